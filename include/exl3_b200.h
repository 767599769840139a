/*
 * exl3_b200.h -- C ABI of libexl3b200.so: the EXL3 (mul1 codebook) trellis weight path on NVIDIA B200 (sm_100a).
 *
 * The entry points are the reference plugin's `quant` seam, one function per QuantTable slot
 * (plugins/turboexl3_qwen38/overlay/mlx_serve/abi/quant.zig:24-108, implemented by plugins/turboexl3_ds41/plugin.zig:28-43),
 * with device buffers in place of MLX arrays and a cudaStream_t in place of the MLX stream.  The reference's kit types
 * (Str, Verdict, Claim, Weight, Source, LoadCtx, Swiglu) are not vendored in its tree; the structs below carry the
 * same fields under plain C types.
 *
 * Conventions
 *   - Every call that can fail returns an exl3_verdict: code EXL3_OK, or a named refusal (`why` is a static string;
 *     the reference's Verdict.refuse / Verdict.named).  An unsupported shape, rate or codebook is refused by name
 *     before any launch; there is no fallback path.
 *   - claims / validate / bill never touch the GPU (quant.zig:22).
 *   - matmul / swiglu enqueue on `stream` and return; they allocate nothing (the per-device workspace is created by
 *     exl3_open or the first weight registered on that device) and do not synchronise.
 *   - Calls that share a device share its workspace: order them on one stream (the reference's single inference
 *     stream), or give concurrent streams their own device via separate processes.
 *   - Activations are f16, bf16 or f32; the output has the input's dtype (linear.zig:17-21).
 */
#ifndef EXL3_B200_H
#define EXL3_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EXL3_ABI_VERSION 1u

/* Str (kit_quant.Str): a byte span, not necessarily NUL-terminated. */
typedef struct exl3_str {
  const char *ptr;
  size_t len;
} exl3_str;

/* Verdict.Code (kit_quant.Verdict): ok, unsupported, failed, too_large. */
typedef enum exl3_code { EXL3_OK = 0, EXL3_UNSUPPORTED = 1, EXL3_FAILED = 2, EXL3_TOO_LARGE = 3 } exl3_code;

typedef struct exl3_verdict {
  int32_t code;    /* exl3_code */
  const char *why; /* static text; NULL when ok */
} exl3_verdict;

/* Claim (kit_quant.Claim): how strongly a format claims a quantization block. */
typedef enum exl3_claim { EXL3_CLAIM_NO = 0, EXL3_CLAIM_BY_MODE = 1, EXL3_CLAIM_BY_MARKER = 2 } exl3_claim;

/* Element types of exl3_tensor / exl3_host_tensor. */
typedef enum exl3_dtype {
  EXL3_F16 = 0,
  EXL3_BF16 = 1,
  EXL3_F32 = 2,
  EXL3_I32 = 3,
  EXL3_U32 = 4,
  EXL3_U16 = 5,
  EXL3_I16 = 6
} exl3_dtype;

/* A device tensor (the ABI's Array): row-major, contiguous. */
typedef struct exl3_tensor {
  void *data;
  int32_t dtype; /* exl3_dtype */
  int32_t ndim;  /* 1..4 */
  int64_t shape[4];
} exl3_tensor;

/* A host tensor handed out by a Source. */
typedef struct exl3_host_tensor {
  const void *data;
  int32_t dtype;
  int32_t ndim;
  int64_t shape[4];
} exl3_host_tensor;

/* Source (kit_quant.Source): where a load reads a pack's tensors.  `tensor` returns 0 and fills `out` when the pack
 * holds `name`, nonzero otherwise.  The data must stay valid until the load call that asked for it returns. */
typedef struct exl3_source {
  void *ctx;
  int (*tensor)(void *ctx, exl3_str name, exl3_host_tensor *out);
} exl3_source;

/* LoadCtx (kit_quant.LoadCtx): one load sequence open -> load_tensor / load_bank* -> close. */
typedef struct exl3_load_ctx {
  uint32_t size; /* sizeof(exl3_load_ctx) */
  exl3_str block_json;
  exl3_str config_json;
  exl3_str model_dir;
  exl3_source source;
  int32_t device;
  void *stream; /* cudaStream_t the uploads run on */
} exl3_load_ctx;

/* Weight flags. */
#define EXL3_WEIGHT_OWNED 1u   /* the library allocated trellis/suh/svh; exl3_release frees them */
#define EXL3_WEIGHT_BANK 2u    /* routed experts stacked on axis 0 (load_bank) */
#define EXL3_WEIGHT_GROUPED 4u /* a grouped linear: x [rows, groups, in] -> y [rows, groups, out] */
/* A narrowed codeword window (the block's "window", 8..16 bits; the codeword is the low w bits of each 16-bit
 * window, expert_exl3.zig Window): bits 8..11 of flags hold 16 - w, 0 for the full window.  The loaders set it from
 * the block; a borrowed weight (exl3_weight_view) sets it by hand.  Such a weight takes the cluster-split decode GEMV
 * (any row count below the GEMM's), the GEMM and the routed experts (gate and up share one window); the
 * grid-stride entry exl3_matmul_noalloc and the dp4a byte sums refuse it. */
/* The mcg codebook (the block's "codebook": "mcg", expert_exl3.zig decodeMcg) instead of mul1; a weight takes the
 * same paths as a narrowed window's. */
#define EXL3_WEIGHT_MCG 16u
#define EXL3_WEIGHT_WINDOW_SHIFT 8
#define EXL3_WEIGHT_WINDOW_MASK 0xF00u
#define EXL3_WEIGHT_WINDOW(w) ((((uint32_t)(16 - (w))) << EXL3_WEIGHT_WINDOW_SHIFT) & EXL3_WEIGHT_WINDOW_MASK)

#define EXL3_MAX_SEGMENTS 4

/* Weight (kit_quant.Weight: w = trellis, scales = suh, biases = svh).  One projection, or `groups` projections of
 * the same shape stacked on axis 0.  A stacked-output weight (exl3_weight_stack: linears that read the same input,
 * the reference's linearShared) has nseg > 1: output columns seg_cols[s]..seg_cols[s+1] use suh row s. */
typedef struct exl3_weight {
  uint32_t size;    /* sizeof(exl3_weight) */
  uint32_t flags;   /* EXL3_WEIGHT_* */
  uint16_t *trellis; /* device, [groups][in/16][out/16][n] (u16 view of the pack's I16) */
  uint16_t *suh;     /* device f16 bits, [groups][nseg][in] */
  uint16_t *svh;     /* device f16 bits, [groups][out] */
  int32_t groups;
  int32_t in_features;
  int32_t out_features;
  int32_t n;         /* halfwords per 16x16 tile = 16 x bits per weight */
  int32_t device;
  int32_t nseg;
  int32_t seg_cols[EXL3_MAX_SEGMENTS + 1];
} exl3_weight;

/* Swiglu options (kit_quant.Swiglu): `limit` > 0 clamps gate above and up symmetrically (moeClamped, 1..128);
 * `verify_rows` keeps the decode chain at any row count. */
typedef struct exl3_swiglu_opts {
  uint32_t size;
  int32_t limit;
  int32_t verify_rows;
} exl3_swiglu_opts;

/* Extra matmul flags (QuantTable.linear_prepared / linear_split(inner)). */
#define EXL3_MATMUL_PREPARED 1u /* x holds f16(H(x*suh)/sqrt(128)) rows: skip the prepare */
#define EXL3_MATMUL_INNER 2u    /* stop at the inner product: y = xp W_hat in f32 (no output Hadamard, no svh) */
#define EXL3_MATMUL_DP4A 4u     /* mul1 byte sums on dp4a instead of the tensor pipe (same bits) */
#define EXL3_MATMUL_GEMV 8u     /* force the decode GEMV at any row count (16 rows per launch) */
#define EXL3_MATMUL_GEMM 16u    /* force the tensor-core GEMM at any row count (the default from 64 rows) */

/* ------------------------------------------------------------------ the quant seam (QuantTable) */

/* claims (plugins/turboexl3_ds41/config.zig:43-47): an EXL3 block (`quant_method` or `format` "exl3") by marker. */
exl3_claim exl3_claims(exl3_str block_json, exl3_str config_json);

/* validate (plugins/turboexl3_ds41/config.zig:49-54; turboexl3_qwen38/config.zig:84-104): refuses by name a codebook
 * other than mul1, a narrowed window, and a rate the kernels do not decode (fractional or above 6 bits). */
exl3_verdict exl3_validate(exl3_str block_json, exl3_str config_json);

/* bill (plugins/turboexl3_ds41/config.zig:57-61): resident bytes once loaded = the bytes the pack stores. */
uint64_t exl3_bill(exl3_str block_json, exl3_str model_dir, uint64_t stored);

/* open / close (plugins/turboexl3_ds41/plugin.zig:52-82): checks the block and creates the device workspace. */
exl3_verdict exl3_open(exl3_load_ctx *ctx);
void exl3_close(exl3_load_ctx *ctx);

/* load_tensor (plugin.zig:86-103): `<name>.trellis` (I16/U16 [in/16, out/16, n]), `<name>.suh` (f16 [in]),
 * `<name>.svh` (f16 [out]) uploaded once to HBM; `in_dim` (0 = any) pins the input width.  A name with no trellis but
 * slices `<name>.slice.<g>` loads as a grouped linear (plugin.zig:107-124). */
exl3_verdict exl3_load_tensor(const exl3_load_ctx *ctx, exl3_str name, uint32_t in_dim, exl3_weight *out);

/* load_bank (plugin.zig:127-185): the routed experts `<prefix>.<e>.<proj>` for e = 0.. stacked on axis 0, refused
 * unless the router `<layer>.gate.weight` scores exactly that many experts. `name` is `<prefix>.<proj>`. */
exl3_verdict exl3_load_bank(const exl3_load_ctx *ctx, exl3_str name, uint32_t in_dim, exl3_weight *out);

/* release (plugin.zig:231-237): frees what the weight owns and zeroes it. */
void exl3_release(exl3_weight *w);

/* matmul (plugin.zig:243-248; quant.zig:41-42): out = x @ W^T.  x [..., in] (f16/bf16/f32) -> out [..., out] in x's
 * dtype; a grouped weight takes x [rows, groups, in].  `out` is caller-allocated. */
exl3_verdict exl3_matmul(const exl3_weight *w, const exl3_tensor *x, void *stream, exl3_tensor *out);

/* moe (plugin.zig:263-265): refused by name -- routed experts run through swiglu. */
exl3_verdict exl3_moe(const exl3_weight *bank, const exl3_tensor *x, const exl3_tensor *lhs, const exl3_tensor *rhs,
                      int32_t sorted, void *stream, exl3_tensor *out);

/* swiglu (plugin.zig:267-283; SX/root.zig:32-167): routed SwiGLU experts.  x [B, S, D]; inds [B, S, K] (i32/u32)
 * and scores [B, S, K] (f32) pick the banks' experts; out [B, S, D] in x's dtype (or f32) is
 * sum_k score * down_e(silu(gate_e(x)) * up_e(x)).  Expert indices outside the bank contribute nothing. */
exl3_verdict exl3_swiglu(const exl3_weight *gate, const exl3_weight *up, const exl3_weight *down,
                         const exl3_tensor *x, const exl3_tensor *inds, const exl3_tensor *scores,
                         const exl3_swiglu_opts *opts, void *stream, exl3_tensor *out);

/* The routed experts at prompt widths (SX/expert_exl3_kernels.zig:2955-3029 moePrefill, expert-sorted windows through
 * a GEMM): reserves, on `device`, the workspace with which exl3_swiglu runs calls of 1024 and more (token, k) slots --
 * up to `max_slots` -- on the tensor cores for banks of up to `experts` experts of hidden -> inter -> hidden: slots
 * sorted by expert into 128-row blocks, the experts' W_hat^T decoded once per call, grouped tcgen05 GEMMs for gate, up
 * and down, the SwiGLU between them.  Memory for speed, like exl3_resident: `bytes` (may be null) receives what it
 * takes (about (max_slots + 127 experts) x (6 hidden + 2 inter) bytes, plus 96 x hidden x inter bytes); max_slots 0
 * frees it.  Without it, or with verify_rows, or for a shared-expert fold, calls take the decode chain in passes.  Not
 * to be called while a call on the device runs. */
exl3_verdict exl3_moe_prefill_reserve(int32_t device, int32_t experts, int32_t hidden, int32_t inter, int32_t max_slots,
                                      uint64_t *bytes);

/* The shared expert beside the routed ones (SharedSwiglu, plugins/turboexl3_qwen38/overlay/mlx_serve/abi/
 * quant.zig:185-199; SX/root.zig:38-68 moeWithShared / moeWithGatedShared, :80-83 moeClampedWithShared). */
typedef struct exl3_shared_swiglu {
  uint32_t size;                /* sizeof(exl3_shared_swiglu) */
  int32_t limit;                /* the routed experts' clamp (exl3_swiglu_opts.limit; 0: none) */
  /* The shared expert's linears (one group each: gate/up [D -> I_s], down [I_s -> D]); all null when `shared` is
   * given instead. */
  const exl3_weight *gate;
  const exl3_weight *up;
  const exl3_weight *down;
  const void *shared;   /* device [B, S, D] in x's dtype: the shared expert's output, already computed */
  const void *logit;    /* device [B, S] in x's dtype: the shared gate's logit per row, or null */
  const void *gate_vec; /* device [D] in x's dtype: logit = x . gate_vec (f32 sum, rounded to x's dtype), or null */
  const void *sigtab;   /* device [65536] in x's dtype: the host's sigmoid of every 16-bit pattern (f16 / bf16
                         * activations), or null: sigmoid in f32 rounded to x's dtype */
} exl3_shared_swiglu;

/* swiglu_shared (quant.zig:95 swiglu_shared): the routed experts (exl3_swiglu) plus the shared expert, folded into
 * the routed output's rounding: out = RN(RN(routed) + g), g = RN(RN(sigmoid(logit)) * shared) with a gate (`logit`
 * or `gate_vec`), else g = shared (RN: to x's dtype; out in x's dtype).  With the shared expert's linears, shared =
 * RN(down(silu(gate(x)) * up(x))) is computed first, into `out`, by the same expert kernels. */
exl3_verdict exl3_swiglu_shared(const exl3_weight *gate, const exl3_weight *up, const exl3_weight *down,
                                const exl3_tensor *x, const exl3_tensor *inds, const exl3_tensor *scores,
                                const exl3_shared_swiglu *opts, void *stream, exl3_tensor *out);

/* ------------------------------------------------------------------ library calls beside the seam */

/* matmul with EXL3_MATMUL_* flags (linear_prepared, linear_split inner: quant.zig:57-66). */
exl3_verdict exl3_matmul_ex(const exl3_weight *w, const exl3_tensor *x, uint32_t flags, void *stream,
                            exl3_tensor *out);

/* matmul_ex with CUDA events recorded on the stream between its launches, for timing a phase without a profiler.
 * events: 4 cudaEvent_t (any may be NULL) -- [0] before the first launch and [3] after the last; on the GEMM path
 * (64 rows and more) [1] after the operand images (prepare + decode) and [2] after the GEMM of the first chunk of
 * rows and columns.  A measurement aid of this library; the reference has no counterpart. */
exl3_verdict exl3_matmul_timed(const exl3_weight *w, const exl3_tensor *x, uint32_t flags, void *stream,
                               exl3_tensor *out, void *const *events);

/* ------------------------------------------------------------------ expert parallelism (beside the seam)
 *
 * The reference runs on one device; these three calls are this library's expert-parallel split of swiglu over ranks
 * (rank r owns experts [r E/world, (r+1) E/world) of every bank), around two equal-split all-to-alls that the caller
 * issues (NCCL).  A dispatch buffer is [world, C + 1, D] in x's dtype: per peer, C token rows in slot order and one
 * metadata row whose 32-bit word j is row j's peer-local expert (-1 = empty).  EXL3_ERR_EP_OVERFLOW in the device
 * error word marks a dispatch that had more than C rows for one peer (the extra slots are dropped). */

/* x [T, D], inds [T, K] (global expert ids; outside 0..experts-1 = absent) -> send [world, C + 1, D] and
 * back_slot [T, K] i32: the row of the returned buffer that holds slot (t, k), -1 if absent or dropped.  With
 * `shared` set, id `experts` is a shared expert that every rank holds at local index experts / world: its slots go to
 * the calling rank's own block. */
exl3_verdict exl3_ep_dispatch(const exl3_tensor *x, const exl3_tensor *inds, int32_t experts, int32_t world,
                              int32_t rank, int32_t shared, void *stream, exl3_tensor *send, exl3_tensor *back_slot);
/* received blocks [world, C + 1, D] -> swiglu's inds [world, C + 1, 1] i32 (metadata rows -1) and scores (all 1). */
exl3_verdict exl3_ep_unpack(const exl3_tensor *recv, void *stream, exl3_tensor *inds, exl3_tensor *scores);
/* out [T, D] = sum_k scores[t, k] * back[back_slot[t, k]] in k order (f32), + shared [T, D] f32 when its data is not
 * NULL; back is f32 [world, C + 1, D] (the owners' swiglu outputs returned by the second all-to-all). */
exl3_verdict exl3_ep_combine(const exl3_tensor *back, const exl3_tensor *back_slot, const exl3_tensor *scores,
                             const exl3_tensor *shared, void *stream, exl3_tensor *out);

/* ------------------------------------------------------------------ expert parallelism over peer memory
 *
 * The same split as above with both all-to-alls done by this library's kernels over NVLink instead of a collective
 * library: every rank holds a receive region [2][world][C + 1][D] (x's dtype) and a return region
 * [2][world][C + 1][D] f32, mapped into the other ranks with CUDA IPC.  Setup as the column-parallel exchange:
 * exl3_epx_create on every rank, exchange the 64-byte handles, exl3_epx_connect.  A step: exl3_epx_dispatch (x's
 * rows straight into the owners' receive regions, then one system-scope release), exl3_epx_receive (bounded wait for
 * every rank's dispatch; the received blocks into the caller's fixed buffer, with swiglu's inds and scores), swiglu
 * on that buffer (f32 out), exl3_epx_return (each block straight back into its source rank's return region, then a
 * release), exl3_epx_combine (bounded wait for every rank's return; the weighted sum).  Stream-ordered kernels with no
 * host synchronisation: a whole step can be captured in a CUDA graph.  A wait that gives up (one second) sets
 * EXL3_ERR_EP_TIMEOUT.  Every rank must run the same steps. */
typedef struct exl3_epx exl3_epx;

/* capacity C rows per (source, owner) pair, hidden D (a multiple of 128), dtype the activations' (f16, bf16, f32). */
exl3_verdict exl3_epx_create(int32_t device, int32_t world, int32_t rank, int32_t cap, int32_t hidden, int32_t dtype,
                             exl3_epx **out, uint8_t *ipc_handle);
/* ipc_handles: world * 64 bytes, rank order (this rank's own entry is ignored). */
exl3_verdict exl3_epx_connect(exl3_epx *ep, const uint8_t *ipc_handles);
void exl3_epx_destroy(exl3_epx *ep);
/* Begins a step: x [T, D], inds [T, K] as exl3_ep_dispatch (shared: id `experts` stays on this rank at local index
 * experts / world) -> back_slot [T, K] i32, the return-region row of slot (t, k), -1 if absent or dropped. */
exl3_verdict exl3_epx_dispatch(exl3_epx *ep, const exl3_tensor *x, const exl3_tensor *inds, int32_t experts,
                               int32_t shared, void *stream, exl3_tensor *back_slot);
/* -> xbuf [world, C + 1, D] (the rows every rank sent here, block q from rank q), inds [world, C + 1, 1] i32 (local
 * expert, -1 = empty) and scores (1), ready for swiglu with this rank's banks. */
exl3_verdict exl3_epx_receive(exl3_epx *ep, void *stream, exl3_tensor *xbuf, exl3_tensor *inds, exl3_tensor *scores);
/* ys: swiglu's f32 output [world, C + 1, D]; block q goes back to rank q. */
exl3_verdict exl3_epx_return(exl3_epx *ep, const exl3_tensor *ys, void *stream);
/* Ends the step: out [T, D] = sum_k scores[t, k] * returned[back_slot[t, k]] in k order (f32). */
exl3_verdict exl3_epx_combine(exl3_epx *ep, const exl3_tensor *back_slot, const exl3_tensor *scores, void *stream,
                              exl3_tensor *out);

/* ------------------------------------------------------------------ column-parallel experts over peer memory
 *
 * Beside the seam: routed experts split by columns instead of by experts, so every rank streams exactly 1/W of the
 * distinct experts' bytes whatever the routing.  Rank r holds, for every expert, gate/up output columns
 * [r inter/W, (r+1) inter/W) and down output columns [r hidden/W, (r+1) hidden/W) (down's input is the whole
 * intermediate).  Setup: exl3_cpx_create on every rank (64-byte IPC handle out), exchange the handles,
 * exl3_cpx_connect.  A call: every rank brings T tokens with K slots (a shared expert is one more bank entry and slot);
 * the library gathers the tokens, runs route / prepare / gate|up on all W T rows (the gate|up epilogue stores its
 * blocks of the down input into every rank's buffer over NVLink), waits for every rank's gate|up, runs down over
 * its output columns and the combine, and returns each token's columns to its owner -- all stream-ordered kernels with
 * no host synchronisation (a whole call fits in a CUDA graph).  A wait that gives up (one second) sets
 * EXL3_ERR_EP_TIMEOUT.  Every rank must make the same calls. */
typedef struct exl3_cpx exl3_cpx;

/* tokens T and slots K per rank per call (W T K <= 512), hidden and inter multiples of 128 W, dtype the activations'. */
exl3_verdict exl3_cpx_create(int32_t device, int32_t world, int32_t rank, int32_t tokens, int32_t topk, int32_t hidden,
                             int32_t inter, int32_t dtype, exl3_cpx **out, uint8_t *ipc_handle);
/* ipc_handles: world * 64 bytes, rank order (this rank's own entry is ignored). */
exl3_verdict exl3_cpx_connect(exl3_cpx *cp, const uint8_t *ipc_handles);
void exl3_cpx_destroy(exl3_cpx *cp);
/* x, out [T, hidden] (the exchange's dtype, 16-byte aligned), inds i32 / scores f32 [T, K] (global expert ids, -1 or
 * past the bank = absent); gate / up: this rank's slices [E, hidden -> inter/W], down [E, inter -> hidden/W]. */
exl3_verdict exl3_swiglu_cp(exl3_cpx *cp, const exl3_weight *gate, const exl3_weight *up, const exl3_weight *down,
                            const exl3_tensor *x, const exl3_tensor *inds, const exl3_tensor *scores,
                            const exl3_swiglu_opts *opts, void *stream, exl3_tensor *out);

/* ------------------------------------------------------------------ column parallelism with a fused all-gather
 *
 * Beside the seam (the reference is single-device): a linear split by output columns over `world` ranks (one process
 * per GPU) whose decode GEMV writes its columns straight into every rank's exchange buffer over NVLink, so no
 * separate all-gather runs.  Setup: exl3_tp_create on every rank (returns a 64-byte CUDA IPC handle), exchange the
 * handles (e.g. torch.distributed), exl3_tp_connect with all of them in rank order.  A step: exl3_tp_begin, the
 * column-parallel matmuls (exl3_matmul_tp, each into its own slot), exl3_tp_gather (publishes this rank's columns,
 * waits for every rank's, then copies the gathered rows out).  All three are stream-ordered kernels with no host
 * synchronisation, so a whole step can be captured in a CUDA graph.  Every rank must run the same steps. */
typedef struct exl3_tp exl3_tp;

/* An exchange of `slots` slots of slot_bytes (a multiple of 16) each, for gathered widths up to 128 * max_cb columns;
 * ipc_handle receives 64 bytes to hand to the other ranks. */
exl3_verdict exl3_tp_create(int32_t device, int32_t world, int32_t rank, int32_t slots, int64_t slot_bytes,
                            int32_t max_cb, exl3_tp **out, uint8_t *ipc_handle);
/* ipc_handles: world * 64 bytes, rank order (this rank's own entry is ignored). */
exl3_verdict exl3_tp_connect(exl3_tp *tp, const uint8_t *ipc_handles);
void exl3_tp_destroy(exl3_tp *tp);
/* The next step (the slots' double buffers flip). */
exl3_verdict exl3_tp_begin(exl3_tp *tp, void *stream);
/* This rank's column shard of a (possibly stacked) linear: x [rows <= 16, in] -> its columns of y, written into slot
 * `slot` of every rank.  seg_col0[s] / seg_total[s] (w->nseg entries, multiples of 128): segment s's first gathered
 * column held by this rank, and the segment's gathered width.  The slot holds the segments back to back, each
 * [rows][seg_total] in x's dtype. */
exl3_verdict exl3_matmul_tp(const exl3_weight *w, const exl3_tensor *x, exl3_tp *tp, int32_t slot,
                            const int64_t *seg_col0, const int64_t *seg_total, void *stream);
/* Ends this rank's step: publishes its columns of every slot of the step to every rank (one system-scope release),
 * waits for every rank's, then copies slots [slot0, slot0 + nslots) to out (device memory, 16-byte aligned): slot i
 * at out + i * slot_bytes.  A step's gathered outputs are readable from its gather on. */
exl3_verdict exl3_tp_gather(exl3_tp *tp, int32_t slot0, int32_t nslots, void *stream, void *out);

/* ------------------------------------------------------------------ exchange timelines
 *
 * An exchange created while EXL3_TRACE=1 is set in the environment records a phase timeline: its kernels write
 * %globaltimer stamps (ns, this GPU's clock) into a device ring of 8 per step for the last 16 steps.  These calls wait
 * for the device and copy the ring into out (128 u64, step-major, oldest step first; steps not yet run read 0); an
 * exchange created without EXL3_TRACE=1 is refused (EXL3_UNSUPPORTED).  Stamps per step --
 *   tp:  0 begin, 1 publish (this rank's GEMVs of the step done), 2 every rank's columns seen, 3 gathered;
 *   epx: 0 dispatch begins, 1 its copies done, 2 every rank's dispatch seen, 3 received, 4 return begins (the
 *        caller's swiglu done), 5 its copies done, 6 every rank's return seen, 7 combined;
 *   cpx: 0 tokens' copies begin, 1 done, 2 every rank's tokens seen, 3 gate|up done, 4 every rank's gate|up seen,
 *        5 down and combine done, 6 every rank's columns seen, 7 copied out.
 * A wait's share (2 - 1, 6 - 5, ...) is the time this rank waited for the slowest peer. */
exl3_verdict exl3_tp_trace(exl3_tp *tp, uint64_t *out);
exl3_verdict exl3_epx_trace(exl3_epx *ep, uint64_t *out);
exl3_verdict exl3_cpx_trace(exl3_cpx *cp, uint64_t *out);

/* ------------------------------------------------------------------ the model seam's parse (linears only)
 *
 * plugins/turboexl3_qwen38/plugin.zig:38-53 ModelTable.claims / parse (config.zig:19-119, src/direct/config.zig:301-420),
 * narrowed to the keys the linears need.  MLX-free and GPU-free; refusals carry the reference's names
 * ("turboexl3_qwen38: NotExl3", "...: Exl3CodebookUnsupported", "...: Exl3WindowUnsupported", "...:
 * Exl3RateUnsupported", "...: Exl3TopKExceedsReduceBank", "...: TrunkQuantNotAnObject", "...: InvalidConfigField",
 * "...: Unsupported", "...: InvalidConfig"). */
typedef struct exl3_model_config {
  uint32_t size; /* sizeof(exl3_model_config), set by the caller */
  uint32_t hidden_size, intermediate_size, num_hidden_layers, num_attention_heads, num_key_value_heads, head_dim;
  uint32_t num_experts, num_experts_per_tok, moe_intermediate_size, shared_expert_intermediate_size;
  uint32_t expert_rate_n; /* the routed banks' halfwords per tile (16 x bits per weight); 0 without expert_quant */
  char weight_prefix[96];  /* NUL-terminated */
} exl3_model_config;
/* A qwen4_exp pack whose config names a trunk_quant block: by marker; everything else: no. */
exl3_claim exl3_model_claims(exl3_str model_type, exl3_str config_json);
exl3_verdict exl3_model_parse(exl3_str config_json, exl3_model_config *out);

/* The model seam's load, bill and forward over the EXL3 linears (ModelTable.bill / load / unload / forward,
 * plugins/turboexl3_qwen38/plugin.zig:38-53, narrowed to the linears: attention, caches, norms and the drafter are the
 * host's).  A pack's tensors are named <prefix>.layers.<i>.<module>.{trellis,suh,svh}; a routed bank's members
 * <bank>.experts.<e>.<proj>.  `names` lists the pack's tensor names (count of them), `source` hands out their data. */
typedef struct exl3_model exl3_model;

/* bill: the resident bytes of every EXL3 tensor of the pack's layers, as the pack stores them (EXL3 weights stay
 * resident as stored, plugins/turboexl3_ds41/config.zig:57-61); 0 for a config exl3_model_parse refuses.  Never
 * touches the GPU. */
uint64_t exl3_model_bill(exl3_str config_json, const exl3_source *source, const exl3_str *names, int32_t count);

/* load: parses the config (exl3_model_parse) and uploads once every EXL3 linear of every layer under the trunk block
 * (trunk_quant) and every routed bank under the expert block (expert_quant, else the trunk's); the linears of a layer
 * that read one input -- <m>.q_proj|k_proj|v_proj and <m>.gate_proj|up_proj -- are also stacked into one launch
 * (SX/linear.zig:39-72).  The dense MLP's intermediate buffers are reserved here for up to `max_rows` rows, so the
 * forward calls allocate nothing.  *out receives the model (free it with exl3_model_unload). */
exl3_verdict exl3_model_load(exl3_str config_json, const exl3_source *source, const exl3_str *names, int32_t count,
                             int32_t device, int32_t max_rows, void *stream, exl3_model **out);
void exl3_model_unload(exl3_model *m);

/* The weight of one module (a linear, or a stack named "a|b|c"), borrowed from the model: 1 when found. */
int32_t exl3_model_weight(const exl3_model *m, int32_t layer, exl3_str module, exl3_weight *out);

/* forward over the linears.  linear: one module, x [..., in] -> out [..., out] in x's dtype.  linears: modules that
 * read one x, out holding each one's [rows, out] back to back -- one stacked launch where the load stacked them.
 * mlp: the dense SwiGLU MLP <module>.{gate,up,down}_proj, down(RN(silu(gate x) * up x)), at most max_rows rows.
 * experts: the routed bank <bank> (exl3_swiglu; x [B, S, D], inds / scores [B, S, K]) plus, when `shared` names a
 * module with gate/up/down_proj, that shared expert folded in by exl3_swiglu_shared -- gated by `shared_logit`
 * (device [B, S] in x's dtype) when given. */
exl3_verdict exl3_model_linear(const exl3_model *m, int32_t layer, exl3_str module, const exl3_tensor *x, void *stream,
                               exl3_tensor *out);
exl3_verdict exl3_model_linears(const exl3_model *m, int32_t layer, const exl3_str *modules, int32_t count,
                                const exl3_tensor *x, void *stream, exl3_tensor *out);
exl3_verdict exl3_model_mlp(const exl3_model *m, int32_t layer, exl3_str module, const exl3_tensor *x, void *stream,
                            exl3_tensor *out);
exl3_verdict exl3_model_experts(const exl3_model *m, int32_t layer, exl3_str bank, exl3_str shared,
                                const exl3_tensor *x, const exl3_tensor *inds, const exl3_tensor *scores,
                                const void *shared_logit, void *stream, exl3_tensor *out);

/* A borrowed view of device arrays already in the pack layout (the reference's shared handles, plugin.zig:213-218):
 * validates the shapes and creates the device workspace; exl3_release on a view frees nothing. */
exl3_verdict exl3_weight_view(uint16_t *trellis, uint16_t *suh, uint16_t *svh, int32_t groups, int32_t in_features,
                              int32_t out_features, int32_t n, int32_t device, exl3_weight *out);

/* Linears that read the same input stacked along the output into one weight (SX/linear.zig:39-72 linearShared):
 * `count` (2..4) one-group weights with equal in_features and n, each out_features a multiple of 128. */
exl3_verdict exl3_weight_stack(const exl3_weight *parts, int32_t count, void *stream, exl3_weight *out);

/* W_hat of group `group`: f16 bits, row-major [in][out] (the decmat / decode_table checks,
 * plugins/turboexl3_ds41/src/exl3/selfcheck.zig:861-930). */
exl3_verdict exl3_decode_dense(const exl3_weight *w, int32_t group, uint16_t *out, uint32_t flags, void *stream);

/* The dense effective W of group `group` (plugins/sushi_ds41/src/sushi/exl3/expert_exl3.zig:440-488
 * reconstructPublic, the dense twin SX/linear.zig:200-224 checks against): f16 bits, row-major [in][out], with
 * x @ W_eff = the linear's output -- W_eff[r][c] = f16(svh[c] * (H128 (suh[r] * (H128 W_hat)[r][.]))[c]), the
 * Hadamards orthonormal, in f32.  One linear (nseg 1). */
exl3_verdict exl3_reconstruct_public(const exl3_weight *w, int32_t group, uint16_t *out, void *stream);

/* Trellis encoder (no counterpart in the reference, which ships no encoder: plugins/turboexl3_ds41/NOTICE:30-32).
 * `target` (device f32, row-major [in][out]) is the matrix the trellis should decode to -- already rotated by the
 * 128-wide Hadamards and scaled to the codebook's unit variance; `trellis` (device) receives [in/16][out/16][n]. */
exl3_verdict exl3_encode_trellis(const float *target, int32_t in_features, int32_t out_features, int32_t n,
                                 uint16_t *trellis, void *stream);

/* matmul without any allocation (no counterpart in the reference): for hosts that cannot let a library call
 * cudaMalloc -- a server that reserves its device memory up front and admits nothing beyond its memory bill, or an
 * embedding runtime whose own allocator owns every device byte.  The same decode and f32 accumulation as
 * exl3_matmul, within the same 2e-3 rel-L2 of the f32 truth but not bit-identical to it (exl3_matmul chooses other
 * kernels by shape, whose sums run in another order); kernel errors land in the word exl3_device_error reads.  The
 * scratch (split partials, counters) lives in one static device array of 8 MiB + 32 KiB that every device loading
 * the library holds until exit; the weight struct may be filled by hand (no exl3_weight_view needed), and its
 * seg_cols must run from 0 to out_features in whole 128-column blocks.  One ungrouped weight (stacked segments
 * allowed), at most 2^24 rows.  A layer needing more partials than the array holds is refused with EXL3_TOO_LARGE.
 * The first call on a device looks the array up (cudaGetSymbolAddress) and clears its counters with a memset on the
 * caller's stream: make it before any stream capture.  All calls share the array: calls that overlap on the GPU
 * race -- order them on one stream. */
exl3_verdict exl3_matmul_noalloc(const exl3_weight *w, const exl3_tensor *x, void *stream, exl3_tensor *out);

/* Resident decoded matrices (QuantTable.resident / resident_pending, plugins/turboexl3_qwen38/overlay/mlx_serve/abi/
 * quant.zig:96-101: memory for speed).  Keeps each of the `count` weights' decoded matrices from its first prefill
 * (GEMM) call on, so later prefill calls skip the weight decode: device memory for the tensor-core GEMM's operand
 * image of W_hat^T, f16, about 2 x in x out bytes per group, is reserved here (calls stay allocation-free) and filled
 * by the first call.  Admitted only if everything kept, old and new, fits in `room` bytes (0: no bound), else refused
 * EXL3_TOO_LARGE and nothing changes; `bytes` (may be null) receives the bytes kept.  A weight already kept is kept
 * once.  `count` 0 drops every kept matrix.  exl3_release drops the matrices of the weight it frees; a borrowed weight
 * (exl3_weight_view) must be dropped before its memory is freed or reused.  The first prefill call on a kept weight
 * fills it on that call's stream: calls on other streams must not run before that call is ordered before them. */
exl3_verdict exl3_resident(const exl3_weight *ws, int32_t count, uint64_t room, void *stream, uint64_t *bytes);

/* The bytes exl3_resident admitted and no prefill call has filled yet (QuantTable.resident_pending). */
uint64_t exl3_resident_pending(void);

/* Device error bits the kernels recorded on `device`; `clear` resets them. */
#define EXL3_ERR_WAIT_TIMEOUT 1u  /* a bounded mbarrier wait gave up (the kernel left its loop and returned) */
#define EXL3_ERR_BAD_SHAPE 2u     /* a launch saw a shape its host validation should have refused */
#define EXL3_ERR_EP_OVERFLOW 4u   /* an expert-parallel dispatch had more rows for one peer than its capacity */
#define EXL3_ERR_TP_TIMEOUT 8u    /* a column-parallel gather gave up waiting (one second) for a peer's columns */
#define EXL3_ERR_EP_TIMEOUT 16u   /* a peer expert-parallel exchange gave up waiting (one second) for a peer's rows */
exl3_verdict exl3_device_error(int32_t device, uint32_t *bits, int32_t clear);

/* The library's build string. */
const char *exl3_version(void);

#ifdef __cplusplus
}
#endif

#endif /* EXL3_B200_H */
