"""The decode path across the GPUs of one box: one process per GPU, torch.distributed over NCCL for the exchanges.

Two splits, the only two the path has (the reference runs on one device; these are this library's):

* Column parallelism for a linear (``ColumnParallelLinear``): rank r keeps the trellis tiles of its 128-aligned range
  of output columns, the whole suh and its slice of svh; x is replicated; every rank computes its columns and one
  all-gather assembles y.  No other exchange: the input Hadamard is per 128-row block of the input and the output
  Hadamard per 128-column block of the output, so both stay inside a shard.

* Expert parallelism for the routed experts (``ExpertParallelSwiglu``): rank r keeps experts
  [r E/world, (r+1) E/world) of every bank; each rank's tokens are dispatched to the experts' owners and the results
  combined back with two equal-split all-to-alls (exl3_ep_dispatch / exl3_ep_unpack / exl3_ep_combine around them).
  A shared expert, when given, runs where the tokens live.

The drivers take their compute as an ``ops`` object (default: the CUDA library) and their exchanges from
torch.distributed, so the same sequence of collectives runs over NCCL on GPUs and over gloo with CPU stand-ins in
the tests.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import quant as Q

COL_BLOCK = 128  # output columns per Hadamard block: the unit a column shard is made of


TRACE_STEPS, TRACE_STAMPS = 16, 8


def read_trace(fn, ptr) -> list[list[int]]:
    """An exchange's phase timeline (created with EXL3_TRACE=1 in the environment): the last 16 steps' %globaltimer
    stamps in ns, 8 per step, oldest step first; steps not yet run are left out.  Which stamp is which: the
    exchange-timeline comment of include/exl3_b200.h."""
    import ctypes
    from . import _lib as L
    buf = (ctypes.c_uint64 * (TRACE_STEPS * TRACE_STAMPS))()
    L.check(fn(ptr, buf))
    steps = [list(buf[i * TRACE_STAMPS:(i + 1) * TRACE_STAMPS]) for i in range(TRACE_STEPS)]
    return [st for st in steps if any(st)]


def column_range(out_features: int, rank: int, world: int) -> tuple[int, int]:
    """Rank r's output columns [c0, c1): whole 128-column blocks, the first (blocks % world) ranks one block more."""
    if out_features % COL_BLOCK:
        raise ValueError("out_features must be a multiple of 128")
    blocks = out_features // COL_BLOCK
    if blocks < world:
        raise ValueError(f"{blocks} column blocks cannot be split over {world} ranks")
    base, extra = divmod(blocks, world)
    b0 = rank * base + min(rank, extra)
    b1 = b0 + base + (1 if rank < extra else 0)
    return b0 * COL_BLOCK, b1 * COL_BLOCK


def shard_columns(tr: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor, rank: int, world: int):
    """This rank's column shard of a linear in the pack layout: trellis [in/16, out/16, n] -> [in/16, cols/16, n],
    suh whole, svh [c0:c1]."""
    c0, c1 = column_range(svh.shape[-1], rank, world)
    return tr[:, c0 // 16:c1 // 16, :].contiguous(), suh, svh[c0:c1].contiguous()


class CudaLinearOps:
    """The compute of the column-parallel linear: the library's matmul."""

    @staticmethod
    def load(tr, suh, svh):
        return Q.weight_from_tensors(tr, suh, svh)

    @staticmethod
    def matmul(w, x, out=None):
        return Q.matmul(w, x, out=out)


class ColumnParallelLinear:
    """y = x @ W^T with W's output columns split over the ranks and y all-gathered.

    Every rank passes the full linear (the pack is readable everywhere) and keeps its shard.  Shards may differ by
    one 128-column block; the gather runs over equal blocks padded to the largest shard and the padding is dropped
    when y is assembled.
    """

    def __init__(self, tr, suh, svh, rank: int, world: int, group=None, ops=None):
        self.rank, self.world, self.group = rank, world, group
        self.ops = ops or CudaLinearOps()
        self.out_features = svh.shape[-1]
        self.ranges = [column_range(self.out_features, r, world) for r in range(world)]
        self.width = max(c1 - c0 for c0, c1 in self.ranges)
        self.weight = self.ops.load(*shard_columns(tr, suh, svh, rank, world))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        rows = x.shape[0]
        c0, c1 = self.ranges[self.rank]
        mine = c1 - c0
        local = torch.empty((rows, self.width), dtype=x.dtype, device=x.device)
        if mine == self.width:
            self.ops.matmul(self.weight, x, local)
        else:
            local[:, mine:].zero_()
            local[:, :mine].copy_(self.ops.matmul(self.weight, x, None))
        if self.world == 1:
            return local
        gathered = torch.empty((self.world * rows, self.width), dtype=x.dtype, device=x.device)  # concatenated form
        dist.all_gather_into_tensor(gathered, local, group=self.group)
        gathered = gathered.view(self.world, rows, self.width)
        return torch.cat([gathered[r, :, :b - a] for r, (a, b) in enumerate(self.ranges)], dim=1)


class TpExchange:
    """Column-parallel outputs gathered inside the decode GEMV (exl3_tp_*): every rank's GEMV writes its columns
    straight into every rank's exchange buffer over NVLink, and a gather kernel waits for all of them.

    One per process (one GPU per rank).  A step is ``begin()``, ``matmul(w, x, slot, ...)`` per column-parallel
    linear (each into its own slot), then ``gather(slot0, n, out)``; no host synchronisation, so whole steps can be
    captured in a CUDA graph.  Every rank must run the same steps.
    """

    def __init__(self, rank: int, world: int, slots: int, slot_bytes: int, max_cb: int, device=None, group=None):
        import ctypes
        from . import _lib as L
        self._L, self._ct = L, ctypes
        self.rank, self.world, self.slots = rank, world, slots
        self.slot_bytes = (int(slot_bytes) + 15) // 16 * 16
        dev = torch.cuda.current_device() if device is None else torch.device(device).index
        handle = (ctypes.c_uint8 * 64)()
        ptr = ctypes.c_void_p()
        L.check(L.lib().exl3_tp_create(dev, world, rank, slots, self.slot_bytes, max_cb, ctypes.byref(ptr), handle))
        self._ptr = ptr
        mine = bytes(handle)
        if world > 1:
            every = [None] * world
            dist.all_gather_object(every, mine, group=group)
        else:
            every = [mine]
        buf = (ctypes.c_uint8 * (64 * world)).from_buffer_copy(b"".join(every))
        L.check(L.lib().exl3_tp_connect(self._ptr, buf))

    def begin(self, stream=None):
        self._L.check(self._L.lib().exl3_tp_begin(self._ptr, Q._stream(stream)))

    def matmul(self, w, x: torch.Tensor, slot: int, seg_col0, seg_total, stream=None):
        """This rank's shard of a (stacked) linear into slot `slot` of every rank: segment s covers gathered
        columns [seg_col0[s], seg_col0[s] + its width) of a segment seg_total[s] wide."""
        ct = self._ct
        c0 = (ct.c_int64 * len(seg_col0))(*[int(v) for v in seg_col0])
        tot = (ct.c_int64 * len(seg_total))(*[int(v) for v in seg_total])
        self._L.check(self._L.lib().exl3_matmul_tp(ct.byref(w.raw), ct.byref(Q._tensor(x)), self._ptr, int(slot), c0,
                                                   tot, Q._stream(stream)))

    def gather(self, slot0: int, nslots: int, out: torch.Tensor, stream=None):
        """Waits for every rank's columns of slots [slot0, slot0 + nslots) and copies them into out (a device buffer
        of nslots * slot_bytes bytes; slot i starts at byte i * slot_bytes)."""
        if out.numel() * out.element_size() < nslots * self.slot_bytes or not out.is_cuda:
            raise ValueError("out holds nslots * slot_bytes bytes on the GPU")
        self._L.check(self._L.lib().exl3_tp_gather(self._ptr, int(slot0), int(nslots), Q._stream(stream),
                                                   out.data_ptr()))

    def trace(self) -> list[list[int]]:
        """Per step: begin, publish (this rank's GEMVs done), every rank's columns seen, gathered (ns)."""
        return read_trace(self._L.lib().exl3_tp_trace, self._ptr)

    def close(self):
        if self._ptr:
            self._L.lib().exl3_tp_destroy(self._ptr)
            self._ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------------ expert parallelism

def expert_range(experts: int, rank: int, world: int) -> tuple[int, int]:
    if experts % world:
        raise ValueError(f"{experts} experts do not split evenly over {world} ranks")
    per = experts // world
    return rank * per, (rank + 1) * per


def ep_capacity(tokens: int, topk: int, experts: int, world: int, shared: bool = False) -> int:
    """Rows one rank can route to one peer: each token sends at most min(K, E/world) distinct experts there (one more,
    its shared-expert slot, to its own rank)."""
    return max(1, tokens * (min(topk, experts // world) + (1 if shared else 0)))


class CudaExpertOps:
    """The compute of the expert-parallel step: the library's dispatch, unpack, swiglu and combine."""

    @staticmethod
    def dispatch(x, inds, experts, world, rank, shared, send, back_slot):
        Q.ep_dispatch(x, inds, experts, world, send, back_slot, rank=rank, shared=shared)

    @staticmethod
    def unpack(recv, inds, scores):
        Q.ep_unpack(recv, inds, scores)

    @staticmethod
    def swiglu(gate, up, down, x, inds, scores, out, limit):
        Q.swiglu(gate, up, down, x, inds, scores, limit=limit, out=out)

    @staticmethod
    def combine(back, back_slot, scores, out):
        Q.ep_combine(back, back_slot, scores, None, out)


class PeerExpertExchange:
    """The two all-to-alls of the expert-parallel step over NVLink peer memory (exl3_epx_*): the dispatch writes each
    token row straight into its owner's receive region and the owners write their outputs straight back, each phase
    published with one system-scope release and awaited with a bounded wait.  One per process (one GPU per rank).
    """

    def __init__(self, rank: int, world: int, cap: int, hidden: int, dtype=torch.float16, device=None, group=None):
        import ctypes
        from . import _lib as L
        self._L, self._ct = L, ctypes
        self.rank, self.world, self.cap, self.hidden = rank, world, cap, hidden
        dev = torch.cuda.current_device() if device is None else torch.device(device).index
        handle = (ctypes.c_uint8 * 64)()
        ptr = ctypes.c_void_p()
        L.check(L.lib().exl3_epx_create(dev, world, rank, cap, hidden, Q._TORCH_DT[dtype], ctypes.byref(ptr), handle))
        self._ptr = ptr
        mine = bytes(handle)
        if world > 1:
            every = [None] * world
            dist.all_gather_object(every, mine, group=group)
        else:
            every = [mine]
        buf = (ctypes.c_uint8 * (64 * world)).from_buffer_copy(b"".join(every))
        L.check(L.lib().exl3_epx_connect(self._ptr, buf))

    def dispatch(self, x, inds, experts: int, shared: bool, back_slot, stream=None):
        self._L.check(self._L.lib().exl3_epx_dispatch(self._ptr, self._ct.byref(Q._tensor(x)),
                                                      self._ct.byref(Q._tensor(inds)), int(experts), int(bool(shared)),
                                                      Q._stream(stream), self._ct.byref(Q._tensor(back_slot))))

    def receive(self, xbuf, inds, scores, stream=None):
        ct = self._ct
        self._L.check(self._L.lib().exl3_epx_receive(self._ptr, Q._stream(stream), ct.byref(Q._tensor(xbuf)),
                                                     ct.byref(Q._tensor(inds)), ct.byref(Q._tensor(scores))))

    def give_back(self, ys, stream=None):
        self._L.check(self._L.lib().exl3_epx_return(self._ptr, self._ct.byref(Q._tensor(ys)), Q._stream(stream)))

    def combine(self, back_slot, scores, out, stream=None):
        ct = self._ct
        self._L.check(self._L.lib().exl3_epx_combine(self._ptr, ct.byref(Q._tensor(back_slot)),
                                                     ct.byref(Q._tensor(scores)), Q._stream(stream),
                                                     ct.byref(Q._tensor(out))))

    def trace(self) -> list[list[int]]:
        """Per step: dispatch begins / copied, every rank's dispatch seen, received, return begins (swiglu done) /
        copied, every rank's return seen, combined (ns)."""
        return read_trace(self._L.lib().exl3_epx_trace, self._ptr)

    def close(self):
        if self._ptr:
            self._L.lib().exl3_epx_destroy(self._ptr)
            self._ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def expert_columns(tr: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor, c0: int, c1: int):
    """A bank's output columns [c0, c1) (multiples of 128): trellis [E, in/16, out/16, n] -> [E, in/16, (c1-c0)/16, n],
    svh [E, out] -> [E, c1-c0]; suh (the input side) whole."""
    if c0 % 128 or c1 % 128:
        raise ValueError("column slices are whole 128-column blocks")
    return tr[:, :, c0 // 16:c1 // 16].contiguous(), suh.contiguous(), svh[:, c0:c1].contiguous()


class ColumnParallelExperts:
    """Routed SwiGLU experts split by columns over the ranks (exl3_cpx_* / exl3_swiglu_cp): rank r holds, for every
    expert, gate/up output columns [r inter/W, (r+1) inter/W) and down output columns [r hidden/W, (r+1) hidden/W)
    (``expert_columns``), so every rank streams 1/W of the distinct experts' bytes whatever the routing.  The tokens
    are gathered, the down input exchanged and the outputs returned over NVLink peer memory inside one call; no host
    synchronisation, so a whole step can be captured in a CUDA graph.  One per process (one GPU per rank).

    gate/up/down: this rank's slices of the banks (the shared expert, when ``shared`` is set, last); ``forward(x [T, D],
    inds, scores)`` -> out [T, D] in x's dtype; inds / scores [T, K], or [T, K + 1] with the shared expert's column.
    """

    def __init__(self, gate, up, down, experts: int, tokens: int, topk: int, hidden: int, inter: int, rank: int,
                 world: int, dtype=torch.float16, device=None, group=None, shared: bool = False, limit: int = 0):
        import ctypes
        from . import _lib as L
        self._L, self._ct = L, ctypes
        self.gate, self.up, self.down, self.shared = gate, up, down, bool(shared)
        self.experts, self.tokens, self.topk, self.hidden, self.inter = experts, tokens, topk, hidden, inter
        self.rank, self.world, self.limit = rank, world, limit
        self.k = topk + (1 if self.shared else 0)
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        index = torch.device(dev).index if torch.device(dev).index is not None else torch.cuda.current_device()
        handle = (ctypes.c_uint8 * 64)()
        ptr = ctypes.c_void_p()
        L.check(L.lib().exl3_cpx_create(index, world, rank, tokens, self.k, hidden, inter, Q._TORCH_DT[dtype],
                                        ctypes.byref(ptr), handle))
        self._ptr = ptr
        mine = bytes(handle)
        if world > 1:
            every = [None] * world
            dist.all_gather_object(every, mine, group=group)
        else:
            every = [mine]
        buf = (ctypes.c_uint8 * (64 * world)).from_buffer_copy(b"".join(every))
        L.check(L.lib().exl3_cpx_connect(self._ptr, buf))
        self._opts = L.SwigluOpts(ctypes.sizeof(L.SwigluOpts), int(limit), 0)
        if self.shared:  # the [T, K + 1] slot lists when the caller passes [T, K]
            self.ext_inds = torch.full((tokens, self.k), experts, dtype=torch.int32, device=dev)
            self.ext_scores = torch.ones((tokens, self.k), dtype=torch.float32, device=dev)

    def forward(self, x: torch.Tensor, inds: torch.Tensor, scores: torch.Tensor, out: torch.Tensor | None = None,
                stream=None):
        if x.shape != (self.tokens, self.hidden) or inds.shape[0] != self.tokens or \
                inds.shape[1] not in (self.topk, self.k):
            raise ValueError("x [tokens, hidden] and inds [tokens, topk (+1 with the shared expert)]")
        if self.shared and inds.shape[1] == self.topk:
            self.ext_inds[:, :self.topk].copy_(inds)
            self.ext_scores[:, :self.topk].copy_(scores)
            inds, scores = self.ext_inds, self.ext_scores
        if out is None:
            out = torch.empty_like(x)
        ct = self._ct
        self._L.check(self._L.lib().exl3_swiglu_cp(
            self._ptr, ct.byref(self.gate.raw), ct.byref(self.up.raw), ct.byref(self.down.raw),
            ct.byref(Q._tensor(x)), ct.byref(Q._tensor(inds)), ct.byref(Q._tensor(scores)), ct.byref(self._opts),
            Q._stream(stream), ct.byref(Q._tensor(out))))
        return out

    def trace(self) -> list[list[int]]:
        """Per step: tokens' copies begin / done, every rank's tokens seen, gate|up done, every rank's gate|up seen,
        down and combine done, every rank's columns seen, copied out (ns)."""
        return read_trace(self._L.lib().exl3_cpx_trace, self._ptr)

    def close(self):
        if self._ptr:
            self._L.lib().exl3_cpx_destroy(self._ptr)
            self._ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class ExpertParallelSwiglu:
    """Routed SwiGLU experts split over the ranks.

    gate/up/down: this rank's banks -- experts [r E/world, (r+1) E/world), followed, when ``shared`` is set, by the
    shared expert (every rank holds it); tokens: the tokens each rank brings per step (the same on every rank, so every
    block of the exchange has the same size).  ``forward(x [T, D], inds, scores)`` returns out [T, D] in x's dtype:
    sum_k scores * expert(x) over the routed experts, plus the shared expert.  inds / scores are [T, K]; with a shared
    expert they may also be [T, K + 1] with the last column already the shared expert (id E, score 1).  A shared slot
    stays on the token's own rank and runs in the same swiglu call as the routed slots.

    ``exchange="nccl"`` moves the rows with two equal-split all_to_all_single calls (any backend, any ``ops``);
    ``exchange="peer"`` with this library's peer-memory kernels (:class:`PeerExpertExchange`, GPUs only).
    """

    def __init__(self, gate, up, down, experts: int, tokens: int, topk: int, hidden: int, rank: int, world: int,
                 dtype=torch.float16, device=None, group=None, shared: bool = False, limit: int = 0, ops=None,
                 exchange: str = "nccl"):
        if exchange not in ("nccl", "peer"):
            raise ValueError("exchange is 'nccl' or 'peer'")
        self.gate, self.up, self.down, self.shared = gate, up, down, bool(shared)
        self.experts, self.tokens, self.topk, self.hidden = experts, tokens, topk, hidden
        self.rank, self.world, self.group, self.limit = rank, world, group, limit
        self.ops = ops or CudaExpertOps()
        self.cap = ep_capacity(tokens, topk, experts, world, self.shared)
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        blk = (world, self.cap + 1, hidden)
        self.send = torch.empty(blk, dtype=dtype, device=dev)
        self.recv = torch.empty(blk, dtype=dtype, device=dev)
        self.ys = torch.empty(blk, dtype=torch.float32, device=dev)
        self.back = torch.empty(blk, dtype=torch.float32, device=dev)
        self.r_inds = torch.empty((world, self.cap + 1, 1), dtype=torch.int32, device=dev)
        self.r_scores = torch.empty((world, self.cap + 1, 1), dtype=torch.float32, device=dev)
        k = topk + (1 if self.shared else 0)
        self.back_slot = torch.empty((tokens, k), dtype=torch.int32, device=dev)
        self.peer = None
        if exchange == "peer":
            self.peer = PeerExpertExchange(rank, world, self.cap, hidden, dtype=dtype, device=dev, group=group)
        if self.shared:  # the [T, K + 1] slot lists when the caller passes [T, K]
            self.ext_inds = torch.full((tokens, k), experts, dtype=torch.int32, device=dev)
            self.ext_scores = torch.ones((tokens, k), dtype=torch.float32, device=dev)

    def _all_to_all(self, out, inp):
        if self.world == 1:
            out.copy_(inp)
        else:
            dist.all_to_all_single(out, inp, group=self.group)

    def forward(self, x: torch.Tensor, inds: torch.Tensor, scores: torch.Tensor, out: torch.Tensor | None = None):
        k = self.topk + (1 if self.shared else 0)
        if x.shape != (self.tokens, self.hidden) or inds.shape[0] != self.tokens or inds.shape[1] not in (self.topk, k):
            raise ValueError("x [tokens, hidden] and inds [tokens, topk (+1 with the shared expert)]")
        if self.shared and inds.shape[1] == self.topk:
            self.ext_inds[:, :self.topk].copy_(inds)
            self.ext_scores[:, :self.topk].copy_(scores)
            inds, scores = self.ext_inds, self.ext_scores
        if out is None:
            out = torch.empty_like(x)
        ops = self.ops
        if self.peer is not None:
            pe = self.peer
            pe.dispatch(x, inds, self.experts, self.shared, self.back_slot)
            pe.receive(self.recv, self.r_inds, self.r_scores)
            ops.swiglu(self.gate, self.up, self.down, self.recv, self.r_inds, self.r_scores, self.ys, self.limit)
            pe.give_back(self.ys)
            pe.combine(self.back_slot, scores, out)
            return out
        ops.dispatch(x, inds, self.experts, self.world, self.rank, self.shared, self.send, self.back_slot)
        self._all_to_all(self.recv, self.send)
        ops.unpack(self.recv, self.r_inds, self.r_scores)
        ops.swiglu(self.gate, self.up, self.down, self.recv, self.r_inds, self.r_scores, self.ys, self.limit)
        self._all_to_all(self.back, self.ys)
        ops.combine(self.back, self.back_slot, scores, out)
        return out
