// exl3_moe.h -- the routed SwiGLU expert path (exl3_moe.cu).
#pragma once
#include "../../include/exl3_b200.h"

namespace exl3 {

// Grows the device's MoE workspace for banks of this shape (load time).
exl3_verdict moe_reserve(int device, int in_features, int out_features);

exl3_verdict moe_swiglu(const exl3_weight* gate, const exl3_weight* up, const exl3_weight* down, const exl3_tensor* x,
                        const exl3_tensor* inds, const exl3_tensor* scores, const exl3_swiglu_opts* opts, void* stream,
                        exl3_tensor* out);

// The routed experts at prompt widths on the tensor cores (exl3_moe_prefill.cu): a workspace for banks of up to
// `experts` experts of hidden x inter and calls of up to max_slots (token, k) slots (0 frees it).
exl3_verdict moe_prefill_reserve(int device, int experts, int hidden, int inter, int max_slots, uint64_t* bytes);
bool moe_prefill_serves(int device, int experts, int hidden, int inter, int64_t slots);
exl3_verdict moe_prefill_run(const exl3_weight* gate, const exl3_weight* up, const exl3_weight* down,
                             const exl3_tensor* x, const exl3_tensor* inds, const exl3_tensor* scores, float limit,
                             void* stream, exl3_tensor* out);
constexpr int64_t kPrefillMinSlots = 1024;  // wider calls take the prefill path where a workspace serves them

// The routed experts with the shared expert folded into the combine (exl3_swiglu_shared).
exl3_verdict moe_swiglu_shared(const exl3_weight* gate, const exl3_weight* up, const exl3_weight* down,
                               const exl3_tensor* x, const exl3_tensor* inds, const exl3_tensor* scores,
                               const exl3_shared_swiglu* opts, void* stream, exl3_tensor* out);

}  // namespace exl3
