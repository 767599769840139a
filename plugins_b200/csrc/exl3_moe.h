// exl3_moe.h -- the routed SwiGLU expert path (exl3_moe.cu).
#pragma once
#include "../../include/exl3_b200.h"

namespace exl3 {

// Grows the device's MoE workspace for banks of this shape (load time).
exl3_verdict moe_reserve(int device, int in_features, int out_features);

exl3_verdict moe_swiglu(const exl3_weight* gate, const exl3_weight* up, const exl3_weight* down, const exl3_tensor* x,
                        const exl3_tensor* inds, const exl3_tensor* scores, const exl3_swiglu_opts* opts, void* stream,
                        exl3_tensor* out);

// The routed experts with the shared expert folded into the combine (exl3_swiglu_shared).
exl3_verdict moe_swiglu_shared(const exl3_weight* gate, const exl3_weight* up, const exl3_weight* down,
                               const exl3_tensor* x, const exl3_tensor* inds, const exl3_tensor* scores,
                               const exl3_shared_swiglu* opts, void* stream, exl3_tensor* out);

}  // namespace exl3
