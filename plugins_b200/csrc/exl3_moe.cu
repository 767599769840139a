// exl3_moe.cu -- routed SwiGLU experts (placeholder until the grouped expert kernels land).
#include "exl3_moe.h"

namespace exl3 {

exl3_verdict moe_reserve(int, int, int) { return {EXL3_OK, nullptr}; }

exl3_verdict moe_swiglu(const exl3_weight*, const exl3_weight*, const exl3_weight*, const exl3_tensor*,
                        const exl3_tensor*, const exl3_tensor*, const exl3_swiglu_opts*, void*, exl3_tensor*) {
  return {EXL3_UNSUPPORTED, "exl3_b200: routed SwiGLU is not built yet"};
}

}  // namespace exl3
