// swiglu_decode.cu -- small-M (decode) SwiGLU kernel (not yet enabled).
#include "decode_kernels.h"

namespace llk_b200 {

int decode_max_m() { return 0; }
bool decode_supported(int64_t, int64_t, int64_t, int) { return false; }
DecodePlan decode_plan(int64_t, int64_t, int64_t, int) { return DecodePlan{0, 0, 64, 0, 1, 0, 0, 0}; }
size_t decode_workspace_bytes(int64_t, int64_t, int64_t, int) { return 0; }
cudaError_t decode_launch(const CUtensorMap &, const CUtensorMap &, const void *, int64_t, void *, int64_t, int,
                          int64_t, int64_t, int64_t, void *, int *, int, cudaStream_t) {
  return cudaErrorNotSupported;
}

}  // namespace llk_b200
