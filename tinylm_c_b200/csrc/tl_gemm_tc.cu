// tl_gemm_tc.cu -- tensor-core (tcgen05, 3xTF32) GEMM engine.  Placeholder
// until the engine lands: reports every shape as unsupported.
#include "tl_gemm.cuh"

namespace tl {
bool gemm_tc_supported(GemmOp, const float *, const float *, const float *, int, int, int) { return false; }
int gemm_tc(DeviceCtx *, GemmOp, float *, const float *, const float *, int, int, int) {
  return set_error(TL_EINVAL, "tensor-core engine not built");
}
}  // namespace tl
