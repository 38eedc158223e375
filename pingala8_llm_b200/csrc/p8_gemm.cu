// p8_gemm.cu -- placeholder until the tcgen05 GEMM lands: ncols > 1 runs the table GEMV per column.
#include "p8_internal.h"

namespace p8 {
bool gemm_supported(const p8_tensor *, int64_t) { return false; }
size_t gemm_workspace(const p8_tensor *, int64_t) { return 0; }
p8_status launch_gemm(const p8_tensor *, const float *, int64_t, int64_t, float *, int64_t, void *, size_t, cudaStream_t) {
    return P8_ERR_UNSUPPORTED;
}
}  // namespace p8
