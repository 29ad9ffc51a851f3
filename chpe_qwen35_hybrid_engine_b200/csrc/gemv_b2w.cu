// 2-bit codes: kernel variants of gemv_impl.cuh with an epilogue every 128
// columns (group 128 and wider).
#include "gemv_impl.cuh"
namespace chpe {
cudaError_t launch_gemv_b2_wide(const GemvPlan &plan, const GemvParams &p, int meta, cudaStream_t st) {
    return launch_gemv_bits<2, kLayoutF16, 128>(plan, p, meta, st);
}
}  // namespace chpe
