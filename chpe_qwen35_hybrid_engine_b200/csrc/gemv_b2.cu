// 2-bit codes: kernel variants of gemv_impl.cuh with an epilogue every 64
// columns (the 128-column variants are in gemv_b2w.cu, compiled in parallel).
#include "gemv_impl.cuh"
namespace chpe {
cudaError_t launch_gemv_b2_wide(const GemvPlan &plan, const GemvParams &p, int meta, cudaStream_t st);
cudaError_t launch_gemv_b2(const GemvPlan &plan, const GemvParams &p, int meta, cudaStream_t st) {
    if (plan.e_cols == 64) return launch_gemv_bits<2, kLayoutF16, 64>(plan, p, meta, st);
    return launch_gemv_b2_wide(plan, p, meta, st);
}
}  // namespace chpe
