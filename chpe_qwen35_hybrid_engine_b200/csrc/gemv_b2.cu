// 2-bit codes: kernel variants of gemv_impl.cuh (epilogue every 64 or 128 columns).
#include "gemv_impl.cuh"
namespace chpe {
cudaError_t launch_gemv_b2(const GemvPlan &plan, const GemvParams &p, int meta, cudaStream_t st) {
    if (plan.e_cols == 64) return launch_gemv_bits<2, kLayoutF16, 64>(plan, p, meta, st);
    return launch_gemv_bits<2, kLayoutF16, 128>(plan, p, meta, st);
}
}  // namespace chpe
