// 4-bit codes: kernel variants of gemv_impl.cuh.
#include "gemv_impl.cuh"
namespace chpe {
cudaError_t launch_gemv_b4(const GemvPlan &plan, const GemvParams &p, int meta, cudaStream_t st) {
    return launch_gemv_bits<4, kLayoutF16, 64>(plan, p, meta, st);
}
}  // namespace chpe
