// int8 x int8 (W8A8): kernel variants of gemv_impl.cuh.
#include "gemv_impl.cuh"
namespace chpe {
cudaError_t launch_gemv_s8(const GemvPlan &plan, const GemvParams &p, int meta, cudaStream_t st) {
    (void)meta;
    return launch_gemv_bits<8, kLayoutS8, 32>(plan, p, kMetaNone, st);
}
}  // namespace chpe
