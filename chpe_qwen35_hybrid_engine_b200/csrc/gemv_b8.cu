// 8-bit codes (fp16 operands): kernel variants of gemv_impl.cuh.
#include "gemv_impl.cuh"
namespace chpe {
cudaError_t launch_gemv_b8(const GemvPlan &plan, const GemvParams &p, int meta, cudaStream_t st) {
    return launch_gemv_bits<8, kLayoutF16, 32>(plan, p, meta, st);
}
}  // namespace chpe
