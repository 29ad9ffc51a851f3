// common.cuh -- sm_100a device helpers shared by the CHPE kernels:
// mbarrier + bulk-copy (TMA engine) wrappers with bounded waits, warp-level
// MMA wrappers and the activation-fragment layout constants.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

namespace chpe {

// A bounded wait gives up after this many nanoseconds of %globaltimer, records
// an error code in the kernel's error word and lets the kernel return.
constexpr unsigned long long kWaitTimeoutNs = 1000000000ull;  // 1 s

enum KernelError : int { kErrNone = 0, kErrWaitFull = 1, kErrWaitEmpty = 2, kErrWaitPrologue = 3 };

// Host side: every kernel launch of the library is counted (process-wide,
// relaxed atomic; defined in abi.cu, read through chpe_kernel_launches).
void note_launch();

// Host side: per-device launch state of one kernel.  A kernel's dynamic
// shared-memory limit (cudaFuncSetAttribute) and its occupancy belong to a
// device context, so a process that launches on several GPUs sets and
// queries them once per device; the lock serialises host threads.
constexpr int kMaxDevices = 64;
struct KernelDeviceState {
    std::mutex mu;
    bool attr_set[kMaxDevices] = {};
    size_t occ_smem[kMaxDevices][8] = {};
    int occ_val[kMaxDevices][8] = {};
};
// The current device (0 when the runtime cannot say; the device's calls then fail anyway).
inline int current_device() {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess) {
        cudaGetLastError();
        d = 0;
    }
    return d;
}
// Sets the kernel's dynamic shared-memory limit to `smem` bytes on the current
// device once, and returns (through *occ, when non-null) its resident blocks
// per SM for `threads` threads and `smem` bytes, cached per device and size.
template <typename Kern>
cudaError_t kernel_prepare(KernelDeviceState &st, Kern kern, int threads, size_t smem_limit, size_t smem, int *occ) {
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(st.mu);
    if (!st.attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_limit);
        if (e != cudaSuccess) return e;
        st.attr_set[dev] = true;
    }
    if (!occ) return cudaSuccess;
    *occ = 0;
    for (int i = 0; i < 8 && st.occ_smem[dev][i]; ++i)
        if (st.occ_smem[dev][i] == smem) *occ = st.occ_val[dev][i];
    if (!*occ) {
        int o = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, kern, threads, smem) != cudaSuccess || o < 1) {
            cudaGetLastError();
            o = 1;
        }
        for (int i = 0; i < 8; ++i)
            if (!st.occ_smem[dev][i]) {
                st.occ_smem[dev][i] = smem;
                st.occ_val[dev][i] = o;
                break;
            }
        *occ = o;
    }
    return cudaSuccess;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Makes mbarrier initialisation visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for the phase with the given parity to complete; false after the
// timeout (never spins forever).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_timer_ns();
    while (true) {
#pragma unroll 1
        for (int i = 0; i < 32; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (global_timer_ns() - t0 > kWaitTimeoutNs) return false;
    }
}

// L2 policy for streamed-once weight bytes: evict first, so activations,
// metadata and split-K partials stay resident.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// 1-D bulk copy global -> this CTA's shared memory, completing `bytes`
// transaction bytes on `bar`.  dst/src 16-byte aligned, bytes % 16 == 0.
// Every bulk copy in this library fills only the issuing CTA's own shared memory.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void bulk_g2s_hint(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Named barrier over `nthreads` threads (id 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// (a & b) | c in one LOP3.
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// D(16x8 f32) += A(16x16 f16, row) * B(16x8 f16, col)
__device__ __forceinline__ void mma_f16_m16n8k16(float d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                 uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D(16x8 s32) += A(16x32 s8, row) * B(32x8 s8, col)
__device__ __forceinline__ void mma_s8_m16n8k32(int d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Atomic add at GPU scope with acquire-release semantics; returns the old
// value.  The release half publishes the writes that the issuing warp made
// before a __syncwarp; the acquire half makes the other CTAs' writes that
// preceded their own releases visible to this warp (after a __syncwarp).
__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned *p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Programmatic dependent launch: wait for the upstream grid's memory.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dependents_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Start of every small kernel of the library: let the next kernel on the
// stream be scheduled right away (its own wait holds it back until this grid
// has finished), then wait for the previous grid's results before touching
// global memory.  The next kernel thereby launches, and a GEMV starts
// fetching weights, while this one runs.
__device__ __forceinline__ void pdl_begin() {
    grid_dependents_launch();
    grid_dependency_wait();
}

// Launch with programmatic stream serialization (the kernel calls pdl_begin
// or grid_dependency_wait before it reads or writes anything another kernel
// produces or consumes).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    note_launch();
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// As launch_pdl, for a kernel whose CTAs form clusters of cluster_x along x.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, unsigned cluster_x, size_t smem,
                               cudaStream_t st, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster_x;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    note_launch();
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// silu(g) = g / (1 + exp(-g)) (src/kernels/neon.zig:705-712), with exp taken
// in double precision and rounded to float: that is the correctly rounded
// float exp except in about one case in 10^9, so every implementation that
// does the same (the oracle's, on the host) gets the same bits.  The W8A8
// path re-quantizes every activation row to int8, where a last-bit
// difference can flip a rounding and grow from there.
constexpr int kCommMaxRanksDev = 8;  // ranks of a tensor-parallel group (= kCommMaxRanks of internal.h)

// Tagged words of the tensor-parallel exchanges: one 64-bit store carries a
// value and the epoch of its exchange (value bits | epoch << 32); naturally
// aligned 64-bit accesses are single-copy atomic, so a reader sees both or
// neither.  System scope: the writer and the reader sit on different GPUs.
__device__ __forceinline__ void st_tagged(unsigned long long *p, float v, unsigned epoch) {
    const unsigned long long w = ((unsigned long long)epoch << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_tagged(const unsigned long long *p) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
// Word w of p, loaded already, once it carries `epoch` (reloading p until
// it does); gives up (ok = false, returns 0) when kWaitTimeoutNs have passed
// since t0, or at once if ok is false.
__device__ __forceinline__ float settle_tagged(const unsigned long long *p, unsigned long long w, unsigned epoch,
                                               unsigned long long t0, bool &ok) {
    if (!ok) return 0.0f;
    while ((unsigned)(w >> 32) != epoch) {
        if (global_timer_ns() - t0 > kWaitTimeoutNs) {
            ok = false;
            return 0.0f;
        }
        __nanosleep(20);
        w = ld_tagged(p);
    }
    return __uint_as_float((unsigned)w);
}

// For each of NV values (index idx[j], valid[j]): the sum over ranks
// r < world, in rank order, of value idx[j] of rank r's slot (own[j] for this
// rank), into sums[j].  Every peer word of every value is loaded before any
// is checked, so all their L2 round trips overlap.
template <int NV>
__device__ __forceinline__ void sum_tagged(const unsigned long long *slots, size_t rstride, const size_t (&idx)[NV],
                                           const bool (&valid)[NV], int world, int rank, const float (&own)[NV],
                                           unsigned epoch, unsigned long long t0, bool &ok, float (&sums)[NV]) {
    unsigned long long w[NV][kCommMaxRanksDev];
#pragma unroll
    for (int j = 0; j < NV; ++j)
#pragma unroll
        for (int r = 0; r < kCommMaxRanksDev; ++r)
            if (valid[j] && r < world && r != rank) w[j][r] = ld_tagged(slots + (size_t)r * rstride + idx[j]);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        float sum = 0.0f;
#pragma unroll
        for (int r = 0; r < kCommMaxRanksDev; ++r)
            if (valid[j] && r < world)
                sum += r == rank ? own[j] : settle_tagged(slots + (size_t)r * rstride + idx[j], w[j][r], epoch, t0, ok);
        sums[j] = sum;
    }
}

__device__ __forceinline__ float exp_rn(float x) { return (float)exp((double)x); }
__device__ __forceinline__ float silu_f(float g) { return __fdiv_rn(g, __fadd_rn(1.0f, exp_rn(-g))); }

}  // namespace chpe
