// gemv.cu -- launch planning and dispatch of the decode/verify GEMV
// (kernel in gemv_impl.cuh, instantiated per code width in gemv_b*.cu).
#include <atomic>

#include "gemv_impl.cuh"

namespace chpe {

// Instantiated in gemv_b8.cu, gemv_b4.cu, gemv_b2.cu and gemv_s8.cu.
cudaError_t launch_gemv_b8(const GemvPlan &plan, const GemvParams &p, int meta, cudaStream_t st);
cudaError_t launch_gemv_b4(const GemvPlan &plan, const GemvParams &p, int meta, cudaStream_t st);
cudaError_t launch_gemv_b2(const GemvPlan &plan, const GemvParams &p, int meta, cudaStream_t st);
cudaError_t launch_gemv_s8(const GemvPlan &plan, const GemvParams &p, int meta, cudaStream_t st);

// SMs of the current device (cached per device).
static int num_sms() {
    static std::atomic<int> cache[kMaxDevices];
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) return 148;
    int n = cache[dev].load(std::memory_order_relaxed);
    if (!n) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = 148;
        }
        cache[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

static int epilogue_cols(const DevMatrix &w) {
    if (w.layout == kLayoutS8) return 32;
    const int kc = chunk_cols(w.bits);
    const int grp = (w.n_groups == 1) ? kc : w.group;
    return std::min(grp, kc);
}

int plan_gemv(const DevMatrix &w, int M, int mode, bool xsplit, GemvPlan *plan, bool allow_xstream) {
    GemvPlan P;
    P.mode = mode;
    P.xsplit = xsplit;
    P.xmode = !xsplit ? 0 : (M <= 4 ? 2 : 1);
    P.e_cols = epilogue_cols(w);
    const int kc = chunk_cols(w.bits);
    const int ne = w.layout == kLayoutS8 ? 0 : kc / P.e_cols;
    P.n_sg = mode == 1 ? ceil_div(w.n_strips, kSG / 2) : ceil_div(w.n_strips, kSG);
    const size_t x_per_block =
        xfrag_bytes_per_block(w.layout, w.bits, M, xsplit) + (size_t)kChunksPerBlock * ne * 32;
    const size_t xmax = M <= 2 ? kXMaxBytes : kXMaxBytesWide;
    const int bpk_max = (int)std::max<size_t>(1, xmax / x_per_block);
    // Fewest K-slices whose activation fragments fit the staging budget, with
    // equal slices; the work counters balance the work, not the slicing.
    int n_ks = std::min(ceil_div(w.n_blocks, std::min(bpk_max, w.n_blocks)), kMaxKs);
    // More than two rows: the activations of all of K rarely fit beside a ring
    // with room for two CTAs per SM, and K-slices cost partial sums.  Instead
    // every ring stage can bring its block's activations along with its
    // weights (re-read from L2 by each strip group): one K-slice, a ring of 3
    // stages -- 2 when 3 would not let two CTAs share an SM.  Resident
    // activations stay where they fit two CTAs per SM in one K-slice, and on
    // matrices of fewer strip groups than half the SMs, which only K-slices
    // spread over the GPU (measured on B200 at M = 4 and 8, Q4 and Q8,
    // 1024..151936 rows, 4096..29568 columns).
    P.sms = num_sms();
    if (M > 2 && allow_xstream) {
        const int bpk_res = ceil_div(w.n_blocks, n_ks);
        const bool res_fits = ceil_div(w.n_blocks, bpk_res) == 1 &&
                              smem_layout(w.layout, w.bits, bpk_res, M, xsplit, P.e_cols, w.block_bytes).total <=
                                  kTwoCtaBytes;
        if (!res_fits && 2 * P.n_sg >= P.sms) {
            P.xstream = 1;
            n_ks = 1;
            P.nstages = 3;
            if (smem_layout(w.layout, w.bits, w.n_blocks, M, xsplit, P.e_cols, w.block_bytes, 1, 3).total >
                kTwoCtaBytes)
                P.nstages = 2;
        }
    }
    const int bpk = ceil_div(w.n_blocks, n_ks);
    n_ks = ceil_div(w.n_blocks, bpk);
    const size_t smem =
        smem_layout(w.layout, w.bits, bpk, M, xsplit, P.e_cols, w.block_bytes, P.xstream, P.nstages).total;
    // at most two CTAs per SM (the kernel's registers: __launch_bounds__(kThreads, 2));
    // each CTA also takes 1 KB of the SM's shared memory for itself
    const int per_sm = std::max(1, (int)std::min<size_t>(2, kSmemPerSm / (smem + 1024)));
    const int nb_last = w.n_blocks - (n_ks - 1) * bpk;
    // upper bound here; the launch recomputes the grid from the kernel's occupancy
    long gk = (long)P.sms * per_sm / n_ks;
    // at least ~4 blocks of work per CTA: small matrices get fewer CTAs
    gk = std::max<long>(1, std::min<long>(gk, std::max<long>(1, (long)P.n_sg * bpk / 4)));
    // Work units.  Whole strip groups (per K-slice) stream fastest -- long
    // runs per strip, no partial sums -- but balance poorly, so they come in
    // rounds of one per CTA covering about 70 % of a CTA's share, with at
    // least one whole strip group's worth of chunks left after a second
    // round (a CTA that draws a whole strip group late then still ends with
    // the others).  The rest is cut into chunks of bc blocks.  Units of one
    // or two blocks cost more in hand-offs and arrival counts than they gain
    // in balance, so chunks are four blocks unless a CTA has fewer than six
    // blocks of work.
    const long per_cta = (long)P.n_sg * bpk / gk;
    P.bc = per_cta >= 6 ? 4 : per_cta >= 3 ? 2 : 1;
    long rounds = per_cta * 7 / (10 * bpk);
    if (rounds >= 2 && per_cta - rounds * bpk < bpk) --rounds;
    P.n_whole = (int)std::min<long>(P.n_sg, rounds * gk);
    // More than two rows, partial sums are summed by chpe_qgemv_reduce_kernel
    // after the GEMV (an arrival count per unit measured slower).  Resident
    // activations: whole strip groups alone (mostly one CTA per SM with many
    // blocks of work), partial sums only across K-slices.  Streamed
    // activations: whole strip groups alone where K is short (at most 8
    // blocks) or where they give the CTAs of each SM about one unit in all,
    // otherwise the rounds of whole strip groups plus chunks.
    if (M > 2) {
        P.rmode = 1;
        if (!P.xstream || w.n_blocks <= 8 || (2 * P.n_sg >= gk && P.n_sg <= gk)) P.n_whole = P.n_sg;
    }
    P.cfull = ceil_div(bpk, P.bc);
    P.ctot = std::max((n_ks - 1) * P.cfull + ceil_div(nb_last, P.bc), n_ks);
    // static units cover the ring's first fill (fetched before the upstream kernel ends)
    P.pref = ceil_div(P.nstages, P.bc);
    if (n_ks == 1 && P.n_whole == P.n_sg) P.ctot = 1;  // every unit covers all of K: no partial sums
    P.items_min = slice_units(P.n_sg, P.n_whole, ceil_div(nb_last, P.bc));
    gk = std::min<long>(gk, P.items_min);
    P.n_ks = n_ks;
    P.bpk = bpk;
    P.grid = (int)(gk * n_ks);
    P.smem = smem;
    P.xf_bytes = (size_t)w.n_blocks * xfrag_bytes_per_block(w.layout, w.bits, M, xsplit);
    P.xs_bytes = w.layout == kLayoutF16 ? (size_t)w.n_blocks * kChunksPerBlock * ne * 32 : 0;
    P.ws_bytes = P.ctot > 1 ? (size_t)P.n_sg * P.ctot * kSG * 16 * M * 4 : 0;
    P.split_counters = P.n_sg + n_ks;
    *plan = P;
    return 0;
}

cudaError_t launch_gemv(const DevMatrix &w0, const DevMatrix *w1, const GemvPlan &plan, const GemvParams &p,
                        cudaStream_t st) {
    (void)w1;
    if (w0.layout == kLayoutS8) return launch_gemv_s8(plan, p, w0.meta_kind, st);
    switch (w0.bits) {
    case 8: return launch_gemv_b8(plan, p, w0.meta_kind, st);
    case 4: return launch_gemv_b4(plan, p, w0.meta_kind, st);
    case 2: return launch_gemv_b2(plan, p, w0.meta_kind, st);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace chpe
