// gemv.cu -- launch planning and dispatch of the decode/verify GEMV
// (kernel in gemv_impl.cuh, instantiated per code width in gemv_b*.cu).
#include "gemv_impl.cuh"

namespace chpe {

// Instantiated in gemv_b8.cu, gemv_b4.cu, gemv_b2.cu and gemv_s8.cu.
cudaError_t launch_gemv_b8(const GemvPlan &plan, const GemvParams &p, int meta, cudaStream_t st);
cudaError_t launch_gemv_b4(const GemvPlan &plan, const GemvParams &p, int meta, cudaStream_t st);
cudaError_t launch_gemv_b2(const GemvPlan &plan, const GemvParams &p, int meta, cudaStream_t st);
cudaError_t launch_gemv_s8(const GemvPlan &plan, const GemvParams &p, int meta, cudaStream_t st);

static int num_sms() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = 148;
        }
    }
    return n;
}

static int epilogue_cols(const DevMatrix &w) {
    if (w.layout == kLayoutS8) return 32;
    const int kc = chunk_cols(w.bits);
    const int grp = (w.n_groups == 1) ? kc : w.group;
    return std::min(grp, kc);
}

int plan_gemv(const DevMatrix &w, int M, int mode, bool xsplit, GemvPlan *plan) {
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
    // equal slices; the stream-K partition balances the work, not the slicing.
    int n_ks = std::min(ceil_div(w.n_blocks, std::min(bpk_max, w.n_blocks)), kMaxKs);
    const int bpk = ceil_div(w.n_blocks, n_ks);
    n_ks = ceil_div(w.n_blocks, bpk);
    const size_t smem = smem_layout(w.layout, w.bits, bpk, M, xsplit, P.e_cols, w.block_bytes).total;
    const int per_sm = std::max(1, (int)std::min<size_t>(4, kSmemBudget / (smem + 1024)));
    // no CTA may get an empty range (the partial counts assume none): at most
    // as many CTAs per slice as the shortest slice has items
    const int nb_last = w.n_blocks - (n_ks - 1) * bpk;
    const long items = (long)P.n_sg * nb_last;
    P.items_min = items;
    P.sms = num_sms();
    // upper bound here; the launch recomputes the grid from the kernel's occupancy
    long gk = std::min<long>((long)P.sms * per_sm / n_ks, items);
    // at least ~4 items per CTA: small matrices get fewer, longer ranges
    gk = std::min<long>(gk, std::max<long>(1, (long)P.n_sg * bpk / 4));
    gk = std::max<long>(1, gk);
    P.n_ks = n_ks;
    // Split-K partials are summed by a second, fully parallel kernel: with
    // several K-slices, or more than two rows, the sums at the end of a CTA's
    // range would keep its epilogue warp (and then its MMA warps) waiting on
    // L2 round trips.  With one slice only the few strip groups cut by range
    // boundaries have partials; the last CTA to arrive sums those.
    P.rmode = (M > 2 || n_ks > 1) ? 1 : 0;
    P.bpk = bpk;
    P.grid = (int)(gk * n_ks);
    P.smem = smem;
    // CTAs of one slice touching one strip group: at most gk / n_sg + 2
    P.maxp = n_ks * (int)(gk / P.n_sg + 2);
    P.xf_bytes = (size_t)w.n_blocks * xfrag_bytes_per_block(w.layout, w.bits, M, xsplit);
    P.xs_bytes = w.layout == kLayoutF16 ? (size_t)w.n_blocks * kChunksPerBlock * ne * 32 : 0;
    P.ws_bytes = (size_t)P.n_sg * P.maxp * kSG * 16 * 8 * 4;
    P.split_counters = P.n_sg;
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
