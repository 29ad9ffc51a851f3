// Host-only driver for the GEMV launch planner (no kernel is launched): for a
// sweep of shapes, formats and activation counts it checks that planning ends
// and that every plan is consistent.  Built and run by tests/test_plan.py.
#include <cstdio>
#include <vector>
#include "../chpe_qwen35_hybrid_engine_b200/csrc/gemv.cu"

using namespace chpe;

// The planner is host code; the kernel launchers are never called here.
namespace chpe {
cudaError_t launch_gemv_b8(const GemvPlan &, const GemvParams &, int, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t launch_gemv_b4(const GemvPlan &, const GemvParams &, int, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t launch_gemv_b2(const GemvPlan &, const GemvParams &, int, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t launch_gemv_s8(const GemvPlan &, const GemvParams &, int, cudaStream_t) { return cudaErrorNotSupported; }
}  // namespace chpe

static DevMatrix make(int bits, int layout, int meta, int N, int K, int group) {
    DevMatrix m;
    m.bits = bits; m.layout = layout; m.meta_kind = meta; m.N = N; m.K = K;
    m.n_strips = ceil_div(N, kStripRows);
    m.span = block_cols(bits);
    m.n_blocks = ceil_div(K, m.span);
    m.group = group;
    m.n_groups = layout == kLayoutS8 ? 0 : K / group;
    if (meta == kMetaNone) { m.gpb = 0; m.gshift = -1; }
    else if (m.n_groups == 1 || group > m.span) { m.gpb = 1; m.gshift = -1; }
    else { m.gpb = m.span / group; int s = 0; while ((1 << s) < group) ++s; m.gshift = s; }
    m.block_bytes = kBlockCodeBytes + 16 * m.gpb * meta_bytes(meta);
    return m;
}

int main() {
    const int Ns[] = {1, 16, 100, 1000, 1024, 4096, 6144, 8192, 12288, 29568, 151936, 152064};
    const int Ks[] = {32, 64, 960, 1000, 2048, 4096, 8192, 12288, 29568};
    struct F { int bits, layout, meta, group; } fmts[] = {
        {8, kLayoutS8, kMetaNone, 0}, {8, kLayoutF16, kMetaS16, 32}, {4, kLayoutF16, kMetaSZ16, 64},
        {2, kLayoutF16, kMetaSZ16, 64}, {2, kLayoutF16, kMetaS16, 128}, {4, kLayoutF16, kMetaF32, 0}};
    long plans = 0, bad = 0;
    for (int N : Ns) for (int K : Ks) for (auto f : fmts) for (int M = 1; M <= 8; ++M) for (int mode = 0; mode < 2; ++mode)
        for (int xs = 0; xs < 2; ++xs) for (int ax = 0; ax < 2; ++ax) {
            int group = f.group ? f.group : K;
            if (f.layout == kLayoutF16 && K % group) continue;
            if (f.layout == kLayoutS8 && xs) continue;
            DevMatrix m = make(f.bits, f.layout, f.meta, N, K, group);
            GemvPlan P;
            plan_gemv(m, M, mode, xs, &P, ax != 0);
            ++plans;
            bool ok = P.n_ks >= 1 && P.n_ks <= kMaxKs && P.bpk >= 1 && (long)P.bpk * P.n_ks >= m.n_blocks &&
                      (long)P.bpk * (P.n_ks - 1) < m.n_blocks && P.grid >= P.n_ks && P.grid % P.n_ks == 0 &&
                      P.smem <= (size_t)kSmemBudget && (P.xstream == 0 || (M > 2 && P.n_ks == 1)) &&
                      P.nstages >= 2 && P.nstages <= kStages;
            // the work units (static ones, then drawn ones, CTAs interleaved
            // in a fixed pseudo-random order) cover every block of every strip
            // group exactly once, every strip group's arrival count reaches its
            // chunk count exactly, and the last draw of each slice is the one
            // that resets its counter
            ok = ok && P.bc >= 1 && P.pref * P.bc >= P.nstages && P.ctot >= P.n_ks && P.n_whole >= 0 &&
                 P.n_whole <= P.n_sg && (P.ctot == 1 || P.ws_bytes >= (size_t)P.n_sg * P.ctot * kSG * 16 * M * 4) &&
                 P.split_counters == P.n_sg + P.n_ks;
            const int Gk = P.grid / P.n_ks;
            const bool deep = (N * (long)K) <= (1L << 26);  // full coverage check on the smaller shapes
            std::vector<int> seen, arrivals(P.n_sg, 0);
            if (ok && deep) seen.assign((size_t)P.n_sg * m.n_blocks, 0);
            for (int k = 0; k < P.n_ks && ok; ++k) {
                const int nbk = std::min(P.bpk, m.n_blocks - k * P.bpk);
                const int C = unit_chunks(nbk, P.bc);
                const int U = slice_units(P.n_sg, P.n_whole, C);
                const int PS = static_units(P.n_whole, Gk, nbk, P.pref, P.nstages);
                const long ntot = grabs_total(U, PS, Gk);
                ok = Gk <= U;
                auto take = [&](long u) {
                    const Unit un = unit_of((int)u, nbk, C, k, P.n_ks, P.n_whole, P.bc, P.cfull, P.ctot);
                    ok = un.sg < P.n_sg && un.gc < un.ctot && un.ctot <= P.ctot && un.bs < un.be && un.be <= nbk &&
                         (un.sg < P.n_whole ? un.ctot == P.n_ks : un.ctot == P.ctot);
                    if (ok) arrivals[un.sg]++;
                    if (ok && deep)
                        for (int b = un.bs; b < un.be; ++b) seen[(size_t)un.sg * m.n_blocks + k * P.bpk + b]++;
                };

                long ctr = 0, draws = 0;
                int resets = 0;
                std::vector<int> pi(Gk, 0);
                std::vector<char> done(Gk, 0);
                int left = Gk;
                unsigned rng = 12345u + k;
                while (left > 0 && ok) {
                    rng = rng * 1103515245u + 12345u;
                    int j = (int)((rng >> 8) % (unsigned)Gk);
                    while (done[j]) j = (j + 1) % Gk;
                    long u;
                    if (pi[j] < PS && j + (long)pi[j] * Gk < U) {
                        u = j + (long)(pi[j]++) * Gk;
                    } else {
                        pi[j] = PS;
                        const long d = ctr++;
                        ++draws;
                        u = (long)PS * Gk + d;
                        if (u >= U) {
                            if (d == ntot - 1) { ++resets; ctr = 0; }
                            done[j] = 1;
                            --left;
                            continue;
                        }
                    }
                    take(u);
                }
                ok = ok && resets == 1 && ctr == 0 && draws == ntot;
            }
            if (ok && deep)
                for (int v : seen) ok = ok && v == 1;
            for (int sg = 0; sg < P.n_sg && ok; ++sg) ok = arrivals[sg] == (sg < P.n_whole ? P.n_ks : P.ctot);
            if (!ok) {
                ++bad;
                if (bad < 20) printf("BAD N=%d K=%d bits=%d M=%d mode=%d xstream=%d n_ks=%d bpk=%d grid=%d smem=%zu\n", N, K, f.bits,
                                     M, mode, P.xstream, P.n_ks, P.bpk, P.grid, P.smem);
            }
        }
    printf("plans=%ld bad=%ld\n", plans, bad);
    return bad ? 1 : 0;
}
