// Host-only driver for the GEMV launch planner (no kernel is launched): for a
// sweep of shapes, formats and activation counts it checks that planning ends
// and that every plan is consistent.  Built and run by tests/test_plan.py.
#include <cstdio>
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
        for (int xs = 0; xs < 2; ++xs) {
            int group = f.group ? f.group : K;
            if (f.layout == kLayoutF16 && K % group) continue;
            if (f.layout == kLayoutS8 && xs) continue;
            DevMatrix m = make(f.bits, f.layout, f.meta, N, K, group);
            GemvPlan P;
            plan_gemv(m, M, mode, xs, &P);
            ++plans;
            bool ok = P.n_ks >= 1 && P.n_ks <= kMaxKs && P.bpk >= 1 && (long)P.bpk * P.n_ks >= m.n_blocks &&
                      (long)P.bpk * (P.n_ks - 1) < m.n_blocks && P.grid >= P.n_ks && P.grid % P.n_ks == 0 &&
                      P.smem <= (size_t)kSmemBudget;
            // the stream-K partition covers every item once and no strip group
            // collects more partial sums than its workspace slots
            const int Gk = P.grid / P.n_ks;
            for (int k = 0; k < P.n_ks && ok; ++k) {
                const int nbk = std::min(P.bpk, m.n_blocks - k * P.bpk);
                const long T = (long)P.n_sg * nbk;
                ok = part_start(T, Gk, 0) == 0 && part_start(T, Gk, Gk) == T;
                for (int j = 0; j < Gk && ok; ++j) ok = part_start(T, Gk, j) < part_start(T, Gk, j + 1);
                for (long x = 0; x < T && ok; x += std::max<long>(1, T / 97)) {
                    const int o = part_owner(T, Gk, x);
                    ok = part_start(T, Gk, o) <= x && x < part_start(T, Gk, o + 1);
                }
            }
            for (int sg = 0; sg < P.n_sg && ok; sg += std::max(1, P.n_sg / 61)) {
                int tot = 0;
                for (int k = 0; k < P.n_ks; ++k)
                    tot += part_count(sg, std::min(P.bpk, m.n_blocks - k * P.bpk), P.n_sg, Gk);
                ok = tot <= P.maxp;
            }
            if (!ok) {
                ++bad;
                if (bad < 20) printf("BAD N=%d K=%d bits=%d M=%d mode=%d n_ks=%d bpk=%d grid=%d smem=%zu\n", N, K, f.bits,
                                     M, mode, P.n_ks, P.bpk, P.grid, P.smem);
            }
        }
    printf("plans=%ld bad=%ld\n", plans, bad);
    return bad ? 1 : 0;
}
