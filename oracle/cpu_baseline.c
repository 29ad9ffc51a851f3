/*
 * cpu_baseline.c -- the reference engine's CPU decode step, restated in C for
 * timing on the GPU host's cores.
 *
 * TEST INFRASTRUCTURE ONLY: bench.py's cpu_baseline leg and its
 * `--impl reference` arm load it (the reference itself is Zig 0.17-dev, which
 * this image cannot build).  It is never part of the product library.
 *
 * What it restates (x86 branches, compiled -O3 -march=native so the portable
 * vector code vectorises as Zig's @Vector code does):
 *   * the worker pool, src/engine.zig:94-174: NUM_WORKERS - 1 persistent
 *     threads spinning on a generation counter, the caller as worker 0;
 *   * the row split, src/engine.zig:188-192: rows / NUM_WORKERS per worker,
 *     the last worker takes the remainder; 4 rows at a time, then the tail;
 *   * dotProductInt8QuadRowNeon / dotProductInt8Neon, src/kernels/neon.zig:
 *     54-255 (x86 `else`: 16-lane int32 accumulators, then the tail);
 *   * dotProductInt8GateUpSwiGLUNeon, :261-350;
 *   * quantizeActivationInt8 :644-670, rmsnorm :673-702;
 *   * Qwen35Engine.step, src/engine.zig:583-734, with its stand-in mixers
 *     (:619-623 attention = V broadcast, :651-654 Gated DeltaNet = qkv * silu(z));
 *   * for the 4-bit 72B-shape model, the fp32 dotTileRow4Bit loop of
 *     src/qwen72b_engine.zig:135-148 (one add per byte: sum += w0*x0 + w1*x1)
 *     over unsigned codes with an fp16 scale and zero per 64 columns, in the
 *     same step structure (80 GQA layers, head-aligned attention stand-in).
 * Weights are seeded pseudo-random bytes filled in parallel.
 */
#include <math.h>
#include <pthread.h>
#include <sched.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef _Float16 f16;

#if defined(__x86_64__) || defined(__i386__)
#define CPU_RELAX() __builtin_ia32_pause()
#else
#define CPU_RELAX() ((void)0)
#endif

/* ---- worker pool (src/engine.zig:94-174) --------------------------------- */
typedef void (*task_fn)(int worker, int nworkers, void *arg);
typedef struct {
    int n;
    pthread_t th[256];
    _Atomic unsigned generation;
    _Atomic unsigned done[256];
    _Atomic int shutdown;
    task_fn fn;
    void *arg;
} pool_t;

typedef struct {
    pool_t *p;
    int id;
} worker_arg;
static worker_arg g_wargs[256];

static void *worker_loop(void *a) {
    worker_arg *wa = (worker_arg *)a;
    pool_t *p = wa->p;
    unsigned last = 0;
    for (;;) {
        unsigned cur = atomic_load_explicit(&p->generation, memory_order_acquire);
        while (cur == last) {
            if (atomic_load_explicit(&p->shutdown, memory_order_acquire)) return NULL;
            CPU_RELAX();
            cur = atomic_load_explicit(&p->generation, memory_order_acquire);
        }
        if (atomic_load_explicit(&p->shutdown, memory_order_acquire)) return NULL;
        p->fn(wa->id, p->n, p->arg);
        last = cur;
        atomic_store_explicit(&p->done[wa->id], cur, memory_order_release);
    }
}

pool_t *cb_pool_create(int n) {
    if (n < 1) n = 1;
    if (n > 256) n = 256;
    pool_t *p = (pool_t *)calloc(1, sizeof(pool_t));
    p->n = n;
    for (int i = 1; i < n; ++i) {
        g_wargs[i].p = p;
        g_wargs[i].id = i;
        pthread_create(&p->th[i], NULL, worker_loop, &g_wargs[i]);
    }
    return p;
}

static void pool_run(pool_t *p, task_fn fn, void *arg) {
    p->fn = fn;
    p->arg = arg;
    unsigned gen = atomic_fetch_add_explicit(&p->generation, 1u, memory_order_acq_rel) + 1u;
    fn(0, p->n, arg);
    for (int i = 1; i < p->n; ++i)
        while (atomic_load_explicit(&p->done[i], memory_order_acquire) != gen) CPU_RELAX();
}

void cb_pool_destroy(pool_t *p) {
    atomic_store(&p->shutdown, 1);
    atomic_fetch_add(&p->generation, 1u);
    for (int i = 1; i < p->n; ++i) pthread_join(p->th[i], NULL);
    free(p);
}

/* ---- int8 dots, x86 branches of src/kernels/neon.zig ---------------------- */
static inline float dot_i8(const int8_t *w, const int8_t *x, size_t n, float norm) {
    int32_t acc[16] = {0};
    size_t i = 0;
    for (; i + 16 <= n; i += 16)
        for (int j = 0; j < 16; ++j) acc[j] += (int32_t)w[i + j] * (int32_t)x[i + j];
    int32_t a = 0;
    for (int j = 0; j < 16; ++j) a += acc[j];
    for (; i < n; ++i) a += (int32_t)w[i] * (int32_t)x[i];
    return (float)a * norm;
}

static inline void dot_i8_quad(const int8_t *w0, const int8_t *w1, const int8_t *w2, const int8_t *w3,
                               const int8_t *x, size_t n, float norm, float *out) {
    int32_t a0[16] = {0}, a1[16] = {0}, a2[16] = {0}, a3[16] = {0};
    size_t i = 0;
    for (; i + 16 <= n; i += 16)
        for (int j = 0; j < 16; ++j) {
            const int32_t xv = x[i + j];
            a0[j] += (int32_t)w0[i + j] * xv;
            a1[j] += (int32_t)w1[i + j] * xv;
            a2[j] += (int32_t)w2[i + j] * xv;
            a3[j] += (int32_t)w3[i + j] * xv;
        }
    int32_t s0 = 0, s1 = 0, s2 = 0, s3 = 0;
    for (int j = 0; j < 16; ++j) {
        s0 += a0[j];
        s1 += a1[j];
        s2 += a2[j];
        s3 += a3[j];
    }
    for (; i < n; ++i) {
        const int32_t xv = x[i];
        s0 += (int32_t)w0[i] * xv;
        s1 += (int32_t)w1[i] * xv;
        s2 += (int32_t)w2[i] * xv;
        s3 += (int32_t)w3[i] * xv;
    }
    out[0] = (float)s0 * norm;
    out[1] = (float)s1 * norm;
    out[2] = (float)s2 * norm;
    out[3] = (float)s3 * norm;
}

static inline float silu(float g) { return g / (1.0f + expf(-g)); }

typedef struct {
    const int8_t *w, *wu;  /* wu: up weights of the fused gate/up, else NULL */
    float sw, su, sx;
    const int8_t *x;
    size_t rows, cols;
    float *out;
} gemv_i8_job;

/* gemvWorkerFn / gemvGateUpWorkerFn, src/engine.zig:188-313 */
static void gemv_i8_task(int wid, int nw, void *a) {
    gemv_i8_job *j = (gemv_i8_job *)a;
    const size_t per = j->rows / (size_t)nw;
    const size_t r0 = (size_t)wid * per, r1 = wid == nw - 1 ? j->rows : r0 + per;
    if (j->wu) {
        const float ng = j->sw * j->sx, nu = j->su * j->sx;
        for (size_t r = r0; r < r1; ++r) {
            const float g = dot_i8(j->w + r * j->cols, j->x, j->cols, ng);
            const float u = dot_i8(j->wu + r * j->cols, j->x, j->cols, nu);
            j->out[r] = silu(g) * u;
        }
        return;
    }
    const float norm = j->sw * j->sx;
    size_t r = r0;
    for (; r + 4 <= r1; r += 4)
        dot_i8_quad(j->w + r * j->cols, j->w + (r + 1) * j->cols, j->w + (r + 2) * j->cols, j->w + (r + 3) * j->cols,
                    j->x, j->cols, norm, j->out + r);
    for (; r < r1; ++r) j->out[r] = dot_i8(j->w + r * j->cols, j->x, j->cols, norm);
}

/* ---- 4-bit rows: the dotTileRow4Bit loop (src/qwen72b_engine.zig:135-148) --
 * one fp32 add per byte, w = (nibble - zero) * scale with the group's fp16
 * scale and zero (64 columns per group). */
typedef struct {
    const uint8_t *codes;
    const uint16_t *s, *z;
    const float *x;
    size_t rows, cols;
    float *out;
} gemv_q4_job;

static void gemv_q4_task(int wid, int nw, void *a) {
    gemv_q4_job *j = (gemv_q4_job *)a;
    const size_t per = j->rows / (size_t)nw;
    const size_t r0 = (size_t)wid * per, r1 = wid == nw - 1 ? j->rows : r0 + per;
    const size_t ng = j->cols / 64, rb = j->cols / 2;
    for (size_t r = r0; r < r1; ++r) {
        const uint8_t *c = j->codes + r * rb;
        float sum = 0.0f;
        for (size_t g = 0; g < ng; ++g) {
            f16 s16, z16;
            memcpy(&s16, &j->s[r * ng + g], 2);
            memcpy(&z16, &j->z[r * ng + g], 2);
            const float s = (float)s16, z = (float)z16;
            for (size_t b = g * 32; b < g * 32 + 32; ++b) {
                const float w0 = ((float)(c[b] & 0x0F) - z) * s;
                const float w1 = ((float)(c[b] >> 4) - z) * s;
                sum += w0 * j->x[2 * b] + w1 * j->x[2 * b + 1];
            }
        }
        j->out[r] = sum;
    }
}

/* ---- element-wise helpers (src/kernels/neon.zig:644-712) ------------------ */
static float quantize_act(const float *x, size_t n, int8_t *q) {
    float mx = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        const float a = fabsf(x[i]);
        if (a > mx) mx = a;
    }
    const float scale = mx > 1e-9f ? mx / 127.0f : 1.0f, inv = 1.0f / scale;
    for (size_t i = 0; i < n; ++i) {
        float r = roundf(x[i] * inv);
        r = r < -128.0f ? -128.0f : (r > 127.0f ? 127.0f : r);
        q[i] = (int8_t)r;
    }
    return scale;
}

static void rmsnorm(const float *x, const float *g, float *y, size_t n, float eps) {
    float lane[4] = {0, 0, 0, 0};
    size_t i = 0;
    for (; i + 4 <= n; i += 4)
        for (int j = 0; j < 4; ++j) lane[j] += x[i + j] * x[i + j];
    float ss = ((lane[0] + lane[1]) + lane[2]) + lane[3];
    for (; i < n; ++i) ss += x[i] * x[i];
    const float inv = 1.0f / sqrtf(ss / (float)n + eps);
    for (i = 0; i < n; ++i) y[i] = x[i] * inv * g[i];
}

/* ---- the model and its step ------------------------------------------------ */
typedef struct {
    int q4;  /* 0: int8 W8A8 hybrid (src/engine.zig); 1: 4-bit GQA (72B shape) */
    int n_layers, attn_every, hidden, ffn, vocab, q_dim, kv_dim, ssm_qkv, ssm_z, head_dim, group;
    int distinct;  /* layers with their own weights; the rest reuse them in turn */
    /* per distinct layer: projections q,k,v,o | qkv,z,out ; gate, up, down */
    uint8_t **w;   /* [distinct][7] weight areas */
    uint16_t **s, **z;
    float *gamma;  /* one RMSNorm gamma vector (all norms) */
    int8_t *embed;
    uint8_t *head;
    uint16_t *head_s, *head_z;
    /* activations */
    float *hidden_v, *norm, *a, *b, *c, *mix, *mlp, *out, *logits;
    int8_t *xq;
} cb_model;

static uint64_t splitmix(uint64_t *s) {
    uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

typedef struct {
    uint8_t *p;
    size_t n;
    uint64_t seed;
} fill_job;
static void fill_task(int wid, int nw, void *a) {
    fill_job *j = (fill_job *)a;
    const size_t per = (j->n / 8 / (size_t)nw) * 8;
    const size_t b0 = (size_t)wid * per, b1 = wid == nw - 1 ? j->n : b0 + per;
    uint64_t st = j->seed ^ (0x1234567ull * (uint64_t)(wid + 1));
    size_t i = b0;
    for (; i + 8 <= b1; i += 8) {
        const uint64_t v = splitmix(&st);
        memcpy(j->p + i, &v, 8);
    }
    for (; i < b1; ++i) j->p[i] = (uint8_t)splitmix(&st);
}
static void fill_bytes(pool_t *p, void *ptr, size_t n, uint64_t seed) {
    fill_job j = {(uint8_t *)ptr, n, seed};
    pool_run(p, fill_task, &j);
}
/* int8 codes in [-64, 63] (keeps activations of the random model tame) */
static void mask_i8(int8_t *p, size_t n) {
    for (size_t i = 0; i < n; ++i) p[i] = (int8_t)(p[i] >> 1);
}
/* fp16 scales around `base` and zero-points in [6, 9] */
static void make_meta(uint16_t *s, uint16_t *z, size_t n, float base, uint64_t seed) {
    uint64_t st = seed;
    for (size_t i = 0; i < n; ++i) {
        const uint64_t r = splitmix(&st);
        const f16 sv = (f16)(base * (0.75f + 0.5f * (float)(r & 0xFFFF) / 65535.0f));
        memcpy(&s[i], &sv, 2);
        if (z) {
            const f16 zv = (f16)(float)(6 + ((r >> 16) & 3));
            memcpy(&z[i], &zv, 2);
        }
    }
}

static size_t proj_rows(const cb_model *m, int kind) {
    switch (kind) {
    case 0: return (size_t)m->q_dim;  /* q | qkv */
    case 1: return (size_t)m->kv_dim; /* k | z */
    case 2: return (size_t)m->kv_dim; /* v */
    case 3: return (size_t)m->hidden; /* o | out */
    case 4: case 5: return (size_t)m->ffn;
    default: return (size_t)m->hidden;
    }
}

/* Builds the model with `distinct` layers of their own weights (the others
 * reuse them in turn).  Returns NULL when memory runs out. */
cb_model *cb_model_create(pool_t *p, int q4, int n_layers, int attn_every, int hidden, int ffn, int vocab, int q_dim,
                          int kv_dim, int ssm_qkv, int ssm_z, int head_dim, int distinct, uint64_t seed) {
    cb_model *m = (cb_model *)calloc(1, sizeof(cb_model));
    m->q4 = q4;
    m->n_layers = n_layers;
    m->attn_every = attn_every;
    m->hidden = hidden;
    m->ffn = ffn;
    m->vocab = vocab;
    m->q_dim = q_dim;
    m->kv_dim = kv_dim;
    m->ssm_qkv = ssm_qkv;
    m->ssm_z = ssm_z;
    m->head_dim = head_dim;
    m->group = 64;
    m->distinct = distinct < 1 ? 1 : (distinct > n_layers ? n_layers : distinct);
    m->w = (uint8_t **)calloc((size_t)m->distinct * 7, sizeof(void *));
    m->s = (uint16_t **)calloc((size_t)m->distinct * 7, sizeof(void *));
    m->z = (uint16_t **)calloc((size_t)m->distinct * 7, sizeof(void *));
    for (int l = 0; l < m->distinct; ++l) {
        const int attn = (l + 1) % attn_every == 0;
        for (int k = 0; k < 7; ++k) {
            size_t rows, cols = (size_t)hidden;
            if (k < 4 && !attn) {
                rows = k == 0 ? (size_t)ssm_qkv : k == 1 ? (size_t)ssm_z : k == 2 ? 0 : (size_t)hidden;
                if (k == 3) cols = (size_t)ssm_z;
            } else {
                rows = proj_rows(m, k);
                if (k == 3) cols = (size_t)q_dim / (q_dim == 2 * hidden ? 2 : 1);
                if (k == 6) cols = (size_t)ffn;
            }
            if (rows == 0) continue;
            const size_t bytes = q4 ? rows * cols / 2 : rows * cols;
            m->w[l * 7 + k] = (uint8_t *)malloc(bytes);
            if (!m->w[l * 7 + k]) return NULL;
            fill_bytes(p, m->w[l * 7 + k], bytes, seed + 97 * (uint64_t)(l * 7 + k));
            if (q4) {
                const size_t ng = rows * (cols / 64);
                m->s[l * 7 + k] = (uint16_t *)malloc(ng * 2);
                m->z[l * 7 + k] = (uint16_t *)malloc(ng * 2);
                make_meta(m->s[l * 7 + k], m->z[l * 7 + k], ng, 0.0067f, seed + (uint64_t)l);
            } else {
                mask_i8((int8_t *)m->w[l * 7 + k], bytes);
            }
        }
    }
    m->gamma = (float *)malloc((size_t)hidden * 4);
    for (int i = 0; i < hidden; ++i) m->gamma[i] = 1.0f + 0.01f * (float)((i * 37) % 11 - 5);
    m->embed = (int8_t *)malloc((size_t)vocab * hidden);
    fill_bytes(p, m->embed, (size_t)vocab * hidden, seed + 7);
    mask_i8(m->embed, (size_t)vocab * hidden);
    const size_t hb = q4 ? (size_t)vocab * hidden / 2 : (size_t)vocab * hidden;
    m->head = (uint8_t *)malloc(hb);
    if (!m->head) return NULL;
    fill_bytes(p, m->head, hb, seed + 11);
    if (q4) {
        const size_t ng = (size_t)vocab * (hidden / 64);
        m->head_s = (uint16_t *)malloc(ng * 2);
        m->head_z = (uint16_t *)malloc(ng * 2);
        make_meta(m->head_s, m->head_z, ng, 0.0067f, seed + 13);
    } else {
        mask_i8((int8_t *)m->head, hb);
    }
    const size_t wide = (size_t)(ffn > q_dim ? ffn : q_dim) + (size_t)ssm_qkv + 16;
    m->hidden_v = (float *)calloc(hidden, 4);
    m->norm = (float *)calloc(wide, 4);
    m->a = (float *)calloc(wide, 4);
    m->b = (float *)calloc(wide, 4);
    m->c = (float *)calloc(wide, 4);
    m->mix = (float *)calloc(wide, 4);
    m->mlp = (float *)calloc(wide, 4);
    m->out = (float *)calloc(wide, 4);
    m->logits = (float *)calloc(vocab, 4);
    m->xq = (int8_t *)calloc(wide, 1);
    return m;
}

void cb_model_destroy(cb_model *m) {
    if (!m) return;
    for (int i = 0; i < m->distinct * 7; ++i) {
        free(m->w[i]);
        free(m->s[i]);
        free(m->z[i]);
    }
    free(m->w);
    free(m->s);
    free(m->z);
    free(m->gamma);
    free(m->embed);
    free(m->head);
    free(m->head_s);
    free(m->head_z);
    free(m->hidden_v);
    free(m->norm);
    free(m->a);
    free(m->b);
    free(m->c);
    free(m->mix);
    free(m->mlp);
    free(m->out);
    free(m->logits);
    free(m->xq);
    free(m);
}

static void gemv_i8(pool_t *p, const uint8_t *w, const int8_t *x, float sx, size_t rows, size_t cols, float *out) {
    gemv_i8_job j = {(const int8_t *)w, NULL, 0.002f, 0.0f, sx, x, rows, cols, out};
    pool_run(p, gemv_i8_task, &j);
}
static void gemv_q4(pool_t *p, const uint8_t *w, const uint16_t *s, const uint16_t *z, const float *x, size_t rows,
                    size_t cols, float *out) {
    gemv_q4_job j = {w, s, z, x, rows, cols, out};
    pool_run(p, gemv_q4_task, &j);
}

/* One decode step for `token` (src/engine.zig:583-734); returns the argmax. */
int cb_step(cb_model *m, pool_t *p, int token) {
    const size_t H = (size_t)m->hidden, F = (size_t)m->ffn;
    const float es = 0.02f * 3.0f / 127.0f;
    for (size_t i = 0; i < H; ++i) m->hidden_v[i] = (float)m->embed[(size_t)token * H + i] * es;
    for (int l = 0; l < m->n_layers; ++l) {
        const int d = l % m->distinct;
        uint8_t **W = m->w + d * 7;
        uint16_t **S = m->s + d * 7, **Z = m->z + d * 7;
        const int attn = (l + 1) % m->attn_every == 0;
        rmsnorm(m->hidden_v, m->gamma, m->norm, H, 1e-6f);
        if (m->q4) {
            if (attn) {
                gemv_q4(p, W[0], S[0], Z[0], m->norm, (size_t)m->q_dim, H, m->a);
                gemv_q4(p, W[1], S[1], Z[1], m->norm, (size_t)m->kv_dim, H, m->b);
                gemv_q4(p, W[2], S[2], Z[2], m->norm, (size_t)m->kv_dim, H, m->c);
                const int hd = m->head_dim, grp = (m->q_dim / hd) / (m->kv_dim / hd);
                for (size_t i = 0; i < H; ++i) m->mix[i] = m->c[((i / hd) / grp) * hd + i % hd];
                gemv_q4(p, W[3], S[3], Z[3], m->mix, H, H, m->out);
            }
            for (size_t i = 0; i < H; ++i) m->hidden_v[i] += m->out[i];
            rmsnorm(m->hidden_v, m->gamma, m->norm, H, 1e-6f);
            gemv_q4(p, W[4], S[4], Z[4], m->norm, F, H, m->a);
            gemv_q4(p, W[5], S[5], Z[5], m->norm, F, H, m->b);
            for (size_t i = 0; i < F; ++i) m->mlp[i] = silu(m->a[i]) * m->b[i];
            gemv_q4(p, W[6], S[6], Z[6], m->mlp, H, F, m->out);
            for (size_t i = 0; i < H; ++i) m->hidden_v[i] += m->out[i];
        } else {
            float sx = quantize_act(m->norm, H, m->xq);
            if (attn) {
                gemv_i8(p, W[0], m->xq, sx, (size_t)m->q_dim, H, m->a);
                gemv_i8(p, W[1], m->xq, sx, (size_t)m->kv_dim, H, m->b);
                gemv_i8(p, W[2], m->xq, sx, (size_t)m->kv_dim, H, m->c);
                for (size_t i = 0; i < H; ++i) m->mix[i] = m->c[i % (size_t)m->kv_dim];
                const float sa = quantize_act(m->mix, H, m->xq);
                gemv_i8(p, W[3], m->xq, sa, H, H, m->out);
            } else {
                gemv_i8(p, W[0], m->xq, sx, (size_t)m->ssm_qkv, H, m->a);
                gemv_i8(p, W[1], m->xq, sx, (size_t)m->ssm_z, H, m->b);
                for (size_t i = 0; i < (size_t)m->ssm_z; ++i) m->mix[i] = m->a[i % (size_t)m->ssm_qkv] * silu(m->b[i]);
                const float sa = quantize_act(m->mix, (size_t)m->ssm_z, m->xq);
                gemv_i8(p, W[3], m->xq, sa, H, (size_t)m->ssm_z, m->out);
            }
            for (size_t i = 0; i < H; ++i) m->hidden_v[i] += m->out[i];
            rmsnorm(m->hidden_v, m->gamma, m->norm, H, 1e-6f);
            sx = quantize_act(m->norm, H, m->xq);
            gemv_i8_job j = {(const int8_t *)W[4], (const int8_t *)W[5], 0.002f, 0.002f, sx, m->xq, F, H, m->mlp};
            pool_run(p, gemv_i8_task, &j);
            const float sm = quantize_act(m->mlp, F, m->xq);
            gemv_i8(p, W[6], m->xq, sm, H, F, m->out);
            for (size_t i = 0; i < H; ++i) m->hidden_v[i] += m->out[i];
        }
    }
    rmsnorm(m->hidden_v, m->gamma, m->norm, H, 1e-6f);
    if (m->q4) {
        gemv_q4(p, m->head, m->head_s, m->head_z, m->norm, (size_t)m->vocab, H, m->logits);
    } else {
        const float sx = quantize_act(m->norm, H, m->xq);
        gemv_i8(p, m->head, m->xq, sx, (size_t)m->vocab, H, m->logits);
    }
    int best = 0;
    for (int v = 1; v < m->vocab; ++v)
        if (m->logits[v] > m->logits[best]) best = v;
    return best;
}
