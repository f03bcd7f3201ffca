/*
 * vmlm_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the VMLM quantised-linear kernels, used as the parity
 * checker by tests/, by __graft_entry__.smoke() and by bench.py's CPU-baseline
 * leg.  Nothing in the product library (sparrow_b200/) links or calls this
 * file; the product path is CUDA only.
 *
 * Every function below restates one reference function, cited by the path
 * inside the shouzugzs-AI/Sparrow tree:
 *
 *   oracle_gemm_nt_int8        ops/src/kernels.rs:1256-1287  (x86_64 AVX2+FMA body)
 *   oracle_gemm_nt_int8_scalar ops/src/kernels.rs:1289-1305  (non-x86 fallback)
 *   oracle_gemm_nt_bf16        ops/src/kernels.rs:1199-1227
 *   bf16_widen_16 / hsum_ps    tensor/src/dtype.rs:12-36
 *   oracle_f32_to_bf16         tensor/src/dtype.rs:38-45 (RNE, no NaN special case)
 *   oracle_quant_int8          tests/src/quant.rs:78-104
 *   oracle_fill_uniform        tests/src/quant.rs:48-55 (lcg, rnd; values lie in [-scale, 0))
 *   oracle_fill_gauss_ref      tests/src/quant.rs:605-613 (Box-Muller on lcg, as written)
 *   oracle_fill_normal         the same lcg with full-range uniforms: true N(0, sigma)
 *   oracle_gemm_naive_f32      tests/src/main.rs:283-295 (naive triple loop)
 *   oracle_gemm_nt_f32_par     ops/src/kernels.rs:947-967 (gemm_nt_scalar: f32
 *                              C = A . B^T, B [n,k], sequential mul then add,
 *                              then `s += c` when acc)
 *   oracle_gemm_f32_par        ops/src/kernels.rs:383-403 (gemm_scalar, the
 *                              whole of gemm NN at :407-419: B [k,n])
 *   oracle_rmsnorm             ops/src/kernels.rs:1346-1370 (sqrt_f :1371-1376 is
 *                              _mm_sqrt_ss: correctly rounded, as sqrtf)
 *   oracle_gemv_f32            core/src/interp.rs:815-827 (OP_GEMV)
 *   oracle_emb                 core/src/interp.rs:1351-1420 (OP_EMB: index
 *                              checks, then the row widened or copied)
 *   parallel split             ops/src/par.rs:44-62 (chunk = ceil(n/nt) over N)
 *   oracle_quant_int4_grouped  tests/src/quant.rs:114-152 (int4, a scale per group)
 *   oracle_gemm_nt_int4_gs     tests/src/quant.rs:298-362 (AVX2 as shipped, or the
 *                              packed order; see the function)
 *   oracle_quant_int8_outliers tests/src/quant.rs:458-515 (LLM.int8 outlier columns)
 *   oracle_gemm_nt_int8_outlier tests/src/quant.rs:524-565
 *   oracle_fill_gauss_k        tests/src/quant.rs:595-602 (Box-Muller / sqrt(k))
 *
 * The AVX2 bodies use the same intrinsic sequence as the reference, so the
 * summation order is the same; the file must be built with -mavx2 -mfma
 * -ffp-contract=off because Rust never contracts a*b+c in the scalar tails.
 *
 * The int8 x int8 -> int32 GEMM (oracle_gemm_i8i8_*) has no counterpart in the
 * reference: it is the exact integer definition, order-free, so it is exact by
 * construction (parity for that kernel is pinned by arithmetic, not by a
 * reference test).
 */
#include <immintrin.h>
#include <math.h>
#include <pthread.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define EXPORT __attribute__((visibility("default")))

/* ---------------------------------------------------------------- dtype */

/* tensor/src/dtype.rs:12-24: one 256-bit load of 16 bf16, each 128-bit half
 * zero-extended to 8 x u32 and shifted left by 16. */
static inline void bf16_widen_16(const uint16_t *p, __m256 *w0, __m256 *w1) {
    __m256i packed = _mm256_loadu_si256((const __m256i *)p);
    __m128i lo128 = _mm256_castsi256_si128(packed);
    __m128i hi128 = _mm256_extracti128_si256(packed, 1);
    __m256i l0 = _mm256_cvtepu16_epi32(lo128);
    __m256i l1 = _mm256_cvtepu16_epi32(hi128);
    *w0 = _mm256_castsi256_ps(_mm256_slli_epi32(l0, 16));
    *w1 = _mm256_castsi256_ps(_mm256_slli_epi32(l1, 16));
}

/* tensor/src/dtype.rs:26-36: (hi128 + lo128) -> + movehl -> lane0 + lane1. */
static inline float hsum_ps(__m256 v) {
    __m128 hi = _mm256_extractf128_ps(v, 1);
    __m128 lo = _mm256_castps256_ps128(v);
    __m128 s4 = _mm_add_ps(hi, lo);
    __m128 sh = _mm_movehl_ps(s4, s4);
    __m128 s2 = _mm_add_ps(s4, sh);
    __m128 s1 = _mm_add_ss(s2, _mm_shuffle_ps(s2, s2, 1));
    return _mm_cvtss_f32(s1);
}

static inline float bf16_bits_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* tensor/src/dtype.rs:38-45: add 0x7fff + lsb, keep the high half. */
EXPORT uint16_t oracle_f32_to_bf16(float v) {
    uint32_t u;
    memcpy(&u, &v, 4);
    uint32_t lsb = (u >> 16) & 1u;
    return (uint16_t)((u + 0x7fffu + lsb) >> 16);
}

EXPORT void oracle_f32_to_bf16_n(const float *x, uint16_t *out, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = oracle_f32_to_bf16(x[i]);
}

EXPORT void oracle_bf16_to_f32_n(const uint16_t *h, float *out, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = bf16_bits_to_f32(h[i]);
}

/* ----------------------------------------------------- reference kernels */

/* ops/src/kernels.rs:1256-1287, restricted to output columns [j0, j1).
 * One 8-lane FMA accumulator over kk+8<=k, hsum_ps, scalar tail with a
 * separate multiply and add, then one multiply by scale[j]. */
static void gemm_nt_int8_cols(const float *a, const int8_t *q, const float *scale,
                              float *c, size_t m, size_t n, size_t k,
                              size_t j0, size_t j1) {
    for (size_t i = 0; i < m; i++) {
        const float *ar = a + i * k;
        for (size_t j = j0; j < j1; j++) {
            const int8_t *qr = q + j * k;
            __m256 acc = _mm256_setzero_ps();
            size_t kk = 0;
            while (kk + 8 <= k) {
                __m128i eight = _mm_loadl_epi64((const __m128i *)(qr + kk));
                __m256i i32v = _mm256_cvtepi8_epi32(eight);
                __m256 lo = _mm256_cvtepi32_ps(i32v);
                __m256 av = _mm256_loadu_ps(ar + kk);
                acc = _mm256_fmadd_ps(av, lo, acc);
                kk += 8;
            }
            float s = hsum_ps(acc);
            while (kk < k) {
                float prod = ar[kk] * (float)qr[kk];
                s = s + prod;
                kk += 1;
            }
            c[i * n + j] = s * scale[j];
        }
    }
}

/* ops/src/kernels.rs:1199-1227, restricted to output columns [j0, j1).
 * Two accumulators (kk..kk+7 and kk+8..kk+15) per 16-wide step. */
static void gemm_nt_bf16_cols(const float *a, const uint16_t *b, float *c,
                              size_t m, size_t n, size_t k, size_t j0, size_t j1) {
    for (size_t i = 0; i < m; i++) {
        const float *ar = a + i * k;
        for (size_t j = j0; j < j1; j++) {
            const uint16_t *br = b + j * k;
            __m256 acc0 = _mm256_setzero_ps();
            __m256 acc1 = _mm256_setzero_ps();
            size_t kk = 0;
            while (kk + 16 <= k) {
                __m256 w0, w1;
                bf16_widen_16(br + kk, &w0, &w1);
                acc0 = _mm256_fmadd_ps(_mm256_loadu_ps(ar + kk), w0, acc0);
                acc1 = _mm256_fmadd_ps(_mm256_loadu_ps(ar + kk + 8), w1, acc1);
                kk += 16;
            }
            float s = hsum_ps(acc0) + hsum_ps(acc1);
            while (kk < k) {
                float prod = ar[kk] * bf16_bits_to_f32(br[kk]);
                s = s + prod;
                kk += 1;
            }
            c[i * n + j] = s;
        }
    }
}

EXPORT void oracle_gemm_nt_int8(const float *a, const int8_t *q, const float *scale,
                                float *c, size_t m, size_t n, size_t k) {
    gemm_nt_int8_cols(a, q, scale, c, m, n, k, 0, n);
}

EXPORT void oracle_gemm_nt_bf16(const float *a, const uint16_t *b, float *c,
                                size_t m, size_t n, size_t k) {
    gemm_nt_bf16_cols(a, b, c, m, n, k, 0, n);
}

/* ops/src/kernels.rs:1289-1305: strictly sequential sum over k. */
EXPORT void oracle_gemm_nt_int8_scalar(const float *a, const int8_t *q, const float *scale,
                                       float *c, size_t m, size_t n, size_t k) {
    for (size_t i = 0; i < m; i++)
        for (size_t j = 0; j < n; j++) {
            float s = 0.0f;
            for (size_t kk = 0; kk < k; kk++) {
                float prod = a[i * k + kk] * (float)q[j * k + kk];
                s = s + prod;
            }
            c[i * n + j] = s * scale[j];
        }
}

/* tests/src/main.rs:283-295: naive f32 NT GEMM used as the regression truth. */
EXPORT void oracle_gemm_naive_f32(const float *a, const float *b, float *c,
                                  size_t m, size_t n, size_t k) {
    for (size_t i = 0; i < m; i++)
        for (size_t j = 0; j < n; j++) {
            float s = 0.0f;
            for (size_t kk = 0; kk < k; kk++) {
                float prod = a[i * k + kk] * b[j * k + kk];
                s = s + prod;
            }
            c[i * n + j] = s;
        }
}

/* ------------------------------------------- int8 x int8 -> int32 (exact) */

static void gemm_i8i8_cols(const int8_t *x, const int8_t *w, const float *scale,
                           int32_t *acc_out, float *c, size_t m, size_t n, size_t k,
                           size_t j0, size_t j1) {
    for (size_t i = 0; i < m; i++) {
        const int8_t *xr = x + i * k;
        for (size_t j = j0; j < j1; j++) {
            const int8_t *wr = w + j * k;
            __m256i acc = _mm256_setzero_si256();
            size_t kk = 0;
            while (kk + 16 <= k) {
                __m256i xv = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i *)(xr + kk)));
                __m256i wv = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i *)(wr + kk)));
                acc = _mm256_add_epi32(acc, _mm256_madd_epi16(xv, wv));
                kk += 16;
            }
            int32_t lanes[8];
            _mm256_storeu_si256((__m256i *)lanes, acc);
            int64_t s = 0;
            for (int t = 0; t < 8; t++) s += lanes[t];
            while (kk < k) {
                s += (int32_t)xr[kk] * (int32_t)wr[kk];
                kk++;
            }
            int32_t s32 = (int32_t)s; /* k*127*128 < 2^31 for k < 132104 */
            if (acc_out) acc_out[i * n + j] = s32;
            if (c) c[i * n + j] = (float)s32 * scale[j];
        }
    }
}

/* C[i][j] = float(sum_k x[i][k]*w[j][k]) * scale[j]; acc_out (optional) gets
 * the int32 sums. Exact integer definition: summation order is irrelevant. */
EXPORT void oracle_gemm_i8i8(const int8_t *x, const int8_t *w, const float *scale,
                             int32_t *acc_out, float *c, size_t m, size_t n, size_t k) {
    gemm_i8i8_cols(x, w, scale, acc_out, c, m, n, k, 0, n);
}

/* ------------------------------------------------------- f32 GEMMs
 * gemm_nt_scalar (ops/src/kernels.rs:947-967) and gemm_scalar (:383-403):
 * per output a sequential sum of separately rounded products, then one add of
 * the old C when acc. (The reference's AVX2 8x8 and packed gemm_nt kernels
 * run FMA chains in other orders; the f32 GEMM's parity is a tolerance.) */
static void gemm_f32_cols(int nn, const float *a, const float *b, float *c, size_t m, size_t n,
                          size_t k, int acc, size_t j0, size_t j1) {
    for (size_t i = 0; i < m; i++)
        for (size_t j = j0; j < j1; j++) {
            float s = 0.0f;
            for (size_t p = 0; p < k; p++) {
                float prod = a[i * k + p] * (nn ? b[p * n + j] : b[j * k + p]);
                s = s + prod;
            }
            if (acc) s = s + c[i * n + j];
            c[i * n + j] = s;
        }
}

/* ------------------------------------------- decode-step neighbours */

/* rmsnorm: per row, ss = sequential sum of v*v, ss /= cols, inv = 1 / sqrt(ss + eps),
 * dst = src * inv * g (left to right). */
EXPORT void oracle_rmsnorm(float *dst, const float *src, const float *g, size_t rows, size_t cols,
                           float eps) {
    for (size_t r = 0; r < rows; r++) {
        const float *p = src + r * cols;
        float *q = dst + r * cols;
        float ss = 0.0f;
        for (size_t i = 0; i < cols; i++) {
            float v = p[i];
            float sq = v * v;
            ss = ss + sq;
        }
        ss = ss / (float)cols;
        float inv = 1.0f / sqrtf(ss + eps);
        for (size_t i = 0; i < cols; i++) {
            float t = p[i] * inv;
            q[i] = t * g[i];
        }
    }
}

/* OP_GEMV: c[i] = sequential sum over p of a[i*k + p] * b[p]. */
EXPORT void oracle_gemv_f32(const float *a, const float *b, float *c, size_t m, size_t k) {
    for (size_t i = 0; i < m; i++) {
        float s = 0.0f;
        for (size_t p = 0; p < k; p++) {
            float prod = a[i * k + p] * b[p];
            s = s + prod;
        }
        c[i] = s;
    }
}

/* OP_EMB for m indices: 0 on success; 1 "row index out of range" (negative, NaN,
 * >= rows); 2 "row index is not an integer". dtype 4: bf16 bits, widened; 0: f32. */
EXPORT int oracle_emb(const void *table, int dtype, size_t rows, size_t cols, const float *idx,
                      size_t m, float *out) {
    for (size_t t = 0; t < m; t++) {
        float rowf = idx[t];
        if (!(rowf >= 0.0f) || rowf >= (float)rows) return 1;
        size_t row = (size_t)rowf;
        if ((float)row != rowf) return 2;
        for (size_t i = 0; i < cols; i++) {
            if (dtype == 4)
                out[t * cols + i] = bf16_bits_to_f32(((const uint16_t *)table)[row * cols + i]);
            else
                out[t * cols + i] = ((const float *)table)[row * cols + i];
        }
    }
    return 0;
}

/* ------------------------------------------------ ops/src/par.rs split */

typedef struct {
    int kind; /* 0 int8, 1 bf16, 2 i8i8, 3 f32 NT, 4 f32 NN */
    const void *a, *b;
    const float *scale;
    int32_t *acc;
    float *c;
    size_t m, n, k, j0, j1;
    int accf; /* f32: C += */
} job_t;

static void *run_job(void *p) {
    job_t *jb = (job_t *)p;
    if (jb->kind == 0)
        gemm_nt_int8_cols((const float *)jb->a, (const int8_t *)jb->b, jb->scale, jb->c,
                          jb->m, jb->n, jb->k, jb->j0, jb->j1);
    else if (jb->kind == 1)
        gemm_nt_bf16_cols((const float *)jb->a, (const uint16_t *)jb->b, jb->c,
                          jb->m, jb->n, jb->k, jb->j0, jb->j1);
    else if (jb->kind == 3 || jb->kind == 4)
        gemm_f32_cols(jb->kind == 4, (const float *)jb->a, (const float *)jb->b, jb->c, jb->m, jb->n,
                      jb->k, jb->accf, jb->j0, jb->j1);
    else
        gemm_i8i8_cols((const int8_t *)jb->a, (const int8_t *)jb->b, jb->scale, jb->acc,
                       jb->c, jb->m, jb->n, jb->k, jb->j0, jb->j1);
    return NULL;
}

/* Columns [0,n) split as chunk = ceil(n/nt) per thread (ops/src/par.rs:44-62);
 * each output element is computed exactly as by the single-thread kernel. */
static void par_run(job_t base, int nt) {
    size_t n = base.n;
    if (nt <= 1 || n <= 1) {
        base.j0 = 0;
        base.j1 = n;
        run_job(&base);
        return;
    }
    if ((size_t)nt > n) nt = (int)n;
    if (nt > 256) nt = 256;
    size_t chunk = (n + (size_t)nt - 1) / (size_t)nt;
    pthread_t th[256];
    job_t jobs[256];
    int started = 0;
    for (int t = 0; t < nt; t++) {
        size_t lo = (size_t)t * chunk, hi = (size_t)(t + 1) * chunk;
        if (hi > n) hi = n;
        if (lo >= hi) break;
        jobs[t] = base;
        jobs[t].j0 = lo;
        jobs[t].j1 = hi;
        if (pthread_create(&th[t], NULL, run_job, &jobs[t]) != 0) {
            run_job(&jobs[t]);
            th[t] = 0;
        }
        started = t + 1;
    }
    for (int t = 0; t < started; t++)
        if (th[t]) pthread_join(th[t], NULL);
}

/* Multi-threaded variants, and column-range variants used to time or check a
 * bounded sample of a large problem ([j0,j1) of n, row stride of c is n). */
EXPORT void oracle_gemm_nt_int8_par(const float *a, const int8_t *q, const float *scale,
                                    float *c, size_t m, size_t n, size_t k, int nt) {
    job_t b = {0, a, q, scale, NULL, c, m, n, k, 0, n, 0};
    par_run(b, nt);
}

EXPORT void oracle_gemm_nt_bf16_par(const float *a, const uint16_t *w, float *c,
                                    size_t m, size_t n, size_t k, int nt) {
    job_t b = {1, a, w, NULL, NULL, c, m, n, k, 0, n, 0};
    par_run(b, nt);
}

EXPORT void oracle_gemm_i8i8_par(const int8_t *x, const int8_t *w, const float *scale,
                                 int32_t *acc, float *c, size_t m, size_t n, size_t k, int nt) {
    job_t b = {2, x, w, scale, acc, c, m, n, k, 0, n, 0};
    par_run(b, nt);
}

EXPORT void oracle_gemm_nt_f32_par(const float *a, const float *b, float *c, size_t m, size_t n,
                                   size_t k, int acc, int nt) {
    job_t jb = {3, a, b, NULL, NULL, c, m, n, k, 0, n, acc};
    par_run(jb, nt);
}

EXPORT void oracle_gemm_f32_par(const float *a, const float *b, float *c, size_t m, size_t n,
                                size_t k, int acc, int nt) {
    job_t jb = {4, a, b, NULL, NULL, c, m, n, k, 0, n, acc};
    par_run(jb, nt);
}

/* ------------------------------------------------------------ generators */

#define LCG_A 6364136223846793005ULL
#define LCG_C 1442695040888963407ULL

/* tests/src/quant.rs:48-51 */
static inline float lcg_next(uint64_t *s) {
    *s = *s * LCG_A + LCG_C;
    return ((float)(uint32_t)(*s >> 33) / (float)(1u << 31)) - 1.0f;
}

/* State after `steps` LCG steps from s (affine map composed by squaring). */
static uint64_t lcg_jump(uint64_t s, uint64_t steps) {
    uint64_t mul = 1, add = 0, cm = LCG_A, ca = LCG_C;
    while (steps) {
        if (steps & 1) {
            mul = mul * cm;
            add = add * cm + ca;
        }
        ca = ca * cm + ca;
        cm = cm * cm;
        steps >>= 1;
    }
    return s * mul + add;
}

typedef struct {
    int kind; /* 0 uniform f32, 1 reference gauss f32, 2 uniform int8, 3 normal f32 */
    uint64_t seed;
    size_t lo, hi;
    float scale;
    void *out;
} gen_t;

static void *gen_range(void *p) {
    gen_t *g = (gen_t *)p;
    if (g->kind == 0) {
        uint64_t s = lcg_jump(g->seed, g->lo);
        float *o = (float *)g->out;
        for (size_t i = g->lo; i < g->hi; i++) o[i] = lcg_next(&s) * g->scale;
    } else if (g->kind == 1) {
        /* tests/src/quant.rs:605-613: two lcg draws per value. */
        uint64_t s = lcg_jump(g->seed, 2 * g->lo);
        float *o = (float *)g->out;
        const float two_pi = 2.0f * 3.14159265358979323846f;
        for (size_t i = g->lo; i < g->hi; i++) {
            float u1 = (lcg_next(&s) + 1.0f) * 0.5f + 1e-9f;
            float u2 = (lcg_next(&s) + 1.0f) * 0.5f;
            float r = sqrtf(-2.0f * logf(u1));
            float arg = two_pi * u2;
            o[i] = r * cosf(arg) * g->scale;
        }
    } else if (g->kind == 4) {
        /* tests/src/quant.rs:595-602: the same draws, r * cos(2 pi u2) / sqrt(k)
         * (scale holds sqrt(k); a division, as written). */
        uint64_t s = lcg_jump(g->seed, 2 * g->lo);
        float *o = (float *)g->out;
        const float two_pi = 2.0f * 3.14159265358979323846f;
        for (size_t i = g->lo; i < g->hi; i++) {
            float u1 = (lcg_next(&s) + 1.0f) * 0.5f + 1e-9f;
            float u2 = (lcg_next(&s) + 1.0f) * 0.5f;
            float r = sqrtf(-2.0f * logf(u1));
            float arg = two_pi * u2;
            o[i] = r * cosf(arg) / g->scale;
        }
    } else if (g->kind == 3) {
        /* Box-Muller on the same lcg, with both uniforms taken from the top 24
         * bits over the full [0,1) range: a true N(0, sigma). */
        uint64_t s = lcg_jump(g->seed, 2 * g->lo);
        float *o = (float *)g->out;
        const float two_pi = 2.0f * 3.14159265358979323846f;
        const float inv24 = 1.0f / 16777216.0f;
        for (size_t i = g->lo; i < g->hi; i++) {
            s = s * LCG_A + LCG_C;
            float u1 = (float)((s >> 40) + 1) * inv24; /* (0, 1] */
            s = s * LCG_A + LCG_C;
            float u2 = (float)(s >> 40) * inv24;       /* [0, 1) */
            o[i] = sqrtf(-2.0f * logf(u1)) * cosf(two_pi * u2) * g->scale;
        }
    } else {
        uint64_t s = lcg_jump(g->seed, g->lo);
        int8_t *o = (int8_t *)g->out;
        for (size_t i = g->lo; i < g->hi; i++) {
            s = s * LCG_A + LCG_C;
            o[i] = (int8_t)((int)((s >> 33) % 255u) - 127);
        }
    }
    return NULL;
}

static void gen_par(gen_t base, size_t n, int nt) {
    if (nt < 1) nt = 1;
    if (nt > 256) nt = 256;
    if ((size_t)nt > n) nt = n ? (int)n : 1;
    size_t chunk = (n + (size_t)nt - 1) / (size_t)nt;
    pthread_t th[256];
    gen_t jobs[256];
    int started = 0;
    for (int t = 0; t < nt; t++) {
        jobs[t] = base;
        jobs[t].lo = (size_t)t * chunk;
        jobs[t].hi = jobs[t].lo + chunk > n ? n : jobs[t].lo + chunk;
        if (jobs[t].lo >= jobs[t].hi) break;
        if (nt == 1 || pthread_create(&th[t], NULL, gen_range, &jobs[t]) != 0) {
            gen_range(&jobs[t]);
            th[t] = 0;
        }
        started = t + 1;
    }
    for (int t = 0; t < started; t++)
        if (th[t]) pthread_join(th[t], NULL);
}

/* rnd(n, seed, scale) of tests/src/quant.rs:52-55: lcg() * scale, which lies in
 * [-scale, 0) because lcg() lies in [-1, 0). */
EXPORT void oracle_fill_uniform(float *out, size_t n, uint64_t seed, float scale, int nt) {
    gen_t g = {0, seed, 0, 0, scale, out};
    gen_par(g, n, nt);
}

/* The reference's Box-Muller (tests/src/quant.rs:605-613), restated as is.
 * Its lcg() returns (s>>33)/2^31 - 1, a 31-bit value over 2^31 minus one, so
 * it lies in [-1, 0): u1, u2 lie in [0, 0.5) and the result is not N(0,1)
 * (r >= sqrt(2 ln 2), std ~1.30). Kept to document that behaviour. */
EXPORT void oracle_fill_gauss_ref(float *out, size_t n, uint64_t seed, float sigma, int nt) {
    gen_t g = {1, seed, 0, 0, sigma, out};
    gen_par(g, n, nt);
}

/* N(0, sigma): Box-Muller on the reference lcg with full-range uniforms. This is
 * the generator for the benchmark configurations' ~N(0, sigma) inputs. */
EXPORT void oracle_fill_normal(float *out, size_t n, uint64_t seed, float sigma, int nt) {
    gen_t g = {3, seed, 0, 0, sigma, out};
    gen_par(g, n, nt);
}

/* The weight generator of the quantisation benchmark (tests/src/quant.rs:595-602):
 * the reference Box-Muller divided by sqrt(k) (sqrt_k = sqrtf(k)). */
EXPORT void oracle_fill_gauss_k(float *out, size_t n, uint64_t seed, float sqrt_k, int nt) {
    gen_t g = {4, seed, 0, 0, sqrt_k, out};
    gen_par(g, n, nt);
}

/* Uniform int8 in [-127,127]: ((s>>33) % 255) - 127 on the lcg stream. */
EXPORT void oracle_fill_int8(int8_t *out, size_t n, uint64_t seed, int nt) {
    gen_t g = {2, seed, 0, 0, 1.0f, out};
    gen_par(g, n, nt);
}

/* ------------------------------------------------------------- quantiser */

typedef struct {
    const float *w;
    int8_t *q;
    float *scale;
    size_t k, r0, r1;
} qjob_t;

/* tests/src/quant.rs:78-104: per row amax (0 -> 1e-30), s = amax/127,
 * q = round(w/s) clamped to [-127,127]; Rust round() is half away from zero,
 * which is C roundf. */
static void *quant_rows(void *p) {
    qjob_t *j = (qjob_t *)p;
    size_t k = j->k;
    for (size_t i = j->r0; i < j->r1; i++) {
        float amax = 0.0f;
        for (size_t t = 0; t < k; t++) {
            float a = fabsf(j->w[i * k + t]);
            if (a > amax) amax = a;
        }
        if (amax == 0.0f) amax = 1e-30f;
        float s = amax / 127.0f;
        j->scale[i] = s;
        for (size_t t = 0; t < k; t++) {
            float v = j->w[i * k + t] / s;
            float r = roundf(v);
            if (r < -127.0f) r = -127.0f;
            if (r > 127.0f) r = 127.0f;
            j->q[i * k + t] = (int8_t)r;
        }
    }
    return NULL;
}

EXPORT void oracle_quant_int8(const float *w, size_t n, size_t k, int8_t *q, float *scale, int nt) {
    if (nt < 1) nt = 1;
    if (nt > 256) nt = 256;
    if ((size_t)nt > n) nt = n ? (int)n : 1;
    size_t chunk = (n + (size_t)nt - 1) / (size_t)nt;
    pthread_t th[256];
    qjob_t jobs[256];
    int started = 0;
    for (int t = 0; t < nt; t++) {
        jobs[t].w = w;
        jobs[t].q = q;
        jobs[t].scale = scale;
        jobs[t].k = k;
        jobs[t].r0 = (size_t)t * chunk;
        jobs[t].r1 = jobs[t].r0 + chunk > n ? n : jobs[t].r0 + chunk;
        if (jobs[t].r0 >= jobs[t].r1) break;
        if (nt == 1 || pthread_create(&th[t], NULL, quant_rows, &jobs[t]) != 0) {
            quant_rows(&jobs[t]);
            th[t] = 0;
        }
        started = t + 1;
    }
    for (int t = 0; t < started; t++)
        if (th[t]) pthread_join(th[t], NULL);
}

/* ------------------------------------------------------ variant kernels */

/* tests/src/quant.rs:114-152: per row and group of `group` columns, amax (0 ->
 * 1e-30), s = amax/7, v = round(w/s) clamped to [-7,7]; two's-complement
 * nibbles packed two per byte, column j in the low nibble when j is even and
 * the high nibble when odd; rows of (k+1)/2 bytes; scale [n][ceil(k/group)]. */
EXPORT void oracle_quant_int4_grouped(const float *w, size_t n, size_t k, size_t group, uint8_t *packed,
                                      float *scale) {
    size_t rowbytes = (k + 1) / 2, gpr = (k + group - 1) / group;
    memset(packed, 0, n * rowbytes);
    for (size_t i = 0; i < n; i++)
        for (size_t g = 0; g < gpr; g++) {
            size_t beg = g * group, end = beg + group < k ? beg + group : k;
            float amax = 0.0f;
            for (size_t j = beg; j < end; j++) {
                float a = fabsf(w[i * k + j]);
                if (a > amax) amax = a;
            }
            if (amax == 0.0f) amax = 1e-30f;
            float s = amax / 7.0f;
            scale[i * gpr + g] = s;
            for (size_t j = beg; j < end; j++) {
                float r = roundf(w[i * k + j] / s);
                if (r < -7.0f) r = -7.0f;
                if (r > 7.0f) r = 7.0f;
                uint8_t nib = (uint8_t)(int8_t)r & 0x0F;
                size_t idx = i * rowbytes + j / 2;
                packed[idx] = (j % 2 == 0) ? (uint8_t)((packed[idx] & 0xF0) | nib)
                                           : (uint8_t)((packed[idx] & 0x0F) | (nib << 4));
            }
        }
}

static inline int nib_value(uint8_t byte, size_t col) {
    int nib = (col % 2 == 0) ? (byte & 0x0F) : ((byte >> 4) & 0x0F);
    return nib > 7 ? nib - 16 : nib;
}

/* tests/src/quant.rs:298-362, gemm_nt_int4_gs. Per (i, j) and per group
 * [g0, min(g0+group, k)): 32-wide steps while kk+32 <= gend, each one 16-byte
 * load at packed + kk/2 and four 8-lane FMAs into one accumulator (lanes kk..+7,
 * +8..+15, +16..+23, +24..+31), hsum_ps, a scalar tail (mul then add), then
 * total += s * scale[group] (mul then add).
 *
 * order 1 is the AVX2 step as shipped (the same intrinsic sequence as
 * :316-333): both 128-bit lanes of the widened load hold the same 16 bytes, so
 * unpacklo/unpackhi repeat bytes 0-3 and 8-11, and the first nibble taken from
 * each byte is the high one; the weights used at step offsets t = 0..31 are the
 * nibbles of byte kk/2 + (t & 16) / 2 + (t & 7) / 2, high nibble for even t.
 * That is not the packer's order (:143-148), which the scalar tail follows.
 * order 0 runs the same arithmetic on the packer's order: offset t uses column
 * kk + t. */
EXPORT void oracle_gemm_nt_int4_gs(const float *a, const uint8_t *packed, const float *scale, float *c,
                                   size_t m, size_t n, size_t k, size_t group, int order) {
    size_t rowbytes = (k + 1) / 2, gpr = (k + group - 1) / group;
    const __m256i lut = _mm256_setr_epi8(0, 1, 2, 3, 4, 5, 6, 7, -8, -7, -6, -5, -4, -3, -2, -1,
                                         0, 1, 2, 3, 4, 5, 6, 7, -8, -7, -6, -5, -4, -3, -2, -1);
    const __m256i mask0f = _mm256_set1_epi8(0x0F);
    for (size_t i = 0; i < m; i++)
        for (size_t j = 0; j < n; j++) {
            const float *ar = a + i * k;
            const uint8_t *pr = packed + j * rowbytes;
            const float *sc = scale + j * gpr;
            float total = 0.0f;
            size_t g0 = 0;
            while (g0 < k) {
                size_t gend = g0 + group < k ? g0 + group : k;
                __m256 acc = _mm256_setzero_ps();
                size_t kk = g0;
                while (kk + 32 <= gend) {
                    __m256i q0, q1, q2, q3;
                    if (order == 1) {
                        __m128i raw = _mm_loadu_si128((const __m128i *)(pr + kk / 2));
                        __m256i v = _mm256_inserti128_si256(_mm256_castsi128_si256(raw), raw, 1);
                        __m256i lo_nib = _mm256_and_si256(_mm256_srli_epi16(v, 4), mask0f);
                        __m256i hi_nib = _mm256_and_si256(v, mask0f);
                        __m256i lo_i8 = _mm256_shuffle_epi8(lut, lo_nib);
                        __m256i hi_i8 = _mm256_shuffle_epi8(lut, hi_nib);
                        __m256i inter_lo = _mm256_unpacklo_epi8(lo_i8, hi_i8);
                        __m256i inter_hi = _mm256_unpackhi_epi8(lo_i8, hi_i8);
                        q0 = _mm256_cvtepi8_epi32(_mm256_castsi256_si128(inter_lo));
                        q1 = _mm256_cvtepi8_epi32(_mm256_extracti128_si256(inter_lo, 1));
                        q2 = _mm256_cvtepi8_epi32(_mm256_castsi256_si128(inter_hi));
                        q3 = _mm256_cvtepi8_epi32(_mm256_extracti128_si256(inter_hi, 1));
                    } else {
                        int8_t t8[32];
                        for (int t = 0; t < 32; t++) t8[t] = (int8_t)nib_value(pr[(kk + t) / 2], kk + t);
                        q0 = _mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i *)(t8 + 0)));
                        q1 = _mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i *)(t8 + 8)));
                        q2 = _mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i *)(t8 + 16)));
                        q3 = _mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i *)(t8 + 24)));
                    }
                    acc = _mm256_fmadd_ps(_mm256_loadu_ps(ar + kk), _mm256_cvtepi32_ps(q0), acc);
                    acc = _mm256_fmadd_ps(_mm256_loadu_ps(ar + kk + 8), _mm256_cvtepi32_ps(q1), acc);
                    acc = _mm256_fmadd_ps(_mm256_loadu_ps(ar + kk + 16), _mm256_cvtepi32_ps(q2), acc);
                    acc = _mm256_fmadd_ps(_mm256_loadu_ps(ar + kk + 24), _mm256_cvtepi32_ps(q3), acc);
                    kk += 32;
                }
                float s = hsum_ps(acc);
                while (kk < gend) {
                    float prod = ar[kk] * (float)nib_value(pr[kk / 2], kk);
                    s = s + prod;
                    kk += 1;
                }
                float part = s * sc[g0 / group];
                total = total + part;
                g0 = gend;
            }
            c[i * n + j] = total;
        }
}

/* tests/src/quant.rs:458-515: column RMS in f64 (sum over rows of w^2, / n,
 * sqrt), mean over columns; a column is an outlier when its RMS exceeds
 * thresh * mean. Per row amax over the other columns (0 -> 1e-30), s =
 * amax/127, q = round(w/s) clamped to +-127, outlier columns quantised to 0.
 * Writes the ascending outlier column indices to idx and returns their count. */
EXPORT size_t oracle_quant_int8_outliers(const float *w, size_t n, size_t k, float thresh, int8_t *q,
                                         float *scale, uint32_t *idx) {
    double tot = 0.0;
    size_t n_out = 0;
    double *col = (double *)calloc(k ? k : 1, sizeof(double));
    if (!col) return (size_t)-1;
    for (size_t i = 0; i < n; i++)
        for (size_t j = 0; j < k; j++) col[j] += (double)w[i * k + j] * (double)w[i * k + j];
    for (size_t j = 0; j < k; j++) {
        col[j] = sqrt(col[j] / (double)n);
        tot += col[j];
    }
    double mean = tot / (double)k;
    for (size_t j = 0; j < k; j++)
        if (col[j] > (double)thresh * mean) idx[n_out++] = (uint32_t)j;
    for (size_t i = 0; i < n; i++) {
        float amax = 0.0f;
        size_t o = 0;
        for (size_t j = 0; j < k; j++) {
            if (o < n_out && idx[o] == j) {
                o++;
                continue;
            }
            float av = fabsf(w[i * k + j]);
            if (av > amax) amax = av;
        }
        if (amax == 0.0f) amax = 1e-30f;
        float s = amax / 127.0f;
        scale[i] = s;
        o = 0;
        for (size_t j = 0; j < k; j++) {
            if (o < n_out && idx[o] == j) {
                o++;
                q[i * k + j] = 0;
                continue;
            }
            float r = roundf(w[i * k + j] / s);
            if (r < -127.0f) r = -127.0f;
            if (r > 127.0f) r = 127.0f;
            q[i * k + j] = (int8_t)r;
        }
    }
    free(col);
    return n_out;
}

/* tests/src/quant.rs:524-565: the int8 body of gemm_nt_int8 (:1256-1287 of the
 * kernels), v = s * scale[j], then v += a[i][jj] * w[j][jj] (mul then add) for
 * each listed outlier column in list order. w is the f32 weight [n][k]. */
EXPORT void oracle_gemm_nt_int8_outlier(const float *a, const int8_t *q, const float *scale, const float *w,
                                        const uint32_t *idx, size_t n_idx, float *c, size_t m, size_t n,
                                        size_t k) {
    gemm_nt_int8_cols(a, q, scale, c, m, n, k, 0, n);
    for (size_t i = 0; i < m; i++)
        for (size_t j = 0; j < n; j++) {
            float v = c[i * n + j];
            for (size_t t = 0; t < n_idx; t++) {
                float prod = a[i * k + idx[t]] * w[j * k + idx[t]];
                v = v + prod;
            }
            c[i * n + j] = v;
        }
}

/* Reference-convention error: max|got-ref| / max|ref| (tests/src/quant.rs:381-418). */
EXPORT double oracle_max_rel_err(const float *got, const float *ref, size_t n) {
    double md = 0.0, mr = 0.0;
    for (size_t i = 0; i < n; i++) {
        double d = fabs((double)got[i] - (double)ref[i]);
        double r = fabs((double)ref[i]);
        if (d > md || d != d) md = d;
        if (r > mr) mr = r;
    }
    return mr > 0 ? md / mr : md;
}
