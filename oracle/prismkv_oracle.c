/*
 * prismkv_oracle.c -- CPU restatement of the PrismKV decode-time retrieval path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library in prismkv_b200/: tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg may call it; the product path never does.
 *
 * Every function restates one function of the reference's portable path,
 * src/prismkv/core.py (cited per function), in plain C with fp32 arithmetic.
 * The reference delegates its arithmetic to PyTorch (torch>=2.4, pinned in the
 * reference's pyproject.toml:10).  Where the reference's result depends on the
 * order in which PyTorch / MKL reduce fp32 values, this file restates the
 * order that the reference's own runtime was observed to use (torch 2.11 CPU,
 * MKL 2024.2, x86-64 AVX-512); tests/golden/make_golden.py generated fixtures
 * from the reference itself and tests/test_oracle_golden.py checks that this
 * file reproduces them bit for bit.  The orders are:
 *
 *   F.linear(x[rows,d], W[F,d])      rows in [2,5]: 16 interleaved FMA chains
 *                                    (chain j takes k = j, j+16, ...), folded
 *                                    as ((c0+c4+c8+c12)+(c1+..)) + ((c2+..)+(c3+..));
 *                                    rows >= 6: one sequential FMA chain over k;
 *                                    bias added after the dot product.
 *   x.mean(0) over [n,d]             per column, PyTorch's 4-level cascade sum
 *                                    (blocks of 2^max(4, ceil(log2 n)/4) rows),
 *                                    for the leading 32*floor(d/32) columns; the
 *                                    remaining columns use the same cascade over
 *                                    groups of 4 rows (4 interleaved partials);
 *                                    then one division by n.
 *   v.sum(-1) over a contiguous row  8-lane vectors, 4 interleaved vector
 *                                    accumulators with the cascade above, lanes
 *                                    added left to right; rows shorter than 8
 *                                    use the scalar 4-partial form.
 *
 * Build: see oracle/Makefile (gcc -O2 -ffp-contract=off -fopenmp).  No
 * -ffast-math: every sum below must keep its written association.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#if defined(__x86_64__)
#include <immintrin.h>
#endif

/* ------------------------------------------------------------------------- */
/* Reduction orders                                                          */
/* ------------------------------------------------------------------------- */

static int64_t ceil_log2(int64_t n) {
    int64_t r = 0, t = 1;
    while (t < n) { t <<= 1; ++r; }
    return r;
}

/* PyTorch's multi-level cascade over `n` groups; each group contributes `width`
 * consecutive partial accumulators (width = 1 for a plain column).  Element
 * (group i, slot k) is at base[(i*width + k) * stride].  Result per slot k in
 * out[k].  Restates the cascade used by torch.sum / torch.mean on CPU. */
static void cascade_groups(const float *base, int64_t n, int width, int64_t stride, float *out) {
    const int levels = 4;
    int64_t lp = ceil_log2(n) / levels;
    if (lp < 4) lp = 4;
    const int64_t step = (int64_t)1 << lp, mask = step - 1;
    float acc[4][8];
    for (int j = 0; j < levels; ++j)
        for (int k = 0; k < width; ++k) acc[j][k] = 0.f;
    int64_t i = 0;
    while (i + step <= n) {
        for (int64_t s = 0; s < step; ++s, ++i)
            for (int k = 0; k < width; ++k) acc[0][k] += base[(i * width + k) * stride];
        for (int j = 1; j < levels; ++j) {
            for (int k = 0; k < width; ++k) { acc[j][k] += acc[j - 1][k]; acc[j - 1][k] = 0.f; }
            if ((i & (mask << (j * lp))) != 0) break;
        }
    }
    for (; i < n; ++i)
        for (int k = 0; k < width; ++k) acc[0][k] += base[(i * width + k) * stride];
    for (int j = 1; j < levels; ++j)
        for (int k = 0; k < width; ++k) acc[0][k] += acc[j][k];
    for (int k = 0; k < width; ++k) out[k] = acc[0][k];
}

/* Column sum of x[n, d] (row-major) for column c, in the order torch.mean(0)
 * uses for a contiguous fp32 matrix. */
static float column_sum(const float *x, int64_t n, int d, int c) {
    int plain = d >= 8 ? (d / 32) * 32 : (d == 4 ? 4 : 0);
    float r[8];
    if (c < plain) {
        cascade_groups(x + c, n, 1, d, r);
        return r[0];
    }
    /* 4 interleaved partials over groups of 4 rows, remainder rows into
     * partial 0, then partials folded left to right. */
    int64_t groups = n / 4;
    cascade_groups(x + c, groups, 4, d, r);
    for (int64_t i = groups * 4; i < n; ++i) r[0] += x[i * d + c];
    return ((r[0] + r[1]) + r[2]) + r[3];
}

/* core.py:80,87,88 -- x.mean(0). */
void orc_colmean(const float *x, int64_t n, int d, float *out) {
    for (int c = 0; c < d; ++c) out[c] = column_sum(x, n, d, c) / (float)n;
}

/* core.py:136 -- val.sum(-1) over one contiguous row of length n. */
float orc_rowsum(const float *x, int64_t n) {
    if (n < 8) {
        float r[8];
        int64_t groups = n / 4;
        cascade_groups(x, groups, 4, 1, r);
        for (int64_t i = groups * 4; i < n; ++i) r[0] += x[i];
        return ((r[0] + r[1]) + r[2]) + r[3];
    }
    const int W = 8;
    int64_t nvec = n / W, nilp = nvec / 4;
    float part[4][8];
    /* cascade over groups of 4 vectors; each "slot" is one (vector, lane). */
    {
        const int levels = 4;
        int64_t lp = ceil_log2(nilp) / levels;
        if (lp < 4) lp = 4;
        const int64_t step = (int64_t)1 << lp, mask = step - 1;
        float acc[4][4][8];
        memset(acc, 0, sizeof(acc));
        int64_t i = 0;
        while (i + step <= nilp) {
            for (int64_t s = 0; s < step; ++s, ++i)
                for (int k = 0; k < 4; ++k)
                    for (int l = 0; l < W; ++l) acc[0][k][l] += x[(i * 4 + k) * W + l];
            for (int j = 1; j < levels; ++j) {
                for (int k = 0; k < 4; ++k)
                    for (int l = 0; l < W; ++l) { acc[j][k][l] += acc[j - 1][k][l]; acc[j - 1][k][l] = 0.f; }
                if ((i & (mask << (j * lp))) != 0) break;
            }
        }
        for (; i < nilp; ++i)
            for (int k = 0; k < 4; ++k)
                for (int l = 0; l < W; ++l) acc[0][k][l] += x[(i * 4 + k) * W + l];
        for (int j = 1; j < levels; ++j)
            for (int k = 0; k < 4; ++k)
                for (int l = 0; l < W; ++l) acc[0][k][l] += acc[j][k][l];
        for (int k = 0; k < 4; ++k)
            for (int l = 0; l < W; ++l) part[k][l] = acc[0][k][l];
    }
    for (int64_t v = nilp * 4; v < nvec; ++v)
        for (int l = 0; l < W; ++l) part[0][l] += x[v * W + l];
    for (int k = 1; k < 4; ++k)
        for (int l = 0; l < W; ++l) part[0][l] += part[k][l];
    float total = 0.f;
    for (int64_t i = nvec * W; i < n; ++i) total += x[i];
    for (int l = 0; l < W; ++l) total += part[0][l];
    return total;
}

/* Dot products in the two orders F.linear was observed to use. */
static float dot_interleaved16(const float *x, const float *w, int d) {
    float c[16];
    for (int j = 0; j < 16; ++j) c[j] = 0.f;
    for (int k = 0; k < d; ++k) c[k & 15] = fmaf(x[k], w[k], c[k & 15]);
    float s[4];
    for (int l = 0; l < 4; ++l) {
        s[l] = c[l];
        s[l] = s[l] + c[l + 4];
        s[l] = s[l] + c[l + 8];
        s[l] = s[l] + c[l + 12];
    }
    return (s[0] + s[1]) + (s[2] + s[3]);
}

static float dot_sequential(const float *x, const float *w, int d) {
    float c = 0.f;
    for (int k = 0; k < d; ++k) c = fmaf(x[k], w[k], c);
    return c;
}

/* core.py:47-48 -- SharedSAE.dense: relu(F.linear(x, W_enc, b_enc)).
 * x[rows, d], W[F, d], b[F] -> out[rows, F]. */
void orc_dense(const float *x, int64_t rows, int d, const float *W, const float *b, int F, float *out) {
    const int interleaved = rows >= 2 && rows <= 5;
    #pragma omp parallel for schedule(static) if (rows * (int64_t)F > 65536)
    for (int64_t r = 0; r < rows; ++r) {
        for (int f = 0; f < F; ++f) {
            float v = interleaved ? dot_interleaved16(x + r * d, W + (int64_t)f * d, d)
                                  : dot_sequential(x + r * d, W + (int64_t)f * d, d);
            v = v + b[f];
            out[r * F + f] = v > 0.f ? v : 0.f;
        }
    }
}

/* ------------------------------------------------------------------------- */
/* core.py:13-26 -- positive_global_topk                                     */
/* ------------------------------------------------------------------------- */

static int cmp_float_desc(const void *a, const void *b) {
    float x = *(const float *)a, y = *(const float *)b;
    return (x < y) - (x > y);
}

/* count-th largest value of a[0..n) (values counted with multiplicity). */
static float kth_largest(const float *a, int64_t n, int64_t count) {
    /* Radix select on an order-preserving key. */
    uint32_t prefix = 0, pmask = 0;
    int64_t need = count;
    uint64_t *hist = (uint64_t *)calloc(65536, sizeof(uint64_t));
    for (int pass = 0; pass < 2; ++pass) {
        int shift = pass == 0 ? 16 : 0;
        memset(hist, 0, 65536 * sizeof(uint64_t));
        for (int64_t i = 0; i < n; ++i) {
            uint32_t u;
            memcpy(&u, &a[i], 4);
            u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
            if ((u & pmask) != prefix) continue;
            hist[(u >> shift) & 0xffffu]++;
        }
        int64_t acc = 0;
        int bin = 65535;
        for (; bin >= 0; --bin) {
            if (acc + (int64_t)hist[bin] >= need) break;
            acc += hist[bin];
        }
        need -= acc;
        prefix |= (uint32_t)bin << shift;
        pmask |= 0xffffu << shift;
    }
    free(hist);
    uint32_t u = prefix;
    u = (u & 0x80000000u) ? (u & 0x7fffffffu) : ~u;
    float v;
    memcpy(&v, &u, 4);
    return v;
}

/* Writes the selected flat indices (ascending strict part, then ties) to out,
 * returns their number.  `out` must hold min(count, n) entries. */
int64_t orc_positive_global_topk(const float *a, int64_t n, int64_t count, int64_t *out) {
    if (count > n) count = n;
    if (count <= 0) return 0;
    float thr = kth_largest(a, n, count);
    int64_t m = 0;
    for (int64_t i = 0; i < n; ++i)
        if (a[i] > thr && a[i] > 0.f) out[m++] = i;
    if (thr > 0.f) {
        int64_t want = count - m;
        for (int64_t i = 0; i < n && want > 0; ++i)
            if (a[i] == thr) { out[m++] = i; --want; }
    }
    return m;
}

/* ------------------------------------------------------------------------- */
/* core.py:76-89 -- summarize (population moments of original keys)         */
/* ------------------------------------------------------------------------- */

/* keys[n, d] fp32 (original keys upcast); CSR lists (offsets[F+1], ids);
 * writes mean[F, d], var[F, d]. */
void orc_summarize(const float *keys, int d, const int64_t *offsets, const int64_t *ids, int F,
                   float *mean, float *var) {
    #pragma omp parallel
    {
        int64_t cap = 0;
        float *x = NULL;
        #pragma omp for schedule(dynamic, 16)
        for (int b = 0; b < F; ++b) {
            int64_t lo = offsets[b], m = offsets[b + 1] - lo;
            float *mu = mean + (int64_t)b * d, *nu = var + (int64_t)b * d;
            if (m == 0) {
                for (int c = 0; c < d; ++c) mu[c] = nu[c] = 0.f;
                continue;
            }
            if (m * d > cap) { cap = m * d; free(x); x = (float *)malloc(cap * sizeof(float)); }
            for (int64_t r = 0; r < m; ++r) memcpy(x + r * d, keys + ids[lo + r] * d, d * sizeof(float));
            orc_colmean(x, m, d, mu);
            for (int64_t r = 0; r < m; ++r)
                for (int c = 0; c < d; ++c) { float t = x[r * d + c] - mu[c]; x[r * d + c] = t * t; }
            orc_colmean(x, m, d, nu);
        }
        free(x);
    }
}

/* ------------------------------------------------------------------------- */
/* core.py:92-103 -- build_index                                             */
/* ------------------------------------------------------------------------- */

/* keys[n, d] fp32 (original keys upcast).  center_in may be NULL (then the
 * keys' own mean, core.py:98).  Outputs: center_out[d], counts[F],
 * offsets[F+1], lists[cap] (token ids, ascending within each feature),
 * optional mean/var[F, d] (NULL to skip).  Returns the number of memberships,
 * or -1 if `cap` is too small, -2 on invalid arguments. */
int64_t orc_build_index(const float *keys, int64_t n, int d, const float *center_in, float key_scale,
                        const float *W, const float *b, int F, int key_mean,
                        float *center_out, int64_t *counts, int64_t *offsets, int64_t *lists, int64_t cap,
                        float *mean, float *var) {
    if (n <= 0 || d <= 0 || F <= 0 || !(key_scale > 0.f)) return -2;
    if (center_in) memcpy(center_out, center_in, d * sizeof(float));
    else orc_colmean(keys, n, d, center_out);
    float *x = (float *)malloc((size_t)n * d * sizeof(float));
    for (int64_t r = 0; r < n; ++r)
        for (int c = 0; c < d; ++c) x[r * d + c] = (keys[r * d + c] - center_out[c]) / key_scale;
    float *act = (float *)malloc((size_t)n * F * sizeof(float));
    orc_dense(x, n, d, W, b, F, act);
    free(x);
    int64_t budget = n * (int64_t)key_mean;
    int64_t total = n * (int64_t)F;
    int64_t want = budget < total ? budget : total;
    int64_t *flat = (int64_t *)malloc((want > 0 ? want : 1) * sizeof(int64_t));
    int64_t m = orc_positive_global_topk(act, total, budget, flat);
    free(act);
    if (m > cap) { free(flat); return -1; }
    /* core.py:101-102: per-feature token lists, sorted ascending. */
    for (int f = 0; f < F; ++f) counts[f] = 0;
    for (int64_t i = 0; i < m; ++i) counts[flat[i] % F]++;
    offsets[0] = 0;
    for (int f = 0; f < F; ++f) offsets[f + 1] = offsets[f] + counts[f];
    unsigned char *member = (unsigned char *)calloc((size_t)total, 1);
    for (int64_t i = 0; i < m; ++i) member[flat[i]] = 1;
    free(flat);
    int64_t *fill = (int64_t *)malloc(F * sizeof(int64_t));
    for (int f = 0; f < F; ++f) fill[f] = offsets[f];
    for (int64_t t = 0; t < n; ++t)
        for (int f = 0; f < F; ++f)
            if (member[t * F + f]) lists[fill[f]++] = t;
    free(fill);
    free(member);
    if (mean && var) orc_summarize(keys, d, offsets, lists, F, mean, var);
    return m;
}

/* ------------------------------------------------------------------------- */
/* core.py:92-103 at scale -- build_index without the [n, F] matrix          */
/* ------------------------------------------------------------------------- */

/* The same index as orc_build_index for n >= 6 rows (the sequential-chain
 * regime of F.linear), computed in token blocks so that memory stays O(n*d +
 * members) instead of n*F floats.  Activations are evaluated twice: pass 1
 * histograms the upper 16 bits of every positive activation to find the bin
 * that holds the count-th largest; pass 2 recomputes them and keeps the
 * entries in or above that bin, from which the exact threshold, the strict
 * members and the first ties in flat order follow as in core.py:13-26.  Each
 * activation is the same fp32 chain as dot_sequential (lane j of a vector
 * accumulator runs feature f+j's chain over k), so the result is bit-identical
 * to orc_build_index. */

#define STREAM_TB 32   /* token rows per block */
#define STREAM_FC 512  /* features per chunk (W^T chunk 256 KB) */

#if defined(__x86_64__)
/* out[r * nf + j] = relu(chain(x[r], W[f0 + j]) + b[f0 + j]) for r < rows,
 * j < nf; WT = W transposed, [d][F]. */
__attribute__((target("avx2,fma")))
static void dense_chunk_avx2(const float *x, int rows, int d, const float *WT, const float *b, int F,
                             int f0, int nf, float *out) {
    int j = 0;
    const __m256 zero = _mm256_setzero_ps();
    for (; j + 16 <= nf; j += 16) {
        const float *wt = WT + f0 + j;
        const __m256 b0 = _mm256_loadu_ps(b + f0 + j), b1 = _mm256_loadu_ps(b + f0 + j + 8);
        int r = 0;
        for (; r + 4 <= rows; r += 4) {
            __m256 a00 = zero, a01 = zero, a10 = zero, a11 = zero;
            __m256 a20 = zero, a21 = zero, a30 = zero, a31 = zero;
            const float *x0 = x + (int64_t)r * d;
            for (int k = 0; k < d; ++k) {
                const __m256 w0 = _mm256_loadu_ps(wt + (int64_t)k * F);
                const __m256 w1 = _mm256_loadu_ps(wt + (int64_t)k * F + 8);
                __m256 xb = _mm256_set1_ps(x0[k]);
                a00 = _mm256_fmadd_ps(xb, w0, a00); a01 = _mm256_fmadd_ps(xb, w1, a01);
                xb = _mm256_set1_ps(x0[d + k]);
                a10 = _mm256_fmadd_ps(xb, w0, a10); a11 = _mm256_fmadd_ps(xb, w1, a11);
                xb = _mm256_set1_ps(x0[2 * d + k]);
                a20 = _mm256_fmadd_ps(xb, w0, a20); a21 = _mm256_fmadd_ps(xb, w1, a21);
                xb = _mm256_set1_ps(x0[3 * d + k]);
                a30 = _mm256_fmadd_ps(xb, w0, a30); a31 = _mm256_fmadd_ps(xb, w1, a31);
            }
            __m256 acc[8] = {a00, a01, a10, a11, a20, a21, a30, a31};
            for (int t = 0; t < 8; ++t) {
                __m256 v = _mm256_add_ps(acc[t], (t & 1) ? b1 : b0);
                v = _mm256_and_ps(v, _mm256_cmp_ps(v, zero, _CMP_GT_OQ));
                _mm256_storeu_ps(out + (int64_t)(r + (t >> 1)) * nf + j + 8 * (t & 1), v);
            }
        }
        for (; r < rows; ++r) {
            __m256 a0 = zero, a1 = zero;
            const float *x0 = x + (int64_t)r * d;
            for (int k = 0; k < d; ++k) {
                const __m256 xb = _mm256_set1_ps(x0[k]);
                a0 = _mm256_fmadd_ps(xb, _mm256_loadu_ps(wt + (int64_t)k * F), a0);
                a1 = _mm256_fmadd_ps(xb, _mm256_loadu_ps(wt + (int64_t)k * F + 8), a1);
            }
            __m256 v0 = _mm256_add_ps(a0, b0), v1 = _mm256_add_ps(a1, b1);
            v0 = _mm256_and_ps(v0, _mm256_cmp_ps(v0, zero, _CMP_GT_OQ));
            v1 = _mm256_and_ps(v1, _mm256_cmp_ps(v1, zero, _CMP_GT_OQ));
            _mm256_storeu_ps(out + (int64_t)r * nf + j, v0);
            _mm256_storeu_ps(out + (int64_t)r * nf + j + 8, v1);
        }
    }
    for (; j < nf; ++j)
        for (int r = 0; r < rows; ++r) {
            float c = 0.f;
            for (int k = 0; k < d; ++k) c = fmaf(x[(int64_t)r * d + k], WT[(int64_t)k * F + f0 + j], c);
            c = c + b[f0 + j];
            out[(int64_t)r * nf + j] = c > 0.f ? c : 0.f;
        }
}
#endif

static void dense_chunk_scalar(const float *x, int rows, int d, const float *WT, const float *b, int F,
                               int f0, int nf, float *out) {
    for (int r = 0; r < rows; ++r)
        for (int j = 0; j < nf; ++j) {
            float c = 0.f;
            for (int k = 0; k < d; ++k) c = fmaf(x[(int64_t)r * d + k], WT[(int64_t)k * F + f0 + j], c);
            c = c + b[f0 + j];
            out[(int64_t)r * nf + j] = c > 0.f ? c : 0.f;
        }
}

static void dense_chunk(const float *x, int rows, int d, const float *WT, const float *b, int F, int f0,
                        int nf, float *out) {
#if defined(__x86_64__)
    if (__builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma")) {
        dense_chunk_avx2(x, rows, d, WT, b, F, f0, nf, out);
        return;
    }
#endif
    dense_chunk_scalar(x, rows, d, WT, b, F, f0, nf, out);
}

typedef struct { int64_t flat; float v; } fv_t;

static int cmp_i64(const void *a, const void *b) {
    int64_t x = *(const int64_t *)a, y = *(const int64_t *)b;
    return (x > y) - (x < y);
}

static int cmp_f32_desc(const void *a, const void *b) {
    float x = *(const float *)a, y = *(const float *)b;
    return (x < y) - (x > y);
}

static inline uint32_t f32_bits(float v) {
    uint32_t u;
    memcpy(&u, &v, 4);
    return u;
}

/* Arguments and return value as orc_build_index. */
int64_t orc_build_index_stream(const float *keys, int64_t n, int d, const float *center_in, float key_scale,
                               const float *W, const float *b, int F, int key_mean,
                               float *center_out, int64_t *counts, int64_t *offsets, int64_t *lists, int64_t cap,
                               float *mean, float *var) {
    if (n <= 0 || d <= 0 || F <= 0 || !(key_scale > 0.f)) return -2;
    if (n < 6)
        return orc_build_index(keys, n, d, center_in, key_scale, W, b, F, key_mean, center_out, counts, offsets,
                               lists, cap, mean, var);
    if (center_in) memcpy(center_out, center_in, d * sizeof(float));
    else orc_colmean(keys, n, d, center_out);
    float *x = (float *)malloc((size_t)n * d * sizeof(float));
    for (int64_t r = 0; r < n; ++r)
        for (int c = 0; c < d; ++c) x[r * d + c] = (keys[r * d + c] - center_out[c]) / key_scale;
    float *WT = (float *)malloc((size_t)F * d * sizeof(float));
    for (int f = 0; f < F; ++f)
        for (int k = 0; k < d; ++k) WT[(int64_t)k * F + f] = W[(int64_t)f * d + k];
    const int64_t total = n * (int64_t)F;
    const int64_t budget = n * (int64_t)key_mean;
    const int64_t count = budget < total ? budget : total;
    const int64_t nblocks = (n + STREAM_TB - 1) / STREAM_TB;

    /* Pass 1: histogram of the upper 16 bits of the positive activations. */
    uint64_t *hist = (uint64_t *)calloc(65536, sizeof(uint64_t));
    #pragma omp parallel
    {
        uint64_t *h = (uint64_t *)calloc(65536, sizeof(uint64_t));
        float *act = (float *)malloc((size_t)STREAM_TB * STREAM_FC * sizeof(float));
        #pragma omp for schedule(dynamic, 4)
        for (int64_t blk = 0; blk < nblocks; ++blk) {
            const int64_t t0 = blk * STREAM_TB;
            const int rows = (int)(n - t0 < STREAM_TB ? n - t0 : STREAM_TB);
            for (int f0 = 0; f0 < F; f0 += STREAM_FC) {
                const int nf = F - f0 < STREAM_FC ? F - f0 : STREAM_FC;
                dense_chunk(x + t0 * d, rows, d, WT, b, F, f0, nf, act);
                for (int64_t i = 0; i < (int64_t)rows * nf; ++i)
                    if (act[i] > 0.f) h[f32_bits(act[i]) >> 16]++;
            }
        }
        #pragma omp critical
        for (int i = 0; i < 65536; ++i) hist[i] += h[i];
        free(h);
        free(act);
    }
    uint64_t positives = 0;
    for (int i = 0; i < 65536; ++i) positives += hist[i];
    /* Positive floats order like their bit patterns.  With fewer positives
     * than `count` the threshold is zero and every positive is a member. */
    const int all_pos = (int64_t)positives <= count;
    int bin = 0;
    int64_t above = 0;
    if (!all_pos) {
        for (bin = 65535; bin > 0; --bin) {
            if (above + (int64_t)hist[bin] >= count) break;
            above += hist[bin];
        }
    }
    free(hist);

    /* Pass 2: keep every positive entry in or above the threshold's bin. */
    int nthreads = 1;
#ifdef _OPENMP
    nthreads = omp_get_max_threads();
#endif
    fv_t **kept = (fv_t **)calloc(nthreads, sizeof(fv_t *));
    int64_t *nkept = (int64_t *)calloc(nthreads, sizeof(int64_t));
    #pragma omp parallel
    {
        int tid = 0;
#ifdef _OPENMP
        tid = omp_get_thread_num();
#endif
        int64_t capk = 1 << 16, m = 0;
        fv_t *buf = (fv_t *)malloc(capk * sizeof(fv_t));
        float *act = (float *)malloc((size_t)STREAM_TB * STREAM_FC * sizeof(float));
        #pragma omp for schedule(dynamic, 4)
        for (int64_t blk = 0; blk < nblocks; ++blk) {
            const int64_t t0 = blk * STREAM_TB;
            const int rows = (int)(n - t0 < STREAM_TB ? n - t0 : STREAM_TB);
            for (int f0 = 0; f0 < F; f0 += STREAM_FC) {
                const int nf = F - f0 < STREAM_FC ? F - f0 : STREAM_FC;
                dense_chunk(x + t0 * d, rows, d, WT, b, F, f0, nf, act);
                for (int r = 0; r < rows; ++r)
                    for (int j = 0; j < nf; ++j) {
                        const float v = act[(int64_t)r * nf + j];
                        if (!(v > 0.f) || (int)(f32_bits(v) >> 16) < bin) continue;
                        if (m == capk) { capk *= 2; buf = (fv_t *)realloc(buf, capk * sizeof(fv_t)); }
                        buf[m].flat = (t0 + r) * (int64_t)F + f0 + j;
                        buf[m].v = v;
                        ++m;
                    }
            }
        }
        kept[tid] = buf;
        nkept[tid] = m;
        free(act);
    }
    free(x);
    free(WT);
    int64_t nk = 0;
    for (int t = 0; t < nthreads; ++t) nk += nkept[t];
    fv_t *all = (fv_t *)malloc((nk > 0 ? nk : 1) * sizeof(fv_t));
    {
        int64_t o = 0;
        for (int t = 0; t < nthreads; ++t) {
            memcpy(all + o, kept[t], nkept[t] * sizeof(fv_t));
            o += nkept[t];
            free(kept[t]);
        }
    }
    free(kept);
    free(nkept);

    /* Exact threshold: the (count - above)-th largest value in the bin. */
    float thr = 0.f;
    if (!all_pos) {
        int64_t inbin = 0;
        for (int64_t i = 0; i < nk; ++i) inbin += (int)(f32_bits(all[i].v) >> 16) == bin;
        float *vals = (float *)malloc((inbin > 0 ? inbin : 1) * sizeof(float));
        int64_t q = 0;
        for (int64_t i = 0; i < nk; ++i)
            if ((int)(f32_bits(all[i].v) >> 16) == bin) vals[q++] = all[i].v;
        qsort(vals, inbin, sizeof(float), cmp_f32_desc);
        thr = vals[count - above - 1];
        free(vals);
    }
    /* Members: strict entries above the threshold, then ties in flat order. */
    int64_t *flat = (int64_t *)malloc((nk > 0 ? nk : 1) * sizeof(int64_t));
    int64_t m = 0, ntie = 0;
    int64_t *tie = (int64_t *)malloc((nk > 0 ? nk : 1) * sizeof(int64_t));
    for (int64_t i = 0; i < nk; ++i) {
        if (all_pos || all[i].v > thr) flat[m++] = all[i].flat;
        else if (all[i].v == thr) tie[ntie++] = all[i].flat;
    }
    free(all);
    if (!all_pos) {
        qsort(tie, ntie, sizeof(int64_t), cmp_i64);
        int64_t want = count - m;
        for (int64_t i = 0; i < ntie && i < want; ++i) flat[m++] = tie[i];
    }
    free(tie);
    if (m > cap) { free(flat); return -1; }
    qsort(flat, m, sizeof(int64_t), cmp_i64);
    for (int f = 0; f < F; ++f) counts[f] = 0;
    for (int64_t i = 0; i < m; ++i) counts[flat[i] % F]++;
    offsets[0] = 0;
    for (int f = 0; f < F; ++f) offsets[f + 1] = offsets[f] + counts[f];
    int64_t *fill = (int64_t *)malloc(F * sizeof(int64_t));
    for (int f = 0; f < F; ++f) fill[f] = offsets[f];
    for (int64_t i = 0; i < m; ++i) lists[fill[flat[i] % F]++] = flat[i] / F;
    free(fill);
    free(flat);
    if (mean && var) orc_summarize(keys, d, offsets, lists, F, mean, var);
    return m;
}

/* core.py:186-201 -- append_index moment merge (elementwise, in the
 * reference's operation order).  counts_a/b are the old/new bucket sizes. */
void orc_merge_moments(const int64_t *counts_a, const float *mean_a, const float *var_a,
                       const int64_t *counts_b, const float *mean_b, const float *var_b,
                       int F, int d, float *mean_out, float *var_out) {
    for (int f = 0; f < F; ++f) {
        float a = (float)counts_a[f], b = (float)counts_b[f];
        float tot = a + b;
        float den = tot > 1.f ? tot : 1.f;
        float w = (a * b) / (den * den);
        for (int c = 0; c < d; ++c) {
            int64_t i = (int64_t)f * d + c;
            float mu = (a * mean_a[i] + b * mean_b[i]) / den;
            float nu = (a * var_a[i] + b * var_b[i]) / den;
            float dm = mean_a[i] - mean_b[i];
            nu = nu + w * (dm * dm);
            mean_out[i] = mu;
            var_out[i] = nu;
        }
    }
}

/* ------------------------------------------------------------------------- */
/* core.py:106-139 -- bucket_scores                                          */
/* ------------------------------------------------------------------------- */

/* Stable descending order of `score` restricted to indices passing `keep`. */
typedef struct { float v; int i; } vi_t;
static int cmp_vi_desc(const void *a, const void *b) {
    const vi_t *x = (const vi_t *)a, *y = (const vi_t *)b;
    if (x->v > y->v) return -1;
    if (x->v < y->v) return 1;
    return (x->i > y->i) - (x->i < y->i);
}

/* q_activation router, core.py:131-139.  q[G, d] fp32 (already upcast),
 * W[F, d], b[F], counts[F] (liveness).  Outputs: score[F];
 * order[<= G*k]; topk_ids[G, k] (per-head picks, rank order).  Returns the
 * number of entries in `order`. */
int orc_route_qact(const float *q, int G, int d, const float *W, const float *b, int F,
                   float query_scale, int k, const int64_t *counts,
                   float *score, int *order, int *topk_ids) {
    if (k > F) k = F;
    float *x = (float *)malloc((size_t)G * d * sizeof(float));
    for (int i = 0; i < G * d; ++i) x[i] = q[i] / query_scale;
    float *a = (float *)malloc((size_t)G * F * sizeof(float));
    orc_dense(x, G, d, W, b, F, a);
    free(x);
    vi_t *tmp = (vi_t *)malloc((size_t)F * sizeof(vi_t));
    float *val = (float *)malloc((size_t)k * sizeof(float));
    for (int f = 0; f < F; ++f) score[f] = 0.f;
    for (int h = 0; h < G; ++h) {
        for (int f = 0; f < F; ++f) { tmp[f].v = a[(int64_t)h * F + f]; tmp[f].i = f; }
        qsort(tmp, F, sizeof(vi_t), cmp_vi_desc);
        for (int r = 0; r < k; ++r) { val[r] = tmp[r].v; topk_ids[h * k + r] = tmp[r].i; }
        float s = orc_rowsum(val, k);
        const float floor_ = 1e-20f;
        if (s < floor_) s = floor_;
        for (int r = 0; r < k; ++r) {
            float v = val[r] / s;
            v = v / (float)G;
            score[topk_ids[h * k + r]] += v;
        }
    }
    for (int f = 0; f < F; ++f) { tmp[f].v = score[f]; tmp[f].i = f; }
    qsort(tmp, F, sizeof(vi_t), cmp_vi_desc);
    int n = 0;
    for (int r = 0; r < F; ++r) {
        int f = tmp[r].i;
        if (tmp[r].v > 0.f && counts[f] > 0) order[n++] = f;
    }
    free(tmp); free(val); free(a);
    return n;
}

/* Ordering half of the moments router, core.py:127-130, applied to given
 * per-bucket scores: stable descending order of live buckets, first k. */
int orc_order_live(const float *score, const int64_t *counts, int F, int k, int *order) {
    vi_t *tmp = (vi_t *)malloc((size_t)F * sizeof(vi_t));
    for (int f = 0; f < F; ++f) { tmp[f].v = score[f]; tmp[f].i = f; }
    qsort(tmp, F, sizeof(vi_t), cmp_vi_desc);
    int n = 0;
    for (int r = 0; r < F && n < k; ++r)
        if (counts[tmp[r].i] > 0) order[n++] = tmp[r].i;
    free(tmp);
    return n;
}

/* moments router scores, core.py:117-128.  terms bit 0 = count, 1 = mean,
 * 2 = variance.  score[F]; writes logits through the softmax in fp32 with the
 * C library's expf (the reference uses PyTorch's vectorised exp; the two agree
 * to about 1 ulp, so this score is compared with a tolerance). */
void orc_moments_score(const float *q, int G, int d, const float *mean, const float *var,
                       const int64_t *counts, int F, int terms, float *score) {
    float *lg = (float *)malloc((size_t)G * F * sizeof(float));
    float *qq = (float *)malloc((size_t)G * d * sizeof(float));
    float *zero = (float *)calloc(F, sizeof(float));
    int live_any = 0;
    for (int f = 0; f < F; ++f) live_any |= counts[f] > 0;
    for (int i = 0; i < G * F; ++i) lg[i] = 0.f;
    if (terms & 1)
        for (int h = 0; h < G; ++h)
            for (int f = 0; f < F; ++f) lg[h * F + f] += logf((float)(counts[f] > 1 ? counts[f] : 1));
    float *t = (float *)malloc((size_t)G * F * sizeof(float));
    if (terms & 2) {
        /* q @ mean.T / sqrt(d) */
        for (int h = 0; h < G; ++h)
            for (int f = 0; f < F; ++f) {
                const float *x = q + h * d, *w = mean + (int64_t)f * d;
                float v = (G >= 2 && G <= 5) ? dot_interleaved16(x, w, d) : dot_sequential(x, w, d);
                t[h * F + f] = v / (float)sqrt((double)d);
            }
        for (int i = 0; i < G * F; ++i) lg[i] += t[i];
    }
    if (terms & 4) {
        for (int i = 0; i < G * d; ++i) qq[i] = q[i] * q[i];
        for (int h = 0; h < G; ++h)
            for (int f = 0; f < F; ++f) {
                const float *x = qq + h * d, *w = var + (int64_t)f * d;
                float v = (G >= 2 && G <= 5) ? dot_interleaved16(x, w, d) : dot_sequential(x, w, d);
                t[h * F + f] = v / (float)(2 * d);
            }
        for (int i = 0; i < G * F; ++i) lg[i] += t[i];
    }
    free(t);
    for (int f = 0; f < F; ++f) score[f] = 0.f;
    if (live_any) {
        for (int h = 0; h < G; ++h) {
            float *row = lg + (int64_t)h * F;
            float mx = -INFINITY;
            for (int f = 0; f < F; ++f) { if (counts[f] <= 0) row[f] = -INFINITY; if (row[f] > mx) mx = row[f]; }
            double den = 0.0;
            for (int f = 0; f < F; ++f) { row[f] = expf(row[f] - mx); den += row[f]; }
            for (int f = 0; f < F; ++f) score[f] += (float)(row[f] / den);
        }
        for (int f = 0; f < F; ++f) score[f] = score[f] / (float)G;
    }
    free(lg); free(qq); free(zero);
}

/* ------------------------------------------------------------------------- */
/* core.py:142-167 -- select_buckets greedy with skip                        */
/* ------------------------------------------------------------------------- */

/* order[n_order] candidate buckets; CSR lists (offsets[F+1], ids) of a
 * history-token index; limit = floor(history * unique_cap) or history.
 * Outputs: out_ids (ascending, unique), features (accepted buckets in
 * acceptance order), *n_features, *raw.  Returns the number of ids. */
int64_t orc_select(const int *order, int n_order, const int64_t *offsets, const int64_t *ids,
                   int64_t history, int64_t limit, int64_t *out_ids, int *features, int *n_features,
                   int64_t *raw) {
    unsigned char *chosen = (unsigned char *)calloc((size_t)(history > 0 ? history : 1), 1);
    int64_t count = 0, rawc = 0;
    int nf = 0;
    for (int c = 0; c < n_order; ++c) {
        int b = order[c];
        int64_t lo = offsets[b], hi = offsets[b + 1], fresh = 0;
        for (int64_t j = lo; j < hi; ++j) fresh += !chosen[ids[j]];
        if (count + fresh > limit) continue;
        for (int64_t j = lo; j < hi; ++j) chosen[ids[j]] = 1;
        count += fresh;
        rawc += hi - lo;
        features[nf++] = b;
    }
    int64_t m = 0;
    for (int64_t t = 0; t < history; ++t)
        if (chosen[t]) out_ids[m++] = t;
    free(chosen);
    *n_features = nf;
    *raw = rawc;
    return m;
}

/* ------------------------------------------------------------------------- */
/* core.py:170-183 -- attend (exact softmax over selected rows + dense tail) */
/* ------------------------------------------------------------------------- */

/* q[G, d], keys/values[total, d] fp32 (upcast), old_ids[n_old] (validated by
 * the caller), history.  Computed in double; out[G, d] in fp32 (the caller
 * casts to the query dtype). */
void orc_attend(const float *q, int G, int d, const float *keys, const float *values, int64_t total,
                const int64_t *old_ids, int64_t n_old, int64_t history, float *out) {
    int64_t rows = n_old + (total - history);
    if (rows <= 0) {
        for (int i = 0; i < G * d; ++i) out[i] = 0.f;
        return;
    }
    double *logit = (double *)malloc((size_t)rows * sizeof(double));
    double scale = 1.0 / sqrt((double)d);
    for (int h = 0; h < G; ++h) {
        double mx = -INFINITY;
        for (int64_t r = 0; r < rows; ++r) {
            int64_t row = r < n_old ? old_ids[r] : history + (r - n_old);
            double s = 0.0;
            for (int c = 0; c < d; ++c) s += (double)q[h * d + c] * (double)keys[row * d + c];
            logit[r] = s * scale;
            if (logit[r] > mx) mx = logit[r];
        }
        double den = 0.0;
        for (int64_t r = 0; r < rows; ++r) { logit[r] = exp(logit[r] - mx); den += logit[r]; }
        for (int c = 0; c < d; ++c) {
            double acc = 0.0;
            for (int64_t r = 0; r < rows; ++r) {
                int64_t row = r < n_old ? old_ids[r] : history + (r - n_old);
                acc += logit[r] * (double)values[row * d + c];
            }
            out[h * d + c] = (float)(acc / den);
        }
    }
    free(logit);
}

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
