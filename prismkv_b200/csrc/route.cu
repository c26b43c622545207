// Query-side routing kernels: q_activation (SAE encode + per-head top-k +
// normalised aggregation) and the moments router.
//
// q_activation restates src/prismkv/core.py:131-139.  The encode reproduces
// the fp32 dot-product order the reference's F.linear takes for a [G, d]
// query block (G in 2..5: sixteen interleaved FMA chains folded pairwise;
// G >= 6: one sequential chain), so the activations -- and with them the
// routed bucket ids -- are bit-identical to the reference's.
#include "common.cuh"
#include "topk.cuh"
#include "mma.cuh"

namespace pk {

constexpr int kEncD = 128;            // head dim compiled for the encoders
constexpr int kEncHeads = 32;         // heads per CTA tile
constexpr int kEncFeat = 128;         // features per CTA tile
constexpr int kEncThreads = 128;      // 4 warps x (8 heads, 4 features/lane)
constexpr int kWPitch = kEncD + 4;    // padded row pitch of the W tile (floats)

enum DotOrder { kInterleaved16 = 0, kSequential = 1 };

// Position of element k of a d=128 row in the chain-major layout used for the
// interleaved order: chain j = k % 16 owns positions 8j .. 8j+7.
__device__ __forceinline__ int perm16(int k) { return 8 * (k & 15) + (k >> 4); }

template <int ORDER, typename QT>
__global__ void __launch_bounds__(kEncThreads)
qact_encode_kernel(const QT* __restrict__ q, const int* __restrict__ units, int n_units, int G,
                   const float* __restrict__ W, const float* __restrict__ bias, float query_scale, int F,
                   float* __restrict__ act) {
    extern __shared__ __align__(16) float smem[];
    float* Xs = smem;                          // [kEncHeads][kEncD]
    float* Ws = smem + kEncHeads * kEncD;      // [kEncFeat][kWPitch]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int f0 = blockIdx.x * kEncFeat;
    const int h0 = blockIdx.y * kEncHeads;
    const int n_heads = n_units * G;

    // Stage the query tile (x = q / query_scale, core.py:133) and W tile.
    for (int e = tid; e < kEncHeads * kEncD; e += kEncThreads) {
        const int hh = e / kEncD, kk = e % kEncD;
        const int h = h0 + hh;
        float x = 0.f;
        if (h < n_heads) {
            const int ui = h / G, g = h % G;
            const int u = units ? units[ui] : ui;
            x = __fdiv_rn(load_f(q, ((int64_t)u * G + g) * kEncD + kk), query_scale);
        }
        const int pos = ORDER == kInterleaved16 ? perm16(kk) : kk;
        Xs[hh * kEncD + pos] = x;
    }
    for (int e = tid; e < kEncFeat * (kEncD / 4); e += kEncThreads) {
        const int ff = e / (kEncD / 4), c = e % (kEncD / 4);
        const int f = f0 + ff;
        float4 w = make_float4(0.f, 0.f, 0.f, 0.f);
        if (f < F) w = reinterpret_cast<const float4*>(W + (int64_t)f * kEncD)[c];
        float* row = Ws + ff * kWPitch;
        const int k = 4 * c;
        if (ORDER == kInterleaved16) {
            row[perm16(k)] = w.x; row[perm16(k + 1)] = w.y; row[perm16(k + 2)] = w.z; row[perm16(k + 3)] = w.w;
        } else {
            *reinterpret_cast<float4*>(row + k) = w;
        }
    }
    __syncthreads();

    // Thread tile: heads warp*8 .. +7 (warp-uniform: broadcast loads),
    // features lane + 32*i (i < 4; conflict-free with the padded pitch).
    const float* xb = Xs + (warp * 8) * kEncD;
    const float* wb = Ws + lane * kWPitch;
    float res[8][4];

    if (ORDER == kInterleaved16) {
        float t0[8][4], t1[8][4], s[8][4];
#pragma unroll 1
        for (int l = 0; l < 4; ++l) {
#pragma unroll 1
            for (int uu = 0; uu < 4; ++uu) {
                const int j = l + 4 * uu;
                float acc[8][4];
#pragma unroll
                for (int a = 0; a < 8; ++a)
#pragma unroll
                    for (int b = 0; b < 4; ++b) acc[a][b] = 0.f;
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const int p = 8 * j + 4 * half;
                    float4 xv[8], wv[4];
#pragma unroll
                    for (int a = 0; a < 8; ++a) xv[a] = *reinterpret_cast<const float4*>(xb + a * kEncD + p);
#pragma unroll
                    for (int b = 0; b < 4; ++b) wv[b] = *reinterpret_cast<const float4*>(wb + b * 32 * kWPitch + p);
#pragma unroll
                    for (int a = 0; a < 8; ++a)
#pragma unroll
                        for (int b = 0; b < 4; ++b) {
                            acc[a][b] = fmaf(xv[a].x, wv[b].x, acc[a][b]);
                            acc[a][b] = fmaf(xv[a].y, wv[b].y, acc[a][b]);
                            acc[a][b] = fmaf(xv[a].z, wv[b].z, acc[a][b]);
                            acc[a][b] = fmaf(xv[a].w, wv[b].w, acc[a][b]);
                        }
                }
#pragma unroll
                for (int a = 0; a < 8; ++a)
#pragma unroll
                    for (int b = 0; b < 4; ++b) s[a][b] = uu == 0 ? acc[a][b] : __fadd_rn(s[a][b], acc[a][b]);
            }
#pragma unroll
            for (int a = 0; a < 8; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    if (l == 0) t0[a][b] = s[a][b];
                    else if (l == 1) t0[a][b] = __fadd_rn(t0[a][b], s[a][b]);
                    else if (l == 2) t1[a][b] = s[a][b];
                    else t1[a][b] = __fadd_rn(t1[a][b], s[a][b]);
                }
        }
#pragma unroll
        for (int a = 0; a < 8; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) res[a][b] = __fadd_rn(t0[a][b], t1[a][b]);
    } else {
#pragma unroll
        for (int a = 0; a < 8; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) res[a][b] = 0.f;
#pragma unroll 4
        for (int p = 0; p < kEncD; p += 4) {
            float4 xv[8], wv[4];
#pragma unroll
            for (int a = 0; a < 8; ++a) xv[a] = *reinterpret_cast<const float4*>(xb + a * kEncD + p);
#pragma unroll
            for (int b = 0; b < 4; ++b) wv[b] = *reinterpret_cast<const float4*>(wb + b * 32 * kWPitch + p);
#pragma unroll
            for (int a = 0; a < 8; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    res[a][b] = fmaf(xv[a].x, wv[b].x, res[a][b]);
                    res[a][b] = fmaf(xv[a].y, wv[b].y, res[a][b]);
                    res[a][b] = fmaf(xv[a].z, wv[b].z, res[a][b]);
                    res[a][b] = fmaf(xv[a].w, wv[b].w, res[a][b]);
                }
        }
    }

    // Epilogue: + bias, ReLU (core.py:48), store act[u, g, f].
#pragma unroll
    for (int a = 0; a < 8; ++a) {
        const int h = h0 + warp * 8 + a;
        if (h >= n_heads) continue;
        const int ui = h / G, g = h % G;
        const int u = units ? units[ui] : ui;
        float* out = act + ((int64_t)u * G + g) * F;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int f = f0 + lane + 32 * b;
            if (f < F) {
                const float v = __fadd_rn(res[a][b], bias[f]);
                out[f] = v > 0.f ? v : 0.f;
            }
        }
    }
}

// Per (unit, head): exact top-k of the head's activations (stable descending,
// ties -> lower feature id, core.py:134), normalisation by the k-slot sum in
// the reference's summation order (core.py:136), division by G (core.py:137).
// The last of the unit's G CTAs aggregates the heads in head order
// (scatter_add_ of core.py:137), keeps score > 0 and live buckets, and emits
// the candidate order (core.py:138-139).
struct QactSmem {
    TopkScratch tk;
    int sel[256];
    uint32_t selkey[256];
    float val[256];
    float norm;
    int is_last;
};

// Given this head's m positive picks in rank order (sm.sel = feature ids,
// sm.selkey = value bits), write the normalised contributions and, in the
// unit's last CTA, aggregate.  `agg` is shared scratch of >= 16*G*k bytes.
__device__ void head_finish(int u, int g, int G, int F, int k, int m, QactSmem& sm, void* agg,
                            const int* __restrict__ counts, int* __restrict__ head_ids, float* __restrict__ head_val,
                            int* __restrict__ unit_done, int* __restrict__ order, int* __restrict__ n_order,
                            int order_stride, float* __restrict__ score) {
    const int tid = threadIdx.x, nt = blockDim.x;
    for (int r = tid; r < k; r += nt) sm.val[r] = r < m ? __uint_as_float(sm.selkey[r]) : 0.f;
    __syncthreads();
    if (tid == 0) {
        const float s = torch_rowsum(sm.val, k);
        const float floor_ = 1e-20f;
        sm.norm = s < floor_ ? floor_ : s;
    }
    __syncthreads();
    const float s = sm.norm;
    int* hid = head_ids + ((int64_t)u * G + g) * k;
    float* hv = head_val + ((int64_t)u * G + g) * k;
    for (int r = tid; r < k; r += nt) {
        float v = r < m ? __uint_as_float(sm.selkey[r]) : 0.f;
        v = __fdiv_rn(v, s);
        v = __fdiv_rn(v, (float)G);
        hid[r] = r < m ? sm.sel[r] : -1;
        hv[r] = v;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) sm.is_last = atomicAdd(&unit_done[u], 1) == G - 1;
    __syncthreads();
    if (!sm.is_last) return;
    __threadfence();

    const int E = G * k;  // <= 256
    int* eid = reinterpret_cast<int*>(agg);            // [E]
    float* ev = reinterpret_cast<float*>(agg) + E;     // [E]
    float* sc = ev + E;                                // [E]
    int* cand = reinterpret_cast<int*>(sc + E);        // [E]
    for (int e = tid; e < E; e += nt) {
        eid[e] = __ldcg(head_ids + (int64_t)u * E + e);
        ev[e] = __ldcg(head_val + (int64_t)u * E + e);
    }
    __syncthreads();
    for (int e = tid; e < E; e += nt) {
        const int f = eid[e];
        const int h = e / k;
        bool first = f >= 0;
        for (int e2 = 0; e2 < h * k && first; ++e2) first = eid[e2] != f;
        float acc = 0.f;
        if (first) {
            for (int hh = 0; hh < G; ++hh)
                for (int r = 0; r < k; ++r)
                    if (eid[hh * k + r] == f) { acc = __fadd_rn(acc, ev[hh * k + r]); break; }
        }
        const bool keep = first && acc > 0.f && counts[(int64_t)u * F + f] > 0;
        sc[e] = acc;
        cand[e] = keep ? f : -1;
        if (score && first) score[(int64_t)u * F + f] = acc;
    }
    __syncthreads();
    // Rank the kept candidates by (score desc, feature asc).
    for (int e = tid; e < E; e += nt) {
        const int f = cand[e];
        if (f < 0) continue;
        const float v = sc[e];
        int r = 0;
        for (int e2 = 0; e2 < E; ++e2) {
            const int f2 = cand[e2];
            if (f2 < 0) continue;
            const float v2 = sc[e2];
            r += (v2 > v) || (v2 == v && f2 < f);
        }
        order[(int64_t)u * order_stride + r] = f;
    }
    int mine = 0;
    for (int e = tid; e < E; e += nt) mine += cand[e] >= 0;
    int tot;
    block_exclusive_scan(mine, sm.tk.scan, &tot);
    if (tid == 0) {
        n_order[u] = tot;
        unit_done[u] = 0;
    }
}

// Exact path: the activations in `act` are the exact ones (qact_encode).
__global__ void __launch_bounds__(256)
qact_select_kernel(const float* __restrict__ act, const int* __restrict__ units, int G, int F, int k,
                   const int* __restrict__ counts, int* __restrict__ head_ids, float* __restrict__ head_val,
                   int* __restrict__ unit_done, int* __restrict__ order, int* __restrict__ n_order, int order_stride,
                   float* __restrict__ score, int* __restrict__ topk_out) {
    extern __shared__ __align__(16) uint32_t vbits[];  // [F] activation bits
    __shared__ QactSmem sm;
    const int tid = threadIdx.x, nt = blockDim.x;
    const int ui = blockIdx.x / G, g = blockIdx.x % G;
    const int u = units ? units[ui] : ui;
    const float* a = act + ((int64_t)u * G + g) * F;
    for (int i = tid; i < F; i += nt) vbits[i] = __float_as_uint(a[i]);
    __syncthreads();

    // Positive activations only: zero-valued picks add nothing to the score.
    const int m = block_topk(
        F, k, [&](int i) { return vbits[i]; }, [&](int i) { return __uint_as_float(vbits[i]) > 0.f; }, sm.sel,
        sm.selkey, sm.tk);
    if (topk_out) {
        // Zero-valued slots take the lowest feature ids whose value is not
        // positive (the rest of the stable descending argsort).
        int* tk = topk_out + ((int64_t)u * G + g) * k;
        for (int r = tid; r < m; r += nt) tk[r] = sm.sel[r];
        if (m < k) {
            int base = 0;
            for (int start = 0; start < F && base < k - m; start += nt) {
                const int i = start + tid;
                const bool z = i < F && !(__uint_as_float(vbits[i]) > 0.f);
                int tot;
                const int at = block_exclusive_scan(z ? 1 : 0, sm.tk.scan, &tot);
                if (z && base + at < k - m) tk[m + base + at] = i;
                base += tot;
            }
        }
    }
    __syncthreads();
    head_finish(u, g, G, F, k, m, sm, vbits, counts, head_ids, head_val, unit_done, order, n_order, order_stride,
                score);
}

// ---------------------------------------------------------------------------
// Bound-filtered routing: approximate activations on the tensor cores, then
// exact fp32 recomputation of the features that can reach the top-k.
// ---------------------------------------------------------------------------

// Per feature: bf16 copy of W_f and an upper bound of ||W_f||_2.
__global__ void sae_prepare_kernel(const float* __restrict__ W, int F, __nv_bfloat16* __restrict__ Wb,
                                   float* __restrict__ wn) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int f = blockIdx.x * (blockDim.x >> 5) + warp;
    if (f >= F) return;
    const float4 w = reinterpret_cast<const float4*>(W + (int64_t)f * kEncD)[lane];
    __nv_bfloat162 lo = __floats2bfloat162_rn(w.x, w.y), hi = __floats2bfloat162_rn(w.z, w.w);
    reinterpret_cast<__nv_bfloat162*>(Wb + (int64_t)f * kEncD)[2 * lane] = lo;
    reinterpret_cast<__nv_bfloat162*>(Wb + (int64_t)f * kEncD)[2 * lane + 1] = hi;
    float ss = fmaf(w.x, w.x, fmaf(w.y, w.y, fmaf(w.z, w.z, w.w * w.w)));
    ss = warp_sum(ss);
    // fp32 sum and sqrt are each within a few ulp: widen by 2^-12.
    if (lane == 0) wn[f] = sqrtf(ss) * (1.0f + 1.0f / 4096.0f);
}

constexpr int kApxHeads = 64, kApxFeat = 128, kApxThreads = 128;

// v[u, g, f] ~= (q/scale) . W_f + b_f with bf16 operands on mma.sync and fp32
// accumulation: a 64-head x 128-feature tile per CTA, 16 heads per warp.
template <typename QT>
__global__ void __launch_bounds__(kApxThreads)
qact_approx_kernel(const QT* __restrict__ q, const int* __restrict__ units, int n_units, int G,
                   const __nv_bfloat16* __restrict__ Wb, const float* __restrict__ bias, float query_scale, int F,
                   float* __restrict__ act) {
    extern __shared__ __align__(128) uint8_t apx_smem[];
    uint8_t* Xs = apx_smem;                     // [64 rows][256 B] swizzled
    uint8_t* Wt = apx_smem + kApxHeads * 256;   // [128 rows][256 B] swizzled
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int f0 = blockIdx.x * kApxFeat, h0 = blockIdx.y * kApxHeads;
    const int n_heads = n_units * G;
    for (int c = tid; c < kApxFeat * 16; c += kApxThreads) {
        const int row = c >> 4, ch = c & 15;
        const int f = f0 + row;
        const bool valid = f < F;
        cp_async_16(smem_addr(Wt) + swz(row, ch), Wb + (int64_t)(valid ? f : 0) * kEncD + ch * 8, valid);
    }
    cp_async_commit_group();
    for (int e = tid; e < kApxHeads * 64; e += kApxThreads) {
        const int row = e >> 6, pc = e & 63;
        const int h = h0 + row;
        float x0 = 0.f, x1 = 0.f;
        if (h < n_heads) {
            const int ui = h / G, g = h % G;
            const int u = units ? units[ui] : ui;
            const int64_t base = ((int64_t)u * G + g) * kEncD + 2 * pc;
            x0 = __fdiv_rn(load_f(q, base), query_scale);
            x1 = __fdiv_rn(load_f(q, base + 1), query_scale);
        }
        *reinterpret_cast<__nv_bfloat162*>(Xs + swz(row, pc >> 2) + (pc & 3) * 4) = __floats2bfloat162_rn(x0, x1);
    }
    cp_async_wait_group<0>();
    __syncthreads();

    float acc[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    const int mi = lane >> 3, r = lane & 7;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
        uint32_t a[4];
        ldsm_x4(smem_addr(Xs) + swz(warp * 16 + (mi & 1) * 8 + r, 2 * kk + (mi >> 1)), a);
#pragma unroll
        for (int np = 0; np < 8; ++np) {
            uint32_t b[4];
            ldsm_x4(smem_addr(Wt) + swz(np * 16 + (mi >> 1) * 8 + r, 2 * kk + (mi & 1)), b);
            mma_16816(acc[2 * np], a, b[0], b[1]);
            mma_16816(acc[2 * np + 1], a, b[2], b[3]);
        }
    }
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        const int h = h0 + warp * 16 + (lane >> 2) + half * 8;
        if (h >= n_heads) continue;
        const int ui = h / G, g = h % G;
        const int u = units ? units[ui] : ui;
        float* out = act + ((int64_t)u * G + g) * F;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int f = f0 + 8 * j + 2 * (lane & 3);
            if (f + 1 < F) {
                *reinterpret_cast<float2*>(out + f) =
                    make_float2(acc[j][2 * half] + bias[f], acc[j][2 * half + 1] + bias[f + 1]);
            } else if (f < F) {
                out[f] = acc[j][2 * half] + bias[f];
            }
        }
    }
}

__device__ __forceinline__ uint32_t fkey(float x) {
    const uint32_t b = __float_as_uint(x);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float fkey_inv(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

template <int ORDER>
__device__ __forceinline__ float exact_dot(const float* __restrict__ x, const float* __restrict__ w) {
    if (ORDER == kInterleaved16) {
        float c[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) c[j] = 0.f;
#pragma unroll
        for (int k4 = 0; k4 < kEncD / 4; ++k4) {
            const float4 wv = reinterpret_cast<const float4*>(w)[k4];
            const int k = 4 * k4;
            c[(k + 0) & 15] = fmaf(x[k + 0], wv.x, c[(k + 0) & 15]);
            c[(k + 1) & 15] = fmaf(x[k + 1], wv.y, c[(k + 1) & 15]);
            c[(k + 2) & 15] = fmaf(x[k + 2], wv.z, c[(k + 2) & 15]);
            c[(k + 3) & 15] = fmaf(x[k + 3], wv.w, c[(k + 3) & 15]);
        }
        float s[4];
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            s[l] = c[l];
            s[l] = __fadd_rn(s[l], c[l + 4]);
            s[l] = __fadd_rn(s[l], c[l + 8]);
            s[l] = __fadd_rn(s[l], c[l + 12]);
        }
        return __fadd_rn(__fadd_rn(s[0], s[1]), __fadd_rn(s[2], s[3]));
    } else {
        float c = 0.f;
#pragma unroll
        for (int k4 = 0; k4 < kEncD / 4; ++k4) {
            const float4 wv = reinterpret_cast<const float4*>(w)[k4];
            const int k = 4 * k4;
            c = fmaf(x[k + 0], wv.x, c);
            c = fmaf(x[k + 1], wv.y, c);
            c = fmaf(x[k + 2], wv.z, c);
            c = fmaf(x[k + 3], wv.w, c);
        }
        return c;
    }
}

constexpr int kCandCap = 2048;

struct FastSmem {
    QactSmem q;
    float x[kEncD];
    float red[32];
    int cand[kCandCap];
    float cval[kCandCap];
    int wc[32];
    int ncand;
};

// Per (unit, head): lambda = k-th largest lower bound; candidates = features
// whose upper bound reaches lambda (a superset of the exact top-k, ties
// included); exact fp32 activations for the candidates in the reference's
// dot-product order; exact top-k among them.  Too many candidates (near-
// degenerate inputs): every feature is recomputed exactly instead.
template <int ORDER, typename QT>
__global__ void __launch_bounds__(256)
qact_select_fast_kernel(const QT* __restrict__ q, const float* __restrict__ act, const int* __restrict__ units, int G,
                        const float* __restrict__ W, const float* __restrict__ bias, const float* __restrict__ wn,
                        float query_scale, int F, int k, const int* __restrict__ counts, int* __restrict__ head_ids,
                        float* __restrict__ head_val, int* __restrict__ unit_done, int* __restrict__ order,
                        int* __restrict__ n_order, int order_stride, float* __restrict__ score, int store_up) {
    // sA[F]: order-preserving keys of the lower bounds (later: exact values
    // if every feature is recomputed); sB[F]: upper bounds when they fit.
    extern __shared__ __align__(16) uint32_t sA[];
    float* sB = reinterpret_cast<float*>(sA + F);
    __shared__ FastSmem sm;
    const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
    const int ui = blockIdx.x / G, g = blockIdx.x % G;
    const int u = units ? units[ui] : ui;
    const float* a = act + ((int64_t)u * G + g) * F;
    float ss = 0.f;
    for (int c = tid; c < kEncD; c += nt) {
        const float x = __fdiv_rn(load_f(q, ((int64_t)u * G + g) * kEncD + c), query_scale);
        sm.x[c] = x;
        ss = fmaf(x, x, ss);
    }
    ss = warp_sum(ss);
    if (lane == 0) sm.red[warp] = ss;
    __syncthreads();
    if (tid == 0) {
        float t = 0.f;
        for (int w = 0; w < nw; ++w) t += sm.red[w];
        sm.red[0] = sqrtf(t) * (1.0f + 1.0f / 4096.0f);
    }
    __syncthreads();
    const float xn = sm.red[0];
    // |v_approx - v_exact| <= eps_f: bf16 operand rounding (2^-8 each),
    // fp32 accumulation and the exact order's own rounding, x2 margin.
    auto eps = [&](int f, float v) { return 0.015625f * xn * wn[f] + 9.5367431640625e-07f * fabsf(v); };
    // One streaming pass (independent, coalesced loads) computes both bounds.
    for (int i = tid; i < F; i += nt) {
        const float v = a[i];
        const float e = eps(i, v);
        sA[i] = fkey(v - e);
        if (store_up) sB[i] = v + e;
    }
    __syncthreads();
    auto upper = [&](int i) { return store_up ? sB[i] : a[i] + eps(i, a[i]); };
    const int m0 = block_topk(
        F, k, [&](int i) { return sA[i]; }, [&](int i) { return true; }, sm.q.sel, sm.q.selkey, sm.q.tk);
    const float lam = m0 >= k ? fkey_inv(sm.q.selkey[k - 1]) : -INFINITY;
    const bool pos_only = !(lam > 0.f);
    // Ordered gather of the candidates (feature order).
    const int seg = ((F + nw - 1) / nw + 31) / 32 * 32;
    const int w0 = min(F, warp * seg), w1 = min(F, w0 + seg);
    int mine = 0;
    for (int base = w0; base < w1; base += 32) {
        const int i = base + lane;
        bool c = false;
        if (i < w1) {
            const float up = upper(i);
            c = pos_only ? up > 0.f : up >= lam;
        }
        mine += __popc(__ballot_sync(0xffffffffu, c));
    }
    if (lane == 0) sm.wc[warp] = mine;
    __syncthreads();
    int before = 0, total = 0;
    for (int w = 0; w < nw; ++w) { if (w < warp) before += sm.wc[w]; total += sm.wc[w]; }
    const bool all_exact = total > kCandCap;
    if (!all_exact) {
        int out = before;
        for (int base = w0; base < w1; base += 32) {
            const int i = base + lane;
            bool c = false;
            if (i < w1) {
                const float up = upper(i);
                c = pos_only ? up > 0.f : up >= lam;
            }
            const unsigned cm = __ballot_sync(0xffffffffu, c);
            if (c) sm.cand[out + __popc(cm & lanemask_lt())] = i;
            out += __popc(cm);
        }
    }
    __syncthreads();
    int m;
    if (!all_exact) {
        for (int c = tid; c < total; c += nt) {
            const int f = sm.cand[c];
            const float z = __fadd_rn(exact_dot<ORDER>(sm.x, W + (int64_t)f * kEncD), bias[f]);
            sm.cval[c] = z > 0.f ? z : 0.f;
        }
        __syncthreads();
        m = block_topk(
            total, k, [&](int i) { return __float_as_uint(sm.cval[i]); }, [&](int i) { return sm.cval[i] > 0.f; },
            sm.q.sel, sm.q.selkey, sm.q.tk);
        for (int r = tid; r < m; r += nt) sm.q.sel[r] = sm.cand[sm.q.sel[r]];
    } else {
        for (int f = tid; f < F; f += nt) {
            const float z = __fadd_rn(exact_dot<ORDER>(sm.x, W + (int64_t)f * kEncD), bias[f]);
            sA[f] = __float_as_uint(z > 0.f ? z : 0.f);
        }
        __syncthreads();
        m = block_topk(
            F, k, [&](int i) { return sA[i]; }, [&](int i) { return __uint_as_float(sA[i]) > 0.f; }, sm.q.sel,
            sm.q.selkey, sm.q.tk);
    }
    __syncthreads();
    head_finish(u, g, G, F, k, m, sm.q, sA, counts, head_ids, head_val, unit_done, order, n_order, order_stride,
                score);
}

__global__ void zero_rows_kernel(float* __restrict__ score, const int* __restrict__ units, int F) {
    const int u = units ? units[blockIdx.x] : blockIdx.x;
    for (int i = threadIdx.x; i < F; i += blockDim.x) score[(int64_t)u * F + i] = 0.f;
}

// ---------------------------------------------------------------------------
// moments router (core.py:117-130)
// ---------------------------------------------------------------------------

// logits[u, g, f] = log(max(n,1)) + q.mu/sqrt(d) + (q*q).var/(2d), -inf for
// empty buckets.  One warp per (unit, feature); lanes split d.
template <typename QT>
__global__ void moments_logits_kernel(const QT* __restrict__ q, const float* __restrict__ mean,
                                      const float* __restrict__ var, const int* __restrict__ counts, int terms,
                                      int G, int d, int F, float* __restrict__ logits) {
    const int u = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int f = blockIdx.x * (blockDim.x >> 5) + warp;
    if (f >= F) return;
    const int n = counts[(int64_t)u * F + f];
    const float* mu = mean + ((int64_t)u * F + f) * d;
    const float* nu = var + ((int64_t)u * F + f) * d;
    const float sq = sqrtf((float)d);
    for (int g = 0; g < G; ++g) {
        float dm = 0.f, dv = 0.f;
        for (int c = lane; c < d; c += 32) {
            const float x = load_f(q, ((int64_t)u * G + g) * d + c);
            if (terms & PK_TERM_MEAN) dm = fmaf(x, mu[c], dm);
            if (terms & PK_TERM_VARIANCE) dv = fmaf(x * x, nu[c], dv);
        }
        dm = warp_sum(dm);
        dv = warp_sum(dv);
        if (lane == 0) {
            float l = 0.f;
            if (terms & PK_TERM_COUNT) l += logf((float)(n > 1 ? n : 1));
            if (terms & PK_TERM_MEAN) l += dm / sq;
            if (terms & PK_TERM_VARIANCE) l += dv / (float)(2 * d);
            logits[((int64_t)u * G + g) * F + f] = n > 0 ? l : -INFINITY;
        }
    }
}

// score[u, f] = mean over heads of softmax(logits[u, g, :]); then the first k
// live buckets by descending score (ties -> lower id).
__global__ void __launch_bounds__(256)
moments_select_kernel(const float* __restrict__ logits, const int* __restrict__ counts, int G, int F, int k,
                      float* __restrict__ score, int* __restrict__ order, int* __restrict__ n_order,
                      int order_stride) {
    extern __shared__ __align__(16) uint32_t sbits[];  // [F]
    __shared__ QactSmem sm;
    __shared__ float red[32];
    const int u = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
    bool any_live = false;
    for (int i = tid; i < F; i += nt) any_live |= counts[(int64_t)u * F + i] > 0;
    any_live = __syncthreads_or(any_live);
    float* sc = score + (int64_t)u * F;
    for (int i = tid; i < F; i += nt) sc[i] = 0.f;
    __syncthreads();
    if (any_live) {
        for (int g = 0; g < G; ++g) {
            const float* l = logits + ((int64_t)u * G + g) * F;
            float mx = -INFINITY;
            for (int i = tid; i < F; i += nt) mx = fmaxf(mx, l[i]);
            mx = warp_max(mx);
            if ((tid & 31) == 0) red[tid >> 5] = mx;
            __syncthreads();
            if (tid < 32) {
                float v = tid < (nt >> 5) ? red[tid] : -INFINITY;
                v = warp_max(v);
                if (tid == 0) red[0] = v;
            }
            __syncthreads();
            mx = red[0];
            __syncthreads();
            float z = 0.f;
            for (int i = tid; i < F; i += nt) z += expf(l[i] - mx);
            z = warp_sum(z);
            if ((tid & 31) == 0) red[tid >> 5] = z;
            __syncthreads();
            if (tid < 32) {
                float v = tid < (nt >> 5) ? red[tid] : 0.f;
                v = warp_sum(v);
                if (tid == 0) red[0] = v;
            }
            __syncthreads();
            z = red[0];
            __syncthreads();
            for (int i = tid; i < F; i += nt) sc[i] += expf(l[i] - mx) / z;
            __syncthreads();
        }
        for (int i = tid; i < F; i += nt) sc[i] = sc[i] / (float)G;
        __syncthreads();
    }
    for (int i = tid; i < F; i += nt) sbits[i] = __float_as_uint(sc[i]);
    __syncthreads();
    const int m = block_topk(
        F, k, [&](int i) { return sbits[i]; }, [&](int i) { return counts[(int64_t)u * F + i] > 0; }, sm.sel,
        sm.selkey, sm.tk);
    for (int r = tid; r < m; r += nt) order[(int64_t)u * order_stride + r] = sm.sel[r];
    if (tid == 0) n_order[u] = m;
}

}  // namespace pk

using namespace pk;

extern "C" size_t pk_route_qact_workspace_bytes(int U, int G, int F, int k) {
    const size_t act = (size_t)U * G * F * sizeof(float);
    const size_t heads = (size_t)U * G * k * (sizeof(int) + sizeof(float));
    const size_t done = (size_t)U * sizeof(int);
    return (act + 255) / 256 * 256 + (heads + 255) / 256 * 256 + (done + 255) / 256 * 256;
}

extern "C" int pk_sae_prepare(uint64_t w_enc, int F, int d, uint64_t w_bf16, uint64_t w_norm, uint64_t stream) {
    if (F < 1 || !w_enc || !w_bf16 || !w_norm) return PK_ERR_ARG;
    if (d != kEncD) return PK_ERR_UNSUPPORTED;
    sae_prepare_kernel<<<(F + 7) / 8, 256, 0, (cudaStream_t)stream>>>((const float*)w_enc, F, (__nv_bfloat16*)w_bf16,
                                                                      (float*)w_norm);
    PK_CHECK_LAUNCH();
    return PK_OK;
}

extern "C" int pk_route_qact(uint64_t q, int q_dtype, uint64_t units, int n_units, uint64_t w_enc, uint64_t b_enc,
                             uint64_t w_bf16, uint64_t w_norm,
                             float query_scale, uint64_t counts, int U, int G, int d, int F, int k,
                             uint64_t workspace, uint64_t workspace_bytes, uint64_t order, uint64_t n_order,
                             int order_stride, uint64_t score, uint64_t topk, uint64_t stream) {
    if (U < 1 || G < 1 || F < 1 || k < 1 || n_units < 0 || n_units > U || !(query_scale > 0.f)) return PK_ERR_ARG;
    if (k > F) k = F;
    if (G * k > 256 || order_stride < G * k) return PK_ERR_ARG;
    if (d != kEncD) return PK_ERR_UNSUPPORTED;
    if ((size_t)F * sizeof(uint32_t) > 200 * 1024) return PK_ERR_UNSUPPORTED;
    if (workspace_bytes < pk_route_qact_workspace_bytes(U, G, F, k)) return PK_ERR_WORKSPACE;
    if (!q || !w_enc || !b_enc || !counts || !workspace || !order || !n_order) return PK_ERR_ARG;
    if (n_units == 0) return PK_OK;
    cudaStream_t st = (cudaStream_t)stream;
    char* ws = (char*)workspace;
    float* act = (float*)ws;
    size_t off = ((size_t)U * G * F * sizeof(float) + 255) / 256 * 256;
    int* hid = (int*)(ws + off);
    float* hval = (float*)(hid + (size_t)U * G * k);
    off += ((size_t)U * G * k * (sizeof(int) + sizeof(float)) + 255) / 256 * 256;
    int* done = (int*)(ws + off);
    const int* ul = (const int*)units;

    // The order F.linear takes for a [G, d] block (see file header).
    const bool inter = G >= 2 && G <= 5;
    if (w_bf16 && w_norm && !topk) {
        // Bound-filtered path: approximate encode on the tensor cores, exact
        // recomputation of the features that can reach the top-k.
        if (q_dtype != PK_BF16 && q_dtype != PK_F32) return PK_ERR_ARG;
        dim3 ag((F + kApxFeat - 1) / kApxFeat, (n_units * G + kApxHeads - 1) / kApxHeads);
        const int asmem = (kApxHeads + kApxFeat) * 256;
        if (q_dtype == PK_BF16) {
            cudaFuncSetAttribute(qact_approx_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, asmem);
            qact_approx_kernel<__nv_bfloat16><<<ag, kApxThreads, asmem, st>>>(
                (const __nv_bfloat16*)q, ul, n_units, G, (const __nv_bfloat16*)w_bf16, (const float*)b_enc,
                query_scale, F, act);
        } else {
            cudaFuncSetAttribute(qact_approx_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, asmem);
            qact_approx_kernel<float><<<ag, kApxThreads, asmem, st>>>((const float*)q, ul, n_units, G,
                                                                      (const __nv_bfloat16*)w_bf16,
                                                                      (const float*)b_enc, query_scale, F, act);
        }
        PK_CHECK_LAUNCH();
        if (score) {
            zero_rows_kernel<<<n_units, 256, 0, st>>>((float*)score, ul, F);
            PK_CHECK_LAUNCH();
        }
        // Lower-bound keys always; upper bounds too when both fit on chip.
        const int store_up = (size_t)8 * F <= 160 * 1024 ? 1 : 0;
        size_t fsmem = (size_t)(store_up ? 8 : 4) * F;
        if ((size_t)16 * G * k > fsmem) fsmem = (size_t)16 * G * k;
#define PK_LAUNCH_FAST(ORD, QT)                                                                                  \
    do {                                                                                                         \
        cudaFuncSetAttribute(qact_select_fast_kernel<ORD, QT>, cudaFuncAttributeMaxDynamicSharedMemorySize,      \
                             (int)fsmem);                                                                        \
        qact_select_fast_kernel<ORD, QT><<<n_units * G, 256, fsmem, st>>>(                                       \
            (const QT*)q, act, ul, G, (const float*)w_enc, (const float*)b_enc, (const float*)w_norm,            \
            query_scale, F, k, (const int*)counts, hid, hval, done, (int*)order, (int*)n_order, order_stride,    \
            (float*)score, store_up);                                                                            \
    } while (0)
        if (q_dtype == PK_BF16) {
            if (inter) PK_LAUNCH_FAST(kInterleaved16, __nv_bfloat16); else PK_LAUNCH_FAST(kSequential, __nv_bfloat16);
        } else {
            if (inter) PK_LAUNCH_FAST(kInterleaved16, float); else PK_LAUNCH_FAST(kSequential, float);
        }
#undef PK_LAUNCH_FAST
        PK_CHECK_LAUNCH();
        return PK_OK;
    }
    dim3 grid((F + kEncFeat - 1) / kEncFeat, (n_units * G + kEncHeads - 1) / kEncHeads);
    const size_t smem = (size_t)(kEncHeads * kEncD + kEncFeat * kWPitch) * sizeof(float);
#define PK_LAUNCH_ENC(ORD, QT)                                                                           \
    do {                                                                                                 \
        cudaFuncSetAttribute(qact_encode_kernel<ORD, QT>, cudaFuncAttributeMaxDynamicSharedMemorySize,   \
                             (int)smem);                                                                 \
        qact_encode_kernel<ORD, QT><<<grid, kEncThreads, smem, st>>>(                                    \
            (const QT*)q, ul, n_units, G, (const float*)w_enc, (const float*)b_enc, query_scale, F, act); \
    } while (0)
    if (q_dtype == PK_BF16) {
        if (inter) PK_LAUNCH_ENC(kInterleaved16, __nv_bfloat16); else PK_LAUNCH_ENC(kSequential, __nv_bfloat16);
    } else if (q_dtype == PK_F32) {
        if (inter) PK_LAUNCH_ENC(kInterleaved16, float); else PK_LAUNCH_ENC(kSequential, float);
    } else {
        return PK_ERR_ARG;
    }
#undef PK_LAUNCH_ENC
    PK_CHECK_LAUNCH();
    if (score) {
        zero_rows_kernel<<<n_units, 256, 0, st>>>((float*)score, ul, F);
        PK_CHECK_LAUNCH();
    }
    size_t ssmem = (size_t)F * sizeof(uint32_t);
    const size_t agg = (size_t)16 * G * k;
    if (agg > ssmem) ssmem = agg;
    cudaFuncSetAttribute(qact_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ssmem);
    qact_select_kernel<<<n_units * G, 256, ssmem, st>>>(act, ul, G, F, k, (const int*)counts, hid, hval, done,
                                                        (int*)order, (int*)n_order, order_stride, (float*)score,
                                                        (int*)topk);
    PK_CHECK_LAUNCH();
    return PK_OK;
}

extern "C" size_t pk_route_moments_workspace_bytes(int U, int G, int F) {
    return ((size_t)U * G * F * sizeof(float) + 255) / 256 * 256;
}

extern "C" int pk_route_moments(uint64_t q, int q_dtype, uint64_t mean, uint64_t var, uint64_t counts, int terms,
                                int U, int G, int d, int F, int k, uint64_t workspace, uint64_t workspace_bytes,
                                uint64_t score, uint64_t order, uint64_t n_order, int order_stride,
                                uint64_t stream) {
    if (U < 1 || G < 1 || d < 1 || F < 1 || k < 1 || terms <= 0 || terms > 7) return PK_ERR_ARG;
    if (k > F) k = F;
    if (k > 256 || order_stride < k) return PK_ERR_ARG;
    if ((size_t)F * sizeof(uint32_t) > 200 * 1024) return PK_ERR_UNSUPPORTED;
    if (workspace_bytes < pk_route_moments_workspace_bytes(U, G, F)) return PK_ERR_WORKSPACE;
    if (!q || !mean || !var || !counts || !workspace || !score || !order || !n_order) return PK_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    float* logits = (float*)workspace;
    dim3 grid((F + 7) / 8, U);
    if (q_dtype == PK_BF16)
        moments_logits_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)q, (const float*)mean,
                                                                   (const float*)var, (const int*)counts, terms,
                                                                   G, d, F, logits);
    else if (q_dtype == PK_F32)
        moments_logits_kernel<float><<<grid, 256, 0, st>>>((const float*)q, (const float*)mean, (const float*)var,
                                                           (const int*)counts, terms, G, d, F, logits);
    else
        return PK_ERR_ARG;
    PK_CHECK_LAUNCH();
    const size_t ssmem = (size_t)F * sizeof(uint32_t);
    cudaFuncSetAttribute(moments_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ssmem);
    moments_select_kernel<<<U, 256, ssmem, st>>>(logits, (const int*)counts, G, F, k, (float*)score, (int*)order,
                                                 (int*)n_order, order_stride);
    PK_CHECK_LAUNCH();
    return PK_OK;
}
