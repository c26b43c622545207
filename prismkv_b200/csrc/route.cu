// Query-side routing kernels: q_activation (SAE encode + per-head top-k +
// normalised aggregation) and the moments router.
//
// q_activation restates src/prismkv/core.py:131-139.  The encode reproduces
// the fp32 dot-product order the reference's F.linear takes for a [G, d]
// query block (G in 2..5: sixteen interleaved FMA chains folded pairwise;
// G >= 6: one sequential chain), so the activations -- and with them the
// routed bucket ids -- are bit-identical to the reference's.
#include <cuda_fp16.h>

#include <cooperative_groups.h>

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

// This head's m positive picks in rank order (sm.sel = feature ids,
// sm.selkey = value bits), normalised by their sum (floored at 1e-20) and
// divided by G, stored in feature order into hid[k] / hv[k], unused slots
// INT_MAX / 0 (the layout the aggregation's binary searches expect).
__device__ void head_picks(int G, int k, int m, QactSmem& sm, int* hid, float* hv) {
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
    for (int r = tid; r < k; r += nt) {
        if (r < m) {
            const int f = sm.sel[r];
            // Position in feature order (a repeated id, which only a
            // malformed merge input can produce, takes the next slot).
            int pos = 0;
            for (int r2 = 0; r2 < m; ++r2) pos += sm.sel[r2] < f || (sm.sel[r2] == f && r2 < r);
            float v = __uint_as_float(sm.selkey[r]);
            v = __fdiv_rn(v, s);
            v = __fdiv_rn(v, (float)G);
            hid[pos] = f;
            hv[pos] = v;
        } else {
            hid[r] = INT32_MAX;
            hv[r] = 0.f;
        }
    }
}

// Scores of the unit's G*k pick entries (eid/ev: G segments of k sorted
// entries in shared memory): score[f] = 0 + v_h1 + v_h2 + ... over the heads
// that picked f, in head order (scatter_add_ of core.py:137), kept at f's
// first entry; cand[e] = f for a first entry with score > 0 and a live
// bucket (live[e], or counts[f] > 0 read here when live is null), else -1.
// One entry per thread; every thread must call it.
__device__ void unit_scores(int u, int G, int F, int k, const int* eid, const float* ev, const int* live,
                            const int* __restrict__ counts, float* sc, int* cand, int e_lo, int e_hi,
                            float* __restrict__ score) {
    const int tid = threadIdx.x, nt = blockDim.x;
    const int E = G * k;
    // Position of feature f in head hh's sorted picks, or -1.
    auto find = [&](int hh, int f) -> int {
        const int* seg = eid + hh * k;
        int lo = 0, hi = k;
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (seg[mid] < f) lo = mid + 1;
            else hi = mid;
        }
        return lo < k && seg[lo] == f ? lo : -1;
    };
    for (int e = tid; e < E; e += nt) {
        const int f = eid[e];
        const int h = e / k;
        bool first = f != INT32_MAX;
        for (int hh = 0; hh < h && first; ++hh) first = find(hh, f) < 0;
        float acc = 0.f;
        if (first) {
            acc = ev[e];
            for (int hh = h + 1; hh < G; ++hh) {
                const int i = find(hh, f);
                if (i >= 0) acc = __fadd_rn(acc, ev[hh * k + i]);
            }
        }
        const bool keep = first && acc > 0.f && (live ? live[e] != 0 : counts[(int64_t)u * F + f] > 0);
        sc[e] = acc;
        cand[e] = keep ? f : -1;
        if (score && first && e >= e_lo && e < e_hi) score[(int64_t)u * F + f] = acc;
    }
    __syncthreads();
}

// order[u, r] = f for the kept entries e in [e_lo, e_hi), r = the rank of
// (score desc, feature asc) among all kept entries; P threads (a power of
// two within a warp) share each entry's comparisons.  Returns the number of
// kept entries (every thread).  Every thread must call it.
__device__ int unit_rank(int u, int E, const float* sc, const int* cand, int e_lo, int e_hi, int* scan,
                         int* __restrict__ order, int order_stride) {
    const int tid = threadIdx.x, nt = blockDim.x;
    const int n_own = e_hi - e_lo;
    int P = 1;
    while (P < 32 && 2 * P * n_own <= nt) P *= 2;
    for (int base = 0; base < n_own * P; base += nt) {
        const int e = e_lo + (base + tid) / P, part = (base + tid) % P;
        int f = -1;
        float v = 0.f;
        if (e < e_hi) {
            f = cand[e];
            v = sc[e];
        }
        int r = 0;
        if (f >= 0) {
            for (int e2 = part; e2 < E; e2 += P) {
                const int f2 = cand[e2];
                if (f2 < 0) continue;
                const float v2 = sc[e2];
                // (A repeated feature id, from a malformed merge input only,
                // ranks by entry: the slots stay distinct.)
                r += (v2 > v) || (v2 == v && (f2 < f || (f2 == f && e2 < e)));
            }
        }
        for (int o = 1; o < P; o <<= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
        if (f >= 0 && part == 0) order[(int64_t)u * order_stride + r] = f;
    }
    int mine = 0;
    for (int e = tid; e < E; e += nt) mine += cand[e] >= 0;
    int tot;
    block_exclusive_scan(mine, scan, &tot);
    return tot;
}

// Given this head's m positive picks in rank order, write the normalised
// contributions to global memory and, in the unit's last CTA (an arrival
// counter), aggregate.  `agg` is shared scratch of >= 16*G*k bytes.
__device__ void head_finish(int u, int g, int G, int F, int k, int m, QactSmem& sm, void* agg,
                            const int* __restrict__ counts, int* __restrict__ head_ids, float* __restrict__ head_val,
                            int* __restrict__ unit_done, int* __restrict__ order, int* __restrict__ n_order,
                            int order_stride, float* __restrict__ score) {
    const int tid = threadIdx.x, nt = blockDim.x;
    head_picks(G, k, m, sm, head_ids + ((int64_t)u * G + g) * k, head_val + ((int64_t)u * G + g) * k);
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
    unit_scores(u, G, F, k, eid, ev, nullptr, counts, sc, cand, 0, E, score);
    const int tot = unit_rank(u, E, sc, cand, 0, E, sm.tk.scan, order, order_stride);
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

constexpr int kApxHeads = 64, kApxFeat = 128, kApxThreads = 256;
constexpr int kMaxGroups = 512;

__device__ __forceinline__ uint32_t fkey(float x) {
    const uint32_t b = __float_as_uint(x);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float fkey_inv(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// Features per group for the routing threshold estimate: the largest of
// 128..8 that leaves at least 4k groups (the k-th largest group maximum is
// then a tight threshold), else the smallest that leaves at least k groups,
// at most kMaxGroups groups either way; 0 if none.
__host__ __device__ __forceinline__ int select_group_size(int F, int k) {
    int best = 0;
    for (int gs = 128; gs >= 8; gs >>= 1) {
        const int ng = (F + gs - 1) / gs;
        if (ng > kMaxGroups) break;
        if (ng >= k) best = gs;
        if (ng >= 4 * k) return gs;
    }
    return best;
}

// Eight consecutive query values as floats (16-byte bf16 or 2x16-byte fp32
// loads; query rows are 16-byte aligned).
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&x)[8]) {
    const uint4 r = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(b[j]);
        x[2 * j] = f.x;
        x[2 * j + 1] = f.y;
    }
}
__device__ __forceinline__ void load8(const float* p, float (&x)[8]) {
    const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

// Tensor-core approximation of the query activations with rigorous bounds.
// v[u, g, f] = (q/scale) . W_f + b_f with bf16 operands on mma.sync and fp32
// accumulation (a 64-head x 128-feature tile per CTA, 16 x 64 per warp)
// differs from the exact fp32 activation by at most
//     e_f = 2^-6 |x| |W_f| + 2^-20 |v|
// (bf16 rounding of both operands, 2^-8 relative each, fp32 accumulation and
// the exact order's own rounding, with a 2x margin; |x| is rounded up by
// 2^-12 and |W_f| comes from pk_sae_prepare).  The kernel writes the upper
// bound U = v + e for every feature and, per head, the maximum lower bound
// L = v - e of every group of gs consecutive features (order-preserving
// keys; gs = 0 skips the groups).
template <typename QT>
__global__ void __launch_bounds__(kApxThreads)
qact_approx_kernel(const QT* __restrict__ q, const int* __restrict__ units, int n_units, int G,
                   const __nv_bfloat16* __restrict__ Wb, const float* __restrict__ bias, const float* __restrict__ wn,
                   float query_scale, int F, int gs, int ngroups, float* __restrict__ upper,
                   uint32_t* __restrict__ gmax) {
    extern __shared__ __align__(128) uint8_t apx_smem[];
    __shared__ float sxn[kApxHeads];
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
    // The 64 query rows, 16-byte chunks of 8 values (all loads of a thread
    // issued before any is used), scaled, rounded to bf16, and their norms.
    constexpr int kChunks = kApxHeads * 16 / kApxThreads;
    float xv[kChunks][8];
#pragma unroll
    for (int t = 0; t < kChunks; ++t) {
        const int c = tid + t * kApxThreads, row = c >> 4, ch = c & 15;
        const int h = h0 + row;
        if (h < n_heads) {
            const int ui = h / G, g = h % G;
            const int u = units ? units[ui] : ui;
            load8(q + ((int64_t)u * G + g) * kEncD + ch * 8, xv[t]);
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) xv[t][j] = 0.f;
        }
    }
    // x = q * (1/scale): within a few ulp of the exact quotient, far inside
    // the bound's margins (the norm's 2^-12, the operands' 2^-8).
    const float inv_scale = 1.0f / query_scale;
#pragma unroll
    for (int t = 0; t < kChunks; ++t) {
        const int c = tid + t * kApxThreads, row = c >> 4, ch = c & 15;
        uint4 packed;
        uint32_t* pw = reinterpret_cast<uint32_t*>(&packed);
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float xa = xv[t][2 * j] * inv_scale, xb = xv[t][2 * j + 1] * inv_scale;
            ss = fmaf(xa, xa, fmaf(xb, xb, ss));
            __nv_bfloat162 b2 = __floats2bfloat162_rn(xa, xb);
            pw[j] = *reinterpret_cast<uint32_t*>(&b2);
        }
        *reinterpret_cast<uint4*>(Xs + swz(row, ch)) = packed;
        // The 16 chunks of a row sit in 16 consecutive lanes.
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (ch == 0) sxn[row] = sqrtf(ss) * (1.0f + 1.0f / 4096.0f);
    }
    cp_async_wait_group<0>();
    __syncthreads();

    // Warp w multiplies head rows 16(w&3).. by feature half fh = w>>2
    // (64 features): eight warps keep twice the loads and stores in flight
    // of a 16 x 128 warp tile at the same register count.
    const int rb = warp & 3, fh = warp >> 2;
    float acc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    const int mi = lane >> 3, r = lane & 7;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
        uint32_t a[4];
        ldsm_x4(smem_addr(Xs) + swz(rb * 16 + (mi & 1) * 8 + r, 2 * kk + (mi >> 1)), a);
#pragma unroll
        for (int np = 0; np < 4; ++np) {
            uint32_t b[4];
            ldsm_x4(smem_addr(Wt) + swz(fh * 64 + np * 16 + (mi >> 1) * 8 + r, 2 * kk + (mi & 1)), b);
            mma_16816(acc[2 * np], a, b[0], b[1]);
            mma_16816(acc[2 * np + 1], a, b[2], b[3]);
        }
    }
    // acc[j][2*half + e] is feature fb + 8j + 2(lane&3) + e of local row
    // rb*16 + (lane>>2) + 8*half, fb = f0 + 64 fh.
    const int fb = f0 + fh * 64;
    float bv[8][2], wv[8][2];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int f = fb + 8 * j + 2 * (lane & 3) + e;
            bv[j][e] = f < F ? bias[f] : 0.f;
            wv[j][e] = f < F ? wn[f] : 0.f;
        }
    // 8-feature blocks per group; a group of 128 spans both feature halves
    // and is finished through shared memory below.
    const int per = gs >> 3, g0 = gs ? f0 / gs : 0;
    const bool split = per == 16;
    uint32_t part[2] = {0u, 0u};
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        const int lrow = rb * 16 + (lane >> 2) + half * 8;
        const int h = h0 + lrow;
        const bool hv = h < n_heads;
        int u = 0, g = 0;
        if (hv) {
            const int ui = h / G;
            g = h % G;
            u = units ? units[ui] : ui;
        }
        const float xn = sxn[lrow];
        float* out = upper + ((int64_t)u * G + g) * F;
        uint32_t* gm = gmax + ((int64_t)u * G + g) * ngroups;
        const bool writer = gs && hv && (lane & 3) == 0;
        uint32_t run = 0u;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int f = fb + 8 * j + 2 * (lane & 3);
            float up[2];
            uint32_t lk = 0u;
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const float v = acc[j][2 * half + e] + bv[j][e];
                const float err = 0.015625f * xn * wv[j][e] + 9.5367431640625e-07f * fabsf(v);
                up[e] = v + err;
                if (f + e < F) lk = max(lk, fkey(v - err));
            }
            if (hv) {
                if ((F & 1) == 0 && f + 1 < F) {
                    *reinterpret_cast<float2*>(out + f) = make_float2(up[0], up[1]);
                } else {
                    if (f < F) out[f] = up[0];
                    if (f + 1 < F) out[f + 1] = up[1];
                }
            }
            // At a group's last 8-feature block, reduce over the quad
            // (the four lanes holding the row's features of each block).
            run = max(run, lk);
            if (gs && !split && ((fh * 8 + j + 1) & (per - 1)) == 0) {
                run = max(run, __shfl_xor_sync(0xffffffffu, run, 1));
                run = max(run, __shfl_xor_sync(0xffffffffu, run, 2));
                const int gi = g0 + (fh * 8 + j + 1) / per - 1;
                if (writer && gi < ngroups) gm[gi] = run;
                run = 0u;
            }
        }
        if (split) {
            run = max(run, __shfl_xor_sync(0xffffffffu, run, 1));
            part[half] = max(run, __shfl_xor_sync(0xffffffffu, run, 2));
        }
    }
    if (split) {
        // Half 0 leaves its row maxima in shared memory; half 1 adds its own
        // and writes the group (g0 < ngroups: the tile starts inside F).
        __shared__ uint32_t sgrp[kApxHeads];
        if (fh == 0 && (lane & 3) == 0) {
            sgrp[rb * 16 + (lane >> 2)] = part[0];
            sgrp[rb * 16 + (lane >> 2) + 8] = part[1];
        }
        __syncthreads();
        if (fh == 1 && (lane & 3) == 0) {
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int lrow = rb * 16 + (lane >> 2) + half * 8;
                const int h = h0 + lrow;
                if (h < n_heads) {
                    const int ui = h / G, g = h % G;
                    const int u = units ? units[ui] : ui;
                    gmax[((int64_t)u * G + g) * ngroups + g0] = max(part[half], sgrp[lrow]);
                }
            }
        }
    }
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
constexpr int kSelThreads = 256;
constexpr int kWarpCand = kCandCap / (kSelThreads / 32);   // candidate slots per warp

struct FastSmem {
    QactSmem q;
    float x[kEncD];
    int cand[kCandCap];
    float cval[kCandCap];
    uint32_t gkey[kMaxGroups];
    int wc[32];
    float lam;
    // Cluster form: this head's sorted picks and their live flags, and a
    // copy of every head's of the unit.
    int hid[256];
    float hv[256];
    int hlive[256];
    int all_id[256];
    float all_v[256];
    int all_live[256];
};

// The unit's share of the routing once a head's m positive picks are in
// sm.q (sel / selkey in rank order): kCluster -- the G head CTAs of the unit
// form a cluster, each copies every head's picks from the others' shared
// memory, computes all entries' scores (the arithmetic of the single-CTA
// aggregation) and ranks and writes the order slots of its own head's
// entries; otherwise the picks go through global memory and the unit's last
// CTA to arrive builds the whole order (head_finish).  Every thread calls it.
template <bool kCluster>
__device__ void qact_unit_tail(int u, int g, int G, int F, int k, int m, FastSmem& sm, uint32_t* sA,
                               const int* __restrict__ counts, int* __restrict__ head_ids,
                               float* __restrict__ head_val, int* __restrict__ unit_done, int* __restrict__ order,
                               int* __restrict__ n_order, int order_stride, float* __restrict__ score) {
    const int tid = threadIdx.x, nt = blockDim.x;
    if constexpr (kCluster) {
        namespace cg = cooperative_groups;
        cg::cluster_group cluster = cg::this_cluster();
        head_picks(G, k, m, sm.q, sm.hid, sm.hv);
        __syncthreads();
        for (int r = tid; r < k; r += nt) {
            const int f = sm.hid[r];
            sm.hlive[r] = f != INT32_MAX && counts[(int64_t)u * F + f] > 0;
        }
        cluster.sync();   // every head's picks are in its CTA's shared memory
        const int E = G * k;
        for (int e = tid; e < E; e += nt) {
            const int h = e / k, r = e - h * k;
            sm.all_id[e] = cluster.map_shared_rank(sm.hid, h)[r];
            sm.all_v[e] = cluster.map_shared_rank(sm.hv, h)[r];
            sm.all_live[e] = cluster.map_shared_rank(sm.hlive, h)[r];
        }
        cluster.sync();   // no CTA exits while another still reads its picks
        float* sc = reinterpret_cast<float*>(sA);
        int* cand = reinterpret_cast<int*>(sA) + E;
        unit_scores(u, G, F, k, sm.all_id, sm.all_v, sm.all_live, counts, sc, cand, g * k, (g + 1) * k, score);
        const int tot = unit_rank(u, E, sc, cand, g * k, (g + 1) * k, sm.q.tk.scan, order, order_stride);
        if (g == 0 && tid == 0) n_order[u] = tot;
    } else {
        head_finish(u, g, G, F, k, m, sm.q, sA, counts, head_ids, head_val, unit_done, order, n_order, order_stride,
                    score);
    }
}

// Per (unit, head), the exact top-k of the activations from the bounds of
// qact_approx_kernel (L_f <= exact_f <= U_f):
//   lambda' = the k-th largest of the per-group maxima of L.  At least k
//             features have L >= lambda', so lambda' <= the k-th largest L
//             <= the k-th largest exact activation.
//   candidates = features with U >= lambda' (and U > 0): every feature whose
//             exact value reaches the k-th largest -- ties included -- is a
//             candidate, so the exact top-k among them (stable descending,
//             ties -> lower feature id, core.py:134) is the exact top-k.
// Candidates get exact fp32 activations in the reference's dot-product
// order.  Too many candidates (near-degenerate inputs): every feature is
// recomputed.
// MINB = 2 when there are more heads than SMs: two CTAs per SM (at most 128
// registers a thread) instead of a second wave.
// kCluster: the G head CTAs of a unit form a thread-block cluster (G <= 8);
// each copies every head's picks from the others' shared memory, computes
// all entries' scores (the same arithmetic as the single-CTA aggregation)
// and ranks and writes the order slots of its own head's entries.
// Otherwise the picks go through global memory and the unit's last CTA to
// arrive builds the whole order.
template <int ORDER, typename QT, int MINB, bool kCluster>
__global__ void __launch_bounds__(kSelThreads, MINB)
qact_select_fast_kernel(const QT* __restrict__ q, const float* __restrict__ upper,
                        const uint32_t* __restrict__ gmax, int ngroups, const int* __restrict__ units, int G,
                        const float* __restrict__ W, const float* __restrict__ bias, float query_scale, int F, int k,
                        const int* __restrict__ counts, int* __restrict__ head_ids, float* __restrict__ head_val,
                        int* __restrict__ unit_done, int* __restrict__ order, int* __restrict__ n_order,
                        int order_stride, float* __restrict__ score, int f_base, int* __restrict__ picks) {
    // sA[F]: exact values when every feature is recomputed; head_finish's
    // aggregation scratch.
    extern __shared__ __align__(16) uint32_t sA[];
    __shared__ FastSmem sm;
    const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
    const int ui = blockIdx.x / G, g = blockIdx.x % G;
    const int u = units ? units[ui] : ui;
    const float* up = upper + ((int64_t)u * G + g) * F;
    const uint32_t* gk = gmax + ((int64_t)u * G + g) * ngroups;
    for (int i = tid; i < ngroups; i += nt) sm.gkey[i] = gk[i];
    for (int c = tid; c < kEncD; c += nt) sm.x[c] = __fdiv_rn(load_f(q, ((int64_t)u * G + g) * kEncD + c), query_scale);
    if (tid == 0) sm.lam = -INFINITY;
    __syncthreads();
    // lambda' = k-th largest group maximum (rank by value, then group index);
    // no groups (too few features): -inf, every positive U is a candidate.
    for (int i = tid; i < ngroups; i += nt) {
        const uint32_t ki = sm.gkey[i];
        int r = 0;
        for (int j = 0; j < ngroups; ++j) {
            const uint32_t kj = sm.gkey[j];
            r += (kj > ki) || (kj == ki && j < i);
        }
        if (r == k - 1) sm.lam = fkey_inv(ki);
    }
    __syncthreads();
    const float lam = sm.lam;
    const bool pos_only = !(lam > 0.f);
    auto is_cand = [&](float u_) { return pos_only ? u_ > 0.f : u_ >= lam; };

    // One pass over U: each warp owns a contiguous segment (a multiple of
    // 128 features) and appends its candidates, in feature order, to its own
    // slots; 16-byte loads, sixteen per lane in flight, when rows are aligned.
    const bool vec = (F & 3) == 0 && (reinterpret_cast<uintptr_t>(up) & 15) == 0;
    const int seg = ((F + nw - 1) / nw + 127) / 128 * 128;
    const int s0 = min(F, warp * seg), s1 = min(F, s0 + seg);
    int* wslot = sm.cand + warp * kWarpCand;
    int mine = 0;
    // Slots in feature order (lane-major, then the lane's four features):
    // the candidates before this lane come from four ballots, no scan.
    const unsigned lt_mask = (1u << lane) - 1u;
    auto take = [&](int base, const float (&v)[4]) {
        unsigned m = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c)
            if (base + 4 * lane + c < s1 && is_cand(v[c])) m |= 1u << c;
        unsigned b[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) b[c] = __ballot_sync(0xffffffffu, (m >> c) & 1u);
        const unsigned any = b[0] | b[1] | b[2] | b[3];
        if (any) {
            int at = mine + __popc(b[0] & lt_mask) + __popc(b[1] & lt_mask) + __popc(b[2] & lt_mask) +
                     __popc(b[3] & lt_mask);
#pragma unroll
            for (int c = 0; c < 4; ++c)
                if (m & (1u << c)) {
                    if (at < kWarpCand) wslot[at] = base + 4 * lane + c;
                    ++at;
                }
            mine += __popc(b[0]) + __popc(b[1]) + __popc(b[2]) + __popc(b[3]);
        }
    };
    if (vec) {
        constexpr int kBatch = 16;  // 16-byte loads in flight per lane
        for (int b0 = s0; b0 < s1; b0 += 128 * kBatch) {
            float4 va[kBatch];
#pragma unroll
            for (int t = 0; t < kBatch; ++t) {
                const int i = b0 + 128 * t + 4 * lane;
                va[t] = i < s1 ? *reinterpret_cast<const float4*>(up + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int t = 0; t < kBatch; ++t) {
                if (b0 + 128 * t >= s1) break;
                const float v[4] = {va[t].x, va[t].y, va[t].z, va[t].w};
                take(b0 + 128 * t, v);
            }
        }
    } else {
        for (int b = s0; b < s1; b += 128) {
            float v[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int i = b + 4 * lane + c;
                v[c] = i < s1 ? up[i] : 0.f;
            }
            take(b, v);
        }
    }
    if (lane == 0) sm.wc[warp] = mine;
    __syncthreads();
    int total = 0;
    bool all_exact = false;
    for (int w = 0; w < nw; ++w) {
        total += sm.wc[w];
        all_exact |= sm.wc[w] > kWarpCand;
    }
    if (!all_exact) {
        // Compact the per-warp slots into feature order.
        constexpr int kPer = kCandCap / kSelThreads;
        int vals[kPer];
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            const int p = tid + i * nt;
            vals[i] = -1;
            if (p < total) {
                int w = 0, before = 0;
                while (before + sm.wc[w] <= p) { before += sm.wc[w]; ++w; }
                vals[i] = sm.cand[w * kWarpCand + (p - before)];
            }
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            const int p = tid + i * nt;
            if (p < total) sm.cand[p] = vals[i];
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
        if (total <= 512) {
            // Exact rank among the candidates: (value desc, feature asc),
            // positive values only; the candidates are in feature order.
            int npos = 0;
            for (int c = tid; c < total; c += nt) npos += sm.cval[c] > 0.f;
            npos = warp_sum(npos);
            if (lane == 0) sm.wc[warp] = npos;
            __syncthreads();
            int all_pos = 0;
            for (int w = 0; w < nw; ++w) all_pos += sm.wc[w];
            m = min(k, all_pos);
            for (int c = tid; c < total; c += nt) {
                const float vc = sm.cval[c];
                if (!(vc > 0.f)) continue;
                int r = 0;
                for (int j = 0; j < total; ++j) {
                    const float vj = sm.cval[j];
                    r += (vj > vc) || (vj == vc && j < c);
                }
                if (r < m) { sm.q.sel[r] = sm.cand[c]; sm.q.selkey[r] = __float_as_uint(vc); }
            }
            __syncthreads();
        } else {
            m = block_topk(
                total, k, [&](int i) { return __float_as_uint(sm.cval[i]); },
                [&](int i) { return sm.cval[i] > 0.f; }, sm.q.sel, sm.q.selkey, sm.q.tk);
            for (int r = tid; r < m; r += nt) sm.q.sel[r] = sm.cand[sm.q.sel[r]];
        }
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
    if constexpr (!kCluster) {
        if (picks) {
            // Feature-sharded routing: this shard's picks of the head, in rank
            // order, as (value bits, feature id); unused slots (0, INT32_MAX).
            int* hp = picks + ((int64_t)u * G + g) * k * 2;
            for (int r = tid; r < k; r += nt) {
                hp[2 * r] = r < m ? (int)sm.q.selkey[r] : 0;
                hp[2 * r + 1] = r < m ? sm.q.sel[r] + f_base : INT32_MAX;
            }
            return;
        }
    }
    qact_unit_tail<kCluster>(u, g, G, F, k, m, sm, sA, counts, head_ids, head_val, unit_done, order, n_order,
                             order_stride, score);
}

__global__ void zero_rows_kernel(float* __restrict__ score, const int* __restrict__ units, int F) {
    const int u = units ? units[blockIdx.x] : blockIdx.x;
    for (int i = threadIdx.x; i < F; i += blockDim.x) score[(int64_t)u * F + i] = 0.f;
}

// Feature-sharded routing, second half.  picks[P][U*G][k] holds, per shard
// and head, the shard's positive top-k as (value bits, feature id) in rank
// order (pk_route_qact_shard), the shards covering disjoint feature ranges.
// Each shard's list holds every feature of its range that can reach the
// head's top-k, so the exact rank (value desc, feature asc, core.py:134) of
// the positive entries over all lists is the unsharded ranking; the first k
// are the head's picks.  The unit's normalisation, aggregation and order
// then follow as in the unsharded route (qact_unit_tail).  One CTA per
// (unit, head); P * k <= kCandCap.
template <bool kCluster>
__global__ void __launch_bounds__(kSelThreads)
qact_merge_kernel(const int* __restrict__ picks, int P, int G, int F, int k, const int* __restrict__ counts,
                  int* __restrict__ head_ids, float* __restrict__ head_val, int* __restrict__ unit_done,
                  int* __restrict__ order, int* __restrict__ n_order, int order_stride, float* __restrict__ score) {
    extern __shared__ __align__(16) uint32_t sA[];   // the tail's aggregation scratch
    __shared__ FastSmem sm;
    const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
    const int u = blockIdx.x / G, g = blockIdx.x % G;
    const int64_t n_heads = gridDim.x;
    const int n = P * k;
    for (int c = tid; c < n; c += nt) {
        const int r = c / k, j = c - r * k;
        const int* e = picks + (((int64_t)r * n_heads + blockIdx.x) * k + j) * 2;
        sm.cval[c] = __uint_as_float((uint32_t)__ldg(e));
        sm.cand[c] = __ldg(e + 1);
    }
    __syncthreads();
    // An entry counts if its value is positive and its feature id lies in
    // [0, F).  Each shard's list is in rank order (value descending,
    // feature ascending) with its counting entries first, so an entry's rank
    // over all lists is its position plus, per other list, a binary search
    // for the entries ahead of it.  Lists that break that form -- only a
    // malformed input can -- take the quadratic rank instead, whose order
    // (value, feature, then entry) keeps the ranks of any input distinct, so
    // the kernel's memory accesses never depend on a malformed input.
    __shared__ int list_len[kCandCap / 8];   // counting entries per list (k >= 8)
    __shared__ int malformed;
    if (tid == 0) malformed = 0;
    for (int r = tid; r < P; r += nt) list_len[r] = k;
    __syncthreads();
    auto counts_ = [&](int c) {
        const int fc = sm.cand[c];
        return sm.cval[c] > 0.f && fc >= 0 && fc < F;
    };
    for (int c = tid; c < n; c += nt) {
        const int r = c / k, j = c - r * k;
        const bool ok = counts_(c);
        if (!ok) atomicMin(&list_len[r], j);
        if (j + 1 < k) {
            const bool okn = counts_(c + 1);
            const float v = sm.cval[c], vn = sm.cval[c + 1];
            const int f = sm.cand[c], fn = sm.cand[c + 1];
            if (okn && (!ok || !(v > vn || (v == vn && f < fn)))) malformed = 1;
        }
    }
    __syncthreads();
    int m;
    if (!malformed) {
        int all_pos = 0;
        for (int r = 0; r < P; ++r) all_pos += list_len[r];
        m = min(k, all_pos);
        for (int c = tid; c < n; c += nt) {
            const int r = c / k, j = c - r * k;
            if (j >= list_len[r]) continue;
            const float v = sm.cval[c];
            const int f = sm.cand[c];
            int rank = j;
            for (int r2 = 0; r2 < P && rank < m; ++r2) {
                if (r2 == r) continue;
                const float* lv = sm.cval + r2 * k;
                const int* lf = sm.cand + r2 * k;
                int lo = 0, hi = list_len[r2];
                while (lo < hi) {
                    const int mid = (lo + hi) >> 1;
                    const float ve = lv[mid];
                    const int fe = lf[mid];
                    if (ve > v || (ve == v && (fe < f || (fe == f && r2 < r)))) lo = mid + 1;
                    else hi = mid;
                }
                rank += lo;
            }
            if (rank < m) { sm.q.sel[rank] = f; sm.q.selkey[rank] = __float_as_uint(v); }
        }
    } else {
        int npos = 0;
        for (int c = tid; c < n; c += nt) {
            const bool ok = counts_(c);
            npos += ok ? 1 : 0;
        }
        __syncthreads();
        for (int c = tid; c < n; c += nt)
            if (!counts_(c)) sm.cval[c] = 0.f;
        npos = warp_sum(npos);
        if (lane == 0) sm.wc[warp] = npos;
        __syncthreads();
        int all_pos = 0;
        for (int w = 0; w < nw; ++w) all_pos += sm.wc[w];
        m = min(k, all_pos);
        for (int c = tid; c < n; c += nt) {
            const float vc = sm.cval[c];
            if (!(vc > 0.f)) continue;
            const int fc = sm.cand[c];
            int r = 0;
            for (int j = 0; j < n; ++j) {
                const float vj = sm.cval[j];
                const int fj = sm.cand[j];
                r += (vj > vc) || (vj == vc && (fj < fc || (fj == fc && j < c)));
            }
            if (r < m) { sm.q.sel[r] = fc; sm.q.selkey[r] = __float_as_uint(vc); }
        }
    }
    __syncthreads();
    qact_unit_tail<kCluster>(u, g, G, F, k, m, sm, sA, counts, head_ids, head_val, unit_done, order, n_order,
                             order_stride, score);
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

// Workspace: activations or upper bounds [U*G, F] fp32, the heads' picks,
// the per-unit arrival counters, the group maxima [U*G, ngroups].
static size_t route_groups(int F, int k) {
    if (k > F) k = F;
    const int gs = select_group_size(F, k);
    return gs ? (size_t)(F + gs - 1) / gs : 0;
}

extern "C" size_t pk_route_qact_workspace_bytes(int U, int G, int F, int k) {
    const size_t act = (size_t)U * G * F * sizeof(float);
    const size_t heads = (size_t)U * G * k * (sizeof(int) + sizeof(float));
    const size_t done = (size_t)U * sizeof(int);
    const size_t groups = (size_t)U * G * route_groups(F, k) * sizeof(uint32_t);
    return (act + 255) / 256 * 256 + (heads + 255) / 256 * 256 + (done + 255) / 256 * 256 +
           (groups + 255) / 256 * 256;
}

extern "C" int pk_sae_prepare(uint64_t w_enc, int F, int d, uint64_t w_bf16, uint64_t w_norm, uint64_t stream) {
    if (F < 1 || !w_enc || !w_bf16 || !w_norm) return PK_ERR_ARG;
    if (d != kEncD) return PK_ERR_UNSUPPORTED;
    sae_prepare_kernel<<<(F + 7) / 8, 256, 0, (cudaStream_t)stream>>>((const float*)w_enc, F, (__nv_bfloat16*)w_bf16,
                                                                      (float*)w_norm);
    PK_CHECK_LAUNCH();
    return PK_OK;
}

// W_enc rounded to fp16 (round to nearest) for the build's tensor-core bounds.
__global__ void sae_half_kernel(const float* __restrict__ W, int64_t n, __half* __restrict__ Wh) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        Wh[i] = __float2half_rn(W[i]);
}

extern "C" int pk_sae_prepare_half(uint64_t w_enc, int F, int d, uint64_t w_half, uint64_t stream) {
    if (F < 1 || !w_enc || !w_half) return PK_ERR_ARG;
    if (d != kEncD) return PK_ERR_UNSUPPORTED;
    const int64_t n = (int64_t)F * d;
    sae_half_kernel<<<(unsigned)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096), 256, 0, (cudaStream_t)stream>>>(
        (const float*)w_enc, n, (__half*)w_half);
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
    off += ((size_t)U * sizeof(int) + 255) / 256 * 256;
    uint32_t* gmax = (uint32_t*)(ws + off);
    const int gs = select_group_size(F, k);
    const int ngroups = (int)route_groups(F, k);
    const int* ul = (const int*)units;

    // The order F.linear takes for a [G, d] block (see file header).
    const bool inter = G >= 2 && G <= 5;
    if (w_bf16 && w_norm && !topk) {
        // Bound-filtered path: approximate encode on the tensor cores, exact
        // recomputation of the features that can reach the top-k.
        if (q_dtype != PK_BF16 && q_dtype != PK_F32) return PK_ERR_ARG;
        if (q % 16 || w_bf16 % 16) return PK_ERR_ARG;   // 16-byte row loads
        dim3 ag((F + kApxFeat - 1) / kApxFeat, (n_units * G + kApxHeads - 1) / kApxHeads);
        const int asmem = (kApxHeads + kApxFeat) * 256;
        if (q_dtype == PK_BF16) {
            cudaFuncSetAttribute(qact_approx_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, asmem);
            qact_approx_kernel<__nv_bfloat16><<<ag, kApxThreads, asmem, st>>>(
                (const __nv_bfloat16*)q, ul, n_units, G, (const __nv_bfloat16*)w_bf16, (const float*)b_enc,
                (const float*)w_norm, query_scale, F, gs, ngroups, act, gmax);
        } else {
            cudaFuncSetAttribute(qact_approx_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, asmem);
            qact_approx_kernel<float><<<ag, kApxThreads, asmem, st>>>(
                (const float*)q, ul, n_units, G, (const __nv_bfloat16*)w_bf16, (const float*)b_enc,
                (const float*)w_norm, query_scale, F, gs, ngroups, act, gmax);
        }
        PK_CHECK_LAUNCH();
        if (score) {
            zero_rows_kernel<<<n_units, 256, 0, st>>>((float*)score, ul, F);
            PK_CHECK_LAUNCH();
        }
        // Shared memory for the all-features fallback and the aggregation.
        size_t fsmem = (size_t)4 * F;
        if ((size_t)16 * G * k > fsmem) fsmem = (size_t)16 * G * k;
        int dev = 0, sms = 148;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        const bool wide = n_units * G > sms;
        // The G head CTAs of a unit as one cluster (G <= 8, portable sizes).
        const bool clustered = G <= 8;
#define PK_LAUNCH_FAST1(ORD, QT, MINB)                                                                           \
    do {                                                                                                         \
        if (clustered) {                                                                                         \
            auto fn = qact_select_fast_kernel<ORD, QT, MINB, true>;                                              \
            cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fsmem);                   \
            cudaLaunchConfig_t cfg = {};                                                                         \
            cfg.gridDim = dim3(n_units * G);                                                                     \
            cfg.blockDim = dim3(kSelThreads);                                                                    \
            cfg.dynamicSmemBytes = fsmem;                                                                        \
            cfg.stream = st;                                                                                     \
            cudaLaunchAttribute attr[1];                                                                         \
            attr[0].id = cudaLaunchAttributeClusterDimension;                                                    \
            attr[0].val.clusterDim.x = G;                                                                        \
            attr[0].val.clusterDim.y = 1;                                                                        \
            attr[0].val.clusterDim.z = 1;                                                                        \
            cfg.attrs = attr;                                                                                    \
            cfg.numAttrs = 1;                                                                                    \
            const cudaError_t e_ = cudaLaunchKernelEx(                                                           \
                &cfg, fn, (const QT*)q, (const float*)act, (const uint32_t*)gmax, ngroups, ul, G,                \
                (const float*)w_enc, (const float*)b_enc, query_scale, F, k, (const int*)counts, hid, hval,      \
                done, (int*)order, (int*)n_order, order_stride, (float*)score, 0, (int*)nullptr);                \
            if (e_ != cudaSuccess) return (int)e_;                                                               \
        } else {                                                                                                 \
            auto fn = qact_select_fast_kernel<ORD, QT, MINB, false>;                                             \
            cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fsmem);                   \
            fn<<<n_units * G, kSelThreads, fsmem, st>>>(                                                         \
                (const QT*)q, act, gmax, ngroups, ul, G, (const float*)w_enc, (const float*)b_enc, query_scale,  \
                F, k, (const int*)counts, hid, hval, done, (int*)order, (int*)n_order, order_stride,             \
                (float*)score, 0, (int*)nullptr);                                                                \
        }                                                                                                        \
    } while (0)
#define PK_LAUNCH_FAST(ORD, QT)                                                                                  \
    do {                                                                                                         \
        if (wide) PK_LAUNCH_FAST1(ORD, QT, 2); else PK_LAUNCH_FAST1(ORD, QT, 1);                                 \
    } while (0)
        if (q_dtype == PK_BF16) {
            if (inter) PK_LAUNCH_FAST(kInterleaved16, __nv_bfloat16); else PK_LAUNCH_FAST(kSequential, __nv_bfloat16);
        } else {
            if (inter) PK_LAUNCH_FAST(kInterleaved16, float); else PK_LAUNCH_FAST(kSequential, float);
        }
#undef PK_LAUNCH_FAST
#undef PK_LAUNCH_FAST1
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

// ---------------------------------------------------------------------------
// Feature-sharded q_activation routing: each of P ranks encodes the features
// [f_lo, f_hi) of every head and exports its picks; after an all-gather of
// the picks every rank merges them into the same order.
// ---------------------------------------------------------------------------

extern "C" size_t pk_route_qact_shard_workspace_bytes(int U, int G, int F_local, int k) {
    if (U < 1 || G < 1 || F_local < 1 || k < 1) return 0;
    const size_t act = (size_t)U * G * F_local * sizeof(float);
    const size_t groups = (size_t)U * G * route_groups(F_local, k) * sizeof(uint32_t);
    return (act + 255) / 256 * 256 + (groups + 255) / 256 * 256;
}

extern "C" int pk_route_qact_shard(uint64_t q, int q_dtype, uint64_t w_enc, uint64_t b_enc, uint64_t w_bf16,
                                   uint64_t w_norm, float query_scale, int U, int G, int d, int F, int k, int f_lo,
                                   int f_hi, uint64_t workspace, uint64_t workspace_bytes, uint64_t picks,
                                   uint64_t stream) {
    if (U < 1 || G < 1 || F < 1 || k < 1 || k > 256 || !(query_scale > 0.f)) return PK_ERR_ARG;
    if (f_lo < 0 || f_hi <= f_lo || f_hi > F) return PK_ERR_ARG;
    if (d != kEncD) return PK_ERR_UNSUPPORTED;
    const int Fl = f_hi - f_lo;
    if ((size_t)Fl * sizeof(uint32_t) > 200 * 1024) return PK_ERR_UNSUPPORTED;
    if (workspace_bytes < pk_route_qact_shard_workspace_bytes(U, G, Fl, k)) return PK_ERR_WORKSPACE;
    if (!q || !w_enc || !b_enc || !w_bf16 || !w_norm || !workspace || !picks) return PK_ERR_ARG;
    if (q_dtype != PK_BF16 && q_dtype != PK_F32) return PK_ERR_ARG;
    if (q % 16 || w_bf16 % 16) return PK_ERR_ARG;   // 16-byte row loads
    cudaStream_t st = (cudaStream_t)stream;
    char* ws = (char*)workspace;
    float* act = (float*)ws;
    uint32_t* gmax = (uint32_t*)(ws + ((size_t)U * G * Fl * sizeof(float) + 255) / 256 * 256);
    const int kl = k < Fl ? k : Fl;
    const int gs = select_group_size(Fl, kl);
    const int ngroups = (int)route_groups(Fl, k);
    // This shard's rows of the SAE (rows are 256 and 512 bytes: the offsets
    // keep the 16-byte alignment of the row loads).
    const __nv_bfloat16* wb = (const __nv_bfloat16*)w_bf16 + (int64_t)f_lo * kEncD;
    const float* wf = (const float*)w_enc + (int64_t)f_lo * kEncD;
    const float* bl = (const float*)b_enc + f_lo;
    const float* wn = (const float*)w_norm + f_lo;
    dim3 ag((Fl + kApxFeat - 1) / kApxFeat, (U * G + kApxHeads - 1) / kApxHeads);
    const int asmem = (kApxHeads + kApxFeat) * 256;
    if (q_dtype == PK_BF16) {
        cudaFuncSetAttribute(qact_approx_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, asmem);
        qact_approx_kernel<__nv_bfloat16><<<ag, kApxThreads, asmem, st>>>(
            (const __nv_bfloat16*)q, nullptr, U, G, wb, bl, wn, query_scale, Fl, gs, ngroups, act, gmax);
    } else {
        cudaFuncSetAttribute(qact_approx_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, asmem);
        qact_approx_kernel<float><<<ag, kApxThreads, asmem, st>>>(
            (const float*)q, nullptr, U, G, wb, bl, wn, query_scale, Fl, gs, ngroups, act, gmax);
    }
    PK_CHECK_LAUNCH();
    const size_t fsmem = (size_t)4 * Fl;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const bool wide = U * G > sms;
    const bool inter = G >= 2 && G <= 5;   // the order F.linear takes for a [G, d] block
#define PK_LAUNCH_SHARD(ORD, QT, MINB)                                                                           \
    do {                                                                                                         \
        auto fn = qact_select_fast_kernel<ORD, QT, MINB, false>;                                                 \
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fsmem);                       \
        fn<<<U * G, kSelThreads, fsmem, st>>>((const QT*)q, act, gmax, ngroups, nullptr, G, wf, bl, query_scale, \
                                               Fl, k, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, 0,   \
                                               nullptr, f_lo, (int*)picks);                                     \
    } while (0)
#define PK_LAUNCH_SHARD2(ORD, QT)                                                                                \
    do {                                                                                                         \
        if (wide) PK_LAUNCH_SHARD(ORD, QT, 2); else PK_LAUNCH_SHARD(ORD, QT, 1);                                 \
    } while (0)
    if (q_dtype == PK_BF16) {
        if (inter) PK_LAUNCH_SHARD2(kInterleaved16, __nv_bfloat16); else PK_LAUNCH_SHARD2(kSequential, __nv_bfloat16);
    } else {
        if (inter) PK_LAUNCH_SHARD2(kInterleaved16, float); else PK_LAUNCH_SHARD2(kSequential, float);
    }
#undef PK_LAUNCH_SHARD2
#undef PK_LAUNCH_SHARD
    PK_CHECK_LAUNCH();
    return PK_OK;
}

extern "C" size_t pk_route_qact_merge_workspace_bytes(int U, int G, int k) {
    if (U < 1 || G < 1 || k < 1) return 0;
    const size_t heads = (size_t)U * G * k * (sizeof(int) + sizeof(float));
    const size_t done = (size_t)U * sizeof(int);
    return (heads + 255) / 256 * 256 + (done + 255) / 256 * 256;
}

extern "C" int pk_route_qact_merge(uint64_t picks, int P, uint64_t counts, int U, int G, int F, int k,
                                   uint64_t workspace, uint64_t workspace_bytes, uint64_t order, uint64_t n_order,
                                   int order_stride, uint64_t score, uint64_t stream) {
    if (P < 1 || U < 1 || G < 1 || F < 1 || k < 1) return PK_ERR_ARG;
    if (G * k > 256 || order_stride < G * k || P * k > kCandCap || P > kCandCap / 8) return PK_ERR_ARG;
    if (workspace_bytes < pk_route_qact_merge_workspace_bytes(U, G, k)) return PK_ERR_WORKSPACE;
    if (!picks || !counts || !workspace || !order || !n_order) return PK_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    char* ws = (char*)workspace;
    int* hid = (int*)ws;
    float* hval = (float*)(hid + (size_t)U * G * k);
    int* done = (int*)(ws + ((size_t)U * G * k * (sizeof(int) + sizeof(float)) + 255) / 256 * 256);
    if (score) {
        zero_rows_kernel<<<U, 256, 0, st>>>((float*)score, nullptr, F);
        PK_CHECK_LAUNCH();
    }
    const size_t msmem = (size_t)16 * G * k;   // the tail's aggregation scratch
    if (G <= 8) {
        // The G head CTAs of a unit as one cluster (portable sizes).
        auto fn = qact_merge_kernel<true>;
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)msmem);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(U * G);
        cfg.blockDim = dim3(kSelThreads);
        cfg.dynamicSmemBytes = msmem;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = G;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        const cudaError_t e = cudaLaunchKernelEx(&cfg, fn, (const int*)picks, P, G, F, k, (const int*)counts, hid,
                                                 hval, done, (int*)order, (int*)n_order, order_stride, (float*)score);
        if (e != cudaSuccess) return (int)e;
    } else {
        auto fn = qact_merge_kernel<false>;
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)msmem);
        fn<<<U * G, kSelThreads, msmem, st>>>((const int*)picks, P, G, F, k, (const int*)counts, hid, hval, done,
                                               (int*)order, (int*)n_order, order_stride, (float*)score);
    }
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
