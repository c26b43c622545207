// Key-side index build and append: src/prismkv/core.py:92-103 (build_index),
// :13-26 (positive_global_topk), :76-89 (summarize), :186-201 (append_index).
//
// The encode a[t, f] = relu(((k_t - c) / s) . W_f + b_f) is recomputed in two
// passes and never stored: pass 1 builds a 2048-bin histogram of the positive
// activations' float bits (>> 20) per unit, which fixes the coarse bin that
// holds the budget's threshold; pass 2 emits every activation above that bin
// as a member and every activation inside it to a boundary buffer as a
// 64-bit key (value descending, flat index ascending).  An exact radix
// select over the boundary keys then takes the remaining members, which is
// the reference's rule: all activations above the count-th largest value,
// then ties at that value by ascending flat index, positives only.  The dot
// products run as one sequential FMA chain over d, the order the reference's
// F.linear takes for a many-row block, so memberships are bit-identical.
#include <cstring>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "mma.cuh"
#include "tc.cuh"

namespace pk {

constexpr int kBD = 128;            // head dim compiled for the build
constexpr int kBT = 128;             // tokens per CTA tile
constexpr int kBF = 128;             // features per CTA tile
constexpr int kBThreads = 256;       // 16 x 16 threads, 8 x 8 outputs each
constexpr int kBPitch = kBT + 4;     // smem pitch (floats) of the k-major tiles
constexpr int kHistBins = 2048;
constexpr int kSortWarpCap = 1024;   // ids a warp sorts in shared memory
constexpr int kSortBigCap = 32768;   // ids one CTA sorts (larger: error)

struct BuildWs {
    int* hist;          // [U, 2048]
    int* cut;           // [U]
    long long* need;    // [U]
    int* n_members;     // [U]
    int* n_boundary;    // [U]
    int* fill;          // [U, F]
    int* flag;          // [4]
    long long* members; // [U, mcap]
    long long* boundary;// [U, bcap]
    int64_t mcap, bcap;
};

template <typename T>
__device__ __forceinline__ float key_at(const T* keys, int64_t unit_stride, int64_t row_stride, int u, int64_t t,
                                        int c) {
    return load_f(keys, (int64_t)u * unit_stride + t * row_stride + c);
}

// center[u, c] = torch-order column mean of the unit's N rows.  The cascade
// of torch_cascade_sum (blocks of 2^lp rows, 4 levels) splits into chunks of
// 2^(3 lp) rows that each add one independent sum to the top accumulator:
// the chunks' sums run in parallel (warp w of the CTA takes chunks w, w+nw,
// ...; lane = column), then lane 0..31 of warp 0 adds them in chunk order
// and runs the cascade over the remaining rows.  Same arithmetic, same order.
template <typename T>
__global__ void __launch_bounds__(1024)
center_kernel(const T* __restrict__ keys, int64_t unit_stride, int64_t row_stride, int64_t N, int d,
              float* __restrict__ center) {
    extern __shared__ float part[];   // [nchunks][32]
    const int u = blockIdx.y, lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int c = blockIdx.x * 32 + lane;
    int lp = ceil_log2_i64(N) / 4;
    if (lp < 4) lp = 4;
    const int64_t step = (int64_t)1 << lp, chunk = step * step * step, mask = step - 1;
    const int64_t nchunks = N / chunk;
    auto get = [&](int64_t i) { return key_at(keys, unit_stride, row_stride, u, i, c); };
    if (c < d) {
        for (int64_t ch = w; ch < nchunks; ch += nw) {
            int64_t i = ch * chunk;
            float a2 = 0.f;
            for (int64_t g = 0; g < step; ++g) {
                float a1 = 0.f;
                for (int64_t b = 0; b < step; ++b) {
                    float a0 = 0.f;
                    for (int64_t s = 0; s < step; ++s, ++i) a0 = __fadd_rn(a0, get(i));
                    a1 = __fadd_rn(a1, a0);
                }
                a2 = __fadd_rn(a2, a1);
            }
            part[ch * 32 + lane] = a2;
        }
    }
    __syncthreads();
    if (w != 0 || c >= d) return;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int64_t ch = 0; ch < nchunks; ++ch) acc[3] = __fadd_rn(acc[3], part[ch * 32 + lane]);
    int64_t i = nchunks * chunk;
    while (i + step <= N) {
        for (int64_t s = 0; s < step; ++s, ++i) acc[0] = __fadd_rn(acc[0], get(i));
        for (int j = 1; j < 4; ++j) {
            acc[j] = __fadd_rn(acc[j], acc[j - 1]);
            acc[j - 1] = 0.f;
            if ((i & (mask << (j * lp))) != 0) break;
        }
    }
    for (; i < N; ++i) acc[0] = __fadd_rn(acc[0], get(i));
    for (int j = 1; j < 4; ++j) acc[0] = __fadd_rn(acc[0], acc[j]);
    center[(int64_t)u * d + c] = __fdiv_rn(acc[0], (float)N);
}

// One tile of 128 tokens x 128 features.  PASS 1: histogram; PASS 2: emit.
template <int PASS, typename T>
__global__ void __launch_bounds__(kBThreads)
build_encode_kernel(const T* __restrict__ keys, int64_t unit_stride, int64_t row_stride, int64_t N,
                    const float* __restrict__ center, float key_scale, const float* __restrict__ W,
                    const float* __restrict__ bias, int F, BuildWs ws, int* __restrict__ lens,
                    int* __restrict__ status) {
    extern __shared__ __align__(16) float sm[];
    float* Xs = sm;                       // [kBD][kBPitch]  x^T
    float* Ws = sm + kBD * kBPitch;       // [kBD][kBPitch]  W^T
    int* hist = reinterpret_cast<int*>(Ws + kBD * kBPitch);  // [2048] (pass 1)
    const int tid = threadIdx.x;
    const int f0 = blockIdx.x * kBF;
    const int64_t t0 = (int64_t)blockIdx.y * kBT;
    const int u = blockIdx.z;
    const float* cu = center + (int64_t)u * kBD;

    if (PASS == 1)
        for (int i = tid; i < kHistBins; i += kBThreads) hist[i] = 0;
    // x = (k - center) / key_scale (core.py:99), transposed into Xs.
    for (int e = tid; e < kBT * kBD; e += kBThreads) {
        const int tt = e / kBD, c = e % kBD;
        const int64_t t = t0 + tt;
        float x = 0.f;
        if (t < N) x = __fdiv_rn(__fsub_rn(key_at(keys, unit_stride, row_stride, u, t, c), cu[c]), key_scale);
        Xs[c * kBPitch + tt] = x;
    }
    for (int e = tid; e < kBF * kBD / 4; e += kBThreads) {
        const int ff = e / (kBD / 4), c4 = e % (kBD / 4);
        const int f = f0 + ff;
        float4 w = make_float4(0.f, 0.f, 0.f, 0.f);
        if (f < F) w = reinterpret_cast<const float4*>(W + (int64_t)f * kBD)[c4];
        Ws[(4 * c4 + 0) * kBPitch + ff] = w.x;
        Ws[(4 * c4 + 1) * kBPitch + ff] = w.y;
        Ws[(4 * c4 + 2) * kBPitch + ff] = w.z;
        Ws[(4 * c4 + 3) * kBPitch + ff] = w.w;
    }
    __syncthreads();

    const int tx = tid & 15, ty = tid >> 4;
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
#pragma unroll 2
    for (int k = 0; k < kBD; ++k) {
        const float4 xa = *reinterpret_cast<const float4*>(Xs + k * kBPitch + ty * 8);
        const float4 xb = *reinterpret_cast<const float4*>(Xs + k * kBPitch + ty * 8 + 4);
        const float4 wa = *reinterpret_cast<const float4*>(Ws + k * kBPitch + tx * 8);
        const float4 wb = *reinterpret_cast<const float4*>(Ws + k * kBPitch + tx * 8 + 4);
        const float xr[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
        const float wr[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(xr[i], wr[j], acc[i][j]);
    }

    const int cut = PASS == 2 ? ws.cut[u] : 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int64_t t = t0 + ty * 8 + i;
        if (t >= N) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int f = f0 + tx * 8 + j;
            if (f >= F) continue;
            const float v = __fadd_rn(acc[i][j], bias[f]);
            if (!(v > 0.f)) continue;
            const uint32_t bits = __float_as_uint(v);
            const int bin = (int)(bits >> 20);
            if (PASS == 1) {
                atomicAdd(&hist[bin], 1);
            } else {
                const long long flat = (long long)t * F + f;
                if (bin > cut) {
                    const int at = atomicAdd(&ws.n_members[u], 1);
                    if (at < ws.mcap) {
                        ws.members[(int64_t)u * ws.mcap + at] = flat;
                        atomicAdd(&lens[(int64_t)u * F + f], 1);
                    } else {
                        atomicOr(status, PK_STATUS_MEMBERS_FULL);
                    }
                } else if (bin == cut) {
                    const int at = atomicAdd(&ws.n_boundary[u], 1);
                    if (at < ws.bcap) {
                        const unsigned long long key =
                            ((unsigned long long)(0xFFFFFu - (bits & 0xFFFFFu)) << 40) | (unsigned long long)flat;
                        ws.boundary[(int64_t)u * ws.bcap + at] = (long long)key;
                    } else {
                        atomicOr(status, PK_STATUS_BOUNDARY_FULL);
                    }
                }
            }
        }
    }
    if (PASS == 1) {
        __syncthreads();
        for (int i = tid; i < kHistBins; i += kBThreads)
            if (hist[i]) atomicAdd(&ws.hist[(int64_t)u * kHistBins + i], hist[i]);
    }
}

// Coarse cut per unit: the bin holding the count-th largest positive value.
__global__ void build_cut_kernel(BuildWs ws, long long count) {
    const int u = blockIdx.x;
    if (threadIdx.x != 0) return;
    const int* h = ws.hist + (int64_t)u * kHistBins;
    long long above = 0;
    int b = kHistBins - 1;
    for (; b >= 0; --b) {
        if (above + h[b] >= count) break;
        above += h[b];
    }
    if (b < 0) {
        ws.cut[u] = -1;  // at most `count` positives: every one is a member
        ws.need[u] = 0;
    } else if (above + h[b] == count && b >= 0) {
        ws.cut[u] = b;   // the bin fills the budget exactly: all of it
        ws.need[u] = h[b];
    } else {
        ws.cut[u] = b;
        ws.need[u] = count - above;
    }
}

// Exact resolution of the boundary bin: the `need` smallest 64-bit keys.
__global__ void __launch_bounds__(1024)
build_resolve_kernel(BuildWs ws, int F, int* __restrict__ lens, int* __restrict__ status) {
    const int u = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
    __shared__ int hist[256];
    __shared__ unsigned long long s_prefix;
    __shared__ long long s_need;
    const long long need0 = ws.need[u];
    const int nb = ws.n_boundary[u];
    if (ws.cut[u] < 0 || need0 <= 0) return;
    if (nb > ws.bcap) {
        // Status already flagged by the encode pass; also stop an append
        // from committing an incomplete member list.
        if (tid == 0) atomicOr(ws.flag, 2);
        return;
    }
    const long long* B = ws.boundary + (int64_t)u * ws.bcap;
    unsigned long long prefix = ~0ull;  // take everything when need >= nb
    if (need0 < nb) {
        unsigned long long pre = 0, pmask = 0;
        long long need = need0;
        for (int pass = 0; pass < 8; ++pass) {
            const int shift = 56 - 8 * pass;
            for (int i = tid; i < 256; i += nt) hist[i] = 0;
            __syncthreads();
            for (int i = tid; i < nb; i += nt) {
                const unsigned long long kk = (unsigned long long)B[i];
                if ((kk & pmask) == pre) atomicAdd(&hist[(kk >> shift) & 255ull], 1);
            }
            __syncthreads();
            if (tid == 0) {
                long long acc = 0;
                int dgt = 0;
                for (; dgt < 256; ++dgt) {
                    if (acc + hist[dgt] >= need) break;
                    acc += hist[dgt];
                }
                s_prefix = pre | ((unsigned long long)dgt << shift);
                s_need = need - acc;
            }
            __syncthreads();
            pre = s_prefix;
            pmask |= 0xFFull << shift;
            need = s_need;
            __syncthreads();
        }
        prefix = pre;
    }
    // Keys are unique (flat indices differ): take every key <= prefix.
    for (int i = tid; i < nb; i += nt) {
        const unsigned long long kk = (unsigned long long)B[i];
        if (kk <= prefix) {
            const long long flat = (long long)(kk & ((1ull << 40) - 1));
            const int at = atomicAdd(&ws.n_members[u], 1);
            if (at < ws.mcap) {
                ws.members[(int64_t)u * ws.mcap + at] = flat;
                atomicAdd(&lens[(int64_t)u * F + (int)(flat % F)], 1);
            } else {
                atomicOr(status, PK_STATUS_MEMBERS_FULL);
            }
        }
    }
}

__host__ __device__ __forceinline__ int bucket_slack(int len, float frac, int smin) {
    return (int)ceilf((float)len * frac) + smin;
}

// offsets[u, f] = exclusive scan of (len + slack) over f; offsets[u, F] = total.
__global__ void __launch_bounds__(1024)
build_offsets_kernel(const int* __restrict__ lens, int F, float frac, int smin, int* __restrict__ offsets,
                     int64_t ids_stride, int* __restrict__ status) {
    const int u = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
    __shared__ int scan[40];
    const int per = (F + nt - 1) / nt;
    const int b0 = min(F, tid * per), b1 = min(F, b0 + per);
    long long mine = 0;
    for (int f = b0; f < b1; ++f) {
        const int l = lens[(int64_t)u * F + f];
        mine += l + bucket_slack(l, frac, smin);
    }
    int total;
    int at = block_exclusive_scan((int)min(mine, (long long)(INT32_MAX / 2)), scan, &total);
    int* off = offsets + (int64_t)u * (F + 1);
    for (int f = b0; f < b1; ++f) {
        off[f] = at;
        const int l = lens[(int64_t)u * F + f];
        at += l + bucket_slack(l, frac, smin);
    }
    if (tid == 0) {
        off[F] = total;
        if ((int64_t)total > ids_stride) atomicOr(status, PK_STATUS_MEMBERS_FULL);
    }
}

// Scatter members into their bucket regions at slot fill[u, f]++.
__global__ void build_scatter_kernel(BuildWs ws, int F, const int* __restrict__ offsets, int* __restrict__ ids,
                                     int64_t ids_stride, long long token_base) {
    const int u = blockIdx.y;
    const int n = (int)min((int64_t)ws.n_members[u], ws.mcap);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const long long flat = ws.members[(int64_t)u * ws.mcap + i];
        const int f = (int)(flat % F);
        const long long t = flat / F;
        const int slot = atomicAdd(&ws.fill[(int64_t)u * F + f], 1);
        ids[(int64_t)u * ids_stride + offsets[(int64_t)u * (F + 1) + f] + slot] = (int)(token_base + t);
    }
}

__device__ __forceinline__ int next_pow2(int x) {
    int p = 1;
    while (p < x) p <<= 1;
    return p;
}

__device__ void bitonic_sort_shared(int* a, int n, int lane, int nthreads, bool warp_only) {
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = lane; i < n / 2; i += nthreads) {
                const int lo = 2 * i - (i & (stride - 1));
                const int hi = lo + stride;
                const bool up = (lo & size) == 0;
                const int x = a[lo], y = a[hi];
                if ((x > y) == up) { a[lo] = y; a[hi] = x; }
            }
            if (warp_only) __syncwarp(); else __syncthreads();
        }
    }
}

// Sort ids[off[f] + start[f] .. + cnt[f]) ascending, one warp per bucket for
// buckets up to kSortWarpCap ids; larger ones go to the CTA sorter.
__global__ void __launch_bounds__(256)
sort_buckets_warp_kernel(int* __restrict__ ids, int64_t ids_stride, const int* __restrict__ offsets,
                         const int* __restrict__ start, const int* __restrict__ cnt, int F) {
    __shared__ int buf[8][kSortWarpCap];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int u = blockIdx.y;
    const int f = blockIdx.x * 8 + warp;
    if (f >= F) return;
    const int L = cnt[(int64_t)u * F + f];
    if (L <= 1 || L > kSortWarpCap) return;
    int* a = buf[warp];
    int* src = ids + (int64_t)u * ids_stride + offsets[(int64_t)u * (F + 1) + f] +
               (start ? start[(int64_t)u * F + f] : 0);
    const int n = next_pow2(L);
    for (int i = lane; i < n; i += 32) a[i] = i < L ? src[i] : INT32_MAX;
    __syncwarp();
    bitonic_sort_shared(a, n, lane, 32, true);
    for (int i = lane; i < L; i += 32) src[i] = a[i];
}

__global__ void __launch_bounds__(1024)
sort_buckets_big_kernel(int* __restrict__ ids, int64_t ids_stride, const int* __restrict__ offsets,
                        const int* __restrict__ start, const int* __restrict__ cnt, int F, int* __restrict__ status) {
    extern __shared__ int big[];
    const int u = blockIdx.y;
    // Grid-stride over the unit's buckets: only the few above the warp
    // kernel's capacity do any work.
    for (int f = blockIdx.x; f < F; f += gridDim.x) {
        const int L = cnt[(int64_t)u * F + f];
        if (L <= kSortWarpCap) continue;
        if (L > kSortBigCap) {
            if (threadIdx.x == 0) atomicOr(status, PK_STATUS_BUCKET_TOO_BIG);
            continue;
        }
        int* src = ids + (int64_t)u * ids_stride + offsets[(int64_t)u * (F + 1) + f] +
                   (start ? start[(int64_t)u * F + f] : 0);
        const int n = next_pow2(L);
        for (int i = threadIdx.x; i < n; i += blockDim.x) big[i] = i < L ? src[i] : INT32_MAX;
        __syncthreads();
        bitonic_sort_shared(big, n, threadIdx.x, blockDim.x, false);
        for (int i = threadIdx.x; i < L; i += blockDim.x) src[i] = big[i];
        __syncthreads();
    }
}

// Moments of the ORIGINAL keys per bucket (core.py:84-88) in torch's order:
// column cascade over the bucket's rows in list order, then / n.  One warp
// per bucket; lane owns dims 4*lane .. 4*lane+3.
template <typename T>
__global__ void __launch_bounds__(256)
summarize_kernel(const T* __restrict__ keys, int64_t unit_stride, int64_t row_stride,
                 const int* __restrict__ offsets, const int* __restrict__ start, const int* __restrict__ cnt,
                 const int* __restrict__ ids, int64_t ids_stride, long long token_base, int F,
                 float* __restrict__ mean, float* __restrict__ var) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int u = blockIdx.y;
    const int f = blockIdx.x * 8 + warp;
    if (f >= F) return;
    const int L = cnt[(int64_t)u * F + f];
    const int* lst = ids + (int64_t)u * ids_stride + offsets[(int64_t)u * (F + 1) + f] +
                     (start ? start[(int64_t)u * F + f] : 0);
    float* mu = mean + ((int64_t)u * F + f) * kBD;
    float* nu = var + ((int64_t)u * F + f) * kBD;
    if (L == 0) {
#pragma unroll
        for (int j = 0; j < 4; ++j) { mu[4 * lane + j] = 0.f; nu[4 * lane + j] = 0.f; }
        return;
    }
#pragma unroll 1
    for (int j = 0; j < 4; ++j) {
        const int c = 4 * lane + j;
        const float s = torch_cascade_sum((int64_t)L, [&](int64_t i) {
            return key_at(keys, unit_stride, row_stride, u, (int64_t)lst[i] - token_base, c);
        });
        const float mj = __fdiv_rn(s, (float)L);
        const float s2 = torch_cascade_sum((int64_t)L, [&](int64_t i) {
            const float x = __fsub_rn(key_at(keys, unit_stride, row_stride, u, (int64_t)lst[i] - token_base, c), mj);
            return __fmul_rn(x, x);
        });
        mu[c] = mj;
        nu[c] = __fdiv_rn(s2, (float)L);
    }
}

// Parallel-formula merge of old and new bucket moments (core.py:194-199),
// in the reference's operation order.  Skipped when the append was refused.
__global__ void merge_moments_kernel(const int* __restrict__ lens_old, const int* __restrict__ cnt_new, int F,
                                     float* __restrict__ mean, float* __restrict__ var,
                                     const float* __restrict__ mean_new, const float* __restrict__ var_new,
                                     const int* __restrict__ flag) {
    if (flag && *flag) return;
    const int u = blockIdx.y;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)F * kBD) return;
    const int f = (int)(i / kBD);
    const float a = (float)lens_old[(int64_t)u * F + f], b = (float)cnt_new[(int64_t)u * F + f];
    const float tot = __fadd_rn(a, b);
    const float den = tot > 1.f ? tot : 1.f;
    const int64_t j = (int64_t)u * F * kBD + i;
    const float ma = mean[j], mb = mean_new[j], va = var[j], vb = var_new[j];
    const float mu = __fdiv_rn(__fadd_rn(__fmul_rn(a, ma), __fmul_rn(b, mb)), den);
    float nv = __fdiv_rn(__fadd_rn(__fmul_rn(a, va), __fmul_rn(b, vb)), den);
    const float w = __fdiv_rn(__fmul_rn(a, b), __fmul_rn(den, den));
    const float dm = __fsub_rn(ma, mb);
    nv = __fadd_rn(nv, __fmul_rn(w, __fmul_rn(dm, dm)));
    mean[j] = mu;
    var[j] = nv;
}

// Append check: every bucket must fit its region; all-or-nothing.
__global__ void append_check_kernel(const int* __restrict__ offsets, const int* __restrict__ lens,
                                    const int* __restrict__ cnt_new, int F, int* __restrict__ flag) {
    const int u = blockIdx.y;
    for (int f = blockIdx.x * blockDim.x + threadIdx.x; f < F; f += gridDim.x * blockDim.x) {
        const int cap = offsets[(int64_t)u * (F + 1) + f + 1] - offsets[(int64_t)u * (F + 1) + f];
        if (lens[(int64_t)u * F + f] + cnt_new[(int64_t)u * F + f] > cap) atomicOr(flag, 1);
    }
}

__global__ void status_gate_kernel(const int* __restrict__ status, int* __restrict__ flag) {
    if (threadIdx.x == 0 && (*status & (PK_STATUS_NEEDS_EXACT | PK_STATUS_BOUNDARY_FULL | PK_STATUS_MEMBERS_FULL)))
        atomicOr(flag, 2);
}

// A refused append zeroes the new counts so nothing downstream (sort,
// moments, commit) touches the index.
__global__ void append_gate_kernel(const int* __restrict__ flag, int* __restrict__ cnt_new, int64_t n) {
    if (!*flag) return;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        cnt_new[i] = 0;
}

__global__ void append_scatter_kernel(BuildWs ws, int F, const int* __restrict__ offsets, const int* __restrict__ lens,
                                      int* __restrict__ ids, int64_t ids_stride, long long token_base) {
    if (*ws.flag) return;
    const int u = blockIdx.y;
    const int n = (int)min((int64_t)ws.n_members[u], ws.mcap);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const long long flat = ws.members[(int64_t)u * ws.mcap + i];
        const int f = (int)(flat % F);
        const long long t = flat / F;
        const int slot = atomicAdd(&ws.fill[(int64_t)u * F + f], 1);
        ids[(int64_t)u * ids_stride + offsets[(int64_t)u * (F + 1) + f] + lens[(int64_t)u * F + f] + slot] =
            (int)(token_base + t);
    }
}

__global__ void append_commit_kernel(const int* __restrict__ flag, int* __restrict__ lens,
                                     const int* __restrict__ cnt_new, int F, int* __restrict__ status) {
    const int u = blockIdx.y;
    const bool full = *flag != 0;
    for (int f = blockIdx.x * blockDim.x + threadIdx.x; f < F; f += gridDim.x * blockDim.x)
        if (!full) lens[(int64_t)u * F + f] += cnt_new[(int64_t)u * F + f];
    if ((*flag & 1) && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) atomicOr(status, PK_STATUS_BUCKET_FULL);
}

// ---------------------------------------------------------------------------
// Host-side helpers
// ---------------------------------------------------------------------------

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

size_t counters_bytes(int U, int F) {
    return align256((size_t)U * kHistBins * 4) + align256((size_t)U * 4) + align256((size_t)U * 8) +
           2 * align256((size_t)U * 4) + align256((size_t)U * F * 4) + align256(16);
}

size_t carve_bytes(int U, int F, int64_t mcap, int64_t bcap) {
    return counters_bytes(U, F) + align256((size_t)U * mcap * 8) + align256((size_t)U * bcap * 8);
}

BuildWs carve(void* base, int U, int F, int64_t mcap, int64_t bcap) {
    BuildWs w;
    char* p = (char*)base;
    w.hist = (int*)p; p += align256((size_t)U * kHistBins * 4);
    w.cut = (int*)p; p += align256((size_t)U * 4);
    w.need = (long long*)p; p += align256((size_t)U * 8);
    w.n_members = (int*)p; p += align256((size_t)U * 4);
    w.n_boundary = (int*)p; p += align256((size_t)U * 4);
    w.fill = (int*)p; p += align256((size_t)U * F * 4);
    w.flag = (int*)p; p += align256(16);
    w.members = (long long*)p; p += align256((size_t)U * mcap * 8);
    w.boundary = (long long*)p;
    w.mcap = mcap;
    w.bcap = bcap;
    return w;
}

template <typename T>
int run_encode_select(const T* keys, int64_t unit_stride, int64_t row_stride, int64_t N, const float* center,
                      float key_scale, const float* W, const float* b, int U, int F, long long count, BuildWs ws,
                      int* lens, int* status, cudaStream_t st) {
    const size_t smem = (size_t)2 * kBD * kBPitch * sizeof(float) + kHistBins * sizeof(int);
    dim3 grid((F + kBF - 1) / kBF, (unsigned)((N + kBT - 1) / kBT), U);
    cudaFuncSetAttribute(build_encode_kernel<1, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(build_encode_kernel<2, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    build_encode_kernel<1, T><<<grid, kBThreads, smem, st>>>(keys, unit_stride, row_stride, N, center, key_scale, W,
                                                             b, F, ws, lens, status);
    PK_CHECK_LAUNCH();
    build_cut_kernel<<<U, 32, 0, st>>>(ws, count);
    PK_CHECK_LAUNCH();
    build_encode_kernel<2, T><<<grid, kBThreads, smem, st>>>(keys, unit_stride, row_stride, N, center, key_scale, W,
                                                             b, F, ws, lens, status);
    PK_CHECK_LAUNCH();
    build_resolve_kernel<<<U, 1024, 0, st>>>(ws, F, lens, status);
    PK_CHECK_LAUNCH();
    return PK_OK;
}

// ---------------------------------------------------------------------------
// Bound-filtered build: approximate activations on the tensor cores with a
// per-entry error bound, global thresholds that bracket the exact budget
// threshold, exact recomputation of only the entries the bounds cannot decide.
//
// Operands are fp16 (unit roundoff 2^-11; x and W_f stay far inside its
// range, which is checked): with fp32 accumulation of exact products,
//   |v - exact| <= e = 2^-9 |x| |W_f| + 2^-21 (|x| + |W_f|) + 2^-20 |v|
// (2^-10 relative from the two roundings and the accumulation, doubled; the
// second term covers fp16 subnormals, the third the reference order's own
// rounding).  Rows with |x_i| >= 60000 or features with |W_f| >= 60000 raise
// PK_STATUS_NEEDS_EXACT (the caller reruns the exact path).
//
// Each CTA holds 128 tokens of one unit (x = (k - c) / s, rounded to fp16)
// and streams every 256-feature tile of W through a double buffer on the
// tcgen05 tensor cores (build_tile_tc_kernel), so a token block's histogram
// and candidates are gathered once per CTA.
//   MODE 0 (sample): histogram of the positive lower bounds of a strided
//     sample of token blocks and feature tiles, all 8192 bins; it places a
//     floor well below the budget threshold.
//   MODE 1: histograms of the lower and upper bounds at or above the floor
//     (a 1024-bin window; the top bin collects everything above); entries
//     whose upper bound reaches the floor are kept, with their bounds, for
//     build_classify_kernel (one tensor-core pass in all).
// ---------------------------------------------------------------------------

constexpr int kFBins = 8192;          // bins of the bounds' float bits >> 18
constexpr int kFShift = 18;
constexpr int kFWin = 1024;           // histogram window above the floor (32 octaves)
constexpr int kFSampleMargin = 2;     // floor: 2x the sample's share of the budget

struct FastWs {
    int* histL;                 // [U, kFWin] lower bounds from floor_bin up
    int* histU;                 // [U, kFWin] upper bounds from floor_bin up
    int* histS;                 // [U, kFBins] sampled positive lower bounds
    int* floor_bin;             // [U]
    int* cutL;                  // [U] bin of the count-th largest lower bound (-1: fewer positives)
    int* cutU;                  // [U] same for the upper bound
    int* n_amb;                 // [U]
    int* n_cand;                // [U]
    long long* amb;             // [U, acap] flat indices to recompute exactly
    float2* cand_hl;            // [U, acap] (U, L) bounds of the entries at or above the floor
    long long* cand_flat;       // [U, acap] their flat indices
    uint8_t* tiles;             // [ceil(F/256)] W_half tile images (64 KB each)
    uint8_t* sides;             // [ceil(F/256)] side records (norms, biases, maxima)
    int64_t acap;
};

size_t fast_counters_bytes(int U) {
    return 2 * align256((size_t)U * kFWin * 4) + align256((size_t)U * kFBins * 4) + align256((size_t)U * 4) +
           4 * align256((size_t)U * 4);
}
size_t fast_bytes(int U, int64_t acap, int F) {
    const size_t ntf = (size_t)((F + 255) / 256);
    return fast_counters_bytes(U) + 2 * align256((size_t)U * acap * 8) + align256((size_t)U * acap * 8) +
           align256(ntf * 256 * 256) + align256(ntf * (2 * 256 * 4 + 16));
}

FastWs carve_fast(void* base, int U, int64_t acap, int F) {
    FastWs w;
    char* p = (char*)base;
    w.histL = (int*)p; p += align256((size_t)U * kFWin * 4);
    w.histU = (int*)p; p += align256((size_t)U * kFWin * 4);
    w.histS = (int*)p; p += align256((size_t)U * kFBins * 4);
    w.floor_bin = (int*)p; p += align256((size_t)U * 4);
    w.cutL = (int*)p; p += align256((size_t)U * 4);
    w.cutU = (int*)p; p += align256((size_t)U * 4);
    w.n_amb = (int*)p; p += align256((size_t)U * 4);
    w.n_cand = (int*)p; p += align256((size_t)U * 4);
    w.amb = (long long*)p; p += align256((size_t)U * acap * 8);
    w.cand_hl = (float2*)p; p += align256((size_t)U * acap * 8);
    w.cand_flat = (long long*)p; p += align256((size_t)U * acap * 8);
    const size_t ntf = (size_t)((F + 255) / 256);
    w.tiles = (uint8_t*)p; p += align256(ntf * 256 * 256);
    w.sides = (uint8_t*)p;
    w.acap = acap;
    return w;
}

__device__ __forceinline__ int fbin(float v) { return (int)(__float_as_uint(v) >> kFShift); }
__device__ __forceinline__ unsigned lane_below() {
    unsigned m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

// v[base + q] for a run-time q in [0, 32): a select tree over the bits of q,
// so that the array stays in registers (no local-memory indexing).
template <int N>
__device__ __forceinline__ float pick32(const float (&v)[N], int base, int q) {
    float a[16], b[8], c[4], e[2];
#pragma unroll
    for (int i = 0; i < 16; ++i) a[i] = (q & 1) ? v[base + 2 * i + 1] : v[base + 2 * i];
#pragma unroll
    for (int i = 0; i < 8; ++i) b[i] = (q & 2) ? a[2 * i + 1] : a[2 * i];
#pragma unroll
    for (int i = 0; i < 4; ++i) c[i] = (q & 4) ? b[2 * i + 1] : b[2 * i];
#pragma unroll
    for (int i = 0; i < 2; ++i) e[i] = (q & 8) ? c[2 * i + 1] : c[2 * i];
    return (q & 16) ? e[1] : e[0];
}

struct TileSample {
    int tb_stride, ft_stride;   // MODE 0: token blocks and feature tiles sampled
};

// Built once per call, per 256-feature tile: a side record of the tile's
// norms, biases (zero past F) and, per 128 features, the largest |W_f| and
// b_f for the epilogue's row tests; and, only when W_half cannot be loaded
// through a tensor map, an image of its rows in the tensor core's shared
// memory layout (two 128-byte-swizzled K-atoms of 256 rows).  W rows out of
// fp16 range raise PK_STATUS_NEEDS_EXACT.
constexpr int kTcFeat = 256;
constexpr int kTcWBytes = kTcFeat * 256;            // 2 K-atoms x 256 rows x 128 B
constexpr int kTcSideBytes = 2 * kTcFeat * 4 + 16;  // norms, biases, 2 x (max |W_f|, max b_f)

__global__ void __launch_bounds__(256)
build_tiles_kernel(const __half* __restrict__ Wh, const float* __restrict__ wn, const float* __restrict__ bias,
                   int F, uint8_t* __restrict__ tiles, uint8_t* __restrict__ sides, int* __restrict__ status,
                   int write_images) {
    const int t = blockIdx.x, row = threadIdx.x, lane = row & 31, warp = row >> 5;
    const int f = t * kTcFeat + row;
    const bool valid = f < F;
    if (write_images) {   // (not needed when the passes load W through a tensor map)
        uint8_t* img = tiles + (int64_t)t * kTcWBytes;
        const uint4* src = reinterpret_cast<const uint4*>(Wh + (int64_t)(valid ? f : 0) * kBD);
#pragma unroll
        for (int ch = 0; ch < 16; ++ch) {
            const uint4 val = valid ? src[ch] : make_uint4(0u, 0u, 0u, 0u);
            *reinterpret_cast<uint4*>(img + (ch >> 3) * (kTcFeat * 128) + sw128_off(row, ch & 7)) = val;
        }
    }
    float* sw = reinterpret_cast<float*>(sides + (int64_t)t * kTcSideBytes);
    const float w = valid ? wn[f] : 0.f, b = valid ? bias[f] : -INFINITY;
    sw[row] = w;
    sw[kTcFeat + row] = valid ? b : 0.f;
    if (w >= 60000.f) atomicOr(status, PK_STATUS_NEEDS_EXACT);
    __shared__ float mw[8], mb[8];
    const float a = warp_max(w), c = warp_max(b);
    if (lane == 0) {
        mw[warp] = a;
        mb[warp] = c;
    }
    __syncthreads();
    if (row < 2) {
        float x = mw[4 * row], y = mb[4 * row];
        for (int i = 1; i < 4; ++i) {
            x = fmaxf(x, mw[4 * row + i]);
            y = fmaxf(y, mb[4 * row + i]);
        }
        reinterpret_cast<float2*>(sw + 2 * kTcFeat)[row] = make_float2(x, y == -INFINITY ? 0.f : y);
    }
}

// The passes run on the 5th-generation tensor cores, one CTA per 128-token
// block of a unit (one CTA per SM), warp-specialised:
//   warp 8 (one thread): loads tile j's W rows straight from W_half with two
//     tensor-map TMA boxes (the K-atoms, 128-byte swizzled by the copy
//     engine) and its side record with a bulk copy into shared-memory buffer
//     j & 1, and issues the eight
//     K=16 MMAs of tile j into TMEM accumulator j & 1 once the copy has
//     landed and the epilogue of tile j-2 has drained that accumulator;
//   warps 0-15: the epilogue of tile j from TMEM -- one token row and 64
//     features per thread (warp w: rows of lane quarter w % 4, features of
//     quarter w / 4) -- then release the accumulator; warps 0-7 also stage
//     the CTA's 128 key rows first.
// The stages meet on mbarriers only (full, MMA done, TMEM empty per buffer);
// every wait is bounded, and a wait that runs out aborts the CTA with
// PK_STATUS_NEEDS_EXACT after the copies and MMAs in flight have landed.
//   MODE 0: histogram of sampled lower bounds (one per 32 columns) to place
//     the floor well below the budget threshold.
//   MODE 1: histograms of the lower and upper bounds at or above the floor
//     (a 1024-bin window; the top bin collects everything above); entries
//     whose upper bound reaches the floor are kept, with their bounds, for
//     build_classify_kernel (one tensor-core pass in all).
constexpr int kTcTokens = 128, kTcEpiWarps = 16, kTcThreads = 32 * (kTcEpiWarps + 1);
constexpr int kTcStageWarps = 8;                                  // warps that stage the key rows (16 each)
constexpr int kTcCols = kTcFeat * 4 / kTcEpiWarps;                // features per epilogue thread
constexpr int kTcChunks = kTcCols / 32;
static_assert(kTcCols == 64, "the epilogue loads its 64 columns with one tmem_ld64_wait");
constexpr int kTcXBytes = kTcTokens * 256;          // 2 K-atoms x 128 rows x 128 B
constexpr int kTcSideSlots = 4;                     // side records: tile j in slot j % 4
constexpr uint64_t kTcWaitNs = 200000000ull;        // 0.2 s: no copy or MMA takes this long
constexpr int kTcStage = 2048;                      // MODE 1: staged candidates per CTA
constexpr int kWarpStage = kTcStage / kTcEpiWarps;  // ... per epilogue warp

__host__ __device__ constexpr int tc_smem(int mode) {
    return 1024 /* alignment slack */ + kTcXBytes + 2 * kTcWBytes + kTcSideSlots * kTcSideBytes + kTcTokens * 4 +
           (mode == 0 ? kFBins * 4 : 2 * kFWin * 4) + 10 * 8 + 16 + (mode == 1 ? kTcStage * 16 : 0);
}

// The W operand's source: a tensor map over W_half [F, d] fp16 (the
// tile's two 128-byte-swizzled K-atoms, 256 feature rows each, loaded by
// the TMA straight into the tensor core's layout; rows past F are filled
// with zeros), or, without one, the tile images of build_tiles_kernel.
struct WSource {
    CUtensorMap map;   // valid when use_map
    int use_map;
};

template <int MODE, typename T>
__global__ void __launch_bounds__(kTcThreads, 1)
build_tile_tc_kernel(const T* __restrict__ keys, int64_t unit_stride, int64_t row_stride, int64_t N,
                     const float* __restrict__ center, float key_scale, int F, FastWs fw, TileSample smp,
                     int* __restrict__ status, const __grid_constant__ WSource wsrc) {
    extern __shared__ uint8_t tc_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* Xs = base;
    uint8_t* Wt = base + kTcXBytes;                                           // [2][kTcWBytes]
    uint8_t* side = Wt + 2 * kTcWBytes;                                       // [4][kTcSideBytes]
    float* xn = reinterpret_cast<float*>(side + kTcSideSlots * kTcSideBytes); // [128]
    int* hA = reinterpret_cast<int*>(xn + kTcTokens);                        // MODE 0: [kFBins]; MODE 1: L [kFWin]
    int* hB = hA + kFWin;                                                    // MODE 1: U [kFWin]
    uint64_t* bars = reinterpret_cast<uint64_t*>(hA + (MODE == 0 ? kFBins : 2 * kFWin));
    uint64_t* full = bars;          // [2] W tile landed
    uint64_t* mma_done = bars + 2;  // [2] MMAs of the tile complete
    uint64_t* tmem_empty = bars + 4; // [2] epilogue drained the accumulator
    uint64_t* side_full = bars + 6;  // [4] side record landed (slot j % 4)
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 10);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);
    float2* stg_hl = reinterpret_cast<float2*>(tslot + 4);                    // MODE 1: [kTcStage]
    long long* stg_flat = reinterpret_cast<long long*>(stg_hl + kTcStage);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int u = blockIdx.y;
    const int64_t t0 = (int64_t)blockIdx.x * (MODE == 0 ? smp.tb_stride : 1) * kTcTokens;
    const float* cu = center + (int64_t)u * kBD;
    const int ntf = (F + kTcFeat - 1) / kTcFeat;
    const int fstep = MODE == 0 ? smp.ft_stride : 1;
    const int ft_first = MODE == 0 ? (int)(blockIdx.x % fstep) : 0;
    const int ntiles = ft_first < ntf ? (ntf - ft_first + fstep - 1) / fstep : 0;
    const bool producer = warp == kTcEpiWarps && lane == 0;
    // Each barrier phase is waited for before the barrier can complete
    // again (a parity wait tells only the current phase from the last):
    // copy j + 2 into W buffer j & 1 follows MMA j, and copy j + 4 into side
    // slot j % 4 follows MMA j + 2, which follows epilogue j.
    auto load_tile = [&](int j) {
        const int t = ft_first + j * fstep;
        const uint32_t wbar = smem_addr(&full[j & 1]), sbar = smem_addr(&side_full[j % kTcSideSlots]);
        mbar_expect_tx(wbar, kTcWBytes);
        const uint32_t wdst = smem_addr(Wt + (j & 1) * kTcWBytes);
        if (wsrc.use_map) {
            // Two boxes of 64 fp16 x 256 rows: the K-atoms of d 0..63, 64..127.
            tma_load_2d(wdst, &wsrc.map, 0, t * kTcFeat, wbar);
            tma_load_2d(wdst + kTcFeat * 128, &wsrc.map, 64, t * kTcFeat, wbar);
        } else {
            bulk_g2s(wdst, fw.tiles + (int64_t)t * kTcWBytes, kTcWBytes, wbar);
        }
        mbar_expect_tx(sbar, kTcSideBytes);
        bulk_g2s(smem_addr(side + (j % kTcSideSlots) * kTcSideBytes), fw.sides + (int64_t)t * kTcSideBytes,
                 kTcSideBytes, sbar);
    };

    if (warp == kTcEpiWarps) tmem_alloc(smem_addr(tslot), 512);
    int n_loaded = 0;
    if (producer) {
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_addr(&full[b]), 1);
            mbar_init(smem_addr(&mma_done[b]), 1);
            mbar_init(smem_addr(&tmem_empty[b]), kTcEpiWarps);
        }
        for (int k = 0; k < kTcSideSlots; ++k) mbar_init(smem_addr(&side_full[k]), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (; n_loaded < 2 && n_loaded < ntiles; ++n_loaded) load_tile(n_loaded);
    }
    if (MODE == 0)
        for (int i = tid; i < kFBins; i += kTcThreads) hA[i] = 0;
    else
        for (int i = tid; i < 2 * kFWin; i += kTcThreads) hA[i] = 0;
    if (warp < kTcStageWarps) {
        // x = (k - center) / key_scale in fp32 (core.py:99), rounded to fp16;
        // this warp's 16 key rows, every load issued before any is used.
        const bool unit_scale = key_scale == 1.0f;
        float kr[16][4];
#pragma unroll
        for (int rr = 0; rr < 16; ++rr) {
            const int64_t t = t0 + warp * 16 + rr;
#pragma unroll
            for (int e = 0; e < 4; ++e)
                kr[rr][e] = t < N ? key_at(keys, unit_stride, row_stride, u, t, 4 * lane + e) : 0.f;
        }
        float cl[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) cl[e] = cu[4 * lane + e];
#pragma unroll
        for (int rr = 0; rr < 16; ++rr) {
            const int row = warp * 16 + rr;
            const int64_t t = t0 + row;
            float x[4] = {0.f, 0.f, 0.f, 0.f};
            if (t < N) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float dlt = __fsub_rn(kr[rr][e], cl[e]);
                    x[e] = unit_scale ? dlt : __fdiv_rn(dlt, key_scale);
                }
            }
            float ss = fmaf(x[0], x[0], fmaf(x[1], x[1], fmaf(x[2], x[2], x[3] * x[3])));
            ss = warp_sum(ss);
            const float amax = warp_max(fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3]))));
            if (lane == 0) {
                xn[row] = sqrtf(ss) * (1.0f + 1.0f / 4096.0f);
                if (!(amax < 60000.f)) atomicOr(status, PK_STATUS_NEEDS_EXACT);
            }
            __half2 p0 = __floats2half2_rn(x[0], x[1]), p1 = __floats2half2_rn(x[2], x[3]);
            uint2 pk2;
            pk2.x = *reinterpret_cast<uint32_t*>(&p0);
            pk2.y = *reinterpret_cast<uint32_t*>(&p1);
            const int chunk = lane >> 1;   // 16-byte chunk of the 256-byte row
            *reinterpret_cast<uint2*>(Xs + (chunk >> 3) * (kTcTokens * 128) + sw128_off(row, chunk & 7) +
                                      (lane & 1) * 8) = pk2;
        }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;

    if (producer) {
        // ------------------------------------------------ copies and MMAs
        const uint32_t idesc = f16_idesc(128, kTcFeat, 0);
        const uint32_t xa = smem_addr(Xs);
        int n_mma = 0;
        for (int j = 0; j < ntiles && !*abort_flag; ++j) {
            const int b = j & 1;
            bool ok = mbar_wait(smem_addr(&full[b]), (j >> 1) & 1, kTcWaitNs);
            if (ok && j >= 2) ok = mbar_wait(smem_addr(&tmem_empty[b]), ((j - 2) >> 1) & 1, kTcWaitNs);
            if (!ok) {
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const uint32_t wa = smem_addr(Wt + b * kTcWBytes);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                const uint32_t koff = (uint32_t)((kk & 3) * 32);   // K=16 step inside the 128-byte atom
                umma_f16(tmem + b * kTcFeat, sw128_desc(xa + (kk >> 2) * (kTcTokens * 128) + koff),
                         sw128_desc(wa + (kk >> 2) * (kTcFeat * 128) + koff), idesc, kk > 0 ? 1u : 0u);
            }
            umma_commit(smem_addr(&mma_done[b]));
            n_mma = j + 1;
            if (j + 2 < ntiles) {
                // Buffer b is free once MMA j has read it; side slot
                // (j + 2) % 4 held tile j - 2, drained before MMA j.
                if (!mbar_wait(smem_addr(&mma_done[b]), (j >> 1) & 1, kTcWaitNs)) {
                    *abort_flag = 1;
                    break;
                }
                load_tile(j + 2);
                n_loaded = j + 3;
            }
        }
        if (*abort_flag) {
            // Let every copy and MMA in flight land before the CTA exits
            // (the last copies into each buffer and slot, the last MMAs).
            for (int j = n_loaded > 2 ? n_loaded - 2 : 0; j < n_loaded; ++j)
                mbar_wait(smem_addr(&full[j & 1]), (j >> 1) & 1, kTcWaitNs);
            for (int j = n_loaded > kTcSideSlots ? n_loaded - kTcSideSlots : 0; j < n_loaded; ++j)
                mbar_wait(smem_addr(&side_full[j % kTcSideSlots]), (j / kTcSideSlots) & 1, kTcWaitNs);
            if (n_mma > 0) mbar_wait(smem_addr(&mma_done[(n_mma - 1) & 1]), ((n_mma - 1) >> 1) & 1, kTcWaitNs);
        }
    } else if (warp < kTcEpiWarps) {
        // ------------------------------------------------------- epilogue
        const int floor_bin = MODE == 1 ? fw.floor_bin[u] : 0;
        const int row = 32 * (warp & 3) + lane, part = warp >> 2, half = part * kTcCols / 128;
        const int64_t trow_t = t0 + row;
        const bool trow = trow_t < N;
        const float xr = xn[row];
        const float cx = 0.001953125f * xr;
        const float fval = __uint_as_float((uint32_t)floor_bin << kFShift);
        float2* whl = stg_hl + warp * kWarpStage;
        long long* wflat = stg_flat + warp * kWarpStage;
        int wcnt = 0;   // this warp's staged candidates (warp-uniform)
        auto warp_flush = [&]() {
            __syncwarp();
            int g = 0;
            if (lane == 0) g = atomicAdd(&fw.n_cand[u], wcnt);
            g = __shfl_sync(0xffffffffu, g, 0);
            for (int e = lane; e < wcnt; e += 32) {
                const int64_t at = (int64_t)g + e;
                if (at < fw.acap) {
                    fw.cand_hl[(int64_t)u * fw.acap + at] = whl[e];
                    fw.cand_flat[(int64_t)u * fw.acap + at] = wflat[e];
                } else if (at == fw.acap) {
                    atomicOr(status, PK_STATUS_BOUNDARY_FULL);
                }
            }
            __syncwarp();
            wcnt = 0;
        };
        for (int j = 0; j < ntiles; ++j) {
            const int b = j & 1;
            bool done = mbar_wait(smem_addr(&mma_done[b]), (j >> 1) & 1, kTcWaitNs);
            if (done)
                done = mbar_wait(smem_addr(&side_full[j % kTcSideSlots]), (j / kTcSideSlots) & 1, kTcWaitNs);
            if (__any_sync(0xffffffffu, !done || *abort_flag)) {   // warp-uniform exit
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const int f0 = (ft_first + j * fstep) * kTcFeat + part * kTcCols;
            const float* sd = reinterpret_cast<const float*>(side + (j % kTcSideSlots) * kTcSideBytes);
            const float* wnb = sd + part * kTcCols;
            const float* bb = sd + kTcFeat + part * kTcCols;
            // The side record's maxima cover 128-feature halves (bounds for
            // any quarter inside).
            const float2 st2 = reinterpret_cast<const float2*>(sd + 2 * kTcFeat)[half];
            const float wm = st2.x, bm = st2.y;
            const float cs = 4.76837158203125e-07f * (xr + wm);
            const float E = cx * wm * (1.0f + 1.0f / 65536.0f) + cs;
            auto err_of = [&](int col, float v) { return fmaf(cx, wnb[col], cs + 9.5367431640625e-07f * fabsf(v)); };
            // MODE 1 keeps v = acc + b_f >= vfloor (U can reach the floor);
            // MODE 0 bins positive v.  Either needs acc >= tau: one compare
            // per entry, the full bound work only for the entries it keeps.
            const float vfloor = fval - 1.001f * E - 3.814697265625e-06f * (fval + E);
            const float tau = vfloor - bm;
            const uint32_t taddr = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)(b * kTcFeat + part * kTcCols);
            // The row's kTcCols accumulators in one TMEM round trip.
            float v[kTcCols];
            __syncwarp();
            tmem_ld64_wait(taddr, v);
            if (MODE == 0) {
                // The sample bins one lower bound per 32 columns, below the
                // largest of theirs (E bounds every column's error).  Counts
                // above any bin then fall short of the entries' -- the floor
                // comes out lower, never unsafe.  Columns past F hold v = 0,
                // which bins nothing.
                if (trow) {
#pragma unroll
                    for (int c = 0; c < kTcChunks; ++c) {
                        float mx = -INFINITY;
#pragma unroll
                        for (int q = 0; q < 32; ++q) mx = fmaxf(mx, v[32 * c + q] + bb[32 * c + q]);
                        if (mx > 0.f) {
                            const float lo = mx - (E + 9.5367431640625e-07f * mx);
                            if (lo > 0.f) atomicAdd(&hA[fbin(lo)], 1);
                        }
                    }
                }
            } else {
                uint32_t m[kTcChunks];
#pragma unroll
                for (int c = 0; c < kTcChunks; ++c) {
                    uint32_t mc = 0;
#pragma unroll
                    for (int q = 0; q < 32; ++q) mc |= (v[32 * c + q] >= tau ? 1u : 0u) << q;
                    const int cols_left = F - (f0 + c * 32);
                    if (!trow || cols_left <= 0) mc = 0;
                    else if (cols_left < 32) mc &= (1u << cols_left) - 1u;
                    m[c] = mc;
                }
                // Slots for every kept entry in this warp's staging buffer
                // (flushed to the unit's list with one global reservation
                // when full; a tile larger than the buffer reserves its own),
                // one scan per tile; entries whose exact U misses the floor
                // get U = -1.  Kept entries are rare: loops over the set bits
                // (a branch per entry, not a predicated body per column).
                int nk = 0;
#pragma unroll
                for (int c = 0; c < kTcChunks; ++c) nk += __popc(m[c]);
                const int inc = warp_inclusive_scan(nk);
                const int wtot = __shfl_sync(0xffffffffu, inc, 31);
                if (wtot > 0) {
                    if (wcnt + wtot > kWarpStage && wcnt > 0) warp_flush();
                    const bool direct = wtot > kWarpStage;
                    int slot;
                    if (direct) {
                        int g = 0;
                        if (lane == 31) g = atomicAdd(&fw.n_cand[u], wtot);
                        slot = __shfl_sync(0xffffffffu, g, 31) + inc - nk;
                    } else {
                        slot = wcnt + inc - nk;
                        wcnt += wtot;
                    }
#pragma unroll
                    for (int c = 0; c < kTcChunks; ++c) {
                        for (uint32_t mm = m[c]; mm; mm &= mm - 1) {
                            const int q = __ffs(mm) - 1;
                            const int col = c * 32 + q;
                            const float vv = pick32(v, 32 * c, q) + bb[col];
                            const float err = err_of(col, vv);
                            const float lo = vv - err, hi = vv + err;
                            bool keep = false;
                            if (hi > 0.f) {
                                const int bh = fbin(hi) - floor_bin;
                                if (bh >= 0) {
                                    atomicAdd(&hB[min(bh, kFWin - 1)], 1);
                                    keep = true;
                                }
                            }
                            if (lo > 0.f) {
                                const int bl = fbin(lo) - floor_bin;
                                if (bl >= 0) atomicAdd(&hA[min(bl, kFWin - 1)], 1);
                            }
                            const float2 hl = make_float2(keep ? hi : -1.f, lo);
                            const long long flat = trow_t * F + f0 + col;
                            if (!direct) {
                                whl[slot] = hl;
                                wflat[slot] = flat;
                            } else if (slot < fw.acap) {
                                fw.cand_hl[(int64_t)u * fw.acap + slot] = hl;
                                fw.cand_flat[(int64_t)u * fw.acap + slot] = flat;
                            } else {
                                atomicOr(status, PK_STATUS_BOUNDARY_FULL);
                            }
                            ++slot;
                        }
                    }
                }
            }
            // Accumulator b drained: MMA j + 2 may overwrite it.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_addr(&tmem_empty[b]));
        }
        if (MODE == 1 && wcnt > 0) warp_flush();
    }
    __syncthreads();
    if (tid == 0 && *abort_flag) atomicOr(status, PK_STATUS_NEEDS_EXACT);
    if (MODE == 0) {
        for (int i = tid; i < kFBins; i += kTcThreads)
            if (hA[i]) atomicAdd(&fw.histS[(int64_t)u * kFBins + i], hA[i]);
    } else {
        for (int i = tid; i < kFWin; i += kTcThreads) {
            if (hA[i]) atomicAdd(&fw.histL[(int64_t)u * kFWin + i], hA[i]);
            if (hB[i]) atomicAdd(&fw.histU[(int64_t)u * kFWin + i], hB[i]);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kTcEpiWarps) tmem_dealloc(tmem, 512);
}

// Per unit: the floor bin.  Scanning the sample's upper-bound histogram from
// the top, the floor is the bin where the count reaches kFSampleMargin times
// the sample's share of the budget (or the lowest sampled positive bin).
// Any floor is correct -- the cut kernel checks that enough bounds lie above
// it -- a low one only costs histogram work.
__global__ void build_floor_kernel(FastWs fw, long long count, double sample_frac) {
    const int u = blockIdx.x;
    if (threadIdx.x != 0) return;
    const int* h = fw.histS + (int64_t)u * kFBins;
    const double target = fmax(1.0, kFSampleMargin * (double)count * sample_frac);
    double acc = 0.0;
    int b = kFBins - 1, lowest = 0;
    int fb = -1;
    for (; b >= 0; --b) {
        if (h[b]) lowest = b;
        acc += h[b];
        if (fb < 0 && acc >= target) fb = b;
    }
    fw.floor_bin[u] = fb >= 0 ? fb : lowest;
}

// Per unit: the bins holding the count-th largest lower / upper bound,
// inside the window above the floor.  Fewer than `count` bounds at or above
// the floor (a floor placed too high, or fewer positive activations than the
// budget -- core.py:23's all-positives case), or a cut in the window's top
// bin (which merges everything above), leave the threshold unbracketed: the
// exact path runs instead.
__global__ void build_fast_cut_kernel(FastWs fw, long long count, int* __restrict__ status) {
    const int u = blockIdx.x;
    if (threadIdx.x != 0) return;
    const int fb = fw.floor_bin[u];
    bool bad = false;
    for (int which = 0; which < 2; ++which) {
        const int* h = (which ? fw.histU : fw.histL) + (int64_t)u * kFWin;
        long long above = 0;
        int b = kFWin - 1;
        for (; b >= 0; --b) {
            if (above + h[b] >= count) break;
            above += h[b];
        }
        if (b < 0 || b == kFWin - 1) bad = true;
        (which ? fw.cutU : fw.cutL)[u] = fb + b;
    }
    if (bad) {
        atomicOr(status, PK_STATUS_NEEDS_EXACT);
        fw.cutL[u] = INT32_MAX;
        fw.cutU[u] = INT32_MAX;
    }
}

// Classification of the candidates kept by the histogram pass (every entry
// whose upper bound reaches the floor): not a member if U is below the lower
// bounds' cut; a member if L is above the upper bounds' cut; otherwise the
// exact value decides.  Appends are aggregated per warp.
__global__ void __launch_bounds__(256)
build_classify_kernel(int F, BuildWs ws, FastWs fw, int* __restrict__ lens, int* __restrict__ status) {
    const int u = blockIdx.y, lane = threadIdx.x & 31;
    const int n = (int)min((int64_t)fw.n_cand[u], fw.acap);
    const int cutL = fw.cutL[u], cutU = fw.cutU[u];
    if (cutL == INT32_MAX) return;  // the exact path runs instead
    const int stride = gridDim.x * blockDim.x;
    for (int base0 = blockIdx.x * blockDim.x; base0 < n; base0 += stride) {
        const int i = base0 + threadIdx.x;
        bool mem = false, amb = false;
        long long flat = 0;
        if (i < n) {
            const float2 hl = fw.cand_hl[(int64_t)u * fw.acap + i];
            flat = fw.cand_flat[(int64_t)u * fw.acap + i];
            const float hi = hl.x, lo = hl.y;
            const bool out = !(hi > 0.f) || fbin(hi) < cutL;
            mem = !out && lo > 0.f && fbin(lo) > cutU;
            amb = !out && !mem;
        }
        const unsigned mm = __ballot_sync(0xffffffffu, mem);
        if (mm) {
            const int lead = __ffs(mm) - 1;
            int base = 0;
            if (lane == lead) base = atomicAdd(&ws.n_members[u], __popc(mm));
            base = __shfl_sync(0xffffffffu, base, lead);
            if (mem) {
                const int at = base + __popc(mm & lane_below());
                if (at < ws.mcap) {
                    ws.members[(int64_t)u * ws.mcap + at] = flat;
                    atomicAdd(&lens[(int64_t)u * F + (int)(flat % F)], 1);
                } else {
                    atomicOr(status, PK_STATUS_MEMBERS_FULL);
                }
            }
        }
        const unsigned am = __ballot_sync(0xffffffffu, amb);
        if (am) {
            const int lead = __ffs(am) - 1;
            int base = 0;
            if (lane == lead) base = atomicAdd(&fw.n_amb[u], __popc(am));
            base = __shfl_sync(0xffffffffu, base, lead);
            if (amb) {
                const int at = base + __popc(am & lane_below());
                if (at < fw.acap) fw.amb[(int64_t)u * fw.acap + at] = flat;
                else atomicOr(status, PK_STATUS_BOUNDARY_FULL);
            }
        }
    }
}

// Exact activations of the undecided entries (sequential FMA over d, as the
// reference); entries the exact value decides go straight to members or are
// dropped, the rest become 64-bit boundary keys (value descending within the
// band, flat index ascending).  Key and W rows are read 32 values at a time
// with 16-byte loads when the key rows are 16-byte aligned.
template <typename T>
__device__ __forceinline__ void load32(const T* p, bool vec, float (&x)[32]) {
    if constexpr (sizeof(T) == 2) {
        if (vec) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint4 r = reinterpret_cast<const uint4*>(p)[q];
                const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 f = __bfloat1622float2(b[j]);
                    x[8 * q + 2 * j] = f.x;
                    x[8 * q + 2 * j + 1] = f.y;
                }
            }
            return;
        }
    } else {
        if (vec) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 r = reinterpret_cast<const float4*>(p)[q];
                x[4 * q] = r.x; x[4 * q + 1] = r.y; x[4 * q + 2] = r.z; x[4 * q + 3] = r.w;
            }
            return;
        }
    }
#pragma unroll
    for (int c = 0; c < 32; ++c) x[c] = load_f(p, c);
}

template <typename T>
__global__ void __launch_bounds__(256)
build_exact_kernel(const T* __restrict__ keys, int64_t unit_stride, int64_t row_stride,
                   const float* __restrict__ center, float key_scale, const float* __restrict__ W,
                   const float* __restrict__ bias, int F, BuildWs ws, FastWs fw, int* __restrict__ lens,
                   int* __restrict__ status, int vec_keys, long long flat_base) {
    __shared__ float cs[kBD];
    const int u = blockIdx.y;
    for (int c = threadIdx.x; c < kBD; c += blockDim.x) cs[c] = center[(int64_t)u * kBD + c];
    __syncthreads();
    const int n = (int)min((int64_t)fw.n_amb[u], fw.acap);
    const int cutL = fw.cutL[u], cutU = fw.cutU[u];
    if (cutL == INT32_MAX) return;  // the exact path runs instead
    const bool unit_scale = key_scale == 1.0f;
    const uint32_t hi_bits = cutU >= 0 ? ((uint32_t)(cutU + 1) << kFShift) : 0x7F800000u;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const long long flat = fw.amb[(int64_t)u * fw.acap + i];
        const long long t = flat / F;
        const int f = (int)(flat % F);
        const T* krow = keys + (int64_t)u * unit_stride + t * row_stride;
        const float4* wrow = reinterpret_cast<const float4*>(W + (int64_t)f * kBD);
        float acc = 0.f;
#pragma unroll 1
        for (int c0 = 0; c0 < kBD; c0 += 32) {
            float kv[32];
            load32(krow + c0, vec_keys != 0, kv);
            float4 wv[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) wv[q] = wrow[c0 / 4 + q];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float w4[4] = {wv[q].x, wv[q].y, wv[q].z, wv[q].w};
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int c = 4 * q + r;
                    const float dlt = __fsub_rn(kv[c], cs[c0 + c]);
                    const float x = unit_scale ? dlt : __fdiv_rn(dlt, key_scale);
                    acc = fmaf(x, w4[r], acc);
                }
            }
        }
        const float y = __fadd_rn(acc, bias[f]);
        if (!(y > 0.f) || fbin(y) < cutL) continue;                 // below the threshold
        if (cutU < 0 || fbin(y) > cutU) {                           // above it (or all positives count)
            const int at = atomicAdd(&ws.n_members[u], 1);
            if (at < ws.mcap) {
                ws.members[(int64_t)u * ws.mcap + at] = flat;
                atomicAdd(&lens[(int64_t)u * F + f], 1);
            } else {
                atomicOr(status, PK_STATUS_MEMBERS_FULL);
            }
            continue;
        }
        // Boundary keys carry the flat index in the whole sequence (flat_base:
        // the shard's first token times F; 0 unsharded) so that ties order
        // the same across shards.
        const uint32_t span = hi_bits - __float_as_uint(y);          // > 0: y lies below the band's top
        const long long gflat = flat + flat_base;
        if (span >= (1u << 28) || gflat >= (1ll << 36)) {
            atomicOr(status, PK_STATUS_NEEDS_EXACT);
            continue;
        }
        const int at = atomicAdd(&ws.n_boundary[u], 1);
        if (at < ws.bcap)
            ws.boundary[(int64_t)u * ws.bcap + at] =
                (long long)(((unsigned long long)span << 36) | (unsigned long long)gflat);
        else
            atomicOr(status, PK_STATUS_BOUNDARY_FULL);
    }
}

// need = count - members so far (the boundary supplies the rest); cut >= 0
// so that the resolve kernel runs.
__global__ void build_fast_need_kernel(BuildWs ws, FastWs fw, long long count) {
    const int u = blockIdx.x;
    if (threadIdx.x != 0) return;
    const long long have = ws.n_members[u];
    ws.need[u] = count - have;
    ws.cut[u] = fw.cutU[u] >= 0 ? 0 : -1;  // all positives: nothing to resolve
}

// Resolve with the fast keys: the `need` smallest keys of the boundary are
// members; key bits [36, 64) hold the value's distance below the band top.
__global__ void __launch_bounds__(1024)
build_fast_resolve_kernel(BuildWs ws, int F, int* __restrict__ lens, int* __restrict__ status) {
    const int u = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
    __shared__ int hist[256];
    __shared__ unsigned long long s_prefix;
    __shared__ long long s_need;
    const long long need0 = ws.need[u];
    const int nb = ws.n_boundary[u];
    if (ws.cut[u] < 0 || need0 <= 0 || nb > ws.bcap) return;
    if (need0 > nb) {
        // The bounds should always leave enough candidates: flag, never guess.
        if (tid == 0) atomicOr(status, PK_STATUS_NEEDS_EXACT);
        return;
    }
    const long long* B = ws.boundary + (int64_t)u * ws.bcap;
    unsigned long long prefix = ~0ull;
    if (need0 < nb) {
        unsigned long long pre = 0, pmask = 0;
        long long need = need0;
        for (int pass = 0; pass < 8; ++pass) {
            const int shift = 56 - 8 * pass;
            for (int i = tid; i < 256; i += nt) hist[i] = 0;
            __syncthreads();
            for (int i = tid; i < nb; i += nt) {
                const unsigned long long kk = (unsigned long long)B[i];
                if ((kk & pmask) == pre) atomicAdd(&hist[(kk >> shift) & 255ull], 1);
            }
            __syncthreads();
            if (tid == 0) {
                long long acc = 0;
                int dgt = 0;
                for (; dgt < 256; ++dgt) {
                    if (acc + hist[dgt] >= need) break;
                    acc += hist[dgt];
                }
                s_prefix = pre | ((unsigned long long)dgt << shift);
                s_need = need - acc;
            }
            __syncthreads();
            pre = s_prefix;
            pmask |= 0xFFull << shift;
            need = s_need;
            __syncthreads();
        }
        prefix = pre;
    }
    for (int i = tid; i < nb; i += nt) {
        const unsigned long long kk = (unsigned long long)B[i];
        if (kk <= prefix) {
            const long long flat = (long long)(kk & ((1ull << 36) - 1));
            const int at = atomicAdd(&ws.n_members[u], 1);
            if (at < ws.mcap) {
                ws.members[(int64_t)u * ws.mcap + at] = flat;
                atomicAdd(&lens[(int64_t)u * F + (int)(flat % F)], 1);
            } else {
                atomicOr(status, PK_STATUS_MEMBERS_FULL);
            }
        }
    }
}

// Sequence-sharded resolve: the boundary keys of every shard, gathered as
// keys[P, U, key_cap] with counts[P, U] (global flat indices), and the
// unit's need = global count - members over all shards.  Every shard runs
// the same radix select over the same keys (so every shard finds the same
// threshold key) and keeps the keys at or below it whose flat index lies in
// its own range [flat_lo, flat_hi).
__global__ void __launch_bounds__(1024)
build_shard_resolve_kernel(const long long* __restrict__ keys, const int* __restrict__ counts, int P, int64_t key_cap,
                           const long long* __restrict__ need_in, long long flat_lo, long long flat_hi, BuildWs ws,
                           FastWs fw, int F, int* __restrict__ lens, int* __restrict__ status) {
    const int u = blockIdx.x, tid = threadIdx.x, nt = blockDim.x, U = gridDim.x;
    __shared__ int hist[256];
    __shared__ unsigned long long s_prefix;
    __shared__ long long s_need;
    if (fw.cutL[u] == INT32_MAX || fw.cutU[u] < 0) return;   // flagged, or all positives (nothing to resolve)
    const long long need0 = need_in[u];
    if (need0 <= 0) return;
    long long total = 0;
    for (int r = 0; r < P; ++r) total += min((int64_t)counts[(int64_t)r * U + u], key_cap);
    if (need0 > total) {
        if (tid == 0) atomicOr(status, PK_STATUS_NEEDS_EXACT);
        return;
    }
    const int64_t nslots = (int64_t)P * key_cap;
    auto key_of = [&](int64_t i, unsigned long long& kk) -> bool {
        const int r = (int)(i / key_cap);
        const int64_t j = i % key_cap;
        if (j >= counts[(int64_t)r * U + u]) return false;
        kk = (unsigned long long)keys[((int64_t)r * U + u) * key_cap + j];
        return true;
    };
    unsigned long long prefix = ~0ull;
    if (need0 < total) {
        unsigned long long pre = 0, pmask = 0;
        long long need = need0;
        for (int pass = 0; pass < 8; ++pass) {
            const int shift = 56 - 8 * pass;
            for (int i = tid; i < 256; i += nt) hist[i] = 0;
            __syncthreads();
            for (int64_t i = tid; i < nslots; i += nt) {
                unsigned long long kk;
                if (key_of(i, kk) && (kk & pmask) == pre) atomicAdd(&hist[(kk >> shift) & 255ull], 1);
            }
            __syncthreads();
            if (tid == 0) {
                long long acc = 0;
                int dgt = 0;
                for (; dgt < 256; ++dgt) {
                    if (acc + hist[dgt] >= need) break;
                    acc += hist[dgt];
                }
                s_prefix = pre | ((unsigned long long)dgt << shift);
                s_need = need - acc;
            }
            __syncthreads();
            pre = s_prefix;
            pmask |= 0xFFull << shift;
            need = s_need;
            __syncthreads();
        }
        prefix = pre;
    }
    for (int64_t i = tid; i < nslots; i += nt) {
        unsigned long long kk;
        if (!key_of(i, kk) || kk > prefix) continue;
        const long long gflat = (long long)(kk & ((1ull << 36) - 1));
        if (gflat < flat_lo || gflat >= flat_hi) continue;
        const long long flat = gflat - flat_lo;
        const int at = atomicAdd(&ws.n_members[u], 1);
        if (at < ws.mcap) {
            ws.members[(int64_t)u * ws.mcap + at] = flat;
            atomicAdd(&lens[(int64_t)u * F + (int)(flat % F)], 1);
        } else {
            atomicOr(status, PK_STATUS_MEMBERS_FULL);
        }
    }
}

__global__ void set_ints_kernel(int* __restrict__ out, int a, int b) {
    out[0] = a;
    out[1] = b;
}

// Chunk sums of the key-center cascade (center_kernel) for a shard of a
// longer sequence: lp comes from the whole sequence's length, and the shard
// holds whole chunks; out[u, ch, c] = the cascade's sum of chunk ch.
template <typename T>
__global__ void __launch_bounds__(1024)
center_chunks_kernel(const T* __restrict__ keys, int64_t unit_stride, int64_t row_stride, int64_t nchunks, int lp,
                     int d, float* __restrict__ out) {
    const int u = blockIdx.y, lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int c = blockIdx.x * 32 + lane;
    const int64_t step = (int64_t)1 << lp, chunk = step * step * step;
    if (c >= d) return;
    for (int64_t ch = w; ch < nchunks; ch += nw) {
        int64_t i = ch * chunk;
        float a2 = 0.f;
        for (int64_t g = 0; g < step; ++g) {
            float a1 = 0.f;
            for (int64_t b = 0; b < step; ++b) {
                float a0 = 0.f;
                for (int64_t s = 0; s < step; ++s, ++i) a0 = __fadd_rn(a0, key_at(keys, unit_stride, row_stride, u, i, c));
                a1 = __fadd_rn(a1, a0);
            }
            a2 = __fadd_rn(a2, a1);
        }
        out[((int64_t)u * nchunks + ch) * d + c] = a2;
    }
}

// The sampled floor's parameters for a shard of N keys: about 64 token
// blocks and every ft_stride-th feature tile (see run_encode_select_fast).
TileSample sample_plan(int64_t N, int F, long long count, int* nsample_out) {
    const int nblocks = (int)((N + 127) / 128);
    const int nft = (F + 255) / 256;
    TileSample smp;
    smp.tb_stride = nblocks > 64 ? nblocks / 64 : 1;
    const int nsample = (nblocks + smp.tb_stride - 1) / smp.tb_stride;
    const double tok_frac = fmin(1.0, (double)nsample * 128.0 / (double)N);
    const double want = kFSampleMargin * (double)count * tok_frac / 8192.0;
    smp.ft_stride = want >= (double)nft ? nft : (want >= 1.0 ? (int)want : 1);
    *nsample_out = nsample;
    return smp;
}

// A tensor map over W_half [F, d] fp16 (rows of 256 bytes, 16-byte aligned):
// boxes of 64 x 256 with the 128-byte swizzle the MMA's K-major descriptors
// read.  Encoded through the driver entry point (no link to libcuda);
// use_map stays 0 when the entry point or the encode is refused, and the
// kernels then copy build_tiles_kernel's images instead.
static WSource make_wsource(const __half* Wh, int F) {
    WSource w;
    memset(&w, 0, sizeof(w));
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    static bool looked_up = false;
    if (!looked_up) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
        cudaGetLastError();
        looked_up = true;
    }
    if (!encode || !Wh || (uintptr_t)Wh % 16 || F < 1) return w;
    const cuuint64_t dims[2] = {(cuuint64_t)kBD, (cuuint64_t)F};
    const cuuint64_t strides[1] = {(cuuint64_t)kBD * sizeof(__half)};
    const cuuint32_t box[2] = {64, (cuuint32_t)kTcFeat};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode(&w.map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void*)Wh, dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    w.use_map = r == CUDA_SUCCESS ? 1 : 0;
    return w;
}

template <typename T>
int run_encode_select_fast(const T* keys, int64_t unit_stride, int64_t row_stride, int64_t N, const float* center,
                           float key_scale, const float* W, const __half* Wh, const float* wn,
                           const float* b, int U, int F, long long count, BuildWs ws, FastWs fw, int* lens,
                           int* status, cudaStream_t st) {
    const int nblocks = (int)((N + 127) / 128);
    const int nft = (F + kTcFeat - 1) / kTcFeat;
    // Floor sample: about 64 token blocks and every ft_stride-th feature
    // tile, the stride chosen so that the sample expects about 8192 entries
    // above the floor (relative noise ~1%, against the floor's 2x margin).
    int nsample = 0;
    const TileSample smp = sample_plan(N, F, count, &nsample);
    const double frac = fmin(1.0, (double)nsample * 128.0 / (double)N) / (double)smp.ft_stride;
    const TileSample none = {1, 1};
    const WSource wsrc = make_wsource(Wh, F);
    build_tiles_kernel<<<nft, 256, 0, st>>>(Wh, wn, b, F, fw.tiles, fw.sides, status, !wsrc.use_map);
    PK_CHECK_LAUNCH();
    cudaFuncSetAttribute(build_tile_tc_kernel<0, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, tc_smem(0));
    cudaFuncSetAttribute(build_tile_tc_kernel<1, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, tc_smem(1));
    build_tile_tc_kernel<0, T><<<dim3(nsample, U), kTcThreads, tc_smem(0), st>>>(
        keys, unit_stride, row_stride, N, center, key_scale, F, fw, smp, status, wsrc);
    PK_CHECK_LAUNCH();
    build_floor_kernel<<<U, 32, 0, st>>>(fw, count, frac);
    PK_CHECK_LAUNCH();
    build_tile_tc_kernel<1, T><<<dim3(nblocks, U), kTcThreads, tc_smem(1), st>>>(
        keys, unit_stride, row_stride, N, center, key_scale, F, fw, none, status, wsrc);
    PK_CHECK_LAUNCH();
    build_fast_cut_kernel<<<U, 32, 0, st>>>(fw, count, status);
    PK_CHECK_LAUNCH();
    build_classify_kernel<<<dim3(256, U), 256, 0, st>>>(F, ws, fw, lens, status);
    PK_CHECK_LAUNCH();
    const size_t esz = sizeof(T);
    const int vec = ((uint64_t)keys % 16 == 0 && (unit_stride * (int64_t)esz) % 16 == 0 &&
                     (row_stride * (int64_t)esz) % 16 == 0) ? 1 : 0;
    build_exact_kernel<T><<<dim3(512, U), 256, 0, st>>>(keys, unit_stride, row_stride, center, key_scale, W, b, F,
                                                        ws, fw, lens, status, vec, 0ll);
    PK_CHECK_LAUNCH();
    build_fast_need_kernel<<<U, 32, 0, st>>>(ws, fw, count);
    PK_CHECK_LAUNCH();
    build_fast_resolve_kernel<<<U, 1024, 0, st>>>(ws, F, lens, status);
    PK_CHECK_LAUNCH();
    return PK_OK;
}

int sort_buckets(int* ids, int64_t ids_stride, const int* offsets, const int* start, const int* cnt, int U, int F,
                 int* status, cudaStream_t st) {
    sort_buckets_warp_kernel<<<dim3((F + 7) / 8, U), 256, 0, st>>>(ids, ids_stride, offsets, start, cnt, F);
    PK_CHECK_LAUNCH();
    const int smem = kSortBigCap * (int)sizeof(int);
    cudaFuncSetAttribute(sort_buckets_big_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    sort_buckets_big_kernel<<<dim3(F < 64 ? F : 64, U), 1024, smem, st>>>(ids, ids_stride, offsets, start, cnt, F,
                                                                          status);
    PK_CHECK_LAUNCH();
    return PK_OK;
}

}  // namespace pk

using namespace pk;

extern "C" int pk_key_center(uint64_t keys, int dtype, int64_t unit_stride, int64_t row_stride, int U, int64_t N,
                             int d, uint64_t center, uint64_t stream) {
    if (U < 1 || N < 1 || d < 1 || !keys || !center || row_stride < d) return PK_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    // 32 columns per CTA, 32 warps share the cascade's independent chunks.
    int lp = ceil_log2_i64(N) / 4;
    if (lp < 4) lp = 4;
    const int64_t nchunks = N >> (3 * lp);
    const size_t smem = (size_t)(nchunks > 0 ? nchunks : 1) * 32 * sizeof(float);
    if (smem > 200 * 1024) return PK_ERR_UNSUPPORTED;
    dim3 grid((d + 31) / 32, U);
    if (dtype == PK_BF16) {
        cudaFuncSetAttribute(center_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        center_kernel<__nv_bfloat16><<<grid, 1024, smem, st>>>((const __nv_bfloat16*)keys, unit_stride, row_stride, N,
                                                               d, (float*)center);
    } else if (dtype == PK_F32) {
        cudaFuncSetAttribute(center_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        center_kernel<float><<<grid, 1024, smem, st>>>((const float*)keys, unit_stride, row_stride, N, d,
                                                       (float*)center);
    } else {
        return PK_ERR_ARG;
    }
    PK_CHECK_LAUNCH();
    return PK_OK;
}

extern "C" int64_t pk_build_ids_capacity(int64_t N, int F, int key_mean, float slack_frac, int slack_min) {
    const int64_t members = N * (int64_t)key_mean;
    return members + (int64_t)ceil((double)members * slack_frac) + (int64_t)F * (slack_min + 1) + 64;
}

extern "C" size_t pk_build_workspace_bytes(int U, int64_t N, int F, int key_mean, int64_t boundary_capacity) {
    const int64_t mcap = N * (int64_t)key_mean;
    const int64_t bcap = boundary_capacity > 0 ? boundary_capacity : 1;
    return carve_bytes(U, F, mcap > 0 ? mcap : 1, bcap) + fast_bytes(U, bcap, F);
}

extern "C" int pk_build_index(uint64_t keys, int dtype, int64_t unit_stride, int64_t row_stride, uint64_t center,
                              float key_scale, uint64_t w_enc, uint64_t b_enc, uint64_t w_half, uint64_t w_norm,
                              int U, int64_t N, int d, int F,
                              int key_mean, int64_t token_base, float slack_frac, int slack_min, uint64_t offsets,
                              uint64_t lens, uint64_t ids, int64_t ids_stride, int64_t boundary_capacity,
                              uint64_t workspace, uint64_t workspace_bytes, uint64_t status, uint64_t stream) {
    if (U < 1 || N < 1 || F < 1 || key_mean < 1 || !(key_scale > 0.f) || slack_frac < 0.f || slack_min < 0)
        return PK_ERR_ARG;
    if (d != kBD) return PK_ERR_UNSUPPORTED;
    if (!keys || !center || !w_enc || !b_enc || !offsets || !lens || !ids || !workspace || !status) return PK_ERR_ARG;
    if ((long long)N * F >= (1ll << 40) || N > INT32_MAX || token_base + N > INT32_MAX || row_stride < d)
        return PK_ERR_ARG;
    if (boundary_capacity < 1) return PK_ERR_ARG;
    if (ids_stride < pk_build_ids_capacity(N, F, key_mean, slack_frac, slack_min)) return PK_ERR_ARG;
    if (workspace_bytes < pk_build_workspace_bytes(U, N, F, key_mean, boundary_capacity)) return PK_ERR_WORKSPACE;
    cudaStream_t st = (cudaStream_t)stream;
    const int64_t mcap = N * (int64_t)key_mean;
    BuildWs ws = carve((void*)workspace, U, F, mcap, boundary_capacity);
    void* fbase = (char*)workspace + carve_bytes(U, F, mcap, boundary_capacity);
    FastWs fw = carve_fast(fbase, U, boundary_capacity, F);
    cudaMemsetAsync((void*)workspace, 0, counters_bytes(U, F), st);
    cudaMemsetAsync(fbase, 0, fast_counters_bytes(U), st);
    cudaMemsetAsync((void*)lens, 0, (size_t)U * F * sizeof(int), st);
    const long long count = (long long)N * key_mean;
    int rc;
    const bool fast = w_half && w_norm;
    if (fast && (w_half % 16)) return PK_ERR_ARG;   // 16-byte row loads
    if (fast && dtype == PK_BF16)
        rc = run_encode_select_fast((const __nv_bfloat16*)keys, unit_stride, row_stride, N, (const float*)center,
                                    key_scale, (const float*)w_enc, (const __half*)w_half,
                                    (const float*)w_norm, (const float*)b_enc, U, F, count, ws, fw, (int*)lens,
                                    (int*)status, st);
    else if (fast && dtype == PK_F32)
        rc = run_encode_select_fast((const float*)keys, unit_stride, row_stride, N, (const float*)center, key_scale,
                                    (const float*)w_enc, (const __half*)w_half, (const float*)w_norm,
                                    (const float*)b_enc, U, F, count, ws, fw, (int*)lens, (int*)status, st);
    else if (dtype == PK_BF16)
        rc = run_encode_select((const __nv_bfloat16*)keys, unit_stride, row_stride, N, (const float*)center, key_scale,
                               (const float*)w_enc, (const float*)b_enc, U, F, count, ws, (int*)lens, (int*)status, st);
    else if (dtype == PK_F32)
        rc = run_encode_select((const float*)keys, unit_stride, row_stride, N, (const float*)center, key_scale,
                               (const float*)w_enc, (const float*)b_enc, U, F, count, ws, (int*)lens, (int*)status, st);
    else
        return PK_ERR_ARG;
    if (rc) return rc;
    build_offsets_kernel<<<U, 1024, 0, st>>>((const int*)lens, F, slack_frac, slack_min, (int*)offsets, ids_stride,
                                             (int*)status);
    PK_CHECK_LAUNCH();
    build_scatter_kernel<<<dim3(64, U), 256, 0, st>>>(ws, F, (const int*)offsets, (int*)ids, ids_stride,
                                                       (long long)token_base);
    PK_CHECK_LAUNCH();
    return sort_buckets((int*)ids, ids_stride, (const int*)offsets, nullptr, (const int*)lens, U, F, (int*)status, st);
}

extern "C" int pk_summarize(uint64_t keys, int dtype, int64_t unit_stride, int64_t row_stride, uint64_t offsets,
                            uint64_t lens, uint64_t ids, int64_t ids_stride, int U, int d, int F, uint64_t mean,
                            uint64_t var, uint64_t stream) {
    if (U < 1 || F < 1 || !keys || !offsets || !lens || !ids || !mean || !var) return PK_ERR_ARG;
    if (d != kBD) return PK_ERR_UNSUPPORTED;
    cudaStream_t st = (cudaStream_t)stream;
    dim3 grid((F + 7) / 8, U);
    if (dtype == PK_BF16)
        summarize_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)keys, unit_stride, row_stride,
                                                             (const int*)offsets, nullptr, (const int*)lens,
                                                             (const int*)ids, ids_stride, 0, F, (float*)mean,
                                                             (float*)var);
    else if (dtype == PK_F32)
        summarize_kernel<float><<<grid, 256, 0, st>>>((const float*)keys, unit_stride, row_stride, (const int*)offsets,
                                                     nullptr, (const int*)lens, (const int*)ids, ids_stride, 0, F,
                                                     (float*)mean, (float*)var);
    else
        return PK_ERR_ARG;
    PK_CHECK_LAUNCH();
    return PK_OK;
}

// Folds one block's bucket moments into a running state with the
// parallel formula of core.py:194-199 (the append_index merge), in place:
// mean/var[U, F, d] of the state (counts_a[U, F]) absorb mean_b/var_b of a
// block with counts_b.  The sequence-sharded index folds its shards' moments
// in token order with it.
extern "C" int pk_merge_moments(uint64_t counts_a, uint64_t mean, uint64_t var, uint64_t counts_b, uint64_t mean_b,
                                uint64_t var_b, int U, int F, int d, uint64_t stream) {
    if (U < 1 || F < 1 || !counts_a || !mean || !var || !counts_b || !mean_b || !var_b) return PK_ERR_ARG;
    if (d != kBD) return PK_ERR_UNSUPPORTED;
    merge_moments_kernel<<<dim3((unsigned)(((int64_t)F * kBD + 255) / 256), U), 256, 0, (cudaStream_t)stream>>>(
        (const int*)counts_a, (const int*)counts_b, F, (float*)mean, (float*)var, (const float*)mean_b,
        (const float*)var_b, nullptr);
    PK_CHECK_LAUNCH();
    return PK_OK;
}

extern "C" size_t pk_append_workspace_bytes(int U, int64_t n_new, int d, int F, int key_mean,
                                            int64_t boundary_capacity) {
    const int64_t mcap = n_new * (int64_t)key_mean;
    const int64_t bcap = boundary_capacity > 0 ? boundary_capacity : 1;
    const size_t base = carve_bytes(U, F, mcap > 0 ? mcap : 1, bcap) + fast_bytes(U, bcap, F);
    // + new-block counts [U, F] + new-block moments [2, U, F, d]
    return base + align256((size_t)U * F * 4) + 2 * align256((size_t)U * F * d * 4);
}

extern "C" int pk_append_index(uint64_t new_keys, int dtype, int64_t unit_stride, int64_t row_stride, int64_t n_new,
                               uint64_t center, float key_scale, uint64_t w_enc, uint64_t b_enc, uint64_t w_half,
                               uint64_t w_norm, int U, int d, int F,
                               int key_mean, int64_t history, uint64_t offsets, uint64_t lens, uint64_t ids,
                               int64_t ids_stride, uint64_t mean, uint64_t var, int64_t boundary_capacity,
                               uint64_t workspace, uint64_t workspace_bytes, uint64_t status, uint64_t stream) {
    if (U < 1 || n_new < 1 || F < 1 || key_mean < 1 || !(key_scale > 0.f) || history < 0) return PK_ERR_ARG;
    if (d != kBD) return PK_ERR_UNSUPPORTED;
    if (!new_keys || !center || !w_enc || !b_enc || !offsets || !lens || !ids || !workspace || !status)
        return PK_ERR_ARG;
    if ((mean == 0) != (var == 0)) return PK_ERR_ARG;
    if ((long long)n_new * F >= (1ll << 40) || history + n_new > INT32_MAX || row_stride < d) return PK_ERR_ARG;
    if (boundary_capacity < 1) return PK_ERR_ARG;
    if (workspace_bytes < pk_append_workspace_bytes(U, n_new, d, F, key_mean, boundary_capacity))
        return PK_ERR_WORKSPACE;
    cudaStream_t st = (cudaStream_t)stream;
    const int64_t mcap = n_new * (int64_t)key_mean;
    BuildWs ws = carve((void*)workspace, U, F, mcap, boundary_capacity);
    void* fbase = (char*)workspace + carve_bytes(U, F, mcap, boundary_capacity);
    FastWs fw = carve_fast(fbase, U, boundary_capacity, F);
    char* extra = (char*)fbase + fast_bytes(U, boundary_capacity, F);
    int* cnt_new = (int*)extra;
    float* mean_new = (float*)(extra + align256((size_t)U * F * 4));
    float* var_new = (float*)(extra + align256((size_t)U * F * 4) + align256((size_t)U * F * d * 4));
    cudaMemsetAsync((void*)workspace, 0, counters_bytes(U, F), st);
    cudaMemsetAsync(cnt_new, 0, (size_t)U * F * 4, st);
    cudaMemsetAsync(fbase, 0, fast_counters_bytes(U), st);
    const long long count = (long long)n_new * key_mean;
    int rc;
    const bool fast = w_half && w_norm;
    if (fast && (w_half % 16)) return PK_ERR_ARG;   // 16-byte row loads
    if (fast && dtype == PK_BF16)
        rc = run_encode_select_fast((const __nv_bfloat16*)new_keys, unit_stride, row_stride, n_new,
                                    (const float*)center, key_scale, (const float*)w_enc,
                                    (const __half*)w_half, (const float*)w_norm, (const float*)b_enc, U, F,
                                    count, ws, fw, cnt_new, (int*)status, st);
    else if (fast && dtype == PK_F32)
        rc = run_encode_select_fast((const float*)new_keys, unit_stride, row_stride, n_new, (const float*)center,
                                    key_scale, (const float*)w_enc, (const __half*)w_half,
                                    (const float*)w_norm, (const float*)b_enc, U, F, count, ws, fw, cnt_new,
                                    (int*)status, st);
    else if (dtype == PK_BF16)
        rc = run_encode_select((const __nv_bfloat16*)new_keys, unit_stride, row_stride, n_new, (const float*)center,
                               key_scale, (const float*)w_enc, (const float*)b_enc, U, F, count, ws, cnt_new,
                               (int*)status, st);
    else if (dtype == PK_F32)
        rc = run_encode_select((const float*)new_keys, unit_stride, row_stride, n_new, (const float*)center, key_scale,
                               (const float*)w_enc, (const float*)b_enc, U, F, count, ws, cnt_new, (int*)status, st);
    else
        return PK_ERR_ARG;
    if (rc) return rc;
    // An incomplete member list (boundary full, or bounds that need the exact
    // path) must not be committed.
    status_gate_kernel<<<1, 32, 0, st>>>((const int*)status, ws.flag);
    PK_CHECK_LAUNCH();
    dim3 g2((F + 255) / 256, U);
    append_check_kernel<<<g2, 256, 0, st>>>((const int*)offsets, (const int*)lens, cnt_new, F, ws.flag);
    PK_CHECK_LAUNCH();
    append_scatter_kernel<<<dim3(64, U), 256, 0, st>>>(ws, F, (const int*)offsets, (const int*)lens, (int*)ids,
                                                        ids_stride, (long long)history);
    PK_CHECK_LAUNCH();
    append_gate_kernel<<<256, 256, 0, st>>>(ws.flag, cnt_new, (int64_t)U * F);
    PK_CHECK_LAUNCH();
    // Sort only the appended tail of each bucket (it follows the old ids,
    // which are all smaller).
    rc = sort_buckets((int*)ids, ids_stride, (const int*)offsets, (const int*)lens, cnt_new, U, F, (int*)status, st);
    if (rc) return rc;
    if (mean) {
        // New-block moments from the appended tails, then the merge.
        if (dtype == PK_BF16)
            summarize_kernel<__nv_bfloat16><<<dim3((F + 7) / 8, U), 256, 0, st>>>(
                (const __nv_bfloat16*)new_keys, unit_stride, row_stride, (const int*)offsets, (const int*)lens,
                cnt_new, (const int*)ids, ids_stride, (long long)history, F, mean_new, var_new);
        else
            summarize_kernel<float><<<dim3((F + 7) / 8, U), 256, 0, st>>>(
                (const float*)new_keys, unit_stride, row_stride, (const int*)offsets, (const int*)lens, cnt_new,
                (const int*)ids, ids_stride, (long long)history, F, mean_new, var_new);
        PK_CHECK_LAUNCH();
        merge_moments_kernel<<<dim3((unsigned)(((int64_t)F * kBD + 255) / 256), U), 256, 0, st>>>(
            (const int*)lens, cnt_new, F, (float*)mean, (float*)var, mean_new, var_new, ws.flag);
        PK_CHECK_LAUNCH();
    }
    append_commit_kernel<<<g2, 256, 0, st>>>(ws.flag, (int*)lens, cnt_new, F, (int*)status);
    PK_CHECK_LAUNCH();
    return PK_OK;
}

// ---------------------------------------------------------------------------
// Sequence-sharded build with the exact global BatchTopK.
// ---------------------------------------------------------------------------

extern "C" size_t pk_build_shard_workspace_bytes(int U, int64_t N, int F, int64_t member_capacity,
                                                  int64_t boundary_capacity) {
    const int64_t mcap = member_capacity > 0 ? member_capacity : 1;
    const int64_t bcap = boundary_capacity > 0 ? boundary_capacity : 1;
    (void)N;
    return carve_bytes(U, F, mcap, bcap) + fast_bytes(U, bcap, F);
}

extern "C" int pk_build_shard_layout(int U, int64_t N, int F, int64_t member_capacity, int64_t boundary_capacity,
                                     uint64_t out) {
    if (U < 1 || N < 1 || F < 1 || member_capacity < 1 || boundary_capacity < 1 || !out) return PK_ERR_ARG;
    const int64_t mcap = member_capacity;
    const size_t fbase = carve_bytes(U, F, mcap, boundary_capacity);
    char* zero = nullptr;
    BuildWs ws = carve(zero, U, F, mcap, boundary_capacity);
    FastWs fw = carve_fast(zero + fbase, U, boundary_capacity, F);
    int64_t* o = (int64_t*)out;
    o[0] = (int64_t)((char*)fw.histS - zero);
    o[1] = (int64_t)((char*)fw.histL - zero);
    o[2] = (int64_t)((char*)fw.histU - zero);
    o[3] = (int64_t)((char*)ws.n_members - zero);
    o[4] = (int64_t)((char*)ws.n_boundary - zero);
    o[5] = (int64_t)((char*)ws.boundary - zero);
    o[6] = (int64_t)((char*)fw.cutU - zero);
    o[7] = (int64_t)((char*)fw.cutL - zero);
    return PK_OK;
}

template <typename T>
int shard_phase(int phase, const T* keys, int64_t us, int64_t rs, const float* center, float key_scale,
                const float* W, const float* b, const __half* Wh, const float* wn, int U, int64_t N, int F,
                BuildWs ws, FastWs fw, long long local_count, long long global_count, double sample_frac,
                long long flat_base, int* lens,
                int* offsets, int* ids, int64_t ids_stride, long long token_base, float slack_frac, int slack_min,
                const long long* all_keys, const int* key_counts, int P, int64_t key_cap, const long long* need,
                int* sample_info, int* status, cudaStream_t st) {
    const int nft = (F + kTcFeat - 1) / kTcFeat;
    const int nblocks = (int)((N + 127) / 128);
    if (phase == 0) {
        // The sample is planned on this shard's own share of the budget.
        int ns = 0;
        const TileSample plan = sample_plan(N, F, local_count, &ns);
        const WSource wsrc = make_wsource(Wh, F);
        build_tiles_kernel<<<nft, 256, 0, st>>>(Wh, wn, b, F, fw.tiles, fw.sides, status, !wsrc.use_map);
        PK_CHECK_LAUNCH();
        cudaFuncSetAttribute(build_tile_tc_kernel<0, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, tc_smem(0));
        build_tile_tc_kernel<0, T><<<dim3(ns, U), kTcThreads, tc_smem(0), st>>>(
            keys, us, rs, N, center, key_scale, F, fw, plan, status, wsrc);
        PK_CHECK_LAUNCH();
        set_ints_kernel<<<1, 1, 0, st>>>(sample_info, ns, plan.ft_stride);
        PK_CHECK_LAUNCH();
        return PK_OK;
    }
    if (phase == 1) {
        const TileSample none = {1, 1};
        build_floor_kernel<<<U, 32, 0, st>>>(fw, global_count, sample_frac);
        PK_CHECK_LAUNCH();
        cudaFuncSetAttribute(build_tile_tc_kernel<1, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, tc_smem(1));
        build_tile_tc_kernel<1, T><<<dim3(nblocks, U), kTcThreads, tc_smem(1), st>>>(
            keys, us, rs, N, center, key_scale, F, fw, none, status, make_wsource(Wh, F));
        PK_CHECK_LAUNCH();
        return PK_OK;
    }
    if (phase == 2) {
        build_fast_cut_kernel<<<U, 32, 0, st>>>(fw, global_count, status);
        PK_CHECK_LAUNCH();
        build_classify_kernel<<<dim3(256, U), 256, 0, st>>>(F, ws, fw, lens, status);
        PK_CHECK_LAUNCH();
        const size_t esz = sizeof(T);
        const int vec = ((uint64_t)keys % 16 == 0 && (us * (int64_t)esz) % 16 == 0 && (rs * (int64_t)esz) % 16 == 0)
                            ? 1 : 0;
        build_exact_kernel<T><<<dim3(512, U), 256, 0, st>>>(keys, us, rs, center, key_scale, W, b, F, ws, fw, lens,
                                                            status, vec, flat_base);
        PK_CHECK_LAUNCH();
        return PK_OK;
    }
    // phase 3: the global resolve, then CSR.
    build_shard_resolve_kernel<<<U, 1024, 0, st>>>(all_keys, key_counts, P, key_cap, need, flat_base,
                                                   flat_base + (long long)N * F, ws, fw, F, lens, status);
    PK_CHECK_LAUNCH();
    build_offsets_kernel<<<U, 1024, 0, st>>>(lens, F, slack_frac, slack_min, offsets, ids_stride, status);
    PK_CHECK_LAUNCH();
    build_scatter_kernel<<<dim3(64, U), 256, 0, st>>>(ws, F, offsets, ids, ids_stride, token_base);
    PK_CHECK_LAUNCH();
    return sort_buckets(ids, ids_stride, offsets, nullptr, lens, U, F, status, st);
}

extern "C" int pk_build_shard_phase(int phase, uint64_t keys, int dtype, int64_t unit_stride, int64_t row_stride,
                                    uint64_t center, float key_scale, uint64_t w_enc, uint64_t b_enc, uint64_t w_half,
                                    uint64_t w_norm, int U, int64_t N, int d, int F, int key_mean,
                                    int64_t member_capacity, int64_t boundary_capacity, uint64_t workspace,
                                    uint64_t workspace_bytes,
                                    long long global_count, double sample_frac, int64_t flat_base, uint64_t lens,
                                    uint64_t offsets, uint64_t ids, int64_t ids_stride, int64_t token_base,
                                    float slack_frac, int slack_min, uint64_t all_keys, uint64_t key_counts, int P,
                                    int64_t key_cap, uint64_t need, uint64_t sample_info, uint64_t status,
                                    uint64_t stream) {
    if (phase < 0 || phase > 3) return PK_ERR_ARG;
    if (U < 1 || N < 1 || F < 1 || key_mean < 1 || !(key_scale > 0.f) || slack_frac < 0.f || slack_min < 0)
        return PK_ERR_ARG;
    if (d != kBD) return PK_ERR_UNSUPPORTED;
    if (!keys || !center || !w_enc || !b_enc || !w_half || !w_norm || !lens || !workspace || !status)
        return PK_ERR_ARG;
    if (w_half % 16 || row_stride < d || N > INT32_MAX || global_count < 1 || flat_base < 0) return PK_ERR_ARG;
    if (flat_base + (long long)N * F >= (1ll << 36)) return PK_ERR_ARG;
    if (boundary_capacity < 1 || member_capacity < 1) return PK_ERR_ARG;
    if (workspace_bytes < pk_build_shard_workspace_bytes(U, N, F, member_capacity, boundary_capacity))
        return PK_ERR_WORKSPACE;
    if (phase == 0 && !sample_info) return PK_ERR_ARG;
    if (phase == 3 && (!offsets || !ids || !all_keys || !key_counts || P < 1 || key_cap < 1 || !need ||
                       ids_stride < 1 || token_base < 0 || token_base + N > INT32_MAX))
        return PK_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    const int64_t mcap = member_capacity;
    BuildWs ws = carve((void*)workspace, U, F, mcap, boundary_capacity);
    void* fbase = (char*)workspace + carve_bytes(U, F, mcap, boundary_capacity);
    FastWs fw = carve_fast(fbase, U, boundary_capacity, F);
    if (phase == 0) {
        cudaMemsetAsync((void*)workspace, 0, counters_bytes(U, F), st);
        cudaMemsetAsync(fbase, 0, fast_counters_bytes(U), st);
        cudaMemsetAsync((void*)lens, 0, (size_t)U * F * sizeof(int), st);
    }
    if (dtype == PK_BF16)
        return shard_phase(phase, (const __nv_bfloat16*)keys, unit_stride, row_stride, (const float*)center,
                           key_scale, (const float*)w_enc, (const float*)b_enc, (const __half*)w_half,
                           (const float*)w_norm, U, N, F, ws, fw, (long long)N * key_mean, global_count, sample_frac,
                           flat_base, (int*)lens,
                           (int*)offsets, (int*)ids, ids_stride, token_base, slack_frac, slack_min,
                           (const long long*)all_keys, (const int*)key_counts, P, key_cap, (const long long*)need,
                           (int*)sample_info, (int*)status, st);
    if (dtype == PK_F32)
        return shard_phase(phase, (const float*)keys, unit_stride, row_stride, (const float*)center, key_scale,
                           (const float*)w_enc, (const float*)b_enc, (const __half*)w_half, (const float*)w_norm, U, N,
                           F, ws, fw, (long long)N * key_mean, global_count, sample_frac, flat_base, (int*)lens,
                           (int*)offsets, (int*)ids,
                           ids_stride, token_base, slack_frac, slack_min, (const long long*)all_keys,
                           (const int*)key_counts, P, key_cap, (const long long*)need, (int*)sample_info,
                           (int*)status, st);
    return PK_ERR_ARG;
}

extern "C" int pk_key_center_chunks(uint64_t keys, int dtype, int64_t unit_stride, int64_t row_stride, int U,
                                    int64_t N, int d, int64_t N_total, uint64_t out, uint64_t stream) {
    if (U < 1 || N < 1 || d < 1 || N_total < N || !keys || !out || row_stride < d) return PK_ERR_ARG;
    int lp = ceil_log2_i64(N_total) / 4;
    if (lp < 4) lp = 4;
    const int64_t chunk = (int64_t)1 << (3 * lp);
    if (N % chunk) return PK_ERR_ARG;   // the shard holds whole chunks
    const int64_t nchunks = N / chunk;
    cudaStream_t st = (cudaStream_t)stream;
    dim3 grid((d + 31) / 32, U);
    if (dtype == PK_BF16)
        center_chunks_kernel<__nv_bfloat16><<<grid, 1024, 0, st>>>((const __nv_bfloat16*)keys, unit_stride,
                                                                   row_stride, nchunks, lp, d, (float*)out);
    else if (dtype == PK_F32)
        center_chunks_kernel<float><<<grid, 1024, 0, st>>>((const float*)keys, unit_stride, row_stride, nchunks, lp,
                                                           d, (float*)out);
    else
        return PK_ERR_ARG;
    PK_CHECK_LAUNCH();
    return PK_OK;
}

extern "C" int64_t pk_key_center_chunk_rows(int64_t N_total) {
    int lp = ceil_log2_i64(N_total) / 4;
    if (lp < 4) lp = 4;
    return (int64_t)1 << (3 * lp);
}
