// Budgeted bucket union: the greedy skip-overflow rule of
// src/prismkv/core.py:152-164, with the union held as a shared-memory bitmap
// over the unit's history and compacted to ascending token ids by a block
// scan (the order of core.py:164's chosen.nonzero()).
//
// The greedy is sequential by definition -- bucket i is accepted iff its
// tokens not yet chosen fit the remaining budget -- but it is computed here
// in parallel, exactly:
//   1. every staged (bucket, token) entry is inserted into a shared-memory
//      hash table that keeps each token's first candidate (atomicMin);
//   2. while no bucket has been skipped, bucket i's new tokens are exactly
//      its tokens whose first candidate is i, so one prefix sum over the
//      candidates finds the first bucket that overflows (i*);
//   3. after i*, the new-token counts of all remaining buckets are recounted
//      in parallel against the bitmap; a warp ballot finds the next bucket
//      that fits; accepting a bucket with no new tokens leaves the bitmap --
//      and so every count -- unchanged, otherwise the bitmap is updated and
//      the remaining counts recounted.
// When the staged lists or the history do not fit on chip, the greedy runs
// in one warp over lists staged chunk by chunk (same result).
#include "common.cuh"

namespace pk {

constexpr int kUnionThreads = 512;
constexpr int kStage = 8192;      // staged token ids (32 KB)
constexpr int kMaxCand = 256;     // candidates per unit (G * k)
constexpr int kHashSlots = 16384; // 2x the staged entries
constexpr int kHashBits = 14;

struct UnionSmem {
    int cand_bucket[kMaxCand];
    int cand_start[kMaxCand];
    int cand_len[kMaxCand];
    int stage_off[kMaxCand + 1];
    int newc[kMaxCand];
    int scan[40];
    long long red[32];
    int flags[8];
};

__device__ __forceinline__ bool test_bit(const uint32_t* bm, int t) { return (bm[t >> 5] >> (t & 31)) & 1u; }
__device__ __forceinline__ void set_bit(uint32_t* bm, int t) { atomicOr(&bm[t >> 5], 1u << (t & 31)); }
__device__ __forceinline__ int hash_slot(int t) { return (int)(((uint32_t)t * 2654435761u) >> (32 - kHashBits)); }

__device__ __forceinline__ void hash_insert(int* hkey, int* hown, int t, int c) {
    int s = hash_slot(t);
    while (true) {
        const int old = atomicCAS(&hkey[s], -1, t);
        if (old == -1 || old == t) {
            atomicMin(&hown[s], c);
            return;
        }
        s = (s + 1) & (kHashSlots - 1);
    }
}

__device__ __forceinline__ int hash_owner(const int* hkey, const int* hown, int t) {
    int s = hash_slot(t);
    while (hkey[s] != t) s = (s + 1) & (kHashSlots - 1);
    return hown[s];
}

__global__ void __launch_bounds__(kUnionThreads)
union_kernel(const int* __restrict__ offsets, const int* __restrict__ lens, const int* __restrict__ ids,
             int64_t ids_stride, const int* __restrict__ order, const int* __restrict__ n_order, int order_stride,
             const int* __restrict__ history, const long long* __restrict__ limit, int F, int max_history,
             int use_hash, int* __restrict__ out_ids, int64_t out_stride, int* __restrict__ out_count,
             int* __restrict__ features, int* __restrict__ n_features, long long* __restrict__ raw,
             int* __restrict__ status) {
    extern __shared__ __align__(16) uint32_t dyn[];
    __shared__ UnionSmem sm;
    const int u = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
    const int lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
    const int H = history[u];
    if (H > max_history || H < 0) {
        // The bitmap was sized for max_history: refuse rather than truncate.
        if (tid == 0) {
            if (status) atomicOr(status, PK_STATUS_HISTORY_TOO_LONG);
            out_count[u] = 0;
            n_features[u] = 0;
            raw[u] = 0;
        }
        return;
    }
    const int W = (H + 31) >> 5;
    const int Wmax = (max_history + 31) >> 5;
    uint32_t* bm = dyn;                                             // [W]
    int* stage = reinterpret_cast<int*>(dyn + ((Wmax + 3) & ~3));   // [kStage]
    int* hkey = stage + kStage;                                     // [kHashSlots] (use_hash)
    int* hown = hkey + kHashSlots;                                  // [kHashSlots]
    const int n = min(n_order[u], kMaxCand);
    const long long lim = limit[u];
    const int* uid = ids + (int64_t)u * ids_stride;
    int* feat = features + (int64_t)u * order_stride;

    for (int i = tid; i < W; i += nt) bm[i] = 0u;
    for (int c = tid; c < n; c += nt) {
        const int b = order[(int64_t)u * order_stride + c];
        sm.cand_bucket[c] = b;
        sm.cand_start[c] = offsets[(int64_t)u * (F + 1) + b];
        sm.cand_len[c] = lens[(int64_t)u * F + b];
    }
    __syncthreads();
    if (tid == 0) {
        long long s = 0;
        sm.stage_off[0] = 0;
        for (int c = 0; c < n; ++c) {
            s += sm.cand_len[c];
            sm.stage_off[c + 1] = (int)min(s, (long long)INT32_MAX);
        }
        sm.red[0] = s;
    }
    __syncthreads();
    const long long raw_total = sm.red[0];
    long long raw_acc = 0;
    int nf = 0;

    if (raw_total <= lim) {
        // Every candidate fits whatever the overlap: the unbudgeted union.
        for (int c = warp; c < n; c += nw) {
            const int L = sm.cand_len[c];
            const int* src = uid + sm.cand_start[c];
            for (int i = lane; i < L; i += 32) {
                const int t = src[i];
                if ((unsigned)t < (unsigned)H) set_bit(bm, t);
            }
        }
        for (int c = tid; c < n; c += nt) feat[c] = sm.cand_bucket[c];
        nf = n;
        raw_acc = raw_total;
    } else if (use_hash && raw_total <= kStage) {
        // ---- 1. stage the lists and record each token's first candidate.
        for (int i = tid; i < kHashSlots; i += nt) { hkey[i] = -1; hown[i] = INT32_MAX; }
        for (int c = warp; c < n; c += nw) {
            const int L = sm.cand_len[c];
            const int* src = uid + sm.cand_start[c];
            int* dst = stage + sm.stage_off[c];
            for (int i = lane; i < L; i += 32) dst[i] = src[i];
        }
        __syncthreads();
        for (int c = warp; c < n; c += nw) {
            const int* lst = stage + sm.stage_off[c];
            const int L = sm.cand_len[c];
            for (int i = lane; i < L; i += 32) {
                const int t = lst[i];
                if ((unsigned)t < (unsigned)H) hash_insert(hkey, hown, t, c);
            }
        }
        __syncthreads();
        // ---- 2. new tokens per candidate while every earlier one is taken.
        for (int c = warp; c < n; c += nw) {
            const int* lst = stage + sm.stage_off[c];
            const int L = sm.cand_len[c];
            int cnt = 0;
            for (int i = lane; i < L; i += 32) {
                const int t = lst[i];
                cnt += ((unsigned)t < (unsigned)H && hash_owner(hkey, hown, t) == c) ? 1 : 0;
            }
            cnt = warp_sum(cnt);
            if (lane == 0) sm.newc[c] = cnt;
        }
        __syncthreads();
        if (warp == 0) {
            // Prefix sum in candidate order; i* = first candidate that overflows.
            long long run = 0;
            int istar = n;
            for (int base = 0; base < n; base += 32) {
                const int c = base + lane;
                int v = c < n ? sm.newc[c] : 0;
                int inc = warp_inclusive_scan(v);
                const bool over = c < n && run + inc > lim;
                const unsigned om = __ballot_sync(0xffffffffu, over);
                if (om) {
                    istar = base + __ffs(om) - 1;
                    const int before = __shfl_sync(0xffffffffu, inc - v, istar - base);
                    run += before;
                    break;
                }
                run += __shfl_sync(0xffffffffu, inc, 31);
            }
            if (lane == 0) {
                sm.flags[0] = istar;
                sm.red[1] = run;   // chosen count after the accepted prefix
            }
        }
        __syncthreads();
        const int istar = sm.flags[0];
        long long count = sm.red[1];
        // Accepted prefix: its tokens into the bitmap.
        for (int c = warp; c < istar; c += nw) {
            const int* lst = stage + sm.stage_off[c];
            const int L = sm.cand_len[c];
            for (int i = lane; i < L; i += 32) {
                const int t = lst[i];
                if ((unsigned)t < (unsigned)H) set_bit(bm, t);
            }
        }
        for (int c = tid; c < istar; c += nt) feat[c] = sm.cand_bucket[c];
        nf = istar;
        raw_acc = sm.stage_off[istar];
        __syncthreads();
        // ---- 3. the tail after the first skipped candidate.
        int pos = istar + 1;
        while (pos < n) {
            // Recount new tokens of candidates pos.. against the bitmap.
            for (int c = pos + warp; c < n; c += nw) {
                const int* lst = stage + sm.stage_off[c];
                const int L = sm.cand_len[c];
                int cnt = 0;
                for (int i = lane; i < L; i += 32) {
                    const int t = lst[i];
                    cnt += ((unsigned)t < (unsigned)H && !test_bit(bm, t)) ? 1 : 0;
                }
                cnt = warp_sum(cnt);
                if (lane == 0) sm.newc[c] = cnt;
            }
            __syncthreads();
            if (warp == 0) {
                // Scan for the next fitting candidate; zero-new acceptances
                // change nothing and are taken inline.
                int next = n;
                while (pos < n) {
                    const int c = pos + lane;
                    const bool fits = c < n && count + sm.newc[c] <= lim;
                    const unsigned fm = __ballot_sync(0xffffffffu, fits);
                    if (!fm) { pos += 32; continue; }
                    const int a = pos + __ffs(fm) - 1;
                    const int add = sm.newc[a];
                    if (lane == 0) feat[nf] = sm.cand_bucket[a];
                    ++nf;
                    raw_acc += sm.cand_len[a];
                    pos = a + 1;
                    if (add > 0) {
                        count += add;
                        next = a;
                        break;
                    }
                }
                if (lane == 0) {
                    sm.flags[1] = next;
                    sm.flags[2] = nf;
                    sm.flags[3] = min(pos, n);
                    sm.red[2] = raw_acc;
                    sm.red[3] = count;
                }
            }
            __syncthreads();
            const int a = sm.flags[1];
            nf = sm.flags[2];
            pos = sm.flags[3];
            raw_acc = sm.red[2];
            count = sm.red[3];
            if (a >= n) break;
            // Candidate a added tokens: set them, then recount.
            {
                const int* lst = stage + sm.stage_off[a];
                const int L = sm.cand_len[a];
                for (int i = tid; i < L; i += nt) {
                    const int t = lst[i];
                    if ((unsigned)t < (unsigned)H) set_bit(bm, t);
                }
            }
            __syncthreads();
        }
    } else {
        // Sequential greedy over lists staged chunk by chunk.
        long long count = 0;
        int c = 0;
        while (c < n) {
            if (tid == 0) {
                int c_end = c, filled = 0;
                sm.flags[4] = 0;
                sm.stage_off[c] = 0;
                while (c_end < n && (filled + sm.cand_len[c_end] <= kStage || c_end == c)) {
                    filled += min(sm.cand_len[c_end], kStage);
                    ++c_end;
                    sm.stage_off[c_end] = filled;
                }
                sm.flags[0] = c_end;
            }
            __syncthreads();
            const int c_end = sm.flags[0];
            for (int cc = c; cc < c_end; ++cc) {
                const int L = min(sm.cand_len[cc], kStage);
                const int* src = uid + sm.cand_start[cc];
                int* dst = stage + sm.stage_off[cc];
                for (int i = tid; i < L; i += nt) dst[i] = src[i];
            }
            __syncthreads();
            if (warp == 0) {
                for (int cc = c; cc < c_end; ++cc) {
                    const int L = sm.cand_len[cc];
                    const int* src = L <= kStage ? stage + sm.stage_off[cc] : uid + sm.cand_start[cc];
                    int fresh = 0;
                    for (int i = lane; i < L; i += 32) {
                        const int t = src[i];
                        fresh += ((unsigned)t < (unsigned)H && !test_bit(bm, t)) ? 1 : 0;
                    }
                    fresh = warp_sum(fresh);
                    if (count + fresh <= lim) {
                        for (int i = lane; i < L; i += 32) {
                            const int t = src[i];
                            if ((unsigned)t < (unsigned)H) set_bit(bm, t);
                        }
                        __syncwarp();
                        count += fresh;
                        raw_acc += L;
                        if (lane == 0) feat[nf] = sm.cand_bucket[cc];
                        ++nf;
                    }
                }
                if (lane == 0) {
                    sm.flags[1] = nf;
                    sm.red[1] = raw_acc;
                    sm.red[2] = count;
                }
            }
            __syncthreads();
            nf = sm.flags[1];
            raw_acc = sm.red[1];
            count = sm.red[2];
            c = c_end;
            __syncthreads();
        }
    }
    __syncthreads();

    // Compaction: each thread owns a contiguous run of words.
    const int per = (W + nt - 1) / nt;
    const int w0 = min(W, tid * per), w1 = min(W, w0 + per);
    int pop = 0;
    for (int w = w0; w < w1; ++w) pop += __popc(bm[w]);
    int total;
    int at = block_exclusive_scan(pop, sm.scan, &total);
    int* dst = out_ids + (int64_t)u * out_stride;
    bool overflow = false;
    for (int w = w0; w < w1; ++w) {
        uint32_t m = bm[w];
        while (m) {
            const int bit = __ffs(m) - 1;
            m &= m - 1;
            if (at < out_stride) dst[at] = w * 32 + bit;
            else overflow = true;
            ++at;
        }
    }
    if (overflow && status) atomicOr(status, PK_STATUS_OUT_FULL);
    if (tid == 0) {
        out_count[u] = total;
        n_features[u] = nf;
        raw[u] = raw_acc;
    }
}

}  // namespace pk

using namespace pk;

extern "C" int pk_union(uint64_t offsets, uint64_t lens, uint64_t ids, int64_t ids_stride, uint64_t order,
                        uint64_t n_order, int order_stride, uint64_t history, uint64_t limit, int U, int F,
                        int max_history, uint64_t out_ids, int64_t out_stride, uint64_t out_count,
                        uint64_t features, uint64_t n_features, uint64_t raw, uint64_t status, uint64_t stream) {
    if (U < 1 || F < 1 || max_history < 0 || order_stride < 1 || out_stride < 0 || ids_stride < 0) return PK_ERR_ARG;
    if (!offsets || !lens || !ids || !order || !n_order || !history || !limit || !out_ids || !out_count ||
        !features || !n_features || !raw)
        return PK_ERR_ARG;
    const int Wmax = (max_history + 31) / 32;
    const size_t base = (size_t)((Wmax + 3) & ~3) * 4 + (size_t)kStage * 4;
    const size_t with_hash = base + (size_t)2 * kHashSlots * 4;
    const size_t cap = 200 * 1024;
    if (base > cap) return PK_ERR_UNSUPPORTED;
    const int use_hash = with_hash <= cap ? 1 : 0;
    const size_t smem = use_hash ? with_hash : base;
    cudaFuncSetAttribute(union_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    union_kernel<<<U, kUnionThreads, smem, (cudaStream_t)stream>>>(
        (const int*)offsets, (const int*)lens, (const int*)ids, ids_stride, (const int*)order, (const int*)n_order,
        order_stride, (const int*)history, (const long long*)limit, F, max_history, use_hash, (int*)out_ids,
        out_stride, (int*)out_count, (int*)features, (int*)n_features, (long long*)raw, (int*)status);
    PK_CHECK_LAUNCH();
    return PK_OK;
}
