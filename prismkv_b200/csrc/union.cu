// Budgeted bucket union: the greedy skip-overflow rule of
// src/prismkv/core.py:152-164, with the union held as a shared-memory bitmap
// over the unit's history and compacted to ascending token ids by a block
// scan (the order of core.py:164's chosen.nonzero()).
//
// The candidates' bucket lists are first staged in shared memory with one
// fully parallel copy.  The greedy -- sequential by definition: bucket i is
// accepted iff its tokens not yet chosen fit the remaining budget -- is then
// computed exactly in two phases:
//   1. while no bucket has been skipped, bucket i's new tokens are its tokens
//      that are neither in the bitmap (earlier rounds) nor in an earlier
//      bucket of the current round.  Rounds take as many buckets as a shared-
//      memory hash (token -> first bucket of the round, atomicMin) can hold;
//      a warp prefix sum over the round's counts finds the first bucket that
//      would overflow (i*), and the buckets before it are OR-ed in.
//   2. after i*, every remaining bucket's new-token count is computed once in
//      parallel; then one warp walks the buckets in order.  A bucket whose
//      count minus the tokens added since cannot fit is skipped at once; any
//      other is re-counted against the current bitmap and taken if it fits.
// Lists that do not fit the staging area are read from global memory by the
// same code paths.
#include "common.cuh"

namespace pk {

constexpr int kUnionThreads = 512;
constexpr int kMaxCand = 256;     // candidates per unit (G * k)

struct UnionSmem {
    int cand_bucket[kMaxCand];
    int cand_start[kMaxCand];
    int cand_len[kMaxCand];
    int cand_stage[kMaxCand];     // offset in the staging area, or -1
    int newc[kMaxCand];
    int scan[40];
    long long red[32];
    int flags[8];
};

__device__ __forceinline__ bool test_bit(const uint32_t* bm, int t) { return (bm[t >> 5] >> (t & 31)) & 1u; }
__device__ __forceinline__ void set_bit(uint32_t* bm, int t) { atomicOr(&bm[t >> 5], 1u << (t & 31)); }

struct Hash {
    int* key;
    int* own;
    int bits;
    __device__ __forceinline__ int slot(int t) const { return (int)(((uint32_t)t * 2654435761u) >> (32 - bits)); }
    __device__ __forceinline__ void insert(int t, int c) const {
        const int mask = (1 << bits) - 1;
        int s = slot(t);
        while (true) {
            const int old = atomicCAS(&key[s], -1, t);
            if (old == -1 || old == t) {
                atomicMin(&own[s], c);
                return;
            }
            s = (s + 1) & mask;
        }
    }
    __device__ __forceinline__ int owner(int t) const {
        const int mask = (1 << bits) - 1;
        int s = slot(t);
        while (key[s] != t) s = (s + 1) & mask;
        return own[s];
    }
};

__global__ void __launch_bounds__(kUnionThreads)
union_kernel(const int* __restrict__ offsets, const int* __restrict__ lens, const int* __restrict__ ids,
             int64_t ids_stride, const int* __restrict__ order, const int* __restrict__ n_order, int order_stride,
             const int* __restrict__ history, const long long* __restrict__ limit, int F, int max_history,
             int hash_bits, int stage_cap, int* __restrict__ out_ids, int64_t out_stride,
             int* __restrict__ out_count, int* __restrict__ features, int* __restrict__ n_features,
             long long* __restrict__ raw, int* __restrict__ status) {
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
    uint32_t* bm = dyn;                                               // [W]
    int* hkeys = reinterpret_cast<int*>(dyn + ((Wmax + 3) & ~3));     // [2^hash_bits]
    int* hown = hkeys + (1 << hash_bits);                             // [2^hash_bits]
    int* stage = hown + (1 << hash_bits);                             // [stage_cap]
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
        int staged = 0;
        for (int c = 0; c < n; ++c) {
            const int L = sm.cand_len[c];
            s += L;
            if (staged + L <= stage_cap) { sm.cand_stage[c] = staged; staged += L; }
            else sm.cand_stage[c] = -1;
        }
        sm.red[0] = s;
    }
    __syncthreads();
    // Stage: one warp per candidate, every load independent.
    for (int c = warp; c < n; c += nw) {
        const int off = sm.cand_stage[c];
        if (off < 0) continue;
        const int L = sm.cand_len[c];
        const int* src = uid + sm.cand_start[c];
        for (int i = lane; i < L; i += 32) stage[off + i] = src[i];
    }
    __syncthreads();
    auto list = [&](int c) -> const int* {
        const int off = sm.cand_stage[c];
        return off >= 0 ? stage + off : uid + sm.cand_start[c];
    };
    const long long raw_total = sm.red[0];
    long long raw_acc = 0;
    int nf = 0;

    if (raw_total <= lim) {
        // Every candidate fits whatever the overlap: the unbudgeted union.
        for (int c = warp; c < n; c += nw) {
            const int L = sm.cand_len[c];
            const int* lst = list(c);
            for (int i = lane; i < L; i += 32) {
                const int t = lst[i];
                if ((unsigned)t < (unsigned)H) set_bit(bm, t);
            }
        }
        for (int c = tid; c < n; c += nt) feat[c] = sm.cand_bucket[c];
        nf = n;
        raw_acc = raw_total;
    } else {
        Hash hs{hkeys, hown, hash_bits};
        const int round_cap = 1 << (hash_bits - 1);  // load factor <= 1/2
        long long count = 0;
        int c0 = 0, istar = n;
        // ---- 1. rounds while every bucket so far was accepted.
        while (c0 < n) {
            if (tid == 0) {
                int c1 = c0, filled = 0;
                while (c1 < n && (filled + sm.cand_len[c1] <= round_cap || c1 == c0)) {
                    filled += sm.cand_len[c1];
                    ++c1;
                }
                sm.flags[0] = c1;
            }
            __syncthreads();
            const int c1 = sm.flags[0];
            const bool single = c1 - c0 == 1;
            if (!single) {
                for (int i = tid; i < (1 << hash_bits); i += nt) { hs.key[i] = -1; hs.own[i] = INT32_MAX; }
                __syncthreads();
                for (int c = c0 + warp; c < c1; c += nw) {
                    const int* lst = list(c);
                    const int L = sm.cand_len[c];
                    for (int i = lane; i < L; i += 32) {
                        const int t = lst[i];
                        if ((unsigned)t < (unsigned)H && !test_bit(bm, t)) hs.insert(t, c);
                    }
                }
                __syncthreads();
            }
            for (int c = c0 + warp; c < c1; c += nw) {
                const int* lst = list(c);
                const int L = sm.cand_len[c];
                int cnt = 0;
                for (int i = lane; i < L; i += 32) {
                    const int t = lst[i];
                    cnt += ((unsigned)t < (unsigned)H && !test_bit(bm, t) && (single || hs.owner(t) == c)) ? 1 : 0;
                }
                cnt = warp_sum(cnt);
                if (lane == 0) sm.newc[c] = cnt;
            }
            __syncthreads();
            if (warp == 0) {
                long long run = count;
                int first_over = c1;
                for (int base = c0; base < c1; base += 32) {
                    const int c = base + lane;
                    const int v = c < c1 ? sm.newc[c] : 0;
                    const int inc = warp_inclusive_scan(v);
                    const bool over = c < c1 && run + inc > lim;
                    const unsigned om = __ballot_sync(0xffffffffu, over);
                    if (om) {
                        first_over = base + __ffs(om) - 1;
                        run += __shfl_sync(0xffffffffu, inc - v, first_over - base);
                        break;
                    }
                    run += __shfl_sync(0xffffffffu, inc, 31);
                }
                if (lane == 0) {
                    sm.flags[1] = first_over;
                    sm.red[1] = run;
                }
            }
            __syncthreads();
            const int acc_end = sm.flags[1];
            count = sm.red[1];
            for (int c = c0 + warp; c < acc_end; c += nw) {
                const int* lst = list(c);
                const int L = sm.cand_len[c];
                for (int i = lane; i < L; i += 32) {
                    const int t = lst[i];
                    if ((unsigned)t < (unsigned)H) set_bit(bm, t);
                }
            }
            for (int c = c0 + tid; c < acc_end; c += nt) feat[c] = sm.cand_bucket[c];
            for (int c = c0; c < acc_end; ++c) raw_acc += sm.cand_len[c];
            nf = acc_end;
            __syncthreads();
            if (acc_end < c1) {
                istar = acc_end;
                break;
            }
            c0 = c1;
        }
        // ---- 2. the tail after the first skipped bucket.
        if (istar + 1 < n) {
            for (int c = istar + 1 + warp; c < n; c += nw) {
                const int* lst = list(c);
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
                // newc[c] was exact when counted; the bitmap has grown by
                // `added` tokens since, so newc[c] - added <= true count.
                long long added = 0;
                for (int c = istar + 1; c < n; ++c) {
                    if ((long long)sm.newc[c] - added > lim - count) continue;
                    const int* lst = list(c);
                    const int L = sm.cand_len[c];
                    int fresh = 0;
                    if (added == 0) {
                        fresh = sm.newc[c];
                    } else {
                        for (int i = lane; i < L; i += 32) {
                            const int t = lst[i];
                            fresh += ((unsigned)t < (unsigned)H && !test_bit(bm, t)) ? 1 : 0;
                        }
                        fresh = warp_sum(fresh);
                    }
                    if (count + fresh > lim) continue;
                    if (fresh > 0) {
                        for (int i = lane; i < L; i += 32) {
                            const int t = lst[i];
                            if ((unsigned)t < (unsigned)H) set_bit(bm, t);
                        }
                        __syncwarp();
                    }
                    count += fresh;
                    added += fresh;
                    raw_acc += L;
                    if (lane == 0) feat[nf] = sm.cand_bucket[c];
                    ++nf;
                }
                if (lane == 0) {
                    sm.flags[3] = nf;
                    sm.red[2] = raw_acc;
                }
            }
            __syncthreads();
            nf = sm.flags[3];
            raw_acc = sm.red[2];
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
    const size_t bitmap = (size_t)((Wmax + 3) & ~3) * 4;
    const size_t cap = 200 * 1024;
    // Hash of 2^13 slots (rounds of <= 4096 list entries) when the bitmap
    // leaves room, else 2^10; the rest stages lists (at least 2048 ids).
    int bits = 0;
    for (int b = 13; b >= 10; --b)
        if (bitmap + ((size_t)2 << b) * 4 + 2048 * 4 <= cap) { bits = b; break; }
    if (!bits) return PK_ERR_UNSUPPORTED;
    const size_t used = bitmap + ((size_t)2 << bits) * 4;
    const int stage_cap = (int)((cap - used) / 4);
    cudaFuncSetAttribute(union_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cap);
    union_kernel<<<U, kUnionThreads, cap, (cudaStream_t)stream>>>(
        (const int*)offsets, (const int*)lens, (const int*)ids, ids_stride, (const int*)order, (const int*)n_order,
        order_stride, (const int*)history, (const long long*)limit, F, max_history, bits, stage_cap, (int*)out_ids,
        out_stride, (int*)out_count, (int*)features, (int*)n_features, (long long*)raw, (int*)status);
    PK_CHECK_LAUNCH();
    return PK_OK;
}
