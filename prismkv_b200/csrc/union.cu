// Budgeted bucket union: the greedy skip-overflow rule of
// src/prismkv/core.py:152-164, with the union held as a shared-memory bitmap
// over the unit's history and compacted to ascending token ids by a block
// scan (the order of core.py:164's chosen.nonzero()).
#include "common.cuh"

namespace pk {

constexpr int kUnionThreads = 512;
constexpr int kStage = 8192;      // staged token ids per chunk (32 KB)
constexpr int kMaxCand = 256;     // candidates per unit (G * k)

struct UnionSmem {
    int cand_bucket[kMaxCand];
    int cand_start[kMaxCand];
    int cand_len[kMaxCand];
    int stage_off[kMaxCand + 1];
    int scan[40];
    long long red[32];
    int flags[4];
};

__device__ __forceinline__ bool test_bit(const uint32_t* bm, int t) { return (bm[t >> 5] >> (t & 31)) & 1u; }
__device__ __forceinline__ void set_bit(uint32_t* bm, int t) { atomicOr(&bm[t >> 5], 1u << (t & 31)); }

__global__ void __launch_bounds__(kUnionThreads)
union_kernel(const int* __restrict__ offsets, const int* __restrict__ lens, const int* __restrict__ ids,
             int64_t ids_stride, const int* __restrict__ order, const int* __restrict__ n_order, int order_stride,
             const int* __restrict__ history, const long long* __restrict__ limit, int F, int max_history,
             int* __restrict__ out_ids, int64_t out_stride, int* __restrict__ out_count,
             int* __restrict__ features, int* __restrict__ n_features, long long* __restrict__ raw,
             int* __restrict__ status) {
    extern __shared__ __align__(16) uint32_t dyn[];
    __shared__ UnionSmem sm;
    const int u = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
    const int lane = tid & 31, warp = tid >> 5;
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
    const int n = min(n_order[u], kMaxCand);
    const long long lim = limit[u];
    const int* uid = ids + (int64_t)u * ids_stride;

    for (int i = tid; i < W; i += nt) bm[i] = 0u;
    for (int c = tid; c < n; c += nt) {
        const int b = order[(int64_t)u * order_stride + c];
        sm.cand_bucket[c] = b;
        sm.cand_start[c] = offsets[(int64_t)u * (F + 1) + b];
        sm.cand_len[c] = lens[(int64_t)u * F + b];
    }
    __syncthreads();
    long long mine = 0;
    for (int c = tid; c < n; c += nt) mine += sm.cand_len[c];
    mine = warp_sum(mine);
    if (lane == 0) sm.red[warp] = mine;
    __syncthreads();
    if (tid == 0) {
        long long s = 0;
        for (int w = 0; w < nt / 32; ++w) s += sm.red[w];
        sm.red[0] = s;
    }
    __syncthreads();
    const long long raw_total = sm.red[0];
    long long raw_acc = 0;
    int nf = 0;
    __syncthreads();

    if (raw_total <= lim) {
        // Every candidate fits whatever the overlap: the unbudgeted union.
        for (int c = 0; c < n; ++c) {
            const int L = sm.cand_len[c];
            const int* src = uid + sm.cand_start[c];
            for (int i = tid; i < L; i += nt) {
                const int t = src[i];
                if ((unsigned)t < (unsigned)H) set_bit(bm, t);
            }
        }
        for (int c = tid; c < n; c += nt) features[(int64_t)u * order_stride + c] = sm.cand_bucket[c];
        nf = n;
        raw_acc = raw_total;
    } else {
        // Sequential greedy; lists are staged in shared memory chunk by chunk
        // so the decision loop only touches on-chip data.
        long long count = 0;
        int c = 0;
        while (c < n) {
            if (tid == 0) {
                int c_end = c, filled = 0;
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
                        if (lane == 0) features[(int64_t)u * order_stride + nf] = sm.cand_bucket[cc];
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
    const size_t smem = (size_t)((Wmax + 3) & ~3) * 4 + (size_t)kStage * 4;
    if (smem > 200 * 1024) return PK_ERR_UNSUPPORTED;
    cudaFuncSetAttribute(union_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    union_kernel<<<U, kUnionThreads, smem, (cudaStream_t)stream>>>(
        (const int*)offsets, (const int*)lens, (const int*)ids, ids_stride, (const int*)order, (const int*)n_order,
        order_stride, (const int*)history, (const long long*)limit, F, max_history, (int*)out_ids, out_stride,
        (int*)out_count, (int*)features, (int*)n_features, (long long*)raw, (int*)status);
    PK_CHECK_LAUNCH();
    return PK_OK;
}
