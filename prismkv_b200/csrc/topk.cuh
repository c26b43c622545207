// Block-wide exact top-k selection over uint32 keys.
#pragma once
#include "common.cuh"

namespace pk {

struct TopkScratch {
    int hist[256];
    int scan[33];
    int misc[8];
};

// Selects the k entries with the largest keys among eligible ones
// (eligible(i) true), ties broken by lower index -- the first k of a stable
// descending argsort restricted to eligible entries.  key(i) must be
// monotone in the ranked value.  Writes the selected indices in rank order
// to out_idx[0..m) and their keys to out_key, returns m = min(k, #eligible).
// out_idx/out_key must hold k entries; k <= 4 * blockDim.x.  All threads of
// the block must call it.
template <typename KeyFn, typename EligFn>
__device__ int block_topk(int n, int k, KeyFn key, EligFn eligible, int* out_idx, uint32_t* out_key,
                          TopkScratch& s) {
    const int tid = threadIdx.x, nt = blockDim.x;
    int local = 0;
    for (int i = tid; i < n; i += nt) local += eligible(i) ? 1 : 0;
    int total;
    block_exclusive_scan(local, s.scan, &total);
    const bool take_all = total <= k;
    uint32_t prefix = 0, pmask = 0;
    int need = take_all ? total : k;
    if (!take_all) {
        // MSB-first radix select of the k-th largest key, 8 bits a pass.
        for (int pass = 0; pass < 4; ++pass) {
            const int shift = 24 - 8 * pass;
            for (int i = tid; i < 256; i += nt) s.hist[i] = 0;
            __syncthreads();
            for (int i = tid; i < n; i += nt) {
                if (!eligible(i)) continue;
                const uint32_t kk = key(i);
                if ((kk & pmask) != prefix) continue;
                atomicAdd(&s.hist[(kk >> shift) & 255u], 1);
            }
            __syncthreads();
            if (tid < 32) {
                // Lane l owns bins 255-8l .. 248-8l (descending).
                int c[8], tot = 0;
#pragma unroll
                for (int j = 0; j < 8; ++j) { c[j] = s.hist[255 - (tid * 8 + j)]; tot += c[j]; }
                const int inc = warp_inclusive_scan(tot);
                const int before = inc - tot;
                if (before < need && inc >= need) {
                    int acc = before, j = 0;
                    for (; j < 8; ++j) {
                        if (acc + c[j] >= need) break;
                        acc += c[j];
                    }
                    s.misc[0] = 255 - (tid * 8 + j);
                    s.misc[1] = need - acc;
                }
            }
            __syncthreads();
            prefix |= (uint32_t)s.misc[0] << shift;
            pmask |= 0xFFu << shift;
            need = s.misc[1];
            __syncthreads();
        }
    }
    // prefix = the k-th largest key; `need` entries equal to it are taken,
    // lowest indices first.  Ordered compaction in index order.
    const uint32_t T = prefix;
    int* sel = out_idx;
    int base = 0, tie_base = 0;
    for (int start = 0; start < n; start += nt) {
        const int i = start + tid;
        const bool el = i < n && eligible(i);
        const uint32_t kk = el ? key(i) : 0u;
        const bool gt = el && (take_all || kk > T);
        const bool eq = el && !take_all && kk == T;
        int eq_total;
        const int eq_rank = block_exclusive_scan(eq ? 1 : 0, s.scan, &eq_total);
        const bool pick = gt || (eq && tie_base + eq_rank < need);
        int pick_total;
        const int at = block_exclusive_scan(pick ? 1 : 0, s.scan, &pick_total);
        if (pick) sel[base + at] = i;
        base += pick_total;
        tie_base += eq_total;
    }
    __syncthreads();
    const int m = base;
    // Sort the m picks by (key desc, index asc): rank by counting.
    for (int i = tid; i < m; i += nt) out_key[i] = key(sel[i]);
    __syncthreads();
    int my_idx[4], my_rank[4], cnt = 0;
    for (int i = tid; i < m; i += nt) {
        const uint32_t ki = out_key[i];
        const int ii = sel[i];
        int r = 0;
        for (int j = 0; j < m; ++j) {
            const uint32_t kj = out_key[j];
            const int ij = sel[j];
            r += (kj > ki) || (kj == ki && ij < ii);
        }
        if (cnt < 4) { my_idx[cnt] = ii; my_rank[cnt] = r; }
        ++cnt;
    }
    __syncthreads();
    for (int c = 0; c < cnt && c < 4; ++c) {
        out_idx[my_rank[c]] = my_idx[c];
        out_key[my_rank[c]] = key(my_idx[c]);
    }
    __syncthreads();
    return m;
}

}  // namespace pk
