// Block-wide exact top-k selection over uint32 keys.
#pragma once
#include "common.cuh"

namespace pk {

constexpr int kTopkCap = 256;   // candidates finished by an exact rank sort

struct TopkScratch {
    int hist[256];
    int wcnt[2][32];            // per-warp counts for ordered compaction
    int misc[8];
    int scan[40];               // block_exclusive_scan scratch for callers
    int cand_idx[kTopkCap];
    uint32_t cand_key[kTopkCap];
};

__device__ __forceinline__ unsigned lanemask_lt() {
    unsigned m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

// Selects the k entries with the largest keys among eligible ones
// (eligible(i) true), ties broken by lower index -- the first k of a stable
// descending argsort restricted to eligible entries.  key(i) must be
// monotone in the ranked value.  Writes the picks in rank order to
// out_idx[0..m) and their keys to out_key, returns m = min(k, #eligible).
// k <= kTopkCap.  All threads of the block must call it; blockDim.x must be
// a multiple of 32.
//
// MSB-first radix select, 8 bits a pass, with warp-aggregated histogram
// updates; as soon as the entries whose key prefix reaches the current
// threshold number at most kTopkCap they are gathered in index order and
// ranked exactly.  If exact ties keep more than kTopkCap entries in play
// after all 32 bits, the strictly greater ones and the lowest-index ties are
// taken directly.
template <typename KeyFn, typename EligFn>
__device__ int block_topk(int n, int k, KeyFn key, EligFn eligible, int* out_idx, uint32_t* out_key,
                          TopkScratch& s) {
    const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
    const int seg = ((n + nw - 1) / nw + 31) / 32 * 32;  // contiguous segment per warp
    const int w0 = min(n, warp * seg), w1 = min(n, w0 + seg);

    uint32_t prefix = 0, pmask = 0;
    int need = k, above = 0;   // entries strictly above the current prefix (all taken)
    int mode = 0;              // 0: undecided, 1: gather prefix >= threshold, 2: exact ties
    int gshift = 0;
    for (int pass = 0; pass < 4 && mode == 0; ++pass) {
        const int shift = 24 - 8 * pass;
        for (int i = tid; i < 256; i += nt) s.hist[i] = 0;
        __syncthreads();
        for (int base = w0; base < w1; base += 32) {
            const int i = base + lane;
            bool part = i < w1 && eligible(i);
            uint32_t kk = part ? key(i) : 0u;
            part = part && (kk & pmask) == prefix;
            const unsigned bin = part ? ((kk >> shift) & 255u) : 256u + lane;
            const unsigned peers = __match_any_sync(0xffffffffu, bin);
            if (part && lane == __ffs(peers) - 1) atomicAdd(&s.hist[bin], __popc(peers));
        }
        __syncthreads();
        if (tid < 32) {
            int c[8], tot = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) { c[j] = s.hist[255 - (tid * 8 + j)]; tot += c[j]; }
            const int inc = warp_inclusive_scan(tot);
            const int all = __shfl_sync(0xffffffffu, inc, 31);
            if (tid == 0) s.misc[2] = all;
            const int before = inc - tot;
            if (all > need && before < need && inc >= need) {
                int acc = before, j = 0;
                for (; j < 8; ++j) {
                    if (acc + c[j] >= need) break;
                    acc += c[j];
                }
                s.misc[0] = 255 - (tid * 8 + j);
                s.misc[1] = acc;          // entries above the digit within this prefix
                s.misc[3] = c[j];         // entries in the digit's bin
            }
        }
        __syncthreads();
        const int in_prefix = s.misc[2];
        if (in_prefix <= need) {
            // Everything still in play is taken: gather by the prefix
            // resolved before this pass (all eligible entries on pass 0).
            mode = 1;
            gshift = pass == 0 ? 32 : shift + 8;
            break;
        }
        const int dgt = s.misc[0], acc = s.misc[1], inbin = s.misc[3];
        prefix |= (uint32_t)dgt << shift;
        pmask |= 0xFFu << shift;
        above += acc;
        need -= acc;
        __syncthreads();
        if (above + inbin <= kTopkCap) {
            mode = 1;
            gshift = shift;
        }
    }
    if (mode == 0) mode = 2;

    // Ordered gather.  Mode 1: every eligible entry whose key, truncated to
    // the resolved prefix bits, is >= the prefix (<= kTopkCap entries, all
    // entries >= the k-th key included).  Mode 2: keys > prefix (exact
    // threshold) plus the lowest-index `need` entries equal to it.
    const uint32_t gmask = gshift >= 32 ? 0u : (0xFFFFFFFFu << gshift);
    const uint32_t gpref = prefix & gmask;
    // Pass A: per-warp counts.
    int my_gt = 0, my_eq = 0;
    for (int base = w0; base < w1; base += 32) {
        const int i = base + lane;
        const bool el = i < w1 && eligible(i);
        const uint32_t kk = el ? key(i) : 0u;
        bool gt, eq;
        if (mode == 1) { gt = el && (kk & gmask) >= gpref; eq = false; }
        else { gt = el && kk > prefix; eq = el && kk == prefix; }
        my_gt += __popc(__ballot_sync(0xffffffffu, gt));
        my_eq += __popc(__ballot_sync(0xffffffffu, eq));
    }
    if (lane == 0) { s.wcnt[0][warp] = my_gt; s.wcnt[1][warp] = my_eq; }
    __syncthreads();
    int gt_base = 0, eq_base = 0, gt_all = 0, eq_all = 0;
    for (int w = 0; w < nw; ++w) {
        if (w < warp) { gt_base += s.wcnt[0][w]; eq_base += s.wcnt[1][w]; }
        gt_all += s.wcnt[0][w];
        eq_all += s.wcnt[1][w];
    }
    // Picks in earlier warps: their greater entries and their share of ties.
    const int out_base = gt_base + min(eq_base, need);
    // Pass B: write picks in index order to the candidate list.
    int out = out_base, eq_seen = eq_base;
    for (int base = w0; base < w1; base += 32) {
        const int i = base + lane;
        const bool el = i < w1 && eligible(i);
        const uint32_t kk = el ? key(i) : 0u;
        bool gt, eq;
        if (mode == 1) { gt = el && (kk & gmask) >= gpref; eq = false; }
        else { gt = el && kk > prefix; eq = el && kk == prefix; }
        const unsigned em = __ballot_sync(0xffffffffu, eq);
        const int my_rank = eq_seen + __popc(em & lanemask_lt());
        const bool pick = gt || (eq && my_rank < need);
        const unsigned pm = __ballot_sync(0xffffffffu, pick);
        if (pick) {
            const int at = out + __popc(pm & lanemask_lt());
            if (at < kTopkCap) { s.cand_idx[at] = i; s.cand_key[at] = kk; }
        }
        out += __popc(pm);
        eq_seen += __popc(em);
    }
    __syncthreads();
    // Mode 1 gathers at most kTopkCap entries; mode 2 takes exactly k.
    const int m_cand = min(kTopkCap, gt_all + (mode == 2 ? min(need, eq_all) : 0));
    // Rank the candidates by (key desc, index asc); keep the first k.
    const int m = min(k, m_cand);
    for (int c = tid; c < m_cand; c += nt) {
        const uint32_t kc = s.cand_key[c];
        const int ic = s.cand_idx[c];
        int r = 0;
        for (int j = 0; j < m_cand; ++j) {
            const uint32_t kj = s.cand_key[j];
            r += (kj > kc) || (kj == kc && s.cand_idx[j] < ic);
        }
        if (r < m) { out_idx[r] = ic; out_key[r] = kc; }
    }
    __syncthreads();
    return m;
}

}  // namespace pk
