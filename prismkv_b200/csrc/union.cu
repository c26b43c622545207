// Budgeted bucket union: the greedy skip-overflow rule of
// src/prismkv/core.py:152-164, with the union held as a shared-memory bitmap
// over the unit's history and compacted to ascending token ids by a block
// scan (the order of core.py:164's chosen.nonzero()).
//
// Candidate bucket i is accepted iff its tokens not yet chosen fit the
// remaining budget.  The kernel computes that sequential rule exactly in two
// phases, with the whole block working on every step:
//   1. the prefix of buckets accepted before the first skip (i*) is found by
//      galloping probes: a probe ORs a range of lists into the bitmap at once
//      and counts the bits it turned on (atomicOr returns the old word, so a
//      token shared by several lists of the range is counted once); if the
//      count overflows the budget the probe's bits are turned off again (each
//      staged entry that turned a bit on carries a flag), and the range
//      halves.  Ranges of more than one bucket run on lists staged in shared
//      memory; a one-bucket probe counts its tokens missing from the bitmap.
//   2. after i*, the tail: each remaining bucket's count of tokens missing
//      from the bitmap is taken once, and a chained hash maps every missing
//      token to the tail entries that hold it.  The block then walks the
//      buckets in order, a batch at a time: the next buckets whose exact
//      counts fit, for as long as their summed counts fit too, are all
//      accepted (each is what the one-at-a-time rule accepts), their tokens
//      are turned on, and each token turned on decrements the counts of the
//      later buckets holding it (two barriers per batch).  When the tail or
//      the hash does not fit in shared memory, rounds run instead: the
//      counts of the next 32 live buckets are retaken from the bitmap (a
//      warp each) and a batch of them is accepted the same way.  A bucket
//      whose count exceeds the remaining budget is dropped for good (its
//      count can shrink by at most what the budget shrinks).
#include "common.cuh"
#include "mma.cuh"

namespace pk {

constexpr int kUnionThreads = 1024;
constexpr int kMaxCand = 256;     // candidates per unit (G * k)
constexpr uint32_t kFlipFlag = 0x80000000u;

struct UnionSmem {
    int cand_bucket[kMaxCand];
    int cand_start[kMaxCand];
    int cand_len[kMaxCand];
    int cand_pre[kMaxCand + 1];   // exclusive prefix of the list lengths
    int newc[kMaxCand];
    unsigned char dead[kMaxCand]; // 1: dropped for good; 2: accepted by the walk or a round
    int cand_pre_win[32];         // the fallback rounds' window of live buckets
    int win_pre[33];              // exclusive prefix of the window lists' 256-entry chunks
    int red[64];
    int flags[8];
    int flip3[3];                 // accepted batches' new-token counts, rotating
};

__device__ __forceinline__ bool test_bit(const uint32_t* bm, int t) { return (bm[t >> 5] >> (t & 31)) & 1u; }
__device__ __forceinline__ void set_bit(uint32_t* bm, int t) { atomicOr(&bm[t >> 5], 1u << (t & 31)); }

// Sum of one non-negative int per thread, returned to every thread: one
// barrier, the warps' sums alternating between two halves of red[64] (a
// half is written again only two calls later, after every thread passed
// the barrier of the call in between).
__device__ __forceinline__ int block_sum(int v, int* red, int& parity) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int* half = red + 32 * parity;
    parity ^= 1;
    v = (int)__reduce_add_sync(0xffffffffu, (unsigned)v);
    if (lane == 0) half[warp] = v;
    __syncthreads();
    return (int)__reduce_add_sync(0xffffffffu, lane < nw ? (unsigned)half[lane] : 0u);
}

// One block of 32 consecutive candidates of a batch (lane = candidate):
// fit says the candidate's count v fits the room rem.  Returns the members:
// the fitting lanes before the first fitting lane at which the running sum
// of the fitting counts (run, carried across blocks, equal in every lane)
// exceeds rem; stop_lane is that lane, or -1 when the whole block joins.
// Counts below 2^26 take 32-bit reductions (a block whose fitting counts
// all fit needs no scan).
__device__ __forceinline__ unsigned batch_block(bool fit, int v, long long rem, long long& run, int& stop_lane) {
    const int lane = threadIdx.x & 31;
    const unsigned fm = __ballot_sync(0xffffffffu, fit);
    unsigned st;
    if (rem < (1ll << 26)) {
        const unsigned tot = __reduce_add_sync(0xffffffffu, fit ? (unsigned)v : 0u);
        if (run + (long long)tot <= rem) {
            run += tot;
            stop_lane = -1;
            return fm;
        }
        int x = fit ? v : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        st = __ballot_sync(0xffffffffu, fit && run + x > rem);
    } else {
        long long x = fit ? v : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const long long y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        st = __ballot_sync(0xffffffffu, fit && run + x > rem);
        if (!st) {
            run += __shfl_sync(0xffffffffu, x, 31);
            stop_lane = -1;
            return fm;
        }
    }
    stop_lane = __ffs(st) - 1;
    return fm & ((1u << stop_lane) - 1u);
}

struct UnionArgs {
    const int* offsets;
    const int* lens;
    const int* ids;
    int64_t ids_stride;
    const int* order;
    const int* n_order;
    int order_stride;
    const int* history;
    const long long* limit;
    int F;
    int max_history;
    int stage_cap;       // staged list entries
    int* out_ids;
    int64_t out_stride;
    int* out_count;
    int* features;
    int* n_features;
    long long* raw;
    int* status;
};

// One unit's union by one CTA of kUnionThreads threads; `dyn` is the
// block's dynamic shared memory (bitmap of max_history bits, then stage_cap
// staged entries), `sm` its static scratch.
__device__ __forceinline__ void union_unit(const UnionArgs& A, int u, uint32_t* dyn, UnionSmem& sm) {
    const int* __restrict__ offsets = A.offsets;
    const int* __restrict__ lens = A.lens;
    const int* __restrict__ ids = A.ids;
    const int64_t ids_stride = A.ids_stride;
    const int* __restrict__ order = A.order;
    const int* __restrict__ n_order = A.n_order;
    const int order_stride = A.order_stride;
    const int* __restrict__ history = A.history;
    const long long* __restrict__ limit = A.limit;
    const int F = A.F, max_history = A.max_history, stage_cap = A.stage_cap;
    int* __restrict__ out_ids = A.out_ids;
    const int64_t out_stride = A.out_stride;
    int* __restrict__ out_count = A.out_count;
    int* __restrict__ features = A.features;
    int* __restrict__ n_features = A.n_features;
    long long* __restrict__ raw = A.raw;
    int* __restrict__ status = A.status;
    const int tid = threadIdx.x, nt = blockDim.x;
    const int lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
    const int H = history[u];
    int red_parity = 0;   // block_sum's half of sm.red
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
    uint32_t* bm = dyn;                                                   // [W]
    uint32_t* stage = dyn + ((Wmax + 3) & ~3);                            // [stage_cap]
    const int n = min(n_order[u], kMaxCand);
    const long long lim = limit[u];
    const int* uid = ids + (int64_t)u * ids_stride;
    int* feat = features + (int64_t)u * order_stride;

    // The bitmap's words, zeroed up to a multiple of 4 (the compaction reads
    // 16 bytes at a time).
    for (int i = tid; i < ((W + 3) & ~3); i += nt) bm[i] = 0u;
    for (int c = tid; c < n; c += nt) {
        const int b = order[(int64_t)u * order_stride + c];
        sm.cand_bucket[c] = b;
        sm.cand_start[c] = offsets[(int64_t)u * (F + 1) + b];
        sm.cand_len[c] = lens[(int64_t)u * F + b];
        sm.dead[c] = 0;
    }
    __syncthreads();
    if (warp == 0) {
        int run = 0;
        for (int base = 0; base < n; base += 32) {
            const int c = base + lane;
            const int L = c < n ? sm.cand_len[c] : 0;
            const int inc = warp_inclusive_scan(L);
            if (c < n) sm.cand_pre[c] = run + inc - L;
            run += __shfl_sync(0xffffffffu, inc, 31);
        }
        if (lane == 0) sm.cand_pre[n] = run;
    }
    __syncthreads();

    // Staging window: buckets [ws0, ws1) whose lists lie back to back in
    // shared memory (entry i of bucket c at cand_pre[c] - cand_pre[ws0] + i).
    int ws0 = 0, ws1 = 0;
    auto stage_from = [&](int c0) {
        // Every warp finds the same window end (the first bucket whose list
        // would end past stage_cap); copies are asynchronous.
        const int base = sm.cand_pre[c0];
        int c1 = n;
        for (int b = c0 + 1; b <= n; b += 32) {
            const int c = b + lane;
            const bool over = c <= n && sm.cand_pre[c] - base > stage_cap;
            const unsigned om = __ballot_sync(0xffffffffu, over);
            if (om) {
                c1 = b + __ffs(om) - 2;
                break;
            }
        }
        for (int c = c0 + warp; c < c1; c += nw) {
            const int off = sm.cand_pre[c] - base;
            const int L = sm.cand_len[c];
            const int* src = uid + sm.cand_start[c];
            for (int i = lane; i < L; i += 32) cp_async_4(smem_addr(stage + off + i), src + i);
        }
        cp_async_wait_all();
        __syncthreads();
        ws0 = c0;
        ws1 = c1;
    };
    // Token i of bucket c (flag bit masked off).
    auto token = [&](int c, int i) -> int {
        if (c >= ws0 && c < ws1) return (int)(stage[sm.cand_pre[c] - sm.cand_pre[ws0] + i] & ~kFlipFlag);
        return uid[sm.cand_start[c] + i];
    };
    // Tokens of bucket c not in the bitmap (lists hold distinct tokens).
    auto missing = [&](int c) -> int {
        const int L = sm.cand_len[c];
        int m = 0;
        for (int i = tid; i < L; i += nt) {
            const int t = token(c, i);
            m += ((unsigned)t < (unsigned)H && !test_bit(bm, t)) ? 1 : 0;
        }
        return block_sum(m, sm.red, red_parity);
    };
    auto or_bucket = [&](int c) {
        const int L = sm.cand_len[c];
        for (int i = tid; i < L; i += nt) {
            const int t = token(c, i);
            if ((unsigned)t < (unsigned)H) set_bit(bm, t);
        }
    };
    // Calls fn(t) for every token of bucket c from one warp (lanes take
    // consecutive entries): a staged list from shared memory, any other from
    // global memory with eight loads a lane in flight (entries past the list
    // give t = -1).
    auto warp_tokens = [&](int c, auto&& fn) {
        const int L = sm.cand_len[c];
        if (c >= ws0 && c < ws1) {
            const uint32_t* src = stage + (sm.cand_pre[c] - sm.cand_pre[ws0]);
            for (int i = lane; i < L; i += 32) fn((int)(src[i] & ~kFlipFlag));
        } else {
            const int* src = uid + sm.cand_start[c];
            for (int i0 = 0; i0 < L; i0 += 256) {
                int tk[8];
#pragma unroll
                for (int b = 0; b < 8; ++b) {
                    const int i = i0 + 32 * b + lane;
                    tk[b] = i < L ? __ldg(src + i) : -1;
                }
#pragma unroll
                for (int b = 0; b < 8; ++b) fn(tk[b]);
            }
        }
    };
    stage_from(0);

    const long long raw_total = sm.cand_pre[n];
    long long raw_acc = 0;
    int nf = 0;
    if (raw_total <= lim) {
        // Every candidate fits whatever the overlap: the unbudgeted union.
        for (int c = warp; c < n; c += nw)
            warp_tokens(c, [&](int t) {
                if ((unsigned)t < (unsigned)H) set_bit(bm, t);
            });
        for (int c = tid; c < n; c += nt) feat[c] = sm.cand_bucket[c];
        nf = n;
        raw_acc = raw_total;
    } else {
        // ---- 1. the prefix accepted before i*.  Buckets whose lists, counted
        // with repeats, fit the budget are accepted whatever the overlap:
        // they are ORed in one pass.
        int sure = n;
        for (int b = 0; b < n; b += 32) {
            const int c = b + lane;
            const unsigned om = __ballot_sync(0xffffffffu, c < n && (long long)sm.cand_pre[c + 1] > lim);
            if (om) {
                sure = b + __ffs(om) - 1;
                break;
            }
        }
        int flips = 0;
        auto flip = [&](int t) {
            if ((unsigned)t < (unsigned)H) {
                const uint32_t bit = 1u << (t & 31);
                flips += (atomicOr(&bm[t >> 5], bit) & bit) ? 0 : 1;
            }
        };
        if (ws0 == 0 && sure <= ws1) {
            // Staged: the prefix's entries are one contiguous run, shared
            // evenly by all threads (a long list is not left to one warp).
            const int e1 = sm.cand_pre[sure];
            for (int e = tid; e < e1; e += nt) flip((int)(stage[e] & ~kFlipFlag));
        } else {
            for (int c = warp; c < sure; c += nw) warp_tokens(c, flip);
        }
        long long count = block_sum(flips, sm.red, red_parity);
        // Galloping probes from there; the first range is sized by the
        // overlap seen so far (tokens per listed entry).
        int lo = sure, fail_hi = n + 1, istar = n;
        int step = 8;
        bool predicted = false;
        if (sure > 0 && sure < n) {
            // Predicted i*: the first bucket whose entries, thinned by the
            // ratio seen so far, exceed the room left.
            const double ratio = (double)count / (double)max(1, sm.cand_pre[sure]);
            const double room = (double)(lim - count) / fmax(ratio, 1e-3);
            int c = n;
            for (int b = sure; b < n; b += 32) {
                const int cc = b + lane;
                const unsigned om = __ballot_sync(
                    0xffffffffu, cc < n && (double)(sm.cand_pre[cc + 1] - sm.cand_pre[sure]) > room);
                if (om) {
                    c = b + __ffs(om) - 1;
                    break;
                }
            }
            step = max(1, c - sure);
            predicted = true;
        }
        __syncthreads();
        while (lo < n) {
            if (fail_hi == lo + 1) { istar = lo; break; }
            int hi = min(min(lo + step, fail_hi - 1), n);
            if (hi > lo + 1 && hi > ws1) {
                if (lo >= ws1) stage_from(lo);
                hi = max(lo + 1, min(hi, ws1));
            }
            if (hi == lo + 1) {
                const int m = missing(lo);
                if (count + m <= lim) {
                    or_bucket(lo);
                    count += m;
                    lo = hi;
                    step = predicted ? 1 : step * 2;
                    predicted = false;
                    __syncthreads();
                } else {
                    istar = lo;
                    break;
                }
            } else {
                const int e0 = sm.cand_pre[lo] - sm.cand_pre[ws0], e1 = sm.cand_pre[hi] - sm.cand_pre[ws0];
                int flips = 0;
                for (int e = e0 + tid; e < e1; e += nt) {
                    const uint32_t t = stage[e] & ~kFlipFlag;
                    if (t < (uint32_t)H) {
                        const uint32_t bit = 1u << (t & 31);
                        if (!(atomicOr(&bm[t >> 5], bit) & bit)) {
                            stage[e] = t | kFlipFlag;
                            ++flips;
                        }
                    }
                }
                const int m = block_sum(flips, sm.red, red_parity);
                if (count + m <= lim) {
                    count += m;
                    lo = hi;
                    step = predicted ? 1 : step * 2;
                    predicted = false;
                } else {
                    for (int e = e0 + tid; e < e1; e += nt) {
                        const uint32_t t = stage[e];
                        if (t & kFlipFlag) {
                            const uint32_t tt = t & ~kFlipFlag;
                            stage[e] = tt;
                            atomicAnd(&bm[tt >> 5], ~(1u << (tt & 31)));
                        }
                    }
                    fail_hi = hi;
                    step = max(1, (hi - lo) / 2);
                    predicted = false;
                }
                __syncthreads();
            }
        }
        for (int c = tid; c < istar; c += nt) feat[c] = sm.cand_bucket[c];
        nf = istar;
        raw_acc = sm.cand_pre[istar];
        // ---- 2. after the first skipped bucket.
        int cpos = istar + 1;
        if (cpos < n && (cpos < ws0 || cpos >= ws1)) stage_from(cpos);
        // Preferred: one warp walks the remaining buckets in order with each
        // bucket's exact count of tokens missing from the bitmap, kept exact
        // by a multimap token -> tail entries (a chained hash over the
        // entries whose token is still missing): accepting a bucket
        // decrements the count of every later bucket holding a token it
        // added.  It needs the tail staged and room for the multimap after
        // the staged lists; otherwise the rounds below run instead.
        // Chain heads: about one per tail entry (only entries whose token is
        // still missing are chained), fewer if space is short.
        const int T = cpos < n ? sm.cand_pre[n] - sm.cand_pre[cpos] : 0;
        const int used = ws1 > ws0 ? sm.cand_pre[ws1] - sm.cand_pre[ws0] : 0;
        int hb_bits = 8;
        while (hb_bits < 16 && (1 << hb_bits) < T) ++hb_bits;
        while (hb_bits > 8 && used + (1 << hb_bits) + T + (T + 3) / 4 > stage_cap) --hb_bits;
        const int need = (1 << hb_bits) + T + (T + 3) / 4;
        if (cpos < n && ws1 == n && cpos >= ws0 && used + need <= stage_cap) {
            int* heads = reinterpret_cast<int*>(stage + used);
            int* nxt = heads + (1 << hb_bits);
            unsigned char* own = reinterpret_cast<unsigned char*>(nxt + T);
            const uint32_t* tail = stage + (sm.cand_pre[cpos] - sm.cand_pre[ws0]);
            for (int i = tid; i < (1 << hb_bits); i += nt) heads[i] = -1;
            __syncthreads();
            auto slot = [&](uint32_t t) { return (int)((t * 2654435761u) >> (32 - hb_bits)); };
            // Every entry's bucket (own), and the counts zeroed; then one
            // flat pass over the tail's entries shared evenly by all threads:
            // an entry whose token is missing is chained, and the lanes of a
            // warp holding entries of one bucket add their missing tokens to
            // its count with one shared-memory atomic.
            for (int c = cpos + warp; c < n; c += nw) {
                const int L = sm.cand_len[c];
                const int e0 = sm.cand_pre[c] - sm.cand_pre[cpos];
                for (int i = lane; i < L; i += 32) own[e0 + i] = (unsigned char)c;
                if (lane == 0) sm.newc[c] = 0;
            }
            __syncthreads();
            for (int base = warp * 32; base < T; base += nt) {
                const int e = base + lane;
                int c = -1;
                bool miss = false;
                if (e < T) {
                    c = own[e];
                    const uint32_t t = tail[e] & ~kFlipFlag;
                    if (t < (uint32_t)H && !test_bit(bm, (int)t)) {
                        miss = true;
                        nxt[e] = atomicExch(&heads[slot(t)], e);
                    }
                }
                const unsigned grp = __match_any_sync(0xffffffffu, c);
                const unsigned mm = __ballot_sync(0xffffffffu, miss);
                if (c >= 0 && lane == __ffs(grp) - 1) {
                    const int k2 = __popc(grp & mm);
                    if (k2) atomicAdd(&sm.newc[c], k2);
                }
            }
            if (tid == 0) sm.flip3[0] = sm.flip3[1] = sm.flip3[2] = 0;
            __syncthreads();
            // The walk accepts a batch of buckets per step: from c on, the
            // buckets whose exact counts fit the room left (rem), in order,
            // for as long as their summed counts fit rem too.  Each member is
            // what the one-at-a-time rule accepts: at its turn its count is at
            // most its count now (counts only shrink), and the room left is at
            // least rem less the earlier members' counts now.  A bucket passed
            // over because its count exceeds rem never fits later (a count
            // shrinks by at most what the room shrinks).  Warp 0 finds the
            // batch [c, cend); the block adds its tokens, and for each token
            // it turns on decrements the counts of the buckets from cend on
            // that hold it.  The members' counts are not touched meanwhile,
            // so every thread tells a member by its count.  Two barriers per
            // batch; the exact growth of the union is the number of bits the
            // batch turned on.
            long long cnt = count;
            for (int c = cpos, it = 0; c < n; ++it) {
                const long long rem = lim - cnt;
                if (warp == 0) {
                    long long run = 0;
                    int cend = n, nadd = 0;
                    for (int b = c; b < n; b += 32) {
                        const int cc = b + lane;
                        const int v = cc < n ? sm.newc[cc] : 0;
                        int stop_lane;
                        const unsigned mem = batch_block(cc < n && (long long)v <= rem, v, rem, run, stop_lane);
                        if ((mem >> lane) & 1u) {
                            feat[nf + nadd + __popc(mem & ((1u << lane) - 1u))] = sm.cand_bucket[cc];
                            sm.dead[cc] = 2;
                        }
                        nadd += __popc(mem);
                        if (stop_lane >= 0) {
                            cend = b + stop_lane;
                            break;
                        }
                    }
                    if (lane == 0) {
                        sm.flags[4] = cend;
                        sm.flags[5] = nadd;
                    }
                }
                __syncthreads();
                const int cend = sm.flags[4];
                nf += sm.flags[5];
                int flips = 0;
                const int e_lo = sm.cand_pre[c] - sm.cand_pre[cpos], e_hi = sm.cand_pre[cend] - sm.cand_pre[cpos];
                for (int e = e_lo + tid; e < e_hi; e += nt) {
                    // Entries of buckets passed over, or of members with
                    // nothing to add, are skipped before their token is read.
                    const int oc0 = sm.newc[own[e]];
                    if (oc0 == 0 || (long long)oc0 > rem) continue;
                    const uint32_t t = tail[e] & ~kFlipFlag;
                    if (t >= (uint32_t)H) continue;
                    const uint32_t bit = 1u << (t & 31);
                    // A bit still off was off when the counts were taken, so
                    // the entry is chained.
                    if (bm[t >> 5] & bit) continue;
                    if (atomicOr(&bm[t >> 5], bit) & bit) continue;
                    ++flips;
                    for (int ce = heads[slot(t)]; ce >= 0; ce = nxt[ce]) {
                        const int oc = own[ce];
                        if (oc >= cend && (tail[ce] & ~kFlipFlag) == t) atomicSub(&sm.newc[oc], 1);
                    }
                }
                flips = warp_sum(flips);
                if (lane == 0 && flips) atomicAdd(&sm.flip3[it % 3], flips);
                if (tid == 0) sm.flip3[(it + 1) % 3] = 0;
                __syncthreads();
                cnt += sm.flip3[it % 3];
                c = cend;
            }
            cpos = n;
        }
        // Rounds over a window of the next 32 live buckets: their exact
        // counts against the bitmap, then a batch of those that fit is
        // accepted.  Every window member over the budget is dropped for good:
        // a count shrinks by at most what the remaining budget shrinks, so a
        // bucket over the budget now never fits later.  The window's lists
        // are cut into chunks of 256 entries dealt to the warps (a long list
        // is shared by several warps); a chunk's tokens are read eight a lane
        // at a time and, when every warp holds at most one chunk, kept in
        // registers for the accepted buckets' OR.
        while (cpos < n) {
            if (warp == 0) {
                // The window: the next 32 buckets from cpos that are not dead,
                // their chunk counts' prefix, their counts zeroed.
                int got = 0;
                for (int base = cpos; base < n && got < 32; base += 32) {
                    const int c = base + lane;
                    const bool live = c < n && !sm.dead[c];
                    const unsigned lm = __ballot_sync(0xffffffffu, live);
                    const int at = got + __popc(lm & ((1u << lane) - 1u));
                    if (live && at < 32) sm.cand_pre_win[at] = c;
                    got += __popc(lm);
                }
                const int nwin = min(got, 32);
                __syncwarp();
                const int c = lane < nwin ? sm.cand_pre_win[lane] : -1;
                const int nch = c >= 0 ? (sm.cand_len[c] + 255) >> 8 : 0;
                sm.win_pre[lane + 1] = warp_inclusive_scan(nch);
                if (c >= 0) sm.newc[c] = 0;
                if (lane == 0) {
                    sm.win_pre[0] = 0;
                    sm.flags[1] = nwin;
                }
            }
            __syncthreads();
            const int nwin = sm.flags[1];
            if (nwin == 0) break;
            const int nchunks = sm.win_pre[nwin];
            // Window slot of chunk q: the last slot whose chunks start at or
            // before q (slots without entries own no chunk).
            auto chunk_slot = [&](int q) {
                int lo = 0, hi = nwin;
                while (hi - lo > 1) {
                    const int mid = (lo + hi) >> 1;
                    if (sm.win_pre[mid] <= q) lo = mid;
                    else hi = mid;
                }
                return lo;
            };
            auto chunk_tokens = [&](int q, int s, int (&tk)[8]) {
                const int c = sm.cand_pre_win[s];
                const int L = sm.cand_len[c];
                const int i0 = (q - sm.win_pre[s]) << 8;
                if (c >= ws0 && c < ws1) {
                    const uint32_t* src = stage + (sm.cand_pre[c] - sm.cand_pre[ws0]);
#pragma unroll
                    for (int b = 0; b < 8; ++b) {
                        const int i = i0 + 32 * b + lane;
                        tk[b] = i < L ? (int)(src[i] & ~kFlipFlag) : -1;
                    }
                } else {
                    const int* src = uid + sm.cand_start[c];
#pragma unroll
                    for (int b = 0; b < 8; ++b) {
                        const int i = i0 + 32 * b + lane;
                        tk[b] = i < L ? __ldg(src + i) : -1;
                    }
                }
            };
            const bool keep = nchunks <= nw;
            int tk[8];
            int my_slot = -1;
            for (int q = warp; q < nchunks; q += nw) {
                const int s = chunk_slot(q);
                chunk_tokens(q, s, tk);
                int m = 0;
#pragma unroll
                for (int b = 0; b < 8; ++b) m += ((unsigned)tk[b] < (unsigned)H && !test_bit(bm, tk[b])) ? 1 : 0;
                m = (int)__reduce_add_sync(0xffffffffu, (unsigned)m);
                if (lane == 0 && m) atomicAdd(&sm.newc[sm.cand_pre_win[s]], m);
                my_slot = s;
            }
            if (tid == 0) sm.flip3[0] = 0;
            __syncthreads();
            // The batch, as in the walk: the window's buckets that fit, in
            // order, while their summed counts fit the room left.  Members
            // over the room are dropped for good; the next window starts at
            // the first bucket that fits alone but not after the batch.
            if (warp == 0) {
                const long long rem = lim - count;
                const int c = lane < nwin ? sm.cand_pre_win[lane] : n;
                const int v = lane < nwin ? sm.newc[c] : 0;
                const bool fits = lane < nwin && (long long)v <= rem;
                long long run = 0;
                int stop_lane;
                const unsigned mem = batch_block(fits, v, rem, run, stop_lane);
                if (lane < nwin && !fits) sm.dead[c] = 1;
                if ((mem >> lane) & 1u) {
                    feat[nf + __popc(mem & ((1u << lane) - 1u))] = sm.cand_bucket[c];
                    sm.dead[c] = 2;
                }
                // Members with tokens to add.
                const unsigned add = __ballot_sync(0xffffffffu, ((mem >> lane) & 1u) && v > 0);
                if (lane == 0) {
                    sm.flags[0] = (int)mem;
                    sm.flags[3] = (int)add;
                    sm.flags[2] = stop_lane >= 0 ? sm.cand_pre_win[stop_lane] : sm.cand_pre_win[nwin - 1] + 1;
                }
            }
            __syncthreads();
            const unsigned mem = (unsigned)sm.flags[0];
            const unsigned add = (unsigned)sm.flags[3];
            nf += __popc(mem);
            cpos = sm.flags[2];
            int flips = 0;
            if (add) {
                for (int q = warp; q < nchunks; q += nw) {
                    const int s = keep ? my_slot : chunk_slot(q);
                    if (!((add >> s) & 1u)) continue;
                    if (!keep) chunk_tokens(q, s, tk);
#pragma unroll
                    for (int b = 0; b < 8; ++b) {
                        const int t = tk[b];
                        if ((unsigned)t < (unsigned)H) {
                            const uint32_t bit = 1u << (t & 31);
                            flips += (atomicOr(&bm[t >> 5], bit) & bit) ? 0 : 1;
                        }
                    }
                }
            }
            flips = (int)__reduce_add_sync(0xffffffffu, (unsigned)flips);
            if (lane == 0 && flips) atomicAdd(&sm.flip3[0], flips);
            __syncthreads();
            count += sm.flip3[0];
        }
    }
    __syncthreads();

    // Compaction: each warp owns a contiguous run of words, each lane
    // reading four consecutive words (16 bytes: conflict-free) of a
    // 128-word chunk; a count pass, the warps' offsets, then the emit pass
    // in word order.  Words past W are zero.
    const int W4 = (W + 3) & ~3;
    const int wper = ((W4 + nw - 1) / nw + 127) & ~127;
    const int ww0 = min(W4, warp * wper), ww1 = min(W4, ww0 + wper);
    int wpop = 0;
    for (int base = ww0; base < ww1; base += 128) {
        const int w = base + 4 * lane;
        if (w < ww1) {
            const uint4 m4 = *reinterpret_cast<const uint4*>(bm + w);
            wpop += __popc(m4.x) + __popc(m4.y) + __popc(m4.z) + __popc(m4.w);
        }
    }
    wpop = warp_sum(wpop);
    if (lane == 0) sm.red[warp] = wpop;
    __syncthreads();
    const int cw = lane < nw ? sm.red[lane] : 0;
    int at = (int)__reduce_add_sync(0xffffffffu, lane < warp ? (unsigned)cw : 0u);
    const int total = (int)__reduce_add_sync(0xffffffffu, (unsigned)cw);
    int* dst = out_ids + (int64_t)u * out_stride;
    bool overflow = false;
    for (int base = ww0; base < ww1; base += 128) {
        const int w = base + 4 * lane;
        const uint4 m4 = w < ww1 ? *reinterpret_cast<const uint4*>(bm + w) : make_uint4(0u, 0u, 0u, 0u);
        const uint32_t mw[4] = {m4.x, m4.y, m4.z, m4.w};
        const int c = __popc(m4.x) + __popc(m4.y) + __popc(m4.z) + __popc(m4.w);
        const int inc = warp_inclusive_scan(c);
        int pos = at + inc - c;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t m = mw[j];
            while (m) {
                const int bit = __ffs(m) - 1;
                m &= m - 1;
                if (pos < out_stride) dst[pos] = (w + j) * 32 + bit;
                else overflow = true;
                ++pos;
            }
        }
        at += __shfl_sync(0xffffffffu, inc, 31);
    }
    if (overflow && status) atomicOr(status, PK_STATUS_OUT_FULL);
    if (warp == 0) {
        // Raw sizes of the buckets the walk or the rounds accepted (marked 2).
        long long r = 0;
        for (int c = lane; c < n; c += 32)
            if (sm.dead[c] == 2) r += sm.cand_len[c];
        raw_acc += warp_sum(r);
    }
    if (tid == 0) {
        out_count[u] = total;
        n_features[u] = nf;
        raw[u] = raw_acc;
    }
}

__global__ void __launch_bounds__(kUnionThreads) union_kernel(UnionArgs A) {
    extern __shared__ __align__(16) uint32_t dyn[];
    __shared__ UnionSmem sm;
    union_unit(A, blockIdx.x, dyn, sm);
}

}  // namespace pk

using namespace pk;

static int union_launch(uint64_t offsets, uint64_t lens, uint64_t ids, int64_t ids_stride, uint64_t order,
                        uint64_t n_order, int order_stride, uint64_t history, uint64_t limit, int U, int F,
                        int max_history, uint64_t out_ids, int64_t out_stride, uint64_t out_count, uint64_t features,
                        uint64_t n_features, uint64_t raw, uint64_t status, uint64_t stream) {
    if (U < 1 || F < 1 || max_history < 0 || order_stride < 1 || out_stride < 0 || ids_stride < 0) return PK_ERR_ARG;
    if (!offsets || !lens || !ids || !order || !n_order || !history || !limit || !out_ids || !out_count ||
        !features || !n_features || !raw)
        return PK_ERR_ARG;
    const int Wmax = (max_history + 31) / 32;
    const size_t bitmap = (size_t)((Wmax + 3) & ~3) * 4;
    // Dynamic shared memory: all a block may hold (227 KB) less the static
    // scratch, rounded down to KB.
    const size_t cap = (227 * 1024 - sizeof(UnionSmem)) / 1024 * 1024;
    // The bitmap, then as many staged list entries as fit (at least 2048).
    if (bitmap + 2048 * 4 > cap) return PK_ERR_UNSUPPORTED;
    const int stage_cap = (int)((cap - bitmap) / 4);
    UnionArgs A;
    A.offsets = (const int*)offsets; A.lens = (const int*)lens; A.ids = (const int*)ids; A.ids_stride = ids_stride;
    A.order = (const int*)order; A.n_order = (const int*)n_order; A.order_stride = order_stride;
    A.history = (const int*)history; A.limit = (const long long*)limit; A.F = F; A.max_history = max_history;
    A.stage_cap = stage_cap; A.out_ids = (int*)out_ids; A.out_stride = out_stride;
    A.out_count = (int*)out_count; A.features = (int*)features; A.n_features = (int*)n_features;
    A.raw = (long long*)raw; A.status = (int*)status;
    cudaFuncSetAttribute(union_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cap);
    union_kernel<<<U, kUnionThreads, cap, (cudaStream_t)stream>>>(A);
    PK_CHECK_LAUNCH();
    return PK_OK;
}

extern "C" int pk_union(uint64_t offsets, uint64_t lens, uint64_t ids, int64_t ids_stride, uint64_t order,
                        uint64_t n_order, int order_stride, uint64_t history, uint64_t limit, int U, int F,
                        int max_history, uint64_t out_ids, int64_t out_stride, uint64_t out_count,
                        uint64_t features, uint64_t n_features, uint64_t raw, uint64_t status, uint64_t stream) {
    return union_launch(offsets, lens, ids, ids_stride, order, n_order, order_stride, history, limit, U, F,
                        max_history, out_ids, out_stride, out_count, features, n_features, raw, status, stream);
}
