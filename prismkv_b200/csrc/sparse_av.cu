// Sparse attention over the selected history rows plus the dense generated
// tail: softmax((Q K_rows^T)/sqrt(d)) V_rows for the G query heads of a unit
// (src/prismkv/core.py:170-183), split across CTAs along the row list with an
// exact log-sum-exp merge (the split-KV scheme of kernels/ppu_8b/av_tuned.cu).
//
// bf16 path: a CTA of four warps streams its split's rows in tiles of 64 K
// rows and 64 V rows, three stages deep.  Each warp gathers its own 16 rows of
// every tile with 16-byte cp.async (rows addressed through the id list, staged
// in shared memory).  For G <= 8 heads, when a unit's splits span several
// clusters its tiles are dealt to the S split CTAs round robin (split s takes
// tiles s, s + S, ...), so a split's tiles are known before the unit's row
// count and their ids are staged in parallel with it; otherwise each split is
// a contiguous run of tiles.  The
// warp also computes on its rows alone, so the warps pipeline independently
// (no CTA barrier per tile): its 16 key rows fill the M = 16 of mma.sync
// m16n8k16 and the heads its N = 8 (S^T = K Q^T, then O^T += V^T P^T with
// P^T formed by movmatrix).  For 9..16 heads the heads fill M, with a CTA
// barrier per tile.  Softmax is online in fp32 and P enters the PV product in
// bf16.  The split CTAs of a unit merge in thread-block clusters of up to 8
// through distributed shared memory; with more splits than one cluster holds,
// each cluster's merged state goes to global memory and, per output slice,
// the last cluster to finish merges the clusters' states.  Without a cluster
// the last CTA of a unit merges the split partials from global memory.  The
// _append entry point fuses the decode KV append: the unit's new rows are
// attended in place of its newest tail row and written into the cache by its
// first split CTA.
#include <cooperative_groups.h>

#include <mutex>

#include "common.cuh"

namespace pk {

constexpr int kAvD = 128;
constexpr int kAvThreads = 128;
constexpr int kAvTile = 64;
constexpr int kAvStages = 3;
constexpr int kAvRowBytes = kAvD * 2;
constexpr int kAvStageBytes = kAvTile * kAvRowBytes * 2;   // K + V
constexpr int kAvMaxG = 16;
constexpr int kAvIdsCap = 2048;   // row ids staged per CTA (longer splits read the rest directly)
constexpr int kAvMaxCluster = 16; // splits merged through distributed shared memory
constexpr int kAvGroupMax = 8;    // CTAs per cluster when clusters are merged through global memory
constexpr int kAvCounters = 8;    // arrival counters per unit (one per cluster rank)
constexpr float kLog2e = 1.4426950408889634f;

struct AvParams {
    const void* q;
    const void* k;
    const void* v;
    int kv_heads;
    int64_t kv_batch_stride, kv_head_stride, kv_row_stride;
    const int* ids;
    int64_t ids_stride;
    const int* count;
    const int* history;
    const int* length;
    int G, S;
    int C;          // CTAs per cluster (G <= 8 kernel; S is a multiple of C)
    int rr;         // G <= 8 kernel: tiles dealt round robin (several clusters per unit)
    float* part;    // [U*G, S, D+2] split partials (log2 domain); cluster states [U, S/C, 3, G*D]
    int* done;      // [U, kAvCounters] arrival counters
    void* out;      // [U, G, D] (dtype of q)
    float* xpart;   // [U*G, D+2] exported partial (natural-log m), or null
    // Fused decode append, or null: unit u's new K/V rows k_new/v_new[u, D]
    // are attended in place of cache row length[u] - 1 (the newest tail row)
    // and written there by the unit's first split CTA.
    const void* k_new;
    const void* v_new;
};

// The row position the fused append fills (-1: none).
__device__ __forceinline__ int fresh_row(const AvParams& p, int H, int len) {
    return p.k_new && len > H ? len - 1 : -1;
}

// The unit's first split CTA writes its new K/V rows into the cache at the
// fresh position with 16-byte vectors (nothing in this launch reads that
// cache row: the loaders take it from k_new/v_new).
template <typename T>
__device__ __forceinline__ void append_fresh_row(const AvParams& p, int u, int64_t ubase, int fresh) {
    if (fresh < 0 || blockIdx.x != 0) return;
    constexpr int kVecs = kAvD * (int)sizeof(T) / 16;
    const int tid = threadIdx.x;
    if (tid >= 2 * kVecs) return;
    const bool isv = tid >= kVecs;
    const int j = isv ? tid - kVecs : tid;
    const uint4* src = reinterpret_cast<const uint4*>((const T*)(isv ? p.v_new : p.k_new) + (int64_t)u * kAvD);
    uint4* dst = reinterpret_cast<uint4*>((T*)(isv ? p.v : p.k) + ubase + (int64_t)fresh * p.kv_row_stride);
    dst[j] = src[j];
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
    const int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(n));
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(dst), "l"(src));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 t = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&t);
}
// Transpose of an 8x8 16-bit matrix held as the warp's mma fragment.
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(y) : "r"(x));
    return y;
}

// Byte offset of (row, 16-byte chunk) inside a 64-row x 256-byte tile, the
// chunk index XOR-swizzled by the row so ldmatrix is bank-conflict free.
__device__ __forceinline__ uint32_t tile_off(int row, int chunk) {
    return (uint32_t)(row * kAvRowBytes + ((chunk ^ (row & 7)) << 4));
}

template <typename OT>
__device__ __forceinline__ OT to_out(float x);
template <>
__device__ __forceinline__ float to_out<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 to_out<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// Combine per-warp (m, l, o) states held in shared memory into this CTA's
// state, then either finish (single split) or store the split partial and
// let the last CTA of the unit merge.  m is in log2 units.
template <typename OT>
__device__ void av_finish(const AvParams& p, int u, int s, float* red, int nwarps) {
    const int G = p.G, S = p.S, tid = threadIdx.x;
    const float* rm = red;
    const float* rl = red + nwarps * kAvMaxG;
    const float* ro = red + 2 * nwarps * kAvMaxG;
    __shared__ int is_last;
    const int dim = tid;  // kAvThreads == kAvD
    for (int h = 0; h < G; ++h) {
        float M = -INFINITY;
        for (int w = 0; w < nwarps; ++w) M = fmaxf(M, rm[w * kAvMaxG + h]);
        float L = 0.f, O = 0.f;
        for (int w = 0; w < nwarps; ++w) {
            const float mw = rm[w * kAvMaxG + h];
            const float sc = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
            L = fmaf(sc, rl[w * kAvMaxG + h], L);
            O = fmaf(sc, ro[(w * kAvMaxG + h) * kAvD + dim], O);
        }
        const int64_t uh = (int64_t)u * G + h;
        if (S == 1) {
            if (p.xpart) {
                float* xp = p.xpart + uh * (kAvD + 2);
                if (dim == 0) { xp[0] = M == -INFINITY ? -INFINITY : M / kLog2e; xp[1] = L; }
                xp[2 + dim] = O;
            } else {
                OT* o = (OT*)p.out + uh * kAvD;
                o[dim] = to_out<OT>(L > 0.f ? O / L : 0.f);
            }
        } else {
            float* pp = p.part + (uh * S + s) * (kAvD + 2);
            if (dim == 0) { pp[0] = M; pp[1] = L; }
            pp[2 + dim] = O;
        }
    }
    if (S == 1) return;
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = atomicAdd(&p.done[u * kAvCounters], 1) == S - 1;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    // Merge the unit's G x S split partials.  Every load is independent of
    // the others, so they are issued in parallel: first all (m, l) pairs into
    // shared memory (reusing `red`, whose per-warp states were consumed
    // above), then the o columns in batches of 16 per thread.  Within a head
    // the splits are still accumulated in ascending order.
    const int GS = G * S;
    float* wt = red;                       // [G*S] m, then merge weights
    float* lt = wt + GS;                   // [G*S] l
    float* Mh = lt + GS;                   // [G]
    float* Lh = Mh + G;                    // [G]
    const float* pu = p.part + (int64_t)u * GS * (kAvD + 2);
    for (int e = tid; e < GS; e += kAvThreads) {
        wt[e] = __ldcg(pu + (int64_t)e * (kAvD + 2));
        lt[e] = __ldcg(pu + (int64_t)e * (kAvD + 2) + 1);
    }
    __syncthreads();
    const int lane = tid & 31, warp = tid >> 5;
    for (int h = warp; h < G; h += kAvThreads / 32) {
        float M = -INFINITY;
        for (int j = lane; j < S; j += 32) M = fmaxf(M, wt[h * S + j]);
        M = warp_max(M);
        __syncwarp();
        float L = 0.f;
        for (int j = lane; j < S; j += 32) {
            const float mj = wt[h * S + j];
            const float sc = (mj == -INFINITY) ? 0.f : exp2f(mj - M);
            wt[h * S + j] = sc;
            L = fmaf(sc, lt[h * S + j], L);
        }
        L = warp_sum(L);
        if (lane == 0) { Mh[h] = M; Lh[h] = L; }
    }
    __syncthreads();
    auto emit = [&](int h, float O) {
        const int64_t uh = (int64_t)u * G + h;
        const float M = Mh[h], L = Lh[h];
        if (p.xpart) {
            float* xp = p.xpart + uh * (kAvD + 2);
            if (dim == 0) { xp[0] = M == -INFINITY ? -INFINITY : M / kLog2e; xp[1] = L; }
            xp[2 + dim] = O;
        } else {
            OT* o = (OT*)p.out + uh * kAvD;
            o[dim] = to_out<OT>(L > 0.f ? O / L : 0.f);
        }
    };
    constexpr int kBatch = 16;
    float O = 0.f;
    int hcur = 0;
    for (int e0 = 0; e0 < GS; e0 += kBatch) {
        float v[kBatch];
#pragma unroll
        for (int t = 0; t < kBatch; ++t)
            v[t] = e0 + t < GS ? __ldcg(pu + (int64_t)(e0 + t) * (kAvD + 2) + 2 + dim) : 0.f;
#pragma unroll
        for (int t = 0; t < kBatch; ++t) {
            const int e = e0 + t;
            if (e < GS) {
                const int h = e / S;
                if (h != hcur) { emit(hcur, O); O = 0.f; hcur = h; }
                O = fmaf(wt[e], v[t], O);
            }
        }
    }
    emit(hcur, O);
    if (tid == 0) p.done[u * kAvCounters] = 0;
}

// Cluster merge: the CTA combines its warps' states into shared memory
// (st: m[kAvMaxG], l[kAvMaxG], o[kAvMaxG][D]), then the cluster's CTAs share
// out the G*D outputs and each reads the S states of its outputs from the
// CTAs' shared memory, accumulating in split order (the same arithmetic as
// the global merge).  The second cluster barrier keeps every CTA's shared
// memory alive until all reads are done.
template <typename OT>
__device__ void av_finish_cluster(const AvParams& p, int u, int s, const float* red, int nwarps, float* st) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    const int G = p.G, S = p.S, tid = threadIdx.x;
    const float* rm = red;
    const float* rl = red + nwarps * kAvMaxG;
    const float* ro = red + 2 * nwarps * kAvMaxG;
    const int dim = tid;  // kAvThreads == kAvD
    for (int h = 0; h < G; ++h) {
        float M = -INFINITY;
        for (int w = 0; w < nwarps; ++w) M = fmaxf(M, rm[w * kAvMaxG + h]);
        float L = 0.f, O = 0.f;
        for (int w = 0; w < nwarps; ++w) {
            const float mw = rm[w * kAvMaxG + h];
            const float sc = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
            L = fmaf(sc, rl[w * kAvMaxG + h], L);
            O = fmaf(sc, ro[(w * kAvMaxG + h) * kAvD + dim], O);
        }
        if (dim == 0) { st[h] = M; st[kAvMaxG + h] = L; }
        st[2 * kAvMaxG + h * kAvD + dim] = O;
    }
    cluster.sync();
    for (int e = s * kAvThreads + tid; e < G * kAvD; e += S * kAvThreads) {
        const int h = e / kAvD, d = e % kAvD;
        float mj[kAvMaxCluster], lj[kAvMaxCluster], oj[kAvMaxCluster];
#pragma unroll
        for (int j = 0; j < kAvMaxCluster; ++j) {
            if (j < S) {
                const float* rst = cluster.map_shared_rank(st, j);
                mj[j] = rst[h];
                lj[j] = rst[kAvMaxG + h];
                oj[j] = rst[2 * kAvMaxG + h * kAvD + d];
            }
        }
        float M = -INFINITY;
#pragma unroll
        for (int j = 0; j < kAvMaxCluster; ++j)
            if (j < S) M = fmaxf(M, mj[j]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int j = 0; j < kAvMaxCluster; ++j) {
            if (j < S) {
                const float sc = (mj[j] == -INFINITY) ? 0.f : exp2f(mj[j] - M);
                L = fmaf(sc, lj[j], L);
                O = fmaf(sc, oj[j], O);
            }
        }
        const int64_t uh = (int64_t)u * G + h;
        if (p.xpart) {
            float* xp = p.xpart + uh * (kAvD + 2);
            if (d == 0) { xp[0] = M == -INFINITY ? -INFINITY : M / kLog2e; xp[1] = L; }
            xp[2 + d] = O;
        } else {
            OT* o = (OT*)p.out + uh * kAvD;
            o[d] = to_out<OT>(L > 0.f ? O / L : 0.f);
        }
    }
    cluster.sync();
}


// Output of one merged (u, h, d) state: the result, or the exported partial
// (natural-log m) for the sequence-sharded merge.
template <typename OT>
__device__ __forceinline__ void av_emit(const AvParams& p, int64_t uh, int d, float M, float L, float O) {
    if (p.xpart) {
        float* xp = p.xpart + uh * (kAvD + 2);
        if (d == 0) { xp[0] = M == -INFINITY ? -INFINITY : M / kLog2e; xp[1] = L; }
        xp[2 + d] = O;
    } else {
        OT* o = (OT*)p.out + uh * kAvD;
        o[d] = to_out<OT>(L > 0.f ? O / L : 0.f);
    }
}

// Push merge (used with the cluster launch of sparse_av_bf16_kernel): the
// C = p.C split CTAs of a cluster share out the unit's G*D output elements,
// element e belonging to cluster rank e / per.  Each CTA combines its warps'
// states, stores its (o) of every element and its (m, l) of every head into
// the owning CTA's receive buffer (pbuf: o_in[C][per], then ml_in[C][G][2]),
// and after one cluster barrier merges the C states of its own elements from
// its own shared memory, in rank order (remote stores instead of remote
// loads, one barrier).  The caller arrived on the cluster barrier at kernel
// start; the wait here, before the first remote store, makes sure every CTA
// of the cluster is running.  With one cluster per unit the merged states
// are the result.  With NC = S / C clusters, each owner stores its elements'
// cluster state (m, l, o) in global memory and counts itself in on its rank's
// arrival counter; the last of the NC owners of a slice merges the NC cluster
// states in cluster order and resets the counter.
template <typename OT>
__device__ void av_finish_push(const AvParams& p, int u, int s, const float* red, int nwarps, float* ml_loc,
                               float* pbuf) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    const int G = p.G, C = p.C, tid = threadIdx.x;
    const int j = (int)cluster.block_rank(), c = s / C, NC = p.S / C;
    const int GD = G * kAvD, per = (GD + C - 1) / C;
    float* o_in = pbuf;
    float* ml_in = pbuf + C * per;
    const float* rm = red;
    const float* rl = red + nwarps * kAvMaxG;
    const float* ro = red + 2 * nwarps * kAvMaxG;
    asm volatile("barrier.cluster.wait;\n" ::: "memory");
    const int dim = tid;  // kAvThreads == kAvD
    for (int h = 0; h < G; ++h) {
        float M = -INFINITY;
        for (int w = 0; w < nwarps; ++w) M = fmaxf(M, rm[w * kAvMaxG + h]);
        float L = 0.f, O = 0.f;
        for (int w = 0; w < nwarps; ++w) {
            const float mw = rm[w * kAvMaxG + h];
            const float sc = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
            L = fmaf(sc, rl[w * kAvMaxG + h], L);
            O = fmaf(sc, ro[(w * kAvMaxG + h) * kAvD + dim], O);
        }
        if (dim == 0) { ml_loc[2 * h] = M; ml_loc[2 * h + 1] = L; }
        const int e = h * kAvD + dim, owner = e / per;
        float* dst = cluster.map_shared_rank(o_in, owner);
        dst[j * per + (e - owner * per)] = O;
    }
    __syncthreads();
    for (int i = tid; i < 2 * G * C; i += kAvThreads) {
        const int r = i / (2 * G), jj = i % (2 * G);
        float* dst = cluster.map_shared_rank(ml_in, r);
        dst[j * 2 * G + jj] = ml_loc[jj];
    }
    cluster.sync();
    float* cst = p.part + (int64_t)(u * NC + c) * 3 * GD;   // this cluster's states [3][GD]
    for (int jj = tid; jj < per && j * per + jj < GD; jj += kAvThreads) {
        const int e = j * per + jj, h = e / kAvD, d = e % kAvD;
        float M = -INFINITY;
        for (int r = 0; r < C; ++r) M = fmaxf(M, ml_in[(r * G + h) * 2]);
        float L = 0.f, O = 0.f;
        for (int r = 0; r < C; ++r) {
            const float mr = ml_in[(r * G + h) * 2];
            const float sc = (mr == -INFINITY) ? 0.f : exp2f(mr - M);
            L = fmaf(sc, ml_in[(r * G + h) * 2 + 1], L);
            O = fmaf(sc, o_in[r * per + jj], O);
        }
        if (NC == 1) {
            av_emit<OT>(p, (int64_t)u * G + h, d, M, L, O);
        } else {
            cst[e] = M;
            cst[GD + e] = L;
            cst[2 * GD + e] = O;
        }
    }
    if (NC == 1) return;
    __shared__ int is_last;
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = atomicAdd(&p.done[u * kAvCounters + j], 1) == NC - 1;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    const float* ust = p.part + (int64_t)u * NC * 3 * GD;
    for (int jj = tid; jj < per && j * per + jj < GD; jj += kAvThreads) {
        const int e = j * per + jj, h = e / kAvD, d = e % kAvD;
        float M = -INFINITY;
        for (int r = 0; r < NC; ++r) M = fmaxf(M, __ldcg(ust + (int64_t)r * 3 * GD + e));
        float L = 0.f, O = 0.f;
        for (int r = 0; r < NC; ++r) {
            const float* sr = ust + (int64_t)r * 3 * GD;
            const float mr = __ldcg(sr + e);
            const float sc = (mr == -INFINITY) ? 0.f : exp2f(mr - M);
            L = fmaf(sc, __ldcg(sr + GD + e), L);
            O = fmaf(sc, __ldcg(sr + 2 * GD + e), O);
        }
        av_emit<OT>(p, (int64_t)u * G + h, d, M, L, O);
    }
    if (tid == 0) p.done[u * kAvCounters + j] = 0;
}

// Receive buffer of av_finish_push, in floats.
__host__ __device__ constexpr int av_push_floats(int G, int S) { return S * ((G * kAvD + S - 1) / S) + 2 * G * S; }

// G <= 8 heads.  Warp w owns rows [16w, 16w + 16) of every tile: it copies
// them in and computes on them, so each warp's stages are its own.  Split s
// takes a contiguous run of the unit's tiles, or, with several clusters per
// unit, the tiles s, s + S, s + 2S, ...
template <bool kCluster>
__global__ void __launch_bounds__(kAvThreads, 2)
sparse_av_bf16_kernel(AvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int s = blockIdx.x, u = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = p.G, S = p.S;
    if constexpr (kCluster) asm volatile("barrier.cluster.arrive.relaxed;\n" ::: "memory");
    const int* idp = p.ids + (int64_t)u * p.ids_stride;
    const __nv_bfloat16* qp = (const __nv_bfloat16*)p.q + (int64_t)u * G * kAvD;
    const int g = lane >> 2, q4 = lane & 3;
    // Q^T as the MMA B operand: n = head g, k = dims.
    uint32_t qb[8][2];
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
#pragma unroll
        for (int r = 0; r < 2; ++r)
            qb[kk][r] = g < G ? *reinterpret_cast<const uint32_t*>(qp + g * kAvD + kk * 16 + r * 8 + 2 * q4) : 0u;
    // Tile j of the split covers 64 consecutive list positions.  With
    // one cluster (or none) per unit the split is a contiguous run of whole
    // tiles [r0, r1); with several clusters (p.rr) the unit's tiles are
    // dealt round robin (split s takes tiles s, s + S, ...), so the split's
    // tiles are known before the unit's row count and their ids are staged
    // in parallel with it: each warp stages the ids of its own rows (16w ..
    // 16w + 15 of each tile) within the id row's stride (entries past the
    // count are not used).  Tiles past the staged ones (more than
    // kAvIdsCap / 64 per split) read their ids directly.
    int* sids = reinterpret_cast<int*>(smem + kAvStages * kAvStageBytes);
    constexpr int kStagedTiles = kAvIdsCap / kAvTile;
    const bool rr = p.rr != 0;
    // List position of row `row` of the split's tile j: base0 + j * tstep + row.
    int base0 = rr ? s * kAvTile : 0;
    const int tstep = rr ? S * kAvTile : kAvTile;
    if (rr) {
        const int64_t tiles_in_stride = (p.ids_stride + kAvTile - 1) / kAvTile;
        const int64_t jcan = s < tiles_in_stride ? (tiles_in_stride - 1 - s) / S + 1 : 0;
        const int jst = (int)(jcan < kStagedTiles ? jcan : kStagedTiles);
        for (int i = lane; i < jst * 16; i += 32) {
            const int j = i >> 4, row = warp * 16 + (i & 15);
            const int64_t r = (int64_t)base0 + (int64_t)j * tstep + row;
            if (r < p.ids_stride) cp_async4(smem_u32(sids + j * kAvTile + row), idp + r);
        }
        cp_async_commit();
    }
    const int H = p.history[u], len = p.length[u], cnt = p.count[u];
    const int rows = len > 0 ? cnt + max(len - H, 0) : 0;
    const int nt_all = (rows + kAvTile - 1) / kAvTile;
    int ntiles, lim;
    if (rr) {
        ntiles = s < nt_all ? (nt_all - 1 - s) / S + 1 : 0;
        lim = rows;
        cp_async_wait<0>();
        __syncwarp();   // the warp's staged ids are visible to all its lanes
    } else {
        // Whole tiles split evenly: the splits differ by at most one tile.
        const int r0 = min(rows, (int)((int64_t)s * nt_all / S) * kAvTile);
        const int r1 = min(rows, (int)((int64_t)(s + 1) * nt_all / S) * kAvTile);
        base0 = r0;
        ntiles = (r1 - r0 + kAvTile - 1) / kAvTile;
        lim = r1;
        // The split's ids, staged by the whole CTA (coalesced, all copies in
        // flight together).
        const int n_staged = min(max(0, min(r1, cnt) - r0), kAvIdsCap);
        for (int i = tid; i < n_staged; i += kAvThreads) cp_async4(smem_u32(sids + i), idp + r0 + i);
        cp_async_commit();
        cp_async_wait<0>();
        __syncthreads();
    }
    // Cache position of row `row` of the split's tile j (-1: past the
    // split): a listed id below the count, then the tail history..length-1.
    auto pos_of = [&](int j, int row) -> int {
        const int r = base0 + j * tstep + row;
        if (r >= lim) return -1;
        if (r >= cnt) return H + (r - cnt);
        return j < kStagedTiles ? sids[j * kAvTile + row] : __ldg(idp + r);
    };
    const int64_t ubase = (int64_t)(u / p.kv_heads) * p.kv_batch_stride + (int64_t)(u % p.kv_heads) * p.kv_head_stride;
    const __nv_bfloat16* kb = (const __nv_bfloat16*)p.k + ubase;
    const __nv_bfloat16* vb = (const __nv_bfloat16*)p.v + ubase;
    const int fresh = fresh_row(p, H, len);
    const __nv_bfloat16* knew = fresh >= 0 ? (const __nv_bfloat16*)p.k_new + (int64_t)u * kAvD : kb;
    const __nv_bfloat16* vnew = fresh >= 0 ? (const __nv_bfloat16*)p.v_new + (int64_t)u * kAvD : vb;
    append_fresh_row<__nv_bfloat16>(p, u, ubase, fresh);

    // Loader: the warp's 16 rows, two 256-byte rows per instruction (16
    // lanes x 16 bytes per row: fully coalesced); rows past the unit's rows
    // are zero-filled.
    const int ld_sub = lane >> 4, ld_ch = lane & 15;
    auto issue = [&](int t) {
        uint8_t* st = smem + (t % kAvStages) * kAvStageBytes;
        const uint32_t kd = smem_u32(st), vd = smem_u32(st + kAvTile * kAvRowBytes);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int row = warp * 16 + 2 * i + ld_sub;
            const int pos = pos_of(t, row);
            const bool valid = pos >= 0, nw = valid && pos == fresh;
            const int64_t off = valid && !nw ? (int64_t)pos * p.kv_row_stride : 0;
            cp_async16(kd + tile_off(row, ld_ch), (nw ? knew : kb) + off + ld_ch * 8, valid);
            cp_async16(vd + tile_off(row, ld_ch), (nw ? vnew : vb) + off + ld_ch * 8, valid);
        }
    };
    if (0 < ntiles) issue(0);
    cp_async_commit();
    if (1 < ntiles) issue(1);
    cp_async_commit();

    // Online softmax state of heads 2*q4 and 2*q4 + 1 (lanes with the same
    // q4 agree); O^T accumulators oc[mt] hold dims mt*16 + g (+8) of them.
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float oc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) oc[j][0] = oc[j][1] = oc[j][2] = oc[j][3] = 0.f;
    const float scale = kLog2e / sqrtf((float)kAvD);
    const int mi = lane >> 3, r8 = lane & 7;
    const int wrow = warp * 16;
    for (int t = 0; t < ntiles; ++t) {
        const int tn = t + kAvStages - 1;
        if (tn < ntiles) issue(tn);
        cp_async_commit();
        cp_async_wait<kAvStages - 1>();
        __syncwarp();   // the warp's own copies of tile t are visible to all its lanes
        const uint8_t* st = smem + (t % kAvStages) * kAvStageBytes;
        const uint32_t kbase = smem_u32(st), vbase = smem_u32(st + kAvTile * kAvRowBytes);
        // S^T = K Q^T, A = the warp's 16 key rows; two accumulation chains.
        float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            uint32_t a[4];
            ldmatrix_x4(kbase + tile_off(wrow + (mi & 1) * 8 + r8, 2 * kk + (mi >> 1)), a);
            if (kk & 1) mma_bf16(sb, a, qb[kk][0], qb[kk][1]);
            else mma_bf16(sa, a, qb[kk][0], qb[kk][1]);
        }
        // Scale, mask rows past the unit's rows (c0/c1: key g, heads 2q4 and
        // 2q4+1; c2/c3: key g+8), online softmax per head.
        const int base_r = base0 + t * tstep + wrow;
        const bool ok0 = base_r + g < lim, ok1 = base_r + g + 8 < lim;
        const float s0 = ok0 ? (sa[0] + sb[0]) * scale : -INFINITY;
        const float s1 = ok0 ? (sa[1] + sb[1]) * scale : -INFINITY;
        const float s2 = ok1 ? (sa[2] + sb[2]) * scale : -INFINITY;
        const float s3 = ok1 ? (sa[3] + sb[3]) * scale : -INFINITY;
        float mx0 = fmaxf(s0, s2), mx1 = fmaxf(s1, s3);
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
        }
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float al0 = mn0 == -INFINITY ? 1.f : exp2f(m0 - mn0);
        const float al1 = mn1 == -INFINITY ? 1.f : exp2f(m1 - mn1);
        const float p0 = mn0 == -INFINITY ? 0.f : exp2f(s0 - mn0);
        const float p2 = mn0 == -INFINITY ? 0.f : exp2f(s2 - mn0);
        const float p1 = mn1 == -INFINITY ? 0.f : exp2f(s1 - mn1);
        const float p3 = mn1 == -INFINITY ? 0.f : exp2f(s3 - mn1);
        float ps0 = p0 + p2, ps1 = p1 + p3;
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            ps0 += __shfl_xor_sync(0xffffffffu, ps0, o);
            ps1 += __shfl_xor_sync(0xffffffffu, ps1, o);
        }
        l0 = fmaf(l0, al0, ps0);
        l1 = fmaf(l1, al1, ps1);
        m0 = mn0;
        m1 = mn1;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            oc[j][0] *= al0; oc[j][1] *= al1;
            oc[j][2] *= al0; oc[j][3] *= al1;
        }
        // P^T as the B operand (k = keys, n = heads), rounded to bf16
        // (relative error 2^-9 per weight, the output's own rounding); l
        // above sums the unrounded fp32 weights.
        const uint32_t pb0 = movmatrix_trans(pack_bf16(p0, p1));
        const uint32_t pb1 = movmatrix_trans(pack_bf16(p2, p3));
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
            uint32_t a[4];
            ldmatrix_x4_trans(vbase + tile_off(wrow + (mi >> 1) * 8 + r8, 2 * mt + (mi & 1)), a);
            mma_bf16(oc[mt], a, pb0, pb1);
        }
        __syncwarp();   // every lane has read the stage before it is refilled
    }
    cp_async_wait<0>();
    __syncthreads();

    // Per-warp states to shared memory (reusing the stage buffers).
    float* red = reinterpret_cast<float*>(smem);
    float* rm = red;
    float* rl = red + 4 * kAvMaxG;
    float* ro = red + 2 * 4 * kAvMaxG;
    const int h0 = 2 * q4, h1 = h0 + 1;
    if (g == 0) {
        if (h0 < G) { rm[warp * kAvMaxG + h0] = m0; rl[warp * kAvMaxG + h0] = l0; }
        if (h1 < G) { rm[warp * kAvMaxG + h1] = m1; rl[warp * kAvMaxG + h1] = l1; }
    }
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
        const int da = mt * 16 + g, db = da + 8;
        if (h0 < G) {
            ro[(warp * kAvMaxG + h0) * kAvD + da] = oc[mt][0];
            ro[(warp * kAvMaxG + h0) * kAvD + db] = oc[mt][2];
        }
        if (h1 < G) {
            ro[(warp * kAvMaxG + h1) * kAvD + da] = oc[mt][1];
            ro[(warp * kAvMaxG + h1) * kAvD + db] = oc[mt][3];
        }
    }
    __syncthreads();
    if constexpr (kCluster) {
        float* pbuf = reinterpret_cast<float*>(smem + kAvStages * kAvStageBytes + kAvIdsCap * sizeof(int));
        av_finish_push<__nv_bfloat16>(p, u, s, red, 4, red + 2 * 4 * kAvMaxG + 4 * kAvMaxG * kAvD, pbuf);
    } else {
        av_finish<__nv_bfloat16>(p, u, s, red, 4);
    }
}

// 9..16 heads: the heads fill the MMA's M = 16 rows.
template <bool kCluster>
__global__ void __launch_bounds__(kAvThreads)
sparse_av_bf16_g16_kernel(AvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int s = blockIdx.x, u = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = p.G;
    const int H = p.history[u], len = p.length[u], cnt = p.count[u];
    const int rows = len > 0 ? cnt + max(len - H, 0) : 0;
    // Whole tiles split evenly: the splits differ by at most one tile.
    const int nt_all = (rows + kAvTile - 1) / kAvTile;
    const int r0 = min(rows, (int)((int64_t)s * nt_all / p.S) * kAvTile);
    const int r1 = min(rows, (int)((int64_t)(s + 1) * nt_all / p.S) * kAvTile);
    const int ntiles = (r1 - r0 + kAvTile - 1) / kAvTile;
    const int64_t ubase = (int64_t)(u / p.kv_heads) * p.kv_batch_stride + (int64_t)(u % p.kv_heads) * p.kv_head_stride;
    const __nv_bfloat16* kb = (const __nv_bfloat16*)p.k + ubase;
    const __nv_bfloat16* vb = (const __nv_bfloat16*)p.v + ubase;
    const int* idp = p.ids + (int64_t)u * p.ids_stride;
    const __nv_bfloat16* qp = (const __nv_bfloat16*)p.q + (int64_t)u * G * kAvD;
    const int fresh = fresh_row(p, H, len);
    const __nv_bfloat16* knew = fresh >= 0 ? (const __nv_bfloat16*)p.k_new + (int64_t)u * kAvD : kb;
    const __nv_bfloat16* vnew = fresh >= 0 ? (const __nv_bfloat16*)p.v_new + (int64_t)u * kAvD : vb;
    append_fresh_row<__nv_bfloat16>(p, u, ubase, fresh);

    // Q as the MMA A operand: rows = heads, columns = dims.
    uint32_t qa[8][4];
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int hh = (lane >> 2) + (r & 1) * 8;
            const int dim = kk * 16 + 2 * (lane & 3) + (r >> 1) * 8;
            qa[kk][r] = hh < G ? *reinterpret_cast<const uint32_t*>(qp + hh * kAvD + dim) : 0u;
        }

    // The split's row ids, staged once in shared memory (all copies in flight
    // together) so that issuing a tile's copies never waits on a global load.
    int* sids = reinterpret_cast<int*>(smem + kAvStages * kAvStageBytes);
    const int n_staged = min(max(0, min(r1, cnt) - r0), kAvIdsCap);
    for (int i = tid; i < n_staged; i += kAvThreads) cp_async4(smem_u32(sids + i), idp + r0 + i);
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    auto pos_of = [&](int r) -> int {
        if (r >= r1) return -1;
        if (r >= cnt) return H + (r - cnt);
        return r - r0 < kAvIdsCap ? sids[r - r0] : idp[r];
    };
    // Loader: each warp moves its 16 rows of the tile, two 256-byte rows per
    // instruction (16 lanes x 16 bytes per row: fully coalesced).
    const int ld_sub = lane >> 4, ld_ch = lane & 15;
    auto issue = [&](int t) {
        uint8_t* st = smem + (t % kAvStages) * kAvStageBytes;
        const uint32_t kd = smem_u32(st), vd = smem_u32(st + kAvTile * kAvRowBytes);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int row = warp * 16 + 2 * i + ld_sub;
            const int pos = pos_of(r0 + t * kAvTile + row);
            const bool valid = pos >= 0, nw = valid && pos == fresh;
            const int64_t off = valid && !nw ? (int64_t)pos * p.kv_row_stride : 0;
            cp_async16(kd + tile_off(row, ld_ch), (nw ? knew : kb) + off + ld_ch * 8, valid);
            cp_async16(vd + tile_off(row, ld_ch), (nw ? vnew : vb) + off + ld_ch * 8, valid);
        }
    };

    if (0 < ntiles) issue(0);
    cp_async_commit();
    if (1 < ntiles) issue(1);
    cp_async_commit();

    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
    float o[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    const float scale = kLog2e / sqrtf((float)kAvD);

    for (int t = 0; t < ntiles; ++t) {
        const int tn = t + kAvStages - 1;
        if (tn < ntiles) issue(tn);
        cp_async_commit();
        cp_async_wait<kAvStages - 1>();
        __syncthreads();

        const uint8_t* st = smem + (t % kAvStages) * kAvStageBytes;
        const uint32_t kbase = smem_u32(st), vbase = smem_u32(st + kAvTile * kAvRowBytes);
        const int wrow = warp * 16;
        float sacc[2][4];
#pragma unroll
        for (int j = 0; j < 2; ++j) sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            uint32_t b[4];
            const int mi = lane >> 3, r = lane & 7;
            const int row = wrow + (mi >> 1) * 8 + r;
            ldmatrix_x4(kbase + tile_off(row, 2 * kk + (mi & 1)), b);
            mma_bf16(sacc[0], qa[kk], b[0], b[1]);
            mma_bf16(sacc[1], qa[kk], b[2], b[3]);
        }
        // Scale, mask rows past the split end, online softmax per head.
        const int base_r = r0 + t * kAvTile + wrow;
        float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const bool ok = base_r + 8 * j + 2 * (lane & 3) + e < r1;
                sacc[j][e] = ok ? sacc[j][e] * scale : -INFINITY;
                sacc[j][2 + e] = ok ? sacc[j][2 + e] * scale : -INFINITY;
                mx_a = fmaxf(mx_a, sacc[j][e]);
                mx_b = fmaxf(mx_b, sacc[j][2 + e]);
            }
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
        const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
        const float al_a = mn_a == -INFINITY ? 1.f : exp2f(m_a - mn_a);
        const float al_b = mn_b == -INFINITY ? 1.f : exp2f(m_b - mn_b);
        float pr[2][4];
        float ps_a = 0.f, ps_b = 0.f;
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                pr[j][e] = mn_a == -INFINITY ? 0.f : exp2f(sacc[j][e] - mn_a);
                pr[j][2 + e] = mn_b == -INFINITY ? 0.f : exp2f(sacc[j][2 + e] - mn_b);
                ps_a += pr[j][e];
                ps_b += pr[j][2 + e];
            }
        ps_a += __shfl_xor_sync(0xffffffffu, ps_a, 1);
        ps_a += __shfl_xor_sync(0xffffffffu, ps_a, 2);
        ps_b += __shfl_xor_sync(0xffffffffu, ps_b, 1);
        ps_b += __shfl_xor_sync(0xffffffffu, ps_b, 2);
        l_a = fmaf(l_a, al_a, ps_a);
        l_b = fmaf(l_b, al_b, ps_b);
        m_a = mn_a;
        m_b = mn_b;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            o[j][0] *= al_a; o[j][1] *= al_a;
            o[j][2] *= al_b; o[j][3] *= al_b;
        }
        // P as the A operand (rows = heads, k = the 16 rows), rounded to
        // bf16 (relative error 2^-9 per weight, the output's own rounding);
        // l above sums the unrounded fp32 weights.
        uint32_t ph[4];
        ph[0] = pack_bf16(pr[0][0], pr[0][1]); ph[1] = pack_bf16(pr[0][2], pr[0][3]);
        ph[2] = pack_bf16(pr[1][0], pr[1][1]); ph[3] = pack_bf16(pr[1][2], pr[1][3]);
#pragma unroll
        for (int np = 0; np < 8; ++np) {
            uint32_t b[4];
            const int mi = lane >> 3, r = lane & 7;
            const int row = wrow + (mi & 1) * 8 + r;
            ldmatrix_x4_trans(vbase + tile_off(row, 2 * np + (mi >> 1)), b);
            mma_bf16(o[2 * np], ph, b[0], b[1]);
            mma_bf16(o[2 * np + 1], ph, b[2], b[3]);
        }
        __syncthreads();
    }
    cp_async_wait<0>();
    __syncthreads();

    // Per-warp states to shared memory (reusing the stage buffers).
    float* red = reinterpret_cast<float*>(smem);
    float* rm = red;
    float* rl = red + 4 * kAvMaxG;
    float* ro = red + 2 * 4 * kAvMaxG;
    const int ha = lane >> 2, hb = ha + 8;
    if ((lane & 3) == 0) {
        if (ha < G) { rm[warp * kAvMaxG + ha] = m_a; rl[warp * kAvMaxG + ha] = l_a; }
        if (hb < G) { rm[warp * kAvMaxG + hb] = m_b; rl[warp * kAvMaxG + hb] = l_b; }
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int dim = 8 * j + 2 * (lane & 3);
        if (ha < G) {
            ro[(warp * kAvMaxG + ha) * kAvD + dim] = o[j][0];
            ro[(warp * kAvMaxG + ha) * kAvD + dim + 1] = o[j][1];
        }
        if (hb < G) {
            ro[(warp * kAvMaxG + hb) * kAvD + dim] = o[j][2];
            ro[(warp * kAvMaxG + hb) * kAvD + dim + 1] = o[j][3];
        }
    }
    __syncthreads();
    if constexpr (kCluster)
        av_finish_cluster<__nv_bfloat16>(p, u, s, red, 4, red + 2 * 4 * kAvMaxG + 4 * kAvMaxG * kAvD);
    else
        av_finish<__nv_bfloat16>(p, u, s, red, 4);
}

// fp32 K/V path (parity shapes such as the CPU fp32 config): one warp per
// row at a time, lane-owned dims, warp-reduced dot products.
__global__ void __launch_bounds__(kAvThreads)
sparse_av_f32_kernel(AvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int s = blockIdx.x, u = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = p.G;
    const int H = p.history[u], len = p.length[u], cnt = p.count[u];
    const int rows = len > 0 ? cnt + max(len - H, 0) : 0;
    const int per = (rows + p.S - 1) / p.S;
    const int r0 = min(rows, s * per), r1 = min(rows, r0 + per);
    const int64_t ubase = (int64_t)(u / p.kv_heads) * p.kv_batch_stride + (int64_t)(u % p.kv_heads) * p.kv_head_stride;
    const float* kb = (const float*)p.k + ubase;
    const float* vb = (const float*)p.v + ubase;
    const int* idp = p.ids + (int64_t)u * p.ids_stride;
    const float* qp = (const float*)p.q + (int64_t)u * G * kAvD;
    const int fresh = fresh_row(p, H, len);
    append_fresh_row<float>(p, u, ubase, fresh);
    float* red = reinterpret_cast<float*>(smem);
    float* rm = red;
    float* rl = red + 4 * kAvMaxG;
    float* ro = red + 2 * 4 * kAvMaxG;
    const float scale = kLog2e / sqrtf((float)kAvD);
    // Heads in groups of four to bound register use.
    for (int h0 = 0; h0 < G; h0 += 4) {
        float4 qv[4], ov[4];
        float m[4], l[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            const int h = h0 + a;
            qv[a] = h < G ? reinterpret_cast<const float4*>(qp + h * kAvD)[lane] : make_float4(0.f, 0.f, 0.f, 0.f);
            ov[a] = make_float4(0.f, 0.f, 0.f, 0.f);
            m[a] = -INFINITY;
            l[a] = 0.f;
        }
        for (int r = r0 + warp; r < r1; r += 4) {
            const int pos = r < cnt ? idp[r] : H + (r - cnt);
            const bool nw = pos == fresh;
            const float* kr = nw ? (const float*)p.k_new + (int64_t)u * kAvD : kb + (int64_t)pos * p.kv_row_stride;
            const float* vr = nw ? (const float*)p.v_new + (int64_t)u * kAvD : vb + (int64_t)pos * p.kv_row_stride;
            const float4 kv = reinterpret_cast<const float4*>(kr)[lane];
            const float4 vv = reinterpret_cast<const float4*>(vr)[lane];
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                float d = qv[a].x * kv.x + qv[a].y * kv.y + qv[a].z * kv.z + qv[a].w * kv.w;
                d = warp_sum(d) * scale;
                const float mn = fmaxf(m[a], d);
                const float al = exp2f(m[a] - mn), pr = exp2f(d - mn);
                l[a] = l[a] * al + pr;
                ov[a].x = ov[a].x * al + pr * vv.x;
                ov[a].y = ov[a].y * al + pr * vv.y;
                ov[a].z = ov[a].z * al + pr * vv.z;
                ov[a].w = ov[a].w * al + pr * vv.w;
                m[a] = mn;
            }
        }
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            const int h = h0 + a;
            if (h >= G) break;
            if (lane == 0) { rm[warp * kAvMaxG + h] = m[a]; rl[warp * kAvMaxG + h] = l[a]; }
            reinterpret_cast<float4*>(ro + (warp * kAvMaxG + h) * kAvD)[lane] = ov[a];
        }
    }
    __syncthreads();
    av_finish<float>(p, u, s, red, 4);
}

__global__ void lse_merge_kernel(const float* __restrict__ part, int P, int UG, float* __restrict__ out_f,
                                 __nv_bfloat16* __restrict__ out_b) {
    const int uh = blockIdx.x, dim = threadIdx.x;
    float M = -INFINITY;
    for (int j = 0; j < P; ++j) M = fmaxf(M, part[((int64_t)j * UG + uh) * (kAvD + 2)]);
    float L = 0.f, O = 0.f;
    for (int j = 0; j < P; ++j) {
        const float* pp = part + ((int64_t)j * UG + uh) * (kAvD + 2);
        const float sc = pp[0] == -INFINITY ? 0.f : expf(pp[0] - M);
        L = fmaf(sc, pp[1], L);
        O = fmaf(sc, pp[2 + dim], O);
    }
    const float r = L > 0.f ? O / L : 0.f;
    if (out_f) out_f[(int64_t)uh * kAvD + dim] = r;
    else out_b[(int64_t)uh * kAvD + dim] = __float2bfloat16_rn(r);
}

// Whether a cluster of S split CTAs of kernel `which` (0: up to 8 heads,
// 1: 9..16 heads; S <= 16, above 8 the non-portable cluster sizes) with
// `smem` bytes each can be resident on the current device; answered once per
// (device, kernel, S, smem) and kept.  Host threads may launch concurrently,
// so the caches below are guarded by one mutex.
static std::mutex g_launch_cache_mu;
constexpr int kMaxDevices = 64;

bool cluster_fits(int which, int S, int smem) {
    static int known[kMaxDevices][2][kAvMaxCluster + 1] = {};   // 0 unknown, 1 yes, 2 no
    static int known_smem[kMaxDevices][2][kAvMaxCluster + 1] = {};
    if (S < 2 || S > kAvMaxCluster) return false;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return false;
    }
    std::lock_guard<std::mutex> lock(g_launch_cache_mu);
    int& state = known[dev][which][S];
    if (known_smem[dev][which][S] != smem) state = 0;
    if (!state) {
        known_smem[dev][which][S] = smem;
        auto fn = which == 0 ? sparse_av_bf16_kernel<true> : sparse_av_bf16_g16_kernel<true>;
        bool ok = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) == cudaSuccess;
        if (ok && S > 8) ok = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess;
        int clusters = 0;
        if (ok) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(S, 1);
            cfg.blockDim = dim3(kAvThreads);
            cfg.dynamicSmemBytes = smem;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = S;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            ok = cudaOccupancyMaxActiveClusters(&clusters, fn, &cfg) == cudaSuccess && clusters > 0;
        }
        cudaGetLastError();   // a refused query leaves no sticky error
        state = ok ? 1 : 2;
    }
    return state == 1;
}

int default_splits(int U) {
    // SM count of the current device, looked up once per device.
    static int sms_of[kMaxDevices] = {};
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < kMaxDevices) {
        std::lock_guard<std::mutex> lock(g_launch_cache_mu);
        if (!sms_of[dev]) {
            int n = 0;
            if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
            sms_of[dev] = n;
        }
        sms = sms_of[dev];
    }
    cudaGetLastError();
    // About one wave of two CTAs per SM across all units: each split pays a
    // fixed prologue (ids, Q, first tile), so more splits than resident slots
    // only add overhead.  Up to 8 splits form one cluster merged on chip;
    // above that, whole clusters of 8 (merged on chip, then across clusters
    // through global memory), at most 64 splits.
    const int s = (2 * sms) / U;
    if (s < 1) return 1;
    return s <= kAvGroupMax ? s : (s / kAvGroupMax * kAvGroupMax > 64 ? 64 : s / kAvGroupMax * kAvGroupMax);
}

// CTAs per cluster of the G <= 8 kernel for S splits: all of them up to 8,
// else the largest divisor of S in [3, 8] (the clusters' states then merge
// through global memory); 0 when there is none (no cluster: the last CTA of
// a unit merges the S split partials).
int av_cluster_size(int S) {
    if (S <= kAvGroupMax) return S;
    for (int c = kAvGroupMax; c >= 3; --c)
        if (S % c == 0) return c;
    return 0;
}

}  // namespace pk

using namespace pk;

extern "C" size_t pk_sparse_av_workspace_bytes(int U, int G, int d, int splits) {
    if (splits <= 0) splits = 256;
    // Split partials [U*G, S, d+2] (the cluster states [U, S/C, 3, G*d] of a
    // clustered launch fit in the same bytes for C >= 3), then kAvCounters
    // arrival counters per unit.
    const size_t part = (size_t)U * G * splits * (d + 2) * sizeof(float);
    return (part + 255) / 256 * 256 + ((size_t)U * kAvCounters * sizeof(int) + 255) / 256 * 256;
}

static int sparse_av_launch(uint64_t q, uint64_t k, uint64_t v, int dtype, int kv_heads, int64_t kv_batch_stride,
                            int64_t kv_head_stride, int64_t kv_row_stride, uint64_t ids, int64_t ids_stride,
                            uint64_t count, uint64_t history, uint64_t length, int U, int G, int d, int splits,
                            uint64_t workspace, uint64_t workspace_bytes, uint64_t out, uint64_t partial,
                            uint64_t k_new, uint64_t v_new, uint64_t stream) {
    if (U < 1 || G < 1 || G > kAvMaxG || kv_heads < 1 || kv_row_stride < d) return PK_ERR_ARG;
    if ((k_new == 0) != (v_new == 0) || (k_new | v_new) % 16) return PK_ERR_ARG;
    if (d != kAvD) return PK_ERR_UNSUPPORTED;
    if (!q || !k || !v || !ids || !count || !history || !length || (!out && !partial)) return PK_ERR_ARG;
    if (splits <= 0) splits = default_splits(U);
    if (splits > 256) return PK_ERR_ARG;
    if (splits > 1 && (!workspace || workspace_bytes < pk_sparse_av_workspace_bytes(U, G, d, splits)))
        return PK_ERR_WORKSPACE;
    AvParams p;
    p.q = (const void*)q; p.k = (const void*)k; p.v = (const void*)v;
    p.kv_heads = kv_heads;
    p.kv_batch_stride = kv_batch_stride; p.kv_head_stride = kv_head_stride; p.kv_row_stride = kv_row_stride;
    p.ids = (const int*)ids; p.ids_stride = ids_stride;
    p.count = (const int*)count; p.history = (const int*)history; p.length = (const int*)length;
    p.G = G; p.S = splits;
    const size_t part_bytes = (size_t)U * G * splits * (d + 2) * sizeof(float);
    p.part = (float*)workspace;
    p.done = workspace ? (int*)((char*)workspace + (part_bytes + 255) / 256 * 256) : nullptr;
    p.out = (void*)out;
    p.xpart = (float*)partial;
    p.k_new = (const void*)k_new;
    p.v_new = (const void*)v_new;
    cudaStream_t st = (cudaStream_t)stream;
    dim3 grid(splits, U);
    p.C = 1;
    p.rr = 0;
    if (dtype == PK_BF16) {
        if (kv_row_stride % 8 || kv_batch_stride % 8 || kv_head_stride % 8 || (k | v) % 16) return PK_ERR_ARG;
        const int which = G <= 8 ? 0 : 1;
        const int base_smem = kAvStages * kAvStageBytes + kAvIdsCap * (int)sizeof(int);
        // Cluster size: the G <= 8 kernel merges clusters of av_cluster_size
        // splits on chip (and the clusters through global memory); the
        // 9..16-head kernel takes all its splits (up to 16) in one cluster.
        const int C = which == 0 ? av_cluster_size(splits) : splits;
        // The cluster form of the G <= 8 kernel adds the push-merge receive buffer.
        const int csmem = base_smem + (which == 0 && C >= 2 ? av_push_floats(G, C) * (int)sizeof(float) : 0);
        if (splits >= 2 && C >= 2 && cluster_fits(which, C, csmem)) {
            p.C = C;
            p.rr = which == 0 && C < splits;
            // The shared-memory limit is one attribute per kernel, shared by
            // every split count: set it for this launch's size.
            auto cfn = which == 0 ? sparse_av_bf16_kernel<true> : sparse_av_bf16_g16_kernel<true>;
            if (cudaFuncSetAttribute(cfn, cudaFuncAttributeMaxDynamicSharedMemorySize, csmem) != cudaSuccess)
                return (int)cudaGetLastError();
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = grid;
            cfg.blockDim = dim3(kAvThreads);
            cfg.dynamicSmemBytes = csmem;
            cfg.stream = st;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = C;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            const cudaError_t e = cudaLaunchKernelEx(
                &cfg, which == 0 ? sparse_av_bf16_kernel<true> : sparse_av_bf16_g16_kernel<true>, p);
            if (e != cudaSuccess) return (int)e;
        } else {
            auto fn = which == 0 ? sparse_av_bf16_kernel<false> : sparse_av_bf16_g16_kernel<false>;
            cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, base_smem);
            fn<<<grid, kAvThreads, base_smem, st>>>(p);
        }
    } else if (dtype == PK_F32) {
        if (kv_row_stride % 4 || kv_batch_stride % 4 || kv_head_stride % 4 || (k | v | q) % 16) return PK_ERR_ARG;
        const int smem = (2 * 4 * kAvMaxG + 4 * kAvMaxG * kAvD) * (int)sizeof(float);
        cudaFuncSetAttribute(sparse_av_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        sparse_av_f32_kernel<<<grid, kAvThreads, smem, st>>>(p);
    } else {
        return PK_ERR_ARG;
    }
    PK_CHECK_LAUNCH();
    return PK_OK;
}

extern "C" int pk_sparse_av(uint64_t q, uint64_t k, uint64_t v, int dtype, int kv_heads, int64_t kv_batch_stride,
                            int64_t kv_head_stride, int64_t kv_row_stride, uint64_t ids, int64_t ids_stride,
                            uint64_t count, uint64_t history, uint64_t length, int U, int G, int d, int splits,
                            uint64_t workspace, uint64_t workspace_bytes, uint64_t out, uint64_t partial,
                            uint64_t stream) {
    return sparse_av_launch(q, k, v, dtype, kv_heads, kv_batch_stride, kv_head_stride, kv_row_stride, ids, ids_stride,
                            count, history, length, U, G, d, splits, workspace, workspace_bytes, out, partial, 0, 0,
                            stream);
}

extern "C" int pk_sparse_av_append(uint64_t q, uint64_t k, uint64_t v, int dtype, int kv_heads,
                                   int64_t kv_batch_stride, int64_t kv_head_stride, int64_t kv_row_stride,
                                   uint64_t ids, int64_t ids_stride, uint64_t count, uint64_t history,
                                   uint64_t length, int U, int G, int d, int splits, uint64_t workspace,
                                   uint64_t workspace_bytes, uint64_t out, uint64_t partial, uint64_t k_new,
                                   uint64_t v_new, uint64_t stream) {
    if (!k_new || !v_new) return PK_ERR_ARG;
    return sparse_av_launch(q, k, v, dtype, kv_heads, kv_batch_stride, kv_head_stride, kv_row_stride, ids, ids_stride,
                            count, history, length, U, G, d, splits, workspace, workspace_bytes, out, partial, k_new,
                            v_new, stream);
}

extern "C" int pk_lse_merge(uint64_t partial, int P, int UG, int d, uint64_t out, int dtype, uint64_t stream) {
    if (P < 1 || UG < 1 || !partial || !out) return PK_ERR_ARG;
    if (d != kAvD) return PK_ERR_UNSUPPORTED;
    if (dtype != PK_F32 && dtype != PK_BF16) return PK_ERR_ARG;
    lse_merge_kernel<<<UG, kAvD, 0, (cudaStream_t)stream>>>(
        (const float*)partial, P, UG, dtype == PK_F32 ? (float*)out : nullptr,
        dtype == PK_BF16 ? (__nv_bfloat16*)out : nullptr);
    PK_CHECK_LAUNCH();
    return PK_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free variant (no counterpart in the reference).  Some embedders
// cannot give the library a workspace -- a host that pre-reserved all device
// memory for its own pool, or a foreign-language caller of this C ABI with no
// device allocator -- so the split scratch lives here, in a file-scope device
// array every GPU that loads the library keeps until exit.
// ---------------------------------------------------------------------------

namespace pk {
static __device__ __align__(256) unsigned char g_av_noalloc_scratch[PK_SPARSE_AV_NOALLOC_SCRATCH_BYTES];

// The array's name is only a host-side stand-in; its device address is looked
// up with the device current.  Outside stream capture every call looks it up
// again (so a device reset, which reloads the module at a new address, is
// followed); inside a capture the address cached by the device's last
// uncaptured call is used, so the first call on a device must come before any
// stream capture.
static void* noalloc_scratch_address(cudaStream_t stream, int* rc) {
    static std::mutex mu;
    static void* addr[kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        *rc = e != cudaSuccess ? (int)e : PK_ERR_ARG;
        return nullptr;
    }
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    e = cudaStreamIsCapturing(stream, &cap);
    if (e != cudaSuccess) {
        *rc = (int)e;
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (cap == cudaStreamCaptureStatusNone) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_av_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            *rc = e != cudaSuccess ? (int)e : PK_ERR_ARG;
            return nullptr;
        }
        addr[dev] = p;
    } else if (!addr[dev]) {
        *rc = PK_ERR_ARG;   // never set up on this device outside a capture
        return nullptr;
    }
    *rc = 0;
    return addr[dev];
}
}  // namespace pk

extern "C" int pk_sparse_av_noalloc(uint64_t q, uint64_t k, uint64_t v, int dtype, int kv_heads,
                                    int64_t kv_batch_stride, int64_t kv_head_stride, int64_t kv_row_stride,
                                    uint64_t ids, int64_t ids_stride, uint64_t count, uint64_t history,
                                    uint64_t length, int U, int G, int d, int splits, uint64_t out,
                                    uint64_t stream) {
    if (U < 1 || G < 1 || G > kAvMaxG || !out) return PK_ERR_ARG;
    if (splits <= 0) splits = default_splits(U);
    if (splits > 256) return PK_ERR_ARG;
    const size_t need = pk_sparse_av_workspace_bytes(U, G, d, splits);
    if (splits > 1 && need > PK_SPARSE_AV_NOALLOC_SCRATCH_BYTES) return PK_ERR_SCRATCH_LIMIT;
    int rc = 0;
    void* scratch = noalloc_scratch_address((cudaStream_t)stream, &rc);
    if (!scratch) return rc;
    if (splits > 1) {
        // The arrival counters must start at zero; the array keeps whatever
        // the previous call left, so clear them on this call's stream.
        const size_t part = (size_t)U * G * splits * (d + 2) * sizeof(float);
        const size_t counters = (part + 255) / 256 * 256;
        cudaError_t e = cudaMemsetAsync((char*)scratch + counters, 0, (size_t)U * kAvCounters * sizeof(int),
                                        (cudaStream_t)stream);
        if (e != cudaSuccess) return (int)e;
    }
    return pk_sparse_av(q, k, v, dtype, kv_heads, kv_batch_stride, kv_head_stride, kv_row_stride, ids, ids_stride,
                        count, history, length, U, G, d, splits, (uint64_t)scratch,
                        (uint64_t)PK_SPARSE_AV_NOALLOC_SCRATCH_BYTES, out, 0, stream);
}
