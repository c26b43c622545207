// Explicit gather of the selected rows and the dense tail into a packed,
// unit-major K/V layout: the reference's layout-control diagnostic
// (kernels/cuda_sm90/native_sources/gather.cu:5-31, driven by
// kernels/cuda_sm90/single.py:24-67).  The sparse attention reads the rows in
// place; this copy exists to compare that with attention over a packed
// layout, and its own rate is the HBM rate of the selected rows' random
// 256-byte reads (the sparse attention's gather ceiling).
#include "common.cuh"

namespace pk {

// One 16-byte vector per thread and step, grid-stride over the packed rows
// of every unit (unit-major, packed_rows slots each); four vectors in flight
// per thread.  Slot r of unit u holds ids[u][r] for r < count[u], then the
// tail rows history[u] + (r - count[u]) up to length[u]; later slots are not
// written.  A unit whose rows exceed packed_rows is truncated and flagged.
__global__ void __launch_bounds__(256)
gather_kv_kernel(const uint4* __restrict__ k, const uint4* __restrict__ v, int kv_heads, int64_t bs, int64_t hs,
                 int64_t rs, const int* __restrict__ ids, int64_t ids_stride, const int* __restrict__ count,
                 const int* __restrict__ history, const int* __restrict__ length, int U, int row_vecs,
                 int64_t packed_rows, uint4* __restrict__ out_k, uint4* __restrict__ out_v, int* __restrict__ status) {
    const int64_t nvec = (int64_t)U * packed_rows * row_vecs;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    constexpr int kUnroll = 4;
    for (int64_t base = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; base < nvec; base += step * kUnroll) {
        uint4 kv[kUnroll], vv[kUnroll];
        int64_t dst[kUnroll];
#pragma unroll
        for (int i = 0; i < kUnroll; ++i) {
            const int64_t e = base + i * step;
            dst[i] = -1;
            if (e >= nvec) continue;
            const int j = (int)(e % row_vecs);
            const int64_t slot = e / row_vecs;
            const int u = (int)(slot / packed_rows);
            const int64_t r = slot % packed_rows;
            const int len = length[u], hist = history[u], cnt = count[u];
            const int64_t rows = len > 0 ? (int64_t)cnt + max(len - hist, 0) : 0;
            if (r >= rows) continue;
            const int64_t pos = r < cnt ? (int64_t)ids[(int64_t)u * ids_stride + r] : hist + (r - cnt);
            const int64_t src = (int64_t)(u / kv_heads) * bs + (int64_t)(u % kv_heads) * hs + pos * rs + j;
            kv[i] = k[src];
            vv[i] = v[src];
            dst[i] = e;
        }
#pragma unroll
        for (int i = 0; i < kUnroll; ++i) {
            if (dst[i] < 0) continue;
            out_k[dst[i]] = kv[i];
            out_v[dst[i]] = vv[i];
        }
    }
    // Truncation check: one thread per unit.
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t < U && status) {
        const int len = length[t], hist = history[t];
        const int64_t rows = len > 0 ? (int64_t)count[t] + max(len - hist, 0) : 0;
        if (rows > packed_rows) atomicOr(status, PK_STATUS_OUT_FULL);
    }
}

// Decode append: slot s's new K and V rows (kv_heads rows of d each,
// contiguous in k_new/v_new) written at row positions[s] of the cache.  One
// CTA per slot, 16-byte vectors; a position outside [0, capacity) leaves the
// slot untouched (an inactive slot), as the reference's append_slots does.
__global__ void __launch_bounds__(128)
kv_append_kernel(const uint4* __restrict__ k_new, const uint4* __restrict__ v_new, uint4* __restrict__ k_cache,
                 uint4* __restrict__ v_cache, int kv_heads, int64_t bs, int64_t hs, int64_t rs,
                 const int* __restrict__ positions, int capacity, int row_vecs) {
    const int slot = blockIdx.x;
    const int pos = positions[slot];
    if (pos < 0 || pos >= capacity) return;
    const int n = kv_heads * row_vecs;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int h = i / row_vecs, j = i % row_vecs;
        const int64_t dst = (int64_t)slot * bs + (int64_t)h * hs + (int64_t)pos * rs + j;
        const int64_t src = ((int64_t)slot * kv_heads + h) * row_vecs + j;
        k_cache[dst] = k_new[src];
        v_cache[dst] = v_new[src];
    }
}

}  // namespace pk

using namespace pk;

extern "C" int pk_gather_kv(uint64_t k, uint64_t v, int dtype, int kv_heads, int64_t kv_batch_stride,
                            int64_t kv_head_stride, int64_t kv_row_stride, uint64_t ids, int64_t ids_stride,
                            uint64_t count, uint64_t history, uint64_t length, int U, int d, int64_t packed_rows,
                            uint64_t out_k, uint64_t out_v, uint64_t status, uint64_t stream) {
    if (U < 1 || d < 1 || kv_heads < 1 || packed_rows < 0 || ids_stride < 0) return PK_ERR_ARG;
    if (!k || !v || !ids || !count || !history || !length || !out_k || !out_v) return PK_ERR_ARG;
    const int esz = dtype == PK_BF16 ? 2 : dtype == PK_F32 ? 4 : 0;
    if (!esz) return PK_ERR_ARG;
    // 16-byte vectors: rows, strides and bases 16-byte aligned.
    if ((d * esz) % 16 || (k | v | out_k | out_v) % 16 || (kv_batch_stride * esz) % 16 ||
        (kv_head_stride * esz) % 16 || (kv_row_stride * esz) % 16)
        return PK_ERR_ARG;
    if (packed_rows == 0) return PK_OK;
    const int row_vecs = d * esz / 16;
    const int per = 16 / esz;   // elements per vector
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t nvec = (int64_t)U * packed_rows * row_vecs;
    int64_t blocks = (nvec + 255) / 256;
    const int64_t cap = (int64_t)sms * 8;
    if (blocks > cap) blocks = cap;
    if (blocks * 256 < U) blocks = (U + 255) / 256;
    gather_kv_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
        (const uint4*)k, (const uint4*)v, kv_heads, kv_batch_stride / per, kv_head_stride / per, kv_row_stride / per,
        (const int*)ids, ids_stride, (const int*)count, (const int*)history, (const int*)length, U, row_vecs,
        packed_rows, (uint4*)out_k, (uint4*)out_v, (int*)status);
    PK_CHECK_LAUNCH();
    return PK_OK;
}

extern "C" int pk_kv_append(uint64_t k_new, uint64_t v_new, uint64_t k_cache, uint64_t v_cache, int dtype,
                            int kv_heads, int64_t kv_batch_stride, int64_t kv_head_stride, int64_t kv_row_stride,
                            uint64_t positions, int slots, int capacity, int d, uint64_t stream) {
    if (slots < 0 || kv_heads < 1 || d < 1 || capacity < 0) return PK_ERR_ARG;
    if (slots == 0) return PK_OK;
    if (!k_new || !v_new || !k_cache || !v_cache || !positions) return PK_ERR_ARG;
    const int esz = dtype == PK_BF16 ? 2 : dtype == PK_F32 ? 4 : 0;
    if (!esz) return PK_ERR_ARG;
    // 16-byte vectors: rows, strides and bases 16-byte aligned.
    if ((d * esz) % 16 || (k_new | v_new | k_cache | v_cache) % 16 || (kv_batch_stride * esz) % 16 ||
        (kv_head_stride * esz) % 16 || (kv_row_stride * esz) % 16)
        return PK_ERR_ARG;
    const int per = 16 / esz;
    kv_append_kernel<<<slots, 128, 0, (cudaStream_t)stream>>>(
        (const uint4*)k_new, (const uint4*)v_new, (uint4*)k_cache, (uint4*)v_cache, kv_heads, kv_batch_stride / per,
        kv_head_stride / per, kv_row_stride / per, (const int*)positions, capacity, d * esz / 16);
    PK_CHECK_LAUNCH();
    return PK_OK;
}
