// Shared device helpers for the PrismKV B200 kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "prismkv_b200.h"

namespace pk {

__device__ __forceinline__ float load_f(const float* p, int64_t i) { return p[i]; }
__device__ __forceinline__ float load_f(const __nv_bfloat16* p, int64_t i) { return __bfloat162float(p[i]); }

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Inclusive prefix sum across a warp.
__device__ __forceinline__ int warp_inclusive_scan(int v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += y;
    }
    return v;
}

// Exclusive block-wide prefix sum of one int per thread.  `scratch` needs
// blockDim.x/32 + 1 ints.  Returns the exclusive prefix; *total gets the sum.
// Every thread of the block must call it.
__device__ __forceinline__ int block_exclusive_scan(int v, int* scratch, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int inc = warp_inclusive_scan(v);
    if (lane == 31) scratch[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        int s = lane < nw ? scratch[lane] : 0;
        int si = warp_inclusive_scan(s);
        if (lane < nw) scratch[lane] = si - s;
        if (lane == nw - 1) scratch[nw] = si;
    }
    __syncthreads();
    int r = scratch[warp] + inc - v;
    *total = scratch[nw];
    __syncthreads();
    return r;
}

// ---------------------------------------------------------------------------
// PyTorch CPU reduction orders, restated so that kernels reproduce the
// reference's fp32 results bit for bit (the same orders as the CPU oracle).
// ---------------------------------------------------------------------------

__host__ __device__ __forceinline__ int ceil_log2_i64(int64_t n) {
    int r = 0;
    int64_t t = 1;
    while (t < n) { t <<= 1; ++r; }
    return r;
}

// Row sum of v[0..n) (n <= 256) in the order torch.sum(-1) uses for a
// contiguous fp32 row: 8-lane vectors, 4 interleaved vector accumulators,
// lanes folded left to right; rows shorter than 8 use the scalar 4-partial
// form.  Sequential code for one thread.
__device__ __forceinline__ float torch_rowsum(const float* v, int n) {
    if (n < 8) {
        float r[4] = {0.f, 0.f, 0.f, 0.f};
        int groups = n / 4;
        for (int i = 0; i < groups; ++i)
            for (int k = 0; k < 4; ++k) r[k] = __fadd_rn(r[k], v[i * 4 + k]);
        for (int i = groups * 4; i < n; ++i) r[0] = __fadd_rn(r[0], v[i]);
        return __fadd_rn(__fadd_rn(__fadd_rn(r[0], r[1]), r[2]), r[3]);
    }
    // n <= 256: at most 8 groups of four 8-lane vectors, below the cascade's
    // first level (16 groups), so each accumulator is a plain running sum.
    float part[4][8];
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int l = 0; l < 8; ++l) part[k][l] = 0.f;
    const int nvec = n / 8, nilp = nvec / 4;
    for (int i = 0; i < nilp; ++i)
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
            for (int l = 0; l < 8; ++l) part[k][l] = __fadd_rn(part[k][l], v[(i * 4 + k) * 8 + l]);
    for (int vv = nilp * 4; vv < nvec; ++vv)
#pragma unroll
        for (int l = 0; l < 8; ++l) part[0][l] = __fadd_rn(part[0][l], v[vv * 8 + l]);
#pragma unroll
    for (int k = 1; k < 4; ++k)
#pragma unroll
        for (int l = 0; l < 8; ++l) part[0][l] = __fadd_rn(part[0][l], part[k][l]);
    float total = 0.f;
    for (int i = nvec * 8; i < n; ++i) total = __fadd_rn(total, v[i]);
#pragma unroll
    for (int l = 0; l < 8; ++l) total = __fadd_rn(total, part[0][l]);
    return total;
}

// The cascade torch.mean(0) applies per column (4 levels, blocks of
// 2^max(4, ceil(log2 n)/4) rows), driven by a functor that yields the
// column's values in row order.  Sequential per thread.
template <typename Get>
__device__ __forceinline__ float torch_cascade_sum(int64_t n, Get get) {
    const int levels = 4;
    int lp = ceil_log2_i64(n) / levels;
    if (lp < 4) lp = 4;
    const int64_t step = (int64_t)1 << lp, mask = step - 1;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int64_t i = 0;
    while (i + step <= n) {
        for (int64_t s = 0; s < step; ++s, ++i) acc[0] = __fadd_rn(acc[0], get(i));
        for (int j = 1; j < levels; ++j) {
            acc[j] = __fadd_rn(acc[j], acc[j - 1]);
            acc[j - 1] = 0.f;
            if ((i & (mask << (j * lp))) != 0) break;
        }
    }
    for (; i < n; ++i) acc[0] = __fadd_rn(acc[0], get(i));
    for (int j = 1; j < levels; ++j) acc[0] = __fadd_rn(acc[0], acc[j]);
    return acc[0];
}

}  // namespace pk

#define PK_CHECK_LAUNCH()                              \
    do {                                               \
        cudaError_t e__ = cudaGetLastError();          \
        if (e__ != cudaSuccess) return (int)e__;       \
    } while (0)
