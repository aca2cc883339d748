// ep.cuh: the device side of expert parallelism. Experts are placed E / N per GPU; every rank routes its own tokens
// (the router is replicated), sends each (token, slot) row to the rank that holds its expert, and sums the returned
// expert outputs in increasing expert id.
//
//  pack     a stable counting sort of the rank's (token, slot) rows by destination rank, and the rows and expert ids
//           in that order (the send buffer of an all-to-all).
//  experts  the expert FFN of rows that arrive in any order, each with its expert id: a stable counting sort by
//           expert, the grouped gate / up products, SwiGLU, the grouped down product (the kernel-level kernels of
//           kernel_api.cuh, the same exact definitions as the layer kernels), the outputs back in arrival order.
//  combine  prefill.cuh's trx_k_pf_combine over the returned rows (the send order's place of each row).
// Every row's arithmetic is the one-GPU road's, so the layer's output is bit for bit the one-GPU output.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include "kernel_api.cuh"

// Stable counting sort of n keys into nk <= 64 buckets by one block of 1024 threads (32 warps, each a contiguous
// chunk of j). key(j) = src64 ? src64[j] / div : src32[j]. Writes offsets[0..nk], place[j] (the row's position in
// bucket order), xmap[place[j]] = j, and counts[b] when counts is not NULL.
__global__ void __launch_bounds__(1024) trx_k_stable_sort(const int64_t *__restrict__ src64, const int32_t *__restrict__ src32,
                                                          int64_t div, int n, int nk, int32_t *__restrict__ offsets,
                                                          int32_t *__restrict__ place, int32_t *__restrict__ xmap,
                                                          int32_t *__restrict__ counts) {
    __shared__ int wc[32][64];
    __shared__ int tot[65];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int chunk = (n + 31) / 32, j0 = warp * chunk, j1 = min(n, j0 + chunk);
    for (int e = lane; e < 64; e += 32) wc[warp][e] = 0;
    __syncwarp();
    auto key = [&](int j) { // a key out of range is dropped (no row of ours carries one)
        const int k = src64 ? (int)(src64[j] / div) : src32[j];
        return k >= 0 && k < nk ? k : -1;
    };
    for (int b = j0; b < j1; b += 32) {
        const int j = b + lane;
        const int k = j < j1 ? key(j) : -1;
        const unsigned peers = __match_any_sync(0xffffffffu, k);
        if (k >= 0 && lane == __ffs(peers) - 1) wc[warp][k] += __popc(peers);
        __syncwarp();
    }
    __syncthreads();
    if (tid < 64) { // bucket tid: its total, and each warp's exclusive start within the bucket
        int s = 0;
        for (int w = 0; w < 32; w++) {
            const int c = wc[w][tid];
            wc[w][tid] = s;
            s += c;
        }
        tot[tid] = tid < nk ? s : 0;
    }
    __syncthreads();
    if (tid == 0) {
        int s = 0;
        for (int e = 0; e < nk; e++) {
            const int c = tot[e];
            tot[e] = s;
            s += c;
        }
        tot[nk] = s;
    }
    __syncthreads();
    if (tid <= nk) offsets[tid] = tot[tid];
    if (counts && tid < nk) counts[tid] = tot[tid + 1] - tot[tid];
    if (tid < 64)
        for (int w = 0; w < 32; w++) wc[w][tid] += tot[tid];
    __syncthreads();
    for (int b = j0; b < j1; b += 32) {
        const int j = b + lane;
        const int k = j < j1 ? key(j) : -1;
        const unsigned peers = __match_any_sync(0xffffffffu, k);
        if (k >= 0) {
            const int pos = wc[warp][k] + __popc(peers & ((1u << lane) - 1u));
            place[j] = pos;
            xmap[pos] = j;
        }
        __syncwarp();
        if (k >= 0 && lane == __ffs(peers) - 1) wc[warp][k] += __popc(peers);
        __syncwarp();
    }
}

// dst row pos = src row xmap[pos] / div (cols floats, cols % 4 == 0); ids_out[pos] = ids_in[xmap[pos]] when given.
// Rows past *n_sorted (the sort's total: rows with a dropped key) are not touched. cap > 0 (the pack's padded form):
// the rows of bucket b = ids_in[j] / kdiv go to b cap + their rank in the bucket instead, and place[j] says so.
__global__ void __launch_bounds__(256) trx_k_gather_rows(const float *__restrict__ src, const int32_t *__restrict__ xmap,
                                                         const int32_t *__restrict__ n_sorted, int div, int cols,
                                                         float *__restrict__ dst, const int64_t *__restrict__ ids_in,
                                                         int32_t *__restrict__ ids_out, const int32_t *__restrict__ offsets,
                                                         int cap, int64_t kdiv, int32_t *__restrict__ place) {
    const int pos = blockIdx.x;
    if (pos >= *n_sorted) return;
    const int j = xmap[pos];
    int dpos = pos;
    if (cap > 0) {
        const int b = (int)(ids_in[j] / kdiv);
        dpos = b * cap + pos - offsets[b];
        if (threadIdx.x == 0) place[j] = dpos;
    }
    const float4 *s = reinterpret_cast<const float4 *>(src + (int64_t)(j / div) * cols);
    float4 *d = reinterpret_cast<float4 *>(dst + (int64_t)dpos * cols);
    for (int i = threadIdx.x; i < cols / 4; i += blockDim.x) d[i] = s[i];
    if (ids_out && threadIdx.x == 0) ids_out[dpos] = (int32_t)ids_in[j];
}

// out row xmap[pos] = src row pos, for pos < *n_sorted
__global__ void __launch_bounds__(256) trx_k_scatter_rows(const float *__restrict__ src, const int32_t *__restrict__ xmap,
                                                          const int32_t *__restrict__ n_sorted, int cols,
                                                          float *__restrict__ out) {
    const int pos = blockIdx.x;
    if (pos >= *n_sorted) return;
    const float4 *s = reinterpret_cast<const float4 *>(src + (int64_t)pos * cols);
    float4 *d = reinterpret_cast<float4 *>(out + (int64_t)xmap[pos] * cols);
    for (int i = threadIdx.x; i < cols / 4; i += blockDim.x) d[i] = s[i];
}
