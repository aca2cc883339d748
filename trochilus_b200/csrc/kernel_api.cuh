// kernel_api.cuh: device side of the kernel-level entry points (tr_matmul_grouped, tr_softmax,
// tr_swiglu), for any shape the reference's API takes with these types: a grouped GEMV where each
// warp or half-warp owns a weight row and every input row of its group, plus element-wise kernels.
// Numerics as the layer kernels (layouts.cuh): Trochilus's scalar definitions, bit for bit.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include "common.cuh"
#include "expf.cuh"
#include "layouts.cuh"

// one warp per 256-block of an input row: Q4_K's prepared rows
__global__ void trx_kapi_prep_q4x(const float *__restrict__ x, int n_in, int cols, uint32_t *__restrict__ q,
                                  double *__restrict__ bf, double *__restrict__ sc) {
    const int nsb = cols / 256;
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int p = gw / nsb, s = gw % nsb;
    if (p >= n_in) return;
    trx_prep_q4x_block(x + (int64_t)p * cols + 256 * s, q + (int64_t)p * cols, s, nsb, bf + (int64_t)p * (cols / 32) + 8 * s,
                       sc + (int64_t)p * nsb + s, threadIdx.x & 31);
}

// A small call's first kernel: its group table and offsets (tab_bytes, a multiple of 4) and its input rows (total
// floats), from mapped pinned host memory (read over the host link) into device memory; lc: the rows go into LC
// order (the Q8_0 and Q6_K dots' input layout), else as they are
__global__ void trx_kapi_pull(const uint32_t *__restrict__ h_tab, int tab_bytes, uint32_t *__restrict__ d_tab,
                              const float *__restrict__ h_x, int64_t total, int cols, float *__restrict__ d_x, int lc) {
    const int64_t i0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x, n = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = i0; i < tab_bytes / 4; i += n) d_tab[i] = h_tab[i];
    for (int64_t i = i0; i < total; i += n) {
        const int64_t p = i / cols;
        const int k = (int)(i % cols);
        d_x[lc ? p * cols + trx_lc_pos(k) : i] = h_x[i];
    }
}

__global__ void trx_kapi_lc(const float *__restrict__ x, int64_t total, int cols, float *__restrict__ y) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t p = i / cols;
        const int k = (int)(i % cols);
        y[p * cols + trx_lc_pos(k)] = x[i];
    }
}

// a Q4_K row of any number of blocks by one warp, 8 blocks a pass
__device__ __forceinline__ float trx_q4k_row_any(const uint8_t *__restrict__ row, int nsb,
                                                 const uint32_t *__restrict__ planes, const double *__restrict__ bf,
                                                 const double *__restrict__ sc, int lane) {
    double y = 0.0;
    const int c = lane & 3;
    for (int s0 = 0; s0 < nsb; s0 += 8) {
        const int s = s0 + (lane >> 2);
        const bool valid = s < nsb;
        int64_t T = 0, M = 0;
        uint4 hdr = make_uint4(0, 0, 0, 0);
        TrxQ4X X;
        X.sc = 0.0;
        if (valid) {
            trx_q4x_load(planes + 2048 * (s >> 3), trx_q4x_lanes(s, nsb), lane, bf + 8 * s, sc + s, X);
            const uint8_t *blk = row + 144 * s;
            hdr = __ldg(reinterpret_cast<const uint4 *>(blk));
            const uint4 q0 = __ldg(reinterpret_cast<const uint4 *>(blk + 16 + 32 * c));
            const uint4 q1 = __ldg(reinterpret_cast<const uint4 *>(blk + 32 + 32 * c));
            trx_q4k_chunk(hdr, q0, q1, c, X, T, M);
        }
        const double v = trx_q4k_value(hdr, T, M, X.sc); // every lane takes part in the shuffles
        for (int i = 0; i < 8 && s0 + i < nsb; i++) y = __dadd_rn(y, trx_shfl_d(v, 4 * i));
    }
    return __double2float_rn(y);
}

template <int TYPE>
__global__ void __launch_bounds__(256) trx_kapi_grouped_k(const uint8_t *const *__restrict__ mats,
                                                          const int32_t *__restrict__ offsets, int rows, int cols,
                                                          const float *__restrict__ x, const uint32_t *__restrict__ xq,
                                                          const double *__restrict__ bf, const double *__restrict__ sc,
                                                          float *__restrict__ y) {
    const int g = blockIdx.y;
    const int p0 = offsets[g], p1 = offsets[g + 1];
    if (p1 <= p0) return;
    const uint8_t *W = mats[g];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t rb = trx_row_bytes(TYPE, cols);
    if (TYPE == TRX_Q4_K) { // one row per warp, 8 rows a block
        const int r = blockIdx.x * 8 + warp;
        if (r >= rows) return;
        const int nsb = cols / 256;
        for (int p = p0; p < p1; p++) {
            const float v = trx_q4k_row_any(W + (int64_t)r * rb, nsb, xq + (int64_t)p * cols, bf + (int64_t)p * (cols / 32),
                                            sc + (int64_t)p * nsb, lane);
            if (lane == 0) y[(int64_t)p * rows + r] = v;
        }
    } else { // a half-warp per row, 16 rows a block
        const int r0 = blockIdx.x * 16 + 2 * warp + (lane >> 4);
        const bool valid = r0 < rows;
        const int r = valid ? r0 : rows - 1; // every lane takes part in the shuffles
        for (int p = p0; p < p1; p++) {
            float v;
            if (TYPE == TRX_Q8_0)
                v = trx_q8l_dot(W + (int64_t)r * rb, reinterpret_cast<const float *>(xq) + (int64_t)p * cols, cols / 256,
                                lane & 15);
            else if (TYPE == TRX_Q6_K)
                v = trx_q6l_dot(W + (int64_t)r * (cols / 256) * 208,
                                W + (int64_t)rows * (cols / 256) * 208 + (int64_t)r * (cols / 256) * 2,
                                reinterpret_cast<const float *>(xq) + (int64_t)p * cols, cols / 256, lane & 15);
            else
                v = trx_plain_dot<TYPE>(W + (int64_t)r * rb, x + (int64_t)p * cols, cols, lane & 15);
            if (valid && (lane & 15) == 0) y[(int64_t)p * rows + r] = v;
        }
    }
}

// prep false (Q4_K): dq, dbf, dsc already hold dx's prepared rows (an earlier call on the same inputs wrote them)
// lc_done: dq already holds dx's rows in LC order (Q8_0, Q6_K: trx_kapi_pull wrote them)
inline bool trx_kapi_grouped(int type, int64_t rows, int64_t cols, const uint8_t *const *dg, const int32_t *doff,
                             int n_groups, int n_in, const float *dx, uint32_t *dq, double *dbf, double *dsc, float *dy,
                             cudaStream_t st, bool prep = true, bool lc_done = false) {
    if (type == TRX_Q4_K) {
        const int64_t warps = (int64_t)n_in * (cols / 256);
        if (prep) trx_kapi_prep_q4x<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(dx, n_in, (int)cols, dq, dbf, dsc);
        dim3 grid((unsigned)((rows + 7) / 8), (unsigned)n_groups);
        trx_kapi_grouped_k<TRX_Q4_K><<<grid, 256, 0, st>>>(dg, doff, (int)rows, (int)cols, dx, dq, dbf, dsc, dy);
        return true;
    }
    dim3 grid((unsigned)((rows + 15) / 16), (unsigned)n_groups);
    if (type == TRX_Q8_0 || type == TRX_Q6_K) {
        const int64_t total = (int64_t)n_in * cols;
        if (!lc_done)
            trx_kapi_lc<<<(unsigned)std::min<int64_t>((total + 255) / 256, 4096), 256, 0, st>>>(
                dx, total, (int)cols, reinterpret_cast<float *>(dq));
        if (type == TRX_Q8_0)
            trx_kapi_grouped_k<TRX_Q8_0><<<grid, 256, 0, st>>>(dg, doff, (int)rows, (int)cols, dx, dq, dbf, dsc, dy);
        else
            trx_kapi_grouped_k<TRX_Q6_K><<<grid, 256, 0, st>>>(dg, doff, (int)rows, (int)cols, dx, dq, dbf, dsc, dy);
        return true;
    }
    if (type == TRX_F32)
        trx_kapi_grouped_k<TRX_F32><<<grid, 256, 0, st>>>(dg, doff, (int)rows, (int)cols, dx, dq, dbf, dsc, dy);
    else if (type == TRX_BF16)
        trx_kapi_grouped_k<TRX_BF16><<<grid, 256, 0, st>>>(dg, doff, (int)rows, (int)cols, dx, dq, dbf, dsc, dy);
    else
        trx_kapi_grouped_k<TRX_F16><<<grid, 256, 0, st>>>(dg, doff, (int)rows, (int)cols, dx, dq, dbf, dsc, dy);
    return true;
}

// dst row p = src row map[p] (cols floats, a multiple of 4; 16-byte aligned rows), a block a row
__global__ void __launch_bounds__(256) trx_kapi_gather_k(const float *__restrict__ src, const int32_t *__restrict__ map,
                                                         int cols, float *__restrict__ dst) {
    const int64_t p = blockIdx.x;
    const float4 *s = reinterpret_cast<const float4 *>(src + (int64_t)map[p] * cols);
    float4 *d = reinterpret_cast<float4 *>(dst + p * cols);
    for (int i = threadIdx.x; i < cols / 4; i += blockDim.x) d[i] = s[i];
}

// tr_softmax over n values by one block of 256 threads: the max as the reference's serial scan from x[0], the exp
// of each difference, the 16-lane sum (lane l adds elements l, l + 16, ... in order), the divisions
__device__ __forceinline__ void trx_softmax_block(float *__restrict__ x, int64_t n) {
    __shared__ float red[8];
    __shared__ float s_m, s_sum;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float m = -__int_as_float(0x7f800000);
    for (int64_t i = tid; i < n; i += blockDim.x)
        if (x[i] == x[i]) m = fmaxf(m, x[i]);
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (tid == 0) {
        float mm = red[0];
        for (int i = 1; i < 8; i++) mm = fmaxf(mm, red[i]);
        s_m = x[0] != x[0] ? x[0] : mm;
    }
    __syncthreads();
    const float mx = s_m;
    for (int64_t i = tid; i < n; i += blockDim.x) x[i] = trx_expf(__fsub_rn(x[i], mx));
    __syncthreads();
    if (warp == 0) {
        float acc = 0.0f;
        if (lane < 16)
            for (int64_t i = lane; i < n; i += 16) acc = __fadd_rn(acc, x[i]);
        acc = trx_lane_tree16(acc);
        if (lane == 0) s_sum = acc;
    }
    __syncthreads();
    const float sum = s_sum;
    for (int64_t i = tid; i < n; i += blockDim.x) x[i] = __fdiv_rn(x[i], sum);
}

__global__ void __launch_bounds__(256) trx_kapi_softmax_k(float *__restrict__ x, int64_t n) { trx_softmax_block(x, n); }

// tr_softmax over each of gridDim.x rows of n values, stride floats apart, a block a row
__global__ void __launch_bounds__(256) trx_softmax_rows_k(float *__restrict__ x, int64_t n, int64_t stride) {
    trx_softmax_block(x + (int64_t)blockIdx.x * stride, n);
}

inline bool trx_kapi_softmax(float *d, int64_t n, cudaStream_t st) {
    trx_kapi_softmax_k<<<1, 256, 0, st>>>(d, n);
    return true;
}

__global__ void trx_kapi_swiglu_k(float *__restrict__ x, const float *__restrict__ y, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float v = x[i];
        const float e = trx_expf(-v);
        x[i] = __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, e)), y[i]);
    }
}

inline bool trx_kapi_swiglu(float *dx, const float *dy, int64_t n, cudaStream_t st) {
    trx_kapi_swiglu_k<<<(unsigned)std::min<int64_t>((n + 255) / 256, 8192), 256, 0, st>>>(dx, dy, n);
    return true;
}
