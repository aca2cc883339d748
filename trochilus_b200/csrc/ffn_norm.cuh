// ffn_norm.cuh: the MoE block's input normalisation (ffn_norm, Trochilus src/models/olmoe.c:1834-1840), so that the
// layer hook can take the residual stream itself: normed = RMSNorm(x) with the layer's ffn_norm weight, per token as
// norm_body applies tr_rmsnorm (olmoe.c:1360-1366, src/kernels/kernels.c:1351-1360):
//   sumsq = the f32 dot of the row with itself under the 16-lane contract (each product rounded, added to lane
//           k mod 16 in order, the lanes joined by the tree; kernels.c:19-23)
//   mean = sumsq / n, inv = 1 / sqrtf(mean + eps), normed[i] = (x[i] * inv) * w[i], every step one IEEE rounding.
#pragma once
#include <cstdint>
#include "common.cuh"

// One block per token (128 threads); x may be device memory or pinned host memory mapped into the device (the
// row is read once, coalesced, into shared memory). Dynamic shared memory: H floats.
__global__ void __launch_bounds__(128) trx_k_ffn_norm(const float *__restrict__ x, const float *__restrict__ w, float eps,
                                                      int H, float *__restrict__ normed) {
    extern __shared__ float sx[];
    __shared__ float s_inv;
    const int t = blockIdx.x, tid = threadIdx.x;
    const float *xr = x + (int64_t)t * H;
    // 16 loads a thread in flight at once (x may be host memory: one round trip over the link, not sixteen)
    for (int base = 0; base < H; base += 16 * (int)blockDim.x) {
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const int i = base + j * (int)blockDim.x + tid;
            v[j] = i < H ? xr[i] : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const int i = base + j * (int)blockDim.x + tid;
            if (i < H) sx[i] = v[j];
        }
    }
    __syncthreads();
    if (tid < 32) {
        float acc = 0.0f;
        if (tid < 16)
            for (int k = tid; k < H; k += 16) acc = __fadd_rn(acc, __fmul_rn(sx[k], sx[k]));
        acc = trx_lane_tree16(acc); // lanes 16-31 join with zeros and are not read
        if (tid == 0) s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, (float)H), eps)));
    }
    __syncthreads();
    const float inv = s_inv;
    for (int i = tid; i < H; i += blockDim.x) normed[(int64_t)t * H + i] = __fmul_rn(__fmul_rn(sx[i], inv), w[i]);
}
