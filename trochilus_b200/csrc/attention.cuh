// attention.cuh: one decode token's attention on the B200 with the CPU's bits (the contract of Trochilus's
// src/backend/gpu_attn.h:1-9: tr_attention_group for a single query, which is tr_attention_head,
// src/kernels/kernels.c:1521-1528, head by head). The session's keys and values live in HBM, per layer and head
// contiguous over positions ([layer][head][pos][head_dim] f32), so that a head's rows stream as one range.
//
//  store    a call's k and v rows ([n_tok][n_head * head_dim]) into their positions of the layer's cache.
//  scores   s[h][t] = dot(q_h, key t) * scale: a half-warp a position, lane l the elements l + 16 m in increasing m
//           (the 16-lane contract, src/kernels/kernels.c:19-23), the lanes joined by the tree, then the scale.
//  softmax  tr_softmax over each head's row (kernel_api.cuh's block softmax).
//  values   out[h][d] = +0, then out = out + p_t v_t[d] in increasing t (k_axpy_f32, kernels.c:34-36): a chain of
//           n_pos rounded steps per output element, which no split may reorder. One CTA a head: a producer warp
//           streams chunks of 64 positions of the head's values (one contiguous 32 KB bulk copy each) and their
//           probabilities into a ring of shared-memory stages; 128 threads, one per element d, run the chains.
// head_dim is 128 (the reference's only supported shape). Every wait is bounded; a give-up sets the error word.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include "bulk.cuh"
#include "common.cuh"

#define TRX_ATTN_HD 128
#define TRX_ATTN_CHUNK 64                                  // positions a stage
#define TRX_ATTN_STAGES 4
#define TRX_ATTN_STAGE_BYTES (TRX_ATTN_CHUNK * TRX_ATTN_HD * 4 + TRX_ATTN_CHUNK * 4)

// src rows [n_tok][n_head * 128] into cache[head][pos0 + i][128] (the layer's part of the cache), a warp a row and
// head, a float4 a lane
__global__ void __launch_bounds__(256) trx_attn_store(const float *__restrict__ src, int n_tok, int n_head,
                                                      int64_t pos0, int64_t n_ctx, float *__restrict__ cache) {
    const int w = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (w >= n_tok * n_head) return;
    const int i = w / n_head, h = w % n_head;
    const float4 v = reinterpret_cast<const float4 *>(src + ((int64_t)i * n_head + h) * TRX_ATTN_HD)[lane];
    reinterpret_cast<float4 *>(cache + ((int64_t)h * n_ctx + pos0 + i) * TRX_ATTN_HD)[lane] = v;
}

// scores[h * s_stride + t] for t < n_pos: 16 positions a block of 256 threads, blockIdx.y the head. The block also
// asks L2 for the same positions' value rows (a bulk prefetch, no data moved to the SM), so that the value kernel's
// few CTAs stream them from L2 rather than HBM.
__global__ void __launch_bounds__(256) trx_attn_scores(const float *__restrict__ q, const float *__restrict__ keys,
                                                       const float *__restrict__ values, int n_pos, int64_t n_ctx,
                                                       float scale, float *__restrict__ scores, int64_t s_stride) {
    const int h = blockIdx.y, l = threadIdx.x & 15;
    if (threadIdx.x == 0) {
        const int first = blockIdx.x * 16, rows = min(16, n_pos - first);
        const float *v = values + ((int64_t)h * n_ctx + first) * TRX_ATTN_HD;
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(v), "r"((uint32_t)rows * TRX_ATTN_HD * 4)
                     : "memory");
    }
    const int t0 = blockIdx.x * 16 + (threadIdx.x >> 4);
    const int t = t0 < n_pos ? t0 : n_pos - 1; // every lane takes part in the tree
    const float *qh = q + (int64_t)h * TRX_ATTN_HD;
    const float *kt = keys + ((int64_t)h * n_ctx + t) * TRX_ATTN_HD;
    float acc = 0.0f;
#pragma unroll
    for (int m = 0; m < TRX_ATTN_HD / 16; m++) acc = __fadd_rn(acc, __fmul_rn(__ldg(qh + l + 16 * m), kt[l + 16 * m]));
    const float s = __fmul_rn(trx_lane_tree16(acc), scale);
    if (l == 0 && t0 < n_pos) scores[(int64_t)h * s_stride + t0] = s;
}

// out[h][d] = the chain over the head's n_pos probabilities and values (one CTA a head: warps 0-3 the 128 chains,
// warp 4 the producer). probs: the softmaxed scores, s_stride floats a head (a multiple of 4, and room up to the
// next multiple of TRX_ATTN_CHUNK); err: set to 9 when a wait gives up
__global__ void __launch_bounds__(160, 1) trx_attn_values(const float *__restrict__ probs, int64_t s_stride,
                                                          const float *__restrict__ values, int n_pos, int64_t n_ctx,
                                                          float *__restrict__ out, int32_t *__restrict__ err) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[TRX_ATTN_STAGES], empty[TRX_ATTN_STAGES];
    __shared__ int s_failed;
    const int h = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n_chunks = (n_pos + TRX_ATTN_CHUNK - 1) / TRX_ATTN_CHUNK;
    if (tid == 0) {
        for (int s = 0; s < TRX_ATTN_STAGES; s++) {
            trx_mbar_init(&full[s], 1);
            trx_mbar_init(&empty[s], 4);
        }
        s_failed = 0;
        trx_fence_barrier_init();
    }
    __syncthreads();
    const float *vh = values + (int64_t)h * n_ctx * TRX_ATTN_HD;
    const float *ph = probs + (int64_t)h * s_stride;
    if (warp == 4) {
        if (lane == 0) {
            int issued = 0;
            for (int c = 0; c < n_chunks; c++) {
                const int s = c % TRX_ATTN_STAGES;
                if (c >= TRX_ATTN_STAGES && !trx_mbar_wait(&empty[s], ((c / TRX_ATTN_STAGES) - 1) & 1, TRX_WAIT_NS)) {
                    atomicExch(&s_failed, 1);
                    break;
                }
                if (*(volatile int *)&s_failed) break;
                const int t0 = c * TRX_ATTN_CHUNK, rows = min(TRX_ATTN_CHUNK, n_pos - t0);
                const uint32_t vbytes = (uint32_t)rows * TRX_ATTN_HD * 4, pbytes = (uint32_t)((rows + 3) / 4) * 16;
                uint8_t *st = smem + (size_t)s * TRX_ATTN_STAGE_BYTES;
                trx_mbar_expect_tx(&full[s], vbytes + pbytes);
                trx_bulk_g2s(st, vh + (int64_t)t0 * TRX_ATTN_HD, vbytes, &full[s]);
                trx_bulk_g2s(st + TRX_ATTN_CHUNK * TRX_ATTN_HD * 4, ph + t0, pbytes, &full[s]);
                issued++;
            }
            // every copy in flight lands before the shared memory goes away: only a stage's latest copy can be in
            // flight (a stage is refilled after its consumers saw the one before land), and only its phase parity is
            // unambiguous
            for (int c = max(0, issued - TRX_ATTN_STAGES); c < issued; c++)
                trx_mbar_wait(&full[c % TRX_ATTN_STAGES], (c / TRX_ATTN_STAGES) & 1, TRX_WAIT_NS);
        }
    } else {
        const int d = tid; // 0..127
        float acc = 0.0f;
        for (int c = 0; c < n_chunks; c++) {
            const int s = c % TRX_ATTN_STAGES;
            const bool ok = trx_mbar_wait(&full[s], (c / TRX_ATTN_STAGES) & 1, TRX_WAIT_NS);
            if (!__all_sync(0xffffffffu, ok)) {
                if (lane == 0) atomicExch(&s_failed, 1);
                break;
            }
            const uint8_t *st = smem + (size_t)s * TRX_ATTN_STAGE_BYTES;
            const float *vs = reinterpret_cast<const float *>(st);
            const float *ps = reinterpret_cast<const float *>(st + TRX_ATTN_CHUNK * TRX_ATTN_HD * 4);
            const int rows = min(TRX_ATTN_CHUNK, n_pos - c * TRX_ATTN_CHUNK);
            for (int r = 0; r < rows; r++) acc = __fadd_rn(acc, __fmul_rn(ps[r], vs[r * TRX_ATTN_HD + d]));
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(trx_smem(&empty[s])) : "memory");
        }
        out[(int64_t)h * TRX_ATTN_HD + d] = acc;
    }
    __syncthreads();
    if (tid == 0 && s_failed) atomicCAS(err, 0, 9);
}

// keeps one warp busy until the host sets *stop (mapped pinned memory) or ns have passed (the reference's warm-up
// of a GPU whose clocks drop between calls, src/backend/gpu_attn.h:14-17): bounded by ns on every path
__global__ void trx_attn_warm(const volatile uint32_t *stop, uint64_t ns) {
    const uint64_t t0 = trx_globaltimer();
    while (*stop == 0u && trx_globaltimer() - t0 < ns) __nanosleep(1000);
}
