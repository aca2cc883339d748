// moe_kernels.cuh: the decode-regime MoE layer as four kernels on one stream.
//
//   trx_k_router   router logits (16-lane contract), then in the last block to finish: the softmax
//                  (correctly rounded exp), top-k by repeated argmax (ties to the lower id), sort of the
//                  k by id, and the stable counting sort of the (token, slot) rows by expert; extra
//                  blocks prepare each token's input row for the expert products
//   trx_k_gateup   per (expert, block of rows): gate and up dots of every row of the expert's segment,
//                  SwiGLU fused, h written (natural order, or the LC order the lane-contract down reads)
//   trx_k_prep     Q4_K down only: h rows prepared for Q4_K's integer definition
//   trx_k_down     per (expert, block of output rows): down dots into h3; the last block to finish a
//                  block of output rows adds the k expert outputs of every token in increasing expert
//                  id and adds the sum to the residual, exactly Trochilus's mix_body
//
// Trochilus references: forward_layer's MoE block src/models/olmoe.c:1845-1933; route_token /
// top_experts olmoe.c:1455-1502; the counting sort olmoe.c:1850-1861; tr_softmax
// src/kernels/kernels.c:1377-1388; SwiGLU kernels.c:1397-1421; mix_body olmoe.c:1432-1446.
#pragma once
#include <cstdint>
#include "common.cuh"
#include "expf.cuh"
#include "layouts.cuh"

#define TRX_MAX_EXPERTS 64
#define TRX_MAX_USED 32
#define TRX_GU_ROWS 32   // gate/up rows per work item (8 warps x 4)
#define TRX_DN_ROWS 64   // down output rows per work item

struct TrxLayer {
    int router_type, gate_type, up_type, down_type;
    const uint8_t *router;
    const float *router_bias; // NULL: none
    const uint8_t *gate, *up, *down; // n_expert matrices each
    int64_t gate_mb, up_mb, down_mb; // bytes per expert matrix
};

struct TrxShape {
    int E, k, H, F, norm_topk;
};

struct TrxWork {
    float *logits;      // [T][E]
    int32_t *sel_id;    // [R]
    float *sel_w;       // [R]
    int32_t *offsets;   // [E + 1]
    int32_t *place;     // [R]
    int32_t *xmap;      // [R] token of grouped row p
    int32_t *active;    // [E]
    int32_t *n_active;  // [1]
    uint32_t *route_cnt;  // [1]
    uint32_t *comb_cnt;   // [H / TRX_DN_ROWS]
    float *x_lc;        // [T][H]
    uint32_t *xq;       // [T][H]
    double *xq_bf;      // [T][H / 32]
    double *xq_sc;      // [T][H / 256]
    float *h;           // [R][F]
    uint32_t *hq;       // [R][F]
    double *hq_bf;      // [R][F / 32]
    double *hq_sc;      // [R][F / 256]
    float *h3;          // [R][H]
    int64_t *out_sel_id;  // optional outputs (NULL: not written)
    float *out_sel_w;
    int64_t *out_offsets;
    int64_t *out_place;
    float *out_logits;
};

__device__ __forceinline__ bool trx_lc_type(int t) { return t == TRX_Q8_0 || t == TRX_Q6_K; }

// ---------------------------------------------------------------------------------------------
// router + route + dispatch

__device__ void trx_route_token(const float *__restrict__ logits, int E, int k, int norm_topk, int lane,
                                int32_t *ids_out, float *w_out) {
    const bool ok0 = lane < E, ok1 = lane + 32 < E;
    const float v0 = ok0 ? __ldcg(logits + lane) : 0.0f, v1 = ok1 ? __ldcg(logits + lane + 32) : 0.0f;
    // max: the reference's serial scan from x[0] with strict > keeps x[0] when it is a NaN, else it is the
    // largest non-NaN value (which x[0] is one of)
    float m = -__int_as_float(0x7f800000);
    if (ok0 && v0 == v0) m = fmaxf(m, v0);
    if (ok1 && v1 == v1) m = fmaxf(m, v1);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float x0 = __shfl_sync(0xffffffffu, v0, 0);
    if (x0 != x0) m = x0;
    const float e0 = ok0 ? trx_expf(__fsub_rn(v0, m)) : 0.0f;
    const float e1 = ok1 ? trx_expf(__fsub_rn(v1, m)) : 0.0f;
    // lane sum: lane l (< 16) adds elements l, l+16, l+32, l+48 in order from +0
    const float b = __shfl_sync(0xffffffffu, e0, (lane & 15) + 16);
    const float d = __shfl_sync(0xffffffffu, e1, (lane & 15) + 16);
    float acc = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(0.0f, e0), b), e1), d);
    acc = trx_lane_tree16(acc);
    const float sum = __shfl_sync(0xffffffffu, acc, 0);
    const float p0 = __fdiv_rn(e0, sum), p1 = __fdiv_rn(e1, sum);
    bool t0 = !ok0, t1 = !ok1; // taken (or absent)
    int ids[TRX_MAX_USED];
    float ws[TRX_MAX_USED];
    for (int s = 0; s < k; s++) {
        const unsigned u0 = __ballot_sync(0xffffffffu, !t0), u1 = __ballot_sync(0xffffffffu, !t1);
        const int f = u0 ? __ffs(u0) - 1 : 32 + __ffs(u1) - 1; // first untaken id
        const float pf = __shfl_sync(0xffffffffu, f < 32 ? p0 : p1, f & 31);
        int best;
        if (pf != pf) {
            best = f;
        } else {
            // largest non-NaN untaken, lowest id among equals
            float bv = 0.0f;
            int bi = 1 << 30;
            if (!t0 && p0 == p0) { bv = p0; bi = lane; }
            if (!t1 && p1 == p1 && (bi == (1 << 30) || p1 > bv)) { bv = p1; bi = lane + 32; }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                const bool take = oi != (1 << 30) && (bi == (1 << 30) || ov > bv || (ov == bv && oi < bi));
                if (take) { bv = ov; bi = oi; }
            }
            best = bi;
        }
        const float pb = __shfl_sync(0xffffffffu, best < 32 ? p0 : p1, best & 31);
        if (best == lane) t0 = true;
        if (best == lane + 32) t1 = true;
        ids[s] = best;
        ws[s] = pb;
    }
    if (lane == 0) {
        if (norm_topk) {
            float sm = 0.0f;
            for (int s = 0; s < k; s++) sm = __fadd_rn(sm, ws[s]);
            for (int s = 0; s < k; s++) ws[s] = __fdiv_rn(ws[s], sm);
        }
        for (int i = 1; i < k; i++) { // insertion sort by id
            const int id = ids[i];
            const float w = ws[i];
            int j = i - 1;
            while (j >= 0 && ids[j] > id) {
                ids[j + 1] = ids[j];
                ws[j + 1] = ws[j];
                j--;
            }
            ids[j + 1] = id;
            ws[j + 1] = w;
        }
        for (int s = 0; s < k; s++) {
            ids_out[s] = ids[s];
            w_out[s] = ws[s];
        }
    }
}

// Stable counting sort of R rows by expert, by one block of 256 threads (8 warps). place[j] = the
// row's position in the grouped order: its expert's start plus the rows of that expert before j.
__device__ void trx_block_counting_sort(const int32_t *__restrict__ sel_id, int R, int E, int k, TrxWork w) {
    __shared__ int cnt[TRX_MAX_EXPERTS + 1];
    __shared__ int run[TRX_MAX_EXPERTS];
    __shared__ int wc[8][TRX_MAX_EXPERTS];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int e = tid; e <= E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int j = tid; j < R; j += blockDim.x) atomicAdd(&cnt[sel_id[j]], 1);
    __syncthreads();
    if (tid == 0) {
        int acc = 0, na = 0;
        for (int e = 0; e < E; e++) {
            const int c = cnt[e];
            w.offsets[e] = acc;
            if (w.out_offsets) w.out_offsets[e] = acc;
            run[e] = acc;
            if (c > 0) w.active[na++] = e;
            acc += c;
        }
        w.offsets[E] = acc;
        if (w.out_offsets) w.out_offsets[E] = acc;
        *w.n_active = na;
    }
    __syncthreads();
    for (int base = 0; base < R; base += blockDim.x) {
        const int j = base + tid;
        const int e = j < R ? sel_id[j] : -1;
        for (int i = tid; i < 8 * TRX_MAX_EXPERTS; i += blockDim.x) (&wc[0][0])[i] = 0;
        __syncthreads();
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const int rank = __popc(peers & ((1u << lane) - 1u));
        if (e >= 0 && rank == 0) wc[warp][e] = __popc(peers);
        __syncthreads();
        if (e >= 0) {
            int pos = run[e] + rank;
            for (int v = 0; v < warp; v++) pos += wc[v][e];
            w.place[j] = pos;
            w.xmap[pos] = j / k;
            if (w.out_place) w.out_place[j] = pos;
        }
        __syncthreads();
        for (int ee = tid; ee < E; ee += blockDim.x) {
            int s = 0;
            for (int v = 0; v < 8; v++) s += wc[v][ee];
            run[ee] += s;
        }
        __syncthreads();
    }
}

// grid: E router blocks + T prep blocks; 256 threads
__global__ void __launch_bounds__(256) trx_k_router(TrxLayer L, TrxShape S, const float *__restrict__ normed, int T,
                                                    TrxWork w) {
    extern __shared__ float srow[]; // H floats
    const int tid = threadIdx.x, lane = tid & 31;
    const int E = S.E, H = S.H;
    if ((int)blockIdx.x >= E) { // input preparation for the gate/up products
        const int t = blockIdx.x - E;
        const float *x = normed + (int64_t)t * H;
        if (L.gate_type == TRX_Q4_K) {
            const int nsb = H / 256;
            for (int s = tid >> 5; s < nsb; s += blockDim.x >> 5)
                trx_prep_q4x_block(x + 256 * s, w.xq + (int64_t)t * H + 256 * s, w.xq_bf + (int64_t)t * (H / 32) + 8 * s,
                                   w.xq_sc + (int64_t)t * (H / 256) + s, lane);
        } else {
            for (int kk = tid; kk < H; kk += blockDim.x) w.x_lc[(int64_t)t * H + trx_lc_pos(kk)] = x[kk];
        }
        return;
    }
    const int e = blockIdx.x;
    const int64_t rb = trx_row_bytes(L.router_type, H);
    const uint8_t *row = L.router + e * rb;
    for (int kk = tid; kk < H; kk += blockDim.x)
        srow[kk] = L.router_type == TRX_F32 ? __ldg(reinterpret_cast<const float *>(row) + kk)
                                            : trx_bf16(__ldg(reinterpret_cast<const uint16_t *>(row) + kk));
    __syncthreads();
    const int tg = tid >> 4, l = tid & 15;
    const float bias = L.router_bias ? L.router_bias[e] : 0.0f;
    for (int t0 = 0; t0 < T; t0 += 16) {
        const int t = t0 + tg < T ? t0 + tg : T - 1;
        const float *x = normed + (int64_t)t * H;
        float acc = 0.0f;
        for (int kk = l; kk < H; kk += 16) acc = __fadd_rn(acc, __fmul_rn(srow[kk], x[kk]));
        acc = trx_lane_tree16(acc);
        if (l == 0 && t0 + tg < T) {
            const float v = L.router_bias ? __fadd_rn(acc, bias) : acc;
            w.logits[(int64_t)t * E + e] = v;
            if (w.out_logits) w.out_logits[(int64_t)t * E + e] = v;
        }
    }
    // the last router block to finish routes every token
    __shared__ int s_last;
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        s_last = atomicAdd(w.route_cnt, 1u) == (unsigned)(E - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const int warp = tid >> 5, k = S.k;
    for (int t = warp; t < T; t += blockDim.x >> 5)
        trx_route_token(w.logits + (int64_t)t * E, E, k, S.norm_topk, lane, w.sel_id + (int64_t)t * k,
                        w.sel_w + (int64_t)t * k);
    __syncthreads();
    const int R = T * k;
    if (w.out_sel_id)
        for (int j = tid; j < R; j += blockDim.x) {
            w.out_sel_id[j] = w.sel_id[j];
            w.out_sel_w[j] = w.sel_w[j];
        }
    trx_block_counting_sort(w.sel_id, R, E, k, w);
    if (tid == 0) *w.route_cnt = 0u;
}

// ---------------------------------------------------------------------------------------------
// gate / up / SwiGLU

__device__ __forceinline__ float trx_silu_mul(float g, float u) {
    const float e = trx_expf(-g);
    const float silu = __fdiv_rn(g, __fadd_rn(1.0f, e));
    return __fmul_rn(silu, u);
}

// Q4_K row of 8 blocks (2048 columns) by one warp: returns float(sum_s v_s) in every lane
__device__ __forceinline__ float trx_q4k_row8(const uint8_t *__restrict__ row, const TrxQ4X &X,
                                              const double *__restrict__ bf, const double *__restrict__ sc, int lane) {
    const int s = lane >> 2, c = lane & 3;
    const uint8_t *blk = row + 144 * s;
    const uint4 hdr = __ldg(reinterpret_cast<const uint4 *>(blk));
    const uint4 q0 = __ldg(reinterpret_cast<const uint4 *>(blk + 16 + 32 * c));
    const uint4 q1 = __ldg(reinterpret_cast<const uint4 *>(blk + 32 + 32 * c));
    int64_t T = trx_q4k_chunk_T(hdr, q0, q1, c, X);
    T += trx_shfl_xor64(T, 1);
    T += trx_shfl_xor64(T, 2);
    double v = 0.0;
    if (c == 0) v = trx_q4k_finish(hdr, T, bf + 8 * s, sc[s]);
    double y = 0.0;
#pragma unroll
    for (int i = 0; i < 8; i++) y = __dadd_rn(y, trx_shfl_d(v, 4 * i));
    return __double2float_rn(y);
}

// Q4_K rows of 4 blocks (1024 columns), two per warp (half-warp each): returns the half's row value
__device__ __forceinline__ float trx_q4k_row4(const uint8_t *__restrict__ row, const TrxQ4X &X,
                                              const double *__restrict__ bf, const double *__restrict__ sc, int lane) {
    const int s = (lane >> 2) & 3, c = lane & 3;
    const uint8_t *blk = row + 144 * s;
    const uint4 hdr = __ldg(reinterpret_cast<const uint4 *>(blk));
    const uint4 q0 = __ldg(reinterpret_cast<const uint4 *>(blk + 16 + 32 * c));
    const uint4 q1 = __ldg(reinterpret_cast<const uint4 *>(blk + 32 + 32 * c));
    int64_t T = trx_q4k_chunk_T(hdr, q0, q1, c, X);
    T += trx_shfl_xor64(T, 1);
    T += trx_shfl_xor64(T, 2);
    double v = 0.0;
    if (c == 0) v = trx_q4k_finish(hdr, T, bf + 8 * s, sc[s]);
    double y = 0.0;
    const int base = lane & 16;
#pragma unroll
    for (int i = 0; i < 4; i++) y = __dadd_rn(y, trx_shfl_d(v, base + 4 * i));
    return __double2float_rn(y);
}

template <int GT, bool DOWN_LC>
__global__ void __launch_bounds__(256) trx_k_gateup(TrxLayer L, TrxShape S, TrxWork w) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int H = S.H, F = S.F;
    const int nrb = F / TRX_GU_ROWS;
    const int n_items = *w.n_active * nrb;
    int cur_t = -1;
    TrxQ4X X;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int e = w.active[item / nrb], rb = item % nrb;
        const int p0 = w.offsets[e], p1 = w.offsets[e + 1];
        const uint8_t *G = L.gate + (int64_t)e * L.gate_mb, *U = L.up + (int64_t)e * L.up_mb;
        for (int rr = warp; rr < TRX_GU_ROWS; rr += 8) {
            const int r = rb * TRX_GU_ROWS + rr;
            for (int p = p0; p < p1; p++) {
                const int t = w.xmap[p];
                float hv;
                if (GT == TRX_Q4_K) {
                    // H == 2048: one row per warp
                    if (t != cur_t) trx_q4x_load(w.xq + (int64_t)t * H + 256 * (lane >> 2), lane & 3, X);
                    cur_t = t;
                    const float g = trx_q4k_row8(G + (int64_t)r * (H / 256) * 144, X, w.xq_bf + (int64_t)t * (H / 32),
                                                 w.xq_sc + (int64_t)t * (H / 256), lane);
                    const float u = trx_q4k_row8(U + (int64_t)r * (H / 256) * 144, X, w.xq_bf + (int64_t)t * (H / 32),
                                                 w.xq_sc + (int64_t)t * (H / 256), lane);
                    hv = trx_silu_mul(g, u);
                } else {
                    // half 0: gate row r, half 1: up row r
                    const uint8_t *M = lane < 16 ? G : U;
                    const float v = trx_q8l_dot(M + (int64_t)r * (H / 256) * 272, w.x_lc + (int64_t)t * H, H / 256,
                                                lane & 15);
                    const float u = __shfl_sync(0xffffffffu, v, 16);
                    hv = trx_silu_mul(v, u);
                }
                if (lane == 0) w.h[(int64_t)p * F + (DOWN_LC ? trx_lc_pos(r) : r)] = hv;
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Q4_K down input: every h row prepared (one warp per (row, 256-block))
__global__ void __launch_bounds__(256) trx_k_prep(TrxShape S, const int *__restrict__ n_rows_dev, int R_max, TrxWork w) {
    const int F = S.F, nsb = F / 256;
    const int R = n_rows_dev ? *n_rows_dev : R_max;
    const int lane = threadIdx.x & 31;
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int p = gw / nsb, s = gw % nsb;
    if (p >= R) return;
    trx_prep_q4x_block(w.h + (int64_t)p * F + 256 * s, w.hq + (int64_t)p * F + 256 * s, w.hq_bf + (int64_t)p * (F / 32) + 8 * s,
                       w.hq_sc + (int64_t)p * (F / 256) + s, lane);
}

// ---------------------------------------------------------------------------------------------
// down + combine + residual

template <int DT>
__global__ void __launch_bounds__(256) trx_k_down(TrxLayer L, TrxShape S, TrxWork w, float *__restrict__ x_io, int T,
                                                  float *__restrict__ ffn_out) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int H = S.H, F = S.F, k = S.k;
    const int nrb = H / TRX_DN_ROWS;
    const int n_act = *w.n_active;
    const int n_items = n_act * nrb;
    __shared__ int s_last;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int e = w.active[item / nrb], rb = item % nrb;
        const int p0 = w.offsets[e], p1 = w.offsets[e + 1];
        const uint8_t *D = L.down + (int64_t)e * L.down_mb;
        // two output rows per warp (a half-warp each): d = rb * 64 + 16 j + 2 warp + half
        for (int p = p0; p < p1; p++) {
            if (DT == TRX_Q4_K) { // F == 1024: 4 blocks a row
                TrxQ4X X;
                trx_q4x_load(w.hq + (int64_t)p * F + 256 * ((lane >> 2) & 3), lane & 3, X);
#pragma unroll 1
                for (int j = 0; j < TRX_DN_ROWS / 16; j++) {
                    const int d = rb * TRX_DN_ROWS + 16 * j + 2 * warp + (lane >> 4);
                    const float v = trx_q4k_row4(D + (int64_t)d * (F / 256) * 144, X, w.hq_bf + (int64_t)p * (F / 32),
                                                 w.hq_sc + (int64_t)p * (F / 256), lane);
                    if ((lane & 15) == 0) w.h3[(int64_t)p * H + d] = v;
                }
            } else {
#pragma unroll 1
                for (int j = 0; j < TRX_DN_ROWS / 16; j++) {
                    const int d = rb * TRX_DN_ROWS + 16 * j + 2 * warp + (lane >> 4);
                    float v;
                    if (DT == TRX_Q8_0)
                        v = trx_q8l_dot(D + (int64_t)d * (F / 256) * 272, w.h + (int64_t)p * F, F / 256, lane & 15);
                    else
                        v = trx_q6l_dot(D + (int64_t)d * (F / 256) * 208,
                                        D + (int64_t)H * (F / 256) * 208 + (int64_t)d * (F / 256) * 2,
                                        w.h + (int64_t)p * F, F / 256, lane & 15);
                    if ((lane & 15) == 0) w.h3[(int64_t)p * H + d] = v;
                }
            }
        }
        // the last block to finish this block of output rows (over all active experts) combines it
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            s_last = atomicAdd(&w.comb_cnt[rb], 1u) == (unsigned)(n_act - 1);
        }
        __syncthreads();
        if (s_last) {
            __threadfence();
            for (int i = tid; i < T * TRX_DN_ROWS; i += blockDim.x) {
                const int t = i / TRX_DN_ROWS, d = rb * TRX_DN_ROWS + i % TRX_DN_ROWS;
                float out = 0.0f;
                for (int s = 0; s < k; s++) {
                    const int j = t * k + s;
                    out = __fadd_rn(out, __fmul_rn(w.sel_w[j], __ldcg(w.h3 + (int64_t)w.place[j] * H + d)));
                }
                if (ffn_out) ffn_out[(int64_t)t * H + d] = out;
                x_io[(int64_t)t * H + d] = __fadd_rn(x_io[(int64_t)t * H + d], out);
            }
            if (tid == 0) w.comb_cnt[rb] = 0u;
        }
        __syncthreads();
    }
}
