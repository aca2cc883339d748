// fused_layer.cuh: one MoE layer call for a short pass (decode, up to TRX_ROUTE_FUSED_MAX tokens) as ONE
// persistent kernel, launched cooperatively so that every CTA is resident and may wait for another.
//
//  phase A  CTAs 0..E-1 compute the router logits of one expert each (trx_router_block); CTAs E..E+T-1
//           prepare one token's input row each; the last of them to finish routes every token and sorts the
//           (token, slot) rows by expert, then publishes the routing (a release store of the call's epoch).
//  phase B  every CTA waits for the routing, takes its share of the routed gate/up rows and of the routed
//           down rows (trx_cta_range over each virtual row space) and arms 1-D TMA bulk copies for BOTH at
//           once: the down weights do not depend on the activations, so they stream from HBM while the
//           gate/up rows are multiplied.
//  gate/up  as trx_k_gateup; each finished chunk adds its rows to its expert's counter (release).
//  down     before a chunk of expert i: wait (acquire) until expert i's F gate/up rows are counted; Q4_K
//           prepares the expert's h rows in shared memory; then the dots into h3 and the id-ordered combine
//           by the last CTA to finish each 16-row block (as trx_k_down).
//  end      the last CTA resets the per-expert counters for the next call.
//
// Every wait is bounded (TRX_SPIN_NS); a CTA that gives up sets the error flag, waits (bounded) for its own
// copies in flight and leaves. The counters a kernel leaves non-zero after an error are reset by
// tr_gpu_moe_check.
#pragma once
#include <cstdint>
#include "bulk.cuh"
#include "moe_kernels.cuh"

#define TRX_SPIN_NS 1000000000ull
#define TRX_FU_SD 4 // down stages

struct TrxSync {
    uint32_t route_cnt;            // router and prep CTAs done in this call
    uint32_t routed;               // the epoch of the last call whose routing is published
    uint32_t finish;               // CTAs done in this call
    uint32_t pad;
    uint32_t gu_done[TRX_MAX_EXPERTS]; // gate/up rows done per active slot
};

__device__ __forceinline__ uint32_t trx_ld_acquire(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void trx_st_release(uint32_t *p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// thread-level bounded wait: *p == target (eq) or *p >= target
__device__ __forceinline__ bool trx_spin(const uint32_t *p, uint32_t target, bool eq) {
    uint64_t t0 = 0;
    for (int it = 0;; it++) {
        const uint32_t v = trx_ld_acquire(p);
        if (eq ? v == target : v >= target) return true;
        if (it == 0) t0 = trx_globaltimer();
        else if (trx_globaltimer() - t0 > TRX_SPIN_NS) return false;
        __nanosleep(32);
    }
}

template <int GT>
__host__ __device__ constexpr int trx_fu_sg() { return GT == TRX_Q4_K ? 4 : 3; }

// dynamic shared memory of the fused kernel (the router phase reuses the stage buffers)
__host__ __device__ inline size_t trx_fused_smem(int gate_type, int down_type, int H, int F, int T) {
    const int rbg = gate_type == TRX_Q4_K ? H / 256 * 144 : H / 32 * 34;
    const int rbd = down_type == TRX_Q4_K ? F / 256 * 144 : down_type == TRX_Q6_K ? F / 256 * 208 : F / 32 * 34;
    const int sg = gate_type == TRX_Q4_K ? 4 : 3;
    size_t stages = (size_t)sg * 2 * TRX_GU_CHUNK * rbg + (size_t)TRX_FU_SD * TRX_DN_CHUNK * rbd;
    const size_t router = (size_t)(1 + (T < TRX_TOK_STAGE ? T : TRX_TOK_STAGE)) * H * 4;
    if (router > stages) stages = router;
    const size_t prep = down_type == TRX_Q4_K ? (size_t)F * 4 + (size_t)(F / 32 + F / 256) * 8 : 0;
    return (stages + 8 * (sg + TRX_FU_SD) + 127) / 128 * 128 + prep;
}

template <int GT, int DT>
__global__ void __launch_bounds__(256, 1) trx_k_layer(TrxLayer L, TrxShape S, const float *__restrict__ normed, int T,
                                                      TrxWork w, TrxSync *sync, float *__restrict__ x_io,
                                                      float *__restrict__ ffn_out, uint32_t epoch) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float res[2][TRX_TOK_GROUP][TRX_GU_CHUNK];
    __shared__ int s_active[TRX_MAX_EXPERTS], s_off[TRX_MAX_EXPERTS + 1], s_nact, s_flag;
    __shared__ float sp[8][96];
    constexpr int CHG = TRX_GU_CHUNK, CHD = TRX_DN_CHUNK, SG = trx_fu_sg<GT>(), SD = TRX_FU_SD;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, hw = tid >> 4;
    const int E = S.E, H = S.H, F = S.F, k = S.k, nsb_d = F / 256;
    const int rbg = GT == TRX_Q4_K ? H / 256 * 144 : H / 32 * 34;
    const int rbd = DT == TRX_Q4_K ? nsb_d * 144 : DT == TRX_Q6_K ? nsb_d * 208 : F / 32 * 34;
    const int gu_half = CHG * rbg, gu_stage = 2 * gu_half, dn_stage = CHD * rbd;
    uint8_t *gu_buf = smem, *dn_buf = smem + SG * gu_stage;
    size_t stage_bytes = (size_t)SG * gu_stage + (size_t)SD * dn_stage;
    const size_t router_bytes = (size_t)(1 + min(T, TRX_TOK_STAGE)) * H * 4;
    if (router_bytes > stage_bytes) stage_bytes = router_bytes;
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + stage_bytes); // SG gate/up, then SD down
    // Q4_K down: one prepared h row, 128-byte aligned (its planes are read 16 bytes at a time)
    uint32_t *s_planes = reinterpret_cast<uint32_t *>(smem + ((stage_bytes + 8 * (SG + SD) + 127) / 128) * 128);
    double *s_bf = reinterpret_cast<double *>(s_planes + F), *s_sc = s_bf + F / 32;

    // ---------------- phase A: router logits, token preparation, routing
    if ((int)blockIdx.x < E + T) {
        if ((int)blockIdx.x < E) trx_router_block(L, S, normed, blockIdx.x, 0, T, w, reinterpret_cast<float *>(smem));
        else trx_prep_token(L, S, normed, blockIdx.x - E, w);
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            s_flag = atomicAdd(&sync->route_cnt, 1u) == (uint32_t)(E + T - 1);
        }
        __syncthreads();
        if (s_flag) {
            __threadfence();
            for (int t = warp; t < T; t += 8)
                trx_route_token(w.logits + (int64_t)t * E, E, k, S.norm_topk, lane, sp[warp], w.sel_id + (int64_t)t * k,
                                w.sel_w + (int64_t)t * k);
            __syncthreads();
            const int R = T * k;
            if (w.out_sel_id)
                for (int j = tid; j < R; j += blockDim.x) {
                    w.out_sel_id[j] = w.sel_id[j];
                    w.out_sel_w[j] = w.sel_w[j];
                }
            trx_block_counting_sort<8>(w.sel_id, R, E, k, w);
            __syncthreads();
            if (tid == 0) {
                sync->route_cnt = 0u;
                __threadfence();
                trx_st_release(&sync->routed, epoch);
            }
        }
    }

    // ---------------- phase B: the routing, this CTA's rows, every copy armed
    if (tid == 0) s_flag = trx_spin(&sync->routed, epoch, true);
    __syncthreads();
    if (!s_flag) {
        if (tid == 0) atomicExch(w.err, 2);
        return;
    }
    if (tid == 0) s_nact = __ldcg(w.n_active);
    if (tid <= E) s_off[tid] = __ldcg(w.offsets + tid);
    if (tid < E) s_active[tid] = __ldcg(w.active + tid);
    __syncthreads();
    const int n_act = s_nact;
    int64_t ag, bg, ad, bd;
    trx_cta_range((int64_t)n_act * F, ag, bg);
    trx_cta_range((int64_t)n_act * H, ad, bd);
    if (tid == 0) {
        for (int s = 0; s < SG + SD; s++) trx_mbar_init(&bar[s], 1);
        trx_fence_barrier_init();
    }
    __syncthreads();
    auto gu_end = [&](int64_t v) { return min(min(v + CHG, bg), (v / F + 1) * F); };
    auto dn_end = [&](int64_t v) { return min(bd, (v / CHD + 1) * CHD); };
    int64_t gu_iv = ag, dn_iv = ad;
    int gu_issued = 0, dn_issued = 0;
    auto issue_gu = [&]() {
        const int64_t ve = gu_end(gu_iv);
        const int e = s_active[gu_iv / F], r0 = (int)(gu_iv % F), n = (int)(ve - gu_iv);
        const int s = gu_issued % SG;
        uint8_t *dst = gu_buf + s * gu_stage;
        trx_mbar_expect_tx(&bar[s], 2u * n * rbg);
        trx_bulk_g2s(dst, L.gate + e * L.gate_mb + (int64_t)r0 * rbg, n * rbg, &bar[s]);
        trx_bulk_g2s(dst + gu_half, L.up + e * L.up_mb + (int64_t)r0 * rbg, n * rbg, &bar[s]);
        gu_iv = ve;
        gu_issued++;
    };
    auto issue_dn = [&]() {
        const int64_t ve = dn_end(dn_iv);
        const int e = s_active[dn_iv / H], d0 = (int)(dn_iv % H), n = (int)(ve - dn_iv);
        const int s = dn_issued % SD;
        trx_mbar_expect_tx(&bar[SG + s], (uint32_t)(n * rbd));
        trx_bulk_g2s(dn_buf + s * dn_stage, L.down + e * L.down_mb + (int64_t)d0 * rbd, n * rbd, &bar[SG + s]);
        dn_iv = ve;
        dn_issued++;
    };
    if (tid == 0) {
        for (int q = 0; q < SG && gu_iv < bg; q++) issue_gu();
        for (int q = 0; q < SD && dn_iv < bd; q++) issue_dn();
    }
    bool failed = false;

    // ---------------- gate / up / SwiGLU
    int cur_t = -1;
    TrxQ4X X;
    int j = 0;
    for (int64_t v = ag; v < bg && !failed; j++) {
        const int64_t ve = gu_end(v);
        const int slot = (int)(v / F), e = s_active[slot], r0 = (int)(v % F), n = (int)(ve - v);
        const int p0 = s_off[e], p1 = s_off[e + 1];
        const int s = j % SG;
        if (GT == TRX_Q4_K && warp < n) {
            const int t0 = __ldcg(w.xmap + p0);
            if (t0 != cur_t) {
                cur_t = t0;
                trx_q4x_load<true>(w.xq + (int64_t)t0 * H + 256 * (lane >> 2), lane & 3, X);
            }
        }
        const bool ok = trx_mbar_wait(&bar[s], (j / SG) & 1, TRX_WAIT_NS);
        if (__syncthreads_or(!ok)) {
            failed = true;
            break;
        }
        const uint8_t *gs = gu_buf + s * gu_stage, *us = gs + gu_half;
        for (int pg = p0; pg < p1; pg += TRX_TOK_GROUP) {
            const int ng = min(TRX_TOK_GROUP, p1 - pg);
            for (int q = 0; q < ng; q++) {
                const int t = __ldcg(w.xmap + pg + q);
                if (GT == TRX_Q4_K) {
                    if (warp < n) {
                        if (t != cur_t) {
                            cur_t = t;
                            trx_q4x_load<true>(w.xq + (int64_t)t * H + 256 * (lane >> 2), lane & 3, X);
                        }
                        const double *bf = w.xq_bf + (int64_t)t * (H / 32), *sc = w.xq_sc + (int64_t)t * (H / 256);
                        const float g = trx_q4k_row8<true, true>(gs + warp * rbg, X, bf, sc, lane);
                        const float u = trx_q4k_row8<true, true>(us + warp * rbg, X, bf, sc, lane);
                        if (lane == 0) {
                            res[0][q][warp] = g;
                            res[1][q][warp] = u;
                        }
                    }
                } else {
                    const int row = hw & 7, mat = hw >> 3;
                    const float vv = trx_q8l_dot<true, true>((mat ? us : gs) + (row < n ? row : 0) * rbg,
                                                             w.x_lc + (int64_t)t * H, H / 256, lane & 15);
                    if (row < n && (lane & 15) == 0) res[mat][q][row] = vv;
                }
            }
            __syncthreads();
            for (int i = tid; i < ng * n; i += blockDim.x) {
                const int q = i / n, row = i % n, r = r0 + row;
                w.h[(int64_t)(pg + q) * F + (DT != TRX_Q4_K ? trx_lc_pos(r) : r)] =
                    trx_silu_mul(res[0][q][row], res[1][q][row]);
            }
            __syncthreads();
        }
        if (tid == 0) {
            __threadfence(); // this chunk's h rows before its count
            atomicAdd(&sync->gu_done[slot], (uint32_t)n);
            if (gu_iv < bg) { // stage s is free again
                trx_fence_proxy_async();
                issue_gu();
            }
        }
        v = ve;
    }

    // ---------------- down + combine + residual
    int prepped_p = -1;
    j = 0;
    for (int64_t v = ad; v < bd && !failed; j++) {
        const int64_t ve = dn_end(v);
        const int slot = (int)(v / H), e = s_active[slot], d0 = (int)(v % H), n = (int)(ve - v);
        const int p0 = s_off[e], p1 = s_off[e + 1];
        const int s = j % SD;
        if (tid == 0) s_flag = trx_spin(&sync->gu_done[slot], (uint32_t)F, false);
        __syncthreads();
        if (!s_flag) {
            failed = true;
            break;
        }
        const bool ok = trx_mbar_wait(&bar[SG + s], (j / SD) & 1, TRX_WAIT_NS);
        if (__syncthreads_or(!ok)) {
            failed = true;
            break;
        }
        const uint8_t *st = dn_buf + s * dn_stage;
        const int row = hw < n ? hw : 0, d = d0 + row;
        for (int p = p0; p < p1; p++) {
            float vv;
            if (DT == TRX_Q4_K) {
                if (p != prepped_p) { // the h row prepared in shared memory (one warp per 256-block)
                    __syncthreads();
                    if (warp < nsb_d)
                        trx_prep_q4x_block<true>(w.h + (int64_t)p * F + 256 * warp, s_planes + 256 * warp, s_bf + 8 * warp,
                                                 s_sc + warp, lane);
                    __syncthreads();
                    prepped_p = p;
                }
                trx_q4x_load(s_planes + 256 * ((lane >> 2) & 3), lane & 3, X);
                vv = trx_q4k_row4<true>(st + row * rbd, X, s_bf, s_sc, lane);
            } else if (DT == TRX_Q8_0) {
                vv = trx_q8l_dot<true, true>(st + row * rbd, w.h + (int64_t)p * F, nsb_d, lane & 15);
            } else {
                const uint8_t *dptr = L.down + e * L.down_mb + (int64_t)H * rbd + (int64_t)d * nsb_d * 2;
                vv = trx_q6l_dot<true, true>(st + row * rbd, dptr, w.h + (int64_t)p * F, nsb_d, lane & 15);
            }
            if (hw < n && (lane & 15) == 0) w.h3[(int64_t)p * H + d] = vv;
        }
        __syncthreads();
        const int blk = d0 / CHD;
        if (tid == 0) {
            __threadfence();
            const uint32_t old = atomicAdd(&w.comb_cnt[blk], (uint32_t)n);
            s_flag = old + (uint32_t)n == (uint32_t)(n_act * CHD);
            if (dn_iv < bd) {
                trx_fence_proxy_async();
                issue_dn();
            }
        }
        __syncthreads();
        if (s_flag) {
            __threadfence();
            for (int i = tid; i < T * CHD; i += blockDim.x) {
                const int t = i / CHD, dd = blk * CHD + i % CHD;
                float out = 0.0f;
                for (int sl = 0; sl < k; sl++) {
                    const int jj = t * k + sl;
                    out = __fadd_rn(out, __fmul_rn(__ldcg(w.sel_w + jj), __ldcg(w.h3 + (int64_t)__ldcg(w.place + jj) * H + dd)));
                }
                if (ffn_out) ffn_out[(int64_t)t * H + dd] = out;
                x_io[(int64_t)t * H + dd] = __fadd_rn(x_io[(int64_t)t * H + dd], out);
            }
            if (tid == 0) w.comb_cnt[blk] = 0u;
        }
        v = ve;
    }

    // ---------------- end
    if (failed) {
        if (tid == 0) {
            atomicExch(w.err, 3);
            // every copy still in flight lands before the CTA's shared memory goes away
            for (int q = 0; q < gu_issued; q++) trx_mbar_wait(&bar[q % SG], (q / SG) & 1, TRX_WAIT_NS);
            for (int q = 0; q < dn_issued; q++) trx_mbar_wait(&bar[SG + q % SD], (q / SD) & 1, TRX_WAIT_NS);
        }
        __syncthreads();
        return;
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(&sync->finish, 1u) == gridDim.x - 1) { // every CTA is past its waits
            for (int i = 0; i < E; i++) sync->gu_done[i] = 0u;
            sync->finish = 0u;
            __threadfence();
        }
    }
}
