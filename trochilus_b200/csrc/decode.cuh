// decode.cuh: a one-token MoE layer call, the decode road's common case, as one compact persistent kernel.
//
// The same results as the general fused kernel (fused_layer.cuh), the same routing code, laid out for one token so
// that its code stays small and no warp waits on another warp's stages; its Q4_K rows run on the integer tensor
// cores (exact integer sums, so the bits are the same).
//
// Exchange between CTAs without fences or counters: every word one CTA publishes for the others (a logit, an h
// value) is a 64-bit store of the value and the call's tag (TrxSync::seq + 1) together, which a reader sees whole or
// not at all; a reader polls until the words it needs carry this call's tag. CTA 0 advances seq as it ends: it can
// end only after it holds h values from every CTA, each stored with a tag derived from that CTA's read of seq, so
// every CTA has read seq by then. (A device-scope fence after a store measured about 1200 cycles on the B200, and a
// fence and a counter at the end of every CTA about 1.3 us a call.) A logit is pushed to every CTA's own row of E
// words, so that each CTA polls lines no other CTA polls: 148 CTAs polling the same 64 words took 3.3 us.
//
// Launched with programmatic dependent launch: the barriers, the expf table and the router row (static weights) are
// set up before trx_griddep_wait, under the previous kernel's tail.
//
//  prologue  a helper warp initialises the barriers; in CTAs 0..E-1 warp 0 loads router row e into registers at
//            once, warps 0-3 stage the token's row in shared memory meanwhile (or, with the ffn_norm in the hook,
//            every CTA normalises the residual row there first), warp 0 forms logit e (the 16-lane contract) and
//            publishes it tagged; warps 4-11 prepare the row for the gate/up dots (all CTAs): Q4_K's integer
//            definition as the tensor cores take it (trx_prep_q4m_block), or Q8_0's inputs in LC order.
//  routing   every CTA, once it holds all E tagged logits, routes the token (softmax, top-k, ids sorted) in shared
//            memory; CTA 0's warp 14 forms the dispatch permutation when the caller asks for it.
//  experts   a CTA owns rows [ga, gb) of every selected expert's gate and up matrices and rows [da, db) of every
//            selected expert's down matrix. Each of 14 consumer warps streams its own units through a ring of
//            shared-memory slots (TMA, no multicast), one mbarrier a slot, so it waits only for its own bytes.
//            Q4_K gate/up: five units a warp, each one 256-block of the CTA's 8 gate rows and the same 8 up rows
//            (two 3-D tile loads), multiplied on the integer tensor cores (trx_q4k_blk_mma); warp 14 adds an
//            expert's block values per row once its units are in and publishes h = silu(g) u tagged. Q8_0
//            gate/up: four units a warp (a gate row and its up row by 1-D bulk copies, the 16-lane contract), whose
//            (g, u) warp 14 turns into h a whole step at once. Then the down: two steps a warp (a half-warp the same
//            row of two experts, trx_q6l_dot_pair_il or trx_q8l_dot_pair_il), or for a Q4_K down three units a warp
//            (a 256-block of the CTA's 16 down rows of one expert, the expert's h block prepared in place, the same
//            tensor-core product). The down weights do not depend on h, so they load while the gate/up rows are
//            multiplied; the h rows come from the helper warp, which gathers expert i's tagged h values into shared
//            memory, experts in order (Q6_K, Q8_0: the rows of experts 2q and 2q + 1 interleaved, the pairs a down
//            step multiplies together).
//  mix       each CTA adds, for its rows [da, db), the k expert outputs in increasing expert id and the sum to the
//            residual (Trochilus's mix_body); CTA 0 advances seq (the host-pointer road: the last CTA, which also
//            posts the host word).
//
// Limits (checked on the host, trx_dec1_takes): one token, no external routing, 2048 columns of gate/up and 256,
// 512 or 1024 of down, Q4_K gate/up with a Q6_K or Q4_K down, or Q8_0 throughout, k even and at most 8, and a grid
// whose shares fit the ring (for Q4_K at most 8 gate/up rows and 16 down rows of an expert a CTA). Every wait is
// bounded; a warp that gives up sets the error flag, waits (bounded) for its own copies in flight and leaves.
//
// Trochilus references: forward_layer's MoE block src/models/olmoe.c:1845-1933 (route_token :1455-1502, the
// counting sort :1850-1861, expert_stages :1642-1689, mix_body :1432-1446); tr_rmsnorm src/kernels/kernels.c:1351-1360.
#pragma once
#include <cstdint>
#include <cuda.h>
#include "fused_layer.cuh"

#define TRX_DC_CWARPS 14  // consumer warps
#define TRX_DC_SILU 14    // the warp that forms h = silu(g) u for the consumers' gate/up units
#define TRX_DC_HELPER 15  // the helper warp (barriers, h gathering)
#define TRX_DC_THREADS 512
#define TRX_DC_NS 3       // slots a consumer warp has in flight (Q4_K_M; Q8_0 weights take 2 larger ones)
#define TRX_DC_SLOT 3456  // Q4_K_M bytes a slot: a gate/up unit (2 x 1152) or a down step (2 x (2 x 832 + 2 x 16))
#define TRX_DC_NS8 2      // Q8_0: slots a consumer warp has in flight
#define TRX_DC_SLOT8 4352 // Q8_0 bytes a slot: a gate/up unit (2 x 2176) or a down step of up to 1024 columns
#define TRX_DC_GU 4       // gate/up units a warp (Q8_0: a gate row and its up row each)
#define TRX_DC_GU4 5      // Q4_K: gate/up units a warp (a 256-block of 8 gate rows and 8 up rows each, on the tensor cores)
#define TRX_DC_DN 2       // down steps a warp (Q6_K, Q8_0: two row pairs each)
#define TRX_DC_DN4 3      // Q4_K down: down units a warp (a 256-block of the CTA's 16 rows of one expert each)
#define TRX_DC_KMAX 8
#define TRX_DC_GRID_MAX 256 // CTAs (the tagged logits: a row of E words for each)
#define TRX_DC_SEQ_MAX 64   // calls of up to this many tokens run one launch a token (faster than the fused kernel)

struct TrxDecPlan {
    uint32_t off_h, off_xq, total; // shared memory: h rows (k x F floats), the prepared token row, the whole
    uint32_t off_v;                // Q4_K: the gate/up units' block values (k x H / 256 x 16 doubles)
    uint32_t off_d;                // Q4_K down: the down units' block values (k x F / 256 x 16 doubles), then the h
                                   // rows' sub-block sums (k x F / 32) and scales (k x F / 256)
    uint32_t slot;                 // bytes a slot
    int ns;                        // slots a consumer warp has in flight
    int ng_max, nd_max;            // the most gate/up and down rows of an expert a CTA takes
};

__host__ __device__ inline uint32_t trx_dc_align(uint32_t v) { return (v + 127u) / 128u * 128u; }

// gate_type Q4_K (with a Q6_K or Q4_K down) or Q8_0 (with a Q8_0 down)
__host__ inline TrxDecPlan trx_dec_plan(int gate_type, int down_type, int H, int F, int k, int grid) {
    TrxDecPlan P{};
    const bool q8 = gate_type == TRX_Q8_0;
    // Q8_0: a gate/up unit is 2 rows of H / 256 272-byte blocks, a down step 2 x 2 rows of F / 256 (no larger for F <= H)
    P.slot = q8 ? TRX_DC_SLOT8 : TRX_DC_SLOT; // (H = 2048)
    P.ns = q8 ? TRX_DC_NS8 : TRX_DC_NS;
    P.off_h = trx_dc_align(TRX_DC_CWARPS * P.ns * P.slot);
    P.off_xq = trx_dc_align(P.off_h + (uint32_t)(k * F * 4 > H * 4 ? k * F * 4 : H * 4));
    // the token's row: Q4_K's digits, sums and scales (trx_prep_q4m_block); Q8_0's inputs in LC order
    P.off_v = trx_dc_align(P.off_xq + (uint32_t)(q8 ? H * 4 : H * 4 + (H / 32) * 8 + (H / 256) * 8));
    P.off_d = q8 ? P.off_v : trx_dc_align(P.off_v + (uint32_t)(k * (H / 256) * 16 * 8));
    P.total = down_type != TRX_Q4_K ? P.off_d
                                    : trx_dc_align(P.off_d + (uint32_t)(k * (F / 256) * 16 * 8 + k * (F / 32) * 8 +
                                                                        k * (F / 256) * 8));
    P.ng_max = (F + grid - 1) / grid;
    P.nd_max = ((H / 2 + grid - 1) / grid) * 2;
    return P;
}

// whether a call takes trx_k_dec1 (the host's part of the limits above)
__host__ inline bool trx_dec1_takes(int gate_type, int down_type, int router_type, int H, int F, int E, int k, int T,
                                    int grid, bool ext) {
    if (T != 1 || ext) return false;
    if (!(gate_type == TRX_Q4_K && (down_type == TRX_Q6_K || down_type == TRX_Q4_K)) &&
        !(gate_type == TRX_Q8_0 && down_type == TRX_Q8_0))
        return false;
    if (router_type != TRX_F32 && router_type != TRX_BF16) return false;
    // (1, 2 or 4 blocks a down row: a row's d values never straddle a 16-byte piece)
    if (H != 2048 || (F != 256 && F != 512 && F != 1024) || E > TRX_MAX_EXPERTS || k < 2 || k % 2 || k > TRX_DC_KMAX)
        return false;
    const TrxDecPlan P = trx_dec_plan(gate_type, down_type, H, F, k, grid);
    // (Q8_0: a unit a gate/up row pair; Q4_K: a unit a 256-block of the CTA's rows, at most 8 of them)
    const bool gu_fits = gate_type == TRX_Q8_0 ? k * P.ng_max <= TRX_DC_CWARPS * TRX_DC_GU
                                               : P.ng_max <= 8 && k * (H / 256) <= TRX_DC_CWARPS * TRX_DC_GU4;
    // (Q4_K down: a unit a 256-block of the CTA's rows of one expert, at most 16 of them; else two row pairs)
    const bool dn_fits = down_type == TRX_Q4_K ? k * (F / 256) <= TRX_DC_CWARPS * TRX_DC_DN4
                                               : (k / 2) * P.nd_max <= 2 * TRX_DC_CWARPS * TRX_DC_DN;
    return P.total <= 206 * 1024 && gu_fits && dn_fits && P.nd_max <= 16 && P.ng_max <= 32 &&
           grid <= TRX_DC_GRID_MAX && F >= grid;
}

// a value and its tag in one 64-bit word (relaxed, device scope; an aligned 64-bit access is never torn)
__device__ __forceinline__ void trx_st_tagged(unsigned long long *p, uint32_t tag, float v) {
    const unsigned long long x = ((unsigned long long)tag << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(x) : "memory");
}
__device__ __forceinline__ unsigned long long trx_ld_tagged(const unsigned long long *p) {
    unsigned long long x;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(x) : "l"(p) : "memory");
    return x;
}
__device__ __forceinline__ ulonglong2 trx_ld_tagged2(const unsigned long long *p) {
    ulonglong2 x;
    asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(x.x), "=l"(x.y) : "l"(p) : "memory");
    return x;
}

// map_gate, map_up (Q4_K): 3-D tensor maps over the layer's gate and up matrices (row bytes, rows, experts), boxes of
// one 256-block of 8 rows (trx_dec1_map); map_down (Q4_K down): the same over the down matrices, boxes of 16 rows;
// unused otherwise
template <int RT, int GT, int DT>
__global__ void __launch_bounds__(TRX_DC_THREADS, 1)
    trx_k_dec1(TrxLayer L, TrxShape S, const float *__restrict__ normed, TrxWork w, TrxSync *sync,
               float *__restrict__ x_io, float *__restrict__ ffn_out, uint32_t epoch, const TrxDecPlan P,
               const __grid_constant__ CUtensorMap map_gate, const __grid_constant__ CUtensorMap map_up,
               const __grid_constant__ CUtensorMap map_down) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr bool Q8 = GT == TRX_Q8_0, DQ4 = DT == TRX_Q4_K;
    constexpr int GU = Q8 ? TRX_DC_GU : TRX_DC_GU4; // gate/up steps a warp
    constexpr int DN = DQ4 ? TRX_DC_DN4 : TRX_DC_DN; // down steps a warp
    __shared__ __align__(8) uint64_t s_full[TRX_DC_CWARPS][TRX_DC_NS];
    __shared__ __align__(8) uint64_t s_hbar[TRX_DC_KMAX];
    __shared__ __align__(8) uint64_t s_gubar[TRX_DC_KMAX]; // Q8_0: step j's gate/up values are in s_gu; Q4_K:
                                                            // expert i's block values are in the v rows
    __shared__ __align__(8) float2 s_gu[TRX_DC_GU * TRX_DC_CWARPS]; // unit u's (gate, up) row values
    __shared__ __align__(16) float sp[96];
    __shared__ __align__(16) float s_q6sc[2 * TRX_DC_CWARPS][32 * TRX_Q6L_SS_BLOCKS];
    __shared__ __align__(16) float s_h3[TRX_DC_KMAX][16];
    __shared__ float s_logit[TRX_MAX_EXPERTS], s_selw[TRX_DC_KMAX], s_inv;
    __shared__ int32_t s_selid[TRX_DC_KMAX], s_off[TRX_MAX_EXPERTS + 1], s_act[TRX_MAX_EXPERTS], s_nact;
    __shared__ int32_t s_place[TRX_DC_KMAX], s_xmap[TRX_DC_KMAX];
    __shared__ int s_flag;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int E = S.E, H = S.H, F = S.F, k = S.k, nsb = F / 256, G = gridDim.x, c = blockIdx.x, NB = H / 256;
    TRX_TRACE(0);
    trx_griddep_launch();
    if (!Q8 && (trx_smem(smem) & 127u) != 0u) { // (the tensor copies need 128-byte aligned slots: report, touch nothing)
        if (threadIdx.x == 0) {
            atomicExch(w.err, 16);
            if (w.host_done) trx_post_done(w.host_done, epoch | 0x80000000u);
        }
        return;
    }
    float *hbuf = reinterpret_cast<float *>(smem + P.off_h); // h rows; before the routing, the token's row
    uint32_t *xq = reinterpret_cast<uint32_t *>(smem + P.off_xq);
    double *xbf = reinterpret_cast<double *>(smem + P.off_xq + H * 4), *xsc = xbf + H / 32;
    // this CTA's rows: [ga, ga + ng) of every gate/up matrix, [da, da + nd) of every down matrix (whole row pairs)
    const int ga = F * c / G, ng = F * (c + 1) / G - ga;
    const int da = (H / 2) * c / G * 2, nd = (H / 2) * (c + 1) / G * 2 - da;
    if (warp == TRX_DC_HELPER && lane == 0) {
        for (int i = 0; i < TRX_DC_CWARPS * TRX_DC_NS; i++) trx_mbar_init(&s_full[0][0] + i, 1);
        for (int i = 0; i < k; i++) trx_mbar_init(&s_hbar[i], 32); // every helper lane arrives
        if (Q8) {
            for (int j = 0; j < TRX_DC_GU; j++) { // a consumer with a unit in step j arrives
                const int n = k * ng - TRX_DC_CWARPS * j;
                trx_mbar_init(&s_gubar[j], (uint32_t)(n < 0 ? 0 : n > TRX_DC_CWARPS ? TRX_DC_CWARPS : n) + (n <= 0));
            }
        } else {
            for (int i = 0; i < k; i++) trx_mbar_init(&s_gubar[i], (uint32_t)(32 * NB)); // every lane of its units
        }
        trx_fence_barrier_init();
    }
    if (warp == 1) trx_expf_prefetch(lane);

    // ---------------- prologue
    const bool router = c < E;
    constexpr int EB = RT == TRX_BF16 ? 2 : 4;
    constexpr int GB = RT == TRX_BF16 ? 8 : 4; // router blocks a group: 16 loads of 16 bytes a lane in flight
    uint4 rr[16];
    const uint8_t *rrow = L.router + (int64_t)c * H * EB;
    const int l16 = lane & 15;
    if (router && warp == 0) { // the row's first group straight into registers, in flight while the input is staged
#pragma unroll
        for (int j = 0; j < 16; j++)
            rr[j] = __ldg(reinterpret_cast<const uint4 *>(rrow + ((size_t)256 * (j / (16 / GB)) + 16 * l16) * EB) + j % (16 / GB));
    }
    trx_griddep_wait(); // what the previous kernels wrote (the input row, x, seq) from here on
    const uint32_t tag = __ldcg(&sync->seq) + 1u; // this call's tag (never 0: a cleared word never matches)
    // residual values of this CTA's output rows, read now (from host memory on the host-pointer road)
    float xres = 0.0f;
    if (tid < nd) xres = x_io[da + tid];
    const float *xrow = normed; // the token's (normalised) row for the preparation: global, or hbuf
    if (S.norm_in) {
        // the ffn_norm: the residual row into hbuf, the 16-lane sum of squares, inv = 1 / sqrtf(sumsq / H + eps),
        // then normed = (x inv) w (Trochilus's tr_rmsnorm)
        for (int i = tid; i < H / 4; i += TRX_DC_THREADS)
            *reinterpret_cast<float4 *>(hbuf + 4 * i) = __ldcg(reinterpret_cast<const float4 *>(normed) + i);
        __syncthreads();
        if (warp == 0) {
            float acc = 0.0f;
            if (lane < 16)
                for (int kk = lane; kk < H; kk += 16) acc = __fadd_rn(acc, __fmul_rn(hbuf[kk], hbuf[kk]));
            acc = trx_lane_tree16(acc);
            if (lane == 0) s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, (float)H), L.norm_eps)));
        }
        __syncthreads();
        const float inv = s_inv;
        for (int i = tid; i < H; i += TRX_DC_THREADS) hbuf[i] = __fmul_rn(__fmul_rn(hbuf[i], inv), __ldg(L.norm_w + i));
        __syncthreads();
        if (c == 0 && w.out_normed)
            for (int i = tid; i < H; i += TRX_DC_THREADS) w.out_normed[i] = hbuf[i];
        xrow = hbuf;
    } else if (router && warp < 4) {
        for (int i = tid; i < H / 4; i += 128)
            *reinterpret_cast<float4 *>(hbuf + 4 * i) = __ldg(reinterpret_cast<const float4 *>(normed) + i);
        asm volatile("bar.sync 1, 128;" ::: "memory");
    }
    if (router && warp == 0) {
        // logit c: lane l adds fl(w x) for k = l + 16 m in increasing k from +0, then the tree (src/kernels/kernels.c:
        // 73-75, 101-109); both half-warps run the same row (the tree needs the whole warp)
        float acc = 0.0f;
        for (int i0 = 0; i0 < H / 256; i0 += GB) {
            if (i0 > 0) {
#pragma unroll
                for (int j = 0; j < 16; j++)
                    rr[j] = __ldg(reinterpret_cast<const uint4 *>(rrow + ((size_t)256 * (i0 + j / (16 / GB)) + 16 * l16) * EB) +
                                  j % (16 / GB));
            }
#pragma unroll
            for (int g = 0; g < GB; g++) {
                float wv[16];
#pragma unroll
                for (int q = 0; q < 16 / GB; q++) {
                    const uint4 v = rr[g * (16 / GB) + q];
                    const uint32_t ws[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int cc = 0; cc < 4; cc++) {
                        if (RT == TRX_BF16) {
                            wv[8 * q + 2 * cc] = __uint_as_float(ws[cc] << 16);
                            wv[8 * q + 2 * cc + 1] = __uint_as_float(ws[cc] & 0xffff0000u);
                        } else {
                            wv[4 * q + cc] = __uint_as_float(ws[cc]);
                        }
                    }
                }
                const float *xb = hbuf + 256 * (i0 + g) + l16; // (staged, or normalised, in hbuf)
#pragma unroll
                for (int m = 0; m < 16; m++) acc = __fadd_rn(acc, __fmul_rn(wv[m], xb[16 * m]));
            }
        }
        acc = trx_lane_tree16(acc); // (in every lane: both half-warps ran the row)
        const float v = L.router_bias ? __fadd_rn(acc, L.router_bias[c]) : acc;
        for (int j = lane; j < G; j += 32) trx_st_tagged(w.tag_logits + (int64_t)j * E + c, tag, v); // every CTA's row
        if (lane == 0 && w.out_logits) w.out_logits[c] = v;
        TRX_TRACE(62);
    }
    constexpr int NS = Q8 ? TRX_DC_NS8 : TRX_DC_NS;           // (the plan's ns and slot, as constants)
    constexpr uint32_t SLOT = Q8 ? TRX_DC_SLOT8 : TRX_DC_SLOT;
    float *xlc = reinterpret_cast<float *>(xq); // (Q8_0: the token's row in LC order)
    uint8_t *xdig = reinterpret_cast<uint8_t *>(xq); // (Q4_K: the token's digits, 1024 bytes a 256-block)
    double *sv = reinterpret_cast<double *>(smem + P.off_v); // (Q4_K: unit (i, b)'s 16 row values at 16 (i NB + b))
    // (Q4_K down: unit (i, b)'s 16 row values at 16 (i nsb + b), then the h blocks' sub-block sums and scales)
    double *dv = reinterpret_cast<double *>(smem + P.off_d), *dbf = dv + 16 * k * nsb, *dsc = dbf + 8 * k * nsb;
    // the token's row prepared for the gate/up dots, warp 4 + s taking 256-block s: Q4_K's integer definition as
    // the tensor cores take it, or Q8_0's inputs in LC order
    if (warp >= 4 && warp < 4 + H / 256) {
        const int sb = warp - 4;
        if (Q8) {
            for (int i = lane; i < 256; i += 32) xlc[256 * sb + trx_lc_pos(i)] = xrow[256 * sb + i];
        } else {
            trx_prep_q4m_block(xrow + 256 * sb, xdig + 1024 * sb, xbf + 8 * sb, xsc + sb, lane);
        }
    }

    // ---------------- routing: once it holds every tagged logit, every CTA routes the token itself
    if (warp == 0) {
        bool got0 = lane >= E, got1 = lane + 32 >= E, ok = true;
        uint64_t t0 = 0;
        for (;;) {
            if (!got0) {
                const unsigned long long x = trx_ld_tagged(w.tag_logits + (int64_t)c * E + lane);
                if ((uint32_t)(x >> 32) == tag) {
                    s_logit[lane] = __uint_as_float((uint32_t)x);
                    got0 = true;
                }
            }
            if (!got1) {
                const unsigned long long x = trx_ld_tagged(w.tag_logits + (int64_t)c * E + lane + 32);
                if ((uint32_t)(x >> 32) == tag) {
                    s_logit[lane + 32] = __uint_as_float((uint32_t)x);
                    got1 = true;
                }
            }
            if (__all_sync(0xffffffffu, got0 && got1)) break;
            const uint64_t now = trx_globaltimer();
            if (t0 == 0) t0 = now;
            else if (now - t0 > TRX_SPIN_NS) {
                ok = false;
                break;
            }
            __nanosleep(20);
        }
        const bool all_ok = __all_sync(0xffffffffu, ok);
        if (lane == 0) s_flag = all_ok ? 1 : 0;
    }
    __syncthreads();
    if (!s_flag) {
        if (tid == 0) {
            atomicExch(w.err, 2);
            if (w.host_done) trx_post_done(w.host_done, epoch | 0x80000000u);
        }
        return;
    }
    TRX_TRACE(1);
    if (warp == 0) {
        trx_route_token<true>(s_logit, E, k, S.norm_topk, lane, sp, s_selid, s_selw);
        __syncwarp();
        const bool out = c == 0;
        if (out && w.out_sel_id && lane < k) {
            w.out_sel_id[lane] = s_selid[lane];
            w.out_sel_w[lane] = s_selw[lane];
        }
    }
    __syncthreads();
    TRX_TRACE(60);

    const uint64_t pol = trx_policy_evict_first(); // the weights are read once a call
    if (warp == TRX_DC_CWARPS && c == 0 && (w.out_offsets || w.out_place)) {
        // the dispatch permutation, when asked for: the ids are sorted already, so only CTA 0 forms it, off the
        // experts' path (the trivial sort, Trochilus's counting sort for one token)
        trx_sort_single(s_selid, E, k, TrxSortOut{s_off, s_act, &s_nact, s_place, s_xmap, w.out_offsets, w.out_place},
                        lane);
    }
    if (warp == TRX_DC_CWARPS) {
        // the CTA's share of every selected expert into L2 at once (gate rows, up rows, down rows, the down rows' d
        // values: lane 4 i + part), so that HBM streams the whole call's weights while the rings start; the rings'
        // copies then read L2
        const int i = lane >> 2, part = lane & 3, rbg = H / 256 * (Q8 ? 272 : 144);
        const int rbd = nsb * (Q8 ? 272 : DQ4 ? 144 : 208);
        if (i < k) {
            const int e = s_selid[i];
            if (part < 2) {
                const uint8_t *mat = part == 0 ? L.gate + e * L.gate_mb : L.up + e * L.up_mb;
                if (ng > 0) trx_bulk_prefetch_l2(mat + (int64_t)ga * rbg, (uint32_t)(ng * rbg));
            } else if (nd > 0) {
                const uint8_t *mat = L.down + e * L.down_mb;
                if (part == 2) {
                    trx_bulk_prefetch_l2(mat + (int64_t)da * rbd, (uint32_t)(nd * rbd));
                } else if (!Q8 && !DQ4) { // the Q6L d values of rows [da, da + nd), widened to 16-byte bounds
                    const int64_t lo = (int64_t)H * rbd + (((int64_t)da * nsb * 2) & ~15ll);
                    const int64_t hi = (int64_t)H * rbd + (((int64_t)(da + nd) * nsb * 2 + 15) & ~15ll);
                    trx_bulk_prefetch_l2(mat + lo, (uint32_t)(hi - lo));
                }
            }
        }
    }
    bool failed = false;
    if (warp < TRX_DC_CWARPS) {
        // ---------------- a consumer warp: GU gate/up units, then DN down steps, through its slots
        uint8_t *slots = smem + (size_t)warp * NS * SLOT;
        // gate/up units (expert-major; Q4_K: an expert's NB blocks), down units (expert pairs; Q4_K down: an
        // expert's nsb blocks)
        const int ngu = Q8 ? k * ng : k * NB, ndn = DQ4 ? k * nsb : (k / 2) * nd;
        // row bytes (Q8L: 272 a block; Q6L: 208 a block, the d values apart) and a half-warp's share of a down step
        const int rbg = H / 256 * (Q8 ? 272 : 144), rbd = nsb * (Q8 ? 272 : 208), rhalf = Q8 ? 2 * rbd : 2 * rbd + 32;
        // lane 0 arms step j in its slot (a step with nothing to load completes at once: zero bytes expected)
        auto issue = [&](int j) {
            if (lane != 0) return;
            uint8_t *dst = slots + (j % NS) * SLOT;
            uint64_t *bar = &s_full[warp][j % NS];
            trx_fence_proxy_async(); // this warp's reads of the slot's last step before the copy rewrites it
            if (j < GU) {
                const int u = warp + TRX_DC_CWARPS * j;
                if (u >= ngu) {
                    trx_mbar_expect_tx(bar, 0u);
                    return;
                }
                if (Q8) {
                    const int i = u / ng, r = ga + u % ng, e = s_selid[i];
                    trx_mbar_expect_tx(bar, 2u * rbg);
                    trx_bulk_g2s_hint(dst, L.gate + e * L.gate_mb + (int64_t)r * rbg, rbg, bar, pol);
                    trx_bulk_g2s_hint(dst + rbg, L.up + e * L.up_mb + (int64_t)r * rbg, rbg, bar, pol);
                } else { // 256-block b of rows ga .. ga + 7 of expert e's gate and up (rows past F read as zeros)
                    const int i = u / NB, b = u % NB, e = s_selid[i];
                    trx_mbar_expect_tx(bar, 2u * 8u * 144u);
                    trx_tma_load_3d_hint(dst, &map_gate, 144 * b, ga, e, bar, pol);
                    trx_tma_load_3d_hint(dst + 8 * 144, &map_up, 144 * b, ga, e, bar, pol);
                }
            } else if (DQ4) { // 256-block b of rows da .. da + 15 of expert e's down (rows past H read as zeros)
                const int v = warp + TRX_DC_CWARPS * (j - GU);
                if (v >= ndn) {
                    trx_mbar_expect_tx(bar, 0u);
                    return;
                }
                const int i = v / nsb, b = v % nsb;
                trx_mbar_expect_tx(bar, 16u * 144u);
                trx_tma_load_3d_hint(dst, &map_down, 144 * b, da, s_selid[i], bar, pol);
            } else {
                uint32_t bytes = 0;
                for (int hh = 0; hh < 2; hh++)
                    if (2 * warp + hh + 2 * TRX_DC_CWARPS * (j - GU) < ndn) bytes += (uint32_t)rhalf;
                trx_mbar_expect_tx(bar, bytes);
                for (int hh = 0; hh < 2; hh++) {
                    const int v = 2 * warp + hh + 2 * TRX_DC_CWARPS * (j - GU);
                    if (v >= ndn) continue;
                    const int q = v / nd, r = da + v % nd;
                    uint8_t *d0 = dst + hh * rhalf;
                    for (int ab = 0; ab < 2; ab++) {
                        const uint8_t *mat = L.down + s_selid[2 * q + ab] * L.down_mb;
                        trx_bulk_g2s_hint(d0 + ab * rbd, mat + (int64_t)r * rbd, rbd, bar, pol);
                        // Q6L: the row's d values, the 16-byte piece that holds them
                        if (!Q8)
                            trx_bulk_g2s_hint(d0 + 2 * rbd + 16 * ab,
                                              mat + (int64_t)H * rbd + ((int64_t)r * nsb * 2 & ~15ll), 16u, bar, pol);
                    }
                }
            }
        };
        int issued = 0;
        for (; issued < NS; issued++) issue(issued);
        float *ss = s_q6sc[2 * warp + (lane >> 4)];
        for (int j = 0; j < GU + DN && !failed; j++) {
            const uint8_t *src = slots + (j % NS) * SLOT;
            if (!__all_sync(0xffffffffu, trx_mbar_wait(&s_full[warp][j % NS], (j / NS) & 1, TRX_WAIT_NS))) {
                failed = true;
                break;
            }
            if (warp == 0) TRX_TRACE(8 + j); // (the timeline: warp 0's step j has its weights)
            if (j < GU) {
                const int u = warp + TRX_DC_CWARPS * j;
                if (u < ngu && Q8) { // the gate row by half-warp 0, the up row by half-warp 1 (16-lane contract each)
                    const float y = trx_q8l_dot<true>(src + (lane >> 4) * rbg, xlc, H / 256, lane & 15);
                    const float yu = __shfl_sync(0xffffffffu, y, 16);
                    if (lane == 0) { // to the silu warp
                        s_gu[u] = make_float2(y, yu);
                        trx_mbar_arrive(&s_gubar[j]);
                    }
                } else if (u < ngu) { // block b of the 8 gate and 8 up rows: lane 4 g holds row g's block values
                    const int i = u / NB, b = u % NB;
                    double vg, vu;
                    trx_q4k_blk_mma(src, src + 8 * 144, xdig + 1024 * b, xbf + 8 * b, xsc[b], lane, vg, vu);
                    if ((lane & 3) == 0 && (lane >> 2) < ng) {
                        sv[16 * (i * NB + b) + (lane >> 2)] = vg;
                        sv[16 * (i * NB + b) + 8 + (lane >> 2)] = vu;
                    }
                    trx_mbar_arrive(&s_gubar[i]); // (every lane: its own stores before the silu warp's reads)
                }
            } else if (DQ4) {
                // a Q4_K down unit: block b of the CTA's 16 rows of expert i against the expert's h, prepared here
                // in place for Q4_K's integer definition (this unit is the block's only reader), on the tensor cores
                const int v = warp + TRX_DC_CWARPS * (j - GU);
                if (v < ndn) {
                    const int i = v / nsb, b = v % nsb, ib = i * nsb + b;
                    if (!__all_sync(0xffffffffu, trx_mbar_wait(&s_hbar[i], 0, TRX_WAIT_NS))) {
                        failed = true;
                        break;
                    }
                    uint8_t *hd = reinterpret_cast<uint8_t *>(hbuf + (size_t)i * F + 256 * b);
                    trx_prep_q4m_block(reinterpret_cast<const float *>(hd), hd, dbf + 8 * ib, dsc + ib, lane);
                    __syncwarp();
                    double v0, v1; // (tile rows g and 8 + g)
                    trx_q4k_blk_mma(src, src + 8 * 144, hd, dbf + 8 * ib, dsc[ib], lane, v0, v1);
                    if ((lane & 3) == 0) {
                        const int g = lane >> 2;
                        if (g < nd) dv[16 * ib + g] = v0;
                        if (8 + g < nd) dv[16 * ib + 8 + g] = v1;
                    }
                }
            } else {
                const int v = 2 * warp + (lane >> 4) + 2 * TRX_DC_CWARPS * (j - GU);
                const int v0 = 2 * warp + 2 * TRX_DC_CWARPS * (j - GU);
                if (v0 < ndn) { // (the warp's first unit exists; a second one past the end computes unstored)
                    const bool valid = v < ndn;
                    const int q = valid ? v / nd : 0, rl = valid ? v % nd : 0, r = da + rl;
                    const bool ok =
                        trx_mbar_wait(&s_hbar[2 * q], 0, TRX_WAIT_NS) && trx_mbar_wait(&s_hbar[2 * q + 1], 0, TRX_WAIT_NS);
                    if (!__all_sync(0xffffffffu, ok)) {
                        failed = true;
                        break;
                    }
                    if (warp == 0) TRX_TRACE(24 + j); // its h rows
                    const uint8_t *d0 = src + (valid ? (lane >> 4) : 0) * rhalf;
                    const uint8_t *rb = d0 + rbd;
                    const float *xab = hbuf + (size_t)q * 2 * F;
                    float2 val;
                    if (Q8) {
                        val = nsb == 4   ? trx_q8l_dot_pair_il<4>(d0, rb, xab, lane & 15)
                              : nsb == 2 ? trx_q8l_dot_pair_il<2>(d0, rb, xab, lane & 15)
                                         : trx_q8l_dot_pair_il<1>(d0, rb, xab, lane & 15);
                    } else {
                        const int dh = (r * nsb * 2) & 15; // the row's d values inside their 16-byte piece
                        const uint8_t *dA = d0 + 2 * rbd + dh, *dB = d0 + 2 * rbd + 16 + dh;
                        val = nsb == 4   ? trx_q6l_dot_pair_il<4>(d0, dA, rb, dB, xab, lane & 15, ss)
                              : nsb == 2 ? trx_q6l_dot_pair_il<2>(d0, dA, rb, dB, xab, lane & 15, ss)
                                         : trx_q6l_dot_pair_il<1>(d0, dA, rb, dB, xab, lane & 15, ss);
                    }
                    if (valid && (lane & 15) == 0) {
                        s_h3[2 * q][rl] = val.x;
                        s_h3[2 * q + 1][rl] = val.y;
                    }
                }
            }
            __syncwarp();
            if (warp == 0) TRX_TRACE(16 + j); // computed
            if (issued < GU + DN) issue(issued++);
        }
        if (failed && lane == 0) { // every copy this warp armed lands before the CTA can leave
            for (int j = 0; j < issued; j++)
                trx_mbar_wait(&s_full[warp][j % NS], (j / NS) & 1, TRX_WAIT_NS);
        }
    } else if (warp == TRX_DC_SILU) {
        // ---------------- h = silu(g) u of a step's gate/up units at once (lane l: unit 14 j + l), published tagged;
        // the consumers go on to their next rows meanwhile
        const int ngu = k * ng;
        for (int j = 0; Q8 && j < TRX_DC_GU && TRX_DC_CWARPS * j < ngu && !failed; j++) {
            if (!__all_sync(0xffffffffu, trx_mbar_wait(&s_gubar[j], 0, TRX_WAIT_NS))) {
                failed = true;
                break;
            }
            const int u = TRX_DC_CWARPS * j + lane;
            if (lane < TRX_DC_CWARPS && u < ngu) {
                const float2 gu = s_gu[u];
                trx_st_tagged(w.tag_h + (int64_t)(u / ng) * F + trx_lc_pos(ga + u % ng), tag, trx_silu_mul(gu.x, gu.y));
            }
        }
        // Q4_K: expert i as soon as its NB units are in, with the experts after it that are in already (at most four
        // in all, when this warp lags behind the consumers), lane 8 e + r taking row ga + r of expert i + e: the
        // block values added in order from +0 (f64), rounded to float once (Trochilus's Q4_K row value), then
        // h = silu(g) u. (Waiting for four experts at a time measured 1.5 us slower a call: the down steps wait for
        // the first experts' h.)
        for (int i = 0; !Q8 && i < k && !failed;) {
            if (!__all_sync(0xffffffffu, trx_mbar_wait(&s_gubar[i], 0, TRX_WAIT_NS))) {
                failed = true;
                break;
            }
            int n = 1;
            if (lane == 0)
                while (n < 4 && i + n < k && trx_mbar_try_wait(&s_gubar[i + n], 0)) n++;
            n = __shfl_sync(0xffffffffu, n, 0);
            const int e = i + (lane >> 3), r = lane & 7;
            // (each lane's own wait on a completed barrier: its acquire of that expert's values)
            if ((lane >> 3) < n && trx_mbar_wait(&s_gubar[e], 0, TRX_WAIT_NS) && r < ng) {
                double ag = 0.0, au = 0.0;
                for (int b = 0; b < NB; b++) {
                    ag = __dadd_rn(ag, sv[16 * (e * NB + b) + r]);
                    au = __dadd_rn(au, sv[16 * (e * NB + b) + 8 + r]);
                }
                // (LC order for a Q6_K down's lane contract; a Q4_K down takes the row in its natural order)
                trx_st_tagged(w.tag_h + (int64_t)e * F + (DQ4 ? ga + r : trx_lc_pos(ga + r)), tag,
                              trx_silu_mul(__double2float_rn(ag), __double2float_rn(au)));
            }
            i += n;
        }
    } else if (warp == TRX_DC_HELPER) {
        // ---------------- the helper: expert i's h into shared memory, experts in order, each value once it carries
        // this call's tag. Lane l takes value pairs l + 32 m (m < F / 64): every load of a poll is issued before the
        // first is looked at, 512 contiguous bytes a warp-wide load; the lane arrives once it holds all its pairs.
        const int npair = F / 64; // 4, 8 or 16
        for (int i = 0; i < k && !failed; i++) {
            const unsigned long long *src = w.tag_h + (int64_t)i * F;
            // expert pairs' rows interleaved (trx_il_off); a Q4_K down takes each expert's row as it is
            float *dst = DQ4 ? hbuf + (size_t)i * F : hbuf + (size_t)(i >> 1) * 2 * F + (i & 1);
            uint32_t want = (1u << npair) - 1u; // the pairs still missing
            uint64_t t0 = 0;
            for (;;) {
                ulonglong2 v[16];
#pragma unroll
                for (int m = 0; m < 16; m++)
                    if (want >> m & 1u) v[m] = trx_ld_tagged2(src + 2 * (lane + 32 * m));
#pragma unroll
                for (int m = 0; m < 16; m++) {
                    if ((want >> m & 1u) && (uint32_t)(v[m].x >> 32) == tag && (uint32_t)(v[m].y >> 32) == tag) {
                        const int pos = 2 * (lane + 32 * m); // (even: pos and pos + 1 are 2 apart in the layout)
                        if (DQ4) {
                            dst[pos] = __uint_as_float((uint32_t)v[m].x);
                            dst[pos + 1] = __uint_as_float((uint32_t)v[m].y);
                        } else {
                            dst[trx_il_off(pos)] = __uint_as_float((uint32_t)v[m].x);
                            dst[trx_il_off(pos) + 2] = __uint_as_float((uint32_t)v[m].y);
                        }
                        want &= ~(1u << m);
                    }
                }
                if (want == 0u) break;
                const uint64_t now = trx_globaltimer();
                if (t0 == 0) t0 = now;
                else if (now - t0 > TRX_SPIN_NS) {
                    failed = true;
                    break;
                }
                __nanosleep(100);
            }
            if (__any_sync(0xffffffffu, failed)) {
                failed = true;
                break;
            }
            if (w.trace != nullptr && lane == 0) w.trace[(size_t)blockIdx.x * 64 + 32 + i] = trx_globaltimer();
            trx_mbar_arrive(&s_hbar[i]); // (each lane its own values: the barrier orders them before the readers)
        }
    }
    TRX_TRACE(6);

    // ---------------- mix and end
    if (__syncthreads_or(failed)) {
        if (tid == 0) {
            atomicCAS(w.err, 0, 3);
            if (w.host_done) trx_post_done(w.host_done, epoch | 0x80000000u);
        }
        return;
    }
    if (tid < nd) { // output row da + tid: the k outputs in increasing expert id, then the residual
        float out = 0.0f;
        for (int i = 0; i < k; i++) {
            float h3 = 0.0f;
            if (DQ4) { // the row's block values added in order from +0 (f64), rounded once
                double a = 0.0;
                for (int b = 0; b < nsb; b++) a = __dadd_rn(a, dv[16 * (i * nsb + b) + tid]);
                h3 = __double2float_rn(a);
            } else {
                h3 = s_h3[i][tid];
            }
            out = __fadd_rn(out, __fmul_rn(s_selw[i], h3));
        }
        if (ffn_out) ffn_out[da + tid] = out;
        x_io[da + tid] = __fadd_rn(xres, out);
    }
    __syncthreads();
    TRX_TRACE(52);
    if (w.host_done == nullptr) {
        if (c == 0 && tid == 0) sync->seq = tag; // the next call's tag: tag + 1 (the next kernel sees it at our end)
        return;
    }
    if (tid == 0) { // the host-pointer road: the host learns the end from a word the last CTA posts
        __threadfence_system(); // the outputs (x may be host memory) before the count
        if (atomicAdd(&sync->finish, 1u) == (uint32_t)G - 1) { // every CTA is past its waits
            sync->seq = tag;
            sync->finish = 0u;
            __threadfence();
            // (a call of several tokens runs one launch a token and only the last posts: it reports any give-up)
            trx_post_done(w.host_done, *(volatile int32_t *)w.err ? (epoch | 0x80000000u) : epoch);
        }
    }
}
