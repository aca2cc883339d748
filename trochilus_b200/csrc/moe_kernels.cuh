// moe_kernels.cuh: Trochilus's OLMoE MoE layer on the GPU, exact, as a few kernels on one stream.
//
//   trx_k_router   router logits under the 16-lane contract (the expert row and the inputs staged in shared
//                  memory, the lane chains fed from registers); for up to TRX_ROUTE_FUSED_MAX tokens the last
//                  router block to finish also routes every token (softmax with the correctly rounded exp,
//                  top-k, ids sorted) and runs the stable counting sort of the (token, slot) rows; extra
//                  blocks prepare each token's input row for the expert products
//   trx_k_route / trx_k_sort / trx_k_prep_tokens   the same steps as separate kernels for longer passes
//   trx_k_gateup   gate and up rows of the routed experts streamed through shared memory by 1-D TMA bulk
//                  copies; SwiGLU fused; h written in the order the down kernel reads
//   trx_k_prep     Q4_K down only: h rows prepared for Q4_K's integer definition
//   trx_k_down     down rows streamed the same way into h3; the last CTA to finish a block of 16 output rows
//                  adds every token's k expert outputs in increasing expert id and adds the sum to the
//                  residual (Trochilus's mix_body)
//
// Work split of the streaming kernels: the routed experts' rows form one virtual row space (slot i of the
// active experts owns rows [i R, (i + 1) R)); CTA c takes the contiguous range [c V / G, (c + 1) V / G), so
// every CTA streams the same number of rows (+-1) whatever the routing, and cuts it into chunks that do not
// cross an expert (nor, for the down, a 16-row combine block). A CTA arms up to TRX_STAGES chunks at once.
//
// Trochilus references: forward_layer's MoE block src/models/olmoe.c:1845-1933; route_token / top_experts
// olmoe.c:1455-1502; the counting sort olmoe.c:1850-1861; tr_softmax src/kernels/kernels.c:1377-1388;
// SwiGLU kernels.c:1397-1421; mix_body olmoe.c:1432-1446.
#pragma once
#include <cstdint>
#include "bulk.cuh"
#include "common.cuh"
#include "expf.cuh"
#include "layouts.cuh"

#define TRX_MAX_EXPERTS 64
#define TRX_MAX_USED 32
#define TRX_GU_CHUNK 8          // gate/up rows a chunk (a warp per row: its gate and up rows)
#define TRX_DN_CHUNK 16         // down output rows a chunk (a half-warp per row); the combine block
#define TRX_STAGES 4            // chunks a CTA has in flight
#define TRX_TOK_GROUP 8         // a segment's rows per epilogue pass
#define TRX_ROUTE_FUSED_MAX 64  // tokens up to which the router kernel routes in its last block
#define TRX_TOK_STAGE 16        // tokens whose inputs a router block stages at once
#define TRX_WAIT_NS 2000000000ull

struct TrxLayer {
    int router_type, gate_type, up_type, down_type;
    const uint8_t *router;
    const float *router_bias;        // NULL: none
    const uint8_t *gate, *up, *down; // n_expert matrices each
    int64_t gate_mb, up_mb, down_mb; // bytes per expert matrix
    const float *norm_w;             // ffn_norm weight (n_embd floats), NULL until set
    float norm_eps;
};

struct TrxShape {
    int E, k, H, F, norm_topk;
    int norm_in; // the fused kernel: the input rows are the residual stream, normalised with L.norm_w first
    int ext;     // the fused kernel: rows routed elsewhere (expert parallelism): row t goes to expert w.ext_ids[t]
                 // alone (k = 1, weight 1; -1: none), the output is the expert's row (ffn_out), no residual
};

struct TrxWork {
    float *logits;       // [T][E]
    int32_t *sel_id;     // [R]
    float *sel_w;        // [R]
    int32_t *offsets;    // [E + 1]
    int32_t *place;      // [R]
    int32_t *xmap;       // [R] token of grouped row p
    int32_t *active;     // [E]
    int32_t *n_active;   // [1]
    uint32_t *route_cnt; // [1]
    uint32_t *comb_cnt;  // [H / TRX_DN_CHUNK]
    int32_t *err;        // [1] nonzero: a kernel gave up waiting for its copies
    float *x_lc;         // [T][H]
    uint32_t *xq;        // [T][H]
    double *xq_bf;       // [T][H / 32]
    double *xq_sc;       // [T][H / 256]
    float *h;            // [R][F]
    uint32_t *hq;        // [R][F]
    double *hq_bf;       // [R][F / 32]
    double *hq_sc;       // [R][F / 256]
    float *h3;           // [R][H]
    int64_t *out_sel_id; // optional outputs (NULL: not written)
    float *out_sel_w;
    int64_t *out_offsets;
    int64_t *out_place;
    float *out_logits;
    uint64_t *trace;     // NULL, or 64 %globaltimer slots per CTA of the fused kernel (tr_gpu_moe_trace)
    float *out_normed;   // NULL, or where the fused kernel (norm_in) writes the normalised rows
    const int32_t *ext_ids; // the fused kernel's external routing (ext): each row's expert, -1 for none
    const struct TrxEpPeers *ep; // ext over peer memory: rows and ids from this rank's exchange region, each output
                                 // row back into its source rank's region, then the sources' return flags
    uint32_t *host_done; // NULL, or a word of mapped pinned host memory: the fused kernel writes its epoch there
                         // once every output is visible to the host (bit 31 set: it gave up)
    unsigned long long *tag_logits; // the one-token kernel (decode.cuh): [E] logits, each with the call's tag
    unsigned long long *tag_h;      // and [k][F] h values (LC order), each with the call's tag
};

// ---------------------------------------------------------------------------------------------
// routing

// One token's routing by one warp: softmax over E <= 64 logits (lane i holds i and i + 32), the k experts,
// their weights, written sorted by id. After the softmax the probabilities are either all NaN (a NaN or an
// infinite logit, or every logit -inf) or none is; the reference's repeated argmax (first untaken id when it
// is NaN, else the largest, ties to the lower id) then picks ids 0..k-1 in the first case and the k largest
// by (value, -id) in the second. The rank of each value among all E gives the latter directly.
// Not inlined: one copy of the code, so that a warp that runs it early (on dummy logits) leaves it in the SM's
// instruction caches for the call's real routing.
template <bool SM = false>
__device__ __noinline__ void trx_route_token(const float *__restrict__ logits, int E, int k, int norm_topk, int lane,
                                float *__restrict__ sp, int32_t *ids_out, float *w_out) {
    const bool ok0 = lane < E, ok1 = lane + 32 < E;
    const float v0 = ok0 ? (SM ? logits[lane] : __ldcg(logits + lane)) : 0.0f;
    const float v1 = ok1 ? (SM ? logits[lane + 32] : __ldcg(logits + lane + 32)) : 0.0f;
    // max: the serial scan from x[0] with strict > keeps x[0] when it is a NaN, else it is the largest
    // non-NaN value (x[0] among them)
    float m = -__int_as_float(0x7f800000);
    if (ok0 && v0 == v0) m = fmaxf(m, v0);
    if (ok1 && v1 == v1) m = fmaxf(m, v1);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float x0 = __shfl_sync(0xffffffffu, v0, 0);
    if (x0 != x0) m = x0;
    const float2 ee = trx_expf2(ok0 ? __fsub_rn(v0, m) : -1.0f, ok1 ? __fsub_rn(v1, m) : -1.0f);
    const float e0 = ok0 ? ee.x : 0.0f, e1 = ok1 ? ee.y : 0.0f;
    // 16-lane sum: lane l (< 16) adds elements l, l+16, l+32, l+48 in order from +0 (absent ones are +0)
    const float b = __shfl_sync(0xffffffffu, e0, (lane & 15) + 16);
    const float d = __shfl_sync(0xffffffffu, e1, (lane & 15) + 16);
    float acc = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(0.0f, e0), b), e1), d);
    acc = trx_lane_tree16(acc);
    const float sum = __shfl_sync(0xffffffffu, acc, 0);
    const float p0 = __fdiv_rn(e0, sum), p1 = __fdiv_rn(e1, sum);
    const bool any_nan = __any_sync(0xffffffffu, (ok0 && p0 != p0) || (ok1 && p1 != p1));
    int r0 = lane, r1 = lane + 32; // selection rank of elements lane and lane + 32
    if (!any_nan) {
        // the rank of each element in the order the k rounds of argmax take them (larger probability first, ties
        // to the lower id): probabilities are in [0, 1], so their bits order them as unsigned integers; key = bits
        // + 1 for a present element, 0 for an absent one (E < 64), which no present element follows
        const uint32_t q0 = ok0 ? __float_as_uint(p0) + 1u : 0u, q1 = ok1 ? __float_as_uint(p1) + 1u : 0u;
        // the 64 keys come by shuffles, all issued independently (the loop fully unrolled, four partial counts a
        // key), so that their latencies overlap
        int c0[4] = {0, 0, 0, 0}, c1[4] = {0, 0, 0, 0};
#pragma unroll
        for (int j = 0; j < 32; j++) {
            const uint32_t a = __shfl_sync(0xffffffffu, q0, j), b = __shfl_sync(0xffffffffu, q1, j); // ids j, j + 32
            c0[j & 3] += (a > q0 || (a == q0 && j < lane)) + (b > q0);
            c1[j & 3] += (a >= q1) + (b > q1 || (b == q1 && j < lane));
        }
        r0 = (c0[0] + c0[1]) + (c0[2] + c0[3]);
        r1 = (c1[0] + c1[1]) + (c1[2] + c1[3]);
    }
    const bool s0 = ok0 && r0 < k, s1 = ok1 && r1 < k;
    float w0 = p0, w1 = p1;
    if (norm_topk) { // the weights summed in selection order, then each divided by the sum
        if (s0) sp[64 + r0] = p0;
        if (s1) sp[64 + r1] = p1;
        __syncwarp();
        float sm = 0.0f;
        for (int i = 0; i < k; i++) sm = __fadd_rn(sm, sp[64 + i]);
        __syncwarp();
        w0 = __fdiv_rn(p0, sm);
        w1 = __fdiv_rn(p1, sm);
    }
    const unsigned b0 = __ballot_sync(0xffffffffu, s0), b1 = __ballot_sync(0xffffffffu, s1);
    const unsigned lt = (1u << lane) - 1u;
    if (s0) {
        const int slot = __popc(b0 & lt);
        ids_out[slot] = lane;
        w_out[slot] = w0;
    }
    if (s1) {
        const int slot = __popc(b0) + __popc(b1 & lt);
        ids_out[slot] = lane + 32;
        w_out[slot] = w1;
    }
}

// Stable counting sort of R rows by expert, by one block of WARPS warps. place[j] = the row's position in
// the grouped order: its expert's start plus the rows of that expert before j.
template <int WARPS>
__device__ void trx_block_counting_sort(const int32_t *__restrict__ sel_id, int R, int E, int k, TrxWork w) {
    __shared__ int cnt[TRX_MAX_EXPERTS + 1];
    __shared__ int run[TRX_MAX_EXPERTS];
    __shared__ int wc[WARPS][TRX_MAX_EXPERTS];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nt = WARPS * 32;
    for (int e = tid; e <= E; e += nt) cnt[e] = 0;
    __syncthreads();
    for (int j = tid; j < R; j += nt) atomicAdd(&cnt[sel_id[j]], 1);
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
    for (int base = 0; base < R; base += nt) {
        const int j = base + tid;
        const int e = j < R ? sel_id[j] : -1;
        for (int i = tid; i < WARPS * TRX_MAX_EXPERTS; i += nt) (&wc[0][0])[i] = 0;
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
        for (int ee = tid; ee < E; ee += nt) {
            int s = 0;
            for (int v = 0; v < WARPS; v++) s += wc[v][ee];
            run[ee] += s;
        }
        __syncthreads();
    }
}

// Where a warp counting sort writes: offsets [E + 1], active [E], n_active [1], place [R], xmap [R] (shared or global
// memory), and the optional int64 copies of offsets and place
struct TrxSortOut {
    int32_t *offsets, *active, *n_active, *place, *xmap;
    int64_t *out_offsets, *out_place;
};

// The sort of a single token's k rows by one warp: its k ids are distinct and already in increasing order, so
// expert sel_id[j] holds row j alone: offsets[e] = the number of selected ids below e, place[j] = j, every row is
// token 0. Not inlined (warmed up early, as trx_route_token).
__device__ __noinline__ void trx_sort_single(const int32_t *__restrict__ sel_id, int E, int k, TrxSortOut w, int lane) {
    const int e0 = lane < k ? sel_id[lane] : TRX_MAX_EXPERTS;
    for (int e = lane; e <= E; e += 32) {
        int c = 0;
        for (int j = 0; j < k; j++) c += sel_id[j] < e;
        w.offsets[e] = c;
        if (w.out_offsets) w.out_offsets[e] = c;
    }
    if (lane < k) {
        w.active[lane] = e0;
        w.place[lane] = lane;
        w.xmap[lane] = 0;
        if (w.out_place) w.out_place[lane] = lane;
    }
    if (lane == 0) *w.n_active = k;
}

// The same by one warp, any R (32 rows a pass, stable by match_any ranks); scnt: 64 ints of shared memory
__device__ void trx_warp_counting_sort(const int32_t *__restrict__ sel_id, int R, int E, int k, TrxSortOut w, int *scnt,
                                       int lane) {
    scnt[lane] = 0;
    scnt[lane + 32] = 0;
    __syncwarp();
    for (int b = 0; b < R; b += 32) {
        const int e = b + lane < R ? sel_id[b + lane] : -1;
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        if (e >= 0 && lane == __ffs(peers) - 1) scnt[e] += __popc(peers);
        __syncwarp();
    }
    const int c0 = lane < E ? scnt[lane] : 0, c1 = lane + 32 < E ? scnt[lane + 32] : 0;
    int i0 = c0, i1 = c1; // inclusive scans
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int a = __shfl_up_sync(0xffffffffu, i0, o), b = __shfl_up_sync(0xffffffffu, i1, o);
        if (lane >= o) {
            i0 += a;
            i1 += b;
        }
    }
    const int total0 = __shfl_sync(0xffffffffu, i0, 31), total = total0 + __shfl_sync(0xffffffffu, i1, 31);
    const int off0 = i0 - c0, off1 = total0 + i1 - c1;
    if (lane < E) {
        w.offsets[lane] = off0;
        if (w.out_offsets) w.out_offsets[lane] = off0;
    }
    if (lane + 32 < E) {
        w.offsets[lane + 32] = off1;
        if (w.out_offsets) w.out_offsets[lane + 32] = off1;
    }
    if (lane == 0) { // the rows with an expert (rows with none, id -1, are left out)
        w.offsets[E] = total;
        if (w.out_offsets) w.out_offsets[E] = total;
    }
    const unsigned a0 = __ballot_sync(0xffffffffu, c0 > 0), a1 = __ballot_sync(0xffffffffu, c1 > 0);
    const unsigned lt = (1u << lane) - 1u;
    if (c0 > 0) w.active[__popc(a0 & lt)] = lane;
    if (c1 > 0) w.active[__popc(a0) + __popc(a1 & lt)] = lane + 32;
    if (lane == 0) *w.n_active = __popc(a0) + __popc(a1);
    __syncwarp();
    scnt[lane] = off0; // the running start of each expert
    scnt[lane + 32] = off1;
    __syncwarp();
    for (int b = 0; b < R; b += 32) {
        const int j = b + lane, e = j < R ? sel_id[j] : -1;
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        if (e >= 0) {
            const int pos = scnt[e] + __popc(peers & lt);
            w.place[j] = pos;
            w.xmap[pos] = j / k;
            if (w.out_place) w.out_place[j] = pos;
        }
        __syncwarp();
        if (e >= 0 && lane == __ffs(peers) - 1) scnt[e] += __popc(peers);
        __syncwarp();
    }
}

// one token's input row prepared for the gate/up products (one block)
__device__ void trx_prep_token(const TrxLayer &L, const TrxShape &S, const float *__restrict__ normed, int t,
                               TrxWork &w) {
    const int tid = threadIdx.x, lane = tid & 31, H = S.H;
    const float *x = normed + (int64_t)t * H;
    if (L.gate_type == TRX_Q4_K) {
        const int nsb = H / 256;
        for (int s = tid >> 5; s < nsb; s += blockDim.x >> 5)
            trx_prep_q4x_block(x + 256 * s, w.xq + (int64_t)t * H, s, nsb, w.xq_bf + (int64_t)t * (H / 32) + 8 * s,
                               w.xq_sc + (int64_t)t * (H / 256) + s, lane);
    } else {
        for (int kk = tid; kk < H; kk += blockDim.x) w.x_lc[(int64_t)t * H + trx_lc_pos(kk)] = x[kk];
    }
}

// Router logits of expert e for tokens [g_begin, g_end) by one block of 256 threads; sdyn: (1 +
// min(tokens, TRX_TOK_STAGE)) * H floats of shared memory.
// nthr: 0 = the whole block takes part; else threads 0 .. nthr - 1 only (a multiple of 32), which meet at named
// barrier 3 instead of the block barrier, so that the others are free meanwhile.
__device__ void trx_router_block(const TrxLayer &L, const TrxShape &S, const float *__restrict__ normed, int e,
                                 int g_begin, int g_end, TrxWork &w, float *sdyn, int nthr = 0) {
    const int tid = threadIdx.x, nt = nthr ? nthr : (int)blockDim.x;
    auto sync = [&]() {
        if (nthr) asm volatile("bar.sync 3, %0;" ::"r"(nthr) : "memory");
        else __syncthreads();
    };
    const int E = S.E, H = S.H;
    float *srow = sdyn, *sx = sdyn + H;
    const int64_t rb = trx_row_bytes(L.router_type, H);
    const uint8_t *row = L.router + e * rb; // lane-row order (trx_repack_lanerows): packed q holds element k below
    auto k_of = [](int q) { return (q & ~255) + ((q >> 4) & 15) + 16 * (q & 15); };
    if (L.router_type == TRX_F32) {
        for (int i = tid; i < H / 4; i += nt) {
            const float4 v = __ldg(reinterpret_cast<const float4 *>(row) + i);
            srow[trx_lc_pos(k_of(4 * i))] = v.x;
            srow[trx_lc_pos(k_of(4 * i + 1))] = v.y;
            srow[trx_lc_pos(k_of(4 * i + 2))] = v.z;
            srow[trx_lc_pos(k_of(4 * i + 3))] = v.w;
        }
    } else { // 8 bfloat16 a load, widened exactly
        for (int i = tid; i < H / 8; i += nt) {
            const uint4 v = __ldg(reinterpret_cast<const uint4 *>(row) + i);
            const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int q = 0; q < 4; q++) {
                srow[trx_lc_pos(k_of(8 * i + 2 * q))] = __uint_as_float(u[q] << 16);
                srow[trx_lc_pos(k_of(8 * i + 2 * q + 1))] = __uint_as_float(u[q] & 0xffff0000u);
            }
        }
    }
    const int tg = tid >> 4, l = tid & 15;
    const float bias = L.router_bias ? L.router_bias[e] : 0.0f;
    const int nch = H / 256;
    for (int g0 = g_begin; g0 < g_end; g0 += TRX_TOK_STAGE) {
        const int ng = min(TRX_TOK_STAGE, g_end - g0);
        if (g0 != g_begin) sync(); // the first group's loads go out with the router row's
        for (int i = tid; i < ng * H / 4; i += nt) { // inputs of the group, LC order
            const int tk = (4 * i) / H, kk = (4 * i) % H;
            const float4 v = *reinterpret_cast<const float4 *>(normed + (int64_t)(g0 + tk) * H + kk);
            float *dst = sx + tk * H;
            dst[trx_lc_pos(kk)] = v.x;
            dst[trx_lc_pos(kk + 1)] = v.y;
            dst[trx_lc_pos(kk + 2)] = v.z;
            dst[trx_lc_pos(kk + 3)] = v.w;
        }
        sync();
        for (int tb = 0; tb < ng; tb += nt / 16) { // a half-warp a token (uniform trip count: the tree's shuffles)
        const int tk = tb + tg < ng ? tb + tg : 0;
        const float *xs = sx + tk * H + 4 * l, *ws = srow + 4 * l;
        float acc = 0.0f;
        for (int i = 0; i < nch; i++) {
            float wv[16], xv[16];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const float4 a = *reinterpret_cast<const float4 *>(ws + 256 * i + 64 * q);
                const float4 c = *reinterpret_cast<const float4 *>(xs + 256 * i + 64 * q);
                wv[4 * q] = a.x; wv[4 * q + 1] = a.y; wv[4 * q + 2] = a.z; wv[4 * q + 3] = a.w;
                xv[4 * q] = c.x; xv[4 * q + 1] = c.y; xv[4 * q + 2] = c.z; xv[4 * q + 3] = c.w;
            }
#pragma unroll
            for (int m = 0; m < 16; m++) acc = __fadd_rn(acc, __fmul_rn(wv[m], xv[m]));
        }
        acc = trx_lane_tree16(acc);
        if (l == 0 && tb + tg < ng) {
            const float v = L.router_bias ? __fadd_rn(acc, bias) : acc;
            w.logits[(int64_t)(g0 + tb + tg) * E + e] = v;
            if (w.out_logits) w.out_logits[(int64_t)(g0 + tb + tg) * E + e] = v;
        }
        }
    }
}

// grid.x: E router blocks (+ T prep blocks when fused); grid.y: token groups of TRX_TOK_STAGE (unfused).
// Dynamic shared memory: (1 + min(T, TRX_TOK_STAGE)) * H floats.
__global__ void __launch_bounds__(256) trx_k_router(TrxLayer L, TrxShape S, const float *__restrict__ normed, int T,
                                                    TrxWork w, int fused) {
    extern __shared__ __align__(16) float sdyn[];
    const int tid = threadIdx.x, lane = tid & 31;
    const int E = S.E;
    if ((int)blockIdx.x >= E) {
        trx_prep_token(L, S, normed, blockIdx.x - E, w);
        return;
    }
    const int g_begin = fused ? 0 : blockIdx.y * TRX_TOK_STAGE, g_end = fused ? T : min(T, g_begin + TRX_TOK_STAGE);
    trx_router_block(L, S, normed, blockIdx.x, g_begin, g_end, w, sdyn);
    if (!fused) return;
    // the last router block to finish routes every token and sorts the rows
    __shared__ int s_last;
    __shared__ float sp[8][96];
    __threadfence(); // every writer's logits visible device-wide before the block is counted
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(w.route_cnt, 1u) == (unsigned)(E - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const int warp = tid >> 5, k = S.k;
    for (int t = warp; t < T; t += blockDim.x >> 5)
        trx_route_token(w.logits + (int64_t)t * E, E, k, S.norm_topk, lane, sp[warp], w.sel_id + (int64_t)t * k,
                        w.sel_w + (int64_t)t * k);
    __syncthreads();
    const int R = T * k;
    if (w.out_sel_id)
        for (int j = tid; j < R; j += blockDim.x) {
            w.out_sel_id[j] = w.sel_id[j];
            w.out_sel_w[j] = w.sel_w[j];
        }
    if (R <= 32) {
        __shared__ int scnt[64];
        const TrxSortOut so{w.offsets, w.active, w.n_active, w.place, w.xmap, w.out_offsets, w.out_place};
        if (warp == 0) trx_warp_counting_sort(w.sel_id, R, E, k, so, scnt, lane);
    } else {
        trx_block_counting_sort<8>(w.sel_id, R, E, k, w);
    }
    if (tid == 0) *w.route_cnt = 0u;
}

// Router logits of a long pass, 16 tokens a block and every expert: thread (t = tid / 16, l = tid % 16) keeps lane l's
// running sums of token t for all E experts in registers while the 256-blocks of H go by in order. For each block the
// 16 tokens' inputs (LC order) and every expert's router columns (lane-row packing) are staged in shared memory with
// coalesced loads, one memory latency a block. Same sums, same order as trx_router_block: the 16-lane contract.
// Dynamic shared memory: TRX_TOK_STAGE * 1024 + E * 256 * sizeof(router element) bytes.
template <int RT>
__global__ void __launch_bounds__(256) trx_k_router_many(TrxLayer L, TrxShape S, const float *__restrict__ normed,
                                                         int T, TrxWork w) {
    extern __shared__ __align__(16) float sdyn[];
    constexpr int WB = RT == TRX_F32 ? 1024 : 512; // bytes of one expert's 256-block
    float *sx = sdyn;
    uint8_t *sw = reinterpret_cast<uint8_t *>(sdyn + TRX_TOK_STAGE * 256);
    const int tid = threadIdx.x, t = tid >> 4, l = tid & 15, t0 = blockIdx.x * TRX_TOK_STAGE;
    const int E = S.E, H = S.H, nb = H / 256;
    const int64_t rb = trx_row_bytes(RT, H);
    float acc[TRX_MAX_EXPERTS];
#pragma unroll
    for (int e = 0; e < TRX_MAX_EXPERTS; e++) acc[e] = 0.0f;
    for (int i = 0; i < nb; i++) {
        __syncthreads();
        for (int j = tid; j < E * (WB / 16); j += blockDim.x) { // every expert's block i, 16 bytes a thread
            const int e = j / (WB / 16), q = j % (WB / 16);
            reinterpret_cast<uint4 *>(sw + e * WB)[q] = __ldg(reinterpret_cast<const uint4 *>(L.router + e * rb + (int64_t)i * WB) + q);
        }
        for (int j = tid; j < TRX_TOK_STAGE * 64; j += blockDim.x) { // block i of the 16 tokens, LC order
            const int tt = j >> 6, k = 4 * (j & 63);
            const float4 v = t0 + tt < T ? __ldg(reinterpret_cast<const float4 *>(normed + (int64_t)(t0 + tt) * H + 256 * i + k))
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
            float *dst = sx + tt * 256;
            dst[trx_lc_pos(k)] = v.x;
            dst[trx_lc_pos(k + 1)] = v.y;
            dst[trx_lc_pos(k + 2)] = v.z;
            dst[trx_lc_pos(k + 3)] = v.w;
        }
        __syncthreads();
        float xv[16];
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const float4 c = *reinterpret_cast<const float4 *>(sx + t * 256 + 64 * q + 4 * l);
            xv[4 * q] = c.x; xv[4 * q + 1] = c.y; xv[4 * q + 2] = c.z; xv[4 * q + 3] = c.w;
        }
#pragma unroll
        for (int e = 0; e < TRX_MAX_EXPERTS; e++) {
            if (e < E) {
                float wv[16];
                if (RT == TRX_F32) {
                    const float4 *wp = reinterpret_cast<const float4 *>(sw + e * WB + 64 * l);
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        const float4 a = wp[q];
                        wv[4 * q] = a.x; wv[4 * q + 1] = a.y; wv[4 * q + 2] = a.z; wv[4 * q + 3] = a.w;
                    }
                } else {
                    const uint4 *wp = reinterpret_cast<const uint4 *>(sw + e * WB + 32 * l);
#pragma unroll
                    for (int q = 0; q < 2; q++) {
                        const uint4 a = wp[q];
                        const uint32_t u[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                        for (int r = 0; r < 4; r++) {
                            wv[8 * q + 2 * r] = __uint_as_float(u[r] << 16);
                            wv[8 * q + 2 * r + 1] = __uint_as_float(u[r] & 0xffff0000u);
                        }
                    }
                }
#pragma unroll
                for (int m = 0; m < 16; m++) acc[e] = __fadd_rn(acc[e], __fmul_rn(wv[m], xv[m]));
            }
        }
    }
    const bool valid = t0 + t < T;
#pragma unroll
    for (int e = 0; e < TRX_MAX_EXPERTS; e++) {
        if (e < E) {
            const float v0 = trx_lane_tree16(acc[e]);
            if (l == 0 && valid) {
                const float v = L.router_bias ? __fadd_rn(v0, L.router_bias[e]) : v0;
                w.logits[(int64_t)(t0 + t) * E + e] = v;
                if (w.out_logits) w.out_logits[(int64_t)(t0 + t) * E + e] = v;
            }
        }
    }
}

__host__ __device__ constexpr size_t trx_router_many_smem(int router_type, int E) {
    return (size_t)TRX_TOK_STAGE * 1024 + (size_t)E * (router_type == TRX_F32 ? 1024 : 512);
}

// longer passes: a warp per token
__global__ void __launch_bounds__(256) trx_k_route(TrxShape S, int T, TrxWork w) {
    __shared__ float sp[8][96];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, t = blockIdx.x * 8 + warp;
    if (t >= T) return;
    trx_route_token(w.logits + (int64_t)t * S.E, S.E, S.k, S.norm_topk, lane, sp[warp], w.sel_id + (int64_t)t * S.k,
                    w.sel_w + (int64_t)t * S.k);
    __syncwarp();
    if (w.out_sel_id && lane < S.k) {
        w.out_sel_id[(int64_t)t * S.k + lane] = w.sel_id[(int64_t)t * S.k + lane];
        w.out_sel_w[(int64_t)t * S.k + lane] = w.sel_w[(int64_t)t * S.k + lane];
    }
}

__global__ void __launch_bounds__(1024) trx_k_sort(TrxShape S, int T, TrxWork w) {
    trx_block_counting_sort<32>(w.sel_id, T * S.k, S.E, S.k, w);
}

__global__ void __launch_bounds__(256) trx_k_prep_tokens(TrxLayer L, TrxShape S, const float *__restrict__ normed,
                                                         TrxWork w) {
    trx_prep_token(L, S, normed, blockIdx.x, w);
}

// ---------------------------------------------------------------------------------------------
// gate / up / SwiGLU

__device__ __noinline__ float trx_silu_mul(float g, float u) {
    const float e = trx_expf(-g);
    const float silu = __fdiv_rn(g, __fadd_rn(1.0f, e));
    return __fmul_rn(silu, u);
}

// Q4_K row of 8 blocks (2048 columns) by one warp: float(sum_s v_s) in every lane
template <bool SM>
__device__ __forceinline__ float trx_q4k_row8(const uint8_t *__restrict__ row, const TrxQ4X &X, int lane) {
    const int s = lane >> 2, c = lane & 3;
    const uint8_t *blk = row + 144 * s;
    const uint4 hdr = trx_ld<SM, uint4>(blk);
    const uint4 q0 = trx_ld<SM, uint4>(blk + 16 + 32 * c);
    const uint4 q1 = trx_ld<SM, uint4>(blk + 32 + 32 * c);
    int64_t T, M;
    trx_q4k_chunk(hdr, q0, q1, c, X, T, M);
    const double v = trx_q4k_value(hdr, T, M, X.sc);
    double y = 0.0;
#pragma unroll
    for (int i = 0; i < 8; i++) y = __dadd_rn(y, trx_shfl_d(v, 4 * i));
    return __double2float_rn(y);
}

// Two Q4_K rows of 8 blocks against the same input (a gate row and its up row), interleaved for ILP
template <bool SM>
__device__ __forceinline__ void trx_q4k_row8x2(const uint8_t *__restrict__ ra, const uint8_t *__restrict__ rb_,
                                               const TrxQ4X &X, int lane, float &ya, float &yb) {
    const int s = lane >> 2, c = lane & 3;
    const uint8_t *ba = ra + 144 * s, *bb = rb_ + 144 * s;
    const uint4 ha = trx_ld<SM, uint4>(ba), hb = trx_ld<SM, uint4>(bb);
    const uint4 a0 = trx_ld<SM, uint4>(ba + 16 + 32 * c), b0 = trx_ld<SM, uint4>(bb + 16 + 32 * c);
    const uint4 a1 = trx_ld<SM, uint4>(ba + 32 + 32 * c), b1 = trx_ld<SM, uint4>(bb + 32 + 32 * c);
    int64_t Ta, Ma, Tb, Mb;
    trx_q4k_chunk(ha, a0, a1, c, X, Ta, Ma);
    trx_q4k_chunk(hb, b0, b1, c, X, Tb, Mb);
    const double va = trx_q4k_value(ha, Ta, Ma, X.sc), vb = trx_q4k_value(hb, Tb, Mb, X.sc);
    double sa = 0.0, sb = 0.0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        sa = __dadd_rn(sa, trx_shfl_d(va, 4 * i));
        sb = __dadd_rn(sb, trx_shfl_d(vb, 4 * i));
    }
    ya = __double2float_rn(sa);
    yb = __double2float_rn(sb);
}

// N Q4_K rows of 8 blocks against the same input (a gate row and its up row, of one or two chunk rows), interleaved
// for ILP: y[i] = float(sum_s v_s) of row i in every lane
template <bool SM, int N>
__device__ __forceinline__ void trx_q4k_row8xn(const uint8_t *const (&rows)[N], const TrxQ4X &X, int lane, float (&y)[N]) {
    const int s = lane >> 2, c = lane & 3;
    uint4 hd[N], q0[N], q1[N];
#pragma unroll
    for (int i = 0; i < N; i++) {
        const uint8_t *b = rows[i] + 144 * s;
        hd[i] = trx_ld<SM, uint4>(b);
        q0[i] = trx_ld<SM, uint4>(b + 16 + 32 * c);
        q1[i] = trx_ld<SM, uint4>(b + 32 + 32 * c);
    }
    double v[N], acc[N];
#pragma unroll
    for (int i = 0; i < N; i++) {
        int64_t T, M;
        trx_q4k_chunk(hd[i], q0[i], q1[i], c, X, T, M);
        v[i] = trx_q4k_value(hd[i], T, M, X.sc);
        acc[i] = 0.0;
    }
#pragma unroll
    for (int j = 0; j < 8; j++)
#pragma unroll
        for (int i = 0; i < N; i++) acc[i] = __dadd_rn(acc[i], trx_shfl_d(v[i], 4 * j));
#pragma unroll
    for (int i = 0; i < N; i++) y[i] = __double2float_rn(acc[i]);
}

// Q4_K rows of 4 blocks (1024 columns), a half-warp each: the half's row value
template <bool SM>
__device__ __forceinline__ float trx_q4k_row4(const uint8_t *__restrict__ row, const TrxQ4X &X, int lane) {
    const int s = (lane >> 2) & 3, c = lane & 3;
    const uint8_t *blk = row + 144 * s;
    const uint4 hdr = trx_ld<SM, uint4>(blk);
    const uint4 q0 = trx_ld<SM, uint4>(blk + 16 + 32 * c);
    const uint4 q1 = trx_ld<SM, uint4>(blk + 32 + 32 * c);
    int64_t T, M;
    trx_q4k_chunk(hdr, q0, q1, c, X, T, M);
    const double v = trx_q4k_value(hdr, T, M, X.sc);
    double y = 0.0;
    const int base = lane & 16;
#pragma unroll
    for (int i = 0; i < 4; i++) y = __dadd_rn(y, trx_shfl_d(v, base + 4 * i));
    return __double2float_rn(y);
}

// the CTA's range of the virtual row space [a, b), V = n_active * rows_per_expert
__device__ __forceinline__ void trx_cta_range(int64_t V, int64_t &a, int64_t &b) {
    a = V * blockIdx.x / gridDim.x;
    b = V * (blockIdx.x + 1) / gridDim.x;
}

// on a timed-out wait: record it, wait (bounded) for this CTA's other copies in flight, leave
__device__ __forceinline__ void trx_bail(TrxWork &w, uint64_t *bar, int from, int issued) {
    if (threadIdx.x == 0) {
        atomicExch(w.err, 1);
        for (int q = from; q < issued; q++) trx_mbar_wait(&bar[q % TRX_STAGES], (q / TRX_STAGES) & 1, TRX_WAIT_NS);
    }
    __syncthreads();
}

// GT: Q4_K or Q8_0 (gate and up share it). Dynamic shared memory: TRX_STAGES * 2 * TRX_GU_CHUNK rows + barriers.
template <int GT, bool DOWN_LC>
__global__ void __launch_bounds__(256) trx_k_gateup(TrxLayer L, TrxShape S, TrxWork w) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float res[2][TRX_TOK_GROUP][TRX_GU_CHUNK];
    constexpr int CH = TRX_GU_CHUNK;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int H = S.H, F = S.F;
    const int rb = GT == TRX_Q4_K ? H / 256 * 144 : H / 32 * 34;
    const int half = CH * rb;
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + TRX_STAGES * 2 * half);
    const int n_act = *w.n_active;
    int64_t a, b;
    trx_cta_range((int64_t)n_act * F, a, b);
    if (tid == 0) {
        for (int s = 0; s < TRX_STAGES; s++) trx_mbar_init(&bar[s], 1);
        trx_fence_barrier_init();
    }
    __syncthreads();
    auto chunk_end = [&](int64_t v) { return min(min(v + CH, b), (v / F + 1) * F); };
    int64_t issue_v = a;
    int issued = 0;
    auto issue = [&]() { // thread 0
        const int64_t ve = chunk_end(issue_v);
        const int e = w.active[issue_v / F], r0 = (int)(issue_v % F), n = (int)(ve - issue_v);
        const int s = issued % TRX_STAGES;
        uint8_t *dst = smem + s * 2 * half;
        trx_mbar_expect_tx(&bar[s], 2u * n * rb);
        trx_bulk_g2s(dst, L.gate + e * L.gate_mb + (int64_t)r0 * rb, n * rb, &bar[s]);
        trx_bulk_g2s(dst + half, L.up + e * L.up_mb + (int64_t)r0 * rb, n * rb, &bar[s]);
        issue_v = ve;
        issued++;
    };
    if (tid == 0)
        for (int q = 0; q < TRX_STAGES && issue_v < b; q++) issue();
    int cur_t = -1;
    TrxQ4X X;
    int j = 0;
    for (int64_t v = a; v < b; j++) {
        const int64_t ve = chunk_end(v);
        const int e = w.active[v / F], r0 = (int)(v % F), n = (int)(ve - v);
        const int p0 = w.offsets[e], p1 = w.offsets[e + 1];
        const int s = j % TRX_STAGES;
        if (GT == TRX_Q4_K && warp < n && w.xmap[p0] != cur_t) { // the first row's input, while the copy lands
            cur_t = w.xmap[p0];
            trx_q4x_load(w.xq + (int64_t)cur_t * H, 32, lane, w.xq_bf + (int64_t)cur_t * (H / 32) + 8 * (lane >> 2),
                         w.xq_sc + (int64_t)cur_t * (H / 256) + (lane >> 2), X);
        }
        const bool ok = trx_mbar_wait(&bar[s], (j / TRX_STAGES) & 1, TRX_WAIT_NS);
        if (__syncthreads_or(!ok)) {
            trx_bail(w, bar, j, issued);
            return;
        }
        const uint8_t *gs = smem + s * 2 * half, *us = gs + half;
        for (int pg = p0; pg < p1; pg += TRX_TOK_GROUP) {
            const int ng = min(TRX_TOK_GROUP, p1 - pg);
            for (int q = 0; q < ng; q++) {
                const int t = w.xmap[pg + q];
                if (GT == TRX_Q4_K) {
                    if (warp < n) {
                        if (t != cur_t) {
                            cur_t = t;
                            trx_q4x_load(w.xq + (int64_t)t * H, 32, lane, w.xq_bf + (int64_t)t * (H / 32) + 8 * (lane >> 2),
                                         w.xq_sc + (int64_t)t * (H / 256) + (lane >> 2), X);
                        }
                        const float g = trx_q4k_row8<true>(gs + warp * rb, X, lane);
                        const float u = trx_q4k_row8<true>(us + warp * rb, X, lane);
                        if (lane == 0) {
                            res[0][q][warp] = g;
                            res[1][q][warp] = u;
                        }
                    }
                } else { // half-warp hw: row hw & 7 of matrix hw >> 3
                    const int hw = tid >> 4, row = hw & 7, mat = hw >> 3;
                    const float vv = trx_q8l_dot<true>((mat ? us : gs) + (row < n ? row : 0) * rb,
                                                       w.x_lc + (int64_t)t * H, H / 256, lane & 15);
                    if (row < n && (lane & 15) == 0) res[mat][q][row] = vv;
                }
            }
            __syncthreads();
            for (int i = tid; i < ng * n; i += blockDim.x) {
                const int q = i / n, row = i % n, r = r0 + row;
                w.h[(int64_t)(pg + q) * F + (DOWN_LC ? trx_lc_pos(r) : r)] = trx_silu_mul(res[0][q][row], res[1][q][row]);
            }
            __syncthreads();
        }
        if (tid == 0 && issue_v < b) { // stage s is free again
            trx_fence_proxy_async();
            issue();
        }
        v = ve;
    }
}

// ---------------------------------------------------------------------------------------------
// Q4_K down input: every h row prepared (one warp per (row, 256-block))
__global__ void __launch_bounds__(256) trx_k_prep(TrxShape S, int R, TrxWork w) {
    const int F = S.F, nsb = F / 256;
    const int lane = threadIdx.x & 31;
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int p = gw / nsb, s = gw % nsb;
    if (p >= R) return;
    trx_prep_q4x_block(w.h + (int64_t)p * F + 256 * s, w.hq + (int64_t)p * F, s, nsb, w.hq_bf + (int64_t)p * (F / 32) + 8 * s,
                       w.hq_sc + (int64_t)p * (F / 256) + s, lane);
}

// ---------------------------------------------------------------------------------------------
// down + combine + residual. DT: Q4_K (F == 1024), Q8_0 or Q6_K. Dynamic shared memory: TRX_STAGES *
// TRX_DN_CHUNK rows + barriers.
template <int DT>
__global__ void __launch_bounds__(256) trx_k_down(TrxLayer L, TrxShape S, TrxWork w, float *__restrict__ x_io, int T,
                                                  float *__restrict__ ffn_out) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int CH = TRX_DN_CHUNK;
    const int tid = threadIdx.x, lane = tid & 31, hw = tid >> 4;
    const int H = S.H, F = S.F, k = S.k, nsb = F / 256;
    const int rb = DT == TRX_Q4_K ? nsb * 144 : DT == TRX_Q6_K ? nsb * 208 : F / 32 * 34;
    const int stage = CH * rb;
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + TRX_STAGES * stage);
    __shared__ int s_last;
    const int n_act = *w.n_active;
    int64_t a, b;
    trx_cta_range((int64_t)n_act * H, a, b);
    if (tid == 0) {
        for (int s = 0; s < TRX_STAGES; s++) trx_mbar_init(&bar[s], 1);
        trx_fence_barrier_init();
    }
    __syncthreads();
    auto chunk_end = [&](int64_t v) { return min(b, (v / CH + 1) * CH); }; // H % CH == 0: never crosses an expert
    int64_t issue_v = a;
    int issued = 0;
    auto issue = [&]() {
        const int64_t ve = chunk_end(issue_v);
        const int e = w.active[issue_v / H], d0 = (int)(issue_v % H), n = (int)(ve - issue_v);
        const int s = issued % TRX_STAGES;
        trx_mbar_expect_tx(&bar[s], (uint32_t)(n * rb));
        trx_bulk_g2s(smem + s * stage, L.down + e * L.down_mb + (int64_t)d0 * rb, n * rb, &bar[s]);
        issue_v = ve;
        issued++;
    };
    if (tid == 0)
        for (int q = 0; q < TRX_STAGES && issue_v < b; q++) issue();
    int cur_p = -1;
    TrxQ4X X;
    int j = 0;
    for (int64_t v = a; v < b; j++) {
        const int64_t ve = chunk_end(v);
        const int e = w.active[v / H], d0 = (int)(v % H), n = (int)(ve - v);
        const int p0 = w.offsets[e], p1 = w.offsets[e + 1];
        const int s = j % TRX_STAGES;
        if (DT == TRX_Q4_K && hw < n && p0 != cur_p) {
            cur_p = p0;
            trx_q4x_load(w.hq + (int64_t)p0 * F, 16, lane & 15, w.hq_bf + (int64_t)p0 * (F / 32) + 8 * ((lane >> 2) & 3),
                         w.hq_sc + (int64_t)p0 * nsb + ((lane >> 2) & 3), X);
        }
        const bool ok = trx_mbar_wait(&bar[s], (j / TRX_STAGES) & 1, TRX_WAIT_NS);
        if (__syncthreads_or(!ok)) {
            trx_bail(w, bar, j, issued);
            return;
        }
        const uint8_t *st = smem + s * stage;
        const int row = hw < n ? hw : 0, d = d0 + row;
        for (int p = p0; p < p1; p++) {
            float vv;
            if (DT == TRX_Q4_K) {
                if (p != cur_p) {
                    cur_p = p;
                    trx_q4x_load(w.hq + (int64_t)p * F, 16, lane & 15, w.hq_bf + (int64_t)p * (F / 32) + 8 * ((lane >> 2) & 3),
                                 w.hq_sc + (int64_t)p * nsb + ((lane >> 2) & 3), X);
                }
                vv = trx_q4k_row4<true>(st + row * rb, X, lane);
            } else if (DT == TRX_Q8_0) {
                vv = trx_q8l_dot<true>(st + row * rb, w.h + (int64_t)p * F, nsb, lane & 15);
            } else {
                const uint8_t *dptr = L.down + e * L.down_mb + (int64_t)H * rb + (int64_t)d * nsb * 2;
                vv = trx_q6l_dot<true>(st + row * rb, dptr, w.h + (int64_t)p * F, nsb, lane & 15);
            }
            if (hw < n && (lane & 15) == 0) w.h3[(int64_t)p * H + d] = vv;
        }
        // count this chunk's rows into its combine block; the CTA completing the block combines it
        __threadfence();
        __syncthreads();
        const int blk = d0 / CH;
        if (tid == 0) {
            const unsigned old = atomicAdd(&w.comb_cnt[blk], (unsigned)n);
            s_last = old + (unsigned)n == (unsigned)(n_act * CH);
            if (issue_v < b) { // stage s is free again
                trx_fence_proxy_async();
                issue();
            }
        }
        __syncthreads();
        if (s_last) {
            __threadfence();
            for (int i = tid; i < T * CH; i += blockDim.x) {
                const int t = i / CH, dd = blk * CH + i % CH;
                float out = 0.0f;
                for (int sl = 0; sl < k; sl++) {
                    const int jj = t * k + sl;
                    out = __fadd_rn(out, __fmul_rn(w.sel_w[jj], __ldcg(w.h3 + (int64_t)w.place[jj] * H + dd)));
                }
                if (ffn_out) ffn_out[(int64_t)t * H + dd] = out;
                x_io[(int64_t)t * H + dd] = __fadd_rn(x_io[(int64_t)t * H + dd], out);
            }
            if (tid == 0) w.comb_cnt[blk] = 0u;
        }
        v = ve;
    }
}
