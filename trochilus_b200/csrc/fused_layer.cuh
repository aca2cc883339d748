// fused_layer.cuh: one MoE layer call for a short pass (decode) as ONE persistent kernel, launched
// cooperatively so that every CTA is resident and may wait for another.
//
//  routing  CTAs 0..E-1 compute the router logits of one expert each (trx_router_block); for calls of more than
//           TRX_FU_LOCAL_PREP tokens CTAs E..E+T-1 prepare one token's input row each, for shorter ones every CTA
//           prepares the inputs itself meanwhile; every writer counts itself in. Once all are in, every CTA reads
//           the logits, routes every token and sorts the (token, slot) rows by expert in its own shared memory (no
//           CTA publishes a routing for the others). Each CTA then takes its share of the routed gate/up rows and of
//           the routed down rows (whole chunks of each virtual row space).
//  then     warp-specialised: a producer warp streams this CTA's gate/up chunks (8 rows of gate and of up) and
//           down chunks (16 rows) from HBM into shared-memory stages with 1-D TMA bulk copies, refilling a stage
//           when its "empty" barrier says its consumers are done with it; the down weights do not depend on the
//           activations, so they stream while the gate/up rows are multiplied. The 8 consumer warps form two groups
//           that take the chunks in turn, each warp two rows of a chunk (two independent chains a warp), with no
//           block-wide barrier: gate/up rows (both matrices, SwiGLU), then the down rows of every chunk once its
//           expert's gate/up rows are all counted (acquire). Short calls (T <= TRX_FU_SEG_MAX) leave their values
//           in shared memory and the producer warp, idle while they multiply, finishes and publishes them: h =
//           silu(g) u per chunk, one fence and count per expert segment of the CTA (the count that completes an
//           expert prepares its Q4_K down inputs), h3 and one fence and count per down chunk. Longer calls publish
//           from the consumers, chunk by chunk.
//  mix      16-row block b is mixed by CTA b mod grid (its producer warp) once all its rows are counted: every
//           token's k expert outputs added in increasing expert id, the sum added to the residual (Trochilus's
//           mix_body).
//  end      the last CTA resets the per-expert counters for the next call and, for the host-pointer road, posts
//           the call's epoch to a pinned host word once every output is visible.
//
// Every wait is bounded (TRX_SPIN_NS, TRX_WAIT_NS); a warp that gives up marks the CTA failed, the producer
// waits (bounded) for every copy it armed, the error flag is set and the CTA leaves. The counters a failed call
// leaves behind are reset by the host (tr_gpu_moe_check, and the host-pointer call on an error).
//
// Trochilus references: forward_layer's MoE block src/models/olmoe.c:1845-1933 (route_token :1455-1502, the
// counting sort :1850-1861, expert_stages :1642-1689, mix_body :1432-1446).
#pragma once
#include <cstdint>
#include "bulk.cuh"
#include "moe_kernels.cuh"
#include "ep.cuh"

#define TRX_SPIN_NS 1000000000ull
#define TRX_FU_CWARPS 8                           // consumer warps
#define TRX_FU_GW (TRX_FU_CWARPS / 2)             // consumer warps a group (two groups take the chunks in turn)
#define TRX_FU_HWARP (TRX_FU_CWARPS + 1)          // the warp that copies short calls' h rows into the down stages
#define TRX_FU_THREADS (32 * (TRX_FU_CWARPS + 2)) // + the producer warp and that one
#define TRX_FU_MAXST 8                            // most stages of either kind
#define TRX_FU_LOCAL_PREP 8                       // tokens up to which every CTA prepares the inputs itself

struct TrxSync {
    uint32_t route_cnt;                // router and prep CTAs done in this call
    uint32_t seq;                      // the one-token kernel's call count: its exchanged words carry seq + 1
    uint32_t finish;                   // CTAs done in this call
    uint32_t pad;
    uint32_t gu_done[TRX_MAX_EXPERTS]; // gate/up rows done per active slot (+1 once Q4_K's down inputs are ready)
};

__device__ __forceinline__ uint32_t trx_ld_acquire(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void trx_st_release(uint32_t *p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// the call's completion word in host memory (after a system-scope fence, so that what came before is visible first)
__device__ __forceinline__ void trx_post_done(uint32_t *word, uint32_t v) {
    __threadfence_system();
    asm volatile("st.volatile.global.u32 [%0], %1;" ::"l"(word), "r"(v) : "memory");
}

__device__ __forceinline__ void trx_mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(trx_smem(bar)) : "memory");
}

// thread-level bounded wait: *p == target (eq) or *p >= target
__device__ __forceinline__ bool trx_spin(const uint32_t *p, uint32_t target, bool eq) {
    uint64_t t0 = 0;
    for (int it = 0;; it++) {
        const uint32_t v = trx_ld_acquire(p);
        if (eq ? v == target : v >= target) return true;
        if (it == 0) t0 = trx_globaltimer();
        else if (trx_globaltimer() - t0 > TRX_SPIN_NS) return false;
        __nanosleep(20);
    }
}

// A CTA's walk over its share of a virtual row space of n_active experts x per rows, in chunks of at most `most`
// rows that stay inside one expert.
//  slot-major (longer calls): the CTA's range [v, end) of the space, chunks aligned to `most`-row blocks when asked;
//           when `most` divides `per` the CTAs share whole chunks. Each expert's rows are done by a few CTAs.
//  expert-major (short calls): the CTA's rows [ra, rb) of EVERY expert (a multiple of `gran` rows), experts in
//           order; the experts are then finished one after another across the grid, and a CTA holds every expert's
//           contribution to its rows. v counts the CTA's rows from 0.
// int32: the spaces hold at most 64 x 2048 rows.
struct TrxWalk {
    int v, end, slot, r, per, most, ra, rb;
    bool aligned, em;
    __device__ void init(int V, int per_, int most_, bool aligned_, bool em_ = false, int gran = 1) {
        per = per_;
        most = most_;
        aligned = aligned_;
        em = em_;
        if (em) { // 32-bit arithmetic: per x grid stays far below 2^32
            const uint32_t units = (uint32_t)(per / gran);
            ra = (int)(units * blockIdx.x / gridDim.x) * gran;
            rb = blockIdx.x + 1 == gridDim.x ? per : (int)(units * (blockIdx.x + 1) / gridDim.x) * gran;
            slot = 0;
            r = ra;
            v = 0;
            end = (V / per) * (rb - ra);
            return;
        }
        uint32_t a, b; // 32-bit: V x grid stays below 2^32 (V <= 64 x 2048)
        const uint32_t units = per_ % most_ == 0 ? (uint32_t)(V / most_) : (uint32_t)V; // whole chunks, or rows
        a = units * blockIdx.x / gridDim.x;
        b = units * (blockIdx.x + 1) / gridDim.x;
        if (per_ % most_ == 0) { // whole chunks: the CTAs' shares differ by one chunk at most, none is partial
            a *= most_;
            b *= most_;
        }
        v = (int)a;
        end = (int)b;
        ra = 0;
        rb = per;
        slot = v / per;
        r = v - slot * per;
    }
    __device__ bool more() const { return v < end; }
    __device__ int n() const {
        if (em) return min(most, rb - r);
        return min(min(aligned ? most - r % most : most, end - v), per - r);
    }
    // whether the current chunk is the CTA's last of its expert
    __device__ bool seg_end() const { return r + n() == rb || v + n() == end; }
    __device__ void next() {
        const int k = n();
        v += k;
        r += k;
        if (r == rb) {
            r = ra;
            slot++;
        }
    }
};

// The fused kernel's dynamic shared memory: the stage buffers (the router phase reuses them), the barriers,
// the call's routing (xmap, sel_w, place, sel_id: R = T k entries each), then the tokens' prepared input rows
// (Q4_K: planes, sums, scales; Q8_0: the LC-ordered row), each region 128-byte aligned.
struct TrxFusedSmem {
    size_t gu_stage, dn_stage, bars, meta, seg, tok, tok_bytes, total;
};

#define TRX_FU_SEG_MAX 4 // tokens up to which a CTA keeps its h values in shared memory and publishes once an expert

// the most gate/up rows one CTA of `grid` takes (whole chunks, or its rows of every expert)
__host__ __device__ inline int trx_fu_rows_g(int E, int k, int T, int F, int grid) {
    const int act = E < T * k ? E : T * k, units = act * F / TRX_GU_CHUNK;
    const int whole = (units + grid - 1) / grid * TRX_GU_CHUNK, em = act * ((F + grid - 1) / grid + 1);
    return whole > em ? whole : em;
}

// short calls: the row granularity of the expert-major down walk (its chunks' Q6_K d values are whole 16-byte
// pieces), and the most down rows a CTA takes of one expert
__host__ __device__ inline int trx_fu_dn_gran(int down_type, int F) {
    return down_type == TRX_Q6_K && F / 256 < 8 ? 8 / (F / 256) : 1;
}
__host__ __device__ inline int trx_fu_rows_d(int down_type, int H, int F, int grid) {
    const int g = trx_fu_dn_gran(down_type, F);
    return (H / g + grid - 1) / grid * g + g;
}


__host__ __device__ inline size_t trx_align128(size_t v) { return (v + 127) / 128 * 128; }

__host__ __device__ inline TrxFusedSmem trx_fused_layout(int gate_type, int down_type, int H, int F, int T, int k, int sg,
                                                         int sd, int E, int grid) {
    const int rbg = gate_type == TRX_Q4_K ? H / 256 * 144 : H / 32 * 34;
    const int rbd = down_type == TRX_Q4_K ? F / 256 * 144 : down_type == TRX_Q6_K ? F / 256 * 208 : F / 32 * 34;
    TrxFusedSmem l;
    l.gu_stage = (size_t)2 * TRX_GU_CHUNK * rbg;
    // Q6_K: the rows' f16 d values (stored after all rows of the matrix) come with them, the 16-row block's
    l.dn_stage = (size_t)TRX_DN_CHUNK * rbd + (down_type == TRX_Q6_K ? (size_t)TRX_DN_CHUNK * (F / 256) * 2 : 0);
    // short calls: the h rows of the chunk's expert come with its weights (not for the Q4_K down, which reads its
    // prepared inputs from L2)
    if (T <= TRX_FU_SEG_MAX && down_type != TRX_Q4_K) l.dn_stage += (size_t)T * F * 4;
    size_t stages = sg * l.gu_stage + sd * l.dn_stage;
    const size_t router = (size_t)(1 + (T < TRX_TOK_STAGE ? T : TRX_TOK_STAGE)) * H * 4;
    if (router > stages) stages = router;
    l.bars = trx_align128(stages);
    l.meta = trx_align128(l.bars + 8 * 4 * TRX_FU_MAXST);
    l.seg = trx_align128(l.meta + (size_t)T * k * 16);
    // short calls: (g, u) of the CTA's gate/up rows, then h3 of its down rows for every grouped row
    const size_t seg_bytes = T <= TRX_FU_SEG_MAX ? (size_t)2 * trx_fu_rows_g(E, k, T, F, grid) * T * 4 +
                                                       (size_t)T * k * trx_fu_rows_d(down_type, H, F, grid) * 4
                                                 : 0;
    l.tok = trx_align128(l.seg + seg_bytes);
    l.tok_bytes = gate_type == TRX_Q4_K ? trx_align128((size_t)H * 4 + (size_t)(H / 32 + H / 256) * 8) : (size_t)H * 4;
    // the tokens' prepared inputs stay in shared memory for short calls (prepared there); longer ones read them from
    // L2, where the prep CTAs wrote them
    l.total = l.tok + (T <= TRX_FU_LOCAL_PREP ? (size_t)T * l.tok_bytes : 0);
    return l;
}

// The routing phase's use of the stage area (free until the barriers): the router's staging ((1 + min(T, 16))
// rows of H floats), the logits' slot, then the routing warm-up's 4 KB of scratch, then (norm_in) the call's
// normalised rows. The offset of those rows; the fused norm needs them to end before the barriers.
__host__ __device__ inline size_t trx_fu_norm_off(int T, int H, int E) {
    const size_t wscr = trx_align128((size_t)(1 + (T < TRX_TOK_STAGE ? T : TRX_TOK_STAGE)) * H * 4 + (size_t)T * E * 4);
    return trx_align128(wscr + 4096);
}

#define TRX_TRACE(slot)                                                                                                \
    do {                                                                                                               \
        if (w.trace != nullptr && threadIdx.x == 0) w.trace[(size_t)blockIdx.x * 64 + (slot)] = trx_globaltimer();     \
    } while (0)

template <int GT, int DT>
__global__ void __launch_bounds__(TRX_FU_THREADS, 1)
    trx_k_layer(TrxLayer L, TrxShape S, const float *__restrict__ normed, int T, TrxWork w, TrxSync *sync,
                float *__restrict__ x_io, float *__restrict__ ffn_out, uint32_t epoch, int SG, int SD) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_active[TRX_MAX_EXPERTS], s_off[TRX_MAX_EXPERTS + 1], s_nact, s_flag;
    __shared__ int s_pact[TRX_MAX_EXPERTS]; // the producer's copy of the active experts
    __shared__ __align__(16) float sp[TRX_FU_CWARPS + 2][96]; // per-warp scratch (16-byte aligned rows)
    __shared__ int s_armed; // down chunks whose stage the producer has armed (read by the h-copy warp)
    __shared__ int scnt[64];
    __shared__ uint32_t s_gcnt[TRX_FU_MAXST], s_dcnt[TRX_FU_MAXST];
    constexpr int CHG = TRX_GU_CHUNK, CHD = TRX_DN_CHUNK;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int E = S.E, H = S.H, F = S.F, k = S.k, nsb_d = F / 256, R = T * k;
    TRX_TRACE(0);
    const long long ck0 = clock64();
#define TRX_CYC(slot)                                                                                                  \
    do {                                                                                                               \
        if (w.trace != nullptr && threadIdx.x == 0) w.trace[(size_t)blockIdx.x * 64 + (slot)] = clock64() - ck0;      \
    } while (0)
    const int rbg = GT == TRX_Q4_K ? H / 256 * 144 : H / 32 * 34;
    const int rbd = DT == TRX_Q4_K ? nsb_d * 144 : DT == TRX_Q6_K ? nsb_d * 208 : F / 32 * 34;
    const TrxFusedSmem lay = trx_fused_layout(GT, DT, H, F, T, k, SG, SD, E, gridDim.x);
    const int gu_half = CHG * rbg;
    uint8_t *gu_buf = smem, *dn_buf = smem + SG * lay.gu_stage;
    uint64_t *full_g = reinterpret_cast<uint64_t *>(smem + lay.bars), *empty_g = full_g + TRX_FU_MAXST;
    uint64_t *full_d = empty_g + TRX_FU_MAXST, *empty_d = full_d + TRX_FU_MAXST;
    int *s_xmap = reinterpret_cast<int *>(smem + lay.meta);
    float *s_selw = reinterpret_cast<float *>(s_xmap + R);
    int *s_place = reinterpret_cast<int *>(s_selw + R);
    int *s_selid = s_place + R;
    uint8_t *s_tok = smem + lay.tok;
    if (tid < TRX_FU_MAXST) s_gcnt[tid] = s_dcnt[tid] = 0u;
    if (tid == 0) s_armed = 0;
    const int nsb_g = H / 256;
    if (tid == 0) { // the pipelines' barriers (their region is not scratch for the routing phase)
        for (int s = 0; s < SG; s++) {
            trx_mbar_init(&full_g[s], 1);
            trx_mbar_init(&empty_g[s], TRX_FU_GW);
        }
        for (int s = 0; s < SD; s++) {
            trx_mbar_init(&full_d[s], 1);
            trx_mbar_init(&empty_d[s], TRX_FU_GW);
        }
        trx_fence_barrier_init();
    }
    if (warp == 1) trx_expf_prefetch(lane); // the softmax's table, before the routing needs it
    // Short calls: the producer warp mixes this CTA's down rows [mra, mrb) of every token (below); their residual
    // values are read now, so that the read (from host memory, in the host-pointer road) is over long before the mix
    const bool seg = T <= TRX_FU_SEG_MAX;
    const int dgran = trx_fu_dn_gran(DT, F), nrmax = trx_fu_rows_d(DT, H, F, gridDim.x);
    int mra, mrb;
    {
        TrxWalk mw;
        mw.init(H, H, CHD, true, true, dgran);
        mra = mw.ra;
        mrb = mw.rb;
    }
    float xpre[2] = {0.0f, 0.0f};
    if (seg && warp == TRX_FU_CWARPS && !S.ext)
#pragma unroll
        for (int q = 0; q < 2; q++) {
            const int i = lane + 32 * q, nr = mrb - mra;
            if (i < nr * T) xpre[q] = x_io[(int64_t)(i / nr) * H + mra + i % nr];
        }

    {
        // ---------------- phase A: CTAs 0..E-1 the logits of one expert each; the tokens' prepared inputs either
        // by every CTA for itself into shared memory (T <= TRX_FU_LOCAL_PREP: from normed, while the logits are
        // computed elsewhere) or by CTAs E..E+T-1 into global memory; every CTA that wrote counts itself in (release)
        // norm_in (short calls, the ffn_norm in the hook): every CTA first normalises the call's residual rows into
        // its shared memory, warp t token t: the row in, lanes 0-15 the lane contract's sum of squares (tree-joined),
        // inv = 1 / sqrtf(sumsq / H + eps), then normed = (x inv) w in place (Trochilus's tr_rmsnorm,
        // src/kernels/kernels.c:1351-1360); CTA 0 also writes them out when asked. The routing phase reads them there.
        // ext over peer memory: every source rank's rows of this step must have arrived (its flag holds the epoch)
        if (w.ep) {
            int why = 0;
            if (tid == 0) {
                const TrxEpHdr *own = reinterpret_cast<const TrxEpHdr *>(w.ep->base[w.ep->rank]);
                s_flag = trx_ep_wait_flags(own->recv_flag, w.ep->n, own->epoch, TRX_EP_WAIT_NS, &why);
            }
            __syncthreads();
            if (!s_flag) {
                if (tid == 0) atomicCAS(w.err, 0, 7 | why); // the first error stays
                return;
            }
        }
        const float *nin = normed;
        if (S.norm_in) {
            float *sn = reinterpret_cast<float *>(smem + trx_fu_norm_off(T, H, E));
            for (int t = warp; t < T; t += TRX_FU_CWARPS + 2) {
                const float *xr = normed + (int64_t)t * H;
                float *row = sn + (size_t)t * H;
                for (int base = 0; base < H; base += 32 * 4 * 8) { // 8 loads a lane in flight
                    float4 v[8];
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const int i = base + (j * 32 + lane) * 4;
                        v[j] = i < H ? __ldcg(reinterpret_cast<const float4 *>(xr + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const int i = base + (j * 32 + lane) * 4;
                        if (i < H) *reinterpret_cast<float4 *>(row + i) = v[j];
                    }
                }
                __syncwarp();
                float acc = 0.0f;
                if (lane < 16)
                    for (int kk = lane; kk < H; kk += 16) acc = __fadd_rn(acc, __fmul_rn(row[kk], row[kk]));
                acc = trx_lane_tree16(acc); // lanes 16-31 join with zeros; lane 0 holds the sum
                const float inv =
                    __shfl_sync(0xffffffffu, __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, (float)H), L.norm_eps))), 0);
                for (int base = 0; base < H; base += 32 * 4 * 8) {
                    float4 wv[8];
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const int i = base + (j * 32 + lane) * 4;
                        wv[j] = i < H ? __ldg(reinterpret_cast<const float4 *>(L.norm_w + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const int i = base + (j * 32 + lane) * 4;
                        if (i < H) {
                            float4 *p = reinterpret_cast<float4 *>(row + i);
                            const float4 xv = *p;
                            *p = make_float4(__fmul_rn(__fmul_rn(xv.x, inv), wv[j].x), __fmul_rn(__fmul_rn(xv.y, inv), wv[j].y),
                                             __fmul_rn(__fmul_rn(xv.z, inv), wv[j].z), __fmul_rn(__fmul_rn(xv.w, inv), wv[j].w));
                        }
                    }
                }
            }
            __syncthreads();
            if (blockIdx.x == 0 && w.out_normed)
                for (int i = tid; i < T * H; i += blockDim.x) w.out_normed[i] = sn[i];
            nin = sn;
        }
        const bool lprep = T <= TRX_FU_LOCAL_PREP;
        const int nrc = S.ext ? 0 : E; // router CTAs (none when the rows come routed)
        const int writers = nrc + (lprep ? 0 : T);
        // short calls: the router CTAs compute the logits with warps 0-3 only, while the others prepare the inputs
        // and warm up the routing code (below)
        const int rthr = lprep ? 128 : 0, w0 = (int)blockIdx.x < nrc && rthr ? rthr / 32 : 0;
        if ((int)blockIdx.x < writers && (rthr == 0 || tid < rthr)) {
            if ((int)blockIdx.x < nrc)
                trx_router_block(L, S, nin, blockIdx.x, 0, T, w, reinterpret_cast<float *>(smem), rthr);
            else trx_prep_token(L, S, normed, blockIdx.x - nrc, w); // (norm_in is for short calls only)
            if (rthr) asm volatile("bar.sync 3, %0;" ::"r"(rthr) : "memory");
            else __syncthreads();
            TRX_TRACE(62);
            if (tid == 0) {
                __threadfence();
                atomicAdd(&sync->route_cnt, 1u);
            }
        }
        if (lprep && warp >= w0) {
            if (GT == TRX_Q4_K) {
                for (int q = warp - w0; q < T * nsb_g; q += TRX_FU_CWARPS + 2 - w0) {
                    const int t = q / nsb_g, s4 = q % nsb_g;
                    uint8_t *tok = s_tok + t * lay.tok_bytes;
                    double *bfd = reinterpret_cast<double *>(tok + (size_t)H * 4);
                    trx_prep_q4x_block(nin + (int64_t)t * H + 256 * s4, reinterpret_cast<uint32_t *>(tok), s4, nsb_g,
                                       bfd + 8 * s4, bfd + H / 32 + s4, lane);
                }
            } else {
                for (int i = tid - 32 * w0; i < T * H / 4; i += blockDim.x - 32 * w0) {
                    const int t = (4 * i) / H, kk = (4 * i) % H;
                    const float4 v = *reinterpret_cast<const float4 *>(nin + (int64_t)t * H + kk);
                    float *dst = reinterpret_cast<float *>(s_tok + t * lay.tok_bytes);
                    dst[trx_lc_pos(kk)] = v.x;
                    dst[trx_lc_pos(kk + 1)] = v.y;
                    dst[trx_lc_pos(kk + 2)] = v.z;
                    dst[trx_lc_pos(kk + 3)] = v.w;
                }
            }
        }
        // While the logits come in, warp 4 (on warp 0's sub-partition) runs the routing steps once on dummy logits,
        // so that the instructions warp 0 runs next are in the SM's instruction caches (run once per call, they
        // would otherwise be fetched cold from L2 line by line)
        // the routing warm-up's scratch: past the router's staging (in use meanwhile) and the logits' slot
        const size_t wscr = trx_align128((size_t)(1 + (T < TRX_TOK_STAGE ? T : TRX_TOK_STAGE)) * H * 4 + (size_t)T * E * 4);
        if (warp == 4 && !S.ext && wscr + 4096 <= lay.bars) {
            float *dl = reinterpret_cast<float *>(smem + wscr);
            int32_t *di = reinterpret_cast<int32_t *>(dl + 64);
            float *dw = dl + 128;
            for (int j = lane; j < 64; j += 32) dl[j] = 0.0f;
            __syncwarp();
            trx_route_token<true>(dl, E, k, S.norm_topk, lane, sp[warp], di, dw);
            __syncwarp();
            if (T == 1) { // and the single-token sort, into dummy arrays after them
                int32_t *dsort = di + 64;
                trx_sort_single(di, E, k, TrxSortOut{dsort, dsort + 72, dsort + 144, dsort + 152, dsort + 224, nullptr, nullptr},
                                lane);
            }
        }
        // ---------------- phase B: every CTA, once all writers are in (acquire), routes and sorts the whole call
        // itself from the logits in L2 (no CTA publishes for the others), and stages the tokens' inputs
        if (tid == 0) s_flag = trx_spin(&sync->route_cnt, (uint32_t)writers, false);
        __syncthreads();
        if (!s_flag) {
            if (tid == 0) {
                atomicExch(w.err, 2);
                if (w.host_done) trx_post_done(w.host_done, epoch | 0x80000000u);
            }
            return;
        }
        TRX_TRACE(1);
        TRX_CYC(53);
        float *slog = reinterpret_cast<float *>(smem); // T x E logits (the stage buffers are free until the barriers)
        if (S.ext) { // routed elsewhere: row t to expert ext_ids[t] alone, weight 1
            for (int j = tid; j < T; j += blockDim.x) {
                s_selid[j] = __ldcg(w.ext_ids + j);
                s_selw[j] = 1.0f;
            }
        } else {
            for (int j = tid; j < T * E; j += blockDim.x) slog[j] = __ldcg(w.logits + j);
        }
        __syncthreads();
        TRX_CYC(54);
        const long long c1 = clock64();
        for (int t = warp; !S.ext && t < T; t += TRX_FU_CWARPS + 2)
            trx_route_token<true>(slog + t * E, E, k, S.norm_topk, lane, sp[warp], s_selid + t * k, s_selw + t * k);
        if (w.trace != nullptr && tid == 0) w.trace[(size_t)blockIdx.x * 64 + 7] = (uint64_t)(clock64() - c1);
        trx_fence_proxy_async(); // the routing's writes to the stage area, before the copies that land there
        __syncthreads();
    }
    TRX_TRACE(60);
    TRX_CYC(55);
    // Both roads: s_selid / s_selw hold the call's routing. The producer derives the active experts from the ids and
    // starts streaming at once; the consumers sort the rows by expert, write the optional outputs and stage the
    // tokens' prepared inputs meanwhile; all meet at bar 1 once the producer's first copies are out.
    const bool lprep = T <= TRX_FU_LOCAL_PREP;
    int n_act;
    if (warp == TRX_FU_CWARPS) {
        if (w.trace != nullptr && lane == 0) w.trace[(size_t)blockIdx.x * 64 + 49] = trx_globaltimer(); // producer on
        uint32_t m0 = 0, m1 = 0; // the selected experts as a 64-bit set
        for (int j = lane; j < R; j += 32) {
            const int e = s_selid[j];
            if (e < 0) continue; // (a row routed nowhere)
            if (e < 32) m0 |= 1u << e;
            else m1 |= 1u << (e - 32);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            m0 |= __shfl_xor_sync(0xffffffffu, m0, o);
            m1 |= __shfl_xor_sync(0xffffffffu, m1, o);
        }
        n_act = __popc(m0) + __popc(m1);
        const unsigned lt = (1u << lane) - 1u;
        if (m0 >> lane & 1u) s_pact[__popc(m0 & lt)] = lane;
        if (m1 >> lane & 1u) s_pact[__popc(m0) + __popc(m1 & lt)] = lane + 32;
        __syncwarp();
        if (w.trace != nullptr && lane == 0) w.trace[(size_t)blockIdx.x * 64 + 61] = trx_globaltimer(); // mask done
    } else if (warp < TRX_FU_CWARPS) {
        const int ctid = tid; // 0..255
        if (warp == 0) {
            const bool out = blockIdx.x == 0;
            const TrxSortOut so{s_off, s_active, &s_nact, s_place, s_xmap, out ? w.out_offsets : nullptr,
                                out ? w.out_place : nullptr};
            TRX_CYC(56);
            const long long c0 = clock64();
            if (T == 1 && !S.ext) {
                trx_sort_single(s_selid, E, k, so, lane);
            } else {
                trx_warp_counting_sort(s_selid, R, E, k, so, scnt, lane);
            }
            if (w.trace != nullptr && lane == 0) w.trace[(size_t)blockIdx.x * 64 + 63] = (uint64_t)(clock64() - c0);
            TRX_TRACE(48);
            TRX_CYC(57);
        } else if (blockIdx.x == 0 && w.out_sel_id) {
            for (int j = ctid - 32; j < R; j += 32 * (TRX_FU_CWARPS - 1)) {
                w.out_sel_id[j] = s_selid[j];
                w.out_sel_w[j] = s_selw[j];
            }
        }
        asm volatile("bar.sync 1, %0;" ::"n"(32 * TRX_FU_CWARPS) : "memory");        // the consumers: sorted
        asm volatile("bar.arrive 2, %0;" ::"n"(TRX_FU_THREADS) : "memory");          // tell the producer
        n_act = s_nact;
        TRX_TRACE(2);
        TRX_CYC(58);
    }
    bool failed = false;
    int issued_g = 0, issued_d = 0; // the producer's counts, for the drain after a failure
    // Short calls (seg): the consumers leave the gate and up values (g, u) and the down values h3 in shared memory
    // and release the stage; the producer warp, idle while they multiply, finishes and publishes them: per gate/up
    // chunk h = silu(g) u, one row a lane, written out, and one device-scope fence and count per expert segment of
    // this CTA; per down chunk h3 written out, one fence and count, and the mix of a 16-row block when its count
    // completes. Longer calls: the consumers finish and publish themselves, chunk by chunk.
    float2 *sgu = reinterpret_cast<float2 *>(smem + lay.seg); // [row of the CTA's gate/up rows][token]: (g, u)
    float *sh3 = reinterpret_cast<float *>(sgu + (size_t)trx_fu_rows_g(E, k, T, F, gridDim.x) * T); // [grouped row][row]
    // short calls, Q8_0 / Q6_K down: the chunk's h rows come into the stage (after the weights and d values)
    const bool hcopy = seg && DT != TRX_Q4_K;
    const int hoff = TRX_DN_CHUNK * rbd + (DT == TRX_Q6_K ? TRX_DN_CHUNK * nsb_d * 2 : 0);
    const uint32_t need = (uint32_t)F + (DT == TRX_Q4_K ? 1u : 0u); // an expert's count once its h is complete
    // where token t's output row goes: ffn_out, or (ext over peer memory) its source rank's region, at [this rank]
    // [its slot]; NULL: nowhere (no ffn_out, or a padding row)
    auto out_row = [&](int t) -> float * {
        if (w.ep == nullptr) return ffn_out ? ffn_out + (int64_t)t * H : nullptr;
        if (s_selid[t] < 0) return nullptr;
        const TrxEpPeers *P = w.ep;
        return reinterpret_cast<float *>(P->base[t / P->cap] + P->off_back) + ((size_t)P->rank * P->cap + t % P->cap) * H;
    };
    // longer calls: the mix of a completed 16-row block (one warp): every token's k outputs in increasing expert id,
    // then the residual
    auto combine = [&](int blk) {
        __threadfence();
        for (int i = lane; i < T * CHD; i += 32) {
            const int t = i / CHD, dd = blk * CHD + i % CHD;
            float out = 0.0f;
            for (int sl = 0; sl < k; sl++) {
                const int jj = t * k + sl;
                if (s_selid[jj] < 0) continue; // (a row routed nowhere)
                out = __fadd_rn(out, __fmul_rn(s_selw[jj], __ldcg(w.h3 + (int64_t)s_place[jj] * H + dd)));
            }
            if (float *o = out_row(t)) o[dd] = out;
            if (!S.ext) x_io[(int64_t)t * H + dd] = __fadd_rn(x_io[(int64_t)t * H + dd], out);
        }
        if (lane == 0) w.comb_cnt[blk] = 0u;
    };

    if (warp == TRX_FU_CWARPS) {
        // ---------------- the producer: every chunk of this CTA, in consumption order (the copies by lane 0; the
        // publication by the whole warp)
        TrxWalk gw, dw; // the next chunk to copy
        gw.init(n_act * F, F, CHG, false, seg);
        dw.init(n_act * H, H, CHD, true, seg, dgran);
        auto issue_g = [&](int s) {
            if (lane == 0) {
                const int e = s_pact[gw.slot], n = gw.n();
                uint8_t *dst = gu_buf + s * lay.gu_stage;
                trx_mbar_expect_tx(&full_g[s], 2u * n * rbg);
                trx_bulk_g2s(dst, L.gate + e * L.gate_mb + (int64_t)gw.r * rbg, n * rbg, &full_g[s]);
                trx_bulk_g2s(dst + gu_half, L.up + e * L.up_mb + (int64_t)gw.r * rbg, n * rbg, &full_g[s]);
            }
        };
        // a down chunk's weights and Q6_K d values (those of its rows: the expert-major chunks start and end on
        // whole 16-byte pieces of them; else those of its 16-row block); with hcopy the stage also waits for the
        // expert's h rows, copied by the h-copy warp once the expert is complete
        auto issue_d = [&](int s) {
            if (lane == 0) {
                const int e = s_active[dw.slot], n = dw.n();
                const int drow = seg ? dw.r : dw.r / CHD * CHD, dbytes = DT == TRX_Q6_K ? (seg ? n : CHD) * nsb_d * 2 : 0;
                const int hbytes = hcopy ? (s_off[e + 1] - s_off[e]) * F * 4 : 0;
                trx_mbar_expect_tx(&full_d[s], (uint32_t)(n * rbd + dbytes + hbytes));
                trx_bulk_g2s(dn_buf + s * lay.dn_stage, L.down + e * L.down_mb + (int64_t)dw.r * rbd, n * rbd, &full_d[s]);
                if (DT == TRX_Q6_K)
                    trx_bulk_g2s(dn_buf + s * lay.dn_stage + CHD * rbd,
                                 L.down + e * L.down_mb + (int64_t)H * rbd + (int64_t)drow * nsb_d * 2, dbytes, &full_d[s]);
            }
        };
        auto wait_all = [&](uint64_t *bar, int parity) {
            return __all_sync(0xffffffffu, trx_mbar_wait(bar, parity, TRX_WAIT_NS));
        };
        if (w.trace != nullptr && lane == 0) w.trace[(size_t)blockIdx.x * 64 + 51] = trx_globaltimer(); // walks set
        for (; issued_g < SG && gw.more(); issued_g++, gw.next()) issue_g(issued_g);
        if (w.trace != nullptr && lane == 0) w.trace[(size_t)blockIdx.x * 64 + 3] = trx_globaltimer(); // copies out
        asm volatile("bar.sync 2, %0;" ::"n"(TRX_FU_THREADS) : "memory"); // the routing is sorted
        // the down weights only after this CTA's first gate/up stages have landed: every CTA's gate/up data then
        // comes first out of HBM, and the down data streams while the gate/up rows are multiplied
        for (int q = 0; q < issued_g && !failed; q++)
            if (!wait_all(&full_g[q], 0)) failed = true;
        for (; !failed && issued_d < SD && dw.more(); issued_d++, dw.next()) issue_d(issued_d);
        if (lane == 0) *(volatile int *)&s_armed = issued_d;
        // gate/up chunks in order: wait for the consumers, publish (seg), refill the stage
        TrxWalk pw;
        pw.init(n_act * F, F, CHG, false, seg);
        const int gv0 = pw.v;
        int seg_v0 = pw.v, seg_slot = pw.slot;
        for (int j = 0; !failed && pw.more(); j++, pw.next()) {
            const int s = j % SG, slot = pw.slot, n = pw.n();
            if (slot != seg_slot) {
                seg_slot = slot;
                seg_v0 = pw.v;
            }
            if (!wait_all(&empty_g[s], (j / SG) & 1)) {
                failed = true;
                break;
            }
            if (seg) {
                const int e = s_active[slot], p0 = s_off[e], np = s_off[e + 1] - p0;
                for (int i = lane; i < n * np; i += 32) {
                    const int rr = i / np, pp = i % np, r = pw.r + rr;
                    const float2 gu = sgu[(pw.v - gv0 + rr) * T + pp];
                    w.h[(int64_t)(p0 + pp) * F + (DT != TRX_Q4_K ? trx_lc_pos(r) : r)] = trx_silu_mul(gu.x, gu.y);
                }
            }
            if (seg && pw.seg_end()) { // this chunk ends the CTA's segment of the expert
                const int e = s_active[slot], p0 = s_off[e], np = s_off[e + 1] - p0, rows = pw.v + n - seg_v0;
                __syncwarp();
                uint32_t old = 0;
                if (lane == 0) {
                    __threadfence(); // the segment's h before its count
                    old = atomicAdd(&sync->gu_done[slot], (uint32_t)rows);
                }
                old = __shfl_sync(0xffffffffu, old, 0);
                if (DT == TRX_Q4_K && old + (uint32_t)rows == (uint32_t)F) {
                    // the expert's last rows: its h is complete; prepare it for the down's integer definition,
                    // then count once more
                    __threadfence();
                    for (int p = p0; p < p0 + np; p++)
                        for (int s4 = 0; s4 < nsb_d; s4++)
                            trx_prep_q4x_block<true>(w.h + (int64_t)p * F + 256 * s4, w.hq + (int64_t)p * F, s4, nsb_d,
                                                     w.hq_bf + (int64_t)p * (F / 32) + 8 * s4, w.hq_sc + (int64_t)p * nsb_d + s4,
                                                     lane);
                    __syncwarp();
                    if (lane == 0) {
                        __threadfence();
                        atomicAdd(&sync->gu_done[slot], 1u);
                    }
                }
            }
            if (gw.more()) {
                issue_g(s);
                issued_g++;
                gw.next();
            }
        }
        if (w.trace != nullptr && lane == 0) w.trace[(size_t)blockIdx.x * 64 + 59] = trx_globaltimer(); // h published
        // down chunks in order: their h rows copied (short calls), wait for the consumers, refill the stage
        TrxWalk pd;
        pd.init(n_act * H, H, CHD, true, seg, dgran);
        int n_mix = 0; // the blocks this CTA mixed (for the timeline)
        for (int j = 0; !failed && pd.more(); j++, pd.next()) {
            const int s = j % SD;
            if (!wait_all(&empty_d[s], (j / SD) & 1)) {
                failed = true;
                break;
            }
            if (dw.more()) {
                issue_d(s);
                issued_d++;
                dw.next();
                if (lane == 0) *(volatile int *)&s_armed = issued_d;
            }
        }
        if (seg) {
            // the mix of this CTA's rows [mra, mrb) of every token: it holds every expert's outputs for them (the
            // empties above: every chunk's h3 is in shared memory); the k outputs in increasing expert id, then the
            // residual (read at the kernel's start)
            const int nr = mrb - mra;
            for (int i = lane; !failed && i < nr * T; i += 32) {
                const int t = i / nr, d = mra + i % nr;
                float out = 0.0f;
                for (int sl = 0; sl < k; sl++) {
                    const int jj = t * k + sl;
                    if (s_selid[jj] < 0) continue; // (a row routed nowhere)
                    out = __fadd_rn(out, __fmul_rn(s_selw[jj], sh3[(size_t)s_place[jj] * nrmax + (d - mra)]));
                }
                if (float *o = out_row(t)) o[d] = out;
                if (!S.ext) {
                    const float xv = i < 32 ? xpre[0] : i < 64 ? xpre[1] : x_io[(int64_t)t * H + d];
                    x_io[(int64_t)t * H + d] = __fadd_rn(xv, out);
                }
            }
            n_mix = 1;
        } else {
            // the mixes: 16-row block b is mixed by CTA b mod grid once all its rows are counted (the mixing spread
            // over the CTAs, none of them waiting for a block before its own rows are out)
            for (int blk = blockIdx.x; !failed && blk < H / CHD; blk += gridDim.x) {
                bool ok = true;
                if (lane == 0) ok = trx_spin(&w.comb_cnt[blk], (uint32_t)(n_act * CHD), false);
                if (!__shfl_sync(0xffffffffu, ok, 0)) {
                    failed = true;
                    break;
                }
                combine(blk);
                n_mix++;
            }
        }
        if (w.trace != nullptr && lane == 0) {
            w.trace[(size_t)blockIdx.x * 64 + 50] = trx_globaltimer(); // the producer's publication done
        }
    } else if (warp == TRX_FU_HWARP) {
        // ---------------- short calls (Q8_0 / Q6_K down): the h rows of each down chunk's expert into its stage, once
        // the producer has armed the stage for the chunk and the expert is complete (chunks in order; the experts
        // complete in that order too)
        asm volatile("bar.sync 2, %0;" ::"n"(TRX_FU_THREADS) : "memory"); // the routing is sorted
        n_act = s_nact;
        if (hcopy) {
            TrxWalk hw;
            hw.init(n_act * H, H, CHD, true, seg, dgran);
            for (int j = 0; !failed && hw.more(); j++, hw.next()) {
                bool ok = true;
                if (lane == 0) {
                    uint64_t t0 = 0;
                    for (int it = 0; *(volatile int *)&s_armed <= j; it++) {
                        if (it == 0) t0 = trx_globaltimer();
                        else if (trx_globaltimer() - t0 > TRX_SPIN_NS) {
                            ok = false;
                            break;
                        }
                        __nanosleep(32);
                    }
                    if (ok) ok = trx_spin(&sync->gu_done[hw.slot], need, false);
                    if (ok) {
                        const int e = s_active[hw.slot], p0 = s_off[e], s = j % SD;
                        // the h the count made visible (generic writes of other CTAs), before the bulk copy reads it
                        asm volatile("fence.proxy.async.global;" ::: "memory");
                        trx_bulk_g2s(dn_buf + s * lay.dn_stage + hoff, w.h + (int64_t)p0 * F, (s_off[e + 1] - p0) * F * 4,
                                     &full_d[s]);
                    }
                }
                if (!__shfl_sync(0xffffffffu, ok, 0)) failed = true;
            }
        }
    } else {
        // ---------------- a consumer warp. The consumers form two groups of TRX_FU_GW warps that take the chunks in
        // turn (group 0 the even ones, group 1 the odd ones), each warp two rows of its group's chunks: two
        // independent chains a warp, two chunks in work at once.
        const int grp = warp / TRX_FU_GW, wl = warp % TRX_FU_GW;
        int cur = -1; // the token (gate/up) or grouped row (down) whose input this warp holds
        TrxQ4X X;
        int jg = 0;
        TrxWalk gw;
        gw.init(n_act * F, F, CHG, false, seg);
        const int gv0 = gw.v;
        // gate / up / SwiGLU: rows wl and wl + TRX_FU_GW of the group's chunks
        for (; gw.more(); jg++, gw.next()) {
            if ((jg & 1) != grp) continue;
            const int slot = gw.slot, e = s_active[slot], r0 = gw.r, n = gw.n();
            const int p0 = s_off[e], p1 = s_off[e + 1];
            const int s = jg % SG;
            if (!__all_sync(0xffffffffu, trx_mbar_wait(&full_g[s], (jg / SG) & 1, TRX_WAIT_NS))) {
                failed = true;
                break;
            }
            if (warp == 0 && jg < 16) TRX_TRACE(8 + jg / 2);
            if (wl < n) {
                const int ra = wl, rb = wl + TRX_FU_GW < n ? wl + TRX_FU_GW : wl; // rb == ra: one row left
                const uint8_t *ga = gu_buf + s * lay.gu_stage + ra * rbg, *gb = gu_buf + s * lay.gu_stage + rb * rbg;
                for (int p = p0; p < p1; p++) {
                    const int t = s_xmap[p];
                    const uint8_t *tok = s_tok + t * lay.tok_bytes;
                    float y[4]; // gate a, up a, gate b, up b
                    if (GT == TRX_Q4_K) {
                        if (t != cur) {
                            if (lprep) {
                                const double *bfd = reinterpret_cast<const double *>(tok + (size_t)H * 4);
                                trx_q4x_load(reinterpret_cast<const uint32_t *>(tok), 32, lane, bfd + 8 * (lane >> 2),
                                             bfd + H / 32 + (lane >> 2), X);
                            } else { // (the prep CTAs' rows in L2)
                                trx_q4x_load<true>(w.xq + (int64_t)t * H, 32, lane,
                                                   w.xq_bf + (int64_t)t * (H / 32) + 8 * (lane >> 2),
                                                   w.xq_sc + (int64_t)t * (H / 256) + (lane >> 2), X);
                            }
                            cur = t;
                        }
                        const uint8_t *const rows[4] = {ga, ga + gu_half, gb, gb + gu_half};
                        trx_q4k_row8xn<true, 4>(rows, X, lane, y);
                    } else { // half 0 the gate rows, half 1 the up rows
                        const float *xt = lprep ? reinterpret_cast<const float *>(tok) : w.x_lc + (int64_t)t * H;
                        const float va = lprep ? trx_q8l_dot<true, false>(lane < 16 ? ga : ga + gu_half, xt, H / 256, lane & 15)
                                               : trx_q8l_dot<true, true>(lane < 16 ? ga : ga + gu_half, xt, H / 256, lane & 15);
                        const float vb = lprep ? trx_q8l_dot<true, false>(lane < 16 ? gb : gb + gu_half, xt, H / 256, lane & 15)
                                               : trx_q8l_dot<true, true>(lane < 16 ? gb : gb + gu_half, xt, H / 256, lane & 15);
                        y[0] = va;
                        y[1] = __shfl_sync(0xffffffffu, va, 16);
                        y[2] = vb;
                        y[3] = __shfl_sync(0xffffffffu, vb, 16);
                    }
                    if (lane < 2 && (lane == 0 || rb != ra)) { // lane 0 row a, lane 1 row b
                        const int rr = lane ? rb : ra, r = r0 + rr;
                        const float g = lane ? y[2] : y[0], u = lane ? y[3] : y[1];
                        if (seg) sgu[(gw.v + rr - gv0) * T + (p - p0)] = make_float2(g, u);
                        else w.h[(int64_t)p * F + (DT != TRX_Q4_K ? trx_lc_pos(r) : r)] = trx_silu_mul(g, u);
                    }
                }
            }
            if (warp == 0 && jg < 16) TRX_TRACE(40 + jg / 2);
            // Longer calls: every warp of the group counts itself into the stage once per chunk (block scope, after
            // its h stores); the last one publishes the chunk's n rows to the expert's count with one device-scope
            // fence and atomic. A stage's uses are TRX_FU_GW counts apart (a warp reaches its next use only after
            // every arrive of the previous one), so the count's residue tells the last warp without a reset.
            __syncwarp();
            if (!seg) {
                uint32_t last = 0;
                if (lane == 0) {
                    __threadfence_block();
                    last = atomicAdd_block(&s_gcnt[s], 1u) % TRX_FU_GW == TRX_FU_GW - 1;
                }
                if (__shfl_sync(0xffffffffu, last, 0)) {
                    uint32_t old = 0;
                    if (lane == 0) {
                        __threadfence(); // the chunk's h rows (this CTA's warps', observed above) before the count
                        old = atomicAdd(&sync->gu_done[slot], (uint32_t)n);
                    }
                    old = __shfl_sync(0xffffffffu, old, 0);
                    if (DT == TRX_Q4_K && old + (uint32_t)n == (uint32_t)F) {
                        // the expert's last chunk: every other row of it is counted, so its h rows are complete;
                        // prepare them for the down's integer definition, then count once more
                        __threadfence();
                        for (int p = p0; p < p1; p++)
                            for (int s4 = 0; s4 < nsb_d; s4++)
                                trx_prep_q4x_block<true>(w.h + (int64_t)p * F + 256 * s4, w.hq + (int64_t)p * F, s4, nsb_d,
                                                         w.hq_bf + (int64_t)p * (F / 32) + 8 * s4,
                                                         w.hq_sc + (int64_t)p * nsb_d + s4, lane);
                        __syncwarp();
                        if (lane == 0) {
                            __threadfence();
                            atomicAdd(&sync->gu_done[slot], 1u);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) trx_mbar_arrive(&empty_g[s]);
            if (warp == 0 && jg < 16) TRX_TRACE(16 + jg / 2);
        }
        if (warp == 0) TRX_TRACE(4);

        // ---------------- down: half-warp hw = 2 wl + lane / 16 of the group takes rows hw and hw + 8 of its chunks
        cur = -1;
        int jd = 0, ready = -1; // ready: the last slot whose gate/up rows this warp saw complete
        TrxWalk dw;
        dw.init(n_act * H, H, CHD, true, seg, dgran);
        for (; dw.more() && !failed; jd++, dw.next()) {
            if ((jd & 1) != grp) continue;
            const int slot = dw.slot, e = s_active[slot], d0 = dw.r, n = dw.n();
            const int p0 = s_off[e], p1 = s_off[e + 1];
            const int s = jd % SD;
            if (slot != ready && !hcopy) { // (with hcopy the stage's barrier includes the expert's h rows)
                bool ok = true;
                if (lane == 0) ok = trx_spin(&sync->gu_done[slot], need, false);
                if (!__shfl_sync(0xffffffffu, ok, 0)) {
                    failed = true;
                    break;
                }
                if (warp == 0 && ready < 0) TRX_TRACE(61); // the first expert's gate/up rows seen complete
                ready = slot;
            }
            if (!__all_sync(0xffffffffu, trx_mbar_wait(&full_d[s], (jd / SD) & 1, TRX_WAIT_NS))) {
                failed = true;
                break;
            }
            if (warp == 0 && jd == 0) TRX_TRACE(5);
            if (warp == 0 && jd < 16) TRX_TRACE(24 + jd / 2);
            const int hw = 2 * wl + (lane >> 4), ra = hw, rb = hw + CHD / 2;
            const int rac = ra < n ? ra : 0, rbc = rb < n ? rb : 0; // a row past the chunk computes row 0, unstored
            if (2 * wl < n) {
                const uint8_t *sta = dn_buf + s * lay.dn_stage + rac * rbd, *stb = dn_buf + s * lay.dn_stage + rbc * rbd;
                const uint8_t *dps = dn_buf + s * lay.dn_stage + CHD * rbd; // the rows' (or block's) Q6_K d values
                const int dbase = seg ? 0 : d0 % CHD, da = dbase + rac, db = dbase + rbc;
                for (int p = p0; p < p1; p++) {
                    float va, vb;
                    if (DT == TRX_Q4_K) {
                        if (p != cur) {
                            trx_q4x_load<true>(w.hq + (int64_t)p * F, 16, lane & 15,
                                               w.hq_bf + (int64_t)p * (F / 32) + 8 * ((lane >> 2) & 3),
                                               w.hq_sc + (int64_t)p * nsb_d + ((lane >> 2) & 3), X);
                            cur = p;
                        }
                        va = trx_q4k_row4<true>(sta, X, lane);
                        vb = trx_q4k_row4<true>(stb, X, lane);
                    } else { // one 256-block an iteration, h through L1 (after the acquire above)
                        const float *hx = hcopy ? reinterpret_cast<const float *>(dn_buf + s * lay.dn_stage + hoff) +
                                                      (int64_t)(p - p0) * F
                                                : w.h + (int64_t)p * F;
                        const float2 v = DT == TRX_Q8_0 ? trx_q8l_dot2(sta, stb, hx, nsb_d, lane & 15)
                                                        : trx_q6l_dot2(sta, stb, dps + da * nsb_d * 2, dps + db * nsb_d * 2,
                                                                       hx, nsb_d, lane & 15);
                        va = v.x;
                        vb = v.y;
                    }
                    if ((lane & 15) == 0) {
                        if (ra < n) {
                            if (seg) sh3[(size_t)p * nrmax + (d0 - dw.ra) + ra] = va;
                            else w.h3[(int64_t)p * H + d0 + ra] = va;
                        }
                        if (rb < n) {
                            if (seg) sh3[(size_t)p * nrmax + (d0 - dw.ra) + rb] = vb;
                            else w.h3[(int64_t)p * H + d0 + rb] = vb;
                        }
                    }
                }
            }
            __syncwarp();

            // longer calls: count the chunk's rows into their 16-row block: the stage's last warp (as for gate/up)
            // adds the chunk's n rows
            if (!seg && lane == 0) {
                __threadfence_block();
                if (atomicAdd_block(&s_dcnt[s], 1u) % TRX_FU_GW == TRX_FU_GW - 1) {
                    __threadfence();
                    atomicAdd(&w.comb_cnt[d0 / CHD], (uint32_t)n);
                }
            }
            __syncwarp();
            if (lane == 0) trx_mbar_arrive(&empty_d[s]);
            if (warp == 0 && jd < 16) TRX_TRACE(32 + jd / 2);
        }
        if (warp == 0) TRX_TRACE(6);
    }

    // ---------------- end
    if (__syncthreads_or(failed)) {
        if (warp == TRX_FU_CWARPS && lane == 0) {
            atomicCAS(w.err, 0, 3 | (w.ep ? 0x100 : 0)); // the first error stays
            // every copy still in flight lands before the CTA's shared memory goes away: only a stage's latest copy
            // can be (a stage is refilled after its consumers saw the one before land), and only its phase parity
            // is unambiguous
            for (int q = max(0, issued_g - SG); q < issued_g; q++)
                trx_mbar_wait(&full_g[q % SG], (q / SG) & 1, TRX_WAIT_NS);
            for (int q = max(0, issued_d - SD); q < issued_d; q++)
                trx_mbar_wait(&full_d[q % SD], (q / SD) & 1, TRX_WAIT_NS);
            if (w.host_done) trx_post_done(w.host_done, epoch | 0x80000000u);
        }
        __syncthreads();
        return;
    }
    TRX_TRACE(52);
    if (tid == 0) {
        // the CTA's outputs (x may be host memory: system scope) before its count
        if (w.host_done || w.ep) __threadfence_system();
        else __threadfence();
        if (atomicAdd(&sync->finish, 1u) == gridDim.x - 1) { // every CTA is past its waits
            __threadfence();
            for (int i = 0; i < E; i++) sync->gu_done[i] = 0u;
            sync->route_cnt = 0u;
            sync->finish = 0u;
            __threadfence();
            if (w.host_done) trx_post_done(w.host_done, epoch); // every CTA's outputs are out
            if (w.ep) { // every output row is in its source's region: the sources' return flags
                const TrxEpPeers *P = w.ep;
                const uint32_t ep_epoch = reinterpret_cast<const TrxEpHdr *>(P->base[P->rank])->epoch;
                __threadfence_system();
                for (int s = 0; s < P->n; s++)
                    trx_st_release_sys(&reinterpret_cast<TrxEpHdr *>(P->base[s])->back_flag[P->rank], ep_epoch);
            }
        }
    }
}
