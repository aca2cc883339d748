// prefill.cuh: a long pass (prefill) of the MoE layer on the 5th-generation tensor cores.
//
// The routing is the exact one (router, top-k, counting sort: moe_kernels.cuh). The expert products are grouped
// GEMMs with tcgen05.mma (kind::tf32, fp32 accumulators in tensor memory) in 3xTF32 split precision: every operand
// v is carried as hi = tf32(v) and lo = tf32(v - hi), and a product as hi.hi + hi.lo + lo.hi (the dropped lo.lo is
// below 2^-22 of it), so the products keep the reference's fp32-activation semantics to about fp32 rounding
// (Trochilus computes them with the 16-lane fp32 contract: src/kernels/kernels.c:125-178 for Q8_0).
//
//  gather    grouped row p of the call (token xmap[p]) as hi/lo planes, its columns in the Q8L order of the weights
//            (position 16 l + m of each 256-block holds column l + 16 m), so that A and B meet in the same K order.
//  gate/up   tile = 128 grouped rows of one expert x (128 gate rows + the 128 up rows of the same outputs):
//            accumulator columns 0..127 gate, 128..255 up. The tile's outputs are h positions 128 n .. 128 n + 127 in
//            the Q8L order of F, so its weight rows are gathered by that order. Epilogue: h = silu(g) u (the
//            reference's tr_swiglu, kernels.c:1397-1421), stored as hi/lo planes: the down GEMM's A.
//  down      tile = 128 grouped rows x 256 down rows; epilogue stores h3 (fp32).
//  combine   the exact mix: out = +0, out += w_slot h3[place] in increasing expert id, x += out (olmoe.c:1432-1446).
//
// A GEMM CTA: warps 0-7 dequantise the tile's Q8L weight rows (d q: exact in fp32; a row per thread) into hi/lo
// tiles in shared memory, then run the epilogue (warp w reads accumulator lanes 32 (w % 4) .. + 31, half the
// columns each); warp 8 brings the A planes with 2-D TMA (128-byte swizzle, no multicast); warp 9 owns the tensor
// memory and issues the MMAs (one thread).
// Two stages of BK = 32 columns; every wait bounded (TRX_WAIT_NS), a failure sets the error flag.
//
// Accumulation: the tensor core's fp32 accumulator does not round each addition to nearest, and over the ~800
// additions of a K = 2048 product its error grows past 1e-5. So the MMAs accumulate one chunk of TRX_PF_CK k-steps
// (128 columns of K) at a time in tensor-memory columns 0..255; the converter warps add each finished chunk into a
// running sum kept in columns 256..511 with round-to-nearest fp32 additions (tcgen05.ld / tcgen05.st), and the MMAs
// of the next chunk wait for that.
#pragma once
#include <cstdint>
#include <cuda.h>
#include "bulk.cuh"
#include "moe_kernels.cuh"

#define TRX_PF_BM 128
#define TRX_PF_BN 256
#define TRX_PF_BK 32
#define TRX_PF_STAGES 2
#define TRX_PF_THREADS 320 // warps 0-7 converters + epilogue, warp 8 TMA, warp 9 MMA
#define TRX_PF_A_BYTES (TRX_PF_BM * TRX_PF_BK * 4)                 // one plane of the A tile: 16 KB
#define TRX_PF_B_BYTES (TRX_PF_BN * TRX_PF_BK * 4)                 // one plane of the B tile: 32 KB
#define TRX_PF_STAGE_BYTES (2 * TRX_PF_A_BYTES + 2 * TRX_PF_B_BYTES) // 96 KB
#define TRX_PF_SMEM (TRX_PF_STAGES * TRX_PF_STAGE_BYTES + 1024 + 256)
#define TRX_PF_CK 4 // k-steps per accumulation chunk (128 columns of K)

// ---- tensor memory, MMA and TMA helpers (inline PTX, sm_100a) ----

__device__ __forceinline__ void trx_tmem_alloc(uint32_t *dst_smem, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(trx_smem(dst_smem)), "r"(cols)
                 : "memory");
}
__device__ __forceinline__ void trx_tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void trx_tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
__device__ __forceinline__ void trx_tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void trx_tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 bytes apart (sm_100 version 1)
__device__ __forceinline__ uint64_t trx_umma_desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3fffu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
           ((uint64_t)2 << 61);
}

// instruction descriptor: D f32, A and B tf32, both K-major, M = 128, N = 256
constexpr uint32_t TRX_PF_IDESC = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(TRX_PF_BN >> 3) << 17) |
                                  ((uint32_t)(TRX_PF_BM >> 4) << 24);

__device__ __forceinline__ void trx_mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                 " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
                 "l"(adesc), "l"(bdesc), "r"(TRX_PF_IDESC), "r"(accumulate)
                 : "memory");
}

// the mbarrier tracks the completion of every MMA this thread issued before
__device__ __forceinline__ void trx_umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(trx_smem(bar))
                 : "memory");
}

// 32 consecutive accumulator columns of this warp's 32 lanes (one row per thread); _nw: without the wait (the
// registers are valid after trx_tmem_wait_ld)
__device__ __forceinline__ void trx_tmem_ld32_nw(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
                 "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
                   "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
                   "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
                   "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void trx_tmem_ld16_nw(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
                 "%14, %15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void trx_tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void trx_tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void trx_tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
                 "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
                   "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
                   "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
                   "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr)
                 : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void trx_tmem_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
                 "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
                 ::"r"(taddr), "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]),
                 "f"(v[8]), "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]),
                 "f"(v[16]), "f"(v[17]), "f"(v[18]), "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]),
                 "f"(v[24]), "f"(v[25]), "f"(v[26]), "f"(v[27]), "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
                 : "memory");
}

__device__ __forceinline__ void trx_tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    trx_tmem_st32(taddr, reinterpret_cast<const float(&)[32]>(v));
}

// 2-D tiled TMA load (no multicast): box at element (x, y) of the tensor map into shared memory
__device__ __forceinline__ void trx_tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(trx_smem(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(trx_smem(bar))
                 : "memory");
}

// tf32 split of an fp32 value: hi rounded to the nearest tf32 (ties away), lo = the remainder rounded the same way
__device__ __forceinline__ float trx_tf32(float v) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
    return __uint_as_float(r);
}
__device__ __forceinline__ void trx_split(float v, float &hi, float &lo) {
    hi = trx_tf32(v);
    lo = trx_tf32(__fsub_rn(v, hi));
}

// h = silu(g) u on the tensor road, which holds a 1e-5 bound rather than the reference's bits: the fast exponential
// and division intrinsics (a few ulp) instead of the correctly rounded trx_expf and an IEEE division
__device__ __forceinline__ float trx_pf_silu_mul(float g, float u) {
    return __fmul_rn(__fdividef(g, __fadd_rn(1.0f, __expf(-g))), u);
}

// the Q8L position of column k within its 256-block, and back
__host__ __device__ __forceinline__ int trx_q8l_pos(int k) { return (k & ~255) + 16 * (k & 15) + ((k >> 4) & 15); }
__host__ __device__ __forceinline__ int trx_q8l_col(int pos) { return (pos & ~255) + ((pos >> 4) & 15) + 16 * (pos & 15); }

struct TrxPfArgs {
    const uint8_t *wa, *wb; // gate/up: the gate and up matrices of expert 0; down: the down matrix (wb unused)
    int64_t wa_mb, wb_mb;   // bytes between consecutive experts' matrices
    int K;                  // columns (H for gate/up, F for down)
    int N;                  // output columns of the GEMM (F for gate/up, H for down)
    const int32_t *offsets, *active, *n_active;
    float *out_hi, *out_lo; // gate/up: h planes [R][F] (Q8L order); down: out_hi = h3 [R][H]
    int32_t *err;
};

// ---- gather: grouped row p's input as hi/lo planes in Q8L column order ----
__global__ void __launch_bounds__(256) trx_k_pf_gather(const float *__restrict__ normed, const int32_t *__restrict__ xmap,
                                                       const int32_t *__restrict__ offsets, int E, int H,
                                                       float *__restrict__ xhi, float *__restrict__ xlo) {
    const int p = blockIdx.x;
    if (p >= offsets[E]) return;
    const float *x = normed + (int64_t)xmap[p] * H;
    for (int pos = threadIdx.x; pos < H; pos += blockDim.x) {
        float hi, lo;
        trx_split(x[trx_q8l_col(pos)], hi, lo);
        xhi[(int64_t)p * H + pos] = hi;
        xlo[(int64_t)p * H + pos] = lo;
    }
}

// ---- combine: out = +0; out += sel_w h3[place] in id order; x += out ----
__global__ void __launch_bounds__(256) trx_k_pf_combine(const float *__restrict__ sel_w, const int32_t *__restrict__ place,
                                                        const float *__restrict__ h3, int T, int k, int H,
                                                        float *__restrict__ x, float *__restrict__ ffn_out) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= (int64_t)T * H) return;
    const int t = (int)(i / H), d = (int)(i % H);
    float out = 0.0f;
    for (int s = 0; s < k; s++)
        out = __fadd_rn(out, __fmul_rn(sel_w[t * k + s], h3[(int64_t)place[t * k + s] * H + d]));
    if (ffn_out) ffn_out[i] = out;
    x[i] = __fadd_rn(x[i], out);
}

// the CTA's m-tile: the active expert whose segment holds it and its first grouped row; false when out of range
__device__ __forceinline__ bool trx_pf_tile(const int32_t *offsets, const int32_t *active, int n_act, int q, int &e,
                                            int &row0, int &rows) {
    for (int i = 0; i < n_act; i++) {
        const int ee = active[i], a = offsets[ee], n = offsets[ee + 1] - a, mt = (n + TRX_PF_BM - 1) / TRX_PF_BM;
        if (q < mt) {
            e = ee;
            row0 = a + q * TRX_PF_BM;
            rows = min(TRX_PF_BM, n - q * TRX_PF_BM);
            return true;
        }
        q -= mt;
    }
    return false;
}

// ---- the grouped GEMM: grid (N / tile outputs, m-tiles upper bound) ----
template <bool GATEUP, int WT>
__global__ void __launch_bounds__(TRX_PF_THREADS, 1)
    trx_k_pf_gemm(const __grid_constant__ CUtensorMap map_hi, const __grid_constant__ CUtensorMap map_lo, TrxPfArgs a) {
    extern __shared__ __align__(1024) uint8_t pf_smem_raw[];
    __shared__ int s_e, s_row0, s_rows, s_ok;
    __shared__ uint32_t s_tmem;
    __shared__ int s_fail;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        int e = 0, row0 = 0, rows = 0;
        s_ok = trx_pf_tile(a.offsets, a.active, *a.n_active, blockIdx.y, e, row0, rows);
        s_e = e;
        s_row0 = row0;
        s_rows = rows;
        s_fail = 0;
    }
    __syncthreads();
    if (!s_ok) return;
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(pf_smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t *full_a = reinterpret_cast<uint64_t *>(smem + TRX_PF_STAGES * TRX_PF_STAGE_BYTES);
    uint64_t *full_b = full_a + TRX_PF_STAGES, *empty = full_b + TRX_PF_STAGES;
    uint64_t *cfull = empty + TRX_PF_STAGES, *cempty = cfull + 1; // a chunk accumulated; a chunk added to the sum
    auto a_hi = [&](int s) { return smem + s * TRX_PF_STAGE_BYTES; };
    auto a_lo = [&](int s) { return smem + s * TRX_PF_STAGE_BYTES + TRX_PF_A_BYTES; };
    auto b_hi = [&](int s) { return smem + s * TRX_PF_STAGE_BYTES + 2 * TRX_PF_A_BYTES; };
    auto b_lo = [&](int s) { return smem + s * TRX_PF_STAGE_BYTES + 2 * TRX_PF_A_BYTES + TRX_PF_B_BYTES; };
    const int e = s_e, row0 = s_row0, rows = s_rows, K = a.K, nk = K / TRX_PF_BK, n = blockIdx.x;
    if (tid == 0) {
        for (int s = 0; s < TRX_PF_STAGES; s++) {
            trx_mbar_init(&full_a[s], 1);
            trx_mbar_init(&full_b[s], 8);
            trx_mbar_init(&empty[s], 1);
        }
        trx_mbar_init(cfull, 1);
        trx_mbar_init(cempty, 8);
        trx_fence_barrier_init();
    }
    if (warp == 9) {
        trx_tmem_alloc(&s_tmem, 2 * TRX_PF_BN);
        trx_tmem_relinquish();
    }
    trx_tc_fence_before();
    __syncthreads();
    trx_tc_fence_after();
    const uint32_t tmem = s_tmem;

    if (warp == 8) {
        // ---- TMA: the A planes of every k-step
        if (lane == 0) {
            int issued = 0;
            for (int ks = 0; ks < nk; ks++, issued++) {
                const int s = ks % TRX_PF_STAGES;
                if (ks >= TRX_PF_STAGES && !trx_mbar_wait(&empty[s], ((ks / TRX_PF_STAGES) - 1) & 1, TRX_WAIT_NS)) {
                    atomicExch(&s_fail, 1);
                    break;
                }
                trx_mbar_expect_tx(&full_a[s], 2u * TRX_PF_A_BYTES);
                trx_tma_load_2d(a_hi(s), &map_hi, ks * TRX_PF_BK, row0, &full_a[s]);
                trx_tma_load_2d(a_lo(s), &map_lo, ks * TRX_PF_BK, row0, &full_a[s]);
            }
            // every copy this thread armed lands before the CTA can leave
            for (int q = max(0, issued - TRX_PF_STAGES); q < issued; q++)
                trx_mbar_wait(&full_a[q % TRX_PF_STAGES], (q / TRX_PF_STAGES) & 1, TRX_WAIT_NS);
        }
    } else if (warp == 9) {
        // ---- MMA issue: 4 k-slices of 8 x 3 split products per k-step, chunk by chunk into columns 0..255
        if (lane == 0) {
            const uint32_t sa = trx_smem(smem);
            for (int ks = 0; ks < nk; ks++) {
                const int s = ks % TRX_PF_STAGES, par = (ks / TRX_PF_STAGES) & 1;
                if (ks % TRX_PF_CK == 0 && ks > 0 &&
                    !trx_mbar_wait(cempty, ((ks / TRX_PF_CK) - 1) & 1, TRX_WAIT_NS)) { // the last chunk was added up
                    atomicExch(&s_fail, 1);
                    break;
                }
                if (!trx_mbar_wait(&full_a[s], par, TRX_WAIT_NS) || !trx_mbar_wait(&full_b[s], par, TRX_WAIT_NS)) {
                    atomicExch(&s_fail, 1);
                    break;
                }
                trx_tc_fence_after();
                const uint32_t ah = sa + s * TRX_PF_STAGE_BYTES, al = ah + TRX_PF_A_BYTES, bh = ah + 2 * TRX_PF_A_BYTES,
                               bl = bh + TRX_PF_B_BYTES;
#pragma unroll
                for (int kk = 0; kk < TRX_PF_BK / 8; kk++) {
                    const uint32_t o = 32u * kk; // 8 tf32 = 32 bytes along the swizzled 128-byte row
                    trx_mma_tf32(tmem, trx_umma_desc_sw128(ah + o), trx_umma_desc_sw128(bh + o),
                                 (ks % TRX_PF_CK) != 0 || kk != 0);
                    trx_mma_tf32(tmem, trx_umma_desc_sw128(ah + o), trx_umma_desc_sw128(bl + o), 1u);
                    trx_mma_tf32(tmem, trx_umma_desc_sw128(al + o), trx_umma_desc_sw128(bh + o), 1u);
                }
                trx_umma_commit(&empty[s]); // the stage is free once these MMAs have read it
                if (ks % TRX_PF_CK == TRX_PF_CK - 1 || ks == nk - 1) trx_umma_commit(cfull);
            }
            if (*(volatile int *)&s_fail) trx_umma_commit(cfull); // wakes the converters (they see the failure)
        }
    } else {
        // ---- converters: this thread's B row r = tid (gate/up: r < 128 the gate row of output 128 n + r, r >= 128
        // the up row of output 128 n + r - 128; down: row 256 n + r), dequantised k-step by k-step into the swizzled
        // hi/lo tiles. K-step j of a 256-block holds Q8L positions 32 j .. 32 j + 31: position 16 l + m is column
        // l + 16 m, the column of lane l's element m in the 16-lane contract (the Q8L and Q6L storage order).
        const int nsb = K / 256;
        const int64_t rb = (int64_t)nsb * (WT == TRX_Q8_0 ? 272 : WT == TRX_Q4_K ? 144 : 208);
        const int r = tid;
        const uint8_t *mat = GATEUP && r >= 128 ? a.wb + e * a.wb_mb : a.wa + e * a.wa_mb;
        const int row = GATEUP ? trx_q8l_col(128 * n + (r & 127)) : 256 * n + r;
        const uint8_t *rp = mat + (int64_t)row * rb;
        // the block's scales: Q8_0 the 8 f16 d of its 32-column groups; Q4_K fl(d sc_j) (0..7) and fl(dmin m_j)
        // (8..15) of its 8 sub-blocks; Q6_K fl(d sc_m) of its 16 sub-blocks (all exact)
        float sc[16];
        uint4 qa, qb; // this k-step's quant bytes
        auto load_q = [&](int ks) {
            const int j = ks & 7, blk = ks >> 3;
            if (WT == TRX_Q8_0) {
                const int64_t o = (int64_t)blk * 272 + 16 + 32 * j;
                qa = __ldg(reinterpret_cast<const uint4 *>(rp + o));
                qb = __ldg(reinterpret_cast<const uint4 *>(rp + o + 16));
            } else if (WT == TRX_Q4_K) {
                // columns 2 j + t + 16 m (t = 0, 1): byte 32 (m >> 2) + 16 (m & 1) + 2 j + t of the block's quants,
                // the high nibble when (m >> 1) & 1; halfword w = 2 (m >> 2) + (m & 1) holds both t
                const uint8_t *q = rp + (int64_t)blk * 144 + 16 + 2 * j;
                uint32_t hw[8];
#pragma unroll
                for (int w2 = 0; w2 < 8; w2++) hw[w2] = __ldg(reinterpret_cast<const uint16_t *>(q + 32 * (w2 >> 1) + 16 * (w2 & 1)));
                qa = make_uint4(hw[0] | hw[1] << 16, hw[2] | hw[3] << 16, hw[4] | hw[5] << 16, hw[6] | hw[7] << 16);
            } else { // Q6L: lanes 2 j and 2 j + 1's low nibbles (8 bytes each) and high bit pairs (4 bytes each)
                qa = __ldg(reinterpret_cast<const uint4 *>(rp + 128 * blk + 16 * j));
                const uint2 h = __ldg(reinterpret_cast<const uint2 *>(rp + 128 * nsb + 64 * blk + 8 * j));
                qb = make_uint4(h.x, h.y, 0u, 0u);
            }
        };
        auto load_d = [&](int blk) {
            if (WT == TRX_Q8_0) {
                const uint4 u = __ldg(reinterpret_cast<const uint4 *>(rp + (int64_t)blk * 272));
                const uint32_t wd[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                for (int b = 0; b < 8; b++) sc[b] = trx_half((uint16_t)(wd[b >> 1] >> (16 * (b & 1))));
            } else if (WT == TRX_Q4_K) {
                const uint4 hdr = __ldg(reinterpret_cast<const uint4 *>(rp + (int64_t)blk * 144));
                const float d = trx_half((uint16_t)(hdr.x & 0xffffu)), dmin = trx_half((uint16_t)(hdr.x >> 16));
                const uint32_t sw[3] = {hdr.y, hdr.z, hdr.w}; // the 12 packed scale bytes
                auto byte = [&](int i) { return (sw[i >> 2] >> (8 * (i & 3))) & 255u; };
#pragma unroll
                for (int jj = 0; jj < 8; jj++) { // Q4_K's 6-bit scale and min of sub-block jj
                    const uint32_t scj = jj < 4 ? byte(jj) & 63u : (byte(jj + 4) & 15u) | ((byte(jj - 4) >> 6) << 4);
                    const uint32_t mj = jj < 4 ? byte(jj + 4) & 63u : (byte(jj + 4) >> 4) | ((byte(jj) >> 6) << 4);
                    sc[jj] = __fmul_rn(d, (float)scj);
                    sc[8 + jj] = __fmul_rn(dmin, (float)mj);
                }
            } else {
                const float d = trx_half(__ldg(reinterpret_cast<const uint16_t *>(mat + (int64_t)a.N * rb) +
                                               (int64_t)row * nsb + blk)); // (the d values follow the N rows)
                const uint4 u = __ldg(reinterpret_cast<const uint4 *>(rp + 192 * nsb + 16 * blk));
                const uint32_t sw[4] = {u.x ^ 0x80808080u, u.y ^ 0x80808080u, u.z ^ 0x80808080u, u.w ^ 0x80808080u};
#pragma unroll
                for (int m = 0; m < 16; m++) sc[m] = __fmul_rn(d, trx_s8_to_f32(sw[m >> 2], m & 3));
            }
        };
        // the weight at position i of the k-step (exact, but Q4_K's d sc q - dmin m, rounded once)
        auto weight = [&](const uint4 ca, const uint4 cb, int i) -> float {
            const uint32_t wa[4] = {ca.x, ca.y, ca.z, ca.w};
            if (WT == TRX_Q8_0) {
                const uint32_t qw = i < 16 ? wa[i >> 2] : (i < 24 ? (i < 20 ? cb.x : cb.y) : (i < 28 ? cb.z : cb.w));
                return __fmul_rn(sc[(i & 15) >> 1], trx_s8_to_f32(qw ^ 0x80808080u, i & 3)); // 19 bits at most
            } else if (WT == TRX_Q4_K) {
                const int t = i >> 4, m = i & 15, w2 = 2 * (m >> 2) + (m & 1);
                const uint32_t q = (wa[w2 >> 1] >> (16 * (w2 & 1) + 8 * t + 4 * ((m >> 1) & 1))) & 15u;
                const float qf = __fsub_rn(__uint_as_float(0x4b000000u | q), 8388608.0f); // exact
                return __fsub_rn(__fmul_rn(sc[m >> 1], qf), sc[8 + (m >> 1)]);
            } else {
                const int lh = i >> 4, m = i & 15;
                uint32_t q4[4];
                trx_q6l_quants(make_uint2(wa[2 * lh], wa[2 * lh + 1]), lh ? cb.y : cb.x, q4);
                const uint32_t q = (q4[m >> 2] >> (8 * (m & 3))) & 255u;
                const float qf = __fsub_rn(__uint_as_float(0x4b000000u | q), 8388640.0f); // q - 32, exact
                return __fmul_rn(sc[m], qf); // exact
            }
        };
        // the row's 32 weights into tile row r
        auto put_row = [&](int s, uint4 ca, uint4 cb) {
            uint8_t *th = b_hi(s) + (r >> 3) * 1024 + (r & 7) * 128, *tlo = b_lo(s) + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
            for (int c = 0; c < 8; c++) { // 16-byte chunk c holds positions 4 c .. 4 c + 3
                float hv[4], lv[4];
#pragma unroll
                for (int i = 0; i < 4; i++) trx_split(weight(ca, cb, 4 * c + i), hv[i], lv[i]);
                const int sw = (c ^ (r & 7)) << 4;
                *reinterpret_cast<float4 *>(th + sw) = make_float4(hv[0], hv[1], hv[2], hv[3]);
                *reinterpret_cast<float4 *>(tlo + sw) = make_float4(lv[0], lv[1], lv[2], lv[3]);
            }
        };
        // warp w's share of the accumulator: lanes 32 (w % 4) .., columns (w / 4) 128 .. + 127
        const uint32_t tl = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
        const int cb = (warp >> 2) * 128;
        // adds finished chunk c (columns 0..255) into the running sum (columns 256..511)
        auto drain = [&](int c) -> bool {
            if (!__all_sync(0xffffffffu, trx_mbar_wait(cfull, c & 1, TRX_WAIT_NS)) || *(volatile int *)&s_fail) return false;
            trx_tc_fence_after();
#pragma unroll 1
            for (int c0 = cb; c0 < cb + 128; c0 += 32) {
                uint32_t v[32], rr[32];
                trx_tmem_ld32_nw(tl + c0, v);
                if (c > 0) trx_tmem_ld32_nw(tl + TRX_PF_BN + c0, rr);
                trx_tmem_wait_ld();
                if (c > 0) {
#pragma unroll
                    for (int i = 0; i < 32; i++) v[i] = __float_as_uint(__fadd_rn(__uint_as_float(rr[i]), __uint_as_float(v[i])));
                }
                trx_tmem_st32(tl + TRX_PF_BN + c0, v); // waited for once, below
            }
            trx_tmem_wait_st();
            trx_tc_fence_before();
            __syncwarp();
            if (lane == 0) trx_mbar_arrive(cempty);
            return true;
        };
        bool failed = false;
        load_d(0);
        load_q(0);
        for (int ks = 0; ks < nk; ks++) {
            const int s = ks % TRX_PF_STAGES;
            const uint4 ca = qa, cbq = qb;
            if (ks + 1 < nk) load_q(ks + 1); // the next k-step's quants in flight while this one is written
            if (ks >= TRX_PF_STAGES &&
                !__all_sync(0xffffffffu, trx_mbar_wait(&empty[s], ((ks / TRX_PF_STAGES) - 1) & 1, TRX_WAIT_NS))) {
                failed = true;
                break;
            }
            if ((ks & 7) == 0 && ks > 0) load_d(ks >> 3);
            put_row(s, ca, cbq);
            trx_fence_proxy_async(); // these generic-proxy writes before the tensor core's reads
            __syncwarp();
            if (lane == 0) trx_mbar_arrive(&full_b[s]);
            // the first k-step of a chunk is written: add the chunk before it into the sum (its MMAs finish
            // meanwhile; the next chunk's wait for this)
            if (ks % TRX_PF_CK == 0 && ks > 0 && !drain(ks / TRX_PF_CK - 1)) {
                failed = true;
                break;
            }
        }
        if (failed) atomicExch(&s_fail, 1);
        // ---- epilogue: the last chunk plus the running sum, this warp's 32 rows and share of the columns
        const int last = (nk - 1) / TRX_PF_CK;
        const bool ok = !failed && __all_sync(0xffffffffu, trx_mbar_wait(cfull, last & 1, TRX_WAIT_NS)) &&
                        !*(volatile int *)&s_fail;
        trx_tc_fence_after();
        if (!ok) {
            atomicExch(&s_fail, 1);
        } else {
            const int m = 32 * (warp & 3) + lane;
            const int64_t p = row0 + m;
            const bool valid = m < rows;
            auto col32 = [&](int c0, float (&v)[32]) { // accumulator column block c0: chunk + sum
                uint32_t u0[32], u1[32];
                trx_tmem_ld32_nw(tl + c0, u0);
                if (last > 0) trx_tmem_ld32_nw(tl + TRX_PF_BN + c0, u1);
                trx_tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; i++)
                    v[i] = last > 0 ? __fadd_rn(__uint_as_float(u1[i]), __uint_as_float(u0[i])) : __uint_as_float(u0[i]);
            };
            if (GATEUP) { // h columns (w / 4) 64 .. + 63: gate at c, up at 128 + c
#pragma unroll 1
                for (int c0 = (warp >> 2) * 64; c0 < (warp >> 2) * 64 + 64; c0 += 32) {
                    float g[32], u[32];
                    col32(c0, g);
                    col32(128 + c0, u);
                    if (valid) {
                        float *oh = a.out_hi + p * a.N + 128 * n + c0, *ol = a.out_lo + p * a.N + 128 * n + c0;
#pragma unroll
                        for (int i = 0; i < 32; i += 4) {
                            float hv[4], lv[4];
#pragma unroll
                            for (int j = 0; j < 4; j++) trx_split(trx_pf_silu_mul(g[i + j], u[i + j]), hv[j], lv[j]);
                            *reinterpret_cast<float4 *>(oh + i) = make_float4(hv[0], hv[1], hv[2], hv[3]);
                            *reinterpret_cast<float4 *>(ol + i) = make_float4(lv[0], lv[1], lv[2], lv[3]);
                        }
                    }
                }
            } else {
#pragma unroll 1
                for (int c0 = cb; c0 < cb + 128; c0 += 32) {
                    float v[32];
                    col32(c0, v);
                    if (valid) {
                        float *o = a.out_hi + p * a.N + 256 * n + c0;
#pragma unroll
                        for (int i = 0; i < 32; i += 4)
                            *reinterpret_cast<float4 *>(o + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
                    }
                }
            }
        }
    }
    trx_tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        trx_tc_fence_after();
        trx_tmem_dealloc(tmem, 2 * TRX_PF_BN);
    }
    if (tid == 0 && s_fail) atomicExch(a.err, 4);
}
