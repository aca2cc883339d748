// layouts.cuh: the weight layouts in HBM, the upload-time repack kernels, and the per-warp dot
// products of one weight row against one input row under Trochilus's numerics.
//
// A GGUF row is read from the host once (tr_gpu_moe_create, or the first kernel-level call that
// names it) and kept in HBM in one of these layouts. Each layout has exactly the GGUF row's bytes;
// only their order changes, so the HBM traffic per weight is the format's own.
//
//  Q4_K  kept as GGUF blocks (144 B = 16 B header + 128 B quants): 16-byte aligned already.
//        Dot: Q4_K's exact-integer definition (Trochilus src/kernels/kernels.h:186-205,
//        src/kernels/kernels.c:196-253). The input row is prepared once (trx_prep_q4x below: per
//        256-block shift, X = nearest-even(x 2^sh), its four bytes as planes); a thread takes one
//        32-byte quant chunk (64 weights of sub-blocks 2c and 2c+1) and forms sum q X exactly with
//        dp4a over the byte planes, the 4 threads of a block add their int64 T exactly (any order),
//        and one thread finishes v = (d T - dmin M) 2^-sh in f64; the row sums v in increasing
//        block order from +0, then rounds to float once.
//  Q8L   from Q8_0 (34 B per 32 weights): per 256 weights (8 blocks), 16 B of the 8 f16 scales, then
//        256 B where byte 16 l + m is q[l + 16 m] (lane l's m-th weight of the chunk). A 16-byte
//        load of a thread of the 16-lane contract is then 16 consecutive terms of its own lane.
//  Q6L   from Q6_K (210 B per 256 weights): per row, for each block s: 128 B low nibbles, then 64 B
//        high bit-pairs, then the 16 int8 scales; the f16 d of every (row, block) after all the rows of
//        the matrix. Lane l's 16 weights m (element l + 16 m) are ordered so that four 6-bit quants come
//        out as the four bytes of a word in two or three logic operations: its 8 low-nibble bytes hold,
//        in byte b < 4, weights b (low nibble) and b + 4 (high nibble), in byte 4 + b weights 8 + b and
//        12 + b; its 4 high-bit bytes hold in byte b the pairs of weights b, b + 4, b + 8, b + 12 at bits
//        0, 2, 4 and 6.
//  F32, BF16 (router): as in the file.
// The lane-contract dots (Q8_0, Q6_K, F32, BF16) take their input row in the "LC order": inside
// every 256 floats, x[l + 16 m] sits at 64 (m >> 2) + 4 l + (m & 3), so that a thread's four
// 16-byte loads hold its lane's 16 inputs and a half-warp's loads are one contiguous 256 B.
#pragma once
#include <cstdint>
#include "common.cuh"

// ---- sizes ----
__host__ __device__ inline int64_t trx_row_bytes(int type, int64_t n) {
    switch (type) {
    case TRX_F32: return n * 4;
    case TRX_F16:
    case TRX_BF16: return n * 2;
    case TRX_Q8_0: return n % 32 ? 0 : n / 32 * 34;
    case TRX_Q4_K: return n % 256 ? 0 : n / 256 * 144;
    case TRX_Q6_K: return n % 256 ? 0 : n / 256 * 210;
    default: return 0;
    }
}

// LC position of natural index k (inside its 256-chunk)
__host__ __device__ inline int trx_lc_pos(int k) {
    const int i = k >> 8, r = k & 255, l = r & 15, m = r >> 4;
    return (i << 8) + ((m >> 2) << 6) + (l << 2) + (m & 3);
}

// a float4 load, through L2 only when CG (data another CTA of the same kernel wrote)
template <bool CG>
__device__ __forceinline__ float4 trx_ldx(const float *p) {
    if (CG) return __ldcg(reinterpret_cast<const float4 *>(p));
    return *reinterpret_cast<const float4 *>(p);
}

// ---- repack kernels (one thread block per row) ----

// Q8_0 rows (GGUF) -> Q8L rows; n % 256 == 0
__global__ void trx_repack_q8l(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst, int64_t rows, int64_t n) {
    const int64_t r = blockIdx.x;
    if (r >= rows) return;
    const int64_t rb = n / 32 * 34;
    const uint8_t *s = src + r * rb;
    uint8_t *d = dst + r * rb;
    for (int64_t k = threadIdx.x; k < n; k += blockDim.x) {
        const int64_t i = k >> 8, rr = k & 255, l = rr & 15, m = rr >> 4, b = k >> 5;
        d[i * 272 + 16 + 16 * l + m] = s[b * 34 + 2 + (k & 31)];
        if ((k & 31) == 0) { // the block's scale
            d[i * 272 + 2 * (b & 7)] = s[b * 34];
            d[i * 272 + 2 * (b & 7) + 1] = s[b * 34 + 1];
        }
    }
}

// Q6_K rows (GGUF) -> Q6L matrix (rows consecutive, then the d's); n % 256 == 0
__global__ void trx_repack_q6l(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst, int64_t rows, int64_t n) {
    const int64_t r = blockIdx.x;
    if (r >= rows) return;
    const int64_t nsb = n / 256;
    const uint8_t *srow = src + r * nsb * 210;
    uint8_t *drow = dst + r * nsb * 208;
    uint8_t *dd = dst + rows * nsb * 208 + r * nsb * 2;
    for (int64_t s = 0; s < nsb; s++) {
        const uint8_t *blk = srow + s * 210;
        // the low nibble and the high bit-pair of weight m of lane l (element i = l + 16 m of the block)
        auto lo4 = [&](int l, int m) -> unsigned {
            const int i = l + 16 * m, hh = i >> 7, c = (i >> 5) & 3, ll = i & 31;
            const unsigned v = blk[64 * hh + 32 * (c & 1) + ll];
            return (c & 2) ? v >> 4 : v & 15u;
        };
        auto hi2 = [&](int l, int m) -> unsigned {
            const int i = l + 16 * m, hh = i >> 7, c = (i >> 5) & 3, ll = i & 31;
            return (blk[128 + 32 * hh + ll] >> (2 * c)) & 3u;
        };
        // lane l's byte t (0..7): weights mb (low nibble) and mb + 4 (high nibble), mb = t < 4 ? t : t + 4
        for (int t = threadIdx.x; t < 128; t += blockDim.x) {
            const int l = t >> 3, b = t & 7, mb = b < 4 ? b : b + 4;
            drow[s * 128 + t] = (uint8_t)(lo4(l, mb) | lo4(l, mb + 4) << 4);
        }
        // lane l's byte b (0..3): the pairs of weights b, b + 4, b + 8, b + 12 at bits 0, 2, 4, 6
        for (int t = threadIdx.x; t < 64; t += blockDim.x) {
            const int l = t >> 2, b = t & 3;
            drow[nsb * 128 + s * 64 + t] =
                (uint8_t)(hi2(l, b) | hi2(l, b + 4) << 2 | hi2(l, b + 8) << 4 | hi2(l, b + 12) << 6);
        }
        for (int t = threadIdx.x; t < 16; t += blockDim.x) drow[nsb * 192 + s * 16 + t] = blk[192 + t];
        if (threadIdx.x == 0) {
            dd[2 * s] = blk[208];
            dd[2 * s + 1] = blk[209];
        }
    }
}

// Router rows (F32 or BF16, n % 256 == 0) -> "lane rows": inside every 256 elements, lane l's 16 elements
// (l + 16 m, m = 0..15) contiguous at 16 l + m, so one thread of a 16-lane chain reads its lane with 16-byte loads
__global__ void trx_repack_lanerows(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst, int64_t rows, int64_t n,
                                    int elem) {
    const int64_t r = blockIdx.x;
    if (r >= rows) return;
    for (int64_t k = threadIdx.x; k < n; k += blockDim.x) {
        const int64_t i = k >> 8, l = k & 15, m = (k >> 4) & 15;
        const int64_t q = (i << 8) + 16 * l + m;
        for (int b = 0; b < elem; b++) dst[(r * n + q) * elem + b] = src[(r * n + k) * elem + b];
    }
}

// ---- input-row preparation ----

// Q4_K's prepared input row of n floats (n % 256 == 0). Per 256-block s: X = nearest-even(x 2^sh_s) as 4 byte
// planes; bf[8 s + j] = the exact sum of X over sub-block j (a double); scale[s] = 2^-sh_s, NaN for a block
// holding a NaN or an infinity (its X then 0). Restated from Trochilus k_q4x_prep (src/kernels/kernels.c:200-239)
// and tr_q4x_shift (src/kernels/kernels_internal.h:150-166).
// The planes are laid out for the warps that read them: a row's blocks go in passes of up to 8 (pass P: blocks
// 8P .. 8P + NB - 1), read by NL = 4 NB lanes, lane L = 4 (s mod 8) + c taking chunk c (64 inputs) of block s as
// 16 words-of-4: its q-th 16 bytes sit at words 2048 P + 4 (q NL + L), so that every 16-byte load of a warp is
// one contiguous NL x 16 bytes. Word j = 16 p + g of a lane holds byte p of X at elements 256 s + 64 c + 4 g .. +3.
__host__ __device__ inline int trx_q4x_lanes(int s, int nsb) {
    const int nb = nsb - (s & ~7);
    return 4 * (nb < 8 ? nb : 8);
}

// 2^n as a double from its bits, for the exponents the preparation takes (|n| < 1022): the same value as
// ldexp(1.0, n), without its library call
__device__ __forceinline__ double trx_pow2d(int n) { return __longlong_as_double((long long)(1023 + n) << 52); }

// The integer form of a 256-block of x, by one warp: lane L holds elements 8 L .. 8 L + 7 in v and gets their
// X = nearest-even(x 2^sh) (0 in a block holding a NaN or an infinity, which sets bad), the block's shift sh chosen
// from max|x| so that every |X| stays at most 2085998640 (Trochilus tr_q4x_shift, src/kernels/kernels_internal.h:
// 150-166, and k_q4x_prep, src/kernels/kernels.c:200-239).
__device__ __forceinline__ void trx_q4x_digitise(const float (&v)[8], int32_t (&X)[8], int &sh, int &bad) {
    float m = 0.0f;
    bad = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const float av = fabsf(v[i]);
        if (!(av <= 3.40282347e38f)) bad = 1;
        else m = fmaxf(m, av);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        bad |= __shfl_xor_sync(0xffffffffu, bad, o);
    }
    sh = 0;
    if (!bad && m != 0.0f) {
        const uint32_t mb = __float_as_uint(m);
        const int field = (int)((mb >> 23) & 255u);
        const int e = field ? field - 126 : (32 - __clz((int)(mb & 0x7fffffu))) - 149;
        sh = 31 - e;
        // m 2^sh is exact in double (a power of two times a float)
        if (__dmul_rn((double)m, trx_pow2d(sh)) > 2085998640.0) sh--;
    }
    const double f = bad ? 0.0 : trx_pow2d(sh);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const double t = __dmul_rn((double)v[i], f); // exact
        X[i] = bad ? 0 : (int32_t)__double2ll_rn(t);   // nearest, ties to even
    }
}

// One warp per 256-block; lane L takes elements 8 L .. 8 L + 7. CG: read x through L2 only (a row another CTA of
// the same kernel wrote). planes_row, bf_blk, sc_blk: the row's planes, the block's sums and scale.
template <bool CG = false>
__device__ __noinline__ void trx_prep_q4x_block(const float *__restrict__ x, uint32_t *__restrict__ planes_row, int s,
                                                   int nsb, double *__restrict__ bf_blk, double *__restrict__ sc_blk,
                                                   int lane) {
    float v[8];
    const float4 a = trx_ldx<CG>(x + 8 * lane);
    const float4 b = trx_ldx<CG>(x + 8 * lane + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    int32_t X[8];
    int sh, bad;
    trx_q4x_digitise(v, X, sh, bad);
    // sub-block sums: sub-block j holds lanes 4 j .. 4 j + 3
    int64_t sum = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) sum += X[i];
    sum += trx_shfl_xor64(sum, 1);
    sum += trx_shfl_xor64(sum, 2);
    if ((lane & 3) == 0) bf_blk[lane >> 2] = (double)sum;
    if (lane == 0) sc_blk[0] = bad ? __longlong_as_double(0x7ff8000000000000ll) : trx_pow2d(-sh);
    // this lane's 8 elements: chunk c = lane / 8, groups g, g + 1 (g = 2 (lane % 8)) of consumer lane 4 (s % 8) + c
    const int c = lane >> 3, g = 2 * (lane & 7), NL = trx_q4x_lanes(s, nsb), L = 4 * (s & 7) + c;
    uint32_t *pass = planes_row + 2048 * (s >> 3);
#pragma unroll
    for (int p = 0; p < 4; p++) {
        uint32_t w0 = 0, w1 = 0;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            w0 |= (((uint32_t)X[i] >> (8 * p)) & 255u) << (8 * i);
            w1 |= (((uint32_t)X[4 + i] >> (8 * p)) & 255u) << (8 * i);
        }
        const int j = 16 * p + g; // g even: words j and j + 1 share a 16-byte group
        *reinterpret_cast<uint2 *>(pass + 4 * ((j >> 2) * NL + L) + (j & 3)) = make_uint2(w0, w1);
    }
}

// ---- dot products ----

// a 16-byte (8-, 4-, 2-byte) load from global memory through the read-only path, or a plain load
// (shared memory: SM = true)
template <bool SM, typename V>
__device__ __forceinline__ V trx_ld(const void *p) {
    if (SM) return *reinterpret_cast<const V *>(p);
    return __ldg(reinterpret_cast<const V *>(p));
}

// Q4_K: the 4 * G lanes of a row group hold G blocks (lane: block s = lane/4 % G, chunk c = lane % 4)
struct TrxQ4X {
    uint32_t w[4][16]; // the thread's 64 inputs as 4 byte planes x 16 words
    int64_t b[2];      // the sums of X over its chunk's sub-blocks 2c and 2c + 1 (exact integers)
    double sc;         // its block's 2^-sh (NaN for a block holding a NaN or an infinity)
};

// The thread's share of a prepared row (trx_prep_q4x_block's layout): lane L of NL reading the pass whose planes
// start at pass_planes, and its block's sub-block sums (bf_blk[0..7]) and scale (*sc_blk). CG: through L2 only
// (__ldcg), for a row another CTA of the same kernel wrote.
template <bool CG = false>
__device__ __forceinline__ void trx_q4x_load(const uint32_t *__restrict__ pass_planes, int NL, int L,
                                             const double *__restrict__ bf_blk, const double *__restrict__ sc_blk,
                                             TrxQ4X &X) {
    const int c = L & 3;
    X.b[0] = trx_d2i(CG ? __ldcg(bf_blk + 2 * c) : bf_blk[2 * c]);
    X.b[1] = trx_d2i(CG ? __ldcg(bf_blk + 2 * c + 1) : bf_blk[2 * c + 1]);
    X.sc = CG ? __ldcg(sc_blk) : *sc_blk;
    const uint4 *src = reinterpret_cast<const uint4 *>(pass_planes) + L;
#pragma unroll
    for (int q = 0; q < 16; q++) {
        const uint4 v = CG ? __ldcg(src + q * NL) : src[q * NL];
        X.w[q >> 2][4 * (q & 3) + 0] = v.x;
        X.w[q >> 2][4 * (q & 3) + 1] = v.y;
        X.w[q >> 2][4 * (q & 3) + 2] = v.z;
        X.w[q >> 2][4 * (q & 3) + 3] = v.w;
    }
}

// One thread's part of a block's T = sum_j sc_j sum q X and M = sum_j m_j sum X, for its 32-byte chunk c (sub-blocks
// 2c: the low nibbles, 2c + 1: the high nibbles) of a block whose header is hdr and quants q0, q1. Both are exact
// integers, so the four chunks' parts add in any order.
__device__ __forceinline__ void trx_q4k_chunk(uint4 hdr, uint4 q0, uint4 q1, int c, const TrxQ4X &X, int64_t &T,
                                              int64_t &M) {
    const uint32_t words[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    uint32_t alo[3] = {0, 0, 0}, ahi[3] = {0, 0, 0};
    int slo = 0, shi = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t lo = words[i] & 0x0f0f0f0fu, hi = (words[i] >> 4) & 0x0f0f0f0fu;
#pragma unroll
        for (int p = 0; p < 3; p++) {
            alo[p] = __dp4a(lo, X.w[p][i], alo[p]);
            ahi[p] = __dp4a(hi, X.w[p][8 + i], ahi[p]);
        }
        slo = __dp4a((int)lo, (int)X.w[3][i], slo);
        shi = __dp4a((int)hi, (int)X.w[3][8 + i], shi);
    }
    // the 6-bit scales and mins of sub-blocks 2c, 2c + 1 from the 12 packed bytes (header words y, z, w):
    // j < 4: sc = byte j & 63, m = byte j + 4 & 63; j >= 4: the low (sc) or high (m) nibble of byte j + 4 and the top
    // two bits of byte j - 4 (sc) or byte j (m)
    const int sh = 16 * (c & 1);
    const uint32_t y2 = hdr.y >> sh, z2 = hdr.z >> sh, w2 = hdr.w >> sh;
    int sc0, sc1, m0, m1;
    if (c < 2) {
        sc0 = (int)(y2 & 63u);
        sc1 = (int)((y2 >> 8) & 63u);
        m0 = (int)(z2 & 63u);
        m1 = (int)((z2 >> 8) & 63u);
    } else {
        sc0 = (int)((w2 & 15u) | (((y2 >> 6) & 3u) << 4));
        sc1 = (int)(((w2 >> 8) & 15u) | (((y2 >> 14) & 3u) << 4));
        m0 = (int)(((w2 >> 4) & 15u) | (((z2 >> 6) & 3u) << 4));
        m1 = (int)(((w2 >> 12) & 15u) | (((z2 >> 14) & 3u) << 4));
    }
    const int64_t b0 = (int64_t)sc0 * alo[0] + (int64_t)sc1 * ahi[0];
    const int64_t b1 = (int64_t)sc0 * alo[1] + (int64_t)sc1 * ahi[1];
    const int64_t b2 = (int64_t)sc0 * alo[2] + (int64_t)sc1 * ahi[2];
    const int64_t b3 = (int64_t)sc0 * slo + (int64_t)sc1 * shi;
    T = b0 + (b1 << 8) + (b2 << 16) + b3 * 16777216ll;
    M = (int64_t)m0 * X.b[0] + (int64_t)m1 * X.b[1];
}

// T and M summed over the 4 threads of a block (xor 1, 2), then v = (d T - dmin M) 2^-sh in f64, in every thread
// of the group (|T| < 2^49, |M| < 2^45: exact as doubles)
__device__ __forceinline__ double trx_q4k_value(uint4 hdr, int64_t T, int64_t M, double sc) {
    T += trx_shfl_xor64(T, 1);
    M += trx_shfl_xor64(M, 1);
    T += trx_shfl_xor64(T, 2);
    M += trx_shfl_xor64(M, 2);
    const double d = trx_half_d((uint16_t)(hdr.x & 0xffffu));
    const double dmin = trx_half_d((uint16_t)(hdr.x >> 16));
    const double val = __dsub_rn(__dmul_rn(d, trx_i2d(T)), __dmul_rn(dmin, trx_i2d(M)));
    return __dmul_rn(val, sc);
}

// ---- Q4_K on the integer tensor cores (one-token decode) ----
//
// T = sum_j sc_j sum_{k in j} q_k X_k is an exact integer, so it may be formed in any order and by any exact
// means: here by mma.sync m16n8k32 (u8 quants x s8 digits, s32 sums), the 32 elements of a sub-block being one
// product's K. X is split into four balanced base-256 digits, X = D0 + 256 D1 + 65536 D2 + 2^24 D3 with every
// D_p in [-128, 127] (|X| <= 2085998640 keeps D3 within 125), which are the four columns of B (the other four are
// zero). The rows of A are 8 gate rows and the same 8 up rows of one 256-block; a high-nibble sub-block enters as
// 16 q (the byte masked in place), its sum then shifted back right by 4, exactly.
//
// The digits' layout, made for the B fragments: product K index k' of thread (g, t) (g = lane / 4, t = lane % 4)
// holds element 8 t + k' (k' < 4) or 8 t + 4 + (k' - 16) (k' >= 16) of the sub-block, the A fragments taking the
// same elements of a quant row. So thread (p, t), p < 4, reads digit plane p's elements 8 t .. 8 t + 7 of every
// sub-block: 64 bytes per block, in four 16-byte chunks (chunk q: sub-blocks 2 q and 2 q + 1), chunk q of lane
// L = 4 p + t stored at 16 (4 L + (q ^ ((L >> 1) & 3))) so that eight lanes' loads of a phase hit distinct banks.
__device__ __forceinline__ int trx_q4m_chunk_off(int L, int q) { return 16 * (4 * L + (q ^ ((L >> 1) & 3))); }

// One warp per 256-block, lane L taking elements 8 L .. 8 L + 7 (the same X as trx_prep_q4x_block): the block's
// digits (1024 bytes at dig), sub-block sums (bf_blk[0..7]) and scale (*sc_blk; NaN for a NaN or an infinity).
__device__ __noinline__ void trx_prep_q4m_block(const float *__restrict__ x, uint8_t *__restrict__ dig,
                                                double *__restrict__ bf_blk, double *__restrict__ sc_blk, int lane) {
    float v[8];
    const float4 a = *reinterpret_cast<const float4 *>(x + 8 * lane);
    const float4 b = *reinterpret_cast<const float4 *>(x + 8 * lane + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    int32_t X[8];
    int sh, bad;
    trx_q4x_digitise(v, X, sh, bad);
    int64_t sum = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) sum += X[i];
    sum += trx_shfl_xor64(sum, 1);
    sum += trx_shfl_xor64(sum, 2);
    if ((lane & 3) == 0) bf_blk[lane >> 2] = (double)sum;
    if (lane == 0) sc_blk[0] = bad ? __longlong_as_double(0x7ff8000000000000ll) : trx_pow2d(-sh);
    // balanced digits: D = ((r + 128) mod 256) - 128, r = (r - D) / 256 (exact: r - D is a multiple of 256)
    uint32_t pw[4][2] = {{0, 0}, {0, 0}, {0, 0}, {0, 0}};
#pragma unroll
    for (int i = 0; i < 8; i++) {
        int32_t r = X[i];
#pragma unroll
        for (int p = 0; p < 4; p++) {
            const int32_t d = p < 3 ? ((r + 128) & 255) - 128 : r;
            r = (r - d) >> 8;
            pw[p][i >> 2] |= ((uint32_t)d & 255u) << (8 * (i & 3));
        }
    }
    // elements 8 L .. 8 L + 7 are sub-block s = L / 4, part t = L % 4: consumer lane 4 p + t, chunk s / 2, half s % 2
    const int sb = lane >> 2, t = lane & 3;
#pragma unroll
    for (int p = 0; p < 4; p++)
        *reinterpret_cast<uint2 *>(dig + trx_q4m_chunk_off(4 * p + t, sb >> 1) + 8 * (sb & 1)) =
            make_uint2(pw[p][0], pw[p][1]);
}

// d = A (16 x 32 u8, row) x B (32 x 8 s8, col), s32, from zero
__device__ __forceinline__ void trx_mma_u8s8(int32_t (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// byte i (0..3) of w, as an int
__device__ __forceinline__ int trx_byte(uint32_t w, int i) { return (int)((w >> (8 * i)) & 255u); }

// One Q4_K block (256 columns) of 8 gate rows and the same 8 up rows against the token's digits, by one warp:
// gate, up: the rows' blocks in shared memory, 144 bytes apart (row g at 144 g); dig, bf, sc: the token's block
// (trx_prep_q4m_block). Lane 4 g gets the block's value v = (d T - dmin M) 2^-sh (f64, Trochilus's definition,
// src/kernels/kernels.c:196-253) of gate row g in vg and of up row g in vu.
__device__ __forceinline__ void trx_q4k_blk_mma(const uint8_t *__restrict__ gate, const uint8_t *__restrict__ up,
                                                const uint8_t *__restrict__ dig, const double *__restrict__ bf,
                                                double sc, int lane, double &vg, double &vu) {
    const int g = lane >> 2, t = lane & 3;
    const uint8_t *rg = gate + 144 * g, *ru = up + 144 * g;
    const uint4 hg = *reinterpret_cast<const uint4 *>(rg), hu = *reinterpret_cast<const uint4 *>(ru);
    uint4 B[4];
#pragma unroll
    for (int q = 0; q < 4; q++)
        B[q] = g < 4 ? *reinterpret_cast<const uint4 *>(dig + trx_q4m_chunk_off(lane, q)) : make_uint4(0, 0, 0, 0);
    // the 6-bit scales of sub-blocks 0..3 and 4..7 and the mins, packed a byte each (Q4_K's 12 scale bytes: j < 4:
    // sc = byte j & 63, m = byte j + 4 & 63; j >= 4: the low (sc) or high (m) nibble of byte j + 4 and the top two
    // bits of byte j - 4 (sc) or byte j (m))
    const uint32_t sg03 = hg.y & 0x3f3f3f3fu, sg47 = (hg.w & 0x0f0f0f0fu) | ((hg.y >> 2) & 0x30303030u);
    const uint32_t su03 = hu.y & 0x3f3f3f3fu, su47 = (hu.w & 0x0f0f0f0fu) | ((hu.y >> 2) & 0x30303030u);
    int32_t lo[4] = {0, 0, 0, 0}, hi[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 4; j++) { // sub-blocks 2 j (low nibbles) and 2 j + 1 (high nibbles) of bytes 32 j .. 32 j + 31
        const uint2 wg = *reinterpret_cast<const uint2 *>(rg + 16 + 32 * j + 8 * t);
        const uint2 wu = *reinterpret_cast<const uint2 *>(ru + 16 + 32 * j + 8 * t);
        const uint32_t pg = j < 2 ? sg03 : sg47, pu = j < 2 ? su03 : su47;
        const int sgl = trx_byte(pg, (2 * j) & 3), sgh = trx_byte(pg, (2 * j + 1) & 3);
        const int sul = trx_byte(pu, (2 * j) & 3), suh = trx_byte(pu, (2 * j + 1) & 3);
        const uint4 bq = B[j]; // chunk j: sub-block 2 j in x, y; 2 j + 1 in z, w
        int32_t c[4];
        trx_mma_u8s8(c, wg.x & 0x0f0f0f0fu, wu.x & 0x0f0f0f0fu, wg.y & 0x0f0f0f0fu, wu.y & 0x0f0f0f0fu, bq.x, bq.y);
        lo[0] += sgl * c[0];
        lo[1] += sgl * c[1];
        lo[2] += sul * c[2];
        lo[3] += sul * c[3];
        trx_mma_u8s8(c, wg.x & 0xf0f0f0f0u, wu.x & 0xf0f0f0f0u, wg.y & 0xf0f0f0f0u, wu.y & 0xf0f0f0f0u, bq.z, bq.w);
        hi[0] += sgh * c[0];
        hi[1] += sgh * c[1];
        hi[2] += suh * c[2];
        hi[3] += suh * c[3];
    }
    // planes 2 t and 2 t + 1 (t < 2; lanes t >= 2 hold the zero columns): the gate row's and the up row's parts
    const int64_t ag = (int64_t)(lo[0] + (hi[0] >> 4)) + 256ll * (int64_t)(lo[1] + (hi[1] >> 4));
    const int64_t au = (int64_t)(lo[2] + (hi[2] >> 4)) + 256ll * (int64_t)(lo[3] + (hi[3] >> 4));
    // (in lane t = 0: its planes 0, 1 and lane t = 1's planes 2, 3)
    const int64_t Tg = ag + 65536ll * trx_shfl_xor64(ag, 1), Tu = au + 65536ll * trx_shfl_xor64(au, 1);
    // M = sum_j m_j S_j, S_j the sub-block sums of X: lane t takes sub-blocks 2 t and 2 t + 1 (exact in f64), whose
    // mins are bytes 2 t, 2 t + 1 (mod 4) of the packed mins of sub-blocks 0..3 or 4..7
    const uint32_t mgp = t < 2 ? (hg.z & 0x3f3f3f3fu) : (((hg.w >> 4) & 0x0f0f0f0fu) | ((hg.z >> 2) & 0x30303030u));
    const uint32_t mup = t < 2 ? (hu.z & 0x3f3f3f3fu) : (((hu.w >> 4) & 0x0f0f0f0fu) | ((hu.z >> 2) & 0x30303030u));
    const int i0 = (2 * t) & 3;
    const double S0 = bf[2 * t], S1 = bf[2 * t + 1];
    double Mg = __dadd_rn(__dmul_rn((double)trx_byte(mgp, i0), S0), __dmul_rn((double)trx_byte(mgp, i0 + 1), S1));
    double Mu = __dadd_rn(__dmul_rn((double)trx_byte(mup, i0), S0), __dmul_rn((double)trx_byte(mup, i0 + 1), S1));
    Mg = __dadd_rn(Mg, __shfl_xor_sync(0xffffffffu, Mg, 1));
    Mu = __dadd_rn(Mu, __shfl_xor_sync(0xffffffffu, Mu, 1));
    Mg = __dadd_rn(Mg, __shfl_xor_sync(0xffffffffu, Mg, 2));
    Mu = __dadd_rn(Mu, __shfl_xor_sync(0xffffffffu, Mu, 2));
    const double dg = trx_half_d((uint16_t)(hg.x & 0xffffu)), dmg = trx_half_d((uint16_t)(hg.x >> 16));
    const double du = trx_half_d((uint16_t)(hu.x & 0xffffu)), dmu = trx_half_d((uint16_t)(hu.x >> 16));
    vg = __dmul_rn(__dsub_rn(__dmul_rn(dg, trx_i2d(Tg)), __dmul_rn(dmg, Mg)), sc);
    vu = __dmul_rn(__dsub_rn(__dmul_rn(du, trx_i2d(Tu)), __dmul_rn(dmu, Mu)), sc);
}

// One 256-block of the lane contract for thread l of a half-warp: its 16 elements k = 256 i + l + 16 m, m = 0..15,
// dequantised and multiplied two at a time with the paired operations (each product rounded on its own), then added
// to the thread's running sum one at a time in order of m.

// Q8L: sc = the block's 8 f16 scales (element m has scale m / 2), q = the thread's 16 quants (byte m = element m)
__device__ __forceinline__ float trx_q8l_block(float acc, uint4 sc, uint4 q, const float (&xv)[16]) {
    const uint32_t qw[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u, q.w ^ 0x80808080u};
    const uint32_t sw[4] = {sc.x, sc.y, sc.z, sc.w};
    const trx_f2 bias = trx_pack2(8388736.0f, 8388736.0f); // 2^23 + 128
#pragma unroll
    for (int m = 0; m < 16; m += 2) {
        const float d = trx_half((uint16_t)(sw[m >> 2] >> (16 * ((m >> 1) & 1))));
        // the int8 quants as floats from their bits: 2^23 + (q + 128), less 2^23 + 128 (exact)
        const trx_f2 qf = trx_sub2(trx_pack2(__uint_as_float(__byte_perm(qw[m >> 2], 0x4b000000u, 0x7440u | (m & 3))),
                                             __uint_as_float(__byte_perm(qw[m >> 2], 0x4b000000u, 0x7440u | ((m + 1) & 3)))),
                                   bias);
        const trx_f2 p = trx_mul2(trx_mul2(trx_pack2(d, d), qf), trx_pack2(xv[m], xv[m + 1]));
        acc = __fadd_rn(acc, trx_lo(p));
        acc = __fadd_rn(acc, trx_hi(p));
    }
    return acc;
}

// Q6L: the thread's 16 six-bit quants as four words of four bytes (word j: weights 4 j .. 4 j + 3), from its 8
// low-nibble bytes ql and its 4 high-bit bytes qh (the layout above)
__device__ __forceinline__ void trx_q6l_quants(uint2 ql, uint32_t qh, uint32_t (&q4)[4]) {
    q4[0] = (ql.x & 0x0f0f0f0fu) | ((qh << 4) & 0x30303030u);
    q4[1] = ((ql.x >> 4) & 0x0f0f0f0fu) | ((qh << 2) & 0x30303030u);
    q4[2] = (ql.y & 0x0f0f0f0fu) | (qh & 0x30303030u);
    q4[3] = ((ql.y >> 4) & 0x0f0f0f0fu) | ((qh >> 2) & 0x30303030u);
}

// One 256-block of a Q6L row for thread l of the half-warp, with the block's 16 sub-block scales fl(d sc_m) given
// (element m has scale m): w = scale (q - 32), exact (d has 11 significant bits, sc 8, q - 32 6); the products
// w x rounded one by one, added in order of m.
__device__ __forceinline__ float trx_q6l_block_sc(float acc, uint2 ql, uint32_t qh, const float (&scale)[16],
                                                  const float (&xv)[16]) {
    uint32_t q4[4];
    trx_q6l_quants(ql, qh, q4);
    const trx_f2 bias6 = trx_pack2(8388640.0f, 8388640.0f); // 2^23 + 32
#pragma unroll
    for (int m = 0; m < 16; m += 2) {
        // 2^23 + q as float bits (byte m & 3 of word m / 4 under the exponent of 2^23), less 2^23 + 32: q - 32
        const trx_f2 qv = trx_sub2(trx_pack2(__uint_as_float(__byte_perm(q4[m >> 2], 0x4b000000u, 0x7440u | (m & 3))),
                                             __uint_as_float(__byte_perm(q4[m >> 2], 0x4b000000u, 0x7440u | ((m + 1) & 3)))),
                                   bias6);
        const trx_f2 p = trx_mul2(trx_mul2(trx_pack2(scale[m], scale[m + 1]), qv), trx_pack2(xv[m], xv[m + 1]));
        acc = __fadd_rn(acc, trx_lo(p));
        acc = __fadd_rn(acc, trx_hi(p));
    }
    return acc;
}

// the block's 16 scales fl(d sc_m) from its int8 scales scv (sc_m in byte m) and its f16 d
__device__ __forceinline__ void trx_q6l_scales(uint4 scv, float d, float (&scale)[16]) {
    const uint32_t scw[4] = {scv.x ^ 0x80808080u, scv.y ^ 0x80808080u, scv.z ^ 0x80808080u, scv.w ^ 0x80808080u};
    const trx_f2 d2 = trx_pack2(d, d), bias8 = trx_pack2(8388736.0f, 8388736.0f); // 2^23 + 128
#pragma unroll
    for (int m = 0; m < 16; m += 2) {
        const trx_f2 scf = trx_sub2(trx_pack2(__uint_as_float(__byte_perm(scw[m >> 2], 0x4b000000u, 0x7440u | (m & 3))),
                                              __uint_as_float(__byte_perm(scw[m >> 2], 0x4b000000u, 0x7440u | ((m + 1) & 3)))),
                                    bias8);
        const trx_f2 sc = trx_mul2(d2, scf); // exact
        scale[m] = trx_lo(sc);
        scale[m + 1] = trx_hi(sc);
    }
}

// Q6L: ql, qh = the thread's low nibbles and high bit pairs, scv = the block's 16 int8 sub-block scales (element m
// has scale m), d = the block's f16 d
__device__ __forceinline__ float trx_q6l_block(float acc, uint2 ql, uint32_t qh, uint4 scv, float d, const float (&xv)[16]) {
    float scale[16];
    trx_q6l_scales(scv, d, scale);
    return trx_q6l_block_sc(acc, ql, qh, scale, xv);
}

// the thread's 16 inputs of block i of an LC-ordered row
template <bool CG>
__device__ __forceinline__ void trx_lc_block(const float *__restrict__ xlc, int i, int l, float (&xv)[16]) {
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const float4 v = trx_ldx<CG>(xlc + 256 * i + 64 * q + 4 * l);
        xv[4 * q] = v.x;
        xv[4 * q + 1] = v.y;
        xv[4 * q + 2] = v.z;
        xv[4 * q + 3] = v.w;
    }
}

// Q8L lane-contract dot of one row (n = 256 * nch) against an LC-ordered input row; thread l of the
// half-warp. Returns the tree sum (same in all 16 threads).
template <bool SM = false, bool CG = false>
__device__ __forceinline__ float trx_q8l_dot(const uint8_t *__restrict__ row, const float *__restrict__ xlc, int nch,
                                             int l) {
    float acc = 0.0f;
    for (int i = 0; i < nch; i++) {
        float xv[16];
        trx_lc_block<CG>(xlc, i, l, xv);
        acc = trx_q8l_block(acc, trx_ld<SM, uint4>(row + 272 * i), trx_ld<SM, uint4>(row + 272 * i + 16 + 16 * l), xv);
    }
    return trx_lane_tree16(acc);
}

// Q6L lane-contract dot (n = 256 * nsb); dptr: this row's nsb f16 d values (in shared memory when DSM)
template <bool SM = false, bool CG = false, bool DSM = false>
__device__ __forceinline__ float trx_q6l_dot(const uint8_t *__restrict__ row, const uint8_t *__restrict__ dptr,
                                             const float *__restrict__ xlc, int nsb, int l) {
    float acc = 0.0f;
    for (int s = 0; s < nsb; s++) {
        float xv[16];
        trx_lc_block<CG>(xlc, s, l, xv);
        acc = trx_q6l_block(acc, trx_ld<SM, uint2>(row + 128 * s + 8 * l), trx_ld<SM, uint32_t>(row + 128 * nsb + 64 * s + 4 * l),
                            trx_ld<SM, uint4>(row + 192 * nsb + 16 * s),
                            trx_half(DSM ? reinterpret_cast<const uint16_t *>(dptr)[s]
                                         : __ldg(reinterpret_cast<const uint16_t *>(dptr) + s)), xv);
    }
    return trx_lane_tree16(acc);
}

// Two Q6L rows a and b (in shared memory, each with its own LC-ordered input row xa, xb and d values da, db), thread l
// of a half-warp: the products of the two rows' element m are formed together by paired operations (each half rounded
// on its own), and each row's chain adds them with scalar additions, so each row's products and sums are exactly the
// single-row road's, in the same order. (A paired addition in the chains gave other bits on sm_100: measured, 239 of
// 256 random row pairs differed from the scalar chain; the chains therefore stay scalar.) The rows' scales are
// computed once into the half-warp's scratch ss (32 nsb floats: row a's, then row b's). Both half-warps of the warp
// call it together (it synchronises the warp). nsb <= TRX_Q6L_SS_BLOCKS.
#define TRX_Q6L_SS_BLOCKS 4
__device__ __noinline__ float2 trx_q6l_dot_pair(const uint8_t *__restrict__ ra, const uint8_t *__restrict__ da,
                                                const float *__restrict__ xa, const uint8_t *__restrict__ rb,
                                                const uint8_t *__restrict__ db, const float *__restrict__ xb, int nsb,
                                                int l, float *__restrict__ ss) {
    float *ssb = ss + 16 * TRX_Q6L_SS_BLOCKS;
    for (int s = 0; s < nsb; s++) {
        const float sca = (float)reinterpret_cast<const int8_t *>(ra + 192 * nsb + 16 * s)[l]; // exact
        const float scb = (float)reinterpret_cast<const int8_t *>(rb + 192 * nsb + 16 * s)[l];
        ss[16 * s + l] = __fmul_rn(trx_half(reinterpret_cast<const uint16_t *>(da)[s]), sca); // exact
        ssb[16 * s + l] = __fmul_rn(trx_half(reinterpret_cast<const uint16_t *>(db)[s]), scb);
    }
    __syncwarp();
    float aa = 0.0f, ab = 0.0f;
    const trx_f2 bias6 = trx_pack2(8388640.0f, 8388640.0f); // 2^23 + 32
#pragma unroll 1
    for (int s = 0; s < nsb; s++) {
        float xva[16], xvb[16], sa[16], sb[16];
        trx_lc_block<false>(xa, s, l, xva);
        trx_lc_block<false>(xb, s, l, xvb);
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const float4 u = *reinterpret_cast<const float4 *>(ss + 16 * s + 4 * q);
            const float4 v = *reinterpret_cast<const float4 *>(ssb + 16 * s + 4 * q);
            sa[4 * q] = u.x; sa[4 * q + 1] = u.y; sa[4 * q + 2] = u.z; sa[4 * q + 3] = u.w;
            sb[4 * q] = v.x; sb[4 * q + 1] = v.y; sb[4 * q + 2] = v.z; sb[4 * q + 3] = v.w;
        }
        uint32_t qa[4], qb[4];
        trx_q6l_quants(*reinterpret_cast<const uint2 *>(ra + 128 * s + 8 * l),
                       *reinterpret_cast<const uint32_t *>(ra + 128 * nsb + 64 * s + 4 * l), qa);
        trx_q6l_quants(*reinterpret_cast<const uint2 *>(rb + 128 * s + 8 * l),
                       *reinterpret_cast<const uint32_t *>(rb + 128 * nsb + 64 * s + 4 * l), qb);
#pragma unroll
        for (int m = 0; m < 16; m++) {
            const uint32_t sel = 0x7440u | (m & 3);
            const trx_f2 qv = trx_sub2(trx_pack2(__uint_as_float(__byte_perm(qa[m >> 2], 0x4b000000u, sel)),
                                                 __uint_as_float(__byte_perm(qb[m >> 2], 0x4b000000u, sel))),
                                       bias6); // (q_a - 32, q_b - 32)
            const trx_f2 p = trx_mul2(trx_mul2(trx_pack2(sa[m], sb[m]), qv), trx_pack2(xva[m], xvb[m]));
            aa = __fadd_rn(aa, trx_lo(p));
            ab = __fadd_rn(ab, trx_hi(p));
        }
    }
    __syncwarp(); // the scratch is free for the warp's next rows
    return make_float2(trx_lane_tree16(aa), trx_lane_tree16(ab));
}

// The interleaved layout of two LC-ordered input rows a, b (trx_q6l_dot_pair_il): within each 64-position group g,
// thread l's positions 4l, 4l+1 as (a, b, a, b) at float offset 128 g + 4 l and 4l+2, 4l+3 at 128 g + 64 + 4 l, so
// that each 16-byte load of a half-warp reads 256 contiguous bytes and yields two ready pairs.
__host__ __device__ inline int trx_il_off(int p) {
    return 128 * (p >> 6) + 64 * ((p & 3) >> 1) + 4 * ((p >> 2) & 15) + 2 * (p & 1);
}

// trx_q6l_dot_pair with both operands laid out for the paired operations: xab holds the rows' inputs interleaved
// (trx_il_off; row a's at even offsets, row b's at odd ones) and the scratch ss receives the scales as pairs
// (sa_m, sb_m), so no value is moved to form a pair; NSB (1, 2 or 4 blocks) unrolled. Same products, same order of
// additions, same bits. (The chains stay scalar: ptxas fuses a paired multiply feeding a paired addition into a
// paired fma, explicit rounding notwithstanding; measured.)
template <int NSB>
__device__ __noinline__ float2 trx_q6l_dot_pair_il(const uint8_t *__restrict__ ra, const uint8_t *__restrict__ da,
                                                   const uint8_t *__restrict__ rb, const uint8_t *__restrict__ db,
                                                   const float *__restrict__ xab, int l, float *__restrict__ ss) {
#pragma unroll
    for (int s = 0; s < NSB; s++) {
        const float sca = (float)reinterpret_cast<const int8_t *>(ra + 192 * NSB + 16 * s)[l]; // exact
        const float scb = (float)reinterpret_cast<const int8_t *>(rb + 192 * NSB + 16 * s)[l];
        *reinterpret_cast<float2 *>(ss + 2 * (16 * s + l)) =
            make_float2(__fmul_rn(trx_half(reinterpret_cast<const uint16_t *>(da)[s]), sca),
                        __fmul_rn(trx_half(reinterpret_cast<const uint16_t *>(db)[s]), scb)); // exact
    }
    __syncwarp();
    float aa = 0.0f, ab = 0.0f;
    const trx_f2 bias6 = trx_pack2(8388640.0f, 8388640.0f); // 2^23 + 32
#pragma unroll
    for (int s = 0; s < NSB; s++) {
        trx_f2 xv[16], sv[16];
#pragma unroll
        for (int q = 0; q < 4; q++) { // element 4 q + j: position 256 s + 64 q + 4 l + j
            const ulonglong2 u = *reinterpret_cast<const ulonglong2 *>(xab + 128 * (4 * s + q) + 4 * l);
            const ulonglong2 v = *reinterpret_cast<const ulonglong2 *>(xab + 128 * (4 * s + q) + 64 + 4 * l);
            xv[4 * q] = u.x;
            xv[4 * q + 1] = u.y;
            xv[4 * q + 2] = v.x;
            xv[4 * q + 3] = v.y;
        }
#pragma unroll
        for (int q = 0; q < 8; q++) {
            const ulonglong2 u = *reinterpret_cast<const ulonglong2 *>(ss + 2 * (16 * s + 2 * q));
            sv[2 * q] = u.x;
            sv[2 * q + 1] = u.y;
        }
        uint32_t qa[4], qb[4];
        trx_q6l_quants(*reinterpret_cast<const uint2 *>(ra + 128 * s + 8 * l),
                       *reinterpret_cast<const uint32_t *>(ra + 128 * NSB + 64 * s + 4 * l), qa);
        trx_q6l_quants(*reinterpret_cast<const uint2 *>(rb + 128 * s + 8 * l),
                       *reinterpret_cast<const uint32_t *>(rb + 128 * NSB + 64 * s + 4 * l), qb);
#pragma unroll
        for (int m = 0; m < 16; m++) {
            const uint32_t sel = 0x7440u | (m & 3);
            const trx_f2 qv = trx_sub2(trx_pack2(__uint_as_float(__byte_perm(qa[m >> 2], 0x4b000000u, sel)),
                                                 __uint_as_float(__byte_perm(qb[m >> 2], 0x4b000000u, sel))),
                                       bias6); // (q_a - 32, q_b - 32)
            const trx_f2 p = trx_mul2(trx_mul2(sv[m], qv), xv[m]);
            aa = __fadd_rn(aa, trx_lo(p));
            ab = __fadd_rn(ab, trx_hi(p));
        }
    }
    __syncwarp(); // the scratch is free for the warp's next rows
    return make_float2(trx_lane_tree16(aa), trx_lane_tree16(ab));
}

// The Q8L counterpart of trx_q6l_dot_pair_il: rows a and b in the Q8L layout (272 bytes a 256-block: the block's
// 8 f16 scales, then its quants in position order, thread l's 16 at bytes 16 l ..), the inputs interleaved
// (trx_il_off). Element m of thread l has scale m / 2; w = fl(d q) (exact), the product fl(w x) rounded, added in
// order of m: trx_q8l_block's arithmetic for each row. NSB: 1, 2 or 4 blocks.
template <int NSB>
__device__ __noinline__ float2 trx_q8l_dot_pair_il(const uint8_t *__restrict__ ra, const uint8_t *__restrict__ rb,
                                                   const float *__restrict__ xab, int l) {
    float aa = 0.0f, ab = 0.0f;
    const trx_f2 bias = trx_pack2(8388736.0f, 8388736.0f); // 2^23 + 128
#pragma unroll
    for (int s = 0; s < NSB; s++) {
        trx_f2 xv[16], dv[8];
#pragma unroll
        for (int q = 0; q < 4; q++) { // element 4 q + j: position 256 s + 64 q + 4 l + j
            const ulonglong2 u = *reinterpret_cast<const ulonglong2 *>(xab + 128 * (4 * s + q) + 4 * l);
            const ulonglong2 v = *reinterpret_cast<const ulonglong2 *>(xab + 128 * (4 * s + q) + 64 + 4 * l);
            xv[4 * q] = u.x;
            xv[4 * q + 1] = u.y;
            xv[4 * q + 2] = v.x;
            xv[4 * q + 3] = v.y;
        }
        const uint4 ha = *reinterpret_cast<const uint4 *>(ra + 272 * s), hb = *reinterpret_cast<const uint4 *>(rb + 272 * s);
        const uint32_t wa[4] = {ha.x, ha.y, ha.z, ha.w}, wb[4] = {hb.x, hb.y, hb.z, hb.w};
#pragma unroll
        for (int i = 0; i < 8; i++) // (d_a, d_b) of scale i
            dv[i] = trx_pack2(trx_half((uint16_t)(wa[i >> 1] >> (16 * (i & 1)))), trx_half((uint16_t)(wb[i >> 1] >> (16 * (i & 1)))));
        const uint4 qa4 = *reinterpret_cast<const uint4 *>(ra + 272 * s + 16 + 16 * l);
        const uint4 qb4 = *reinterpret_cast<const uint4 *>(rb + 272 * s + 16 + 16 * l);
        const uint32_t qa[4] = {qa4.x ^ 0x80808080u, qa4.y ^ 0x80808080u, qa4.z ^ 0x80808080u, qa4.w ^ 0x80808080u};
        const uint32_t qb[4] = {qb4.x ^ 0x80808080u, qb4.y ^ 0x80808080u, qb4.z ^ 0x80808080u, qb4.w ^ 0x80808080u};
#pragma unroll
        for (int m = 0; m < 16; m++) {
            const uint32_t sel = 0x7440u | (m & 3);
            const trx_f2 qv = trx_sub2(trx_pack2(__uint_as_float(__byte_perm(qa[m >> 2], 0x4b000000u, sel)),
                                                 __uint_as_float(__byte_perm(qb[m >> 2], 0x4b000000u, sel))),
                                       bias); // (q_a, q_b), exact
            const trx_f2 p = trx_mul2(trx_mul2(dv[m >> 1], qv), xv[m]);
            aa = __fadd_rn(aa, trx_lo(p));
            ab = __fadd_rn(ab, trx_hi(p));
        }
    }
    return make_float2(trx_lane_tree16(aa), trx_lane_tree16(ab));
}

// Two rows (a, b in shared memory) of the same width against one LC-ordered input row read through L1 (each
// 256-block's inputs loaded once for both rows), one 256-block an iteration (a small loop body). Q6L: da, db the
// rows' f16 d values in shared memory. Returns both tree sums (the same in all 16 threads of the half-warp).
__device__ __forceinline__ float2 trx_q6l_dot2(const uint8_t *__restrict__ ra, const uint8_t *__restrict__ rb,
                                               const uint8_t *__restrict__ da, const uint8_t *__restrict__ db,
                                               const float *__restrict__ xlc, int nsb, int l) {
    float aa = 0.0f, ab = 0.0f;
#pragma unroll 1
    for (int s = 0; s < nsb; s++) {
        float xv[16];
        trx_lc_block<false>(xlc, s, l, xv);
        aa = trx_q6l_block(aa, *reinterpret_cast<const uint2 *>(ra + 128 * s + 8 * l),
                           *reinterpret_cast<const uint32_t *>(ra + 128 * nsb + 64 * s + 4 * l),
                           *reinterpret_cast<const uint4 *>(ra + 192 * nsb + 16 * s),
                           trx_half(reinterpret_cast<const uint16_t *>(da)[s]), xv);
        ab = trx_q6l_block(ab, *reinterpret_cast<const uint2 *>(rb + 128 * s + 8 * l),
                           *reinterpret_cast<const uint32_t *>(rb + 128 * nsb + 64 * s + 4 * l),
                           *reinterpret_cast<const uint4 *>(rb + 192 * nsb + 16 * s),
                           trx_half(reinterpret_cast<const uint16_t *>(db)[s]), xv);
    }
    return make_float2(trx_lane_tree16(aa), trx_lane_tree16(ab));
}

__device__ __forceinline__ float2 trx_q8l_dot2(const uint8_t *__restrict__ ra, const uint8_t *__restrict__ rb,
                                               const float *__restrict__ xlc, int nch, int l) {
    float aa = 0.0f, ab = 0.0f;
#pragma unroll 1
    for (int i = 0; i < nch; i++) {
        float xv[16];
        trx_lc_block<false>(xlc, i, l, xv);
        aa = trx_q8l_block(aa, *reinterpret_cast<const uint4 *>(ra + 272 * i),
                           *reinterpret_cast<const uint4 *>(ra + 272 * i + 16 + 16 * l), xv);
        ab = trx_q8l_block(ab, *reinterpret_cast<const uint4 *>(rb + 272 * i),
                           *reinterpret_cast<const uint4 *>(rb + 272 * i + 16 + 16 * l), xv);
    }
    return make_float2(trx_lane_tree16(aa), trx_lane_tree16(ab));
}

// The thread's 16 inputs of each of NCH 256-chunks of an LC-ordered row, in registers (CG: through L2)
template <int NCH, bool CG>
__device__ __forceinline__ void trx_lc_load(const float *__restrict__ xlc, int l, float (&xr)[NCH * 16]) {
#pragma unroll
    for (int i = 0; i < NCH; i++)
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const float4 v = trx_ldx<CG>(xlc + 256 * i + 64 * q + 4 * l);
            xr[16 * i + 4 * q] = v.x;
            xr[16 * i + 4 * q + 1] = v.y;
            xr[16 * i + 4 * q + 2] = v.z;
            xr[16 * i + 4 * q + 3] = v.w;
        }
}

// trx_q8l_dot / trx_q6l_dot of a row in shared memory against inputs already in registers
template <int NCH>
__device__ __forceinline__ float trx_q8l_dot_reg(const uint8_t *__restrict__ row, const float (&xr)[NCH * 16], int l) {
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < NCH; i++) {
        float xv[16];
#pragma unroll
        for (int m = 0; m < 16; m++) xv[m] = xr[16 * i + m];
        acc = trx_q8l_block(acc, *reinterpret_cast<const uint4 *>(row + 272 * i),
                            *reinterpret_cast<const uint4 *>(row + 272 * i + 16 + 16 * l), xv);
    }
    return trx_lane_tree16(acc);
}

template <int NSB, bool DSM = false>
__device__ __forceinline__ float trx_q6l_dot_reg(const uint8_t *__restrict__ row, const uint8_t *__restrict__ dptr,
                                                 const float (&xr)[NSB * 16], int l) {
    float acc = 0.0f;
#pragma unroll
    for (int s = 0; s < NSB; s++) {
        float xv[16];
#pragma unroll
        for (int m = 0; m < 16; m++) xv[m] = xr[16 * s + m];
        acc = trx_q6l_block(acc, *reinterpret_cast<const uint2 *>(row + 128 * s + 8 * l),
                            *reinterpret_cast<const uint32_t *>(row + 128 * NSB + 64 * s + 4 * l),
                            *reinterpret_cast<const uint4 *>(row + 192 * NSB + 16 * s),
                            trx_half(DSM ? reinterpret_cast<const uint16_t *>(dptr)[s]
                                         : __ldg(reinterpret_cast<const uint16_t *>(dptr) + s)), xv);
    }
    return trx_lane_tree16(acc);
}

// F32 / F16 / BF16 row, natural-order input, thread l of the half-warp (n % 16 == 0)
template <int TYPE>
__device__ __forceinline__ float trx_plain_dot(const uint8_t *__restrict__ row, const float *__restrict__ x, int n,
                                               int l) {
    float acc = 0.0f;
    for (int k = l; k < n; k += 16) {
        float w;
        if (TYPE == TRX_F32) w = __ldg(reinterpret_cast<const float *>(row) + k);
        else if (TYPE == TRX_F16) w = trx_half(__ldg(reinterpret_cast<const uint16_t *>(row) + k));
        else w = trx_bf16(__ldg(reinterpret_cast<const uint16_t *>(row) + k));
        acc = __fadd_rn(acc, __fmul_rn(w, x[k]));
    }
    return trx_lane_tree16(acc);
}
