// common.cuh: shared device helpers for the MoE-layer kernels (sm_100a).
//
// Exactness: every float and double operation on an exact path is written with an explicit
// rounding intrinsic (__fadd_rn, __fmul_rn, __fdiv_rn, __dadd_rn, ...). The compiler never fuses
// those into FMAs, which is what the reference's 16-lane contract requires (Trochilus
// src/kernels/kernels.h:3-22: separate multiply and add, each rounded). The library is also built
// with -fmad=false, so plain float expressions are not contracted either.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

#define TRX_LANES 16

// ggml type numbers (Trochilus src/format/gguf.h:16-27)
enum : int { TRX_F32 = 0, TRX_F16 = 1, TRX_Q8_0 = 8, TRX_Q4_K = 12, TRX_Q6_K = 14, TRX_BF16 = 30 };

// IEEE half to float and to double, exact (every half is a float): the conversion instruction, which takes no
// branch for the rare classes (subnormals, infinities, NaNs)
__device__ __forceinline__ float trx_half(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ double trx_half_d(uint16_t h) { return (double)__half2float(__ushort_as_half(h)); }

// Two floats in one 64-bit register and the sm_100 paired operations on them: each half rounded to nearest even
// on its own, exactly as the scalar __fadd_rn / __fsub_rn / __fmul_rn would (no contraction, subnormals kept)
typedef unsigned long long trx_f2;
__device__ __forceinline__ trx_f2 trx_pack2(float lo, float hi) {
    return (trx_f2)__float_as_uint(lo) | ((trx_f2)__float_as_uint(hi) << 32);
}
__device__ __forceinline__ float trx_lo(trx_f2 v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float trx_hi(trx_f2 v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ trx_f2 trx_mul2(trx_f2 a, trx_f2 b) {
    trx_f2 d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ trx_f2 trx_sub2(trx_f2 a, trx_f2 b) {
    trx_f2 d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// an integer |v| < 2^51 to double and back, exactly, through the 1.5 * 2^52 bias (integer and double adds only)
__device__ __forceinline__ double trx_i2d(int64_t v) {
    return __dsub_rn(__longlong_as_double(v + 0x4338000000000000ll), 6755399441055744.0);
}
__device__ __forceinline__ int64_t trx_d2i(double x) {
    return __double_as_longlong(__dadd_rn(x, 6755399441055744.0)) - 0x4338000000000000ll;
}
__device__ __forceinline__ float trx_bf16(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

// The 16-lane tree ((l0+l1)+(l2+l3))+((l4+l5)+(l6+l7)), same for 8..15, halves last
// (Trochilus src/kernels/kernels_internal.h:219-230), over the 16 threads of an aligned
// half-warp holding one lane each: xor 1 pairs (l0,l1), xor 2 pairs the pair sums, and so on.
// Float addition is commutative, so a + b == b + a bit for bit and every thread ends with the
// same tree sum.
__device__ __forceinline__ float trx_lane_tree16(float v) {
    v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
    v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
    v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
    v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 8));
    return v;
}

__device__ __forceinline__ int64_t trx_shfl_xor64(int64_t v, int m) {
    int lo = (int)(uint32_t)(uint64_t)v, hi = (int)(uint32_t)((uint64_t)v >> 32);
    lo = __shfl_xor_sync(0xffffffffu, lo, m);
    hi = __shfl_xor_sync(0xffffffffu, hi, m);
    return (int64_t)(((uint64_t)(uint32_t)hi << 32) | (uint32_t)lo);
}

__device__ __forceinline__ double trx_shfl_d(double v, int src) {
    return __shfl_sync(0xffffffffu, v, src);
}

// the byte of a packed int8 (two's complement) as float, exactly: 2^23 + (q + 128) built from bits,
// less 2^23 + 128 (both exact, the difference exact)
__device__ __forceinline__ float trx_s8_to_f32(uint32_t word_xor80, int byte) {
    uint32_t b = __byte_perm(word_xor80, 0x4b000000u, 0x7440u | (uint32_t)byte);
    return __fsub_rn(__uint_as_float(b), 8388736.0f);
}

struct TrxError {
    // written by kernels that give up on a bounded wait; read and cleared by the host
    int code;
    int where;
};
