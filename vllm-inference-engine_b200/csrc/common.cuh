// Shared device helpers for the pagedkv sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/pagedkv.h"

namespace pagedkv {

// Kernels never trap on a bad index: they skip the access and OR a
// PAGEDKV_EFLAG_* bit into the device error word whose address the ABI layer
// passes in (see pagedkv_read_error_flags).
__device__ __forceinline__ void set_error(unsigned int *err, unsigned int bit) {
  atomicOr(err, bit);
}

// 16-byte streaming load through the read-only path. The KV pool is read once
// per decode call, so it is marked evict-first in L1.
__device__ __forceinline__ uint4 ldg_stream16(const void *p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint4 ldg16(const void *p) {
  return __ldg(reinterpret_cast<const uint4 *>(p));
}

__device__ __forceinline__ void stg16(void *p, uint4 v) {
  *reinterpret_cast<uint4 *>(p) = v;
}

// Element type traits: unpack 8 packed 16-bit values into fp32 and pack back.
template <typename T> struct Elem;

template <> struct Elem<__half> {
  static constexpr int kDtype = PAGEDKV_DTYPE_F16;
  __device__ __forceinline__ static void unpack8(const uint4 &r, float (&f)[8]) {
    const __half2 *h = reinterpret_cast<const __half2 *>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 v = __half22float2(h[i]);
      f[2 * i] = v.x;
      f[2 * i + 1] = v.y;
    }
  }
  __device__ __forceinline__ static uint4 pack8(const float (&f)[8]) {
    uint4 r;
    __half2 *h = reinterpret_cast<__half2 *>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    return r;
  }
  __device__ __forceinline__ static float to_float(__half x) { return __half2float(x); }
  __device__ __forceinline__ static __half from_float(float x) { return __float2half_rn(x); }
};

template <> struct Elem<__nv_bfloat16> {
  static constexpr int kDtype = PAGEDKV_DTYPE_BF16;
  __device__ __forceinline__ static void unpack8(const uint4 &r, float (&f)[8]) {
    const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 v = __bfloat1622float2(h[i]);
      f[2 * i] = v.x;
      f[2 * i + 1] = v.y;
    }
  }
  __device__ __forceinline__ static uint4 pack8(const float (&f)[8]) {
    uint4 r;
    __nv_bfloat162 *h = reinterpret_cast<__nv_bfloat162 *>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    return r;
  }
  __device__ __forceinline__ static float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ __forceinline__ static __nv_bfloat16 from_float(float x) { return __float2bfloat16_rn(x); }
};

// transformers' apply_rotary_pos_emb, x * cos + rotate_half(x) * sin, on
// packed 16-bit pairs, rounded exactly as its 16-bit tensor ops:
// r(r(x * c) + r(xp' * s)), with xp' the rotation partner xp, negated when
// `lo` (the first half of the head). Each op is one correctly rounded f16x2 /
// bf16x2 instruction (explicit .rn, so nothing is contracted into an fma),
// which equals the fp32 form of the tensor ops (products rounded to T, summed
// in fp32, the sum rounded to T): the product of two 16-bit values is exact
// in fp32 (for bf16 products below fp32's normal range the significand
// product has under 16 bits, so rounding it to fp32 first changes no bf16
// rounding), and an fp32 sum rounded to 16 bits is the correctly rounded
// 16-bit sum (24 >= 2 * 11 + 2). Shared by every kernel that rotates, so their
// results are bit-identical.
template <typename T>
__device__ __forceinline__ uint32_t mul2_rn(uint32_t a, uint32_t b) {
  uint32_t r;
  if constexpr (Elem<T>::kDtype == PAGEDKV_DTYPE_F16)
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  else
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

template <typename T>
__device__ __forceinline__ uint32_t add2_rn(uint32_t a, uint32_t b) {
  uint32_t r;
  if constexpr (Elem<T>::kDtype == PAGEDKV_DTYPE_F16)
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  else
    asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

template <typename T>
__device__ __forceinline__ uint4 rope8(const uint4 &x, const uint4 &xp, const uint4 &c, const uint4 &s, bool lo) {
  const uint32_t neg = lo ? 0x80008000u : 0u;  // sign bits of both halves
  uint4 r;
  r.x = add2_rn<T>(mul2_rn<T>(x.x, c.x), mul2_rn<T>(xp.x ^ neg, s.x));
  r.y = add2_rn<T>(mul2_rn<T>(x.y, c.y), mul2_rn<T>(xp.y ^ neg, s.y));
  r.z = add2_rn<T>(mul2_rn<T>(x.z, c.z), mul2_rn<T>(xp.z ^ neg, s.z));
  r.w = add2_rn<T>(mul2_rn<T>(x.w, c.w), mul2_rn<T>(xp.w ^ neg, s.w));
  return r;
}

// log2(e): scores are kept in the base-2 domain so exp() becomes one exp2f.
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kNegInf = -__builtin_huge_valf();

}  // namespace pagedkv
