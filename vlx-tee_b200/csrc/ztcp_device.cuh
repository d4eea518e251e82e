// ztcp_device.cuh -- device primitives of the ZTCP codec for sm_100a.
//
//  * ChaCha20 (RFC 8439 section 2.3) keystream blocks, one 64-byte block per thread, counter-indexed
//    so any block of a page's keystream is computed independently (reference: csrc:113-189).
//  * SipHash-2-4 with 128-bit output as a serial per-lane chain over 64-bit words (csrc:401-471),
//    written on 32-bit halves with explicit carry so each 64-bit add is one add.cc/addc pair and each
//    rotate two funnel shifts (rotate by 32 is a register swap).
//  * Group-16 INT8 / INT4 quantizers and dequantizers bit-exact with the reference's scalar x86 path
//    (csrc:734-754, 771-777, 805-825, 845-854), including its handling of NaN products.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace ztcp {

// ------------------------------------------------------------------------------------------------
// ChaCha20
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t rotl32(uint32_t x, int b) { return __funnelshift_l(x, x, b); }

#define ZTCP_QR(a, b, c, d)   \
  a += b; d = rotl32(d ^ a, 16); \
  c += d; b = rotl32(b ^ c, 12); \
  a += b; d = rotl32(d ^ a, 8);  \
  c += d; b = rotl32(b ^ c, 7);

// 64-byte keystream block as 16 little-endian words: key[8] from the 256-bit key, nonce words
// [seq lo, seq hi, layer << 16 | head_group] (csrc:101-110), counter = 1 + block index (csrc:497).
__device__ __forceinline__ void chacha20_block(const uint32_t key[8], uint32_t counter, uint32_t n0, uint32_t n1,
                                               uint32_t n2, uint32_t out[16]) {
  uint32_t x0 = 0x61707865u, x1 = 0x3320646eu, x2 = 0x79622d32u, x3 = 0x6b206574u;
  uint32_t x4 = key[0], x5 = key[1], x6 = key[2], x7 = key[3];
  uint32_t x8 = key[4], x9 = key[5], x10 = key[6], x11 = key[7];
  uint32_t x12 = counter, x13 = n0, x14 = n1, x15 = n2;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    ZTCP_QR(x0, x4, x8, x12);
    ZTCP_QR(x1, x5, x9, x13);
    ZTCP_QR(x2, x6, x10, x14);
    ZTCP_QR(x3, x7, x11, x15);
    ZTCP_QR(x0, x5, x10, x15);
    ZTCP_QR(x1, x6, x11, x12);
    ZTCP_QR(x2, x7, x8, x13);
    ZTCP_QR(x3, x4, x9, x14);
  }
  out[0] = x0 + 0x61707865u;  out[1] = x1 + 0x3320646eu;
  out[2] = x2 + 0x79622d32u;  out[3] = x3 + 0x6b206574u;
  out[4] = x4 + key[0];       out[5] = x5 + key[1];
  out[6] = x6 + key[2];       out[7] = x7 + key[3];
  out[8] = x8 + key[4];       out[9] = x9 + key[5];
  out[10] = x10 + key[6];     out[11] = x11 + key[7];
  out[12] = x12 + counter;    out[13] = x13 + n0;
  out[14] = x14 + n1;         out[15] = x15 + n2;
}
#undef ZTCP_QR

// ------------------------------------------------------------------------------------------------
// SipHash-2-4-128
// ------------------------------------------------------------------------------------------------
struct W64 {
  uint32_t lo, hi;
};

__device__ __forceinline__ W64 w64(uint64_t v) { return W64{(uint32_t)v, (uint32_t)(v >> 32)}; }
__device__ __forceinline__ uint64_t u64(W64 v) { return ((uint64_t)v.hi << 32) | v.lo; }

__device__ __forceinline__ W64 add64(W64 a, W64 b) {
  W64 r;
  asm("add.cc.u32 %0, %2, %4;\n\taddc.u32 %1, %3, %5;"
      : "=r"(r.lo), "=r"(r.hi)
      : "r"(a.lo), "r"(a.hi), "r"(b.lo), "r"(b.hi));
  return r;
}
template <int B>
__device__ __forceinline__ W64 rotl64(W64 x) {
  if (B == 32) return W64{x.hi, x.lo};
  return W64{__funnelshift_l(x.hi, x.lo, B), __funnelshift_l(x.lo, x.hi, B)};
}
__device__ __forceinline__ W64 xor64(W64 a, W64 b) { return W64{a.lo ^ b.lo, a.hi ^ b.hi}; }

struct SipState {
  W64 v0, v1, v2, v3;

  __device__ __forceinline__ void init(uint64_t k0, uint64_t k1) {
    v0 = w64(0x736f6d6570736575ull ^ k0);
    v1 = w64(0x646f72616e646f6dull ^ k1 ^ 0xeeull);
    v2 = w64(0x6c7967656e657261ull ^ k0);
    v3 = w64(0x7465646279746573ull ^ k1);
  }
  __device__ __forceinline__ void round() {
    v0 = add64(v0, v1); v1 = xor64(rotl64<13>(v1), v0); v0 = rotl64<32>(v0);
    v2 = add64(v2, v3); v3 = xor64(rotl64<16>(v3), v2);
    v0 = add64(v0, v3); v3 = xor64(rotl64<21>(v3), v0);
    v2 = add64(v2, v1); v1 = xor64(rotl64<17>(v1), v2); v2 = rotl64<32>(v2);
  }
  __device__ __forceinline__ void absorb(W64 m) {
    v3 = xor64(v3, m);
    round();
    round();
    v0 = xor64(v0, m);
  }
  __device__ __forceinline__ void absorb(uint32_t lo, uint32_t hi) { absorb(W64{lo, hi}); }
  // finalization: v2 ^= 0xee, 4 rounds -> low half; v1 ^= 0xdd, 4 rounds -> high half (csrc:458-470)
  __device__ __forceinline__ void finish(uint32_t tag[4]) {
    v2.lo ^= 0xeeu;
    round(); round(); round(); round();
    tag[0] = v0.lo ^ v1.lo ^ v2.lo ^ v3.lo;
    tag[1] = v0.hi ^ v1.hi ^ v2.hi ^ v3.hi;
    v1.lo ^= 0xddu;
    round(); round(); round(); round();
    tag[2] = v0.lo ^ v1.lo ^ v2.lo ^ v3.lo;
    tag[3] = v0.hi ^ v1.hi ^ v2.hi ^ v3.hi;
  }
};

// ------------------------------------------------------------------------------------------------
// fp16 helpers and group quantizers
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint16_t bf16_bits_to_f16_bits(uint16_t b) {
  return __half_as_ushort(__float2half_rn(__uint_as_float((uint32_t)b << 16)));
}
__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// float -> int32 as x86-64 cvttss2si converts it (the reference's static_cast on its x86 build):
// NaN and values outside [-2^31, 2^31) give INT32_MIN.
__device__ __forceinline__ int32_t x86_cvtt(float f) {
  if (!(f >= -2147483648.0f && f < 2147483648.0f)) return INT32_MIN;
  return __float2int_rz(f);
}

// Loads 16 consecutive elements (fp16 or bf16 bits) as fp16 bit patterns.  src must be 16-byte aligned.
template <bool BF16>
__device__ __forceinline__ void load_group16(const uint16_t* src, uint16_t h[16]) {
  const uint4 a = __ldg(reinterpret_cast<const uint4*>(src));
  const uint4 b = __ldg(reinterpret_cast<const uint4*>(src) + 1);
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    h[2 * i] = (uint16_t)(w[i] & 0xFFFFu);
    h[2 * i + 1] = (uint16_t)(w[i] >> 16);
    if (BF16) {
      h[2 * i] = bf16_bits_to_f16_bits(h[2 * i]);
      h[2 * i + 1] = bf16_bits_to_f16_bits(h[2 * i + 1]);
    }
  }
}

// amax with a 1e-6 floor; NaN elements never compare greater (csrc:737-744 / 808-815)
__device__ __forceinline__ float group_amax(const uint16_t h[16]) {
  float amax = 1e-6f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float av = fabsf(f16_bits_to_f32(h[i]));
    amax = av > amax ? av : amax;
  }
  return amax;
}

// INT8: scale = fp16(amax / 127), q = clamp(rint(x * (1 / scale)), -127, 127); a NaN product
// quantizes to +127 (reference x86 build, pinned by the oracle).
__device__ __forceinline__ uint16_t quant_int8(const uint16_t h[16], uint32_t q[4]) {
  const float amax = group_amax(h);
  const __half sh = __float2half_rn(__fdiv_rn(amax, 127.0f));
  const float inv = __frcp_rn(__half2float(sh));
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float qf = rintf(__fmul_rn(f16_bits_to_f32(h[4 * w + j]), inv));
      if (qf != qf) qf = 127.0f;
      qf = fminf(fmaxf(qf, -127.0f), 127.0f);
      word |= ((uint32_t)(__float2int_rz(qf)) & 0xFFu) << (8 * j);
    }
    q[w] = word;
  }
  return __half_as_ushort(sh);
}

// INT4: scale = fp16(amax / 7), u = clamp(int(rint(x * (1 / scale)) + 8), 0, 15) with x86 float->int
// conversion; byte i = u[2i] | u[2i+1] << 4.
__device__ __forceinline__ uint16_t quant_int4(const uint16_t h[16], uint32_t q[2]) {
  const float amax = group_amax(h);
  const __half sh = __float2half_rn(__fdiv_rn(amax, 7.0f));
  const float inv = __frcp_rn(__half2float(sh));
#pragma unroll
  for (int w = 0; w < 2; ++w) {
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float qf = __fadd_rn(rintf(__fmul_rn(f16_bits_to_f32(h[8 * w + j]), inv)), 8.0f);
      const int32_t u = min(max(x86_cvtt(qf), 0), 15);
      word |= (uint32_t)u << (4 * j);
    }
    q[w] = word;
  }
  return __half_as_ushort(sh);
}

// fp16(float(q) * float(scale)); a NaN product (zero times an infinite scale) is written as 0xFE00,
// the half the reference's x86 build produces from the default NaN.
__device__ __forceinline__ uint16_t dequant_one(float q, float s) {
  const float p = __fmul_rn(q, s);
  if (p != p) return 0xFE00u;
  return __half_as_ushort(__float2half_rn(p));
}

__device__ __forceinline__ void dequant_int8(const uint32_t q[4], uint16_t scale, uint32_t out[8]) {
  const float s = f16_bits_to_f32(scale);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t w = q[i / 2] >> (16 * (i & 1));
    const float a = (float)(int8_t)(w & 0xFFu), b = (float)(int8_t)((w >> 8) & 0xFFu);
    out[i] = (uint32_t)dequant_one(a, s) | ((uint32_t)dequant_one(b, s) << 16);
  }
}

__device__ __forceinline__ void dequant_int4(const uint32_t q[2], uint16_t scale, uint32_t out[8]) {
  const float s = f16_bits_to_f32(scale);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t byte = (q[i / 4] >> (8 * (i & 3))) & 0xFFu;
    const float a = (float)(int)(byte & 0xFu) - 8.0f, b = (float)(int)(byte >> 4) - 8.0f;
    out[i] = (uint32_t)dequant_one(a, s) | ((uint32_t)dequant_one(b, s) << 16);
  }
}

}  // namespace ztcp
