// ztcp_device.cuh -- device primitives of the ZTCP codec for sm_100a.
//
//  * ChaCha20 (RFC 8439 section 2.3) keystream blocks, one 64-byte block per thread, counter-indexed
//    so any block of a page's keystream is computed independently (reference: csrc:113-189).
//  * SipHash-2-4 with 128-bit output as a serial per-lane chain over 64-bit words (csrc:401-471),
//    written on 32-bit halves with explicit carry: each 64-bit add is one add.cc/addc pair, each
//    rotate two funnel shifts or byte permutes (rotate by 32 is a register swap).  The chain is bound
//    by the ALU pipe (~42 ALU instructions per word, 2 cycles each per warp on a sub-partition).
//  * Group-16 INT8 / INT4 quantizers and dequantizers bit-exact with the reference's scalar x86 path
//    (csrc:734-754, 771-777, 805-825, 845-854), including its handling of NaN products.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "ztcp_layout.h"

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
  // One SipRound.  The 64-bit rotate by 16 is two byte permutes; rotates by 13, 17 and 21 are funnel
  // shifts; rotate by 32 swaps halves.  `pre` is XORed into v3 by the last instruction that writes it
  // (a 3-input LOP3), which lets the next word's `v3 ^= m` ride along for free.
  __device__ __forceinline__ void round(W64 pre = W64{0u, 0u}) {
    v0 = add64(v0, v1); v1 = xor64(rotl64<13>(v1), v0); v0 = rotl64<32>(v0);
    v2 = add64(v2, v3);
    v3 = W64{__byte_perm(v3.hi, v3.lo, 0x5432) ^ v2.lo, __byte_perm(v3.lo, v3.hi, 0x5432) ^ v2.hi};
    v0 = add64(v0, v3);
    {
      const W64 r = rotl64<21>(v3);
      v3 = W64{r.lo ^ v0.lo ^ pre.lo, r.hi ^ v0.hi ^ pre.hi};
    }
    v2 = add64(v2, v1); v1 = xor64(rotl64<17>(v1), v2); v2 = rotl64<32>(v2);
  }
  __device__ __forceinline__ void absorb(W64 m) {
    v3 = xor64(v3, m);
    round();
    round();
    v0 = xor64(v0, m);
  }
  __device__ __forceinline__ void absorb(uint32_t lo, uint32_t hi) { absorb(W64{lo, hi}); }
  // Absorb m into a state whose v3 already carries m, and fold the following word into v3.
  __device__ __forceinline__ void absorb_pre(W64 m, W64 next) {
    round();
    round(next);
    v0 = xor64(v0, m);
  }
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

// ------------------------------------------------------------------------------------------------
// Group loads: 16 consecutive elements as eight fp16x2 words (bf16 input rounded to fp16 first)
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t w) {
  const float2 f = make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
  const __half2 h = __float22half2_rn(f);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// src must be 16-byte aligned.
template <bool BF16>
__device__ __forceinline__ void load_group16(const uint16_t* src, uint32_t w[8]) {
  const uint4 a = __ldg(reinterpret_cast<const uint4*>(src));
  const uint4 b = __ldg(reinterpret_cast<const uint4*>(src) + 1);
  w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
  w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
  if (BF16) {
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = bf16x2_to_f16x2(w[i]);
  }
}

__device__ __forceinline__ uint16_t lo16(uint32_t w) { return (uint16_t)(w & 0xFFFFu); }
__device__ __forceinline__ uint16_t hi16(uint32_t w) { return (uint16_t)(w >> 16); }

// Largest |x| bit pattern of the group's 16 fp16 (BF16W = false) or bf16 (BF16W = true) elements, as a
// tree of packed half-precision NaN-propagating maxima of |x| (half the instructions of an integer max of
// masked bit patterns, and off the integer ALU pipe that ChaCha20 saturates).  For non-negative IEEE halves
// the bit patterns order like the values, +inf above every finite value and NaN above +inf, so for fp16 a
// result >= 0x7C00 flags a non-finite element (a NaN anywhere gives a NaN); likewise 0x7F80 for bf16.
template <bool BF16W>
__device__ __forceinline__ uint32_t group_amax_bits(const uint32_t w[8]) {
  if (BF16W) {
    __nv_bfloat162 v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __habs2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
    const __nv_bfloat162 a = __hmax2_nan(__hmax2_nan(v[0], v[1]), __hmax2_nan(v[2], v[3]));
    const __nv_bfloat162 b = __hmax2_nan(__hmax2_nan(v[4], v[5]), __hmax2_nan(v[6], v[7]));
    const __nv_bfloat162 m = __hmax2_nan(a, b);
    return (uint32_t)__bfloat16_as_ushort(__hmax_nan(__low2bfloat16(m), __high2bfloat16(m)));
  } else {
    __half2 v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __habs2(*reinterpret_cast<const __half2*>(&w[i]));
    const __half2 a = __hmax2_nan(__hmax2_nan(v[0], v[1]), __hmax2_nan(v[2], v[3]));
    const __half2 b = __hmax2_nan(__hmax2_nan(v[4], v[5]), __hmax2_nan(v[6], v[7]));
    const __half2 m = __hmax2_nan(a, b);
    return (uint32_t)__half_as_ushort(__hmax_nan(__low2half(m), __high2half(m)));
  }
}

// ------------------------------------------------------------------------------------------------
// Exact scalar quantizers (the reference's x86 semantics, including NaN products); used for groups
// whose scale is subnormal, zero or non-finite, or that hold a non-finite element.
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ float f16_at(const uint32_t* w, int i) {
  return f16_bits_to_f32((i & 1) ? hi16(w[i >> 1]) : lo16(w[i >> 1]));
}

// amax of NW fp16x2 words with a 1e-6 floor; NaN elements never compare greater (csrc:737-744 /
// 808-815)
template <int NW>
__device__ __forceinline__ float amax_exact(const uint32_t* w) {
  float amax = 1e-6f;
#pragma unroll
  for (int i = 0; i < 2 * NW; ++i) {
    const float av = fabsf(f16_at(w, i));
    amax = av > amax ? av : amax;
  }
  return amax;
}

// INT8: q = clamp(rint(x * inv), -127, 127); a NaN product quantizes to +127.  NQ output words.
template <int NQ>
__device__ __forceinline__ void quant_int8_exact(const uint32_t* w, float inv, uint32_t* q) {
#pragma unroll
  for (int k = 0; k < NQ; ++k) {
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float qf = rintf(__fmul_rn(f16_at(w, 4 * k + j), inv));
      if (qf != qf) qf = 127.0f;
      qf = fminf(fmaxf(qf, -127.0f), 127.0f);
      word |= ((uint32_t)(__float2int_rz(qf)) & 0xFFu) << (8 * j);
    }
    q[k] = word;
  }
}

// INT4: u = clamp(int(rint(x * inv) + 8), 0, 15) with x86 float->int conversion (NaN -> 0).  NQ output
// words.
template <int NQ>
__device__ __forceinline__ void quant_int4_exact(const uint32_t* w, float inv, uint32_t* q) {
#pragma unroll
  for (int k = 0; k < NQ; ++k) {
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float qf = __fadd_rn(rintf(__fmul_rn(f16_at(w, 8 * k + j), inv)), 8.0f);
      word |= (uint32_t)min(max(x86_cvtt(qf), 0), 15) << (4 * j);
    }
    q[k] = word;
  }
}

// ------------------------------------------------------------------------------------------------
// Group-16 quantizers.  scale = fp16(amax / qmax) and inv = 1 / float(scale) (IEEE reciprocal).
// Fast path: every element finite and scale a normal fp16.  Then the scale is within 2^-11 of
// amax / qmax, so |x * inv| <= qmax * (1 + 2^-11) + tiny < qmax + 0.5 and no clamp can fire.  fp16(amax /
// qmax) equals fp16(amax * (1 / qmax)) for every fp16 amax and the 1e-6 floor (checked exhaustively by the
// CPU tests), so the scale is one multiply.
//
// Rounding and packing.  p = x * inv rounded to fp32, then p + M with M = 2^23 + c rounded again: the sum
// lies in [2^23, 2^24), where the fp32 spacing is 1, so the FADD rounds p to the nearest integer with ties
// to even (M is even) and the sum's bit pattern is 0x4B000000 + (M - 2^23) + rint(p).  With c = qmax + 1
// (8 for INT4, 128 for INT8) the low bits hold u = rint(p) + c, in [1, 15] or [1, 255].  The stored word is
// then the sum of the element patterns weighted 16^i (INT4 nibble i) or 256^i (INT8 byte i), mod 2^32:
// the u terms land in their own nibbles or bytes without carries, and the constant parts cancel because
// one element's magic carries an extra offset (0x500000 at nibble 1, 0xB500 at byte 2) chosen so that
// the sum of all constant terms is 2^32.  So each element costs one multiply, one add and one integer
// multiply-add.  INT4 stores u itself (the format's q + 8); INT8 stores q = u - 128 as a two's-complement
// byte, which is u with its top bit flipped (one XOR per word).  The multiply and the add are the scalar
// _rn intrinsics, never contracted into a fused multiply-add: a fused x * inv + M would break rounding
// ties with the unrounded product.  (Packed f32x2 multiply and add were observed to be fused on sm_100a
// even with explicit .rn, so they are not used.)  The integer weights come from the kernel parameters
// (PackMul) rather than literals: with a literal power of two the compiler turns each multiply-add into a
// shift-and-add on the integer ALU pipe, which ChaCha20 already saturates; as IMADs they run on the FMA pipe.
// ------------------------------------------------------------------------------------------------
constexpr float kPackM4 = 8388616.0f;             // 2^23 + 8
constexpr float kPackM4n1 = 8388616.0f + 5242880.0f;  // 2^23 + 8 + 0x500000 (nibble 1)
constexpr float kPackM8 = 8388736.0f;             // 2^23 + 128
constexpr float kPackM8b2 = 8388736.0f + 46336.0f;    // 2^23 + 128 + 0xB500 (byte 2)

__device__ __forceinline__ uint32_t pack_bits(float x, float inv, float m) {
  return __float_as_uint(__fadd_rn(__fmul_rn(x, inv), m));
}

// Element pairs (lo = element 2j, hi = element 2j + 1) of one output word: INT4 eight elements from four
// pairs, INT8 four elements from two pairs.
__device__ __forceinline__ uint32_t pack_int4_word(const float lo[4], const float hi[4], float inv, const PackMul& mu) {
  uint32_t acc = pack_bits(hi[3], inv, kPackM4);
  acc = acc * mu.m16 + pack_bits(lo[3], inv, kPackM4);
#pragma unroll
  for (int j = 2; j >= 0; --j) {
    acc = acc * mu.m16 + pack_bits(hi[j], inv, j == 0 ? kPackM4n1 : kPackM4);
    acc = acc * mu.m16 + pack_bits(lo[j], inv, kPackM4);
  }
  return acc;
}

__device__ __forceinline__ uint32_t pack_int8_word(float e0, float e1, float e2, float e3, float inv,
                                                   const PackMul& mu) {
  uint32_t acc = pack_bits(e3, inv, kPackM8);
  acc = acc * mu.m256 + pack_bits(e2, inv, kPackM8b2);
  acc = acc * mu.m256 + pack_bits(e1, inv, kPackM8);
  acc = acc * mu.m256 + pack_bits(e0, inv, kPackM8);
  return acc ^ 0x80808080u;
}

__device__ __forceinline__ bool group_scale(const uint32_t w[8], float rq, __half* sh, float* inv) {
  const uint32_t amax_bits = group_amax_bits<false>(w);
  if (amax_bits >= 0x7C00u) {  // inf or NaN element: exact path computes everything
    *sh = __float2half_rn(__fmul_rn(amax_exact<8>(w), rq));
    *inv = __frcp_rn(__half2float(*sh));
    return false;
  }
  const float amax = fmaxf(f16_bits_to_f32((uint16_t)amax_bits), 1e-6f);
  *sh = __float2half_rn(__fmul_rn(amax, rq));
  *inv = __frcp_rn(__half2float(*sh));
  return __half_as_ushort(*sh) >= 0x0400u;  // normal scale (finite: amax <= 65504)
}

__device__ __forceinline__ uint16_t quant_int8(const uint32_t w[8], uint32_t q[4], const PackMul& mu) {
  __half sh;
  float inv;
  if (!group_scale(w, 1.0f / 127.0f, &sh, &inv)) {
    quant_int8_exact<4>(w, inv, q);
    return __half_as_ushort(sh);
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&w[2 * k]));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&w[2 * k + 1]));
    q[k] = pack_int8_word(a.x, a.y, b.x, b.y, inv, mu);
  }
  return __half_as_ushort(sh);
}

__device__ __forceinline__ uint16_t quant_int4(const uint32_t w[8], uint32_t q[2], const PackMul& mu) {
  __half sh;
  float inv;
  if (!group_scale(w, 1.0f / 7.0f, &sh, &inv)) {
    quant_int4_exact<2>(w, inv, q);
    return __half_as_ushort(sh);
  }
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    float lo[4], hi[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&w[4 * k + j]));
      lo[j] = x.x;
      hi[j] = x.y;
    }
    q[k] = pack_int4_word(lo, hi, inv, mu);
  }
  return __half_as_ushort(sh);
}

// ------------------------------------------------------------------------------------------------
// bf16 input without the round trip through fp16.  A bf16 value in fp16's normal range converts to
// fp16 exactly, so only elements below 2^-14 (or above 65504) could change.  With the group amax in
// [2^-9, 65280] (INT4) or [2^-5, 65280] (INT8) -- at least 4 * qmax * 2^-14 -- every element below
// 2^-14 has |x * inv| < 0.26 and quantizes to 0 from either value, and the amax is itself an exact fp16
// value, so the scale and every q equal the fp16 path's.  Other groups convert and take that path.
// ------------------------------------------------------------------------------------------------
constexpr uint32_t kBf16MaxFp16 = 0x477Fu;  // largest bf16 <= 65504

__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// true when the direct path applied; w holds raw bf16 pairs
__device__ __forceinline__ bool quant_int4_bf16(const uint32_t w[8], uint32_t q[2], uint16_t* scale,
                                                const PackMul& mu) {
  const uint32_t ab = group_amax_bits<true>(w);
  if (ab < 0x3B00u || ab > kBf16MaxFp16) return false;
  const __half sh = __float2half_rn(__fmul_rn(__uint_as_float(ab << 16), 1.0f / 7.0f));
  const float inv = __frcp_rn(__half2float(sh));
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    float lo[4], hi[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      lo[j] = __uint_as_float(w[4 * k + j] * mu.m64k);  // the low bf16 moved up: an IMAD, not an ALU shift
      hi[j] = bf16_hi(w[4 * k + j]);
    }
    q[k] = pack_int4_word(lo, hi, inv, mu);
  }
  *scale = __half_as_ushort(sh);
  return true;
}

__device__ __forceinline__ bool quant_int8_bf16(const uint32_t w[8], uint32_t q[4], uint16_t* scale,
                                                const PackMul& mu) {
  const uint32_t ab = group_amax_bits<true>(w);
  if (ab < 0x3D00u || ab > kBf16MaxFp16) return false;
  const __half sh = __float2half_rn(__fmul_rn(__uint_as_float(ab << 16), 1.0f / 127.0f));
  const float inv = __frcp_rn(__half2float(sh));
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t a = w[2 * k], b = w[2 * k + 1];
    q[k] = pack_int8_word(__uint_as_float(a * mu.m64k), bf16_hi(a), __uint_as_float(b * mu.m64k), bf16_hi(b), inv, mu);
  }
  *scale = __half_as_ushort(sh);
  return true;
}

// ------------------------------------------------------------------------------------------------
// Group-16 quantizers with the reference's ARM NEON fp16 arithmetic (csrc:718-733 INT8, :786-803 INT4;
// the multi-group NEON paths :905-1039 take the same per-group steps): |x| max in fp16 with NaN
// propagating, the 1e-6 floor through std::max, scale = fp16(amax * (1/qmax)), inv = fp16(1/scale),
// each product x*inv rounded to fp16 (the product of two fp16 values is exact in fp32), then
// round-to-nearest-even to int16 (NaN -> 0, saturating) and the saturating narrowings of vqmovn /
// vqmovun.  Selected per call; dequantization is the same in both arithmetics.
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ float neon_amax(const uint32_t w[8]) {
  float m = fabsf(f16_at(w, 0));
#pragma unroll
  for (int i = 1; i < 16; ++i) {
    const float a = fabsf(f16_at(w, i));
    m = (m != m || a != a) ? __int_as_float(0x7FC00000) : (a > m ? a : m);
  }
  return m < 1e-6f ? 1e-6f : m;
}

__device__ __forceinline__ int32_t neon_cvtn_s16(float p) {
  if (p != p) return 0;
  return (int32_t)fminf(fmaxf(rintf(p), -32768.0f), 32767.0f);
}

// fp16(x * inv) for fp16 x and inv, as an fp32 value
__device__ __forceinline__ float neon_mul(float x, float inv) { return __half2float(__float2half_rn(__fmul_rn(x, inv))); }

__device__ __forceinline__ uint16_t quant_int8_neon(const uint32_t w[8], uint32_t q[4]) {
  const __half sh = __float2half_rn(__fmul_rn(neon_amax(w), 1.0f / 127.0f));
  const float inv = __half2float(__float2half_rn(__frcp_rn(__half2float(sh))));
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int32_t s = max(min(neon_cvtn_s16(neon_mul(f16_at(w, 4 * k + j), inv)), 127), -127);
      word |= ((uint32_t)s & 0xFFu) << (8 * j);
    }
    q[k] = word;
  }
  return __half_as_ushort(sh);
}

__device__ __forceinline__ uint16_t quant_int4_neon(const uint32_t w[8], uint32_t q[2]) {
  const __half sh = __float2half_rn(__fmul_rn(neon_amax(w), 1.0f / 7.0f));
  const float inv = __half2float(__float2half_rn(__frcp_rn(__half2float(sh))));
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int32_t s = (int16_t)(neon_cvtn_s16(neon_mul(f16_at(w, 8 * k + j), inv)) + 8);  // int16 add wraps
      word |= (uint32_t)min(max(s, 0), 15) << (4 * j);
    }
    q[k] = word;
  }
  return __half_as_ushort(sh);
}

// ------------------------------------------------------------------------------------------------
// Dequantizers: fp16(float(q) * float(scale)).  float(q) * float(scale) is exact in fp32 (<= 8 + 11
// significant bits), so one IEEE half multiply of half(q) by the scale rounds it identically; half(q)
// is built exactly as (1024 + u) - bias from the bit pattern 0x6400 | u.  A non-finite scale takes the
// exact path, which writes a NaN product as 0xFE00 -- the half the reference's x86 build produces from
// the default NaN.
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint16_t dequant_one(float q, float s) {
  const float p = __fmul_rn(q, s);
  if (p != p) return 0xFE00u;
  return __half_as_ushort(__float2half_rn(p));
}

// NOUT output words (2 * NOUT elements).
template <int NOUT>
__device__ __forceinline__ void dequant_exact(const uint32_t* q, int bits, uint16_t scale, uint32_t* out) {
  const float s = f16_bits_to_f32(scale);
#pragma unroll
  for (int i = 0; i < NOUT; ++i) {
    float a, b;
    if (bits == 8) {
      const uint32_t w = q[i / 2] >> (16 * (i & 1));
      a = (float)(int8_t)(w & 0xFFu);
      b = (float)(int8_t)((w >> 8) & 0xFFu);
    } else {
      const uint32_t byte = (q[i / 4] >> (8 * (i & 3))) & 0xFFu;
      a = (float)(int)(byte & 0xFu) - 8.0f;
      b = (float)(int)(byte >> 4) - 8.0f;
    }
    out[i] = (uint32_t)dequant_one(a, s) | ((uint32_t)dequant_one(b, s) << 16);
  }
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<const uint32_t*>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<const __half2*>(&u); }

// NQ q words (4 elements each) -> 2 * NQ output words.
template <int NQ>
__device__ __forceinline__ void dequant_int8(const uint32_t* q, uint16_t scale, uint32_t* out) {
  if ((scale & 0x7C00u) == 0x7C00u) {
    dequant_exact<2 * NQ>(q, 8, scale, out);
    return;
  }
  const __half2 s2 = __half2half2(__ushort_as_half(scale));
  const __half2 bias = __float2half2_rn(1152.0f);  // 0x6400 | (q ^ 0x80) = 1152 + q
#pragma unroll
  for (int k = 0; k < NQ; ++k) {
    const uint32_t u = q[k] ^ 0x80808080u;
    const uint32_t lo = __byte_perm(u, 0x64646464u, 0x5140), hi = __byte_perm(u, 0x64646464u, 0x7362);
    out[2 * k] = h2_bits(__hmul2_rn(__hsub2(bits_h2(lo), bias), s2));
    out[2 * k + 1] = h2_bits(__hmul2_rn(__hsub2(bits_h2(hi), bias), s2));
  }
}

// NQ q words (8 elements each) -> 4 * NQ output words.
template <int NQ>
__device__ __forceinline__ void dequant_int4(const uint32_t* q, uint16_t scale, uint32_t* out) {
  if ((scale & 0x7C00u) == 0x7C00u) {
    dequant_exact<4 * NQ>(q, 4, scale, out);
    return;
  }
  if ((scale & 0x7C00u) >= 0x1400u) {
    // scale / 16 is a normal fp16 (exponent field >= 5; subtracting 0x1000 lowers it by 4, exactly).  Output
    // pair j (elements 2j, 2j + 1) comes from byte j copied into every byte: the low half keeps its low
    // nibble (1024 + u), the high half its high nibble at bits 20-23 (1024 + 16u).  16 (u - 8) * (scale / 16)
    // is then the same exact product as (u - 8) * scale, rounded once (every nibble and every such scale
    // checked against the direct form on the CPU), with one permute and one mask per pair and no
    // reordering of the results.
    const __half2 s2 = bits_h2((uint32_t)scale | ((uint32_t)(scale - 0x1000u) << 16));
    const __half2 bias = bits_h2(0x64806408u);  // (1032, 1152)
#pragma unroll
    for (int k = 0; k < NQ; ++k) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t p = (__byte_perm(q[k], 0u, 0x1111u * j) & 0x00F0000Fu) | 0x64006400u;
        out[4 * k + j] = h2_bits(__hmul2_rn(__hsub2(bits_h2(p), bias), s2));
      }
    }
    return;
  }
  // scales below 2^-10: the pairs (e0, e4) .. (e3, e7) at unit weight, reordered after the multiply
  const __half2 s2 = __half2half2(__ushort_as_half(scale));
  const __half2 bias = __float2half2_rn(1032.0f);  // 0x6400 | u = 1024 + u, q = u - 8
#pragma unroll
  for (int k = 0; k < NQ; ++k) {
    const uint32_t w = q[k];  // nibbles e0..e7 of this word, element i at bits 4i
    // (e0,e4) (e1,e5) (e2,e6) (e3,e7) as fp16 pairs 1024 + u
    const uint32_t p0 = (w & 0x000F000Fu) | 0x64006400u;
    const uint32_t p1 = ((w >> 4) & 0x000F000Fu) | 0x64006400u;
    const uint32_t p2 = ((w >> 8) & 0x000F000Fu) | 0x64006400u;
    const uint32_t p3 = ((w >> 12) & 0x000F000Fu) | 0x64006400u;
    const __half2 v0 = __hmul2_rn(__hsub2(bits_h2(p0), bias), s2);
    const __half2 v1 = __hmul2_rn(__hsub2(bits_h2(p1), bias), s2);
    const __half2 v2 = __hmul2_rn(__hsub2(bits_h2(p2), bias), s2);
    const __half2 v3 = __hmul2_rn(__hsub2(bits_h2(p3), bias), s2);
    out[4 * k + 0] = __byte_perm(h2_bits(v0), h2_bits(v1), 0x5410);  // (e0, e1)
    out[4 * k + 1] = __byte_perm(h2_bits(v2), h2_bits(v3), 0x5410);  // (e2, e3)
    out[4 * k + 2] = __byte_perm(h2_bits(v0), h2_bits(v1), 0x7632);  // (e4, e5)
    out[4 * k + 3] = __byte_perm(h2_bits(v2), h2_bits(v3), 0x7632);  // (e6, e7)
  }
}

}  // namespace ztcp
