/*
 * ztcp_oracle.c -- CPU restatement of the ZTCP cold-page codec.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * codec: tests, __graft_entry__.smoke() and bench.py's cpu_baseline leg may
 * call it; the product path never does.
 *
 * It restates the reference's *scalar* (non-NEON) code path, which is the
 * path the reference compiles to on x86-64 and therefore the one whose wire
 * bytes are reproducible on this hardware.  Every function cites the
 * reference lines it follows (paths relative to the reference project root,
 * `research/baseline_codec/...`).  The code is written from the algorithm,
 * not translated: the encoder builds the whole plaintext payload first, then
 * encrypts it with one keystream pass, then MACs header||ciphertext -- the
 * reference interleaves these three per byte, which yields the same bytes.
 *
 * Pinned against: the reference codec compiled from its own source in this
 * container (oracle/_ref), and the golden vectors in tests/golden/.
 *
 * Build: gcc -O2 -std=c11 -fPIC -shared (no -ffast-math: every float op here
 * must be IEEE round-to-nearest-even, as in the reference's scalar path).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ZO_HEADER_BYTES 32
#define ZO_TAG_BYTES 16
#define ZO_MAGIC 0x5A54u
#define ZO_VERSION 1u
#define ZO_GROUP 16

/* ------------------------------------------------------------------ */
/* IEEE binary16 / bfloat16 conversions (round-to-nearest-even).       */
/* at::Half conversion semantics used by the reference (csrc:741,812). */
/* ------------------------------------------------------------------ */
static uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

float zo_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  if (exp == 0x1Fu) return bits_f32(sign | 0x7F800000u | (man << 13)); /* inf / nan */
  if (exp != 0) return bits_f32(sign | ((exp + 112u) << 23) | (man << 13));
  if (man == 0) return bits_f32(sign);
  /* subnormal: value = man * 2^-24, exact in binary32 */
  float v = (float)man * 5.9604644775390625e-08f;
  return (h & 0x8000u) ? -v : v;
}

uint16_t zo_f32_to_f16(float f) {
  uint32_t x = f32_bits(f);
  uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  uint32_t ax = x & 0x7FFFFFFFu;
  if (ax > 0x7F800000u) return (uint16_t)(sign | 0x7E00u | ((ax >> 13) & 0x3FFu)); /* nan, quiet */
  if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* rounds to >= 65520 -> inf */
  if (ax >= 0x38800000u) {
    /* normal half range: rebias exponent, round 13 dropped bits to nearest-even */
    uint32_t mant = ax & 0x7FFFFFu;
    uint32_t e = (ax >> 23) - 112u;
    uint32_t h = (e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u; /* carry may bump exponent: correct */
    return (uint16_t)(sign | h);
  }
  /* subnormal or zero half: value / 2^-24, rounded to nearest-even integer */
  {
    float a = bits_f32(ax);
    float scaled = a * 16777216.0f; /* exact: power-of-two scaling of a float >= 2^-149 */
    float r = nearbyintf(scaled);    /* default rounding mode is nearest-even */
    return (uint16_t)(sign | (uint16_t)r); /* r <= 1024 -> 1024 is the smallest normal, still correct */
  }
}

float zo_bf16_to_f32(uint16_t b) { return bits_f32((uint32_t)b << 16); }

uint16_t zo_bf16_to_f16(uint16_t b) { return zo_f32_to_f16(zo_bf16_to_f32(b)); }

/* ------------------------------------------------------------------ */
/* ChaCha20, RFC 8439 section 2.3.  Reference: csrc:113-189 (scalar    */
/* branch 157-188), key/nonce words csrc:85-110.                       */
/* ------------------------------------------------------------------ */
static uint32_t rotl32(uint32_t x, int b) { return (x << b) | (x >> (32 - b)); }

void zo_chacha20_block(const uint32_t key[8], uint32_t counter, const uint32_t nonce[3], uint8_t out[64]) {
  uint32_t s[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u,
                    key[0], key[1], key[2], key[3], key[4], key[5], key[6], key[7],
                    counter, nonce[0], nonce[1], nonce[2]};
  uint32_t x[16];
  memcpy(x, s, sizeof(s));
  static const int idx[8][4] = {{0, 4, 8, 12}, {1, 5, 9, 13}, {2, 6, 10, 14}, {3, 7, 11, 15},
                                {0, 5, 10, 15}, {1, 6, 11, 12}, {2, 7, 8, 13}, {3, 4, 9, 14}};
  for (int dr = 0; dr < 10; ++dr) {
    for (int q = 0; q < 8; ++q) {
      uint32_t *a = &x[idx[q][0]], *b = &x[idx[q][1]], *c = &x[idx[q][2]], *d = &x[idx[q][3]];
      *a += *b; *d = rotl32(*d ^ *a, 16);
      *c += *d; *b = rotl32(*b ^ *c, 12);
      *a += *b; *d = rotl32(*d ^ *a, 8);
      *c += *d; *b = rotl32(*b ^ *c, 7);
    }
  }
  for (int i = 0; i < 16; ++i) {
    uint32_t w = x[i] + s[i];
    out[4 * i + 0] = (uint8_t)w;
    out[4 * i + 1] = (uint8_t)(w >> 8);
    out[4 * i + 2] = (uint8_t)(w >> 16);
    out[4 * i + 3] = (uint8_t)(w >> 24);
  }
}

/* keystream XOR of an arbitrary-length buffer: csrc:356-398 */
void zo_chacha20_xor(const uint8_t* src, uint8_t* dst, size_t len, const uint32_t key[8],
                     uint32_t counter0, const uint32_t nonce[3]) {
  uint8_t ks[64];
  for (size_t off = 0; off < len; off += 64) {
    zo_chacha20_block(key, counter0 + (uint32_t)(off / 64), nonce, ks);
    size_t n = len - off < 64 ? len - off : 64;
    for (size_t j = 0; j < n; ++j) dst[off + j] = src[off + j] ^ ks[j];
  }
}

/* key words from the four u64 key limbs: csrc:85-99 */
static void key_words_from_u64(const uint64_t k[4], uint32_t kw[8]) {
  for (int i = 0; i < 4; ++i) {
    kw[2 * i] = (uint32_t)k[i];
    kw[2 * i + 1] = (uint32_t)(k[i] >> 32);
  }
}

/* nonce derivation from the header: csrc:101-110 */
static void nonce_words(uint64_t seq, uint16_t layer, uint16_t head_group, uint32_t nw[3]) {
  nw[0] = (uint32_t)seq;
  nw[1] = (uint32_t)(seq >> 32);
  nw[2] = ((uint32_t)layer << 16) | head_group;
}

/* ------------------------------------------------------------------ */
/* SipHash-2-4 with 128-bit output.  Reference: csrc:401-471.          */
/* ------------------------------------------------------------------ */
static uint64_t rotl64(uint64_t x, int b) { return (x << b) | (x >> (64 - b)); }

typedef struct { uint64_t v0, v1, v2, v3; } zo_sip;

static void sip_round(zo_sip* s) {
  s->v0 += s->v1; s->v1 = rotl64(s->v1, 13); s->v1 ^= s->v0; s->v0 = rotl64(s->v0, 32);
  s->v2 += s->v3; s->v3 = rotl64(s->v3, 16); s->v3 ^= s->v2;
  s->v0 += s->v3; s->v3 = rotl64(s->v3, 21); s->v3 ^= s->v0;
  s->v2 += s->v1; s->v1 = rotl64(s->v1, 17); s->v1 ^= s->v2; s->v2 = rotl64(s->v2, 32);
}

static void sip_absorb(zo_sip* s, uint64_t m) {
  s->v3 ^= m; sip_round(s); sip_round(s); s->v0 ^= m;
}

static uint64_t load_le64(const uint8_t* p) {
  uint64_t w = 0;
  for (int i = 7; i >= 0; --i) w = (w << 8) | p[i];
  return w;
}

void zo_siphash128(uint64_t k0, uint64_t k1, const uint8_t* data, size_t len, uint8_t out[16]) {
  zo_sip s = {0x736f6d6570736575ull ^ k0, 0x646f72616e646f6dull ^ k1 ^ 0xeeull,
              0x6c7967656e657261ull ^ k0, 0x7465646279746573ull ^ k1};
  size_t n_words = len / 8;
  for (size_t i = 0; i < n_words; ++i) sip_absorb(&s, load_le64(data + 8 * i));
  uint64_t last = (uint64_t)(len & 0xff) << 56;
  for (size_t b = 0; b < (len & 7); ++b) last |= (uint64_t)data[8 * n_words + b] << (8 * b);
  sip_absorb(&s, last);
  s.v2 ^= 0xee;
  for (int i = 0; i < 4; ++i) sip_round(&s);
  uint64_t lo = s.v0 ^ s.v1 ^ s.v2 ^ s.v3;
  s.v1 ^= 0xdd;
  for (int i = 0; i < 4; ++i) sip_round(&s);
  uint64_t hi = s.v0 ^ s.v1 ^ s.v2 ^ s.v3;
  for (int i = 0; i < 8; ++i) { out[i] = (uint8_t)(lo >> (8 * i)); out[8 + i] = (uint8_t)(hi >> (8 * i)); }
}

/* ------------------------------------------------------------------ */
/* Group-16 quantizers, scalar semantics.                              */
/* INT8: csrc:734-754 (dequant 771-777); INT4: csrc:805-825 (845-854). */
/* ------------------------------------------------------------------ */
static float group_amax(const uint16_t* src) {
  float amax = 1e-6f;
  for (int i = 0; i < ZO_GROUP; ++i) {
    float av = fabsf(zo_f16_to_f32(src[i]));
    if (av > amax) amax = av; /* NaN never compares greater: ignored, as in the reference */
  }
  return amax;
}

/* float -> integer conversion as x86-64 cvttss2si does it (the reference's
 * static_cast on its x86 build): NaN and out-of-range give INT32_MIN. */
static int32_t x86_cvtt(float f) {
  if (!(f >= -2147483648.0f && f < 2147483648.0f)) return INT32_MIN;
  return (int32_t)f;
}

/*
 * INT8.  A product x*inv that is NaN -- an all-zero or tiny group whose fp16
 * scale underflows to 0 (0 * inf), or an infinite element times the zero
 * inverse of an infinite scale -- quantizes to +127 in the reference as built
 * on x86-64 with its -ffast-math flags (probed against oracle/_ref).  NaN
 * *inputs* are outside the parity contract: the reference's vectorized amax
 * reduction gives compiler-dependent results for them.
 */
static void quant_group_int8(const uint16_t* src, uint8_t* q, uint16_t* scale) {
  float amax = group_amax(src);
  uint16_t sh = zo_f32_to_f16(amax / 127.0f);
  float inv = 1.0f / zo_f16_to_f32(sh);
  *scale = sh;
  for (int i = 0; i < ZO_GROUP; ++i) {
    float qf = nearbyintf(zo_f16_to_f32(src[i]) * inv);
    if (isnan(qf)) qf = 127.0f;
    if (qf < -127.0f) qf = -127.0f;
    if (qf > 127.0f) qf = 127.0f;
    q[i] = (uint8_t)(int8_t)x86_cvtt(qf);
  }
}

static int clamp_i(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

static void quant_group_int4(const uint16_t* src, uint8_t* q, uint16_t* scale) {
  float amax = group_amax(src);
  uint16_t sh = zo_f32_to_f16(amax / 7.0f);
  float inv = 1.0f / zo_f16_to_f32(sh);
  *scale = sh;
  for (int i = 0; i < ZO_GROUP / 2; ++i) {
    float q0 = nearbyintf(zo_f16_to_f32(src[2 * i]) * inv) + 8.0f;
    float q1 = nearbyintf(zo_f16_to_f32(src[2 * i + 1]) * inv) + 8.0f;
    int u0 = clamp_i(x86_cvtt(q0), 0, 15);
    int u1 = clamp_i(x86_cvtt(q1), 0, 15);
    q[i] = (uint8_t)((u0 & 0xF) | ((u1 & 0xF) << 4));
  }
}

/* ------------------------------------------------------------------ */
/* Group-16 quantizers, ARM NEON semantics (the reference built with     */
/* __ARM_FEATURE_FP16_VECTOR_ARITHMETIC: csrc:718-733 INT8, :786-803 INT4; */
/* its dual- and quad-group paths :905-1039 take the same per-group      */
/* steps).  |x| max in fp16 with NaN propagating (FMAX), the 1e-6 floor  */
/* through std::max, scale = fp16(amax * (1/qmax)), inv = fp16(1/scale) */
/* held in an fp16 register, the product x*inv rounded to fp16 (the     */
/* product of two fp16 values is exact in float), then vcvtn (nearest,  */
/* ties to even, NaN -> 0, saturating to int16) and vqmovn / vqmovun    */
/* narrowing.  Dequantization is the same as the scalar path's: the      */
/* fp16 product of q and the scale is rounded once either way.           */
/* Not checked against an ARM build (none runs here).                    */
/* ------------------------------------------------------------------ */
static float neon_amax(const uint16_t* src) {
  float m = fabsf(zo_f16_to_f32(src[0]));
  for (int i = 1; i < ZO_GROUP; ++i) {
    float a = fabsf(zo_f16_to_f32(src[i]));
    m = (isnan(m) || isnan(a)) ? NAN : (a > m ? a : m);
  }
  return m < 1e-6f ? 1e-6f : m; /* std::max(amax, 1e-6f) keeps a NaN */
}

static int32_t neon_cvtn_s16(uint16_t h) {
  float f = zo_f16_to_f32(h);
  if (isnan(f)) return 0;
  float r = nearbyintf(f);
  if (r > 32767.0f) return 32767;
  if (r < -32768.0f) return -32768;
  return (int32_t)r;
}

static uint16_t neon_inv(uint16_t sh) { return zo_f32_to_f16(1.0f / zo_f16_to_f32(sh)); }

static void quant_group_int8_neon(const uint16_t* src, uint8_t* q, uint16_t* scale) {
  uint16_t sh = zo_f32_to_f16(neon_amax(src) * (1.0f / 127.0f));
  float inv = zo_f16_to_f32(neon_inv(sh));
  *scale = sh;
  for (int i = 0; i < ZO_GROUP; ++i) {
    int32_t s = neon_cvtn_s16(zo_f32_to_f16(zo_f16_to_f32(src[i]) * inv));
    s = s > 127 ? 127 : (s < -128 ? -128 : s); /* vqmovn_s16 */
    if (s < -127) s = -127;                     /* vmaxq_s8(q, -127) */
    q[i] = (uint8_t)(int8_t)s;
  }
}

static void quant_group_int4_neon(const uint16_t* src, uint8_t* q, uint16_t* scale) {
  uint16_t sh = zo_f32_to_f16(neon_amax(src) * (1.0f / 7.0f));
  float inv = zo_f16_to_f32(neon_inv(sh));
  *scale = sh;
  int u[ZO_GROUP];
  for (int i = 0; i < ZO_GROUP; ++i) {
    int16_t s = (int16_t)(neon_cvtn_s16(zo_f32_to_f16(zo_f16_to_f32(src[i]) * inv)) + 8); /* vaddq_s16 wraps */
    int v = s < 0 ? 0 : (s > 255 ? 255 : s);                                                /* vqmovun_s16 */
    u[i] = v > 15 ? 15 : v;                                                                 /* vminq_u8 */
  }
  for (int i = 0; i < ZO_GROUP / 2; ++i) q[i] = (uint8_t)(u[2 * i] | (u[2 * i + 1] << 4));
}

static void dequant_group_int8(const uint8_t* q, uint16_t scale, uint16_t* dst) {
  float s = zo_f16_to_f32(scale);
  for (int i = 0; i < ZO_GROUP; ++i) dst[i] = zo_f32_to_f16((float)(int8_t)q[i] * s);
}

static void dequant_group_int4(const uint8_t* q, uint16_t scale, uint16_t* dst) {
  float s = zo_f16_to_f32(scale);
  for (int i = 0; i < ZO_GROUP / 2; ++i) {
    dst[2 * i] = zo_f32_to_f16(((float)(q[i] & 0xF) - 8.0f) * s);
    dst[2 * i + 1] = zo_f32_to_f16(((float)(q[i] >> 4) - 8.0f) * s);
  }
}

/* ------------------------------------------------------------------ */
/* Payload size contract.  csrc:1439-1474 (minimum, no padding) and    */
/* cold_page_spec.py:203-246 (same sum, padded to a 4-byte multiple).  */
/* Returns -1 for invalid preset / rope_mode.                          */
/* ------------------------------------------------------------------ */
int64_t zo_min_payload_bytes(int preset, int rope_mode, int64_t vecs, int64_t head_dim, int64_t rope_dim, int has_v) {
  if (preset < 1 || preset > 3 || rope_mode < 0 || rope_mode > 2) return -1;
  int64_t total = 0;
  int64_t nope = head_dim - rope_dim;
  if (rope_mode == 2 && rope_dim > 0) total += vecs * rope_dim * 2;
  else if (rope_mode == 1 && rope_dim > 0) total += vecs * rope_dim + vecs * (rope_dim / ZO_GROUP) * 2;
  int64_t kq = rope_mode == 0 ? head_dim : nope;
  if (kq > 0) total += (preset == 1 ? vecs * (kq / 2) : vecs * kq) + vecs * (kq / ZO_GROUP) * 2;
  if (has_v) total += (preset == 3 ? vecs * head_dim : vecs * (head_dim / 2)) + vecs * (head_dim / ZO_GROUP) * 2;
  return total;
}

int64_t zo_spec_payload_bytes(int preset, int rope_mode, int64_t vecs, int64_t head_dim, int64_t rope_dim, int has_v) {
  int64_t m = zo_min_payload_bytes(preset, rope_mode, vecs, head_dim, rope_dim, has_v);
  if (m < 0) return m;
  return (m + 3) / 4 * 4;
}

/* ------------------------------------------------------------------ */
/* Section walk shared by encode and decode: csrc:1376-1409 (encode),  */
/* csrc:2420-2461 (decode).  kind: 0 raw fp16, 1 int8, 2 int4.         */
/* ------------------------------------------------------------------ */
typedef struct { int buf; int kind; int64_t col; int64_t dim; } zo_section;

static int build_sections(int preset, int rope_mode, int64_t head_dim, int64_t rope_dim, int has_v, zo_section sec[3]) {
  int n = 0;
  if (rope_mode == 2 && rope_dim > 0) sec[n++] = (zo_section){0, 0, 0, rope_dim};
  else if (rope_mode == 1 && rope_dim > 0) sec[n++] = (zo_section){0, 1, 0, rope_dim};
  int64_t kq = rope_mode == 0 ? head_dim : head_dim - rope_dim;
  int64_t kc = rope_mode == 0 ? 0 : rope_dim;
  if (kq > 0) sec[n++] = (zo_section){0, preset == 1 ? 2 : 1, kc, kq};
  if (has_v) sec[n++] = (zo_section){1, preset == 3 ? 1 : 2, 0, head_dim};
  return n;
}

static void write_header(uint8_t* h, int preset, int rope_mode, uint32_t tenant, uint32_t model, uint16_t layer,
                         uint16_t head_group, uint64_t tok, uint64_t seq) {
  /* struct <HBBIIHHQQ, cold_page_spec.py:51 / csrc:61-75 */
  uint8_t flags = (uint8_t)((preset & 0x0F) | ((rope_mode & 0x0F) << 4));
  h[0] = (uint8_t)(ZO_MAGIC & 0xFF); h[1] = (uint8_t)(ZO_MAGIC >> 8);
  h[2] = (uint8_t)ZO_VERSION; h[3] = flags;
  for (int i = 0; i < 4; ++i) { h[4 + i] = (uint8_t)(tenant >> (8 * i)); h[8 + i] = (uint8_t)(model >> (8 * i)); }
  h[12] = (uint8_t)layer; h[13] = (uint8_t)(layer >> 8);
  h[14] = (uint8_t)head_group; h[15] = (uint8_t)(head_group >> 8);
  for (int i = 0; i < 8; ++i) { h[16 + i] = (uint8_t)(tok >> (8 * i)); h[24 + i] = (uint8_t)(seq >> (8 * i)); }
}

/*
 * Encode one page (csrc:1103-1426).  k, v: fp16 bit patterns [vecs, head_dim]
 * (v may be NULL for a single-buffer MLA page).  blob_out must hold
 * 32 + expected_payload + 16 bytes.  Returns 0, or -1 on invalid arguments.
 */
static int encode_page(const uint16_t* k, const uint16_t* v, int64_t vecs, int64_t head_dim, int64_t rope_dim,
                       int preset, int rope_mode, int64_t expected_payload, uint32_t tenant, uint32_t model,
                       uint16_t layer, uint16_t head_group, uint64_t tok, uint64_t seq, const uint64_t key[4],
                       uint64_t mk0, uint64_t mk1, uint8_t* blob_out, int neon) {
  int64_t min_p = zo_min_payload_bytes(preset, rope_mode, vecs, head_dim, rope_dim, v != NULL);
  if (min_p < 0 || expected_payload < min_p) return -1;
  uint8_t* hdr = blob_out;
  uint8_t* payload = blob_out + ZO_HEADER_BYTES;
  write_header(hdr, preset, rope_mode, tenant, model, layer, head_group, tok, seq);
  memset(payload, 0, (size_t)expected_payload); /* pad bytes are plaintext zeros (csrc:1411-1422) */

  zo_section sec[3];
  int ns = build_sections(preset, rope_mode, head_dim, rope_dim, v != NULL, sec);
  int64_t off = 0;
  for (int si = 0; si < ns; ++si) {
    const uint16_t* buf = sec[si].buf == 0 ? k : v;
    int64_t dim = sec[si].dim, groups = dim / ZO_GROUP;
    if (sec[si].kind == 0) {
      for (int64_t r = 0; r < vecs; ++r)
        for (int64_t c = 0; c < dim; ++c) {
          uint16_t h = buf[r * head_dim + sec[si].col + c];
          payload[off + 2 * (r * dim + c)] = (uint8_t)h;
          payload[off + 2 * (r * dim + c) + 1] = (uint8_t)(h >> 8);
        }
      off += vecs * dim * 2;
      continue;
    }
    int64_t qpg = sec[si].kind == 1 ? 16 : 8; /* q bytes per group */
    uint8_t* qbase = payload + off;
    uint8_t* sbase = qbase + vecs * groups * qpg;
    for (int64_t r = 0; r < vecs; ++r)
      for (int64_t g = 0; g < groups; ++g) {
        const uint16_t* src = buf + r * head_dim + sec[si].col + g * ZO_GROUP;
        uint16_t sc;
        uint8_t* qd = qbase + (r * groups + g) * qpg;
        if (sec[si].kind == 1) (neon ? quant_group_int8_neon : quant_group_int8)(src, qd, &sc);
        else (neon ? quant_group_int4_neon : quant_group_int4)(src, qd, &sc);
        sbase[2 * (r * groups + g)] = (uint8_t)sc;
        sbase[2 * (r * groups + g) + 1] = (uint8_t)(sc >> 8);
      }
    off += vecs * groups * (qpg + 2);
  }

  uint32_t kw[8], nw[3];
  key_words_from_u64(key, kw);
  nonce_words(seq, layer, head_group, nw);
  zo_chacha20_xor(payload, payload, (size_t)expected_payload, kw, 1u, nw); /* counter starts at 1 (csrc:497) */
  zo_siphash128(mk0, mk1, blob_out, (size_t)(ZO_HEADER_BYTES + expected_payload),
                blob_out + ZO_HEADER_BYTES + expected_payload);
  return 0;
}

int zo_encode_page(const uint16_t* k, const uint16_t* v, int64_t vecs, int64_t head_dim, int64_t rope_dim,
                   int preset, int rope_mode, int64_t expected_payload, uint32_t tenant, uint32_t model,
                   uint16_t layer, uint16_t head_group, uint64_t tok, uint64_t seq, const uint64_t key[4],
                   uint64_t mk0, uint64_t mk1, uint8_t* blob_out) {
  return encode_page(k, v, vecs, head_dim, rope_dim, preset, rope_mode, expected_payload, tenant, model, layer,
                     head_group, tok, seq, key, mk0, mk1, blob_out, 0);
}

/*
 * Decode one blob with the batch-decoder's check order (csrc:2309-2463):
 * magic/version -> 1, AAD mismatch -> 2, MAC -> 3, invalid flags -> 4,
 * payload shorter than the flags require -> 5 (the reference folds 4 and 5
 * into its status 1).  On status 0 writes k_out (and v_out when v_out is not
 * NULL, i.e. the page is not a single-buffer MLA page).  Outputs are not
 * touched on failure.
 */
int zo_decode_page(const uint8_t* blob, int64_t blob_len, int64_t vecs, int64_t head_dim, int64_t rope_dim,
                   int is_mla, uint32_t exp_tenant, uint32_t exp_model, uint16_t exp_layer, uint64_t exp_tok,
                   const uint64_t key[4], uint64_t mk0, uint64_t mk1, uint16_t* k_out, uint16_t* v_out) {
  if (blob_len <= ZO_HEADER_BYTES + ZO_TAG_BYTES) return 1;
  int64_t payload_len = blob_len - ZO_HEADER_BYTES - ZO_TAG_BYTES;
  uint16_t magic = (uint16_t)(blob[0] | (blob[1] << 8));
  if (magic != ZO_MAGIC || blob[2] != ZO_VERSION) return 1;
  uint32_t tenant = (uint32_t)load_le64(blob + 4) & 0xFFFFFFFFu;
  uint32_t model = (uint32_t)load_le64(blob + 8) & 0xFFFFFFFFu;
  uint16_t layer = (uint16_t)(blob[12] | (blob[13] << 8));
  uint16_t head_group = (uint16_t)(blob[14] | (blob[15] << 8));
  uint64_t tok = load_le64(blob + 16), seq = load_le64(blob + 24);
  if (tenant != exp_tenant || model != exp_model || layer != exp_layer || tok != exp_tok) return 2;

  uint8_t tag[16];
  zo_siphash128(mk0, mk1, blob, (size_t)(ZO_HEADER_BYTES + payload_len), tag);
  uint8_t diff = 0;
  for (int i = 0; i < 16; ++i) diff |= (uint8_t)(tag[i] ^ blob[ZO_HEADER_BYTES + payload_len + i]);
  if (diff) return 3;

  int preset = blob[3] & 0x0F, rope_mode = (blob[3] >> 4) & 0x0F;
  int64_t min_p = zo_min_payload_bytes(preset, rope_mode, vecs, head_dim, rope_dim, !is_mla);
  if (min_p < 0) return 4;
  if (payload_len < min_p) return 5;

  uint8_t* plain = (uint8_t*)malloc((size_t)payload_len);
  if (!plain) return -1;
  uint32_t kw[8], nw[3];
  key_words_from_u64(key, kw);
  nonce_words(seq, layer, head_group, nw);
  zo_chacha20_xor(blob + ZO_HEADER_BYTES, plain, (size_t)payload_len, kw, 1u, nw);

  zo_section sec[3];
  int ns = build_sections(preset, rope_mode, head_dim, rope_dim, !is_mla, sec);
  int64_t off = 0;
  for (int si = 0; si < ns; ++si) {
    uint16_t* dst = sec[si].buf == 0 ? k_out : v_out;
    int64_t dim = sec[si].dim, groups = dim / ZO_GROUP;
    if (sec[si].kind == 0) {
      for (int64_t r = 0; r < vecs; ++r)
        for (int64_t c = 0; c < dim; ++c)
          dst[r * head_dim + sec[si].col + c] =
              (uint16_t)(plain[off + 2 * (r * dim + c)] | (plain[off + 2 * (r * dim + c) + 1] << 8));
      off += vecs * dim * 2;
      continue;
    }
    int64_t qpg = sec[si].kind == 1 ? 16 : 8;
    const uint8_t* qbase = plain + off;
    const uint8_t* sbase = qbase + vecs * groups * qpg;
    for (int64_t r = 0; r < vecs; ++r)
      for (int64_t g = 0; g < groups; ++g) {
        uint16_t sc = (uint16_t)(sbase[2 * (r * groups + g)] | (sbase[2 * (r * groups + g) + 1] << 8));
        uint16_t* out = dst + r * head_dim + sec[si].col + g * ZO_GROUP;
        if (sec[si].kind == 1) dequant_group_int8(qbase + (r * groups + g) * qpg, sc, out);
        else dequant_group_int4(qbase + (r * groups + g) * qpg, sc, out);
      }
    off += vecs * groups * (qpg + 2);
  }
  memset(plain, 0, (size_t)payload_len);
  free(plain);
  return 0;
}

/*
 * Batch wrappers with the reference's batch semantics
 * (csrc:1904-2004 encode: page b gets seq = base + b;
 *  csrc:2250-2496 decode: any failing page zeroes every output).
 * Decode returns the index of the first failing page, or -1 when all pass;
 * per-page statuses go to status_out.
 */
/* arith: 0 = the reference's scalar (x86-64) quantizers, 1 = its ARM NEON fp16 quantizers */
int zo_encode_batch_arith(const uint16_t* k, const uint16_t* v, int64_t batch, int64_t vecs, int64_t head_dim,
                          int64_t rope_dim, int preset, int rope_mode, int64_t expected_payload, uint32_t tenant,
                          uint32_t model, uint16_t layer, uint16_t head_group, const uint64_t* tok,
                          uint64_t base_seq, const uint64_t key[4], uint64_t mk0, uint64_t mk1, uint8_t* blobs_out,
                          int arith) {
  int64_t page = vecs * head_dim, blob = ZO_HEADER_BYTES + expected_payload + ZO_TAG_BYTES;
  for (int64_t b = 0; b < batch; ++b) {
    int rc = encode_page(k + b * page, v ? v + b * page : NULL, vecs, head_dim, rope_dim, preset, rope_mode,
                         expected_payload, tenant, model, layer, head_group, tok[b], base_seq + (uint64_t)b, key,
                         mk0, mk1, blobs_out + b * blob, arith);
    if (rc) return rc;
  }
  return 0;
}

int zo_encode_batch(const uint16_t* k, const uint16_t* v, int64_t batch, int64_t vecs, int64_t head_dim,
                    int64_t rope_dim, int preset, int rope_mode, int64_t expected_payload, uint32_t tenant,
                    uint32_t model, uint16_t layer, uint16_t head_group, const uint64_t* tok, uint64_t base_seq,
                    const uint64_t key[4], uint64_t mk0, uint64_t mk1, uint8_t* blobs_out) {
  return zo_encode_batch_arith(k, v, batch, vecs, head_dim, rope_dim, preset, rope_mode, expected_payload, tenant,
                               model, layer, head_group, tok, base_seq, key, mk0, mk1, blobs_out, 0);
}

int64_t zo_decode_batch(const uint8_t* blobs, int64_t batch, int64_t blob_len, int64_t vecs, int64_t head_dim,
                        int64_t rope_dim, int is_mla, uint32_t exp_tenant, uint32_t exp_model, uint16_t exp_layer,
                        const uint64_t* exp_tok, const uint64_t key[4], uint64_t mk0, uint64_t mk1,
                        uint16_t* k_out, uint16_t* v_out, int32_t* status_out) {
  int64_t page = vecs * head_dim, first_bad = -1;
  for (int64_t b = 0; b < batch; ++b) {
    status_out[b] = zo_decode_page(blobs + b * blob_len, blob_len, vecs, head_dim, rope_dim, is_mla, exp_tenant,
                                   exp_model, exp_layer, exp_tok[b], key, mk0, mk1, k_out + b * page,
                                   is_mla ? NULL : v_out + b * page);
    if (status_out[b] != 0 && first_bad < 0) first_bad = b;
  }
  if (first_bad >= 0) {
    memset(k_out, 0, (size_t)(batch * page) * 2);
    if (!is_mla) memset(v_out, 0, (size_t)(batch * page) * 2);
  }
  return first_bad;
}
