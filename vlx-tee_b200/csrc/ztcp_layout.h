// ztcp_layout.h -- ZTCP cold-page wire layout, shared by host and device code.
//
// Wire format (research/baseline_codec/cold_page_spec.py:17-37, csrc:61-75):
//   [32-byte header][payload, `payload_len` bytes, ChaCha20-encrypted][16-byte SipHash-2-4-128 tag]
// Header: struct <HBBIIHHQQ: magic 0x5A54, version 1, flags (preset | rope_mode << 4),
//   tenant_id_hash u32, model_id_hash u32, layer_id u16, head_group_id u16,
//   page_token_hash u64, sequence_nonce u64.
// Payload: up to three sections in this order (csrc:1376-1409):
//   K RoPE columns [0, rope_dim)  -- raw fp16 (rope_mode 2) or INT8 (rope_mode 1)
//   K quantized columns           -- NoPE [rope_dim, head_dim) (or all of K when rope_mode 0);
//                                    INT4 for preset 1, INT8 for presets 2 and 3
//   V (absent for a single-buffer MLA page) -- INT4 for presets 1 and 2, INT8 for preset 3
// Each quantized section is [q bytes for every (vec, group)] followed by [fp16 scale per (vec, group)],
// vec-major then group-major; a raw section is the fp16 rows back to back.  Zero bytes pad the
// payload to `payload_len` (csrc:1411-1422).
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define ZTCP_HD constexpr __host__ __device__ __forceinline__
#else
#define ZTCP_HD constexpr inline
#endif

namespace ztcp {

constexpr uint16_t kMagic = 0x5A54;
constexpr uint8_t kVersion = 1;
constexpr int64_t kHeaderBytes = 32;
constexpr int64_t kTagBytes = 16;
constexpr int kGroup = 16;

enum SectionKind : int32_t { kRaw = 0, kInt8 = 1, kInt4 = 2 };

// Integer weights of the quantizers' multiply-add packing (16, 256 and 65536), handed to the kernels as
// parameters so that the compiler keeps each weighted sum as an integer multiply-add.
struct PackMul {
  uint32_t m16, m256, m64k;
};

struct Section {
  int32_t kind = 0;   // SectionKind
  int32_t buf = 0;    // 0 = K, 1 = V
  int32_t col = 0;    // first source column
  int32_t dim = 0;    // number of source columns (multiple of 16)
  int64_t q_off = 0;  // payload offset of the q (or raw) region
  int64_t s_off = 0;  // payload offset of the scale region (== end of the q region)
  int32_t q_bpv = 0;  // q bytes per vec (raw: dim*2, int8: dim, int4: dim/2)
  int32_t s_bpv = 0;  // scale bytes per vec (groups*2; 0 for raw)
};

struct Layout {
  int32_t n = 0;          // number of sections (0..3)
  Section sec[3] = {};
  int64_t data_end = 0;   // first payload byte after the last section (minimum payload)
};

// Section walk for (preset, rope_mode) -- csrc:1376-1409 and required_payload_bytes_for_flags
// (csrc:1439-1474).  Returns false for an invalid preset / rope_mode.
ZTCP_HD bool build_layout(int preset, int rope_mode, int64_t vecs, int64_t head_dim, int64_t rope_dim,
                          bool has_v, Layout* L) {
  L->n = 0;
  L->data_end = 0;
  if (preset < 1 || preset > 3 || rope_mode < 0 || rope_mode > 2) return false;
  int64_t off = 0;
  auto add = [&](int32_t kind, int32_t buf, int64_t col, int64_t dim) {
    Section& s = L->sec[L->n++];
    s.kind = kind;
    s.buf = buf;
    s.col = (int32_t)col;
    s.dim = (int32_t)dim;
    s.q_bpv = kind == kRaw ? (int32_t)(dim * 2) : (kind == kInt8 ? (int32_t)dim : (int32_t)(dim / 2));
    s.s_bpv = kind == kRaw ? 0 : (int32_t)(dim / kGroup * 2);
    s.q_off = off;
    s.s_off = off + vecs * s.q_bpv;
    off = s.s_off + vecs * s.s_bpv;
  };
  if (rope_mode == 2 && rope_dim > 0) add(kRaw, 0, 0, rope_dim);
  else if (rope_mode == 1 && rope_dim > 0) add(kInt8, 0, 0, rope_dim);
  const int64_t kq = rope_mode == 0 ? head_dim : head_dim - rope_dim;
  const int64_t kc = rope_mode == 0 ? 0 : rope_dim;
  if (kq > 0) add(preset == 1 ? kInt4 : kInt8, 0, kc, kq);
  if (has_v) add(preset == 3 ? kInt8 : kInt4, 1, 0, head_dim);
  L->data_end = off;
  return true;
}

// Payload size the reference's Python spec computes (cold_page_spec.py:203-246): the minimum
// rounded up to a 4-byte multiple.  Returns -1 for invalid flags.
ZTCP_HD int64_t spec_payload_bytes(int preset, int rope_mode, int64_t vecs, int64_t head_dim,
                                   int64_t rope_dim, bool has_v) {
  Layout L{};
  if (!build_layout(preset, rope_mode, vecs, head_dim, rope_dim, has_v, &L)) return -1;
  return (L.data_end + 3) / 4 * 4;
}

// Staging bytes one vec needs across all sections (q + scales).
ZTCP_HD int64_t stage_bytes_per_vec(const Layout& L) {
  int64_t b = 0;
  for (int i = 0; i < L.n; ++i) b += L.sec[i].q_bpv + L.sec[i].s_bpv;
  return b;
}

// Largest stage_bytes_per_vec over every valid (preset, rope_mode): ingress reads flags from each
// blob's header, so its tile staging is sized for the worst case.
ZTCP_HD int64_t worst_stage_bytes_per_vec(int64_t head_dim, int64_t rope_dim, bool has_v) {
  int64_t worst = 0;
  for (int p = 1; p <= 3; ++p)
    for (int r = 0; r <= 2; ++r) {
      Layout L{};
      build_layout(p, r, 1, head_dim, rope_dim, has_v, &L);
      int64_t b = stage_bytes_per_vec(L);
      if (b > worst) worst = b;
    }
  return worst;
}

}  // namespace ztcp
