// ztcp_kernels.cuh -- kernel parameter blocks shared by the kernels and the host launchers.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "ztcp_layout.h"

namespace ztcp {

// Per-page metadata of a batch.  Device pointers may be null: kv_block -> identity, sequence_nonce ->
// seq_base + page index (the reference's batch rule, csrc:1994), layer_id -> layer_uniform.  pool_pages > 0:
// blocks outside [0, pool_pages) are rejected on the device before any access.
struct PageMeta {
  const int32_t* kv_block;
  int64_t pool_pages;
  const uint64_t* token_hash;
  const uint64_t* sequence_nonce;
  const uint16_t* layer_id;
  uint64_t seq_base;
  uint32_t tenant;
  uint32_t model;
  uint16_t layer_uniform;
  uint16_t head_group;
};

constexpr int kTileThreads = 256;

// Keystream work of a full tile when every byte range it owns is whole 64-byte blocks (true for the
// standard geometries): range i covers the tile's blocks [first[i], first[i+1]), starting at keystream block
// kb0[i] + tile * (first[i+1] - first[i]), with its plaintext at staging offset stage[i].  Built on the host,
// so a CTA maps a block to its range by comparisons instead of a table that one thread builds while the
// others wait.  ok == 0: the kernels take the general path (ragged or unaligned ranges, padded tails).
struct TilePlan {
  int32_t ok = 0;
  int32_t n = 0;
  int32_t first[7] = {};
  int32_t kb0[6] = {};
  int32_t stage[6] = {};
};

struct EgressParams {
  const uint16_t* k;        // KV pool (fp16 or bf16 bits), page p at k + kv_block[p] * page_elems
  const uint16_t* v;        // null for a single-buffer MLA page
  int64_t page_elems;
  uint8_t* out;             // blobs, page p at out + p * blob_stride
  int64_t blob_stride;
  int64_t payload_len;
  int64_t vecs;
  int32_t head_dim;
  int32_t flags;            // header flags byte
  Layout L;
  PageMeta meta;
  uint32_t key[8];
  int32_t tile_vecs;
  int32_t n_tiles;
  int64_t n_pages;
  int32_t stage_q[3];       // shared-memory staging offsets (bytes) for a full tile
  int32_t stage_s[3];
  int32_t gshift[3];        // log2(groups per row) of each section, -1 when not a power of two
  int32_t stage_bytes;
  int32_t neon_arith;       // quantize with the reference's ARM NEON fp16 arithmetic
  PackMul mul;              // integer packing weights {16, 256, 65536}
  TilePlan plan;            // full tiles of L restricted to sections [sec_lo, sec_hi) (blobs 16-byte aligned)
  // What one launch produces: sections [sec_lo, sec_hi) of tiles [tile_lo, tile_lo + tiles) of every page
  // (grid = n_pages * tiles).  A whole-page launch is sections [0, L.n) of tiles [0, n_tiles) with the
  // header; a wire-order egress splits a batch into launches of one section and a tile range each and
  // leaves the header to its last tag segment.
  int32_t sec_lo, sec_hi;
  int32_t tile_lo, tiles;
  int32_t write_header;
};

struct MacParams {
  uint8_t* blobs;           // written (tag) in sign mode, read-only in verify mode
  int64_t blob_stride;
  int64_t payload_len;
  int64_t n_pages;
  uint64_t mk0, mk1;
  PageMeta meta;            // sign mode: block range only (an out-of-range page gets a zero tag)
  // segment mode (mac_segment_kernel): absorb blob bytes [seg_from, seg_to) into each page's chain; the
  // state between segments lives in the page's 32-byte header slot; the first segment starts the chain with
  // the header built from meta, the last one absorbs the length word, writes the tag and then the header
  int64_t seg_from, seg_to;
  int32_t seg_first, seg_last;
  int32_t flags;            // header flags byte (segment mode)
  // verify mode only
  int64_t vecs;
  int64_t head_dim;
  int64_t rope_dim;
  int32_t has_v;
  int32_t* status;          // [n_pages]
  int32_t* any_fail;        // [1], zeroed by the launcher
};

struct IngressParams {
  const uint8_t* blobs;
  int64_t blob_stride;
  int64_t payload_len;
  uint16_t* k_out;          // fp16 outputs, page p at k_out + kv_block[p] * page_elems
  uint16_t* v_out;
  int64_t page_elems;
  int64_t vecs;
  int32_t head_dim;
  int32_t rope_dim;
  int32_t has_v;
  PageMeta meta;
  uint32_t key[8];
  const int32_t* any_fail;
  const int32_t* status;     // per-page verify status (read when page_fallback)
  int32_t page_fallback;     // zero only failing pages instead of the whole batch
  int32_t tile_vecs;
  int32_t n_tiles;
  int64_t n_pages;
  int32_t stage_bytes;
  // layout and staging plan of every valid header flags byte, indexed by (preset - 1) * 3 + rope_mode
  // (every page reaching the decrypt pass has been verified, so its flags select a valid entry)
  Layout lay[9];
  int32_t lay_q[9][3];
  int32_t lay_s[9][3];
  TilePlan plan[9];         // full tiles of each layout (blobs 16-byte aligned)
};

void launch_egress(const EgressParams& P, bool bf16, cudaStream_t stream);
void launch_mac(const MacParams& P, bool verify, cudaStream_t stream);
void launch_mac_segment(const MacParams& P, cudaStream_t stream);
void launch_ingress(const IngressParams& P, cudaStream_t stream);
void launch_chacha20_xor(const uint8_t* src, uint8_t* dst, int64_t len, const uint32_t key[8], uint32_t counter0,
                         const uint32_t nonce[3], cudaStream_t stream);
void launch_siphash(const uint8_t* src, int64_t len, uint64_t k0, uint64_t k1, uint8_t* out16, cudaStream_t stream);

// Sets the calling thread's ztcp_last_error message and returns `code` (ztcp_capi.cu).
int32_t set_last_error(int32_t code, const std::string& msg);
// Records the phase event armed by ztcp_mark_phase on `stream`, if any, and disarms it (ztcp_measure.cu).
void take_phase_mark(cudaStream_t stream);

// Staging layout of one tile: 16-byte aligned q and scale areas per section.
ZTCP_HD int32_t plan_stage(const Layout& L, int32_t tile_vecs, int32_t stage_q[3], int32_t stage_s[3]) {
  int64_t off = 0;
  for (int i = 0; i < 3; ++i) {
    stage_q[i] = stage_s[i] = 0;
    if (i >= L.n) continue;
    stage_q[i] = (int32_t)off;
    off += ((int64_t)tile_vecs * L.sec[i].q_bpv + 15) / 16 * 16;
    stage_s[i] = (int32_t)off;
    off += ((int64_t)tile_vecs * L.sec[i].s_bpv + 15) / 16 * 16;
  }
  return (int32_t)off;
}

// Tile plan of a layout for full tiles of tile_vecs vecs and sections [sec_lo, sec_hi) (see TilePlan); ok stays 0
// when a range is not whole 64-byte blocks, block indices would not fit 32 bits, or aligned is false (blobs not
// 16-byte aligned).
ZTCP_HD void build_tile_plan(const Layout& L, int32_t tile_vecs, const int32_t stage_q[3], const int32_t stage_s[3],
                             bool aligned, TilePlan* T, int sec_lo = 0, int sec_hi = 3) {
  T->ok = 0;
  T->n = 0;
  int64_t acc = 0;
  bool good = aligned;
  for (int i = sec_lo; i < L.n && i < sec_hi; ++i) {
    const Section& S = L.sec[i];
    for (int part = 0; part < 2; ++part) {
      if (part == 1 && S.kind == kRaw) break;
      const int64_t a0 = part == 0 ? S.q_off : S.s_off;
      const int64_t bytes = (int64_t)tile_vecs * (part == 0 ? S.q_bpv : S.s_bpv);
      if (a0 % 64 != 0 || bytes % 64 != 0 || bytes == 0 || a0 / 64 > 0x3FFFFFFF) good = false;
      T->first[T->n] = (int32_t)acc;
      T->kb0[T->n] = (int32_t)(a0 / 64);
      T->stage[T->n] = part == 0 ? stage_q[i] : stage_s[i];
      acc += bytes / 64;
      ++T->n;
    }
  }
  T->first[T->n] = (int32_t)acc;
  if (L.data_end / 64 > 0x3FFFFFFF) good = false;
  T->ok = good && T->n > 0 ? 1 : 0;
}

// Vecs per CTA tile: 64 rows (a whole page when it is smaller), fewer when the staging would exceed
// 96 KB of shared memory.
ZTCP_HD int32_t pick_tile_vecs(int64_t vecs, int64_t stage_per_vec) {
  int64_t tv = vecs < 64 ? vecs : 64;
  while (tv > 1 && tv * stage_per_vec > 96 * 1024) tv = (tv + 1) / 2;
  return (int32_t)tv;
}

ZTCP_HD int32_t log2_or_minus1(int64_t x) {
  if (x <= 0 || (x & (x - 1)) != 0) return -1;
  int32_t k = 0;
  while (((int64_t)1 << k) < x) ++k;
  return k;
}

// ------------------------------------------------------------------------------------------------
// Page geometries compiled into their own tile kernels
// ------------------------------------------------------------------------------------------------
// The tile kernels read the wire layout, tiling and staging plan of a launch from their parameters, which costs
// address and index arithmetic on every group and keystream block.  For the benchmark configurations' page
// geometries and formats the same values are also compile-time constants: a second instantiation of each tile
// kernel reads them from a table the compiler folds, and the launchers pick it when a launch's parameters equal a
// table entry (the generic kernel otherwise).  The values are computed by the same functions the host uses.
struct StaticGeometry {
  int32_t num_tokens = 0, num_heads = 0, head_dim = 0, rope_dim = 0;
  bool has_v = false;
};
constexpr StaticGeometry kGqa64x8x128{64, 8, 128, 64, true};    // benchmark configurations 0, 1, 2, 4
constexpr StaticGeometry kMla64x1x576{64, 1, 576, 64, false};   // benchmark configuration 3

// Egress: a whole-batch launch (every section and tile, with the header) of one format and geometry.
struct StaticEgress {
  Layout L{};
  TilePlan plan{};
  int32_t stage_q[3] = {}, stage_s[3] = {}, gshift[3] = {};
  int32_t tile_vecs = 0, n_tiles = 0, head_dim = 0, flags = 0, stage_bytes = 0;
  int64_t vecs = 0, page_elems = 0;
  // Staged rows: a full tile's K and V rows (tile_vecs x head_dim each, contiguous in the pool) are copied to
  // shared memory after the staging area by two bulk copies while every thread computes its keystream block
  // (one block per thread: the plan's blocks fit the CTA).  rows_smem = the launch's dynamic shared memory.
  int32_t rows_ok = 0, rows_bytes = 0, rows_smem = 0;
};

ZTCP_HD StaticEgress make_static_egress(int preset, int rope_mode, StaticGeometry g) {
  StaticEgress e{};
  e.vecs = (int64_t)g.num_tokens * g.num_heads;
  e.head_dim = g.head_dim;
  e.page_elems = e.vecs * g.head_dim;
  e.flags = (preset & 0x0F) | ((rope_mode & 0x0F) << 4);
  build_layout(preset, rope_mode, e.vecs, g.head_dim, g.rope_dim, g.has_v, &e.L);
  e.tile_vecs = pick_tile_vecs(e.vecs, stage_bytes_per_vec(e.L));
  e.n_tiles = (int32_t)((e.vecs + e.tile_vecs - 1) / e.tile_vecs);
  e.stage_bytes = plan_stage(e.L, e.tile_vecs, e.stage_q, e.stage_s);
  build_tile_plan(e.L, e.tile_vecs, e.stage_q, e.stage_s, true, &e.plan);
  for (int i = 0; i < 3; ++i) e.gshift[i] = i < e.L.n ? log2_or_minus1(e.L.sec[i].dim / kGroup) : -1;
  e.rows_bytes = e.tile_vecs * g.head_dim * 2;
  e.rows_ok = e.plan.ok && e.plan.first[e.plan.n] <= kTileThreads && e.stage_bytes % 16 == 0 && e.rows_bytes % 16 == 0 &&
              e.stage_bytes + (g.has_v ? 2 : 1) * e.rows_bytes <= 48 * 1024;
  e.rows_smem = e.rows_ok ? e.stage_bytes + (g.has_v ? 2 : 1) * e.rows_bytes : e.stage_bytes;
  return e;
}


// (preset, rope_mode) and geometry of each compiled egress: INT4_SYM and K8V4_ASYM with PRESERVE_FP8 on GQA
// pages, INT4_SYM with PRESERVE_FP8 on MLA pages.
constexpr int kStaticEgressCount = 3;
constexpr int kStaticEgressKeys[kStaticEgressCount][2] = {{1, 1}, {2, 1}, {1, 1}};
constexpr StaticGeometry kStaticEgressGeometry[kStaticEgressCount] = {kGqa64x8x128, kGqa64x8x128, kMla64x1x576};

// Resident CTAs per SM the compiled egress kernel is built for: 5 with staged rows (45-47 KB of shared memory
// and up to 48 registers per thread), 7 otherwise.
ZTCP_HD int egress_min_blocks(int cfg) {
  return cfg > 0 && make_static_egress(kStaticEgressKeys[cfg - 1][0], kStaticEgressKeys[cfg - 1][1],
                                       kStaticEgressGeometry[cfg - 1]).rows_ok
             ? 5
             : 7;
}

// Ingress: a geometry with the layouts of every flags byte a header may carry, two of them (the benchmark
// formats) compiled into their own copies of the tile code.
struct StaticIngress {
  Layout lay[9] = {};
  int32_t lay_q[9][3] = {}, lay_s[9][3] = {};
  TilePlan plan[9] = {};
  int32_t tile_vecs = 0, n_tiles = 0, head_dim = 0, has_v = 0, stage_bytes = 0;
  int64_t vecs = 0, page_elems = 0;
};

ZTCP_HD StaticIngress make_static_ingress(StaticGeometry g) {
  StaticIngress s{};
  s.vecs = (int64_t)g.num_tokens * g.num_heads;
  s.head_dim = g.head_dim;
  s.page_elems = s.vecs * g.head_dim;
  s.has_v = g.has_v ? 1 : 0;
  const int64_t worst = worst_stage_bytes_per_vec(g.head_dim, g.rope_dim, g.has_v);
  s.tile_vecs = pick_tile_vecs(s.vecs, worst);
  s.n_tiles = (int32_t)((s.vecs + s.tile_vecs - 1) / s.tile_vecs);
  s.stage_bytes = (int32_t)(s.tile_vecs * worst + 6 * 16);
  for (int p = 1; p <= 3; ++p)
    for (int r = 0; r <= 2; ++r) {
      const int i = (p - 1) * 3 + r;
      build_layout(p, r, s.vecs, g.head_dim, g.rope_dim, g.has_v, &s.lay[i]);
      plan_stage(s.lay[i], s.tile_vecs, s.lay_q[i], s.lay_s[i]);
      build_tile_plan(s.lay[i], s.tile_vecs, s.lay_q[i], s.lay_s[i], true, &s.plan[i]);
    }
  return s;
}

constexpr int kStaticIngressCount = 2;
constexpr StaticGeometry kStaticIngressGeometry[kStaticIngressCount] = {kGqa64x8x128, kMla64x1x576};
// layout indices ((preset - 1) * 3 + rope_mode) with their own copy of the ingress tile code:
// INT4_SYM + PRESERVE_FP8 and K8V4_ASYM + PRESERVE_FP8
constexpr int kStaticIngressFast0 = 1, kStaticIngressFast1 = 4;

// Index + 1 of the compiled egress / ingress whose values a launch's parameters equal, or 0.
int static_egress_index(const EgressParams& P);
int static_ingress_index(const IngressParams& P);

}  // namespace ztcp
