// ztcp_kernels.cu -- sm_100a kernels of the ZTCP cold-page codec.
//
// Egress  = egress_tile_kernel (quantize + pack + ChaCha20, per (page, vec-tile))
//         + mac_kernel<sign>    (one SipHash-2-4-128 chain per lane = per page, writes the tag)
// Ingress = mac_kernel<verify>  (header / AAD / tag / flags checks, per-page status, batch fail flag)
//         + ingress_tile_kernel (decrypt + dequantize per (page, vec-tile); zeroes every output when
//                                any page of the batch failed -- the reference's all-or-nothing rule,
//                                csrc:2481-2495 -- or, with the page-fallback option, only the failed pages)
//
// Tiling.  A CTA owns `tile_vecs` consecutive vecs (token x head rows) of one page.  Those rows map
// to one contiguous byte range per q region and per scale region of every section (the payload is
// vec-major within a region), so a CTA quantizes its rows into shared memory and then encrypts its
// own byte ranges.  ChaCha20 is counter-indexed (payload byte x uses block 1 + x / 64), so every
// 64-byte keystream block is computed by exactly the threads that need it; a block straddling two
// tiles is computed by both and each writes only its own bytes.
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

#include "ztcp_device.cuh"
#include "ztcp_kernels.cuh"

namespace ztcp {

namespace {

// Pool block of batch page `page`, or -1 when the block table points outside the pool (the page is then
// neither read nor written in the pool).
__device__ __forceinline__ int64_t page_block(const PageMeta& m, int64_t page) {
  const int64_t b = m.kv_block ? (int64_t)m.kv_block[page] : page;
  return (m.pool_pages > 0 && (b < 0 || b >= m.pool_pages)) ? -1 : b;
}
__device__ __forceinline__ uint64_t page_seq(const PageMeta& m, int64_t page) {
  return m.sequence_nonce ? m.sequence_nonce[page] : m.seq_base + (uint64_t)page;
}
__device__ __forceinline__ uint16_t page_layer(const PageMeta& m, int64_t page) {
  return m.layer_id ? m.layer_id[page] : m.layer_uniform;
}

__device__ __forceinline__ Section pick(const Layout& L, int s) {
  return s == 0 ? L.sec[0] : (s == 1 ? L.sec[1] : L.sec[2]);
}

// A payload byte range [a, b) owned by one tile, backed by shared-memory staging (or zeros).
struct Range {
  int64_t a, b;
  int32_t stage;
  int32_t zero;
};

__device__ __forceinline__ int tile_ranges(const Layout& L, int64_t v0, int tv, const int32_t sq[3],
                                           const int32_t ss[3], bool with_pad, int64_t payload_len, Range r[7],
                                           int sec_lo, int sec_hi) {
  int n = 0;
#pragma unroll
  for (int s = 0; s < 3; ++s) {
    if (s >= L.n || s >= sec_hi) break;
    if (s < sec_lo) continue;
    const Section S = pick(L, s);
    r[n++] = Range{S.q_off + v0 * S.q_bpv, S.q_off + (v0 + tv) * S.q_bpv, sq[s], 0};
    if (S.kind != kRaw) r[n++] = Range{S.s_off + v0 * S.s_bpv, S.s_off + (v0 + tv) * S.s_bpv, ss[s], 0};
  }
  if (with_pad && payload_len > L.data_end) r[n++] = Range{L.data_end, payload_len, 0, 1};
  return n;
}

__device__ __forceinline__ int64_t range_blocks(const Range& r) {
  return r.b > r.a ? ((r.b - 1) >> 6) - (r.a >> 6) + 1 : 0;
}

// A tile's byte ranges and the prefix sums of their 64-byte keystream blocks, built once per CTA in
// shared memory; threads then map a flat keystream-block index to (range, block) by a short scan.
struct RangeTable {
  Range r[7];
  int64_t first[8];  // first[i] = flat index of range i's first block; first[n] = total blocks
  int32_t n;
};

__device__ __forceinline__ void build_range_table(RangeTable& T, const Layout& L, int64_t v0, int tv,
                                                  const int32_t sq[3], const int32_t ss[3], bool with_pad,
                                                  int64_t payload_len, int sec_lo = 0, int sec_hi = 3) {
  T.n = tile_ranges(L, v0, tv, sq, ss, with_pad, payload_len, T.r, sec_lo, sec_hi);
  int64_t acc = 0;
  for (int i = 0; i < T.n; ++i) {
    T.first[i] = acc;
    acc += range_blocks(T.r[i]);
  }
  T.first[T.n] = acc;
}

__device__ __forceinline__ int find_range(const RangeTable& T, int64_t bi) {
  int i = 0;
  while (i + 1 < T.n && bi >= T.first[i + 1]) ++i;
  return i;
}

// XOR one keystream block into bytes [lo, hi) of dst, taking plaintext from src (nullptr = zeros).
// Both pointers address payload byte 64*kb (block start); bytes outside [lo, hi) are untouched.
__device__ __forceinline__ void xor_block_bytes(uint8_t* dst, const uint8_t* src, const uint32_t ks[16], int lo,
                                                int hi) {
#pragma unroll
  for (int w = 0; w < 16; ++w) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int x = 4 * w + j;
      if (x >= lo && x < hi) dst[x] = (uint8_t)((src ? src[x] : 0) ^ (uint8_t)(ks[w] >> (8 * j)));
    }
  }
}

// Range of flat block bi in a tile plan (ranges are few: compare against every boundary).
__device__ __forceinline__ int plan_range(const TilePlan& T, int bi) {
  int i = 0;
#pragma unroll
  for (int j = 1; j < 6; ++j) i += (j < T.n && bi >= T.first[j]) ? 1 : 0;
  return i;
}

// One section's slice of a tile: source rows, staging areas and the (vec, group) index split.
struct SectionTile {
  const uint16_t* src;  // first source element of the tile's first row in this section
  uint8_t* q;           // staging of the q (or raw) region for the tile
  uint8_t* sc;          // staging of the scale region for the tile
  int32_t row_stride;   // elements between rows (head_dim)
  int32_t q_bpv, s_bpv; // staging bytes per vec
  int32_t groups;       // 16-element groups per row in this section
  int32_t gshift;       // log2(groups), or -1 when groups is not a power of two
  int32_t tv;           // vecs in this tile
};

__device__ __forceinline__ void split_item(int it, const SectionTile& t, int& vec, int& g) {
  if (t.gshift >= 0) {
    vec = it >> t.gshift;
    g = it & (t.groups - 1);
  } else {
    vec = it / t.groups;
    g = it - vec * t.groups;
  }
}

// STAGED: the tile's rows are in shared memory (t.src points there); otherwise they are read from the KV
// pool through the read-only data path.
template <int KIND, bool BF16, bool NEON, bool STAGED = false>
__device__ __forceinline__ void quantize_section(const SectionTile& t, const PackMul& mu) {
  const int items = t.tv * t.groups;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    int vec, g;
    split_item(it, t, vec, g);
    uint32_t w[8];  // raw bits
    if (STAGED) {
      const uint4* p = reinterpret_cast<const uint4*>(t.src + vec * t.row_stride + g * 16);
      const uint4 a = p[0], b = p[1];
      w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
      w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
    } else {
      load_group16<false>(t.src + vec * t.row_stride + g * 16, w);
    }
    uint8_t* qd = t.q + vec * t.q_bpv;
    if (KIND == kRaw) {
      if (BF16) {
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = bf16x2_to_f16x2(w[i]);
      }
      uint4* d = reinterpret_cast<uint4*>(qd + g * 32);
      d[0] = make_uint4(w[0], w[1], w[2], w[3]);
      d[1] = make_uint4(w[4], w[5], w[6], w[7]);
    } else if (KIND == kInt8) {
      uint32_t q[4];
      uint16_t sc;
      if (NEON || !BF16 || !quant_int8_bf16(w, q, &sc, mu)) {
        if (BF16) {
#pragma unroll
          for (int i = 0; i < 8; ++i) w[i] = bf16x2_to_f16x2(w[i]);
        }
        sc = NEON ? quant_int8_neon(w, q) : quant_int8(w, q, mu);
      }
      *reinterpret_cast<uint4*>(qd + g * 16) = make_uint4(q[0], q[1], q[2], q[3]);
      *reinterpret_cast<uint16_t*>(t.sc + vec * t.s_bpv + g * 2) = sc;
    } else {
      uint32_t q[2];
      uint16_t sc;
      if (NEON || !BF16 || !quant_int4_bf16(w, q, &sc, mu)) {
        if (BF16) {
#pragma unroll
          for (int i = 0; i < 8; ++i) w[i] = bf16x2_to_f16x2(w[i]);
        }
        sc = NEON ? quant_int4_neon(w, q) : quant_int4(w, q, mu);
      }
      *reinterpret_cast<uint2*>(qd + g * 8) = make_uint2(q[0], q[1]);
      *reinterpret_cast<uint16_t*>(t.sc + vec * t.s_bpv + g * 2) = sc;
    }
  }
}

// Dequantize one section's slice of a tile from staging into the KV pool rows.
template <int KIND>
__device__ __forceinline__ void dequantize_section(const SectionTile& t, uint16_t* dst) {
  const int items = t.tv * t.groups;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    int vec, g;
    split_item(it, t, vec, g);
    uint4* d = reinterpret_cast<uint4*>(dst + vec * t.row_stride + g * 16);
    const uint8_t* qs = t.q + vec * t.q_bpv;
    if (KIND == kRaw) {
      const uint4* q = reinterpret_cast<const uint4*>(qs + g * 32);
      d[0] = q[0];
      d[1] = q[1];
      continue;
    }
    const uint16_t scale = *reinterpret_cast<const uint16_t*>(t.sc + vec * t.s_bpv + g * 2);
    uint32_t o[8];
    if (KIND == kInt8) {
      const uint4 q = *reinterpret_cast<const uint4*>(qs + g * 16);
      const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
      dequant_int8<4>(qw, scale, o);
    } else {
      const uint2 q = *reinterpret_cast<const uint2*>(qs + g * 8);
      const uint32_t qw[2] = {q.x, q.y};
      dequant_int4<2>(qw, scale, o);
    }
    d[0] = make_uint4(o[0], o[1], o[2], o[3]);
    d[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

__device__ __forceinline__ int32_t log2_if_pow2(int32_t x) {
  return (x > 0 && (x & (x - 1)) == 0) ? __ffs(x) - 1 : -1;
}

// The compiled geometries' tables (ztcp_kernels.cuh): constant memory the compiler reads at compile time
// wherever a kernel indexes them with constants.
__constant__ constexpr StaticEgress kStaticEgress[kStaticEgressCount] = {
    make_static_egress(kStaticEgressKeys[0][0], kStaticEgressKeys[0][1], kStaticEgressGeometry[0]),
    make_static_egress(kStaticEgressKeys[1][0], kStaticEgressKeys[1][1], kStaticEgressGeometry[1]),
    make_static_egress(kStaticEgressKeys[2][0], kStaticEgressKeys[2][1], kStaticEgressGeometry[2])};
__constant__ constexpr StaticIngress kStaticIngress[kStaticIngressCount] = {
    make_static_ingress(kStaticIngressGeometry[0]), make_static_ingress(kStaticIngressGeometry[1])};

// The 32-byte header of a page (csrc:61-75, :1129-1140).
__device__ __forceinline__ void write_header(uint8_t* blob, int32_t flags, const PageMeta& m, int64_t page, uint64_t seq,
                                             uint16_t layer) {
  const uint64_t tok = m.token_hash[page];
  const uint32_t hw[8] = {(uint32_t)kMagic | ((uint32_t)kVersion << 16) | ((uint32_t)flags << 24),
                          m.tenant,
                          m.model,
                          (uint32_t)layer | ((uint32_t)m.head_group << 16),
                          (uint32_t)tok,
                          (uint32_t)(tok >> 32),
                          (uint32_t)seq,
                          (uint32_t)(seq >> 32)};
  if ((reinterpret_cast<uintptr_t>(blob) & 3) == 0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) reinterpret_cast<uint32_t*>(blob)[i] = hw[i];
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) blob[i] = (uint8_t)(hw[i >> 2] >> (8 * (i & 3)));
  }
}

// Waits for phase 0 of a shared-memory mbarrier for at most 2^31 SM clock cycles (about a second at the
// B200's 1.97 GHz; each try_wait may suspend the thread for a while); true when the phase completed.
__device__ __forceinline__ bool mbar_wait_parity0(uint32_t bar) {
  const long long t0 = clock64();
  for (;;) {
    uint32_t done;
    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0; selp.u32 %0, 1, 0, p; }"
                 : "=r"(done)
                 : "r"(bar)
                 : "memory");
    if (done) return true;
    if (clock64() - t0 > (1ll << 31)) return false;
  }
}

// ------------------------------------------------------------------------------------------------
// Egress: quantize + pack + encrypt one (page, vec-tile)
// ------------------------------------------------------------------------------------------------
// 7 resident CTAs per SM (the register cap this implies was measured ~5 % faster than 6), 5 for the compiled
// geometries that stage their rows (egress_min_blocks).
// CFG = 0: layout, tiling and staging plan from the launch parameters; CFG = i > 0: those of kStaticEgress[i - 1]
// as compile-time constants (a whole-batch launch of that geometry and format), so their address and index
// arithmetic folds away.
template <bool BF16, bool NEON, int CFG>
__global__ void __launch_bounds__(kTileThreads, egress_min_blocks(CFG)) egress_tile_kernel(const __grid_constant__ EgressParams P) {
  extern __shared__ __align__(16) uint8_t stage[];
  __shared__ RangeTable T;
  const StaticEgress& G = kStaticEgress[CFG > 0 ? CFG - 1 : 0];
  const Layout& L = CFG ? G.L : P.L;
  const TilePlan& plan = CFG ? G.plan : P.plan;
  const int32_t(&stage_q)[3] = CFG ? G.stage_q : P.stage_q;
  const int32_t(&stage_s)[3] = CFG ? G.stage_s : P.stage_s;
  const int32_t(&gshift)[3] = CFG ? G.gshift : P.gshift;
  const int tile_vecs = CFG ? G.tile_vecs : P.tile_vecs;
  const int n_tiles = CFG ? G.n_tiles : P.n_tiles;
  const int64_t vecs = CFG ? G.vecs : P.vecs;
  const int head_dim = CFG ? G.head_dim : P.head_dim;
  const int64_t page_elems = CFG ? G.page_elems : P.page_elems;
  const int sec_lo = CFG ? 0 : P.sec_lo, sec_hi = CFG ? G.L.n : P.sec_hi;
  const int tile_lo = CFG ? 0 : P.tile_lo, tiles = CFG ? G.n_tiles : P.tiles;
  const int64_t page = blockIdx.x / tiles;
  const int tile = tile_lo + (int)(blockIdx.x - page * tiles);
  const int64_t v0 = (int64_t)tile * tile_vecs;
  const int tv = (int)min((int64_t)tile_vecs, vecs - v0);
  const bool with_pad = tile == n_tiles - 1 && sec_hi == L.n;  // the last tile of the last section pads
  const bool padded = with_pad && P.payload_len > L.data_end;
  const bool planned = plan.ok && tv == tile_vecs && !padded;
  const int64_t blk = page_block(P.meta, page);
  uint8_t* blob = P.out + page * P.blob_stride;
  if (blk < 0) {  // block outside the pool: this tile's share of the blob becomes zeros (magic 0)
    if (sec_lo == 0) {  // once per tile (a wire-order egress produces the other sections in later launches)
      const int64_t chunk = (P.blob_stride + n_tiles - 1) / n_tiles;
      const int64_t a = (int64_t)tile * chunk, b = min(a + chunk, P.blob_stride);
      for (int64_t x = a + threadIdx.x; x < b; x += blockDim.x) blob[x] = 0;
    }
    return;
  }
  if (!planned && threadIdx.x == 0)
    build_range_table(T, L, v0, tv, stage_q, stage_s, with_pad, P.payload_len, sec_lo, sec_hi);
  const uint16_t* kp = P.k + blk * page_elems;
  const uint16_t* vp = P.v ? P.v + blk * page_elems : nullptr;

  if (CFG && G.rows_ok && planned) {
    // Staged rows: one thread starts two bulk copies of the tile's K and V rows into shared memory, completing
    // on an mbarrier, and every thread computes its keystream block while they land -- the load latency that
    // the quantizer would otherwise wait out hides under the keystream.
    __shared__ __align__(8) uint64_t rows_bar;
    uint8_t* kin = stage + G.stage_bytes;
    uint8_t* vin = kin + G.rows_bytes;
    const uint32_t bar = (uint32_t)__cvta_generic_to_shared(&rows_bar);
    if (threadIdx.x == 0) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                   "r"((uint32_t)(vp ? 2 * G.rows_bytes : G.rows_bytes))
                   : "memory");
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                       (uint32_t)__cvta_generic_to_shared(kin)),
                   "l"(kp + v0 * head_dim), "r"((uint32_t)G.rows_bytes), "r"(bar)
                   : "memory");
      if (vp)
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         (uint32_t)__cvta_generic_to_shared(vin)),
                     "l"(vp + v0 * head_dim), "r"((uint32_t)G.rows_bytes), "r"(bar)
                     : "memory");
    }
    const uint64_t seq = page_seq(P.meta, page);
    const uint16_t layer = page_layer(P.meta, page);
    const uint32_t n2 = ((uint32_t)layer << 16) | P.meta.head_group;
    const int bi = threadIdx.x;  // this thread's block of the tile (one per thread: rows_ok)
    const bool has_block = bi < plan.first[plan.n];
    uint32_t ks[16];
    int kb = 0, soff = 0;
    if (has_block) {
      const int i = plan_range(plan, bi);
      const int rel = bi - plan.first[i];
      kb = plan.kb0[i] + tile * (plan.first[i + 1] - plan.first[i]) + rel;
      soff = plan.stage[i] + rel * 64;
      chacha20_block(P.key, (uint32_t)(1 + kb), (uint32_t)seq, (uint32_t)(seq >> 32), n2, ks);
    }
    __syncthreads();  // the barrier's initialization is visible to every thread
    // Bounded wait: each try_wait suspends for a while, and the copies read valid pool memory, so they land
    // within microseconds.  Should they not within the limit, the threads copy the rows themselves -- the
    // same bytes the bulk copies carry, so a copy landing late changes nothing -- and thread 0 waits once
    // more, with the same limit, before the CTA gives up its shared memory.
    const bool landed = __syncthreads_and(mbar_wait_parity0(bar));
    if (!landed) {
      const uint4* ks16 = reinterpret_cast<const uint4*>(kp + v0 * head_dim);
      const uint4* vs16 = vp ? reinterpret_cast<const uint4*>(vp + v0 * head_dim) : nullptr;
      for (int c = threadIdx.x; c < G.rows_bytes / 16; c += kTileThreads) {
        reinterpret_cast<uint4*>(kin)[c] = __ldg(ks16 + c);
        if (vs16) reinterpret_cast<uint4*>(vin)[c] = __ldg(vs16 + c);
      }
      __syncthreads();
    }
#pragma unroll
    for (int s = 0; s < 3; ++s) {
      if (s >= L.n) break;
      const Section S = L.sec[s];
      const SectionTile st{reinterpret_cast<const uint16_t*>(S.buf ? vin : kin) + S.col, stage + stage_q[s],
                           stage + stage_s[s], head_dim, S.q_bpv, S.s_bpv, S.dim >> 4, gshift[s], tv};
      if (S.kind == kInt4) quantize_section<kInt4, BF16, NEON, true>(st, P.mul);
      else if (S.kind == kInt8) quantize_section<kInt8, BF16, NEON, true>(st, P.mul);
      else quantize_section<kRaw, BF16, NEON, true>(st, P.mul);
    }
    if (tile == 0 && threadIdx.x == 0) write_header(blob, G.flags, P.meta, page, seq, layer);
    __syncthreads();
    if (has_block) {
      const uint4* src = reinterpret_cast<const uint4*>(stage + soff);
      uint4* dst = reinterpret_cast<uint4*>(blob + kHeaderBytes + (int64_t)kb * 64);
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        uint4 pt = src[w];
        pt.x ^= ks[4 * w]; pt.y ^= ks[4 * w + 1]; pt.z ^= ks[4 * w + 2]; pt.w ^= ks[4 * w + 3];
        dst[w] = pt;
      }
    }
    if (!landed && threadIdx.x == 0) mbar_wait_parity0(bar);
    return;
  }

  // ---- phase 1: quantize this tile's rows of every section this launch produces into shared memory
#pragma unroll
  for (int s = 0; s < 3; ++s) {
    if (s >= sec_hi) break;
    if (s < sec_lo) continue;
    const Section S = L.sec[s];
    const SectionTile st{(S.buf ? vp : kp) + v0 * head_dim + S.col, stage + stage_q[s], stage + stage_s[s],
                         head_dim, S.q_bpv, S.s_bpv, S.dim >> 4, gshift[s], tv};
    if (S.kind == kInt4) quantize_section<kInt4, BF16, NEON>(st, P.mul);
    else if (S.kind == kInt8) quantize_section<kInt8, BF16, NEON>(st, P.mul);
    else quantize_section<kRaw, BF16, NEON>(st, P.mul);
  }

  // header (32 bytes) by tile 0 (a wire-order egress leaves it to its last tag segment)
  const uint64_t seq = page_seq(P.meta, page);
  const uint16_t layer = page_layer(P.meta, page);
  if (tile == 0 && threadIdx.x == 0 && (CFG || P.write_header))
    write_header(blob, CFG ? G.flags : P.flags, P.meta, page, seq, layer);
  __syncthreads();

  // ---- phase 2: encrypt this tile's byte ranges
  const uint32_t n2 = ((uint32_t)layer << 16) | P.meta.head_group;
  uint8_t* payload = blob + kHeaderBytes;
  if (planned) {  // whole, 16-byte aligned blocks
    const int total = plan.first[plan.n];
    for (int bi = threadIdx.x; bi < total; bi += blockDim.x) {
      const int i = plan_range(plan, bi);
      const int rel = bi - plan.first[i];
      const int kb = plan.kb0[i] + tile * (plan.first[i + 1] - plan.first[i]) + rel;
      uint32_t ks[16];
      chacha20_block(P.key, (uint32_t)(1 + kb), (uint32_t)seq, (uint32_t)(seq >> 32), n2, ks);
      const uint4* src = reinterpret_cast<const uint4*>(stage + plan.stage[i] + rel * 64);
      uint4* dst = reinterpret_cast<uint4*>(payload + (int64_t)kb * 64);
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        uint4 pt = src[w];
        pt.x ^= ks[4 * w]; pt.y ^= ks[4 * w + 1]; pt.z ^= ks[4 * w + 2]; pt.w ^= ks[4 * w + 3];
        dst[w] = pt;
      }
    }
    return;
  }
  const int64_t total_blocks = T.first[T.n];
  for (int64_t bi = threadIdx.x; bi < total_blocks; bi += blockDim.x) {
    const int i = find_range(T, bi);
    const Range r = T.r[i];
    const int64_t kb = (r.a >> 6) + (bi - T.first[i]);
    uint32_t ks[16];
    chacha20_block(P.key, (uint32_t)(1 + kb), (uint32_t)seq, (uint32_t)(seq >> 32), n2, ks);
    const int64_t base = kb << 6;
    const int lo = (int)(max(r.a, base) - base), hi = (int)(min(r.b, base + 64) - base);
    uint8_t* dst = payload + base;
    const uint8_t* src = r.zero ? nullptr : stage + r.stage + (base - r.a);  // only bytes [lo, hi) are read
    const bool full = lo == 0 && hi == 64;
    if (full && ((reinterpret_cast<uintptr_t>(dst) | (r.zero ? 0 : reinterpret_cast<uintptr_t>(src))) & 15) == 0) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        uint4 pt = r.zero ? make_uint4(0, 0, 0, 0) : reinterpret_cast<const uint4*>(src)[w];
        pt.x ^= ks[4 * w]; pt.y ^= ks[4 * w + 1]; pt.z ^= ks[4 * w + 2]; pt.w ^= ks[4 * w + 3];
        reinterpret_cast<uint4*>(dst)[w] = pt;
      }
    } else {
      xor_block_bytes(dst, src, ks, lo, hi);
    }
  }
}

// ------------------------------------------------------------------------------------------------
// SipHash-2-4-128 chains: one lane per page
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t ld_u32_any(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

__device__ __forceinline__ W64 load_word_any(const uint8_t* p) { return W64{ld_u32_any(p), ld_u32_any(p + 4)}; }

// Shared-memory ring of one chain lane: kRing chunks of 128 bytes (16 words), filled ahead of the chain
// by per-thread asynchronous copies (cp.async, 16 bytes each, completed by cp.async.wait_group -- a
// wait on the thread's own copies, which always finish).  The chain consumes ~8 bytes per ~86 cycles,
// so 7 chunks in flight are ~9.6k cycles of lookahead: DRAM latency is hidden whether or not the blob
// is L2-resident.  Lanes' rings are kRingStride apart (1040 = 65 x 16 bytes) so that the 16-byte reads
// of 8 consecutive lanes fall in distinct bank quads.
constexpr int kChunk = 128;
constexpr int kRing = 8;
constexpr int kRingStride = kRing * kChunk + 16;
constexpr int kChainThreads = 128;
constexpr int kRingBytes = kChainThreads * kRingStride;  // 133,120 bytes per chain CTA

__device__ __forceinline__ void cp_async16(uint32_t smem_addr, const void* gptr) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr), "l"(gptr) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ring_fill(uint32_t ring, const uint8_t* p, int64_t chunk, int64_t n_chunks) {
  if (chunk < n_chunks) {
    const uint32_t dst = ring + (uint32_t)(chunk & (kRing - 1)) * kChunk;
    const uint8_t* src = p + chunk * kChunk;
#pragma unroll
    for (int j = 0; j < kChunk / 16; ++j) cp_async16(dst + 16 * j, src + 16 * j);
  }
  cp_async_commit();  // empty groups past the end keep the group count uniform
}

// SipHash-2-4-128 of bytes [0, len) of p: little-endian words, then the length word (csrc:425-442),
// then finalization.  Each word's `v3 ^= m` is folded into the previous word (absorb_pre), so the
// stream is walked with one word of lookahead.  With a 16-byte-aligned p (and a ring, i.e. in the
// chain kernel), whole 128-byte chunks stream through the lane's shared-memory ring; the remainder
// and unaligned blobs use direct loads.
__device__ __forceinline__ void siphash_bytes(SipState& st, const uint8_t* p, int64_t len, uint32_t tag[4],
                                              uint8_t* ring_ptr) {
  const int64_t n_words = len >> 3;
  W64 fin{0u, (uint32_t)(len & 0xff) << 24};
  {
    const int rem = (int)(len & 7);
    const uint8_t* t = p + n_words * 8;
    for (int b = 0; b < rem; ++b) {
      if (b < 4) fin.lo |= (uint32_t)t[b] << (8 * b);
      else fin.hi |= (uint32_t)t[b] << (8 * (b - 4));
    }
  }
  int64_t i0 = 0;  // first word not yet absorbed
  if (ring_ptr != nullptr && (reinterpret_cast<uintptr_t>(p) & 15) == 0 && n_words >= 32) {
    const int64_t n_chunks = n_words >> 4;
    const uint32_t ring = (uint32_t)__cvta_generic_to_shared(ring_ptr);
    auto slot = [&](int64_t c) { return reinterpret_cast<const uint4*>(ring_ptr + (c & (kRing - 1)) * kChunk); };
#pragma unroll 1
    for (int c = 0; c < kRing - 1; ++c) ring_fill(ring, p, c, n_chunks);
    const W64 after = n_chunks * 16 < n_words ? load_word_any(p + n_chunks * kChunk) : fin;
    cp_async_wait<kRing - 2>();  // chunk 0 landed
    st.v3 = xor64(st.v3, load_word_any(p));  // word 0
    // Chunk c is read from the ring a 16-byte pair at a time right before its words are absorbed (the
    // shared-memory loads hide under the previous word's rounds); its last word looks ahead into chunk
    // c+1, which has landed too.  The loop body absorbs four words: the chain runs concurrently with the
    // tile kernels of other batches, and its code footprint costs them instruction-fetch bandwidth.
    // Measured in the 32-batch bench (same call): 4 words per pass 1,791-1,808 GB/s, 8 words 1,714-1,720,
    // 16 words 1,644-1,680, 32 words 1,450-1,466, 2 words 1,764, 1 word 1,731-1,748 -- although the chain
    // alone is fastest at 16 or 32 words (95.6 vs 99.9 cycles/word at 4).
#pragma unroll 1
    for (int64_t c = 0; c < n_chunks; ++c) {
      ring_fill(ring, p, c + kRing - 1, n_chunks);
      cp_async_wait<kRing - 2>();  // chunks c and c+1 landed
      const uint4* w = slot(c);
      const W64 last = c + 1 < n_chunks ? W64{slot(c + 1)[0].x, slot(c + 1)[0].y} : after;
#pragma unroll 1
      for (int h = 0; h < 4; ++h) {  // four words per pass: a short loop body (see below)
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const int j = 2 * h + jj;
          const uint4 q = w[j];
          st.absorb_pre(W64{q.x, q.y}, W64{q.z, q.w});
          W64 nx;
          if (j < 7) {
            const uint4 r = w[j + 1];
            nx = W64{r.x, r.y};
          } else {
            nx = last;
          }
          st.absorb_pre(W64{q.z, q.w}, nx);
        }
      }
    }
    cp_async_wait<0>();
    i0 = n_chunks * 16;
  } else {
    st.v3 = xor64(st.v3, n_words > 0 ? load_word_any(p) : fin);
  }
  for (int64_t i = i0; i < n_words; ++i)
    st.absorb_pre(load_word_any(p + 8 * i), i + 1 < n_words ? load_word_any(p + 8 * (i + 1)) : fin);
  st.absorb_pre(fin, W64{0u, 0u});
  st.finish(tag);
}

template <bool VERIFY>
__global__ void __launch_bounds__(kChainThreads, 1) mac_kernel(const __grid_constant__ MacParams P) {
  extern __shared__ __align__(16) uint8_t rings[];
  const int64_t page = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (page >= P.n_pages) return;
  uint8_t* blob = P.blobs + page * P.blob_stride;
  const int64_t mac_len = kHeaderBytes + P.payload_len;
  int32_t status = 0;
  if (page_block(P.meta, page) < 0) {  // block outside the pool
    if (VERIFY) {
      P.status[page] = 6;  // ZTCP_PAGE_BAD_BLOCK
      atomicOr(P.any_fail, 1);
    } else {
      for (int i = 0; i < (int)kTagBytes; ++i) blob[mac_len + i] = 0;
    }
    return;
  }
  if (VERIFY) {
    uint32_t h[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = ld_u32_any(blob + 4 * i);
    const uint64_t tok = ((uint64_t)h[5] << 32) | h[4];
    if ((h[0] & 0xFFFFu) != kMagic || ((h[0] >> 16) & 0xFFu) != kVersion) status = 1;
    else if (h[1] != P.meta.tenant || h[2] != P.meta.model || (h[3] & 0xFFFFu) != page_layer(P.meta, page) ||
             tok != P.meta.token_hash[page])
      status = 2;
    if (status != 0) {
      P.status[page] = status;
      atomicOr(P.any_fail, 1);
      return;
    }
  }
  SipState st;
  st.init(P.mk0, P.mk1);
  uint32_t tag[4];
  siphash_bytes(st, blob, mac_len, tag, rings + threadIdx.x * kRingStride);
  uint8_t* tag_ptr = blob + mac_len;
  if (!VERIFY) {
    if ((reinterpret_cast<uintptr_t>(tag_ptr) & 3) == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i) reinterpret_cast<uint32_t*>(tag_ptr)[i] = tag[i];
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) tag_ptr[i] = (uint8_t)(tag[i >> 2] >> (8 * (i & 3)));
    }
    return;
  }
  uint32_t diff = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) diff |= tag[i] ^ ld_u32_any(tag_ptr + 4 * i);
  if (diff != 0) {
    status = 3;
  } else {
    const uint8_t flags = blob[3];
    Layout L;
    if (!build_layout(flags & 0x0F, (flags >> 4) & 0x0F, P.vecs, P.head_dim, P.rope_dim, P.has_v != 0, &L))
      status = 4;
    else if (P.payload_len < L.data_end)
      status = 5;
  }
  P.status[page] = status;
  if (status != 0) atomicOr(P.any_fail, 1);
}

// ------------------------------------------------------------------------------------------------
// Tag chains of a wire-order egress, one segment per launch
// ------------------------------------------------------------------------------------------------
// Absorbs n_words little-endian words of p (16-byte aligned, or direct loads otherwise) into st and leaves
// the state clean (the last word folds nothing ahead), so a later launch can continue from it.
__device__ __forceinline__ void sip_absorb_words(SipState& st, const uint8_t* p, int64_t n_words, uint8_t* ring_ptr) {
  if (n_words <= 0) return;
  int64_t i0 = 0;
  if ((reinterpret_cast<uintptr_t>(p) & 15) == 0 && n_words >= 32) {
    const int64_t n_chunks = n_words >> 4;
    const uint32_t ring = (uint32_t)__cvta_generic_to_shared(ring_ptr);
    auto slot = [&](int64_t c) { return reinterpret_cast<const uint4*>(ring_ptr + (c & (kRing - 1)) * kChunk); };
#pragma unroll 1
    for (int c = 0; c < kRing - 1; ++c) ring_fill(ring, p, c, n_chunks);
    const W64 after = n_chunks * 16 < n_words ? load_word_any(p + n_chunks * kChunk) : W64{0u, 0u};
    cp_async_wait<kRing - 2>();
    st.v3 = xor64(st.v3, load_word_any(p));
#pragma unroll 1
    for (int64_t c = 0; c < n_chunks; ++c) {
      ring_fill(ring, p, c + kRing - 1, n_chunks);
      cp_async_wait<kRing - 2>();
      const uint4* w = slot(c);
      const W64 last = c + 1 < n_chunks ? W64{slot(c + 1)[0].x, slot(c + 1)[0].y} : after;
#pragma unroll 1
      for (int h = 0; h < 4; ++h) {
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const int j = 2 * h + jj;
          const uint4 q = w[j];
          st.absorb_pre(W64{q.x, q.y}, W64{q.z, q.w});
          W64 nx;
          if (j < 7) {
            const uint4 r = w[j + 1];
            nx = W64{r.x, r.y};
          } else {
            nx = last;
          }
          st.absorb_pre(W64{q.z, q.w}, nx);
        }
      }
    }
    cp_async_wait<0>();
    i0 = n_chunks * 16;
    if (i0 == n_words) return;
  } else {
    st.v3 = xor64(st.v3, load_word_any(p));
  }
  for (int64_t i = i0; i < n_words; ++i)
    st.absorb_pre(load_word_any(p + 8 * i), i + 1 < n_words ? load_word_any(p + 8 * (i + 1)) : W64{0u, 0u});
}

__device__ __forceinline__ void header_words(const PageMeta& m, int64_t page, int32_t flags, uint32_t hw[8]) {
  const uint64_t tok = m.token_hash[page];
  const uint64_t seq = page_seq(m, page);
  hw[0] = (uint32_t)kMagic | ((uint32_t)kVersion << 16) | ((uint32_t)flags << 24);
  hw[1] = m.tenant;
  hw[2] = m.model;
  hw[3] = (uint32_t)page_layer(m, page) | ((uint32_t)m.head_group << 16);
  hw[4] = (uint32_t)tok;
  hw[5] = (uint32_t)(tok >> 32);
  hw[6] = (uint32_t)seq;
  hw[7] = (uint32_t)(seq >> 32);
}

// One segment of the tag chains (one lane per page, the shape of mac_kernel): blob bytes [seg_from, seg_to)
// are absorbed after the production launches that write them have finished (stream order).  Between launches a
// page's chain state (v0..v3, 32 bytes) waits in its blob's header slot, which nothing else reads until the
// last segment writes the real header there after the tag.
__global__ void __launch_bounds__(kChainThreads, 1) mac_segment_kernel(const __grid_constant__ MacParams P) {
  extern __shared__ __align__(16) uint8_t rings[];
  const int64_t page = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (page >= P.n_pages) return;
  uint8_t* blob = P.blobs + page * P.blob_stride;
  const int64_t mac_len = kHeaderBytes + P.payload_len;
  uint32_t* slot = reinterpret_cast<uint32_t*>(blob);  // 16-byte aligned: checked by the host
  if (page_block(P.meta, page) < 0) {  // block outside the pool: the blob stays zero (written by the tile kernel)
    if (P.seg_last)
      for (int i = 0; i < (int)kTagBytes; ++i) blob[mac_len + i] = 0;
    return;
  }
  SipState st;
  int64_t from = P.seg_from;
  if (P.seg_first) {
    uint32_t hw[8];
    header_words(P.meta, page, P.flags, hw);
    st.init(P.mk0, P.mk1);
#pragma unroll
    for (int i = 0; i < 4; ++i) st.absorb(hw[2 * i], hw[2 * i + 1]);
    from = kHeaderBytes;
  } else {
    const uint4 a = reinterpret_cast<const uint4*>(slot)[0], b = reinterpret_cast<const uint4*>(slot)[1];
    st.v0 = W64{a.x, a.y};
    st.v1 = W64{a.z, a.w};
    st.v2 = W64{b.x, b.y};
    st.v3 = W64{b.z, b.w};
  }
  const int64_t n_words = (P.seg_to - from) >> 3;
  sip_absorb_words(st, blob + from, n_words, rings + threadIdx.x * kRingStride);
  if (!P.seg_last) {
    reinterpret_cast<uint4*>(slot)[0] = make_uint4(st.v0.lo, st.v0.hi, st.v1.lo, st.v1.hi);
    reinterpret_cast<uint4*>(slot)[1] = make_uint4(st.v2.lo, st.v2.hi, st.v3.lo, st.v3.hi);
    return;
  }
  // the length word: (mac_len & 0xff) << 56 | the bytes after the last whole word (csrc:425-442)
  W64 fin{0u, (uint32_t)(mac_len & 0xff) << 24};
  const uint8_t* t = blob + from + 8 * n_words;
  const int rem = (int)(P.seg_to - from - 8 * n_words);
  for (int b = 0; b < rem; ++b) {
    if (b < 4) fin.lo |= (uint32_t)t[b] << (8 * b);
    else fin.hi |= (uint32_t)t[b] << (8 * (b - 4));
  }
  st.absorb(fin);
  uint32_t tag[4];
  st.finish(tag);
  uint8_t* tag_ptr = blob + mac_len;
  if ((reinterpret_cast<uintptr_t>(tag_ptr) & 3) == 0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) reinterpret_cast<uint32_t*>(tag_ptr)[i] = tag[i];
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) tag_ptr[i] = (uint8_t)(tag[i >> 2] >> (8 * (i & 3)));
  }
  uint32_t hw[8];
  header_words(P.meta, page, P.flags, hw);
  reinterpret_cast<uint4*>(slot)[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
  reinterpret_cast<uint4*>(slot)[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
}

// ------------------------------------------------------------------------------------------------
// Ingress: decrypt + dequantize one (page, vec-tile), or zero it when the batch failed
// ------------------------------------------------------------------------------------------------
// Decrypt + dequantize one verified (page, vec-tile) with layout L, its staging offsets and tile plan: either the
// launch parameters' entry for the page's flags, or a compile-time one (the same code with constants).
__device__ __forceinline__ void ingress_tile(const IngressParams& P, RangeTable& T, const Layout& L,
                                             const int32_t (&sq)[3], const int32_t (&ss)[3], const TilePlan& TP,
                                             int tile, int64_t v0, int tv, int tile_vecs, int head_dim,
                                             const uint8_t* payload, uint32_t n0, uint32_t n1, uint32_t n2,
                                             uint16_t* kd, uint16_t* vd) {
  extern __shared__ __align__(16) uint8_t stage[];
  const bool planned = TP.ok && tv == tile_vecs;

  // ---- phase 1: decrypt this tile's byte ranges into shared memory (loads issued before the keystream)
  if (planned) {  // whole, 16-byte aligned blocks
    const int total = TP.first[TP.n];
    for (int bi = threadIdx.x; bi < total; bi += blockDim.x) {
      const int i = plan_range(TP, bi);
      const int rel = bi - TP.first[i];
      const int kb = TP.kb0[i] + tile * (TP.first[i + 1] - TP.first[i]) + rel;
      const uint4* src = reinterpret_cast<const uint4*>(payload + (int64_t)kb * 64);
      uint4 c[4];
#pragma unroll
      for (int w = 0; w < 4; ++w) c[w] = __ldg(src + w);
      uint32_t ks[16];
      chacha20_block(P.key, (uint32_t)(1 + kb), n0, n1, n2, ks);
      uint4* dst = reinterpret_cast<uint4*>(stage + TP.stage[i] + rel * 64);
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        c[w].x ^= ks[4 * w]; c[w].y ^= ks[4 * w + 1]; c[w].z ^= ks[4 * w + 2]; c[w].w ^= ks[4 * w + 3];
        dst[w] = c[w];
      }
    }
  } else {
    if (threadIdx.x == 0) build_range_table(T, L, v0, tv, sq, ss, false, P.payload_len);
    __syncthreads();
    const int64_t total_blocks = T.first[T.n];
    for (int64_t bi = threadIdx.x; bi < total_blocks; bi += blockDim.x) {
      const int i = find_range(T, bi);
      const Range r = T.r[i];
      const int64_t kb = (r.a >> 6) + (bi - T.first[i]);
      uint32_t ks[16];
      const int64_t base = kb << 6;
      const int lo = (int)(max(r.a, base) - base), hi = (int)(min(r.b, base + 64) - base);
      const uint8_t* src = payload + base;
      uint8_t* dst = stage + r.stage + (base - r.a);  // only bytes [lo, hi) are written
      if (lo == 0 && hi == 64 &&
          ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0) {
        uint4 c[4];
#pragma unroll
        for (int w = 0; w < 4; ++w) c[w] = __ldg(reinterpret_cast<const uint4*>(src) + w);
        chacha20_block(P.key, (uint32_t)(1 + kb), n0, n1, n2, ks);
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          c[w].x ^= ks[4 * w]; c[w].y ^= ks[4 * w + 1]; c[w].z ^= ks[4 * w + 2]; c[w].w ^= ks[4 * w + 3];
          reinterpret_cast<uint4*>(dst)[w] = c[w];
        }
      } else {
        chacha20_block(P.key, (uint32_t)(1 + kb), n0, n1, n2, ks);
#pragma unroll
        for (int w = 0; w < 16; ++w) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int x = 4 * w + j;
            if (x >= lo && x < hi) dst[x] = (uint8_t)(src[x] ^ (uint8_t)(ks[w] >> (8 * j)));
          }
        }
      }
    }
  }
  __syncthreads();

  // ---- phase 2: dequantize into the paged KV layout
#pragma unroll
  for (int s = 0; s < 3; ++s) {
    if (s >= L.n) break;
    const Section S = L.sec[s];
    const int32_t groups = S.dim >> 4;
    const SectionTile st{nullptr, stage + sq[s], stage + ss[s], head_dim, S.q_bpv, S.s_bpv, groups,
                         log2_if_pow2(groups), tv};
    uint16_t* dst = (S.buf ? vd : kd) + v0 * head_dim + S.col;
    if (S.kind == kInt4) dequantize_section<kInt4>(st, dst);
    else if (S.kind == kInt8) dequantize_section<kInt8>(st, dst);
    else dequantize_section<kRaw>(st, dst);
  }
}

// 6 resident CTAs per SM (measured ~9 % faster than the 5 its unconstrained register count allows).
// CFG = 0: geometry, tiling and the layouts of every header flags byte from the launch parameters; CFG = i > 0:
// those of kStaticIngress[i - 1] as compile-time constants, with the layouts of the formats it lists (the
// benchmark configurations' flags) each in its own copy of the tile code.
template <int CFG>
__global__ void __launch_bounds__(kTileThreads, 6) ingress_tile_kernel(const __grid_constant__ IngressParams P) {
  __shared__ RangeTable T;
  const StaticIngress& G = kStaticIngress[CFG > 0 ? CFG - 1 : 0];
  const int tile_vecs = CFG ? G.tile_vecs : P.tile_vecs;
  const int n_tiles = CFG ? G.n_tiles : P.n_tiles;
  const int64_t vecs = CFG ? G.vecs : P.vecs;
  const int head_dim = CFG ? G.head_dim : P.head_dim;
  const int64_t page_elems = CFG ? G.page_elems : P.page_elems;
  const int64_t page = blockIdx.x / n_tiles;
  const int tile = (int)(blockIdx.x - page * n_tiles);
  const int64_t v0 = (int64_t)tile * tile_vecs;
  const int tv = (int)min((int64_t)tile_vecs, vecs - v0);
  const int64_t blk = page_block(P.meta, page);
  if (blk < 0) return;  // block outside the pool: never written (status ZTCP_PAGE_BAD_BLOCK)
  uint16_t* kd = P.k_out + blk * page_elems;
  uint16_t* vd = P.v_out ? P.v_out + blk * page_elems : nullptr;

  if (P.page_fallback ? P.status[page] != 0 : *P.any_fail != 0) {
    const int64_t n16 = (int64_t)tv * head_dim / 8;  // uint4 per buffer
    uint4* kz = reinterpret_cast<uint4*>(kd + v0 * head_dim);
    uint4* vz = vd ? reinterpret_cast<uint4*>(vd + v0 * head_dim) : nullptr;
    for (int64_t i = threadIdx.x; i < n16; i += blockDim.x) {
      kz[i] = make_uint4(0, 0, 0, 0);
      if (vz) vz[i] = make_uint4(0, 0, 0, 0);
    }
    return;
  }

  // header: the flags byte selects the page's layout; nonce words for the keystream (seq lo, seq hi,
  // layer_id << 16 | head_group_id)
  const uint8_t* blob = P.blobs + page * P.blob_stride;
  uint32_t h0, h3, h6, h7;
  if ((reinterpret_cast<uintptr_t>(blob) & 15) == 0) {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(blob));
    const uint4 b = __ldg(reinterpret_cast<const uint4*>(blob) + 1);
    h0 = a.x; h3 = a.w; h6 = b.z; h7 = b.w;
  } else {
    h0 = ld_u32_any(blob); h3 = ld_u32_any(blob + 12); h6 = ld_u32_any(blob + 24); h7 = ld_u32_any(blob + 28);
  }
  const uint32_t flags = h0 >> 24;
  const int li = (int)((flags & 0x0Fu) - 1u) * 3 + (int)((flags >> 4) & 0x0Fu);
  const uint32_t n0 = h6, n1 = h7, n2 = (h3 << 16) | (h3 >> 16);
  const uint8_t* payload = blob + kHeaderBytes;
  if (CFG && li == kStaticIngressFast0) {
    constexpr int F = kStaticIngressFast0;
    ingress_tile(P, T, G.lay[F], G.lay_q[F], G.lay_s[F], G.plan[F], tile, v0, tv, tile_vecs, head_dim, payload,
                 n0, n1, n2, kd, vd);
  } else if (CFG && li == kStaticIngressFast1) {
    constexpr int F = kStaticIngressFast1;
    ingress_tile(P, T, G.lay[F], G.lay_q[F], G.lay_s[F], G.plan[F], tile, v0, tv, tile_vecs, head_dim, payload,
                 n0, n1, n2, kd, vd);
  } else {
    ingress_tile(P, T, P.lay[li], P.lay_q[li], P.lay_s[li], P.plan[li], tile, v0, tv, tile_vecs, head_dim, payload,
                 n0, n1, n2, kd, vd);
  }
}

// ------------------------------------------------------------------------------------------------
// Known-answer entry points (csrc:2499-2538)
// ------------------------------------------------------------------------------------------------
__global__ void chacha20_xor_kernel(const uint8_t* src, uint8_t* dst, int64_t len, const uint32_t k0, uint32_t k1,
                                    uint32_t k2, uint32_t k3, uint32_t k4, uint32_t k5, uint32_t k6, uint32_t k7,
                                    uint32_t counter0, uint32_t n0, uint32_t n1, uint32_t n2) {
  const int64_t kb = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (kb * 64 >= len) return;
  const uint32_t key[8] = {k0, k1, k2, k3, k4, k5, k6, k7};
  uint32_t ks[16];
  chacha20_block(key, counter0 + (uint32_t)kb, n0, n1, n2, ks);
  const int hi = (int)min((int64_t)64, len - kb * 64);
  const uint8_t* s = src + kb * 64;
  uint8_t* d = dst + kb * 64;
#pragma unroll
  for (int w = 0; w < 16; ++w) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int x = 4 * w + j;
      if (x < hi) d[x] = (uint8_t)(s[x] ^ (uint8_t)(ks[w] >> (8 * j)));
    }
  }
}

__global__ void siphash_kernel(const uint8_t* src, int64_t len, uint64_t k0, uint64_t k1, uint8_t* out16) {
  if (blockIdx.x != 0 || threadIdx.x != 0) return;
  SipState st;
  st.init(k0, k1);
  uint32_t tag[4];
  siphash_bytes(st, src, len, tag, nullptr);
#pragma unroll
  for (int i = 0; i < 16; ++i) out16[i] = (uint8_t)(tag[i >> 2] >> (8 * (i & 3)));
}

// Shared memory a chain CTA takes: the sm_100 per-CTA maximum (227 KB), so it owns its SM.
constexpr int kMacReserveBytes = 227 * 1024;

// Dynamic shared memory above 48 KB needs a per-kernel, per-device opt-in.  It is raised, never lowered (a
// lower setting would fail the launches of larger tiles made before), and set only when a launch needs more
// than the kernel was opened to on this device.
struct OptIn {
  const void* fn;
  int dev;
  int32_t bytes;
};
std::mutex g_optin_mu;
OptIn g_optin[64];
int g_optin_n = 0;

template <typename K>
void ensure_smem(K kernel, int32_t bytes) {
  if (bytes <= 48 * 1024) return;
  const void* fn = reinterpret_cast<const void*>(kernel);
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(g_optin_mu);
  OptIn* rec = nullptr;
  for (int i = 0; i < g_optin_n; ++i)
    if (g_optin[i].fn == fn && g_optin[i].dev == dev) rec = &g_optin[i];
  if (rec && rec->bytes >= bytes) return;
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (rec) rec->bytes = bytes;
  else if (g_optin_n < 64) g_optin[g_optin_n++] = OptIn{fn, dev, bytes};
}

}  // namespace

namespace {

// Host copies of the compiled tables (the same compile-time values), for matching launches against them.
constexpr StaticEgress kStaticEgressHost[kStaticEgressCount] = {
    make_static_egress(kStaticEgressKeys[0][0], kStaticEgressKeys[0][1], kStaticEgressGeometry[0]),
    make_static_egress(kStaticEgressKeys[1][0], kStaticEgressKeys[1][1], kStaticEgressGeometry[1]),
    make_static_egress(kStaticEgressKeys[2][0], kStaticEgressKeys[2][1], kStaticEgressGeometry[2])};
constexpr StaticIngress kStaticIngressHost[kStaticIngressCount] = {
    make_static_ingress(kStaticIngressGeometry[0]), make_static_ingress(kStaticIngressGeometry[1])};

bool same(const Section& a, const Section& b) {
  return a.kind == b.kind && a.buf == b.buf && a.col == b.col && a.dim == b.dim && a.q_off == b.q_off &&
         a.s_off == b.s_off && a.q_bpv == b.q_bpv && a.s_bpv == b.s_bpv;
}
bool same(const Layout& a, const Layout& b) {
  if (a.n != b.n || a.data_end != b.data_end) return false;
  for (int i = 0; i < a.n; ++i)
    if (!same(a.sec[i], b.sec[i])) return false;
  return true;
}
bool same(const TilePlan& a, const TilePlan& b) {
  if (a.ok != b.ok || a.n != b.n) return false;
  if (!a.ok) return true;
  for (int i = 0; i <= a.n; ++i)
    if (a.first[i] != b.first[i]) return false;
  for (int i = 0; i < a.n; ++i)
    if (a.kb0[i] != b.kb0[i] || a.stage[i] != b.stage[i]) return false;
  return true;
}
bool same3(const int32_t (&a)[3], const int32_t (&b)[3]) { return a[0] == b[0] && a[1] == b[1] && a[2] == b[2]; }

template <bool BF16, bool NEON, int CFG>
void launch_egress_t(const EgressParams& P, cudaStream_t stream) {
  const int64_t grid = P.n_pages * P.tiles;
  // a compiled geometry that stages its rows takes their room after the staging area
  const int32_t smem = CFG ? kStaticEgressHost[CFG - 1].rows_smem : P.stage_bytes;
  ensure_smem(egress_tile_kernel<BF16, NEON, CFG>, smem);
  egress_tile_kernel<BF16, NEON, CFG><<<(unsigned)grid, kTileThreads, smem, stream>>>(P);
}

template <bool BF16>
void launch_egress_x86(const EgressParams& P, cudaStream_t stream) {
  switch (static_egress_index(P)) {
    case 1: launch_egress_t<BF16, false, 1>(P, stream); break;
    case 2: launch_egress_t<BF16, false, 2>(P, stream); break;
    case 3: launch_egress_t<BF16, false, 3>(P, stream); break;
    default: launch_egress_t<BF16, false, 0>(P, stream); break;
  }
}

}  // namespace

int static_egress_index(const EgressParams& P) {
  if (P.neon_arith || P.sec_lo != 0 || P.sec_hi != P.L.n || P.tile_lo != 0 || P.tiles != P.n_tiles || !P.write_header)
    return 0;
  for (int i = 0; i < kStaticEgressCount; ++i) {
    const StaticEgress& S = kStaticEgressHost[i];
    if (P.vecs == S.vecs && P.head_dim == S.head_dim && P.page_elems == S.page_elems && P.flags == S.flags &&
        P.tile_vecs == S.tile_vecs && P.n_tiles == S.n_tiles && P.stage_bytes == S.stage_bytes && same(P.L, S.L) &&
        same(P.plan, S.plan) && same3(P.stage_q, S.stage_q) && same3(P.stage_s, S.stage_s) && same3(P.gshift, S.gshift))
      return i + 1;
  }
  return 0;
}

int static_ingress_index(const IngressParams& P) {
  for (int i = 0; i < kStaticIngressCount; ++i) {
    const StaticIngress& S = kStaticIngressHost[i];
    if (P.vecs != S.vecs || P.head_dim != S.head_dim || P.page_elems != S.page_elems || P.has_v != S.has_v ||
        P.tile_vecs != S.tile_vecs || P.n_tiles != S.n_tiles || P.stage_bytes != S.stage_bytes)
      continue;
    bool eq = true;
    for (int l = 0; l < 9 && eq; ++l)
      eq = same(P.lay[l], S.lay[l]) && same(P.plan[l], S.plan[l]) && same3(P.lay_q[l], S.lay_q[l]) &&
           same3(P.lay_s[l], S.lay_s[l]);
    if (eq) return i + 1;
  }
  return 0;
}

void launch_egress(const EgressParams& P, bool bf16, cudaStream_t stream) {
  if (P.neon_arith) {
    if (bf16) launch_egress_t<true, true, 0>(P, stream);
    else launch_egress_t<false, true, 0>(P, stream);
  } else {
    if (bf16) launch_egress_x86<true>(P, stream);
    else launch_egress_x86<false>(P, stream);
  }
}

void launch_mac(const MacParams& P, bool verify, cudaStream_t stream) {
  // A chain CTA is four warps, one per SM sub-partition, each running 32 independent per-page chains
  // that keep the sub-partition's ALU pipe busy.  The CTA takes the SM's whole shared memory (its
  // lanes' input rings use 133 KB of it) so that no other CTA -- another chain CTA or a tile kernel
  // running concurrently on another stream -- is co-scheduled on its sub-partitions.
  static_assert(kRingBytes <= kMacReserveBytes, "chain rings must fit the reserved shared memory");
  const unsigned grid = (unsigned)((P.n_pages + kChainThreads - 1) / kChainThreads);
  // the shared-memory opt-in is a per-device property of each kernel: set it on a device's first launch
  static std::atomic<uint64_t> opted[2];
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = dev < 64 ? (uint64_t)1 << dev : 0;
  if (!bit || !(opted[verify].load(std::memory_order_relaxed) & bit)) {
    if (verify) cudaFuncSetAttribute(mac_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMacReserveBytes);
    else cudaFuncSetAttribute(mac_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMacReserveBytes);
    opted[verify].fetch_or(bit, std::memory_order_relaxed);
  }
  if (verify) mac_kernel<true><<<grid, kChainThreads, kMacReserveBytes, stream>>>(P);
  else mac_kernel<false><<<grid, kChainThreads, kMacReserveBytes, stream>>>(P);
}

void launch_mac_segment(const MacParams& P, cudaStream_t stream) {
  const unsigned grid = (unsigned)((P.n_pages + kChainThreads - 1) / kChainThreads);
  static std::atomic<uint64_t> opted;
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = dev < 64 ? (uint64_t)1 << dev : 0;
  if (!bit || !(opted.load(std::memory_order_relaxed) & bit)) {
    cudaFuncSetAttribute(mac_segment_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMacReserveBytes);
    opted.fetch_or(bit, std::memory_order_relaxed);
  }
  mac_segment_kernel<<<grid, kChainThreads, kMacReserveBytes, stream>>>(P);
}

namespace {

template <int CFG>
void launch_ingress_t(const IngressParams& P, cudaStream_t stream) {
  const int64_t grid = P.n_pages * P.n_tiles;
  ensure_smem(ingress_tile_kernel<CFG>, P.stage_bytes);
  ingress_tile_kernel<CFG><<<(unsigned)grid, kTileThreads, P.stage_bytes, stream>>>(P);
}

}  // namespace

void launch_ingress(const IngressParams& P, cudaStream_t stream) {
  switch (static_ingress_index(P)) {
    case 1: launch_ingress_t<1>(P, stream); break;
    case 2: launch_ingress_t<2>(P, stream); break;
    default: launch_ingress_t<0>(P, stream); break;
  }
}

void launch_chacha20_xor(const uint8_t* src, uint8_t* dst, int64_t len, const uint32_t key[8], uint32_t counter0,
                         const uint32_t nonce[3], cudaStream_t stream) {
  const int64_t blocks = (len + 63) / 64;
  const unsigned grid = (unsigned)((blocks + 127) / 128);
  chacha20_xor_kernel<<<grid, 128, 0, stream>>>(src, dst, len, key[0], key[1], key[2], key[3], key[4], key[5],
                                                key[6], key[7], counter0, nonce[0], nonce[1], nonce[2]);
}

void launch_siphash(const uint8_t* src, int64_t len, uint64_t k0, uint64_t k1, uint8_t* out16, cudaStream_t stream) {
  siphash_kernel<<<1, 32, 0, stream>>>(src, len, k0, k1, out16);
}

}  // namespace ztcp
