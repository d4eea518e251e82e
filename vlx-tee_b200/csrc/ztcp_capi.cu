// ztcp_capi.cu -- host layer of the C-ABI declared in include/ztcp_b200.h.
//
// Validates arguments with the reference's TORCH_CHECK rules and messages (csrc:1499-1507,
// 1925-1957, 2269-2296), plans the tiling and launches the kernels on the caller's stream.  Nothing
// here allocates device memory or synchronizes.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "../../include/ztcp_b200.h"
#include "ztcp_kernels.cuh"
#include "ztcp_layout.h"

static_assert(sizeof(ztcp::IngressParams) <= 4096 && sizeof(ztcp::EgressParams) <= 4096,
              "kernel parameter blocks must fit the classic 4 KB limit");

namespace {

thread_local std::string g_last_error;

// Shared memory one tile may stage (the sm_100 opt-in limit is 227 KB per CTA).
constexpr int64_t kMaxStageBytes = 200 * 1024;

int32_t fail(int32_t code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Geometry rule of the reference (csrc:1507, :1930): positive tokens/heads, head_dim a positive multiple
// of 16, rope_dim a multiple of 16 in [0, head_dim].
int32_t check_geometry(const ztcp_geometry* g, const char* dims_msg) {
  if (!g) return fail(ZTCP_EINVAL, "geometry must not be NULL");
  if (!(g->num_tokens > 0 && g->num_heads > 0 && g->head_dim >= 16 && (g->head_dim % 16) == 0))
    return fail(ZTCP_EINVAL, dims_msg);
  if (!(g->rope_dim >= 0 && g->rope_dim <= g->head_dim && (g->rope_dim % 16) == 0))
    return fail(ZTCP_EINVAL, "Invalid rope_dim");
  const int64_t vecs = g->num_tokens * g->num_heads;
  if (vecs > (int64_t)1 << 31 || g->head_dim > (int64_t)1 << 20) return fail(ZTCP_EINVAL, "KV page geometry too large");
  return ZTCP_OK;
}

int32_t check_batch(const ztcp_page_batch* b) {
  if (!b) return fail(ZTCP_EINVAL, "page batch must not be NULL");
  if (b->n_pages <= 0) return fail(ZTCP_EINVAL, "batch must hold at least one page");
  if (!b->token_hash) return fail(ZTCP_EINVAL, "page_token_hashes must not be NULL");
  if (b->options & ~(ZTCP_OPT_NEON_ARITH | ZTCP_OPT_PAGE_FALLBACK)) return fail(ZTCP_EINVAL, "unknown page batch options");
  if (b->kv_pool_pages < 0) return fail(ZTCP_EINVAL, "kv_pool_pages must be non-negative");
  if (b->kv_block && b->kv_pool_pages == 0)
    return fail(ZTCP_EINVAL, "kv_pool_pages is required with a block table (kv_block entries are checked against it)");
  if (!b->kv_block && b->kv_pool_pages > 0 && b->n_pages > b->kv_pool_pages)
    return fail(ZTCP_EINVAL, "batch has more pages than kv_pool_pages");
  return ZTCP_OK;
}

ztcp::PageMeta to_meta(const ztcp_page_batch* b) {
  ztcp::PageMeta m;
  m.kv_block = b->kv_block;
  m.pool_pages = b->kv_pool_pages;
  m.token_hash = b->token_hash;
  m.sequence_nonce = b->sequence_nonce;
  m.layer_id = b->layer_id;
  m.seq_base = b->base_sequence_nonce;
  m.tenant = b->tenant_id_hash;
  m.model = b->model_id_hash;
  m.layer_uniform = b->layer_id_uniform;
  m.head_group = b->head_group_id;
  return m;
}

void key_words(const ztcp_keys* k, uint32_t out[8]) {
  for (int i = 0; i < 4; ++i) {
    out[2 * i] = (uint32_t)k->enc[i];
    out[2 * i + 1] = (uint32_t)(k->enc[i] >> 32);
  }
}

int32_t launch_status(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(ZTCP_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return ZTCP_OK;
}

}  // namespace

int32_t ztcp::set_last_error(int32_t code, const std::string& msg) { return fail(code, msg); }

// ------------------------------------------------------------------------------------------------
// Wire-order egress of large batches
// ------------------------------------------------------------------------------------------------
// A page's tag is one serial SipHash chain over its blob (~0.6 ms for a cfg0 page), and it can only absorb
// bytes that are final.  Produced page by page (tile kernel, then chain), a large batch's chains start only
// once all of its tiles are done, so its egress takes the production time plus a chain.  In wire order --
// one launch per (section, tile range) of every page, in the blob's byte order -- each launch finalizes the
// next byte range of every page, and the chains follow it segment by segment on a high-priority side
// stream, so they run while the rest of the batch is produced: egress takes about max(production, chain).
// Ordering is by stream events only (no kernel waits on another), and the chain state between segments
// lives in each blob's header slot (the last segment writes the header), so no memory is allocated.
namespace {

constexpr int64_t kWireOrderMinPages = 1024;  // 8 chain CTAs; smaller batches gain little over one pass
constexpr int kMaxLaunches = 16;              // production launches of one wire-order egress
constexpr int kMaxSideDevices = 64;
constexpr int32_t kNotWireOrder = 1;          // encode_wire_order: not applicable, take the single pass

struct Launch {
  int32_t sec, tile_vecs, t0, t1;  // section sec of tiles [t0, t1) (of tile_vecs vecs) in every page
  int64_t frontier;                // blob bytes [0, frontier) of every page are final once this launch is done
};

struct ChainSeg {
  int64_t from, to;  // blob bytes the tag chains absorb
  int32_t after;     // the production launch whose completion (and all before it) the segment waits for
};

// Vecs per tile of a one-section launch: about 1,024 groups per CTA, as a whole-page tile of the standard
// geometry holds, so a CTA's fixed costs weigh the same; staging stays under 96 KB.
int32_t section_tile_vecs(const ztcp::EgressParams& P, int s) {
  const ztcp::Section& S = P.L.sec[s];
  int64_t tv = std::min<int64_t>(std::max<int64_t>(1024 / std::max(S.dim / ztcp::kGroup, 1), 1), P.vecs);
  while (tv > 1 && tv * (S.q_bpv + S.s_bpv) + 32 > 96 * 1024) tv = (tv + 1) / 2;
  return (int32_t)tv;
}

// Production launches in wire order, one per tile of each section's tiling (up to four per section).  Chain
// segments: the first two launches' bytes one segment each (the chains start as soon as the first launch is
// done and stay just behind production), then the remaining launches in two segments -- each segment costs
// ~15-20 us of launch, SM hand-over and ring start-up on top of its words, and production stays ahead of the
// chains from there on (a 4,096-page cfg0 egress: ~0.52 ms of production on the SMs the chains leave, 0.62 ms
// of chain).  Returns false when a boundary is not 16-byte aligned (the chains stream whole 16-byte units
// through their rings).
bool plan_wire_order(const ztcp::EgressParams& P, Launch L[kMaxLaunches], int* nl, ChainSeg C[kMaxLaunches], int* nc) {
  const int64_t mac_len = ztcp::kHeaderBytes + P.payload_len;
  int n = 0;
  for (int s = 0; s < P.L.n; ++s) {
    const ztcp::Section& S = P.L.sec[s];
    const int32_t tv = section_tile_vecs(P, s);
    const int32_t T = (int32_t)((P.vecs + tv - 1) / tv);
    const int32_t g = std::min<int32_t>(T, 4);
    for (int k = 0; k < g; ++k) {
      const int32_t t0 = (int32_t)((int64_t)T * k / g), t1 = (int32_t)((int64_t)T * (k + 1) / g);
      if (n == kMaxLaunches) return false;
      const int64_t frontier = t1 < T ? ztcp::kHeaderBytes + S.q_off + std::min<int64_t>((int64_t)t1 * tv, P.vecs) * S.q_bpv
                                      : (s + 1 < P.L.n ? ztcp::kHeaderBytes + P.L.sec[s + 1].q_off : mac_len);
      if (frontier % 16 != 0 && frontier != mac_len) return false;
      L[n++] = Launch{s, tv, t0, t1, frontier};
    }
  }
  int m = 0;
  int64_t from = 0;
  const int rest = n - 2, half = (rest + 1) / 2;
  for (int j = 0; j < n; ++j) {
    const bool ends = j < 2 || j == n - 1 || (rest > 1 && j == 1 + half);
    if (!ends) continue;
    C[m++] = ChainSeg{from, L[j].frontier, j};
    from = L[j].frontier;
  }
  *nl = n;
  *nc = m;
  return m >= 2;
}

// One production launch with its section's own tiling and staging, no header.
void section_launch(const ztcp::EgressParams& P, const Launch& l, bool aligned, ztcp::EgressParams* Q) {
  *Q = P;
  const int s = l.sec;
  Q->tile_vecs = l.tile_vecs;
  Q->n_tiles = (int32_t)((P.vecs + l.tile_vecs - 1) / l.tile_vecs);
  Q->sec_lo = s;
  Q->sec_hi = s + 1;
  Q->tile_lo = l.t0;
  Q->tiles = l.t1 - l.t0;
  Q->write_header = 0;
  const ztcp::Section& S = P.L.sec[s];
  for (int i = 0; i < 3; ++i) Q->stage_q[i] = Q->stage_s[i] = 0;
  Q->stage_s[s] = (int32_t)(((int64_t)Q->tile_vecs * S.q_bpv + 15) / 16 * 16);
  Q->stage_bytes = Q->stage_s[s] + (int32_t)(((int64_t)Q->tile_vecs * S.s_bpv + 15) / 16 * 16);
  ztcp::build_tile_plan(Q->L, Q->tile_vecs, Q->stage_q, Q->stage_s, aligned, &Q->plan, s, s + 1);
}

// Per device: the chains' side stream (highest priority), a second production stream (consecutive production
// launches alternate between the caller's stream and it, so one launch's last wave overlaps the next one's
// first) and the events that order them.  Created on a device's first wire-order egress and kept until the
// process exits (driver objects, no device memory of the caller's).
struct SideStream {
  cudaStream_t chain = nullptr, prod = nullptr;
  cudaEvent_t ev[kMaxLaunches + 3] = {};
  bool ready = false;
};
std::mutex g_side_mu;
SideStream g_side[kMaxSideDevices];

// The current device's side streams and events, created on first use; null on failure.
SideStream* side_streams() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxSideDevices) return nullptr;
  SideStream& S = g_side[dev];
  if (S.ready) return &S;
  int least = 0, greatest = 0;
  cudaDeviceGetStreamPriorityRange(&least, &greatest);
  if (!S.chain && cudaStreamCreateWithPriority(&S.chain, cudaStreamNonBlocking, greatest) != cudaSuccess) return nullptr;
  if (!S.prod && cudaStreamCreateWithFlags(&S.prod, cudaStreamNonBlocking) != cudaSuccess) return nullptr;
  for (auto& e : S.ev)
    if (!e && cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return nullptr;
  S.ready = true;
  return &S;
}

int32_t encode_wire_order(const ztcp::EgressParams& P, const ztcp::MacParams& M, bool bf16, cudaStream_t s) {
  Launch L[kMaxLaunches];
  ChainSeg C[kMaxLaunches];
  int nl = 0, nc = 0;
  const bool aligned = ((reinterpret_cast<uintptr_t>(P.out) | (uintptr_t)P.blob_stride) % 16) == 0;
  if (!aligned || !plan_wire_order(P, L, &nl, C, &nc)) return kNotWireOrder;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return kNotWireOrder;  // a captured call stays on the caller's stream
  }
  // one call's records and waits are enqueued together: the side streams and events are shared per device
  std::lock_guard<std::mutex> lock(g_side_mu);
  SideStream* side = side_streams();
  if (!side) {
    cudaGetLastError();
    return kNotWireOrder;
  }
  // ev[j]: production launch j done; ev[nl]: chains done; ev[nl + 1]: call start; ev[nl + 2]: second stream done
  cudaEvent_t* ev = side->ev;
  auto record_wait = [](cudaEvent_t e, cudaStream_t from, cudaStream_t to) {
    if (cudaEventRecord(e, from) != cudaSuccess || cudaStreamWaitEvent(to, e, 0) != cudaSuccess)
      return launch_status("cudaStreamWaitEvent");
    return (int32_t)ZTCP_OK;
  };
  int32_t rc = record_wait(ev[nl + 1], s, side->prod);  // the second production stream follows the caller's work
  if (rc != ZTCP_OK) return rc;
  // On a failure after the first launch, the caller's stream still waits for what the side streams hold, so no
  // work of this call runs after the caller's next operation on its buffers.
  auto fail_joined = [&](int32_t code) {
    const std::string msg = g_last_error;
    cudaEventRecord(ev[nl + 2], side->prod);
    cudaStreamWaitEvent(s, ev[nl + 2], 0);
    cudaEventRecord(ev[nl], side->chain);
    cudaStreamWaitEvent(s, ev[nl], 0);
    g_last_error = msg;
    return code;
  };
  int c = 0;
  for (int j = 0; j < nl; ++j) {
    ztcp::EgressParams Q;
    section_launch(P, L[j], aligned, &Q);
    cudaStream_t ps = (j & 1) ? side->prod : s;
    ztcp::launch_egress(Q, bf16, ps);
    if ((rc = launch_status("egress_tile_kernel")) != ZTCP_OK) return fail_joined(rc);
    if ((rc = record_wait(ev[j], ps, side->chain)) != ZTCP_OK) return fail_joined(rc);  // the chains wait for every launch
    if (c < nc && C[c].after == j) {
      ztcp::MacParams K = M;
      K.seg_from = C[c].from;
      K.seg_to = C[c].to;
      K.seg_first = c == 0;
      K.seg_last = c == nc - 1;
      ztcp::launch_mac_segment(K, side->chain);
      if ((rc = launch_status("mac_segment_kernel")) != ZTCP_OK) return fail_joined(rc);
      ++c;
    }
  }
  if ((rc = record_wait(ev[nl + 2], side->prod, s)) != ZTCP_OK) return fail_joined(rc);
  ztcp::take_phase_mark(s);
  if ((rc = record_wait(ev[nl], side->chain, s)) != ZTCP_OK) return fail_joined(rc);
  return ZTCP_OK;
}

}  // namespace

extern "C" {

const char* ztcp_last_error(void) { return g_last_error.c_str(); }

int32_t ztcp_version(void) { return 100; }

int64_t ztcp_min_payload_bytes(int32_t preset, int32_t rope_mode, const ztcp_geometry* geom, int32_t has_v) {
  if (!geom) return -1;
  ztcp::Layout L;
  if (!ztcp::build_layout(preset, rope_mode, geom->num_tokens * geom->num_heads, geom->head_dim, geom->rope_dim,
                          has_v != 0, &L))
    return -1;
  return L.data_end;
}

int64_t ztcp_spec_payload_bytes(int32_t preset, int32_t rope_mode, const ztcp_geometry* geom, int32_t has_v) {
  if (!geom) return -1;
  return ztcp::spec_payload_bytes(preset, rope_mode, geom->num_tokens * geom->num_heads, geom->head_dim,
                                  geom->rope_dim, has_v != 0);
}

int32_t ztcp_encode_pages(const void* k_pages, const void* v_pages, int32_t kv_dtype, const ztcp_geometry* geom,
                          const ztcp_page_batch* batch, int32_t preset, int32_t rope_mode,
                          int64_t expected_payload_bytes, const ztcp_keys* keys, uint8_t* out_blobs, void* stream) {
  int32_t rc = check_geometry(geom, "Invalid k_pages dimensions");
  if (rc != ZTCP_OK) return rc;
  if ((rc = check_batch(batch)) != ZTCP_OK) return rc;
  if (!keys) return fail(ZTCP_EINVAL, "keys must not be NULL");
  if (!k_pages || !out_blobs) return fail(ZTCP_EINVAL, "k_pages and out_blobs must not be NULL");
  if (kv_dtype != ZTCP_DTYPE_F16 && kv_dtype != ZTCP_DTYPE_BF16)
    return fail(ZTCP_EINVAL, "k_pages must be float16 or bfloat16");
  if (!aligned16(k_pages) || (v_pages && !aligned16(v_pages)))
    return fail(ZTCP_EINVAL, "k_pages / v_pages must be 16-byte aligned");
  if (preset < 1 || preset > 3) return fail(ZTCP_EINVAL, "Invalid preset (must be 1..3)");
  if (rope_mode < 0 || rope_mode > 2) return fail(ZTCP_EINVAL, "Invalid rope_mode (must be 0..2)");
  const int64_t vecs = geom->num_tokens * geom->num_heads;
  ztcp::EgressParams P;
  memset(&P, 0, sizeof(P));
  ztcp::build_layout(preset, rope_mode, vecs, geom->head_dim, geom->rope_dim, v_pages != nullptr, &P.L);
  if (expected_payload_bytes < P.L.data_end)
    return fail(ZTCP_EINVAL, "expected_payload_bytes smaller than required payload");
  if (expected_payload_bytes > ((int64_t)1 << 36))
    return fail(ZTCP_EINVAL, "expected_payload_bytes too large");
  P.k = static_cast<const uint16_t*>(k_pages);
  P.v = static_cast<const uint16_t*>(v_pages);
  P.page_elems = vecs * geom->head_dim;
  P.out = out_blobs;
  P.blob_stride = ztcp::kHeaderBytes + expected_payload_bytes + ztcp::kTagBytes;
  P.payload_len = expected_payload_bytes;
  P.vecs = vecs;
  P.head_dim = (int32_t)geom->head_dim;
  P.flags = (preset & 0x0F) | ((rope_mode & 0x0F) << 4);
  P.meta = to_meta(batch);
  P.neon_arith = (batch->options & ZTCP_OPT_NEON_ARITH) != 0;
  P.mul = ztcp::PackMul{16u, 256u, 65536u};
  key_words(keys, P.key);
  P.tile_vecs = ztcp::pick_tile_vecs(vecs, ztcp::stage_bytes_per_vec(P.L));
  P.n_tiles = (int32_t)((vecs + P.tile_vecs - 1) / P.tile_vecs);
  P.n_pages = batch->n_pages;
  P.stage_bytes = ztcp::plan_stage(P.L, P.tile_vecs, P.stage_q, P.stage_s);
  ztcp::build_tile_plan(P.L, P.tile_vecs, P.stage_q, P.stage_s,
                        (reinterpret_cast<uintptr_t>(P.out) | (uintptr_t)P.blob_stride) % 16 == 0, &P.plan);
  for (int i = 0; i < 3; ++i) {
    const int64_t groups = i < P.L.n ? P.L.sec[i].dim / ztcp::kGroup : 0;
    P.gshift[i] = groups > 0 ? ztcp::log2_or_minus1(groups) : -1;
  }
  if (P.stage_bytes > kMaxStageBytes) return fail(ZTCP_EINVAL, "head_dim too large for one tile");
  if (P.n_pages * P.n_tiles > 0x7FFFFFFFLL) return fail(ZTCP_EINVAL, "batch too large for one launch");
  P.sec_lo = 0;
  P.sec_hi = P.L.n;
  P.tile_lo = 0;
  P.tiles = P.n_tiles;
  P.write_header = 1;

  ztcp::MacParams M;
  memset(&M, 0, sizeof(M));
  M.blobs = out_blobs;
  M.blob_stride = P.blob_stride;
  M.payload_len = expected_payload_bytes;
  M.n_pages = batch->n_pages;
  M.mk0 = keys->mac[0];
  M.mk1 = keys->mac[1];
  M.meta = P.meta;
  M.flags = P.flags;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool bf16 = kv_dtype == ZTCP_DTYPE_BF16;
  if (P.n_pages >= kWireOrderMinPages) {
    rc = encode_wire_order(P, M, bf16, s);
    if (rc != kNotWireOrder) return rc;
  }
  ztcp::launch_egress(P, bf16, s);
  if ((rc = launch_status("egress_tile_kernel")) != ZTCP_OK) return rc;
  ztcp::take_phase_mark(s);
  ztcp::launch_mac(M, false, s);
  return launch_status("mac_kernel<sign>");
}

}  // extern "C"

namespace {

// Shared argument checks and verify-pass parameters of ztcp_verify_pages / ztcp_decode_pages.
int32_t prepare_verify(const uint8_t* blobs, int64_t blob_bytes, const ztcp_geometry* geom,
                       const ztcp_page_batch* batch, const ztcp_keys* keys, int32_t* status, int32_t* any_fail,
                       ztcp::MacParams* M) {
  int32_t rc = check_geometry(geom, "Invalid out_k_pages dimensions");
  if (rc != ZTCP_OK) return rc;
  if ((rc = check_batch(batch)) != ZTCP_OK) return rc;
  if (!keys) return fail(ZTCP_EINVAL, "keys must not be NULL");
  if (!blobs || !status || !any_fail) return fail(ZTCP_EINVAL, "cold_blobs, status and any_fail must not be NULL");
  if (blob_bytes <= ztcp::kHeaderBytes + ztcp::kTagBytes) return fail(ZTCP_EINVAL, "cold_blob too small");
  memset(M, 0, sizeof(*M));
  M->blobs = const_cast<uint8_t*>(blobs);
  M->blob_stride = blob_bytes;
  M->payload_len = blob_bytes - ztcp::kHeaderBytes - ztcp::kTagBytes;
  M->n_pages = batch->n_pages;
  M->mk0 = keys->mac[0];
  M->mk1 = keys->mac[1];
  M->meta = to_meta(batch);
  M->vecs = geom->num_tokens * geom->num_heads;
  M->head_dim = geom->head_dim;
  M->rope_dim = geom->rope_dim;
  M->has_v = geom->is_mla_single_buffer == 0;
  M->status = status;
  M->any_fail = any_fail;
  return ZTCP_OK;
}

int32_t launch_verify(const ztcp::MacParams& M, cudaStream_t s) {
  if (cudaMemsetAsync(M.any_fail, 0, sizeof(int32_t), s) != cudaSuccess) return launch_status("memset any_fail");
  ztcp::launch_mac(M, true, s);
  return launch_status("mac_kernel<verify>");
}

}  // namespace

extern "C" {

int32_t ztcp_verify_pages(const uint8_t* blobs, int64_t blob_bytes, const ztcp_geometry* geom,
                          const ztcp_page_batch* batch, const ztcp_keys* keys, int32_t* status, int32_t* any_fail,
                          void* stream) {
  ztcp::MacParams M;
  const int32_t rc = prepare_verify(blobs, blob_bytes, geom, batch, keys, status, any_fail, &M);
  if (rc != ZTCP_OK) return rc;
  return launch_verify(M, static_cast<cudaStream_t>(stream));
}

int32_t ztcp_decode_pages(const uint8_t* blobs, int64_t blob_bytes, const ztcp_geometry* geom,
                          const ztcp_page_batch* batch, const ztcp_keys* keys, uint16_t* out_k, uint16_t* out_v,
                          int32_t* status, int32_t* any_fail, void* stream) {
  ztcp::MacParams M;
  int32_t rc = prepare_verify(blobs, blob_bytes, geom, batch, keys, status, any_fail, &M);
  if (rc != ZTCP_OK) return rc;
  if (!out_k) return fail(ZTCP_EINVAL, "out_k_pages must not be NULL");
  const bool has_v = geom->is_mla_single_buffer == 0;
  if (has_v && !out_v) return fail(ZTCP_EINVAL, "out_v_pages is required for non-MLA geometry");
  if (!has_v && out_v) return fail(ZTCP_EINVAL, "out_v_pages must be NULL for a single-buffer MLA geometry");
  if (!aligned16(out_k) || (out_v && !aligned16(out_v)))
    return fail(ZTCP_EINVAL, "out_k_pages / out_v_pages must be 16-byte aligned");
  const int64_t vecs = geom->num_tokens * geom->num_heads;

  ztcp::IngressParams P;
  memset(&P, 0, sizeof(P));
  P.blobs = blobs;
  P.blob_stride = blob_bytes;
  P.payload_len = M.payload_len;
  P.k_out = out_k;
  P.v_out = out_v;
  P.page_elems = vecs * geom->head_dim;
  P.vecs = vecs;
  P.head_dim = (int32_t)geom->head_dim;
  P.rope_dim = (int32_t)geom->rope_dim;
  P.has_v = has_v;
  P.meta = to_meta(batch);
  key_words(keys, P.key);
  P.any_fail = any_fail;
  P.status = status;
  P.page_fallback = (batch->options & ZTCP_OPT_PAGE_FALLBACK) != 0;
  const int64_t worst = ztcp::worst_stage_bytes_per_vec(geom->head_dim, geom->rope_dim, has_v);
  P.tile_vecs = ztcp::pick_tile_vecs(vecs, worst);
  P.n_tiles = (int32_t)((vecs + P.tile_vecs - 1) / P.tile_vecs);
  P.n_pages = batch->n_pages;
  // worst case over every (preset, rope_mode) a header may carry, plus 16-byte rounding per area
  if (P.tile_vecs * worst + 6 * 16 > kMaxStageBytes) return fail(ZTCP_EINVAL, "head_dim too large for one tile");
  P.stage_bytes = (int32_t)(P.tile_vecs * worst + 6 * 16);
  // layouts and staging plans of every flags byte a verified header may carry
  for (int p = 1; p <= 3; ++p)
    for (int r = 0; r <= 2; ++r) {
      const int i = (p - 1) * 3 + r;
      ztcp::build_layout(p, r, vecs, geom->head_dim, geom->rope_dim, has_v, &P.lay[i]);
      ztcp::plan_stage(P.lay[i], P.tile_vecs, P.lay_q[i], P.lay_s[i]);
      ztcp::build_tile_plan(P.lay[i], P.tile_vecs, P.lay_q[i], P.lay_s[i],
                            (reinterpret_cast<uintptr_t>(P.blobs) | (uintptr_t)P.blob_stride) % 16 == 0, &P.plan[i]);
    }
  if (P.n_pages * P.n_tiles > 0x7FFFFFFFLL) return fail(ZTCP_EINVAL, "batch too large for one launch");

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((rc = launch_verify(M, s)) != ZTCP_OK) return rc;
  ztcp::take_phase_mark(s);
  ztcp::launch_ingress(P, s);
  return launch_status("ingress_tile_kernel");
}

int32_t ztcp_chacha20_xor(const uint8_t* src, uint8_t* dst, int64_t len, const uint8_t key32[32], uint32_t counter,
                          const uint8_t nonce12[12], void* stream) {
  if (len < 0) return fail(ZTCP_EINVAL, "len must be non-negative");
  if (!key32 || !nonce12) return fail(ZTCP_EINVAL, "key_u8 must be 32-byte and nonce_u8 12-byte");
  if (len == 0) return ZTCP_OK;
  if (!src || !dst) return fail(ZTCP_EINVAL, "data must not be NULL");
  uint32_t key[8], nonce[3];
  memcpy(key, key32, 32);
  memcpy(nonce, nonce12, 12);
  ztcp::launch_chacha20_xor(src, dst, len, key, counter, nonce, static_cast<cudaStream_t>(stream));
  return launch_status("chacha20_xor_kernel");
}

int32_t ztcp_siphash24_128(const uint8_t* src, int64_t len, uint64_t mk0, uint64_t mk1, uint8_t* out16,
                           void* stream) {
  if (len < 0) return fail(ZTCP_EINVAL, "len must be non-negative");
  if (!out16 || (len > 0 && !src)) return fail(ZTCP_EINVAL, "data and out must not be NULL");
  ztcp::launch_siphash(src, len, mk0, mk1, out16, static_cast<cudaStream_t>(stream));
  return launch_status("siphash_kernel");
}

int32_t ztcp_gather(uint8_t* dst, int32_t dst_device, const uint8_t* const* srcs, const int32_t* src_devices,
                    const int64_t* bytes, int32_t n, void* stream) {
  if (n < 0 || (n > 0 && (!dst || !srcs || !src_devices || !bytes))) return fail(ZTCP_EINVAL, "gather arguments must not be NULL");
  int64_t off = 0;
  for (int32_t i = 0; i < n; ++i) {
    if (bytes[i] < 0 || (bytes[i] > 0 && !srcs[i])) return fail(ZTCP_EINVAL, "gather part sizes must be non-negative");
    if (bytes[i] == 0) continue;
    const cudaError_t e = cudaMemcpyPeerAsync(dst + off, dst_device, srcs[i], src_devices[i], (size_t)bytes[i],
                                              static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return fail(ZTCP_ECUDA, std::string("cudaMemcpyPeerAsync: ") + cudaGetErrorString(e));
    off += bytes[i];
  }
  return ZTCP_OK;
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------
// Decode for callers that cannot allocate device memory (no counterpart in the reference)
// ------------------------------------------------------------------------------------------------
// ztcp_decode_pages takes from its caller the per-page status array through which the tag-check kernel
// tells the decrypt kernel which pages failed.  ztcp_decode_pages_noalloc keeps that array here instead:
// one per GPU, ZTCP_NOALLOC_MAX_PAGES entries (256 KiB), resident on every GPU that loads this library
// until the process exits.  Host code may not use the array's name as a device address; its address on
// each device is looked up once, with that device current, and handed to the unchanged decode path.  The
// address is cached for the life of the process: after a cudaDeviceReset the module (and this array) could
// be loaded elsewhere, so a reset after the first call on a device is documented as unsupported.
static __device__ __align__(256) int32_t g_noalloc_status[ZTCP_NOALLOC_MAX_PAGES];

namespace {

constexpr int kNoallocDevices = 64;
std::mutex g_noalloc_mu;
int32_t* g_noalloc_addr[kNoallocDevices];  // g_noalloc_status on device i, once looked up

int32_t noalloc_status_array(int32_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(ZTCP_ECUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (dev >= 0 && dev < kNoallocDevices && g_noalloc_addr[dev]) {
    *out = g_noalloc_addr[dev];
    return ZTCP_OK;
  }
  int32_t* ptr = nullptr;
  e = cudaGetSymbolAddress((void**)&ptr, g_noalloc_status);
  if (e != cudaSuccess || ptr == nullptr)
    return fail(ZTCP_ECUDA, std::string("cudaGetSymbolAddress of the no-allocation status array: ") +
                                cudaGetErrorString(e));
  if (dev >= 0 && dev < kNoallocDevices) g_noalloc_addr[dev] = ptr;
  *out = ptr;
  return ZTCP_OK;
}

}  // namespace

extern "C" {

int32_t ztcp_decode_pages_noalloc(const uint8_t* blobs, int64_t blob_bytes, const ztcp_geometry* geom,
                                  const ztcp_page_batch* batch, const ztcp_keys* keys, uint16_t* out_k,
                                  uint16_t* out_v, int32_t* any_fail, void* stream) {
  if (!batch) return fail(ZTCP_EINVAL, "page batch must not be NULL");
  if (batch->n_pages > ZTCP_NOALLOC_MAX_PAGES)
    return fail(ZTCP_EINVAL, "batch of " + std::to_string(batch->n_pages) +
                                 " pages exceeds the no-allocation decode's limit of " +
                                 std::to_string(ZTCP_NOALLOC_MAX_PAGES) + " pages per call");
  if (!any_fail) return fail(ZTCP_EINVAL, "any_fail must not be NULL");
  int32_t* status = nullptr;
  const int32_t rc = noalloc_status_array(&status);
  if (rc != ZTCP_OK) return rc;
  // every page's status is written by the tag check before the decrypt pass reads it, and any_fail is
  // zeroed by the decode itself, so nothing left over from an earlier call is read
  return ztcp_decode_pages(blobs, blob_bytes, geom, batch, keys, out_k, out_v, status, any_fail, stream);
}

}  // extern "C"

