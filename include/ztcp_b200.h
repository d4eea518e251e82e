/*
 * ztcp_b200.h -- C-ABI of the B200 (sm_100a) ZTCP cold-page codec.
 *
 * Drop-in boundary: these entry points replace the reference's native codec module
 * (research/baseline_codec/csrc/fused_cold_page_cpu.cpp, bound by pybind at :2540-2683 and loaded
 * into NativeCppFusedColdPageCodec._ext by research/baseline_codec/native_fused_codec.py:43-78).
 * The reference's eight module functions map onto them as:
 *
 *   fused_encode_cold_pages_peak_into_cpu (csrc:1904-2004)  -> ztcp_encode_pages
 *   fused_encode_cold_pages_batch_cpu     (csrc:1775-1902)  -> ztcp_encode_pages (caller allocates)
 *   fused_encode_cold_page_cpu            (csrc:1478-1555)  -> ztcp_encode_pages with n_pages = 1
 *   fused_decode_cold_pages_peak_into_cpu (csrc:2250-2496)  -> ztcp_decode_pages
 *   fused_decode_cold_pages_batch_cpu     (csrc:2006-2248)  -> ztcp_decode_pages (caller allocates)
 *   fused_decode_cold_page_cpu            (csrc:1557-1773)  -> ztcp_decode_pages with n_pages = 1
 *   chacha20_rfc8439_xor_cpu              (csrc:2499-2523)  -> ztcp_chacha20_xor
 *   siphash24_128_cpu                     (csrc:2525-2538)  -> ztcp_siphash24_128
 *
 * Conventions.  Every pointer named "device" is CUDA device memory on the current device; every
 * call only enqueues work on `stream` (a cudaStream_t; NULL = the legacy default stream) and returns
 * ZTCP_OK, or a negative code with a message from ztcp_last_error() when an argument is invalid or a
 * launch fails.  No call allocates memory or synchronizes.  Validation messages repeat the
 * reference's TORCH_CHECK texts.  Wire bytes equal the reference codec's x86 build.
 */
#ifndef ZTCP_B200_H
#define ZTCP_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ZTCP_OK 0
#define ZTCP_EINVAL (-1)  /* invalid argument (message in ztcp_last_error) */
#define ZTCP_ECUDA (-2)   /* CUDA launch error (message in ztcp_last_error) */

#define ZTCP_DTYPE_F16 0
#define ZTCP_DTYPE_BF16 1

/* Per-page decode status, in the reference's check order (csrc:2309-2355).  The reference reports
 * 4 and 5 as its status 1 ("Invalid cold-page header magic, version, or flags"). */
#define ZTCP_PAGE_OK 0
#define ZTCP_PAGE_BAD_MAGIC 1      /* magic or version */
#define ZTCP_PAGE_AAD_MISMATCH 2   /* tenant / model / layer / token hash differ from the expected AAD */
#define ZTCP_PAGE_MAC_FAILED 3     /* SipHash-2-4-128 tag mismatch */
#define ZTCP_PAGE_BAD_FLAGS 4      /* preset or rope_mode out of range */
#define ZTCP_PAGE_TRUNCATED 5      /* payload shorter than the flags require */
#define ZTCP_PAGE_BAD_BLOCK 6      /* kv_block[i] outside [0, kv_pool_pages): the page is neither read nor written
                                      (an extension: the reference's batch calls take contiguous pages) */

/* KV page geometry: a page is num_tokens x num_heads x head_dim elements per buffer. */
typedef struct ztcp_geometry {
  int64_t num_tokens;
  int64_t num_heads;
  int64_t head_dim;            /* multiple of 16 */
  int64_t rope_dim;            /* leading RoPE columns of K, multiple of 16, <= head_dim */
  int32_t is_mla_single_buffer; /* decode: no V buffer (encode infers this from v_pages == NULL) */
  int32_t reserved;
} ztcp_geometry;

/* Session keys: 256-bit ChaCha20 key as four little-endian u64 limbs (k0..k3) and the 128-bit
 * SipHash key (mk0, mk1) -- the reference's (k0, k1, k2, k3, mk0, mk1) arguments. */
typedef struct ztcp_keys {
  uint64_t enc[4];
  uint64_t mac[2];
} ztcp_keys;

/* One batch of pages and its AAD.  Page i of the batch:
 *   KV block     kv_block[i]        (device int32; NULL = i)          -- block-table addressing
 *   token hash   token_hash[i]      (device uint64; required)
 *   seq nonce    sequence_nonce[i]  (device uint64; NULL = base_sequence_nonce + i, csrc:1994)
 *   layer id     layer_id[i]        (device uint16; NULL = layer_id_uniform)
 * tenant / model hash and head group are shared by the batch.  For decode these are the EXPECTED
 * values the header must carry.
 * kv_pool_pages: pages in the KV pool(s) the batch addresses.  Required (> 0) with a block table: the
 * kernels check every kv_block entry against it before any access, on the device.  A page whose entry
 * lies outside [0, kv_pool_pages) is never read or written in the pool: encode writes that page's blob
 * as all-zero bytes (magic 0, which every decode rejects), decode reports ZTCP_PAGE_BAD_BLOCK for it
 * and sets *any_fail.  Without a block table, 0 means "not given"; a positive value must be >= n_pages.
 * options: ZTCP_OPT_* bits (0 = the reference's scalar x86-64 arithmetic, bit-exact with its build). */
#define ZTCP_OPT_NEON_ARITH 1 /* egress: quantize with the reference's ARM NEON fp16 arithmetic (its build with
                                 __ARM_FEATURE_FP16_VECTOR_ARITHMETIC, csrc:718-733 / :786-803); decode ignores it */
#define ZTCP_OPT_PAGE_FALLBACK 2 /* decode: zero only the pages that fail (status != 0) and decode the others,
                                    for a caller that recomputes failed pages instead of dropping the batch
                                    (the per-page fallback of the reference's design, paper main.tex:174);
                                    without it any failing page zeroes every output page, as the reference's
                                    decoders do (csrc:2481-2495).  any_fail is set either way; egress ignores it */
typedef struct ztcp_page_batch {
  int64_t n_pages;
  const int32_t* kv_block;
  const uint64_t* token_hash;
  const uint64_t* sequence_nonce;
  const uint16_t* layer_id;
  uint64_t base_sequence_nonce;
  uint32_t tenant_id_hash;
  uint32_t model_id_hash;
  uint16_t layer_id_uniform;
  uint16_t head_group_id;
  int32_t options;
  int64_t kv_pool_pages;
} ztcp_page_batch;

/* Message of the last failed call on this thread ("" when none). */
const char* ztcp_last_error(void);

/* Library version, major * 10000 + minor * 100 + patch. */
int32_t ztcp_version(void);

/* Minimum payload bytes for (preset, rope_mode) and geometry -- required_payload_bytes_for_flags
 * (csrc:1439-1474).  Returns -1 for an invalid preset / rope_mode. */
int64_t ztcp_min_payload_bytes(int32_t preset, int32_t rope_mode, const ztcp_geometry* geom, int32_t has_v);

/* Payload bytes of the reference's Python spec (cold_page_spec.py:203-246): the minimum rounded up
 * to a multiple of 4.  A blob is 32 + payload + 16 bytes. */
int64_t ztcp_spec_payload_bytes(int32_t preset, int32_t rope_mode, const ztcp_geometry* geom, int32_t has_v);

/* Egress.  Quantizes, packs, encrypts (ChaCha20, counter from 1, nonce [seq lo, seq hi,
 * layer << 16 | head_group]) and tags (SipHash-2-4-128 over header || ciphertext) every page of
 * `batch` into out_blobs (device, [n_pages, 32 + expected_payload_bytes + 16], dense).
 *   k_pages, v_pages: device KV pools (fp16 or bf16 per kv_dtype; bf16 is rounded to fp16 with
 *   round-to-nearest-even first), page b at base + kv_block[b] * num_tokens*num_heads*head_dim
 *   elements; 16-byte aligned.  v_pages = NULL encodes a single-buffer (MLA) page.
 * Replaces fused_encode_cold_pages_peak_into_cpu (csrc:1904-2004) and, with n_pages = 1,
 * fused_encode_cold_page_cpu (csrc:1478-1555). */
int32_t ztcp_encode_pages(const void* k_pages, const void* v_pages, int32_t kv_dtype, const ztcp_geometry* geom,
                          const ztcp_page_batch* batch, int32_t preset, int32_t rope_mode,
                          int64_t expected_payload_bytes, const ztcp_keys* keys, uint8_t* out_blobs, void* stream);

/* Ingress.  For every blob (device, [n_pages, blob_bytes], dense): checks magic/version, the AAD
 * against `batch`, the SipHash tag, then flags and length; writes status[i] (device int32,
 * ZTCP_PAGE_*) and sets *any_fail (device int32, zeroed by this call) when any page fails.  Only
 * then decrypts and dequantizes into out_k / out_v (device fp16, page i at kv_block[i]); when any
 * page of the batch failed, every output page of the batch is zeroed instead (csrc:2481-2495) -- or,
 * with ZTCP_OPT_PAGE_FALLBACK in batch->options, only the failed pages.
 * out_v must be NULL for a single-buffer MLA geometry and non-NULL otherwise.
 * Replaces fused_decode_cold_pages_peak_into_cpu (csrc:2250-2496) and, with n_pages = 1,
 * fused_decode_cold_page_cpu (csrc:1557-1773). */
int32_t ztcp_decode_pages(const uint8_t* blobs, int64_t blob_bytes, const ztcp_geometry* geom,
                          const ztcp_page_batch* batch, const ztcp_keys* keys, uint16_t* out_k, uint16_t* out_v,
                          int32_t* status, int32_t* any_fail, void* stream);

/* Integrity check only: the checks of ztcp_decode_pages (magic/version, AAD, SipHash tag, flags,
 * length) without decrypting -- status[i] and *any_fail as ztcp_decode_pages writes them.  Replaces
 * the verification steps of the reference's decoders (csrc:2312-2355) for scrubbing stored blobs. */
int32_t ztcp_verify_pages(const uint8_t* blobs, int64_t blob_bytes, const ztcp_geometry* geom,
                          const ztcp_page_batch* batch, const ztcp_keys* keys, int32_t* status, int32_t* any_fail,
                          void* stream);

/* RFC 8439 ChaCha20 keystream XOR of `len` device bytes (src may equal dst).  key32 and nonce12 are
 * host arrays.  Replaces chacha20_rfc8439_xor_cpu (csrc:2499-2523). */
int32_t ztcp_chacha20_xor(const uint8_t* src, uint8_t* dst, int64_t len, const uint8_t key32[32], uint32_t counter,
                          const uint8_t nonce12[12], void* stream);

/* SipHash-2-4 with 128-bit output of `len` device bytes into out16 (device).  Replaces
 * siphash24_128_cpu (csrc:2525-2538). */
int32_t ztcp_siphash24_128(const uint8_t* src, int64_t len, uint64_t mk0, uint64_t mk1, uint8_t* out16,
                           void* stream);

/* Peer gather of blobs encoded on several GPUs into one buffer on `dst_device` (the offload path's
 * "one sender" step; the reference has no GPU, this has no reference counterpart): part i
 * (`bytes[i]` bytes at `srcs[i]` on `src_devices[i]`) lands at dst + bytes[0] + ... + bytes[i-1].  One
 * cudaMemcpyPeerAsync per part, enqueued on `stream` (a stream of dst_device): copy-engine transfers,
 * no kernel reads another GPU's memory. */
int32_t ztcp_gather(uint8_t* dst, int32_t dst_device, const uint8_t* const* srcs, const int32_t* src_devices,
                    const int64_t* bytes, int32_t n, void* stream);

/* Largest batch ztcp_decode_pages_noalloc takes in one call. */
#define ZTCP_NOALLOC_MAX_PAGES 65536

/* Ingress that needs no device memory from the caller beyond its inputs, its K/V outputs and a one-word
 * any_fail flag -- an addition of this library with no counterpart in the reference.  ztcp_decode_pages
 * asks for a per-page status array (the tag check's verdicts, read by the decrypt pass); this variant
 * keeps those verdicts in a buffer inside the library, so it suits callers that cannot call cudaMalloc on
 * the decode path: a serving engine that hands all device memory to its KV pool at start-up and allows no
 * allocation while requests run (one could fail or stall on a full device), or a plugin loaded into such
 * an engine that only sees the engine's buffers.  Otherwise it behaves as ztcp_decode_pages: same checks,
 * same outputs, *any_fail (device int32) zeroed by the call and set when a page fails, every output page
 * zeroed then (only the failed ones with ZTCP_OPT_PAGE_FALLBACK); per-page statuses are not returned.
 * Limits: at most ZTCP_NOALLOC_MAX_PAGES pages per call (larger batches return ZTCP_EINVAL; split them);
 * the buffer (ZTCP_NOALLOC_MAX_PAGES x 4 bytes = 256 KiB) stays on every GPU that loads the library
 * until the process exits.  All calls on a device share that one buffer and each overwrites it, so calls
 * that overlap on the GPU (streams not ordered against each other) race and can decode or zero the wrong
 * pages: issue them on one stream or order them with events.  The first call on each device looks up the
 * buffer's address there (a one-time set-up, done with that device current); make that first call before
 * any stream capture.  The address is kept for the life of the process, so resetting a device
 * (cudaDeviceReset) after its first call is not supported: the library's device memory may move. */
int32_t ztcp_decode_pages_noalloc(const uint8_t* blobs, int64_t blob_bytes, const ztcp_geometry* geom,
                                  const ztcp_page_batch* batch, const ztcp_keys* keys, uint16_t* out_k,
                                  uint16_t* out_v, int32_t* any_fail, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ZTCP_B200_H */
