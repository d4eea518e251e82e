/* ztcp_ledger.h -- host-side nonce and freshness ledger of the ZTCP session keyring, C ABI.
 *
 * The reference keeps, per (tenant, session), a set of burned 96-bit ChaCha20 nonces, a freshness
 * watermark per KV slot (model_id_hash, layer_id, head_group_id, page_token_hash) and the session's
 * largest sequence nonce, and walks them page by page in Python
 * (research/baseline_codec/fused_quant_crypto.py: preflight_validate_egress :263-342, commit_egress
 * :397-434, verify_and_update_freshness :458-541, verify_and_update_freshness_batch :543-603,
 * next_sequence_nonce :248-261).  This ledger holds the same tables in C++ and applies each batch
 * operation all-or-nothing, with the reference's check order, so the caller can raise the reference's
 * exceptions from the returned error record.  Key material, generations and crypto-shredding stay with
 * the caller (they are per call, not per page).
 *
 * Sessions are named by a caller-chosen 64-bit id.  All functions are thread-safe (one mutex per
 * ledger) and never throw; they return ZTCP_LEDGER_OK or a negative ZTCP_LEDGER_E* code.
 */
#ifndef ZTCP_LEDGER_H
#define ZTCP_LEDGER_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ZTCP_LEDGER_OK 0
#define ZTCP_LEDGER_ESTALE (-1)       /* sequence nonce older than the slot's watermark or the minimum */
#define ZTCP_LEDGER_EREUSE (-2)       /* 96-bit nonce already burned under the session */
#define ZTCP_LEDGER_ENOSESSION (-3)   /* session id not open */
#define ZTCP_LEDGER_EINVAL (-4)       /* NULL pointer or empty batch */
#define ZTCP_LEDGER_EMISMATCH (-5)    /* sequence nonce differs from the expected one */

/* What failed and on which page: `seq` the page's sequence nonce, `ref` the watermark or minimum it is
 * below (ESTALE) or the expected value (EMISMATCH), `loc` the nonce's layer_id << 16 | head_group_id
 * word (EREUSE), `index` the page within the batch, `kind` for ESTALE: 0 = slot watermark, 1 = minimum. */
typedef struct ztcp_ledger_error {
  int32_t code;
  int32_t kind;
  int64_t index;
  uint64_t seq;
  uint64_t ref;
  uint32_t loc;
  uint32_t reserved;
} ztcp_ledger_error;

/* One decoded page header's freshness fields. */
typedef struct ztcp_fresh_record {
  uint32_t model_id_hash;
  uint16_t layer_id;
  uint16_t head_group_id;
  uint64_t page_token_hash;
  uint64_t sequence_nonce;
} ztcp_fresh_record;

typedef struct ztcp_ledger ztcp_ledger;
typedef struct ztcp_reservation ztcp_reservation;

ztcp_ledger* ztcp_ledger_create(void);
void ztcp_ledger_destroy(ztcp_ledger* ledger);

/* Open empty tables for `session` (replacing any it had; the keyring's derive_or_get :202-246). */
int32_t ztcp_ledger_open(ztcp_ledger* ledger, uint64_t session);
/* Drop the session's tables (crypto-shred, _zeroize_and_remove_session :605-635).  Returns 1 when the
 * session was open, 0 otherwise. */
int32_t ztcp_ledger_close(ztcp_ledger* ledger, uint64_t session);
int32_t ztcp_ledger_is_open(const ztcp_ledger* ledger, uint64_t session);

/* next_sequence_nonce (:248-261): base = max + 1, max = base + count - 1.  The reference does this on
 * unbounded Python integers, so past 2^64 - 1 it hands out 2^64, 2^64 + 1, ...; the ledger keeps the
 * session maximum as a 128-bit value to give the same answers (base = *base_hi << 64 | *base_lo). */
int32_t ztcp_ledger_next_nonce(ztcp_ledger* ledger, uint64_t session, uint64_t count, uint64_t* base_lo,
                               uint64_t* base_hi);
int32_t ztcp_ledger_max_nonce(const ztcp_ledger* ledger, uint64_t session, uint64_t* max_lo, uint64_t* max_hi);

/* preflight_validate_egress (:263-342) for pages i = 0..n-1 with sequence nonce base + i: every page
 * must be no older than its slot's watermark (or an earlier page of the batch in the same slot) and
 * carry an unburned nonce.  On success the batch's nonces are burned, the session maximum is raised to
 * the last page's nonce and *out holds the staged slot watermarks for ztcp_ledger_commit; on failure
 * nothing changes and *err says why. */
int32_t ztcp_ledger_preflight(ztcp_ledger* ledger, uint64_t session, uint32_t model_id_hash, uint16_t layer_id,
                              uint16_t head_group_id, uint64_t base_sequence_nonce, const uint64_t* token_hashes,
                              int64_t n, ztcp_reservation** out, ztcp_ledger_error* err);
uint64_t ztcp_reservation_last_seq(const ztcp_reservation* r);
int64_t ztcp_reservation_pages(const ztcp_reservation* r);
/* commit_egress (:397-434): raise each staged slot's watermark (never lower it) and the session maximum. */
int32_t ztcp_ledger_commit(ztcp_ledger* ledger, uint64_t session, const ztcp_reservation* r);
void ztcp_reservation_free(ztcp_reservation* r);

/* verify_and_update_freshness_batch (:543-603): every record must be >= the minimum (when has_min) and
 * >= its slot's watermark (as updated by earlier records of the batch); on success raise the watermarks
 * and the session maximum, on failure change nothing. */
int32_t ztcp_ledger_freshness_batch(ztcp_ledger* ledger, uint64_t session, const ztcp_fresh_record* records,
                                    int64_t n, int32_t has_min, uint64_t min_sequence_nonce, ztcp_ledger_error* err);
/* verify_and_update_freshness (:458-541), one page: the expected nonce (when has_expected) is checked
 * first, then the minimum, then the slot watermark. */
int32_t ztcp_ledger_freshness_one(ztcp_ledger* ledger, uint64_t session, const ztcp_fresh_record* record,
                                  int32_t has_min, uint64_t min_sequence_nonce, int32_t has_expected,
                                  uint64_t expected_sequence_nonce, ztcp_ledger_error* err);

/* Freshness records of n blobs from their 32-byte headers (cold_page_spec.py:117-161 field order);
 * blob i starts at blobs + i * stride.  The batch decode wrapper parses these per page in Python
 * (native_fused_codec.py:335-343, :424-430). */
int32_t ztcp_ledger_parse_headers(const uint8_t* blobs, int64_t stride, int64_t n, ztcp_fresh_record* out);

#ifdef __cplusplus
}
#endif

#endif /* ZTCP_LEDGER_H */
