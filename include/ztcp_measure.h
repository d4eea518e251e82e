/*
 * ztcp_measure.h -- measurement entry points of the B200 ZTCP codec library (libztcp_b200.so).
 *
 * Neither has a counterpart in the reference (research/baseline_codec/csrc/fused_cold_page_cpu.cpp has no
 * GPU and no roofline).  They give a benchmark the integer ceilings of the codec's own primitives on the
 * GPU at hand, and the split of one codec call's time between its two kernels, so every roofline
 * fraction it reports is measured in the same run.  Not part of the drop-in boundary.
 */
#ifndef ZTCP_MEASURE_H
#define ZTCP_MEASURE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Scratch (device bytes) ztcp_measure_int_peaks needs. */
#define ZTCP_MEASURE_SCRATCH_BYTES (8 << 20)

typedef struct ztcp_int_peaks {
  double chacha20_blocks_per_s;    /* RFC 8439 keystream blocks per second, every SM busy, no memory traffic */
  double sip_words_per_s;          /* SipHash-2-4 64-bit words per second over the GPU, one chain warp per
                                      SM sub-partition (32 independent chains each), no memory traffic */
  double sip_chain_cycles_per_word; /* SM cycles per word of one such chain: the latency floor of a page tag */
  double sip_chain_ms;             /* duration of one 12,293-word chain (one cfg0 page) at the clock seen */
  int32_t sms;                     /* streaming multiprocessors of the device */
  int32_t reserved;
} ztcp_int_peaks;

/* Runs three short calibration kernels on the current device (about 10 ms in all) with the codec's own
 * ChaCha20 block function and SipHash round (the device code of ztcp_encode_pages / ztcp_decode_pages),
 * synchronizes, and fills *out.  scratch: at least ZTCP_MEASURE_SCRATCH_BYTES of device memory, 16-byte
 * aligned (the kernels write their results there so nothing is optimized away).  Returns ZTCP_OK or a
 * negative code with ztcp_last_error() set. */
int32_t ztcp_measure_int_peaks(void* scratch, int64_t scratch_bytes, ztcp_int_peaks* out);

/* Arms a one-shot phase mark for the calling thread: the next ztcp_encode_pages, ztcp_decode_pages or
 * ztcp_decode_pages_noalloc call made on this thread records `event` (a cudaEvent_t) on its stream between
 * its two kernels -- after the egress tile kernel and before the tag chain (encode), after the tag
 * check and before the decrypt kernel (decode) -- and then disarms it.  A call that fails before
 * launching leaves it armed.  event = NULL disarms. */
int32_t ztcp_mark_phase(void* event);

#ifdef __cplusplus
}
#endif

#endif /* ZTCP_MEASURE_H */
