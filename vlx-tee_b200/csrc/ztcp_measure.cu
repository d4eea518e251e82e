// ztcp_measure.cu -- measurement entry points (include/ztcp_measure.h): integer ceilings of the codec's
// primitives on the current GPU, and the one-shot phase mark the codec calls record between their kernels.
//
// The calibration kernels call the same device functions as the codec kernels (ztcp_device.cuh):
//  * chacha20_block with every SM full of threads and no memory traffic -> keystream blocks per second,
//    the integer-ALU ceiling of the tile kernels' keystream work;
//  * SipState::absorb_pre over words generated in registers, one warp of 32 chains per SM sub-partition
//    (the tag kernels' shape) -> words per second over the GPU and cycles per word of one chain, the
//    latency floor of a page's tag.
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/ztcp_b200.h"
#include "../../include/ztcp_measure.h"
#include "ztcp_device.cuh"
#include "ztcp_kernels.cuh"

namespace ztcp {

namespace {

thread_local cudaEvent_t g_phase_event = nullptr;

constexpr int kPeakChachaThreads = 256;
constexpr int kPeakChachaCtasPerSm = 8;
constexpr int kPeakChachaBlocksPerThread = 64;
constexpr int kPeakSipThreads = 128;     // one warp per SM sub-partition
constexpr int kPeakSipWords = 12293;     // one cfg0 page: header + payload + length word

__global__ void __launch_bounds__(kPeakChachaThreads) peak_chacha_kernel(uint32_t* out, uint32_t seed) {
  const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t key[8] = {seed, seed + 1u, seed + 2u, seed + 3u, seed + 4u, seed + 5u, seed + 6u, seed + 7u};
  uint32_t acc = 0;
  for (int i = 0; i < kPeakChachaBlocksPerThread; ++i) {
    uint32_t ks[16];
    chacha20_block(key, t * kPeakChachaBlocksPerThread + i, seed, ~seed, t, ks);
#pragma unroll
    for (int w = 0; w < 16; ++w) acc ^= ks[w];
  }
  out[t] = acc;
}

__global__ void __launch_bounds__(kPeakSipThreads) peak_sip_kernel(uint64_t* out, long long* cycles) {
  const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
  SipState st;
  st.init(0x0706050403020100ull ^ t, 0x0f0e0d0c0b0a0908ull);
  W64 m{t, 0x9e3779b9u};
  st.v3 = xor64(st.v3, m);
  const long long c0 = clock64();
  for (int i = 0; i < kPeakSipWords; ++i) {
    const W64 next{m.lo + 0x9e3779b9u, m.hi ^ (uint32_t)i};
    st.absorb_pre(m, next);
    m = next;
  }
  const long long c1 = clock64();
  out[t] = u64(st.v0) ^ u64(st.v1) ^ u64(st.v2) ^ u64(st.v3);
  cycles[t] = c1 - c0;
}

}  // namespace

// Records the armed phase event (if any) on `stream` and disarms it; called by the codec entry points
// between their two kernels.
void take_phase_mark(cudaStream_t stream) {
  if (g_phase_event != nullptr) {
    cudaEventRecord(g_phase_event, stream);
    g_phase_event = nullptr;
  }
}

}  // namespace ztcp

namespace {

int32_t measure_fail(const std::string& what, cudaError_t e) {
  return ztcp::set_last_error(ZTCP_ECUDA, what + ": " + cudaGetErrorString(e));
}

}  // namespace

extern "C" {

int32_t ztcp_mark_phase(void* event) {
  ztcp::g_phase_event = static_cast<cudaEvent_t>(event);
  return ZTCP_OK;
}

int32_t ztcp_measure_int_peaks(void* scratch, int64_t scratch_bytes, ztcp_int_peaks* out) {
  using ztcp::set_last_error;
  if (!scratch || !out) return set_last_error(ZTCP_EINVAL, "scratch and out must not be NULL");
  if ((reinterpret_cast<uintptr_t>(scratch) & 15) != 0)
    return set_last_error(ZTCP_EINVAL, "scratch must be 16-byte aligned");
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return measure_fail("device query", e);
  const int64_t chacha_threads = (int64_t)sms * ztcp::kPeakChachaCtasPerSm * ztcp::kPeakChachaThreads;
  const int64_t sip_threads = (int64_t)sms * ztcp::kPeakSipThreads;
  const int64_t need = chacha_threads * 4 + sip_threads * 16;
  if (scratch_bytes < need || need > ZTCP_MEASURE_SCRATCH_BYTES)
    return set_last_error(ZTCP_EINVAL, "scratch smaller than ZTCP_MEASURE_SCRATCH_BYTES");
  uint32_t* o32 = static_cast<uint32_t*>(scratch);
  uint64_t* o64 = reinterpret_cast<uint64_t*>(static_cast<uint8_t*>(scratch) + ((chacha_threads * 4 + 15) / 16) * 16);
  long long* cyc = reinterpret_cast<long long*>(o64 + sip_threads);

  cudaStream_t s = nullptr;
  cudaEvent_t a = nullptr, b = nullptr;
  if ((e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking)) != cudaSuccess) return measure_fail("stream", e);
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  float chacha_ms = 0.f, sip_ms = 0.f;
  long long c0 = 0;
  const unsigned chacha_grid = (unsigned)(sms * ztcp::kPeakChachaCtasPerSm);
  // one untimed launch each (module load, clocks up), then timed repetitions
  ztcp::peak_chacha_kernel<<<chacha_grid, ztcp::kPeakChachaThreads, 0, s>>>(o32, 0x12345u);
  ztcp::peak_sip_kernel<<<(unsigned)sms, ztcp::kPeakSipThreads, 0, s>>>(o64, cyc);
  constexpr int kReps = 3;
  cudaEventRecord(a, s);
  for (int r = 0; r < kReps; ++r) ztcp::peak_chacha_kernel<<<chacha_grid, ztcp::kPeakChachaThreads, 0, s>>>(o32, 0x777u + r);
  cudaEventRecord(b, s);
  e = cudaEventSynchronize(b);
  if (e == cudaSuccess) e = cudaEventElapsedTime(&chacha_ms, a, b);
  if (e == cudaSuccess) {
    cudaEventRecord(a, s);
    for (int r = 0; r < kReps; ++r) ztcp::peak_sip_kernel<<<(unsigned)sms, ztcp::kPeakSipThreads, 0, s>>>(o64, cyc);
    cudaEventRecord(b, s);
    e = cudaEventSynchronize(b);
  }
  if (e == cudaSuccess) e = cudaEventElapsedTime(&sip_ms, a, b);
  if (e == cudaSuccess) e = cudaMemcpyAsync(&c0, cyc, sizeof(c0), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaGetLastError();
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  cudaStreamDestroy(s);
  if (e != cudaSuccess) return measure_fail("calibration kernels", e);
  chacha_ms /= kReps;
  sip_ms /= kReps;
  out->chacha20_blocks_per_s = (double)chacha_threads * ztcp::kPeakChachaBlocksPerThread / (chacha_ms * 1e-3);
  out->sip_words_per_s = (double)sip_threads * ztcp::kPeakSipWords / (sip_ms * 1e-3);
  out->sip_chain_cycles_per_word = (double)c0 / ztcp::kPeakSipWords;
  out->sip_chain_ms = sip_ms;
  out->sms = sms;
  out->reserved = 0;
  return ZTCP_OK;
}

}  // extern "C"
