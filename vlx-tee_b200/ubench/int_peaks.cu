// int_peaks.cu -- integer-pipe ceilings of the ZTCP codec's primitives on one B200 (sm_100a).
//
// Measures, with the codec's own device code (csrc/ztcp_device.cuh):
//   * chacha20_blocks_per_s: ChaCha20 keystream blocks per second with every SM busy (no memory
//     traffic) -- the ALU ceiling of the egress/ingress tile kernels' keystream work;
//   * sip_chain_cycles_per_word: cycles per 64-bit word of one SipHash-2-4 chain when each SM
//     sub-partition runs one warp of 32 chains -- the latency floor of one page's tag;
//   * sip_words_per_s: SipHash words per second for 1, 2 and 4 chain warps per sub-partition;
//   * alu / fma pipe rates of the instruction classes the chains use (xor3, funnel shift, byte permute,
//     integer multiply-add), in warp instructions per cycle per SM.
// Each line printed is one JSON object.  Build and run:
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -o /tmp/int_peaks vlx-tee_b200/ubench/int_peaks.cu && /tmp/int_peaks
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

#include "../csrc/ztcp_device.cuh"

using namespace ztcp;

#define CK(x)                                                                  \
  do {                                                                         \
    cudaError_t e = (x);                                                       \
    if (e != cudaSuccess) {                                                    \
      printf("{\"error\":\"%s\",\"line\":%d}\n", cudaGetErrorString(e), __LINE__); \
      return 1;                                                                \
    }                                                                          \
  } while (0)

__global__ void chacha_kernel(uint32_t* out, int blocks_per_thread, uint32_t seed) {
  const uint32_t tid = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t key[8] = {seed, seed ^ 1u, seed ^ 2u, seed ^ 3u, seed ^ 4u, seed ^ 5u, seed ^ 6u, seed ^ 7u};
  uint32_t acc = 0;
  for (int it = 0; it < blocks_per_thread; ++it) {
    uint32_t ks[16];
    chacha20_block(key, tid * blocks_per_thread + it, seed, ~seed, tid, ks);
#pragma unroll
    for (int i = 0; i < 16; ++i) acc ^= ks[i];
  }
  out[tid] = acc;
}

// One chain per lane over `words` words generated in registers (no memory traffic).
__global__ void sip_kernel(uint64_t* out, long long* cycles, int words) {
  const uint32_t g = blockIdx.x * blockDim.x + threadIdx.x;
  SipState st;
  st.init(0x0706050403020100ull ^ g, 0x0f0e0d0c0b0a0908ull);
  W64 m{g, 0x9e3779b9u};
  st.v3 = xor64(st.v3, m);
  const long long t0 = clock64();
  for (int i = 0; i < words; ++i) {
    const W64 nx{m.lo + 0x9e3779b9u, m.hi ^ (uint32_t)i};
    st.absorb_pre(m, nx);
    m = nx;
  }
  const long long t1 = clock64();
  out[g] = u64(st.v0) ^ u64(st.v1) ^ u64(st.v2) ^ u64(st.v3);
  cycles[g] = t1 - t0;
}

__device__ __forceinline__ uint32_t lop3_xor3(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm volatile("lop3.b32 %0, %1, %2, %3, 0x96;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

template <int OP>
__global__ void op_kernel(uint32_t* out, int iters, uint32_t k) {
  uint32_t a[8], b[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) { a[j] = threadIdx.x * 7 + j; b[j] = threadIdx.x * 3 + 5 * j; }
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (OP == 0) a[j] = lop3_xor3(a[j], b[j], k);
      if (OP == 1) a[j] = __funnelshift_l(a[j], b[j], 13);
      if (OP == 2) a[j] = __byte_perm(a[j], b[j], 0x5432);
      if (OP == 3) a[j] = a[j] * k + b[j];
    }
  }
  uint32_t r = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) r ^= a[j] ^ b[j];
  out[blockIdx.x * blockDim.x + threadIdx.x] = r;
}

template <typename F>
static float time_ms(F f, int reps) {
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  f();
  cudaDeviceSynchronize();
  cudaEventRecord(a);
  for (int i = 0; i < reps; ++i) f();
  cudaEventRecord(b);
  cudaEventSynchronize(b);
  float ms;
  cudaEventElapsedTime(&ms, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  return ms / reps;
}

int main() {
  cudaDeviceProp p;
  CK(cudaGetDeviceProperties(&p, 0));
  const int sms = p.multiProcessorCount;
  int clk_khz = 0;
  cudaDeviceGetAttribute(&clk_khz, cudaDevAttrClockRate, 0);
  printf("{\"device\":\"%s\",\"sms\":%d,\"max_clock_mhz\":%.0f}\n", p.name, sms, clk_khz / 1e3);
  const int max_threads = sms * 2048;
  uint32_t* o32;
  uint64_t* o64;
  long long* cyc;
  CK(cudaMalloc(&o32, sizeof(uint32_t) * max_threads));
  CK(cudaMalloc(&o64, sizeof(uint64_t) * max_threads));
  CK(cudaMalloc(&cyc, sizeof(long long) * max_threads));

  {
    const int block = 256, grid = sms * (2048 / block), bpt = 64;
    const double blocks = (double)grid * block * bpt;
    const float ms = time_ms([&] { chacha_kernel<<<grid, block>>>(o32, bpt, 0x12345u); }, 5);
    CK(cudaGetLastError());
    printf("{\"metric\":\"chacha20_blocks_per_s\",\"value\":%.4g,\"keystream_GBps\":%.1f,\"ms\":%.4f}\n",
           blocks / (ms * 1e-3), 64.0 * blocks / (ms * 1e-3) / 1e9, ms);
  }
  {
    const int words = 12293;  // one GQA INT4_SYM+PRESERVE_FP8 page: header + payload + length word
    for (int warps_per_smsp : {1, 2, 4}) {
      const int block = 128 * warps_per_smsp;
      const float ms = time_ms([&] { sip_kernel<<<sms, block>>>(o64, cyc, words); }, 3);
      CK(cudaGetLastError());
      long long c0;
      CK(cudaMemcpy(&c0, cyc, sizeof(c0), cudaMemcpyDeviceToHost));
      const double chains = (double)sms * block;
      printf("{\"metric\":\"sip_chain\",\"warps_per_smsp\":%d,\"sip_chain_cycles_per_word\":%.2f,"
             "\"page_chain_ms\":%.4f,\"sip_words_per_s\":%.4g}\n",
             warps_per_smsp, (double)c0 / words, ms, chains * words / (ms * 1e-3));
    }
  }
  {
    const int block = 256, grid = sms * 8, iters = 4096;
    const double ops = (double)grid * block * iters * 8;
    const char* names[4] = {"lop3_xor3", "shf_funnel", "prmt", "imad"};
    float ms[4];
    ms[0] = time_ms([&] { op_kernel<0><<<grid, block>>>(o32, iters, 0x1234567u); }, 5);
    ms[1] = time_ms([&] { op_kernel<1><<<grid, block>>>(o32, iters, 0x1234567u); }, 5);
    ms[2] = time_ms([&] { op_kernel<2><<<grid, block>>>(o32, iters, 0x1234567u); }, 5);
    ms[3] = time_ms([&] { op_kernel<3><<<grid, block>>>(o32, iters, 0x1234567u); }, 5);
    CK(cudaGetLastError());
    for (int i = 0; i < 4; ++i)
      printf("{\"metric\":\"op_rate\",\"op\":\"%s\",\"warp_inst_per_clk_per_sm_at_max_clock\":%.2f}\n", names[i],
             ops / 32.0 / (ms[i] * 1e-3) / sms / (clk_khz * 1e3));
  }
  CK(cudaDeviceSynchronize());
  return 0;
}
