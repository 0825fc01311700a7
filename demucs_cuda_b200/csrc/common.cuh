// Shared helpers of the sm_100a backend: error handling, the backend stream, launch
// accounting and fp16 conversion.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/dc_b200.h"

namespace dcb {

// ------------------------------------------------------------------ errors
// The reference aborts through dc_die on any failure (cuda_common.cuh:17-26).  The same
// is the default here; a host may instead ask for the error to be recorded and the call to
// return (dcb_set_error_mode).
void fail(const char *fmt, ...);
bool failed();  // an error is pending in return mode
// number of errors this thread has recorded (return mode); a call that compares it before
// and after knows whether it raised one itself, whatever error was already pending
uint64_t error_count();
cudaStream_t stream();
void count_launch();
void add_launches(uint64_t n);
uint64_t launches_now();
void set_stream_override(cudaStream_t s);
cudaStream_t stream_override_get();

#define DCB_CUDA(call)                                                                   \
  do {                                                                                   \
    cudaError_t e_ = (call);                                                             \
    if (e_ != cudaSuccess) {                                                             \
      ::dcb::fail("CUDA error %s at %s:%d: %s", cudaGetErrorName(e_), __FILE__, __LINE__, \
                  cudaGetErrorString(e_));                                               \
    }                                                                                    \
  } while (0)

#define DCB_LAUNCHED()                  \
  do {                                  \
    ::dcb::count_launch();              \
    DCB_CUDA(cudaGetLastError());       \
  } while (0)

#define DCB_REQUIRE(cond, ...)  \
  do {                          \
    if (!(cond)) {              \
      ::dcb::fail(__VA_ARGS__); \
      return;                   \
    }                           \
  } while (0)

// option values (dcb_set_option)
extern int g_opt_simt;
extern int g_opt_graphs;
extern int g_opt_streams;
extern int g_opt_dconv_rows;
extern int g_opt_generic_epi;  // channels-last convs take the generic epilogue

// device fault word written by bounded waits (see umma.cuh); the library is one
// translation unit (all.cu), so the definition lives here
__device__ uint32_t g_dev_fault = 0;
// limit of every bounded wait in nanoseconds (option "wait_limit_ms"; default 2 s)
__device__ uint64_t g_wait_ns = 2000000000ull;
// One-shot test hook (option "test_withhold_arrive"): while non-zero, the first tensor-core
// GEMM CTA that reaches its first operand stage consumes the flag and does not release that
// stage, so the producer's next wait on it can only end by the bounded-wait limit.
__device__ uint32_t g_test_withhold = 0;

static inline unsigned grid_for(int64_t n, int threads, int64_t cap = 148 * 32) {
  int64_t b = (n + threads - 1) / threads;
  if (b > cap) b = cap;
  return (unsigned)(b < 1 ? 1 : b);
}

#define DCB_GRID_STRIDE(i, n) \
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (n); \
       i += (int64_t)blockDim.x * gridDim.x)

// ------------------------------------------------------------------ numerics
// GELU in the erf form the reference uses (backend_cpu.c:144, cuda_common.cuh:42-44).
// 2^x by the hardware approximation (ex2.approx.ftz: relative error ~2^-22, results below
// 2^-126 flush to zero)
static __device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// GELU, x Phi(x) with Phi(x) = (1 + erf(x / sqrt 2)) / 2 (the exact form of layers.c).
// erf(z), z >= 0, from Abramowitz & Stegun 7.1.26: 1 - (a1 t + ... + a5 t^5) exp(-z^2),
// t = 1 / (1 + p z), |error| <= 1.5e-7.  The tail h = (1 - erf(|x| / sqrt 2)) / 2 is formed
// directly (coefficients pre-halved), so Phi = 1 - h for x >= 0 and h for x < 0 without
// cancellation.  |GELU error| <= 3e-7 (|x| + 1) against float64 erf (pinned by a GPU test).
static __device__ __forceinline__ float gelu_f(float x) {
  const float z = fabsf(x) * 0.70710678118654752f;
  const float t = __fdividef(1.0f, fmaf(0.3275911f, z, 1.0f));
  float p = fmaf(0.5307027145f, t, -0.7265760135f);  // a5 / 2, a4 / 2
  p = fmaf(p, t, 0.7107068705f);                      // a3 / 2
  p = fmaf(p, t, -0.142248368f);                      // a2 / 2
  p = fmaf(p, t, 0.127414796f);                       // a1 / 2
  const float h = p * t * ex2_approx(x * x * -0.72134752044448170f);  // exp(-x^2 / 2)
  return x * (x >= 0.f ? 1.0f - h : h);
}
static __device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }
// fp32 -> fp16 bits, round to nearest even (the reference's dc_f32_to_f16 rule).
static __device__ __forceinline__ uint16_t f2h_bits(float v) {
  return __half_as_ushort(__float2half_rn(v));
}
static __device__ __forceinline__ float h2f_bits(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}
// (c0, c1) += (a0, a1) * (b0, b1) by one packed fp32 FMA (sm_100 fma.rn.f32x2; each lane
// rounds as fmaf does)
static __device__ __forceinline__ void ffma2(float &c0, float &c1, float a0, float a1, float b0,
                                             float b1) {
  asm("{\n\t.reg .b64 ra, rb, rc;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%0, %1};\n\t"
      "fma.rn.f32x2 rc, ra, rb, rc;\n\t"
      "mov.b64 {%0, %1}, rc;\n\t}"
      : "+f"(c0), "+f"(c1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}
// two floats -> packed fp16x2 (low = a)
static __device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  // one packed conversion (both halves round to nearest even): d = {hi: b, lo: a}
  uint32_t d;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(b), "f"(a));
  return d;
}

// host side RNE conversion (IEEE 754 binary32 -> binary16)
uint16_t host_f2h(float f);
float host_h2f(uint16_t h);

}  // namespace dcb
