// Runtime part of the backend.h ABI (backend.h:28-40) plus the dcb_* control calls.
// One process drives one GPU (multi-GPU runs one process per GPU), so the backend state
// is process-global like the reference's (backend_cuda.cu:8-46).
#include <nvtx3/nvToolsExt.h>
#include <stdarg.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "common.cuh"

namespace dcb {

static cudaStream_t g_own_stream = nullptr;
static cudaStream_t g_ext_stream = nullptr;
static bool g_use_ext = false;
static char g_name[256] = "cuda-sm100a";
static int g_err_mode = DCB_ERRORS_FATAL;
static thread_local char g_err[1024] = "";
static thread_local uint64_t g_err_count = 0;  // errors recorded on this thread so far
static std::atomic<uint64_t> g_launches{0};
int g_opt_simt = 0;
int g_opt_graphs = 0;
int g_opt_generic_epi = 0;
int g_opt_streams = 1;
int g_opt_dconv_rows = 1;
extern int g_stream_istft;

void fail(const char *fmt, ...) {
  char msg[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(msg, sizeof(msg), fmt, ap);
  va_end(ap);
  if (g_err_mode == DCB_ERRORS_FATAL) {
    fprintf(stderr, "demucs-b200: %s\n", msg);
    fflush(stderr);
    exit(1);
  }
  g_err_count++;
  if (!g_err[0]) {
    snprintf(g_err, sizeof(g_err), "%s", msg);
  }
}

bool failed() { return g_err[0] != 0; }
uint64_t error_count() { return g_err_count; }

static cudaStream_t g_override = nullptr;  // capture stream while a CUDA graph is recorded

void set_stream_override(cudaStream_t s) { g_override = s; }
cudaStream_t stream_override_get() { return g_override; }

cudaStream_t stream() {
  if (g_override) return g_override;
  if (g_use_ext) return g_ext_stream;
  if (!g_own_stream) {
    DCB_CUDA(cudaStreamCreateWithFlags(&g_own_stream, cudaStreamNonBlocking));
  }
  return g_own_stream;
}

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
void add_launches(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
uint64_t launches_now() { return g_launches.load(); }

uint16_t host_f2h(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ex = (x >> 23) & 0xffu;
  uint32_t man = x & 0x7fffffu;
  if (ex == 0xffu) return (uint16_t)(sign | 0x7c00u | (man ? 0x200u : 0u));  // inf / qNaN
  int32_t e = (int32_t)ex - 112;  // rebias 127 -> 15
  if (e >= 31) return (uint16_t)(sign | 0x7c00u);
  if (e <= 0) {  // fp16 subnormal or zero
    if (e < -10) return (uint16_t)sign;
    man |= 0x800000u;
    uint32_t sh = (uint32_t)(14 - e);
    uint32_t q = man >> sh, r = man & ((1u << sh) - 1u), halfway = 1u << (sh - 1u);
    if (r > halfway || (r == halfway && (q & 1u))) q++;
    return (uint16_t)(sign | q);
  }
  uint32_t h = sign | ((uint32_t)e << 10) | (man >> 13);
  uint32_t r = man & 0x1fffu;
  if (r > 0x1000u || (r == 0x1000u && (h & 1u))) h++;  // carry may round up the exponent
  return (uint16_t)h;
}

float host_h2f(uint16_t h) {
  uint32_t sign = ((uint32_t)h & 0x8000u) << 16, ex = (h >> 10) & 0x1fu, man = h & 0x3ffu, x;
  if (ex == 0) {
    if (!man) {
      x = sign;
    } else {
      int e = 0;
      while (!(man & 0x400u)) {
        man <<= 1;
        e++;
      }
      x = sign | ((uint32_t)(113 - e) << 23) | ((man & 0x3ffu) << 13);
    }
  } else if (ex == 31) {
    x = sign | 0x7f800000u | (man << 13);
  } else {
    x = sign | ((ex + 112) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &x, 4);
  return f;
}

}  // namespace dcb

using namespace dcb;

extern "C" {

dc_half dk_pack_half(float v, int weight) {
  (void)weight;
  return host_f2h(v);
}

int dk_init(int device, char *name, size_t name_cap) {
  int count = 0;
  cudaError_t err = cudaGetDeviceCount(&count);
  if (err != cudaSuccess || count == 0) {
    if (name && name_cap) {
      snprintf(name, name_cap, "no NVIDIA GPU / driver found (%s)",
               err != cudaSuccess ? cudaGetErrorString(err) : "0 devices");
    }
    return -1;
  }
  if (device < 0 || device >= count) {
    if (name && name_cap) snprintf(name, name_cap, "device %d out of range (%d)", device, count);
    return -1;
  }
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) {
    if (name && name_cap) snprintf(name, name_cap, "cannot query device %d", device);
    return -1;
  }
  if (prop.major != 10) {
    // the kernels are built for sm_100a only (tcgen05 / TMEM / TMA)
    if (name && name_cap) {
      snprintf(name, name_cap, "%s is sm_%d%d; this backend requires sm_100 (B200/GB200)",
               prop.name, prop.major, prop.minor);
    }
    return -1;
  }
  err = cudaSetDevice(device);
  if (err == cudaSuccess) err = cudaFree(0);
  if (err != cudaSuccess) {
    if (name && name_cap) {
      snprintf(name, name_cap, "cannot create a CUDA context: %s", cudaGetErrorString(err));
    }
    return -1;
  }
  if (!g_own_stream) {
    DCB_CUDA(cudaStreamCreateWithFlags(&g_own_stream, cudaStreamNonBlocking));
  }
  snprintf(g_name, sizeof(g_name), "%.200s sm_%d%d %.1fGiB", prop.name, prop.major, prop.minor,
           (double)prop.totalGlobalMem / (double)(1u << 30));
  if (name && name_cap) snprintf(name, name_cap, "%s", g_name);
  return 0;
}

const char *dk_backend_name(void) { return "cuda-sm100a"; }

void dk_sync(void) { DCB_CUDA(cudaStreamSynchronize(stream())); }

void *dk_raw_malloc(size_t bytes) {
  void *p = nullptr;
  if (cudaMalloc(&p, bytes ? bytes : 1) != cudaSuccess) {
    (void)cudaGetLastError();
    return nullptr;
  }
  return p;
}

void dk_raw_free(void *p) {
  if (p) {
    DCB_CUDA(cudaStreamSynchronize(stream()));
    DCB_CUDA(cudaFree(p));
  }
}

void dk_memcpy_h2d(void *dst, const void *src, size_t bytes) {
  if (bytes) {
    DCB_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, stream()));
    DCB_CUDA(cudaStreamSynchronize(stream()));
  }
}

void dk_memcpy_d2h(void *dst, const void *src, size_t bytes) {
  if (bytes) {
    DCB_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, stream()));
    DCB_CUDA(cudaStreamSynchronize(stream()));
  }
}

void dk_memcpy_d2d(void *dst, const void *src, size_t bytes) {
  if (bytes) DCB_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, stream()));
}

void dk_memset0(void *dst, size_t bytes) {
  if (bytes) DCB_CUDA(cudaMemsetAsync(dst, 0, bytes, stream()));
}

int dk_mem_info(size_t *free_bytes, size_t *total_bytes) {
  return cudaMemGetInfo(free_bytes, total_bytes) == cudaSuccess ? 0 : -1;
}

void dk_range_push(const char *name) { nvtxRangePushA(name); }
void dk_range_pop(void) { nvtxRangePop(); }

void dcb_set_error_mode(int mode) { g_err_mode = mode; }

const char *dcb_last_error(int clear) {
  static thread_local char copy[1024];
  snprintf(copy, sizeof(copy), "%s", g_err);
  if (clear) g_err[0] = 0;
  return copy;
}

void dcb_set_stream(void *s) {
  g_ext_stream = (cudaStream_t)s;
  g_use_ext = true;
}

void dcb_use_own_stream(void) { g_use_ext = false; }

void *dcb_get_stream(void) { return (void *)stream(); }

int dcb_set_option(const char *name, int value) {
  int old = -1;
  if (!strcmp(name, "simt")) {
    old = g_opt_simt;
    g_opt_simt = value;
  } else if (!strcmp(name, "graphs")) {
    old = g_opt_graphs;
    g_opt_graphs = value;
  } else if (!strcmp(name, "stream_istft")) {
    old = g_stream_istft;
    g_stream_istft = value;
  } else if (!strcmp(name, "streams")) {
    // 1: the time branch's layers run on a second stream beside the frequency branch's
    old = g_opt_streams;
    g_opt_streams = value;
  } else if (!strcmp(name, "dconv_rows")) {
    // 1: frequency-branch DConv levels that fit take the fused one-CTA-per-row kernel
    old = g_opt_dconv_rows;
    g_opt_dconv_rows = value;
  } else if (!strcmp(name, "generic_epilogue")) {
    old = g_opt_generic_epi;
    g_opt_generic_epi = value;
  } else if (!strcmp(name, "wait_limit_ms")) {
    // limit of every bounded device-side wait (default 2000 ms)
    if (value < 1) {
      fail("wait_limit_ms must be >= 1 (got %d)", value);
      return -1;
    }
    uint64_t ns = 0;
    DCB_CUDA(cudaMemcpyFromSymbol(&ns, g_wait_ns, sizeof(ns)));
    old = (int)(ns / 1000000ull);
    ns = (uint64_t)value * 1000000ull;
    DCB_CUDA(cudaMemcpyToSymbol(g_wait_ns, &ns, sizeof(ns)));
  } else if (!strcmp(name, "test_withhold_arrive")) {
    // test hook: the next tensor-core GEMM CTA keeps its first operand stage (see umma.cuh)
    uint32_t v = value ? 1u : 0u, prev = 0;
    DCB_CUDA(cudaMemcpyFromSymbol(&prev, g_test_withhold, sizeof(prev)));
    DCB_CUDA(cudaMemcpyToSymbol(g_test_withhold, &v, sizeof(v)));
    old = (int)prev;
  } else {
    fail("unknown option '%s'", name);
  }
  return old;
}

uint64_t dcb_kernel_launches(void) { return g_launches.load(); }

uint32_t dcb_device_fault(int clear) {
  uint32_t v = 0;
  DCB_CUDA(cudaMemcpyFromSymbol(&v, g_dev_fault, sizeof(v)));
  if (clear && v) {
    uint32_t z = 0;
    DCB_CUDA(cudaMemcpyToSymbol(g_dev_fault, &z, sizeof(z)));
  }
  return v;
}

}  // extern "C"
