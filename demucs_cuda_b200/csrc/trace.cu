// Per-kernel-class CUDA-event trace.  When a class is enabled (dcb_trace_start), every
// launch of that class is bracketed by two events on the launching stream and tagged with
// its algorithmic FLOPs and bytes (unpadded problem sizes), so a host can measure achieved
// TFLOP/s or GB/s of a kernel family inside a timed region.
#include <vector>

#include "common.cuh"

namespace dcb {

// classes 0-4 are tensor-core kernels (FLOPs and minimum bytes), 5-7 the memory-bound glue
// of the forward (minimum bytes: each input read once, each output written once): the STFT /
// inverse STFT and their layout passes, the DConv GroupNorm statistics and CUDA-core tail,
// and the transformer's LayerNorms / GroupNorm
enum TraceClass : int {
  TR_CONV = 0, TR_CONVTR, TR_LINEAR, TR_ATTN, TR_GEMM, TR_SPECTRAL, TR_DCONV, TR_NORM,
  TR_NCLASS
};

struct TraceRec {
  int cls;
  cudaEvent_t a, b;
  double flops, bytes;
  int64_t M, N, K;  // problem extents of the launch (for per-shape breakdowns)
};

static uint32_t g_trace_mask = 0;
static std::vector<TraceRec> g_trace;
static std::vector<cudaEvent_t> g_event_pool;

static cudaEvent_t trace_event() {
  if (!g_event_pool.empty()) {
    cudaEvent_t e = g_event_pool.back();
    g_event_pool.pop_back();
    return e;
  }
  cudaEvent_t e;
  DCB_CUDA(cudaEventCreate(&e));
  return e;
}

struct TraceScope {
  bool on;
  TraceRec rec;
  TraceScope(int cls, double flops, double bytes, int64_t M = 0, int64_t N = 0, int64_t K = 0)
      : on((g_trace_mask >> cls) & 1u) {
    if (!on) return;
    rec.M = M;
    rec.N = N;
    rec.K = K;
    rec.cls = cls;
    rec.flops = flops;
    rec.bytes = bytes;
    rec.a = trace_event();
    rec.b = trace_event();
    DCB_CUDA(cudaEventRecord(rec.a, stream()));
  }
  ~TraceScope() {
    if (!on) return;
    DCB_CUDA(cudaEventRecord(rec.b, stream()));
    g_trace.push_back(rec);
  }
};

}  // namespace dcb

using namespace dcb;

extern "C" {

void dcb_trace_start(uint32_t mask) {
  g_trace_mask = mask;
  for (auto &r : g_trace) {
    g_event_pool.push_back(r.a);
    g_event_pool.push_back(r.b);
  }
  g_trace.clear();
}

int dcb_trace_stop(double *ms, double *flops, double *bytes, int *launches, int ncls) {
  g_trace_mask = 0;
  DCB_CUDA(cudaStreamSynchronize(stream()));
  for (int c = 0; c < ncls; c++) {
    ms[c] = flops[c] = bytes[c] = 0.0;
    launches[c] = 0;
  }
  for (auto &r : g_trace) {
    if (r.cls >= ncls) continue;
    float t = 0.f;
    DCB_CUDA(cudaEventElapsedTime(&t, r.a, r.b));
    ms[r.cls] += t;
    flops[r.cls] += r.flops;
    bytes[r.cls] += r.bytes;
    launches[r.cls] += 1;
  }
  return (int)g_trace.size();
}

int dcb_trace_dump(const char *path) {
  FILE *f = fopen(path, "w");
  if (!f) return -1;
  DCB_CUDA(cudaStreamSynchronize(stream()));
  fprintf(f, "class,ms,flops,bytes,M,N,K\n");
  for (auto &r : g_trace) {
    float t = 0.f;
    DCB_CUDA(cudaEventElapsedTime(&t, r.a, r.b));
    fprintf(f, "%d,%.6f,%.0f,%.0f,%lld,%lld,%lld\n", r.cls, t, r.flops, r.bytes,
            (long long)r.M, (long long)r.N, (long long)r.K);
  }
  fclose(f);
  return (int)g_trace.size();
}

}  // extern "C"
