// Normalisation part of the backend.h ABI (backend.h:72-89).
//
// Row statistics follow the reference's two-pass definition (mean, then the mean squared
// deviation, backend_cpu.c:227-243) with the row split into chunks: each CTA computes its
// chunk's mean and centred sum of squares from registers, and a second kernel merges the
// chunks with Chan's parallel formula in double (norm.cu:42-107 does the same merge).
#include <atomic>

#include "common.cuh"

namespace dcb {

constexpr int kStatChunk = 8192;  // elements per CTA
constexpr int kStatThreads = 256;

template <typename T>
static __device__ __forceinline__ T block_sum(T v, T *sh) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  T r = 0;
  int nw = blockDim.x >> 5;
  for (int i = 0; i < nw; i++) r += sh[i];
  return r;
}

// partial[row][chunk] = {count, mean, M2}; one CTA per (row, chunk) pair, the pairs
// flattened on grid.x so the row count is not bounded by grid.y's 65535
__global__ void __launch_bounds__(kStatThreads)
    k_chunk_stats(const float *__restrict__ x, int64_t L, int nchunks, double *partial) {
  __shared__ double sh[kStatThreads / 32];
  const int64_t row = blockIdx.x / (unsigned)nchunks;
  const int chunk = (int)(blockIdx.x - row * nchunks);
  int64_t c0 = (int64_t)chunk * kStatChunk;
  int64_t n = L - c0 < kStatChunk ? L - c0 : kStatChunk;
  const float *p = x + row * L + c0;
  constexpr int PER = kStatChunk / kStatThreads;
  float v[PER];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < PER; i++) {
    int64_t j = (int64_t)i * kStatThreads + threadIdx.x;
    v[i] = j < n ? p[j] : 0.f;
    s += v[i];
  }
  double tot = block_sum<double>((double)s, sh);
  double mean = tot / (double)n;
  float mf = (float)mean;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < PER; i++) {
    int64_t j = (int64_t)i * kStatThreads + threadIdx.x;
    if (j < n) {
      float d = v[i] - mf;
      q += d * d;
    }
  }
  double m2 = block_sum<double>((double)q, sh);
  // correct the centring for the float rounding of the mean: sum (x - mf)^2 =
  // M2 + n (mean - mf)^2
  double dm = mean - (double)mf;
  m2 -= (double)n * dm * dm;
  if (threadIdx.x == 0) {
    double *o = partial + (row * nchunks + chunk) * 3;
    o[0] = (double)n;
    o[1] = mean;
    o[2] = m2 > 0 ? m2 : 0.0;
  }
}

// Chan's parallel merge of (count, mean, M2) pairs
static __device__ __forceinline__ void chan_merge(double &n, double &m, double &m2, double nb,
                                                  double mb, double m2b) {
  if (nb == 0.0) return;
  if (n == 0.0) {
    n = nb;
    m = mb;
    m2 = m2b;
    return;
  }
  const double nt = n + nb, d = mb - m;
  m += d * nb / nt;
  m2 += m2b + d * d * n * nb / nt;
  n = nt;
}

// one warp per row: each lane merges a strided subset of the chunk partials, then a
// shuffle tree merges the 32 lane results
static __device__ __forceinline__ void warp_merge_row(const double *p, int nchunks, double &n,
                                                      double &m, double &m2) {
  const int lane = threadIdx.x & 31;
  n = m = m2 = 0.0;
  for (int c = lane; c < nchunks; c += 32) chan_merge(n, m, m2, p[c * 3], p[c * 3 + 1], p[c * 3 + 2]);
  for (int o = 16; o > 0; o >>= 1) {
    const double nb = __shfl_xor_sync(0xffffffffu, n, o);
    const double mb = __shfl_xor_sync(0xffffffffu, m, o);
    const double m2b = __shfl_xor_sync(0xffffffffu, m2, o);
    chan_merge(n, m, m2, nb, mb, m2b);
  }
}

__global__ void k_combine_stats(const double *partial, int64_t rows, int nchunks, float *mean,
                                float *var) {
  const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (r >= rows) return;
  double n, m, m2;
  warp_merge_row(partial + r * nchunks * 3, nchunks, n, m, m2);
  if ((threadIdx.x & 31) == 0) {
    mean[r] = (float)m;
    var[r] = (float)(m2 / n);
  }
}

// the per-chunk partials live in stream-ordered memory of the call's stream (calls on two
// streams never share them)
void row_stats(const float *x, int64_t rows, int64_t L, float *mean, float *var) {
  if (rows <= 0 || L <= 0) return;
  DCB_REQUIRE(L / kStatChunk < 0x7fffffff && rows < 0x7fffffff &&
                  rows * ((L + kStatChunk - 1) / kStatChunk) < 0x7fffffff,
              "row_stats: %lld rows of %lld elements exceed the launch limits",
              (long long)rows, (long long)L);
  int nchunks = (int)((L + kStatChunk - 1) / kStatChunk);
  const size_t need = (size_t)rows * nchunks * 3 * sizeof(double);
  double *part = nullptr;
  DCB_CUDA(cudaMallocAsync(&part, need, stream()));
  k_chunk_stats<<<(unsigned)(rows * nchunks), kStatThreads, 0, stream()>>>(x, L, nchunks, part);
  DCB_LAUNCHED();
  k_combine_stats<<<grid_for(rows * 32, 128, 1 << 30), 128, 0, stream()>>>(part, rows, nchunks,
                                                                     mean, var);
  DCB_LAUNCHED();
  DCB_CUDA(cudaFreeAsync(part, stream()));
}

// ---- allocation-free row statistics (dk_row_stats_noalloc)
// Some hosts cannot let a library allocate device memory: a real-time audio thread that
// must never block (cudaMalloc / cudaFree may synchronise the whole device), or a host
// application that hands all device memory to its own pool and budgets it exactly.  For
// them the chunk partials of the row statistics live in this fixed array instead of the
// buffer row_stats grows with cudaMalloc.  It is reserved on every GPU that loads the
// library, for the life of the process: 1 MiB = kNoAllocPartials (row, chunk) partials of
// three doubles each.
constexpr int64_t kNoAllocPartials = 43690;
static __device__ __align__(256) double g_rowstat_noalloc[kNoAllocPartials * 3];

// Device address of g_rowstat_noalloc, looked up once per device with that device current
// (on the host the array's name is only a stand-in for the device symbol, so kernels must
// be given this address).  Entries are published with release ordering, so two host
// threads that race on a device's first call both see a complete pointer (at worst both
// look it up).  The cache does not survive cudaDeviceReset: a host that resets a device
// must not call this entry point on it again in the same process.
static std::atomic<double *> g_rowstat_noalloc_ptr[64];

static double *rowstat_noalloc_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    fail("dk_row_stats_noalloc: no usable current CUDA device");
    return nullptr;
  }
  double *cached = g_rowstat_noalloc_ptr[dev].load(std::memory_order_acquire);
  if (cached) return cached;
  void *p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_rowstat_noalloc);
  if (e != cudaSuccess || !p) {
    fail("dk_row_stats_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
         cudaGetErrorString(e));
    return nullptr;
  }
  g_rowstat_noalloc_ptr[dev].store((double *)p, std::memory_order_release);
  return (double *)p;
}

int row_stats_noalloc(const float *x, int64_t rows, int64_t L, float *mean, float *var) {
  if (rows <= 0 || L <= 0) return 0;
  // errors raised by this call, not one an earlier call left pending on this thread
  const uint64_t err0 = error_count();
  const int64_t nchunks = (L + kStatChunk - 1) / kStatChunk;
  // each factor is checked before the product, so the product cannot overflow
  if (rows > kNoAllocPartials || nchunks > kNoAllocPartials ||
      rows * nchunks > kNoAllocPartials) {
    fail("dk_row_stats_noalloc: %lld rows x %lld chunks of %d elements need more than the "
         "%lld partials this entry point reserves; use dk_row_stats",
         (long long)rows, (long long)nchunks, kStatChunk, (long long)kNoAllocPartials);
    return -1;
  }
  double *part = rowstat_noalloc_ptr();
  if (!part) return -1;
  // every (row, chunk) slot used below is written by k_chunk_stats before k_combine_stats
  // reads it, so the previous call's contents never leak into this one
  k_chunk_stats<<<(unsigned)(rows * nchunks), kStatThreads, 0, stream()>>>(x, L, (int)nchunks,
                                                                          part);
  DCB_LAUNCHED();
  k_combine_stats<<<grid_for(rows * 32, 128, 1 << 30), 128, 0, stream()>>>(part, rows, (int)nchunks,
                                                                     mean, var);
  DCB_LAUNCHED();
  return error_count() != err0 ? -1 : 0;
}

// ---- row-segment kernels of the ABI's apply steps (GroupNorm apply, GroupNorm(1) over the
// last axis, per-row affine).  The work unit is one (row, segment) pair: a warp takes a
// unit, loads the row's normalisation constants once, and streams the segment's
// kSegFloats elements (float4 steps when the row length and the pointers allow it).
constexpr int64_t kSegFloats = 2048;

static inline unsigned seg_grid(int64_t units) {
  return grid_for(units * 32, 256, 148 * 16);
}

static __device__ __forceinline__ float gn_one(float v, float m, float rs, float wc, float bc,
                                               int act) {
  const float n = (v - m) * rs * wc + bc;
  return act == 1 ? gelu_f(n) : n;
}

// GroupNorm apply over x [B][C][S] (act 0 plain, 1 GELU); rows = B * C
__global__ void __launch_bounds__(256)
    k_gn_apply_rows(const float *__restrict__ x, float *__restrict__ y,
                    const float *__restrict__ mean, const float *__restrict__ var,
                    const float *__restrict__ w, const float *__restrict__ b, int64_t C,
                    int64_t S, int64_t G, float eps, int act, int64_t rows, int64_t nseg,
                    int vec) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t cpg = C / G;
  for (int64_t u = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; u < rows * nseg;
       u += nwarps) {
    const int64_t r = u / nseg, sg = u - r * nseg;
    const int64_t bi = r / C, c = r - bi * C, gi = bi * G + c / cpg;
    const float m = mean[gi], rs = 1.0f / sqrtf(var[gi] + eps), wc = w[c], bc = b[c];
    const float *xr = x + r * S;
    float *yr = y + r * S;
    const int64_t e0 = sg * kSegFloats, e1 = e0 + kSegFloats < S ? e0 + kSegFloats : S;
    if (vec) {
      for (int64_t j = e0 / 4 + lane; j < e1 / 4; j += 32) {
        float4 v = ((const float4 *)xr)[j];
        v.x = gn_one(v.x, m, rs, wc, bc, act);
        v.y = gn_one(v.y, m, rs, wc, bc, act);
        v.z = gn_one(v.z, m, rs, wc, bc, act);
        v.w = gn_one(v.w, m, rs, wc, bc, act);
        ((float4 *)yr)[j] = v;
      }
    } else {
      for (int64_t j = e0 + lane; j < e1; j += 32) yr[j] = gn_one(xr[j], m, rs, wc, bc, act);
    }
  }
}

// GroupNorm + GLU over the channel halves: y [B][C/2][S] from x [B][C][S]; rows = B * C/2,
// each output row reads its value row c and gate row c + C/2
__global__ void __launch_bounds__(256)
    k_gn_glu_rows(const float *__restrict__ x, float *__restrict__ y,
                  const float *__restrict__ mean, const float *__restrict__ var,
                  const float *__restrict__ w, const float *__restrict__ b, int64_t C,
                  int64_t S, int64_t G, float eps, int64_t rows, int64_t nseg, int vec) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t H = C / 2, cpg = C / G;
  for (int64_t u = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; u < rows * nseg;
       u += nwarps) {
    const int64_t r = u / nseg, sg = u - r * nseg;
    const int64_t bi = r / H, c = r - bi * H;
    const int64_t ga = bi * G + c / cpg, gb = bi * G + (c + H) / cpg;
    const float ma = mean[ga], ra = 1.0f / sqrtf(var[ga] + eps), wa = w[c], ba = b[c];
    const float mb = mean[gb], rb = 1.0f / sqrtf(var[gb] + eps), wb = w[c + H], bb = b[c + H];
    const float *xa = x + (bi * C + c) * S, *xb = xa + H * S;
    float *yr = y + r * S;
    const int64_t e0 = sg * kSegFloats, e1 = e0 + kSegFloats < S ? e0 + kSegFloats : S;
    if (vec) {
      for (int64_t j = e0 / 4 + lane; j < e1 / 4; j += 32) {
        const float4 va = ((const float4 *)xa)[j], vb = ((const float4 *)xb)[j];
        float4 o;
        o.x = gn_one(va.x, ma, ra, wa, ba, 0) * sigmoid_f(gn_one(vb.x, mb, rb, wb, bb, 0));
        o.y = gn_one(va.y, ma, ra, wa, ba, 0) * sigmoid_f(gn_one(vb.y, mb, rb, wb, bb, 0));
        o.z = gn_one(va.z, ma, ra, wa, ba, 0) * sigmoid_f(gn_one(vb.z, mb, rb, wb, bb, 0));
        o.w = gn_one(va.w, ma, ra, wa, ba, 0) * sigmoid_f(gn_one(vb.w, mb, rb, wb, bb, 0));
        ((float4 *)yr)[j] = o;
      }
    } else {
      for (int64_t j = e0 + lane; j < e1; j += 32) {
        yr[j] = gn_one(xa[j], ma, ra, wa, ba, 0) * sigmoid_f(gn_one(xb[j], mb, rb, wb, bb, 0));
      }
    }
  }
}

// Normalisation over whole rows of L elements with an affine on the last axis of length C
// (channel j % C): the scalar path of dk_norm_apply_last for rows that k_norm_last4 does not
// take.  A lane's channel index starts at (e0 + lane) % C and advances by 32 % C per step.
__global__ void __launch_bounds__(256)
    k_norm_last(const float *__restrict__ x, float *__restrict__ y,
                const float *__restrict__ mean, const float *__restrict__ var,
                const float *__restrict__ w, const float *__restrict__ b, int64_t rows,
                int64_t L, int64_t C, float eps, int64_t nseg) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t step = 32 % C;
  for (int64_t u = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; u < rows * nseg;
       u += nwarps) {
    const int64_t r = u / nseg, sg = u - r * nseg;
    const float m = mean[r], rs = 1.0f / sqrtf(var[r] + eps);
    const float *xr = x + r * L;
    float *yr = y + r * L;
    const int64_t e0 = sg * kSegFloats, e1 = e0 + kSegFloats < L ? e0 + kSegFloats : L;
    int64_t c = (e0 + lane) % C;
    for (int64_t j = e0 + lane; j < e1; j += 32) {
      float v = (xr[j] - m) * rs;
      if (w) v *= w[c];
      if (b) v += b[c];
      yr[j] = v;
      c += step;
      if (c >= C) c -= C;
    }
  }
}

// k_norm_last for rows of L = n * C floats with C % 4 == 0 (16-byte aligned): grid (blocks,
// rows), float4 per thread step, the channel index advanced incrementally (no divisions in
// the loop)
// (sums: the row's statistics as fp64 sum and sum of squares of its L values, in place of
// mean / var, split over kSumSlots slots [row][slot][2])
constexpr int kSumSlots = 16;
static __device__ __forceinline__ void stats_from_sums(const double *sums, int64_t r,
                                                       double inv_n, float &m, float &v) {
  double s = 0.0, q = 0.0;
  const double *p = sums + 2 * kSumSlots * r;
#pragma unroll
  for (int i = 0; i < kSumSlots; i++) {
    s += p[2 * i];
    q += p[2 * i + 1];
  }
  const double md = s * inv_n;
  const double vd = q * inv_n - md * md;
  m = (float)md;
  v = vd > 0.0 ? (float)vd : 0.f;
}

__global__ void k_norm_last4(const float4 *__restrict__ x, float4 *__restrict__ y,
                             const float *__restrict__ mean, const float *__restrict__ var,
                             const float *__restrict__ w, const float *__restrict__ b, int L4,
                             int C4, float eps, const double *__restrict__ sums, double inv_n) {
  const int r = blockIdx.y;
  float m, vr;
  if (sums) {
    stats_from_sums(sums, r, inv_n, m, vr);
  } else {
    m = mean[r];
    vr = var[r];
  }
  const float rs = 1.0f / sqrtf(vr + eps);
  const float4 *xr = x + (int64_t)r * L4;
  float4 *yr = y + (int64_t)r * L4;
  const float4 *w4 = (const float4 *)w, *b4 = (const float4 *)b;
  const int stride = gridDim.x * blockDim.x;
  const int cstep = stride % C4;
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  int c = i % C4;
  for (; i < L4; i += stride) {
    const float4 v = xr[i];
    float4 o = make_float4((v.x - m) * rs, (v.y - m) * rs, (v.z - m) * rs, (v.w - m) * rs);
    if (w4) {
      const float4 g = w4[c];
      o.x *= g.x;
      o.y *= g.y;
      o.z *= g.z;
      o.w *= g.w;
    }
    if (b4) {
      const float4 h = b4[c];
      o.x += h.x;
      o.y += h.y;
      o.z += h.z;
      o.w += h.w;
    }
    yr[i] = o;
    c += cstep;
    if (c >= C4) c -= C4;
  }
}

// HTDemucs input normalisation / output denormalisation per row (x - m) / (sd + eps) or
// x (sd + eps) + m with sd = sqrt(var): one warp per (row, segment) unit, the row's
// constants formed once per unit
__global__ void __launch_bounds__(256)
    k_affine_rows(const float *__restrict__ x, float *__restrict__ y,
                  const float *__restrict__ mean, const float *__restrict__ var, int64_t rows,
                  int64_t L, float eps, int denorm, int64_t nseg, int vec) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t u = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; u < rows * nseg;
       u += nwarps) {
    const int64_t r = u / nseg, sg = u - r * nseg;
    const float sd = sqrtf(var[r]) + eps, m = mean[r];
    const float *xr = x + r * L;
    float *yr = y + r * L;
    const int64_t e0 = sg * kSegFloats, e1 = e0 + kSegFloats < L ? e0 + kSegFloats : L;
    if (vec) {
      for (int64_t j = e0 / 4 + lane; j < e1 / 4; j += 32) {
        float4 v = ((const float4 *)xr)[j];
        if (denorm) {
          v = make_float4(v.x * sd + m, v.y * sd + m, v.z * sd + m, v.w * sd + m);
        } else {
          v = make_float4((v.x - m) / sd, (v.y - m) / sd, (v.z - m) / sd, (v.w - m) / sd);
        }
        ((float4 *)yr)[j] = v;
      }
    } else {
      for (int64_t j = e0 + lane; j < e1; j += 32) {
        const float v = xr[j];
        yr[j] = denorm ? v * sd + m : (v - m) / sd;
      }
    }
  }
}

// LayerNorm, one warp per row, row kept in registers (C <= 32 * 32 * 4 = 4096 floats per
// warp in float4 chunks; larger rows fall back to row_stats + apply).  Output either fp32
// or fp16 (the latter is the GEMM A operand of the next linear, rounded exactly as
// dk_to_half_rows would round the fp32 result).
template <bool HALF_OUT>
__global__ void k_layernorm(const float *__restrict__ x, void *__restrict__ yv,
                            const float *__restrict__ w, const float *__restrict__ b,
                            int64_t rows, int C, float eps, int ld_out) {
  int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float *p = x + row * C;
  constexpr int MAXV = 32;
  float v[MAXV];
  int nv = 0;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; i++) {
    int c = i * 32 + lane;
    v[i] = c < C ? p[c] : 0.f;
    s += v[i];
    nv = i;
  }
  (void)nv;
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  double mean_d = (double)s / (double)C;
  float m = (float)mean_d;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; i++) {
    int c = i * 32 + lane;
    if (c < C) {
      float d = v[i] - m;
      q += d * d;
    }
  }
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  double dm = mean_d - (double)m;
  double m2 = (double)q - (double)C * dm * dm;
  float var = (float)((m2 > 0 ? m2 : 0.0) / (double)C);
  float rs = 1.0f / sqrtf(var + eps);
#pragma unroll
  for (int i = 0; i < MAXV; i++) {
    int c = i * 32 + lane;
    if (c < C) {
      float n = (v[i] - m) * rs;
      if (w) n *= w[c];
      if (b) n += b[c];
      if (HALF_OUT) {
        ((uint16_t *)yv)[row * ld_out + c] = f2h_bits(n);
      } else {
        ((float *)yv)[row * ld_out + c] = n;
      }
    } else if (HALF_OUT && c < ld_out) {
      ((uint16_t *)yv)[row * ld_out + c] = 0;
    }
  }
}

// Rows of C = 128 * NV floats: each lane holds NV float4 (16-byte loads; fp16 output as
// 8-byte stores).  Same statistics as k_layernorm (sum in fp32 across lanes, the second
// moment about the fp32 mean with the fp64 correction).
template <int NV, bool HALF_OUT>
__global__ void __launch_bounds__(128)
    k_layernorm_v4(const float *__restrict__ x, void *__restrict__ yv,
                   const float *__restrict__ w, const float *__restrict__ b, int64_t rows,
                   float eps, int ld_out) {
  constexpr int C = 128 * NV;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float4 *p = (const float4 *)(x + row * C);
  float4 v[NV];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; i++) {
    v[i] = p[i * 32 + lane];
    s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const double mean_d = (double)s / (double)C;
  const float m = (float)mean_d;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < NV; i++) {
    const float a = v[i].x - m, bq = v[i].y - m, c = v[i].z - m, d = v[i].w - m;
    q += (a * a + bq * bq) + (c * c + d * d);
  }
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const double dm = mean_d - (double)m;
  const double m2 = (double)q - (double)C * dm * dm;
  const float var = (float)((m2 > 0 ? m2 : 0.0) / (double)C);
  const float rs = 1.0f / sqrtf(var + eps);
#pragma unroll
  for (int i = 0; i < NV; i++) {
    const int c0 = (i * 32 + lane) * 4;
    float n[4] = {(v[i].x - m) * rs, (v[i].y - m) * rs, (v[i].z - m) * rs, (v[i].w - m) * rs};
    if (w) {
      const float4 wv = *(const float4 *)(w + c0);
      n[0] *= wv.x;
      n[1] *= wv.y;
      n[2] *= wv.z;
      n[3] *= wv.w;
    }
    if (b) {
      const float4 bv = *(const float4 *)(b + c0);
      n[0] += bv.x;
      n[1] += bv.y;
      n[2] += bv.z;
      n[3] += bv.w;
    }
    if (HALF_OUT) {
      *(uint2 *)((uint16_t *)yv + row * ld_out + c0) =
          make_uint2(pack_h2(n[0], n[1]), pack_h2(n[2], n[3]));
    } else {
      *(float4 *)((float *)yv + row * ld_out + c0) = make_float4(n[0], n[1], n[2], n[3]);
    }
  }
}

void layernorm(const float *x, void *y, const float *w, const float *b, int64_t rows, int C,
               float eps, bool half_out, int ld_out) {
  if (rows <= 0) return;
  TraceScope ts(TR_NORM, 0.0, (double)rows * C * (4.0 + (half_out ? 2.0 : 4.0)), rows, C, 0);
  // vector path: C = 128 * NV with aligned rows and parameters (and no output padding)
  const bool vec = C % 128 == 0 && C <= 1024 && ld_out == C && ((uintptr_t)x & 15) == 0 &&
                   ((uintptr_t)y & 15) == 0 && (!w || ((uintptr_t)w & 15) == 0) &&
                   (!b || ((uintptr_t)b & 15) == 0);
  if (vec) {
    const unsigned blocks = (unsigned)((rows + 3) / 4);
#define DCB_LNV(NV)                                                                       \
  if (half_out)                                                                           \
    k_layernorm_v4<NV, true><<<blocks, 128, 0, stream()>>>(x, y, w, b, rows, eps, ld_out);  \
  else                                                                                    \
    k_layernorm_v4<NV, false><<<blocks, 128, 0, stream()>>>(x, y, w, b, rows, eps, ld_out)
    switch (C / 128) {
      case 1: DCB_LNV(1); break;
      case 2: DCB_LNV(2); break;
      case 3: DCB_LNV(3); break;
      case 4: DCB_LNV(4); break;
      case 5: DCB_LNV(5); break;
      case 6: DCB_LNV(6); break;
      case 7: DCB_LNV(7); break;
      default: DCB_LNV(8); break;
    }
#undef DCB_LNV
    DCB_LAUNCHED();
    return;
  }
  if (C <= 1024) {
    unsigned blocks = (unsigned)((rows + 3) / 4);
    if (half_out) {
      k_layernorm<true><<<blocks, 128, 0, stream()>>>(x, y, w, b, rows, C, eps, ld_out);
    } else {
      k_layernorm<false><<<blocks, 128, 0, stream()>>>(x, y, w, b, rows, C, eps, ld_out);
    }
    DCB_LAUNCHED();
    return;
  }
  // long rows: generic two kernels (fp32 output only)
  DCB_REQUIRE(!half_out, "layernorm: fp16 output needs C <= 1024");
  float *st = nullptr;
  DCB_CUDA(cudaMallocAsync(&st, (size_t)rows * 2 * sizeof(float), stream()));
  row_stats(x, rows, C, st, st + rows);
  const int64_t nseg = (C + kSegFloats - 1) / kSegFloats;
  k_norm_last<<<seg_grid(rows * nseg), 256, 0, stream()>>>(x, (float *)y, st, st + rows, w, b,
                                                           rows, C, C, eps, nseg);
  DCB_LAUNCHED();
  DCB_CUDA(cudaFreeAsync(st, stream()));
}

}  // namespace dcb

using namespace dcb;

extern "C" {

void dk_row_stats(const float *x, int64_t rows, int64_t L, float *mean, float *var) {
  row_stats(x, rows, L, mean, var);
}

int dk_row_stats_noalloc(const float *x, int64_t rows, int64_t L, float *mean, float *var) {
  return row_stats_noalloc(x, rows, L, mean, var);
}

void dk_groupnorm_apply(const float *x, float *y, const float *mean, const float *var,
                        const float *w, const float *b, int64_t B, int64_t C, int64_t S,
                        int64_t G, float eps, int act) {
  if (B <= 0 || C <= 0 || S <= 0) return;
  DCB_REQUIRE(G > 0 && C % G == 0 && (act != 2 || C % 2 == 0),
              "groupnorm_apply: C %lld, groups %lld, act %d", (long long)C, (long long)G, act);
  const int64_t nseg = (S + kSegFloats - 1) / kSegFloats;
  const int vec = S % 4 == 0 && (((uintptr_t)x | (uintptr_t)y) & 15) == 0;
  if (act == 2) {
    const int64_t rows = B * (C / 2);
    k_gn_glu_rows<<<seg_grid(rows * nseg), 256, 0, stream()>>>(x, y, mean, var, w, b, C, S, G,
                                                               eps, rows, nseg, vec);
  } else {
    const int64_t rows = B * C;
    k_gn_apply_rows<<<seg_grid(rows * nseg), 256, 0, stream()>>>(x, y, mean, var, w, b, C, S,
                                                                 G, eps, act, rows, nseg, vec);
  }
  DCB_LAUNCHED();
}

void dk_norm_apply_last(const float *x, float *y, const float *mean, const float *var,
                        const float *w, const float *b, int64_t rows, int64_t L, int64_t C,
                        float eps) {
  if (rows <= 0 || L <= 0) return;
  DCB_REQUIRE(C > 0, "norm_apply_last: C %lld", (long long)C);
  const bool al = ((uintptr_t)x | (uintptr_t)y | (uintptr_t)w | (uintptr_t)b) % 16 == 0;
  if (al && C % 4 == 0 && L % C == 0 && L / 4 < (1ll << 31) && rows <= 65535) {
    const int L4 = (int)(L / 4), C4 = (int)(C / 4);
    const unsigned bx = grid_for(L4, 256, (148 * 8 + rows - 1) / rows);
    k_norm_last4<<<dim3(bx, (unsigned)rows), 256, 0, stream()>>>(
        (const float4 *)x, (float4 *)y, mean, var, w, b, L4, C4, eps, nullptr, 0.0);
  } else {
    const int64_t nseg = (L + kSegFloats - 1) / kSegFloats;
    k_norm_last<<<seg_grid(rows * nseg), 256, 0, stream()>>>(x, y, mean, var, w, b, rows, L, C,
                                                             eps, nseg);
  }
  DCB_LAUNCHED();
}

__global__ void k_sums_to_stats(const double *__restrict__ sums, int64_t rows, double inv_n,
                                float *__restrict__ mean, float *__restrict__ var) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r < rows) stats_from_sums(sums, r, inv_n, mean[r], var[r]);
}

// dk_norm_apply_last with each row's statistics given as fp64 sums [rows][kSumSlots][2]
// (partial sums and sums of squares of its L values, added over the slots), e.g. formed by
// the producing GEMM's epilogue
void norm_apply_last_sums(const float *x, float *y, const double *sums, const float *w,
                          const float *b, int64_t rows, int64_t L, int64_t C, float eps) {
  if (rows <= 0 || L <= 0) return;
  DCB_REQUIRE(C > 0, "norm_apply_last: C %lld", (long long)C);
  const double inv_n = 1.0 / (double)L;
  const bool al = ((uintptr_t)x | (uintptr_t)y | (uintptr_t)w | (uintptr_t)b) % 16 == 0;
  if (al && C % 4 == 0 && L % C == 0 && L / 4 < (1ll << 31) && rows <= 65535) {
    const int L4 = (int)(L / 4), C4 = (int)(C / 4);
    const unsigned bx = grid_for(L4, 256, (148 * 8 + rows - 1) / rows);
    k_norm_last4<<<dim3(bx, (unsigned)rows), 256, 0, stream()>>>(
        (const float4 *)x, (float4 *)y, nullptr, nullptr, w, b, L4, C4, eps, sums, inv_n);
    DCB_LAUNCHED();
    return;
  }
  float *st = nullptr;
  DCB_CUDA(cudaMallocAsync(&st, (size_t)rows * 2 * sizeof(float), stream()));
  k_sums_to_stats<<<grid_for(rows, 128, 1 << 30), 128, 0, stream()>>>(sums, rows, inv_n, st,
                                                                      st + rows);
  DCB_LAUNCHED();
  dk_norm_apply_last(x, y, st, st + rows, w, b, rows, L, C, eps);
  DCB_CUDA(cudaFreeAsync(st, stream()));
}

void dk_affine_rows(const float *x, float *y, const float *mean, const float *var,
                    int64_t rows, int64_t L, float eps, int denorm) {
  if (rows <= 0 || L <= 0) return;
  const int64_t nseg = (L + kSegFloats - 1) / kSegFloats;
  const int vec = L % 4 == 0 && (((uintptr_t)x | (uintptr_t)y) & 15) == 0;
  k_affine_rows<<<seg_grid(rows * nseg), 256, 0, stream()>>>(x, y, mean, var, rows, L, eps,
                                                             denorm, nseg, vec);
  DCB_LAUNCHED();
}

void dk_layernorm(const float *x, float *y, const float *w, const float *b, int64_t rows,
                  int64_t C, float eps) {
  layernorm(x, y, w, b, rows, (int)C, eps, false, (int)C);
}

}  // extern "C"
