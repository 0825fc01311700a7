// Spectral part of the backend.h ABI (backend.h:133-144): Hann-windowed STFT, inverse
// frames and overlap-add.  One CTA transforms one frame in shared memory (iterative radix-2
// decimation in time over bit-reversed input, the same butterfly order as the reference's
// fft_radix2, backend_cpu.c:549-567); twiddles exp(-2 pi i k / n) are evaluated in double
// on the host and stored as float (fft.cu:9-63 does the same).
#include <math.h>

#include <vector>

#include "common.cuh"

namespace dcb {

static float2 *g_tw = nullptr;
static int g_tw_n = 0;

const float2 *twiddles(int n) {
  if (g_tw_n == n) return g_tw;
  if (n <= 1 || (n & (n - 1)) || n > 8192) {
    fail("fft size %d must be a power of two <= 8192", n);
    return nullptr;
  }
  std::vector<float2> h(n / 2);
  for (int k = 0; k < n / 2; k++) {
    double a = -2.0 * 3.14159265358979323846 * (double)k / (double)n;
    h[k] = make_float2((float)cos(a), (float)sin(a));
  }
  if (g_tw) {
    DCB_CUDA(cudaStreamSynchronize(stream()));
    DCB_CUDA(cudaFree(g_tw));
  }
  DCB_CUDA(cudaMalloc(&g_tw, (n / 2) * sizeof(float2)));
  DCB_CUDA(cudaMemcpy(g_tw, h.data(), (n / 2) * sizeof(float2), cudaMemcpyHostToDevice));
  g_tw_n = n;
  return g_tw;
}

static __device__ __forceinline__ int bitrev(int i, int bits) {
  return (int)(__brev((unsigned)i) >> (32 - bits));
}

// in-place forward DFT of bit-reversed data in shared memory
static __device__ void fft_smem(float2 *buf, int n, const float2 *__restrict__ tw) {
  for (int half = 1; half < n; half <<= 1) {
    __syncthreads();
    int step = n / (2 * half);
    for (int j = threadIdx.x; j < n / 2; j += blockDim.x) {
      int pos = j & (half - 1);
      int i0 = (j / half) * 2 * half + pos, i1 = i0 + half;
      float2 w = tw[pos * step];
      float2 a = buf[i0], b = buf[i1];
      float tr = w.x * b.x - w.y * b.y, ti = w.x * b.y + w.y * b.x;
      buf[i1] = make_float2(a.x - tr, a.y - ti);
      buf[i0] = make_float2(a.x + tr, a.y + ti);
    }
  }
  __syncthreads();
}

__global__ void k_stft(const float *__restrict__ sig, float *__restrict__ out, int64_t L,
                       int n, int bits, int hop, int frame0, int nframes, int nbins,
                       const float *__restrict__ window, const float2 *__restrict__ tw) {
  extern __shared__ float2 buf[];
  int f = blockIdx.x;
  int64_t r = blockIdx.y;
  int64_t start = (int64_t)(frame0 + f) * hop;
  const float *s = sig + r * L;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    int64_t t = start + i;
    float v = t < L ? s[t] * window[i] : 0.f;
    buf[bitrev(i, bits)] = make_float2(v, 0.f);
  }
  fft_smem(buf, n, tw);
  float *ore = out + r * 2 * (int64_t)nbins * nframes;
  float *oim = ore + (int64_t)nbins * nframes;
  for (int k = threadIdx.x; k < nbins; k += blockDim.x) {
    ore[(int64_t)k * nframes + f] = buf[k].x;
    oim[(int64_t)k * nframes + f] = buf[k].y;
  }
}

__global__ void k_istft_frames(const float *__restrict__ spec, float *__restrict__ frames,
                               int nbins, int nframes, int pad_frames, int n, int bits,
                               const float *__restrict__ window,
                               const float2 *__restrict__ tw) {
  extern __shared__ float2 buf[];
  int NF = nframes + 2 * pad_frames;
  int f = blockIdx.x;
  int64_t r = blockIdx.y;
  float *dst = frames + (r * NF + f) * (int64_t)n;
  int fi = f - pad_frames;
  if (fi < 0 || fi >= nframes) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = 0.f;
    return;
  }
  const float *sre = spec + r * 2 * (int64_t)nbins * nframes;
  const float *sim = sre + (int64_t)nbins * nframes;
  for (int k = threadIdx.x; k < n; k += blockDim.x) {
    int kk = k <= n / 2 ? k : n - k;
    float xr = 0.f, xi = 0.f;
    if (kk < nbins) {
      xr = sre[(int64_t)kk * nframes + fi];
      xi = sim[(int64_t)kk * nframes + fi];
    }
    if (k > n / 2) xi = -xi;
    buf[bitrev(k, bits)] = make_float2(xr, -xi);
  }
  fft_smem(buf, n, tw);
  float inv_n = 1.0f / (float)n;
  for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = buf[i].x * inv_n * window[i];
}

__global__ void k_ola(const float *__restrict__ frames, float *__restrict__ out, int64_t R,
                      int nframes, int n, int hop, const float *__restrict__ window,
                      int64_t start, int64_t length) {
  int64_t out_len = (int64_t)hop * (nframes - 1) + n, total = R * length;
  DCB_GRID_STRIDE(e, total) {
    int64_t r = e / length, t = e - r * length, idx = start + t;
    float num = 0.f, den = 0.f;
    if (idx < out_len) {
      int64_t f_hi = idx / hop;
      if (f_hi > nframes - 1) f_hi = nframes - 1;
      int64_t f_lo = idx - n + 1 <= 0 ? 0 : (idx - n + hop) / hop;
      for (int64_t f = f_lo; f <= f_hi; f++) {
        int64_t i = idx - f * hop;
        if (i < 0 || i >= n) continue;
        num += frames[(r * nframes + f) * n + i];
        den += window[i] * window[i];
      }
    }
    out[e] = den > 0.f ? num / den : 0.f;
  }
}

// Decoder output x [B][S*2C][F][N] (channel 2q = real, 2q+1 = imaginary of row q = (s, c))
// -> z [B*S*C][N][F] complex, frame-major, denormalised per batch
// (v * (sqrt(var) + eps) + mean, htdemucs.c:251): 32x32 shared-memory tiles, coalesced on
// both sides.
__global__ void k_spec_frames_major(const float *__restrict__ x, float2 *__restrict__ z,
                                    const float *__restrict__ mean,
                                    const float *__restrict__ var, int rows_per_b, int F,
                                    int N, float eps) {
  __shared__ float tre[32][33], tim[32][33];
  const int r = blockIdx.z;
  const int b = r / rows_per_b, q = r - b * rows_per_b;
  const int f0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
  const float sd = sqrtf(var[b]) + eps, m = mean[b];
  const float *xre = x + ((int64_t)b * 2 * rows_per_b + 2 * q) * F * (int64_t)N;
  const float *xim = xre + (int64_t)F * N;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int f = f0 + i, n = n0 + threadIdx.x;
    if (f < F && n < N) {
      tre[i][threadIdx.x] = xre[(int64_t)f * N + n] * sd + m;
      tim[i][threadIdx.x] = xim[(int64_t)f * N + n] * sd + m;
    }
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int n = n0 + i, f = f0 + threadIdx.x;
    if (f < F && n < N)
      z[((int64_t)r * N + n) * F + f] = make_float2(tre[threadIdx.x][i], tim[threadIdx.x][i]);
  }
}

// Fused inverse STFT + overlap-add (dk_istft_frames + dk_ola, backend_cpu.c:596-662): CTA =
// one row and kOlaHops consecutive hops of the padded OLA signal.  Every frame touching
// them (pad frames are zero) is inverse-transformed in shared memory (conjugate -> forward
// FFT -> conjugate, real part, 1/n, window) and added into the CTA's accumulator in
// ascending frame order; outputs are divided by the summed squared window.
constexpr int kOlaHops = 8;

__global__ void __launch_bounds__(512)
    k_istft_ola(const float2 *__restrict__ z, float *__restrict__ out, int N, int F, int n,
                int bits, int hop, const float *__restrict__ window,
                const float2 *__restrict__ tw, int64_t start, int64_t length, int j_first) {
  extern __shared__ float2 sbuf[];
  float *acc = (float *)(sbuf + n);
  const int64_t r = blockIdx.y;
  const int j0 = j_first + blockIdx.x * kOlaHops;
  const int NF = N + 4;  // two zero pad frames on each side (stft.c:55-60)
  const int span = kOlaHops * hop;
  const int64_t a0 = (int64_t)j0 * hop;
  for (int i = threadIdx.x; i < span; i += blockDim.x) acc[i] = 0.f;
  const float inv_n = 1.0f / (float)n;
  const int frames_per_window = n / hop;
  int f_beg = j0 - frames_per_window + 1;
  if (f_beg < 0) f_beg = 0;
  int f_end = j0 + kOlaHops - 1;
  if (f_end > NF - 1) f_end = NF - 1;
  for (int f = f_beg; f <= f_end; f++) {
    const int fi = f - 2;
    if (fi < 0 || fi >= N) continue;  // pad frame: contributes zero
    const float2 *zr = z + ((int64_t)r * N + fi) * F;
    __syncthreads();  // previous frame's accumulate finished reading sbuf
    for (int k = threadIdx.x; k < n; k += blockDim.x) {
      const int kk = k <= n / 2 ? k : n - k;
      float2 v = kk < F ? zr[kk] : make_float2(0.f, 0.f);
      if (k > n / 2) v.y = -v.y;
      sbuf[(int)(__brev((unsigned)k) >> (32 - bits))] = make_float2(v.x, -v.y);
    }
    fft_smem(sbuf, n, tw);
    const int64_t fpos = (int64_t)f * hop;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const int64_t rel = fpos + i - a0;
      if (rel >= 0 && rel < span) acc[rel] += sbuf[i].x * inv_n * window[i];
    }
  }
  __syncthreads();
  const int64_t out_len = (int64_t)hop * (NF - 1) + n;
  for (int i = threadIdx.x; i < span; i += blockDim.x) {
    const int64_t idx = a0 + i, t = idx - start;
    if (t < 0 || t >= length) continue;
    float den = 0.f;
    if (idx < out_len) {
      int64_t f_hi = idx / hop;
      if (f_hi > NF - 1) f_hi = NF - 1;
      const int64_t f_lo = idx - n + 1 <= 0 ? 0 : (idx - n + hop) / hop;
      for (int64_t f = f_lo; f <= f_hi; f++) {
        const int64_t w = idx - f * hop;
        if (w < 0 || w >= n) continue;
        den += window[w] * window[w];
      }
    }
    out[r * length + t] = den > 0.f ? acc[i] / den : 0.f;
  }
}

// ---------------------------------------------------------------- 4096-point Stockham FFT
// Radix-16 Stockham autosort FFT for n = 4096 with 256 threads: three passes, each thread
// holds 16 points in registers, applies the pass twiddles, does a 16-point DFT (radix 4 x 4)
// and writes back to the same shared buffer after a barrier.  The buffer index is padded by
// one element per 16 so every pass's loads and stores are (nearly) free of bank conflicts,
// and the result comes out in natural order (no bit reversal).
constexpr int kFftN = 4096;
constexpr int kFftThreads = 256;
constexpr int kFftPadded = kFftN + kFftN / 16;

static __device__ __forceinline__ int fpad(int i) { return i + (i >> 4); }
static __device__ __forceinline__ float2 cmulf(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}
// in-place 4-point DFT (forward sign) of (a, b, c, d)
static __device__ __forceinline__ void dft4(float2 &a, float2 &b, float2 &c, float2 &d) {
  const float2 s0 = make_float2(a.x + c.x, a.y + c.y), d0 = make_float2(a.x - c.x, a.y - c.y);
  const float2 s1 = make_float2(b.x + d.x, b.y + d.y), d1 = make_float2(b.x - d.x, b.y - d.y);
  a = make_float2(s0.x + s1.x, s0.y + s1.y);
  c = make_float2(s0.x - s1.x, s0.y - s1.y);
  b = make_float2(d0.x + d1.y, d0.y - d1.x);  // d0 - i d1
  d = make_float2(d0.x - d1.y, d0.y + d1.x);  // d0 + i d1
}
// 16-point forward DFT; on return X[k1 + 4 k2] sits in v[4 k1 + k2]
static __device__ __forceinline__ void dft16(float2 (&v)[16]) {
  // cos / sin of pi/8 and of pi/4
  const float c1 = 0.92387953251128674f, s1 = 0.38268343236508978f, h = 0.70710678118654752f;
#pragma unroll
  for (int n2 = 0; n2 < 4; n2++) dft4(v[n2], v[n2 + 4], v[n2 + 8], v[n2 + 12]);
  // twiddles W16^(n2 k1) at v[n2 + 4 k1]
  v[5] = cmulf(v[5], make_float2(c1, -s1));    // W^1
  v[9] = cmulf(v[9], make_float2(h, -h));      // W^2
  v[13] = cmulf(v[13], make_float2(s1, -c1));  // W^3
  v[6] = cmulf(v[6], make_float2(h, -h));      // W^2
  v[10] = make_float2(v[10].y, -v[10].x);      // W^4 = -i
  v[14] = cmulf(v[14], make_float2(-h, -h));   // W^6
  v[7] = cmulf(v[7], make_float2(s1, -c1));    // W^3
  v[11] = cmulf(v[11], make_float2(-h, -h));   // W^6
  v[15] = cmulf(v[15], make_float2(-c1, s1));  // W^9
#pragma unroll
  for (int k1 = 0; k1 < 4; k1++) dft4(v[4 * k1], v[4 * k1 + 1], v[4 * k1 + 2], v[4 * k1 + 3]);
}
// Pass twiddles of fft4096, laid out [pass][r][k] so that a warp's load of twiddle r for its
// 32 consecutive k falls in one or two 128-byte lines: pass 1 (Ns = 16) holds
// exp(-2 pi i k r / 256) at (r - 1) * 16 + k, pass 2 (Ns = 256) holds exp(-2 pi i k r / 4096)
// at kTwPass2 + (r - 1) * 256 + k, for r = 1..15.
constexpr int kTwPass2 = 15 * 16;
constexpr int kTwEntries = kTwPass2 + 15 * 256;

// forward DFT of buf (padded layout, natural order in and out); tw: the pass tables above
static __device__ __forceinline__ void fft4096(float2 *buf, const float2 *__restrict__ tw) {
  const int j = threadIdx.x;
#pragma unroll
  for (int pass = 0; pass < 3; pass++) {
    const int lg = 4 * pass, Ns = 1 << lg;
    float2 v[16];
#pragma unroll
    for (int r = 0; r < 16; r++) v[r] = buf[fpad(j + 256 * r)];
    const int k = j & (Ns - 1);
    if (pass > 0) {
      const float2 *twp = tw + (pass == 1 ? 0 : kTwPass2) + k;
#pragma unroll
      for (int r = 1; r < 16; r++) v[r] = cmulf(v[r], __ldg(twp + (r - 1) * Ns));
    }
    dft16(v);
    __syncthreads();
    const int idxD = ((j >> lg) << (lg + 4)) + k;
#pragma unroll
    for (int r = 0; r < 16; r++) buf[fpad(idxD + r * Ns)] = v[4 * (r & 3) + (r >> 2)];
    __syncthreads();
  }
}

static float2 *g_tw_full = nullptr;

// exp(-2 pi i e / 4096) for e < 4096, evaluated in double on the host
// fft4096's pass tables, evaluated in double on the host (entry of pass p, r, k:
// exp(-2 pi i e / 4096) with e = k r 4096 / (16 Ns), Ns = 16^p)
static const float2 *twiddles4096() {
  if (g_tw_full) return g_tw_full;
  std::vector<float2> h(kTwEntries);
  for (int pass = 1; pass < 3; pass++) {
    const int Ns = 1 << (4 * pass), base = pass == 1 ? 0 : kTwPass2;
    for (int r = 1; r < 16; r++)
      for (int k = 0; k < Ns; k++) {
        const int e = (k * r) << (8 - 4 * pass);
        const double a = -2.0 * 3.14159265358979323846 * (double)e / (double)kFftN;
        h[base + (r - 1) * Ns + k] = make_float2((float)cos(a), (float)sin(a));
      }
  }
  DCB_CUDA(cudaMalloc(&g_tw_full, kTwEntries * sizeof(float2)));
  DCB_CUDA(cudaMemcpy(g_tw_full, h.data(), kTwEntries * sizeof(float2),
                      cudaMemcpyHostToDevice));
  return g_tw_full;
}

// Hann-windowed STFT frames of sig [R][L] (frame f starts at (frame0 + f) * hop), written
// frame-major: z [R][nframes][nbins] complex (coalesced stores).
__global__ void __launch_bounds__(kFftThreads)
    k_stft_fm(const float *__restrict__ sig, float2 *__restrict__ z, int64_t L, int hop,
              int frame0, int nframes, int nbins, const float *__restrict__ window,
              const float2 *__restrict__ tw) {
  __shared__ float2 buf[kFftPadded];
  const int f = blockIdx.x;
  const int64_t r = blockIdx.y;
  const int64_t start = (int64_t)(frame0 + f) * hop;
  const float *s = sig + r * L;
#pragma unroll
  for (int q = 0; q < 16; q++) {
    const int i = threadIdx.x + 256 * q;
    const int64_t t = start + i;
    buf[fpad(i)] = make_float2(t < L ? s[t] * window[i] : 0.f, 0.f);
  }
  __syncthreads();
  fft4096(buf, tw);
  float2 *out = z + (r * nframes + f) * (int64_t)nbins;
  for (int k = threadIdx.x; k < nbins; k += kFftThreads) out[k] = buf[fpad(k)];
}

// z [R][N][F] complex (frame-major) -> x [B][2C][F][N] normalised per batch, (v - m) / sd
// with sd = sqrt(var) + eps (the spectrogram normalisation of htdemucs.c:152-154)
__global__ void k_fm_to_chw(const float2 *__restrict__ z, float *__restrict__ x,
                            const float *__restrict__ mean, const float *__restrict__ var,
                            int rows_per_b, int F, int N, float eps, int normalise) {
  __shared__ float tre[32][33], tim[32][33];
  const int r = blockIdx.z;
  const int b = r / rows_per_b, q = r - b * rows_per_b;
  const int f0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
  float sd = 1.f, m = 0.f;
  if (normalise) {
    sd = sqrtf(var[b]) + eps;
    m = mean[b];
  }
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int n = n0 + i, f = f0 + threadIdx.x;
    if (f < F && n < N) {
      const float2 v = z[((int64_t)r * N + n) * F + f];
      tre[threadIdx.x][i] = v.x;
      tim[threadIdx.x][i] = v.y;
    }
  }
  __syncthreads();
  float *xre = x + ((int64_t)b * 2 * rows_per_b + 2 * q) * F * (int64_t)N;
  float *xim = xre + (int64_t)F * N;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int f = f0 + i, n = n0 + threadIdx.x;
    if (f < F && n < N) {
      xre[(int64_t)f * N + n] = (tre[i][threadIdx.x] - m) / sd;
      xim[(int64_t)f * N + n] = (tim[i][threadIdx.x] - m) / sd;
    }
  }
}


// inverse STFT for n = 4096, hop 1024, in two passes.  Pass 1: one CTA per (row, pair of
// output frames f, f + 1) inverts both spectra with one complex FFT (Y = X_f + i X_{f+1},
// both Hermitian-extended; IFFT(Y) = conj(FFT(conj(Y))) / n, real part frame f, imaginary
// part frame f + 1) and writes the windowed frames fw[row][f - f_lo][4096].  Output frame f
// uses spectrum frame f - 2 (the two frames of padding of the reference's istft).
__global__ void __launch_bounds__(kFftThreads)
    k_ifft_frames4096(const float2 *__restrict__ z, float *__restrict__ fw, int N, int F,
                      const float *__restrict__ window, const float2 *__restrict__ tw,
                      int f_lo, int nfw) {
  __shared__ float2 buf[kFftPadded];
  constexpr int n = kFftN;
  const int64_t r = blockIdx.y;
  const int f = f_lo + 2 * blockIdx.x;
  const int fa = f - 2, fb = f - 1;
  const bool va = fa >= 0 && fa < N, vb = f + 1 < f_lo + nfw && fb >= 0 && fb < N;
  if (!va && !vb) return;  // pass 2 skips frames without a spectrum
  const float2 *za = z + (r * N + fa) * F;
  const float2 *zb = z + (r * N + fb) * F;
#pragma unroll
  for (int q = 0; q < 16; q++) {
    const int k = threadIdx.x + 256 * q;
    const int kk = k <= n / 2 ? k : n - k;
    float2 a = va && kk < F ? za[kk] : make_float2(0.f, 0.f);
    float2 b = vb && kk < F ? zb[kk] : make_float2(0.f, 0.f);
    if (k > n / 2) {
      a.y = -a.y;
      b.y = -b.y;
    } else if (k == 0) {
      // the reference keeps the real part of a complex IFFT, which drops the DC bin's
      // imaginary part; in the two-frame pairing it would leak into the other frame
      a.y = 0.f;
      b.y = 0.f;
    }
    buf[fpad(k)] = make_float2(a.x - b.y, -(a.y + b.x));
  }
  __syncthreads();
  fft4096(buf, tw);
  const float inv_n = 1.0f / (float)n;
  float *oa = fw + (r * nfw + (f - f_lo)) * (int64_t)n;
  float *ob = oa + n;
#pragma unroll
  for (int q = 0; q < 16; q++) {
    const int i = threadIdx.x + 256 * q;
    const float2 v = buf[fpad(i)];
    const float wi = window[i] * inv_n;
    if (va) oa[i] = v.x * wi;
    if (vb) ob[i] = -v.y * wi;
  }
}

// Pass 2: out[row][t] = sum of the windowed frames covering start + t (frames with a
// spectrum) / sum of the squared window over every frame covering it (the reference's
// window-sum division), for t in [0, length)
__global__ void k_ola_frames4096(const float *__restrict__ fw, float *__restrict__ out,
                                 int64_t R, int N, int NF, const float *__restrict__ window,
                                 int f_lo, int nfw, int64_t start, int64_t length) {
  constexpr int n = kFftN, hop = 1024;
  const int64_t total = R * length;
  const int64_t out_len = (int64_t)hop * (NF - 1) + n;
  DCB_GRID_STRIDE(i, total) {
    const int64_t r = i / length, t = i - r * length, idx = start + t;
    float acc = 0.f, den = 0.f;
    if (idx < out_len) {
      int64_t g_hi = idx / hop;
      if (g_hi > NF - 1) g_hi = NF - 1;
      const int64_t g_lo = idx - n + 1 <= 0 ? 0 : (idx - n + hop) / hop;
      for (int64_t g = g_lo; g <= g_hi; g++) {
        const int64_t w = idx - g * hop;
        if (w < 0 || w >= n) continue;
        den += window[w] * window[w];
        const int64_t fi = g - 2;
        if (fi >= 0 && fi < N && g >= f_lo && g < f_lo + nfw)
          acc += fw[(r * nfw + (g - f_lo)) * (int64_t)n + w];
      }
    }
    out[r * length + t] = den > 0.f ? acc / den : 0.f;
  }
}

// Fused inverse STFT + overlap-add for n = 4096, hop 1024 (the reference's istft with its
// window-sum division): one CTA per (row, run of `hops` consecutive output hops).  The
// CTA inverts the frames covering its hops in ascending order, two real frames per complex
// FFT (as k_ifft_frames4096), adds each windowed frame into a ring of four hop
// accumulators in shared memory, and writes hop g as soon as frame g (its last
// contributor) is in; the three frames before the run are recomputed by the CTA (3 of
// hops + 3 frames), so no frame buffer goes through HBM.  The run length is chosen per
// call (stream_hops) so the CTAs fill whole waves of the GPU.

// The output stage (htdemucs.c:262-279) fused into the streamed inverse STFT: with y set,
// sample t of row r goes to y[r][t - off] (t - off in [0, keep)) as the time branch's
// de-normalised output plus the spectral branch's, xt[r][t - off] (sqrt(var[b]) + eps) +
// mean[b] + istft, b = r / rows; nothing else is written
struct StreamCombine {
  float *y = nullptr;
  const float *xt = nullptr, *mean = nullptr, *var = nullptr;
  int rows = 1;
  int64_t Lt = 0, off = 0, keep = 0;
  float eps = 0.f;
};
int g_stream_istft = 1;  // 0: the two-pass inverse STFT (frames through HBM), for A/B checks

__global__ void __launch_bounds__(kFftThreads, 4)
    k_istft_stream4096(const float2 *__restrict__ z, float *__restrict__ out, int N, int F,
                       int NF, const float *__restrict__ window,
                       const float2 *__restrict__ tw, int64_t start, int64_t length,
                       int g_first, int hops, const StreamCombine cb) {
  // [kFftPadded] FFT buffer, then the ring [4][1024], then 1 / (sum of the squared window
  // over the four frames covering a sample) for the hops whose four frames all exist
  extern __shared__ float2 sbuf[];
  float2 *buf = sbuf;
  float *ring = (float *)(sbuf + kFftPadded);
  float *sinv = ring + 4 * 1024;
  constexpr int n = kFftN, hop = 1024;
  const int64_t r = blockIdx.y;
  const int k0 = g_first + blockIdx.x * hops;  // first output hop of this CTA
  const int k1 = min(k0 + hops, NF + 3);       // hops past NF + 2 hold no samples
  const float inv_n = 1.0f / (float)n;
  for (int i = threadIdx.x; i < 4 * hop; i += kFftThreads) ring[i] = 0.f;
  for (int w = threadIdx.x; w < hop; w += kFftThreads) {
    float den = 0.f;  // ascending frames (i = 3 .. 0), as below
#pragma unroll
    for (int i = 3; i >= 0; i--) {
      const float wv = window[i * hop + w];
      den += wv * wv;
    }
    sinv[w] = den > 0.f ? 1.0f / den : 0.f;
  }
  // the output stage's constants of this row
  const float cb_sd = cb.y ? sqrtf(cb.var[r / cb.rows]) + cb.eps : 0.f;
  const float cb_mu = cb.y ? cb.mean[r / cb.rows] : 0.f;
  int g = k0 - 3 < 0 ? 0 : k0 - 3;
  __syncthreads();
  for (; g < k1; g += 2) {
    // frames g and g + 1 (those past NF - 1 do not exist; spectra of frame g: g - 2)
    const int fa = g - 2, fb = g - 1;
    // (frame g + 1 enters the FFT whenever it has a spectrum, so every frame comes out of
    // the same pair, and rounding, as in k_ifft_frames4096; it is added only inside the run)
    const bool va = g < NF && fa >= 0 && fa < N;
    const bool vb = g + 1 < NF && fb >= 0 && fb < N;
    if (va || vb) {
      const float2 *za = z + (r * N + fa) * F;
      const float2 *zb = z + (r * N + fb) * F;
#pragma unroll
      for (int q = 0; q < 16; q++) {
        const int k = threadIdx.x + 256 * q;
        const int kk = k <= n / 2 ? k : n - k;
        float2 a = va && kk < F ? za[kk] : make_float2(0.f, 0.f);
        float2 b = vb && kk < F ? zb[kk] : make_float2(0.f, 0.f);
        if (k > n / 2) {
          a.y = -a.y;
          b.y = -b.y;
        } else if (k == 0) {
          // the reference keeps the real part of a complex IFFT, which drops the DC bin's
          // imaginary part; in the two-frame pairing it would leak into the other frame
          a.y = 0.f;
          b.y = 0.f;
        }
        buf[fpad(k)] = make_float2(a.x - b.y, -(a.y + b.x));
      }
      __syncthreads();
      fft4096(buf, tw);
    }
    // add frame g (real part) then frame g + 1 (imaginary part), finishing one hop each
#pragma unroll
    for (int e = 0; e < 2; e++) {
      const int ge = g + e;
      if (ge >= k1) break;
      if (e == 0 ? va : vb) {  // (ge < k1 here)
#pragma unroll
        for (int q = 0; q < 16; q++) {
          const int i = threadIdx.x + 256 * q;
          const float2 v = buf[fpad(i)];
          const float x = (e == 0 ? v.x : -v.y) * (window[i] * inv_n);
          ring[(((ge + (i >> 10)) & 3) << 10) + (i & 1023)] += x;
        }
      }
      __syncthreads();
      // hop ge is complete: samples ge * hop + w, divided by the squared-window sum of
      // every frame covering them
      if (ge >= k0) {
        float *slot = ring + ((ge & 3) << 10);
        const bool inner = ge >= 3 && ge <= NF - 1;  // all four frames of the hop exist
        for (int w = threadIdx.x; w < hop; w += kFftThreads) {
          const int64_t idx = (int64_t)ge * hop + w;
          const int64_t t = idx - start;
          if (t >= 0 && t < length) {
            float val;
            if (inner) {
              val = slot[w] * sinv[w];
            } else {
              float den = 0.f;  // ascending frames, as the two-pass overlap-add sums
#pragma unroll
              for (int i = 3; i >= 0; i--) {
                const int gi = ge - i;
                if (gi >= 0 && gi < NF) {
                  const float wv = window[i * hop + w];
                  den += wv * wv;
                }
              }
              val = den > 0.f ? slot[w] / den : 0.f;
            }
            if (cb.y) {
              const int64_t tt = t - cb.off;
              if (tt >= 0 && tt < cb.keep)
                cb.y[r * cb.keep + tt] = fmaf(cb.xt[r * cb.Lt + tt], cb_sd, cb_mu) + val;
            } else {
              out[r * length + t] = val;
            }
          }
          slot[w] = 0.f;
        }
      } else {
        // a hop before the run: only cleared (its other frames belong to the previous CTA)
        float *slot = ring + ((ge & 3) << 10);
        for (int w = threadIdx.x; w < hop; w += kFftThreads) slot[w] = 0.f;
      }
      __syncthreads();
    }
  }
}

static int log2i(int n) {
  int b = 0;
  while ((1 << b) < n) b++;
  return b;
}

// Whether the streamed inverse STFT (k_istft_stream4096) covers a call: n_fft 4096, hop
// 1024, and output samples within the signal's hops
bool ispec_stream_ok(int n_fft, int hop, int N, int64_t start, int64_t length) {
  return n_fft == kFftN && hop == 1024 && g_stream_istft &&
         (start + length - 1) / hop <= (int64_t)N + 6;
}

// Streamed inverse STFT + overlap-add of a frame-major spectrum z [R][N][F] (bins F <=
// 2049; the decoder's F = 2048 leaves the Nyquist bin zero) -> out [R][length], samples
// start .. start + length of the signal (ispec_stream_ok must hold)
void ispec_frames(const float2 *z, float *out, int64_t R, int F, int N, const float *window,
                  int64_t start, int64_t length, const StreamCombine &cb) {
  constexpr int hop = 1024;
  DCB_REQUIRE(R <= 65535 && F <= kFftN / 2 + 1, "ispec: %lld rows, %d bins", (long long)R, F);
  // output frames NF = N + 4 (two of padding on each side); hops covering the samples
  // (the signal ends with hop NF + 2)
  const int NF = N + 4;
  const int g_first = (int)(start / hop);
  const int g_last = (int)((start + length - 1) / hop);
  const size_t sm = (size_t)kFftPadded * sizeof(float2) + 5 * 1024 * sizeof(float);
  static int slots = 0;  // resident CTAs of the whole GPU
  if (!slots) {
    DCB_CUDA(cudaFuncSetAttribute(k_istft_stream4096,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
    int per_sm = 0;
    DCB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_istft_stream4096,
                                                           kFftThreads, sm));
    int dev = 0, nsm = 0;
    DCB_CUDA(cudaGetDevice(&dev));
    DCB_CUDA(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
    slots = (per_sm > 0 ? per_sm : 1) * (nsm > 0 ? nsm : 1);
  }
  // run length: the least waves x (hops + 3 frames) over the possible run counts (a CTA's
  // time is about its frame count; every CTA of a wave runs at once)
  const int total = g_last - g_first + 1;
  int hops = total;
  int64_t best = -1;
  for (int runs = 1; runs <= total; runs++) {
    const int hr = (total + runs - 1) / runs;
    if ((total + hr - 1) / hr != runs) continue;  // same hop count as a smaller run count
    const int64_t waves = ((int64_t)runs * R + slots - 1) / slots;
    const int64_t cost = waves * (hr + 3);
    if (best < 0 || cost < best) {
      best = cost;
      hops = hr;
    }
  }
  const int runs = (total + hops - 1) / hops;
  TraceScope ts(TR_SPECTRAL, 0.0,
                (double)R * N * F * 8.0 + (cb.y ? (double)R * cb.keep * 8.0 : (double)R * length * 4.0),
                R, F, length);
  k_istft_stream4096<<<dim3((unsigned)runs, (unsigned)R), kFftThreads, sm, stream()>>>(
      z, out, N, F, NF, window, twiddles4096(), start, length, g_first, hops, cb);
  DCB_LAUNCHED();
}

// denormalise + inverse STFT + OLA of the decoder output (the engine's _ispec path):
// x [B][2*rows_per_b][F][N] -> out [B*rows_per_b][length]
void ispec_fused(const float *x, float *out, const float *mean, const float *var, int B,
                 int rows_per_b, int F, int N, int n_fft, int hop, const float *window,
                 int64_t start, int64_t length, float eps) {
  const float2 *tw = twiddles(n_fft);
  if (!tw) return;
  const int64_t R = (int64_t)B * rows_per_b;
  DCB_REQUIRE(R <= 65535 && F <= n_fft / 2 + 1, "ispec: %lld rows, %d bins", (long long)R, F);
  float2 *z = nullptr;
  DCB_CUDA(cudaMallocAsync(&z, (size_t)R * N * F * sizeof(float2), stream()));
  dim3 tg((unsigned)((N + 31) / 32), (unsigned)((F + 31) / 32), (unsigned)R);
  {
    TraceScope ts(TR_SPECTRAL, 0.0, 2.0 * R * N * F * 8.0, R, F, N);
    k_spec_frames_major<<<tg, dim3(32, 8), 0, stream()>>>(x, z, mean, var, rows_per_b, F, N,
                                                           eps);
    DCB_LAUNCHED();
  }
  const int j_first = (int)(start / hop);
  const int j_last = (int)((start + length - 1) / hop);
  const int groups = (j_last - j_first + 1 + kOlaHops - 1) / kOlaHops;
  const size_t smem = (size_t)n_fft * sizeof(float2) + (size_t)kOlaHops * hop * sizeof(float);
  static size_t attr = 0;
  if (smem > attr) {
    DCB_CUDA(cudaFuncSetAttribute(k_istft_ola, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)smem));
    attr = smem;
  }
  if (ispec_stream_ok(n_fft, hop, N, start, length)) {
    ispec_frames(z, out, R, F, N, window, start, length, StreamCombine{});
    DCB_CUDA(cudaFreeAsync(z, stream()));
    return;
  }
  if (n_fft == kFftN && hop == 1024) {
    // frames covering [start, start + length): NF = N + 4 output frames in all
    const int NF = N + 4;
    // first frame reaching past start: floor((start - n) / hop) + 1
    const int64_t a = start - n_fft;
    int f_lo = (int)((a >= 0 ? a / hop : -((-a + hop - 1) / hop))) + 1;
    if (f_lo < 0) f_lo = 0;
    int f_hi = (int)((start + length - 1) / hop);
    if (f_hi > NF - 1) f_hi = NF - 1;
    const int nfw = f_hi - f_lo + 1;
    float *fw = nullptr;
    DCB_CUDA(cudaMallocAsync(&fw, (size_t)R * nfw * n_fft * sizeof(float), stream()));
    k_ifft_frames4096<<<dim3((unsigned)((nfw + 1) / 2), (unsigned)R), kFftThreads, 0,
                        stream()>>>(z, fw, N, F, window, twiddles4096(), f_lo, nfw);
    DCB_LAUNCHED();
    k_ola_frames4096<<<grid_for(R * length, 256), 256, 0, stream()>>>(
        fw, out, R, N, NF, window, f_lo, nfw, start, length);
    DCB_LAUNCHED();
    DCB_CUDA(cudaFreeAsync(fw, stream()));
  } else {
    k_istft_ola<<<dim3((unsigned)groups, (unsigned)R), 512, smem, stream()>>>(
        z, out, N, F, n_fft, log2i(n_fft), hop, window, tw, start, length, j_first);
  }
  DCB_LAUNCHED();
  DCB_CUDA(cudaFreeAsync(z, stream()));
}

// HTDemucs _spec + per-segment normalisation (stft.c:29-47, htdemucs.c:152-154): the
// padded signal xc [R = B*C][L] -> x [B][2C][nbins][nframes] normalised; mean/var receive
// the per-batch statistics; mag (optional) receives the unnormalised spectrogram.
void spec_normalised(const float *xc, int B, int C, int64_t L, int n_fft, int hop, int frame0,
                     int nframes, int nbins, const float *window, float *x, float *mean,
                     float *var, float *mag) {
  const int64_t R = (int64_t)B * C;
  DCB_REQUIRE(n_fft == kFftN && R <= 65535, "spec: n_fft %d (this path needs 4096)", n_fft);
  float2 *z = nullptr;
  DCB_CUDA(cudaMallocAsync(&z, (size_t)R * nframes * nbins * sizeof(float2), stream()));
  const double zb = (double)R * nframes * nbins * 8.0;
  {
    TraceScope ts(TR_SPECTRAL, 0.0, (double)R * L * 4.0 + zb, R, nbins, nframes);
    k_stft_fm<<<dim3((unsigned)nframes, (unsigned)R), kFftThreads, 0, stream()>>>(
        xc, z, L, hop, frame0, nframes, nbins, window, twiddles4096());
    DCB_LAUNCHED();
  }
  {
    // the statistics cover the same elements in any order
    TraceScope ts(TR_SPECTRAL, 0.0, zb, R, nbins, nframes);
    row_stats((const float *)z, B, (int64_t)C * nframes * nbins * 2, mean, var);
  }
  dim3 tg((unsigned)((nframes + 31) / 32), (unsigned)((nbins + 31) / 32), (unsigned)R);
  if (mag) {
    TraceScope ts(TR_SPECTRAL, 0.0, 2.0 * zb, R, nbins, nframes);
    k_fm_to_chw<<<tg, dim3(32, 8), 0, stream()>>>(z, mag, mean, var, C, nbins, nframes, 0.f, 0);
    DCB_LAUNCHED();
  }
  {
    TraceScope ts(TR_SPECTRAL, 0.0, 2.0 * zb, R, nbins, nframes);
    k_fm_to_chw<<<tg, dim3(32, 8), 0, stream()>>>(z, x, mean, var, C, nbins, nframes, 1e-5f,
                                                  1);
    DCB_LAUNCHED();
  }
  DCB_CUDA(cudaFreeAsync(z, stream()));
}

}  // namespace dcb

using namespace dcb;

extern "C" {

void dk_stft(const float *sig, float *out, int64_t R, int64_t L, int n_fft, int hop,
             int frame0, int nframes, int nbins, const float *window) {
  if (R <= 0 || nframes <= 0) return;
  const float2 *tw = twiddles(n_fft);
  if (!tw) return;
  DCB_REQUIRE(R <= 65535, "stft: %lld rows", (long long)R);
  dim3 grid((unsigned)nframes, (unsigned)R);
  size_t sm = (size_t)n_fft * sizeof(float2);
  if (sm > 48 * 1024) DCB_CUDA(cudaFuncSetAttribute(k_stft, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
  k_stft<<<grid, 512, sm, stream()>>>(sig, out, L, n_fft, log2i(n_fft), hop, frame0, nframes,
                                      nbins, window, tw);
  DCB_LAUNCHED();
}

void dk_istft_frames(const float *spec, float *frames, int64_t R, int nbins, int nframes,
                     int pad_frames, int n_fft, const float *window) {
  if (R <= 0) return;
  const float2 *tw = twiddles(n_fft);
  if (!tw) return;
  DCB_REQUIRE(R <= 65535, "istft: %lld rows", (long long)R);
  dim3 grid((unsigned)(nframes + 2 * pad_frames), (unsigned)R);
  size_t sm = (size_t)n_fft * sizeof(float2);
  if (sm > 48 * 1024) DCB_CUDA(cudaFuncSetAttribute(k_istft_frames, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
  k_istft_frames<<<grid, 512, sm, stream()>>>(spec, frames, nbins, nframes, pad_frames, n_fft,
                                              log2i(n_fft), window, tw);
  DCB_LAUNCHED();
}

void dk_ola(const float *frames, float *out, int64_t R, int nframes, int n_fft, int hop,
            const float *window, int64_t start, int64_t length) {
  if (R * length <= 0) return;
  k_ola<<<grid_for(R * length, 256), 256, 0, stream()>>>(frames, out, R, nframes, n_fft, hop,
                                                         window, start, length);
  DCB_LAUNCHED();
}

}  // extern "C"
