// Memory-bound glue of the model engine: GroupNorm over strided rows (so the DConv of the
// frequency branch runs on [B, C, Fr, T] without the transposes of layers.c:3-20), fused
// GN + GLU + LayerScale residual, token transposes with LayerNorm and positional
// embedding, the frequency embedding, and the final denormalise / combine step.
#include "common.cuh"

namespace dcb {

// A "row" r = (b, f) of a [B, C, Fr, T]-like tensor: element (c, t) lives at
// b * sB + f * sF + c * sC + t.
struct RowView {
  const float *x;
  int Fr;
  int64_t sB, sF, sC;
  int C, T;
};

constexpr int kGnChunk = 8192;
constexpr int kGnThreads = 256;

template <typename Tv>
static __device__ __forceinline__ Tv blk_sum(Tv v, Tv *sh) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  Tv r = 0;
  for (int i = 0; i < (int)(blockDim.x >> 5); i++) r += sh[i];
  return r;
}

// two-pass statistics of one chunk of one row -> (count, mean, M2) partial in double
__global__ void __launch_bounds__(kGnThreads)
    k_rowview_stats(RowView v, int nchunks, double *partial) {
  __shared__ double sh[kGnThreads / 32];
  const int64_t row = blockIdx.y;
  const int chunk = blockIdx.x;
  const int64_t L = (int64_t)v.C * v.T;
  const int64_t e0 = (int64_t)chunk * kGnChunk;
  const int64_t n = L - e0 < kGnChunk ? L - e0 : kGnChunk;
  const int64_t b = row / v.Fr, f = row - b * v.Fr;
  const float *base = v.x + b * v.sB + f * v.sF;
  constexpr int PER = kGnChunk / kGnThreads;
  float val[PER];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < PER; i++) {
    const int64_t j = (int64_t)i * kGnThreads + threadIdx.x;
    float t = 0.f;
    if (j < n) {
      const int64_t e = e0 + j;
      const int64_t c = e / v.T, tt = e - c * v.T;
      t = base[c * v.sC + tt];
    }
    val[i] = t;
    s += t;
  }
  const double tot = blk_sum<double>((double)s, sh);
  const double mean = tot / (double)n;
  const float mf = (float)mean;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < PER; i++) {
    const int64_t j = (int64_t)i * kGnThreads + threadIdx.x;
    if (j < n) {
      const float d = val[i] - mf;
      q += d * d;
    }
  }
  double m2 = blk_sum<double>((double)q, sh);
  const double dm = mean - (double)mf;
  m2 -= (double)n * dm * dm;
  if (threadIdx.x == 0) {
    double *o = partial + (row * nchunks + chunk) * 3;
    o[0] = (double)n;
    o[1] = mean;
    o[2] = m2 > 0 ? m2 : 0.0;
  }
}

// Chan merge of the chunk partials -> mean, rstd = 1/sqrt(var + eps) (float, as the
// reference's apply computes it, backend_cpu.c:254)
__global__ void k_rowview_combine(const double *partial, int64_t rows, int nchunks, float eps,
                                  float *mean, float *rstd, float *var) {
  const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (r >= rows) return;
  double n, m, m2;
  warp_merge_row(partial + r * nchunks * 3, nchunks, n, m, m2);
  if ((threadIdx.x & 31) == 0) {
    const float vf = (float)(m2 / n);
    mean[r] = (float)m;
    if (var) var[r] = vf;
    if (rstd) rstd[r] = 1.0f / sqrtf(vf + eps);
  }
}

// statistics of B*Fr rows; mean/rstd/var are device arrays of rows entries (var optional);
// the per-chunk partials live in stream-ordered memory of the call's stream
void rowview_stats(const RowView &v, int B, float eps, float *mean, float *rstd, float *var) {
  const int64_t rows = (int64_t)B * v.Fr;
  const int64_t L = (int64_t)v.C * v.T;
  if (rows <= 0 || L <= 0) return;
  const int nchunks = (int)((L + kGnChunk - 1) / kGnChunk);
  DCB_REQUIRE(rows <= 65535, "group norm: %lld rows", (long long)rows);
  double *part = nullptr;
  DCB_CUDA(cudaMallocAsync(&part, (size_t)rows * nchunks * 3 * sizeof(double), stream()));
  dim3 grid(nchunks, (unsigned)rows);
  k_rowview_stats<<<grid, kGnThreads, 0, stream()>>>(v, nchunks, part);
  DCB_LAUNCHED();
  k_rowview_combine<<<grid_for(rows * 32, 128, 1 << 30), 128, 0, stream()>>>(part, rows, nchunks,
                                                                       eps, mean, rstd, var);
  DCB_LAUNCHED();
  DCB_CUDA(cudaFreeAsync(part, stream()));
}

// y = GELU(GN(x)) in the same strided layout (x and y share strides)
__global__ void k_gn_gelu(RowView v, float *__restrict__ y, const float *__restrict__ mean,
                          const float *__restrict__ rstd, const float *__restrict__ w,
                          const float *__restrict__ bb, int B) {
  const int64_t per = (int64_t)v.C * v.T, total = (int64_t)B * v.Fr * per;
  DCB_GRID_STRIDE(i, total) {
    const int64_t row = i / per, e = i - row * per;
    const int64_t c = e / v.T, t = e - c * v.T;
    const int64_t b = row / v.Fr, f = row - b * v.Fr;
    const int64_t off = b * v.sB + f * v.sF + c * v.sC + t;
    const float n = (v.x[off] - mean[row]) * rstd[row] * w[c] + bb[c];
    y[off] = gelu_f(n);
  }
}


// threads of the one-CTA-per-row GroupNorm kernels
constexpr int kGnFusedThreads = 256;

// Upper-triangle entry p of a hid x hid Gram matrix -> (j, k), j <= k, in the order
// (0,0), (0,1), .., (0,hid-1), (1,1), ..: entry (j, j) is at j hid - j (j - 1) / 2, so j is
// the root of that quadratic (fp32 estimate, corrected by at most a step either way).
static __device__ __forceinline__ void gram_pair(int p, int hid, int &j, int &k) {
  const float b = 2.0f * (float)hid + 1.0f;
  int jj = (int)((b - sqrtf(fmaxf(b * b - 8.0f * (float)p, 0.f))) * 0.5f);
  if (jj < 0) jj = 0;
  if (jj > hid - 1) jj = hid - 1;
  while (jj > 0 && jj * hid - jj * (jj - 1) / 2 > p) jj--;
  while (jj + 1 < hid && (jj + 1) * hid - (jj + 1) * jj / 2 <= p) jj++;
  j = jj;
  k = jj + (p - (jj * hid - jj * (jj - 1) / 2));
}

// DConv hidden rows (layers.c:24-53, the freq branch viewed as B*Fr rows [hid][T]):
// GroupNorm(1) + GELU in place, one CTA per row, and the GroupNorm(1) statistics of the
// row's next 1x1 conv output z = W16 . fp16(h) + b without forming z.  With S_j the sums
// and Q the Gram matrix of fp16(h) over t, and zc = {G = W16^T W16, u = column sums of
// W16, v = W16^T b, sum b, sum b^2} (fp64):
//   sum z   = T sum(b) + u . S
//   sum z^2 = <G, Q> + 2 v . S + T sum(b^2)
// zmean / zrstd receive the mean and 1 / sqrt(var + eps) of z over its C2 * T values.
__global__ void __launch_bounds__(kGnFusedThreads)
    k_gn_gelu_zstats(RowView v, float *__restrict__ y, const float *__restrict__ w,
                     const float *__restrict__ bb, float eps, const double *__restrict__ zc,
                     int C2, float *__restrict__ zmean, float *__restrict__ zrstd,
                     uint16_t *__restrict__ h16, int hidp) {
  extern __shared__ float hs[];  // [hid][T]: fp16-rounded GELU outputs of this row
  __shared__ double sh[2][kGnFusedThreads / 32];
  const int64_t row = blockIdx.x;
  const int64_t b = row / v.Fr, f = row - b * v.Fr;
  const float *xr = v.x + b * v.sB + f * v.sF;
  const int hid = v.C, T = v.T;
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
  double s = 0.0, ss = 0.0;
  for (int c = 0; c < hid; c++) {
    const float *xc = xr + c * v.sC;
    for (int t = threadIdx.x; t < T; t += kGnFusedThreads) {
      const double a = (double)xc[t];
      s += a;
      ss += a * a;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    ss += __shfl_xor_sync(0xffffffffu, ss, o);
  }
  if (lane == 0) {
    sh[0][wid] = s;
    sh[1][wid] = ss;
  }
  __syncthreads();
  s = 0.0;
  ss = 0.0;
  for (int i = 0; i < kGnFusedThreads / 32; i++) {
    s += sh[0][i];
    ss += sh[1][i];
  }
  const double n = (double)hid * T;
  const double md = s / n;
  double vd = ss / n - md * md;
  if (vd < 0.0) vd = 0.0;
  const float m = (float)md;
  const float rs = 1.0f / sqrtf((float)vd + eps);
  float *yr = y + b * v.sB + f * v.sF;
  for (int c = 0; c < hid; c++) {
    const float *xc = xr + c * v.sC;
    float *yc = yr + c * v.sC;
    const float wc = w[c], bc = bb[c];
    for (int t = threadIdx.x; t < T; t += kGnFusedThreads) {
      const float h = gelu_f((xc[t] - m) * rs * wc + bc);
      yc[t] = h;
      hs[c * T + t] = __half2float(__float2half_rn(h));
    }
  }
  __syncthreads();  // every thread has read sh[] and written hs[]
  // fp16 channels-last copy of the row (the 1x1 conv's A operand): h16[(row T + t) hidp + c],
  // channels hid..hidp-1 zero
  if (h16) {
    for (int t = threadIdx.x; t < T; t += kGnFusedThreads) {
      uint16_t *dst = h16 + ((int64_t)row * T + t) * hidp;
      for (int c8 = 0; c8 < hidp; c8 += 8) {
        float q[8];
#pragma unroll
        for (int k = 0; k < 8; k++) q[k] = c8 + k < hid ? hs[(c8 + k) * T + t] : 0.f;
        *(uint4 *)(dst + c8) = make_uint4(pack_h2(q[0], q[1]), pack_h2(q[2], q[3]),
                                          pack_h2(q[4], q[5]), pack_h2(q[6], q[7]));
      }
    }
  }
  // one warp per entry: the hid (hid + 1) / 2 upper Gram entries, then the hid sums
  const double *G = zc, *u = zc + hid * hid, *vv = u + hid;
  const int npair = hid * (hid + 1) / 2;
  double psum = 0.0, psq = 0.0;
  for (int p = wid; p < npair + hid; p += kGnFusedThreads / 32) {
    int j, k;
    if (p < npair) {
      gram_pair(p, hid, j, k);
    } else {
      j = p - npair;
      k = -1;
    }
    const float *hj = hs + j * T;
    const float *hk = k >= 0 ? hs + k * T : nullptr;
    double acc = 0.0;
    for (int t = lane; t < T; t += 32) acc += (double)(hk ? hj[t] * hk[t] : hj[t]);
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (k >= 0) {
      psq += (j == k ? 1.0 : 2.0) * G[j * hid + k] * acc;
    } else {
      psum += u[j] * acc;
      psq += 2.0 * vv[j] * acc;
    }
  }
  __syncthreads();  // sh[] is reused
  if (lane == 0) {
    sh[0][wid] = psum;
    sh[1][wid] = psq;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double sz = 0.0, szz = 0.0;
    for (int i = 0; i < kGnFusedThreads / 32; i++) {
      sz += sh[0][i];
      szz += sh[1][i];
    }
    const double sb = zc[hid * hid + 2 * hid], sb2 = zc[hid * hid + 2 * hid + 1];
    sz += (double)T * sb;
    szz += (double)T * sb2;
    const double nz = (double)C2 * T;
    const double mz = sz / nz;
    double vz = szz / nz - mz * mz;
    if (vz < 0.0) vz = 0.0;
    zmean[row] = (float)mz;
    zrstd[row] = 1.0f / sqrtf((float)vz + eps);
  }
}

// Sums S_j and upper Gram entries Q_jk (j <= k) of fp16(h) over one chunk of a DConv
// hidden row [hid][T], accumulated in fp64 into acc[row][npair + hid] (npair = hid (hid +
// 1) / 2, the sums last): the statistics of z = W16 . fp16(h) + b for rows too long for
// one CTA.  Block (chunk, row, group of kGramPairs entries); the chunk is staged in shared
// memory [hid][len].
constexpr int kGramChunk = 1024;
constexpr int kGramPairs = 64;  // Gram entries per block (8 per warp)
__global__ void __launch_bounds__(256)
    k_gram_chunk(RowView v, int chunk, double *__restrict__ acc) {
  extern __shared__ float hs[];
  const int64_t row = blockIdx.y;
  const int64_t b = row / v.Fr, f = row - b * v.Fr;
  const int hid = v.C;
  const int64_t t0 = (int64_t)blockIdx.x * chunk;
  const int len = (int)(v.T - t0 < chunk ? v.T - t0 : chunk);
  const float *xr = v.x + b * v.sB + f * v.sF + t0;
  for (int i = threadIdx.x; i < hid * len; i += blockDim.x) {
    const int j = i / len, t = i - j * len;
    hs[j * len + t] = __half2float(__float2half_rn(xr[(int64_t)j * v.sC + t]));
  }
  __syncthreads();
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int npair = hid * (hid + 1) / 2;
  const int p_end = min(npair + hid, (int)(blockIdx.z + 1) * kGramPairs);
  for (int p = blockIdx.z * kGramPairs + wid; p < p_end; p += blockDim.x / 32) {
    int j, k;
    if (p < npair) {
      gram_pair(p, hid, j, k);
    } else {
      j = p - npair;
      k = -1;
    }
    const float *hj = hs + j * len;
    const float *hk = k >= 0 ? hs + k * len : nullptr;
    // products of fp16 values are exact in fp32; a lane's <= 32 terms are summed in fp32,
    // lanes and chunks in fp64
    float a32 = 0.f;
    if (hk) {
      for (int t = lane; t < len; t += 32) a32 = fmaf(hj[t], hk[t], a32);
    } else {
      for (int t = lane; t < len; t += 32) a32 += hj[t];
    }
    double a = (double)a32;
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if (lane == 0) atomicAdd(&acc[row * (npair + hid) + p], a);
  }
}

// z statistics of one DConv row (see k_gn_gelu_zstats) from its accumulated sums and upper
// Gram entries a[npair + hid], by all 256 threads of a CTA: warp w takes the Gram rows j =
// w, w + 8, .., its lanes the entries (j, k >= j), addressed directly (entry (j, k) of the
// upper triangle sits at j hid - j (j - 1) / 2 + k - j); fp64 shuffle and shared-memory
// reduction, thread 0 writes the mean and 1 / sqrt(var + eps) of z over its C2 T values
static __device__ __forceinline__ void zstats_row(const double *__restrict__ a,
                                                  const double *__restrict__ zc, int hid,
                                                  int64_t T, int C2, float eps, float *zmean,
                                                  float *zrstd, double (*red)[8]) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int npair = hid * (hid + 1) / 2;
  const double *G = zc, *u = zc + hid * hid, *vv = u + hid;
  double sz = 0.0, szz = 0.0;
  for (int j = wid; j < hid; j += 8) {
    const int base = j * hid - j * (j - 1) / 2;
    for (int k = j + lane; k < hid; k += 32)
      szz += (k == j ? 1.0 : 2.0) * G[j * hid + k] * __ldcg(a + base + (k - j));
  }
  if (wid == 0) {
    for (int j = lane; j < hid; j += 32) {
      const double sj = __ldcg(a + npair + j);
      sz += u[j] * sj;
      szz += 2.0 * vv[j] * sj;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    sz += __shfl_xor_sync(0xffffffffu, sz, o);
    szz += __shfl_xor_sync(0xffffffffu, szz, o);
  }
  if (lane == 0) {
    red[0][wid] = sz;
    red[1][wid] = szz;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    sz = 0.0;
    szz = 0.0;
    for (int w = 0; w < 8; w++) {
      sz += red[0][w];
      szz += red[1][w];
    }
    sz += (double)T * zc[hid * hid + 2 * hid];
    szz += (double)T * zc[hid * hid + 2 * hid + 1];
    const double nz = (double)C2 * T;
    const double mz = sz / nz;
    double vz = szz / nz - mz * mz;
    if (vz < 0.0) vz = 0.0;
    *zmean = (float)mz;
    *zrstd = 1.0f / sqrtf((float)vz + eps);
  }
}

// GroupNorm statistics of z from the accumulated sums, one CTA of 256 threads per row
__global__ void __launch_bounds__(256)
    k_zstats_final(const double *__restrict__ acc, const double *__restrict__ zc, int hid,
                   int64_t T, int C2, int rows, float eps, float *__restrict__ zmean,
                   float *__restrict__ zrstd) {
  __shared__ double red[2][8];
  const int row = blockIdx.x;
  if (row >= rows) return;
  const int npair = hid * (hid + 1) / 2;
  zstats_row(acc + (int64_t)row * (npair + hid), zc, hid, T, C2, eps, zmean + row,
             zrstd + row, red);
}

// DConv hidden rows [hid][T] after the k3 conv, whose epilogue summed each row's values and
// squares into hstat (layers.c:24-53): GroupNorm(1) + GELU into hg (same layout as the
// input), the fp16 channels-last copy (the 1x1 conv's A operand), and the sums S_j and
// upper Gram entries Q_jk of fp16(h) (the z statistics, see k_gn_gelu_zstats) added into
// acc[row] in fp64.  Block = (chunk of `chunk` positions, row, group of `egroup` Gram
// entries): every block of a chunk forms its GELU outputs in shared memory, the group-0
// block writes them out; a thread sums one entry over a slice of the positions (products of
// fp16 values are exact in fp32, 32 of them are summed in fp32, the rest in fp64).  The
// last block of a row to finish (a counter per row) turns acc[row] into zmean / zrstd.
// hstat, acc and cnt start at zero.
constexpr int kDgThreads = 256;
__global__ void __launch_bounds__(kDgThreads)
    k_dconv_gn_gram(RowView v, float *__restrict__ hg, const float *__restrict__ w,
                    const float *__restrict__ bb, float eps, const double *__restrict__ hstat,
                    double *__restrict__ acc, unsigned *__restrict__ cnt, int chunk, int egroup,
                    const double *__restrict__ zc, int C2, float *__restrict__ zmean,
                    float *__restrict__ zrstd, uint16_t *__restrict__ h16, int hidp) {
  extern __shared__ float hs[];  // [hid][ld]: fp16-rounded GELU outputs of the chunk
  __shared__ double red[2][8];
  __shared__ unsigned s_last;
  const int64_t row = blockIdx.y;
  const int64_t b = row / v.Fr, f = row - b * v.Fr;
  const int hid = v.C, T = v.T;
  const int t0 = blockIdx.x * chunk;
  const int len = T - t0 < chunk ? T - t0 : chunk;
  const int ld = len | 1;  // odd row pitch: threads on consecutive channels hit distinct banks
  const bool writer = blockIdx.z == 0;
  // the row's GroupNorm statistics (same formulas as k_gn_gelu_zstats)
  const double n = (double)hid * T;
  const double md = __ldcg(hstat + 2 * row) / n;
  double vd = __ldcg(hstat + 2 * row + 1) / n - md * md;
  if (vd < 0.0) vd = 0.0;
  const float m = (float)md;
  const float rs = 1.0f / sqrtf((float)vd + eps);
  const int64_t off = b * v.sB + f * v.sF + t0;
  const float *__restrict__ xr = v.x + off;
  float *__restrict__ yr = hg + off;
  // eight elements per thread at a time: their loads are all in flight before the first
  // result is stored (the input and the output are distinct buffers).  Element i of the
  // chunk is (channel i / len, position i % len); a thread steps i by kDgThreads, so its
  // (channel, position) pair advances by subtraction (no division in the loop)
  const int nel = hid * len;
  int cn = 0, tn = (int)threadIdx.x;
  while (tn >= len) {
    tn -= len;
    cn++;
  }
  for (int i0 = 0; i0 < nel; i0 += 8 * kDgThreads) {
    float xv[8];
    int cc[8], tt[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const int i = i0 + k * kDgThreads + (int)threadIdx.x;
      cc[k] = cn;
      tt[k] = tn;
      xv[k] = i < nel ? xr[(int64_t)cn * v.sC + tn] : 0.f;
      tn += kDgThreads;
      while (tn >= len) {
        tn -= len;
        cn++;
      }
    }
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const int i = i0 + k * kDgThreads + (int)threadIdx.x;
      if (i < nel) {
        const int c = cc[k];
        const float h = gelu_f((xv[k] - m) * rs * w[c] + bb[c]);
        if (writer) yr[(int64_t)c * v.sC + tt[k]] = h;
        hs[c * ld + tt[k]] = __half2float(__float2half_rn(h));
      }
    }
  }
  __syncthreads();
  if (writer && h16) {
    for (int t = threadIdx.x; t < len; t += kDgThreads) {
      uint16_t *dst = h16 + (row * T + t0 + t) * hidp;
      for (int c8 = 0; c8 < hidp; c8 += 8) {
        float q[8];
#pragma unroll
        for (int k = 0; k < 8; k++) q[k] = c8 + k < hid ? hs[(c8 + k) * ld + t] : 0.f;
        *(uint4 *)(dst + c8) = make_uint4(pack_h2(q[0], q[1]), pack_h2(q[2], q[3]),
                                          pack_h2(q[4], q[5]), pack_h2(q[6], q[7]));
      }
    }
  }
  // this block's Gram entries [e0, e1), `slices` threads per entry
  const int npair = hid * (hid + 1) / 2, ntot = npair + hid;
  const int e0 = blockIdx.z * egroup;
  const int e1 = e0 + egroup < ntot ? e0 + egroup : ntot;
  const int ne = e1 - e0;
  const int slices = ne >= kDgThreads ? 1 : kDgThreads / ne;
  double *ar = acc + row * ntot;
  if (threadIdx.x < ne * slices) {
    const int p = e0 + (int)threadIdx.x % ne, sl = (int)threadIdx.x / ne;
    int j, k;
    if (p < npair) {
      gram_pair(p, hid, j, k);
    } else {
      j = p - npair;
      k = -1;
    }
    const float *hj = hs + j * ld;
    const float *hk = hs + (k >= 0 ? k : j) * ld;
    const float one = k >= 0 ? 0.f : 1.f;  // sums: hj[t] * 1 (hk = hj, weight 0)
    double a = 0.0;
    for (int tb = sl; tb < len; tb += 32 * slices) {
      // 32 terms of this slice in fp32, four independent chains
      float a4[4] = {0.f, 0.f, 0.f, 0.f};
      const int te = tb + 32 * slices < len ? tb + 32 * slices : len;
      int t = tb;
      for (; t + 3 * slices < te; t += 4 * slices) {
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const float x = hj[t + q * slices];
          a4[q] = fmaf(x, fmaf(hk[t + q * slices], 1.f - one, one), a4[q]);
        }
      }
      for (; t < te; t += slices) a4[0] = fmaf(hj[t], fmaf(hk[t], 1.f - one, one), a4[0]);
      a += (double)((a4[0] + a4[1]) + (a4[2] + a4[3]));
    }
    atomicAdd(ar + p, a);
  }
  // the row's last block: every block's atomics are visible once its count is (the CTA
  // barrier orders this block's atomics before thread 0's fence, which is cumulative, and
  // the fence before the count)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicAdd(cnt + row, 1u) == gridDim.x * gridDim.z - 1 ? 1u : 0u;
  }
  __syncthreads();
  if (s_last) {
    __threadfence();
    zstats_row(ar, zc, hid, T, C2, eps, zmean + row, zrstd + row, red);
  }
}

// Both layers of a frequency-branch DConv (layers.c:24-53) for one row (b, f) of T
// positions per CTA, when the row fits in shared memory (C = 48 or 96, hid = C / 8): the
// row's fp16 channels-last copy stays in shared memory from the first layer's k3 conv to
// the second layer's, and per layer the CTA forms h = conv_k3(fp16 y) + b on CUDA cores
// (products of fp16 values exact in fp32, summed in fp32 as the tensor core does), its
// GroupNorm(1) statistics (fp64), GELU, fp16(h), the z statistics from the sums and Gram
// matrix of fp16(h) (see k_gn_gelu_zstats), and the 1x1 conv + GroupNorm + GLU +
// LayerScale + residual of k_dconv_tail, reading the residual from and writing the result
// to y; the final fp16 copy goes to yh.  Nothing else touches HBM.
struct DconvRowLayer {
  const uint16_t *w0;  // k3 conv weights [hid][ld0], element (o, kw C + c)
  int64_t ld0;
  const float *b0, *g1w, *g1b;  // conv bias, first GroupNorm affine [hid]
  const double *zc;             // z statistics constants (see k_gn_gelu_zstats)
  const uint16_t *w3;           // 1x1 conv [2C][ld3]
  int64_t ld3;
  const float *b3, *g4w, *g4b, *scale;  // [2C], [2C], [2C], [C]
  int dil;
};
struct DconvRowArgs {
  float *y;      // [B][C][Fr][T]
  uint16_t *yh;  // [B][Fr][T][C] fp16 (channels-last, T unpadded)
  int Fr, T;
  int64_t ysB, ysC;  // y strides of b and c
  DconvRowLayer L[2];
};
// 192 threads, each with positions t and t + 192 of the row (rows up to 384 positions); the
// row's fp16 copy in shared memory has a pitch of C + 8 halves (an odd number of 16-byte
// units), so a warp's 16-byte loads of 32 consecutive positions hit distinct banks
constexpr int kDrThreads = 192;
constexpr int kDrMaxT = 2 * kDrThreads;

template <int C, int HID, int HIDP>
__global__ void __launch_bounds__(kDrThreads, 4)
    k_dconv_rows(const DconvRowArgs a) {
  static_assert(HIDP % 4 == 0 && HIDP >= HID && C % 8 == 0, "k_dconv_rows shape");
  constexpr int NPAIR = HID * (HID + 1) / 2, NTOT = NPAIR + HID;
  constexpr int SP = C + 8;  // pitch of the fp16 row copy (halves)
  extern __shared__ __align__(16) uint8_t dsm[];
  const int T = a.T;
  uint16_t *sy = (uint16_t *)dsm;                        // [T][SP] fp16 y of this row
  float *sh = (float *)(dsm + (size_t)T * SP * 2);       // [HID][T] h, then fp16(GELU)
  float *sw0 = sh + (size_t)HID * T;                     // [3][C][HIDP]
  float *sw3 = sw0 + 3 * C * HIDP;                       // [2C][HIDP]
  float *sb3 = sw3 + 2 * C * HIDP;                       // [2C]
  float *sg4w = sb3 + 2 * C, *sg4b = sg4w + 2 * C;       // [2C] each
  float *ssc = sg4b + 2 * C;                             // [C]
  __shared__ double dred[2][kDrThreads / 32];
  __shared__ double dent[kDrThreads];  // Gram partial sums, then the entry totals
  __shared__ float s_par[4];           // GroupNorm mean / rstd, z mean / rstd
  const int row = blockIdx.x;
  const int b = row / a.Fr, f = row - b * a.Fr;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  float *yrow = a.y + (int64_t)b * a.ysB + (int64_t)f * T;  // element (c, t): yrow[c ysC + t]
  uint16_t *yhrow = a.yh + (int64_t)row * T * C;
  // the row's fp16 copy into shared memory (16-byte chunks)
  for (int i = tid; i < T * C / 8; i += kDrThreads) {
    const int t = i / (C / 8), c8 = i - t * (C / 8);
    *(uint4 *)(sy + (size_t)t * SP + 8 * c8) = ((const uint4 *)yhrow)[i];
  }
  for (int l = 0; l < 2; l++) {
    const DconvRowLayer &L = a.L[l];
    // this layer's weights as fp32: k3 conv [kw][c][o], 1x1 conv [c'][j] (o, j padded with 0)
    for (int i = tid; i < 3 * C * HIDP; i += kDrThreads) {
      const int o = i % HIDP, c = (i / HIDP) % C, kw = i / (HIDP * C);
      sw0[i] = o < HID ? h2f_bits(L.w0[(int64_t)o * L.ld0 + kw * C + c]) : 0.f;
    }
    for (int i = tid; i < 2 * C * HIDP; i += kDrThreads) {
      const int j = i % HIDP, c = i / HIDP;
      sw3[i] = j < HID ? h2f_bits(L.w3[(int64_t)c * L.ld3 + j]) : 0.f;
    }
    for (int i = tid; i < 2 * C; i += kDrThreads) {
      sb3[i] = L.b3[i];
      sg4w[i] = L.g4w[i];
      sg4b[i] = L.g4b[i];
      if (i < C) ssc[i] = L.scale[i];
    }
    __syncthreads();
    // h[o][t] = b0[o] + sum over taps kw and channels c of w0[o][kw][c] y[t + (kw - 1) dil][c]
    // for this thread's positions t0 = tid and t1 = tid + kDrThreads (every weight load serves
    // both)
    double s1 = 0.0, s2 = 0.0;
    {
      const int t0 = tid, t1 = tid + kDrThreads;
      const bool v0 = t0 < T, v1 = t1 < T;
      float acc0[HIDP], acc1[HIDP];
#pragma unroll
      for (int o = 0; o < HIDP; o++) {
        const float bo = o < HID ? L.b0[o] : 0.f;
        acc0[o] = bo;
        acc1[o] = bo;
      }
#pragma unroll
      for (int kw = 0; kw < 3; kw++) {
        const int ta = t0 + (kw - 1) * L.dil, tb = t1 + (kw - 1) * L.dil;
        const bool ia = v0 && ta >= 0 && ta < T, ib = v1 && tb >= 0 && tb < T;
        const uint4 *ya = (const uint4 *)(sy + (size_t)(ia ? ta : 0) * SP);
        const uint4 *yb = (const uint4 *)(sy + (size_t)(ib ? tb : 0) * SP);
        const float4 *wp = (const float4 *)(sw0 + (kw * C) * HIDP);
#pragma unroll 1
        for (int c8 = 0; c8 < C / 8; c8++) {
          const uint4 ua = ia ? ya[c8] : make_uint4(0u, 0u, 0u, 0u);
          const uint4 ub = ib ? yb[c8] : make_uint4(0u, 0u, 0u, 0u);
          const uint32_t wa[4] = {ua.x, ua.y, ua.z, ua.w}, wb[4] = {ub.x, ub.y, ub.z, ub.w};
#pragma unroll
          for (int k = 0; k < 8; k++) {
            const float xa = __half2float(__ushort_as_half((uint16_t)(wa[k >> 1] >> (16 * (k & 1)))));
            const float xb = __half2float(__ushort_as_half((uint16_t)(wb[k >> 1] >> (16 * (k & 1)))));
#pragma unroll
            for (int q = 0; q < HIDP / 4; q++) {
              // both positions per instruction (packed FMA, each lane rounds as fmaf)
              const float4 w = wp[(8 * c8 + k) * (HIDP / 4) + q];
              ffma2(acc0[4 * q], acc1[4 * q], w.x, w.x, xa, xb);
              ffma2(acc0[4 * q + 1], acc1[4 * q + 1], w.y, w.y, xa, xb);
              ffma2(acc0[4 * q + 2], acc1[4 * q + 2], w.z, w.z, xa, xb);
              ffma2(acc0[4 * q + 3], acc1[4 * q + 3], w.w, w.w, xa, xb);
            }
          }
        }
      }
#pragma unroll
      for (int o = 0; o < HID; o++) {
        if (v0) {
          sh[o * T + t0] = acc0[o];
          s1 += (double)acc0[o];
          s2 += (double)acc0[o] * acc0[o];
        }
        if (v1) {
          sh[o * T + t1] = acc1[o];
          s1 += (double)acc1[o];
          s2 += (double)acc1[o] * acc1[o];
        }
      }
    }
    // GroupNorm(1) statistics of h over hid x T (the formulas of k_gn_gelu_zstats)
    for (int o = 16; o > 0; o >>= 1) {
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
      s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    }
    if (lane == 0) {
      dred[0][wid] = s1;
      dred[1][wid] = s2;
    }
    __syncthreads();
    if (tid == 0) {
      double t1 = 0.0, t2 = 0.0;
      for (int w = 0; w < kDrThreads / 32; w++) {
        t1 += dred[0][w];
        t2 += dred[1][w];
      }
      const double n = (double)HID * T;
      const double md = t1 / n;
      double vd = t2 / n - md * md;
      if (vd < 0.0) vd = 0.0;
      s_par[0] = (float)md;
      s_par[1] = 1.0f / sqrtf((float)vd + 1e-5f);
    }
    __syncthreads();
    {
      const float m = s_par[0], rs = s_par[1];
      for (int i = tid; i < HID * T; i += kDrThreads) {
        const int o = i / T;
        sh[i] = __half2float(__float2half_rn(gelu_f((sh[i] - m) * rs * L.g1w[o] + L.g1b[o])));
      }
    }
    __syncthreads();
    // sums S_j and upper Gram entries Q_jk of fp16(h): entry e = tid % NTOT over the
    // positions t = slice, slice + slices, ..; 32 terms in fp32, the rest in fp64
    {
      constexpr int SL = kDrThreads / NTOT > 0 ? kDrThreads / NTOT : 1;
      double acc = 0.0;
      if (tid < NTOT * SL) {
        const int e = tid % NTOT, sl = tid / NTOT;
        int j, k;
        if (e < NPAIR) {
          gram_pair(e, HID, j, k);
        } else {
          j = e - NPAIR;
          k = -1;
        }
        const float *hj = sh + j * T, *hk = sh + (k >= 0 ? k : j) * T;
        const float one = k >= 0 ? 0.f : 1.f;
        for (int tb = sl; tb < T; tb += 32 * SL) {
          float a32 = 0.f;
          const int te = tb + 32 * SL < T ? tb + 32 * SL : T;
          for (int t = tb; t < te; t += SL) a32 = fmaf(hj[t], fmaf(hk[t], 1.f - one, one), a32);
          acc += (double)a32;
        }
      }
      dent[tid] = acc;
      __syncthreads();
      if (tid < NTOT) {
        double tot = 0.0;
        for (int sl = 0; sl < SL; sl++) tot += dent[sl * NTOT + tid];
        dent[tid] = tot;  // (slice 0's own slot: only this thread reads and writes it)
      }
      __syncthreads();
      // z statistics (zstats_row's sums, from shared memory)
      const double *G = L.zc, *u = L.zc + HID * HID, *vv = u + HID;
      double sz = 0.0, szz = 0.0;
      for (int e = tid; e < NTOT; e += kDrThreads) {
        if (e < NPAIR) {
          int j, k;
          gram_pair(e, HID, j, k);
          szz += (k == j ? 1.0 : 2.0) * G[j * HID + k] * dent[e];
        } else {
          const int j = e - NPAIR;
          sz += u[j] * dent[e];
          szz += 2.0 * vv[j] * dent[e];
        }
      }
      for (int o = 16; o > 0; o >>= 1) {
        sz += __shfl_xor_sync(0xffffffffu, sz, o);
        szz += __shfl_xor_sync(0xffffffffu, szz, o);
      }
      __syncthreads();  // (every thread has read dred from the previous use)
      if (lane == 0) {
        dred[0][wid] = sz;
        dred[1][wid] = szz;
      }
      __syncthreads();
      if (tid == 0) {
        double z1 = 0.0, z2 = 0.0;
        for (int w = 0; w < kDrThreads / 32; w++) {
          z1 += dred[0][w];
          z2 += dred[1][w];
        }
        z1 += (double)T * L.zc[HID * HID + 2 * HID];
        z2 += (double)T * L.zc[HID * HID + 2 * HID + 1];
        const double nz = (double)(2 * C) * T;
        const double mz = z1 / nz;
        double vz = z2 / nz - mz * mz;
        if (vz < 0.0) vz = 0.0;
        s_par[2] = (float)mz;
        s_par[3] = 1.0f / sqrtf((float)vz + 1e-5f);
      }
      __syncthreads();
    }
    // 1x1 conv + GroupNorm + GLU + LayerScale + residual (k_dconv_tail's arithmetic) for this
    // thread's positions t0 and t1 = t0 + kDrThreads together, 8 channels at a time with the
    // next 8 channels' residuals loaded ahead (the residual loads are the tail's latency);
    // the fp16 copy of the result into shared memory (the next layer's input) and, after
    // the last layer, to yh
    {
      const float mu = s_par[2], rs = s_par[3];
      const int t0 = tid, t1 = tid + kDrThreads;
      const bool v0 = t0 < T, v1 = t1 < T;
      float h0[HIDP], h1[HIDP];
#pragma unroll
      for (int j = 0; j < HIDP; j++) {
        h0[j] = j < HID && v0 ? sh[j * T + t0] : 0.f;
        h1[j] = j < HID && v1 ? sh[j * T + t1] : 0.f;
      }
      float *yp0 = yrow + (v0 ? t0 : 0), *yp1 = yrow + (v1 ? t1 : 0);
      float yn0[8], yn1[8];
#pragma unroll
      for (int k = 0; k < 8; k++) {
        yn0[k] = v0 ? yp0[(int64_t)k * a.ysC] : 0.f;
        yn1[k] = v1 ? yp1[(int64_t)k * a.ysC] : 0.f;
      }
#pragma unroll 1
      for (int c0 = 0; c0 < C; c0 += 8) {
        float y0[8], y1[8];
#pragma unroll
        for (int k = 0; k < 8; k++) {
          y0[k] = yn0[k];
          y1[k] = yn1[k];
        }
        if (c0 + 8 < C) {
#pragma unroll
          for (int k = 0; k < 8; k++) {
            yn0[k] = v0 ? yp0[(int64_t)(c0 + 8 + k) * a.ysC] : 0.f;
            yn1[k] = v1 ? yp1[(int64_t)(c0 + 8 + k) * a.ysC] : 0.f;
          }
        }
        float n0[8], n1[8];
#pragma unroll
        for (int k = 0; k < 8; k++) {
          const int c = c0 + k;
          const float4 *wa = (const float4 *)(sw3 + c * HIDP);
          const float4 *wb = (const float4 *)(sw3 + (C + c) * HIDP);
          float x0 = 0.f, g0 = 0.f, x1 = 0.f, g1 = 0.f;
#pragma unroll
          for (int j = 0; j < HIDP / 4; j++) {
            // the GLU's two halves per instruction (packed FMA, each lane rounds as fmaf)
            const float4 p = wa[j], z = wb[j];
            ffma2(x0, g0, p.x, z.x, h0[4 * j], h0[4 * j]);
            ffma2(x0, g0, p.y, z.y, h0[4 * j + 1], h0[4 * j + 1]);
            ffma2(x0, g0, p.z, z.z, h0[4 * j + 2], h0[4 * j + 2]);
            ffma2(x0, g0, p.w, z.w, h0[4 * j + 3], h0[4 * j + 3]);
            ffma2(x1, g1, p.x, z.x, h1[4 * j], h1[4 * j]);
            ffma2(x1, g1, p.y, z.y, h1[4 * j + 1], h1[4 * j + 1]);
            ffma2(x1, g1, p.z, z.z, h1[4 * j + 2], h1[4 * j + 2]);
            ffma2(x1, g1, p.w, z.w, h1[4 * j + 3], h1[4 * j + 3]);
          }
          x0 = (x0 + sb3[c] - mu) * rs * sg4w[c] + sg4b[c];
          g0 = (g0 + sb3[C + c] - mu) * rs * sg4w[C + c] + sg4b[C + c];
          x1 = (x1 + sb3[c] - mu) * rs * sg4w[c] + sg4b[c];
          g1 = (g1 + sb3[C + c] - mu) * rs * sg4w[C + c] + sg4b[C + c];
          n0[k] = y0[k] + ssc[c] * (x0 * __fdividef(1.0f, 1.0f + __expf(-g0)));
          n1[k] = y1[k] + ssc[c] * (x1 * __fdividef(1.0f, 1.0f + __expf(-g1)));
        }
        if (v0) {
#pragma unroll
          for (int k = 0; k < 8; k++) yp0[(int64_t)(c0 + k) * a.ysC] = n0[k];
          const uint4 q0 = make_uint4(pack_h2(n0[0], n0[1]), pack_h2(n0[2], n0[3]),
                                      pack_h2(n0[4], n0[5]), pack_h2(n0[6], n0[7]));
          *(uint4 *)(sy + (size_t)t0 * SP + c0) = q0;
          if (l == 1) *(uint4 *)(yhrow + (size_t)t0 * C + c0) = q0;
        }
        if (v1) {
#pragma unroll
          for (int k = 0; k < 8; k++) yp1[(int64_t)(c0 + k) * a.ysC] = n1[k];
          const uint4 q1 = make_uint4(pack_h2(n1[0], n1[1]), pack_h2(n1[2], n1[3]),
                                      pack_h2(n1[4], n1[5]), pack_h2(n1[6], n1[7]));
          *(uint4 *)(sy + (size_t)t1 * SP + c0) = q1;
          if (l == 1) *(uint4 *)(yhrow + (size_t)t1 * C + c0) = q1;
        }
      }
    }
    __syncthreads();
  }
}

// DConv tail on CUDA cores for small hidden widths (layers.c:24-53, hid = C / 8 <= 24):
// y[c] += scale[c] * GLU(GroupNorm(W16 . fp16(h) + b)) per position, with the GroupNorm
// statistics of each row (b, f) precomputed.  A 1x1 conv of K = hid is a handful of MACs
// per output, too few for a tensor-core tile; here one thread per position keeps fp16(h)
// in registers and reads the weights [2C][HIDP] as fp32 from shared memory (broadcast).
// Products of fp16 values are exact in fp32 and summed in fp32, as the tensor cores do.
template <int HIDP>
__global__ void __launch_bounds__(256)
    k_dconv_tail(const float *__restrict__ h, float *__restrict__ y, const uint16_t *__restrict__ w16,
                 int64_t ldw, const float *__restrict__ bias, const float *__restrict__ gw,
                 const float *__restrict__ gb, const float *__restrict__ scale,
                 const float *__restrict__ zmean, const float *__restrict__ zrstd, int B, int C,
                 int hid, int Fr, int64_t T, int64_t hsB, int64_t hsC, int64_t ysB,
                 int64_t ysC, uint16_t *__restrict__ yh, int64_t yh_pitch) {
  extern __shared__ float sm[];
  float *sw = sm;                    // [2C][HIDP]
  float *sbias = sw + 2 * C * HIDP;  // [2C]
  float *sgw = sbias + 2 * C;        // [2C]
  float *sgb = sgw + 2 * C;          // [2C]
  float *ssc = sgb + 2 * C;          // [C]
  for (int i = threadIdx.x; i < 2 * C * HIDP; i += blockDim.x) {
    const int c = i / HIDP, j = i - c * HIDP;
    sw[i] = j < hid ? h2f_bits(w16[(int64_t)c * ldw + j]) : 0.f;
  }
  for (int i = threadIdx.x; i < 2 * C; i += blockDim.x) {
    sbias[i] = bias[i];
    sgw[i] = gw[i];
    sgb[i] = gb[i];
    if (i < C) ssc[i] = scale[i];
  }
  __syncthreads();
  const int64_t total = (int64_t)B * Fr * T;
  for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < total;
       p += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = p / T, t = p - row * T;
    const int64_t b = row / Fr, f = row - b * Fr;
    const float mu = zmean[row], rs = zrstd[row];
    const float *hp = h + b * hsB + f * T + t;
    float hv[HIDP];
#pragma unroll
    for (int j = 0; j < HIDP; j++)
      hv[j] = j < hid ? __half2float(__float2half_rn(hp[(int64_t)j * hsC])) : 0.f;
    float *yp = y + b * ysB + f * T + t;
    // fp16 channels-last copy of the updated row: yh[(row * yh_pitch + t) * C + c]
    uint16_t *yhp = yh ? yh + ((int64_t)row * yh_pitch + t) * C : nullptr;
    // 8 channels per step: their residual loads are issued together (C % 8 == 0), one
    // step ahead of the step that uses them
    float yn[8];
#pragma unroll
    for (int k = 0; k < 8; k++) yn[k] = yp[(int64_t)k * ysC];
    for (int c0 = 0; c0 < C; c0 += 8) {
      float yv[8];
#pragma unroll
      for (int k = 0; k < 8; k++) yv[k] = yn[k];
      if (c0 + 8 < C) {
#pragma unroll
        for (int k = 0; k < 8; k++) yn[k] = yp[(int64_t)(c0 + 8 + k) * ysC];
      }
      float nv[8];
#pragma unroll
      for (int k = 0; k < 8; k++) {
        const int c = c0 + k;
        const float4 *wa = (const float4 *)(sw + c * HIDP);
        const float4 *wb = (const float4 *)(sw + (C + c) * HIDP);
        float a = 0.f, g = 0.f;
#pragma unroll
        for (int j = 0; j < HIDP / 4; j++) {
          const float4 x = wa[j], z = wb[j];
          a = fmaf(x.x, hv[4 * j], a);
          a = fmaf(x.y, hv[4 * j + 1], a);
          a = fmaf(x.z, hv[4 * j + 2], a);
          a = fmaf(x.w, hv[4 * j + 3], a);
          g = fmaf(z.x, hv[4 * j], g);
          g = fmaf(z.y, hv[4 * j + 1], g);
          g = fmaf(z.z, hv[4 * j + 2], g);
          g = fmaf(z.w, hv[4 * j + 3], g);
        }
        a = (a + sbias[c] - mu) * rs * sgw[c] + sgb[c];
        g = (g + sbias[C + c] - mu) * rs * sgw[C + c] + sgb[C + c];
        nv[k] = yv[k] + ssc[c] * (a * __fdividef(1.0f, 1.0f + __expf(-g)));
      }
#pragma unroll
      for (int k = 0; k < 8; k++) yp[(int64_t)(c0 + k) * ysC] = nv[k];
      if (yhp)
        *(uint4 *)(yhp + c0) = make_uint4(pack_h2(nv[0], nv[1]), pack_h2(nv[2], nv[3]),
                                          pack_h2(nv[4], nv[5]), pack_h2(nv[6], nv[7]));
    }
  }
}

// x[b][c][f][t] += emb[f][c] * alpha   (dc_add_freq_emb, htdemucs.c:114-134)
__global__ void k_add_freq_emb(float *x, const float *__restrict__ emb, float alpha, int B,
                               int C, int Fr, int T, int emb_cols) {
  const int64_t total = (int64_t)B * C * Fr * T;
  DCB_GRID_STRIDE(i, total) {
    const int64_t r = i / T, f = r % Fr, c = (r / Fr) % C;
    x[i] = x[i] + emb[f * emb_cols + c] * alpha;
  }
}

// tokens: x [B, C, Fr, T1] -> tok[b][t*Fr + f][c] = LN(x[b, :, f, t]) + pos[t*Fr + f][c]
// (transformer.c:164-185), C <= 1024.  Fr = 1 gives the time branch ([B, C, T2] ->
// [B, T2, C]).  CTA = kTokT consecutive t of one (b, f): its warps read the tile channel
// by channel (128-byte rows along t) into shared memory [C][kTokT + 1] (odd pitch: both
// the row writes and the per-token column reads are free of bank conflicts), then one warp
// per token normalises it (lane sums over channels c = 32 i + lane, then a shuffle tree)
// and writes the token's row contiguously.
constexpr int kTokT = 32;
__global__ void __launch_bounds__(256)
    k_tokens_ln_pos(const float *__restrict__ x, float *__restrict__ tok,
                    const float *__restrict__ w, const float *__restrict__ bb,
                    const float *__restrict__ pos, int B, int C, int Fr, int T1, float eps) {
  extern __shared__ float tile[];  // [C][kTokT + 1]
  constexpr int P = kTokT + 1;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int t0 = blockIdx.x * kTokT, f = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int nt = T1 - t0 < kTokT ? T1 - t0 : kTokT;
  const int64_t sc = (int64_t)Fr * T1;
  const float *xb = x + b * (int64_t)C * sc + (int64_t)f * T1 + t0;
  // eight channel rows per warp in flight before the first is stored
  for (int c0 = warp; c0 < C; c0 += 8 * nw) {
    float r[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const int c = c0 + k * nw;
      r[k] = c < C && lane < nt ? xb[c * sc + lane] : 0.f;
    }
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const int c = c0 + k * nw;
      if (c < C) tile[c * P + lane] = r[k];
    }
  }
  __syncthreads();
  const int64_t ntok = (int64_t)Fr * T1;
  for (int j = warp; j < nt; j += nw) {
    const int64_t tk = (int64_t)(t0 + j) * Fr + f;
    float v[32];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 32; i++) {
      const int c = i * 32 + lane;
      v[i] = c < C ? tile[c * P + j] : 0.f;
      s += v[i];
    }
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const double md = (double)s / (double)C;
    const float m = (float)md;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < 32; i++) {
      const int c = i * 32 + lane;
      if (c < C) {
        const float d = v[i] - m;
        q += d * d;
      }
    }
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    const double dm = md - (double)m;
    double m2 = (double)q - (double)C * dm * dm;
    const float var = (float)((m2 > 0 ? m2 : 0.0) / (double)C);
    const float rs = 1.0f / sqrtf(var + eps);
    float *o = tok + (b * ntok + tk) * C;
    const float *pp = pos + tk * C;
#pragma unroll
    for (int i = 0; i < 32; i++) {
      const int c = i * 32 + lane;
      if (c < C) o[c] = ((v[i] - m) * rs * w[c] + bb[c]) + pp[c];
    }
  }
}

// fp32 [n][Cs][H][W] (strides sN, sC, sH, 1; optional addend laid out the same) ->
// fp16 channels-last [n][H][Wp][C], round to nearest even: the A operand of the next conv
// (the reference rounds the same fp32 values in dk_im2col_half).  Channels Cs..C-1 are
// zero (C, a multiple of 8, pads inputs with few channels).  One thread per (position,
// 8 channels).
__global__ void k_to_half_cl(const float *__restrict__ x, const float *__restrict__ add,
                             uint16_t *__restrict__ y, int64_t images, int C, int H, int W,
                             int Wp, int64_t sN, int64_t sC, int64_t sH, int Cs) {
  const int C8 = C / 8;
  const int64_t total = images * H * (int64_t)W * C8;
  DCB_GRID_STRIDE(i, total) {
    const int64_t w = i % W, r = i / W;
    const int c8 = (int)(r % C8);
    const int64_t r2 = r / C8;
    const int64_t h = r2 % H, n = r2 / H;
    const int64_t src = n * sN + (int64_t)c8 * 8 * sC + h * sH + w;
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
      v[k] = 0.f;
      if (c8 * 8 + k < Cs) {
        v[k] = x[src + k * sC];
        if (add) v[k] += add[src + k * sC];
      }
    }
    uint4 *d = (uint4 *)(y + ((n * H + h) * Wp + w) * C + c8 * 8);
    *d = make_uint4(pack_h2(v[0], v[1]), pack_h2(v[2], v[3]), pack_h2(v[4], v[5]),
                    pack_h2(v[6], v[7]));
  }
}

// im2col of a few-channel fp32 input [n][C][H][W] (C <= 8) for an 8-tap conv, as the fp16
// A operand of a 1x1 conv: y[n][ho][wo][tap * 8 + c], round to nearest even; taps along H
// (axis 0: h = ho S - P + tap, w = wo) or along W (axis 1: h = ho, w = wo S - P + tap);
// taps outside the input and channels c >= C are zero (the conv's zero padding).  Threads
// run over positions fastest (coalesced reads), one (position, tap) each.
__global__ void k_im2col8_half(const float *__restrict__ x, uint16_t *__restrict__ y,
                               int64_t images, int C, int H, int W, int Ho, int Wo, int S, int P,
                               int axis) {
  const int64_t npos = images * Ho * (int64_t)Wo;
  const int64_t total = npos * 8;
  DCB_GRID_STRIDE(i, total) {
    const int tap = (int)(i / npos);
    const int64_t pos = i - (int64_t)tap * npos;
    const int64_t wo = pos % Wo, r = pos / Wo;
    const int64_t ho = r % Ho, n = r / Ho;
    const int64_t h = axis == 0 ? ho * S - P + tap : ho;
    const int64_t w = axis == 0 ? wo : wo * S - P + tap;
    float v[8];
    const bool in = h >= 0 && h < H && w >= 0 && w < W;
#pragma unroll
    for (int c = 0; c < 8; c++)
      v[c] = in && c < C ? x[((n * C + c) * H + h) * (int64_t)W + w] : 0.f;
    *(uint4 *)(y + pos * 64 + tap * 8) = make_uint4(pack_h2(v[0], v[1]), pack_h2(v[2], v[3]),
                                                   pack_h2(v[4], v[5]), pack_h2(v[6], v[7]));
  }
}

// tok [B, Fr*T1, C] (token t*Fr + f) -> x [B, C, Fr, T1]: CTA = kTokT consecutive t of one
// (b, f); warps read token rows (contiguous channels) into shared memory [C][kTokT + 1],
// then write channel rows (contiguous t)
__global__ void __launch_bounds__(256)
    k_tokens_to_chw(const float *__restrict__ tok, float *__restrict__ x, int B, int C, int Fr,
                    int T1) {
  extern __shared__ float tile[];  // [C][kTokT + 1]
  constexpr int P = kTokT + 1;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int t0 = blockIdx.x * kTokT, f = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int nt = T1 - t0 < kTokT ? T1 - t0 : kTokT;
  const int64_t ntok = (int64_t)Fr * T1;
  // eight loads per lane in flight before the first is stored
  for (int j = warp; j < nt; j += nw) {
    const float *row = tok + (b * ntok + (int64_t)(t0 + j) * Fr + f) * C;
    for (int c0 = lane; c0 < C; c0 += 8 * 32) {
      float r[8];
#pragma unroll
      for (int k = 0; k < 8; k++) {
        const int c = c0 + 32 * k;
        r[k] = c < C ? row[c] : 0.f;
      }
#pragma unroll
      for (int k = 0; k < 8; k++) {
        const int c = c0 + 32 * k;
        if (c < C) tile[c * P + j] = r[k];
      }
    }
  }
  __syncthreads();
  const int64_t sc = (int64_t)Fr * T1;
  float *xb = x + b * (int64_t)C * sc + (int64_t)f * T1 + t0;
  for (int c = warp; c < C; c += nw)
    if (lane < nt) xb[c * sc + lane] = tile[c * P + lane];
}

// y[b][s][c][t] = xt_denorm + center_trim(xi) with denorm x * (sqrt(var) + eps) + mean per
// batch (htdemucs.c:258-268); xi has length Li >= T, centre-trimmed.
__global__ void k_final_combine(const float *__restrict__ xt, const float *__restrict__ xi,
                                float *__restrict__ y, const float *__restrict__ meant,
                                const float *__restrict__ vart, int B, int64_t per, int T,
                                int Li, int keep, float eps) {
  const int64_t rows_per_b = per / T;
  const int64_t total = (int64_t)B * rows_per_b * keep;
  const int off = (Li - T) / 2;
  DCB_GRID_STRIDE(i, total) {
    const int64_t t = i % keep, r = i / keep, b = r / rows_per_b;
    const float sd = sqrtf(vart[b]) + eps;
    const float a = xt[r * T + t] * sd + meant[b];
    y[i] = a + xi[r * Li + off + t];
  }
}

// segment gather with zero padding: out[b][c][t] = mix[b][c][start + t] or 0 outside
// [0, total) (apply.c:135-154 padded_chunk)
__global__ void k_chunk(const float *__restrict__ mix, float *__restrict__ out, int Bm, int C,
                        int64_t total, int64_t start, int64_t len, int64_t ob_stride) {
  const int64_t n = (int64_t)Bm * C * len;
  DCB_GRID_STRIDE(i, n) {
    const int64_t t = i % len, r = i / len, c = r % C, b = r / C;
    const int64_t s = start + t;
    out[b * ob_stride + c * len + t] = (s >= 0 && s < total) ? mix[(b * C + c) * total + s] : 0.f;
  }
}

// One segment forward of dc_apply_model placed in the final output (see Sched in
// forward.cu): chunk start in the mix, output / view position of its first kept sample,
// centre-trim offset and kept length, and the pass it belongs to.
struct SegItem {
  int64_t start, out0, view0, y0, n;
  int pass;
};

// the items of one forward call, by value in the kernel parameters
struct BatchItems {
  int64_t start[32];  // first mix sample of the item's padded chunk
  int64_t out0[32];   // output position of the item's first kept sample
  int64_t view0[32];  // its position in the item's pass view (weight-sum index)
  int64_t y0[32];     // first kept sample inside the item's model output
  int64_t n[32];      // kept samples
  int noff[32];       // segments of the item's pass
  int cnt;
};

// every item's padded chunk of mix (zeros outside [0, total)) into flat[k][b][c][len]
// (apply.c:135-154 padded_chunk); blockIdx.y = item
__global__ void k_chunk_batch(const float *__restrict__ mix, float *__restrict__ flat, int Bm,
                              int C, int64_t total, int64_t len, BatchItems bi) {
  const int k = blockIdx.y;
  const int64_t n = (int64_t)Bm * C * len;
  float *out = flat + (int64_t)k * n;
  const int64_t start = bi.start[k];
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i % len, r = i / len;
    const int64_t s = start + t;
    out[i] = (s >= 0 && s < total) ? mix[r * total + s] : 0.f;
  }
}

// Inverse of a pass's summed transition weights at view position p: the segments at
// offsets q stride (q < noff) that cover p, summed in fp64 in segment order as
// apply.c:295-300 sums them.
static __device__ __forceinline__ float inv_weight_sum(const float *__restrict__ w, int64_t p,
                                                       int seg, int stride, int noff) {
  const int64_t qlo = p < seg ? 0 : (p - seg) / stride + 1;
  int64_t qhi = p / stride;
  if (qhi > noff - 1) qhi = noff - 1;
  double s = 0.0;
  for (int64_t q = qlo; q <= qhi; q++) s += (double)w[p - q * stride];
  return s > 0.0 ? (float)(1.0 / s) : 0.0f;
}

// win[r][t - lo] += y[k][r][y0_k + u] * w[u] * inv_sum_k(view0_k + u) * scale, u = t - out0_k,
// for every item k of the call that covers output position t in [t0, t1) (accumulate,
// apply.c:157-169; the weight-sum division, apply.c:295-306; the shift average,
// apply.c:203-207), in item order
__global__ void k_accumulate_items(float *win, int64_t ld, int64_t lo,
                                   const float *__restrict__ y, const float *__restrict__ w,
                                   int rows, int64_t y_len, int64_t t0, int64_t t1, int seg,
                                   int stride, float scale, BatchItems bi) {
  DCB_GRID_STRIDE(i, t1 - t0) {
    const int64_t t = t0 + i;
    float *col = win + (t - lo);
    for (int k = 0; k < bi.cnt; k++) {
      const int64_t u = t - bi.out0[k];
      if (u < 0 || u >= bi.n[k]) continue;
      const float cw = w[u] * inv_weight_sum(w, bi.view0[k] + u, seg, stride, bi.noff[k]) * scale;
      const float *yk = y + (int64_t)k * rows * y_len + bi.y0[k] + u;
      for (int r = 0; r < rows; r++) col[r * ld] += yk[(int64_t)r * y_len] * cw;
    }
  }
}

// output windows of the shards (sorted by lo)
struct WinList {
  int64_t lo[64], hi[64];
  int n;
};

// out[r][t] = sum over windows w covering t of wins[w * wstride + r * ld + t - lo_w]
// (zero where none does): the root's overlap-add of the gathered shard outputs
__global__ void k_merge_windows(float *__restrict__ out, int64_t rows, int64_t T,
                                const float *__restrict__ wins, int64_t ld, int64_t wstride,
                                WinList wl) {
  DCB_GRID_STRIDE(t, T) {
    for (int64_t r = 0; r < rows; r++) {
      float acc = 0.f;
      for (int i = 0; i < wl.n; i++)
        if (t >= wl.lo[i] && t < wl.hi[i])
          acc += wins[(int64_t)i * wstride + r * ld + (t - wl.lo[i])];
      out[r * T + t] = acc;
    }
  }
}

}  // namespace dcb
