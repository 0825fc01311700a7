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

static double *g_part = nullptr;
static size_t g_part_cap = 0;

// statistics of B*Fr rows; mean/rstd/var are device arrays of rows entries (var optional)
void rowview_stats(const RowView &v, int B, float eps, float *mean, float *rstd, float *var) {
  const int64_t rows = (int64_t)B * v.Fr;
  const int64_t L = (int64_t)v.C * v.T;
  if (rows <= 0 || L <= 0) return;
  const int nchunks = (int)((L + kGnChunk - 1) / kGnChunk);
  const size_t need = (size_t)rows * nchunks * 3 * sizeof(double);
  if (need > g_part_cap) {
    if (g_part) {
      DCB_CUDA(cudaStreamSynchronize(stream()));
      DCB_CUDA(cudaFree(g_part));
    }
    g_part_cap = need < ((size_t)4 << 20) ? ((size_t)4 << 20) : need * 2;
    DCB_CUDA(cudaMalloc(&g_part, g_part_cap));
  }
  DCB_REQUIRE(rows <= 65535, "group norm: %lld rows", (long long)rows);
  dim3 grid(nchunks, (unsigned)rows);
  k_rowview_stats<<<grid, kGnThreads, 0, stream()>>>(v, nchunks, g_part);
  DCB_LAUNCHED();
  k_rowview_combine<<<grid_for(rows * 32, 128, 1 << 30), 128, 0, stream()>>>(g_part, rows, nchunks,
                                                                       eps, mean, rstd, var);
  DCB_LAUNCHED();
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

// res[c] += scale[c] * (GN(x)[c] * sigmoid(GN(x)[c + C/2])) for c < C/2 (DConv tail,
// layers.c:38-44); res has C/2 channels with channel stride rsC and the same b/f/t strides
// pattern given by (rsB, rsF).
__global__ void k_gn_glu_res(RowView v, const float *__restrict__ mean,
                             const float *__restrict__ rstd, const float *__restrict__ w,
                             const float *__restrict__ bb, const float *__restrict__ scale,
                             float *__restrict__ res, int64_t rsB, int64_t rsF, int64_t rsC,
                             int B) {
  const int H = v.C / 2;
  const int64_t per = (int64_t)H * v.T, total = (int64_t)B * v.Fr * per;
  DCB_GRID_STRIDE(i, total) {
    const int64_t row = i / per, e = i - row * per;
    const int64_t c = e / v.T, t = e - c * v.T;
    const int64_t b = row / v.Fr, f = row - b * v.Fr;
    const float *xb = v.x + b * v.sB + f * v.sF + t;
    const float m = mean[row], rs = rstd[row];
    const float na = (xb[c * v.sC] - m) * rs * w[c] + bb[c];
    const float nb = (xb[(c + H) * v.sC] - m) * rs * w[c + H] + bb[c + H];
    const float g = na * sigmoid_f(nb);
    float *rp = res + b * rsB + f * rsF + c * rsC + t;
    *rp = *rp + g * scale[c];
  }
}

// GroupNorm(1) of one strided row per CTA, fused with its consumer (DConv,
// layers.c:31-44): statistics over the row's C x T elements in double (sum and sum of
// squares; the reference's two passes in double agree to ~1e-15 for these magnitudes),
// then a second pass over the now L2-resident row applies
//   mode 0:  y = GELU(GN(x))                            (same layout as x, in place allowed)
//   mode 1:  res[c] += scale[c] * GN(x)[c] * sigmoid(GN(x)[c + C/2]),  c < C/2
constexpr int kGnFusedThreads = 256;

template <int MODE>
__global__ void __launch_bounds__(kGnFusedThreads)
    k_gn_fused(RowView v, float *__restrict__ y, const float *__restrict__ w,
               const float *__restrict__ bb, const float *__restrict__ scale, int64_t rsB,
               int64_t rsF, int64_t rsC, float eps) {
  __shared__ double sh[2][kGnFusedThreads / 32];
  const int64_t row = blockIdx.x;
  const int64_t b = row / v.Fr, f = row - b * v.Fr;
  const float *xr = v.x + b * v.sB + f * v.sF;
  double s = 0.0, ss = 0.0;
  for (int c = 0; c < v.C; c++) {
    const float *xc = xr + c * v.sC;
    for (int t = threadIdx.x; t < v.T; t += kGnFusedThreads) {
      const double a = (double)xc[t];
      s += a;
      ss += a * a;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    ss += __shfl_xor_sync(0xffffffffu, ss, o);
  }
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
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
  const double n = (double)v.C * v.T;
  const double md = s / n;
  double vd = ss / n - md * md;
  if (vd < 0.0) vd = 0.0;
  const float m = (float)md;
  const float rs = 1.0f / sqrtf((float)vd + eps);
  if (MODE == 0) {
    float *yr = y + b * v.sB + f * v.sF;
    for (int c = 0; c < v.C; c++) {
      const float *xc = xr + c * v.sC;
      float *yc = yr + c * v.sC;
      const float wc = w[c], bc = bb[c];
      for (int t = threadIdx.x; t < v.T; t += kGnFusedThreads)
        yc[t] = gelu_f((xc[t] - m) * rs * wc + bc);
    }
  } else {
    const int H = v.C / 2;
    float *rr = y + b * rsB + f * rsF;
    for (int c = 0; c < H; c++) {
      const float *xa = xr + c * v.sC, *xb = xr + (c + H) * v.sC;
      float *rc = rr + c * rsC;
      const float wa = w[c], ba = bb[c], wb = w[c + H], bbv = bb[c + H], sc = scale[c];
      for (int t = threadIdx.x; t < v.T; t += kGnFusedThreads) {
        const float na = (xa[t] - m) * rs * wa + ba;
        const float nb = (xb[t] - m) * rs * wb + bbv;
        rc[t] = rc[t] + na * sigmoid_f(nb) * sc;
      }
    }
  }
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
                     int C2, float *__restrict__ zmean, float *__restrict__ zrstd) {
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
  // one warp per entry: the hid (hid + 1) / 2 upper Gram entries, then the hid sums
  const double *G = zc, *u = zc + hid * hid, *vv = u + hid;
  const int npair = hid * (hid + 1) / 2;
  double psum = 0.0, psq = 0.0;
  for (int p = wid; p < npair + hid; p += kGnFusedThreads / 32) {
    int j, k;
    if (p < npair) {
      j = 0;
      int q = p;
      while (q >= hid - j) {
        q -= hid - j;
        j++;
      }
      k = j + q;
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
// (transformer.c:164-185); one warp per token, C <= 1024.  Fr = 1 gives the time branch
// ([B, C, T2] -> [B, T2, C]).
__global__ void k_tokens_ln_pos(const float *__restrict__ x, float *__restrict__ tok,
                                const float *__restrict__ w, const float *__restrict__ bb,
                                const float *__restrict__ pos, int B, int C, int Fr, int T1,
                                float eps) {
  const int64_t ntok = (int64_t)Fr * T1;
  const int64_t gt = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (gt >= (int64_t)B * ntok) return;
  const int64_t b = gt / ntok, tk = gt - b * ntok;
  const int64_t t = tk / Fr, f = tk - t * Fr;
  const float *xb = x + b * (int64_t)C * Fr * T1 + f * T1 + t;
  const int64_t sc = (int64_t)Fr * T1;
  float v[32];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 32; i++) {
    const int c = i * 32 + lane;
    v[i] = c < C ? xb[c * sc] : 0.f;
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
  float *o = tok + gt * C;
  const float *pp = pos + tk * C;
#pragma unroll
  for (int i = 0; i < 32; i++) {
    const int c = i * 32 + lane;
    if (c < C) o[c] = ((v[i] - m) * rs * w[c] + bb[c]) + pp[c];
  }
}

// tok [B, Fr*T1, C] (token t*Fr + f) -> x [B, C, Fr, T1]
__global__ void k_tokens_to_chw(const float *__restrict__ tok, float *__restrict__ x, int B,
                                int C, int Fr, int T1) {
  const int64_t total = (int64_t)B * C * Fr * T1;
  DCB_GRID_STRIDE(i, total) {
    const int64_t t = i % T1, r = i / T1, f = r % Fr, r2 = r / Fr, c = r2 % C, b = r2 / C;
    x[i] = tok[(b * (int64_t)Fr * T1 + t * Fr + f) * C + c];
  }
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

// out[b][src][c][off + t] += y[b][src][c][y0 + t] * w[t], t < n  (apply.c:157-169)
__global__ void k_accumulate(float *out, const float *__restrict__ y,
                             const float *__restrict__ w, int rows, int64_t out_len,
                             int64_t y_len, int64_t off, int64_t y0, int64_t n) {
  const int64_t total = (int64_t)rows * n;
  DCB_GRID_STRIDE(i, total) {
    const int64_t t = i % n, r = i / n;
    out[r * out_len + off + t] += y[r * y_len + y0 + t] * w[t];
  }
}

// y = x * s[t] (final division by the summed transition weights)
// x[r][t] *= 1 / sum_i w[t - off_i] over the segments i covering t (offsets i * stride,
// i < noff): the weight normalisation of dc_apply_model (apply.c:295-300), summed in fp64
// in segment order as the reference does, without a host-side weight-sum array.
__global__ void k_scale_ola(float *x, const float *__restrict__ w, int64_t rows, int64_t L,
                            int seg, int stride, int noff) {
  DCB_GRID_STRIDE(t, L) {
    const int64_t lo = t < seg ? 0 : (t - seg) / stride + 1;
    int64_t hi = t / stride;
    if (hi > noff - 1) hi = noff - 1;
    double s = 0.0;
    for (int64_t i = lo; i <= hi; i++) s += (double)w[t - i * stride];
    const float inv = s > 0.0 ? (float)(1.0 / s) : 0.0f;
    for (int64_t r = 0; r < rows; r++) x[r * L + t] *= inv;
  }
}

__global__ void k_scale_time(float *x, const float *__restrict__ s, int64_t rows, int64_t L) {
  const int64_t total = rows * L;
  DCB_GRID_STRIDE(i, total) { x[i] = x[i] * s[i % L]; }
}

}  // namespace dcb
