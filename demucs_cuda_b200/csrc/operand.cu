// GEMM operand preparation and attention helpers of the backend.h ABI
// (backend.h:91-131).  The model engine in this library does not call these (its conv,
// transposed-conv and attention kernels gather operands on the fly); they exist so the
// reference's unchanged ops.c runs on this backend with identical results.
#include "common.cuh"

namespace dcb {

__global__ void k_to_half_rows(const float *__restrict__ x, uint16_t *__restrict__ y,
                               int64_t rows, int64_t C, int64_t Cp) {
  int64_t n = rows * Cp;
  DCB_GRID_STRIDE(i, n) {
    int64_t r = i / Cp, c = i - r * Cp;
    y[i] = c < C ? f2h_bits(x[r * C + c]) : (uint16_t)0;
  }
}

// [b][C][P] fp32 -> [b][P][Cp] fp16 through a 32x32 shared tile
__global__ void k_transpose_to_half(const float *__restrict__ x, uint16_t *__restrict__ y,
                                    int64_t C, int64_t P, int64_t Cp) {
  __shared__ float tile[32][33];
  int64_t b = blockIdx.z;
  int64_t p0 = (int64_t)blockIdx.x * 32, c0 = (int64_t)blockIdx.y * 32;
  const float *xb = x + b * C * P;
  uint16_t *yb = y + b * P * Cp;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    int64_t c = c0 + i, p = p0 + threadIdx.x;
    tile[i][threadIdx.x] = (c < C && p < P) ? xb[c * P + p] : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    int64_t p = p0 + i, c = c0 + threadIdx.x;
    if (p < P && c < Cp) yb[p * Cp + c] = c < C ? f2h_bits(tile[threadIdx.x][i]) : (uint16_t)0;
  }
}

__global__ void k_im2col(const float *__restrict__ x, uint16_t *__restrict__ col, DkConvGeom g,
                         int64_t n0, int64_t nb, int64_t p0, int64_t np) {
  int64_t K = (int64_t)g.KH * g.KW * g.C, plane = (int64_t)g.H * g.W;
  int64_t total = nb * np * g.Kp;
  DCB_GRID_STRIDE(e, total) {
    int64_t k = e % g.Kp, t = e / g.Kp, pi = t % np, bi = t / np;
    float v = 0.f;
    if (k < K) {
      int64_t p = p0 + pi;
      int ho = (int)(p / g.Wo), wo = (int)(p % g.Wo);
      int c = (int)(k % g.C), kk = (int)(k / g.C);
      int kh = kk / g.KW, kw = kk % g.KW;
      int h = ho * g.SH - g.PH + kh * g.DH, w = wo * g.SW - g.PW + kw * g.DW;
      if (h >= 0 && h < g.H && w >= 0 && w < g.W) {
        v = x[(n0 + bi) * g.C * plane + c * plane + (int64_t)h * g.W + w];
      }
    }
    col[e] = f2h_bits(v);
  }
}

__global__ void k_col2im_tr(const float *__restrict__ cols, float *__restrict__ y,
                            const float *__restrict__ bias, int64_t nb, int O, DkConvGeom g) {
  int64_t P = (int64_t)g.H * g.W, M = (int64_t)O * g.KH * g.KW;
  int64_t per = (int64_t)O * g.Ho * g.Wo, total = nb * per;
  DCB_GRID_STRIDE(e, total) {
    int64_t bi = e / per, r = e - bi * per;
    int o = (int)(r / ((int64_t)g.Ho * g.Wo));
    int64_t hw = r - (int64_t)o * g.Ho * g.Wo;
    int ho = (int)(hw / g.Wo), wo = (int)(hw % g.Wo);
    const float *cb = cols + bi * M * P;
    float acc = bias ? bias[o] : 0.f;
    int hf = ho + g.PH, wf = wo + g.PW;
    for (int kh = 0; kh < g.KH; kh++) {
      int hs = hf - kh;
      if (hs < 0 || hs % g.SH) continue;
      int h = hs / g.SH;
      if (h >= g.H) continue;
      for (int kw = 0; kw < g.KW; kw++) {
        int ws = wf - kw;
        if (ws < 0 || ws % g.SW) continue;
        int w = ws / g.SW;
        if (w >= g.W) continue;
        acc += cb[((int64_t)(o * g.KH + kh) * g.KW + kw) * P + (int64_t)h * g.W + w];
      }
    }
    y[e] = acc;
  }
}

// softmax(scale * s) per row -> fp16, pad columns zeroed; one CTA per row
__global__ void k_softmax_to_half(const float *__restrict__ s, int64_t lds,
                                  uint16_t *__restrict__ p, int64_t ldp, int64_t L, float scale) {
  __shared__ float red[32];
  __shared__ double redd[32];
  int64_t r = blockIdx.x;
  const float *row = s + r * lds;
  float mx = -INFINITY;
  for (int64_t j = threadIdx.x; j < L; j += blockDim.x) mx = fmaxf(mx, row[j] * scale);
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (l == 0) red[w] = mx;
  __syncthreads();
  mx = red[0];
  for (int i = 1; i < nw; i++) mx = fmaxf(mx, red[i]);
  double sum = 0.0;
  for (int64_t j = threadIdx.x; j < L; j += blockDim.x) sum += (double)expf(row[j] * scale - mx);
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (l == 0) redd[w] = sum;
  __syncthreads();
  sum = 0.0;
  for (int i = 0; i < nw; i++) sum += redd[i];
  float inv = (float)(1.0 / sum);
  for (int64_t j = threadIdx.x; j < ldp; j += blockDim.x) {
    p[r * ldp + j] = j < L ? f2h_bits(expf(row[j] * scale - mx) * inv) : (uint16_t)0;
  }
}

__global__ void k_split_heads(const float *__restrict__ x, uint16_t *__restrict__ y, int64_t B,
                              int64_t T, int H, int hd, int hdp, int64_t Tp, int transpose) {
  int64_t D = (int64_t)H * hd;
  if (!transpose) {
    int64_t n = B * H * T * hdp;
    DCB_GRID_STRIDE(e, n) {
      int d = (int)(e % hdp);
      int64_t t = (e / hdp) % T, bh = e / (hdp * T);
      int64_t b = bh / H, h = bh % H;
      y[e] = d < hd ? f2h_bits(x[(b * T + t) * D + h * hd + d]) : (uint16_t)0;
    }
  } else {
    int64_t n = B * H * hd * Tp;
    DCB_GRID_STRIDE(e, n) {
      int64_t t = e % Tp, d = (e / Tp) % hd, bh = e / (Tp * hd);
      int64_t b = bh / H, h = bh % H;
      y[e] = t < T ? f2h_bits(x[(b * T + t) * D + h * hd + d]) : (uint16_t)0;
    }
  }
}

}  // namespace dcb

using namespace dcb;

extern "C" {

void dk_to_half_rows(const float *x, dc_half *y, int64_t rows, int64_t C, int64_t Cp) {
  if (rows * Cp <= 0) return;
  k_to_half_rows<<<grid_for(rows * Cp, 256), 256, 0, stream()>>>(x, y, rows, C, Cp);
  DCB_LAUNCHED();
}

void dk_transpose_to_half(const float *x, dc_half *y, int64_t batch, int64_t C, int64_t P,
                          int64_t Cp) {
  if (batch <= 0 || P <= 0) return;
  DCB_REQUIRE(batch <= 65535, "transpose_to_half: batch %lld > 65535", (long long)batch);
  dim3 grid((unsigned)((P + 31) / 32), (unsigned)((Cp + 31) / 32), (unsigned)batch);
  k_transpose_to_half<<<grid, dim3(32, 8), 0, stream()>>>(x, y, C, P, Cp);
  DCB_LAUNCHED();
}

void dk_im2col_half(const float *x, dc_half *col, const DkConvGeom *g, int64_t n0, int64_t nb,
                    int64_t p0, int64_t np) {
  int64_t total = nb * np * g->Kp;
  if (total <= 0) return;
  k_im2col<<<grid_for(total, 256), 256, 0, stream()>>>(x, col, *g, n0, nb, p0, np);
  DCB_LAUNCHED();
}

void dk_col2im_tr(const float *cols, float *y, const float *bias, int64_t nb, int O,
                  const DkConvGeom *g) {
  int64_t total = nb * (int64_t)O * g->Ho * g->Wo;
  if (total <= 0) return;
  k_col2im_tr<<<grid_for(total, 256), 256, 0, stream()>>>(cols, y, bias, nb, O, *g);
  DCB_LAUNCHED();
}

void dk_softmax_to_half(const float *s, int64_t lds, dc_half *p, int64_t ldp, int64_t rows,
                        int64_t L, float scale) {
  if (rows <= 0) return;
  DCB_REQUIRE(rows <= 0x7fffffff, "softmax_to_half: too many rows");
  k_softmax_to_half<<<(unsigned)rows, 256, 0, stream()>>>(s, lds, p, ldp, L, scale);
  DCB_LAUNCHED();
}

void dk_split_heads_half(const float *x, dc_half *y, int64_t B, int64_t T, int H, int hd,
                         int hdp, int64_t Tp, int transpose) {
  int64_t n = transpose ? B * H * hd * Tp : B * H * T * hdp;
  if (n <= 0) return;
  k_split_heads<<<grid_for(n, 256), 256, 0, stream()>>>(x, y, B, T, H, hd, hdp, Tp, transpose);
  DCB_LAUNCHED();
}

}  // extern "C"
