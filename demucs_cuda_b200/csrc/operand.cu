// GEMM operand preparation and attention helpers of the backend.h ABI
// (backend.h:91-131; reference semantics backend_cpu.c:324-506).  The model engine in this
// library does not call these (its conv, transposed-conv and attention kernels gather
// operands on the fly); they exist so the reference's unchanged ops.c runs on this backend
// with identical results.
//
// Every fp16 operand row here is written in 16-byte groups of eight elements (one uint4
// store per thread and group) when the row length and the destination allow it; the
// fp32 sources are read along their contiguous axis.
#include "common.cuh"

namespace dcb {

// eight floats -> eight fp16 (RNE) in one 16-byte word
static __device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  return make_uint4(pack_h2(v[0], v[1]), pack_h2(v[2], v[3]), pack_h2(v[4], v[5]),
                    pack_h2(v[6], v[7]));
}

// ---------------------------------------------------------------- to_half_rows
// y[r][c] = fp16(x[r][c]) for c < C, 0 for C <= c < Cp.  Thread = (row, group of 8 output
// columns); groups = ceil(Cp / 8) per row.
__global__ void k_to_half_rows(const float *__restrict__ x, uint16_t *__restrict__ y,
                               int64_t rows, int64_t C, int64_t Cp, int vec) {
  const int64_t groups = (Cp + 7) / 8;
  DCB_GRID_STRIDE(u, rows * groups) {
    const int64_t r = u / groups, c0 = (u - r * groups) * 8;
    const float *xr = x + r * C;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = c0 + i < C ? xr[c0 + i] : 0.f;
    if (vec) {
      *(uint4 *)(y + r * Cp + c0) = pack8(v);
    } else {
      for (int i = 0; i < 8 && c0 + i < Cp; i++) y[r * Cp + c0 + i] = f2h_bits(v[i]);
    }
  }
}

// ---------------------------------------------------------------- transpose_to_half
// x [b][C][P] fp32 -> y [b][P][Cp] fp16, channels >= C zero.  CTA tile: 64 positions x 64
// channels.  Load phase: each warp reads channel rows of the tile along P (coalesced) and
// stores them converted to fp16 as sm[c][p].  Store phase: a thread owns (position, group of
// 8 channels) and writes that group as one 16-byte word of the output row.
constexpr int kTpP = 64, kTpC = 64;
__global__ void __launch_bounds__(256)
    k_transpose_to_half(const float *__restrict__ x, uint16_t *__restrict__ y, int64_t C,
                        int64_t P, int64_t Cp, int vec) {
  __shared__ uint16_t sm[kTpC][kTpP + 2];  // +2 halves: rows start on distinct banks
  const int64_t b = blockIdx.z;
  const int64_t p0 = (int64_t)blockIdx.x * kTpP, c0 = (int64_t)blockIdx.y * kTpC;
  const float *xb = x + b * C * P;
  uint16_t *yb = y + b * P * Cp;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int cr = warp; cr < kTpC; cr += 8) {
    const int64_t c = c0 + cr;
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const int pp = h * 32 + lane;
      const int64_t p = p0 + pp;
      sm[cr][pp] = f2h_bits(c < C && p < P ? xb[c * P + p] : 0.f);
    }
  }
  __syncthreads();
  // 64 positions x 8 channel groups = 512 (position, group) words, two per thread
#pragma unroll
  for (int k = 0; k < 2; k++) {
    const int u = k * 256 + threadIdx.x;
    const int pp = u >> 3, grp = u & 7;
    const int64_t p = p0 + pp, cg = c0 + grp * 8;
    if (p >= P || cg >= Cp) continue;
    uint16_t h[8];
#pragma unroll
    for (int i = 0; i < 8; i++) h[i] = cg + i < C ? sm[grp * 8 + i][pp] : (uint16_t)0;
    if (vec) {
      *(uint4 *)(yb + p * Cp + cg) =
          make_uint4(h[0] | ((uint32_t)h[1] << 16), h[2] | ((uint32_t)h[3] << 16),
                     h[4] | ((uint32_t)h[5] << 16), h[6] | ((uint32_t)h[7] << 16));
    } else {
      for (int i = 0; i < 8 && cg + i < Cp; i++) yb[p * Cp + cg + i] = h[i];
    }
  }
}

// ---------------------------------------------------------------- im2col
// col[bi][pi][k] with k = (kh KW + kw) C + c (backend.h:107-110).  Thread = (item, position,
// group of 8 consecutive k); the group's (c, kw, kh) is decoded once and then stepped.
__global__ void k_im2col(const float *__restrict__ x, uint16_t *__restrict__ col, DkConvGeom g,
                         int64_t n0, int64_t nb, int64_t p0, int64_t np, int vec) {
  const int64_t K = (int64_t)g.KH * g.KW * g.C, plane = (int64_t)g.H * g.W;
  const int64_t groups = (g.Kp + 7) / 8;
  DCB_GRID_STRIDE(u, nb * np * groups) {
    const int64_t row = u / groups, k0 = (u - row * groups) * 8;
    const int64_t bi = row / np, p = p0 + (row - bi * np);
    const int ho = (int)(p / g.Wo), wo = (int)(p - (int64_t)ho * g.Wo);
    const float *xb = x + (n0 + bi) * g.C * plane;
    int c = (int)(k0 % g.C), t = (int)(k0 / g.C);
    int kw = t % g.KW, kh = t / g.KW;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
      float e = 0.f;
      if (k0 + i < K) {
        const int h = ho * g.SH - g.PH + kh * g.DH, w = wo * g.SW - g.PW + kw * g.DW;
        if (h >= 0 && h < g.H && w >= 0 && w < g.W) e = xb[c * plane + (int64_t)h * g.W + w];
      }
      v[i] = e;
      if (++c == g.C) {
        c = 0;
        if (++kw == g.KW) {
          kw = 0;
          kh++;
        }
      }
    }
    uint16_t *dst = col + row * g.Kp + k0;
    if (vec) {
      *(uint4 *)dst = pack8(v);
    } else {
      for (int i = 0; i < 8 && k0 + i < g.Kp; i++) dst[i] = f2h_bits(v[i]);
    }
  }
}

// ---------------------------------------------------------------- col2im (transposed conv)
// y[bi][o][ho][wo] = bias[o] + sum of cols[bi][(o, kh, kw)][h][w] over the taps with
// ho + PH = h SH + kh and wo + PW = w SW + kw.  Only taps in the output's stride phase can
// contribute, so the tap loops start at the phase residue and step by the stride (at most
// ceil(KH / SH) x ceil(KW / SW) taps, no divisibility tests), in ascending (kh, kw) order.
// CTA = one output row (bi, o, ho); threads stride over wo.
__global__ void __launch_bounds__(128)
    k_col2im_tr(const float *__restrict__ cols, float *__restrict__ y,
                const float *__restrict__ bias, int O, DkConvGeom g) {
  const int64_t P = (int64_t)g.H * g.W, taps = (int64_t)g.KH * g.KW;
  const int64_t rowid = blockIdx.x;  // (bi, o, ho)
  const int ho = (int)(rowid % g.Ho);
  const int64_t bo = rowid / g.Ho;
  const int o = (int)(bo % O);
  const int64_t bi = bo / O;
  const float *cb = cols + (bi * O + o) * taps * P;
  float *yr = y + rowid * g.Wo;
  const float b0 = bias ? bias[o] : 0.f;
  const int hf = ho + g.PH;
  // smallest kh >= 0 of this phase whose input row h = (hf - kh) / SH is < H
  int kh_lo = hf % g.SH;
  const int hmax_k = hf - g.SH * (g.H - 1);  // kh below this gives h >= H
  if (kh_lo < hmax_k) kh_lo += ((hmax_k - kh_lo + g.SH - 1) / g.SH) * g.SH;
  for (int wo = threadIdx.x; wo < g.Wo; wo += blockDim.x) {
    const int wf = wo + g.PW;
    int kw_lo = wf % g.SW;
    const int wmax_k = wf - g.SW * (g.W - 1);
    if (kw_lo < wmax_k) kw_lo += ((wmax_k - kw_lo + g.SW - 1) / g.SW) * g.SW;
    float acc = b0;
    for (int kh = kh_lo; kh < g.KH && kh <= hf; kh += g.SH) {
      const int h = (hf - kh) / g.SH;
      const float *ck = cb + (int64_t)kh * g.KW * P + (int64_t)h * g.W;
      for (int kw = kw_lo; kw < g.KW && kw <= wf; kw += g.SW) {
        acc += ck[(int64_t)kw * P + (wf - kw) / g.SW];
      }
    }
    yr[wo] = acc;
  }
}

// ---------------------------------------------------------------- softmax -> fp16
// P = softmax(scale * S) per row, fp16, columns L..ldp-1 zeroed.  One warp per row (eight
// rows per CTA): lane-strided passes for the maximum and the sum of exponentials (lane sums
// in fp32, combined across lanes in double), then the normalised row in fp16 pairs.
__global__ void __launch_bounds__(256)
    k_softmax_to_half(const float *__restrict__ s, int64_t lds, uint16_t *__restrict__ p,
                      int64_t ldp, int64_t rows, int64_t L, float scale, int pairs) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const float *row = s + r * lds;
  uint16_t *out = p + r * ldp;
  float mx = -INFINITY;
  for (int64_t j = lane; j < L; j += 32) mx = fmaxf(mx, row[j] * scale);
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float part = 0.f;
  for (int64_t j = lane; j < L; j += 32) part += expf(row[j] * scale - mx);
  double sum = (double)part;
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float inv = (float)(1.0 / sum);
  if (pairs) {
    for (int64_t j = 2 * lane; j < ldp; j += 64) {
      const float a = j < L ? expf(row[j] * scale - mx) * inv : 0.f;
      const float b = j + 1 < L ? expf(row[j + 1] * scale - mx) * inv : 0.f;
      *(uint32_t *)(out + j) = pack_h2(a, b);
    }
  } else {
    for (int64_t j = lane; j < ldp; j += 32) {
      out[j] = j < L ? f2h_bits(expf(row[j] * scale - mx) * inv) : (uint16_t)0;
    }
  }
}

// ---------------------------------------------------------------- split heads
// x [B][T][H hd] fp32 -> y [B][H][T][hdp] fp16 (d >= hd zero).  One warp per token row
// (b, t): the lanes read the row's H hd floats in order and write each head's slice.
__global__ void __launch_bounds__(256)
    k_split_heads_rows(const float *__restrict__ x, uint16_t *__restrict__ y, int64_t B,
                       int64_t T, int H, int hd, int hdp) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t D = (int64_t)H * hd;
  for (int64_t bt = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; bt < B * T;
       bt += nwarps) {
    const int64_t b = bt / T, t = bt - b * T;
    const float *xr = x + bt * D;
    for (int64_t e = lane; e < (int64_t)H * hdp; e += 32) {
      const int h = (int)(e / hdp), d = (int)(e - (int64_t)h * hdp);
      y[((b * H + h) * T + t) * hdp + d] = d < hd ? f2h_bits(xr[(int64_t)h * hd + d]) : (uint16_t)0;
    }
  }
}

// x [B][T][H hd] fp32 -> y [B][H][hd][Tp] fp16 (t >= T zero).  CTA tile: 32 tokens x 32
// feature columns of one b, read along the features and written along the tokens through a
// shared tile, so both sides are coalesced; tiles cover t up to Tp (the zero padding).
__global__ void __launch_bounds__(256)
    k_split_heads_t(const float *__restrict__ x, uint16_t *__restrict__ y, int64_t T, int H,
                    int hd, int64_t Tp) {
  __shared__ float sm[32][33];
  const int64_t b = blockIdx.z;
  const int64_t t0 = (int64_t)blockIdx.x * 32;
  const int64_t f0 = (int64_t)blockIdx.y * 32;
  const int64_t D = (int64_t)H * hd;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int i = ty; i < 32; i += 8) {
    const int64_t t = t0 + i, f = f0 + tx;
    sm[i][tx] = (t < T && f < D) ? x[(b * T + t) * D + f] : 0.f;
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int64_t f = f0 + i, t = t0 + tx;
    if (f >= D || t >= Tp) continue;
    const int h = (int)(f / hd), d = (int)(f - (int64_t)h * hd);
    y[((b * H + h) * hd + d) * Tp + t] = f2h_bits(sm[tx][i]);
  }
}

}  // namespace dcb

using namespace dcb;

extern "C" {

void dk_to_half_rows(const float *x, dc_half *y, int64_t rows, int64_t C, int64_t Cp) {
  if (rows <= 0 || Cp <= 0) return;
  const int vec = Cp % 8 == 0 && ((uintptr_t)y & 15) == 0;
  const int64_t groups = (Cp + 7) / 8;
  k_to_half_rows<<<grid_for(rows * groups, 256), 256, 0, stream()>>>(x, y, rows, C, Cp, vec);
  DCB_LAUNCHED();
}

void dk_transpose_to_half(const float *x, dc_half *y, int64_t batch, int64_t C, int64_t P,
                          int64_t Cp) {
  if (batch <= 0 || P <= 0 || Cp <= 0) return;
  DCB_REQUIRE(batch <= 65535, "transpose_to_half: batch %lld > 65535", (long long)batch);
  const int vec = Cp % 8 == 0 && ((uintptr_t)y & 15) == 0;
  dim3 grid((unsigned)((P + kTpP - 1) / kTpP), (unsigned)((Cp + kTpC - 1) / kTpC),
            (unsigned)batch);
  k_transpose_to_half<<<grid, 256, 0, stream()>>>(x, y, C, P, Cp, vec);
  DCB_LAUNCHED();
}

void dk_im2col_half(const float *x, dc_half *col, const DkConvGeom *g, int64_t n0, int64_t nb,
                    int64_t p0, int64_t np) {
  const int64_t groups = (g->Kp + 7) / 8;
  if (nb <= 0 || np <= 0 || groups <= 0) return;
  const int vec = g->Kp % 8 == 0 && ((uintptr_t)col & 15) == 0;
  k_im2col<<<grid_for(nb * np * groups, 256), 256, 0, stream()>>>(x, col, *g, n0, nb, p0, np,
                                                                   vec);
  DCB_LAUNCHED();
}

void dk_col2im_tr(const float *cols, float *y, const float *bias, int64_t nb, int O,
                  const DkConvGeom *g) {
  const int64_t rows = nb * (int64_t)O * g->Ho;
  if (rows <= 0 || g->Wo <= 0) return;
  DCB_REQUIRE(rows < 0x7fffffff && g->SH > 0 && g->SW > 0,
              "col2im_tr: %lld output rows, strides %d x %d", (long long)rows, g->SH, g->SW);
  k_col2im_tr<<<(unsigned)rows, 128, 0, stream()>>>(cols, y, bias, O, *g);
  DCB_LAUNCHED();
}

void dk_softmax_to_half(const float *s, int64_t lds, dc_half *p, int64_t ldp, int64_t rows,
                        int64_t L, float scale) {
  if (rows <= 0) return;
  DCB_REQUIRE((rows + 7) / 8 <= 0x7fffffff, "softmax_to_half: too many rows");
  const int pairs = ldp % 2 == 0 && ((uintptr_t)p & 3) == 0;
  k_softmax_to_half<<<(unsigned)((rows + 7) / 8), 256, 0, stream()>>>(s, lds, p, ldp, rows, L,
                                                                      scale, pairs);
  DCB_LAUNCHED();
}

void dk_split_heads_half(const float *x, dc_half *y, int64_t B, int64_t T, int H, int hd,
                         int hdp, int64_t Tp, int transpose) {
  if (B <= 0 || H <= 0 || hd <= 0) return;
  if (!transpose) {
    if (T <= 0 || hdp <= 0) return;
    k_split_heads_rows<<<grid_for(B * T * 32, 256), 256, 0, stream()>>>(x, y, B, T, H, hd,
                                                                        hdp);
  } else {
    if (Tp <= 0) return;
    DCB_REQUIRE(B <= 65535, "split_heads_half: batch %lld > 65535", (long long)B);
    const int64_t D = (int64_t)H * hd;
    dim3 grid((unsigned)((Tp + 31) / 32), (unsigned)((D + 31) / 32), (unsigned)B);
    k_split_heads_t<<<grid, 256, 0, stream()>>>(x, y, T, H, hd, Tp);
  }
  DCB_LAUNCHED();
}

}  // extern "C"
