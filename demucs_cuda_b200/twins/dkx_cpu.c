/* CPU twins of the fused entry points (include/dc_b200.h Part 2) for the reference's CPU
 * backend.  The reference's link model keeps its CUDA and CPU backends interchangeable: a
 * model layer that calls dkx_conv2d / dkx_conv_tr / dkx_linear / dkx_attention must also
 * link against backend_cpu.c.  Each twin composes Part-1 calls exactly as the reference's
 * ops.c composes the unfused operation it replaces, then applies the fused epilogue the same
 * way the reference's layers do after it:
 *
 *   dkx_conv2d    conv_core (ops.c:31-77): dk_im2col_half + dk_gemm_half + dk_channel_bias,
 *                 then GELU (layers.c:120, dk_unary) or channel GLU (layers.c:134, dk_glu)
 *   dkx_conv_tr   conv_tr_core (ops.c:143-177): dk_transpose_to_half + dk_gemm_half +
 *                 dk_col2im_tr with the decoder crop (layers.c:201-211) as the col2im output
 *                 offset, then GELU (layers.c:212-216)
 *   dkx_linear    dc_linear (ops.c:234-257)
 *   dkx_attention dc_attention (ops.c:390-443): split heads, S = Q K^T, softmax to fp16,
 *                 O = P V, heads merged back with dk_strided_copy
 *
 * Build it next to backend_cpu.c (same include path, backend.h):
 *   gcc -O3 -std=gnu11 -I worker-cuda/src -c dkx_cpu.c
 * Scratch comes from dk_raw_malloc / dk_raw_free, which the CPU backend serves from the host
 * heap; one batch item is processed at a time, so the scratch is that of one item. */
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "backend.h"

/* the epilogue selector of dkx_conv2d (values of include/dc_b200.h) */
enum { DKX_ACT_NONE = 0, DKX_ACT_GELU = 1, DKX_ACT_GLU = 2 };

void dkx_conv2d(const float *x, int N, const DkConvGeom *g, const dc_half *weight, int O,
                const float *bias, int act, float *y) {
  const int64_t P = (int64_t)g->Ho * g->Wo;
  if (N <= 0 || P <= 0) return;
  dc_half *col = (dc_half *)dk_raw_malloc((size_t)(P * g->Kp) * sizeof(dc_half));
  /* the O pre-activation channels: y itself unless a GLU halves them */
  float *z = act == DKX_ACT_GLU ? (float *)dk_raw_malloc((size_t)(N * O * P) * sizeof(float))
                                : y;
  for (int64_t n = 0; n < N; n++) {
    dk_im2col_half(x, col, g, n, 1, 0, P);
    dk_gemm_half(O, P, g->Kp, 1.0f, weight, g->Kp, 0, col, g->Kp, 0, 0.0f, z + n * O * P, P, 0,
                 1);
  }
  dk_raw_free(col);
  if (bias) dk_channel_bias(z, bias, N, O, P);
  if (act == DKX_ACT_GELU) {
    dk_unary(DK_UN_GELU, z, z, (int64_t)N * O * P, 1.0f, 0.0f);
  } else if (act == DKX_ACT_GLU) {
    dk_glu(z, y, N, O / 2, P);
    dk_raw_free(z);
  }
}

void dkx_conv_tr(const float *x, int N, int C, int H, int W, const dc_half *weight, int O,
                 int KH, int KW, int stride, const float *bias, int crop, int out_len,
                 int gelu, float *y) {
  const int axis_h = KW == 1;
  DkConvGeom g;
  memset(&g, 0, sizeof(g));
  g.C = C;
  g.H = H;
  g.W = W;
  g.KH = KH;
  g.KW = KW;
  g.SH = axis_h ? stride : 1;
  g.SW = axis_h ? 1 : stride;
  g.PH = axis_h ? crop : 0; /* col2im output offset along the stride axis: the crop */
  g.PW = axis_h ? 0 : crop;
  g.DH = g.DW = 1;
  g.Ho = axis_h ? out_len : H;
  g.Wo = axis_h ? W : out_len;
  g.Kp = (C + 7) / 8 * 8; /* the loader's padding of the reduction over input channels */
  const int64_t P = (int64_t)H * W, M = (int64_t)O * KH * KW;
  if (N <= 0 || P <= 0) return;
  dc_half *xt = (dc_half *)dk_raw_malloc((size_t)(P * g.Kp) * sizeof(dc_half));
  float *cols = (float *)dk_raw_malloc((size_t)(M * P) * sizeof(float));
  const int64_t out_item = (int64_t)O * g.Ho * g.Wo;
  for (int64_t n = 0; n < N; n++) {
    dk_transpose_to_half(x + n * C * P, xt, 1, C, P, g.Kp);
    dk_gemm_half(M, P, g.Kp, 1.0f, weight, g.Kp, 0, xt, g.Kp, 0, 0.0f, cols, P, 0, 1);
    dk_col2im_tr(cols, y + n * out_item, bias, 1, O, &g);
  }
  dk_raw_free(xt);
  dk_raw_free(cols);
  if (gelu) dk_unary(DK_UN_GELU, y, y, (int64_t)N * out_item, 1.0f, 0.0f);
}

void dkx_linear(const float *x, int64_t R, int in, const dc_half *weight, int64_t kp, int out,
                const float *bias, float *y) {
  if (R <= 0) return;
  dc_half *xh = (dc_half *)dk_raw_malloc((size_t)(R * kp) * sizeof(dc_half));
  dk_to_half_rows(x, xh, R, in, kp);
  dk_gemm_half(R, out, kp, 1.0f, xh, kp, 0, weight, kp, 0, 0.0f, y, out, 0, 1);
  dk_raw_free(xh);
  if (bias) dk_channel_bias(y, bias, R, out, 1);
}

void dkx_attention(const float *q, const float *k, const float *v, int B, int Tq, int Tk,
                   int H, int hd, float *y) {
  if (B <= 0 || Tq <= 0 || Tk <= 0) return;
  const int hdp = (hd + 7) / 8 * 8;
  const int64_t Tkp = ((int64_t)Tk + 7) / 8 * 8, BH = (int64_t)B * H, D = (int64_t)H * hd;
  dc_half *qh = (dc_half *)dk_raw_malloc((size_t)(BH * Tq * hdp) * sizeof(dc_half));
  dc_half *kh = (dc_half *)dk_raw_malloc((size_t)(BH * Tk * hdp) * sizeof(dc_half));
  dc_half *vt = (dc_half *)dk_raw_malloc((size_t)(BH * hd * Tkp) * sizeof(dc_half));
  float *s = (float *)dk_raw_malloc((size_t)((int64_t)Tq * Tk) * sizeof(float));
  dc_half *p = (dc_half *)dk_raw_malloc((size_t)((int64_t)Tq * Tkp) * sizeof(dc_half));
  float *o = (float *)dk_raw_malloc((size_t)(BH * Tq * hd) * sizeof(float));
  dk_split_heads_half(q, qh, B, Tq, H, hd, hdp, 0, 0);
  dk_split_heads_half(k, kh, B, Tk, H, hd, hdp, 0, 0);
  dk_split_heads_half(v, vt, B, Tk, H, hd, hdp, Tkp, 1);
  const float scale = 1.0f / sqrtf((float)hd);
  for (int64_t bh = 0; bh < BH; bh++) {
    dk_gemm_half(Tq, Tk, hdp, 1.0f, qh + bh * Tq * hdp, hdp, 0, kh + bh * Tk * hdp, hdp, 0,
                 0.0f, s, Tk, 0, 1);
    dk_softmax_to_half(s, Tk, p, Tkp, Tq, Tk, scale);
    dk_gemm_half(Tq, hd, Tkp, 1.0f, p, Tkp, 0, vt + bh * hd * Tkp, Tkp, 0, 0.0f,
                 o + bh * Tq * hd, hd, 0, 1);
  }
  /* o [B][H][Tq][hd] -> y [B][Tq][H * hd] */
  DkStrided st;
  memset(&st, 0, sizeof(st));
  st.ndim = 4;
  st.shape[0] = B;
  st.shape[1] = H;
  st.shape[2] = Tq;
  st.shape[3] = hd;
  st.a_strides[0] = (int64_t)H * Tq * hd;
  st.a_strides[1] = (int64_t)Tq * hd;
  st.a_strides[2] = hd;
  st.a_strides[3] = 1;
  st.b_strides[0] = (int64_t)Tq * D;
  st.b_strides[1] = hd;
  st.b_strides[2] = D;
  st.b_strides[3] = 1;
  dk_strided_copy(&st, o, y, 0);
  dk_raw_free(qh);
  dk_raw_free(kh);
  dk_raw_free(vt);
  dk_raw_free(s);
  dk_raw_free(p);
  dk_raw_free(o);
}
