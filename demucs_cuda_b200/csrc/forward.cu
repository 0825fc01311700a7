// Forward pass of the htdemucs_6s engine (htdemucs.c:136-280 order), the teacher-forced
// single-stage entry points used by the parity tests (test_compare.c:139-216 order) and
// the segment scheduler (apply.c:179-306).
#include <math.h>

#include <algorithm>
#include <string>
#include <vector>

#include "common.cuh"
#include "gemm.cuh"

namespace dcb {


// ------------------------------------------------------------------ device memory
static float *dalloc(size_t n) {
  void *p = nullptr;
  DCB_CUDA(cudaMallocAsync(&p, (n ? n : 1) * sizeof(float), stream()));
  return (float *)p;
}
static uint16_t *halloc(size_t n) {
  void *p = nullptr;
  DCB_CUDA(cudaMallocAsync(&p, (n ? n : 1) * sizeof(uint16_t), stream()));
  return (uint16_t *)p;
}
static void dfree(void *p) {
  if (p) DCB_CUDA(cudaFreeAsync(p, stream()));
}

// The frequency and time branches are independent from the spectrogram to the transformer,
// inside each transformer layer, and through the decoders: the time branch's layers are
// issued on a second stream (option "streams"), forked from and joined back to the current
// one with events, so its kernels fill the GPU beside the frequency branch's (inside a CUDA
// graph capture the second stream joins the capture through the fork).
static cudaStream_t aux_stream() {
  static cudaStream_t s = nullptr;
  if (!s) DCB_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  return s;
}
// the second stream of overlapped forward batches (see apply_window)
static cudaStream_t batch_stream() {
  static cudaStream_t s = nullptr;
  if (!s) DCB_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  return s;
}
// `waiter` waits for everything issued so far on `on`
static void stream_wait(cudaStream_t waiter, cudaStream_t on) {
  static cudaEvent_t ev[16] = {};
  static int next = 0;
  cudaEvent_t &e = ev[next];
  next = (next + 1) % 16;
  if (!e) DCB_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  DCB_CUDA(cudaEventRecord(e, on));
  DCB_CUDA(cudaStreamWaitEvent(waiter, e, 0));
}
// issue on `s` for the lifetime of the scope (when `on`), then back to the previous stream
struct OnStream {
  cudaStream_t prev = nullptr;
  bool on;
  OnStream(cudaStream_t s, bool on_) : on(on_) {
    if (!on) return;
    prev = stream_override_get();
    set_stream_override(s);
  }
  ~OnStream() {
    if (on) set_stream_override(prev);
  }
};

void ispec_fused(const float *x, float *out, const float *mean, const float *var, int B,
                 int rows_per_b, int F, int N, int n_fft, int hop, const float *window,
                 int64_t start, int64_t length, float eps);
bool ispec_stream_ok(int n_fft, int hop, int N, int64_t start, int64_t length);
void ispec_frames(const float2 *z, float *out, int64_t R, int F, int N, const float *window,
                  int64_t start, int64_t length, const StreamCombine &cb);
void spec_normalised(const float *xc, int B, int C, int64_t L, int n_fft, int hop, int frame0,
                     int nframes, int nbins, const float *window, float *x, float *mean,
                     float *var, float *mag);

struct Stage {
  DcbStageFn fn = nullptr;
  void *user = nullptr;
  void emit(const char *name, const float *p, std::initializer_list<int> shape) {
    if (!fn) return;
    DCB_CUDA(cudaStreamSynchronize(stream()));
    int s[8];
    int n = 0;
    for (int v : shape) s[n++] = v;
    fn(name, p, n, s, user);
  }
};

// ------------------------------------------------------------------ conv helpers
// conv over images of x viewed as [n1][n2] -> (c, h, w) with the given strides, output
// written through the same kind of view; act: 0 none, 1 gelu, 2 glu (weights interleaved)
struct Img {
  int N1 = 1, N2 = 1;
  int64_t sN1 = 0, sN2 = 0, sC = 0, sH = 0;
  int C = 0, H = 1, W = 1;
};

static Img contiguous(int N, int C, int H, int W) {
  Img v;
  v.N1 = N;
  v.N2 = 1;
  v.sN1 = (int64_t)C * H * W;
  v.sC = (int64_t)H * W;
  v.sH = W;
  v.C = C;
  v.H = H;
  v.W = W;
  return v;
}
// [B, C, Fr, T] seen as B*Fr images [C][1][T] (the DConv view of layers.c:3-20)
static Img freq_rows(int B, int C, int Fr, int T) {
  Img v;
  v.N1 = B;
  v.N2 = Fr;
  v.sN1 = (int64_t)C * Fr * T;
  v.sN2 = T;
  v.sC = (int64_t)Fr * T;
  v.sH = 0;
  v.C = C;
  v.H = 1;
  v.W = T;
  return v;
}

static void conv(const ConvW &cw, const float *x, const float *x2, const Img &in, int SH, int SW,
                 int PH, int PW, int DH, int DW, int Ho, int Wo, float *y, const Img &out,
                 int act, const float *res = nullptr, const float *scale = nullptr,
                 const float *gn_mean = nullptr, const float *gn_rstd = nullptr,
                 const NormW *gn = nullptr) {
  Gather g{};
  g.x = x;
  g.x2 = x2;
  g.N2 = in.N2;
  g.sN1 = in.sN1;
  g.sN2 = in.sN2;
  g.sC = in.sC;
  g.sH = in.sH;
  g.C = in.C;
  g.H = in.H;
  g.W = in.W;
  g.KH = cw.KH;
  g.KW = cw.KW;
  g.SH = SH;
  g.SW = SW;
  g.PH = PH;
  g.PW = PW;
  g.DH = DH;
  g.DW = DW;
  g.Ho = Ho;
  g.Wo = Wo;
  g.K = cw.K;
  Epi e;
  e.mode = EPI_CONV;
  e.bias = cw.bias;
  e.act = act;
  e.y = y;
  e.oN2 = out.N2;
  e.oN1 = out.sN1;
  e.oN2s = out.sN2;
  e.oC = out.sC;
  e.oH = out.sH;
  e.O = act >= 2 ? cw.O / 2 : cw.O;
  e.Ho = Ho;
  e.Wo = Wo;
  e.res = res;
  e.scale = scale;
  e.gn_mean = gn_mean;
  e.gn_rstd = gn_rstd;
  e.gn_w = gn ? gn->w : nullptr;
  e.gn_b = gn ? gn->b : nullptr;
  const int64_t M = (int64_t)in.N1 * in.N2 * Ho * Wo;
  gemm_gather(g, M, cw.w, cw.rows, cw.ld, e, act >= 2 ? cw.glu_bn : 0, cw.wt, cw.ldt, cw.ncb);
}

// stride-phase transposed conv along H (freq) or W (time), crop + optional GELU
static void conv_tr(const ConvW &cw, const float *x, const Img &in, bool axis_h, int S,
                    int crop, int out_len, bool gelu, float *y, const Img &out) {
  Gather g{};
  g.x = x;
  g.N2 = in.N2;
  g.sN1 = in.sN1;
  g.sN2 = in.sN2;
  g.sC = in.sC;
  g.sH = in.sH;
  g.C = in.C;
  g.H = in.H;
  g.W = in.W;
  g.KH = axis_h ? 2 : 1;
  g.KW = axis_h ? 1 : 2;
  g.SH = g.SW = 1;
  g.PH = axis_h ? 1 : 0;
  g.PW = axis_h ? 0 : 1;
  g.DH = g.DW = 1;
  g.Ho = axis_h ? in.H + 1 : in.H;
  g.Wo = axis_h ? in.W : in.W + 1;
  g.K = 2 * in.C;
  Epi e;
  e.mode = EPI_CONVTR;
  e.bias = cw.bias;
  e.act = gelu ? 1 : 0;
  e.y = y;
  e.oN2 = out.N2;
  e.oN1 = out.sN1;
  e.oN2s = out.sN2;
  e.oC = out.sC;
  e.oH = out.sH;
  e.O = cw.O;
  e.Ho = g.Ho;
  e.Wo = g.Wo;
  e.stride = S;
  e.crop = crop;
  e.out_len = out_len;
  e.axis_h = axis_h ? 1 : 0;
  gemm_gather(g, (int64_t)in.N1 * in.N2 * g.Ho * g.Wo, cw.w, cw.rows, cw.ld, e, 0, cw.wt,
              cw.ldt, cw.ncb);
}

// ------------------------------------------------------------------ fp16 companions
// fp16 channels-last copy of an activation [images][C][H][W]: [images][H][Wp][C] (Wp = W,
// or W rounded up to a multiple of 4 with zero positions past W where a stride-4 conv
// reads it), written by the producing kernel and read by the next conv through TMA.
struct Half16 {
  uint16_t *p = nullptr;
  int64_t images = 0;
  int C = 0, H = 1, W = 0, Wp = 0;
  int im2col = 0;  // 1: the 8-tap im2col of a few-channel input, read by a 1x1 conv
  HalfAct act() const { return HalfAct{p, images, C, H, W, Wp}; }
  // [images * H][1][Wp][C]: the DConv view (frequency rows are images)
  HalfAct rows() const { return HalfAct{p, images * H, C, 1, W, Wp}; }
};

static Half16 half_alloc(int64_t images, int C, int H, int W, bool pad4) {
  Half16 h;
  if (C % 8) return h;  // no companion: the convs read the fp32 tensor
  h.images = images;
  h.C = C;
  h.H = H;
  h.W = W;
  h.Wp = pad4 ? (W + 3) / 4 * 4 : W;
  const size_t n = (size_t)images * H * h.Wp * C;
  h.p = halloc(n);
  if (h.Wp != W) DCB_CUDA(cudaMemsetAsync(h.p, 0, n * 2, stream()));
  return h;
}

// fp16 companion of an fp32 NCHW tensor [images][Cs][H][W] (+ addend of the same layout)
// with C >= Cs channels (the extra ones zero; C = Cs when Cs is a multiple of 8)
static Half16 to_half(const float *x, const float *add, int64_t images, int Cs, int H, int W,
                      bool pad4, int C = 0) {
  if (C == 0) C = Cs;
  Half16 h = half_alloc(images, C, H, W, pad4);
  if (!h.p) return h;
  const int64_t n = images * H * (int64_t)W * (C / 8);
  k_to_half_cl<<<grid_for(n, 256), 256, 0, stream()>>>(x, add, h.p, images, C, H, W, h.Wp,
                                                       (int64_t)Cs * H * W, (int64_t)H * W, W,
                                                       Cs);
  DCB_LAUNCHED();
  return h;
}

// im2col'd fp16 copy of a few-channel input for an 8-tap, stride-S conv along H (axis 0) or
// W (axis 1): [images][Ho][Wo][64]
static Half16 im2col8(const float *x, int64_t images, int C, int H, int W, int Ho, int Wo,
                      int S, int P, int axis) {
  Half16 h = half_alloc(images, 64, Ho, Wo, false);
  h.im2col = 1;
  const int64_t n = images * Ho * (int64_t)Wo * 8;
  k_im2col8_half<<<grid_for(n, 256), 256, 0, stream()>>>(x, h.p, images, C, H, W, Ho, Wo, S, P,
                                                         axis);
  DCB_LAUNCHED();
  return h;
}

// point the epilogue's fp16 copy at h (its [images][H][Wp][C] layout)
static void epi_half(Epi &e, const Half16 &h) {
  e.yh = h.p;
  e.yhH = h.H;
  e.yhW = h.Wp;
  e.yhC = h.C;
}

// conv through the fp16 companion when the TMA kernel covers it, else the gather kernel on
// the fp32 tensor (then the companion, if wanted, is converted from the fp32 output)
// Returns whether the channels-last tensor-core conv ran (only it sums row_stats: the
// per-image output sums of a rows view, see Epi::row_stats; the caller falls back otherwise)
static bool conv_any(const ConvW &cw, const float *x, const Half16 *xh, const Img &in, int SH,
                     int SW, int PH, int PW, int DH, int DW, int Ho, int Wo, float *y,
                     const Img &out, int act, Half16 *yh, bool rows_view,
                     const float *emb = nullptr, float emb_alpha = 0.f, int emb_ld = 0,
                     double *row_stats = nullptr) {
  Epi e;
  e.mode = EPI_CONV;
  e.bias = cw.bias;
  e.act = act;
  e.y = y;
  e.oN2 = out.N2;
  e.oN1 = out.sN1;
  e.oN2s = out.sN2;
  e.oC = out.sC;
  e.oH = out.sH;
  e.O = act >= 2 ? cw.O / 2 : cw.O;
  e.Ho = Ho;
  e.Wo = Wo;
  e.emb = emb;
  e.emb_alpha = emb_alpha;
  e.emb_ld = emb_ld;
  e.row_stats = rows_view ? row_stats : nullptr;
  if (yh && yh->p) epi_half(e, *yh);
  if (xh && xh->p && xh->im2col && cw.wi) {
    // the input is already im2col'd: a 1x1 conv with K = 8 taps x 8 channels
    if (conv_half(xh->act(), 1, 1, 1, 1, 0, 0, 1, 1, Ho, Wo, cw.wi, cw.rows, 64, 1, e, 0))
      return true;
  } else if (xh && xh->p && cw.wt) {
    const HalfAct a = rows_view ? xh->rows() : xh->act();
    if (conv_half(a, cw.KH, cw.KW, SH, SW, PH, PW, DH, DW, Ho, Wo, cw.wt, cw.rows, cw.ldt,
                  cw.ncb, e, act >= 2 ? cw.glu_bn : 0))
      return true;
    if (e.row_stats) {
      // an epilogue without the row sums: the conv alone (the caller forms the statistics)
      e.row_stats = nullptr;
      if (conv_half(a, cw.KH, cw.KW, SH, SW, PH, PW, DH, DW, Ho, Wo, cw.wt, cw.rows, cw.ldt,
                    cw.ncb, e, act >= 2 ? cw.glu_bn : 0))
        return false;
    }
  }
  if (x == nullptr || y == nullptr) {
    fail("conv: the gather kernel needs fp32 tensors");
    return false;
  }
  conv(cw, x, nullptr, in, SH, SW, PH, PW, DH, DW, Ho, Wo, y, out, act);
  if (emb) {
    const int64_t n = (int64_t)out.N1 * e.O * Ho * Wo;
    k_add_freq_emb<<<grid_for(n, 256), 256, 0, stream()>>>(y, emb, emb_alpha, out.N1, e.O, Ho,
                                                          Wo, emb_ld);
    DCB_LAUNCHED();
  }
  if (yh && yh->p) {
    // fp32 output -> companion; out is contiguous [N1*N2 images][C][Ho][Wo] or rows
    const int64_t n = (int64_t)yh->images * yh->H * yh->W * (yh->C / 8);
    k_to_half_cl<<<grid_for(n, 256), 256, 0, stream()>>>(
        y, nullptr, yh->p, yh->images, yh->C, yh->H, yh->W, yh->Wp, out.sN1,
        rows_view ? (int64_t)yh->H * yh->W : out.sC, yh->W, yh->C);
    DCB_LAUNCHED();
  }
  return false;
}

// ------------------------------------------------------------------ layers
// y += scale * GLU(GroupNorm(conv1x1(h))) of a DConv layer on CUDA cores (hid <= 24), also
// refreshing the fp16 companion of y
static void dconv_tail(const DConvW &dw, const float *h, float *y, int B, int C, int hid,
                       int Fr, int T, const float *zmean, const float *zrstd, Half16 *yh) {
  const int hidp = (hid + 3) / 4 * 4;
  const size_t sm = ((size_t)2 * C * hidp + 7 * (size_t)C) * sizeof(float);
  const int64_t total = (int64_t)B * Fr * T;
  const unsigned grid = grid_for(total, 256, 148 * 8);
  const int64_t hsB = (int64_t)hid * Fr * T, hsC = (int64_t)Fr * T;
  const int64_t ysB = (int64_t)C * Fr * T, ysC = (int64_t)Fr * T;
  uint16_t *yhp = yh ? yh->p : nullptr;
  const int64_t pitch = yh ? yh->Wp : 0;
  // minimum bytes: h read once, y read and rewritten, its fp16 companion written
  TraceScope ts(TR_DCONV, 0.0,
                (double)total * ((double)hid * 4.0 + (double)C * 8.0 + (yhp ? C * 2.0 : 0.0)),
                total, C, hid);
#define DCB_TAIL(P)                                                                            \
  k_dconv_tail<P><<<grid, 256, sm, stream()>>>(h, y, dw.c3.w, dw.c3.ld, dw.c3.bias, dw.gn4.w, \
                                              dw.gn4.b, dw.scale, zmean, zrstd, B, C, hid,   \
                                              Fr, T, hsB, hsC, ysB, ysC, yhp, pitch)
  switch (hidp) {
    case 4: DCB_TAIL(4); break;
    case 8: DCB_TAIL(8); break;
    case 12: DCB_TAIL(12); break;
    case 16: DCB_TAIL(16); break;
    case 20: DCB_TAIL(20); break;
    default: DCB_TAIL(24); break;
  }
#undef DCB_TAIL
  DCB_LAUNCHED();
}

// DConv residual branch (layers.c:24-53) applied in place on y [B, C, Fr, T] (Fr = 1 for
// the time branch) and its fp16 companion yh ([B][Fr][Wp][C], read by the k3 convs):
// conv k3 (dilation 2^d) -> GroupNorm(1) + GELU -> conv 1x1 -> GroupNorm(1) + GLU ->
// LayerScale -> residual.  The second GroupNorm's statistics come from the sums and Gram
// matrix of the hidden rows (the 1x1 conv output is never formed), and the 1x1 conv runs
// fused with everything after it: on CUDA cores for hidden widths <= 24, as a tensor-core
// conv with a GroupNorm + GLU epilogue above.
// Both DConv layers of a frequency-branch level in one kernel, one CTA per row (b, f), for
// the first level (k_dconv_rows: C = 48, hid = 6, k3 convs of dilation 1 and 2, rows of at
// most kDrMaxT positions).  Returns false (nothing launched) otherwise.  (At C = 96 the
// same kernel is slower than the per-layer path: two CTAs of six warps per SM leave the
// CUDA-core k3 conv latency-bound.)
static bool dconv_rows(const EncW &E, float *y, Half16 *yh, int B, int C, int Fr, int T) {
  if (g_opt_simt || E.ndconv != 2 || Fr <= 1 || !yh || !yh->p || yh->Wp != T || yh->C != C ||
      C != 48 || T > kDrMaxT)
    return false;
  DconvRowArgs a{};
  for (int l = 0; l < 2; l++) {
    const DConvW &dw = E.dconv[l];
    if (!dw.c0.w || !dw.c3.w || !dw.zc || dw.c0.O != C / 8 || dw.c0.KW != 3 ||
        dw.c0.KH != 1 || dw.c0.C != C || dw.c3.O != 2 * C)
      return false;
    DconvRowLayer &L = a.L[l];
    L.w0 = dw.c0.w;
    L.ld0 = dw.c0.ld;
    L.b0 = dw.c0.bias;
    L.g1w = dw.gn1.w;
    L.g1b = dw.gn1.b;
    L.zc = dw.zc;
    L.w3 = dw.c3.w;
    L.ld3 = dw.c3.ld;
    L.b3 = dw.c3.bias;
    L.g4w = dw.gn4.w;
    L.g4b = dw.gn4.b;
    L.scale = dw.scale;
    L.dil = 1 << l;
  }
  a.y = y;
  a.yh = yh->p;
  a.Fr = Fr;
  a.T = T;
  a.ysB = (int64_t)C * Fr * T;
  a.ysC = (int64_t)Fr * T;
  const int hid = C / 8, hidp = (hid + 3) / 4 * 4;
  const size_t sm = (size_t)T * (C + 8) * 2 + (size_t)hid * T * 4 +
                    ((size_t)5 * C * hidp + 7 * (size_t)C) * 4;
  if (sm > 200 * 1024) return false;
  const unsigned rows = (unsigned)((int64_t)B * Fr);
  // minimum bytes: the fp16 row read and written once, y read and written per layer
  TraceScope ts(TR_DCONV, 0.0, (double)rows * T * C * (2.0 * 2 + 8.0 * 2), rows, C, T);
  static size_t attr = 0;
  if (sm > 48 * 1024 && sm > attr) {
    DCB_CUDA(cudaFuncSetAttribute(k_dconv_rows<48, 6, 8>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
    attr = sm;
  }
  k_dconv_rows<48, 6, 8><<<rows, kDrThreads, sm, stream()>>>(a);
  DCB_LAUNCHED();
  return true;
}

static void dconv(const EncW &E, float *y, Half16 *yh, int B, int C, int Fr, int T) {
  if (g_opt_dconv_rows && dconv_rows(E, y, yh, B, C, Fr, T)) return;
  const Img v = freq_rows(B, C, Fr, T);
  const unsigned rows = (unsigned)((int64_t)B * Fr);
  // one CTA per row when there are many short rows (frequency branch); chunked statistics
  // across CTAs when a few rows are long (time branch, lowest frequency level)
  const bool fused = rows >= 128 && (int64_t)2 * C * T <= (256 << 10);
  float *stat = dalloc((size_t)rows * 2);
  for (int d = 0; d < E.ndconv; d++) {
    const DConvW &dw = E.dconv[d];
    const int dil = 1 << d;
    const int hid = dw.c0.O, C2 = dw.c3.O;
    DCB_REQUIRE(dw.zc != nullptr, "dconv: the 1x1 conv of layer %d is not 1x1", d);
    // conv k3, dilation 2^d, padding 2^d -> h [B, hid, Fr, T]; its epilogue also sums each
    // row's values and squares (the first GroupNorm's statistics) into hstat.  Row
    // accumulators (zeroed): hstat [rows][2], the Gram sums acc [rows][npair + hid] and a
    // block counter per row
    const int npair = hid * (hid + 1) / 2;
    const size_t nacc = (size_t)rows * (2 + npair + hid);
    double *hstat = (double *)dalloc(nacc * 2 + rows);
    double *gacc = hstat + 2 * (size_t)rows;
    unsigned *gcnt = (unsigned *)(hstat + nacc);
    DCB_CUDA(cudaMemsetAsync(hstat, 0, nacc * sizeof(double) + rows * sizeof(unsigned),
                             stream()));
    float *h = dalloc((size_t)B * hid * Fr * T);
    const Img hv = freq_rows(B, hid, Fr, T);
    const bool hsums =
        conv_any(dw.c0, y, yh, v, 1, 1, 0, dil, 1, dil, 1, T, h, hv, 0, nullptr, true, nullptr,
                 0.f, 0, hstat);
    RowView rh{h, Fr, (int64_t)hid * Fr * T, T, (int64_t)Fr * T, hid, T};
    // hidden widths >= 24: the hidden rows as fp16 channels-last (channels padded to 8),
    // the A operand of a tensor-core 1x1 conv (narrower ones run on CUDA cores, where the
    // few MACs per output are cheaper than the tensor-core epilogue)
    const int hidp = (hid + 7) / 8 * 8;
    Half16 h16 =
        hid >= 24 && dw.c3g.wt && yh && yh->p ? half_alloc(B, hidp, Fr, T, false) : Half16{};
    float *hg = nullptr;  // the GELU outputs (the new kernel does not work in place)
    if (hsums) {
      // GroupNorm(1) + GELU, the fp16 copy and the z statistics, by chunks of the rows and
      // groups of Gram entries across CTAs (the last CTA of a row finishes its z statistics)
      int chunk = 12288 / hid;
      chunk = chunk > 1024 ? 1024 : chunk / 32 * 32;
      if (chunk > T) chunk = T;
      const int ntot = npair + hid, groups = (ntot + kDgThreads - 1) / kDgThreads;
      const int egroup = (ntot + groups - 1) / groups;
      const size_t sm = (size_t)hid * (chunk | 1) * sizeof(float);
      static size_t attr = 0;
      if (sm > 40 * 1024 && sm > attr) {
        DCB_CUDA(cudaFuncSetAttribute(k_dconv_gn_gram,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
        attr = sm;
      }
      TraceScope ts(TR_DCONV, 0.0,
                    (double)rows * T * ((double)hid * 8.0 + (h16.p ? hidp * 2.0 : 0.0)),
                    rows, hid, T);
      hg = dalloc((size_t)B * hid * Fr * T);
      const dim3 grid((unsigned)((T + chunk - 1) / chunk), rows, (unsigned)groups);
      k_dconv_gn_gram<<<grid, kDgThreads, sm, stream()>>>(rh, hg, dw.gn1.w, dw.gn1.b, 1e-5f,
                                                           hstat, gacc, gcnt, chunk, egroup,
                                                           dw.zc, C2, stat, stat + rows, h16.p,
                                                           hidp);
      DCB_LAUNCHED();
      std::swap(h, hg);  // h: the GELU outputs from here on
    } else if (fused) {
      // GroupNorm(1) + GELU in place with the z statistics, one CTA per row
      const size_t sm = (size_t)hid * T * sizeof(float);
      static size_t attr = 0;
      if (sm > 48 * 1024 && sm > attr) {
        DCB_CUDA(cudaFuncSetAttribute(k_gn_gelu_zstats,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
        attr = sm;
      }
      TraceScope ts(TR_DCONV, 0.0,
                    (double)rows * T * ((double)hid * 8.0 + (h16.p ? hidp * 2.0 : 0.0)),
                    rows, hid, T);
      k_gn_gelu_zstats<<<rows, kGnFusedThreads, sm, stream()>>>(
          rh, h, dw.gn1.w, dw.gn1.b, 1e-5f, dw.zc, C2, stat, stat + rows, h16.p, hidp);
      DCB_LAUNCHED();
    } else {
      const int64_t n = (int64_t)B * hid * Fr * T;
      {
        TraceScope ts(TR_DCONV, 0.0, (double)n * 4.0, rows, hid, T);
        rowview_stats(rh, B, 1e-5f, stat, stat + rows, nullptr);
      }
      {
        TraceScope ts(TR_DCONV, 0.0, (double)n * 8.0, rows, hid, T);
        k_gn_gelu<<<grid_for(n, 256), 256, 0, stream()>>>(rh, h, stat, stat + rows, dw.gn1.w,
                                                         dw.gn1.b, B);
        DCB_LAUNCHED();
      }
      if (h16.p) {
        const int64_t nh = (int64_t)B * Fr * T * (hidp / 8);
        k_to_half_cl<<<grid_for(nh, 256), 256, 0, stream()>>>(
            h, nullptr, h16.p, B, hidp, Fr, T, T, (int64_t)hid * Fr * T, (int64_t)Fr * T, T, hid);
        DCB_LAUNCHED();
      }
      // z statistics from the Gram matrix of fp16(h), accumulated over chunks of each row
      const int chunk = kGramChunk * 6 / hid >= kGramChunk ? kGramChunk : 12288 / hid;
      double *acc = (double *)dalloc((size_t)rows * (npair + hid) * 2);
      DCB_CUDA(cudaMemsetAsync(acc, 0, (size_t)rows * (npair + hid) * sizeof(double), stream()));
      const dim3 gg((unsigned)((T + chunk - 1) / chunk), rows,
                    (unsigned)((npair + hid + kGramPairs - 1) / kGramPairs));
      {
        TraceScope ts(TR_DCONV, 0.0, (double)n * 4.0, rows, hid, T);
        k_gram_chunk<<<gg, 256, (size_t)hid * chunk * sizeof(float), stream()>>>(rh, chunk,
                                                                                  acc);
        DCB_LAUNCHED();
      }
      k_zstats_final<<<(unsigned)rows, 256, 0, stream()>>>(acc, dw.zc, hid, T, C2, (int)rows,
                                                            1e-5f, stat, stat + rows);
      DCB_LAUNCHED();
      dfree(acc);
    }
    bool done = false;
    if (h16.p) {
      // 1x1 conv + GroupNorm + GLU + LayerScale + residual in one tensor-core conv epilogue
      Epi e;
      e.mode = EPI_CONV;
      e.bias = dw.c3g.bias;
      e.act = 3;
      e.y = y;
      e.oN2 = v.N2;
      e.oN1 = v.sN1;
      e.oN2s = v.sN2;
      e.oC = v.sC;
      e.oH = v.sH;
      e.O = C;
      e.Ho = 1;
      e.Wo = T;
      e.res = y;
      e.scale = dw.scale;
      e.gn_mean = stat;
      e.gn_rstd = stat + rows;
      e.gn_w = dw.gn4.w;
      e.gn_b = dw.gn4.b;
      epi_half(e, *yh);
      e.yhH = 1;  // images are the rows (b, f) of yh's [B][Fr][T][C] layout
      done = conv_half(h16.rows(), 1, 1, 1, 1, 0, 0, 1, 1, 1, T, dw.c3g.wt, dw.c3g.rows,
                       dw.c3g.ldt, dw.c3g.ncb, e, dw.c3g.glu_bn);
    }
    dfree(h16.p);
    if (done) {
    } else if (hid <= 24) {
      dconv_tail(dw, h, y, B, C, hid, Fr, T, stat, stat + rows, yh);
    } else {
      conv(dw.c3g, h, nullptr, hv, 1, 1, 0, 0, 1, 1, 1, T, y, v, 3, y, dw.scale, stat,
           stat + rows, &dw.gn4);
      if (yh && yh->p) {
        const int64_t n = rows * (int64_t)T * (C / 8);
        k_to_half_cl<<<grid_for(n, 256), 256, 0, stream()>>>(y, nullptr, yh->p, B, C, Fr, T,
                                                             yh->Wp, (int64_t)C * Fr * T,
                                                             (int64_t)Fr * T, T, C);
        DCB_LAUNCHED();
      }
    }
    dfree(h);
    dfree(hg);
    dfree(hstat);
  }
  dfree(stat);
}

// fp16 copy of a first encoder's input: the im2col'd form when its conv has 8 taps over
// <= 8 channels (the model inputs), else the channel-padded channels-last form
static Half16 first_input(DcbModel *m, bool freq, const float *x, int B, int C, int H, int W) {
  const EncW &E = freq ? m->enc[0] : m->tenc[0];
  const int S = m->cfg.stride, K = m->cfg.kernel_size, pad = K / 4;
  if (E.conv.wi && C <= 8 && K == 8) {
    if (freq) return im2col8(x, B, C, H, W, (H + 2 * pad - K) / S + 1, W, S, pad, 0);
    const int Lp = (W + S - 1) / S * S;
    return im2col8(x, B, C, 1, W, 1, (Lp + 2 * pad - K) / S + 1, S, pad, 1);
  }
  return to_half(x, nullptr, B, C, H, W, !freq, (C + 7) / 8 * 8);
}

// freq encoder (dc_henc with freq = 1): x [B, Cin, H, W] (+ fp16 companion xh, or null) ->
// z [B, Cout, H/S, W] and its companion zh
static float *enc_freq(DcbModel *m, int idx, const float *x, const Half16 *xh, int B, int H,
                       int W, int *Ho_out, Half16 *zh) {
  const EncW &E = m->enc[idx];
  const int S = m->cfg.stride, K = m->cfg.kernel_size, pad = K / 4;
  const int Ho = (H + 2 * pad - K) / S + 1;
  const int C = E.Cout;
  float *y = dalloc((size_t)B * C * Ho * W);
  Half16 yh = half_alloc(B, C, Ho, W, false);
  conv_any(E.conv, x, xh, contiguous(B, E.Cin, H, W), S, 1, pad, 0, 1, 1, Ho, W, y,
           contiguous(B, C, Ho, W), 1, &yh, false);
  dconv(E, y, &yh, B, C, Ho, W);
  float *z = dalloc((size_t)B * C * Ho * W);
  *zh = half_alloc(B, C, Ho, W, false);
  const int ce = m->cfg.context_enc;
  const bool emb = idx == 0 && m->freq_emb;
  conv_any(E.rewrite, y, &yh, contiguous(B, C, Ho, W), 1, 1, ce, ce, 1, 1, Ho, W, z,
           contiguous(B, C, Ho, W), 2, zh, false, emb ? m->freq_emb : nullptr,
           m->cfg.freq_emb * m->cfg.emb_scale, m->fe_cols);
  dfree(y);
  dfree(yh.p);
  *Ho_out = Ho;
  return z;
}

// time encoder: x [B, Cin, L] (+ companion) -> z [B, Cout, ceil(L/S)] and its companion
static float *enc_time(DcbModel *m, int idx, const float *x, const Half16 *xh, int B, int L,
                       int *Lo_out, Half16 *zh) {
  const EncW &E = m->tenc[idx];
  const int S = m->cfg.stride, K = m->cfg.kernel_size, pad = K / 4;
  const int Lp = (L + S - 1) / S * S;  // zero pad to a multiple of the stride (layers.c:88-94)
  const int Lo = (Lp + 2 * pad - K) / S + 1;
  const int C = E.Cout;
  float *y = dalloc((size_t)B * C * Lo);
  Half16 yh = half_alloc(B, C, 1, Lo, false);
  conv_any(E.conv, x, xh, contiguous(B, E.Cin, 1, L), 1, S, 0, pad, 1, 1, 1, Lo, y,
           contiguous(B, C, 1, Lo), 1, &yh, false);
  dconv(E, y, &yh, B, C, 1, Lo);
  float *z = dalloc((size_t)B * C * Lo);
  *zh = half_alloc(B, C, 1, Lo, true);  // read with stride 4 by the next encoder
  const int ce = m->cfg.context_enc;
  conv_any(E.rewrite, y, &yh, contiguous(B, C, 1, Lo), 1, 1, 0, ce, 1, 1, 1, Lo, z,
           contiguous(B, C, 1, Lo), 2, zh, false);
  dfree(y);
  dfree(yh.p);
  *Lo_out = Lo;
  return z;
}

// The last frequency decoder's output written straight as the inverse STFT's frame-major
// spectrum (de-normalised), in place of the NCHW tensor: z [B * rows][frames][bins]
struct SpecOut {
  float2 *z = nullptr;
  int rows = 0;  // complex rows per batch item (sources x audio channels)
  const float *mean = nullptr, *var = nullptr;
  float eps = 0.f;
  bool done = false;  // the decoder wrote z (else it produced y as usual)
};

// transposed conv of a decoder from the fp16 companion zh of its input: y (fp32, optional)
// and the fp16 companion of (y + skip_next) for the next decoder (optional), or the
// spectrum of spec (y, skip_next and yh absent)
static bool convtr_half(const ConvW &cw, const Half16 &zh, bool axis_h, int S, int crop,
                        int out_len, bool gelu, float *y, const Img &out, const float *skip_next,
                        Half16 *yh, const SpecOut *spec = nullptr) {
  Epi e;
  e.mode = EPI_CONVTR;
  e.bias = cw.bias;
  e.bias_x = cw.bias_x;
  e.act = gelu ? 1 : 0;
  e.y = y;
  e.oN2 = out.N2;
  e.oN1 = out.sN1;
  e.oN2s = out.sN2;
  e.oC = out.sC;
  e.oH = out.sH;
  e.O = cw.O;
  e.stride = S;
  e.crop = crop;
  e.out_len = out_len;
  e.axis_h = axis_h ? 1 : 0;
  e.hskip = skip_next;
  if (yh) epi_half(e, *yh);
  if (spec) {
    // the frequency transposed conv run along W over a view of zh with H and W swapped
    // (lines = time frames, positions = bins), so that a lane's output bins are
    // contiguous in the frame-major spectrum; one 64-channel block (the K blocks of the
    // two axes are the same taps in the same order only then)
    if (!axis_h || y || yh || skip_next || cw.ncb != 1) return false;
    e.spec_z = spec->z;
    e.spec_rows = spec->rows;
    e.spec_frames = zh.W;
    e.spec_bins = out_len;
    e.spec_mean = spec->mean;
    e.spec_var = spec->var;
    e.spec_eps = spec->eps;
    e.axis_h = 0;
    e.Ho = zh.W;
    e.Wo = zh.H + 1;
    HalfAct v{zh.p, zh.images, zh.C, zh.W, zh.H, zh.H};
    v.sW = zh.Wp;
    v.sH = 1;
    v.sN = (int64_t)zh.H * zh.Wp;
    return conv_half(v, 1, 2, 1, 1, 0, 1, 1, 1, zh.W, zh.H + 1, cw.wt, cw.rows, cw.ldt, cw.ncb,
                     e, 128);
  }
  const int Ho = axis_h ? zh.H + 1 : 1, Wo = axis_h ? zh.W : zh.W + 1;
  e.Ho = Ho;
  e.Wo = Wo;
  return conv_half(zh.act(), axis_h ? 2 : 1, axis_h ? 1 : 2, 1, 1, axis_h ? 1 : 0,
                   axis_h ? 0 : 1, 1, 1, Ho, Wo, cw.wt, cw.rows, cw.ldt, cw.ncb, e, 0);
}

// freq decoder (dc_hdec, layers.c:143-220): input x + skip given as its fp16 companion xs
// (x, skip fp32 for the fallback path) -> y [B, Cout, S*H, W] (fp32 when want_y) and, when
// skip_next is given, the companion of y + skip_next for the next decoder.  With spec (the
// last decoder), the output goes to spec's frame-major spectrum when the tensor-core path
// takes it (spec->done; nullptr returned), else to y as usual.
static float *dec_freq(DcbModel *m, int idx, const float *x, const float *skip, const Half16 *xs,
                       int B, int H, int W, bool last, bool want_y, const float *skip_next,
                       Half16 *yh, SpecOut *spec = nullptr) {
  const DecW &D = m->dec[idx];
  const int C = D.Cin, S = m->cfg.stride, c = m->cfg.context, pad = m->cfg.kernel_size / 4;
  const int out_len = (H - 1) * S + m->cfg.kernel_size - 2 * pad;
  const Img oimg = contiguous(B, D.Cout, out_len, W);
  const bool tma = xs && xs->p && D.rewrite.wt && D.convtr.wt;
  float *y = (want_y && !(spec && tma)) || !tma ? dalloc((size_t)B * D.Cout * out_len * W)
                                               : nullptr;
  if (tma) {
    if (yh) *yh = half_alloc(B, D.Cout, out_len, W, false);
    Half16 zh = half_alloc(B, C, H, W, false);
    conv_any(D.rewrite, nullptr, xs, contiguous(B, C, H, W), 1, 1, c, c, 1, 1, H, W, nullptr,
             contiguous(B, C, H, W), 2, &zh, false);
    if (spec && !skip_next && !yh &&
        convtr_half(D.convtr, zh, true, S, pad, out_len, !last, nullptr, oimg, nullptr,
                    nullptr, spec)) {
      spec->done = true;
      dfree(zh.p);
      return nullptr;
    }
    if (!y) y = dalloc((size_t)B * D.Cout * out_len * W);
    if (!convtr_half(D.convtr, zh, true, S, pad, out_len, !last, y, oimg, skip_next, yh))
      fail("decoder %d: transposed conv not supported", idx);
    dfree(zh.p);
    return y;
  }
  // fp32 path (channel counts the TMA kernel does not take)
  float *z = dalloc((size_t)B * C * H * W);
  conv(D.rewrite, x, skip, contiguous(B, C, H, W), 1, 1, c, c, 1, 1, H, W, z,
       contiguous(B, C, H, W), 2);
  conv_tr(D.convtr, z, contiguous(B, C, H, W), true, S, pad, out_len, !last, y, oimg);
  dfree(z);
  if (yh) *yh = to_half(y, skip_next, B, D.Cout, out_len, W, false);
  return y;
}

// time decoder: input x + skip as the companion xs -> y [B, Cout, length]
static float *dec_time(DcbModel *m, int idx, const float *x, const float *skip, const Half16 *xs,
                       int B, int L, int length, bool last, bool want_y, const float *skip_next,
                       Half16 *yh) {
  const DecW &D = m->tdec[idx];
  const int C = D.Cin, S = m->cfg.stride, c = m->cfg.context, pad = m->cfg.kernel_size / 4;
  const Img oimg = contiguous(B, D.Cout, 1, length);
  const bool tma = xs && xs->p && D.rewrite.wt && D.convtr.wt;
  float *y = want_y || !tma ? dalloc((size_t)B * D.Cout * length) : nullptr;
  if (tma) {
    if (yh) *yh = half_alloc(B, D.Cout, 1, length, false);
    Half16 zh = half_alloc(B, C, 1, L, false);
    conv_any(D.rewrite, nullptr, xs, contiguous(B, C, 1, L), 1, 1, 0, c, 1, 1, 1, L, nullptr,
             contiguous(B, C, 1, L), 2, &zh, false);
    if (!convtr_half(D.convtr, zh, false, S, pad, length, !last, y, oimg, skip_next, yh))
      fail("time decoder %d: transposed conv not supported", idx);
    dfree(zh.p);
    return y;
  }
  float *z = dalloc((size_t)B * C * L);
  conv(D.rewrite, x, skip, contiguous(B, C, 1, L), 1, 1, 0, c, 1, 1, 1, L, z,
       contiguous(B, C, 1, L), 2);
  conv_tr(D.convtr, z, contiguous(B, C, 1, L), false, S, pad, length, !last, y, oimg);
  dfree(z);
  if (yh) *yh = to_half(y, skip_next, B, D.Cout, 1, length, false);
  return y;
}

// ------------------------------------------------------------------ transformer
// positional embeddings (transformer.c:107-158), computed once per token grid on the host
// with the reference's float32 formulas and cached on the device
static const float *pos_2d(DcbModel *m, int C, int Fr, int T1) {
  const long long key = ((long long)1 << 62) | ((long long)C << 40) | ((long long)Fr << 24) | T1;
  auto it = m->pos_cache.find(key);
  if (it != m->pos_cache.end()) return it->second;
  const int half = C / 2, nterm = half / 2;
  std::vector<float> div(nterm), pe((size_t)T1 * Fr * C);
  const float sc = -logf(m->cfg.t_max_period) / (float)half;
  for (int j = 0; j < nterm; j++) div[j] = expf((float)(2 * j) * sc);
  const float wgt = m->cfg.t_weight_pos_embed;
  for (int t = 0; t < T1; t++)
    for (int f = 0; f < Fr; f++) {
      float *row = &pe[((size_t)t * Fr + f) * C];
      for (int c = 0; c < C; c++) {
        const int cc = c < half ? c : c - half;
        const float pos = c < half ? (float)t : (float)f;
        const float ang = pos * div[cc / 2];
        row[c] = ((cc % 2) == 0 ? sinf(ang) : cosf(ang)) * wgt;
      }
    }
  float *d = nullptr;
  DCB_CUDA(cudaMalloc(&d, pe.size() * sizeof(float)));
  DCB_CUDA(cudaMemcpy(d, pe.data(), pe.size() * sizeof(float), cudaMemcpyHostToDevice));
  m->pos_cache[key] = d;
  return d;
}

static const float *pos_1d(DcbModel *m, int C, int T) {
  const long long key = ((long long)C << 40) | T;
  auto it = m->pos_cache.find(key);
  if (it != m->pos_cache.end()) return it->second;
  const int half = C / 2;
  std::vector<float> pe((size_t)T * C);
  const float wgt = m->cfg.t_weight_pos_embed;
  for (int t = 0; t < T; t++)
    for (int j = 0; j < half; j++) {
      const float den = powf(m->cfg.t_max_period, (float)j / (float)(half - 1));
      const float ph = (float)t / den;
      pe[(size_t)t * C + j] = cosf(ph) * wgt;
      pe[(size_t)t * C + half + j] = sinf(ph) * wgt;
    }
  float *d = nullptr;
  DCB_CUDA(cudaMalloc(&d, pe.size() * sizeof(float)));
  DCB_CUDA(cudaMemcpy(d, pe.data(), pe.size() * sizeof(float), cudaMemcpyHostToDevice));
  m->pos_cache[key] = d;
  return d;
}

static void linear_rows(const LinW &lw, const uint16_t *x16, int64_t R, Epi e) {
  RowsA a{x16, (int64_t)lw.ld, 0};
  RowsA b{lw.w, lw.ld, 0};
  e.bias = lw.bias;
  gemm_rows(R, lw.out, lw.in, a, b, 1, e);
}

// Per-branch work buffers of one transformer layer
struct TBuf {
  uint16_t *ln = nullptr;   // [R][ld] fp16 LN output (query side)
  uint16_t *lnk = nullptr;  // [R][ld] fp16 LN output of the key/value side (cross)
  uint16_t *q = nullptr, *k = nullptr, *vt = nullptr;
  uint16_t *att = nullptr;  // [R][D] fp16 attention output
  uint16_t *hid = nullptr;  // [R][hidden] fp16 FFN hidden
};

// one branch of layer l: x [B, Tq, D] (updated in place); kv side tokens Tk, its LN output
// already in b.lnk for cross layers
static void tlayer_branch(DcbModel *m, const TLayerW &tl, float *x, int B, int Tq, int Tk,
                          TBuf &b) {
  const int D = m->D, H = m->cfg.t_heads, hd = D / H;
  const int64_t R = (int64_t)B * Tq;
  const int64_t Tkp = (Tk + 7) / 8 * 8;
  // attention projections with the head split fused in the epilogue
  Epi eh;
  eh.mode = EPI_HEADS;
  eh.heads = H;
  eh.hd = hd;
  eh.sec_cols = D;
  if (!tl.cross) {
    eh.T = Tq;
    eh.Tp = Tkp;
    eh.sec_ptr[0] = b.q;
    eh.sec_ptr[1] = b.k;
    eh.sec_ptr[2] = b.vt;
    eh.sec_layout[2] = 1;
    linear_rows(tl.qkv, b.ln, R, eh);
  } else {
    eh.T = Tq;
    eh.sec_ptr[0] = b.q;
    linear_rows(tl.qkv, b.ln, R, eh);
    Epi ek = eh;
    ek.T = Tk;
    ek.Tp = Tkp;
    ek.sec_ptr[0] = b.k;
    ek.sec_ptr[1] = b.vt;
    ek.sec_layout[0] = 0;
    ek.sec_layout[1] = 1;
    linear_rows(tl.kv, b.lnk, (int64_t)B * Tk, ek);
  }
  flash_attention(b.q, b.k, b.vt, B, H, Tq, Tk, hd, Tkp, b.att, nullptr);
  // x = x + gamma_1 * (att W_o^T + b_o)
  Epi er;
  er.mode = EPI_ROWS_F32;
  er.out = x;
  er.ldo = D;
  er.res = x;
  er.ldr = D;
  er.gamma = tl.gamma1;
  RowsA a{b.att, D, 0};
  {
    Epi e2 = er;
    e2.bias = tl.out.bias;
    gemm_rows(R, tl.out.out, tl.out.in, a, RowsA{tl.out.w, tl.out.ld, 0}, 1, e2);
  }
  // feed forward: LN -> linear1 + GELU (fp16) -> linear2 + LayerScale residual
  const NormW &nf = tl.cross ? tl.norm3 : tl.norm2;
  layernorm(x, b.ln, nf.w, nf.b, R, D, 1e-5f, true, (int)tl.lin1.ld);
  Epi eg;
  eg.mode = EPI_ROWS_F16;
  eg.act = 1;
  eg.out = b.hid;
  eg.ldo = tl.lin2.ld;
  linear_rows(tl.lin1, b.ln, R, eg);
  // GroupNorm(1) over [Tq, D] per batch, affine on D (norm_out): linear2's epilogue sums
  // each batch item's Tq rows of the updated x (fp64 sums, zeroed here), the apply pass
  // forms the mean and variance from them
  static_assert(kStatSlots == kSumSlots, "row-group sums: slot counts of producer and consumer");
  double *gs = (double *)dalloc((size_t)B * kStatSlots * 4);
  DCB_CUDA(cudaMemsetAsync(gs, 0, (size_t)B * kStatSlots * 2 * sizeof(double), stream()));
  Epi e3 = er;
  e3.gamma = tl.gamma2;
  e3.row_stats = gs;
  e3.stat_rows = Tq;
  linear_rows(tl.lin2, b.hid, R, e3);
  {
    TraceScope ts(TR_NORM, 0.0, (double)B * Tq * D * 8.0, B, D, Tq);  // apply
    norm_apply_last_sums(x, x, gs, tl.norm_out.w, tl.norm_out.b, B, (int64_t)Tq * D, D, 1e-5f);
  }
  dfree(gs);
}

// dc_crosstransformer (transformer.c:160-216): x [B, C, Fr, T1], xt [B, C, T2] in place.
// With `aux`, each layer's time-branch half runs on that stream beside the frequency
// branch's (forked and joined per layer: a cross layer reads both branches' tokens).
static void crosstransformer(DcbModel *m, float *x, float *xt, int B, int Fr, int T1, int T2,
                             cudaStream_t aux) {
  const int D = m->D, H = m->cfg.t_heads, hd = D / H;
  const int N1 = Fr * T1, N2 = T2;
  // with the branches on two streams, each branch's linears take one persistent CTA per SM
  // (the other branch's kernels run beside them); restored on return
  struct UmmaCtas {
    int prev;
    explicit UmmaCtas(int n) : prev(g_umma_ctas_per_sm) { g_umma_ctas_per_sm = n; }
    ~UmmaCtas() { g_umma_ctas_per_sm = prev; }
  } umma_ctas(aux ? 1 : 2);
  float *tx = dalloc((size_t)B * N1 * D), *tt = dalloc((size_t)B * N2 * D);
  // token layout kernels: CTA = kTokT positions of one (b, f), a [D][kTokT + 1] fp32 tile
  DCB_REQUIRE(D <= 1024 && B <= 65535 && Fr <= 65535, "transformer: D %d, B %d, Fr %d", D, B,
              Fr);
  const size_t tok_sm = (size_t)D * (kTokT + 1) * sizeof(float);
  {
    static size_t attr = 0;
    if (tok_sm > 48 * 1024 && tok_sm > attr) {
      DCB_CUDA(cudaFuncSetAttribute(k_tokens_ln_pos,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tok_sm));
      DCB_CUDA(cudaFuncSetAttribute(k_tokens_to_chw,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tok_sm));
      attr = tok_sm;
    }
  }
  {
    k_tokens_ln_pos<<<dim3((unsigned)((T1 + kTokT - 1) / kTokT), (unsigned)Fr, (unsigned)B), 256,
                      tok_sm, stream()>>>(x, tx, m->norm_in.w, m->norm_in.b,
                                          pos_2d(m, D, Fr, T1), B, D, Fr, T1, 1e-5f);
    DCB_LAUNCHED();
    k_tokens_ln_pos<<<dim3((unsigned)((T2 + kTokT - 1) / kTokT), 1u, (unsigned)B), 256, tok_sm,
                      stream()>>>(xt, tt, m->norm_in_t.w, m->norm_in_t.b, pos_1d(m, D, T2), B, D,
                                  1, T2, 1e-5f);
    DCB_LAUNCHED();
  }
  const int ldl = (D + 7) / 8 * 8;
  const int hidden = m->hidden, ldh = (hidden + 7) / 8 * 8;
  TBuf bx, bt;
  const int64_t R1 = (int64_t)B * N1, R2 = (int64_t)B * N2;
  const int64_t Np1 = (N1 + 7) / 8 * 8, Np2 = (N2 + 7) / 8 * 8;
  const int64_t Nmax = N1 > N2 ? N1 : N2, Npmax = Np1 > Np2 ? Np1 : Np2;
  for (TBuf *b : {&bx, &bt}) {
    const int64_t R = b == &bx ? R1 : R2;
    b->ln = halloc((size_t)R * ldl);
    b->lnk = halloc((size_t)(R1 > R2 ? R1 : R2) * ldl);
    b->q = halloc((size_t)B * H * Nmax * hd);
    b->k = halloc((size_t)B * H * Nmax * hd);
    b->vt = halloc((size_t)B * H * hd * Npmax);
    b->att = halloc((size_t)R * D);
    b->hid = halloc((size_t)R * ldh);
  }
  const cudaStream_t s_main = stream();
  for (int l = 0; l < m->cfg.t_layers; l++) {
    const TLayerW &lx = m->layers[0][l], &lt = m->layers[1][l];
    if (!lx.cross) {
      if (aux) stream_wait(aux, s_main);
      layernorm(tx, bx.ln, lx.norm1.w, lx.norm1.b, R1, D, 1e-5f, true, ldl);
      tlayer_branch(m, lx, tx, B, N1, N1, bx);
      {
        OnStream os(aux, aux != nullptr);
        layernorm(tt, bt.ln, lt.norm1.w, lt.norm1.b, R2, D, 1e-5f, true, ldl);
        tlayer_branch(m, lt, tt, B, N2, N2, bt);
      }
    } else {
      // both branches read the previous layer's tokens: every LN runs before either branch
      // updates its tokens (two on each stream, then each stream waits for the other's)
      if (aux) stream_wait(aux, s_main);
      layernorm(tx, bx.ln, lx.norm1.w, lx.norm1.b, R1, D, 1e-5f, true, ldl);
      layernorm(tt, bx.lnk, lx.norm2.w, lx.norm2.b, R2, D, 1e-5f, true, ldl);
      {
        OnStream os(aux, aux != nullptr);
        layernorm(tt, bt.ln, lt.norm1.w, lt.norm1.b, R2, D, 1e-5f, true, ldl);
        layernorm(tx, bt.lnk, lt.norm2.w, lt.norm2.b, R1, D, 1e-5f, true, ldl);
      }
      if (aux) {
        stream_wait(s_main, aux);
        stream_wait(aux, s_main);
      }
      tlayer_branch(m, lx, tx, B, N1, N2, bx);
      {
        OnStream os(aux, aux != nullptr);
        tlayer_branch(m, lt, tt, B, N2, N1, bt);
      }
    }
    if (aux) stream_wait(s_main, aux);
  }
  {
    k_tokens_to_chw<<<dim3((unsigned)((T1 + kTokT - 1) / kTokT), (unsigned)Fr, (unsigned)B), 256,
                      tok_sm, stream()>>>(tx, x, B, D, Fr, T1);
    DCB_LAUNCHED();
    k_tokens_to_chw<<<dim3((unsigned)((T2 + kTokT - 1) / kTokT), 1u, (unsigned)B), 256, tok_sm,
                      stream()>>>(tt, xt, B, D, 1, T2);
    DCB_LAUNCHED();
  }
  for (TBuf *b : {&bx, &bt}) {
    dfree(b->ln);
    dfree(b->lnk);
    dfree(b->q);
    dfree(b->k);
    dfree(b->vt);
    dfree(b->att);
    dfree(b->hid);
  }
  dfree(tx);
  dfree(tt);
}

// ------------------------------------------------------------------ forward
static int forward(DcbModel *m, const float *mix_in, int B, int T, float *out, Stage &sg) {
  const Cfg &c = m->cfg;
  const int C = c.audio_channels, L = c.valid_length, nfft = c.nfft, hop = c.hop;
  const int depth = m->depth;
  if (T > L) {
    fail("forward: input length %d exceeds the training length %d", T, L);
    return -1;
  }
  // mix padded to the training length (htdemucs.c:141-147)
  const float *mix = mix_in;
  float *mixp = nullptr;
  if (T < L) {
    mixp = dalloc((size_t)B * C * L);
    k_chunk<<<grid_for((int64_t)B * C * L, 256), 256, 0, stream()>>>(mix_in, mixp, B, C, T, 0, L,
                                                                     (int64_t)C * L);
    DCB_LAUNCHED();
    mix = mixp;
  }
  // spectrogram (stft.c:29-47): two reflect pads then the STFT
  const int le = (L + hop - 1) / hop;
  const int pad = (hop / 2) * 3, extra = pad + le * hop - L;
  const int L1 = L + pad + extra, L2 = L1 + nfft;
  const int nb = nfft / 2;
  float *xp = dalloc((size_t)B * C * L1), *xc = dalloc((size_t)B * C * L2);
  dk_reflect_pad(mix, xp, (int64_t)B * C, L, pad, extra);
  dk_reflect_pad(xp, xc, (int64_t)B * C, L1, nfft / 2, nfft / 2);
  dfree(xp);
  float *stats = dalloc((size_t)B * 4);
  float *mean = stats, *var = stats + B, *meant = stats + 2 * B, *vart = stats + 3 * B;
  const int64_t per_mag = (int64_t)2 * C * nb * le;
  float *x = dalloc((size_t)B * per_mag);
  float *mag = sg.fn ? dalloc((size_t)B * per_mag) : nullptr;
  spec_normalised(xc, B, C, L2, nfft, hop, 2, le, nb, m->window, x, mean, var, mag);
  dfree(xc);
  if (mag) {
    sg.emit("mag", mag, {B, 2 * C, nb, le});
    dfree(mag);
  }
  sg.emit("x_norm", x, {B, 2 * C, nb, le});
  // from here to the transformer the time branch runs on the second stream (the stage
  // callbacks of the tests keep one stream)
  const bool two = g_opt_streams && !sg.fn;
  const cudaStream_t s_main = stream();
  const cudaStream_t s_aux = two ? aux_stream() : s_main;
  if (two) stream_wait(s_aux, s_main);
  std::vector<float *> saved, saved_t;
  std::vector<int> fr_len, t_len;  // H of the freq input, length of the time input
  int H = nb, W = le, Lt = L;
  char name[32];
  float *xt = nullptr;
  {
    // time branch: normalised input, then the encoders
    OnStream os(s_aux, two);
    row_stats(mix, B, (int64_t)C * L, meant, vart);
    xt = dalloc((size_t)B * C * L);
    dk_affine_rows(mix, xt, meant, vart, B, (int64_t)C * L, 1e-5f, 0);
    sg.emit("xt_norm", xt, {B, C, L});
    // fp16 channels-last companion of each encoder input (the first: the normalised input
    // with its few channels padded to 8, or its im2col form)
    Half16 xh_t = first_input(m, false, xt, B, C, 1, L);
    for (int i = 0; i < depth; i++) {
      t_len.push_back(Lt);
      int Lo;
      Half16 zt;
      float *xt2 = enc_time(m, i, xt, &xh_t, B, Lt, &Lo, &zt);
      if (i == 0) dfree(xt);  // the normalised input; encoder outputs live on as skips
      dfree(xh_t.p);
      xh_t = zt;
      xt = xt2;
      Lt = Lo;
      saved_t.push_back(xt);
      snprintf(name, sizeof(name), "tenc_%d", i);
      sg.emit(name, xt, {B, m->tenc[i].Cout, Lt});
    }
    dfree(xh_t.p);
  }
  {
    // frequency branch encoders
    Half16 xh_f = first_input(m, true, x, B, 2 * C, nb, le);
    for (int i = 0; i < depth; i++) {
      fr_len.push_back(H);
      int Ho;
      Half16 zf;
      float *x2 = enc_freq(m, i, x, &xh_f, B, H, W, &Ho, &zf);
      if (i == 0) dfree(x);
      dfree(xh_f.p);
      xh_f = zf;
      x = x2;
      H = Ho;
      saved.push_back(x);
      snprintf(name, sizeof(name), "enc_%d", i);
      sg.emit(name, x, {B, m->enc[i].Cout, H, W});
    }
    dfree(xh_f.p);
  }
  if (two) stream_wait(s_main, s_aux);
  // the encoder outputs are kept as skips; the transformer works on copies
  const int D = m->D;
  float *tx = dalloc((size_t)B * D * H * W), *txt = dalloc((size_t)B * D * Lt);
  DCB_CUDA(cudaMemcpyAsync(tx, x, (size_t)B * D * H * W * 4, cudaMemcpyDeviceToDevice, stream()));
  DCB_CUDA(cudaMemcpyAsync(txt, xt, (size_t)B * D * Lt * 4, cudaMemcpyDeviceToDevice, stream()));
  if (c.t_layers > 0) crosstransformer(m, tx, txt, B, H, W, Lt, two ? s_aux : nullptr);
  sg.emit("transformer_x", tx, {B, D, H, W});
  sg.emit("transformer_xt", txt, {B, D, Lt});
  x = tx;
  xt = txt;
  // decoders (htdemucs.c:198-237).  Each decoder reads x + skip as an fp16 companion, which
  // the previous decoder's transposed conv writes (the first: a conversion of the
  // transformer output); the fp32 outputs are formed only where something reads them.
  // a decoder also writes its fp32 output when the next one reads fp32 (its channel counts
  // take the gather kernel)
  auto tma_dec = [&](const DecW &d) {
    return d.rewrite.wt && d.convtr.wt && d.Cin % 8 == 0;
  };
  // time branch decoders on the second stream
  if (two) stream_wait(s_aux, s_main);
  {
    OnStream os(s_aux, two);
    Half16 xs_t = to_half(xt, saved_t.back(), B, D, 1, Lt, false);
    for (int i = 0; i < depth; i++) {
      const bool last = i == depth - 1;
      const bool want_yt = last || sg.fn || !tma_dec(m->tdec[i + 1]);
      float *skip_t = saved_t.back();
      saved_t.pop_back();
      const int Lin = Lt;
      Lt = t_len.back();
      t_len.pop_back();
      Half16 yt;
      float *xt2 = dec_time(m, i, xt, skip_t, &xs_t, B, Lin, Lt, last, want_yt,
                            last ? nullptr : saved_t.back(), last ? nullptr : &yt);
      dfree(xt);
      dfree(skip_t);
      dfree(xs_t.p);
      xs_t = yt;
      xt = xt2;
      snprintf(name, sizeof(name), "tdec_%d", i);
      if (xt) sg.emit(name, xt, {B, m->tdec[i].Cout, Lt});
    }
    dfree(xs_t.p);
  }
  Half16 xs_f = to_half(x, saved.back(), B, D, H, W, false);
  SpecOut spec;
  for (int i = 0; i < depth; i++) {
    const bool last = i == depth - 1;
    const bool want_y = last || sg.fn || !tma_dec(m->dec[i + 1]);
    float *skip = saved.back();
    saved.pop_back();
    const int Hin = H;
    H = fr_len.back();
    fr_len.pop_back();
    Half16 ys;
    if (last && !sg.fn && m->dec[i].Cout % 2 == 0 && H <= nfft / 2 + 1 &&
        ispec_stream_ok(nfft, hop, W, (int64_t)nfft / 2 + pad, L)) {
      // the inverse STFT reads the decoder's output as a frame-major spectrum, which the
      // transposed conv's epilogue writes directly (de-normalised)
      spec.rows = m->dec[i].Cout / 2;
      spec.mean = mean;
      spec.var = var;
      spec.eps = 1e-5f;
      spec.z = (float2 *)dalloc((size_t)2 * B * spec.rows * W * H);
    }
    float *x2 = dec_freq(m, i, x, skip, &xs_f, B, Hin, W, last, want_y,
                         last ? nullptr : saved.back(), last ? nullptr : &ys,
                         spec.z ? &spec : nullptr);
    dfree(x);
    dfree(skip);
    dfree(xs_f.p);
    xs_f = ys;
    x = x2;
    if (H != (Hin - 1) * c.stride + c.kernel_size - 2 * (c.kernel_size / 4)) {
      fail("decoder %d: frequency length mismatch", i);
    }
    snprintf(name, sizeof(name), "dec_%d", i);
    if (x) sg.emit(name, x, {B, m->dec[i].Cout, H, W});
  }
  dfree(xs_f.p);
  if (two) stream_wait(s_main, s_aux);
  // output (htdemucs.c:242-279)
  const int S = c.n_sources;
  const int Ctot = m->dec[depth - 1].Cout;  // S * 2C
  const int64_t R = (int64_t)B * S * (Ctot / S / 2);
  const int keep = T < L ? T : L;
  const int64_t per = (int64_t)m->tdec[depth - 1].Cout * Lt;
  float *xi = nullptr;
  if (spec.done && !sg.fn) {
    // the output stage (time branch + spectral branch, de-normalised) written by the
    // streamed inverse STFT itself
    StreamCombine cb;
    cb.y = out;
    cb.xt = xt;
    cb.mean = meant;
    cb.var = vart;
    cb.rows = (int)(per / Lt);
    cb.Lt = Lt;
    cb.off = (L - Lt) / 2;
    cb.keep = keep;
    cb.eps = 1e-5f;
    ispec_frames(spec.z, nullptr, R, H, W, m->window, (int64_t)nfft / 2 + pad, L, cb);
  } else {
    xi = dalloc((size_t)R * L);
    if (spec.done)
      ispec_frames(spec.z, xi, R, H, W, m->window, (int64_t)nfft / 2 + pad, L,
                   StreamCombine{});
    else
      ispec_fused(x, xi, mean, var, B, Ctot / 2, H, W, nfft, hop, m->window,
                  (int64_t)nfft / 2 + pad, L, 1e-5f);
    sg.emit("ispec", xi, {B, S, (int)(Ctot / S / 2), L});
    const int64_t n = (int64_t)B * (per / Lt) * keep;
    k_final_combine<<<grid_for(n, 256), 256, 0, stream()>>>(xt, xi, out, meant, vart, B, per, Lt,
                                                           L, keep, 1e-5f);
    DCB_LAUNCHED();
  }
  dfree(spec.z);
  dfree(x);
  sg.emit("stems", out, {B, S, C, keep});
  dfree(xi);
  dfree(xt);
  dfree(stats);
  dfree(mixp);
  return keep;
}

// ------------------------------------------------------------------ graph replay
// Persistent in/out buffers of the forward for a batch shape and slot (allocated once; two
// slots per shape let consecutive batches overlap, each with its own graph).
static FwdGraph *forward_slot(DcbModel *m, int B, int T, int idx) {
  for (auto &g : m->graphs)
    if (g.B == B && g.T == T && g.idx == idx) return &g;
  const Cfg &c = m->cfg;
  FwdGraph g;
  g.B = B;
  g.T = T;
  g.idx = idx;
  if (cudaMalloc(&g.in, (size_t)B * c.audio_channels * T * 4) != cudaSuccess ||
      cudaMalloc(&g.out, (size_t)B * c.n_sources * c.audio_channels * T * 4) != cudaSuccess) {
    (void)cudaGetLastError();
    fail("forward: out of device memory for the %d-segment buffers", B);
    return nullptr;
  }
  m->graphs.push_back(g);
  return &m->graphs.back();
}

// Run the forward on slot->in -> slot->out.  With the "graphs" option the first call runs
// eagerly (growing every lazily sized scratch buffer and cache), the second records the
// whole forward into a CUDA graph on a private stream, and every call from then on replays
// it on the caller's stream; kernel tracing forces the eager path.
static int forward_slot_run(DcbModel *m, FwdGraph *g) {
  Stage none;
  if (!g_opt_graphs || g_trace_mask || !g->warmed) {
    const int r = forward(m, g->in, g->B, g->T, g->out, none);
    g->warmed = true;
    return r;
  }
  if (!m->cap) {
    DCB_CUDA(cudaStreamCreateWithFlags(&m->cap, cudaStreamNonBlocking));
    DCB_CUDA(cudaEventCreateWithFlags(&m->ev_in, cudaEventDisableTiming));
    DCB_CUDA(cudaEventCreateWithFlags(&m->ev_out, cudaEventDisableTiming));
  }
  const cudaStream_t user = stream();
  if (!g->exec) {
    cudaGraph_t graph = nullptr;
    const cudaStream_t prev = stream_override_get();
    // the capture stream starts behind everything issued so far on the caller's stream
    DCB_CUDA(cudaEventRecord(m->ev_in, user));
    DCB_CUDA(cudaStreamWaitEvent(m->cap, m->ev_in, 0));
    set_stream_override(m->cap);
    const uint64_t n0 = launches_now();
    cudaError_t e = cudaStreamBeginCapture(m->cap, cudaStreamCaptureModeThreadLocal);
    int r = -1;
    if (e == cudaSuccess) {
      r = forward(m, g->in, g->B, g->T, g->out, none);
      e = cudaStreamEndCapture(m->cap, &graph);
    }
    set_stream_override(prev);
    if (e != cudaSuccess || r < 0 || !graph) {
      if (graph) cudaGraphDestroy(graph);
      (void)cudaGetLastError();
      fail("forward: CUDA graph capture failed (%s)", cudaGetErrorString(e));
      return -1;
    }
    g->launches = launches_now() - n0;
    add_launches(0 - g->launches);  // recorded, not run: the replay below counts them
    e = cudaGraphInstantiate(&g->exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) {
      g->exec = nullptr;
      fail("forward: CUDA graph instantiation failed (%s)", cudaGetErrorString(e));
      return -1;
    }
  }
  DCB_CUDA(cudaGraphLaunch(g->exec, user));
  add_launches(g->launches);
  return g->T;
}

// ------------------------------------------------------------------ segment scheduler
// CPython's random.Random(seed).randint (MT19937, Matsumoto & Nishimura 1998; seeding by
// init_by_array over the seed's 32-bit words; randbelow by rejection on getrandbits(k)),
// which apply.c:5-107 restates so that shifts match the Python original.
struct Mt {
  uint32_t s[624];
  int i = 625;
  void init(uint32_t v) {
    s[0] = v;
    for (int k = 1; k < 624; k++) s[k] = 1812433253u * (s[k - 1] ^ (s[k - 1] >> 30)) + (uint32_t)k;
    i = 624;
  }
  void seed(uint64_t n) {
    uint32_t key[2];
    int nk = 0;
    if (n == 0) key[nk++] = 0;
    while (n && nk < 2) {
      key[nk++] = (uint32_t)(n & 0xffffffffu);
      n >>= 32;
    }
    init(19650218u);
    int a = 1, b = 0;
    for (int k = 624 > nk ? 624 : nk; k; k--) {
      s[a] = (s[a] ^ ((s[a - 1] ^ (s[a - 1] >> 30)) * 1664525u)) + key[b] + (uint32_t)b;
      a++;
      b++;
      if (a >= 624) {
        s[0] = s[623];
        a = 1;
      }
      if (b >= nk) b = 0;
    }
    for (int k = 623; k; k--) {
      s[a] = (s[a] ^ ((s[a - 1] ^ (s[a - 1] >> 30)) * 1566083941u)) - (uint32_t)a;
      a++;
      if (a >= 624) {
        s[0] = s[623];
        a = 1;
      }
    }
    s[0] = 0x80000000u;
  }
  uint32_t next() {
    if (i >= 624) {
      for (int k = 0; k < 624; k++) {
        const uint32_t y = (s[k] & 0x80000000u) | (s[(k + 1) % 624] & 0x7fffffffu);
        s[k] = s[(k + 397) % 624] ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
      }
      i = 0;
    }
    uint32_t y = s[i++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
  }
  int randint(int lo, int hi) {
    const uint32_t n = (uint32_t)(hi - lo + 1);
    int k = 0;
    for (uint32_t t = n; t; t >>= 1) k++;
    uint32_t v;
    do {
      v = k == 0 ? 0 : next() >> (32 - k);
    } while (v >= n);
    return lo + (int)v;
  }
};

// Fewest groups of at most bs of the items v, in order, sizes differing by at most one:
// every segment is padded to the training length (tails centred, as apply.c:282-293 pads
// them), so full segments and tails share one forward shape, and a segment's result does
// not depend on its batch (normalisation and every kernel are per item).
static std::vector<std::vector<int>> balanced_batches(const std::vector<int> &v, int bs) {
  std::vector<std::vector<int>> out;
  const int n = (int)v.size();
  bs = bs < 1 ? 1 : (bs > 32 ? 32 : bs);
  if (n == 0) return out;
  const int nb = (n + bs - 1) / bs, q = n / nb, r = n % nb;
  int at = 0;
  for (int b = 0; b < nb; b++) {
    const int sz = q + (b < r ? 1 : 0);
    out.emplace_back(v.begin() + at, v.begin() + at + sz);
    at += sz;
  }
  return out;
}

// Items [b, e) of n that shard s of cnt runs: one contiguous block, sizes within one.
static void shard_block(int n, const DcbApplyOpts &o, int &b, int &e) {
  const int cnt = o.shard_count > 1 ? o.shard_count : 1;
  const int s = cnt > 1 ? o.shard_index : 0;
  b = (int)((int64_t)n * s / cnt);
  e = (int)((int64_t)n * (s + 1) / cnt);
}

// One split pass over `length` samples (apply.c:223-237): segment offsets, and this shard's
// forward calls as indices into them.
struct Plan {
  int seg = 0, stride = 0;
  std::vector<int> offsets;
  std::vector<std::vector<int>> batches;
};

static Plan make_plan(const Cfg &c, int length, const DcbApplyOpts &o) {
  Plan p;
  p.seg = (int)((float)c.samplerate * c.segment);
  p.stride = (int)((1.0f - o.overlap) * (float)p.seg);
  if (p.stride <= 0) return p;
  for (int off = 0; off < length; off += p.stride) p.offsets.push_back(off);
  int b, e;
  shard_block((int)p.offsets.size(), o, b, e);
  std::vector<int> mine;
  for (int i = b; i < e; i++) mine.push_back(i);
  p.batches = balanced_batches(mine, o.batch_size);
  return p;
}

// triangular transition weights (apply.c:116-133), float32 math
static std::vector<float> ola_weight(int n, float power) {
  std::vector<float> w(n);
  const int half = n / 2;
  float mx = 0.f;
  for (int i = 0; i < half; i++) w[i] = (float)(i + 1);
  for (int i = half; i < n; i++) w[i] = (float)(n - i);
  for (float v : w) mx = v > mx ? v : mx;
  for (float &v : w) v = powf(v / mx, power);
  return w;
}

// The whole of dc_apply_model's plan (apply.c:179-306) in the coordinates of the final
// output.  Shift pass i (apply.c:184-207) views the track, padded by max_shift zeros on
// both sides, from offset off_i: view position p holds mix[p - d_i] with
// d_i = max_shift - off_i, over a view of T + d_i samples, which is split into segments at
// offsets 0, stride, 2 stride, ...  Each segment is one item: its padded chunk is read
// straight from the mix (no padded or shifted copies of the track) and its kept samples
// land at output positions p - d_i, weighted by the transition weight, the inverse of its
// pass's weight sum (apply.c:295-300) and 1 / shifts (the average over passes).  The items
// of all passes are ordered by output position; a shard runs one contiguous block of them,
// so its output window [lo, hi) spans about 1 / shard_count of the track.
struct Sched {
  int seg = 0, stride = 0;
  float scale = 1.f;
  std::vector<int> pass_noff;  // segments of each pass (their weights sum at each position)
  std::vector<SegItem> items;
  std::vector<std::vector<int>> batches;  // this shard's forward calls (indices into items)
  int64_t lo = 0, hi = 0;                 // this shard's output window
};

static bool make_sched(const Cfg &c, int T, const DcbApplyOpts &o, Sched &sc) {
  sc.seg = (int)((float)c.samplerate * c.segment);
  sc.stride = (int)((1.0f - o.overlap) * (float)sc.seg);
  if (sc.stride <= 0 || sc.seg <= 0) {
    fail("apply: invalid overlap %f", (double)o.overlap);
    return false;
  }
  const int Lv = c.valid_length;
  const int npass = o.shifts > 0 ? o.shifts : 1;
  const int max_shift = o.shifts > 0 ? (int)(0.5f * (float)c.samplerate) : 0;
  sc.scale = 1.0f / (float)npass;
  Mt rng;
  rng.seed(o.use_seed ? (uint64_t)o.seed : 1u);
  for (int i = 0; i < npass; i++) {
    const int64_t d = o.shifts > 0 ? max_shift - rng.randint(0, max_shift) : 0;
    const int64_t L = (int64_t)T + d;  // view length: length + max_shift - offset
    int noff = 0;
    for (int64_t off = 0; off < L; off += sc.stride, noff++) {
      SegItem it;
      it.n = L - off < sc.seg ? L - off : sc.seg;
      if (it.n > Lv) {
        fail("apply: segment longer than the training length");
        return false;
      }
      it.y0 = (Lv - it.n) / 2;  // padded_chunk centring / center_trim
      it.view0 = off;
      it.out0 = off - d;
      it.start = off - it.y0 - d;
      it.pass = i;
      sc.items.push_back(it);
    }
    sc.pass_noff.push_back(noff);
  }
  std::stable_sort(sc.items.begin(), sc.items.end(),
                   [](const SegItem &a, const SegItem &b) { return a.out0 < b.out0; });
  int b, e;
  shard_block((int)sc.items.size(), o, b, e);
  std::vector<int> mine;
  sc.lo = T;
  sc.hi = 0;
  for (int k = b; k < e; k++) {
    mine.push_back(k);
    const SegItem &it = sc.items[k];
    const int64_t a0 = it.out0 < 0 ? 0 : it.out0;
    const int64_t a1 = it.out0 + it.n > T ? T : it.out0 + it.n;
    if (a0 < sc.lo) sc.lo = a0;
    if (a1 > sc.hi) sc.hi = a1;
  }
  if (o.shard_count <= 1) {
    sc.lo = 0;
    sc.hi = T;
  }
  if (sc.hi < sc.lo) sc.hi = sc.lo;
  sc.batches = balanced_batches(mine, o.batch_size);
  return true;
}

// The shard's weighted segments of mix [B, C, T] into its window: win[r][j] += (share of
// output position lo + j) for rows r < B S C, j < hi - lo (row stride ld; the caller zeroes
// the window first).
// Optional per-batch hooks of apply_window: before(k) runs on the host before batch k is
// enqueued (after the batch's input span is known), after(k) once its accumulation is.
struct BatchHooks {
  virtual void before(int k, int64_t in_lo, int64_t in_hi) = 0;
  virtual void after(int k) = 0;
  virtual ~BatchHooks() {}
};

static int apply_window(DcbModel *m, const float *mix, int B, int T, const Sched &sc,
                        float *win, int64_t ld, float power, BatchHooks *hooks = nullptr) {
  const Cfg &c = m->cfg;
  const int C = c.audio_channels, S = c.n_sources, Lv = c.valid_length;
  if (!m->ola_w || m->ola_seg != sc.seg || m->ola_pow != power) {
    // the weights depend only on (segment, power): computed on the host once (float math
    // as apply.c:116-133) and kept on the device
    std::vector<float> w = ola_weight(sc.seg, power);
    DCB_CUDA(cudaStreamSynchronize(stream()));
    cudaFree(m->ola_w);
    m->ola_w = nullptr;
    DCB_CUDA(cudaMalloc(&m->ola_w, (size_t)sc.seg * 4));
    DCB_CUDA(cudaMemcpy(m->ola_w, w.data(), (size_t)sc.seg * 4, cudaMemcpyHostToDevice));
    m->ola_seg = sc.seg;
    m->ola_pow = power;
  }
  const int rows = B * S * C;
  // consecutive batches alternate between the caller's stream and a second one (each with
  // its own slot and graph), so one batch's forward overlaps the next one's; the
  // accumulations into the shared window stay in batch order (each waits for the previous
  // batch), and the caller's stream joins the second one at the end
  const int nb = (int)sc.batches.size();
  const bool ovl = g_opt_streams && nb > 1;
  const cudaStream_t bs0 = stream();
  const cudaStream_t bs1 = ovl ? batch_stream() : bs0;
  if (ovl) stream_wait(bs1, bs0);
  for (int kb = 0; kb < nb; kb++) {
    const auto &bt = sc.batches[kb];
    const int nbt = (int)bt.size();
    const cudaStream_t bsk = (kb & 1) ? bs1 : bs0;
    OnStream os(bsk, ovl);
    FwdGraph *slot = forward_slot(m, nbt * B, Lv, ovl ? (kb & 1) : 0);
    if (!slot) return -1;
    BatchItems bi{};
    bi.cnt = nbt;
    int64_t t0 = sc.hi, t1 = sc.lo;
    for (int k = 0; k < nbt; k++) {
      const SegItem &it = sc.items[bt[k]];
      bi.start[k] = it.start;
      bi.out0[k] = it.out0;
      bi.view0[k] = it.view0;
      bi.y0[k] = it.y0;
      bi.n[k] = it.n;
      bi.noff[k] = sc.pass_noff[it.pass];
      t0 = it.out0 < t0 ? it.out0 : t0;
      t1 = it.out0 + it.n > t1 ? it.out0 + it.n : t1;
    }
    t0 = t0 < sc.lo ? sc.lo : t0;
    t1 = t1 > sc.hi ? sc.hi : t1;
    const int64_t per = (int64_t)B * C * Lv;
    if (hooks) {
      int64_t in_lo = T, in_hi = 0;
      for (int k = 0; k < nbt; k++) {
        in_lo = bi.start[k] < in_lo ? bi.start[k] : in_lo;
        in_hi = bi.start[k] + Lv > in_hi ? bi.start[k] + Lv : in_hi;
      }
      hooks->before(kb, in_lo < 0 ? 0 : in_lo, in_hi > T ? T : in_hi);
    }
    k_chunk_batch<<<dim3(grid_for(per, 256, 148 * 8), (unsigned)nbt), 256, 0, stream()>>>(
        mix, slot->in, B, C, T, Lv, bi);
    DCB_LAUNCHED();
    if (forward_slot_run(m, slot) < 0) return -1;
    if (ovl && kb > 0) stream_wait(bsk, (kb & 1) ? bs0 : bs1);  // batch kb - 1 accumulated
    if (t1 > t0) {
      k_accumulate_items<<<grid_for(t1 - t0, 256, 148 * 16), 256, 0, stream()>>>(
          win, ld, sc.lo, slot->out, m->ola_w, rows, Lv, t0, t1, sc.seg, sc.stride, sc.scale,
          bi);
      DCB_LAUNCHED();
    }
    if (hooks) hooks->after(kb);
  }
  if (ovl) stream_wait(bs0, bs1);
  return 0;
}

// dcb_apply_host's copy pipeline on two copy streams (one per direction, so an upload never
// queues behind a download): before batch k, the part of the track it reads that is not on
// the device yet goes host -> device and the batch waits for it; after batch k, the output
// samples that no later batch touches (those before the first output position of batch
// k + 1; segments are in output order) go device -> host while the next batches compute.
struct HostPipe : BatchHooks {
  DcbModel *m;
  const Sched *sc;
  const float *mix_h;
  float *out_h;
  int64_t T = 0, rows_in = 0, rows_out = 0, in_done = 0, out_done = 0;
  void before(int k, int64_t lo, int64_t hi) override {
    (void)k;
    (void)lo;
    if (hi > in_done) {
      DCB_CUDA(cudaMemcpy2DAsync(m->hmix + in_done, (size_t)T * 4, mix_h + in_done,
                                 (size_t)T * 4, (size_t)(hi - in_done) * 4, (size_t)rows_in,
                                 cudaMemcpyHostToDevice, m->hcp));
      in_done = hi;
      DCB_CUDA(cudaEventRecord(m->hev_in, m->hcp));
      DCB_CUDA(cudaStreamWaitEvent(stream(), m->hev_in, 0));
    }
  }
  void after(int k) override {
    int64_t fin = T;
    if (k + 1 < (int)sc->batches.size()) {
      for (int i : sc->batches[k + 1]) fin = sc->items[i].out0 < fin ? sc->items[i].out0 : fin;
    }
    if (fin < 0) fin = 0;
    if (fin > out_done) flush(fin);
  }
  void flush(int64_t fin) {
    DCB_CUDA(cudaEventRecord(m->hev_out, stream()));
    DCB_CUDA(cudaStreamWaitEvent(m->hcd, m->hev_out, 0));
    DCB_CUDA(cudaMemcpy2DAsync(out_h + out_done, (size_t)T * 4, m->hout + out_done,
                               (size_t)T * 4, (size_t)(fin - out_done) * 4, (size_t)rows_out,
                               cudaMemcpyDeviceToHost, m->hcd));
    out_done = fin;
  }
};

}  // namespace dcb

using namespace dcb;

extern "C" {

int dcb_forward(DcbModel *m, const float *mix, int B, int T, float *out, DcbStageFn fn,
                void *user) {
  if (!m || B <= 0 || T <= 0) return -1;
  Stage sg;
  sg.fn = fn;
  sg.user = user;
  const int r = forward(m, mix, B, T, out, sg);
  return failed() ? -1 : r;
}

int dcb_stage_encoder(DcbModel *m, int branch, int idx, const float *x, int B, int C, int H,
                      int W, float *y, int *out_shape) {
  if (!m || idx < 0 || idx >= m->depth) return -1;
  if (branch == 0) {
    const EncW &E = m->enc[idx];
    if (C != E.Cin) return -1;
    const int S = m->cfg.stride, K = m->cfg.kernel_size;
    const int Ho = (H + 2 * (K / 4) - K) / S + 1;
    out_shape[0] = B;
    out_shape[1] = E.Cout;
    out_shape[2] = Ho;
    out_shape[3] = W;
    if (!y) return 0;
    int ho;
    Half16 xh = idx == 0 ? first_input(m, true, x, B, C, H, W)
                         : to_half(x, nullptr, B, C, H, W, false, (C + 7) / 8 * 8);
    Half16 zh;
    float *z = enc_freq(m, idx, x, &xh, B, H, W, &ho, &zh);
    DCB_CUDA(cudaMemcpyAsync(y, z, (size_t)B * E.Cout * Ho * W * 4, cudaMemcpyDeviceToDevice,
                             stream()));
    dfree(z);
    dfree(zh.p);
    dfree(xh.p);
  } else {
    const EncW &E = m->tenc[idx];
    if (C != E.Cin) return -1;
    const int S = m->cfg.stride, L = W;
    const int Lo = (L + S - 1) / S;
    out_shape[0] = B;
    out_shape[1] = E.Cout;
    out_shape[2] = Lo;
    out_shape[3] = 0;
    if (!y) return 0;
    int lo;
    Half16 xh = idx == 0 ? first_input(m, false, x, B, C, 1, L)
                         : to_half(x, nullptr, B, C, 1, L, true, (C + 7) / 8 * 8);
    Half16 zh;
    float *z = enc_time(m, idx, x, &xh, B, L, &lo, &zh);
    DCB_CUDA(cudaMemcpyAsync(y, z, (size_t)B * E.Cout * Lo * 4, cudaMemcpyDeviceToDevice,
                             stream()));
    dfree(z);
    dfree(zh.p);
    dfree(xh.p);
  }
  DCB_CUDA(cudaStreamSynchronize(stream()));
  return failed() ? -1 : 0;
}

int dcb_stage_decoder(DcbModel *m, int branch, int idx, const float *x, const float *skip,
                      int B, int C, int H, int W, int length, float *y, int *out_shape) {
  if (!m || idx < 0 || idx >= m->depth) return -1;
  const bool last = idx == m->depth - 1;
  const int S = m->cfg.stride, K = m->cfg.kernel_size;
  if (branch == 0) {
    const DecW &D = m->dec[idx];
    if (C != D.Cin) return -1;
    const int Ho = (H - 1) * S + K - 2 * (K / 4);
    out_shape[0] = B;
    out_shape[1] = D.Cout;
    out_shape[2] = Ho;
    out_shape[3] = W;
    if (!y) return 0;
    Half16 xs = to_half(x, skip, B, C, H, W, false);
    float *z = dec_freq(m, idx, x, skip, &xs, B, H, W, last, true, nullptr, nullptr);
    DCB_CUDA(cudaMemcpyAsync(y, z, (size_t)B * D.Cout * Ho * W * 4, cudaMemcpyDeviceToDevice,
                             stream()));
    dfree(z);
    dfree(xs.p);
  } else {
    const DecW &D = m->tdec[idx];
    if (C != D.Cin) return -1;
    out_shape[0] = B;
    out_shape[1] = D.Cout;
    out_shape[2] = length;
    out_shape[3] = 0;
    if (!y) return 0;
    Half16 xs = to_half(x, skip, B, C, 1, W, false);
    float *z = dec_time(m, idx, x, skip, &xs, B, W, length, last, true, nullptr, nullptr);
    DCB_CUDA(cudaMemcpyAsync(y, z, (size_t)B * D.Cout * length * 4, cudaMemcpyDeviceToDevice,
                             stream()));
    dfree(z);
    dfree(xs.p);
  }
  DCB_CUDA(cudaStreamSynchronize(stream()));
  return failed() ? -1 : 0;
}

int dcb_stage_transformer(DcbModel *m, float *x, float *xt, int B, int C, int Fr, int T1,
                          int T2) {
  if (!m || C != m->D) return -1;
  crosstransformer(m, x, xt, B, Fr, T1, T2, nullptr);
  DCB_CUDA(cudaStreamSynchronize(stream()));
  return failed() ? -1 : 0;
}

void dcb_apply_defaults(DcbApplyOpts *o) {
  o->shifts = 1;
  o->split = 1;
  o->overlap = 0.25f;
  o->transition_power = 1.0f;
  o->batch_size = 8;
  o->seed = 1;
  o->use_seed = 0;
  o->shard_index = 0;
  o->shard_count = 1;
}

int dcb_py_randint(uint64_t seed, int lo, int hi, int n, int *out) {
  if (hi < lo || n < 0 || !out) return -1;
  Mt rng;
  rng.seed(seed);
  for (int i = 0; i < n; i++) out[i] = rng.randint(lo, hi);
  return 0;
}

int dcb_segment_plan(int samplerate, float segment, int length, const DcbApplyOpts *o,
                     int *offsets, int *call_of, int cap) {
  if (!o || length <= 0) return -1;
  Cfg c;
  c.samplerate = samplerate;
  c.segment = segment;
  Plan p = make_plan(c, length, *o);
  if (p.stride <= 0) return -1;
  const int n = (int)p.offsets.size();
  if (n > cap) return n;
  for (int i = 0; i < n; i++) {
    offsets[i] = p.offsets[i];
    call_of[i] = -1;
  }
  int call = 0;
  for (auto &b : p.batches) {
    for (int i : b) call_of[i] = call;
    call++;
  }
  return n;
}

int dcb_apply_plan(DcbModel *m, int T, const DcbApplyOpts *o, int *n_forwards, int *n_batched) {
  if (!m || !o || T <= 0) return -1;
  Sched sc;
  if (!make_sched(m->cfg, T, *o, sc)) return -1;
  int fw = 0;
  for (auto &b : sc.batches) fw += (int)b.size();
  if (n_forwards) *n_forwards = fw;
  if (n_batched) *n_batched = (int)sc.batches.size();
  return 0;
}

int dcb_apply_window(int samplerate, float segment, int valid_length, int T,
                     const DcbApplyOpts *o, int64_t *lo, int64_t *hi) {
  if (!o || T <= 0 || samplerate <= 0 || valid_length <= 0) return -1;
  Cfg c;
  c.samplerate = samplerate;
  c.segment = segment;
  c.valid_length = valid_length;
  Sched sc;
  if (!make_sched(c, T, *o, sc)) return -1;
  if (lo) *lo = sc.lo;
  if (hi) *hi = sc.hi;
  return 0;
}

// dc_apply_model (apply.c:179-306): the whole output, or (shard_count > 1) this shard's
// share of it with zeros elsewhere, so that the shards' outputs sum to the full result
int dcb_apply(DcbModel *m, const float *mix, int B, int T, float *out, const DcbApplyOpts *o) {
  if (!m || !o || B <= 0 || T <= 0) return -1;
  if (!o->split) {
    fail("apply: split=0 is not supported by this engine");
    return -1;
  }
  Sched sc;
  if (!make_sched(m->cfg, T, *o, sc)) return -1;
  const int64_t rows = (int64_t)B * m->cfg.n_sources * m->cfg.audio_channels;
  DCB_CUDA(cudaMemsetAsync(out, 0, (size_t)rows * T * 4, stream()));
  if (apply_window(m, mix, B, T, sc, out + sc.lo, T, o->transition_power) < 0) return -1;
  DCB_CUDA(cudaStreamSynchronize(stream()));
  return failed() ? -1 : 0;
}

int dcb_apply_host(DcbModel *m, const float *mix_h, int B, int T, float *out_h,
                   const DcbApplyOpts *o) {
  if (!m || !o || !mix_h || !out_h || B <= 0 || T <= 0) return -1;
  if (!o->split || o->shard_count > 1) {
    fail("apply_host: needs split=1 and the whole track (shards use dcb_apply_shard)");
    return -1;
  }
  Sched sc;
  if (!make_sched(m->cfg, T, *o, sc)) return -1;
  const int C = m->cfg.audio_channels;
  const int64_t rows = (int64_t)B * m->cfg.n_sources * C;
  const size_t nin = (size_t)B * C * T, nout = (size_t)rows * T;
  if (!m->hcp) {
    DCB_CUDA(cudaStreamCreateWithFlags(&m->hcp, cudaStreamNonBlocking));
    DCB_CUDA(cudaStreamCreateWithFlags(&m->hcd, cudaStreamNonBlocking));
    DCB_CUDA(cudaEventCreateWithFlags(&m->hev_in, cudaEventDisableTiming));
    DCB_CUDA(cudaEventCreateWithFlags(&m->hev_out, cudaEventDisableTiming));
  }
  if (nin > m->hmix_cap || nout > m->hout_cap) {
    DCB_CUDA(cudaStreamSynchronize(stream()));
    DCB_CUDA(cudaStreamSynchronize(m->hcp));
    DCB_CUDA(cudaStreamSynchronize(m->hcd));
    if (nin > m->hmix_cap) {
      cudaFree(m->hmix);
      m->hmix = nullptr;
      m->hmix_cap = 0;
      if (cudaMalloc(&m->hmix, nin * 4) != cudaSuccess) {
        (void)cudaGetLastError();
        fail("apply_host: out of device memory for the track (%.1f MB)", nin * 4 / 1e6);
        return -1;
      }
      m->hmix_cap = nin;
    }
    if (nout > m->hout_cap) {
      cudaFree(m->hout);
      m->hout = nullptr;
      m->hout_cap = 0;
      if (cudaMalloc(&m->hout, nout * 4) != cudaSuccess) {
        (void)cudaGetLastError();
        fail("apply_host: out of device memory for the stems (%.1f MB)", nout * 4 / 1e6);
        return -1;
      }
      m->hout_cap = nout;
    }
  }
  if (failed()) return -1;
  // the copy streams start after everything already queued on the caller's stream
  DCB_CUDA(cudaEventRecord(m->hev_out, stream()));
  DCB_CUDA(cudaStreamWaitEvent(m->hcp, m->hev_out, 0));
  DCB_CUDA(cudaStreamWaitEvent(m->hcd, m->hev_out, 0));
  HostPipe hp;
  hp.m = m;
  hp.sc = &sc;
  hp.mix_h = mix_h;
  hp.out_h = out_h;
  hp.T = T;
  hp.rows_in = (int64_t)B * C;
  hp.rows_out = rows;
  DCB_CUDA(cudaMemsetAsync(m->hout, 0, nout * 4, stream()));
  if (apply_window(m, m->hmix, B, T, sc, m->hout, T, o->transition_power, &hp) < 0) return -1;
  if (hp.out_done < T) hp.flush(T);
  DCB_CUDA(cudaStreamSynchronize(m->hcp));
  DCB_CUDA(cudaStreamSynchronize(m->hcd));
  DCB_CUDA(cudaStreamSynchronize(stream()));
  return failed() ? -1 : 0;
}

int dcb_apply_shard(DcbModel *m, const float *mix, int B, int T, float *win, int64_t ld,
                    const DcbApplyOpts *o) {
  if (!m || !o || B <= 0 || T <= 0 || !win) return -1;
  if (!o->split) {
    fail("apply: split=0 is not supported by this engine");
    return -1;
  }
  Sched sc;
  if (!make_sched(m->cfg, T, *o, sc)) return -1;
  if (ld < sc.hi - sc.lo) {
    fail("apply_shard: row stride %lld is shorter than the window (%lld samples)",
         (long long)ld, (long long)(sc.hi - sc.lo));
    return -1;
  }
  const int64_t rows = (int64_t)B * m->cfg.n_sources * m->cfg.audio_channels;
  if (sc.hi > sc.lo) {
    DCB_CUDA(cudaMemset2DAsync(win, (size_t)ld * 4, 0, (size_t)(sc.hi - sc.lo) * 4,
                               (size_t)rows, stream()));
  }
  if (apply_window(m, mix, B, T, sc, win, ld, o->transition_power) < 0) return -1;
  return failed() ? -1 : 0;
}

int dcb_merge_windows(float *out, int64_t rows, int64_t T, const float *wins, int64_t ld,
                      int64_t win_stride, const int64_t *lo, const int64_t *hi, int n) {
  if (!out || rows <= 0 || T <= 0 || n < 0 || n > 64 || (n > 0 && (!wins || !lo || !hi))) {
    fail("merge_windows: invalid arguments (n = %d, at most 64 windows)", n);
    return -1;
  }
  WinList wl{};
  wl.n = n;
  for (int i = 0; i < n; i++) {
    if (lo[i] < 0 || hi[i] > T || hi[i] - lo[i] > ld) {
      fail("merge_windows: window %d [%lld, %lld) outside the track or wider than %lld", i,
           (long long)lo[i], (long long)hi[i], (long long)ld);
      return -1;
    }
    wl.lo[i] = lo[i];
    wl.hi[i] = hi[i];
  }
  k_merge_windows<<<grid_for(T, 256, 148 * 16), 256, 0, stream()>>>(out, rows, T, wins, ld,
                                                                    win_stride, wl);
  DCB_LAUNCHED();
  return failed() ? -1 : 0;
}

}  // extern "C"
