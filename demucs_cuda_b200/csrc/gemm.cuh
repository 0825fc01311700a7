// Tensor-core GEMM family (tcgen05 / TMEM / TMA) shared by dk_gemm_half, the
// implicit-GEMM convolutions, the stride-phase transposed convolutions and the transformer
// linears.  Internal C++ interface; the C ABI wrappers are in gemm.cu.
#pragma once

#include "common.cuh"

namespace dcb {

// Implicit im2col over x viewed as images [n][c][h][w] (w contiguous).  Image n is
// n1 * N2 + n2 with element offset n1 * sN1 + n2 * sN2, so a [B, C, Fr, T] tensor can be
// read as B*Fr images [C][T] without the transposes of layers.c:3-20.  The GEMM row is
// the output position p = (n, ho, wo) and the reduction index k = (kh*KW + kw)*C + c,
// matching the packed weight layout (weights.c:298-311, backend.h:108-109).
struct Gather {
  const float *x;
  const float *x2;  // optional second input added element-wise before rounding (decoder skip)
  int N2;
  int64_t sN1, sN2, sC, sH;
  int C, H, W;
  int KH, KW, SH, SW, PH, PW, DH, DW;
  int Ho, Wo;
  int K;  // KH*KW*C
};

enum EpiMode : int {
  EPI_GEMM = 0,    // C = alpha acc + beta C (dk_gemm_half); swapped -> transposed store
  EPI_CONV = 1,    // y[n][o][ho][wo] = act(acc + bias); GLU pairs interleaved columns
  EPI_CONVTR = 2,  // stride-phase scatter: column (r, o) -> output t = S q + r - crop
  EPI_ROWS_F32 = 3,  // out[m][n] = acc + bias (+ res[m][n] + gamma[n] * (...))
  EPI_ROWS_F16 = 4,  // out16[m][n] = fp16(act(acc + bias))
  EPI_HEADS = 5,     // fp16 head-split sections [B][H][T][hd] / [B][H][hd][Tp]
};

constexpr int kStatSlots = 16;

struct Epi {
  int mode = EPI_GEMM;
  int vec = 0;  // 16-column vector stores allowed (set by the launcher after checks)
  const float *bias = nullptr;
  // EPI_CONVTR: the bias per GEMM column (phase, channel), 16-byte aligned (the
  // specialised channels-last epilogue reads it; null: bias[channel])
  const float *bias_x = nullptr;
  int y_al = 0;  // NCHW rows of y are 16-byte aligned (set by the channels-last launcher)
  int cvec = 0;  // row modes: vector stores and 16-byte aligned column constants (launcher)
  int act = 0;  // 0 none, 1 gelu, 2 glu, 3 GroupNorm + glu (EPI_CONV)
  // EPI_GEMM
  float *C = nullptr;
  int64_t ldc = 0, strideC = 0;
  float alpha = 1.f, beta = 0.f;
  int swapped = 0;
  // EPI_CONV / EPI_CONVTR output view: (n, o, h, w) -> n1*oN1 + n2*oN2 + o*oC + h*oH + w
  float *y = nullptr;
  int oN2 = 1;
  int64_t oN1 = 0, oN2s = 0, oC = 0, oH = 0;
  int O = 0;          // output channels (after GLU halving)
  int Ho = 1, Wo = 1;  // GEMM row -> (n, ho, wo)
  int glu_half = 0;    // columns per half inside one N tile (GLU)
  const float *res = nullptr;  // EPI_CONV: y = res + scale[o] * value (DConv residual)
  const float *scale = nullptr;
  // act 3: GroupNorm(1) of the pre-GLU output with per-image statistics (image = row /
  // (Ho * Wo)) and the affine of all 2 * O channels, then GLU
  const float *gn_mean = nullptr, *gn_rstd = nullptr, *gn_w = nullptr, *gn_b = nullptr;
  // EPI_CONVTR
  int stride = 4, crop = 0, out_len = 0, axis_h = 1;
  // fp16 channels-last copy of an EPI_CONV / EPI_CONVTR output (the A operand of the next
  // conv): element (n, o, h, w) of the output at yh[((n * yhH + h) * yhW + w) * yhC + o];
  // hskip (fp32, laid out like y) is added first (the decoders' skip connections).  y may
  // be null when only the copy is needed.
  uint16_t *yh = nullptr;
  int yhH = 1, yhW = 1, yhC = 0;
  const float *hskip = nullptr;
  // EPI_CONV with Ho = 1 (images are rows): per image, the sum and the sum of squares of the
  // output values, added in fp64 to row_stats[2 n], [2 n + 1] (the GroupNorm(1)
  // statistics of a DConv hidden row, formed while the conv writes it)
  // EPI_ROWS_F32: the same sums per group of stat_rows consecutive output rows (group
  // m / stat_rows; the GroupNorm(1) statistics of a transformer branch's [T, D] output),
  // spread over kStatSlots slots per group (row_stats[(g * kStatSlots + slot) * 2 + 0/1],
  // slot = CTA index % kStatSlots) so the atomics of many CTAs do not meet on one address
  double *row_stats = nullptr;
  int64_t stat_rows = 0;
  // EPI_CONVTR along W over a view with the frequency axis as W (the last frequency
  // decoder): instead of y, the de-normalised complex spectrum frame-major,
  // spec_z[(n * spec_rows + o / 2) * spec_frames + h][w] = (v(o) sd + mean, v(o + 1) sd +
  // mean) for even o, h the time frame and w the bin, sd = sqrt(spec_var[n]) + spec_eps,
  // mean = spec_mean[n] (htdemucs.c:242-252) -- the inverse STFT's input, so the decoder
  // output never goes through the NCHW layout
  float2 *spec_z = nullptr;
  int spec_rows = 0, spec_frames = 0, spec_bins = 0;
  const float *spec_mean = nullptr, *spec_var = nullptr;
  float spec_eps = 0.f;
  // frequency embedding added to the output (first frequency encoder, htdemucs.c:114-134):
  // value += emb_alpha * emb[h * emb_ld + o]
  const float *emb = nullptr;
  float emb_alpha = 0.f;
  int emb_ld = 0;
  // EPI_ROWS_*
  void *out = nullptr;
  int64_t ldo = 0, ldr = 0;
  const float *gamma = nullptr;
  // EPI_HEADS
  int T = 0, heads = 0, hd = 0, sec_cols = 0;
  int64_t Tp = 0;
  uint16_t *sec_ptr[3] = {nullptr, nullptr, nullptr};
  int sec_layout[3] = {0, 0, 0};
};

// A operand source for the row-major (TMA) path
struct RowsA {
  const uint16_t *p;
  int64_t ld, stride;  // elements; stride 0 = shared across the batch
};

// C = A . B^T with A [M][K] fp16 rows (TMA), B [N][K] fp16 rows (TMA)
void gemm_rows(int64_t M, int64_t N, int64_t K, RowsA a, RowsA b, int64_t batch, const Epi &e);
// C = gather(x) . B^T with B [N][K] fp16 rows (TMA); M = images * Ho * Wo
void gemm_gather(const Gather &g, int64_t M, const uint16_t *w, int64_t N, int64_t ldw,
                 const Epi &e, int bn_hint = 0, const uint16_t *wt = nullptr,
                 int64_t ldt = 0, int ncb = 0);
// fp16 channels-last activation [images][H][W][C] (W padded to Wp with zeros) feeding the
// TMA implicit-GEMM conv
struct HalfAct {
  const uint16_t *p = nullptr;
  int64_t images = 0;
  int C = 0, H = 1, W = 0, Wp = 0;
  // position strides of a strided view along W, H and images (0: [images][H][Wp]
  // contiguous); e.g. W and H swapped to run a conv along the stored H axis
  int64_t sW = 0, sH = 0, sN = 0;
};
// conv / transposed conv over a HalfAct: taps (KH, KW), stride SH along H and SW (1 or 4)
// along W, padding PH/PW, dilation DH/DW; B = weights in the TMA K order (ldt, ncb).
// Returns false (nothing launched) when the call is outside what the kernel covers.
bool conv_half(const HalfAct &x, int KH, int KW, int SH, int SW, int PH, int PW, int DH, int DW,
               int Ho, int Wo, const uint16_t *wt, int64_t N, int64_t ldt, int ncb, const Epi &e,
               int bn_hint);

// N tile used by gemm_gather for a given column count (the GLU interleave depends on it)
int gather_bn(int64_t M, int64_t N, bool glu);

}  // namespace dcb
