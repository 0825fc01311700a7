/* Checker-side driver over the reference's own C implementation (CPU backend).
 *
 * TEST INFRASTRUCTURE ONLY.  This file is compiled together with the reference's
 * unchanged sources (worker-cuda/src/*.c, backend_cpu.c) by oracle/Makefile into
 * oracle/_ref/libdcref.so.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg load that library, always as the checker or the timed CPU baseline,
 * never as the product path.  The Makefile's `abi` target links the same file and the
 * same reference model sources against libdc_b200.so instead of backend_cpu.c
 * (oracle/_ref/abi/dcabi): the reference's own model code driving this library through
 * its backend.h ABI, which the GPU tests compare with the CPU build.
 *
 * It exposes plain-pointer entry points (host float arrays, since the CPU backend's
 * "device" pointers are host pointers, backend_cpu.c:46-51) so Python can call:
 *   - the model forward with per-stage dumps, in the order test_compare.c:116-226 checks
 *     (mag, x_norm, xt_norm, enc_i, tenc_i, transformer_x/xt, dec_i, tdec_i, stems),
 *     following dc_htdemucs_forward (htdemucs.c:136-280) call by call;
 *   - dc_apply_model (apply.c:179-306) on a whole track;
 *   - the ops-level conv / conv_tr / linear / attention / norm / spectral wrappers
 *     (ops.c, stft.c) with weights packed by dc_weight_from_host (weights.c:444-489),
 *     i.e. exactly the loader's fp16 rule.
 * Errors inside the reference call dc_die -> exit(1) (util.c:40-55); inputs passed here
 * are validated by the Python side first.
 */
#include "apply.h"
#include "htdemucs.h"
#include "ops.h"

#include <math.h>

typedef void (*dcref_stage_fn)(const char *name, const float *data, int ndim, const int *shape,
                               void *user);

static DcWeights g_w;
static DcModel g_m;
static int g_loaded = 0;

/* Copies go through dc_to_host (tensor.c), so this driver runs unchanged over either
 * backend: the reference's CPU backend (host pointers) or a GPU backend linked in its place
 * (device pointers). */
static void to_host(DcTensor t, float *out) {
  float *h = dc_to_host(t);
  memcpy(out, h, (size_t)dc_numel(t) * sizeof(float));
  free(h);
}

static void emit(dcref_stage_fn fn, void *user, const char *name, DcTensor t) {
  if (!fn) {
    return;
  }
  float *h = dc_to_host(t);
  fn(name, h, t.ndim, t.shape, user);
  free(h);
}

int dcref_load(const char *weights, const char *config) {
  char dev[64];
  dk_init(0, dev, sizeof(dev));
  if (g_loaded) {
    dc_model_free(&g_m);
    dc_weights_free(&g_w);
    g_loaded = 0;
  }
  dc_weights_load(&g_w, weights, config);
  dc_model_init(&g_m, &g_w);
  g_loaded = 1;
  return 0;
}

int dcref_n_sources(void) { return g_loaded ? g_w.cfg.n_sources : -1; }
int dcref_valid_length(void) { return g_loaded ? g_w.cfg.valid_length : -1; }
size_t dcref_weight_block_bytes(void) { return g_loaded ? g_w.block_bytes : 0; }

/* mix [B][C][T] -> stems written to out [B][S][C][Tout]; returns Tout.
 * The stage sequence mirrors htdemucs.c:136-280 so each intermediate can be dumped. */
int dcref_forward(const float *mix_h, int B, int C, int T, float *out, dcref_stage_fn fn,
                  void *user) {
  if (!g_loaded) {
    return -1;
  }
  DcModel *m = &g_m;
  const DcConfig *cfg = &g_w.cfg;
  int s3[3] = {B, C, T};
  DcTensor mix = dc_from_host(mix_h, s3, 3);
  int length_pre_pad = 0;
  int training_length = cfg->valid_length;
  if (cfg->use_train_segment && T < training_length) {
    length_pre_pad = T;
    DcTensor p = dc_pad1d(mix, 0, training_length - T, 0);
    dc_free(mix);
    mix = p;
  }
  DcTensor mag = dc_htdemucs_spec_cac(&m->stft, mix);
  emit(fn, user, "mag", mag);
  int Fq = mag.shape[2], Tf = mag.shape[3];
  DcTensor mean, var, meant, vart;
  dc_batch_stats(mag, &mean, &var);
  DcTensor x = dc_batch_normalize(mag, mean, var, 1e-5f, 0);
  dc_free(mag);
  emit(fn, user, "x_norm", x);
  dc_batch_stats(mix, &meant, &vart);
  DcTensor xt = dc_batch_normalize(mix, meant, vart, 1e-5f, 0);
  dc_free(mix);
  emit(fn, user, "xt_norm", xt);

  DcTensor saved[DC_MAX_DEPTH], saved_t[DC_MAX_DEPTH];
  int lengths[DC_MAX_DEPTH], lengths_t[DC_MAX_DEPTH];
  int n_saved = 0, n_saved_t = 0, n_len = 0, n_lent = 0;
  char name[32];
  for (int idx = 0; idx < m->n_enc; idx++) {
    lengths[n_len++] = x.shape[x.ndim - 1];
    DcTensor inject = dc_empty();
    if (idx < m->n_tenc) {
      lengths_t[n_lent++] = xt.shape[xt.ndim - 1];
      DcTensor xt2 = dc_henc(xt, dc_empty(), m->w, &m->tencoder[idx]);
      dc_free(xt);
      xt = xt2;
      if (!m->tencoder[idx].empty) {
        saved_t[n_saved_t++] = dc_ref(xt);
        snprintf(name, sizeof(name), "tenc_%d", idx);
        emit(fn, user, name, xt);
      } else {
        inject = xt;
      }
    }
    DcTensor x2 = dc_henc(x, inject, m->w, &m->encoder[idx]);
    dc_free(x);
    x = x2;
    if (idx == 0) {
      DcTensor x3 = dc_add_freq_emb(m, x);
      dc_free(x);
      x = x3;
    }
    saved[n_saved++] = dc_ref(x);
    snprintf(name, sizeof(name), "enc_%d", idx);
    emit(fn, user, name, x);
  }
  if (cfg->t_layers > 0) {
    dc_crosstransformer(&x, &xt, m->w, cfg);
    emit(fn, user, "transformer_x", x);
    emit(fn, user, "transformer_xt", xt);
  }
  int offset = m->n_enc - m->n_tdec;
  for (int idx = 0; idx < m->n_dec; idx++) {
    DcTensor skip = saved[--n_saved];
    int len = lengths[--n_len];
    DcTensor pre = dc_empty();
    DcTensor x2 = dc_hdec(x, skip, len, m->w, &m->decoder[idx], &pre);
    dc_free(x);
    dc_free(skip);
    x = x2;
    snprintf(name, sizeof(name), "dec_%d", idx);
    emit(fn, user, name, x);
    if (idx >= offset) {
      DcLayerSpec *tdec = &m->tdecoder[idx - offset];
      int length_t = lengths_t[--n_lent];
      DcTensor xt2;
      if (tdec->empty) {
        DcTensor pre0 = dc_slice_axis(pre, 2, 0, 1);
        DcTensor pre_s = dc_squeeze_axis(pre0, 2);
        dc_free(pre0);
        xt2 = dc_hdec(pre_s, dc_empty(), length_t, m->w, tdec, NULL);
        dc_free(pre_s);
      } else {
        DcTensor skip_t = saved_t[--n_saved_t];
        xt2 = dc_hdec(xt, skip_t, length_t, m->w, tdec, NULL);
        dc_free(skip_t);
      }
      dc_free(xt);
      xt = xt2;
      snprintf(name, sizeof(name), "tdec_%d", idx - offset);
      emit(fn, user, name, xt);
    }
    dc_free(pre);
  }
  int S = cfg->n_sources;
  int Ctot = x.shape[1];
  int r5[5] = {B, S, Ctot / S, Fq, Tf};
  DcTensor xr = dc_reshape(x, r5, 5);
  dc_free(x);
  DcTensor xden = dc_batch_normalize(xr, mean, var, 1e-5f, 1);
  dc_free(xr);
  DcTensor xi = dc_htdemucs_ispec_cac(&m->stft, xden, training_length);
  dc_free(xden);
  emit(fn, user, "ispec", xi);
  int actual = xt.shape[xt.ndim - 1];
  int r4[4] = {B, S, xt.shape[1] / S, actual};
  DcTensor xtr = dc_reshape(xt, r4, 4);
  dc_free(xt);
  DcTensor xtd = dc_batch_normalize(xtr, meant, vart, 1e-5f, 1);
  dc_free(xtr);
  DcTensor xtrim = dc_center_trim(xi, xtd.shape[3]);
  dc_free(xi);
  DcTensor y = dc_add(xtd, xtrim);
  dc_free(xtd);
  dc_free(xtrim);
  int keep = length_pre_pad ? length_pre_pad : training_length;
  if (y.shape[3] > keep) {
    DcTensor y2 = dc_slice_axis(y, 3, 0, keep);
    dc_free(y);
    y = y2;
  }
  emit(fn, user, "stems", y);
  int tout = y.shape[3];
  if (out) {
    to_host(y, out);
  }
  dc_free(y);
  dc_free(mean);
  dc_free(var);
  dc_free(meant);
  dc_free(vart);
  return tout;
}

/* The reference's own forward, unmodified (htdemucs.c:136-280). */
int dcref_forward_plain(const float *mix_h, int B, int C, int T, float *out) {
  if (!g_loaded) {
    return -1;
  }
  int s3[3] = {B, C, T};
  DcTensor mix = dc_from_host(mix_h, s3, 3);
  DcTensor y = dc_htdemucs_forward(&g_m, mix);
  to_host(y, out);
  int tout = y.shape[3];
  dc_free(y);
  dc_free(mix);
  return tout;
}

/* dc_apply_model on mix [B][C][T] -> out [B][S][C][T] (apply.c:179-306). */
int dcref_apply(const float *mix_h, int B, int C, int T, float *out, int shifts, int split,
                float overlap, float transition_power, int batch_size, unsigned seed,
                int use_seed) {
  if (!g_loaded) {
    return -1;
  }
  DcApplyOpts o;
  memset(&o, 0, sizeof(o));
  o.shifts = shifts;
  o.split = split;
  o.overlap = overlap;
  o.transition_power = transition_power;
  o.segment = 0.0f;
  o.batch_size = batch_size;
  o.seed = seed;
  o.use_seed = use_seed;
  int s3[3] = {B, C, T};
  DcTensor mix = dc_from_host(mix_h, s3, 3);
  DcTensor y = dc_apply_model(&g_m, mix, &o);
  to_host(y, out);
  dc_free(y);
  dc_free(mix);
  return 0;
}

/* ------------------------------------------------------------ ops level */

static void copy_out(DcTensor y, float *out) {
  to_host(y, out);
  dc_free(y);
}

int dcref_conv1d(const float *x, int N, int C, int L, const float *w, int O, int K,
                 const float *b, int stride, int pad, int dil, float *y) {
  int xs[3] = {N, C, L}, ws[3] = {O, K, C}, bs[1] = {O};
  DcTensor xt = dc_from_host(x, xs, 3);
  DcWeight W, Bw;
  dc_weight_from_host(&W, "t.conv.weight", w, ws, 3);
  if (b) {
    dc_weight_from_host(&Bw, "t.conv.bias", b, bs, 1);
  }
  DcTensor yt = dc_conv1d(xt, &W, b ? &Bw : NULL, stride, pad, dil);
  int lo = yt.shape[2];
  copy_out(yt, y);
  dc_free(xt);
  dc_weight_release(&W);
  if (b) {
    dc_weight_release(&Bw);
  }
  return lo;
}

int dcref_conv2d(const float *x, int N, int C, int H, int Wd, const float *w, int O, int KH,
                 int KW, const float *b, int sh, int sw, int ph, int pw, float *y) {
  int xs[4] = {N, C, H, Wd}, ws[4] = {O, KH, KW, C}, bs[1] = {O};
  DcTensor xt = dc_from_host(x, xs, 4);
  DcWeight W, Bw;
  dc_weight_from_host(&W, "t.conv.weight", w, ws, 4);
  if (b) {
    dc_weight_from_host(&Bw, "t.conv.bias", b, bs, 1);
  }
  DcTensor yt = dc_conv2d(xt, &W, b ? &Bw : NULL, sh, sw, ph, pw);
  copy_out(yt, y);
  dc_free(xt);
  dc_weight_release(&W);
  if (b) {
    dc_weight_release(&Bw);
  }
  return 0;
}

int dcref_conv_tr2d(const float *x, int N, int C, int H, int Wd, const float *w, int O, int KH,
                    int KW, const float *b, int sh, int sw, float *y) {
  int xs[4] = {N, C, H, Wd}, ws[4] = {O, KH, KW, C}, bs[1] = {O};
  DcTensor xt = dc_from_host(x, xs, 4);
  DcWeight W, Bw;
  dc_weight_from_host(&W, "t.conv_tr.weight", w, ws, 4);
  if (b) {
    dc_weight_from_host(&Bw, "t.conv_tr.bias", b, bs, 1);
  }
  DcTensor yt = dc_conv_tr2d(xt, &W, b ? &Bw : NULL, sh, sw);
  copy_out(yt, y);
  dc_free(xt);
  dc_weight_release(&W);
  if (b) {
    dc_weight_release(&Bw);
  }
  return 0;
}

int dcref_conv_tr1d(const float *x, int N, int C, int L, const float *w, int O, int K,
                    const float *b, int stride, float *y) {
  int xs[3] = {N, C, L}, ws[3] = {O, K, C}, bs[1] = {O};
  DcTensor xt = dc_from_host(x, xs, 3);
  DcWeight W, Bw;
  dc_weight_from_host(&W, "t.conv_tr.weight", w, ws, 3);
  if (b) {
    dc_weight_from_host(&Bw, "t.conv_tr.bias", b, bs, 1);
  }
  DcTensor yt = dc_conv_tr1d(xt, &W, b ? &Bw : NULL, stride);
  copy_out(yt, y);
  dc_free(xt);
  dc_weight_release(&W);
  if (b) {
    dc_weight_release(&Bw);
  }
  return 0;
}

int dcref_linear(const float *x, int R, int IN, const float *w, int OUT, const float *b,
                 float *y) {
  int xs[2] = {R, IN}, ws[2] = {OUT, IN}, bs[1] = {OUT};
  DcTensor xt = dc_from_host(x, xs, 2);
  DcWeight W, Bw;
  dc_weight_from_host(&W, "t.weight", w, ws, 2);
  if (b) {
    dc_weight_from_host(&Bw, "t.bias", b, bs, 1);
  }
  DcTensor yt = dc_linear(xt, &W, b ? &Bw : NULL);
  copy_out(yt, y);
  dc_free(xt);
  dc_weight_release(&W);
  if (b) {
    dc_weight_release(&Bw);
  }
  return 0;
}

int dcref_attention(const float *q, const float *k, const float *v, int B, int Tq, int Tk,
                    int D, int H, float *y) {
  int qs[3] = {B, Tq, D}, ks[3] = {B, Tk, D};
  DcTensor qt = dc_from_host(q, qs, 3), kt = dc_from_host(k, ks, 3), vt = dc_from_host(v, ks, 3);
  DcTensor yt = dc_attention(qt, kt, vt, H);
  copy_out(yt, y);
  dc_free(qt);
  dc_free(kt);
  dc_free(vt);
  return 0;
}

int dcref_groupnorm(const float *x, int B, int C, int S, const float *w, const float *b, int G,
                    int act, float *y) {
  int xs[3] = {B, C, S}, cs[1] = {C};
  DcTensor xt = dc_from_host(x, xs, 3), wt = dc_from_host(w, cs, 1), bt = dc_from_host(b, cs, 1);
  DcTensor yt = dc_groupnorm(xt, wt, bt, G, 1e-5f, act);
  copy_out(yt, y);
  dc_free(xt);
  dc_free(wt);
  dc_free(bt);
  return 0;
}

int dcref_groupnorm_last(const float *x, int B, int T, int C, const float *w, const float *b,
                         float *y) {
  int xs[3] = {B, T, C}, cs[1] = {C};
  DcTensor xt = dc_from_host(x, xs, 3), wt = dc_from_host(w, cs, 1), bt = dc_from_host(b, cs, 1);
  DcTensor yt = dc_groupnorm_last(xt, wt, bt, 1e-5f);
  copy_out(yt, y);
  dc_free(xt);
  dc_free(wt);
  dc_free(bt);
  return 0;
}

int dcref_layernorm(const float *x, int R, int C, const float *w, const float *b, float *y) {
  int xs[2] = {R, C}, cs[1] = {C};
  DcTensor xt = dc_from_host(x, xs, 2), wt = dc_from_host(w, cs, 1), bt = dc_from_host(b, cs, 1);
  DcTensor yt = dc_layer_norm(xt, wt, bt, 1e-5f);
  copy_out(yt, y);
  dc_free(xt);
  dc_free(wt);
  dc_free(bt);
  return 0;
}

/* HTDemucs _spec (cac): mix [B][C][T] -> z [B][2C][nfft/2][frames]; returns frames. */
int dcref_spec(const float *mix, int B, int C, int T, int nfft, float *out) {
  DcStft st = dc_stft_new(nfft, nfft / 4);
  int s3[3] = {B, C, T};
  DcTensor mt = dc_from_host(mix, s3, 3);
  DcTensor z = dc_htdemucs_spec_cac(&st, mt);
  int frames = z.shape[3];
  if (out) {
    to_host(z, out);
  }
  dc_free(z);
  dc_free(mt);
  dc_stft_free(&st);
  return frames;
}

/* HTDemucs _ispec (cac): z [B][S][2C][F][N] -> y [B][S][C][length]. */
int dcref_ispec(const float *z, int B, int S, int C2, int F, int N, int nfft, int length,
                float *y) {
  DcStft st = dc_stft_new(nfft, nfft / 4);
  int s5[5] = {B, S, C2, F, N};
  DcTensor zt = dc_from_host(z, s5, 5);
  DcTensor yt = dc_htdemucs_ispec_cac(&st, zt, length);
  copy_out(yt, y);
  dc_free(zt);
  dc_stft_free(&st);
  return 0;
}

/* fp16 round trip exactly as the reference packs GEMM operands (util.c:246-306). */
void dcref_round_half(const float *x, float *y, int64_t n) {
  for (int64_t i = 0; i < n; i++) {
    y[i] = dc_f16_to_f32(dc_f32_to_f16(x[i]));
  }
}
