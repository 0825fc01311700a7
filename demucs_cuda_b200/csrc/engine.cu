// htdemucs_6s model engine on the sm_100a kernels: weight loading and packing, the forward
// pass and the segment scheduler.
//
// Mirrors the reference's model layer (htdemucs.c, layers.c, transformer.c, stft.c,
// apply.c) operation by operation, but every GEMM-shaped step is one fused tensor-core
// kernel:
//   encoder conv      implicit-GEMM conv + bias + GELU                    (layers.c:96-121)
//   DConv             k3 conv -> GN+GELU -> 1x1 conv -> GN+GLU+LayerScale residual,
//                     run directly on [B, C, Fr, T] (no transposes)       (layers.c:24-68)
//   rewrite           1x1 / 3x3 conv + bias + GLU (decoder: + skip add in the gather)
//   conv_tr           stride-phase GEMM + bias + crop + GELU              (layers.c:192-216)
//   attention block   LN -> fused QKV GEMM (head-split fp16 epilogue) -> flash attention
//                     -> out-proj GEMM + LayerScale residual -> LN -> linear1 + GELU (fp16)
//                     -> linear2 + LayerScale residual -> GroupNorm(1)   (transformer.c)
// Activations stay fp32 between layers exactly like the reference; every GEMM operand is
// rounded to fp16 (RNE) where the reference rounds it.
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "gemm.cuh"

namespace dcb {

// defined in the other translation-unit parts of the library
void row_stats(const float *x, int64_t rows, int64_t L, float *mean, float *var);
void layernorm(const float *x, void *y, const float *w, const float *b, int64_t rows, int C,
               float eps, bool half_out, int ld_out);
void flash_attention(const uint16_t *q, const uint16_t *k, const uint16_t *vt, int B, int H,
                     int Tq, int Tk, int hd, int64_t Tkp, uint16_t *o16, float *o32);

// ------------------------------------------------------------------ config (config.c:11-264)
struct Cfg {
  int n_sources = 6, samplerate = 44100, nfft = 4096, hop = 1024, audio_channels = 2;
  float segment = 7.8f;
  int channels = 48, channels_time = 0, growth = 2, depth = 4, kernel_size = 8, stride = 4;
  int time_stride = 2, context = 1, context_enc = 0, norm_groups = 4, norm_starts = 4;
  int dconv_mode = 1, dconv_depth = 2, dconv_comp = 8;
  float dconv_init = 1e-3f;
  int rewrite = 1, cac = 1;
  float freq_emb = 0.2f, emb_scale = 10.0f;
  int t_layers = 5, t_heads = 8;
  float t_hidden_scale = 4.0f, t_max_period = 10000.0f, t_weight_pos_embed = 1.0f;
  int t_gelu = 1, t_cross_first = 0, bottom_channels = 0, use_train_segment = 1;
  int wiener_iters = 0, valid_length = 0;
};

// The reference's tolerant key scanner: first occurrence of "key" anywhere, value after
// the colon; "kwargs" entries override (config.c:11-104, 157-264).
static const char *find_key(const char *js, const char *key) {
  char pat[128];
  snprintf(pat, sizeof(pat), "\"%s\"", key);
  const char *p = strstr(js, pat);
  if (!p) return nullptr;
  p = strchr(p + strlen(pat), ':');
  if (!p) return nullptr;
  p++;
  while (*p == ' ' || *p == '\n' || *p == '\t' || *p == '\r') p++;
  return p;
}
static int key_int(const char *js, const char *key, int fb) {
  const char *p = find_key(js, key);
  if (!p) return fb;
  if (!strncmp(p, "true", 4)) return 1;
  if (!strncmp(p, "false", 5)) return 0;
  if (!strncmp(p, "null", 4)) return fb;
  return (int)strtol(p, nullptr, 10);
}
static float key_float(const char *js, const char *key, float fb) {
  const char *p = find_key(js, key);
  if (!p || !strncmp(p, "null", 4)) return fb;
  return strtof(p, nullptr);
}
static int key_str_array_len(const char *js, const char *key) {
  const char *p = find_key(js, key);
  if (!p || *p != '[') return 0;
  int n = 0;
  p++;
  while (*p && *p != ']') {
    while (*p == ' ' || *p == '\n' || *p == '\t' || *p == ',' || *p == '\r') p++;
    if (*p != '"') break;
    p++;
    while (*p && *p != '"') p++;
    if (*p == '"') p++;
    n++;
  }
  return n;
}

static void apply_keys(Cfg &c, const char *js, bool kw) {
#define KI(name) c.name = key_int(js, #name, c.name)
#define KF(name) c.name = key_float(js, #name, c.name)
  if (!kw) {
    int ns = key_str_array_len(js, "sources");
    if (ns > 0) c.n_sources = ns;
    KI(samplerate);
    KF(segment);
    KI(nfft);
    c.hop = key_int(js, "hop_length", c.hop);
    KI(audio_channels);
    KI(valid_length);
  }
  KI(channels);
  KI(channels_time);
  KI(growth);
  KI(depth);
  KI(kernel_size);
  KI(stride);
  KI(time_stride);
  KI(context);
  KI(context_enc);
  KI(norm_groups);
  KI(norm_starts);
  KI(dconv_mode);
  KI(dconv_depth);
  KI(dconv_comp);
  KF(dconv_init);
  KI(rewrite);
  KI(cac);
  KF(freq_emb);
  KF(emb_scale);
  KI(t_layers);
  KI(t_heads);
  KF(t_hidden_scale);
  KF(t_max_period);
  KF(t_weight_pos_embed);
  KI(t_gelu);
  KI(t_cross_first);
  KI(bottom_channels);
  KI(use_train_segment);
  KI(wiener_iters);
  if (kw) {
    KI(nfft);
    KI(samplerate);
  }
#undef KI
#undef KF
}

// The model JSON's text (empty text = the htdemucs_6s defaults).
static bool read_text(const char *path, std::string &js) {
  js.clear();
  if (!path || !path[0]) return true;
  FILE *f = fopen(path, "rb");
  if (!f) {
    fail("cannot read config %s", path);
    return false;
  }
  char buf[4096];
  size_t n;
  while ((n = fread(buf, 1, sizeof(buf), f)) > 0) js.append(buf, n);
  fclose(f);
  return true;
}

static bool load_config(const std::string &js, Cfg &c) {
  c = Cfg();
  c.valid_length = (int)(c.segment * (float)c.samplerate);
  if (!js.empty()) {
    apply_keys(c, js.c_str(), false);
    const char *kw = find_key(js.c_str(), "kwargs");
    if (kw) apply_keys(c, kw, true);
  }
  c.hop = c.nfft / 4;
  if (c.valid_length <= 0) c.valid_length = (int)(c.segment * (float)c.samplerate);
  // this engine implements the htdemucs_6s layer structure
  const char *why = nullptr;
  if (c.wiener_iters != 0) why = "wiener_iters != 0";
  else if (!c.use_train_segment) why = "use_train_segment = 0";
  else if (c.norm_starts < c.depth) why = "outer GroupNorm layers (norm_starts < depth)";
  else if (c.dconv_mode != 1) why = "dconv_mode other than encoder-only";
  else if (!c.cac || !c.rewrite || !c.t_gelu) why = "cac/rewrite/t_gelu disabled";
  else if (c.channels_time && c.channels_time != c.channels) why = "channels_time";
  else if (c.bottom_channels) why = "bottom_channels";
  else if (c.kernel_size != 2 * c.stride) why = "kernel_size != 2 * stride";
  else if (c.depth > 8) why = "depth > 8";
  if (why) {
    fail("unsupported model configuration: %s", why);
    return false;
  }
  return true;
}

// ------------------------------------------------------------------ safetensors
struct StEntry {
  std::string dtype;
  std::vector<int> shape;
  size_t begin = 0, end = 0;
};

static void skip_ws(const char *&p, const char *e) {
  while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) p++;
}
static bool parse_str(const char *&p, const char *e, std::string &out) {
  skip_ws(p, e);
  if (p >= e || *p != '"') return false;
  p++;
  out.clear();
  while (p < e && *p != '"') {
    char ch = *p++;
    if (ch == '\\' && p < e) ch = *p++;
    out.push_back(ch);
  }
  if (p >= e) return false;
  p++;
  return true;
}
static bool parse_u64(const char *&p, const char *e, uint64_t &v) {
  skip_ws(p, e);
  v = 0;
  bool any = false;
  while (p < e && *p >= '0' && *p <= '9') {
    v = v * 10 + (uint64_t)(*p++ - '0');
    any = true;
  }
  return any;
}
static void skip_value(const char *&p, const char *e) {
  skip_ws(p, e);
  int depth = 0;
  bool in_str = false;
  for (; p < e; p++) {
    char ch = *p;
    if (in_str) {
      if (ch == '\\') p++;
      else if (ch == '"') {
        in_str = false;
        if (depth == 0) {
          p++;
          return;
        }
      }
      continue;
    }
    if (ch == '"') in_str = true;
    else if (ch == '{' || ch == '[') depth++;
    else if (ch == '}' || ch == ']') {
      if (--depth <= 0) {
        p++;
        return;
      }
    } else if (depth == 0 && (ch == ',')) return;
  }
}
static bool expect(const char *&p, const char *e, char ch) {
  skip_ws(p, e);
  if (p < e && *p == ch) {
    p++;
    return true;
  }
  return false;
}

static bool parse_st_header(const char *js, size_t len, std::unordered_map<std::string, StEntry> &out) {
  const char *p = js, *e = js + len;
  if (!expect(p, e, '{')) return false;
  while (true) {
    if (expect(p, e, '}')) break;
    std::string key;
    if (!parse_str(p, e, key) || !expect(p, e, ':')) return false;
    if (key == "__metadata__") {
      skip_value(p, e);
    } else {
      StEntry en;
      if (!expect(p, e, '{')) return false;
      while (!expect(p, e, '}')) {
        std::string field;
        if (!parse_str(p, e, field)) return false;
        expect(p, e, ':');
        if (field == "dtype") {
          if (!parse_str(p, e, en.dtype)) return false;
        } else if (field == "shape") {
          expect(p, e, '[');
          while (!expect(p, e, ']')) {
            uint64_t v;
            if (!parse_u64(p, e, v)) return false;
            en.shape.push_back((int)v);
            expect(p, e, ',');
          }
        } else if (field == "data_offsets") {
          uint64_t a, b;
          expect(p, e, '[');
          if (!parse_u64(p, e, a)) return false;
          expect(p, e, ',');
          if (!parse_u64(p, e, b)) return false;
          expect(p, e, ']');
          en.begin = a;
          en.end = b;
        } else {
          skip_value(p, e);
        }
        expect(p, e, ',');
      }
      out[key] = en;
    }
    expect(p, e, ',');
  }
  return true;
}

// ------------------------------------------------------------------ packed layers
struct ConvW {             // B operand of a conv GEMM plus its epilogue constants
  uint16_t *w = nullptr;   // [rows][ld] fp16
  int64_t ld = 0;
  int rows = 0;            // B rows (columns of the GEMM)
  int O = 0, C = 0, KH = 1, KW = 1, K = 0;
  float *bias = nullptr;
  float *bias_x = nullptr; // transposed convs: bias per GEMM column (phase, channel)
  int glu_bn = 0;          // N tile of the GLU interleave (0 = plain)
  // the same rows in the TMA conv kernels' K order (kh, channel block, kw, channel), the
  // channels zero-padded to ncb blocks of 64
  uint16_t *wt = nullptr;
  int64_t ldt = 0;
  int ncb = 0;
  // 8-tap convs over <= 8 input channels (the first encoders): K = (tap, channel padded to
  // 8) = 64, matching the im2col'd fp16 copy of their input
  uint16_t *wi = nullptr;
};
struct LinW {
  uint16_t *w = nullptr;   // [out][ld]
  int64_t ld = 0;
  int out = 0, in = 0;
  float *bias = nullptr;
};
struct NormW {
  float *w = nullptr, *b = nullptr;
};
struct DConvW {
  ConvW c0, c3;
  ConvW c3g;  // c3 with its output halves interleaved for a GLU epilogue
  NormW gn1, gn4;
  float *scale = nullptr;
  // fp64 constants of c3 (fp16 weights W16 [2C][hid], bias b) giving the GroupNorm
  // statistics of z = W16 . h + b from the sums and Gram matrix of h:
  // G = W16^T W16 [hid][hid], u = column sums of W16, v = W16^T b, sum(b), sum(b^2)
  double *zc = nullptr;
};
struct EncW {
  ConvW conv, rewrite;
  DConvW dconv[4];
  int ndconv = 0;
  int Cin = 0, Cout = 0;
};
struct DecW {
  ConvW rewrite, convtr;  // convtr in the stride-phase layout
  int Cin = 0, Cout = 0;
};
struct TLayerW {
  bool cross = false;
  NormW norm1, norm2, norm3, norm_out;
  LinW qkv;  // self: [3D][D]; cross: q only [D][D]
  LinW kv;   // cross: [2D][D]
  LinW out, lin1, lin2;
  float *gamma1 = nullptr, *gamma2 = nullptr;
};

// One captured forward (htdemucs.c:136-280) for a batch shape, with persistent input and
// output buffers so the graph's pointers stay valid across replays.
struct FwdGraph {
  int B = 0, T = 0;
  int idx = 0;  // which of the two alternating slots of this shape (overlapped batches)
  float *in = nullptr, *out = nullptr;
  bool warmed = false;
  cudaGraphExec_t exec = nullptr;
  uint64_t launches = 0;  // kernels per replay
};

}  // namespace dcb

struct DcbModel {
  dcb::Cfg cfg;
  void *block = nullptr;
  size_t block_bytes = 0;
  // what the layout was built from (kept for the packed on-disk image)
  std::string cfg_text, st_header;
  uint64_t st_data_len = 0;
  int depth = 0;
  dcb::EncW enc[8], tenc[8];
  dcb::DecW dec[8], tdec[8];
  float *freq_emb = nullptr;
  int fe_rows = 0, fe_cols = 0;
  dcb::NormW norm_in, norm_in_t;
  dcb::TLayerW layers[2][16];
  float *window = nullptr;
  int D = 0, hidden = 0;
  // cached positional embeddings, keyed by token-grid shape
  std::unordered_map<long long, float *> pos_cache;
  // transition weights of the overlap-add for (segment length, power), on the device
  float *ola_w = nullptr;
  int ola_seg = 0;
  float ola_pow = 0.f;
  // CUDA graphs of the segment forward (option "graphs"), replayed on `cap`
  std::vector<dcb::FwdGraph> graphs;
  cudaStream_t cap = nullptr;
  cudaEvent_t ev_in = nullptr, ev_out = nullptr;
  // dcb_apply_host: upload (hcp) and download (hcd) streams, their events and the device
  // track / stems buffers
  cudaStream_t hcp = nullptr, hcd = nullptr;
  cudaEvent_t hev_in = nullptr, hev_out = nullptr;
  float *hmix = nullptr, *hout = nullptr;
  size_t hmix_cap = 0, hout_cap = 0;
};

namespace dcb {

// staging of the single device block (weights.c:316-360 keeps one 256-aligned block too)
struct Staging {
  std::vector<uint8_t> bytes;
  std::vector<std::pair<size_t, void **>> fix;  // offset -> pointer slot to patch
  size_t add(const void *src, size_t n, void **slot) {
    size_t off = (bytes.size() + 255) & ~(size_t)255;
    bytes.resize(off + n);
    if (src) memcpy(bytes.data() + off, src, n);
    fix.push_back({off, slot});
    return off;
  }
};

struct Loader {
  std::unordered_map<std::string, StEntry> ents;
  const uint8_t *data = nullptr;  // null: layout only (every element reads as zero)
  size_t data_len = 0;
  std::string missing;

  bool has(const std::string &n) const { return ents.count(n) != 0; }
  // element i as float (F32 / F16 / BF16, weights.c:216-236)
  float at(const StEntry &e, size_t i) const {
    if (!data) return 0.f;
    const uint8_t *p = data + e.begin;
    if (e.dtype == "F32") {
      float v;
      memcpy(&v, p + i * 4, 4);
      return v;
    }
    uint16_t h;
    memcpy(&h, p + i * 2, 2);
    if (e.dtype == "F16") return host_h2f(h);
    uint32_t x = (uint32_t)h << 16;
    float v;
    memcpy(&v, &x, 4);
    return v;
  }
  const StEntry *get(const std::string &n) {
    auto it = ents.find(n);
    if (it == ents.end()) {
      if (missing.empty()) missing = n;
      return nullptr;
    }
    return &it->second;
  }
  std::vector<float> f32(const std::string &n, size_t expect_numel = 0) {
    const StEntry *e = get(n);
    std::vector<float> v;
    if (!e) return v;
    size_t numel = 1;
    for (int s : e->shape) numel *= (size_t)s;
    if (expect_numel && numel != expect_numel) {
      if (missing.empty()) missing = n + " (shape)";
      return v;
    }
    v.resize(numel);
    for (size_t i = 0; i < numel; i++) v[i] = at(*e, i);
    return v;
  }
};

static size_t dtype_size(const std::string &d) { return d == "F32" ? 4 : 2; }

static void stage_f32(Staging &st, const std::vector<float> &v, float **slot) {
  st.add(v.data(), v.size() * sizeof(float), (void **)slot);
}

// rows [rows][kp] with K = (kh, kw, c) (channels fastest) -> the TMA im2col K order
// (kh, channel block, kw, c) with channels zero-padded to ncb = ceil(C / 64) blocks
static void stage_tma_order(Staging &st, ConvW &cw, const std::vector<uint16_t> &packed,
                            int rows, int64_t kp, int KH, int KW, int C) {
  const int ncb = (C + 63) / 64;
  const int64_t ldt = (int64_t)KH * KW * ncb * 64;
  std::vector<uint16_t> t((size_t)rows * ldt, 0);
  for (int r = 0; r < rows; r++)
    for (int kh = 0; kh < KH; kh++)
      for (int kw = 0; kw < KW; kw++)
        for (int cb = 0; cb < ncb; cb++) {
          const int n = C - cb * 64 < 64 ? C - cb * 64 : 64;
          memcpy(&t[(size_t)r * ldt + (((size_t)kh * ncb + cb) * KW + kw) * 64],
                 &packed[(size_t)r * kp + ((size_t)kh * KW + kw) * C + (size_t)cb * 64],
                 (size_t)n * 2);
        }
  cw.ncb = ncb;
  cw.ldt = ldt;
  st.add(t.data(), t.size() * 2, (void **)&cw.wt);
}

// GEMM weight in the loader layout: rows o, reduction over the flattened rest, fp16 RNE,
// K padded to 8 (weights.c:306-310, 338-347)
static std::vector<uint16_t> pack_rows(const std::vector<float> &w, int rows, int K, int64_t kp) {
  std::vector<uint16_t> out((size_t)rows * kp, 0);
  for (int r = 0; r < rows; r++)
    for (int k = 0; k < K; k++) out[(size_t)r * kp + k] = host_f2h(w[(size_t)r * K + k]);
  return out;
}

static bool load_conv(Loader &L, Staging &st, const std::string &prefix, ConvW &cw,
                      bool glu, int glu_bn_hint) {
  const StEntry *e = L.get(prefix + ".conv.weight");
  if (!e) return false;
  const int nd = (int)e->shape.size();
  cw.O = e->shape[0];
  cw.C = e->shape[nd - 1];
  cw.KH = nd == 4 ? e->shape[1] : 1;
  cw.KW = nd == 4 ? e->shape[2] : e->shape[1];
  cw.K = cw.KH * cw.KW * cw.C;
  std::vector<float> w = L.f32(prefix + ".conv.weight");
  std::vector<float> b = L.f32(prefix + ".conv.bias", (size_t)cw.O);
  if (w.empty() || b.empty()) return false;
  const int64_t kp = (cw.K + 7) / 8 * 8;
  std::vector<uint16_t> packed = pack_rows(w, cw.O, cw.K, kp);
  cw.ld = kp;
  if (glu) {
    // interleave [a | b] halves per N tile so each tile holds matching GLU pairs
    const int O2 = cw.O / 2, bn = glu_bn_hint, hb = bn / 2, ntiles = (O2 + hb - 1) / hb;
    std::vector<uint16_t> il((size_t)ntiles * bn * kp, 0);
    for (int t = 0; t < ntiles; t++)
      for (int j = 0; j < bn; j++) {
        const int o = t * hb + (j < hb ? j : j - hb);
        if (o >= O2) continue;
        const int src = j < hb ? o : O2 + o;
        memcpy(&il[((size_t)t * bn + j) * kp], &packed[(size_t)src * kp], kp * 2);
      }
    packed.swap(il);
    cw.rows = ntiles * bn;
    cw.glu_bn = bn;
  } else {
    cw.rows = cw.O;
  }
  st.add(packed.data(), packed.size() * 2, (void **)&cw.w);
  stage_tma_order(st, cw, packed, cw.rows, kp, cw.KH, cw.KW, cw.C);
  if (cw.C <= 8 && cw.KH * cw.KW == 8) {
    std::vector<uint16_t> t((size_t)cw.rows * 64, 0);
    for (int r = 0; r < cw.rows; r++)
      for (int tap = 0; tap < 8; tap++)
        memcpy(&t[(size_t)r * 64 + tap * 8], &packed[(size_t)r * kp + (size_t)tap * cw.C],
               (size_t)cw.C * 2);
    st.add(t.data(), t.size() * 2, (void **)&cw.wi);
  }
  stage_f32(st, b, &cw.bias);
  return true;
}

// transposed conv weight [O][Ktaps][(1)][C] -> phase matrix B[(r, o)][(j', c)] =
// W[o][r + S (1 - j')][c] (tap j' = 0 reads input q-1, j' = 1 reads input q)
static bool load_convtr(Loader &L, Staging &st, const std::string &prefix, ConvW &cw, int S,
                        bool axis_h) {
  const StEntry *e = L.get(prefix + ".conv.weight");
  if (!e) return false;
  const int nd = (int)e->shape.size();
  const int O = e->shape[0], C = e->shape[nd - 1];
  const int Kt = nd == 4 ? e->shape[1] * e->shape[2] : e->shape[1];
  if (Kt != 2 * S) {
    fail("%s: transposed-conv kernel %d is not 2 * stride", prefix.c_str(), Kt);
    return false;
  }
  std::vector<float> w = L.f32(prefix + ".conv.weight");
  std::vector<float> b = L.f32(prefix + ".conv.bias", (size_t)O);
  if (w.empty() || b.empty()) return false;
  const int64_t ld = (2 * C + 7) / 8 * 8;
  std::vector<uint16_t> ph((size_t)O * S * ld, 0);
  for (int o = 0; o < O; o++)
    for (int r = 0; r < S; r++)
      for (int jp = 0; jp < 2; jp++) {
        const int tap = r + S * (1 - jp);
        for (int c = 0; c < C; c++)
          ph[((size_t)r * O + o) * ld + jp * C + c] = host_f2h(w[((size_t)o * Kt + tap) * C + c]);
      }
  cw.O = O;
  cw.C = C;
  cw.K = 2 * C;
  cw.ld = ld;
  cw.rows = O * S;
  st.add(ph.data(), ph.size() * 2, (void **)&cw.w);
  // the two taps run along H (frequency decoders) or W (time decoders)
  stage_tma_order(st, cw, ph, cw.rows, ld, axis_h ? 2 : 1, axis_h ? 1 : 2, C);
  stage_f32(st, b, &cw.bias);
  // the bias per GEMM column (phase r, channel o)
  std::vector<float> bx((size_t)O * S);
  for (int r = 0; r < S; r++)
    for (int o = 0; o < O; o++) bx[(size_t)r * O + o] = b[o];
  stage_f32(st, bx, &cw.bias_x);
  return true;
}

static bool load_linear_cat(Loader &L, Staging &st, const std::vector<std::string> &prefixes,
                            LinW &lw) {
  std::vector<float> W, B;
  int in = 0, out = 0;
  for (const auto &p : prefixes) {
    const StEntry *e = L.get(p + ".weight");
    if (!e || e->shape.size() != 2) return false;
    if (in && e->shape[1] != in) return false;
    in = e->shape[1];
    std::vector<float> w = L.f32(p + ".weight");
    std::vector<float> b = L.has(p + ".bias") ? L.f32(p + ".bias", (size_t)e->shape[0])
                                               : std::vector<float>((size_t)e->shape[0], 0.f);
    W.insert(W.end(), w.begin(), w.end());
    B.insert(B.end(), b.begin(), b.end());
    out += e->shape[0];
  }
  const int64_t kp = (in + 7) / 8 * 8;
  std::vector<uint16_t> packed = pack_rows(W, out, in, kp);
  lw.out = out;
  lw.in = in;
  lw.ld = kp;
  st.add(packed.data(), packed.size() * 2, (void **)&lw.w);
  stage_f32(st, B, &lw.bias);
  return true;
}

static bool load_norm(Loader &L, Staging &st, const std::string &p, NormW &nw, int C) {
  std::vector<float> w = L.f32(p + ".weight", (size_t)C), b = L.f32(p + ".bias", (size_t)C);
  if (w.empty() || b.empty()) return false;
  stage_f32(st, w, &nw.w);
  stage_f32(st, b, &nw.b);
  return true;
}

// DConvW::zc for the 1x1 conv at `prefix` (weights [2C][hid] rounded to fp16 as the GEMM
// uses them)
static bool dconv_zconst(Loader &L, Staging &st, const std::string &prefix, DConvW &dw) {
  const int O = dw.c3.O, hid = dw.c3.K;
  if (dw.c3.KH != 1 || dw.c3.KW != 1) return true;  // not a 1x1 conv: no fused statistics
  std::vector<float> w = L.f32(prefix + ".conv.weight");
  std::vector<float> b = L.f32(prefix + ".conv.bias", (size_t)O);
  if (w.size() != (size_t)O * hid || b.empty()) return false;
  std::vector<double> zc((size_t)hid * hid + 2 * hid + 2, 0.0);
  double *G = zc.data(), *u = G + hid * hid, *v = u + hid;
  for (int c = 0; c < O; c++) {
    for (int j = 0; j < hid; j++) {
      const double wj = host_h2f(host_f2h(w[(size_t)c * hid + j]));
      u[j] += wj;
      v[j] += (double)b[c] * wj;
      for (int k = 0; k < hid; k++) G[j * hid + k] += wj * host_h2f(host_f2h(w[(size_t)c * hid + k]));
    }
    zc[(size_t)hid * hid + 2 * hid] += b[c];
    zc[(size_t)hid * hid + 2 * hid + 1] += (double)b[c] * b[c];
  }
  st.add(zc.data(), zc.size() * sizeof(double), (void **)&dw.zc);
  return true;
}

static int glu_bn_for(int O2) {
  // fixed N tile for GLU convs: 2*O2 columns rounded up to a power of two, at most 128, or
  // 96 where that pads fewer columns (O2 = 48, 96: the channels-last conv kernel takes it;
  // the gather path then runs on CUDA cores)
  int bn = 32;
  while (bn < 128 && bn < 2 * O2) bn *= 2;
  const int64_t pad = (2 * O2 + bn - 1) / bn * bn, pad96 = (2 * O2 + 95) / 96 * 96;
  if (2 * O2 > 64 && pad96 < pad) bn = 96;
  return bn;
}

// Every GEMM operand and parameter of the model staged into `st` in the device block's
// layout (the loader rule of weights.c:298-349 plus this engine's derived forms).  With a
// layout-only loader (no tensor data) the layout is the same and the bytes are zeros.
static bool stage_model(DcbModel *m, Loader &L, Staging &st, const char *what) {
  const Cfg &c = m->cfg;
  char p[160];
  bool ok = true;
  m->depth = c.depth;
  for (int i = 0; i < c.depth && ok; i++) {
    EncW &e = m->enc[i];
    snprintf(p, sizeof(p), "encoder.%d.conv", i);
    ok &= load_conv(L, st, p, e.conv, false, 0);
    snprintf(p, sizeof(p), "encoder.%d.rewrite", i);
    if (ok) ok &= load_conv(L, st, p, e.rewrite, true, glu_bn_for(e.conv.O));
    e.Cin = e.conv.C;
    e.Cout = e.conv.O;
    EncW &t = m->tenc[i];
    snprintf(p, sizeof(p), "tencoder.%d.conv", i);
    if (ok) ok &= load_conv(L, st, p, t.conv, false, 0);
    snprintf(p, sizeof(p), "tencoder.%d.rewrite", i);
    if (ok) ok &= load_conv(L, st, p, t.rewrite, true, glu_bn_for(t.conv.O));
    t.Cin = t.conv.C;
    t.Cout = t.conv.O;
    for (int br = 0; br < 2 && ok; br++) {
      EncW &E = br ? t : e;
      E.ndconv = c.dconv_depth;
      for (int d = 0; d < c.dconv_depth && ok; d++) {
        DConvW &dw = E.dconv[d];
        snprintf(p, sizeof(p), "%s.%d.dconv.layers.%d.layers", br ? "tencoder" : "encoder", i, d);
        std::string base(p);
        ok &= load_conv(L, st, base + ".0", dw.c0, false, 0);
        if (ok) ok &= load_conv(L, st, base + ".3", dw.c3, false, 0);
        if (ok) ok &= load_conv(L, st, base + ".3", dw.c3g, true, glu_bn_for(dw.c3.O / 2));
        if (ok) ok &= dconv_zconst(L, st, base + ".3", dw);
        if (ok) ok &= load_norm(L, st, base + ".1", dw.gn1, dw.c0.O);
        if (ok) ok &= load_norm(L, st, base + ".4", dw.gn4, dw.c3.O);
        if (ok) {
          std::vector<float> sc = L.f32(base + ".6.scale", (size_t)E.Cout);
          ok &= !sc.empty();
          if (ok) stage_f32(st, sc, &dw.scale);
        }
      }
    }
  }
  for (int i = 0; i < c.depth && ok; i++) {
    DecW &d = m->dec[i];
    snprintf(p, sizeof(p), "decoder.%d.rewrite", i);
    const StEntry *rw = L.get(std::string(p) + ".conv.weight");
    ok &= rw != nullptr;
    if (ok) ok &= load_conv(L, st, p, d.rewrite, true, glu_bn_for(rw->shape[0] / 2));
    snprintf(p, sizeof(p), "decoder.%d.conv_tr", i);
    if (ok) ok &= load_convtr(L, st, p, d.convtr, c.stride, true);
    d.Cin = d.rewrite.C;
    d.Cout = d.convtr.O;
    DecW &t = m->tdec[i];
    snprintf(p, sizeof(p), "tdecoder.%d.rewrite", i);
    const StEntry *rt = ok ? L.get(std::string(p) + ".conv.weight") : nullptr;
    ok &= rt != nullptr;
    if (ok) ok &= load_conv(L, st, p, t.rewrite, true, glu_bn_for(rt->shape[0] / 2));
    snprintf(p, sizeof(p), "tdecoder.%d.conv_tr", i);
    if (ok) ok &= load_convtr(L, st, p, t.convtr, c.stride, false);
    t.Cin = t.rewrite.C;
    t.Cout = t.convtr.O;
  }
  if (ok && c.freq_emb != 0.0f && L.has("freq_emb.embedding.weight")) {
    const StEntry *e = L.get("freq_emb.embedding.weight");
    m->fe_rows = e->shape[0];
    m->fe_cols = e->shape[1];
    stage_f32(st, L.f32("freq_emb.embedding.weight"), &m->freq_emb);
  }
  m->D = m->enc[c.depth - 1].Cout;
  if (ok && c.t_layers > 0) {
    const int D = m->D;
    ok &= load_norm(L, st, "crosstransformer.norm_in", m->norm_in, D);
    if (ok) ok &= load_norm(L, st, "crosstransformer.norm_in_t", m->norm_in_t, D);
    for (int br = 0; br < 2 && ok; br++) {
      for (int l = 0; l < c.t_layers && ok; l++) {
        TLayerW &tl = m->layers[br][l];
        snprintf(p, sizeof(p), "crosstransformer.%s.%d", br ? "layers_t" : "layers", l);
        std::string b(p);
        tl.cross = (l % 2) != (c.t_cross_first ? 1 : 0);
        const std::string a = b + (tl.cross ? ".cross_attn" : ".attn");
        if (tl.cross) {
          ok &= load_linear_cat(L, st, {a + ".query_proj"}, tl.qkv);
          if (ok) ok &= load_linear_cat(L, st, {a + ".key_proj", a + ".value_proj"}, tl.kv);
        } else {
          ok &= load_linear_cat(L, st, {a + ".query_proj", a + ".key_proj", a + ".value_proj"},
                                tl.qkv);
        }
        if (ok) ok &= load_linear_cat(L, st, {a + ".out_proj"}, tl.out);
        if (ok) ok &= load_linear_cat(L, st, {b + ".linear1"}, tl.lin1);
        if (ok) ok &= load_linear_cat(L, st, {b + ".linear2"}, tl.lin2);
        if (ok) ok &= load_norm(L, st, b + ".norm1", tl.norm1, D);
        if (ok) ok &= load_norm(L, st, b + ".norm2", tl.norm2, D);
        if (ok && tl.cross) ok &= load_norm(L, st, b + ".norm3", tl.norm3, D);
        if (ok) ok &= load_norm(L, st, b + ".norm_out.gn", tl.norm_out, D);
        if (ok) {
          std::vector<float> g1 = L.f32(b + ".gamma_1.scale", (size_t)D);
          std::vector<float> g2 = L.f32(b + ".gamma_2.scale", (size_t)D);
          ok &= !g1.empty() && !g2.empty();
          if (ok) {
            stage_f32(st, g1, &tl.gamma1);
            stage_f32(st, g2, &tl.gamma2);
          }
        }
      }
    }
    m->hidden = m->layers[0][0].lin1.out;
  }
  if (!ok) {
    fail("weights %s: missing or malformed tensor '%s'", what, L.missing.c_str());
    return false;
  }
  // periodic Hann window in double, stored as float (stft.c:5-20)
  std::vector<float> win(c.nfft);
  for (int i = 0; i < c.nfft; i++)
    win[i] = (float)(0.5 - 0.5 * cos(2.0 * 3.14159265358979323846 * (double)i / (double)c.nfft));
  stage_f32(st, win, &m->window);
  return true;
}

// Allocate the device block, fill it from `src` (st's bytes, a packed image, or nothing: a
// zeroed block that a broadcast fills) and point every staged slot into it.
static bool upload_block(DcbModel *m, Staging &st, const uint8_t *src) {
  m->block_bytes = st.bytes.size();
  if (cudaMalloc(&m->block, m->block_bytes ? m->block_bytes : 1) != cudaSuccess) {
    (void)cudaGetLastError();
    fail("out of device memory uploading weights (%.1f MB)", (double)m->block_bytes / 1048576.0);
    return false;
  }
  if (src) {
    DCB_CUDA(cudaMemcpy(m->block, src, m->block_bytes, cudaMemcpyHostToDevice));
  } else {
    DCB_CUDA(cudaMemset(m->block, 0, m->block_bytes));
  }
  for (auto &fx : st.fix) *fx.second = (uint8_t *)m->block + fx.first;
  // the stream-ordered pool keeps freed activation memory for reuse
  cudaMemPool_t pool;
  int dev = 0;
  cudaGetDevice(&dev);
  if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
    uint64_t thr = UINT64_MAX;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
  }
  return !failed();
}

// A model from its config text and safetensors header; `data` (the tensor bytes, or null
// for layout only) and `block` (a packed block image to upload instead of the staged
// bytes, or null).
static DcbModel *build_model(const std::string &cfg_text, const std::string &header,
                             const uint8_t *data, uint64_t data_len, const uint8_t *block,
                             uint64_t block_bytes, bool zero_block, const char *what) {
  DcbModel *m = new DcbModel();
  if (!load_config(cfg_text, m->cfg)) {
    delete m;
    return nullptr;
  }
  m->cfg_text = cfg_text;
  m->st_header = header;
  m->st_data_len = data_len;
  Loader L;
  if (!parse_st_header(header.data(), header.size(), L.ents)) {
    fail("corrupt safetensors header in %s", what);
    delete m;
    return nullptr;
  }
  L.data = data;
  L.data_len = data_len;
  for (auto &kv : L.ents) {
    size_t numel = 1;
    for (int s : kv.second.shape) numel *= (size_t)s;
    const StEntry &e = kv.second;
    if ((e.dtype != "F32" && e.dtype != "F16" && e.dtype != "BF16") || e.end < e.begin ||
        e.end > L.data_len || e.end - e.begin != numel * dtype_size(e.dtype)) {
      fail("bad tensor entry %s (%s)", kv.first.c_str(), e.dtype.c_str());
      delete m;
      return nullptr;
    }
  }
  Staging st;
  if (!stage_model(m, L, st, what)) {
    delete m;
    return nullptr;
  }
  if (block && block_bytes != st.bytes.size()) {
    fail("%s: packed block of %llu bytes, the layout needs %zu", what,
         (unsigned long long)block_bytes, st.bytes.size());
    delete m;
    return nullptr;
  }
  if (!upload_block(m, st, block ? block : (zero_block ? nullptr : st.bytes.data()))) {
    dcb_model_free(m);
    return nullptr;
  }
  return m;
}

// safetensors file: 8-byte little-endian header length, JSON header, tensor data
static bool read_st(const char *path, bool header_only, std::string &header,
                    std::vector<uint8_t> &data, uint64_t &data_len) {
  FILE *f = fopen(path, "rb");
  if (!f) {
    fail("cannot read weights %s", path);
    return false;
  }
  uint8_t lb[8];
  bool ok = fread(lb, 1, 8, f) == 8;
  uint64_t hlen = 0;
  for (int i = 7; i >= 0; i--) hlen = (hlen << 8) | lb[i];
  fseeko(f, 0, SEEK_END);
  const uint64_t size = (uint64_t)ftello(f);
  ok = ok && hlen <= size - 8 && size >= 8;
  if (ok) {
    header.resize(hlen);
    fseeko(f, 8, SEEK_SET);
    ok = fread(&header[0], 1, hlen, f) == hlen;
  }
  data_len = ok ? size - 8 - hlen : 0;
  if (ok && !header_only) {
    data.resize(data_len);
    ok = fread(data.data(), 1, data_len, f) == data_len;
  }
  fclose(f);
  if (!ok) fail("weights file %s is truncated or not safetensors", path);
  return ok;
}

static DcbModel *load_model(const char *st_path, const char *cfg_path, bool layout_only) {
  std::string cfg_text, header;
  std::vector<uint8_t> data;
  uint64_t data_len = 0;
  if (!read_text(cfg_path, cfg_text) || !read_st(st_path, layout_only, header, data, data_len))
    return nullptr;
  return build_model(cfg_text, header, layout_only ? nullptr : data.data(), data_len, nullptr, 0,
                     layout_only, st_path);
}

}  // namespace dcb

using namespace dcb;

extern "C" {

DcbModel *dcb_model_load(const char *st_path, const char *cfg_path) {
  return dcb::load_model(st_path, cfg_path, false);
}

DcbModel *dcb_model_load_layout(const char *st_path, const char *cfg_path) {
  return dcb::load_model(st_path, cfg_path, true);
}

// Packed image: "DCBPACK1", then u64-length-prefixed config text, safetensors header,
// safetensors data length (u64), block bytes, and an FNV-1a 64 checksum of the block.
static const char kPackMagic[8] = {'D', 'C', 'B', 'P', 'A', 'C', 'K', '1'};

static uint64_t fnv1a64(const uint8_t *p, size_t n) {
  uint64_t h = 1469598103934665603ull;
  for (size_t i = 0; i < n; i++) {
    h ^= p[i];
    h *= 1099511628211ull;
  }
  return h;
}

int dcb_model_save_packed(const DcbModel *m, const char *path) {
  if (!m || !m->block || !path) return -1;
  std::vector<uint8_t> blk(m->block_bytes);
  DCB_CUDA(cudaDeviceSynchronize());
  DCB_CUDA(cudaMemcpy(blk.data(), m->block, m->block_bytes, cudaMemcpyDeviceToHost));
  if (failed()) return -1;
  FILE *f = fopen(path, "wb");
  if (!f) {
    fail("cannot write %s", path);
    return -1;
  }
  auto put64 = [&](uint64_t v) {
    uint8_t b[8];
    for (int i = 0; i < 8; i++) b[i] = (uint8_t)(v >> (8 * i));
    return fwrite(b, 1, 8, f) == 8;
  };
  bool ok = fwrite(kPackMagic, 1, 8, f) == 8;
  ok = ok && put64(m->cfg_text.size()) &&
       fwrite(m->cfg_text.data(), 1, m->cfg_text.size(), f) == m->cfg_text.size();
  ok = ok && put64(m->st_header.size()) &&
       fwrite(m->st_header.data(), 1, m->st_header.size(), f) == m->st_header.size();
  ok = ok && put64(m->st_data_len) && put64(blk.size()) &&
       fwrite(blk.data(), 1, blk.size(), f) == blk.size();
  ok = ok && put64(fnv1a64(blk.data(), blk.size()));
  ok = (fclose(f) == 0) && ok;
  if (!ok) {
    fail("short write to %s", path);
    return -1;
  }
  return 0;
}

DcbModel *dcb_model_load_packed(const char *path) {
  FILE *f = path ? fopen(path, "rb") : nullptr;
  if (!f) {
    fail("cannot read packed weights %s", path ? path : "(null)");
    return nullptr;
  }
  auto get64 = [&](uint64_t &v) {
    uint8_t b[8];
    if (fread(b, 1, 8, f) != 8) return false;
    v = 0;
    for (int i = 7; i >= 0; i--) v = (v << 8) | b[i];
    return true;
  };
  char magic[8];
  std::string cfg_text, header;
  std::vector<uint8_t> blk;
  uint64_t n = 0, data_len = 0, sum = 0;
  bool ok = fread(magic, 1, 8, f) == 8 && !memcmp(magic, kPackMagic, 8);
  ok = ok && get64(n) && n < (1u << 24);
  if (ok) {
    cfg_text.resize(n);
    ok = fread(&cfg_text[0], 1, n, f) == n;
  }
  ok = ok && get64(n) && n < (1u << 28);
  if (ok) {
    header.resize(n);
    ok = fread(&header[0], 1, n, f) == n;
  }
  ok = ok && get64(data_len) && get64(n) && n < ((uint64_t)1 << 36);
  if (ok) {
    blk.resize(n);
    ok = fread(blk.data(), 1, n, f) == n;
  }
  ok = ok && get64(sum);
  fclose(f);
  if (!ok) {
    fail("%s is not a packed weight image (or is truncated)", path);
    return nullptr;
  }
  if (fnv1a64(blk.data(), blk.size()) != sum) {
    fail("%s: packed block checksum mismatch", path);
    return nullptr;
  }
  return dcb::build_model(cfg_text, header, nullptr, data_len, blk.data(), blk.size(), false,
                          path);
}

void dcb_model_free(DcbModel *m) {
  if (!m) return;
  cudaStreamSynchronize(stream());
  if (m->cap) cudaStreamSynchronize(m->cap);
  for (auto &g : m->graphs) {
    if (g.exec) cudaGraphExecDestroy(g.exec);
    cudaFree(g.in);
    cudaFree(g.out);
  }
  if (m->ev_in) cudaEventDestroy(m->ev_in);
  if (m->ev_out) cudaEventDestroy(m->ev_out);
  if (m->cap) cudaStreamDestroy(m->cap);
  for (auto &kv : m->pos_cache) cudaFree(kv.second);
  if (m->hcp) cudaStreamSynchronize(m->hcp);
  if (m->hcd) cudaStreamSynchronize(m->hcd);
  if (m->hev_in) cudaEventDestroy(m->hev_in);
  if (m->hev_out) cudaEventDestroy(m->hev_out);
  if (m->hcp) cudaStreamDestroy(m->hcp);
  if (m->hcd) cudaStreamDestroy(m->hcd);
  cudaFree(m->hmix);
  cudaFree(m->hout);
  cudaFree(m->ola_w);
  if (m->block) cudaFree(m->block);
  delete m;
}

int dcb_model_info(const DcbModel *m, int *n_sources, int *audio_channels, int *valid_length,
                   int *samplerate, float *segment) {
  if (!m) return -1;
  if (n_sources) *n_sources = m->cfg.n_sources;
  if (audio_channels) *audio_channels = m->cfg.audio_channels;
  if (valid_length) *valid_length = m->cfg.valid_length;
  if (samplerate) *samplerate = m->cfg.samplerate;
  if (segment) *segment = m->cfg.segment;
  return 0;
}

size_t dcb_model_weight_bytes(const DcbModel *m) { return m ? m->block_bytes : 0; }
void *dcb_model_weight_block(DcbModel *m) { return m ? m->block : nullptr; }

}  // extern "C"
