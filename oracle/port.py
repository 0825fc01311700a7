"""numpy restatement of the reference's htdemucs_6s forward and segment scheduler.

TEST INFRASTRUCTURE ONLY (the checker): imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg.  The product path never imports it.

Every function restates the reference algorithm it cites (paths relative to
worker-cuda/src/ of nicapotato/demucs-cuda), keeping the reference's numerics:

* GEMM operands are rounded to fp16 with round-to-nearest-even exactly where the reference
  rounds them (weights at load, weights.c:338-347; activations in dk_im2col_half,
  dk_to_half_rows, dk_transpose_to_half, dk_split_heads_half, dk_softmax_to_half), products
  are accumulated in fp32 (numpy float32 GEMM; the reference uses a sequential fp32 sum,
  backend_cpu.c:444-455, so sums agree to fp32 rounding only);
* row statistics are two-pass in double and stored as float (backend_cpu.c:227-243);
* activations, norms and the STFT are fp32.

Pinned against the reference itself: tests/test_oracle.py compares this port with
oracle/_ref (the reference's own C code) per stage on committed golden fixtures and on a
freshly generated model.
"""
from __future__ import annotations

import math

import numpy as np

F32 = np.float32


def half(x):
    """fp32 -> fp16 (RNE) -> fp32, as dc_f32_to_f16/dc_f16_to_f32 (util.c:246-306)."""
    return np.asarray(x, dtype=F32).astype(np.float16).astype(F32)


def erf32(x):
    from scipy.special import erf
    return erf(x.astype(np.float64)).astype(F32)


def gelu(x):
    """0.5 x (1 + erf(x / sqrt 2)) (backend_cpu.c:144)."""
    x = np.asarray(x, dtype=F32)
    return (F32(0.5) * x * (F32(1.0) + erf32(x * F32(0.70710678118654752)))).astype(F32)


def sigmoid(x):
    x = np.asarray(x, dtype=F32)
    return (F32(1.0) / (F32(1.0) + np.exp(-x))).astype(F32)


def glu(x, axis=1):
    """a * sigmoid(b) over the two halves of `axis` (backend_cpu.c:173-182)."""
    a, b = np.split(x, 2, axis=axis)
    return (a * sigmoid(b)).astype(F32)


def row_stats(x2d):
    """Per-row mean and biased variance, two-pass in double (backend_cpu.c:227-243)."""
    xd = x2d.astype(np.float64)
    m = xd.mean(axis=1)
    v = ((xd - m[:, None]) ** 2).mean(axis=1)
    return m.astype(F32), v.astype(F32)


# ---------------------------------------------------------------- GEMM family


def gemm(a16, b16):
    """C = A . B^T on fp16-valued fp32 operands, fp32 result (dk_gemm_half contract,
    backend.h:117-122)."""
    return np.matmul(a16, b16.T).astype(F32)


def conv2d(x, w, b, sh, sw, ph, pw, dh=1, dw=1):
    """conv_core (ops.c:31-77): im2col with k = (kh*KW + kw)*C + c (backend_cpu.c:346-372),
    fp16 operands, then bias.  x [N,C,H,W], w [O,KH,KW,C]."""
    N, C, H, W = x.shape
    O, KH, KW, _ = w.shape
    Ho = (H + 2 * ph - dh * (KH - 1) - 1) // sh + 1
    Wo = (W + 2 * pw - dw * (KW - 1) - 1) // sw + 1
    xp = np.pad(half(x), ((0, 0), (0, 0), (ph, ph), (pw, pw)))
    cols = np.empty((N, Ho, Wo, KH, KW, C), dtype=F32)
    for kh in range(KH):
        for kw in range(KW):
            h0, w0 = kh * dh, kw * dw
            sl = xp[:, :, h0:h0 + sh * (Ho - 1) + 1:sh, w0:w0 + sw * (Wo - 1) + 1:sw]
            cols[:, :, :, kh, kw, :] = sl.transpose(0, 2, 3, 1)
    A = half(w).reshape(O, -1)
    y = np.matmul(cols.reshape(N, Ho * Wo, -1), A.T).astype(F32)  # [N, P, O]
    y = y.transpose(0, 2, 1).reshape(N, O, Ho, Wo)
    if b is not None:
        y = (y + np.asarray(b, F32)[None, :, None, None]).astype(F32)
    return y


def conv1d(x, w, b, stride, pad, dil):
    """dc_conv1d (ops.c:79-111): conv2d with H = 1.  x [N,C,L], w [O,K,C]."""
    y = conv2d(x[:, :, None, :], w[:, None, :, :], b, 1, stride, 0, pad, 1, dil)
    return y[:, :, 0, :]


def conv_tr2d(x, w, b, sh, sw):
    """conv_tr_core (ops.c:143-177): cols = W[O*KH*KW][C] . x^T (fp16), then col2im with
    bias first and taps summed in (kh, kw) order (backend_cpu.c:374-411)."""
    N, C, H, W = x.shape
    O, KH, KW, _ = w.shape
    Ho, Wo = (H - 1) * sh + KH, (W - 1) * sw + KW
    A = half(w).reshape(O * KH * KW, C)
    xt = half(x).reshape(N, C, H * W)
    cols = np.matmul(A[None], xt).astype(F32).reshape(N, O, KH, KW, H, W)
    y = np.zeros((N, O, Ho, Wo), dtype=F32)
    if b is not None:
        y += np.asarray(b, F32)[None, :, None, None]
    for kh in range(KH):
        for kw in range(KW):
            y[:, :, kh:kh + sh * (H - 1) + 1:sh, kw:kw + sw * (W - 1) + 1:sw] += cols[:, :, kh, kw]
    return y


def conv_tr1d(x, w, b, stride):
    """dc_conv_tr1d (ops.c:179-206)."""
    return conv_tr2d(x[:, :, None, :], w[:, None, :, :], b, 1, stride)[:, :, 0, :]


def linear(x, w, b):
    """dc_linear (ops.c:234-257): fp16 rows . fp16 weight^T + bias."""
    shp = x.shape
    y = gemm(half(x.reshape(-1, shp[-1])), half(w))
    if b is not None:
        y = (y + np.asarray(b, F32)[None, :]).astype(F32)
    return y.reshape(shp[:-1] + (w.shape[0],))


def attention(q, k, v, heads):
    """dc_attention (ops.c:390-443): split heads to fp16, S = Q K^T (fp32),
    softmax(S / sqrt(hd)) written as fp16 (backend_cpu.c:462-480: max in float, sum of
    expf in double, inv = (float)(1/sum)), O = P V."""
    B, Tq, D = q.shape
    Tk = k.shape[1]
    hd = D // heads
    scale = F32(1.0) / F32(math.sqrt(hd))
    qh = half(q).reshape(B, Tq, heads, hd).transpose(0, 2, 1, 3)
    kh = half(k).reshape(B, Tk, heads, hd).transpose(0, 2, 1, 3)
    vh = half(v).reshape(B, Tk, heads, hd).transpose(0, 2, 1, 3)
    s = np.matmul(qh, kh.transpose(0, 1, 3, 2)).astype(F32) * scale
    mx = s.max(axis=-1, keepdims=True)
    e = np.exp((s - mx).astype(F32)).astype(F32)
    inv = (1.0 / e.astype(np.float64).sum(axis=-1, keepdims=True)).astype(F32)
    p = half(e * inv)
    o = np.matmul(p, vh).astype(F32)
    return o.transpose(0, 2, 1, 3).reshape(B, Tq, D)


# ---------------------------------------------------------------- norms


def groupnorm(x, w, b, groups, act, eps=1e-5):
    """dc_groupnorm (ops.c:306-334) + dk_groupnorm_apply (backend_cpu.c:245-282).
    act 0 none, 1 GELU, 2 GLU over channels."""
    B, C = x.shape[:2]
    xs = x.reshape(B, C, -1)
    m, v = row_stats(xs.reshape(B * groups, -1))
    m = m.reshape(B, groups)
    rs = (F32(1.0) / np.sqrt(v + F32(eps))).astype(F32).reshape(B, groups)
    g = np.arange(C) // (C // groups)
    n = ((xs - m[:, g, None]) * rs[:, g, None] * np.asarray(w, F32)[None, :, None]
         + np.asarray(b, F32)[None, :, None]).astype(F32)
    if act == 1:
        n = gelu(n)
    elif act == 2:
        n = glu(n, axis=1)
    return n.reshape((B, n.shape[1]) + x.shape[2:])


def layernorm(x, w, b, eps=1e-5):
    """dk_layernorm (backend_cpu.c:316-323): row stats then (x-m)*rs*w + b."""
    shp = x.shape
    x2 = x.reshape(-1, shp[-1])
    m, v = row_stats(x2)
    rs = (F32(1.0) / np.sqrt(v + F32(eps))).astype(F32)
    y = ((x2 - m[:, None]) * rs[:, None] * np.asarray(w, F32) + np.asarray(b, F32)).astype(F32)
    return y.reshape(shp)


def groupnorm_last(x, w, b, eps=1e-5):
    """dc_groupnorm_last (ops.c:336-350): one group over all non-batch dims, affine on the
    last dim (transformer norm_out)."""
    B = x.shape[0]
    m, v = row_stats(x.reshape(B, -1))
    rs = (F32(1.0) / np.sqrt(v + F32(eps))).astype(F32)
    sh = (B,) + (1,) * (x.ndim - 1)
    return ((x - m.reshape(sh)) * rs.reshape(sh) * np.asarray(w, F32)
            + np.asarray(b, F32)).astype(F32)


def batch_stats(x):
    """dc_batch_stats (ops.c:369-375)."""
    return row_stats(x.reshape(x.shape[0], -1))


def batch_normalize(x, m, v, eps, denorm):
    """dk_affine_rows (backend_cpu.c:304-314): sd = sqrtf(var) + eps."""
    sd = (np.sqrt(v) + F32(eps)).astype(F32)
    sh = (x.shape[0],) + (1,) * (x.ndim - 1)
    if denorm:
        return (x * sd.reshape(sh) + m.reshape(sh)).astype(F32)
    return ((x - m.reshape(sh)) / sd.reshape(sh)).astype(F32)


# ---------------------------------------------------------------- spectral


def reflect_pad1d(x, left, right):
    """dc_pad1d(reflect) (tensor.c:442-474), including its zero pre-pad when the signal is
    not longer than the pad."""
    L = x.shape[-1]
    mx = max(left, right)
    if L <= mx:
        extra = mx - L + 1
        er = min(right, extra)
        el = extra - er
        left -= el
        right -= er
        x = np.pad(x, [(0, 0)] * (x.ndim - 1) + [(el, er)])
    if left == 0 and right == 0:
        return x
    return np.pad(x, [(0, 0)] * (x.ndim - 1) + [(left, right)], mode="reflect")


def hann(n):
    """Periodic Hann window in double, stored as float (stft.c:5-20)."""
    i = np.arange(n, dtype=np.float64)
    return (0.5 - 0.5 * np.cos(2.0 * math.pi * i / n)).astype(F32)


def spec(mix, nfft):
    """dc_htdemucs_spec_cac (stft.c:29-47) + dk_stft (backend_cpu.c:569-594):
    [B,C,T] -> [B, 2C, nfft/2, le] with (re, im) planes per channel."""
    B, C, T = mix.shape
    hl = nfft // 4
    le = -(-T // hl)
    pad = (hl // 2) * 3
    xp = reflect_pad1d(mix, pad, pad + le * hl - T)
    xc = reflect_pad1d(xp, nfft // 2, nfft // 2)
    L = xc.shape[-1]
    win = hann(nfft).astype(np.float64)
    starts = (2 + np.arange(le)) * hl
    idx = starts[:, None] + np.arange(nfft)[None, :]
    sig = np.zeros((B * C, L + nfft), dtype=np.float64)
    sig[:, :L] = xc.reshape(B * C, L)
    fr = sig[:, idx] * win  # [R, le, nfft]
    X = np.fft.fft(fr, axis=-1)[:, :, : nfft // 2]  # [R, le, nbins]
    out = np.stack([X.real, X.imag], axis=1).transpose(0, 1, 3, 2)  # [R, 2, nbins, le]
    return out.reshape(B, 2 * C, nfft // 2, le).astype(F32)


def ispec(z, nfft, length):
    """dc_htdemucs_ispec_cac (stft.c:49-69) + dk_istft_frames / dk_ola
    (backend_cpu.c:596-662): irfft of the Nyquist-less spectrum, windowed, 2 zero pad
    frames each side, overlap-add divided by the summed squared window."""
    B, S, C2, F, N = z.shape
    C = C2 // 2
    hop = nfft // 4
    R = B * S * C
    zz = z.reshape(R, 2, F, N).astype(np.float64)
    spec_full = np.zeros((R, N, nfft // 2 + 1), dtype=np.complex128)
    spec_full[:, :, :F] = (zz[:, 0] + 1j * zz[:, 1]).transpose(0, 2, 1)
    win = hann(nfft).astype(np.float64)
    frames = np.fft.irfft(spec_full, n=nfft, axis=-1) * win  # [R, N, nfft]
    NF = N + 4
    out_len = hop * (NF - 1) + nfft
    num = np.zeros((R, out_len))
    den = np.zeros(out_len)
    for f in range(NF):
        den[f * hop:f * hop + nfft] += win ** 2
        if 2 <= f < N + 2:
            num[:, f * hop:f * hop + nfft] += frames[:, f - 2]
    start = nfft // 2 + (hop // 2) * 3
    seg = slice(start, start + length)
    n_ = num[:, seg]
    d_ = den[seg]
    y = np.where(d_ > 0, n_ / np.where(d_ > 0, d_, 1.0), 0.0)
    return y.reshape(B, S, C, length).astype(F32)


# ---------------------------------------------------------------- model


class Config:
    """Values the forward needs from the model JSON (config.c:106-264 defaults)."""

    def __init__(self, d: dict):
        g = d.get
        self.n_sources = len(g("sources", [0] * 6))
        self.samplerate = g("samplerate", 44100)
        self.segment = g("segment", 7.8)
        self.nfft = g("nfft", 4096)
        self.audio_channels = g("audio_channels", 2)
        self.channels = g("channels", 48)
        self.depth = g("depth", 4)
        self.kernel_size = g("kernel_size", 8)
        self.stride = g("stride", 4)
        self.context = g("context", 1)
        self.context_enc = g("context_enc", 0)
        self.dconv_depth = g("dconv_depth", 2)
        self.t_layers = g("t_layers", 5)
        self.t_heads = g("t_heads", 8)
        self.freq_emb = g("freq_emb", 0.2)
        self.emb_scale = g("emb_scale", 10.0)
        self.t_max_period = g("t_max_period", 10000.0)
        self.t_weight_pos_embed = g("t_weight_pos_embed", 1.0)
        self.valid_length = g("valid_length", 0) or int(F32(self.segment) * F32(self.samplerate))


def dconv(x, W, prefix, depth):
    """dc_dconv (layers.c:24-53) on [N, C, T]."""
    y = x.copy()
    for d in range(depth):
        dil = 1 << d
        p = f"{prefix}.layers.{d}.layers"
        h = conv1d(y, W[f"{p}.0.conv.weight"], W[f"{p}.0.conv.bias"], 1, dil, dil)
        h = groupnorm(h, W[f"{p}.1.weight"], W[f"{p}.1.bias"], 1, 1)
        h = conv1d(h, W[f"{p}.3.conv.weight"], W[f"{p}.3.conv.bias"], 1, 0, 1)
        h = groupnorm(h, W[f"{p}.4.weight"], W[f"{p}.4.bias"], 1, 2)
        y = (y + h * W[f"{p}.6.scale"][None, :, None]).astype(F32)
    return y


def henc(x, W, prefix, freq, cfg: Config):
    """dc_henc (layers.c:80-141) for htdemucs_6s layers (no outer norm, rewrite + DConv)."""
    K, S = cfg.kernel_size, cfg.stride
    if not freq:
        le = x.shape[-1]
        if le % S:
            x = np.pad(x, ((0, 0), (0, 0), (0, S - le % S)))
        y = conv1d(x, W[f"{prefix}.conv.conv.weight"], W[f"{prefix}.conv.conv.bias"], S,
                   K // 4, 1)
    else:
        y = conv2d(x, W[f"{prefix}.conv.conv.weight"], W[f"{prefix}.conv.conv.bias"], S, 1,
                   K // 4, 0)
    y = gelu(y)
    if freq:
        B, C, Fr, T = y.shape
        yr = y.transpose(0, 2, 1, 3).reshape(B * Fr, C, T)
        yd = dconv(yr, W, f"{prefix}.dconv", cfg.dconv_depth)
        y = yd.reshape(B, Fr, C, T).transpose(0, 2, 1, 3)
    else:
        y = dconv(y, W, f"{prefix}.dconv", cfg.dconv_depth)
    ce = cfg.context_enc
    if freq:
        z = conv2d(y, W[f"{prefix}.rewrite.conv.weight"], W[f"{prefix}.rewrite.conv.bias"], 1,
                   1, ce, ce)
    else:
        z = conv1d(y, W[f"{prefix}.rewrite.conv.weight"], W[f"{prefix}.rewrite.conv.bias"], 1,
                   ce, 1)
    return glu(z, axis=1)


def hdec(x, skip, length, W, prefix, freq, last, cfg: Config):
    """dc_hdec (layers.c:143-220): + skip, rewrite (3x3 / k3) + GLU, conv_tr, crop, GELU."""
    x = (x + skip).astype(F32)
    c = cfg.context
    if freq:
        z = conv2d(x, W[f"{prefix}.rewrite.conv.weight"], W[f"{prefix}.rewrite.conv.bias"], 1,
                   1, c, c)
    else:
        z = conv1d(x, W[f"{prefix}.rewrite.conv.weight"], W[f"{prefix}.rewrite.conv.bias"], 1,
                   c, 1)
    y = glu(z, axis=1)
    pad = cfg.kernel_size // 4
    if freq:
        z = conv_tr2d(y, W[f"{prefix}.conv_tr.conv.weight"], W[f"{prefix}.conv_tr.conv.bias"],
                      cfg.stride, 1)
        z = z[:, :, pad:z.shape[2] - pad]
    else:
        z = conv_tr1d(y, W[f"{prefix}.conv_tr.conv.weight"], W[f"{prefix}.conv_tr.conv.bias"],
                      cfg.stride)
        z = z[:, :, pad:pad + length]
    if not last:
        z = gelu(z)
    return np.ascontiguousarray(z)


def sin_embedding(length, dim, max_period, weight):
    """transformer.c:108-126, float32 arithmetic."""
    half_ = dim // 2
    t = np.arange(length, dtype=F32)[:, None]
    j = np.arange(half_, dtype=F32)[None, :]
    den = np.power(F32(max_period), j / F32(half_ - 1)).astype(F32)
    ph = (t / den).astype(F32)
    return np.concatenate([np.cos(ph) * F32(weight), np.sin(ph) * F32(weight)], axis=1)[None]


def sin_embedding_2d(d_model, height, width, max_period, weight):
    """transformer.c:128-158: tokens ordered t * height + f."""
    half_ = d_model // 2
    nterm = half_ // 2
    sc = F32(-np.log(F32(max_period)) / F32(half_))
    div = np.exp(F32(2) * np.arange(nterm, dtype=F32) * sc).astype(F32)
    c = np.arange(d_model)
    cc = np.where(c < half_, c, c - half_)
    t = np.arange(width, dtype=F32)[:, None, None]
    f = np.arange(height, dtype=F32)[None, :, None]
    pos = np.where((c < half_)[None, None, :], t, f)
    ang = (pos * div[cc // 2][None, None, :]).astype(F32)
    val = np.where((cc % 2 == 0)[None, None, :], np.sin(ang), np.cos(ang)) * F32(weight)
    return val.reshape(1, width * height, d_model).astype(F32)


def _mha(q, kv, W, p, heads):
    """mha_pref (transformer.c:18-35)."""
    qq = linear(q, W[f"{p}.query_proj.weight"], W[f"{p}.query_proj.bias"])
    kk = linear(kv, W[f"{p}.key_proj.weight"], W[f"{p}.key_proj.bias"])
    vv = linear(kv, W[f"{p}.value_proj.weight"], W[f"{p}.value_proj.bias"])
    a = attention(qq, kk, vv, heads)
    return linear(a, W[f"{p}.out_proj.weight"], W[f"{p}.out_proj.bias"])


def _residual(x, a, W, gamma):
    return (x + a * W[f"{gamma}.scale"]).astype(F32)


def _ffn(x, W, p, norm):
    """feed_forward (transformer.c:37-54)."""
    xn = layernorm(x, W[f"{p}.{norm}.weight"], W[f"{p}.{norm}.bias"])
    h = gelu(linear(xn, W[f"{p}.linear1.weight"], W[f"{p}.linear1.bias"]))
    h2 = linear(h, W[f"{p}.linear2.weight"], W[f"{p}.linear2.bias"])
    return _residual(x, h2, W, f"{p}.gamma_2")


def _norm_out(x, W, p):
    return groupnorm_last(x, W[f"{p}.norm_out.gn.weight"], W[f"{p}.norm_out.gn.bias"])


def crosstransformer(x, xt, W, cfg: Config):
    """dc_crosstransformer (transformer.c:160-216): 5 layers, even self / odd cross."""
    B, C, Fr, T1 = x.shape
    xf = x.transpose(0, 3, 2, 1).reshape(B, T1 * Fr, C)
    cur = layernorm(xf, W["crosstransformer.norm_in.weight"], W["crosstransformer.norm_in.bias"])
    cur = (cur + sin_embedding_2d(C, Fr, T1, cfg.t_max_period, cfg.t_weight_pos_embed)).astype(F32)
    Ct, T2 = xt.shape[1], xt.shape[2]
    xtt = xt.transpose(0, 2, 1)
    curt = layernorm(xtt, W["crosstransformer.norm_in_t.weight"],
                     W["crosstransformer.norm_in_t.bias"])
    curt = (curt + sin_embedding(T2, Ct, cfg.t_max_period, cfg.t_weight_pos_embed)).astype(F32)
    H = cfg.t_heads
    for idx in range(cfg.t_layers):
        lp, lpt = f"crosstransformer.layers.{idx}", f"crosstransformer.layers_t.{idx}"
        if idx % 2 == 0:
            outs = []
            for p, v in ((lp, cur), (lpt, curt)):
                xn = layernorm(v, W[f"{p}.norm1.weight"], W[f"{p}.norm1.bias"])
                a = _mha(xn, xn, W, f"{p}.attn", H)
                x1 = _residual(v, a, W, f"{p}.gamma_1")
                outs.append(_norm_out(_ffn(x1, W, p, "norm2"), W, p))
        else:
            outs = []
            for p, q, k in ((lp, cur, curt), (lpt, curt, cur)):
                qn = layernorm(q, W[f"{p}.norm1.weight"], W[f"{p}.norm1.bias"])
                kn = layernorm(k, W[f"{p}.norm2.weight"], W[f"{p}.norm2.bias"])
                a = _mha(qn, kn, W, f"{p}.cross_attn", H)
                x1 = _residual(q, a, W, f"{p}.gamma_1")
                outs.append(_norm_out(_ffn(x1, W, p, "norm3"), W, p))
        cur, curt = outs
    xo = cur.reshape(B, T1, Fr, C).transpose(0, 3, 2, 1)
    return np.ascontiguousarray(xo), np.ascontiguousarray(curt.transpose(0, 2, 1))


def forward(mix, W, cfg: Config, stages=None):
    """dc_htdemucs_forward (htdemucs.c:136-280); `stages` (dict) receives the intermediate
    tensors under test_compare.c's keys."""
    st = stages if stages is not None else {}
    mix = np.asarray(mix, F32)
    B, _, length = mix.shape
    L = cfg.valid_length
    pre = 0
    if length < L:
        pre = length
        mix = np.pad(mix, ((0, 0), (0, 0), (0, L - length)))
    mag = spec(mix, cfg.nfft)
    st["mag"] = mag
    Fq, Tf = mag.shape[2], mag.shape[3]
    mean, var = batch_stats(mag)
    x = batch_normalize(mag, mean, var, 1e-5, 0)
    st["x_norm"] = x
    meant, vart = batch_stats(mix)
    xt = batch_normalize(mix, meant, vart, 1e-5, 0)
    st["xt_norm"] = xt
    saved, saved_t, lens, lens_t = [], [], [], []
    for idx in range(cfg.depth):
        lens.append(x.shape[-1])
        lens_t.append(xt.shape[-1])
        xt = henc(xt, W, f"tencoder.{idx}", False, cfg)
        saved_t.append(xt)
        st[f"tenc_{idx}"] = xt
        x = henc(x, W, f"encoder.{idx}", True, cfg)
        if idx == 0:
            emb = W["freq_emb.embedding.weight"][: x.shape[2]].T
            scaled = (emb * F32(cfg.freq_emb * cfg.emb_scale)).astype(F32)
            x = (x + scaled[None, :, :, None]).astype(F32)
        saved.append(x)
        st[f"enc_{idx}"] = x
    if cfg.t_layers > 0:
        x, xt = crosstransformer(x, xt, W, cfg)
        st["transformer_x"] = x
        st["transformer_xt"] = xt
    for idx in range(cfg.depth):
        last = idx == cfg.depth - 1
        x = hdec(x, saved.pop(), lens.pop(), W, f"decoder.{idx}", True, last, cfg)
        st[f"dec_{idx}"] = x
        xt = hdec(xt, saved_t.pop(), lens_t.pop(), W, f"tdecoder.{idx}", False, last, cfg)
        st[f"tdec_{idx}"] = xt
    S = cfg.n_sources
    xr = x.reshape(B, S, -1, Fq, Tf)
    xden = batch_normalize(xr, mean, var, 1e-5, 1)
    xi = ispec(xden, cfg.nfft, L)
    st["ispec"] = xi
    xtr = xt.reshape(B, S, -1, xt.shape[-1])
    xtd = batch_normalize(xtr, meant, vart, 1e-5, 1)
    d = xi.shape[-1] - xtd.shape[-1]
    xtrim = xi[..., d // 2: xi.shape[-1] - (d - d // 2)]
    y = (xtd + xtrim).astype(F32)
    keep = pre if pre else L
    y = np.ascontiguousarray(y[..., :keep])
    st["stems"] = y
    return y


# ---------------------------------------------------------------- apply


class PyRandom:
    """CPython's random.Random(seed).randint (apply.c:5-107 restates MT19937 for it)."""

    def __init__(self, seed):
        import random
        self.r = random.Random(seed)

    def randint(self, lo, hi):
        return self.r.randint(lo, hi)


def ola_weight(n, power):
    """Triangular transition weights (apply.c:116-133), float32 math."""
    half_ = n // 2
    w = np.concatenate([np.arange(1, half_ + 1), n - np.arange(half_, n)]).astype(F32)
    return np.power(w / w.max(), F32(power)).astype(F32)


def padded_chunk(mix, offset, chunk_len, target_len):
    """apply.c:135-154."""
    total = mix.shape[-1]
    delta = target_len - chunk_len
    start = offset - delta // 2
    end = start + target_len
    cs, ce = max(start, 0), min(end, total)
    sl = mix[..., cs:ce]
    pl, pr = cs - start, end - ce
    if pl or pr:
        sl = np.pad(sl, [(0, 0)] * (sl.ndim - 1) + [(pl, pr)])
    return sl


def center_trim(y, n):
    d = y.shape[-1] - n
    return y[..., d // 2: y.shape[-1] - (d - d // 2)]


def segment_plan(length, cfg: Config, overlap=0.25, batch_size=8):
    """Offsets and forward batches of dc_apply_model's split loop (apply.c:223-296):
    full segments batched up to batch_size, each tail segment alone."""
    seg = int(F32(cfg.samplerate) * F32(cfg.segment))
    stride = int((F32(1.0) - F32(overlap)) * F32(seg))
    offsets = list(range(0, length, stride))
    batches, cur = [], []
    for i in range(len(offsets) + 1):
        full = i < len(offsets) and length - offsets[i] >= seg
        flush = not full
        if full:
            cur.append(i)
            flush = len(cur) >= batch_size
        if flush and cur:
            batches.append(("full", cur))
            cur = []
        if i < len(offsets) and not full:
            batches.append(("tail", [i]))
    return seg, stride, offsets, batches


def apply_model(mix, W, cfg: Config, shifts=1, overlap=0.25, transition_power=1.0,
                batch_size=8, seed=1, forward_fn=None, shard=(0, 1)):
    """dc_apply_model (apply.c:179-306) with split=True.  shard = (index, count) keeps only
    the segments of one contiguous block of the offsets, [n index / count, n (index + 1) /
    count) (the weight sum stays global), so the shards' outputs add up to the unsharded
    result; with shifts = 0 this is the engine's data-parallel split."""
    fwd = forward_fn or (lambda x: forward(x, W, cfg))
    B, C, length = mix.shape
    if shifts > 0:
        max_shift = int(F32(0.5) * F32(cfg.samplerate))
        padded = padded_chunk(mix, 0, length, length + 2 * max_shift)
        rng = PyRandom(seed)
        acc = None
        for _ in range(shifts):
            off = rng.randint(0, max_shift)
            shifted = padded_chunk(padded, off, length + max_shift - off,
                                   length + max_shift - off)
            out = apply_model(shifted, W, cfg, 0, overlap, transition_power, batch_size,
                              seed, forward_fn, shard)
            tr = out[..., max_shift - off:]
            acc = tr if acc is None else (acc + tr).astype(F32)
        return (acc * F32(1.0 / shifts)).astype(F32)
    seg, stride, offsets, batches = segment_plan(length, cfg, overlap, batch_size)
    weight = ola_weight(seg, transition_power)
    sumw = np.zeros(length, dtype=np.float64)
    for off in offsets:  # every segment's weight, whichever shard runs it
        n = min(seg, length - off)
        sumw[off:off + n] += weight[:n]
    out = np.zeros((B, cfg.n_sources, C, length), dtype=F32)
    si, sc = shard
    b0, b1 = len(offsets) * si // sc, len(offsets) * (si + 1) // sc
    for kind, idxs in batches:
        idxs = [i for i in idxs if b0 <= i < b1]
        if not idxs:
            continue
        if kind == "full":
            flat = np.concatenate([padded_chunk(mix, offsets[i], seg, cfg.valid_length)
                                   for i in idxs], axis=0)
            y = fwd(flat)
            for k, i in enumerate(idxs):
                off = offsets[i]
                yk = center_trim(y[k * B:(k + 1) * B], seg)
                out[..., off:off + seg] += (yk * weight).astype(F32)
        else:
            i = idxs[0]
            this = length - offsets[i]
            valid = max(cfg.valid_length, this)
            y = fwd(padded_chunk(mix, offsets[i], this, valid))
            yk = center_trim(y, this)
            out[..., offsets[i]:] += (yk * weight[:this]).astype(F32)
    inv = np.where(sumw > 0, 1.0 / np.where(sumw > 0, sumw, 1), 0).astype(F32)
    return (out * inv).astype(F32)
