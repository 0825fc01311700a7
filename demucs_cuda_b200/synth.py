"""Seeded synthetic inputs and random-init htdemucs_6s weights.

No checkpoint or dataset is reachable here, so every run uses generated data with the
reference's shapes:

* weights: the htdemucs_6s tensor set the reference loader expects (names and MLX layouts
  as read by weights.c:258-372 and looked up by layers.c / transformer.c / htdemucs.c),
  Kaiming-uniform (bound 1/sqrt(fan_in), PyTorch's conv/linear default) from a numpy
  PCG64 stream, written as an fp32 safetensors file plus the model JSON
  (config.c:106-155 keys);
* inputs: the benchmark configurations -- a U[-0.5, 0.5] stereo segment (one forward) and a
  240 s sum of sinusoids plus noise (config 4).

Both the reference oracle and this package load the same files, so both see identical
bytes.
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass, field, asdict

import numpy as np


@dataclass
class ModelConfig:
    """Subset of the reference DcConfig (config.h:6-51) that shapes the weights."""

    n_sources: int = 6
    samplerate: int = 44100
    segment: float = 7.8
    nfft: int = 4096
    audio_channels: int = 2
    channels: int = 48
    growth: int = 2
    depth: int = 4
    kernel_size: int = 8
    stride: int = 4
    context: int = 1
    context_enc: int = 0
    dconv_depth: int = 2
    dconv_comp: int = 8
    dconv_init: float = 1e-3
    t_layers: int = 5
    t_heads: int = 8
    t_hidden_scale: float = 4.0
    freq_emb: float = 0.2
    emb_scale: float = 10.0
    valid_length: int = 0
    sources: list = field(default_factory=lambda: ["drums", "bass", "other", "vocals",
                                                   "guitar", "piano"])

    def __post_init__(self):
        if self.valid_length <= 0:
            # float32 arithmetic as config.c:154 does it
            self.valid_length = int(np.float32(self.segment) * np.float32(self.samplerate))

    def to_json(self) -> str:
        d = asdict(self)
        d["model"] = "htdemucs_6s"
        d["sources"] = self.sources[: self.n_sources]
        d["hop_length"] = self.nfft // 4
        d["cac"] = 1
        d["rewrite"] = 1
        d["dconv_mode"] = 1
        d["norm_starts"] = 4
        d["norm_groups"] = 4
        d["t_cross_first"] = 0
        d["t_gelu"] = 1
        d["use_train_segment"] = 1
        d["wiener_iters"] = 0
        return json.dumps(d, indent=1)


FULL = ModelConfig()
# Same architecture and widths, 1 s segments: every layer shape of the real model with a
# shorter time axis (used for fast parity of the full-width kernels).
SHORT = ModelConfig(segment=1.0)
# Narrow (channels 8, transformer dim 64, head dim 8) and 0.5 s: a full forward the CPU
# reference finishes in well under a second.
TINY = ModelConfig(channels=8, segment=0.5)


def weight_specs(cfg: ModelConfig):
    """(name, shape, kind) for every tensor, following the htdemucs construction that
    htdemucs.c:29-106 mirrors (channel counts come from the original HTDemucs: decoder 0's
    output is audio_channels*n_sources*2 under cac).  kind: 'conv'/'linear' (Kaiming
    weight), 'bias', 'gn_w', 'gn_b', 'scale_dconv', 'scale_t', 'emb'."""
    specs = []
    ach = cfg.audio_channels
    chin, chin_z = ach, ach * 2
    chout = chout_z = cfg.channels
    freqs = cfg.nfft // 2
    K, S = cfg.kernel_size, cfg.stride
    for index in range(cfg.depth):
        freq = freqs > 1
        ker = K
        if freq and freqs <= K:
            ker = freqs
        # encoder (freq), conv weight [O, KH, KW, I]
        specs.append((f"encoder.{index}.conv.conv.weight", (chout_z, ker, 1, chin_z), "conv"))
        specs.append((f"encoder.{index}.conv.conv.bias", (chout_z,), "bias"))
        ce = 1 + 2 * cfg.context_enc
        specs.append((f"encoder.{index}.rewrite.conv.weight", (2 * chout_z, ce, ce, chout_z),
                      "conv"))
        specs.append((f"encoder.{index}.rewrite.conv.bias", (2 * chout_z,), "bias"))
        specs += _dconv_specs(f"encoder.{index}.dconv", chout_z, cfg)
        if freq:
            specs.append((f"tencoder.{index}.conv.conv.weight", (chout, K, chin), "conv"))
            specs.append((f"tencoder.{index}.conv.conv.bias", (chout,), "bias"))
            specs.append((f"tencoder.{index}.rewrite.conv.weight", (2 * chout, ce, chout),
                          "conv"))
            specs.append((f"tencoder.{index}.rewrite.conv.bias", (2 * chout,), "bias"))
            specs += _dconv_specs(f"tencoder.{index}.dconv", chout, cfg)
        if index == 0:
            chin = ach * cfg.n_sources
            chin_z = chin * 2
        dec = cfg.depth - 1 - index  # decoder.insert(0, ...)
        cc = 1 + 2 * cfg.context
        specs.append((f"decoder.{dec}.rewrite.conv.weight", (2 * chout_z, cc, cc, chout_z),
                      "conv"))
        specs.append((f"decoder.{dec}.rewrite.conv.bias", (2 * chout_z,), "bias"))
        specs.append((f"decoder.{dec}.conv_tr.conv.weight", (chin_z, ker, 1, chout_z), "conv"))
        specs.append((f"decoder.{dec}.conv_tr.conv.bias", (chin_z,), "bias"))
        if freq:
            specs.append((f"tdecoder.{dec}.rewrite.conv.weight", (2 * chout, cc, chout),
                          "conv"))
            specs.append((f"tdecoder.{dec}.rewrite.conv.bias", (2 * chout,), "bias"))
            specs.append((f"tdecoder.{dec}.conv_tr.conv.weight", (chin, K, chout), "conv"))
            specs.append((f"tdecoder.{dec}.conv_tr.conv.bias", (chin,), "bias"))
        chin, chin_z = chout, chout_z
        chout *= cfg.growth
        chout_z *= cfg.growth
        if freq:
            freqs = 1 if freqs <= K else freqs // S
    # frequency embedding after encoder 0: [n_freq_after_enc0, channels]
    specs.append(("freq_emb.embedding.weight", (cfg.nfft // 2 // S, cfg.channels), "emb"))
    D = cfg.channels * cfg.growth ** (cfg.depth - 1)
    H = int(D * cfg.t_hidden_scale)
    for br in ("", "_t"):
        specs.append((f"crosstransformer.norm_in{br}.weight", (D,), "gn_w"))
        specs.append((f"crosstransformer.norm_in{br}.bias", (D,), "gn_b"))
    for br in ("layers", "layers_t"):
        for l in range(cfg.t_layers):
            p = f"crosstransformer.{br}.{l}"
            attn = "attn" if l % 2 == 0 else "cross_attn"
            for proj in ("query_proj", "key_proj", "value_proj", "out_proj"):
                specs.append((f"{p}.{attn}.{proj}.weight", (D, D), "linear"))
                specs.append((f"{p}.{attn}.{proj}.bias", (D,), "bias"))
            norms = ["norm1", "norm2"] + ([] if l % 2 == 0 else ["norm3"])
            for n in norms:
                specs.append((f"{p}.{n}.weight", (D,), "gn_w"))
                specs.append((f"{p}.{n}.bias", (D,), "gn_b"))
            specs.append((f"{p}.linear1.weight", (H, D), "linear"))
            specs.append((f"{p}.linear1.bias", (H,), "bias"))
            specs.append((f"{p}.linear2.weight", (D, H), "linear"))
            specs.append((f"{p}.linear2.bias", (D,), "bias"))
            specs.append((f"{p}.gamma_1.scale", (D,), "scale_t"))
            specs.append((f"{p}.gamma_2.scale", (D,), "scale_t"))
            specs.append((f"{p}.norm_out.gn.weight", (D,), "gn_w"))
            specs.append((f"{p}.norm_out.gn.bias", (D,), "gn_b"))
    return specs


def _dconv_specs(prefix, C, cfg):
    hid = C // cfg.dconv_comp
    out = []
    for d in range(cfg.dconv_depth):
        p = f"{prefix}.layers.{d}.layers"
        out.append((f"{p}.0.conv.weight", (hid, 3, C), "conv"))
        out.append((f"{p}.0.conv.bias", (hid,), "bias"))
        out.append((f"{p}.1.weight", (hid,), "gn_w"))
        out.append((f"{p}.1.bias", (hid,), "gn_b"))
        out.append((f"{p}.3.conv.weight", (2 * C, 1, hid), "conv"))
        out.append((f"{p}.3.conv.bias", (2 * C,), "bias"))
        out.append((f"{p}.4.weight", (2 * C,), "gn_w"))
        out.append((f"{p}.4.bias", (2 * C,), "gn_b"))
        out.append((f"{p}.6.scale", (C,), "scale_dconv"))
    return out


def make_weights(cfg: ModelConfig, seed: int = 1, layer_scale: float | None = None,
                 affine_jitter: float = 0.1):
    """Random-init weights.  layer_scale=None keeps the HTDemucs inits (DConv LayerScale
    dconv_init, transformer LayerScale 1e-4); a larger value makes every residual branch
    visible in the output, which parity tests use so a branch error cannot hide."""
    rng = np.random.default_rng(seed)
    specs = weight_specs(cfg)
    fan = {}
    for name, shape, kind in specs:
        if kind in ("conv", "linear"):
            fan[name.rsplit(".", 1)[0]] = int(np.prod(shape[1:]))
    out = {}
    for name, shape, kind in specs:
        if kind in ("conv", "linear"):
            b = 1.0 / np.sqrt(np.prod(shape[1:]))
            v = rng.uniform(-b, b, shape)
        elif kind == "bias":
            b = 1.0 / np.sqrt(fan[name.rsplit(".", 1)[0]])
            v = rng.uniform(-b, b, shape)
        elif kind == "gn_w":
            v = 1.0 + rng.uniform(-affine_jitter, affine_jitter, shape)
        elif kind == "gn_b":
            v = rng.uniform(-affine_jitter, affine_jitter, shape)
        elif kind == "scale_dconv":
            s = cfg.dconv_init if layer_scale is None else layer_scale
            v = np.full(shape, s) * (1.0 + rng.uniform(-0.5, 0.5, shape))
        elif kind == "scale_t":
            s = 1e-4 if layer_scale is None else layer_scale
            v = np.full(shape, s) * (1.0 + rng.uniform(-0.5, 0.5, shape))
        elif kind == "emb":
            # ScaledEmbedding(smooth=True): cumulative sum / sqrt(index), divided by scale
            e = rng.standard_normal(shape)
            e = np.cumsum(e, axis=0) / np.sqrt(np.arange(1, shape[0] + 1))[:, None]
            v = e / cfg.emb_scale
        else:
            raise ValueError(kind)
        out[name] = np.asarray(v, dtype=np.float32)
    return out


def save_safetensors(path: str, tensors: dict):
    """Minimal safetensors writer (F32 only): 8-byte LE header length, JSON header,
    concatenated little-endian data."""
    header = {}
    off = 0
    blobs = []
    for name, arr in tensors.items():
        a = np.ascontiguousarray(arr, dtype="<f4")
        n = a.nbytes
        header[name] = {"dtype": "F32", "shape": list(a.shape), "data_offsets": [off, off + n]}
        blobs.append(a.tobytes())
        off += n
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def load_safetensors(path: str) -> dict:
    with open(path, "rb") as f:
        raw = f.read()
    hl = struct.unpack("<Q", raw[:8])[0]
    header = json.loads(raw[8:8 + hl])
    data = raw[8 + hl:]
    out = {}
    for name, e in header.items():
        if name == "__metadata__":
            continue
        b, en = e["data_offsets"]
        dt = {"F32": "<f4", "F16": "<f2"}[e["dtype"]]
        out[name] = np.frombuffer(data[b:en], dtype=dt).reshape(e["shape"]).astype(np.float32)
    return out


def write_model(dirpath: str, cfg: ModelConfig, seed: int = 1, layer_scale=None):
    """Write <dir>/model.safetensors and <dir>/model.json; returns the two paths.
    Skips the work when both files already exist with the same generation key."""
    os.makedirs(dirpath, exist_ok=True)
    wpath = os.path.join(dirpath, "model.safetensors")
    cpath = os.path.join(dirpath, "model.json")
    key = json.dumps([asdict(cfg), seed, layer_scale], sort_keys=True)
    kpath = os.path.join(dirpath, "gen.key")
    if os.path.exists(wpath) and os.path.exists(cpath) and os.path.exists(kpath):
        with open(kpath) as f:
            if f.read() == key:
                return wpath, cpath
    save_safetensors(wpath, make_weights(cfg, seed, layer_scale))
    with open(cpath, "w") as f:
        f.write(cfg.to_json())
    with open(kpath, "w") as f:
        f.write(key)
    return wpath, cpath


def segment_input(cfg: ModelConfig = FULL, batch: int = 1, seed: int = 0) -> np.ndarray:
    """Config 0: i.i.d. U[-0.5, 0.5] stereo segment(s) of valid_length samples."""
    rng = np.random.default_rng(seed)
    return rng.uniform(-0.5, 0.5, (batch, cfg.audio_channels, cfg.valid_length)).astype(
        np.float32)


def track_input(seconds: float = 240.0, samplerate: int = 44100, seed: int = 0,
                n_sines: int = 40) -> np.ndarray:
    """Config 4: a seeded sum of n_sines sinusoids in 40-8000 Hz plus uniform noise,
    stereo, |x| <= 0.9.  Returns [1, 2, T] float32."""
    T = int(round(seconds * samplerate))
    rng = np.random.default_rng(seed)
    t = np.arange(T, dtype=np.float64) / samplerate
    out = np.zeros((2, T), dtype=np.float64)
    for ch in range(2):
        f = rng.uniform(40.0, 8000.0, n_sines)
        ph = rng.uniform(0, 2 * np.pi, n_sines)
        a = rng.uniform(0.2, 1.0, n_sines)
        acc = np.zeros(T)
        for i in range(n_sines):
            acc += a[i] * np.sin(2 * np.pi * f[i] * t + ph[i])
        acc += rng.uniform(-1.0, 1.0, T) * 2.0
        out[ch] = acc
    out *= 0.9 / np.max(np.abs(out))
    return out[None].astype(np.float32)
