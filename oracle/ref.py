"""ctypes access to the reference's own CPU implementation (oracle/_ref/libdcref.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's CPU
baseline leg, as the checker / timed CPU baseline.  The product never imports this.

The library is the reference's unchanged C sources (backend_cpu.c + model/ops/tensor
files) compiled by oracle/Makefile, plus oracle/refdrv.c.  All pointers are host memory.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_ref", "libdcref.so")
BIN_PATH = os.path.join(HERE, "_ref", "dcref")

_F = C.POINTER(C.c_float)
STAGE_FN = C.CFUNCTYPE(None, C.c_char_p, _F, C.c_int, C.POINTER(C.c_int), C.c_void_p)
_lib = None


def available() -> bool:
    return os.path.exists(LIB_PATH)


def lib():
    global _lib
    if _lib is None:
        if not available():
            raise FileNotFoundError(
                f"{LIB_PATH} missing: build it with `make -C oracle` where the reference "
                "sources are present")
        _lib = C.CDLL(LIB_PATH)
        _lib.dcref_forward.restype = C.c_int
        _lib.dcref_forward.argtypes = [_F, C.c_int, C.c_int, C.c_int, _F, STAGE_FN, C.c_void_p]
        _lib.dcref_forward_plain.argtypes = [_F, C.c_int, C.c_int, C.c_int, _F]
        _lib.dcref_apply.argtypes = [_F, C.c_int, C.c_int, C.c_int, _F, C.c_int, C.c_int,
                                     C.c_float, C.c_float, C.c_int, C.c_uint, C.c_int]
        _lib.dcref_weight_block_bytes.restype = C.c_size_t
        _lib.dk_gemm_half.argtypes = [C.c_int64, C.c_int64, C.c_int64, C.c_float, C.c_void_p,
                                      C.c_int64, C.c_int64, C.c_void_p, C.c_int64, C.c_int64,
                                      C.c_float, C.c_void_p, C.c_int64, C.c_int64, C.c_int64]
        _lib.dcref_round_half.argtypes = [_F, _F, C.c_int64]
    return _lib


def _p(a):
    return a.ctypes.data_as(_F)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def load(weights: str, config: str):
    lib().dcref_load(weights.encode(), config.encode())


def n_sources() -> int:
    return lib().dcref_n_sources()


def valid_length() -> int:
    return lib().dcref_valid_length()


def forward(mix: np.ndarray, stages: bool = False):
    """Reference forward on mix [B, C, T]; returns stems (and a dict of stage outputs)."""
    mix = _f32(mix)
    B, Cc, T = mix.shape
    S = n_sources()
    out = np.zeros((B, S, Cc, max(T, valid_length())), dtype=np.float32)
    got = {}

    def cb(name, data, ndim, shape, user):
        shp = tuple(shape[i] for i in range(ndim))
        n = int(np.prod(shp))
        got[name.decode()] = np.ctypeslib.as_array(data, shape=(n,)).copy().reshape(shp)

    fn = STAGE_FN(cb) if stages else STAGE_FN(0)
    tout = lib().dcref_forward(_p(mix), B, Cc, T, _p(out), fn, None)
    stems = np.ascontiguousarray(out.reshape(-1)[: B * S * Cc * tout].reshape(B, S, Cc, tout))
    return (stems, got) if stages else stems


def apply_model(mix, shifts=1, split=True, overlap=0.25, transition_power=1.0, batch_size=8,
                seed=1, use_seed=False):
    mix = _f32(mix)
    B, Cc, T = mix.shape
    out = np.zeros((B, n_sources(), Cc, T), dtype=np.float32)
    lib().dcref_apply(_p(mix), B, Cc, T, _p(out), shifts, int(split), overlap,
                      transition_power, batch_size, seed, int(use_seed))
    return out


def round_half(x):
    x = _f32(x)
    y = np.empty_like(x)
    lib().dcref_round_half(_p(x), _p(y), x.size)
    return y


def conv1d(x, w, b, stride, pad, dil):
    x, w = _f32(x), _f32(w)
    N, Cc, L = x.shape
    O, K, _ = w.shape
    Lo = (L + 2 * pad - dil * (K - 1) - 1) // stride + 1
    y = np.zeros((N, O, Lo), dtype=np.float32)
    bb = _f32(b) if b is not None else None
    lib().dcref_conv1d(_p(x), N, Cc, L, _p(w), O, K, _p(bb) if bb is not None else None,
                       stride, pad, dil, _p(y))
    return y


def conv2d(x, w, b, sh, sw, ph, pw):
    x, w = _f32(x), _f32(w)
    N, Cc, H, W = x.shape
    O, KH, KW, _ = w.shape
    Ho = (H + 2 * ph - KH) // sh + 1
    Wo = (W + 2 * pw - KW) // sw + 1
    y = np.zeros((N, O, Ho, Wo), dtype=np.float32)
    bb = _f32(b) if b is not None else None
    lib().dcref_conv2d(_p(x), N, Cc, H, W, _p(w), O, KH, KW,
                       _p(bb) if bb is not None else None, sh, sw, ph, pw, _p(y))
    return y


def conv_tr2d(x, w, b, sh, sw):
    x, w = _f32(x), _f32(w)
    N, Cc, H, W = x.shape
    O, KH, KW, _ = w.shape
    y = np.zeros((N, O, (H - 1) * sh + KH, (W - 1) * sw + KW), dtype=np.float32)
    bb = _f32(b) if b is not None else None
    lib().dcref_conv_tr2d(_p(x), N, Cc, H, W, _p(w), O, KH, KW,
                          _p(bb) if bb is not None else None, sh, sw, _p(y))
    return y


def conv_tr1d(x, w, b, stride):
    x, w = _f32(x), _f32(w)
    N, Cc, L = x.shape
    O, K, _ = w.shape
    y = np.zeros((N, O, (L - 1) * stride + K), dtype=np.float32)
    bb = _f32(b) if b is not None else None
    lib().dcref_conv_tr1d(_p(x), N, Cc, L, _p(w), O, K, _p(bb) if bb is not None else None,
                          stride, _p(y))
    return y


def linear(x, w, b):
    x, w = _f32(x), _f32(w)
    R, IN = x.shape
    OUT = w.shape[0]
    y = np.zeros((R, OUT), dtype=np.float32)
    bb = _f32(b) if b is not None else None
    lib().dcref_linear(_p(x), R, IN, _p(w), OUT, _p(bb) if bb is not None else None, _p(y))
    return y


def attention(q, k, v, heads):
    q, k, v = _f32(q), _f32(k), _f32(v)
    B, Tq, D = q.shape
    Tk = k.shape[1]
    y = np.zeros((B, Tq, D), dtype=np.float32)
    lib().dcref_attention(_p(q), _p(k), _p(v), B, Tq, Tk, D, heads, _p(y))
    return y


def groupnorm(x, w, b, groups, act):
    x = _f32(x)
    B, Cc = x.shape[:2]
    S = int(np.prod(x.shape[2:]))
    Co = Cc // 2 if act == 2 else Cc
    y = np.zeros((B, Co) + x.shape[2:], dtype=np.float32)
    lib().dcref_groupnorm(_p(x), B, Cc, S, _p(_f32(w)), _p(_f32(b)), groups, act, _p(y))
    return y


def groupnorm_last(x, w, b):
    x = _f32(x)
    B, T, Cc = x.shape
    y = np.zeros_like(x)
    lib().dcref_groupnorm_last(_p(x), B, T, Cc, _p(_f32(w)), _p(_f32(b)), _p(y))
    return y


def layernorm(x, w, b):
    x = _f32(x)
    R, Cc = x.shape
    y = np.zeros_like(x)
    lib().dcref_layernorm(_p(x), R, Cc, _p(_f32(w)), _p(_f32(b)), _p(y))
    return y


def spec(mix, nfft=4096):
    mix = _f32(mix)
    B, Cc, T = mix.shape
    frames = lib().dcref_spec(_p(mix), B, Cc, T, nfft, None)
    out = np.zeros((B, 2 * Cc, nfft // 2, frames), dtype=np.float32)
    lib().dcref_spec(_p(mix), B, Cc, T, nfft, _p(out))
    return out


def ispec(z, length, nfft=4096):
    z = _f32(z)
    B, S, C2, F, N = z.shape
    y = np.zeros((B, S, C2 // 2, length), dtype=np.float32)
    lib().dcref_ispec(_p(z), B, S, C2, F, N, nfft, length, _p(y))
    return y
