"""The CPU twins of the fused entry points (demucs_cuda_b200/twins/dkx_cpu.c), which keep
the reference's CPU backend interchangeable with this library when its model layer calls
dkx_*: each twin, compiled against the reference's backend.h and linked with its CPU
backend (oracle/_ref), must give what the reference computes with the unfused calls it
replaces (ops.c conv_core / conv_tr_core / dc_linear / dc_attention, then the layer's
activation).  CPU only; skipped where the reference tree or its CPU build is absent."""
import ctypes as C
import os
import subprocess

import numpy as np
import pytest

from conftest import ROOT, rel_l2

from oracle import REFERENCE_SRC as REF_SRC
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libdcref.so")
TWINS = os.path.join(ROOT, "demucs_cuda_b200", "twins", "dkx_cpu.c")

pytestmark = pytest.mark.skipif(
    not (os.path.exists(os.path.join(REF_SRC, "backend.h")) and os.path.exists(REF_LIB)),
    reason="reference sources or oracle/_ref not present")


@pytest.fixture(scope="module")
def twins(tmp_path_factory):
    from oracle import ref
    ref.lib()  # the reference CPU backend, loaded first: the twins bind to its dk_* symbols
    out = str(tmp_path_factory.mktemp("twins") / "libdkxcpu.so")
    subprocess.run(["gcc", "-O3", "-std=gnu11", "-fPIC", "-shared", "-ffp-contract=off",
                    "-I", REF_SRC, TWINS, "-o", out, REF_LIB, "-lm",
                    f"-Wl,-rpath,{os.path.dirname(REF_LIB)}"], check=True)
    return C.CDLL(out)


def _geom(C_, H, W, KH, KW, SH, SW, PH, PW, DH=1, DW=1):
    from demucs_cuda_b200 import DkConvGeom
    g = DkConvGeom()
    g.C, g.H, g.W, g.KH, g.KW, g.SH, g.SW, g.PH, g.PW, g.DH, g.DW = (C_, H, W, KH, KW, SH, SW,
                                                                     PH, PW, DH, DW)
    g.Ho = (H + 2 * PH - DH * (KH - 1) - 1) // SH + 1
    g.Wo = (W + 2 * PW - DW * (KW - 1) - 1) // SW + 1
    g.Kp = (KH * KW * C_ + 7) // 8 * 8
    return g


def _pack(w2d):
    """fp16 rows padded to a multiple of 8 (the loader rule, weights.c:306-310)."""
    rows, K = w2d.shape
    kp = (K + 7) // 8 * 8
    out = np.zeros((rows, kp), np.float16)
    out[:, :K] = w2d.astype(np.float32).astype(np.float16)
    return np.ascontiguousarray(out), kp


def _p(a):
    return C.c_void_p(a.ctypes.data) if a is not None else None


@pytest.mark.parametrize("N,C_,H,W,O,KH,KW,SH,SW,PH,PW,act", [
    (2, 4, 64, 9, 24, 8, 1, 4, 1, 2, 0, 0),     # freq encoder conv k(8,1) s(4,1) p(2,0)
    (1, 9, 11, 13, 10, 3, 3, 1, 1, 1, 1, 1),    # 3x3 + GELU
    (1, 48, 16, 20, 96, 1, 1, 1, 1, 0, 0, 2),   # encoder rewrite 1x1 + GLU
    (1, 24, 8, 10, 48, 3, 3, 1, 1, 1, 1, 2),    # decoder rewrite 3x3 + GLU
])
def test_conv2d_twin(twins, N, C_, H, W, O, KH, KW, SH, SW, PH, PW, act):
    from oracle import port, ref
    rng = np.random.default_rng(N * 100 + C_ + O)
    x = rng.uniform(-1, 1, (N, C_, H, W)).astype(np.float32)
    w = (rng.uniform(-1, 1, (O, KH, KW, C_)) / np.sqrt(KH * KW * C_)).astype(np.float32)
    b = rng.uniform(-1, 1, O).astype(np.float32)
    r = ref.conv2d(x, w, b, SH, SW, PH, PW)
    if act == 1:
        r = port.gelu(r)
    elif act == 2:
        r = port.glu(r, axis=1)
    g = _geom(C_, H, W, KH, KW, SH, SW, PH, PW)
    wp, _ = _pack(w.reshape(O, -1))
    y = np.zeros(r.shape, np.float32)
    twins.dkx_conv2d(_p(x), N, C.byref(g), _p(wp), O, _p(b), act, _p(y))
    assert rel_l2(y, r) < 1e-6


@pytest.mark.parametrize("N,C_,H,W,O,axis_h,gelu", [
    (2, 24, 16, 9, 12, True, False),     # frequency decoder k(8,1) s4, crop 2
    (1, 16, 8, 7, 24, True, True),       # with GELU
    (2, 19, 1, 23, 11, False, False),    # time decoder k8 s4 (1-D as H = 1)
    (1, 12, 1, 30, 8, False, True),
])
def test_conv_tr_twin(twins, N, C_, H, W, O, axis_h, gelu):
    from oracle import port, ref
    rng = np.random.default_rng(N * 77 + C_ + O)
    S, K, crop = 4, 8, 2
    x = rng.uniform(-1, 1, (N, C_, H, W)).astype(np.float32)
    wshape = (O, K, 1, C_) if axis_h else (O, 1, K, C_)
    w = (rng.uniform(-1, 1, wshape) / np.sqrt(C_)).astype(np.float32)
    b = rng.uniform(-1, 1, O).astype(np.float32)
    full = ref.conv_tr2d(x, w, b, S if axis_h else 1, 1 if axis_h else S)
    if axis_h:
        out_len = full.shape[2] - 2 * crop
        r = full[:, :, crop:crop + out_len]
    else:
        out_len = full.shape[3] - 2 * crop - 1
        r = full[:, :, :, crop:crop + out_len]
    if gelu:
        r = port.gelu(r)
    r = np.ascontiguousarray(r)
    wp, _ = _pack(w.reshape(O * K, C_))
    KH, KW = (K, 1) if axis_h else (1, K)
    y = np.zeros(r.shape, np.float32)
    twins.dkx_conv_tr(_p(x), N, C_, H, W, _p(wp), O, KH, KW, S, _p(b), crop, out_len,
                      int(gelu), _p(y))
    assert rel_l2(y, r) < 1e-6


@pytest.mark.parametrize("R,IN,OUT", [(37, 50, 29), (130, 384, 96)])
def test_linear_twin(twins, R, IN, OUT):
    from oracle import ref
    rng = np.random.default_rng(R + IN + OUT)
    x = rng.uniform(-1, 1, (R, IN)).astype(np.float32)
    w = (rng.uniform(-1, 1, (OUT, IN)) / np.sqrt(IN)).astype(np.float32)
    b = rng.uniform(-1, 1, OUT).astype(np.float32)
    r = ref.linear(x, w, b)
    wp, kp = _pack(w)
    y = np.zeros((R, OUT), np.float32)
    twins.dkx_linear(_p(x), C.c_int64(R), IN, _p(wp), C.c_int64(kp), OUT, _p(b), _p(y))
    assert rel_l2(y, r) < 1e-6


@pytest.mark.parametrize("B,Tq,Tk,H,hd", [(1, 37, 50, 2, 12), (2, 64, 40, 4, 8)])
def test_attention_twin(twins, B, Tq, Tk, H, hd):
    from oracle import ref
    rng = np.random.default_rng(B * 1000 + Tq + Tk)
    D = H * hd
    q = rng.standard_normal((B, Tq, D)).astype(np.float32)
    k = rng.standard_normal((B, Tk, D)).astype(np.float32)
    v = rng.standard_normal((B, Tk, D)).astype(np.float32)
    r = ref.attention(q, k, v, H)
    y = np.zeros((B, Tq, D), np.float32)
    twins.dkx_attention(_p(q), _p(k), _p(v), B, Tq, Tk, H, hd, _p(y))
    assert rel_l2(y, r) < 1e-6
