"""Isolated kernel timings of the hot path on one B200: the conv GEMM shapes of the
htdemucs_6s encoders/decoders, one cross-transformer layer pair at dim 512 (8 heads, head
dim 64, FFN 2048, batch 8), and the fused attention at the model's shapes.

    python -m demucs_cuda_b200.kernel_bench [--cases conv,convx,layer,attn] [--reps 20]

Every number is device time from CUDA events around the kernel launches only (the library's
per-class launch trace, dcb_trace_*), averaged over `reps` launches after two warm-up
launches, with L2 flushed (a 256 MB buffer rewritten) between launches; each result is
printed as one JSON line as soon as it is measured.  Parity is checked on reduced shapes
against a float64 torch product of the same fp16 operands, never at full size.  Fractions
are of the measured peaks (MEASURED_PEAKS.json beside the repository root: HBM copy GB/s,
dense bf16 TFLOP/s burst).

Shapes: conv GEMMs through dk_gemm_half as ops.c calls it (A = weights [M][K], B = im2col
positions [N][K], C fp32 [M][N]; reference gemm.cu:162-195) and the same convolutions
through the implicit-GEMM entry point dkx_conv2d from the fp32 NCHW input (no im2col buffer);
the transformer layer through the engine's cross transformer (transformer.c:160-216) on a
synthetic model of channels 64 (dim 512 at the bottom); attention through dkx_attention.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, M, N, K): rows (output channels) x positions x reduction, from the model's layers
CONV_GEMMS = [
    ("enc0_freq", 48, 172032, 32),
    ("enc1_freq", 96, 43008, 384),
    ("enc2_freq", 192, 10752, 768),
    ("enc3_freq", 384, 2688, 1536),
    ("tenc0", 48, 85995, 16),
    ("tenc1", 96, 21499, 384),
    ("rewrite0_freq", 96, 172032, 48),
    ("dec3_rewrite_freq", 96, 172032, 432),
    ("dec0_rewrite_freq", 768, 2688, 3456),
    ("convtr3_freq", 192, 172032, 48),
    ("convtr2_freq", 384, 43008, 96),
    ("convtr3_time", 96, 85995, 48),
]

# implicit-GEMM convs from fp32 NCHW: (name, N, C, H, W, O, KH, KW, SH, SW, PH, PW, act)
CONVS = [
    ("enc0_freq_k8s4", 1, 4, 2048, 336, 48, 8, 1, 4, 1, 2, 0, 1),
    ("enc1_freq_k8s4", 1, 48, 512, 336, 96, 8, 1, 4, 1, 2, 0, 1),
    ("rewrite0_freq_1x1_glu", 1, 48, 512, 336, 96, 1, 1, 1, 1, 0, 0, 2),
    ("dec3_rewrite_3x3_glu", 1, 48, 512, 336, 96, 3, 3, 1, 1, 1, 1, 2),
    ("dec0_rewrite_3x3_glu", 1, 384, 8, 336, 768, 3, 3, 1, 1, 1, 1, 2),
]


def _peaks():
    p = os.path.join(os.path.dirname(HERE), "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


def _emit(rec):
    print(json.dumps(rec), flush=True)


class Flusher:
    """Rewrites a buffer larger than L2 so every timed launch starts from DRAM."""

    def __init__(self, torch):
        self.buf = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")

    def __call__(self):
        self.buf.fill_(1.0)


def _timed(dcb, torch, fn, cls, reps, flush):
    """Mean device ms per launch of trace class `cls` inside fn, and the traced totals."""
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    ms = fl = by = 0.0
    n = 0
    for _ in range(reps):
        flush()
        torch.cuda.synchronize()
        dcb.trace_start([cls])
        fn()
        t = dcb.trace_stop()[cls]
        ms += t["ms"]
        fl += t["flops"]
        by += t["bytes"]
        n += t["launches"]
    if n == 0:
        raise RuntimeError(f"no {cls} launch traced")
    return ms / reps, fl / reps, by / reps, n / reps


def _rates(rec, ms, flops, nbytes, hbm, tf, kind):
    rec.update({"ms": ms, "tflops": flops / ms / 1e9, "gbs": nbytes / ms / 1e6,
                "algorithmic_flops": flops, "algorithmic_bytes": nbytes})
    ai = flops / max(nbytes, 1.0)
    roof = min(tf, ai * hbm / 1e3)   # TFLOP/s attainable at this arithmetic intensity
    rec["frac_of_tensor_peak"] = rec["tflops"] / tf
    rec["frac_of_roofline"] = rec["tflops"] / roof
    rec["bound"] = "tensor" if ai * hbm / 1e3 >= tf else "hbm"
    rec["peaks"] = {"hbm_gbs": hbm, "tflops": tf, "kind": kind}
    return rec


def case_conv_gemm(dcb, torch, reps, flush, hbm, tf, kind):
    """dk_gemm_half at the conv shapes (fp16 operands in memory, fp32 C)."""
    rng = torch.Generator(device="cuda").manual_seed(0)
    # parity on a reduced shape of every kind of call: shared weights, batched positions
    A = torch.randn((96, 384), generator=rng, device="cuda").half()
    B = torch.randn((2, 1000, 384), generator=rng, device="cuda").half()
    got = dcb.gemm_half(A, B)
    want = torch.matmul(A.double(), B.double().transpose(1, 2))
    err = float((got.double() - want).norm() / want.norm())
    _emit({"case": "conv_gemm_parity", "shape": [96, 1000, 384, 2], "rel_l2": err,
           "ok": err < 2e-5})
    for name, M, N, K in CONV_GEMMS:
        Kp = (K + 7) // 8 * 8
        A = torch.randn((M, Kp), generator=rng, device="cuda").half()
        Bm = torch.randn((N, Kp), generator=rng, device="cuda").half()
        Cm = torch.empty((1, M, N), device="cuda", dtype=torch.float32)
        if Kp != K:
            A[:, K:] = 0
            Bm[:, K:] = 0
        ms, fl, by, n = _timed(dcb, torch, lambda: dcb.gemm_half(A, Bm, Cm), "gemm_half", reps,
                               flush)
        _emit(_rates({"case": "conv_gemm", "name": name, "M": M, "N": N, "K": K,
                      "entry": "dk_gemm_half"}, ms, fl, by, hbm, tf, kind))


def case_convx(dcb, torch, reps, flush, hbm, tf, kind):
    """dkx_conv2d: implicit-GEMM conv from fp32 NCHW with the fused epilogue."""
    rng = torch.Generator(device="cuda").manual_seed(1)
    L = dcb.lib()
    for name, N, Cc, H, W, O, KH, KW, SH, SW, PH, PW, act in CONVS:
        g = dcb.DkConvGeom()
        g.C, g.H, g.W, g.KH, g.KW, g.SH, g.SW, g.PH, g.PW, g.DH, g.DW = (Cc, H, W, KH, KW, SH,
                                                                         SW, PH, PW, 1, 1)
        g.Ho = (H + 2 * PH - KH) // SH + 1
        g.Wo = (W + 2 * PW - KW) // SW + 1
        g.Kp = (KH * KW * Cc + 7) // 8 * 8
        x = torch.randn((N, Cc, H, W), generator=rng, device="cuda")
        w = (torch.randn((O, g.Kp), generator=rng, device="cuda") / np.sqrt(KH * KW * Cc)).half()
        w[:, KH * KW * Cc:] = 0
        b = torch.randn((O,), generator=rng, device="cuda")
        Oy = O // 2 if act == 2 else O
        y = torch.empty((N, Oy, g.Ho, g.Wo), device="cuda")

        def run():
            L.dkx_conv2d(C.c_void_p(x.data_ptr()), N, C.byref(g), C.c_void_p(w.data_ptr()), O,
                         C.c_void_p(b.data_ptr()), act, C.c_void_p(y.data_ptr()))

        ms, fl, by, n = _timed(dcb, torch, run, "conv", reps, flush)
        dcb.check(True, name)
        _emit(_rates({"case": "conv_implicit", "name": name, "M": O,
                      "N": N * g.Ho * g.Wo, "K": KH * KW * Cc, "entry": "dkx_conv2d"},
                     ms, fl, by, hbm, tf, kind))


def case_attention(dcb, torch, reps, flush, hbm, tf, kind):
    """dkx_attention (fused flash kernel) at the model's shapes; parity on a reduced one."""
    rng = torch.Generator(device="cuda").manual_seed(2)
    L = dcb.lib()

    def attn(q, k, v, H):
        B_, Tq, D = q.shape
        y = torch.empty_like(q)
        L.dkx_attention(C.c_void_p(q.data_ptr()), C.c_void_p(k.data_ptr()),
                        C.c_void_p(v.data_ptr()), B_, Tq, k.shape[1], H, D // H,
                        C.c_void_p(y.data_ptr()))
        return y

    for hd in (48, 64):
        D, H = 8 * hd, 8
        q = torch.randn((1, 300, D), generator=rng, device="cuda")
        k = torch.randn((1, 257, D), generator=rng, device="cuda")
        v = torch.randn((1, 257, D), generator=rng, device="cuda")
        got = attn(q, k, v, H)
        qh = q.half().double().view(1, 300, H, hd).transpose(1, 2)
        kh = k.half().double().view(1, 257, H, hd).transpose(1, 2)
        vh = v.half().double().view(1, 257, H, hd).transpose(1, 2)
        p = torch.softmax(qh @ kh.transpose(-1, -2) / np.sqrt(hd), dim=-1)
        want = (p @ vh).transpose(1, 2).reshape(1, 300, D)
        err = float((got.double() - want).norm() / want.norm())
        _emit({"case": "attention_parity", "head_dim": hd, "rel_l2": err, "ok": err < 2e-3})
    shapes = [("freq_self_hd48", 8, 2688, 2688, 48), ("time_self_hd48", 8, 1344, 1344, 48),
              ("cross_f_t_hd48", 8, 2688, 1344, 48), ("freq_self_hd64", 8, 2688, 2688, 64),
              ("cross_f_t_hd64", 8, 2688, 1343, 64)]
    for name, B_, Tq, Tk, hd in shapes:
        D, H = 8 * hd, 8
        q = torch.randn((B_, Tq, D), generator=rng, device="cuda")
        k = torch.randn((B_, Tk, D), generator=rng, device="cuda")
        v = torch.randn((B_, Tk, D), generator=rng, device="cuda")
        ms, fl, by, n = _timed(dcb, torch, lambda: attn(q, k, v, H), "attention", reps, flush)
        _emit(_rates({"case": "attention", "name": name, "batch": B_, "heads": H, "Tq": Tq,
                      "Tk": Tk, "head_dim": hd, "entry": "dkx_attention (flash kernel only)"},
                     ms, fl, by, hbm, tf, kind))


def case_layer(dcb, torch, reps, flush, hbm, tf, kind):
    """One self + one cross layer per branch of the cross transformer at dim 512, batch 8:
    freq tokens 8 x 336 = 2688, time tokens 1344 (QKV [8 2688, 512] x [512, 1536], FFN
    512 -> 2048 -> 512, 8 heads of 64)."""
    from demucs_cuda_b200 import synth
    cfg = synth.ModelConfig(channels=64, t_layers=2, segment=1.0)
    d = os.path.join(tempfile.gettempdir(), "demucs_b200_kernel_bench", "layer_d512")
    w, c = synth.write_model(d, cfg, seed=1)
    model = dcb.Model(w, c)
    rng = torch.Generator(device="cuda").manual_seed(3)
    Bn, D = 8, 512
    x0 = torch.randn((Bn, D, 8, 336), generator=rng, device="cuda")
    xt0 = torch.randn((Bn, D, 1344), generator=rng, device="cuda")
    assert model.n_sources == 6
    classes = ["linear", "attention"]

    def run():
        model.stage_transformer(x0, xt0)

    for _ in range(2):
        run()
    torch.cuda.synchronize()
    tot = {k: [0.0, 0.0, 0.0] for k in classes}
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wall = 0.0
    for _ in range(reps):
        flush()
        torch.cuda.synchronize()
        dcb.trace_start(classes)
        e0.record()
        run()
        e1.record()
        tr = dcb.trace_stop()
        wall += e0.elapsed_time(e1)
        for k in classes:
            tot[k][0] += tr[k]["ms"]
            tot[k][1] += tr[k]["flops"]
            tot[k][2] += tr[k]["bytes"]
    rec = {"case": "transformer_layer_pair", "dim": D, "heads": 8, "head_dim": 64, "ffn": 2048,
           "batch": Bn, "freq_tokens": 2688, "time_tokens": 1344,
           "ms_per_call_events": wall / reps, "entry": "dcb_stage_transformer (2 layers)"}
    for k in classes:
        ms, fl, by = (v / reps for v in tot[k])
        rec[k] = _rates({}, ms, fl, by, hbm, tf, kind)
    _emit(rec)
    model.close()


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--cases", default="conv,convx,layer,attn")
    ap.add_argument("--reps", type=int, default=20)
    args = ap.parse_args(argv)
    import torch
    sys.path.insert(0, os.path.dirname(HERE))
    import demucs_cuda_b200 as dcb
    dcb.require_gpu()
    hbm, tf, kind = _peaks()
    flush = Flusher(torch)
    table = {"conv": case_conv_gemm, "convx": case_convx, "layer": case_layer,
             "attn": case_attention}
    for name in args.cases.split(","):
        table[name](dcb, torch, args.reps, flush, hbm, tf, kind)
    fault = dcb.device_fault()
    _emit({"case": "done", "device_fault": fault})
    return 1 if fault else 0


if __name__ == "__main__":
    sys.exit(main())
