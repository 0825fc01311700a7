"""Parity of the configuration bench.py times: full-width htdemucs_6s forwards of several
segments per call, replayed as CUDA graphs (option "graphs"), through dc_apply_model.

* short configuration (every layer at full width, 1 s segments): dcb_apply with batches of
  8 segments and shifts 1, graphs on, over three calls (eager warm-up, capture + replay,
  replay), against the reference's own apply.c on its CPU backend;
* full configuration (7.8 s segments, the benchmark's shapes): dcb_apply running the 7
  segments of a 43 s track as ONE batched forward replayed from a graph, against the same
  track with every segment forwarded alone and eagerly -- that single-segment path is the
  one tests/test_gpu_model.py pins to the reference's digest at this size.  The two agree
  to fp16 rounding noise, not bit for bit: the first stage that differs is the first
  encoder whose DConv runs as a tensor-core conv (frequency encoder 2), where the batch
  changes how tiles map to CTAs and so the order of its fp32 partial sums; a last-bit
  difference before an fp16 operand rounding moves that operand by one unit, and the
  forward carries it to about 5e-5 of the stems (the path's own error against the
  reference is of the same size).  Each run is bit-reproducible.
"""
import numpy as np
import pytest

from conftest import model_files, rel_l2

pytestmark = pytest.mark.gpu

STEMS_GATE = 1e-3


def _apply(torch, model, mix, **kw):
    out = model.apply(torch.from_numpy(mix).cuda(), **kw)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_short_batched_graph_apply_vs_reference(torch_cuda):
    torch = torch_cuda
    import demucs_cuda_b200 as dcb
    from oracle import ref
    cfg, w, c = model_files("short")
    rng = np.random.default_rng(21)
    T = 220000   # 7-8 segment offsets of 1 s at stride 0.75 s (shifts 1 lengthens the view)
    mix = rng.uniform(-0.5, 0.5, (1, 2, T)).astype(np.float32)
    ref.load(w, c)
    want = ref.apply_model(mix, shifts=1, overlap=0.25, batch_size=8)
    model = dcb.Model(w, c)
    nf, nb = model.apply_plan(T, shifts=1, batch_size=8)
    assert nb == 1 and nf >= 7, (nf, nb)   # one batched forward call
    prev = dcb.set_option("graphs", 1)
    try:
        n0 = dcb.kernel_launches()
        outs = [_apply(torch, model, mix, shifts=1, batch_size=8) for _ in range(3)]
        launched = dcb.kernel_launches() - n0
    finally:
        dcb.set_option("graphs", prev)
    for i, o in enumerate(outs):
        e = rel_l2(o, want)
        print(f"call {i}: batched graph apply vs reference apply.c rel_l2 {e:.3e}")
        assert e < STEMS_GATE
    assert rel_l2(outs[2], outs[0]) < 1e-6   # replay == eager
    assert launched > 0 and dcb.device_fault() == 0


def test_full_width_batch7_graph_replay_matches_single_segments(torch_cuda):
    torch = torch_cuda
    import demucs_cuda_b200 as dcb
    from demucs_cuda_b200 import synth
    cfg, w, c = model_files("full")
    seg = cfg.valid_length
    stride = int(0.75 * seg)
    T = 7 * stride - 1000                # offsets 0 .. 6 stride: 7 segments, the last a tail
    mix = synth.track_input(T / cfg.samplerate, cfg.samplerate, seed=3)[:, :, :T]
    mix = np.ascontiguousarray(mix, np.float32)
    model = dcb.Model(w, c)
    nf, nb = model.apply_plan(T, shifts=0, batch_size=8)
    assert (nf, nb) == (7, 1), (nf, nb)
    dcb.set_option("graphs", 0)
    single = _apply(torch, model, mix, shifts=0, batch_size=1)
    prev = dcb.set_option("graphs", 1)
    try:
        outs = [_apply(torch, model, mix, shifts=0, batch_size=8) for _ in range(3)]
    finally:
        dcb.set_option("graphs", prev)
    for i, o in enumerate(outs):
        e = rel_l2(o, single)
        print(f"call {i}: batch-7 forward (graphs) vs 7 single forwards rel_l2 {e:.3e}")
        assert e < 2e-4
    assert rel_l2(outs[2], outs[0]) < 1e-6   # replay == eager capture, same batch
    assert dcb.device_fault() == 0
    del model
