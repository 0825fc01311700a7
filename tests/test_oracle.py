"""The CPU oracle (oracle/port.py) pinned against the reference itself (CPU, no GPU).

* committed digests of reference runs (tests/golden/*_digest.json, made by
  tests/golden/make_golden.py from oracle/_ref) -- always available;
* the reference's own CPU build (oracle/_ref/libdcref.so) when it has been built: op-level
  cases on the reference's test_kernels.c shapes, teacher-forced model stages as
  test_compare.c runs them, and dc_apply_model on a short track.
"""
import json
import os

import numpy as np
import pytest

from conftest import ROOT, model_files, rel_l2

GOLDEN = os.path.join(ROOT, "tests", "golden")


def _ref():
    from oracle import ref
    if not ref.available():
        pytest.skip("oracle/_ref not built (make -C oracle)")
    return ref


def _port_model(name):
    from demucs_cuda_b200 import synth
    from oracle import port
    cfg, w, c = model_files(name)
    return cfg, w, c, synth.load_safetensors(w), port.Config(json.load(open(c)))


def test_port_vs_committed_tiny_digest():
    """port forward vs the reference run recorded in tiny_digest.json (no reference build
    needed): every stage's samples and energy."""
    from demucs_cuda_b200 import synth
    from oracle import port
    dg = json.load(open(os.path.join(GOLDEN, "tiny_digest.json")))
    cfg, w, c, W, pc = _port_model("tiny")
    mix = synth.segment_input(cfg, 1, dg["input_seed"])
    st = {}
    port.forward(mix, W, pc, st)
    for k, d in dg["stages"].items():
        a = np.ascontiguousarray(st[k], np.float32).ravel()
        assert list(st[k].shape) == d["shape"], k
        idx = np.linspace(0, a.size - 1, d["idx_count"]).astype(np.int64)
        e = rel_l2(a[idx], np.array(d["samples"]))
        energy = abs(float((a.astype(np.float64) ** 2).sum()) / d["sumsq"] - 1.0)
        gate = 2e-4 if k == "stems" else 2e-3  # non-teacher-forced stage drift
        assert e < gate and energy < gate, (k, e, energy)


def test_digest_files_consistent():
    for name in ("tiny", "short", "full"):
        p = os.path.join(GOLDEN, f"{name}_digest.json")
        dg = json.load(open(p))
        st = dg["stages"]
        assert st["stems"]["shape"][:3] == [1, 6, 2]
        for k, d in st.items():
            assert np.isfinite(d["sumsq"]) and d["sumsq"] > 0, (name, k)


@pytest.mark.parametrize("case", ["conv1d", "conv2d", "conv_tr2d", "conv_tr1d", "linear",
                                  "attention", "groupnorm", "layernorm", "spec", "ispec"])
def test_port_ops_vs_reference(case):
    """The port's ops against the reference ops.c / backend_cpu.c on the shapes of the
    reference's tests/test_kernels.c."""
    ref = _ref()
    from oracle import port
    rng = np.random.default_rng(12345)
    u = lambda *s: rng.uniform(-1, 1, s).astype(np.float32)  # noqa: E731
    tol = 1e-5
    if case == "conv1d":
        x, w, b = u(2, 13, 101), u(17, 8, 13), u(17)
        got, want = port.conv1d(x, w, b, 4, 2, 1), ref.conv1d(x, w, b, 4, 2, 1)
    elif case == "conv2d":
        x, w, b = u(1, 9, 11, 13), u(10, 3, 3, 9), u(10)
        got, want = port.conv2d(x, w, b, 1, 1, 1, 1), ref.conv2d(x, w, b, 1, 1, 1, 1)
    elif case == "conv_tr2d":
        x, w, b = u(2, 24, 16, 9), u(12, 8, 1, 24), u(12)
        got, want = port.conv_tr2d(x, w, b, 4, 1), ref.conv_tr2d(x, w, b, 4, 1)
    elif case == "conv_tr1d":
        x, w, b = u(2, 19, 23), u(11, 8, 19), u(11)
        got, want = port.conv_tr1d(x, w, b, 4), ref.conv_tr1d(x, w, b, 4)
    elif case == "linear":
        x, w, b = u(130, 384), u(1536, 384), u(1536)
        got, want = port.linear(x, w, b), ref.linear(x, w, b)
    elif case == "attention":
        q, k, v = u(2, 33, 64), u(2, 47, 64), u(2, 47, 64)
        got, want = port.attention(q, k, v, 8), ref.attention(q, k, v, 8)
        tol = 1e-4  # numpy exp vs glibc expf may flip an fp16 rounding of P
    elif case == "groupnorm":
        x, w, b = u(2, 16, 33) * 3 + 0.5, u(16), u(16)
        for act in (0, 1, 2):
            assert rel_l2(port.groupnorm(x, w, b, 1, act), ref.groupnorm(x, w, b, 1, act)) < tol
        got, want = port.groupnorm(x, w, b, 4, 1), ref.groupnorm(x, w, b, 4, 1)
    elif case == "layernorm":
        x, w, b = u(45, 384), u(384), u(384)
        got, want = port.layernorm(x, w, b), ref.layernorm(x, w, b)
    elif case == "spec":
        mix = u(1, 2, 44100) * 0.5
        got, want = port.spec(mix, 4096), ref.spec(mix)
    else:
        z = rng.standard_normal((1, 2, 4, 2048, 44)).astype(np.float32)
        got, want = port.ispec(z, 4096, 44100), ref.ispec(z, 44100)
    assert got.shape == want.shape
    assert rel_l2(got, want) < tol


def test_port_teacher_forced_stages_vs_reference():
    """Each model stage of the port fed the reference's previous-stage output, as
    test_compare.c does, against the reference's stage output (stage gate 8e-4)."""
    ref = _ref()
    from demucs_cuda_b200 import synth
    from oracle import port
    cfg, w, c, W, pc = _port_model("tiny")
    ref.load(w, c)
    mix = synth.segment_input(cfg, 1, 0)
    _, R = ref.forward(mix, stages=True)
    errs = {}
    for i in range(pc.depth):
        xin = R["x_norm"] if i == 0 else R[f"enc_{i - 1}"]
        y = port.henc(xin, W, f"encoder.{i}", True, pc)
        if i == 0:
            emb = W["freq_emb.embedding.weight"][: y.shape[2]].T
            y = (y + (emb * np.float32(pc.freq_emb * pc.emb_scale))[None, :, :, None]).astype(
                np.float32)
        errs[f"enc_{i}"] = rel_l2(y, R[f"enc_{i}"])
        tin = R["xt_norm"] if i == 0 else R[f"tenc_{i - 1}"]
        errs[f"tenc_{i}"] = rel_l2(port.henc(tin, W, f"tencoder.{i}", False, pc), R[f"tenc_{i}"])
    x, xt = port.crosstransformer(R["enc_3"], R["tenc_3"], W, pc)
    errs["transformer_x"] = rel_l2(x, R["transformer_x"])
    errs["transformer_xt"] = rel_l2(xt, R["transformer_xt"])
    tl = [R["xt_norm"].shape[-1]] + [R[f"tenc_{i}"].shape[-1] for i in range(3)]
    for i in range(pc.depth):
        last = i == pc.depth - 1
        xin = R["transformer_x"] if i == 0 else R[f"dec_{i - 1}"]
        y = port.hdec(xin, R[f"enc_{3 - i}"], 0, W, f"decoder.{i}", True, last, pc)
        errs[f"dec_{i}"] = rel_l2(y, R[f"dec_{i}"])
        tin = R["transformer_xt"] if i == 0 else R[f"tdec_{i - 1}"]
        y = port.hdec(tin, R[f"tenc_{3 - i}"], tl[3 - i], W, f"tdecoder.{i}", False, last, pc)
        errs[f"tdec_{i}"] = rel_l2(y, R[f"tdec_{i}"])
    bad = {k: v for k, v in errs.items() if not v < 8e-4}
    assert not bad, bad


def test_port_apply_vs_reference():
    """dc_apply_model (shifts 1, overlap 0.25, batches, tail segments) on a 2.2 s track."""
    ref = _ref()
    from oracle import port
    cfg, w, c, W, pc = _port_model("tiny")
    ref.load(w, c)
    rng = np.random.default_rng(3)
    mix = (rng.uniform(-0.5, 0.5, (1, 2, 97000))).astype(np.float32)
    want = ref.apply_model(mix, shifts=1, overlap=0.25, batch_size=2)
    got = port.apply_model(mix, W, pc, shifts=1, overlap=0.25, batch_size=2)
    assert got.shape == want.shape
    assert rel_l2(got, want) < 2e-4


def test_port_shards_sum_to_full():
    from oracle import port
    cfg, w, c, W, pc = _port_model("tiny")
    rng = np.random.default_rng(4)
    mix = (rng.uniform(-0.5, 0.5, (1, 2, 60000))).astype(np.float32)
    full = port.apply_model(mix, W, pc, shifts=0, batch_size=3)
    parts = sum(port.apply_model(mix, W, pc, shifts=0, batch_size=3, shard=(i, 3))
                for i in range(3))
    assert rel_l2(parts, full) < 1e-6
