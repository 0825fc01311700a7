"""The reference's own C code driving libdc_b200.so through the backend.h ABI on the GPU.

oracle/Makefile's `abi` target links the reference's unchanged sources (util, config,
tensor, weights, ops, stft, layers, transformer, htdemucs, apply .c) and its own test
programs against libdc_b200.so in place of its CPU backend, as a downstream build of the
reference would link the drop-in library.  No Python or PyTorch is in those processes.

* tests/test_kernels.c and tests/test_stft.c run unchanged and must pass their own gates;
* tests/test_compare.c runs unchanged on goldens that the reference's CPU build writes
  for the same weights and input (every key it reads: mix, mag, x_norm, xt_norm, enc_i,
  tenc_i, transformer_x/xt, dec_i, tdec_i, stems); its teacher-forced stages must meet the
  8e-4 stage gate and the stems the 1e-3 gate (SNR >= 60 dB), tighter than its built-in
  2e-3;
* the refmain.c runner (oracle/_ref/abi/dcabi) runs dc_apply_model (apply.c) on a track,
  compared with the same runner over the CPU backend.
"""
import os
import re
import subprocess

import numpy as np
import pytest

from conftest import CACHE, ROOT, model_files, rel_l2

pytestmark = pytest.mark.gpu

ABI = os.path.join(ROOT, "oracle", "_ref", "abi")
STAGE_GATE = 8e-4
STEMS_GATE = 1e-3


def _bin(name):
    path = os.path.join(ABI, name)
    if not os.path.exists(path):
        pytest.fail(f"{path} missing: build it with `make -C oracle abi` where the reference "
                    "sources are present (it travels with the repository snapshot)")
    return path


def _run(args, timeout=900):
    r = subprocess.run(args, capture_output=True, text=True, timeout=timeout)
    print(r.stdout[-4000:])
    if r.stderr:
        print(r.stderr[-2000:])
    return r


@pytest.mark.parametrize("prog", ["test_kernels", "test_stft"])
def test_reference_kernel_tests_on_b200(torch_cuda, prog):
    r = _run([_bin(prog)])
    assert r.returncode == 0, r.stderr[-500:]
    assert "backend cuda-sm100a" in r.stdout
    checks = [ln for ln in r.stdout.splitlines() if "rel_l2=" in ln or "rel=" in ln]
    assert checks, "no checks printed"
    assert not [ln for ln in checks if "FAIL" in ln]
    assert f"{prog}: OK" in r.stdout


def _goldens(name):
    """Goldens with test_compare.c's keys from the reference's CPU build (cached per
    configuration and weight file)."""
    from demucs_cuda_b200 import synth
    from oracle import ref
    cfg, w, c = model_files(name)
    path = os.path.join(CACHE, f"goldens_{name}.safetensors")
    if not os.path.exists(path) or os.path.getmtime(path) < os.path.getmtime(w):
        ref.load(w, c)
        mix = synth.segment_input(cfg, 1, 0)
        stems, st = ref.forward(mix, stages=True)
        g = {k: np.ascontiguousarray(v, np.float32) for k, v in st.items()}
        g["mix"] = np.ascontiguousarray(mix[0], np.float32)
        g["stems"] = np.ascontiguousarray(stems, np.float32)
        synth.save_safetensors(path + ".tmp", g)
        os.replace(path + ".tmp", path)
    return w, c, path


@pytest.mark.parametrize("name", ["tiny", "short"])
def test_reference_test_compare_on_b200(torch_cuda, name):
    w, c, g = _goldens(name)
    r = _run([_bin("test_compare"), w, c, g])
    assert r.returncode == 0, r.stderr[-500:]
    rel = {}
    for ln in r.stdout.splitlines():
        m = re.match(r"^(\S+)(?: \(end to end\))?\s+rel_l2=([0-9.e+-]+)", ln)
        if m:
            rel[m.group(1)] = float(m.group(2))
    expect = {"mag", "x_norm", "xt_norm", "transformer_x", "transformer_xt", "stems"}
    expect |= {f"{k}_{i}" for k in ("enc", "tenc", "dec", "tdec") for i in range(4)}
    assert expect <= set(rel), expect - set(rel)
    for k, v in rel.items():
        gate = 1e-5 if k in ("mag", "x_norm", "xt_norm") else (
            STEMS_GATE if k == "stems" else STAGE_GATE)
        assert v <= gate, (k, v, gate)
    assert "test_compare: OK" in r.stdout


def test_reference_apply_on_b200(torch_cuda, tmp_path):
    """dc_apply_model (apply.c, shifts 1, overlap 0.25, batches of 2 plus tails) of the
    reference's model code: over libdc_b200.so on the GPU and over backend_cpu.c."""
    cfg, w, c = model_files("tiny")
    rng = np.random.default_rng(5)
    T = 97000
    mix = rng.uniform(-0.5, 0.5, (1, 2, T)).astype("<f4")
    mpath = str(tmp_path / "mix.f32")
    mix.tofile(mpath)
    outs = {}
    for kind, exe in (("gpu", _bin("dcabi")),
                      ("cpu", os.path.join(ROOT, "oracle", "_ref", "dcref"))):
        out = str(tmp_path / f"{kind}.f32")
        r = _run([exe, "apply", w, c, mpath, "1", "2", str(T), out, "1", "2"])
        assert r.returncode == 0, (kind, r.stderr[-500:])
        outs[kind] = np.fromfile(out, "<f4").reshape(1, cfg.n_sources, 2, T)
    e = rel_l2(outs["gpu"], outs["cpu"])
    print(f"apply.c over libdc_b200.so vs over backend_cpu.c: rel_l2 {e:.3e}")
    assert e < STEMS_GATE
