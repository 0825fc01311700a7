"""The C-ABI library loads without a GPU and exports every function include/dc_b200.h
declares (no compute calls here)."""
import os
import re
import subprocess

import pytest

from conftest import ROOT
from oracle import REFERENCE_SRC

HEADER = os.path.join(ROOT, "include", "dc_b200.h")
REF_BACKEND_H = os.path.join(REFERENCE_SRC, "backend.h")


def declared_functions(path):
    src = open(path).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = set(re.findall(r"\b((?:dk|dkx|dcb)_[a-z0-9_]+)\s*\(", src))
    return names


def test_header_and_python_list_agree():
    import demucs_cuda_b200 as d
    assert declared_functions(HEADER) == set(d.ALL_SYMBOLS)


def test_library_exports_every_declared_symbol():
    import demucs_cuda_b200 as d
    L = d.lib(load_only=True)
    for name in declared_functions(HEADER):
        assert hasattr(L, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", d.LIB_PATH], capture_output=True,
                         text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    missing = declared_functions(HEADER) - exported
    assert not missing, missing


@pytest.mark.skipif(not os.path.exists(REF_BACKEND_H), reason="reference tree not mounted")
def test_covers_reference_backend_h():
    """Every function of the reference kernel interface has a definition here."""
    ref = declared_functions(REF_BACKEND_H)
    assert ref, "no functions parsed from backend.h"
    assert ref <= declared_functions(HEADER), ref - declared_functions(HEADER)


def test_pack_half_rounding_matches_reference_rule():
    """dk_pack_half is host code: round-to-nearest-even fp16, same bits as numpy's IEEE
    conversion (and as the reference's dc_f32_to_f16, util.c:246-279) including
    subnormals, ties, overflow and NaN."""
    import numpy as np
    import demucs_cuda_b200 as d
    L = d.lib(load_only=True)
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        rng.standard_normal(4000).astype(np.float32) * 10,
        (rng.standard_normal(2000) * 1e-5).astype(np.float32),          # subnormal range
        np.array([65504, 65519.99, 65520, 1e9, -1e9, 0.0, -0.0, np.inf, -np.inf],
                 np.float32),
        np.array([1 + 2 ** -11, 1 + 3 * 2 ** -11, 2 ** -24, 2 ** -25, 3 * 2 ** -25],
                 np.float32),                                             # ties / edges
    ])
    want = vals.astype(np.float16).view(np.uint16)
    got = np.array([L.dk_pack_half(float(v), 1) for v in vals], np.uint16)
    assert (got == want).all()
    nan = L.dk_pack_half(float("nan"), 0)
    assert (nan & 0x7c00) == 0x7c00 and (nan & 0x3ff) != 0


def test_backend_options_round_trip():
    """dcb_set_option (host-only) takes every option include/dc_b200.h documents and returns
    the previous value, so A/B tests can switch a path and put it back."""
    import ctypes
    import demucs_cuda_b200 as d
    L = d.lib(load_only=True)
    L.dcb_set_option.argtypes = [ctypes.c_char_p, ctypes.c_int]
    L.dcb_set_option.restype = ctypes.c_int
    header = open(HEADER).read()
    defaults = {"simt": 0, "graphs": 0, "generic_epilogue": 0, "stream_istft": 1}
    for name, default in defaults.items():
        assert f'"{name}"' in header, name
        old = L.dcb_set_option(name.encode(), 1 - default)
        assert old == default, (name, old)
        assert L.dcb_set_option(name.encode(), old) == 1 - default, name
