"""Every backend.h function of the drop-in boundary, run on the GPU through libdc_b200.so and
compared with the reference's own CPU backend (backend_cpu.c, built into oracle/_ref) on
the same seeded inputs.

The sizes are odd on purpose, as the reference's tests/test_kernels.c chooses them, so that
K padding, partial tiles, ragged rows and both the vector and the scalar paths of each
kernel run.  Bars: data movement and fp16 conversions are bit-exact (the same
round-to-nearest-even rule); float arithmetic agrees to fp32 rounding (rel L2 <= 1e-6,
the GPU contracts a * b + c into one fused multiply-add where the CPU build rounds twice);
softmax probabilities, rounded to fp16 after an exponential, within one fp16 unit.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

F32 = np.float32


@pytest.fixture(scope="module")
def env(torch_cuda):
    import demucs_cuda_b200 as dcb
    from oracle import ref
    cpu = ref.lib()
    for name, (res, args) in dcb.signatures().items():
        if name.startswith("dk_") and hasattr(cpu, name) and name != "dk_row_stats_noalloc":
            fn = getattr(cpu, name)
            fn.restype, fn.argtypes = res, args
    return {"gpu": dcb.lib(), "cpu": cpu, "torch": torch_cuda, "dcb": dcb}


def _dev(env, a):
    return env["torch"].from_numpy(np.ascontiguousarray(a)).cuda()


def _p(t):
    return C.c_void_p(t.data_ptr())


def _np(a):
    return C.c_void_p(a.ctypes.data)


def _done(env, what):
    env["torch"].cuda.synchronize()
    env["dcb"].check(True, what)
    assert env["dcb"].device_fault() == 0


def _strided(shape, a_strides, b_strides):
    from demucs_cuda_b200 import DkStrided
    p = DkStrided()
    p.ndim = len(shape)
    for i, (n, sa, sb) in enumerate(zip(shape, a_strides, b_strides)):
        p.shape[i], p.a_strides[i], p.b_strides[i] = n, sa, sb
    return p


def _cstrides(shape):
    st, acc = [], 1
    for n in reversed(shape):
        st.append(acc)
        acc *= n
    return list(reversed(st))


# ------------------------------------------------------------------ elementwise / copies
@pytest.mark.parametrize("accumulate", [0, 1])
def test_strided_copy(env, accumulate):
    """A 4-D permutation (copy of a transposed view, tensor.c dc_transpose) and a broadcast
    source (stride 0, dc_broadcast_to), plain and accumulating."""
    rng = np.random.default_rng(1)
    src = rng.standard_normal((3, 5, 7, 11)).astype(F32)
    shape = [11, 3, 7, 5]                      # dst = src.transpose(3, 0, 2, 1)
    sst = _cstrides(src.shape)
    a_str = [sst[3], sst[0], sst[2], sst[1]]
    cases = [(shape, a_str), ([4, 3, 5, 7, 11], [0] + sst)]   # broadcast over a new axis
    for shp, ast in cases:
        n = int(np.prod(shp))
        dst0 = rng.standard_normal(n).astype(F32)
        p = _strided(shp, ast, _cstrides(shp))
        want = dst0.copy()
        env["cpu"].dk_strided_copy(C.byref(p), _np(src), _np(want), accumulate)
        s_t, d_t = _dev(env, src), _dev(env, dst0)
        env["gpu"].dk_strided_copy(C.byref(p), _p(s_t), _p(d_t), accumulate)
        _done(env, "dk_strided_copy")
        got = d_t.cpu().numpy()
        if accumulate:
            assert rel_l2(got, want) < 1e-7
        else:
            assert np.array_equal(got, want)


@pytest.mark.parametrize("op", [0, 1, 2, 3, 4])
def test_binary_broadcast(env, op):
    rng = np.random.default_rng(2 + op)
    shape = [2, 13, 37]
    a = rng.standard_normal(shape).astype(F32)
    b = (rng.standard_normal((13, 1)) + (3.0 if op == 3 else 0.0)).astype(F32)
    p = _strided(shape, _cstrides(shape), [0, 1, 0])       # b [13, 1] broadcast
    n = int(np.prod(shape))
    want = np.zeros(n, F32)
    env["cpu"].dk_binary(op, C.byref(p), _np(a), _np(b), _np(want))
    at, bt = _dev(env, a), _dev(env, b)
    yt = env["torch"].zeros(n, device="cuda")
    env["gpu"].dk_binary(op, C.byref(p), _p(at), _p(bt), _p(yt))
    _done(env, "dk_binary")
    assert np.array_equal(yt.cpu().numpy(), want) or rel_l2(yt.cpu().numpy(), want) < 1e-7


@pytest.mark.parametrize("op,alpha,beta", [(0, 1.7, -0.3), (1, 0, 0), (2, 0, 0), (3, 0, 0)])
def test_unary(env, op, alpha, beta):
    rng = np.random.default_rng(10 + op)
    x = (rng.standard_normal(1001) * 3).astype(F32)
    want = np.zeros_like(x)
    env["cpu"].dk_unary(op, _np(x), _np(want), x.size, alpha, beta)
    xt = _dev(env, x)
    yt = env["torch"].zeros_like(xt)
    env["gpu"].dk_unary(op, _p(xt), _p(yt), x.size, alpha, beta)
    _done(env, "dk_unary")
    assert rel_l2(yt.cpu().numpy(), want) < 1e-6


def test_fill_and_memory(env):
    """dk_fill, dk_memset0, the dk_memcpy family and dk_raw_malloc/free on odd sizes."""
    torch, L = env["torch"], env["gpu"]
    yt = torch.zeros(1003, device="cuda")
    L.dk_fill(_p(yt), 1001, C.c_float(2.5))
    _done(env, "dk_fill")
    y = yt.cpu().numpy()
    assert (y[:1001] == 2.5).all() and (y[1001:] == 0).all()
    n = 777
    host = np.arange(n, dtype=F32)
    back = np.zeros(n, F32)
    d0 = L.dk_raw_malloc(n * 4)
    d1 = L.dk_raw_malloc(n * 4)
    assert d0 and d1
    L.dk_memcpy_h2d(C.c_void_p(d0), _np(host), n * 4)
    L.dk_memcpy_d2d(C.c_void_p(d1), C.c_void_p(d0), n * 4)
    L.dk_memset0(C.c_void_p(d0), 100 * 4)
    L.dk_sync()
    L.dk_memcpy_d2h(_np(back), C.c_void_p(d1), n * 4)
    assert np.array_equal(back, host)
    L.dk_memcpy_d2h(_np(back), C.c_void_p(d0), n * 4)
    assert (back[:100] == 0).all() and np.array_equal(back[100:], host[100:])
    L.dk_raw_free(C.c_void_p(d0))
    L.dk_raw_free(C.c_void_p(d1))
    fr, tot = C.c_size_t(), C.c_size_t()
    assert L.dk_mem_info(C.byref(fr), C.byref(tot)) == 0 and 0 < fr.value <= tot.value
    L.dk_range_push(b"abi-test")
    L.dk_range_pop()
    assert L.dk_backend_name() == b"cuda-sm100a"
    env["dcb"].check(True, "memory")


@pytest.mark.parametrize("outer,half,inner", [(3, 7, 11), (2, 48, 336), (1, 5, 1)])
def test_glu(env, outer, half, inner):
    rng = np.random.default_rng(outer * 100 + half)
    x = rng.standard_normal((outer, 2 * half, inner)).astype(F32) * 2
    want = np.zeros((outer, half, inner), F32)
    env["cpu"].dk_glu(_np(x), _np(want), outer, half, inner)
    xt = _dev(env, x)
    yt = env["torch"].zeros(want.shape, device="cuda")
    env["gpu"].dk_glu(_p(xt), _p(yt), outer, half, inner)
    _done(env, "dk_glu")
    assert rel_l2(yt.cpu().numpy(), want) < 1e-6


@pytest.mark.parametrize("outer,Cc,inner", [(3, 7, 11), (2, 48, 1000), (5, 1, 3)])
def test_channel_bias_and_scale_add(env, outer, Cc, inner):
    rng = np.random.default_rng(outer + Cc + inner)
    y0 = rng.standard_normal((outer, Cc, inner)).astype(F32)
    x = rng.standard_normal((outer, Cc, inner)).astype(F32)
    bias = rng.standard_normal(Cc).astype(F32)
    scale = rng.standard_normal(Cc).astype(F32)
    want_b = y0.copy()
    env["cpu"].dk_channel_bias(_np(want_b), _np(bias), outer, Cc, inner)
    want_s = y0.copy()
    env["cpu"].dk_scale_add(_np(want_s), _np(x), _np(scale), outer, Cc, inner)
    yb, ys = _dev(env, y0), _dev(env, y0)
    keep = [_dev(env, bias), _dev(env, x), _dev(env, scale)]
    env["gpu"].dk_channel_bias(_p(yb), _p(keep[0]), outer, Cc, inner)
    env["gpu"].dk_scale_add(_p(ys), _p(keep[1]), _p(keep[2]), outer, Cc, inner)
    _done(env, "bias/scale_add")
    assert np.array_equal(yb.cpu().numpy(), want_b)
    assert rel_l2(ys.cpu().numpy(), want_s) < 1e-7


@pytest.mark.parametrize("rows,L,left,right", [(3, 37, 5, 9), (4, 351232 // 64, 1536, 1620)])
def test_reflect_pad(env, rows, L, left, right):
    rng = np.random.default_rng(rows + L)
    x = rng.standard_normal((rows, L)).astype(F32)
    want = np.zeros((rows, L + left + right), F32)
    env["cpu"].dk_reflect_pad(_np(x), _np(want), rows, L, left, right)
    xt = _dev(env, x)
    yt = env["torch"].zeros(want.shape, device="cuda")
    env["gpu"].dk_reflect_pad(_p(xt), _p(yt), rows, L, left, right)
    _done(env, "dk_reflect_pad")
    assert np.array_equal(yt.cpu().numpy(), want)


# ------------------------------------------------------------------ normalisation
@pytest.mark.parametrize("rows,L", [(70001, 3), (5, 50001), (1, 8192 * 3 + 1)])
def test_row_stats(env, rows, L):
    """Including more rows than a grid's y dimension holds (70001 > 65535)."""
    rng = np.random.default_rng(rows)
    x = (rng.standard_normal((rows, L)) * 2 + 0.7).astype(F32)
    m0, v0 = np.zeros(rows, F32), np.zeros(rows, F32)
    env["cpu"].dk_row_stats(_np(x), rows, L, _np(m0), _np(v0))
    xt = _dev(env, x)
    st = env["torch"].zeros(2 * rows, device="cuda")
    env["gpu"].dk_row_stats(_p(xt), rows, L, _p(st), C.c_void_p(st.data_ptr() + 4 * rows))
    _done(env, "dk_row_stats")
    s = st.cpu().numpy()
    assert np.abs(s[:rows] - m0).max() <= 1e-6 * (1 + np.abs(m0).max())
    assert rel_l2(s[rows:], v0) < 1e-6


@pytest.mark.parametrize("B,Cc,S,G,act", [(2, 12, 37, 1, 0), (2, 12, 36, 1, 1), (3, 16, 33, 4, 2),
                                          (2, 16, 1000, 4, 2), (1, 6, 4097, 2, 1)])
def test_groupnorm_apply(env, B, Cc, S, G, act):
    rng = np.random.default_rng(B * Cc * S + act)
    x = (rng.standard_normal((B, Cc, S)) * 3 + 0.5).astype(F32)
    mean = rng.standard_normal(B * G).astype(F32)
    var = rng.uniform(0.5, 2.0, B * G).astype(F32)
    w = rng.standard_normal(Cc).astype(F32)
    b = rng.standard_normal(Cc).astype(F32)
    Co = Cc // 2 if act == 2 else Cc
    want = np.zeros((B, Co, S), F32)
    env["cpu"].dk_groupnorm_apply(_np(x), _np(want), _np(mean), _np(var), _np(w), _np(b), B, Cc,
                                  S, G, C.c_float(1e-5), act)
    keep = [_dev(env, a) for a in (x, mean, var, w, b)]
    yt = env["torch"].zeros(want.shape, device="cuda")
    env["gpu"].dk_groupnorm_apply(_p(keep[0]), _p(yt), *[_p(k) for k in keep[1:]], B, Cc, S, G,
                                  C.c_float(1e-5), act)
    _done(env, "dk_groupnorm_apply")
    assert rel_l2(yt.cpu().numpy(), want) < 1e-6


@pytest.mark.parametrize("rows,L,Cc,affine", [(3, 384 * 5, 384, True), (3, 50 * 7, 50, True),
                                              (2, 37, 37, False), (4, 6 * 9, 6, True)])
def test_norm_apply_last(env, rows, L, Cc, affine):
    rng = np.random.default_rng(rows * L + Cc)
    x = rng.standard_normal((rows, L)).astype(F32)
    mean = rng.standard_normal(rows).astype(F32)
    var = rng.uniform(0.5, 2.0, rows).astype(F32)
    w = rng.standard_normal(Cc).astype(F32)
    b = rng.standard_normal(Cc).astype(F32)
    want = np.zeros_like(x)
    env["cpu"].dk_norm_apply_last(_np(x), _np(want), _np(mean), _np(var),
                                  _np(w) if affine else None, _np(b) if affine else None, rows,
                                  L, Cc, C.c_float(1e-5))
    keep = [_dev(env, a) for a in (x, mean, var, w, b)]
    yt = env["torch"].zeros(want.shape, device="cuda")
    env["gpu"].dk_norm_apply_last(_p(keep[0]), _p(yt), _p(keep[1]), _p(keep[2]),
                                  _p(keep[3]) if affine else None,
                                  _p(keep[4]) if affine else None, rows, L, Cc, C.c_float(1e-5))
    _done(env, "dk_norm_apply_last")
    assert rel_l2(yt.cpu().numpy(), want) < 1e-6


@pytest.mark.parametrize("rows,L,denorm", [(2, 343980 * 2, 0), (2, 4099, 1), (3, 36, 1)])
def test_affine_rows(env, rows, L, denorm):
    rng = np.random.default_rng(rows + L + denorm)
    x = rng.standard_normal((rows, L)).astype(F32)
    mean = rng.standard_normal(rows).astype(F32)
    var = rng.uniform(0.01, 2.0, rows).astype(F32)
    want = np.zeros_like(x)
    env["cpu"].dk_affine_rows(_np(x), _np(want), _np(mean), _np(var), rows, L, C.c_float(1e-5),
                              denorm)
    keep = [_dev(env, a) for a in (x, mean, var)]
    yt = env["torch"].zeros(want.shape, device="cuda")
    env["gpu"].dk_affine_rows(_p(keep[0]), _p(yt), _p(keep[1]), _p(keep[2]), rows, L,
                              C.c_float(1e-5), denorm)
    _done(env, "dk_affine_rows")
    assert rel_l2(yt.cpu().numpy(), want) < 1e-6


@pytest.mark.parametrize("R,Cc", [(45, 384), (13, 50), (5, 1536)])
def test_layernorm_paths(env, R, Cc):
    """Vector rows (C a multiple of 128), scalar rows, and rows longer than a warp holds."""
    rng = np.random.default_rng(R + Cc)
    x = rng.standard_normal((R, Cc)).astype(F32)
    w = rng.standard_normal(Cc).astype(F32)
    b = rng.standard_normal(Cc).astype(F32)
    want = np.zeros_like(x)
    env["cpu"].dk_layernorm(_np(x), _np(want), _np(w), _np(b), R, Cc, C.c_float(1e-5))
    keep = [_dev(env, a) for a in (x, w, b)]
    yt = env["torch"].zeros(want.shape, device="cuda")
    env["gpu"].dk_layernorm(_p(keep[0]), _p(yt), _p(keep[1]), _p(keep[2]), R, Cc,
                            C.c_float(1e-5))
    _done(env, "dk_layernorm")
    assert rel_l2(yt.cpu().numpy(), want) < 2e-6


# ------------------------------------------------------------------ GEMM operand preparation
def _u16(env, shape):
    return env["torch"].zeros(shape, dtype=env["torch"].int16, device="cuda")


def _bits(t):
    return t.cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("rows,Cc,Cp", [(37, 50, 56), (5, 384, 384), (7, 13, 21)])
def test_to_half_rows(env, rows, Cc, Cp):
    rng = np.random.default_rng(rows + Cc)
    x = (rng.standard_normal((rows, Cc)) * 100).astype(F32)
    want = np.zeros((rows, Cp), np.uint16)
    env["cpu"].dk_to_half_rows(_np(x), _np(want), rows, Cc, Cp)
    xt = _dev(env, x)
    yt = _u16(env, (rows, Cp))
    env["gpu"].dk_to_half_rows(_p(xt), _p(yt), rows, Cc, Cp)
    _done(env, "dk_to_half_rows")
    assert np.array_equal(_bits(yt), want)


@pytest.mark.parametrize("batch,Cc,P,Cp", [(3, 19, 101, 24), (1, 64, 130, 64), (2, 5, 7, 9)])
def test_transpose_to_half(env, batch, Cc, P, Cp):
    rng = np.random.default_rng(batch * Cc + P)
    x = (rng.standard_normal((batch, Cc, P)) * 10).astype(F32)
    want = np.zeros((batch, P, Cp), np.uint16)
    env["cpu"].dk_transpose_to_half(_np(x), _np(want), batch, Cc, P, Cp)
    xt = _dev(env, x)
    yt = _u16(env, (batch, P, Cp))
    env["gpu"].dk_transpose_to_half(_p(xt), _p(yt), batch, Cc, P, Cp)
    _done(env, "dk_transpose_to_half")
    assert np.array_equal(_bits(yt), want)


def _geom(Cc, H, W, KH, KW, SH, SW, PH, PW, DH=1, DW=1, transposed=False):
    from demucs_cuda_b200 import DkConvGeom
    g = DkConvGeom()
    g.C, g.H, g.W, g.KH, g.KW, g.SH, g.SW, g.PH, g.PW, g.DH, g.DW = (Cc, H, W, KH, KW, SH, SW,
                                                                     PH, PW, DH, DW)
    if transposed:   # full output minus the crop on both sides
        g.Ho = (H - 1) * SH + KH - 2 * PH
        g.Wo = (W - 1) * SW + KW - 2 * PW
    else:
        g.Ho = (H + 2 * PH - DH * (KH - 1) - 1) // SH + 1
        g.Wo = (W + 2 * PW - DW * (KW - 1) - 1) // SW + 1
    g.Kp = (KH * KW * Cc + 7) // 8 * 8
    return g


@pytest.mark.parametrize("N,n0,nb,p0,np_,geom", [
    (2, 0, 2, 0, None, (4, 64, 9, 8, 1, 4, 1, 2, 0)),        # conv2d k8x1 s4 p2
    (1, 0, 1, 0, None, (9, 11, 13, 3, 3, 1, 1, 1, 1)),       # conv2d 3x3 pad 1
    (3, 1, 2, 17, 40, (13, 1, 101, 1, 8, 1, 4, 0, 2)),       # conv1d k8 s4, item/position slice
    (1, 0, 1, 0, None, (24, 1, 64, 1, 3, 1, 1, 0, 4, 1, 4)),  # conv1d k3 dilation 4
])
def test_im2col_half(env, N, n0, nb, p0, np_, geom):
    g = _geom(*geom)
    rng = np.random.default_rng(g.C * g.H + g.W)
    x = rng.standard_normal((N, g.C, g.H, g.W)).astype(F32)
    npos = np_ if np_ is not None else g.Ho * g.Wo
    want = np.zeros((nb, npos, g.Kp), np.uint16)
    env["cpu"].dk_im2col_half(_np(x), _np(want), C.byref(g), n0, nb, p0, npos)
    xt = _dev(env, x)
    yt = _u16(env, (nb, npos, g.Kp))
    env["gpu"].dk_im2col_half(_p(xt), _p(yt), C.byref(g), n0, nb, p0, npos)
    _done(env, "dk_im2col_half")
    assert np.array_equal(_bits(yt), want)


@pytest.mark.parametrize("nb,O,geom", [
    (2, 12, (24, 16, 9, 8, 1, 4, 1, 2, 0)),     # freq decoder: k8x1 s4, crop 2 rows
    (2, 11, (19, 1, 23, 1, 8, 1, 4, 0, 2)),     # time decoder: k1x8 s1x4, crop 2 columns
    (1, 5, (7, 6, 5, 3, 3, 2, 2, 1, 0)),        # generic 3x3 stride 2, uneven crop
    (1, 3, (4, 5, 4, 2, 2, 2, 2, 0, 0)),        # kernel = stride (one tap per output)
])
def test_col2im_tr(env, nb, O, geom):
    g = _geom(*geom, transposed=True)
    rng = np.random.default_rng(nb * O + g.H)
    M = O * g.KH * g.KW
    cols = rng.standard_normal((nb, M, g.H * g.W)).astype(F32)
    bias = rng.standard_normal(O).astype(F32)
    for with_bias in (True, False):
        want = np.zeros((nb, O, g.Ho, g.Wo), F32)
        env["cpu"].dk_col2im_tr(_np(cols), _np(want), _np(bias) if with_bias else None, nb, O,
                                C.byref(g))
        keep = [_dev(env, cols), _dev(env, bias)]
        yt = env["torch"].zeros(want.shape, device="cuda")
        env["gpu"].dk_col2im_tr(_p(keep[0]), _p(yt), _p(keep[1]) if with_bias else None, nb, O,
                                C.byref(g))
        _done(env, "dk_col2im_tr")
        assert np.array_equal(yt.cpu().numpy(), want)  # same taps, same summation order


@pytest.mark.parametrize("rows,L,lds,ldp", [(37, 47, 47, 48), (9, 300, 304, 304),
                                            (5, 1343, 1344, 1351)])
def test_softmax_to_half(env, rows, L, lds, ldp):
    rng = np.random.default_rng(rows + L)
    s = (rng.standard_normal((rows, lds)) * 4).astype(F32)
    want = np.zeros((rows, ldp), np.uint16)
    scale = C.c_float(1.0 / np.sqrt(48.0))
    env["cpu"].dk_softmax_to_half(_np(s), lds, _np(want), ldp, rows, L, scale)
    st = _dev(env, s)
    yt = _u16(env, (rows, ldp))
    env["gpu"].dk_softmax_to_half(_p(st), lds, _p(yt), ldp, rows, L, scale)
    _done(env, "dk_softmax_to_half")
    got = _bits(yt)
    assert (got[:, L:] == 0).all()
    g32 = got.view(np.float16).astype(np.float64)
    w32 = want.view(np.float16).astype(np.float64)
    ulp = np.maximum(np.spacing(np.abs(w32).astype(np.float16)).astype(np.float64), 2.0 ** -24)
    assert (np.abs(g32 - w32) <= ulp).all()
    assert rel_l2(g32, w32) < 1e-3


@pytest.mark.parametrize("transpose,B,T,H,hd,hdp,Tp", [(0, 2, 47, 8, 48, 48, 0),
                                                      (0, 1, 33, 8, 8, 16, 0),
                                                      (1, 2, 47, 8, 48, 0, 48),
                                                      (1, 1, 1343, 8, 48, 0, 1344),
                                                      (1, 2, 33, 3, 5, 0, 40)])
def test_split_heads_half(env, transpose, B, T, H, hd, hdp, Tp):
    rng = np.random.default_rng(B * T + hd)
    x = rng.standard_normal((B, T, H * hd)).astype(F32)
    shape = (B, H, hd, Tp) if transpose else (B, H, T, hdp)
    want = np.zeros(shape, np.uint16)
    env["cpu"].dk_split_heads_half(_np(x), _np(want), B, T, H, hd, hdp, Tp, transpose)
    xt = _dev(env, x)
    yt = _u16(env, shape)
    env["gpu"].dk_split_heads_half(_p(xt), _p(yt), B, T, H, hd, hdp, Tp, transpose)
    _done(env, "dk_split_heads_half")
    assert np.array_equal(_bits(yt), want)
