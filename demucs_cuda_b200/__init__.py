"""B200 (sm_100a) backend for demucs-cuda's htdemucs_6s hot path.

The product is the C-ABI library libdc_b200.so (include/dc_b200.h): the reference's
backend.h kernel interface, fused tensor-core entry points and an htdemucs_6s engine.
This module is the Python host side over that ABI (ctypes), mirroring the reference's
model-level calls: load weights (dc_weights_load + dc_model_init), forward
(dc_htdemucs_forward), per-stage calls (dc_henc / dc_hdec / dc_crosstransformer as
test_compare.c uses them) and the segment scheduler (dc_apply_model).

PyTorch only provides device memory and the stream; there is no fallback: if the CUDA
library is missing or no sm_100 GPU is present, every call raises.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdc_b200.so")

_F = C.c_void_p
STAGE_FN = C.CFUNCTYPE(None, C.c_char_p, C.c_void_p, C.c_int, C.POINTER(C.c_int), C.c_void_p)

# every symbol include/dc_b200.h declares (checked by tests/test_abi.py)
BACKEND_SYMBOLS = [
    "dk_pack_half", "dk_init", "dk_backend_name", "dk_sync", "dk_raw_malloc", "dk_raw_free",
    "dk_memcpy_h2d", "dk_memcpy_d2h", "dk_memcpy_d2d", "dk_memset0", "dk_mem_info",
    "dk_range_push", "dk_range_pop", "dk_strided_copy", "dk_binary", "dk_unary", "dk_fill",
    "dk_glu", "dk_channel_bias", "dk_scale_add", "dk_reflect_pad", "dk_row_stats",
    "dk_groupnorm_apply", "dk_norm_apply_last", "dk_affine_rows", "dk_layernorm",
    "dk_to_half_rows", "dk_transpose_to_half", "dk_im2col_half", "dk_col2im_tr",
    "dk_gemm_half", "dk_softmax_to_half", "dk_split_heads_half", "dk_stft",
    "dk_istft_frames", "dk_ola",
]
FUSED_SYMBOLS = ["dkx_conv2d", "dkx_conv_tr", "dkx_linear", "dkx_attention"]
NOALLOC_SYMBOLS = ["dk_row_stats_noalloc"]
ENGINE_SYMBOLS = [
    "dcb_set_error_mode", "dcb_last_error", "dcb_set_stream", "dcb_use_own_stream",
    "dcb_get_stream",
    "dcb_set_option", "dcb_kernel_launches", "dcb_device_fault", "dcb_trace_start",
    "dcb_trace_stop", "dcb_trace_dump", "dcb_model_load", "dcb_model_load_layout",
    "dcb_model_save_packed", "dcb_model_load_packed",
    "dcb_model_free", "dcb_model_info", "dcb_model_weight_bytes", "dcb_model_weight_block",
    "dcb_forward", "dcb_stage_encoder", "dcb_stage_decoder", "dcb_stage_transformer",
    "dcb_apply_defaults", "dcb_apply", "dcb_apply_plan", "dcb_py_randint", "dcb_segment_plan",
    "dcb_apply_window", "dcb_apply_shard", "dcb_merge_windows", "dcb_apply_host",
]
ALL_SYMBOLS = BACKEND_SYMBOLS + NOALLOC_SYMBOLS + FUSED_SYMBOLS + ENGINE_SYMBOLS


class DkStrided(C.Structure):
    _fields_ = [("ndim", C.c_int), ("shape", C.c_int64 * 8), ("a_strides", C.c_int64 * 8),
                ("b_strides", C.c_int64 * 8)]


class DkConvGeom(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("C", "H", "W", "KH", "KW", "SH", "SW", "PH", "PW",
                                       "DH", "DW", "Ho", "Wo")] + [("Kp", C.c_int64)]


class DcbApplyOpts(C.Structure):
    _fields_ = [("shifts", C.c_int), ("split", C.c_int), ("overlap", C.c_float),
                ("transition_power", C.c_float), ("batch_size", C.c_int), ("seed", C.c_uint),
                ("use_seed", C.c_int), ("shard_index", C.c_int), ("shard_count", C.c_int)]


_lib = None


class BackendError(RuntimeError):
    pass


def lib(load_only: bool = False):
    """Load libdc_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise BackendError(f"{LIB_PATH} is missing: build it with `python -m "
                           "demucs_cuda_b200.build` (or __graft_entry__.build())")
    L = C.CDLL(LIB_PATH)
    for name, (res, args) in signatures().items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    if not load_only:
        L.dcb_set_error_mode(1)  # record errors; Python raises them
    _lib = L
    return L


def signatures():
    """ctypes (restype, argtypes) of every exported function, by name.  The Part-1 entries
    are the reference backend.h signatures, so the same table also binds the reference's
    own CPU backend for side-by-side checks."""
    i64, i32, f32, vp, sz = C.c_int64, C.c_int, C.c_float, C.c_void_p, C.c_size_t
    return {
        "dk_pack_half": (C.c_uint16, [f32, i32]),
        "dk_init": (i32, [i32, C.c_char_p, sz]),
        "dk_backend_name": (C.c_char_p, []),
        "dk_sync": (None, []),
        "dk_raw_malloc": (vp, [sz]),
        "dk_raw_free": (None, [vp]),
        "dk_memcpy_h2d": (None, [vp, vp, sz]),
        "dk_memcpy_d2h": (None, [vp, vp, sz]),
        "dk_memcpy_d2d": (None, [vp, vp, sz]),
        "dk_memset0": (None, [vp, sz]),
        "dk_mem_info": (i32, [C.POINTER(sz), C.POINTER(sz)]),
        "dk_range_push": (None, [C.c_char_p]),
        "dk_range_pop": (None, []),
        "dk_strided_copy": (None, [C.POINTER(DkStrided), vp, vp, i32]),
        "dk_binary": (None, [i32, C.POINTER(DkStrided), vp, vp, vp]),
        "dk_unary": (None, [i32, vp, vp, i64, f32, f32]),
        "dk_fill": (None, [vp, i64, f32]),
        "dk_glu": (None, [vp, vp, i64, i64, i64]),
        "dk_channel_bias": (None, [vp, vp, i64, i64, i64]),
        "dk_scale_add": (None, [vp, vp, vp, i64, i64, i64]),
        "dk_reflect_pad": (None, [vp, vp, i64, i64, i64, i64]),
        "dk_row_stats": (None, [vp, i64, i64, vp, vp]),
        "dk_row_stats_noalloc": (i32, [vp, i64, i64, vp, vp]),
        "dk_groupnorm_apply": (None, [vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, f32, i32]),
        "dk_norm_apply_last": (None, [vp, vp, vp, vp, vp, vp, i64, i64, i64, f32]),
        "dk_affine_rows": (None, [vp, vp, vp, vp, i64, i64, f32, i32]),
        "dk_layernorm": (None, [vp, vp, vp, vp, i64, i64, f32]),
        "dk_to_half_rows": (None, [vp, vp, i64, i64, i64]),
        "dk_transpose_to_half": (None, [vp, vp, i64, i64, i64, i64]),
        "dk_im2col_half": (None, [vp, vp, C.POINTER(DkConvGeom), i64, i64, i64, i64]),
        "dk_col2im_tr": (None, [vp, vp, vp, i64, i32, C.POINTER(DkConvGeom)]),
        "dk_gemm_half": (None, [i64, i64, i64, f32, vp, i64, i64, vp, i64, i64, f32, vp, i64,
                                i64, i64]),
        "dk_softmax_to_half": (None, [vp, i64, vp, i64, i64, i64, f32]),
        "dk_split_heads_half": (None, [vp, vp, i64, i64, i32, i32, i32, i64, i32]),
        "dk_stft": (None, [vp, vp, i64, i64, i32, i32, i32, i32, i32, vp]),
        "dk_istft_frames": (None, [vp, vp, i64, i32, i32, i32, i32, vp]),
        "dk_ola": (None, [vp, vp, i64, i32, i32, i32, vp, i64, i64]),
        "dkx_conv2d": (None, [vp, i32, C.POINTER(DkConvGeom), vp, i32, vp, i32, vp]),
        "dkx_conv_tr": (None, [vp, i32, i32, i32, i32, vp, i32, i32, i32, i32, vp, i32, i32,
                               i32, vp]),
        "dkx_linear": (None, [vp, i64, i32, vp, i64, i32, vp, vp]),
        "dkx_attention": (None, [vp, vp, vp, i32, i32, i32, i32, i32, vp]),
        "dcb_set_error_mode": (None, [i32]),
        "dcb_last_error": (C.c_char_p, [i32]),
        "dcb_set_stream": (None, [vp]),
        "dcb_use_own_stream": (None, []),
        "dcb_get_stream": (vp, []),
        "dcb_set_option": (i32, [C.c_char_p, i32]),
        "dcb_kernel_launches": (C.c_uint64, []),
        "dcb_device_fault": (C.c_uint32, [i32]),
        "dcb_trace_start": (None, [C.c_uint32]),
        "dcb_trace_stop": (i32, [C.POINTER(C.c_double), C.POINTER(C.c_double),
                                 C.POINTER(C.c_double), C.POINTER(i32), i32]),
        "dcb_trace_dump": (i32, [C.c_char_p]),
        "dcb_model_load": (vp, [C.c_char_p, C.c_char_p]),
        "dcb_model_load_layout": (vp, [C.c_char_p, C.c_char_p]),
        "dcb_model_save_packed": (i32, [vp, C.c_char_p]),
        "dcb_model_load_packed": (vp, [C.c_char_p]),
        "dcb_model_free": (None, [vp]),
        "dcb_model_info": (i32, [vp, C.POINTER(i32), C.POINTER(i32), C.POINTER(i32),
                                 C.POINTER(i32), C.POINTER(f32)]),
        "dcb_model_weight_bytes": (sz, [vp]),
        "dcb_model_weight_block": (vp, [vp]),
        "dcb_forward": (i32, [vp, vp, i32, i32, vp, STAGE_FN, vp]),
        "dcb_stage_encoder": (i32, [vp, i32, i32, vp, i32, i32, i32, i32, vp, C.POINTER(i32)]),
        "dcb_stage_decoder": (i32, [vp, i32, i32, vp, vp, i32, i32, i32, i32, i32, vp,
                                    C.POINTER(i32)]),
        "dcb_stage_transformer": (i32, [vp, vp, vp, i32, i32, i32, i32, i32]),
        "dcb_py_randint": (i32, [C.c_uint64, i32, i32, i32, C.POINTER(i32)]),
        "dcb_segment_plan": (i32, [i32, f32, i32, C.POINTER(DcbApplyOpts), C.POINTER(i32),
                                   C.POINTER(i32), i32]),
        "dcb_apply_defaults": (None, [C.POINTER(DcbApplyOpts)]),
        "dcb_apply": (i32, [vp, vp, i32, i32, vp, C.POINTER(DcbApplyOpts)]),
        "dcb_apply_plan": (i32, [vp, i32, C.POINTER(DcbApplyOpts), C.POINTER(i32),
                                 C.POINTER(i32)]),
        "dcb_apply_window": (i32, [i32, f32, i32, i32, C.POINTER(DcbApplyOpts),
                                   C.POINTER(i64), C.POINTER(i64)]),
        "dcb_apply_shard": (i32, [vp, vp, i32, i32, vp, i64, C.POINTER(DcbApplyOpts)]),
        "dcb_apply_host": (i32, [vp, vp, i32, i32, vp, C.POINTER(DcbApplyOpts)]),
        "dcb_merge_windows": (i32, [vp, i64, i64, vp, i64, i64, C.POINTER(i64),
                                    C.POINTER(i64), i32]),
    }


def check(ok=True, what="call"):
    """Raise BackendError if the library recorded an error (or ok is False)."""
    L = lib()
    msg = L.dcb_last_error(1).decode()
    if msg or not ok:
        raise BackendError(f"{what}: {msg or 'failed'}")


def use_torch_stream():
    """Run the backend on PyTorch's current stream so torch ops and kernels are ordered."""
    import torch
    lib().dcb_set_stream(C.c_void_p(torch.cuda.current_stream().cuda_stream))


def require_gpu():
    import torch
    if not torch.cuda.is_available():
        raise BackendError("no CUDA device: this backend runs only on sm_100 GPUs")
    major, _ = torch.cuda.get_device_capability()
    if major != 10:
        raise BackendError("this backend is built for sm_100a (B200) only")
    use_torch_stream()


def _ptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


class Model:
    """htdemucs_6s on the B200 engine (weights packed once on the device).

    Model(weights, config) reads and packs a safetensors file; with layout_only=True only
    its header is read and the device block is left zeroed for the caller to fill (the
    data-parallel ranks receive rank 0's block by broadcast); Model.from_packed(path) loads
    a pre-packed image written by save_packed()."""

    def __init__(self, weights: str, config: str = "", layout_only: bool = False,
                 packed: str = ""):
        require_gpu()
        L = lib()
        if packed:
            self._h = L.dcb_model_load_packed(packed.encode())
        elif layout_only:
            self._h = L.dcb_model_load_layout(weights.encode(), config.encode())
        else:
            self._h = L.dcb_model_load(weights.encode(), config.encode())
        if not self._h:
            check(False, "model load")
        ns, ac, vl, sr = C.c_int(), C.c_int(), C.c_int(), C.c_int()
        seg = C.c_float()
        L.dcb_model_info(self._h, C.byref(ns), C.byref(ac), C.byref(vl), C.byref(sr),
                         C.byref(seg))
        self.n_sources, self.audio_channels = ns.value, ac.value
        self.valid_length, self.samplerate, self.segment = vl.value, sr.value, seg.value

    @classmethod
    def from_packed(cls, path: str) -> "Model":
        return cls("", packed=path)

    def save_packed(self, path: str):
        """Write the pre-packed on-disk image (dcb_model_save_packed)."""
        r = lib().dcb_model_save_packed(self._h, path.encode())
        check(r == 0, "save_packed")

    def close(self):
        if getattr(self, "_h", None):
            lib().dcb_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def weight_bytes(self) -> int:
        return lib().dcb_model_weight_bytes(self._h)

    def weight_block(self):
        """(device pointer, bytes) of the packed weight block (the broadcast payload)."""
        return lib().dcb_model_weight_block(self._h), self.weight_bytes

    def forward(self, mix, stages: bool = False, out=None):
        """mix [B, C, T] float32 CUDA tensor -> stems [B, S, C, min(T, valid_length)]."""
        import torch
        use_torch_stream()
        mix = mix.contiguous()
        B, Cc, T = mix.shape
        keep = min(T, self.valid_length)
        if out is None:
            out = torch.empty((B, self.n_sources, Cc, keep), device=mix.device,
                              dtype=torch.float32)
        got = {}

        def cb(name, data, ndim, shape, user):
            shp = tuple(shape[i] for i in range(ndim))
            n = 1
            for s in shp:
                n *= s
            buf = torch.empty(n, device=mix.device, dtype=torch.float32)
            lib().dk_memcpy_d2d(C.c_void_p(buf.data_ptr()), C.c_void_p(data), n * 4)
            torch.cuda.current_stream().synchronize()
            got[name.decode()] = buf.reshape(shp)

        fn = STAGE_FN(cb) if stages else STAGE_FN(0)
        r = lib().dcb_forward(self._h, _ptr(mix), B, T, _ptr(out), fn, None)
        check(r >= 0, "forward")
        return (out, got) if stages else out

    def stage_encoder(self, branch: int, idx: int, x):
        import torch
        use_torch_stream()
        x = x.contiguous()
        shp = (C.c_int * 4)()
        B, Cc = x.shape[0], x.shape[1]
        H, W = (x.shape[2], x.shape[3]) if branch == 0 else (1, x.shape[2])
        r = lib().dcb_stage_encoder(self._h, branch, idx, _ptr(x), B, Cc, H, W, None, shp)
        check(r == 0, "stage_encoder")
        oshape = tuple(shp[i] for i in range(4 if branch == 0 else 3))
        y = torch.empty(oshape, device=x.device, dtype=torch.float32)
        r = lib().dcb_stage_encoder(self._h, branch, idx, _ptr(x), B, Cc, H, W, _ptr(y), shp)
        check(r == 0, "stage_encoder")
        return y

    def stage_decoder(self, branch: int, idx: int, x, skip, length: int = 0):
        import torch
        use_torch_stream()
        x, skip = x.contiguous(), skip.contiguous()
        shp = (C.c_int * 4)()
        B, Cc = x.shape[0], x.shape[1]
        H, W = (x.shape[2], x.shape[3]) if branch == 0 else (1, x.shape[2])
        r = lib().dcb_stage_decoder(self._h, branch, idx, _ptr(x), _ptr(skip), B, Cc, H, W,
                                    length, None, shp)
        check(r == 0, "stage_decoder")
        oshape = tuple(shp[i] for i in range(4 if branch == 0 else 3))
        y = torch.empty(oshape, device=x.device, dtype=torch.float32)
        r = lib().dcb_stage_decoder(self._h, branch, idx, _ptr(x), _ptr(skip), B, Cc, H, W,
                                    length, _ptr(y), shp)
        check(r == 0, "stage_decoder")
        return y

    def stage_transformer(self, x, xt):
        use_torch_stream()
        x, xt = x.contiguous().clone(), xt.contiguous().clone()
        B, Cc, Fr, T1 = x.shape
        r = lib().dcb_stage_transformer(self._h, _ptr(x), _ptr(xt), B, Cc, Fr, T1, xt.shape[2])
        check(r == 0, "stage_transformer")
        return x, xt

    def apply_opts(self, shifts=1, overlap=0.25, transition_power=1.0, batch_size=8, seed=1,
                   use_seed=False, shard_index=0, shard_count=1):
        o = DcbApplyOpts()
        lib().dcb_apply_defaults(C.byref(o))
        o.shifts, o.split, o.overlap = shifts, 1, overlap
        o.transition_power, o.batch_size = transition_power, batch_size
        o.seed, o.use_seed = seed, int(use_seed)
        o.shard_index, o.shard_count = shard_index, shard_count
        return o

    def apply(self, mix, out=None, **kw):
        """dc_apply_model on mix [B, C, T] (CUDA) -> [B, S, C, T].  With shard_count > 1 the
        result holds this shard's share; summing all shards gives the full output."""
        import torch
        use_torch_stream()
        mix = mix.contiguous()
        B, Cc, T = mix.shape
        if out is None:
            out = torch.empty((B, self.n_sources, Cc, T), device=mix.device,
                              dtype=torch.float32)
        o = self.apply_opts(**kw)
        r = lib().dcb_apply(self._h, _ptr(mix), B, T, _ptr(out), C.byref(o))
        check(r == 0, "apply")
        return out

    def apply_host(self, mix_h, out_h, **kw):
        """dc_apply_model on host (CPU) tensors mix_h [B, C, T] -> out_h [B, S, C, T], the
        copies overlapped with the compute (dcb_apply_host); pinned tensors overlap best."""
        use_torch_stream()
        assert not mix_h.is_cuda and not out_h.is_cuda
        assert mix_h.is_contiguous() and out_h.is_contiguous()
        B, Cc, T = mix_h.shape
        o = self.apply_opts(**kw)
        r = lib().dcb_apply_host(self._h, _ptr(mix_h), B, T, _ptr(out_h), C.byref(o))
        check(r == 0, "apply_host")
        return out_h

    def apply_window(self, T: int, **kw):
        """(lo, hi): the output window of this shard's share (dcb_apply_window)."""
        o = self.apply_opts(**kw)
        lo, hi = C.c_int64(), C.c_int64()
        r = lib().dcb_apply_window(self.samplerate, self.segment, self.valid_length, T,
                                   C.byref(o), C.byref(lo), C.byref(hi))
        check(r == 0, "apply_window")
        return lo.value, hi.value

    def apply_shard(self, mix, win, **kw):
        """This shard's share of apply() over its window only: win [B*S*C, ld] (CUDA),
        column j = time lo + j (dcb_apply_shard)."""
        use_torch_stream()
        mix = mix.contiguous()
        B, Cc, T = mix.shape
        o = self.apply_opts(**kw)
        r = lib().dcb_apply_shard(self._h, _ptr(mix), B, T, _ptr(win), win.stride(0),
                                  C.byref(o))
        check(r == 0, "apply_shard")
        return win

    def apply_plan(self, T: int, **kw):
        o = self.apply_opts(**kw)
        nf, nb = C.c_int(), C.c_int()
        lib().dcb_apply_plan(self._h, T, C.byref(o), C.byref(nf), C.byref(nb))
        return nf.value, nb.value


def gemm_half(A, B, C_=None, alpha=1.0, beta=0.0):
    """dk_gemm_half on torch fp16 tensors: A [b, M, K] (or [M, K] shared), B [b, N, K]
    -> C [b, M, N] fp32 (strides from the tensors)."""
    import torch
    use_torch_stream()
    if A.dim() == 2:
        A3, sa = A.unsqueeze(0), 0
    else:
        A3, sa = A, A.stride(0)
    if B.dim() == 2:
        B3, sb = B.unsqueeze(0), 0
    else:
        B3, sb = B, B.stride(0)
    batch = max(A3.shape[0], B3.shape[0])
    M, K = A3.shape[1], A3.shape[2]
    N = B3.shape[1]
    if C_ is None:
        C_ = torch.zeros((batch, M, N), device=A.device, dtype=torch.float32)
    lib().dk_gemm_half(M, N, K, alpha, _ptr(A3), A3.stride(1), sa, _ptr(B3), B3.stride(1), sb,
                       beta, _ptr(C_), C_.stride(1), C_.stride(0), batch)
    check(True, "dk_gemm_half")
    return C_


def merge_windows(out, wins, lo, hi):
    """out [rows, T] = overlap-add of the gathered shard windows wins [n, rows, ld] placed at
    lo[i] .. hi[i] (dcb_merge_windows)."""
    use_torch_stream()
    n = len(lo)
    los, his = (C.c_int64 * n)(*lo), (C.c_int64 * n)(*hi)
    o2 = out.reshape(-1, out.shape[-1])   # a view of the contiguous [.., T] output
    rows, T = o2.shape
    r = lib().dcb_merge_windows(_ptr(o2), rows, T, _ptr(wins), wins.stride(1),
                                wins.stride(0), los, his, n)
    check(r == 0, "merge_windows")
    return out


def apply_opts(shifts=1, overlap=0.25, transition_power=1.0, batch_size=8, seed=1,
               use_seed=False, shard_index=0, shard_count=1):
    o = DcbApplyOpts()
    lib(load_only=True).dcb_apply_defaults(C.byref(o))
    o.shifts, o.split, o.overlap = shifts, 1, overlap
    o.transition_power, o.batch_size = transition_power, batch_size
    o.seed, o.use_seed = seed, int(use_seed)
    o.shard_index, o.shard_count = shard_index, shard_count
    return o


def py_randint(seed: int, lo: int, hi: int, n: int):
    """CPython random.Random(seed).randint draws as the engine computes them (host only)."""
    out = (C.c_int * n)()
    lib(load_only=True).dcb_py_randint(seed, lo, hi, n, out)
    return list(out)


def segment_plan(length: int, samplerate=44100, segment=7.8, **kw):
    """(offsets, call index per offset on this shard or -1) of the engine's scheduler."""
    o = apply_opts(**kw)
    L = lib(load_only=True)
    n = L.dcb_segment_plan(samplerate, segment, length, C.byref(o), None, None, 0)
    offs, calls = (C.c_int * n)(), (C.c_int * n)()
    L.dcb_segment_plan(samplerate, segment, length, C.byref(o), offs, calls, n)
    return list(offs), list(calls)


def set_option(name: str, value: int) -> int:
    return lib().dcb_set_option(name.encode(), int(value))


def kernel_launches() -> int:
    return lib().dcb_kernel_launches()


TRACE_CLASSES = ["conv", "conv_tr", "linear", "attention", "gemm_half", "spectral", "dconv",
                 "norm"]
GLUE_CLASSES = ("spectral", "dconv", "norm")


def trace_start(classes=tuple(TRACE_CLASSES)):
    mask = 0
    for c in classes:
        mask |= 1 << TRACE_CLASSES.index(c)
    lib().dcb_trace_start(mask)


def trace_stop():
    """Per-class {ms, flops, bytes, launches} of the traced launches."""
    n = len(TRACE_CLASSES)
    ms, fl, by = (C.c_double * n)(), (C.c_double * n)(), (C.c_double * n)()
    ln = (C.c_int * n)()
    lib().dcb_trace_stop(ms, fl, by, ln, n)
    check(True, "trace")
    return {c: {"ms": ms[i], "flops": fl[i], "bytes": by[i], "launches": ln[i]}
            for i, c in enumerate(TRACE_CLASSES)}


def trace_dump(path: str) -> int:
    return lib().dcb_trace_dump(path.encode())


def device_fault(clear: bool = True) -> int:
    return lib().dcb_device_fault(int(clear))
