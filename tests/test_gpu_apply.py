"""dc_apply_model on the GPU engine (dcb_apply) against the reference's own apply.c run on
the CPU (oracle/_ref, apply.c:179-306 over backend_cpu.c): shifts, overlap
with the transition-weighted overlap-add, full batches and tail segments, shards, and the
CUDA-graph replay of the segment forward (option "graphs")."""
import numpy as np
import pytest

from conftest import model_files, rel_l2

pytestmark = pytest.mark.gpu

STEMS_GATE = 1e-3  # SNR >= 60 dB, the end-to-end gate of the forward


@pytest.fixture(scope="module")
def tiny_apply(torch_cuda):
    import demucs_cuda_b200 as dcb
    from oracle import ref
    cfg, w, c = model_files("tiny")
    ref.load(w, c)
    rng = np.random.default_rng(3)
    mix = rng.uniform(-0.5, 0.5, (1, 2, 97000)).astype(np.float32)
    return {"torch": torch_cuda, "model": dcb.Model(w, c), "mix": mix, "ref": ref}


def _apply(env, **kw):
    torch = env["torch"]
    out = env["model"].apply(torch.from_numpy(env["mix"]).cuda(), **kw)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("shifts,batch", [(0, 2), (1, 2), (2, 3)])
def test_apply_vs_reference(tiny_apply, shifts, batch):
    import demucs_cuda_b200 as dcb
    dcb.set_option("graphs", 0)
    want = tiny_apply["ref"].apply_model(tiny_apply["mix"], shifts=shifts, overlap=0.25,
                                         batch_size=batch)
    got = _apply(tiny_apply, shifts=shifts, overlap=0.25, batch_size=batch)
    assert got.shape == want.shape
    assert rel_l2(got, want) < STEMS_GATE


def test_apply_graph_replay_matches_eager(tiny_apply):
    """The captured forward replays the same kernels on the same persistent buffers: three
    calls (eager warm-up, capture + replay, replay) give the eager result."""
    import demucs_cuda_b200 as dcb
    dcb.set_option("graphs", 0)
    eager = _apply(tiny_apply, shifts=1, batch_size=2)
    prev = dcb.set_option("graphs", 1)
    try:
        n0 = dcb.kernel_launches()
        outs = [_apply(tiny_apply, shifts=1, batch_size=2) for _ in range(3)]
        n1 = dcb.kernel_launches()
    finally:
        dcb.set_option("graphs", prev)
    for o in outs:
        assert rel_l2(o, eager) < 1e-6
    assert n1 > n0
    assert dcb.device_fault() == 0


def test_apply_shards_sum_to_full(tiny_apply):
    """Segment data parallelism: the shards' outputs add up to the unsharded result."""
    import demucs_cuda_b200 as dcb
    dcb.set_option("graphs", 1)
    full = _apply(tiny_apply, shifts=0, batch_size=2)
    parts = sum(_apply(tiny_apply, shifts=0, batch_size=2, shard_index=i, shard_count=3)
                for i in range(3))
    dcb.set_option("graphs", 0)
    assert rel_l2(parts, full) < 1e-6


def test_apply_short_track_single_segment(tiny_apply):
    """A track shorter than one segment: one tail forward, zero padded (apply.c:282-293)."""
    import demucs_cuda_b200 as dcb
    dcb.set_option("graphs", 0)
    mix = tiny_apply["mix"][:, :, :5000].copy()
    want = tiny_apply["ref"].apply_model(mix, shifts=0, batch_size=2)
    torch = tiny_apply["torch"]
    got = tiny_apply["model"].apply(torch.from_numpy(mix).cuda(), shifts=0,
                                    batch_size=2).cpu().numpy()
    assert rel_l2(got, want) < STEMS_GATE


def _block(model):
    """uint8 view of the model's packed device block."""
    import torch
    ptr, nbytes = model.weight_block()

    class _CAI:
        __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                    "data": (ptr, False), "version": 3}

    return torch.as_tensor(_CAI(), device="cuda")


@pytest.mark.parametrize("shifts,count", [(0, 3), (2, 4)])
def test_shard_windows_gather_merge(tiny_apply, shifts, count):
    """The data-parallel path bench.py runs at N GPUs, on one GPU: each shard's share over
    its window only (dcb_apply_shard), the windows padded to one width as a gather leaves
    them, and the root's overlap-add (dcb_merge_windows) give the unsharded result; each
    window matches the shard's full-length share (dcb_apply with shard_count)."""
    import demucs_cuda_b200 as dcb
    torch = tiny_apply["torch"]
    model = tiny_apply["model"]
    dcb.set_option("graphs", 1)
    mix = torch.from_numpy(tiny_apply["mix"]).cuda()
    T = mix.shape[-1]
    kw = dict(shifts=shifts, batch_size=2, shard_count=count)
    full = model.apply(mix, shifts=shifts, batch_size=2)
    spans = [model.apply_window(T, shard_index=r, **kw) for r in range(count)]
    assert spans[0][0] == 0 and spans[-1][1] == T
    assert all(spans[r][0] <= spans[r + 1][0] for r in range(count - 1))
    wmax = max(h - l for l, h in spans)
    rows = model.n_sources * 2
    wins = torch.full((count, rows, wmax), float("nan"), device="cuda")
    for r, (lo, hi) in enumerate(spans):
        wins[r, :, :hi - lo] = 0.0
        model.apply_shard(mix, wins[r], shard_index=r, **kw)
        share = model.apply(mix, shard_index=r, **kw).reshape(rows, T)
        assert torch.count_nonzero(share[:, :lo]) == 0 and torch.count_nonzero(share[:, hi:]) == 0
        assert rel_l2(wins[r, :, :hi - lo].cpu().numpy(), share[:, lo:hi].cpu().numpy()) < 1e-6
    out = torch.full((1, model.n_sources, 2, T), float("nan"), device="cuda")
    dcb.merge_windows(out, wins, [l for l, _ in spans], [h for _, h in spans])
    torch.cuda.synchronize()
    dcb.set_option("graphs", 0)
    assert rel_l2(out.cpu().numpy(), full.cpu().numpy()) < 1e-6
    assert dcb.device_fault() == 0


def test_layout_only_load_and_packed_image(tiny_apply, tmp_path):
    """A layout-only model (safetensors header only) has the same block size with zeros in
    it; once rank 0's block is copied in -- what the broadcast does -- it computes the same
    stems.  The pre-packed on-disk image reloads to the identical block and result."""
    import demucs_cuda_b200 as dcb
    torch = tiny_apply["torch"]
    cfg, w, c = model_files("tiny")
    ref_model = tiny_apply["model"]
    mix = torch.from_numpy(tiny_apply["mix"][:, :, :cfg.valid_length]).cuda()
    want = ref_model.forward(mix).cpu().numpy()
    lay = dcb.Model(w, c, layout_only=True)
    assert lay.weight_bytes == ref_model.weight_bytes
    assert torch.count_nonzero(_block(lay)) == 0
    _block(lay).copy_(_block(ref_model))
    torch.cuda.synchronize()
    # (the DConv statistics accumulate with atomics: equal to fp32 reassociation)
    assert rel_l2(lay.forward(mix).cpu().numpy(), want) < 1e-6
    path = str(tmp_path / "tiny.dcbpack")
    ref_model.save_packed(path)
    pk = dcb.Model.from_packed(path)
    assert torch.equal(_block(pk), _block(ref_model))
    assert rel_l2(pk.forward(mix).cpu().numpy(), want) < 1e-6
    # a damaged image is refused (checksum), not loaded
    raw = bytearray(open(path, "rb").read())
    raw[-100] ^= 0xFF
    bad = str(tmp_path / "bad.dcbpack")
    open(bad, "wb").write(bytes(raw))
    with pytest.raises(dcb.BackendError, match="checksum"):
        dcb.Model.from_packed(bad)
    del lay, pk


def test_apply_host_buffers_match_device_apply(tiny_apply):
    """dcb_apply_host (host input and output, copies overlapped with the batches on a second
    stream) gives dcb_apply's result, with page-locked and with ordinary host tensors, and
    leaves the rest of the output buffer's contents irrelevant (every sample is written)."""
    import demucs_cuda_b200 as dcb
    torch = tiny_apply["torch"]
    model = tiny_apply["model"]
    dcb.set_option("graphs", 1)
    mix = tiny_apply["mix"]
    want = model.apply(torch.from_numpy(mix).cuda(), shifts=1, batch_size=2).cpu().numpy()
    for pinned in (True, False):
        mh = torch.from_numpy(mix.copy())
        oh = torch.full((1, model.n_sources, 2, mix.shape[-1]), float("nan"))
        if pinned:
            mh, oh = mh.pin_memory(), oh.pin_memory()
        for _ in range(2):
            model.apply_host(mh, oh, shifts=1, batch_size=2)
            assert rel_l2(oh.numpy(), want) < 1e-6
    dcb.set_option("graphs", 0)
    assert dcb.device_fault() == 0
