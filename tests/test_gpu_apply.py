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
