"""Data-parallel host logic on CPU with world_size 2 (gloo), the same steps bench.py runs
over NCCL on GPUs: rank 0's weights reach the other rank only through a broadcast; the
engine's scheduler (dcb_segment_plan, dcb_apply_window) assigns each rank one contiguous
block of segments and an output window; each rank's share of dc_apply_model is zero outside
its window; the windows, padded to one width, are gathered to rank 0 and overlap-added
there, which reproduces the single-process result."""
import json
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import model_files, rel_l2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _window(length, pc, rank, world):
    import ctypes as C
    import demucs_cuda_b200 as d
    o = d.apply_opts(shifts=0, batch_size=2, shard_index=rank, shard_count=world)
    lo, hi = C.c_int64(), C.c_int64()
    r = d.lib(load_only=True).dcb_apply_window(pc.samplerate, pc.segment, pc.valid_length,
                                               length, C.byref(o), C.byref(lo), C.byref(hi))
    assert r == 0
    return lo.value, hi.value


def _worker(rank, world, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=300))
    try:
        from demucs_cuda_b200 import synth
        import demucs_cuda_b200 as d
        from oracle import port as P
        cfg, w, c = model_files("tiny")
        W = synth.load_safetensors(w)
        # rank 0's weights reach every rank through a broadcast (ranks > 0 start from zeros)
        names = sorted(W)
        flat = torch.from_numpy(np.concatenate([W[n].ravel() for n in names]))
        if rank != 0:
            flat.zero_()
        dist.broadcast(flat, src=0)
        off = 0
        for n in names:
            k = W[n].size
            W[n] = flat[off:off + k].numpy().reshape(W[n].shape)
            off += k
        pc = P.Config(json.load(open(c)))
        length = 70000
        rng = np.random.default_rng(5)
        mix = rng.uniform(-0.5, 0.5, (1, 2, length)).astype(np.float32)
        # the shard assignment and windows come from the engine's own scheduler
        offs, calls = d.segment_plan(length, pc.samplerate, pc.segment, shifts=0,
                                     batch_size=2, shard_index=rank, shard_count=world)
        mine = [i for i, cidx in enumerate(calls) if cidx >= 0]
        assert mine == list(range(mine[0], mine[-1] + 1))   # one contiguous block
        spans = [_window(length, pc, r, world) for r in range(world)]
        lo, hi = spans[rank]
        part = P.apply_model(mix, W, pc, shifts=0, batch_size=2, shard=(rank, world))
        outside = np.concatenate([part[..., :lo].ravel(), part[..., hi:].ravel()])
        assert not outside.any()   # the share is zero outside the window
        wmax = max(h - l for l, h in spans)
        win = np.zeros((part.shape[1] * part.shape[2], wmax), np.float32)
        win[:, :hi - lo] = part.reshape(-1, length)[:, lo:hi]
        t = torch.from_numpy(win)
        gl = [torch.empty_like(t) for _ in range(world)] if rank == 0 else None
        dist.gather(t, gather_list=gl, dst=0)
        if rank == 0:
            merged = np.zeros((win.shape[0], length), np.float32)
            for (l, h), g in zip(spans, gl):
                merged[:, l:h] += g.numpy()[:, :h - l]
            full = P.apply_model(mix, W, pc, shifts=0, batch_size=2)
            with open(out_path, "w") as f:
                json.dump({"rel": rel_l2(merged, full.reshape(-1, length)),
                           "n_mine": len(mine), "spans": spans}, f)
    finally:
        dist.destroy_process_group()


def test_two_rank_sharded_apply(tmp_path):
    out = str(tmp_path / "res.json")
    mp.spawn(_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    res = json.load(open(out))
    assert res["n_mine"] >= 1
    assert res["rel"] < 1e-6
    (l0, h0), (l1, h1) = res["spans"]
    assert l0 == 0 and h1 == 70000 and l1 < h0   # the windows overlap where segments do
