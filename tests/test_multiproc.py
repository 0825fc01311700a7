"""Data-parallel host logic on CPU with world_size 2 (gloo): the weight broadcast from rank 0,
the engine's segment sharding (dcb_segment_plan) and the stem reduction reproduce the
single-process dc_apply_model result.  Same steps bench.py runs over NCCL on GPUs."""
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


def _worker(rank, world, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
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
        rng = np.random.default_rng(5)
        mix = rng.uniform(-0.5, 0.5, (1, 2, 70000)).astype(np.float32)
        # the shard assignment comes from the engine's own scheduler
        _, calls = d.segment_plan(70000, pc.samplerate, pc.segment, shifts=0, batch_size=2,
                                  shard_index=rank, shard_count=world)
        mine = [i for i, cidx in enumerate(calls) if cidx >= 0]
        assert all(i % world == rank for i in mine)
        part = P.apply_model(mix, W, pc, shifts=0, batch_size=2, shard=(rank, world))
        t = torch.from_numpy(part.copy())
        dist.reduce(t, dst=0)
        if rank == 0:
            full = P.apply_model(mix, W, pc, shifts=0, batch_size=2)
            with open(out_path, "w") as f:
                json.dump({"rel": rel_l2(t.numpy(), full), "n_mine": len(mine)}, f)
    finally:
        dist.destroy_process_group()


def test_two_rank_sharded_apply(tmp_path):
    out = str(tmp_path / "res.json")
    mp.spawn(_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    res = json.load(open(out))
    assert res["n_mine"] >= 1
    assert res["rel"] < 1e-6
