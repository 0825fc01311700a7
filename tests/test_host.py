"""Host-side scheduler logic of the engine (no GPU): shift RNG and segment plan."""
import random

import numpy as np
import pytest


@pytest.mark.parametrize("seed", [0, 1, 12345, 2 ** 32 + 5])
def test_shift_rng_is_cpython_randint(seed):
    import demucs_cuda_b200 as d
    r = random.Random(seed)
    want = [r.randint(0, 22050) for _ in range(50)]
    assert d.py_randint(seed, 0, 22050, 50) == want


@pytest.mark.parametrize("length", [10_584_000, 343_980, 400_000, 1000, 1_000_001])
def test_segment_plan_matches_port(length):
    import demucs_cuda_b200 as d
    from oracle import port
    pc = port.Config({})
    seg, stride, offsets, batches = port.segment_plan(length, pc, 0.25, 8)
    offs, calls = d.segment_plan(length, overlap=0.25, batch_size=8)
    assert offs == offsets
    # one shard: the same forward calls as dc_apply_model (full segments batched, tails alone)
    groups = {}
    for i, c in enumerate(calls):
        groups.setdefault(c, []).append(i)
    assert sorted(groups.values()) == sorted(idx for _, idx in batches)


@pytest.mark.parametrize("count", [2, 3, 4, 8])
def test_shards_cover_every_segment_once(count):
    import demucs_cuda_b200 as d
    length = 10_584_000
    seen = np.zeros(len(d.segment_plan(length)[0]), int)
    for s in range(count):
        _, calls = d.segment_plan(length, shard_index=s, shard_count=count)
        seen += np.array(calls) >= 0
    assert (seen == 1).all()


def test_240s_track_plan_counts():
    """42 segment forwards (40 full + 2 tails) per shift."""
    import demucs_cuda_b200 as d
    offs, calls = d.segment_plan(10_584_000 + 22050 - 7000)  # shifted track length range
    assert len(offs) in (42, 43)
    offs, calls = d.segment_plan(10_584_000)
    assert len(offs) == 42 and max(calls) + 1 == 7  # 5 batches of 8 + 2 tails
