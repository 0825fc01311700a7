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
@pytest.mark.parametrize("bs", [1, 3, 8])
def test_segment_plan_matches_port(length, bs):
    """Same segment offsets as dc_apply_model; every segment in exactly one forward call,
    calls of at most batch_size segments, as few calls as possible, sizes within one of
    each other (tails are padded to the training length like full segments, so they batch
    with them; a segment's result does not depend on its batch)."""
    import demucs_cuda_b200 as d
    from oracle import port
    pc = port.Config({})
    seg, stride, offsets, batches = port.segment_plan(length, pc, 0.25, bs)
    offs, calls = d.segment_plan(length, overlap=0.25, batch_size=bs)
    assert offs == offsets
    groups = {}
    for i, c in enumerate(calls):
        groups.setdefault(c, []).append(i)
    assert sorted(i for g in groups.values() for i in g) == list(range(len(offs)))
    sizes = [len(g) for g in groups.values()]
    assert max(sizes) <= bs and max(sizes) - min(sizes) <= 1
    assert len(groups) == -(-len(offs) // bs)


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
    """The 240 s benchmark track: 42 segment forwards (40 full + 2 tails) per shift, in 6 forward
    calls of 7 segments at batch size 8."""
    import demucs_cuda_b200 as d
    offs, calls = d.segment_plan(10_584_000 + 22050 - 7000)  # shifted track length range
    assert len(offs) in (42, 43)
    offs, calls = d.segment_plan(10_584_000)
    assert len(offs) == 42 and max(calls) + 1 == 6
    assert all(calls.count(c) == 7 for c in range(6))
