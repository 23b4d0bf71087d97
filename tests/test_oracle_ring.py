"""CPU: the host ring model reproduces the reference's recorded digests.

crates/lumen-mlx/src/native_cache/golden_tests.rs:465-497 records twelve
FNV-1a digests of NativeRotatingKvCacheTurboQuant driven through three plans
with step-prealloc on and off. The oracle's ring model must give the same
twelve numbers bit for bit; the GPU ring is then checked against the same
recording (tests/test_gpu_ring.py).
"""
import pytest


@pytest.mark.parametrize("qjl", [False, True], ids=["stage1", "qjl"])
def test_ring_model_matches_recorded_digests(orc, qjl):
    import ring_model as rm

    got = rm.digests(rm.ModelCase, qjl)
    rec = rm.RECORDED_TQ_QJL if qjl else rm.RECORDED_TQ
    assert {k: hex(v) for k, v in got.items()} == {k: hex(v) for k, v in rec.items()}


def test_ring_model_refusals(orc):
    import numpy as np
    import ring_model as rm

    r = rm.RingModel(1, 12, 2)
    one = np.zeros((1, 1, 1, 4), np.uint8)
    for _ in range(5):
        r.update([one], True)
    assert not r.truncate_to(6)          # target > offset
    assert r.truncate_to(5)              # no-op
    assert r.truncate_to(3) and r.offset == 3 and r.idx == 3
    for _ in range(20):
        r.update([one], True)
    assert r.offset > r.max_size
    assert not r.truncate_to(10)         # post-rotation rollback refused


def test_ring_geometry_checks(orc):
    import ring_model as rm

    with pytest.raises(rm.RingError):
        rm.RingModel(1, 0, 0)
    with pytest.raises(rm.RingError):
        rm.RingModel(1, 4, 4)
