"""Device membership digests (the order-free part of every capture task hash,
P/tessa_capture.rs:274-293) and capture sampling from a device leaf batch."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_membership_digests_match_restatement():
    import torch
    from shear_b200 import capture as cap, ops
    rng = np.random.default_rng(1)
    sizes = np.array([0, 1, 5, 257, 1000, 4097, 300], np.uint64)
    starts = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.uint64)
    rows = int(sizes.sum())
    members = rng.permutation(rows).astype(np.uint32)
    gids = rng.choice(2**32 - 1, rows, replace=False).astype(np.uint32)
    dev = torch.device("cuda:0")
    t = lambda a: torch.from_numpy(a.view(np.int32)).to(dev)
    got = ops.membership_digests(t(members), starts, sizes, global_ids=t(gids))
    for l, (s, n) in enumerate(zip(starts, sizes)):
        want = cap.membership_digest(gids[members[int(s):int(s + n)]])
        assert tuple(int(v) for v in got[l]) == want
    direct = ops.membership_digests(t(members), starts, sizes)
    for l, (s, n) in enumerate(zip(starts, sizes)):
        assert tuple(int(v) for v in direct[l]) == cap.membership_digest(members[int(s):int(s + n)])


def test_capture_leaf_batch_equals_host_sampling():
    import torch
    from shear_b200 import capture as cap
    rng = np.random.default_rng(2)
    sizes = rng.integers(150, 1400, 400).astype(np.uint64)
    starts = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.uint64)
    rows = int(sizes.sum())
    members = rng.permutation(rows).astype(np.uint32)
    gids = rng.choice(5_000_000, rows, replace=False).astype(np.uint32)
    dev = torch.device("cuda:0")
    t = lambda a: torch.from_numpy(a.view(np.int32)).to(dev)
    a = cap.TessaCaptureSampler(9)
    cap.capture_leaf_batch(a, t(members), starts, sizes, 8, 768, global_ids=t(gids))
    b = cap.TessaCaptureSampler(9)
    for s, n in zip(starts, sizes):
        b.observe_leaf(cap.TessaLeafTask(0, 0, 8, 768, list(gids[members[int(s):int(s + n)]])))
    fa, fb = a.finish(), b.finish()
    assert fa.leaf_tasks == fb.leaf_tasks and fa.bin_counts == fb.bin_counts
    assert len(fa.leaf_tasks) == sum(fa.bin_counts["leaf_selected"]) > 0
