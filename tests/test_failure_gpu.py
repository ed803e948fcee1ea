"""The bounded-wait failure path on the B200, exercised without a GPU fault.

Every spin-wait in this library's kernels is bounded by wall time; when one
runs out the kernel records TESSA_DEVERR_TIMEOUT, its other roles leave, and
the call returns TESSA_ERR_TIMEOUT with the context still usable (the
reference's watchdog likewise gives up with a status, CB:5883-5930).  The
probe waits on a barrier that nothing arrives on -- no copy or MMA is in
flight -- so running out its limit is safe; the leaf call after it must still
be bit-exact with the oracle.
"""
import ctypes

import numpy as np
import pytest

from leafcases import make_leaf_batch, oracle_leaf

pytestmark = pytest.mark.gpu


def _leaf(c, k, ctx):
    import torch
    from shear_b200 import ops
    dev = torch.device("cuda:0")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    ids, d = ops.leaf_topk_sq8(t(c["codes"]), t(c["scales"]), t(c["norms"]), t(c["gids"].view(np.int32)),
                               t(c["members"].view(np.int32)), c["starts"], c["sizes"], k, ctx=ctx)
    torch.cuda.synchronize()
    return ops.as_u32(ids), d.cpu().numpy()


def test_wait_that_runs_out_returns_timeout_and_context_stays_usable(oracle):
    from shear_b200 import _capi as C
    from shear_b200 import ops
    ctx = ops.context(0)
    lib = C.load()
    c = make_leaf_batch(oracle, [700, 300], 768, seed=19, dup=True, permute=True)
    want = oracle_leaf(oracle, c, 8)
    for limit_ns in (50_000_000, 200_000):
        elapsed = ctypes.c_uint64()
        rc = lib.tessa_check_bounded_wait(ctx.handle, limit_ns, ctypes.byref(elapsed), None)
        assert rc == -4, C.ERRORS.get(rc, rc)  # TESSA_ERR_TIMEOUT
        assert b"timed out" in lib.tessa_last_error_message()
        # the first waiter gave up at its limit; the second left through the
        # abort flag long before its own (20x + 2 s) limit
        assert limit_ns <= elapsed.value < limit_ns + 500_000_000
        got = _leaf(c, 8, ctx)
        assert np.array_equal(got[0], want[0])
        assert np.array_equal(got[1].view(np.uint32), want[1].view(np.uint32))


def test_wait_limit_setter_validates_and_applies(oracle):
    from shear_b200 import _capi as C
    from shear_b200 import ops
    ctx = ops.context(0)
    lib = C.load()
    assert lib.tessa_set_wait_timeout_ns(ctx.handle, 1_000) == -1          # below the 10 ms floor
    assert lib.tessa_set_wait_timeout_ns(ctx.handle, 10 ** 12) == -1       # above the 60 s ceiling
    c = make_leaf_batch(oracle, [300, 129], 256, seed=23, permute=True)
    want = oracle_leaf(oracle, c, 16)
    try:
        assert lib.tessa_set_wait_timeout_ns(ctx.handle, 20_000_000) == 0  # 20 ms: normal work fits easily
        got = _leaf(c, 16, ctx)
        assert np.array_equal(got[0], want[0])
        assert np.array_equal(got[1].view(np.uint32), want[1].view(np.uint32))
    finally:
        assert lib.tessa_set_wait_timeout_ns(ctx.handle, 0) == 0            # default restored
