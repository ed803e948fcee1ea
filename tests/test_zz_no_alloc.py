"""The allocation-free leaf entry point (tessa_leaf_topk_sq8_noalloc).

It serves callers that must not allocate device memory -- hosts whose
allocator already owns the device, latency-critical threads that cannot afford
cudaMalloc's possible device synchronisation, embedders with a fixed footprint
-- by keeping its scratch in a static 64 MiB device array.  These tests call it
through the C ABI and check it against the allocating entry point
(tessa_leaf_topk_sq8) and against the CPU oracle, bit for bit, on batches in a
row (a call must not see the previous call's leftovers), with and without the
caller's leaf-ordered codes and with rows that take the exact fallback.  The
file is named so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest

from leafcases import make_leaf_batch, oracle_leaf

pytestmark = pytest.mark.gpu


def _tensors(c):
    import torch
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return dict(codes=t(c["codes"]), scales=t(c["scales"]), norms=t(c["norms"]),
                gids=t(c["gids"].view(np.int32)), members=t(c["members"].view(np.int32)),
                ordered=t(c["codes"][c["members"].astype(np.int64)]))


def _noalloc(c, d, k, leaf_ordered=False):
    import torch
    from shear_b200 import _capi
    rows = int(c["members"].shape[0])
    ids = torch.full((rows * k,), -7, dtype=torch.int32, device="cuda")
    dists = torch.full((rows * k,), -7.0, dtype=torch.float32, device="cuda")
    starts = np.ascontiguousarray(c["starts"], np.uint64)
    sizes = np.ascontiguousarray(c["sizes"], np.uint64)
    a = _capi.LeafArgs(codes=d["codes"].data_ptr(), scales=d["scales"].data_ptr(), norms=d["norms"].data_ptr(),
                       global_ids=d["gids"].data_ptr(), resident_rows=c["codes"].shape[0],
                       padded_dim=c["codes"].shape[1], k=k, leaf_members=d["members"].data_ptr(),
                       leaf_starts=starts.ctypes.data, leaf_sizes=sizes.ctypes.data, leaf_count=starts.shape[0],
                       leaf_rows=rows, topk_ids=ids.data_ptr(), topk_dists=dists.data_ptr(),
                       leaf_ordered_codes=d["ordered"].data_ptr() if leaf_ordered else None)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _capi.check(_capi.load().tessa_leaf_topk_sq8_noalloc(ctypes.byref(a), stream))
    return ids.cpu().numpy().view(np.uint32), dists.cpu().numpy()


def _allocating(c, d, k):
    import torch
    from shear_b200 import ops
    ids, dists = ops.leaf_topk_sq8(d["codes"], d["scales"], d["norms"], d["gids"], d["members"], c["starts"],
                                   c["sizes"], k)
    torch.cuda.synchronize()
    return ops.as_u32(ids), dists.cpu().numpy()


def test_noalloc_matches_allocating_entry_point_on_two_calls(oracle):
    # Permuted members force the gather of leaf-ordered codes into the static
    # scratch; the batches differ in shape, data and k.  The allocation-free
    # call runs the four-warp leaf kernel, the allocating call the
    # column-split kernel and its finishing kernel: the two must agree bit
    # for bit.
    for sizes, dim, k, seed in (([300, 257, 129], 768, 32, 41), ([640, 100], 256, 4, 42),
                                ([2048, 700], 768, 32, 43), ([500, 129], 1024, 16, 44)):
        c = make_leaf_batch(oracle, sizes, dim, seed=seed, dup=True, permute=True)
        d = _tensors(c)
        want_ids, want_d = _allocating(c, d, k)
        got_ids, got_d = _noalloc(c, d, k)
        assert np.array_equal(got_ids, want_ids)
        assert np.array_equal(got_d.view(np.uint32), want_d.view(np.uint32))
        wi, wd = oracle_leaf(oracle, c, k)
        assert np.array_equal(got_ids, wi)
        assert np.array_equal(got_d.view(np.uint32), wd.view(np.uint32))


def test_noalloc_leaf_ordered_codes_and_exact_fallback_rows(oracle):
    # Nearly identical rows put many rows on eps-tie chains, which the kernel
    # hands to the exact sequential fallback through the static scratch; with
    # the caller's leaf-ordered codes no gather region is reserved.
    rng = np.random.default_rng(77)

    def formula(rows, dim):
        base = rng.standard_normal(dim).astype(np.float32)
        x = base[None, :] + rng.standard_normal((rows, dim)).astype(np.float32) * np.float32(2e-3)
        return x / np.linalg.norm(x, axis=1, keepdims=True)
    for k, ordered in ((4, False), (32, True), (8, True)):
        c = make_leaf_batch(oracle, [700, 300], 128, seed=k, formula=formula, permute=True)
        d = _tensors(c)
        got_ids, got_d = _noalloc(c, d, k, leaf_ordered=ordered)
        want_ids, want_d = _allocating(c, d, k)
        wi, wd = oracle_leaf(oracle, c, k)
        assert np.array_equal(got_ids, want_ids) and np.array_equal(got_ids, wi)
        assert np.array_equal(got_d.view(np.uint32), want_d.view(np.uint32))
        assert np.array_equal(got_d.view(np.uint32), wd.view(np.uint32))


def test_noalloc_rejects_batches_beyond_the_static_scratch(oracle):
    from shear_b200 import _capi
    c = make_leaf_batch(oracle, [64], 768, seed=3, permute=True)
    d = _tensors(c)
    # Claim two leaves of 50,000 member rows: the gather alone would need
    # 76.8 MB > 64 MiB.  The size check runs before any device access.
    c_big = dict(c)
    c_big["starts"] = np.array([0, 50000], np.uint64)
    c_big["sizes"] = np.array([50000, 50000], np.uint64)
    c_big["members"] = np.zeros(100000, np.uint32)
    with pytest.raises(_capi.TessaError, match="UNSUPPORTED.*static"):
        _noalloc(c_big, d, 4)
