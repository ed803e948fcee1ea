"""SQ8 leaf top-k on the B200 (tcgen05 kernel through the C ABI) vs the oracle.

Bit-exact: ids equal and distance bits equal for every output slot.
"""
import numpy as np
import pytest

from leafcases import make_leaf_batch, oracle_leaf

pytestmark = pytest.mark.gpu


def _device_run(c, k, leaf_ordered=False):
    import torch
    from shear_b200 import ops
    dev = torch.device("cuda:0")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    codes = t(c["codes"])
    lo = None
    if leaf_ordered:
        lo = t(c["codes"][c["members"].astype(np.int64)])
    ids, dists = ops.leaf_topk_sq8(codes, t(c["scales"]), t(c["norms"]), t(c["gids"].view(np.int32)),
                                   t(c["members"].view(np.int32)), c["starts"], c["sizes"], k,
                                   leaf_ordered_codes=lo)
    torch.cuda.synchronize()
    return ops.as_u32(ids), dists.cpu().numpy()


def _assert_same(got, want):
    gi, gd = got
    wi, wd = want
    bad = np.nonzero((gi != wi) | (gd.view(np.uint32) != wd.view(np.uint32)))[0]
    assert bad.size == 0, f"{bad.size} mismatching slots, first at {bad[:5]}: got {gi[bad[:5]]} " \
                          f"{gd[bad[:5]]} want {wi[bad[:5]]} {wd[bad[:5]]}"


CASES = [
    # (sizes, dim, k, dup, permute)
    ([2], 16, 1, False, False),
    ([3, 5], 16, 4, False, False),
    ([33], 128, 2, True, False),
    ([128], 128, 32, False, False),
    ([129], 768, 8, True, True),
    ([255, 256, 257], 768, 16, False, True),
    ([1, 300, 2], 100, 4, False, True),
    ([740, 728, 641], 1024, 2, False, False),
    ([2048], 768, 32, True, False),
    ([512, 513], 512, 7, False, True),
]


@pytest.mark.parametrize("sizes,dim,k,dup,permute", CASES)
def test_leaf_matches_oracle(oracle, sizes, dim, k, dup, permute):
    c = make_leaf_batch(oracle, sizes, dim, seed=sum(sizes) + dim + k, dup=dup, permute=permute)
    _assert_same(_device_run(c, k), oracle_leaf(oracle, c, k))


@pytest.mark.parametrize("dim,k", [(256, 2), (768, 2), (768, 32), (1024, 2), (512, 9)])
def test_leaf_many_tiles_per_cta_match_oracle(oracle, dim, k):
    # More than three times as many 128-row tiles as SMs, of ragged leaves: every
    # persistent CTA runs several tiles back to back, so each tile's A tile is
    # copied into tensor memory over the previous tile's once that tile's MMAs
    # have completed (ring deeper than the A slabs at k = 2, shallower at k = 32).
    rng = np.random.default_rng(dim * 7 + k)
    sizes = [int(s) for s in rng.integers(100, 400, size=300)]
    rows_per_leaf = np.array(sizes)
    assert int(((rows_per_leaf + 127) // 128).sum()) > 3 * 148
    c = make_leaf_batch(oracle, sizes, dim, seed=dim + k, dup=True, permute=True)
    _assert_same(_device_run(c, k), oracle_leaf(oracle, c, k))


def test_leaf_ordered_codes_path_matches_gather_path(oracle):
    c = make_leaf_batch(oracle, [300, 200], 256, seed=11, permute=True)
    a = _device_run(c, 8)
    b = _device_run(c, 8, leaf_ordered=True)
    _assert_same(a, b)
    _assert_same(a, oracle_leaf(oracle, c, 8))


def test_leaf_host_api_matches_oracle(oracle):
    from shear_b200 import ops
    c = make_leaf_batch(oracle, [700, 300], 768, seed=5, dup=True, permute=True)
    got = ops.leaf_topk_sq8_host(c["codes"], c["scales"], c["norms"], c["gids"], c["members"], c["starts"],
                                 c["sizes"], 32)
    _assert_same(got, oracle_leaf(oracle, c, 32))


def _host_run(c, k, batch_bytes=None):
    from shear_b200 import ops
    try:
        return ops.leaf_topk_sq8_host(c["codes"], c["scales"], c["norms"], c["gids"], c["members"], c["starts"],
                                      c["sizes"], k, batch_bytes=batch_bytes)
    finally:
        ops.set_host_batch_bytes(0)


@pytest.mark.parametrize("k", [2, 9, 32])
def test_leaf_host_pipeline_batches_match_oracle(oracle, k):
    # identity members + ordered leaves take the batched upload/kernel/download
    # pipeline; ~256 rows of codes per batch gives many batches of whole leaves
    c = make_leaf_batch(oracle, [300, 129, 512, 77, 1000, 2, 640, 128], 768, seed=31 + k, dup=True)
    want = oracle_leaf(oracle, c, k)
    _assert_same(_host_run(c, k, batch_bytes=256 * 768), want)
    _assert_same(_host_run(c, k, batch_bytes=1), want)
    _assert_same(_host_run(c, k), want)


def test_leaf_host_pipeline_with_gaps_between_leaves(oracle):
    # rows outside every leaf are not compared (no leaf writes them)
    c = make_leaf_batch(oracle, [850], 256, seed=8)
    c["starts"] = np.array([5, 300, 700], np.uint64)
    c["sizes"] = np.array([200, 390, 100], np.uint64)
    k = 6
    wi, wd = oracle_leaf(oracle, c, k)
    gi, gd = _host_run(c, k, batch_bytes=150 * 256)
    rows = np.concatenate([np.arange(int(s), int(s + n)) for s, n in zip(c["starts"], c["sizes"])])
    slots = (rows[:, None] * k + np.arange(k)[None, :]).ravel()
    _assert_same((gi[slots], gd[slots]), (wi[slots], wd[slots]))


def test_leaf_host_unordered_leaves_take_serial_path(oracle):
    c = make_leaf_batch(oracle, [200, 300, 100], 128, seed=4)
    c["starts"] = np.array([500, 0, 200], np.uint64)
    c["sizes"] = np.array([100, 200, 300], np.uint64)
    _assert_same(_host_run(c, 5, batch_bytes=64 * 128), oracle_leaf(oracle, c, 5))


def test_leaf_host_pipeline_sums_fallback_rows(oracle):
    from shear_b200 import ops
    rng = np.random.default_rng(78)
    def formula(rows, dim):
        base = rng.standard_normal(dim).astype(np.float32)
        x = base[None, :] + rng.standard_normal((rows, dim)).astype(np.float32) * np.float32(2e-3)
        return x / np.linalg.norm(x, axis=1, keepdims=True)
    c = make_leaf_batch(oracle, [700, 300, 500], 128, seed=3, formula=formula)
    _device_run(c, 8)
    want_fb = ops.leaf_last_fallback_rows()
    assert want_fb > 0
    got = _host_run(c, 8, batch_bytes=128 * 300)
    assert ops.leaf_last_fallback_rows() == want_fb
    _assert_same(got, oracle_leaf(oracle, c, 8))


def test_leaf_duplicate_local_ids_are_all_skipped(oracle):
    # CB:9569-9650 skips every column whose local id equals the row's
    c = make_leaf_batch(oracle, [40], 64, seed=9)
    c["members"] = np.array(list(range(20)) + list(range(20)), np.uint32)
    _assert_same(_device_run(c, 4), oracle_leaf(oracle, c, 4))


def test_reference_replay_fixture_607x1024_duplicate_rows(oracle):
    # P/tessa_replay.rs:1794-1894 input: row 7 duplicates row 6, k = 2
    def formula(rows, dim):
        r = np.arange(rows)[:, None]
        a = np.arange(dim)[None, :]
        src = np.where(r == 7, 6, r)
        return (((src * 17 + a * 13) % 97).astype(np.float32) * np.float32(0.03125) - np.float32(1.0))
    c = make_leaf_batch(oracle, [607], 1024, seed=0, formula=formula)
    c["gids"] = np.arange(607, dtype=np.uint32)
    _assert_same(_device_run(c, 2), oracle_leaf(oracle, c, 2))


def test_reference_staged_fixture_740_728_641(oracle):
    # P/tessa_replay.rs:1898-1999 input (staged multi-leaf offsets), k = 2
    def formula(rows, dim):
        r = np.arange(rows)[:, None]
        a = np.arange(dim)[None, :]
        return (((r * 131 + a * 17 + r * a * 3) % 251).astype(np.float32) * np.float32(0.0078125)
                - np.float32(0.75))
    c = make_leaf_batch(oracle, [740, 728, 641], 1024, seed=0, formula=formula)
    c["gids"] = np.arange(740 + 728 + 641, dtype=np.uint32)
    want = oracle_leaf(oracle, c, 2)
    _assert_same(_device_run(c, 2), want)
    # The staged merge order of the reference gives the same lists here.
    staged = oracle.leaf_topk_sq8(c["codes"], c["scales"], c["norms"], c["gids"], c["members"], c["starts"],
                                  c["sizes"], 2, 128)
    _assert_same(want, staged)


def test_leaf_tie_chains_go_through_exact_fallback(oracle):
    # Nearly identical rows: SQ8 distances cluster within the 2e-5 tie window,
    # so many rows have non-transitive tie chains and need the sequential rule.
    from shear_b200 import ops
    rng = np.random.default_rng(77)
    def formula(rows, dim):
        base = rng.standard_normal(dim).astype(np.float32)
        x = base[None, :] + rng.standard_normal((rows, dim)).astype(np.float32) * np.float32(2e-3)
        return x / np.linalg.norm(x, axis=1, keepdims=True)
    for k in (4, 32):
        c = make_leaf_batch(oracle, [700, 300], 128, seed=k, formula=formula)
        got = _device_run(c, k)
        _assert_same(got, oracle_leaf(oracle, c, k))
        assert ops.leaf_last_fallback_rows() > 0


@pytest.mark.parametrize("k", [3, 5, 12, 17, 24, 31])
def test_leaf_k_between_register_widths(oracle, k):
    # k below its register width (the merge of the two column halves then
    # inserts the other half's values one pair at a time instead of the
    # bitonic merge used when k fills the width); ragged leaves and repeated
    # members
    c = make_leaf_batch(oracle, [700, 129, 300, 64, 40], 256, seed=100 + k, dup=True, permute=True)
    _assert_same(_device_run(c, k), oracle_leaf(oracle, c, k))


def test_leaf_config2_shape_sample(oracle):
    # 16 leaves of the 4096 x 2048 x 768 k=32 benchmark workload
    from shear_b200 import ops
    c = make_leaf_batch(oracle, [2048] * 16, 768, seed=2026)
    _assert_same(_device_run(c, 32), oracle_leaf(oracle, c, 32))
    # On random rows the exact fallback is the exception (about 1 row in
    # 2000): a regression that sends many rows there stays correct but slow.
    assert ops.leaf_last_fallback_rows() < 16 * 2048 // 200


def test_leaf_large_single_leaf(oracle):
    # one leaf four times the reference's largest staged leaf (2048 rows)
    c = make_leaf_batch(oracle, [8192], 128, seed=8192, dup=True)
    _assert_same(_device_run(c, 32), oracle_leaf(oracle, c, 32))


def test_leaf_empty_batch_is_a_no_op():
    import torch
    from shear_b200 import ops
    dev = torch.device("cuda:0")
    codes = torch.zeros((4, 16), dtype=torch.int8, device=dev)
    f = torch.zeros(4, device=dev)
    g = torch.zeros(4, dtype=torch.int32, device=dev)
    ids, dists = ops.leaf_topk_sq8(codes, f, f, g, g[:0], np.zeros(0, np.uint64), np.zeros(0, np.uint64), 4)
    torch.cuda.synchronize()
    assert ids.numel() == 0 and dists.numel() == 0


def test_leaf_rejects_bad_arguments(oracle):
    from shear_b200 import ops, TessaError
    c = make_leaf_batch(oracle, [10], 32, seed=1)
    for k in (0, 33):
        with pytest.raises(TessaError, match="INVALID_ARG"):
            _device_run(c, k)
    bad = dict(c)
    bad["members"] = c["members"].copy()
    bad["members"][3] = 10**6
    with pytest.raises(TessaError, match="BAD_ROW"):
        ops.leaf_topk_sq8_host(bad["codes"], bad["scales"], bad["norms"], bad["gids"], bad["members"],
                               bad["starts"], bad["sizes"], 2)
    big = make_leaf_batch(oracle, [4], 2048, seed=1)
    with pytest.raises(TessaError, match="UNSUPPORTED"):
        _device_run(big, 2)


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("sizes,dim,k,seed", [
    ([300, 129, 1000, 257], 768, 2, 1),      # odd tile counts: the last pair's second CTA holds no rows
    ([2048, 700, 100, 1500], 768, 32, 2),
    ([513, 255, 1], 128, 8, 3),
    ([900, 900, 900], 1024, 16, 4),
])
def test_leaf_pair_and_single_cta_kernels_match_oracle(oracle, mode, sizes, dim, k, seed):
    # mode 0: the column-split kernel on CTA pairs (tcgen05 cta_group::2, each
    # CTA loading half of every B chunk); mode 1: one CTA per 128-row tile.
    from shear_b200 import ops
    c = make_leaf_batch(oracle, sizes, dim, seed=seed, dup=True, permute=True)
    want = oracle_leaf(oracle, c, k)
    ops.set_leaf_kernel(mode)
    try:
        _assert_same(_device_run(c, k), want)
        _assert_same(_device_run(c, k, leaf_ordered=True), want)
    finally:
        ops.set_leaf_kernel(1)
