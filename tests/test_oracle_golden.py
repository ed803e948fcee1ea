"""Pins the CPU checker (oracle/) to the reference's own golden values.

Each test restates a reference unit test (file:line in the reference project)
with the same inputs and expected values, or checks the C restatement against
an independent pure-Python transliteration on small cases.
"""
import numpy as np
import pytest

EPS = np.float32(2e-5)


def test_sq8_quantizes_per_vector_with_padding_and_zero_scale(oracle):
    # shear-core/src/algorithm/pipnn/dco_sq_int8.rs:3261-3282
    codes, scales, norms = oracle.quantize_sq8(np.array([[0, 0, 0], [1, -1, 0.5]], np.float32), k_align=8)
    assert codes.shape == (2, 8)
    assert scales[0] == np.float32(1.0)
    assert norms[0] == np.float32(0.0)
    assert codes[0].tolist() == [0] * 8
    assert scales[1] == np.float32(1.0) / np.float32(127.0)
    assert norms[1] == np.float32(2.25)
    assert codes[1].tolist() == [127, -127, 64, 0, 0, 0, 0, 0]


def test_sq8_quantization_bits_control_effective_code_range(oracle):
    # dco_sq_int8.rs:3285-3298
    codes8, s8, _ = oracle.quantize_sq8(np.array([[1.0, -1.0, 0.5]], np.float32), k_align=8, bits=8)
    assert s8[0] == np.float32(1.0) / np.float32(127.0)
    assert codes8[0].tolist() == [127, -127, 64, 0, 0, 0, 0, 0]
    codes4, s4, _ = oracle.quantize_sq8(np.array([[1.0, -1.0, 0.5]], np.float32), k_align=8, bits=4)
    assert s4[0] == np.float32(1.0) / np.float32(7.0)
    assert codes4[0][0] == 7 and codes4[0][1] == -7
    assert all(-7 <= c <= 7 for c in codes4[0])


def test_sq8_dot_and_approx_l2_use_exact_norms_and_scales(oracle):
    # dco_sq_int8.rs:3301-3323
    codes, scales, norms = oracle.quantize_sq8(np.array([[1.0, 0.5], [0.5, 1.0]], np.float32), k_align=4)
    dot = oracle.sq8_dot(codes[0], codes[1])
    assert dot == 127 * 64 + 64 * 127
    approx = oracle.sq8_l2_from_dot(dot, scales[0], norms[0], scales[1], norms[1])
    expected_dot = np.float32(dot) * scales[0] * scales[1]
    expected = norms[0] + norms[1] - np.float32(2.0) * expected_dot
    assert abs(float(approx) - float(expected)) < 1e-6


def test_padded_dim_rounds_up_to_k_align(oracle):
    # dco_sq_int8.rs:1216-1224
    assert oracle.padded_dim(768) == 768
    assert oracle.padded_dim(100) == 112
    assert oracle.padded_dim(3, 8) == 8
    assert oracle.padded_dim(1, 1) == 1


def test_quantizer_round_half_away_and_sequential_norm(oracle):
    # Rust f32::round is half-away-from-zero; norm is a left-to-right f32 sum.
    x = np.array([[2.5, -2.5, 127.0, 0.1, -0.3]], np.float32)
    codes, scales, norms = oracle.quantize_sq8(x)
    scale = np.float32(127.0) / np.float32(127.0)
    want = [int(np.sign(v) * np.floor(abs(np.float32(v) / scale) + 0.5)) for v in x[0]]
    assert codes[0][:5].tolist() == want
    s = np.float32(0)
    for v in x[0]:
        s = np.float32(s + np.float32(v * v))
    assert norms[0] == s


def test_quantizer_rejects_non_finite(oracle):
    with pytest.raises(ValueError):
        oracle.quantize_sq8(np.array([[1.0, np.inf]], np.float32))


def _better(d, i, od, oi):
    delta = np.float32(np.float32(d) - np.float32(od))
    return (i < oi) if abs(delta) <= EPS else (d < od)


def _py_leaf(codes, scales, norms, gids, members, k):
    """Transliteration of CB:9569-9650 + CB:7229-7259 for one leaf."""
    n = len(members)
    ids = np.full((n, k), 0xFFFFFFFF, np.uint32)
    dists = np.full((n, k), np.float32(3.402823466e38), np.float32)
    for r in range(n):
        li = members[r]
        bd = [np.float32(3.402823466e38)] * k
        bi = [0xFFFFFFFF] * k
        for c in range(n):
            lj = members[c]
            if lj == li:
                continue
            dot = int(np.dot(codes[li].astype(np.int64), codes[lj].astype(np.int64)))
            ss = np.float32(scales[li] * scales[lj])
            sd = np.float32(ss * np.float32(dot))
            d = np.float32(np.float32(norms[li] + norms[lj]) + np.float32(np.float32(-2.0) * sd))
            if d <= 0:
                d = np.float32(0)
            g = int(gids[lj])
            if not _better(d, g, bd[k - 1], bi[k - 1]):
                continue
            pos = k - 1
            while pos > 0 and _better(d, g, bd[pos - 1], bi[pos - 1]):
                bd[pos] = bd[pos - 1]
                bi[pos] = bi[pos - 1]
                pos -= 1
            bd[pos] = d
            bi[pos] = g
        ids[r] = bi
        dists[r] = bd
    return ids, dists


@pytest.mark.parametrize("n,k,dup", [(9, 2, False), (20, 4, True), (33, 8, True), (5, 4, False)])
def test_oracle_leaf_matches_transliteration(oracle, n, k, dup):
    rng = np.random.default_rng(n * 100 + k)
    x = rng.standard_normal((n, 24)).astype(np.float32)
    if dup:  # CB:41953-42137 forces ties with duplicate rows (2==1, 5==4)
        x[2] = x[1]
        x[min(5, n - 1)] = x[4]
    codes, scales, norms = oracle.quantize_sq8(x)
    gids = rng.permutation(1000)[:n].astype(np.uint32)
    members = rng.permutation(n).astype(np.uint32)
    ids, dists = oracle.leaf_topk_sq8(codes, scales, norms, gids, members, [0], [n], k)
    want_ids, want_d = _py_leaf(codes, scales, norms, gids, members, k)
    assert np.array_equal(ids.reshape(n, k), want_ids)
    assert np.array_equal(dists.reshape(n, k).view(np.uint32), want_d.view(np.uint32))


def test_oracle_staged_equals_sequential_without_tie_chains(oracle):
    # For generic data the reference's staged 128-column merge (CB:35199-35203,
    # CB:7261-7309) and the sequential order agree.
    rng = np.random.default_rng(3)
    n, k = 600, 4
    x = rng.standard_normal((n, 64)).astype(np.float32)
    codes, scales, norms = oracle.quantize_sq8(x)
    gids = np.arange(n, dtype=np.uint32)
    m = np.arange(n, dtype=np.uint32)
    a = oracle.leaf_topk_sq8(codes, scales, norms, gids, m, [0], [n], k, 0)
    b = oracle.leaf_topk_sq8(codes, scales, norms, gids, m, [0], [n], k, 128)
    assert np.array_equal(a[0], b[0])
    assert np.array_equal(a[1].view(np.uint32), b[1].view(np.uint32))


def test_oracle_leaf_short_leaf_keeps_empty_slots(oracle):
    x = np.eye(3, 16, dtype=np.float32)
    codes, scales, norms = oracle.quantize_sq8(x)
    ids, dists = oracle.leaf_topk_sq8(codes, scales, norms, np.arange(3, dtype=np.uint32),
                                      np.arange(3, dtype=np.uint32), [0], [3], 4)
    ids = ids.reshape(3, 4)
    assert (ids[:, 2:] == 0xFFFFFFFF).all()
    assert (dists.reshape(3, 4)[:, 2:] == np.float32(3.402823466e38)).all()


def _splitmix(v):
    m = (1 << 64) - 1
    v ^= v >> 30
    v = (v * 0xBF58476D1CE4E5B9) & m
    v ^= v >> 27
    v = (v * 0x94D049BB133111EB) & m
    return v ^ (v >> 31)


def test_assignment_tie_key_is_splitmix64_of_point_and_leader(oracle):
    # CB:5983-5989, CB:6510-6520
    for p, l in [(0, 0), (7, 3), (123456, 77), (2**32 - 1, 2**32 - 1)]:
        want = _splitmix(((p << 32) ^ l ^ 0x9E3779B97F4A7C15) & ((1 << 64) - 1))
        assert oracle.tie_key(p, l) == want
    assert oracle.hash64(0) == 0


def _py_assign(x, norms, leaders_local, point, fp32=True, codes=None, scales=None, fused=True):
    best = [(np.float32(3.402823466e38), 0xFFFFFFFF, 0xFFFFFFFF)] * 4
    key = lambda l: _splitmix(((int(point) << 32) ^ int(l) ^ 0x9E3779B97F4A7C15) & ((1 << 64) - 1))
    for slot, l in enumerate(int(v) for v in leaders_local):
        if fp32:
            dot = np.float32(0)
            for a in range(x.shape[1]):
                dot = np.float32(dot + np.float32(x[point, a] * x[l, a]))
            d = np.float32(np.float32(norms[point] + norms[l]) + np.float32(-2.0) * dot)
        else:
            idot = int(np.dot(codes[point].astype(np.int64), codes[l].astype(np.int64)))
            t = np.float32(np.float32(2.0 * scales[point]) * scales[l])
            d = np.float32(np.float32(norms[point] + norms[l]) - np.float32(t * np.float32(idot)))
        d = max(d, np.float32(0))

        def bt(d, l, od, ol):
            if abs(np.float32(d - od)) <= EPS:
                return key(l) < key(ol) or (key(l) == key(ol) and l < ol)
            return d < od
        if not bt(d, l, best[3][0], best[3][2]):
            continue
        pos = 3
        while pos > 0 and bt(d, l, best[pos - 1][0], best[pos - 1][2]):
            pos -= 1
        best = best[:pos] + [(d, slot, l)] + best[pos:3]
    return best


def test_oracle_assignment_fp32_matches_transliteration(oracle):
    rng = np.random.default_rng(5)
    rows, dim = 40, 20
    x = rng.standard_normal((rows, dim)).astype(np.float32)
    x[7] = x[6]  # P/tessa_replay.rs:1803-1810 duplicates a row to force ties
    norms = oracle.raw_norms(x)
    codes, scales, qn = oracle.quantize_sq8(x)
    gids = (np.arange(rows) * 3 + 1).astype(np.uint32)
    members = np.arange(rows, dtype=np.uint32)
    leaders = np.array([6, 7, 1, 2, 3, 9, 11], np.uint32)
    ids, dists = oracle.assign(0, x, norms, codes, scales, gids, members, leaders, [0], [rows], [0],
                               [len(leaders)], [2], [0], rows * 2)
    for p in range(rows):
        best = _py_assign(x, norms, leaders, p)
        for r in range(2):
            assert ids[p * 2 + r] == gids[best[r][2]]
            assert dists[p * 2 + r] == best[r][0]
    sids, sd = oracle.assign(2, x, qn, codes, scales, gids, members, leaders, [0], [rows], [0],
                             [len(leaders)], [2], [0], rows * 2)
    for p in range(rows):
        best = _py_assign(x, qn, leaders, p, fp32=False, codes=codes, scales=scales)
        for r in range(2):
            assert sids[p * 2 + r] == gids[best[r][2]]
            assert sd[p * 2 + r] == best[r][0]


# ------------------------------------------------------------- global D0

def test_d0_reference_assigns_by_sq_distance_with_stable_ties(oracle):
    # P/dco_sq_int8.rs:3422-3453 sq_gpu_d0_reference_assigns_by_sq_distance_with_stable_ties
    leaders = np.array([[1.0, 0.0], [-1.0, 0.0]], np.float32)
    payload = oracle.quantize_sq8(leaders)
    r = oracle.d0_assign(np.array([[0.0, 0.0], [1.0, 0.0]], np.float32), [0, 1], [5, 3], leaders, 1,
                         leader_payload=payload)
    frags = list(zip(r["child_ids"].ravel().tolist(), r["point_ids"].ravel().tolist()))
    assert frags == [(1, 0), (0, 1)]
    assert r["codes"].shape == (2, 16)


@pytest.mark.parametrize("fanout", [1, 6, 17, 32])
def test_d0_oracle_matches_sorting_reference_on_compute_backend_fixture(oracle, fanout):
    # compute_backend.rs:43857-43940 fixture (duplicate leader, row equal to a leader)
    from d0cases import reference_fixture_43857, py_d0_sort
    raw, gids, lids, lv = reference_fixture_43857()
    r = oracle.d0_assign(raw, gids, lids, lv, fanout)
    lc, ls, ln = oracle.quantize_sq8(lv)
    want = py_d0_sort(r["codes"], r["scales"], r["norms"], lc, ls, ln, lids, fanout)
    assert np.array_equal(r["child_ids"], want)
    assert np.array_equal(r["point_ids"], np.repeat(gids, fanout).reshape(-1, fanout))
    # leader 1 (id 100) ties leader 0 (id 90000) exactly: the smaller id wins
    assert r["child_ids"][0, 0] == 1


@pytest.mark.parametrize("rows,dim,leaders,fanout,seed", [(40, 24, 19, 3, 1), (25, 100, 64, 8, 2),
                                                           (30, 16, 5, 5, 3)])
def test_d0_oracle_matches_sorting_reference_on_random_rows(oracle, rows, dim, leaders, fanout, seed):
    from d0cases import random_case, py_d0_sort
    raw, gids, lids, lv = random_case(rows, dim, leaders, seed)
    r = oracle.d0_assign(raw, gids, lids, lv, fanout)
    lc, ls, ln = oracle.quantize_sq8(lv)
    assert np.array_equal(r["child_ids"], py_d0_sort(r["codes"], r["scales"], r["norms"], lc, ls, ln, lids,
                                                      fanout))


def test_d0_oracle_rejects_invalid_requests(oracle):
    # P/dco_sq_int8.rs:1932-1960
    lv = np.ones((2, 4), np.float32)
    with pytest.raises(ValueError, match="at least one input row"):
        oracle.d0_assign(np.zeros((0, 4), np.float32), [], [1, 2], lv, 1)
    with pytest.raises(ValueError, match="at least one global D0 leader"):
        oracle.d0_assign(np.ones((1, 4), np.float32), [0], [], np.zeros((0, 4), np.float32), 1)
    for f in (0, 3):
        with pytest.raises(ValueError, match="fanout must be in"):
            oracle.d0_assign(np.ones((1, 4), np.float32), [0], [1, 2], lv, f)


# ------------------------------------------------------------ candidate edges

def _test_sketches(num_points, width):
    # P/leaf_build.rs:2900-2908 build_test_sketches: point * 0.1 + bit (f32)
    return np.array([[np.float32(p) * np.float32(0.1) + np.float32(b) for b in range(width)]
                     for p in range(num_points)], np.float32)


def test_flush_edges_reference_fixture(oracle):
    # P/leaf_build.rs:3126-3137 fixture, 12-bit hashes: every valid slot gives
    # (i -> j, hash(s_i, s_j)) then (j -> i, hash(s_j, s_i)); the (30, u32::MAX,
    # inf) slot is skipped.
    sk = _test_sketches(31, 12)
    p, c, h, d = oracle.flush_edges([10, 20, 30], [20, 30, 30, 10, 20, 0xFFFFFFFF],
                                    [1.0, 2.0, 1.5, 1.0, 1.5, np.inf], 2, sk, 12)
    assert list(zip(p.tolist(), c.tolist())) == [(10, 20), (20, 10), (10, 30), (30, 10), (20, 30), (30, 20),
                                                 (20, 10), (10, 20), (30, 20), (20, 30)]
    assert d.tolist() == [1.0, 1.0, 2.0, 2.0, 1.5, 1.5, 1.0, 1.0, 1.5, 1.5]
    # higher point ids have larger sketches in every bit: forward to a larger id = all ones
    assert h.tolist() == [0xFFF, 0, 0xFFF, 0, 0xFFF, 0, 0, 0xFFF, 0, 0xFFF]


def test_compute_hash_and_sketch_transliteration(oracle):
    rng = np.random.default_rng(4)
    a = rng.standard_normal(16).astype(np.float32)
    b = a.copy()
    b[3] = a[3] + np.float32(1e-3)
    b[5] = np.nextafter(a[5], np.float32(-np.inf), dtype=np.float32)
    want = sum(1 << i for i in range(16) if np.float32(b[i] - a[i]) >= 0)
    assert oracle.compute_hash(a, b, 16) == want
    assert oracle.compute_hash(a, b, 4) == want & 0xF
    x = rng.standard_normal((5, 37)).astype(np.float32)
    planes = rng.uniform(-1, 1, (12, 37)).astype(np.float32)
    got = oracle.sketch_rows(x, planes)
    for i in range(5):
        for hh in range(12):
            acc = np.float32(0)
            for ax in range(37):
                acc = np.float32(acc + np.float32(x[i, ax] * planes[hh, ax]))
            assert got[i, hh].view(np.uint32) == acc.view(np.uint32)


def test_library_expand_edges_matches_oracle_flush(oracle):
    # host-only entry point of the library (no device work)
    from shear_b200 import ops
    rng = np.random.default_rng(9)
    rows, k, n = 300, 7, 1000
    sk = rng.standard_normal((n, 12)).astype(np.float32)
    pid = rng.permutation(n)[:rows].astype(np.uint32)
    ids = rng.integers(0, n, rows * k).astype(np.uint32)
    ds = rng.uniform(0, 2, rows * k).astype(np.float32)
    ids[::11] = 0xFFFFFFFF
    ds[5::13] = np.inf
    ds[7::17] = np.nan
    hf = np.array([oracle.compute_hash(sk[pid[s // k]], sk[ids[s]], 12) if ids[s] != 0xFFFFFFFF else 0
                   for s in range(rows * k)], np.uint16)
    hr = np.array([oracle.compute_hash(sk[ids[s]], sk[pid[s // k]], 12) if ids[s] != 0xFFFFFFFF else 0
                   for s in range(rows * k)], np.uint16)
    want = oracle.flush_edges(pid, ids, ds, k, sk, 12)
    for threads in (1, 3, 8):
        got = ops.expand_edges(pid, ids, ds, hf, hr, k, threads=threads)
        for g, w in zip(got, want):
            assert np.array_equal(g.view(np.uint8), w.view(np.uint8))
