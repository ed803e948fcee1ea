"""Device HashPrune reservoirs (tessa_reduce_records / tessa_reduce_grouped)
on the B200.

The reference reduces candidate edges on the CPU, one insert_inner call per
edge (P/hash_prune.rs:1326-1452).  The device reduction must leave the same
slots: against the line-by-line Python restatement of insert_inner on small
cases (targets, hashes and distances of every slot), against the host reducer
on larger ones, and through its own merge path (reservoirs of pieces merged
again equal the reservoirs of the whole), with distance ties, colliding hashes,
negative and signed-zero distances, missing and non-finite slots.
"""
import numpy as np
import pytest

from oracle import hashprune as HP

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda:0")


def _records(batch):
    pid, ids, ds, hf, hr, k = batch
    return (_dev(pid.view(np.int32)), _dev(ids.view(np.int32).reshape(-1)), _dev(ds.reshape(-1)),
            _dev(hf.view(np.int16).reshape(-1)), _dev(hr.view(np.int16).reshape(-1)), k)


def _concat(batches):
    k = batches[0][5]
    cat = lambda i: np.concatenate([b[i] for b in batches])
    return cat(0), cat(1), cat(2), cat(3), cat(4), k


def _host(offsets, nb, sl, count):
    from shear_b200 import ops
    off = offsets.cpu().numpy().view(np.uint64)
    assert int(off[-1]) == count
    n = nb[:count].cpu().numpy().view(np.uint32) if nb is not None else None
    s = sl[:count * 12].cpu().numpy().view(ops.EDGE_DTYPE) if sl is not None else None
    return off, n, s


def _signed_dists(rng, shape):
    d = (rng.random(shape).astype(np.float32) - np.float32(0.1))  # some negative (SQ8 rounding can give them)
    d[rng.random(shape) < 0.03] = np.float32(0.0)
    d[rng.random(shape) < 0.03] = np.float32(-0.0)
    d[rng.random(shape) < 0.02] = np.nan
    return d


@pytest.mark.parametrize("points,l_max,m_bits,dup", [(50, 8, 4, False), (200, 16, 6, True), (30, 64, 12, False),
                                                     (120, 5, 3, True), (40, 1, 2, True)])
def test_device_reservoirs_equal_insert_inner_restatement(points, l_max, m_bits, dup):
    from shear_b200 import ops
    from test_reducer import _batches
    rng = np.random.default_rng(points * 7 + l_max + m_bits)
    batches = _batches(rng, points, 300, 3, 4, m_bits, dup)
    if not dup:
        for b in batches:
            b[2][...] = _signed_dists(rng, b[2].shape)
    want = HP.reduce_leaf_batches(points, l_max, batches, slots=True)
    whole = _concat(batches)
    off, nb, sl = _host(*ops.reduce_records(*_records(whole), points, l_max, slots=True))
    for p in range(points):
        a, b = int(off[p]), int(off[p + 1])
        w = want[p]
        assert nb[a:b].tolist() == [t for t, _, _ in w], p
        assert sl["target"][a:b].tolist() == [t for t, _, _ in w], p
        assert sl["hash"][a:b].tolist() == [h for _, h, _ in w], p
        assert sl["dist"][a:b].view(np.uint32).tolist() == \
            np.array([d for _, _, d in w], np.float32).view(np.uint32).tolist(), p


def test_device_reservoirs_equal_host_reducer_at_scale():
    from shear_b200 import ops
    from test_reducer import _batches
    rng = np.random.default_rng(11)
    points, k, l_max = 20000, 2, 64
    batches = _batches(rng, points, 100000, k, 3, 12, dup_dist=True)
    # overlapping leaves: repeat records exactly
    b0 = batches[0]
    rep = rng.integers(0, b0[0].size, 50000)
    batches.append(tuple(a[rep] for a in b0[:5]) + (k,))
    red = ops.Reducer(points, l_max, 4)
    for b in batches:
        red.add(*b)
    want_off, want_nb = red.finish()
    red.close()
    off, nb, _ = _host(*ops.reduce_records(*_records(_concat(batches)), points, l_max))
    assert np.array_equal(off, want_off.astype(np.uint64))
    assert np.array_equal(nb, want_nb)


def test_hub_selection_with_equal_values_and_small_l_max():
    # One source receives thousands of edges: many share distance and target
    # under different hashes, so the l_max-th best is decided by the hash.
    from shear_b200 import ops
    rng = np.random.default_rng(5)
    rows, k = 6000, 2
    pid = np.zeros(rows, np.uint32)
    ids = rng.integers(1, 40, (rows, k)).astype(np.uint32)
    ds = (np.round(rng.random((rows, k)) * 3) / 4).astype(np.float32)
    hf = rng.integers(0, 1 << 16, (rows, k)).astype(np.uint16)
    hr = rng.integers(0, 1 << 16, (rows, k)).astype(np.uint16)
    batch = (pid, ids, ds, hf, hr, k)
    for l_max in (1, 7, 33, 255):
        want = HP.reduce_leaf_batches(40, l_max, [batch], slots=True)
        off, nb, sl = _host(*ops.reduce_records(*_records(batch), 40, l_max, slots=True))
        for p in range(40):
            a, b = int(off[p]), int(off[p + 1])
            assert list(zip(sl["target"][a:b].tolist(), sl["hash"][a:b].tolist())) == \
                [(t, h) for t, h, _ in want[p]], (l_max, p)


def test_merging_reservoirs_of_pieces_equals_whole():
    # min over hashes and the l_max best commute with splitting the edges:
    # reservoirs of three pieces, merged, equal the reservoirs of all edges;
    # so do the grouped records of tessa_group_edges.
    from shear_b200 import ops
    from test_reducer import _batches
    rng = np.random.default_rng(21)
    points, k, l_max = 3000, 3, 24
    batches = _batches(rng, points, 20000, k, 3, 8, dup_dist=True)
    whole = _concat(batches)
    off_w, nb_w, sl_w, cnt_w = ops.reduce_records(*_records(whole), points, l_max, slots=True)
    pieces = [ops.reduce_records(*_records(b), points, l_max, slots=True) for b in batches]
    merged = ops.reduce_grouped([(o, s, c) for o, _, s, c in pieces], points, l_max, slots=True)
    a, b = _host(off_w, nb_w, sl_w, cnt_w), _host(*merged)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    assert np.array_equal(a[2].view(np.uint8), b[2].view(np.uint8))
    goff, gedges = ops.group_edges(*_records(whole)[:5], k, points)
    total = int(goff[-1].item())
    c = _host(*ops.reduce_grouped([(goff, gedges, total)], points, l_max))
    assert np.array_equal(a[0], c[0]) and np.array_equal(a[1], c[1])


def test_grouped_offsets_need_not_start_at_zero():
    # a slice of a larger CSR (one owner's range of points) is a valid piece
    import torch
    from shear_b200 import ops
    from test_reducer import _batches
    rng = np.random.default_rng(8)
    points, l_max = 1000, 16
    (batch,) = _batches(rng, points, 6000, 2, 1, 10)
    off, _, sl, cnt = ops.reduce_records(*_records(batch), points, l_max, slots=True)
    lo, hi = 300, 700
    base = int(off[lo].item())
    piece = (off[lo:hi + 1].contiguous(), sl[base * 12:], int(off[hi].item()) - base)
    got = _host(*ops.reduce_grouped([piece], hi - lo, l_max))
    full = _host(off, None, sl, cnt)
    want_nb = full[2]["target"][base:int(off[hi].item())]
    assert np.array_equal(got[1], want_nb)
    assert np.array_equal(got[0], full[0][lo:hi + 1] - np.uint64(base))
    torch.cuda.synchronize()


def test_empty_input_and_errors():
    import torch
    from shear_b200 import ops, TessaError
    dev = torch.device("cuda:0")
    e = torch.empty(0, dtype=torch.int32, device=dev)
    h = torch.empty(0, dtype=torch.int16, device=dev)
    off, nb, _, cnt = ops.reduce_records(e, e, torch.empty(0, device=dev), h, h, 2, 10, 8)
    assert cnt == 0 and not off.any()
    pid = torch.tensor([0, 1], dtype=torch.int32, device=dev)
    ids = torch.tensor([1, 7], dtype=torch.int32, device=dev)
    ds = torch.tensor([0.5, 0.25], device=dev)
    h2 = torch.zeros(2, dtype=torch.int16, device=dev)
    with pytest.raises(TessaError, match="BAD_ROW"):
        ops.reduce_records(pid, ids, ds, h2, h2, 1, 4, 8)
    ids = torch.tensor([1, 2], dtype=torch.int32, device=dev)
    hf = torch.tensor([1, 2], dtype=torch.int16, device=dev)
    small = (torch.empty(5, dtype=torch.int64, device=dev), torch.empty(1, dtype=torch.int32, device=dev), None)
    with pytest.raises(TessaError, match="capacity"):
        ops.reduce_records(pid, ids, ds, hf, hf, 1, 4, 8, out=small)
    with pytest.raises(TessaError, match="l_max"):
        ops.reduce_records(pid, ids, ds, hf, hf, 1, 4, 0)
