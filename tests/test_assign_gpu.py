"""TESSA assignment replay on the B200 vs the oracle.

FP32: bit-exact with the reference's FP32 SIMT executor order.  SQ8: bit-exact
with the contracted (single FFMA) form of CB:14676-14678; ids equal to the
uncontracted form except where two leaders are within the 2e-5 tie window.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _tasks(rng, rows, ntasks):
    moff, mcnt, loff, lcnt, rh, out = [], [], [], [], [], []
    members, leaders = [], []
    o = 0
    for t in range(ntasks):
        m = int(rng.integers(1, 300))
        l = int(rng.integers(1, 100))
        r = int(rng.integers(1, min(4, l) + 1))
        moff.append(len(members)); mcnt.append(m)
        loff.append(len(leaders)); lcnt.append(l)
        rh.append(r); out.append(o)
        members += rng.integers(0, rows, m).tolist()
        leaders += rng.choice(rows, l, replace=False).tolist()
        o += m * r
    return (np.array(members, np.uint32), np.array(leaders, np.uint32), moff, mcnt, loff, lcnt, rh,
            np.array(out, np.uint64), o)


@pytest.mark.parametrize("dim", [20, 128, 768])
def test_assignment_fp32_and_sq8_match_oracle(oracle, dim):
    import torch
    from shear_b200 import ops
    from shear_b200._capi import ASSIGN_FP32, ASSIGN_SQ8
    rng = np.random.default_rng(dim)
    rows = 2000
    x = rng.standard_normal((rows, dim)).astype(np.float32)
    x[7] = x[6]
    raw = oracle.raw_norms(x)
    codes, scales, qn = oracle.quantize_sq8(x)
    gids = rng.permutation(10 * rows)[:rows].astype(np.uint32)
    members, leaders, moff, mcnt, loff, lcnt, rh, out, n = _tasks(rng, rows, 6)
    dv = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    common = dict(global_ids=dv(gids.view(np.int32)), members=dv(members.view(np.int32)),
                  leaders=dv(leaders.view(np.int32)), task_member_offsets=moff, task_member_counts=mcnt,
                  task_leader_offsets=loff, task_leader_counts=lcnt, task_rh=rh, task_output_offsets=out,
                  output_len=n)
    ids, d = ops.assign(ASSIGN_FP32, x=dv(x), raw_norms=dv(raw), **common)
    wi, wd = oracle.assign(0, x, raw, codes, scales, gids, members, leaders, moff, mcnt, loff, lcnt, rh, out, n)
    assert np.array_equal(ops.as_u32(ids), wi)
    assert np.array_equal(d.cpu().numpy().view(np.uint32), wd.view(np.uint32))
    ids, d = ops.assign(ASSIGN_SQ8, codes=dv(codes), scales=dv(scales), sq8_norms=dv(qn), **common)
    wi, wd = oracle.assign(3, x, qn, codes, scales, gids, members, leaders, moff, mcnt, loff, lcnt, rh, out, n)
    assert np.array_equal(ops.as_u32(ids), wi)
    assert np.array_equal(d.cpu().numpy().view(np.uint32), wd.view(np.uint32))
    ui, ud = oracle.assign(2, x, qn, codes, scales, gids, members, leaders, moff, mcnt, loff, lcnt, rh, out, n)
    # Against the uncontracted form: same leader wherever no two leaders sit
    # inside the 2e-5 tie window, and distances a few ulp apart there.
    same = ops.as_u32(ids) == ui
    assert same.mean() > 0.99
    assert np.allclose(d.cpu().numpy()[same], ud[same], rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("leaders,dim", [(16, 768), (16, 128), (32, 768), (60, 256), (128, 784)])
def test_sq8_assignment_many_items_per_cta(oracle, leaders, dim):
    """Enough 128-row work items that every CTA of the persistent tensor-core
    kernel takes several (ring wrap-around, both accumulator buffers, slabs
    pending across item boundaries), with ragged member counts, one leader
    width per launch (16, 32, 64 and 128 leader slots) and a K tail
    (784 = 6 slabs + 16 bytes)."""
    import torch
    from shear_b200 import ops
    from shear_b200._capi import ASSIGN_SQ8
    rng = np.random.default_rng(1000 + leaders + dim)
    rows = 6000
    x = rng.standard_normal((rows, dim)).astype(np.float32)
    codes, scales, qn = oracle.quantize_sq8(x)
    gids = rng.permutation(10 * rows)[:rows].astype(np.uint32)
    ntasks = 420
    moff, mcnt, loff, lcnt, rh, out = [], [], [], [], [], []
    members, lead = [], []
    o = 0
    for t in range(ntasks):
        m = int(rng.integers(1, 400))
        r = int(rng.integers(1, 5))
        moff.append(len(members)); mcnt.append(m)
        loff.append(len(lead)); lcnt.append(leaders)
        rh.append(r); out.append(o)
        members += rng.integers(0, rows, m).tolist()
        lead += rng.choice(rows, leaders, replace=False).tolist()
        o += m * r
    members = np.array(members, np.uint32)
    lead = np.array(lead, np.uint32)
    out = np.array(out, np.uint64)
    dv = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    ids, d = ops.assign(ASSIGN_SQ8, codes=dv(codes), scales=dv(scales), sq8_norms=dv(qn),
                        global_ids=dv(gids.view(np.int32)), members=dv(members.view(np.int32)),
                        leaders=dv(lead.view(np.int32)), task_member_offsets=moff, task_member_counts=mcnt,
                        task_leader_offsets=loff, task_leader_counts=lcnt, task_rh=rh, task_output_offsets=out,
                        output_len=o)
    wi, wd = oracle.assign(3, x, qn, codes, scales, gids, members, lead, moff, mcnt, loff, lcnt, rh, out, o)
    assert np.array_equal(ops.as_u32(ids), wi)
    assert np.array_equal(d.cpu().numpy().view(np.uint32), wd.view(np.uint32))


@pytest.mark.parametrize("leaders", [16, 60])
def test_sq8_assignment_exact_leader_ties(oracle, leaders):
    """Every row has an identical twin and the tasks' leaders include both
    twins, so many candidates tie exactly (and within 2e-5) with a held slot:
    the insertion must take the reference's hash-tie rule (CB:6524-6578) for
    those and the plain distance order elsewhere."""
    import torch
    from shear_b200 import ops
    from shear_b200._capi import ASSIGN_SQ8
    rng = np.random.default_rng(77 + leaders)
    rows, dim = 4000, 128
    x = rng.standard_normal((rows, dim)).astype(np.float32)
    x[1::2] = x[0::2]
    codes, scales, qn = oracle.quantize_sq8(x)
    gids = rng.permutation(10 * rows)[:rows].astype(np.uint32)
    ntasks = 300
    moff, mcnt, loff, lcnt, rh, out = [], [], [], [], [], []
    members, lead = [], []
    o = 0
    for t in range(ntasks):
        m = int(rng.integers(1, 300))
        moff.append(len(members)); mcnt.append(m)
        loff.append(len(lead)); lcnt.append(leaders)
        r = 4
        rh.append(r); out.append(o)
        members += rng.integers(0, rows, m).tolist()
        base = rng.choice(rows // 2, leaders // 2, replace=False) * 2
        lead += np.stack([base, base + 1], 1).reshape(-1).tolist()
        o += m * r
    members = np.array(members, np.uint32)
    lead = np.array(lead, np.uint32)
    out = np.array(out, np.uint64)
    dv = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    ids, d = ops.assign(ASSIGN_SQ8, codes=dv(codes), scales=dv(scales), sq8_norms=dv(qn),
                        global_ids=dv(gids.view(np.int32)), members=dv(members.view(np.int32)),
                        leaders=dv(lead.view(np.int32)), task_member_offsets=moff, task_member_counts=mcnt,
                        task_leader_offsets=loff, task_leader_counts=lcnt, task_rh=rh, task_output_offsets=out,
                        output_len=o)
    wi, wd = oracle.assign(3, x, qn, codes, scales, gids, members, lead, moff, mcnt, loff, lcnt, rh, out, o)
    assert np.array_equal(ops.as_u32(ids), wi)
    assert np.array_equal(d.cpu().numpy().view(np.uint32), wd.view(np.uint32))
    # the twins really tie: a row's two best slots are almost always the two
    # copies of its nearest leader, ordered by the tie key
    got = ops.as_u32(ids).reshape(-1, 4)
    twin_of = dict(zip(gids[0::2].tolist(), gids[1::2].tolist()))
    twin_of.update(zip(gids[1::2].tolist(), gids[0::2].tolist()))
    pairs = np.array([twin_of.get(a) == b for a, b in got[:, :2].tolist()])
    assert pairs.mean() > 0.9
