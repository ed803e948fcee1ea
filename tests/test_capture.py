"""TESSA capture restatement (shear_b200/capture.py) against the reference's
own capture tests (P/tessa_capture.rs:1103-1454), and the digest path."""
import json
import os

import numpy as np
import pytest

from shear_b200 import capture as cap


def hex_digest(b):
    return f"{b:02x}" * 32


def dataset():
    return {"canonical_base_path": "/data/base.fbin", "rows": 1_000_000, "dimension": 1024,
            "header_sha256": hex_digest(0x11)}


def provenance():
    return {"seed": 42, "git_commit": "0123456789abcdef", "binary_sha256": hex_digest(0x22),
            "command_sha256": hex_digest(0x33), "root_leader_hash": 11, "d0_partition_hash": 13,
            "d0_task_list_hash": 17}


def assignment_task(i, rows, leaders):
    return cap.make_tessa_assignment_task(42, 1, i, min(leaders, 8), 1024,
                                          [((i * 10_007 + r) % 1_000_000) for r in range(rows)][::-1],
                                          [((i * 257 + l) % 1_000_000) for l in range(leaders)])


def leaf_task(i, rows):
    return cap.make_tessa_leaf_task(42, 2, 1024, [((i * 4099 + r) % 1_000_000) for r in range(rows)][::-1])


def small_selection():
    s = cap.TessaCaptureSampler(42)
    s.observe_assignment(assignment_task(1, 256, 16))
    s.observe_assignment(assignment_task(2, 513, 17))
    s.observe_leaf(leaf_task(3, 256))
    return s.finish()


def test_bin_boundaries_are_exact():
    assert [cap.assignment_row_bin(v) for v in (255, 256, 1024, 1025, 8192, 8193)] == [None, 0, 0, 1, 1, 2]
    assert [cap.assignment_leader_bin(v) for v in (0, 16, 17, 32, 33, 64, 65, 128, 129)] == \
        [None, 0, 1, 1, 2, 2, 3, 3, None]
    assert [cap.leaf_size_bin(v) for v in (255, 256, 512, 513, 896, 897, 1280, 1281)] == \
        [None, 0, 0, 1, 1, 2, 2, None]


def test_dataset_metadata_hashes_the_canonical_fbin_header(tmp_path):
    import hashlib
    import struct
    path = tmp_path / "base.fbin"
    path.write_bytes(struct.pack("<ii", 3, 2) + bytes(3 * 2 * 4))
    m = cap.tessa_capture_dataset_metadata(str(path))
    assert (m["rows"], m["dimension"]) == (3, 2)
    assert m["canonical_base_path"] == os.path.realpath(str(path))
    assert m["header_sha256"] == hashlib.sha256(struct.pack("<ii", 3, 2)).hexdigest()


def test_bottom_k_is_order_independent_and_bounded():
    assignments, leaves, i = [], [], 0
    for rows in (256, 1025, 8193):
        for leaders in (16, 17, 33, 65):
            for _ in range(20):
                assignments.append(assignment_task(i, rows, leaders))
                i += 1
    for rows in (256, 513, 897):
        for _ in range(70):
            leaves.append(leaf_task(i, rows))
            i += 1

    def select(a_order, l_order):
        s = cap.TessaCaptureSampler(42)
        for j in a_order:
            s.observe_assignment(assignments[j])
        for j in l_order:
            s.observe_leaf(leaves[j])
        return s.finish()

    fwd = select(range(len(assignments)), range(len(leaves)))
    rev = select(reversed(range(len(assignments))), reversed(range(len(leaves))))
    shuf = select(sorted(range(len(assignments)), key=lambda j: assignments[j].priority ^ 0xA5A5A5A5),
                  sorted(range(len(leaves)), key=lambda j: leaves[j].priority ^ 0x5A5A5A5A))
    ah = lambda s: [t.task_hash for t in s.assignment_tasks]
    lh = lambda s: [t.task_hash for t in s.leaf_tasks]
    assert ah(fwd) == ah(rev) == ah(shuf)
    assert lh(fwd) == lh(rev) == lh(shuf)
    assert len(fwd.assignment_tasks) == 12 * 16 and len(fwd.leaf_tasks) == 3 * 64
    assert fwd.bin_counts["assignment_observed"] == [[20] * 4] * 3
    assert fwd.bin_counts["assignment_selected"] == [[16] * 4] * 3
    assert fwd.bin_counts["leaf_observed"] == [70] * 3 and fwd.bin_counts["leaf_selected"] == [64] * 3


def test_fragment_round_trip_merge_and_idempotency(tmp_path):
    d = str(tmp_path)
    first = small_selection()
    p1 = cap.write_tessa_capture_fragment(d, 0x11, first)
    b1 = open(p1, "rb").read()
    assert cap.write_tessa_capture_fragment(d, 0x11, first) == p1
    assert open(p1, "rb").read() == b1
    conflicting = cap.TessaCaptureSelection(first.assignment_tasks, first.leaf_tasks,
                                            json.loads(json.dumps(first.bin_counts)))
    conflicting.bin_counts["leaf_observed"][0] += 1
    with pytest.raises(cap.CaptureError):
        cap.write_tessa_capture_fragment(d, 0x11, conflicting)
    s2 = cap.TessaCaptureSampler(42)
    s2.observe_assignment(assignment_task(4, 1025, 33))
    s2.observe_leaf(leaf_task(5, 513))
    cap.write_tessa_capture_fragment(d, 0x22, s2.finish())
    m = cap.merge_tessa_capture_fragments(d, 42)
    assert len(m.assignment_tasks) == 3 and len(m.leaf_tasks) == 2
    bc = m.bin_counts
    assert (bc["assignment_observed"][0][0], bc["assignment_observed"][0][1], bc["assignment_observed"][1][2]) == \
        (1, 1, 1)
    assert bc["leaf_observed"] == [1, 1, 0] and bc["leaf_selected"] == [1, 1, 0]
    assert (bc["assignment_selected"][0][0], bc["assignment_selected"][0][1], bc["assignment_selected"][1][2]) == \
        (1, 1, 1)
    # serde_json's pretty layout: two-space indent, one array element per line, trailing newline
    text = b1.decode()
    assert text.startswith('{\n  "version": 1,\n  "request_hash": 17,\n  "selection": {\n') and text.endswith("}\n")


def test_round_trip_is_little_endian_and_byte_stable(tmp_path):
    a, b = str(tmp_path / "a"), str(tmp_path / "b")
    sel = small_selection()
    cap.write_tessa_capture(a, dataset(), provenance(), sel)
    cap.write_tessa_capture(b, dataset(), provenance(), sel)
    _, at, lt = cap.load_tessa_capture(a, dataset())
    assert at == sel.assignment_tasks and lt == sel.leaf_tasks
    first = sel.assignment_tasks[0].member_ids[0]
    assert open(os.path.join(a, cap.TESSA_ASSIGNMENT_MEMBERS_FILE), "rb").read()[:4] == first.to_bytes(4, "little")
    for f in (cap.TESSA_CAPTURE_MANIFEST_FILE, cap.TESSA_ASSIGNMENT_MEMBERS_FILE, cap.TESSA_ASSIGNMENT_LEADERS_FILE,
              cap.TESSA_LEAF_MEMBERS_FILE):
        assert open(os.path.join(a, f), "rb").read() == open(os.path.join(b, f), "rb").read()
    alias = dataset()
    alias["canonical_base_path"] = "/same/data/through/another/mount.fbin"
    cap.load_tessa_capture(a, alias)


def _corrupt(d, update):
    p = os.path.join(d, cap.TESSA_CAPTURE_MANIFEST_FILE)
    v = json.loads(open(p, "rb").read())
    update(v)
    open(p, "wb").write((json.dumps(v, indent=2) + "\n").encode())


def test_rejects_corrupt_or_mismatched_inputs(tmp_path):
    def fresh(name):
        d = str(tmp_path / name)
        cap.write_tessa_capture(d, dataset(), provenance(), small_selection())
        return d

    d = fresh("version")
    _corrupt(d, lambda v: v.__setitem__("version", 2))
    with pytest.raises(cap.CaptureError):
        cap.load_tessa_capture(d)
    d = fresh("length")
    p = os.path.join(d, cap.TESSA_ASSIGNMENT_MEMBERS_FILE)
    open(p, "wb").write(open(p, "rb").read()[:-4])
    with pytest.raises(cap.CaptureError):
        cap.load_tessa_capture(d)
    d = fresh("dup")
    _corrupt(d, lambda v: v["assignment_tasks"][1].__setitem__("task_hash", v["assignment_tasks"][0]["task_hash"]))
    with pytest.raises(cap.CaptureError):
        cap.load_tessa_capture(d)
    d = fresh("range")
    p = os.path.join(d, cap.TESSA_ASSIGNMENT_MEMBERS_FILE)
    data = bytearray(open(p, "rb").read())
    data[:4] = dataset()["rows"].to_bytes(4, "little")
    open(p, "wb").write(bytes(data))
    with pytest.raises(cap.CaptureError):
        cap.load_tessa_capture(d)
    d = fresh("mismatch")
    e = dataset()
    e["header_sha256"] = hex_digest(0xFF)
    with pytest.raises(cap.CaptureError):
        cap.load_tessa_capture(d, e)


def test_digest_observation_equals_task_observation():
    rng = np.random.default_rng(3)
    sizes = list(rng.integers(200, 1400, 300))
    members = [rng.choice(1_000_000, n, replace=False).astype(np.uint32) for n in sizes]
    a = cap.TessaCaptureSampler(7)
    for m in members:
        a.observe_leaf(cap.TessaLeafTask(0, 0, 4, 768, list(m)))
    b = cap.TessaCaptureSampler(7)
    digests = np.array([cap.membership_digest(m) for m in members], dtype=np.uint64)
    calls = []
    b.observe_leaf_digests(4, 768, sizes, digests, lambda l: (calls.append(l), members[l])[1])
    fa, fb = a.finish(), b.finish()
    assert [t.task_hash for t in fa.leaf_tasks] == [t.task_hash for t in fb.leaf_tasks]
    assert fa.leaf_tasks == fb.leaf_tasks and fa.bin_counts == fb.bin_counts
    assert len(calls) < len(sizes)  # member lists copied only for candidates of a bin


def test_membership_digest_matches_scalar_restatement():
    ids = [0, 1, 63, 64, 65, 0xFFFFFFFF, 123456789]
    n, s, x = cap.membership_digest(ids)
    ss = xx = 0
    for i in ids:
        m = cap.mix_membership_id(i)
        ss = (ss + m) & ((1 << 64) - 1)
        r = i & 63
        xx ^= ((m << r) | (m >> (64 - r))) & ((1 << 64) - 1) if r else m
    assert (n, s, x) == (len(ids), ss, xx)
