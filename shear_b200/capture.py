"""TESSA capture: bounded, order-independent samples of the assignment and leaf
tasks a build runs, written in the reference's on-disk format so replay
fixtures can come from B200 runs.

Restates shear-core/src/algorithm/pipnn/tessa_capture.rs (P/tessa_capture.rs):
task hashes and priorities (stable FNV-1a 64 over a domain tag, :177-300),
row / leader / size bins (:206-232), the bottom-k sampler (:350-458), JSON
fragments and their merge (:460-597), the capture directory (manifest.json and
three little-endian u32 files, :599-687) and its loader with validation
(:689-1099).  JSON is written as serde_json's pretty printer writes it (two
space indent, one array element per line, trailing newline), so fragments and
manifests are byte-compatible with the reference's.

The device side: the membership digest that enters every task hash (a sum and
an xor of splitmix-mixed ids, :274-293) does not depend on member order, so
``ops.membership_digests`` computes it per leaf on the GPU from the device
member arrays; ``observe_leaf_digests`` then ranks every leaf by priority on
the host and copies out only the member lists of the tasks the sampler keeps.
"""
from __future__ import annotations

import dataclasses
import hashlib
import json
import os
import struct
from typing import Callable, Iterable, Sequence

import numpy as np

TESSA_CAPTURE_VERSION = 1
TESSA_CAPTURE_MANIFEST_FILE = "manifest.json"
TESSA_ASSIGNMENT_MEMBERS_FILE = "assignment_members.u32le"
TESSA_ASSIGNMENT_LEADERS_FILE = "assignment_leaders.u32le"
TESSA_LEAF_MEMBERS_FILE = "leaf_members.u32le"
TESSA_ASSIGNMENT_ROW_BINS = 3
TESSA_ASSIGNMENT_LEADER_BINS = 4
TESSA_LEAF_SIZE_BINS = 3
TESSA_ASSIGNMENT_BIN_LIMIT = 16
TESSA_LEAF_BIN_LIMIT = 64

_FNV_OFFSET = 0xCBF29CE484222325
_FNV_PRIME = 0x100000001B3
_M64 = (1 << 64) - 1


class CaptureError(ValueError):
    """A capture file or request the reference would reject (message prefix as its)."""

    def __init__(self, message: str):
        super().__init__(f"TESSA capture: {message}")


# ---------------------------------------------------------------- hashing

class _Fnv1a64:
    """P/tessa_capture.rs:177-204 StableFnv1a64 (a zero result becomes 1)."""

    def __init__(self, domain: bytes):
        self.h = _FNV_OFFSET
        self.write(domain)

    def write(self, data: bytes) -> None:
        h = self.h
        for b in data:
            h = ((h ^ b) * _FNV_PRIME) & _M64
        self.h = h

    def u32(self, v: int) -> None:
        self.write(struct.pack("<I", v & 0xFFFFFFFF))

    def u64(self, v: int) -> None:
        self.write(struct.pack("<Q", v & _M64))

    def finish(self) -> int:
        return self.h if self.h != 0 else 1


def mix_membership_id(value: int) -> int:
    """P/tessa_capture.rs:274-279 (splitmix64 finaliser of id + golden ratio)."""
    m = (value + 0x9E3779B97F4A7C15) & _M64
    m = ((m ^ (m >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    m = ((m ^ (m >> 27)) * 0x94D049BB133111EB) & _M64
    return m ^ (m >> 31)


def _rotl(v: int, r: int) -> int:
    r &= 63
    return ((v << r) | (v >> (64 - r))) & _M64 if r else v


def membership_digest(ids: Iterable[int]) -> tuple[int, int, int]:
    """(count, wrapping sum, xor of rotations) of P/tessa_capture.rs:281-293."""
    a = np.asarray(list(ids) if not isinstance(ids, np.ndarray) else ids, dtype=np.uint64)
    if a.size == 0:
        return 0, 0, 0
    with np.errstate(over="ignore"):
        m = a + np.uint64(0x9E3779B97F4A7C15)
        m = (m ^ (m >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        m = (m ^ (m >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        m = m ^ (m >> np.uint64(31))
        r = a & np.uint64(63)
        rot = np.where(r == 0, m, (m << r) | (m >> ((np.uint64(64) - r) & np.uint64(63))))
        s = int(np.sum(m, dtype=np.uint64))
    return int(a.size), s, int(np.bitwise_xor.reduce(rot))


def _write_digest(h: _Fnv1a64, digest) -> None:
    n, s, x = digest
    h.u64(n)
    h.u64(s)
    h.u64(x)


def priority_for_task(seed: int, task_hash: int) -> int:
    h = _Fnv1a64(b"SHEAR-TESSA-PRIORITY\0")
    h.u64(seed)
    h.u64(task_hash)
    return h.finish()


def assignment_task_hash(seed, depth, retry, r_h, padded_dim, member_ids, leader_ids) -> int:
    h = _Fnv1a64(b"SHEAR-TESSA-ASSIGNMENT\0")
    h.u64(seed)
    h.u32(depth)
    h.u32(retry)
    h.u32(r_h)
    h.u32(padded_dim)
    _write_digest(h, membership_digest(member_ids))
    h.u64(len(leader_ids))
    for lid in leader_ids:
        h.u32(int(lid))
    return h.finish()


def leaf_task_hash_from_digest(seed: int, k: int, padded_dim: int, digest) -> int:
    h = _Fnv1a64(b"SHEAR-TESSA-LEAF\0")
    h.u64(seed)
    h.u32(k)
    h.u32(padded_dim)
    _write_digest(h, digest)
    return h.finish()


def leaf_task_hash(seed, k, padded_dim, member_ids) -> int:
    return leaf_task_hash_from_digest(seed, k, padded_dim, membership_digest(member_ids))


def tessa_request_hash(seed: int, member_ids) -> int:
    h = _Fnv1a64(b"SHEAR-TESSA-REQUEST\0")
    h.u64(seed)
    _write_digest(h, membership_digest(member_ids))
    return h.finish()


# ---------------------------------------------------------------- bins

def assignment_row_bin(rows: int):
    if 256 <= rows <= 1024:
        return 0
    if 1025 <= rows <= 8192:
        return 1
    if rows >= 8193:
        return 2
    return None


def assignment_leader_bin(leaders: int):
    for b, hi in enumerate((16, 32, 64, 128)):
        if leaders <= hi:
            return b if leaders >= 1 else None
    return None


def leaf_size_bin(rows: int):
    if 256 <= rows <= 512:
        return 0
    if 513 <= rows <= 896:
        return 1
    if 897 <= rows <= 1280:
        return 2
    return None


# ---------------------------------------------------------------- records

@dataclasses.dataclass
class TessaAssignmentTask:
    task_hash: int
    priority: int
    depth: int
    retry: int
    r_h: int
    padded_dim: int
    member_ids: list
    leader_ids: list


@dataclasses.dataclass
class TessaLeafTask:
    task_hash: int
    priority: int
    k: int
    padded_dim: int
    member_ids: list


def make_tessa_assignment_task(seed, depth, retry, r_h, padded_dim, member_ids, leader_ids) -> TessaAssignmentTask:
    members = sorted(int(v) for v in member_ids)
    leaders = [int(v) for v in leader_ids]
    th = assignment_task_hash(seed, depth, retry, r_h, padded_dim, members, leaders)
    return TessaAssignmentTask(th, priority_for_task(seed, th), depth, retry, r_h, padded_dim, members, leaders)


def make_tessa_leaf_task(seed, k, padded_dim, member_ids) -> TessaLeafTask:
    members = sorted(int(v) for v in member_ids)
    th = leaf_task_hash(seed, k, padded_dim, members)
    return TessaLeafTask(th, priority_for_task(seed, th), k, padded_dim, members)


def _zeros_counts():
    return {
        "assignment_observed": [[0] * TESSA_ASSIGNMENT_LEADER_BINS for _ in range(TESSA_ASSIGNMENT_ROW_BINS)],
        "assignment_selected": [[0] * TESSA_ASSIGNMENT_LEADER_BINS for _ in range(TESSA_ASSIGNMENT_ROW_BINS)],
        "leaf_observed": [0] * TESSA_LEAF_SIZE_BINS,
        "leaf_selected": [0] * TESSA_LEAF_SIZE_BINS,
    }


@dataclasses.dataclass
class TessaCaptureSelection:
    assignment_tasks: list
    leaf_tasks: list
    bin_counts: dict


def _key(task):
    return (task.priority, task.task_hash)


class TessaCaptureSampler:
    """P/tessa_capture.rs:350-458: per bin, the tasks with the smallest
    (priority, task hash), at most TESSA_*_BIN_LIMIT; independent of the
    order tasks are observed in."""

    def __init__(self, seed: int):
        self.seed = seed
        self.assignment_bins = [[[] for _ in range(TESSA_ASSIGNMENT_LEADER_BINS)]
                                for _ in range(TESSA_ASSIGNMENT_ROW_BINS)]
        self.leaf_bins = [[] for _ in range(TESSA_LEAF_SIZE_BINS)]
        self.bin_counts = _zeros_counts()

    def observe_assignment(self, task: TessaAssignmentTask) -> bool:
        t = make_tessa_assignment_task(self.seed, task.depth, task.retry, task.r_h, task.padded_dim,
                                       task.member_ids, task.leader_ids)
        rb, lb = assignment_row_bin(len(t.member_ids)), assignment_leader_bin(len(t.leader_ids))
        if rb is None or lb is None:
            return False
        self.bin_counts["assignment_observed"][rb][lb] += 1
        return self._admit(self.assignment_bins[rb][lb], t, TESSA_ASSIGNMENT_BIN_LIMIT, "assignment")

    def observe_leaf(self, task: TessaLeafTask) -> bool:
        t = make_tessa_leaf_task(self.seed, task.k, task.padded_dim, task.member_ids)
        b = leaf_size_bin(len(t.member_ids))
        if b is None:
            return False
        self.bin_counts["leaf_observed"][b] += 1
        return self._admit(self.leaf_bins[b], t, TESSA_LEAF_BIN_LIMIT, "leaf")

    @staticmethod
    def _admit(bin_, t, limit, kind) -> bool:
        for existing in bin_:
            if existing.task_hash == t.task_hash:
                if existing != t:
                    raise CaptureError(f"{kind} task hash collision for {t.task_hash}")
                return False
        bin_.append(t)
        bin_.sort(key=_key)
        if len(bin_) > limit:
            bin_.pop()
        return True

    def observe_leaf_digests(self, k: int, padded_dim: int, sizes: Sequence[int], digests,
                             members_of: Callable[[int], Sequence[int]]) -> int:
        """Observe many leaf tasks from their membership digests ((count, sum,
        xor) per leaf, e.g. from the GPU); members_of(l) is called only for
        leaves that can enter their bin (or collide with a kept hash).  The
        result equals observe_leaf on every leaf.  Returns tasks kept."""
        kept = 0
        for l, n in enumerate(sizes):
            b = leaf_size_bin(int(n))
            if b is None:
                continue
            dg = tuple(int(v) for v in digests[l])
            th = leaf_task_hash_from_digest(self.seed, k, padded_dim, dg)
            pr = priority_for_task(self.seed, th)
            bin_ = self.leaf_bins[b]
            full = len(bin_) >= TESSA_LEAF_BIN_LIMIT
            if full and (pr, th) > _key(bin_[-1]) and all(e.task_hash != th for e in bin_):
                self.bin_counts["leaf_observed"][b] += 1  # would be pushed and popped at once
                continue
            self.bin_counts["leaf_observed"][b] += 1
            t = make_tessa_leaf_task(self.seed, k, padded_dim, members_of(l))
            if t.task_hash != th:
                raise CaptureError(f"leaf digest does not match the members of leaf {l}")
            kept += self._admit(bin_, t, TESSA_LEAF_BIN_LIMIT, "leaf")
        return kept

    def finish(self) -> TessaCaptureSelection:
        a, leaves = [], []
        for rb in range(TESSA_ASSIGNMENT_ROW_BINS):
            for lb in range(TESSA_ASSIGNMENT_LEADER_BINS):
                bin_ = sorted(self.assignment_bins[rb][lb], key=_key)
                self.bin_counts["assignment_selected"][rb][lb] = len(bin_)
                a.extend(bin_)
        for b in range(TESSA_LEAF_SIZE_BINS):
            bin_ = sorted(self.leaf_bins[b], key=_key)
            self.bin_counts["leaf_selected"][b] = len(bin_)
            leaves.extend(bin_)
        return TessaCaptureSelection(a, leaves, self.bin_counts)


# ---------------------------------------------------------------- JSON

def _dumps(obj) -> bytes:
    """serde_json::to_vec_pretty + b'\\n'."""
    return (json.dumps(obj, indent=2, ensure_ascii=False) + "\n").encode("utf-8")


def _task_json(t) -> dict:
    return dataclasses.asdict(t)


def _selection_json(sel: TessaCaptureSelection) -> dict:
    return {"assignment_tasks": [_task_json(t) for t in sel.assignment_tasks],
            "leaf_tasks": [_task_json(t) for t in sel.leaf_tasks],
            "bin_counts": sel.bin_counts}


def _selection_from_json(d) -> TessaCaptureSelection:
    return TessaCaptureSelection([TessaAssignmentTask(**t) for t in d["assignment_tasks"]],
                                 [TessaLeafTask(**t) for t in d["leaf_tasks"]], d["bin_counts"])


def write_tessa_capture_fragment(directory: str, request_hash: int, selection: TessaCaptureSelection) -> str:
    """P/tessa_capture.rs:460-519: fragment-<hash>.json, created once; an
    existing fragment must hold the same bytes."""
    os.makedirs(directory, exist_ok=True)
    data = _dumps({"version": TESSA_CAPTURE_VERSION, "request_hash": request_hash,
                   "selection": _selection_json(selection)})
    path = os.path.join(directory, f"fragment-{request_hash:016x}.json")
    try:
        fd = os.open(path, os.O_WRONLY | os.O_CREAT | os.O_EXCL, 0o644)
    except FileExistsError:
        with open(path, "rb") as f:
            if f.read() != data:
                raise CaptureError(f"existing TESSA fragment {path} differs from request {request_hash:016x}")
        return path
    with os.fdopen(fd, "wb") as f:
        f.write(data)
        f.flush()
        os.fsync(f.fileno())
    return path


def merge_tessa_capture_fragments(directory: str, seed: int) -> TessaCaptureSelection:
    """P/tessa_capture.rs:521-597."""
    try:
        names = sorted(n for n in os.listdir(directory) if n.startswith("fragment-") and n.endswith(".json"))
    except OSError as e:
        raise CaptureError(f"failed to read TESSA fragment directory {directory}: {e}")
    if not names:
        raise CaptureError(f"no TESSA capture fragments found in {directory}")
    sampler = TessaCaptureSampler(seed)
    observed = _zeros_counts()
    seen = set()
    for n in names:
        path = os.path.join(directory, n)
        with open(path, "rb") as f:
            frag = json.loads(f.read())
        if frag["version"] != TESSA_CAPTURE_VERSION:
            raise CaptureError(f"unsupported TESSA fragment version {frag['version']} in {path}")
        if frag["request_hash"] in seen:
            raise CaptureError(f"duplicate TESSA request hash {frag['request_hash']:016x}")
        seen.add(frag["request_hash"])
        bc = frag["selection"]["bin_counts"]
        for rb in range(TESSA_ASSIGNMENT_ROW_BINS):
            for lb in range(TESSA_ASSIGNMENT_LEADER_BINS):
                observed["assignment_observed"][rb][lb] += bc["assignment_observed"][rb][lb]
        for b in range(TESSA_LEAF_SIZE_BINS):
            observed["leaf_observed"][b] += bc["leaf_observed"][b]
        sel = _selection_from_json(frag["selection"])
        for t in sel.assignment_tasks:
            sampler.observe_assignment(t)
        for t in sel.leaf_tasks:
            sampler.observe_leaf(t)
    out = sampler.finish()
    out.bin_counts["assignment_observed"] = observed["assignment_observed"]
    out.bin_counts["leaf_observed"] = observed["leaf_observed"]
    return out


# ---------------------------------------------------------------- capture dir

def tessa_capture_dataset_metadata(path: str) -> dict:
    """P/tessa_capture.rs:62-93: canonical path, rows and dimension from the
    fbin header, SHA-256 of the 8 header bytes."""
    canonical = os.path.realpath(path)
    with open(canonical, "rb") as f:
        header = f.read(8)
    if len(header) != 8:
        raise CaptureError(f"failed to hash capture dataset header {canonical}")
    rows, dim = struct.unpack("<ii", header)
    meta = {"canonical_base_path": canonical, "rows": rows, "dimension": dim,
            "header_sha256": hashlib.sha256(header).hexdigest()}
    _validate_dataset(meta)
    return meta


def _is_sha256(v) -> bool:
    return isinstance(v, str) and len(v) == 64 and all(c in "0123456789abcdefABCDEF" for c in v)


def _validate_dataset(d) -> None:
    if (not d["canonical_base_path"] or not os.path.isabs(d["canonical_base_path"]) or d["rows"] == 0
            or d["dimension"] == 0 or not _is_sha256(d["header_sha256"])):
        raise CaptureError(f"invalid capture dataset metadata: path='{d['canonical_base_path']}' rows={d['rows']} "
                           f"dim={d['dimension']} header_sha256='{d['header_sha256']}'")


def _validate_provenance(p) -> None:
    if (not p["git_commit"] or not _is_sha256(p["binary_sha256"]) or not _is_sha256(p["command_sha256"])
            or p["root_leader_hash"] == 0 or p["d0_partition_hash"] == 0 or p["d0_task_list_hash"] == 0):
        raise CaptureError("invalid TESSA capture provenance")


def _validate_selection(sel: TessaCaptureSelection, seed: int, rows: int) -> None:
    """P/tessa_capture.rs:835-947."""
    hashes = set()
    sel_a = [[0] * TESSA_ASSIGNMENT_LEADER_BINS for _ in range(TESSA_ASSIGNMENT_ROW_BINS)]
    for t in sel.assignment_tasks:
        rb, lb = assignment_row_bin(len(t.member_ids)), assignment_leader_bin(len(t.leader_ids))
        if rb is None:
            raise CaptureError("assignment task is outside configured row bins")
        if lb is None:
            raise CaptureError("assignment task is outside configured leader bins")
        sel_a[rb][lb] += 1
        if sel_a[rb][lb] > TESSA_ASSIGNMENT_BIN_LIMIT:
            raise CaptureError(f"assignment capture bin ({rb}, {lb}) exceeds limit {TESSA_ASSIGNMENT_BIN_LIMIT}")
        _sorted(t.member_ids, "assignment members")
        _ids(t.member_ids, rows, "assignment member")
        _ids(t.leader_ids, rows, "assignment leader")
        if t.r_h == 0 or t.r_h > len(t.leader_ids):
            raise CaptureError(f"assignment task {t.task_hash} has invalid r_h {t.r_h} for {len(t.leader_ids)} leaders")
        if t.padded_dim == 0:
            raise CaptureError(f"assignment task {t.task_hash} has zero padded_dim")
        exp = assignment_task_hash(seed, t.depth, t.retry, t.r_h, t.padded_dim, t.member_ids, t.leader_ids)
        _hash_priority(t.task_hash, t.priority, exp, seed)
        if t.task_hash in hashes:
            raise CaptureError(f"duplicate TESSA task hash {t.task_hash}")
        hashes.add(t.task_hash)
    sel_l = [0] * TESSA_LEAF_SIZE_BINS
    for t in sel.leaf_tasks:
        b = leaf_size_bin(len(t.member_ids))
        if b is None:
            raise CaptureError("leaf task is outside configured size bins")
        sel_l[b] += 1
        if sel_l[b] > TESSA_LEAF_BIN_LIMIT:
            raise CaptureError(f"leaf capture bin {b} exceeds limit {TESSA_LEAF_BIN_LIMIT}")
        _sorted(t.member_ids, "leaf members")
        _ids(t.member_ids, rows, "leaf member")
        if t.k == 0 or t.k >= len(t.member_ids) or t.padded_dim == 0:
            raise CaptureError(f"leaf task {t.task_hash} has invalid k {t.k} or padded_dim {t.padded_dim} for "
                               f"{len(t.member_ids)} members")
        _hash_priority(t.task_hash, t.priority, leaf_task_hash(seed, t.k, t.padded_dim, t.member_ids), seed)
        if t.task_hash in hashes:
            raise CaptureError(f"duplicate TESSA task hash {t.task_hash}")
        hashes.add(t.task_hash)
    bc = sel.bin_counts
    if bc["assignment_selected"] != sel_a or bc["leaf_selected"] != sel_l:
        raise CaptureError("capture selected bin counts do not match task records")
    for rb in range(TESSA_ASSIGNMENT_ROW_BINS):
        for lb in range(TESSA_ASSIGNMENT_LEADER_BINS):
            if bc["assignment_observed"][rb][lb] < sel_a[rb][lb]:
                raise CaptureError("capture assignment observed count is smaller than selected count")
    for o, s in zip(bc["leaf_observed"], sel_l):
        if o < s:
            raise CaptureError("capture leaf observed count is smaller than selected count")


def _sorted(ids, label) -> None:
    if any(a > b for a, b in zip(ids, ids[1:])):
        raise CaptureError(f"{label} are not in canonical sorted order")


def _ids(ids, rows, label) -> None:
    for v in ids:
        if v >= rows:
            raise CaptureError(f"{label} id {v} is outside dataset rows {rows}")


def _hash_priority(task_hash, priority, expected, seed) -> None:
    if task_hash != expected or priority != priority_for_task(seed, expected):
        raise CaptureError(f"TESSA task hash or priority mismatch for task {task_hash}")


def _write_u32le(path: str, values) -> None:
    with open(path, "wb") as f:
        f.write(np.asarray(values, dtype="<u4").tobytes())


def _read_u32le(path: str) -> np.ndarray:
    with open(path, "rb") as f:
        data = f.read()
    if len(data) % 4:
        raise CaptureError(f"capture binary {path} has non-u32 byte length {len(data)}")
    return np.frombuffer(data, dtype="<u4")


def _assignment_sort_key(t):
    rb, lb = assignment_row_bin(len(t.member_ids)), assignment_leader_bin(len(t.leader_ids))
    big = 1 << 64
    return (big if rb is None else rb, big if lb is None else lb, t.priority, t.task_hash)


def _leaf_sort_key(t):
    b = leaf_size_bin(len(t.member_ids))
    return (1 << 64 if b is None else b, t.priority, t.task_hash)


def write_tessa_capture(directory: str, dataset: dict, provenance: dict, selection: TessaCaptureSelection) -> str:
    """P/tessa_capture.rs:599-687."""
    _validate_dataset(dataset)
    _validate_provenance(provenance)
    sel = TessaCaptureSelection(sorted(selection.assignment_tasks, key=_assignment_sort_key),
                                sorted(selection.leaf_tasks, key=_leaf_sort_key), selection.bin_counts)
    _validate_selection(sel, provenance["seed"], dataset["rows"])
    os.makedirs(directory, exist_ok=True)
    am, al, lm, a_meta, l_meta = [], [], [], [], []
    for t in sel.assignment_tasks:
        a_meta.append({"task_hash": t.task_hash, "priority": t.priority, "depth": t.depth, "retry": t.retry,
                       "r_h": t.r_h, "padded_dim": t.padded_dim, "member_offset": len(am),
                       "member_len": len(t.member_ids), "leader_offset": len(al), "leader_len": len(t.leader_ids)})
        am.extend(t.member_ids)
        al.extend(t.leader_ids)
    for t in sel.leaf_tasks:
        l_meta.append({"task_hash": t.task_hash, "priority": t.priority, "k": t.k, "padded_dim": t.padded_dim,
                       "member_offset": len(lm), "member_len": len(t.member_ids)})
        lm.extend(t.member_ids)
    files = {"assignment_members": TESSA_ASSIGNMENT_MEMBERS_FILE,
             "assignment_leaders": TESSA_ASSIGNMENT_LEADERS_FILE, "leaf_members": TESSA_LEAF_MEMBERS_FILE}
    _write_u32le(os.path.join(directory, files["assignment_members"]), am)
    _write_u32le(os.path.join(directory, files["assignment_leaders"]), al)
    _write_u32le(os.path.join(directory, files["leaf_members"]), lm)
    manifest = {"version": TESSA_CAPTURE_VERSION, "dataset": dataset, "provenance": provenance,
                "bin_counts": sel.bin_counts, "files": files, "assignment_tasks": a_meta, "leaf_tasks": l_meta}
    path = os.path.join(directory, TESSA_CAPTURE_MANIFEST_FILE)
    with open(path, "wb") as f:
        f.write(_dumps(manifest))
    return path


def _relative_name(name: str) -> None:
    if not name or os.path.isabs(name) or name in (".", "..") or "/" in name or "\\" in name:
        raise CaptureError(f"capture file name must be one relative path component: {name}")


def _exact_slice(values, offset, length, next_offset, label):
    if offset != next_offset:
        raise CaptureError(f"{label} metadata is not contiguous: expected offset {next_offset}, got {offset}")
    end = offset + length
    if end > len(values):
        raise CaptureError(f"{label} range [{offset}, {end}) exceeds {len(values)} words")
    return [int(v) for v in values[offset:end]], end


def load_tessa_capture(directory: str, expected_dataset: dict | None = None):
    """P/tessa_capture.rs:689-816: returns (manifest, assignment_tasks, leaf_tasks)."""
    path = os.path.join(directory, TESSA_CAPTURE_MANIFEST_FILE)
    try:
        with open(path, "rb") as f:
            manifest = json.loads(f.read())
    except (OSError, ValueError) as e:
        raise CaptureError(f"failed to read capture manifest {path}: {e}")
    if manifest.get("version") != TESSA_CAPTURE_VERSION:
        raise CaptureError(f"unsupported TESSA capture version {manifest.get('version')}")
    _validate_dataset(manifest["dataset"])
    _validate_provenance(manifest["provenance"])
    if expected_dataset is not None:
        _validate_dataset(expected_dataset)
        d, e = manifest["dataset"], expected_dataset
        if (d["rows"], d["dimension"], d["header_sha256"]) != (e["rows"], e["dimension"], e["header_sha256"]):
            raise CaptureError(
                f"capture dataset identity mismatch: captured rows={d['rows']} dim={d['dimension']} "
                f"header_sha256={d['header_sha256']}, expected rows={e['rows']} dim={e['dimension']} "
                f"header_sha256={e['header_sha256']}")
    files = manifest["files"]
    for key in ("assignment_members", "assignment_leaders", "leaf_members"):
        _relative_name(files[key])
    am = _read_u32le(os.path.join(directory, files["assignment_members"]))
    al = _read_u32le(os.path.join(directory, files["assignment_leaders"]))
    lm = _read_u32le(os.path.join(directory, files["leaf_members"]))
    a_tasks, mo, lo = [], 0, 0
    for m in manifest["assignment_tasks"]:
        members, mo = _exact_slice(am, m["member_offset"], m["member_len"], mo, "assignment members")
        leaders, lo = _exact_slice(al, m["leader_offset"], m["leader_len"], lo, "assignment leaders")
        a_tasks.append(TessaAssignmentTask(m["task_hash"], m["priority"], m["depth"], m["retry"], m["r_h"],
                                           m["padded_dim"], members, leaders))
    if mo != len(am) or lo != len(al):
        raise CaptureError(f"capture assignment binary lengths do not match metadata: members {mo} of {len(am)}, "
                           f"leaders {lo} of {len(al)}")
    l_tasks, fo = [], 0
    for m in manifest["leaf_tasks"]:
        members, fo = _exact_slice(lm, m["member_offset"], m["member_len"], fo, "leaf members")
        l_tasks.append(TessaLeafTask(m["task_hash"], m["priority"], m["k"], m["padded_dim"], members))
    if fo != len(lm):
        raise CaptureError(f"capture leaf binary length does not match metadata: {fo} of {len(lm)}")
    _validate_selection(TessaCaptureSelection(a_tasks, l_tasks, manifest["bin_counts"]),
                        manifest["provenance"]["seed"], manifest["dataset"]["rows"])
    return manifest, a_tasks, l_tasks


def capture_leaf_batch(sampler: TessaCaptureSampler, members, leaf_starts, leaf_sizes, k: int, padded_dim: int,
                       global_ids=None, ctx=None) -> int:
    """Offer every leaf of a device leaf batch (the leaf operator's layout:
    member local ids in leaf order, global id = global_ids[member]) to the
    sampler as a TessaLeafTask (k, padded_dim, member global ids).  Digests are
    computed on the GPU; a leaf's member list is copied to the host only if the
    task can enter its bin.  Returns the tasks kept."""
    from . import ops

    starts = np.ascontiguousarray(leaf_starts, np.uint64)
    sizes = np.ascontiguousarray(leaf_sizes, np.uint64)
    digests = ops.membership_digests(members, starts, sizes, global_ids=global_ids, ctx=ctx)

    def members_of(l):
        lo, n = int(starts[l]), int(sizes[l])
        local = members[lo:lo + n].long()
        ids = global_ids[local] if global_ids is not None else members[lo:lo + n]
        return ids.cpu().numpy().view(np.uint32)

    return sampler.observe_leaf_digests(k, padded_dim, [int(n) for n in sizes], digests, members_of)
