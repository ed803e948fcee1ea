"""Device-tensor and host-buffer entry points over the C ABI.

Device forms take CUDA tensors (torch is used only for device memory and
streams) and run on the tensors' current stream.  Host forms take numpy arrays
and are the reference-facing calls: they copy in, run and copy out inside the
call, like the compute-backend trait method they replace
(``PiPNNComputeBackend::process_quantized_subtree_l2_compact_topk``,
shear-core/src/algorithm/pipnn/compute_backend.rs:3693-3884).

uint32 data (ids) travel in torch as int32 tensors with the same bit pattern;
``as_u32`` turns them back into numpy uint32.
"""
from __future__ import annotations

import ctypes
import threading

import numpy as np

from . import _capi as C

_tls = threading.local()


class Context:
    """One library context (one device, one host thread)."""

    def __init__(self, device: int = 0):
        lib = C.load()
        h = ctypes.c_void_p()
        C.check(lib.tessa_create(int(device), ctypes.byref(h)))
        self.handle = h
        self.device = int(device)

    def close(self) -> None:
        if self.handle:
            C.load().tessa_destroy(self.handle)
            self.handle = None

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass


def context(device: int = 0) -> Context:
    cache = getattr(_tls, "ctx", None)
    if cache is None:
        cache = _tls.ctx = {}
    if device not in cache:
        cache[device] = Context(device)
    return cache[device]


def _stream_ptr(torch, device):
    """torch's current stream as the C ABI's stream argument (its default
    stream is 0, which the C ABI reads as the legacy default stream)."""
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p()


def _np_ptr(a):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else ctypes.c_void_p()


def as_u32(t) -> np.ndarray:
    """int32 torch tensor (or numpy) holding uint32 bits -> numpy uint32."""
    a = t.detach().cpu().numpy() if hasattr(t, "detach") else np.asarray(t)
    return a.view(np.uint32)


def padded_dim(dim: int, k_align: int = 16) -> int:
    """P/dco_sq_int8.rs:1216-1224 sq_int8_padded_dim."""
    if dim <= 0:
        raise ValueError("SQ-int8 quantization requires dim > 0")
    k_align = max(1, int(k_align))
    return (dim + k_align - 1) // k_align * k_align


# ----------------------------------------------------------------- SQ8 quant

def quantize_sq8(x, k_align: int = 16, bits: int = 8, ctx: Context | None = None):
    """GPU quantize_sq_int8_matrix_with_bits (P/dco_sq_int8.rs:1331-1375).

    x: CUDA float32 tensor [rows, dim].  Returns (codes int8 [rows, padded],
    scales f32 [rows], norms f32 [rows]) on the same device, bit-exact with the
    reference CPU quantizer.
    """
    import torch

    if not x.is_cuda or x.dtype != torch.float32 or x.dim() != 2:
        raise ValueError("x must be a 2-D float32 CUDA tensor")
    x = x.contiguous()
    rows, dim = x.shape
    dev = x.device.index
    ctx = ctx or context(dev)
    pd = padded_dim(dim, k_align)
    codes = torch.empty((rows, pd), dtype=torch.int8, device=x.device)
    scales = torch.empty(rows, dtype=torch.float32, device=x.device)
    norms = torch.empty(rows, dtype=torch.float32, device=x.device)
    C.check(C.load().tessa_quantize_sq8(ctx.handle, _ptr(x), rows, dim, k_align, bits, _ptr(codes),
                                        _ptr(scales), _ptr(norms), _stream_ptr(torch, dev)))
    return codes, scales, norms


def quantize_sq8_host(x: np.ndarray, k_align: int = 16, bits: int = 8, device: int = 0):
    """Host-buffer form of :func:`quantize_sq8` (numpy in, numpy out)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, dim = x.shape
    pd = padded_dim(dim, k_align)
    codes = np.zeros((rows, pd), dtype=np.int8)
    scales = np.zeros(rows, dtype=np.float32)
    norms = np.zeros(rows, dtype=np.float32)
    C.check(C.load().tessa_quantize_sq8_host(context(device).handle, _np_ptr(x), rows, dim, k_align, bits,
                                             _np_ptr(codes), _np_ptr(scales), _np_ptr(norms)))
    return codes, scales, norms


# -------------------------------------------------------------- leaf top-k

def _layout(leaf_starts, leaf_sizes):
    starts = np.ascontiguousarray(leaf_starts, dtype=np.uint64)
    sizes = np.ascontiguousarray(leaf_sizes, dtype=np.uint64)
    if starts.shape != sizes.shape or starts.ndim != 1:
        raise ValueError("leaf_starts and leaf_sizes must be 1-D and of equal length")
    return starts, sizes


def leaf_topk_sq8(codes, scales, norms, global_ids, leaf_members, leaf_starts, leaf_sizes, k: int,
                  leaf_ordered_codes=None, out=None, ctx: Context | None = None):
    """Fused SQ8 leaf top-k on device tensors (see tessa_leaf_topk_sq8).

    codes int8 [resident_rows, padded_dim]; scales / norms f32 and global_ids
    int32(uint32 bits) [resident_rows]; leaf_members int32(uint32) [leaf_rows];
    leaf_starts / leaf_sizes host sequences.  Returns (ids int32-bits,
    dists f32), each [leaf_rows * k].
    """
    import torch

    starts, sizes = _layout(leaf_starts, leaf_sizes)
    dev = codes.device.index
    ctx = ctx or context(dev)
    leaf_rows = int(leaf_members.numel())
    if out is None:
        ids = torch.empty(leaf_rows * k, dtype=torch.int32, device=codes.device)
        dists = torch.empty(leaf_rows * k, dtype=torch.float32, device=codes.device)
    else:
        ids, dists = out
    a = C.LeafArgs(codes=codes.data_ptr(), scales=scales.data_ptr(), norms=norms.data_ptr(),
                   global_ids=global_ids.data_ptr(), resident_rows=codes.shape[0],
                   padded_dim=codes.shape[1], k=k, leaf_members=leaf_members.data_ptr(),
                   leaf_starts=starts.ctypes.data, leaf_sizes=sizes.ctypes.data,
                   leaf_count=starts.shape[0], leaf_rows=leaf_rows, topk_ids=ids.data_ptr(),
                   topk_dists=dists.data_ptr(),
                   leaf_ordered_codes=leaf_ordered_codes.data_ptr() if leaf_ordered_codes is not None else None)
    C.check(C.load().tessa_leaf_topk_sq8(ctx.handle, ctypes.byref(a), _stream_ptr(torch, dev)))
    return ids, dists


def leaf_topk_sq8_host(codes, scales, norms, global_ids, leaf_members, leaf_starts, leaf_sizes, k: int,
                       device: int = 0, out=None, batch_bytes: int | None = None):
    """Host-buffer form: numpy arrays in, numpy (ids uint32, dists f32) out.

    Pinned host arrays (e.g. ``torch.empty(..., pin_memory=True).numpy()``)
    make the copies inside the call run at full link speed.  With identity
    members and ordered, disjoint leaves the call pipelines upload, kernel and
    download in batches of ``batch_bytes`` bytes of codes (None keeps the
    context's setting; 0 restores the 128 MiB default).
    """
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    scales = np.ascontiguousarray(scales, dtype=np.float32)
    norms = np.ascontiguousarray(norms, dtype=np.float32)
    gids = np.ascontiguousarray(global_ids, dtype=np.uint32)
    members = np.ascontiguousarray(leaf_members, dtype=np.uint32)
    starts, sizes = _layout(leaf_starts, leaf_sizes)
    n = members.shape[0] * k
    if out is None:
        ids = np.empty(n, dtype=np.uint32)
        dists = np.empty(n, dtype=np.float32)
    else:
        ids, dists = out
    a = C.LeafArgs(codes=codes.ctypes.data, scales=scales.ctypes.data, norms=norms.ctypes.data,
                   global_ids=gids.ctypes.data, resident_rows=codes.shape[0], padded_dim=codes.shape[1],
                   k=k, leaf_members=members.ctypes.data, leaf_starts=starts.ctypes.data,
                   leaf_sizes=sizes.ctypes.data, leaf_count=starts.shape[0], leaf_rows=members.shape[0],
                   topk_ids=ids.ctypes.data, topk_dists=dists.ctypes.data, leaf_ordered_codes=None)
    if batch_bytes is not None:
        set_host_batch_bytes(batch_bytes, device=device)
    C.check(C.load().tessa_leaf_topk_sq8_host(context(device).handle, ctypes.byref(a)))
    return ids, dists


def set_host_batch_bytes(batch_bytes: int, ctx: Context | None = None, device: int = 0) -> None:
    """Bytes of codes per batch of the host-buffer pipeline (0 = default 128 MiB)."""
    ctx = ctx or context(device)
    C.check(C.load().tessa_set_host_batch_bytes(ctx.handle, int(batch_bytes)))


def set_leaf_kernel(mode: int, ctx: Context | None = None, device: int = 0) -> None:
    """tessa_set_leaf_kernel: 0 = column-split kernel on CTA pairs (default), 1 = one CTA per tile."""
    ctx = ctx or context(device)
    C.check(C.load().tessa_set_leaf_kernel(ctx.handle, int(mode)))


def leaf_last_fallback_rows(ctx: Context | None = None, device: int = 0) -> int:
    """Rows of the last leaf call on `ctx` recomputed by the exact sequential fallback."""
    ctx = ctx or context(device)
    n = ctypes.c_uint64()
    C.check(C.load().tessa_leaf_last_fallback_rows(ctx.handle, ctypes.byref(n)))
    return int(n.value)


# -------------------------------------------------------------- assignment

def assign(source: int, *, x=None, raw_norms=None, codes=None, scales=None, sq8_norms=None, global_ids,
           members, leaders, task_member_offsets, task_member_counts, task_leader_offsets,
           task_leader_counts, task_rh, task_output_offsets, output_len: int, ctx: Context | None = None):
    """Assignment replay (tessa_assign) on device tensors; task arrays are host sequences.

    source: ``ASSIGN_FP32`` (x, raw_norms) or ``ASSIGN_SQ8`` (codes, scales,
    sq8_norms).  Returns (ids int32-bits, dists f32) of output_len entries.
    """
    import torch

    dev = global_ids.device.index
    ctx = ctx or context(dev)
    u32 = lambda v: np.ascontiguousarray(v, dtype=np.uint32)
    moff, mcnt, loff, lcnt, rh = (u32(task_member_offsets), u32(task_member_counts),
                                  u32(task_leader_offsets), u32(task_leader_counts), u32(task_rh))
    outoff = np.ascontiguousarray(task_output_offsets, dtype=np.uint64)
    ids = torch.full((output_len,), -1, dtype=torch.int32, device=global_ids.device)
    dists = torch.full((output_len,), 3.402823466e38, dtype=torch.float32, device=global_ids.device)
    ref = x if x is not None else codes
    a = C.AssignArgs(x=_ptr(x).value, raw_norms=_ptr(raw_norms).value, codes=_ptr(codes).value,
                     scales=_ptr(scales).value, sq8_norms=_ptr(sq8_norms).value,
                     global_ids=global_ids.data_ptr(), resident_rows=ref.shape[0],
                     dim=x.shape[1] if x is not None else 0,
                     padded_dim=codes.shape[1] if codes is not None else 0,
                     members=members.data_ptr(), leaders=leaders.data_ptr(),
                     task_member_offsets=moff.ctypes.data, task_member_counts=mcnt.ctypes.data,
                     task_leader_offsets=loff.ctypes.data, task_leader_counts=lcnt.ctypes.data,
                     task_rh=rh.ctypes.data, task_output_offsets=outoff.ctypes.data,
                     task_count=moff.shape[0], member_rows=int(members.numel()),
                     out_ids=ids.data_ptr(), out_dists=dists.data_ptr())
    C.check(C.load().tessa_assign(ctx.handle, int(source), ctypes.byref(a), _stream_ptr(torch, dev)))
    return ids, dists


# ------------------------------------------------------------- global D0

class D0Result:
    """SqGpuD0QuantizeAssignResult (P/dco_sq_int8.rs:1929-2070): the SQ8 matrix
    of the batch and its D0 assignment fragments.

    codes [rows, padded_dim] int8, scales / norms [rows] f32, child_ids
    [rows, fanout] leader indices (best first), point_ids [rows, fanout]
    (the row's global id), dists [rows, fanout] SQ8 distances.
    """

    def __init__(self, codes, scales, norms, child_ids, point_ids, dists, dim):
        self.codes, self.scales, self.norms = codes, scales, norms
        self.child_ids, self.point_ids, self.dists = child_ids, point_ids, dists
        self.rows = int(codes.shape[0])
        self.dim = int(dim)
        self.padded_dim = int(codes.shape[1])

    def fragments(self):
        """[(child_id, point_id), ...] in the reference's order (row-major, best first)."""
        c = np.asarray(self.child_ids).reshape(-1)
        p = np.asarray(self.point_ids).reshape(-1)
        return list(zip(c.tolist(), p.tolist()))


def d0_last_profile(ctx: Context | None = None, device: int = 0) -> dict:
    """Event-timed phases of the context's last D0 call (SqGpuD0StagingProfile's device walls)."""
    ctx = ctx or context(device)
    p = C.D0Profile()
    C.check(C.load().tessa_d0_last_profile(ctx.handle, ctypes.byref(p)))
    return {n: getattr(p, n) for n, _ in C.D0Profile._fields_}


def _d0_leaders(leader_count, dim, leader_vectors, leader_payload):
    if leader_payload is None:
        if leader_vectors is None:
            raise ValueError("global D0 leaders need leader vectors or a leader payload")
        return leader_vectors, None, None, None
    codes, scales, norms = leader_payload
    pd = padded_dim(dim)
    if tuple(codes.shape) != (leader_count, pd) or scales.shape[0] != leader_count or norms.shape[0] != leader_count:
        raise ValueError(f"SQ GPU-D0 staging leader payload shape mismatch: codes {tuple(codes.shape)} "
                         f"expected ({leader_count}, {pd})")
    return None, codes, scales, norms


def quantize_sq8_and_assign_global_d0(raw_vectors, global_ids, global_d0_leader_ids, global_d0_leader_vectors,
                                      fanout_top: int, leader_payload=None, device: int = 0, out=None) -> D0Result:
    """Host form of the trait method quantize_sq8_and_assign_global_d0
    (compute_backend.rs:3828-3837; CUDA implementation :24281-24760; CPU
    reference P/dco_sq_int8.rs:1929-2070): numpy in, numpy out.

    raw_vectors [rows, dim] f32; global_ids [rows]; global_d0_leader_ids
    [leaders]; global_d0_leader_vectors [leaders, dim] f32 (ignored when
    leader_payload = (codes, scales, norms) is given).  out = (codes, scales,
    norms, child_ids, point_ids, dists) preallocated numpy arrays (e.g. pinned).
    """
    raw = np.ascontiguousarray(raw_vectors, dtype=np.float32)
    gids = np.ascontiguousarray(global_ids, dtype=np.uint32)
    lids = np.ascontiguousarray(global_d0_leader_ids, dtype=np.uint32)
    rows, leaders = gids.shape[0], lids.shape[0]
    if raw.ndim != 2:
        raw = raw.reshape(rows, -1) if rows else raw.reshape(0, 0)
    dim = raw.shape[1] if raw.ndim == 2 else 0
    if raw.shape[0] != rows:
        raise ValueError(f"SQ GPU-D0 staging raw vector shape mismatch: rows={rows} values={raw.size}")
    lv, lc, ls, ln = _d0_leaders(leaders, dim, global_d0_leader_vectors, leader_payload)
    if lv is not None:
        lv = np.ascontiguousarray(lv, dtype=np.float32)
        if lv.size != leaders * dim:
            raise ValueError(f"SQ GPU-D0 staging leader vector shape mismatch: leaders={leaders} dim={dim} "
                             f"values={lv.size}")
    else:
        lc = np.ascontiguousarray(lc, dtype=np.int8)
        ls = np.ascontiguousarray(ls, dtype=np.float32)
        ln = np.ascontiguousarray(ln, dtype=np.float32)
    f = int(fanout_top)
    pd = padded_dim(dim) if dim > 0 else 0
    n = rows * max(f, 0)
    if out is None:
        codes = np.zeros((rows, pd), dtype=np.int8)
        scales = np.zeros(rows, dtype=np.float32)
        norms = np.zeros(rows, dtype=np.float32)
        child = np.zeros(n, dtype=np.uint32)
        point = np.zeros(n, dtype=np.uint32)
        dists = np.zeros(n, dtype=np.float32)
    else:
        codes, scales, norms, child, point, dists = out
        if codes.size != rows * pd or scales.size != rows or norms.size != rows or child.size != n or \
                point.size != n or dists.size != n:
            raise ValueError("D0 output buffers have the wrong sizes")
        codes = codes.reshape(rows, pd)
    a = C.D0Args(raw_vectors=raw.ctypes.data, global_ids=gids.ctypes.data, rows=rows, dim=dim, fanout_top=f,
                 leader_ids=lids.ctypes.data, leader_vectors=_np_ptr(lv).value, leader_codes=_np_ptr(lc).value,
                 leader_scales=_np_ptr(ls).value, leader_norms=_np_ptr(ln).value, leader_count=leaders,
                 codes=codes.ctypes.data, scales=scales.ctypes.data, norms=norms.ctypes.data,
                 child_ids=child.ctypes.data, point_ids=point.ctypes.data, dists=dists.ctypes.data)
    C.check(C.load().tessa_quantize_sq8_assign_d0_host(context(device).handle, ctypes.byref(a)))
    shape = (rows, f)
    return D0Result(codes, scales, norms, child.reshape(shape), point.reshape(shape), dists.reshape(shape), dim)


def quantize_sq8_assign_d0(x, global_ids, leader_ids, fanout_top: int, leader_vectors=None, leader_payload=None,
                           ctx: Context | None = None, out=None) -> D0Result:
    """Device form: CUDA tensors in (x [rows, dim] f32, global_ids / leader_ids
    int32 bit patterns of uint32, leader_vectors [leaders, dim] f32 or
    leader_payload (codes, scales, norms)), CUDA tensors out, on the tensors'
    current stream.  out = (codes, scales, norms, child_ids, point_ids, dists)
    preallocated CUDA tensors."""
    import torch

    if not x.is_cuda or x.dtype != torch.float32 or x.dim() != 2:
        raise ValueError("x must be a 2-D float32 CUDA tensor")
    x = x.contiguous()
    rows, dim = x.shape
    dev = x.device.index
    ctx = ctx or context(dev)
    leaders = int(leader_ids.numel())
    lv, lc, ls, ln = _d0_leaders(leaders, dim, leader_vectors, leader_payload)
    f = int(fanout_top)
    pd = padded_dim(dim)
    n = rows * max(f, 0)
    if out is None:
        codes = torch.empty((rows, pd), dtype=torch.int8, device=x.device)
        scales = torch.empty(rows, dtype=torch.float32, device=x.device)
        norms = torch.empty(rows, dtype=torch.float32, device=x.device)
        child = torch.empty(n, dtype=torch.int32, device=x.device)
        point = torch.empty(n, dtype=torch.int32, device=x.device)
        dists = torch.empty(n, dtype=torch.float32, device=x.device)
    else:
        codes, scales, norms, child, point, dists = out
        if codes.numel() != rows * pd or scales.numel() != rows or norms.numel() != rows or \
                child.numel() != n or point.numel() != n or dists.numel() != n:
            raise ValueError("D0 output tensors have the wrong sizes")
        if not all(t.is_contiguous() and t.is_cuda for t in out):
            raise ValueError("D0 output tensors must be contiguous CUDA tensors")
        codes = codes.view(rows, pd)
    c = lambda t: t.contiguous() if t is not None else None
    lv, lc, ls, ln = c(lv), c(lc), c(ls), c(ln)
    gid = global_ids.contiguous()
    lid = leader_ids.contiguous()
    a = C.D0Args(raw_vectors=x.data_ptr(), global_ids=gid.data_ptr(), rows=rows, dim=dim, fanout_top=f,
                 leader_ids=lid.data_ptr(), leader_vectors=_ptr(lv).value, leader_codes=_ptr(lc).value,
                 leader_scales=_ptr(ls).value, leader_norms=_ptr(ln).value, leader_count=leaders,
                 codes=codes.data_ptr(), scales=scales.data_ptr(), norms=norms.data_ptr(),
                 child_ids=child.data_ptr(), point_ids=point.data_ptr(), dists=dists.data_ptr())
    C.check(C.load().tessa_quantize_sq8_assign_d0(ctx.handle, ctypes.byref(a), _stream_ptr(torch, dev)))
    shape = (rows, f)
    return D0Result(codes, scales, norms, child.view(shape), point.view(shape), dists.view(shape), dim)


# ------------------------------------------------------- candidate edges

def sketch_rows(x, hyperplanes, ctx: Context | None = None, out=None):
    """Per-point sketches (fill_sketch_row, hash_prune.rs:2208-2232) on the GPU.

    x: CUDA f32 [rows, dim]; hyperplanes: CUDA f32 [m, dim] (m <= 16).
    Returns CUDA f32 [rows, m], bit-exact with the reference's sequential sums.
    """
    import torch

    x = x.contiguous()
    planes = hyperplanes.contiguous()
    rows, dim = x.shape
    m = planes.shape[0]
    ctx = ctx or context(x.device.index)
    if out is None:
        out = torch.empty((rows, m), dtype=torch.float32, device=x.device)
    C.check(C.load().tessa_sketch_rows(ctx.handle, _ptr(x), rows, dim, _ptr(planes), m, _ptr(out),
                                       _stream_ptr(torch, x.device.index)))
    return out


def edge_hashes(point_ids, topk_ids, k: int, sketches, m_bits: int, leaf_starts=None, leaf_sizes=None,
                ctx: Context | None = None, out=None):
    """Forward / reverse hashes of every leaf slot (int32-bit CUDA tensors in,
    (hash_fwd, hash_rev) int16-bit CUDA tensors of rows * k out).  Sketch rows
    are indexed by global point id.  With the leaf layout (host sequences)
    each leaf's sketches are staged once in shared memory and candidates must
    be members of their leaf."""
    import torch

    rows = int(point_ids.numel())
    ctx = ctx or context(point_ids.device.index)
    if out is None:
        out = (torch.empty(rows * k, dtype=torch.int16, device=point_ids.device),
               torch.empty(rows * k, dtype=torch.int16, device=point_ids.device))
    sk = sketches.contiguous()
    if leaf_starts is None:
        starts = sizes = np.zeros(0, np.uint64)
    else:
        starts, sizes = _layout(leaf_starts, leaf_sizes)
    C.check(C.load().tessa_edge_hashes(ctx.handle, _ptr(point_ids.contiguous()), _ptr(topk_ids.contiguous()), rows, k,
                                       _np_ptr(starts), _np_ptr(sizes), starts.shape[0], _ptr(sk), sk.shape[0],
                                       sk.shape[1], m_bits, _ptr(out[0]), _ptr(out[1]),
                                       _stream_ptr(torch, point_ids.device.index)))
    return out


def expand_edges(point_ids, topk_ids, topk_dists, hash_fwd, hash_rev, k: int, threads: int = 0):
    """Host edge expansion in the reference's order (numpy in / out):
    returns (p uint32, c uint32, hash uint16, dist f32)."""
    import os
    pid = np.ascontiguousarray(point_ids, np.uint32)
    ids = np.ascontiguousarray(topk_ids).view(np.uint32).reshape(-1)
    ds = np.ascontiguousarray(topk_dists, np.float32).reshape(-1)
    hf = np.ascontiguousarray(hash_fwd).view(np.uint16).reshape(-1)
    hr = np.ascontiguousarray(hash_rev).view(np.uint16).reshape(-1)
    rows = pid.shape[0]
    if ids.shape[0] != rows * k or ds.shape[0] != rows * k or hf.shape[0] != rows * k or hr.shape[0] != rows * k:
        raise ValueError("edge inputs must hold rows * k slots")
    threads = threads or min(32, os.cpu_count() or 1)
    n = ctypes.c_uint64()
    lib = C.load()
    args = (_np_ptr(pid), _np_ptr(ids), _np_ptr(ds), _np_ptr(hf), _np_ptr(hr), rows, k, threads)
    C.check(lib.tessa_expand_edges(*args, None, None, None, None, 0, ctypes.byref(n)))
    p, c = np.empty(n.value, np.uint32), np.empty(n.value, np.uint32)
    h, d = np.empty(n.value, np.uint16), np.empty(n.value, np.float32)
    C.check(lib.tessa_expand_edges(*args, _np_ptr(p), _np_ptr(c), _np_ptr(h), _np_ptr(d), n.value, ctypes.byref(n)))
    return p, c, h, d


# ---------------------------------------------------------------- capture

def membership_digests(ids, leaf_starts, leaf_sizes, global_ids=None, ctx: Context | None = None):
    """Per-leaf (count, sum, xor) membership digests of device member arrays
    (int32-bit CUDA tensors; member id = global_ids[ids[i]] when given) ->
    numpy uint64 [leaves, 3], the input of TessaCaptureSampler.observe_leaf_digests."""
    import torch

    starts, sizes = _layout(leaf_starts, leaf_sizes)
    ctx = ctx or context(ids.device.index)
    n = starts.shape[0]
    out = torch.empty((2, max(n, 1)), dtype=torch.int64, device=ids.device)
    gid = global_ids.contiguous() if global_ids is not None else None
    C.check(C.load().tessa_membership_digests(ctx.handle, _ptr(ids.contiguous()), _ptr(gid), _np_ptr(starts),
                                              _np_ptr(sizes), n, _ptr(out[0]), _ptr(out[1]),
                                              _stream_ptr(torch, ids.device.index)))
    d = out[:, :n].cpu().numpy().view(np.uint64)
    return np.stack([sizes.astype(np.uint64), d[0], d[1]], axis=1)


# -------------------------------------------------------- subtree partition

class SubtreeParams:
    """Persistent-subtree plan values (CB:1309-1340 with the PiPNNParams
    defaults of P/params.rs:3342-3368): leaf_max = max(256, c_max), leaf_min 64,
    max_depth 10, max_leaders min(1000, 128), fanout_second 3, root_depth 1
    (D1+ tasks), small_node_limit 4096, psamp_fraction 0.001."""

    def __init__(self, c_max=2048, leaf_min=64, max_depth=10, max_leaders=1000, fanout_second=3, root_depth=1,
                 small_node_limit=4096, psamp_fraction=0.001):
        self.leaf_max = max(256, int(c_max))
        self.leaf_min = int(leaf_min)
        self.max_depth = int(max_depth)
        self.max_leaders = min(int(max_leaders), 128)
        self.fanout_second = int(fanout_second)
        self.root_depth = int(root_depth)
        self.small_node_limit = int(small_node_limit)
        self.psamp_fraction = float(psamp_fraction)

    def as_array(self):
        return np.array([self.leaf_max, self.leaf_min, self.max_depth, self.max_leaders, self.fanout_second,
                         self.root_depth, self.small_node_limit], np.uint32)


def subtree_leaf_capacity(member_rows: int, params: SubtreeParams | None = None) -> int:
    """Rows of the leaf arena subtree_partition allocates for member_rows task rows."""
    prm = params or SubtreeParams()
    return max(prm.fanout_second, 1) * int(member_rows) + 16


def _leaf_codes_ptr(leaf_codes, cap: int, codes):
    if leaf_codes is None:
        return None
    if not leaf_codes.is_cuda or leaf_codes.dtype != codes.dtype or not leaf_codes.is_contiguous() or \
            leaf_codes.numel() < cap * codes.shape[1]:
        raise ValueError(f"leaf_codes must be a contiguous int8 CUDA tensor of at least {cap} x {codes.shape[1]}")
    return leaf_codes.data_ptr()


def subtree_root_seed(random_seed: int, depth: int, rows: int, parent_points: int, min_recurse_size: int) -> int:
    """gpu_queue_root_seed (CB:1597-1603)."""
    def rotl(v, r):
        v &= (1 << 64) - 1
        return ((v << r) | (v >> (64 - r))) & ((1 << 64) - 1)
    return (random_seed ^ ((depth * 0x9E3779B97F4A7C15) & ((1 << 64) - 1)) ^ rotl(rows, 17)
            ^ rotl(parent_points, 7) ^ rotl(min_recurse_size, 29)) & ((1 << 64) - 1)


def subtree_partition(codes, scales, norms, task_members, task_offsets, task_counts, task_seeds,
                      params: SubtreeParams | None = None, ctx: Context | None = None, leaf_codes=None):
    """tessa_subtree_partition on device tensors (codes/scales/norms/task_members);
    task arrays are host sequences.  Returns (leaf_rows device int32 tensor of the
    used extent, leaf_starts u64, leaf_sizes u32, leaf_tasks u32, stats dict)."""
    import torch

    prm = params or SubtreeParams()
    dev = codes.device.index
    ctx = ctx or context(dev)
    toff = np.ascontiguousarray(task_offsets, np.uint64)
    tcnt = np.ascontiguousarray(task_counts, np.uint32)
    tseed = np.ascontiguousarray(task_seeds, np.uint64)
    member_rows = int(task_members.numel())
    # every task row lands in at most fanout_second leaves (replication only at the subtree root)
    cap = subtree_leaf_capacity(int(tcnt.astype(np.uint64).sum()), prm)
    leaf_rows = torch.empty(cap, dtype=torch.int32, device=codes.device)
    starts = np.zeros(cap, np.uint64)
    sizes = np.zeros(cap, np.uint32)
    tasks = np.zeros(cap, np.uint32)
    a = C.SubtreeArgs(codes=codes.data_ptr(), scales=scales.data_ptr(), sq8_norms=norms.data_ptr(),
                      resident_rows=codes.shape[0], padded_dim=codes.shape[1], task_members=task_members.data_ptr(),
                      member_rows=member_rows, task_offsets=toff.ctypes.data, task_counts=tcnt.ctypes.data,
                      task_seeds=tseed.ctypes.data, task_count=tcnt.size, leaf_max=prm.leaf_max,
                      leaf_min=prm.leaf_min, max_depth=prm.max_depth, max_leaders=prm.max_leaders,
                      fanout_second=prm.fanout_second, root_depth=prm.root_depth,
                      small_node_limit=prm.small_node_limit, psamp_fraction=prm.psamp_fraction,
                      leaf_rows=leaf_rows.data_ptr(), leaf_rows_capacity=cap, leaf_starts=starts.ctypes.data,
                      leaf_sizes=sizes.ctypes.data, leaf_tasks=tasks.ctypes.data, leaf_capacity=cap,
                      leaf_codes=_leaf_codes_ptr(leaf_codes, cap, codes))
    r = C.SubtreeResult()
    C.check(C.load().tessa_subtree_partition(ctx.handle, ctypes.byref(a), ctypes.byref(r), _stream_ptr(torch, dev)))
    n = int(r.leaf_count)
    stats = {f: int(getattr(r, f)) for f in ("rounds", "large_assignments", "retries", "balanced", "small_nodes",
                                             "leaf_rows_used", "kernel_launches")}
    stats.update({f: round(float(getattr(r, f)), 3) for f in ("assign_ms", "scatter_ms", "small_ms", "wall_ms",
                                                          "host_prep_ms", "host_decide_ms", "sync_wait_ms")})
    return leaf_rows[:int(r.leaf_rows_used)], starts[:n].copy(), sizes[:n].copy(), tasks[:n].copy(), stats


# ------------------------------------------------------ subtree submissions

_SUBMITTED: dict = {}  # (context handle, ticket) -> the device tensors the submission reads


def subtree_submit(codes, scales, norms, global_ids, task_members, task_offsets, task_counts, task_seeds, k: int,
                   params: SubtreeParams | None = None, ctx: Context | None = None) -> int:
    """tessa_subtree_submit: partition + leaf top-k of a batch of subtree tasks,
    queued on the context's submission worker.  Returns the ticket; the device
    tensors are kept alive here until the ticket is polled."""
    import torch

    prm = params or SubtreeParams()
    dev = codes.device.index
    ctx = ctx or context(dev)
    toff = np.ascontiguousarray(task_offsets, np.uint64)
    tcnt = np.ascontiguousarray(task_counts, np.uint32)
    tseed = np.ascontiguousarray(task_seeds, np.uint64)
    a = C.SubtreeArgs(codes=codes.data_ptr(), scales=scales.data_ptr(), sq8_norms=norms.data_ptr(),
                      resident_rows=codes.shape[0], padded_dim=codes.shape[1], task_members=task_members.data_ptr(),
                      member_rows=int(task_members.numel()), task_offsets=toff.ctypes.data,
                      task_counts=tcnt.ctypes.data, task_seeds=tseed.ctypes.data, task_count=tcnt.size,
                      leaf_max=prm.leaf_max, leaf_min=prm.leaf_min, max_depth=prm.max_depth,
                      max_leaders=prm.max_leaders, fanout_second=prm.fanout_second, root_depth=prm.root_depth,
                      small_node_limit=prm.small_node_limit, psamp_fraction=prm.psamp_fraction)
    req = C.SubtreeRequest(partition=a, global_ids=global_ids.data_ptr(), k=int(k))
    ticket = ctypes.c_uint64()
    C.check(C.load().tessa_subtree_submit(ctx.handle, ctypes.byref(req), ctypes.byref(ticket),
                                          _stream_ptr(torch, dev)))
    _SUBMITTED[(ctx.handle.value, ticket.value)] = (codes, scales, norms, global_ids, task_members)
    return int(ticket.value)


def subtree_poll(ticket: int, wait: bool = True, ctx: Context | None = None, device: int = 0):
    """tessa_subtree_poll: None while the submission runs (wait=False), else a
    dict of the CompactTopKBatch as numpy views of the slot's pinned memory
    (valid until subtree_release) plus the partition stats."""
    ctx = ctx or context(device)
    v = C.CompactView()
    rc = C.load().tessa_subtree_poll(ctx.handle, int(ticket), 1 if wait else 0, ctypes.byref(v))
    if rc == -11 and not wait:
        return None
    _SUBMITTED.pop((ctx.handle.value, int(ticket)), None)
    C.check(rc)
    rows, k, nl = int(v.rows), int(v.k), int(v.leaf_count)

    def arr(ptr, n, ct, dt):
        if n == 0 or not ptr:
            return np.zeros(0, dt)
        return np.ctypeslib.as_array(ctypes.cast(ptr, ctypes.POINTER(ct)), shape=(n,)).view(dt)
    stats = {f: getattr(v.partition, f) for f, _ in C.SubtreeResult._fields_}
    return dict(ticket=int(v.ticket), rows=rows, k=k, leaf_starts=arr(v.leaf_starts, nl, ctypes.c_uint64, np.uint64),
                leaf_sizes=arr(v.leaf_sizes, nl, ctypes.c_uint32, np.uint32),
                leaf_tasks=arr(v.leaf_tasks, nl, ctypes.c_uint32, np.uint32),
                point_ids=arr(v.point_ids, rows, ctypes.c_uint32, np.uint32),
                topk_ids=arr(v.topk_ids, rows * k, ctypes.c_uint32, np.uint32),
                topk_dists=arr(v.topk_dists, rows * k, ctypes.c_float, np.float32),
                partition=stats, fallback_rows=int(v.fallback_rows))


def subtree_release(ticket: int, ctx: Context | None = None, device: int = 0) -> None:
    ctx = ctx or context(device)
    C.check(C.load().tessa_subtree_release(ctx.handle, int(ticket)))


# ---------------------------------------------------------- host reduction

class Reducer:
    """HashPrune reservoirs on the host (tessa_reducer_*): add leaf batches
    (numpy arrays), then finish() -> CSR (offsets u64 [n+1], neighbors u32)."""

    def __init__(self, num_points: int, l_max: int = 64, threads: int = 0):
        import os
        self.handle = ctypes.c_void_p()
        self.lib = C.load()
        threads = threads or min(64, os.cpu_count() or 1)
        C.check(self.lib.tessa_reducer_create(num_points, l_max, threads, ctypes.byref(self.handle)))
        self.num_points = num_points

    def add(self, point_ids, topk_ids, topk_dists, hash_fwd, hash_rev, k: int):
        pid = np.ascontiguousarray(point_ids).view(np.uint32).reshape(-1)
        ids = np.ascontiguousarray(topk_ids).view(np.uint32).reshape(-1)
        ds = np.ascontiguousarray(topk_dists, np.float32).reshape(-1)
        hf = np.ascontiguousarray(hash_fwd).view(np.uint16).reshape(-1)
        hr = np.ascontiguousarray(hash_rev).view(np.uint16).reshape(-1)
        rows = pid.shape[0]
        if ids.shape[0] != rows * k or ds.shape[0] != rows * k or hf.shape[0] != rows * k or hr.shape[0] != rows * k:
            raise ValueError("reducer inputs must hold rows * k slots")
        C.check(self.lib.tessa_reducer_add(self.handle, _np_ptr(pid), _np_ptr(ids), _np_ptr(ds), _np_ptr(hf),
                                           _np_ptr(hr), rows, k))

    def add_grouped(self, offsets, edges):
        """Edges grouped by reservoir (host copies of group_edges' outputs:
        offsets uint64 [n+1], edges as the 12-byte tessa_edge records)."""
        off = np.ascontiguousarray(offsets, np.uint64)
        e = np.ascontiguousarray(edges)
        if off.shape[0] != self.num_points + 1:
            raise ValueError("offsets must hold num_points + 1 entries")
        C.check(self.lib.tessa_reducer_add_grouped(self.handle, _np_ptr(off), _np_ptr(e)))

    def edges(self) -> int:
        n = ctypes.c_uint64()
        C.check(self.lib.tessa_reducer_edges(self.handle, ctypes.byref(n)))
        return int(n.value)

    def finish(self):
        offsets = np.zeros(self.num_points + 1, np.uint64)
        n = ctypes.c_uint64()
        C.check(self.lib.tessa_reducer_finish(self.handle, _np_ptr(offsets), None, 0, ctypes.byref(n)))
        nb = np.zeros(max(int(n.value), 1), np.uint32)
        C.check(self.lib.tessa_reducer_finish(self.handle, _np_ptr(offsets), _np_ptr(nb), nb.shape[0],
                                              ctypes.byref(n)))
        return offsets, nb[:int(n.value)]

    def close(self):
        if self.handle:
            self.lib.tessa_reducer_destroy(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass


EDGE_DTYPE = np.dtype([("target", "<u4"), ("dist", "<f4"), ("hash", "<u2"), ("reserved", "<u2")])


def group_edges(point_ids, topk_ids, topk_dists, hash_fwd, hash_rev, k: int, num_points: int,
                ctx: Context | None = None, out=None):
    """tessa_group_edges on device tensors: (offsets int64 [n+1], edges uint8 [cap * 12])
    CUDA tensors; point p's edges are edges[offsets[p]:offsets[p+1]] (tessa_edge records)."""
    import torch

    rows = int(point_ids.numel())
    dev = point_ids.device
    ctx = ctx or context(dev.index)
    cap = 2 * rows * k
    if out is None:
        offsets = torch.empty(num_points + 1, dtype=torch.int64, device=dev)
        edges = torch.empty(max(cap, 1) * 12, dtype=torch.uint8, device=dev)
    else:
        offsets, edges = out
    C.check(C.load().tessa_group_edges(ctx.handle, _ptr(point_ids), _ptr(topk_ids), _ptr(topk_dists),
                                       _ptr(hash_fwd), _ptr(hash_rev), rows, k, num_points, _ptr(offsets),
                                       _ptr(edges), cap, _stream_ptr(torch, dev.index)))
    return offsets, edges


def _reduce_outputs(torch, dev, num_points, cap, neighbors, slots, out):
    if out is not None:
        return out
    offsets = torch.empty(num_points + 1, dtype=torch.int64, device=dev)
    nb = torch.empty(max(cap, 1), dtype=torch.int32, device=dev) if neighbors else None
    sl = torch.empty(max(cap, 1) * 12, dtype=torch.uint8, device=dev) if slots else None
    return offsets, nb, sl


def reduce_records(point_ids, topk_ids, topk_dists, hash_fwd, hash_rev, k: int, num_points: int, l_max: int,
                   ctx: Context | None = None, neighbors: bool = True, slots: bool = False, out=None):
    """tessa_reduce_records: HashPrune reservoirs of leaf records on the device.

    Returns (offsets int64 [n+1], neighbors int32 [cap] or None, slots uint8
    [cap * 12] (tessa_edge) or None, slot_count); point p's slots are
    [offsets[p], offsets[p+1]), in hash order."""
    import torch

    rows = int(point_ids.numel())
    dev = point_ids.device
    ctx = ctx or context(dev.index)
    cap = min(2 * rows * k, num_points * l_max)
    offsets, nb, sl = _reduce_outputs(torch, dev, num_points, cap, neighbors, slots, out)
    if out is not None:
        cap = min(nb.numel() if nb is not None else cap, sl.numel() // 12 if sl is not None else cap)
    count = ctypes.c_uint64()
    C.check(C.load().tessa_reduce_records(ctx.handle, _ptr(point_ids), _ptr(topk_ids), _ptr(topk_dists),
                                          _ptr(hash_fwd), _ptr(hash_rev), rows, k, num_points, l_max, _ptr(offsets),
                                          _ptr(nb) if nb is not None else None,
                                          _ptr(sl) if sl is not None else None, cap, ctypes.byref(count),
                                          _stream_ptr(torch, dev.index)))
    return offsets, nb, sl, int(count.value)


def reduce_grouped(pieces, num_points: int, l_max: int, ctx: Context | None = None, neighbors: bool = True,
                   slots: bool = False, out=None):
    """tessa_reduce_grouped: merge edges grouped by source -- `pieces` is a
    list of (offsets int64 [n+1] CUDA tensor, edges uint8 CUDA tensor of
    tessa_edge records, edge count) -- into reservoirs on the device.  Same
    returns as reduce_records."""
    import torch

    dev = pieces[0][0].device
    ctx = ctx or context(dev.index)
    g = len(pieces)
    offs = (ctypes.c_void_p * g)(*[p[0].data_ptr() for p in pieces])
    eds = (ctypes.c_void_p * g)(*[p[1].data_ptr() if int(p[2]) else None for p in pieces])
    cnt = (ctypes.c_uint64 * g)(*[int(p[2]) for p in pieces])
    m = sum(int(p[2]) for p in pieces)
    cap = min(m, num_points * l_max)
    offsets, nb, sl = _reduce_outputs(torch, dev, num_points, cap, neighbors, slots, out)
    if out is not None:
        cap = min(nb.numel() if nb is not None else cap, sl.numel() // 12 if sl is not None else cap)
    count = ctypes.c_uint64()
    C.check(C.load().tessa_reduce_grouped(ctx.handle, g, offs, eds, cnt, num_points, l_max, _ptr(offsets),
                                          _ptr(nb) if nb is not None else None,
                                          _ptr(sl) if sl is not None else None, cap, ctypes.byref(count),
                                          _stream_ptr(torch, dev.index)))
    return offsets, nb, sl, int(count.value)
