"""Seeded global-D0 staging inputs shared by the oracle pins and GPU parity tests."""
import functools

import numpy as np

TIE_EPS = np.float32(2e-5)


def reference_fixture_43857():
    """Inputs of cuda_backend_sq8_d0_wmma_matches_scalar_and_reference_for_dynamic_fanout
    (shear-core/src/algorithm/pipnn/compute_backend.rs:43857-43940): 13 rows x 32,
    35 leaders, leader 1 duplicates leader 0, row 0 equals leader 0, leader ids
    20000+j except ids[0] = 90000 and ids[1] = 100."""
    dim, rows, leaders = 32, 13, 35
    r = np.arange(rows)[:, None]
    a = np.arange(dim)[None, :]
    raw = ((((r * 17 + a * 5 + 3) % 29).astype(np.float32) - np.float32(14.0)) * np.float32(0.125))
    lj = np.arange(leaders)[:, None]
    lv = ((((lj * 11 + a * 7 + 1) % 31).astype(np.float32) - np.float32(15.0)) * np.float32(0.125))
    lv[1] = lv[0]
    raw[0] = lv[0]
    gids = (10_000 + np.arange(rows)).astype(np.uint32)
    lids = (20_000 + np.arange(leaders)).astype(np.uint32)
    lids[0] = 90_000
    lids[1] = 100
    return raw.astype(np.float32), gids, lids, lv.astype(np.float32)


def random_case(rows, dim, leaders, seed, *, normalize=True, near_dup_leaders=0):
    rng = np.random.default_rng(seed)
    raw = rng.standard_normal((rows, dim)).astype(np.float32)
    lv = rng.standard_normal((leaders, dim)).astype(np.float32)
    if near_dup_leaders:
        # groups of leaders within ~1e-4 of each other: SQ8 distances inside the eps window
        for j in range(1, min(near_dup_leaders, leaders)):
            lv[j] = lv[0] + rng.standard_normal(dim).astype(np.float32) * np.float32(1e-4)
    if normalize:
        raw /= np.linalg.norm(raw, axis=1, keepdims=True)
        lv /= np.linalg.norm(lv, axis=1, keepdims=True)
    gids = rng.permutation(rows * 4)[:rows].astype(np.uint32)
    lids = rng.permutation(rows * 4 + leaders * 4)[:leaders].astype(np.uint32)
    return raw, gids, lids, lv


def stable_distance_order(ld, lt, rd, rt):
    """P/mod.rs:417-428 (f32 subtraction, eps 2e-5, then ids; else total_cmp)."""
    if abs(np.float32(np.float32(ld) - np.float32(rd))) <= TIE_EPS:
        return int(lt > rt) - int(lt < rt)
    return int(ld > rd) - int(ld < rd)


def py_d0_sort(codes, scales, norms, lcodes, lscales, lnorms, lids, fanout):
    """Independent transliteration of quantize_sq8_and_assign_global_d0_reference's
    assignment loop (P/dco_sq_int8.rs:2037-2061): all candidates, sorted by
    stable_distance_order, first `fanout` leader indices."""
    rows = codes.shape[0]
    out = np.zeros((rows, fanout), np.uint32)
    for r in range(rows):
        cands = []
        for j in range(lcodes.shape[0]):
            dot = int(np.dot(codes[r].astype(np.int64), lcodes[j].astype(np.int64)))
            ss = np.float32(scales[r] * lscales[j])
            sd = np.float32(ss * np.float32(dot))
            d = np.float32(np.float32(norms[r] + lnorms[j]) + np.float32(np.float32(-2.0) * sd))
            if d <= 0:
                d = np.float32(0)
            cands.append((j, d))
        cands.sort(key=functools.cmp_to_key(
            lambda x, y: stable_distance_order(x[1], int(lids[x[0]]), y[1], int(lids[y[0]]))))
        out[r] = [j for j, _ in cands[:fanout]]
    return out
