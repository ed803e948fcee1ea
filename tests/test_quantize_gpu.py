"""GPU SQ8 quantizer vs the reference CPU quantizer restatement (bit-exact)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,dim", [(2, 3), (257, 100), (1000, 768), (64, 1024), (400_000, 8), (3, 2000),
                                      (1001, 4), (77, 12), (50_000, 768), (300, 4096), (33, 36),
                                      # enough rows that every CTA reuses its buffers (3, 4, 6 and 8 of them)
                                      (40_000, 1024), (3_000, 4096), (30_000, 2000), (200_000, 128),
                                      (100_000, 100), (60_000, 512)])
def test_quantize_matches_cpu_bits(oracle, rows, dim):
    import torch
    from shear_b200 import ops
    rng = np.random.default_rng(rows + dim)
    x = (rng.standard_normal((rows, dim)) * rng.uniform(0.01, 100, (rows, 1))).astype(np.float32)
    x[0] = 0.0
    codes, scales, norms = ops.quantize_sq8(torch.from_numpy(x).cuda())
    wc, ws, wn = oracle.quantize_sq8(x)
    assert np.array_equal(codes.cpu().numpy(), wc)
    assert np.array_equal(scales.cpu().numpy().view(np.uint32), ws.view(np.uint32))
    assert np.array_equal(norms.cpu().numpy().view(np.uint32), wn.view(np.uint32))


@pytest.mark.parametrize("k_align", [1, 3, 16])
def test_quantize_k_align_and_unaligned_base(oracle, k_align):
    # odd paddings (byte stores) and an x base that is not 16-byte aligned
    # (the row-streaming path needs aligned rows; the other path takes it)
    import torch
    from shear_b200 import ops
    rng = np.random.default_rng(k_align)
    x = rng.standard_normal((500, 64)).astype(np.float32)
    t = torch.from_numpy(x).cuda()
    codes, scales, norms = ops.quantize_sq8(t, k_align=k_align)
    wc, ws, wn = oracle.quantize_sq8(x, k_align=k_align)
    assert np.array_equal(codes.cpu().numpy(), wc)
    assert np.array_equal(norms.cpu().numpy().view(np.uint32), wn.view(np.uint32))
    big = torch.from_numpy(rng.standard_normal(500 * 64 + 1).astype(np.float32)).cuda()
    off = big[1:].view(500, 64)  # 4-byte offset: not 16-byte aligned
    codes2, _, norms2 = ops.quantize_sq8(off, k_align=k_align)
    wc2, _, wn2 = oracle.quantize_sq8(big[1:].cpu().numpy().reshape(500, 64), k_align=k_align)
    assert np.array_equal(codes2.cpu().numpy(), wc2)
    assert np.array_equal(norms2.cpu().numpy().view(np.uint32), wn2.view(np.uint32))


def test_quantize_half_integer_boundaries_and_tiny_scales(oracle):
    # Elements whose quotient x / scale sits on or within a few ulps of a
    # half-integer (where rounding the quotient first matters), rows whose
    # scale is subnormal, and rows of mixed magnitude.
    import torch
    from shear_b200 import ops
    rng = np.random.default_rng(11)
    rows, dim = 4096, 128
    x = np.zeros((rows, dim), np.float32)
    for r in range(rows):
        mx = np.float32(rng.choice([1.0, 0.37, 3.0e-3, 1.0e5, 7.7e-37, 2.0e-38, 1.5e-39]))
        sc = np.float32(mx / np.float32(127.0))
        k = rng.integers(-127, 127, dim - 1).astype(np.float32)
        v = ((k + np.float32(0.5)) * sc).astype(np.float32)
        steps = rng.integers(-3, 4, dim - 1)
        v = np.array([np.float32(a) if s == 0 else
                      np.nextafter(np.float32(a), np.float32(np.inf if s > 0 else -np.inf), dtype=np.float32)
                      for a, s in zip(v, steps)], np.float32)
        x[r, 0] = mx
        x[r, 1:] = np.clip(v, -mx, mx)
    x = x[:, rng.permutation(dim)]
    codes, scales, norms = ops.quantize_sq8(torch.from_numpy(x).cuda())
    wc, ws, wn = oracle.quantize_sq8(x)
    bad = np.argwhere(codes.cpu().numpy() != wc)
    assert bad.size == 0, f"{len(bad)} code mismatches, first {bad[:3].tolist()}"
    assert np.array_equal(scales.cpu().numpy().view(np.uint32), ws.view(np.uint32))
    assert np.array_equal(norms.cpu().numpy().view(np.uint32), wn.view(np.uint32))


def test_quantize_golden_and_host_api():
    from shear_b200 import ops
    codes, scales, norms = ops.quantize_sq8_host(np.array([[0, 0, 0], [1, -1, 0.5]], np.float32), k_align=8)
    assert codes[1].tolist() == [127, -127, 64, 0, 0, 0, 0, 0]
    assert scales[1] == np.float32(1) / np.float32(127) and norms[1] == np.float32(2.25)
    assert scales[0] == 1.0 and norms[0] == 0.0


def test_quantize_rejects_non_finite():
    from shear_b200 import ops, TessaError
    with pytest.raises(TessaError, match="NONFINITE"):
        ops.quantize_sq8_host(np.array([[1.0, np.nan, 2.0]], np.float32))
