"""GPU SQ8 quantizer vs the reference CPU quantizer restatement (bit-exact)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,dim", [(2, 3), (257, 100), (1000, 768), (64, 1024), (400_000, 8)])
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
