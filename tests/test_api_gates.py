"""API gates and SmoothQuant helpers, on CPU: the same ValueError gates and
message substrings as the reference's tests (tests/test_sc_smoke.py:76-129,
tests/test_smoothquant.py), raised before any device work."""
from __future__ import annotations

import pytest
import torch

from scmp_kernels_b200 import sc_matmul
from scmp_kernels_b200.quant.smoothquant import (accumulate_act_scales, apply_smoothing,
                                                 apply_smoothing_offline, compute_smooth_scales)


def test_import_surface():
    from scmp_kernels_b200 import sc_matmul  # noqa: F401
    from scmp_kernels_b200.sc import clear_rng_cache, det_kernel_tuning, sc_matmul  # noqa: F401,F811
    from scmp_kernels_b200.quant import (fused_quantize_bipolar, fused_quantize_bipolar_perrow,  # noqa: F401
                                         fused_quantize_unipolar, _grouped_symmetric_quant)
    from scmp_kernels_b200.sc.kernels import fused_quantize_bipolar as f2  # noqa: F401  (re-export)
    with det_kernel_tuning():
        with det_kernel_tuning():
            pass


@pytest.mark.parametrize("kw,shape,match", [
    (dict(granularity="per_tensor", chunk_d=72), "2d", "chunk_d"),
    (dict(granularity="per_row", mode="unipolar", chunk_d=72), "2d", "chunk_d"),
    (dict(granularity="per_row", chunk_d=72), "3d", "chunk_d"),
    (dict(granularity="per_head"), "2d", "per_head"),
    (dict(granularity="per_head", mode="unipolar"), "3d", "per_head"),
    (dict(granularity="per_block"), "2d", "granularity"),
    (dict(mode="ternary"), "2d", "mode"),
])
def test_value_error_gates(kw, shape, match):
    if shape == "2d":
        a, b = torch.randn(64, 1024), torch.randn(128, 1024)
    else:
        a, b = torch.randn(4, 64, 1024), torch.randn(4, 128, 1024)
    with pytest.raises(ValueError, match=match):
        sc_matmul(a, b, **kw)


def test_device_mismatch_and_smoothing_shape():
    a, b = torch.randn(4, 8), torch.randn(4, 8)
    with pytest.raises(ValueError):
        sc_matmul(a, b, smooth_scales=torch.ones(7))
    with pytest.raises(ValueError):
        sc_matmul(a, b, smooth_scales=torch.ones(2, 8))


def test_no_cpu_fallback():
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(RuntimeError, match="CUDA device"):
        sc_matmul(torch.randn(4, 8), torch.randn(5, 8))


def test_accumulate_act_scales():
    torch.manual_seed(0)
    x1, x2 = torch.randn(8, 16), torch.randn(8, 16) * 3.0
    r = accumulate_act_scales(x2, accumulate_act_scales(x1))
    assert torch.allclose(r, torch.maximum(x1.abs().amax(0), x2.abs().amax(0)))


def test_compute_smooth_scales_closed_forms():
    torch.manual_seed(1)
    act, w = torch.rand(16) + 0.1, torch.randn(32, 16)
    s = compute_smooth_scales(act, w, alpha=0.5)
    assert s.shape == (16,) and torch.all(s > 0)
    assert torch.allclose(compute_smooth_scales(act, w, 0.0), 1.0 / w.abs().amax(0).clamp(min=1e-5))
    assert torch.allclose(compute_smooth_scales(act, w, 1.0), act.clamp(min=1e-5))


def test_apply_smoothing_identities():
    torch.manual_seed(2)
    a, b = torch.randn(4, 32, dtype=torch.float64), torch.randn(6, 32, dtype=torch.float64)
    s = torch.rand(32, dtype=torch.float64) + 0.5
    a_s, b_s = apply_smoothing(a, b, s)
    assert (a @ b.T - a_s @ b_s.T).abs().max() < 1e-10
    a3, b3 = torch.randn(2, 4, 32, dtype=torch.float64), torch.randn(2, 6, 32, dtype=torch.float64)
    a3s, b3s = apply_smoothing(a3, b3, s)
    assert (a3 @ b3.transpose(-1, -2) - a3s @ b3s.transpose(-1, -2)).abs().max() < 1e-10
    w = apply_smoothing_offline(b, s)
    assert ((a / s) @ w.T - a @ b.T).abs().max() < 1e-10


def test_smoothing_invalid_args():
    with pytest.raises(ValueError):
        compute_smooth_scales(torch.ones(8), torch.ones(4, 8), alpha=1.5)
    with pytest.raises(ValueError):
        compute_smooth_scales(torch.ones(8), torch.ones(4, 9))
    with pytest.raises(ValueError):
        apply_smoothing(torch.zeros(2, 8), torch.zeros(3, 8), torch.zeros(2, 8))


def test_prepare_weight_argument_checks():
    from scmp_kernels_b200 import prepare_weight
    with pytest.raises(ValueError, match="mode"):
        prepare_weight(torch.zeros(4, 8), mode="ternary")
    with pytest.raises(ValueError, match="2D"):
        prepare_weight(torch.zeros(2, 4, 8))
    with pytest.raises(ValueError, match="float32"):
        prepare_weight(torch.zeros(4, 8, dtype=torch.float16), smooth_scales=torch.ones(8))
    with pytest.raises(ValueError, match="smooth_scales"):
        prepare_weight(torch.zeros(4, 8), smooth_scales=torch.ones(7))
