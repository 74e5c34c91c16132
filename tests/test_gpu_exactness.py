"""Where the exactness of the native path is most exposed, on the GPU.

* The default GEMM accumulates products of e2m1 values (0, +1, -1) in the
  float32 accumulator of tcgen05.mma.kind::mxf4; that is exact only while
  every partial sum stays an integer below 2^24 in magnitude and the tensor
  core adds at full float32 precision. These tests drive the production
  kernels (e2m1, int8, CUDA cores) to accumulators of 2^23 (every stream bit
  set, checked against the closed form) and past 2^22 with mixed signs and
  odd increments (checked against the C restatement of the reference's
  accumulator, sc/kernels.py:216-252).
* The full-size benchmark outputs at their far corners (the last output
  tiles: whole tiles for config 2, whose last wave fills 72 of 74 SM pairs;
  pieces of the stream-K tail for config 2 with 10048 rows of b and for
  config 5's 512-row run) against the CPU oracle.
* enable_matmul on quantised operands, per_tensor 3D (kernels.py:1207-1226)
  and the SC_OWEN_MODE=random masks against the reference's own function on
  the same CUDA device (kernels.py:646-704; the reference installed in
  baseline/_ref, skipped when it is not).
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest
import torch

from oracle import c_oracle as CO
from oracle import sc_oracle as O

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from scmp_kernels_b200 import _lib, sc_matmul  # noqa: E402
from scmp_kernels_b200.sc import clear_rng_cache  # noqa: E402
from scmp_kernels_b200.sc import kernels as K  # noqa: E402

DEV = "cuda:0"
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(params=["e2m1", "int8", "simt"])
def variant(request, monkeypatch):
    monkeypatch.setattr(K, "_FORCE_SIMT", request.param == "simt")
    monkeypatch.setenv("SCMP_TC_INT8", "1" if request.param == "int8" else "0")
    monkeypatch.setenv("SCMP_TC_ATMEM", "0")
    monkeypatch.delenv("SCMP_TC_SINGLE", raising=False)
    for k in ("SC_OWEN_MODE", "SC_DISABLE_OWEN", "SC_SCRAMBLE_RESCALE"):
        monkeypatch.delenv(k, raising=False)
    clear_rng_cache()
    yield request.param
    clear_rng_cache()


def test_saturated_accumulator_2p23_closed_form(variant):
    """Every operand at full scale: each boundary saturates (k = L, every
    stream bit set), so S = +-D*L = +-2^23 exactly (D = 32768, L = 256), and
    the output is fl32(fl32(S * fl32(q^2/L)) * fl32(sa * sb)) with
    sa = sb = fl32(1 / 127). A single 256 x 256 output tile: the default
    GEMM shares its K range over eight SM pairs (stream-K pieces summed in
    int32), the others accumulate it whole."""
    d, n, m = 32768, 256, 256
    a = torch.ones(n, d, device=DEV)
    b = torch.ones(m, d, device=DEV)
    a[1::2] = -1.0                      # odd rows of a negative: S = -2^23 there
    b[::3] = -1.0
    y = sc_matmul(a, b, "per_row", mode="bipolar", sc_prec=8)
    f32 = np.float32
    s = f32(1.0) / f32(127)
    sign = np.where(np.arange(n) % 2 == 1, -1, 1)[:, None] * np.where(np.arange(m) % 3 == 0, -1, 1)[None, :]
    S = (sign * d * 256).astype(f32)
    expect = (S * (f32(127 * 127) / f32(256))) * (s * s)
    assert np.array_equal(y.cpu().numpy(), expect.astype(f32))
    assert _lib.device_error() == 0


def test_mixed_sign_accumulator_past_2p22_vs_c_oracle(variant):
    """Operands near full scale with a few negative dimensions: integer sums
    between 4.0e6 and 4.3e6 (past 2^22), built from odd per-dimension counts
    (boundaries below the saturation point), checked against the C
    restatement of the reference's accumulator."""
    d, n, m = 17001, 64, 96
    g = torch.Generator().manual_seed(61)
    a = 1.0 - 0.006 * torch.rand(n, d, generator=g)
    b = 1.0 - 0.006 * torch.rand(m, d, generator=g)
    flip = torch.rand(m, d, generator=g) < 0.01
    b[flip] = -b[flip]
    y = sc_matmul(a.to(DEV), b.to(DEV), "per_row", mode="bipolar", sc_prec=8).cpu().numpy()
    ref = CO.sc_matmul(a.numpy(), b.numpy(), "per_row", mode="bipolar", sc_prec=8)
    assert np.array_equal(y, ref)
    # the sums really are past 2^22 and odd in places: out / (fl32(q^2/L) *
    # sa * sb) recovers S to within a fraction of one
    sa = a.abs().amax(1).double().numpy() / 127
    sb = b.abs().amax(1).double().numpy() / 127
    S = y.astype(np.float64) / (16129.0 / 256.0) / (sa[:, None] * sb[None, :])
    assert np.abs(S).max() > 2 ** 22
    assert (np.rint(S) % 2 == 1).any()
    assert _lib.device_error() == 0


@pytest.mark.parametrize("workload", ["config2", "config2_tail", "config5"])
def test_full_size_far_corner_vs_oracle(workload, monkeypatch):
    """The last 64 x 64 block of the full config-2 output (its last wave is
    whole tiles), of config 2 with 10048 rows of b (336 tiles: a last wave of
    40 tiles that the stream-K tail shares over the 74 SM pairs) and of
    config 5's 512-row run (a tail as well) equal the CPU oracle's."""
    for k in ("SC_OWEN_MODE", "SC_DISABLE_OWEN", "SC_SCRAMBLE_RESCALE", "SCMP_TC_INT8", "SCMP_TC_ATMEM",
              "SCMP_TC_SINGLE"):
        monkeypatch.delenv(k, raising=False)
    monkeypatch.setattr(K, "_FORCE_SIMT", False)
    from scmp_kernels_b200 import workloads as W
    if workload.startswith("config2"):
        a, b = W.config2(DEV)
        if workload == "config2_tail":
            b = b[:10048].contiguous()
        kw = dict(mode="bipolar", sc_prec=8)
        s = None
    else:
        a, b, s = W.config5(DEV)
        a = a[:512].contiguous()
        kw = dict(mode="unipolar", sc_prec=6, stoc_len=64)
    y = sc_matmul(a, b, "per_row", smooth_scales=s, **kw)
    blk = y[-64:, -64:].cpu().numpy()
    del y
    ref = CO.sc_matmul(a[-64:].cpu().numpy(), b[-64:].cpu().numpy(), "per_row",
                       smooth_scales=None if s is None else s.cpu().numpy(), **kw)
    assert np.array_equal(blk, ref)
    assert _lib.device_error() == 0


@pytest.mark.parametrize("bip", [True, False])
def test_enable_matmul_vs_oracle(bip):
    """enable_matmul (enable_matmul_triton's counterpart) on quantised
    operands: fl32(S * fl32(q^2 / L)) with S the reference's accumulator."""
    from scmp_kernels_b200.sc.config_helpers import make_sobol_simple_config
    clear_rng_cache()
    n, m, d, L, G = 70, 130, 200, 128, 256
    cfg = make_sobol_simple_config(d, d, 8)
    t = K._get_cached_enable_tables(cfg, 8, torch.device(DEV), L, G)
    g = torch.Generator().manual_seed(71)
    ba = torch.randint(0, G + 1, (n, d), generator=g, dtype=torch.int16)
    bb = torch.randint(0, G + 1, (m, d), generator=g, dtype=torch.int16)
    sa = (torch.randint(0, 2, (n, d), generator=g) * 2 - 1).to(torch.int8)
    sb = (torch.randint(0, 2, (m, d), generator=g) * 2 - 1).to(torch.int8)
    q2 = 127.0 * 127.0
    y = K.enable_matmul(t, ba.to(DEV), bb.to(DEV), sa.to(DEV) if bip else None, sb.to(DEV) if bip else None,
                        n, m, d, L, q2, bip).cpu().numpy()
    T = O.Tables(cfg, 8, L, G, env={})
    S = T.S(ba.numpy().astype(np.int64), bb.numpy().astype(np.int64),
            sa.numpy() if bip else None, sb.numpy() if bip else None)
    assert np.array_equal(y, O.scaled(S, 127, L))
    assert _lib.device_error() == 0


@pytest.mark.parametrize("mode,p", [("bipolar", 8), ("unipolar", 6)])
def test_per_tensor_3d_vs_oracle(mode, p):
    """per_tensor with (B, N, D) operands: one range over the whole tensors,
    every batch entry quantised with it (kernels.py:1207-1226, run there on
    one CUDA stream per entry, which the CPU interpreter cannot run)."""
    clear_rng_cache()
    g = torch.Generator().manual_seed(73)
    a = torch.randn(3, 21, 45, generator=g)
    b = torch.randn(3, 17, 45, generator=g) * 0.3
    y = sc_matmul(a.to(DEV), b.to(DEV), "per_tensor", mode=mode, sc_prec=p).cpu().numpy()
    ref = O.sc_matmul(a.numpy(), b.numpy(), "per_tensor", mode=mode, sc_prec=p, env={})
    assert np.array_equal(y, ref)
    assert _lib.device_error() == 0


def _reference_kernels():
    ref = os.path.join(REPO, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "scmp_kernels")):
        pytest.skip("the reference is not installed in baseline/_ref")
    if ref not in sys.path:
        sys.path.append(ref)
    import scmp_kernels.sc.kernels as RK
    return RK


@pytest.mark.parametrize("L,G", [(64, 256), (100, 128), (40, 100)])
def test_owen_random_masks_match_reference_on_device(L, G, monkeypatch):
    """SC_OWEN_MODE=random draws its masks from a seeded torch generator on
    the operands' device; the prepared sequences here equal the reference's
    _prepare_rng_prefix run on the same CUDA device, and the device tables
    built from them equal the oracle's tables of those sequences."""
    RK = _reference_kernels()
    monkeypatch.setenv("SC_OWEN_MODE", "random")
    monkeypatch.delenv("SC_DISABLE_OWEN", raising=False)
    monkeypatch.delenv("SC_SCRAMBLE_RESCALE", raising=False)
    from scmp_kernels_b200.sc.config_helpers import make_sobol_simple_config
    clear_rng_cache()
    d = 48
    cfg = make_sobol_simple_config(d, d, 8)
    qa, kb = K._get_cached_sequences(cfg, 8, DEV)
    for seq in (qa, kb):
        ours = K._prepare_rng_prefix(seq, 8, L, G, DEV)
        ref = RK._prepare_rng_prefix(torch.from_numpy(seq).to(DEV), 8, L, G).cpu().numpy()
        assert np.array_equal(ours, ref)
    t = K._get_cached_enable_tables(cfg, 8, torch.device(DEV), L, G)
    ra = K._prepare_rng_prefix(qa, 8, L, G, DEV)
    V = t.vcap + 1
    kt = O.k_table(ra, L, V)
    assert np.array_equal(t.ktab.cpu().numpy()[t.amap.cpu().numpy()], kt.astype(np.int16))
    clear_rng_cache()
