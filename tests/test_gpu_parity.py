"""Parity of the native B200 path with the reference, on the GPU.

* every golden fixture (outputs of the reference's own sc_matmul) through the
  tcgen05 path and through the CUDA-core path: bit-exact float32;
* device tables against the reference's k_table / cum_indicator;
* seeded random cases against the CPU oracle, bit-exact;
* the quantiser API against the oracle's restatements.
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, golden_names, load_golden
from oracle import sc_oracle as O

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from scmp_kernels_b200 import _lib, sc_matmul  # noqa: E402
from scmp_kernels_b200.sc import clear_rng_cache  # noqa: E402
from scmp_kernels_b200.sc import kernels as K  # noqa: E402

DEV = "cuda:0"


@pytest.fixture(params=["tc2", "tc2int8", "tc2atmem", "tc1", "simt"])
def impl(request, monkeypatch):
    """tc2: tcgen05 on SM pairs (default: e2m1 operands for streams of 64
    positions or more, 480-wide tiles for long tiles, two accumulators for
    short ones); tc2int8: the same with int8 operands (512-wide tiles);
    tc2atmem: SM pairs with a in tensor memory for long tiles; tc1: tcgen05
    on single SMs; simt: CUDA cores."""
    monkeypatch.setattr(K, "_FORCE_SIMT", request.param == "simt")
    monkeypatch.setenv("SCMP_TC_ATMEM", "1" if request.param == "tc2atmem" else "0")
    monkeypatch.setenv("SCMP_TC_INT8", "1" if request.param == "tc2int8" else "0")
    if request.param == "tc1":
        monkeypatch.setenv("SCMP_TC_SINGLE", "1")
    else:
        monkeypatch.delenv("SCMP_TC_SINGLE", raising=False)
    clear_rng_cache()
    yield request.param
    clear_rng_cache()


def _run(a, b, p, s=None):
    p = dict(p)
    g = p.pop("granularity")
    ta = torch.from_numpy(a).to(DEV)
    tb = torch.from_numpy(b).to(DEV)
    ts = torch.from_numpy(s).to(DEV) if s is not None else None
    y = sc_matmul(ta, tb, g, smooth_scales=ts, **p)
    assert y.device == ta.device and y.dtype == torch.float32
    out = y.cpu().numpy()
    assert _lib.device_error() == 0
    return out


@pytest.mark.parametrize("name", golden_names())
def test_golden(name, impl, env_vars):
    a, b, p, out, s, env = load_golden(name)
    env_vars(env)
    y = _run(a, b, p, s)
    assert y.shape == out.shape
    bad = np.argwhere(y != out)
    assert bad.size == 0, f"{len(bad)} mismatches, first at {bad[0]}: {y[tuple(bad[0])]} vs {out[tuple(bad[0])]}"


RNG = np.load(os.path.join(GOLDEN, "rng_golden.npz"))


@pytest.mark.parametrize("L,G", [(256, 256), (64, 256), (64, 64), (100, 128), (256, 300), (40, 100)])
def test_device_tables_reproduce_reference(L, G, env_vars):
    env_vars({})
    from scmp_kernels_b200.sc.config_helpers import make_sobol_simple_config
    clear_rng_cache()
    t = K._get_cached_enable_tables(make_sobol_simple_config(6, 6, 8), 8, torch.device(DEV), L, G)
    kt = t.ktab.cpu().numpy()[t.amap.cpu().numpy()]
    ref_k = RNG[f"ktab_L{L}_G{G}"]
    assert np.array_equal(kt[:, :G + 1], ref_k[:, :G + 1])
    pat = t.pattern.cpu().numpy().view(np.uint32)[t.bmap.cpu().numpy()]   # (6, vcap+1, lw)
    sliced = np.unpackbits(pat.view(np.uint8), axis=-1, bitorder="little")  # (6, vcap+1, lp), bit order
    # word bit 8i + 4h + q holds position 16h + 4q + i of the word
    l = np.arange(32)
    perm = 8 * (l & 3) + 4 * (l >> 4) + ((l >> 2) & 3)
    idx = (np.arange(sliced.shape[-1]) // 32) * 32 + perm[np.arange(sliced.shape[-1]) % 32]
    bits = sliced[..., idx]                                               # position order
    # e2m1-sliced copy: word bit 4i + q holds position 8q + i of the word
    pat4 = t.pattern4.cpu().numpy().view(np.uint32)[t.bmap.cpu().numpy()]
    s4 = np.unpackbits(pat4.view(np.uint8), axis=-1, bitorder="little")
    perm4 = 4 * (l & 7) + (l >> 3)
    idx4 = (np.arange(s4.shape[-1]) // 32) * 32 + perm4[np.arange(s4.shape[-1]) % 32]
    assert np.array_equal(s4[..., idx4], bits)
    cum = np.concatenate([np.zeros(bits.shape[:2] + (1,), np.int64), np.cumsum(bits, -1)], -1)
    ref = RNG[f"cum_L{L}_G{G}"]                                           # (6, L+1, V)
    vv = min(ref.shape[2], t.vcap + 1)
    assert np.array_equal(cum[:, :vv, :L + 1].transpose(0, 2, 1), ref[:, :, :vv])


CASES = [
    dict(granularity="per_row", mode="bipolar", sc_prec=8, n=37, m=53, d=300),
    dict(granularity="per_row", mode="unipolar", sc_prec=6, n=33, m=65, d=129, stoc_len=64),
    dict(granularity="per_row", mode="bipolar", sc_prec=8, n=130, m=260, d=64, group_a=3, group_b=7),
    dict(granularity="per_tensor", mode="bipolar", sc_prec=8, n=20, m=300, d=77),
    dict(granularity="per_tensor", mode="unipolar", sc_prec=7, n=129, m=31, d=95),
    dict(granularity="per_row", mode="bipolar", sc_prec=8, n=40, m=33, d=200, chunk_d=64, stoc_len=128,
         rng_levels=128),
    dict(granularity="per_row", mode="bipolar", sc_prec=8, n=17, m=29, d=150, chunk_d=72),
    dict(granularity="per_head", mode="bipolar", sc_prec=8, bh=3, n=23, m=41, d=19),
    dict(granularity="per_row", mode="bipolar", sc_prec=8, bh=2, n=9, m=140, d=31, stoc_len=32),
    dict(granularity="per_row", mode="bipolar", sc_prec=5, n=140, m=270, d=48, stoc_len=20),
    dict(granularity="per_row", mode="bipolar", sc_prec=9, n=40, m=270, d=24),
]


@pytest.mark.parametrize("case", range(len(CASES)))
def test_random_vs_oracle(case, impl, env_vars):
    env_vars({})
    c = dict(CASES[case])
    g = torch.Generator().manual_seed(1000 + case)
    bh = c.pop("bh", None)
    n, m, d = c.pop("n"), c.pop("m"), c.pop("d")
    sa = (bh, n, d) if bh else (n, d)
    sb = (bh, m, d) if bh else (m, d)
    a = (torch.randn(*sa, generator=g) * 2).numpy()
    b = (torch.randn(*sb, generator=g) * 0.05).numpy()
    a.reshape(-1)[::97] = 0.0
    y = _run(a, b, c)
    p = dict(c)
    gran = p.pop("granularity")
    ref = O.sc_matmul(a, b, gran, env={}, **p)
    assert np.array_equal(y, ref), f"max |diff| {np.abs(y - ref).max()}"


@pytest.mark.parametrize("smooth", [False, True])
def test_per_head_one_pass_params_vs_oracle(smooth, impl, env_vars):
    """per_head scales from the one-pass head kernel: heads that start off a
    16-byte boundary (odd d), an all-zero head on each side, with and without
    SmoothQuant scales, against the oracle bit for bit."""
    env_vars({})
    g = torch.Generator().manual_seed(77)
    a = (torch.randn(4, 31, 13, generator=g) * 2).numpy()
    b = (torch.randn(4, 17, 13, generator=g) * 0.5).numpy()
    a[2] = 0.0
    b[1] = 0.0
    s = (torch.rand(13, generator=g) + 0.5).numpy() if smooth else None
    y = _run(a, b, dict(granularity="per_head", sc_prec=8), s)
    ref = O.sc_matmul(a, b, "per_head", sc_prec=8, smooth_scales=s, env={})
    assert np.array_equal(y, ref), f"max |diff| {np.abs(y - ref).max()}"


@pytest.mark.parametrize("shape,kw", [
    ((600, 1100, 1024), dict(granularity="per_row", sc_prec=8)),                       # 512 stages per tile
    ((530, 700, 4096), dict(granularity="per_row", mode="unipolar", sc_prec=6, stoc_len=64)),
])
def test_narrow_long_tiles_equal_default(shape, kw, monkeypatch, env_vars):
    """The opt-in narrow kernel for long tiles (SCMP_TC_NARROW=1: 240-wide
    tiles on the unrolled two-buffer kernel, whole tiles only) gives the
    default wide kernel's bits."""
    env_vars({})
    monkeypatch.setattr(K, "_FORCE_SIMT", False)
    n, m, d = shape
    g = torch.Generator(device=DEV).manual_seed(21)
    a = torch.randn(n, d, device=DEV, generator=g)
    b = torch.randn(m, d, device=DEV, generator=g) * 0.03
    y_wide = sc_matmul(a, b, **kw)
    monkeypatch.setenv("SCMP_TC_NARROW", "1")
    y_narrow = sc_matmul(a, b, **kw)
    assert torch.equal(y_wide, y_narrow)
    assert _lib.device_error() == 0


@pytest.mark.parametrize("shape,kw", [
    ((300, 520, 1000), dict(granularity="per_row", sc_prec=8)),
    ((700, 1300, 512), dict(granularity="per_row", mode="unipolar", sc_prec=6, stoc_len=64)),
    ((260, 600, 640), dict(granularity="per_row", sc_prec=8, chunk_d=64, stoc_len=128, rng_levels=128)),
])
def test_tc_variants_match_simt_at_size(shape, kw, monkeypatch, env_vars):
    env_vars({})
    n, m, d = shape
    g = torch.Generator(device=DEV).manual_seed(7)
    a = torch.randn(n, d, device=DEV, generator=g)
    b = torch.randn(m, d, device=DEV, generator=g) * 0.02
    outs = []
    # CUDA cores; SM pairs (default, e2m1); SM pairs with int8 operands; SM
    # pairs with a in tensor memory; single SMs
    for simt, single, atmem, i8 in ((True, "0", "0", "0"), (False, "0", "0", "0"), (False, "0", "0", "1"),
                                    (False, "0", "1", "0"), (False, "1", "0", "0")):
        monkeypatch.setattr(K, "_FORCE_SIMT", simt)
        monkeypatch.setenv("SCMP_TC_SINGLE", single)
        monkeypatch.setenv("SCMP_TC_ATMEM", atmem)
        monkeypatch.setenv("SCMP_TC_INT8", i8)
        outs.append(sc_matmul(a, b, **kw))
    for i, o in enumerate(outs[1:], 1):
        assert torch.equal(outs[0], o), f"variant {i} differs from the CUDA-core GEMM"
    assert _lib.device_error() == 0


@pytest.mark.parametrize("shape,kw", [
    ((1000, 5000, 512), dict(granularity="per_row", sc_prec=8)),                 # fewer tiles than workers
    ((2048, 11008, 1024), dict(granularity="per_row", sc_prec=8)),               # 2 waves + a 28-tile tail
    ((600, 300, 1000), dict(granularity="per_tensor", mode="unipolar", sc_prec=7)),  # 6 tiles, all shared
    ((9, 197, 197, 640), dict(granularity="per_head", sc_prec=8)),                 # 9 heads, one tile each
    ((300, 700, 40), dict(granularity="per_row", sc_prec=8)),                    # 5 blocks: no tail
])
@pytest.mark.parametrize("single,i8", [("0", "0"), ("0", "1"), ("1", "0")])
def test_split_last_wave_matches_whole_tiles(shape, kw, single, i8, monkeypatch, env_vars):
    """The last wave's tiles shared over K by all workers (pieces of uneven
    length, a worker's range spanning two tiles, the pieces' accumulators
    summed by the last to finish) give the same bits as whole tiles."""
    env_vars({})
    g = torch.Generator(device=DEV).manual_seed(5)
    if len(shape) == 4:
        bh, n, m, d = shape
        a = torch.randn(bh, n, d, device=DEV, generator=g)
        b = torch.randn(bh, m, d, device=DEV, generator=g)
    else:
        n, m, d = shape
        a = torch.randn(n, d, device=DEV, generator=g)
        b = torch.randn(m, d, device=DEV, generator=g) * 0.05
    monkeypatch.setattr(K, "_FORCE_SIMT", False)
    monkeypatch.setenv("SCMP_TC_SINGLE", single)
    monkeypatch.setenv("SCMP_TC_INT8", i8)
    monkeypatch.setenv("SCMP_TC_NO_SPLIT", "0")
    y_split = sc_matmul(a, b, **kw)
    monkeypatch.setenv("SCMP_TC_NO_SPLIT", "1")
    y_whole = sc_matmul(a, b, **kw)
    assert torch.equal(y_split, y_whole)
    assert _lib.device_error() == 0


@pytest.mark.parametrize("shape,kw", [
    ((2048, 11008, 1024), dict(granularity="per_row", sc_prec=8)),                # 8 bands, 23 tiles each
    ((1800, 3000, 640), dict(granularity="per_row", mode="unipolar", sc_prec=6, stoc_len=64)),  # ragged
    ((5, 197, 197, 640), dict(granularity="per_head", sc_prec=8)),                # one band per head
])
@pytest.mark.parametrize("group", ["3", "8"])
def test_band_grouped_tile_order_matches_default(shape, kw, group, monkeypatch, env_vars):
    """Tiles taken in groups of bands of a (each b tile for every band of a
    group, SCMP_TC_BAND_GROUP) give the bits of the band-by-band order, the
    split last wave included."""
    env_vars({})
    g = torch.Generator(device=DEV).manual_seed(6)
    if len(shape) == 4:
        bh, n, m, d = shape
        a, b = torch.randn(bh, n, d, device=DEV, generator=g), torch.randn(bh, m, d, device=DEV, generator=g)
    else:
        n, m, d = shape
        a, b = torch.randn(n, d, device=DEV, generator=g), torch.randn(m, d, device=DEV, generator=g) * 0.05
    monkeypatch.setattr(K, "_FORCE_SIMT", False)
    monkeypatch.setenv("SCMP_TC_BAND_GROUP", "1")
    y1 = sc_matmul(a, b, **kw)
    monkeypatch.setenv("SCMP_TC_BAND_GROUP", group)
    yg = sc_matmul(a, b, **kw)
    assert torch.equal(y1, yg)
    assert _lib.device_error() == 0


@pytest.mark.parametrize("shape,kw", [
    ((300, 520, 4096), dict(granularity="per_row", sc_prec=8)),                          # 2 blocks per thread
    ((129, 77, 8192), dict(granularity="per_row", mode="unipolar", sc_prec=6, stoc_len=64, smooth=True)),
    ((70, 90, 301), dict(granularity="per_row", sc_prec=8, group_a=3, group_b=7)),      # ragged d: scalar loads
    ((50, 60, 16384), dict(granularity="per_row", sc_prec=8)),                          # 8 blocks per thread
    ((20000 // 100, 40, 20000), dict(granularity="per_row", sc_prec=7)),                # too long: warp kernel
    ((64, 48, 3000), dict(granularity="per_row", sc_prec=10)),                          # q > 256: no table
    ((33, 90, 130), dict(granularity="per_tensor", mode="unipolar", sc_prec=7)),
    ((3, 40, 50, 64), dict(granularity="per_head", sc_prec=8)),
    ((2, 9, 140, 31), dict(granularity="per_row", sc_prec=8)),                           # 3D per_row
    # short rows: 8, 16 or 32 threads per row, several rows per block, the
    # last block partly past the rows
    ((70, 33, 64), dict(granularity="per_row", mode="unipolar", sc_prec=6, stoc_len=64)),
    ((45, 37, 100), dict(granularity="per_row", mode="unipolar", sc_prec=6, stoc_len=64, smooth=True)),
    ((77, 50, 256), dict(granularity="per_row", sc_prec=8, group_a=3, group_b=7)),
    ((61, 29, 200), dict(granularity="per_row", mode="unipolar", sc_prec=7, group_a=2, group_b=5)),
    ((3, 197, 64, 197), dict(granularity="per_head", sc_prec=8)),
    ((5, 197, 197, 64), dict(granularity="per_head", sc_prec=8)),
])
def test_row_block_quantiser_matches_warp_quantiser(shape, kw, monkeypatch, env_vars):
    """The default quantiser (one block per row, the row in registers, one
    pass) and the warp-per-row one (SCMP_QUANT_WARP=1) give the same bits."""
    env_vars({})
    kw = dict(kw)
    g = torch.Generator(device=DEV).manual_seed(12)
    if len(shape) == 4:
        bh, n, m, d = shape
        a, b = torch.randn(bh, n, d, device=DEV, generator=g), torch.randn(bh, m, d, device=DEV, generator=g)
    else:
        n, m, d = shape
        a, b = torch.randn(n, d, device=DEV, generator=g), torch.randn(m, d, device=DEV, generator=g) * 0.05
    if kw.pop("smooth", False):
        kw["smooth_scales"] = torch.rand(a.shape[-1], device=DEV, generator=g) + 0.5
    monkeypatch.setattr(K, "_FORCE_SIMT", False)
    monkeypatch.setenv("SCMP_QUANT_WARP", "0")
    y_staged = sc_matmul(a, b, **kw)
    monkeypatch.setenv("SCMP_QUANT_WARP", "1")
    y_warp = sc_matmul(a, b, **kw)
    assert torch.equal(y_staged, y_warp)
    assert _lib.device_error() == 0


@pytest.mark.parametrize("gran,shape", [("per_row", (70, 300, 500)), ("per_tensor", (33, 90, 130)),
                                        ("per_head", (3, 40, 50, 64))])
@pytest.mark.parametrize("simt", [False, True])
def test_result_scattered_to_several_buffers(gran, shape, simt, monkeypatch, env_vars):
    """The epilogue's multi-destination store (the fused all-gather's
    mechanism, exercised here with two buffers on one device): every buffer
    receives the result at the given offset and row stride, nothing else."""
    env_vars({})
    monkeypatch.setattr(K, "_FORCE_SIMT", simt)
    g = torch.Generator(device=DEV).manual_seed(9)
    if gran == "per_head":
        bh, n, m, d = shape
        a, b = torch.randn(bh, n, d, device=DEV, generator=g), torch.randn(bh, m, d, device=DEV, generator=g)
    else:
        n, m, d = shape
        bh = 1
        a, b = torch.randn(n, d, device=DEV, generator=g), torch.randn(m, d, device=DEV, generator=g)
    ref = sc_matmul(a, b, gran, sc_prec=8)
    ld, off = m + 37, 11
    bufs = [torch.full((off + bh * n * ld + 5,), float("nan"), device=DEV) for _ in range(2)]
    with K.output_to([x.data_ptr() for x in bufs], off, ld, bufs[0]):
        sc_matmul(a, b, gran, sc_prec=8)
    torch.cuda.synchronize()
    for x in bufs:
        blk = x[off:off + bh * n * ld].view(bh * n, ld)
        assert torch.equal(blk[:, :m], ref.reshape(bh * n, m))
        assert torch.isnan(blk[:, m:]).all() and torch.isnan(x[:off]).all()
        assert torch.isnan(x[off + bh * n * ld:]).all()
    assert _lib.device_error() == 0


@pytest.mark.parametrize("kw", [dict(sc_prec=8), dict(sc_prec=6, mode="unipolar", stoc_len=64, group_b=7),
                                dict(sc_prec=8, chunk_d=64, stoc_len=128, rng_levels=128),
                                dict(sc_prec=8, group_a=5), dict(sc_prec=6, mode="unipolar", stoc_len=32, group_a=3),
                                dict(sc_prec=6, mode="unipolar", stoc_len=64, smooth=True)])
def test_host_operands_pipelined_equal_device_result(kw, env_vars):
    """Pinned host operands take the streamed path (b and the result moved in
    blocks while blocks compute); the result equals the device call's. With
    SmoothQuant scales in pinned host memory too."""
    env_vars({})
    from scmp_kernels_b200.sc import matmul as MM
    kw = dict(kw)
    g = torch.Generator().manual_seed(4)
    m = MM._HOST_MIN_ROWS + 333
    a = torch.randn(MM._HOST_MIN_ROWS + 77, 256, generator=g).pin_memory()
    b = (torch.randn(m, 256, generator=g) * 0.05).pin_memory()
    s = (torch.rand(256, generator=g) + 0.5).pin_memory() if kw.pop("smooth", False) else None
    assert MM._host_pipelined_applies(a, b)
    y_host = sc_matmul(a, b, "per_row", smooth_scales=s, **kw)
    assert y_host.device.type == "cpu" and y_host.shape == (a.shape[0], m)
    y_dev = sc_matmul(a.to(DEV), b.to(DEV), "per_row", smooth_scales=s.to(DEV) if s is not None else None, **kw)
    assert torch.equal(y_host, y_dev.cpu())
    assert _lib.device_error() == 0


def test_host_pipelined_waits_for_work_queued_on_freed_blocks(env_vars):
    """The streamed path's device staging buffers come from the caller's
    stream's memory pool; a block freed there may still be written by work
    queued on that stream. The copies into the staging buffers run on another
    stream and must start only after that work: here a spin kernel delays
    writes of huge values into two freed tensors of the staging buffers'
    sizes, and the result must still equal the device call's."""
    env_vars({})
    from scmp_kernels_b200.sc import matmul as MM
    g = torch.Generator().manual_seed(8)
    n, m, d = MM._HOST_MIN_ROWS + 77, MM._HOST_MIN_ROWS + 333, 256
    a = torch.randn(n, d, generator=g).pin_memory()
    b = (torch.randn(m, d, generator=g) * 0.05).pin_memory()
    ref = sc_matmul(a.to(DEV), b.to(DEV), "per_row", sc_prec=8).cpu()
    junk_a = torch.full((n, d), 1e30, device=DEV)
    junk_b = torch.full((m, d), -1e30, device=DEV)
    for _ in range(3):
        x = torch.empty(n, d, device=DEV)
        y = torch.empty(m, d, device=DEV)
        torch.cuda._sleep(20_000_000)  # a bounded spin (about 10 ms) on the current stream
        x.copy_(junk_a)
        y.copy_(junk_b)
        del x, y
        out = sc_matmul(a, b, "per_row", sc_prec=8)
        assert torch.equal(out, ref)
    assert _lib.device_error() == 0


def test_native_kernels_do_the_work():
    """One per_row call launches the library's own kernels: two quantisers,
    the padded row map and the SC-GEMM."""
    a = torch.randn(64, 300, device=DEV)
    b = torch.randn(96, 300, device=DEV)
    sc_matmul(a, b, "per_row", sc_prec=8)  # tables built and cached
    n0 = _lib.launch_count()
    sc_matmul(a, b, "per_row", sc_prec=8)
    torch.cuda.synchronize()
    assert _lib.launch_count() - n0 == 4


@pytest.mark.parametrize("workload,rows", [("config2", None), ("config5", 512), ("config3qk", None),
                                            ("config3av", None)])
def test_full_size_workloads_agree_across_gemm_variants(workload, rows, monkeypatch, env_vars):
    """The benchmark workloads at their full sizes (config 5: its first 512
    rows of a against all of b; per_row quantisation is row-local, so a row
    slice is an exact sub-problem): the default GEMM (SM pairs, 480-wide
    tiles, stream-K tail, e2m1 operands), the same with int8 operands, SM
    pairs with a in tensor memory, and the CUDA-core GEMM give the same bits,
    and every output is finite."""
    env_vars({})
    from scmp_kernels_b200 import workloads as W
    if workload == "config2":
        a, b = W.config2(DEV)
        kw = dict(granularity="per_row", mode="bipolar", sc_prec=8)
    elif workload == "config5":
        a, b, s5 = W.config5(DEV)
        a = a[:rows].contiguous()
        kw = dict(granularity="per_row", mode="unipolar", sc_prec=6, stoc_len=64, smooth_scales=s5)
    else:
        q, k, probs, v_t = W.config3(DEV)
        a, b = (q, k) if workload == "config3qk" else (probs, v_t)
        kw = dict(granularity="per_head", sc_prec=8)
    outs = []
    for simt, atmem, i8 in ((False, "0", "0"), (False, "0", "1"), (False, "1", "0"), (True, "0", "0")):
        monkeypatch.setattr(K, "_FORCE_SIMT", simt)
        monkeypatch.setenv("SCMP_TC_ATMEM", atmem)
        monkeypatch.setenv("SCMP_TC_INT8", i8)
        outs.append(sc_matmul(a, b, **kw))
    assert torch.isfinite(outs[0]).all()
    for i, o in enumerate(outs[1:], 1):
        assert torch.equal(outs[0], o), f"variant {i} differs"
    assert _lib.device_error() == 0


def test_quantiser_api_vs_oracle():
    from scmp_kernels_b200 import quant as Q
    g = torch.Generator().manual_seed(3)
    x = torch.randn(37, 90, generator=g)
    xn = x.numpy()
    bnd, sgn, sc = Q.fused_quantize_bipolar(x.to(DEV), float(x.abs().max()), 8)
    rb, rs, rsc = O.fused_quantize_bipolar(xn, float(x.abs().max()), 8, 256)
    assert np.array_equal(bnd.cpu().numpy(), rb) and np.array_equal(sgn.cpu().numpy(), rs) and sc == rsc
    bnd, sgn, scr = Q.fused_quantize_bipolar_perrow(x.to(DEV), 8, rng_levels=64)
    rb, rs, rsc = O.fused_quantize_bipolar_perrow(xn, 8, 64)
    assert np.array_equal(bnd.cpu().numpy(), rb) and np.array_equal(scr.cpu().numpy(), rsc)
    bnd, sc, zp, rsum = Q.fused_quantize_unipolar(x.to(DEV), float(x.max()), float(x.min()), 6,
                                                  compute_sum=True)
    rb, rsc, rzp, rrs = O.fused_quantize_unipolar(xn, float(x.max()), float(x.min()), 6, 64)
    assert np.array_equal(bnd.cpu().numpy(), rb) and sc == rsc and zp == rzp
    assert np.array_equal(rsum.cpu().numpy(), rrs)
    for G in (1, 4, 37, 100):
        s, xi, sg = Q._grouped_symmetric_quant(x.to(DEV), G, 127)
        rs_, rxi, rsg = O.grouped_symmetric_quant(xn, G, 127)
        assert np.array_equal(s.cpu().numpy(), rs_) and np.array_equal(xi.cpu().numpy(), rxi)
        assert np.array_equal(sg.cpu().numpy(), rsg)
        s, zp, xi = Q._grouped_asymmetric_quant(x.to(DEV), G, 255)
        rs_, rzp, rxi = O.grouped_asymmetric_quant(xn, G, 255)
        assert np.array_equal(s.cpu().numpy(), rs_) and np.array_equal(zp.cpu().numpy(), rzp)
        assert np.array_equal(xi.cpu().numpy(), rxi)
    x3 = torch.randn(3, 11, 20, generator=g)
    inv = (1.0 / (x3.abs().amax(dim=(1, 2)).clamp(min=1e-5) / 127)).float()
    bnd, sgn = Q.fused_quant_bipolar_batched(x3.to(DEV), inv.to(DEV), 8)
    rb, rs = O.fused_quant_bipolar_batched(x3.numpy(), inv.numpy(), 8, 256)
    assert np.array_equal(bnd.cpu().numpy(), rb.transpose(0, 2, 1))
    assert np.array_equal(sgn.cpu().numpy(), rs.transpose(0, 2, 1))
    assert _lib.device_error() == 0


def test_cpu_inputs_round_trip_and_device_guard():
    a, b = torch.randn(8, 64), torch.randn(16, 64)
    y = sc_matmul(a, b, "per_row")
    assert y.device.type == "cpu" and y.shape == (8, 16)
    assert torch.cuda.current_device() == 0
    y2 = sc_matmul(a.cuda(), b.cuda(), "per_row")
    assert torch.equal(y, y2.cpu())


@pytest.mark.parametrize("shape,self_index", [((4096, 3000, 640), 1), ((600, 1700, 1000), 0), ((300, 520, 700), 2)])
def test_deferred_peer_copies_fill_every_buffer(shape, self_index, env_vars):
    """With one destination marked as this device's own, the wide-tile GEMM
    stores each whole tile there and its epilogue warps copy it to the other
    destinations while the next tile computes (tail pieces store to all
    directly): every buffer gets the result at its offset and row stride."""
    env_vars({})
    n, m, d = shape
    g = torch.Generator(device=DEV).manual_seed(19)
    a, b = torch.randn(n, d, device=DEV, generator=g), torch.randn(m, d, device=DEV, generator=g) * 0.05
    ref = sc_matmul(a, b, "per_row", sc_prec=8)
    # one case with 16-byte-aligned rows (whole-vector copies), the others not
    ld, off = (m + 4, 8) if self_index == 0 else (m + 13, 7)
    bufs = [torch.full((off + n * ld + 3,), float("nan"), device=DEV) for _ in range(3)]
    with K.output_to([x.data_ptr() for x in bufs], off, ld, bufs[0], self_index=self_index):
        sc_matmul(a, b, "per_row", sc_prec=8)
    torch.cuda.synchronize()
    for x in bufs:
        blk = x[off:off + n * ld].view(n, ld)
        assert torch.equal(blk[:, :m], ref)
        assert torch.isnan(blk[:, m:]).all() and torch.isnan(x[:off]).all()
    assert _lib.device_error() == 0


@pytest.mark.parametrize("kw", [
    dict(mode="bipolar", sc_prec=8),
    dict(mode="unipolar", sc_prec=6, stoc_len=64, group_b=4),
    dict(mode="bipolar", sc_prec=8, smooth=True),
])
def test_prepared_weight_matches_sc_matmul(kw, env_vars):
    """A weight quantised once (prepare_weight / sc_matmul_prepared, the
    library's SCMP_FLAG_B_READY) gives the bits of sc_matmul on every call: a
    sequence of a's with growing and shrinking row counts (the workspace grows
    once, b is quantised again then), and, once quantised, b is not read
    (zeroing it leaves the results unchanged)."""
    from scmp_kernels_b200 import prepare_weight, sc_matmul_prepared
    env_vars({})
    kw = dict(kw)
    g = torch.Generator(device=DEV).manual_seed(21)
    d, m = 640, 1100
    b = torch.randn(m, d, device=DEV, generator=g) * 0.03
    if kw.pop("smooth", False):
        kw["smooth_scales"] = torch.rand(d, device=DEV, generator=g) + 0.5
    w = prepare_weight(b, **kw)
    refs = {}
    for n in (300, 1500, 64, 1500):
        a = torch.randn(n, d, device=DEV, generator=torch.Generator(device=DEV).manual_seed(n))
        ref = sc_matmul(a, b, "per_row", **kw)
        y = sc_matmul_prepared(a, w)
        assert torch.equal(y, ref), f"n={n}"
        refs[n] = (a, ref)
    b.zero_()  # the prepared weight refers to b; the workspace already holds it quantised
    for n in (300, 64):
        a, ref = refs[n]
        assert torch.equal(sc_matmul_prepared(a, w), ref)
    assert _lib.device_error() == 0
