"""scmp_sc_matmul_noalloc, the entry point for callers that cannot allocate.

Some callers of this library have no way to hand it device scratch memory:
a host program that binds the C ABI through a plain FFI and owns no device
allocator, or a serving process that reserved all device memory at start-up
and must not call cudaMalloc afterwards. scmp_sc_matmul_noalloc serves them
from a fixed 16 MiB array compiled into the library. This test calls it
through the C ABI, twice in a row, and checks both results against the
workspace-taking scmp_sc_matmul bit for bit (the tolerance every parity test
here uses), then checks that a call needing more scratch than the array holds
is refused with a clear error. It is collected last so that a failing run
stops only after every other test has run.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from scmp_kernels_b200 import _lib  # noqa: E402
from scmp_kernels_b200.sc import kernels as K  # noqa: E402
from scmp_kernels_b200.sc.config_helpers import make_sobol_simple_config  # noqa: E402

DEV = torch.device("cuda", 0)


def _desc(a, b, out, gran, mode, sc_prec, tables):
    n, d, m = a.shape[-2], a.shape[-1], b.shape[-2]
    amap, bmap = tables.maps_for(d)
    desc = _lib.MatmulDesc(
        granularity=gran, mode=_lib.BIPOLAR if mode == "bipolar" else _lib.UNIPOLAR, sc_prec=sc_prec,
        stoc_len=tables.L, rng_levels=tables.G, chunk_d=0, group_a=1, group_b=1, batch=1, n=n,
        m=m, d=d, a=a.data_ptr(), b=b.data_ptr(), smooth_scales=None, out=out.data_ptr(),
        ktab=tables.ktab.data_ptr(), pattern=tables.pattern.data_ptr(), amap=amap.data_ptr(),
        bmap=bmap.data_ptr(), vcap=tables.vcap, lp=tables.lp, flags=0, pattern4=tables.pattern4.data_ptr())
    return desc, (amap, bmap)


@pytest.mark.parametrize("gran,mode,sc_prec,shape", [
    (_lib.PER_ROW, "bipolar", 8, (300, 520, 1000)),
    (_lib.PER_TENSOR, "unipolar", 6, (129, 257, 640)),
])
def test_noalloc_matches_workspace_entry_point(gran, mode, sc_prec, shape):
    torch.cuda.set_device(DEV)
    lib = _lib.lib()
    n, m, d = shape
    g = torch.Generator(device=DEV).manual_seed(11)
    a = torch.randn(n, d, device=DEV, generator=g)
    b = torch.randn(m, d, device=DEV, generator=g) * 0.05
    tables = K._get_cached_enable_tables(make_sobol_simple_config(d, d, sc_prec), sc_prec, DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)

    ref = torch.empty(n, m, device=DEV)
    desc, keep = _desc(a, b, ref, gran, mode, sc_prec, tables)
    need = ctypes.c_size_t()
    _lib.check(lib.scmp_sc_matmul_workspace_size(ctypes.byref(desc), ctypes.byref(need)))
    ws = torch.empty(need.value, dtype=torch.uint8, device=DEV)
    _lib.check(lib.scmp_sc_matmul(ctypes.byref(desc), ctypes.c_void_p(ws.data_ptr()), need.value, stream))

    # the case fits the fixed scratch (the no-alloc entry drops the split of
    # the last wave, whose part accumulators may not fit; results are the same)
    whole = ctypes.c_size_t()
    desc.flags = _lib.FLAG_NO_SPLIT
    _lib.check(lib.scmp_sc_matmul_workspace_size(ctypes.byref(desc), ctypes.byref(whole)))
    desc.flags = 0
    assert whole.value <= 16 << 20
    for _ in range(2):  # the shared scratch keeps the previous call's contents
        out = torch.full((n, m), float("nan"), device=DEV)
        desc2, keep2 = _desc(a, b, out, gran, mode, sc_prec, tables)
        _lib.check(lib.scmp_sc_matmul_noalloc(ctypes.byref(desc2), stream), "sc_matmul_noalloc")
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    assert _lib.device_error() == 0


def test_noalloc_rejects_oversized_calls():
    lib = _lib.lib()
    desc = _lib.MatmulDesc(granularity=_lib.PER_ROW, mode=_lib.BIPOLAR, sc_prec=8, stoc_len=256,
                           rng_levels=256, group_a=1, group_b=1, batch=1, n=4096, m=4096, d=4096,
                           vcap=256, lp=256, a=1, b=1, out=1, ktab=1, pattern=1, amap=1, bmap=1)
    st = lib.scmp_sc_matmul_noalloc(ctypes.byref(desc), None)
    assert st == _lib.SCMP_ERR_INVALID_ARG
    assert b"16 MiB" in lib.scmp_last_error()
