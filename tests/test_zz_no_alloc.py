"""The allocation-free LayerNorm backward (C symbol ``dtb_layernorm_bwd_noalloc``).

It exists for callers that must not allocate device memory while they run
(runtimes that own the whole GPU through their own pool, latency-critical loops
that cannot take cudaMalloc's device-wide synchronisation, plain-C callers).
This file is named so that pytest collects it last.  It calls the exported
symbol through ctypes - not through torch - and checks its outputs against the
regular ``layernorm_bwd`` entry point on two calls in a row: the scratch array
is shared by every call and keeps the previous call's contents, so the second
call checks that nothing stale leaks into its result.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

from dtrain_b200.ops import _ext  # noqa: E402
from dtrain_b200.ops import kernels as K  # noqa: E402


def _symbol():
    _ext.lib()  # make sure the library (and libtorch) is loaded into the process
    so = ctypes.CDLL(_ext.built_path())
    fn = so.dtb_layernorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 9 + [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    return fn


def _inputs(rows, C, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, C, device="cuda", generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(C, device="cuda", generator=g)).bfloat16()
    b = (0.1 * torch.randn(C, device="cuda", generator=g)).bfloat16()
    _, mean, rstd = K.layernorm_fwd(x, w, b)
    dy = torch.randn(rows, C, device="cuda", generator=g).bfloat16()
    dres = torch.randn(rows, C, device="cuda", generator=g).bfloat16()
    return x, w, mean, rstd, dy, dres


def _call(fn, x, w, mean, rstd, dy, dres, dx, dw, db, accumulate=0):
    stream = torch.cuda.current_stream().cuda_stream
    return fn(dy.data_ptr(), x.data_ptr(), w.data_ptr(), mean.data_ptr(), rstd.data_ptr(),
              dres.data_ptr() if dres is not None else None, dx.data_ptr(), dw.data_ptr(), db.data_ptr(),
              x.shape[0], x.shape[1], accumulate, stream)


def test_noalloc_layernorm_bwd_matches_regular_entry_point_twice():
    fn = _symbol()
    # two calls in a row with different shapes and data; the second one reuses the scratch array
    for call, (rows, C, seed) in enumerate([(4096, 768, 1), (1000, 1024, 2)]):
        x, w, mean, rstd, dy, dres = _inputs(rows, C, seed)
        dw_ref = torch.empty(C, device="cuda")
        db_ref = torch.empty(C, device="cuda")
        dx_ref = K.layernorm_bwd(dy, x, w, mean, rstd, dres, dw_ref, db_ref)
        dx = torch.empty_like(x)
        dw = torch.full((C,), float("nan"), device="cuda")
        db = torch.full((C,), float("nan"), device="cuda")
        rc = _call(fn, x, w, mean, rstd, dy, dres, dx, dw, db)
        torch.cuda.synchronize()
        assert rc == 0, f"call {call}: return code {rc}"
        torch.testing.assert_close(dx.float(), dx_ref.float(), rtol=1e-2, atol=1e-2)
        torch.testing.assert_close(dw, dw_ref, rtol=1e-4, atol=1e-4)
        torch.testing.assert_close(db, db_ref, rtol=1e-4, atol=1e-4)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    fn = _symbol()
    rows, C = 40000, 2048  # needs 2 * 625 * 2048 floats > the 1 Mi-float scratch
    x = torch.empty(64, C, device="cuda", dtype=torch.bfloat16)  # never read: rejected before launch
    mean = torch.empty(64, device="cuda")
    dw = torch.empty(C, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(x.data_ptr(), x.data_ptr(), x.data_ptr(), mean.data_ptr(), mean.data_ptr(), None, x.data_ptr(),
            dw.data_ptr(), dw.data_ptr(), rows, C, 0, stream)
    assert rc == -2
