"""The allocation-free LayerNorm backward (C symbol ``dtb_layernorm_bwd_noalloc``).

It exists for callers that must not allocate device memory while they run
(runtimes that own the whole GPU through their own pool, latency-critical loops
that cannot take cudaMalloc's device-wide synchronisation, plain-C callers).
This file is named so that pytest collects it last.  It calls the exported
symbol through ctypes - not through torch - with the return codes declared in
csrc/dtb_noalloc.h, and checks its outputs against the regular ``layernorm_bwd``
entry point (itself checked against fp32 PyTorch in test_kernels_gpu.py) on
calls in a row: the scratch array is shared by every call and keeps the previous
call's contents, so each later call checks that nothing stale leaks into its
result.  The calls cover the residual-gradient input present and absent, and
dw/db written or accumulated.
"""
import ctypes
import os
import re

import pytest
import torch

pytestmark = pytest.mark.gpu

from dtrain_b200.ops import _ext  # noqa: E402
from dtrain_b200.ops import kernels as K  # noqa: E402

HEADER = os.path.join(os.path.dirname(_ext.__file__), "..", "csrc", "dtb_noalloc.h")


def _codes() -> dict:
    text = open(HEADER).read()
    return {m.group(1): int(m.group(2)) for m in re.finditer(r"#define (DTB_NOALLOC_\w+) \(?(-?\d+)\)?", text)}


def _symbol():
    _ext.lib()  # make sure the library (and libtorch) is loaded into the process
    so = ctypes.CDLL(_ext.built_path())
    fn = so.dtb_layernorm_bwd_noalloc
    fn.restype = ctypes.c_int
    # the prototype in dtb_noalloc.h: 9 pointers, rows, C, accumulate, stream
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


# (rows, C, seed, with dresid, accumulate into dw/db)
CALLS = [(4096, 768, 1, True, False), (1000, 1024, 2, False, False), (2500, 512, 3, True, True),
         (777, 768, 4, False, True)]


def test_noalloc_layernorm_bwd_matches_regular_entry_point_on_calls_in_a_row():
    fn = _symbol()
    ok = _codes()["DTB_NOALLOC_OK"]
    for call, (rows, C, seed, with_res, acc) in enumerate(CALLS):
        x, w, mean, rstd, dy, dres = _inputs(rows, C, seed)
        dres = dres if with_res else None
        start_w = torch.randn(C, device="cuda") if acc else torch.full((C,), float("nan"), device="cuda")
        start_b = torch.randn(C, device="cuda") if acc else torch.full((C,), float("nan"), device="cuda")
        dw_ref, db_ref = start_w.clone(), start_b.clone()
        dx_ref = K.layernorm_bwd(dy, x, w, mean, rstd, dres, dw_ref, db_ref, accumulate=acc)
        dx = torch.empty_like(x)
        dw, db = start_w.clone(), start_b.clone()
        rc = _call(fn, x, w, mean, rstd, dy, dres, dx, dw, db, accumulate=int(acc))
        torch.cuda.synchronize()
        assert rc == ok, f"call {call}: return code {rc}"
        torch.testing.assert_close(dx.float(), dx_ref.float(), rtol=1e-2, atol=1e-2)
        torch.testing.assert_close(dw, dw_ref, rtol=1e-4, atol=1e-4)
        torch.testing.assert_close(db, db_ref, rtol=1e-4, atol=1e-4)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    fn = _symbol()
    codes = _codes()
    rows, C = 43_649, 768  # ceil(rows / 64) = 683 blocks: 2 * 683 * 768 floats > 2^20
    x = torch.empty(64, C, device="cuda", dtype=torch.bfloat16)  # never read: rejected before launch
    mean = torch.empty(64, device="cuda")
    dw = torch.empty(C, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(x.data_ptr(), x.data_ptr(), x.data_ptr(), mean.data_ptr(), mean.data_ptr(), None, x.data_ptr(),
            dw.data_ptr(), dw.data_ptr(), rows, C, 0, stream)
    assert rc == codes["DTB_NOALLOC_TOO_LARGE"]
    rc = fn(None, x.data_ptr(), x.data_ptr(), mean.data_ptr(), mean.data_ptr(), None, x.data_ptr(),
            dw.data_ptr(), dw.data_ptr(), 64, C, 0, stream)
    assert rc == codes["DTB_NOALLOC_BAD_ARGUMENT"]
