"""rf_newton_schulz_noalloc: the Newton-Schulz entry point for callers that
cannot allocate device memory (e.g. an XLA FFI handler whose framework has
reserved the GPU for its own pool, or a fixed-budget deployment).  It takes
its workspace from a static device array instead of a caller buffer.

Checked through the C ABI against the ordinary rf_newton_schulz (caller
workspace) on the same input, on two calls in a row (the array is shared
and keeps the previous call's contents), plus the size limit.  This file is
collected last so a failure here leaves every other test already run.
"""

import ctypes

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


def _call_existing(lib, _lib, x, out, coeffs, rows, prec, stream):
    n = ctypes.c_size_t()
    b, r, c = x.shape
    _lib.check(lib.rf_newton_schulz_workspace_size(b, r, c, prec, ctypes.byref(n)))
    ws = torch.empty(n.value, dtype=torch.uint8, device=x.device)
    _lib.check(lib.rf_newton_schulz(x.data_ptr(), _lib.RF_F32, out.data_ptr(), _lib.RF_F32, b, r, c, coeffs, rows,
                                    5, 1e-8, _lib.RF_PRECOND_FROBENIUS, prec, ws.data_ptr(), ws.numel(), stream))
    return ws


def test_noalloc_matches_workspace_entry_point_twice():
    from rollfast_b200 import _lib

    lib = _lib.load()
    dev = torch.device("cuda:0")
    stream = torch.cuda.current_stream(dev).cuda_stream
    c = O.resolve_ns_coeffs("polar_express", 5)
    coeffs = (ctypes.c_float * c.size)(*c.reshape(-1).tolist())
    rows = c.shape[0]
    for prec in (_lib.RF_NS_F16, _lib.RF_NS_F32):
        for call, (shape, seed) in enumerate((((2, 256, 768), 1), ((3, 640, 200), 2))):
            x = torch.from_numpy(np.random.default_rng(seed).standard_normal(shape).astype(np.float32)).to(dev)
            ref = torch.empty_like(x)
            ws = _call_existing(lib, _lib, x, ref, coeffs, rows, prec, stream)
            got = torch.full_like(x, float("nan"))
            b, r, cc = shape
            _lib.check(lib.rf_newton_schulz_noalloc(x.data_ptr(), _lib.RF_F32, got.data_ptr(), _lib.RF_F32, b, r,
                                                    cc, coeffs, rows, 5, 1e-8, prec, stream))
            torch.cuda.synchronize()
            _lib.sync_check(stream)
            del ws
            err = float(torch.linalg.vector_norm(got - ref) / torch.linalg.vector_norm(ref))
            # Same kernels on the same data: identical up to the 16-bit path's tolerance.
            assert err <= 1e-5, (prec, call, err)
            oracle = O.quintic_newton_schulz(x.cpu().numpy(), c, 5)
            e_or = float(np.linalg.norm(got.cpu().numpy() - oracle) / np.linalg.norm(oracle))
            assert e_or <= (1e-2 if prec == _lib.RF_NS_F16 else 1e-5), (prec, call, e_or)


def test_noalloc_rejects_problems_beyond_the_static_scratch():
    from rollfast_b200 import _lib

    lib = _lib.load()
    dev = torch.device("cuda:0")
    n = ctypes.c_size_t()
    _lib.check(lib.rf_newton_schulz_workspace_size(1, 4096, 4096, _lib.RF_NS_F16, ctypes.byref(n)))
    assert n.value > (32 << 20)
    x = torch.zeros((1, 8, 8), device=dev)  # pointers only; the size check comes first
    c = (ctypes.c_float * 3)(3.4445, -4.7750, 2.0315)
    st = lib.rf_newton_schulz_noalloc(x.data_ptr(), _lib.RF_F32, x.data_ptr(), _lib.RF_F32, 1, 4096, 4096, c, 0, 5,
                                      1e-8, _lib.RF_NS_F16, torch.cuda.current_stream(dev).cuda_stream)
    assert st == _lib.RF_EINVAL
    assert b"static scratch" in lib.rf_last_error()
