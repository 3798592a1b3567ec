"""Newton-Schulz coefficients and the ``orthogonalize_fn`` plugin seam
(restates src/rollfast/optim/orthogonalization.py).

Coefficient schedules are host-side float64 NumPy, exactly as the reference
computes them (orthogonalization.py:58-147).  ``orthogonalize_via_newton_schulz``
runs on the GPU through ``rf_newton_schulz``.
"""

from __future__ import annotations

import ctypes
from typing import Any, Callable, Literal, Sequence

import numpy as np
import torch

from . import _lib, _runtime
from .base import rf_dtype, require_cuda, stream_handle
from .dimension_numbers import MatrixDimensionNumbers, _compute_matrix_layout
from .tree import is_aux_leaf

MuonPreconditioning = Literal["frobenius", "spectral", "aol", "schatten"]
NsCoeffTriple = tuple
NsCoeffs = Any
MuonNsCoeffs = NsCoeffs
OrthogonalizeFn = Callable[..., torch.Tensor]

MUON_NS_COEFFS = (3.4445, -4.7750, 2.0315)  # orthogonalization.py:42
DION_NS_COEFFS = (  # orthogonalization.py:43-49
    (4.0848, -6.8946, 2.9270),
    (3.9505, -6.3029, 2.6377),
    (3.7418, -5.5913, 2.3037),
    (2.8769, -3.1427, 1.2046),
    (2.8366, -3.0525, 1.2012),
)
NS_COEFFS_PRESETS = {"standard": MUON_NS_COEFFS, "dion": DION_NS_COEFFS}
_PRECONDITIONINGS = ("frobenius", "spectral", "aol", "schatten")


def _optimal_quintic(l: float, u: float) -> tuple[float, float, float]:
    """orthogonalization.py:58-84: odd quintic with equal-ripple error on
    [l, u], by Remez exchange on the two interior extrema."""
    if not 0 < l <= u:
        raise ValueError(f"l must satisfy 0 < l <= u, got l={l}, u={u}.")
    if l / u >= 1 - 1e-5:
        return (15 / 8) / u, (-10 / 8) / (u**3), (3 / 8) / (u**5)
    q, r = (3 * l + u) / 4, (l + 3 * u) / 4
    err, prev = np.inf, None
    a = b = c = 0.0
    for _ in range(1000):
        if prev is not None and abs(prev - err) <= 1e-15:
            break
        prev = err
        system = np.array(
            [[l, l**3, l**5, 1], [q, q**3, q**5, -1], [r, r**3, r**5, 1], [u, u**3, u**5, -1]]
        )
        a, b, c, err = np.linalg.solve(system, np.ones(4))
        q, r = np.sqrt((-3 * b + np.array([-1, 1]) * np.sqrt(9 * b**2 - 20 * a * c)) / (10 * c))
    return float(a), float(b), float(c)


def polar_express_coeffs(l: float = 1e-3, num_iters: int = 8, *, safety_factor_eps: float = 2e-2,
                         cushion: float = 0.02407327424182761) -> list[tuple[float, float, float]]:
    """orthogonalization.py:87-119: PolarExpress per-step coefficients."""
    u = 1.0
    if not 0 < l <= u:
        raise ValueError(f"l must satisfy 0 < l <= 1, got {l}.")
    if num_iters < 1:
        raise ValueError(f"num_iters must be >= 1, got {num_iters}.")
    sf = 1 + safety_factor_eps
    out = []
    for i in range(num_iters):
        a, b, c = _optimal_quintic(max(l, cushion * u), u)
        if cushion * u > l:
            pl = a * l + b * l**3 + c * l**5
            pu = a * u + b * u**3 + c * u**5
            k = 2 / (pl + pu)
            a, b, c = a * k, b * k, c * k
        if i < num_iters - 1:
            a, b, c = a / sf, b / sf**3, c / sf**5
        out.append((a, b, c))
        l = a * l + b * l**3 + c * l**5
        u = 2 - l
    return out


def resolve_ns_coeffs(ns_coeffs: NsCoeffs, ns_steps) -> torch.Tensor:
    """orthogonalization.py:122-147: preset / triple / ordered schedule ->
    float32 (3,) or (n, 3) tensor (host)."""
    n = int(ns_steps)
    if isinstance(ns_coeffs, str):
        if ns_coeffs == "polar_express":
            coeffs = polar_express_coeffs(num_iters=n)
        elif ns_coeffs in NS_COEFFS_PRESETS:
            coeffs = NS_COEFFS_PRESETS[ns_coeffs]
        else:
            raise ValueError(f"Unknown ns_coeff preset string: {ns_coeffs}")
    elif isinstance(ns_coeffs, torch.Tensor):
        coeffs = ns_coeffs.detach().cpu().numpy()
    else:
        coeffs = ns_coeffs
    arr = np.asarray(coeffs, dtype=np.float32)
    if arr.ndim > 2 or arr.shape[-1] != 3:
        raise ValueError(f"ns_coeffs must have shape (3,) or (n, 3), got {tuple(arr.shape)}")
    if arr.ndim == 2:
        if arr.shape[0] < n:
            raise ValueError(f"Not enough coeffs to perform {ns_steps} steps")
        arr = arr[:n]
    return torch.from_numpy(np.ascontiguousarray(arr))


_resolve_ns_coeffs = resolve_ns_coeffs


def coeff_buffer(ns_coeffs):
    """(ctypes float array, n_coeff_rows) for the C ABI: rows 0 marks a single
    (3,) triple repeated ns_steps times (orthogonalization.py:253-260); an
    (n, 3) schedule runs all n rows in order (orthogonalization.py:262-269)."""
    c = torch.as_tensor(ns_coeffs).detach().to("cpu", torch.float32).contiguous()
    if c.ndim not in (1, 2) or c.shape[-1] != 3 or (c.ndim == 2 and c.shape[0] == 0):
        raise ValueError(
            f"Newton-Schulz coefficients must have shape (3,) or (n, 3), got {tuple(c.shape)}."
        )
    flat = c.reshape(-1).tolist()
    return (ctypes.c_float * len(flat))(*flat), (0 if c.ndim == 1 else c.shape[0])


def quintic_newton_schulz(x: torch.Tensor, ns_coeffs: torch.Tensor, ns_steps: int = 5,
                          preconditioning: MuonPreconditioning = "frobenius", eps: float = 1e-8,
                          *, out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """orthogonalization.py:211-273 over the last two axes of ``x`` (fp32
    output, like the reference's float32 iteration), with any of the
    reference's preconditionings (frobenius, spectral, aol, schatten)."""
    if preconditioning not in _PRECONDITIONINGS:
        raise ValueError(f"Unknown preconditioning {preconditioning!r}.")
    if x.ndim < 2:
        raise ValueError(f"Input must have rank >= 2, got shape={tuple(x.shape)}.")
    require_cuda(x, "x")
    cbuf, rows = coeff_buffer(ns_coeffs)
    xc = x.contiguous()
    if xc.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        xc = xc.float()
    batch = int(np.prod(xc.shape[:-2])) if xc.ndim > 2 else 1
    r, c = int(xc.shape[-2]), int(xc.shape[-1])
    out = torch.empty(xc.shape, dtype=out_dtype, device=xc.device)
    lib = _lib.load()
    prec = _runtime.ns_precision()
    nbytes = ctypes.c_size_t()
    _lib.check(lib.rf_newton_schulz_workspace_size(batch, r, c, prec, ctypes.byref(nbytes)))
    ws = _runtime.workspace(xc.device, nbytes.value)
    _lib.check(lib.rf_newton_schulz(xc.data_ptr(), rf_dtype(xc), out.data_ptr(), rf_dtype(out), batch, r, c,
                                    cbuf, rows, int(ns_steps), float(eps),
                                    _lib.PRECONDITIONING_CODES[preconditioning], prec, ws.data_ptr(), ws.numel(),
                                    stream_handle(xc)))
    return out


def orthogonalize_via_newton_schulz(x, ns_coeffs, ns_steps=5, preconditioning: MuonPreconditioning = "frobenius",
                                    eps=1e-8, dimension_numbers: MatrixDimensionNumbers | None = None):
    """orthogonalization.py:276-305."""
    if is_aux_leaf(x):
        return x
    if x.ndim != 2 and not isinstance(dimension_numbers, MatrixDimensionNumbers):
        raise ValueError(
            "Input must have shape (m, n) or weight dimension numbers must be "
            f"provided. Got shape={tuple(x.shape)} and dimension_numbers={dimension_numbers}."
        )
    if x.ndim == 2:
        dimension_numbers = MatrixDimensionNumbers(reduction_axis=0, output_axis=1)
    lay = _compute_matrix_layout(x.shape, x.dtype, dimension_numbers)
    mat = x.permute(lay.perm).reshape(lay.flat_shape) if not lay.is_identity else x.reshape(lay.flat_shape)
    ortho = quintic_newton_schulz(mat, ns_coeffs, ns_steps, preconditioning, eps)
    return ortho.reshape(lay.unflat_shape).permute(lay.inv_perm)


__all__ = [
    "DION_NS_COEFFS",
    "MUON_NS_COEFFS",
    "MuonNsCoeffs",
    "MuonPreconditioning",
    "NS_COEFFS_PRESETS",
    "NsCoeffs",
    "OrthogonalizeFn",
    "orthogonalize_via_newton_schulz",
    "polar_express_coeffs",
    "quintic_newton_schulz",
    "resolve_ns_coeffs",
]
