"""Runtime configuration shared by the transforms: workspace cache and the
Newton-Schulz operand precision.

The C ABI never allocates; the host keeps one growable device workspace per
(device, stream) and hands it to every call on that stream.
"""

from __future__ import annotations

import os
import threading

import torch

from . import _lib

_lock = threading.Lock()
_workspaces: dict = {}

_DEFAULT_PRECISION = os.environ.get("ROLLFAST_NS_PRECISION", "f16").lower()
if _DEFAULT_PRECISION not in _lib.PRECISIONS:
    raise ValueError(f"ROLLFAST_NS_PRECISION={_DEFAULT_PRECISION!r}: expected one of f16, bf16, f32")
_precision = _lib.PRECISIONS[_DEFAULT_PRECISION]


def set_ns_precision(name: str) -> None:
    """Newton-Schulz operand precision for subsequent updates:
    ``"f16"`` (default; 16-bit tensor-core operands, fp32 accumulation,
    power-of-two operand scaling), ``"bf16"``, or ``"f32"`` (CUDA-core fp32,
    for reference-grade parity with the reference's float32 iteration)."""
    global _precision
    key = name.lower()
    if key not in _lib.PRECISIONS:
        raise ValueError(f"unknown NS precision {name!r}")
    _precision = _lib.PRECISIONS[key]


def ns_precision() -> int:
    return _precision


def ns_precision_name(p: int | None = None) -> str:
    p = _precision if p is None else p
    return {_lib.RF_NS_F16: "f16", _lib.RF_NS_BF16: "bf16", _lib.RF_NS_F32: "f32"}[p]


_aux_streams: dict = {}


def pipelined() -> bool:
    """Overlap HBM-bound preparation / AdamW with the Newton-Schulz GEMMs on
    a second stream (ROLLFAST_PIPELINE=1; off by default: under the 1 kW power
    cap the concurrent HBM traffic costs the GEMMs more clock than it saves)."""
    return os.environ.get("ROLLFAST_PIPELINE", "0") != "0"


def aux_stream(device: torch.device) -> torch.cuda.Stream:
    """The persistent second stream of ``device``."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    with _lock:
        s = _aux_streams.get(idx)
        if s is None:
            s = torch.cuda.Stream(device=torch.device("cuda", idx))
            _aux_streams[idx] = s
        return s


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """A device buffer of at least ``nbytes`` for the current stream."""
    stream = torch.cuda.current_stream(device)
    key = (device.index if device.index is not None else torch.cuda.current_device(), stream.cuda_stream)
    with _lock:
        buf = _workspaces.get(key)
        if buf is None or buf.numel() < nbytes:
            # Round up to 2 MiB to limit re-allocations as shapes vary.
            size = max(int(nbytes), 1)
            size = (size + (1 << 21) - 1) // (1 << 21) * (1 << 21)
            buf = torch.empty(size, dtype=torch.uint8, device=device)
            _workspaces[key] = buf
        return buf


def release_workspaces() -> None:
    with _lock:
        _workspaces.clear()
