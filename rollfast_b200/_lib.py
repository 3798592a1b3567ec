"""ctypes binding of ``librollfast_b200.so`` (the C ABI in ``include/rollfast_b200.h``).

This is the same surface an XLA FFI registration would bind; every call
checks the returned ``rf_status`` and raises with the library's message.
There is no fallback: if the shared library is missing, importing the
compute entry points raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "librollfast_b200.so")

RF_OK, RF_EINVAL, RF_ECUDA, RF_ETIMEOUT, RF_ENOTSUP = 0, 1, 2, 3, 4
RF_F32, RF_BF16, RF_F16 = 0, 1, 2
RF_EMA, RF_HEAVY_BALL = 0, 1
RF_NS_F16, RF_NS_BF16, RF_NS_F32 = 0, 1, 2
RF_PRECOND_FROBENIUS, RF_PRECOND_SPECTRAL, RF_PRECOND_AOL, RF_PRECOND_SCHATTEN = 0, 1, 2, 3
PRECONDITIONING_CODES = {"frobenius": RF_PRECOND_FROBENIUS, "spectral": RF_PRECOND_SPECTRAL,
                         "aol": RF_PRECOND_AOL, "schatten": RF_PRECOND_SCHATTEN}

PRECISIONS = {"f16": RF_NS_F16, "fp16": RF_NS_F16, "float16": RF_NS_F16,
              "bf16": RF_NS_BF16, "bfloat16": RF_NS_BF16,
              "f32": RF_NS_F32, "fp32": RF_NS_F32, "float32": RF_NS_F32}

# Exported symbols of include/rollfast_b200.h (checked by the CPU test-suite).
EXPORTED = (
    "rf_muon_workspace_size",
    "rf_muon_update",
    "rf_muon_direction",
    "rf_newton_schulz_workspace_size",
    "rf_newton_schulz",
    "rf_newton_schulz_noalloc",
    "rf_muon_tail",
    "rf_adamw_update",
    "rf_adamw_workspace_size",
    "rf_last_error",
    "rf_version",
    "rf_kernel_launch_count",
    "rf_sync_check",
    "rf_error_snapshot",
    "rf_profile_begin",
    "rf_profile_end",
    "rf_apply_updates",
    "rf_ipc_export",
    "rf_ipc_open",
    "rf_ipc_close",
    "rf_peer_copy",
    "rf_flags_signal",
    "rf_flags_wait",
)


class RfApplyLeaf(ctypes.Structure):
    _fields_ = [
        ("param", ctypes.c_void_p),
        ("update", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("n", ctypes.c_int64),
        ("param_dtype", ctypes.c_int32),
        ("update_dtype", ctypes.c_int32),
        ("seed", ctypes.c_uint64),
    ]


class RfIpcHandle(ctypes.Structure):
    _fields_ = [("bytes", ctypes.c_ubyte * 64)]


class RfMuonLeaf(ctypes.Structure):
    _fields_ = [
        ("grad", ctypes.c_void_p),
        ("mu", ctypes.c_void_p),
        ("param", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("batch", ctypes.c_int64),
        ("rows", ctypes.c_int64),
        ("cols", ctypes.c_int64),
        ("grad_dtype", ctypes.c_int32),
        ("param_dtype", ctypes.c_int32),
        ("out_dtype", ctypes.c_int32),
        ("shape_scale", ctypes.c_float),
        ("decay", ctypes.c_float),
        ("skip_ns", ctypes.c_int32),
        ("mu_dtype", ctypes.c_int32),
        ("sr_seed", ctypes.c_uint64),
        ("decay_in_f32", ctypes.c_int32),
        ("magma_score", ctypes.c_void_p),
        ("magma_keep", ctypes.c_int32),
        ("apply_mode", ctypes.c_int32),
        ("apply_seed", ctypes.c_uint64),
    ]


class RfMuonParams(ctypes.Structure):
    _fields_ = [
        ("beta", ctypes.c_float),
        ("eps", ctypes.c_float),
        ("count", ctypes.c_int32),
        ("nesterov", ctypes.c_int32),
        ("accumulator", ctypes.c_int32),
        ("ns_steps", ctypes.c_int32),
        ("n_coeff_rows", ctypes.c_int32),
        ("coeffs", ctypes.POINTER(ctypes.c_float)),
        ("precision", ctypes.c_int32),
        ("lr", ctypes.c_float),
        ("fuse_tail", ctypes.c_int32),
        ("aux_stream", ctypes.c_void_p),
        ("reserve_sms", ctypes.c_int32),
        ("preconditioning", ctypes.c_int32),
        ("adaptive", ctypes.c_int32),
        ("magma_tau", ctypes.c_float),
    ]


class RfTailLeaf(ctypes.Structure):
    _fields_ = [
        ("o", ctypes.c_void_p),
        ("param", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("n", ctypes.c_int64),
        ("o_dtype", ctypes.c_int32),
        ("param_dtype", ctypes.c_int32),
        ("out_dtype", ctypes.c_int32),
        ("shape_scale", ctypes.c_float),
        ("decay", ctypes.c_float),
        ("decay_in_f32", ctypes.c_int32),
    ]


class RfAdamLeaf(ctypes.Structure):
    _fields_ = [
        ("grad", ctypes.c_void_p),
        ("mu", ctypes.c_void_p),
        ("nu", ctypes.c_void_p),
        ("param", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("n", ctypes.c_int64),
        ("grad_dtype", ctypes.c_int32),
        ("param_dtype", ctypes.c_int32),
        ("out_dtype", ctypes.c_int32),
        ("decay", ctypes.c_float),
        ("decay_rounding", ctypes.c_int32),
        ("state_dtype", ctypes.c_int32),
        ("sr_seed_mu", ctypes.c_uint64),
        ("sr_seed_nu", ctypes.c_uint64),
        ("decay_mask", ctypes.c_void_p),
        ("magma_score", ctypes.c_void_p),
        ("magma_keep", ctypes.c_int32),
        ("apply_mode", ctypes.c_int32),
        ("apply_seed", ctypes.c_uint64),
    ]


class RfAdamParams(ctypes.Structure):
    _fields_ = [
        ("b1", ctypes.c_double),
        ("b2", ctypes.c_double),
        ("eps", ctypes.c_float),
        ("eps_root", ctypes.c_float),
        ("count", ctypes.c_int32),
        ("nesterov", ctypes.c_int32),
        ("lr", ctypes.c_float),
        ("max_ctas_per_sm", ctypes.c_int32),
        ("magma_tau", ctypes.c_float),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
    ]


class RollfastError(RuntimeError):
    """A non-OK rf_status from the native library."""

    def __init__(self, status: int, message: str):
        super().__init__(f"rollfast_b200: status {status}: {message}")
        self.status = status


_lock = threading.Lock()
_lib = None


def load(path: str | None = None):
    """Load (once) and return the native library; raise if it is absent."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise ImportError(
                f"{p} not found: build it with `python -m rollfast_b200.build` "
                "(there is no non-CUDA implementation of this path)"
            )
        lib = ctypes.CDLL(p)
        vp, i32, i64, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t
        lib.rf_last_error.restype = ctypes.c_char_p
        lib.rf_last_error.argtypes = []
        lib.rf_version.argtypes = [ctypes.POINTER(i32)] * 3
        lib.rf_kernel_launch_count.restype = i64
        lib.rf_kernel_launch_count.argtypes = []
        lib.rf_sync_check.argtypes = [vp]
        lib.rf_error_snapshot.argtypes = [vp, vp]
        lib.rf_profile_begin.argtypes = []
        lib.rf_profile_end.argtypes = [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(i64),
                                       ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]
        lib.rf_muon_workspace_size.argtypes = [ctypes.POINTER(RfMuonLeaf), i32, i32, i32, ctypes.POINTER(sz)]
        lib.rf_muon_update.argtypes = [ctypes.POINTER(RfMuonLeaf), i32, ctypes.POINTER(RfMuonParams), vp, sz, vp]
        lib.rf_muon_direction.argtypes = [ctypes.POINTER(RfMuonLeaf), i32, ctypes.POINTER(RfMuonParams), vp]
        lib.rf_newton_schulz_workspace_size.argtypes = [i64, i64, i64, i32, ctypes.POINTER(sz)]
        lib.rf_newton_schulz.argtypes = [vp, i32, vp, i32, i64, i64, i64, ctypes.POINTER(ctypes.c_float), i32,
                                         i32, ctypes.c_float, i32, i32, vp, sz, vp]
        lib.rf_newton_schulz_noalloc.argtypes = [vp, i32, vp, i32, i64, i64, i64, ctypes.POINTER(ctypes.c_float),
                                                 i32, i32, ctypes.c_float, i32, vp]
        lib.rf_muon_tail.argtypes = [ctypes.POINTER(RfTailLeaf), i32, ctypes.c_float, i32, vp]
        lib.rf_adamw_update.argtypes = [ctypes.POINTER(RfAdamLeaf), i32, ctypes.POINTER(RfAdamParams), vp]
        lib.rf_adamw_workspace_size.argtypes = [ctypes.POINTER(RfAdamLeaf), i32, ctypes.POINTER(sz)]
        lib.rf_apply_updates.argtypes = [ctypes.POINTER(RfApplyLeaf), i32, i32, vp]
        lib.rf_ipc_export.argtypes = [vp, ctypes.POINTER(RfIpcHandle), ctypes.POINTER(sz)]
        lib.rf_ipc_open.argtypes = [ctypes.POINTER(RfIpcHandle), ctypes.POINTER(vp)]
        lib.rf_ipc_close.argtypes = [vp]
        lib.rf_peer_copy.argtypes = [vp, vp, sz, vp]
        lib.rf_flags_signal.argtypes = [ctypes.POINTER(vp), i32, ctypes.c_uint32, vp]
        lib.rf_flags_wait.argtypes = [vp, i32, i32, ctypes.c_uint32, ctypes.c_double, vp]
        for name in EXPORTED:
            f = getattr(lib, name)
            if name not in ("rf_last_error", "rf_kernel_launch_count"):
                f.restype = ctypes.c_int
        _lib = lib
        return lib


def check(status: int) -> None:
    if status != RF_OK:
        msg = load().rf_last_error().decode("utf-8", "replace")
        if status == RF_EINVAL:
            raise ValueError(f"rollfast_b200: {msg}")
        raise RollfastError(status, msg)


def version() -> tuple[int, int, int]:
    a, b, c = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
    check(load().rf_version(ctypes.byref(a), ctypes.byref(b), ctypes.byref(c)))
    return a.value, b.value, c.value


def kernel_launch_count() -> int:
    return int(load().rf_kernel_launch_count())


def sync_check(stream_handle: int) -> None:
    check(load().rf_sync_check(ctypes.c_void_p(stream_handle)))


def error_snapshot(dst_ptr: int, stream_handle: int) -> None:
    """Enqueue a copy of the two device error words to ``dst_ptr`` (2 int32)."""
    check(load().rf_error_snapshot(ctypes.c_void_p(dst_ptr), ctypes.c_void_p(stream_handle)))


def profile_begin() -> None:
    check(load().rf_profile_begin())


def profile_end() -> dict:
    ms, n = ctypes.c_double(), ctypes.c_int64()
    alg, exe = ctypes.c_double(), ctypes.c_double()
    check(load().rf_profile_end(ctypes.byref(ms), ctypes.byref(n), ctypes.byref(alg), ctypes.byref(exe)))
    return {"gemm_ms": ms.value, "launches": n.value, "algorithmic_flops": alg.value, "executed_flops": exe.value}


# ---------------------------------------------------------------------------
# Peer transport (multi-GPU sharded update)
# ---------------------------------------------------------------------------


def ipc_export(ptr: int) -> tuple[bytes, int]:
    """(64-byte IPC handle of the allocation holding ``ptr``, offset of ``ptr`` in it)."""
    h, off = RfIpcHandle(), ctypes.c_size_t()
    check(load().rf_ipc_export(ctypes.c_void_p(ptr), ctypes.byref(h), ctypes.byref(off)))
    return bytes(h.bytes), int(off.value)


def ipc_open(handle: bytes) -> int:
    """Base address of another process's allocation mapped into the current device."""
    if len(handle) != 64:
        raise ValueError("an IPC handle is 64 bytes")
    h = RfIpcHandle()
    ctypes.memmove(h.bytes, handle, 64)
    base = ctypes.c_void_p()
    check(load().rf_ipc_open(ctypes.byref(h), ctypes.byref(base)))
    return int(base.value)


def ipc_close(base: int) -> None:
    check(load().rf_ipc_close(ctypes.c_void_p(base)))


def peer_copy(dst: int, src: int, nbytes: int, stream_handle: int) -> None:
    check(load().rf_peer_copy(ctypes.c_void_p(dst), ctypes.c_void_p(src), ctypes.c_size_t(nbytes),
                              ctypes.c_void_p(stream_handle)))


def flags_signal(addrs, value: int, stream_handle: int) -> None:
    arr = (ctypes.c_void_p * max(len(addrs), 1))(*addrs)
    check(load().rf_flags_signal(arr, len(addrs), ctypes.c_uint32(value & 0xFFFFFFFF),
                                 ctypes.c_void_p(stream_handle)))


def flags_wait(addr: int, n: int, skip: int, target: int, timeout_s: float, stream_handle: int) -> None:
    check(load().rf_flags_wait(ctypes.c_void_p(addr), n, skip, ctypes.c_uint32(target & 0xFFFFFFFF),
                               float(timeout_s), ctypes.c_void_p(stream_handle)))
