"""rollfast_b200: B200-native Muon update hot path with rollfast's API.

Drop-in names (rollfast/__init__.py:54-72 for the Muon path):
``muon``, ``scale_by_muon``, ``scale_by_muon_shape``, ``MuonState``,
``MuonDimensionNumbers`` / ``MatrixDimensionNumbers``,
``orthogonalize_via_newton_schulz``, ``polar_express_coeffs``,
``resolve_ns_coeffs``, ``MUON_NS_COEFFS``, ``adamw``, ``scale_by_adam``.
Leaves are CUDA ``torch.Tensor`` buffers; the compute runs in
``librollfast_b200.so`` (hand-written sm_100a CUDA behind a C ABI).
"""

from . import distributed
from ._runtime import set_ns_precision
from .adam import ScaleByAdamState, adamw, scale_by_adam
from .base import GradientTransformation, apply_updates, update_and_apply
from .dimension_numbers import MatrixDimensionNumbers, MuonDimensionNumbers, WeightDimNumOrFn
from .muon import MuonState, muon, scale_by_muon, scale_by_muon_shape, scale_by_shape
from .orthogonalization import (
    DION_NS_COEFFS,
    MUON_NS_COEFFS,
    MuonNsCoeffs,
    NsCoeffs,
    orthogonalize_via_newton_schulz,
    polar_express_coeffs,
    resolve_ns_coeffs,
)
from .tree import MaskedNode

MomentumAccumulator = str

__version__ = "0.1.0"

__all__ = [
    "DION_NS_COEFFS",
    "GradientTransformation",
    "MUON_NS_COEFFS",
    "MaskedNode",
    "MatrixDimensionNumbers",
    "MomentumAccumulator",
    "MuonDimensionNumbers",
    "MuonNsCoeffs",
    "MuonState",
    "NsCoeffs",
    "ScaleByAdamState",
    "WeightDimNumOrFn",
    "adamw",
    "apply_updates",
    "distributed",
    "muon",
    "orthogonalize_via_newton_schulz",
    "polar_express_coeffs",
    "resolve_ns_coeffs",
    "scale_by_adam",
    "scale_by_muon",
    "scale_by_muon_shape",
    "scale_by_shape",
    "set_ns_precision",
    "update_and_apply",
]
