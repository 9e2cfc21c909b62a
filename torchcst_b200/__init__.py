"""B200-native (sm_100a) backend for torchcst's radius cell-mass CSTLinear hot path.

Public surface mirrors the reference names for this path::

    from torchcst_b200 import CSTLinear, CSTAdamW, ChebyshevSpec, RadiusBounds, chart_presets, kernels

Compute runs in the native library ``torchcst_b200/lib/libtcst_b200.so`` through
the C ABI declared in ``include/tcst_b200.h``; there is no CPU fallback.
"""

from .spec import (  # noqa: F401
    CellMass,
    ChebyshevSpec,
    KernelSpec,
    PolarRadius,
    RadiusBounds,
    RationalRadius,
    RegularGrid,
    chart_presets,
    kernels,
    radius_cell_mass_axes,
)

__all__ = [
    "CSTAdamW",
    "CSTLinear",
    "ChebyshevSpec",
    "RadiusBounds",
    "chart_presets",
    "kernels",
]


def __getattr__(name):
    # torch-dependent pieces load lazily so declarations stay importable without CUDA.
    if name == "CSTLinear":
        from .linear import CSTLinear
        return CSTLinear
    if name == "CSTAdamW":
        from .optim import CSTAdamW
        return CSTAdamW
    raise AttributeError(name)
