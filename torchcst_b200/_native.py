"""ctypes binding of the C ABI in ``include/tcst_b200.h``.

The shared object is ``torchcst_b200/lib/libtcst_b200.so`` (built in-tree by
``torchcst_b200/build.py``). There is no CPU fallback: every compute entry point
raises if the library or a CUDA device is missing.
"""

from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libtcst_b200.so")

TCST_RATIONAL = 0
TCST_POLAR = 1

STATUS_NONFINITE = 1
STATUS_BOUNDS = 2
STATUS_RADIUS = 4
STATUS_TIMEOUT = 8
STATUS_FOOTPRINT = 16
STATUS_SEQUENCE = 32


class Axis(ctypes.Structure):
    _fields_ = [
        ("site_count", ctypes.c_int32),
        ("base_tile_sites", ctypes.c_int32),
        ("merge_factor", ctypes.c_int32),
        ("modes", ctypes.c_int32),
        ("spacing", ctypes.c_double),
        ("origin", ctypes.c_double),
    ]


class Coordinates(ctypes.Structure):
    _fields_ = [
        ("kind", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("amplitude_max", ctypes.c_double),
        ("radius_min", ctypes.c_double),
        ("radius_birth", ctypes.c_double),
        ("radius_max", ctypes.c_double),
        ("w_c", ctypes.c_double),
        ("kappa", ctypes.c_double),
        ("lower_kappa", ctypes.c_double),
        ("upper_decay_power", ctypes.c_double),
        ("out_bounds", ctypes.c_double * 4),
        ("in_bounds", ctypes.c_double * 4),
    ]


class AdamW(ctypes.Structure):
    _fields_ = [
        ("lerp_weight", ctypes.c_float),
        ("beta2", ctypes.c_float),
        ("one_minus_beta2", ctypes.c_float),
        ("neg_step_size", ctypes.c_float),
        ("bias2_sqrt", ctypes.c_float),
        ("eps", ctypes.c_float),
        ("decay_factor", ctypes.c_float),
        ("has_decay", ctypes.c_int32),
        ("field_ratio", ctypes.c_float * 4),
        ("field_mask", ctypes.c_int32),
        ("amplitude_cap", ctypes.c_float),
        ("polar_amplitude_max", ctypes.c_float),
        ("polar_w_c", ctypes.c_float),
        ("polar_activity_gain", ctypes.c_float),
        ("polar_dormant_q_scale", ctypes.c_float),
        ("polar_decay", ctypes.c_float),
        ("polar_energy_step", ctypes.c_float),
        ("period_out", ctypes.c_float),
        ("period_in", ctypes.c_float),
        ("amplitude_decay", ctypes.c_float),
    ]


P = ctypes.c_void_p
I64 = ctypes.c_int64
I32 = ctypes.c_int32

# name -> (restype, argtypes); mirrors include/tcst_b200.h exactly.
SIGNATURES = {
    "tcst_version": (ctypes.c_char_p, []),
    "tcst_last_error": (ctypes.c_char_p, []),
    "tcst_atom_table_bytes": (I64, [I64, ctypes.POINTER(Axis), ctypes.POINTER(Axis)]),
    "tcst_decode_route": (ctypes.c_int, [P, I64, ctypes.POINTER(Axis), ctypes.POINTER(Axis),
                                         ctypes.POINTER(Coordinates), P, P, P, P, P]),
    "tcst_weight_scratch_bytes": (I64, [I64, ctypes.POINTER(Axis), ctypes.POINTER(Axis)]),
    "tcst_assemble_weight": (ctypes.c_int, [P, I64, ctypes.POINTER(Axis), ctypes.POINTER(Axis),
                                            P, I64, P, I64, P, P, I64, P]),
    "tcst_assemble_weight_static": (ctypes.c_int, [P, I64, ctypes.POINTER(Axis),
                                                   ctypes.POINTER(Axis), P, I64, P, P, I64, P]),
    "tcst_static_weight_scratch_bytes": (I64, []),
    "tcst_split_tf32": (ctypes.c_int, [P, I64, I64, I64, P, P, I64, P]),
    "tcst_gemm_tf32x3": (ctypes.c_int, [I64, I64, I64, P, P, I64, I32, P, P, I64, I32,
                                        P, I64, I32, I64, P, P]),
    "tcst_gemm_f16x3": (ctypes.c_int, [I64, I64, I64, P, P, I64, I32, P, P, P, I64, I32, P, P,
                                       I64, I32, I64, P, P]),
    "tcst_gemm_f16x3_mse": (ctypes.c_int, [I64, I64, I64, P, P, I64, P, P, P, I64, P, P, I64,
                                           ctypes.c_float, P, I64, P, ctypes.POINTER(I32), P,
                                           P, P]),
    "tcst_assemble_weight_f16": (ctypes.c_int, [P, I64, ctypes.POINTER(Axis), ctypes.POINTER(Axis),
                                                P, I64, P, I64, P, P, P, I64, P, P]),
    "tcst_assemble_weight_window_f16": (ctypes.c_int, [P, I64, ctypes.POINTER(Axis),
                                                       ctypes.POINTER(Axis), P, I64, I64, I64,
                                                       I64, I64, P, I64, P, P, P, I64, P, P]),
    "tcst_absmax": (ctypes.c_int, [P, I64, I64, I64, P, P]),
    "tcst_split_f16": (ctypes.c_int, [P, I64, I64, I64, P, P, P, I64, P, P]),
    "tcst_mse_grad_f32": (ctypes.c_int, [P, P, I64, I64, I64, ctypes.c_float, P, I64, P,
                                         ctypes.POINTER(I32), P, P]),
    "tcst_pullback": (ctypes.c_int, [P, I64, ctypes.POINTER(Axis), ctypes.POINTER(Axis),
                                     P, I64, I32, I64, P, P]),
    "tcst_pullback_band": (ctypes.c_int, [P, I64, ctypes.POINTER(Axis), ctypes.POINTER(Axis),
                                          P, I64, I32, I64, I64, I64, P, P]),
    "tcst_optimizer_step": (ctypes.c_int, [P, P, P, P, I64, I32, ctypes.POINTER(AdamW), P]),
    "tcst_optimizer_step_device": (ctypes.c_int, [P, P, P, P, I64, I32, P, P]),
    "tcst_scalar_ring_fetch": (ctypes.c_int, [P, I32, I64, P, P, P]),
    "tcst_optimizer_step_ring": (ctypes.c_int, [P, P, P, P, I64, I32, P, P]),
    "tcst_coordinate_update": (ctypes.c_int, [P, P, I64, I32, ctypes.POINTER(AdamW), P]),
    "tcst_mse_grad": (ctypes.c_int, [P, P, I64, I64, I64, ctypes.c_float, P, P, I64, P,
                                     ctypes.POINTER(I32), P]),
    "tcst_atom_energies": (ctypes.c_int, [P, I64, ctypes.POINTER(Axis), ctypes.POINTER(Axis),
                                          P, P]),
}

_lock = threading.Lock()
_lib = None


def load(path: str = LIB_PATH):
    """Load the native library once; raise with a clear message if it is missing."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(
                f"torchcst_b200 native library not found at {path}; run "
                "`python -m torchcst_b200.build` (this backend has no CPU fallback)")
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


class NativeError(RuntimeError):
    pass


def check(rc: int, what: str):
    if rc != 0:
        msg = load().tcst_last_error().decode(errors="replace")
        kind = {1: ValueError, 2: NativeError, 3: NotImplementedError}.get(rc, NativeError)
        raise kind(f"{what}: {msg}")


def call(name: str, *args):
    rc = getattr(load(), name)(*args)
    check(rc, name)
    return rc


def exported_symbols():
    return tuple(SIGNATURES)
