"""Thin host wrappers over the C ABI: shapes, workspaces and stream plumbing.

Tensors are allocated with torch (device memory and the current CUDA stream are
torch's); every computation happens in the native sm_100a library. There is no
CPU path: calling these with CPU tensors raises.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _native as N
from .spec import AxisDecl, KernelSpec, PolarRadius, RationalRadius, _f32


def pad4(n: int) -> int:
    return (int(n) + 3) & ~3


def _vp(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device=None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def on_device(device):
    """Context that makes ``device`` the current CUDA device for the native calls
    inside it (the C ABI works on the current device and its streams); free when
    it already is."""
    return torch.cuda.device(device)


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and (not t.is_cuda):
            raise ValueError("the B200 backend requires CUDA tensors (it has no CPU fallback)")


def native_axis(a: AxisDecl) -> N.Axis:
    return N.Axis(a.site_count, a.base_tile_sites, a.merge_factor, a.modes, float(a.spacing),
                  float(a.origin))


def native_coordinates(kernel: KernelSpec) -> N.Coordinates:
    c = kernel.coordinates
    out = N.Coordinates()
    if isinstance(c, RationalRadius):
        out.kind = N.TCST_RATIONAL
        out.amplitude_max = _f32(c.amplitude_max)
        out.radius_min = _f32(c.radius_min)
        out.radius_birth = _f32(c.radius_birth)
        out.radius_max = _f32(c.radius_max)
    elif isinstance(c, PolarRadius):
        out.kind = N.TCST_POLAR
        out.amplitude_max = _f32(c.amplitude_max)
        out.w_c = _f32(c.w_c)
        out.kappa = _f32(c.kappa)
        out.lower_kappa = _f32(c.lower_kappa)
        out.upper_decay_power = _f32(c.upper_decay_power)
        ob, ib = c.output_bounds, c.input_bounds
        for i, v in enumerate((ob.minimum, ob.birth, ob.maximum, ob.upper_floor)):
            out.out_bounds[i] = _f32(v)
        for i, v in enumerate((ib.minimum, ib.birth, ib.maximum, ib.upper_floor)):
            out.in_bounds[i] = _f32(v)
    else:
        raise TypeError("unsupported coordinates")
    return out


@dataclass
class Plan:
    """Static native description of one layer."""

    out_axis: N.Axis
    in_axis: N.Axis
    coords: N.Coordinates
    n_out: int
    n_in: int
    kind: int

    @classmethod
    def make(cls, axes, kernel):
        oa, ia = axes
        return cls(native_axis(oa), native_axis(ia), native_coordinates(kernel), oa.site_count,
                   ia.site_count, native_coordinates(kernel).kind)

    def table_bytes(self, atoms: int) -> int:
        return int(N.load().tcst_atom_table_bytes(atoms, ctypes.byref(self.out_axis),
                                                   ctypes.byref(self.in_axis)))


class Workspace:
    """Persistent per-device scratch of one layer: the weight assembly's
    fixed-point plane for wide atoms and the status word."""

    def __init__(self, plan: Plan, device):
        self.plan = plan
        self.device = torch.device(device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._scratch = None

    def scratch(self, atoms: int):
        need = int(N.load().tcst_weight_scratch_bytes(atoms, ctypes.byref(self.plan.out_axis),
                                                       ctypes.byref(self.plan.in_axis)))
        if self._scratch is None or self._scratch.numel() * 4 < need:
            self._scratch = torch.empty((need + 15) // 16 * 4, dtype=torch.int32, device=self.device)
        return self._scratch


def decode_route(plan: Plan, p, status, *, owner_keys=None, routing=None):
    require_cuda(p)
    atoms = p.shape[0]
    table = torch.empty(max(plan.table_bytes(atoms) // 4, 1), dtype=torch.float32, device=p.device)
    N.call("tcst_decode_route", _vp(p), atoms, ctypes.byref(plan.out_axis),
           ctypes.byref(plan.in_axis), ctypes.byref(plan.coords), _vp(table), _vp(owner_keys),
           _vp(routing), _vp(status), _stream(p.device))
    return table


def assemble_weight(plan: Plan, table, atoms, ws: Workspace, *, dense=False, split=True):
    dev = ws.device
    scratch = ws.scratch(atoms)
    ld = pad4(plan.n_in)
    w = torch.empty(plan.n_out, plan.n_in, dtype=torch.float32, device=dev) if dense else None
    hi = lo = None
    if split:
        hi = torch.empty(plan.n_out, ld, dtype=torch.float32, device=dev)
        lo = torch.empty(plan.n_out, ld, dtype=torch.float32, device=dev)
    N.call("tcst_assemble_weight", _vp(table), atoms, ctypes.byref(plan.out_axis),
           ctypes.byref(plan.in_axis), _vp(scratch), scratch.numel() * 4, _vp(w), plan.n_in,
           _vp(hi), _vp(lo), ld, _stream(dev))
    return w, hi, lo, ld


def assemble_weight_f16(plan: Plan, table, atoms, ws: Workspace):
    """W assembled straight into f16 split planes (with max |W| and its scale)."""
    dev = ws.device
    scratch = ws.scratch(atoms)
    w = torch.empty(plan.n_out, plan.n_in, dtype=torch.float32, device=dev)
    sp = F16Split(plan.n_out, plan.n_in, dev)
    sp.amax.zero_()
    N.call("tcst_assemble_weight_f16", _vp(table), atoms, ctypes.byref(plan.out_axis),
           ctypes.byref(plan.in_axis), _vp(scratch), scratch.numel() * 4, _vp(w), plan.n_in,
           _vp(sp.amax), _vp(sp.hi), _vp(sp.lo), sp.ld, _vp(sp.scale), _stream(dev))
    return sp


def assemble_weight_window_f16(plan: Plan, table, atoms, ws: Workspace, row0, rows, col0, cols):
    """W[row0 : row0 + rows, col0 : col0 + cols] (fp32) and its f16 split planes."""
    dev = ws.device
    scratch = ws.scratch(atoms)
    w = torch.empty(rows, cols, dtype=torch.float32, device=dev)
    sp = F16Split(rows, cols, dev)
    sp.amax.zero_()
    N.call("tcst_assemble_weight_window_f16", _vp(table), atoms, ctypes.byref(plan.out_axis),
           ctypes.byref(plan.in_axis), _vp(scratch), scratch.numel() * 4, row0, rows, col0,
           cols, _vp(w), cols, _vp(sp.amax), _vp(sp.hi), _vp(sp.lo), sp.ld, _vp(sp.scale),
           _stream(dev))
    return w, sp


def split_tf32(x):
    """Two-term TF32 split of a 2-D float32 CUDA tensor into padded planes."""
    require_cuda(x)
    rows, cols = x.shape
    ld = pad4(cols)
    hi = torch.empty(rows, ld, dtype=torch.float32, device=x.device)
    lo = torch.empty(rows, ld, dtype=torch.float32, device=x.device)
    if rows * cols == 0:
        return hi, lo, ld
    if x.stride(1) != 1:
        x = x.contiguous()
    N.call("tcst_split_tf32", _vp(x), rows, cols, x.stride(0), _vp(hi), _vp(lo), ld,
           _stream(x.device))
    return hi, lo, ld


def pad8(n: int) -> int:
    return (n + 7) // 8 * 8


class F16Split:
    """F16 hi/lo planes of one float32 matrix plus its device-side absmax and
    power-of-two scale (own storage, or views into a caller's buffers)."""

    def __init__(self, rows, cols, device, *, amax=None, scale=None):
        self.rows, self.cols, self.ld = rows, cols, pad8(cols)
        self.hi = torch.empty(rows, self.ld, dtype=torch.float16, device=device)
        self.lo = torch.empty_like(self.hi)
        if amax is None:
            words = torch.zeros(2, dtype=torch.float32, device=device)
            amax, scale = words[0:1], words[1:2]
        self.amax, self.scale = amax, scale

    @property
    def scale_ptr(self):
        return self.scale.data_ptr()

    def fill(self, x, *, amax_ready=False):
        """Split float32 x [rows][cols] (strided rows); with ``amax_ready`` the
        caller already folded max |x| into a zeroed ``self.amax``."""
        st = _stream(x.device)
        if not amax_ready:
            self.amax.zero_()
            N.call("tcst_absmax", _vp(x), self.rows, self.cols, x.stride(0), _vp(self.amax), st)
        N.call("tcst_split_f16", _vp(x), self.rows, self.cols, x.stride(0), _vp(self.amax),
               _vp(self.hi), _vp(self.lo), self.ld, _vp(self.scale), st)
        return self


def gemm_f16(M, N_, K, a: F16Split, a_mn, b: F16Split, b_mn, c, ldc, status, *, split_k=1,
             split_stride=0):
    N.call("tcst_gemm_f16x3", M, N_, K, _vp(a.hi), _vp(a.lo), a.ld, int(a_mn),
           ctypes.c_void_p(a.scale_ptr), _vp(b.hi), _vp(b.lo), b.ld, int(b_mn),
           ctypes.c_void_p(b.scale_ptr), _vp(c), ldc, split_k, split_stride, _vp(status),
           _stream(c.device))


def gemm(M, N_, K, a, lda, a_mn, b, ldb, b_mn, c, ldc, status, *, split_k=1, split_stride=0):
    """C[s] = A B^T over a K slice s (three-product TF32 split on tcgen05)."""
    N.call("tcst_gemm_tf32x3", M, N_, K, _vp(a[0]), _vp(a[1]), lda, int(a_mn), _vp(b[0]),
           _vp(b[1]), ldb, int(b_mn), _vp(c), ldc, split_k, split_stride, _vp(status),
           _stream(c.device))


def pullback(plan: Plan, table, atoms, g, ldg, split, split_stride, device):
    grad = torch.empty(atoms, 4, dtype=torch.float32, device=device)
    N.call("tcst_pullback", _vp(table), atoms, ctypes.byref(plan.out_axis),
           ctypes.byref(plan.in_axis), _vp(g), ldg, split, split_stride, _vp(grad),
           _stream(device))
    return grad


def pullback_band(plan: Plan, table, atoms, g, ldg, split, split_stride, row0, rows, device):
    """Atom gradients from the G rows [row0, row0 + rows) alone (g holds them)."""
    grad = torch.empty(atoms, 4, dtype=torch.float32, device=device)
    N.call("tcst_pullback_band", _vp(table), atoms, ctypes.byref(plan.out_axis),
           ctypes.byref(plan.in_axis), _vp(g), ldg, split, split_stride, row0, rows, _vp(grad),
           _stream(device))
    return grad


def weight_split_k(plan: Plan, rows: int, sm_count: int = 148) -> int:
    """Split-K factor of the dW = dY^T X GEMM: enough CTAs to cover the SMs."""
    tiles = -(-plan.n_out // 128) * -(-plan.n_in // 256)
    kblocks = max(1, -(-rows // 32))
    return int(max(1, min(8, kblocks, sm_count // max(tiles, 1))))


def atom_energies(plan: Plan, table, atoms, device):
    e = torch.empty(atoms, dtype=torch.float64, device=device)
    N.call("tcst_atom_energies", _vp(table), atoms, ctypes.byref(plan.out_axis),
           ctypes.byref(plan.in_axis), _vp(e), _stream(device))
    return e


class ScalarRing:
    """Per-launch optimizer scalars for steps replayed from a CUDA graph, with no
    host-to-device copy in front of the replay: a ring of slots in pinned host
    memory, a device state block that ``fetch`` (``tcst_scalar_ring_fetch``, one
    CTA reading the ring through its device mapping) fills from the next slot
    and that ``launch`` (``tcst_optimizer_step_ring``) reads, and one event per
    slot marking when its fetch has run. Every ``write`` must be followed by
    exactly one ``fetch`` execution (eager or replayed), before its ``launch``."""

    SLOTS = 64

    def __init__(self, device):
        size = ctypes.sizeof(N.AdamW)
        self.seq_offset = (size + 15) // 16 * 16
        self.slot_bytes = self.seq_offset + 16
        self.host = torch.zeros(self.SLOTS, self.slot_bytes, dtype=torch.uint8).pin_memory()
        # [use count, valid, -, -, tcst_adamw]
        self.state = torch.zeros((16 + self.seq_offset) // 4, dtype=torch.int32, device=device)
        self.events = [None] * self.SLOTS
        self.uses = 0
        self._pending = None

    def write(self, h):
        """Fill the next fetch's slot from the ``N.AdamW`` struct ``h`` (host
        side, before that fetch is enqueued on the current stream)."""
        if self._pending is not None:
            # Recorded after the previous fetch was enqueued: it fires once
            # that fetch has read its slot.
            ev = torch.cuda.Event()
            ev.record()
            self.events[self._pending] = ev
        slot = self.uses % self.SLOTS
        ev = self.events[slot]
        if ev is not None:
            ev.synchronize()
        base = self.host[slot].data_ptr()
        ctypes.memmove(base, ctypes.addressof(h), ctypes.sizeof(h))
        ctypes.c_uint32.from_address(base + self.seq_offset).value = self.uses & 0xFFFFFFFF
        self._pending = slot
        self.uses += 1

    def fetch(self, status, stream):
        """Enqueue the copy of the next slot into the device state (capturable)."""
        N.call("tcst_scalar_ring_fetch", _vp(self.host), self.SLOTS, self.slot_bytes,
               _vp(self.state), _vp(status), stream)

    def launch(self, p, grad, exp_avg, exp_avg_sq, kind, stream):
        """Enqueue the optimizer step on the fetched scalars (capturable)."""
        N.call("tcst_optimizer_step_ring", _vp(p), _vp(grad), _vp(exp_avg), _vp(exp_avg_sq),
               p.shape[0], kind, _vp(self.state), stream)


def status_error(code: int) -> str | None:
    if code == 0:
        return None
    parts = []
    if code & N.STATUS_NONFINITE:
        parts.append("atom parameters must be finite")
    if code & N.STATUS_BOUNDS:
        parts.append("rational radius requires finite rows, q in [0,1] and bounded amplitude")
    if code & N.STATUS_RADIUS:
        parts.append("radius must lie in (0, chart period/2]")
    if code & N.STATUS_TIMEOUT:
        parts.append("a bounded device wait expired")
    if code & N.STATUS_FOOTPRINT:
        parts.append("footprint exceeds this build's limits")
    if code & N.STATUS_SEQUENCE:
        parts.append("an optimizer scalar ring slot was out of step (no update applied)")
    return "; ".join(parts)


def f32(x) -> float:
    return float(np.float32(x))
