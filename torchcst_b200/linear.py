"""CSTLinear on the B200 backend: a drop-in for torchcst's radius cell-mass Linear.

``CSTLinear(charts=(out, in), atoms=..., kernel=product(cell_mass(...), coordinates=...))``
keeps the reference constructor, atom layout ([A, 4] float32 rows in the original
order, reachable as ``layer.atoms.p`` and saved under ``atom_state.atoms.p``),
constructor-default initialization (same torch RNG calls as
_backends/torch/kernels/radius_cell_mass.py:126-159 and polar_amp_width.py:25-50)
and forward semantics (nn/linear.py:384-417). Forward and backward run the
native sm_100a path; there is no CPU fallback.
"""

from __future__ import annotations

import math

import torch
from torch import nn
from torch.autograd.function import once_differentiable

from . import runtime as R
from .spec import KernelSpec, PolarRadius, RationalRadius, RegularGrid, radius_cell_mass_axes


class _CellMassLinear(torch.autograd.Function):
    """Y = X W^T with W assembled from atoms; backward gives dX and p.grad.

    X, W and dY enter the tensor cores as f16 hi/lo planes with per-tensor
    power-of-two scales (three products, float32-accurate; see
    ``tcst_gemm_f16x3``)."""

    @staticmethod
    def forward(ctx, x, p, layer):
        ws = layer._workspace(x.device)
        plan = layer._plan
        atoms = p.shape[0]
        dev = x.device
        table = R.decode_route(plan, p, ws.status)
        layer._maybe_check(ws)
        w16 = R.assemble_weight_f16(plan, table, atoms, ws)
        rows = x.shape[0]
        x16 = R.F16Split(rows, plan.n_in, dev)
        if rows:
            x16.fill(x)
        y = torch.empty(rows, plan.n_out, dtype=torch.float32, device=dev)
        R.gemm_f16(rows, plan.n_out, plan.n_in, x16, False, w16, False, y, plan.n_out, ws.status)
        ctx.save_for_backward(table)
        ctx.splits = (x16, w16)
        ctx.meta = (layer, rows, atoms)
        return y

    @staticmethod
    @once_differentiable
    def backward(ctx, dy):
        (table,) = ctx.saved_tensors
        x16, w16 = ctx.splits
        layer, rows, atoms = ctx.meta
        plan = layer._plan
        ws = layer._workspace(dy.device)
        dy = dy.contiguous()
        dy16 = R.F16Split(rows, plan.n_out, dy.device)
        if rows:
            dy16.fill(dy)
        dx = grad = None
        if ctx.needs_input_grad[0]:
            dx = torch.empty(rows, plan.n_in, dtype=torch.float32, device=dy.device)
            R.gemm_f16(rows, plan.n_in, plan.n_out, dy16, False, w16, True, dx, plan.n_in,
                       ws.status)
        if ctx.needs_input_grad[1]:
            split = R.weight_split_k(plan, rows)
            ldg = R.pad4(plan.n_in)
            stride = plan.n_out * ldg
            g = torch.empty(split * stride, dtype=torch.float32, device=dy.device)
            R.gemm_f16(plan.n_out, plan.n_in, rows, dy16, True, x16, True, g, ldg, ws.status,
                       split_k=split, split_stride=stride)
            grad = R.pullback(plan, table, atoms, g, ldg, split, stride, dy.device)
        ctx.splits = None
        return dx, grad, None


class _Atoms(nn.Module):
    def __init__(self, p):
        super().__init__()
        self.p = nn.Parameter(p)


class _AtomState(nn.Module):
    """Holds the Parameter under the reference's state-dict key atom_state.atoms.p."""

    def __init__(self, p):
        super().__init__()
        self.atoms = _Atoms(p)


def _initial_atoms(kernel: KernelSpec, axes, atoms: int, atom_init: str):
    """Constructor-default atoms on CPU float32, with the reference's RNG calls."""
    out_axis, in_axis = axes
    c = kernel.coordinates
    if isinstance(c, RationalRadius):
        # _backends/torch/kernels/radius_cell_mass.py:134-146.
        p = torch.empty((atoms, 4), dtype=torch.float32)
        p[:, 0].normal_(0, float(torch.tensor(c.amplitude_std, dtype=torch.float32)))
        cap = torch.tensor(c.amplitude_max, dtype=torch.float32)
        if cap.double() > c.amplitude_max:
            cap = torch.nextafter(cap, torch.zeros_like(cap))
        p[:, 0].clamp_(-cap, cap)
        p[:, 1].fill_(float(torch.tensor(c.radius_fraction, dtype=torch.float32)))
        p[:, 2].uniform_(out_axis.origin, out_axis.origin + out_axis.period)
        p[:, 3].uniform_(in_axis.origin, in_axis.origin + in_axis.period)
        return p
    # Polar: _backends/torch/kernels/polar_amp_width.py:25-50 with regular-grid
    # centers (_backends/torch/charts/regular_grid.py:47-75).
    if atom_init not in ("balanced", "uniform"):
        raise ValueError("mode must be 'balanced' or 'uniform'")

    def centers(axis, mode):
        if mode == "uniform":
            spacing = torch.tensor(axis.spacing, dtype=torch.float32)
            extent = spacing.new_tensor((axis.period,))
            return torch.tensor(axis.origin, dtype=torch.float32) + torch.rand(
                atoms, 1, dtype=torch.float32) * extent
        idx = torch.linspace(0, axis.site_count - 1, atoms, dtype=torch.float64).round().long()
        return (torch.tensor(axis.origin, dtype=torch.float32)
                + idx.to(torch.float32) * torch.tensor(axis.spacing, dtype=torch.float32))[:, None]

    out_p = centers(out_axis, atom_init)
    in_p = centers(in_axis, "uniform")
    amplitude = out_p.new_empty(atoms)
    amplitude.normal_(mean=0.0, std=0.1 / math.sqrt(atoms))
    maximum = torch.tensor(c.amplitude_max, dtype=torch.float32)
    ratio = (amplitude / maximum).clamp(-1 + 1e-6, 1 - 1e-6)
    polar = torch.stack((ratio, (1 - ratio.square()).sqrt()), dim=-1)
    polar = polar * (1.0 + 3.0 * torch.tensor(c.alpha_init, dtype=torch.float32)).sqrt()
    return torch.cat((polar, out_p, in_p), dim=-1)


class CSTLinear(nn.Module):
    """Radius cell-mass CSTLinear executed by the sm_100a backend.

    ``validate``: "sync" (default) reads the device status word after decoding
    and raises ``ValueError`` for invalid atoms like the reference; "off" skips
    the host read (status stays available through :meth:`check_status`).
    """

    def __init__(self, output_chart=None, input_chart=None, *, charts=None, atoms,
                 kernel: KernelSpec, atom_init="balanced", device=None,
                 dtype=torch.float32, validate="sync"):
        super().__init__()
        if charts is not None:
            if output_chart is not None or input_chart is not None:
                raise ValueError("charts cannot be combined with output_chart, input_chart")
            if not isinstance(charts, tuple) or len(charts) != 2:
                raise ValueError("radius cell masses require an (output, input) chart pair")
            output_chart, input_chart = charts
        if not isinstance(output_chart, RegularGrid) or not isinstance(input_chart, RegularGrid):
            raise TypeError("charts must be regular_grid(..., geometry='flat_torus') charts")
        if not isinstance(kernel, KernelSpec):
            raise TypeError("kernel must be a KernelSpec")
        if dtype != torch.float32:
            raise TypeError("the B200 backend computes the float32 CSTLinear contract")
        if validate not in ("sync", "off"):
            raise ValueError("validate must be 'sync' or 'off'")
        self.output_chart, self.input_chart = output_chart, input_chart
        self.kernel = kernel
        self.axes = radius_cell_mass_axes((output_chart, input_chart), kernel)
        self.validate = validate
        if isinstance(atoms, bool) or not isinstance(atoms, (int, torch.Tensor)):
            raise TypeError("atoms must be an integer, Tensor or Parameter")
        if isinstance(atoms, int):
            if atoms < 1:
                raise ValueError("atoms must be positive")
            p = _initial_atoms(kernel, self.axes, atoms, atom_init)
        else:
            p = atoms.detach().to(torch.float32).clone()
            if p.ndim != 2 or p.shape[1] != 4:
                raise ValueError("atom parameters must have shape [atoms, 4]")
        self.atom_state = _AtomState(p.to(device) if device is not None else p)
        self._plan = R.Plan.make(self.axes, kernel)
        self._workspaces = {}

    @property
    def atoms(self):
        return self.atom_state.atoms

    @property
    def in_features(self):
        return self.input_chart.features

    @property
    def out_features(self):
        return self.output_chart.features

    def cst_charts(self):
        return self.output_chart, self.input_chart

    def _workspace(self, device):
        key = torch.device(device).index
        ws = self._workspaces.get(key)
        if ws is None:
            ws = self._workspaces[key] = R.Workspace(self._plan, device)
        return ws

    def _maybe_check(self, ws):
        # Inside a CUDA graph capture the status stays on the device (read it
        # later with check_status); a host read there would break the capture.
        if self.validate == "sync" and not torch.cuda.is_current_stream_capturing():
            self.check_status(ws)

    def check_status(self, ws=None):
        """Raise ValueError if a kernel flagged an invalid atom or a timeout."""
        ws = ws or self._workspace(self.atoms.p.device)
        code = int(ws.status.item())
        if code:
            ws.status.zero_()
            raise ValueError(R.status_error(code))

    def forward(self, x):
        if x.shape[-1] != self.in_features:
            raise ValueError(f"expected input features {self.in_features}, got {x.shape[-1]}")
        p = self.atoms.p
        R.require_cuda(x, p)
        if x.dtype != torch.float32:
            raise TypeError("the B200 backend computes the float32 CSTLinear contract")
        flat = x.reshape(-1, self.in_features).contiguous()
        with R.on_device(p.device):  # the backward runs on the device's autograd thread
            y = _CellMassLinear.apply(flat, p, self)
        return y.reshape(*x.shape[:-1], self.out_features)

    # -- diagnostics ---------------------------------------------------------------

    @torch.no_grad()
    def weight(self):
        """Dense float32 W [out, in] assembled on the device."""
        p = self.atoms.p
        ws = self._workspace(p.device)
        with R.on_device(p.device):
            table = R.decode_route(self._plan, p, ws.status)
            self._maybe_check(ws)
            w, _, _, _ = R.assemble_weight(self._plan, table, p.shape[0], ws, dense=True,
                                           split=False)
        return w

    @torch.no_grad()
    def routing(self):
        """(routing [A, 6] int32, owner keys [A] int64) computed on the device."""
        p = self.atoms.p
        ws = self._workspace(p.device)
        routing = torch.empty(p.shape[0], 6, dtype=torch.int32, device=p.device)
        keys = torch.empty(p.shape[0], dtype=torch.int64, device=p.device)
        with R.on_device(p.device):
            R.decode_route(self._plan, p, ws.status, owner_keys=keys, routing=routing)
            self._maybe_check(ws)
        return routing, keys

    def extra_repr(self):
        c = self.kernel.coordinates
        return (f"out={self.out_features}, in={self.in_features}, atoms={self.atoms.p.shape[0]}, "
                f"coordinates={c.id}")


def is_polar(layer: CSTLinear) -> bool:
    return isinstance(layer.kernel.coordinates, PolarRadius)
