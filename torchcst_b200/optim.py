"""CSTAdamW for B200 CSTLinear sites: AdamW + field_lrs + coordinate law in one kernel.

Mirrors torchcst's ``CSTAdamW(params, model=..., lr=..., field_lrs=...)``
(optim/adamw.py:26-360): atom groups default to raw ``weight_decay=0``,
``field_lrs`` are absolute rates relative to the group ``lr`` recorded when the
group is configured (optim/_field_lrs.py:29-38), ``amplitude_weight_decay`` is
the decoupled Polar amplitude decay (optim/adamw.py:41,146-183; raw
``weight_decay`` must stay 0 on atom groups), per-parameter state is torch's
``step`` / ``exp_avg`` / ``exp_avg_sq`` (so ``state_dict`` round-trips), and
ordinary parameters take torch's own functional AdamW. Atom parameters of
``torchcst_b200.CSTLinear`` sites are updated by ``tcst_optimizer_step``: the
AdamW proposal, the field rescale and the rational projection or Polar
activity law in one pass over HBM.
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import torch
from torch.optim import AdamW

from . import _native as N
from . import runtime as R
from .linear import CSTLinear
from .spec import PolarRadius, RationalRadius

REFERENCE = "_cst_field_lr_reference"


def _f32(x) -> float:
    """Round a Python float to float32 (round to nearest even), as torch.tensor does."""
    return float(np.float32(x))


def law_fields(h: N.AdamW, coords, axes, lr: float, amplitude_weight_decay: float = 0.0):
    """Fill the coordinate-law fields of a tcst_adamw block: the rational
    amplitude cap (_backends/torch/updates/rational_radius.py:10-29), the Polar
    activity-law scalars at step size ``lr`` with torch's float32 scalar
    arithmetic (_backends/torch/algorithms/polar_update/executor.py:42-112), the
    chart periods of the torus retraction and the float32 Polar amplitude decay
    ``lr * amplitude_weight_decay`` (executor.py:18-41)."""
    if amplitude_weight_decay:
        if not isinstance(coords, PolarRadius):
            # operators/atom_update.py:42-66: decay is a Polar-only law.
            raise ValueError("amplitude decay requires Polar atoms")
        h.amplitude_decay = _f32(lr * amplitude_weight_decay)
    oa, ia = axes
    h.period_out = _f32(oa.period)
    h.period_in = _f32(ia.period)
    if isinstance(coords, RationalRadius):
        cap = torch.tensor(coords.amplitude_max, dtype=torch.float32)
        if cap.double() > coords.amplitude_max:
            cap = torch.nextafter(cap, torch.zeros_like(cap))
        h.amplitude_cap = float(cap)
    else:
        p32 = torch.float32
        h.polar_amplitude_max = _f32(coords.amplitude_max)
        h.polar_w_c = _f32(coords.w_c)
        h.polar_activity_gain = _f32(coords.activity_gain)
        rate = torch.tensor(coords.dormant_expansion_rate, dtype=p32)
        h.polar_dormant_q_scale = float(3.0 * rate * torch.tensor(lr, dtype=p32))
        rr = torch.tensor(coords.radial_regularization, dtype=p32)
        h.polar_decay = float(torch.exp(-4.0 * rr * torch.tensor(lr, dtype=p32)))
        h.polar_energy_step = _f32(lr) if coords.activity_mode == "time_energy" else 0.0
    return h


def coordinate_update_(proposal, previous, coords, axes, step_size: float,
                       amplitude_weight_decay: float = 0.0):
    """Apply the coordinate law in place: ``proposal`` (an outside optimizer's
    AdamW + field-rate point) becomes the law's result from ``previous``, on the
    current CUDA stream (``tcst_coordinate_update``)."""
    R.require_cuda(proposal, previous)
    if proposal.dtype != torch.float32 or previous.dtype != torch.float32:
        raise TypeError("the B200 update computes float32 atoms")
    if not proposal.is_contiguous() or not previous.is_contiguous():
        raise ValueError("the B200 update needs contiguous [atoms, 4] tensors")
    if proposal.shape != previous.shape or proposal.ndim != 2 or proposal.shape[1] != 4:
        raise ValueError("previous point must match the bound atom shape")
    h = law_fields(N.AdamW(), coords, axes, step_size, amplitude_weight_decay)
    kind = N.TCST_POLAR if isinstance(coords, PolarRadius) else N.TCST_RATIONAL
    with R.on_device(proposal.device):
        N.call("tcst_coordinate_update", R._vp(proposal), R._vp(previous), proposal.shape[0],
               kind, ctypes.byref(h), R._stream(proposal.device))
    return proposal


class CSTAdamW(AdamW):
    def __init__(self, params, *, model, amplitude_weight_decay: float = 0.0, field_lrs=None,
                 check_finite: bool = False, **adamw_options):
        if not isinstance(model, torch.nn.Module):
            raise TypeError("model must be a torch.nn.Module")
        self._validate_decay(amplitude_weight_decay)
        self.model = model
        self.check_finite = check_finite
        self._sites = {id(m.atoms.p): m for m in model.modules() if isinstance(m, CSTLinear)}
        self._field_lrs = self._rates(field_lrs)
        if self._field_lrs and not self._sites:
            raise ValueError("field_lrs requires managed CST sites")
        params = list(params)
        if not params:
            raise ValueError("optimizer got an empty parameter list")
        groups = params if isinstance(params[0], dict) else [{"params": params}]
        default_lr = adamw_options.get("lr", 1e-3)
        for g in groups:
            g["params"] = list(g["params"]) if not isinstance(g["params"], torch.Tensor) else [g["params"]]
            if any(id(p) in self._sites for p in g["params"]):
                g.setdefault("weight_decay", adamw_options.get("weight_decay", 0.0))
                g.setdefault("amplitude_weight_decay", amplitude_weight_decay)
                if "field_lrs" not in g and self._field_lrs:
                    g["field_lrs"] = dict(self._field_lrs)
                if g.get("field_lrs"):
                    g["field_lrs"] = self._rates(g["field_lrs"])
                    g.setdefault(REFERENCE, g.get("lr", default_lr))
        super().__init__(groups, **adamw_options)

    @staticmethod
    def _validate_decay(decay):
        """optim/adamw.py:126-131."""
        if type(decay) not in (int, float) or not math.isfinite(decay) or decay < 0:
            raise ValueError("amplitude_weight_decay must be a finite nonnegative Python scalar")

    def _validate_group(self, group):
        """The per-step group rules of optim/adamw.py:146-183: atom groups keep raw
        weight_decay=0 and take the decoupled Polar amplitude decay instead."""
        has_atoms = any(id(p) in self._sites for p in group["params"])
        if "amplitude_weight_decay" in group:
            if not has_atoms:
                raise ValueError("amplitude_weight_decay requires an atom group")
            decay = group["amplitude_weight_decay"]
            self._validate_decay(decay)
            rate = group.get("lr", self.defaults["lr"])
            if (type(rate) not in (int, float) or not math.isfinite(rate) or rate < 0
                    or rate * decay > 1):
                raise ValueError(
                    "lr * amplitude_weight_decay must be in [0, 1] with finite Python lr")
        if has_atoms:
            raw = group.get("weight_decay", self.defaults["weight_decay"])
            if type(raw) not in (int, float) or raw != 0:
                raise ValueError(
                    "managed atoms require raw weight_decay=0; use amplitude_weight_decay")

    @staticmethod
    def _rates(value):
        if value is None:
            return {}
        out = {}
        for name, rate in dict(value).items():
            if not isinstance(name, str) or not name:
                raise ValueError("field_lrs names must be nonempty strings")
            if type(rate) not in (int, float) or not math.isfinite(rate) or rate < 0:
                raise ValueError("field_lrs values must be finite nonnegative Python scalars")
            out[name] = float(rate)
        return out

    def _native_params(self, site: CSTLinear, group, step: int) -> N.AdamW:
        lr = group["lr"]
        beta1, beta2 = group["betas"]
        key = (id(site), lr, beta1, beta2, group["eps"], group["weight_decay"],
               group.get("amplitude_weight_decay", 0.0),
               tuple(sorted((group.get("field_lrs") or {}).items())), group.get(REFERENCE))
        cache = self.__dict__.setdefault("_params_cache", {})
        base = cache.get(key)
        if base is None:
            if len(cache) >= 64:  # learning-rate schedules create a key per rate
                cache.clear()
            base = cache[key] = self._step_free_params(site, group)
        h = N.AdamW.from_buffer_copy(base)
        bc1 = 1 - beta1 ** step
        bc2 = 1 - beta2 ** step
        h.neg_step_size = _f32(-(lr / bc1))
        h.bias2_sqrt = _f32(bc2 ** 0.5)
        return h

    def _step_free_params(self, site: CSTLinear, group) -> N.AdamW:
        """Every tcst_adamw field except the two bias corrections."""
        lr = group["lr"]
        beta1, beta2 = group["betas"]
        h = N.AdamW()
        h.lerp_weight = _f32(1 - beta1)
        h.beta2 = _f32(beta2)
        h.one_minus_beta2 = _f32(1 - beta2)
        h.eps = _f32(group["eps"])
        wd = group["weight_decay"]
        h.has_decay = int(wd != 0)
        h.decay_factor = _f32(1 - lr * wd)
        coords = site.kernel.coordinates
        configured = group.get("field_lrs") or {}
        mask = 0
        if configured:
            reference = group[REFERENCE]
            for name, start, stop in coords.optimizer_fields:
                if name in configured and configured[name] != reference:
                    for c in range(start, stop):
                        h.field_ratio[c] = _f32(configured[name] / reference)
                        mask |= 1 << c
            unknown = set(configured) - {f[0] for f in coords.optimizer_fields}
            if unknown:
                raise ValueError(f"unknown field_lrs {sorted(unknown)}")
        h.field_mask = mask
        law_fields(h, coords, site.axes, lr, group.get("amplitude_weight_decay", 0.0))
        return h

    def site_step(self, p):
        """Advance the step count of atom parameter ``p`` exactly as :meth:`step`
        does and return ``(params, state, kind)`` for ``tcst_optimizer_step*``, or
        ``None`` when the group's learning rate is 0 (no update)."""
        site = self._sites.get(id(p))
        if site is None:
            raise ValueError("not an atom parameter of a managed CSTLinear")
        group = next(g for g in self.param_groups if any(q is p for q in g["params"]))
        self._validate_group(group)
        if group.get("amsgrad") or group.get("maximize"):
            raise NotImplementedError("amsgrad/maximize are not implemented for atom groups")
        lr = group["lr"]
        if type(lr) not in (int, float) or not math.isfinite(lr) or lr < 0:
            raise ValueError("CST learning rates must be finite nonnegative Python scalars")
        state = self.state[p]
        if not state:
            state["step"] = torch.tensor(0.0, dtype=torch.float32)
            state["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
            state["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
        state["step"] += 1
        if lr == 0:
            return None
        h = self._native_params(site, group, int(state["step"].item()))
        kind = N.TCST_POLAR if isinstance(site.kernel.coordinates, PolarRadius) else N.TCST_RATIONAL
        return h, state, kind

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            self._validate_group(group)
        for group in self.param_groups:
            if group.get("amsgrad") or group.get("maximize"):
                if any(id(p) in self._sites for p in group["params"]):
                    raise NotImplementedError("amsgrad/maximize are not implemented for atom groups")
            lr = group["lr"]
            if type(lr) not in (int, float) or not math.isfinite(lr) or lr < 0:
                raise ValueError("CST learning rates must be finite nonnegative Python scalars")
            plain = ([], [], [], [], [])
            capturing = torch.cuda.is_current_stream_capturing()
            for p in group["params"]:
                if p.grad is None:
                    continue
                site = self._sites.get(id(p))
                state = self.state[p]
                if not state:
                    # torch's AdamW keeps a capturable group's step count on the device.
                    on_device = site is None and group["capturable"]
                    state["step"] = (torch.zeros((), dtype=torch.float32, device=p.device)
                                     if on_device else torch.tensor(0.0, dtype=torch.float32))
                    state["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                    state["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                if capturing and site is None and not group["capturable"]:
                    raise RuntimeError("capturing a CSTAdamW step needs capturable=True for "
                                       "the groups of ordinary parameters")
                if capturing and site is not None:
                    self._capture_site_step(p, site, state)
                    continue
                if site is None:
                    plain[0].append(p)
                    plain[1].append(p.grad)
                    plain[2].append(state["exp_avg"])
                    plain[3].append(state["exp_avg_sq"])
                    plain[4].append(state["step"])
                    continue
                if p.is_cuda:
                    self._graph_entry(p)  # ready for a later capture
                if self.check_finite and not bool(torch.isfinite(p.grad).all()):
                    raise FloatingPointError("non-finite parameter gradient")
                if p.grad.is_sparse:
                    raise ValueError("CST coordinate policies require strided atom gradients")
                state["step"] += 1
                if lr == 0:
                    continue
                h = self._native_params(site, group, int(state["step"].item()))
                kind = N.TCST_POLAR if isinstance(site.kernel.coordinates, PolarRadius) else N.TCST_RATIONAL
                grad = p.grad.contiguous()
                with R.on_device(p.device):
                    N.call("tcst_optimizer_step", R._vp(p), R._vp(grad),
                           R._vp(state["exp_avg"]), R._vp(state["exp_avg_sq"]), p.shape[0],
                           kind, ctypes.byref(h), R._stream(p.device))
            if plain[0]:
                beta1, beta2 = group["betas"]
                torch.optim._functional.adamw(
                    plain[0], plain[1], plain[2], plain[3], [], plain[4],
                    foreach=group["foreach"], capturable=group["capturable"],
                    differentiable=group["differentiable"], fused=group["fused"],
                    amsgrad=group["amsgrad"], beta1=beta1, beta2=beta2, lr=lr,
                    weight_decay=group["weight_decay"], eps=group["eps"],
                    maximize=group["maximize"], has_complex=False)
        return loss

    # -- CUDA graph capture ------------------------------------------------------

    def _graph_entry(self, p):
        """The scalar ring of atom site ``p`` for captured steps (pinned host
        slots the captured optimizer kernel reads through their device mapping,
        and its device use counter). Made by an eager step: an allocation inside
        a capture would come with an initialising kernel that every replay
        would run."""
        entries = self.__dict__.setdefault("_graph_entries", {})
        entry = entries.get(id(p))
        if entry is None:
            entry = entries[id(p)] = {"p": p, "ring": R.ScalarRing(p.device)}
        return entry

    def _capture_site_step(self, p, site, state):
        """Record the atom update of ``p`` into the CUDA graph being captured.
        The kernel reads its per-step scalars from the ring slot that
        :meth:`refresh_captured` writes before every replay; the step count is
        advanced there too, once per replay, not here."""
        entry = self.__dict__.get("_graph_entries", {}).get(id(p))
        if entry is None:
            raise RuntimeError("run one eager CSTAdamW step before capturing one")
        self.__dict__.setdefault("_graph_sites", {})[id(p)] = entry
        kind = N.TCST_POLAR if isinstance(site.kernel.coordinates, PolarRadius) else N.TCST_RATIONAL
        if not p.grad.is_contiguous():
            raise ValueError("captured atom updates need a contiguous gradient")
        with R.on_device(p.device):
            stream = R._stream(p.device)
            entry["ring"].fetch(site._workspace(p.device).status, stream)
            entry["ring"].launch(p, p.grad, state["exp_avg"], state["exp_avg_sq"], kind, stream)

    def refresh_captured(self):
        """Host half of one replayed step of every captured atom site: advance its
        step count exactly as :meth:`step` does and write the step's scalars
        (bias corrections, rates) into the ring slot the replay's optimizer
        kernel reads. Call it once before every replay."""
        for entry in self.__dict__.get("_graph_sites", {}).values():
            out = self.site_step(entry["p"])
            if out is None:
                raise ValueError("a captured CSTAdamW step needs a positive learning rate")
            entry["ring"].write(out[0])

    def get_field_lrs(self):
        out = []
        for group in self.param_groups:
            configured = group.get("field_lrs") or {}
            if not configured:
                out.append({})
                continue
            scale = group["lr"] / group[REFERENCE]
            out.append({k: v * scale for k, v in configured.items()})
        return out
