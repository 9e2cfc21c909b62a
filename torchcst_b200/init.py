"""He/Xavier variance-matching initialization of B200 CSTLinear atoms.

Same contract and search as torchcst's ``init.variance_scaling_`` /
``kaiming_normal_`` / ``xavier_normal_`` (init.py:40-125,
_backends/torch/initialization.py:16-139): draw one standard-normal proposal per
atom on the CPU generator, then bisect an amplitude scale until the summed atom
operator energy sum_a amp_a^2 |m_out,a|^2 |m_in,a|^2 is within 0.5% of
variance * N_out * N_in. The per-atom energies are evaluated on the device by
``tcst_atom_energies`` (images folded before squaring, like
radius_cell_mass.py:162-205), so the search costs milliseconds instead of
seconds per trial.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, replace

import torch

from . import runtime as R
from .linear import CSTLinear
from .spec import PolarRadius, RationalRadius


@dataclass(frozen=True)
class InitializationReport:
    scheme: str
    q: float
    variance: float
    target_energy: float
    expected_energy: float
    relative_error: float
    amplitude_scale: float
    amplitude_rms: float
    clipped_atoms: int
    atom_count: int
    evaluations: int


_SCALES = (0.0, 0.025, 0.05, 0.1, 0.2, 0.4, 0.8, 1.6, 3.2, 6.4, 12.8, 32.0)


@torch.no_grad()
def variance_scaling_(module: CSTLinear, variance, *, q=0.0, generator=None):
    if not isinstance(module, CSTLinear):
        raise TypeError("variance initialization requires a CSTLinear")
    if isinstance(variance, bool) or not isinstance(variance, (int, float)) or not math.isfinite(
            variance) or variance <= 0:
        raise ValueError("positive finite Dense weight variance required")
    if isinstance(q, bool) or not isinstance(q, (int, float)) or not math.isfinite(q) or not 0 <= q <= 1:
        raise ValueError("q must be a finite fraction in [0,1]")
    p = module.atoms.p
    if p.grad is not None:
        raise ValueError("initialize before backward and optimizer construction")
    coords = module.kernel.coordinates
    maximum = float(torch.tensor(coords.amplitude_max, dtype=torch.float32))
    noise = torch.randn(p.shape[0], dtype=p.dtype, device="cpu", generator=generator)
    target = variance * module.out_features * module.in_features
    rho = math.sqrt(1 + 3 * q)
    tolerance = 0.005
    device = p.device if p.is_cuda else torch.device("cuda")
    plan = module._plan
    ws = module._workspace(device)
    original = p.detach().to("cpu").clone()
    history = []

    def trial(scale):
        ratio_unclipped = noise * (scale / maximum)
        ratio = ratio_unclipped.clamp(-1 + 1e-6, 1 - 1e-6)
        cand = original.clone()
        if isinstance(coords, RationalRadius):
            cand[:, 0] = ratio * maximum
            cand[:, 1] = q
        else:
            cand[:, :2] = torch.stack((ratio, (1 - ratio.square()).sqrt()), -1) * rho
        dev = cand.to(device)
        with R.on_device(device):
            table = R.decode_route(plan, dev, ws.status)
            energies = R.atom_energies(plan, table, cand.shape[0], device)
        energy = float(energies.sum())
        code = int(ws.status.item())
        if code:
            ws.status.zero_()
            raise ValueError(R.status_error(code))
        if not math.isfinite(energy) or energy < 0:
            raise ValueError("nonfinite initial Atom energy")
        error = abs(energy / target - 1)
        history.append((scale, energy, error))
        return cand, energy, error, int((ratio_unclipped.abs() >= 1 - 1e-6).sum())

    low, high, accepted = 0.0, None, None
    for relative in _SCALES:
        scale = relative * maximum
        value = trial(scale)
        if value[2] <= tolerance:
            accepted = (scale, value)
            break
        if value[1] >= target:
            high = scale
            break
        low = scale
    if accepted is None and high is not None:
        for _ in range(32):
            scale = (low + high) / 2
            value = trial(scale)
            if value[2] <= tolerance:
                accepted = (scale, value)
                break
            if value[1] < target:
                low = scale
            else:
                high = scale
    if accepted is None:
        raise ValueError("variance target not reached in the bounded scale search; module "
                         f"unchanged. Search history: {history}")
    scale, (cand, energy, error, clipped) = accepted
    if isinstance(coords, PolarRadius):
        pair = cand[:, :2].double()
        amp = maximum * pair[:, 0] / pair.square().sum(-1).sqrt()
    else:
        amp = cand[:, 0].double()
    p.copy_(cand.to(p.device))
    return InitializationReport("variance_scaling", float(q), float(variance), target, energy,
                                error, scale, float(amp.square().mean().sqrt()), clipped,
                                cand.shape[0], len(history))


def kaiming_normal_(module, a=0.0, mode="fan_in", nonlinearity="leaky_relu", *, q=0.0,
                    generator=None):
    if mode not in ("fan_in", "fan_out"):
        raise ValueError("mode must be fan_in or fan_out")
    gain = torch.nn.init.calculate_gain(nonlinearity, a)
    fan = module.in_features if mode == "fan_in" else module.out_features
    report = variance_scaling_(module, gain ** 2 / fan, q=q, generator=generator)
    return replace(report, scheme="kaiming_normal")


def xavier_normal_(module, gain=1.0, *, q=0.0, generator=None):
    if isinstance(gain, bool) or not isinstance(gain, (float, int)) or not math.isfinite(
            gain) or gain <= 0:
        raise ValueError("positive finite gain required")
    variance = gain ** 2 * 2 / (module.in_features + module.out_features)
    report = variance_scaling_(module, variance, q=q, generator=generator)
    return replace(report, scheme="xavier_normal")
