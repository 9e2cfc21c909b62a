"""Generate golden vectors by running the torchcst reference itself.

Run in a container where the reference source tree is available:

    PYTHONPATH=<torchcst>/src python tests/golden/make_golden.py            # base cases
    PYTHONPATH=<torchcst>/src python tests/golden/make_golden.py config3_decay config2_init \
        trajectory1 trajectory_mid                                          # extra cases

It writes ``tests/golden/*.npz``. The GPU box never runs this script; the tests
only read the committed fixtures. Each case records the reference inputs
(atoms, rows, upstream gradient), the reference outputs (Y, dX, p.grad, the
atoms after one CSTAdamW step) and the dense float64 factors, whose support
pins the integer routing (level, K, first tile) of every atom.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _imports():
    import torchcst  # noqa: F401
    from torchcst import CSTAdamW, CSTLinear, ChebyshevSpec, RadiusBounds, chart_presets, kernels
    from torchcst import init as cst_init
    return CSTAdamW, CSTLinear, ChebyshevSpec, RadiusBounds, chart_presets, kernels, cst_init


def _factors64(layer):
    from torchcst._backends.torch.kernels import execution
    import copy
    p = layer.atoms.p.detach().double()
    k64 = copy.deepcopy(layer.kernel).double()
    c64 = tuple(copy.deepcopy(c).double() for c in layer.cst_charts())
    phi_in, phi_out = execution.factors(k64, *c64, p)
    return phi_in.numpy(), phi_out.numpy()


def _reference_routing(layer):
    """Per-atom (level, K, first_tile) on both axes, as the reference computes it.

    Wraps the reference's ``integrated_cells`` while its own ``factors`` runs
    (radius_cell_mass.py:97-114): each call receives one (level, K) group's
    radii, relative centers, local period and unwrapped sites. Rows are mapped
    back to atoms through the reference's own decoded radius and relative
    center of every atom, which are unique for random data.
    """
    from torchcst._backends.torch.kernels import radius_cell_mass as rcm
    from torchcst._backends.torch.parameterizations.radius_cell_mass import decoded_values
    from torchcst.kernels.radius_cell_mass import radius_cell_mass_axes
    charts = layer.cst_charts()
    axes = radius_cell_mass_axes(tuple(c.declaration() for c in charts),
                                 layer.kernel.declaration())
    p = layer.atoms.p.detach()
    _, r_in, r_out = decoded_values(layer.kernel, p)
    calls = []
    original = rcm.integrated_cells

    def recording(profile, radius, centers, period, sites, spacing):
        calls.append((radius.detach().double().numpy().copy(),
                      centers.detach().double().numpy().copy(), float(period),
                      sites[:, 0].numpy().copy(), int(sites.shape[1])))
        return original(profile, radius, centers, period, sites, spacing)

    rcm.integrated_cells = recording
    try:
        with torch.no_grad():
            rcm.factors(layer.kernel, *charts, p)
    finally:
        rcm.integrated_cells = original
    out = {}
    # factors() evaluates the output axis first, then the input axis.
    split = None
    total = 0
    for i, call in enumerate(calls):
        total += len(call[0])
        if total == len(p):
            split = i + 1
            break
    for name, axis, radius, center_col, group in (
            ("out", axes[0], r_out, 2, calls[:split]),
            ("in", axes[1], r_in, 3, calls[split:])):
        rel = rcm._relative_centers(p[:, center_col], axis.origin, axis.period).numpy()
        lookup = {}
        for a, key in enumerate(zip(radius.detach().double().numpy().tolist(), rel.tolist())):
            lookup.setdefault(key, []).append(a)
        level = np.full(len(p), -1, np.int16)
        count = np.zeros(len(p), np.int8)
        first = np.zeros(len(p), np.int32)
        tiles = []
        t = axis.binding.base_tile_sites
        while t <= axis.site_count:
            tiles.append(t)
            t *= axis.binding.merge_factor
        for radius_g, centers_g, period, first_site, length in group:
            for r, c, f in zip(radius_g.tolist(), centers_g.tolist(), first_site.tolist()):
                for a in lookup[(r, c)]:
                    k = None
                    for lv, tile in enumerate(tiles):
                        if length % tile == 0 and length // tile in (2, 3) and \
                                abs((length // tile) * tile * axis.spacing - period) == 0:
                            if r <= tile * axis.spacing and (lv == 0 or r > tiles[lv - 1] * axis.spacing):
                                k = (lv, length // tile, f // tile)
                    assert k is not None
                    level[a], count[a], first[a] = k
        assert (level >= 0).all()
        out[f"route_{name}_level"] = level
        out[f"route_{name}_count"] = count
        out[f"route_{name}_first_tile"] = first
    return out


def run_case(layer, x, dy, *, lr, field_lrs=None, need_dx=True, sample=None,
             factors=True, seed=0):
    CSTAdamW = _imports()[0]
    x = x.clone().requires_grad_(need_dx)
    p0 = layer.atoms.p.detach().clone()
    y = layer(x)
    y.backward(dy)
    grad = layer.atoms.p.grad.detach().clone()
    opt = CSTAdamW(layer.parameters(), model=layer, lr=lr,
                   **({"field_lrs": field_lrs} if field_lrs else {}))
    opt.step()
    p1 = layer.atoms.p.detach().clone()
    out = dict(p0=p0.numpy(), x=x.detach().numpy(), dy=dy.numpy(), y=y.detach().numpy(),
               lr=np.float64(lr))
    if need_dx:
        out["dx"] = x.grad.numpy()
    if sample is None:
        out["grad"] = grad.numpy()
        out["p1"] = p1.numpy()
    else:
        g = torch.Generator().manual_seed(seed)
        rows = torch.randperm(len(p0), generator=g)[:sample].sort().values
        out["rows"] = rows.numpy()
        out["grad"] = grad[rows].numpy()
        out["p1"] = p1[rows].numpy()
        out["grad_colsum"] = grad.double().sum(0).numpy()
        out["grad_colsq"] = grad.double().square().sum(0).numpy()
    if field_lrs:
        out["field_amplitude"] = np.float64(field_lrs.get("amplitude", np.nan))
        out["field_radius_fraction"] = np.float64(field_lrs.get("radius_fraction", np.nan))
    if factors:
        layer.zero_grad(set_to_none=True)
        with torch.no_grad():
            layer.atoms.p.copy_(p0)
        out.update(_reference_routing(layer))
        phi_in, phi_out = _factors64(layer)
        g = torch.Generator().manual_seed(seed + 100)
        cols = torch.randperm(len(p0), generator=g)[:min(len(p0), 256)].sort().values.numpy()
        out["phi_cols"] = cols
        out["phi_in"], out["phi_out"] = phi_in[:, cols], phi_out[:, cols]
    return out


def rational_layer(n_out, n_in, atoms, *, radius_max, q=0.0, seed=0, init=None,
                   base=(1, 1), merge=(2, 2), spacing=(1.0, 1.0), origin=(0.0, 0.0)):
    (CSTAdamW, CSTLinear, ChebyshevSpec, RadiusBounds, chart_presets, kernels,
     cst_init) = _imports()
    torch.manual_seed(seed)
    out_f = kernels.cell_mass(ChebyshevSpec(modes=8), base_tile_sites=base[0],
                              merge_factor=merge[0])
    in_f = kernels.cell_mass(ChebyshevSpec(modes=8), base_tile_sites=base[1],
                             merge_factor=merge[1])
    layer = CSTLinear(
        charts=(chart_presets.regular_grid(n_out, geometry="flat_torus", spacing=spacing[0],
                                           origin=origin[0]),
                chart_presets.regular_grid(n_in, geometry="flat_torus", spacing=spacing[1],
                                           origin=origin[1])),
        atoms=atoms,
        kernel=kernels.product(out_f, in_f, coordinates=kernels.rational_radius(
            radius_max=radius_max, radius_fraction=q)),
        backend="factored")
    if init == "kaiming":
        cst_init.kaiming_normal_(layer, nonlinearity="relu", q=q)
    elif init == "xavier":
        cst_init.xavier_normal_(layer, gain=1.0, q=q)
    return layer


def polar_layer(n_out, n_in, atoms, *, seed=0, in_base=49):
    (CSTAdamW, CSTLinear, ChebyshevSpec, RadiusBounds, chart_presets, kernels,
     cst_init) = _imports()
    torch.manual_seed(seed)
    out_f = kernels.cell_mass(ChebyshevSpec(modes=8))
    in_f = kernels.cell_mass(ChebyshevSpec(modes=8), base_tile_sites=in_base, merge_factor=2)
    coords = kernels.polar(amplitude_max=1.0, w_c=0.3, bounds=RadiusBounds(
        minimum=0.5, birth=4.0, maximum=50.0, upper_floor=1.0))
    return CSTLinear(
        charts=(chart_presets.regular_grid(n_out, geometry="flat_torus"),
                chart_presets.regular_grid(n_in, geometry="flat_torus")),
        atoms=atoms, kernel=kernels.product(out_f, in_f, coordinates=coords),
        backend="factored")


def synthetic_images(batch, generator):
    """~19% nonzero pixels, U[0,1], inside the central 20x20 crop of 28x28."""
    x = torch.zeros(batch, 28, 28)
    crop = torch.rand(batch, 20, 20, generator=generator)
    keep = torch.rand(batch, 20, 20, generator=generator) < (149 / 400)
    x[:, 4:24, 4:24] = crop * keep
    return x.reshape(batch, 784)


def decay_case():
    """Polar config-3 layer, three CSTAdamW steps with amplitude_weight_decay on
    fixed synthetic gradients: the atoms after every step."""
    CSTAdamW = _imports()[0]
    layer = polar_layer(1024, 784, 16384)
    p0 = layer.atoms.p.detach().clone()
    g = torch.Generator().manual_seed(11)
    grads = torch.randn(3, 16384, 4, generator=g) * 1e-2
    opt = CSTAdamW(layer.parameters(), model=layer, lr=2e-3, amplitude_weight_decay=0.25)
    rows = slice(0, 4096)  # the update is row by row: the first 4096 rows suffice
    out = dict(p0=p0[rows].numpy(), grads=grads[:, rows].numpy(), lr=np.float64(2e-3),
               amplitude_weight_decay=np.float64(0.25))
    for step in range(3):
        layer.atoms.p.grad = grads[step].clone()
        opt.step()
        out[f"p{step + 1}"] = layer.atoms.p.detach()[rows].clone().numpy()
    # The decay law alone on fixed inputs (executor.py:18-41), bit for bit.
    from torchcst._backends.torch.algorithms.polar_update.executor import decay_amplitude
    prev = torch.randn(4096, 4, generator=g)
    upd = prev + torch.randn(4096, 4, generator=g) * 1e-2
    out["decay_previous"], out["decay_updated"] = prev.numpy(), upd.numpy()
    out["decay_amount"] = np.float64(2e-3 * 0.25)
    out["decay_out"] = decay_amplitude(prev, upd, amount=2e-3 * 0.25).numpy()
    return out


def init_case():
    """The reference's He initialisation report at config 2 (seed 0): the scale
    its bounded search accepted and the energy it matched (p0 is config2's)."""
    _, _, _, _, _, _, cst_init = _imports()
    layer = rational_layer(1024, 1024, 65536, radius_max=512.0)
    report = cst_init.kaiming_normal_(layer, nonlinearity="relu", q=0.0)
    out = {k: np.float64(getattr(report, k)) for k in
           ("amplitude_scale", "relative_error", "target_energy", "expected_energy",
            "amplitude_rms")}
    out["evaluations"] = np.int64(report.evaluations)
    # The atoms themselves equal config2's p0 (same seed and calls).
    assert np.array_equal(layer.atoms.p.detach().numpy(),
                          np.load(os.path.join(HERE, "config2.npz"))["p0"])
    return out


def trajectory_case(n_out, n_in, atoms, *, radius_max, rows, steps, lr, field_lrs, seed,
                    keep=1):
    """An MSE training trajectory of the reference (fixed X and target): the
    loss of every step and the atoms after every step. With a large radius
    field rate the footprints widen through several bin classes on the way."""
    CSTAdamW = _imports()[0]
    layer = rational_layer(n_out, n_in, atoms, radius_max=radius_max, init="kaiming",
                           seed=seed)
    g = torch.Generator().manual_seed(seed + 1)
    x = torch.randn(rows, n_in, generator=g)
    target = torch.randn(rows, n_out, generator=g)
    opt = CSTAdamW(layer.parameters(), model=layer, lr=lr,
                   **({"field_lrs": field_lrs} if field_lrs else {}))
    out = dict(p0=layer.atoms.p.detach().clone().numpy(), x=x.numpy(), target=target.numpy(),
               lr=np.float64(lr))
    if field_lrs:
        out["field_amplitude"] = np.float64(field_lrs.get("amplitude", np.nan))
        out["field_radius_fraction"] = np.float64(field_lrs.get("radius_fraction", np.nan))
    losses, ps = [], []
    for _ in range(steps):
        opt.zero_grad(set_to_none=True)
        loss = (layer(x) - target).square().mean()
        loss.backward()
        opt.step()
        losses.append(loss.item())
        if len(losses) % keep == 0:
            ps.append(layer.atoms.p.detach().clone().numpy())
    out["losses"] = np.asarray(losses)
    out["p_steps"] = np.stack(ps)  # atoms after steps keep, 2 keep, ...
    out["keep"] = np.int64(keep)
    return out


def reference_file():
    """The config-1 reference layer (seed 0) saved as a Safetensors file the way
    a torchcst user saves one: every tensor of its state dict, after an atom
    relayout (the row-to-id maps are in the file)."""
    from safetensors.torch import save_file
    layer = rational_layer(8, 16, 12, radius_max=4.0)
    layer.atom_state.relayout(torch.arange(11, -1, -1))
    path = os.path.join(HERE, "config1_reference.safetensors")
    save_file({k: v.detach().contiguous() for k, v in layer.state_dict().items()
               if torch.is_tensor(v)}, path)
    # The relayout reversed the rows (the sum over atoms, the model, is the same).
    assert np.array_equal(layer.atoms.p.detach().numpy(),
                          np.load(os.path.join(HERE, "config1.npz"))["p0"][::-1])
    return None


EXTRA_CASES = {
    "config1_reference_file": reference_file,
    "config3_decay": decay_case,
    "config2_init": init_case,
    "trajectory1": lambda: trajectory_case(8, 16, 12, radius_max=4.0, rows=4, steps=20,
                                           lr=1e-2, field_lrs=None, seed=0),
    "trajectory_mid": lambda: trajectory_case(
        256, 256, 4096, radius_max=128.0, rows=64, steps=12, lr=1e-2,
        field_lrs={"amplitude": 1e-2, "radius_fraction": 6e-2}, seed=3, keep=4),
}


def main():
    torch.set_num_threads(os.cpu_count() or 1)
    only = [a for a in sys.argv[1:] if not a.startswith("-")]
    if only:
        for name in only:
            value = EXTRA_CASES[name]()
            if value is None:
                continue
            path = os.path.join(HERE, f"{name}.npz")
            np.savez_compressed(path, **value)
            print(name, os.path.getsize(path), "bytes", sorted(value))
        return 0
    cases = {}

    # Config 1: README example (16 -> 8, 12 atoms, radius_max 4, seed 0).
    layer = rational_layer(8, 16, 12, radius_max=4.0)
    x, target = torch.randn(4, 16), torch.randn(4, 8)
    with torch.no_grad():
        y0 = layer(x)
    dy = 2 * (y0 - target) / y0.numel()
    c = run_case(layer, x, dy, lr=1e-3)
    c["target"] = target.numpy()
    cases["config1"] = c

    # Config 2 (headline): 1024^2, 64N atoms, He init q=0, field_lrs; 16 rows.
    layer = rational_layer(1024, 1024, 65536, radius_max=512.0, init="kaiming")
    g = torch.Generator().manual_seed(1)
    x = torch.randn(16, 1024, generator=g)
    dy = torch.randn(16, 1024, generator=g) * 1e-3
    cases["config2"] = run_case(
        layer, x, dy, lr=1e-3, field_lrs={"amplitude": 2.4e-3, "radius_fraction": 9.6e-3},
        sample=4096)

    # Config 3: Polar 784 -> 1024 (input base tile 49, merge 2), 16384 atoms.
    layer = polar_layer(1024, 784, 16384)
    g = torch.Generator().manual_seed(2)
    x = synthetic_images(32, g)
    dy = torch.randn(32, 1024, generator=g) * 1e-3
    cases["config3"] = run_case(layer, x, dy, lr=1e-3, need_dx=False, sample=4096)

    # Config 4 shape, reduced: 256 -> 1024, radius_max 128, q=0.25, Xavier.
    layer = rational_layer(1024, 256, 4096, radius_max=128.0, q=0.25, init="xavier")
    g = torch.Generator().manual_seed(3)
    x = torch.randn(8, 256, generator=g)
    dy = torch.randn(8, 1024, generator=g) * 1e-3
    cases["config4s"] = run_case(layer, x, dy, lr=1e-3)

    # Config 5 shape, reduced: 512^2, radius_max 256, q ~ U[0,1] (wide, folded).
    layer = rational_layer(512, 512, 2048, radius_max=256.0, init="kaiming")
    with torch.no_grad():
        layer.atoms.p[:, 1].uniform_(0, 1, generator=torch.Generator().manual_seed(4))
    g = torch.Generator().manual_seed(5)
    x = torch.randn(8, 512, generator=g)
    dy = torch.randn(8, 512, generator=g) * 1e-3
    cases["config5s"] = run_case(layer, x, dy, lr=1e-3)

    # Hierarchy edge cases: merge 3, base 3, spacing 0.5, origin offsets,
    # centers outside [0, Q), radii at tile thresholds.
    layer = rational_layer(81, 54, 96, radius_max=13.0, q=0.0, base=(1, 2), merge=(3, 3),
                           spacing=(0.5, 1.0), origin=(-3.25, 7.0))
    with torch.no_grad():
        p = layer.atoms.p
        gen = torch.Generator().manual_seed(6)
        p[:, 1].uniform_(0, 1, generator=gen)
        p[:8, 1] = torch.tensor([0.0, 1.0, 0.5, 0.25, 0.75, 1.0, 0.0, 0.1])
        p[:, 2] = (torch.rand(96, generator=gen) * 3 - 1) * 40.5
        p[:, 3] = (torch.rand(96, generator=gen) * 3 - 1) * 54
        p[8:12, 2] = torch.tensor([-3.25, 37.25, 0.0, -44.0])
    g = torch.Generator().manual_seed(7)
    x = torch.randn(4, 54, generator=g)
    dy = torch.randn(4, 81, generator=g) * 1e-2
    cases["hierarchy"] = run_case(layer, x, dy, lr=1e-3)

    for name, value in cases.items():
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **value)
        print(name, os.path.getsize(path), "bytes", sorted(value))


if __name__ == "__main__":
    sys.exit(main())
