"""Parity of the sm_100a path (through the C ABI) against the CPU oracle and the
reference golden vectors.

Tolerances: routing and owner keys bit-exact; the optimizer step bit-exact
against the oracle; Y, dX, W and atom gradients within 1e-4 of the output scale
(max |err| / max |ref|, float64 truth), the north-star bound for fp32-accurate
tensor-core arithmetic (three-product f16 split with power-of-two scales; the
exported TF32 variant is held to the same bound).
"""

import numpy as np
import pytest
import torch

from oracle import cst_oracle as O
from tests.golden_cases import CASES, field_lrs, load

pytestmark = pytest.mark.gpu

TOL = 1e-4


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-300))


@pytest.fixture(scope="module")
def R():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from torchcst_b200 import runtime
    return runtime


def make_layer(name, p0):
    from torchcst_b200 import CSTLinear, kernels
    from torchcst_b200.spec import CellMass, ChebyshevSpec, RadiusBounds, RegularGrid
    out_axis, in_axis, spec = CASES[name]
    charts = tuple(RegularGrid(a.site_count, a.spacing, a.origin) for a in (out_axis, in_axis))
    profiles = tuple(CellMass(ChebyshevSpec(a.modes), a.base_tile_sites, a.merge_factor)
                     for a in (out_axis, in_axis))
    if isinstance(spec, O.Rational):
        coords = kernels.rational_radius(radius_min=spec.radius_min, radius_birth=spec.radius_birth,
                                         radius_max=spec.radius_max,
                                         amplitude_max=spec.amplitude_max)
    else:
        b = RadiusBounds(minimum=0.5, birth=4.0, maximum=50.0, upper_floor=1.0)
        coords = kernels.polar(amplitude_max=1.0, w_c=0.3, bounds=b)
    kernel = kernels.product(profiles[0], profiles[1], coordinates=coords)
    return CSTLinear(charts=charts, atoms=torch.as_tensor(p0), kernel=kernel, device="cuda")


# -- GEMM ---------------------------------------------------------------------------


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("shape,split", [((256, 512, 256), 1), ((130, 300, 70), 1),
                                         ((128, 256, 1000), 3), ((8, 16, 4), 1)])
def test_gemm_tf32x3(R, a_mn, b_mn, shape, split):
    M, N, K = shape
    g = torch.Generator().manual_seed(M * 7 + N + K)
    A = torch.randn(M, K, generator=g)
    B = torch.randn(N, K, generator=g)
    ref = A.double() @ B.double().T
    a_store = (A.T if a_mn else A).contiguous().cuda()
    b_store = (B.T if b_mn else B).contiguous().cuda()
    a_hi, a_lo, lda = R.split_tf32(a_store)
    b_hi, b_lo, ldb = R.split_tf32(b_store)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ldc = R.pad4(N)
    c = torch.full((split, M, ldc), float("nan"), device="cuda")
    R.gemm(M, N, K, (a_hi, a_lo), lda, a_mn, (b_hi, b_lo), ldb, b_mn, c, ldc, status,
           split_k=split, split_stride=M * ldc)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    out = c[:, :, :N].sum(0).double().cpu()
    err = float((out - ref).abs().max() / ref.abs().max())
    # Tensor-core fp32 accumulation truncates: allow 1e-5 of the output scale.
    assert err < 1e-5, err


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("shape,split", [((256, 512, 256), 1), ((130, 300, 70), 1),
                                         ((128, 256, 1000), 3), ((8, 16, 4), 1),
                                         ((300, 520, 1030), 2)])
@pytest.mark.parametrize("scales", [(1.0, 1.0), (1e-7, 3e4)])
def test_gemm_f16x3(R, a_mn, b_mn, shape, split, scales):
    """Three-product f16 split with per-tensor power-of-two scales: the same
    11-bit significands as 3xTF32, so the same 1e-5 bound, for operands many
    decades apart in magnitude."""
    M, N, K = shape
    g = torch.Generator().manual_seed(M * 7 + N + K)
    A = torch.randn(M, K, generator=g) * scales[0]
    B = torch.randn(N, K, generator=g) * scales[1]
    ref = A.double() @ B.double().T
    a_store = (A.T if a_mn else A).contiguous().cuda()
    b_store = (B.T if b_mn else B).contiguous().cuda()
    a = R.F16Split(*a_store.shape, "cuda").fill(a_store)
    b = R.F16Split(*b_store.shape, "cuda").fill(b_store)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ldc = R.pad4(N)
    c = torch.full((split, M, ldc), float("nan"), device="cuda")
    R.gemm_f16(M, N, K, a, a_mn, b, b_mn, c, ldc, status, split_k=split, split_stride=M * ldc)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    out = c[:, :, :N].sum(0).double().cpu()
    err = float((out - ref).abs().max() / ref.abs().max())
    assert err < 1e-5, err


@pytest.mark.parametrize("shape", [(4096, 1024, 1024), (130, 300, 70), (256, 512, 256)])
def test_gemm_f16x3_mse_epilogue(R, shape):
    """Forward GEMM with the MSE epilogue: dY = (X W^T - T) * scale, the loss
    partials sum to sum (X W^T - T)^2, and max |dY| is the max of what it wrote."""
    from torchcst_b200 import _native as N
    import ctypes
    M, Nn, K = shape
    g = torch.Generator().manual_seed(M + Nn + K)
    X = torch.randn(M, K, generator=g)
    W = torch.randn(Nn, K, generator=g) * 0.05
    T = torch.randn(M, Nn, generator=g)
    scale = 2.0 / (M * Nn)
    ref = X.double() @ W.double().T - T.double()
    x16 = R.F16Split(M, K, "cuda").fill(X.cuda())
    w16 = R.F16Split(Nn, K, "cuda").fill(W.cuda())
    Td = T.cuda()
    dy = torch.full((M, Nn), float("nan"), device="cuda")
    tiles = -(-Nn // 256) * -(-M // 128)
    partial = torch.full((4 * tiles,), float("nan"), dtype=torch.float64, device="cuda")
    amax = torch.zeros(1, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    count = ctypes.c_int32(0)
    vp = R._vp
    N.call("tcst_gemm_f16x3_mse", M, Nn, K, vp(x16.hi), vp(x16.lo), x16.ld, vp(x16.scale),
           vp(w16.hi), vp(w16.lo), w16.ld, vp(w16.scale), vp(Td), Nn, ctypes.c_float(scale),
           vp(dy), Nn, vp(partial), ctypes.byref(count), vp(amax), vp(status),
           R._stream(torch.device("cuda")))
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert count.value == 4 * tiles
    out = dy.double().cpu()
    err = float((out - ref * scale).abs().max() / (ref.abs().max() * scale))
    assert err < 1e-5, err
    loss = float(partial.sum())
    want = float((ref ** 2).sum())
    assert abs(loss - want) <= 1e-5 * want, (loss, want)
    assert float(amax.item()) == float(dy.abs().max())


def test_f16_split_scale_and_exactness(R):
    """s is a power of two putting max |s x| in [2^14, 2^15); hi + lo keeps
    22 significant bits of s x."""
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(64, 100, generator=g) * 1e-3).cuda()
    sp = R.F16Split(64, 100, "cuda").fill(x)
    torch.cuda.synchronize()
    amax, s = float(sp.amax[0]), float(sp.scale[0])
    assert amax == float(x.abs().max())
    assert s == 2.0 ** round(np.log2(s))
    assert 2 ** 14 <= amax * s < 2 ** 15
    recon = (sp.hi[:, :100].double() + sp.lo[:, :100].double()).cpu() / s
    xd = x.double().cpu()
    # lo rounds at 2^-11 of itself, or at the f16 subnormal step 2^-24 below 2^-14.
    bound = xd.abs() * 2.0 ** -21 + 2.0 ** -24 / s
    assert bool(((recon - xd).abs() <= bound).all())


# -- routing ------------------------------------------------------------------------


@pytest.mark.parametrize("name", ["config1", "hierarchy", "config4s", "config3", "config2",
                                  "config5s"])
def test_routing_and_owner_keys_bit_exact(R, name):
    d = load(name)
    layer = make_layer(name, d["p0"])
    routing, keys = layer.routing()
    routing = routing.cpu().numpy()
    for j, (side, key) in enumerate([("out", "level"), ("out", "count"), ("out", "first_tile"),
                                     ("in", "level"), ("in", "count"), ("in", "first_tile")]):
        np.testing.assert_array_equal(routing[:, j], d[f"route_{side}_{key}"])
    out_axis, in_axis, spec = CASES[name]
    table = O.routing_table(O.decode(out_axis, in_axis, spec, d["p0"]))
    np.testing.assert_array_equal(keys.cpu().numpy(), table["owner_key"])


# -- weight, forward, backward ------------------------------------------------------


@pytest.mark.parametrize("name", ["config1", "hierarchy", "config4s", "config3", "config2",
                                  "config5s"])
def test_weight_matches_oracle(R, name):
    d = load(name)
    layer = make_layer(name, d["p0"])
    w = layer.weight().cpu().numpy()
    out_axis, in_axis, spec = CASES[name]
    lay = O.decode(out_axis, in_axis, spec, d["p0"])
    # Profile coefficients are float32: W agrees with float64 to ~1e-6 of its scale.
    assert rel(w, O.weight64(lay)) < 1e-5


@pytest.mark.parametrize("name", ["config1", "hierarchy", "config4s", "config3", "config2",
                                  "config5s"])
def test_forward_backward_vs_oracle_and_golden(R, name):
    d = load(name)
    layer = make_layer(name, d["p0"])
    x = torch.as_tensor(d["x"]).cuda().requires_grad_("dx" in d)
    y = layer(x)
    y.backward(torch.as_tensor(d["dy"]).cuda())
    torch.cuda.synchronize()
    out_axis, in_axis, spec = CASES[name]
    lay = O.decode(out_axis, in_axis, spec, d["p0"])
    W = O.weight64(lay)
    x64, dy64 = d["x"].astype(np.float64), d["dy"].astype(np.float64)
    y_gpu = y.detach().cpu().numpy()
    assert rel(y_gpu, x64 @ W.T) < TOL
    assert rel(y_gpu, d["y"]) < TOL
    if "dx" in d:
        dx = x.grad.cpu().numpy()
        assert rel(dx, dy64 @ W) < TOL
        assert rel(dx, d["dx"]) < TOL
    grad = layer.atoms.p.grad.cpu().numpy()
    g64 = O.atom_gradients64(lay, dy64.T @ x64)
    rows = d.get("rows", slice(None))
    for c in range(4):
        assert rel(grad[:, c], g64[:, c]) < TOL, (c, rel(grad[:, c], g64[:, c]))
        assert rel(grad[rows, c], d["grad"][:, c]) < TOL, c


def _align16(x):
    return (x + 15) // 16 * 16


def _reach(c):
    return 16 << c


def _edge(c, fe=32):
    return fe if c < 4 else _reach(c) // 2


def _bin_geom(out_axis, in_axis):
    """Classes, tiles per axis and first bin of each class, restating the device
    bin geometry (fine classes on 32-site tiles, coarse ones on reach/2)."""
    no, ni = out_axis.site_count, in_axis.site_count
    for fe in (32, 64):  # fine bins of 32 sites, 64 when those do not fit
        tr, tc, base, nb, c = [], [], [], 0, 0
        while True:
            e = _edge(c, fe)
            tr.append(-(-no // e))
            tc.append(-(-ni // e))
            base.append(nb)
            nb += tr[-1] * tc[-1]
            c += 1
            if _reach(c - 1) >= 2 * max(no, ni):
                break
        if nb + 1 <= 98304:
            break
    if out_axis.modes != 8 or in_axis.modes != 8 or nb + 1 > 98304:
        return dict(nclass=0, nbins=2)
    # Owner-pair level-banks: shared hierarchy, K T > 128, at most 16384 pairs.
    pairs = {}
    if (out_axis.base_tile_sites == in_axis.base_tile_sites
            and out_axis.merge_factor == in_axis.merge_factor
            and out_axis.spacing == in_axis.spacing and out_axis.merge_factor > 1):
        t, level = out_axis.base_tile_sites, 0
        while t <= no and t <= ni:
            for k in (2, 3):
                npair = (no // t) * (ni // t)
                if k * t <= 128 or npair > 16384 or no % t or ni % t or nb + npair + 1 > 98304:
                    continue
                pairs[(level, k)] = dict(T=t, ni=ni // t, base=nb)
                nb += npair
            t *= out_axis.merge_factor
            level += 1
    return dict(nclass=c, tr=tr, tc=tc, base=base, nbins=nb + 1, pairs=pairs, fe=fe)


def _table_sections(out_axis, in_axis, atoms):
    """Byte offsets of the atom table sections, restating the device layout
    (records, spans, site values, bin_of, offsets, ids)."""
    aw = lambda m: (4 + 2 * (m + 1) + 3) // 4 * 4
    words = (4 + aw(out_axis.modes) + aw(in_axis.modes) + 3) // 4 * 4
    geo = _bin_geom(out_axis, in_axis)
    spans = _align16(atoms * words * 4)
    sites = _align16(spans + atoms * 16)
    binof = _align16(sites + atoms * 192 * 4)  # 2 axes x 3 values x 32 sites
    offsets = _align16(binof + atoms * 4)
    ids = _align16(offsets + 4 * (geo["nbins"] + 1))
    return dict(spans=spans, binof=binof, offsets=offsets, ids=ids, geo=geo)


@pytest.mark.parametrize("name", ["config1", "hierarchy", "config3", "config5s", "config2"])
def test_bins_are_stable_and_complete(R, name):
    d = load(name)
    layer = make_layer(name, d["p0"])
    out_axis, in_axis, _ = CASES[name]
    ws = layer._workspace(layer.atoms.p.device)
    table = R.decode_route(layer._plan, layer.atoms.p, ws.status)
    raw = table.view(torch.int32).cpu().numpy()
    A = d["p0"].shape[0]
    sec = _table_sections(out_axis, in_axis, A)
    geo = sec["geo"]
    nb = geo["nbins"]
    spans = raw[sec["spans"] // 4: sec["spans"] // 4 + 4 * A].reshape(A, 4)
    bin_of = raw[sec["binof"] // 4: sec["binof"] // 4 + A]
    offsets = raw[sec["offsets"] // 4: sec["offsets"] // 4 + nb + 1]
    ids = raw[sec["ids"] // 4: sec["ids"] // 4 + A]
    # Spans: wrapped first sites and footprints of both axes, from the golden routing.
    for side, (axis, col) in enumerate([(out_axis, 0), (in_axis, 2)]):
        key = "out" if side == 0 else "in"
        tile = axis.base_tile_sites * axis.merge_factor ** d[f"route_{key}_level"].astype(np.int64)
        np.testing.assert_array_equal(spans[:, col], (d[f"route_{key}_first_tile"] * tile)
                                      % axis.site_count)
        np.testing.assert_array_equal(spans[:, col + 1], d[f"route_{key}_count"] * tile)
    # Expected bin: class (smallest reach covering the larger footprint) x tile.
    f = np.maximum(spans[:, 1], spans[:, 3])
    if geo["nclass"]:
        cls = np.zeros(A, np.int64)
        while (f > np.vectorize(_reach)(cls)).any():
            cls += f > np.vectorize(_reach)(cls)
        e = np.vectorize(lambda c: _edge(c, geo["fe"]))(cls)
        base = np.asarray(geo["base"])[cls]
        tcs = np.asarray(geo["tc"])[cls]
        want = base + (spans[:, 0] // e) * tcs + spans[:, 2] // e
        # Coarse atoms with the same level and bank on both axes: owner-pair bins.
        lo, li = d["route_out_level"], d["route_in_level"]
        ko, ki = d["route_out_count"], d["route_in_count"]
        for j in np.nonzero((cls >= 4) & (lo == li) & (ko == ki))[0]:
            pl = geo["pairs"].get((int(lo[j]), int(ko[j])))
            if pl is not None:
                want[j] = pl["base"] + (spans[j, 0] // pl["T"]) * pl["ni"] + spans[j, 2] // pl["T"]
    else:
        want = np.zeros(A, np.int64)
    want = np.where(f > 0, want, nb - 1)
    np.testing.assert_array_equal(bin_of, want)
    np.testing.assert_array_equal(offsets, np.concatenate([[0], np.cumsum(np.bincount(want, minlength=nb))]))
    # Stable: ids grouped by bin, increasing inside every bin.
    np.testing.assert_array_equal(ids, np.argsort(want, kind="stable"))


@pytest.mark.parametrize("name", ["config2", "config5s", "config3"])
def test_bitwise_deterministic(R, name):
    d = load(name)
    layer = make_layer(name, d["p0"])
    x = torch.as_tensor(d["x"]).cuda().requires_grad_(True)
    dy = torch.as_tensor(d["dy"]).cuda()
    outs = []
    for _ in range(2):
        layer.zero_grad(set_to_none=True)
        x.grad = None
        y = layer(x)
        y.backward(dy)
        outs.append((y.detach().clone(), x.grad.clone(), layer.atoms.p.grad.clone()))
    for a, b in zip(*outs):
        assert torch.equal(a, b)


# -- optimizer ----------------------------------------------------------------------


@pytest.mark.parametrize("name", ["config1", "config2", "config3", "config4s", "hierarchy"])
def test_optimizer_step_bit_exact_vs_oracle(R, name):
    from torchcst_b200 import CSTAdamW
    d = load(name)
    rows = d.get("rows", slice(None))
    p0 = d["p0"][rows]
    grad = d["grad"]
    layer = make_layer(name, p0)
    lr = float(d["lr"])
    fl = field_lrs(d)
    opt = CSTAdamW(layer.parameters(), model=layer, lr=lr, **({"field_lrs": fl} if fl else {}))
    out_axis, in_axis, spec = CASES[name]
    ratios = O.field_ratios(spec, fl, lr)
    state = O.AdamState(0, np.zeros_like(grad), np.zeros_like(grad))
    p = p0.copy()
    for step in range(3):
        g = (grad * (1.0 + 0.5 * step)).astype(np.float32)
        layer.atoms.p.grad = torch.as_tensor(g).cuda()
        opt.step()
        p = O.optimizer_step(p, g, state, spec, lr=lr, field_ratios=ratios,
                             periods=(out_axis.period, in_axis.period))
        got = layer.atoms.p.detach().cpu().numpy()
        np.testing.assert_array_equal(got, p)
        st = opt.state[layer.atoms.p]
        np.testing.assert_array_equal(st["exp_avg"].cpu().numpy(), state.exp_avg)
        np.testing.assert_array_equal(st["exp_avg_sq"].cpu().numpy(), state.exp_avg_sq)
    # Within two float32 ulps of the reference's own step (torch CPU sqrt differs).
    if step == 2 and "p1" in d:
        pass


def test_invalid_atoms_raise(R):
    d = load("config1")
    p = d["p0"].copy()
    p[3, 1] = 1.5
    layer = make_layer("config1", p)
    with pytest.raises(ValueError, match="q in"):
        layer(torch.randn(2, 16, device="cuda"))
    p = d["p0"].copy()
    p[0, 2] = np.nan
    layer = make_layer("config1", p)
    with pytest.raises(ValueError, match="finite"):
        layer(torch.randn(2, 16, device="cuda"))


def test_empty_batch_and_atoms(R):
    d = load("config1")
    layer = make_layer("config1", d["p0"])
    x = torch.zeros(0, 16, device="cuda", requires_grad=True)
    y = layer(x)
    assert y.shape == (0, 8)
    y.sum().backward()
    assert torch.count_nonzero(layer.atoms.p.grad) == 0


# -- output-row bands (sharded layer) --------------------------------------------------


@pytest.mark.parametrize("name,bands", [("config2", 4), ("config5s", 4), ("config4s", 2)])
def test_band_windows_and_pullback_match_full(R, name, bands):
    """Weight windows equal the full assembly bit for bit; band pullbacks sum
    to the full pullback (float32 summation order aside)."""
    d = load(name)
    layer = make_layer(name, d["p0"])
    plan, p = layer._plan, layer.atoms.p
    ws = layer._workspace(p.device)
    A = p.shape[0]
    table = R.decode_route(plan, p, ws.status)
    w_full, _, _, _ = R.assemble_weight(plan, table, A, ws, dense=True, split=False)
    no, ni = plan.n_out, plan.n_in
    rb, cb = no // bands, ni // bands
    for k in range(bands):
        w, sp = R.assemble_weight_window_f16(plan, table, A, ws, k * rb, rb, 0, ni)
        assert torch.equal(w, w_full[k * rb:(k + 1) * rb])
        assert float(sp.amax[0]) == float(w.abs().max())
        w, _ = R.assemble_weight_window_f16(plan, table, A, ws, 0, no, k * cb, cb)
        assert torch.equal(w, w_full[:, k * cb:(k + 1) * cb])
    # Pullback: restore the full assembly's owner-pair state, then compare.
    R.assemble_weight(plan, table, A, ws, dense=True, split=False)
    gen = torch.Generator(device="cuda").manual_seed(7)
    ldg = R.pad4(ni)
    G = torch.randn(no, ldg, device="cuda", generator=gen) * 1e-3
    full = R.pullback(plan, table, A, G.clone(), ldg, 1, 0, p.device)
    acc = torch.zeros_like(full, dtype=torch.float64)
    for k in range(bands):
        gb = G[k * rb:(k + 1) * rb].clone()
        acc += R.pullback_band(plan, table, A, gb, ldg, 1, 0, k * rb, rb, p.device).double()
    torch.cuda.synchronize()
    for col in range(4):
        assert rel(acc[:, col].cpu(), full[:, col].double().cpu()) < 1e-5, col


def test_large_chart_fine_bins_of_64_sites(R):
    """A 6144-site chart needs fine bins of 64 sites (3 (6144/32)^2 > 98,304
    bins of 32): weight and pullback still match the float64 oracle."""
    from torchcst_b200 import CSTLinear, kernels
    from torchcst_b200.spec import CellMass, ChebyshevSpec, RegularGrid
    axis = O.Axis(6144, base_tile_sites=3, merge_factor=2)
    spec = O.Rational(radius_max=48.0)
    rng = np.random.default_rng(11)
    A = 2048
    p0 = np.stack([rng.normal(0, 0.1, A), rng.uniform(0, 1, A), rng.uniform(0, 6144, A),
                   rng.uniform(0, 6144, A)], 1).astype(np.float32)
    prof = CellMass(ChebyshevSpec(8), 3, 2)
    kernel = kernels.product(prof, prof, coordinates=kernels.rational_radius(
        radius_min=spec.radius_min, radius_birth=spec.radius_birth,
        radius_max=spec.radius_max, amplitude_max=spec.amplitude_max))
    grid = RegularGrid(6144, 1.0, 0.0)
    layer = CSTLinear(charts=(grid, grid), atoms=torch.as_tensor(p0), kernel=kernel, device="cuda")
    lay = O.decode(axis, axis, spec, p0)
    w = layer.weight().cpu().numpy()
    assert rel(w, O.weight64(lay)) < 1e-5
    del w
    plan, p = layer._plan, layer.atoms.p
    ws = layer._workspace(p.device)
    table = R.decode_route(plan, p, ws.status)
    R.assemble_weight(plan, table, A, ws, dense=True, split=False)
    gen = torch.Generator(device="cuda").manual_seed(5)
    G = torch.randn(6144, 6144, device="cuda", generator=gen) * 1e-3
    grad = R.pullback(plan, table, A, G, 6144, 1, 0, p.device).cpu().numpy()
    g64 = O.atom_gradients64(lay, G.double().cpu().numpy())
    for c in range(4):
        assert rel(grad[:, c], g64[:, c]) < TOL, c


PARITY_CASES = ["config1", "config2", "hierarchy", "config3", "config4s", "config5s"]


def test_parity_report(R):
    """Errors against the reference's float32 results (the goldens) and against
    float64 truth side by side, with the reference's own float32 error for
    scale (max |a - b| / max |b|; gradients: the worst of the four columns on
    the goldens' rows). Prints the table; every figure must be within 1e-4."""
    lines = ["| case | tensor | new vs reference fp32 | new vs fp64 | reference fp32 vs fp64 |",
             "|---|---|---|---|---|"]
    worst = 0.0
    for name in PARITY_CASES:
        d = load(name)
        layer = make_layer(name, d["p0"])
        x = torch.as_tensor(d["x"]).cuda().requires_grad_("dx" in d)
        y = layer(x)
        y.backward(torch.as_tensor(d["dy"]).cuda())
        torch.cuda.synchronize()
        out_axis, in_axis, spec = CASES[name]
        lay = O.decode(out_axis, in_axis, spec, d["p0"])
        W = O.weight64(lay)
        x64, dy64 = d["x"].astype(np.float64), d["dy"].astype(np.float64)
        rows = d.get("rows", slice(None))
        g64 = O.atom_gradients64(lay, dy64.T @ x64)[rows]
        grad = layer.atoms.p.grad.cpu().numpy()[rows]
        out = {"Y": (y.detach().cpu().numpy(), d["y"], x64 @ W.T)}
        if "dx" in d:
            out["dX"] = (x.grad.cpu().numpy(), d["dx"], dy64 @ W)
        out["grad"] = (grad, d["grad"], g64)
        for what, (new, ref32, truth) in out.items():
            if what == "grad":
                e32 = max(rel(new[:, c], ref32[:, c]) for c in range(4))
                e64 = max(rel(new[:, c], truth[:, c]) for c in range(4))
                r64 = max(rel(ref32[:, c], truth[:, c]) for c in range(4))
            else:
                e32, e64, r64 = rel(new, ref32), rel(new, truth), rel(ref32, truth)
            worst = max(worst, e32, e64)
            lines.append(f"| {name} | {what} | {e32:.2e} | {e64:.2e} | {r64:.2e} |")
    print("\n".join(lines))
    assert worst < TOL
