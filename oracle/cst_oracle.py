"""numpy restatement of torchcst's radius cell-mass Linear hot path (CPU oracle).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py`` (CPU baseline / reference arm). The product package never
imports it.

Every function names the reference source it restates (paths relative to the
torchcst source tree ``src/torchcst``). Two arithmetic modes are provided:

* ``*64`` helpers evaluate the mathematics in float64 ("truth"), used as the
  parity target for the CUDA path at tolerance;
* ``reference_step`` re-runs the reference's own *factored* algorithm in its
  own precision mix (float64 factors cast to float32, float32 GEMMs, float64
  factor backward, float32 AdamW) and is what the CPU baseline times.

Integer routing (level, bank, first tile, owner key) is evaluated with the same
float64 operation order as the reference, so it is bit-exact.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

F32 = np.float32
F64 = np.float64
TINY32 = float(np.finfo(np.float32).tiny)


def f32(value):
    """Round a Python float the way torchcst's float32 KernelState buffers do."""
    return float(np.float32(value))


# ---------------------------------------------------------------------------
# Declarations (kernels/radius_cell_mass.py:16-93, kernels/spec.py:133-157)
# ---------------------------------------------------------------------------


@dataclass(frozen=True)
class Axis:
    """One fixed 1-D flat-torus regular grid with its cell-mass hierarchy.

    Mirrors ``RadiusCellMassGrid`` (kernels/radius_cell_mass.py:16-26) plus the
    binding fields ``base_tile_sites``/``merge_factor`` and ``ChebyshevSpec.modes``.
    """

    site_count: int
    spacing: float = 1.0
    origin: float = 0.0
    base_tile_sites: int = 1
    merge_factor: int = 2
    modes: int = 8

    @property
    def period(self) -> float:
        return self.site_count * self.spacing

    def validate(self):
        """kernels/radius_cell_mass.py:55-66."""
        if self.site_count % self.base_tile_sites:
            raise ValueError("base_tile_sites must divide the chart site count")
        ratio = self.site_count // self.base_tile_sites
        while ratio > 1 and ratio % self.merge_factor == 0:
            ratio //= self.merge_factor
        if ratio != 1:
            raise ValueError("chart/base tile ratio must be a power of merge_factor")

    def tiles(self):
        """Tile site counts of every hierarchy level, base first."""
        out, tile = [], self.base_tile_sites
        while tile <= self.site_count:
            out.append(tile)
            tile *= self.merge_factor
        return out

    def banks(self):
        """(tile_sites, count K, node_offset, tile_count, level) per bank.

        Same enumeration as the reference CUDA twin ``parse_axis``
        (_backends/cuda/algorithms/linear/radius_cell_mass/common.cuh:51-60):
        per level, K=2 then K=3, each bank owning ``sites/tile`` nodes.
        """
        out, offset = [], 0
        for level, tile in enumerate(self.tiles()):
            for count in (2, 3):
                out.append((tile, count, offset, self.site_count // tile, level))
                offset += self.site_count // tile
        return out

    def node_count(self):
        return sum(self.site_count // t for t in self.tiles()) * 2


@dataclass(frozen=True)
class Rational:
    """RationalRadiusSpec (kernels/parameterizations/rational_radius.py:9-32).

    Scalars are stored as the float32 KernelState buffers hold them.
    """

    radius_min: float = 0.5
    radius_birth: float = 4.0
    radius_max: float = 50.0
    amplitude_max: float = 32.0

    def __post_init__(self):
        for name in ("radius_min", "radius_birth", "radius_max", "amplitude_max"):
            object.__setattr__(self, name, f32(getattr(self, name)))


@dataclass(frozen=True)
class Polar:
    """PolarAmpRadiusSpec with the rational envelope and its update settings.

    kernels/factories.py:403-460 (defaults), kernels/parameterizations/
    activity_width.py:68. ``input``/``output`` are (minimum, birth, maximum,
    upper_floor) RadiusBounds. Scalars are float32 buffers as in KernelState.
    """

    amplitude_max: float = 1.0
    w_c: float = 0.3
    kappa: float = 3.0
    lower_kappa: float = 3.0
    upper_decay_power: float = 1.0
    input: tuple = (0.5, 4.0, 50.0, 1.0)
    output: tuple = (0.5, 4.0, 50.0, 1.0)
    radial_regularization: float = 0.1
    activity_gain: float = 1.0
    activity_mode: str = "finite_chord"
    dormant_expansion_rate: float = 0.0

    def __post_init__(self):
        for name in ("amplitude_max", "w_c", "kappa", "lower_kappa",
                     "upper_decay_power", "radial_regularization",
                     "activity_gain", "dormant_expansion_rate"):
            object.__setattr__(self, name, f32(getattr(self, name)))
        object.__setattr__(self, "input", tuple(f32(v) for v in self.input))
        object.__setattr__(self, "output", tuple(f32(v) for v in self.output))


# ---------------------------------------------------------------------------
# Coordinate decode
# ---------------------------------------------------------------------------


def rational_decode(p, spec: Rational, dtype=F32):
    """Physical amplitude/radius of rational rows [a, q, mu_out, mu_in].

    _backends/torch/parameterizations/rational_radius.py:6-38. The radius is
    computed in float64, rounded to the parameter dtype (float32) and clamped
    to the representable closed interval with a straight-through gradient.
    Returns amplitude (f64), radius (f32 value as f64), dr/da and dr/dq (f64,
    the analytic Jacobian of the raw expression).
    """
    p = np.asarray(p)
    a = p[:, 0].astype(F64)
    q = p[:, 1].astype(F64)
    low, birth, high, cap = (spec.radius_min, spec.radius_birth,
                             spec.radius_max, spec.amplitude_max)
    if (not np.isfinite(p).all()) or np.any((q < 0) | (q > 1) | (np.abs(a) > cap)):
        raise ValueError(
            "rational radius requires finite rows, q in [0,1] and bounded amplitude")
    ratio = np.square(a / 0.3)
    denom = 1.0 + 3.0 * ratio
    lower = low + (birth - low) / denom
    log_lower = np.log(lower)
    log_high = math.log(high)
    raw = np.exp((1 - q) * log_lower + q * log_high)
    value = np.where(q == 0, lower, np.where(q == 1, high, raw))
    lo = dtype(low)
    if float(lo) < low:
        lo = np.nextafter(lo, dtype(np.inf))
    hi = dtype(high)
    if float(hi) > high:
        hi = np.nextafter(hi, dtype(0))
    if lo > hi:
        raise ValueError("radius interval has no representable value in parameter dtype")
    encoded = value.astype(dtype)
    radius = np.clip(encoded, lo, hi)
    dlower_da = -(birth - low) * (3.0 * 2.0 * a / 0.09) / np.square(denom)
    dr_da = raw * (1 - q) / lower * dlower_da
    dr_dq = raw * (log_high - log_lower)
    return dict(amplitude=a, radius_in=radius.astype(F64), radius_out=radius.astype(F64),
                radius32=radius, dr_da=dr_da, dr_dq=dr_dq)


def polar_amplitude_alpha(pair, amplitude_max, tiny=TINY32):
    """_backends/torch/parameterizations/polar_amp_width.py:127-139 (float64)."""
    s, t = pair[:, 0], pair[:, 1]
    radius_square = s * s + t * t
    safe = np.maximum(radius_square, tiny)
    amplitude = amplitude_max * s / np.sqrt(safe)
    alpha = np.clip((radius_square - 1.0) / 3.0, 0.0, 1.0)
    return amplitude, alpha, radius_square


def polar_radius(amplitude, alpha, bounds, spec: Polar):
    """Rational Polar width law, _width_bounds (polar_amp_width.py:158-244)."""
    minimum, birth, maximum, floor = bounds
    x = np.square(amplitude / spec.w_c)
    lower_delta = birth - minimum
    upper_delta = maximum - minimum
    upper_x = np.power(x, spec.upper_decay_power)
    upper = minimum + upper_delta * spec.kappa / (spec.kappa + upper_x)
    lower = minimum + lower_delta / (1.0 + spec.lower_kappa * x)
    upper = np.maximum(upper, floor)
    upper = np.maximum(upper, lower)
    sigma = np.exp((1.0 - alpha) * np.log(lower) + alpha * np.log(upper))
    return np.minimum(np.maximum(sigma, lower), upper)


def polar_decode(p, spec: Polar):
    """Amplitude (f64), detached radii and d amplitude/d(s,t) of Polar rows.

    _backends/torch/parameterizations/radius_cell_mass.py:10-28; radii are
    detached by _backends/torch/kernels/radius_cell_mass.py:241-243.
    """
    pair = np.asarray(p)[:, :2].astype(F64)
    amplitude, alpha, rs = polar_amplitude_alpha(pair, spec.amplitude_max)
    r_in = polar_radius(amplitude, alpha, spec.input, spec)
    r_out = polar_radius(amplitude, alpha, spec.output, spec)
    s, t = pair[:, 0], pair[:, 1]
    live = rs > TINY32
    r = np.sqrt(np.maximum(rs, TINY32))
    damp_ds = np.where(live, spec.amplitude_max * (1.0 / r - s * s / r**3),
                       spec.amplitude_max / r)
    damp_dt = np.where(live, -spec.amplitude_max * s * t / r**3, 0.0)
    return dict(amplitude=amplitude, radius_in=r_in, radius_out=r_out,
                damp_ds=damp_ds, damp_dt=damp_dt)


# ---------------------------------------------------------------------------
# Routing (_backends/torch/kernels/radius_cell_mass.py:17-123)
# ---------------------------------------------------------------------------


def relative_centers(centers, origin, period):
    """Stable float64 modular-relative coordinates (radius_cell_mass.py:17-63).

    Finite-period branch: fmod(fmod(mu, Q) - fmod(origin, Q), Q), negative
    results shifted by +Q (which can round to exactly Q).
    """
    encoded = np.asarray(centers).astype(F64)
    residue = np.fmod(encoded, period)
    origin_residue = math.fmod(origin, period)
    relative = np.fmod(residue - origin_residue, period)
    return np.where(relative < 0, relative + period, relative)


def route(axis: Axis, radius, centers):
    """Level, count K, first tile and owner node of every atom on one axis.

    radius_cell_mass.py:81-123 selects the smallest tile width >= R (float64
    compare of the routing radius), K = ceil(2R/T)+1 and
    first_tile = floor((mu_rel + s/2)/T - (K-1)/2). The owner node follows the
    reference CUDA twin ``classify`` (common.cuh:131-138, pipeline.cu:75-80).
    """
    R = np.asarray(radius, dtype=F64)
    if not np.isfinite(R).all() or not np.isfinite(np.asarray(centers, F64)).all():
        raise ValueError("radius and centers must be finite")
    if np.any((R <= 0) | (R > axis.period / 2)):
        raise ValueError("radius must lie in (0, chart period/2]")
    n = len(R)
    level = np.full(n, -1, np.int64)
    tile_sites = np.zeros(n, np.int64)
    count = np.zeros(n, np.int64)
    remaining = np.ones(n, bool)
    for lvl, tile in enumerate(axis.tiles()):
        width = tile * axis.spacing
        selected = remaining & (R <= width)
        level[selected] = lvl
        tile_sites[selected] = tile
        count[selected] = (np.ceil(2 * R[selected] / width)).astype(np.int64) + 1
        remaining &= ~selected
    if remaining.any():
        raise ValueError("radius does not fit the declared hierarchy")
    local = relative_centers(centers, axis.origin, axis.period)
    width = tile_sites * axis.spacing
    first_tile = np.floor((local + axis.spacing / 2) / width - (count - 1) / 2).astype(np.int64)
    bank = 2 * level + (count - 2)
    offsets = np.array([b[2] for b in axis.banks()], np.int64)
    tile_count = axis.site_count // tile_sites
    node = offsets[bank] + np.mod(first_tile, tile_count)
    return dict(level=level, tile_sites=tile_sites, count=count, first_tile=first_tile,
                bank=bank, node=node, local_center=local,
                period=(count * tile_sites) * axis.spacing)


def owner_keys(out_route, in_route, in_axis: Axis):
    """Owner key ``no * input_node_count + ni`` (pipeline.cu:75-80)."""
    return out_route["node"] * in_axis.node_count() + in_route["node"]


# ---------------------------------------------------------------------------
# Profile (_backends/torch/profiles/radius_fourier.py:14-72)
# ---------------------------------------------------------------------------


def density_coefficients(radius, period, modes):
    """Normalized Chebyshev-square Fourier coefficients c_0..c_M and dc/dR.

    radius_fourier.py:14-58: sample the scaled Chebyshev recurrence with
    z = cos^2(pi R/P) at 2M+1 points, square, FFT, symmetrize, normalize so
    c_0 = 1/P. ``period`` may be per atom. The derivative differentiates the
    same recurrence (the detached ``scale`` cancels in the normalization).
    """
    R = np.asarray(radius, F64)[:, None]
    P = np.broadcast_to(np.asarray(period, F64), (R.shape[0],))[:, None]
    n = 2 * modes + 1
    theta = 2 * np.pi * np.arange(n, dtype=F64) / n
    cosine = np.cos(theta / 2)[None, :]
    arg = np.pi * R / P
    ibs = np.square(np.cos(arg))
    dibs = -(np.pi / P) * np.sin(2 * arg)
    prev = np.full_like(ibs + cosine, 2.0)
    dprev = np.zeros_like(prev)
    cur = np.broadcast_to(cosine, prev.shape).copy()
    dcur = np.zeros_like(prev)
    for _ in range(2, modes + 1):
        nxt = cosine * cur - ibs * prev / 4
        dnxt = cosine * dcur - (dibs * prev + ibs * dprev) / 4
        prev, cur = cur, nxt
        dprev, dcur = dcur, dnxt
    scale = np.abs(cur).max(axis=-1, keepdims=True)
    density = np.square(cur / scale)
    ddensity = 2 * (cur / scale) * (dcur / scale)
    coef = np.fft.fftshift(np.fft.fft(density, axis=-1), axes=-1).real / n
    dcoef = np.fft.fftshift(np.fft.fft(ddensity, axis=-1), axes=-1).real / n
    coef = (coef + coef[:, ::-1]) / 2
    dcoef = (dcoef + dcoef[:, ::-1]) / 2
    c0 = coef[:, modes:modes + 1]
    dc0 = dcoef[:, modes:modes + 1]
    c = coef[:, modes:] / (P * c0)
    dc = (dcoef[:, modes:] * c0 - coef[:, modes:] * dc0) / (P * c0 * c0)
    return c, dc


def integrated_cells(c, dc, local_center, period, sites, spacing, modes):
    """Whole-cell masses m, dm/dmu and dm/dR on unwrapped sites.

    radius_fourier.py:61-72: m = s*(c_0 + 2 sum_k c_k sinc(k s/P) cos(2 pi k (n s - mu)/P)).
    """
    k = np.arange(1, modes + 1, dtype=F64)
    P = np.asarray(period, F64)[:, None]
    disp = sites.astype(F64) * spacing - np.asarray(local_center, F64)[:, None]
    phase = (2 * np.pi / P)[..., None] * disp[..., None] * k
    cell = np.sinc(k[None, :] * spacing / P)[:, None, :]
    ck = c[:, None, 1:] * cell
    dck = dc[:, None, 1:] * cell
    cosp, sinp = np.cos(phase), np.sin(phase)
    m = spacing * (c[:, :1] + 2 * (ck * cosp).sum(-1))
    dm_dR = spacing * (dc[:, :1] + 2 * (dck * cosp).sum(-1))
    omega = (2 * np.pi / P)[..., None] * k
    dm_dmu = spacing * 2 * (ck * sinp * omega).sum(-1)
    return m, dm_dmu, dm_dR


@dataclass
class AxisProfiles:
    """Per-atom footprints on one axis, grouped by footprint length.

    ``groups`` holds (atom indices, sites mod N [A_g,F], m, dm/dmu, dm/dR).
    """

    axis: Axis
    routing: dict
    groups: list = field(default_factory=list)

    def dense(self, atoms, which=0):
        """Dense [N, A] float64 matrix of column ``which`` (0=m, 1=dmu, 2=dR)."""
        n = self.axis.site_count
        out = np.zeros(n * atoms, F64)
        for idx, sites, *vals in self.groups:
            flat = (sites * atoms + idx[:, None]).ravel()
            out += np.bincount(flat, weights=vals[which].ravel(), minlength=n * atoms)
        return out.reshape(n, atoms)


def axis_profiles(axis: Axis, radius, centers):
    """radius_cell_mass.py:66-123 with derivatives, kept sparse per atom."""
    r = route(axis, radius, centers)
    prof = AxisProfiles(axis, r)
    key = r["tile_sites"] * 4 + r["count"]
    for value in np.unique(key):
        idx = np.nonzero(key == value)[0]
        tile, count = int(value // 4), int(value % 4)
        P = count * tile * axis.spacing
        c, dc = density_coefficients(np.asarray(radius, F64)[idx], P, axis.modes)
        sites = r["first_tile"][idx, None] * tile + np.arange(count * tile)
        m, dmu, dR = integrated_cells(c, dc, r["local_center"][idx],
                                      np.full(len(idx), P), sites, axis.spacing,
                                      axis.modes)
        prof.groups.append((idx, np.mod(sites, axis.site_count), m, dmu, dR))
    return prof


# ---------------------------------------------------------------------------
# Layer math
# ---------------------------------------------------------------------------


@dataclass
class Layer:
    """A decoded layer: axes, coordinates and per-axis profiles."""

    out_axis: Axis
    in_axis: Axis
    spec: object
    p: np.ndarray
    dec: dict = None
    out_prof: AxisProfiles = None
    in_prof: AxisProfiles = None

    @property
    def atoms(self):
        return self.p.shape[0]


def decode(out_axis: Axis, in_axis: Axis, spec, p, dtype=F32) -> Layer:
    """Decode coordinates and evaluate both axes' cell-mass footprints.

    ``dtype`` is the parameter dtype of the emulated reference model: float32
    rounds the rational radius to float32 before routing (the CSTLinear
    default), float64 keeps it in double (a ``.double()`` model).
    """
    out_axis.validate()
    in_axis.validate()
    p = np.asarray(p, dtype)
    if p.ndim != 2 or p.shape[1] != 4:
        raise ValueError("radius cell masses require floating-point [atom,4] rows")
    if not np.isfinite(p).all():
        raise ValueError("atom parameters must be finite")
    dec = (rational_decode(p, spec, dtype) if isinstance(spec, Rational)
           else polar_decode(p, spec))
    lay = Layer(out_axis, in_axis, spec, p, dec)
    lay.out_prof = axis_profiles(out_axis, dec["radius_out"], p[:, 2])
    lay.in_prof = axis_profiles(in_axis, dec["radius_in"], p[:, 3])
    return lay


def routing_table(lay: Layer):
    """Integer routing of every atom: [level, K, first_tile] per axis + owner key."""
    ro, ri = lay.out_prof.routing, lay.in_prof.routing
    return dict(
        out_level=ro["level"], out_count=ro["count"], out_first_tile=ro["first_tile"],
        in_level=ri["level"], in_count=ri["count"], in_first_tile=ri["first_tile"],
        owner_key=owner_keys(ro, ri, lay.in_axis),
    )


def routing_only(out_axis: Axis, in_axis: Axis, spec, p, dtype=F32):
    """Integer routing and owner keys without evaluating any profile, for layers
    too large for :func:`decode` (every atom of a 262,144-atom layer): the
    decode of rational_radius.py:6-38 or polar_amp_width.py:127-245 and the
    routing expressions of radius_cell_mass.py:81-123, nothing else."""
    out_axis.validate()
    in_axis.validate()
    p = np.asarray(p, dtype)
    dec = (rational_decode(p, spec, dtype) if isinstance(spec, Rational)
           else polar_decode(p, spec))
    ro = route(out_axis, dec["radius_out"], p[:, 2])
    ri = route(in_axis, dec["radius_in"], p[:, 3])
    return dict(out_level=ro["level"], out_count=ro["count"], out_first_tile=ro["first_tile"],
                in_level=ri["level"], in_count=ri["count"], in_first_tile=ri["first_tile"],
                owner_key=owner_keys(ro, ri, in_axis))


def factored64(lay: Layer, x, dy):
    """(Y, dX, p.grad) in float64 through dense factors, the association of the
    reference's factored path (_backends/torch/operators/linear.py:47-66):
    Y = (X phi_in) phi_out^T with phi_out = amp m_out. Its cost is O(B A N)
    rather than O(A F_out F_in), so it serves layers of few atoms with wide
    (folded) footprints, such as the 128-atom model of a wide-layer check."""
    x = np.asarray(x, F64)
    dy = np.asarray(dy, F64)
    A = lay.atoms
    amp = lay.dec["amplitude"]
    m_out, dmu_out, dR_out = (lay.out_prof.dense(A, k) for k in range(3))
    m_in, dmu_in, dR_in = (lay.in_prof.dense(A, k) for k in range(3))
    u = x @ m_in          # [B, A] atom values before the amplitude
    v = dy @ m_out        # [B, A] upstream cotangent per atom
    y = (u * amp) @ m_out.T
    dx = (v * amp) @ m_in.T
    d_amp = (u * v).sum(0)
    d_mu_out = amp * (u * (dy @ dmu_out)).sum(0)
    d_mu_in = amp * (v * (x @ dmu_in)).sum(0)
    d_R = amp * ((u * (dy @ dR_out)).sum(0) + (v * (x @ dR_in)).sum(0))
    grad = np.zeros((A, 4))
    if isinstance(lay.spec, Rational):
        grad[:, 0] = d_amp + d_R * lay.dec["dr_da"]
        grad[:, 1] = d_R * lay.dec["dr_dq"]
    else:
        grad[:, 0] = d_amp * lay.dec["damp_ds"]
        grad[:, 1] = d_amp * lay.dec["damp_dt"]
    grad[:, 2] = d_mu_out
    grad[:, 3] = d_mu_in
    return y, dx, grad


def _pairs(lay: Layer):
    """Yield matched (indices, out sites, out vals, in sites, in vals) chunks."""
    out_map = {}
    for g in lay.out_prof.groups:
        for j, a in enumerate(g[0]):
            out_map[a] = (g, j)
    for gi in lay.in_prof.groups:
        idx_in = gi[0]
        fo = {}
        for j, a in enumerate(idx_in):
            go, jo = out_map[a]
            fo.setdefault(id(go), (go, []))[1].append((j, jo))
        for go, lst in fo.values():
            ji = np.array([x[0] for x in lst])
            jo = np.array([x[1] for x in lst])
            yield (idx_in[ji], [v[jo] for v in go[1:]], [v[ji] for v in gi[1:]])


def weight64(lay: Layer):
    """Dense W[o,i] = sum_a amp_a m_out,a(o) m_in,a(i) in float64.

    Equivalent to phi_out @ phi_in.T of radius_cell_mass.py:225-263 with images
    folded modulo N.
    """
    W = np.zeros((lay.out_axis.site_count, lay.in_axis.site_count), F64)
    amp = lay.dec["amplitude"]
    for idx, (so, mo, _, _), (si, mi, _, _) in _pairs(lay):
        for start in range(0, len(idx), 4096):
            sl = slice(start, start + 4096)
            vals = amp[idx[sl], None, None] * mo[sl, :, None] * mi[sl, None, :]
            rows = np.broadcast_to(so[sl, :, None], vals.shape)
            cols = np.broadcast_to(si[sl, None, :], vals.shape)
            np.add.at(W, (rows, cols), vals)
    return W


def forward64(lay: Layer, x):
    return np.asarray(x, F64) @ weight64(lay).T


def atom_gradients64(lay: Layer, G):
    """Atom-parameter gradient from G = dY^T X (float64), [A, 4] float64.

    Restates the autograd chain of radius_cell_mass.py:225-247 through
    integrated_cells / density_coefficients / physical_parameters:
    d amp = m_out^T G m_in, d mu_out = amp m_out'^T G m_in, d mu_in likewise,
    d R = amp (dR m_out^T G m_in + m_out^T G dR m_in); then the rational chain
    (a, q) or the Polar amplitude chain (s, t) with detached radii.
    """
    A = lay.atoms
    amp = lay.dec["amplitude"]
    d_amp = np.zeros(A)
    d_mu_out = np.zeros(A)
    d_mu_in = np.zeros(A)
    d_R = np.zeros(A)
    for idx, (so, mo, dmo, dRo), (si, mi, dmi, dRi) in _pairs(lay):
        for start in range(0, len(idx), 2048):
            sl = slice(start, start + 2048)
            g = G[so[sl][:, :, None], si[sl][:, None, :]]
            gm = np.einsum("aoi,ai->ao", g, mi[sl])
            d_amp[idx[sl]] = np.einsum("ao,ao->a", gm, mo[sl])
            d_mu_out[idx[sl]] = amp[idx[sl]] * np.einsum("ao,ao->a", gm, dmo[sl])
            d_mu_in[idx[sl]] = amp[idx[sl]] * np.einsum(
                "aoi,ao,ai->a", g, mo[sl], dmi[sl])
            d_R[idx[sl]] = amp[idx[sl]] * (np.einsum("ao,ao->a", gm, dRo[sl])
                                           + np.einsum("aoi,ao,ai->a", g, mo[sl], dRi[sl]))
    grad = np.zeros((A, 4))
    if isinstance(lay.spec, Rational):
        grad[:, 0] = d_amp + d_R * lay.dec["dr_da"]
        grad[:, 1] = d_R * lay.dec["dr_dq"]
    else:
        grad[:, 0] = d_amp * lay.dec["damp_ds"]
        grad[:, 1] = d_amp * lay.dec["damp_dt"]
    grad[:, 2] = d_mu_out
    grad[:, 3] = d_mu_in
    return grad


def backward64(lay: Layer, x, dy):
    """(dX, p.grad) in float64 for upstream gradient dY."""
    x = np.asarray(x, F64)
    dy = np.asarray(dy, F64)
    W = weight64(lay)
    G = dy.T @ x
    return dy @ W, atom_gradients64(lay, G)


# ---------------------------------------------------------------------------
# Reference factored algorithm in the reference's precision mix (CPU baseline)
# ---------------------------------------------------------------------------


def factors32(lay: Layer):
    """phi_in [N_in, A], phi_out [N_out, A] as float32 (radius_cell_mass.py:245-247)."""
    amp = lay.dec["amplitude"]
    phi_in = lay.in_prof.dense(lay.atoms).astype(F32)
    phi_out = (lay.out_prof.dense(lay.atoms) * amp[None, :]).astype(F32)
    return phi_in, phi_out


def factored_forward32(lay: Layer, x):
    """_backends/torch/operators/linear.py:47-66: (X phi_in) phi_out^T in float32."""
    phi_in, phi_out = factors32(lay)
    atom_values = np.asarray(x, F32) @ phi_in
    return atom_values @ phi_out.T, (phi_in, phi_out, atom_values)


def factored_backward_gemms32(x, dy, saved):
    """The four float32 GEMMs of the factored path's autograd backward."""
    phi_in, phi_out, atom_values = saved
    x = np.asarray(x, F32)
    dy = np.asarray(dy, F32)
    d_atom_values = dy @ phi_out
    d_phi_out = dy.T @ atom_values
    dx = d_atom_values @ phi_in.T
    d_phi_in = x.T @ d_atom_values
    return dx, d_phi_out, d_phi_in


def factor_chain(lay: Layer, d_phi_out, d_phi_in):
    """float64 chain from d phi to d p (the ``.to(p.dtype)`` cast backward
    promotes to float64): gather each atom's footprint entries and contract with
    dm/d(amp, mu, R), then the rational or Polar coordinate chain."""
    A = lay.atoms
    amp = lay.dec["amplitude"]
    d_amp = np.zeros(A)
    d_mu_out = np.zeros(A)
    d_mu_in = np.zeros(A)
    d_R = np.zeros(A)
    fo = np.ascontiguousarray(d_phi_out).ravel()
    fi = np.ascontiguousarray(d_phi_in).ravel()
    for idx, sites, m, dmu, dR in lay.out_prof.groups:
        g = fo[sites * A + idx[:, None]].astype(F64)
        d_amp[idx] += (g * m).sum(-1)
        d_mu_out[idx] += amp[idx] * (g * dmu).sum(-1)
        d_R[idx] += amp[idx] * (g * dR).sum(-1)
    for idx, sites, m, dmu, dR in lay.in_prof.groups:
        g = fi[sites * A + idx[:, None]].astype(F64)
        d_mu_in[idx] += (g * dmu).sum(-1)
        d_R[idx] += (g * dR).sum(-1)
    grad = np.zeros((A, 4))
    if isinstance(lay.spec, Rational):
        grad[:, 0] = d_amp + d_R * lay.dec["dr_da"]
        grad[:, 1] = d_R * lay.dec["dr_dq"]
    else:
        grad[:, 0] = d_amp * lay.dec["damp_ds"]
        grad[:, 1] = d_amp * lay.dec["damp_dt"]
    grad[:, 2] = d_mu_out
    grad[:, 3] = d_mu_in
    return grad.astype(F32)


def factored_backward32(lay: Layer, x, dy, saved):
    """Autograd backward of the factored path: four float32 GEMMs, then the
    float64 factor chain."""
    dx, d_phi_out, d_phi_in = factored_backward_gemms32(x, dy, saved)
    return dx, factor_chain(lay, d_phi_out, d_phi_in)


# ---------------------------------------------------------------------------
# Optimizer (optim/adamw.py:230-294, optim/_field_lrs.py:128-134,
# _backends/torch/updates/rational_radius.py:10-29,
# _backends/torch/algorithms/polar_update/executor.py:18-176)
# ---------------------------------------------------------------------------


@dataclass
class AdamState:
    step: int
    exp_avg: np.ndarray
    exp_avg_sq: np.ndarray


def _fma32(a, b, c):
    """Single-rounding float32 fused multiply-add (vectorized torch lerp)."""
    return (a.astype(F64) * b.astype(F64) + c.astype(F64)).astype(F32)


def adamw32(p, g, state: AdamState, *, lr, beta1=0.9, beta2=0.999, eps=1e-8,
            weight_decay=0.0):
    """torch.optim.adam._single_tensor_adam (decoupled decay, non-capturable).

    Operation order: step += 1; p *= 1 - lr wd; m = lerp(m, g, 1-beta1)
    (fma form); v = v*beta2 + ((1-beta2)*g)*g; denom = sqrt(v)/sqrt(bc2)+eps;
    p += ((-lr/bc1) * m) / denom (addcdiv order). Scalars cast to float32 as
    torch does. ``sqrt`` is the IEEE correctly rounded one; torch's CPU
    vectorized sqrt differs from it by one ulp on a fraction of a percent of
    elements, so the reference's own atoms after a step agree to ~1 ulp.
    """
    p = p.astype(F32).copy()
    g = g.astype(F32)
    state.step += 1
    if weight_decay != 0:
        p = (p * F32(1 - lr * weight_decay)).astype(F32)
    m = _fma32(np.full_like(g, F32(1 - beta1)), (g - state.exp_avg).astype(F32), state.exp_avg)
    v = (state.exp_avg_sq * F32(beta2)).astype(F32)
    v = (v + ((F32(1 - beta2) * g).astype(F32) * g).astype(F32)).astype(F32)
    bc1 = 1 - beta1 ** state.step
    bc2 = 1 - beta2 ** state.step
    step_size = lr / bc1
    bc2s = bc2 ** 0.5
    denom = (np.sqrt(v) / F32(bc2s)).astype(F32)
    denom = (denom + F32(eps)).astype(F32)
    upd = ((F32(-step_size) * m).astype(F32) / denom).astype(F32)
    p = (p + upd).astype(F32)
    state.exp_avg = m
    state.exp_avg_sq = v
    return p


def apply_field_lrs(point, previous, ratios):
    """optim/_field_lrs.py:128-134: old + (proposal - old) * ratio per block."""
    point = point.copy()
    for first, last, ratio in ratios:
        old = previous[:, first:last]
        point[:, first:last] = (old + ((point[:, first:last] - old).astype(F32)
                                       * F32(ratio)).astype(F32)).astype(F32)
    return point


def rational_update(previous, point, spec: Rational):
    """_backends/torch/updates/rational_radius.py:10-29 (a clamp, q in [0,1])."""
    displacement = (point - previous).astype(F32)
    proposal = (previous + displacement).astype(F32)
    cap = np.float32(spec.amplitude_max)
    if float(cap) > spec.amplitude_max:
        cap = np.nextafter(cap, np.float32(0))
    out = proposal.copy()
    out[:, 0] = np.clip(proposal[:, 0], -cap, cap)
    out[:, 1] = np.clip(proposal[:, 1], F32(0), F32(1))
    return out


def torus_remainder32(x, period):
    """torch.remainder for float32 (Python-style modulus)."""
    x = x.astype(F32)
    b = F32(period)
    mod = np.fmod(x, b).astype(F32)
    fix = (mod != 0) & ((mod < 0) != (b < 0))
    return np.where(fix, (mod + b).astype(F32), mod).astype(F32)


def polar_update(previous, point, spec: Polar, *, step_size, periods):
    """Polar activity law + flat-torus retraction in float32.

    _backends/torch/algorithms/polar_update/executor.py:42-112 and 168-176,
    _backends/torch/geometry/flat_torus.py:30-35.
    """
    prev = previous.astype(F32)
    disp = (point.astype(F32) - prev).astype(F32)
    one = F32(1)
    pair = prev[:, :2]
    rs = (pair[:, :1] * pair[:, :1] + pair[:, 1:] * pair[:, 1:]).astype(F32)
    tiny = F32(TINY32)
    safe_r = np.sqrt(np.maximum(rs, tiny)).astype(F32)
    fallback = np.zeros_like(pair)
    fallback[:, 1] = 1
    unit = np.where(rs > tiny, (pair / safe_r).astype(F32), fallback)
    polar = (unit * np.clip(safe_r, F32(1), F32(2))).astype(F32)
    raw = disp[:, :2]
    radius_square = (polar[:, :1] * polar[:, :1] + polar[:, 1:] * polar[:, 1:]).astype(F32)
    dot = (raw[:, :1] * polar[:, :1]).astype(F32) + (raw[:, 1:] * polar[:, 1:]).astype(F32)
    radial_coefficient = (dot.astype(F32) / radius_square).astype(F32)
    tangent = (raw - (radial_coefficient * polar).astype(F32)).astype(F32)
    chord = (polar + tangent).astype(F32)
    chord_q = (chord[:, :1] * chord[:, :1] + chord[:, 1:] * chord[:, 1:]).astype(F32)
    direction = (chord / np.sqrt(chord_q)).astype(F32)
    energy = (tangent[:, :1] * tangent[:, :1] + tangent[:, 1:] * tangent[:, 1:]).astype(F32)
    if spec.activity_mode == "time_energy":
        energy = (energy / F32(step_size)).astype(F32)
    drs = (direction[:, :1] * direction[:, :1] + direction[:, 1:] * direction[:, 1:]).astype(F32)
    dsafe = np.maximum(drs, tiny)
    proposed_amp = ((F32(spec.amplitude_max) * direction[:, :1]).astype(F32)
                    / np.sqrt(dsafe).astype(F32)).astype(F32)
    dormant_weight = (one / (one + np.square((proposed_amp / F32(spec.w_c)).astype(F32)))).astype(F32)
    c3 = (F32(3.0) * F32(spec.dormant_expansion_rate)).astype(F32)
    c3 = (c3 * F32(step_size)).astype(F32)
    dormant_q = (c3 * dormant_weight).astype(F32)
    task_q = (radius_square + (F32(spec.activity_gain) * energy).astype(F32)).astype(F32)
    task_q = np.clip((task_q + dormant_q).astype(F32), F32(1), F32(4))
    task_polar = (direction * np.sqrt(task_q)).astype(F32)
    decay_arg = (F32(-4.0) * F32(spec.radial_regularization)).astype(F32)
    decay_arg = (decay_arg * F32(step_size)).astype(F32)
    decay = np.exp(decay_arg).astype(F32)
    activity = ((task_q - one).astype(F32) / task_q).astype(F32)
    regularized_q = (one / (one - (activity * decay).astype(F32)).astype(F32)).astype(F32)
    ratio = np.sqrt((regularized_q / task_q).astype(F32)).astype(F32)
    regularized_polar = (task_polar * ratio).astype(F32)
    out = np.empty_like(prev)
    out[:, :2] = regularized_polar
    out[:, 2] = torus_remainder32((prev[:, 2] + disp[:, 2]).astype(F32), periods[0])
    out[:, 3] = torus_remainder32((prev[:, 3] + disp[:, 3]).astype(F32), periods[1])
    return out


def decay_amplitude(previous, updated, amount):
    """Decoupled Polar amplitude decay in float32 at the accepted radius
    (_backends/torch/algorithms/polar_update/executor.py:18-41): the normalized
    first coordinate loses ``amount`` times its old value, t keeps its sign."""
    if amount == 0:
        return updated
    prev = previous.astype(F32)
    out = updated.astype(F32).copy()
    tiny = F32(TINY32)
    one = F32(1)
    old_r = np.sqrt(np.maximum((prev[:, 0] * prev[:, 0] + prev[:, 1] * prev[:, 1]).astype(F32),
                               tiny)).astype(F32)
    new_r = np.sqrt(np.maximum((out[:, 0] * out[:, 0] + out[:, 1] * out[:, 1]).astype(F32),
                               tiny)).astype(F32)
    old_amp = (prev[:, 0] / old_r).astype(F32)
    target = ((out[:, 0] / new_r).astype(F32) - (F32(amount) * old_amp).astype(F32)).astype(F32)
    target = np.clip(target, F32(-1), one)
    absolute = np.abs(target)
    room = np.maximum(((one - absolute).astype(F32) * (one + absolute).astype(F32)).astype(F32),
                      F32(0))
    magnitude = (new_r * np.sqrt(room).astype(F32)).astype(F32)
    s = (new_r * target).astype(F32)
    out[:, 1] = np.copysign(magnitude, out[:, 1]).astype(F32)
    out[:, 0] = s
    return out


def optimizer_step(p, grad, state: AdamState, spec, *, lr, field_ratios=(),
                   betas=(0.9, 0.999), eps=1e-8, periods=None, amplitude_weight_decay=0.0):
    """One CSTAdamW step on an atom table (optim/adamw.py:230-247): AdamW, the
    field rates, the coordinate law and, for Polar rows, the amplitude decay
    (_backends/torch/algorithms/atom_update/algorithm.py:58-83)."""
    previous = p.astype(F32).copy()
    point = adamw32(p, grad, state, lr=lr, beta1=betas[0], beta2=betas[1], eps=eps)
    if field_ratios:
        point = apply_field_lrs(point, previous, field_ratios)
    if isinstance(spec, Rational):
        if amplitude_weight_decay:
            raise ValueError("amplitude decay requires Polar atoms")
        return rational_update(previous, point, spec)
    out = polar_update(previous, point, spec, step_size=lr, periods=periods)
    return decay_amplitude(previous, out, lr * amplitude_weight_decay)


def field_ratios(spec, field_lrs, lr):
    """(start, stop, ratio) blocks (optim/_field_lrs.py:115-125,
    kernels/parameterizations/base.py:24-47)."""
    if not field_lrs:
        return ()
    names = ((("amplitude", 0, 1), ("radius_fraction", 1, 2)) if isinstance(spec, Rational)
             else (("amplitude", 0, 2),))
    layout = names + (("output_center", 2, 3), ("input_center", 3, 4))
    return tuple((s, e, field_lrs[n] / lr) for n, s, e in layout
                 if n in field_lrs and field_lrs[n] != lr)


# ---------------------------------------------------------------------------
# Whole step (reference algorithm) -- what the CPU baseline times
# ---------------------------------------------------------------------------


def reference_step(out_axis, in_axis, spec, p, x, target, state: AdamState, *, lr,
                   field_lrs=None):
    """MSE forward, factored backward, one CSTAdamW step; returns (loss, y, dx, grad, p')."""
    lay = decode(out_axis, in_axis, spec, p)
    y, saved = factored_forward32(lay, x)
    diff = (y - np.asarray(target, F32)).astype(F32)
    loss = float(np.mean(np.square(diff, dtype=F32), dtype=F32))
    dy = (diff * F32(2.0 / diff.size)).astype(F32)
    dx, grad = factored_backward32(lay, x, dy, saved)
    ratios = field_ratios(spec, field_lrs, lr)
    new_p = optimizer_step(p, grad, state, spec, lr=lr, field_ratios=ratios,
                           periods=(out_axis.period, in_axis.period))
    return loss, y, dx, grad, new_p
