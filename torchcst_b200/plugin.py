"""torchcst backend plugin: the sm_100a radius cell-mass Linear as a registered Algorithm.

torchcst selects Linear implementations through its own registry: an
``Algorithm`` (``_backends/algorithm.py:17-93``) registered with
``Registry.register`` (``_backends/registry.py:17-23``) and chosen by an
``ExecutionPlan`` through a selector (``_backends/dispatch/select.py:6-21``).
This module defines that Algorithm for the B200 path, mirroring the reference's
``FactoredAlgorithm`` (``_backends/torch/algorithms/linear/factored/
algorithm.py:17-61``): same ``operation_id`` and ``semantics_id``, metadata-only
``supports``, and an ``execute`` that returns Y connected to autograd, with dX
and ``p.grad`` from the native backward. A reference layer then runs on the
GPU without code changes::

    registry, plan = torchcst_b200.plugin.register(torchcst._backends.catalog.make_registry())
    layer = torchcst.CSTLinear(..., selector=FixedSelector(plan, registry=registry))

torchcst itself is imported only when these functions are called; nothing here
is needed by ``torchcst_b200``'s own ``CSTLinear``.
"""

from __future__ import annotations

import weakref
from dataclasses import dataclass
from functools import lru_cache

import torch

from . import runtime as R
from .spec import (CellMass, ChebyshevSpec, KernelSpec, PolarRadius, RadiusBounds,
                   RationalRadius, RegularGrid, radius_cell_mass_axes)

ALGORITHM_ID = "b200_radius_cell_mass"
REVISION = "v1"


@dataclass(frozen=True)
class B200Recipe:
    """JSON-native settings of the B200 Algorithm (``Registry.dump_plan`` needs a
    dataclass of plain fields). ``validate``: "sync" reads the device status word
    after decoding and raises ``ValueError`` for invalid atoms like the
    reference; "off" leaves it on the device."""

    validate: str = "sync"


def _chart_declaration(chart):
    return chart.declaration() if hasattr(chart, "declaration") else chart


def spec_from_reference(charts, kernel):
    """(axes, KernelSpec) of this package from torchcst declarations.

    ``charts``: the (output, input) ``RegularGridChartSpec`` pair (or chart
    modules); ``kernel``: a ``KernelSpec`` declaration
    (``kernels/radius_cell_mass.py:29-93`` defines what is accepted).
    """
    decls = [_chart_declaration(c) for c in charts]
    grids = []
    for d in decls:
        if getattr(d, "kind", None) != "regular_grid" or len(d.shape) != 1:
            raise ValueError("radius cell masses require fixed one-dimensional torus grids")
        if getattr(d.geometry, "id", None) != "flat_torus":
            raise ValueError("radius cell masses require fixed one-dimensional torus grids")
        grids.append(RegularGrid(int(d.shape[0]), float(d.spacing[0]), float(d.origin[0])))
    profiles = []
    for b in kernel.profiles:
        if getattr(b.profile, "id", None) != "chebyshev":
            raise ValueError("the B200 path evaluates Chebyshev cell masses")
        profiles.append(CellMass(ChebyshevSpec(int(b.profile.modes)), int(b.base_tile_sites),
                                 int(b.merge_factor)))
    par = kernel.parameterization
    pid = getattr(par, "id", None)
    if pid == "rational_radius" and kernel.revision == 8:
        coords = RationalRadius(float(par.radius_min), float(par.radius_birth),
                                float(par.radius_max), float(par.amplitude_max))
    elif pid == "polar_activity_radius" and kernel.revision == 7:
        if getattr(par, "radius_envelope", "rational") != "rational":
            raise ValueError("the B200 path implements the rational Polar radius envelope")

        def bounds(b):
            return RadiusBounds(float(b.minimum), float(b.birth), float(b.maximum),
                                float(b.upper_floor))

        update = dict(getattr(kernel.update, "settings", ()) or ())
        init = dict(getattr(kernel.initialization, "settings", ()) or ())
        coords = PolarRadius(
            float(par.amplitude_max), float(par.w_c), bounds(par.input_bounds),
            bounds(par.output_bounds), float(par.kappa), float(par.lower_kappa),
            float(par.upper_decay_power), float(init.get("alpha_init", 0.0)),
            float(update.get("radial_regularization", 0.1)),
            float(update.get("activity_gain", 1.0)),
            str(update.get("activity_mode", "finite_chord")),
            float(update.get("dormant_expansion_rate", 0.0)))
    else:
        raise ValueError("the B200 path implements rational (revision 8) and Polar "
                         "(revision 7) radius coordinates")
    if kernel.composition != "separable":
        raise ValueError("radius cell masses require a separable product kernel")
    spec = KernelSpec(tuple(profiles), coords)
    return radius_cell_mass_axes(tuple(grids), spec), spec


class NativeBinding:
    """The per-binding state the native autograd Function needs (plan, device
    workspaces, validation mode), kept in the torchcst AlgorithmState."""

    def __init__(self, axes, kernel: KernelSpec, validate: str):
        self.axes, self.kernel = axes, kernel
        self._plan = R.Plan.make(axes, kernel)
        self.validate = validate
        self._workspaces = {}

    def _workspace(self, device):
        key = torch.device(device).index
        ws = self._workspaces.get(key)
        if ws is None:
            ws = self._workspaces[key] = R.Workspace(self._plan, device)
        return ws

    def _maybe_check(self, ws):
        if self.validate == "sync":
            code = int(ws.status.item())
            if code:
                ws.status.zero_()
                raise ValueError(R.status_error(code))


_BINDINGS: "weakref.WeakKeyDictionary" = weakref.WeakKeyDictionary()


@lru_cache(maxsize=1)
def algorithm_class():
    """The Algorithm subclass (created on first use: it derives from torchcst's)."""
    from torchcst._backends.algorithm import Algorithm
    from torchcst._backends.schema import SupportResult
    from torchcst.operators.context import LinearContext
    from torchcst.operators.execution import (LinearInputs, linear_execution,
                                              validate_live_operator)

    @dataclass(frozen=True)
    class B200RadiusCellMassAlgorithm(Algorithm):
        id: str = ALGORITHM_ID
        revision: str = REVISION
        operation_id: str = "linear"
        semantics_id: str = "kernel-atom-sum-v1"
        recipe_type: type = B200Recipe
        input_type: type = LinearInputs

        def validate_recipe(self, recipe):
            if type(recipe) is not B200Recipe:
                raise ValueError("expected a B200Recipe")
            if recipe.validate not in ("sync", "off"):
                raise ValueError("validate must be 'sync' or 'off'")

        def validate_configuration(self, site):
            spec_from_reference(site.cst_charts(), site.kernel.declaration())

        def supports(self, context, recipe):
            if not isinstance(context, LinearContext):
                return SupportResult(("requires a LinearContext",))
            reasons = []
            dev = context.device
            if dev.type != "cuda" or dev.compute_capability != (10, 0):
                reasons.append("requires an sm_100 (B200) CUDA device")
            if context.dtype != torch.float32:
                reasons.append("computes the float32 contract")
            op = context.operator
            if len(op.charts) != 2:
                reasons.append("requires factorized input/output charts")
            else:
                try:
                    spec_from_reference(op.charts, op.kernel)
                except (ValueError, TypeError, AttributeError) as exc:
                    reasons.append(str(exc))
            if context.parameter_dim != 4:
                reasons.append("atom rows must have four coordinates")
            return SupportResult(tuple(reasons))

        def workspace_bound(self, context, recipe):
            return None

        def validate_inputs(self, state, inputs):
            super().validate_inputs(state, inputs)
            validate_live_operator(state, inputs)

        def execute(self, state, inputs):
            from .linear import _CellMassLinear

            x, p, operator, site = linear_execution(state, inputs)
            native = _BINDINGS.get(site)
            key = (operator, state.recipe)
            if native is None or native[0] != key:
                axes, spec = spec_from_reference(operator.charts, operator.kernel)
                native = (key, NativeBinding(axes, spec, state.recipe.validate))
                _BINDINGS[site] = native
            R.require_cuda(x, p)
            flat = x.reshape(-1, x.shape[-1]).contiguous()
            with R.on_device(p.device):
                return _CellMassLinear.apply(flat, p, native[1])

    return B200RadiusCellMassAlgorithm


def algorithm():
    return algorithm_class()()


def plan(recipe: B200Recipe | None = None):
    """The ExecutionPlan that selects this Algorithm."""
    from torchcst._backends.schema import ExecutionPlan
    return ExecutionPlan(ALGORITHM_ID, REVISION, recipe or B200Recipe())


def register(registry=None, recipe: B200Recipe | None = None):
    """Register the Algorithm (into a fresh catalog registry by default) and
    return ``(registry, plan)``."""
    if registry is None:
        from torchcst._backends.catalog import make_registry
        registry = make_registry()
    registry.register(algorithm())
    return registry, plan(recipe)


def selector(registry=None, recipe: B200Recipe | None = None):
    """A torchcst ``FixedSelector`` that picks this Algorithm."""
    from torchcst._backends.dispatch.select import FixedSelector
    registry, p = register(registry, recipe)
    return FixedSelector(p, registry=registry)
