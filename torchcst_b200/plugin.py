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
    opt = torchcst.CSTAdamW(layer.parameters(), model=layer,
                            update_selector=torchcst_b200.plugin.update_selector(registry))

or, for every layer of a model at once (B200 on sm_100, the reference's own
choice elsewhere): ``torchcst_b200.plugin.use_b200(model)``. The atom_update
Algorithm (``_backends/torch/algorithms/atom_update/algorithm.py:13-83``) runs
the coordinate law of a reference ``CSTAdamW`` step in one native kernel.

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
        if self.validate == "sync" and not torch.cuda.is_current_stream_capturing():
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
            x, p, operator, site = linear_execution(state, inputs)
            return execute_linear(site, x, p, operator.charts, operator.kernel, state.recipe)

    return B200RadiusCellMassAlgorithm


def execute_linear(site, x, p, charts, kernel, recipe):
    """The Linear Algorithm's execute without torchcst's dispatch objects: Y of
    a radius cell-mass layer given its live input ``x`` [..., N_in], atoms ``p``
    and its (output, input) chart and kernel declarations (the attribute
    structure of torchcst's declarations). ``site`` keys the cached native
    binding (the layer module). Y is connected to autograd: dX and p.grad come
    from the native backward."""
    from .linear import _CellMassLinear

    native = _BINDINGS.get(site)
    key = (charts, kernel, recipe)
    if native is None or native[0] != key:
        axes, spec = spec_from_reference(charts, kernel)
        native = (key, NativeBinding(axes, spec, recipe.validate))
        _BINDINGS[site] = native
    R.require_cuda(x, p)
    flat = x.reshape(-1, x.shape[-1]).contiguous()
    with R.on_device(p.device):
        return _CellMassLinear.apply(flat, p, native[1])


# -- atom_update ------------------------------------------------------------------

UPDATE_ALGORITHM_ID = "b200_atom_update"
UPDATE_REVISION = "v1"


def update_atoms_(proposal, previous, charts, kernel, step_size, amplitude_weight_decay=0.0):
    """The update Algorithm's execute without torchcst's dispatch objects: the
    declared coordinate law (rational projection, or the Polar activity law
    with torus retraction and amplitude decay) applied in place to ``proposal``
    from ``previous`` by one native kernel, as the torch atom_update Algorithm
    does with several torch ops (_backends/torch/algorithms/atom_update/
    algorithm.py:58-83). Returns ``proposal``."""
    from .optim import coordinate_update_

    axes, spec = spec_from_reference(charts, kernel)
    coordinate_update_(proposal, previous, spec.coordinates, axes, step_size,
                       amplitude_weight_decay)
    return proposal


def _is_sm100(device_info):
    cc = getattr(device_info, "compute_capability", None)
    if cc is None and device_info.type == "cuda" and torch.cuda.is_available():
        cc = torch.cuda.get_device_capability(device_info.index or 0)
    return device_info.type == "cuda" and tuple(cc or ()) == (10, 0)


@lru_cache(maxsize=1)
def update_algorithm_class():
    """The atom_update Algorithm (created on first use: it derives from torchcst's)."""
    from torchcst._backends.algorithm import Algorithm
    from torchcst._backends.schema import DefaultRecipe, SupportResult
    from torchcst.operators.atom_update import (AtomUpdateContext, AtomUpdateInputs,
                                                amplitude_decay_amount)

    @dataclass(frozen=True)
    class B200AtomUpdateAlgorithm(Algorithm):
        id: str = UPDATE_ALGORITHM_ID
        revision: str = UPDATE_REVISION
        operation_id: str = "atom_update"
        semantics_id: str = "kernel-coordinate-update-v2"
        recipe_type: type = DefaultRecipe
        input_type: type = AtomUpdateInputs

        def validate_recipe(self, recipe):
            if type(recipe) is not DefaultRecipe:
                raise ValueError("the B200 atom update has no tunable recipe")

        def supports(self, context, recipe):
            if not isinstance(context, AtomUpdateContext):
                return SupportResult(("requires AtomUpdateContext",))
            reasons = []
            if not _is_sm100(context.device):
                reasons.append("requires an sm_100 (B200) CUDA device")
            if context.dtype != torch.float32 or not context.contiguous:
                reasons.append("requires contiguous float32 atoms")
            if len(context.parameter_shape) != 2 or context.parameter_shape[1] != 4:
                reasons.append("atom rows must have four coordinates")
            if context.execution_mode != "eager":
                reasons.append("runs in eager mode")
            kernel = context.kernel
            par = getattr(kernel, "parameterization", None)
            pid = getattr(par, "id", None)
            if not ((pid == "rational_radius" and kernel.revision == 8)
                    or (pid == "polar_activity_radius" and kernel.revision == 7)):
                reasons.append("implements rational (revision 8) and Polar (revision 7) "
                               "radius coordinates")
            elif context.amplitude_decay and pid != "polar_activity_radius":
                reasons.append("amplitude decay requires Polar atoms")
            if getattr(kernel, "composition", None) != "separable" or len(
                    context.geometries) != 2 or any(
                    type(g).__name__ != "FlatTorusGeometrySpec" for g in context.geometries):
                reasons.append("requires two one-dimensional FlatTorus charts")
            return SupportResult(tuple(reasons))

        def workspace_bound(self, context, recipe):
            return 0

        @torch.no_grad()
        def execute(self, state, inputs):
            decay = amplitude_decay_amount(state.context, inputs)
            binding = state.binding
            decl = binding.execution_declaration()
            proposal = binding.execution_parameters()
            update_atoms_(proposal, inputs.previous, decl.charts, decl.kernel,
                          inputs.step_size, inputs.amplitude_weight_decay if decay else 0.0)
            return proposal.detach()

        def prepare_optimizer_program(self, dispatcher, cached, adapter, site=None):
            return OptimizerProgram(dispatcher, cached)

    return B200AtomUpdateAlgorithm


class OptimizerProgram:
    """The certified fast path a torchcst CSTAdamW takes for this update
    (optim/_coordinate_step.py:75-104,143-168): after the first dispatched step
    the optimizer asks the selected Algorithm for a program, and later steps call
    ``preflight`` (before AdamW) and ``run`` (after AdamW and the field rates)
    instead of dispatching again. The laws here leave the optimizer state where
    it is (the flat-torus and rational transports are the identity), so
    ``transport_required`` stays False."""

    transport_required = False

    def __init__(self, dispatcher, cached):
        self.dispatcher = dispatcher
        self.state = cached.state
        self.plan = cached.decision.plan
        self.context = cached.context
        self.binding = cached.state.binding
        self.point = self.binding.execution_parameters()

    def preflight(self, dispatcher, adapter, point, gradient, decay):
        if dispatcher is not self.dispatcher or point is not self.point:
            return False
        if type(gradient) is not torch.Tensor or gradient.layout != torch.strided or (
                gradient.shape != point.shape or gradient.dtype != point.dtype
                or gradient.device != point.device):
            return False
        keys = getattr(adapter, "vector_keys", None)
        if type(keys) is not tuple or not set(keys) <= {"exp_avg"}:
            return False
        if (decay != 0) != self.context.amplitude_decay:
            return False
        return not torch.cuda.is_current_stream_capturing()

    def validate_inputs(self, inputs):
        self.binding.validate_inputs(inputs)
        return True

    def run(self, dispatcher, adapter, inputs, state):
        """Apply the law to the bound atoms; None asks for ordinary dispatch."""
        if dispatcher is not self.dispatcher or self.binding.execution_parameters() is not (
                self.point):
            return None
        return self.state.algorithm.execute(self.state, inputs)

    def transport_is_identity(self, dispatcher, adapter, point, inputs, state):
        return True


def update_algorithm():
    return update_algorithm_class()()


def update_plan():
    """The ExecutionPlan that selects the B200 atom update."""
    from torchcst._backends.schema import DefaultRecipe, ExecutionPlan
    return ExecutionPlan(UPDATE_ALGORITHM_ID, UPDATE_REVISION, DefaultRecipe())


def update_selector(registry=None):
    """A torchcst ``FixedSelector`` for ``CSTAdamW(..., update_selector=...)``."""
    from torchcst._backends.dispatch.select import FixedSelector
    registry = install(registry)
    return FixedSelector(update_plan(), registry=registry)


# -- registration and selection -------------------------------------------------------


def install(registry=None):
    """Register both Algorithms (Linear and atom_update) into ``registry`` (the
    global torchcst registry by default) unless already there; returns it."""
    if registry is None:
        from torchcst._backends.catalog import get_registry
        registry = get_registry()
    for make, key in ((algorithm, (ALGORITHM_ID, REVISION)),
                      (update_algorithm, (UPDATE_ALGORITHM_ID, UPDATE_REVISION))):
        try:
            registry.get(key[0], revision=key[1])
        except ValueError:
            registry.register(make())
    return registry


@lru_cache(maxsize=1)
def _first_selector_class():
    from torchcst._backends.dispatch.base import Match, Selector

    class B200FirstSelector(Selector):
        """``backend="auto"`` with the B200 plan first: the plan is proposed
        whenever its Algorithm supports the context (an sm_100 CUDA device and
        a supported declaration); otherwise the reference's own default
        selector decides (nn/linear.py:45-57)."""

        def __init__(self, plan, fallback, *, registry):
            super().__init__(revision="b200-first-v1", registry=registry)
            if fallback.registry is not registry:
                raise ValueError("the fallback selector must use the same Registry")
            registry.validate_plan(plan)
            self._plan, self._fallback = plan, fallback

        def _match(self, context):
            algorithm = self.registry.validate_plan(self._plan)
            if algorithm.matches(context, self._plan.recipe):
                return Match(self._plan, ("b200", self._plan.algorithm_id),
                             "sm_100 device with a supported radius cell-mass declaration")
            return self._fallback._match(context)

    return B200FirstSelector


def auto_selector(recipe: B200Recipe | None = None):
    """The reference's automatic Linear selection with the B200 plan preferred
    on sm_100: registers the Algorithms into torchcst's global registry (once)
    and wraps the reference's default selector."""
    from torchcst.nn.linear import _default_selector
    fallback = _default_selector()
    registry = install(fallback.registry)
    return _first_selector_class()(plan(recipe), fallback, registry=registry)


def use_b200(model, recipe: B200Recipe | None = None):
    """One call for a whole model: every torchcst ``CSTLinear`` in ``model``
    gets :func:`auto_selector` (B200 on sm_100, the reference's choice
    elsewhere). Returns the number of layers routed."""
    from torchcst.nn.linear import CSTLinear as ReferenceLinear
    selector = auto_selector(recipe)
    count = 0
    for module in model.modules():
        if isinstance(module, ReferenceLinear):
            module.selector = selector
            count += 1
    return count


def algorithm():
    return algorithm_class()()


def plan(recipe: B200Recipe | None = None):
    """The ExecutionPlan that selects this Algorithm."""
    from torchcst._backends.schema import ExecutionPlan
    return ExecutionPlan(ALGORITHM_ID, REVISION, recipe or B200Recipe())


def register(registry=None, recipe: B200Recipe | None = None):
    """Register the Linear and atom_update Algorithms (into a fresh catalog
    registry by default) and return ``(registry, plan)``."""
    if registry is None:
        from torchcst._backends.catalog import make_registry
        registry = make_registry()
    registry.register(algorithm())
    registry.register(update_algorithm())
    return registry, plan(recipe)


def selector(registry=None, recipe: B200Recipe | None = None):
    """A torchcst ``FixedSelector`` that picks this Algorithm."""
    from torchcst._backends.dispatch.select import FixedSelector
    registry, p = register(registry, recipe)
    return FixedSelector(p, registry=registry)
