"""The weight-assembly entry point that allocates nothing.

Callers that cannot hand the library device memory (for example a plugin whose
host framework owns every device allocation) use tcst_assemble_weight_static,
whose scratch is an array built into the library. This test calls it
through the C ABI twice in a row and checks each result against
tcst_assemble_weight run with caller-provided scratch. Both run the same
kernels in the same fixed order, so the outputs must agree bit for bit
(tighter than the 1e-4 tolerance the other parity tests use). The cases cover
every footprint class, including the mid-size classes whose masses live in the
scratch. It must pass in a fresh process and after the rest of the suite,
which is why it sits in the last test file.
"""

import ctypes

import numpy as np
import pytest
import torch

from tests.golden_cases import load

pytestmark = pytest.mark.gpu


def _layer(p0, n_out, n_in, radius_max):
    from torchcst_b200 import CSTLinear, ChebyshevSpec, chart_presets, kernels
    return CSTLinear(
        charts=(chart_presets.regular_grid(n_out, geometry="flat_torus"),
                chart_presets.regular_grid(n_in, geometry="flat_torus")),
        atoms=torch.as_tensor(p0), device="cuda",
        kernel=kernels.product(kernels.cell_mass(ChebyshevSpec(modes=8)),
                               coordinates=kernels.rational_radius(radius_max=radius_max)))


def _planes(plan, dev):
    ld = (plan.n_in + 3) & ~3
    w = torch.full((plan.n_out, plan.n_in), float("nan"), device=dev)
    hi = torch.full((plan.n_out, ld), float("nan"), device=dev)
    lo = torch.full((plan.n_out, ld), float("nan"), device=dev)
    return w, hi, lo, ld


@pytest.mark.parametrize("case,n_out,n_in,radius_max", [("config5s", 512, 512, 256.0),
                                                        ("config4s", 1024, 256, 128.0),
                                                        ("config1", 8, 16, 4.0)])
def test_static_weight_matches_caller_scratch(case, n_out, n_in, radius_max):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from torchcst_b200 import _native as N
    from torchcst_b200 import runtime as R
    lib = N.load()
    d = load(case)
    layer = _layer(d["p0"], n_out, n_in, radius_max)
    p = layer.atoms.p.detach()
    plan = layer._plan
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    table = R.decode_route(plan, p, status)
    stream = R._stream(p.device)
    oa, ia = ctypes.byref(plan.out_axis), ctypes.byref(plan.in_axis)

    need = lib.tcst_weight_scratch_bytes(p.shape[0], oa, ia)
    scratch = torch.zeros((need + 3) // 4, dtype=torch.int32, device="cuda")
    w_ref, hi_ref, lo_ref, ld = _planes(plan, p.device)
    N.check(lib.tcst_assemble_weight(R._vp(table), p.shape[0], oa, ia, R._vp(scratch), need,
                                     R._vp(w_ref), plan.n_in, R._vp(hi_ref), R._vp(lo_ref), ld,
                                     stream), "tcst_assemble_weight")
    for _ in range(2):
        w, hi, lo, ld = _planes(plan, p.device)
        N.check(lib.tcst_assemble_weight_static(R._vp(table), p.shape[0], oa, ia, R._vp(w),
                                                plan.n_in, R._vp(hi), R._vp(lo), ld, stream),
                "tcst_assemble_weight_static")
        torch.cuda.synchronize()
        assert torch.equal(w, w_ref)
        assert torch.equal(hi[:, :plan.n_in], hi_ref[:, :plan.n_in])
        assert torch.equal(lo[:, :plan.n_in], lo_ref[:, :plan.n_in])
    assert int(status.item()) == 0
    assert np.isfinite(w.cpu().numpy()).all()


def test_static_weight_rejects_oversized_layers():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from torchcst_b200 import _native as N
    lib = N.load()
    limit = lib.tcst_static_weight_scratch_bytes()
    assert limit == 32 << 20
    axis = N.Axis(1024, 1, 2, 8, 1.0, 0.0)
    fits, too_many = 32768, 65536
    assert lib.tcst_weight_scratch_bytes(fits, ctypes.byref(axis), ctypes.byref(axis)) <= limit
    assert lib.tcst_weight_scratch_bytes(too_many, ctypes.byref(axis), ctypes.byref(axis)) > limit
    rc = lib.tcst_assemble_weight_static(None, too_many, ctypes.byref(axis), ctypes.byref(axis),
                                         None, 0, None, None, 0, None)
    assert rc == 3
    assert b"more than the built-in" in lib.tcst_last_error()
