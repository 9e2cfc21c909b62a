"""The plugin's Algorithm bodies on the GPU, and the amplitude decay.

The reference package is not installed on the GPU box, so these run the Linear
and atom_update Algorithms' execute bodies (``plugin.execute_linear``,
``plugin.update_atoms_``) with stand-in declarations of the same attribute
structure (tests/reference_decls.py; tests/test_plugin_cpu.py pins them to the
reference's own declarations). Tolerances: Y, dX and gradients within 1e-4 of
the output scale against the reference's float32 goldens and the float64
oracle; coordinate laws and optimizer steps bit-exact against the oracle.
"""

import numpy as np
import pytest
import torch

from oracle import cst_oracle as O
from tests import reference_decls as D
from tests.golden_cases import CASES, load

pytestmark = pytest.mark.gpu

TOL = 1e-4


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-300))


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda", 0)


class Site(torch.nn.Module):
    def __init__(self, p):
        super().__init__()
        self.p = torch.nn.Parameter(torch.as_tensor(p).cuda())


DECLS = {
    "config1": ((D.chart(8), D.chart(16)), D.rational_kernel(4.0)),
    "config2": ((D.chart(1024), D.chart(1024)), D.rational_kernel(512.0)),
    "config3": ((D.chart(1024), D.chart(784)), D.polar_kernel()),
}


@pytest.mark.parametrize("name", ["config1", "config2", "config3"])
def test_linear_algorithm_execute_matches_goldens(cuda, name):
    from torchcst_b200 import plugin
    d = load(name)
    charts, kernel = DECLS[name]
    site = Site(d["p0"])
    x = torch.as_tensor(d["x"]).cuda().requires_grad_("dx" in d)
    y = plugin.execute_linear(site, x, site.p, charts, kernel, D.recipe())
    y.backward(torch.as_tensor(d["dy"]).cuda())
    torch.cuda.synchronize()
    out_axis, in_axis, spec = CASES[name]
    lay = O.decode(out_axis, in_axis, spec, d["p0"])
    W = O.weight64(lay)
    x64, dy64 = d["x"].astype(np.float64), d["dy"].astype(np.float64)
    assert rel(y.detach().cpu(), d["y"]) < TOL
    assert rel(y.detach().cpu(), x64 @ W.T) < TOL
    if "dx" in d:
        assert rel(x.grad.cpu(), d["dx"]) < TOL
    rows = d.get("rows", slice(None))
    grad = site.p.grad.cpu().numpy()
    g64 = O.atom_gradients64(lay, dy64.T @ x64)
    for c in range(4):
        assert rel(grad[rows, c], d["grad"][:, c]) < TOL, c
        assert rel(grad[:, c], g64[:, c]) < TOL, c


@pytest.mark.parametrize("name,decay", [("config1", 0.0), ("config2", 0.0), ("config3", 0.0),
                                        ("config3", 0.25)])
def test_update_algorithm_execute_bit_exact(cuda, name, decay):
    """The coordinate law alone (what a torchcst CSTAdamW dispatches after its
    own AdamW and field rates) equals the oracle's law bit for bit."""
    from torchcst_b200 import plugin
    d = load(name)
    charts, kernel = DECLS[name]
    out_axis, in_axis, spec = CASES[name]
    rows = d.get("rows", slice(None))
    previous = d["p0"][rows].astype(np.float32)
    g = np.random.default_rng(1)
    proposal = (previous + g.standard_normal(previous.shape) * 3e-3).astype(np.float32)
    if isinstance(spec, O.Rational):
        proposal[:5, 1] = [-0.1, 1.2, 0.5, 1.0, 0.0]  # q projected onto [0, 1]
        want = O.rational_update(previous, proposal, spec)
    else:
        lr = 2e-3
        want = O.polar_update(previous, proposal, spec, step_size=lr,
                              periods=(out_axis.period, in_axis.period))
        want = O.decay_amplitude(previous, want, lr * decay)
    lr = 2e-3 if not isinstance(spec, O.Rational) else 1e-3
    prop = torch.as_tensor(proposal).cuda()
    prev = torch.as_tensor(previous).cuda()
    plugin.update_atoms_(prop, prev, charts, kernel, lr, decay)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(prop.cpu().numpy(), want)


def test_cstadamw_amplitude_decay_bit_exact_and_vs_reference(cuda):
    """CSTAdamW(amplitude_weight_decay=...) on Polar atoms: three fused steps
    equal the oracle bit for bit, and the reference's own steps within the
    oracle's pinned bound (tests/test_oracle_golden.py)."""
    from torchcst_b200 import CSTAdamW
    from tests.test_gpu_parity import make_layer
    d = load("config3_decay")
    layer = make_layer("config3", d["p0"])
    lr, decay = float(d["lr"]), float(d["amplitude_weight_decay"])
    opt = CSTAdamW(layer.parameters(), model=layer, lr=lr, amplitude_weight_decay=decay)
    out_axis, in_axis, spec = CASES["config3"]
    p = d["p0"].copy()
    state = O.AdamState(0, np.zeros_like(p), np.zeros_like(p))
    for step in range(3):
        layer.atoms.p.grad = torch.as_tensor(d["grads"][step]).cuda()
        opt.step()
        p = O.optimizer_step(p, d["grads"][step], state, spec, lr=lr,
                             periods=(out_axis.period, in_axis.period),
                             amplitude_weight_decay=decay)
        got = layer.atoms.p.detach().cpu().numpy()
        np.testing.assert_array_equal(got, p)
        ref = d[f"p{step + 1}"]
        ulp = np.spacing(np.abs(ref).astype(np.float32)).astype(np.float64)
        assert (np.abs(got.astype(np.float64) - ref) <= 8 * ulp + 1e-9).all()


def test_amplitude_decay_group_rules(cuda):
    from torchcst_b200 import CSTAdamW
    from tests.test_gpu_parity import make_layer
    d = load("config1")
    layer = make_layer("config1", d["p0"])
    opt = CSTAdamW(layer.parameters(), model=layer, lr=1e-3, amplitude_weight_decay=0.1)
    layer.atoms.p.grad = torch.as_tensor(d["grad"]).cuda()
    with pytest.raises(ValueError, match="Polar"):
        opt.step()
    with pytest.raises(ValueError, match="nonnegative"):
        CSTAdamW(layer.parameters(), model=layer, amplitude_weight_decay=-1.0)
    opt = CSTAdamW(layer.parameters(), model=layer, lr=1e-3, weight_decay=0.01)
    with pytest.raises(ValueError, match="raw weight_decay=0"):
        opt.step()
    layer3 = make_layer("config3", load("config3")["p0"])
    opt = CSTAdamW(layer3.parameters(), model=layer3, lr=0.5, amplitude_weight_decay=4.0)
    layer3.atoms.p.grad = torch.zeros_like(layer3.atoms.p)
    with pytest.raises(ValueError, match=r"lr \* amplitude_weight_decay"):
        opt.step()
