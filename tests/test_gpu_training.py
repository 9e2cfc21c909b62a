"""Training-level parity on the GPU: the He initialisation, multi-step
trajectories against the reference's own, and a reference-saved checkpoint
loaded onto the device and stepped.

* Initialisation: the device variance-matching search reproduces the
  reference's (``match_variance``, _backends/torch/initialization.py:16-139)
  at config 2: the same accepted scale after the same number of trials, the
  same relative energy error to 1e-6, and so the same atoms bit for bit.
* Trajectories: the reference's own CSTAdamW training (fixed X and target,
  recorded by tests/golden/make_golden.py) against the same steps through this
  package's drop-in API. Every step's loss within 1e-5 (relative); the atoms
  within 2e-3 of the reference's (a fifth of the largest per-step move) with
  99.9% of coordinates within 1e-4. Adam normalises each coordinate's step, so a
  coordinate whose gradient is near zero can move by up to a step size on last-
  bit differences; these bounds allow that and nothing systematic.
* Checkpoint: a Safetensors file saved from a reference layer (relaid-out
  atoms) loads onto the device, runs forward to 1e-4 of the reference's Y and
  takes the oracle's optimizer step bit for bit.
"""

import os

import numpy as np
import pytest
import torch

from oracle import cst_oracle as O
from tests.golden_cases import CASES, GOLDEN, field_lrs, load

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda", 0)


def _layer(n_out, n_in, atoms, radius_max, device="cuda"):
    from torchcst_b200 import CSTLinear, ChebyshevSpec, chart_presets, kernels
    grid = lambda n: chart_presets.regular_grid(n, geometry="flat_torus")
    return CSTLinear(charts=(grid(n_out), grid(n_in)), atoms=atoms, device=device,
                     kernel=kernels.product(kernels.cell_mass(ChebyshevSpec(modes=8)),
                                            coordinates=kernels.rational_radius(
                                                radius_max=radius_max)))


def test_he_init_reproduces_the_reference_search(cuda):
    from torchcst_b200.init import kaiming_normal_
    want = load("config2_init")
    torch.manual_seed(0)
    layer = _layer(1024, 1024, 65536, 512.0)
    report = kaiming_normal_(layer, nonlinearity="relu", q=0.0)
    print("init:", report)
    assert report.amplitude_scale == float(want["amplitude_scale"])
    assert report.evaluations == int(want["evaluations"])
    assert abs(report.relative_error - float(want["relative_error"])) < 1e-6
    assert abs(report.expected_energy / float(want["expected_energy"]) - 1) < 1e-6
    np.testing.assert_array_equal(layer.atoms.p.detach().cpu().numpy(), load("config2")["p0"])


TRAJECTORIES = {
    "trajectory1": (8, 16, 12, 4.0),
    "trajectory_mid": (256, 256, 4096, 128.0),
}


@pytest.mark.parametrize("name", sorted(TRAJECTORIES))
def test_training_trajectory_follows_the_reference(cuda, name):
    from torchcst_b200 import CSTAdamW
    n_out, n_in, atoms, radius_max = TRAJECTORIES[name]
    d = load(name)
    layer = _layer(n_out, n_in, torch.as_tensor(d["p0"]), radius_max)
    lr, keep = float(d["lr"]), int(d["keep"])
    fl = field_lrs(d)
    opt = CSTAdamW(layer.parameters(), model=layer, lr=lr, **({"field_lrs": fl} if fl else {}))
    x, t = torch.as_tensor(d["x"]).cuda(), torch.as_tensor(d["target"]).cuda()
    worst = []
    for step, want in enumerate(d["losses"]):
        opt.zero_grad(set_to_none=True)
        loss = (layer(x) - t).square().mean()
        loss.backward()
        opt.step()
        assert abs(float(loss) - want) <= 1e-5 * want, (step, float(loss), want)
        if (step + 1) % keep == 0:
            got = layer.atoms.p.detach().cpu().numpy()
            diff = np.abs(got - d["p_steps"][(step + 1) // keep - 1])
            worst.append((step + 1, float(diff.max()), float(np.quantile(diff, 0.999))))
            assert diff.max() <= 2e-3, worst[-1]
            assert np.quantile(diff, 0.999) <= 1e-4, worst[-1]
    print(name, "worst |dp| per kept step (step, max, 99.9%):", worst)


def test_reference_checkpoint_loads_and_steps_on_device(cuda):
    from torchcst_b200 import CSTAdamW, hub
    d = load("config1")
    model = hub.load_safetensors(os.path.join(GOLDEN, "config1_reference.safetensors"),
                                 model_factory=lambda: _layer(8, 16, 12, 4.0, device="cpu"),
                                 device=cuda)
    p = model.atoms.p.detach().cpu().numpy()
    np.testing.assert_array_equal(p, d["p0"][::-1])  # the saved relayout
    model.train()
    x = torch.as_tensor(d["x"]).cuda()
    y = model(x)
    out_axis, in_axis, spec = CASES["config1"]
    rel = float(np.abs(y.detach().cpu().numpy() - d["y"]).max() / np.abs(d["y"]).max())
    assert rel < 1e-4
    opt = CSTAdamW(model.parameters(), model=model, lr=1e-3)
    loss = (y - torch.as_tensor(d["target"]).cuda()).square().mean()
    loss.backward()
    grad = model.atoms.p.grad.cpu().numpy()
    opt.step()
    state = O.AdamState(0, np.zeros_like(grad), np.zeros_like(grad))
    want = O.optimizer_step(p, grad, state, spec, lr=1e-3)
    np.testing.assert_array_equal(model.atoms.p.detach().cpu().numpy(), want)
    # And the optimizer state round-trips through its state dict on the device.
    sd = opt.state_dict()
    opt2 = CSTAdamW(model.parameters(), model=model, lr=1e-3)
    opt2.load_state_dict(sd)
    st, st2 = opt.state[model.atoms.p], opt2.state[model.atoms.p]
    for key in ("exp_avg", "exp_avg_sq"):
        assert torch.equal(st[key], st2[key])
    assert float(st["step"]) == float(st2["step"]) == 1.0
