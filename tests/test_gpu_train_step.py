"""The fused MSE train step: eager launches, CUDA-graph replays and the drop-in
autograd API take the same step.

Eager and replayed steps run the same kernels on the same buffers, so atoms and
optimizer moments must agree bit for bit. The autograd path forms dY with torch
ops instead of the fused loss kernel, so it agrees to float32 rounding.
"""

import numpy as np
import pytest
import torch

from tests.golden_cases import load

pytestmark = pytest.mark.gpu


def _setup(seed=0):
    from torchcst_b200 import CSTAdamW, CSTLinear, ChebyshevSpec, chart_presets, kernels
    d = load("config5s")
    grid = chart_presets.regular_grid(512, geometry="flat_torus")
    layer = CSTLinear(charts=(grid, grid), atoms=torch.as_tensor(d["p0"]), device="cuda",
                      validate="off",
                      kernel=kernels.product(kernels.cell_mass(ChebyshevSpec(modes=8)),
                                             coordinates=kernels.rational_radius(radius_max=256.0)))
    opt = CSTAdamW(layer.parameters(), model=layer, lr=1e-3,
                   field_lrs={"amplitude": 2.4e-3, "radius_fraction": 9.6e-3})
    g = torch.Generator(device="cuda").manual_seed(seed)
    xs = [torch.randn(256, 512, device="cuda", generator=g) for _ in range(2)]
    ts = [torch.randn(256, 512, device="cuda", generator=g) for _ in range(2)]
    return layer, opt, xs, ts


def _state(layer, opt):
    p = layer.atoms.p
    st = opt.state[p]
    return [p.detach().clone(), st["exp_avg"].clone(), st["exp_avg_sq"].clone()]


def test_graph_replay_matches_eager_steps():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from torchcst_b200.train import MSETrainStep
    runs = []
    for graphs in (False, True):
        layer, opt, xs, ts = _setup()
        step = MSETrainStep(layer, opt, 256)
        losses = [float(step(xs[0], ts[0]))]
        if graphs:
            step.capture(list(zip(xs, ts)))
        for i in range(1, 5):
            losses.append(float(step(xs[i % 2], ts[i % 2])))
        torch.cuda.synchronize()
        assert step.check_status() == 0
        runs.append((losses, _state(layer, opt), int(opt.state[layer.atoms.p]["step"])))
        step.release()
    (l0, s0, n0), (l1, s1, n1) = runs
    assert n0 == n1 == 5
    assert l0 == l1
    for a, b in zip(s0, s1):
        assert torch.equal(a, b)


def test_fused_step_matches_autograd_api():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from torchcst_b200.train import MSETrainStep
    layer, opt, xs, ts = _setup()
    step = MSETrainStep(layer, opt, 256)
    fused_loss = float(step(xs[0], ts[0]))
    assert step.check_status() == 0
    fused = _state(layer, opt)

    layer2, opt2, _, _ = _setup()
    y = layer2(xs[0])
    loss = (y - ts[0]).square().mean()
    loss.backward()
    opt2.step()
    api = _state(layer2, opt2)
    api_loss = float(loss.detach())
    assert abs(fused_loss - api_loss) <= 1e-6 * abs(api_loss)
    # Same update up to float32 rounding of dY (torch ops vs the fused loss kernel).
    for a, b in zip(fused, api):
        a, b = a.cpu().numpy().astype(np.float64), b.cpu().numpy().astype(np.float64)
        assert np.abs(a - b).max() <= 1e-4 * max(np.abs(b).max(), 1e-30)


def _graphed_vs_eager(build, steps=7):
    """Run the same drop-in step function eagerly and through GraphedStep
    (3 eager warm-up calls, then captured replays over two buffer sets)."""
    from torchcst_b200.train import GraphedStep
    runs = []
    for graphed in (False, True):
        model, opt, step_fn, xs, ts = build()
        call = GraphedStep(step_fn, opt) if graphed else step_fn
        losses = [float(call(xs[i % 2], ts[i % 2])) for i in range(steps)]
        torch.cuda.synchronize()
        state = [t.detach().clone() for t in model.parameters()]
        for p in model.parameters():
            st = opt.state[p]
            state += [st["exp_avg"].clone(), st["exp_avg_sq"].clone()]
        runs.append((losses, state))
        if graphed:
            call.release()
    (l0, s0), (l1, s1) = runs
    assert l0 == l1
    for a, b in zip(s0, s1):
        assert torch.equal(a, b)


def test_graphed_autograd_step_matches_eager_mse():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")

    def build():
        layer, opt, xs, ts = _setup()

        def step(x, t):
            opt.zero_grad(set_to_none=True)
            loss = (layer(x) - t).square().mean()
            loss.backward()
            opt.step()
            return loss

        return layer, opt, step, xs, ts

    _graphed_vs_eager(build)


def test_graphed_autograd_step_matches_eager_classifier():
    """The config-3 shape of model (Polar CSTLinear, ReLU, dense head,
    cross-entropy) with a capturable group for the dense parameters."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from tests.test_gpu_parity import make_layer
    import torch.nn.functional as F
    from torchcst_b200 import CSTAdamW

    def build():
        d = load("config3")
        torch.manual_seed(0)
        layer = make_layer("config3", d["p0"])
        layer.validate = "off"
        head = torch.nn.Linear(1024, 10).cuda()
        model = torch.nn.Sequential(layer, torch.nn.ReLU(), head)
        opt = CSTAdamW(model.parameters(), model=model, lr=1e-3, capturable=True)
        g = torch.Generator(device="cuda").manual_seed(3)
        xs = [torch.rand(64, 784, device="cuda", generator=g) for _ in range(2)]
        ts = [torch.randint(0, 10, (64,), device="cuda", generator=g) for _ in range(2)]

        def step(x, t):
            opt.zero_grad(set_to_none=True)
            loss = F.cross_entropy(model(x), t)
            loss.backward()
            opt.step()
            return loss

        return model, opt, step, xs, ts

    _graphed_vs_eager(build)



def test_scalar_ring_matches_host_scalars_and_flags_stale_slots():
    """tcst_scalar_ring_fetch + tcst_optimizer_step_ring take each launch's
    scalars from its ring slot: three launches equal three host-scalar steps bit
    for bit, and a slot whose sequence number is not the fetch's raises
    TCST_STATUS_SEQUENCE and leaves the atoms and moments unchanged (the use
    count still advances)."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import ctypes
    from torchcst_b200 import _native as N
    from torchcst_b200 import runtime as R
    layer, opt, _, _ = _setup()
    p = layer.atoms.p
    g = torch.Generator(device="cuda").manual_seed(3)
    grads = [torch.randn(p.shape, device="cuda", generator=g) * 1e-3 for _ in range(3)]
    kind = N.TCST_RATIONAL
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = R._stream(p.device)
    host = [p.detach().clone(), torch.zeros_like(p), torch.zeros_like(p)]
    dev = [t.clone() for t in host]
    ring = R.ScalarRing(p.device)
    for step, grad in enumerate(grads, start=1):
        h = opt._native_params(layer, opt.param_groups[0], step)
        N.call("tcst_optimizer_step", R._vp(host[0]), R._vp(grad), R._vp(host[1]),
               R._vp(host[2]), p.shape[0], kind, ctypes.byref(h), stream)
        ring.write(h)
        ring.fetch(status, stream)
        ring.launch(dev[0], grad, dev[1], dev[2], kind, stream)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert int(ring.state[0].item()) == 3
    for a, b in zip(host, dev):
        assert torch.equal(a, b)
    # A slot written for another launch: flagged, nothing updated.
    h = opt._native_params(layer, opt.param_groups[0], 4)
    ring.write(h)
    slot = ring.host[(ring.uses - 1) % ring.SLOTS]
    ctypes.c_uint32.from_address(slot.data_ptr() + ring.seq_offset).value = 12345
    before = [t.clone() for t in dev]
    ring.fetch(status, stream)
    ring.launch(dev[0], grads[0], dev[1], dev[2], kind, stream)
    torch.cuda.synchronize()
    assert int(status.item()) == N.STATUS_SEQUENCE
    assert int(ring.state[0].item()) == 4
    for a, b in zip(before, dev):
        assert torch.equal(a, b)
