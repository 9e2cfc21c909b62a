"""Safetensors loading (torchcst_b200.hub) on CPU.

Own files round-trip with the reference's key, shape and dtype rules; files
saved from reference layers (the reference source tree, when present) load
into the B200 layers that declare the same kernel, and a differing declaration
is refused.
"""

import pytest
import torch
from torch import nn

from safetensors.torch import save_file

from torchcst_b200 import CSTLinear, ChebyshevSpec, RadiusBounds, chart_presets, kernels
from torchcst_b200 import hub

from test_plugin_cpu import _reference_layer, tc  # noqa: F401 (fixture)


def _grid(n):
    return chart_presets.regular_grid(n, geometry="flat_torus")


def _rational_layer(n_out=8, n_in=16, atoms=12, seed=0, radius_max=4.0, **kw):
    torch.manual_seed(seed)
    return CSTLinear(charts=(_grid(n_out), _grid(n_in)), atoms=atoms,
                     kernel=kernels.product(kernels.cell_mass(ChebyshevSpec(modes=8)),
                                            coordinates=kernels.rational_radius(
                                                radius_max=radius_max, **kw)))


def _save(path, module):
    save_file({k: v.detach().contiguous() for k, v in module.state_dict().items()
               if torch.is_tensor(v)}, str(path))


def test_own_file_round_trips(tmp_path):
    src = _rational_layer(seed=1)
    _save(tmp_path / "m.safetensors", src)
    out = hub.load_safetensors(tmp_path / "m.safetensors",
                               model_factory=lambda: _rational_layer(seed=2))
    assert torch.equal(out.atoms.p.detach(), src.atoms.p.detach())
    assert not out.training


def test_key_shape_and_dtype_errors(tmp_path):
    layer = _rational_layer()
    p = layer.atoms.p.detach()
    save_file({"atom_state.atoms.p": p, "extra": torch.zeros(1)}, str(tmp_path / "a.safetensors"))
    with pytest.raises(ValueError, match="keys do not match the model.*Unexpected: \\['extra'\\]"):
        hub.load_safetensors(tmp_path / "a.safetensors", model_factory=_rational_layer)
    save_file({"atom_state.atoms.p": p[:6].contiguous()}, str(tmp_path / "b.safetensors"))
    with pytest.raises(ValueError, match="has shape \\(6, 4\\)"):
        hub.load_safetensors(tmp_path / "b.safetensors", model_factory=_rational_layer)
    save_file({"atom_state.atoms.p": p.double()}, str(tmp_path / "c.safetensors"))
    with pytest.raises(ValueError, match="dtype torch.float64"):
        hub.load_safetensors(tmp_path / "c.safetensors", model_factory=_rational_layer)


def test_nested_layer_prefix(tmp_path):
    def model():
        torch.manual_seed(3)
        return nn.Sequential(_rational_layer(seed=3), nn.ReLU(), nn.Linear(8, 2))

    src = model()
    with torch.no_grad():
        src[0].atoms.p.add_(0.25)
        src[2].weight.mul_(2.0)
    _save(tmp_path / "s.safetensors", src)
    out = hub.load_safetensors(tmp_path / "s.safetensors", model_factory=model)
    for k, v in src.state_dict().items():
        assert torch.equal(out.state_dict()[k], v)


def test_reference_rational_file_loads(tc, tmp_path):  # noqa: F811
    from torchcst import kernels as rk
    ref = _reference_layer(tc, 8, 16, rk.rational_radius(radius_max=4.0, radius_fraction=0.0),
                           atoms=12)
    # A relaid-out reference layer: rows stay the model, ids only label them.
    ref.atom_state.relayout(torch.arange(11, -1, -1))
    _save(tmp_path / "r.safetensors", ref)
    out = hub.load_safetensors(tmp_path / "r.safetensors", model_factory=_rational_layer)
    assert torch.equal(out.atoms.p.detach(), ref.state_dict()["atom_state.atoms.p"])
    # A layer declaring another coordinate rule does not take the file.
    with pytest.raises(ValueError, match="kernel.amplitude_max"):
        hub.load_safetensors(tmp_path / "r.safetensors",
                             model_factory=lambda: _rational_layer(amplitude_max=16.0))


def test_reference_polar_file_loads(tc, tmp_path):  # noqa: F811
    from torchcst import kernels as rk
    from torchcst.kernels import RadiusBounds as RB
    ref = _reference_layer(tc, 64, 64, rk.polar(amplitude_max=1.0, w_c=0.3, bounds=RB(
        minimum=0.5, birth=4.0, maximum=16.0, upper_floor=1.0)), atoms=12)
    _save(tmp_path / "p.safetensors", ref)

    def own(w_c=0.3):
        b = RadiusBounds(minimum=0.5, birth=4.0, maximum=16.0, upper_floor=1.0)
        return CSTLinear(charts=(_grid(64), _grid(64)), atoms=12,
                         kernel=kernels.product(kernels.cell_mass(ChebyshevSpec(modes=8)),
                                                coordinates=kernels.polar(
                                                    amplitude_max=1.0, w_c=w_c, bounds=b)))

    out = hub.load_safetensors(tmp_path / "p.safetensors", model_factory=own)
    assert torch.equal(out.atoms.p.detach(), ref.state_dict()["atom_state.atoms.p"])
    with pytest.raises(ValueError, match="kernel.w_c"):
        hub.load_safetensors(tmp_path / "p.safetensors", model_factory=lambda: own(w_c=0.25))


def test_broken_row_map_is_refused(tmp_path):
    layer = _rational_layer()
    entries = {"atom_state.atoms.p": layer.atoms.p.detach(),
               "atom_state._row_to_id": torch.zeros(12, dtype=torch.int64),
               "atom_state._id_to_row": torch.arange(12)}
    save_file(entries, str(tmp_path / "m.safetensors"))
    with pytest.raises(ValueError, match="not an atom-id permutation"):
        hub.load_safetensors(tmp_path / "m.safetensors", model_factory=_rational_layer)


def test_from_pretrained_uses_the_hub_download(tmp_path, monkeypatch):
    import huggingface_hub
    src = _rational_layer(seed=4)
    _save(tmp_path / "model.safetensors", src)
    calls = []

    def fake_download(*, repo_id, filename, revision, token):
        calls.append((repo_id, filename, revision, token))
        return str(tmp_path / filename)

    monkeypatch.setattr(huggingface_hub, "hf_hub_download", fake_download)
    out = hub.from_pretrained("org/model", model_factory=lambda: _rational_layer(seed=5),
                              revision="main")
    assert calls == [("org/model", "model.safetensors", "main", None)]
    assert torch.equal(out.atoms.p.detach(), src.atoms.p.detach())
