"""Safetensors loading for models built from torchcst_b200 layers.

Mirrors ``torchcst.hub`` (hub.py:17-82): ``load_safetensors`` builds the model
with a factory, checks the file's tensors against the model's state dict
(same keys, shapes and dtypes) and returns the model in eval mode on
``device``; ``from_pretrained`` downloads the file from the Hugging Face Hub
first. The same error messages are raised.

A file saved from a *reference* model also loads into the B200 model that
declares the same layers. A reference ``CSTLinear`` holds tensors that the B200
layer keeps as plain declaration values or does not need:

* ``kernel.<name>`` scalar buffers: the coordinate rule's settings
  (rational: the radius bounds, ``amplitude_max``, ``radius_fraction``,
  ``amplitude_std``; Polar:
  ``amplitude_max``, ``w_c``, the envelope and radius bounds of both axes and
  the update settings). Each must equal the B200 layer's declared value in the
  file's dtype, otherwise loading fails naming the entry: a checkpoint is not
  silently run under another rule.
* ``atom_state._row_to_id`` / ``atom_state._id_to_row``: the reference's stable
  atom-id permutation. The atom rows themselves (``atom_state.atoms.p``) are
  the model; the permutation only labels them, so it is checked (a permutation
  and its inverse) and not stored.

Every other tensor follows the reference rule exactly.
"""

from __future__ import annotations

from collections.abc import Callable
from pathlib import Path
from typing import TypeVar

import torch
from torch import nn

from .spec import PolarRadius, RationalRadius

__all__ = ["from_pretrained", "load_safetensors"]

_Model = TypeVar("_Model", bound=nn.Module)

_ROW_MAPS = ("atom_state._row_to_id", "atom_state._id_to_row")


def _kernel_scalars(coordinates) -> dict[str, float]:
    """The reference's ``kernel.<name>`` buffers of a coordinate rule, by name."""
    if isinstance(coordinates, RationalRadius):
        return {"radius_min": coordinates.radius_min,
                "radius_birth": coordinates.radius_birth,
                "radius_max": coordinates.radius_max,
                "amplitude_max": coordinates.amplitude_max,
                "radius_fraction": coordinates.radius_fraction,
                "amplitude_std": coordinates.amplitude_std}
    if isinstance(coordinates, PolarRadius):
        out = {"amplitude_max": coordinates.amplitude_max, "w_c": coordinates.w_c,
               "kappa": coordinates.kappa, "lower_kappa": coordinates.lower_kappa,
               "upper_decay_power": coordinates.upper_decay_power}
        for side, b in (("input", coordinates.input_bounds),
                        ("output", coordinates.output_bounds)):
            out[f"radius_min_{side}"] = b.minimum
            out[f"radius_birth_{side}"] = b.birth
            out[f"radius_max_{side}"] = b.maximum
            out[f"radius_upper_floor_{side}"] = b.upper_floor
        out.update(alpha_init=coordinates.alpha_init,
                   radial_regularization=coordinates.radial_regularization,
                   activity_gain=coordinates.activity_gain,
                   dormant_expansion_rate=coordinates.dormant_expansion_rate)
        return out
    return {}


def _accept_reference_entries(model: nn.Module, tensors: dict, expected: dict) -> dict:
    """Drop (after checking) the reference-layer tensors the B200 layers do not hold."""
    from .linear import CSTLinear

    tensors = dict(tensors)
    for prefix, module in model.named_modules():
        if not isinstance(module, CSTLinear):
            continue
        pre = f"{prefix}." if prefix else ""
        scalars = _kernel_scalars(module.kernel.coordinates)
        for name, value in scalars.items():
            key = f"{pre}kernel.{name}"
            if key not in tensors or key in expected:
                continue
            stored = tensors[key]
            if stored.numel() != 1 or not stored.is_floating_point():
                raise ValueError(f"Safetensors tensor {key!r} is not a floating-point scalar.")
            declared = torch.tensor(float(value), dtype=stored.dtype)
            if not torch.equal(stored.reshape(()), declared):
                raise ValueError(
                    f"Safetensors tensor {key!r} holds {stored.item()!r}, but the model "
                    f"declares {float(value)!r}.")
            del tensors[key]
        maps = [f"{pre}{m}" for m in _ROW_MAPS]
        if any(k in tensors and k not in expected for k in maps):
            if not all(k in tensors for k in maps):
                raise ValueError(
                    f"Safetensors file holds only one of {maps[0]!r} and {maps[1]!r}.")
            row_to_id, id_to_row = tensors[maps[0]], tensors[maps[1]]
            count = module.atoms.p.shape[0]
            ids = torch.arange(count)
            if (row_to_id.dtype != torch.int64 or id_to_row.dtype != torch.int64
                    or tuple(row_to_id.shape) != (count,) or tuple(id_to_row.shape) != (count,)
                    or not torch.equal(row_to_id.sort().values, ids)
                    or not torch.equal(id_to_row[row_to_id], ids)):
                raise ValueError(
                    f"Safetensors tensors {maps[0]!r} / {maps[1]!r} are not an atom-id "
                    f"permutation of {count} atoms and its inverse.")
            for k in maps:
                del tensors[k]
    return tensors


def _require(module: str, what: str):
    """Import an optional dependency of the hub path, with the reference's hint."""
    import importlib

    try:
        return importlib.import_module(module)
    except ImportError as error:
        raise ImportError(f"Install torchcst[hub] to {what}.") from error


def _check_entries(stored: dict, wanted: dict) -> None:
    """Same keys, then per key the same shape and dtype (the reference's messages)."""
    if stored.keys() != wanted.keys():
        missing = sorted(set(wanted) - set(stored))
        unexpected = sorted(set(stored) - set(wanted))
        raise ValueError("Safetensors keys do not match the model. "
                         f"Missing: {missing}. Unexpected: {unexpected}.")
    for key in stored:
        have, need = stored[key], wanted[key]
        if have.shape == need.shape and have.dtype == need.dtype:
            continue
        raise ValueError(f"Safetensors tensor {key!r} has shape {tuple(have.shape)} "
                         f"and dtype {have.dtype}, expected {tuple(need.shape)} "
                         f"and {need.dtype}.")


def load_safetensors(
    path: str | Path,
    *,
    model_factory: Callable[[], _Model],
    device: str | torch.device = "cpu",
) -> _Model:
    """Build the model with ``model_factory``, load the file's tensors into it and
    return it in eval mode on ``device``. The file holds every tensor of the
    model's state dict and nothing else (a reference model's file may add the
    entries described in the module docstring); non-tensor extra state comes
    from the factory."""
    st = _require("safetensors.torch", "load Safetensors")
    stored = st.load_file(path, device="cpu")
    model = model_factory()
    state = model.state_dict()
    wanted = {key: value for key, value in state.items() if torch.is_tensor(value)}
    stored = _accept_reference_entries(model, stored, wanted)
    _check_entries(stored, wanted)
    state.update(stored)
    model.load_state_dict(state)
    return model.to(device).eval()


def from_pretrained(
    repo_id: str,
    *,
    model_factory: Callable[[], _Model],
    filename: str = "model.safetensors",
    revision: str | None = None,
    device: str | torch.device = "cpu",
    token: str | bool | None = None,
) -> _Model:
    """Fetch ``filename`` of ``repo_id`` from the Hugging Face Hub (or its local
    cache), then ``load_safetensors`` it."""
    hub = _require("huggingface_hub", "download model weights")
    local = hub.hf_hub_download(repo_id=repo_id, filename=filename, revision=revision,
                                token=token)
    return load_safetensors(local, model_factory=model_factory, device=device)
