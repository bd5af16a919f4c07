"""Mixer registry: plugs this package's layers into archbench's registry (the drop-in boundary,
archbench/layers/__init__.py:1-26) or builds them standalone.

    import archbench_b200.registry as r
    r.install()          # archbench's build_mixer("gdn" | "nsgdn", ...) now builds the B200 layers

Builders keep archbench's signature ``builder(d_model, layer_idx, n_layer, **layer_kwargs)`` so
``Block.__init__`` (archbench/model.py:40) and the configs' ``model.layer`` keys work unchanged.
The ``gdn`` module is wrapped like archbench's FLAMixer (``.layer`` attribute, tensor output) so
state-dict keys match the fla-backed original.
"""

from __future__ import annotations

import inspect

import torch.nn as nn

from .layers import GatedDeltaNet, NStepGDN


class MixerWrapper(nn.Module):
    """Same attribute name and output contract as archbench's FLAMixer (fla.py:11-18)."""

    def __init__(self, layer: nn.Module):
        super().__init__()
        self.layer = layer

    def forward(self, x, *args, **kwargs):
        out = self.layer(x, *args, **kwargs)
        return out[0] if isinstance(out, tuple) else out


def build_nsgdn(d_model: int, layer_idx: int, n_layer: int, **kwargs) -> nn.Module:
    """archbench/layers/nsgdn.py:545-547."""
    return NStepGDN(d_model, layer_idx=layer_idx, **kwargs)


def build_gdn(d_model: int, layer_idx: int, n_layer: int, **kwargs) -> nn.Module:
    """archbench/layers/fla.py:36-38 + build_fla's keyword filling (fla.py:21-33)."""
    accepted = inspect.signature(GatedDeltaNet).parameters
    auto = {"hidden_size": d_model, "layer_idx": layer_idx, "num_hidden_layers": n_layer}
    kwargs = {**{k: v for k, v in auto.items() if k in accepted}, **kwargs}
    wrapper = MixerWrapper
    try:  # use archbench's own wrapper class when archbench is importable (its init logic keys on it)
        from archbench.layers.fla import FLAMixer

        wrapper = FLAMixer
    except Exception:
        pass
    return wrapper(GatedDeltaNet(**kwargs))


BUILDERS = {"gdn": build_gdn, "nsgdn": build_nsgdn}


def build_mixer(name: str, d_model: int, layer_idx: int, n_layer: int, **kwargs) -> nn.Module:
    if name not in BUILDERS:
        raise KeyError(f"unknown arch {name!r}; available: {sorted(BUILDERS)}")
    return BUILDERS[name](d_model=d_model, layer_idx=layer_idx, n_layer=n_layer, **kwargs)


def install() -> None:
    """Point archbench's registry entries ``gdn`` and ``nsgdn`` at the B200 layers."""
    from archbench import layers as L

    for name, fn in BUILDERS.items():
        L._REGISTRY[name] = fn
