"""Deterministic parameters for the layer-level golden fixtures.

``make_golden.py`` builds archbench's own ``NStepGDN`` (archbench/layers/nsgdn.py:473-515), fills
every parameter with ``fill(module, seed)`` and records its forward output; the tests build this
package's drop-in ``NStepGDN`` with the same keywords, fill it with the same call and compare.  The
values come from one seeded ``torch.Generator`` walked over the state dict in name order, so only
the seed has to be stored, and the fixture records a digest of the filled values to pin it.

Distributions follow the reference's own initialisers (nsgdn.py:458-515), widened where the
reference starts from a constant so that every term of the layer is exercised:
  in_proj, o_proj   U(-1/sqrt(fan_in), 1/sqrt(fan_in))  (nn.Linear's default bound)
  conv.weight       U(-1/sqrt(size), 1/sqrt(size))
  A_log             log U(1, 16)
  dt_bias           softplus^-1 of dt, dt = exp(U(log 1e-3, log 0.1))
  b_bias            N(0, 0.5)    (zeros in the reference)
  lam               softplus^-1 of U(0.5, 1.5)    (softplus^-1(1) in the reference)
  norm.weight       1 + N(0, 0.1)  (ones in the reference)
"""

from __future__ import annotations

import hashlib
import math

import numpy as np
import torch


def values(name: str, shape, g: torch.Generator) -> torch.Tensor:
    f = dict(generator=g, dtype=torch.float32)
    if name.endswith("proj.weight"):
        b = 1.0 / math.sqrt(shape[-1])
        return (torch.rand(shape, **f) * 2 - 1) * b
    if name == "conv.weight":
        b = 1.0 / math.sqrt(shape[-1])
        return (torch.rand(shape, **f) * 2 - 1) * b
    if name == "A_log":
        return (torch.rand(shape, **f) * 15 + 1).log()
    if name == "dt_bias":
        dt = torch.exp(torch.rand(shape, **f) * (math.log(0.1) - math.log(0.001)) + math.log(0.001))
        return dt + torch.log(-torch.expm1(-dt))
    if name == "b_bias":
        return torch.randn(shape, **f) * 0.5
    if name == "lam":
        lam = torch.rand(shape, **f) + 0.5
        return torch.log(torch.expm1(lam))
    if name == "norm.weight":
        return 1 + 0.1 * torch.randn(shape, **f)
    raise KeyError(f"no generator for parameter {name!r}")


def fill(module: torch.nn.Module, seed: int) -> str:
    """Overwrite every parameter of ``module`` in name order; returns the sha256 of the values."""
    g = torch.Generator().manual_seed(seed)
    h = hashlib.sha256()
    sd = module.state_dict()
    new = {}
    for name in sorted(sd):
        t = values(name, tuple(sd[name].shape), g)
        new[name] = t
        h.update(name.encode())
        h.update(np.ascontiguousarray(t.numpy()).tobytes())
    module.load_state_dict(new)
    return h.hexdigest()


def layer_input(B: int, T: int, d_model: int, seed: int) -> torch.Tensor:
    """The layer input x ~ N(0, 1), (B, T, d_model) float32."""
    return torch.randn(B, T, d_model, generator=torch.Generator().manual_seed(seed))
