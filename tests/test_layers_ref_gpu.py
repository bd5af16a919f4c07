"""The drop-in NStepGDN against archbench's own NStepGDN.forward (archbench/layers/nsgdn.py:517-542).

``tests/golden/nsgdn_layer.npz`` holds the reference layer's float32 outputs on CPU (where its
``pick_scan`` runs ``nsgdn_ref``), made by ``tests/golden/make_golden.py`` with the parameters of
``tests/golden/layer_params.py``.  Here the same parameters go into this package's layer, which
runs on the B200 kernels:

* ``scan_impl="ref"`` maps to the fp32 recurrent kernel with the fp32 prologue/epilogue kernels:
  rel-L2 <= 1e-4 on the layer output (fp32 arithmetic throughout; the GEMMs are cuBLAS fp32);
* the default ``scan_impl="chunk"`` runs the tensor-core chunk kernels on bf16 q, k, u, v, as the
  reference's own chunk path casts them (nsgdn.py:400-405): rel-L2 <= 1e-2 and max-abs <= 2e-2
  on the layer output, which carries that input rounding (about 2e-3 per element) through the
  output norm and projection;
* the same in a training forward (autograd graph: the whole-mixer autograd node).

Cases: n_steps 1 and 2, expand_v 1 and 2, ragged T = 100, with and without the output gate.
The host test ``test_layer_params_digest`` (no GPU) checks that the parameter generator fills this
package's layer with exactly the values the fixture was made from."""

import os
import sys

import numpy as np
import pytest
import torch

from archbench_b200.layers import NStepGDN

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import layer_params  # noqa: E402
from make_golden import LAYER_CASES  # noqa: E402

FIX = np.load(os.path.join(HERE, "golden", "nsgdn_layer.npz"))


def _build(i):
    name, B, T, D, kw = LAYER_CASES[i]
    m = NStepGDN(D, **kw)
    digest = layer_params.fill(m, 500 + i)
    x = layer_params.layer_input(B, T, D, 600 + i)
    return name, m, x, digest


def _err(got, want):
    d = got.double().cpu() - torch.from_numpy(want).double()
    return d.abs().max().item(), (d.norm() / torch.from_numpy(want).double().norm()).item()


@pytest.mark.parametrize("i", range(len(LAYER_CASES)))
def test_layer_params_digest(i):
    name, m, x, digest = _build(i)
    assert digest == FIX[f"{name}_params_sha256"].item().decode()
    assert abs(x.double().sum().item() - float(FIX[f"{name}_x_sum"])) < 1e-9


@pytest.mark.gpu
@pytest.mark.parametrize("i", range(len(LAYER_CASES)))
def test_nsgdn_layer_fp32_scan_matches_reference_layer(i):
    name, m, x, _ = _build(i)
    m.scan_impl, m._impl = "ref", "recurrent"
    m = m.cuda()
    with torch.no_grad():
        y = m(x.cuda())
    torch.cuda.synchronize()
    mx, rel = _err(y, FIX[f"{name}_y"])
    assert rel <= 1e-4, f"{name}: max-abs {mx:.3e} rel-L2 {rel:.3e}"


@pytest.mark.gpu
@pytest.mark.parametrize("train", [False, True])
@pytest.mark.parametrize("i", range(len(LAYER_CASES)))
def test_nsgdn_layer_chunk_scan_matches_reference_layer(i, train):
    name, m, x, _ = _build(i)
    m = m.cuda()
    xc = x.cuda()
    if train:
        y = m(xc.requires_grad_(True))
        y.float().square().mean().backward()  # the backward runs too; its values are tested elsewhere
        y = y.detach()
    else:
        with torch.no_grad():
            y = m(xc)
    torch.cuda.synchronize()
    mx, rel = _err(y, FIX[f"{name}_y"])
    assert rel <= 1e-2 and mx <= 2e-2, f"{name} train={train}: max-abs {mx:.3e} rel-L2 {rel:.3e}"
