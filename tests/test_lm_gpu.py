"""Configuration 4's decoder LM (archbench_b200.lm, the structure of archbench/model.py:18-149 with
``gdn`` mixers) through cached greedy decoding (archbench_b200.decode).

* A reduced variant (2 blocks, d_model 256, 2 heads of 128, vocabulary 512, fp32 weights): the
  logits every new token is chosen from against a float64 CPU recompute of the whole sequence in
  which each mixer's token mixing is the oracle recurrence (on q, k, v rounded to bf16 as the layer
  hands them to the kernel), rel-L2 <= 5e-3; every greedy token equals the float64 argmax wherever
  the float64 top-2 margin exceeds 1e-3.
* The full configuration-4 model (24 blocks, d_model 1024, 8 heads, SwiGLU 2816, vocabulary 50304,
  bf16 weights), batch 2, a 256-token prompt and 4 greedy steps: cached decoding against re-running
  the whole sequence on the same kernels, rel-L2 <= 6e-2 (bf16 GEMMs of a one-token call and a
  full-sequence call round differently, and the difference grows through 24 bf16 blocks: 3.6e-2
  measured)."""

import copy
import os
import sys

import pytest
import torch

from archbench_b200.decode import greedy_decode
from archbench_b200.lm import LM, config4_lm

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from test_layers_gpu import gdn_cpu  # noqa: E402

pytestmark = pytest.mark.gpu


def lm_cpu64(m: LM, idx):
    m64 = copy.deepcopy(m).double().cpu()
    with torch.no_grad():
        x = m64.embed(idx.cpu())
        for blk in m64.blocks:
            x = x + gdn_cpu(blk.mixer.layer, blk.norm1(x))
            x = x + blk.mlp(blk.norm2(x))
        return m64.lm_head(m64.norm(x))


def rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return ((a - b).norm() / b.norm()).item()


def test_reduced_config4_greedy_decode_against_float64_recompute():
    torch.manual_seed(31)
    m = LM(arch="gdn", d_model=256, n_layer=2, vocab_size=512,
           layer=dict(num_heads=2, head_dim=128, expand_v=1.0)).cuda().eval()
    idx = torch.randint(0, 512, (2, 100), device="cuda", generator=torch.Generator(device="cuda").manual_seed(32))
    steps = 8
    ids, got = greedy_decode(m, idx, steps, return_logits=True)
    want = lm_cpu64(m, ids[:, :-1])[:, idx.shape[1] - 1:]
    r = rel(got, want)
    assert r <= 5e-3, r
    top2 = want.topk(2, -1).values
    sure = (top2[..., 0] - top2[..., 1]) > 1e-3
    assert torch.equal(ids[:, 100:].cpu()[sure], want.argmax(-1)[sure])


def test_config4_model_cached_decode_against_recompute():
    torch.manual_seed(33)
    m = config4_lm()
    n_params = sum(p.numel() for p in m.parameters())
    assert 3.5e8 < n_params < 4.2e8, n_params  # the 380M class
    idx = torch.randint(0, 50304, (2, 256), device="cuda", generator=torch.Generator(device="cuda").manual_seed(34))
    with torch.no_grad():
        ids, got = greedy_decode(m, idx, 4, return_logits=True)
        want = m(ids[:, :-1])[0][:, idx.shape[1] - 1:]
    assert torch.isfinite(got).all()
    assert torch.equal(ids[:, 256:], got.argmax(-1))
    r = rel(got.float(), want.float())
    assert r <= 6e-2, r


def test_graph_decode_matches_eager_decode():
    """Decode steps replayed from one captured CUDA graph (decode.GraphDecoder) against eager calls."""
    torch.manual_seed(35)
    for arch, layer in (("gdn", dict(num_heads=2, head_dim=128, expand_v=1.0)),
                        ("nsgdn", dict(num_heads=2, head_dim=128, expand_v=2.0, n_steps=2))):
        m = LM(arch=arch, d_model=256, n_layer=2, vocab_size=512, layer=layer).cuda().eval()
        idx = torch.randint(0, 512, (3, 70), device="cuda", generator=torch.Generator(device="cuda").manual_seed(36))
        ids_e, lg_e = greedy_decode(m, idx, 12, return_logits=True)
        ids_g, lg_g = greedy_decode(m, idx, 12, return_logits=True, graph=True)
        assert torch.equal(ids_e, ids_g), arch
        assert rel(lg_g, lg_e) <= 1e-5, (arch, rel(lg_g, lg_e))

