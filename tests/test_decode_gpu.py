"""Greedy decoding through bound caches (archbench_b200.decode) against re-running the whole
sequence, the way archbench's generation loop does (archbench/core_eval.py:136-142).

The model is a stand-in with the structure of archbench's LM (archbench/model.py:36-149: embedding,
pre-norm blocks of mixer + SwiGLU MLP with the optional per-layer residual scalars, final RMSNorm,
lm_head, forward(idx) -> (logits, loss)) and mixers from this package's registry.  Tolerance: the
logits each new token is chosen from against the full-sequence logits at the same positions,
rel-L2 <= 5e-3 in fp32 and <= 2e-2 under bf16 autocast (GEMMs of a one-token call and a
full-sequence call round differently)."""

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from archbench_b200.decode import bind_caches, greedy_decode
from archbench_b200.registry import build_mixer

pytestmark = pytest.mark.gpu


class Block(nn.Module):
    def __init__(self, arch, d, i, n, **kw):
        super().__init__()
        self.norm1, self.norm2 = nn.RMSNorm(d, eps=1e-6), nn.RMSNorm(d, eps=1e-6)
        self.mixer = build_mixer(arch, d, i, n, **kw)
        self.up, self.down = nn.Linear(d, 2 * 512, bias=False), nn.Linear(512, d, bias=False)

    def forward(self, x):
        x = x + self.mixer(self.norm1(x))
        a, b = self.up(self.norm2(x)).chunk(2, -1)
        return x + self.down(F.silu(a) * b)


class TinyLM(nn.Module):
    def __init__(self, arch, d=256, n=2, vocab=512, **kw):
        super().__init__()
        self.embed = nn.Embedding(vocab, d)
        self.blocks = nn.ModuleList(Block(arch, d, i, n, **kw) for i in range(n))
        self.norm = nn.RMSNorm(d, eps=1e-6)
        self.lm_head = nn.Linear(d, vocab, bias=False)
        self.resid_lambdas = nn.Parameter(torch.tensor([1.15, 1.05]))
        self.x0_lambdas = nn.Parameter(torch.tensor([0.2, 0.05]))
        self.smear_gate = None

    def forward(self, idx, targets=None):
        x = x0 = self.embed(idx)
        for i, b in enumerate(self.blocks):
            x = b(self.resid_lambdas[i] * x + self.x0_lambdas[i] * x0)
        return self.lm_head(self.norm(x)), None


def rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm()).item()


@pytest.mark.parametrize("arch,kw", [("nsgdn", dict(num_heads=2, head_dim=128, n_steps=1)),
                                     ("nsgdn", dict(num_heads=2, head_dim=128, n_steps=2)),
                                     ("gdn", dict(num_heads=2, head_dim=128, expand_v=1))])
@pytest.mark.parametrize("autocast", [False, True])
def test_greedy_decode_matches_full_recompute(arch, kw, autocast):
    torch.manual_seed(21)
    m = TinyLM(arch, **kw).cuda().eval()
    g = torch.Generator(device="cuda").manual_seed(22)
    idx = torch.randint(0, 512, (2, 100), device="cuda", generator=g)
    steps = 8
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
        ids, got = greedy_decode(m, idx, steps, return_logits=True)
        want = m(ids[:, :-1])[0][:, idx.shape[1] - 1:]
    assert ids.shape == (2, 100 + steps) and torch.equal(ids[:, :100], idx)
    assert torch.equal(ids[:, 100:], got.argmax(-1))
    r = rel(got.float(), want.float())
    assert r <= (2e-2 if autocast else 5e-3), r


def test_bound_caches_hold_state_and_unbind():
    torch.manual_seed(23)
    m = TinyLM("nsgdn", num_heads=2, head_dim=128).cuda().eval()
    idx = torch.randint(0, 512, (2, 70), device="cuda")
    with torch.no_grad():
        with bind_caches(m) as caches:
            m(idx)
            assert len(caches) == 2 and all(c.seen == 70 and c.state is not None for c in caches)
            assert caches[0].state.shape == (2, 2, 256, 128)
        m(idx)  # unbound again: no cache is touched
        assert all(c.seen == 70 for c in caches)
