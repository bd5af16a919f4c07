"""The decoder LM of benchmark configuration 4, for the bench and the tests.

archbench's own ``LM`` (archbench/model.py:18-149) picks this package's mixers up unchanged
through ``registry.install()``; that tree is not present where the benchmarks run, so this module
restates the part of it configuration 4 uses, with the same module names and maths:

    x = embed(idx); for each block: x = x + mixer(norm1(x)); x = x + mlp(norm2(x))
    logits = lm_head(norm(x)), lm_head tied to the embedding          (model.py:36-48, 122-149)
    mlp: SwiGLU, hidden = round_up(2/3 * mlp_ratio * d_model, 64)      (model.py:18-33)

archbench's optional extras (per-layer residual scalars, the mid-depth backout, embedding norm)
are available as keywords; the embedding smear is not, since cached decoding cannot serve it
(``decode.bind_caches``).  Configuration 4: 24 ``gdn`` blocks, d_model 1024, 8 heads of
head_dim 128 with expand_v 1, short convolutions of width 4, output gate, RMSNorm, SwiGLU hidden
2816 (mlp_ratio 4.125), vocabulary 50304, bf16 weights ~ N(0, 0.02) (``config4_lm``).
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from .registry import build_mixer


class MLP(nn.Module):
    def __init__(self, d_model: int, ratio: float):
        super().__init__()
        hidden = (int(2 / 3 * ratio * d_model) + 63) // 64 * 64
        self.up = nn.Linear(d_model, 2 * hidden, bias=False)
        self.down = nn.Linear(hidden, d_model, bias=False)

    def forward(self, x):
        a, b = self.up(x).chunk(2, dim=-1)
        return self.down(F.silu(a) * b)


class Block(nn.Module):
    def __init__(self, arch: str, d_model: int, layer_idx: int, n_layer: int, mlp_ratio: float, norm_eps: float, layer: dict):
        super().__init__()
        self.norm1 = nn.RMSNorm(d_model, eps=norm_eps)
        self.mixer = build_mixer(arch, d_model, layer_idx, n_layer, **layer)
        self.norm2 = nn.RMSNorm(d_model, eps=norm_eps)
        self.mlp = MLP(d_model, mlp_ratio)

    def forward(self, x):
        x = x + self.mixer(self.norm1(x))
        return x + self.mlp(self.norm2(x))


class LM(nn.Module):
    def __init__(self, arch="gdn", d_model=1024, n_layer=24, vocab_size=50304, mlp_ratio=4.125, norm_eps=1e-5,
                 layer=None, resid_scalars=False, backout=False, embed_norm=False, init_std=0.02):
        super().__init__()
        self.n_layer, self.embed_norm = n_layer, embed_norm
        self.embed = nn.Embedding(vocab_size, d_model)
        self.blocks = nn.ModuleList(Block(arch, d_model, i, n_layer, mlp_ratio, norm_eps, dict(layer or {}))
                                    for i in range(n_layer))
        self.norm = nn.RMSNorm(d_model, eps=norm_eps)
        self.lm_head = nn.Linear(d_model, vocab_size, bias=False)
        self.lm_head.weight = self.embed.weight
        self.resid_lambdas = self.x0_lambdas = self.backout_lambda = self.smear_gate = None
        L = n_layer
        if resid_scalars:  # model.py:68-70
            self.resid_lambdas = nn.Parameter(torch.tensor([1.15 - 0.10 * i / max(L - 1, 1) for i in range(L)]))
            self.x0_lambdas = nn.Parameter(torch.tensor([0.20 - 0.15 * i / max(L - 1, 1) for i in range(L)]))
        if backout:
            self.backout_lambda = nn.Parameter(torch.full((1,), 0.2))
        for m in self.modules():  # every projection and the embedding ~ N(0, init_std)
            if isinstance(m, (nn.Linear, nn.Embedding)):
                nn.init.normal_(m.weight, mean=0.0, std=init_std)

    def forward(self, idx: torch.Tensor, targets=None):
        x = self.embed(idx)
        if self.embed_norm:
            x = F.rms_norm(x, (x.size(-1),))
        x0, x_mid = x, None
        for i, block in enumerate(self.blocks):
            if self.resid_lambdas is not None:
                x = self.resid_lambdas[i] * x + self.x0_lambdas[i] * x0
            x = block(x)
            if i == self.n_layer // 2:
                x_mid = x
        if self.backout_lambda is not None:
            x = x - self.backout_lambda * x_mid
        logits = self.lm_head(self.norm(x))
        loss = None
        if targets is not None:
            loss = F.cross_entropy(logits.float().flatten(0, 1), targets.flatten())
        return logits, loss


CONFIG4 = dict(arch="gdn", d_model=1024, n_layer=24, vocab_size=50304, mlp_ratio=4.125,
               layer=dict(num_heads=8, head_dim=128, expand_v=1.0, use_gate=True, use_short_conv=True, conv_size=4))


def config4_lm(device="cuda", dtype=torch.bfloat16, **overrides) -> LM:
    """Configuration 4's model (random init), optionally with fewer layers etc. for tests."""
    kw = {**CONFIG4, **overrides}
    return LM(**kw).to(device=device, dtype=dtype).eval()
