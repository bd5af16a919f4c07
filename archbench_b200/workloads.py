"""Seeded synthetic workloads with the value distributions of the benchmark configurations.

Distributions (the same for every configuration):
    q, k ~ N(0, 1), L2-normalised per head; q then scaled by DK^-1/2 (as the nsgdn layer does,
        archbench/layers/nsgdn.py:527)
    v ~ N(0, 1)
    beta = sigmoid(N(0, 1))
    la = log alpha = logsigmoid(N(0, 1) + 4) / 8
    S_0 = 0
Draw order is q, k, v, beta, la from one ``torch.Generator`` seeded with ``seed``; the values
are drawn in float32 and then rounded to ``dtype`` (q, k, v only; beta and la stay float32).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F


@dataclass(frozen=True)
class Config:
    name: str
    B: int
    T: int
    H: int
    DK: int
    DV: int
    dtype: torch.dtype
    note: str


CONFIGS = {
    "cfg0": Config("cfg0", 2, 512, 4, 64, 64, torch.float32, "single-layer forward, fp32, chunk 64 (CPU-runnable case)"),
    "cfg1": Config("cfg1", 8, 4096, 8, 128, 128, torch.bfloat16, "chunkwise prefill, bf16 q/k/v, fp32 gates and state"),
    "cfg2": Config("cfg2", 256, 1, 16, 128, 128, torch.bfloat16, "recurrent decode step; state from a 1024-token prefill"),
    "cfg3": Config("cfg3", 1, 65536, 32, 128, 128, torch.bfloat16, "long-context prefill, heads sharded over GPUs"),
}

DECODE_PREFILL_T = 1024
DECODE_STEPS = 1024


def make_inputs(B, T, H, DK, DV, seed=0, dtype=torch.bfloat16, device="cpu"):
    """dict(q, k, v, beta, la) with the distributions above; q/k/v in ``dtype``, gates fp32."""
    g = torch.Generator(device=device).manual_seed(seed)
    f32 = dict(generator=g, device=device, dtype=torch.float32)
    q = F.normalize(torch.randn(B, T, H, DK, **f32), dim=-1) * DK**-0.5
    k = F.normalize(torch.randn(B, T, H, DK, **f32), dim=-1)
    v = torch.randn(B, T, H, DV, **f32)
    beta = torch.sigmoid(torch.randn(B, T, H, **f32))
    la = F.logsigmoid(torch.randn(B, T, H, **f32) + 4) / 8
    return dict(q=q.to(dtype), k=k.to(dtype), v=v.to(dtype), beta=beta, la=la)


def make_config_inputs(cfg: Config | str, seed=0, device="cpu", T=None, B=None, H=None):
    """Inputs of a named configuration, optionally with a smaller B, T or H."""
    c = CONFIGS[cfg] if isinstance(cfg, str) else cfg
    return make_inputs(B or c.B, T or c.T, H or c.H, c.DK, c.DV, seed=seed, dtype=c.dtype, device=device)


def prefill_flops_per_token_head(DK=128, DV=128, C=64):
    """Algorithmic tensor FLOPs per token and head of the chunked prefill at chunk size C.

    2 * (C*DK [Q U^T] + C*DK [K U^T] + C*DK [W = T (gamma K)] + C*DV [U_wy = T V]
         + C*DV [intra-chunk output] + 3*DK*DV [W S^T, Q S^T, R^T U state update]).
    """
    return 2 * (3 * C * DK + 2 * C * DV + 3 * DK * DV)


def prefill_bytes_per_token_head(DK=128, DV=128, in_bytes=2, out_bytes=2):
    """Algorithmic HBM bytes per token and head: q, k, v in, y out, beta and la (fp32) in."""
    return in_bytes * (2 * DK + DV) + out_bytes * DV + 8


def decode_bytes_per_token_head(DK=128, DV=128, in_bytes=2, out_bytes=2):
    """Algorithmic HBM bytes per decode step and head: fp32 state read and written once,
    plus q, k, v, beta, la in and y out."""
    return 2 * 4 * DK * DV + in_bytes * (2 * DK + DV) + out_bytes * DV + 8


def backward_flops_per_chunk(C=64, D=128):
    """Tensor FLOPs the chunked backward executes per (b, h, chunk) with DK = DV = D:
    2 * (10 C D^2 + 17 C^2 D + 2 C^3) multiply-adds.  C D^2 products: the prep pass's dY^T Gamma Q, the
    forward chain's R and state update, the backward chain's d U dS^T and dR^T W, and in the local pass
    R, dR, dY S0, R dS1, dR S0; C^2 D products: the prep pass's K U^T, Q U^T, T Gamma K, T V, A^T dY and
    twelve in the local pass; C^3: the two products of dL = -T^T dT T^T."""
    return 2 * (10 * C * D * D + 17 * C * C * D + 2 * C**3)


def backward_bytes_per_token_head(D=128, in_bytes=2, dy_bytes=2):
    """Algorithmic HBM bytes of the backward per token and head: q, k, v, dy and the gates in; fp32 dq,
    dk, dv, dla and dbeta out (the chunk workspace traffic is extra)."""
    return in_bytes * 3 * D + dy_bytes * D + 8 + 4 * 3 * D + 8
