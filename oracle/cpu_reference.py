"""Timed CPU baseline -- TEST/BENCH INFRASTRUCTURE ONLY.

A PyTorch restatement of archbench's own CPU path for this op, ``nsgdn_ref``
(archbench/layers/nsgdn.py:408-417): a Python loop over tokens of batched fp32 matmuls on
(B, H, DV, DK) states, run on the host's cores through torch's intra-op thread pool.  It is
what ``NStepGDN.forward`` executes on a CPU tensor (``pick_scan`` returns ``nsgdn_ref``,
nsgdn.py:54-55).  ``bench.py`` times it as ``cpu_baseline`` and as the ``--impl reference``
arm; the reference tree itself is not available on the GPU host, so this restatement stands
in for it (same operations, same order, same dtype).  It also accepts an initial state and
returns the final state, which the bench's decode workload needs.
"""

from __future__ import annotations

import torch


@torch.no_grad()
def nsgdn_ref_torch(q, k, u, v, la, s0=None):
    """y (B,T,H,DV), S_T (B,H,DV,DK) -- the loop of nsgdn.py:410-417 with an initial state."""
    B, T, H, DK = q.shape
    S = q.new_zeros(B, H, v.shape[-1], DK) if s0 is None else s0.clone()
    ys = []
    for t in range(T):
        S = la[:, t].exp()[..., None, None] * S
        r = v[:, t] - (S @ k[:, t][..., None]).squeeze(-1)
        S = S + r[..., :, None] * u[:, t][..., None, :]
        ys.append((S @ q[:, t][..., None]).squeeze(-1))
    return torch.stack(ys, 1), S
