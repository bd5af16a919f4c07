"""Write vectors of the N-step gated delta rule (archbench/layers/nsgdn.py:61-75).

u_1 = beta k; each further step u <- u - lam beta (p.u) p_perp with p = k_{t-1} and
p_perp = p - (p.k) k, which keeps k.u = beta while shrinking the disturbance p.u to the previous
read.  n_steps = 1 is plain GDN (the kernels then take beta directly and form u = beta k
on chip).  Elementwise and O(T * DK): it stays in PyTorch."""

import torch


def write_direction(k: torch.Tensor, p: torch.Tensor, beta: torch.Tensor, lam: torch.Tensor, n_steps: int) -> torch.Tensor:
    b = beta[..., None]
    l = lam[None, None, :, None]
    u = b * k
    if n_steps > 1:
        p_perp = p - (p * k).sum(-1, keepdim=True) * k
        for _ in range(n_steps - 1):
            pu = (p * u).sum(-1, keepdim=True)
            u = u - l * b * pu * p_perp
    return u
