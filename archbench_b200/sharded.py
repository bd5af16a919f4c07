"""Head-sharded multi-GPU execution of the gated delta rule.

Every (b, h) recurrence is independent (archbench/layers/nsgdn.py:408-417 never mixes heads),
so heads are partitioned over ranks and each rank runs the prefill kernel on its own heads
with no inter-GPU traffic inside the recurrence.  The one collective is an NCCL all-gather of
the outputs, issued only when a caller needs all heads on every rank.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops


def head_slice(H: int, rank: int, world: int) -> slice:
    """Heads owned by ``rank``: a contiguous block of H / world heads."""
    if H % world:
        raise ValueError(f"H={H} heads do not split over {world} ranks")
    n = H // world
    return slice(rank * n, (rank + 1) * n)


def gather_heads(y_local: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """All-gather head shards (B, T, H/world, DV) into a contiguous (B, T, H, DV) tensor.

    NCCL gathers rank-major blocks; one permute-copy then interleaves them into the
    (B, T, H, DV) layout the caller expects."""
    if world == 1:
        return y_local
    y_local = y_local.contiguous()
    B, T, hl, DV = y_local.shape
    buf = torch.empty((world * B, T, hl, DV), dtype=y_local.dtype, device=y_local.device)
    dist.all_gather_into_tensor(buf, y_local, group=group)  # rank-major blocks along dim 0
    return buf.view(world, B, T, hl, DV).permute(1, 2, 0, 3, 4).reshape(B, T, world * hl, DV)


def sharded_prefill(q, k, v, la, beta=None, u=None, initial_state=None, output_final_state=False, gather=True, group=None,
                    impl="auto", layout="bthd"):
    """Run this rank's heads of a full-head problem and optionally all-gather y.

    q, k, v, la, beta, u, initial_state hold ALL heads (every rank passes the same logical
    tensors, e.g. views of a replicated activation); each rank computes heads
    ``head_slice(H, rank, world)``.  Returns (y, S_T_local): S_T_local covers this rank's heads; y is
    this rank's (B, T, H/world, DV) without ``gather``, else every head:
      layout "bthd"  (B, T, H, DV): NCCL gathers rank-major blocks, one permute-copy interleaves them;
      layout "hbtd"  (H, B, T, DV), head-major: the kernel writes this rank's heads straight into its
                     slice of the gather buffer and the all-gather runs in place -- no copy at all."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    if layout not in ("bthd", "hbtd"):
        raise ValueError(f"layout must be 'bthd' or 'hbtd', got {layout!r}")
    H = q.shape[2]
    hs = head_slice(H, rank, world)
    sel = lambda t: None if t is None else t[:, :, hs]
    s0 = None if initial_state is None else initial_state[:, hs]
    if gather and layout == "hbtd":
        B, T, DV = q.shape[0], q.shape[1], v.shape[-1]
        full = torch.empty((H, B, T, DV), dtype=q.dtype, device=q.device)
        mine = full[hs]
        S = ops.gdn_prefill_into(mine.permute(1, 2, 0, 3), sel(q), sel(k), sel(v), sel(la), beta=sel(beta), u=sel(u),
                                 initial_state=s0, output_final_state=output_final_state, impl=impl)
        if world > 1:
            dist.all_gather_into_tensor(full, mine, group=group)  # in place: rank r's block is already there
        return full, S
    y, S = ops.gdn_prefill(sel(q), sel(k), sel(v), sel(la), beta=sel(beta), u=sel(u), initial_state=s0,
                           output_final_state=output_final_state, impl=impl)
    if gather:
        y = gather_heads(y, world, group)
    return y, S
