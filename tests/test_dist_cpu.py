"""Multi-rank host logic on CPU with the gloo backend (world size 2), no GPU.

* head sharding + all-gather reassemble the full (B, T, H, DV) output on every rank;
* sharded_prefill runs each rank's heads only (the kernel call is replaced by the CPU oracle
  here, since this host has no GPU) and the gathered result equals the unsharded oracle, in the
  (B, T, H, DV) layout and in the head-major layout whose gather runs in place (the kernel's output
  view is this rank's slice of the gather buffer);
* failure detection: when one rank raises before the collective, the other rank's collective
  ends with an error within the process group's short timeout instead of hanging.
"""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _worker_gather(rank, world, port, q):
    try:
        _init(rank, world, port)
        from archbench_b200.sharded import gather_heads

        B, T, hl, DV = 2, 5, 3, 4
        y = torch.full((B, T, hl, DV), float(rank)) + torch.arange(hl).view(1, 1, hl, 1) * 10
        full = gather_heads(y, world)
        expect = torch.cat([torch.full((B, T, hl, DV), float(r)) + torch.arange(hl).view(1, 1, hl, 1) * 10 for r in range(world)], 2)
        q.put((rank, bool(torch.equal(full, expect)), None))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, False, repr(e)))


def _worker_sharded(rank, world, port, q):
    try:
        _init(rank, world, port)
        from archbench_b200 import ops, sharded
        from archbench_b200.workloads import make_inputs
        from oracle import oracle as O

        calls = []

        def fake_prefill(q_, k, v, la, beta=None, u=None, initial_state=None, output_final_state=False, impl="auto"):
            calls.append(q_.shape[2])
            y, S = O.recurrence(q_.numpy(), k.numpy(), v.numpy(), la.numpy(), beta=beta.numpy())
            return torch.from_numpy(y).float(), (torch.from_numpy(S).float() if output_final_state else None)

        ops.gdn_prefill = fake_prefill
        x = make_inputs(1, 24, 4, 16, 8, seed=5, dtype=torch.float32)
        y, _ = sharded.sharded_prefill(x["q"], x["k"], x["v"], x["la"], beta=x["beta"])
        y_ref, _ = O.recurrence(x["q"].numpy(), x["k"].numpy(), x["v"].numpy(), x["la"].numpy(), beta=x["beta"].numpy())
        ok = calls == [2] and np.allclose(y.numpy(), y_ref, atol=1e-6)
        q.put((rank, bool(ok), None))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover
        q.put((rank, False, repr(e)))


def _worker_sharded_head_major(rank, world, port, q):
    try:
        _init(rank, world, port)
        from archbench_b200 import ops, sharded
        from archbench_b200.workloads import make_inputs
        from oracle import oracle as O

        seen = []

        def fake_prefill_into(y, q_, k, v, la, beta=None, u=None, initial_state=None, output_final_state=False, impl="auto"):
            seen.append((tuple(y.shape), y.stride()))
            out, S = O.recurrence(q_.numpy(), k.numpy(), v.numpy(), la.numpy(), beta=beta.numpy())
            y.copy_(torch.from_numpy(out).float())  # through the strided view: into the gather buffer
            return torch.from_numpy(S).float() if output_final_state else None

        ops.gdn_prefill_into = fake_prefill_into
        x = make_inputs(2, 24, 4, 16, 8, seed=6, dtype=torch.float32)
        full, _ = sharded.sharded_prefill(x["q"], x["k"], x["v"], x["la"], beta=x["beta"], layout="hbtd")
        y_ref, _ = O.recurrence(x["q"].numpy(), x["k"].numpy(), x["v"].numpy(), x["la"].numpy(), beta=x["beta"].numpy())
        ok = (tuple(full.shape) == (4, 2, 24, 8) and seen == [((2, 24, 2, 8), (24 * 8, 8, 2 * 24 * 8, 1))]
              and np.allclose(full.permute(1, 2, 0, 3).numpy(), y_ref, atol=1e-6))
        q.put((rank, bool(ok), None))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover
        q.put((rank, False, repr(e)))


def _worker_failure(rank, world, port, q):
    _init(rank, world, port, timeout_s=4)
    if rank == 1:
        q.put((rank, "raised", None))
        raise SystemExit(3)  # this rank dies before the collective
    from archbench_b200.sharded import gather_heads

    try:
        gather_heads(torch.zeros(1, 2, 1, 4), world)
        q.put((rank, "no-error", None))
    except Exception as e:
        q.put((rank, "error", type(e).__name__))


def _run(fn, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=timeout) for _ in range(world)]
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return sorted(out, key=lambda t: t[0])


def test_gather_heads_two_ranks():
    res = _run(_worker_gather)
    assert all(ok for _, ok, _ in res), res


def test_sharded_prefill_matches_unsharded():
    res = _run(_worker_sharded)
    assert all(ok for _, ok, _ in res), res


def test_sharded_prefill_head_major_gathers_in_place():
    res = _run(_worker_sharded_head_major)
    assert all(ok for _, ok, _ in res), res


def test_dead_rank_is_detected_not_hung():
    res = _run(_worker_failure)
    by_rank = {r: (status, detail) for r, status, detail in res}
    assert by_rank[1][0] == "raised"
    assert by_rank[0][0] == "error", by_rank
