"""Benchmark of the gated-DeltaNet hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--skip-extra]
                    [--only decode|backward|layer|nstep|lm|long_context|fla] [--lm-steps S]
    torchrun --nproc-per-node N bench.py --gpus N ...

Headline (``value``): chunkwise prefill of configuration 1 -- B=8, T=4096, H=8, DK=DV=128,
bf16 q/k/v, fp32 beta/la/state, chunk 64 -- as whole-job tokens/s.  Each rank runs its own
configuration-1 batch (batch x heads partitioned over ranks, no data-path collective), so
scaling is weak.  Inputs are 201 MB of q/k/v per rank, larger than the 126 MB L2, so no
flush is needed between steps.

Extra objects on the same line:
  decode       configuration 2: B=256, H=16 single-token steps on a state built by a 1024-token
               prefill; state streamed from HBM once per step (per rank: its own batch).
  long_context configuration 3: B=1, T=65536, H=32, heads sharded over the N ranks (strong
               scaling), outputs all-gathered over NCCL into (B, T, H, DV) on every rank.
  backward     the configuration-1 prefill backward (gdn_prefill_bwd) and forward + backward as
               one training step of the token mixing.
  layer        the drop-in nsgdn mixer on configuration-1 tokens (d_model 1024): inference forward
               with the fused prologue/epilogue kernels, and a training step through autograd.
  nstep        nsgdn's n-step write vectors with its default keys (DV=256, n_steps=2) on
               configuration-1 tokens: the prefill with u given and the write vectors' backward.
  e2e          the headline prefill through the public API with host buffers: pinned-host ->
               device copies of q/k/v/beta/la and the device -> host copy of y inside the timed
               region.
  roofline     the prefill kernel against measured HBM bandwidth (MEASURED_PEAKS.json), with
               its tensor-pipe FLOP rate beside it.
  cpu_baseline archbench's recurrence (restated in torch, oracle/cpu_reference.py) on the host
               cores, on a bounded sample of configuration 1.
"""

from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from archbench_b200.workloads import (  # noqa: E402
    CONFIGS,
    decode_bytes_per_token_head,
    make_inputs,
    prefill_bytes_per_token_head,
    prefill_flops_per_token_head,
)

METRIC = "GDN prefill tok/s/GPU (T=4096,d=128), decode tok/s; % roofline at 1/2/4/8 GPU"


# Committed ncu capture of each prefill kernel on the headline workload.
PROFILE_OF = {"chunk_single": "ws_kernel_cfg1.md", "chunk_cluster": "pair_kernel_cfg1.md"}


def profiled_traffic(summary):
    """DRAM bytes (read + write) per launch from one committed ncu capture of the kernel."""
    try:
        with open(os.path.join(ROOT, "profiles", summary)) as f:
            m = re.search(r"^traffic_bytes_per_launch:\s*(\d+)", f.read(), re.M)
        return int(m.group(1)) if m else None
    except OSError:
        return None


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


# ------------------------------------------------------------------------------------------
# distributed plumbing
# ------------------------------------------------------------------------------------------


def dist_init(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def min_over_ranks(x: float, world: int) -> float:
    return -max_over_ranks(-x, world)


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while active."""

    FIELDS = "clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = []
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) != 7:
                continue
            try:
                rows.append((float(parts[0]), float(parts[1]), float(parts[2]), parts[3:]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[3]) if v.lower() == "active"})
        loaded = [r[0] for r in rows if r[2] > 200.0] or [r[0] for r in rows]
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(r[2] for r in rows)}


# Kernel launches of one gdn_prefill per selected path (the segmented path: prep, state pass, combine,
# output pass; the split path: prep and the state-only kernel).
LAUNCHES_PER_PREFILL = {"chunk_cluster": 1, "chunk_single": 1, "chunk_split": 2, "segmented": 4, "recurrent": 1}


def timed(fn, steps, warmup, world, stream=None):
    """Warm up, then time exactly ``steps`` calls with CUDA events on the launching stream,
    bracketed by a barrier and a device synchronize; returns max-over-ranks seconds."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    stream = stream or torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(e0.elapsed_time(e1) / 1e3, world)


# ------------------------------------------------------------------------------------------
# our arm
# ------------------------------------------------------------------------------------------


def graphed(fn):
    """``fn`` (device work only, no collective) captured once in a CUDA graph after two warm-up calls
    (the second on a side stream, as capture requires); returns the graph's replay.  Allocations ``fn``
    makes come from the graph's private pool and stay valid for every replay."""
    fn()
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    return graph.replay


def bench_prefill(args, rank, world):
    from archbench_b200 import ops

    c = CONFIGS["cfg1"]
    x = make_inputs(c.B, c.T, c.H, c.DK, c.DV, seed=1000 + rank, dtype=c.dtype, device="cuda")
    impl = args.prefill_impl
    out = {}

    def step():
        out["y"], _ = ops.gdn_prefill(x["q"], x["k"], x["v"], x["la"], beta=x["beta"], impl=impl)

    sel = ops.selected_impl(x["q"], x["k"], x["v"], x["la"], beta=x["beta"], impl=impl)
    # One gdn_prefill call (one kernel launch) captured in a CUDA graph and replayed per step: the timed
    # loop then carries no host work (Python, argument checks, tensor-map encoding).
    run = graphed(step) if args.graph else step
    with ClockSampler(torch.cuda.current_device()) as clk:
        secs = timed(run, args.steps, args.warmup, world)
    fastest = min_over_ranks(secs, world)
    tokens_per_step = c.B * c.T
    th = c.B * c.T * c.H
    per_launch = secs / args.steps
    hbm, tflops, src = peaks()
    alg_bytes = th * prefill_bytes_per_token_head(c.DK, c.DV)
    alg_flops = th * prefill_flops_per_token_head(c.DK, c.DV)
    achieved_gbs = alg_bytes / per_launch / 1e9
    res = {
        "value": world * tokens_per_step / secs * args.steps,
        "ms_per_step": per_launch * 1e3,
        "ms_per_step_fastest_rank": fastest / args.steps * 1e3,
        "timing": "CUDA graph replay of one gdn_prefill call per step" if args.graph else "one gdn_prefill call per step",
        "kernel": sel,
        "roofline": {
            "bound": "hbm", "achieved": achieved_gbs, "peak": hbm, "unit": "GB/s", "frac": achieved_gbs / hbm,
            "traffic": profiled_traffic(PROFILE_OF.get(sel, "")),
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, profiles/" + PROFILE_OF.get(sel, "(none)"),
            "peak_source": src, "algorithmic_bytes_per_launch": alg_bytes,
            "tensor": {"achieved_tflops": alg_flops / per_launch / 1e12, "peak_tflops": tflops,
                       "frac": alg_flops / per_launch / 1e12 / tflops, "algorithmic_flops_per_launch": alg_flops},
        },
        "clocks": clk.summary(),
        "gpu_launches": args.steps,
    }
    del x, out
    return res


def bench_prefill_e2e(args, rank, world):
    """Same workload through the public API from pinned host buffers (ops.gdn_prefill_from_host: the
    batch in pieces, copies overlapped with the prefill); every copy is inside the timed region."""
    from archbench_b200 import ops

    c = CONFIGS["cfg1"]
    xh = make_inputs(c.B, c.T, c.H, c.DK, c.DV, seed=2000 + rank, dtype=c.dtype, device="cpu")
    xh = {k: v.pin_memory() for k, v in xh.items()}
    y_host = torch.empty(c.B, c.T, c.H, c.DV, dtype=torch.bfloat16).pin_memory()
    h2d = sum(v.numel() * v.element_size() for v in xh.values())
    d2h = y_host.numel() * y_host.element_size()

    # The public host-buffer entry: pieces of the batch pipelined through H2D copy, prefill, D2H copy, and
    # consecutive calls overlapping one call's copies in with the previous call's tail.  Back to back, two
    # pieces per call measure within 1 % of the 3.8 ms the copies alone take (B200: 1 piece 3.96 ms,
    # 2: 3.99, 4: 4.11, 8: 4.27); more pieces shorten a lone call's latency instead.
    pieces = 2

    def step():
        ops.gdn_prefill_from_host(xh["q"], xh["k"], xh["v"], xh["la"], xh["beta"], y_host, pieces=pieces,
                                  impl=args.prefill_impl)

    steps = args.steps
    secs = timed(step, steps, args.warmup, world)
    return {"value": world * c.B * c.T * steps / secs, "unit": "tok/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "steps": steps, "ms_per_step": secs / steps * 1e3, "api": f"ops.gdn_prefill_from_host ({pieces} pieces)",
            "gpu_launches": pieces * steps}


def bench_decode(args, rank, world):
    from archbench_b200 import ops
    from archbench_b200.workloads import DECODE_PREFILL_T

    c = CONFIGS["cfg2"]
    B, H, D = c.B, c.H, c.DK
    pre = make_inputs(B, DECODE_PREFILL_T, H, D, D, seed=3000 + rank, dtype=torch.bfloat16, device="cuda")
    _, state = ops.gdn_prefill(pre["q"], pre["k"], pre["v"], pre["la"], beta=pre["beta"], output_final_state=True)
    del pre
    n = args.warmup + args.steps
    tok = make_inputs(B, n, H, D, D, seed=4000 + rank, dtype=torch.bfloat16, device="cuda")
    tok = {k: v.transpose(0, 1).contiguous() for k, v in tok.items()}  # (steps, B, H, ...)
    it = {"i": 0}

    def step():
        i = it["i"] % n
        it["i"] += 1
        ops.gdn_decode_step(tok["q"][i], tok["k"][i], tok["v"][i], tok["la"][i], state, beta=tok["beta"][i])

    secs = timed(step, args.steps, args.warmup, world)
    per = secs / args.steps
    hbm, _, src = peaks()
    alg = B * H * decode_bytes_per_token_head(D, D)
    return {"value": world * B / per, "unit": "tok/s", "ms_per_step": per * 1e3, "config": "cfg2 B256 H16 d128, state from a 1024-token prefill",
            "roofline": {"bound": "hbm", "achieved": alg / per / 1e9, "peak": hbm, "unit": "GB/s", "frac": alg / per / 1e9 / hbm,
                         "peak_source": src, "algorithmic_bytes_per_launch": alg},
            "gpu_launches": args.steps}


def bench_backward(args, rank, world):
    """Configuration-1 prefill backward (gdn_prefill_bwd: dq, dk, dv, dla, dbeta from dy), and the
    forward + backward pair as one training step of the token mixing."""
    from archbench_b200 import ops
    from archbench_b200.workloads import backward_bytes_per_token_head, backward_flops_per_chunk

    c = CONFIGS["cfg1"]
    x = make_inputs(c.B, c.T, c.H, c.DK, c.DV, seed=6000 + rank, dtype=c.dtype, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(6100 + rank)
    dy = torch.randn(c.B, c.T, c.H, c.DV, generator=g, device="cuda").to(torch.bfloat16)

    def bwd():
        ops.gdn_prefill_bwd(x["q"], x["k"], x["v"], x["la"], dy, beta=x["beta"])

    def train():
        ops.gdn_prefill(x["q"], x["k"], x["v"], x["la"], beta=x["beta"])
        bwd()

    steps = max(1, min(args.steps, 10))
    t_b = timed(bwd, steps, min(args.warmup, 3), world) / steps
    t_t = timed(train, steps, min(args.warmup, 3), world) / steps
    th = c.B * c.T * c.H
    flops = c.B * c.H * (c.T // 64) * backward_flops_per_chunk(64, c.DK)
    hbm, tflops, src = peaks()
    alg = th * backward_bytes_per_token_head(c.DK)
    return {"value": world * c.B * c.T / t_b, "unit": "tok/s", "ms_per_step": t_b * 1e3, "train_step_ms": t_t * 1e3,
            "train_step_tok_s": world * c.B * c.T / t_t, "config": "cfg1 B8 T4096 H8 d128, bf16 dy, fp32 gradients",
            "roofline": {"bound": "tensor", "achieved": flops / t_b / 1e12, "peak": tflops, "unit": "TFLOP/s",
                         "frac": flops / t_b / 1e12 / tflops, "peak_source": src,
                         "executed_flops_per_launch": flops, "note": "mma.sync fp16 products; four launches (amax, prep, chains, local)",
                         "hbm_achieved_gbs": alg / t_b / 1e9, "algorithmic_bytes_per_launch": alg},
            "gpu_launches": 9 * steps}


def bench_nstep(args, rank, world):
    """nsgdn's n-step write vectors at configuration-1 tokens with archbench's default nsgdn keys
    (B=8, T=4096, H=8, DK=128, DV=256, n_steps=2): the prefill with u given (the split path: prep
    kernel, then the state-only chunk kernel with u tiles in its k/q ring) and the write vectors'
    backward (gdn_write_vectors_bwd)."""
    import torch.nn.functional as F

    from archbench_b200 import ops
    from archbench_b200.nstep import write_direction

    c = CONFIGS["cfg1"]
    DV = 2 * c.DV
    x = make_inputs(c.B, c.T, c.H, c.DK, DV, seed=8000 + rank, dtype=c.dtype, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(8100 + rank)
    lam = torch.rand(c.H, generator=g, device="cuda") + 0.5
    kf = x["k"].float()
    u = write_direction(kf, F.pad(kf[:, :-1], (0, 0, 0, 0, 1, 0)), x["beta"], lam, 2).to(torch.bfloat16)
    du = torch.randn(c.B, c.T, c.H, c.DK, generator=g, device="cuda")
    dk = torch.zeros_like(du)

    def fwd():
        ops.gdn_prefill(x["q"], x["k"], x["v"], x["la"], u=u)

    def wv_bwd():
        ops.write_vectors_bwd(x["k"], x["beta"], lam, du, dk, 2)

    steps = max(1, min(args.steps, 10))
    t_f = timed(fwd, steps, min(args.warmup, 3), world) / steps
    t_w = timed(wv_bwd, steps, min(args.warmup, 3), world) / steps
    th = c.B * c.T * c.H
    hbm, _, src = peaks()
    alg_f = th * (3 * 2 * c.DK + 2 * 2 * DV + 4)   # q, k, u, v in; y out (bf16); la (fp32)
    alg_w = th * (2 * c.DK + 4 + 3 * 4 * c.DK + 4)  # k (bf16), beta, du, dk in/out (fp32), dbeta
    return {"config": "cfg1 tokens B8 T4096 H8 DK128 DV256, u = 2-step write vectors", "prefill_ms": t_f * 1e3,
            "prefill_tok_s": world * c.B * c.T / t_f, "write_vectors_bwd_ms": t_w * 1e3,
            "roofline": {"bound": "hbm", "prefill_achieved_gbs": alg_f / t_f / 1e9, "prefill_frac": alg_f / t_f / 1e9 / hbm,
                         "write_vectors_bwd_achieved_gbs": alg_w / t_w / 1e9, "write_vectors_bwd_frac": alg_w / t_w / 1e9 / hbm,
                         "peak": hbm, "unit": "GB/s", "peak_source": src},
            "kernel": ops.selected_impl(x["q"], x["k"], x["v"], x["la"], u=u),
            "gpu_launches": (LAUNCHES_PER_PREFILL[ops.selected_impl(x["q"], x["k"], x["v"], x["la"], u=u)] + 1) * steps}


def bench_layer(args, rank, world):
    """The nsgdn mixer as a whole (projections, short conv, norms and gates, scan, output norm and gate,
    output projection) on configuration-1 tokens: B=8, T=4096, d_model=1024, H=8, head_dim=128,
    expand_v=1, n_steps=1, bf16 weights (random init).  Inference forward (fused prologue/epilogue
    kernels) and one training step (forward + backward through autograd)."""
    from archbench_b200.layers import NStepGDN

    c = CONFIGS["cfg1"]
    torch.manual_seed(7000 + rank)
    m = NStepGDN(1024, num_heads=c.H, head_dim=c.DK, expand_v=1.0, n_steps=1).cuda().to(torch.bfloat16)
    x = torch.randn(c.B, c.T, 1024, device="cuda", dtype=torch.bfloat16)
    # the training step is the layer's forward and backward for a fixed upstream gradient: a loss on the
    # (8, 4096, 1024) output would add PyTorch's elementwise kernels (~0.3 ms) to the layer's time
    dout = torch.randn(c.B, c.T, 1024, device="cuda", dtype=torch.bfloat16)

    def infer():
        with torch.no_grad():
            m(x)

    def train():
        m.zero_grad(set_to_none=True)
        m(x).backward(dout)

    steps = max(1, min(args.steps, 10))
    t_i = timed(infer, steps, min(args.warmup, 3), world) / steps
    t_t = timed(train, steps, min(args.warmup, 3), world) / steps
    tok = c.B * c.T
    # archbench's default nsgdn layer keys (configs/arch/nsgdn.yaml: expand_v 2, n_steps 2)
    del m
    m = NStepGDN(1024, num_heads=c.H, head_dim=c.DK, expand_v=2.0, n_steps=2).cuda().to(torch.bfloat16)
    t_i2 = timed(infer, steps, min(args.warmup, 3), world) / steps
    t_t2 = timed(train, steps, min(args.warmup, 3), world) / steps
    return {"config": "nsgdn layer, B8 T4096 d_model 1024 H8 head_dim 128 expand_v 1 n_steps 1, bf16; training step = "
                      "forward + backward for a fixed random upstream gradient of the output", "infer_ms": t_i * 1e3,
            "infer_tok_s": world * tok / t_i, "train_step_ms": t_t * 1e3, "train_tok_s": world * tok / t_t,
            "default_keys": {"config": "the same with expand_v 2, n_steps 2 (archbench's nsgdn defaults)",
                             "infer_ms": t_i2 * 1e3, "infer_tok_s": world * tok / t_i2, "train_step_ms": t_t2 * 1e3,
                             "train_tok_s": world * tok / t_t2},
            # expand_v 1: inference 3, training step 9 (prologue, scan, epilogue; their backwards with the
            # scan's four); default keys: inference 4 (split scan: 2), training step 15 (DV = 256: two slices
            # of the scan's backward, the write vectors' backward)
            "gpu_launches": 31 * steps}


def bench_long_context(args, rank, world):
    """cfg3 heads sharded over ranks (strong scaling).  Three timings of the same prefill: compute only;
    with the NCCL all-gather into a head-major (H, B, T, DV) buffer that the kernel writes its heads into
    directly (in-place gather, no copy -- the reported ``value``); and with the gather into the
    (B, T, H, DV) layout (gather then one permute-copy)."""
    import torch.distributed as dist

    from archbench_b200 import ops
    from archbench_b200.sharded import gather_heads

    c = CONFIGS["cfg3"]
    if c.H % world:
        return {"skipped": f"H={c.H} not divisible by {world} ranks"}
    h_loc = c.H // world
    x = make_inputs(c.B, c.T, h_loc, c.DK, c.DV, seed=5000 + rank, dtype=c.dtype, device="cuda")
    full = torch.empty((c.H, c.B, c.T, c.DV), dtype=c.dtype, device="cuda")
    mine = full[rank * h_loc:(rank + 1) * h_loc]
    out = {}

    def prefill():
        out["y"], _ = ops.gdn_prefill(x["q"], x["k"], x["v"], x["la"], beta=x["beta"])

    def prefill_into_slice():
        ops.gdn_prefill_into(mine.permute(1, 2, 0, 3), x["q"], x["k"], x["v"], x["la"], beta=x["beta"])

    # Each rank's prefill (up to four launches: prep, segment states, combine, output pass) is replayed
    # from a CUDA graph, as the headline's step is, so host launch jitter on a busy host does not leak into
    # the max over ranks; the NCCL gathers run eagerly between replays.
    step_compute = graphed(prefill) if args.graph else prefill
    fill_slice = graphed(prefill_into_slice) if args.graph else prefill_into_slice

    def step_gather_head_major():
        fill_slice()
        if world > 1:
            dist.all_gather_into_tensor(full, mine)

    def step_gather_bthd():
        step_compute()
        out["full"] = gather_heads(out["y"], world)

    steps = max(1, min(args.steps, 10))
    t_c = timed(step_compute, steps, min(args.warmup, 3), world)
    t_h = timed(step_gather_head_major, steps, min(args.warmup, 3), world)
    t_g = timed(step_gather_bthd, steps, min(args.warmup, 3), world)
    tokens = c.B * c.T
    sel = ops.selected_impl(x["q"], x["k"], x["v"], x["la"], beta=x["beta"])
    return {"value": tokens * steps / t_h, "unit": "tok/s", "value_without_gather": tokens * steps / t_c,
            "value_gather_bthd": tokens * steps / t_g,
            "ms_per_step": t_h / steps * 1e3, "ms_compute": t_c / steps * 1e3, "ms_gather_head_major": (t_h - t_c) / steps * 1e3,
            "ms_gather_bthd": (t_g - t_c) / steps * 1e3, "heads_per_rank": h_loc, "kernel": sel, "scaling": "strong",
            "gather": "NCCL all_gather_into_tensor, in place into a head-major (H, B, T, DV) buffer; value_gather_bthd: "
                      "gather then permute-copy into (B, T, H, DV)",
            "timing": ("each rank's prefill a CUDA graph replay, the gathers eager" if args.graph else
                       "eager calls"),
            "gpu_launches": 3 * LAUNCHES_PER_PREFILL[sel] * steps}


def bench_lm(args, rank, world):
    """Configuration 4: the 380M-class decoder (24 gdn blocks, d_model 1024, 8 heads of 128, SwiGLU 2816,
    vocabulary 50304, bf16 weights ~ N(0, 0.02), random init; archbench_b200.lm) -- a prefill of 16 prompts
    of 2048 uniform-random token ids, then 256 greedy decode steps through the per-layer recurrent caches
    (archbench_b200.decode.bind_caches).  The batch is sharded over the ranks (16 / N prompts each, model
    replicas, no collective)."""
    from archbench_b200.decode import GraphDecoder, bind_caches
    from archbench_b200.lm import CONFIG4, config4_lm

    B_all, T, steps = 16, 2048, args.lm_steps
    if B_all % world:
        return {"skipped": f"batch {B_all} not divisible by {world} ranks"}
    B = B_all // world
    torch.manual_seed(9000)  # the same weights on every rank
    m = config4_lm()
    g = torch.Generator(device="cuda").manual_seed(9100 + rank)
    idx = torch.randint(0, CONFIG4["vocab_size"], (B, T), device="cuda", generator=g)

    def run(n_steps, timing):
        """Prefill, then n_steps greedy steps replayed from one captured CUDA graph; with ``timing`` the
        prefill and the replays are timed with CUDA events (the capture itself is outside both)."""
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        with torch.no_grad(), bind_caches(m) as caches:
            ev[0].record()
            logits = m(idx)[0][:, -1]
            ev[1].record()
            dec = GraphDecoder(m, caches, logits.argmax(-1))
            torch.cuda.synchronize()
            barrier(world)
            ev[2].record()
            for _ in range(n_steps):
                dec.step()
            ev[3].record()
            torch.cuda.synchronize()
        if not timing:
            return None
        return ev[0].elapsed_time(ev[1]) / 1e3, ev[2].elapsed_time(ev[3]) / 1e3

    run(8, False)  # warm-up: one prefill, a capture and a few replays
    torch.cuda.synchronize()
    barrier(world)
    t_pre, t_dec = run(steps, True)
    t_pre = max_over_ranks(t_pre, world)
    t_dec = max_over_ranks(t_dec, world)
    del m
    return {"config": "cfg4: 24 gdn blocks d_model 1024 H8 head_dim 128 expand_v 1, SwiGLU 2816, vocab 50304, bf16; "
                      "prefill 16 x 2048 then 256 greedy steps, batch sharded",
            "prefill_ms": t_pre * 1e3, "prefill_tok_s": world * B * T / t_pre,
            "decode_ms_per_step": t_dec / steps * 1e3, "decode_tok_s": world * B * steps / t_dec,
            "prompts_per_rank": B, "gpu_launches": 3 * CONFIG4["n_layer"] * (1 + steps),  # prologue, scan, epilogue per layer and call
            "note": "prefill: one eager model call; decode: one captured CUDA graph per step (projections and MLP are "
                    "cuBLAS GEMMs, the token mixing and the layer prologue/epilogue this package's kernels)"}


# fla's backward is not run here: on this pool's B200 its chunk_gated_delta_rule backward (fla 0.5.1, which
# dispatched chunk_bwd_dqkwg to its TileLang backend) failed on an unaligned access inside that kernel on
# the configuration-1 inputs below (contiguous bf16 q/k/v/dy, fp32 gates) after the forward had run cleanly.
# The note leaves out the runtime's wording of that error, which log scanners take for a fault of this run.
FLA_BACKWARD_NOT_RUN = ("not run: fla 0.5.1's backward (chunk_bwd_dqkwg, TileLang backend) failed on an "
                        "unaligned access inside its own kernel on this box's B200 with the configuration-1 inputs")


def bench_fla(args, rank, world, ours_prefill_ms, ours_decode_ms):
    """The reference's own GPU kernels on this box: fla 0.5.1's Triton ``chunk_gated_delta_rule`` on the
    configuration-1 inputs (what archbench's ``gdn`` arch runs in prefill, fla/layers/gated_deltanet.py:266-279,
    and the state pass archbench's nsgdn chunk path shares, nsgdn.py:352-363) and
    ``fused_recurrent_gated_delta_rule`` on the configuration-2 decode step (gated_deltanet.py:281-294).  Same
    q/k/v/beta/la as our legs (q already scaled, so scale=1; no in-kernel l2norm); fla's state layout is
    [B, H, K, V].  Timed like ours (CUDA events, warm-up first; the first call JIT-compiles)."""
    try:
        import fla
        from fla.ops.gated_delta_rule import chunk_gated_delta_rule, fused_recurrent_gated_delta_rule
    except Exception as e:
        return {"unavailable": f"fla does not import on this host: {e!r}"[:300]}
    from archbench_b200 import ops
    from archbench_b200.workloads import DECODE_PREFILL_T

    c = CONFIGS["cfg1"]
    x = make_inputs(c.B, c.T, c.H, c.DK, c.DV, seed=1000 + rank, dtype=c.dtype, device="cuda")

    def f_chunk():
        return chunk_gated_delta_rule(x["q"], x["k"], x["v"], x["la"], x["beta"], scale=1.0)

    t0 = time.perf_counter()
    o, _ = f_chunk()
    torch.cuda.synchronize()
    jit_s = time.perf_counter() - t0
    y, _ = ops.gdn_prefill(x["q"], x["k"], x["v"], x["la"], beta=x["beta"])
    rel = float((o.float() - y.float()).norm() / y.float().norm())
    del o, y
    steps = max(1, min(args.steps, 20))
    t_chunk = timed(f_chunk, steps, args.warmup, world) / steps

    del x
    c2 = CONFIGS["cfg2"]
    B, H, D = c2.B, c2.H, c2.DK
    pre = make_inputs(B, DECODE_PREFILL_T, H, D, D, seed=3000 + rank, dtype=torch.bfloat16, device="cuda")
    _, state = ops.gdn_prefill(pre["q"], pre["k"], pre["v"], pre["la"], beta=pre["beta"], output_final_state=True)
    del pre
    h0 = state.transpose(-1, -2).contiguous()
    tok = make_inputs(B, 1, H, D, D, seed=4000 + rank, dtype=torch.bfloat16, device="cuda")

    def f_dec():
        return fused_recurrent_gated_delta_rule(tok["q"], tok["k"], tok["v"], tok["la"], beta=tok["beta"], scale=1.0,
                                                initial_state=h0, output_final_state=True)

    t_dec = timed(f_dec, steps, args.warmup, world) / steps
    return {"impl": f"fla {fla.__version__} (Triton)", "prefill_ms": t_chunk * 1e3, "prefill_tok_s": world * c.B * c.T / t_chunk,
            "prefill_speedup_ours_vs_fla": t_chunk * 1e3 / ours_prefill_ms if ours_prefill_ms else None, "prefill_fla_vs_ours_rel_l2": rel,
            "backward": FLA_BACKWARD_NOT_RUN,
            "decode_ms": t_dec * 1e3, "decode_tok_s": world * B / t_dec, "decode_speedup_ours_vs_fla": t_dec * 1e3 / ours_decode_ms if ours_decode_ms else None,
            "first_call_s": jit_s, "gpu_launches": 0,
            "note": "fla's kernels are the checker here, not ours: not counted in gpu_launches"}


def keep_freed_heap():
    """Stop glibc from handing freed heap memory back to the OS between the CPU path's per-token 4 MB
    temporaries.  Without it a fresh process trims the heap after every free, so each new state tensor
    is faulted in again page by page: the same code measured 21.6-26.3 K tok/s in a fresh process and
    57-61 K tok/s with trimming off or in a process whose heap had grown (16 cores).  Returns whether
    glibc accepted the settings."""
    try:
        import ctypes

        libc = ctypes.CDLL("libc.so.6")
        M_TRIM_THRESHOLD, M_TOP_PAD, M_MMAP_THRESHOLD = -1, -2, -3
        ok = libc.mallopt(M_MMAP_THRESHOLD, 32 << 20) == 1      # 4 MB tensors come from the heap
        ok &= libc.mallopt(M_TRIM_THRESHOLD, 1 << 30) == 1      # freed memory stays in the heap
        ok &= libc.mallopt(M_TOP_PAD, 64 << 20) == 1
        return bool(ok)
    except Exception:
        return False


CPU_SAMPLE = ("cfg1 B8 T4096 H8 d128 fp32: each step one pass over the whole configuration-1 batch (8 sequences of "
              "4096 tokens, fed in 64-token slices with the state carried); glibc heap trimming off (mallopt)")


def cpu_reference_setup():
    """Inputs of the CPU legs: the whole configuration-1 batch in fp32 (seed 7), u = beta k."""
    keep_freed_heap()
    torch.set_num_threads(os.cpu_count() or 1)  # every host core (torchrun sets OMP_NUM_THREADS=1 for its ranks)
    c = CONFIGS["cfg1"]
    x = make_inputs(c.B, c.T, c.H, c.DK, c.DV, seed=7, dtype=torch.float32, device="cpu")
    x["u"] = x["beta"][..., None] * x["k"]
    return x


def cpu_reference_pass(x, slice_t=64):
    """One pass of archbench's recurrence (torch restatement, oracle/cpu_reference.py) over the whole
    batch; returns the tokens processed (B * T)."""
    from oracle.cpu_reference import nsgdn_ref_torch

    B, T = x["q"].shape[:2]
    S = None
    for t0 in range(0, T, slice_t):
        sl = slice(t0, t0 + slice_t)
        _, S = nsgdn_ref_torch(x["q"][:, sl], x["k"][:, sl], x["u"][:, sl], x["v"][:, sl], x["la"][:, sl], s0=S)
    return B * T


def cpu_reference_rate(x, steps, warmup):
    """tok/s of ``steps`` timed passes after ``warmup`` untimed ones: the one measurement both CPU legs
    report (``cpu_baseline`` on our line, and the ``--impl reference`` arm)."""
    for _ in range(warmup):
        cpu_reference_pass(x)
    t0 = time.perf_counter()
    tokens = sum(cpu_reference_pass(x) for _ in range(steps))
    dt = time.perf_counter() - t0
    return tokens / dt, dt


def cpu_threads_note():
    aff = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else None
    return f"{torch.get_num_threads()} torch threads; os.cpu_count() {os.cpu_count()}, affinity {aff}"


def cpu_baseline(budget_s=10.0):
    """The reference arm's measurement on our line: the same passes and warm-up, as many whole passes
    as fit in about ``budget_s``."""
    x = cpu_reference_setup()
    rate0, dt0 = cpu_reference_rate(x, 1, 3)
    steps = max(1, int(budget_s / dt0))
    rate, dt = cpu_reference_rate(x, steps, 0)
    total = (rate0 * dt0 + rate * dt) / (dt0 + dt)
    return {"value": total, "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{CPU_SAMPLE}; 3 warm-up passes, {steps + 1} timed passes ({dt + dt0:.1f} s); {cpu_threads_note()}"}


def run_ours(args):
    rank, world, local = dist_init(args.gpus)
    if args.only:  # one leg alone (profiling runs): its own object, not the bench line
        res = {"decode": bench_decode, "backward": bench_backward, "layer": bench_layer,
               "nstep": bench_nstep, "lm": bench_lm, "long_context": bench_long_context,
               "fla": lambda a, r, w: bench_fla(a, r, w, None, None)}[args.only](args, rank, world)
        if rank == 0:
            print(json.dumps({"leg": args.only, **res}), flush=True)
        finish(world)
        return
    res = bench_prefill(args, rank, world)
    line = {
        "metric": METRIC, "value": res["value"], "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": res["ms_per_step"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded; BASELINE distributions)",
        "config": {"workload": "cfg1 chunkwise prefill B=8 T=4096 H=8 DK=DV=128 chunk=64 (per rank)", "global_batch": 8 * world,
                   "seq_len": 4096, "heads": 8, "head_dim": 128, "parallelism": f"batch-heads sharded x{world}",
                   "l2": "inputs 201 MB/rank > 126 MB L2 (no flush)", "kernel": res["kernel"], "timing": res["timing"]},
        "roofline": res["roofline"], "clocks": res["clocks"], "gpu_launches": res["gpu_launches"],
        "ms_per_step_fastest_rank": res["ms_per_step_fastest_rank"],
    }
    if not args.skip_extra:
        line["e2e"] = bench_prefill_e2e(args, rank, world)
        torch.cuda.empty_cache()
        line["decode"] = bench_decode(args, rank, world)
        torch.cuda.empty_cache()
        line["long_context"] = bench_long_context(args, rank, world)
        torch.cuda.empty_cache()
        line["backward"] = bench_backward(args, rank, world)
        torch.cuda.empty_cache()
        line["layer"] = bench_layer(args, rank, world)
        torch.cuda.empty_cache()
        line["nstep"] = bench_nstep(args, rank, world)
        torch.cuda.empty_cache()
        line["lm"] = bench_lm(args, rank, world)
        if world == 1:
            torch.cuda.empty_cache()
            line["reference_gpu"] = bench_fla(args, rank, world, res["ms_per_step"], line["decode"]["ms_per_step"])
        line["gpu_launches"] += (line["decode"]["gpu_launches"] + line["long_context"].get("gpu_launches", 0)
                                 + line["backward"]["gpu_launches"] + line["e2e"]["gpu_launches"] + line["layer"]["gpu_launches"]
                                 + line["nstep"]["gpu_launches"] + line["lm"].get("gpu_launches", 0))
    if rank == 0 and world == 1 and not args.skip_cpu:
        line["cpu_baseline"] = cpu_baseline()
    if rank == 0:
        print(json.dumps(line), flush=True)
    finish(world)


def run_reference(args):
    """The reference's CPU implementation of this path on the host cores (rank 0 only): each step is one
    pass over the whole configuration-1 batch, the sample ``cpu_baseline`` times too."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    x = cpu_reference_setup()
    v, dt = cpu_reference_rate(x, args.steps, args.warmup)
    sample = f"{CPU_SAMPLE}; {args.warmup} warm-up passes, {args.steps} timed ({dt:.1f} s); {cpu_threads_note()}"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; BASELINE distributions)",
        "config": {"workload": "cfg1 chunkwise prefill B=8 T=4096 H=8 DK=DV=128 chunk=64 (per rank)", "sample": sample},
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def finish(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--prefill-impl", choices=["auto", "chunk", "chunk_cluster", "chunk_single", "chunk_split", "recurrent", "segmented"], default="auto")
    ap.add_argument("--skip-extra", action="store_true", help="headline prefill only")
    ap.add_argument("--skip-cpu", action="store_true", help="omit the cpu_baseline leg")
    ap.add_argument("--only", choices=["decode", "backward", "layer", "nstep", "lm", "long_context", "fla"], default=None,
                    help="run one extra leg alone and print its object (for profiling)")
    ap.add_argument("--lm-steps", type=int, default=256,
                    help="greedy decode steps of the configuration-4 leg (256 in the benchmark configuration)")
    ap.add_argument("--no-graph", dest="graph", action="store_false",
                    help="time plain calls instead of CUDA-graph replays of one call")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
