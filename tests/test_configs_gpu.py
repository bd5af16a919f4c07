"""Benchmark configurations 2 and 3 at their full sizes, checked head by head against the float64
C oracle (the restatement of archbench's nsgdn_ref, archbench/layers/nsgdn.py:408-417).

* Configuration 2: B=256, H=16, d=128; the state comes from a 1024-token chunked prefill, then
  256 single-token decode steps (bf16 q/k/v, fresh beta/la each step) on the full batch.  The
  oracle replays the same 1024 + 256 tokens on a subset of (b, h) pairs, so the check covers the
  prefill's state hand-off and the error growth over the decode run.
* Configuration 3: B=1, T=65536, H=32, d=128 in one launch (the one-GPU shape: the cluster
  kernel), and the 4-head shard of an 8-GPU job (the segmented path), with heads checked
  against the oracle over the whole 65536-token sequence.

Tolerance: max-abs <= 2e-3 and rel-L2 <= 1e-3 on y (fp32 outputs) and on the state, as for the
other chunk-kernel tests."""

import numpy as np
import pytest
import torch

from archbench_b200 import ops
from archbench_b200.workloads import make_inputs
from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL_MAX, TOL_REL = 2e-3, 1e-3


def np32(t):
    return t.detach().float().cpu().numpy()


def check(got, want, what):
    mx, rel = O.errors(np32(got) if isinstance(got, torch.Tensor) else got, want)
    assert mx <= TOL_MAX and rel <= TOL_REL, f"{what}: max-abs {mx:.3e} rel-L2 {rel:.3e}"


def test_cfg2_decode_after_prefill_against_oracle():
    B, H, D, T_pre, steps = 256, 16, 128, 1024, 256
    pre = make_inputs(B, T_pre, H, D, D, seed=3000, dtype=torch.bfloat16, device="cuda")
    tok = make_inputs(B, steps, H, D, D, seed=4000, dtype=torch.bfloat16, device="cuda")
    bs, hs = [0, 97, 255], [0, 7, 15]
    sub = lambda x: x[bs][:, :, hs]
    ref_in = {n: torch.cat([sub(pre[n]), sub(tok[n])], 1) for n in pre}
    _, state = ops.gdn_prefill(pre["q"], pre["k"], pre["v"], pre["la"], beta=pre["beta"], output_final_state=True)
    assert ops.selected_impl(pre["q"], pre["k"], pre["v"], pre["la"], beta=pre["beta"]) in ("chunk_cluster", "chunk_single", "chunk_split")
    del pre
    ys = []
    for t in range(steps):
        ys.append(ops.gdn_decode_step(tok["q"][:, t], tok["k"][:, t], tok["v"][:, t], tok["la"][:, t], state,
                                      beta=tok["beta"][:, t], out_dtype=torch.float32)[bs][:, hs])
    y = torch.stack(ys, 1)
    torch.cuda.synchronize()
    y_o, S_o = O.recurrence_c(*(np32(ref_in[n]) for n in ("q", "k", "v", "la")), beta=np32(ref_in["beta"]))
    check(y, y_o[:, T_pre:], "decode y over 256 steps")
    check(y[:, -1], y_o[:, -1], "decode y at the last step")
    check(state[bs][:, hs], S_o, "state after 1024 + 256 tokens")
    assert ops.device_status() == 0


@pytest.mark.parametrize("H,impl,heads", [(32, "chunk_cluster", [0, 31]), (4, "segmented", [0, 3])])
def test_cfg3_long_context_heads_against_oracle(H, impl, heads):
    B, T, D = 1, 65536, 128
    x = make_inputs(B, T, H, D, D, seed=5000 + H, dtype=torch.bfloat16, device="cuda")
    assert ops.selected_impl(x["q"], x["k"], x["v"], x["la"], beta=x["beta"]) == impl
    y, S = ops.gdn_prefill(x["q"], x["k"], x["v"], x["la"], beta=x["beta"], output_final_state=True,
                           out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    sub = {n: x[n][:, :, heads] for n in x}
    y_o, S_o = O.recurrence_c(*(np32(sub[n]) for n in ("q", "k", "v", "la")), beta=np32(sub["beta"]))
    check(y[:, :, heads], y_o, f"H={H} y")
    check(y[:, -4096:, heads], y_o[:, -4096:], f"H={H} y over the last 4096 tokens")
    check(S[:, heads], S_o, f"H={H} S_T")
