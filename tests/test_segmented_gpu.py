"""The segment-parallel prefill (few long sequences) against the CPU oracle and the fp32
recurrent kernel.  Same tolerance as the single-pass chunk kernel: max-abs <= 2e-3 and
rel-L2 <= 1e-3 on y and S_T (fp32 outputs)."""

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


@pytest.mark.parametrize("T,DV,s0", [(40 * 64, 128, False), (40 * 64 + 37, 128, True), (24 * 64, 256, True)])
def test_segmented_against_oracle(T, DV, s0):
    B, H = 1, 2
    x = make_inputs(B, T, H, 128, DV, seed=T + DV, dtype=torch.bfloat16)
    S0 = torch.randn(B, H, DV, 128, generator=torch.Generator().manual_seed(7)) * 0.3 if s0 else None
    y_o, S_o = O.recurrence_c(*(np32(x[n]) for n in ("q", "k", "v", "la")), beta=np32(x["beta"]), s0=None if S0 is None else S0.numpy())
    g = {k: v.cuda() for k, v in x.items()}
    assert ops.selected_impl(g["q"], g["k"], g["v"], g["la"], beta=g["beta"]) == "segmented"
    y, S = ops.gdn_prefill(g["q"], g["k"], g["v"], g["la"], beta=g["beta"], initial_state=None if S0 is None else S0.cuda(),
                           output_final_state=True, out_dtype=torch.float32, impl="segmented")
    torch.cuda.synchronize()
    check(y, y_o, "y")
    check(S, S_o, "S_T")
    assert ops.device_status() == 0


def test_segmented_long_context_against_recurrent():
    """Configuration-3 sequence length (T = 65536) with 4 heads, as one of 8 GPUs holds them."""
    g = make_inputs(1, 65536, 4, 128, 128, seed=3, dtype=torch.bfloat16, device="cuda")
    y_s, S_s = ops.gdn_prefill(g["q"], g["k"], g["v"], g["la"], beta=g["beta"], output_final_state=True, out_dtype=torch.float32)
    y_r, S_r = ops.gdn_prefill(g["q"], g["k"], g["v"], g["la"], beta=g["beta"], output_final_state=True, out_dtype=torch.float32, impl="recurrent")
    for a, b_, what in ((y_s, y_r, "y"), (S_s, S_r, "S_T")):
        d = (a - b_).double()
        mx, rel = d.abs().max().item(), (d.norm() / b_.double().norm()).item()
        assert mx <= TOL_MAX and rel <= TOL_REL, f"{what}: max-abs {mx:.3e} rel-L2 {rel:.3e}"


def test_segmented_equals_single_pass_bf16_output():
    g = make_inputs(1, 32 * 64, 2, 128, 128, seed=11, dtype=torch.bfloat16, device="cuda")
    y1, _ = ops.gdn_prefill(g["q"], g["k"], g["v"], g["la"], beta=g["beta"], impl="chunk")
    y2, _ = ops.gdn_prefill(g["q"], g["k"], g["v"], g["la"], beta=g["beta"], impl="segmented")
    d = (y1.float() - y2.float())
    assert (d.norm() / y1.float().norm()).item() < 3e-3


@pytest.mark.parametrize("T,DV", [(40 * 64 + 37, 128), (24 * 64, 256)])
def test_segmented_write_vectors_against_oracle(T, DV):
    """Explicit n-step write vectors (nsgdn n_steps = 2, archbench/layers/nsgdn.py:61-75) on the
    segmented path: both passes run the single-CTA kernel with u tiles."""
    B, H = 1, 2
    x = make_inputs(B, T, H, 128, DV, seed=T + 3 * DV, dtype=torch.bfloat16)
    k = np32(x["k"]).astype(np.float64)
    p = np.pad(k[:, :-1], ((0, 0), (1, 0), (0, 0), (0, 0)))
    u = O.write_direction(k, p, np32(x["beta"]).astype(np.float64), np.array([1.0, 0.7]), 2)
    u_bf = torch.from_numpy(u.astype(np.float32)).to(torch.bfloat16)
    S0 = torch.randn(B, H, DV, 128, generator=torch.Generator().manual_seed(9)) * 0.3
    y_o, S_o = O.recurrence_c(*(np32(x[n]) for n in ("q", "k", "v", "la")), u=np32(u_bf), s0=S0.numpy())
    g = {k_: v.cuda() for k_, v in x.items()}
    assert ops.selected_impl(g["q"], g["k"], g["v"], g["la"], u=u_bf.cuda()) == "segmented"
    y, S = ops.gdn_prefill(g["q"], g["k"], g["v"], g["la"], u=u_bf.cuda(), initial_state=S0.cuda(), output_final_state=True,
                           out_dtype=torch.float32)
    torch.cuda.synchronize()
    check(y, y_o, "y")
    check(S, S_o, "S_T")
    assert ops.device_status() == 0
