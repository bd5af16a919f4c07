"""Parity of the token-serial CUDA kernel (prefill and decode) with the CPU oracle.

fp32 inputs: max-abs and rel-L2 <= 1e-5 on y and S_T (the north-star fp32 tolerance).
bf16 inputs: the kernel still computes in fp32, so the same 1e-5 bound holds against the
oracle run on the bf16-rounded inputs (input rounding is not counted as error)."""

import os

import numpy as np
import pytest
import torch

from archbench_b200 import ops
from archbench_b200.workloads import make_inputs
from oracle import oracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
TOL32 = 1e-5


def dev(x):
    return {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in x.items()}


def np32(t):
    return t.detach().float().cpu().numpy()


def check(got, want, tol_max, tol_rel, what):
    mx, rel = O.errors(np32(got) if isinstance(got, torch.Tensor) else got, want)
    assert mx <= tol_max and rel <= tol_rel, f"{what}: max-abs {mx:.3e} rel-L2 {rel:.3e}"


def test_cfg0_fp32_against_oracle():
    x = make_inputs(2, 512, 4, 64, 64, seed=0, dtype=torch.float32)
    y_o, S_o = O.recurrence_c(*(x[n].numpy() for n in ("q", "k", "v", "la")), beta=x["beta"].numpy())
    g = dev(x)
    y, S = ops.gdn_prefill(g["q"], g["k"], g["v"], g["la"], beta=g["beta"], output_final_state=True, impl="recurrent")
    torch.cuda.synchronize()
    assert y.dtype == torch.float32
    check(y, y_o, TOL32, TOL32, "y")
    check(S, S_o, TOL32, TOL32, "S_T")


def test_cfg0_against_reference_golden():
    d = np.load(os.path.join(GOLD, "cfg0.npz"))
    x = dev(make_inputs(2, 512, 4, 64, 64, seed=0, dtype=torch.float32))
    y, S = ops.gdn_prefill(x["q"], x["k"], x["v"], x["la"], beta=x["beta"], output_final_state=True)
    check(y[:, ::8], d["y_every8"], TOL32, TOL32, "y")
    check(S, d["sT"], TOL32, TOL32, "S_T")


def test_golden_initial_state_ragged_T():
    d = np.load(os.path.join(GOLD, "gdn_small.npz"))
    t = {k: torch.from_numpy(d[k]).cuda() for k in ("q", "k", "v", "beta", "la", "s0")}
    y, S = ops.gdn_prefill(t["q"], t["k"], t["v"], t["la"], beta=t["beta"], initial_state=t["s0"], output_final_state=True)
    check(y, d["y"], TOL32, TOL32, "y")
    check(S, d["sT"], TOL32, TOL32, "S_T")


def test_golden_nstep_write_vectors():
    d = np.load(os.path.join(GOLD, "nstep_small.npz"))
    t = {k: torch.from_numpy(d[k]).cuda() for k in ("q", "k", "v", "u", "la")}
    y, S = ops.gdn_prefill(t["q"], t["k"], t["v"], t["la"], u=t["u"], output_final_state=True)
    check(y, d["y"], TOL32, TOL32, "y")
    check(S, d["sT"], TOL32, TOL32, "S_T")


@pytest.mark.parametrize("DK,DV", [(32, 16), (64, 64), (128, 128), (256, 128), (128, 100)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_head_sizes(DK, DV, dtype):
    x = make_inputs(2, 37, 3, DK, DV, seed=DK + DV, dtype=dtype)
    s0 = torch.randn(2, 3, DV, DK, generator=torch.Generator().manual_seed(5)) * 0.3
    y_o, S_o = O.recurrence_c(*(np32(x[n]) for n in ("q", "k", "v", "la")), beta=np32(x["beta"]), s0=s0.numpy())
    g = dev(x)
    y, S = ops.gdn_prefill(g["q"], g["k"], g["v"], g["la"], beta=g["beta"], initial_state=s0.cuda(), output_final_state=True, out_dtype=torch.float32, impl="recurrent")
    check(y, y_o, TOL32, TOL32, "y")
    check(S, S_o, TOL32, TOL32, "S_T")


def test_strided_views_and_bf16_output():
    B, T, H, D = 2, 50, 2, 128
    x = make_inputs(B, T, H, D, D, seed=9, dtype=torch.bfloat16)
    # q/k/v as column slices of one fused projection, as the nsgdn layer produces them.
    fused = torch.cat([x["q"].reshape(B, T, -1), x["k"].reshape(B, T, -1), x["v"].reshape(B, T, -1)], -1).cuda()
    q, k, v = (fused[..., i * H * D : (i + 1) * H * D].view(B, T, H, D) for i in range(3))
    assert not q.is_contiguous()
    y, S = ops.gdn_prefill(q, k, v, x["la"].cuda(), beta=x["beta"].cuda(), output_final_state=True, impl="recurrent")
    assert y.dtype == torch.bfloat16
    y_o, S_o = O.recurrence_c(*(np32(x[n]) for n in ("q", "k", "v", "la")), beta=np32(x["beta"]))
    check(y, y_o, 2e-3, 4e-3, "y (bf16 output rounding)")
    check(S, S_o, TOL32, TOL32, "S_T")


def test_T0_copies_state_and_T1():
    x = dev(make_inputs(1, 1, 2, 64, 64, seed=1, dtype=torch.float32))
    s0 = torch.randn(1, 2, 64, 64, device="cuda")
    e = {n: x[n][:, :0] for n in ("q", "k", "v", "beta", "la")}
    _, S = ops.gdn_prefill(e["q"], e["k"], e["v"], e["la"], beta=e["beta"], initial_state=s0, output_final_state=True)
    assert torch.equal(S, s0)
    _, S = ops.gdn_prefill(e["q"], e["k"], e["v"], e["la"], beta=e["beta"], output_final_state=True)
    assert torch.count_nonzero(S) == 0
    y, S1 = ops.gdn_prefill(x["q"], x["k"], x["v"], x["la"], beta=x["beta"], initial_state=s0, output_final_state=True)
    y_o, S_o = O.recurrence(*(np32(x[n]) for n in ("q", "k", "v", "la")), beta=np32(x["beta"]), s0=np32(s0))
    check(y, y_o, TOL32, TOL32, "y")
    check(S1, S_o, TOL32, TOL32, "S")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("with_u", [False, True])
def test_decode_steps_against_oracle(dtype, with_u):
    B, H, D, steps = 4, 3, 128, 12
    x = make_inputs(B, steps, H, D, D, seed=77, dtype=dtype)
    S0 = torch.randn(B, H, D, D, generator=torch.Generator().manual_seed(8)) * 0.2
    u = (x["beta"][..., None] * x["k"].float()).to(dtype) if with_u else None
    y_o, S_o = O.recurrence(*(np32(x[n]) for n in ("q", "k", "v", "la")), beta=None if with_u else np32(x["beta"]), u=None if u is None else np32(u), s0=S0.numpy())
    g = dev(x)
    state = S0.cuda().contiguous()
    ys = []
    for t in range(steps):
        ys.append(ops.gdn_decode_step(g["q"][:, t], g["k"][:, t], g["v"][:, t], g["la"][:, t], state,
                                      beta=None if with_u else g["beta"][:, t], u=None if u is None else u[:, t].cuda(), out_dtype=torch.float32))
    y = torch.stack(ys, 1)
    check(y, y_o, TOL32, TOL32, "decode y")
    check(state, S_o, TOL32, TOL32, "decode state")


def test_decode_matches_prefill_state():
    B, T, H, D = 3, 20, 2, 128
    x = dev(make_inputs(B, T + 1, H, D, D, seed=4, dtype=torch.bfloat16))
    sl = lambda a, s: a[:, s]
    _, S = ops.gdn_prefill(*(sl(x[n], slice(0, T)) for n in ("q", "k", "v", "la")), beta=sl(x["beta"], slice(0, T)), output_final_state=True, impl="recurrent")
    y_d = ops.gdn_decode_step(*(x[n][:, T] for n in ("q", "k", "v", "la")), S, beta=x["beta"][:, T], out_dtype=torch.float32)
    y_p, S_p = ops.gdn_prefill(x["q"], x["k"], x["v"], x["la"], beta=x["beta"], output_final_state=True, out_dtype=torch.float32, impl="recurrent")
    torch.testing.assert_close(y_d, y_p[:, T], rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(S, S_p, rtol=1e-5, atol=1e-6)


def test_errors_raise():
    x = dev(make_inputs(1, 4, 1, 96, 64, seed=0, dtype=torch.float32))
    with pytest.raises(ops.GdnError):
        ops.gdn_prefill(x["q"], x["k"], x["v"], x["la"], beta=x["beta"])
