"""Parity of the chunked prefill backward (gdn_prefill_bwd) with the CPU oracle's backward.

The oracle (oracle.recurrence_bwd, float64) restates archbench's own backward of the recurrence and is
pinned to float64 autograd through archbench's nsgdn_ref (tests/test_oracle.py).  The kernels take
bf16 (or fp32) q/k/v and dy, run every product on fp16 tensor-core operands with fp32 accumulation and
return fp32 gradients; the oracle runs in float64 on the same bf16-rounded inputs.

Tolerance per gradient (dq, dk, du or dbeta, dv, dla, ds0): rel-L2 <= 2e-3 and max-abs <= 1e-2 of the
gradient's largest magnitude.
"""

import numpy as np
import pytest
import torch

from archbench_b200 import ops
from archbench_b200.workloads import make_inputs
from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL_REL, TOL_MAX_FRAC = 2e-3, 1e-2
D = 128


def np64(t):
    return t.detach().double().cpu().numpy()


def check(got, want, what):
    got = np64(got)
    mx, rel = O.errors(got, want)
    scale = float(np.abs(want).max(initial=0.0)) or 1.0
    assert rel <= TOL_REL and mx <= TOL_MAX_FRAC * scale, f"{what}: rel-L2 {rel:.3e} max-abs {mx:.3e} (max |ref| {scale:.3e})"
    return rel


def case(B, T, H, seed, s0=True, dsT=True, with_u=False, dy_scale=1.0, dy_dtype=torch.bfloat16, in_dtype=torch.bfloat16,
         DV=D):
    x = make_inputs(B, T, H, D, DV, seed=seed, dtype=in_dtype)
    g = torch.Generator().manual_seed(seed + 7)
    S0 = 0.3 * torch.randn(B, H, DV, D, generator=g) if s0 else None
    dS = torch.randn(B, H, DV, D, generator=g) * dy_scale if dsT else None
    dy = (torch.randn(B, T, H, DV, generator=g) * dy_scale).to(dy_dtype)
    u = None
    if with_u:
        u = torch.nn.functional.normalize(0.7 * x["k"].float() + 0.1 * torch.randn(B, T, H, D, generator=g), dim=-1)
        u = (u * x["beta"][..., None]).to(in_dtype)
    return x, S0, dS, dy, u


def run(x, S0, dS, dy, u):
    gpu = lambda t: None if t is None else t.cuda()
    grads = ops.gdn_prefill_bwd(gpu(x["q"]), gpu(x["k"]), gpu(x["v"]), gpu(x["la"]), gpu(dy),
                                beta=None if u is not None else gpu(x["beta"]), u=gpu(u), initial_state=gpu(S0),
                                ds_T=gpu(dS), want_ds0=True)
    torch.cuda.synchronize()
    want = O.recurrence_bwd(np64(x["q"]), np64(x["k"]), np64(x["v"]), np64(x["la"]), np64(dy),
                            beta=None if u is not None else np64(x["beta"]), u=None if u is None else np64(u),
                            s0=None if S0 is None else np64(S0), ds_T=None if dS is None else np64(dS))
    return grads, want


def check_all(grads, want, tag):
    rels = {}
    for n, w in want.items():
        rels[n] = check(grads[n], w, f"{tag} {n}")
    return rels


@pytest.mark.parametrize("T", [64, 1, 63, 100, 130, 192])
def test_backward_lengths(T):
    grads, want = run(*case(2, T, 2, seed=T))
    check_all(grads, want, f"T={T}")


def test_backward_without_states():
    grads, want = run(*case(2, 256, 2, seed=5, s0=False, dsT=False))
    check_all(grads, want, "no S0, no dS_T")


def test_backward_write_vector_given():
    grads, want = run(*case(1, 160, 3, seed=9, with_u=True))
    assert "du" in grads and "dbeta" not in grads
    check_all(grads, want, "u given")


@pytest.mark.parametrize("dy_scale", [1e-6, 1e3])
def test_backward_gradient_scale(dy_scale):
    """Tiny (bf16 training) and large incoming gradients keep their relative accuracy: the kernels
    scale (dy, dS_T) by a power of two per (b, h) before fp16 operands."""
    grads, want = run(*case(1, 128, 2, seed=11, dy_scale=dy_scale))
    check_all(grads, want, f"dy x {dy_scale:g}")


@pytest.mark.parametrize("with_u", [False, True])
def test_backward_wide_state(with_u):
    """DV = 256 (head_dim 128, expand_v 2 as in archbench's gdn and nsgdn configs): two 128-row state
    slices whose shared-input gradients add up."""
    grads, want = run(*case(1, 130, 2, seed=29, with_u=with_u, DV=256))
    check_all(grads, want, f"DV=256 u={with_u}")


def test_backward_fp32_inputs_and_dy():
    grads, want = run(*case(1, 96, 2, seed=13, dy_dtype=torch.float32, in_dtype=torch.float32))
    check_all(grads, want, "fp32 I/O")


@pytest.mark.parametrize("DV,with_u", [(D, False), (2 * D, False), (2 * D, True)])
def test_backward_deterministic(DV, with_u):
    """Bitwise the same gradients on a second call, also when a later 128-row state slice adds its part
    of dq, dk, du, dla and dbeta to the earlier slice's outputs."""
    x, S0, dS, dy, u = case(1, 192, 2, seed=17, DV=DV, with_u=with_u)
    a, _ = run(x, S0, dS, dy, u)
    b, _ = run(x, S0, dS, dy, u)
    for n in a:
        assert torch.equal(a[n], b[n]), n


def test_autograd_through_prefill_op():
    """torch.autograd through ops.gdn_prefill gives the backward kernels' gradients."""
    x, S0, dS, dy, _ = case(2, 130, 2, seed=19)
    q, k, v = (x[n].cuda().requires_grad_(True) for n in ("q", "k", "v"))
    la, beta = x["la"].cuda().requires_grad_(True), x["beta"].cuda().requires_grad_(True)
    s0 = S0.cuda().requires_grad_(True)
    y, S = ops.gdn_prefill(q, k, v, la, beta=beta, initial_state=s0, output_final_state=True)
    loss = (y.float() * dy.cuda().float()).sum() + (S * dS.cuda()).sum()
    gq, gk, gv, gla, gb, gs0 = torch.autograd.grad(loss, [q, k, v, la, beta, s0])
    assert gq.dtype == torch.bfloat16 and gla.dtype == torch.float32 and gs0.shape == s0.shape
    direct = ops.gdn_prefill_bwd(q.detach(), k.detach(), v.detach(), la.detach(), dy.cuda(), beta=beta.detach(),
                                 initial_state=s0.detach(), ds_T=dS.cuda(), want_ds0=True)
    # y is bf16, so autograd hands the kernels dy rounded to bf16: dy here is bf16 already.
    for got, n in ((gq, "dq"), (gk, "dk"), (gv, "dv"), (gla, "dla"), (gb, "dbeta"), (gs0, "ds0")):
        assert torch.equal(got.float(), direct[n].to(got.dtype).float()), n


def test_backward_configuration1_slice():
    """Full configuration-1 backward (B=8, T=4096, H=8); one (b, h) sequence against the oracle
    (every (b, h) is independent, so its gradients are those of the single-sequence problem)."""
    x = make_inputs(8, 4096, 8, D, D, seed=23, dtype=torch.bfloat16)
    dy = torch.randn(8, 4096, 8, D, generator=torch.Generator().manual_seed(24)).to(torch.bfloat16)
    gpu = {n: t.cuda() for n, t in x.items()}
    grads = ops.gdn_prefill_bwd(gpu["q"], gpu["k"], gpu["v"], gpu["la"], dy.cuda(), beta=gpu["beta"])
    torch.cuda.synchronize()
    b, h = 5, 3
    sl = lambda t: np64(t[b : b + 1, :, h : h + 1])
    want = O.recurrence_bwd(sl(x["q"]), sl(x["k"]), sl(x["v"]), sl(x["la"]), sl(dy), beta=sl(x["beta"]))
    for n in ("dq", "dk", "dv", "dla", "dbeta"):
        check(grads[n][b : b + 1, :, h : h + 1], want[n], f"cfg1 (b={b}, h={h}) {n}")
    for n, t in grads.items():
        assert torch.isfinite(t).all(), n


def _torch_recurrence(q, k, v, la, beta=None, u=None, initial_state=None, output_final_state=False, **kw):
    """float64 autograd reference of the scan (the per-token loop of nsgdn_ref) on the GPU."""
    qd, kd, vd = q.double(), k.double(), v.double()
    uu = (beta.double()[..., None] * kd) if u is None else u.double()
    B, T, H, DK = q.shape
    S = qd.new_zeros(B, H, v.shape[-1], DK) if initial_state is None else initial_state.double()
    ys = []
    for t in range(T):
        S = la[:, t].double().exp()[..., None, None] * S
        r = vd[:, t] - (S @ kd[:, t][..., None]).squeeze(-1)
        S = S + r[..., :, None] * uu[:, t][..., None, :]
        ys.append((S @ qd[:, t][..., None]).squeeze(-1))
    y = torch.stack(ys, 1).to(q.dtype)
    return y, (S.float() if output_final_state else None)


@pytest.mark.parametrize("layer", ["nsgdn1", "nsgdn2", "gdn", "nsgdn_ref_config", "gdn_ref_config"])
def test_layer_parameter_gradients(layer, monkeypatch):
    """A training step of the drop-in layers: parameter gradients through the CUDA backward against
    the same layer with its scan replaced by a float64 autograd recurrence."""
    from archbench_b200 import layers

    torch.manual_seed(0)
    if layer == "gdn":
        m = layers.GatedDeltaNet(hidden_size=256, expand_v=1, head_dim=128, num_heads=2).cuda()
    elif layer == "gdn_ref_config":  # archbench configs/arch/gdn.yaml: head_dim 128, expand_v 2
        m = layers.GatedDeltaNet(hidden_size=256, expand_v=2.0, head_dim=128, num_heads=2, use_gate=True, conv_size=4).cuda()
    elif layer == "nsgdn_ref_config":  # archbench configs/arch/nsgdn.yaml: head_dim 128, expand_v 2, n_steps 2
        m = layers.NStepGDN(256, num_heads=2, head_dim=128, expand_v=2.0, n_steps=2, lam=1.0, conv_size=4).cuda()
    else:
        m = layers.NStepGDN(256, num_heads=2, head_dim=128, expand_v=1.0, n_steps=1 if layer == "nsgdn1" else 2).cuda()
    x = torch.randn(2, 96, 256, device="cuda")
    m.fused_io = False  # the scan is the part under test: keep the rest on the PyTorch path

    def grads():
        m.zero_grad()
        y = m(x)
        (y.float().square().mean()).backward()
        return {n: p.grad.detach().clone() for n, p in m.named_parameters() if p.grad is not None}

    got = grads()
    monkeypatch.setattr(layers.ops, "gdn_prefill", _torch_recurrence)
    want = grads()
    assert set(got) == set(want) and len(got) >= 5
    for n in want:
        mx, rel = O.errors(np64(got[n]), np64(want[n]))
        assert rel <= 2e-2, f"{layer} {n}: rel-L2 {rel:.3e}"
