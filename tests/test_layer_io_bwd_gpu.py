"""Backward of the layer prologue and epilogue kernels against autograd through the PyTorch ops they
replace (the layers' PyTorch path: conv in the projection dtype, norms and gates in fp32).

Tolerance: fp32 projections rel-L2 <= 1e-4 per gradient (fast exp/divide in the kernels); bf16
projections rel-L2 <= 2e-2 (the PyTorch path rounds the conv output and its gradients to bf16, the
kernels keep fp32 from the bf16 inputs).  Layer level: parameter gradients of the fused training path
against the same layer on its PyTorch path, rel-L2 <= 2e-2."""

import pytest
import torch
import torch.nn.functional as F

from archbench_b200 import ops
from archbench_b200.layers import GatedDeltaNet, NStepGDN
from test_layer_io_gpu import make, rel, torch_prologue

pytestmark = pytest.mark.gpu


def cotangents(outs, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(o.shape, device="cuda", generator=g) for o in outs]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("T,conv_size", [(37, 4), (100, 4), (64, 1), (20, 3)])
@pytest.mark.parametrize("DV", [128, 256])
def test_prologue_backward_matches_torch(dtype, T, conv_size, DV):
    B, H, DK = 2, 2, 128
    xq, xk, xv, xa, xb, conv, A_log, dt_bias, b_bias = make(B, T, H, DK, DV, dtype, conv_size=conv_size, seed=T + DV,
                                                            fused_proj=False)
    if conv_size == 1:
        conv = None
    la_min = -1.0
    grads = []
    for impl in ("cuda", "torch"):
        leaves = [t.detach().clone().requires_grad_(True) for t in (xq, xk, xv, xa, xb, A_log, dt_bias, b_bias)]
        cw = None if conv is None else [w.detach().clone().requires_grad_(True) for w in conv]
        lq, lk, lv, la_, lb, lA, ldt, lbb = leaves
        if impl == "cuda":
            outs = ops.layer_prologue_train(lq, lk, lv, la_, lb, lA, ldt, H=H, DK=DK, DV=DV, b_bias=lbb, conv=cw,
                                            q_scale=DK**-0.5, la_min=la_min, out_dtype=torch.float32)
        else:
            outs = torch_prologue(lq, lk, lv, la_, lb, lA, ldt, H, DK, DV, b_bias=lbb, conv=cw, q_scale=DK**-0.5,
                                  la_min=la_min)[:5]
        loss = sum((o.float() * c).sum() for o, c in zip(outs, cotangents(outs, 5)))
        params = leaves + ([] if cw is None else cw)
        grads.append(torch.autograd.grad(loss, params))
    names = ["xq", "xk", "xv", "xa", "xb", "A_log", "dt_bias", "b_bias", "wq", "wk", "wv"]
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    for n, got, want in zip(names, grads[0], grads[1]):
        r = rel(got.float(), want.float())
        assert r <= tol, f"{n}: rel-L2 {r:.3e}"


@pytest.mark.parametrize("ydt,gate", [(torch.float32, True), (torch.bfloat16, True), (torch.float32, False)])
def test_epilogue_backward_matches_torch(ydt, gate):
    B, T, H, DV = 2, 45, 3, 256
    g_ = torch.Generator(device="cuda").manual_seed(9)
    y0 = torch.randn(B, T, H, DV, device="cuda", generator=g_).to(ydt)
    g0 = torch.randn(B, T, H * DV, device="cuda", generator=g_).to(ydt) if gate else None
    w0 = torch.rand(DV, device="cuda", generator=g_) + 0.5
    do = torch.randn(B, T, H * DV, device="cuda", generator=g_)
    res = []
    for impl in ("cuda", "torch"):
        y, w = y0.clone().requires_grad_(True), w0.clone().requires_grad_(True)
        g = None if g0 is None else g0.clone().requires_grad_(True)
        if impl == "cuda":
            o = ops.layer_epilogue_train(y, w, g, eps=1e-5, out_dtype=torch.float32)
        else:
            yf = y.float()
            o = yf * torch.rsqrt(yf.square().mean(-1, keepdim=True) + 1e-5) * w
            if gate:
                o = o * F.silu(g.float().view(B, T, H, DV))
            o = o.reshape(B, T, H * DV)
        params = [y, w] + ([g] if gate else [])
        res.append(torch.autograd.grad((o.float() * do).sum(), params))
    tol = 1e-4 if ydt == torch.float32 else 2e-2
    for n, got, want in zip(["y", "weight", "g"], res[0], res[1]):
        r = rel(got.float(), want.float())
        assert r <= tol, f"{n}: rel-L2 {r:.3e}"


@pytest.mark.parametrize("cls,expand_v,n_steps", [("nsgdn", 1.0, 1), ("nsgdn", 2.0, 1), ("nsgdn", 2.0, 2), ("nsgdn", 1.0, 3), ("nsgdn", 2.0, 8),
                                                   ("gdn", 1.0, 1), ("gdn", 2.0, 1)])
def test_layer_training_fused_matches_torch_path(cls, expand_v, n_steps):
    """Parameter gradients of a training step on the fused kernels (prologue, scan, epilogue forward and
    backward; nsgdn's n-step write vectors through autograd between prologue and scan) against the
    same layer with its prologue/epilogue in PyTorch."""
    torch.manual_seed(3)
    if cls == "nsgdn":
        m = NStepGDN(256, num_heads=2, head_dim=128, expand_v=expand_v, n_steps=n_steps).cuda()
    else:
        m = GatedDeltaNet(hidden_size=256, expand_v=expand_v, head_dim=128, num_heads=2).cuda()
    x = torch.randn(2, 100, 256, device="cuda")

    def grads(fused):
        m.fused_io = fused
        m.zero_grad()
        m(x).float().square().mean().backward()
        return {n: p.grad.detach().clone() for n, p in m.named_parameters() if p.grad is not None}

    got, want = grads(True), grads(False)
    assert set(got) == set(want) and len(got) >= 6
    for n in want:
        r = rel(got[n], want[n])
        assert r <= 2e-2, f"{cls} expand_v={expand_v} n_steps={n_steps} {n}: rel-L2 {r:.3e}"


@pytest.mark.parametrize("kdt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("T,n_steps,DK", [(37, 2, 128), (100, 3, 128), (16, 5, 128), (64, 2, 64), (1, 2, 128)])
def test_write_vectors_backward_matches_autograd(kdt, T, n_steps, DK):
    """gdn_write_vectors_bwd against autograd through write_direction (archbench/layers/nsgdn.py:61-75)
    on the same (possibly bf16-rounded) keys: dk (own and successor's share), dbeta, dlam to fp32
    rounding (rel-L2 <= 1e-5)."""
    from archbench_b200.nstep import write_direction

    B, H = 2, 3
    g_ = torch.Generator(device="cuda").manual_seed(T * 7 + n_steps)
    k = F.normalize(torch.randn(B, T, H, DK, device="cuda", generator=g_), dim=-1).to(kdt)
    beta = torch.rand(B, T, H, device="cuda", generator=g_)
    lam = torch.rand(H, device="cuda", generator=g_) + 0.5
    du = torch.randn(B, T, H, DK, device="cuda", generator=g_)
    dk0 = torch.randn(B, T, H, DK, device="cuda", generator=g_)
    kr, br, lr = (t.float().clone().requires_grad_(True) for t in (k, beta, lam))
    p = F.pad(kr[:, :-1], (0, 0, 0, 0, 1, 0))
    dk_w, db_w, dl_w = torch.autograd.grad(write_direction(kr, p, br, lr, n_steps), (kr, br, lr), du)
    dk = dk0.clone()
    dbeta, dlam = ops.write_vectors_bwd(k, beta, lam, du, dk, n_steps)
    for n, got, want in (("dk", dk, dk0 + dk_w), ("dbeta", dbeta, db_w), ("dlam", dlam, dl_w)):
        if want.abs().max().item() == 0.0:  # T = 1: no previous key, so lam has no effect
            assert got.abs().max().item() == 0.0, n
            continue
        r = rel(got, want)
        assert r <= 1e-5, f"{n}: rel-L2 {r:.3e}"
