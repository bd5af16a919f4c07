"""The layer prologue and epilogue kernels against the PyTorch ops they replace.

Prologue: SiLU(short causal conv) of the projections computed in the projection dtype (F.conv1d,
F.silu), l2-normalised q (times DK^-1/2) and k, la = -softplus(a + dt_bias) exp(A_log) (clamped),
beta = sigmoid(b + b_bias) -- archbench/layers/nsgdn.py:457-470, 520-536 and the fla gdn mixer's
equivalents.  Epilogue: RMSNorm over DV times SiLU(g).  fp32 projections match to fp32 rounding;
bf16 projections to one bf16 rounding of the conv output (the summation order of the taps may
differ from cuDNN's), so those comparisons allow a few bf16 ulps."""

import pytest
import torch
import torch.nn.functional as F

from archbench_b200 import ops
from archbench_b200.layers import GatedDeltaNet, GDNCache, NStepGDN

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_grad():
    with torch.no_grad():
        yield


def torch_prologue(xq, xk, xv, xa, xb, A_log, dt_bias, H, DK, DV, b_bias=None, conv=None, state=None, q_scale=1.0,
                   l2_eps=1e-12, la_min=None, beta_scale=1.0):
    """The PyTorch path of the layers (conv in the projection dtype, then fp32)."""
    B, T, _ = xq.shape
    outs, new_state = [], []
    for i, x in enumerate((xq, xk, xv)):
        if conv is None:
            y = F.silu(x)
        else:
            w = conv[i].reshape(conv[i].shape[0], 1, -1).to(x.dtype)
            K = w.shape[-1]
            pre = state[i].to(x.dtype) if state is not None else x.new_zeros(B, x.shape[2], K - 1)
            xp = torch.cat([pre, x.transpose(1, 2)], -1)
            y = F.silu(F.conv1d(xp, w, None, groups=x.shape[2])).transpose(1, 2)
            new_state.append(xp[..., -(K - 1):])
        outs.append(y.float())
    q = F.normalize(outs[0].view(B, T, H, DK), dim=-1, eps=l2_eps) * q_scale
    k = F.normalize(outs[1].view(B, T, H, DK), dim=-1, eps=l2_eps)
    v = outs[2].view(B, T, H, DV)
    la = -F.softplus(xa.float() + dt_bias) * A_log.exp()
    if la_min is not None:
        la = la.clamp_min(la_min)
    beta = torch.sigmoid(xb.float() + (0.0 if b_bias is None else b_bias)) * beta_scale
    return q, k, v, la, beta, new_state


def make(B, T, H, DK, DV, dtype, conv_size=4, seed=0, fused_proj=True):
    g = torch.Generator(device="cuda").manual_seed(seed)
    r = lambda *s: torch.randn(*s, device="cuda", generator=g)
    if fused_proj:  # one projection, column slices as in NStepGDN (width padded to x8)
        width = (2 * H * DK + H * DV + 2 * H + 7) // 8 * 8
        proj = r(B, T, width).to(dtype)
        xq, xk, xv = proj[..., :H * DK], proj[..., H * DK:2 * H * DK], proj[..., 2 * H * DK:2 * H * DK + H * DV]
        o = 2 * H * DK + H * DV
        xa, xb = proj[..., o:o + H], proj[..., o + H:o + 2 * H]
    else:
        xq, xk, xv, xa, xb = r(B, T, H * DK).to(dtype), r(B, T, H * DK).to(dtype), r(B, T, H * DV).to(dtype), \
            r(B, T, H).to(dtype), r(B, T, H).to(dtype)
    conv = (r(H * DK, conv_size) * 0.5, r(H * DK, conv_size) * 0.5, r(H * DV, conv_size) * 0.5) if conv_size else None
    A_log, dt_bias, b_bias = r(H).abs().log1p(), r(H) * 0.5, r(H) * 0.5
    return xq, xk, xv, xa, xb, conv, A_log, dt_bias, b_bias


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("T", [1, 37, 100])
@pytest.mark.parametrize("flavor", ["nsgdn", "gdn"])
def test_prologue_matches_torch(dtype, T, flavor):
    B, H, DK = 2, 3, 128
    DV = 256 if flavor == "nsgdn" else 128
    xq, xk, xv, xa, xb, conv, A_log, dt_bias, b_bias = make(B, T, H, DK, DV, dtype, seed=T, fused_proj=flavor == "nsgdn")
    kw = dict(q_scale=DK**-0.5)
    if flavor == "nsgdn":
        kw.update(b_bias=b_bias, la_min=-3.0)
    else:
        kw.update(l2_eps=1e-6, beta_scale=2.0)
    state = tuple(torch.randn(B, c, 3, device="cuda").to(dtype) for c in (H * DK, H * DK, H * DV))
    got = ops.layer_prologue(xq, xk, xv, xa, xb, A_log, dt_bias, H=H, DK=DK, DV=DV, conv=conv, conv_state=state,
                             want_state=True, out_dtype=torch.float32, **kw)
    want = torch_prologue(xq, xk, xv, xa, xb, A_log, dt_bias, H, DK, DV, conv=conv, state=state, **kw)
    for name, a, b in zip("qkv", got[:3], want[:3]):
        if dtype == torch.float32:
            assert (a - b).abs().max().item() <= 1e-5 * max(1.0, b.abs().max().item()), name
        else:  # a bf16 conv output may round one ulp (2^-8 relative) apart
            assert ((a - b).abs() <= b.abs() * 2**-6 + 2e-3).all(), name
    assert torch.allclose(got[3], want[3], rtol=1e-5, atol=1e-6) and torch.allclose(got[4], want[4], rtol=1e-5, atol=1e-6)
    for a, b in zip(got[5], want[5]):
        assert torch.equal(a, b.contiguous())


def test_prologue_state_continues_a_sequence():
    """Two calls through the conv state give the one-call result exactly."""
    B, T, H, DK, DV = 2, 70, 2, 128, 256
    xq, xk, xv, xa, xb, conv, A_log, dt_bias, b_bias = make(B, T, H, DK, DV, torch.bfloat16, seed=5)
    sl = lambda t, a, b: t[:, a:b]
    full = ops.layer_prologue(xq, xk, xv, xa, xb, A_log, dt_bias, H=H, DK=DK, DV=DV, conv=conv, b_bias=b_bias)
    first = ops.layer_prologue(*(sl(t, 0, 33) for t in (xq, xk, xv, xa, xb)), A_log, dt_bias, H=H, DK=DK, DV=DV,
                               conv=conv, b_bias=b_bias, want_state=True)
    second = ops.layer_prologue(*(sl(t, 33, T) for t in (xq, xk, xv, xa, xb)), A_log, dt_bias, H=H, DK=DK, DV=DV,
                                conv=conv, b_bias=b_bias, conv_state=first[5])
    for i in range(5):
        assert torch.equal(torch.cat([first[i], second[i]], 1), full[i]), i


@pytest.mark.parametrize("ydt,gate,odt", [(torch.bfloat16, True, torch.bfloat16), (torch.float32, True, torch.float32),
                                           (torch.float32, False, torch.bfloat16)])
def test_epilogue_matches_torch(ydt, gate, odt):
    B, T, H, DV = 2, 45, 3, 256
    g_ = torch.Generator(device="cuda").manual_seed(9)
    y = torch.randn(B, T, H, DV, device="cuda", generator=g_).to(ydt)
    g = torch.randn(B, T, H * DV, device="cuda", generator=g_).to(torch.bfloat16) if gate else None
    w = torch.rand(DV, device="cuda", generator=g_) + 0.5
    got = ops.layer_epilogue(y, w, g, eps=1e-5, out_dtype=odt).float()
    yf = y.float()
    want = yf * torch.rsqrt(yf.square().mean(-1, keepdim=True) + 1e-5) * w
    if gate:
        want = want * F.silu(g.float().view(B, T, H, DV))
    want = want.reshape(B, T, H * DV)
    tol = 1e-5 if odt == torch.float32 else 8e-3
    assert ((got - want).abs() / (want.abs() + 1e-2)).max().item() < tol


def rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm()).item()


@pytest.mark.parametrize("cls", ["nsgdn", "gdn"])
@pytest.mark.parametrize("autocast", [False, True])
def test_layers_fused_match_torch_path(cls, autocast):
    torch.manual_seed(11)
    if cls == "nsgdn":
        m = NStepGDN(256, num_heads=2, head_dim=128, expand_v=2.0, n_steps=1, la_min=-4.0).cuda()
    else:
        m = GatedDeltaNet(hidden_size=256, expand_v=1, head_dim=128, num_heads=2, allow_neg_eigval=True).cuda()
    x = torch.randn(2, 100, 256, device="cuda")
    with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
        m.fused_io = True
        a = m(x)
        m.fused_io = False
        b = m(x)
    assert a.dtype == b.dtype
    assert rel(a, b) < (3e-2 if autocast else 2e-3), rel(a, b)


@pytest.mark.parametrize("cls", ["nsgdn", "gdn"])
def test_fused_cache_decode_equals_prefill(cls):
    torch.manual_seed(12)
    if cls == "nsgdn":
        m = NStepGDN(256, num_heads=2, head_dim=128, expand_v=2.0, n_steps=1).cuda()
    else:
        m = GatedDeltaNet(hidden_size=256, expand_v=1, head_dim=128, num_heads=2).cuda()
    x = torch.randn(2, 72, 256, device="cuda")
    full = m(x)
    cache = GDNCache()
    parts = [m(x[:, :64], cache=cache)] + [m(x[:, t:t + 1], cache=cache) for t in range(64, 72)]
    assert rel(torch.cat(parts, 1), full) < 5e-3


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("T,conv_size", [(1, 4), (37, 4), (100, 4), (64, 1)])
@pytest.mark.parametrize("n_steps,with_prev", [(2, False), (2, True), (3, True)])
def test_prologue_nstep_write_vectors(dtype, T, conv_size, n_steps, with_prev):
    """nsgdn write vectors u (archbench/layers/nsgdn.py:472-487): u = beta k, then n-1 corrections
    u -= lam beta (p.u) (p - (p.k) k) with p the previous token's normalised k (the previous call's
    last k for the first token, zero at the start of a sequence)."""
    from archbench_b200.nstep import write_direction
    B, H, DK, DV = 2, 3, 128, 256
    xq, xk, xv, xa, xb, conv, A_log, dt_bias, b_bias = make(B, T, H, DK, DV, dtype, conv_size=conv_size, seed=T + n_steps)
    if conv_size == 1:
        conv = None
    g_ = torch.Generator(device="cuda").manual_seed(17)
    lam = torch.rand(H, device="cuda", generator=g_) + 0.5
    kp = F.normalize(torch.randn(B, H, DK, device="cuda", generator=g_), dim=-1) if with_prev else None
    kw = dict(q_scale=DK**-0.5, b_bias=b_bias, la_min=-3.0)
    got = ops.layer_prologue(xq, xk, xv, xa, xb, A_log, dt_bias, H=H, DK=DK, DV=DV, conv=conv, want_state=True,
                             out_dtype=torch.float32, n_steps=n_steps, lam=lam, k_prev=kp, **kw)
    assert len(got) == 8
    want = torch_prologue(xq, xk, xv, xa, xb, A_log, dt_bias, H, DK, DV, conv=conv, **kw)
    k = want[1]
    p = torch.cat([(kp if kp is not None else torch.zeros_like(k[:, 0]))[:, None], k[:, :-1]], 1)
    u = write_direction(k, p, want[4], lam, n_steps)
    if dtype == torch.float32:
        assert (got[6] - u).abs().max().item() <= 1e-5, (got[6] - u).abs().max().item()
        assert (got[7] - k[:, -1]).abs().max().item() <= 1e-5
    else:  # k itself may differ by one bf16 rounding of the conv output
        assert rel(got[6], u) < 2e-2 and rel(got[7], k[:, -1]) < 2e-2


@pytest.mark.parametrize("expand_v", [1.0, 2.0])
@pytest.mark.parametrize("n_steps", [2, 3])
def test_nstep_layer_fused_matches_torch_path(expand_v, n_steps):
    torch.manual_seed(13)
    m = NStepGDN(256, num_heads=2, head_dim=128, expand_v=expand_v, n_steps=n_steps, la_min=-4.0).cuda()
    x = torch.randn(2, 100, 256, device="cuda")
    m.fused_io = True
    a = m(x)
    m.fused_io = False
    b = m(x)
    assert rel(a, b) < 2e-3, rel(a, b)


@pytest.mark.parametrize("fused_prefill,fused_decode", [(True, True), (True, False), (False, True)])
def test_nstep_cache_decode_equals_prefill(fused_prefill, fused_decode):
    """A prefill then token-by-token decode through the cache (conv state and the last k carried between
    calls) gives the one-call output; the fused and PyTorch paths share the cache layout."""
    torch.manual_seed(14)
    m = NStepGDN(256, num_heads=2, head_dim=128, expand_v=2.0, n_steps=2).cuda()
    x = torch.randn(2, 72, 256, device="cuda")
    m.fused_io = True
    full = m(x)
    cache = GDNCache()
    m.fused_io = fused_prefill
    parts = [m(x[:, :64], cache=cache)]
    m.fused_io = fused_decode
    parts += [m(x[:, t:t + 1], cache=cache) for t in range(64, 72)]
    assert rel(torch.cat(parts, 1), full) < 5e-3
