"""The drop-in mixers end to end on the GPU.

Each layer's forward is compared with the same layer computed on the CPU in float64 where the
token mixing is the oracle recurrence: the projections, short convolution, l2norm, gate and
norms follow archbench/layers/nsgdn.py:517-542 (nsgdn) and fla/layers/gated_deltanet.py:201-316
(gdn).  Decode through a cache must reproduce the prefill of the longer sequence."""

import copy

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from archbench_b200.layers import GatedDeltaNet, GDNCache, NStepGDN
from archbench_b200.nstep import write_direction
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _inference_mode():
    with torch.no_grad():
        yield


def conv_silu(x, w, bias=None):
    T = x.shape[1]
    y = F.conv1d(x.transpose(1, 2), w, bias, padding=w.shape[-1] - 1, groups=x.shape[2])
    return F.silu(y[..., :T].transpose(1, 2))


def scan64(q, k, v, la, beta=None, u=None):
    """Oracle token mixing on inputs rounded to bf16 exactly as the layer hands them to the kernel."""
    r = lambda t: t.detach().to(torch.bfloat16).double().numpy()
    y, _ = O.recurrence(r(q), r(k), r(v), la.detach().double().numpy(), beta=None if beta is None else beta.detach().double().numpy(),
                        u=None if u is None else r(u))
    return torch.from_numpy(y)


def nsgdn_cpu(m: NStepGDN, x):
    m = copy.deepcopy(m).double().cpu()
    x = x.double().cpu()
    B, T, _ = x.shape
    H, DK, DV = m.H, m.DK, m.DV
    n_qkv = 2 * m.qk_dim + m.v_dim
    proj = m.in_proj(x)
    qkv, g, ab = proj[..., :n_qkv], proj[..., n_qkv:n_qkv + m.n_gate], proj[..., n_qkv + m.n_gate:n_qkv + m.n_gate + 2 * H]
    qkv = conv_silu(qkv, m.conv.weight)
    q = F.normalize(qkv[..., :m.qk_dim].view(B, T, H, DK), dim=-1) * DK**-0.5
    k = F.normalize(qkv[..., m.qk_dim:2 * m.qk_dim].view(B, T, H, DK), dim=-1)
    v = qkv[..., 2 * m.qk_dim:].view(B, T, H, DV)
    la = -F.softplus(ab[..., :H] + m.dt_bias) * m.A_log.exp()
    beta = torch.sigmoid(ab[..., H:] + m.b_bias)
    if m.n_steps > 1:
        p = F.pad(k[:, :-1], (0, 0, 0, 0, 1, 0))
        y = scan64(q, k, v, la, u=write_direction(k, p, beta, F.softplus(m.lam), m.n_steps))
    else:
        y = scan64(q, k, v, la, beta=beta)
    y = m.norm(y)
    y = y * F.silu(g).view(B, T, H, DV)
    return m.o_proj(y.reshape(B, T, -1))


def rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return ((a - b).norm() / b.norm()).item()


@pytest.mark.parametrize("n_steps", [1, 2])
def test_nsgdn_forward_matches_cpu(n_steps):
    torch.manual_seed(0)
    m = NStepGDN(256, num_heads=2, head_dim=128, expand_v=1.0, n_steps=n_steps).cuda()
    x = torch.randn(2, 160, 256, device="cuda")
    y = m(x)
    want = nsgdn_cpu(m, x)
    assert y.shape == (2, 160, 256)
    assert rel(y, want) < 5e-3, rel(y, want)


def test_nsgdn_reference_yaml_keys_dv256():
    """configs/arch/nsgdn.yaml keys (expand_v 2.0 -> DV 256, n_steps 2) construct and run."""
    torch.manual_seed(1)
    m = NStepGDN(512, head_dim=128, expand_v=2.0, n_steps=2, lam=1.0, use_gate=True, use_short_conv=True, conv_size=4, num_heads=2).cuda()
    x = torch.randn(1, 96, 512, device="cuda")
    assert rel(m(x), nsgdn_cpu(m, x)) < 5e-3


def gdn_cpu(m: GatedDeltaNet, x):
    m = copy.deepcopy(m).double().cpu()
    x = x.double().cpu()
    B, T, _ = x.shape
    H, DK, DV = m.num_heads, m.head_k_dim, m.head_v_dim
    q = conv_silu(m.q_proj(x), m.q_conv1d.weight)
    k = conv_silu(m.k_proj(x), m.k_conv1d.weight)
    v = conv_silu(m.v_proj(x), m.v_conv1d.weight)
    q = F.normalize(q.view(B, T, H, DK), dim=-1, eps=1e-6) * DK**-0.5
    k = F.normalize(k.view(B, T, H, DK), dim=-1, eps=1e-6)
    beta = m.b_proj(x).sigmoid()
    la = -m.A_log.exp() * F.softplus(m.a_proj(x) + m.dt_bias)
    o = scan64(q, k, v.view(B, T, H, DV), la, beta=beta)
    g = m.g_proj(x).view(B, T, H, DV)
    o = o * torch.rsqrt(o.square().mean(-1, keepdim=True) + m.o_norm.eps) * m.o_norm.weight * F.silu(g)
    return m.o_proj(o.reshape(B, T, -1))


def test_gdn_forward_matches_cpu():
    torch.manual_seed(2)
    m = GatedDeltaNet(hidden_size=256, expand_v=1, head_dim=128, num_heads=2).cuda()
    x = torch.randn(2, 130, 256, device="cuda")
    assert rel(m(x), gdn_cpu(m, x)) < 5e-3


@pytest.mark.parametrize("cls", ["nsgdn", "gdn"])
def test_cache_decode_equals_prefill(cls):
    torch.manual_seed(3)
    if cls == "nsgdn":
        m = NStepGDN(256, num_heads=2, head_dim=128, expand_v=1.0, n_steps=2).cuda()
    else:
        m = GatedDeltaNet(hidden_size=256, expand_v=1, head_dim=128, num_heads=2).cuda()
    x = torch.randn(2, 80, 256, device="cuda")
    full = m(x)
    cache = GDNCache()
    parts = [m(x[:, :64], cache=cache)]
    for t in range(64, 80):
        parts.append(m(x[:, t:t + 1], cache=cache))
    got = torch.cat(parts, 1)
    assert cache.seen == 80
    assert rel(got, full) < 5e-3, rel(got, full)


def test_bf16_autocast_forward():
    torch.manual_seed(4)
    m = NStepGDN(256, num_heads=2, head_dim=128, expand_v=1.0, n_steps=1).cuda()
    x = torch.randn(2, 128, 256, device="cuda")
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = m(x)
    assert y.dtype == torch.bfloat16 and torch.isfinite(y).all()
    assert rel(y.float(), nsgdn_cpu(m, x)) < 3e-2
