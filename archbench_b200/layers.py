"""Drop-in gated-DeltaNet mixers running the token mixing on this package's CUDA kernels.

``NStepGDN``      -- archbench's ``nsgdn`` mixer (archbench/layers/nsgdn.py:473-542): same
                     constructor keywords, same parameter names and shapes, same maths.
``GatedDeltaNet`` -- the ``gdn`` mixer archbench takes from fla (fla/layers/gated_deltanet.py:
                     100-316 via archbench/layers/fla.py:36-38): same keywords and parameter
                     names (q/k/v/a/b/g_proj, q/k/v_conv1d, A_log, dt_bias, o_norm, o_proj).

Both keep ``forward(x) -> y`` (B, T, D) and add an optional ``cache`` argument (a
``GDNCache``) that carries the recurrent state and the short-convolution state between calls:
a call with a cache continues from it (prefill of any length, or one-token decode) and leaves
the updated state in it.  The projections are PyTorch GEMMs; the short convolution, the q/k
norms and the gates run as one CUDA kernel (``ops.layer_prologue``), the token mixing is
``ops.gdn_prefill`` / ``ops.gdn_decode_step``, and the output norm and gate one more kernel
(``ops.layer_epilogue``); the prologue kernel also computes nsgdn's n-step write vectors, and in
training ``gdn_write_vectors_bwd`` differentiates them (fp32 fallbacks for other head sizes use
PyTorch ops there).  ``fused_io = False`` on a module (or a configuration the kernels do not serve:
conv bias, odd head sizes) keeps those parts in PyTorch.  Calls that
build an autograd graph (training) run the prologue, scan and epilogue forward and backward on the
CUDA kernels (DK = 128; DV = DK or 2 DK for the fused prologue/epilogue, a multiple of 128 for the
scan); without a backward kernel for a configuration, those parts run in PyTorch.  There is no
CPU path.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops


@dataclass
class GDNCache:
    """Per-layer decode state: fp32 recurrent state (B, H, DV, DK) and the last conv_size-1
    inputs of each short convolution (B, channels, conv_size-1)."""

    state: Optional[torch.Tensor] = None
    conv: dict = field(default_factory=dict)
    seen: int = 0
    # A static cache keeps its tensors: decode steps overwrite the recurrent state and the conv
    # states in place, so a decode step captured in a CUDA graph reads and writes the same buffers
    # on every replay (decode.GraphDecoder).
    static: bool = False


def _put(cache: GDNCache, key: str, value: torch.Tensor) -> None:
    """Store a conv-state entry; a static cache overwrites the tensor it already holds."""
    old = cache.conv.get(key)
    if old is not None and old.shape == value.shape and old.data_ptr() == value.data_ptr():
        return  # written in place by the kernel
    if cache.static and old is not None and old.shape == value.shape:
        old.copy_(value)
    else:
        cache.conv[key] = value


class ShortConv(nn.Module):
    """Depthwise causal convolution + SiLU (archbench/layers/nsgdn.py:457-470).

    ``weight`` is (dim, 1, size) as in the reference.  With ``state`` (B, dim, size-1) the
    convolution continues a previous call; the new state is returned alongside."""

    def __init__(self, dim: int, size: int, bias: bool = False):
        super().__init__()
        self.size = size
        self.weight = nn.Parameter(torch.empty(dim, 1, size).uniform_(-1 / math.sqrt(size), 1 / math.sqrt(size)))
        self.bias = nn.Parameter(torch.zeros(dim)) if bias else None

    def forward(self, x: torch.Tensor, state: Optional[torch.Tensor] = None, want_state: bool = False):
        B, T, Dm = x.shape
        xt = x.transpose(1, 2)
        pre = state.to(x.dtype) if state is not None else x.new_zeros(B, Dm, self.size - 1)
        xp = torch.cat([pre, xt], -1)
        y = F.conv1d(xp, self.weight.to(x.dtype), None if self.bias is None else self.bias.to(x.dtype), groups=Dm)
        y = F.silu(y).transpose(1, 2)
        new_state = xp[..., -(self.size - 1):].contiguous() if want_state and self.size > 1 else None
        return y, new_state


def _scan_impl(name: str) -> str:
    """archbench's scan_impl values (nsgdn.py:52-58) mapped onto this package's kernels: the
    chunked tensor-core kernel for 'chunk'/'dplr', the fp32 recurrent kernel for 'triton'/'ref'."""
    if name in ("chunk", "dplr"):
        return "auto"
    if name in ("triton", "ref"):
        return "recurrent"
    raise ValueError(f"unknown scan_impl {name!r}")


def _fused_ok(DK: int, DV: int) -> bool:
    """Head sizes the layer prologue/epilogue kernels serve."""
    return DK in (64, 128, 256) and DV in (64, 128, 256, 512) and DK <= DV <= 2 * DK


def _training(x: torch.Tensor, m: nn.Module) -> bool:
    """True when this call builds an autograd graph (the scan, ``ops.gdn_prefill``, is always
    differentiable; the fused prologue/epilogue use their differentiable variants)."""
    return torch.is_grad_enabled() and (x.requires_grad or any(p.requires_grad for p in m.parameters()))


def _fused_allowed(x: torch.Tensor, m: nn.Module, cache, DK: int, DV: int, conv_size: int) -> bool:
    """The fused prologue/epilogue serve this call: always without autograd; with autograd (training)
    when their backward kernels serve the head sizes and no decode cache is carried."""
    if not _training(x, m):
        return True
    return cache is None and ops.layer_io_trainable(DK, DV, conv_size)


def _mix(q, k, v, la, beta, u, cache: Optional[GDNCache], impl: str):
    """Token mixing with an optional cache: prefill (T > 1 or no state) or one decode step."""
    B, T, H, DK = q.shape
    if cache is None:
        y, _ = ops.gdn_prefill(q, k, v, la, beta=beta, u=u, impl=impl)
        return y
    if cache.state is not None and T == 1:
        y = ops.gdn_decode_step(q[:, 0], k[:, 0], v[:, 0], la[:, 0], cache.state,
                                beta=None if beta is None else beta[:, 0], u=None if u is None else u[:, 0])
        return y[:, None]
    y, S = ops.gdn_prefill(q, k, v, la, beta=beta, u=u, initial_state=cache.state, output_final_state=True, impl=impl)
    cache.state = S
    return y


class NStepGDN(nn.Module):
    """archbench's N-step gated DeltaNet mixer (nsgdn.py:473-542) on the CUDA kernels."""

    def __init__(self, d_model: int, num_heads: int = 8, head_dim: int = 128, expand_v: float = 2.0, n_steps: int = 2,
                 lam: float = 1.0, use_gate: bool = True, use_short_conv: bool = True, conv_size: int = 4,
                 norm_eps: float = 1e-5, scan_impl: str = "chunk", la_min: float | None = None, layer_idx: int | None = None):
        super().__init__()
        DK, DV = head_dim, int(head_dim * expand_v)
        if DK & (DK - 1) or DV & (DV - 1):
            raise ValueError("head_dim and head_dim * expand_v must be powers of 2")
        if n_steps < 1:
            raise ValueError("n_steps must be >= 1")
        if lam <= 0:
            raise ValueError("lam must be > 0")
        self.H, self.DK, self.DV, self.n_steps = num_heads, DK, DV, n_steps
        self.qk_dim, self.v_dim = num_heads * DK, num_heads * DV
        self.use_gate = use_gate
        self.n_gate = self.v_dim if use_gate else 0
        width = 2 * self.qk_dim + self.v_dim + self.n_gate + 2 * num_heads
        self.in_proj = nn.Linear(d_model, (width + 7) // 8 * 8, bias=False)
        self.conv = ShortConv(2 * self.qk_dim + self.v_dim, conv_size) if use_short_conv else None
        self.A_log = nn.Parameter(torch.empty(num_heads).uniform_(1, 16).log())
        dt = torch.exp(torch.rand(num_heads) * (math.log(0.1) - math.log(0.001)) + math.log(0.001))
        self.dt_bias = nn.Parameter(dt + torch.log(-torch.expm1(-dt)))
        self.b_bias = nn.Parameter(torch.zeros(num_heads))
        self.lam = nn.Parameter(torch.full((num_heads,), math.log(math.expm1(lam))))
        self.norm = nn.RMSNorm(DV, eps=norm_eps)
        self.scan_impl = scan_impl
        self._impl = _scan_impl(scan_impl)
        self.la_min = la_min
        self.o_proj = nn.Linear(self.v_dim, d_model, bias=False)
        self.layer_idx = layer_idx
        self.fused_io = True

    @torch.compiler.disable  # ctypes kernel calls run eagerly; the compiled graph breaks around them
    def _forward_fused(self, x: torch.Tensor, proj: torch.Tensor, cache: Optional[GDNCache]) -> torch.Tensor:
        B, T, _ = x.shape
        H, DK, DV = self.H, self.DK, self.DV
        qd, n_qkv = self.qk_dim, 2 * self.qk_dim + self.v_dim
        ab0 = n_qkv + self.n_gate
        conv = state = None
        if self.conv is not None:
            w = self.conv.weight.reshape(n_qkv, -1)
            conv = (w[:qd], w[qd:2 * qd], w[2 * qd:])
            st = cache.conv.get("qkv") if cache is not None else None
            if st is not None:
                state = (st[:, :qd], st[:, qd:2 * qd], st[:, 2 * qd:])
        dt = torch.bfloat16 if (DK == 128 and self._impl != "recurrent") else torch.float32
        parts = (proj[..., :qd], proj[..., qd:2 * qd], proj[..., 2 * qd:n_qkv], proj[..., ab0:ab0 + H], proj[..., ab0 + H:ab0 + 2 * H])
        train = _training(x, self)
        if train and dt == torch.bfloat16:
            # the whole mixer as one autograd node: the projection's gradient is written once
            cw = None if self.conv is None else self.conv.weight.reshape(n_qkv, -1).float()
            o = ops.NsgdnMixerTrain.apply(proj, cw, self.A_log, self.dt_bias, self.b_bias, self.norm.weight,
                                          F.softplus(self.lam.float()),
                                          (H, DK, DV, self.n_gate, DK**-0.5, self.la_min, self.norm.eps, self._impl, self.n_steps))
            return self.o_proj(o)
        u = None
        if train:
            q, k, v, la, beta = ops.layer_prologue_train(*parts, self.A_log, self.dt_bias, H=H, DK=DK, DV=DV, b_bias=self.b_bias,
                                                         conv=conv, q_scale=DK**-0.5, la_min=self.la_min, out_dtype=dt)
            new_state = None
            if self.n_steps > 1:  # write vectors through autograd (no cache in training: zero before token 0)
                from .nstep import write_direction

                kf = k.float()
                p = F.pad(kf[:, :-1], (0, 0, 0, 0, 1, 0))
                u = write_direction(kf, p, beta, F.softplus(self.lam.float()), self.n_steps).to(dt)
        elif self.n_steps > 1:  # n-step write vectors computed by the prologue kernel
            kp = cache.conv.get("k_prev") if cache is not None else None
            q, k, v, la, beta, new_state, u, k_last = ops.layer_prologue(
                *parts, self.A_log, self.dt_bias, H=H, DK=DK, DV=DV, b_bias=self.b_bias, conv=conv, conv_state=state,
                want_state=cache is not None, q_scale=DK**-0.5, la_min=self.la_min, out_dtype=dt, n_steps=self.n_steps,
                lam=ops._cached(self.lam, "softplus", lambda t: F.softplus(t.float())),
                k_prev=None if kp is None else kp.reshape(B, H, DK), in_place=cache is not None and cache.static)
            if cache is not None:
                _put(cache, "k_prev", k_last.reshape(B, 1, H, DK))
        else:
            q, k, v, la, beta, new_state = ops.layer_prologue(
                *parts, self.A_log, self.dt_bias, H=H, DK=DK, DV=DV, b_bias=self.b_bias, conv=conv, conv_state=state,
                want_state=cache is not None, q_scale=DK**-0.5, la_min=self.la_min, out_dtype=dt,
                in_place=cache is not None and cache.static)
        if cache is not None and new_state is not None and not (state is not None and new_state[0] is state[0]):
            _put(cache, "qkv", torch.cat(new_state, 1))
        y = _mix(q, k, v, la, None if u is not None else beta, u, cache, self._impl)
        if cache is not None:
            cache.seen += T
        g = proj[..., n_qkv:n_qkv + self.n_gate] if self.use_gate else None
        epi = ops.layer_epilogue_train if train else ops.layer_epilogue
        o = epi(y, self.norm.weight, g, eps=self.norm.eps, out_dtype=x.dtype)
        return self.o_proj(o)

    bound_cache: Optional[GDNCache] = None  # used when called without a cache (decode.bind_caches)

    def forward(self, x: torch.Tensor, cache: Optional[GDNCache] = None) -> torch.Tensor:
        if cache is None:
            cache = self.bound_cache
        B, T, _ = x.shape
        H, DK, DV = self.H, self.DK, self.DV
        n_qkv = 2 * self.qk_dim + self.v_dim
        proj = self.in_proj(x)
        if (self.fused_io and _fused_ok(DK, DV) and proj.dtype in (torch.bfloat16, torch.float32)
                and (self.conv is None or (self.conv.bias is None and self.conv.size <= 4))
                and self.n_steps <= 8
                and _fused_allowed(x, self, cache, DK, DV, self.conv.size if self.conv is not None else 1)):
            return self._forward_fused(x, proj, cache)
        qkv, g, ab = proj[..., :n_qkv], proj[..., n_qkv:n_qkv + self.n_gate], proj[..., n_qkv + self.n_gate:n_qkv + self.n_gate + 2 * H]
        if self.conv is not None:
            qkv, st = self.conv(qkv, None if cache is None else cache.conv.get("qkv"), want_state=cache is not None)
            if cache is not None:
                _put(cache, "qkv", st)
        with torch.autocast(x.device.type, enabled=False):
            qkv = qkv.float()
            q = F.normalize(qkv[..., :self.qk_dim].view(B, T, H, DK), dim=-1) * DK**-0.5
            k = F.normalize(qkv[..., self.qk_dim:2 * self.qk_dim].view(B, T, H, DK), dim=-1)
            v = qkv[..., 2 * self.qk_dim:].view(B, T, H, DV)
            ab = ab.float()
            la = -F.softplus(ab[..., :H] + self.dt_bias) * self.A_log.exp()
            if self.la_min is not None:
                la = la.clamp_min(self.la_min)
            beta = torch.sigmoid(ab[..., H:] + self.b_bias)
            u = None
            if self.n_steps > 1:
                from .nstep import write_direction

                prev = cache.conv.get("k_prev") if cache is not None else None
                p = torch.cat([prev if prev is not None else torch.zeros_like(k[:, :1]), k[:, :-1]], 1)
                u = write_direction(k, p, beta, F.softplus(self.lam.float()), self.n_steps)
                if cache is not None:
                    _put(cache, "k_prev", k[:, -1:].detach())
            dt = torch.bfloat16 if (DK == 128 and self._impl != "recurrent") else torch.float32
            y = _mix(q.to(dt), k.to(dt), v.to(dt), la, None if u is not None else beta, None if u is None else u.to(dt), cache, self._impl)
        if cache is not None:
            cache.seen += T
        y = self.norm(y.to(x.dtype))
        if self.use_gate:
            y = y * F.silu(g).view(B, T, H, DV)
        return self.o_proj(y.reshape(B, T, -1))


class FusedRMSNormGated(nn.Module):
    """RMSNorm over the head dimension times SiLU(gate) (fla's FusedRMSNormGated semantics,
    swish activation): o = x / rms(x) * weight * g * sigmoid(g)."""

    def __init__(self, hidden: int, eps: float = 1e-5):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden))
        self.eps = eps

    def forward(self, x, g=None):
        xf = x.float()
        y = xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + self.eps) * self.weight.float()
        if g is not None:
            y = y * F.silu(g.float())
        return y.to(x.dtype)


class GatedDeltaNet(nn.Module):
    """The ``gdn`` mixer (fla's GatedDeltaNet, fla/layers/gated_deltanet.py:100-316) on the
    CUDA kernels.  Keyword set and parameter names follow fla so state dicts interchange."""

    def __init__(self, hidden_size: int = 2048, expand_v: float = 2, head_dim: int = 256, num_heads: int = 6,
                 num_v_heads: int | None = None, mode: str = "chunk", use_gate: bool = True, use_short_conv: bool = True,
                 allow_neg_eigval: bool = False, conv_size: int = 4, conv_bias: bool = False, layer_idx: int | None = None,
                 norm_eps: float = 1e-5, **kwargs):
        super().__init__()
        if mode not in ("chunk", "fused_recurrent"):
            raise ValueError(f"Not supported mode `{mode}`.")
        self.mode = mode
        self.allow_neg_eigval = allow_neg_eigval
        self.hidden_size = hidden_size
        self.expand_v = expand_v
        self.use_gate, self.use_short_conv, self.conv_size, self.conv_bias = use_gate, use_short_conv, conv_size, conv_bias
        self.head_dim, self.num_heads = head_dim, num_heads
        self.num_v_heads = num_v_heads if num_v_heads is not None else num_heads
        if self.num_v_heads != self.num_heads:
            raise ValueError("num_v_heads != num_heads (grouped value heads) is not supported by this build")
        self.head_k_dim = head_dim
        self.head_v_dim = int(head_dim * expand_v)
        self.key_dim = num_heads * self.head_k_dim
        self.value_dim = self.num_v_heads * self.head_v_dim
        self.layer_idx = layer_idx
        if not math.isclose(head_dim * expand_v, self.head_v_dim, rel_tol=1e-5):
            raise ValueError(f"expand_v={expand_v} does not give an integer head_v_dim")
        self.q_proj = nn.Linear(hidden_size, self.key_dim, bias=False)
        self.k_proj = nn.Linear(hidden_size, self.key_dim, bias=False)
        self.v_proj = nn.Linear(hidden_size, self.value_dim, bias=False)
        self.a_proj = nn.Linear(hidden_size, self.num_v_heads, bias=False)
        self.b_proj = nn.Linear(hidden_size, self.num_v_heads, bias=False)
        self.A_log = nn.Parameter(torch.log(torch.empty(self.num_v_heads).uniform_(0, 16)))
        dt = torch.exp(torch.rand(self.num_v_heads) * (math.log(0.1) - math.log(0.001)) + math.log(0.001)).clamp(min=1e-4)
        self.dt_bias = nn.Parameter(dt + torch.log(-torch.expm1(-dt)))
        if use_short_conv:
            self.q_conv1d = ShortConv(self.key_dim, conv_size, conv_bias)
            self.k_conv1d = ShortConv(self.key_dim, conv_size, conv_bias)
            self.v_conv1d = ShortConv(self.value_dim, conv_size, conv_bias)
        if use_gate:
            self.g_proj = nn.Linear(hidden_size, self.value_dim, bias=False)
        self.o_norm = FusedRMSNormGated(self.head_v_dim, eps=norm_eps)
        self.o_proj = nn.Linear(self.value_dim, hidden_size, bias=False)
        self.fused_io = True

    @torch.compiler.disable  # ctypes kernel calls run eagerly; the compiled graph breaks around them
    def _forward_fused(self, x: torch.Tensor, cache: Optional[GDNCache]) -> torch.Tensor:
        B, T, _ = x.shape
        H, DK, DV = self.num_heads, self.head_k_dim, self.head_v_dim
        conv = state = None
        if self.use_short_conv:
            conv = (self.q_conv1d.weight, self.k_conv1d.weight, self.v_conv1d.weight)
            if cache is not None and cache.conv.get("q") is not None:
                state = (cache.conv["q"], cache.conv["k"], cache.conv["v"])
        dt = torch.bfloat16 if DK == 128 else torch.float32
        train = _training(x, self)
        g = None
        if train:
            xq, xk, xv, xa, xb = self.q_proj(x), self.k_proj(x), self.v_proj(x), self.a_proj(x), self.b_proj(x)
        else:  # one GEMM for all six projections (their weights concatenated once, kept while unchanged)
            proj = F.linear(x, self._projection_weight())
            kd, vd, nh = self.key_dim, self.value_dim, self.num_v_heads
            xq, xk, xv = proj[..., :kd], proj[..., kd:2 * kd], proj[..., 2 * kd:2 * kd + vd]
            o0 = 2 * kd + vd
            if self.use_gate:
                g, o0 = proj[..., o0:o0 + vd], o0 + vd
            xa, xb = proj[..., o0:o0 + nh], proj[..., o0 + nh:o0 + 2 * nh]
        if train:
            q, k, v, la, beta = ops.layer_prologue_train(
                xq, xk, xv, xa.to(xq.dtype), xb.to(xq.dtype), self.A_log, self.dt_bias, H=H, DK=DK, DV=DV, conv=conv,
                q_scale=DK**-0.5, l2_eps=1e-6, beta_scale=2.0 if self.allow_neg_eigval else 1.0, out_dtype=dt)
            new_state = None
        else:
            q, k, v, la, beta, new_state = ops.layer_prologue(
                xq, xk, xv, xa.to(xq.dtype), xb.to(xq.dtype), self.A_log, self.dt_bias, H=H, DK=DK, DV=DV, conv=conv,
                conv_state=state, want_state=cache is not None, q_scale=DK**-0.5, l2_eps=1e-6,
                beta_scale=2.0 if self.allow_neg_eigval else 1.0, out_dtype=dt, in_place=cache is not None and cache.static)
        if cache is not None and new_state is not None:
            for key, st in zip("qkv", new_state):
                _put(cache, key, st)
        o = _mix(q, k, v, la, beta, None, cache, "auto")
        if cache is not None:
            cache.seen += T
        if train and self.use_gate:
            g = self.g_proj(x)
        epi = ops.layer_epilogue_train if train else ops.layer_epilogue
        o = epi(o, self.o_norm.weight, g, eps=self.o_norm.eps, out_dtype=x.dtype)
        return self.o_proj(o)

    bound_cache: Optional[GDNCache] = None  # used when called without a cache (decode.bind_caches)

    def _projection_weight(self) -> torch.Tensor:
        """[q; k; v; g; a; b] projection weights in one matrix, rebuilt when any of them changes."""
        ws = [self.q_proj.weight, self.k_proj.weight, self.v_proj.weight]
        ws += [self.g_proj.weight] if self.use_gate else []
        ws += [self.a_proj.weight, self.b_proj.weight]
        key = tuple((w.data_ptr(), w._version, w.dtype, w.device) for w in ws)
        hit = getattr(self, "_proj_cat", None)
        if hit is None or hit[0] != key:
            with torch.no_grad():
                hit = (key, torch.cat(ws, 0))
            self._proj_cat = hit
        return hit[1]

    def forward(self, hidden_states: torch.Tensor, cache: Optional[GDNCache] = None, **kwargs) -> torch.Tensor:
        if cache is None:
            cache = self.bound_cache
        x = hidden_states
        B, T, _ = x.shape
        want = cache is not None
        if (self.fused_io and _fused_ok(self.head_k_dim, self.head_v_dim) and not self.conv_bias and self.conv_size <= 4
                and self.q_proj.weight.dtype in (torch.bfloat16, torch.float32)
                and _fused_allowed(x, self, cache, self.head_k_dim, self.head_v_dim, self.conv_size if self.use_short_conv else 1)):
            return self._forward_fused(x, cache)
        if self.use_short_conv:
            q, sq = self.q_conv1d(self.q_proj(x), None if cache is None else cache.conv.get("q"), want)
            k, sk = self.k_conv1d(self.k_proj(x), None if cache is None else cache.conv.get("k"), want)
            v, sv = self.v_conv1d(self.v_proj(x), None if cache is None else cache.conv.get("v"), want)
            if want:
                for key, st in zip("qkv", (sq, sk, sv)):
                    _put(cache, key, st)
        else:
            q, k, v = F.silu(self.q_proj(x)), F.silu(self.k_proj(x)), F.silu(self.v_proj(x))
        H, DK, DV = self.num_heads, self.head_k_dim, self.head_v_dim
        with torch.autocast(x.device.type, enabled=False):
            # fla normalises q, k inside its kernel (use_qk_l2norm_in_kernel) and scales q by
            # DK^-1/2 (its default scale); the gate is -exp(A_log) softplus(a + dt_bias)
            # (fla/ops/gated_delta_rule/gate.py:naive_gdn_gate).
            qf = F.normalize(q.float().view(B, T, H, DK), dim=-1, eps=1e-6) * DK**-0.5
            kf = F.normalize(k.float().view(B, T, H, DK), dim=-1, eps=1e-6)
            vf = v.float().view(B, T, H, DV)
            beta = self.b_proj(x).float().sigmoid()
            if self.allow_neg_eigval:
                beta = beta * 2.0
            la = -self.A_log.float().exp() * F.softplus(self.a_proj(x).float() + self.dt_bias.float())
            dt = torch.bfloat16 if DK == 128 else torch.float32
            o = _mix(qf.to(dt), kf.to(dt), vf.to(dt), la, beta, None, cache, "auto")
        if cache is not None:
            cache.seen += T
        if self.use_gate:
            o = self.o_norm(o.to(x.dtype), self.g_proj(x).view(B, T, H, DV))
        else:
            o = self.o_norm(o.to(x.dtype))
        return self.o_proj(o.reshape(B, T, -1))
