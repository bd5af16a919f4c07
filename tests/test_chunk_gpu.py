"""Parity of the chunked tcgen05/TMEM prefill kernel with the CPU oracle.

Tolerance (north-star, bf16 I/O with fp32 state): max-abs <= 2e-3 and rel-L2 <= 1e-3 on y and
on the final state, measured on fp32 outputs against the float64 oracle run on the same
bf16-rounded inputs.  A bf16 output adds its own rounding (rel-L2 ~1.7e-3 for a perfect
result), so bf16 outputs are held to max-abs <= 2e-3 and rel-L2 <= 3e-3."""

import numpy as np
import pytest
import torch

from archbench_b200 import ops
from archbench_b200.workloads import make_inputs
from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL_MAX, TOL_REL = 2e-3, 1e-3
TOL_REL_BF16_OUT = 3e-3
# The chunk kernels: a two-CTA cluster per sequence (DV = 128, u = beta k), one CTA per sequence
# and 128-row state slice, and the split path (every chunk's products in one parallel pass, then
# one state-only CTA per sequence and state slice).
VARIANTS = ["chunk_cluster", "chunk_single", "chunk_split"]


def np32(t):
    return t.detach().float().cpu().numpy()


def check(got, want, what, tol_max=TOL_MAX, tol_rel=TOL_REL):
    mx, rel = O.errors(np32(got), want)
    assert mx <= tol_max and rel <= tol_rel, f"{what}: max-abs {mx:.3e} rel-L2 {rel:.3e}"
    return mx, rel


def run_case(B, T, H, seed=0, s0=False, with_u=False, out_dtype=torch.float32, impl="chunk"):
    x = make_inputs(B, T, H, 128, 128, seed=seed, dtype=torch.bfloat16)
    S0 = (torch.randn(B, H, 128, 128, generator=torch.Generator().manual_seed(seed + 1)) * 0.3) if s0 else None
    u = (x["beta"][..., None] * x["k"].float()).to(torch.bfloat16) if with_u else None
    y_o, S_o = O.recurrence_c(*(np32(x[n]) for n in ("q", "k", "v", "la")),
                              beta=None if with_u else np32(x["beta"]), u=None if u is None else np32(u),
                              s0=None if S0 is None else S0.numpy())
    g = {k: v.cuda() for k, v in x.items()}
    y, S = ops.gdn_prefill(g["q"], g["k"], g["v"], g["la"], beta=None if with_u else g["beta"],
                           u=None if u is None else u.cuda(), initial_state=None if S0 is None else S0.cuda(),
                           output_final_state=True, out_dtype=out_dtype, impl=impl)
    torch.cuda.synchronize()
    return y, S, y_o, S_o


def test_chunk_kernel_is_selected():
    x = make_inputs(1, 64, 1, 128, 128, dtype=torch.bfloat16)
    g = {k: v.cuda() for k, v in x.items()}
    assert ops.selected_impl(g["q"], g["k"], g["v"], g["la"], beta=g["beta"]) == "chunk_cluster"
    assert ops.selected_impl(g["q"], g["k"], g["v"], g["la"], beta=g["beta"], impl="chunk_single") == "chunk_single"


@pytest.mark.parametrize("impl", VARIANTS)
@pytest.mark.parametrize("T", [64, 192, 1, 63, 65, 100, 130])
def test_lengths(T, impl):
    y, S, y_o, S_o = run_case(2, T, 2, seed=T, impl=impl)
    check(y, y_o, f"y T={T}")
    check(S, S_o, f"S_T T={T}")
    assert ops.device_status() == 0


@pytest.mark.parametrize("impl", VARIANTS)
def test_initial_state(impl):
    y, S, y_o, S_o = run_case(1, 256, 3, seed=5, s0=True, impl=impl)
    check(y, y_o, "y")
    check(S, S_o, "S_T")


@pytest.mark.parametrize("impl", ["chunk", "chunk_split"])
def test_write_vector_given(impl):
    y, S, y_o, S_o = run_case(2, 160, 2, seed=6, with_u=True, impl=impl)
    check(y, y_o, "y (u given)")
    check(S, S_o, "S_T (u given)")


@pytest.mark.parametrize("impl", ["chunk", "chunk_split"])
def test_nstep_write_vectors(impl):
    """n_steps = 2 write vectors (archbench/layers/nsgdn.py:61-75): u is not parallel to k."""
    B, T, H = 1, 128, 2
    x = make_inputs(B, T, H, 128, 128, seed=17, dtype=torch.bfloat16)
    k = np32(x["k"]).astype(np.float64)
    p = np.pad(k[:, :-1], ((0, 0), (1, 0), (0, 0), (0, 0)))
    u = O.write_direction(k, p, np32(x["beta"]).astype(np.float64), np.array([1.0, 0.7]), 2)
    u_bf = torch.from_numpy(u.astype(np.float32)).to(torch.bfloat16)
    y_o, S_o = O.recurrence_c(*(np32(x[n]) for n in ("q", "k", "v", "la")), u=np32(u_bf))
    g = {k_: v.cuda() for k_, v in x.items()}
    y, S = ops.gdn_prefill(g["q"], g["k"], g["v"], g["la"], u=u_bf.cuda(), output_final_state=True, out_dtype=torch.float32, impl=impl)
    check(y, y_o, "y")
    check(S, S_o, "S_T")


@pytest.mark.parametrize("impl", VARIANTS)
def test_bf16_output(impl):
    y, S, y_o, S_o = run_case(2, 128, 2, seed=7, out_dtype=torch.bfloat16, impl=impl)
    assert y.dtype == torch.bfloat16
    check(y, y_o, "y bf16", tol_rel=TOL_REL_BF16_OUT)
    check(S, S_o, "S_T")


@pytest.mark.parametrize("impl", VARIANTS)
def test_strided_views(impl):
    B, T, H, D = 2, 128, 2, 128
    x = make_inputs(B, T, H, D, D, seed=9, dtype=torch.bfloat16)
    fused = torch.cat([x["q"].reshape(B, T, -1), x["k"].reshape(B, T, -1), x["v"].reshape(B, T, -1)], -1).cuda()
    q, k, v = (fused[..., i * H * D : (i + 1) * H * D].view(B, T, H, D) for i in range(3))
    assert not q.is_contiguous()
    assert ops.selected_impl(q, k, v, x["la"].cuda(), beta=x["beta"].cuda(), impl=impl) == impl
    y, S = ops.gdn_prefill(q, k, v, x["la"].cuda(), beta=x["beta"].cuda(), output_final_state=True, out_dtype=torch.float32, impl=impl)
    y_o, S_o = O.recurrence_c(*(np32(x[n]) for n in ("q", "k", "v", "la")), beta=np32(x["beta"]))
    check(y, y_o, "y")
    check(S, S_o, "S_T")


@pytest.mark.parametrize("impl", VARIANTS)
def test_cfg1_heads_against_oracle(impl):
    """Configuration-1 sequence length and heads (T=4096, H=8) for one batch row."""
    x = make_inputs(1, 4096, 8, 128, 128, seed=41, dtype=torch.bfloat16)
    y_o, S_o = O.recurrence_c(*(np32(x[n]) for n in ("q", "k", "v", "la")), beta=np32(x["beta"]))
    g = {k: v.cuda() for k, v in x.items()}
    y, S = ops.gdn_prefill(g["q"], g["k"], g["v"], g["la"], beta=g["beta"], output_final_state=True, out_dtype=torch.float32, impl=impl)
    check(y, y_o, "y cfg1 row")
    check(S, S_o, "S_T cfg1 row")


@pytest.mark.parametrize("impl", VARIANTS)
def test_cfg1_full_size_against_recurrent_kernel(impl):
    """Full configuration 1 (B=8, T=4096, H=8): the chunk kernel against the fp32 recurrent
    kernel (itself pinned to the oracle at 1e-5), same tolerance."""
    g = make_inputs(8, 4096, 8, 128, 128, seed=1000, dtype=torch.bfloat16, device="cuda")
    y_c, S_c = ops.gdn_prefill(g["q"], g["k"], g["v"], g["la"], beta=g["beta"], output_final_state=True, out_dtype=torch.float32, impl=impl)
    y_r, S_r = ops.gdn_prefill(g["q"], g["k"], g["v"], g["la"], beta=g["beta"], output_final_state=True, out_dtype=torch.float32, impl="recurrent")
    for a, b_, what in ((y_c, y_r, "y"), (S_c, S_r, "S_T")):
        d = (a - b_).double()
        mx = d.abs().max().item()
        rel = (d.norm() / b_.double().norm()).item()
        assert mx <= TOL_MAX and rel <= TOL_REL, f"{what}: max-abs {mx:.3e} rel-L2 {rel:.3e}"
    assert ops.device_status() == 0


@pytest.mark.parametrize("impl", VARIANTS)
def test_deterministic(impl):
    g = make_inputs(2, 256, 4, 128, 128, seed=3, dtype=torch.bfloat16, device="cuda")
    y1, S1 = ops.gdn_prefill(g["q"], g["k"], g["v"], g["la"], beta=g["beta"], output_final_state=True, impl=impl)
    y2, S2 = ops.gdn_prefill(g["q"], g["k"], g["v"], g["la"], beta=g["beta"], output_final_state=True, impl=impl)
    assert torch.equal(y1, y2) and torch.equal(S1, S2)


def test_state_in_place_and_chaining():
    """Two prefill calls chained through the state equal one call over the concatenation."""
    g = make_inputs(2, 320, 2, 128, 128, seed=12, dtype=torch.bfloat16, device="cuda")
    cut = 192
    sl = lambda n, s: g[n][:, s]
    y_a, S = ops.gdn_prefill(*(sl(n, slice(0, cut)) for n in ("q", "k", "v", "la")), beta=sl("beta", slice(0, cut)), output_final_state=True, out_dtype=torch.float32)
    y_b, S2 = ops.gdn_prefill(*(sl(n, slice(cut, None)) for n in ("q", "k", "v", "la")), beta=sl("beta", slice(cut, None)), initial_state=S, output_final_state=True, out_dtype=torch.float32)
    y_f, S_f = ops.gdn_prefill(g["q"], g["k"], g["v"], g["la"], beta=g["beta"], output_final_state=True, out_dtype=torch.float32)
    torch.testing.assert_close(torch.cat([y_a, y_b], 1), y_f, rtol=0, atol=2e-3)
    torch.testing.assert_close(S2, S_f, rtol=0, atol=2e-3)


def test_bounded_wait_times_out_and_context_survives():
    """Failure detection on the device: a wait on a barrier nothing arrives on gives up after its
    cycle limit, the status word reports GDN_ERR_TIMEOUT, and the GPU keeps working."""
    assert ops.selftest_bounded_wait(2_000_000) == ops.GdnError(-8, "").status
    assert ops.device_status() == 0  # the read above cleared it
    y, S, y_o, S_o = run_case(1, 64, 1, seed=99)
    check(y, y_o, "y after timeout self test")


@pytest.mark.parametrize("impl", ["auto", "chunk_single"])
@pytest.mark.parametrize("DV", [256, 384])
def test_value_dim_multiple_of_128(DV, impl):
    """expand_v > 1 (configs/arch/nsgdn.yaml uses DV = 2 DK): one CTA per 128-row state slice (the
    split path under auto, the single-CTA kernel on request)."""
    x = make_inputs(2, 130, 2, 128, DV, seed=DV, dtype=torch.bfloat16)
    S0 = torch.randn(2, 2, DV, 128, generator=torch.Generator().manual_seed(3)) * 0.2
    y_o, S_o = O.recurrence_c(*(np32(x[n]) for n in ("q", "k", "v", "la")), beta=np32(x["beta"]), s0=S0.numpy())
    g = {k: v.cuda() for k, v in x.items()}
    want = "chunk_split" if impl == "auto" else impl
    assert ops.selected_impl(g["q"], g["k"], g["v"], g["la"], beta=g["beta"], impl=impl) == want
    y, S = ops.gdn_prefill(g["q"], g["k"], g["v"], g["la"], beta=g["beta"], initial_state=S0.cuda(), output_final_state=True,
                           out_dtype=torch.float32, impl=impl)
    check(y, y_o, f"y DV={DV}")
    check(S, S_o, f"S_T DV={DV}")


@pytest.mark.parametrize("impl", ["auto", "chunk_single"])
@pytest.mark.parametrize("DV", [256, 384])
def test_write_vectors_with_wide_state(DV, impl):
    """n_steps = 2 write vectors with DV = 2 DK (configs/arch/nsgdn.yaml: head_dim 128, expand_v 2,
    n_steps 2): the explicit-u kernel runs once per 128-row state slice; bf16 output, initial state
    updated in place."""
    B, T, H = 2, 130, 2
    x = make_inputs(B, T, H, 128, DV, seed=31 + DV, dtype=torch.bfloat16)
    k = np32(x["k"]).astype(np.float64)
    p = np.pad(k[:, :-1], ((0, 0), (1, 0), (0, 0), (0, 0)))
    u = O.write_direction(k, p, np32(x["beta"]).astype(np.float64), np.array([1.0, 0.7]), 2)
    u_bf = torch.from_numpy(u.astype(np.float32)).to(torch.bfloat16)
    S0 = torch.randn(B, H, DV, 128, generator=torch.Generator().manual_seed(4)) * 0.2
    y_o, S_o = O.recurrence_c(*(np32(x[n]) for n in ("q", "k", "v", "la")), u=np32(u_bf), s0=S0.numpy())
    g = {k_: v.cuda() for k_, v in x.items()}
    want = "chunk_split" if impl == "auto" else impl
    assert ops.selected_impl(g["q"], g["k"], g["v"], g["la"], u=u_bf.cuda(), impl=impl) == want
    s = S0.cuda()
    y, S = ops.gdn_prefill(g["q"], g["k"], g["v"], g["la"], u=u_bf.cuda(), initial_state=s, output_final_state=True,
                           out_dtype=torch.float32, impl=impl)
    check(y, y_o, f"y DV={DV} (u given)")
    check(S, S_o, f"S_T DV={DV} (u given)")


@pytest.mark.parametrize("pieces", [1, 3, 8])
def test_prefill_from_host_buffers(pieces):
    """ops.gdn_prefill_from_host (pinned host in, host out, copies pipelined with the prefill) returns
    exactly what gdn_prefill returns for each piece of the batch."""
    B, T, H = 8, 200, 2
    x = {n: t.pin_memory() for n, t in make_inputs(B, T, H, 128, 128, seed=41, dtype=torch.bfloat16).items()}
    y_host = torch.empty(B, T, H, 128, dtype=torch.bfloat16).pin_memory()
    ops.gdn_prefill_from_host(x["q"], x["k"], x["v"], x["la"], x["beta"], y_host, pieces=pieces)
    torch.cuda.synchronize()
    cuts = [B * i // pieces for i in range(pieces + 1)]
    for b0, b1 in zip(cuts[:-1], cuts[1:]):
        g = {n: t[b0:b1].cuda() for n, t in x.items()}
        y, _ = ops.gdn_prefill(g["q"], g["k"], g["v"], g["la"], beta=g["beta"])
        assert torch.equal(y.cpu(), y_host[b0:b1]), (b0, b1)


def test_prefill_from_host_back_to_back_and_after_device_work():
    """Consecutive host-buffer calls overlap one call's copies in with the previous call's tail: two calls
    enqueued without a synchronisation in between each return what gdn_prefill returns; with
    wait_current=True a call reads inputs that a device-to-host copy on the current stream is still
    writing only after that copy."""
    B, T, H = 4, 200, 2
    xs = [{n: t.pin_memory() for n, t in make_inputs(B, T, H, 128, 128, seed=51 + i, dtype=torch.bfloat16).items()}
          for i in range(2)]
    ys = [torch.empty(B, T, H, 128, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    for x, y in zip(xs, ys):
        ops.gdn_prefill_from_host(x["q"], x["k"], x["v"], x["la"], x["beta"], y, pieces=2)
    torch.cuda.synchronize()
    for x, y in zip(xs, ys):
        g = {n: t.cuda() for n, t in x.items()}
        want, _ = ops.gdn_prefill(g["q"], g["k"], g["v"], g["la"], beta=g["beta"])
        assert torch.equal(want.cpu(), y)
    # q produced on the device and copied to pinned host memory on the current stream, not yet complete
    gq = make_inputs(B, T, H, 128, 128, seed=60, dtype=torch.bfloat16, device="cuda")["q"]
    xs[0]["q"].copy_(gq, non_blocking=True)
    ops.gdn_prefill_from_host(xs[0]["q"], xs[0]["k"], xs[0]["v"], xs[0]["la"], xs[0]["beta"], ys[0], pieces=2,
                              wait_current=True)
    torch.cuda.synchronize()
    g = {n: t.cuda() for n, t in xs[0].items()}
    want, _ = ops.gdn_prefill(gq, g["k"], g["v"], g["la"], beta=g["beta"])
    assert torch.equal(want.cpu(), ys[0])


@pytest.mark.parametrize("impl", ["auto"] + VARIANTS)
def test_empty_inputs(impl):
    """T = 0: no token is read or written and S_T = S_0; B = 0: empty outputs."""
    B, H = 2, 2
    x = make_inputs(B, 64, H, 128, 128, seed=5, dtype=torch.bfloat16, device="cuda")
    S0 = torch.randn(B, H, 128, 128, device="cuda")
    e = {n: t[:, :0] for n, t in x.items()}
    y, S = ops.gdn_prefill(e["q"], e["k"], e["v"], e["la"], beta=e["beta"], initial_state=S0, output_final_state=True,
                           impl=impl)
    assert y.shape == (B, 0, H, 128) and torch.equal(S, S0)
    e = {n: t[:0] for n, t in x.items()}
    y, S = ops.gdn_prefill(e["q"], e["k"], e["v"], e["la"], beta=e["beta"], output_final_state=True, impl=impl)
    assert y.shape == (0, 64, H, 128) and S.shape == (0, H, 128, 128)
    assert ops.device_status() == 0


@pytest.mark.parametrize("T", [100, 192])
@pytest.mark.parametrize("with_u", [True, False])
def test_unaligned_y_rows(T, with_u):
    """y rows that are not 16-byte aligned (fp32 y with a row stride of 129 elements) cannot be TMA
    stores: the single-CTA kernel writes them with its own stores (auto selection), for an explicit u
    and for u = beta k."""
    import ctypes

    B, H = 2, 2
    x = make_inputs(B, T, H, 128, 128, seed=31 + T, dtype=torch.bfloat16)
    u = (x["beta"][..., None] * x["k"].float()).to(torch.bfloat16) if with_u else None
    y_o, S_o = O.recurrence_c(*(np32(x[n]) for n in ("q", "k", "v", "la")), u=None if u is None else np32(u),
                              beta=None if with_u else np32(x["beta"]))
    g = {k: v.cuda() for k, v in x.items()}
    a, _, s_out, keep = ops._prepare(g["q"], g["k"], None if u is None else u.cuda(), g["v"], g["la"],
                                     None if with_u else g["beta"], None, True, torch.float32, "auto")
    ybuf = torch.full((B, T, H, 129), float("nan"), device="cuda")
    a.y, a.sy = ybuf.data_ptr(), ops.Strides(T * H * 129, H * 129, 129)
    lib = ops.load_library()
    assert lib.gdn_prefill_select_impl(ctypes.byref(a)) == 5  # GDN_IMPL_CHUNK_SINGLE
    ops._check(lib.gdn_prefill_fwd(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    what = "u given" if with_u else "u = beta k"
    check(ybuf[..., :128], y_o, f"y ({what}, unaligned y rows)")
    check(s_out, S_o, f"S_T ({what}, unaligned y rows)")
    assert torch.isnan(ybuf[..., 128]).all()
    assert ops.device_status() == 0


@pytest.mark.parametrize("T,s0", [(1, False), (63, True), (64, False), (130, True), (4096, False)])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_split_equals_cluster_bitwise(T, s0, out_dtype):
    """The prep kernel restates the cluster kernel's prep CTA operation for operation and the state-only
    kernel is that kernel's state CTA: for DV = 128 and u = beta k both paths give the same bits."""
    B, H = 2, 3
    g = make_inputs(B, T, H, 128, 128, seed=50 + T, dtype=torch.bfloat16, device="cuda")
    S0 = torch.randn(B, H, 128, 128, device="cuda", generator=torch.Generator(device="cuda").manual_seed(T)) * 0.3 if s0 else None
    out = {}
    for impl in ("chunk_cluster", "chunk_split"):
        out[impl] = ops.gdn_prefill(g["q"], g["k"], g["v"], g["la"], beta=g["beta"], initial_state=S0, output_final_state=True,
                                    out_dtype=out_dtype, impl=impl)
    torch.cuda.synchronize()
    assert torch.equal(out["chunk_cluster"][0], out["chunk_split"][0])
    assert torch.equal(out["chunk_cluster"][1], out["chunk_split"][1])
    assert ops.device_status() == 0


def test_split_selected_for_more_sequences_than_clusters():
    """More sequences than two-CTA clusters fit at once (configuration 4's prefill: B=16, H=8): AUTO runs
    the split path, one state-only CTA per sequence in one wave, with the cluster kernel's bits."""
    B, T, H = 16, 200, 8
    g = make_inputs(B, T, H, 128, 128, seed=77, dtype=torch.bfloat16, device="cuda")
    assert ops.selected_impl(g["q"], g["k"], g["v"], g["la"], beta=g["beta"]) == "chunk_split"
    y_a, S_a = ops.gdn_prefill(g["q"], g["k"], g["v"], g["la"], beta=g["beta"], output_final_state=True)
    y_c, S_c = ops.gdn_prefill(g["q"], g["k"], g["v"], g["la"], beta=g["beta"], output_final_state=True,
                               impl="chunk_cluster")
    torch.cuda.synchronize()
    assert torch.equal(y_a, y_c) and torch.equal(S_a, S_c)
    assert ops.device_status() == 0
