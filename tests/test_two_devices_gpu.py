"""Two GPUs driven from one process: every kernel that needs more than 48 KB of dynamic shared memory
opts in per device (a function attribute belongs to the function as loaded in one device's
context), so launches on the second device must work after the first device has set up its own.

The same calls run on cuda:0 and then on cuda:1 -- the cluster and single-CTA chunk kernels, the
split path (prep kernel and state-only chunk kernel), the segmented path, the allocation-free entry
point, the backward and the fused layer prologue and epilogue -- and must give bitwise the same
results on both devices (the kernels are deterministic);
the prefill is also checked against the float64 oracle.  No peer memory is touched.  Skipped with
fewer than two GPUs."""

import ctypes

import pytest
import torch

from archbench_b200 import ops
from archbench_b200.layers import NStepGDN
from archbench_b200.workloads import make_inputs
from oracle import oracle as O

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two GPUs")]


def _run_all(dev):
    out = {}
    with torch.cuda.device(dev):
        x = make_inputs(2, 320, 3, 128, 128, seed=41, dtype=torch.bfloat16, device=dev)
        for impl in ("chunk_cluster", "chunk_single", "chunk_split"):
            y, S = ops.gdn_prefill(x["q"], x["k"], x["v"], x["la"], beta=x["beta"], output_final_state=True,
                                   out_dtype=torch.float32, impl=impl)
            out[f"y_{impl}"], out[f"S_{impl}"] = y, S
        xs = make_inputs(1, 40 * 64, 2, 128, 128, seed=42, dtype=torch.bfloat16, device=dev)
        y, S = ops.gdn_prefill(xs["q"], xs["k"], xs["v"], xs["la"], beta=xs["beta"], output_final_state=True,
                               out_dtype=torch.float32, impl="segmented")
        out["y_segmented"], out["S_segmented"] = y, S
        lib = ops.load_library()
        args, y_static, s_static, keep = ops.prefill_args(xs["q"], xs["k"], xs["v"], xs["la"], beta=xs["beta"],
                                                          output_final_state=True, out_dtype=torch.float32)
        rc = lib.gdn_prefill_fwd_static_workspace(ctypes.byref(args), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == 0, lib.gdn_status_string(rc)
        out["y_static"], out["S_static"] = y_static, s_static
        dy = torch.randn(2, 320, 3, 128, device=dev, generator=torch.Generator(device=dev).manual_seed(43)).to(torch.bfloat16)
        for n, g in ops.gdn_prefill_bwd(x["q"], x["k"], x["v"], x["la"], dy, beta=x["beta"]).items():
            out[n] = g
        torch.manual_seed(44)
        m = NStepGDN(256, num_heads=2, head_dim=128, expand_v=1.0, n_steps=2).to(dev)
        xin = torch.randn(2, 96, 256, device=dev, generator=torch.Generator(device=dev).manual_seed(45))
        with torch.no_grad():
            out["layer"] = m(xin)
        torch.cuda.synchronize(dev)
        assert ops.device_status() == 0
    return {k: v.cpu() for k, v in out.items()}, {k: v.float().cpu() for k, v in x.items()}, {k: v.float().cpu() for k, v in xs.items()}


def test_every_kernel_runs_on_both_devices_with_equal_results():
    r0, x0, xs0 = _run_all(torch.device("cuda", 0))
    r1, _, _ = _run_all(torch.device("cuda", 1))
    assert r0.keys() == r1.keys()
    for k in r0:
        assert torch.equal(r0[k], r1[k]), f"{k} differs between cuda:0 and cuda:1"
    y_o, S_o = O.recurrence_c(*(x0[n].numpy() for n in ("q", "k", "v", "la")), beta=x0["beta"].numpy())
    for impl in ("chunk_cluster", "chunk_single", "chunk_split"):
        for got, want, what in ((r0[f"y_{impl}"], y_o, "y"), (r0[f"S_{impl}"], S_o, "S")):
            mx, rel = O.errors(got.numpy(), want)
            assert mx <= 2e-3 and rel <= 1e-3, f"{impl} {what}: max-abs {mx:.3e} rel-L2 {rel:.3e}"
    y_o, S_o = O.recurrence_c(*(xs0[n].numpy() for n in ("q", "k", "v", "la")), beta=xs0["beta"].numpy())
    for name in ("segmented", "static"):
        for got, want, what in ((r0[f"y_{name}"], y_o, "y"), (r0[f"S_{name}"], S_o, "S")):
            mx, rel = O.errors(got.numpy(), want)
            assert mx <= 2e-3 and rel <= 1e-3, f"{name} {what}: max-abs {mx:.3e} rel-L2 {rel:.3e}"
