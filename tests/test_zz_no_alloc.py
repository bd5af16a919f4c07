"""gdn_prefill_fwd_static_workspace: the segmented prefill for callers that cannot allocate
device memory when they call -- e.g. a plugin whose host framework owns all device memory and
passes only input and output pointers, or a serving loop that forbids cudaMalloc after start-up
(an allocation there synchronises the device and upsets a pre-planned memory pool).  Its scratch
is a fixed array inside the library instead of a caller-provided workspace.

Every case calls it through the C ABI (ctypes), twice in a row (the second call reuses the array
the first one left behind), and compares it with the workspace-taking entry point gdn_prefill_fwd
and with the float64 C oracle on the same inputs, at the tolerance of the other chunk-kernel tests
(max-abs <= 2e-3, rel-L2 <= 1e-3, fp32 outputs).  This file is collected last so that a run that
stops at its first failure has run every other test before it."""

import ctypes

import numpy as np
import pytest
import torch

from archbench_b200 import ops
from archbench_b200.nstep import write_direction
from archbench_b200.workloads import make_inputs
from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL_MAX, TOL_REL = 2e-3, 1e-3
GDN_ERR_UNSUPPORTED = -5
STATIC_BYTES = 16 << 20  # GDN_STATIC_WORKSPACE_BYTES


def _errors(a, b):
    a = torch.as_tensor(a).double().cpu()
    b = torch.as_tensor(b).double().cpu()
    d = a - b
    return d.abs().max().item(), (d.norm() / b.norm()).item()


def _check(got, want, what):
    mx, rel = _errors(got, want)
    assert mx <= TOL_MAX and rel <= TOL_REL, f"{what}: max-abs {mx:.3e} rel-L2 {rel:.3e}"


def _np32(t):
    return t.detach().float().cpu().numpy()


def _call_static(lib, g, s0, impl="auto", u=None):
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    beta = None if u is not None else g["beta"]
    args, y, s_out, keep = ops.prefill_args(g["q"], g["k"], g["v"], g["la"], beta=beta, u=u, initial_state=s0,
                                            output_final_state=True, out_dtype=torch.float32)
    if impl == "invalid":
        args.impl = 99  # ignored by this entry point
    rc = lib.gdn_prefill_fwd_static_workspace(ctypes.byref(args), stream)
    torch.cuda.synchronize()
    del keep
    return rc, y, s_out


@pytest.mark.parametrize("B,T,H,DV,with_u", [
    (1, 48 * 64 + 21, 2, 128, False),  # few, long sequences; ragged last chunk
    (1, 40 * 64, 1, 256, True),        # nsgdn's write vectors (n_steps 2) and expand_v 2
])
def test_static_workspace_entry_point_matches_oracle_and_workspace_entry_point(B, T, H, DV, with_u):
    g = make_inputs(B, T, H, 128, DV, seed=77 + DV, dtype=torch.bfloat16, device="cuda")
    s0 = torch.randn(B, H, DV, 128, device="cuda", generator=torch.Generator(device="cuda").manual_seed(3)) * 0.2
    u = None
    if with_u:
        kf = g["k"].float()
        prev = torch.nn.functional.pad(kf[:, :-1], (0, 0, 0, 0, 1, 0))
        lam = torch.full((H,), 0.8, device="cuda")
        u = write_direction(kf, prev, g["beta"], lam, 2).to(torch.bfloat16)
    y_ws, s_ws = ops.gdn_prefill(g["q"], g["k"], g["v"], g["la"], beta=None if with_u else g["beta"], u=u,
                                 initial_state=s0, output_final_state=True, out_dtype=torch.float32, impl="segmented")
    y_o, s_o = O.recurrence_c(*(_np32(g[n]) for n in ("q", "k", "v", "la")),
                              beta=None if with_u else _np32(g["beta"]), u=None if u is None else _np32(u),
                              s0=_np32(s0).astype(np.float64))
    lib = ops.load_library()
    for call in range(2):
        rc, y, s_out = _call_static(lib, g, s0, u=u)
        assert rc == 0, lib.gdn_status_string(rc)
        _check(y, y_ws, f"call {call} y vs gdn_prefill_fwd")
        _check(s_out, s_ws, f"call {call} S_T vs gdn_prefill_fwd")
        _check(y, y_o, f"call {call} y vs oracle")
        _check(s_out, s_o, f"call {call} S_T vs oracle")
    assert ops.device_status() == 0


def test_static_workspace_uses_fewer_longer_segments_when_the_usual_plan_does_not_fit():
    # One sequence of 592 chunks (4 per SM of a 148-SM B200, last one ragged): the usual plan (one
    # segment per SM) needs 147 segment-state slots of 128 KB, more scratch than the array holds,
    # so the entry point must cut the sequence into fewer, longer segments.
    B, T, H = 1, 592 * 64 - 20, 1
    g = make_inputs(B, T, H, 128, 128, seed=91, dtype=torch.bfloat16, device="cuda")
    args, _, _, keep = ops.prefill_args(g["q"], g["k"], g["v"], g["la"], beta=g["beta"], impl="segmented")
    lib = ops.load_library()
    need = ctypes.c_size_t(0)
    assert lib.gdn_prefill_workspace_bytes(ctypes.byref(args), ctypes.byref(need)) == 0
    del keep
    assert need.value > STATIC_BYTES, f"the usual plan needs {need.value} B; pick a longer T for this case"
    y_o, s_o = O.recurrence_c(*(_np32(g[n]) for n in ("q", "k", "v", "la")), beta=_np32(g["beta"]))
    for call in range(2):
        rc, y, s_out = _call_static(lib, g, None, impl="invalid" if call else "auto")
        assert rc == 0, lib.gdn_status_string(rc)
        _check(y, y_o, f"call {call} y vs oracle")
        _check(s_out, s_o, f"call {call} S_T vs oracle")
    assert ops.device_status() == 0


def test_static_workspace_entry_point_rejects_what_it_does_not_serve():
    lib = ops.load_library()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    g = make_inputs(8, 256, 8, 128, 128, seed=1, dtype=torch.bfloat16, device="cuda")  # many short sequences
    args, _, _, keep = ops.prefill_args(g["q"], g["k"], g["v"], g["la"], beta=g["beta"])
    assert lib.gdn_prefill_fwd_static_workspace(ctypes.byref(args), stream) == GDN_ERR_UNSUPPORTED
    del keep
