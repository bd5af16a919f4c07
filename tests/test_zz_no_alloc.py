"""gdn_prefill_fwd_static_workspace: the segmented prefill for callers that cannot allocate
device memory when they call -- e.g. a plugin whose host framework owns all device memory and
passes only input and output pointers, or a serving loop that forbids cudaMalloc after start-up.
Its scratch is a fixed array inside the library instead of a caller-provided workspace.

Called through the C ABI (ctypes), twice in a row, and compared with the workspace-taking entry
point gdn_prefill_fwd on the same inputs, at the tolerance of the other chunk-kernel tests
(max-abs <= 2e-3, rel-L2 <= 1e-3, fp32 outputs).  This file is collected last so that a run that
stops at its first failure has run every other test before it."""

import ctypes

import pytest
import torch

from archbench_b200 import ops
from archbench_b200.workloads import make_inputs

pytestmark = pytest.mark.gpu
TOL_MAX, TOL_REL = 2e-3, 1e-3


def _errors(a, b):
    d = (a - b).double()
    return d.abs().max().item(), (d.norm() / b.double().norm()).item()


def test_static_workspace_entry_point_matches_workspace_entry_point():
    B, T, H = 1, 48 * 64 + 21, 2  # few, long sequences: the segmented path; ragged last chunk
    g = make_inputs(B, T, H, 128, 128, seed=77, dtype=torch.bfloat16, device="cuda")
    s0 = torch.randn(B, H, 128, 128, device="cuda", generator=torch.Generator(device="cuda").manual_seed(3)) * 0.2
    y_ref, s_ref = ops.gdn_prefill(g["q"], g["k"], g["v"], g["la"], beta=g["beta"], initial_state=s0,
                                   output_final_state=True, out_dtype=torch.float32, impl="segmented")
    lib = ops.load_library()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):  # the second call reuses the array the first one left behind
        args, y, s_out, keep = ops.prefill_args(g["q"], g["k"], g["v"], g["la"], beta=g["beta"], initial_state=s0,
                                                output_final_state=True, out_dtype=torch.float32)
        rc = lib.gdn_prefill_fwd_static_workspace(ctypes.byref(args), stream)
        assert rc == 0, lib.gdn_status_string(rc)
        torch.cuda.synchronize()
        for got, want, what in ((y, y_ref, "y"), (s_out, s_ref, "S_T")):
            mx, rel = _errors(got, want)
            assert mx <= TOL_MAX and rel <= TOL_REL, f"call {call} {what}: max-abs {mx:.3e} rel-L2 {rel:.3e}"
        del keep
    assert ops.device_status() == 0


def test_static_workspace_entry_point_rejects_what_it_does_not_serve():
    lib = ops.load_library()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    g = make_inputs(8, 256, 8, 128, 128, seed=1, dtype=torch.bfloat16, device="cuda")  # many short sequences
    args, _, _, keep = ops.prefill_args(g["q"], g["k"], g["v"], g["la"], beta=g["beta"])
    assert lib.gdn_prefill_fwd_static_workspace(ctypes.byref(args), stream) == -5  # GDN_ERR_UNSUPPORTED
    del keep
