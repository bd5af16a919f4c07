"""The prefill and decode ops under CUDA-graph capture: a captured call replayed on new inputs
(copied into the captured input buffers) gives the same outputs as an eager call.  Serving
loops and the bench time graph replays, so the C-ABI path must be capturable: no allocation,
no host synchronisation and no stream other than the caller's inside a call."""

import pytest
import torch

from archbench_b200 import ops
from archbench_b200.workloads import make_inputs

pytestmark = pytest.mark.gpu


def _capture(fn):
    fn()  # first call: library load, kernel attributes, caches
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = fn()
    return g, out


@pytest.mark.parametrize("impl", ["chunk_cluster", "chunk_single"])
def test_prefill_graph_replay_matches_eager(impl):
    B, T, H = 2, 320, 4
    a = make_inputs(B, T, H, 128, 128, seed=31, dtype=torch.bfloat16, device="cuda")
    b = make_inputs(B, T, H, 128, 128, seed=32, dtype=torch.bfloat16, device="cuda")
    bufs = {k: v.clone() for k, v in a.items()}
    g, out = _capture(lambda: ops.gdn_prefill(bufs["q"], bufs["k"], bufs["v"], bufs["la"], beta=bufs["beta"],
                                              output_final_state=True, out_dtype=torch.float32, impl=impl))
    for src in (b, a):  # replay on new inputs, then on the first ones again
        for k in bufs:
            bufs[k].copy_(src[k])
        g.replay()
        y_e, s_e = ops.gdn_prefill(src["q"], src["k"], src["v"], src["la"], beta=src["beta"], output_final_state=True,
                                   out_dtype=torch.float32, impl=impl)
        torch.cuda.synchronize()
        assert torch.equal(out[0], y_e) and torch.equal(out[1], s_e)
    assert ops.device_status() == 0


def test_decode_graph_replay_matches_eager():
    B, H = 8, 4
    x = make_inputs(B, 4, H, 128, 128, seed=33, dtype=torch.bfloat16, device="cuda")
    state0 = torch.randn(B, H, 128, 128, device="cuda", generator=torch.Generator(device="cuda").manual_seed(4)) * 0.1
    st_g, st_e = state0.clone(), state0.clone()
    tok = {k: v[:, 0].clone() for k, v in x.items()}
    g, y_g = _capture(lambda: ops.gdn_decode_step(tok["q"], tok["k"], tok["v"], tok["la"], st_g, beta=tok["beta"],
                                                  out_dtype=torch.float32))
    st_g.copy_(state0)  # the capture warm-up calls advanced it
    for t in range(4):
        for k in tok:
            tok[k].copy_(x[k][:, t])
        g.replay()
        y_e = ops.gdn_decode_step(x["q"][:, t], x["k"][:, t], x["v"][:, t], x["la"][:, t], st_e, beta=x["beta"][:, t],
                                  out_dtype=torch.float32)
        torch.cuda.synchronize()
        assert torch.equal(y_g, y_e)
    assert torch.equal(st_g, st_e)
