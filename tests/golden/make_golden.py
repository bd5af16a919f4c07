"""Generate the golden fixtures in this directory from the reference's own code.

Run where the reference tree is available:
    python tests/golden/make_golden.py [/path/to/archbench-checkout]

What it records (all float32 arithmetic, CPU):
  * archbench's naive recurrence ``nsgdn_ref`` (archbench/layers/nsgdn.py:408-417) on seeded
    inputs.  ``nsgdn_ref`` takes no initial state and returns no final state, so both are
    expressed through its own inputs:
      - prefix tokens j = 0..DK-1 with k = u = e_j, v = S0[:, j], la = 0 write column j of the
        state (r = S0[:, j] - S e_j = S0[:, j] while column j is still zero), so the state
        after the prefix is exactly S0;
      - suffix tokens j = 0..DK-1 with k = u = v = 0, la = 0 leave the state unchanged and
        read y = S e_j = column j of the final state.
  * the write vectors of ``write_direction`` (nsgdn.py:61-75) for n_steps = 2, used as u;
  * fla 0.5.1's ``naive_recurrent_gated_delta_rule`` (fla/ops/gated_delta_rule/naive.py:13),
    which takes an initial state and returns the final state directly (state layout [K, V]);
  * gradients of ``nsgdn_ref`` (float64 torch autograd through the reference's own loop, with the
    same prefix/suffix tokens for S0 and S_T) for given incoming gradients dy and dS_T: the
    gradient of S0 is the gradient of the prefix tokens' v, and dS_T enters as the suffix
    tokens' dy.  Once with u a leaf (du), once with u = beta k from ``write_direction``
    (dbeta, and dk including the write-vector path).

  * archbench's own ``NStepGDN`` layer (nsgdn.py:473-542) forward on CPU in float32 (where
    ``pick_scan`` takes ``nsgdn_ref``), parameters from ``layer_params.fill`` and seeded inputs,
    for n_steps 1 and 2, expand_v 1 and 2 and a ragged T: ``nsgdn_layer.npz``.

    python tests/golden/make_golden.py [/path/to/archbench-checkout] [--only NAME]

The checkout defaults to the environment variable ARCHBENCH_REFERENCE.
"""

from __future__ import annotations

import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from archbench_b200.workloads import make_inputs  # noqa: E402


def _ref_modules(ref_root):
    sys.path.insert(0, ref_root)
    from archbench.layers.nsgdn import nsgdn_ref, write_direction  # noqa: E402

    return nsgdn_ref, write_direction


def run_with_state(nsgdn_ref, q, k, u, v, la, s0):
    """nsgdn_ref with an initial state (prefix) and a final-state readout (suffix)."""
    B, T, H, DK = q.shape
    DV = v.shape[-1]
    eye = torch.eye(DK)
    pre_k = eye[None, :, None, :].expand(B, DK, H, DK)
    pre_v = s0.permute(0, 3, 1, 2)  # (B, DK=j, H, DV): column j of S0 for prefix token j
    zk = torch.zeros(B, DK, H, DK)
    qq = torch.cat([zk, q, eye[None, :, None, :].expand(B, DK, H, DK)], 1)
    kk = torch.cat([pre_k, k, zk], 1)
    uu = torch.cat([pre_k, u, zk], 1)
    vv = torch.cat([pre_v, v, torch.zeros(B, DK, H, DV)], 1)
    ll = torch.cat([torch.zeros(B, DK, H), la, torch.zeros(B, DK, H)], 1)
    yy = nsgdn_ref(qq.contiguous(), kk.contiguous(), uu.contiguous(), vv.contiguous(), ll.contiguous())
    y = yy[:, DK : DK + T]
    sT = yy[:, DK + T :].permute(0, 2, 3, 1)  # (B, H, DV, DK): S_T[:, :, :, j] = y of readout j
    return y.contiguous(), sT.contiguous()


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def bwd_fixture(nsgdn_ref, write_direction):
    """Gradients of archbench's nsgdn_ref (float64) with an initial state and a final-state readout."""
    B, T, H, DK, DV = 1, 100, 2, 32, 32
    x = {n: t.double() for n, t in make_inputs(B, T, H, DK, DV, seed=41, dtype=torch.float64).items()}
    g = torch.Generator().manual_seed(42)
    s0 = 0.5 * torch.randn(B, H, DV, DK, generator=g, dtype=torch.float64)
    dy = torch.randn(B, T, H, DV, generator=g, dtype=torch.float64)
    dsT = torch.randn(B, H, DV, DK, generator=g, dtype=torch.float64)
    u_leaf = 0.7 * x["k"] + 0.1 * torch.randn(B, T, H, DK, generator=g, dtype=torch.float64)
    d = dict(q=x["q"], k=x["k"], v=x["v"], beta=x["beta"], la=x["la"], s0=s0, dy=dy, dsT=dsT, u=u_leaf)
    for mode in ("u", "beta"):
        leaves = {n: d[n].clone().requires_grad_(True) for n in ("q", "k", "v", "la", "s0", "u" if mode == "u" else "beta")}
        if mode == "u":
            u = leaves["u"]
        else:
            u = write_direction(leaves["k"], torch.zeros_like(leaves["k"]), leaves["beta"], torch.ones(H, dtype=torch.float64), 1)
        y, sT = run_with_state(nsgdn_ref, leaves["q"], leaves["k"], u, leaves["v"], leaves["la"], leaves["s0"])
        loss = (y * dy).sum() + (sT * dsT).sum()
        grads = torch.autograd.grad(loss, list(leaves.values()))
        for n, gr in zip(leaves, grads):
            d[f"{mode}_d{n}"] = gr.detach()
    return d


# Layer cases: (name, B, T, d_model, keywords).  head_dim 128 puts the scan on the tensor-core kernels.
LAYER_CASES = [
    ("e1_n1", 2, 128, 64, dict(num_heads=2, head_dim=128, expand_v=1.0, n_steps=1)),
    ("e1_n2_ragged", 2, 100, 64, dict(num_heads=2, head_dim=128, expand_v=1.0, n_steps=2)),
    ("e2_n2", 1, 128, 64, dict(num_heads=2, head_dim=128, expand_v=2.0, n_steps=2)),
    ("e2_n1_ragged", 1, 100, 64, dict(num_heads=1, head_dim=128, expand_v=2.0, n_steps=1, use_gate=False)),
]


def layer_fixture(ref_root):
    """archbench's NStepGDN.forward (CPU, float32) on seeded parameters and inputs."""
    sys.path.insert(0, HERE)
    import layer_params  # noqa: E402

    sys.path.insert(0, ref_root)
    from archbench.layers.nsgdn import NStepGDN as RefNStepGDN  # noqa: E402

    d = {}
    for i, (name, B, T, D, kw) in enumerate(LAYER_CASES):
        m = RefNStepGDN(D, **kw)
        digest_w = layer_params.fill(m, 500 + i)
        x = layer_params.layer_input(B, T, D, 600 + i)
        with torch.no_grad():
            y = m(x)
        d[f"{name}_y"] = y
        d[f"{name}_x_sum"] = np.float64(x.double().sum())
        d[f"{name}_params_sha256"] = np.bytes_(digest_w)
    return d


def main(ref_root):
    torch.manual_seed(0)
    nsgdn_ref, write_direction = _ref_modules(ref_root)
    out = {}

    # A: plain GDN write vector u = beta k, random initial state, ragged T.
    B, T, H, DK, DV = 2, 100, 2, 32, 32
    x = make_inputs(B, T, H, DK, DV, seed=11, dtype=torch.float32)
    g = torch.Generator().manual_seed(12)
    s0 = 0.5 * torch.randn(B, H, DV, DK, generator=g)
    lam = torch.ones(H)
    u = write_direction(x["k"], torch.zeros_like(x["k"]), x["beta"], lam, 1)
    y, sT = run_with_state(nsgdn_ref, x["q"], x["k"], u, x["v"], x["la"], s0)
    out["gdn_small"] = dict(q=x["q"], k=x["k"], v=x["v"], beta=x["beta"], la=x["la"], s0=s0, u=u, y=y, sT=sT)

    # B: n_steps = 2 write vectors from the reference's write_direction, S0 = 0.
    B, T, H, DK, DV = 1, 80, 3, 32, 64
    x = make_inputs(B, T, H, DK, DV, seed=21, dtype=torch.float32)
    lam = torch.tensor([0.5, 1.0, 1.7])
    p = torch.nn.functional.pad(x["k"][:, :-1], (0, 0, 0, 0, 1, 0))
    u = write_direction(x["k"], p, x["beta"], lam, 2)
    y = nsgdn_ref(x["q"], x["k"], u, x["v"], x["la"])
    _, sT = run_with_state(nsgdn_ref, x["q"], x["k"], u, x["v"], x["la"], torch.zeros(B, H, DV, DK))
    out["nstep_small"] = dict(q=x["q"], k=x["k"], v=x["v"], beta=x["beta"], la=x["la"], lam=lam, u=u, y=y, sT=sT)

    # C: configuration 0 (B2 T512 H4 d64 fp32, seed 0).  Inputs are regenerated from the
    # seed by the tests; their digest pins the generator.  y is stored every 8th token.
    x = make_inputs(2, 512, 4, 64, 64, seed=0, dtype=torch.float32)
    u = x["beta"][..., None] * x["k"]
    y, sT = run_with_state(nsgdn_ref, x["q"], x["k"], u, x["v"], x["la"], torch.zeros(2, 4, 64, 64))
    y_plain = nsgdn_ref(x["q"], x["k"], u, x["v"], x["la"])
    assert torch.equal(y, y_plain) or torch.allclose(y, y_plain, atol=1e-6), "prefix/suffix changed y"
    out["cfg0"] = dict(
        y_every8=y[:, ::8],
        y_sum=np.float64(y.double().sum()),
        y_sumsq=np.float64(y.double().square().sum()),
        sT=sT,
        inputs_sha256=np.bytes_(digest(*(x[n].numpy() for n in ("q", "k", "v", "beta", "la")))),
    )

    # D: fla's naive recurrence (second oracle), initial state in, final state out.
    from fla.ops.gated_delta_rule.naive import naive_recurrent_gated_delta_rule

    B, T, H, K, V = 1, 64, 2, 32, 32
    x = make_inputs(B, T, H, K, V, seed=31, dtype=torch.float32)
    h0 = 0.3 * torch.randn(B, H, K, V, generator=torch.Generator().manual_seed(32))
    o, hT = naive_recurrent_gated_delta_rule(x["q"], x["k"], x["v"], x["beta"], x["la"], scale=1.0, initial_state=h0, output_final_state=True)
    out["fla_naive"] = dict(q=x["q"], k=x["k"], v=x["v"], beta=x["beta"], la=x["la"], h0=h0, y=o, hT=hT)

    out["bwd_small"] = bwd_fixture(nsgdn_ref, write_direction)

    if ONLY in (None, "nsgdn_layer"):
        out["nsgdn_layer"] = layer_fixture(ref_root)

    for name, d in out.items():
        if ONLY and name != ONLY:
            continue
        arrs = {k: (v.numpy() if isinstance(v, torch.Tensor) else v) for k, v in d.items()}
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrs)
        print(name, {k: getattr(v, "shape", ()) for k, v in arrs.items()})


ONLY = None

if __name__ == "__main__":
    argv = sys.argv[1:]
    if "--only" in argv:
        i = argv.index("--only")
        ONLY = argv[i + 1]
        del argv[i : i + 2]
    root = argv[0] if argv else os.environ.get("ARCHBENCH_REFERENCE")
    if not root:
        sys.exit("give the archbench checkout as an argument or in ARCHBENCH_REFERENCE")
    main(root)
