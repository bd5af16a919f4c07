"""The CPU oracle against the golden vectors produced by the reference's own code."""

import hashlib
import os

import numpy as np
import pytest
import torch

from archbench_b200.workloads import make_inputs
from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")
# The goldens are archbench's fp32 arithmetic; the oracle is fp64.  Their gap is fp32 rounding.
TOL_MAX, TOL_REL = 5e-6, 1e-6


def load(name):
    return np.load(os.path.join(GOLD, f"{name}.npz"))


@pytest.mark.parametrize("impl", ["numpy", "c"])
def test_gdn_small_initial_and_final_state(impl):
    d = load("gdn_small")
    f = O.recurrence if impl == "numpy" else O.recurrence_c
    y, S = f(d["q"], d["k"], d["v"], d["la"], beta=d["beta"], s0=d["s0"])
    for got, want in ((y, d["y"]), (S, d["sT"])):
        mx, rel = O.errors(got, want)
        assert mx < TOL_MAX and rel < TOL_REL, (mx, rel)


def test_gdn_small_u_equals_beta_k():
    d = load("gdn_small")
    y1, S1 = O.recurrence(d["q"], d["k"], d["v"], d["la"], u=d["u"], s0=d["s0"])
    y2, S2 = O.recurrence(d["q"], d["k"], d["v"], d["la"], beta=d["beta"], s0=d["s0"])
    assert O.errors(y1, y2)[1] < 1e-6 and O.errors(S1, S2)[1] < 1e-6


@pytest.mark.parametrize("impl", ["numpy", "c"])
def test_nstep_write_vectors(impl):
    d = load("nstep_small")
    f = O.recurrence if impl == "numpy" else O.recurrence_c
    y, S = f(d["q"], d["k"], d["v"], d["la"], u=d["u"])
    for got, want in ((y, d["y"]), (S, d["sT"])):
        mx, rel = O.errors(got, want)
        assert mx < TOL_MAX and rel < TOL_REL, (mx, rel)


def test_write_direction_matches_reference():
    d = load("nstep_small")
    k = d["k"].astype(np.float64)
    p = np.pad(k[:, :-1], ((0, 0), (1, 0), (0, 0), (0, 0)))
    u = O.write_direction(k, p, d["beta"].astype(np.float64), d["lam"].astype(np.float64), 2)
    mx, rel = O.errors(u, d["u"])
    assert mx < 1e-6 and rel < 1e-6


def test_fla_naive_second_oracle():
    d = load("fla_naive")
    # fla's state is [K, V]: the transpose of the (DV, DK) layout used here.
    y, S = O.recurrence(d["q"], d["k"], d["v"], d["la"], beta=d["beta"], s0=np.swapaxes(d["h0"], -1, -2))
    assert O.errors(y, d["y"])[1] < TOL_REL
    assert O.errors(S, np.swapaxes(d["hT"], -1, -2))[1] < TOL_REL


def test_cfg0_generator_and_recurrence():
    d = load("cfg0")
    x = make_inputs(2, 512, 4, 64, 64, seed=0, dtype=torch.float32)
    h = hashlib.sha256()
    for n in ("q", "k", "v", "beta", "la"):
        h.update(np.ascontiguousarray(x[n].numpy()).tobytes())
    assert h.hexdigest() == d["inputs_sha256"].item().decode(), "seeded input generator drifted"
    y, S = O.recurrence_c(*(x[n].numpy() for n in ("q", "k", "v", "la")), beta=x["beta"].numpy())
    mx, rel = O.errors(y[:, ::8], d["y_every8"])
    assert mx < TOL_MAX and rel < TOL_REL
    mx, rel = O.errors(S, d["sT"])
    assert mx < TOL_MAX and rel < TOL_REL
    assert abs(y.sum() - d["y_sum"]) < 1e-3 and abs((y**2).sum() / d["y_sumsq"] - 1) < 1e-6


def test_decode_steps_equal_recurrence():
    x = make_inputs(2, 5, 3, 32, 16, seed=3, dtype=torch.float32)
    q, k, v, la, beta = (x[n].numpy() for n in ("q", "k", "v", "la", "beta"))
    y_full, S_full = O.recurrence(q, k, v, la, beta=beta)
    y_dec, S_dec = O.decode_steps(*(np.swapaxes(a, 0, 1) for a in (q, k, v, la)), np.zeros((2, 3, 16, 32)), beta=np.swapaxes(beta, 0, 1))
    assert np.allclose(np.swapaxes(y_dec, 0, 1), y_full) and np.allclose(S_dec, S_full)


def test_errors_helper():
    assert O.errors(np.ones(3), np.ones(3)) == (0.0, 0.0)
    mx, rel = O.errors(np.array([1.0, 2.0]), np.array([1.0, 1.0]))
    assert mx == 1.0 and abs(rel - 1 / np.sqrt(2)) < 1e-12


@pytest.mark.parametrize("mode", ["u", "beta"])
def test_backward_oracle_matches_reference_autograd(mode):
    """The oracle's backward against float64 autograd through archbench's own nsgdn_ref."""
    d = load("bwd_small")
    kw = dict(u=d["u"]) if mode == "u" else dict(beta=d["beta"])
    for chunk in (64, 16):
        g = O.recurrence_bwd(d["q"], d["k"], d["v"], d["la"], d["dy"], s0=d["s0"], ds_T=d["dsT"], chunk=chunk, **kw)
        names = ["dq", "dk", "dv", "dla", "ds0", "du" if mode == "u" else "dbeta"]
        for n in names:
            mx, rel = O.errors(g[n], d[f"{mode}_{n}"])
            assert mx < 1e-10 and rel < 1e-12, (n, chunk, mx, rel)
