"""CPU oracle for the gated delta rule -- TEST INFRASTRUCTURE ONLY.

This module restates, in float64 numpy, the per-token recurrence that archbench uses as its
own ground truth (archbench/layers/nsgdn.py:408-417, ``nsgdn_ref``) together with the write
vector of nsgdn.py:61-75 (``write_direction``).  It exists to check the CUDA kernels; only
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs
of ``bench.py`` may import it.  The product path (``archbench_b200``) never calls it.

Pinning: ``tests/golden/make_golden.py`` ran archbench's own ``nsgdn_ref`` (and fla 0.5.1's
``naive_recurrent_gated_delta_rule``, a second, independent naive recurrence) on seeded
inputs and stored the outputs under ``tests/golden/``; ``tests/test_oracle.py`` checks this
module against them.

Recurrence, per (b, h), state S of shape (DV, DK) (nsgdn.py:410):
    S = exp(la_t) * S                       nsgdn.py:413
    r = v_t - S @ k_t                       nsgdn.py:414
    S = S + outer(r, u_t)                   nsgdn.py:415
    y_t = S @ q_t                           nsgdn.py:416
"""

from __future__ import annotations

import numpy as np


def write_direction(k: np.ndarray, p: np.ndarray, beta: np.ndarray, lam: np.ndarray, n_steps: int) -> np.ndarray:
    """u_1 = beta k, then n_steps-1 projected steps (archbench/layers/nsgdn.py:61-75).

    k, p: (B, T, H, DK); beta: (B, T, H); lam: (H,).  p is k shifted one token right with a
    zero first token (nsgdn.py:535).
    """
    b = beta[..., None]
    lm = lam[None, None, :, None]
    u = b * k
    if n_steps > 1:
        p_perp = p - (p * k).sum(-1, keepdims=True) * k
        for _ in range(n_steps - 1):
            pu = (p * u).sum(-1, keepdims=True)
            u = u - lm * b * pu * p_perp
    return u


def recurrence(q, k, v, la, beta=None, u=None, s0=None, dtype=np.float64):
    """Token-serial gated delta rule.  Returns (y (B,T,H,DV), S_T (B,H,DV,DK)).

    q, k (and u): (B, T, H, DK); v: (B, T, H, DV); la, beta: (B, T, H); s0: (B, H, DV, DK).
    Exactly one of ``beta`` (u = beta * k) and ``u`` must be given.  Arithmetic is carried out
    in ``dtype`` (float64 by default) on the values given; callers round inputs to the kernel's
    input dtype first so that input rounding is not counted as kernel error.
    """
    q, k, v, la = (np.asarray(a, dtype=dtype) for a in (q, k, v, la))
    if (beta is None) == (u is None):
        raise ValueError("give exactly one of beta and u")
    u = np.asarray(beta, dtype=dtype)[..., None] * k if u is None else np.asarray(u, dtype=dtype)
    B, T, H, DK = q.shape
    DV = v.shape[-1]
    S = np.zeros((B, H, DV, DK), dtype=dtype) if s0 is None else np.array(s0, dtype=dtype, copy=True)
    y = np.empty((B, T, H, DV), dtype=dtype)
    for t in range(T):
        S *= np.exp(la[:, t])[..., None, None]
        r = v[:, t] - np.einsum("bhij,bhj->bhi", S, k[:, t])
        S += r[..., :, None] * u[:, t][..., None, :]
        y[:, t] = np.einsum("bhij,bhj->bhi", S, q[:, t])
    return y, S


def decode_steps(q, k, v, la, state, beta=None, u=None, dtype=np.float64):
    """Apply ``T`` single-token steps to ``state`` (B,H,DV,DK); same maths as ``recurrence``.

    q, k, v: (T, B, H, D) stacks of per-step tokens; la, beta: (T, B, H).  Returns
    (y (T,B,H,DV), new state).  The state is not modified in place.
    """
    swap = lambda a: None if a is None else np.swapaxes(np.asarray(a), 0, 1)
    y, S = recurrence(swap(q), swap(k), swap(v), swap(la), beta=swap(beta), u=swap(u), s0=state, dtype=dtype)
    return np.swapaxes(y, 0, 1), S


def errors(got: np.ndarray, want: np.ndarray) -> tuple[float, float]:
    """(max-abs error, relative L2 error) of ``got`` against ``want``."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    d = got - want
    den = float(np.linalg.norm(want.ravel()))
    return float(np.abs(d).max(initial=0.0)), float(np.linalg.norm(d.ravel()) / den) if den > 0 else float(np.linalg.norm(d.ravel()))


# ---------------------------------------------------------------------------------------------
# C restatement (oracle/gdn_oracle.c): same recurrence, float64, threaded over (b, h).
# ---------------------------------------------------------------------------------------------

_C_LIB = None


def _c_lib():
    global _C_LIB
    if _C_LIB is None:
        import ctypes
        import os

        path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libgdn_oracle.so")
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle`")
        lib = ctypes.CDLL(path)
        f = lib.gdn_oracle_recurrence
        P = ctypes.c_void_p
        I64 = ctypes.c_int64
        f.argtypes = [P, P, P, P, P, P, P, P, P, I64, I64, I64, I64, I64, ctypes.c_int]
        f.restype = ctypes.c_int
        _C_LIB = lib
    return _C_LIB


def recurrence_c(q, k, v, la, beta=None, u=None, s0=None, nthreads=None):
    """``recurrence`` through the C oracle: float32 inputs, float64 arithmetic and outputs."""
    import os

    lib = _c_lib()
    f32 = lambda a: None if a is None else np.ascontiguousarray(a, dtype=np.float32)
    q, k, v, la, beta, u = map(f32, (q, k, v, la, beta, u))
    if (beta is None) == (u is None):
        raise ValueError("give exactly one of beta and u")
    B, T, H, DK = q.shape
    DV = v.shape[-1]
    y = np.empty((B, T, H, DV), dtype=np.float64)
    S = np.empty((B, H, DV, DK), dtype=np.float64)
    s0 = None if s0 is None else np.ascontiguousarray(s0, dtype=np.float64)
    ptr = lambda a: None if a is None else a.ctypes.data
    n = nthreads if nthreads else (os.cpu_count() or 1)
    rc = lib.gdn_oracle_recurrence(ptr(q), ptr(k), ptr(u), ptr(beta), ptr(v), ptr(la), ptr(s0), ptr(y), ptr(S), B, T, H, DK, DV, n)
    if rc != 0:
        raise RuntimeError(f"gdn_oracle_recurrence failed ({rc})")
    return y, S


# ---------------------------------------------------------------------------------------------
# Backward of the recurrence (float64 numpy), for checking the CUDA backward.
# ---------------------------------------------------------------------------------------------


def recurrence_bwd(q, k, v, la, dy, beta=None, u=None, s0=None, ds_T=None, chunk=64, dtype=np.float64):
    """Gradients of the token-serial recurrence for incoming gradients ``dy`` (of y) and ``ds_T``
    (of the final state).

    Restates archbench's own backward of the recurrence (archbench/layers/nsgdn.py:112-155,
    ``_nsgdn_bwd_kernel``): states are checkpointed at chunk starts in a forward sweep; each chunk,
    last to first, recomputes its per-token states and then walks its tokens backwards with the
    state gradient G (DV x DK per (b, h)):

        G += dy_t q_t^T;  dr = G u_t (= dv_t);  du_t = G^T r_t;  G -= dr k_t^T;
        dk_t = -Sp_t^T dr;  dla_t = <G, Sp_t>;  G = alpha_t G

    with Sp_t = alpha_t S_{t-1} the decayed state and dq_t = S_t^T dy_t (nsgdn.py:130-134).
    With ``beta`` (u = beta k) the write-vector gradient is folded in: dk += beta du and
    dbeta = du . k.

    Returns a dict with dq, dk, dv, dla, ds0 and du (``u`` given) or dbeta (``beta`` given).
    """
    q, k, v, la, dy = (np.asarray(a, dtype=dtype) for a in (q, k, v, la, dy))
    if (beta is None) == (u is None):
        raise ValueError("give exactly one of beta and u")
    uu = np.asarray(beta, dtype=dtype)[..., None] * k if u is None else np.asarray(u, dtype=dtype)
    B, T, H, DK = q.shape
    DV = v.shape[-1]
    S = np.zeros((B, H, DV, DK), dtype=dtype) if s0 is None else np.array(s0, dtype=dtype, copy=True)
    starts = list(range(0, T, chunk))
    ckpt = []
    for c0 in starts:  # forward sweep: state at every chunk start
        ckpt.append(S.copy())
        for t in range(c0, min(T, c0 + chunk)):
            S *= np.exp(la[:, t])[..., None, None]
            r = v[:, t] - np.einsum("bhij,bhj->bhi", S, k[:, t])
            S += r[..., :, None] * uu[:, t][..., None, :]
    dq, dk, du = np.zeros_like(q), np.zeros_like(q), np.zeros_like(q)
    dv, dla = np.zeros_like(v), np.zeros_like(la)
    G = np.zeros((B, H, DV, DK), dtype=dtype) if ds_T is None else np.array(ds_T, dtype=dtype, copy=True)
    for c0, S0 in zip(reversed(starts), reversed(ckpt)):
        ts = list(range(c0, min(T, c0 + chunk)))
        S = S0.copy()
        Sp, R = [], []
        for t in ts:  # recompute the chunk: decayed states and residuals
            S *= np.exp(la[:, t])[..., None, None]
            r = v[:, t] - np.einsum("bhij,bhj->bhi", S, k[:, t])
            Sp.append(S.copy())
            R.append(r)
            S += r[..., :, None] * uu[:, t][..., None, :]
            dq[:, t] = np.einsum("bhij,bhi->bhj", S, dy[:, t])
        for i in reversed(range(len(ts))):
            t = ts[i]
            G += dy[:, t][..., :, None] * q[:, t][..., None, :]
            dr = np.einsum("bhij,bhj->bhi", G, uu[:, t])
            dv[:, t] = dr
            du[:, t] = np.einsum("bhij,bhi->bhj", G, R[i])
            G -= dr[..., :, None] * k[:, t][..., None, :]
            dk[:, t] = -np.einsum("bhij,bhi->bhj", Sp[i], dr)
            dla[:, t] = np.einsum("bhij,bhij->bh", G, Sp[i])
            G *= np.exp(la[:, t])[..., None, None]
    out = {"dq": dq, "dv": dv, "dla": dla, "ds0": G}
    if u is None:
        b = np.asarray(beta, dtype=dtype)
        out["dk"] = dk + b[..., None] * du
        out["dbeta"] = (du * k).sum(-1)
    else:
        out["dk"] = dk
        out["du"] = du
    return out
