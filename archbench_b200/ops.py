"""Python/PyTorch side of the gated-DeltaNet kernels: a thin ctypes layer over the C ABI of
``include/gdn_b200.h`` (``libgdn_b200.so``) plus ``torch.library`` custom ops.

There is no CPU path and no other backend: every function here requires CUDA tensors and the
native library, and raises if either is missing.  Under ``torch.compile`` the kernels are opaque:
custom ops with fake implementations, or host functions the compiler does not trace
(``torch.compiler.disable``: the ctypes calls run eagerly between compiled regions).

Public functions
  gdn_prefill(q, k, v, la, beta=None, u=None, initial_state=None, output_final_state=False,
              out_dtype=None, impl="auto") -> (y, S_T | None)
  gdn_decode_step(q, k, v, la, state, beta=None, u=None, out_dtype=None) -> y   (state in place)
  nsgdn_scan(q, k, u, v, la) -> y      # same signature and meaning as the scan functions of
                                       # archbench/layers/nsgdn.py:219,400,408
Custom ops (for torch.compile, mirroring archbench/layers/nsgdn.py:162-216,352-367)
  torch.ops.archbench_b200.prefill, torch.ops.archbench_b200.decode_step
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional

import torch

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libgdn_b200.so")

GDN_DTYPE_F32, GDN_DTYPE_BF16 = 0, 1
IMPLS = {"auto": 0, "chunk": 1, "recurrent": 2, "segmented": 3, "chunk_cluster": 4, "chunk_single": 5, "chunk_split": 6}
IMPL_NAMES = {1: "chunk", 2: "recurrent", 3: "segmented", 4: "chunk_cluster", 5: "chunk_single", 6: "chunk_split"}
# impl values whose calls may need a workspace (gdn_prefill_workspace_bytes), allocated per call
_WORKSPACE_IMPLS = ("auto", "segmented", "chunk_split")
_DT = {torch.float32: GDN_DTYPE_F32, torch.bfloat16: GDN_DTYPE_BF16}


class GdnError(RuntimeError):
    """A gdn_status error returned by the native library."""

    def __init__(self, status: int, msg: str):
        super().__init__(f"gdn_b200 error {status}: {msg}")
        self.status = status


class Strides(ctypes.Structure):
    _fields_ = [("b", ctypes.c_int64), ("t", ctypes.c_int64), ("h", ctypes.c_int64)]


class PrefillArgs(ctypes.Structure):
    """Mirror of gdn_prefill_args (include/gdn_b200.h)."""

    _fields_ = [
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("u", ctypes.c_void_p), ("v", ctypes.c_void_p),
        ("beta", ctypes.c_void_p), ("la", ctypes.c_void_p), ("s0", ctypes.c_void_p), ("y", ctypes.c_void_p),
        ("s_out", ctypes.c_void_p),
        ("sq", Strides), ("sk", Strides), ("su", Strides), ("sv", Strides), ("sy", Strides),
        ("B", ctypes.c_int64), ("T", ctypes.c_int64), ("H", ctypes.c_int64), ("DK", ctypes.c_int64), ("DV", ctypes.c_int64),
        ("in_dtype", ctypes.c_int32), ("out_dtype", ctypes.c_int32), ("impl", ctypes.c_int32), ("reserved", ctypes.c_int32),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_uint64),
    ]


class DecodeArgs(ctypes.Structure):
    """Mirror of gdn_decode_args (include/gdn_b200.h)."""

    _fields_ = [
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("u", ctypes.c_void_p), ("v", ctypes.c_void_p),
        ("beta", ctypes.c_void_p), ("la", ctypes.c_void_p), ("state", ctypes.c_void_p), ("y", ctypes.c_void_p),
        ("sq", Strides), ("sk", Strides), ("su", Strides), ("sv", Strides), ("sy", Strides),
        ("B", ctypes.c_int64), ("H", ctypes.c_int64), ("DK", ctypes.c_int64), ("DV", ctypes.c_int64),
        ("in_dtype", ctypes.c_int32), ("out_dtype", ctypes.c_int32),
    ]


class PrologueArgs(ctypes.Structure):
    """Mirror of gdn_prologue_args (include/gdn_b200.h)."""

    _fields_ = [(n, ctypes.c_void_p) for n in ("xq", "xk", "xv")] + \
               [(n, ctypes.c_int64) for n in ("sxq_b", "sxq_t", "sxk_b", "sxk_t", "sxv_b", "sxv_t")] + \
               [(n, ctypes.c_void_p) for n in ("xa", "xb")] + \
               [(n, ctypes.c_int64) for n in ("sxa_b", "sxa_t", "sxb_b", "sxb_t")] + \
               [(n, ctypes.c_void_p) for n in ("wq", "wk", "wv", "cq_in", "ck_in", "cv_in", "cq_out", "ck_out", "cv_out")] + \
               [(n, ctypes.c_int64) for n in ("scq_b", "sck_b", "scv_b")] + \
               [(n, ctypes.c_void_p) for n in ("A_log", "dt_bias", "b_bias", "q", "k", "v", "la", "beta")] + \
               [(n, ctypes.c_int64) for n in ("B", "T", "H", "DK", "DV")] + \
               [(n, ctypes.c_int32) for n in ("conv_size", "flags", "in_dtype", "out_dtype")] + \
               [(n, ctypes.c_float) for n in ("q_scale", "l2_eps", "la_min", "beta_scale")] + \
               [(n, ctypes.c_void_p) for n in ("u", "lam", "k_prev_in", "k_prev_out")] + \
               [("n_steps", ctypes.c_int32), ("reserved", ctypes.c_int32)]


class EpilogueArgs(ctypes.Structure):
    """Mirror of gdn_epilogue_args (include/gdn_b200.h)."""

    _fields_ = [("y", ctypes.c_void_p), ("sy", Strides), ("g", ctypes.c_void_p), ("sg_b", ctypes.c_int64),
                ("sg_t", ctypes.c_int64), ("weight", ctypes.c_void_p), ("o", ctypes.c_void_p), ("so_b", ctypes.c_int64),
                ("so_t", ctypes.c_int64)] + \
               [(n, ctypes.c_int64) for n in ("B", "T", "H", "DV")] + \
               [(n, ctypes.c_int32) for n in ("y_dtype", "g_dtype", "o_dtype")] + [("eps", ctypes.c_float)]


class BackwardArgs(ctypes.Structure):
    """Mirror of gdn_backward_args (include/gdn_b200.h)."""

    _fields_ = [(n, ctypes.c_void_p) for n in ("q", "k", "u", "v", "beta", "la", "s0", "dy", "ds_T",
                                                 "dq", "dk", "du", "dv", "dbeta", "dla", "ds0")] + \
               [(n, Strides) for n in ("sq", "sk", "su", "sv", "sdy")] + \
               [(n, ctypes.c_int64) for n in ("B", "T", "H", "DK", "DV")] + \
               [("in_dtype", ctypes.c_int32), ("dy_dtype", ctypes.c_int32), ("workspace", ctypes.c_void_p),
                ("workspace_bytes", ctypes.c_uint64)]


class PrologueBwdArgs(ctypes.Structure):
    """Mirror of gdn_prologue_bwd_args (include/gdn_b200.h)."""

    _fields_ = [(n, ctypes.c_void_p) for n in ("xq", "xk", "xv")] + \
               [(n, ctypes.c_int64) for n in ("sxq_b", "sxq_t", "sxk_b", "sxk_t", "sxv_b", "sxv_t")] + \
               [(n, ctypes.c_void_p) for n in ("xa", "xb")] + \
               [(n, ctypes.c_int64) for n in ("sxa_b", "sxa_t", "sxb_b", "sxb_t")] + \
               [(n, ctypes.c_void_p) for n in ("wq", "wk", "wv", "A_log", "dt_bias", "b_bias", "dq", "dk", "dv", "dla", "dbeta",
                                                 "dxq", "dxk", "dxv")] + \
               [(n, ctypes.c_int64) for n in ("sdxq_b", "sdxq_t", "sdxk_b", "sdxk_t", "sdxv_b", "sdxv_t")] + \
               [(n, ctypes.c_void_p) for n in ("dxa", "dxb")] + \
               [(n, ctypes.c_int64) for n in ("sdxa_b", "sdxa_t", "sdxb_b", "sdxb_t")] + \
               [(n, ctypes.c_void_p) for n in ("dwq", "dwk", "dwv", "dA_log", "ddt_bias", "db_bias")] + \
               [(n, ctypes.c_int64) for n in ("B", "T", "H", "DK", "DV")] + \
               [(n, ctypes.c_int32) for n in ("conv_size", "flags", "in_dtype", "grad_dtype")] + \
               [(n, ctypes.c_float) for n in ("q_scale", "l2_eps", "la_min", "beta_scale")]


class WriteVectorsBwdArgs(ctypes.Structure):
    """Mirror of gdn_write_vectors_bwd_args (include/gdn_b200.h)."""

    _fields_ = [(n, ctypes.c_void_p) for n in ("k", "beta", "lam", "du", "dk", "dbeta", "dlam")] + \
               [(n, ctypes.c_int64) for n in ("B", "T", "H", "DK")] + [("k_dtype", ctypes.c_int32), ("n_steps", ctypes.c_int32)]


class EpilogueBwdArgs(ctypes.Structure):
    """Mirror of gdn_epilogue_bwd_args (include/gdn_b200.h)."""

    _fields_ = [("y", ctypes.c_void_p), ("sy", Strides), ("g", ctypes.c_void_p), ("sg_b", ctypes.c_int64),
                ("sg_t", ctypes.c_int64), ("weight", ctypes.c_void_p), ("dout", ctypes.c_void_p), ("sdo_b", ctypes.c_int64),
                ("sdo_t", ctypes.c_int64), ("dy", ctypes.c_void_p), ("dg", ctypes.c_void_p), ("sdg_b", ctypes.c_int64),
                ("sdg_t", ctypes.c_int64), ("dweight", ctypes.c_void_p)] + \
               [(n, ctypes.c_int64) for n in ("B", "T", "H", "DV")] + \
               [(n, ctypes.c_int32) for n in ("y_dtype", "g_dtype", "do_dtype")] + [("eps", ctypes.c_float)]


GDN_PROLOGUE_CLAMP_LA = 1

# Every symbol include/gdn_b200.h declares, with its ctypes signature.
SYMBOLS = {
    "gdn_prefill_fwd": ([ctypes.POINTER(PrefillArgs), ctypes.c_void_p], ctypes.c_int),
    "gdn_decode_step": ([ctypes.POINTER(DecodeArgs), ctypes.c_void_p], ctypes.c_int),
    "gdn_prefill_workspace_bytes": ([ctypes.POINTER(PrefillArgs), ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
    "gdn_prefill_select_impl": ([ctypes.POINTER(PrefillArgs)], ctypes.c_int),
    "gdn_device_status": ([ctypes.POINTER(ctypes.c_int), ctypes.c_int], ctypes.c_int),
    "gdn_selftest_bounded_wait": ([ctypes.c_longlong, ctypes.c_void_p], ctypes.c_int),
    "gdn_prefill_fwd_static_workspace": ([ctypes.POINTER(PrefillArgs), ctypes.c_void_p], ctypes.c_int),
    "gdn_status_string": ([ctypes.c_int], ctypes.c_char_p),
    "gdn_write_vectors_bwd": ([ctypes.POINTER(WriteVectorsBwdArgs), ctypes.c_void_p], ctypes.c_int),
    "gdn_abi_version": ([], ctypes.c_int),
    "gdn_layer_prologue": ([ctypes.POINTER(PrologueArgs), ctypes.c_void_p], ctypes.c_int),
    "gdn_layer_epilogue": ([ctypes.POINTER(EpilogueArgs), ctypes.c_void_p], ctypes.c_int),
    "gdn_prefill_bwd_workspace_bytes": ([ctypes.POINTER(BackwardArgs), ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
    "gdn_prefill_bwd": ([ctypes.POINTER(BackwardArgs), ctypes.c_void_p], ctypes.c_int),
    "gdn_layer_prologue_bwd": ([ctypes.POINTER(PrologueBwdArgs), ctypes.c_void_p], ctypes.c_int),
    "gdn_layer_epilogue_bwd": ([ctypes.POINTER(EpilogueBwdArgs), ctypes.c_void_p], ctypes.c_int),
}

_LIB = None


def load_library(path: str = LIB_PATH):
    """Load libgdn_b200.so (built by ``python -m archbench_b200.build``); raises if absent."""
    global _LIB
    if _LIB is not None and path == LIB_PATH:
        return _LIB
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} is missing: build it with `python -m archbench_b200.build`")
    lib = ctypes.CDLL(path)
    for name, (argtypes, restype) in SYMBOLS.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = restype
    if path == LIB_PATH:
        _LIB = lib
    return lib


def _check(status: int):
    if status != 0:
        msg = load_library().gdn_status_string(status)
        raise GdnError(status, msg.decode() if msg else "?")


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _tok_strides(t: torch.Tensor) -> Strides:
    """(b, t, h) element strides of a [B][T][H][D] view."""
    return Strides(t.stride(0), t.stride(1), t.stride(2))


def _aligned16(t: torch.Tensor) -> bool:
    es = t.element_size()
    return t.data_ptr() % 16 == 0 and all((s * es) % 16 == 0 for s in t.stride()[:-1])


def _prep_token(t: torch.Tensor, name: str, dtype: torch.dtype) -> torch.Tensor:
    """A [B,T,H,D] tensor in ``dtype`` with unit last stride and 16-byte aligned rows."""
    if t.dim() != 4:
        raise ValueError(f"{name} must be (B, T, H, D), got {tuple(t.shape)}")
    if t.dtype != dtype:
        t = t.to(dtype)
    if t.stride(-1) != 1 or not _aligned16(t):
        t = t.contiguous()
    return t


def _check_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("archbench_b200 ops run on CUDA tensors only (no CPU path)")


def prefill_args(q, k, v, la, beta=None, u=None, initial_state=None, output_final_state=False, out_dtype=None, impl="auto"):
    """Build the C-ABI argument block for a prefill: returns (PrefillArgs, y, S_T or None, keep),
    with y and S_T freshly allocated and `keep` holding the (possibly converted) inputs alive for
    as long as the block is used.  For callers that drive the C entry points directly."""
    out_dtype = q.dtype if out_dtype is None else out_dtype
    return _prepare(q, k, u, v, la, beta, initial_state, bool(output_final_state), out_dtype, impl)


def _prepare(q, k, u, v, la, beta, s0, output_final_state: bool, out_dtype: torch.dtype, impl: str, y_out=None):
    _check_cuda(q, k, u, v, la, beta, s0, y_out)
    in_dtype = torch.bfloat16 if q.dtype == torch.bfloat16 else torch.float32
    q, k, v = (_prep_token(t, n, in_dtype) for t, n in ((q, "q"), (k, "k"), (v, "v")))
    if u is not None:
        u = _prep_token(u, "u", in_dtype)
    B, T, H, DK = q.shape
    DV = v.shape[-1]
    if k.shape != q.shape or v.shape[:3] != q.shape[:3] or (u is not None and u.shape != q.shape):
        raise ValueError("q, k, u must be (B, T, H, DK) and v (B, T, H, DV)")
    la = la.float().contiguous()
    if la.shape != (B, T, H):
        raise ValueError(f"la must be (B, T, H) = {(B, T, H)}, got {tuple(la.shape)}")
    if u is None:
        if beta is None:
            raise ValueError("give beta (u = beta * k) or u")
        beta = beta.float().contiguous()
        if beta.shape != (B, T, H):
            raise ValueError("beta must be (B, T, H)")
    else:
        beta = None
    if s0 is not None:
        s0 = s0.float().contiguous()
        if s0.shape != (B, H, DV, DK):
            raise ValueError(f"initial_state must be (B, H, DV, DK) = {(B, H, DV, DK)}")
    if y_out is None:
        y = torch.empty(B, T, H, DV, device=q.device, dtype=out_dtype)
    else:
        if tuple(y_out.shape) != (B, T, H, DV) or y_out.dtype not in _DT or y_out.device != q.device:
            raise ValueError(f"y must be a float32 or bfloat16 (B, T, H, DV) = {(B, T, H, DV)} tensor on {q.device}")
        if y_out.stride(-1) != 1:
            raise ValueError("y must have a unit last stride")
        y, out_dtype = y_out, y_out.dtype
    s_out = torch.empty(B, H, DV, DK, device=q.device, dtype=torch.float32) if output_final_state else None
    a = PrefillArgs(
        _ptr(q), _ptr(k), _ptr(u), _ptr(v), _ptr(beta), _ptr(la), _ptr(s0), _ptr(y), _ptr(s_out),
        _tok_strides(q), _tok_strides(k), _tok_strides(u) if u is not None else Strides(0, 0, 0), _tok_strides(v), _tok_strides(y),
        B, T, H, DK, DV, _DT[in_dtype], _DT[out_dtype], IMPLS[impl], 0,
    )
    return a, y, s_out, (q, k, u, v, la, beta, s0)


def _prefill_impl(q, k, u, v, la, beta, s0, output_final_state: bool, out_dtype: torch.dtype, impl: str, y_out=None):
    a, y, s_out, _keep = _prepare(q, k, u, v, la, beta, s0, output_final_state, out_dtype, impl, y_out)
    lib = load_library()
    if a.B == 0 or a.H == 0:  # an empty batch: empty outputs, nothing to launch
        return y, s_out
    ws = None
    with torch.cuda.device(q.device):
        if impl in _WORKSPACE_IMPLS:
            need = ctypes.c_size_t(0)
            _check(lib.gdn_prefill_workspace_bytes(ctypes.byref(a), ctypes.byref(need)))
            if need.value > 0:  # scratch through torch's caching allocator; the library allocates nothing
                ws = torch.empty(need.value, dtype=torch.uint8, device=q.device)
                a.workspace, a.workspace_bytes = ws.data_ptr(), need.value
        _check(lib.gdn_prefill_fwd(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream(q.device).cuda_stream)))
    return y, s_out


def _prefill_bwd_impl(q, k, u, v, la, beta, s0, dy, ds_T, want_ds0: bool):
    """Gradients of a prefill (see gdn_prefill_bwd): (dq, dk, du_or_dbeta, dv, dla, ds0), fp32;
    du_or_dbeta is du (B, T, H, DK) when u is given, else dbeta (B, T, H); ds0 is empty unless
    ``want_ds0``."""
    _check_cuda(q, k, u, v, la, beta, s0, dy, ds_T)
    in_dtype = torch.bfloat16 if q.dtype == torch.bfloat16 else torch.float32
    q, k, v = (_prep_token(t, n, in_dtype) for t, n in ((q, "q"), (k, "k"), (v, "v")))
    u = None if u is None else _prep_token(u, "u", in_dtype)
    dy = _prep_token(dy, "dy", torch.bfloat16 if dy.dtype == torch.bfloat16 else torch.float32)
    B, T, H, DK = q.shape
    DV = v.shape[-1]
    if DK != 128 or DV % 128 or DV > 1024:
        raise NotImplementedError(f"the prefill backward serves DK = 128, DV a multiple of 128 up to 1024 (got DK={DK}, DV={DV})")
    if dy.shape != (B, T, H, DV):
        raise ValueError(f"dy must be {(B, T, H, DV)}, got {tuple(dy.shape)}")
    la = la.float().contiguous()
    beta = None if u is not None else beta.float().contiguous()
    s0 = None if s0 is None else s0.float().contiguous()
    ds_T = None if ds_T is None else ds_T.float().contiguous()
    dev = q.device
    dq = torch.empty(B, T, H, DK, device=dev, dtype=torch.float32)
    dk = torch.empty_like(dq)
    dv = torch.empty(B, T, H, DV, device=dev, dtype=torch.float32)
    dla = torch.empty(B, T, H, device=dev, dtype=torch.float32)
    du = torch.empty_like(dq) if u is not None else None
    dbeta = torch.empty(B, T, H, device=dev, dtype=torch.float32) if u is None else None
    ds0 = torch.empty(B, H, DV, DK, device=dev, dtype=torch.float32) if want_ds0 else None
    a = BackwardArgs(
        _ptr(q), _ptr(k), _ptr(u), _ptr(v), _ptr(beta), _ptr(la), _ptr(s0), _ptr(dy), _ptr(ds_T),
        _ptr(dq), _ptr(dk), _ptr(du), _ptr(dv), _ptr(dbeta), _ptr(dla), _ptr(ds0),
        _tok_strides(q), _tok_strides(k), _tok_strides(u) if u is not None else Strides(0, 0, 0), _tok_strides(v), _tok_strides(dy),
        B, T, H, DK, DV, _DT[in_dtype], _DT[dy.dtype], None, 0)
    lib = load_library()
    with torch.cuda.device(dev):
        need = ctypes.c_size_t(0)
        _check(lib.gdn_prefill_bwd_workspace_bytes(ctypes.byref(a), ctypes.byref(need)))
        ws = torch.empty(max(need.value, 1), dtype=torch.uint8, device=dev)  # through torch's caching allocator
        a.workspace, a.workspace_bytes = ws.data_ptr(), need.value
        _check(lib.gdn_prefill_bwd(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)))
    empty = q.new_empty(0, dtype=torch.float32)
    return dq, dk, (du if u is not None else dbeta), dv, dla, (ds0 if ds0 is not None else empty)


def _dec_strides(t: torch.Tensor) -> Strides:
    return Strides(t.stride(0), 0, t.stride(1))


def _decode_impl(q, k, u, v, la, beta, state, out_dtype):
    _check_cuda(q, k, u, v, la, beta, state)
    if q.dim() == 4:  # (B, 1, H, D) accepted as well as (B, H, D)
        q, k, v = q[:, 0], k[:, 0], v[:, 0]
        u = None if u is None else u[:, 0]
        la = la[:, 0] if la.dim() == 3 else la
        beta = None if beta is None else (beta[:, 0] if beta.dim() == 3 else beta)
    in_dtype = torch.bfloat16 if q.dtype == torch.bfloat16 else torch.float32
    fix = lambda t: None if t is None else (t.to(in_dtype) if t.dtype != in_dtype else t).contiguous()
    q, k, v, u = fix(q), fix(k), fix(v), fix(u)
    B, H, DK = q.shape
    DV = v.shape[-1]
    if state.dtype != torch.float32 or not state.is_contiguous() or state.shape != (B, H, DV, DK):
        raise ValueError(f"state must be a contiguous fp32 (B, H, DV, DK) = {(B, H, DV, DK)} tensor")
    la = la.float().contiguous()
    beta = None if (u is not None or beta is None) else beta.float().contiguous()
    if u is None and beta is None:
        raise ValueError("give beta (u = beta * k) or u")
    y = torch.empty(B, H, DV, device=q.device, dtype=out_dtype)
    a = DecodeArgs(
        _ptr(q), _ptr(k), _ptr(u), _ptr(v), _ptr(beta), _ptr(la), _ptr(state), _ptr(y),
        _dec_strides(q), _dec_strides(k), _dec_strides(u) if u is not None else Strides(0, 0, 0), _dec_strides(v), _dec_strides(y),
        B, H, DK, DV, _DT[in_dtype], _DT[out_dtype],
    )
    lib = load_library()
    with torch.cuda.device(q.device):
        _check(lib.gdn_decode_step(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream(q.device).cuda_stream)))
    return y


# ------------------------------------------------------------------------------------------------
# torch.library custom ops (opaque to torch.compile; fake impls give output metadata)
# ------------------------------------------------------------------------------------------------

_DTYPE_CODE = {0: torch.float32, 1: torch.bfloat16}


@torch.library.custom_op("archbench_b200::prefill", mutates_args=())
def _prefill_op(
    q: torch.Tensor, k: torch.Tensor, u: Optional[torch.Tensor], v: torch.Tensor, la: torch.Tensor,
    beta: Optional[torch.Tensor], s0: Optional[torch.Tensor], output_final_state: bool, out_dtype_code: int, impl: str,
) -> tuple[torch.Tensor, torch.Tensor]:
    y, s = _prefill_impl(q, k, u, v, la, beta, s0, output_final_state, _DTYPE_CODE[out_dtype_code], impl)
    return y, (s if s is not None else q.new_empty(0, dtype=torch.float32))


@_prefill_op.register_fake
def _(q, k, u, v, la, beta, s0, output_final_state, out_dtype_code, impl):
    B, T, H, DK = q.shape
    DV = v.shape[-1]
    y = q.new_empty(B, T, H, DV, dtype=_DTYPE_CODE[out_dtype_code])
    s = q.new_empty(B, H, DV, DK, dtype=torch.float32) if output_final_state else q.new_empty(0, dtype=torch.float32)
    return y, s


@torch.library.custom_op("archbench_b200::prefill_bwd", mutates_args=())
def _prefill_bwd_op(
    q: torch.Tensor, k: torch.Tensor, u: Optional[torch.Tensor], v: torch.Tensor, la: torch.Tensor,
    beta: Optional[torch.Tensor], s0: Optional[torch.Tensor], dy: torch.Tensor, ds_T: Optional[torch.Tensor], want_ds0: bool,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    return _prefill_bwd_impl(q, k, u, v, la, beta, s0, dy, ds_T, want_ds0)


@_prefill_bwd_op.register_fake
def _(q, k, u, v, la, beta, s0, dy, ds_T, want_ds0):
    B, T, H, DK = q.shape
    DV = v.shape[-1]
    f = lambda *shape: q.new_empty(*shape, dtype=torch.float32)
    return (f(B, T, H, DK), f(B, T, H, DK), f(B, T, H, DK) if u is not None else f(B, T, H), f(B, T, H, DV), f(B, T, H),
            f(B, H, DV, DK) if want_ds0 else f(0))


def _prefill_setup(ctx, inputs, output):
    q, k, u, v, la, beta, s0, output_final_state, out_dtype_code, impl = inputs
    ctx.output_final_state = output_final_state
    ctx.has = (u is not None, beta is not None, s0 is not None)
    ctx.save_for_backward(q, k, u, v, la, beta, s0)


def _prefill_backward(ctx, gy, gs):
    """Autograd of archbench_b200::prefill: the chunked backward kernels (gdn_prefill_bwd).
    Mirrors the autograd registration of archbench's scan ops (archbench/layers/nsgdn.py:206-216,
    386-397)."""
    q, k, u, v, la, beta, s0 = ctx.saved_tensors
    if gy is None:
        gy = torch.zeros(*q.shape[:3], v.shape[-1], device=q.device, dtype=torch.float32)
    ds_T = gs if (ctx.output_final_state and gs is not None and gs.numel() > 0) else None
    dq, dk, dub, dv, dla, ds0 = _prefill_bwd_op(q, k, u, v, la, beta, s0, gy, ds_T, s0 is not None)
    cast = lambda g, ref: None if ref is None else g.to(ref.dtype)
    return (cast(dq, q), cast(dk, k), cast(dub, u) if u is not None else None, cast(dv, v), cast(dla, la),
            cast(dub, beta) if u is None and beta is not None else None, cast(ds0, s0) if s0 is not None else None,
            None, None, None)


_prefill_op.register_autograd(_prefill_backward, setup_context=_prefill_setup)


def gdn_prefill_bwd(q, k, v, la, dy, beta=None, u=None, initial_state=None, ds_T=None, want_ds0=False):
    """Gradients of ``gdn_prefill`` for incoming dy (B, T, H, DV) and ds_T (B, H, DV, DK) or None.
    Returns a dict of fp32 tensors: dq, dk, dv, dla, du (u given) or dbeta, and ds0 if ``want_ds0``.
    DK = 128, DV a multiple of 128."""
    if (u is None) == (beta is None):
        raise ValueError("give exactly one of beta (u = beta * k) and u")
    dq, dk, dub, dv, dla, ds0 = _prefill_bwd_op(q, k, u, v, la, beta, initial_state, dy, ds_T, bool(want_ds0))
    out = {"dq": dq, "dk": dk, "dv": dv, "dla": dla, ("du" if u is not None else "dbeta"): dub}
    if want_ds0:
        out["ds0"] = ds0
    return out


@torch.library.custom_op("archbench_b200::decode_step", mutates_args=("state",))
def _decode_op(
    q: torch.Tensor, k: torch.Tensor, u: Optional[torch.Tensor], v: torch.Tensor, la: torch.Tensor,
    beta: Optional[torch.Tensor], state: torch.Tensor, out_dtype_code: int,
) -> torch.Tensor:
    return _decode_impl(q, k, u, v, la, beta, state, _DTYPE_CODE[out_dtype_code])


@_decode_op.register_fake
def _(q, k, u, v, la, beta, state, out_dtype_code):
    B, H, DV = state.shape[0], state.shape[1], state.shape[2]
    return q.new_empty(B, H, DV, dtype=_DTYPE_CODE[out_dtype_code])


def _code(dt: Optional[torch.dtype], default: torch.dtype) -> int:
    dt = default if dt is None else dt
    if dt not in _DT:
        raise ValueError(f"out_dtype must be float32 or bfloat16, got {dt}")
    return _DT[dt]


def gdn_prefill(q, k, v, la, beta=None, u=None, initial_state=None, output_final_state=False, out_dtype=None, impl="auto"):
    """Gated delta rule over a whole sequence block.

    q, k, u: (B, T, H, DK); v: (B, T, H, DV); la, beta: (B, T, H) fp32; initial_state:
    (B, H, DV, DK) fp32.  q/k/u/v in bf16 run the chunked tcgen05 kernel (DK = DV = 128) or
    the recurrent kernel; fp32 inputs run the recurrent kernel.  Returns (y, S_T or None);
    y defaults to the input dtype.
    """
    if impl not in IMPLS:
        raise ValueError(f"impl must be one of {sorted(IMPLS)}")
    # (workspace for the segmented path is sized and allocated per call by _prefill_impl)
    y, s = _prefill_op(q, k, u, v, la, beta, initial_state, bool(output_final_state), _code(out_dtype, q.dtype if q.dtype in _DT else torch.float32), impl)
    return y, (s if output_final_state else None)


@torch.compiler.disable
def gdn_prefill_into(y, q, k, v, la, beta=None, u=None, initial_state=None, output_final_state=False, impl="auto"):
    """``gdn_prefill`` writing its output into ``y``, a (B, T, H, DV) tensor or view with any element
    strides and a unit last stride (e.g. this rank's slice of a head-major all-gather buffer, seen
    through a permute).  No autograd.  Returns S_T or None."""
    if impl not in IMPLS:
        raise ValueError(f"impl must be one of {sorted(IMPLS)}")
    _, s = _prefill_impl(q, k, u, v, la, beta, initial_state, bool(output_final_state), y.dtype, impl, y_out=y)
    return s


_COPY_STREAMS = {}


def _copy_streams(dev: torch.device):
    if dev.index not in _COPY_STREAMS:
        _COPY_STREAMS[dev.index] = (torch.cuda.Stream(dev), torch.cuda.Stream(dev))
    return _COPY_STREAMS[dev.index]


@torch.compiler.disable
def gdn_prefill_from_host(q, k, v, la, beta, y_out, pieces=8, impl="auto", device=None, wait_current=False):
    """Prefill of host tensors (pinned, for asynchronous copies) into the host tensor ``y_out``.

    The batch is cut into ``pieces`` along B: each piece's inputs are copied to the GPU on one copy
    stream, its prefill runs on the current stream and its output is copied back on another, so the
    host-to-device copies of later pieces overlap the prefill and the device-to-host copies of earlier
    ones (PCIe carries both directions at once).  Returns after enqueueing; the current stream waits
    for the last copy back, so synchronising it (or an event recorded on it) covers the whole call.
    Same arguments and result as ``gdn_prefill(q, k, v, la, beta=beta)`` with y in ``y_out``'s dtype.

    The copies in start at once: the host inputs must hold their values when the call is made, as they
    do when the host wrote them, so consecutive calls overlap one call's copies in with the previous
    call's last prefill and copy back.  ``wait_current=True`` starts them only after the work already
    queued on the current stream -- for inputs that a device-to-host copy ordered on that stream is
    still writing.  The copies back always follow the current stream's earlier work."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    cur = torch.cuda.current_stream(dev)
    h2d, d2h = _copy_streams(dev)
    B = q.shape[0]
    pieces = max(1, min(int(pieces), B))
    cuts = [B * i // pieces for i in range(pieces + 1)]
    if wait_current:
        h2d.wait_stream(cur)
    d2h.wait_stream(cur)
    for b0, b1 in zip(cuts[:-1], cuts[1:]):
        if b1 == b0:
            continue
        with torch.cuda.stream(h2d):
            g = [t[b0:b1].to(dev, non_blocking=True) for t in (q, k, v, la, beta)]
        cur.wait_stream(h2d)
        for t in g:
            t.record_stream(cur)
        y, _ = gdn_prefill(*g[:4], beta=g[4], out_dtype=y_out.dtype, impl=impl)
        d2h.wait_stream(cur)
        y.record_stream(d2h)
        with torch.cuda.stream(d2h):
            y_out[b0:b1].copy_(y, non_blocking=True)
    cur.wait_stream(d2h)
    return y_out


def gdn_decode_step(q, k, v, la, state, beta=None, u=None, out_dtype=None):
    """One token per sequence: q, k, u (B, H, DK), v (B, H, DV), la/beta (B, H); ``state``
    (B, H, DV, DK) fp32 is updated in place.  Returns y (B, H, DV)."""
    return _decode_op(q, k, u, v, la, beta, state, _code(out_dtype, q.dtype if q.dtype in _DT else torch.float32))


def nsgdn_scan(q, k, u, v, la) -> torch.Tensor:
    """Drop-in for archbench's scan ops (archbench/layers/nsgdn.py:219 nsgdn_scan, :400
    nsgdn_scan_chunk, :408 nsgdn_ref): y (B, T, H, DV) for q, k, u (B, T, H, DK), v, la.

    Like nsgdn_scan_chunk, q/k/u/v are cast to bf16 and y is bf16 (fp32 inputs with
    DK != 128 or DV != 128 keep fp32 and run the recurrent kernel)."""
    if q.shape[-1] == 128 and v.shape[-1] == 128:
        dt = torch.bfloat16
        q, k, u, v = (t.to(dt) for t in (q, k, u, v))
    return gdn_prefill(q, k, v, la, u=u)[0]


@torch.compiler.disable
def selected_impl(q, k, v, la, beta=None, u=None, impl="auto") -> str:
    """Name of the kernel ``gdn_prefill`` runs for these arguments ("chunk_cluster", "chunk_single",
    "chunk_split", "segmented" or "recurrent")."""
    _check_cuda(q, k, u, v, la, beta)
    in_dtype = torch.bfloat16 if q.dtype == torch.bfloat16 else torch.float32
    q, k, v = (_prep_token(t, n, in_dtype) for t, n in ((q, "q"), (k, "k"), (v, "v")))
    u = None if u is None else _prep_token(u, "u", in_dtype)
    B, T, H, DK = q.shape
    DV = v.shape[-1]
    a = PrefillArgs(
        _ptr(q), _ptr(k), _ptr(u), _ptr(v), _ptr(beta), _ptr(la), None, 0x100, None,
        _tok_strides(q), _tok_strides(k), _tok_strides(u) if u is not None else Strides(0, 0, 0), _tok_strides(v),
        Strides(T * H * DV, H * DV, DV), B, T, H, DK, DV, _DT[in_dtype], _DT[in_dtype], IMPLS[impl], 0,
    )
    lib = load_library()
    if impl in _WORKSPACE_IMPLS:
        need = ctypes.c_size_t(0)
        _check(lib.gdn_prefill_workspace_bytes(ctypes.byref(a), ctypes.byref(need)))
        if need.value > 0:  # the caller of gdn_prefill always supplies it
            a.workspace, a.workspace_bytes = 0x100, need.value
    r = lib.gdn_prefill_select_impl(ctypes.byref(a))
    if r < 0:
        _check(r)
    return IMPL_NAMES[r]


@torch.compiler.disable
def device_status(reset: bool = False) -> int:
    """The sticky device-side status word (0 = no kernel reported a bounded-wait timeout)."""
    out = ctypes.c_int(0)
    _check(load_library().gdn_device_status(ctypes.byref(out), int(bool(reset))))
    return out.value


@torch.compiler.disable
def selftest_bounded_wait(max_cycles: int = 2_000_000) -> int:
    """Run the device-side bounded-wait self test and return the status word it leaves
    (GDN_ERR_TIMEOUT = -8 when the wait gave up as designed).  Clears the word first."""
    device_status(reset=True)
    lib = load_library()
    _check(lib.gdn_selftest_bounded_wait(int(max_cycles), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    st = device_status(reset=True)
    return st


# ------------------------------------------------------------------------------------------------
# Layer prologue / epilogue (the torch ops around the scan in NStepGDN / GatedDeltaNet.forward)

_DTC = {torch.bfloat16: GDN_DTYPE_BF16, torch.float32: GDN_DTYPE_F32}


def _cached(t: torch.Tensor, kind: str, make):
    """``make(t)`` (a derived copy of a parameter: fp32, transposed, ...), kept on the tensor object and
    reused while the tensor is unchanged (same storage and version counter).  Calls that record
    autograd history on ``t`` compute afresh.  Inference and CUDA-graph decode steps then launch no
    conversion kernels for the layer's constants."""
    if torch.is_grad_enabled() and t.requires_grad:
        return make(t)
    key = (t.data_ptr(), t._version, tuple(t.shape), t.dtype, t.device)
    store = getattr(t, "_gdn_derived", None)
    if store is None:
        store = {}
        try:
            t._gdn_derived = store
        except (AttributeError, RuntimeError):
            return make(t)
    hit = store.get(kind)
    if hit is not None and hit[0] == key:
        return hit[1]
    val = make(t)
    store[kind] = (key, val)
    return val


def _f32(t: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    return None if t is None else _cached(t, "f32", lambda x: x.float().contiguous())


def _rows16(t: torch.Tensor) -> torch.Tensor:
    """A (B, T, C) view with unit channel stride and 16-byte aligned (b, t) strides, else a copy."""
    es = t.element_size()
    if t.stride(-1) != 1 or t.data_ptr() % 16 or (t.stride(0) * es) % 16 or (t.stride(1) * es) % 16:
        t = t.contiguous()
    return t


@torch.compiler.disable
def layer_prologue(xq, xk, xv, xa, xb, A_log, dt_bias, *, H, DK, DV, b_bias=None, conv=None, conv_state=None,
                   want_state=False, q_scale=1.0, l2_eps=1e-12, la_min=None, beta_scale=1.0, out_dtype=torch.bfloat16,
                   n_steps=1, lam=None, k_prev=None, in_place=False):
    """q, k, v (B, T, H, D) in ``out_dtype`` and la, beta (B, T, H) fp32 from the layer's
    projections, in one CUDA kernel: SiLU(short causal conv) of each projection, l2-normalised q
    (times ``q_scale``) and k, la = -softplus(a + dt_bias) exp(A_log) (clamped at ``la_min``),
    beta = sigmoid(b + b_bias) * beta_scale.  ``conv`` = (wq, wk, wv) weights of shape
    (channels, conv_size) (or the layer's (channels, 1, conv_size)) or None (SiLU only); ``conv_state`` = (cq, ck, cv) of shape
    (B, channels, conv_size - 1) continues a previous call.  Returns (q, k, v, la, beta, new_state)
    with new_state None unless ``want_state``.  With ``n_steps`` > 1 (nsgdn write vectors, ``lam`` the
    per-head step sizes, ``k_prev`` (B, H, DK) the previous call's last normalised k or None) it returns
    (q, k, v, la, beta, new_state, u, k_last) with k_last (B, H, DK) fp32 when ``want_state``.
    ``in_place`` (one token, ``want_state``, a conv state given): the new conv state (and k_last) are
    written over ``conv_state`` (and ``k_prev``) and those tensors are returned; a one-token call is
    one run of one warp per (b, h), which reads the old state before it writes the new one."""
    _check_cuda(xq, xk, xv, xa, xb)
    dt = xq.dtype
    if dt not in _DTC or any(t.dtype != dt for t in (xk, xv, xa, xb)):
        raise ValueError("projections must share one dtype, bf16 or fp32")
    xq, xk, xv = _rows16(xq), _rows16(xk), _rows16(xv)
    B, T, _ = xq.shape
    dev = xq.device
    q = torch.empty(B, T, H, DK, device=dev, dtype=out_dtype)
    k = torch.empty(B, T, H, DK, device=dev, dtype=out_dtype)
    v = torch.empty(B, T, H, DV, device=dev, dtype=out_dtype)
    la = torch.empty(B, T, H, device=dev, dtype=torch.float32)
    beta = torch.empty(B, T, H, device=dev, dtype=torch.float32)
    taps = 1 if conv is None else conv[0].shape[-1]
    ws = [None, None, None] if conv is None else [
        _cached(w, f"convT{taps}", lambda x: x.reshape(x.shape[0], taps).float().t().contiguous()) for w in conv]
    nstep = int(n_steps) > 1
    in_place = bool(in_place) and T == 1 and want_state and taps > 1 and conv_state is not None
    if in_place:  # the state tensors are read and rewritten by the kernel: channel stride taps - 1, unit last
        for c, ch in zip(conv_state, (H * DK, H * DK, H * DV)):
            if c.dtype != dt or tuple(c.shape) != (B, ch, taps - 1) or c.stride(2) != 1 or c.stride(1) != taps - 1:
                in_place = False
        if nstep and k_prev is not None and (k_prev.dtype != torch.float32 or not k_prev.is_contiguous()):
            in_place = False
    if in_place:
        cin = list(conv_state)
        cout = list(conv_state)
    else:
        cin = [None, None, None] if conv_state is None else [c.to(dt).contiguous() for c in conv_state]
        cout = [None, None, None]
        if want_state and taps > 1:
            cout = [torch.empty(B, ch, taps - 1, device=dev, dtype=dt) for ch in (H * DK, H * DK, H * DV)]
    A_log, dt_bias, b_bias = _f32(A_log), _f32(dt_bias), _f32(b_bias)
    st = lambda c: 0 if c is None else c.stride(0)
    u = torch.empty(B, T, H, DK, device=dev, dtype=out_dtype) if nstep else None
    lam32 = lam.float().contiguous() if nstep else None
    kp_in = k_prev.reshape(B, H, DK).float().contiguous() if (nstep and k_prev is not None) else None
    kp_out = None
    if nstep and want_state:
        kp_out = kp_in if (in_place and kp_in is not None) else torch.empty(B, H, DK, device=dev, dtype=torch.float32)
    a = PrologueArgs(
        _ptr(xq), _ptr(xk), _ptr(xv), xq.stride(0), xq.stride(1), xk.stride(0), xk.stride(1), xv.stride(0), xv.stride(1),
        _ptr(xa), _ptr(xb), xa.stride(0), xa.stride(1), xb.stride(0), xb.stride(1),
        *[_ptr(w) for w in ws], *[_ptr(c) for c in cin], *[_ptr(c) for c in cout],
        st(cout[0] if cout[0] is not None else cin[0]), st(cout[1] if cout[1] is not None else cin[1]),
        st(cout[2] if cout[2] is not None else cin[2]),
        _ptr(A_log), _ptr(dt_bias), _ptr(b_bias), _ptr(q), _ptr(k), _ptr(v), _ptr(la), _ptr(beta),
        B, T, H, DK, DV, taps, GDN_PROLOGUE_CLAMP_LA if la_min is not None else 0, _DTC[dt], _DTC[out_dtype],
        float(q_scale), float(l2_eps), float(la_min if la_min is not None else 0.0), float(beta_scale),
        _ptr(u), _ptr(lam32), _ptr(kp_in), _ptr(kp_out), int(n_steps) if nstep else 1, 0)
    for t in (xa, xb):
        if t.stride(-1) != 1:
            raise ValueError("gate projections need a unit last stride")
    _check(load_library().gdn_layer_prologue(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)))
    st = tuple(cout) if want_state and taps > 1 else None
    if nstep:
        return q, k, v, la, beta, st, u, kp_out
    return q, k, v, la, beta, st


@torch.compiler.disable
def layer_epilogue(y, weight, g=None, eps=1e-5, out_dtype=torch.bfloat16):
    """o (B, T, H*DV) = RMSNorm over each head's DV values of y (B, T, H, DV) times ``weight``,
    times SiLU(g) when g (B, T, H*DV) is given; fp32 arithmetic, one rounding to ``out_dtype``."""
    _check_cuda(y, g)
    if y.dtype not in _DTC or (g is not None and g.dtype not in _DTC):
        raise ValueError("y and g must be bf16 or fp32")
    B, T, H, DV = y.shape
    y = _prep_token(y, "y", y.dtype)
    if g is not None:
        g = _rows16(g.reshape(B, T, H * DV))
    o = torch.empty(B, T, H * DV, device=y.device, dtype=out_dtype)
    w = _f32(weight)
    a = EpilogueArgs(_ptr(y), _tok_strides(y), _ptr(g), 0 if g is None else g.stride(0), 0 if g is None else g.stride(1),
                     _ptr(w), _ptr(o), o.stride(0), o.stride(1), B, T, H, DV, _DTC[y.dtype],
                     _DTC[g.dtype] if g is not None else GDN_DTYPE_F32, _DTC[out_dtype], float(eps))
    _check(load_library().gdn_layer_epilogue(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream(y.device).cuda_stream)))
    return o


# ------------------------------------------------------------------------------------------------
# Differentiable prologue / epilogue (training through the fused kernels)
# ------------------------------------------------------------------------------------------------


def layer_io_trainable(DK: int, DV: int, conv_size: int) -> bool:
    """Head sizes and conv widths the prologue/epilogue backward kernels serve."""
    return DK in (64, 128) and DV in (DK, 2 * DK) and 1 <= conv_size <= 4


@torch.library.custom_op("archbench_b200::layer_prologue_train", mutates_args=())
def _prologue_train_op(
    xq: torch.Tensor, xk: torch.Tensor, xv: torch.Tensor, xa: torch.Tensor, xb: torch.Tensor,
    wq: Optional[torch.Tensor], wk: Optional[torch.Tensor], wv: Optional[torch.Tensor],
    A_log: torch.Tensor, dt_bias: torch.Tensor, b_bias: Optional[torch.Tensor], H: int, DK: int, DV: int,
    q_scale: float, l2_eps: float, la_min: Optional[float], beta_scale: float, out_dtype_code: int,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    conv = None if wq is None else tuple(w.t() for w in (wq, wk, wv))  # tap-major -> (channels, taps)
    q, k, v, la, beta, _ = layer_prologue(xq, xk, xv, xa, xb, A_log, dt_bias, H=H, DK=DK, DV=DV, b_bias=b_bias, conv=conv,
                                          q_scale=q_scale, l2_eps=l2_eps, la_min=la_min, beta_scale=beta_scale,
                                          out_dtype=_DTYPE_CODE[out_dtype_code])
    return q, k, v, la, beta


@_prologue_train_op.register_fake
def _(xq, xk, xv, xa, xb, wq, wk, wv, A_log, dt_bias, b_bias, H, DK, DV, q_scale, l2_eps, la_min, beta_scale, out_dtype_code):
    B, T = xq.shape[:2]
    od = _DTYPE_CODE[out_dtype_code]
    e = lambda *sh, dt=od: xq.new_empty(*sh, dtype=dt)
    return e(B, T, H, DK), e(B, T, H, DK), e(B, T, H, DV), e(B, T, H, dt=torch.float32), e(B, T, H, dt=torch.float32)


def _prologue_train_setup(ctx, inputs, output):
    xq, xk, xv, xa, xb, wq, wk, wv, A_log, dt_bias, b_bias, H, DK, DV, q_scale, l2_eps, la_min, beta_scale, _ = inputs
    ctx.save_for_backward(xq, xk, xv, xa, xb, wq, wk, wv, A_log, dt_bias, b_bias)
    ctx.cfg = (H, DK, DV, q_scale, l2_eps, la_min, beta_scale)


def _run_prologue_bwd(xs, ws, A_log, dt_bias, b_bias, grads, outs, H, DK, DV, q_scale, l2_eps, la_min, beta_scale):
    """gdn_layer_prologue_bwd: xs = (xq, xk, xv, xa, xb) forward inputs; ws = tap-major fp32 conv weights
    or Nones; grads = (dq, dk, dv, dla, dbeta); outs = (dxq, dxk, dxv, dxa, dxb) to write (any b/t strides).
    Returns (dws, dA_log, ddt_bias, db_bias) in fp32."""
    xq, xk, xv, xa, xb = xs
    B, T, _ = xq.shape
    dev, dt = xq.device, xq.dtype
    dq, dk, dv, dla, dbeta = grads
    gd = dq.dtype if dq is not None else torch.float32
    dq = torch.zeros(B, T, H, DK, device=dev, dtype=gd) if dq is None else dq.contiguous()
    dk = torch.zeros(B, T, H, DK, device=dev, dtype=gd) if dk is None else dk.to(gd).contiguous()
    dv = torch.zeros(B, T, H, DV, device=dev, dtype=gd) if dv is None else dv.to(gd).contiguous()
    dla = torch.zeros(B, T, H, device=dev) if dla is None else dla.float().contiguous()
    dbeta = torch.zeros(B, T, H, device=dev) if dbeta is None else dbeta.float().contiguous()
    xq, xk, xv = _rows16(xq), _rows16(xk), _rows16(xv)
    dxq, dxk, dxv, dxa, dxb = outs
    taps = 1 if ws[0] is None else ws[0].shape[0]
    dws = [None, None, None] if ws[0] is None else [torch.empty_like(w) for w in ws]
    dA, ddt = torch.empty(H, device=dev), torch.empty(H, device=dev)
    dbb = None if b_bias is None else torch.empty(H, device=dev)
    A32, dt32 = A_log.float().contiguous(), dt_bias.float().contiguous()
    bb32 = None if b_bias is None else b_bias.float().contiguous()
    ws = [None if w is None else w.contiguous() for w in ws]
    a = PrologueBwdArgs(
        _ptr(xq), _ptr(xk), _ptr(xv), xq.stride(0), xq.stride(1), xk.stride(0), xk.stride(1), xv.stride(0), xv.stride(1),
        _ptr(xa), _ptr(xb), xa.stride(0), xa.stride(1), xb.stride(0), xb.stride(1),
        *[_ptr(w) for w in ws], _ptr(A32), _ptr(dt32), _ptr(bb32), _ptr(dq), _ptr(dk), _ptr(dv), _ptr(dla), _ptr(dbeta),
        _ptr(dxq), _ptr(dxk), _ptr(dxv), dxq.stride(0), dxq.stride(1), dxk.stride(0), dxk.stride(1), dxv.stride(0), dxv.stride(1),
        _ptr(dxa), _ptr(dxb), dxa.stride(0), dxa.stride(1), dxb.stride(0), dxb.stride(1),
        *[_ptr(w) for w in dws], _ptr(dA), _ptr(ddt), _ptr(dbb),
        B, T, H, DK, DV, taps, GDN_PROLOGUE_CLAMP_LA if la_min is not None else 0, _DTC[dt], _DTC[gd],
        float(q_scale), float(l2_eps), float(la_min if la_min is not None else 0.0), float(beta_scale))
    _check(load_library().gdn_layer_prologue_bwd(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)))
    return dws, dA, ddt, dbb


def _prologue_train_backward(ctx, dq, dk, dv, dla, dbeta):
    """The prologue's backward kernel (gdn_layer_prologue_bwd): projection, gate, conv-weight and
    A_log / dt_bias / b_bias gradients in one pass."""
    xq, xk, xv, xa, xb, wq, wk, wv, A_log, dt_bias, b_bias = ctx.saved_tensors
    H, DK, DV, q_scale, l2_eps, la_min, beta_scale = ctx.cfg
    B, T, _ = xq.shape
    dev, dt = xq.device, xq.dtype
    outs = (torch.empty(B, T, H * DK, device=dev, dtype=dt), torch.empty(B, T, H * DK, device=dev, dtype=dt),
            torch.empty(B, T, H * DV, device=dev, dtype=dt), torch.empty(B, T, H, device=dev, dtype=dt),
            torch.empty(B, T, H, device=dev, dtype=dt))
    dws, dA, ddt, dbb = _run_prologue_bwd((xq, xk, xv, xa, xb), (wq, wk, wv), A_log, dt_bias, b_bias,
                                          (dq, dk, dv, dla, dbeta), outs, H, DK, DV, q_scale, l2_eps, la_min, beta_scale)
    return (*outs, dws[0], dws[1], dws[2], dA.to(A_log.dtype), ddt.to(dt_bias.dtype),
            None if dbb is None else dbb.to(b_bias.dtype), None, None, None, None, None, None, None, None)


_prologue_train_op.register_autograd(_prologue_train_backward, setup_context=_prologue_train_setup)


@torch.library.custom_op("archbench_b200::layer_epilogue_train", mutates_args=())
def _epilogue_train_op(y: torch.Tensor, weight: torch.Tensor, g: Optional[torch.Tensor], eps: float, out_dtype_code: int) -> torch.Tensor:
    return layer_epilogue(y, weight, g, eps=eps, out_dtype=_DTYPE_CODE[out_dtype_code])


@_epilogue_train_op.register_fake
def _(y, weight, g, eps, out_dtype_code):
    B, T, H, DV = y.shape
    return y.new_empty(B, T, H * DV, dtype=_DTYPE_CODE[out_dtype_code])


def _epilogue_train_setup(ctx, inputs, output):
    y, weight, g, eps, _ = inputs
    ctx.save_for_backward(y, weight, g)
    ctx.eps = eps


def _run_epilogue_bwd(y, weight, g, do, dy, dg, eps):
    """gdn_layer_epilogue_bwd: writes dy (contiguous (B, T, H, DV)) and dg (any b/t strides) and returns
    the fp32 gradient of the norm weight."""
    B, T, H, DV = y.shape
    yv = _prep_token(y, "y", y.dtype)
    gv = None if g is None else _rows16(g.reshape(B, T, H * DV))
    do = _rows16(do.reshape(B, T, H * DV))
    if do.dtype not in _DTC:
        do = do.float()
    dw = torch.empty(DV, device=y.device)
    w = weight.float().contiguous()
    a = EpilogueBwdArgs(_ptr(yv), _tok_strides(yv), _ptr(gv), 0 if gv is None else gv.stride(0), 0 if gv is None else gv.stride(1),
                        _ptr(w), _ptr(do), do.stride(0), do.stride(1), _ptr(dy), _ptr(dg), 0 if dg is None else dg.stride(0),
                        0 if dg is None else dg.stride(1), _ptr(dw), B, T, H, DV,
                        _DTC[y.dtype], _DTC[gv.dtype] if gv is not None else GDN_DTYPE_F32, _DTC[do.dtype], float(eps))
    _check(load_library().gdn_layer_epilogue_bwd(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream(y.device).cuda_stream)))
    return dw


@torch.compiler.disable
def write_vectors_bwd(k, beta, lam, du, dk, n_steps):
    """Backward of the n-step write vectors u(k, beta, lam) (archbench/layers/nsgdn.py:61-75, p = the
    previous token's k, zero before the first) in one CUDA kernel (gdn_write_vectors_bwd): adds
    their share of dk into ``dk`` ((B, T, H, DK) fp32 contiguous, in place) and returns
    (dbeta (B, T, H), dlam (H,)) in fp32."""
    _check_cuda(k, beta, lam, du, dk)
    B, T, H, DK = k.shape
    k = k.contiguous() if k.dtype in (torch.bfloat16, torch.float32) else k.float().contiguous()
    beta, lam, du = beta.float().contiguous(), lam.float().contiguous(), du.float().contiguous()
    if dk.dtype != torch.float32 or not dk.is_contiguous() or dk.shape != (B, T, H, DK):
        raise ValueError("dk must be a contiguous fp32 (B, T, H, DK) tensor")
    dbeta = torch.empty(B, T, H, device=k.device)
    dlam = torch.empty(H, device=k.device)
    a = WriteVectorsBwdArgs(_ptr(k), _ptr(beta), _ptr(lam), _ptr(du), _ptr(dk), _ptr(dbeta), _ptr(dlam), B, T, H, DK,
                            _DTC[k.dtype], int(n_steps))
    _check(load_library().gdn_write_vectors_bwd(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream(k.device).cuda_stream)))
    return dbeta, dlam


def _epilogue_train_backward(ctx, do):
    """The epilogue's backward kernel (gdn_layer_epilogue_bwd): dy, dg and the norm weight's gradient."""
    y, weight, g = ctx.saved_tensors
    B, T, H, DV = y.shape
    dy = torch.empty(B, T, H, DV, device=y.device, dtype=y.dtype)
    dg = None if g is None else torch.empty(B, T, H * DV, device=y.device, dtype=g.dtype)
    dw = _run_epilogue_bwd(y, weight, g, do, dy, dg, ctx.eps)
    return dy, dw.to(weight.dtype), (None if g is None else dg.reshape(g.shape)), None, None


_epilogue_train_op.register_autograd(_epilogue_train_backward, setup_context=_epilogue_train_setup)


def layer_prologue_train(xq, xk, xv, xa, xb, A_log, dt_bias, *, H, DK, DV, b_bias=None, conv=None, q_scale=1.0,
                         l2_eps=1e-12, la_min=None, beta_scale=1.0, out_dtype=torch.bfloat16):
    """``layer_prologue`` without conv state, differentiable: its backward is one CUDA kernel.  ``conv`` =
    (wq, wk, wv) of shape (channels, conv_size) (or the layer's (channels, 1, conv_size)), or None."""
    ws = (None, None, None)
    if conv is not None:
        ws = tuple(w.reshape(w.shape[0], w.shape[-1]).float().t().contiguous() for w in conv)  # tap-major fp32
    return _prologue_train_op(xq, xk, xv, xa, xb, *ws, A_log, dt_bias, b_bias, H, DK, DV, float(q_scale), float(l2_eps),
                              None if la_min is None else float(la_min), float(beta_scale), _DTC[out_dtype])


def layer_epilogue_train(y, weight, g=None, eps=1e-5, out_dtype=torch.bfloat16):
    """``layer_epilogue``, differentiable: its backward is one CUDA kernel."""
    return _epilogue_train_op(y, weight, g, float(eps), _DTC[out_dtype])


class NsgdnMixerTrain(torch.autograd.Function):
    """The nsgdn mixer between its fused input projection and its output projection: prologue,
    scan and epilogue forward and backward on the CUDA kernels.  The gradient of the projection is
    written once, column block by column block, by the three backward kernels (no per-slice
    accumulation).  Inputs: proj (B, T, width) with columns [q | k | v | g | a | b | pad], conv
    weight (3 H DK.., taps) fp32 or None, A_log, dt_bias, b_bias, norm weight, softplus(lam) (H,)
    fp32; output o (B, T, H DV) in proj's dtype.  With n_steps > 1 the prologue kernel also forms the
    write vectors (archbench/layers/nsgdn.py:61-75, previous token's k, zero before the first) and
    ``write_vectors_bwd`` differentiates them."""

    @staticmethod
    def forward(ctx, proj, conv_w, A_log, dt_bias, b_bias, norm_w, lam_sp, cfg):
        H, DK, DV, n_gate, q_scale, la_min, eps, impl, n_steps = cfg
        qd = H * DK
        n_qkv = 2 * qd + H * DV
        ab0 = n_qkv + n_gate
        xs = (proj[..., :qd], proj[..., qd:2 * qd], proj[..., 2 * qd:n_qkv], proj[..., ab0:ab0 + H], proj[..., ab0 + H:ab0 + 2 * H])
        conv = None if conv_w is None else (conv_w[:qd], conv_w[qd:2 * qd], conv_w[2 * qd:])
        u = None
        if n_steps > 1:  # the prologue kernel also forms the write vectors
            q, k, v, la, beta, _, u, _ = layer_prologue(*xs, A_log, dt_bias, H=H, DK=DK, DV=DV, b_bias=b_bias, conv=conv,
                                                        q_scale=q_scale, la_min=la_min, out_dtype=torch.bfloat16,
                                                        n_steps=n_steps, lam=lam_sp)
        else:
            q, k, v, la, beta, _ = layer_prologue(*xs, A_log, dt_bias, H=H, DK=DK, DV=DV, b_bias=b_bias, conv=conv,
                                                  q_scale=q_scale, la_min=la_min, out_dtype=torch.bfloat16)
        y, _ = _prefill_impl(q, k, u, v, la, None if u is not None else beta, None, False, torch.bfloat16, impl)
        g = proj[..., n_qkv:n_qkv + n_gate] if n_gate else None
        o = layer_epilogue(y, norm_w, g, eps=eps, out_dtype=proj.dtype)
        ctx.save_for_backward(proj, conv_w, A_log, dt_bias, b_bias, norm_w, q, k, v, la, beta, y, u, lam_sp)
        ctx.cfg = cfg
        return o

    @staticmethod
    def backward(ctx, do):
        proj, conv_w, A_log, dt_bias, b_bias, norm_w, q, k, v, la, beta, y, u, lam_sp = ctx.saved_tensors
        H, DK, DV, n_gate, q_scale, la_min, eps, impl, n_steps = ctx.cfg
        B, T, width = proj.shape
        qd = H * DK
        n_qkv = 2 * qd + H * DV
        ab0 = n_qkv + n_gate
        dproj = torch.empty_like(proj)
        if width > ab0 + 2 * H:
            dproj[..., ab0 + 2 * H:].zero_()
        g = proj[..., n_qkv:n_qkv + n_gate] if n_gate else None
        dy = torch.empty_like(y)
        dnorm = _run_epilogue_bwd(y, norm_w, g, do, dy, dproj[..., n_qkv:n_qkv + n_gate] if n_gate else None, eps)
        dlam = None
        if u is None:
            dq, dk, dbeta, dv, dla, _ = _prefill_bwd_impl(q, k, None, v, la, beta, None, dy, None, False)
        else:
            dq, dk, du, dv, dla, _ = _prefill_bwd_impl(q, k, u, v, la, None, None, dy, None, False)
            dbeta, dlam = write_vectors_bwd(k, beta, lam_sp, du, dk, n_steps)
        xs = (proj[..., :qd], proj[..., qd:2 * qd], proj[..., 2 * qd:n_qkv], proj[..., ab0:ab0 + H], proj[..., ab0 + H:ab0 + 2 * H])
        outs = (dproj[..., :qd], dproj[..., qd:2 * qd], dproj[..., 2 * qd:n_qkv], dproj[..., ab0:ab0 + H], dproj[..., ab0 + H:ab0 + 2 * H])
        ws = (None, None, None) if conv_w is None else tuple(w.t().contiguous() for w in (conv_w[:qd], conv_w[qd:2 * qd], conv_w[2 * qd:]))
        dws, dA, ddt, dbb = _run_prologue_bwd(xs, ws, A_log, dt_bias, b_bias, (dq, dk, dv, dla, dbeta), outs, H, DK, DV,
                                              q_scale, 1e-12, la_min, 1.0)
        dconv = None if conv_w is None else torch.cat([w.t() for w in dws], 0).to(conv_w.dtype)
        return (dproj, dconv, dA.to(A_log.dtype), ddt.to(dt_bias.dtype), None if dbb is None else dbb.to(b_bias.dtype),
                dnorm.to(norm_w.dtype), dlam, None)
