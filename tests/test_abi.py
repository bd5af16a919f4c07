"""The C-ABI library: it loads, exports every symbol include/gdn_b200.h declares, and its
host-side argument checks answer without a GPU (no compute call is made here)."""

import ctypes
import os
import re

import pytest

from archbench_b200 import ops

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gdn_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(gdn_\w+)\s*\(", src, flags=re.M)))


def test_header_declares_the_expected_api():
    assert declared_functions() == sorted(ops.SYMBOLS), declared_functions()


def test_library_exports_every_declared_symbol():
    lib = ops.load_library()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert lib.gdn_abi_version() == 2


def test_struct_layout_matches_header():
    # pointers 9*8, strides 5*24, sizes 5*8, ints 4*4
    assert ctypes.sizeof(ops.PrefillArgs) == 9 * 8 + 5 * 24 + 5 * 8 + 4 * 4 + 8 + 8
    assert ctypes.sizeof(ops.DecodeArgs) == 8 * 8 + 5 * 24 + 4 * 8 + 2 * 4
    # pointers 22*8, int64 18*8, 4 int32 + 4 float
    assert ctypes.sizeof(ops.PrologueArgs) == 22 * 8 + 18 * 8 + 4 * 4 + 4 * 4 + 4 * 8 + 2 * 4
    assert ctypes.sizeof(ops.WriteVectorsBwdArgs) == 7 * 8 + 4 * 8 + 2 * 4
    assert ctypes.sizeof(ops.EpilogueArgs) == 4 * 8 + 24 + 8 * 8 + 3 * 4 + 4


def test_layer_io_argument_checks():
    lib = ops.load_library()
    a = ops.PrologueArgs()
    assert lib.gdn_layer_prologue(ctypes.byref(a), None) == -1
    e = ops.EpilogueArgs()
    assert lib.gdn_layer_epilogue(ctypes.byref(e), None) == -1
    assert lib.gdn_layer_prologue(None, None) == -1 and lib.gdn_layer_epilogue(None, None) == -1
    # all pointers set (never dereferenced), bad conv size and head size answer before any device use
    ptrs = {n: 0x10000 * (i + 1) for i, n in enumerate(("xq", "xk", "xv", "xa", "xb", "A_log", "dt_bias", "q", "k", "v", "la", "beta"))}
    a = ops.PrologueArgs(**ptrs, B=1, T=8, H=2, DK=128, DV=128, conv_size=9, in_dtype=1, out_dtype=1)
    assert lib.gdn_layer_prologue(ctypes.byref(a), None) == -2
    a.conv_size, a.DK = 4, 96
    assert lib.gdn_layer_prologue(ctypes.byref(a), None) == -2
    a.DK, a.in_dtype = 128, 7
    assert lib.gdn_layer_prologue(ctypes.byref(a), None) == -3
    e = ops.EpilogueArgs(y=0x10000, weight=0x20000, o=0x30000, B=1, T=1, H=1, DV=100, y_dtype=1, g_dtype=1, o_dtype=1)
    assert lib.gdn_layer_epilogue(ctypes.byref(e), None) == -2


def fake_args(**kw):
    """Valid-looking prefill args with fake (never dereferenced) 256-aligned pointers."""
    B, T, H, DK, DV = kw.pop("shape", (2, 128, 4, 128, 128))
    st = ops.Strides(T * H * DK, H * DK, DK)
    a = ops.PrefillArgs(
        0x10000, 0x20000, None, 0x30000, 0x40000, 0x50000, None, 0x60000, None,
        st, st, ops.Strides(0, 0, 0), ops.Strides(T * H * DV, H * DV, DV), ops.Strides(T * H * DV, H * DV, DV),
        B, T, H, DK, DV, ops.GDN_DTYPE_BF16, ops.GDN_DTYPE_BF16, 0, 0, None, 0,
    )
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def status(a):
    return ops.load_library().gdn_prefill_select_impl(ctypes.byref(a))


def test_validation_codes():
    assert status(fake_args()) in (2, 4, 5)
    assert status(fake_args(q=None)) == -1
    assert status(fake_args(beta=None)) == -1  # no u and no beta
    assert status(fake_args(B=0)) == -2
    assert status(fake_args(T=-1)) == -2
    assert status(fake_args(DK=96)) == -5
    assert status(fake_args(DV=0)) == -5
    assert status(fake_args(in_dtype=7)) == -3
    assert status(fake_args(impl=9)) == -5
    assert status(fake_args(impl=7)) == -5
    assert status(fake_args(impl=6)) == -2  # the split path without its workspace
    assert status(fake_args(q=0x10002)) == -4  # misaligned vector loads


def test_recurrent_selected_for_fp32_and_small_heads():
    assert status(fake_args(in_dtype=ops.GDN_DTYPE_F32, out_dtype=ops.GDN_DTYPE_F32)) == 2
    assert status(fake_args(shape=(2, 64, 4, 64, 64))) == 2
    assert status(fake_args(shape=(2, 64, 4, 64, 64), impl=1)) == -5  # chunk forced, not covered
    assert status(fake_args(impl=3)) == -5  # segmented forced where it does not apply


def test_chunk_variant_selection():
    # DV = 128, u = beta k: the two-CTA cluster kernel; "chunk" resolves to it
    assert status(fake_args()) == 4
    assert status(fake_args(impl=1)) == 4
    assert status(fake_args(impl=4)) == 4
    assert status(fake_args(impl=5)) == 5
    # DV = 256 or an explicit write vector: only the single-CTA kernel
    wide = (2, 128, 4, 128, 256)
    assert status(fake_args(shape=wide)) == 5
    assert status(fake_args(shape=wide, impl=4)) == -5
    st = ops.Strides(128 * 4 * 128, 4 * 128, 128)
    assert status(fake_args(u=0x70000, su=st)) == 5
    assert status(fake_args(u=0x70000, su=st, impl=4)) == -5


def test_workspace_query():
    lib = ops.load_library()
    n = ctypes.c_size_t(123)
    # 64 (b, h) units on a 148-SM part: the single-pass kernel, no workspace
    assert lib.gdn_prefill_workspace_bytes(ctypes.byref(fake_args()), ctypes.byref(n)) == 0
    assert n.value == 0
    # one long sequence: segmented, (P - 1) slots of (DV + 128) x 128 fp32
    a = fake_args(shape=(1, 4096, 2, 128, 128))
    assert lib.gdn_prefill_workspace_bytes(ctypes.byref(a), ctypes.byref(n)) == 0
    assert n.value > 0 and n.value % (256 * 128 * 4 * 2) == 0
    assert status(a) == 4  # no workspace supplied: the single-pass (cluster) chunk kernel
    a.workspace, a.workspace_bytes = 0x100000, n.value
    assert status(a) == 3
    a.impl = 3
    a.workspace_bytes = n.value - 1
    assert status(a) == -2


def test_cluster_kernel_preferred_over_segments_for_enough_sequences():
    lib = ops.load_library()
    n = ctypes.c_size_t(123)
    # 32 (b, h) units on 148 SMs (configuration 3 on one GPU): the cluster kernel, no workspace
    a = fake_args(shape=(1, 65536, 32, 128, 128))
    assert lib.gdn_prefill_workspace_bytes(ctypes.byref(a), ctypes.byref(n)) == 0
    assert n.value == 0
    assert status(a) == 4
    # the segmented path still plans when asked for explicitly
    a.impl = 3
    assert lib.gdn_prefill_workspace_bytes(ctypes.byref(a), ctypes.byref(n)) == 0
    assert n.value > 0


def test_status_strings():
    lib = ops.load_library()
    for s in range(-8, 1):
        assert lib.gdn_status_string(s) and b"unknown" not in lib.gdn_status_string(s)


def test_null_args_rejected_before_device_use():
    lib = ops.load_library()
    assert lib.gdn_prefill_fwd(None, None) == -1
    assert lib.gdn_decode_step(None, None) == -1


def test_ops_refuse_cpu_tensors():
    import torch

    x = torch.zeros(1, 4, 1, 32)
    with pytest.raises(ValueError, match="CUDA"):
        ops.gdn_prefill(x, x, x, torch.zeros(1, 4, 1), beta=torch.zeros(1, 4, 1))


def test_split_path_workspace_and_selection():
    """DV > 128 (or explicit write vectors) under auto: the split path when the caller supplies the
    workspace gdn_prefill_workspace_bytes reports (24 KB per (b, h, chunk)), else the single-CTA kernel."""
    lib = ops.load_library()
    B, T, H, DV = 2, 130, 4, 256
    a = fake_args(shape=(B, T, H, 128, DV))
    need = ctypes.c_size_t(0)
    assert lib.gdn_prefill_workspace_bytes(ctypes.byref(a), ctypes.byref(need)) == 0
    assert need.value == B * H * 3 * 24576
    assert status(a) == 5  # no workspace: the single-CTA kernel
    a.workspace, a.workspace_bytes = 0x100000, need.value
    assert status(a) == 6
    a.workspace_bytes = need.value - 16
    assert status(a) == 5
    # DV = 128, u = beta k: the cluster kernel, no workspace
    b = fake_args(shape=(B, T, H, 128, 128))
    assert lib.gdn_prefill_workspace_bytes(ctypes.byref(b), ctypes.byref(need)) == 0 and need.value == 0
    assert status(b) == 4
    # the same with the split path requested
    b.impl = 6
    assert lib.gdn_prefill_workspace_bytes(ctypes.byref(b), ctypes.byref(need)) == 0
    assert need.value == B * H * 3 * 24576
    b.workspace, b.workspace_bytes = 0x100000, need.value
    assert status(b) == 6
