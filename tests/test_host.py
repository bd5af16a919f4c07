"""Host-side logic that needs no GPU: layer construction and parameter names against the
reference's layers, the registry boundary, the custom-op fake implementations, sharding maths
and the bench's roofline arithmetic."""

import os
import sys

import pytest
import torch

from archbench_b200 import ops, registry, workloads
from archbench_b200.layers import GatedDeltaNet, NStepGDN
from archbench_b200.sharded import head_slice

# An archbench checkout, for the tests that import the reference's own layers (skipped without one;
# tests/test_layers_ref_gpu.py::test_layer_params_digest pins the parameter names and shapes
# through committed fixtures instead).
REF = os.environ.get("ARCHBENCH_REFERENCE", "")


def reference_nsgdn():
    if not REF or not os.path.isdir(REF):
        pytest.skip("no archbench checkout (set ARCHBENCH_REFERENCE)")
    if REF not in sys.path:
        sys.path.insert(0, REF)
    from archbench.layers.nsgdn import NStepGDN as RefNStepGDN

    return RefNStepGDN


@pytest.mark.parametrize("kw", [dict(), dict(expand_v=1.0, n_steps=1), dict(use_gate=False, conv_size=2), dict(num_heads=4, head_dim=64)])
def test_nsgdn_parameters_match_reference(kw):
    Ref = reference_nsgdn()
    torch.manual_seed(0)
    ours = NStepGDN(256, **kw)
    ref = Ref(256, **kw)
    a = {k: tuple(v.shape) for k, v in ours.state_dict().items()}
    b = {k: tuple(v.shape) for k, v in ref.state_dict().items()}
    assert a == b
    ours.load_state_dict(ref.state_dict())  # interchangeable checkpoints


def test_nsgdn_constructor_validation_matches_reference():
    for bad in (dict(head_dim=96), dict(n_steps=0), dict(lam=0.0), dict(scan_impl="nope")):
        with pytest.raises(ValueError):
            NStepGDN(128, **bad)


def test_gdn_parameter_names_match_fla():
    m = GatedDeltaNet(hidden_size=256, expand_v=2, head_dim=128, num_heads=2)
    names = set(m.state_dict())
    for n in ("q_proj.weight", "k_proj.weight", "v_proj.weight", "a_proj.weight", "b_proj.weight", "A_log", "dt_bias",
              "q_conv1d.weight", "k_conv1d.weight", "v_conv1d.weight", "g_proj.weight", "o_norm.weight", "o_proj.weight"):
        assert n in names, n
    assert tuple(m.q_conv1d.weight.shape) == (256, 1, 4)
    assert tuple(m.v_proj.weight.shape) == (512, 256)


def test_registry_builders_and_wrapper():
    m = registry.build_mixer("gdn", d_model=256, layer_idx=0, n_layer=2, head_dim=128, expand_v=1.0, num_heads=2)
    assert hasattr(m, "layer") and isinstance(m.layer, GatedDeltaNet)
    n = registry.build_mixer("nsgdn", d_model=256, layer_idx=0, n_layer=2, head_dim=128, expand_v=1.0, num_heads=2, n_steps=1)
    assert isinstance(n, NStepGDN)
    with pytest.raises(KeyError):
        registry.build_mixer("mamba", 256, 0, 1)


def test_registry_installs_into_archbench():
    reference_nsgdn()
    from archbench import layers as L

    saved = dict(L._REGISTRY)
    try:
        registry.install()
        m = L.build_mixer("nsgdn", 256, 0, 2, head_dim=128, expand_v=1.0, num_heads=2)
        assert isinstance(m, NStepGDN)
        g = L.build_mixer("gdn", 256, 0, 2, head_dim=128, expand_v=1.0, num_heads=2)
        assert isinstance(g.layer, GatedDeltaNet)
    finally:
        L._REGISTRY.clear()
        L._REGISTRY.update(saved)


def test_fake_impls_give_output_metadata():
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        q = torch.empty(2, 64, 4, 128, dtype=torch.bfloat16)
        la = torch.empty(2, 64, 4)
        y, s = torch.ops.archbench_b200.prefill(q, q, None, q, la, la, None, True, 1, "auto")
        assert y.shape == (2, 64, 4, 128) and y.dtype == torch.bfloat16 and s.shape == (2, 4, 128, 128)
        st = torch.empty(2, 4, 128, 128)
        yd = torch.ops.archbench_b200.decode_step(q[:, 0], q[:, 0], None, q[:, 0], la[:, 0], la[:, 0], st, 0)
        assert yd.shape == (2, 4, 128) and yd.dtype == torch.float32


def test_head_slices_partition_heads():
    H, world = 32, 8
    seen = []
    for r in range(world):
        s = head_slice(H, r, world)
        seen += list(range(H))[s]
    assert seen == list(range(H))
    with pytest.raises(ValueError):
        head_slice(30, 0, 8)


def test_algorithmic_counts():
    assert workloads.prefill_flops_per_token_head(128, 128, 64) == 180224
    assert workloads.prefill_bytes_per_token_head(128, 128) == 1032
    assert workloads.decode_bytes_per_token_head(128, 128) == 132104


def test_config_table_matches_baseline():
    c = workloads.CONFIGS
    assert (c["cfg1"].B, c["cfg1"].T, c["cfg1"].H, c["cfg1"].DK) == (8, 4096, 8, 128)
    assert (c["cfg2"].B, c["cfg2"].H) == (256, 16)
    assert (c["cfg3"].B, c["cfg3"].T, c["cfg3"].H) == (1, 65536, 32)


def test_bind_caches_host_checks():
    """Cache binding is host logic: every mixer must carry state; smear must be off."""
    import torch.nn as nn

    from archbench_b200.decode import bind_caches
    from archbench_b200.registry import build_mixer

    class Blk(nn.Module):
        def __init__(self, mixer):
            super().__init__()
            self.mixer = mixer

    m = nn.Module()
    m.blocks = nn.ModuleList([Blk(build_mixer("nsgdn", 256, 0, 2, num_heads=2, head_dim=128)),
                              Blk(build_mixer("gdn", 256, 1, 2, num_heads=2, head_dim=128))])
    m.smear_gate = None
    with bind_caches(m) as caches:
        assert len(caches) == 2
        assert m.blocks[0].mixer.bound_cache is caches[0] and m.blocks[1].mixer.layer.bound_cache is caches[1]
        with pytest.raises(RuntimeError):
            with bind_caches(m):
                pass
    assert m.blocks[0].mixer.bound_cache is None and m.blocks[1].mixer.layer.bound_cache is None
    m.smear_gate = nn.Linear(24, 1)
    with pytest.raises(ValueError, match="smear"):
        with bind_caches(m):
            pass
    m.smear_gate = None
    m.blocks.append(Blk(nn.Linear(256, 256)))
    with pytest.raises(ValueError, match="no recurrent state"):
        with bind_caches(m):
            pass


def test_nstep_write_direction_matches_golden():
    """The torch restatement of the write vectors (the autograd reference of the write-vector
    backward kernel's parity test) against the reference's own output in tests/golden."""
    import numpy as np

    from archbench_b200.nstep import write_direction

    d = np.load(os.path.join(os.path.dirname(__file__), "golden", "nstep_small.npz"))
    k = torch.from_numpy(d["k"]).double()
    p = torch.nn.functional.pad(k[:, :-1], (0, 0, 0, 0, 1, 0))
    u = write_direction(k, p, torch.from_numpy(d["beta"]).double(), torch.from_numpy(d["lam"]).double(), 2)
    assert torch.allclose(u, torch.from_numpy(d["u"]).double(), rtol=0, atol=1e-6)
