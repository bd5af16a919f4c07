"""The drop-in ``gdn`` mixer against fla's own GatedDeltaNet layer (fla 0.5.1,
fla/layers/gated_deltanet.py:201-316), the class archbench's ``gdn`` arch builds
(archbench/layers/fla.py:36-38).

One fla layer is built (float32 parameters), its state dict is loaded into this package's
GatedDeltaNet, and both run the same input on the GPU (fla on its Triton kernels, as the checker;
ours on the B200 kernels):

* T <= 64 in eval mode, where fla takes ``fused_recurrent_gated_delta_rule`` (float32 state and
  arithmetic): rel-L2 <= 1e-2 on the layer output.  The gap is this package's scan taking bf16
  q, k, v (about 2e-3 per element), as archbench's chunk path does (nsgdn.py:400-405);
* T = 256 in eval mode, where fla takes ``chunk_gated_delta_rule``: rel-L2 <= 3e-2.  fla's chunk
  kernels keep their per-chunk states and intermediates in the input dtype; at configuration 1
  in bf16 they differ from this package's kernel by 2.3e-2 rel-L2 while this package's kernel is
  within 3.7e-4 of the float64 oracle, so the looser bound here is fla's.

fla must import on the GPU host (it does on this pool's B200 image); without it the tests skip."""

import pytest
import torch

from archbench_b200.layers import GatedDeltaNet

pytestmark = pytest.mark.gpu


def _fla_layer():
    try:
        from fla.layers.gated_deltanet import GatedDeltaNet as FlaGatedDeltaNet
    except Exception as e:  # pragma: no cover - depends on the host image
        pytest.skip(f"fla unavailable: {e!r}")
    return FlaGatedDeltaNet


@pytest.mark.parametrize("expand_v", [1.0, 2.0])
@pytest.mark.parametrize("T,tol", [(64, 1e-2), (37, 1e-2), (256, 3e-2)])
def test_gdn_layer_matches_fla_layer(expand_v, T, tol):
    Fla = _fla_layer()
    torch.manual_seed(11)
    kw = dict(hidden_size=256, expand_v=expand_v, head_dim=128, num_heads=2, mode="chunk", use_gate=True,
              use_short_conv=True, conv_size=4)
    ref = Fla(**kw).cuda().eval()
    ours = GatedDeltaNet(**kw).cuda().eval()
    missing, unexpected = ours.load_state_dict(ref.state_dict(), strict=True)
    assert not missing and not unexpected
    x = torch.randn(2, T, 256, device="cuda", generator=torch.Generator(device="cuda").manual_seed(12))
    with torch.no_grad():
        y_ref = ref(x)[0].float()
        y = ours(x).float()
    torch.cuda.synchronize()
    d = (y - y_ref).double()
    rel = (d.norm() / y_ref.double().norm()).item()
    assert rel <= tol, f"T={T} expand_v={expand_v}: rel-L2 {rel:.3e} (max-abs {d.abs().max().item():.3e})"


def test_gdn_layer_decode_continues_fla_prefill_output():
    """Our layer's cached decode steps against fla's layer run over the whole sequence."""
    from archbench_b200.layers import GDNCache

    Fla = _fla_layer()
    torch.manual_seed(13)
    kw = dict(hidden_size=256, expand_v=1.0, head_dim=128, num_heads=2, mode="chunk")
    ref = Fla(**kw).cuda().eval()
    ours = GatedDeltaNet(**kw).cuda().eval()
    ours.load_state_dict(ref.state_dict())
    T0, steps = 40, 8
    x = torch.randn(2, T0 + steps, 256, device="cuda", generator=torch.Generator(device="cuda").manual_seed(14))
    with torch.no_grad():
        y_ref = ref(x)[0].float()  # T <= 64: fla's fused recurrent path
        cache = GDNCache()
        ys = [ours(x[:, :T0], cache=cache)]
        for t in range(T0, T0 + steps):
            ys.append(ours(x[:, t:t + 1], cache=cache))
        y = torch.cat(ys, 1).float()
    d = (y - y_ref).double()
    rel = (d.norm() / y_ref.double().norm()).item()
    assert rel <= 1e-2, f"rel-L2 {rel:.3e}"
