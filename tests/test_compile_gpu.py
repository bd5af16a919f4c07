"""The drop-in mixers under ``torch.compile``, as archbench's trainer runs its model
(archbench/trainer.py:94-95: ``torch.compile(model, dynamic=False)``): a training step (loss and
parameter gradients) and an evaluation forward of a compiled two-block LM give the same results as
the eager model.  The token mixing and the layer prologue/epilogue stay opaque to the compiler
(``torch.library`` custom ops and autograd functions around this package's kernels); the
projections, norms and MLPs are compiled.  Tolerance: rel-L2 <= 1e-3 on the loss and <= 5e-3 on the
logits and every parameter gradient (fp32 weights; the compiled graph fuses and reorders the
elementwise work around the same kernels, and the mixer rounds q, k, v to bf16 for the chunk
kernel, so a one-ulp fp32 difference upstream can move a bf16 rounding: measured up to 1.05e-3)."""

import copy

import pytest
import torch

from archbench_b200.lm import LM

pytestmark = pytest.mark.gpu


def rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


@pytest.mark.parametrize("arch,layer", [
    ("nsgdn", dict(num_heads=2, head_dim=128, expand_v=1.0, n_steps=1)),
    ("nsgdn", dict(num_heads=2, head_dim=128, expand_v=2.0, n_steps=2)),
    ("gdn", dict(num_heads=2, head_dim=128, expand_v=1.0)),
])
def test_compiled_training_step_and_eval_match_eager(arch, layer):
    torch.manual_seed(51)
    eager = LM(arch=arch, d_model=256, n_layer=2, vocab_size=512, layer=layer).cuda()
    comp_model = copy.deepcopy(eager)
    compiled = torch.compile(comp_model, dynamic=False)
    g = torch.Generator(device="cuda").manual_seed(52)
    idx = torch.randint(0, 512, (2, 192), device="cuda", generator=g)
    tgt = torch.randint(0, 512, (2, 192), device="cuda", generator=g)

    _, loss_e = eager(idx, tgt)
    loss_e.backward()
    _, loss_c = compiled(idx, tgt)
    loss_c.backward()
    assert rel(loss_c.detach(), loss_e.detach()) <= 1e-3
    pe = dict(eager.named_parameters())
    for n, p in comp_model.named_parameters():
        if pe[n].grad is None:
            assert p.grad is None, n
            continue
        assert p.grad is not None, n
        assert rel(p.grad, pe[n].grad) <= 5e-3, (n, rel(p.grad, pe[n].grad))

    with torch.no_grad():
        eager.eval()
        compiled.eval()
        le, _ = eager(idx)
        lc, _ = compiled(idx)
    assert rel(lc, le) <= 5e-3
