"""Recurrent-state cache plumbing for greedy decoding through an unmodified archbench LM.

archbench's ``LM.forward(idx)`` (archbench/model.py:122-149) calls every block's mixer as
``mixer(x)`` with no state argument, and its generation loop (archbench/core_eval.py:136-142)
re-runs the whole prefix for every new token.  ``bind_caches(model)`` gives every mixer of this
package in a model its own ``GDNCache`` for the duration of a ``with`` block; a mixer called without
an explicit cache uses the bound one.  Inside the block ``model(prompt)`` runs the prompt through
the chunked prefill and leaves each layer's recurrent state and conv state in its cache, and
``model(next_ids[:, None])`` then advances every layer by one token (the decode kernel and the conv
state) instead of re-running the prefix.  ``greedy_decode`` is that loop; ``GraphDecoder`` captures
its one-token step as a CUDA graph.

Only models whose token mixing all carries state this way can be decoded like this: every mixer
must be one of this package's layers, and archbench's embedding smear (a token shift over the
embeddings, model.py:131-133, which needs the previous token's embedding) must be off."""

from __future__ import annotations

import contextlib
from typing import Iterator, List

import torch
import torch.nn as nn

from .layers import GatedDeltaNet, GDNCache, NStepGDN


def _stateful_layers(model: nn.Module) -> List[nn.Module]:
    layers = [m for m in model.modules() if isinstance(m, (NStepGDN, GatedDeltaNet))]
    for name, m in model.named_modules():
        if name.split(".")[-1] == "mixer" and not any(l is m or any(l is c for c in m.modules()) for l in layers):
            raise ValueError(f"{name} ({type(m).__name__}) keeps no recurrent state across calls; "
                             "cached decoding needs every mixer to be a B200 gdn/nsgdn layer")
    if getattr(model, "smear_gate", None) is not None:
        raise ValueError("the embedding smear mixes each token with the previous one's embedding, "
                         "which a one-token call does not see; cached decoding needs smear off")
    if not layers:
        raise ValueError("model has no B200 gdn/nsgdn layers")
    return layers


@contextlib.contextmanager
def bind_caches(model: nn.Module) -> Iterator[List[GDNCache]]:
    """Bind a fresh ``GDNCache`` to every gdn/nsgdn layer of ``model`` (yielded in module order);
    the bindings are removed on exit."""
    layers = _stateful_layers(model)
    if any(l.bound_cache is not None for l in layers):
        raise RuntimeError("caches are already bound to this model")
    caches = [GDNCache() for _ in layers]
    for l, c in zip(layers, caches):
        l.bound_cache = c
    try:
        yield caches
    finally:
        for l in layers:
            l.bound_cache = None


def _logits(out) -> torch.Tensor:
    return out[0] if isinstance(out, (tuple, list)) else out


class GraphDecoder:
    """One greedy decode step of a model with bound, filled caches, captured once as a CUDA graph and
    replayed per token: the step's few hundred launches (projections, the layer kernels, the MLPs)
    then cost one graph launch instead of one host round trip each.

    ``token`` (B,) holds the current token; each ``step()`` runs the model on it, leaves the step's
    last-position logits in ``logits`` and the greedy next token in ``token``, and advances every
    cache by one token.  The caches are switched to static (in-place updates), so the captured
    kernels read and write the same state buffers on every replay.  Capturing does not advance the
    caches: the warm-up call that precedes the capture runs on saved copies, which are put back."""

    def __init__(self, model: nn.Module, caches: List[GDNCache], token: torch.Tensor):
        self.model = model
        self.token = token.clone()
        for c in caches:
            c.static = True
        saved = [(c.state.clone(), {k: v.clone() for k, v in c.conv.items()}, c.seen) for c in caches]
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):  # warm-up: cuBLAS handles, library state, allocator pool
            self._run()
        torch.cuda.current_stream().wait_stream(side)
        for c, (st, conv, seen) in zip(caches, saved):
            c.state.copy_(st)
            for k, v in conv.items():
                c.conv[k].copy_(v)
            c.seen = seen
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.logits = self._run()
        for c, (_, _, seen) in zip(caches, saved):  # the capture ran no kernel; undo its host bookkeeping
            c.seen = seen
        self.caches = caches

    def _run(self) -> torch.Tensor:
        logits = _logits(self.model(self.token[:, None]))[:, -1]
        self.token.copy_(logits.argmax(-1))
        return logits

    def step(self) -> torch.Tensor:
        self.graph.replay()
        for c in self.caches:
            c.seen += 1
        return self.logits


@torch.no_grad()
def greedy_decode(model: nn.Module, idx: torch.Tensor, steps: int, return_logits: bool = False, graph: bool = False):
    """Greedy continuation of ``idx`` (B, T) by ``steps`` tokens: one prefill call, then one
    one-token call per step through the bound caches (replays of one captured step with ``graph``).
    Returns the (B, T + steps) ids, and with ``return_logits`` also the (B, steps, vocab) logits each
    new token was chosen from."""
    if steps < 1:
        raise ValueError("steps must be >= 1")
    with bind_caches(model) as caches:
        logits = _logits(model(idx))[:, -1]
        toks, seen = [logits.argmax(-1)], [logits]
        if graph and steps > 1:
            dec = GraphDecoder(model, caches, toks[0])
            for _ in range(steps - 1):
                lg = dec.step()
                toks.append(dec.token.clone())
                if return_logits:
                    seen.append(lg.clone())
        else:
            for _ in range(steps - 1):
                logits = _logits(model(toks[-1][:, None]))[:, -1]
                toks.append(logits.argmax(-1))
                seen.append(logits)
    ids = torch.cat([idx, torch.stack(toks, 1)], 1)
    return (ids, torch.stack(seen, 1)) if return_logits else ids
