"""Plan-driven executor: runs one microbatch of a joint plan through the model.

For every layer the hidden rows are resharded from the previous layer's
attention layout to this layer's attention layout (identity routes are free),
the mixer runs with its ``LocalLayout`` (ring attention / GDN state passing
over the layer's CP team), the MLP optionally runs in its own placement, and
before the head the rows return to the ingress layout so labels and loss
weights line up (reference: joint_cp/adapter.py:125-186, without Megatron
monkeypatching). Local layouts are cached per (layout, lengths).
"""

from __future__ import annotations

import torch
import torch.utils.checkpoint

from ..parallel.layout import LocalLayout
from ..parallel.transport import move
from ..planner.joint.ir import Microbatch
from ..utils.tracing import nvtx


class LayoutCache:
    def __init__(self, world: int, rank: int, device, teams=None):
        self.world, self.rank, self.device, self.teams = world, rank, device, teams
        self._cache: dict = {}

    def get(self, layout, lengths: dict) -> LocalLayout:
        key = (layout, tuple(sorted(lengths.items())))
        hit = self._cache.get(key)
        if hit is None:
            if len(self._cache) > 4096:
                self._cache.clear()
            hit = LocalLayout(layout, lengths, self.world, self.rank, self.device, self.teams)
            self._cache[key] = hit
        return hit


class MicrobatchRun:
    """One microbatch of a plan on this rank. With ``recompute_tokens`` set, a microbatch that
    holds more tokens than that on some rank (in any of its layouts) keeps only each layer's input
    and recomputes the layer's forward in the backward (the cost model prices the same rule,
    ``joint.cost.Model.recompute_tokens``)."""

    def __init__(self, mb: Microbatch, lengths: dict, cache: LayoutCache, first_layer: int = 0,
                 num_layers: int | None = None, recompute_tokens: int | None = None):
        self.lengths = {s: lengths[s] for g in mb.ingress.groups for s in g.samples}
        self.ingress = cache.get(mb.ingress, self.lengths)
        layers = mb.layers[first_layer:first_layer + num_layers] if num_layers else mb.layers[first_layer:]
        self.contexts = [cache.get(a, self.lengths) for a, _ in layers]
        self.mlp_contexts = [None if m == a else cache.get(m, self.lengths) for a, m in layers]
        self.recompute = recompute_tokens is not None and recomputes(mb, self.lengths, cache.world,
                                                                     recompute_tokens)

    def forward_layers(self, model, x, start_ctx=None):
        prev = start_ctx or self.ingress
        for i, (layer, ctx, mctx) in enumerate(zip(model.layers, self.contexts, self.mlp_contexts)):
            if ctx is not prev:
                with nvtx(f"route cp{getattr(prev, 'cp', '?')}->cp{getattr(ctx, 'cp', '?')}"):
                    x = move(x, prev, ctx)
            with nvtx(f"layer {i} {type(layer).__name__} cp{getattr(ctx, 'cp', '?')}"):
                if self.recompute and x.requires_grad:
                    x = torch.utils.checkpoint.checkpoint(layer, x, ctx, mctx, use_reentrant=False)
                else:
                    x = layer(x, ctx, mctx)
            prev = ctx
        return x, prev

    def forward(self, model, tokens, labels, weights, packet=None, version: int = 0):
        """Loss of this microbatch; ``packet`` (an ``audits.PacketAccounting``) counts the forward
        at the embedding output and samples memory at forward end and around the loss."""
        x = model.embed(tokens)
        if packet is not None:
            x = packet.forward(x, version)
        x, prev = self.forward_layers(model, x)
        x = move(x, prev, self.ingress)
        if packet is None:
            return model.loss(x, labels, weights)
        packet.sample("F_end", packet.forwards)
        packet.sample("CE_before", packet.forwards)
        out = model.loss(x, labels, weights)
        packet.sample("CE_after", packet.forwards)
        return out


def recomputes(mb: Microbatch, lengths: dict, world: int, limit: int) -> bool:
    """Whether some rank holds more than ``limit`` tokens of ``mb`` in one of its layouts."""
    layouts = [mb.ingress] + [x for pair in mb.layers for x in pair]
    return max(max(x.tokens(lengths, world)) for x in layouts) > limit
