"""Synthetic global batches and their per-rank microbatch inputs.

Two workloads:
* fixed: ``num_seqs`` documents of ``seq_len`` tokens;
* log-normal: documents with log-normal lengths (median, sigma), clipped to
  ``[lo, hi]`` and rounded up to the CP alignment, drawn until the batch holds
  ``total_tokens`` tokens (seeded).
Token ids are uniform over the vocabulary; labels are the next token of the
same document stream (the last label wraps to the first token); every token
carries loss weight ``1 / global_loss_tokens`` (per-token loss over the update).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from ..planner.joint.ir import spans


@dataclass
class GlobalBatch:
    lengths: dict[int, int]
    tokens: dict[int, torch.Tensor]     # host int64 [L] (pinned when built for CUDA)
    labels: dict[int, torch.Tensor]
    loss_tokens: int
    masks: dict[int, torch.Tensor] | None = None   # optional per-token loss mask (1 = counted)

    @property
    def total_tokens(self) -> int:
        return sum(self.lengths.values())


def fixed_lengths(num_seqs: int, seq_len: int) -> list[int]:
    return [seq_len] * num_seqs


def lognormal_lengths(total_tokens: int, median: int, sigma: float, lo: int, hi: int, align: int,
                      seed: int) -> list[int]:
    rng = np.random.default_rng(seed)
    out, acc = [], 0
    while acc < total_tokens:
        n = int(round(math.exp(math.log(median) + sigma * rng.standard_normal())))
        n = max(lo, min(hi, n))
        n = (n + align - 1) // align * align
        n = min(n, total_tokens - acc) if total_tokens - acc >= lo else n
        n = max(align, n // align * align)
        out.append(n)
        acc += n
    return out


def make_batch(lengths: list[int], vocab: int, seed: int, pin: bool = False) -> GlobalBatch:
    gen = torch.Generator(device="cpu")
    gen.manual_seed(seed)
    toks, labs = {}, {}
    for i, n in enumerate(lengths):
        t = torch.randint(0, vocab, (n,), generator=gen, dtype=torch.int64)
        l = torch.roll(t, -1)
        if pin:
            t, l = t.pin_memory(), l.pin_memory()
        toks[i], labs[i] = t, l
    return GlobalBatch(dict(enumerate(lengths)), toks, labs, sum(lengths))


@dataclass
class HostInputs:
    tokens: torch.Tensor
    labels: torch.Tensor
    weights: torch.Tensor

    def to(self, device, non_blocking=True) -> "HostInputs":
        return HostInputs(self.tokens.to(device, non_blocking=non_blocking),
                          self.labels.to(device, non_blocking=non_blocking),
                          self.weights.to(device, non_blocking=non_blocking))

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.tokens, self.labels, self.weights))


def local_inputs(batch: GlobalBatch, ingress_layout, world: int, rank: int, pin: bool = False) -> HostInputs:
    """This rank's ingress-ordered tokens, labels and loss weights (host tensors)."""
    rows = spans(ingress_layout, batch.lengths, world)[rank]
    t = torch.cat([batch.tokens[s][b:b + c] for s, b, _, c in rows]) if rows else torch.empty(0, dtype=torch.int64)
    l = torch.cat([batch.labels[s][b:b + c] for s, b, _, c in rows]) if rows else torch.empty(0, dtype=torch.int64)
    if batch.masks is None:
        w = torch.full((t.numel(),), 1.0 / batch.loss_tokens, dtype=torch.float32)
    else:
        m = torch.cat([batch.masks[s][b:b + c] for s, b, _, c in rows]) if rows else torch.empty(0)
        w = m.float() / batch.loss_tokens
    if pin:
        t, l, w = t.pin_memory(), l.pin_memory(), w.pin_memory()
    return HostInputs(t, l, w)


def manifest_batch(manifest: dict, pin: bool = False) -> GlobalBatch:
    """Whole-update batch of a ``joint_cp_inputs_v1`` manifest (LCG64 content, first-half loss mask)."""
    from ..planner.content import vector_fields
    toks, labs, masks = {}, {}, {}
    for s in manifest["samples"]:
        f = vector_fields(manifest, s["sample_id"], torch.arange(s["length"]))
        t, l, m = f["tokens"], f["labels"], f["loss_mask"] > 0
        if pin:
            t, l = t.pin_memory(), l.pin_memory()
        toks[s["sample_id"]], labs[s["sample_id"]], masks[s["sample_id"]] = t, l, m
    lengths = {s["sample_id"]: s["length"] for s in manifest["samples"]}
    return GlobalBatch(lengths, toks, labs, manifest["loss_tokens"], masks)
