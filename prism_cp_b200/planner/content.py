"""Deterministic synthetic token content (``lcg64_next_token_v1``).

Every sample has its own stream of a 64-bit linear congruential generator
``x <- a x + c (mod 2^64)`` with the PCG/Knuth MMIX constants, starting at the
manifest seed advanced by ``sample_id * 2^32`` steps. Token at position ``p``
is ``(state_{p+1} >> 32) % vocab``; the label is the token at ``p + 1`` of the
same stream. Jump-ahead uses the standard O(log n) composition of affine maps
(Brown, "Random number generation with arbitrary strides", 1994), so any span
of any sample is generated without touching the rest.

The constants, stream stride and token/label rule match the reference's frozen
content rule (experiments/sequence_dynamic_cp/two_dimensional_inputs.py:3-44)
so that manifests and packets are interchangeable.
"""

from __future__ import annotations

from functools import lru_cache

MODULUS = 1 << 64
MULTIPLIER = 6364136223846793005
INCREMENT = 1442695040888963407
SAMPLE_STRIDE = 1 << 32
MASK = MODULUS - 1


def affine_power(steps: int, mult: int = MULTIPLIER, inc: int = INCREMENT) -> tuple[int, int]:
    """(A, C) with x_{n+steps} = A x_n + C (mod 2^64)."""
    if steps < 0:
        raise ValueError("negative stream offset")
    acc_a, acc_c = 1, 0
    a, c = mult, inc
    while steps:
        if steps & 1:
            acc_a, acc_c = (acc_a * a) & MASK, (acc_c * a + c) & MASK
        a, c = (a * a) & MASK, (c * (a + 1)) & MASK
        steps >>= 1
    return acc_a, acc_c


def advance(state: int, steps: int) -> int:
    a, c = affine_power(steps)
    return (a * state + c) & MASK


def materialize_span(manifest: dict, sample_id: int, start: int, stop: int) -> dict:
    """Tokens, labels, positions and loss mask of one sample slice (plain lists)."""
    sample = next((s for s in manifest["samples"] if s["sample_id"] == sample_id), None)
    if sample is None or not 0 <= start <= stop <= sample["length"]:
        raise ValueError("invalid sample or span bounds")
    rule = manifest["content_rule"]
    state = advance(rule["initial_state"], sample_id * SAMPLE_STRIDE + start + 1)
    stream = []
    for _ in range(stop - start + 1):
        stream.append((state >> 32) % rule["vocab_size"])
        state = (state * MULTIPLIER + INCREMENT) & MASK
    return {"tokens": stream[:-1], "labels": stream[1:], "positions": list(range(start, stop)),
            "loss_mask": [int(p < sample["loss_prefix_tokens"]) for p in range(start, stop)]}


# ---------------------------------------------------------------- vectorised (torch)
def _signed(v: int) -> int:
    v &= MASK
    return v - MODULUS if v >= MODULUS // 2 else v


def _jump_table(count: int, stride: int):
    """Per-index affine coefficients for index*stride steps (int64 wrap == mod 2^64)."""
    import torch
    idx = torch.arange(count, dtype=torch.int64)
    mul = torch.ones(count, dtype=torch.int64)
    add = torch.zeros(count, dtype=torch.int64)
    a, c = affine_power(stride)
    bit = 1
    while bit < count:
        sel = (idx & bit) != 0
        mul = torch.where(sel, mul * _signed(a), mul)
        add = torch.where(sel, add * _signed(a) + _signed(c), add)
        a, c = (a * a) & MASK, (c * (a + 1)) & MASK
        bit <<= 1
    return mul, add


@lru_cache(maxsize=1)
def _low_table():
    return _jump_table(256, 1)


def vector_fields(manifest: dict, sample_id: int, positions, device="cpu") -> dict:
    """Fields at arbitrary positions with O(N) tensor work (256-entry low table +
    a high table of O(max_position / 256) entries)."""
    import torch
    sample = next((s for s in manifest["samples"] if s["sample_id"] == sample_id), None)
    if sample is None:
        raise ValueError("unknown stable sample ID")
    pos = torch.as_tensor(positions, dtype=torch.int64, device="cpu").reshape(-1)
    if pos.numel() and (bool((pos < 0).any()) or bool((pos >= sample["length"]).any())):
        raise ValueError("sample position outside length")
    rule = manifest["content_rule"]
    base = advance(rule["initial_state"], sample_id * SAMPLE_STRIDE)
    off = pos + 1
    hi, lo = off // 256, off % 256
    hmul, hadd = _jump_table(int(hi.max()) + 1 if hi.numel() else 1, 256)
    lmul, ladd = _low_table()
    states = (_signed(base) * hmul[hi] + hadd[hi]) * lmul[lo] + ladd[lo]
    vocab = rule["vocab_size"]
    tokens = ((states >> 32) & 0xFFFFFFFF) % vocab
    nxt = states * _signed(MULTIPLIER) + _signed(INCREMENT)
    labels = ((nxt >> 32) & 0xFFFFFFFF) % vocab
    return {"tokens": tokens.to(device), "labels": labels.to(device), "position_ids": pos.to(device),
            "loss_mask": (pos < sample["loss_prefix_tokens"]).float().to(device)}
