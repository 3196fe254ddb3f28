"""Input manifests (``joint_cp_inputs_v1``), whole-update packets and plan identities.

* ``build_manifest`` / ``validate_manifest``: explicit sample lengths with stable
  ids/uids, ``alignment_tokens = 2 * world`` and a loss mask on the first half
  of each sample; content is the LCG64 rule of ``content.py``. Field names and
  checks are the reference's (joint_cp/inputs.py:6-60) so manifests written by
  either tool validate in both.
* ``PacketSource``: repeats the same frozen whole-update packet every update
  (reference: two_dimensional_packet.py:76-123), producing per-rank inputs for
  the executor directly instead of patching a Megatron dataset.
* ``structural_identity``: reversible raw-DEFLATE encoding of a plan's packed
  shapes (reference: mixed_global_batch.py:8-14); ``fingerprint`` is its
  sha256 variant used by the measured-cost tables.
"""

from __future__ import annotations

import base64
import hashlib
import json
import zlib
from pathlib import Path

from .content import INCREMENT, MODULUS, MULTIPLIER, SAMPLE_STRIDE, vector_fields

CONTENT_RULE_NAME = "lcg64_next_token_v1"


def _content_rule(seed: int, vocab: int = 32768) -> dict:
    return {"name": CONTENT_RULE_NAME, "vocab_size": vocab, "initial_state": seed, "modulus": MODULUS,
            "multiplier": MULTIPLIER, "increment": INCREMENT, "sample_stride": SAMPLE_STRIDE,
            "token": "upper_32_bits_mod_vocab", "label": "token_at_position_plus_one_in_same_sample_stream",
            "position": "zero_based_sample_position", "loss_mask": "position < length // 2"}


def build_manifest(lengths, case_id: str, world: int, seed: int = 1234, vocab: int = 32768) -> dict:
    m = {"schema": "joint_cp_inputs_v1", "case_id": case_id, "world": world, "seed": seed,
         "variant": "frozen_lengths", "grouping_constraint": False, "alignment_tokens": 2 * world,
         "backend_alignments": {"joint_attention": 2 * world}, "input_tokens": sum(lengths),
         "loss_tokens": sum(n // 2 for n in lengths), "content_rule": _content_rule(seed, vocab),
         "samples": [{"sample_id": i, "sample_uid": f"{case_id}:{i:06d}", "length": n, "original_length": n,
                      "loss_prefix_tokens": n // 2} for i, n in enumerate(lengths)]}
    validate_manifest(m)
    return m


def validate_manifest(m: dict) -> None:
    if m.get("schema") != "joint_cp_inputs_v1" or m.get("variant") != "frozen_lengths":
        raise ValueError("Unknown joint input schema")
    world = m.get("world")
    if world not in (1, 2, 4, 8, 16, 32) or type(m.get("seed")) is not int or not 0 <= m["seed"] < MODULUS:
        raise ValueError("Invalid joint world or seed")
    if m.get("grouping_constraint") is not False or m.get("alignment_tokens") != 2 * world:
        raise ValueError("Joint grouping/alignment contract changed")
    if m.get("backend_alignments") != {"joint_attention": 2 * world}:
        raise ValueError("Joint backend alignment changed")
    samples = m.get("samples", [])
    if not samples or [s["sample_id"] for s in samples] != list(range(len(samples))):
        raise ValueError("Joint input must contain ascending unique sample IDs")
    for s in samples:
        n = s["length"]
        if (type(n) is not int or n <= 0 or n % (2 * world) or n >= SAMPLE_STRIDE - 1
                or s["original_length"] != n or s["loss_prefix_tokens"] != n // 2
                or s["sample_uid"] != f"{m['case_id']}:{s['sample_id']:06d}"):
            raise ValueError("Joint sample length, mask or identity changed")
    if m["content_rule"] != _content_rule(m["seed"], m["content_rule"].get("vocab_size", 32768)):
        raise ValueError("Joint deterministic content rule changed")
    if (m["input_tokens"] != sum(s["length"] for s in samples)
            or m["loss_tokens"] != sum(s["loss_prefix_tokens"] for s in samples)):
        raise ValueError("Joint token total changed")


def packet_launch_metadata(manifest: dict, world: int, capacity: int) -> tuple:
    """(micro batch, sequence capacity, tokens per rank, input tokens, loss tokens, alignment, fixture)."""
    validate_manifest(manifest)
    if world != manifest.get("world", 16) or capacity <= 0:
        raise ValueError("Packet launch world/capacity mismatch")
    if max(s["length"] for s in manifest["samples"]) > world * capacity:
        raise ValueError("Ingress allocation cannot hold the longest sample")
    return (1, world * capacity, manifest["input_tokens"] // world, manifest["input_tokens"],
            manifest["loss_tokens"], str(2 * world),
            {"mode": "packed_cp_case", "lengths": [2 * world], "prompt_lengths": [world]})


class PacketSource:
    """The same frozen whole-update packet for every update of a run."""

    def __init__(self, manifest, updates: int):
        if type(updates) is not int or updates <= 0:
            raise ValueError("updates must be a positive integer")
        if isinstance(manifest, (str, Path)):
            manifest = json.loads(Path(manifest).read_text())
        validate_manifest(manifest)
        self.manifest = manifest
        self.updates = updates
        self.lengths = {s["sample_id"]: s["length"] for s in manifest["samples"]}
        self.streams = [{"id": "TWO_DIMENSIONAL", "updates": [
            {"update": u + 1, "input_tokens": manifest["input_tokens"], "loss_tokens": manifest["loss_tokens"],
             "recipe_ids": [], "logical_sample_ids": list(self.lengths), "repeat_same_frozen_samples": True}
            for u in range(updates)]}]

    def __len__(self):
        return self.updates

    def fields(self, sample_id: int, positions, device="cpu") -> dict:
        return vector_fields(self.manifest, sample_id, positions, device)

    def rank_inputs(self, update: int, ingress_layout, world: int, rank: int, device="cpu"):
        """Ingress-ordered (tokens, labels, positions, loss weights) of one rank for one update."""
        import torch
        from .joint.ir import spans
        if not 1 <= update <= self.updates:
            raise IndexError("whole-update packet exhausted")
        rows = spans(ingress_layout, self.lengths, world)[rank]
        parts = [self.fields(s, torch.arange(b, b + c), device) for s, b, _, c in rows]
        cat = lambda key: torch.cat([p[key] for p in parts]) if parts else torch.empty(0)
        mask = cat("loss_mask")
        return cat("tokens"), cat("labels"), cat("position_ids"), mask / max(1, self.manifest["loss_tokens"])


def structural_identity(plan, lengths) -> str:
    """Reversible (raw DEFLATE, no checksum) encoding of packed shapes and placement."""
    shape = [[{"ranks": list(g.ranks), "lengths": [lengths[i] for i in g.ids]} for g in row] for row in plan]
    payload = json.dumps(shape, sort_keys=True, separators=(",", ":")).encode()
    enc = zlib.compressobj(level=6, wbits=-15)
    return "structure_v1:" + base64.b64encode(enc.compress(payload) + enc.flush()).decode()


def decode_identity(identity: str):
    if not identity.startswith("structure_v1:"):
        raise ValueError("unknown identity encoding")
    raw = zlib.decompress(base64.b64decode(identity.split(":", 1)[1]), wbits=-15)
    return json.loads(raw)


def fingerprint(plan, lengths) -> str:
    """sha256 of exact packed shapes, sample order, placement and microbatch order."""
    shape = [[{"ranks": list(g.ranks), "lengths": [lengths[i] for i in g.ids]} for g in row] for row in plan]
    return hashlib.sha256(json.dumps(shape, sort_keys=True, separators=(",", ":")).encode()).hexdigest()


def packet_collate(items):
    if len(items) != 1 or not isinstance(items[0], list):
        raise ValueError("Packet loader requires exactly one packet per batch")
    return items[0]
