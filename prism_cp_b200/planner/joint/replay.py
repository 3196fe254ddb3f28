"""Compile a solved joint plan into per-update replay rows, and validate them.

A replay row is what the executor consumes: stream ``TWO_DIMENSIONAL``, role
``S``, one ``rank_ids`` list per microbatch (ingress ownership), the derived
ingress allocation bound ``capacity_tokens``, one execution round per
microbatch and the embedded ``joint_cp_v1`` plan. ``validate_replay`` rejects
any tampering with world, pattern, ownership, rounds or capacity (field names
and rules as the reference: joint_cp/replay.py:6-46).
"""

from __future__ import annotations

from .ir import Plan, validate_plan


def compile_replay(result: dict, manifest: dict, updates: int = 3, candidate_id: str = "joint_cp") -> list[dict]:
    if updates < 1 or result.get("plan") is None:
        raise ValueError("Replay requires a feasible plan and positive update count")
    plan = Plan.from_dict(result["plan"])
    lengths = dict(enumerate(s["length"] for s in manifest["samples"]))
    stable = [s["sample_id"] for s in manifest["samples"]]
    if len(set(stable)) != len(stable):
        raise ValueError("Duplicate stable sample IDs")
    validate_plan(plan, lengths)
    rank_ids = [mb.ingress.rank_ids(plan.world) for mb in plan.microbatches]
    # an allocation bound for ingress tensors derived after the search, not a search constraint
    capacity = max(max(mb.ingress.tokens(lengths, plan.world)) for mb in plan.microbatches)
    if manifest["input_tokens"] != sum(lengths.values()):
        raise ValueError("Manifest input total differs from sample lengths")
    rows = []
    for step in range(1, updates + 1):
        rows.append({
            "step": step, "stream_id": "TWO_DIMENSIONAL", "architecture": "gdngqa_gpt", "role": "S",
            "candidate_id": candidate_id, "case_id": manifest["case_id"], "seed": manifest["seed"],
            "capacity_tokens": capacity, "capacity_semantics": "derived_ingress_allocation_bound",
            "rank_ids": rank_ids, "expected_lengths": list(lengths.values()), "logical_sample_ids": stable,
            "stable_to_scheduler_ordinal": [{"stable_sample_id": s, "scheduler_ordinal": i}
                                            for i, s in enumerate(stable)],
            "native_verified_cpu": False, "execution_rounds": [[i] for i in range(len(rank_ids))],
            "source_microbatches": len(rank_ids), "merged_microbatches": len(rank_ids),
            "input_tokens": manifest["input_tokens"], "loss_tokens": manifest["loss_tokens"],
            "repeat_same_frozen_content": True, "joint_plan": plan.to_dict(),
            "status": "CPU_ONLY_NOT_GPU_ADMITTED"})
    return rows


def validate_replay(row: dict, world: int, pattern: str | None = None) -> Plan:
    plan = Plan.from_dict(row["joint_plan"])
    if plan.world != world:
        raise ValueError("Joint replay world was changed")
    lengths = dict(enumerate(row["expected_lengths"]))
    validate_plan(plan, lengths)
    expected = [mb.ingress.rank_ids(world) for mb in plan.microbatches]
    capacity = max(max(mb.ingress.tokens(lengths, world)) for mb in plan.microbatches)
    if ((pattern is not None and plan.pattern != pattern) or row["rank_ids"] != expected
            or row["capacity_tokens"] != capacity or row["execution_rounds"] != [[i] for i in range(len(expected))]
            or row["role"] != "S" or row.get("capacity_semantics") != "derived_ingress_allocation_bound"):
        raise ValueError("Joint replay ingress, world, pattern, rounds or capacity was changed")
    return plan
