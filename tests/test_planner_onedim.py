"""1-D planner, native N re-derivation, policies, content rule and manifests (CPU)."""

import json
import random
from pathlib import Path

import pytest

from prism_cp_b200.planner import content, inputs
from prism_cp_b200.planner.mixed import coalesce_rounds, to_joint
from prism_cp_b200.planner.native import replay
from prism_cp_b200.planner.onedim import (Constraints, ExactCosts, Group, ProxyCost, export_plan, fingerprint,
                                          from_rank_ids, native_plan, pack_layout, search, select, to_rank_ids,
                                          validate)
from prism_cp_b200.planner.policy import capacity_shortlist, integrate, select as policy_select, tradeoff

GOLDEN = json.loads((Path(__file__).parent / "data" / "native_golden_plans.json").read_text())
HYBRID = ProxyCost("hybrid", 0.05, 4.0)


@pytest.mark.parametrize("case", GOLDEN, ids=[c["source"].split("/")[-1] for c in GOLDEN])
def test_native_matches_frozen_reference_plans(case):
    got = replay(list(enumerate(case["lengths"])), case["world"], case["capacity_tokens"])
    assert got == case["rank_ids"]


def test_native_unit_regressions():
    assert replay([(0, 6144), (1, 2048)], 2, 4096) == [[[0, 1], [0, 1]]]
    assert replay([(0, 50), (1, 50)], 14, 100) == [[[0, 1]] * 14]


def test_square_and_token_weighted_native_plans_differ_on_the_counterexample():
    """One 16K sample among 128 2K samples, 16 ranks, K = 32K: the square workload packs the short
    samples to the token capacity and the idle ranks then double the long sample's group (CP2, a
    32K-token rank); weighting tokens (the 1-GQA + 3-GDN stack coefficients, beta = 10.107 / 0.05545
    * 1024 tokens) spreads them, so the long sample keeps one rank and no rank holds more than 18K."""
    lengths = {0: 16384, **{i: 2048 for i in range(1, 129)}}
    limits = Constraints(16, 32768, alignment=32)
    square = native_plan(lengths, limits, ProxyCost("square", 1.0, 0.0))
    weighted = native_plan(lengths, limits, ProxyCost("hybrid", 0.05545098956660255, 10.106780354385673))
    assert len(square) == len(weighted) == 1
    assert len(next(g for g in square[0] if 0 in g.ids).ranks) == 2
    assert len(next(g for g in weighted[0] if 0 in g.ids).ranks) == 1
    assert max(sum(lengths[i] for i in g.ids) / len(g.ranks) for g in square[0]) == 32768
    assert max(sum(lengths[i] for i in g.ids) / len(g.ranks) for g in weighted[0]) == 18432


@pytest.mark.parametrize("plan,reason", [
    (((Group((0,), (0,)), Group((1,), (0,))),), "exactly once"),
    (((Group((0,), (0,)),),), "All ranks"),
    (((Group((1, 2), (0, 1)), Group((0, 3), (2,))),), "aligned"),
    (((Group((0, 1), (0, 1, 2)),),), "capacity"),
])
def test_illegal_plans(plan, reason):
    lengths = {0: 4096, 1: 4096, 2: 4096}
    limits = Constraints(4 if reason == "aligned" else 2, 4096)
    with pytest.raises(ValueError, match=reason):
        validate(plan, lengths, limits)


@pytest.mark.parametrize("world,min_cp", [(2, 1), (4, 1), (8, 2), (16, 4)])
def test_search_candidates_are_legal_and_never_worse_than_native(world, min_cp):
    rng = random.Random(4242 + world)
    for _ in range(6):
        lengths = {i: rng.choice([2048, 4096, 8192, 16384, 32768]) for i in range(rng.randint(1, 30))}
        limits = Constraints(world, 16384, min_cp, alignment=2 * world)
        res = search(lengths, limits, HYBRID, local_evaluations=16)
        for c in res["candidates"]:
            validate(c["plan"], lengths, limits)
            assert from_rank_ids(to_rank_ids(c["plan"], world)) == c["plan"]
        native = [c for c in res["candidates"] if c["name"] == "native_square"]
        if native:
            assert res["selected"]["proxy_cost"] <= HYBRID.evaluate(native[0]["plan"], lengths) + 1e-8


def test_selection_prefers_measured_then_proxy_then_native():
    lengths = {0: 8192, 1: 8192, 2: 4096, 3: 4096}
    limits = Constraints(2, 8192, alignment=4)
    res = search(lengths, limits, HYBRID, local_evaluations=8)
    plan, why = select(res, lengths)
    assert why == "native_fallback_unknown_distributed_cost" and plan["name"] == "native_square"
    assert select(res, lengths, allow_proxy=True)[1] == "experimental_compute_proxy"
    contract = {"model": "x"}
    records = [{"fingerprint": c["fingerprint"], "status": "ok", "numerical_pass": True,
                "milliseconds": 10.0 + i} for i, c in enumerate(res["candidates"])]
    records[-1]["milliseconds"] = 1.0
    table = ExactCosts({"contract": contract, "scope": "complete step", "records": records}, contract)
    chosen, why = select(res, lengths, table)
    assert why == "measured_complete_plan" and chosen is res["candidates"][-1]
    with pytest.raises(ValueError):
        ExactCosts({"contract": {"model": "y"}, "scope": "", "records": []}, contract)


def test_pack_layout_and_export():
    lengths = {i: 4096 for i in range(6)}
    limits = Constraints(4, 8192, alignment=8)
    plan = pack_layout(lengths, limits, (2, 1, 1), HYBRID)
    validate(plan, lengths, limits)
    out = export_plan(plan, lengths, HYBRID, 8)
    assert out["fingerprint"] == fingerprint(plan, lengths)
    assert all(g["placement"] == "intra_node" for b in out["microbatches"] for g in b["groups"])


def test_coalesce_rounds_respects_capacity():
    lengths = {0: 4096, 1: 4096, 2: 2048, 3: 2048}
    plan = ((Group((0, 1), (0,)),), (Group((0,), (2,)), Group((1,), (3,))), (Group((0, 1), (1,)),))
    windows = coalesce_rounds(plan, lengths, 2, 4096)
    assert windows == ((0, 1), (2,))
    joint = to_joint(plan, lengths, 2, "G*")
    assert len(joint.microbatches) == 3


def test_tradeoff_rule():
    assert tradeoff(100, 10, 80, 11, min_gain_per_memory_growth=2.0)["accepted"]      # +25% for +10%
    assert not tradeoff(100, 10, 95, 11, min_gain_per_memory_growth=2.0)["accepted"]  # +5% for +10%
    assert tradeoff(100, 10, 100, 9)["reason"] == "no_memory_increase"
    assert tradeoff(100, 10, 90, 20, fits=False)["reason"] == "physical_memory_rejected"
    sel = policy_select([{"id": "N", "kind": "native", "time": 100, "peak": 10, "fits": True},
                         {"id": "J", "kind": "joint", "time": 80, "peak": 10.5, "fits": True}], "N")
    assert sel["selected"] == "J" and sel["best_native"] == "N"


def test_capacity_shortlist_keeps_fractional_thresholds():
    values = capacity_shortlist([248 * 1024] * 8 + [4096] * 64)
    assert 15872 in values and 31 * 1024 in values
    assert all(v % 32 == 0 and v * 16 >= 248 * 1024 for v in values)


def test_integrate_is_ratio_of_expectations():
    def row(name, t, peak, cap=None):
        return {"id": name, "capacity_tokens": cap,
                "scores": {"p": {"predicted_update_ms": t, "peak_gib": peak, "model_fits": True}}}
    cases = [{"case": "a", "input_tokens": 100, "simple_capacity_tokens": [16384, 24576],
              "native": [row("N_K16", 100, 10, 16384), row("N_K24", 80, 20, 24576)], "joint": [row("J_a", 40, 15)]},
             {"case": "b", "input_tokens": 900, "simple_capacity_tokens": [16384, 24576],
              "native": [row("N_K16", 200, 30, 16384), row("N_K24", 240, 40, 24576)], "joint": [row("J_b", 220, 25)]}]
    res = integrate(cases, {"a": 0.5, "b": 0.5}, "p", "physical")
    assert res["fixed_capacity_tokens"] == 16384
    assert res["fixed"]["expected_update_ms"] == 150
    assert res["simple"]["expected_update_ms"] == 140
    assert res["selected"]["expected_update_ms"] == 120
    assert res["selection_gain_vs_simple_pct"] == pytest.approx(100 / 6)
    assert res["joint_selected_probability"] == 0.5


def test_lcg_jump_and_vector_fields_agree():
    m = inputs.build_manifest([64, 32], "case", 2, seed=99, vocab=4096)
    span = content.materialize_span(m, 1, 5, 20)
    state = content.advance(99, 1 * content.SAMPLE_STRIDE + 6)
    assert span["tokens"][0] == (state >> 32) % 4096
    vec = content.vector_fields(m, 1, list(range(5, 20)))
    assert vec["tokens"].tolist() == span["tokens"] and vec["labels"].tolist() == span["labels"]
    assert span["loss_mask"] == [int(p < 16) for p in range(5, 20)]
    # stepping once equals a one-step jump
    assert content.advance(7, 1) == (7 * content.MULTIPLIER + content.INCREMENT) % content.MODULUS


def test_manifest_validation_and_identity():
    m = inputs.build_manifest([64, 128], "id", 2)
    bad = json.loads(json.dumps(m))
    bad["samples"][0]["length"] = 63
    with pytest.raises(ValueError):
        inputs.validate_manifest(bad)
    plan = ((Group((0, 1), (0, 1)),),)
    ident = inputs.structural_identity(plan, {0: 64, 1: 128})
    assert inputs.decode_identity(ident) == [[{"ranks": [0, 1], "lengths": [64, 128]}]]
    src = inputs.PacketSource(m, 2)
    from prism_cp_b200.planner.joint.ir import Group as JG, Layout
    t, l, p, w = src.rank_inputs(1, Layout((JG((0, 1), (0, 1)),), "zigzag"), 2, 1)
    # rank 1 holds sample 0 positions 16..47 (mask: < 32) and sample 1 positions 32..95 (mask: < 64)
    assert t.numel() == 96 and float(w.sum()) * m["loss_tokens"] == pytest.approx(16 + 32)
