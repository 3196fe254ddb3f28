"""Joint 2-D planner: IR, cost model, exact/bounded solver, replay (CPU only)."""

import json
from dataclasses import replace
from itertools import product

import pytest

from prism_cp_b200.planner.joint import (Evaluator, Group, Layout, Microbatch, Model, Plan, SearchLimit,
                                         SearchOptions, layout_candidates, route, solve, spans, validate_layout,
                                         validate_plan)
from prism_cp_b200.planner.joint.analysis import describe, measure
from prism_cp_b200.planner.joint.replay import compile_replay, validate_replay


def small_model(**kw):
    return Model(hidden=4, ffn=8, vocab=16, q_heads=2, kv_heads=1, head_dim=2, gdn_heads=1, gdn_dim=2,
                 static_bytes=0, external_bytes=0, margin_bytes=0, **kw)


def token_labels(layout, lengths, world):
    return [[(s, b + k) for s, b, _, c in row for k in range(c)] for row in spans(layout, lengths, world)]


def test_every_route_is_an_exact_permutation():
    lengths = {0: 16, 1: 8, 2: 8}
    cands = layout_candidates(lengths, lengths, 4, True, 100)
    assert len(cands) > 10
    for src in cands:
        for dst in cands:
            dst = dst.with_mode("contiguous")
            have, want = token_labels(src, lengths, 4), token_labels(dst, lengths, 4)
            got = [[None] * len(r) for r in want]
            for s, d, a, b, n in route(src, dst, lengths, 4):
                assert all(x is None for x in got[d][b:b + n])
                got[d][b:b + n] = have[s][a:a + n]
            assert got == want


def test_zigzag_spans_balance_causal_work():
    lengths = {0: 32}
    lay = Layout((Group((0, 1, 2, 3), (0,)),), "zigzag")
    rows = spans(lay, lengths, 4)
    assert rows[0] == ((0, 0, 0, 4), (0, 28, 4, 4))
    assert rows[3] == ((0, 12, 0, 4), (0, 16, 4, 4))


def test_exact_solver_equals_brute_force():
    lengths, world, pattern, model = {0: 8, 1: 4}, 2, "G*", small_model()
    best_total = float("inf")
    for packing in (((0, 1),), ((0,), (1,))):
        total = model.update_ms
        for ids in packing:
            lays = layout_candidates(ids, lengths, world, True, 100)
            mlps = tuple(dict.fromkeys(x.with_mode(m) for x in lays for m in ("zigzag", "contiguous")))
            best = float("inf")
            for ing, a1, a2, m1, m2 in product(lays, lays, lays, mlps, mlps):
                mb = Microbatch(ing, ((a1.with_mode("contiguous"), m1), (a2, m2)))
                row = Evaluator(model, lengths, world, pattern).evaluate(mb)
                if row["fits"]:
                    best = min(best, row["predicted_ms"])
            total += best
        best_total = min(best_total, total)
    res = solve(lengths, world, pattern, model, SearchOptions(mode="exact"))
    assert res["status"] == "optimal_in_declared_domain"
    assert res["predicted_update_ms"] == pytest.approx(best_total)
    validate_plan(Plan.from_dict(json.loads(json.dumps(res["plan"]))), lengths)


def test_capacity_comes_from_memory_model_and_peak_accumulates():
    lengths = {0: 65536}
    grp = (Group((0, 1), (0,)),)
    mb = Microbatch(Layout(grp, "zigzag"), ((Layout(grp, "contiguous"),) * 2,) * 8)
    model = small_model()
    res = solve(lengths, 2, "G*", model, SearchOptions(mode="exact"))
    assert max(Plan.from_dict(res["plan"]).microbatches[0].ingress.tokens(lengths, 2)) > 24576
    row = Evaluator(model, lengths, 2, "G" * 8).evaluate(mb)
    assert row["points"][7]["saved_live_bytes"][0] > 7 * row["points"][0]["saved_live_bytes"][0]
    peak = max(row["peak_bytes"])
    tight = replace(model, device_bytes=8 * 1024 ** 3 + peak - 1)
    assert not Evaluator(tight, lengths, 2, "G" * 8).evaluate(mb)["fits"]


def test_solver_picks_different_cp_per_layer(monkeypatch):
    import prism_cp_b200.planner.joint.solver as solver_mod

    class Forced(Evaluator):
        def operator(self, symbol, layout):
            cp = len(layout.groups[0].ranks)
            table = {"G": {1: 1.0, 2: 9.0}, "*": {1: 9.0, 2: 1.0}, "M": {1: 1.0, 2: 1.0}}
            return table[symbol][cp], (1, 1), (0, 0)

        def transfer(self, source, target):
            return (0.0 if source == target else 0.01), (0, 0)

    monkeypatch.setattr(solver_mod, "Evaluator", Forced)
    res = solve({0: 8, 1: 8}, 2, "G*", small_model(), SearchOptions(mode="exact"))
    assert res["predicted_update_ms"] < 6.0
    mb = Plan.from_dict(res["plan"]).microbatches[0]
    assert len(mb.layers[0][0].groups[0].ranks) == 1 and len(mb.layers[1][0].groups[0].ranks) == 2


def test_replay_round_trip_and_tamper_rejection():
    lengths = {0: 8, 1: 4}
    res = solve(lengths, 2, "G*", small_model(), SearchOptions(mode="exact"))
    manifest = {"samples": [{"sample_id": 17, "length": 8}, {"sample_id": 23, "length": 4}], "input_tokens": 12,
                "loss_tokens": 6, "case_id": "t", "seed": 3}
    rows = compile_replay(res, manifest)
    for row in rows:
        validate_replay(row, 2, "G*")
        assert row["logical_sample_ids"] == [17, 23]
    rows[0]["capacity_tokens"] += 1
    with pytest.raises(ValueError, match="changed"):
        validate_replay(rows[0], 2)


def test_bounded_search_status_and_budget():
    lengths, model = {i: 32 for i in range(8)}, small_model()
    res = solve(lengths, 2, "G*", model)
    validate_plan(Plan.from_dict(res["plan"]), lengths)
    assert res["status"] == "best_found_no_optimality_certificate"
    out = solve(lengths, 2, "G*", model, SearchOptions(max_states=1))
    assert out["status"] == "search_budget_exhausted" and out["plan"] is None
    with pytest.raises(SearchLimit):
        solve({0: 8, 1: 8}, 2, "G*", model, SearchOptions(mode="exact", max_states=1))


def test_ownership_validation():
    with pytest.raises(ValueError, match="alignment"):
        validate_layout(Layout((Group((0, 1), (0,)),), "zigzag"), {0: 7}, 2)
    with pytest.raises(ValueError, match="exactly once"):
        validate_plan(Plan(2, "G", ()), {0: 8})
    with pytest.raises(ValueError, match="dyadic"):
        validate_layout(Layout((Group((1, 2), (0,)), Group((0, 3), (1,))), "zigzag"), {0: 8, 1: 8}, 4)


def test_incumbent_survives_budget_interruption(monkeypatch):
    from prism_cp_b200.planner.joint.solver import _Search
    lengths, model = {0: 8, 1: 4}, small_model()
    original = _Search.batch
    seen = {}

    def interrupt(search, ids):
        if search.incumbent is not None:
            seen["score"] = search.incumbent[0] + model.update_ms
            raise SearchLimit("stop after the first complete packing")
        return original(search, ids)

    monkeypatch.setattr(_Search, "batch", interrupt)
    res = solve(lengths, 2, "G*", model, SearchOptions(homogeneous_packing=True))
    assert res["state_budget_exhausted"] and res["predicted_update_ms"] == seen["score"]
    validate_plan(Plan.from_dict(res["plan"]), lengths)


def test_node_affine_candidates_avoid_cross_node_routes():
    lengths = dict(enumerate([32768] + [512] * 448))

    def uniform(affine):
        lays = layout_candidates(lengths, lengths, 16, False, 6, 8 if affine else None)
        return {len(x.groups[0].ranks): x for x in lays if len({len(g.ranks) for g in x.groups}) == 1}

    plain, local = uniform(False), uniform(True)

    def remote(lays):
        return sum(n for s, d, _, _, n in route(lays[2].with_mode("contiguous"), lays[8], lengths, 16)
                   if s // 8 != d // 8)

    assert remote(plain) > 0 and remote(local) == 0


def test_stage_accounting_sums_to_score():
    lengths = {0: 64, 1: 32, 2: 32}
    model = small_model()
    res = solve(lengths, 2, "GG*", model)
    desc = describe(res, lengths, model)
    assert desc["predicted_update_ms"] == pytest.approx(sum(desc["stage_costs"].values()))
    total, _ = measure(Plan.from_dict(res["plan"]), lengths, model)
    assert total == pytest.approx(res["predicted_update_ms"])


def test_default_model_chooses_heterogeneous_cp():
    lengths = dict(enumerate([32768] + [512] * 448))
    res = solve(lengths, 16, "GGG*GGG*", Model(), SearchOptions(beam=16, layouts=6, node_affinity=True,
                                                                homogeneous_packing=True))
    assert not res["state_budget_exhausted"]
    plan = Plan.from_dict(res["plan"])
    validate_plan(plan, lengths)
    assert any(len({a.sample_cp() for a, _ in mb.layers}) > 1 for mb in plan.microbatches)
