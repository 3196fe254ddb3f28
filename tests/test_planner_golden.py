"""The planner reproduces the reference planner's outputs on a fixed corpus of inputs.

``tests/data/planner_golden.json`` holds what the reference's own planner code
returned for every case (generated once by ``tests/data/make_planner_golden.py``):
joint 2-D solves in exact and bounded mode over several models and hardware
profiles (their plans, predicted update times, search counters, memory
tie-break, stage accounting and CP-response evidence), the memory tie-break on
hand-made CP1 plans, 1-D searches (every candidate's fingerprint and proxy
cost, the selected plan, short-sequence refinement, export, selection rules and
round coalescing) and the memory/throughput policy rules. This package must
give the same answers: plans exactly, scores to 1e-9 relative. Free-text fields
(scope and provenance notes, anything containing a space) are descriptions, not
results, and are not compared.
"""

from __future__ import annotations

import json
import math
from pathlib import Path

import pytest

from prism_cp_b200.planner import mixed, onedim, policy
from prism_cp_b200.planner.joint.analysis import describe
from prism_cp_b200.planner.joint.cost import Model
from prism_cp_b200.planner.joint.ir import Plan
from prism_cp_b200.planner.joint.memory_selection import prefer_lower_memory
from prism_cp_b200.planner.joint.solver import SearchLimit, SearchOptions, solve

GOLDEN = json.loads((Path(__file__).parent / "data" / "planner_golden.json").read_text())


def close(a, b, rel=1e-9):
    if isinstance(a, dict):
        assert isinstance(b, dict) and set(a) == set(b), (sorted(a), sorted(b))
        for k in a:
            close(a[k], b[k], rel)
        return
    if isinstance(a, (list, tuple)):
        assert isinstance(b, (list, tuple)) and len(a) == len(b), (a, b)
        for x, y in zip(a, b):
            close(x, y, rel)
        return
    if isinstance(a, float) or isinstance(b, float):
        if a is None or b is None:
            assert a is None and b is None, (a, b)
            return
        assert math.isclose(a, b, rel_tol=rel, abs_tol=1e-9), (a, b)
        return
    if isinstance(a, str) and isinstance(b, str) and (" " in a or " " in b):
        return
    assert a == b, (a, b)


def jsonable(x):
    return json.loads(json.dumps(x, default=list))


def _model(name):
    return Model(**GOLDEN["models"][name])


def _lengths(case):
    return {int(k): v for k, v in case["lengths"].items()}


@pytest.mark.parametrize("case", GOLDEN["joint"], ids=[c["name"] for c in GOLDEN["joint"]])
def test_joint_solve_matches_reference(case):
    lengths, model = _lengths(case), _model(case["model"])
    options = SearchOptions(**case["options"])
    if "error" in case:
        with pytest.raises(SearchLimit if case["error"] == "SearchLimit" else Exception):
            solve(lengths, case["world"], case["pattern"], model, options)
        return
    result = solve(lengths, case["world"], case["pattern"], model, options)
    assert result["status"] == case["status"]
    assert jsonable(result["plan"]) == case["plan"]
    for key in ("states_examined", "pool_packings_examined", "microbatch_shapes_solved", "beam_pruned"):
        assert result[key] == case[key], key
    if case["plan"] is None:
        return
    close(result["predicted_update_ms"], case["predicted_update_ms"])
    close(jsonable(result.get("memory_selection")), case["memory_selection"])
    close(jsonable(result["resource_metrics"]), case["resource_metrics"])
    close(jsonable(result["cp_response_evidence"]), case["cp_response_evidence"])
    assert [list(e["peak_bytes"]) for e in result["microbatch_evidence"]] == case["peaks"]
    close(jsonable(describe(result, lengths, model)), case["describe"])


@pytest.mark.parametrize("case", GOLDEN["memory"])
def test_memory_tie_break_matches_reference(case):
    lengths = _lengths(case)
    plan = Plan.from_dict(case["plan"])
    chosen, meta = prefer_lower_memory(plan, lengths, Model(), case["tolerance"])
    assert jsonable(chosen.to_dict()) == case["selected"]
    close(jsonable(meta), case["meta"])


def _proxy(name):
    c = GOLDEN["proxy_costs"][name]
    return onedim.ProxyCost(name, c["a"], c["b"], c["provenance"])


@pytest.mark.parametrize("case", GOLDEN["onedim"], ids=[c["name"] for c in GOLDEN["onedim"]])
def test_onedim_search_matches_reference(case):
    lengths = _lengths(case)
    limits = onedim.Constraints(case["world"], case["token_cap"], case["min_cp"], case["max_sequences"],
                                case["alignment"])
    cost = _proxy(case["cost"])
    if "error" in case:
        with pytest.raises(ValueError):
            onedim.search(lengths, limits, cost, case["local_evaluations"], case["rounds"])
        return
    result = onedim.search(lengths, limits, cost, case["local_evaluations"], case["rounds"])
    got = [(c["name"], c["fingerprint"]) for c in result["candidates"]]
    assert got == [(c["name"], c["fingerprint"]) for c in case["candidates"]]
    close([c["proxy_cost"] for c in result["candidates"]], [c["proxy_cost"] for c in case["candidates"]])
    sel = result["selected"]
    assert (sel["name"], sel["fingerprint"]) == (case["selected"]["name"], case["selected"]["fingerprint"])
    assert onedim.to_rank_ids(sel["plan"], case["world"]) == case["selected"]["rank_ids"]
    assert jsonable(result["failures"]) == case["failures"]
    assert result["local_evaluations"] == case["local_evaluations"]
    refinement = {k: v for k, v in result["short_sequence_refinement"].items() if k != "planning_ms"}
    close(jsonable(refinement), case["refinement"])
    close(jsonable(onedim.export_plan(sel["plan"], lengths, cost, 8)), case["export"])
    assert onedim.select(result, lengths, None, True)[1] == case["proxy_select"]
    if case["native_select"] is not None:
        assert onedim.select(result, lengths, None, False)[1] == case["native_select"]
    rounds = mixed.coalesce_rounds(sel["plan"], lengths, case["world"], case["token_cap"], case["max_sequences"])
    assert jsonable(rounds) == case["coalesced"]


def test_policy_rules_match_reference():
    g = GOLDEN["policy"]
    for c in g["tradeoff"]:
        got = policy.tradeoff(*c["args"], min_gain_per_memory_growth=c["multiplier"], fits=c["fits"])
        close(jsonable(got), c["result"])
    for s in g["select"]:
        if "error" in s["result"]:
            with pytest.raises(ValueError):
                policy.select(s["candidates"], s["reference"], s["multiplier"])
            continue
        close(jsonable(policy.select(s["candidates"], s["reference"], s["multiplier"])), s["result"])
    for s in g["shortlists"]:
        assert policy.capacity_shortlist(s["lengths"]) == s["result"]
    cases = {c["case"]: c for c in g["cases"]}
    for row in g["choose"]:
        close(jsonable(policy.choose(cases[row["case"]], row["policy"], row["preference"])), row["result"])
    for key, want in g["integrate"].items():
        p, m = key.split("/")
        close(jsonable(policy.integrate(g["cases"], g["weights"], p, m)), want)
