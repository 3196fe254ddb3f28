"""Joint 2-D planner properties on CPU: ownership IR, memory model, solver optimality and limits.

Equality with the reference planner's outputs is pinned separately by the golden corpus
(``test_planner_golden.py``); these tests check the invariants any correct planner must keep,
over generated inputs (hypothesis) where the domain is small enough to enumerate.
"""

import itertools
import json
from dataclasses import replace

import pytest
from hypothesis import given, settings
from hypothesis import strategies as st

from prism_cp_b200.planner.joint import (Evaluator, Group, Layout, Microbatch, Model, Plan, SearchLimit,
                                         SearchOptions, layout_candidates, route, solve, spans, validate_layout,
                                         validate_plan)
from prism_cp_b200.planner.joint.analysis import describe, measure
from prism_cp_b200.planner.joint.replay import compile_replay, validate_replay

TINY = dict(hidden=4, ffn=8, vocab=16, q_heads=2, kv_heads=1, head_dim=2, gdn_heads=1, gdn_dim=2, static_bytes=0,
            external_bytes=0, margin_bytes=0)


def tiny(**overrides) -> Model:
    return Model(**{**TINY, **overrides})


def owned_tokens(layout, lengths, world):
    """Per rank, the (sample, position) of every local row in local order."""
    return [[(s, b + k) for s, b, _, c in row for k in range(c)] for row in spans(layout, lengths, world)]


lengths_st = st.lists(st.sampled_from((8, 16, 24, 32)), min_size=1, max_size=3).map(lambda xs: dict(enumerate(xs)))


# ------------------------------------------------------------------ ownership IR
class TestOwnership:
    @settings(max_examples=25, deadline=None)
    @given(lengths=lengths_st, world=st.sampled_from((2, 4)), data=st.data())
    def test_routes_move_every_token_exactly_once(self, lengths, world, data):
        layouts = layout_candidates(lengths, lengths, world, True, 1000)
        if not layouts:
            return
        src = data.draw(st.sampled_from(layouts))
        dst = data.draw(st.sampled_from(layouts)).with_mode(data.draw(st.sampled_from(("zigzag", "contiguous"))))
        have, want = owned_tokens(src, lengths, world), owned_tokens(dst, lengths, world)
        filled = [[None] * len(row) for row in want]
        for s, d, a, b, n in route(src, dst, lengths, world):
            assert all(x is None for x in filled[d][b:b + n]), "a destination row was written twice"
            filled[d][b:b + n] = have[s][a:a + n]
        assert filled == want

    @settings(max_examples=30, deadline=None)
    @given(cp=st.sampled_from((1, 2, 4, 8)), chunk=st.integers(1, 16))
    def test_zigzag_gives_every_rank_the_same_causal_work(self, cp, chunk):
        n = 2 * cp * chunk
        layout = Layout((Group(tuple(range(cp)), (0,)),), "zigzag")
        rows = spans(layout, {0: n}, cp)
        work = [sum(b + k + 1 for _, b, _, c in row for k in range(c)) for row in rows]
        assert len(set(work)) == 1 and sum(c for row in rows for _, _, _, c in row) == n

    @pytest.mark.parametrize("layout,lengths,world,message", [
        (Layout((Group((0, 1), (0,)),), "zigzag"), {0: 7}, 2, "alignment"),
        (Layout((Group((1, 2), (0,)), Group((0, 3), (1,))), "zigzag"), {0: 8, 1: 8}, 4, "dyadic"),
    ])
    def test_illegal_layouts_are_named(self, layout, lengths, world, message):
        with pytest.raises(ValueError, match=message):
            validate_layout(layout, lengths, world)

    def test_a_plan_must_cover_every_sample(self):
        with pytest.raises(ValueError, match="exactly once"):
            validate_plan(Plan(2, "G", ()), {0: 8})


# ------------------------------------------------------------------ memory model
class TestMemory:
    def _one_group(self, layers):
        g = (Group((0, 1), (0,)),)
        return Microbatch(Layout(g, "zigzag"), ((Layout(g, "contiguous"),) * 2,) * layers)

    def test_saved_bytes_grow_with_depth_and_the_budget_decides_fit(self):
        lengths, model = {0: 65536}, tiny()
        mb = self._one_group(8)
        row = Evaluator(model, lengths, 2, "G" * 8).evaluate(mb)
        saved = [p["saved_live_bytes"][0] for p in row["points"]]
        assert saved == sorted(saved) and saved[-1] > 7 * saved[0]
        peak = max(row["peak_bytes"])
        exact_fit = replace(model, device_bytes=8 * 1024 ** 3 + peak)
        one_short = replace(model, device_bytes=8 * 1024 ** 3 + peak - 1)
        assert Evaluator(exact_fit, lengths, 2, "G" * 8).evaluate(mb)["fits"]
        assert not Evaluator(one_short, lengths, 2, "G" * 8).evaluate(mb)["fits"]

    def test_capacity_follows_the_memory_model_not_a_token_cap(self):
        res = solve({0: 65536}, 2, "G*", tiny(), SearchOptions(mode="exact"))
        ingress = Plan.from_dict(res["plan"]).microbatches[0].ingress
        assert max(ingress.tokens({0: 65536}, 2)) > 24576


# ------------------------------------------------------------------ solver
def brute_force(lengths, world, pattern, model) -> float:
    """Cheapest plan by enumerating every packing, layout and layer path."""
    ids = sorted(lengths)
    ev = Evaluator(model, lengths, world, pattern)

    def best_microbatch(pack):
        layouts = layout_candidates(pack, lengths, world, True, 10 ** 6)
        mlps = tuple({x.with_mode(m): None for x in layouts for m in ("zigzag", "contiguous")})
        best = float("inf")
        for ingress in layouts:
            for path in itertools.product(layouts, repeat=len(pattern)):
                for mlp_path in itertools.product(mlps, repeat=len(pattern)):
                    layers = tuple((a.with_mode("contiguous" if s == "G" else "zigzag"), m)
                                   for s, a, m in zip(pattern, path, mlp_path))
                    row = ev.evaluate(Microbatch(ingress, layers))
                    if row["fits"]:
                        best = min(best, row["predicted_ms"])
        return best

    def partitions(items):
        if not items:
            yield []
            return
        head, rest = items[0], items[1:]
        for k in range(len(rest) + 1):
            for others in itertools.combinations(rest, k):
                remaining = [x for x in rest if x not in others]
                for tail in partitions(remaining):
                    yield [(head, *others)] + tail

    return model.update_ms + min(sum(best_microbatch(p) for p in packing) for packing in partitions(ids))


class TestSolver:
    @settings(max_examples=6, deadline=None)
    @given(lengths=st.lists(st.sampled_from((4, 8, 12)), min_size=1, max_size=2).map(lambda x: dict(enumerate(x))),
           pattern=st.sampled_from(("G*", "*G")))
    def test_exact_mode_is_optimal(self, lengths, pattern):
        model = tiny()
        res = solve(lengths, 2, pattern, model, SearchOptions(mode="exact"))
        assert res["status"] == "optimal_in_declared_domain"
        assert res["predicted_update_ms"] == pytest.approx(brute_force(lengths, 2, pattern, model))
        validate_plan(Plan.from_dict(json.loads(json.dumps(res["plan"]))), lengths)

    @pytest.mark.parametrize("gdn_prefers,gqa_prefers", [(1, 2), (2, 1)])
    def test_each_layer_gets_its_own_cp_degree(self, monkeypatch, gdn_prefers, gqa_prefers):
        import prism_cp_b200.planner.joint.solver as solver_mod

        class Priced(Evaluator):
            def operator(self, symbol, layout):
                cp = len(layout.groups[0].ranks)
                favourite = {"G": gdn_prefers, "*": gqa_prefers, "M": cp}[symbol]
                return (1.0 if cp == favourite else 9.0), (1, 1), (0, 0)

            def transfer(self, source, target):
                return (0.0 if source == target else 0.01), (0, 0)

        monkeypatch.setattr(solver_mod, "Evaluator", Priced)
        res = solve({0: 8, 1: 8}, 2, "G*", tiny(), SearchOptions(mode="exact"))
        layers = Plan.from_dict(res["plan"]).microbatches[0].layers
        assert [len(a.groups[0].ranks) for a, _ in layers] == [gdn_prefers, gqa_prefers]

    def test_budget_exhaustion(self):
        lengths, model = {i: 32 for i in range(8)}, tiny()
        assert solve(lengths, 2, "G*", model)["status"] == "best_found_no_optimality_certificate"
        starved = solve(lengths, 2, "G*", model, SearchOptions(max_states=1))
        assert starved["status"] == "search_budget_exhausted" and starved["plan"] is None
        with pytest.raises(SearchLimit):
            solve({0: 8, 1: 8}, 2, "G*", model, SearchOptions(mode="exact", max_states=1))

    def test_an_interrupted_bounded_search_returns_its_incumbent(self, monkeypatch):
        from prism_cp_b200.planner.joint.solver import _Search
        model, calls = tiny(), {}
        solve_batch = _Search.batch

        def stop_after_first_packing(search, ids):
            if search.incumbent is not None:
                calls["incumbent_ms"] = search.incumbent[0] + model.update_ms
                raise SearchLimit("interrupted")
            return solve_batch(search, ids)

        monkeypatch.setattr(_Search, "batch", stop_after_first_packing)
        res = solve({0: 8, 1: 4}, 2, "G*", model, SearchOptions(homogeneous_packing=True))
        assert res["state_budget_exhausted"] and res["predicted_update_ms"] == calls["incumbent_ms"]

    def test_node_affinity_keeps_samples_on_their_node(self):
        lengths = dict(enumerate([32768] + [512] * 448))

        def cross_node_rows(affine):
            lays = layout_candidates(lengths, lengths, 16, False, 6, 8 if affine else None)
            by_width = {len(x.groups[0].ranks): x for x in lays if len({len(g.ranks) for g in x.groups}) == 1}
            edges = route(by_width[2].with_mode("contiguous"), by_width[8], lengths, 16)
            return sum(n for s, d, _, _, n in edges if s // 8 != d // 8)

        assert cross_node_rows(False) > 0 and cross_node_rows(True) == 0

    def test_a_long_document_among_short_ones_gets_mixed_cp(self):
        lengths = dict(enumerate([32768] + [512] * 448))
        options = SearchOptions(beam=16, layouts=6, node_affinity=True, homogeneous_packing=True)
        res = solve(lengths, 16, "GGG*GGG*", Model(), options)
        plan = Plan.from_dict(res["plan"])
        validate_plan(plan, lengths)
        assert not res["state_budget_exhausted"]
        assert any(len({a.sample_cp() for a, _ in mb.layers}) > 1 for mb in plan.microbatches)


# ------------------------------------------------------------------ accounting and replay
def test_stage_costs_add_up_and_rescoring_agrees():
    lengths, model = {0: 64, 1: 32, 2: 32}, tiny()
    res = solve(lengths, 2, "GG*", model)
    assert sum(describe(res, lengths, model)["stage_costs"].values()) == pytest.approx(res["predicted_update_ms"])
    assert measure(Plan.from_dict(res["plan"]), lengths, model)[0] == pytest.approx(res["predicted_update_ms"])


def test_replay_rows_keep_logical_ids_and_reject_edits():
    res = solve({0: 8, 1: 4}, 2, "G*", tiny(), SearchOptions(mode="exact"))
    manifest = {"samples": [{"sample_id": 17, "length": 8}, {"sample_id": 23, "length": 4}], "input_tokens": 12,
                "loss_tokens": 6, "case_id": "t", "seed": 3}
    rows = compile_replay(res, manifest)
    for row in rows:
        validate_replay(row, 2, "G*")
        assert row["logical_sample_ids"] == [17, 23]
    rows[-1]["capacity_tokens"] += 1
    with pytest.raises(ValueError, match="changed"):
        validate_replay(rows[-1], 2)


def test_solver_rejects_recompute_priced_models():
    """Recompute depends on every layout of a microbatch at once, which the solver's layer-by-layer
    objective cannot price: such a model is refused with a clear error instead of a wrong plan."""
    from dataclasses import replace
    import pytest as _pytest
    from prism_cp_b200.models.config import hybrid_tiny
    from prism_cp_b200.planner.joint.cost import model_from_config
    from prism_cp_b200.planner.joint.solver import solve
    cfg = hybrid_tiny()
    m = replace(model_from_config(cfg, 80 << 30), recompute_tokens=1024)
    with _pytest.raises(ValueError, match="recompute"):
        solve({0: 2048, 1: 1024}, 2, cfg.pattern, m)
