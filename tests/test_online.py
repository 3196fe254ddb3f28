"""Online per-batch CP selection."""

import pytest

from prism_cp_b200.planner.joint import Model
from prism_cp_b200.planner.joint.cost import model_from_config
from prism_cp_b200.planner.joint.ir import validate_plan
from prism_cp_b200.planner.online import candidate_plan, select
from prism_cp_b200.runtime.batch import lognormal_lengths
from prism_cp_b200.models.config import hybrid_1p3b


def test_every_candidate_is_a_valid_plan():
    lengths = dict(enumerate([4096, 2048, 1024, 1024, 512, 512, 8192, 256]))
    for cg in (1, 2, 4, 8):
        for ca in (1, 2, 4, 8):
            plan = candidate_plan(lengths, 8, "GGG*GGG*", cg, ca, 8192)
            if plan is not None:
                validate_plan(plan, lengths)


def test_selection_is_deterministic_and_prefers_cp1_for_short_documents():
    model = Model()
    short = dict(enumerate([2048] * 64))
    sel = select(short, 8, "GGG*GGG*", model)
    assert (sel.cp_gdn, sel.cp_gqa) == (1, 1)
    assert select(short, 8, "GGG*GGG*", model).plan == sel.plan


def test_long_documents_force_context_parallelism():
    model = model_from_config(hybrid_1p3b(), device_bytes=180 * 1024 ** 3)
    lengths = dict(enumerate(lognormal_lengths(1 << 20, 4096, 1.0, 512, 131072, 16, 3) + [131072]))
    sel = select(lengths, 8, hybrid_1p3b().pattern, model, capacity=32768, dynamic=False)
    assert max(sel.cp_gdn, sel.cp_gqa) >= 4
    assert any(r["fits"] for r in sel.candidates)


def test_selection_shrinks_capacity_until_a_plan_fits_the_calibrated_memory():
    """On the calibrated B200 model the token ceiling alone packs microbatches that do not fit;
    the selector backs off to a smaller per-rank capacity and returns a plan that fits."""
    from prism_cp_b200.models.config import PRESETS
    from prism_cp_b200.planner.calibrate import calibrated
    from prism_cp_b200.planner.cli import B200_ENVELOPE
    from prism_cp_b200.planner.joint.cost import Evaluator, model_from_config
    from prism_cp_b200.planner.online import select
    from prism_cp_b200.runtime.batch import lognormal_lengths
    cfg = PRESETS["hybrid-1.3b"]()
    model = calibrated(model_from_config(cfg, B200_ENVELOPE["device_bytes"],
                                         **{k: v for k, v in B200_ENVELOPE.items() if k != "device_bytes"}))
    lengths = dict(enumerate(lognormal_lengths(1 << 20, 4096, 1.0, 512, 131072, 8, 1234)))
    sel = select(lengths, 4, cfg.pattern, model)
    ev = Evaluator(model, lengths, 4, cfg.pattern)
    assert all(ev.evaluate(mb)["fits"] for mb in sel.plan.microbatches)
    placed = sorted(s for mb in sel.plan.microbatches for g in mb.ingress.groups for s in g.samples)
    assert placed == sorted(lengths)


def test_dynamic_plan_gives_long_documents_big_teams_and_short_ones_cp1():
    """One long document among short ones: the per-document plan runs the long one on a large team
    and the short ones on CP1 ranks in the same microbatches, and is chosen when predicted faster."""
    from prism_cp_b200.planner.online import dynamic_candidates
    model = model_from_config(hybrid_1p3b(), device_bytes=180 * 1024 ** 3)
    lengths = {0: 65536, **{i: 2048 for i in range(1, 97)}}
    cands = dynamic_candidates(lengths, 8, hybrid_1p3b().pattern, model)
    assert cands
    _, cap, plan, _ = min(cands, key=lambda c: c[0])
    validate_plan(plan, lengths)
    first = plan.microbatches[0]
    degree = {s: cp for s, cp in first.layers[3][0].sample_cp()}
    assert degree[0] >= 65536 // cap and min(degree.values()) == 1
    sel = select(lengths, 8, hybrid_1p3b().pattern, model)
    uniform = select(lengths, 8, hybrid_1p3b().pattern, model, dynamic=False)
    assert sel.predicted_update_ms <= uniform.predicted_update_ms
    assert (sel.dynamic_capacity is not None) == (sel.predicted_update_ms < uniform.predicted_update_ms)


def test_full_recompute_keeps_the_memory_bounded_capacity():
    """With every microbatch recomputing (recompute_tokens = 0, ``--recompute-granularity full``) the
    packing capacity comes from the memory model, not from the threshold: the batch is not split
    into one document per microbatch."""
    from dataclasses import replace
    from prism_cp_b200.planner.calibrate import calibrated
    from prism_cp_b200.planner.cli import B200_ENVELOPE
    cfg = hybrid_1p3b()
    m = calibrated(model_from_config(cfg, B200_ENVELOPE["device_bytes"],
                                     **{k: v for k, v in B200_ENVELOPE.items() if k != "device_bytes"}))
    lengths = dict(enumerate(lognormal_lengths(1 << 20, 8192, 1.0, 512, 131072, 8, 1237)))
    full = select(lengths, 4, cfg.pattern, replace(m, recompute_tokens=0))
    assert len(full.plan.microbatches) < len(lengths) // 2, len(full.plan.microbatches)
    threshold = select(lengths, 4, cfg.pattern, replace(m, recompute_tokens=32768))
    assert len(full.plan.microbatches) <= len(threshold.plan.microbatches) + 2


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_benchmark_workload_builds_the_planned_batch(world):
    """The benchmark's default workload: 1M tokens of log-normal documents (the same lengths at every
    N), an online plan that validates, covers every document once and fits the calibrated memory
    model, with its predicted step time."""
    from prism_cp_b200.runtime.workload import build
    cfg = hybrid_1p3b()
    wl = build(cfg, world, "lognormal", "online", pin=False)
    assert sum(wl.batch.lengths.values()) == wl.description["global_batch_tokens"] <= 1 << 20
    assert wl.description["seq_len"] == max(wl.batch.lengths.values())
    validate_plan(wl.plan, wl.batch.lengths)
    seen = sorted(s for mb in wl.plan.microbatches for g in mb.ingress.groups for s in g.samples)
    assert seen == sorted(wl.batch.lengths)
    assert wl.predicted_ms and wl.predicted_ms > 0 and wl.parallelism.startswith("online")
    fixed = build(cfg, world, "fixed", "uniform", seqs=8, seq_len=32768, pin=False)
    assert fixed.parallelism == f"cp{world}" and fixed.predicted_ms is None
    validate_plan(fixed.plan, fixed.batch.lengths)
