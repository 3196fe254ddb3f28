"""Planner CLI, catalogue cover, cost fit, profile builder and handoff self-check (CPU)."""

import itertools
import json
import math

import pytest

from prism_cp_b200.planner import cli, costfit, handoff, profile_builder, studies
from prism_cp_b200.planner.inputs import build_manifest
from prism_cp_b200.planner.joint.cost import Model
from prism_cp_b200.planner.joint.ir import Plan, validate_plan

SMALL = Model(hidden=1024, ffn=4096, vocab=32000, q_heads=8, kv_heads=2, head_dim=128, gdn_heads=8, gdn_dim=128,
              device_bytes=180 * 10 ** 9)


def test_count_cover_matches_brute_force():
    templates = [(1, 0, 5.0, "a"), (0, 2, 3.0, "b"), (1, 2, 7.5, "c"), (0, 1, 1.8, "d"), (2, 1, 9.0, "e")]
    for n_long, n_short in [(2, 3), (3, 4), (1, 5)]:
        best = math.inf
        for counts in itertools.product(range(6), repeat=len(templates)):
            h = sum(c * t[0] for c, t in zip(counts, templates))
            s = sum(c * t[1] for c, t in zip(counts, templates))
            if (h, s) == (n_long, n_short):
                best = min(best, sum(c * t[2] for c, t in zip(counts, templates)))
        score, chosen = studies.count_cover(templates, n_long, n_short)
        assert math.isclose(score, best)
        by_id = {t[3]: t for t in templates}
        assert sum(by_id[i][0] for i in chosen) == n_long and sum(by_id[i][1] for i in chosen) == n_short


def test_count_cover_rejects_uncoverable():
    with pytest.raises(ValueError):
        studies.count_cover([(2, 0, 1.0, 0)], 3, 0)


def test_costfit_recovers_and_refuses():
    s = [2048 * k for k in range(1, 11)]
    t = [3e-4 * x + 0.2 for x in s]
    f = costfit.fit("M", s, t, "linear", holdout_every=3)
    assert abs(f.coefficients["S"] - 3e-4) < 1e-10 and abs(f.coefficients["1"] - 0.2) < 1e-8
    assert math.isclose(f.query(8192), 3e-4 * 8192 + 0.2, rel_tol=1e-9)
    with pytest.raises(ValueError, match="CP"):
        f.query(8192, cp=4)
    with pytest.raises(ValueError, match="outside"):
        f.query(10 ** 7)


def test_nnls_keeps_coefficients_nonnegative():
    import numpy as np
    A = np.array([[1.0, 1.0], [2.0, 1.0], [3.0, 1.0]])
    b = np.array([3.0, 2.0, 1.0])  # decreasing: the unconstrained slope is negative
    x = costfit.nnls_exact(A, b)
    assert (x >= 0).all() and x[0] == 0.0 and math.isclose(x[1], 2.0)


def test_profile_builder_medians_and_validates():
    records = []
    for module in ("GQA", "GDN"):
        for cp, ms in ((1, 80.0), (2, 42.0), (4, 22.0), (8, 12.0)):
            for rep in range(3):
                records.append({"module": module, "cp": cp, "tokens": 65536, "fb_ms": ms + rep})
    shape = (1024, 8, 2, 128, 8, 128)
    prof = profile_builder.build(records, 65536, shape)
    assert prof["anchors"]["GQA"]["milliseconds"]["4"] == 23.0
    from dataclasses import replace
    m = replace(SMALL, cp_response=prof)  # validates in __post_init__
    assert m.cp_response["hardware"] == "B200"


def test_handoff_self_check_passes():
    report = handoff.run()
    assert report["ok"], report


def test_cli_search_writes_result_replay_executor(tmp_path):
    manifest = build_manifest([8192, 4096, 2048, 2048], "cli", 2)
    mpath = tmp_path / "m.json"
    mpath.write_text(json.dumps(manifest))
    prof = tmp_path / "model.json"
    from dataclasses import asdict
    prof.write_text(json.dumps(asdict(SMALL)))
    out = tmp_path / "run"
    rc = cli.main(["search", "--manifest", str(mpath), "--output", str(out), "--world", "2", "--pattern", "G*",
                   "--model-profile", str(prof), "--updates", "2"])
    assert rc == 0
    result = json.loads((out / "result.json").read_text())
    plan = Plan.from_dict(result["plan"])
    validate_plan(plan, dict(enumerate([8192, 4096, 2048, 2048])))
    assert len(json.loads((out / "replay.json").read_text())) == 2
    assert json.loads((out / "executor.json").read_text())["mode"] == "joint"


def test_cli_study_reports_alpha_selection(tmp_path):
    manifest = build_manifest([16384, 4096, 4096, 2048, 2048, 1024, 1024], "study", 4)
    mpath = tmp_path / "m.json"
    mpath.write_text(json.dumps(manifest))
    prof = tmp_path / "model.json"
    from dataclasses import asdict
    prof.write_text(json.dumps(asdict(SMALL)))
    out = tmp_path / "study"
    rc = cli.main(["study", "--manifest", str(mpath), "--output", str(out), "--world", "4", "--pattern", "GGG*",
                   "--model-profile", str(prof), "--capacities", "4096", "8192", "16384",
                   "--reference-capacity", "8192", "--beam", "4", "--layouts", "4"])
    assert rc == 0
    report = json.loads((out / "study.json").read_text())
    ids = {c["id"] for c in report["candidates"]}
    assert {"native_K4096", "native_K8192", "native_K16384", "joint"} <= ids
    assert report["decision"]["selected"] in ids
    assert (out / "REPORT.md").read_text().startswith("# Native N vs joint plan")


def test_b200_cp1_costfit_reproduces_measured_records():
    """The committed B200 CP1 fit (from measured module records) matches its own measurements."""
    import json
    from pathlib import Path
    import pytest
    from prism_cp_b200.planner.costfit import CostFit
    root = Path(__file__).resolve().parents[1] / "prism_cp_b200" / "planner" / "data"
    fits = {m: CostFit(**f) for m, f in json.loads((root / "b200_cp1_costfit.json").read_text())["fits"].items()}
    recs = json.loads((root / "b200_module_records.json").read_text())
    for key, module in (("gqa", "GQA"), ("gdn", "GDN")):
        for r in recs[key]["records"]:
            if r.get("sequences", 1) == 1:
                assert abs(fits[module].query(r["tokens"]) - r["fb_ms"]) <= 0.15 * r["fb_ms"] + 0.5
    with pytest.raises(ValueError):
        fits["GQA"].query(8192, cp=2)


def test_b200_operator_calibration_reproduces_module_times():
    """Evaluator costs with the committed calibration match the newest measured CP = 1 module times, and
    the older multi-length records up to the factor the calibration was moved by (faster kernels)."""
    import json
    from dataclasses import replace
    from pathlib import Path
    from prism_cp_b200.models.config import PRESETS
    from prism_cp_b200.planner.calibrate import load_default
    from prism_cp_b200.planner.cli import B200_ENVELOPE
    from prism_cp_b200.planner.joint.cost import Evaluator, model_from_config
    from prism_cp_b200.planner.joint.ir import Group, Layout
    model = model_from_config(PRESETS["hybrid-1.3b"](), B200_ENVELOPE["device_bytes"],
                              **{k: v for k, v in B200_ENVELOPE.items() if k != "device_bytes"})
    cal = {k: {x: v[x] for x in ("linear", "quadratic", "fixed_ms") if x in v} for k, v in load_default().items()}
    calibrated = replace(model, operator_calibration=cal)
    root = Path(__file__).resolve().parents[1] / "prism_cp_b200" / "planner" / "data"
    recs = json.loads((root / "b200_module_records.json").read_text())
    moved = {k: v.get("rescaled_by", 1.0) for k, v in load_default().items()}
    for key, sym in (("gqa", "*"), ("gdn", "G"), ("mlp", "M")):
        for r in recs[key]["records"]:
            if r.get("sequences", 1) != 1:
                continue
            ev = Evaluator(calibrated, {0: r["tokens"]}, 1, "G*")
            ms, _, _ = ev.operator(sym, Layout((Group((0,), (0,)),), "zigzag"))
            want = r["fb_ms"] * moved[sym]
            assert abs(ms - want) <= 0.2 * want + 0.5, (sym, r["tokens"], ms, want)
    newest = json.loads((root / "b200_anchor_records.json").read_text())["records"]
    for r in (r for r in newest if r["cp"] == 1):
        sym = {"GQA": "*", "GDN": "G"}[r["module"]]
        ms, _, _ = Evaluator(calibrated, {0: r["tokens"]}, 1, "G*").operator(sym, Layout((Group((0,), (0,)),), "zigzag"))
        assert abs(ms - r["fb_ms"]) <= 0.05 * r["fb_ms"], (sym, ms, r["fb_ms"])
    # the uncalibrated envelope is much more optimistic for the GDN recurrence
    ev0 = Evaluator(model, {0: 32768}, 1, "G*")
    ms0, _, _ = ev0.operator("G", Layout((Group((0,), (0,)),), "zigzag"))
    assert ms0 < 0.5 * [r for r in recs["gdn"]["records"] if r["tokens"] == 32768 and r["sequences"] == 1][0]["fb_ms"]


def test_b200_calibrated_memory_matches_the_measured_peak():
    """With the committed byte scale, one 32K-token CP = 1 microbatch of the 1.3B model is priced at the
    141.15 GiB peak the bench measured, inside the HBM budget; the uncalibrated model underestimates it."""
    from prism_cp_b200.models.config import PRESETS
    from prism_cp_b200.planner.calibrate import calibrated
    from prism_cp_b200.planner.cli import B200_ENVELOPE
    from prism_cp_b200.planner.joint.cost import Evaluator, model_from_config
    from prism_cp_b200.planner.joint.ir import Group, Layout, Microbatch
    cfg = PRESETS["hybrid-1.3b"]()
    raw = model_from_config(cfg, B200_ENVELOPE["device_bytes"],
                            **{k: v for k, v in B200_ENVELOPE.items() if k != "device_bytes"})
    one = Layout((Group((0,), (0,)),), "zigzag")
    mb = Microbatch(one, tuple((one, one) for _ in cfg.pattern))
    gib = 2 ** 30
    peak = max(Evaluator(calibrated(raw), {0: 32768}, 1, cfg.pattern).evaluate(mb)["peak_bytes"]) / gib
    assert abs(peak - 141.15) < 0.5 and peak * gib <= calibrated(raw).budget
    assert max(Evaluator(raw, {0: 32768}, 1, cfg.pattern).evaluate(mb)["peak_bytes"]) / gib < 100


def test_calibrated_planner_prices_the_measured_bench_steps():
    """The committed B200 calibration prices the bench's measured steps (1M tokens of log-normal
    documents, the online plan it chooses at 1, 2, 4 and 8 GPUs) within 10 %."""
    import json
    from dataclasses import replace
    from prism_cp_b200.models.config import PRESETS
    from prism_cp_b200.planner.calibrate import DEFAULT, calibrated
    from prism_cp_b200.planner.cli import B200_ENVELOPE
    from prism_cp_b200.planner.joint.cost import model_from_config
    from prism_cp_b200.planner.online import select
    from prism_cp_b200.runtime.batch import lognormal_lengths
    cfg = PRESETS["hybrid-1.3b"]()
    m = replace(calibrated(model_from_config(cfg, B200_ENVELOPE["device_bytes"],
                                             **{k: v for k, v in B200_ENVELOPE.items() if k != "device_bytes"})),
                recompute_tokens=32768)
    measured = json.loads(DEFAULT.read_text())["bench_steps_ms"]
    for world in (1, 2, 4, 8):
        lengths = dict(enumerate(lognormal_lengths(1 << 20, 4096, 1.0, 512, 131072, 2 * max(world, 8), 1234)))
        ms = select(lengths, world, cfg.pattern, m).predicted_update_ms
        assert abs(ms - measured[str(world)]) <= 0.10 * measured[str(world)], (world, ms, measured[str(world)])


def test_cp_overhead_factor_lookup_and_measured_ratio():
    """Flat and per-operator factor tables; the committed factors reproduce the measured module
    anchors at every measured CP degree."""
    import json
    from pathlib import Path
    from prism_cp_b200.models.config import PRESETS
    from prism_cp_b200.planner import calibrate
    from prism_cp_b200.planner.calibrate import calibrated
    from prism_cp_b200.planner.cli import B200_ENVELOPE
    from prism_cp_b200.planner.joint.cost import Evaluator, cp_overhead_factor, model_from_config
    from prism_cp_b200.planner.joint.ir import Group, Layout
    table = {"2": 1.1, "8": 1.3}
    assert cp_overhead_factor(table, 2) == 1.1 and cp_overhead_factor(table, 4) == 1.1 and cp_overhead_factor(table, 8) == 1.3
    assert cp_overhead_factor({"4": 1.2}, 2) == 1.2
    cfg = PRESETS["hybrid-1.3b"]()
    m = calibrated(model_from_config(cfg, B200_ENVELOPE["device_bytes"],
                                     **{k: v for k, v in B200_ENVELOPE.items() if k != "device_bytes"}))
    data = Path(calibrate.__file__).resolve().parent / "data" / "b200_anchor_records.json"
    for r in json.loads(data.read_text())["records"]:
        if r["cp"] == 1 or r["tokens"] != 65536:
            continue
        sym = "G" if r["module"] == "GDN" else "*"
        lay = Layout((Group(tuple(range(r["cp"])), (0,)),), "contiguous" if sym == "G" else "zigzag")
        got = Evaluator(m, {0: r["tokens"]}, r["cp"], sym).operator(sym, lay)[0]
        assert abs(got - r["fb_ms"]) <= 0.10 * r["fb_ms"], (r, got)


def test_calibration_cli_reproduces_the_committed_file(tmp_path):
    import json
    from pathlib import Path
    from prism_cp_b200.planner import calibrate
    data = Path(calibrate.__file__).resolve().parent / "data"
    out = tmp_path / "cal.json"
    anchors = str(data / "b200_anchor_records.json")
    assert calibrate.main(["--records", str(data / "b200_module_records.json"), "--output", str(out),
                           "--peak-gib", "141.15", "--rescale-records", anchors, "--cp-records", anchors]) == 0
    got, committed = json.loads(out.read_text()), json.loads((data / "b200_operator_calibration.json").read_text())
    assert got["calibration"] == committed["calibration"]
    assert abs(got["byte_scale"] - committed["byte_scale"]) < 1e-9
    assert got["cp_overhead"] == committed["cp_overhead"]


def test_cp_factors_fit_from_module_anchors():
    """Per-operator CP factors are the measured/predicted ratio of one-sequence CP module records;
    the evaluator then prices each operator with its own factor (and 1 without one)."""
    from dataclasses import replace
    from prism_cp_b200.models.config import PRESETS
    from prism_cp_b200.planner.calibrate import calibrated, fit_cp_factors
    from prism_cp_b200.planner.cli import B200_ENVELOPE
    from prism_cp_b200.planner.joint.cost import Evaluator, cp_overhead_factor, model_from_config
    from prism_cp_b200.planner.joint.ir import Group, Layout
    cfg = PRESETS["hybrid-1.3b"]()
    m = replace(calibrated(model_from_config(cfg, B200_ENVELOPE["device_bytes"],
                                             **{k: v for k, v in B200_ENVELOPE.items() if k != "device_bytes"})),
                cp_overhead=None)

    def predicted(sym, cp, tokens):
        lay = Layout((Group(tuple(range(cp)), (0,)),), "contiguous" if sym == "G" else "zigzag")
        return Evaluator(m, {0: tokens}, cp, sym).operator(sym, lay)[0]

    scale = {("G", 2): 1.3, ("G", 4): 1.5, ("*", 2): 1.1, ("*", 4): 1.2}
    records = [{"module": "GDN" if s == "G" else "GQA", "cp": cp, "tokens": n, "sequences": 1,
                "fb_ms": f * predicted(s, cp, n)} for (s, cp), f in scale.items() for n in (65536, 131072)]
    records.append({"module": "GQA", "cp": 1, "tokens": 65536, "sequences": 1, "fb_ms": 1.0})  # ignored
    table = fit_cp_factors(m, records)
    for (s, cp), f in scale.items():
        assert abs(table[s][str(cp)] - f) < 1e-9
    assert cp_overhead_factor(table, 8, "G") == table["G"]["4"]
    assert cp_overhead_factor(table, 2, "M") == 1.0
    priced = replace(m, cp_overhead=table)
    lay = Layout((Group((0, 1), (0,)),), "contiguous")
    got = Evaluator(priced, {0: 65536}, 2, "G").operator("G", lay)[0]
    assert abs(got - 1.3 * predicted("G", 2, 65536)) < 1e-9


def test_committed_b200_anchor_profile_prices_its_own_anchors():
    """The B200 anchor profile built from the committed module records validates against the 1.3B
    model and, used as the CP response, prices a 65,536-token sequence at every measured CP degree at
    exactly its measured time."""
    import json
    from dataclasses import replace
    from pathlib import Path
    from prism_cp_b200.models.config import PRESETS
    from prism_cp_b200.planner import profile_builder
    from prism_cp_b200.planner.cli import B200_ENVELOPE
    from prism_cp_b200.planner.joint.cost import Evaluator, model_from_config
    from prism_cp_b200.planner.joint.ir import Group, Layout
    data = Path(profile_builder.__file__).resolve().parent / "data"
    committed = json.loads((data / "b200_cp_anchors.json").read_text())
    records = json.loads((data / "b200_anchor_records.json").read_text())
    rebuilt = profile_builder.build(records["records"], 65536, records["model_shape"], committed["name"],
                                    committed["source"])
    assert rebuilt == committed
    cfg = PRESETS["hybrid-1.3b"]()
    m = replace(model_from_config(cfg, B200_ENVELOPE["device_bytes"],
                                  **{k: v for k, v in B200_ENVELOPE.items() if k != "device_bytes"}),
                cp_response=committed)
    for kind, sym in (("GQA", "*"), ("GDN", "G")):
        for cp, ms in committed["anchors"][kind]["milliseconds"].items():
            cp = int(cp)
            lay = Layout((Group(tuple(range(cp)), (0,)),), "zigzag" if sym == "*" else "contiguous")
            got = Evaluator(m, {0: 65536}, cp, sym).operator(sym, lay)[0]
            assert abs(got - ms) < 1e-6 * ms, (kind, cp, got, ms)
