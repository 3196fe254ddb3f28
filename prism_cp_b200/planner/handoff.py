"""CPU self-check of the planner stack before plans are handed to GPUs.

The reference re-validates its fit observations, response profiles, a cached
plan score, a small solve + replay and the frozen native/joint plans
(experiments/sequence_dynamic_cp/handoff_check.py:33-144). This check covers
the same ground for this framework's own artefacts:

* native fixed-N re-derivation reproduces every frozen reference plan shipped
  in ``planner/data/native_golden_plans.json``;
* an exact and a bounded joint solve on a small pool agree with an
  independent re-score, and the compiled replay validates;
* the catalogue cover and the memory tie-break run on a tiny pool;
* every response profile in ``planner/configs`` validates against its model;
* the CP1 cost fit recovers known coefficients exactly;
* the LCG content stream is deterministic across span boundaries.

``python -m prism_cp_b200.planner.handoff`` prints a JSON report and exits 1
on the first failed check class.
"""

from __future__ import annotations

import json
import math
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def check_native() -> dict:
    from .native import replay
    cases = json.loads((HERE / "data" / "native_golden_plans.json").read_text())
    bad = [c["source"] for c in cases
           if replay(list(enumerate(c["lengths"])), c["world"], c["capacity_tokens"]) != c["rank_ids"]]
    return {"frozen_plans": len(cases), "mismatches": bad, "ok": not bad}


def check_solve() -> dict:
    from .inputs import build_manifest
    from .joint.cost import Evaluator, Model
    from .joint.replay import compile_replay, validate_replay
    from .joint.solver import SearchOptions, solve
    from .joint.ir import Plan
    model = Model(hidden=1024, ffn=4096, vocab=32000, q_heads=8, kv_heads=2, head_dim=128, gdn_heads=8,
                  gdn_dim=128, device_bytes=180 * 10 ** 9, compute_tflops=1400.0, intra_gbps=770.0,
                  memory_gbps=6500.0)
    lengths = [8192, 4096, 2048]
    pool = dict(enumerate(lengths))
    out = {}
    for mode in ("exact", "bounded"):
        res = solve(pool, 2, "G*", model, SearchOptions(mode=mode, max_states=4_000_000))
        plan = Plan.from_dict(res["plan"])
        ev = Evaluator(model, pool, 2, "G*")
        rescored = sum(ev.evaluate(b)["predicted_ms"] for b in plan.microbatches) + model.update_ms
        out[mode] = {"status": res["status"], "predicted_update_ms": res["predicted_update_ms"],
                     "rescored_ms": rescored, "agree": math.isclose(rescored, res["predicted_update_ms"],
                                                                    rel_tol=1e-9)}
    manifest = build_manifest(lengths, "handoff", 2)
    rows = compile_replay(dict(plan=res["plan"]), manifest, 2, "handoff")
    for row in rows:
        validate_replay(row, 2, "G*")
    out["replay_rows"] = len(rows)
    out["exact_not_worse"] = out["exact"]["predicted_update_ms"] <= out["bounded"]["predicted_update_ms"] + 1e-9
    out["ok"] = out["exact"]["agree"] and out["bounded"]["agree"] and out["exact_not_worse"]
    return out


def check_catalogue() -> dict:
    from .joint.cost import Model
    from .joint.ir import Plan
    from .joint.solver import SearchOptions, solve
    from .studies import audit_catalogue, catalogue_template
    model = Model(hidden=1024, ffn=4096, vocab=32000, q_heads=8, kv_heads=2, head_dim=128, gdn_heads=8,
                  gdn_dim=128, device_bytes=180 * 10 ** 9)
    lengths = dict(enumerate([16384, 16384, 2048, 2048, 2048, 2048]))
    res = solve(lengths, 4, "GGG*", model, SearchOptions(beam=4, layouts=4))
    cat = catalogue_template(Plan.from_dict(res["plan"]), lengths, 16384, 2048)
    audit = audit_catalogue(cat, 2, 16384, 4, 2048, 4, "GGG*", model)
    return {"templates": len(cat), "audit_ms": audit["predicted_update_ms"],
            "search_ms": res["predicted_update_ms"],
            "ok": audit["predicted_update_ms"] <= res["predicted_update_ms"] * (1 + 1e-9)}


def check_profiles() -> dict:
    from .joint.cost import Model
    from .joint.response import validate_response
    found, bad = [], []
    for path in sorted((HERE / "configs").glob("*.json")) if (HERE / "configs").is_dir() else []:
        data = json.loads(path.read_text())
        try:
            model = Model(**{k: v for k, v in data.get("model", {}).items()})
            validate_response(data["cp_response"] if "cp_response" in data else data, model)
            found.append(path.name)
        except (ValueError, KeyError, TypeError) as err:
            bad.append(f"{path.name}: {err}")
    return {"profiles": found, "errors": bad, "ok": not bad}


def check_costfit() -> dict:
    from .costfit import fit
    s = [1024 * k for k in range(1, 13)]
    t = [2e-8 * x * x + 3e-4 * x + 0.5 for x in s]
    f = fit("GQA", s, t, "quadratic", holdout_every=4)
    ok = (abs(f.coefficients["S2"] - 2e-8) < 1e-12 and abs(f.coefficients["S"] - 3e-4) < 1e-9
          and f.holdout_max_relative_error is not None and f.holdout_max_relative_error < 1e-9)
    refused = False
    try:
        f.query(4096, cp=2)
    except ValueError:
        refused = True
    return {"coefficients": f.coefficients, "refuses_cp2": refused, "ok": ok and refused}


def check_content() -> dict:
    from .content import materialize_span
    from .inputs import build_manifest
    m = build_manifest([4096, 1024], "handoff_content", 2)
    whole = materialize_span(m, 0, 0, 4096)
    a, b = materialize_span(m, 0, 0, 1000), materialize_span(m, 0, 1000, 4096)
    ok = list(whole["tokens"]) == list(a["tokens"]) + list(b["tokens"])
    return {"ok": ok}


CHECKS = {"native": check_native, "solve": check_solve, "catalogue": check_catalogue, "profiles": check_profiles,
          "costfit": check_costfit, "content": check_content}


def run() -> dict:
    report = {}
    for name, fn in CHECKS.items():
        try:
            report[name] = fn()
        except Exception as err:  # a crash is a failed check, reported with its reason
            report[name] = {"ok": False, "error": f"{type(err).__name__}: {err}"}
    report["ok"] = all(r["ok"] for r in report.values())
    return report


def main(argv=None) -> int:
    report = run()
    print(json.dumps(report, indent=2, default=str))
    return 0 if report["ok"] else 1


if __name__ == "__main__":
    sys.exit(main())
