"""Planner command line: ``python -m prism_cp_b200.planner.cli <command> ...``.

Commands
  search   joint sequence x layer search over a frozen input manifest; writes
           result.json, replay.json and executor.json (flags follow the reference
           experiments/sequence_dynamic_cp/joint_cp_search.py:16-85)
  scale    free-pool scale search over (long, short) sample pools
  audit    catalogue cover of a (long, short) pool from saved scale results
  study    native fixed-N (capacity grid) versus the joint plan, alpha-rule selection
  native   the native fixed-N plan of a manifest at one capacity, as a joint plan
  profile  build a B200 CP response profile from module-bench records
  fit      fit CP1 module costs from module-bench records
  handoff  CPU self-check of the planner stack

Hardware models: ``--hardware B200`` uses this framework's B200 envelope
(180 GB HBM3e, NVLink 5 through NVSwitch) with operator costs calibrated to
measured single-GPU module times of this framework's kernels
(``calibrate.py``; ``--uncalibrated`` keeps the analytic envelope);
``--model-profile`` loads any Model JSON, including the reference's H100/H800
profiles, which share the schema.
"""

from __future__ import annotations

import argparse
import json
import sys
from dataclasses import asdict, replace
from pathlib import Path

from .inputs import validate_manifest
from .joint.cost import Model, execution_contract, model_from_config
from .joint.ir import Plan
from .joint.replay import compile_replay
from .joint.solver import SearchLimit, SearchOptions, solve

B200_ENVELOPE = dict(device_bytes=180 * 10 ** 9, compute_tflops=1400.0, intra_gbps=770.0, inter_gbps=50.0,
                     memory_gbps=6500.0, ranks_per_node=8,
                     provenance="B200 envelope: measured copy/GEMM peaks, NVLink 5 peer bandwidth; analytic terms")


def build_model(args) -> Model:
    fields = {}
    if getattr(args, "model_profile", None):
        fields = json.loads(Path(args.model_profile).read_text())
        return Model(**fields)
    if getattr(args, "model_config", None):
        from ..models.config import PRESETS
        cfg = PRESETS[args.model_config]()
        model = model_from_config(cfg, B200_ENVELOPE["device_bytes"],
                                  **{k: v for k, v in B200_ENVELOPE.items() if k != "device_bytes"})
    else:
        model = Model(**B200_ENVELOPE)
    if not getattr(args, "uncalibrated", False) and getattr(args, "hardware", "B200") == "B200":
        from .calibrate import calibrated
        model = replace(calibrated(model),
                        provenance=model.provenance + "; operator costs and activation bytes calibrated to "
                                                      "measured B200 module times and peak memory")
    if getattr(args, "cp_response", None):
        profile = json.loads(Path(args.cp_response).read_text())
        model = replace(model, cp_response=profile,
                        provenance=model.provenance + "; CP response: " + profile.get("name", "profile"))
    return model


def search_options(args) -> SearchOptions:
    return SearchOptions(mode=args.mode, beam=args.beam, layouts=args.layouts, max_states=args.max_states,
                         node_affinity=args.node_affinity, homogeneous_packing=args.homogeneous_packing,
                         balanced_packing=args.balanced_packing, heavy_tail_packing=args.heavy_tail_packing,
                         max_attention_cp=args.max_attention_cp, memory_time_tolerance=args.memory_time_tolerance)


def _model_args(ap):
    g = ap.add_mutually_exclusive_group()
    g.add_argument("--model-profile", type=Path, help="Model JSON (reference H100/H800 profiles load unchanged)")
    g.add_argument("--hardware", choices=("B200",), default="B200")
    ap.add_argument("--model-config", help="framework model preset (e.g. hybrid-1.3b) for the model shape")
    ap.add_argument("--cp-response", type=Path, help="CP response profile JSON (e.g. a B200 anchor profile)")
    ap.add_argument("--uncalibrated", action="store_true",
                    help="analytic operator costs at the B200 envelope, without the measured module calibration")


def _search_args(ap):
    ap.add_argument("--mode", choices=("exact", "bounded"), default="bounded")
    ap.add_argument("--node-affinity", action="store_true")
    ap.add_argument("--homogeneous-packing", action="store_true")
    ap.add_argument("--balanced-packing", action="store_true")
    ap.add_argument("--heavy-tail-packing", action="store_true")
    ap.add_argument("--max-attention-cp", type=int)
    ap.add_argument("--memory-time-tolerance", type=float, default=0.001)
    ap.add_argument("--beam", type=int, default=8)
    ap.add_argument("--layouts", type=int, default=8)
    ap.add_argument("--max-states", type=int, default=1_000_000)


def cmd_search(args) -> int:
    manifest = json.loads(args.manifest.read_text())
    validate_manifest(manifest)
    model = build_model(args)
    options = search_options(args)
    lengths = dict(enumerate(s["length"] for s in manifest["samples"]))
    args.output.mkdir(parents=True, exist_ok=False)
    try:
        result = solve(lengths, args.world, args.pattern, model, options)
    except SearchLimit as err:
        result = dict(status="search_budget_exhausted", plan=None, reason=str(err), gpu_admitted=False)
    result.update(model=asdict(model), search_options=asdict(options), input_manifest=str(args.manifest.resolve()),
                  input_tokens=sum(lengths.values()))
    (args.output / "result.json").write_text(json.dumps(result, indent=2) + "\n")
    if result["plan"] is None:
        print(json.dumps(dict(status=result["status"], gpu_admitted=False)))
        return 2
    replay = compile_replay(result, manifest, args.updates, args.output.name)
    (args.output / "replay.json").write_text(json.dumps(replay, separators=(",", ":")) + "\n")
    executor = dict(mode="joint", model_contract=execution_contract(model), vocab_size=model.vocab,
                    model_provenance=model.provenance)
    (args.output / "executor.json").write_text(json.dumps(executor, indent=2) + "\n")
    print(json.dumps(dict(status=result["status"], microbatches=len(result["plan"]["microbatches"]),
                          ingress_allocation_tokens=replay[0]["capacity_tokens"],
                          predicted_update_ms=result["predicted_update_ms"],
                          resource_metrics=result["resource_metrics"], gpu_admitted=False)))
    return 0


def cmd_scale(args) -> int:
    from .studies import catalogue_template, scale_case
    model = build_model(args)
    args.output.mkdir(parents=True, exist_ok=False)
    summary, catalogue = [], []
    for case in args.cases:
        n_long, long_len, n_short, short_len = (int(x) for x in case.split(":"))
        out = scale_case(n_long, long_len, n_short, short_len, args.world, args.pattern, model,
                         search_options(args))
        name = f"{n_long}x{long_len}_{n_short}x{short_len}"
        (args.output / f"{name}_result.json").write_text(json.dumps(out["result"], separators=(",", ":")) + "\n")
        if out["result"]["plan"] is not None:
            lengths = dict(enumerate([long_len] * n_long + [short_len] * n_short))
            catalogue += catalogue_template(Plan.from_dict(out["result"]["plan"]), lengths, long_len, short_len)
        summary.append(dict(out["row"], case=name))
        print(json.dumps(summary[-1]), flush=True)
    (args.output / "summary.json").write_text(json.dumps(summary, indent=2) + "\n")
    (args.output / "catalogue.json").write_text(json.dumps(catalogue) + "\n")
    return 0


def cmd_audit(args) -> int:
    from .studies import audit_catalogue
    model = build_model(args)
    catalogue = []
    for path in args.catalogues:
        catalogue += json.loads(Path(path).read_text())
    n_long, long_len, n_short, short_len = (int(x) for x in args.case.split(":"))
    result = audit_catalogue(catalogue, n_long, long_len, n_short, short_len, args.world, args.pattern, model,
                             args.max_attention_cp, args.memory_time_tolerance)
    args.output.write_text(json.dumps(result, separators=(",", ":")) + "\n")
    print(json.dumps({k: result[k] for k in ("status", "predicted_update_ms", "catalogue_templates",
                                            "usable_templates")}))
    return 0


def _manifest_lengths(path: Path) -> dict:
    manifest = json.loads(path.read_text())
    validate_manifest(manifest)
    return dict(enumerate(s["length"] for s in manifest["samples"]))


def cmd_study(args) -> int:
    from .studies import native_vs_joint, report_markdown
    model = build_model(args)
    lengths = _manifest_lengths(args.manifest)
    report = native_vs_joint(lengths, args.world, args.pattern, model, args.capacities, args.reference_capacity,
                             args.alpha, search_options(args))
    args.output.mkdir(parents=True, exist_ok=False)
    (args.output / "study.json").write_text(json.dumps(report, indent=2, default=float) + "\n")
    (args.output / "REPORT.md").write_text(report_markdown(report))
    print(json.dumps({"selected": report["decision"]["selected"],
                      "joint_speedup_vs_reference": report["joint_speedup_vs_reference"]}))
    return 0


def cmd_native(args) -> int:
    from .studies import native_joint_plan, plan_score
    model = build_model(args)
    lengths = _manifest_lengths(args.manifest)
    plan = native_joint_plan(lengths, args.world, args.pattern, args.capacity)
    score = plan_score(plan, lengths, model)
    args.output.write_text(json.dumps({"plan": plan.to_dict(), "score": score}) + "\n")
    print(json.dumps(score))
    return 0


def resolve_pattern(args) -> None:
    """A plan covers the model's own layers: the preset's pattern unless one is given."""
    if getattr(args, "pattern", "unset") is None:
        if getattr(args, "model_config", None):
            from ..models.config import PRESETS
            args.pattern = PRESETS[args.model_config]().pattern
        else:
            args.pattern = "GGG*GGG*"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="prism_cp_b200.planner.cli", description=__doc__.splitlines()[0])
    sub = ap.add_subparsers(dest="command", required=True)

    s = sub.add_parser("search", help="joint search over a frozen manifest")
    s.add_argument("--manifest", type=Path, required=True)
    s.add_argument("--output", type=Path, required=True)
    s.add_argument("--world", type=int, default=8)
    s.add_argument("--pattern", default=None,
                   help="layer pattern (default: the --model-config preset's, else GGG*GGG*)")
    s.add_argument("--updates", type=int, default=3)
    _search_args(s)
    _model_args(s)
    s.set_defaults(fn=cmd_search)

    sc = sub.add_parser("scale", help="free-pool scale search; CASE = n_long:long_len:n_short:short_len")
    sc.add_argument("--output", type=Path, required=True)
    sc.add_argument("--cases", nargs="+", required=True)
    sc.add_argument("--world", type=int, default=8)
    sc.add_argument("--pattern", default=None,
                   help="layer pattern (default: the --model-config preset's, else GGG*GGG*)")
    _search_args(sc)
    _model_args(sc)
    sc.set_defaults(fn=cmd_scale)

    au = sub.add_parser("audit", help="catalogue cover and audit of one pool")
    au.add_argument("--catalogues", nargs="+", required=True)
    au.add_argument("--case", required=True)
    au.add_argument("--output", type=Path, required=True)
    au.add_argument("--world", type=int, default=8)
    au.add_argument("--pattern", default=None,
                   help="layer pattern (default: the --model-config preset's, else GGG*GGG*)")
    au.add_argument("--max-attention-cp", type=int)
    au.add_argument("--memory-time-tolerance", type=float, default=0.001)
    _model_args(au)
    au.set_defaults(fn=cmd_audit)

    st = sub.add_parser("study", help="native N capacity grid versus the joint plan")
    st.add_argument("--manifest", type=Path, required=True)
    st.add_argument("--output", type=Path, required=True)
    st.add_argument("--world", type=int, default=8)
    st.add_argument("--pattern", default=None,
                   help="layer pattern (default: the --model-config preset's, else GGG*GGG*)")
    st.add_argument("--capacities", type=int, nargs="+", default=[8192, 16384, 24576, 32768, 40960])
    st.add_argument("--reference-capacity", type=int, default=16384)
    st.add_argument("--alpha", type=float, default=2.0)
    _search_args(st)
    _model_args(st)
    st.set_defaults(fn=cmd_study)

    nv = sub.add_parser("native", help="native fixed-N plan of a manifest")
    nv.add_argument("--manifest", type=Path, required=True)
    nv.add_argument("--output", type=Path, required=True)
    nv.add_argument("--world", type=int, default=8)
    nv.add_argument("--pattern", default=None,
                   help="layer pattern (default: the --model-config preset's, else GGG*GGG*)")
    nv.add_argument("--capacity", type=int, default=16384)
    _model_args(nv)
    nv.set_defaults(fn=cmd_native)

    pr = sub.add_parser("profile", help="B200 CP response profile from module-bench records")
    pr.add_argument("rest", nargs=argparse.REMAINDER)
    pr.set_defaults(fn=lambda a: __import__("prism_cp_b200.planner.profile_builder",
                                            fromlist=["main"]).main(a.rest) or 0)
    ft = sub.add_parser("fit", help="CP1 module cost fit")
    ft.add_argument("rest", nargs=argparse.REMAINDER)
    ft.set_defaults(fn=lambda a: __import__("prism_cp_b200.planner.costfit", fromlist=["main"]).main(a.rest) or 0)
    ho = sub.add_parser("handoff", help="CPU self-check of the planner stack")
    ho.add_argument("rest", nargs=argparse.REMAINDER)
    ho.set_defaults(fn=lambda a: __import__("prism_cp_b200.planner.handoff", fromlist=["main"]).main(a.rest))

    args = ap.parse_args(argv)
    resolve_pattern(args)
    return int(args.fn(args) or 0)


if __name__ == "__main__":
    sys.exit(main())
