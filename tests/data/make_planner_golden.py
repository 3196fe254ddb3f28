"""Golden outputs of the reference planner over a fixed corpus of inputs.

Run once on CPU against a checkout of the reference (LiJunscs/prism-cp):

    python tests/data/make_planner_golden.py /root/reference tests/data/planner_golden.json

It imports the reference's own planner modules (experiments/sequence_dynamic_cp:
joint_cp.solver / model / response / memory_selection / analysis, planner.py,
short_sequence.py, mixed_plan.py, memory_performance_policy.py,
random_batch_capacity_analysis.py) and records what they return for every case
of the corpus below. ``tests/test_planner_golden.py`` replays the same cases
through this package's planner and requires identical plans and scores.

The reference's 1-D search seeds itself with Megatron's native scheduler, which
it compiles from a Megatron source tree outside its repository; that tree is
not available, so the generator hands the reference this package's re-derived
native scheduler (``prism_cp_b200.planner.native.replay``, checked separately
against the reference's frozen native plans). Everything downstream of the
native seed - layouts, LPT packing, local search, short-sequence refinement,
selection and export - is the reference's code.
"""

from __future__ import annotations

import json
import random
import sys
from pathlib import Path

GiB = 1024 ** 3


def _jsonable(x):
    if isinstance(x, dict):
        return {str(k): _jsonable(v) for k, v in x.items()}
    if isinstance(x, (list, tuple)):
        return [_jsonable(v) for v in x]
    if isinstance(x, float) and x != x:
        return None
    return x


# ------------------------------------------------------------------ corpus
def joint_cases(configs: dict) -> list[dict]:
    rng = random.Random(20261202)
    cases = []

    def add(name, lengths, world, pattern, model, **options):
        cases.append(dict(name=name, lengths={str(k): v for k, v in lengths.items()}, world=world, pattern=pattern,
                          model=model, options=options))

    # exact domain: <= 6 samples, <= 4 ranks
    add("exact_w2_two", {0: 4096, 1: 8192}, 2, "G*", "default", mode="exact")
    add("exact_w4_pair", {0: 16384, 1: 4096}, 4, "G*", "default", mode="exact")
    add("exact_w2_three", {0: 65536, 1: 8192, 2: 8192}, 2, "G*", "small", mode="exact")
    add("exact_w4_budget", {0: 16384, 1: 4096, 2: 4096, 3: 8192}, 4, "GGG*", "default", mode="exact",
        max_states=200000)
    # bounded: uniform, mixed, heavy-tailed and irregular pools on 2..16 ranks
    add("uniform_w8", {i: 8192 for i in range(16)}, 8, "GGG*GGG*", "default")
    add("uniform_w4_long", {i: 32768 for i in range(6)}, 4, "GGG*", "default")
    for world in (2, 4, 8, 16):
        for trial in range(3):
            n = rng.randint(3, 24)
            lengths = {i: rng.choice((1024, 2048, 4096, 8192, 16384, 32768, 65536)) for i in range(n)}
            add(f"mixed_w{world}_{trial}", lengths, world, "GGG*GGG*", "default")
    for world in (8, 16):
        lengths = {0: 262144, 1: 131072, **{i: 4096 for i in range(2, 34)}}
        add(f"heavy_w{world}", lengths, world, "GGG*GGG*", "default")
        add(f"heavy_w{world}_balanced", lengths, world, "GGG*GGG*", "default", balanced_packing=True)
        add(f"heavy_w{world}_heavytail", lengths, world, "GGG*GGG*", "default", heavy_tail_packing=True)
    irregular = {i: n for i, n in enumerate((40960, 49152, 57344, 65536) * 2)}
    irregular.update({8 + i: 2048 for i in range(32)})
    add("irregular_w16_measured", irregular, 16, "GGG*GGG*", "measured16")
    add("irregular_w16_h100", irregular, 16, "GGG*GGG*", "h100_16")
    add("irregular_w16_h100_homog", irregular, 16, "GGG*GGG*", "h100_16", homogeneous_packing=True)
    add("irregular_w16_rpn4_affine", irregular, 16, "GGG*GGG*", "rpn4", node_affinity=True)
    add("irregular_w16_maxcp2", irregular, 16, "GGG*GGG*", "default", max_attention_cp=2)
    add("irregular_w16_beam4", irregular, 16, "GGG*GGG*", "default", beam=4, layouts=4)
    long_pool = {0: 262144, 1: 262144, **{i: 8192 for i in range(2, 18)}}
    add("long_w32_h100", long_pool, 32, "GGG*GGG*", "h100_32")
    add("long_w16_small", {0: 131072, 1: 65536, 2: 16384, 3: 16384}, 16, "GGG*", "small")
    add("short_pattern_w4", {i: rng.choice((2048, 4096, 6144, 8192)) for i in range(10)}, 4, "G*G*", "default")
    add("mixed_w8_tolerance", {i: rng.choice((4096, 8192, 16384)) for i in range(20)}, 8, "GGG*GGG*", "default",
        memory_time_tolerance=0.05)
    return cases


def model_specs(ref: Path) -> dict:
    cfg = ref / "experiments/sequence_dynamic_cp/configs"
    load = lambda name: json.loads((cfg / name).read_text())  # noqa: E731
    return {
        "default": {},
        "small": {"device_bytes": 40 * GiB},
        "rpn4": {"ranks_per_node": 4},
        "measured16": load("joint_16gpu_measured.json"),
        "h100_16": load("joint_16gpu_h100.json"),
        "h100_32": load("joint_32gpu_h100.json"),
    }


def onedim_cases() -> list[dict]:
    rng = random.Random(20261203)
    cases = []
    for world, min_cp in ((2, 1), (4, 1), (8, 2), (16, 4), (16, 1)):
        for trial in range(3):
            n = rng.randint(1, 40)
            lengths = {i: rng.choice((2048, 4096, 8192, 16384, 32768)) for i in range(n)}
            cases.append(dict(name=f"w{world}_min{min_cp}_{trial}", lengths={str(k): v for k, v in lengths.items()},
                              world=world, token_cap=16384, min_cp=min_cp, max_sequences=None,
                              alignment=2 * world, cost="hybrid", local_evaluations=24, rounds=2))
    cases.append(dict(name="square_counterexample_shape", lengths={str(i): (16384 if i == 0 else 2048)
                                                                    for i in range(40)},
                      world=16, token_cap=32768, min_cp=1, max_sequences=None, alignment=32, cost="gpt",
                      local_evaluations=64, rounds=2))
    cases.append(dict(name="max_sequences", lengths={str(i): rng.choice((1024, 2048, 4096)) for i in range(30)},
                      world=4, token_cap=8192, min_cp=1, max_sequences=3, alignment=8, cost="hybrid",
                      local_evaluations=128, rounds=3))
    return cases


def policy_cases() -> dict:
    rng = random.Random(7)
    trade = []
    for _ in range(40):
        rt, rp = rng.uniform(50, 200), rng.uniform(20, 80)
        ct, cpk = rt * rng.uniform(0.6, 1.4), rp * rng.uniform(0.7, 1.6)
        trade.append(dict(args=[rt, rp, ct, cpk], multiplier=rng.choice((0.0, 1.0, 2.0, 3.5)),
                          fits=rng.random() > 0.2))
    sets = []
    for s in range(6):
        cands = [dict(id="N_ref", kind="native", time=100.0, peak=50.0, fits=True)]
        for j in range(rng.randint(3, 9)):
            kind = rng.choice(("native", "joint"))
            cands.append(dict(id=f"{'N' if kind == 'native' else 'J'}_{s}_{j}", kind=kind,
                              time=rng.uniform(70, 130), peak=rng.uniform(35, 90), fits=rng.random() > 0.15))
        sets.append(dict(candidates=cands, reference="N_ref", multiplier=rng.choice((1.0, 2.0))))
    shortlists = [sorted(rng.choice((4096, 8192, 24576, 40960, 65536, 98304, 131072, 262144))
                         for _ in range(rng.randint(1, 12))) for _ in range(10)]
    # capacity cases for choose / integrate
    cases = []
    for c in range(5):
        native = []
        for k in (8192, 12288, 16384, 20480, 24576, 32768):
            scores = {p: dict(predicted_update_ms=rng.uniform(5000, 9000), peak_gib=rng.uniform(30, 80),
                              model_fits=rng.random() > 0.1) for p in ("paired_linear", "paired_quadratic")}
            if k == 16384:
                for sc in scores.values():
                    sc["model_fits"] = True
            native.append(dict(id=f"N_K{k // 1024}", capacity_tokens=k, scores=scores))
        joint = [dict(id=f"J_{c}_{j}", scores={p: dict(predicted_update_ms=rng.uniform(4500, 9500),
                                                        peak_gib=rng.uniform(30, 80), model_fits=rng.random() > 0.2)
                                                for p in ("paired_linear", "paired_quadratic")})
                 for j in range(3)]
        cases.append(dict(case=f"case{c}", input_tokens=rng.randint(1500000, 2500000), native=native, joint=joint,
                          simple_capacity_tokens=[8192, 16384, 24576]))
    weights = {f"case{c}": w for c, w in zip(range(5), (0.1, 0.2, 0.3, 0.25, 0.15))}
    return dict(tradeoff=trade, select=sets, shortlists=shortlists, cases=cases, weights=weights)


# ------------------------------------------------------------------ generation
def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    ref, out = Path(argv[0]), Path(argv[1])
    sd = ref / "experiments/sequence_dynamic_cp"
    sys.path.insert(0, str(sd))
    sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
    from prism_cp_b200.planner.native import replay as native_replay
    import native as ref_native
    ref_native.replay = native_replay
    import planner as ref_planner
    ref_planner.replay = native_replay
    from joint_cp.model import Model
    from joint_cp.solver import SearchOptions, solve
    from joint_cp.analysis import describe
    from joint_cp.memory_selection import prefer_lower_memory
    from joint_cp.ir import Plan
    import mixed_plan
    import memory_performance_policy as mpp
    import random_batch_capacity_analysis as rbca

    specs = model_specs(ref)
    golden = dict(models=specs, joint=[], onedim=[], memory=[], mixed=[], policy={})

    for case in joint_cases(specs):
        lengths = {int(k): v for k, v in case["lengths"].items()}
        model = Model(**specs[case["model"]])
        try:
            result = solve(lengths, case["world"], case["pattern"], model, SearchOptions(**case["options"]))
        except Exception as error:  # recorded: the rewrite must raise the same way
            golden["joint"].append(_jsonable(dict(case, error=type(error).__name__, message=str(error))))
            print("joint", case["name"], "raised", type(error).__name__, flush=True)
            continue
        row = dict(case, status=result["status"], plan=result["plan"],
                   predicted_update_ms=result.get("predicted_update_ms"),
                   states_examined=result["states_examined"],
                   pool_packings_examined=result["pool_packings_examined"],
                   microbatch_shapes_solved=result["microbatch_shapes_solved"],
                   beam_pruned=result["beam_pruned"], memory_selection=result.get("memory_selection"),
                   resource_metrics=result.get("resource_metrics"),
                   cp_response_evidence=result.get("cp_response_evidence"),
                   peaks=[list(e["peak_bytes"]) for e in result.get("microbatch_evidence", [])],
                   describe=describe(result, lengths, model) if result["plan"] else None)
        golden["joint"].append(_jsonable(row))
        print("joint", case["name"], result["status"], result.get("predicted_update_ms"), flush=True)

    # the memory tie-break on hand-made CP1 plans (rank-resident homogeneous families)
    from joint_cp.ir import Group, Layout, Microbatch
    for world, n, length in ((4, 24, 4096), (8, 40, 8192), (2, 9, 16384)):
        lengths = {i: length for i in range(n)}
        per = -(-n // world)
        batches = []
        for start in range(0, per, 3):
            groups = []
            for r in range(world):
                ids = tuple(i for i in range(r * per + start, min(r * per + start + 3, (r + 1) * per)) if i < n)
                groups.append(Group((r,), ids))
            if any(not g.samples for g in groups):
                continue
            ing = Layout(tuple(groups), "zigzag")
            con = ing.with_mode("contiguous")
            batches.append(Microbatch(ing, tuple((con if c == "G" else ing, con) for c in "GGG*")))
        covered = {s for b in batches for g in b.ingress.groups for s in g.samples}
        lengths = {s: lengths[s] for s in covered}
        plan = Plan(world, "GGG*", tuple(batches))
        for tol in (0.0, 0.001, 0.2):
            chosen, meta = prefer_lower_memory(plan, lengths, Model(), tol)
            golden["memory"].append(_jsonable(dict(world=world, lengths={str(k): v for k, v in lengths.items()},
                                                   plan=plan.to_dict(), tolerance=tol, selected=chosen.to_dict(),
                                                   meta=meta)))

    costs = ref_planner.models(ref / "experiments/performance_model/results/cp1_20261009_p1_v2/"
                                     "stack_coefficients.json")
    golden["proxy_costs"] = {k: dict(a=v.a, b=v.b, provenance=v.provenance) for k, v in costs.items()}
    for case in onedim_cases():
        lengths = {int(k): v for k, v in case["lengths"].items()}
        limits = ref_planner.Constraints(case["world"], case["token_cap"], case["min_cp"], case["max_sequences"],
                                         case["alignment"])
        cost = costs[case["cost"]]
        try:
            result = ref_planner.search(lengths, limits, cost, case["local_evaluations"], case["rounds"])
        except ValueError as error:
            golden["onedim"].append(dict(case, error=str(error)))
            continue
        sel = result["selected"]
        row = dict(case, selected=dict(name=sel["name"], fingerprint=sel["fingerprint"],
                                       proxy_cost=sel["proxy_cost"],
                                       rank_ids=ref_planner.to_rank_ids(sel["plan"], case["world"])),
                   candidates=[dict(name=c["name"], fingerprint=c["fingerprint"], proxy_cost=c["proxy_cost"])
                               for c in result["candidates"]],
                   failures=result["failures"], local_evaluations=result["local_evaluations"],
                   refinement={k: v for k, v in result["short_sequence_refinement"].items() if k != "planning_ms"},
                   export=ref_planner.export_plan(sel["plan"], lengths, cost, 8),
                   proxy_select=ref_planner.select(result, lengths, None, True)[1],
                   native_select=ref_planner.select(result, lengths, None, False)[1]
                   if any(c["name"] == "native_square" for c in result["candidates"]) else None)
        rounds = mixed_plan.coalesce_rounds(sel["plan"], lengths, case["world"], case["token_cap"],
                                            case["max_sequences"])
        row["coalesced"] = rounds
        golden["onedim"].append(_jsonable(row))
        print("onedim", case["name"], sel["name"], sel["proxy_cost"], flush=True)

    pc = policy_cases()
    golden["policy"]["tradeoff"] = [dict(c, result=mpp.tradeoff(*c["args"], min_gain_per_memory_growth=c["multiplier"],
                                                                fits=c["fits"])) for c in pc["tradeoff"]]
    sel_rows = []
    for s in pc["select"]:
        try:
            res = mpp.select(s["candidates"], s["reference"], s["multiplier"])
        except ValueError as error:
            res = dict(error=str(error))
        sel_rows.append(dict(s, result=res))
    golden["policy"]["select"] = sel_rows
    golden["policy"]["shortlists"] = [dict(lengths=ls, result=rbca.capacity_shortlist(ls))
                                      for ls in pc["shortlists"]]
    golden["policy"]["choose"] = []
    for case in pc["cases"]:
        for p in ("paired_linear", "paired_quadratic"):
            for m in ("physical", "alpha2"):
                golden["policy"]["choose"].append(dict(case=case["case"], policy=p, preference=m,
                                                       result=rbca.choose(case, p, m)))
    golden["policy"]["integrate"] = {f"{p}/{m}": rbca.integrate(pc["cases"], pc["weights"], p, m)
                                     for p in ("paired_linear", "paired_quadratic") for m in ("physical", "alpha2")}
    golden["policy"]["cases"] = pc["cases"]
    golden["policy"]["weights"] = pc["weights"]
    out.write_text(json.dumps(_jsonable(golden), sort_keys=True) + "\n")
    print("wrote", out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
