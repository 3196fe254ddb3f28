"""Calibrate the planner's operator costs to measured single-GPU (CP = 1) module times.

The evaluator prices an operator from analytic FLOPs at ``Model.compute_tflops``
(token-linear work, plus causal-attention work for GQA) and analytic CP
communication. ``calibrate(records, model)`` fits, per operator, the measured
forward + backward milliseconds of single-sequence module-bench records as

    ms = linear_flops / (e_lin * rate) + quadratic_flops / (e_quad * rate) + fixed_ms

with non-negative coefficients (exact active-set NNLS, ``costfit.nnls_exact``),
so ``e_lin`` / ``e_quad`` are the fractions of the envelope the kernels reach
and ``fixed_ms`` the per-call overhead. The result goes into
``Model.operator_calibration``; CP > 1 keeps the analytic communication terms
(at the measured NVLink bandwidth) unless a measured CP response profile is
given. ``fit_byte_scale`` does the same for memory: the activation-byte scale at
which the evaluator's peak of one microbatch equals a measured peak.
``rescale`` moves the multi-length CP = 1 fit to newer one-length records of the
same modules (the kernels got faster since the fit), and ``fit_cp_factors``
gives every CP operator and degree its measured/predicted factor from module
anchors at CP 2/4/8. The committed ``data/b200_operator_calibration.json``
holds all of them, for this framework's own kernels on B200 and the 1.3B shape;
it is regenerated with

    python -m prism_cp_b200.planner.calibrate \
        --records prism_cp_b200/planner/data/b200_module_records.json \
        --output prism_cp_b200/planner/data/b200_operator_calibration.json --peak-gib 141.15 \
        --rescale-records prism_cp_b200/planner/data/b200_anchor_records.json \
        --cp-records prism_cp_b200/planner/data/b200_anchor_records.json
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path

import numpy as np

from .costfit import nnls_exact
from .joint.cost import Evaluator, Model

DEFAULT = Path(__file__).resolve().parent / "data" / "b200_operator_calibration.json"

MODULES = {"GDN": "G", "GQA": "*", "M": "M", "MLP": "M"}


def _analytic_ms(model: Model, symbol: str, tokens: int) -> tuple[float, float]:
    """(linear ms, quadratic ms) the uncalibrated evaluator assigns one CP = 1 sequence of ``tokens``."""
    m = model
    h, f, d = m.hidden, m.ffn, m.gdn_heads * m.gdn_dim
    n = tokens
    rate = m.compute_tflops * 1e9
    if symbol == "M":
        return 18 * n * h * f / rate, 0.0
    if symbol == "*":
        proj = 6 * n * (h * (m.q_heads + 2 * m.kv_heads) * m.head_dim + h * h)
        quad = 6 * m.q_heads * m.head_dim * n * n
        return proj / rate, quad / rate
    return 6 * n * (6 * h * d + 4 * m.gdn_heads * m.gdn_dim ** 2) / rate, 0.0


def load_default() -> dict:
    """The committed B200 operator calibration (fitted on the 1.3B shape)."""
    return json.loads(DEFAULT.read_text())["calibration"]


def load_byte_scale() -> float:
    """The committed activation-byte scale (measured peak of one 32K-token microbatch, 1.3B)."""
    return float(json.loads(DEFAULT.read_text()).get("byte_scale", 1.0))


def calibrated(model: Model) -> Model:
    """``model`` with the committed operator calibration and activation-byte scale."""
    from dataclasses import replace
    cal = {k: {x: v[x] for x in ("linear", "quadratic", "fixed_ms") if x in v} for k, v in load_default().items()}
    cp = json.loads(DEFAULT.read_text()).get("cp_overhead")
    return replace(model, operator_calibration=cal, byte_scale=load_byte_scale(), cp_overhead=cp)


def fit_byte_scale(model: Model, pattern: str, tokens: int, peak_bytes: int) -> float:
    """Activation-byte scale that makes the evaluator's peak of one CP = 1 microbatch of ``tokens``
    equal a measured peak (bisection; the peak grows monotonically with the scale)."""
    from dataclasses import replace
    from .joint.ir import Group, Layout, Microbatch
    one = Layout((Group((0,), (0,)),), "zigzag")
    mb = Microbatch(one, tuple((one, one) for _ in pattern))

    def peak(scale):
        ev = Evaluator(replace(model, byte_scale=scale), {0: tokens}, 1, pattern)
        return max(ev.evaluate(mb)["peak_bytes"])
    lo, hi = 0.05, 20.0
    if not peak(lo) <= peak_bytes <= peak(hi):
        raise ValueError("the measured peak is outside what a byte scale can reach")
    for _ in range(60):
        mid = 0.5 * (lo + hi)
        if peak(mid) < peak_bytes:
            lo = mid
        else:
            hi = mid
    return 0.5 * (lo + hi)


def calibrate(records: list[dict], model: Model) -> dict:
    out = {}
    by_sym: dict = {}
    for r in records:
        if int(r.get("cp", 1)) != 1 or int(r.get("sequences", 1)) != 1:
            continue
        sym = MODULES.get(r["module"])
        if sym is not None:
            by_sym.setdefault(sym, []).append((int(r["tokens"]), float(r["fb_ms"])))
    for sym, pts in sorted(by_sym.items()):
        rows, b = [], []
        for tokens, ms in pts:
            lin, quad = _analytic_ms(model, sym, tokens)
            rows.append([lin, quad, 1.0] if sym == "*" else [lin, 1.0])
            b.append(ms)
        coef = nnls_exact(np.asarray(rows), np.asarray(b))
        if sym == "*":
            a, q, c = (float(x) for x in coef)
        else:
            (a, c), q = (float(x) for x in coef), 0.0
        if a <= 0:
            raise ValueError(f"{sym}: the token-linear term vanished; the records cannot calibrate it")
        cal = {"linear": 1.0 / a, "fixed_ms": c, "points": len(pts)}
        if sym == "*":
            if q <= 0:
                raise ValueError("GQA: the quadratic term vanished")
            cal["quadratic"] = 1.0 / q
        out[sym] = cal
    return out


def fit_cp_overhead(model: Model, pattern: str, lengths: dict, world: int, step_ms: float, cp1_step_ms: float,
                    tokens_per_rank: int) -> float:
    """CP overhead factor on the GDN and attention operators at CP = ``world`` that makes the model's
    CP = world / CP = 1 step ratio for ``lengths`` equal the measured ``step_ms / cp1_step_ms``."""
    from dataclasses import replace
    from .fixed import uniform_plan

    def step(m, w):
        plan = uniform_plan(lengths, w, w, tokens_per_rank, pattern)
        ev = Evaluator(m, lengths, w, pattern)
        return sum(ev.evaluate(mb)["predicted_ms"] for mb in plan.microbatches)
    base = replace(model, cp_overhead=None)
    target = step_ms * step(base, 1) / cp1_step_ms
    lo, hi = 0.5, 3.0
    for _ in range(60):
        mid = 0.5 * (lo + hi)
        if step(replace(base, cp_overhead={str(world): mid}), world) < target:
            lo = mid
        else:
            hi = mid
    return 0.5 * (lo + hi)


def rescale(cal: dict, model: Model, records: list[dict]) -> dict:
    """The CP = 1 calibration moved to newer measurements of the same modules.

    The multi-length fit keeps its shape (the ratio of token-linear, quadratic and fixed terms); each
    operator with newer one-sequence CP = 1 records is scaled so that its price matches their median
    measured/predicted ratio (faster kernels since the fit divide every term by the same factor).
    Operators without newer records keep their fit."""
    import statistics
    from dataclasses import replace
    out = {k: dict(v) for k, v in cal.items()}
    m = replace(model, operator_calibration={k: {x: v[x] for x in ("linear", "quadratic", "fixed_ms") if x in v}
                                             for k, v in cal.items()}, cp_overhead=None)
    ratios: dict = {}
    for r in records:
        sym = MODULES.get(r["module"])
        if int(r.get("cp", 1)) != 1 or int(r.get("sequences", 1)) != 1 or sym not in out:
            continue
        lin, quad = _analytic_ms(m, sym, int(r["tokens"]))
        c = out[sym]
        predicted = lin / c["linear"] + (quad / c["quadratic"] if "quadratic" in c else 0.0) + c.get("fixed_ms", 0.0)
        ratios.setdefault(sym, []).append(float(r["fb_ms"]) / predicted)
    for sym, v in ratios.items():
        f = statistics.median(v)
        c = out[sym]
        c["linear"] /= f
        if "quadratic" in c:
            c["quadratic"] /= f
        c["fixed_ms"] = c.get("fixed_ms", 0.0) * f
        c["rescaled_by"] = f
    return out


def fit_cp_factors(model: Model, records: list[dict]) -> dict:
    """Per operator and CP degree: measured module time over the calibrated model's price.

    ``records`` are module-bench rows at CP > 1 (one sequence of ``tokens`` over a team of ``cp``
    ranks, forward + backward, max over ranks). The factor of (operator, cp) is the median over
    the measured lengths of ``fb_ms / predicted``, where ``predicted`` is what ``model`` (with its
    CP = 1 calibration, without CP factors) assigns the same group; the evaluator multiplies CP
    prices by it. This replaces a single factor fitted to whole-step times with one measured
    anchor set per operator and degree."""
    from dataclasses import replace
    import statistics
    from .joint.ir import Group, Layout
    base = replace(model, cp_overhead=None)
    ratios: dict = {}
    for r in records:
        cp, sym = int(r.get("cp", 1)), MODULES.get(r["module"])
        if cp <= 1 or sym not in ("G", "*") or int(r.get("sequences", 1)) != 1:
            continue
        tokens = int(r["tokens"])
        ev = Evaluator(base, {0: tokens}, cp, sym)
        layout = Layout((Group(tuple(range(cp)), (0,)),), "contiguous" if sym == "G" else "zigzag")
        predicted = ev.operator(sym, layout)[0]
        ratios.setdefault(sym, {}).setdefault(str(cp), []).append(float(r["fb_ms"]) / predicted)
    return {sym: {cp: statistics.median(v) for cp, v in sorted(per.items(), key=lambda kv: int(kv[0]))}
            for sym, per in sorted(ratios.items())}


def _records_of(path: Path) -> list[dict]:
    data = json.loads(path.read_text())
    if "records" in data:
        return list(data["records"])
    return [r for v in data.values() if isinstance(v, dict) for r in v.get("records", [])]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--records", type=Path, required=True, help="module records (one file per module or combined)")
    ap.add_argument("--model-config", default="hybrid-1.3b")
    ap.add_argument("--output", type=Path, required=True)
    ap.add_argument("--peak-gib", type=float, default=None,
                    help="measured peak_allocated of one CP = 1 microbatch (bench.py) for the byte scale")
    ap.add_argument("--peak-tokens", type=int, default=32768)
    ap.add_argument("--bench-steps", type=float, nargs=2, default=None, metavar=("CP1_MS", "CP2_MS"),
                    help="measured bench.py ms/step on one GPU and on two (CP = 2), 8 x 32K tokens")
    ap.add_argument("--rescale-records", type=Path, nargs="*", default=None,
                    help="newer module-bench JSON files: their CP = 1 rows rescale the fitted operators")
    ap.add_argument("--cp-records", type=Path, nargs="*", default=None,
                    help="module-bench JSON files at CP > 1: per-operator, per-degree factors (replaces "
                         "--bench-steps)")
    args = ap.parse_args(argv)
    from dataclasses import replace
    from ..models.config import PRESETS
    from .cli import B200_ENVELOPE
    from .joint.cost import model_from_config
    records = _records_of(args.records)
    cfg = PRESETS[args.model_config]()
    model = model_from_config(cfg, B200_ENVELOPE["device_bytes"],
                              **{k: v for k, v in B200_ENVELOPE.items() if k != "device_bytes"})
    cal = calibrate(records, model)
    out = {"model_config": args.model_config, "compute_tflops": model.compute_tflops,
           "source": str(args.records), "calibration": cal}
    if args.rescale_records:
        cal = rescale(cal, model, [r for path in args.rescale_records for r in _records_of(path)])
        out["calibration"] = cal
        out["rescale_source"] = ", ".join(str(p) for p in args.rescale_records)
    model = replace(model, operator_calibration={k: {x: v[x] for x in ("linear", "quadratic", "fixed_ms") if x in v}
                                                 for k, v in cal.items()})
    if args.peak_gib is not None:
        out["byte_scale"] = fit_byte_scale(model, cfg.pattern, args.peak_tokens, int(args.peak_gib * 2 ** 30))
        out["byte_scale_source"] = f"measured peak_allocated {args.peak_gib} GiB, one {args.peak_tokens}-token microbatch"
        model = replace(model, byte_scale=out["byte_scale"])
    if args.cp_records:
        cp_rows = [r for path in args.cp_records for r in _records_of(path)]
        out["cp_overhead"] = fit_cp_factors(model, cp_rows)
        out["cp_overhead_source"] = ("module bench at CP > 1 (one sequence over a team, forward + backward, max over "
                                     "ranks): " + ", ".join(str(p) for p in args.cp_records))
    elif args.bench_steps is not None:
        lengths = {i: 32768 for i in range(8)}
        out["cp_overhead"] = {"2": fit_cp_overhead(model, cfg.pattern, lengths, 2, args.bench_steps[1],
                                                   args.bench_steps[0], 32768)}
        out["cp_overhead_source"] = (f"bench.py, 8 x 32K tokens: {args.bench_steps[0]} ms per step on one GPU, "
                                     f"{args.bench_steps[1]} ms on two (CP = 2); CP 4 and 8 use it until measured")
    args.output.write_text(json.dumps(out, indent=1) + "\n")
    print(json.dumps({k: out[k] for k in out if k in ("calibration", "byte_scale", "cp_overhead")}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
