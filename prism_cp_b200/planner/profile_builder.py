"""Build a B200 CP response profile (``b200_operator_anchors_v1``) from module-bench records.

The reference builds its H100 profiles from per-node module medians
(experiments/sequence_dynamic_cp/build_h100_cp_profile.py:17-76). On one
8-GPU NVSwitch box every CP degree 1/2/4/8 is measured directly, so the
profile keeps one anchor per (operator, CP): the median over repeats (and over
ranks' max, which the bench already records) of the module's forward+backward
time at ``anchor_tokens`` tokens. No CP is extrapolated; shapes other than the
anchor scale by declared useful work (``operator_work``) in the evaluator.
"""

from __future__ import annotations

import argparse
import json
import statistics
from pathlib import Path

from .joint.response import B200_SCHEMA


def build(records: list[dict], anchor_tokens: int, model_shape, name: str = "b200_module_bench",
          source: str = "") -> dict:
    """records: dicts with module ('GQA'/'GDN'), cp, tokens, fb_ms (max over ranks)."""
    anchors = {}
    for module in ("GQA", "GDN"):
        per_cp: dict[str, list] = {}
        for r in records:
            if r["module"] == module and int(r["tokens"]) == anchor_tokens:
                per_cp.setdefault(str(int(r["cp"])), []).append(float(r["fb_ms"]))
        if not per_cp:
            raise ValueError(f"no {module} records at {anchor_tokens} tokens")
        anchors[module] = {"milliseconds": {cp: statistics.median(v) for cp, v in sorted(per_cp.items(),
                                                                                         key=lambda kv: int(kv[0]))},
                           "repeats": {cp: len(v) for cp, v in per_cp.items()}}
    if set(anchors["GQA"]["milliseconds"]) != set(anchors["GDN"]["milliseconds"]):
        raise ValueError("GQA and GDN must be measured at the same CP degrees")
    return {"schema": B200_SCHEMA, "name": name, "hardware": "B200", "anchor_tokens": anchor_tokens,
            "model_shape": list(model_shape), "anchors": anchors, "source": source,
            "shape_policy": "useful_work_scaling", "unmeasured_cp_policy": "rejected"}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--records", type=Path, nargs="+", required=True,
                    help="module bench JSON files (one per module and CP degree, or combined)")
    ap.add_argument("--anchor-tokens", type=int, required=True)
    ap.add_argument("--output", type=Path, required=True)
    ap.add_argument("--name", default="b200_module_bench")
    args = ap.parse_args(argv)
    records, shape = [], None
    for path in args.records:
        data = json.loads(path.read_text())
        records += data["records"]
        if shape is not None and list(data["model_shape"]) != list(shape):
            raise ValueError(f"{path}: measured for a different model shape")
        shape = data["model_shape"]
    prof = build(records, args.anchor_tokens, shape, args.name, ", ".join(str(p) for p in args.records))
    args.output.write_text(json.dumps(prof, indent=2) + "\n")
    print(json.dumps({k: prof["anchors"][k]["milliseconds"] for k in prof["anchors"]}))


if __name__ == "__main__":
    main()
