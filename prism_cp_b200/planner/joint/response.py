"""Hardware CP response: turn measured module timings into per-operator cost.

Three profile schemas are understood (all JSON-serialisable dicts carried in
``Model.cp_response``):

* ``joint_cp_response_v1`` - residual fits per CP 2/4/8 on top of the analytic
  cost (``quadratic_fraction``, ``token_fraction``, ``fixed_ms``), optional
  paired CP16 GQA anchors (linear or quadratic residual) and explicit CP32
  hypotheses (reference schema: joint_cp/response.py:57-122,153-199).
* ``h100_operator_anchors_v1`` - full-module F+B anchors at one length for
  CP 8/16(/32); other shapes scale by declared useful work, CP 1/2/4 by
  ``T8 * 8 / p`` (reference: joint_cp/response.py:32-54,157-170).
* ``b200_operator_anchors_v1`` - this framework's own profile, written by
  ``prism_cp_b200.planner.profile_builder`` from the B200 module bench: anchors
  measured at every CP in the profile's domain (1, 2, 4, 8 on one NVSwitch
  box), so no CP is extrapolated; other shapes scale by useful work.

``operator_work`` is the declared useful F+B FLOPs per operator, identical to
the reference's definition so scores stay comparable.
"""

from __future__ import annotations

import math

H100_SCHEMA = "h100_operator_anchors_v1"
B200_SCHEMA = "b200_operator_anchors_v1"
RESIDUAL_SCHEMA = "joint_cp_response_v1"
ANCHOR_SCHEMAS = (H100_SCHEMA, B200_SCHEMA)
REFERENCE_SHAPE = (4096, 32, 8, 128, 16, 128, 8)


def operator_work(model, symbol: str, tokens: int, squares: int) -> float:
    """Declared useful forward+backward FLOPs of one operator over a token set."""
    h, d = model.hidden, model.gdn_heads * model.gdn_dim
    if symbol == "*":
        proj = h * (model.q_heads + 2 * model.kv_heads) * model.head_dim + h * h
        return 6 * proj * tokens + 6 * model.q_heads * model.head_dim * squares
    if symbol == "G":
        return 6 * (6 * h * d + 4 * model.gdn_heads * model.gdn_dim ** 2) * tokens
    if symbol == "M":
        return 18 * h * model.ffn * tokens
    raise ValueError("Unknown operator")


def _shape(model):
    return (model.hidden, model.q_heads, model.kv_heads, model.head_dim, model.gdn_heads, model.gdn_dim,
            model.ranks_per_node)


def _check_anchor_times(anchors, domain):
    for anchor in anchors.values():
        if set(anchor["milliseconds"]) != domain:
            raise ValueError("GQA/GDN measured CP domains must match")
        for t in anchor["milliseconds"].values():
            if not math.isfinite(t) or t <= 0:
                raise ValueError("Anchor times must be finite and positive")


def validate_anchor_response(profile: dict, model) -> None:
    schema = profile.get("schema")
    anchors = profile.get("anchors", {})
    if set(anchors) != {"GQA", "GDN"}:
        raise ValueError("Anchor profiles require separate GQA and GDN anchors")
    domain = set(anchors["GQA"]["milliseconds"])
    if schema == H100_SCHEMA:
        if _shape(model) != REFERENCE_SHAPE:
            raise ValueError("H100 anchors require H4096/Q32/KV8/D128/GDN16x128 and 8 GPUs per node")
        if profile.get("hardware") != "H100" or profile.get("anchor_tokens") != 262144:
            raise ValueError("Unknown H100 anchor hardware or length")
        if (profile.get("shape_policy") != "useful_work_scaling_unvalidated"
                or profile.get("unmeasured_cp_policy") != "constant_cp8_per_gpu_efficiency"):
            raise ValueError("H100 extrapolation must have an explicit supported policy")
        if domain not in ({"8", "16"}, {"8", "16", "32"}):
            raise ValueError("H100 measured CP domain must be 8/16 or 8/16/32")
        if "32" in domain and not profile.get("cp32_source"):
            raise ValueError("H100 CP32 requires its independent measured source")
    else:
        shape = profile.get("model_shape")
        if shape is not None and tuple(shape) != _shape(model)[:6]:
            raise ValueError("B200 anchors were measured for a different model shape")
        if profile.get("hardware") != "B200" or int(profile.get("anchor_tokens", 0)) <= 0:
            raise ValueError("Unknown B200 anchor hardware or length")
        if not domain or any(int(c) & (int(c) - 1) for c in domain):
            raise ValueError("B200 measured CP domain must be powers of two")
        if max(int(c) for c in domain) > model.ranks_per_node:
            raise ValueError("B200 anchors cover one NVSwitch box only")
    _check_anchor_times(anchors, domain)


def validate_response(profile: dict, model) -> None:
    schema = profile.get("schema")
    if schema in ANCHOR_SCHEMAS:
        validate_anchor_response(profile, model)
        return
    if schema != RESIDUAL_SCHEMA:
        raise ValueError("Unknown CP response schema")
    if profile.get("cp16_policy") not in ("carry8", "paired_linear", "paired_quadratic"):
        raise ValueError("Unknown CP16 response policy")
    if profile.get("cp32_policy") not in (None, "work_scaling", "carry_residual", "double_residual"):
        raise ValueError("Unknown CP32 hypothesis")
    mult = profile.get("gdn32_multiplier", 1.0)
    if not math.isfinite(mult) or mult < 1:
        raise ValueError("CP32 GDN stress multiplier must be finite and >=1")
    if profile.get("cp32_policy") and profile["cp16_policy"] == "carry8":
        raise ValueError("CP32 hypotheses require a paired CP16 GQA response")
    if _shape(model) != REFERENCE_SHAPE:
        raise ValueError("CP profiling transfer requires H4096/Q32/KV8/D128/GDN16x128 and 8 GPUs per node")
    fits = profile.get("fits", {})
    if not fits or set(fits) - {"GQA", "GDN"}:
        raise ValueError("No profiling evidence for requested operator")
    for fit in fits.values():
        for cp in ("2", "4", "8"):
            p = fit["parameters"][cp]
            for key in ("quadratic_fraction", "token_fraction", "fixed_ms"):
                if not math.isfinite(p[key]) or p[key] < 0:
                    raise ValueError("Invalid profiling response coefficient")
    if profile["cp16_policy"] != "carry8":
        pairs = profile.get("paired_anchors", [])
        if "GQA" not in fits or len(pairs) != 2 or sorted(p["length"] for p in pairs) != [65536, 262144]:
            raise ValueError("Paired CP16 transfer requires the two GQA anchors")
        if any(not math.isfinite(p["ratio"]) or p["ratio"] <= 0 for p in pairs):
            raise ValueError("Invalid paired CP ratio")


def residual_profile(fits: dict, paired_anchors: list, *, name: str, cp16: str = "paired_linear",
                     cp32: str | None = None, gdn32_multiplier: float = 1.0, include_gdn: bool = True,
                     scope: str = "", gdn_transfer: str = "", packing_extrapolation: str = "") -> dict:
    """Assemble a ``joint_cp_response_v1`` profile from fit data (cf. load_response)."""
    if cp16 not in ("carry8", "paired_linear", "paired_quadratic"):
        raise ValueError("Unknown CP16 response policy")
    if cp32 not in (None, "work_scaling", "carry_residual", "double_residual"):
        raise ValueError("Unknown CP32 hypothesis")
    chosen = dict(fits) if include_gdn else {"GQA": fits["GQA"]}
    suffix = "" if include_gdn else "_gqa_only"
    if cp32:
        suffix += f"_cp32_{cp32}_gdn{gdn32_multiplier:g}"
    return {"schema": RESIDUAL_SCHEMA, "name": name + suffix, "fits": chosen, "cp16_policy": cp16,
            "paired_anchors": list(paired_anchors), "cp32_policy": cp32, "gdn32_multiplier": gdn32_multiplier,
            "scope": scope, "gdn_transfer": gdn_transfer if include_gdn else "not transferred",
            "packing_extrapolation": packing_extrapolation}


class Response:
    """Prices one operator group call given its analytic components (milliseconds)."""

    def __init__(self, model):
        self.model = model
        self.profile = model.cp_response
        self.anchor_fit = None
        if self.profile is None or self.profile.get("schema") in ANCHOR_SCHEMAS:
            return
        if self.profile["cp16_policy"] != "carry8":
            self.anchor_fit = self._paired_fit()

    def _paired_fit(self):
        m = self.model
        p8 = self.profile["fits"]["GQA"]["parameters"]["8"]
        rate = m.compute_tflops * 1e9
        a = 6 * (m.hidden * (m.q_heads + 2 * m.kv_heads) * m.head_dim + m.hidden * m.hidden) / rate
        b = 6 * m.q_heads * m.head_dim / rate
        power = 1 if self.profile["cp16_policy"] == "paired_linear" else 2
        points = []
        for pair in sorted(self.profile["paired_anchors"], key=lambda r: r["length"]):
            n = pair["length"]
            t8 = ((1 + p8["token_fraction"]) * a * n + (1 + p8["quadratic_fraction"]) * b * n * n) / 8 + p8["fixed_ms"]
            target, ideal = t8 * pair["ratio"], (a * n + b * n * n) / 16
            points.append({"length": n, "coordinate": n ** power / 16, "reference_cp8_ms": t8,
                           "target_ms": target, "ideal_ms": ideal, "residual_ms": target - ideal,
                           "observed_ratio": pair["ratio"]})
        lo, hi = points
        slope = (hi["residual_ms"] - lo["residual_ms"]) / (hi["coordinate"] - lo["coordinate"])
        intercept = lo["residual_ms"] - slope * lo["coordinate"]
        if min(slope, intercept) < 0:
            raise ValueError("Paired response transfer produced a negative residual")
        return {"power": power, "slope": slope, "fixed_ms": intercept, "anchors": points}

    def _anchor_cost(self, symbol, cp, tokens, squares, cross_node, fallback):
        kind = {"G": "GDN", "*": "GQA"}.get(symbol)
        if kind is None:
            return fallback
        anchor = self.profile["anchors"][kind]["milliseconds"]
        n = self.profile["anchor_tokens"]
        if self.profile["schema"] == H100_SCHEMA:
            if cp not in (1, 2, 4) and str(cp) not in anchor:
                raise ValueError(f"H100 CP>{max(map(int, anchor))} requires new evidence or an explicit new hypothesis")
            if cp <= 8 and cross_node:
                raise ValueError("H100 CP<=8 anchor/extrapolation requires node-local groups")
            ms = anchor[str(cp)] if str(cp) in anchor else anchor["8"] * 8 / cp
        else:
            if str(cp) not in anchor:
                raise ValueError(f"B200 profile has no measured CP{cp} anchor")
            ms = anchor[str(cp)]
        # anchors include the module's own CP communication: scale by useful work only
        return ms * operator_work(self.model, symbol, tokens, squares) / operator_work(self.model, symbol, n, n * n)

    def cost(self, symbol, cp, linear_ms, quadratic_ms, communication_ms, local_communication_ms, tokens, squares,
             cross_node=None):
        ideal = linear_ms + quadratic_ms
        if self.profile is not None and self.profile.get("schema") in ANCHOR_SCHEMAS:
            return self._anchor_cost(symbol, cp, tokens, squares, cross_node, ideal + communication_ms)
        kind = {"G": "GDN", "*": "GQA"}.get(symbol)
        if self.profile is None or cp == 1 or kind not in self.profile["fits"]:
            return ideal + communication_ms
        if cp == 32:
            policy = self.profile.get("cp32_policy")
            if policy is None:
                raise ValueError("CP32 requires an explicit unmeasured response hypothesis")
            if kind == "GQA":
                f = self.anchor_fit
                variable = f["slope"] * (tokens if f["power"] == 1 else squares) / 16
                residual = {"work_scaling": variable / 2 + f["fixed_ms"],
                            "carry_residual": variable + f["fixed_ms"]}.get(policy, 2 * (variable + f["fixed_ms"]))
                return ideal + residual
        elif cp not in (2, 4, 8, 16):
            raise ValueError("CP response transfer supports CP<=32 only")
        if cp == 16 and kind == "GQA" and self.anchor_fit is not None:
            f = self.anchor_fit
            return ideal + f["slope"] * (tokens if f["power"] == 1 else squares) / 16 + f["fixed_ms"]
        p = self.profile["fits"][kind]["parameters"][str(min(cp, 8))]
        residual = p["token_fraction"] * linear_ms + p["quadratic_fraction"] * quadratic_ms + p["fixed_ms"]
        value = ideal + residual + max(0.0, communication_ms - local_communication_ms)
        return value * self.profile.get("gdn32_multiplier", 1.0) if cp == 32 else value


def response_coverage(plan, lengths, model) -> dict:
    """How many group calls fall inside the measured domain (calls, not samples)."""
    prof = model.cp_response
    if prof is None:
        return {"policy": "analytic_unvalidated"}
    if prof.get("schema") in ANCHOR_SCHEMAS:
        domain = tuple(int(c) for c in prof["anchors"]["GQA"]["milliseconds"])
        counts = {"anchor_domain_group_calls": 0, "shape_extrapolated_group_calls": 0,
                  "cp_extrapolated_group_calls": 0, "packed_group_calls": 0,
                  "cp16_gqa_calls": 0, "cp16_gdn_calls": 0}
        if 32 in domain:
            counts.update(cp32_gqa_calls=0, cp32_gdn_calls=0)
        n = prof["anchor_tokens"]
        for mb in plan.microbatches:
            for symbol, (layout, _) in zip(plan.pattern, mb.layers):
                for g in layout.groups:
                    cp = len(g.ranks)
                    at_shape = len(g.samples) == 1 and lengths[g.samples[0]] == n
                    counts["anchor_domain_group_calls"] += int(at_shape and cp in domain)
                    counts["shape_extrapolated_group_calls"] += int(not at_shape)
                    counts["cp_extrapolated_group_calls"] += int(cp not in domain)
                    counts["packed_group_calls"] += int(len(g.samples) > 1)
                    counts["cp16_gdn_calls" if symbol == "G" else "cp16_gqa_calls"] += int(cp == 16)
                    if cp == 32:
                        counts["cp32_gdn_calls" if symbol == "G" else "cp32_gqa_calls"] += 1
        return {"policy": prof["name"], "hardware": prof["hardware"], "counts": counts,
                "source": prof.get("source"), "anchors": prof["anchors"], "cp32_source": prof.get("cp32_source"),
                "shape_policy": prof.get("shape_policy"), "unmeasured_cp_policy": prof.get("unmeasured_cp_policy"),
                "other_terms": "MLP, head, routing, update and memory are analytic estimates",
                "gpu_measured": prof["schema"] == B200_SCHEMA}
    counts = {"calibrated_group_calls": 0, "packed_group_calls": 0, "outside_length_domain_calls": 0,
              "cp16_gqa_calls": 0, "cp16_gdn_calls": 0, "cp32_gqa_calls": 0, "cp32_gdn_calls": 0,
              "uncalibrated_gdn_calls": 0}
    for mb in plan.microbatches:
        for symbol, (layout, _) in zip(plan.pattern, mb.layers):
            kind = "GDN" if symbol == "G" else "GQA"
            for g in layout.groups:
                cp = len(g.ranks)
                if cp == 1:
                    continue
                if kind not in prof["fits"]:
                    counts["uncalibrated_gdn_calls"] += 1
                    continue
                counts["calibrated_group_calls"] += 1
                counts["packed_group_calls"] += int(len(g.samples) > 1)
                lo, hi = prof["fits"][kind]["sequence_domain_ki"]
                if cp == 16:
                    counts["cp16_gdn_calls" if kind == "GDN" else "cp16_gqa_calls"] += 1
                    if kind == "GQA" and prof["cp16_policy"] != "carry8":
                        lo, hi = 64, 256
                elif cp == 32:
                    counts["cp32_gdn_calls" if kind == "GDN" else "cp32_gqa_calls"] += 1
                    if kind == "GQA":
                        lo, hi = 64, 256
                counts["outside_length_domain_calls"] += int(any(not lo * 1024 <= lengths[s] <= hi * 1024
                                                                 for s in g.samples))
    return {"policy": prof["name"], "counts": counts, "gdn_head_transfer": prof.get("gdn_transfer"),
            "anchor_fit": Response(model).anchor_fit, "cp32_policy": prof.get("cp32_policy"),
            "cp32_scope": prof.get("cp32_scope"), "gpu_measured": False}
