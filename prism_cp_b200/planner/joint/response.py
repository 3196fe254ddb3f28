"""Hardware CP response: measured module timings turned into per-operator cost.

``Model.cp_response`` is a JSON-serialisable profile in one of three schemas.
Each schema is one profile class here; ``profile_of(model)`` returns the right
one and the evaluator only ever calls ``price`` on it:

* no profile (``Analytic``) - the analytic time: useful FLOPs at the declared
  throughput plus CP communication at the declared link bandwidth;
* ``joint_cp_response_v1`` (``Residual``) - per CP 2/4/8 residual fits on top of
  the analytic time (a fraction of the token-linear time, a fraction of the
  quadratic time, a fixed cost), CP16 GQA from two paired anchors (a residual
  linear in tokens or in squared tokens) and explicit CP32 hypotheses
  (reference schema: joint_cp/response.py:57-122,153-199);
* ``h100_operator_anchors_v1`` / ``b200_operator_anchors_v1`` (``Anchors``) -
  full-module F+B times at one anchor length for a set of CP degrees; other
  shapes scale by declared useful work. The H100 profile extrapolates CP 1/2/4
  as ``T8 * 8 / p`` (reference: joint_cp/response.py:32-54,157-170); the B200
  profile (written by ``prism_cp_b200.planner.profile_builder`` from this
  framework's module bench) must measure every CP it is asked for.

``operator_work`` is the declared useful F+B FLOPs per operator; its formula is
the reference's, so predicted scores stay comparable between the two tools.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

H100_SCHEMA = "h100_operator_anchors_v1"
B200_SCHEMA = "b200_operator_anchors_v1"
RESIDUAL_SCHEMA = "joint_cp_response_v1"
ANCHOR_SCHEMAS = (H100_SCHEMA, B200_SCHEMA)
# hidden, q heads, kv heads, head dim, GDN heads, GDN head dim, ranks per node of the
# model the reference's H800/H100 profiles were measured on
REFERENCE_SHAPE = (4096, 32, 8, 128, 16, 128, 8)
KIND = {"G": "GDN", "*": "GQA"}
CP16_POLICIES = ("carry8", "paired_linear", "paired_quadratic")
CP32_POLICIES = (None, "work_scaling", "carry_residual", "double_residual")


def operator_work(model, symbol: str, tokens: int, squares: int) -> float:
    """Declared useful forward+backward FLOPs of one operator over a token set."""
    h = model.hidden
    if symbol == "M":
        return 18 * h * model.ffn * tokens
    if symbol == "G":
        d = model.gdn_heads * model.gdn_dim
        return 6 * (6 * h * d + 4 * model.gdn_heads * model.gdn_dim ** 2) * tokens
    if symbol == "*":
        projection = h * (model.q_heads + 2 * model.kv_heads) * model.head_dim + h * h
        return 6 * projection * tokens + 6 * model.q_heads * model.head_dim * squares
    raise ValueError("Unknown operator")


def model_shape(model) -> tuple:
    return (model.hidden, model.q_heads, model.kv_heads, model.head_dim, model.gdn_heads, model.gdn_dim,
            model.ranks_per_node)


@dataclass(frozen=True)
class Parts:
    """Analytic pieces of one group call (milliseconds)."""

    linear: float          # token-linear compute
    quadratic: float       # causal-attention compute
    comm: float            # CP communication on the group's own links
    comm_local: float      # the same traffic priced at intra-node bandwidth

    @property
    def ideal(self) -> float:
        return self.linear + self.quadratic


class Analytic:
    name = "analytic_unvalidated"

    def validate(self) -> None:
        pass

    def prepare(self) -> "Analytic":
        return self

    def price(self, symbol, cp, parts: Parts, tokens, squares, cross_node) -> float:
        return parts.ideal + parts.comm

    def allows_attention_cp(self, cp: int) -> bool:
        return True

    def coverage(self, plan, lengths) -> dict:
        return {"policy": self.name}


def _finite_nonnegative(x) -> bool:
    return math.isfinite(x) and x >= 0


class Residual:
    """``joint_cp_response_v1``: residual fits over the analytic time per CP degree."""

    def __init__(self, profile: dict, model):
        self.profile, self.model = profile, model
        self.name = profile.get("name")
        self.fits = profile.get("fits", {})
        self.cp16 = profile.get("cp16_policy")
        self.cp32 = profile.get("cp32_policy")
        self.gdn32 = profile.get("gdn32_multiplier", 1.0)
        self.anchor_fit = None

    # ---------------------------------------------------------------- validation
    def validate(self) -> None:
        if self.cp16 not in CP16_POLICIES:
            raise ValueError("Unknown CP16 response policy")
        if self.cp32 not in CP32_POLICIES:
            raise ValueError("Unknown CP32 hypothesis")
        if not (math.isfinite(self.gdn32) and self.gdn32 >= 1):
            raise ValueError("CP32 GDN stress multiplier must be finite and >=1")
        if self.cp32 and self.cp16 == "carry8":
            raise ValueError("CP32 hypotheses require a paired CP16 GQA response")
        if model_shape(self.model) != REFERENCE_SHAPE:
            raise ValueError("CP profiling transfer requires H4096/Q32/KV8/D128/GDN16x128 and 8 GPUs per node")
        if not self.fits or not set(self.fits) <= {"GQA", "GDN"}:
            raise ValueError("No profiling evidence for requested operator")
        coefficients = [p[k] for fit in self.fits.values() for cp in ("2", "4", "8")
                        for p in (fit["parameters"][cp],) for k in ("quadratic_fraction", "token_fraction", "fixed_ms")]
        if not all(_finite_nonnegative(c) for c in coefficients):
            raise ValueError("Invalid profiling response coefficient")
        if self.cp16 == "carry8":
            return
        pairs = self.profile.get("paired_anchors", [])
        if "GQA" not in self.fits or len(pairs) != 2 or sorted(p["length"] for p in pairs) != [65536, 262144]:
            raise ValueError("Paired CP16 transfer requires the two GQA anchors")
        if not all(math.isfinite(p["ratio"]) and p["ratio"] > 0 for p in pairs):
            raise ValueError("Invalid paired CP ratio")

    def prepare(self) -> "Residual":
        if self.cp16 != "carry8":
            self.anchor_fit = self._paired_fit()
        return self

    def _paired_fit(self) -> dict:
        """Line through the residuals of the two paired CP16/CP8 GQA anchors, in tokens
        (``paired_linear``) or squared tokens (``paired_quadratic``) per CP16 rank."""
        m = self.model
        rate = m.compute_tflops * 1e9
        a = 6 * (m.hidden * (m.q_heads + 2 * m.kv_heads) * m.head_dim + m.hidden * m.hidden) / rate
        b = 6 * m.q_heads * m.head_dim / rate
        p8 = self.fits["GQA"]["parameters"]["8"]
        power = 1 if self.cp16 == "paired_linear" else 2

        def anchor(pair):
            n = pair["length"]
            t8 = ((1 + p8["token_fraction"]) * a * n + (1 + p8["quadratic_fraction"]) * b * n * n) / 8 \
                + p8["fixed_ms"]
            target, ideal = t8 * pair["ratio"], (a * n + b * n * n) / 16
            return {"length": n, "coordinate": n ** power / 16, "reference_cp8_ms": t8, "target_ms": target,
                    "ideal_ms": ideal, "residual_ms": target - ideal, "observed_ratio": pair["ratio"]}

        short, long_ = (anchor(p) for p in sorted(self.profile["paired_anchors"], key=lambda r: r["length"]))
        slope = (long_["residual_ms"] - short["residual_ms"]) / (long_["coordinate"] - short["coordinate"])
        intercept = short["residual_ms"] - slope * short["coordinate"]
        if slope < 0 or intercept < 0:
            raise ValueError("Paired response transfer produced a negative residual")
        return {"power": power, "slope": slope, "fixed_ms": intercept, "anchors": [short, long_]}

    # ---------------------------------------------------------------- pricing
    def _paired_variable(self, tokens, squares) -> float:
        f = self.anchor_fit
        return f["slope"] * (tokens if f["power"] == 1 else squares) / 16

    def price(self, symbol, cp, parts: Parts, tokens, squares, cross_node) -> float:
        kind = KIND.get(symbol)
        ideal = parts.ideal
        if cp == 1 or kind not in self.fits:
            return ideal + parts.comm
        if cp not in (2, 4, 8, 16, 32):
            raise ValueError("CP response transfer supports CP<=32 only")
        if cp == 32 and self.cp32 is None:
            raise ValueError("CP32 requires an explicit unmeasured response hypothesis")
        if kind == "GQA" and cp == 32:
            variable, fixed = self._paired_variable(tokens, squares), self.anchor_fit["fixed_ms"]
            if self.cp32 == "work_scaling":
                return ideal + (variable / 2 + fixed)
            if self.cp32 == "carry_residual":
                return ideal + (variable + fixed)
            return ideal + 2 * (variable + fixed)
        if kind == "GQA" and cp == 16 and self.anchor_fit is not None:
            return ideal + self._paired_variable(tokens, squares) + self.anchor_fit["fixed_ms"]
        p = self.fits[kind]["parameters"][str(min(cp, 8))]
        residual = p["token_fraction"] * parts.linear + p["quadratic_fraction"] * parts.quadratic + p["fixed_ms"]
        value = ideal + residual + max(0.0, parts.comm - parts.comm_local)
        return value * self.gdn32 if cp == 32 else value

    def allows_attention_cp(self, cp: int) -> bool:
        return True

    # ---------------------------------------------------------------- evidence
    def coverage(self, plan, lengths) -> dict:
        names = ("calibrated_group_calls", "packed_group_calls", "outside_length_domain_calls", "cp16_gqa_calls",
                 "cp16_gdn_calls", "cp32_gqa_calls", "cp32_gdn_calls", "uncalibrated_gdn_calls")
        counts = dict.fromkeys(names, 0)
        for symbol, layout in _attention_calls(plan):
            kind = KIND[symbol]
            for g in layout.groups:
                cp = len(g.ranks)
                if cp == 1:
                    continue
                if kind not in self.fits:
                    counts["uncalibrated_gdn_calls"] += 1
                    continue
                counts["calibrated_group_calls"] += 1
                counts["packed_group_calls"] += len(g.samples) > 1
                window = tuple(self.fits[kind]["sequence_domain_ki"])
                if cp in (16, 32):
                    counts[f"cp{cp}_{kind.lower()}_calls"] += 1
                    paired = kind == "GQA" and (cp == 32 or self.cp16 != "carry8")
                    window = (64, 256) if paired else window
                lo, hi = window
                counts["outside_length_domain_calls"] += any(
                    not lo * 1024 <= lengths[s] <= hi * 1024 for s in g.samples)
        return {"policy": self.name, "counts": counts, "gdn_head_transfer": self.profile.get("gdn_transfer"),
                "anchor_fit": self.anchor_fit, "cp32_policy": self.cp32,
                "cp32_scope": self.profile.get("cp32_scope"), "gpu_measured": False}


def _attention_calls(plan):
    """(symbol, attention layout) of every layer of every microbatch, in plan order."""
    for mb in plan.microbatches:
        for symbol, (layout, _) in zip(plan.pattern, mb.layers):
            yield symbol, layout


class Anchors:
    """Full-module anchor profiles (H100 from the reference's measurements, B200 from this
    framework's module bench): time at one anchor length per measured CP degree."""

    def __init__(self, profile: dict, model):
        self.profile, self.model = profile, model
        self.schema = profile.get("schema")
        self.name = profile.get("name")
        self.anchors = profile.get("anchors", {})
        self.tokens = profile.get("anchor_tokens")

    @property
    def domain(self) -> set:
        return set(self.anchors["GQA"]["milliseconds"])

    def validate(self) -> None:
        if set(self.anchors) != {"GQA", "GDN"}:
            raise ValueError("Anchor profiles require separate GQA and GDN anchors")
        domain, p = self.domain, self.profile
        if self.schema == H100_SCHEMA:
            checks = (
                (model_shape(self.model) == REFERENCE_SHAPE,
                 "H100 anchors require H4096/Q32/KV8/D128/GDN16x128 and 8 GPUs per node"),
                (p.get("hardware") == "H100" and self.tokens == 262144, "Unknown H100 anchor hardware or length"),
                (p.get("shape_policy") == "useful_work_scaling_unvalidated"
                 and p.get("unmeasured_cp_policy") == "constant_cp8_per_gpu_efficiency",
                 "H100 extrapolation must have an explicit supported policy"),
                (domain in ({"8", "16"}, {"8", "16", "32"}), "H100 measured CP domain must be 8/16 or 8/16/32"),
                ("32" not in domain or bool(p.get("cp32_source")), "H100 CP32 requires its independent measured source"),
            )
        else:
            shape = p.get("model_shape")
            degrees = [int(c) for c in domain]
            checks = (
                (shape is None or tuple(shape) == model_shape(self.model)[:6],
                 "B200 anchors were measured for a different model shape"),
                (p.get("hardware") == "B200" and int(self.tokens or 0) > 0, "Unknown B200 anchor hardware or length"),
                (bool(degrees) and all(c & (c - 1) == 0 for c in degrees),
                 "B200 measured CP domain must be powers of two"),
                (not degrees or max(degrees) <= self.model.ranks_per_node, "B200 anchors cover one NVSwitch box only"),
            )
        for ok, message in checks:
            if not ok:
                raise ValueError(message)
        for anchor in self.anchors.values():
            times = anchor["milliseconds"]
            if set(times) != domain:
                raise ValueError("GQA/GDN measured CP domains must match")
            if not all(math.isfinite(t) and t > 0 for t in times.values()):
                raise ValueError("Anchor times must be finite and positive")

    def prepare(self) -> "Anchors":
        return self

    def _anchor_ms(self, kind, cp, cross_node) -> float:
        times = self.anchors[kind]["milliseconds"]
        if self.schema != H100_SCHEMA:
            if str(cp) not in times:
                raise ValueError(f"B200 profile has no measured CP{cp} anchor")
            return times[str(cp)]
        if str(cp) not in times and cp not in (1, 2, 4):
            raise ValueError(f"H100 CP>{max(map(int, times))} requires new evidence or an explicit new hypothesis")
        if cross_node and cp <= 8:
            raise ValueError("H100 CP<=8 anchor/extrapolation requires node-local groups")
        # unmeasured CP 1/2/4 keep the measured CP8 per-GPU efficiency
        return times[str(cp)] if str(cp) in times else times["8"] * 8 / cp

    def price(self, symbol, cp, parts: Parts, tokens, squares, cross_node) -> float:
        kind = KIND.get(symbol)
        if kind is None:
            return parts.ideal + parts.comm
        # the anchors include the module's own CP communication: scale by useful work only
        at_anchor = operator_work(self.model, symbol, self.tokens, self.tokens * self.tokens)
        return self._anchor_ms(kind, cp, cross_node) * operator_work(self.model, symbol, tokens, squares) / at_anchor

    def allows_attention_cp(self, cp: int) -> bool:
        """Attention CP stays within the profile's largest measured degree (the reference's rule
        for its H100 profile); the B200 profile also needs that exact degree measured."""
        measured = self.anchors["GQA"]["milliseconds"]
        if cp > max(map(int, measured)):
            return False
        return self.schema == H100_SCHEMA or str(cp) in measured

    def coverage(self, plan, lengths) -> dict:
        domain = tuple(int(c) for c in self.anchors["GQA"]["milliseconds"])
        names = ["anchor_domain_group_calls", "shape_extrapolated_group_calls", "cp_extrapolated_group_calls",
                 "packed_group_calls", "cp16_gqa_calls", "cp16_gdn_calls"]
        if 32 in domain:
            names += ["cp32_gqa_calls", "cp32_gdn_calls"]
        counts = dict.fromkeys(names, 0)
        for symbol, layout in _attention_calls(plan):
            for g in layout.groups:
                cp = len(g.ranks)
                at_shape = len(g.samples) == 1 and lengths[g.samples[0]] == self.tokens
                counts["anchor_domain_group_calls"] += at_shape and cp in domain
                counts["shape_extrapolated_group_calls"] += not at_shape
                counts["cp_extrapolated_group_calls"] += cp not in domain
                counts["packed_group_calls"] += len(g.samples) > 1
                if cp in (16, 32):
                    counts[f"cp{cp}_{KIND[symbol].lower()}_calls"] += 1
        p = self.profile
        return {"policy": self.name, "hardware": p["hardware"], "counts": counts, "source": p.get("source"),
                "anchors": self.anchors, "cp32_source": p.get("cp32_source"), "shape_policy": p.get("shape_policy"),
                "unmeasured_cp_policy": p.get("unmeasured_cp_policy"),
                "other_terms": "MLP, head, routing, update and memory are analytic estimates",
                "gpu_measured": self.schema == B200_SCHEMA}


def _profile(profile: dict | None, model):
    if profile is None:
        return Analytic()
    schema = profile.get("schema")
    if schema in ANCHOR_SCHEMAS:
        return Anchors(profile, model)
    if schema == RESIDUAL_SCHEMA:
        return Residual(profile, model)
    raise ValueError("Unknown CP response schema")


def validate_response(profile: dict, model) -> None:
    """Raise ValueError unless ``profile`` is a supported CP response for ``model``."""
    _profile(profile, model).validate()


def profile_of(model):
    """The pricing object of ``model.cp_response`` (validated when the model was built)."""
    return _profile(model.cp_response, model).prepare()


def response_coverage(plan, lengths, model) -> dict:
    """How many group calls fall inside the profile's measured domain (calls, not samples)."""
    return profile_of(model).coverage(plan, lengths)


def residual_profile(fits: dict, paired_anchors: list, *, name: str, cp16: str = "paired_linear",
                     cp32: str | None = None, gdn32_multiplier: float = 1.0, include_gdn: bool = True,
                     scope: str = "", gdn_transfer: str = "", packing_extrapolation: str = "") -> dict:
    """Assemble a ``joint_cp_response_v1`` profile from residual fits and paired GQA anchors."""
    if cp16 not in CP16_POLICIES:
        raise ValueError("Unknown CP16 response policy")
    if cp32 not in CP32_POLICIES:
        raise ValueError("Unknown CP32 hypothesis")
    suffix = ("" if include_gdn else "_gqa_only") + (f"_cp32_{cp32}_gdn{gdn32_multiplier:g}" if cp32 else "")
    return {"schema": RESIDUAL_SCHEMA, "name": name + suffix,
            "fits": dict(fits) if include_gdn else {"GQA": fits["GQA"]}, "cp16_policy": cp16,
            "paired_anchors": list(paired_anchors), "cp32_policy": cp32, "gdn32_multiplier": gdn32_multiplier,
            "scope": scope, "gdn_transfer": gdn_transfer if include_gdn else "not transferred",
            "packing_extrapolation": packing_extrapolation}
