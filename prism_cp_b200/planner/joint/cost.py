"""Cost and whole forward/backward memory model of a joint plan.

``Model`` holds the model shape, the device bytes and reservations, throughput
and link assumptions and an optional hardware CP-response profile (the field
set is the planner's config format, shared with the reference's
joint_cp/model.py so its configs load unchanged). ``Evaluator`` prices one
microbatch:

* every operator call of a layout is described by a ``Sheet`` (useful FLOPs,
  the causal-attention part of them, CP bytes on the wire, bytes saved for the
  backward and transient workspace per rank) from a per-operator formula, then
  priced by the response profile (``response.profile_of``);
* a layout change is priced by its route: the busiest rank's injected or
  received bytes per link class, the local pack/unpack copy, a latency, all
  twice (the backward runs the inverse route);
* memory is a per-rank walk: the residual stream and every layer's saved
  activations accumulate, and at each step of a layer (route in, operator,
  route to the MLP, MLP, route back) the step's workspace sits on top.

Times are milliseconds of forward + backward. The formulas and constants are
the reference's (joint_cp/model.py:56-228), evaluated in the same arithmetic
order, so identical plans get identical predicted times in both tools.
``byte_scale``, ``operator_calibration`` and ``cp_overhead`` fit the model to
this framework's measured B200 kernels (``planner/calibrate.py``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, fields
from functools import lru_cache
from typing import NamedTuple

from .ir import identity_route, route
from .response import Parts, operator_work, profile_of, validate_response

GIB = 1024 ** 3
_POSITIVE = ("hidden", "ffn", "vocab", "q_heads", "kv_heads", "head_dim", "gdn_heads", "gdn_dim", "device_bytes",
             "compute_tflops", "intra_gbps", "inter_gbps", "memory_gbps", "ranks_per_node", "byte_scale")


@dataclass(frozen=True)
class Model:
    hidden: int = 4096
    ffn: int = 16384
    vocab: int = 32768
    q_heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    gdn_heads: int = 16
    gdn_dim: int = 128
    device_bytes: int = 80 * GIB
    external_bytes: int = 2 * GIB
    margin_bytes: int = 2 * GIB
    static_bytes: int | None = None
    compute_tflops: float = 300.0
    intra_gbps: float = 300.0
    inter_gbps: float = 25.0
    memory_gbps: float = 1500.0
    ranks_per_node: int = 8
    latency_ms: float = 0.01
    microbatch_ms: float = 0.1
    update_ms: float = 1.0
    provenance: str = "analytic_unvalidated; throughput, link and storage envelopes are assumptions"
    cp_response: dict | None = None
    byte_scale: float = 1.0
    # measured single-GPU efficiency per operator ("G", "*", "M"): {"linear": fraction of
    # compute_tflops reached by the token-linear work, "quadratic": the same for causal attention,
    # "fixed_ms": per-call overhead}; None keeps the analytic envelope
    operator_calibration: dict | None = None
    # measured step-time factor of CP > 1 operators over the analytic CP terms, keyed by CP degree
    # ("2": 1.07); degrees without an entry use the largest measured degree's factor
    cp_overhead: dict | None = None
    # microbatches with more tokens than this on some rank (in any of their layouts) keep only
    # every layer's input and recompute the layer's forward in the backward; None: never
    recompute_tokens: int | None = None

    def __post_init__(self):
        numbers = {f.name: getattr(self, f.name) for f in fields(self)}
        for key, value in numbers.items():
            if isinstance(value, bool) or not isinstance(value, (int, float)):
                continue
            if not math.isfinite(value) or value < 0:
                raise ValueError(f"Invalid model field {key}")
        zero = next((k for k in _POSITIVE if numbers[k] <= 0), None)
        if zero is not None:
            raise ValueError(f"Model field must be positive: {zero}")
        if self.cp_response is not None:
            validate_response(self.cp_response, self)
        for symbol, cal in (self.operator_calibration or {}).items():
            sane = cal.get("linear", 0) > 0 and cal.get("quadratic", 1) > 0 and cal.get("fixed_ms", 0) >= 0
            if symbol not in ("G", "*", "M") or not sane:
                raise ValueError(f"invalid operator calibration for {symbol!r}: {cal}")

    @property
    def gdn_width(self) -> int:
        return self.gdn_heads * self.gdn_dim

    @property
    def budget(self) -> int:
        """Admission budget of one device: 90 % of it, and at least 8 GiB left free."""
        return min(int(0.9 * self.device_bytes), self.device_bytes - 8 * GIB)

    def params(self, pattern: str) -> int:
        h, d = self.hidden, self.gdn_width
        per_symbol = {"*": h * (self.q_heads + 2 * self.kv_heads) * self.head_dim + h * h,
                      "G": h * 5 * d + d * h + 4 * 3 * d + 2 * self.gdn_heads}
        mixers = sum(per_symbol[s] * pattern.count(s) for s in ("*", "G"))
        return 2 * self.vocab * h + len(pattern) * (3 * h * self.ffn + 4 * h) + mixers + h

    def static(self, pattern: str, world: int) -> int:
        """bf16 weights, fp32 gradients, fp32 master/m/v sharded over the world, a buffer reserve."""
        if self.static_bytes is not None:
            return self.static_bytes
        return math.ceil(self.params(pattern) * (6 + 12 / world)) + 256 * 1024 ** 2

    def saved_per_token(self, pattern: str) -> float:
        h, d = self.hidden, self.gdn_width
        qkv = (self.q_heads + 2 * self.kv_heads) * self.head_dim
        per_layer = {"G": 2 * (8 * h + 5 * d), "*": 2 * (8 * h + qkv) + 4 * self.q_heads}
        mixers = per_layer["G"] * pattern.count("G") + per_layer["*"] * pattern.count("*")
        return self.byte_scale * (4 * h + mixers + len(pattern) * 2 * (4 * h + 3 * self.ffn))

    def token_capacity_upper_bound(self, pattern: str, world: int) -> int:
        """Necessary (not sufficient) token ceiling: average live storage at the output head."""
        room = self.budget - self.static(pattern, world) - self.external_bytes - self.margin_bytes
        per_token = self.saved_per_token(pattern) + 4 * self.vocab + 4 * self.hidden
        return max(0, int(room * world // per_token))


class Sheet(NamedTuple):
    """One operator call of one CP group, per rank of the group."""

    flops: float        # useful F+B FLOPs per rank
    quadratic: float    # the causal-attention part of ``flops``
    comm: float         # CP bytes per rank on the group's links
    saved: int          # bytes kept for the backward
    work: int           # transient workspace bytes


def _mlp_sheet(m: Model, n: int, squares: int, nseq: int, cp: int) -> Sheet:
    h, f = m.hidden, m.ffn
    return Sheet(18 * n * h * f, 0, 0, n * 2 * (4 * h + 3 * f), n * 2 * (2 * h + 2 * f))


def _gqa_sheet(m: Model, n: int, squares: int, nseq: int, cp: int) -> Sheet:
    h, kv = m.hidden, m.kv_heads * m.head_dim
    qkv = (m.q_heads + 2 * m.kv_heads) * m.head_dim
    quadratic = 6 * m.q_heads * m.head_dim * squares / cp
    return Sheet(6 * n * (h * qkv + h * h) + quadratic, quadratic,
                 3 * (cp - 1) * n * 4 * kv,                      # K/V ring forward + K/V and dK/dV backward
                 n * (2 * (8 * h + qkv) + 4 * m.q_heads),
                 n * (4 * h + 8 * kv * max(1, cp - 1)))


def _gdn_sheet(m: Model, n: int, squares: int, nseq: int, cp: int) -> Sheet:
    h, d = m.hidden, m.gdn_width
    state = 4 * m.gdn_heads * m.gdn_dim ** 2                    # one fp32 recurrent state
    return Sheet(6 * n * (6 * h * d + state), 0,
                 2 * (cp - 1) * nseq * (state + 6 * 3 * d),     # state pass + conv halo, F and B
                 n * 2 * (8 * h + 5 * d),
                 n * 4 * (h + 5 * d) + nseq * cp * state)


SHEETS = {"M": _mlp_sheet, "*": _gqa_sheet, "G": _gdn_sheet}


def cp_overhead_factor(table: dict, cp: int, symbol: str | None = None) -> float:
    """Measured CP overhead factor for degree ``cp``: its own entry, else the largest measured
    degree below it, else the smallest measured degree. ``table`` is either one table for every
    CP operator ({"2": f, ...}) or one per operator symbol ({"G": {"2": f}, "*": {...}}); an
    operator without its own table gets 1."""
    if table and all(isinstance(v, dict) for v in table.values()):
        table = table.get(symbol) if symbol is not None else None
        if not table:
            return 1.0
    measured = sorted(int(k) for k in table)
    usable = [k for k in measured if k <= cp] or measured[:1]
    return float(table[str(usable[-1])])


def _plus(a, b) -> tuple:
    return tuple(x + y for x, y in zip(a, b))


class Evaluator:
    """Prices microbatches of one batch (``lengths``) on ``world`` ranks for one layer ``pattern``."""

    def __init__(self, model: Model, lengths: dict, world: int, pattern: str):
        self.model, self.lengths, self.world, self.pattern = model, lengths, world, pattern
        self.base = model.static(pattern, world) + model.external_bytes + model.margin_bytes
        self.profile = profile_of(model)
        self._none = (0,) * world

    @lru_cache(maxsize=4096)
    def tokens(self, layout) -> tuple[int, ...]:
        return layout.tokens(self.lengths, self.world)

    def _scaled(self, nbytes) -> int:
        return int(self.model.byte_scale * nbytes)

    # ------------------------------------------------------------------ routes
    @lru_cache(maxsize=8192)
    def transfer(self, source, target):
        """(ms of the route and its inverse, per-rank workspace bytes) of a layout change."""
        if source == target:
            return 0.0, self._none
        edges = route(source, target, self.lengths, self.world)
        if identity_route(edges):
            return 0.0, self._none
        m = self.model
        row = 2 * m.hidden
        # per rank: [sent intra, received intra, sent inter, received inter] bytes
        load = [[0, 0, 0, 0] for _ in range(self.world)]
        for src, dst, _, _, count in edges:
            if src == dst:
                continue
            lane = 2 if src // m.ranks_per_node != dst // m.ranks_per_node else 0
            load[src][lane] += count * row
            load[dst][lane + 1] += count * row
        # the busiest rank sets the pace: injection or reception, per link class
        link_ms = max((max(r[0], r[1]) / (m.intra_gbps * 1e6) + max(r[2], r[3]) / (m.inter_gbps * 1e6)
                       for r in load), default=0)
        # the local pack and unpack copies (forward and inverse backward)
        work = tuple(self._scaled(2 * row * (a + b)) for a, b in zip(self.tokens(source), self.tokens(target)))
        copy_ms = max(work) / (m.memory_gbps * 1e6)
        return 2 * (link_ms + copy_ms + m.latency_ms), work

    # ------------------------------------------------------------------ operators
    def _call_ms(self, symbol: str, cp: int, sheet: Sheet, tokens: int, squares: int, cross: bool) -> float:
        m = self.model
        rate = m.compute_tflops * 1e9
        linear, quadratic = (sheet.flops - sheet.quadratic) / rate, sheet.quadratic / rate
        cal = (m.operator_calibration or {}).get(symbol)
        if cal is not None:
            linear = linear / cal["linear"] + cal.get("fixed_ms", 0.0)
            quadratic = quadratic / cal.get("quadratic", 1.0)
        latency = 2 * m.latency_ms * (cp - 1) if symbol != "M" else 0.0
        bandwidth = m.inter_gbps if cross else m.intra_gbps
        parts = Parts(linear, quadratic, sheet.comm / (bandwidth * 1e6) + latency,
                      sheet.comm / (m.intra_gbps * 1e6) + latency)
        ms = self.profile.price(symbol, cp, parts, tokens, squares, cross)
        if cp > 1 and symbol != "M" and m.cp_overhead:
            ms *= cp_overhead_factor(m.cp_overhead, cp, symbol)
        return ms

    @lru_cache(maxsize=4096)
    def operator(self, symbol: str, layout):
        """(ms of the slowest group, saved bytes per rank, workspace bytes per rank) of one operator."""
        m = self.model
        saved, work = [0] * self.world, [0] * self.world
        slowest = None
        for g in layout.groups:
            cp = len(g.ranks)
            sizes = [self.lengths[s] for s in g.samples]
            total, squares = sum(sizes), sum(x * x for x in sizes)
            sheet = SHEETS[symbol](m, total // cp, squares, len(sizes), cp)
            cross = g.ranks[0] // m.ranks_per_node != g.ranks[-1] // m.ranks_per_node
            ms = self._call_ms(symbol, cp, sheet, total, squares, cross)
            slowest = ms if slowest is None else max(slowest, ms)
            for r in g.ranks:
                saved[r], work[r] = self._scaled(sheet.saved), self._scaled(sheet.work)
        return slowest, tuple(saved), tuple(work)

    # ------------------------------------------------------------------ memory walk
    def initial(self, ingress) -> tuple[int, ...]:
        """Live bytes before the first layer: static state plus the residual stream, which
        stays alive through the whole stack."""
        return tuple(self.base + self._scaled(n * 4 * self.model.hidden) for n in self.tokens(ingress))

    def layer(self, live, previous, attention, mlp, symbol):
        """(ms, live bytes after, peak bytes) of one layer entered from layout ``previous``."""
        a_ms, a_saved, a_work = self.operator(symbol, attention)
        m_ms, m_saved, m_work = self.operator("M", mlp)
        in_ms, in_work = self.transfer(previous, attention)
        out_ms, out_work = self.transfer(attention, mlp)
        after_mixer = _plus(live, a_saved)
        after_mlp = _plus(after_mixer, m_saved)
        # forward steps and their backward points: route in, mixer, route to the MLP, MLP, route back
        peak = tuple(max(l0 + i, l1 + max(aw, ow), l2 + max(mw, ow))
                     for l0, l1, l2, i, aw, ow, mw in zip(live, after_mixer, after_mlp, in_work, a_work, out_work,
                                                          m_work))
        # the MLP output returns to the attention placement: two routes each in F and B
        return in_ms + a_ms + m_ms + 2 * out_ms, after_mlp, peak

    def finish(self, live, previous, ingress):
        """(ms, peak bytes) of the return to the ingress layout, the head and the per-microbatch cost."""
        m = self.model
        back_ms, back_work = self.transfer(previous, ingress)
        tokens = self.tokens(ingress)
        logits = [self._scaled(n * (4 * m.vocab + 4 * m.hidden)) for n in tokens]
        peak = tuple(x + max(w, lg) for x, w, lg in zip(live, back_work, logits))
        head_ms = max(tokens) * 6 * m.hidden * m.vocab / (m.compute_tflops * 1e9)
        return back_ms + head_ms + m.microbatch_ms, peak

    def recomputes(self, batch) -> bool:
        """Whether ``batch`` runs with per-layer recompute (``Model.recompute_tokens``)."""
        limit = self.model.recompute_tokens
        if limit is None:
            return False
        layouts = [batch.ingress] + [x for pair in batch.layers for x in pair]
        return max(max(self.tokens(x)) for x in layouts) > limit

    def _evaluate_recompute(self, batch) -> dict:
        """Per-layer recompute: between forward and backward every layer keeps only its input
        (bf16 rows of its attention layout); in the backward one layer at a time is rebuilt, so
        the peak is the checkpoints plus the largest single layer's own walk on top of them, and
        each layer pays its forward (a third of its F+B time) once more."""
        m = self.model
        start, previous = self.initial(batch.ingress), batch.ingress
        checkpoints = [0] * self.world
        for attention, _ in batch.layers:
            checkpoints = [c + self._scaled(n * 2 * m.hidden) for c, n in zip(checkpoints, self.tokens(attention))]
        held = _plus(start, checkpoints)
        peak, total, points = held, 0.0, []
        for index, symbol in enumerate(self.pattern):
            attention, mlp = batch.layers[index]
            ms, _, here = self.layer(held, previous, attention, mlp, symbol)
            rebuild = (self.operator(symbol, attention)[0] + self.operator("M", mlp)[0]) / 3
            total += ms + rebuild
            peak = tuple(map(max, peak, here))
            points.append({"layer": index, "saved_live_bytes": list(held), "peak_bytes": list(here),
                           "attention_tokens": self.tokens(attention), "mlp_tokens": self.tokens(mlp)})
            previous = attention
        ms, here = self.finish(held, previous, batch.ingress)
        peak = tuple(map(max, peak, here))
        return {"predicted_ms": total + ms, "peak_bytes": peak, "fits": max(peak) <= m.budget, "points": points,
                "head_peak_bytes": here, "includes_margin": True, "recompute": True,
                "memory_status": "structural_forward_backward_envelope_not_measured"}

    def evaluate(self, batch) -> dict:
        if self.recomputes(batch):
            return self._evaluate_recompute(batch)
        live, previous = self.initial(batch.ingress), batch.ingress
        peak, total, points = live, 0.0, []
        for index, symbol in enumerate(self.pattern):
            attention, mlp = batch.layers[index]
            ms, live, here = self.layer(live, previous, attention, mlp, symbol)
            total += ms
            peak = tuple(map(max, peak, here))
            points.append({"layer": index, "saved_live_bytes": list(live), "peak_bytes": list(here),
                           "attention_tokens": self.tokens(attention), "mlp_tokens": self.tokens(mlp)})
            previous = attention
        ms, here = self.finish(live, previous, batch.ingress)
        peak = tuple(map(max, peak, here))
        return {"predicted_ms": total + ms, "peak_bytes": peak, "fits": max(peak) <= self.model.budget,
                "points": points, "head_peak_bytes": here, "includes_margin": True,
                "memory_status": "structural_forward_backward_envelope_not_measured"}


def execution_contract(model: Model) -> dict:
    """Model fields the executor must match before replaying a plan (Megatron names)."""
    return {"hidden_size": model.hidden, "ffn_hidden_size": model.ffn, "num_attention_heads": model.q_heads,
            "num_query_groups": model.kv_heads, "kv_channels": model.head_dim,
            "linear_num_key_heads": model.gdn_heads, "linear_num_value_heads": model.gdn_heads,
            "linear_key_head_dim": model.gdn_dim, "linear_value_head_dim": model.gdn_dim,
            "linear_conv_kernel_dim": 4}


def resource_metrics(lengths: dict, world: int, pattern: str, model: Model, predicted_ms: float) -> dict:
    """Whole allocated world (idle ranks included); useful work is plan-invariant."""
    tokens = sum(lengths.values())
    squares = sum(n * n for n in lengths.values())
    flops = sum(operator_work(model, s, tokens, squares) for s in pattern)
    flops += len(pattern) * operator_work(model, "M", tokens, squares)
    flops += 6 * tokens * model.hidden * model.vocab
    gpu_ms = world * predicted_ms
    return {"allocated_gpus": world, "predicted_gpu_ms": gpu_ms, "declared_useful_flops": flops,
            "predicted_useful_tflops_per_gpu": flops / (gpu_ms * 1e9), "status": "modeled_not_measured",
            "flop_scope": "GQA projection/causal attention, GDN projection/recurrence, MLP and output GEMM; "
                          "no CP communication or redundant FLOPs",
            "mfu": None, "mfu_note": "fixed-work same-hardware MFU ratios equal inverse GPU-time ratios"}


def model_from_config(cfg, device_bytes: int, **overrides) -> Model:
    """Planner model for a ``HybridConfig`` (GDN key dim used for the GDN width)."""
    return Model(hidden=cfg.hidden_size, ffn=cfg.ffn_hidden_size, vocab=cfg.vocab_size,
                 q_heads=cfg.num_attention_heads, kv_heads=cfg.num_query_groups, head_dim=cfg.kv_channels,
                 gdn_heads=cfg.linear_num_key_heads, gdn_dim=cfg.linear_key_head_dim,
                 device_bytes=device_bytes, **overrides)
