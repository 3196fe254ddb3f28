"""Cost and whole forward/backward memory model of a joint plan.

``Model`` holds the model shape, device bytes, external/margin reservations,
throughput and link assumptions, and an optional hardware CP response
profile. ``Evaluator`` prices a microbatch layer by layer: the operator time of
each layout (analytic FLOPs and CP communication, replaced or corrected by the
response profile), the transfer time of every layout change (forward route
and its inverse in the backward), and a per-rank memory envelope that
accumulates saved activations layer by layer and adds each step's workspace,
both for the forward prefix and the matching backward point. All times are
milliseconds of forward + backward.

Formulas and constants follow the reference evaluator
(experiments/sequence_dynamic_cp/joint_cp/model.py:17-228) so predicted update
times of identical plans agree; ``Model.byte_scale`` lets a measured B200
profile rescale the activation terms of this framework's own kernels.
"""

from __future__ import annotations

import math
from dataclasses import asdict, dataclass
from functools import lru_cache

from .ir import identity_route, route
from .response import Response, operator_work, validate_response

GIB = 1024 ** 3


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

    def __post_init__(self):
        for key, value in asdict(self).items():
            if isinstance(value, (int, float)) and not isinstance(value, bool):
                if not math.isfinite(value) or value < 0:
                    raise ValueError(f"Invalid model field {key}")
        for key in ("hidden", "ffn", "vocab", "q_heads", "kv_heads", "head_dim", "gdn_heads", "gdn_dim",
                    "device_bytes", "compute_tflops", "intra_gbps", "inter_gbps", "memory_gbps",
                    "ranks_per_node", "byte_scale"):
            if getattr(self, key) <= 0:
                raise ValueError(f"Model field must be positive: {key}")
        if self.cp_response is not None:
            validate_response(self.cp_response, self)
        for sym, cal in (self.operator_calibration or {}).items():
            if sym not in ("G", "*", "M") or not (cal.get("linear", 0) > 0 and cal.get("quadratic", 1) > 0
                                                  and cal.get("fixed_ms", 0) >= 0):
                raise ValueError(f"invalid operator calibration for {sym!r}: {cal}")

    @property
    def budget(self) -> int:
        return min(int(0.9 * self.device_bytes), self.device_bytes - 8 * GIB)

    def params(self, pattern: str) -> int:
        h, d = self.hidden, self.gdn_heads * self.gdn_dim
        gqa = h * (self.q_heads + 2 * self.kv_heads) * self.head_dim + h * h
        gdn = h * 5 * d + d * h + 4 * 3 * d + 2 * self.gdn_heads
        return (2 * self.vocab * h + len(pattern) * (3 * h * self.ffn + 4 * h)
                + pattern.count("*") * gqa + pattern.count("G") * gdn + h)

    def static(self, pattern: str, world: int) -> int:
        if self.static_bytes is not None:
            return self.static_bytes
        # bf16 weights, fp32 gradients, fp32 master/m/v sharded over the world, buffer reserve
        return math.ceil(self.params(pattern) * (6 + 12 / world)) + 256 * 1024 ** 2

    def saved_per_token(self, pattern: str) -> float:
        h, d = self.hidden, self.gdn_heads * self.gdn_dim
        gqa_io = (self.q_heads + 2 * self.kv_heads) * self.head_dim
        return self.byte_scale * (4 * h + pattern.count("G") * 2 * (8 * h + 5 * d)
                                  + pattern.count("*") * (2 * (8 * h + gqa_io) + 4 * self.q_heads)
                                  + len(pattern) * 2 * (4 * h + 3 * self.ffn))

    def token_capacity_upper_bound(self, pattern: str, world: int) -> int:
        """Necessary (not sufficient) token ceiling from average live storage at the head."""
        head = 4 * self.vocab + 4 * self.hidden
        room = self.budget - self.static(pattern, world) - self.external_bytes - self.margin_bytes
        return max(0, int(room * world // (self.saved_per_token(pattern) + head)))


def _cp_factor(table: dict, cp: int) -> float:
    """Measured CP overhead factor for degree ``cp``: its own entry, else the largest measured degree
    below it, else the smallest measured degree."""
    known = sorted(int(k) for k in table)
    below = [k for k in known if k <= cp]
    return float(table[str(cp if cp in known else (below[-1] if below else known[0]))])


class Evaluator:
    def __init__(self, model: Model, lengths: dict, world: int, pattern: str):
        self.model, self.lengths, self.world, self.pattern = model, lengths, world, pattern
        self.base = model.static(pattern, world) + model.external_bytes + model.margin_bytes
        self.response = Response(model)
        self._zeros = (0,) * world

    @lru_cache(maxsize=4096)
    def tokens(self, layout) -> tuple[int, ...]:
        return layout.tokens(self.lengths, self.world)

    @lru_cache(maxsize=8192)
    def transfer(self, source, target):
        """(ms forward+inverse, per-rank workspace bytes) of a layout change."""
        m = self.model
        if source == target:
            return 0.0, self._zeros
        edges = route(source, target, self.lengths, self.world)
        if identity_route(edges):
            return 0.0, self._zeros
        row = 2 * m.hidden
        out_intra, out_inter = [0] * self.world, [0] * self.world
        in_intra, in_inter = [0] * self.world, [0] * self.world
        for src, dst, _, _, n in edges:
            if src == dst:
                continue
            cross = src // m.ranks_per_node != dst // m.ranks_per_node
            (out_inter if cross else out_intra)[src] += n * row
            (in_inter if cross else in_intra)[dst] += n * row
        # the critical rank's injection/receive time, not the sum over GPUs
        link_ms = max((max(a, b) / (m.intra_gbps * 1e6) + max(c, d) / (m.inter_gbps * 1e6)
                       for a, b, c, d in zip(out_intra, in_intra, out_inter, in_inter)), default=0.0)
        work = tuple(int(m.byte_scale * 2 * row * (a + b)) for a, b in zip(self.tokens(source), self.tokens(target)))
        copy_ms = max(work) / (m.memory_gbps * 1e6)
        return 2 * (link_ms + copy_ms + m.latency_ms), work

    @lru_cache(maxsize=4096)
    def operator(self, symbol: str, layout):
        """(ms, saved bytes per rank, workspace bytes per rank) of one layer operator."""
        m = self.model
        times = []
        saved, work = [0] * self.world, [0] * self.world
        h, f, d = m.hidden, m.ffn, m.gdn_heads * m.gdn_dim
        bs = m.byte_scale
        for g in layout.groups:
            cp = len(g.ranks)
            lens = [self.lengths[s] for s in g.samples]
            n = sum(lens) // cp
            squares = sum(x * x for x in lens)
            quadratic = 0
            if symbol == "M":
                flops, comm = 18 * n * h * f, 0
                save, ws = n * 2 * (4 * h + 3 * f), n * 2 * (2 * h + 2 * f)
            elif symbol == "*":
                proj = 6 * n * (h * (m.q_heads + 2 * m.kv_heads) * m.head_dim + h * h)
                quadratic = 6 * m.q_heads * m.head_dim * squares / cp
                flops = proj + quadratic
                comm = 3 * (cp - 1) * n * 4 * m.kv_heads * m.head_dim
                save = n * (2 * (8 * h + (m.q_heads + 2 * m.kv_heads) * m.head_dim) + 4 * m.q_heads)
                ws = n * (4 * h + 8 * m.kv_heads * m.head_dim * max(1, cp - 1))
            else:
                flops = 6 * n * (6 * h * d + 4 * m.gdn_heads * m.gdn_dim ** 2)
                comm = 2 * (cp - 1) * len(lens) * (4 * m.gdn_heads * m.gdn_dim ** 2 + 6 * 3 * d)
                save = n * 2 * (8 * h + 5 * d)
                ws = n * 4 * (h + 5 * d) + len(lens) * cp * 4 * m.gdn_heads * m.gdn_dim ** 2
            cross = g.ranks[0] // m.ranks_per_node != g.ranks[-1] // m.ranks_per_node
            bandwidth = m.inter_gbps if cross else m.intra_gbps
            latency = 2 * m.latency_ms * (cp - 1) if symbol != "M" else 0.0
            rate = m.compute_tflops * 1e9
            lin_ms, quad_ms = (flops - quadratic) / rate, quadratic / rate
            cal = (m.operator_calibration or {}).get(symbol)
            if cal is not None:
                lin_ms = lin_ms / cal["linear"] + cal.get("fixed_ms", 0.0)
                quad_ms = quad_ms / cal.get("quadratic", 1.0)
            ms = self.response.cost(symbol, cp, lin_ms, quad_ms,
                                    comm / (bandwidth * 1e6) + latency, comm / (m.intra_gbps * 1e6) + latency,
                                    sum(lens), squares, cross_node=cross)
            if cp > 1 and m.cp_overhead and symbol != "M":
                ms *= _cp_factor(m.cp_overhead, cp)
            times.append(ms)
            for r in g.ranks:
                saved[r], work[r] = int(bs * save), int(bs * ws)
        return max(times), tuple(saved), tuple(work)

    def initial(self, ingress) -> tuple[int, ...]:
        # the embedding output / residual stays alive through the whole stack
        return tuple(self.base + int(self.model.byte_scale * n * 4 * self.model.hidden)
                     for n in self.tokens(ingress))

    def layer(self, live, previous, attention, mlp, symbol):
        a_ms, a_save, a_ws = self.operator(symbol, attention)
        m_ms, m_save, m_ws = self.operator("M", mlp)
        in_ms, in_ws = self.transfer(previous, attention)
        out_ms, out_ws = self.transfer(attention, mlp)
        after_a = tuple(x + y for x, y in zip(live, a_save))
        after_m = tuple(x + y for x, y in zip(after_a, m_save))
        points = (tuple(x + y for x, y in zip(live, in_ws)),
                  tuple(x + y for x, y in zip(after_a, a_ws)),
                  tuple(x + y for x, y in zip(after_a, out_ws)),
                  tuple(x + y for x, y in zip(after_m, m_ws)),
                  tuple(x + y for x, y in zip(after_m, out_ws)))
        peak = tuple(max(col) for col in zip(*points))
        # the MLP output returns to the attention placement: two routes each in F and B
        return in_ms + a_ms + m_ms + 2 * out_ms, after_m, peak

    def finish(self, live, previous, ingress):
        back_ms, back_ws = self.transfer(previous, ingress)
        m, tokens = self.model, self.tokens(ingress)
        peak = tuple(a + max(b, int(m.byte_scale * n * (4 * m.vocab + 4 * m.hidden)))
                     for a, b, n in zip(live, back_ws, tokens))
        head_ms = max(tokens) * 6 * m.hidden * m.vocab / (m.compute_tflops * 1e9)
        return back_ms + head_ms + m.microbatch_ms, peak

    def evaluate(self, batch) -> dict:
        live, previous = self.initial(batch.ingress), batch.ingress
        peak, total, points = live, 0.0, []
        for index, (symbol, (attention, mlp)) in enumerate(zip(self.pattern, batch.layers)):
            cost, live, here = self.layer(live, previous, attention, mlp, symbol)
            peak = tuple(max(a, b) for a, b in zip(peak, here))
            total += cost
            points.append({"layer": index, "saved_live_bytes": list(live), "peak_bytes": list(here),
                           "attention_tokens": self.tokens(attention), "mlp_tokens": self.tokens(mlp)})
            previous = attention
        cost, here = self.finish(live, previous, batch.ingress)
        peak = tuple(max(a, b) for a, b in zip(peak, here))
        return {"predicted_ms": total + cost, "peak_bytes": peak, "fits": max(peak) <= self.model.budget,
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
