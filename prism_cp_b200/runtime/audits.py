"""Run-time audits: collective inventory, accumulation ordering, input integrity.

* ``CommunicationAudit`` records every torch.distributed collective issued
  inside its context (name, shapes, bytes, group size, caller) - the
  reference's one-step collective inventory (communication_audit.py:8-63).
* ``AccumulationAudit`` checks the update contract the reference enforces
  around Megatron's DDP (accumulation_audit.py:8-174): no gradient
  reduce-scatter before the last backward of the update, exactly one
  reduce-scatter, one optimizer step and one parameter all-gather per update,
  and the loss-token count.
* ``check_packet_inputs`` compares a rank's materialised tokens, labels,
  positions and loss mask exactly with the deterministic content rule
  (stream_integrity.py / mixed_packet_integrity.py).
"""

from __future__ import annotations

import contextlib
import time
import traceback

import torch
import torch.distributed as dist

_COLLECTIVES = ("all_reduce", "all_gather", "all_gather_into_tensor", "reduce_scatter_tensor", "all_to_all_single",
                "broadcast", "barrier", "batch_isend_irecv", "send", "recv", "isend", "irecv")


def _nbytes(obj) -> int:
    if isinstance(obj, torch.Tensor):
        return obj.numel() * obj.element_size()
    if isinstance(obj, (list, tuple)):
        return sum(_nbytes(x) for x in obj)
    if isinstance(obj, dist.P2POp):
        return _nbytes(obj.tensor)
    return 0


class CommunicationAudit(contextlib.AbstractContextManager):
    def __init__(self, stacks: bool = False):
        self.events: list[dict] = []
        self.stacks = stacks
        self._saved = {}

    def __enter__(self):
        for name in _COLLECTIVES:
            fn = getattr(dist, name, None)
            if fn is None:
                continue
            self._saved[name] = fn

            def wrapper(*args, __fn=fn, __name=name, **kwargs):
                group = kwargs.get("group")
                size = dist.get_world_size(group) if dist.is_initialized() else 1
                ev = {"op": __name, "bytes": sum(_nbytes(a) for a in args), "group_size": size,
                      "shapes": [list(a.shape) for a in args if isinstance(a, torch.Tensor)]}
                if self.stacks:
                    ev["stack"] = traceback.format_stack(limit=6)[:-1]
                self.events.append(ev)
                return __fn(*args, **kwargs)

            setattr(dist, name, wrapper)
        return self

    def __exit__(self, *exc):
        for name, fn in self._saved.items():
            setattr(dist, name, fn)
        return False

    def summary(self) -> dict:
        out: dict = {}
        for ev in self.events:
            row = out.setdefault(ev["op"], {"calls": 0, "bytes": 0})
            row["calls"] += 1
            row["bytes"] += ev["bytes"]
        return out


class AccumulationAudit:
    """Event log of one update with the ordering rules of a complete update."""

    def __init__(self):
        self.events: list[tuple] = []
        self.times: list[int] = []      # host nanoseconds of each event (the bucket timeline)

    def _add(self, ev: tuple):
        self.events.append(ev)
        self.times.append(time.perf_counter_ns())

    def backward(self, microbatch: int):
        self._add(("backward", microbatch))

    def reduce_scatter(self, nbytes: int):
        self._add(("reduce_scatter", nbytes))

    def optimizer_step(self):
        self._add(("optimizer_step",))

    def all_gather(self, nbytes: int):
        self._add(("all_gather", nbytes))

    def timeline(self) -> list[dict]:
        t0 = self.times[0] if self.times else 0
        return [{"event": ev[0], "arg": ev[1] if len(ev) > 1 else None, "host_ns": t - t0}
                for ev, t in zip(self.events, self.times)]

    def check(self, microbatches: int, loss_tokens: int | None = None, observed_loss_tokens: int | None = None):
        kinds = [e[0] for e in self.events]
        backwards = [i for i, k in enumerate(kinds) if k == "backward"]
        rs = [i for i, k in enumerate(kinds) if k == "reduce_scatter"]
        if len(backwards) != microbatches:
            raise AssertionError(f"expected {microbatches} backward passes, saw {len(backwards)}")
        if len(rs) != 1 or rs[0] < backwards[-1]:
            raise AssertionError("gradient reduce-scatter must run once, after the last backward")
        if kinds.count("optimizer_step") != 1 or kinds.index("optimizer_step") < rs[0]:
            raise AssertionError("exactly one optimizer step after the reduce-scatter")
        if kinds.count("all_gather") != 1 or kinds.index("all_gather") < kinds.index("optimizer_step"):
            raise AssertionError("exactly one parameter all-gather after the optimizer step")
        if loss_tokens is not None and observed_loss_tokens != loss_tokens:
            raise AssertionError(f"loss tokens {observed_loss_tokens} != {loss_tokens}")
        return True


def check_packet_inputs(source, update: int, ingress_layout, world: int, rank: int, tokens, labels, positions,
                        weights) -> None:
    """Exact comparison of one rank's inputs with the manifest's content rule."""
    t, l, p, w = source.rank_inputs(update, ingress_layout, world, rank)
    for name, a, b in (("tokens", tokens, t), ("labels", labels, l), ("positions", positions, p)):
        if not torch.equal(a.cpu().to(b.dtype), b):
            raise AssertionError(f"input integrity: {name} differ from the deterministic content rule")
    if not torch.equal(weights.cpu().float() > 0, w > 0):
        raise AssertionError("input integrity: loss mask differs from the content rule")


def _in_backward() -> bool:
    """True while the autograd engine runs a backward (e.g. a checkpointed layer recomputing)."""
    return torch._C._current_graph_task_id() != -1


class TokenwiseFusionAudit:
    """Every tokenwise operator (a layer's mixer projections and its MLP) runs exactly once per
    executed microbatch on all of the rank's rows, whatever mix of CP teams the microbatch uses
    (the executor never splits a tokenwise GEMM per CP segment). Counts forward calls of the
    layers' mixer and MLP modules; recomputation inside a backward is not a new call. The
    reference enforces the same on the first step of a mixed-CP run (runtime.py:372-391, 423-426)."""

    def __init__(self, model):
        self.calls: dict[str, int] = {}
        self.handles = []
        for index, layer in enumerate(getattr(model, "layers", [])):
            for name in ("mixer", "mlp"):
                module = getattr(layer, name, None)
                if module is None:
                    continue
                key = f"layer{index}.{name}"
                self.calls[key] = 0
                self.handles.append(module.register_forward_hook(self._counter(key)))

    def _counter(self, key: str):
        def hook(module, inputs, output):
            if not _in_backward():
                self.calls[key] += 1
        return hook

    def reset(self) -> None:
        for key in self.calls:
            self.calls[key] = 0

    def check(self, microbatches: int) -> None:
        wrong = {k: v for k, v in self.calls.items() if v != microbatches}
        if wrong:
            raise ValueError(f"Tokenwise operators were not fused per microbatch (expected {microbatches}): {wrong}")

    def close(self) -> None:
        for h in self.handles:
            h.remove()
        self.handles = []


class PacketAccounting:
    """Forward/backward accounting of one update's microbatches (the reference's packet F/B
    checks, mixed_packet_integrity.py:21-47,99-101):

    * the parameter version (optimizer steps taken) must not change between the first forward
      and the last backward of an update;
    * every microbatch runs exactly one forward and one backward (counted at the embedding
      output, so recomputed layers do not count twice);
    * with ``memory_samples``, allocator state is sampled at forward end, before and after the
      loss and at backward end, for microbatches 1, 2, every 8th and the last."""

    def __init__(self, memory_samples: bool = False):
        self.memory_samples = memory_samples
        self.samples: list[dict] = []
        self.version = None
        self.forwards = self.backwards = 0
        self.expected = 0

    def begin(self, version: int, microbatches: int) -> None:
        self.version, self.expected = version, microbatches
        self.forwards = self.backwards = 0
        self.samples = []

    def _wanted(self, ordinal: int) -> bool:
        return ordinal <= 2 or ordinal % 8 == 0 or ordinal == self.expected

    def sample(self, phase: str, ordinal: int) -> None:
        if not (self.memory_samples and torch.cuda.is_available() and torch.cuda.is_initialized()):
            return
        if self._wanted(ordinal):
            stats = torch.cuda.memory_stats()
            self.samples.append({"phase": phase, "microbatch": ordinal, "allocated": torch.cuda.memory_allocated(),
                                 "reserved": torch.cuda.memory_reserved(),
                                 "active": stats.get("active_bytes.all.current", 0),
                                 "inactive_split": stats.get("inactive_split_bytes.all.current", 0),
                                 "free_total": list(torch.cuda.mem_get_info())})

    def forward(self, embedded: torch.Tensor, version: int) -> torch.Tensor:
        """Count a microbatch forward at its embedding output and arm the backward count."""
        if version != self.version:
            raise ValueError("Parameter version changed inside packet")
        self.forwards += 1
        ordinal = self.forwards
        if embedded.requires_grad:
            def on_backward(grad, ordinal=ordinal):
                self.backwards += 1
                if version != self.version:
                    raise ValueError("Parameter version changed during backward")
                self.sample("B_end", ordinal)
                return grad
            embedded.register_hook(on_backward)
        return embedded

    def finish(self, version: int) -> dict:
        if version != self.version:
            raise ValueError("Parameter version changed inside packet")
        if self.forwards != self.expected or self.backwards != self.expected:
            raise ValueError(f"Packet F/B mismatch {self.forwards}/{self.backwards}/{self.expected}")
        return {"forwards": self.forwards, "backwards": self.backwards, "parameter_version": self.version,
                "memory_boundary_samples": list(self.samples)}
