"""The benchmark workloads: one global batch and the plan that runs it on ``world`` ranks.

* ``fixed``: ``seqs`` documents of ``seq_len`` tokens, CP = world for every layer (``uniform``).
* ``lognormal``: one global batch of ``total_tokens`` tokens of variable-length documents
  (log-normal lengths, median 4096, sigma 1.0, clipped to 512..131072, seeded, multiples of 16
  tokens so the same batch runs at every world size up to 8); the online planner picks the CP degree
  of the GDN and of the GQA layers from the calibrated B200 cost model (``online``), and microbatches
  above ``recompute_tokens`` per rank recompute their layers in the backward.

Used by ``bench.py`` and by the multi-rank step breakdown (``utils/tracing.py``) so both time the
same thing.
"""

from __future__ import annotations

from dataclasses import dataclass, replace


@dataclass
class Workload:
    batch: object
    plan: object
    description: dict
    parallelism: str
    predicted_ms: float | None


def build(cfg, world: int, workload: str = "lognormal", plan: str = "online", *, seqs: int = 8,
          seq_len: int = 32768, tokens_per_rank: int = 32768, total_tokens: int = 1 << 20, seed: int = 1234,
          recompute_tokens: int | None = 32768, pin: bool = True) -> Workload:
    from ..planner.fixed import uniform_plan
    from .batch import fixed_lengths, lognormal_lengths, make_batch

    if workload == "fixed":
        lengths = fixed_lengths(seqs, seq_len)
        desc = {"global_batch": seqs, "seq_len": seq_len}
    elif workload == "lognormal":
        lengths = lognormal_lengths(total_tokens, 4096, 1.0, 512, 131072, 2 * max(world, 8), seed)
        desc = {"global_batch": len(lengths), "global_batch_tokens": sum(lengths), "seq_len": max(lengths),
                "lengths": "log-normal median 4096 sigma 1.0 clipped 512..131072"}
    else:
        raise ValueError(f"unknown workload {workload!r}")
    batch = make_batch(lengths, cfg.vocab_size, seed, pin=pin)
    if plan == "uniform":
        return Workload(batch, uniform_plan(batch.lengths, world, world, tokens_per_rank, cfg.pattern), desc,
                        f"cp{world}", None)
    if plan != "online":
        raise ValueError(f"unknown plan {plan!r}")
    from ..planner.calibrate import calibrated
    from ..planner.cli import B200_ENVELOPE
    from ..planner.joint.cost import model_from_config
    from ..planner.online import select
    pm = calibrated(model_from_config(cfg, B200_ENVELOPE["device_bytes"],
                                      **{k: v for k, v in B200_ENVELOPE.items() if k != "device_bytes"}))
    pm = replace(pm, recompute_tokens=recompute_tokens)
    try:
        sel = select(batch.lengths, world, cfg.pattern, pm)
    except ValueError as err:
        raise ValueError(f"no (cp_gdn, cp_gqa) plan of this batch fits {world} GPU(s) under the calibrated "
                         f"memory model ({err}); use more GPUs or shorter documents") from err
    return Workload(batch, sel.plan, desc, f"online {sel.description} over {world}", sel.predicted_update_ms)
