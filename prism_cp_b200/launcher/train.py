"""Training entry point (``python -m prism_cp_b200.launcher.train <Megatron-style flags>``).

Run one process per GPU under ``torchrun`` (``--master-addr 127.0.0.1`` on one
box). Every update: build or load the global batch, plan it with the selected
scheduler, and run ``Trainer.train_step``:

* ``--sequence-packing-scheduler default_dynamic_cp``: native N with per-rank
  capacity ``--max-seqlen-per-dp-cp-rank`` and ``--min-dynamic-context-parallel-size``,
  rounds coalesced into mixed-CP microbatches;
* ``joint``: the frozen replay rows of ``--joint-replay`` (validated against the
  world and layer pattern);
* ``fixed``: one CP degree ``--context-parallel-size`` for every layer.

Data: ``--packet-manifest`` (deterministic LCG64 content with the first-half
loss mask), ``--varlen-mock-dataset-config-json`` (log-normal or explicit
lengths) or fixed ``--global-batch-size x --seq-length`` documents.
"""

from __future__ import annotations

import datetime
import json
import os
import sys
import time
from pathlib import Path

import torch
import torch.distributed as dist

from ..models.hybrid import HybridModel
from ..parallel.teams import Teams
from ..planner.fixed import uniform_plan
from ..planner.joint.replay import validate_replay
from ..planner.mixed import to_joint
from ..planner.native import replay as native_replay
from ..planner.onedim import from_rank_ids
from ..runtime import checkpoint
from ..runtime.batch import fixed_lengths, lognormal_lengths, make_batch, manifest_batch
from ..runtime.trainer import Trainer
from ..utils.tracing import ProfileWindow, enable_nvtx, nvtx, nvtx_enabled
from .args import build_parser, model_config, validate


def global_batch(args, world: int, step: int, pin: bool):
    if args.packet_manifest:
        manifest = json.loads(Path(args.packet_manifest).read_text())
        from ..planner.inputs import validate_manifest
        validate_manifest(manifest)
        return manifest_batch(manifest, pin=pin)
    if args.varlen_mock_dataset_config_json:
        cfg = json.loads(Path(args.varlen_mock_dataset_config_json).read_text())
        if "lengths" in cfg:
            lengths = list(cfg["lengths"])
        else:
            lengths = lognormal_lengths(cfg.get("total_tokens", 1 << 20), cfg.get("median", 4096),
                                        cfg.get("sigma", 1.0), cfg.get("min", 512), cfg.get("max", 131072),
                                        2 * world, args.seed + step)
        return make_batch(lengths, args.vocab_size, args.seed + step, pin=pin)
    return make_batch(fixed_lengths(args.global_batch_size, args.seq_length), args.vocab_size, args.seed + step,
                      pin=pin)


_PLANNER_MODEL: dict = {}


def _planner_model(args, world: int):
    """The planner's cost model of this run's model shape on B200 (calibrated operator costs)."""
    key = world
    if key not in _PLANNER_MODEL:
        from ..planner.calibrate import calibrated
        from ..planner.cli import B200_ENVELOPE
        from ..planner.joint.cost import model_from_config
        m = model_from_config(model_config(args), B200_ENVELOPE["device_bytes"],
                              **{k: v for k, v in B200_ENVELOPE.items() if k != "device_bytes"})
        m = calibrated(m)
        limit = recompute_limit(args)
        if limit is not None:
            from dataclasses import replace
            m = replace(m, recompute_tokens=limit)
        _PLANNER_MODEL[key] = m
    return _PLANNER_MODEL[key]


def recompute_limit(args) -> int | None:
    """Tokens per rank above which a microbatch recomputes its layers in the backward (None: never)."""
    if args.recompute_granularity == "full":
        return 0
    return args.recompute_tokens


def plan_for(args, batch, world: int, pattern: str, step: int, replays):
    if args.sequence_packing_scheduler == "joint":
        row = replays[(step - 1) % len(replays)]
        plan = validate_replay(row, world, pattern)
        if list(batch.lengths.values()) != row["expected_lengths"]:
            raise SystemExit("joint replay lengths differ from the batch")
        return plan
    if args.sequence_packing_scheduler == "online":
        # per-batch (cp_gdn, cp_gqa) from the calibrated B200 cost model; the dyadic teams already
        # exist, so a new degree needs no new process group
        from ..planner.online import select
        sel = select(batch.lengths, world, pattern, _planner_model(args, world))
        if int(os.environ.get("RANK", "0")) == 0 and (step == 1 or step % max(1, args.log_interval) == 0):
            print(json.dumps({"step": step, "online_cp": {"gdn": sel.cp_gdn, "gqa": sel.cp_gqa},
                              "plan": sel.description,
                              "predicted_update_ms": round(sel.predicted_update_ms, 3)}), flush=True)
        return sel.plan
    if args.sequence_packing_scheduler == "fixed":
        cp = args.context_parallel_size or world
        return uniform_plan(batch.lengths, world, cp, args.max_seqlen_per_dp_cp_rank, pattern)
    rounds = from_rank_ids(native_replay(list(batch.lengths.items()), world, args.max_seqlen_per_dp_cp_rank,
                                         args.min_dynamic_context_parallel_size))
    return to_joint(rounds, batch.lengths, world, pattern, token_cap=args.max_seqlen_per_dp_cp_rank)


def main(argv=None) -> int:
    args = build_parser().parse_args(argv)
    validate(args)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cuda = args.device == "cuda"
    device = torch.device("cuda", local) if cuda else torch.device("cpu")
    if cuda:
        torch.cuda.set_device(device)
    if world > 1:
        backend = args.distributed_backend if cuda else "gloo"
        dist.init_process_group(backend, device_id=device if cuda else None,
                                timeout=datetime.timedelta(minutes=args.distributed_timeout_minutes))
    cfg = model_config(args)
    if rank == 0 and (args.records or args.save):
        # the run's full configuration beside its records / checkpoints (the reference's launch
        # recipe writes its config and command files the same way)
        out = Path(args.records or args.save)
        out.mkdir(parents=True, exist_ok=True)
        env = {k: v for k, v in os.environ.items() if k.startswith(("PRISM_", "NCCL_", "CUDA_VISIBLE"))}
        (out / "launch_config.json").write_text(json.dumps(
            {"argv": list(sys.argv if argv is None else argv), "args": vars(args), "world": world,
             "model": {"name": cfg.name, "pattern": cfg.pattern, "parameters": cfg.parameter_count()},
             "environment": env}, indent=1, default=str))
    dtype = torch.bfloat16 if (args.bf16 and cuda) else torch.float32
    tp_size, pp_size = args.tensor_model_parallel_size, args.pipeline_model_parallel_size
    pipeline = None
    if pp_size > 1:
        # 1F1B over stages of world / pp ranks; each stage builds only its own layers
        from ..runtime.pipeline import PipelineTrainer, make_stage
        info = make_stage(pp_size, cfg.num_layers)
        model = HybridModel(cfg, dtype=dtype, device=device, seed=args.seed,
                            layers=range(info.first_layer, info.first_layer + info.num_layers),
                            pre_process=info.stage == 0, post_process=info.stage == pp_size - 1)
        pipeline = PipelineTrainer(model, info, device, lr=args.lr, min_lr=args.min_lr,
                                   weight_decay=args.weight_decay, clip_grad=args.clip_grad,
                                   warmup_steps=args.lr_warmup_iters,
                                   decay_steps=args.lr_decay_iters or args.train_iters, records=args.records,
                                   recompute_tokens=recompute_limit(args))
        plan_world = info.stage_world
        trainer = pipeline
    else:
        tpc = None
        if tp_size > 1:
            from ..parallel.tensor import make_tp
            tpc = make_tp(tp_size)
        model = HybridModel(cfg, dtype=dtype, device=device, seed=args.seed, tp=tpc)
        teams = Teams(world, tp=tpc) if tpc is not None else Teams(world)
        plan_world = world // tp_size
        trainer = Trainer(model, teams, device, lr=args.lr, min_lr=args.min_lr, weight_decay=args.weight_decay,
                          clip_grad=args.clip_grad, warmup_steps=args.lr_warmup_iters,
                          decay_steps=args.lr_decay_iters or args.train_iters, records=args.records,
                          overlap_grad_reduce=args.overlap_grad_reduce,
                          overlap_param_gather=args.overlap_param_gather,
                          bucket_bytes=(args.ddp_bucket_size or (64 << 20)) * 4,
                          recompute_tokens=recompute_limit(args))
    replays = json.loads(Path(args.joint_replay).read_text()) if args.joint_replay else None
    start = 1
    if args.load and checkpoint.latest(args.load) is not None:
        start = checkpoint.load(trainer, checkpoint.latest(args.load)) + 1
    enable_nvtx(args.nvtx_ranges or nvtx_enabled())
    window = ProfileWindow(args.profile_step_start, args.profile_step_end, args.profile_ranks, rank,
                           enabled=args.profile and cuda)
    for step in range(start, args.train_iters + 1):
        batch = global_batch(args, world, step, pin=cuda)
        plan = plan_for(args, batch, plan_world, cfg.pattern, step, replays)
        window.before(step)
        t0 = time.perf_counter()
        with nvtx(f"step {step}"):
            res = trainer.train_step(batch, plan)
        step_ms = res.elapsed_ms
        if step_ms is None:
            # wall time of the step on this rank (train_step reads the loss, so the device has finished),
            # max over ranks
            if cuda:
                torch.cuda.synchronize(device)
            ms = torch.tensor([(time.perf_counter() - t0) * 1000.0], dtype=torch.float64, device=device)
            if world > 1:
                dist.all_reduce(ms, op=dist.ReduceOp.MAX)
            step_ms = float(ms.item())
        window.after(step)
        if rank == 0 and step % args.log_interval == 0:
            line = {"step": step, "loss": res.loss, "lr": res.lr, "tokens": res.tokens,
                    "microbatches": res.microbatches, "step_ms": round(step_ms, 3),
                    "tokens_per_s": round(res.tokens / step_ms * 1000.0, 1) if step_ms else None}
            for key in ("bubble_fraction", "exposed_p2p_ms", "compute_ms", "pipeline_stages"):
                if key in (res.extra or {}):
                    line[key] = res.extra[key]
            print(json.dumps(line), flush=True)
        if args.save and args.save_interval and step % args.save_interval == 0:
            checkpoint.save(trainer, args.save, plan_cursor=step)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
