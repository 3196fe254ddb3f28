"""Trainer records, audits, contracts and guards on CPU."""

import json

import pytest
import torch

from prism_cp_b200.models.config import hybrid_tiny
from prism_cp_b200.models.hybrid import HybridModel
from prism_cp_b200.parallel.teams import Teams
from prism_cp_b200.planner.fixed import uniform_plan
from prism_cp_b200.runtime import numerics, records
from prism_cp_b200.runtime.audits import AccumulationAudit, CommunicationAudit
from prism_cp_b200.runtime.batch import make_batch
from prism_cp_b200.runtime.trainer import Trainer


def _trainer(tmp_path, **kw):
    cfg = hybrid_tiny()
    model = HybridModel(cfg, dtype=torch.float32, device="cpu", seed=0)
    batch = make_batch([256, 128, 128], cfg.vocab_size, seed=1)
    plan = uniform_plan(batch.lengths, 1, 1, 256, cfg.pattern)
    return Trainer(model, Teams(1), torch.device("cpu"), **kw), batch, plan


def test_records_audit_and_summary(tmp_path):
    tr, batch, plan = _trainer(tmp_path, records=str(tmp_path), audit=True)
    losses = [tr.train_step(batch, plan).loss for _ in range(3)]
    assert losses[-1] < losses[0]
    rows = [json.loads(x) for x in (tmp_path / "steps_rank0.jsonl").read_text().splitlines()]
    assert [r["step"] for r in rows] == [1, 2, 3] and all(r["finite"] for r in rows)
    records.compress(tmp_path, 1)
    manifest = {"input_tokens": batch.total_tokens, "loss_tokens": batch.loss_tokens}
    summary = records.summarize_records(tmp_path, manifest, 3, [2, 3], len(plan.microbatches), world=1)
    assert summary["status"] == "complete" and len(summary["rankmax_seconds"]) == 2


def test_accumulation_audit_rejects_early_reduce_scatter():
    audit = AccumulationAudit()
    audit.backward(0)
    audit.reduce_scatter(10)
    audit.backward(1)
    audit.optimizer_step()
    audit.all_gather(10)
    with pytest.raises(AssertionError, match="after the last backward"):
        audit.check(2)


def test_communication_audit_counts_nothing_without_collectives(tmp_path):
    tr, batch, plan = _trainer(tmp_path)
    with CommunicationAudit() as audit:
        tr.train_step(batch, plan)
    assert audit.summary() == {}


def test_contracts_are_frozen_and_gate_compares(tmp_path):
    c = numerics.contract("cp_bf16_v2")
    assert c["optimizer"]["gradients"]["relative"] == 0.06
    path = tmp_path / "c.json"
    path.write_text(json.dumps(c))
    assert numerics.load_contract(path) == c
    c["logical"]["decoder_Y"] = 0.5
    path.write_text(json.dumps(c))
    with pytest.raises(ValueError, match="frozen"):
        numerics.load_contract(path)
    tr, batch, plan = _trainer(tmp_path)
    gate_w = numerics.TrainingNumerics(tmp_path / "ref", "write", steps=2)
    for step in (1, 2):
        tr.train_step(batch, plan)
        gate_w.observe(step, tr.optimizer)
    tr2, _, _ = _trainer(tmp_path)
    gate_r = numerics.TrainingNumerics(tmp_path / "run", "read", reference=tmp_path / "ref", steps=2)
    for step in (1, 2):
        tr2.train_step(batch, plan)
        gate_r.observe(step, tr2.optimizer)
    assert not gate_r.failures
    assert records.finite({"a": [1.0, torch.ones(2)]}) and not records.finite([float("nan")])


def test_checkpoint_resume_restores_training_state(tmp_path):
    from prism_cp_b200.runtime import checkpoint
    tr, batch, plan = _trainer(tmp_path)
    tr.train_step(batch, plan)
    checkpoint.save(tr, tmp_path / "ck", plan_cursor=1)
    after_save = tr.train_step(batch, plan).loss
    tr2, _, _ = _trainer(tmp_path)
    cursor = checkpoint.load(tr2, checkpoint.latest(tmp_path / "ck"))
    assert cursor == 1 and tr2.optimizer.step_count == 1
    assert abs(tr2.train_step(batch, plan).loss - after_save) < 1e-6


def test_launcher_runs_native_and_fixed_schedulers(capsys):
    from prism_cp_b200.launcher.train import main
    common = ["--device", "cpu", "--num-layers", "4", "--hidden-size", "256", "--ffn-hidden-size", "512",
              "--vocab-size", "4096", "--num-attention-heads", "4", "--num-query-groups", "2", "--kv-channels", "64",
              "--linear-num-key-heads", "4", "--linear-num-value-heads", "4", "--linear-key-head-dim", "64",
              "--linear-value-head-dim", "64", "--global-batch-size", "3", "--seq-length", "256",
              "--max-seqlen-per-dp-cp-rank", "512", "--train-iters", "2"]
    assert main(common) == 0
    assert main(common + ["--sequence-packing-scheduler", "fixed", "--context-parallel-size", "1"]) == 0
    lines = [json.loads(x) for x in capsys.readouterr().out.splitlines() if x.startswith("{")]
    assert len(lines) == 4 and all(x["tokens"] == 768 for x in lines)


def test_overlapped_bucket_reduce_matches_single_bucket():
    """Bucketed ownership with overlapped reduce-scatter and parameter all-gather gives the same
    update as one bucket."""
    import torch
    from prism_cp_b200.models.config import hybrid_tiny
    from prism_cp_b200.models.hybrid import HybridModel
    from prism_cp_b200.parallel.teams import Teams
    from prism_cp_b200.planner.fixed import uniform_plan
    from prism_cp_b200.runtime.batch import make_batch
    from prism_cp_b200.runtime.trainer import Trainer
    cfg = hybrid_tiny()
    batch = make_batch([512, 256, 256], cfg.vocab_size, seed=3)
    plan = uniform_plan(batch.lengths, 1, 1, 512, cfg.pattern)
    results = []
    for grads, params_overlap in ((False, False), (True, False), (True, True), (False, True)):
        model = HybridModel(cfg, dtype=torch.float32, device="cpu", seed=0)
        tr = Trainer(model, Teams(1), torch.device("cpu"), overlap_grad_reduce=grads,
                     overlap_param_gather=params_overlap, bucket_bytes=64 << 10)
        if grads or params_overlap:
            assert len(tr.flat.buckets) > 2
        if params_overlap:
            # the model's own parameters are gathered before the layers'
            pg = tr.param_gather
            assert pg.order[:len(pg.top)] == list(pg.top) and sorted(pg.order) == list(range(len(tr.flat.buckets)))
        losses = [tr.train_step(batch, plan).loss for _ in range(2)]
        params = torch.cat([p.detach().reshape(-1) for p in model.parameters()])
        results.append((losses, params))
    l0, p0 = results[0]
    for l1, p1 in results[1:]:
        assert l0 == pytest.approx(l1, rel=1e-6)
        assert torch.allclose(p0, p1, rtol=1e-5, atol=1e-6)


def test_logical_gate_flags_a_different_model(tmp_path):
    """The logical gate passes against itself and fails against a differently initialised model."""
    import pytest
    import torch
    from prism_cp_b200.models.config import hybrid_tiny
    from prism_cp_b200.models.hybrid import HybridModel
    from prism_cp_b200.planner.fixed import uniform_plan
    from prism_cp_b200.runtime.batch import make_batch
    from prism_cp_b200.runtime.numerics import LogicalNumerics
    from prism_cp_b200.runtime.trainer import Trainer

    class Solo:
        world, rank, initialized = 1, 0, False

        def team(self, ranks):
            return None

    cfg = hybrid_tiny()
    batch = make_batch([384, 256], cfg.vocab_size, seed=3)
    plan = uniform_plan(batch.lengths, 1, 1, 1024, cfg.pattern)

    def step(seed, mode):
        gate = LogicalNumerics(tmp_path, mode=mode, steps=1)
        Trainer(HybridModel(cfg, dtype=torch.float32, device="cpu", seed=seed), Solo(), torch.device("cpu"),
                logical=gate).train_step(batch, plan)
        return gate

    step(0, "write")
    assert not step(0, "read").failures
    with pytest.raises(AssertionError, match="logical numerics gate failed"):
        step(1, "read")


def test_auxiliary_run_records(tmp_path):
    """Inventory, mixed-execution, bucket, timeline and optimizer-memory records beside the step records."""
    tr, batch, plan = _trainer(tmp_path, records=str(tmp_path), audit=True)
    for _ in range(2):
        tr.train_step(batch, plan)
    inv = json.loads((tmp_path / "model_inventory.json").read_text())
    assert inv["total_numel"] == sum(p.numel() for p in tr.model.parameters())
    mixed = [json.loads(x) for x in (tmp_path / "mixed_execution.jsonl").read_text().splitlines()]
    assert [m["step"] for m in mixed] == [1, 2]
    assert len(mixed[0]["microbatches"]) == len(plan.microbatches)
    assert len(mixed[0]["microbatches"][0]["layer_cp"]) == len(tr.model.cfg.pattern)
    buckets = [json.loads(x) for x in (tmp_path / "buckets_rank0.jsonl").read_text().splitlines()]
    assert buckets[-1]["buckets"] and buckets[-1]["buckets"][0]["bytes"] > 0
    timeline = [json.loads(x) for x in (tmp_path / "timeline_rank0.jsonl").read_text().splitlines()]
    events = [e["event"] for e in timeline[-1]["events"]]
    assert events.count("backward") == len(plan.microbatches) and "optimizer_step" in events
    assert all(b["host_ns"] >= a["host_ns"] for a, b in zip(timeline[-1]["events"], timeline[-1]["events"][1:]))
    mem = [json.loads(x) for x in (tmp_path / "optimizer_memory_rank0.jsonl").read_text().splitlines()]
    assert mem[-1]["master"] == mem[-1]["exp_avg"] == mem[-1]["exp_avg_sq"] > 0


def test_launcher_writes_its_run_configuration(tmp_path):
    from prism_cp_b200.launcher.train import main
    rec = tmp_path / "rec"
    argv = ["--device", "cpu", "--num-layers", "4", "--hidden-size", "256", "--ffn-hidden-size", "512",
            "--vocab-size", "4096", "--num-attention-heads", "4", "--num-query-groups", "2", "--kv-channels", "64",
            "--linear-num-key-heads", "4", "--linear-num-value-heads", "4", "--linear-key-head-dim", "64",
            "--linear-value-head-dim", "64", "--global-batch-size", "2", "--seq-length", "256",
            "--max-seqlen-per-dp-cp-rank", "512", "--train-iters", "1", "--records", str(rec)]
    assert main(argv) == 0
    cfg = json.loads((rec / "launch_config.json").read_text())
    assert cfg["argv"] == argv and cfg["args"]["train_iters"] == 1 and cfg["model"]["pattern"] == "GGG*"
    assert (rec / "steps_rank0.jsonl").exists()


def test_recomputed_microbatches_match_stored_activations():
    """A microbatch above the recompute threshold keeps only layer inputs and rebuilds each
    layer in the backward: loss and every gradient equal the stored-activation run."""
    from prism_cp_b200.runtime.executor import recomputes
    grads = {}
    for limit in (None, 128):
        cfg = hybrid_tiny()
        model = HybridModel(cfg, dtype=torch.float32, device="cpu", seed=0)
        batch = make_batch([256, 128, 128], cfg.vocab_size, seed=1)
        plan = uniform_plan(batch.lengths, 1, 1, 256, cfg.pattern)
        tr = Trainer(model, Teams(1), torch.device("cpu"), recompute_tokens=limit)
        if limit is not None:
            assert all(recomputes(mb, batch.lengths, 1, limit) for mb in plan.microbatches)
        tr.flat.zero_grad()
        loss = tr.forward_backward(batch.lengths, plan, tr.prepare(batch, plan, pin=False))
        tr.flat.fold_param_grads()
        grads[limit] = (float(loss), tr.flat.grad.clone())
    assert grads[None][0] == pytest.approx(grads[128][0], rel=1e-6)
    assert torch.allclose(grads[None][1], grads[128][1], rtol=1e-5, atol=1e-7)


def test_planner_prices_recompute_for_oversize_documents():
    from dataclasses import replace
    from prism_cp_b200.models.config import PRESETS
    from prism_cp_b200.planner.joint.cost import Evaluator, Model
    from prism_cp_b200.planner.online import select
    cfg = PRESETS["hybrid-1.3b"]()
    base = Model(hidden=cfg.hidden_size, ffn=cfg.ffn_hidden_size, vocab=cfg.vocab_size, q_heads=16, kv_heads=4,
                 head_dim=128, gdn_heads=16, gdn_dim=128, device_bytes=180 * 10 ** 9, compute_tflops=1400.0)
    lengths = {0: 131072, **{i: 4096 for i in range(1, 17)}}
    with pytest.raises(ValueError):
        select(lengths, 1, cfg.pattern, base, degrees=(1,))
    sel = select(lengths, 1, cfg.pattern, replace(base, recompute_tokens=32768), degrees=(1,))
    ev = Evaluator(replace(base, recompute_tokens=32768), lengths, 1, cfg.pattern)
    rows = [ev.evaluate(mb) for mb in sel.plan.microbatches]
    assert [bool(r.get("recompute")) for r in rows].count(True) == 1 and all(r["fits"] for r in rows)
    long_mb = next(mb for mb, r in zip(sel.plan.microbatches, rows) if r.get("recompute"))
    assert 0 in long_mb.ingress.groups[0].samples


def test_tokenwise_fusion_and_packet_accounting():
    """Audited steps: every mixer / MLP runs once per microbatch (not per CP segment), every
    microbatch runs one forward and one backward, and the parameter version holds within the update."""
    from prism_cp_b200.runtime.audits import PacketAccounting, TokenwiseFusionAudit
    tr, batch, plan = _trainer(None, audit=True)
    tr.train_step(batch, plan)
    assert all(v == len(plan.microbatches) for v in tr.fusion.calls.values()) and tr.fusion.calls
    assert tr.last_packet["forwards"] == tr.last_packet["backwards"] == len(plan.microbatches)
    # a mixer called twice in one microbatch (split per segment) is caught
    tr.fusion.reset()
    tr.fusion.calls["layer0.mixer"] = 2 * len(plan.microbatches)
    with pytest.raises(ValueError, match="not fused"):
        tr.fusion.check(len(plan.microbatches))
    # a parameter update between forward and backward is caught
    acct = PacketAccounting()
    acct.begin(version=3, microbatches=1)
    x = torch.ones(2, requires_grad=True)
    y = acct.forward(x * 2, 3)
    acct.version = 4
    with pytest.raises(ValueError, match="during backward"):
        y.sum().backward()
    acct2 = PacketAccounting()
    acct2.begin(version=0, microbatches=2)
    acct2.forward(torch.ones(2, requires_grad=True) * 1, 0).sum().backward()
    with pytest.raises(ValueError, match="F/B mismatch"):
        acct2.finish(0)
    # recomputed layers are not counted twice
    cfg_tr = Trainer(HybridModel(hybrid_tiny(), dtype=torch.float32, device="cpu", seed=0), Teams(1),
                     torch.device("cpu"), audit=True, recompute_tokens=64)
    cfg_tr.train_step(batch, plan)
    assert all(v == len(plan.microbatches) for v in cfg_tr.fusion.calls.values())
