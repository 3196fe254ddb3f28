"""The Megatron-style launcher with tensor and pipeline parallelism on two CPU ranks (gloo)."""

import os
import socket
import traceback

import torch.multiprocessing as mp

TINY = ["--device", "cpu", "--num-layers", "4", "--hidden-size", "256", "--ffn-hidden-size", "512",
        "--vocab-size", "4096", "--num-attention-heads", "4", "--num-query-groups", "2", "--kv-channels", "64",
        "--linear-num-key-heads", "4", "--linear-num-value-heads", "4", "--linear-key-head-dim", "64",
        "--linear-value-head-dim", "64", "--global-batch-size", "3", "--seq-length", "256",
        "--max-seqlen-per-dp-cp-rank", "512", "--train-iters", "2", "--sequence-packing-scheduler", "fixed"]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, argv, queue):
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    try:
        from prism_cp_b200.launcher.train import main
        queue.put((rank, main(argv)))
    except BaseException:  # pragma: no cover - reported to the parent
        queue.put((rank, traceback.format_exc()))


def _run(argv, world=2):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, argv, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(30)
    assert all(v == 0 for v in results.values()), results


def test_launcher_tensor_parallel_two_ranks():
    _run(TINY + ["--tensor-model-parallel-size", "2", "--context-parallel-size", "1"])


def test_launcher_pipeline_parallel_two_ranks():
    _run(TINY + ["--pipeline-model-parallel-size", "2", "--context-parallel-size", "1"])


def test_launcher_online_scheduler_two_ranks():
    """Per-batch CP degrees chosen online by the calibrated cost model, applied on pre-built teams."""
    argv = [a for a in TINY]
    i = argv.index("--sequence-packing-scheduler")
    argv[i + 1] = "online"
    _run(argv + ["--use-varlen-dataset"])


def test_launcher_tensor_parallel_records_save_and_resume(tmp_path):
    """TP = 2 through the launcher: one record file per process, a checkpoint, and a resumed run."""
    rec, ck = tmp_path / "rec", tmp_path / "ck"
    base = TINY + ["--tensor-model-parallel-size", "2", "--context-parallel-size", "1"]
    _run(base + ["--records", str(rec), "--save", str(ck), "--save-interval", "2"])
    assert (rec / "steps_rank0.jsonl").exists() and (rec / "steps_rank1.jsonl").exists()
    assert (ck / "latest_checkpointed_iteration.txt").read_text().strip() == "2"
    argv = list(base)
    argv[argv.index("--train-iters") + 1] = "3"
    _run(argv + ["--load", str(ck)])


def test_launcher_pipeline_parallel_with_full_recompute():
    """``--recompute-granularity full`` reaches the pipeline stages (every stage layer recomputes)."""
    _run(TINY + ["--pipeline-model-parallel-size", "2", "--context-parallel-size", "1",
                 "--recompute-granularity", "full"])


def test_launcher_online_scheduler_with_full_recompute():
    """The online planner with every microbatch recomputing packs by its memory model (no capacity
    collapse) and the trainer recomputes every microbatch."""
    argv = [a for a in TINY]
    i = argv.index("--sequence-packing-scheduler")
    argv[i + 1] = "online"
    _run(argv + ["--use-varlen-dataset", "--recompute-granularity", "full"])
