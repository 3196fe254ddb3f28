"""Failure detection on the host: a rank that raises, a peer that never joins, an HBM budget
rejection agreed across ranks. Every fault here is made on CPU ranks (gloo); nothing faults a GPU."""

import datetime
import os
import socket
import time
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tiny_trainer(world):
    from prism_cp_b200.models.config import hybrid_tiny
    from prism_cp_b200.models.hybrid import HybridModel
    from prism_cp_b200.parallel.teams import Teams
    from prism_cp_b200.planner.fixed import uniform_plan
    from prism_cp_b200.runtime.batch import make_batch
    from prism_cp_b200.runtime.trainer import Trainer
    cfg = hybrid_tiny()
    batch = make_batch([512, 512], cfg.vocab_size, seed=1)
    plan = uniform_plan(batch.lengths, world, world, 512, cfg.pattern)
    tr = Trainer(HybridModel(cfg, dtype=torch.float32, device="cpu", seed=0), Teams(world), torch.device("cpu"))
    return tr, batch, plan


def _raiser(rank, world, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
        tr, batch, plan = _tiny_trainer(world)
        tr.train_step(batch, plan)
        if rank == 1:
            raise RuntimeError("injected failure on rank 1 between steps")
        t0 = time.monotonic()
        try:
            tr.train_step(batch, plan)
            queue.put((rank, "no error"))
        except Exception as err:  # the peer is gone: the next collective must fail, not hang
            queue.put((rank, f"error after {time.monotonic() - t0:.1f}s: {type(err).__name__}"))
    except RuntimeError as err:
        queue.put((rank, f"raised: {err}"))
    except Exception:
        queue.put((rank, traceback.format_exc()))


def test_a_rank_that_raises_ends_its_peers_next_collective_with_an_error():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_raiser, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(queue.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(30)
        if p.is_alive():
            p.kill()
    assert out[1].startswith("raised: injected failure"), out
    assert out[0].startswith("error after"), out
    assert float(out[0].split()[2].rstrip("s:")) < 60, out


def _lonely(port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    t0 = time.monotonic()
    try:
        dist.init_process_group("gloo", rank=0, world_size=2, timeout=datetime.timedelta(seconds=3))
        queue.put("joined")
    except Exception as err:
        queue.put(f"error after {time.monotonic() - t0:.1f}s: {type(err).__name__}")


def test_a_peer_that_never_joins_times_out_the_rendezvous():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    p = ctx.Process(target=_lonely, args=(_free_port(), queue))
    p.start()
    msg = queue.get(timeout=120)
    p.join(30)
    if p.is_alive():
        p.kill()
    assert msg.startswith("error after"), msg


def _admission_rank(rank, world, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        tr, _, _ = _tiny_trainer(world)
        gib = 1024 ** 3
        # fake device memory queries: rank 1 has an external process holding most of the GPU
        total = 180 * gib
        free = (150 if rank == 0 else 10) * gib
        torch.cuda.mem_get_info = lambda device=None: (free, total)
        torch.cuda.max_memory_allocated = lambda device=None: 20 * gib
        torch.cuda.memory_reserved = lambda device=None: 25 * gib
        tr.hbm_guard = True
        ok, mem = tr.admission()
        queue.put((rank, (ok, mem["budget"], mem["required"])))
    except Exception:
        queue.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_hbm_admission_is_agreed_across_ranks():
    from prism_cp_b200.runtime.trainer import hbm_budget
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_admission_rank, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(queue.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(30)
    gib = 1024 ** 3
    assert hbm_budget(180 * gib) == 162 * gib
    # rank 0 alone would be admitted (20 + 5 GiB external); rank 1 (20 + 145 GiB) is not: both reject
    assert out[0][0] is False and out[1][0] is False, out
    assert out[0][2] == 25 * gib and out[1][2] == 165 * gib
