"""Host-side fault injection for the tensor-parallel runner (CPU, gloo ranks).

A rank that dies between decode steps must not hang the others: rank 1 exits
abruptly right after the process group forms; rank 0 then enters the o/down
exchange (the sum all-reduce the decoder performs after its row-split
projections) and must get an error from the collective within the process
group's short timeout instead of waiting forever. No GPU involved.
"""

import json
import multiprocessing
import os
import socket
import sys
import time
from datetime import timedelta

import pytest

torch = pytest.importorskip("torch")
dist = pytest.importorskip("torch.distributed")

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    sys.path[:0] = [os.path.join(HERE, ".."), os.path.join(HERE, "..", "spark-mlx-llm_b200")]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # dies without a word, between steps
    from spark_b200 import tp
    from spark_b200.decoder import DecoderConfig

    cfg = DecoderConfig.small()
    sp = tp.plan(cfg, rank, world)
    part = torch.ones((1, cfg.hidden), dtype=torch.float32) * sp.o_cols[1]
    t0 = time.perf_counter()
    try:
        dist.all_reduce(part)
        outcome = "completed"
    except Exception as exc:  # the collective reports the dead peer
        outcome = type(exc).__name__
    with open(os.path.join(out_dir, "rank0.json"), "w") as f:
        json.dump({"outcome": outcome, "seconds": time.perf_counter() - t0}, f)
    os._exit(0)  # the group is broken: skip its teardown


def test_dead_rank_fails_the_next_collective(tmp_path):
    ctx = multiprocessing.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    deadline = time.time() + 120
    for p in procs:
        p.join(max(1.0, deadline - time.time()))
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
        p.join(5)
    assert not alive, "a rank hung after its peer died"
    assert procs[1].exitcode == 3
    result = json.loads((tmp_path / "rank0.json").read_text())
    assert result["outcome"] != "completed", result
    assert result["seconds"] < 60, result
