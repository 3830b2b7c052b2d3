"""Episode sharding and the multi-rank host plumbing, on CPU with gloo
(world_size 2): the shard plan, max-over-ranks timing, and a rank that fails
before a collective surfacing as an error on its peer instead of a hang."""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import pytest
import torch.multiprocessing as mp

from tarmac_b200 import shard

PKG = str(Path(__file__).resolve().parents[1] / "topk-tarmac_b200")


def test_shard_range_covers_batch_exactly():
    for B in (1, 7, 256, 1024, 4096, 1023):
        for world in (1, 2, 4, 8):
            seen = []
            for r in range(world):
                b0, b1 = shard.shard_range(B, world, r)
                assert 0 <= b0 <= b1 <= B
                seen.extend(range(b0, b1))
            assert seen == list(range(B))
    with pytest.raises(ValueError):
        shard.shard_range(8, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, fail_rank, q):
    sys.path.insert(0, PKG)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                      RANK=str(rank), LOCAL_RANK=str(rank),
                      WORLD_SIZE=str(world))
    from tarmac_b200 import shard as sh
    try:
        sh.init("gloo", timeout_s=10)
        b0, b1 = sh.shard_range(1024, world, rank)
        sh.barrier()
        t = sh.max_over_ranks(float(rank + 1) * 1.5)
        rows = sh.sum_over_ranks(float(b1 - b0))
        if rank == fail_rank:
            raise RuntimeError("injected failure before the next collective")
        sh.barrier()
        q.put((rank, "ok", t, rows))
    except Exception as e:  # reported to the parent, never swallowed
        q.put((rank, "error", type(e).__name__, str(e)[:200]))
    finally:
        try:
            sh.shutdown()
        except Exception:
            pass


def _run(world, fail_rank):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, fail_rank, q))
          for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(res)


def test_two_ranks_max_and_sum():
    res = _run(2, fail_rank=-1)
    assert [r[1] for r in res] == ["ok", "ok"]
    assert all(r[2] == 3.0 for r in res)        # max over ranks of 1.5, 3.0
    assert all(r[3] == 1024.0 for r in res)     # shards cover the batch


def test_failed_rank_surfaces_as_error_on_peer():
    res = _run(2, fail_rank=1)
    status = {r[0]: r[1] for r in res}
    assert status[1] == "error"
    assert status[0] == "error"  # its barrier fails (peer gone / timeout)


class _FakeNvml:
    """NVML stand-in: the GPU at bus id 0000001B:00 is local to CPUs 0-3 and
    64; everything else is unknown."""

    def __init__(self):
        self.shutdown = False

    def nvmlInit(self):
        pass

    def nvmlShutdown(self):
        self.shutdown = True

    def nvmlDeviceGetHandleByPciBusId(self, bus):
        if not bus.endswith(":1B:00.0"):
            raise RuntimeError("not found")
        return "h"

    def nvmlDeviceGetCpuAffinity(self, h, words):
        return [0b1111, 0b1] + [0] * (words - 2)


def test_local_cpus_reads_nvml_mask_within_current_affinity():
    fake = _FakeNvml()
    allowed = set(os.sched_getaffinity(0))
    cpus = shard.local_cpus("00000000:1B:00.0", nvml=fake)
    want = sorted({0, 1, 2, 3, 64} & allowed)
    assert cpus == (want or None)
    assert fake.shutdown
    assert shard.local_cpus("00000000:2C:00.0", nvml=_FakeNvml()) is None
