"""Multi-GPU host logic on CPU: the batched-decode bench splits independent
sequences evenly over ranks (no collective on the data path) and reports the
max over ranks of the device time.  Run here as two gloo ranks on 127.0.0.1;
on a GPU box the same code runs with NCCL, one process per GPU."""
import os
import socket
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    sys.path.insert(0, ROOT)
    import bench
    return bench


def test_shard_partition():
    bench = _bench()
    for world in (1, 2, 4, 8):
        parts = [bench.shard(64, world, r) for r in range(world)]
        assert [i for p in parts for i in p] == list(range(64))
        assert len({len(p) for p in parts}) == 1
    with pytest.raises(ValueError):
        bench.shard(64, 3, 0)
    with pytest.raises(ValueError):
        bench.shard(64, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    try:
        import numpy as np
        import torch
        import torch.distributed as dist
        bench = _bench()
        d = bench.Dist(world, backend="gloo")
        ids = bench.shard(64, d.world, d.rank)
        # every rank derives its prompts from the same seeded global set
        rng = np.random.default_rng(1234)
        allp = rng.integers(0, 262144, size=(64, 16), dtype=np.int32)
        mine = torch.from_numpy(np.ascontiguousarray(allp[ids.start:ids.stop]))
        got = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(got, mine)
        whole = torch.cat(got).numpy()
        d.barrier()
        ms = d.max(10.0 + rank)  # the slowest rank's time
        d.close()
        q.put((rank, bool((whole == allp).all()), ms, len(ids)))
    except Exception as ex:  # reported to the parent, which fails the test
        q.put((rank, repr(ex), None, None))


@pytest.mark.parametrize("world", [2])
def test_gloo_ranks_shard_and_max(world):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok, ms, n in res:
        assert ok is True, ok
        assert ms == 10.0 + world - 1
        assert n == 64 // world


def test_clock_summary_and_streamed_bytes():
    """Bench host helpers: the clock record's reasons and median, and the
    per-step weight bytes (every tensor once, only the gathered rows of the
    per-layer token table)."""
    bench = _bench()
    c = bench.ClockSampler(0)
    c.rows = [["0", "1965", "1965", "", "0x0", "Not Active", "Not Active", "Not Active", "Not Active"],
              ["0", "1800", "1965", "", "0x4", "Not Active", "Not Active", "Not Active", "Active"],
              ["0", "1965", "1965", "", "0x0", "Not Active", "Not Active", "Not Active", "Not Active"]]
    s = c.summary()
    assert s["sm_mhz"] == 1965.0 and s["sm_max_mhz"] == 1965.0 and s["samples"] == 3
    assert s["reasons"] == ["sw_power_cap"]
    assert bench.ClockSampler(0).summary()["reasons"] == ["unsampled"]

    g4 = bench.load_pkg()
    m = g4.synth.make_model(g4.synth.TINY, seed=1)
    ple = m.t["ple_tok"]
    row = ple.nbytes // ple.shape[0]
    assert m.streamed_bytes(4) == m.weight_bytes() - ple.nbytes + 4 * row
