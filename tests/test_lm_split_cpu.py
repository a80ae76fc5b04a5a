"""Row-split LM head, host side, on CPU: two gloo ranks each hold a slice of
the vocabulary rows (g4_lm_split_rows), compute the packed (value, first
index) key of every sequence's largest logit in their slice (the device
epilogue's key, g4_argmax_keys), all-gather the keys and merge them for
their own sequences (g4_lm_split_merge, the function the device merge kernel
runs).  The merged token must be the first index of the largest logit over
the whole vocabulary, the reference's greedy rule (sample_token with
temp <= 0, gemma4-4b/cpu-blas/main.c:2045-2050), including ties that straddle
the slice boundary."""
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _pkg():
    sys.path.insert(0, ROOT)
    import bench
    return bench.load_pkg()


def _logits(world, B, V):
    rng = np.random.default_rng(77)
    L = rng.standard_normal((world * B, V)).astype(np.float32)
    chunk, _, _ = _pkg().lm_split_rows(V, world, 0)
    L[0, [5, chunk + 3]] = 9.0           # tie across the slice boundary: the lower index wins
    L[1, [chunk + 7, chunk + 2]] = 8.5   # tie inside one slice
    L[2, :] = 0.0
    L[2, chunk + 1] = -0.0               # -0 and +0 are equal: index 0 wins
    L[3, V - 1] = 50.0                   # the last row of the last slice
    return L


def test_split_rows_cover_vocab():
    g4 = _pkg()
    for V in (262144, 4096, 1000):
        for world in (2, 4, 8):
            spans = [g4.lm_split_rows(V, world, r)[1:] for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == V
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, B, V, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank))
    try:
        import torch
        import torch.distributed as dist
        g4 = _pkg()
        dist.init_process_group("gloo", rank=rank, world_size=world)
        L = _logits(world, B, V)
        chunk, r0, r1 = g4.lm_split_rows(V, world, rank)
        # this rank's slice for every rank's sequences; keys carry slice-local row indices
        mine = np.array([g4.argmax_key(L[s, r0:r1]) if r1 > r0 else 0 for s in range(world * B)], np.uint64)
        got = [torch.zeros(world * B, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(got, torch.from_numpy(mine.view(np.int64)))
        keys_all = np.stack([g.numpy().view(np.uint64) for g in got])
        merged = g4.lm_split_merge(keys_all, world, rank, B, chunk)
        toks = [0xffffffff - int(k & np.uint64(0xffffffff)) for k in merged]
        want = [int(np.argmax(L[rank * B + b])) for b in range(B)]
        dist.destroy_process_group()
        q.put((rank, toks, want))
    except Exception as ex:
        q.put((rank, repr(ex), None))


@pytest.mark.parametrize("world", [2])
def test_gloo_split_argmax_merge(world):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    B, V = 4, 4096
    procs = [ctx.Process(target=_rank, args=(r, world, port, B, V, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, toks, want in res:
        assert toks == want, (rank, toks, want)
