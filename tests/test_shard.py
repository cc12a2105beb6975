"""Stream sharding across ranks (the multi-GPU plan) on CPU with gloo.

Each rank decodes its contiguous shard of the streams independently (here
with the CPU oracle standing in for the per-GPU decoder); gathering the
shards must reproduce the single-process result token for token, which is
the "1 vs N GPUs gives identical per-stream tokens" property.  Also checks
the failure path: a rank that raises leaves the others with an error from a
short process-group timeout instead of a hang."""

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from noetic_b200.shard import shard_plan, shard_range

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CFG = dict(vocab=29, d_model=16, n_layer=2, expand=2, conv_k=3, mlp_mult=2, eps=1e-5, tau_max=8.0)


def test_shard_plan_covers_every_stream_once():
    for n in [1, 7, 16, 16384, 16385]:
        for world in [1, 2, 3, 4, 8]:
            plan = shard_plan(n, world)
            seen = [s for first, count in plan for s in range(first, first + count)]
            assert seen == list(range(n))
            counts = [c for _, c in plan]
            assert max(counts) - min(counts) <= 1
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def _decode_streams(first, count, steps):
    import sys

    sys.path.insert(0, ROOT)
    import oracle as O
    from noetic_b200.prompts import uniform_prompts

    m = O.Model(O.LmConfig(**CFG), seed=5)
    ids = uniform_prompts(count, 6, CFG["vocab"], 100, first=first)
    out = np.zeros((count, steps), dtype=np.int64)
    for i in range(count):
        d = O.Decoder(m)
        for t in ids[i]:
            lg = d.step(int(t))
        tok = O.argmax(lg)
        for j in range(steps):
            out[i, j] = tok
            tok = O.argmax(d.step(tok))
    return out


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n_streams, steps, result_path, fail_rank):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        if rank == fail_rank:
            raise RuntimeError("injected rank failure")
        first, count = shard_range(n_streams, world, rank)
        mine = torch.from_numpy(_decode_streams(first, count, steps))
        parts = [None] * world
        dist.all_gather_object(parts, mine)
        if rank == 0:
            np.save(result_path, torch.cat(parts).numpy())
    except RuntimeError as e:
        if rank == 0:
            with open(result_path + ".err", "w") as f:
                f.write(str(e))
        if rank == fail_rank:
            os._exit(3)
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_two_rank_sharded_decode_matches_single_process(tmp_path):
    n_streams, steps = 5, 4
    path = str(tmp_path / "tokens.npy")
    mp.start_processes(_worker, args=(2, _free_port(), n_streams, steps, path, -1), nprocs=2, start_method="spawn")
    gathered = np.load(path)
    single = _decode_streams(0, n_streams, steps)
    assert np.array_equal(gathered, single)


def test_a_failing_rank_surfaces_as_an_error_not_a_hang(tmp_path):
    path = str(tmp_path / "tokens.npy")
    with pytest.raises(Exception):
        mp.start_processes(_worker, args=(2, _free_port(), 4, 2, path, 1), nprocs=2, start_method="spawn")
    assert not os.path.exists(path)
