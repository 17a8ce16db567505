"""CPU tests of the multi-GPU decode plumbing with world_size 2 over gloo.

Each rank decodes its LPT shard of the sequences with the C oracle (standing
in for the CUDA kernel, which needs a GPU), then the outputs are gathered with
shard.OutputGather -- the exact collective bench.py runs over NCCL -- and
compared with a single-process decode of all sequences.  A second test makes
one rank leave before the collective and checks that the other rank's
collective ends with an error inside the process-group timeout (failure made
on the host, no GPU involved).
"""
import os
import socket
import sys
from datetime import timedelta

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
NH, NKV, HD = 32, 4, 64
QD, KVD = NH * HD, NKV * HD


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def make_inputs(seed=21, n=7, equal=False):
    rng = np.random.default_rng(seed)
    lengths = np.full(n, 150) if equal else rng.integers(1, 300, n)
    caps = [int(L) + 3 for L in lengths]
    kcs = [rng.standard_normal((1, c, KVD), dtype=np.float32) for c in caps]
    vcs = [rng.standard_normal((1, c, KVD), dtype=np.float32) for c in caps]
    q = rng.standard_normal((n, QD), dtype=np.float32)
    k = rng.standard_normal((n, KVD), dtype=np.float32)
    v = rng.standard_normal((n, KVD), dtype=np.float32)
    return lengths, caps, kcs, vcs, q, k, v


def _worker(rank, world, port, result_path, equal=False):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, os.path.join(ROOT, "tinyllama-engine_b200"))
    import torch
    import torch.distributed as dist
    import oracle
    import shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    lengths, caps, kcs, vcs, q, k, v = make_inputs(n=8 if equal else 7, equal=equal)
    p = shard.plan(lengths, world)
    mine = p.mine(rank)
    gather = shard.OutputGather(p, QD, "cpu")
    # equal lengths: decode straight into this rank's slot (in-place gather)
    out = gather.local_slot(rank).numpy() if equal else np.zeros((p.max_local, QD), np.float32)
    if mine:
        part = np.zeros((len(mine), QD), np.float32)
        oracle.port().decode_batch([kcs[s] for s in mine], [vcs[s] for s in mine],
                                   [caps[s] for s in mine], [int(lengths[s]) - 1 for s in mine],
                                   q[mine].copy(), k[mine].copy(), v[mine].copy(), part, 0)
        out[:len(mine)] = part
    full = gather(gather.local_slot(rank) if equal else torch.from_numpy(out))
    if rank == 0:
        np.save(result_path, full.numpy())
    dist.barrier()
    dist.destroy_process_group()


def _deserter(rank, world, port, result_path):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        return  # leaves between steps: never joins the collective
    buf = torch.zeros(4)
    try:
        dist.all_reduce(buf)
        msg = "no error"
    except Exception as e:  # noqa: BLE001  (gloo raises RuntimeError/DistBackendError)
        msg = "error: " + type(e).__name__
    with open(result_path, "w") as f:
        f.write(msg)


@pytest.mark.parametrize("equal", [False, True])
def test_sharded_decode_gather_matches_single_process(tmp_path, equal):
    """Ragged lengths: LPT shards, gather + reorder.  Equal lengths (the
    config-5 shape): contiguous blocks decoded into the gather buffer's own
    slots, gathered in place and already in sequence order."""
    import torch.multiprocessing as mp
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, os.path.join(ROOT, "tinyllama-engine_b200"))
    import oracle
    import shard
    res = str(tmp_path / "gathered.npy")
    mp.start_processes(_worker, args=(2, free_port(), res, equal), nprocs=2, start_method="spawn")
    got = np.load(res)
    lengths, caps, kcs, vcs, q, k, v = make_inputs(n=8 if equal else 7, equal=equal)
    if equal:
        p = shard.plan(lengths, 2)
        assert p.local == [[0, 1, 2, 3], [4, 5, 6, 7]]
        assert shard.OutputGather(p, QD, "cpu").in_order
    want = np.zeros((len(lengths), QD), np.float32)
    oracle.port().decode_batch(kcs, vcs, caps, [int(L) - 1 for L in lengths], q.copy(), k.copy(),
                               v, want, 0)
    assert np.array_equal(got, want)


def test_rank_leaving_before_collective_is_detected(tmp_path):
    import torch.multiprocessing as mp
    res = str(tmp_path / "msg.txt")
    mp.start_processes(_deserter, args=(2, free_port(), res), nprocs=2, start_method="spawn")
    assert open(res).read().startswith("error"), open(res).read()


def test_plan_gather_rows_are_a_permutation():
    sys.path.insert(0, os.path.join(ROOT, "tinyllama-engine_b200"))
    import shard
    lengths = np.random.default_rng(0).integers(128, 2049, 64)
    for world in (1, 2, 4, 8):
        p = shard.plan(lengths, world)
        rows = sorted(p.gather_row)
        assert len(set(rows)) == len(lengths)
        assert all(0 <= r < world * p.max_local for r in rows)
        for r in range(world):
            for i, s in enumerate(p.local[r]):
                assert p.gather_row[s] == r * p.max_local + i


def test_context_plan_covers_rows_and_last_rank_holds_newest():
    import shard
    for n, w in [(10, 3), (8, 8), (32768, 8), (1000003, 7)]:
        p = shard.context_plan(n, w)
        assert p.bounds[0][0] == 0 and p.bounds[-1][1] == n
        assert all(p.bounds[r][1] == p.bounds[r + 1][0] for r in range(w - 1))
        sizes = [b - a for a, b in p.bounds]
        assert max(sizes) - min(sizes) <= 1 and min(sizes) >= 1
    with pytest.raises(ValueError):
        shard.context_plan(3, 4)
