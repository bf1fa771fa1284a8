"""The N > 1 path of bench.py on CPU: two gloo ranks split the pairs of the workload with
shard_pairs (every pair on exactly one rank, token loads balanced) and agree on the step time
through a MAX all-reduce, as the NCCL ranks do on the GPU box. The encoder forward itself has no
collective: ranks run disjoint pairs (pure data parallelism)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import bench


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out_dir: str):
    import datetime

    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from kleinhirn_b200 import synthetic
        lens = synthetic.seq_lengths("mminilm-l12-xlmr", 4096, 7)
        mine = bench.shard_pairs(lens, world, rank)
        # every rank's index list, padded to a common length, gathered on all ranks
        n = torch.tensor([len(mine)], dtype=torch.int64)
        sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(sizes, n)
        cap = int(max(s.item() for s in sizes))
        pad = torch.full((cap,), -1, dtype=torch.int64)
        pad[: len(mine)] = torch.from_numpy(mine)
        got = [torch.empty(cap, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(got, pad)
        # the step time every rank reports is the max over ranks
        t = torch.tensor([10.0 + rank], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), lens=lens,
                 shards=np.stack([g.numpy() for g in got]), tmax=t.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_two_rank_sharding(tmp_path, world):
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    ref = None
    for r in range(world):
        d = np.load(tmp_path / f"rank{r}.npz")
        if ref is None:
            ref = d
        # every rank saw the same shards (deterministic split) and the same max time
        assert np.array_equal(d["shards"], ref["shards"])
        assert float(d["tmax"][0]) == 10.0 + world - 1
    lens = ref["lens"]
    owned = [s[s >= 0] for s in ref["shards"]]
    allidx = np.concatenate(owned)
    assert np.array_equal(np.sort(allidx), np.arange(len(lens))), "a pair is missing or on two ranks"
    loads = [int(lens[o].sum()) for o in owned]
    assert max(loads) - min(loads) <= int(lens.max()), f"token loads unbalanced: {loads}"
    for o in owned:  # each rank runs its pairs shortest first
        assert np.all(np.diff(lens[o]) >= 0)


def test_shard_single_rank_identity():
    lens = np.array([5, 3, 9, 1], dtype=np.int64)
    mine = bench.shard_pairs(lens, 1, 0)
    assert sorted(mine.tolist()) == [0, 1, 2, 3]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_chunks_are_even_and_bounded(world):
    """Each rank's rows go in even bulk chunks of at most 524,288 (+ one bucket of room for the
    sequence that does not fit exactly): the full C5 step on 1 GPU, and its shares on 2, 4, 8."""
    from kleinhirn_b200 import synthetic
    lens = synthetic.seq_lengths(bench.WORKLOAD, 65536, 1234)
    for rank in range(world):
        mine = bench.shard_pairs(lens, world, rank)
        rows = int(lens[mine].sum())
        chunk = bench.chunk_size(rows, 0)
        n = -(-rows // chunk)
        assert chunk <= 524288 + bench.BUCKET
        # greedy packing of whole sequences fills the chunks: no short extra one
        filled, count = 0, 1
        for ln in lens[mine]:
            if filled + ln > chunk:
                count, filled = count + 1, 0
            filled += int(ln)
        assert count == n, (rows, chunk, count, n)
    assert bench.chunk_size(3960, 0) >= 3960
    assert bench.chunk_size(10, 777) == 777
