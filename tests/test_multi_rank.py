"""The data-parallel host layer (kleinhirn_b200/dp.py) on CPU, with gloo ranks and a TCPStore as on
the GPU box:

- the ranks split the sequences with shard_sequences (every sequence on exactly one rank, token
  loads balanced) and agree on the step time through a MAX all-reduce;
- OutputGather assembles every rank's outputs in input order on rank 0 (the host gather of the
  multi-GPU run, src/encoder.ts:461-474 puts results back in input order);
- failure between steps: a rank that leaves after a step (it exits without announcing itself
  for the next one) is detected by the coordinator's bounded wait on the store, the survivors
  re-shard its sequences among themselves, and the step's outputs are complete.
The encoder forward itself has no collective: ranks run disjoint sequences."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from kleinhirn_b200 import dp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def fake_output(idx: np.ndarray, cols: int) -> np.ndarray:
    """Stand-in for the forward of sequences `idx`: a value only that sequence has."""
    return (np.asarray(idx, dtype=np.float32)[:, None] * 0.5 + np.arange(cols, dtype=np.float32)[None, :] + 1.0)


def _rank_main(rank: int, world: int, port: int, out_dir: str):
    import datetime

    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from kleinhirn_b200 import synthetic
        lens = synthetic.seq_lengths("mminilm-l12-xlmr", 4096, 7)
        shards = [dp.shard_sequences(lens, world, r) for r in range(world)]
        mine = shards[rank]
        # every rank's index list, padded to a common length, gathered on all ranks
        cap = max(len(s) for s in shards)
        pad = torch.full((cap,), -1, dtype=torch.int64)
        pad[: len(mine)] = torch.from_numpy(mine)
        got = [torch.empty(cap, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(got, pad)
        # the step time every rank reports is the max over ranks
        t = torch.tensor([10.0 + rank], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        # the host gather of the outputs in input order on rank 0
        cols = 3
        g = dp.OutputGather(dist, None, rank, shards, cols)
        g.local.numpy()[: len(mine) * cols] = fake_output(mine, cols).ravel()
        out = g.gather()
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), lens=lens,
                 shards=np.stack([x.numpy() for x in got]), tmax=t.numpy(),
                 out=out if out is not None else np.zeros(0))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_two_rank_sharding_and_gather(tmp_path, world):
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
    assert np.array_equal(np.sort(allidx), np.arange(len(lens))), "a sequence is missing or on two ranks"
    loads = [int(lens[o].sum()) for o in owned]
    assert max(loads) - min(loads) <= int(lens.max()), f"token loads unbalanced: {loads}"
    for o in owned:  # each rank runs its sequences shortest first
        assert np.all(np.diff(lens[o]) >= 0)
    # rank 0 holds every sequence's output, in input order
    assert np.array_equal(ref["out"], fake_output(np.arange(len(lens)), 3))


def _failing_rank_main(rank: int, world: int, port: int, out_dir: str, leaver: int):
    import datetime

    import torch.distributed as dist
    store = dist.TCPStore("127.0.0.1", port, world, is_master=(rank == 0), timeout=datetime.timedelta(seconds=60))
    from kleinhirn_b200 import synthetic
    lens = synthetic.seq_lengths("mminilm-l12-xlmr", 1000, 11)
    cols = 2
    mem = dp.Membership(store, rank, world, timeout_s=2.0)
    results = {}
    for step in range(3):
        if rank == leaver and step == 1:
            return  # leaves between steps: nothing in flight, no announcement for step 1
        members = mem.join(step)
        mine = dp.reshard(lens, members, rank)
        out = dp.store_gather(store, step, rank, members, mine, fake_output(mine, cols), cols, len(lens))
        if rank == 0:
            results[step] = (members, out)
    if rank == 0:
        np.savez(os.path.join(out_dir, "coordinator.npz"),
                 **{f"members{s}": np.array(m) for s, (m, _) in results.items()},
                 **{f"out{s}": o for s, (_, o) in results.items()}, lens=lens)
    store.set(f"done/{rank}", b"1")
    if rank == 0:  # the store lives in rank 0's process: keep it up until the survivors are done
        import time
        for r in range(world):
            if r == leaver:
                continue
            while not store.check([f"done/{r}"]):
                time.sleep(0.01)


def test_rank_that_leaves_between_steps_is_resharded(tmp_path):
    world, leaver = 3, 2
    mp.start_processes(_failing_rank_main, args=(world, _free_port(), str(tmp_path), leaver), nprocs=world,
                       start_method="spawn", join=True)
    d = np.load(tmp_path / "coordinator.npz")
    n = len(d["lens"])
    want = fake_output(np.arange(n), 2)
    assert list(d["members0"]) == [0, 1, 2]
    assert list(d["members1"]) == [0, 1] and list(d["members2"]) == [0, 1]
    for s in range(3):  # every step, before and after the loss, has every sequence's output
        assert np.array_equal(d[f"out{s}"], want), f"step {s}"
    # after the loss the two survivors share all sequences, balanced
    lens = d["lens"]
    a, b = dp.reshard(lens, [0, 1], 0), dp.reshard(lens, [0, 1], 1)
    assert np.array_equal(np.sort(np.concatenate([a, b])), np.arange(n))
    assert abs(int(lens[a].sum()) - int(lens[b].sum())) <= int(lens.max())


def test_shard_single_rank_identity():
    lens = np.array([5, 3, 9, 1], dtype=np.int64)
    mine = dp.shard_sequences(lens, 1, 0)
    assert sorted(mine.tolist()) == [0, 1, 2, 3]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_chunks_are_even_and_bounded(world):
    """Each rank's rows go in even bulk chunks of at most 1,048,576 (+ one bucket of room for the
    sequence that does not fit exactly): the full C5 step on 1 GPU, and its shares on 2, 4, 8."""
    from kleinhirn_b200 import synthetic
    lens = synthetic.seq_lengths("mminilm-l12-xlmr", 65536, 1234)
    for rank in range(world):
        mine = dp.shard_sequences(lens, world, rank)
        rows = int(lens[mine].sum())
        chunk = dp.chunk_size(rows, 0)
        n = -(-rows // chunk)
        assert chunk <= 1048576 + 512
        # greedy packing of whole sequences fills the chunks: no short extra one
        filled, count = 0, 1
        for ln in lens[mine]:
            if filled + ln > chunk:
                count, filled = count + 1, 0
            filled += int(ln)
        assert count == n, (rows, chunk, count, n)
    assert dp.chunk_size(3960, 0) >= 3960
    assert dp.chunk_size(10, 777) == 777


FWD_CFG = {"model_type": "bert", "hidden_size": 64, "num_hidden_layers": 2, "num_attention_heads": 2,
           "intermediate_size": 128, "hidden_act": "gelu", "vocab_size": 120, "max_position_embeddings": 66,
           "type_vocab_size": 2, "layer_norm_eps": 1e-12, "num_labels": 3}


def _fwd_inputs():
    rng = np.random.default_rng(21)
    lens = rng.integers(3, 60, 11)
    return [list(rng.integers(3, 120, int(n))) for n in lens]


def _forward_rank_main(rank: int, world: int, port: int, out_dir: str):
    import datetime

    import torch.distributed as dist
    from harness import Model, oracle_forward
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        m = Model(FWD_CFG, {"task": "sequence-classification"}, seed=4, f16=False)
        ids = _fwd_inputs()
        lens = np.array([len(x) for x in ids])
        shards = [dp.shard_sequences(lens, world, r) for r in range(world)]
        mine = shards[rank]
        out_mine = oracle_forward(m, [ids[i] for i in mine], 64, threads=1)
        g = dp.OutputGather(dist, None, rank, shards, m.cols)
        g.local.numpy()[: len(mine) * m.cols] = np.asarray(out_mine, dtype=np.float32).ravel()
        out = g.gather()
        np.save(os.path.join(out_dir, f"fwd{rank}.npy"), out if out is not None else np.zeros(0))
    finally:
        dist.destroy_process_group()


def test_two_rank_forward_equals_one_process(tmp_path):
    """The sharded forward (each rank runs its own sequences, rank 0 gathers them in input
    order) gives the same outputs as one process running every sequence: the path has no
    collective, so each sequence's result does not depend on the rank that ran it."""
    from harness import Model, oracle_forward
    world = 2
    mp.start_processes(_forward_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    m = Model(FWD_CFG, {"task": "sequence-classification"}, seed=4, f16=False)
    want = np.asarray(oracle_forward(m, _fwd_inputs(), 64, threads=1), dtype=np.float32)
    got = np.load(tmp_path / "fwd0.npy").reshape(want.shape)
    assert np.array_equal(got, want)
