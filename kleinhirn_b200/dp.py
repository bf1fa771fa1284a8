"""Data parallelism over independent sequences: one process per GPU, each with a full weight
replica, no collective on the data path.

This is the multi-GPU form of ``EncoderModel.runIdsBatch`` (src/encoder.ts:461-474: sort the
inputs by length, run them in chunks, put the results back in input order):

- ``shard_sequences``: which sequences a rank runs; longest first onto the least-loaded rank by
  token count, so the ranks finish together; each rank packs its share shortest first.
- ``chunk_size``: packed rows per bulk chunk of a rank.
- ``OutputGather``: the host gather of every rank's outputs into input order on rank 0 (over a
  CPU process group: gloo), the only communication of a step.
- ``Membership`` and ``reshard``: failure handling between steps. Before a step every rank
  announces itself on the job's key-value store; rank 0 (the coordinator, which also holds the
  gathered outputs) waits a bounded time for the announcements and publishes the step's members;
  a rank that did not announce in time is out, and the survivors re-shard its sequences among
  themselves. ``store_gather`` moves outputs through the store, so a step after a loss does not
  depend on a process group that still counts the lost rank.

Failures are made and detected on the host: a rank that exits, never joins, or raises. A rank
leaves only between steps, with none of its kernels in flight.
"""
from __future__ import annotations

import time

import numpy as np


def shard_sequences(lens: np.ndarray, world: int, rank: int) -> np.ndarray:
    """Indices of the sequences rank `rank` of `world` runs, shortest first; deterministic, so
    every rank computes every rank's share without communication."""
    lens = np.asarray(lens)
    order = np.argsort(-lens, kind="stable")
    load = np.zeros(world, dtype=np.int64)
    owner = np.empty(len(lens), dtype=np.int64)
    for i in order:
        r = int(np.argmin(load))
        owner[i] = r
        load[r] += int(lens[i])
    mine = np.nonzero(owner == rank)[0]
    return mine[np.argsort(lens[mine], kind="stable")]


def chunk_size(tokens: int, requested: int = 0, bucket: int = 512, max_rows: int = 1048576) -> int:
    """Packed rows per bulk chunk: as requested, or the rank's rows in even chunks of at most
    `max_rows` (long launches keep the tail waves of the GEMMs small; even chunks avoid a short
    last one), plus one bucket of room for the sequence that does not fit exactly."""
    if requested > 0:
        return requested
    n = max(1, -(-tokens // max_rows))
    return max(bucket, -(-tokens // n) + bucket)


class OutputGather:
    """Gathers every rank's outputs (rows of `cols` floats, its shard in shard order) into one
    array in input order on rank 0, through a CPU process group. Buffers are made once: `local`
    is the rank's padded output buffer (write the shard's rows to its front)."""

    def __init__(self, dist, group, rank: int, shards: list[np.ndarray], cols: int, pin: bool = False):
        import torch
        self.dist, self.group, self.rank, self.shards, self.cols = dist, group, rank, shards, cols
        n = max(len(s) for s in shards)
        self.local = torch.zeros(n * cols, dtype=torch.float32, pin_memory=pin)
        self.parts = [torch.zeros(n * cols, dtype=torch.float32) for _ in shards] if rank == 0 else None
        self.out = np.zeros((sum(len(s) for s in shards), cols), dtype=np.float32) if rank == 0 else None

    def gather(self) -> np.ndarray | None:
        """Rank 0: the outputs of every sequence in input order; other ranks: None."""
        if self.dist is None:
            s = self.shards[0]
            self.out[s] = self.local.numpy()[:len(s) * self.cols].reshape(-1, self.cols)
            return self.out
        self.dist.gather(self.local, self.parts if self.rank == 0 else None, dst=0, group=self.group)
        if self.rank != 0:
            return None
        for r, s in enumerate(self.shards):
            self.out[s] = self.parts[r].numpy()[:len(s) * self.cols].reshape(-1, self.cols)
        return self.out


class Membership:
    """Which ranks take part in each step, decided by rank 0 on the job's store (a
    torch.distributed Store: TCPStore, FileStore). Every rank calls ``join(step)`` before the
    step; rank 0 waits up to `timeout_s` for the others' announcements and publishes the members;
    the others wait for that list. A rank missing from it is out for good: it raises
    ``LeftJob``. Rank 0 is the coordinator: if it is lost the job ends."""

    class LeftJob(RuntimeError):
        pass

    def __init__(self, store, rank: int, world: int, timeout_s: float = 5.0, poll_s: float = 0.01):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.poll_s = timeout_s, poll_s
        self.members = list(range(world))

    def _has(self, key: str) -> bool:
        return bool(self.store.check([key]))

    def join(self, step: int) -> list[int]:
        self.store.set(f"dp/alive/{step}/{self.rank}", b"1")
        if self.rank == 0:
            deadline = time.monotonic() + self.timeout_s
            pending = [r for r in self.members if r != 0]
            while pending and time.monotonic() < deadline:
                pending = [r for r in pending if not self._has(f"dp/alive/{step}/{r}")]
                if pending:
                    time.sleep(self.poll_s)
            members = [r for r in self.members if r not in pending]
            self.store.set(f"dp/members/{step}", ",".join(map(str, members)).encode())
        else:
            key = f"dp/members/{step}"
            deadline = time.monotonic() + max(60.0, 4 * self.timeout_s)
            while not self._has(key):
                if time.monotonic() > deadline:
                    raise TimeoutError(f"rank {self.rank}: no member list for step {step} (coordinator lost)")
                time.sleep(self.poll_s)
            members = [int(x) for x in self.store.get(key).decode().split(",") if x]
        self.members = members
        if self.rank not in members:
            raise Membership.LeftJob(f"rank {self.rank} is not a member of step {step}")
        return members


def reshard(lens: np.ndarray, members: list[int], rank: int) -> np.ndarray:
    """This rank's sequences when only `members` (sorted rank ids) take part: the sequences of the
    whole job shared among the members as shard_sequences shares them among that many ranks."""
    slot = members.index(rank)
    return shard_sequences(lens, len(members), slot)


def store_gather(store, step: int, rank: int, members: list[int], idx: np.ndarray, out: np.ndarray, cols: int,
                 total: int, timeout_s: float = 60.0, poll_s: float = 0.01) -> np.ndarray | None:
    """Outputs (rows of `cols` floats) of the step's members into input order on rank 0, through
    the store: each member publishes its sequence indices and output rows; rank 0 assembles them
    (rows nobody sent stay NaN); None on the other ranks."""
    idx = np.asarray(idx, dtype=np.int64)
    out = np.ascontiguousarray(out, dtype=np.float32).reshape(len(idx), cols)
    if rank != 0:
        store.set(f"dp/out/{step}/{rank}", idx.tobytes() + out.tobytes())
        return None
    res = np.full((total, cols), np.nan, dtype=np.float32)
    res[idx] = out
    deadline = time.monotonic() + timeout_s
    for r in members:
        if r == 0:
            continue
        key = f"dp/out/{step}/{r}"
        while not store.check([key]):
            if time.monotonic() > deadline:
                raise TimeoutError(f"no outputs of rank {r} for step {step}")
            time.sleep(poll_s)
        raw = store.get(key)
        n = len(raw) // (8 + 4 * cols)
        res[np.frombuffer(raw[:8 * n], dtype=np.int64)] = np.frombuffer(raw[8 * n:], dtype=np.float32).reshape(n, cols)
    return res
