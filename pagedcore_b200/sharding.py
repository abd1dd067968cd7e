"""Sequences across GPUs: one process per GPU, each with its own pool.

Sequences are independent (attention reads only a row's own blocks), so the
KV path shards with no collective on it.  Rank r of N owns the requests at
batch positions i with i % N == r, with its own ``KVAllocator``, pool, block
tables and stream.  The one exchange of a decode step is the gather of every
row's next-token id (int64, a few KB) once the step's logits exist: NCCL on
GPUs, gloo on CPU.

Failure handling is on the host and between steps.  A rank whose step fails
marks the run failed in the process group's key-value store before it exits;
before every exchange each rank announces itself for that step in the store
and waits, bounded, until all ranks have announced themselves or one has
marked a failure.  So a rank that failed is reported to the others as an
error before they enter a collective it will never join, and a rank that
dies without marking anything ends the others' wait with a timeout.
"""

from __future__ import annotations

import time
from collections.abc import Sequence
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

_FAILED = "pagedkv/failed"


def shard_positions(count: int, rank: int, world: int) -> np.ndarray:
    """Batch positions owned by ``rank``: i with i % world == rank, ascending."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must lie in [0, world)")
    if count < 0:
        raise ValueError("count must be non-negative")
    return np.arange(rank, count, world, dtype=np.int64)


def shard(items: Sequence, rank: int, world: int) -> tuple:
    """The rank's share of ``items`` (e.g. request ids), in batch order."""
    return tuple(items[i] for i in shard_positions(len(items), rank, world))


class StepExchange:
    """Per-step exchange of next-token ids between the ranks of a decode.

    ``store`` is the process group's key-value store (the default group's
    when omitted); ``wait`` bounds how long a rank waits for the others
    before an exchange.  The ranks announce themselves in the store before
    every ``check_every``-th exchange (every one by default); a decode loop
    that must not pay a store round trip per step checks less often, and a
    failure is then noticed at the next checked step or by the process
    group's timeout.
    """

    def __init__(
        self,
        group: dist.ProcessGroup | None = None,
        store: dist.Store | None = None,
        wait: timedelta = timedelta(seconds=60),
        check_every: int = 1,
    ) -> None:
        if type(check_every) is not int or check_every < 1:
            raise ValueError("check_every must be a positive integer")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if store is None:
            store = dist.distributed_c10d._get_default_store()
        self.store = store
        self.wait = wait
        self.check_every = check_every
        self.step = 0
        self._buffers: dict = {}

    # -- failure marks ---------------------------------------------------------
    def fail(self, error: BaseException | str) -> None:
        """Mark the run failed (call from the failing rank, before it exits)."""
        self.store.set(_FAILED, f"rank {self.rank}: {error}")

    def check(self) -> None:
        """Raise if any rank has marked the run failed."""
        if self.store.check([_FAILED]):
            raise RuntimeError(f"decode aborted: {self.store.get(_FAILED).decode()}")

    def _await_peers(self) -> None:
        key = f"pagedkv/ready/{self.step}"
        self.store.add(key, 1)
        start = time.monotonic()
        deadline = start + self.wait.total_seconds()
        while True:
            self.check()
            if self.store.add(key, 0) >= self.world:
                return
            now = time.monotonic()
            if now > deadline:
                raise TimeoutError(
                    f"decode step {self.step}: only {self.store.add(key, 0)} of {self.world} ranks reached the "
                    f"token exchange within {self.wait.total_seconds():.0f} s"
                )
            # Ranks reach a step within microseconds of each other in a healthy
            # run: poll back to back for the first 2 ms, then every millisecond.
            if now - start > 0.002:
                time.sleep(0.001)

    # -- the exchange ----------------------------------------------------------
    def gather_tokens(self, local: torch.Tensor, count: int) -> torch.Tensor:
        """Every row's token id, in batch order, from each rank's own rows.

        ``local`` holds this rank's ids (int64, one per owned position, as
        :func:`shard_positions` orders them); returns int64 ``[count]``.
        """
        if local.dtype != torch.int64 or local.dim() != 1:
            raise ValueError("token ids must be a 1-D int64 tensor")
        owned = len(shard_positions(count, self.rank, self.world))
        if local.numel() != owned:
            raise ValueError(f"rank {self.rank} owns {owned} of {count} rows, got {local.numel()} ids")
        if self.step % self.check_every == 0:
            self._await_peers()
        per_rank = -(-count // self.world)
        # The collective's buffers are kept from step to step (same addresses
        # every step), each step's result is returned as a copy.
        key = (count, local.device)
        if self._buffers.get("key") != key:
            self._buffers = {
                "key": key,
                "padded": torch.full((per_rank,), -1, dtype=torch.int64, device=local.device),
                "gathered": torch.empty(self.world * per_rank, dtype=torch.int64, device=local.device),
            }
        padded, gathered = self._buffers["padded"], self._buffers["gathered"]
        padded[:owned] = local
        dist.all_gather_into_tensor(gathered, padded, group=self.group)
        self.step += 1
        # Rank r's j-th id belongs to batch position r + j*world.
        return gathered.view(self.world, per_rank).t().reshape(-1)[:count].clone()


class ShardedGreedyDecoder:
    """Greedy decode of one batch spread over the ranks, one token per row per step.

    Rank r owns batch positions i % N == r (``shard``): their requests live in
    this rank's own ``KVAllocator`` (pool, ledger, stream) and its decoder
    step is a ``graph.DecoderStepGraph`` over them.  Each step picks every
    owned row's next token on the device (the first maximal logit, the
    reference's greedy choice, decoder.py:87-100) and the ranks then gather
    the ids of the whole batch once (``StepExchange.gather_tokens``, NCCL on
    GPUs): the only data that crosses GPUs.  A rank's own ids feed its next
    step without leaving the device.
    """

    def __init__(self, decoder, allocator, requests: Sequence, exchange: StepExchange | None = None, *,
                 graph=None) -> None:
        self.exchange = exchange
        world = 1 if exchange is None else exchange.world
        rank = 0 if exchange is None else exchange.rank
        self.count = len(requests)
        if self.count < world:
            raise ValueError("every rank needs at least one row of the batch")
        self.requests = shard(requests, rank, world)
        if graph is None:  # anything with DecoderStepGraph's step(ids, requests) -> logits [B, 1, V]
            from pagedcore_b200.graph import DecoderStepGraph

            graph = DecoderStepGraph(decoder, allocator, rows=len(self.requests))
        self.graph = graph

    @torch.inference_mode()
    def step(self, input_ids: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """One step for this rank's rows (int64 [owned, 1] ids on its device).

        Returns (this rank's next ids int64 [owned, 1], the whole batch's next
        ids int64 [count] in batch order); both stay on the device.
        """
        logits = self.graph.step(input_ids, self.requests)
        local = logits[:, 0].argmax(dim=-1)
        gathered = local if self.exchange is None else self.exchange.gather_tokens(local, self.count)
        return local.view(-1, 1), gathered
