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
    before an exchange.
    """

    def __init__(
        self,
        group: dist.ProcessGroup | None = None,
        store: dist.Store | None = None,
        wait: timedelta = timedelta(seconds=60),
    ) -> None:
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if store is None:
            store = dist.distributed_c10d._get_default_store()
        self.store = store
        self.wait = wait
        self.step = 0

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
        deadline = time.monotonic() + self.wait.total_seconds()
        while True:
            self.check()
            if self.store.add(key, 0) >= self.world:
                return
            if time.monotonic() > deadline:
                raise TimeoutError(
                    f"decode step {self.step}: only {self.store.add(key, 0)} of {self.world} ranks reached the "
                    f"token exchange within {self.wait.total_seconds():.0f} s"
                )
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
        self._await_peers()
        per_rank = -(-count // self.world)
        padded = torch.full((per_rank,), -1, dtype=torch.int64, device=local.device)
        padded[:owned] = local
        gathered = torch.empty(self.world * per_rank, dtype=torch.int64, device=local.device)
        dist.all_gather_into_tensor(gathered, padded, group=self.group)
        self.step += 1
        # Rank r's j-th id belongs to batch position r + j*world.
        return gathered.view(self.world, per_rank).t().reshape(-1)[:count]
