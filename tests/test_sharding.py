"""Sharding of a decode batch across ranks, on CPU with the gloo backend.

Rank r of N owns batch positions i % N == r; the one per-step exchange is
the gather of next-token ids.  The failure tests make the failure on the host
(a rank that raises, or one that leaves without a word) and check that the
other rank gets an error instead of waiting in a collective.
"""

from __future__ import annotations

import multiprocessing as mp
import socket
import time
from datetime import timedelta

import numpy as np
import pytest

from pagedcore_b200.sharding import shard, shard_positions

WORLD = 2


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shards_cover_every_position_once_in_batch_order(world: int) -> None:
    for count in range(0, 20):
        shares = [shard_positions(count, rank, world) for rank in range(world)]
        joined = np.sort(np.concatenate(shares))
        assert np.array_equal(joined, np.arange(count))
        assert max(len(s) for s in shares) - min(len(s) for s in shares) <= 1
        for share in shares:
            assert np.all(np.diff(share) > 0)
    assert shard(("a", "b", "c", "d", "e"), 1, 2) == ("b", "d")


def test_shard_rejects_a_rank_outside_the_world() -> None:
    with pytest.raises(ValueError, match="rank"):
        shard_positions(4, 2, 2)


# -- multi-process (spawned ranks, gloo) ----------------------------------------
def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(scenario: str, rank: int, port: int, queue) -> None:
    import torch
    import torch.distributed as dist

    from pagedcore_b200.sharding import StepExchange, shard_positions

    store = dist.TCPStore("127.0.0.1", port, WORLD, rank == 0, timeout=timedelta(seconds=30))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=WORLD, timeout=timedelta(seconds=20))
    exchange = StepExchange(store=store, wait=timedelta(seconds=4 if scenario == "vanish" else 20),
                            check_every=3 if scenario == "greedy" else 1)
    count = 7
    try:
        if scenario == "greedy":
            queue.put((rank, ("ok", _greedy_steps(exchange, count))))
            return
        # Step 0: every rank contributes ids for its own rows (id = 100 * position).
        mine = torch.from_numpy(shard_positions(count, rank, WORLD) * 100)
        first = exchange.gather_tokens(mine, count).tolist()
        if scenario == "gather":
            second = exchange.gather_tokens(mine + 1, count).tolist()
            queue.put((rank, ("ok", first, second)))
        elif rank == 1:
            if scenario == "raise":
                try:
                    raise ValueError("injected failure in the step")
                except ValueError as error:
                    exchange.fail(error)
                    queue.put((rank, ("failed", str(error))))
            else:  # "vanish": leave without marking anything
                queue.put((rank, ("left",)))
        else:
            start = time.monotonic()
            try:
                exchange.gather_tokens(mine, count)
                queue.put((rank, ("no error",)))
            except (RuntimeError, TimeoutError) as error:
                queue.put((rank, (type(error).__name__, str(error), time.monotonic() - start)))
    finally:
        dist.destroy_process_group()


class _FakeStepGraph:
    """DecoderStepGraph's step contract on the CPU: logits [B, 1, V] whose
    greedy choice for request ``rNN`` at input id x is (x + NN) % V (ties to
    the lower id, as argmax resolves them)."""

    VOCAB = 50

    def __init__(self) -> None:
        self.calls = []

    def step(self, input_ids, requests):
        import torch

        self.calls.append(tuple(requests))
        logits = torch.zeros((len(requests), 1, self.VOCAB), dtype=torch.float16)
        for row, request in enumerate(requests):
            best = (int(input_ids[row, 0]) + int(request[1:])) % self.VOCAB
            logits[row, 0, best:best + 2] = 1.0  # a tie with the next id: the lower one wins
        return logits


def _greedy_steps(exchange, count: int) -> list:
    import torch

    from pagedcore_b200.sharding import ShardedGreedyDecoder

    requests = tuple(f"r{i}" for i in range(count))
    graph = _FakeStepGraph()
    decoder = ShardedGreedyDecoder(None, None, requests, exchange, graph=graph)
    ids = torch.tensor([[i] for i in range(exchange.rank, count, exchange.world)], dtype=torch.int64)
    history = []
    for _ in range(5):
        ids, gathered = decoder.step(ids)
        history.append(gathered.tolist())
    assert all(call == decoder.requests for call in graph.calls)
    return history


def _run(scenario: str) -> dict:
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(scenario, rank, port, queue)) for rank in range(WORLD)]
    for proc in procs:
        proc.start()
    results = {}
    try:
        for _ in range(WORLD):
            rank, value = queue.get(timeout=90)
            results[rank] = value
    finally:
        for proc in procs:
            proc.join(timeout=30)
            if proc.is_alive():
                proc.kill()
    return results


def test_token_gather_returns_every_row_in_batch_order() -> None:
    results = _run("gather")
    expected = [100 * i for i in range(7)]
    for rank in range(WORLD):
        status, first, second = results[rank]
        assert status == "ok"
        assert first == expected
        assert second == [x + 1 for x in expected]


def test_a_rank_that_fails_is_reported_before_the_next_exchange() -> None:
    results = _run("raise")
    assert results[1][0] == "failed"
    kind, message, seconds = results[0]
    assert kind == "RuntimeError"
    assert "rank 1" in message and "injected failure" in message
    assert seconds < 10  # well inside the 20 s wait bound: the mark ends the wait


def test_a_rank_that_leaves_silently_ends_the_wait_with_a_timeout() -> None:
    results = _run("vanish")
    assert results[1] == ("left",)
    kind, message, seconds = results[0]
    assert kind == "TimeoutError"
    assert "1 of 2 ranks" in message
    assert 3 < seconds < 20


def test_sharded_greedy_decode_gathers_the_whole_batch_every_step() -> None:
    # Each rank decodes only its own rows; every rank sees all rows' tokens, in
    # batch order, after every step (peers checked on every third exchange).
    results = _run("greedy")
    vocab, count = _FakeStepGraph.VOCAB, 7
    ids, expected = list(range(count)), []
    for _ in range(5):
        ids = [(x + i) % vocab for i, x in enumerate(ids)]
        expected.append(ids)
    for rank in range(WORLD):
        status, history = results[rank]
        assert status == "ok"
        assert history == expected
