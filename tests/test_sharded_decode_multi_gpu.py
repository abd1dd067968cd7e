"""Sharded greedy decode over two GPUs: the per-step NCCL token gather and a rank failure.

Two spawned ranks, one GPU each, NCCL with NVLS off.  Rank r decodes the batch
positions i % 2 == r of a four-row batch of the reduced model
(``ShardedGreedyDecoder`` over ``DecoderStepGraph``) and gathers every row's
greedy token each step.

* agree: on both ranks every gathered step equals the one-GPU greedy decode of
  the whole batch, which each rank also runs on its own GPU.
* fail: rank 1 stops between steps (its kernels finished, no collective in
  flight), marks the run failed in the store and leaves; rank 0 must raise at
  its next step, before it enters the gather, naming rank 1 and the error.

Skipped with fewer than two GPUs.  The failure is made on the host; no GPU is
faulted.
"""

from __future__ import annotations

import multiprocessing as mp
import os
import socket
import time
from datetime import timedelta

import pytest

pytestmark = pytest.mark.gpu

WORLD = 2
LENGTHS = (1, 16, 49, 70)
STEPS = 5
FAIL_AFTER = 2  # rank 1 leaves after this many steps


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(scenario: str, rank: int, port: int, queue) -> None:
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch
    import torch.distributed as dist
    from dataclasses import replace

    from pagedcore_b200.decoder import BatchedDecoder, prefill_paged
    from pagedcore_b200.engine_types import KVReservation, RequestId
    from pagedcore_b200.graph import DecoderStepGraph
    from pagedcore_b200.kv_cache import KVAllocator
    from pagedcore_b200.sharding import ShardedGreedyDecoder, StepExchange, shard
    from pagedcore_b200.weights import random_weights

    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    store = dist.TCPStore("127.0.0.1", port, WORLD, rank == 0, timeout=timedelta(seconds=60))
    dist.init_process_group("nccl", store=store, rank=rank, world_size=WORLD, timeout=timedelta(seconds=60),
                            device_id=device)
    try:
        small = random_weights(5, device, layers=2, vocab=31, intermediate=32)
        weights = replace(small, layers=small.layers * 11)
        engine = BatchedDecoder(weights)
        batch = tuple(RequestId(f"row{i}") for i in range(len(LENGTHS)))

        def prefilled(requests):
            lengths = [LENGTHS[batch.index(r)] for r in requests]
            blocks = sum(-(-(n + STEPS + 1) // 16) for n in lengths) + 2
            pool = torch.full((22, 2, blocks, 16, 4, 64), torch.nan, dtype=torch.float16, device=device)
            allocator = KVAllocator(pool)
            for request, length in zip(requests, lengths, strict=True):
                allocator.create(KVReservation(request, -(-(length + STEPS + 1) // 16)))
                prompt = ((torch.arange(length) * 7 + length) % 31)[None].to(device)
                prefill_paged(prompt, weights, allocator, request)
            return allocator

        cache = prefilled(shard(batch, rank, WORLD))
        sharded = ShardedGreedyDecoder(engine, cache, batch, StepExchange(store=store, wait=timedelta(seconds=30)))
        whole = prefilled(batch)
        plain = DecoderStepGraph(engine, whole, rows=len(batch))
        first = torch.tensor([[3 + i] for i in range(len(batch))], dtype=torch.int64, device=device)
        local = first[rank::WORLD].contiguous()
        expected = first
        for step in range(STEPS):
            if scenario == "fail" and rank == 1 and step == FAIL_AFTER:
                torch.cuda.synchronize(device)  # nothing of this rank in flight
                error = ValueError("injected failure between steps")
                sharded.exchange.fail(error)
                queue.put((rank, ("failed", step)))
                return
            start = time.monotonic()
            try:
                local, gathered = sharded.step(local)
            except (RuntimeError, TimeoutError) as error:
                queue.put((rank, (type(error).__name__, str(error), step, time.monotonic() - start)))
                return
            expected = plain.step(expected, batch)[:, 0].argmax(dim=-1).view(-1, 1)
            if not torch.equal(gathered, expected.view(-1)) or not torch.equal(local, expected[rank::WORLD]):
                queue.put((rank, ("mismatch", step, gathered.tolist(), expected.view(-1).tolist())))
                return
        torch.cuda.synchronize(device)
        cache.check_device_errors()
        queue.put((rank, ("ok", sharded.exchange.step)))
    finally:
        dist.destroy_process_group()


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
            rank, value = queue.get(timeout=240)
            results[rank] = value
    finally:
        for proc in procs:
            proc.join(timeout=60)
            if proc.is_alive():
                proc.kill()
    return results


def _two_gpus() -> bool:
    import torch

    return torch.cuda.is_available() and torch.cuda.device_count() >= WORLD


@pytest.mark.skipif(not _two_gpus(), reason="needs two GPUs")
def test_two_ranks_gather_the_one_gpu_greedy_tokens_every_step() -> None:
    results = _run("agree")
    for rank in range(WORLD):
        assert results[rank] == ("ok", STEPS), results[rank]


@pytest.mark.skipif(not _two_gpus(), reason="needs two GPUs")
def test_a_rank_that_fails_between_steps_stops_the_other_before_its_next_gather() -> None:
    results = _run("fail")
    assert results[1] == ("failed", FAIL_AFTER)
    kind, message, step, seconds = results[0]
    assert kind == "RuntimeError", results[0]
    assert step == FAIL_AFTER
    assert "rank 1" in message and "injected failure" in message
    assert seconds < 25  # the failure mark ends the wait well inside its 30 s bound
