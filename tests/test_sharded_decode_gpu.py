"""Sharded greedy decode with its per-step NCCL token gather, on one GPU.

``ShardedGreedyDecoder`` runs a rank's rows through ``DecoderStepGraph``,
takes each row's greedy token on the device and gathers the whole batch's
tokens over NCCL once per step.  On one rank (an NCCL group of one) it must
reproduce, token for token, the one-GPU greedy decode it shards: the same
graph-replayed decoder step followed by argmax.  The multi-rank gather and its
failure handling are covered on CPU with gloo ranks (tests/test_sharding.py).
"""

from __future__ import annotations

import socket
from dataclasses import replace
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist

from pagedcore_b200.decoder import BatchedDecoder, prefill_paged
from pagedcore_b200.engine_types import KVReservation, RequestId
from pagedcore_b200.graph import DecoderStepGraph
from pagedcore_b200.kv_cache import KVAllocator
from pagedcore_b200.sharding import ShardedGreedyDecoder, StepExchange
from pagedcore_b200.weights import random_weights
from tests.conftest import cuda_device

pytestmark = pytest.mark.gpu

LENGTHS = (1, 16, 49, 70)
STEPS = 6


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _prefilled(weights, device) -> tuple[KVAllocator, tuple[RequestId, ...]]:
    blocks = sum(-(-(n + STEPS + 1) // 16) for n in LENGTHS) + 2
    allocator = KVAllocator(torch.full((22, 2, blocks, 16, 4, 64), torch.nan, dtype=torch.float16, device=device))
    requests = tuple(RequestId(f"row{i}") for i in range(len(LENGTHS)))
    for request, length in zip(requests, LENGTHS, strict=True):
        allocator.create(KVReservation(request, -(-(length + STEPS + 1) // 16)))
        prompt = ((torch.arange(length) * 7 + length) % 31)[None].to(device)
        prefill_paged(prompt, weights, allocator, request)
    return allocator, requests


def test_sharded_greedy_decode_on_one_rank_reproduces_the_one_gpu_tokens() -> None:
    device = cuda_device()
    small = random_weights(5, device, layers=2, vocab=31, intermediate=32)
    weights = replace(small, layers=small.layers * 11)
    engine = BatchedDecoder(weights)
    store = dist.TCPStore("127.0.0.1", _free_port(), 1, True, timeout=timedelta(seconds=30))
    dist.init_process_group("nccl", store=store, rank=0, world_size=1, timeout=timedelta(seconds=60),
                            device_id=device)
    try:
        sharded_cache, requests = _prefilled(weights, device)
        plain_cache, _ = _prefilled(weights, device)
        sharded = ShardedGreedyDecoder(engine, sharded_cache, requests, StepExchange(store=store))
        plain = DecoderStepGraph(engine, plain_cache, rows=len(requests))
        ids = torch.tensor([[3 + i] for i in range(len(requests))], dtype=torch.int64, device=device)
        local, expected = ids, ids
        for _ in range(STEPS):
            local, gathered = sharded.step(local)
            expected = plain.step(expected, requests)[:, 0].argmax(dim=-1).view(-1, 1)
            assert torch.equal(gathered, expected.view(-1))
            assert torch.equal(local, expected)
        assert [sharded_cache.cached_length(r) for r in requests] == [n + STEPS for n in LENGTHS]
        assert sharded.exchange.step == STEPS
        sharded_cache.check_device_errors()
    finally:
        dist.destroy_process_group()
