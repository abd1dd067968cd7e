"""BASELINE config 5 on one GPU: sustained decode under allocator churn.

Per GPU (the box's 1024 sequences over 8 GPUs): 128 sequences at full
2048-token context, a pool of 90 % of the blocks they need (0.9 * 128 * 128),
so admission is credit-bound.  Every request reserves its full context
(prompt + max_new = 2048) and finishes at a seeded random step (EOS); its
credits admit the next queued request, a 512-token prompt.  The worker loop is
``scheduler.Worker`` (strict FIFO, one prefill per iteration, one decode step
for every active sequence); the prefill is a paged write of the prompt's K/V
with RoPE (synthetic K/V: the KV path, not the dense model), the decode step
the 22 fused decode-layer launches of ``DecodeStepGraph``, one CUDA graph
replay whatever the active batch.  Reported: decode tokens/s over the
timed iterations, the attention's algorithmic bytes per second, admissions
and completions.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from pagedcore_b200 import workloads
from pagedcore_b200.engine_types import RequestId
from pagedcore_b200.graph import DecodeStepGraph
from pagedcore_b200.kv_cache import KVAllocator
from pagedcore_b200.scheduler import EOS_TOKEN, Request, Worker, required_blocks

ROWS = 128
CONTEXT = 2048
NEW_PROMPT = 512
POOL_SHARE = 0.9
LAYERS = 22


@dataclass
class StressResult:
    iterations: int
    seconds: float
    decode_tokens: int
    prefill_tokens: int
    admitted: int
    completed: int
    attention_bytes: float
    active_mean: float

    @property
    def tokens_per_second(self) -> float:
        return self.decode_tokens / self.seconds

    @property
    def attention_gbs(self) -> float:
        return self.attention_bytes / self.seconds / 1e9


class StressRun:
    """The config 5 workload on one device, driven through ``Worker``."""

    def __init__(self, device: torch.device, seed: int = 5, rows: int = ROWS, context: int = CONTEXT,
                 new_prompt: int = NEW_PROMPT, balance: str = "measured") -> None:
        self.device = device
        self.rng = workloads.rng(seed, 50)
        self.context = context
        self.new_prompt = new_prompt
        blocks = int(POOL_SHARE * rows * (context // 16))
        pool = torch.empty((LAYERS, 2, blocks, 16, 4, 64), dtype=torch.float16, device=device)
        self.allocator = KVAllocator(pool, validation="incremental", balance=balance)
        generator = torch.Generator(device=device).manual_seed(seed)
        self.kv = torch.randn(LAYERS, context, 4, 64, dtype=torch.float16, device=device, generator=generator)
        self.q = torch.randn(LAYERS, rows, 32, 64, dtype=torch.float16, device=device, generator=generator)
        self.k = torch.randn(LAYERS, rows, 4, 64, dtype=torch.float16, device=device, generator=generator)
        self.out = torch.empty(LAYERS, rows, 32, 64, dtype=torch.float16, device=device)
        self.graph = DecodeStepGraph(self.allocator, rows=rows)
        self.finish_at: dict[RequestId, int] = {}
        self.lengths: dict[RequestId, int] = {}
        self.next_id = 0
        self.decode_tokens = 0
        self.prefill_tokens = 0
        self.attention_bytes = 0.0
        self.active_sum = 0
        self.worker = Worker(self.allocator, self._prefill, self._decode, max_active=rows)
        # The initial sequences: long prompts, each finishing at a seeded step.
        for prompt in self.rng.integers(1, context - context // 4, size=rows):
            self.submit(int(prompt))

    def submit(self, prompt: int) -> None:
        request_id = RequestId(f"r{self.next_id}")
        self.next_id += 1
        max_new = self.context - prompt
        self.finish_at[request_id] = int(self.rng.integers(1, max_new + 1))
        self.worker.submit(Request(request_id, prompt, max_new))

    def _prefill(self, request: Request) -> int:
        length = request.prompt_tokens
        self.allocator.append(request.request_id, self.kv[:, :length], self.kv[:, :length], rotate=True)
        self.lengths[request.request_id] = length
        self.prefill_tokens += length
        return EOS_TOKEN if self.finish_at[request.request_id] <= 1 else 7

    def _decode(self, batch) -> list[int]:
        count = len(batch)
        ids = tuple(request.request_id for request in batch)
        self.graph.step(self.q, self.k, self.k, self.out, ids)
        tokens = []
        for request in batch:
            length = self.lengths[request.request_id] = self.lengths[request.request_id] + 1
            # K/V streamed + table entries + Q in and out + new token in and written, per layer.
            self.attention_bytes += LAYERS * (1024 * length + 4 * -(-length // 16) + 2 * 4096 + 2 * 1024 + 8)
            tokens.append(EOS_TOKEN if len(request.output) + 1 >= self.finish_at[request.request_id] else 7)
        self.decode_tokens += count
        self.active_sum += count
        return tokens

    def iterate(self) -> None:
        """One worker iteration; finished requests are replaced by 512-token prompts."""
        completed = len(self.worker.completed)
        self.worker.iterate()
        for _ in range(len(self.worker.completed) - completed):
            self.submit(self.new_prompt)

    def warm(self, iterations: int) -> None:
        """Untimed iterations, then wait for the device."""
        for _ in range(iterations):
            self.iterate()
        torch.cuda.synchronize(self.device)

    def run(self, warmup: int, iterations: int) -> StressResult:
        self.warm(warmup)
        base = (self.decode_tokens, self.prefill_tokens, self.attention_bytes, self.active_sum,
                self.next_id - len(self.worker.pending), len(self.worker.completed))
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        stream = torch.cuda.current_stream(self.device)
        start.record(stream)
        for _ in range(iterations):
            self.iterate()
        end.record(stream)
        torch.cuda.synchronize(self.device)
        self.allocator.check_device_errors()
        return StressResult(
            iterations=iterations,
            seconds=start.elapsed_time(end) / 1000.0,
            decode_tokens=self.decode_tokens - base[0],
            prefill_tokens=self.prefill_tokens - base[1],
            admitted=self.next_id - len(self.worker.pending) - base[4],
            completed=len(self.worker.completed) - base[5],
            attention_bytes=self.attention_bytes - base[2],
            active_mean=(self.active_sum - base[3]) / iterations,
        )


def pool_blocks(rows: int = ROWS) -> int:
    return int(POOL_SHARE * rows * (CONTEXT // 16))


def full_context_credits() -> int:
    return required_blocks(NEW_PROMPT, CONTEXT - NEW_PROMPT)

