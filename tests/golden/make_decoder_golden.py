"""Generate the decoder golden fixtures by running PagedCore's decoder on the CPU.

Run from the repository root, with the reference checkout importable:

    PAGEDCORE_REFERENCE=/path/to/PagedCore/src python tests/golden/make_decoder_golden.py

The reference's ``prefill``, ``prefill_paged`` and ``decode_paged``
(src/pagedcore/decoder.py) run unmodified on CPU pools, with weights from
``pagedcore_b200.weights.random_weights`` (drawn on the CPU from a seed, so the
GPU tests rebuild the same bits).  Outputs:

- decoder_small.npz   a reduced model (2 layers repeated 11 times, vocabulary
                      31, MLP width 32; the reference tests' geometry): prefill
                      logits of five prompts, and decode_paged logits of a
                      three-row batch over three steps.
- decoder_cfg3.json   BASELINE config 3: the full TinyLlama shape with N(0, 0.02)
                      weights (norm weights 1.0), a 128-token prompt of random
                      ids, 128 greedy tokens at batch 1 through prefill_paged and
                      decode_paged; per step the top-8 token ids and logits.
"""

from __future__ import annotations

import json
import os
import sys
import time
from dataclasses import replace
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
if not os.environ.get("PAGEDCORE_REFERENCE"):
    raise SystemExit("set PAGEDCORE_REFERENCE to the reference checkout's src directory (the one holding pagedcore/)")
sys.path.insert(0, os.environ["PAGEDCORE_REFERENCE"])

from pagedcore.decoder import decode_paged, prefill, prefill_paged  # noqa: E402  (the reference)
from pagedcore.engine_types import KVReservation, RequestId  # noqa: E402
from pagedcore.kv_cache import KVAllocator  # noqa: E402

from pagedcore_b200.weights import random_weights  # noqa: E402

OUT = Path(__file__).resolve().parent

SMALL_SEED = 5
SMALL_PROMPTS = (1, 15, 16, 17, 49)
SMALL_ROWS = (1, 16, 49)
SMALL_STEPS = 3
CFG3_SEED = 3
CFG3_PROMPT = 128
CFG3_NEW = 128
TOP = 8


def small_weights():
    weights = random_weights(SMALL_SEED, layers=2, vocab=31, intermediate=32)
    return replace(weights, layers=weights.layers * 11)


def small_prompt(tokens: int) -> torch.Tensor:
    return (torch.arange(tokens)[None] + tokens) % 31


def small_step_tokens(step: int, order: tuple[int, ...]) -> torch.Tensor:
    return torch.tensor([[3 + row + step] for row in order])


def cfg3_prompt() -> torch.Tensor:
    generator = torch.Generator().manual_seed(CFG3_SEED * 1000 + 1)
    return torch.randint(0, 32000, (1, CFG3_PROMPT), generator=generator, dtype=torch.int64)


def make_small() -> None:
    weights = small_weights()
    out = {}
    for tokens in SMALL_PROMPTS:
        logits, _ = prefill(small_prompt(tokens), weights)
        out[f"prefill_{tokens}"] = logits[0].float().numpy()
    pool = torch.full((22, 2, 16, 16, 4, 64), torch.nan, dtype=torch.float16)
    allocator = KVAllocator(pool)
    requests = tuple(RequestId(f"row{row}") for row in range(len(SMALL_ROWS)))
    for request, length in zip(requests, SMALL_ROWS, strict=True):
        allocator.create(KVReservation(request, (length + SMALL_STEPS + 15) // 16))
        prefill_paged(small_prompt(length), weights, allocator, request)
    for step in range(SMALL_STEPS):
        order = tuple(range(len(requests))) if step % 2 == 0 else tuple(reversed(range(len(requests))))
        logits = decode_paged(small_step_tokens(step, order), weights, allocator, tuple(requests[r] for r in order))
        out[f"decode_{step}"] = logits[:, 0].float().numpy()
        out[f"decode_{step}_order"] = np.asarray(order)
    np.savez_compressed(OUT / "decoder_small.npz", **out)


def top(logits: torch.Tensor) -> tuple[list[int], list[float]]:
    values, ids = logits.float().topk(TOP)
    return ids.tolist(), values.tolist()


def make_cfg3() -> None:
    start = time.time()
    weights = random_weights(CFG3_SEED)
    prompt = cfg3_prompt()
    pool = torch.full((22, 2, 20, 16, 4, 64), torch.nan, dtype=torch.float16)
    allocator = KVAllocator(pool)
    request = RequestId("cfg3")
    allocator.create(KVReservation(request, (CFG3_PROMPT + CFG3_NEW + 15) // 16))
    logits = prefill_paged(prompt, weights, allocator, request)[0, -1]
    steps = []
    for step in range(CFG3_NEW):
        ids, values = top(logits)
        steps.append({"top_ids": ids, "top_logits": values})
        if step + 1 < CFG3_NEW:
            token = torch.tensor([[ids[0]]], dtype=torch.int64)
            logits = decode_paged(token, weights, allocator, (request,))[0, 0]
    record = {
        "seed": CFG3_SEED,
        "prompt_seed": CFG3_SEED * 1000 + 1,
        "prompt": prompt[0].tolist(),
        "greedy_ids": [s["top_ids"][0] for s in steps],
        "steps": steps,
        "note": "reference prefill_paged + decode_paged on CPU (torch %s), %.0f s" % (torch.__version__,
                                                                                  time.time() - start),
    }
    (OUT / "decoder_cfg3.json").write_text(json.dumps(record))


if __name__ == "__main__":
    torch.set_num_threads(os.cpu_count() or 1)
    make_small()
    make_cfg3()
