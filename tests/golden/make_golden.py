"""Generate the golden fixtures by running PagedCore's own code on the CPU.

Run from the repository root, with the reference checkout importable:

    PAGEDCORE_REFERENCE=/path/to/PagedCore/src python tests/golden/make_golden.py

It imports the reference's ``pagedcore.kv_cache``, ``pagedcore.attention``
and ``pagedcore.dense`` unmodified and feeds them the seeded workloads of
``pagedcore_b200.workloads``.  Outputs (all small):

- rope_table.npz      FP16 cos/sin [2, 2048, 32] read back from the
                      reference's apply_rope (dense.py:33-61).
- attention_cfg1.npz  config 1: the reference's paged_attention outputs at
                      layers 0 and 21, block tables, and FP64 dense outputs.
- append_cfg2.json    config 2: tables, lengths, capacity and SHA-256 of the
                      whole pool after churn, after the prompt writes and after
                      the one-token appends (reference KVAllocator + apply_rope).
- append_small.npz    a small append case: SHA-256 of its whole pool, and
                      its layers 0 and 21 in full.

The fixtures are inputs to tests only; nothing at run time reads the
reference.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
if not os.environ.get("PAGEDCORE_REFERENCE"):
    raise SystemExit("set PAGEDCORE_REFERENCE to the reference checkout's src directory (the one holding pagedcore/)")
sys.path.insert(0, os.environ["PAGEDCORE_REFERENCE"])

from pagedcore.attention import paged_attention  # noqa: E402  (the reference)
from pagedcore.dense import apply_rope  # noqa: E402
from pagedcore.engine_types import KVReservation, RequestId  # noqa: E402
from pagedcore.kv_cache import KVAllocator  # noqa: E402

from pagedcore_b200 import workloads  # noqa: E402

OUT = Path(__file__).resolve().parent
SMALL_CASE = dict(seed=7, num_blocks=48, churn_count=200, prompt_count=3, decode_rows=8, max_prompt=64,
                  churn_tokens=15)


def sha256(array: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(array).view(np.uint8)).hexdigest()


def capacity(allocator: KVAllocator) -> list[int]:
    c = allocator.capacity()
    return [c.total_blocks, c.free_blocks, c.owned_blocks, c.reserved_blocks, c.active_slots,
            c.live_cached_token_slots]


def rope_table() -> None:
    key = torch.zeros(1, 1, 2048, 64, dtype=torch.float16)
    key[..., :32] = 1
    query = torch.zeros(1, 1, 2048, 64, dtype=torch.float16)
    _, rotated = apply_rope(query, key, torch.arange(2048)[None])
    cos = rotated[0, 0, :, :32].numpy()
    sin = rotated[0, 0, :, 32:].numpy()
    np.savez_compressed(OUT / "rope_table.npz", table=np.stack((cos, sin)))


def rotate_reference(key: np.ndarray, positions: np.ndarray) -> torch.Tensor:
    """apply_rope on K [22, T, 4, 64] at positions [T] (all layers at once)."""
    k = torch.from_numpy(key).transpose(1, 2)  # [22, 4, T, 64]
    q = torch.zeros(k.shape[0], 1, k.shape[2], 64, dtype=torch.float16)
    _, rotated = apply_rope(q, k, torch.from_numpy(positions.astype(np.int64))[None])
    return rotated.transpose(1, 2).contiguous()


def attention_cfg1() -> None:
    case = workloads.attention_case()
    pool = torch.full((22, 2, case.num_blocks, 16, 4, 64), torch.nan, dtype=torch.float16)
    allocator = KVAllocator(pool)
    # Seeded fragmentation: the reference treats the free list as a set.
    allocator._free_blocks = [int(b) for b in case.free_order]
    requests = [RequestId(f"row{i}") for i in range(len(case.lengths))]
    for request, length, key, value in zip(requests, case.lengths, case.keys, case.values, strict=True):
        allocator.create(KVReservation(request, workloads.blocks_for(length)))
        allocator.append(request, torch.from_numpy(key), torch.from_numpy(value))
    tables = [list(allocator.block_table(r)) for r in requests]
    outputs = {}
    dense = {}
    for layer in (0, 21):
        outs = []
        dens = []
        for row, request in enumerate(requests):
            q = torch.from_numpy(case.query[row]).reshape(1, 32, 1, 64)
            outs.append(paged_attention(q, allocator, request, layer_index=layer).reshape(32, 64).numpy())
            k = case.keys[row][layer].astype(np.float64)
            v = case.values[row][layer].astype(np.float64)
            heads = []
            for h in range(32):
                s = case.query[row][h].astype(np.float64) @ k[:, h // 8].T / 8.0
                w = np.exp(s - s.max())
                w /= w.sum()
                heads.append(w @ v[:, h // 8])
            dens.append(np.stack(heads).astype(np.float16))
        outputs[layer] = np.stack(outs)
        dense[layer] = np.stack(dens)
    flat = np.concatenate([np.asarray(t, dtype=np.int32) for t in tables])
    np.savez_compressed(
        OUT / "attention_cfg1.npz",
        lengths=np.asarray(case.lengths, dtype=np.int32),
        tables=flat,
        out_layer0=outputs[0],
        out_layer21=outputs[21],
        dense_layer0=dense[0],
        dense_layer21=dense[21],
    )


def replay_cfg2(case: workloads.AppendCase) -> dict:
    pool = torch.full((22, 2, case.num_blocks, 16, 4, 64), torch.nan, dtype=torch.float16)
    allocator = KVAllocator(pool)
    result: dict = {}
    t0 = time.time()
    for index, op in enumerate(case.churn):
        rid = RequestId(str(op.request))
        if op.kind == "create":
            allocator.create(KVReservation(rid, op.credits))
            key, value = workloads.churn_fill(index, op.tokens)
            allocator.append(rid, torch.from_numpy(key), torch.from_numpy(value))
        else:
            allocator.release_all(rid)
    print(f"churn replayed in {time.time() - t0:.1f}s", file=sys.stderr)
    result["after_churn"] = {
        "capacity": capacity(allocator),
        "free_list": [int(b) for b in allocator._free_blocks],
        "pool_sha256": sha256(pool.numpy()),
    }
    for prompt in case.prompts:
        rid = RequestId(str(prompt.request))
        allocator.create(KVReservation(rid, prompt.credits))
        tokens = prompt.key.shape[1]
        rotated = rotate_reference(prompt.key, np.arange(tokens))
        allocator.append(rid, rotated, torch.from_numpy(prompt.value))
    result["after_prompts"] = {
        "capacity": capacity(allocator),
        "tables": {str(p.request): list(allocator.block_table(RequestId(str(p.request)))) for p in case.prompts},
        "pool_sha256": sha256(pool.numpy()),
    }
    requests = tuple(RequestId(str(r)) for r in case.decode.requests)
    positions = np.array([allocator.cached_length(r) for r in requests], dtype=np.int64)
    with allocator.append_decode(requests):
        for layer in range(22):
            k = torch.from_numpy(case.decode.key[layer])[:, :, None]  # [B, 4, 1, 64]
            q = torch.zeros(len(requests), 1, 1, 64, dtype=torch.float16)
            _, rotated = apply_rope(q, k, torch.from_numpy(positions)[:, None])
            for row, request in enumerate(requests):
                allocator.write_decode_layer(
                    request, layer, rotated[row, :, 0], torch.from_numpy(case.decode.value[layer, row])
                )
    result["after_decode"] = {
        "capacity": capacity(allocator),
        "tables": {str(r): list(allocator.block_table(r)) for r in requests},
        "lengths": {str(r): allocator.cached_length(r) for r in requests},
        "free_list_sha256": hashlib.sha256(np.asarray(allocator._free_blocks, dtype=np.int64)).hexdigest(),
        "pool_sha256": sha256(pool.numpy()),
    }
    return result


def append_cfg2() -> None:
    case = workloads.append_case()
    result = replay_cfg2(case)
    result["workload"] = {"seed": 2, "num_blocks": case.num_blocks, "churn": len(case.churn),
                          "prompts": [p.key.shape[1] for p in case.prompts], "decode_rows": len(case.decode.requests)}
    (OUT / "append_cfg2.json").write_text(json.dumps(result, indent=1, sort_keys=True))


def append_small() -> None:
    case = workloads.append_case(**SMALL_CASE)
    pool = torch.full((22, 2, case.num_blocks, 16, 4, 64), torch.nan, dtype=torch.float16)
    allocator = KVAllocator(pool)
    for index, op in enumerate(case.churn):
        rid = RequestId(str(op.request))
        if op.kind == "create":
            allocator.create(KVReservation(rid, op.credits))
            key, value = workloads.churn_fill(index, op.tokens)
            allocator.append(rid, torch.from_numpy(key), torch.from_numpy(value))
        else:
            allocator.release_all(rid)
    for prompt in case.prompts:
        rid = RequestId(str(prompt.request))
        allocator.create(KVReservation(rid, prompt.credits))
        allocator.append(rid, rotate_reference(prompt.key, np.arange(prompt.key.shape[1])),
                         torch.from_numpy(prompt.value))
    requests = tuple(RequestId(str(r)) for r in case.decode.requests)
    positions = np.array([allocator.cached_length(r) for r in requests], dtype=np.int64)
    with allocator.append_decode(requests):
        for layer in range(22):
            k = torch.from_numpy(case.decode.key[layer])[:, :, None]
            q = torch.zeros(len(requests), 1, 1, 64, dtype=torch.float16)
            _, rotated = apply_rope(q, k, torch.from_numpy(positions)[:, None])
            for row, request in enumerate(requests):
                allocator.write_decode_layer(request, layer, rotated[row, :, 0],
                                             torch.from_numpy(case.decode.value[layer, row]))
    np.savez_compressed(
        OUT / "append_small.npz",
        pool_sha256=np.frombuffer(bytes.fromhex(sha256(pool.numpy())), dtype=np.uint8),
        pool_layer0=pool[0].numpy(),
        pool_layer21=pool[21].numpy(),
        capacity=np.asarray(capacity(allocator), dtype=np.int64),
        free_list=np.asarray(allocator._free_blocks, dtype=np.int32),
    )


if __name__ == "__main__":
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    steps = sys.argv[1:] or ["rope", "attention", "small", "append"]
    if "rope" in steps:
        rope_table()
    if "attention" in steps:
        attention_cfg1()
    if "small" in steps:
        append_small()
    if "append" in steps:
        append_cfg2()
    print("golden fixtures written to", OUT)
