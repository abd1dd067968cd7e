"""Speed of the oracle port against the reference's own CPU code, same rows, one thread.

Test infrastructure, run by hand where the reference checkout is importable:

    PAGEDCORE_REFERENCE=/path/to/PagedCore/src python oracle/calibrate_port.py [rows] [steps]

bench.py's CPU baseline and its reference arm time the oracle restatement of
the reference's CPU path, because the reference cannot be installed on the
GPU box.  This script runs the same decode steps of the same config 4 rows
(seed 4: contexts, churned pool size) through both:

- the reference: ``kv_cache.KVAllocator`` on a CPU pool (full re-validation
  on every call, kv_cache.py:314-357), ``dense.apply_rope`` on each row's
  query and key, ``write_decode_layer`` and ``attention.paged_attention``
  per (row, layer) inside one ``append_decode`` per step (the KV path of
  decoder.py:156-199, without its dense GEMMs);
- the port: ``oracle.allocator``, ``oracle.rope``, ``oracle.kv_write`` and
  ``oracle.attention`` as bench.py's ``oracle_decode_rows`` drives them;

and prints both times per decode token and their ratio as one JSON line.
"""

from __future__ import annotations

import json
import os
import sys
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
if not os.environ.get("PAGEDCORE_REFERENCE"):
    raise SystemExit("set PAGEDCORE_REFERENCE to the reference checkout's src directory (the one holding pagedcore/)")
sys.path.insert(0, os.environ["PAGEDCORE_REFERENCE"])

from pagedcore.attention import paged_attention  # noqa: E402  (the reference)
from pagedcore.dense import apply_rope  # noqa: E402
from pagedcore.engine_types import KVReservation, RequestId  # noqa: E402
from pagedcore.kv_cache import KVAllocator  # noqa: E402

from pagedcore_b200 import workloads  # noqa: E402

LAYERS = 22


def reference_seconds(lengths: list[int], num_blocks: int, steps: int, seed: int) -> float:
    pool = torch.empty((LAYERS, 2, num_blocks, 16, 4, 64), dtype=torch.float16)
    allocator = KVAllocator(pool)
    pattern = torch.from_numpy(workloads.normal_f16(workloads.rng(seed, 9), (LAYERS, 16, 4, 64)))
    rids = tuple(RequestId(f"r{i}") for i in range(len(lengths)))
    for rid, length in zip(rids, lengths, strict=True):
        allocator.create(KVReservation(rid, workloads.blocks_for(length + steps)))
        chunk = pattern.repeat(1, -(-length // 16), 1, 1)[:, :length].contiguous()
        allocator.append(rid, chunk, chunk)
    q, k, v = (torch.from_numpy(x) for x in workloads.decode_step_inputs(seed, len(rids), 0))
    elapsed = 0.0
    with torch.inference_mode():
        for _ in range(steps):
            begin = time.perf_counter()
            positions = [allocator.cached_length(rid) for rid in rids]
            with allocator.append_decode(rids):
                for layer in range(LAYERS):
                    for row, rid in enumerate(rids):
                        position = torch.tensor([[positions[row]]], dtype=torch.int64)
                        query, key = apply_rope(q[layer, row][None, :, None], k[layer, row][None, :, None], position)
                        allocator.write_decode_layer(rid, layer, key[0, :, 0], v[layer, row])
                        paged_attention(query, allocator, rid, layer_index=layer)
            elapsed += time.perf_counter() - begin
    return elapsed


def main() -> None:
    rows = int(sys.argv[1]) if len(sys.argv) > 1 else 8
    steps = int(sys.argv[2]) if len(sys.argv) > 2 else 2
    torch.set_num_threads(1)
    from threadpoolctl import threadpool_limits

    sys.path.insert(0, str(ROOT))
    from bench import oracle_decode_rows

    case = workloads.decode_case(seed=4, batch=256, steps=steps)
    lengths = [int(n) for n in case.lengths[:rows]]
    with threadpool_limits(1):
        port = oracle_decode_rows(lengths, case.num_blocks, steps=steps, warmup=0, seed=4)
    reference = reference_seconds(lengths, case.num_blocks, steps, seed=4)
    tokens = rows * steps
    print(json.dumps({
        "rows": rows, "steps": steps, "tokens": tokens, "contexts": lengths, "pool_blocks": case.num_blocks,
        "threads": 1, "reference_s_per_token": reference / tokens, "port_s_per_token": port / tokens,
        "port_over_reference_speed": reference / port, "torch": torch.__version__,
    }))


if __name__ == "__main__":
    main()
