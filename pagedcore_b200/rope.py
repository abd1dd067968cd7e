"""FP16 RoPE table for the fused K/Q rotation of the append kernel.

PagedCore rotates K (and Q) in FP16 with cos/sin computed in FP32 and then
rounded to FP16 (src/pagedcore/dense.py:46-59).  The FP32 ``cos``/``sin``
and ``pow`` of ATen's CPU kernels are not correctly rounded, and a few table
entries differ in their last FP16 bit from any other implementation, so the
table is built here with the reference's own op sequence on the CPU:

    inverse = 1 / (10000 ** (arange(0, 64, 2).float() / 64))
    angles  = positions.float()[..., None] * inverse;  angles = cat(angles, angles)
    cos     = angles.cos().half();  sin = angles.sin().half()

for every position 0..2047.  Only the first 32 columns are kept (the second
half duplicates them).  The device copy is FP16 cos[2048][32] followed by
sin[2048][32], the layout ``pkv_append_kv`` reads.
"""

from __future__ import annotations

import torch

_CONTEXT_LIMIT = 2048
_HEAD_DIM = 64

_device_tables: dict[torch.device, torch.Tensor] = {}


def rope_cos_sin(positions: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """FP16 cos/sin [..., 64] at int64 positions, as dense.apply_rope makes them."""
    with torch.autocast(device_type=positions.device.type, enabled=False):
        inverse = 1.0 / (
            10000.0 ** (torch.arange(0, _HEAD_DIM, 2, device=positions.device).float() / _HEAD_DIM)
        )
        angles = positions.float().unsqueeze(-1) * inverse
        angles = torch.cat((angles, angles), dim=-1)
        return angles.cos().to(torch.float16), angles.sin().to(torch.float16)


def host_table() -> torch.Tensor:
    """The [2, 2048, 32] FP16 (cos, sin) table, computed on the CPU."""
    positions = torch.arange(_CONTEXT_LIMIT, dtype=torch.int64)[None]
    cos, sin = rope_cos_sin(positions)
    return torch.stack((cos[0, :, : _HEAD_DIM // 2], sin[0, :, : _HEAD_DIM // 2])).contiguous()


def device_table(device: torch.device) -> torch.Tensor:
    """The table resident on ``device`` (built once per device)."""
    device = torch.device(device)
    table = _device_tables.get(device)
    if table is None:
        table = host_table().to(device)
        _device_tables[device] = table
    return table
