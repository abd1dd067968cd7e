"""Boundary value types of the paged KV path.

Same names, fields and validation as PagedCore's engine_types
(src/pagedcore/engine_types.py:7-11, 63-65, 170-219), so values built by a
caller of the reference are accepted unchanged.  The other request-lifecycle
types of that module belong to the service layer and are not part of this path.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import StrEnum
from typing import NewType, TypeAlias

RequestId = NewType("RequestId", str)
BlockId = NewType("BlockId", int)
BlockTable: TypeAlias = tuple[BlockId, ...]


class FinishReason(StrEnum):
    """Why a generation stopped (engine_types.py:63-65)."""

    EOS = "eos"
    LENGTH = "length"


@dataclass(frozen=True, slots=True)
class KVReservation:
    """Maximum capacity credits granted at admission, including owned blocks.

    Credits do not assign physical blocks (engine_types.py:170-187).
    """

    request_id: RequestId
    maximum_block_credits: int

    def __post_init__(self) -> None:
        credits = self.maximum_block_credits
        if not isinstance(credits, int) or isinstance(credits, bool) or credits <= 0:
            raise ValueError("maximum_block_credits must be a positive integer")


@dataclass(frozen=True, slots=True)
class CapacityCounts:
    """Snapshot of ownership and credits (engine_types.py:190-219)."""

    total_blocks: int
    free_blocks: int
    owned_blocks: int
    reserved_blocks: int
    active_slots: int
    live_cached_token_slots: int

    def __post_init__(self) -> None:
        for name, value in (
            ("total_blocks", self.total_blocks),
            ("free_blocks", self.free_blocks),
            ("owned_blocks", self.owned_blocks),
            ("reserved_blocks", self.reserved_blocks),
            ("active_slots", self.active_slots),
            ("live_cached_token_slots", self.live_cached_token_slots),
        ):
            if not isinstance(value, int) or isinstance(value, bool) or value < 0:
                raise ValueError(f"{name} must be a nonnegative integer")
        if self.free_blocks + self.owned_blocks != self.total_blocks:
            raise ValueError("free_blocks + owned_blocks must equal total_blocks")
        if not self.owned_blocks <= self.reserved_blocks <= self.total_blocks:
            raise ValueError("owned_blocks <= reserved_blocks <= total_blocks must hold")
