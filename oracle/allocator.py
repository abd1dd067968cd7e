"""Oracle of KVAllocator's bookkeeping (src/pagedcore/kv_cache.py:63-357).

Test infrastructure only.  Pure Python; request ids are any hashable value.
Data movement is separate (``oracle.kv_write``): the methods here return the
slot ids (physical_block * 16 + slot) that the reference's copies target.
"""

from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class _Sequence:
    credits: int
    blocks: list[int] = field(default_factory=list)
    length: int = 0


class OracleAllocator:
    def __init__(self, num_blocks: int, *, audit: bool = True) -> None:
        self.num_blocks = num_blocks
        self.audit_every_call = audit
        # kv_cache.py:86 - reversed(range(N)): block 0 on top of the stack.
        self.free: list[int] = list(reversed(range(num_blocks)))
        self.sequences: dict[object, _Sequence] = {}
        self.owners: dict[int, object] = {}
        self.staged: dict[object, tuple[list[int], int]] | None = None
        self.staged_additional = 0

    # kv_cache.py:314-357
    def audit(self) -> tuple[int, int, int, int, int, int]:
        for sequence in self.sequences.values():
            if (
                not 0 <= sequence.length <= 2048
                or len(sequence.blocks) != (sequence.length + 15) // 16
                or not len(sequence.blocks) <= sequence.credits <= 128
            ):
                raise RuntimeError("corrupt KV block table or reservation")
        assigned = [b for s in self.sequences.values() for b in s.blocks]
        if any(not 0 <= b < self.num_blocks for b in self.free + assigned):
            raise RuntimeError("invalid physical KV block")
        owned, free = set(assigned), set(self.free)
        if len(assigned) != len(owned):
            raise RuntimeError("physical KV blocks must have unique owners")
        if len(self.free) != len(free):
            raise RuntimeError("free KV blocks must be unique")
        if not free.isdisjoint(owned):
            raise RuntimeError("owned KV blocks must not be free")
        if free | owned != set(range(self.num_blocks)):
            raise RuntimeError("KV blocks must cover the pool")
        owners = {b: r for r, s in self.sequences.items() for b in s.blocks}
        if owners != self.owners:
            raise RuntimeError("KV blocks are not owned by the recorded requests")
        return self.capacity_unchecked()

    def _check(self) -> None:
        if self.audit_every_call:
            self.audit()

    def capacity_unchecked(self) -> tuple[int, int, int, int, int, int]:
        return (
            self.num_blocks,
            len(self.free),
            sum(len(s.blocks) for s in self.sequences.values()),
            sum(s.credits for s in self.sequences.values()),
            len(self.sequences),
            sum(s.length for s in self.sequences.values()),
        )

    def capacity(self) -> tuple[int, int, int, int, int, int]:
        self._check()
        return self.capacity_unchecked()

    def _mutation(self) -> None:
        if self.staged is not None:
            raise RuntimeError("KV mutation is not allowed during a staged decode append")

    # kv_cache.py:92-110
    def create(self, request: object, credits: int) -> None:
        self._mutation()
        if request in self.sequences:
            raise ValueError("request already has a KV cache")
        total, _, _, reserved, _, _ = self.capacity()
        if credits > total:
            raise ValueError("reservation exceeds total KV pool capacity")
        if credits > 128:
            raise ValueError("reservation exceeds KV context capacity")
        if credits > total - reserved:
            raise RuntimeError("KV pool has insufficient unreserved blocks")
        self.sequences[request] = _Sequence(credits)
        self._check()

    def table(self, request: object) -> tuple[int, ...]:
        self._check()
        return tuple(self.sequences[request].blocks)

    def length(self, request: object) -> int:
        self._check()
        return self.sequences[request].length

    # kv_cache.py:127-179 (bookkeeping; the copy is kv_write.write_rows)
    def append(self, request: object, tokens: int) -> list[int]:
        """Publish ``tokens`` positions; return their slot ids in position order."""
        self._mutation()
        self._check()
        sequence = self.sequences[request]
        if tokens < 1:
            raise ValueError("K and V must share FP16 [22, tokens, 4, 64] on the pool device")
        length = sequence.length + tokens
        if length > 2048:
            raise ValueError("KV cache must not exceed 2048 token positions")
        required = (length + 15) // 16
        if required > sequence.credits:
            raise RuntimeError("KV append exceeds request reservation")
        additional = required - len(sequence.blocks)
        if additional > len(self.free):
            raise RuntimeError("KV pool has insufficient free blocks")
        new_blocks = list(reversed(self.free[-additional:])) if additional else []
        blocks = sequence.blocks + new_blocks
        slots = [blocks[p // 16] * 16 + p % 16 for p in range(sequence.length, length)]
        if additional:
            del self.free[-additional:]
        for block in new_blocks:
            self.owners[block] = request
        sequence.blocks = blocks
        sequence.length = length
        self._check()
        return slots

    # kv_cache.py:181-205
    def decode_begin(self, requests: tuple[object, ...]) -> tuple[list[int], list[int]]:
        """Stage length+1 per request; return (slot ids, RoPE positions)."""
        self._mutation()
        self._check()
        if not requests or len(set(requests)) != len(requests):
            raise ValueError("decode requires nonempty, distinct request IDs")
        staged = {}
        additional = 0
        slots, positions = [], []
        for request in requests:
            sequence = self.sequences[request]
            if not 1 <= sequence.length < 2048:
                raise ValueError("decode requires 1 to 2047 cached token positions")
            if (sequence.length + 16) // 16 > sequence.credits:
                raise RuntimeError("KV append exceeds request reservation")
            blocks = list(sequence.blocks)
            if sequence.length % 16 == 0:
                additional += 1
                if additional > len(self.free):
                    raise RuntimeError("KV pool has insufficient free blocks")
                blocks.append(self.free[-additional])
            staged[request] = (blocks, sequence.length + 1)
            slots.append(blocks[sequence.length // 16] * 16 + sequence.length % 16)
            positions.append(sequence.length)
        self.staged = staged
        self.staged_additional = additional
        return slots, positions

    # kv_cache.py:208-219
    def decode_commit(self) -> None:
        assert self.staged is not None
        if self.staged_additional:
            del self.free[-self.staged_additional :]
        for request, (blocks, length) in self.staged.items():
            sequence = self.sequences[request]
            for block in blocks[len(sequence.blocks) :]:
                self.owners[block] = request
            sequence.blocks = blocks
            sequence.length = length
        self.staged = None
        self._check()

    def decode_abort(self) -> None:
        self.staged = None

    def view(self, request: object) -> tuple[list[int], int]:
        """Table and length seen by attention (staged view when staged)."""
        if self.staged is not None and request in self.staged:
            blocks, length = self.staged[request]
            return list(blocks), length
        sequence = self.sequences[request]
        return list(sequence.blocks), sequence.length

    # kv_cache.py:286-298
    def release(self, request: object) -> None:
        self._mutation()
        self._check()
        sequence = self.sequences.pop(request)
        for block in sequence.blocks:
            del self.owners[block]
        self.free.extend(reversed(sequence.blocks))
        self._check()
