"""Pool-sizing configuration of the paged KV path.

Mirrors the fields of PagedCore's frozen ``PagedCoreConfig`` that size and
shape the KV pool (src/pagedcore/config.py:24-89): ``kv_pool_mib``,
``workspace_margin_mib`` and the fixed ``block_tokens``/``context_limit``,
with the same ``PAGEDCORE_*`` environment variables (config.py:111-128).
Model identity, service limits and logging belong to the layers above this
path.
"""

from __future__ import annotations

import os
from collections.abc import Mapping
from dataclasses import dataclass


class ConfigurationError(ValueError):
    pass


@dataclass(frozen=True, slots=True)
class PagedCoreConfig:
    context_limit: int = 2048
    block_tokens: int = 16
    kv_pool_mib: int = 8192
    workspace_margin_mib: int = 1536

    def __post_init__(self) -> None:
        for name, value in (
            ("context_limit", self.context_limit),
            ("block_tokens", self.block_tokens),
            ("kv_pool_mib", self.kv_pool_mib),
            ("workspace_margin_mib", self.workspace_margin_mib),
        ):
            if not isinstance(value, int) or isinstance(value, bool):
                raise ConfigurationError(f"{name} must be an integer")
        for name, value, expected in (
            ("context_limit", self.context_limit, 2048),
            ("block_tokens", self.block_tokens, 16),
        ):
            if value != expected:
                raise ConfigurationError(f"{name} is fixed at {expected!r}")
        for name, value in (
            ("kv_pool_mib", self.kv_pool_mib),
            ("workspace_margin_mib", self.workspace_margin_mib),
        ):
            if value <= 0:
                raise ConfigurationError(f"{name} must be greater than zero")


def _read_int(environment: Mapping[str, str], name: str, default: int) -> int:
    raw = environment.get(name)
    if raw is None:
        return default
    try:
        return int(raw)
    except ValueError as error:
        raise ConfigurationError(f"{name} must be an integer") from error


def load_config(environment: Mapping[str, str] | None = None) -> PagedCoreConfig:
    source = os.environ if environment is None else environment
    return PagedCoreConfig(
        context_limit=_read_int(source, "PAGEDCORE_CONTEXT_LIMIT", 2048),
        block_tokens=_read_int(source, "PAGEDCORE_BLOCK_TOKENS", 16),
        kv_pool_mib=_read_int(source, "PAGEDCORE_KV_POOL_MIB", 8192),
        workspace_margin_mib=_read_int(source, "PAGEDCORE_WORKSPACE_MARGIN_MIB", 1536),
    )
