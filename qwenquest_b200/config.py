"""``--hisparse-config`` parsing with the defaults and checks of ``src/qwenquest/config.py:267-359``.

The backends accept the reference's ``SparseConfig`` objects directly (any
object with the same attributes); JSON strings, dicts and ``None`` are parsed
here into :class:`SparseConfig` with the upstream defaults: ``top_k=2048``,
``device_buffer_size=2*top_k``, ``quest_page_size=64`` for
``algorithm == "quest"``, ``top_k % quest_page_size == 0``; unknown keys land
in ``sparse_extra_config`` (which carries ``avoid_recent_overlap``).
"""

from __future__ import annotations

import json
from collections.abc import Mapping
from dataclasses import dataclass, field
from typing import Any


@dataclass(frozen=True)
class SparseConfig:
    top_k: int = 2048
    device_buffer_size: int = 4096
    host_to_device_ratio: int = 2
    swap_in_block_size: int = 960
    algorithm: str | None = None
    backend: str | None = None
    page_size: int | None = None
    min_sparse_prompt_len: int | None = None
    quest_page_size: int | None = None
    sparse_extra_config: dict[str, Any] = field(default_factory=dict, hash=False)

    @property
    def avoid_recent_overlap(self) -> bool:
        return bool(self.sparse_extra_config.get("avoid_recent_overlap", False))


def parse_hisparse_config(config) -> Any:
    """Returns ``config`` itself when it already is a parsed config object."""
    if config is not None and not isinstance(config, (str, Mapping)):
        return config
    if config is None:
        extra: dict[str, Any] = {}
    elif isinstance(config, str):
        try:
            extra = dict(json.loads(config))
        except json.JSONDecodeError as e:
            raise ValueError(f"Failed to parse hisparse_config: {e}") from e
    else:
        extra = dict(config)
    top_k = extra.pop("top_k", 2048)
    device_buffer_size = extra.pop("device_buffer_size", 2 * top_k)
    host_to_device_ratio = extra.pop("host_to_device_ratio", 2)
    swap_in_block_size = extra.pop("swap_in_block_size", 960)
    if device_buffer_size < top_k:
        raise ValueError(
            f"device_buffer_size ({device_buffer_size}) must be no smaller than top_k ({top_k})"
        )
    if not isinstance(swap_in_block_size, int) or isinstance(swap_in_block_size, bool):
        raise ValueError(f"swap_in_block_size must be an integer, got {swap_in_block_size!r}")
    if swap_in_block_size <= 0 or swap_in_block_size > 1024:
        raise ValueError(f"swap_in_block_size ({swap_in_block_size}) must be in the range [1, 1024]")
    algorithm = extra.pop("algorithm", None)
    backend = extra.pop("backend", None)
    min_sparse_prompt_len = extra.pop("min_sparse_prompt_len", None)
    page_size = extra.pop("page_size", None)
    quest_page_size = extra.pop("quest_page_size", None)
    if algorithm == "quest":
        if quest_page_size is None:
            quest_page_size = 64
        if quest_page_size <= 0 or top_k % quest_page_size != 0:
            raise ValueError(
                f"hisparse_config: top_k ({top_k}) must be divisible by "
                f"quest_page_size ({quest_page_size}) for algorithm='quest'."
            )
    return SparseConfig(
        top_k=top_k,
        device_buffer_size=device_buffer_size,
        host_to_device_ratio=host_to_device_ratio,
        swap_in_block_size=swap_in_block_size,
        algorithm=algorithm,
        backend=backend,
        page_size=page_size,
        min_sparse_prompt_len=min_sparse_prompt_len,
        quest_page_size=quest_page_size,
        sparse_extra_config=extra,
    )


def avoid_recent_overlap(cfg) -> bool:
    v = getattr(cfg, "avoid_recent_overlap", None)
    if v is None:
        v = (getattr(cfg, "sparse_extra_config", None) or {}).get("avoid_recent_overlap", False)
    return bool(v)
