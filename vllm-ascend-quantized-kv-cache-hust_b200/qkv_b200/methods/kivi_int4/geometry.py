"""KIVI INT4 layout invariants (pure Python, no torch).

The five rules of the reference's geometry.py:22-60, with its messages:
group % 8 (eight int4 lanes per int32 word), residual % group (whole-group
key flush), head % 8, head % group (value groups along head_size), and
block % group (a key group never straddles a page).
"""

from __future__ import annotations

from typing import Any


def validate_kivi_geometry(*, head_size: int, group_size: int, residual_length: int,
                           block_size: int | None = None) -> None:
    if group_size <= 0 or group_size % 8:
        raise ValueError(f"kivi_int4 requires group_size divisible by 8, got {group_size}")
    if residual_length % group_size:
        raise ValueError(
            f"kivi_int4 requires residual_length ({residual_length}) "
            f"to be divisible by group_size ({group_size})"
        )
    if head_size % 8:
        raise ValueError(f"kivi_int4 requires head_size divisible by 8, got {head_size}")
    if head_size % group_size:
        raise ValueError(
            f"kivi_int4 requires head_size ({head_size}) to be divisible by group_size ({group_size})"
        )
    if block_size is not None and block_size % group_size:
        raise ValueError(
            f"kivi_int4 requires block_size ({block_size}) to be divisible by group_size ({group_size})"
        )


def validate_kivi_config(config: Any) -> None:
    """Accepts a MethodConfig or a live impl (``kivi_*`` attribute names)."""
    group_size = getattr(config, "group_size", None)
    if group_size is None:
        group_size = getattr(config, "kivi_group_size", None)
    residual_length = getattr(config, "residual_length", None)
    if residual_length is None:
        residual_length = getattr(config, "kivi_residual_length", None)
    if group_size is None or residual_length is None:
        raise ValueError(
            "kivi_int4 config must define group_size/residual_length "
            "(or kivi_group_size/kivi_residual_length)"
        )
    validate_kivi_geometry(
        head_size=config.head_size,
        group_size=group_size,
        residual_length=residual_length,
        block_size=getattr(config, "block_size", None),
    )


__all__ = ["validate_kivi_config", "validate_kivi_geometry"]
