"""Fused B200 execution of the GPT modules (filled in by the kernel layer)."""

from __future__ import annotations

import torch


def should_fuse(x: torch.Tensor) -> bool:
    return False
