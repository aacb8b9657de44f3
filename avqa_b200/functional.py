"""Functional entry point (reference ``src/avqa/functional.py:24-66``).

Like the reference, each call builds a fresh ``AVQAttention`` without
projections -- and therefore with the default codebook -- unless a
``codebook`` (parents, children) pair is given.  ``kv_cache`` is extended in
place.
"""
from __future__ import annotations

import torch

from avqa_b200.attention_module import AVQAttention
from avqa_b200.cache import KVCache
from avqa_b200.config import AVQConfig


def attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, config: AVQConfig,
              mask: torch.Tensor | None = None, kv_cache: KVCache | None = None,
              codebook: tuple[torch.Tensor, torch.Tensor] | None = None) -> torch.Tensor:
    module = AVQAttention(config, in_proj=False, out_proj=False)
    if codebook is not None:
        module.codebook.parents, module.codebook.children = codebook
    return module(query, key, value, mask=mask, kv_cache=kv_cache)


__all__ = ["attention"]
