"""avqa_b200: AVQ attention (sachncs/avqa's hot path) on B200 CUDA kernels.

Public API mirrors the reference package ``avqa``:

- :class:`AVQAttention`            the attention module
- :func:`avqa_b200.functional.attention`
- :class:`AVQConfig` and its sub-configs
- :class:`Backend`, :class:`CUDABackend`, :class:`QuantizationResult`
- :class:`HierarchicalCodebook`, KV caches, the error hierarchy
- :class:`StreamingVQBuffer`       causal incremental VQ (``avqa.streaming_vq``)

The compute runs in ``libavqa_b200.so`` (C ABI: ``include/avqa_b200.h``),
built in-tree by ``python -m avqa_b200.build_ext``.
"""
from __future__ import annotations

from avqa_b200.attention_module import AVQAttention
from avqa_b200.backend import Backend, CUDABackend, QuantizationResult
from avqa_b200.cache import InMemoryKVCache, KVCache, PagedKVCache
from avqa_b200.codebook import HierarchicalCodebook, codebook_from_keys
from avqa_b200.config import AVQConfig
from avqa_b200.exceptions import (AVQAError, BackendError, CodebookError, ConfigurationError, DeviceError, DtypeError,
                                  MergeError, NotInitializedError, RoutingError, ShapeError)
from avqa_b200.streaming_vq import StreamingVQBuffer

__version__ = "0.1.0"
Codebook = HierarchicalCodebook

__all__ = [
    "AVQAError", "AVQAttention", "AVQConfig", "Backend", "BackendError", "CUDABackend", "Codebook", "CodebookError",
    "ConfigurationError", "DeviceError", "DtypeError", "HierarchicalCodebook", "InMemoryKVCache", "KVCache",
    "MergeError", "NotInitializedError", "PagedKVCache", "QuantizationResult", "RoutingError", "ShapeError", "StreamingVQBuffer",
    "__version__", "codebook_from_keys",
]
