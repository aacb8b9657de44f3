"""KV caches with the reference's interface (``src/avqa/cache.py:39-331``).

Both caches keep raw keys/values in head layout ``[B, H, S, D]`` and return
them from :meth:`lookup` in append order.  In addition each cache carries the
device quantization state of the AVQ modules that decode through it, so a
decode step quantizes only the appended token (bit-identical to the
reference's full re-quantization, see ``csrc/avq_decode.cu``).

Unlike the reference's ``PagedKVCache`` (whose pages are allocated as
``[1, H, 0, D]`` fp32 and therefore reject B > 1 and bf16 appends), pages
here are ``[B, H, page_size, D]`` device tensors in the cache dtype; decode
appends are written into the current page by the append kernel.
"""
from __future__ import annotations

from abc import ABC, abstractmethod

import torch

from avqa_b200.exceptions import ConfigurationError, NotInitializedError, ShapeError


class KVCache(ABC):
    """Abstract KV cache."""

    def __init__(self) -> None:
        self.quant_states: dict = {}  # module key -> ops.QuantState

    @abstractmethod
    def append(self, key: torch.Tensor, value: torch.Tensor) -> None: ...

    @abstractmethod
    def lookup(self) -> tuple[torch.Tensor, torch.Tensor]: ...

    @abstractmethod
    def reset(self) -> None: ...

    @abstractmethod
    def state_dict(self) -> dict[str, torch.Tensor]: ...

    @abstractmethod
    def load_state_dict(self, state: dict[str, torch.Tensor]) -> None: ...

    @property
    @abstractmethod
    def size(self) -> int: ...


class InMemoryKVCache(KVCache):
    """Contiguous cache; keys/values concatenated along the sequence axis."""

    def __init__(self, num_heads: int = 1, head_dim_k: int = 64, head_dim_v: int = 64, max_size: int = 0,
                 device: str | torch.device = "cpu", dtype: torch.dtype = torch.float32) -> None:
        super().__init__()
        self.num_heads, self.head_dim_k, self.head_dim_v = num_heads, head_dim_k, head_dim_v
        self.max_size, self.device, self.dtype = max_size, device, dtype
        self.cache_key = torch.empty(0, num_heads, 0, head_dim_k, device=device, dtype=dtype)
        self.cache_value = torch.empty(0, num_heads, 0, head_dim_v, device=device, dtype=dtype)

    def append(self, key: torch.Tensor, value: torch.Tensor) -> None:
        if tuple(key.shape) != (*value.shape[:-1], self.head_dim_k):
            raise ShapeError(f"key/value shape mismatch: key={tuple(key.shape)}, value={tuple(value.shape)}",
                             expected=(*value.shape[:-1], self.head_dim_k), actual=tuple(key.shape))
        if self.cache_key.numel() == 0:
            self.cache_key = key.to(device=self.device, dtype=self.dtype)
            self.cache_value = value.to(device=self.device, dtype=self.dtype)
        else:
            self.cache_key = torch.cat([self.cache_key, key.to(self.cache_key.dtype)], dim=-2)
            self.cache_value = torch.cat([self.cache_value, value.to(self.cache_value.dtype)], dim=-2)
        if self.max_size > 0 and self.size > self.max_size:
            excess = self.size - self.max_size
            self.cache_key = self.cache_key[..., excess:, :].contiguous()
            self.cache_value = self.cache_value[..., excess:, :].contiguous()
            self.quant_states.clear()  # evicted keys leave the buckets: re-quantize next time

    def lookup(self) -> tuple[torch.Tensor, torch.Tensor]:
        if self.cache_key.numel() == 0 or self.cache_value.numel() == 0:
            return (torch.zeros(1, self.num_heads, 0, self.head_dim_k, dtype=self.dtype, device=self.device),
                    torch.zeros(1, self.num_heads, 0, self.head_dim_v, dtype=self.dtype, device=self.device))
        return self.cache_key, self.cache_value

    def reset(self) -> None:
        self.cache_key = torch.empty(0, self.num_heads, 0, self.head_dim_k, device=self.device, dtype=self.dtype)
        self.cache_value = torch.empty(0, self.num_heads, 0, self.head_dim_v, device=self.device, dtype=self.dtype)
        self.quant_states.clear()

    def state_dict(self) -> dict[str, torch.Tensor]:
        return {"schema_version": torch.tensor(1, dtype=torch.int32),
                "num_heads": torch.tensor(self.num_heads, dtype=torch.int32),
                "head_dim_k": torch.tensor(self.head_dim_k, dtype=torch.int32),
                "head_dim_v": torch.tensor(self.head_dim_v, dtype=torch.int32),
                "size": torch.tensor(self.size, dtype=torch.int32),
                "cache_key": self.cache_key.detach().clone(), "cache_value": self.cache_value.detach().clone()}

    def load_state_dict(self, state: dict[str, torch.Tensor]) -> None:
        for name in ("num_heads", "head_dim_k", "head_dim_v"):
            if name in state and int(state[name]) != getattr(self, name):
                raise ShapeError(f"{name} mismatch", expected=getattr(self, name), actual=int(state[name]))
        k, v = state.get("cache_key"), state.get("cache_value")
        self.quant_states.clear()
        if k is not None and v is not None and k.numel() > 0:
            self.cache_key = k.to(device=self.device, dtype=self.dtype)
            self.cache_value = v.to(device=self.device, dtype=self.dtype)
        else:
            self.reset()

    @property
    def size(self) -> int:
        return 0 if self.cache_key.numel() == 0 else int(self.cache_key.shape[-2])


class PagedKVCache(KVCache):
    """Fixed-size pages ``[B, H, page_size, D]`` on the cache device."""

    def __init__(self, page_size: int = 16, num_heads: int = 1, head_dim_k: int = 64, head_dim_v: int = 64,
                 max_pages: int = 0, device: str | torch.device = "cpu", dtype: torch.dtype = torch.float32) -> None:
        super().__init__()
        if page_size <= 0:
            raise ConfigurationError(f"page_size must be > 0, got {page_size}", {"page_size": page_size})
        self.page_size, self.num_heads = page_size, num_heads
        self.head_dim_k, self.head_dim_v = head_dim_k, head_dim_v
        self.max_pages, self.device, self.dtype = max_pages, device, dtype
        self.key_pages: list[torch.Tensor] = []
        self.value_pages: list[torch.Tensor] = []
        self.batch = 0
        self.fill = 0  # tokens in the last page

    # -- page management -------------------------------------------------------

    def allocate_page(self, batch: int) -> None:
        if self.max_pages > 0 and len(self.key_pages) >= self.max_pages:
            raise NotInitializedError(f"paged KV cache is full ({self.max_pages} pages)")
        shape_k = (batch, self.num_heads, self.page_size, self.head_dim_k)
        shape_v = (batch, self.num_heads, self.page_size, self.head_dim_v)
        self.key_pages.append(torch.zeros(shape_k, dtype=self.dtype, device=self.device))
        self.value_pages.append(torch.zeros(shape_v, dtype=self.dtype, device=self.device))
        self.batch = batch
        self.fill = 0

    def reserve(self, batch: int, n: int) -> list[tuple[int, int, int]]:
        """Claim ``n`` slots; returns ``(page, slot0, count)`` runs in order."""
        if self.key_pages and batch != self.batch:
            raise ShapeError("batch size changed inside a paged cache", expected=self.batch, actual=batch)
        runs = []
        while n > 0:
            if not self.key_pages or self.fill == self.page_size:
                self.allocate_page(batch)
            take = min(n, self.page_size - self.fill)
            runs.append((len(self.key_pages) - 1, self.fill, take))
            self.fill += take
            n -= take
        return runs

    def append(self, key: torch.Tensor, value: torch.Tensor) -> None:
        B, _, T, _ = key.shape
        cursor = 0
        for page, slot0, take in self.reserve(B, T):
            self.key_pages[page][:, :, slot0:slot0 + take] = key[:, :, cursor:cursor + take].to(self.dtype)
            self.value_pages[page][:, :, slot0:slot0 + take] = value[:, :, cursor:cursor + take].to(self.dtype)
            cursor += take

    def lookup(self) -> tuple[torch.Tensor, torch.Tensor]:
        if not self.key_pages:
            return (torch.zeros(1, self.num_heads, 0, self.head_dim_k, dtype=self.dtype, device=self.device),
                    torch.zeros(1, self.num_heads, 0, self.head_dim_v, dtype=self.dtype, device=self.device))
        ks = self.key_pages[:-1] + [self.key_pages[-1][:, :, :self.fill]]
        vs = self.value_pages[:-1] + [self.value_pages[-1][:, :, :self.fill]]
        return torch.cat(ks, dim=-2), torch.cat(vs, dim=-2)

    def reset(self) -> None:
        self.key_pages, self.value_pages = [], []
        self.fill = 0
        self.quant_states.clear()

    def state_dict(self) -> dict[str, torch.Tensor]:
        return {"schema_version": torch.tensor(1, dtype=torch.int32),
                "page_size": torch.tensor(self.page_size, dtype=torch.int32),
                "num_pages": torch.tensor(len(self.key_pages), dtype=torch.int32),
                "size": torch.tensor(self.size, dtype=torch.int32)}

    def load_state_dict(self, state: dict[str, torch.Tensor]) -> None:
        if "page_size" in state and int(state["page_size"]) != self.page_size:
            raise ShapeError("page_size mismatch", expected=self.page_size, actual=int(state["page_size"]))
        self.reset()

    @property
    def size(self) -> int:
        return 0 if not self.key_pages else (len(self.key_pages) - 1) * self.page_size + self.fill

    @property
    def num_pages(self) -> int:
        return len(self.key_pages)


__all__ = ["InMemoryKVCache", "KVCache", "PagedKVCache"]
