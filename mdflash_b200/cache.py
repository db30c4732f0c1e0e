"""Static-capacity KV cache for tree verification.

transformers' DynamicLayer.update concatenates (transformers/cache_utils.py:102-121), which
reallocates and copies every layer's whole K and V on every verify step.  TreeKVLayer
keeps DynamicLayer's interface (``keys`` / ``values`` views of the live rows, ``update``,
``crop``, ``get_seq_length``) but writes new rows in place into a buffer allocated once
per request, so the reference's ``compact_dynamic_cache`` (ddtree.py:325-333) and this
package's compaction kernel both work on it unchanged, and the K/V base pointers stay
fixed between steps (the compaction pointer table is built once).
"""
from __future__ import annotations

import torch
from transformers.cache_utils import DynamicCache, DynamicLayer

from . import kernels as K


class TreeKVLayer(DynamicLayer):
    def __init__(self, capacity: int):
        super().__init__()
        self.capacity = int(capacity)
        self.length = 0
        self.k_buf: torch.Tensor | None = None
        self.v_buf: torch.Tensor | None = None

    def lazy_initialization(self, key_states: torch.Tensor, value_states: torch.Tensor) -> None:
        self.dtype, self.device = key_states.dtype, key_states.device
        b, h, _, d = key_states.shape
        self.k_buf = torch.zeros((b, h, self.capacity, d), dtype=self.dtype, device=self.device)
        self.v_buf = torch.zeros((b, h, self.capacity, value_states.shape[-1]), dtype=self.dtype,
                                 device=self.device)
        self.length = 0
        self.keys = self.k_buf[..., :0, :]
        self.values = self.v_buf[..., :0, :]
        self.is_initialized = True

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args, **kwargs):
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        n = key_states.shape[-2]
        end = self.length + n
        if end > self.capacity:
            raise RuntimeError(f"TreeKVLayer capacity {self.capacity} exceeded ({end})")
        self.k_buf[..., self.length:end, :].copy_(key_states)
        self.v_buf[..., self.length:end, :].copy_(value_states)
        self.length = end
        self.keys = self.k_buf[..., :end, :]
        self.values = self.v_buf[..., :end, :]
        return self.keys, self.values

    def get_seq_length(self) -> int:
        return self.length if self.is_initialized else 0

    def get_max_cache_shape(self) -> int:
        return self.capacity

    def crop(self, max_length: int) -> None:
        if max_length < 0:
            max_length = self.get_seq_length() - abs(max_length)
        if not self.is_initialized or self.length <= max_length:
            return
        self.length = max(0, max_length)
        self.keys = self.k_buf[..., :self.length, :]
        self.values = self.v_buf[..., :self.length, :]

    def reset(self) -> None:
        self.length = 0
        if self.is_initialized:
            self.keys = self.k_buf[..., :0, :]
            self.values = self.v_buf[..., :0, :]


class TreeKVCache(DynamicCache):
    """A DynamicCache whose layers are TreeKVLayer with a fixed row capacity."""

    def __init__(self, num_layers: int, capacity: int):
        super().__init__()
        self.layers = [TreeKVLayer(capacity) for _ in range(num_layers)]
        self.layer_class_to_replicate = None
        self._table: K.KvTable | None = None

    def allocate(self, kv_heads: int, head_dim: int, dtype: torch.dtype, device,
                 batch: int = 1) -> "TreeKVCache":
        """Allocates every layer's buffers up front (instead of on the first update)."""
        proto = torch.empty((batch, kv_heads, 0, head_dim), dtype=dtype, device=device)
        for layer in self.layers:
            if not layer.is_initialized:
                layer.lazy_initialization(proto, proto)
        return self

    def kv_table(self) -> K.KvTable:
        """Pointer table of every layer's K and V buffers (stable across steps)."""
        if self._table is None:
            ts = []
            for layer in self.layers:
                if not layer.is_initialized:
                    raise RuntimeError("cache layers are not initialised yet")
                ts += [layer.k_buf, layer.v_buf]
            self._table = K.KvTable(ts)
        return self._table
