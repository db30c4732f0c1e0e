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
    """``keys`` / ``values`` are views of the live rows, built when read: a decode loop sets
    the length every round, and building two views per layer there cost ~5 us each on the
    host (0.35 ms per round at 36 layers)."""

    def __init__(self, capacity: int):
        super().__init__()
        self.capacity = int(capacity)
        self.length = 0
        self.k_buf: torch.Tensor | None = None
        self.v_buf: torch.Tensor | None = None
        self._views: tuple[int, torch.Tensor, torch.Tensor] | None = None

    def _live(self, i: int):
        if getattr(self, "k_buf", None) is None:
            return self.__dict__.get("_unset_kv", (None, None))[i]
        if self._views is None or self._views[0] != self.length:
            self._views = (self.length, self.k_buf[..., :self.length, :],
                           self.v_buf[..., :self.length, :])
        return self._views[1 + i]

    @property
    def keys(self):
        return self._live(0)

    @keys.setter
    def keys(self, t):  # before the buffers exist (the base class sets None)
        self.__dict__["_unset_kv"] = (t, self.__dict__.get("_unset_kv", (None, None))[1])

    @property
    def values(self):
        return self._live(1)

    @values.setter
    def values(self, t):
        self.__dict__["_unset_kv"] = (self.__dict__.get("_unset_kv", (None, None))[0], t)

    def lazy_initialization(self, key_states: torch.Tensor, value_states: torch.Tensor) -> None:
        self.dtype, self.device = key_states.dtype, key_states.device
        b, h, _, d = key_states.shape
        self.k_buf = torch.zeros((b, h, self.capacity, d), dtype=self.dtype, device=self.device)
        self.v_buf = torch.zeros((b, h, self.capacity, value_states.shape[-1]), dtype=self.dtype,
                                 device=self.device)
        self.length = 0
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

    def set_length(self, length: int) -> None:
        """Sets the live row count (shorter or longer), for rows that a device-side step
        wrote without telling the host (a step recorded with a device prefix length)."""
        if not self.is_initialized:
            raise RuntimeError("cache layer is not initialised yet")
        if not 0 <= length <= self.capacity:
            raise ValueError(f"length {length} outside [0, {self.capacity}]")
        self.length = int(length)

    def reset(self) -> None:
        self.length = 0


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

    def set_seq_length(self, length: int) -> None:
        """TreeKVLayer.set_length on every layer."""
        for layer in self.layers:
            layer.set_length(length)

    @property
    def capacity(self) -> int:
        return self.layers[0].capacity

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
