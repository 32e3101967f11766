"""In-place KV cache over one device slab, with O(1) crop and a capture-safe append.

Layout: every layer's K and V live in ONE allocation, a slab of shape
[layers, 2, batch, kv_heads, capacity, head_dim] (bf16). A layer's K and V are
views of it, so a 36-layer cache is one 3.7 GB block of HBM (cfg4, 8 episodes)
rather than 72 allocations, and nothing is ever re-allocated or concatenated:
  * a write claims slots [pos, pos + n) of every row with `reserve(n)` and the
    umic_kv_append kernel (or the fused attention-input kernel) fills them;
  * `crop(n)` moves the write position back; the data stays where it is;
  * reads are prefix views [:, :, :len, :] that the attention backends take as
    strided tensors -- no per-step copy of the prefix.

Graph decode: `enable_graph_mode(pos_t)` binds every layer to one shared
`DeviceCursor` holding a device int64 position. One-token appends then write at
*pos_t as read on the device at execution time, so a CUDA graph captured for a
KV length replays correctly while the position advances. `set_graph_len` sets
the length the captured graph's attention reads; `set_pos` resynchronises the
host position after replays.

The classes subclass transformers' DynamicLayer / DynamicCache so its mask and
attention-backend selection treat them as the dynamic cache they replace. The
public surface (class and method names, the overflow message) is the one of the
reference's InplaceLayer / InplaceKVCache (src/umic/cache.py:25-160).
"""

from __future__ import annotations

import logging
from dataclasses import dataclass

import torch
from transformers.cache_utils import DynamicCache, DynamicLayer

from .kernels.kv import kv_append

logger = logging.getLogger(__name__)


@dataclass
class DeviceCursor:
    """The write position of graph-mode appends, shared by every layer of one cache.

    pos_t: device int64 tensor [1] the captured kernels read; length: the KV length the
    graph being captured or replayed attends over; active: whether appends use it."""

    pos_t: torch.Tensor | None = None
    length: int = 0
    active: bool = False


class InplaceLayer(DynamicLayer):
    """One layer's K and V: views [batch, kv_heads, capacity, head_dim] of the cache slab
    (or any preallocated buffers), a host write position and the cache's DeviceCursor."""

    def __init__(self, k_buf: torch.Tensor, v_buf: torch.Tensor, base_len: int,
                 cursor: DeviceCursor | None = None) -> None:
        super().__init__()
        if k_buf.shape != v_buf.shape:
            raise ValueError("InplaceLayer: K and V buffers differ in shape")
        self.k_buf, self.v_buf = k_buf, v_buf
        self.cursor = cursor if cursor is not None else DeviceCursor()
        self.dtype, self.device = k_buf.dtype, k_buf.device
        self.is_initialized = True
        self._fill = 0
        self._show(base_len)

    # ---------------------------------------------------------------- state

    @property
    def capacity(self) -> int:
        return self.k_buf.shape[2]

    @property
    def graph_mode(self) -> bool:
        return self.cursor.active

    def _show(self, length: int) -> None:
        """Sets the host position and points keys / values at the first `length` slots."""
        self._fill = length
        self._expose(length)

    def _expose(self, length: int) -> None:
        self.keys = self.k_buf[:, :, :length]
        self.values = self.v_buf[:, :, :length]

    # ------------------------------------------------------------- writes

    def reserve(self, n: int):
        """Claims the slots of `n` new tokens for a kernel that writes K/V itself.

        Returns (k_buf, v_buf, pos): pos is the host position (an int), or, for a
        one-token step in graph mode, the cursor's device position tensor. keys / values
        already cover the new slots when this returns; the caller must fill them before
        attention reads. Overflow raises before anything moves."""
        cur = self.cursor
        if cur.active and n == 1 and cur.pos_t is not None:
            self._expose(cur.length)
            return self.k_buf, self.v_buf, cur.pos_t
        start = self._fill
        if start + n > self.capacity:
            raise RuntimeError(f"InplaceLayer overflow: pos {start} + new {n} > "
                               f"buffer {self.capacity}")
        self._show(start + n)
        return self.k_buf, self.v_buf, start

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args, **kwargs):
        """Appends [batch, kv_heads, n, head_dim] keys / values in place; returns the
        prefix views (never a copy)."""
        k_buf, v_buf, pos = self.reserve(key_states.shape[2])
        kv_append(k_buf, v_buf, key_states, value_states, pos)
        return self.keys, self.values

    def lazy_initialization(self, key_states, value_states) -> None:
        return None  # the buffers exist from construction

    # --------------------------------------------------------------- reads

    def get_seq_length(self, *args, **kwargs) -> int:
        return self._fill

    def get_max_cache_shape(self) -> int:
        return -1

    def crop(self, max_length: int) -> None:
        """Moves the write position back to `max_length` (negative: that many tokens
        from the end), clamped to [0, current]; O(1), nothing is copied."""
        target = self._fill + max_length if max_length < 0 else max_length
        self._show(min(self._fill, max(0, target)))


class InplaceKVCache(DynamicCache):
    """DynamicCache whose layers are InplaceLayers over one slab."""

    def __init__(self, layers: list[InplaceLayer], slab: torch.Tensor | None = None) -> None:
        super().__init__()
        self.layers = layers
        self.slab = slab
        self.cursor = layers[0].cursor if layers else DeviceCursor()
        for lyr in layers:
            lyr.cursor = self.cursor

    # ---------------------------------------------------------- construction

    @staticmethod
    def _slab(num_layers: int, batch: int, heads: int, head_dim: int, capacity: int,
              device, dtype) -> torch.Tensor:
        return torch.empty(num_layers, 2, batch, heads, capacity, head_dim, device=device,
                           dtype=dtype)

    @classmethod
    def _over(cls, slab: torch.Tensor, base_len: int) -> "InplaceKVCache":
        cursor = DeviceCursor()
        return cls([InplaceLayer(slab[i, 0], slab[i, 1], base_len, cursor)
                    for i in range(slab.shape[0])], slab)

    @classmethod
    def allocate(cls, num_layers: int, batch: int, heads: int, head_dim: int, capacity: int,
                 device, dtype=torch.bfloat16) -> "InplaceKVCache":
        """An empty cache with room for `capacity` tokens per row and layer, for a prefill
        that writes straight into it."""
        return cls._over(cls._slab(num_layers, batch, heads, head_dim, capacity, device, dtype), 0)

    @classmethod
    def from_dynamic(cls, cache: DynamicCache, extra_tokens: int,
                     margin: int = 8) -> "InplaceKVCache":
        """Moves a filled DynamicCache into a slab with `extra_tokens + margin` free
        slots per layer (one copy of the prefix, once; src/umic/cache.py:104-130)."""
        first = cache.layers[0].keys
        b, h, base, d = first.shape
        slab = cls._slab(len(cache.layers), b, h, d, base + extra_tokens + margin,
                         first.device, first.dtype)
        for i, lyr in enumerate(cache.layers):
            slab[i, 0, :, :, :base].copy_(lyr.keys)
            slab[i, 1, :, :, :base].copy_(lyr.values)
        out = cls._over(slab, base)
        logger.info("InplaceKVCache: %d layers x %d + %d slots, %.0f MB", slab.shape[0], base,
                    extra_tokens + margin, slab.numel() * slab.element_size() / 1e6)
        return out

    # ------------------------------------------------------------ position

    def crop(self, max_length: int) -> None:
        for lyr in self.layers:
            lyr.crop(max_length)

    def set_pos(self, n: int) -> None:
        """Host write position of every layer (after graph replays advanced the device)."""
        for lyr in self.layers:
            if self.cursor.active:
                lyr._fill = n  # the views follow the cursor's length while graphs run
            else:
                lyr._show(n)

    def get_seq_length(self, layer_idx: int = 0, *args, **kwargs) -> int:
        return self.layers[layer_idx].get_seq_length()

    # ------------------------------------------------------- graph decode

    def enable_graph_mode(self, pos_t: torch.Tensor) -> None:
        """One-token appends write at the device position pos_t from now on."""
        self.cursor.pos_t = pos_t
        self.cursor.active = True

    def disable_graph_mode(self) -> None:
        """Back to host-position appends; keys / values show the host length again."""
        self.cursor.active = False
        for lyr in self.layers:
            lyr._show(lyr._fill)

    def set_graph_len(self, n: int) -> None:
        """KV length the captured / replayed decode step attends over."""
        self.cursor.length = n
