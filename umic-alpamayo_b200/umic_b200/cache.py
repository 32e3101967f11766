"""In-place KV cache: preallocated buffers, in-place appends, O(1) crop.

Mirrors src/umic/cache.py of soonhong99/umic-alpamayo (InplaceLayer /
InplaceKVCache, HF DynamicLayer / DynamicCache subclasses so HF mask and
attention-backend selection stay unchanged). Appends run on the B200
umic_kv_append kernel:
  * eager mode writes at the host-tracked position; overflow raises
    RuntimeError before anything is written (cache.py:64-68);
  * graph mode (driven by DecodeGraphRunner) writes one token per step at a
    device position tensor, so one captured graph per KV length replays while
    the position advances (cache.py:53-63).
Unlike the reference, reads never copy: update() returns prefix views of the
buffer in both modes (the reference returned a fresh .contiguous() copy of the
whole prefix on every decode step, about 466 MB per step at 3.1 k tokens for
the 36-layer LM); the attention backend reads the strided view directly.
"""

from __future__ import annotations

import logging

import torch
from transformers.cache_utils import DynamicCache, DynamicLayer

from .kernels.kv import kv_append

logger = logging.getLogger(__name__)


class InplaceLayer(DynamicLayer):
    """One layer's KV in a preallocated [B, H, capacity, D] buffer."""

    def __init__(self, k_buf: torch.Tensor, v_buf: torch.Tensor, base_len: int) -> None:
        super().__init__()
        self._k_buf = k_buf
        self._v_buf = v_buf
        self._pos = base_len
        self.dtype, self.device = k_buf.dtype, k_buf.device
        self.is_initialized = True
        self.keys = k_buf[:, :, :base_len, :]
        self.values = v_buf[:, :, :base_len, :]
        self.graph_mode = False
        self._pos_t: torch.Tensor | None = None
        self._graph_len = 0

    @property
    def capacity(self) -> int:
        return self._k_buf.shape[2]

    def lazy_initialization(self, key_states, value_states) -> None:  # buffers exist already
        return None

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args, **kwargs):
        n = key_states.shape[2]
        if self.graph_mode and n == 1 and self._pos_t is not None:
            kv_append(self._k_buf, self._v_buf, key_states, value_states, self._pos_t)
            self.keys = self._k_buf[:, :, :self._graph_len, :]
            self.values = self._v_buf[:, :, :self._graph_len, :]
            return self.keys, self.values
        pos = self._pos
        kv_append(self._k_buf, self._v_buf, key_states, value_states, pos)  # raises on overflow
        self._pos = pos + n
        self.keys = self._k_buf[:, :, :self._pos, :]
        self.values = self._v_buf[:, :, :self._pos, :]
        return self.keys, self.values

    def reserve(self, n: int):
        """Claims the slots of n new tokens for a kernel that writes K/V itself.

        Returns (k_buf, v_buf, pos): pos is an int, or the device position
        tensor in graph mode (one token per step). The visible keys /
        values are advanced exactly as update() would; the caller must write the
        slots before the attention reads them."""
        if self.graph_mode and n == 1 and self._pos_t is not None:
            self.keys = self._k_buf[:, :, :self._graph_len, :]
            self.values = self._v_buf[:, :, :self._graph_len, :]
            return self._k_buf, self._v_buf, self._pos_t
        pos = self._pos
        if pos + n > self.capacity:
            raise RuntimeError(f"InplaceLayer overflow: pos {pos} + new {n} > "
                               f"buffer {self.capacity}")
        self._pos = pos + n
        self.keys = self._k_buf[:, :, :self._pos, :]
        self.values = self._v_buf[:, :, :self._pos, :]
        return self._k_buf, self._v_buf, pos

    def get_seq_length(self, *args, **kwargs) -> int:
        return self._pos

    def get_max_cache_shape(self) -> int:
        return -1

    def crop(self, max_length: int) -> None:
        """O(1): move the write pointer back (negative counts from the end)."""
        if max_length < 0:
            max_length = self._pos + max_length
        self._pos = max(0, min(self._pos, max_length))
        self.keys = self._k_buf[:, :, :self._pos, :]
        self.values = self._v_buf[:, :, :self._pos, :]


class InplaceKVCache(DynamicCache):
    """DynamicCache whose layers are preallocated InplaceLayers (cache.py:94-160)."""

    def __init__(self, layers: list[InplaceLayer]) -> None:
        super().__init__()
        self.layers = layers

    @classmethod
    def allocate(cls, num_layers: int, batch: int, heads: int, head_dim: int, capacity: int,
                 device, dtype=torch.bfloat16) -> "InplaceKVCache":
        """Empty cache with room for `capacity` tokens per layer (for a prefill that
        writes straight into it, with no DynamicCache conversion)."""
        layers = []
        for _ in range(num_layers):
            kb = torch.empty(batch, heads, capacity, head_dim, device=device, dtype=dtype)
            layers.append(InplaceLayer(kb, torch.empty_like(kb), 0))
        return cls(layers)

    @classmethod
    def from_dynamic(cls, cache: DynamicCache, extra_tokens: int,
                     margin: int = 8) -> "InplaceKVCache":
        """One-time conversion: allocate base + extra + margin tokens and copy the
        existing prefix (cache.py:104-128)."""
        layers: list[InplaceLayer] = []
        alloc = 0
        for lyr in cache.layers:
            k, v = lyr.keys, lyr.values
            b, h, base_len, d = k.shape
            kb = torch.empty(b, h, base_len + extra_tokens + margin, d, device=k.device,
                             dtype=k.dtype)
            vb = torch.empty_like(kb)
            kb[:, :, :base_len, :] = k
            vb[:, :, :base_len, :] = v
            layers.append(InplaceLayer(kb, vb, base_len))
            alloc += kb.numel() * kb.element_size() * 2
        logger.info("InplaceKVCache: %d layers, base_len=%d, alloc=%.0f MB", len(layers),
                    layers[0]._pos if layers else 0, alloc / 1e6)
        return cls(layers)

    def crop(self, max_length: int) -> None:
        for lyr in self.layers:
            lyr.crop(max_length)

    # --- CUDA-graph mode plumbing (driven by umic_b200.graph) -------------

    def enable_graph_mode(self, pos_t: torch.Tensor) -> None:
        for lyr in self.layers:
            lyr.graph_mode = True
            lyr._pos_t = pos_t

    def disable_graph_mode(self) -> None:
        for lyr in self.layers:
            lyr.graph_mode = False
            lyr.keys = lyr._k_buf[:, :, :lyr._pos, :]
            lyr.values = lyr._v_buf[:, :, :lyr._pos, :]

    def set_pos(self, n: int) -> None:
        for lyr in self.layers:
            lyr._pos = n

    def set_graph_len(self, n: int) -> None:
        for lyr in self.layers:
            lyr._graph_len = n

    def get_seq_length(self, layer_idx: int = 0, *args, **kwargs) -> int:
        return self.layers[layer_idx].get_seq_length()
