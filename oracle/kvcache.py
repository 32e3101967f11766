"""Host restatement of the reference's in-place KV cache bookkeeping (test infrastructure).

Follows InplaceLayer (src/umic/cache.py:25-91): a preallocated buffer of
base + extra + margin tokens; update() writes n tokens at the write pointer and
advances it, raising on overflow (cache.py:64-71); crop() only moves the
pointer back, negative lengths counting from the end (cache.py:85-91); the
visible keys/values are the prefix [0, pos). Graph mode writes one token at a
device position and exposes an exact graph_len prefix (cache.py:53-63).
"""

from __future__ import annotations

import torch


class KVCacheOracle:
    def __init__(self, k: torch.Tensor, v: torch.Tensor, extra: int, margin: int = 8):
        b, h, base, d = k.shape
        self.cap = base + extra + margin
        self.k = torch.zeros(b, h, self.cap, d, dtype=k.dtype)
        self.v = torch.zeros_like(self.k)
        self.k[:, :, :base] = k
        self.v[:, :, :base] = v
        self.pos = base

    def update(self, k_new: torch.Tensor, v_new: torch.Tensor):
        n = k_new.shape[2]
        if self.pos + n > self.cap:
            raise RuntimeError(f"InplaceLayer overflow: pos {self.pos} + new {n} > "
                               f"buffer {self.cap}")
        self.k[:, :, self.pos:self.pos + n] = k_new
        self.v[:, :, self.pos:self.pos + n] = v_new
        self.pos += n
        return self.k[:, :, :self.pos], self.v[:, :, :self.pos]

    def graph_update(self, k_new, v_new, pos: int, graph_len: int):
        self.k[:, :, pos:pos + 1] = k_new
        self.v[:, :, pos:pos + 1] = v_new
        return self.k[:, :, :graph_len], self.v[:, :, :graph_len]

    def crop(self, max_length: int) -> None:
        if max_length < 0:
            max_length = self.pos + max_length
        self.pos = min(self.pos, max_length)

    def get_seq_length(self) -> int:
        return self.pos
