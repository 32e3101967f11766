"""Per-KV-length CUDA-graph decode, persistent across inferences.

Mirrors src/umic/graph.py of soonhong99/umic-alpamayo (DecodeGraphRunner,
fuse_decode_graph): the VLM's forward is wrapped; during decode every step
with a given KV length replays one captured graph (captured on first sight,
in one shared memory pool); sampling stays outside the graph. KV buffers,
static inputs and the rope-delta tensor live in the runner, so a later
inference only copies its prefill KV into them and replays.

Differences from the reference, all on the host side:
  * decode batches of B >= 1 rows (input_ids [B, 1]), not only B == 1;
  * the step position comes from the cache's host-tracked length instead of
    cache_position.item(), so a decode step makes no host synchronisation;
  * the KV written inside the graph goes through umic_kv_append with a device
    position (no index_copy_), and the attention reads the buffer prefix as a
    view instead of a per-step contiguous copy;
  * FlowStepGraph (graph.py:179-253 of the reference, never wired there) is
    provided and used by workloads.flow_sample(graph=True), which captures a
    whole Euler step (expert pass + update) once and replays it.
"""

from __future__ import annotations

import logging
from typing import Any

import torch
from transformers.cache_utils import DynamicCache

from .cache import InplaceKVCache

logger = logging.getLogger(__name__)

_DYNAMIC_KEYS = ("input_ids", "attention_mask", "cache_position", "past_key_values",
                 "position_ids", "use_cache")

DECODE_ATTN = "umic_decode_sdpa"


def _decode_attention(module, query, key, value, attention_mask, dropout=0.0, scaling=None,
                      is_causal=None, **kwargs):
    """Attention for the captured decode step: each row's single query token attends
    to the whole exact-length KV prefix (the runner checked that no row is padded),
    so no mask is built and SDPA keeps its GQA path, reading the K/V buffer views in
    place. transformers 5.x builds an explicit mask whenever a CUDA stream is
    capturing, which would otherwise force a K/V head-expansion copy per layer."""
    out = torch.nn.functional.scaled_dot_product_attention(
        query, key, value, attn_mask=None, dropout_p=0.0, scale=scaling,
        is_causal=query.shape[2] > 1, enable_gqa=query.shape[1] != key.shape[1])
    return out.transpose(1, 2).contiguous(), None


def _register_decode_attention() -> None:
    from transformers import AttentionInterface

    AttentionInterface.register(DECODE_ATTN, _decode_attention)


def _text_configs(vlm: torch.nn.Module) -> list:
    seen = {}
    for m in vlm.modules():
        c = getattr(m, "config", None)
        if c is not None and type(c).__name__.endswith("TextConfig"):
            seen[id(c)] = c
    return list(seen.values())


class DecodeGraphRunner:
    """Wraps a VLM's forward; replays per-KV-length graphs for decode steps."""

    def __init__(self, vlm: torch.nn.Module, max_new_tokens: int = 96,
                 warmup_steps: int = 2) -> None:
        self.vlm = vlm
        self.orig_forward = vlm.forward
        self.max_new = max_new_tokens
        self.warmup_steps = warmup_steps
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.outs: dict[int, Any] = {}
        self.pool = None
        self.cache: InplaceKVCache | None = None
        self.base_len: int | None = None
        self.batch: int | None = None
        self.in_decode = False
        self.step = 0
        self.s_ids = self.s_pos = self.s_rope = None
        self.const_kwargs: dict[str, Any] = {}
        self.mrope = hasattr(getattr(vlm, "model", None), "rope_deltas")
        _register_decode_attention()
        self._configs = _text_configs(vlm)
        vlm.forward = self.__call__
        orig_generate = getattr(vlm, "generate", None)
        if orig_generate is not None:
            def _generate(*a: Any, **kw: Any):
                out = orig_generate(*a, **kw)
                self.finish()
                return out
            vlm.generate = _generate

    # ------------------------------------------------------------------

    def finish(self) -> None:
        """Decode finished: hand the cache back in dynamic mode (graph.py:68-73)."""
        if self.cache is not None:
            self.cache.disable_graph_mode()
        self.in_decode = False
        self.step = 0

    def release(self) -> None:
        """Drop every captured graph and the persistent buffers."""
        self.finish()
        self.graphs.clear()
        self.outs.clear()
        self.pool = None
        self.cache = None
        self.base_len = None

    def _rope_deltas(self, batch: int, dev) -> torch.Tensor:
        model = getattr(self.vlm, "model", None)
        rd = getattr(model, "rope_deltas", None)
        if rd is None:
            return torch.zeros(batch, 1, dtype=torch.long, device=dev)
        rd = rd.reshape(-1, 1).to(dev)
        if rd.shape[0] != batch:
            rd = rd.repeat_interleave(batch // rd.shape[0], dim=0)
        return rd

    def _begin_inference(self, kwargs: dict[str, Any]) -> bool:
        pkv = kwargs.get("past_key_values")
        if not (isinstance(pkv, DynamicCache) and getattr(pkv, "layers", None)
                and all(getattr(lyr, "keys", None) is not None for lyr in pkv.layers)):
            return False
        mask = kwargs.get("attention_mask")
        if mask is not None and not bool((mask == 1).all().item()):
            logger.warning("DecodeGraphRunner: padded input mask - bypassing")
            return False
        ids = kwargs["input_ids"]
        batch, dev = ids.shape[0], ids.device
        base = pkv.get_seq_length()
        same_shape = (self.cache is not None and base == self.base_len and batch == self.batch)
        if same_shape and pkv is not self.cache:
            # Reuse the persistent buffers (captured graphs baked their addresses).
            for dst, src in zip(self.cache.layers, pkv.layers):
                dst._k_buf[:, :, :base, :].copy_(src.keys[:, :, :base, :])
                dst._v_buf[:, :, :base, :].copy_(src.values[:, :, :base, :])
            self.cache.set_pos(base)
        elif not same_shape:
            if self.cache is not None:
                logger.info("DecodeGraphRunner: shape changed, rebuilding graphs")
                self.graphs.clear()
                self.outs.clear()
                self.pool = None
            if isinstance(pkv, InplaceKVCache) and all(
                    lyr.capacity >= base + self.max_new for lyr in pkv.layers):
                self.cache = pkv
            else:
                self.cache = InplaceKVCache.from_dynamic(pkv, extra_tokens=self.max_new)
            self.base_len = base
            self.batch = batch
            self.s_ids = torch.zeros(batch, 1, dtype=torch.long, device=dev)
            self.s_pos = torch.zeros(1, dtype=torch.long, device=dev)
            self.s_rope = torch.zeros(batch, 1, dtype=torch.long, device=dev)
        self.s_rope.copy_(self._rope_deltas(batch, dev))
        self.cache.enable_graph_mode(self.s_pos)
        self.const_kwargs = {k: v for k, v in kwargs.items() if k not in _DYNAMIC_KEYS}
        self.in_decode = True
        return True

    def _static_call(self):
        # position ids from device tensors only: no host value enters the graph
        pos = (self.s_pos + self.s_rope).reshape(self.batch, 1)
        position_ids = pos.unsqueeze(0).expand(3, self.batch, 1) if self.mrope else pos
        saved = [c._attn_implementation_internal for c in self._configs]
        for c in self._configs:
            c._attn_implementation_internal = DECODE_ATTN
        try:
            return self.orig_forward(input_ids=self.s_ids, attention_mask=None,
                                     past_key_values=self.cache, position_ids=position_ids,
                                     use_cache=True, **self.const_kwargs)
        finally:
            for c, v in zip(self._configs, saved):
                c._attn_implementation_internal = v

    # ------------------------------------------------------------------

    def __call__(self, *args: Any, **kwargs: Any):
        ids = kwargs.get("input_ids")
        if (args or ids is None or ids.dim() != 2 or ids.shape[1] != 1
                or kwargs.get("past_key_values") is None or not ids.is_cuda):
            return self.orig_forward(*args, **kwargs)
        if not self.in_decode and not self._begin_inference(kwargs):
            return self.orig_forward(*args, **kwargs)
        if ids.shape[0] != self.batch:
            return self.orig_forward(*args, **kwargs)
        pos = self.cache.get_seq_length()
        kv_len = pos + 1
        if kv_len > self.cache.layers[0].capacity:
            raise RuntimeError(f"DecodeGraphRunner: KV length {kv_len} exceeds the cache "
                               f"capacity {self.cache.layers[0].capacity}")
        self.s_ids.copy_(ids)
        self.s_pos.fill_(pos)
        self.cache.set_graph_len(kv_len)
        if not self.graphs and self.step < self.warmup_steps:
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                out = self._static_call()
            torch.cuda.current_stream().wait_stream(s)
        elif kv_len not in self.graphs:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=self.pool, capture_error_mode="relaxed"):
                self.outs[kv_len] = self._static_call()
            if self.pool is None:
                self.pool = g.pool()
            g.replay()
            self.graphs[kv_len] = g
            out = self.outs[kv_len]
        else:
            self.graphs[kv_len].replay()
            out = self.outs[kv_len]
        self.step += 1
        self.cache.set_pos(kv_len)
        return out


def fuse_decode_graph(vlm: torch.nn.Module, max_new_tokens: int = 96) -> DecodeGraphRunner:
    """Install the per-length decode CUDA-graph runner (graph.py:174-176)."""
    return DecodeGraphRunner(vlm, max_new_tokens=max_new_tokens)


class FlowStepGraph:
    """Capture one fixed-shape flow ODE step and replay it (graph.py:179-253).

    Every step runs the expert on the same shapes with the same buffer
    addresses (the prefix KV is read-only; the action tokens are appended at
    [base, base + n) and cropped back), so a single graph serves all steps;
    only the values of x and t change. Capture failure falls back to eager.
    """

    def __init__(self, step_fn, warmup: int = 2) -> None:
        self.step_fn = step_fn
        self.warmup = warmup
        self.n = 0
        self.graph: torch.cuda.CUDAGraph | None = None
        self.xs = self.ts = self.out = None
        self.failed = False

    def __call__(self, x: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
        if self.failed or (self.graph is None and self.n < self.warmup):
            self.n += 1
            return self.step_fn(x=x, t=t)
        if self.graph is None:
            try:
                self.xs = x.clone()
                self.ts = t.clone()
                s = torch.cuda.Stream()
                s.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(s):
                    self.step_fn(x=self.xs, t=self.ts)
                torch.cuda.current_stream().wait_stream(s)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, capture_error_mode="relaxed"):
                    self.out = self.step_fn(x=self.xs, t=self.ts)
                self.graph = g
            except Exception as exc:  # noqa: BLE001 - correctness over speed
                logger.warning("FlowStepGraph capture failed (%s); eager fallback", exc)
                self.failed = True
                return self.step_fn(x=x, t=t)
        self.xs.copy_(x)
        self.ts.copy_(t)
        self.graph.replay()
        return self.out.clone()
