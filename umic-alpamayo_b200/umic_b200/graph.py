"""CUDA-graph decode per KV length, and the flow-step graph.

Two pieces share one mechanism, `GraphBank`: graphs keyed by a shape key, each
captured the first time its key is seen, all into one memory pool, replayed
afterwards; the first capture is preceded by eager warm-up calls on a side
stream (lazy library initialisation must not happen inside a capture).

`DecodeGraphRunner` (drop-in for the reference's runner, src/umic/graph.py:36-176)
wraps a VLM's forward. A decode step -- input_ids [B, 1] against a populated
cache with no padding -- is a pure function of (token ids, position, KV length),
so the runner keeps those inputs in persistent device tensors (`DecodeState`)
together with the in-place KV cache the graphs write into, and replays the graph
of the step's KV length. The state outlives an inference: the next inference
with the same prefill length and batch copies its prefill KV into the same
buffers and replays graphs captured earlier. What this build does differently:
batches of B >= 1 rows; the position comes from the cache's host length, so a
step never synchronises with the device; appends go through umic_kv_append /
umic_qk_norm_rope_kv at a device position, and attention reads the buffer
prefix as a view (no per-step contiguous copy).

`FlowStepGraph` replays a whole fixed-shape Euler step of the flow sampler (the
reference defines one but never wires it, src/umic/graph.py:179-253): every step
runs the expert over the same shapes and buffer addresses, so one graph serves
them all and only the values of x and t change.
"""

from __future__ import annotations

import logging
from dataclasses import dataclass, field
from typing import Any, Callable

import torch
from transformers.cache_utils import DynamicCache

from .cache import InplaceKVCache

logger = logging.getLogger(__name__)

DECODE_ATTN = "umic_decode_sdpa"

# forward() arguments a decode step supplies itself; everything else is passed through
_STEP_ARGS = frozenset(("input_ids", "attention_mask", "cache_position", "past_key_values",
                        "position_ids", "use_cache"))


def on_side_stream(fn: Callable[[], Any]) -> Any:
    """Runs fn on a fresh stream ordered after (and joined back into) the current one."""
    main = torch.cuda.current_stream()
    side = torch.cuda.Stream()
    side.wait_stream(main)
    with torch.cuda.stream(side):
        out = fn()
    main.wait_stream(side)
    return out


@dataclass
class GraphBank:
    """CUDA graphs by key, captured on first use into one shared pool."""

    graphs: dict = field(default_factory=dict)
    outputs: dict = field(default_factory=dict)
    pool: Any = None

    def run(self, key, fn: Callable[[], Any]) -> Any:
        """Replays the graph of `key`, capturing fn() for it first if it has none."""
        graph = self.graphs.get(key)
        if graph is None:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, pool=self.pool, capture_error_mode="relaxed"):
                self.outputs[key] = fn()
            if self.pool is None:
                self.pool = graph.pool()
            self.graphs[key] = graph
        graph.replay()
        return self.outputs[key]

    def clear(self) -> None:
        self.graphs.clear()
        self.outputs.clear()
        self.pool = None


# ------------------------------------------------------------ decode attention

def _decode_attention(module, query, key, value, attention_mask, dropout=0.0, scaling=None,
                      is_causal=None, **kwargs):
    """The captured decode step's attention: each row's single query token attends to the
    whole exact-length KV prefix (the runner only graphs unpadded batches), so no mask is
    needed and SDPA keeps its grouped-query path over the K/V buffer views. transformers
    5.x builds an explicit mask whenever a stream is capturing, which would force a K/V
    head expansion copy per layer."""
    out = torch.nn.functional.scaled_dot_product_attention(
        query, key, value, attn_mask=None, dropout_p=0.0, scale=scaling,
        is_causal=query.shape[2] > 1, enable_gqa=query.shape[1] != key.shape[1])
    return out.transpose(1, 2).contiguous(), None


def _text_configs(vlm: torch.nn.Module) -> list:
    """Every distinct text config in the model (their attention backend is switched to
    DECODE_ATTN while a step is captured or run)."""
    found = {}
    for m in vlm.modules():
        cfg = getattr(m, "config", None)
        if cfg is not None and type(cfg).__name__.endswith("TextConfig"):
            found.setdefault(id(cfg), cfg)
    return list(found.values())


# ------------------------------------------------------------------- decode

@dataclass
class DecodeState:
    """What a captured decode graph reads and writes, kept across inferences."""

    cache: InplaceKVCache
    base_len: int
    batch: int
    ids: torch.Tensor  # [B, 1] token ids of the step
    pos: torch.Tensor  # [1] device write position
    rope_delta: torch.Tensor  # [B, 1] MRoPE offset of each row
    passthrough: dict = field(default_factory=dict)  # other forward() kwargs


def _populated(pkv) -> bool:
    layers = getattr(pkv, "layers", None)
    return (isinstance(pkv, DynamicCache) and bool(layers)
            and all(getattr(l, "keys", None) is not None for l in layers))


class DecodeGraphRunner:
    """Wraps vlm.forward; decode steps replay per-KV-length CUDA graphs."""

    def __init__(self, vlm: torch.nn.Module, max_new_tokens: int = 96,
                 warmup_steps: int = 2) -> None:
        from transformers import AttentionInterface

        AttentionInterface.register(DECODE_ATTN, _decode_attention)
        self.vlm = vlm
        self.max_new = max_new_tokens
        self.bank = GraphBank()
        self.state: DecodeState | None = None
        self.in_decode = False
        self._eager_left = warmup_steps  # side-stream warm-up steps before the first capture
        self._configs = _text_configs(vlm)
        self._mrope = hasattr(getattr(vlm, "model", None), "rope_deltas")
        self._inner = vlm.forward
        vlm.forward = self.__call__
        generate = getattr(vlm, "generate", None)
        if generate is not None:
            def generate_then_finish(*a: Any, **kw: Any):
                try:
                    return generate(*a, **kw)
                finally:
                    self.finish()
            vlm.generate = generate_then_finish

    @property
    def graphs(self) -> dict:
        return self.bank.graphs

    @property
    def cache(self) -> InplaceKVCache | None:
        return None if self.state is None else self.state.cache

    # ----------------------------------------------------------- lifecycle

    def finish(self) -> None:
        """End of an inference's decode: the cache returns to host-position appends
        (src/umic/graph.py:68-73)."""
        if self.state is not None:
            self.state.cache.disable_graph_mode()
        self.in_decode = False

    def release(self) -> None:
        """Drops every captured graph and the persistent state."""
        self.finish()
        self.bank.clear()
        self.state = None

    # -------------------------------------------------------------- entry

    def _step_ids(self, args: tuple, kwargs: dict) -> torch.Tensor | None:
        """The [B, 1] token ids of a call that is a graphable decode step, else None."""
        ids = kwargs.get("input_ids")
        if args or ids is None or ids.dim() != 2 or ids.shape[1] != 1 or not ids.is_cuda:
            return None
        return ids if kwargs.get("past_key_values") is not None else None

    def __call__(self, *args: Any, **kwargs: Any):
        ids = self._step_ids(args, kwargs)
        if ids is None or (not self.in_decode and not self._open(kwargs)):
            return self._inner(*args, **kwargs)
        st = self.state
        if ids.shape[0] != st.batch:
            return self._inner(*args, **kwargs)
        kv_len = st.cache.get_seq_length() + 1
        if kv_len > st.cache.layers[0].capacity:
            raise RuntimeError(f"DecodeGraphRunner: KV length {kv_len} exceeds the cache "
                               f"capacity {st.cache.layers[0].capacity}")
        st.ids.copy_(ids)
        st.pos.fill_(kv_len - 1)
        st.cache.set_graph_len(kv_len)
        if self._eager_left > 0 and not self.bank.graphs:
            self._eager_left -= 1
            out = on_side_stream(self._step)
        else:
            out = self.bank.run(kv_len, self._step)
        st.cache.set_pos(kv_len)
        return out

    # ------------------------------------------------------------ internals

    def _open(self, kwargs: dict) -> bool:
        """Starts an inference's decode phase on its prefill cache; False leaves the call
        to the wrapped forward (cache not populated, or padded rows)."""
        pkv = kwargs.get("past_key_values")
        if not _populated(pkv):
            return False
        mask = kwargs.get("attention_mask")
        if mask is not None and not bool(mask.bool().all().item()):
            logger.warning("DecodeGraphRunner: padded rows, decode runs without graphs")
            return False
        ids = kwargs["input_ids"]
        batch, base = ids.shape[0], pkv.get_seq_length()
        st = self.state
        if st is not None and (st.base_len, st.batch) == (base, batch):
            if pkv is not st.cache:  # same shapes: refill the buffers the graphs point at
                for dst, src in zip(st.cache.layers, pkv.layers):
                    dst.k_buf[:, :, :base].copy_(src.keys[:, :, :base])
                    dst.v_buf[:, :, :base].copy_(src.values[:, :, :base])
                st.cache.set_pos(base)
        else:
            if st is not None:
                logger.info("DecodeGraphRunner: new prefill length / batch, graphs dropped")
                self.bank.clear()
            self.state = st = self._new_state(pkv, ids, base)
        st.rope_delta.copy_(self._rope_deltas(batch, ids.device))
        st.passthrough = {k: v for k, v in kwargs.items() if k not in _STEP_ARGS}
        st.cache.enable_graph_mode(st.pos)
        self.in_decode = True
        return True

    def _new_state(self, pkv, ids: torch.Tensor, base: int) -> DecodeState:
        roomy = isinstance(pkv, InplaceKVCache) and all(
            l.capacity >= base + self.max_new for l in pkv.layers)
        cache = pkv if roomy else InplaceKVCache.from_dynamic(pkv, extra_tokens=self.max_new)
        b, dev = ids.shape[0], ids.device
        return DecodeState(cache, base, b, torch.zeros(b, 1, dtype=torch.long, device=dev),
                           torch.zeros(1, dtype=torch.long, device=dev),
                           torch.zeros(b, 1, dtype=torch.long, device=dev))

    def _rope_deltas(self, batch: int, dev) -> torch.Tensor:
        rd = getattr(getattr(self.vlm, "model", None), "rope_deltas", None)
        if rd is None:
            return torch.zeros(batch, 1, dtype=torch.long, device=dev)
        rd = rd.reshape(-1, 1).to(dev)
        return rd if rd.shape[0] == batch else rd.repeat_interleave(batch // rd.shape[0], dim=0)

    def _step(self):
        """One decode step from the persistent tensors only: no host value is read, so
        the same work replays from a graph (position ids = position + rope delta)."""
        st = self.state
        rows = (st.pos + st.rope_delta).view(st.batch, 1)
        position_ids = rows.unsqueeze(0).expand(3, st.batch, 1) if self._mrope else rows
        saved = [c._attn_implementation_internal for c in self._configs]
        for c in self._configs:
            c._attn_implementation_internal = DECODE_ATTN
        try:
            return self._inner(input_ids=st.ids, attention_mask=None, past_key_values=st.cache,
                               position_ids=position_ids, use_cache=True, **st.passthrough)
        finally:
            for c, v in zip(self._configs, saved):
                c._attn_implementation_internal = v


def fuse_decode_graph(vlm: torch.nn.Module, max_new_tokens: int = 96) -> DecodeGraphRunner:
    """Installs the per-length decode graph runner on `vlm` (src/umic/graph.py:174-176)."""
    return DecodeGraphRunner(vlm, max_new_tokens=max_new_tokens)


# ---------------------------------------------------------------------- flow

class FlowStepGraph:
    """step_fn(x=x, t=t) replayed from one CUDA graph after `warmup` eager calls.

    The inputs are copied into persistent tensors the graph reads; the output is cloned
    out of the graph's pool, so callers may keep it across steps. If the capture fails
    the step stays eager for good (correctness first)."""

    def __init__(self, step_fn: Callable[..., torch.Tensor], warmup: int = 2) -> None:
        self.step_fn = step_fn
        self.warmup = warmup
        self.calls = 0
        self.bank = GraphBank()
        self.inputs: tuple[torch.Tensor, torch.Tensor] | None = None
        self.failed = False

    @property
    def graph(self):
        return self.bank.graphs.get(0)

    def _captured_step(self) -> torch.Tensor:
        xs, ts = self.inputs
        return self.step_fn(x=xs, t=ts)

    def __call__(self, x: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
        self.calls += 1
        if self.failed or (self.graph is None and self.calls <= self.warmup):
            return self.step_fn(x=x, t=t)
        if self.inputs is None:
            self.inputs = (x.clone(), t.clone())
            try:
                on_side_stream(self._captured_step)
                return self.bank.run(0, self._captured_step).clone()
            except RuntimeError as exc:
                logger.warning("FlowStepGraph: capture failed (%s); the step stays eager", exc)
                self.failed = True
                self.bank.clear()
                return self.step_fn(x=x, t=t)
        self.inputs[0].copy_(x)
        self.inputs[1].copy_(t)
        return self.bank.run(0, self._captured_step).clone()


def fuse_flow_graph(model: torch.nn.Module, warmup: int = 2) -> None:
    """Replay every ODE step of `model.diffusion.sample` from a CUDA graph
    (src/umic/graph.py:235-253): the step callables the model hands to its sampler
    (`step_fn`, `unguided_step_fn`) are wrapped in FlowStepGraph for the duration of each
    sample() call; the sampler itself is untouched."""
    sampler = model.diffusion
    inner = sampler.sample

    def sample_with_step_graphs(*args: Any, **kwargs: Any):
        for key in ("step_fn", "unguided_step_fn"):
            if kwargs.get(key) is not None:
                kwargs[key] = FlowStepGraph(kwargs[key], warmup)
        return inner(*args, **kwargs)

    sampler.sample = sample_with_step_graphs
    logger.info("fuse_flow_graph: ODE steps of %s.sample replay from CUDA graphs",
                type(sampler).__name__)
