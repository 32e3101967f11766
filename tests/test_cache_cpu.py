"""Host bookkeeping of InplaceKVCache / DecodeGraphRunner on CPU.

The device write (umic_kv_append) is replaced, in this file only, by a CPU
stand-in with the same contract, so the pointer / crop / graph-mode logic can
be checked against the oracle without a GPU. The real wrapper refuses CPU
tensors (no CPU path in the product); that is checked too."""

import pytest
import torch
from transformers.cache_utils import DynamicCache

import oracle
from umic_b200 import cache as cache_mod
from umic_b200.cache import InplaceKVCache


def _fake_kv_append(k_buf, v_buf, k_new, v_new, pos):
    n = k_new.shape[2]
    p = int(pos.item()) if isinstance(pos, torch.Tensor) else int(pos)
    if p + n > k_buf.shape[2]:
        raise RuntimeError(f"InplaceLayer overflow: pos {p} + new {n} > buffer {k_buf.shape[2]}")
    k_buf[:, :, p:p + n] = k_new
    v_buf[:, :, p:p + n] = v_new


@pytest.fixture
def fake_kernel(monkeypatch):
    monkeypatch.setattr(cache_mod, "kv_append", _fake_kv_append)


def _dyn(b=2, h=3, base=5, d=8, layers=2, seed=0):
    g = torch.Generator().manual_seed(seed)
    dyn = DynamicCache()
    ks = []
    for i in range(layers):
        k = torch.randn(b, h, base, d, generator=g)
        v = torch.randn(b, h, base, d, generator=g)
        dyn.update(k, v, i)
        ks.append((k, v))
    return dyn, ks


def test_real_append_refuses_cpu_tensors():
    from umic_b200.kernels import kv_append

    z = torch.zeros(1, 1, 4, 8, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="no CPU path"):
        kv_append(z, z, z[:, :, :1], z[:, :, :1], 0)


def test_append_crop_matches_oracle(fake_kernel):
    dyn, ks = _dyn()
    c = InplaceKVCache.from_dynamic(dyn, extra_tokens=4, margin=2)
    ref = oracle.KVCacheOracle(ks[0][0], ks[0][1], extra=4, margin=2)
    assert c.layers[0].capacity == ref.cap == 11
    g = torch.Generator().manual_seed(1)
    for n in (2, 1, 3):
        kn, vn = torch.randn(2, 3, n, 8, generator=g), torch.randn(2, 3, n, 8, generator=g)
        k, v = c.layers[0].update(kn, vn)
        rk, rv = ref.update(kn, vn)
        assert torch.equal(k, rk) and torch.equal(v, rv)
        assert c.get_seq_length() == ref.get_seq_length()
        c.crop(-1)
        ref.crop(-1)
        assert c.get_seq_length() == ref.get_seq_length()
    with pytest.raises(RuntimeError, match="overflow"):
        c.layers[0].update(torch.zeros(2, 3, 9, 8), torch.zeros(2, 3, 9, 8))
    assert c.get_seq_length() == ref.get_seq_length()  # failed append moved nothing


def test_views_not_copies(fake_kernel):
    dyn, _ = _dyn()
    c = InplaceKVCache.from_dynamic(dyn, extra_tokens=4)
    k, _ = c.layers[0].update(torch.ones(2, 3, 1, 8), torch.ones(2, 3, 1, 8))
    assert k.data_ptr() == c.layers[0].k_buf.data_ptr()  # a prefix view of the buffer


def test_graph_mode_writes_at_device_position(fake_kernel):
    dyn, _ = _dyn()
    c = InplaceKVCache.from_dynamic(dyn, extra_tokens=4)
    pos_t = torch.tensor([5])
    c.enable_graph_mode(pos_t)
    c.set_graph_len(6)
    kn = torch.full((2, 3, 1, 8), 7.0)
    k, _ = c.layers[0].update(kn, kn)
    assert k.shape[2] == 6 and torch.equal(k[:, :, 5:6], kn)
    c.set_pos(6)
    c.disable_graph_mode()
    assert c.get_seq_length() == 6 and c.layers[0].keys.shape[2] == 6


def test_allocate_then_prefill_and_crop(fake_kernel):
    c = InplaceKVCache.allocate(num_layers=3, batch=2, heads=2, head_dim=4, capacity=10,
                                device="cpu", dtype=torch.float32)
    assert c.get_seq_length() == 0
    x = torch.randn(2, 2, 7, 4)
    for lyr in c.layers:
        lyr.update(x, x)
    assert c.get_seq_length() == 7
    c.crop(0)
    assert c.get_seq_length() == 0 and c.layers[2].keys.shape[2] == 0


def test_repeat_cache_hook_converts_once_and_resyncs(fake_kernel):
    from torch import nn

    from umic_b200 import integrate

    seen = []

    class Expert(nn.Module):
        def forward(self, inputs_embeds=None, past_key_values=None):
            seen.append(past_key_values)
            return inputs_embeds

    ex = Expert()
    integrate.fuse_repeat_cache(ex, extra_tokens_hint=4)
    dyn, _ = _dyn()
    emb = torch.zeros(2, 3, 8)
    ex(inputs_embeds=emb, past_key_values=dyn)
    ex(inputs_embeds=emb, past_key_values=dyn)
    assert isinstance(seen[0], InplaceKVCache) and seen[0] is seen[1]
    assert seen[0].layers[0].capacity == 5 + 4 + 8
    seen[0].layers[0].update(torch.zeros(2, 3, 2, 8), torch.zeros(2, 3, 2, 8))
    ex(inputs_embeds=emb, past_key_values=dyn)  # re-sync: crop back to the caller's length
    assert seen[2].get_seq_length() == 5


def test_fuse_flow_graph_wraps_the_sampler_step_callables():
    """The reference's fuse_flow_graph contract: sample() receives its step callables
    wrapped in FlowStepGraph; the first `warmup` calls of a step run eagerly (no CUDA)."""
    from types import SimpleNamespace

    from umic_b200.graph import FlowStepGraph, fuse_flow_graph

    seen = {}

    def sample(x, step_fn=None, unguided_step_fn=None):
        seen["step"], seen["unguided"] = step_fn, unguided_step_fn
        t = torch.zeros(1)
        for _ in range(2):
            x = step_fn(x=x, t=t)
        return x

    model = SimpleNamespace(diffusion=SimpleNamespace(sample=sample))
    fuse_flow_graph(model, warmup=2)
    out = model.diffusion.sample(torch.ones(3), step_fn=lambda x, t: x * 2)
    assert isinstance(seen["step"], FlowStepGraph) and seen["unguided"] is None
    assert torch.equal(out, torch.full((3,), 4.0)) and seen["step"].graph is None
