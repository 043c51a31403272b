"""CPU tests of the HuggingFace patch (transformers 5.x).

The fast path normally needs CUDA; here it is enabled on CPU with the kernel
call replaced by the CPU oracle, so the routing, masking rules, GQA expansion
and fallbacks are checked without a GPU.  tests/test_patch_hf_gpu.py runs the
same models through the real kernels.
"""
import math

import pytest
import torch

from flash_attn_volta_b200 import patch_hf
from oracle.attention_oracle import attention_fwd
from tests.hf_models import tiny_model

FAMILIES = ["llama", "qwen2", "qwen3", "gpt2"]


def _oracle_flash_attn(q, k, v, causal=False, sm_scale=None):
    # the kernel's grouped-query contract: query head h reads K/V head h // group
    g = q.shape[2] // k.shape[2]
    k, v = k.repeat_interleave(g, dim=2), v.repeat_interleave(g, dim=2)
    o, _ = attention_fwd(q.float(), k.float(), v.float(), causal=causal, scale=sm_scale)
    return o.to(q.dtype)


@pytest.fixture
def cpu_fast_path(monkeypatch):
    calls = []

    def fake(q, k, v, causal=False, sm_scale=None):
        calls.append((tuple(q.shape), causal, sm_scale, k.shape[2]))
        return _oracle_flash_attn(q, k, v, causal, sm_scale)

    monkeypatch.setattr(patch_hf, "flash_attn", fake)
    monkeypatch.setattr(patch_hf, "_kernel_device_ok", lambda t: True)
    return calls


@pytest.mark.parametrize("family", FAMILIES)
@pytest.mark.parametrize("impl", ["sdpa", "eager"])
def test_patched_logits_match(family, impl, cpu_fast_path):
    model = tiny_model(family, impl)
    ids = torch.randint(0, 128, (2, 24), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = model(ids).logits
        fam, n = patch_hf.patch_model(model)
        assert fam == family and n == 2
        out = model(ids).logits
    assert len(cpu_fast_path) == 2  # one kernel call per layer
    assert all(c[1] for c in cpu_fast_path)  # causal
    assert (out - ref).abs().max() < 2e-2  # q/k/v are rounded to fp16 on the fast path
    assert patch_hf.unpatch_gpt2(model) + patch_hf.unpatch_qwen2(model) + \
        patch_hf.unpatch_qwen3(model) + patch_hf.unpatch_llama(model) == 2
    with torch.no_grad():
        assert torch.equal(model(ids).logits, ref)


def test_gqa_and_scale_forwarded(cpu_fast_path):
    model = tiny_model("llama")
    patch_hf.patch_llama(model)
    with torch.no_grad():
        model(torch.randint(0, 128, (1, 10)))
    shape, causal, scale, kv_heads = cpu_fast_path[0]
    assert shape == (1, 10, 4, 32)
    assert kv_heads == 2  # the 2 K/V heads reach the kernel unexpanded (grouped-query path)
    assert scale == pytest.approx(1 / math.sqrt(32))


def test_padding_mask_and_decode_fall_back(cpu_fast_path):
    model = tiny_model("qwen2")
    ids = torch.randint(0, 128, (2, 16), generator=torch.Generator().manual_seed(2))
    am = torch.ones_like(ids)
    am[0, :4] = 0  # left padding: not a pure causal mask
    with torch.no_grad():
        ref = model(ids, attention_mask=am).logits
        patch_hf.patch_qwen2(model)
        out = model(ids, attention_mask=am).logits
    assert len(cpu_fast_path) == 0
    assert torch.equal(out, ref)
    # prefill takes the fast path, the cached decode steps (q_len 1) fall back
    with torch.no_grad():
        gen = model.generate(ids[:1], max_new_tokens=4, do_sample=False)
    assert gen.shape == (1, 20)
    assert len(cpu_fast_path) == 2


def test_training_backward_through_patch(cpu_fast_path):
    model = tiny_model("llama").train()
    patch_hf.patch_llama(model)
    ids = torch.randint(0, 128, (2, 12))
    loss = model(ids, labels=ids).loss
    loss.backward()
    assert all(p.grad is not None for p in model.parameters() if p.requires_grad)


def test_is_causal_only_mask_forms():
    n = 6
    tri = torch.tril(torch.ones(n, n, dtype=torch.bool))
    assert patch_hf._is_causal_only_mask(tri[None, None], n)
    assert not patch_hf._is_causal_only_mask(torch.ones(1, 1, n, n, dtype=torch.bool), n)
    add = torch.zeros(1, 1, n, n).masked_fill(~tri, torch.finfo(torch.float32).min)
    assert patch_hf._is_causal_only_mask(add, n)
    assert not patch_hf._is_causal_only_mask(torch.zeros(1, 1, n, n), n)
    assert not patch_hf._is_causal_only_mask(add[:, :, :, :3], n)


def test_refuses_state_space_models():
    import transformers as T
    cfg = T.MambaConfig(vocab_size=64, hidden_size=32, num_hidden_layers=1, state_size=4)
    model = T.MambaForCausalLM(cfg)
    assert patch_hf._linear_attn_family(model) == "mamba"
    with pytest.raises(RuntimeError):
        patch_hf.patch_model(model)


def test_unknown_family():
    with pytest.raises(ValueError):
        patch_hf.patch_model(torch.nn.Linear(2, 2))
