"""Route HuggingFace transformers attention through the B200 kernels.

Drop-in for flash_attn_volta/patch_hf.py (public names kept: ``patch_gpt2``,
``patch_qwen2``, ``patch_qwen3``, ``patch_llama``, the ``unpatch_*``
counterparts, ``patch_model``, ``_is_causal_only_mask``,
``_linear_attn_family``), rewritten for the transformers 5.x module API.

The reference replaced each attention module's ``forward`` (or GPT-2's
``_attn``) with a copy that read ``self.num_heads`` / ``self.rotary_emb`` and
returned a 3-tuple (patch_hf.py:122-201, 425-480).  Transformers 5.x removed
those attributes: every attention module now computes q/k/v (rotary applied,
KV-cache updated) and hands ``(B, H, S, D)`` tensors to a function looked up by
``config._attn_implementation`` in ``AttentionInterface``.  So here the kernel
is registered once in that registry under ``IMPL_NAME``, and ``patch_*`` gives
each target attention module a private copy of its config that selects it.
Everything the module does around attention (projections, QK-norm, rotary,
cache, output projection) stays the model's own code.

The registered function keeps the reference's fast-path rules
(patch_hf.py:29-48, 63-71, 138-155): it calls ``flash_attn(..., causal=True)``
only for square self-attention (prefill / training; ``q_len == kv_len``) with no
mask or a pure causal mask, no attention-probability output, no attention
dropout, no sliding window and a supported head_dim on CUDA; anything else (a
KV-cache decode step, padding masks, cross-attention, ...) goes to the model's
original attention implementation.  GQA/MQA K/V go to the kernel with their
own head count (query head h reads K/V head h // group), where the reference
first expanded them to the query heads with ``repeat_kv`` (patch_hf.py:187-188).
"""
from __future__ import annotations

import copy
import sys
from typing import Optional, Tuple

import torch

from .autograd import flash_attn

IMPL_NAME = "flash_attn_volta_b200"


def _kernel_device_ok(t: torch.Tensor) -> bool:
    """Whether tensors on t's device can take the kernel path (CUDA only)."""
    return t.is_cuda


_FAMILIES = {
    "gpt2": {"GPT2Attention"},
    "qwen2": {"Qwen2Attention", "Qwen2SdpaAttention", "Qwen2FlashAttention2"},
    "qwen3": {"Qwen3Attention", "Qwen3SdpaAttention", "Qwen3FlashAttention2"},
    "llama": {"LlamaAttention", "LlamaSdpaAttention", "LlamaFlashAttention2"},
}


def _is_causal_only_mask(mask: torch.Tensor, q_len: int) -> bool:
    """True if ``mask`` (4-D, ``(.., q_len, kv_len >= q_len)``) is the plain causal
    mask on its top-left ``q_len x q_len`` block.

    Accepts both HF mask forms: additive float (0 kept, very negative masked;
    patch_hf.py:29-48 of the reference) and boolean (True = attend).
    """
    if mask is None:
        return True
    if mask.dim() != 4 or mask.size(-2) != q_len or mask.size(-1) < q_len:
        return False
    m = mask[..., :q_len, :q_len]
    tri = torch.tril(torch.ones(q_len, q_len, device=mask.device, dtype=torch.bool))
    if m.dtype == torch.bool:
        return bool(m[..., tri].all()) and not bool(m[..., ~tri].any())
    if (m[..., tri].abs() > 1e-3).any():
        return False
    if (m[..., ~tri] > -1.0).any():
        return False
    return True


def _original_attention(module, impl: str):
    """The attention function the module used before patching."""
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    if impl != "eager" and impl in ALL_ATTENTION_FUNCTIONS:
        return ALL_ATTENTION_FUNCTIONS[impl]
    return sys.modules[type(module).__module__].eager_attention_forward


def flash_attention_forward(module, query, key, value, attention_mask, scaling=None,
                            dropout: float = 0.0, **kwargs):
    """AttentionInterface function: (B, H, S, D) q/k/v -> ((B, S, H, D) out, None)."""
    q_len, kv_len = query.shape[-2], key.shape[-2]
    head_dim = query.shape[-1]
    fast = (
        _kernel_device_ok(query)
        and q_len == kv_len
        and head_dim in (16, 32, 64, 128)
        and value.shape[-1] == head_dim
        and getattr(module, "is_causal", True)
        and not getattr(module, "is_cross_attention", False)
        and not getattr(module, "reorder_and_upcast_attn", False)
        and not (dropout and module.training)
        and kwargs.get("sliding_window") is None
        and not kwargs.get("output_attentions", False)
        and kwargs.get("head_mask") is None
        and query.shape[1] % key.shape[1] == 0
        and _is_causal_only_mask(attention_mask, q_len)
    )
    if not fast:
        fn = _original_attention(module, module._fa_orig_impl)
        return fn(module, query, key, value, attention_mask, scaling=scaling, dropout=dropout,
                  **kwargs)
    # bf16 models stay in bf16 (the kernels take both); anything else runs in fp16
    dt = torch.bfloat16 if query.dtype == torch.bfloat16 else torch.float16
    q = query.transpose(1, 2).to(dt)
    k = key.transpose(1, 2).to(dt)
    v = value.transpose(1, 2).to(dt)
    sm_scale = float(scaling) if scaling is not None else head_dim ** -0.5
    out = flash_attn(q, k, v, causal=True, sm_scale=sm_scale)
    return out.to(query.dtype), None


def _register() -> None:
    from transformers import AttentionInterface
    AttentionInterface.register(IMPL_NAME, flash_attention_forward)


def _patch_family(model: torch.nn.Module, names: set) -> int:
    _register()
    n = 0
    for mod in model.modules():
        if type(mod).__name__ in names and hasattr(mod, "config"):
            if not hasattr(mod, "_fa_orig_config"):
                mod._fa_orig_config = mod.config
                mod._fa_orig_impl = mod.config._attn_implementation or "eager"
                cfg = copy.copy(mod.config)
                cfg._attn_implementation = IMPL_NAME
                mod.config = cfg
            n += 1
    return n


def _unpatch_family(model: torch.nn.Module, names: set) -> int:
    n = 0
    for mod in model.modules():
        if type(mod).__name__ in names and hasattr(mod, "_fa_orig_config"):
            mod.config = mod._fa_orig_config
            del mod._fa_orig_config
            del mod._fa_orig_impl
            n += 1
    return n


def patch_gpt2(model: torch.nn.Module) -> int:
    """Patch every GPT2Attention block on ``model``. Returns count patched."""
    return _patch_family(model, _FAMILIES["gpt2"])


def unpatch_gpt2(model: torch.nn.Module) -> int:
    return _unpatch_family(model, _FAMILIES["gpt2"])


def patch_qwen2(model: torch.nn.Module) -> int:
    """Patch every Qwen2 attention block on ``model``. Returns count patched."""
    return _patch_family(model, _FAMILIES["qwen2"])


def unpatch_qwen2(model: torch.nn.Module) -> int:
    return _unpatch_family(model, _FAMILIES["qwen2"])


def patch_qwen3(model: torch.nn.Module) -> int:
    """Patch every Qwen3 attention block (QK-norm stays the model's own code)."""
    return _patch_family(model, _FAMILIES["qwen3"])


def unpatch_qwen3(model: torch.nn.Module) -> int:
    return _unpatch_family(model, _FAMILIES["qwen3"])


def patch_llama(model: torch.nn.Module) -> int:
    """Patch every Llama attention block on ``model``. Returns count patched."""
    return _patch_family(model, _FAMILIES["llama"])


def unpatch_llama(model: torch.nn.Module) -> int:
    return _unpatch_family(model, _FAMILIES["llama"])


# Linear-attention / state-space models (patch_hf.py:353-387 of the reference):
# the kernel computes softmax attention only, so patch_model refuses these.
# Module class name -> the family reported in the refusal.
_NON_SOFTMAX_MIXERS = {
    "MambaMixer": "mamba",
    "Mamba2Mixer": "mamba2",
    "RwkvSelfAttention": "rwkv",
    "RwkvLinearAttention": "rwkv",
    "RecurrentGemmaRecurrentBlock": "recurrent_gemma",
    "RetNetAttention": "retnet",
}


def _linear_attn_family(model: torch.nn.Module) -> Optional[str]:
    """Family name (mamba / mamba2 / rwkv / recurrent_gemma / retnet) of a
    linear-attention or state-space model, else None."""
    for m in (model, *model.modules()):
        fam = _NON_SOFTMAX_MIXERS.get(type(m).__name__)
        if fam is not None:
            return fam
    return None


def patch_model(model: torch.nn.Module) -> Tuple[str, int]:
    """Detect the model family and patch it. Returns ``(family, n_patched)``.

    Raises RuntimeError for linear-attention / state-space architectures and
    ValueError for an unknown family (patch_hf.py:394-417 of the reference).
    """
    fam = _linear_attn_family(model)
    if fam is not None:
        raise RuntimeError(
            f"cannot patch a {fam} model: this library replaces softmax attention "
            "(multi-head or grouped-query) and the model mixes tokens with a "
            "linear-attention / state-space layer instead")
    present = {type(m).__name__ for m in model.modules()}
    for fam_name, patch in (("gpt2", patch_gpt2), ("qwen3", patch_qwen3),
                            ("qwen2", patch_qwen2), ("llama", patch_llama)):
        if present & _FAMILIES[fam_name]:
            return fam_name, patch(model)
    raise ValueError(f"no patch known for model class {type(model).__name__}")
