"""Tiny random-init HF models of each patched family (no downloads)."""
import torch


def tiny_model(family, impl="sdpa", dtype=torch.float32, head_dim=32):
    import transformers as T
    common = dict(vocab_size=128, num_hidden_layers=2)
    if family == "llama":
        cfg = T.LlamaConfig(hidden_size=4 * head_dim, intermediate_size=256, num_attention_heads=4,
                            num_key_value_heads=2, head_dim=head_dim, **common)
        cls = T.LlamaForCausalLM
    elif family == "qwen2":
        cfg = T.Qwen2Config(hidden_size=4 * head_dim, intermediate_size=256, num_attention_heads=4,
                            num_key_value_heads=1, **common)
        cls = T.Qwen2ForCausalLM
    elif family == "qwen3":
        cfg = T.Qwen3Config(hidden_size=4 * head_dim, intermediate_size=256, num_attention_heads=4,
                            num_key_value_heads=2, head_dim=head_dim, **common)
        cls = T.Qwen3ForCausalLM
    elif family == "gpt2":
        cfg = T.GPT2Config(n_embd=4 * head_dim, n_head=4, n_layer=2, vocab_size=128,
                           n_positions=512)
        cls = T.GPT2LMHeadModel
    else:
        raise ValueError(family)
    cfg._attn_implementation = impl
    torch.manual_seed(0)
    return cls(cfg).to(dtype).eval()
