"""HF models patched onto the B200 kernels vs the same models unpatched (fp16, CUDA)."""
import pytest
import torch

from flash_attn_volta_b200 import patch_hf
from tests.hf_models import tiny_model

pytestmark = pytest.mark.gpu

FAMILIES = ["llama", "qwen2", "qwen3", "gpt2"]


@pytest.mark.parametrize("family", FAMILIES)
@pytest.mark.parametrize("head_dim", [64, 128])
def test_logits_and_grads_match_unpatched(family, head_dim):
    dev = torch.device("cuda", 0)
    model = tiny_model(family, "sdpa", torch.float16, head_dim=head_dim).to(dev)
    ids = torch.randint(0, 128, (2, 200), generator=torch.Generator().manual_seed(3)).to(dev)

    def run():
        model.zero_grad(set_to_none=True)
        out = model(ids, labels=ids)
        out.loss.backward()
        g = torch.cat([p.grad.float().flatten() for p in model.parameters() if p.grad is not None])
        return out.logits.float().detach(), out.loss.item(), g

    ref_logits, ref_loss, ref_g = run()
    calls = []
    orig = patch_hf.flash_attn
    patch_hf.flash_attn = lambda *a, **k: calls.append(1) or orig(*a, **k)
    try:
        fam, n = patch_hf.patch_model(model)
        logits, loss, g = run()
    finally:
        patch_hf.flash_attn = orig
    assert fam == family and n == 2 and len(calls) == 2
    cos = torch.nn.functional.cosine_similarity(logits.flatten(), ref_logits.flatten(), dim=0)
    assert cos > 0.9999
    assert (logits - ref_logits).abs().max() < 2e-2
    assert abs(loss - ref_loss) < 1e-3
    gcos = torch.nn.functional.cosine_similarity(g, ref_g, dim=0)
    assert gcos > 0.999


@pytest.mark.parametrize("family", ["llama", "qwen3"])
def test_greedy_generation_unchanged(family):
    dev = torch.device("cuda", 0)
    model = tiny_model(family, "sdpa", torch.float16).to(dev)
    ids = torch.randint(0, 128, (1, 64), generator=torch.Generator().manual_seed(4)).to(dev)
    with torch.no_grad():
        ref = model.generate(ids, max_new_tokens=16, do_sample=False)
        patch_hf.patch_model(model)
        out = model.generate(ids, max_new_tokens=16, do_sample=False)
    assert (out == ref).float().mean() >= 0.95  # fp16 rounding may flip a late near-tie
