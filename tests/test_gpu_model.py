"""Whole-model drop-in on GPU: a GPT-NeoX model with the reference's gate at mlp.act,
switched to the sm_100a kernels with install(model) (and SparseHead for embed_out),
gives the logits of the unfused model within tolerance, for the prefill and for
cached decode steps (T = 1 token per call, the smallest shapes the kernels see)."""
from __future__ import annotations

import pytest
import torch

from oracle import mlp as omlp

pytestmark = pytest.mark.gpu


class FixedOneSidedThreshold(torch.nn.Module):  # the reference gate module's name, attribute and rule
    def __init__(self, kappa):
        super().__init__()
        self.kappa = kappa

    def forward(self, x):
        return x.masked_fill(x < self.kappa, 0)


def _model(dtype):
    import transformers

    cfg = transformers.GPTNeoXConfig(hidden_size=256, intermediate_size=1024, num_hidden_layers=3,
                                     num_attention_heads=4, vocab_size=1024, use_parallel_residual=True,
                                     attn_implementation="eager")
    torch.manual_seed(9)
    model = transformers.GPTNeoXForCausalLM(cfg).to(dtype).cuda().eval()
    for layer in model.gpt_neox.layers:
        layer.mlp.act = FixedOneSidedThreshold(0.05)
    return model


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_install_matches_unfused_model_for_prefill_and_decode(dtype):
    from sparsity_spillover_b200 import SparseHead, install

    model = _model(dtype)
    ids = torch.randint(0, 1024, (2, 96), device="cuda")
    nxt = torch.randint(0, 1024, (2, 1), device="cuda")
    with torch.inference_mode():
        ref = model(ids, use_cache=True)
        ref_step = model(nxt, past_key_values=ref.past_key_values, use_cache=True).logits.float()
        ref_logits = ref.logits.float()
        meta = install(model)
        model.embed_out = SparseHead(model.embed_out, dtype=dtype)
        out = model(ids, use_cache=True)
        step = model(nxt, past_key_values=out.past_key_values, use_cache=True).logits.float()
        step2 = model(step.argmax(-1)[:, -1:], past_key_values=out.past_key_values, use_cache=True).logits
    tol = {torch.float16: 4e-3, torch.bfloat16: 2e-2}[dtype]  # three layers and the head, each within its own bound
    assert meta["gates"][0]["operator"] == "one_sided_threshold"
    assert omlp.max_rel_error(out.logits.float().cpu(), ref_logits.cpu()) <= tol
    assert omlp.max_rel_error(step.cpu(), ref_step.cpu()) <= tol
    assert step2.shape == (2, 1, 1024) and bool(torch.isfinite(step2).all())


@pytest.mark.parametrize("mode", ["custom_sparse", "custom_no_skip", "dense"])
def test_install_head_matches_the_oracle_on_the_final_hidden_states(mode):
    """install_head(model, mode, config) as the reference's head installer: the fp32 model's
    final hidden states, their 16x16 corner certificates (custom modes) and an fp16 projection
    give the oracle's logits."""
    import transformers

    from oracle import head as ohead
    from sparsity_spillover_b200 import install_head

    cfg = transformers.GPTNeoXConfig(hidden_size=128, intermediate_size=512, num_hidden_layers=2,
                                     num_attention_heads=4, vocab_size=2048, attn_implementation="eager")
    torch.manual_seed(68)
    model = transformers.GPTNeoXForCausalLM(cfg).cuda().eval()
    kappa = 0.25
    model.config.head_input_gate = {"operator": "tile_corner_threshold", "kappa": kappa, "tile_tokens": 16,
                                    "tile_features": 16}
    ids = torch.randint(0, 2048, (1, 128), device="cuda")
    with torch.inference_mode():
        hidden = model.gpt_neox(ids).last_hidden_state.float().cpu()[0]
        meta = install_head(model, mode, {"kernel_tile_tokens": 16, "kernel_tile_vocabulary": 256})
        logits = model(ids).logits.float().cpu()[0]
    w = model.embed_out.weight.detach().cpu().half()
    if mode == "dense":
        ref = ohead.logits(hidden.half(), w)
    else:
        x_ref, _ = ohead.prepare(hidden, kappa, torch.float16)
        ref = ohead.logits(x_ref, w)
        assert meta["gate"]["kappa"] == kappa
    assert omlp.max_rel_error(logits, ref.float()) <= 2e-3
