"""GPU parity of the folded LayerNorm prologue of the up projection.

* spmlp_row_stats: per-token mean and rstd within fp32 rounding of torch's.
* spmlp_up_gate_ln: z within the north-star tolerance of the fp32 oracle of
  dense_h_to_4h(post_attention_layernorm(x)) (rows with large mean offsets
  included), h exactly the gate of the kernel's own z, and the 16x64 bitmap
  exactly that of h.
* install_joint(fuse_layernorm=True) reproduces the unfused GPT-NeoX model.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import bitmap as obit
from oracle import gates as og
from oracle import mlp as omlp

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}


def _inputs(t, d, f, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(t, d, generator=g) + 4.0 * torch.randn(t, 1, generator=g)  # per-token offsets
    gamma = 1.0 + 0.1 * torch.randn(d, generator=g)
    beta = 0.1 * torch.randn(d, generator=g)
    w = torch.randn(f, d, generator=g) * 0.02
    b = torch.randn(f, generator=g) * 0.02
    return x.to(dtype), gamma.to(dtype), beta.to(dtype), w.to(dtype), b.to(dtype)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_row_stats_match_torch(dtype):
    from sparsity_spillover_b200 import ops

    x, *_ = _inputs(1000, 512, 64, dtype, seed=1)
    mean, rstd = ops.row_stats(x.cuda(), 1e-5)
    xf = x.double()
    ref_mean = xf.mean(1)
    ref_rstd = 1.0 / torch.sqrt(xf.var(1, unbiased=False) + 1e-5)
    assert torch.allclose(mean.cpu().double(), ref_mean, rtol=1e-5, atol=1e-5)
    assert torch.allclose(rstd.cpu().double(), ref_rstd, rtol=1e-5)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("gate", [{"operator": "one_sided_threshold", "kappa": 0.05}, {"operator": "gelu"}])
@pytest.mark.parametrize("t,d,f", [(1000, 512, 2048), (4096, 1024, 4096)])
def test_up_gate_ln_matches_the_unfused_oracle(dtype, gate, t, d, f):
    from sparsity_spillover_b200 import gates, ops

    x, gamma, beta, w, b = _inputs(t, d, f, dtype, seed=t + d)
    folded = ops.FoldedLayerNorm(gamma.cuda(), beta.cuda(), 1e-5, w.cuda(), b.cuda())
    z = torch.empty(t, f, dtype=dtype, device="cuda")
    h, bits = ops.up_gate_ln(x.cuda(), folded, gate, z_out=z)
    ref = omlp.layer_norm_linear(x, gamma, beta, 1e-5, w, b)
    assert omlp.max_rel_error(z.cpu(), ref) <= TOL[dtype]
    spec = gates.resolve(gate)
    h_k = h.cpu()
    if spec.op == og.GELU:  # erf GELU of the kernel's z, within the up projection tests' bound
        expect = og.apply(z.cpu().float(), spec.op).to(dtype)
        assert (h_k.float() - expect.float()).abs().max() <= 2 * og.ulp(float(expect.float().abs().max()), dtype)
    else:  # threshold gates: exactly the reference gate of the kernel's own z
        expect = og.apply(z.cpu(), spec.op, spec.kappa_for(dtype))
        assert torch.equal(h_k.view(torch.int16), expect.view(torch.int16))
    np.testing.assert_array_equal(bits.cpu().numpy().view(np.uint32), obit.tile_bits(h_k))


def test_install_joint_with_folded_layernorm():
    import transformers

    from sparsity_spillover_b200 import install_joint

    class FixedOneSidedThreshold(torch.nn.Module):
        def __init__(self, kappa):
            super().__init__()
            self.kappa = kappa

        def forward(self, x):
            return x.masked_fill(x < self.kappa, 0)

    cfg = transformers.GPTNeoXConfig(hidden_size=256, intermediate_size=1024, num_hidden_layers=2,
                                     num_attention_heads=4, vocab_size=512, use_parallel_residual=True,
                                     attn_implementation="eager")
    torch.manual_seed(6)
    model = transformers.GPTNeoXForCausalLM(cfg).to(torch.bfloat16).cuda().eval()
    for layer in model.gpt_neox.layers:
        layer.mlp.act = FixedOneSidedThreshold(0.05)
        with torch.no_grad():
            layer.post_attention_layernorm.weight.normal_(1.0, 0.1)
            layer.post_attention_layernorm.bias.normal_(0.0, 0.1)
    ids = torch.randint(0, 512, (2, 128), device="cuda")
    with torch.inference_mode():
        ref = model.gpt_neox(ids, use_cache=False).last_hidden_state.float()
        meta = install_joint(model, fuse_layernorm=True)
        out = model.gpt_neox(ids, use_cache=False).last_hidden_state.float()
    assert meta["fuse_layernorm"]
    assert omlp.max_rel_error(out.cpu(), ref.cpu()) <= 2 * TOL[torch.bfloat16]
