"""GPU parity of the joint consumer and the elementwise gate against the CPU oracle.

* spmlp_gate: gated values bit-exact against the reference's gate modules
  restated in the oracle (ties at kappa, -0.0, NaN), and the 16x64 bitmap of the
  result bit-exact against the oracle's tile occupancy; in place and out of place.
* spmlp_joint: out = round(round(round(h W2^T + b2) + round(z Wo^T + bo)) + r)
  within the north-star tolerance of the oracle's restatement of the reference
  joint (runs/042-2026-09-20-pythia70m-sparse-scale/controls.py:19-26, pinned by
  golden vectors), for every skip mode, ragged T, with and without biases and
  residual; on tile-structured h the issued / skipped K16 counts equal the
  oracle's accounting.
* JointConsumer keeps the reference Joint's contract (ungated h and z in, both
  gates applied inside) and install_joint reproduces an unfused GPT-NeoX model.
"""
from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import bitmap as obit
from oracle import gates as og
from oracle import mlp as omlp

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}
DTYPES = [torch.float16, torch.bfloat16]


def _same(a: torch.Tensor, b: torch.Tensor) -> bool:
    """Equal values with NaN in the same places (-0.0 and 0.0 are both zeros)."""
    a, b = a.cpu().float(), b.cpu().float()
    nan = torch.isnan(a)
    return bool(torch.equal(nan, torch.isnan(b)) and torch.equal(a[~nan], b[~nan]))


def _layer(t, d, f, dtype, seed, density=0.1):
    g = torch.Generator().manual_seed(seed)
    h = torch.randn(t, f, generator=g)
    h = torch.where(torch.rand(t, f, generator=g) < density, h, torch.zeros(()))
    z = torch.randn(t, d, generator=g)
    w2 = torch.randn(d, f, generator=g) * (0.02 / 3.5)
    b2 = torch.randn(d, generator=g) * 0.02
    wo = torch.randn(d, d, generator=g) * 0.02
    bo = torch.randn(d, generator=g) * 0.02
    r = torch.randn(t, d, generator=g)
    return [v.to(dtype) for v in (h, z, w2, b2, wo, bo, r)]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("op,kappa", [("one_sided_threshold", 0.5), ("symmetric_threshold", 0.5),
                                      ("relu", None), ("identity", None)])
def test_gate_is_bit_exact_and_writes_the_bitmap(dtype, op, kappa):
    from sparsity_spillover_b200 import gates, ops

    spec = gates.resolve({"operator": op} if kappa is None else {"operator": op, "kappa": kappa})
    g = torch.Generator().manual_seed(3)
    x = torch.randn(1000, 512, generator=g)
    x[::7, ::5] = 0.5                 # ties at kappa survive the one-sided gate
    x[1, :8] = torch.tensor([-0.0, float("nan"), -0.5, 0.4999, 0.5001, -1.0, 1.0, 0.0])
    x[64:80, 128:192] = -2.0          # a tile the one-sided gate clears entirely
    x = x.to(dtype)
    k = spec.kappa_for(dtype)
    expect = {"one_sided_threshold": lambda v: og.one_sided(v, k), "symmetric_threshold": lambda v: og.symmetric(v, k),
              "relu": og.relu, "identity": lambda v: v.clone()}[op](x)
    bits = torch.empty(ops.tile_bits_size(*x.shape), dtype=torch.int32, device="cuda")
    out = ops.gate(x.cuda(), spec, bits=bits)
    assert _same(out, expect)
    np.testing.assert_array_equal(bits.cpu().numpy().view(np.uint32), obit.tile_bits(expect.float()))
    inplace = x.cuda()
    ops.gate(inplace, spec, out=inplace)
    assert _same(inplace, expect)


def test_gate_rejects_tile_gates_and_overlap():
    from sparsity_spillover_b200 import ops

    x = torch.zeros(64, 128, dtype=torch.float16, device="cuda")
    with pytest.raises(ValueError):
        ops.gate(x, {"operator": "gelu"})
    from sparsity_spillover_b200._lib import SpmlpError

    big = torch.zeros(64 * 128 + 64, dtype=torch.float16, device="cuda")
    with pytest.raises(SpmlpError, match="overlap"):
        ops.gate(big[:64 * 128].view(64, 128), {"operator": "relu"}, out=big[64:].view(64, 128))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("skip", [False, True, "fine"])
@pytest.mark.parametrize("t,d,f", [(1000, 512, 2048), (4096, 256, 1024)])
def test_joint_matches_oracle(dtype, skip, t, d, f):
    from sparsity_spillover_b200 import ops

    h, z, w2, b2, wo, bo, r = _layer(t, d, f, dtype, seed=t + d)
    bits = ops.tile_bits_from_h(h.cuda())
    out = ops.joint(h.cuda(), bits, z.cuda(), w2.cuda(), b2.cuda(), wo.cuda(), bo.cuda(), r.cuda(), skip=skip)
    ref = omlp.joint(h, z, w2, b2, wo, bo, r, 0.0, 0.0, False, False)
    assert omlp.max_rel_error(out.cpu(), ref) <= TOL[dtype]


@pytest.mark.parametrize("dtype", DTYPES)
def test_joint_without_biases_or_residual(dtype):
    from sparsity_spillover_b200 import ops

    h, z, w2, _, wo, _, _ = _layer(512, 512, 2048, dtype, seed=9)
    out = ops.joint(h.cuda(), ops.tile_bits_from_h(h.cuda()), z.cuda(), w2.cuda(), None, wo.cuda(), None, None)
    a = omlp.linear(h, w2, None).to(dtype)
    b = omlp.linear(z, wo, None).to(dtype)
    ref = (a.float() + b.float()).to(dtype)
    assert omlp.max_rel_error(out.cpu(), ref) <= TOL[dtype]


@pytest.mark.parametrize("skip", [True, "fine"])
def test_joint_skips_dead_tiles_of_h_and_counts_them(skip):
    from sparsity_spillover_b200 import ops, workloads

    dtype, t, d, f = torch.bfloat16, 4096, 512, 2048
    h, _ = workloads.tile_structured_h(t, f, 0.2, seed=11, device="cpu")
    _, z, w2, b2, wo, bo, r = _layer(t, d, f, dtype, seed=12)
    h = h.to(dtype)
    bits = ops.tile_bits_from_h(h.cuda())
    stats = torch.zeros(2, dtype=torch.int64, device="cuda")
    out = ops.joint(h.cuda(), bits, z.cuda(), w2.cuda(), b2.cuda(), wo.cuda(), bo.cuda(), r.cuda(), skip=skip,
                    stats=stats)
    ref = omlp.joint(h, z, w2, b2, wo, bo, r, 0.0, 0.0, False, False)
    assert omlp.max_rel_error(out.cpu(), ref) <= TOL[dtype]
    mask = obit.tile_mask(h.float(), 16, 64)
    issued, skipped = obit.skip_counts(mask, f, n_tiles=d // 256, m_tile=ops.down_tile_tokens(skip))
    assert stats.cpu().tolist() == [issued, skipped]
    assert skipped > 0


@pytest.mark.parametrize("skip", [True, "fine"])
def test_joint_last_round_split_items_match_the_oracle(skip):
    """At T=32768, d=512 the joint's persistent grid runs its last round of tiles as
    half-width items (both products, both column halves): the final token blocks match
    the oracle, and the issued / skipped counters equal the oracle's accounting over
    all tokens (tile-structured h, so whole K-blocks are skipped)."""
    from sparsity_spillover_b200 import ops, workloads

    dtype, t, d, f = torch.bfloat16, 32768, 512, 2048
    h, _ = workloads.tile_structured_h(t, f, 0.3, seed=21, device="cuda", dtype=dtype)
    g = torch.Generator().manual_seed(22)
    z = torch.randn(t, d, generator=g).to(dtype)
    w2 = (torch.randn(d, f, generator=g) * 0.02).to(dtype)
    b2 = (torch.randn(d, generator=g) * 0.02).to(dtype)
    wo = (torch.randn(d, d, generator=g) * 0.02).to(dtype)
    bo = (torch.randn(d, generator=g) * 0.02).to(dtype)
    r = torch.randn(t, d, generator=g).to(dtype)
    bits = ops.tile_bits_from_h(h)
    stats = torch.zeros(2, dtype=torch.int64, device="cuda")
    out = ops.joint(h, bits, z.cuda(), w2.cuda(), b2.cuda(), wo.cuda(), bo.cuda(), r.cuda(), skip=skip, stats=stats)
    torch.cuda.synchronize()
    h_c = h.cpu()
    tail = slice(t - 4096, t)
    ref = omlp.joint(h_c[tail], z[tail], w2, b2, wo, bo, r[tail], 0.0, 0.0, False, False)
    assert omlp.max_rel_error(out.cpu()[tail], ref) <= TOL[dtype]
    head = slice(0, 1024)
    ref0 = omlp.joint(h_c[head], z[head], w2, b2, wo, bo, r[head], 0.0, 0.0, False, False)
    assert omlp.max_rel_error(out.cpu()[head], ref0) <= TOL[dtype]
    issued, skipped = obit.skip_counts(obit.tile_mask(h_c.float(), 16, 64), f, n_tiles=d // 256,
                                       m_tile=ops.down_tile_tokens(skip))
    assert stats.cpu().tolist() == [issued, skipped]


class FixedOneSidedThreshold(torch.nn.Module):  # the reference gate module's name, attribute and rule
    def __init__(self, kappa):
        super().__init__()
        self.kappa = kappa

    def forward(self, x):
        return x.masked_fill(x < self.kappa, 0)


@pytest.mark.parametrize("dtype", DTYPES)
def test_joint_consumer_keeps_the_reference_contract(dtype):
    """Joint(layer)(h, z, residual) with ungated h and z: both gates applied inside."""
    from sparsity_spillover_b200 import JointConsumer

    t, d, f = 768, 512, 2048
    g = torch.Generator().manual_seed(21)
    h = torch.randn(t, f, generator=g).to(dtype)
    _, z, w2, b2, wo, bo, r = _layer(t, d, f, dtype, seed=22)
    lin2 = torch.nn.Linear(f, d).to(dtype).cuda()
    lino = torch.nn.Linear(d, d).to(dtype).cuda()
    with torch.no_grad():
        lin2.weight.copy_(w2)
        lin2.bias.copy_(b2)
        lino.weight.copy_(wo)
        lino.bias.copy_(bo)
    th, tz = 1.25, 0.5
    layer = SimpleNamespace(mlp=SimpleNamespace(dense_4h_to_h=lin2, act=FixedOneSidedThreshold(th)),
                            attention=SimpleNamespace(dense=lino, z_gate=FixedOneSidedThreshold(tz)))
    joint = JointConsumer(layer)
    assert joint.gh and joint.gz and joint.th == th and joint.tz == tz
    with torch.inference_mode():
        out = joint(h.cuda().view(3, 256, f), z.cuda().view(3, 256, d), r.cuda().view(3, 256, d))
    assert out.shape == (3, 256, d)
    ref = omlp.joint(h, z, w2, b2, wo, bo, r, og.round_kappa(th, dtype), og.round_kappa(tz, dtype), True, True)
    assert omlp.max_rel_error(out.reshape(t, d).cpu(), ref) <= TOL[dtype]


def test_install_joint_reproduces_the_unfused_model():
    import transformers

    from sparsity_spillover_b200 import install_joint

    cfg = transformers.GPTNeoXConfig(hidden_size=256, intermediate_size=1024, num_hidden_layers=2,
                                     num_attention_heads=4, vocab_size=512, use_parallel_residual=True,
                                     attn_implementation="eager")
    torch.manual_seed(5)
    model = transformers.GPTNeoXForCausalLM(cfg).to(torch.bfloat16).cuda().eval()
    for layer in model.gpt_neox.layers:
        layer.mlp.act = FixedOneSidedThreshold(0.05)
        with torch.no_grad():
            layer.mlp.dense_h_to_4h.bias.normal_(0, 0.02)
    ids = torch.randint(0, 512, (2, 128), device="cuda")
    with torch.inference_mode():
        ref = model.gpt_neox(ids, use_cache=False).last_hidden_state.float()
        meta = install_joint(model)
        out = model.gpt_neox(ids, use_cache=False).last_hidden_state.float()
    assert meta["gates"][0]["h"]["operator"] == "one_sided_threshold"
    assert omlp.max_rel_error(out.cpu(), ref.cpu()) <= 2 * TOL[torch.bfloat16]
