"""The allocation-free MLP forward, called through the C ABI.

spmlp_mlp_forward_noalloc serves callers that cannot allocate device memory at
the call (a global-mode CUDA graph capture, a framework whose allocator owns
the GPU's memory, a foreign-language host without a device allocator): its
workspace is a static device buffer inside the library.  These tests call it
through ctypes with raw device pointers and check, on two calls in a row, that
it returns what the allocating entry point spmlp_mlp_forward returns, within
the north-star tolerance (max|err| / max|ref| <= 2e-3 for fp16, 1e-2 for bf16).
The second call uses fewer tokens and different inputs, so stale workspace
contents from the first call (h or bitmap bits) would show up as errors.

They also check it against the CPU oracle (fp32 GEMMs, the reference gate on
the kernel's dtype-rounded z), and at the largest token count the static buffer holds
for F = 2048 (8191 tokens: 2*T*F bytes of h plus the bitmap within 32 MiB),
with one token more rejected.

This file sorts last so that a run stopping at its first failure has already
run every other test; it also passes on its own in a fresh process.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}
CODES = {torch.float16: 0, torch.bfloat16: 1}
ONE_SIDED, DOWN_SKIP = 2, 1


def _layer(t, d, f, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(t, d, generator=g, device="cuda").to(dtype)
    w_in = (torch.randn(f, d, generator=g, device="cuda") * 0.02).to(dtype)
    b_in = (torch.randn(f, generator=g, device="cuda") * 0.05).to(dtype)
    w_out = (torch.randn(d, f, generator=g, device="cuda") * 0.006).to(dtype)
    b_out = (torch.randn(d, generator=g, device="cuda") * 0.05).to(dtype)
    r = torch.randn(t, d, generator=g, device="cuda").to(dtype)
    return x, w_in, b_in, w_out, b_out, r


def _reference(lib, args, kappa, dtype):
    """The allocating entry point with caller-owned workspace."""
    x, w_in, b_in, w_out, b_out, r = args
    t, d = x.shape
    f = w_in.shape[0]
    y = torch.empty(t, d, dtype=dtype, device="cuda")
    h = torch.empty(t, f, dtype=dtype, device="cuda")
    bits = torch.empty(int(lib.spmlp_tile_bits_size(t, f)), dtype=torch.int32, device="cuda")
    rc = lib.spmlp_mlp_forward(x.data_ptr(), w_in.data_ptr(), b_in.data_ptr(), w_out.data_ptr(), b_out.data_ptr(),
                               r.data_ptr(), y.data_ptr(), h.data_ptr(), bits.data_ptr(), t, d, f, CODES[dtype],
                               ONE_SIDED, ctypes.c_float(kappa), t, DOWN_SKIP, None,
                               torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.spmlp_last_error()
    return y


def _noalloc(lib, args, kappa, dtype):
    x, w_in, b_in, w_out, b_out, r = args
    t, d = x.shape
    f = w_in.shape[0]
    y = torch.empty(t, d, dtype=dtype, device="cuda")
    rc = lib.spmlp_mlp_forward_noalloc(x.data_ptr(), w_in.data_ptr(), b_in.data_ptr(), w_out.data_ptr(),
                                       b_out.data_ptr(), r.data_ptr(), y.data_ptr(), t, d, f, CODES[dtype],
                                       ONE_SIDED, ctypes.c_float(kappa), t, DOWN_SKIP, None,
                                       torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.spmlp_last_error()
    return y


def _max_rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_noalloc_matches_allocating_entry_point_on_two_calls(lib, dtype):
    torch.cuda.init()
    kappa = float(torch.tensor(0.58, dtype=dtype))  # about 10% density for these inputs
    calls = [(_layer(4096, 512, 2048, dtype, seed=1), kappa), (_layer(1000, 512, 2048, dtype, seed=2), kappa)]
    for args, k in calls:
        y_ref = _reference(lib, args, k, dtype)
        y = _noalloc(lib, args, k, dtype)
        torch.cuda.synchronize()
        assert _max_rel(y, y_ref) <= TOL[dtype]
        assert torch.equal(y, y_ref)  # same kernels, same inputs: deterministic


def _oracle(lib, args, kappa, dtype):
    """fp32 oracle of the same forward, on the kernel's own rounded z (the parity
    convention of this library's tests: a z one ulp away from the oracle's can flip a
    gate decision at kappa, so the gate is applied to the z the up projection
    computed): h = one-sided gate of z, y = h w_out^T + b_out + r in fp32.  z comes
    from spmlp_up_gate's z_out through the C ABI."""
    from oracle import gates as og
    from oracle import mlp as omlp

    x, w_in, b_in, w_out, b_out, r = args
    t, d = x.shape
    f = w_in.shape[0]
    h = torch.empty(t, f, dtype=dtype, device="cuda")
    z = torch.empty(t, f, dtype=dtype, device="cuda")
    bits = torch.empty(int(lib.spmlp_tile_bits_size(t, f)), dtype=torch.int32, device="cuda")
    rc = lib.spmlp_up_gate(x.data_ptr(), w_in.data_ptr(), b_in.data_ptr(), h.data_ptr(), bits.data_ptr(),
                           z.data_ptr(), t, d, f, CODES[dtype], ONE_SIDED, ctypes.c_float(kappa), t,
                           torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.spmlp_last_error()
    torch.cuda.synchronize()
    z_c = z.cpu()
    assert _max_rel(z_c, omlp.linear(x.cpu(), w_in.cpu(), b_in.cpu())) <= TOL[dtype]
    h_ref = og.apply(z_c, og.ONE_SIDED, kappa)
    return omlp.down_from_h(h_ref, w_out.cpu(), b_out.cpu(), residual=r.cpu())


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_noalloc_matches_the_oracle_up_to_the_buffer_limit(lib, dtype):
    torch.cuda.init()
    kappa = float(torch.tensor(0.58, dtype=dtype))
    for t in (8191, 513):  # 8191 tokens fill the 32 MiB buffer at F = 2048; then a smaller call
        args = _layer(t, 512, 2048, dtype, seed=t)
        y = _noalloc(lib, args, kappa, dtype)
        torch.cuda.synchronize()
        assert _max_rel(y.cpu(), _oracle(lib, args, kappa, dtype)) <= TOL[dtype]
    args = _layer(8192, 512, 2048, dtype, seed=5)
    x, w_in, b_in, w_out, b_out, r = args
    y = torch.empty(8192, 512, dtype=dtype, device="cuda")
    rc = lib.spmlp_mlp_forward_noalloc(x.data_ptr(), w_in.data_ptr(), b_in.data_ptr(), w_out.data_ptr(),
                                       b_out.data_ptr(), r.data_ptr(), y.data_ptr(), 8192, 512, 2048, CODES[dtype],
                                       ONE_SIDED, ctypes.c_float(kappa), 8192, DOWN_SKIP, None,
                                       torch.cuda.current_stream().cuda_stream)
    assert rc == -2  # one token past the limit: SPMLP_ESHAPE, nothing launched


def test_noalloc_rejects_sizes_beyond_the_static_buffer(lib):
    torch.cuda.init()
    args = _layer(64, 512, 2048, torch.float16, seed=3)
    x, w_in, b_in, w_out, b_out, r = args
    too_many_tokens = 1 << 20  # 2 * T * F bytes far above the buffer: rejected before any launch
    y = torch.empty(64, 512, dtype=torch.float16, device="cuda")
    rc = lib.spmlp_mlp_forward_noalloc(x.data_ptr(), w_in.data_ptr(), b_in.data_ptr(), w_out.data_ptr(),
                                       b_out.data_ptr(), r.data_ptr(), y.data_ptr(), too_many_tokens, 512, 2048, 0,
                                       ONE_SIDED, ctypes.c_float(0.5), too_many_tokens, DOWN_SKIP, None,
                                       torch.cuda.current_stream().cuda_stream)
    assert rc == -2  # SPMLP_ESHAPE
    assert b"static buffer" in lib.spmlp_last_error()
