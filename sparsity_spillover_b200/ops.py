"""Tensor-level entry points over libspmlp.so, plus ``torch.ops.spmlp.*`` registrations.

Each function mirrors the reference's kernel-adapter contract
(runs/042-2026-09-20-pythia70m-sparse-scale/kernel/joint/joint.cu:141-149 TORCH_CHECKs,
candidate.py:26-33): CUDA tensors, contiguous, one device and dtype, launched on
the caller's current stream, errors raised as exceptions.  Inference only.
There is no CPU path: a tensor that is not on a CUDA device is an error.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .gates import OPERATORS, GateSpec, resolve

_DTYPES = {torch.float16: _lib.F16, torch.bfloat16: _lib.BF16}


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _check(name: str, t: torch.Tensor, dtype: torch.dtype | None, device: torch.device, shape=None) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a tensor")
    if t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")
    if dtype is not None and t.dtype != dtype:
        raise ValueError(f"{name} has dtype {t.dtype}, expected {dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if shape is not None and tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {tuple(shape)}")


def _device_dtype(x: torch.Tensor) -> tuple[torch.device, torch.dtype, int]:
    if not x.is_cuda:
        raise ValueError("libspmlp runs on CUDA tensors only (no CPU fallback)")
    if x.dtype not in _DTYPES:
        raise ValueError(f"unsupported dtype {x.dtype}; use float16 or bfloat16")
    return x.device, x.dtype, _DTYPES[x.dtype]


def tile_bits_size(tokens: int, features: int) -> int:
    return int(_lib.load().spmlp_tile_bits_size(tokens, features))


_COMPACT_MODES = {"compact": _lib.DOWN_COMPACT, "compact_fine": _lib.DOWN_COMPACT_FINE}


def _down_mode(skip: bool | str) -> int:
    if skip is False:
        return _lib.DOWN_DENSE
    if skip is True or skip == "coarse":
        return _lib.DOWN_SKIP
    if skip == "fine":
        return _lib.DOWN_SKIP_FINE
    if isinstance(skip, str) and skip in _COMPACT_MODES:
        return _COMPACT_MODES[skip]
    raise ValueError("skip must be True/'coarse', 'fine', 'compact', 'compact_fine' or False")


def _bits_size(skip: bool | str, tokens: int, features: int) -> int:
    """Words of the bitmap a down mode reads: 16x16 tiles for the compact modes, else 16x64."""
    if isinstance(skip, str) and skip in _COMPACT_MODES:
        return tile_bits16_size(tokens, features)
    return tile_bits_size(tokens, features)


def down_tile_tokens(skip: bool | str = True) -> int:
    """Tokens per down-projection tile for a skip setting: the granularity of
    K-block skipping and of the issued/skipped counters."""
    return int(_lib.load().spmlp_down_tile_tokens(_down_mode(skip)))


def tile_bits_words(features: int) -> int:
    return int(_lib.load().spmlp_tile_bits_words(features))


def tile_bits16_size(tokens: int, features: int) -> int:
    return int(_lib.load().spmlp_tile_bits16_size(tokens, features))


def tile_bits16_from_h(h: torch.Tensor, bits: torch.Tensor | None = None) -> torch.Tensor:
    """16x16 tile bitmap of h [T,F] (int32 words) for the compact down modes."""
    device, dtype, code = _device_dtype(h)
    _check("h", h, dtype, device)
    t, f = h.shape
    if bits is None:
        bits = torch.empty((tile_bits16_size(t, f),), device=device, dtype=torch.int32)
    _check("bits", bits, torch.int32, device, (tile_bits16_size(t, f),))
    with torch.cuda.device(device):
        _lib.call("spmlp_tile_bits16_from_h", _ptr(h), _ptr(bits), t, f, _stream(device))
    return bits


def tile_bits_from_h(h: torch.Tensor, bits: torch.Tensor | None = None) -> torch.Tensor:
    """16x64 tile bitmap of an existing h [T,F] (int32 words, layout of include/spmlp.h)."""
    device, dtype, code = _device_dtype(h)
    _check("h", h, dtype, device)
    t, f = h.shape
    if bits is None:
        bits = torch.empty((tile_bits_size(t, f),), device=device, dtype=torch.int32)
    _check("bits", bits, torch.int32, device, (tile_bits_size(t, f),))
    with torch.cuda.device(device):
        _lib.call("spmlp_tile_bits_from_h", _ptr(h), _ptr(bits), t, f, code, _stream(device))
    return bits


_MASK_ENCODINGS = {"raw": _lib.MASK_RAW, "runs": _lib.MASK_ROW_RUNS}


def encode_mask(bits: torch.Tensor, tokens: int, features: int, encoding: str = "raw") -> bytes:
    """Serialise a 16x64 tile bitmap (device or host int32[tile_bits_size(T, F)]) into the
    self-describing byte format of include/spmlp.h: "raw" words or lossless "runs" of
    identical 16-row groups."""
    if encoding not in _MASK_ENCODINGS:
        raise ValueError(f"encoding must be one of {sorted(_MASK_ENCODINGS)}")
    host = bits.detach().to("cpu", torch.int32).contiguous()
    if host.numel() != tile_bits_size(tokens, features):
        raise ValueError("bits does not match tile_bits_size(tokens, features)")
    code = _MASK_ENCODINGS[encoding]
    size = _lib.call_size("spmlp_mask_encoded_size", host.data_ptr(), tokens, features, code)
    out = (ctypes.c_uint8 * size)()
    _lib.call_size("spmlp_mask_encode", host.data_ptr(), tokens, features, code, ctypes.addressof(out), size)
    return bytes(out)


def decode_mask(data: bytes, device: torch.device | str | None = None) -> tuple[torch.Tensor, int, int]:
    """(bits, T, F) from a serialised bitmap; bits on ``device`` (host when None)."""
    buf = ctypes.create_string_buffer(bytes(data), len(data))
    t, f, enc = ctypes.c_int64(0), ctypes.c_int(0), ctypes.c_int(0)
    _lib.call("spmlp_mask_decode_header", ctypes.addressof(buf), len(data), ctypes.byref(t), ctypes.byref(f),
              ctypes.byref(enc))
    bits = torch.empty(tile_bits_size(t.value, f.value), dtype=torch.int32)
    _lib.call("spmlp_mask_decode", ctypes.addressof(buf), len(data), bits.data_ptr(), bits.numel())
    return (bits if device is None else bits.to(device)), t.value, f.value


def save_mask(path, bits: torch.Tensor, tokens: int, features: int, encoding: str = "raw") -> int:
    """Write a tile bitmap to ``path``; returns the bytes written."""
    data = encode_mask(bits, tokens, features, encoding)
    with open(path, "wb") as fh:
        fh.write(data)
    return len(data)


def load_mask(path, device: torch.device | str | None = None) -> tuple[torch.Tensor, int, int]:
    """(bits, T, F) read from a file written by ``save_mask``."""
    with open(path, "rb") as fh:
        return decode_mask(fh.read(), device)


def up_gate(x: torch.Tensor, w_in: torch.Tensor, b_in: torch.Tensor | None, gate=None, *,
            h: torch.Tensor | None = None, bits: torch.Tensor | None = None, z_out: torch.Tensor | None = None,
            seq_len: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """h = gate(round(x w_in^T + b_in)) and the 16x64 tile bitmap of h.

    x [T,d], w_in [F,d] (nn.Linear layout), b_in [F] or None.  ``gate`` is a
    GateSpec, a reference gate spec mapping, a reference gate module, or None
    (ungated A0: GELU).  z_out, when given, receives the pre-gate z.
    """
    device, dtype, code = _device_dtype(x)
    spec: GateSpec = resolve(gate)
    t, d = x.shape
    f = w_in.shape[0]
    _check("x", x, dtype, device)
    _check("w_in", w_in, dtype, device, (f, d))
    if b_in is not None:
        _check("b_in", b_in, dtype, device, (f,))
    if h is None:
        h = torch.empty((t, f), device=device, dtype=dtype)
    _check("h", h, dtype, device, (t, f))
    if bits is None:
        bits = torch.empty((tile_bits_size(t, f),), device=device, dtype=torch.int32)
    _check("bits", bits, torch.int32, device, (tile_bits_size(t, f),))
    if z_out is not None:
        _check("z_out", z_out, dtype, device, (t, f))
    with torch.cuda.device(device):
        _lib.call("spmlp_up_gate", _ptr(x), _ptr(w_in), _ptr(b_in), _ptr(h), _ptr(bits), _ptr(z_out),
                  t, d, f, code, spec.op, ctypes.c_float(spec.kappa_for(dtype)),
                  int(seq_len or t), _stream(device))
    return h, bits


class FoldedLayerNorm:
    """A LayerNorm folded into the linear layer it feeds (weight preparation, done once).

    For z = LN(x) W^T + b with LN(x) = (x - mean) * rstd * gamma + beta:
    z = rstd * (x (W diag(gamma))^T - mean * s) + c with s[f] = sum_k (W diag(gamma))[f, k]
    and c = b + W beta.  ``w_fold`` is stored in the activation dtype; ``s`` is summed
    from the stored (rounded) ``w_fold`` so the mean subtraction matches what the GEMM
    accumulates; ``s`` and ``c`` stay fp32.
    """

    def __init__(self, ln_weight: torch.Tensor | None, ln_bias: torch.Tensor | None, eps: float,
                 weight: torch.Tensor, bias: torch.Tensor | None, dtype: torch.dtype | None = None):
        dtype = dtype or weight.dtype
        w = weight.detach().float()
        gamma = torch.ones(w.shape[1], device=w.device) if ln_weight is None else ln_weight.detach().float()
        beta = torch.zeros(w.shape[1], device=w.device) if ln_bias is None else ln_bias.detach().float()
        self.w_fold = (w * gamma[None, :]).to(dtype).contiguous()
        self.s = self.w_fold.float().sum(dim=1).contiguous()
        c = w @ beta
        if bias is not None:
            c = c + bias.detach().float()
        self.c = c.contiguous()
        self.eps = float(eps)

    @classmethod
    def from_modules(cls, layer_norm: torch.nn.LayerNorm, linear: torch.nn.Linear, dtype=None) -> "FoldedLayerNorm":
        return cls(layer_norm.weight, layer_norm.bias, layer_norm.eps, linear.weight, linear.bias, dtype)


def row_stats(x: torch.Tensor, eps: float, mean: torch.Tensor | None = None,
              rstd: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-token LayerNorm statistics of x [T, d]: fp32 mean and 1/sqrt(var + eps)."""
    device, dtype, code = _device_dtype(x)
    t, d = x.shape
    _check("x", x, dtype, device)
    if mean is None:
        mean = torch.empty(t, device=device, dtype=torch.float32)
    if rstd is None:
        rstd = torch.empty(t, device=device, dtype=torch.float32)
    _check("mean", mean, torch.float32, device, (t,))
    _check("rstd", rstd, torch.float32, device, (t,))
    with torch.cuda.device(device):
        _lib.call("spmlp_row_stats", _ptr(x), _ptr(mean), _ptr(rstd), t, d, code, ctypes.c_float(eps), _stream(device))
    return mean, rstd


def up_gate_ln(x: torch.Tensor, folded: FoldedLayerNorm, gate=None, *, h: torch.Tensor | None = None,
               bits: torch.Tensor | None = None, z_out: torch.Tensor | None = None, seq_len: int | None = None,
               stats: tuple[torch.Tensor, torch.Tensor] | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """h = gate(LN(x) W_in^T + b_in) with the LayerNorm folded in: reads the raw x [T, d]."""
    spec = resolve(gate)
    device, dtype, code = _device_dtype(x)
    t, d = x.shape
    f = folded.w_fold.shape[0]
    _check("x", x, dtype, device)
    _check("w_fold", folded.w_fold, dtype, device, (f, d))
    _check("ln_s", folded.s, torch.float32, device, (f,))
    _check("ln_c", folded.c, torch.float32, device, (f,))
    mean, rstd = stats if stats is not None else row_stats(x, folded.eps)
    if h is None:
        h = torch.empty((t, f), device=device, dtype=dtype)
    if bits is None:
        bits = torch.empty((tile_bits_size(t, f),), device=device, dtype=torch.int32)
    _check("h", h, dtype, device, (t, f))
    _check("bits", bits, torch.int32, device, (tile_bits_size(t, f),))
    if z_out is not None:
        _check("z_out", z_out, dtype, device, (t, f))
    with torch.cuda.device(device):
        _lib.call("spmlp_up_gate_ln", _ptr(x), _ptr(folded.w_fold), _ptr(folded.s), _ptr(folded.c), _ptr(mean),
                  _ptr(rstd), _ptr(h), _ptr(bits), _ptr(z_out), t, d, f, code, spec.op,
                  ctypes.c_float(spec.kappa_for(dtype)), int(seq_len or t), _stream(device))
    return h, bits


def down_sparse(h: torch.Tensor, bits: torch.Tensor | None, w_out: torch.Tensor, b_out: torch.Tensor | None,
                residual: torch.Tensor | None = None, *, skip: bool | str = True, y: torch.Tensor | None = None,
                stats: torch.Tensor | None = None) -> torch.Tensor:
    """y = round(h w_out^T + b_out) [then round(y + residual)], skipping dead 16x64 K-tiles.

    h [T,F], w_out [d,F], b_out [d] or None, residual [T,d] or None.
    skip: True / "coarse" (256-token tiles on CTA pairs), "fine" (128-token tiles,
    finer skipping for token-blocked zeros), "compact" / "compact_fine" (the same
    tiles gathering only live 16-feature granules; ``bits`` is then the 16x16 bitmap
    of ``tile_bits16_from_h``) or False (dense).
    stats: optional int64[2] device tensor accumulating issued / skipped K16 steps.
    """
    device, dtype, code = _device_dtype(h)
    t, f = h.shape
    d = w_out.shape[0]
    _check("h", h, dtype, device)
    _check("w_out", w_out, dtype, device, (d, f))
    if b_out is not None:
        _check("b_out", b_out, dtype, device, (d,))
    if residual is not None:
        _check("residual", residual, dtype, device, (t, d))
    mode = _down_mode(skip)
    if mode != _lib.DOWN_DENSE:
        if bits is None:
            raise ValueError("skipping needs the tile bitmap")
        _check("bits", bits, torch.int32, device, (_bits_size(skip, t, f),))
    if y is None:
        y = torch.empty((t, d), device=device, dtype=dtype)
    _check("y", y, dtype, device, (t, d))
    if stats is not None:
        _check("stats", stats, torch.int64, device, (2,))
    with torch.cuda.device(device):
        _lib.call("spmlp_down_sparse", _ptr(h), _ptr(bits) if mode != _lib.DOWN_DENSE else None, _ptr(w_out),
                  _ptr(b_out), _ptr(residual), _ptr(y), t, f, d, code, mode, _ptr(stats), _stream(device))
    return y


def _pointer_array(ptrs: list[int]):
    arr = (ctypes.c_void_p * len(ptrs))(*ptrs)
    return ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p)), arr


def down_scatter(h: torch.Tensor, bits: torch.Tensor | None, w_out: torch.Tensor, slots: list[int], *,
                 skip: bool | str = True, stats: torch.Tensor | None = None) -> None:
    """Partial down projection of a d_ff slice, scattered by token block: the rounded
    partial of tokens [j T/w, (j+1) T/w) is stored at device address ``slots[j]``
    (this rank's slot in rank j's receive buffer, typically peer memory)."""
    device, dtype, code = _device_dtype(h)
    t, f = h.shape
    d = w_out.shape[0]
    _check("h", h, dtype, device)
    _check("w_out", w_out, dtype, device, (d, f))
    mode = _down_mode(skip)
    if mode != _lib.DOWN_DENSE:
        if bits is None:
            raise ValueError("skipping needs the tile bitmap")
        _check("bits", bits, torch.int32, device, (tile_bits_size(t, f),))
    if stats is not None:
        _check("stats", stats, torch.int64, device, (2,))
    arr, keep = _pointer_array([int(v) for v in slots])
    with torch.cuda.device(device):
        _lib.call("spmlp_down_scatter", _ptr(h), _ptr(bits) if mode != _lib.DOWN_DENSE else None, _ptr(w_out), arr,
                  len(slots), t, f, d, code, mode, _ptr(stats), _stream(device))
    del keep


def reduce_broadcast(recv: torch.Tensor, b_out: torch.Tensor | None, residual: torch.Tensor | None,
                     targets: list[int]) -> None:
    """y = round(round(sum_r recv[r] + b_out) + residual) for recv [world, rows, d],
    written to each device address in ``targets`` (rows x d each)."""
    device, dtype, code = _device_dtype(recv)
    world, rows, d = recv.shape
    _check("recv", recv, dtype, device)
    if b_out is not None:
        _check("b_out", b_out, dtype, device, (d,))
    if residual is not None:
        _check("residual", residual, dtype, device, (rows, d))
    arr, keep = _pointer_array([int(v) for v in targets])
    with torch.cuda.device(device):
        _lib.call("spmlp_reduce_broadcast", _ptr(recv), world, rows, d, _ptr(b_out), _ptr(residual), arr, len(targets),
                  code, _stream(device))
    del keep


def reduce_broadcast_multicast(mc_part: int, mc_x: int, rows: int, d: int, b_out: torch.Tensor | None,
                               residual: torch.Tensor | None, dtype: torch.dtype, device: torch.device) -> None:
    """The d_ff split's reduction + broadcast through NVSwitch multicast (include/spmlp.h):
    ``mc_part`` / ``mc_x`` are this rank's block addresses in the multicast mappings of the
    partial buffer and of the next layer's input; ``residual`` is the block in the local copy."""
    code = _DTYPES[dtype] if dtype in _DTYPES else None
    if code is None:
        raise TypeError(f"unsupported dtype {dtype}")
    if b_out is not None:
        _check("b_out", b_out, dtype, device, (d,))
    if residual is not None:
        _check("residual", residual, dtype, device, (rows, d))
    if not mc_part or not mc_x:
        raise ValueError("multicast addresses must be nonzero")
    with torch.cuda.device(device):
        _lib.call("spmlp_reduce_broadcast_multicast", int(mc_part), int(mc_x), _ptr(residual), int(rows), int(d),
                  _ptr(b_out), code, _stream(device))


def peer_barrier(peer_slots: list[int], local_flags: torch.Tensor, epoch: int) -> None:
    """Device-side barrier of the fused d_ff split over NVLink (see include/spmlp.h)."""
    device = local_flags.device
    _check("local_flags", local_flags, torch.int64, device, (len(peer_slots),))
    arr, keep = _pointer_array([int(v) for v in peer_slots])
    with torch.cuda.device(device):
        _lib.call("spmlp_peer_barrier", arr, _ptr(local_flags), len(peer_slots), int(epoch), _stream(device))
    del keep


def joint(h: torch.Tensor, bits: torch.Tensor | None, z: torch.Tensor, w2: torch.Tensor, b2: torch.Tensor | None,
          wo: torch.Tensor, bo: torch.Tensor | None, residual: torch.Tensor | None = None, *,
          skip: bool | str = True, out: torch.Tensor | None = None,
          stats: torch.Tensor | None = None) -> torch.Tensor:
    """out = round(round(round(h w2^T + b2) + round(z wo^T + bo)) + residual) in one kernel.

    The joint consumer of a GPT-NeoX layer with parallel residual: h [T,F] (already
    gated; bits its 16x64 tile bitmap), z [T,d] the attention context before its
    output projection, w2 [d,F] / b2 [d] (dense_4h_to_h), wo [d,d] / bo [d]
    (attention.dense), residual [T,d].  skip and stats as in ``down_sparse`` (the
    z branch is dense).
    """
    device, dtype, code = _device_dtype(h)
    t, f = h.shape
    d = w2.shape[0]
    _check("h", h, dtype, device)
    _check("z", z, dtype, device, (t, d))
    _check("w2", w2, dtype, device, (d, f))
    _check("wo", wo, dtype, device, (d, d))
    if b2 is not None:
        _check("b2", b2, dtype, device, (d,))
    if bo is not None:
        _check("bo", bo, dtype, device, (d,))
    if residual is not None:
        _check("residual", residual, dtype, device, (t, d))
    mode = _down_mode(skip)
    if mode != _lib.DOWN_DENSE:
        if bits is None:
            raise ValueError("skipping needs the tile bitmap")
        _check("bits", bits, torch.int32, device, (tile_bits_size(t, f),))
    if out is None:
        out = torch.empty((t, d), device=device, dtype=dtype)
    _check("out", out, dtype, device, (t, d))
    if stats is not None:
        _check("stats", stats, torch.int64, device, (2,))
    with torch.cuda.device(device):
        _lib.call("spmlp_joint", _ptr(h), _ptr(bits) if mode != _lib.DOWN_DENSE else None, _ptr(z), _ptr(w2),
                  _ptr(b2), _ptr(wo), _ptr(bo), _ptr(residual), _ptr(out), t, f, d, code, mode, _ptr(stats),
                  _stream(device))
    return out


_ELEMENTWISE_GATES = (_lib.GATE_IDENTITY, _lib.GATE_ONE_SIDED, _lib.GATE_SYMMETRIC, _lib.GATE_RELU)


def gate(x: torch.Tensor, gate, *, out: torch.Tensor | None = None,
         bits: torch.Tensor | None = None) -> torch.Tensor:
    """out = gate(x) for an elementwise gate (identity, one-sided, symmetric, ReLU);
    ``out=x`` gates in place.  With ``bits`` (int32[tile_bits_size(T, F)]) the 16x64
    tile bitmap of the result is written too."""
    spec = resolve(gate)
    if spec.op not in _ELEMENTWISE_GATES:
        raise ValueError(f"spmlp gate takes an elementwise threshold gate or ReLU, not {spec.operator!r}")
    device, dtype, code = _device_dtype(x)
    t, f = x.shape
    _check("x", x, dtype, device)
    if out is None:
        out = torch.empty_like(x)
    _check("out", out, dtype, device, (t, f))
    if bits is not None:
        _check("bits", bits, torch.int32, device, (tile_bits_size(t, f),))
    with torch.cuda.device(device):
        _lib.call("spmlp_gate", _ptr(x), _ptr(out), _ptr(bits), t, f, code, spec.op,
                  ctypes.c_float(spec.kappa_for(dtype)), _stream(device))
    return out


def mlp_forward(x: torch.Tensor, w_in: torch.Tensor, b_in: torch.Tensor | None, w_out: torch.Tensor,
                b_out: torch.Tensor | None, gate=None, *, residual: torch.Tensor | None = None, skip: bool | str = True,
                h: torch.Tensor | None = None, bits: torch.Tensor | None = None, y: torch.Tensor | None = None,
                stats: torch.Tensor | None = None, seq_len: int | None = None) -> torch.Tensor:
    """GPTNeoXMLP.forward with a fused gate: both kernels, h/bits as reusable workspace."""
    h, bits = up_gate(x, w_in, b_in, gate, h=h, bits=bits, seq_len=seq_len)
    return down_sparse(h, bits, w_out, b_out, residual, skip=skip, y=y, stats=stats)


def head_support_words(d: int) -> int:
    return int(_lib.load().spmlp_head_support_words(d))


def head_prepare(x: torch.Tensor, kappa: float, dtype: torch.dtype = torch.float16, *,
                 x_out: torch.Tensor | None = None, support: torch.Tensor | None = None):
    """fp32 head input -> (dtype input with dead 16x16 tiles zeroed, support bits).

    kappa is compared in fp32 (float(torch.tensor(kappa, dtype=float32)),
    runs/068-2026-10-08-pythia14m-aligned-vocabulary-tiles/inference/head.py:20-29).
    """
    if not x.is_cuda or x.dtype != torch.float32:
        raise ValueError("head_prepare takes a CUDA float32 input")
    if dtype not in _DTYPES:
        raise ValueError("dtype must be float16 or bfloat16")
    device = x.device
    t, d = x.shape
    _check("x", x, torch.float32, device)
    words = head_support_words(d)
    if x_out is None:
        x_out = torch.empty((t, d), device=device, dtype=dtype)
    _check("x_out", x_out, dtype, device, (t, d))
    if support is None:
        support = torch.empty(((t + 15) // 16) * words, device=device, dtype=torch.int32)
    _check("support", support, torch.int32, device, (((t + 15) // 16) * words,))
    k32 = float(torch.tensor(kappa, dtype=torch.float32))
    with torch.cuda.device(device):
        _lib.call("spmlp_head_prepare", _ptr(x), _ptr(x_out), _ptr(support), t, d, _DTYPES[dtype],
                  ctypes.c_float(k32), _stream(device))
    return x_out, support


def head_sparse(x: torch.Tensor, w_vocab: torch.Tensor, *, support: torch.Tensor | None = None,
                active_tiles: torch.Tensor | None = None, logits: torch.Tensor | None = None,
                stats: torch.Tensor | None = None) -> torch.Tensor:
    """logits = x w_vocab^T (embed_out), optionally K-gated (support) or N-gated (active_tiles)."""
    device, dtype, code = _device_dtype(x)
    t, d = x.shape
    v = w_vocab.shape[0]
    _check("x", x, dtype, device)
    _check("w_vocab", w_vocab, dtype, device, (v, d))
    if support is not None and active_tiles is not None:
        raise ValueError("give support (K gate) or active_tiles (N gate), not both")
    axis = _lib.HEAD_GATE_NONE
    n_active = 0
    if support is not None:
        axis = _lib.HEAD_GATE_K
        _check("support", support, torch.int32, device, (((t + 15) // 16) * head_support_words(d),))
    if active_tiles is not None:
        axis = _lib.HEAD_GATE_N
        _check("active_tiles", active_tiles, torch.int32, device)
        n_active = active_tiles.numel()
    if logits is None:
        logits = torch.empty((t, v), device=device, dtype=dtype)
    _check("logits", logits, dtype, device, (t, v))
    if stats is not None:
        _check("stats", stats, torch.int64, device, (2,))
    with torch.cuda.device(device):
        _lib.call("spmlp_head_sparse", _ptr(x), _ptr(support), _ptr(w_vocab), _ptr(logits), _ptr(active_tiles),
                  n_active, t, d, v, code, axis, _ptr(stats), _stream(device))
    return logits


def head_fill(logits: torch.Tensor, tiles: torch.Tensor, value: float) -> torch.Tensor:
    """Write ``value`` into the listed 128-column vocabulary tiles of logits."""
    device, dtype, code = _device_dtype(logits)
    t, v = logits.shape
    _check("logits", logits, dtype, device)
    _check("tiles", tiles, torch.int32, device)
    with torch.cuda.device(device):
        _lib.call("spmlp_head_fill", _ptr(logits), _ptr(tiles), tiles.numel(), t, v, code, ctypes.c_float(value),
                  _stream(device))
    return logits


def set_sm_count_target(sms: int, device: int | None = None) -> None:
    """Cap the persistent GEMMs launched afterwards on ``device`` at ``sms`` SMs (0 = all)."""
    dev = torch.cuda.current_device() if device is None else int(device)
    with torch.cuda.device(dev):
        _lib.call("spmlp_set_sm_count_target", int(sms))


def device_status(device: int | None = None) -> int:
    """Status word written by kernels that gave up on a bounded wait (0 = none)."""
    dev = torch.cuda.current_device() if device is None else int(device)
    out = ctypes.c_int(0)
    _lib.call("spmlp_device_status", dev, ctypes.byref(out))
    return out.value


def selftest_wait(device: int | None = None) -> None:
    """Launch the bounded-wait self-test (see include/spmlp.h) on the current stream."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
    with torch.cuda.device(dev):
        _lib.call("spmlp_selftest_wait", _stream(dev))


def clear_device_status(device: int | None = None) -> None:
    dev = torch.cuda.current_device() if device is None else int(device)
    _lib.call("spmlp_clear_device_status", dev)


# ---------------------------------------------------------------- torch.library ops
# Functional custom ops so the kernels appear as torch.ops.spmlp.* (e.g. inside
# user graphs); each allocates its outputs and calls the functions above.
_LIB = torch.library.Library("spmlp", "DEF")
_LIB.define("up_gate(Tensor x, Tensor w_in, Tensor? b_in, int gate_op, float kappa, int seq_len) -> (Tensor, Tensor)")
_LIB.define("down_sparse(Tensor h, Tensor? bits, Tensor w_out, Tensor? b_out, Tensor? residual, bool skip) -> Tensor")
_LIB.define("head_sparse(Tensor x, Tensor w_vocab, Tensor? support, Tensor? active_tiles) -> Tensor")
_LIB.define("joint(Tensor h, Tensor? bits, Tensor z, Tensor w2, Tensor? b2, Tensor wo, Tensor? bo, "
            "Tensor? residual, bool skip) -> Tensor")

_OP_NAMES = {v: k for k, v in OPERATORS.items()}


def _up_gate_op(x, w_in, b_in, gate_op, kappa, seq_len):
    op_name = _OP_NAMES[int(gate_op)]
    spec = GateSpec(op_name, int(gate_op), float(kappa))
    return up_gate(x, w_in, b_in, spec, seq_len=int(seq_len) or None)


def _down_sparse_op(h, bits, w_out, b_out, residual, skip):
    return down_sparse(h, bits, w_out, b_out, residual, skip=bool(skip))


def _head_sparse_op(x, w_vocab, support, active_tiles):
    return head_sparse(x, w_vocab, support=support, active_tiles=active_tiles)


_LIB.impl("up_gate", _up_gate_op, "CUDA")
_LIB.impl("down_sparse", _down_sparse_op, "CUDA")
_LIB.impl("head_sparse", _head_sparse_op, "CUDA")


def _joint_op(h, bits, z, w2, b2, wo, bo, residual, skip):
    return joint(h, bits, z, w2, b2, wo, bo, residual, skip=bool(skip))


_LIB.impl("joint", _joint_op, "CUDA")
