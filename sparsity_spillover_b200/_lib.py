"""ctypes binding of libspmlp.so (the C ABI declared in include/spmlp.h).

Loading fails loudly: there is no CPU or PyTorch fallback for any entry point.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

from .build import LIB

_c = ctypes
VP = _c.c_void_p
I64 = _c.c_int64
I32 = _c.c_int
F32 = _c.c_float

# name -> (restype, argtypes); mirrors include/spmlp.h one to one.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "spmlp_version": (I32, []),
    "spmlp_last_error": (_c.c_char_p, []),
    "spmlp_tile_bits_words": (I32, [I32]),
    "spmlp_down_tile_tokens": (I32, [I32]),
    "spmlp_tile_bits_size": (I64, [I64, I32]),
    "spmlp_mask_encoded_size": (I64, [VP, I64, I32, I32]),
    "spmlp_mask_encode": (I64, [VP, I64, I32, I32, VP, I64]),
    "spmlp_mask_decode_header": (I32, [VP, I64, _c.POINTER(I64), _c.POINTER(I32), _c.POINTER(I32)]),
    "spmlp_mask_decode": (I32, [VP, I64, VP, I64]),
    "spmlp_tile_bits_from_h": (I32, [VP, VP, I64, I32, I32, VP]),
    "spmlp_tile_bits16_words": (I32, [I32]),
    "spmlp_tile_bits16_size": (I64, [I64, I32]),
    "spmlp_tile_bits16_from_h": (I32, [VP, VP, I64, I32, VP]),
    "spmlp_up_gate": (I32, [VP, VP, VP, VP, VP, VP, I64, I32, I32, I32, I32, F32, I64, VP]),
    "spmlp_row_stats": (I32, [VP, VP, VP, I64, I32, I32, F32, VP]),
    "spmlp_up_gate_ln": (I32, [VP, VP, VP, VP, VP, VP, VP, VP, VP, I64, I32, I32, I32, I32, F32, I64, VP]),
    "spmlp_down_sparse": (I32, [VP, VP, VP, VP, VP, VP, I64, I32, I32, I32, I32, VP, VP]),
    "spmlp_down_scatter": (I32, [VP, VP, VP, _c.POINTER(VP), I32, I64, I32, I32, I32, I32, VP, VP]),
    "spmlp_reduce_broadcast": (I32, [VP, I32, I64, I32, VP, VP, _c.POINTER(VP), I32, I32, VP]),
    "spmlp_reduce_broadcast_multicast": (I32, [VP, VP, VP, I64, I32, VP, I32, VP]),
    "spmlp_peer_barrier": (I32, [_c.POINTER(VP), VP, I32, I64, VP]),
    "spmlp_joint": (I32, [VP, VP, VP, VP, VP, VP, VP, VP, VP, I64, I32, I32, I32, I32, VP, VP]),
    "spmlp_gate": (I32, [VP, VP, VP, I64, I32, I32, I32, F32, VP]),
    "spmlp_mlp_forward": (I32, [VP, VP, VP, VP, VP, VP, VP, VP, VP, I64, I32, I32, I32, I32, F32, I64, I32, VP, VP]),
    "spmlp_mlp_forward_noalloc": (I32, [VP, VP, VP, VP, VP, VP, VP, I64, I32, I32, I32, I32, F32, I64, I32, VP, VP]),
    "spmlp_head_support_words": (I32, [I32]),
    "spmlp_head_fill": (I32, [VP, VP, I32, I64, I32, I32, F32, VP]),
    "spmlp_head_prepare": (I32, [VP, VP, VP, I64, I32, I32, F32, VP]),
    "spmlp_head_sparse": (I32, [VP, VP, VP, VP, VP, I32, I64, I32, I32, I32, I32, VP, VP]),
    "spmlp_selftest_wait": (I32, [VP]),
    "spmlp_set_sm_count_target": (I32, [I32]),
    "spmlp_device_status": (I32, [I32, _c.POINTER(I32)]),
    "spmlp_clear_device_status": (I32, [I32]),
}

# Constants of include/spmlp.h.
F16, BF16 = 0, 1
GATE_IDENTITY, GATE_GELU, GATE_ONE_SIDED, GATE_SYMMETRIC, GATE_RELU, GATE_GELU_MASKED, GATE_CORNER = range(7)
DOWN_DENSE, DOWN_SKIP, DOWN_SKIP_FINE, DOWN_COMPACT, DOWN_COMPACT_FINE = 0, 1, 2, 3, 4
MASK_RAW, MASK_ROW_RUNS = 0, 1
HEAD_GATE_NONE, HEAD_GATE_K, HEAD_GATE_N = 0, 1, 2

_lib: ctypes.CDLL | None = None


class SpmlpError(RuntimeError):
    """A libspmlp entry point returned a nonzero status."""

    def __init__(self, name: str, code: int, message: str):
        super().__init__(f"{name} failed with status {code}: {message}")
        self.code = code


def library_path() -> Path:
    return LIB


def load() -> ctypes.CDLL:
    """Load libspmlp.so (built in-tree by ``__graft_entry__.build``)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB.exists():
        raise RuntimeError(
            f"{LIB} is missing: build it with `python -m sparsity_spillover_b200.build` "
            "(there is no CPU fallback)"
        )
    lib = ctypes.CDLL(str(LIB))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _lib = lib
    return lib


def call(name: str, *args) -> None:
    """Call an entry point and raise SpmlpError on a nonzero status."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != 0:
        raise SpmlpError(name, rc, lib.spmlp_last_error().decode(errors="replace"))


def call_size(name: str, *args) -> int:
    """Call an entry point that returns a byte count; raise SpmlpError when it is negative."""
    lib = load()
    n = getattr(lib, name)(*args)
    if n < 0:
        raise SpmlpError(name, n, lib.spmlp_last_error().decode(errors="replace"))
    return n


def exported_symbols() -> list[str]:
    return list(SIGNATURES)
