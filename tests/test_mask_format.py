"""The persisted tile-bitmap format (host code of libspmlp.so, no GPU needed):
lossless round trips in both encodings against the oracle's packed bitmap, the
header fields, and rejection of malformed or corrupted input."""
from __future__ import annotations

import struct

import numpy as np
import pytest
import torch

from oracle import bitmap as obit


def _bits_of(mask: np.ndarray) -> torch.Tensor:
    """Packed kernel-layout words of a boolean [row_groups, tiles] mask, via the oracle."""
    return torch.from_numpy(obit.pack_bits(mask).reshape(-1).view(np.int32).copy())


@pytest.mark.parametrize("encoding", ["raw", "runs"])
@pytest.mark.parametrize("t,f,p", [(4096, 2048, 0.1), (1000, 320, 0.5), (16, 64, 1.0), (17, 4096, 0.02),
                                   (512, 2048, 0.0)])
def test_round_trip_is_lossless(encoding, t, f, p):
    from sparsity_spillover_b200 import ops

    rng = np.random.default_rng(t + f)
    mask = rng.random(((t + 15) // 16, f // 64)) < p
    bits = _bits_of(mask)
    data = ops.encode_mask(bits, t, f, encoding)
    back, t2, f2 = ops.decode_mask(data)
    assert (t2, f2) == (t, f)
    assert torch.equal(back, bits)
    magic, version, enc, rows, cols, f_h, t_h, words, _, pbytes, live = struct.unpack_from("<IHHHHIQIIQQ", data)
    assert magic == 0x424D5053 and version == 1 and enc == {"raw": 0, "runs": 1}[encoding]
    assert (rows, cols, f_h, t_h) == (16, 64, f, t)
    assert words == ops.tile_bits_words(f) and pbytes == len(data) - 64 and live == int(mask.sum())


def test_row_runs_compress_the_benchmark_mask_shapes():
    from sparsity_spillover_b200 import ops

    rng = np.random.default_rng(7)
    t, f = 65536, 2048
    every_tile = _bits_of(np.ones((t // 16, f // 64), dtype=bool))  # element-random 10 % density
    assert len(ops.encode_mask(every_tile, t, f, "runs")) == 64 + 4 + 8
    blocks = np.repeat(rng.random((t // 64, f // 64)) < 0.1, 4, axis=0)  # 64-token x 64-feature tiles (cfg2)
    blocked = _bits_of(blocks)
    raw, runs = len(ops.encode_mask(blocked, t, f, "raw")), len(ops.encode_mask(blocked, t, f, "runs"))
    assert runs <= 64 + 4 + (t // 64) * 8 and runs < raw
    noise = _bits_of(rng.random((t // 16, f // 64)) < 0.5)  # no two groups alike: runs cost more
    assert len(ops.encode_mask(noise, t, f, "runs")) > len(ops.encode_mask(noise, t, f, "raw"))


def test_file_round_trip(tmp_path):
    from sparsity_spillover_b200 import ops

    rng = np.random.default_rng(3)
    bits = _bits_of(rng.random((64, 32)) < 0.3)
    n = ops.save_mask(tmp_path / "layer0.spmb", bits, 1024, 2048, "runs")
    assert n == (tmp_path / "layer0.spmb").stat().st_size
    back, t, f = ops.load_mask(tmp_path / "layer0.spmb")
    assert (t, f) == (1024, 2048) and torch.equal(back, bits)


@pytest.mark.parametrize("encoding", ["raw", "runs"])
def test_corruption_is_rejected(encoding):
    from sparsity_spillover_b200 import ops
    from sparsity_spillover_b200._lib import SpmlpError

    rng = np.random.default_rng(11)
    bits = _bits_of(rng.random((64, 32)) < 0.3)
    data = bytearray(ops.encode_mask(bits, 1024, 2048, encoding))
    flipped = bytearray(data)
    flipped[len(data) - 3] ^= 0x10
    with pytest.raises(SpmlpError, match="checksum"):
        ops.decode_mask(bytes(flipped))
    with pytest.raises(SpmlpError, match="truncated"):
        ops.decode_mask(bytes(data[:-4]))
    with pytest.raises(SpmlpError, match="magic"):
        ops.decode_mask(b"XXXX" + bytes(data[4:]))
    bad_version = bytearray(data)
    bad_version[4] = 9
    with pytest.raises(SpmlpError, match="version"):
        ops.decode_mask(bytes(bad_version))
    with pytest.raises(SpmlpError):
        ops.decode_mask(bytes(data[:40]))


def test_encode_argument_errors():
    from sparsity_spillover_b200 import ops
    from sparsity_spillover_b200._lib import SpmlpError

    bits = torch.zeros(ops.tile_bits_size(64, 512), dtype=torch.int32)
    with pytest.raises(ValueError):
        ops.encode_mask(bits, 64, 512, "zip")
    with pytest.raises(ValueError):
        ops.encode_mask(bits, 128, 512)  # wrong size for T
    with pytest.raises(SpmlpError, match="multiple of 64"):
        ops.encode_mask(torch.zeros(4, dtype=torch.int32), 64, 100)
