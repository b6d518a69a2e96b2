// Standalone 16x64 tile-bitmap builder for an existing activation h [T, F].
//
// spmlp_up_gate emits the bitmap as a by-product of its epilogue; this kernel
// serves callers whose h comes from elsewhere (e.g. a tile-structured h fed
// straight to the down-projection).  Bit semantics are the same: a tile's bit
// is set iff one of its elements is nonzero (-0.0 counts as zero).
#pragma once

#include <stdint.h>

#include "gemm_sm100.cuh"

namespace spmlp {

// One CTA per 16-row group; each warp scans whole 16x64 tiles: lane l reads the
// 64-byte half (l & 1) of row (l >> 1), i.e. four 16-byte vectors.
__global__ void __launch_bounds__(256) tile_bits_kernel(const uint16_t* __restrict__ h, uint32_t* __restrict__ bits,
                                                        int T, int F, int words) {
  extern __shared__ uint32_t s_words[];
  const int rg = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  for (int w = threadIdx.x; w < words; w += blockDim.x) s_words[w] = 0u;
  __syncthreads();
  const int tiles = F / 64;
  const int row = rg * 16 + (lane >> 1);
  for (int g = warp; g < tiles; g += nwarps) {
    uint32_t acc = 0;
    if (row < T) {
      const uint4* p = reinterpret_cast<const uint4*>(h + static_cast<size_t>(row) * F + g * 64 + (lane & 1) * 32);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 v = __ldcs(p + i);  // streamed once: do not keep in L1/L2
        acc |= (v.x | v.y | v.z | v.w) & 0x7fff7fffu;
      }
    }
    if (__any_sync(0xffffffffu, acc != 0) && lane == 0) atomicOr(&s_words[g >> 5], 1u << (g & 31));
  }
  __syncthreads();
  for (int w = threadIdx.x; w < words; w += blockDim.x) bits[static_cast<size_t>(rg) * words + w] = s_words[w];
}

// Elementwise gate of an activation x [T, F] into out (which may alias x), and
// optionally the 16x64 tile bitmap of the gated values.  Gates: identity, one-
// sided (keep z >= kappa), symmetric (keep |z| >= kappa), ReLU -- the same packed
// comparisons as the up-projection epilogue, so NaN is kept and -0.0 counts as
// zero.  This serves inputs gated outside the up projection: the joint
// consumer's h and attention-output z branches.  Same grid as tile_bits_kernel.
template <bool BF16>
__global__ void __launch_bounds__(256) gate_bits_kernel(const uint16_t* x, uint16_t* out, uint32_t* __restrict__ bits,
                                                        int T, int F, int words, int gate_op, float kappa) {
  using D = DType<BF16>;
  extern __shared__ uint32_t s_words[];
  const int rg = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  if (bits != nullptr) {
    for (int w = threadIdx.x; w < words; w += blockDim.x) s_words[w] = 0u;
    __syncthreads();
  }
  const uint32_t k2 = D::pack_rn(kappa, kappa);  // exact: kappa is already a dtype value
  auto gate = [&](uint32_t w) -> uint32_t {
    switch (gate_op) {
      case GATE_ONE_SIDED:
        return w & ~D::lt_mask(w, k2);
      case GATE_SYMMETRIC:
        return w & ~D::lt_mask(w & 0x7fff7fffu, k2);
      case GATE_RELU:
        return w & ~D::lt_mask(w, 0u);
      default:
        return w;
    }
  };
  const int tiles = F / 64;
  const int row = rg * 16 + (lane >> 1);
  for (int g = warp; g < tiles; g += nwarps) {
    uint32_t acc = 0;
    if (row < T) {
      const size_t off = static_cast<size_t>(row) * F + g * 64 + (lane & 1) * 32;
      const uint4* src = reinterpret_cast<const uint4*>(x + off);
      uint4* dst = reinterpret_cast<uint4*>(out + off);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 v = __ldcs(src + i);
        v.x = gate(v.x);
        v.y = gate(v.y);
        v.z = gate(v.z);
        v.w = gate(v.w);
        dst[i] = v;
        acc |= (v.x | v.y | v.z | v.w) & 0x7fff7fffu;
      }
    }
    if (bits != nullptr && __any_sync(0xffffffffu, acc != 0) && lane == 0) atomicOr(&s_words[g >> 5], 1u << (g & 31));
  }
  if (bits != nullptr) {
    __syncthreads();
    for (int w = threadIdx.x; w < words; w += blockDim.x) bits[static_cast<size_t>(rg) * words + w] = s_words[w];
  }
}

// The corner-tile gate (8-token x 16-feature tiles, kept iff the tile's top-left z >
// kappa) applied in place to z [T, F], with the 16x64 tile bitmap of the result.
// Token blocks restart at every sequence start (row multiple of seq_len), so with
// seq_len % 8 != 0 a block's corner row can lie in another up-projection tile, where
// the fused epilogue cannot see it; this pass serves that case after an ungated up
// projection.  The last block of a sequence may be shorter than 8 tokens and is
// decided by its own first row, as in the reference gate.  In place is safe: a
// corner that is rejected (z <= kappa, or NaN) may be zeroed by its own thread while
// others read it, and 0 > kappa is false for every kappa >= 0, so every reader
// reaches the same decision.  Same grid as tile_bits_kernel.
template <bool BF16>
__global__ void __launch_bounds__(256) corner_gate_kernel(uint16_t* z, uint32_t* __restrict__ bits, int T, int F,
                                                          int words, int seq_len, float kappa) {
  using D = DType<BF16>;
  extern __shared__ uint32_t s_words[];
  const int rg = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  for (int w = threadIdx.x; w < words; w += blockDim.x) s_words[w] = 0u;
  __syncthreads();
  const int tiles = F / 64;
  const int row = rg * 16 + (lane >> 1);
  int corner_row = row;
  if (row < T) {
    const int s0 = (row / seq_len) * seq_len;
    corner_row = s0 + ((row - s0) / 8) * 8;
  }
  for (int g = warp; g < tiles; g += nwarps) {
    uint32_t acc = 0;
    if (row < T) {
      const int col = g * 64 + (lane & 1) * 32;  // two 16-feature tiles per lane
      const volatile uint16_t* cz = z + static_cast<size_t>(corner_row) * F + col;
      const uint32_t keep0 = D::to_float(cz[0]) > kappa ? 0xffffffffu : 0u;
      const uint32_t keep1 = D::to_float(cz[16]) > kappa ? 0xffffffffu : 0u;
      uint4* p = reinterpret_cast<uint4*>(z + static_cast<size_t>(row) * F + col);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t keep = i < 2 ? keep0 : keep1;
        uint4 v = p[i];
        v.x &= keep;
        v.y &= keep;
        v.z &= keep;
        v.w &= keep;
        p[i] = v;
        acc |= (v.x | v.y | v.z | v.w) & 0x7fff7fffu;
      }
    }
    if (__any_sync(0xffffffffu, acc != 0) && lane == 0) atomicOr(&s_words[g >> 5], 1u << (g & 31));
  }
  __syncthreads();
  for (int w = threadIdx.x; w < words; w += blockDim.x) bits[static_cast<size_t>(rg) * words + w] = s_words[w];
}

// The 16x16 tile bitmap of h (the compact down mode's): one bit per 16-row x 16-feature
// tile, bit g % 32 of word r * words + g / 32 set iff the tile holds a nonzero (-0.0
// counts as zero).  One CTA per 16-row group; each warp scans two tiles per pass: lane l
// reads the 16-byte half (l & 1) of row (l >> 1) & 15 of tile 2 pass + l / 32 ... as two
// 16-lane halves, one tile each.
__global__ void __launch_bounds__(256) tile_bits16_kernel(const uint16_t* __restrict__ h, uint32_t* __restrict__ bits,
                                                          int T, int F, int words) {
  extern __shared__ uint32_t s_words[];
  const int rg = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  for (int w = threadIdx.x; w < words; w += blockDim.x) s_words[w] = 0u;
  __syncthreads();
  const int tiles = F / 16;
  const int half = lane >> 4;            // which of the pass's two tiles
  const int row = rg * 16 + (lane & 15);  // one row of the tile per lane (32 bytes)
  for (int g0 = 2 * warp; g0 < tiles; g0 += 2 * nwarps) {
    const int g = g0 + half;
    uint32_t acc = 0;
    if (row < T && g < tiles) {
      const uint4* p = reinterpret_cast<const uint4*>(h + static_cast<size_t>(row) * F + g * 16);
      const uint4 a = __ldcs(p), b = __ldcs(p + 1);
      acc = (a.x | a.y | a.z | a.w | b.x | b.y | b.z | b.w) & 0x7fff7fffu;
    }
    const uint32_t ball = __ballot_sync(0xffffffffu, acc != 0);
    if (lane == 0) {
      if (ball & 0x0000ffffu) atomicOr(&s_words[g0 >> 5], 1u << (g0 & 31));
      if ((ball & 0xffff0000u) && g0 + 1 < tiles) atomicOr(&s_words[(g0 + 1) >> 5], 1u << ((g0 + 1) & 31));
    }
  }
  __syncthreads();
  for (int w = threadIdx.x; w < words; w += blockDim.x) bits[static_cast<size_t>(rg) * words + w] = s_words[w];
}

}  // namespace spmlp
