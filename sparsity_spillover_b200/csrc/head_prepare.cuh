// Corner certificates of the vocabulary-head input and its cast to fp16/bf16.
//
// Reference semantics (runs/068-2026-10-08-pythia14m-aligned-vocabulary-tiles/
// inference/head.cu:9-16 and head.py:20-29, gate runs/063-.../tile_gate.py:20-33):
// the head input x (fp32, after the final LayerNorm) is gated in 16-token x
// 16-feature tiles; a tile is live iff its top-left fp32 value is > kappa
// (fp32 comparison, before any cast).  Live tiles keep every signed value.
//
// Output: x_out = cast(x) with dead tiles zeroed, and support bits: bit (j % 32)
// of word [r * words + j / 32] is set iff tile (r, j) is live.
#pragma once

#include "gemm_sm100.cuh"

namespace spmlp {

template <bool BF16>
__global__ void __launch_bounds__(256) head_prepare_kernel(const float* __restrict__ x, uint16_t* __restrict__ x_out,
                                                           uint32_t* __restrict__ support, int T, int d, int words,
                                                           float kappa) {
  using D = DType<BF16>;
  extern __shared__ uint32_t s_words[];  // [words]
  const int rg = blockIdx.x;             // 16-row group
  const int row0 = rg * 16;
  const int granules = d / 16;
  for (int w = threadIdx.x; w < words; w += blockDim.x) s_words[w] = 0u;
  __syncthreads();
  for (int j = threadIdx.x; j < granules; j += blockDim.x) {
    const float corner = x[static_cast<size_t>(row0) * d + j * 16];
    if (corner > kappa) atomicOr(&s_words[j >> 5], 1u << (j & 31));
  }
  __syncthreads();
  for (int w = threadIdx.x; w < words; w += blockDim.x) support[static_cast<size_t>(rg) * words + w] = s_words[w];
  // Cast four consecutive features per thread; a tile never splits a quad.
  const int rows = min(16, T - row0);
  const int quads = rows * (d / 4);
  for (int q = threadIdx.x; q < quads; q += blockDim.x) {
    const int r = q / (d / 4);
    const int c = (q - r * (d / 4)) * 4;
    const size_t off = static_cast<size_t>(row0 + r) * d + c;
    const bool live = (s_words[(c >> 4) >> 5] >> ((c >> 4) & 31)) & 1u;
    const float4 v = *reinterpret_cast<const float4*>(x + off);
    uint2 o;
    if (live) {
      o.x = uint32_t(D::round_bits(v.x)) | (uint32_t(D::round_bits(v.y)) << 16);
      o.y = uint32_t(D::round_bits(v.z)) | (uint32_t(D::round_bits(v.w)) << 16);
    } else {
      o.x = 0u;
      o.y = 0u;
    }
    *reinterpret_cast<uint2*>(x_out + off) = o;
  }
}

// Write `value` (already in the activation dtype's bit pattern) into the listed
// 128-column tiles of logits [T, V]: used to mask vocabulary tiles the N-gated
// head does not compute.
__global__ void __launch_bounds__(256) head_fill_kernel(uint16_t* __restrict__ logits, const int* __restrict__ tiles,
                                                        int n_tiles, int T, int V, uint16_t value) {
  const int tile = blockIdx.y;
  if (tile >= n_tiles) return;
  const int col0 = __ldg(tiles + tile) * 128;
  const uint32_t v2 = uint32_t(value) | (uint32_t(value) << 16);
  const uint4 v8 = make_uint4(v2, v2, v2, v2);
  // 16 threads x 8 halves cover one 128-column row segment.
  const int lane16 = threadIdx.x & 15;
  const int col = col0 + lane16 * 8;
  if (col >= V) return;
  for (int row = blockIdx.x * 16 + (threadIdx.x >> 4); row < T; row += gridDim.x * 16)
    *reinterpret_cast<uint4*>(logits + static_cast<size_t>(row) * V + col) = v8;
}

}  // namespace spmlp
