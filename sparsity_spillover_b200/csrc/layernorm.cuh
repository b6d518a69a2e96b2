// Per-token LayerNorm statistics for the up projection's folded LayerNorm.
//
// GPT-NeoX feeds dense_h_to_4h with post_attention_layernorm(x) (the reference
// computes it in a paired LayerNorm kernel, runs/035-2026-09-18-pythia70m-k050-port/
// kernel/norm/norm.cu:23-60).  Folding gamma into the weight and beta into a
// per-feature constant leaves only two numbers per token for the GEMM epilogue:
// mean and rstd = 1 / sqrt(var + eps) (biased variance, fp32, as
// torch.nn.LayerNorm).  One warp per token, two passes over the row (the second
// one hits L1), so the normalized activation is never written to memory.
#pragma once

#include <stdint.h>

#include "gemm_sm100.cuh"

namespace spmlp {

template <bool BF16>
__global__ void __launch_bounds__(256) row_stats_kernel(const uint16_t* __restrict__ x, float* __restrict__ mean,
                                                        float* __restrict__ rstd, int T, int d, float eps) {
  using D = DType<BF16>;
  const int token = static_cast<int>((blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (token >= T) return;  // whole warps leave together
  const uint16_t* row = x + static_cast<size_t>(token) * d;
  float sum = 0.f;
  for (int c = lane * 8; c < d; c += 256) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(row + c));
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) sum += D::lo(w[j]) + D::hi(w[j]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float mu = sum / static_cast<float>(d);
  float sq = 0.f;
  for (int c = lane * 8; c < d; c += 256) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(row + c));
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a = D::lo(w[j]) - mu, b = D::hi(w[j]) - mu;
      sq = fmaf(a, a, fmaf(b, b, sq));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  if (lane == 0) {
    mean[token] = mu;
    rstd[token] = rsqrtf(sq / static_cast<float>(d) + eps);
  }
}

}  // namespace spmlp
