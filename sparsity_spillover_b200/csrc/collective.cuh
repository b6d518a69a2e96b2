// Reduction side of the d_ff split's fused reduce-scatter.
//
// Each rank's scattering down projection (GemmParams::scatter_rows) has written
// its rounded partial of this rank's token block into slot r of this rank's
// receive buffer recv [world, rows, d].  This kernel finishes the layer for the
// block: y = round(round(sum_r recv[r] + b_out) + residual), the sum in fp32 in
// rank order (deterministic), and writes y to every target -- each rank's copy
// of the next layer's input, so the reduction and the all-gather of the next
// input are one pass over NVLink.
#pragma once

#include <stdint.h>

#include "gemm_sm100.cuh"

namespace spmlp {

struct BroadcastTargets {
  void* dst[kMaxRanks];  // this rank's token block inside each target buffer
  int n;
};

// Vectors (8 elements, 16 bytes) each thread has in flight per pass of the grid-stride
// loops below: the loads of kVecsInFlight vectors are issued before any is used, so
// that a grid squeezed onto a few SMs (beside a persistent GEMM of another token
// slice) still keeps enough NVLink / HBM requests outstanding.
constexpr int kVecsInFlight = 4;

template <bool BF16>
__global__ void __launch_bounds__(256) reduce_broadcast_kernel(const uint16_t* __restrict__ recv, int world,
                                                               int64_t elems, int d, const uint16_t* __restrict__ bias,
                                                               const uint16_t* residual, BroadcastTargets targets) {
  using D = DType<BF16>;
  constexpr int U = kVecsInFlight;
  const int64_t vecs = elems / 8;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i0 = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i0 < vecs; i0 += U * stride) {
    float acc[U][8];
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[u][e] = 0.f;
    for (int r = 0; r < world; ++r) {
      uint4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t i = i0 + u * stride;
        v[u] = i < vecs ? __ldcs(reinterpret_cast<const uint4*>(recv + r * elems) + i) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[u][2 * j] += D::lo(w[j]);
          acc[u][2 * j + 1] += D::hi(w[j]);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = i0 + u * stride;
      if (i >= vecs) break;
      uint32_t out[4];
      const int col = static_cast<int>((i * 8) % d);
      uint4 b = make_uint4(0u, 0u, 0u, 0u);
      if (bias != nullptr) b = __ldg(reinterpret_cast<const uint4*>(bias + col));
      const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) out[j] = D::pack_rn(acc[u][2 * j] + D::lo(bw[j]), acc[u][2 * j + 1] + D::hi(bw[j]));
      if (residual != nullptr) {
        const uint4 rv = reinterpret_cast<const uint4*>(residual)[i];
        const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) out[j] = D::pack_rn(D::lo(out[j]) + D::lo(rw[j]), D::hi(out[j]) + D::hi(rw[j]));
      }
      const uint4 o = make_uint4(out[0], out[1], out[2], out[3]);
      for (int k = 0; k < targets.n; ++k) reinterpret_cast<uint4*>(targets.dst[k])[i] = o;
    }
  }
  __threadfence_system();  // peer stores are performed before the kernel completes
}

// The same finish of the layer through NVLink SHARP (NVSwitch multicast objects):
// every rank has written its rounded partial of ALL tokens into its own copy of a
// multicast-bound buffer; for this rank's block, multimem.ld_reduce returns the sum
// of every rank's copy, reduced inside the switch in fp32 (.acc::f32) and rounded
// once to the dtype; then y = round(round(sum + b_out) + residual) goes to every
// rank's copy of the next layer's input with one multimem.st.  Per rank, the partial
// tokens cross NVLink once into the switch and the result once out of it, instead
// of one peer store per rank for each.  The switch's reduction order is fixed per
// address, so every run gives the same y; it is not the rank order of
// reduce_broadcast_kernel, and the sum is rounded once more before b_out is added.
// mc_part / mc_x: this rank's block inside the multicast mappings; residual: this
// rank's block of its local copy of the layer input (read before mc_x overwrites it).
template <bool BF16>
__device__ __forceinline__ uint4 multimem_ld_reduce_add_v4(const uint16_t* mc) {
  uint4 v;
  if constexpr (BF16)
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(mc) : "memory");
  else
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(mc) : "memory");
  return v;
}

template <bool BF16>
__device__ __forceinline__ void multimem_st_v4(uint16_t* mc, const uint4& v) {
  if constexpr (BF16)
    asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};"
                 :: "l"(mc), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
  else
    asm volatile("multimem.st.relaxed.sys.global.v4.f16x2 [%0], {%1, %2, %3, %4};"
                 :: "l"(mc), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

template <bool BF16>
__global__ void __launch_bounds__(256) multicast_reduce_broadcast_kernel(const uint16_t* mc_part, uint16_t* mc_x,
                                                                         int64_t elems, int d,
                                                                         const uint16_t* __restrict__ bias,
                                                                         const uint16_t* residual) {
  using D = DType<BF16>;
  constexpr int U = kVecsInFlight;
  const int64_t vecs = elems / 8;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i0 = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i0 < vecs; i0 += U * stride) {
    uint4 sv[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < vecs) sv[u] = multimem_ld_reduce_add_v4<BF16>(mc_part + 8 * i);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = i0 + u * stride;
      if (i >= vecs) break;
      const uint32_t sw[4] = {sv[u].x, sv[u].y, sv[u].z, sv[u].w};
      const int col = static_cast<int>((i * 8) % d);
      uint4 b = make_uint4(0u, 0u, 0u, 0u);
      if (bias != nullptr) b = __ldg(reinterpret_cast<const uint4*>(bias + col));
      const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
      uint32_t out[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) out[j] = D::pack_rn(D::lo(sw[j]) + D::lo(bw[j]), D::hi(sw[j]) + D::hi(bw[j]));
      if (residual != nullptr) {
        const uint4 rv = reinterpret_cast<const uint4*>(residual)[i];
        const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) out[j] = D::pack_rn(D::lo(out[j]) + D::lo(rw[j]), D::hi(out[j]) + D::hi(rw[j]));
      }
      multimem_st_v4<BF16>(mc_x + 8 * i, make_uint4(out[0], out[1], out[2], out[3]));
    }
  }
  __threadfence_system();  // the multicast stores are performed before the kernel completes
}

struct PeerFlags {
  long long* dst[kMaxRanks];  // this rank's slot in each rank's flag array (peer memory)
};

// Barrier over NVLink peer memory: thread j stores `epoch` into this rank's slot of
// rank j's flags (after a system-scope fence, so this rank's earlier peer stores
// are visible first), then waits until rank j's epoch has arrived in `local`.
// Every wait is bounded: after SPMLP_WAIT_NS it records kDevTimeoutPeer and gives up.
__global__ void peer_barrier_kernel(PeerFlags peers, const long long* local, int world, long long epoch,
                                    int* status) {
  const int j = threadIdx.x;
  if (j >= world) return;
  const int base = status_base(status);  // errors of earlier launches are not this barrier's
  __threadfence_system();
  asm volatile("st.release.sys.global.b64 [%0], %1;" ::"l"(peers.dst[j]), "l"(epoch) : "memory");
  const uint64_t start = global_timer_ns();
  while (true) {
    long long seen;
    asm volatile("ld.acquire.sys.global.b64 %0, [%1];" : "=l"(seen) : "l"(local + j) : "memory");
    if (seen >= epoch) break;
    if (status_changed(status, base)) break;  // another wait of this barrier already failed
    if (global_timer_ns() - start > SPMLP_WAIT_NS) {
      status_record(status, base, kDevTimeoutPeer);
      break;
    }
    __nanosleep(100);
  }
}

}  // namespace spmlp
