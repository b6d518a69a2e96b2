// Persistent, warp-specialised sm_100a GEMM used by every kernel of the sparse
// gated MLP:  C[M,N] = A[M,K] * B[N,K]^T  with both operands K-major fp16/bf16.
//
//   warp 0      TMA producer: walks the live K-blocks of each tile (bitmap
//               driven, ballot/popc scheduled) and loads only those A/B tiles
//               into a STAGES-deep shared-memory ring, so the ring holds the
//               surviving tiles back to back (compaction through smem).
//   warp 1      MMA issuer: one elected thread issues tcgen05.mma (M=128,
//               or M=256 over a CTA pair, N=BN, K=16) into TMEM accumulators,
//               double-buffered across tiles when two tiles' worth fit.
//   warps 2..   epilogue (4 or 8 warps): tcgen05.ld the accumulator (one
//               token row per thread, software-pipelined), apply the
//               kind-specific epilogue, stage 32x32 chunks in shared memory
//               and write them with TMA bulk stores.
//
// Kinds:
//   KIND_UP    z = round(acc + b_in); h = gate(z); writes h, the 16x64 tile
//              nonzero bitmap, and optionally z.      (GPTNeoXMLP.dense_h_to_4h + act)
//   KIND_DOWN  y = round(acc + b_out) [then round(y + residual)], skipping
//              K-blocks whose 16x64 tiles are all zero for the whole M-tile.
//                                                     (GPTNeoXMLP.dense_4h_to_h)
//   KIND_HEAD  logits = round(acc) over an explicit list of active 128-column
//              vocabulary tiles, optionally skipping dead K16 groups of the
//              head input (corner certificates).        (GPTNeoXForCausalLM.embed_out)
//   KIND_JOINT out = round(round(round(h W2^T + b2) + round(z Wo^T + bo)) + r):
//              the MLP's down projection (tile-skipping over h) and the
//              attention output projection in two TMEM accumulators of the
//              same tile, with GPT-NeoX's parallel residual.  (the joint consumer)
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "sm100.cuh"

namespace spmlp {

enum Kind : int { KIND_UP = 0, KIND_DOWN = 1, KIND_HEAD = 2, KIND_JOINT = 3 };

// Gate operators applied to the rounded up-projection output z.
enum GateOp : int {
  GATE_IDENTITY = 0,     // h = z
  GATE_GELU = 1,         // h = gelu_erf(z)                         (A0, ungated GPT-NeoX)
  GATE_ONE_SIDED = 2,    // h = z if z >= kappa else 0              (FixedOneSidedThreshold)
  GATE_SYMMETRIC = 3,    // h = z if |z| >= kappa else 0            (FixedSymmetricThreshold)
  GATE_RELU = 4,         // h = z if z > 0 else 0                   (torch.nn.ReLU)
  GATE_GELU_MASKED = 5,  // h = gelu_erf(z) if z > kappa else 0     (gelu-then-mask variant)
  GATE_CORNER = 6,       // 8x16 tile kept iff its top-left z > kappa (CornerTileThreshold)
};

constexpr int kBM = 128;       // tokens per tile (UMMA M)
constexpr int kBK = 64;        // K elements per pipeline stage (one 128-byte swizzle row)
constexpr int kBitsRows = 16;  // bitmap tile height (tokens)
constexpr int kBitsCols = 64;  // bitmap tile width (features)
constexpr int kMaxRanks = 8;   // ranks a scattering down projection can address
constexpr int kPrefetchAhead = 8;  // K-blocks of h brought into L2 ahead of their TMA loads

struct GemmParams {
  int M, N, K;            // tokens, output columns, reduction length
  int m_tiles, n_tiles;   // n_tiles = entries of col_tiles for KIND_HEAD
  // Work items: tiles [0, tail_from) as they are, then each remaining tile as two
  // half-width (BN/2-column) items, so the last round of a persistent grid is not
  // left half idle.  work_items = tail_from + 2 * (m_tiles * n_tiles - tail_from).
  int tail_from, work_items;
  int split_tail;         // host: 1 = may split the last round's tiles (set from the launch shape)
  const void* bias;       // [N] in the activation dtype, nullable
  void* out;              // [M, N] row-major output (h, y or logits)
  void* z_out;            // KIND_UP: optional pre-gate z [M, N]
  const void* residual;   // KIND_DOWN / KIND_JOINT: optional [M, N]
  int K2;                 // KIND_JOINT: reduction length of the second product (z Wo^T)
  const void* bias2;      // KIND_JOINT: [N] bias of the second product, nullable
  // KIND_UP with a LayerNorm folded into the weight (B = W diag(gamma)): z =
  // round(rstd[m] * (acc - mean[m] * ln_s[n]) + ln_c[n]) instead of round(acc + b),
  // with ln_s = sum_k B[n, k] and ln_c = b + W beta (fp32).  Null: no LayerNorm.
  const float* ln_mean;   // [M]
  const float* ln_rstd;   // [M]
  const float* ln_s;      // [N]
  const float* ln_c;      // [N]
  uint32_t* bits_out;     // KIND_UP: 16x64 tile bitmap, zeroed by the host
  const uint32_t* bits_in;  // KIND_DOWN / KIND_JOINT: 16x64 bitmap of A; KIND_HEAD: 16x16 support bits
  int bits_words;         // words per 16-row group in bits_out / bits_in
  int skip;               // KIND_DOWN/HEAD: 1 = skip dead K granules
  const int* col_tiles;   // KIND_HEAD: active BN-column tile indices
  int gate_op;
  float kappa;            // already rounded to the activation dtype
  int seq_len;            // GATE_CORNER: tokens per sequence (blocks restart per sequence)
  unsigned long long* stats;  // nullable: [0] issued K granules, [1] skipped K granules
  // KIND_DOWN, d_ff split: with scatter_rows > 0 the rounded partial tile of tokens
  // [j * scatter_rows, (j + 1) * scatter_rows) goes to scatter_out[j] (this rank's
  // slot in rank j's receive buffer, [scatter_rows, N], usually peer memory)
  // instead of `out`; bias and residual are added after the reduction.
  void* scatter_out[kMaxRanks];
  int scatter_rows;
  int* status;            // device status word
};

template <bool BF16>
struct DType;
template <>
struct DType<false> {
  using T = __half;
  __device__ static __forceinline__ uint16_t round_bits(float f) { return __half_as_ushort(__float2half_rn(f)); }
  __device__ static __forceinline__ float to_float(uint16_t b) { return __half2float(__ushort_as_half(b)); }
  // Two fp32 values rounded (RN) into one packed word, low half first.
  __device__ static __forceinline__ uint32_t pack_rn(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  __device__ static __forceinline__ __half2 h2(uint32_t w) { return *reinterpret_cast<const __half2*>(&w); }
  // 0xFFFF in each half where a < b (false for NaN operands).
  __device__ static __forceinline__ uint32_t lt_mask(uint32_t a, uint32_t b) { return __hlt2_mask(h2(a), h2(b)); }
  __device__ static __forceinline__ uint32_t gt_mask(uint32_t a, uint32_t b) { return __hgt2_mask(h2(a), h2(b)); }
  __device__ static __forceinline__ float lo(uint32_t w) { return to_float(static_cast<uint16_t>(w & 0xffffu)); }
  __device__ static __forceinline__ float hi(uint32_t w) { return to_float(static_cast<uint16_t>(w >> 16)); }
};
template <>
struct DType<true> {
  using T = __nv_bfloat16;
  __device__ static __forceinline__ uint16_t round_bits(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
  }
  __device__ static __forceinline__ float to_float(uint16_t b) { return __bfloat162float(__ushort_as_bfloat16(b)); }
  __device__ static __forceinline__ uint32_t pack_rn(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  __device__ static __forceinline__ __nv_bfloat162 h2(uint32_t w) {
    return *reinterpret_cast<const __nv_bfloat162*>(&w);
  }
  __device__ static __forceinline__ uint32_t lt_mask(uint32_t a, uint32_t b) { return __hlt2_mask(h2(a), h2(b)); }
  __device__ static __forceinline__ uint32_t gt_mask(uint32_t a, uint32_t b) { return __hgt2_mask(h2(a), h2(b)); }
  __device__ static __forceinline__ float lo(uint32_t w) { return __uint_as_float(w << 16); }
  __device__ static __forceinline__ float hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
};

__device__ __forceinline__ float gelu_erf(float z) { return 0.5f * z * (1.0f + erff(z * 0.70710678118654752f)); }

// Granule size of the K-skip bitmap for each kind (features per bit).
template <int KIND>
struct KGran {
  static constexpr int value = (KIND == KIND_HEAD) ? 16 : kBitsCols;
};

// Live-K mask of one 32-granule chunk for M-tile m_blk of GROUPS 16-row groups.
// Warp-collective: lane j tests granule 32*chunk+j across the tile's row groups
// and __ballot_sync gathers the answer.  Rows past the last row group are absent.
template <int GROUPS>
__device__ __forceinline__ uint32_t live_chunk(const uint32_t* bits, int words, int row_groups, int m_blk,
                                               int chunk, int granules, int lane) {
  const int g = chunk * 32 + lane;
  uint32_t live = 0;
  if (g < granules) {
    const int rg0 = m_blk * GROUPS;
#pragma unroll
    for (int r = 0; r < GROUPS; ++r) {
      const int rg = rg0 + r;
      if (rg < row_groups) live |= (__ldg(bits + static_cast<size_t>(rg) * words + chunk) >> lane) & 1u;
    }
  }
  return __ballot_sync(0xffffffffu, live != 0);
}

// Expand a granule mask (16-feature granules) to a 64-wide K-block mask.
__device__ __forceinline__ uint32_t kblocks_of_k16(uint32_t m16) {
  uint32_t kb = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if ((m16 >> (4 * i)) & 0xFu) kb |= 1u << i;
  return kb;
}

// RING = 0: each epilogue warp stages its whole tile (kWarpChunks chunks) in
// shared memory, and the down projection's residual is TMA-loaded there.
// RING > 0: each warp cycles through RING single-chunk slots (one TMA store per
// chunk), and the residual is read into registers; the shared memory saved
// goes to deeper operand pipelines.
template <int KIND, int BN, int STAGES, bool BF16, int EPI = 4, int CG = 1, int RING = 0>
struct GemmTraits {
  static constexpr int kTileM = kBM * CG;                   // tokens per (cluster) tile
  static constexpr uint32_t kABytes = kBM * kBK * 2;         // this CTA's 128 rows of A per stage
  static constexpr uint32_t kBBytes = (BN / CG) * kBK * 2;   // this CTA's share of B per stage
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr int kAccs = KIND == KIND_JOINT ? 2 : 1;     // accumulators per tile
  static constexpr uint32_t kAccCols = kAccs * BN;               // TMEM columns of one tile's accumulators
  // Double-buffered when two tiles' accumulators fit in TMEM's 512 columns (this
  // CTA's M half); a joint tile of BN = 256 fills TMEM alone and is single-buffered.
  static constexpr int kAccBufs = 2 * kAccCols <= 512 ? 2 : 1;
  static constexpr uint32_t kTmemCols = kAccBufs * kAccCols;
  static constexpr int kEpiWarps = EPI;          // 4: one warp per TMEM lane quarter; 8: two, splitting columns
  static constexpr int kThreads = 64 + 32 * EPI;
  static constexpr uint32_t kStageOutBytes = 32 * 32 * 2;  // one 32-row x 32-column output chunk
  static constexpr int kWarpChunks = (BN / 32) / (EPI / 4);  // chunks one epilogue warp handles per tile
  static constexpr int kFlush = kWarpChunks < 4 ? kWarpChunks : 4;  // chunks per fence + store batch (RING = 0)
  static constexpr int kSlabChunks = RING > 0 ? RING : kWarpChunks;  // staged chunks per epilogue warp
  static constexpr uint32_t kEpiBytes = EPI * kSlabChunks * kStageOutBytes;
  // Per-column fp32 vectors staged per warp: the bias (two for the joint; the
  // up projection's folded LayerNorm uses two: ln_s and ln_c).
  static constexpr int kColVecs = (KIND == KIND_JOINT || KIND == KIND_UP) ? 2 : 1;
  static constexpr uint32_t kBiasBytes = kColVecs * EPI * kWarpChunks * 32 * 4;  // each warp's own columns
  static constexpr uint32_t kBarrierBytes = 256;
  static_assert((2 * STAGES + 5 + EPI) * 8 + 4 <= kBarrierBytes, "barrier region too small");
  static constexpr uint32_t kSmemBytes =
      STAGES * kStageBytes + kEpiBytes + kBiasBytes + kBarrierBytes + 1024;  // +1 KiB for alignment
  static_assert(BN == 128 || BN == 256, "BN must be 128 or 256");
  static_assert(CG == 1 || CG == 2, "one CTA or a CTA pair");
  static_assert(EPI == 4 || EPI == 8, "4 or 8 epilogue warps");
  static_assert(kTmemCols <= 512, "TMEM has 512 columns");
  static_assert(RING == 0 || (RING >= 2 && RING <= kWarpChunks), "a ring has 2 .. kWarpChunks slots");
  static_assert(!(KIND == KIND_HEAD && BN == 256) || RING > 0,
                "a head work item of two vocabulary tiles writes through an output ring");
  static_assert(kSmemBytes <= 232448, "exceeds the 227 KiB shared-memory limit");
};

// Number of K granules (bitmap bits) in the reduction dimension.
template <int KIND>
__device__ __forceinline__ int k_granules(int K) {
  return K / KGran<KIND>::value;
}

// Enumerate the live K-blocks (64-wide) of an M-tile of GROUPS 16-row groups, calling f(kb, k16_mask)
// for each; k16_mask says which of the block's four K16 steps to issue.
// Warp-collective (all 32 lanes must call it with the same arguments).
template <int KIND, int GROUPS, class F>
__device__ __forceinline__ bool for_each_live_kblock(const GemmParams& p, int m_blk, int lane, F&& f) {
  const int kblocks = p.K / kBK;
  if (!p.skip || p.bits_in == nullptr) {
    for (int kb = 0; kb < kblocks; ++kb)
      if (!f(kb, 0xFu)) return false;
    return true;
  }
  const int row_groups = (p.M + kBitsRows - 1) / kBitsRows;
  const int granules = k_granules<KIND>(p.K);
  const int chunks = (granules + 31) / 32;
  for (int c = 0; c < chunks; ++c) {
    const uint32_t mask = live_chunk<GROUPS>(p.bits_in, p.bits_words, row_groups, m_blk, c, granules, lane);
    if constexpr (KGran<KIND>::value == kBK) {
      uint32_t pending = mask;
      while (pending) {
        const int kb = c * 32 + __ffs(pending) - 1;
        pending &= pending - 1;
        if (!f(kb, 0xFu)) return false;
      }
    } else {
      // 16-feature granules: 32 granules = 8 K-blocks per chunk.
      uint32_t pending = kblocks_of_k16(mask);
      while (pending) {
        const int i = __ffs(pending) - 1;
        pending &= pending - 1;
        if (!f(c * 8 + i, (mask >> (4 * i)) & 0xFu)) return false;
      }
    }
  }
  return true;
}

// for_each_live_kblock for the TMA producer, which also calls pf(kb) for the live
// K-block AHEAD positions further on in the same 32-granule chunk of the bitmap (the
// first AHEAD blocks of a chunk as it starts), so that their operand tiles can be
// brought into L2 before the shared-memory ring has room for them.
template <int KIND, int GROUPS, int AHEAD, class F, class P>
__device__ __forceinline__ bool for_each_live_kblock_ahead(const GemmParams& p, int m_blk, int lane, F&& f, P&& pf) {
  const int kblocks = p.K / kBK;
  if (!p.skip || p.bits_in == nullptr) {
    for (int kb = 0; kb < AHEAD && kb < kblocks; ++kb) pf(kb);
    for (int kb = 0; kb < kblocks; ++kb) {
      if (kb + AHEAD < kblocks) pf(kb + AHEAD);
      if (!f(kb, 0xFu)) return false;
    }
    return true;
  }
  const int row_groups = (p.M + kBitsRows - 1) / kBitsRows;
  const int granules = k_granules<KIND>(p.K);
  const int chunks = (granules + 31) / 32;
  constexpr int kPerChunk = KGran<KIND>::value == kBK ? 32 : 8;  // K-blocks per chunk of 32 granules
  for (int c = 0; c < chunks; ++c) {
    const uint32_t mask = live_chunk<GROUPS>(p.bits_in, p.bits_words, row_groups, m_blk, c, granules, lane);
    uint32_t pending = KGran<KIND>::value == kBK ? mask : kblocks_of_k16(mask);
    uint32_t ahead = pending;
    for (int i = 0; i < AHEAD && ahead; ++i) {
      pf(c * kPerChunk + __ffs(ahead) - 1);
      ahead &= ahead - 1;
    }
    while (pending) {
      const int i = __ffs(pending) - 1;
      pending &= pending - 1;
      if (ahead) {
        pf(c * kPerChunk + __ffs(ahead) - 1);
        ahead &= ahead - 1;
      }
      const uint32_t k16 = KGran<KIND>::value == kBK ? 0xFu : (mask >> (4 * i)) & 0xFu;
      if (!f(c * kPerChunk + i, k16)) return false;
    }
  }
  return true;
}

// Enumerate the live 16-feature granules of an M-tile of GROUPS 16-row groups in
// increasing K (16x16 bitmap), calling f(g); without skipping every granule.
// Warp-collective (all 32 lanes must call it with the same arguments).
template <int GROUPS, class F>
__device__ __forceinline__ bool for_each_live_g16(const GemmParams& p, int m_blk, int lane, F&& f) {
  const int granules = p.K / 16;
  if (!p.skip || p.bits_in == nullptr) {
    for (int g = 0; g < granules; ++g)
      if (!f(g)) return false;
    return true;
  }
  const int row_groups = (p.M + kBitsRows - 1) / kBitsRows;
  const int chunks = (granules + 31) / 32;
  for (int c = 0; c < chunks; ++c) {
    uint32_t pending = live_chunk<GROUPS>(p.bits_in, p.bits_words, row_groups, m_blk, c, granules, lane);
    while (pending) {
      const int g = c * 32 + __ffs(pending) - 1;
      pending &= pending - 1;
      if (!f(g)) return false;
    }
  }
  return true;
}

// Whether an M-tile of GROUPS 16-row groups has any live K granule (warp-collective),
// i.e. whether for_each_live_kblock would visit any K-block: one bitmap word per lane
// (lane i reads word i of the tile's GROUPS x chunks words) instead of GROUPS per lane.
template <int KIND, int GROUPS, bool G16 = false>
__device__ __forceinline__ bool any_live(const GemmParams& p, int m_blk, int lane) {
  if (!p.skip || p.bits_in == nullptr) return p.K >= kBK;
  const int row_groups = (p.M + kBitsRows - 1) / kBitsRows;
  const int granules = G16 ? p.K / 16 : k_granules<KIND>(p.K);
  const int chunks = (granules + 31) / 32;
  uint32_t any = 0;
  for (int i = lane; i < GROUPS * chunks; i += 32) {
    const int r = i % GROUPS, c = i / GROUPS;
    const int rg = m_blk * GROUPS + r;
    if (rg < row_groups) {
      const int valid = granules - 32 * c;  // granule bits of this word that exist
      const uint32_t mask = valid >= 32 ? 0xffffffffu : ((1u << valid) - 1u);
      any |= __ldg(p.bits_in + static_cast<size_t>(rg) * p.bits_words + c) & mask;
    }
  }
  return __ballot_sync(0xffffffffu, any != 0) != 0;
}

template <int KIND, int BN>
__device__ __forceinline__ void tile_coords(const GemmParams& p, int t, int& m_blk, int& n_col0);

// KIND_HEAD with BN = 256 (a CTA pair): work item t covers entries 2j and 2j + 1 of
// the list of 128-column vocabulary tiles (col_tiles, or every tile in order), one
// per CTA of the pair; an odd list leaves the last item with one tile, which runs
// as a half-width item.  n_tiles counts 128-column tiles.  Returns the half flag.
__device__ __forceinline__ bool head_pair_coords(const GemmParams& p, int t, int& m_blk, int& col0, int& col1) {
  const int items = (p.n_tiles + 1) >> 1;
  m_blk = t / items;
  const int i0 = 2 * (t - m_blk * items);
  col0 = (p.col_tiles != nullptr ? __ldg(p.col_tiles + i0) : i0) * 128;
  const bool single = i0 + 1 >= p.n_tiles;
  col1 = single ? col0 : (p.col_tiles != nullptr ? __ldg(p.col_tiles + i0 + 1) : i0 + 1) * 128;
  return single;
}

template <int KIND, int BN>
__host__ __device__ constexpr bool head_pairs() { return KIND == KIND_HEAD && BN == 256; }

// Work item t -> its tile's M-block and first column; true for a half-width item.
template <int KIND, int BN>
__device__ __forceinline__ bool work_coords(const GemmParams& p, int t, int& m_blk, int& n_col0) {
  if constexpr (head_pairs<KIND, BN>()) {
    int col1;
    return head_pair_coords(p, t, m_blk, n_col0, col1);
  }
  if (t < p.tail_from) {
    tile_coords<KIND, BN>(p, t, m_blk, n_col0);
    return false;
  }
  const int u = t - p.tail_from;
  tile_coords<KIND, BN>(p, p.tail_from + (u >> 1), m_blk, n_col0);
  n_col0 += (u & 1) * (BN / 2);
  return true;
}

template <int KIND, int BN>
__device__ __forceinline__ void tile_coords(const GemmParams& p, int t, int& m_blk, int& n_col0) {
  m_blk = t / p.n_tiles;
  const int n_sel = t - m_blk * p.n_tiles;
  if (KIND == KIND_HEAD && p.col_tiles != nullptr) {
    n_col0 = __ldg(p.col_tiles + n_sel) * BN;
  } else {
    n_col0 = n_sel * BN;
  }
}

// ------------------------------------------------------------------ epilogues
// One call turns 32 accumulator columns of one token row into 16 packed output
// words (32 fp16/bf16 values).  `acc` holds fp32 bit patterns (all zero for a
// tile without live K-blocks); `bias` points at the 32 fp32 bias values of the
// chunk in shared memory; `res` holds the chunk's 32 residual values.  The up
// epilogue returns whether the row's 32 outputs hold a nonzero (bitmap).
template <bool BF16, int GATE>
struct UpEpilogue {
  using D = DType<BF16>;
  // z = round(acc + b) two values per word; h = gate(z) computed on packed
  // words: a comparison mask clears rejected halves (NaN compares false, so
  // masked_fill(z < kappa, 0) keeps it, as torch does).
  // With a folded LayerNorm (ln_c non-null) `bias` holds ln_s and the row's mean
  // and rstd are given.
  __device__ __forceinline__ static bool apply(const GemmParams& p, int row, int col0, int lane, bool row_ok,
                                               const uint32_t (&acc)[32], const float* bias, uint32_t k2,
                                               uint32_t (&out)[16], const float* ln_c = nullptr,
                                               float mean = 0.f, float rstd = 0.f) {
    uint32_t z[16];
    if (ln_c != nullptr) {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float a = fmaf(-mean, bias[2 * j], __uint_as_float(acc[2 * j]));
        const float b = fmaf(-mean, bias[2 * j + 1], __uint_as_float(acc[2 * j + 1]));
        z[j] = D::pack_rn(fmaf(rstd, a, ln_c[2 * j]), fmaf(rstd, b, ln_c[2 * j + 1]));
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j)
        z[j] = D::pack_rn(__uint_as_float(acc[2 * j]) + bias[2 * j], __uint_as_float(acc[2 * j + 1]) + bias[2 * j + 1]);
    }
    if constexpr (GATE == GATE_ONE_SIDED) {
#pragma unroll
      for (int j = 0; j < 16; ++j) out[j] = z[j] & ~D::lt_mask(z[j], k2);
    } else if constexpr (GATE == GATE_SYMMETRIC) {
#pragma unroll
      for (int j = 0; j < 16; ++j) out[j] = z[j] & ~D::lt_mask(z[j] & 0x7fff7fffu, k2);
    } else if constexpr (GATE == GATE_RELU) {
#pragma unroll
      for (int j = 0; j < 16; ++j) out[j] = z[j] & ~D::lt_mask(z[j], 0u);
    } else if constexpr (GATE == GATE_GELU) {
#pragma unroll
      for (int j = 0; j < 16; ++j) out[j] = D::pack_rn(gelu_erf(D::lo(z[j])), gelu_erf(D::hi(z[j])));
    } else if constexpr (GATE == GATE_GELU_MASKED) {
#pragma unroll
      for (int j = 0; j < 16; ++j)
        out[j] = D::pack_rn(gelu_erf(D::lo(z[j])), gelu_erf(D::hi(z[j]))) & D::gt_mask(z[j], k2);
    } else if constexpr (GATE == GATE_CORNER) {
      // Tiles are 8 tokens x 16 features; the corner row of this thread's
      // block lives in lane (lane & ~7) of the same warp because blocks and
      // warp row-quarters are both 8-aligned (the host runs this epilogue only
      // for seq_len % 8 == 0 or a single sequence, and a separate pass otherwise).
      // Columns 0 and 16 of the chunk are corners.
      const int src = lane & ~7;
      const uint32_t c0 = __shfl_sync(0xffffffffu, z[0], src);
      const uint32_t c1 = __shfl_sync(0xffffffffu, z[8], src);
      const uint32_t keep0 = D::lo(c0) > p.kappa ? 0xffffffffu : 0u;
      const uint32_t keep1 = D::lo(c1) > p.kappa ? 0xffffffffu : 0u;
#pragma unroll
      for (int j = 0; j < 8; ++j) out[j] = z[j] & keep0;
#pragma unroll
      for (int j = 8; j < 16; ++j) out[j] = z[j] & keep1;
    } else {  // GATE_IDENTITY
#pragma unroll
      for (int j = 0; j < 16; ++j) out[j] = z[j];
    }
    uint32_t any = 0;
#pragma unroll
    for (int j = 0; j < 16; ++j) any |= out[j];
    if (p.z_out != nullptr && row_ok) {  // check/debug export of the pre-gate z
      uint4* zo = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.z_out) + static_cast<size_t>(row) * p.N + col0);
#pragma unroll
      for (int j = 0; j < 4; ++j) zo[j] = make_uint4(z[4 * j], z[4 * j + 1], z[4 * j + 2], z[4 * j + 3]);
    }
    return row_ok && (any & 0x7fff7fffu) != 0;  // -0.0 is a zero
  }
};

template <bool BF16>
struct DownEpilogue {
  using D = DType<BF16>;
  // y = round(acc + b); with a residual, round(y + r) computed in fp32 like torch's add.
  __device__ __forceinline__ static void apply(const GemmParams& p, const uint32_t (&acc)[32], const float* bias,
                                               const uint4 (&res)[4], uint32_t (&out)[16]) {
#pragma unroll
    for (int j = 0; j < 16; ++j)
      out[j] = D::pack_rn(__uint_as_float(acc[2 * j]) + bias[2 * j], __uint_as_float(acc[2 * j + 1]) + bias[2 * j + 1]);
    if (p.residual != nullptr) {
      const uint32_t* r = reinterpret_cast<const uint32_t*>(&res[0]);
#pragma unroll
      for (int j = 0; j < 16; ++j) out[j] = D::pack_rn(D::lo(out[j]) + D::lo(r[j]), D::hi(out[j]) + D::hi(r[j]));
    }
  }
};

template <bool BF16>
struct HeadEpilogue {
  using D = DType<BF16>;
  __device__ __forceinline__ static void apply(const uint32_t (&acc)[32], uint32_t (&out)[16]) {
#pragma unroll
    for (int j = 0; j < 16; ++j) out[j] = D::pack_rn(__uint_as_float(acc[2 * j]), __uint_as_float(acc[2 * j + 1]));
  }
};

// The joint consumer in the reference's rounding order (torch's bf16/fp16 ops):
// a = round(acc_h + b2), b = round(acc_z + bo), s = round(a + b), out = round(s + r),
// every addition in fp32.
template <bool BF16>
struct JointEpilogue {
  using D = DType<BF16>;
  __device__ __forceinline__ static void apply(const uint32_t (&acc_h)[32], const uint32_t (&acc_z)[32],
                                               const float* bias_h, const float* bias_z, const uint4 (&res)[4],
                                               bool with_res, uint32_t (&out)[16]) {
    const uint32_t* r = reinterpret_cast<const uint32_t*>(&res[0]);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint32_t a = D::pack_rn(__uint_as_float(acc_h[2 * j]) + bias_h[2 * j],
                                    __uint_as_float(acc_h[2 * j + 1]) + bias_h[2 * j + 1]);
      const uint32_t b = D::pack_rn(__uint_as_float(acc_z[2 * j]) + bias_z[2 * j],
                                    __uint_as_float(acc_z[2 * j + 1]) + bias_z[2 * j + 1]);
      uint32_t sum = D::pack_rn(D::lo(a) + D::lo(b), D::hi(a) + D::hi(b));
      if (with_res) sum = D::pack_rn(D::lo(sum) + D::lo(r[j]), D::hi(sum) + D::hi(r[j]));
      out[j] = sum;
    }
  }
};

// ------------------------------------------------------------------ kernel
// CG = 1: one CTA per 128 x BN tile.  CG = 2: a CTA pair (cluster of 2) per
// 256 x BN tile: each CTA loads its 128 rows of A and BN/2 rows of B, the
// leader's single thread issues tcgen05.mma.cta_group::2 (M = 256) over both
// CTAs' shared memory, and each CTA's TMEM receives its 128-row half.  Stage
// completion is counted on the leader's barriers; commits multicast to both.
// LN (KIND_UP only): the epilogue applies a LayerNorm folded into the weight
// (GemmParams::ln_*); a compile-time switch so the plain up projection carries none of it.
// G16 (KIND_DOWN): the compact mode -- the skip bitmap has 16x16 granules and each stage
// gathers four live 16-feature granules of K (A and B boxes of 16 columns, 32-byte
// swizzle), one K16 MMA each, so only live granules are loaded and multiplied.
template <int KIND, int GATE, int BN, int STAGES, bool BF16, int EPI, int CG, int RING = 0, bool LN = false,
          bool G16 = false>
__global__ void __launch_bounds__(GemmTraits<KIND, BN, STAGES, BF16, EPI, CG, RING>::kThreads, 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                      const __grid_constant__ CUtensorMap tm_c, const __grid_constant__ CUtensorMap tm_r,
                      const __grid_constant__ CUtensorMap tm_a2, const __grid_constant__ CUtensorMap tm_b2,
                      const __grid_constant__ CUtensorMap tm_bh, const __grid_constant__ CUtensorMap tm_b2h,
                      const GemmParams p) {
  using Tr = GemmTraits<KIND, BN, STAGES, BF16, EPI, CG, RING>;
  constexpr int kGroups = Tr::kTileM / kBitsRows;  // 16-row bitmap groups per tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_a = smem;
  uint8_t* s_b = smem + STAGES * Tr::kABytes;
  uint8_t* s_out = smem + STAGES * Tr::kStageBytes;  // [EPI][kSlabChunks][32x32] staged output chunks
  float* s_bias = reinterpret_cast<float*>(s_out + Tr::kEpiBytes);  // [EPI][kWarpChunks * 32]
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(s_bias) + Tr::kBiasBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2] (the leader's are the ones used)
  uint64_t* drain = acc_empty + 2;      // [1]
  uint64_t* res_full = drain + 1;       // [EPI]: residual slab loaded (KIND_DOWN)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(res_full + EPI);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int total_tiles = p.work_items;  // work items (tiles, the tail split in halves)
  const uint32_t rank = (CG == 1) ? 0u : cluster_ctarank();
  const bool leader = rank == 0;
  const int unit = (CG == 1) ? static_cast<int>(blockIdx.x) : static_cast<int>(cluster_id_x());
  const int units = (CG == 1) ? static_cast<int>(gridDim.x) : static_cast<int>(nclusters_x());

  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
    tma_prefetch_desc(&tm_c);
    if ((KIND == KIND_DOWN || KIND == KIND_JOINT) && RING == 0 && p.residual != nullptr) tma_prefetch_desc(&tm_r);
    if (KIND == KIND_JOINT) {
      tma_prefetch_desc(&tm_a2);
      tma_prefetch_desc(&tm_b2);
    }
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], CG * EPI);  // one arrival per epilogue warp of each CTA
    }
    mbar_init(drain, 1);
    for (int i = 0; i < EPI; ++i) mbar_init(&res_full[i], 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc<CG>(tmem_slot, Tr::kTmemCols);
  tc_fence_before();
  if constexpr (CG == 1)
    __syncthreads();
  else
    cluster_sync();  // both CTAs' barriers exist before any cross-CTA arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Everything above may overlap the tail of the previous kernel in the stream;
  // nothing below reads global memory before that kernel has completed.
  grid_dependency_wait();
  grid_launch_dependents();
  // Status word as this launch found it: errors of earlier launches are not this one's.
  const int st0 = status_base(p.status);

  if (warp == 0) {
    // ------------------------------------------------ TMA producer (both CTAs)
    const uint64_t pol_b = l2_policy_evict_last();  // weights: reused by every tile
    int stage = 0;
    uint32_t phase = 0;
    int issued = 0;
    bool ok = true;
    for (int t = unit; t < total_tiles && ok; t += units) {
      int m_blk, n_col0;
      const bool half = work_coords<KIND, BN>(p, t, m_blk, n_col0);
      const int a_row = m_blk * Tr::kTileM + static_cast<int>(rank) * kBM;
      int b_row = n_col0 + static_cast<int>(rank) * ((half ? BN / 2 : BN) / CG);
      int b_row2 = b_row;  // KIND_HEAD, one CTA: the second vocabulary tile of the item
      if constexpr (head_pairs<KIND, BN>()) {
        // A CTA pair: each CTA loads its own vocabulary tile (BN / CG = 128 rows).  One
        // CTA: both tiles, as two 128-row boxes stacked in the stage.
        int mb, c0, c1;
        head_pair_coords(p, t, mb, c0, c1);
        if (!half) {
          b_row = (CG == 1 || rank == 0) ? c0 : c1;
          b_row2 = c1;
        }
      }
      // A half-width item loads half of B (and of the joint's B2) through maps with a
      // box of BN/2/CG rows.
      const CUtensorMap* map_b = half ? &tm_bh : &tm_b;
      const uint32_t stage_bytes = half ? Tr::kABytes + Tr::kBBytes / 2 : Tr::kStageBytes;
      // Load K-block kb of (ma, mb) into the next ring stage (warp-collective).
      auto issue = [&](const CUtensorMap* ma, const CUtensorMap* mb, int kb) -> bool {
        bool good = true;
        if (lane == 0) {
          good = mbar_wait(&empty[stage], phase ^ 1u, p.status, st0, kDevTimeoutProducer);
          if (good) {
            if constexpr (CG == 1) {
              mbar_arrive_expect_tx(&full[stage], stage_bytes);
              tma_load_2d(s_a + stage * Tr::kABytes, ma, &full[stage], kb * kBK, a_row, 0ull);
              tma_load_2d(s_b + stage * Tr::kBBytes, mb, &full[stage], kb * kBK, b_row, pol_b);
              if constexpr (head_pairs<KIND, BN>()) {
                if (!half)
                  tma_load_2d(s_b + stage * Tr::kBBytes + (BN / 2) * kBK * 2, mb, &full[stage], kb * kBK, b_row2,
                              pol_b);
              }
            } else {
              // Both CTAs' bytes land on the leader's barrier; only the leader arrives.
              if (leader) mbar_arrive_expect_tx(&full[stage], CG * stage_bytes);
              const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
              tma_load_2d_pair(s_a + stage * Tr::kABytes, ma, bar, kb * kBK, a_row, 0ull);
              tma_load_2d_pair(s_b + stage * Tr::kBBytes, mb, bar, kb * kBK, b_row, pol_b);
            }
          }
        }
        good = __shfl_sync(0xffffffffu, good, 0);
        if (good) {
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        return good;
      };
      if constexpr (KIND == KIND_JOINT) {
        // The attention-output branch first: every K-block of z and Wo.
        for (int kb = 0; kb < p.K2 / kBK && ok; ++kb) ok = issue(&tm_a2, half ? &tm_b2h : &tm_b2, kb);
        if (!ok) break;
      }
      if constexpr (G16) {
        // Four live 16-feature granules per stage: slot j holds the granule's 128 rows of
        // A (4 KiB) and BN/CG rows of B, each a 32B-swizzled box of 16 columns.
        constexpr uint32_t kSlotA = kBM * 32, kSlotB = (BN / CG) * 32;
        const uint32_t slot_bytes = kSlotA + (half ? kSlotB / 2 : kSlotB);
        int j = 0;
        auto flush = [&]() -> bool {  // the stage holds j granules: arm its barrier, move on
          if (lane == 0) {
            if constexpr (CG == 1)
              mbar_arrive_expect_tx(&full[stage], static_cast<uint32_t>(j) * slot_bytes);
            else if (leader)
              mbar_arrive_expect_tx(&full[stage], static_cast<uint32_t>(CG * j) * slot_bytes);
          }
          __syncwarp();
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
          j = 0;
          return true;
        };
        ok = for_each_live_g16<kGroups>(p, m_blk, lane, [&](int g) -> bool {
          bool good = true;
          if (lane == 0) {
            if (j == 0) good = mbar_wait(&empty[stage], phase ^ 1u, p.status, st0, kDevTimeoutProducer);
            if (good) {
              uint8_t* a_dst = s_a + stage * Tr::kABytes + j * kSlotA;
              uint8_t* b_dst = s_b + stage * Tr::kBBytes + j * kSlotB;
              if constexpr (CG == 1) {
                tma_load_2d(a_dst, &tm_a, &full[stage], g * 16, a_row, 0ull);
                tma_load_2d(b_dst, map_b, &full[stage], g * 16, b_row, pol_b);
              } else {
                const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
                tma_load_2d_pair(a_dst, &tm_a, bar, g * 16, a_row, 0ull);
                tma_load_2d_pair(b_dst, map_b, bar, g * 16, b_row, pol_b);
              }
            }
          }
          good = __shfl_sync(0xffffffffu, good, 0);
          if (!good) return false;
          if (++j == 4) flush();
          return true;
        });
        if (ok && j > 0) flush();
      } else if constexpr ((KIND == KIND_DOWN || KIND == KIND_JOINT) && CG == 1) {
        // A is h, mostly in HBM (written by the up projection, larger than L2): bring
        // its tiles into L2 kPrefetchAhead live K-blocks ahead of the loads.  This pays
        // for the single-CTA skipping kernels (4-6 % on tile-structured h); the pair
        // kernels are bound by the L2-to-SM operand stream instead, and lose 2-7 %.
        ok = for_each_live_kblock_ahead<KIND, kGroups, kPrefetchAhead>(
            p, m_blk, lane, [&](int kb, uint32_t) { return issue(&tm_a, map_b, kb); },
            [&](int kb) {
              if (lane == 0) tma_prefetch_l2_2d(&tm_a, kb * kBK, a_row);
            });
      } else {
        ok = for_each_live_kblock<KIND, kGroups>(p, m_blk, lane,
                                                 [&](int kb, uint32_t) { return issue(&tm_a, map_b, kb); });
      }
    }
    if (!ok && lane == 0) {
      // Error path: let the copies this warp started land before the CTA exits.
      if constexpr (CG == 1) {
        const int outstanding = issued < STAGES ? issued : STAGES;
        int s = stage;
        uint32_t ph = phase;
        for (int i = 0; i < outstanding; ++i) {
          if (--s < 0) {
            s = STAGES - 1;
            ph ^= 1u;
          }
          const uint64_t start = global_timer_ns();
          while (!mbar_try_wait(&full[s], ph)) {
            if (global_timer_ns() - start > SPMLP_WAIT_NS) {
              status_record(p.status, st0, kDevTimeoutDrain);
              break;
            }
          }
        }
      } else {
        // A pair's copies complete on the leader's barriers, which this CTA
        // cannot poll; give in-flight bulk copies (microseconds) time to land.
        const uint64_t start = global_timer_ns();
        while (global_timer_ns() - start < 200000ull) __nanosleep(1000);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer (leader CTA only)
    constexpr uint32_t idesc_full = umma_idesc_f16(Tr::kTileM, BN, BF16);
    constexpr uint32_t idesc_half = umma_idesc_f16(Tr::kTileM, BN / 2, BF16);
    if (leader) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      unsigned long long issued_steps = 0, skipped_steps = 0;
      const int k_steps_total = p.K / 16;
      for (int t = unit; t < total_tiles && ok; t += units) {
        int m_blk, n_col0;
        const bool half = work_coords<KIND, BN>(p, t, m_blk, n_col0);
        const uint32_t idesc = half ? idesc_half : idesc_full;
        // Counted per whole tile: a split tile's second half adds nothing.  A head
        // item counts per 128-token x 128-column tile, as the single-CTA head does:
        // its vocabulary tiles times the 128-token halves of its M-block in range.
        unsigned long long weight = (!half || ((t - p.tail_from) & 1) == 0) ? 1ull : 0ull;
        if constexpr (head_pairs<KIND, BN>())
          weight = (half ? 1ull : 2ull) * (CG == 2 && m_blk * Tr::kTileM + kBM < p.M ? 2ull : 1ull);
        // A tile without live K-blocks needs no MMA: the epilogue writes the
        // zero-accumulator result itself (the joint always has its z branch).  The live
        // K16 steps of the others are counted while their MMAs are issued below.
        if (KIND != KIND_JOINT && !any_live<KIND, kGroups, G16>(p, m_blk, lane)) {
          skipped_steps += weight * static_cast<unsigned long long>(k_steps_total);
          continue;
        }
        if (lane == 0) ok = mbar_wait(&acc_empty[acc], acc_phase ^ 1u, p.status, st0, kDevTimeoutMma);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc) * Tr::kAccCols;
        // MMAs of the next ring stage into accumulator d (warp-collective).
        auto mma_stage = [&](uint32_t d, uint32_t k16, uint32_t& accumulate) -> bool {
          bool good = true;
          if (lane == 0) {
            good = mbar_wait(&full[stage], phase, p.status, st0, kDevTimeoutMma);
            if (good) {
              tc_fence_after();
              const uint64_t a_desc = sw128_kmajor_desc(smem_u32(s_a + stage * Tr::kABytes));
              const uint64_t b_desc = sw128_kmajor_desc(smem_u32(s_b + stage * Tr::kBBytes));
#pragma unroll
              for (int k = 0; k < kBK / 16; ++k) {
                if ((k16 >> k) & 1u) {
                  // +32 bytes per K16 step inside the 128-byte swizzled row (>>4 encoded)
                  umma_f16<CG>(d, a_desc + static_cast<uint64_t>(2 * k), b_desc + static_cast<uint64_t>(2 * k), idesc,
                               accumulate);
                  accumulate = 1;
                }
              }
              umma_commit<CG>(&empty[stage]);
            }
          }
          good = __shfl_sync(0xffffffffu, good, 0);
          if (good && ++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
          return good;
        };
        if constexpr (KIND == KIND_JOINT) {
          // z Wo^T into the second accumulator, in the order the producer loaded it.
          uint32_t accumulate_z = 0;
          for (int kb = 0; kb < p.K2 / kBK && ok; ++kb) ok = mma_stage(d_tmem + BN, 0xFu, accumulate_z);
          if (!ok) break;
        }
        uint32_t accumulate = 0;
        int live_steps = 0;
        if constexpr (G16) {
          // One K16 MMA per gathered granule, four per stage (the producer's grouping).
          constexpr uint32_t kSlotA = kBM * 32, kSlotB = (BN / CG) * 32;
          int j = 0;
          auto release_stage = [&]() {
            if (lane == 0) umma_commit<CG>(&empty[stage]);
            __syncwarp();
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
            j = 0;
          };
          ok = for_each_live_g16<kGroups>(p, m_blk, lane, [&](int) -> bool {
            bool good = true;
            if (lane == 0) {
              if (j == 0) {
                good = mbar_wait(&full[stage], phase, p.status, st0, kDevTimeoutMma);
                if (good) tc_fence_after();
              }
              if (good) {
                const uint64_t a_desc = sw32_kmajor_desc(smem_u32(s_a + stage * Tr::kABytes + j * kSlotA));
                const uint64_t b_desc = sw32_kmajor_desc(smem_u32(s_b + stage * Tr::kBBytes + j * kSlotB));
                umma_f16<CG>(d_tmem, a_desc, b_desc, idesc, accumulate);
                accumulate = 1;
              }
            }
            good = __shfl_sync(0xffffffffu, good, 0);
            if (!good) return false;
            ++live_steps;
            if (++j == 4) release_stage();
            return true;
          });
          if (ok && j > 0) release_stage();
        } else {
          ok = for_each_live_kblock<KIND, kGroups>(p, m_blk, lane, [&](int, uint32_t k16) {
            live_steps += __popc(k16);
            return mma_stage(d_tmem, k16, accumulate);
          });
        }
        if (!ok) break;
        skipped_steps += weight * static_cast<unsigned long long>(k_steps_total - live_steps);
        issued_steps += weight * static_cast<unsigned long long>(live_steps);
        if (lane == 0) umma_commit<CG>(&acc_full[acc]);
        __syncwarp();
        if (++acc == Tr::kAccBufs) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (lane == 0) {
        // Wait for every MMA this thread issued before TMEM is released.
        umma_commit_local<CG>(drain);
        const uint64_t start = global_timer_ns();
        while (!mbar_try_wait(drain, 0)) {
          if (global_timer_ns() - start > SPMLP_WAIT_NS) {
            status_record(p.status, st0, kDevTimeoutDrain);
            break;
          }
        }
        if (p.stats != nullptr && KIND != KIND_UP) {
          atomicAdd(p.stats + 0, issued_steps);
          atomicAdd(p.stats + 1, skipped_steps);
        }
      }
    }
  } else {
    // ------------------------------------------------ epilogue warps (both CTAs)
    const int ew = warp - 2;               // 0 .. EPI-1
    const int quarter = warp & 3;          // TMEM lanes 32*quarter .. +31 (hardware rule: warp id % 4)
    constexpr int kMyChunks = Tr::kWarpChunks;
    constexpr int kBatches = (kMyChunks + Tr::kFlush - 1) / Tr::kFlush;
    // EPI == 8: the two warps of a quarter split the columns of a tile (or of a
    // half-width item) in two; this warp's first chunk of an item:
    const int col_part = ew / 4;
    auto first_chunk = [&](bool half) { return col_part * (half ? kMyChunks / 2 : kMyChunks); };
    constexpr bool kRing = RING > 0;
    uint8_t* stage_out = s_out + ew * Tr::kSlabChunks * Tr::kStageOutBytes;
    float* bias_s = s_bias + ew * kMyChunks * 32;  // this warp's columns, from its first chunk on
    float* bias2_s = bias_s + EPI * kMyChunks * 32;  // KIND_JOINT: the second product's bias; KIND_UP: ln_c
    constexpr bool ln = LN && KIND == KIND_UP;
    constexpr bool kHasRes = KIND == KIND_DOWN || KIND == KIND_JOINT;
    const bool with_res = kHasRes && p.residual != nullptr;
    const bool scatter = KIND == KIND_DOWN && p.scatter_rows > 0;
    int ring_slot = 0;  // RING > 0: next slot of this warp's ring (carries across tiles)
    // The accumulator-release barriers live in the leader CTA.
    // The two barriers are adjacent, so the leader's copy of barrier i is at base + 8 i
    // (computed rather than indexed from an array, which would live in local memory).
    const uint32_t acc_empty_leader = (CG == 1) ? smem_u32(&acc_empty[0]) : mapa_shared(smem_u32(&acc_empty[0]), 0);
    int acc = 0;
    uint32_t acc_phase = 0, res_phase = 0;
    const uint32_t k2 = DType<BF16>::pack_rn(p.kappa, p.kappa);  // kappa in both halves (exact: pre-rounded)

    // Bias of one tile's columns for this warp: lane l holds 8 values (one 16-byte vector).
    const bool bias_lane = KIND != KIND_HEAD && lane * 8 < kMyChunks * 32;
    auto load_bias = [&](const void* bias, int t) -> uint4 {
      uint4 raw = make_uint4(0u, 0u, 0u, 0u);
      if (bias_lane && bias != nullptr && t < total_tiles) {
        int mb, nc;
        const bool hf = work_coords<KIND, BN>(p, t, mb, nc);
        const int col = nc + first_chunk(hf) * 32 + lane * 8;
        if (col < p.N) raw = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(bias) + col));
      }
      return raw;
    };
    // Eight packed dtype values -> eight fp32 values at dst.
    auto store_bias = [&](const uint4& raw, float* dst) {
      const uint16_t* hb = reinterpret_cast<const uint16_t*>(&raw);
      float b[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) b[i] = DType<BF16>::to_float(hb[i]);
      reinterpret_cast<float4*>(dst)[0] = make_float4(b[0], b[1], b[2], b[3]);
      reinterpret_cast<float4*>(dst)[1] = make_float4(b[4], b[5], b[6], b[7]);
    };
    uint4 bias_next = load_bias(p.bias, unit);
    uint4 bias2_next = KIND == KIND_JOINT ? load_bias(p.bias2, unit) : make_uint4(0u, 0u, 0u, 0u);
    // Folded LayerNorm: eight fp32 columns of ln_s and ln_c per lane, one tile ahead.
    float4 lns_next[2], lnc_next[2];
    auto load_ln = [&](int t) {
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      lns_next[0] = lns_next[1] = lnc_next[0] = lnc_next[1] = z;
      if (bias_lane && t < total_tiles) {
        int mb, nc;
        const bool hf = work_coords<KIND, BN>(p, t, mb, nc);
        const int col = nc + first_chunk(hf) * 32 + lane * 8;
        if (col < p.N) {
          const float4* sp = reinterpret_cast<const float4*>(p.ln_s + col);
          const float4* cp = reinterpret_cast<const float4*>(p.ln_c + col);
          lns_next[0] = __ldg(sp);
          lns_next[1] = __ldg(sp + 1);
          lnc_next[0] = __ldg(cp);
          lnc_next[1] = __ldg(cp + 1);
        }
      }
    };
    if constexpr (ln) load_ln(unit);

    for (int t = unit; t < total_tiles; t += units) {
      int m_blk, n_col0;
      const bool half = work_coords<KIND, BN>(p, t, m_blk, n_col0);
      // Output column of chunk ch: a pair of vocabulary tiles maps chunks 4.. to the second tile.
      int n_col1 = n_col0;
      if constexpr (head_pairs<KIND, BN>()) {
        int mb, c0;
        head_pair_coords(p, t, mb, c0, n_col1);
      }
      auto chunk_col = [&](int ch) {
        if constexpr (head_pairs<KIND, BN>()) return ch < 4 ? n_col0 + ch * 32 : n_col1 + (ch - 4) * 32;
        return n_col0 + ch * 32;
      };
      int live_blocks = 1;  // > 0: the MMA warp wrote this item's accumulator
      if constexpr (KIND != KIND_UP) live_blocks = any_live<KIND, kGroups, G16>(p, m_blk, lane) ? 1 : 0;
      const int row0 = m_blk * Tr::kTileM + static_cast<int>(rank) * kBM + quarter * 32;
      const int row = row0 + lane;
      const bool row_ok = row < p.M;
      const bool has_acc = KIND == KIND_JOINT || live_blocks > 0;  // the joint's z branch is never empty
      // Folded LayerNorm: this thread's row statistics.
      const float row_mean = (ln && row_ok) ? __ldg(p.ln_mean + row) : 0.f;
      const float row_rstd = (ln && row_ok) ? __ldg(p.ln_rstd + row) : 0.f;
      const bool has_h = live_blocks > 0;                             // KIND_JOINT: the h accumulator was written
      const int ch_begin = first_chunk(half);
      const int ch_end = ch_begin + (half ? kMyChunks / 2 : kMyChunks);
      // RING > 0: the residual of chunk ch (this thread's row, 32 values) into registers.
      auto load_res = [&](int ch, uint4 (&r)[4]) {
        if constexpr (kRing && kHasRes) {
          const int col0 = n_col0 + ch * 32;
          if (with_res && row_ok && ch < ch_end && col0 < p.N) {
            const uint4* rp = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.residual) +
                                                             static_cast<size_t>(row) * p.N + col0);
#pragma unroll
            for (int c = 0; c < 4; ++c) r[c] = __ldg(rp + c);
          }
        }
      };
      // Residual registers of the two chunks in flight, fetched before the accumulator wait.
      const uint4 z4 = make_uint4(0u, 0u, 0u, 0u);
      uint4 res_a[4] = {z4, z4, z4, z4};
      uint4 res_b[4] = {z4, z4, z4, z4};
      load_res(ch_begin, res_a);
      load_res(ch_begin + 1, res_b);

      // Residual: TMA it into this warp's output slab while the MMAs run.  The
      // previous tile's stores must first have read the slab.
      if (!kRing && with_res) {
        if (lane == 0) {
          bulk_wait_group_read<0>();
          if (row0 < p.M) {
            int n_in = 0;
            for (int i = 0; i < kMyChunks; ++i) n_in += (n_col0 + (ch_begin + i) * 32 < p.N) ? 1 : 0;
            mbar_arrive_expect_tx(&res_full[ew], n_in * Tr::kStageOutBytes);
            for (int i = 0; i < kMyChunks; ++i) {
              const int c0 = n_col0 + (ch_begin + i) * 32;
              if (c0 < p.N) tma_load_2d(stage_out + i * Tr::kStageOutBytes, &tm_r, &res_full[ew], c0, row0, 0ull);
            }
          }
        }
        __syncwarp();
      }

      // Bias of this tile -> shared memory (fp32); the next tile's is fetched now.
      if constexpr (KIND != KIND_HEAD) {
        __syncwarp();  // every lane is done with the previous tile's bias
        if (lane * 8 < kMyChunks * 32) {
          if constexpr (ln) {
            reinterpret_cast<float4*>(bias_s + lane * 8)[0] = lns_next[0];
            reinterpret_cast<float4*>(bias_s + lane * 8)[1] = lns_next[1];
            reinterpret_cast<float4*>(bias2_s + lane * 8)[0] = lnc_next[0];
            reinterpret_cast<float4*>(bias2_s + lane * 8)[1] = lnc_next[1];
          } else {
            store_bias(bias_next, bias_s + lane * 8);
          }
          if constexpr (KIND == KIND_JOINT) store_bias(bias2_next, bias2_s + lane * 8);
        }
        __syncwarp();
        bias_next = load_bias(p.bias, t + units);
        if constexpr (KIND == KIND_JOINT) bias2_next = load_bias(p.bias2, t + units);
        if constexpr (ln) load_ln(t + units);
      }

      if (has_acc) {
        // Every lane observes the barrier itself before reading TMEM.
        const bool good = __all_sync(0xffffffffu, mbar_wait(&acc_full[acc], acc_phase, p.status, st0, kDevTimeoutEpilogue));
        if (!good) break;
        tc_fence_after();
      }
      if (!kRing && with_res && row0 < p.M) {
        const bool good = __all_sync(0xffffffffu, mbar_wait(&res_full[ew], res_phase, p.status, st0, kDevTimeoutEpilogue));
        res_phase ^= 1u;
        if (!good) break;
      }
      const uint32_t t_row =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc) * Tr::kAccCols;

      // Release the accumulator (once per warp) when its last TMEM load completed.
      auto release_acc = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (CG == 1)
            mbar_arrive(&acc_empty[acc]);
          else
            mbar_arrive_cluster(acc_empty_leader + 8u * static_cast<uint32_t>(acc));
        }
      };

      uint32_t nz_bits = 0;  // KIND_UP: bit (2*group + half) per 64-column group of the tile
      const int sw = (lane >> 1) & 3;  // 64-byte swizzle of this lane's row in a 32x32 chunk
      // v: the chunk's accumulator values (KIND_JOINT: of h W2^T, with v2 those of z Wo^T).
      auto process = [&](int ch, const uint32_t (&v)[32], const uint32_t (&v2)[32], const uint4 (&res_regs)[4]) {
        const int col0 = chunk_col(ch);
        const int slot = ch - ch_begin;
        uint8_t* buf = stage_out + (kRing ? ring_slot : slot) * Tr::kStageOutBytes;
        if constexpr (kRing) {
          // The store that last used this slot, RING chunks ago, has read it.
          if (lane == 0) bulk_wait_group_read<(RING > 0 ? RING - 1 : 0)>();
          __syncwarp();
        } else if (!with_res && slot % Tr::kFlush == 0) {
          // The store batch that last used these slots has read them.
          if (lane == 0) bulk_wait_group_read<kBatches - 1>();
          __syncwarp();
        }
        if (col0 < p.N) {  // N is a multiple of 64: a chunk is wholly in or out of range
          uint32_t packed[16];
          bool nz = false;
          if constexpr (KIND == KIND_UP) {
            nz = UpEpilogue<BF16, GATE>::apply(p, row, col0, lane, row_ok, v, bias_s + slot * 32, k2, packed,
                                               ln ? bias2_s + slot * 32 : nullptr, row_mean, row_rstd);
          } else if constexpr (KIND == KIND_DOWN) {
            uint4 r[4] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u),
                          make_uint4(0u, 0u, 0u, 0u)};
            if (with_res) {
#pragma unroll
              for (int c = 0; c < 4; ++c)
                r[c] = kRing ? res_regs[c] : *reinterpret_cast<const uint4*>(buf + lane * 64 + ((c ^ sw) << 4));
            }
            DownEpilogue<BF16>::apply(p, v, bias_s + slot * 32, r, packed);
          } else if constexpr (KIND == KIND_JOINT) {
            const uint4 z4r = make_uint4(0u, 0u, 0u, 0u);
            uint4 r[4] = {z4r, z4r, z4r, z4r};
            if (with_res) {
#pragma unroll
              for (int c = 0; c < 4; ++c)
                r[c] = kRing ? res_regs[c] : *reinterpret_cast<const uint4*>(buf + lane * 64 + ((c ^ sw) << 4));
            }
            JointEpilogue<BF16>::apply(v, v2, bias_s + slot * 32, bias2_s + slot * 32, r, with_res, packed);
          } else {
            HeadEpilogue<BF16>::apply(v, packed);
          }
          if constexpr (KIND == KIND_UP) {
            const uint32_t ball = __ballot_sync(0xffffffffu, nz);
            const int grp = ch >> 1;
            if (ball & 0x0000ffffu) nz_bits |= 1u << (2 * grp);
            if (ball & 0xffff0000u) nz_bits |= 1u << (2 * grp + 1);
          }
          // Stage the 32x32 chunk (64-byte rows, 64-byte swizzle) in this warp's tile slab.
#pragma unroll
          for (int c = 0; c < 4; ++c)
            *reinterpret_cast<uint4*>(buf + lane * 64 + ((c ^ sw) << 4)) =
                make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
          if (scatter) {
            // The partial chunk goes to its token block's owner (peer memory over
            // NVLink), read back from the slab so that one store instruction writes
            // eight whole 64-byte row segments: lane l moves 16 bytes of row l / 4.
            __syncwarp();
            const int owner = row0 / p.scatter_rows;  // token blocks hold whole tiles
            uint16_t* dst_base = static_cast<uint16_t*>(p.scatter_out[owner]) +
                                 static_cast<size_t>(row0 - owner * p.scatter_rows) * p.N + col0;
            const int piece = lane & 3;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int r = 8 * i + (lane >> 2);
              if (row0 + r < p.M) {
                const uint4 v = *reinterpret_cast<const uint4*>(buf + r * 64 + ((piece ^ ((r >> 1) & 3)) << 4));
                *reinterpret_cast<uint4*>(dst_base + static_cast<size_t>(r) * p.N + piece * 8) = v;
              }
            }
            __syncwarp();  // the slot is rewritten by the next chunk
          }
        }
        if (scatter) return;  // nothing staged for a TMA store
        if constexpr (kRing) {
          // One fence and one TMA store per chunk; the slot is reused RING chunks later.
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (row0 < p.M && col0 < p.N) tma_store_2d(&tm_c, buf, col0, row0);
            bulk_commit_group();
          }
          ring_slot = ring_slot + 1 == RING ? 0 : ring_slot + 1;
        } else if ((slot + 1) % Tr::kFlush == 0 || slot + 1 == kMyChunks) {
          // Every kFlush chunks: one fence and one batch of TMA stores for the staged chunks.
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && row0 < p.M) {
            for (int i = slot - slot % Tr::kFlush; i <= slot; ++i) {
              const int c0 = n_col0 + (ch_begin + i) * 32;
              if (c0 < p.N) tma_store_2d(&tm_c, stage_out + i * Tr::kStageOutBytes, c0, row0);
            }
          }
          if (lane == 0) bulk_commit_group();
        }
      };

      if constexpr (KIND == KIND_JOINT) {
        // Two accumulators per chunk: h W2^T at t_row, z Wo^T at t_row + BN.
        auto joint_chunk = [&](int ch, const uint4 (&res_regs)[4]) {
          uint32_t vh[32], vz[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) vh[j] = 0u;  // h without live K-blocks contributes zero
          if (has_h) tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(ch * 32), vh);
          tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(BN + ch * 32), vz);
          tmem_wait_ld(vz);
          tmem_pin(vh);
          if (ch + 1 == ch_end) release_acc();
          process(ch, vh, vz, res_regs);
        };
#pragma unroll 1
        for (int ch = ch_begin; ch < ch_end; ch += 2) {
          joint_chunk(ch, res_a);
          load_res(ch + 2, res_a);
          if (ch + 1 < ch_end) {
            joint_chunk(ch + 1, res_b);
            load_res(ch + 3, res_b);
          }
        }
      } else {
        uint32_t va[32], vb[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) va[j] = vb[j] = 0u;
        if (has_acc) tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(ch_begin * 32), va);
#pragma unroll 1
        for (int ch = ch_begin; ch < ch_end; ch += 2) {
          // even chunk: va
          if (has_acc) {
            tmem_wait_ld(va);
            if (ch + 1 < ch_end) tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>((ch + 1) * 32), vb);
            if (ch + 1 >= ch_end) release_acc();
          }
          process(ch, va, va, res_a);
          load_res(ch + 2, res_a);
          if (ch + 1 < ch_end) {
            // odd chunk: vb
            if (has_acc) {
              tmem_wait_ld(vb);
              if (ch + 2 < ch_end) tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>((ch + 2) * 32), va);
              if (ch + 2 >= ch_end) release_acc();
            }
            process(ch + 1, vb, vb, res_b);
            load_res(ch + 3, res_b);
          }
        }
      }
      if constexpr (KIND == KIND_UP) {
        // Publish this warp's 16x64 bits: two 16-row groups per warp quarter.  Every bit
        // of the bitmap belongs to exactly one warp (its 64 columns, its 16 rows), which
        // writes it whether set or clear: an AND clears the warp's dead groups and an OR
        // sets its live ones, so the buffer needs no clearing before the launch and
        // whatever it held is overwritten.
        if (lane == 0) {
          const int g0 = n_col0 / kBitsCols;  // first 64-column group of the tile
          const int word = g0 >> 5;
          const int shift = g0 & 31;          // BN/64 <= 4 groups stay inside one word
          const int row_groups = (p.M + kBitsRows - 1) / kBitsRows;
          uint32_t own = 0;                   // this warp's groups (two 32-column chunks each)
          for (int grp = ch_begin >> 1; grp < (ch_end >> 1); ++grp)
            if (n_col0 + grp * kBitsCols < p.N) own |= 1u << (shift + grp);
          // The owner of the last 64-column group also clears the unused bits above it.
          const int g_last = p.N / kBitsCols - 1;
          if ((g_last >> 5) == word && ((own >> (g_last & 31)) & 1u)) own |= ~((2u << (g_last & 31)) - 1u);
          for (int half = 0; half < 2; ++half) {
            const int rg = (row0 >> 4) + half;
            if (rg >= row_groups || own == 0) continue;
            uint32_t w = 0;
            for (int grp = 0; grp < BN / kBitsCols; ++grp)
              if ((nz_bits >> (2 * grp + half)) & 1u) w |= 1u << (shift + grp);
            uint32_t* wp = p.bits_out + static_cast<size_t>(rg) * p.bits_words + word;
            if (w != own) atomicAnd(wp, ~own | w);
            if (w != 0) atomicOr(wp, w);
          }
        }
      }
      if (has_acc && ++acc == Tr::kAccBufs) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (scatter) __threadfence_system();  // peer stores are performed before the kernel completes
    if (lane == 0) bulk_wait_group<0>();  // stores complete before the CTA's shared memory goes away
    __syncwarp();
  }

  tc_fence_before();
  if constexpr (CG == 1)
    __syncthreads();
  else
    cluster_sync();  // the pair's MMAs and cross-CTA arrivals are finished
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<CG>(tmem_base, Tr::kTmemCols);
  }
}

}  // namespace spmlp
