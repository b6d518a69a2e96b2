// Host side of libspmlp.so: argument checks, TMA tensor maps, launches and the
// extern "C" entry points declared in include/spmlp.h.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <mutex>
#include <string>

#include "gemm_sm100.cuh"
#include "head_prepare.cuh"
#include "bitmap.cuh"
#include "collective.cuh"
#include "layernorm.cuh"
#include "mask_format.cuh"
#include "spmlp.h"

namespace spmlp {

// One status word per device, written only by kernels that give up on a wait.
__device__ int g_device_status = 0;

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
  return static_cast<int>(e);
}

constexpr int kMaxDevices = 64;
constexpr int kProgrammaticLaunch = 1;  // GEMM launches overlap the previous kernel's tail

// Tile configuration of the up-projection: pipeline stages, epilogue warps,
// CTAs per tile, output ring slots per epilogue warp (0 = whole-tile slab).
constexpr int kUpBN = 256, kUpStages = 4, kUpEpiWarps = 8, kUpCG = 2, kUpRing = 0;
// Up-projection with few tiles (e.g. the 14M shape): 128 x 128 tiles on single CTAs.
constexpr int kUpSmallBN = 128;
// Down-projection, dense and coarse-skip modes: 256-token tiles on CTA pairs.
// Its long reduction (K = d_ff) leaves the epilogue idle most of the time, so
// four epilogue warps and a two-slot output ring suffice, and the shared memory
// goes to six operand stages (the loads of h are the bound).
constexpr int kDownStages = 6, kDownEpiWarps = 4, kDownCG = 2, kDownRing = 2;
// Down-projection with d <= 128 (the 14M shape): 128-column tiles on the pairs; each
// stage is 16 KiB of h and 8 KiB of W_out per CTA.  Eight epilogue warps (two chunks each:
// few tiles, so the epilogue is on the critical path) and seven stages fit.
constexpr int kDownNarrowBN = 128, kDownNarrowStages = 7, kDownNarrowEpiWarps = 8;
// Down-projection, fine-skip mode: 128-token tiles on single CTAs.
constexpr int kDownFineBN = 256, kDownFineStages = 4, kDownFineEpiWarps = 4, kDownFineRing = 2;
// Vocabulary head: 128 x 128 tiles on single CTAs.
constexpr int kHeadStages = 4, kHeadEpiWarps = 8, kHeadRing = 2;
// Dense and N-gated head: work items of two vocabulary tiles on a CTA pair (256 x 256).
constexpr int kHeadPairStages = 5, kHeadPairEpiWarps = 8, kHeadPairRing = 2;
// Head on one CTA with two vocabulary tiles per item (dense and N gate below kHeadPairMinD,
// the K gate always; 0 = one tile per item).  Measured on B200, cfg4 shapes: 1.2-1.4x faster
// than one tile per item at d = 128 (N gate, 5-100 % active tiles), 1.6-1.9x for the K gate,
// 1.1-1.2x faster than the pair kernel at d = 256; the pair kernel wins at d = 512 (its
// operand stream is half).
constexpr int kHeadWide = 1, kHeadWideStages = 3, kHeadWideEpiWarps = 8, kHeadWideRing = 2;
constexpr int kHeadPairMinD = 512;  // d from which the pair kernel is faster
// Joint consumer: 256 output columns per tile, so that h is read by only d/256
// column tiles; the tile's two accumulators then fill TMEM's 512 columns and are
// single-buffered (measured on cfg1: 96 us against 121 us for double-buffered
// 128-column tiles, which read h twice as often).
constexpr int kJointBN = 256, kJointStages = 5, kJointEpiWarps = 8, kJointRing = 2;
constexpr int kJointFineStages = 4, kJointFineEpiWarps = 4;

struct DeviceInfo {
  int sm_count = 0;
  int sm_target = 0;    // spmlp_set_sm_count_target: SMs the persistent GEMMs may use (0 = all)
  int* status = nullptr;
  void* ctx = nullptr;  // the context the cached addresses belong to
  bool ok = false;
};

std::mutex g_dev_mutex;
DeviceInfo g_dev[kMaxDevices];

// The calling thread's current CUDA context (driver handle), or null.  Device
// addresses of this module's __device__ variables belong to one context: after a
// cudaDeviceReset the runtime loads the module again into a new primary context,
// and addresses cached for the old one are stale.
void* current_context() {
  typedef int (*CtxGetCurrentFn)(void**);
  static CtxGetCurrentFn fn = []() -> CtxGetCurrentFn {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<CtxGetCurrentFn>(ptr);
  }();
  void* ctx = nullptr;
  if (fn == nullptr || fn(&ctx) != 0) return nullptr;
  return ctx;
}

int current_device_info(DeviceInfo** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(SPMLP_EDEVICE, "device index %d out of range", dev);
  // Null until the runtime has made the device's primary context current on this
  // thread; the symbol lookup below does that, so the entry is then refreshed once.
  void* ctx = current_context();
  std::lock_guard<std::mutex> lock(g_dev_mutex);
  DeviceInfo& info = g_dev[dev];
  if (!info.ok || ctx == nullptr || info.ctx != ctx) {
    info.ok = false;
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major != 10 || minor != 0)
      return fail(SPMLP_EDEVICE, "device %d is sm_%d%d; libspmlp is built for sm_100a only", dev, major, minor);
    e = cudaDeviceGetAttribute(&info.sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
    void* addr = nullptr;
    e = cudaGetSymbolAddress(&addr, g_device_status);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(status word)");
    info.status = static_cast<int*>(addr);
    info.ctx = current_context();
    info.ok = true;
  }
  *out = &info;
  return 0;
}

// ---------------------------------------------------------------- tensor maps
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(ptr);
  }();
  return fn;
}

// K-major operand [rows, k] -> box of 64 (k) x box_rows, 128-byte swizzle; with
// box_k = 16, a box of one K16 step (32 bytes per row) and 32-byte swizzle.
int make_kmajor_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t k, int box_rows, bool bf16,
                    int box_k = kBK) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(SPMLP_EDRIVER, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(k) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_k), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = box_k == 16 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_128B;
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SPMLP_EDRIVER, "cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
  return 0;
}

// Row-major output [rows, cols] written in 32-row x 32-column boxes with 64-byte swizzle.
int make_out_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, bool bf16) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(SPMLP_EDRIVER, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SPMLP_EDRIVER, "cuTensorMapEncodeTiled (output) failed (CUresult %d)", static_cast<int>(r));
  return 0;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------- launch
template <int KIND, int GATE, int BN, int STAGES, bool BF16, int EPI, int CG, int RING = 0, bool LN = false,
          bool G16 = false>
int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, GemmParams p,
                cudaStream_t stream, DeviceInfo* dev, const CUtensorMap* tr = nullptr,
                const CUtensorMap* ta2 = nullptr, const CUtensorMap* tb2 = nullptr,
                const CUtensorMap* tbh = nullptr, const CUtensorMap* tb2h = nullptr) {
  using Tr = GemmTraits<KIND, BN, STAGES, BF16, EPI, CG, RING>;
  auto kernel = gemm_sm100_kernel<KIND, GATE, BN, STAGES, BF16, EPI, CG, RING, LN, G16>;
  // Setting the attribute is per function; cheap and idempotent.
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Tr::kSmemBytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(max dynamic smem)");
  p.m_tiles = (p.M + Tr::kTileM - 1) / Tr::kTileM;
  // A head work item of BN = 256 holds two 128-column vocabulary tiles (n_tiles counts those).
  const int n_items = head_pairs<KIND, BN>() ? (p.n_tiles + 1) / 2 : p.n_tiles;
  const int tiles = p.m_tiles * n_items;
  if (tiles == 0) return 0;
  p.tail_from = p.work_items = tiles;
  p.status = dev->status;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  cfg.blockDim = dim3(Tr::kThreads);
  cfg.dynamicSmemBytes = Tr::kSmemBytes;
  cfg.stream = stream;
  // Programmatic dependent launch: this kernel's set-up may overlap the previous
  // kernel's tail (the kernel waits with griddepcontrol.wait before reading inputs).
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = kProgrammaticLaunch;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int units = dev->sm_count;  // persistent: one CTA (or CTA pair) per SM (pair)
  if constexpr (CG > 1) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(cluster size)");
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = CG;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
    // Clusters that can be resident at once, queried once per device for this kernel.
    static int max_clusters[kMaxDevices] = {};
    int dev_id = 0;
    cudaGetDevice(&dev_id);
    if (max_clusters[dev_id] == 0) {
      cudaLaunchConfig_t query = cfg;  // the cluster shape alone decides residency
      query.gridDim = dim3(dev->sm_count);
      query.attrs = &attr[1];
      query.numAttrs = 1;
      int n = 0;
      e = cudaOccupancyMaxActiveClusters(&n, kernel, &query);
      if (e != cudaSuccess || n <= 0) return cuda_fail(e == cudaSuccess ? cudaErrorInvalidConfiguration : e,
                                                       "cudaOccupancyMaxActiveClusters");
      max_clusters[dev_id] = n;
    }
    units = max_clusters[dev_id];
  }
  // A caller that runs other kernels beside the GEMMs (a reduction over NVLink on another
  // stream) leaves them SMs by capping the persistent grid.
  if (dev->sm_target > 0) units = std::min(units, std::max(1, dev->sm_target / CG));
  // The last round of the persistent grid: when it would leave at least half of the
  // units idle, its tiles run as two half-width items each (the down projection and
  // the joint consumer, whose epilogue warps write through an output ring).
  if constexpr ((KIND == KIND_DOWN || KIND == KIND_JOINT) && RING > 0) {
    if (p.split_tail && tiles > units) {
      const int rem = tiles % units;
      if (rem > 0 && 2 * rem <= units) {
        p.tail_from = tiles - rem;
        p.work_items = tiles + rem;
      }
    }
  }
  if (p.work_items < units) units = p.work_items;
  cfg.gridDim = dim3(units * CG);
  e = cudaLaunchKernelEx(&cfg, kernel, ta, tb, tc, tr != nullptr ? *tr : tc, ta2 != nullptr ? *ta2 : ta,
                         tb2 != nullptr ? *tb2 : tb, tbh != nullptr ? *tbh : tb, tb2h != nullptr ? *tb2h : tb, p);
  if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
  return 0;
}

// Up-projection launch with the gate operator (and the folded LayerNorm) as
// compile-time parameters.
template <int BN, int G, bool SMALL>
int launch_up_gate(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmParams& p,
                   bool bf16, bool ln, cudaStream_t stream, DeviceInfo* dev) {
  constexpr int S = kUpStages, E = kUpEpiWarps, C = SMALL ? 1 : kUpCG, R = kUpRing;
  if (ln)
    return bf16 ? launch_gemm<KIND_UP, G, BN, S, true, E, C, R, true>(ta, tb, tc, p, stream, dev)
                : launch_gemm<KIND_UP, G, BN, S, false, E, C, R, true>(ta, tb, tc, p, stream, dev);
  return bf16 ? launch_gemm<KIND_UP, G, BN, S, true, E, C, R>(ta, tb, tc, p, stream, dev)
              : launch_gemm<KIND_UP, G, BN, S, false, E, C, R>(ta, tb, tc, p, stream, dev);
}

template <int BN, bool SMALL>
int launch_up(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmParams& p, int gate_op,
              bool bf16, cudaStream_t stream, DeviceInfo* dev) {
  const bool ln = p.ln_c != nullptr;
#define SPMLP_UP_CASE(G) \
  case G:                \
    return launch_up_gate<BN, G, SMALL>(ta, tb, tc, p, bf16, ln, stream, dev);
  switch (gate_op) {
    SPMLP_UP_CASE(GATE_IDENTITY)
    SPMLP_UP_CASE(GATE_GELU)
    SPMLP_UP_CASE(GATE_ONE_SIDED)
    SPMLP_UP_CASE(GATE_SYMMETRIC)
    SPMLP_UP_CASE(GATE_RELU)
    SPMLP_UP_CASE(GATE_GELU_MASKED)
    SPMLP_UP_CASE(GATE_CORNER)
    default:
      return fail(SPMLP_EINVAL, "unknown gate_op %d", gate_op);
  }
#undef SPMLP_UP_CASE
}

int check_dtype(int dtype) {
  if (dtype != SPMLP_F16 && dtype != SPMLP_BF16) return fail(SPMLP_EINVAL, "dtype must be SPMLP_F16 or SPMLP_BF16");
  return 0;
}

int check_gate(int gate_op, float kappa, int64_t T, int64_t seq_len) {
  if (gate_op < SPMLP_GATE_IDENTITY || gate_op > SPMLP_GATE_CORNER) return fail(SPMLP_EINVAL, "unknown gate_op %d", gate_op);
  const bool uses_kappa = gate_op == SPMLP_GATE_ONE_SIDED || gate_op == SPMLP_GATE_SYMMETRIC ||
                          gate_op == SPMLP_GATE_GELU_MASKED || gate_op == SPMLP_GATE_CORNER;
  if (uses_kappa && (!std::isfinite(kappa) || kappa < 0.f))
    return fail(SPMLP_EINVAL, "kappa must be a finite nonnegative number");
  if (gate_op == SPMLP_GATE_CORNER) {
    if (seq_len <= 0) return fail(SPMLP_EINVAL, "corner gate needs seq_len > 0");
    if (T % seq_len != 0) return fail(SPMLP_ESHAPE, "T=%lld is not a multiple of seq_len=%lld", (long long)T, (long long)seq_len);
  }
  return 0;
}

int check_mk(int64_t T, int K, int N, const char* kname, const char* nname) {
  if (T < 1 || T >= (int64_t(1) << 31)) return fail(SPMLP_ESHAPE, "T=%lld must be in [1, 2^31)", (long long)T);
  if (K < kBK || K % kBK != 0) return fail(SPMLP_ESHAPE, "%s=%d must be a positive multiple of 64", kname, K);
  if (N < kBitsCols || N % kBitsCols != 0) return fail(SPMLP_ESHAPE, "%s=%d must be a positive multiple of 64", nname, N);
  return 0;
}

}  // namespace

// ln_s != nullptr: the folded-LayerNorm form (w_in = W diag(gamma), b_in unused; see GemmParams).
int up_gate_impl(const void* x, const void* w_in, const void* b_in, void* h, uint32_t* bits, void* z_out, int64_t T,
                 int d, int F, int dtype, int gate_op, float kappa, int64_t seq_len, cudaStream_t stream,
                 const float* ln_s = nullptr, const float* ln_c = nullptr, const float* ln_mean = nullptr,
                 const float* ln_rstd = nullptr) {
  int rc;
  if (!x || !w_in || !h || !bits) return fail(SPMLP_EINVAL, "x, w_in, h and tile_bits must be non-null");
  if ((rc = check_dtype(dtype))) return rc;
  if ((rc = check_mk(T, d, F, "d", "F"))) return rc;
  if ((rc = check_gate(gate_op, kappa, T, seq_len))) return rc;
  if (!aligned16(x) || !aligned16(w_in) || !aligned16(h) || (b_in && !aligned16(b_in)) || (z_out && !aligned16(z_out)))
    return fail(SPMLP_EALIGN, "x, w_in, b_in, h and z_out must be 16-byte aligned");
  const bool ln = ln_s != nullptr;
  if (ln) {
    if (!ln_c || !ln_mean || !ln_rstd) return fail(SPMLP_EINVAL, "ln_s, ln_c, row_mean and row_rstd must be non-null");
    if (!aligned16(ln_s) || !aligned16(ln_c)) return fail(SPMLP_EALIGN, "ln_s and ln_c must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(ln_mean) % 4 || reinterpret_cast<uintptr_t>(ln_rstd) % 4)
      return fail(SPMLP_EALIGN, "row_mean and row_rstd must be 4-byte aligned");
  }
  DeviceInfo* dev = nullptr;
  if ((rc = current_device_info(&dev))) return rc;
  const bool bf16 = dtype == SPMLP_BF16;
  // Few tiles: 128 x 128 tiles on single CTAs, so that more SMs share the work and each
  // epilogue warp handles half as many chunks.  Chosen when those tiles fit in one round of
  // the SMs, or when K <= 128 and the 256 x 256 pair tiles would not fill the CTA pairs.
  // Measured (fp16, us per launch, pair / small): T x d x F = 4096x128x512 6.7 / 4.9,
  // 8192x128x512 7.3 / 6.6, 16384x128x512 10.1 / 10.3, 1024x512x2048 8.6 / 7.2,
  // 2048x512x2048 9.4 / 10.7, 4096x512x2048 13.1 / 17.2, 2048x256x1024 7.3 / 5.6.
  const int64_t pair_tiles = ((T + 2 * kBM - 1) / (2 * kBM)) * ((F + kUpBN - 1) / kUpBN);
  const int64_t small_tiles = ((T + kBM - 1) / kBM) * ((F + kUpSmallBN - 1) / kUpSmallBN);
  const bool small = small_tiles <= dev->sm_count || (d <= 128 && pair_tiles * kUpCG <= dev->sm_count);
  const int bn = small ? kUpSmallBN : kUpBN;
  CUtensorMap ta, tb;
  if ((rc = make_kmajor_map(&ta, x, T, d, kBM, bf16))) return rc;
  // B rows per CTA: kUpBN / kUpCG on a pair, kUpSmallBN on one CTA (both 128).
  if ((rc = make_kmajor_map(&tb, w_in, F, d, small ? kUpSmallBN : kUpBN / kUpCG, bf16))) return rc;
  CUtensorMap tc;
  if ((rc = make_out_map(&tc, h, T, F, bf16))) return rc;
  const int words = spmlp_tile_bits_words(F);
  // No clear of tile_bits first: the kernel writes every bit of it, set or clear.
  cudaError_t e;
  GemmParams p{};
  p.M = static_cast<int>(T);
  p.N = F;
  p.K = d;
  p.n_tiles = (F + bn - 1) / bn;
  p.bias = ln ? nullptr : b_in;
  p.ln_s = ln_s;
  p.ln_c = ln_c;
  p.ln_mean = ln_mean;
  p.ln_rstd = ln_rstd;
  p.out = h;
  p.z_out = z_out;
  p.bits_out = bits;
  p.bits_words = words;
  p.gate_op = gate_op;
  p.kappa = kappa;
  p.seq_len = static_cast<int>(seq_len > 0 ? seq_len : T);
  // Corner gate over several sequences whose length is not a multiple of 8: a token
  // block's corner row may belong to another tile, so the up projection writes the
  // ungated z and corner_gate_kernel gates it in place and rebuilds the bitmap.
  const bool corner_pass = gate_op == SPMLP_GATE_CORNER && seq_len != T && seq_len % 8 != 0;
  const int op = corner_pass ? SPMLP_GATE_IDENTITY : gate_op;
  rc = small ? launch_up<kUpSmallBN, true>(ta, tb, tc, p, op, bf16, stream, dev)
             : launch_up<kUpBN, false>(ta, tb, tc, p, op, bf16, stream, dev);
  if (rc || !corner_pass) return rc;
  const int groups = static_cast<int>((T + kBitsRows - 1) / kBitsRows);
  const size_t smem = static_cast<size_t>(words) * 4;
  uint16_t* hz = static_cast<uint16_t*>(h);
  if (bf16)
    corner_gate_kernel<true><<<groups, 256, smem, stream>>>(hz, bits, static_cast<int>(T), F, words,
                                                            static_cast<int>(seq_len), kappa);
  else
    corner_gate_kernel<false><<<groups, 256, smem, stream>>>(hz, bits, static_cast<int>(T), F, words,
                                                             static_cast<int>(seq_len), kappa);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "corner_gate_kernel launch");
  return 0;
}

// slots != nullptr: the d_ff split's scattering mode (see GemmParams::scatter_out);
// y is then unused and bias and residual must be null.
int down_impl(const void* h, const uint32_t* bits, const void* w_out, const void* b_out, const void* residual, void* y,
              int64_t T, int F, int d, int dtype, int mode, uint64_t* stats, cudaStream_t stream,
              void* const* slots = nullptr, int world = 0) {
  int rc;
  if (slots != nullptr) {
    if (world < 1 || world > kMaxRanks) return fail(SPMLP_EINVAL, "world=%d must be in [1, %d]", world, kMaxRanks);
    if (T % world) return fail(SPMLP_ESHAPE, "T=%lld must divide evenly over %d ranks", (long long)T, world);
    if ((T / world) % (kBM * kDownCG))
      return fail(SPMLP_ESHAPE, "tokens per rank (%lld) must be a multiple of %d", (long long)(T / world), kBM * kDownCG);
    for (int j = 0; j < world; ++j)
      if (!slots[j] || !aligned16(slots[j])) return fail(SPMLP_EALIGN, "receive slot %d must be non-null and 16-byte aligned", j);
    y = slots[0];  // the output map is encoded but not stored through in this mode
  }
  if (!h || !w_out || !y) return fail(SPMLP_EINVAL, "h, w_out and y must be non-null");
  if (mode < SPMLP_DOWN_DENSE || mode > SPMLP_DOWN_COMPACT_FINE) return fail(SPMLP_EINVAL, "unknown down mode %d", mode);
  const bool compact = mode == SPMLP_DOWN_COMPACT || mode == SPMLP_DOWN_COMPACT_FINE;
  if (compact && slots != nullptr) return fail(SPMLP_EINVAL, "the scattering down projection takes the 16x64 modes");
  if (mode != SPMLP_DOWN_DENSE && !bits) return fail(SPMLP_EINVAL, "the skipping down modes need tile_bits");
  if ((rc = check_dtype(dtype))) return rc;
  if ((rc = check_mk(T, F, d, "F", "d"))) return rc;
  if (!aligned16(h) || !aligned16(w_out) || !aligned16(y) || (b_out && !aligned16(b_out)) ||
      (residual && !aligned16(residual)))
    return fail(SPMLP_EALIGN, "h, w_out, b_out, residual and y must be 16-byte aligned");
  if (stats && (reinterpret_cast<uintptr_t>(stats) & 7u)) return fail(SPMLP_EALIGN, "stats must be 8-byte aligned");
  DeviceInfo* dev = nullptr;
  if ((rc = current_device_info(&dev))) return rc;
  const bool bf16 = dtype == SPMLP_BF16;
  constexpr int BN = 256, BNF = kDownFineBN;
  const bool fine = mode == SPMLP_DOWN_SKIP_FINE || mode == SPMLP_DOWN_COMPACT_FINE;
  // d <= 128 on CTA pairs (the dense and 256-token skip modes): 128-column tiles, so that no
  // MMA runs on the empty half of a 256-column tile.  Same token tile, same skip accounting.
  const bool narrow = !fine && !compact && slots == nullptr && d <= kDownNarrowBN;
  const int bn = fine ? BNF : (narrow ? kDownNarrowBN : BN);
  const int box_k = compact ? 16 : kBK;  // compact: gathered K16 granules, 32-byte swizzle
  CUtensorMap ta, tb;
  if ((rc = make_kmajor_map(&ta, h, T, F, kBM, bf16, box_k))) return rc;
  const int cg = fine ? 1 : kDownCG;
  if ((rc = make_kmajor_map(&tb, w_out, d, F, bn / cg, bf16, box_k))) return rc;
  CUtensorMap tb_half;  // half-width tail items load bn/2 columns of w_out
  if ((rc = make_kmajor_map(&tb_half, w_out, d, F, bn / 2 / cg, bf16, box_k))) return rc;
  CUtensorMap tc, tr;
  if ((rc = make_out_map(&tc, y, T, d, bf16))) return rc;
  if (residual != nullptr && (rc = make_out_map(&tr, residual, T, d, bf16))) return rc;
  GemmParams p{};
  p.M = static_cast<int>(T);
  p.N = d;
  p.K = F;
  p.n_tiles = (d + bn - 1) / bn;
  p.bias = b_out;
  p.out = y;
  p.residual = residual;
  p.bits_in = bits;
  p.bits_words = compact ? spmlp_tile_bits16_words(F) : spmlp_tile_bits_words(F);
  p.skip = mode == SPMLP_DOWN_DENSE ? 0 : 1;
  p.stats = reinterpret_cast<unsigned long long*>(stats);
  p.split_tail = 1;
  if (slots != nullptr) {
    p.scatter_rows = static_cast<int>(T / world);
    for (int j = 0; j < world; ++j) p.scatter_out[j] = slots[j];
  }
  constexpr int S = kDownStages, E = kDownEpiWarps, C = kDownCG, R = kDownRing;
  constexpr int SF = kDownFineStages, EF = kDownFineEpiWarps, RF = kDownFineRing;
  const CUtensorMap* trp = residual != nullptr ? &tr : nullptr;
  if (compact) {
    if (fine) {
      if (bf16) return launch_gemm<KIND_DOWN, 0, BNF, SF, true, EF, 1, RF, false, true>(ta, tb, tc, p, stream, dev, trp, &ta, &tb, &tb_half);
      return launch_gemm<KIND_DOWN, 0, BNF, SF, false, EF, 1, RF, false, true>(ta, tb, tc, p, stream, dev, trp, &ta, &tb, &tb_half);
    }
    if (bf16) return launch_gemm<KIND_DOWN, 0, BN, S, true, E, C, R, false, true>(ta, tb, tc, p, stream, dev, trp, &ta, &tb, &tb_half);
    return launch_gemm<KIND_DOWN, 0, BN, S, false, E, C, R, false, true>(ta, tb, tc, p, stream, dev, trp, &ta, &tb, &tb_half);
  }
  if (fine) {
    if (bf16) return launch_gemm<KIND_DOWN, 0, BNF, SF, true, EF, 1, RF>(ta, tb, tc, p, stream, dev, trp, &ta, &tb, &tb_half);
    return launch_gemm<KIND_DOWN, 0, BNF, SF, false, EF, 1, RF>(ta, tb, tc, p, stream, dev, trp, &ta, &tb, &tb_half);
  }
  if (narrow) {
    constexpr int BNN = kDownNarrowBN, SN = kDownNarrowStages, EN = kDownNarrowEpiWarps;
    if (bf16) return launch_gemm<KIND_DOWN, 0, BNN, SN, true, EN, C, R>(ta, tb, tc, p, stream, dev, trp, &ta, &tb, &tb_half);
    return launch_gemm<KIND_DOWN, 0, BNN, SN, false, EN, C, R>(ta, tb, tc, p, stream, dev, trp, &ta, &tb, &tb_half);
  }
  if (bf16) return launch_gemm<KIND_DOWN, 0, BN, S, true, E, C, R>(ta, tb, tc, p, stream, dev, trp, &ta, &tb, &tb_half);
  return launch_gemm<KIND_DOWN, 0, BN, S, false, E, C, R>(ta, tb, tc, p, stream, dev, trp, &ta, &tb, &tb_half);
}

int joint_impl(const void* h, const uint32_t* bits, const void* z, const void* w2, const void* b2, const void* wo,
               const void* bo, const void* residual, void* out, int64_t T, int F, int d, int dtype, int mode,
               uint64_t* stats, cudaStream_t stream) {
  int rc;
  if (!h || !z || !w2 || !wo || !out) return fail(SPMLP_EINVAL, "h, z, w2, wo and out must be non-null");
  if (mode != SPMLP_DOWN_DENSE && mode != SPMLP_DOWN_SKIP && mode != SPMLP_DOWN_SKIP_FINE)
    return fail(SPMLP_EINVAL, "unknown joint mode %d", mode);
  if (mode != SPMLP_DOWN_DENSE && !bits) return fail(SPMLP_EINVAL, "the skipping joint modes need tile_bits");
  if ((rc = check_dtype(dtype))) return rc;
  if ((rc = check_mk(T, F, d, "F", "d"))) return rc;
  if (!aligned16(h) || !aligned16(z) || !aligned16(w2) || !aligned16(wo) || !aligned16(out) ||
      (b2 && !aligned16(b2)) || (bo && !aligned16(bo)) || (residual && !aligned16(residual)))
    return fail(SPMLP_EALIGN, "h, z, w2, b2, wo, bo, residual and out must be 16-byte aligned");
  if (stats && (reinterpret_cast<uintptr_t>(stats) & 7u)) return fail(SPMLP_EALIGN, "stats must be 8-byte aligned");
  DeviceInfo* dev = nullptr;
  if ((rc = current_device_info(&dev))) return rc;
  const bool bf16 = dtype == SPMLP_BF16;
  constexpr int BN = kJointBN;
  const int cg = mode == SPMLP_DOWN_SKIP_FINE ? 1 : 2;
  CUtensorMap ta, tb, ta2, tb2, tc, tr, tb_half, tb2_half;
  if ((rc = make_kmajor_map(&ta, h, T, F, kBM, bf16))) return rc;
  if ((rc = make_kmajor_map(&tb, w2, d, F, BN / cg, bf16))) return rc;
  if ((rc = make_kmajor_map(&ta2, z, T, d, kBM, bf16))) return rc;
  if ((rc = make_kmajor_map(&tb2, wo, d, d, BN / cg, bf16))) return rc;
  // half-width tail items (the last round of the persistent grid) load half of each B
  if ((rc = make_kmajor_map(&tb_half, w2, d, F, BN / 2 / cg, bf16))) return rc;
  if ((rc = make_kmajor_map(&tb2_half, wo, d, d, BN / 2 / cg, bf16))) return rc;
  if ((rc = make_out_map(&tc, out, T, d, bf16))) return rc;
  if (residual != nullptr && (rc = make_out_map(&tr, residual, T, d, bf16))) return rc;
  GemmParams p{};
  p.M = static_cast<int>(T);
  p.N = d;
  p.K = F;
  p.K2 = d;
  p.n_tiles = (d + BN - 1) / BN;
  p.bias = b2;
  p.bias2 = bo;
  p.out = out;
  p.residual = residual;
  p.bits_in = bits;
  p.bits_words = spmlp_tile_bits_words(F);
  p.skip = mode == SPMLP_DOWN_DENSE ? 0 : 1;
  p.stats = reinterpret_cast<unsigned long long*>(stats);
  p.split_tail = 1;
  constexpr int R = kJointRing;
  const CUtensorMap* trp = residual != nullptr ? &tr : nullptr;
  if (mode == SPMLP_DOWN_SKIP_FINE) {
    constexpr int S = kJointFineStages, E = kJointFineEpiWarps;
    if (bf16) return launch_gemm<KIND_JOINT, 0, BN, S, true, E, 1, R>(ta, tb, tc, p, stream, dev, trp, &ta2, &tb2, &tb_half, &tb2_half);
    return launch_gemm<KIND_JOINT, 0, BN, S, false, E, 1, R>(ta, tb, tc, p, stream, dev, trp, &ta2, &tb2, &tb_half, &tb2_half);
  }
  constexpr int S = kJointStages, E = kJointEpiWarps;
  if (bf16) return launch_gemm<KIND_JOINT, 0, BN, S, true, E, 2, R>(ta, tb, tc, p, stream, dev, trp, &ta2, &tb2, &tb_half, &tb2_half);
  return launch_gemm<KIND_JOINT, 0, BN, S, false, E, 2, R>(ta, tb, tc, p, stream, dev, trp, &ta2, &tb2, &tb_half, &tb2_half);
}

// A bounded wait on an mbarrier that nothing arrives on: the same wait helper every
// kernel uses gives up after SPMLP_WAIT_NS, records kDevTimeoutProbe in the status
// word and the kernel returns normally.
__global__ void wait_probe_kernel(int* status) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) (void)mbar_wait(&bar, 0, status, status_base(status), kDevTimeoutProbe);
}

int row_stats_impl(const void* x, float* mean, float* rstd, int64_t T, int d, int dtype, float eps,
                   cudaStream_t stream) {
  int rc;
  if (!x || !mean || !rstd) return fail(SPMLP_EINVAL, "x, mean and rstd must be non-null");
  if ((rc = check_dtype(dtype))) return rc;
  if (T < 1 || T >= (int64_t(1) << 31)) return fail(SPMLP_ESHAPE, "T must be in [1, 2^31)");
  if (d < kBK || d % kBK) return fail(SPMLP_ESHAPE, "d=%d must be a positive multiple of 64", d);
  if (!std::isfinite(eps) || eps <= 0.f) return fail(SPMLP_EINVAL, "eps must be a finite positive number");
  if (!aligned16(x)) return fail(SPMLP_EALIGN, "x must be 16-byte aligned");
  DeviceInfo* dev = nullptr;
  if ((rc = current_device_info(&dev))) return rc;
  const int blocks = static_cast<int>((T + 7) / 8);  // eight tokens (warps) per 256-thread block
  const uint16_t* xs = static_cast<const uint16_t*>(x);
  if (dtype == SPMLP_BF16)
    row_stats_kernel<true><<<blocks, 256, 0, stream>>>(xs, mean, rstd, static_cast<int>(T), d, eps);
  else
    row_stats_kernel<false><<<blocks, 256, 0, stream>>>(xs, mean, rstd, static_cast<int>(T), d, eps);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "row_stats_kernel launch");
  return 0;
}

int multicast_reduce_broadcast_impl(const void* mc_part, void* mc_x, const void* residual, int64_t rows, int d,
                                    const void* b_out, int dtype, cudaStream_t stream) {
  int rc;
  if (!mc_part || !mc_x) return fail(SPMLP_EINVAL, "mc_part and mc_x must be non-null multicast addresses");
  if ((rc = check_dtype(dtype))) return rc;
  if (rows < 1 || rows >= (int64_t(1) << 31)) return fail(SPMLP_ESHAPE, "rows must be in [1, 2^31)");
  if (d < kBitsCols || d % kBitsCols) return fail(SPMLP_ESHAPE, "d=%d must be a positive multiple of 64", d);
  if (!aligned16(mc_part) || !aligned16(mc_x) || (b_out && !aligned16(b_out)) || (residual && !aligned16(residual)))
    return fail(SPMLP_EALIGN, "mc_part, mc_x, b_out and residual must be 16-byte aligned");
  DeviceInfo* dev = nullptr;
  if ((rc = current_device_info(&dev))) return rc;
  const int64_t elems = rows * d;
  const int64_t vecs = elems / 8;
  const int blocks = static_cast<int>(std::min<int64_t>((vecs + 255) / 256, int64_t(dev->sm_count) * 8));
  const uint16_t* pv = static_cast<const uint16_t*>(mc_part);
  uint16_t* xv = static_cast<uint16_t*>(mc_x);
  const uint16_t* bv = static_cast<const uint16_t*>(b_out);
  const uint16_t* resv = static_cast<const uint16_t*>(residual);
  if (dtype == SPMLP_BF16)
    multicast_reduce_broadcast_kernel<true><<<blocks, 256, 0, stream>>>(pv, xv, elems, d, bv, resv);
  else
    multicast_reduce_broadcast_kernel<false><<<blocks, 256, 0, stream>>>(pv, xv, elems, d, bv, resv);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "multicast_reduce_broadcast_kernel launch");
  return 0;
}

int reduce_broadcast_impl(const void* recv, int world, int64_t rows, int d, const void* b_out, const void* residual,
                          void* const* targets, int n_targets, int dtype, cudaStream_t stream) {
  int rc;
  if (!recv || !targets) return fail(SPMLP_EINVAL, "recv and targets must be non-null");
  if ((rc = check_dtype(dtype))) return rc;
  if (world < 1 || world > kMaxRanks) return fail(SPMLP_EINVAL, "world=%d must be in [1, %d]", world, kMaxRanks);
  if (n_targets < 1 || n_targets > kMaxRanks)
    return fail(SPMLP_EINVAL, "n_targets=%d must be in [1, %d]", n_targets, kMaxRanks);
  if (rows < 1 || rows >= (int64_t(1) << 31)) return fail(SPMLP_ESHAPE, "rows must be in [1, 2^31)");
  if (d < kBitsCols || d % kBitsCols) return fail(SPMLP_ESHAPE, "d=%d must be a positive multiple of 64", d);
  if (!aligned16(recv) || (b_out && !aligned16(b_out)) || (residual && !aligned16(residual)))
    return fail(SPMLP_EALIGN, "recv, b_out and residual must be 16-byte aligned");
  BroadcastTargets tg{};
  tg.n = n_targets;
  for (int k = 0; k < n_targets; ++k) {
    if (!targets[k] || !aligned16(targets[k])) return fail(SPMLP_EALIGN, "target %d must be non-null and 16-byte aligned", k);
    tg.dst[k] = targets[k];
  }
  DeviceInfo* dev = nullptr;
  if ((rc = current_device_info(&dev))) return rc;
  const int64_t elems = rows * d;
  const int64_t vecs = elems / 8;
  const int blocks = static_cast<int>(std::min<int64_t>((vecs + 255) / 256, int64_t(dev->sm_count) * 8));
  const uint16_t* rv = static_cast<const uint16_t*>(recv);
  const uint16_t* bv = static_cast<const uint16_t*>(b_out);
  const uint16_t* resv = static_cast<const uint16_t*>(residual);
  if (dtype == SPMLP_BF16)
    reduce_broadcast_kernel<true><<<blocks, 256, 0, stream>>>(rv, world, elems, d, bv, resv, tg);
  else
    reduce_broadcast_kernel<false><<<blocks, 256, 0, stream>>>(rv, world, elems, d, bv, resv, tg);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "reduce_broadcast_kernel launch");
  return 0;
}

int gate_impl(const void* x, void* out, uint32_t* bits, int64_t T, int F, int dtype, int gate_op, float kappa,
              cudaStream_t stream) {
  int rc;
  if (!x || !out) return fail(SPMLP_EINVAL, "x and out must be non-null");
  if ((rc = check_dtype(dtype))) return rc;
  if (gate_op != SPMLP_GATE_IDENTITY && gate_op != SPMLP_GATE_ONE_SIDED && gate_op != SPMLP_GATE_SYMMETRIC &&
      gate_op != SPMLP_GATE_RELU)
    return fail(SPMLP_EINVAL, "spmlp_gate takes the identity, one-sided, symmetric or ReLU gate (got %d)", gate_op);
  if (!std::isfinite(kappa) || kappa < 0.f) return fail(SPMLP_EINVAL, "kappa must be a finite nonnegative number");
  if (T < 1 || T >= (int64_t(1) << 31)) return fail(SPMLP_ESHAPE, "T must be in [1, 2^31)");
  if (F < kBitsCols || F % kBitsCols) return fail(SPMLP_ESHAPE, "F=%d must be a positive multiple of 64", F);
  if (!aligned16(x) || !aligned16(out)) return fail(SPMLP_EALIGN, "x and out must be 16-byte aligned");
  if (x != out) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(x), b = reinterpret_cast<uintptr_t>(out);
    const uintptr_t n = static_cast<uintptr_t>(T) * F * 2;
    if (a < b + n && b < a + n) return fail(SPMLP_EINVAL, "x and out must be the same buffer or not overlap");
  }
  DeviceInfo* dev = nullptr;
  if ((rc = current_device_info(&dev))) return rc;
  const int words = spmlp_tile_bits_words(F);
  const int groups = static_cast<int>((T + kBitsRows - 1) / kBitsRows);
  const size_t smem = bits != nullptr ? static_cast<size_t>(words) * 4 : 0;
  const uint16_t* xs = static_cast<const uint16_t*>(x);
  uint16_t* os = static_cast<uint16_t*>(out);
  if (dtype == SPMLP_BF16)
    gate_bits_kernel<true><<<groups, 256, smem, stream>>>(xs, os, bits, static_cast<int>(T), F, words, gate_op, kappa);
  else
    gate_bits_kernel<false><<<groups, 256, smem, stream>>>(xs, os, bits, static_cast<int>(T), F, words, gate_op, kappa);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "gate_bits_kernel launch");
  return 0;
}

int tile_bits_impl(const void* h, uint32_t* bits, int64_t T, int F, int dtype, cudaStream_t stream) {
  int rc;
  if (!h || !bits) return fail(SPMLP_EINVAL, "h and tile_bits must be non-null");
  if ((rc = check_dtype(dtype))) return rc;
  if (T < 1 || T >= (int64_t(1) << 31)) return fail(SPMLP_ESHAPE, "T must be in [1, 2^31)");
  if (F < kBitsCols || F % kBitsCols) return fail(SPMLP_ESHAPE, "F=%d must be a positive multiple of 64", F);
  if (!aligned16(h)) return fail(SPMLP_EALIGN, "h must be 16-byte aligned");
  DeviceInfo* dev = nullptr;
  if ((rc = current_device_info(&dev))) return rc;
  const int words = spmlp_tile_bits_words(F);
  const int groups = static_cast<int>((T + kBitsRows - 1) / kBitsRows);
  tile_bits_kernel<<<groups, 256, static_cast<size_t>(words) * 4, stream>>>(static_cast<const uint16_t*>(h), bits,
                                                                            static_cast<int>(T), F, words);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "tile_bits_kernel launch");
  return 0;
}

int tile_bits16_impl(const void* h, uint32_t* bits, int64_t T, int F, cudaStream_t stream) {
  int rc;
  if (!h || !bits) return fail(SPMLP_EINVAL, "h and tile_bits16 must be non-null");
  if (T < 1 || T >= (int64_t(1) << 31)) return fail(SPMLP_ESHAPE, "T must be in [1, 2^31)");
  if (F < kBitsCols || F % kBitsCols) return fail(SPMLP_ESHAPE, "F=%d must be a positive multiple of 64", F);
  if (!aligned16(h)) return fail(SPMLP_EALIGN, "h must be 16-byte aligned");
  DeviceInfo* dev = nullptr;
  if ((rc = current_device_info(&dev))) return rc;
  const int words = spmlp_tile_bits16_words(F);
  const int groups = static_cast<int>((T + kBitsRows - 1) / kBitsRows);
  tile_bits16_kernel<<<groups, 256, static_cast<size_t>(words) * 4, stream>>>(static_cast<const uint16_t*>(h), bits,
                                                                              static_cast<int>(T), F, words);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "tile_bits16_kernel launch");
  return 0;
}

int head_prepare_impl(const float* x, void* x_out, uint32_t* support, int64_t T, int d, int dtype, float kappa,
                      cudaStream_t stream) {
  int rc;
  if (!x || !x_out || !support) return fail(SPMLP_EINVAL, "x, x_out and support must be non-null");
  if ((rc = check_dtype(dtype))) return rc;
  if (T < 1 || T >= (int64_t(1) << 31)) return fail(SPMLP_ESHAPE, "T must be in [1, 2^31)");
  if (d < kBK || d % kBK) return fail(SPMLP_ESHAPE, "d=%d must be a positive multiple of 64", d);
  if (!std::isfinite(kappa) || kappa < 0.f) return fail(SPMLP_EINVAL, "kappa must be a finite nonnegative number");
  if (!aligned16(x) || !aligned16(x_out)) return fail(SPMLP_EALIGN, "x and x_out must be 16-byte aligned");
  DeviceInfo* dev = nullptr;
  if ((rc = current_device_info(&dev))) return rc;
  const int words = spmlp_head_support_words(d);
  const int groups = static_cast<int>((T + 15) / 16);
  const size_t smem = static_cast<size_t>(words) * 4;
  if (dtype == SPMLP_BF16)
    head_prepare_kernel<true><<<groups, 256, smem, stream>>>(x, static_cast<uint16_t*>(x_out), support,
                                                             static_cast<int>(T), d, words, kappa);
  else
    head_prepare_kernel<false><<<groups, 256, smem, stream>>>(x, static_cast<uint16_t*>(x_out), support,
                                                              static_cast<int>(T), d, words, kappa);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "head_prepare_kernel launch");
  return 0;
}

int head_impl(const void* x, const uint32_t* support, const void* w, void* logits, const int32_t* active,
              int n_active, int64_t T, int d, int V, int dtype, int gate_axis, uint64_t* stats,
              cudaStream_t stream) {
  int rc;
  if (!x || !w || !logits) return fail(SPMLP_EINVAL, "x, w_vocab and logits must be non-null");
  if ((rc = check_dtype(dtype))) return rc;
  if ((rc = check_mk(T, d, V, "d", "V"))) return rc;
  if (V % 128 != 0) return fail(SPMLP_ESHAPE, "V=%d must be a multiple of 128", V);
  if (gate_axis < SPMLP_HEAD_DENSE || gate_axis > SPMLP_HEAD_GATE_N)
    return fail(SPMLP_EINVAL, "unknown gate_axis %d", gate_axis);
  if (gate_axis == SPMLP_HEAD_GATE_K && !support) return fail(SPMLP_EINVAL, "SPMLP_HEAD_GATE_K needs support bits");
  if (gate_axis == SPMLP_HEAD_GATE_N && (n_active < 0 || (n_active > 0 && !active)))
    return fail(SPMLP_EINVAL, "SPMLP_HEAD_GATE_N needs a device list of n_active >= 0 tiles");
  if (gate_axis == SPMLP_HEAD_GATE_N && n_active > V / 128)
    return fail(SPMLP_EINVAL, "n_active=%d exceeds the %d vocabulary tiles", n_active, V / 128);
  if (!aligned16(x) || !aligned16(w) || !aligned16(logits)) return fail(SPMLP_EALIGN, "x, w_vocab and logits must be 16-byte aligned");
  if (stats && (reinterpret_cast<uintptr_t>(stats) & 7u)) return fail(SPMLP_EALIGN, "stats must be 8-byte aligned");
  DeviceInfo* dev = nullptr;
  if ((rc = current_device_info(&dev))) return rc;
  const bool bf16 = dtype == SPMLP_BF16;
  constexpr int BN = 128;
  // Every form runs two vocabulary tiles per work item.  The dense and N-gated heads
  // with d >= kHeadPairMinD do so on a CTA pair (each CTA loads one tile of w_vocab,
  // 128 rows), which halves the operand traffic per MMA.  Below it, and for the
  // K-gated head at any d (it skips K16 groups dead for its 128 tokens, a granule a
  // pair would double), one CTA loads both tiles stacked in the stage: one 256-column
  // item halves the epilogue's per-item cost where the logit stores bound the head.
  const bool pairs = gate_axis != SPMLP_HEAD_GATE_K && d >= kHeadPairMinD;
  CUtensorMap ta, tb, tb_half;
  if ((rc = make_kmajor_map(&ta, x, T, d, kBM, bf16))) return rc;
  if ((rc = make_kmajor_map(&tb, w, V, d, BN, bf16))) return rc;
  if ((rc = make_kmajor_map(&tb_half, w, V, d, BN / 2, bf16))) return rc;  // a lone tile split over the pair
  CUtensorMap tc;
  if ((rc = make_out_map(&tc, logits, T, V, bf16))) return rc;
  GemmParams p{};
  p.M = static_cast<int>(T);
  p.N = V;
  p.K = d;
  p.n_tiles = gate_axis == SPMLP_HEAD_GATE_N ? n_active : V / BN;
  p.out = logits;
  p.col_tiles = gate_axis == SPMLP_HEAD_GATE_N ? active : nullptr;
  p.bits_in = gate_axis == SPMLP_HEAD_GATE_K ? support : nullptr;
  p.bits_words = spmlp_head_support_words(d);
  p.skip = gate_axis == SPMLP_HEAD_GATE_K ? 1 : 0;
  p.stats = reinterpret_cast<unsigned long long*>(stats);
  // Eight epilogue warps (two 32-column chunks each) and a two-slot output ring:
  // the logit stores, not the MMAs, bound the head at d = 128.
  if (kHeadWide && !pairs) {
    constexpr int SW = kHeadWideStages, EW = kHeadWideEpiWarps, RW = kHeadWideRing;
    if (bf16) return launch_gemm<KIND_HEAD, 0, 2 * BN, SW, true, EW, 1, RW>(ta, tb, tc, p, stream, dev, nullptr, &ta, &tb);
    return launch_gemm<KIND_HEAD, 0, 2 * BN, SW, false, EW, 1, RW>(ta, tb, tc, p, stream, dev, nullptr, &ta, &tb);
  }
  if (pairs) {
    constexpr int SP = kHeadPairStages, EP = kHeadPairEpiWarps, RP = kHeadPairRing;
    if (bf16) return launch_gemm<KIND_HEAD, 0, 2 * BN, SP, true, EP, 2, RP>(ta, tb, tc, p, stream, dev, nullptr, &ta, &tb, &tb_half);
    return launch_gemm<KIND_HEAD, 0, 2 * BN, SP, false, EP, 2, RP>(ta, tb, tc, p, stream, dev, nullptr, &ta, &tb, &tb_half);
  }
  constexpr int S = kHeadStages, E = kHeadEpiWarps, R = kHeadRing;
  if (bf16) return launch_gemm<KIND_HEAD, 0, BN, S, true, E, 1, R>(ta, tb, tc, p, stream, dev);
  return launch_gemm<KIND_HEAD, 0, BN, S, false, E, 1, R>(ta, tb, tc, p, stream, dev);
}

int head_fill_impl(void* logits, const int32_t* tiles, int n_tiles, int64_t T, int V, int dtype, float value,
                   cudaStream_t stream) {
  int rc;
  if (!logits || (n_tiles > 0 && !tiles)) return fail(SPMLP_EINVAL, "logits and tiles must be non-null");
  if ((rc = check_dtype(dtype))) return rc;
  if (T < 1 || T >= (int64_t(1) << 31)) return fail(SPMLP_ESHAPE, "T must be in [1, 2^31)");
  if (V < 128 || V % 128) return fail(SPMLP_ESHAPE, "V=%d must be a positive multiple of 128", V);
  if (n_tiles < 0 || n_tiles > V / 128) return fail(SPMLP_EINVAL, "n_tiles=%d out of range", n_tiles);
  if (!aligned16(logits)) return fail(SPMLP_EALIGN, "logits must be 16-byte aligned");
  if (n_tiles == 0) return 0;
  DeviceInfo* dev = nullptr;
  if ((rc = current_device_info(&dev))) return rc;
  uint16_t bits;
  if (dtype == SPMLP_BF16) {
    __nv_bfloat16 b = __float2bfloat16_rn(value);
    std::memcpy(&bits, &b, 2);
  } else {
    __half hv = __float2half_rn(value);
    std::memcpy(&bits, &hv, 2);
  }
  const int row_blocks = static_cast<int>(std::min<int64_t>((T + 15) / 16, 4096));
  dim3 grid(row_blocks, n_tiles);
  head_fill_kernel<<<grid, 256, 0, stream>>>(static_cast<uint16_t*>(logits), tiles, n_tiles, static_cast<int>(T), V,
                                             bits);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "head_fill_kernel launch");
  return 0;
}

// ------------------------------------------------------------ allocation-free MLP forward
// Workspace of spmlp_mlp_forward_noalloc: h [T, F] (256-byte aligned) followed by
// the tile bitmap.  A file-scope device array, so the library never calls
// cudaMalloc for it: the CUDA runtime reserves it on every device where this
// module is loaded, and it stays reserved until the process exits.
constexpr size_t kNoAllocScratchBytes = SPMLP_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[64] = {};
void* g_noalloc_ctx[64] = {};

// Device address of g_noalloc_scratch on the current device.  The host-side
// symbol is only a stand-in, never a device address; the real address is looked
// up (cudaGetSymbolAddress, with that device current) once per device and
// context, and looked up again when the context changes (after a device reset
// the runtime loads this module again, at a new address).
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(SPMLP_EDEVICE, "device index %d out of range", dev);
  void* ctx = current_context();
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_ptr[dev] == nullptr || ctx == nullptr || g_noalloc_ctx[dev] != ctx) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
    g_noalloc_ptr[dev] = ptr;
    g_noalloc_ctx[dev] = current_context();
  }
  *out = g_noalloc_ptr[dev];
  return 0;
}

int mlp_forward_noalloc_impl(const void* x, const void* w_in, const void* b_in, const void* w_out, const void* b_out,
                             const void* residual, void* y, int64_t T, int d, int F, int dtype, int gate_op,
                             float kappa, int64_t seq_len, int mode, uint64_t* stats, cudaStream_t stream) {
  if (T < 1 || T >= (int64_t(1) << 31)) return fail(SPMLP_ESHAPE, "T=%lld must be in [1, 2^31)", (long long)T);
  if (F < kBitsCols || F % kBitsCols != 0) return fail(SPMLP_ESHAPE, "F=%d must be a positive multiple of 64", F);
  const size_t h_bytes = ((static_cast<size_t>(T) * static_cast<size_t>(F) * 2) + 255) & ~size_t(255);
  const size_t bits_bytes = static_cast<size_t>(spmlp_tile_bits_size(T, F)) * 4;
  if (h_bytes + bits_bytes > kNoAllocScratchBytes)
    return fail(SPMLP_ESHAPE,
                "spmlp_mlp_forward_noalloc: T=%lld x F=%d needs %zu bytes of workspace but the static buffer "
                "holds %zu; split the tokens into smaller calls or use spmlp_mlp_forward",
                (long long)T, F, h_bytes + bits_bytes, kNoAllocScratchBytes);
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  void* h = scratch;
  uint32_t* bits = reinterpret_cast<uint32_t*>(static_cast<unsigned char*>(scratch) + h_bytes);
  // up_gate writes every bit of the bitmap, set or clear, so nothing the previous
  // call left in the buffer is read.
  rc = up_gate_impl(x, w_in, b_in, h, bits, nullptr, T, d, F, dtype, gate_op, kappa, seq_len, stream);
  if (rc) return rc;
  return down_impl(h, bits, w_out, b_out, residual, y, T, F, d, dtype, mode, stats, stream);
}

}  // namespace spmlp

using namespace spmlp;

extern "C" {

int spmlp_version(void) { return 100; }

int spmlp_down_tile_tokens(int mode) {
  return (mode == SPMLP_DOWN_SKIP_FINE || mode == SPMLP_DOWN_COMPACT_FINE) ? kBM : kBM * kDownCG;
}

const char* spmlp_last_error(void) { return g_last_error.c_str(); }

int spmlp_tile_bits_words(int F) {
  if (F <= 0) return 0;
  const int groups = (F + kBitsCols - 1) / kBitsCols;
  return (groups + 31) / 32;
}

int64_t spmlp_tile_bits_size(int64_t T, int F) {
  if (T <= 0 || F <= 0) return 0;
  return ((T + kBitsRows - 1) / kBitsRows) * static_cast<int64_t>(spmlp_tile_bits_words(F));
}

static int check_mask_geometry(int64_t T, int F, int encoding) {
  if (T < 1 || T >= (int64_t(1) << 40)) return fail(SPMLP_ESHAPE, "T=%lld must be in [1, 2^40)", (long long)T);
  if (F < kBitsCols || F % kBitsCols || F / kBitsCols > 65536)
    return fail(SPMLP_ESHAPE, "F=%d must be a positive multiple of 64 with at most 65536 tiles", F);
  if (encoding != SPMLP_MASK_RAW && encoding != SPMLP_MASK_ROW_RUNS)
    return fail(SPMLP_EINVAL, "unknown mask encoding %d", encoding);
  return 0;
}

int64_t spmlp_mask_encoded_size(const uint32_t* tile_bits, int64_t T, int F, int encoding) {
  int rc;
  if (!tile_bits) return fail(SPMLP_EINVAL, "tile_bits must be non-null");
  if ((rc = check_mask_geometry(T, F, encoding))) return rc;
  return mask::kHeaderBytes + mask::payload_bytes(tile_bits, T, spmlp_tile_bits_words(F), encoding);
}

int64_t spmlp_mask_encode(const uint32_t* tile_bits, int64_t T, int F, int encoding, void* out, int64_t capacity) {
  const int64_t size = spmlp_mask_encoded_size(tile_bits, T, F, encoding);
  if (size < 0) return size;
  if (!out) return fail(SPMLP_EINVAL, "out must be non-null");
  if (capacity < size) return fail(SPMLP_ESHAPE, "out holds %lld bytes, %lld needed", (long long)capacity, (long long)size);
  const int words = spmlp_tile_bits_words(F);
  uint8_t* o = static_cast<uint8_t*>(out);
  uint8_t* payload = o + mask::kHeaderBytes;
  mask::write_payload(tile_bits, T, words, encoding, payload);
  const int64_t pbytes = size - mask::kHeaderBytes;
  std::memset(o, 0, mask::kHeaderBytes);
  mask::put<uint32_t>(o + 0, mask::kMagic);
  mask::put<uint16_t>(o + 4, mask::kVersion);
  mask::put<uint16_t>(o + 6, static_cast<uint16_t>(encoding));
  mask::put<uint16_t>(o + 8, static_cast<uint16_t>(kBitsRows));
  mask::put<uint16_t>(o + 10, static_cast<uint16_t>(kBitsCols));
  mask::put<uint32_t>(o + 12, static_cast<uint32_t>(F));
  mask::put<uint64_t>(o + 16, static_cast<uint64_t>(T));
  mask::put<uint32_t>(o + 24, static_cast<uint32_t>(words));
  mask::put<uint32_t>(o + 28, mask::crc32(payload, static_cast<size_t>(pbytes)));
  mask::put<uint64_t>(o + 32, static_cast<uint64_t>(pbytes));
  mask::put<uint64_t>(o + 40, static_cast<uint64_t>(mask::popcount_all(tile_bits, mask::groups_of(T) * words)));
  return size;
}

int spmlp_mask_decode_header(const void* data, int64_t n, int64_t* T, int* F, int* encoding) {
  if (!data) return fail(SPMLP_EINVAL, "data must be non-null");
  const uint8_t* b = static_cast<const uint8_t*>(data);
  if (n < mask::kHeaderBytes || mask::get<uint32_t>(b) != mask::kMagic)
    return fail(SPMLP_EFORMAT, "not a serialized tile bitmap (bad magic or short header)");
  if (mask::get<uint16_t>(b + 4) != mask::kVersion)
    return fail(SPMLP_EFORMAT, "unsupported mask format version %u", unsigned(mask::get<uint16_t>(b + 4)));
  if (mask::get<uint16_t>(b + 8) != kBitsRows || mask::get<uint16_t>(b + 10) != kBitsCols)
    return fail(SPMLP_EFORMAT, "mask tiles are %ux%u, this library uses %dx%d", unsigned(mask::get<uint16_t>(b + 8)),
                unsigned(mask::get<uint16_t>(b + 10)), kBitsRows, kBitsCols);
  const int enc = mask::get<uint16_t>(b + 6);
  const int64_t t = static_cast<int64_t>(mask::get<uint64_t>(b + 16));
  const uint32_t f = mask::get<uint32_t>(b + 12);
  if (f > 0x7fffffffu || check_mask_geometry(t, static_cast<int>(f), enc))
    return fail(SPMLP_EFORMAT, "mask header holds an invalid shape or encoding");
  if (static_cast<int>(mask::get<uint32_t>(b + 24)) != spmlp_tile_bits_words(static_cast<int>(f)))
    return fail(SPMLP_EFORMAT, "mask header word count does not match F");
  const uint64_t pbytes = mask::get<uint64_t>(b + 32);
  if (pbytes > static_cast<uint64_t>(n - mask::kHeaderBytes)) return fail(SPMLP_EFORMAT, "mask payload is truncated");
  if (T) *T = t;
  if (F) *F = static_cast<int>(f);
  if (encoding) *encoding = enc;
  return 0;
}

int spmlp_mask_decode(const void* data, int64_t n, uint32_t* tile_bits, int64_t capacity_words) {
  int64_t T = 0;
  int F = 0, enc = 0;
  int rc = spmlp_mask_decode_header(data, n, &T, &F, &enc);
  if (rc) return rc;
  if (!tile_bits) return fail(SPMLP_EINVAL, "tile_bits must be non-null");
  const uint8_t* b = static_cast<const uint8_t*>(data);
  const uint8_t* payload = b + mask::kHeaderBytes;
  const int64_t pbytes = static_cast<int64_t>(mask::get<uint64_t>(b + 32));
  if (mask::crc32(payload, static_cast<size_t>(pbytes)) != mask::get<uint32_t>(b + 28))
    return fail(SPMLP_EFORMAT, "mask payload checksum mismatch");
  const int words = spmlp_tile_bits_words(F);
  const int64_t groups = mask::groups_of(T);
  if (capacity_words < groups * words)
    return fail(SPMLP_ESHAPE, "tile_bits holds %lld words, %lld needed", (long long)capacity_words,
                (long long)(groups * words));
  if (enc == SPMLP_MASK_RAW) {
    if (pbytes != groups * words * 4) return fail(SPMLP_EFORMAT, "raw mask payload has the wrong size");
    std::memcpy(tile_bits, payload, static_cast<size_t>(pbytes));
  } else {
    if (pbytes < 4) return fail(SPMLP_EFORMAT, "row-run mask payload is truncated");
    const int64_t runs = mask::get<uint32_t>(payload);
    if (4 + runs * (1 + words) * 4 != pbytes) return fail(SPMLP_EFORMAT, "row-run mask payload has the wrong size");
    const uint8_t* o = payload + 4;
    int64_t r = 0;
    for (int64_t i = 0; i < runs; ++i, o += (1 + words) * 4) {
      const int64_t len = mask::get<uint32_t>(o);
      if (len < 1 || len > groups - r) return fail(SPMLP_EFORMAT, "row runs do not cover the token groups");
      for (int64_t k = 0; k < len; ++k, ++r) std::memcpy(tile_bits + r * words, o + 4, static_cast<size_t>(words) * 4);
    }
    if (r != groups) return fail(SPMLP_EFORMAT, "row runs do not cover the token groups");
  }
  // Bits past the last 64-feature tile of a group must be clear.
  const int tiles = F / kBitsCols;
  if (tiles % 32) {
    const uint32_t spare = ~((1u << (tiles % 32)) - 1u);
    for (int64_t r = 0; r < groups; ++r)
      if (tile_bits[r * words + words - 1] & spare) return fail(SPMLP_EFORMAT, "mask sets bits past the last tile");
  }
  return 0;
}

int spmlp_tile_bits_from_h(const void* h, uint32_t* tile_bits, int64_t T, int F, int dtype, void* stream) {
  return tile_bits_impl(h, tile_bits, T, F, dtype, static_cast<cudaStream_t>(stream));
}

int spmlp_tile_bits16_words(int F) {
  if (F <= 0) return 0;
  return (F / 16 + 31) / 32;
}

int64_t spmlp_tile_bits16_size(int64_t T, int F) {
  if (T <= 0 || F <= 0) return 0;
  return ((T + kBitsRows - 1) / kBitsRows) * static_cast<int64_t>(spmlp_tile_bits16_words(F));
}

int spmlp_tile_bits16_from_h(const void* h, uint32_t* tile_bits16, int64_t T, int F, void* stream) {
  return tile_bits16_impl(h, tile_bits16, T, F, static_cast<cudaStream_t>(stream));
}

int spmlp_up_gate(const void* x, const void* w_in, const void* b_in, void* h, uint32_t* tile_bits, void* z_out,
                  int64_t T, int d, int F, int dtype, int gate_op, float kappa, int64_t seq_len, void* stream) {
  return up_gate_impl(x, w_in, b_in, h, tile_bits, z_out, T, d, F, dtype, gate_op, kappa, seq_len,
                      static_cast<cudaStream_t>(stream));
}

int spmlp_row_stats(const void* x, float* mean, float* rstd, int64_t T, int d, int dtype, float eps, void* stream) {
  return row_stats_impl(x, mean, rstd, T, d, dtype, eps, static_cast<cudaStream_t>(stream));
}

int spmlp_up_gate_ln(const void* x, const void* w_fold, const float* ln_s, const float* ln_c, const float* row_mean,
                     const float* row_rstd, void* h, uint32_t* tile_bits, void* z_out, int64_t T, int d, int F,
                     int dtype, int gate_op, float kappa, int64_t seq_len, void* stream) {
  if (!ln_s) return fail(SPMLP_EINVAL, "ln_s must be non-null");
  return up_gate_impl(x, w_fold, nullptr, h, tile_bits, z_out, T, d, F, dtype, gate_op, kappa, seq_len,
                      static_cast<cudaStream_t>(stream), ln_s, ln_c, row_mean, row_rstd);
}

int spmlp_down_sparse(const void* h, const uint32_t* tile_bits, const void* w_out, const void* b_out,
                      const void* residual, void* y, int64_t T, int F, int d, int dtype, int mode, uint64_t* stats,
                      void* stream) {
  return down_impl(h, tile_bits, w_out, b_out, residual, y, T, F, d, dtype, mode, stats,
                   static_cast<cudaStream_t>(stream));
}

int spmlp_down_scatter(const void* h, const uint32_t* tile_bits, const void* w_out, void* const* slots, int world,
                       int64_t T, int F, int d, int dtype, int mode, uint64_t* stats, void* stream) {
  if (!slots) return fail(SPMLP_EINVAL, "slots must be non-null");
  return down_impl(h, tile_bits, w_out, nullptr, nullptr, nullptr, T, F, d, dtype, mode, stats,
                   static_cast<cudaStream_t>(stream), slots, world);
}

int spmlp_reduce_broadcast(const void* recv, int world, int64_t rows, int d, const void* b_out, const void* residual,
                           void* const* targets, int n_targets, int dtype, void* stream) {
  return reduce_broadcast_impl(recv, world, rows, d, b_out, residual, targets, n_targets, dtype,
                               static_cast<cudaStream_t>(stream));
}

int spmlp_reduce_broadcast_multicast(const void* mc_part, void* mc_x, const void* residual, int64_t rows, int d,
                                     const void* b_out, int dtype, void* stream) {
  return multicast_reduce_broadcast_impl(mc_part, mc_x, residual, rows, d, b_out, dtype,
                                         static_cast<cudaStream_t>(stream));
}

int spmlp_joint(const void* h, const uint32_t* tile_bits, const void* z, const void* w2, const void* b2,
                const void* wo, const void* bo, const void* residual, void* out, int64_t T, int F, int d, int dtype,
                int mode, uint64_t* stats, void* stream) {
  return joint_impl(h, tile_bits, z, w2, b2, wo, bo, residual, out, T, F, d, dtype, mode, stats,
                    static_cast<cudaStream_t>(stream));
}

int spmlp_gate(const void* x, void* out, uint32_t* tile_bits, int64_t T, int F, int dtype, int gate_op, float kappa,
               void* stream) {
  return gate_impl(x, out, tile_bits, T, F, dtype, gate_op, kappa, static_cast<cudaStream_t>(stream));
}

int spmlp_mlp_forward(const void* x, const void* w_in, const void* b_in, const void* w_out, const void* b_out,
                      const void* residual, void* y, void* h_workspace, uint32_t* bits_workspace, int64_t T, int d,
                      int F, int dtype, int gate_op, float kappa, int64_t seq_len, int mode, uint64_t* stats,
                      void* stream) {
  int rc = up_gate_impl(x, w_in, b_in, h_workspace, bits_workspace, nullptr, T, d, F, dtype, gate_op, kappa, seq_len,
                        static_cast<cudaStream_t>(stream));
  if (rc) return rc;
  return down_impl(h_workspace, bits_workspace, w_out, b_out, residual, y, T, F, d, dtype, mode, stats,
                   static_cast<cudaStream_t>(stream));
}

int spmlp_mlp_forward_noalloc(const void* x, const void* w_in, const void* b_in, const void* w_out,
                              const void* b_out, const void* residual, void* y, int64_t T, int d, int F, int dtype,
                              int gate_op, float kappa, int64_t seq_len, int mode, uint64_t* stats, void* stream) {
  return mlp_forward_noalloc_impl(x, w_in, b_in, w_out, b_out, residual, y, T, d, F, dtype, gate_op, kappa, seq_len,
                                  mode, stats, static_cast<cudaStream_t>(stream));
}

int spmlp_head_support_words(int d) {
  if (d <= 0) return 0;
  return (d / 16 + 31) / 32;
}

int spmlp_head_prepare(const float* x, void* x_out, uint32_t* support, int64_t T, int d, int dtype, float kappa,
                       void* stream) {
  return head_prepare_impl(x, x_out, support, T, d, dtype, kappa, static_cast<cudaStream_t>(stream));
}

int spmlp_head_sparse(const void* x, const uint32_t* support, const void* w_vocab, void* logits,
                      const int32_t* active_tiles, int n_active, int64_t T, int d, int V, int dtype, int gate_axis,
                      uint64_t* stats, void* stream) {
  return head_impl(x, support, w_vocab, logits, active_tiles, n_active, T, d, V, dtype, gate_axis, stats,
                   static_cast<cudaStream_t>(stream));
}

int spmlp_head_fill(void* logits, const int32_t* tiles, int n_tiles, int64_t T, int V, int dtype, float value,
                    void* stream) {
  return head_fill_impl(logits, tiles, n_tiles, T, V, dtype, value, static_cast<cudaStream_t>(stream));
}

int spmlp_peer_barrier(long long* const* peer_slots, const long long* local_flags, int world, long long epoch,
                       void* stream) {
  if (!peer_slots || !local_flags) return fail(SPMLP_EINVAL, "peer_slots and local_flags must be non-null");
  if (world < 1 || world > kMaxRanks) return fail(SPMLP_EINVAL, "world=%d must be in [1, %d]", world, kMaxRanks);
  if (epoch < 1) return fail(SPMLP_EINVAL, "epoch must be positive and increase from call to call");
  PeerFlags pf{};
  for (int j = 0; j < world; ++j) {
    if (!peer_slots[j] || (reinterpret_cast<uintptr_t>(peer_slots[j]) & 7u))
      return fail(SPMLP_EALIGN, "peer slot %d must be non-null and 8-byte aligned", j);
    pf.dst[j] = peer_slots[j];
  }
  if (reinterpret_cast<uintptr_t>(local_flags) & 7u) return fail(SPMLP_EALIGN, "local_flags must be 8-byte aligned");
  DeviceInfo* dev = nullptr;
  int rc = current_device_info(&dev);
  if (rc) return rc;
  peer_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(pf, local_flags, world, epoch, dev->status);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "peer_barrier_kernel launch");
  return 0;
}

int spmlp_selftest_wait(void* stream) {
  DeviceInfo* dev = nullptr;
  int rc = current_device_info(&dev);
  if (rc) return rc;
  wait_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(dev->status);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "wait_probe_kernel launch");
  return 0;
}

int spmlp_set_sm_count_target(int sms) {
  if (sms < 0) return fail(SPMLP_EINVAL, "sms=%d must be >= 0 (0 = every SM)", sms);
  DeviceInfo* dev = nullptr;
  int rc = current_device_info(&dev);
  if (rc) return rc;
  dev->sm_target = sms;
  return 0;
}

int spmlp_device_status(int device, int* status_out) {
  if (!status_out) return fail(SPMLP_EINVAL, "status_out must be non-null");
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if ((e = cudaSetDevice(device)) != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int));
  cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyFromSymbol(status word)");
  *status_out = v & 0xff;  // the code; the bits above count the events
  return 0;
}

int spmlp_clear_device_status(int device) {
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if ((e = cudaSetDevice(device)) != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  const int zero = 0;
  e = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int));
  cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyToSymbol(status word)");
  return 0;
}

}  // extern "C"
