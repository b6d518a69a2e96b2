/*
 * spmlp.h — C ABI of the B200 (sm_100a) activation-sparse GPT-NeoX MLP kernels.
 *
 * The library (libspmlp.so) replaces, for CUDA tensors, the forward path of
 *   GPTNeoXMLP.forward = dense_4h_to_h(act(dense_h_to_4h(m)))
 * (transformers/models/gpt_neox/modeling_gpt_neox.py, class GPTNeoXMLP) with
 * `act` one of the reference's gate modules
 * (src/sparsity_research/sites.py:86-107, runs/063-2026-10-07-pythia14m-tile-specialized-kernel/tile_gate.py:9-33),
 * and the reference's sparse consumer / vocabulary-head kernels
 * (runs/042-2026-09-20-pythia70m-sparse-scale/kernel/joint/joint.cu:138-157, runs/068-2026-10-08-pythia14m-aligned-vocabulary-tiles/inference/head.cu:79-118).
 *
 * Conventions shared by every entry point
 *   - All tensors are device pointers, row-major and contiguous, 16-byte aligned.
 *   - Activations and weights share one dtype: SPMLP_F16 or SPMLP_BF16.
 *     Accumulation is fp32; each output is rounded once (bias added first),
 *     matching torch.nn.Linear on CUDA.
 *   - Weights use torch.nn.Linear's layout: [out_features, in_features].
 *   - `stream` is a cudaStream_t (NULL = legacy default stream); kernels are
 *     launched on it and nothing synchronises the host.
 *   - Return value: 0 on success, a negative SPMLP_E* code for an argument
 *     error (nothing launched), or a positive cudaError_t.  The message of the
 *     last failure on the calling thread is returned by spmlp_last_error().
 *   - No entry point allocates device memory except where stated.
 *   - The kernels never trap: a device-side wait that does not finish within
 *     2 s records a code in the per-device status word (spmlp_device_status)
 *     and the kernel returns early, leaving its outputs incomplete.  The code
 *     stays set until spmlp_clear_device_status; kernels launched afterwards
 *     run normally (each compares the word against the value it found at
 *     launch).  A caller that must know whether a result is good reads the
 *     status word after the work it depends on.
 */
#ifndef SPMLP_H_
#define SPMLP_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dtypes */
#define SPMLP_F16 0
#define SPMLP_BF16 1

/* gate operators applied to z = round(x W_in^T + b_in) (the `act` slot of GPTNeoXMLP) */
#define SPMLP_GATE_IDENTITY 0    /* h = z                                                */
#define SPMLP_GATE_GELU 1        /* h = gelu_erf(z): ungated A0 (ACT2FN["gelu"])          */
#define SPMLP_GATE_ONE_SIDED 2   /* h = z if z >= kappa else 0: sites.py:86-94            */
#define SPMLP_GATE_SYMMETRIC 3   /* h = z if |z| >= kappa else 0: sites.py:97-107         */
#define SPMLP_GATE_RELU 4        /* h = max(z, 0): torch.nn.ReLU (sites.py:221-222)       */
#define SPMLP_GATE_GELU_MASKED 5 /* h = gelu_erf(z) if z > kappa else 0                   */
#define SPMLP_GATE_CORNER 6      /* 8x16 tile kept iff its top-left z > kappa: runs/063-2026-10-07-pythia14m-tile-specialized-kernel/tile_gate.py:20-33 */

/* down-projection modes */
#define SPMLP_DOWN_DENSE 0 /* every K-block multiplied (skipping disabled)          */
#define SPMLP_DOWN_SKIP 1  /* K-blocks whose 16x64 tiles are all zero for the whole
                              down-projection tile (spmlp_down_tile_tokens(mode)
                              tokens) are neither loaded nor multiplied; 256-token
                              tiles on CTA pairs (fastest dense throughput)        */
#define SPMLP_DOWN_SKIP_FINE 2 /* as SPMLP_DOWN_SKIP with 128-token tiles on single
                              CTAs: skips more K-blocks when zeros come in token
                              blocks narrower than 256 (e.g. 64-token tiles)        */
#define SPMLP_DOWN_COMPACT 3 /* compact mode: live K granules gathered; the bitmap
                              is the 16x16 one (spmlp_tile_bits16_from_h); each
                              pipeline stage gathers four live 16-feature granules of
                              the tile (the union over its tokens) into shared memory,
                              and only those are loaded and multiplied; 256-token tiles
                              on CTA pairs.  For zeros structured at 16 features, e.g.
                              the reference's 8x16 corner-tile gate
                              (runs/063-2026-10-07-pythia14m-tile-specialized-kernel/tile_gate.py:9-33) */
#define SPMLP_DOWN_COMPACT_FINE 4 /* SPMLP_DOWN_COMPACT with 128-token tiles on single CTAs */

/* error codes (negative returns) */
#define SPMLP_EINVAL -1   /* bad argument (null pointer, bad enum, non-finite kappa) */
#define SPMLP_ESHAPE -2   /* unsupported shape (alignment / divisibility)            */
#define SPMLP_EALIGN -3   /* pointer not 16-byte aligned                              */
#define SPMLP_EDEVICE -4  /* current device is not an sm_100 GPU                      */
#define SPMLP_EDRIVER -5  /* tensor-map encoding unavailable or failed                */
#define SPMLP_EFORMAT -6  /* serialized mask malformed, truncated or checksum mismatch */

/* Tile bitmap geometry.  Bit (g % 32) of word [r * words + g / 32] is set iff
 * the 16-token x 64-feature tile (rows 16r.., features 64g..) of h holds a
 * nonzero.  words = spmlp_tile_bits_words(F); the buffer holds
 * ceil(T/16) * words uint32 words. */
int spmlp_tile_bits_words(int F);
int64_t spmlp_tile_bits_size(int64_t T, int F);

/* Persisted tile bitmaps (host memory, no GPU needed).  No counterpart in the
 * reference, which recomputes its masks on every forward; this is the format
 * for keeping a bitmap across calls or processes (e.g. a cached prefill).  The
 * byte string is self-describing: a 64-byte header ("SPMB", version 1,
 * encoding, 16x64 tile geometry, T, F, words per row group, CRC-32 of the
 * payload, payload bytes, live tiles) and the payload.
 *   SPMLP_MASK_RAW:      the bitmap words as above.
 *   SPMLP_MASK_ROW_RUNS: runs of identical 16-row groups (u32 run count, then
 *                        per run a u32 length and the group's words); lossless.
 *                        Element-random masks (all groups alike) become one run,
 *                        token-blocked masks shrink by their block height.
 * encode returns the bytes written; decode rebuilds the exact words and rejects
 * malformed or corrupted input with SPMLP_EFORMAT. */
#define SPMLP_MASK_RAW 0
#define SPMLP_MASK_ROW_RUNS 1
int64_t spmlp_mask_encoded_size(const uint32_t* tile_bits, int64_t T, int F, int encoding);
int64_t spmlp_mask_encode(const uint32_t* tile_bits, int64_t T, int F, int encoding, void* out, int64_t capacity);
int spmlp_mask_decode_header(const void* data, int64_t n, int64_t* T, int* F, int* encoding);
int spmlp_mask_decode(const void* data, int64_t n, uint32_t* tile_bits, int64_t capacity_words);

/* 16x16 tile bitmap of an existing h [T,F] for the compact down modes: bit g % 32 of
 * word r * spmlp_tile_bits16_words(F) + g / 32 is set iff tile (16-row group r,
 * 16-feature group g) holds a nonzero (-0.0 counts as zero); every word is written.
 * spmlp_tile_bits16_size gives the words for T tokens.  No reference counterpart:
 * the reference derives its K16 masks inside the consumer
 * (runs/042-2026-09-20-pythia70m-sparse-scale/kernel/joint/joint.cu:14-31). */
int spmlp_tile_bits16_words(int F);
int64_t spmlp_tile_bits16_size(int64_t T, int F);
int spmlp_tile_bits16_from_h(const void* h, uint32_t* tile_bits16, int64_t T, int F, void* stream);

/* Tile bitmap of an existing h [T,F] (same bit semantics as spmlp_up_gate's;
 * for callers whose h does not come from spmlp_up_gate).  Overwrites every
 * word of tile_bits.  Requires F % 64 == 0.  No reference counterpart: the
 * reference derives its K16 masks inside the consumer
 * (runs/042-2026-09-20-pythia70m-sparse-scale/kernel/joint/joint.cu:14-31). */
int spmlp_tile_bits_from_h(const void* h, uint32_t* tile_bits, int64_t T, int F, int dtype, void* stream);

/* Up-projection fused with bias, rounding, gate and tile bitmap.
 * Replaces GPTNeoXMLP.dense_h_to_4h followed by GPTNeoXMLP.act
 * (pythia.py:76-77 installs the gate as mlp.act).
 *   x [T,d], w_in [F,d], b_in [F] (nullable) -> h [T,F], tile_bits (zeroed
 *   here, then filled), z_out [T,F] (nullable: the pre-gate z, for checks).
 *   kappa must already be rounded to the activation dtype (runs/063-2026-10-07-pythia14m-tile-specialized-kernel/kernel.py:17-19).
 *   seq_len: tokens per sequence for SPMLP_GATE_CORNER (T a multiple of it;
 *   8-token blocks restart at each sequence, and a sequence whose length is not
 *   a multiple of 8 ends with a shorter block decided by its own first row, as
 *   runs/063-2026-10-07-pythia14m-tile-specialized-kernel/tile_gate.py:25-28
 *   allows; with several such sequences the gate runs as a second in-place pass
 *   over h), ignored otherwise.
 *   Requires d % 64 == 0, F % 64 == 0, 1 <= T < 2^31. */
int spmlp_up_gate(const void* x, const void* w_in, const void* b_in, void* h, uint32_t* tile_bits,
                  void* z_out, int64_t T, int d, int F, int dtype, int gate_op, float kappa,
                  int64_t seq_len, void* stream);

/* Up projection with the MLP's LayerNorm folded in, so that the normalized
 * activation m = post_attention_layernorm(x) is never materialised.  Replaces
 * the reference's paired LayerNorm (runs/035-2026-09-18-pythia70m-k050-port/kernel/norm/norm.cu:23-60,
 * its MLP output m) followed by dense_h_to_4h + gate.
 *   spmlp_row_stats: per token of x [T,d], mean and rstd = 1/sqrt(var + eps)
 *   (fp32, biased variance as torch.nn.LayerNorm).
 *   spmlp_up_gate_ln: as spmlp_up_gate on the raw x with w_fold = W_in diag(gamma)
 *   [F,d] in the activation dtype, ln_s[f] = sum_k w_fold[f,k] and
 *   ln_c = b_in + W_in beta (fp32 [F]):
 *     z = round(rstd * (x w_fold^T - mean * ln_s) + ln_c), then the gate, bitmap
 *     and optional z export as spmlp_up_gate.
 *   z differs from the unfused round(round(LN(x)) W_in^T + b_in) by the rounding
 *   of m that the fold skips. */
int spmlp_row_stats(const void* x, float* mean, float* rstd, int64_t T, int d, int dtype, float eps, void* stream);
int spmlp_up_gate_ln(const void* x, const void* w_fold, const float* ln_s, const float* ln_c, const float* row_mean,
                     const float* row_rstd, void* h, uint32_t* tile_bits, void* z_out, int64_t T, int d, int F,
                     int dtype, int gate_op, float kappa, int64_t seq_len, void* stream);

/* Sparse down-projection.  Replaces GPTNeoXMLP.dense_4h_to_h and the h branch
 * of the reference's joint consumer (runs/042-2026-09-20-pythia70m-sparse-scale/kernel/joint/joint.cu:138-157,
 * adapter call runs/042-2026-09-20-pythia70m-sparse-scale/kernel/joint/candidate.py:26-33).
 *   h [T,F], tile_bits from spmlp_up_gate (ignored for SPMLP_DOWN_DENSE),
 *   w_out [d,F], b_out [d] (nullable), residual [T,d] (nullable) -> y [T,d]
 *   y = round(h w_out^T + b_out), then round(y + residual) when given.
 *   A K-block (64 features) is skipped for a tile of spmlp_down_tile_tokens(mode)
 *   tokens when every 16x64 bitmap tile of it in that token range is zero; in the
 *   compact modes tile_bits is the 16x16 bitmap and a 16-feature granule is skipped
 *   when every 16x16 tile of it in that token range is zero.
 *   stats (nullable, 2 x uint64, accumulated): [0] issued K16 MMA steps,
 *   [1] skipped K16 MMA steps; one step is one tcgen05.mma over a
 *   spmlp_down_tile_tokens(mode) x 256 output tile.
 *   Skipping is exact for finite weights (0 * w == 0). */
int spmlp_down_tile_tokens(int mode);
int spmlp_down_sparse(const void* h, const uint32_t* tile_bits, const void* w_out, const void* b_out,
                      const void* residual, void* y, int64_t T, int F, int d, int dtype, int mode,
                      uint64_t* stats, void* stream);

/* d_ff split with the reduce-scatter fused into the down projection.  No
 * counterpart in the reference (it runs on one GPU); it replaces the partial
 * down projection followed by an NCCL reduce-scatter (ncclReduceScatter of the
 * partial y over tokens) that a d_ff split of GPTNeoXMLP.dense_4h_to_h needs.
 *   spmlp_down_scatter: as spmlp_down_sparse without bias and residual, but the
 *   rounded partial of tokens [j*T/world, (j+1)*T/world) is stored into
 *   slots[j] ([T/world, d], this rank's slot in rank j's receive buffer, peer
 *   memory reachable over NVLink) while the other tiles are still computing.
 *   T/world must be a multiple of 256.
 *   spmlp_reduce_broadcast: after every rank's scatter has completed (the caller
 *   orders it, e.g. with a one-element all-reduce), for this rank's token block:
 *   y = round(round(sum_r recv[r] + b_out) + residual), the sum in fp32 in rank
 *   order, written to each of targets[0..n_targets) (this rank's block of each
 *   rank's copy of the next layer's input: the all-gather of the next input in
 *   the same pass).  recv [world, rows, d]; residual may be one of the targets. */
int spmlp_down_scatter(const void* h, const uint32_t* tile_bits, const void* w_out, void* const* slots, int world,
                       int64_t T, int F, int d, int dtype, int mode, uint64_t* stats, void* stream);
int spmlp_reduce_broadcast(const void* recv, int world, int64_t rows, int d, const void* b_out,
                           const void* residual, void* const* targets, int n_targets, int dtype, void* stream);
/* The same finish of the layer through NVLink SHARP, replacing the reduce-scatter +
 * all-gather pair (ncclReduceScatter / ncclAllGather) of a d_ff split where the
 * GPUs' memory is bound to an NVSwitch multicast object.  Every rank has written
 * its rounded partial of all T tokens ([T, d], no bias, e.g. spmlp_down_sparse)
 * into its own copy of a multicast-bound buffer, and the caller has ordered those
 * writes before this call on every rank (spmlp_peer_barrier).  For this rank's
 * block (rows tokens): mc_part is the block's address in the partial buffer's
 * multicast mapping, mc_x in the next input's; residual is the block in this
 * rank's local copy of the layer input (nullable).  y = round(round(s + b_out) +
 * residual) with s = round(sum over ranks), reduced in fp32 inside the switch
 * (multimem.ld_reduce .acc::f32), then written to every rank's copy (multimem.st). */
int spmlp_reduce_broadcast_multicast(const void* mc_part, void* mc_x, const void* residual, int64_t rows, int d,
                                     const void* b_out, int dtype, void* stream);
/* Barrier between the ranks of the fused d_ff split over NVLink peer memory,
 * ordered on `stream`: this rank stores `epoch` into peer_slots[j] (its slot in
 * rank j's int64 flag array, [world]) after a system-scope fence, then waits until
 * local_flags[j] >= epoch for every j.  epoch must grow from call to call (flags
 * start at 0).  Each wait gives up after about 2 s with SPMLP_STATUS_TIMEOUT_PEER
 * in the status word; nothing faults.  One rank per GPU: two ranks sharing a
 * GPU are not guaranteed to run at the same time, so one would wait out the 2 s
 * limit and give up; that is not supported. */
int spmlp_peer_barrier(long long* const* peer_slots, const long long* local_flags, int world, long long epoch,
                       void* stream);

/* Joint consumer: the MLP's down projection and the attention output
 * projection of one GPT-NeoX layer, summed with its parallel residual, in one
 * kernel.  Replaces the reference's joint (the k018 Joint.__call__ of
 * runs/026-2026-09-06-pythia14m-fused-sparse-kernel/autoresearch/candidates/k018/candidate.py:32-46
 * called from layer_forward :48-56, and the K042 kernel
 * runs/042-2026-09-20-pythia70m-sparse-scale/kernel/joint/joint.cu:88-137 behind
 * runs/042-2026-09-20-pythia70m-sparse-scale/kernel/joint/candidate.py:26-33).
 *   h [T,F] with tile_bits (ignored for SPMLP_DOWN_DENSE), z [T,d] (the
 *   attention context before its dense projection), w2 [d,F], b2 [d], wo [d,d],
 *   bo [d] (biases nullable), residual [T,d] (nullable) -> out [T,d]
 *   out = round(round(round(h w2^T + b2) + round(z wo^T + bo)) + residual),
 *   every addition in fp32: the rounding order of
 *   runs/027-2026-09-06-pythia14m-kernel-sparsity-characterization/test_adapter.py:19-24
 *   and runs/042-2026-09-20-pythia70m-sparse-scale/controls.py:19-26.
 *   The reference's input gates (h < th and z < tz set to zero) are applied
 *   beforehand with spmlp_gate.  mode and stats as spmlp_down_sparse (over the
 *   h branch; z is dense); output tiles are spmlp_down_tile_tokens(mode) x 256. */
int spmlp_joint(const void* h, const uint32_t* tile_bits, const void* z, const void* w2, const void* b2,
                const void* wo, const void* bo, const void* residual, void* out, int64_t T, int F, int d,
                int dtype, int mode, uint64_t* stats, void* stream);

/* Elementwise gate of an activation x [T,F] into out (the same buffer, or one
 * that does not overlap it), and, when tile_bits is non-null, the 16x64 tile
 * bitmap of the gated values (layout as spmlp_up_gate's).  gate_op is one of
 * SPMLP_GATE_IDENTITY, _ONE_SIDED, _SYMMETRIC, _RELU with kappa rounded to
 * dtype: the reference's FixedOneSidedThreshold / FixedSymmetricThreshold /
 * ReLU (src/sparsity_research/sites.py:86-107, 221-222) as the joint consumer
 * applies them to its h and z inputs (runs/042-2026-09-20-pythia70m-sparse-scale/controls.py:20-23).
 * F must be a positive multiple of 64. */
int spmlp_gate(const void* x, void* out, uint32_t* tile_bits, int64_t T, int F, int dtype, int gate_op,
               float kappa, void* stream);

/* Whole gated MLP forward: spmlp_up_gate then spmlp_down_sparse, with the
 * caller's h and tile-bit buffers as workspace (GPTNeoXMLP.forward). */
int spmlp_mlp_forward(const void* x, const void* w_in, const void* b_in, const void* w_out,
                      const void* b_out, const void* residual, void* y, void* h_workspace,
                      uint32_t* bits_workspace, int64_t T, int d, int F, int dtype, int gate_op,
                      float kappa, int64_t seq_len, int mode, uint64_t* stats, void* stream);

/* Allocation-free variant of spmlp_mlp_forward.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory at the
 * point of the call, for example code running while a stream is being captured
 * into a CUDA graph (cudaMalloc is not permitted during a global-mode capture),
 * code inside a framework or serving engine whose own allocator already holds
 * the GPU's memory (a raw cudaMalloc can fail there, and cudaFree synchronises
 * the device), or a foreign-language host with no binding to a device
 * allocator.  Such callers pass only inputs and outputs.
 *
 * The workspace (h and the tile bitmap) lives in one static device buffer of
 * SPMLP_NOALLOC_SCRATCH_BYTES inside the library, reserved on every GPU where
 * the library's module is loaded and held until the process exits; the call
 * itself allocates nothing.  Calls with 2*T*F (rounded up to 256) plus
 * 4*spmlp_tile_bits_size(T, F) bytes above that size are rejected with
 * SPMLP_ESHAPE: at F = 2048 that is about 8190 tokens per call.
 *
 * The first call on each device looks up the buffer's device address
 * (cudaGetSymbolAddress with that device current) and caches it; make that
 * first call before any stream capture.  Every call on a device shares the one
 * buffer, which keeps the last call's contents (every bit of the bitmap is
 * rewritten on each call): calls that can overlap on the GPU — on different streams or from
 * different host threads, on the same device — race on it and must be
 * serialised by the caller.  Arguments and results are as spmlp_mlp_forward's. */
#define SPMLP_NOALLOC_SCRATCH_BYTES (32u * 1024u * 1024u)
int spmlp_mlp_forward_noalloc(const void* x, const void* w_in, const void* b_in, const void* w_out,
                              const void* b_out, const void* residual, void* y, int64_t T, int d, int F,
                              int dtype, int gate_op, float kappa, int64_t seq_len, int mode,
                              uint64_t* stats, void* stream);

/* head gate axes for spmlp_head_sparse */
#define SPMLP_HEAD_DENSE 0  /* every K16 group and every vocabulary column                  */
#define SPMLP_HEAD_GATE_K 1 /* skip 16x16 head-input tiles whose corner certificate failed  */
#define SPMLP_HEAD_GATE_N 2 /* compute only the listed 128-column vocabulary tiles          */

/* Corner certificates + cast of the vocabulary-head input.  Replaces the
 * reference's prepare step (runs/068-2026-10-08-pythia14m-aligned-vocabulary-tiles/inference/head.cu:9-16,79-91;
 * Head.forward at .../inference/head.py:64-79).
 *   x [T,d] fp32 -> x_out [T,d] in dtype with dead 16x16 tiles zeroed, and
 *   support bits: bit (j%32) of word [r*spmlp_head_support_words(d) + j/32]
 *   set iff x[16r, 16j] > kappa (fp32 comparison before the cast).
 *   Requires d % 64 == 0. */
int spmlp_head_support_words(int d);
int spmlp_head_prepare(const float* x, void* x_out, uint32_t* support, int64_t T, int d, int dtype,
                       float kappa, void* stream);

/* Vocabulary projection logits [T,V] = x [T,d] w_vocab[V,d]^T (embed_out, no
 * bias), fp32 accumulation, one rounding to dtype.  Replaces Head.project /
 * project_kernel (runs/068-2026-10-08-pythia14m-aligned-vocabulary-tiles/inference/head.cu:18-77,104-118).
 *   gate_axis SPMLP_HEAD_DENSE: all columns.
 *   SPMLP_HEAD_GATE_K: K16 steps whose 16x16 tile is dead for all 128 tokens
 *     of a tile are skipped (support from spmlp_head_prepare).
 *   SPMLP_HEAD_GATE_N: only the n_active 128-column tiles listed (device int32,
 *     indices < ceil(V/128)) are computed; other logits are left unwritten
 *     (spmlp_head_fill masks them).
 *   stats (nullable): [0] issued K16 steps, [1] skipped K16 steps.
 *   Requires d % 64 == 0, V % 128 == 0. */
int spmlp_head_sparse(const void* x, const uint32_t* support, const void* w_vocab, void* logits,
                      const int32_t* active_tiles, int n_active, int64_t T, int d, int V, int dtype,
                      int gate_axis, uint64_t* stats, void* stream);

/* Write `value` (rounded to dtype) into the listed 128-column tiles of logits [T,V]. */
int spmlp_head_fill(void* logits, const int32_t* tiles, int n_tiles, int64_t T, int V, int dtype,
                    float value, void* stream);

/* At most `sms` SMs of the current device for the persistent GEMMs launched afterwards
 * on it (0 = every SM, the default), like cuBLAS's cublasSetSmCountTarget: a caller that
 * runs other kernels concurrently on another stream (the d_ff split's reduction over
 * NVLink beside the next token slice's projections) leaves them SMs.  A CTA pair counts
 * two.  No reference counterpart. */
int spmlp_set_sm_count_target(int sms);

/* Status word of `device` written by kernels that gave up on a bounded wait
 * (0 = none; otherwise the code of the most recent wait that gave up, which
 * stays until cleared).  Within one launch, the first wait that gives up makes
 * the launch's other waits give up at once, so a failed launch unwinds quickly;
 * later launches are not affected by a code that is already set.  Reading
 * synchronises that device.  clear resets it to 0. */
#define SPMLP_STATUS_OK 0
#define SPMLP_STATUS_TIMEOUT_PRODUCER 1 /* TMA warp: no free pipeline stage          */
#define SPMLP_STATUS_TIMEOUT_MMA 2      /* MMA warp: no loaded stage / free TMEM     */
#define SPMLP_STATUS_TIMEOUT_EPILOGUE 3 /* epilogue: no finished accumulator         */
#define SPMLP_STATUS_TIMEOUT_DRAIN 4    /* teardown: in-flight copies / MMAs pending */
#define SPMLP_STATUS_TIMEOUT_PROBE 5    /* spmlp_selftest_wait                       */
#define SPMLP_STATUS_TIMEOUT_PEER 6     /* spmlp_peer_barrier: a peer did not signal */
int spmlp_device_status(int device, int* status_out);
int spmlp_clear_device_status(int device);

/* Self-test of failure detection (no counterpart in the reference): one kernel
 * waits, with the bounded wait every kernel here uses, on a barrier that nothing
 * completes.  After about 2 s it gives up, records SPMLP_STATUS_TIMEOUT_PROBE in
 * the status word and returns; the context stays usable.  Nothing faults or
 * traps.  It waits the full 2 s whether or not the status word is already set. */
int spmlp_selftest_wait(void* stream);

/* Message of the last failed call on this thread ("" if none). */
const char* spmlp_last_error(void);

/* Library ABI version (major * 100 + minor). */
int spmlp_version(void);

#ifdef __cplusplus
}
#endif

#endif /* SPMLP_H_ */
