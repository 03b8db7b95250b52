/*
 * gdn.h -- C ABI of the B200 GatedDeltaNet (GDN) layer step.
 *
 * This is the drop-in boundary for the GDN path of qwen-mlx.  It replaces:
 *   - the recurrence entry point  gated_delta_kernel   (src/models/metal_gdn.rs:170-218)
 *   - the fused S=1 / S>1 layer body between the projections of
 *     GatedDeltaNet::forward_with_cache                (src/models/qwen3_5.rs:588-665)
 *   - the compiled beta/g closure  compiled_beta_g     (src/models/compiled_ops.rs:68-94)
 *   - the executor's per-step stack/unstack of per-sequence states
 *     Qwen35Executor::{stack_caches,unstack_caches}    (src/scheduler/mlx_executor.rs:92-130)
 *     by a device-resident, slot-indexed state pool.
 *
 * Conventions
 *   - bf16 tensors are passed as uint16_t bit patterns (gdn_bf16).
 *   - Every function returns GDN_OK (0) or a GDN_E_* code; nothing throws or
 *     aborts across the ABI.  gdn_last_error() returns a message for the last
 *     failure on the calling thread.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *     Compute calls are asynchronous on that stream and take DEVICE pointers;
 *     calls documented as "synchronous" take host pointers.
 *   - A pool belongs to one device; calls switch to that device and restore
 *     the caller's current device before returning.
 *   - Only head_k_dim = head_v_dim = 128 and conv_kernel = 4 are specialised;
 *     other shapes return GDN_E_UNSUPPORTED.
 *
 * Layouts (row-major, the reference's own):
 *   recurrent state of one (slot, layer):  [Hv][dv][dk] f32   (metal_gdn.rs:144-152)
 *   conv state of one (slot, layer):       [K-1][D] bf16      (qwen3_5.rs:598-604)
 *   conv weight:                           [D][K] bf16        (qwen3_5.rs:1058-1066, [D,K,1])
 *   D = 2*Hk*dk + Hv*dv channels in the order q | k | v       (qwen3_5.rs:513, :627-629)
 */
#ifndef GDN_B200_H
#define GDN_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__) || defined(__clang__)
#define GDN_API __attribute__((visibility("default")))
#else
#define GDN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define GDN_OK 0
#define GDN_E_INVALID 1     /* null pointer, negative size, inconsistent arguments */
#define GDN_E_UNSUPPORTED 2 /* shape not specialised on this build */
#define GDN_E_BAD_SLOT 3    /* slot id out of range, or used twice in one batch */
#define GDN_E_BAD_SEQLENS 4 /* cu_seqlens not starting at 0, decreasing, or not ending at n_tokens */
#define GDN_E_CUDA 5        /* CUDA runtime error (message in gdn_last_error) */
#define GDN_E_NOMEM 6       /* device allocation failed */
#define GDN_E_DEVICE 7      /* a device-side bounds check tripped (see gdn_pool_check) */

typedef uint16_t gdn_bf16;

/* Model shapes.  Mirrors the GDN fields of Qwen35Config (src/models/qwen3_5.rs:30-70). */
typedef struct gdn_config {
    int32_t hidden;       /* hidden_size */
    int32_t n_k_heads;    /* linear_num_key_heads */
    int32_t n_v_heads;    /* linear_num_value_heads (multiple of n_k_heads) */
    int32_t head_k_dim;   /* linear_key_head_dim  (128) */
    int32_t head_v_dim;   /* linear_value_head_dim (128) */
    int32_t conv_kernel;  /* linear_conv_kernel_dim (4) */
    int32_t n_layers;     /* number of GDN layers held by a pool */
    float rms_norm_eps;   /* rms_norm_eps of the gated output norm */
} gdn_config;

/* Per-layer parameters of the fused step (GatedDeltaNet fields, qwen3_5.rs:466-490). Device pointers. */
typedef struct gdn_layer_weights {
    const gdn_bf16* conv_w; /* [D][K]  conv1d.weight */
    const float* A_log;     /* [Hv]    A_log */
    const float* dt_bias;   /* [Hv]    dt_bias, as f32 values (a bf16 parameter widened exactly) */
    const gdn_bf16* norm_w; /* [dv]    norm.weight (RMSNormGated) */
    /* Non-zero when the checkpoint stores dt_bias in bf16.  MLX then adds a + dt_bias and takes its exp
     * as bf16 ops, each rounded to bf16, before the f32 log(. + 1) (compiled_ops.rs:36-40); with 0 the
     * add and exp are f32, as for an f32 dt_bias. */
    int32_t dt_bias_bf16;
} gdn_layer_weights;

/* Projection outputs feeding one layer step and its output, packed by token.
 * Each buffer is [n_tokens][ld] with its own row stride (elements), so a single
 * merged projection output [N][D + Hv*dv + 2*Hv] can be passed three times.
 * ab holds b in columns [0,Hv) and a in [Hv,2Hv): the reference's merged
 * order (qwen3_5.rs:583, :1038). */
typedef struct gdn_step_io {
    const gdn_bf16* qkv; int64_t ld_qkv; /* [N][D]     in_proj_qkv output (pre-conv) */
    const gdn_bf16* z;   int64_t ld_z;   /* [N][Hv*dv] in_proj_z output */
    const gdn_bf16* ab;  int64_t ld_ab;  /* [N][2*Hv]  in_proj_b | in_proj_a outputs */
    gdn_bf16* out;       int64_t ld_out; /* [N][Hv*dv] silu(z) * rms_norm(y): input of out_proj */
} gdn_step_io;

typedef struct gdn_pool gdn_pool;

/* Message of the last failing call on this thread ("" if none). */
GDN_API const char* gdn_last_error(void);

/* Library version string. */
GDN_API const char* gdn_version(void);

/* ---------------------------------------------------------------- state pool
 * Replaces the executor's per-sequence Qwen35State caches (mlx_executor.rs:19-21)
 * and their stack/unstack (mlx_executor.rs:92-130): a sequence's state lives in
 * a fixed slot for its whole life, and a step addresses slots by id.
 * Device layout: rec  [n_layers][n_slots][Hv][dv][dk] f32
 *                conv [n_layers][n_slots][K-1][D] bf16
 * A new pool is zeroed (the reference's missing-cache zeros, qwen3_5.rs:598-601, :644-648). */
GDN_API int gdn_pool_create(int device, const gdn_config* cfg, int32_t n_slots, gdn_pool** out);
GDN_API int gdn_pool_destroy(gdn_pool* pool);

/* Size the pool's step scratch for up to `max_tokens` packed tokens per call
 * (a new pool holds max(n_slots, 1024)).  The scratch holds one 1056-byte record
 * per (v-head, token): 33 KiB per token for Hv = 32.  Synchronous; call it before
 * capturing a step into a CUDA graph, never while a step is in flight. */
GDN_API int gdn_pool_reserve_tokens(gdn_pool* pool, int32_t max_tokens);

/* Device pointers to one layer's slice of the pool (slot 0 of that layer). */
GDN_API int gdn_pool_layer_state(gdn_pool* pool, int32_t layer, float** rec, gdn_bf16** conv);

/* Bytes of device memory held by the pool (states + bookkeeping). */
GDN_API int gdn_pool_bytes(const gdn_pool* pool, size_t* bytes);

/* Zero the state of `n` slots (all layers): admission of a new sequence
 * (replaces qwen3_5.rs:598-601, :644-648).  slots: host array. Asynchronous. */
GDN_API int gdn_slot_reset(gdn_pool* pool, const int32_t* slots, int32_t n, void* stream);

/* Copy one (slot, layer) state out of / into the pool in the reference layout:
 * rec [Hv][dv][dk] f32 (the reference's [1,Hv,dv,dk] cache.1) and conv [K-1][D]
 * bf16 (cache.0).  Host pointers; synchronous.  Either pointer may be NULL. */
GDN_API int gdn_slot_export(gdn_pool* pool, int32_t slot, int32_t layer, float* rec, gdn_bf16* conv);
GDN_API int gdn_slot_import(gdn_pool* pool, int32_t slot, int32_t layer, const float* rec, const gdn_bf16* conv);

/* Host-side check of a batch's routing tables (host pointers): every slot in
 * range and used once, cu_seqlens[0] == 0, non-decreasing, cu_seqlens[n_seq] == n_tokens. */
GDN_API int gdn_validate_batch(const gdn_pool* pool, const int32_t* slot_ids, const int32_t* cu_seqlens, int32_t n_seq,
                       int32_t n_tokens);

/* The same check without a pool (n_slots given directly); needs no GPU. */
GDN_API int gdn_validate_tables(int32_t n_slots, const int32_t* slot_ids, const int32_t* cu_seqlens, int32_t n_seq,
                                int32_t n_tokens);

/* Read and optionally clear the pool's device error word (synchronous).  Kernels
 * skip any sequence whose slot id or token range fails their bounds checks and
 * record GDN_E_BAD_SLOT / GDN_E_BAD_SEQLENS as bit (1 << code) in this word. */
GDN_API int gdn_pool_check(gdn_pool* pool, int32_t* flags, int reset);

/* ---------------------------------------------------------------- compute */

/* One fused GDN layer step over a packed ragged batch (qwen3_5.rs:588-665 and
 * compiled_ops.rs:12-49): causal depthwise conv + SiLU with the conv state
 * update, q/k RMSNorm (gains 1/dk and dk^-1/2), beta = sigmoid(b),
 * g = exp(-exp(A_log) * softplus(a + dt_bias)), the gated delta rule on the
 * slot's f32 state (in place), and silu(z) * rms_norm(y, norm_w, eps).
 * Sequence i owns tokens [cu_seqlens[i], cu_seqlens[i+1]) and slot slot_ids[i].
 * A sequence of one token uses the reference's S=1 conv rounding
 * (qwen3_5.rs:593-610), a longer one its conv1d rounding (:611-624).
 * slot_ids / cu_seqlens: DEVICE arrays.  Asynchronous on `stream`. */
GDN_API int gdn_layer_step(gdn_pool* pool, int32_t layer, const gdn_layer_weights* w, const gdn_step_io* io,
                   const int32_t* slot_ids, const int32_t* cu_seqlens, int32_t n_seq, int32_t n_tokens,
                   void* stream);

/* gdn_layer_step with flags.  GDN_STEP_TABLES_STABLE: the routing tables were already used by
 * an earlier GDN call of this step after they were last written, and the call before this one on
 * the stream was for a different layer (typically layers 2..L of a step whose tables were uploaded
 * before layer 1).  The step then reads its routing entries and conv windows while the preceding
 * kernel is still running, and only the token inputs after it.  Same results as gdn_layer_step.
 * (An executor feature of this library; the reference's per-layer call is gated_delta_kernel,
 * metal_gdn.rs:170-218.) */
#define GDN_STEP_TABLES_STABLE 1u
GDN_API int gdn_layer_step_ex(gdn_pool* pool, int32_t layer, const gdn_layer_weights* w, const gdn_step_io* io,
                              const int32_t* slot_ids, const int32_t* cu_seqlens, int32_t n_seq, int32_t n_tokens,
                              uint32_t flags, void* stream);

/* Parameters of a whole mixer layer (GatedDeltaNet, qwen3_5.rs:466-503) and of its
 * decoder-layer input norm.  Device pointers.  w_in holds the four input
 * projections stacked by rows in the reference's merged order (qwen3_5.rs:1038-1047):
 * in_proj_qkv (D rows) | in_proj_z (Hv*dv) | in_proj_b (Hv) | in_proj_a (Hv).
 * Each projection may also (or instead) be given in a tiled form:
 *   *_q4    gdn_weight_tile_q4 tiles of the MLX 4-bit quantized weight (the reference's
 *           4-bit checkpoint, qwen3_5.rs:929-935): used for every call when present (streamed by
 *           the weight-streaming kernel for calls of at most 64 tokens on a weight of at least
 *           64 * #SMs rows; otherwise expanded to bf16 in the pool's scratch, then cuBLASLt);
 *   *_tiles gdn_weight_tile tiles of the bf16 weight: used for calls of at most 64 tokens.
 * Otherwise (and for longer calls without 4-bit tiles) the row-major bf16 weight runs on
 * cuBLASLt, so a row-major weight may be NULL only when one of the tiled forms covers
 * every call made. */
typedef struct gdn_mixer_weights {
    gdn_layer_weights step;      /* conv_w, A_log, dt_bias, norm_w */
    const gdn_bf16* w_in;        /* [D + Hv*dv + 2*Hv][hidden] or NULL */
    const gdn_bf16* w_out;       /* [hidden][Hv*dv]  out_proj, or NULL */
    const gdn_bf16* pre_norm_w;  /* [hidden] input_layernorm gain (used by gdn_stack_step) */
    const void* w_in_tiles;      /* gdn_weight_tile(D + Hv*dv + 2*Hv, hidden) of w_in, or NULL */
    const void* w_out_tiles;     /* gdn_weight_tile(hidden, Hv*dv) of w_out, or NULL */
    const void* w_in_q4;         /* gdn_weight_tile_q4 of the quantized w_in, or NULL */
    const void* w_out_q4;        /* gdn_weight_tile_q4 of the quantized w_out, or NULL */
} gdn_mixer_weights;

/* One projection (nn::Linear without bias, qwen3_5.rs:572-586, :668):
 * y[m][n] = bf16(sum_k x[m][k] * w[n][k]) with f32 accumulation, for m < n_tokens,
 * n < n_out, k < n_in.  x [n_tokens][ld_x], w [n_out][n_in], y [n_tokens][ld_y] bf16.
 * Runs cuBLASLt (library GEMM) on the pool's handle and stream.  Asynchronous. */
GDN_API int gdn_linear(gdn_pool* pool, int32_t n_tokens, int32_t n_out, int32_t n_in, const gdn_bf16* x,
                       int64_t ld_x, const gdn_bf16* w, gdn_bf16* y, int64_t ld_y, void* stream);

/* Bytes of the tiled copy of a bf16 projection weight w [n_out][n_in] (0 for a bad shape). */
GDN_API int64_t gdn_weight_tile_bytes(int32_t n_out, int32_t n_in);

/* Write the tiled copy of w [n_out][n_in] bf16 (row-major, device) into `tiles`
 * (gdn_weight_tile_bytes bytes, 16-byte aligned, device): the layout the
 * weight-streaming tensor-core kernel reads.  Blocks of 8 rows x 64 columns, 1 KB
 * each, block (kt, rg) (columns [64 kt, +64), rows [8 rg, +8)) at
 * (kt * ceil(n_out/8) + rg) * 1024; inside it element (8 rg + r, 64 kt + 8 c + e) at
 * byte c*128 + r*16 + e*2; rows >= n_out and columns >= n_in are zero.  Done once
 * when weights are loaded.  Asynchronous. */
GDN_API int gdn_weight_tile(int32_t n_out, int32_t n_in, const gdn_bf16* w, void* tiles, void* stream);

/* Bytes of the tiled copy of an MLX 4-bit weight of logical shape [n_out][n_in]
 * (n_in a multiple of 64; 0 otherwise). */
GDN_API int64_t gdn_weight_tile_q4_bytes(int32_t n_out, int32_t n_in);

/* Tile an MLX affine 4-bit weight (bits 4, group size 64, as nn::QuantizedLinear holds it after
 * quantize, qwen3_5.rs:929-935): w_q [n_out][n_in/8] uint32 (column k in bits 4*(k%8) of word
 * k/8), scales and biases [n_out][n_in/64] bf16; weight = scale * q + bias.  Blocks of 8 rows x
 * one group, 288 B each, block (kt, rg) at (kt * ceil(n_out/8) + rg) * 288: word (c, r) at
 * c*32 + r*4 holds the codes of row 8 rg + r, columns 64 kt + 8c .. +7 (column 8c+e in nibble
 * e/2 for even e, 4 + e/2 for odd e), then the 8 scales at 256 and the 8 biases at 272; rows
 * >= n_out are zero.  Device pointers, 16-byte aligned tiles.  Asynchronous. */
GDN_API int gdn_weight_tile_q4(int32_t n_out, int32_t n_in, const uint32_t* w_q, const gdn_bf16* scales,
                               const gdn_bf16* biases, void* tiles, void* stream);

/* gdn_linear on a bf16 tiled weight, on the weight-streaming tensor-core kernel
 * (tokens in blocks of 64, each block streams the weight once):
 * y[m][n] = bf16(sum_k x[m][k] * w[n][k]), f32 accumulation.  n_in % 8 == 0, x rows
 * 16-byte aligned (ld_x % 8 == 0).  The sum order is fixed per shape and device, so
 * results repeat bit for bit.  Asynchronous. */
GDN_API int gdn_linear_tiled(gdn_pool* pool, int32_t n_tokens, int32_t n_out, int32_t n_in, const gdn_bf16* x,
                             int64_t ld_x, const void* w_tiles, gdn_bf16* y, int64_t ld_y, void* stream);

/* The 4-bit quantized projection (MLX quantized_matmul with transpose, bits 4, group 64,
 * qwen3_5.rs:572-586 / :668 on the quantized checkpoint): each weight is dequantized once to
 * bf16 (scale * q + bias, one rounding), then y[m][n] = bf16(sum_k x[m][k] * w[n][k]) with
 * f32 accumulation on the tensor cores.  w_q4_tiles from gdn_weight_tile_q4; n_in % 64 == 0,
 * x rows 16-byte aligned.  Tokens in blocks of 64.  Deterministic.  Asynchronous. */
GDN_API int gdn_linear_q4(gdn_pool* pool, int32_t n_tokens, int32_t n_out, int32_t n_in, const gdn_bf16* x,
                          int64_t ld_x, const void* w_q4_tiles, gdn_bf16* y, int64_t ld_y, void* stream);

/* A whole mixer layer (GatedDeltaNet::forward_with_cache, qwen3_5.rs:559-669):
 * y = out_proj(gdn_layer_step(in_proj(x))) over a packed ragged batch.
 * x [n_tokens][ld_x], y [n_tokens][ld_y] bf16, hidden columns.  The projections run as
 * gdn_mixer_weights says: 4-bit tiles on the weight-streaming kernel (or expanded to bf16 for
 * cuBLASLt, see above), bf16 tiles on it for calls of at most 64 tokens, otherwise cuBLASLt
 * (library GEMM), all with f32 accumulation.
 * Asynchronous. */
GDN_API int gdn_mixer_step(gdn_pool* pool, int32_t layer, const gdn_mixer_weights* w, const gdn_bf16* x,
                           int64_t ld_x, gdn_bf16* y, int64_t ld_y, const int32_t* slot_ids,
                           const int32_t* cu_seqlens, int32_t n_seq, int32_t n_tokens, void* stream);

/* The residual GDN stack: for l = 0 .. n_layers-1,
 *   h <- h + mixer_l(rms_norm(h, layers[l].pre_norm_w, rms_norm_eps))
 * (the decoder layer of qwen3_5.rs:729-739 restricted to its mixer), in place on
 * h [n_tokens][ld_h] bf16.  layers: n_layers entries (host array of device pointers). */
GDN_API int gdn_stack_step(gdn_pool* pool, const gdn_mixer_weights* layers, gdn_bf16* h, int64_t ld_h,
                           const int32_t* slot_ids, const int32_t* cu_seqlens, int32_t n_seq, int32_t n_tokens,
                           void* stream);

/* The gated delta recurrence alone on pool state (metal_gdn.rs:10-67), packed
 * and ragged: q,k [N][Hk][dk] bf16, v [N][Hv][dv] bf16, g [N][Hv] f32,
 * beta [N][Hv] bf16 -> y [N][Hv][dv] bf16; state of slot_ids[i] updated in place. */
GDN_API int gdn_recurrence(gdn_pool* pool, int32_t layer, const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v,
                   const float* g, const gdn_bf16* beta, const int32_t* slot_ids, const int32_t* cu_seqlens,
                   int32_t n_seq, int32_t n_tokens, gdn_bf16* y, void* stream);

/* Reference-shaped recurrence: the argument meaning of gated_delta_kernel
 * (metal_gdn.rs:170-173).  q,k [B,T,Hk,dk], v [B,T,Hv,dv], g [B,T,Hv] f32,
 * beta [B,T,Hv] bf16, state_in [B,Hv,dv,dk] f32 -> y [B,T,Hv,dv] bf16 and
 * state_out [B,Hv,dv,dk] f32.  state_out may equal state_in (in place) or be a
 * separate buffer (the reference's functional form).  Device pointers. */
GDN_API int gdn_gated_delta_kernel(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v, const float* g,
                           const gdn_bf16* beta, const float* state_in, int32_t seq_len, int32_t batch, int32_t hk,
                           int32_t hv, int32_t dk, int32_t dv, gdn_bf16* y, float* state_out, void* stream);

/* beta and g alone (compiled_beta_g, compiled_ops.rs:68-94): ab [N][ld_ab] (b | a)
 * -> beta [N][Hv] bf16, g [N][Hv] f32.  Device pointers. */
GDN_API int gdn_beta_g(const gdn_bf16* ab, int64_t ld_ab, int32_t n_tokens, int32_t hv, const float* A_log,
               const float* dt_bias, gdn_bf16* beta, float* g, void* stream);

/* gdn_beta_g for a dt_bias stored in bf16 (dt_bias_bf16 != 0, see gdn_layer_weights): the same
 * closure (compiled_ops.rs:12-49) with a + dt_bias and its exp rounded to bf16. */
GDN_API int gdn_beta_g_ex(const gdn_bf16* ab, int64_t ld_ab, int32_t n_tokens, int32_t hv, const float* A_log,
                          const float* dt_bias, int32_t dt_bias_bf16, gdn_bf16* beta, float* g, void* stream);

/* Which kernel runs decode-only calls (n_tokens == n_seq) of gdn_layer_step and the entry points
 * built on it: 0 (default) by batch size -- fewer than 64 sequences the split kernel (each
 * (sequence, v-head) state tile split by dv rows over 4 CTAs of a cluster; Hv/Hk <= 2), 64 or
 * more the fused one-kernel step; 1 always the split kernel; 2 always the fused kernel; 3 the
 * two-kernel step (prep, then recurrence).  Results agree within f32 rounding.  Process-wide;
 * set it before capturing graphs.  (A tuning and test control of this library; the reference
 * has one kernel, metal_gdn.rs:170-218.) */
GDN_API int gdn_set_decode_kernel(int mode);

/* Failure-detection tests only (no counterpart in the reference).  Shortens the bound of the split
 * kernel's state wait to `wait_ns` and makes CTA `skip_block` of it arm its barrier without
 * issuing the copy, so that wait runs out: the kernel records 1 << 7 in the pool's error word
 * (gdn_pool_check), leaves that CTA's 32 state rows and outputs unwritten and returns.
 * gdn_test_set_wait_fault(-1, 2000000000) restores normal operation.  Process-wide. */
GDN_API int gdn_test_set_wait_fault(int32_t skip_block, int64_t wait_ns);

/* ------------------------------------------------------- no-allocation variant
 * No counterpart in the reference.  The fused layer step of gdn_layer_step for
 * callers that may not allocate device memory -- e.g. an engine that reserves a
 * fixed device arena at start-up and forbids cudaMalloc afterwards, or a host
 * framework whose caching allocator owns all device memory.  The caller passes
 * the state of ONE layer in memory it owns: rec_state [n_slots][Hv][dv][dk] f32
 * (16-byte aligned) and conv_state [n_slots][K-1][D] bf16, plus the same weights,
 * step buffers and DEVICE routing tables as gdn_layer_step.  The step's scratch
 * comes from a fixed array compiled into this library (4,259,840 bytes on every
 * device that loads it, kept until exit): at most 4096 records, i.e.
 * n_tokens * n_v_heads <= 4096 (128 tokens per call at 32 v-heads); larger calls
 * return GDN_E_INVALID.  This function never allocates.  Its first call on a
 * device looks up the scratch's device address; make that first call before
 * capturing a stream into a CUDA graph.  All calls share the scratch, so calls
 * that overlap on the GPU (other streams or threads) race: serialise them.
 * Asynchronous on `stream`.  The kernels' bounds checks and bounded waits record
 * failures in an error word inside the same array (read it with gdn_noalloc_check);
 * validate the tables with gdn_validate_tables before the call. */
GDN_API int gdn_layer_step_noalloc(const gdn_config* cfg, int32_t n_slots, float* rec_state, gdn_bf16* conv_state,
                                   const gdn_layer_weights* w, const gdn_step_io* io, const int32_t* slot_ids,
                                   const int32_t* cu_seqlens, int32_t n_seq, int32_t n_tokens, void* stream);

/* No counterpart in the reference.  The device error word of gdn_layer_step_noalloc on the
 * current device: bits (1 << GDN_E_BAD_SLOT) / (1 << GDN_E_BAD_SEQLENS) when a kernel skipped a
 * sequence whose slot or token range failed its bounds check, (1 << 7) when a bounded device
 * wait gave up.  A call that set a bit returned GDN_OK, but its outputs and the states it
 * touched are not to be trusted.  Synchronous (waits for the device); clears the word when
 * `reset` is non-zero.  Allocates nothing.  The word is shared by every no-alloc call on the
 * device and keeps its bits until cleared. */
GDN_API int gdn_noalloc_check(int32_t* flags, int reset);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_H */
