/*
 * gdn_hybrid.h -- C ABI of the other two layer kinds of the hybrid Qwen3.5 decoder, so that a
 * continuously batched step can run every layer of the model on this library:
 *
 *   - the full-attention mixer body between its projections (Qwen35Attention::forward_with_cache,
 *     src/models/qwen3_5.rs:377-459): q/k RMSNorm, partial RoPE, the per-sequence KV cache,
 *     scaled dot-product attention and the sigmoid output gate.  The reference's batched executor
 *     stacks ragged KV caches by zero padding and runs SDPA without a mask
 *     (src/scheduler/mlx_executor.rs:57-86), so padded keys take softmax weight; here each token
 *     attends to exactly the keys of its own sequence up to its own position.
 *   - the sparse MoE block (SparseMoeBlock::forward, src/models/qwen3_5.rs:262-302): router
 *     softmax, top-k selection and renormalisation, the selected MLX 4-bit experts
 *     (SwitchMlp::forward, :127-160, gather_qmm with group 64), silu(gate) * up
 *     (compiled_ops.rs:99-143), and the sigmoid-gated shared expert (:218-228, :296-300).
 *
 * Conventions are those of gdn.h: bf16 as uint16_t bit patterns, GDN_OK / GDN_E_* return codes,
 * gdn_last_error() for the message, `stream` a cudaStream_t as void*.  Tensors are DEVICE
 * pointers; the routing tables of gdn_attn_step are HOST arrays (they size the launch).
 */
#ifndef GDN_B200_HYBRID_H
#define GDN_B200_HYBRID_H

#include "gdn.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- full attention */

/* Attention shapes: the attention fields of Qwen35Config (qwen3_5.rs:30-45) and the KV-cache capacity. */
typedef struct gdn_attn_config {
    int32_t n_heads;      /* num_attention_heads (16) */
    int32_t n_kv_heads;   /* num_key_value_heads (2); n_heads / n_kv_heads <= 16 */
    int32_t head_dim;     /* head_dim: 64, 128 or 256 */
    int32_t rotary_dim;   /* head_dim * partial_rotary_factor (64): even, <= head_dim */
    float rope_theta;     /* rope_theta (1e7) */
    float rms_norm_eps;   /* rms_norm_eps of q_norm / k_norm */
    int32_t max_ctx;      /* positions per slot in the KV cache */
} gdn_attn_config;

/* Workspace bytes of one gdn_attn_step over `n_tokens` packed tokens whose longest context (cached
 * keys + own tokens) is `max_kv_len`.  Needs no GPU. */
GDN_API int gdn_attn_workspace_bytes(const gdn_attn_config* cfg, int32_t n_tokens, int32_t max_kv_len,
                                     int64_t* bytes);

/* One attention layer body over a packed ragged batch.  Sequence i owns tokens
 * [cu_seqlens[i], cu_seqlens[i+1]), KV-cache slot slot_ids[i], and has positions[i] keys cached;
 * its token j is at position positions[i] + j.  For every token:
 *   q, gate = q_full row split per head [q (hd) | gate (hd)]        (qwen3_5.rs:387-391)
 *   q = rope(rms_norm(q, q_norm_w)), k = rope(rms_norm(k, k_norm_w)) (:393-416; first rotary_dim dims,
 *       rotate-half pairing, angle = position * rope_theta^(-2i/rotary_dim))
 *   k, v written to the cache at the token's position                (:419-424)
 *   o = softmax(q k^T / sqrt(hd)) v over keys [0, position]          (:427-449; GQA groups of n_heads/n_kv_heads)
 *   out = o * sigmoid(gate)                                          (:455-456)
 * q_full [N][2*nh*hd], k_in / v_in [N][nkv*hd], out [N][nh*hd] (input of o_proj), q_norm_w / k_norm_w [hd];
 * k_cache / v_cache [n_slots][nkv][max_ctx][hd] bf16.  slot_ids, cu_seqlens, positions: HOST arrays,
 * checked (slots in range and distinct, positions[i] + tokens <= max_ctx).  The workspace holds
 * gdn_attn_workspace_bytes(cfg, N, max over i of positions[i] + tokens_i) bytes.  The per-token
 * (slot, position) table is copied into the workspace from host memory during the call, and that
 * copy waits for the work already queued on `stream`; the kernels then run asynchronously.  Not
 * capturable in a CUDA graph for that reason. */
GDN_API int gdn_attn_step(const gdn_attn_config* cfg, const gdn_bf16* q_full, const gdn_bf16* k_in,
                          const gdn_bf16* v_in, const gdn_bf16* q_norm_w, const gdn_bf16* k_norm_w,
                          gdn_bf16* k_cache, gdn_bf16* v_cache, int32_t n_slots, const int32_t* slot_ids,
                          const int32_t* cu_seqlens, const int32_t* positions, int32_t n_seq, int32_t n_tokens,
                          gdn_bf16* out, void* workspace, int64_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- sparse MoE */

/* MoE shapes: the MoE fields of Qwen35Config (qwen3_5.rs:55-63). */
typedef struct gdn_moe_config {
    int32_t hidden;          /* hidden_size: multiple of 64 */
    int32_t n_experts;       /* num_experts (256); <= 1024 */
    int32_t top_k;           /* num_experts_per_tok (8); <= 16 */
    int32_t moe_inter;       /* moe_intermediate_size (512): multiple of 64 */
    int32_t shared_inter;    /* shared_expert_intermediate_size (512): multiple of 64 */
    int32_t norm_topk_prob;  /* norm_topk_prob */
} gdn_moe_config;

/* One MLX affine 4-bit matrix [rows][cols], groups of 64 columns: w = scale * q + bias, q = bits
 * 4*(c%8) of word c/8 of the row (the checkpoint's weight / scales / biases, qwen3_5.rs:929-935). */
typedef struct gdn_q4_matrix {
    const uint32_t* q;        /* [rows][cols/8] */
    const gdn_bf16* scales;   /* [rows][cols/64] */
    const gdn_bf16* biases;   /* [rows][cols/64] */
} gdn_q4_matrix;

/* The MoE block's parameters (SparseMoeBlock fields, qwen3_5.rs:232-248).  Experts are stacked by
 * expert as in the checkpoint's switch_mlp tensors: gate / up [E][moe_inter][hidden], down
 * [E][hidden][moe_inter].  router: mlp.gate as bf16 [E][hidden]; shared_gate: shared_expert_gate as
 * bf16 [hidden]. */
typedef struct gdn_moe_weights {
    const gdn_bf16* router;
    gdn_q4_matrix gate, up, down;
    gdn_q4_matrix sh_gate, sh_up, sh_down;   /* [shared_inter][hidden], [hidden][shared_inter] */
    const gdn_bf16* shared_gate;
} gdn_moe_weights;

GDN_API int gdn_moe_workspace_bytes(const gdn_moe_config* cfg, int32_t n_tokens, int64_t* bytes);

/* Routing only (qwen3_5.rs:268-284): logits = x router^T (bf16), p = softmax(logits) (bf16), the top_k
 * experts by p (descending, lower index first among equal p), their p renormalised to sum 1 when
 * norm_topk_prob.  x [N][hidden]; logits [N][E] (may be NULL), ids [N][top_k] int32, weights
 * [N][top_k] bf16.  Asynchronous. */
GDN_API int gdn_moe_route(const gdn_moe_config* cfg, const gdn_moe_weights* w, const gdn_bf16* x, int32_t n_tokens,
                          gdn_bf16* logits, int32_t* ids, gdn_bf16* weights, void* stream);

/* The whole MoE block: out = sum_j weight_j * expert_{id_j}(x) + sigmoid(x . shared_gate) * shared(x),
 * expert(x) = down(silu(gate x) * up x).  When `route_ids` / `route_weights` are non-NULL they are
 * used as the routing (e.g. from gdn_moe_route) and the router is not run.  Asynchronous. */
GDN_API int gdn_moe_step(const gdn_moe_config* cfg, const gdn_moe_weights* w, const gdn_bf16* x, int32_t n_tokens,
                         const int32_t* route_ids, const gdn_bf16* route_weights, gdn_bf16* out, void* workspace,
                         int64_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_HYBRID_H */
