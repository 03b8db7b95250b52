// gdn_internal.h -- kernel argument blocks and launchers shared between the
// kernels (.cu) and the C ABI implementation (gdn_api.cu).  Not installed.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {

// Head dimensions the kernels are specialised for (checked at the ABI).
constexpr int DK_ABI = 128;
constexpr int DV_ABI = 128;

// Arguments of the stand-alone recurrence kernel.  Pointers are device pointers.
struct StepArgs {
    // state (one layer's slice of the pool, or dense [B] arrays for the functional form)
    float* rec;            // [n_slots][Hv][DV][DK] f32, written
    const float* rec_in;   // read from here when non-null (functional form), else from rec
    // routing
    const int32_t* slot_ids;    // [n_seq]; null: slot = sequence index
    const int32_t* cu_seqlens;  // [n_seq+1]; null: T_dense tokens per sequence
    int32_t n_seq, n_slots, T_dense, n_tokens;
    int32_t hk, hv;
    // inputs / output
    const uint16_t* q;
    const uint16_t* k;
    const uint16_t* v;
    const float* g;
    const uint16_t* beta;
    uint16_t* y;
    // device error word (atomicOr of 1 << GDN_E_*)
    int32_t* err;
};

// Per-(v-head, token) record written by the prep kernel and streamed by the
// recurrence kernels: q | k | v | silu(z) (bf16 x 128 each) | g f32 | beta f32 | log g f32 | pad (20 bytes).
// 33 DRAM sectors of 32 bytes, so every field starts on a sector and no store covers part of one (a partly
// written sector costs the memory a read-modify-write).
constexpr int REC_BYTES = 1056;
static_assert(REC_BYTES % 32 == 0, "records sector-aligned");
constexpr int REC_PER_STAGE = 4;   // token records staged with each state tile

struct PrepArgs {
    const uint16_t* qkv; long long ld_qkv;
    const uint16_t* z; long long ld_z;
    const uint16_t* ab; long long ld_ab;
    uint16_t* conv;              // layer slice of the conv-state pool [n_slots][KC-1][D]
    const uint16_t* conv_w;
    const float* A_log;
    const float* dt_bias;
    const int32_t* slot_ids;
    const int32_t* cu_seqlens;
    int32_t n_seq, n_slots, n_tokens;
    int32_t hk, hv, D;
    uint8_t* rec;                // scratch records [Hv][rec_cap][REC_BYTES]
    long long rec_cap;
    int32_t* err;
    int32_t tables_stable;       // routing tables and this layer's conv state may be read before the PDL wait
    int32_t dt_bf16;             // dt_bias is a bf16 parameter: a + dt_bias and its exp round to bf16 (gate_softplus)
    int32_t z_skip_min_t;        // > 0: tokens of segments at least this long get no silu(z) record (the chunked
                                 // pass reads z itself); honoured by gdn_prep_vec_kernel, the others write it anyway
};

struct RecurArgs {
    float* rec;                  // state written here [n_slots][Hv][DV][DK]
    const float* rec_in;         // read from here when non-null, else from rec
    uint16_t* conv;              // conv-state pool slice (windows written back)
    const uint16_t* qkv; long long ld_qkv;
    const uint8_t* recs;
    long long rec_cap;
    const uint16_t* norm_w;
    float eps;
    uint16_t* out; long long ld_out;
    const int32_t* slot_ids;
    const int32_t* cu_seqlens;
    int32_t n_seq, n_slots, n_tokens;
    int32_t hk, hv, D;
    int32_t* err;
    const uint16_t* z;           // non-null: the chunked kernel reads z [n_tokens][ld_z] and applies SiLU itself
    long long ld_z;              // (wy_z_direct), else it reads silu(z) from the records
    int32_t wy_min_t;            // > 0: segments of at least this many tokens go to the chunked kernel
    int32_t* wy_counter;         // chunked kernel's work-ticket counter (zeroed by the plan kernel)
    uint8_t* wy_tiles;           // per (chunk, v-head) tile sets of the chunk-parallel pass [wy_cap_chunks][Hv][48 KiB]
    long long wy_cap_chunks;     // chunks the tile scratch holds
    int32_t* wy_cb;              // [n_seq] chunk prefix per sequence (plan kernel)
    int2* wy_chunks;             // [wy_cap_chunks] (first token row, tokens) of every chunk (plan kernel)
    int32_t* wy_plan;            // [0] chunks, [1] qualifying sequences, [2..] them longest first
};

// Sequences the plan kernel ranks longest first (more run in call order); tile set per (chunk, v-head).
constexpr int WY_SORT_CAP = 1024;
constexpr int WY_TILESET_BYTES = 6 * 8192;
constexpr int WY_PLAN_INTS = 2 + WY_SORT_CAP;

// Sequences of at least this many tokens in one call run the chunked (WY) tensor-core kernel.
constexpr int WY_MIN_T = 32;

// The chunked kernel can load z rows by TMA straight from the caller's tensor: 16-byte aligned base and rows.
inline bool wy_z_direct(const void* z, long long ld_z) {
    return z != nullptr && (reinterpret_cast<uintptr_t>(z) & 15u) == 0 && ld_z > 0 && ld_z % 8 == 0;
}

cudaError_t launch_wy(const RecurArgs& r, cudaStream_t stream);
cudaError_t launch_layer_step_v2(const PrepArgs& p, const RecurArgs& r, cudaStream_t stream);
// Decode-only calls (n_tokens == n_seq) with at least FUSED_MIN_SEQ sequences: prep and recurrence in
// one persistent kernel (gdn_fused.cu).
constexpr int FUSED_MIN_SEQ = 64;
cudaError_t launch_decode_fused(const PrepArgs& p, const RecurArgs& r, cudaStream_t stream);
// Decode-only calls of few sequences, Hv/Hk <= 2: each (sequence, v-head) tile split by dv rows over 4 CTAs of a
// cluster (gdn_split.cu).
struct SplitCtl {
    unsigned long long wait_ns;  // bound of the state-slice wait (2 s; shortened only by failure-detection tests)
    int skip_block;              // failure-detection tests: this CTA's state copy is never issued (-1: none)
};
cudaError_t launch_decode_split(const PrepArgs& p, const RecurArgs& r, const SplitCtl& ctl, cudaStream_t stream);
// Which decode-only kernel launch_layer_step_v2 uses (gdn_set_decode_kernel): 0 by batch size, 1 split, 2 fused
// (>= 1 sequence), 3 the two-kernel step.
extern int g_decode_kernel;
// Sequences below which decode-only calls take the split kernel (by-batch-size selection).
constexpr int SPLIT_MAX_SEQ = 8;
extern SplitCtl g_split_ctl;

// Projections and the decoder pre-norm / residual (gdn_proj.cu).
struct GemmCtx;
GemmCtx* gemm_create(void* workspace, size_t ws_bytes);
void gemm_destroy(GemmCtx* g);
int gemm_bf16_nt(GemmCtx* g, int M, int N, int K, const uint16_t* x, long long ldx, const uint16_t* w,
                 uint16_t* out, long long ldo, cudaStream_t stream);
cudaError_t launch_add_rmsnorm(const uint16_t* h_in, long long ld_h, const uint16_t* o, long long ld_o,
                               uint16_t* h_out, const uint16_t* w, uint16_t* hn, long long ld_hn, int rows, int H,
                               float eps, cudaStream_t stream);

// Weight-streaming projection GEMM for calls of at most WG_MAX_M tokens on a tiled weight
// (gdn_wgemm.cu): y[m][n] = bf16(sum_k x[m][k] w[n][k]).  x rows 16-byte aligned (ldx % 8 == 0,
// K % 8 == 0; K % 64 == 0 for 4-bit tiles); ws holds wg_workspace_floats(n_sm) floats, cnt one
// zeroed int per 128 rows of w.
constexpr int WG_MAX_M = 64;
struct WgGemm {
    const uint8_t* tiles;        // bf16 tiles (wg_tile_bytes) or 4-bit tiles (wq_tile_bytes)
    bool q4;
    const uint16_t* x; long long ldx;
    uint16_t* y; long long ldy;
    int M, N, K;
    int n_sm;
    float* ws;
    int* cnt;
    int* err;
};
long long wg_tile_bytes(int N, int K);
long long wq_tile_bytes(int N, int K);
long long wg_workspace_floats(int n_sm);
int wg_num_slabs(int NRG, int n_sm);  // row slabs of the weight-streaming GEMM (one arrival counter each)
cudaError_t launch_wg_tile(const uint16_t* w, int N, int K, uint8_t* tiles, cudaStream_t stream);
cudaError_t launch_wq_tile(const uint32_t* wq, const uint16_t* scales, const uint16_t* biases, int N, int K,
                           uint8_t* tiles, cudaStream_t stream);
cudaError_t launch_wg_gemm(const WgGemm& g, cudaStream_t stream);
// Tiled TMA tensor map over a row-major bf16 matrix [rows][cols] (row stride ld_bytes, a multiple of 16; base
// 16-byte aligned): box of box_cols (<= 64) x box_rows with 128-byte swizzle, out-of-range elements read as zero.
// False when the driver's encoder is unavailable or rejects the arguments (gdn_tmap.cu).
bool tmap_bf16_2d_sw128(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t ld_bytes,
                        uint32_t box_cols, uint32_t box_rows);
// TMA tensor map over the token records [n_heads][rec_cap][rec_bytes] as 4-D u16 elements (e: 8 per 16-byte
// chunk, t: token row < n_tokens, c: 16-byte chunk of the record, h: head), box {8, box_tokens, box_chunks, 1}:
// a box lands as offset(t, c, e) = c * box_tokens * 16 + t * 16 + e * 2, the no-swizzle core-matrix layout with
// token rows 16 bytes apart; rows >= n_tokens read as zero (gdn_tmap.cu).
bool tmap_records(CUtensorMap* map, const void* recs, int n_tokens, long long rec_cap, int n_heads, int rec_bytes,
                  uint32_t box_tokens, uint32_t box_chunks);
// The 4-bit projection for calls of at most 16 tokens with the dequantized weight in tensor memory
// (gdn_wq16.cu); same arguments as launch_wg_gemm (q4 tiles).
bool wq16_supported(int M, int N, int K);
cudaError_t launch_wq16(const WgGemm& g, cudaStream_t stream);
// bf16 tiles (wg_tile_bytes layout, K % 64 == 0), at most 16 tokens: the weight streamed by bulk copy into a
// ring of shared-memory stages that the MMA reads as its A operand (gdn_wq16.cu).  cudaErrorNotSupported when a
// split's tokens do not fit in shared memory.
bool wb16_supported(int M, int N, int K);
cudaError_t launch_wb16(const WgGemm& g, cudaStream_t stream);
// 4-bit tiles (wq_tile_bytes layout, K % 64 == 0) -> row-major bf16 weight w [N][K], 16-byte aligned.
cudaError_t launch_wq_untile(const void* tiles, int N, int K, uint16_t* w, cudaStream_t stream);

// Set the calling thread's gdn_last_error() message and return `code` / GDN_OK.
int record_error(int code, const char* msg);
int record_ok();
cudaError_t launch_recurrence(const StepArgs& a, cudaStream_t stream);
cudaError_t launch_beta_g(const uint16_t* ab, long long ld_ab, int n_tokens, int hv, const float* A_log,
                          const float* dt_bias, int dt_bf16, uint16_t* beta, float* g, cudaStream_t stream);

}  // namespace gdn
