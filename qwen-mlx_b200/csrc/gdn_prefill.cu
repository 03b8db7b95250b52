// gdn_prefill.cu -- chunked (WY) gated delta rule on tcgen05 tensor cores for the
// multi-token sequences of a packed step (sm_100a).
//
// The recurrence of metal_gdn.rs:37-62, S_t = g_t S_{t-1} + d_t k_t^T with
// d_t = beta_t (v_t - g_t S_{t-1} k_t) and y_t = S_t q_t, is evaluated 64 tokens
// at a time.  With lg_t = sum_{j<=t} log g_j inside the chunk, gamma_t = exp(lg_t)
// and S0 the state entering the chunk:
//   G = K K^T, QK = Q K^T                                (tensor cores, exact bf16 inputs)
//   M[t][s] = beta_t exp(lg_t - lg_s) G[t][s]  (s < t),  T = (I + M)^-1   (CUDA cores, blocked)
//   U = T diag(beta) V,  W = T diag(beta gamma) K          (tensor cores)
//   D = U - W S0^T                                        (accumulated onto U in TMEM)
//   Y = diag(gamma) Q S0^T + P (.) QK D,  P[t][s] = exp(lg_t - lg_s) (s <= t)
//   S_C = gamma_C S0 + D^T diag(exp(lg_C - lg_s)) K
// f32 operands (T beta, T beta gamma, W, S0, D, P (.) QK) enter the bf16 MMAs as hi + lo bf16
// pairs (hi = bf16(x), lo = bf16(x - hi)); products of two split operands drop lo*lo.  Decays
// stay in log space, so long chunks of strong decay cannot underflow into 0/0.
//
// Everything up to T beta, T beta gamma and P (.) QK depends only on the chunk's own inputs, so it
// is computed for every chunk at once; only D, Y and the state update need the state entering the
// chunk.  A call with long segments runs three kernels after the prep:
//   gdn_wy_plan_kernel   (one CTA) numbers the chunks of the qualifying segments (an exclusive
//                        prefix over the sequences), ranks the sequences longest first, and zeroes
//                        the sequential kernel's work ticket;
//   gdn_wy_chunk_kernel  (chunk-parallel, 2 CTAs per SM, work item = (chunk, k-head)): G and QK of
//                        the k-head once, then for each of its v-heads (two at a time, one per warp
//                        group) M, the blocked inverse
//                        T = (I + M)^-1 and the tiles T beta, T beta gamma and P (.) QK as hi / lo
//                        bf16 pairs, stored to global memory in the exact shared-memory layout the
//                        sequential kernel multiplies from (48 KiB per chunk and v-head);
//   gdn_wy_kernel        (sequential, one CTA per SM, work item = (sequence, v-head), longest
//                        chains first): per chunk one bulk copy brings the chunk's tiles, then
//                        U, W, D, Q S0^T, P D and the state update on the tensor cores, and the
//                        epilogue rounds y to bf16 (metal_gdn.rs:54) and applies
//                        silu(z) * rms_norm(y, norm_w, eps) (qwen3_5.rs:660-665).
// The f32 state S lives in TMEM for the whole sequence: each chunk scales it by gamma_C in place and
// the state-update MMA accumulates onto it.
//
// Every operand tile is stored token-major ([t][d], [t][v], [s][v]) in the core-matrix layout of
// gdn_umma.cuh and read K-major or MN-major as each product needs, so no tile is ever transposed and
// every shared-memory store is a 16-byte vector.  Every product is an M = 128 MMA whose 128 rows are
// v, d or [Q; K] stacked, so every TMEM lane carries data: G and QK come out of one [Q; K] K^T
// product, and U, W, D, Q S0^T and P D are formed transposed (U^T = V^T (T beta)^T,
// W^T = K^T (T beta gamma)^T, D^T = U^T - S0 W^T, (Q S0^T)^T = S0 Q^T, (P D)^T = D^T P^T).
//
// Shared memory of gdn_wy_kernel (bytes):
//   R_QK  64K  [Q [64 t][128 d] | K [64 s][128 d]] x 2 (chunk parity), token-major TMA boxes
//   R_V   16K  V [64 s][128 v], token-major TMA box
//   R_Z   32K  z [64 t][128 v] x 2 (chunk parity), token-major TMA boxes for the epilogue: raw rows of the
//              caller's z (turned into silu(z) in place by the compute warps while the chunk's D runs) or
//              silu(z) from the records when z rows are not 16-byte aligned
//   R_T   17K  y [64 t][128 v] bf16 (row stride LDY), the epilogue's transpose
//   R_TB  32K  (T beta) hi, lo; (T beta gamma) hi, lo [64 t][64 s] (bulk copy) -> -W^T hi, -W^T lo [128 d][64 t]
//   R_P   16K  (P (.) QK) hi, lo [64 t][64 s] (same bulk copy)
// TMEM (cta_group::1, all 128 lanes): S [0,128) = state [v][d]; U [192,256) = U^T then D^T;
// W [256,320) = W^T; QS [320,384) = (Q S0^T)^T; PD [384,448) = (P D)^T; the hi/lo A operands of Q S0^T, D,
// P D and the state update (S0, then D^T and Dd^T) in [128,192) and [448,512).
#include "gdn_device.cuh"
#include "gdn_internal.h"
#include "gdn_ptx.cuh"
#include "gdn_umma.cuh"

namespace gdn {

constexpr int WC = 64;                 // tokens per chunk
constexpr int WY_THREADS = 256;       // compute threads of the sequential pass (and of the chunk pass)
constexpr int WY_ISSUER_WARP = WY_THREADS / 32;        // the sequential pass: warp 8 issues the MMAs,
constexpr int WY_EPI_WARP = WY_ISSUER_WARP + 1;         // warps 9 and 10 run the per-token epilogue
constexpr int WY_EPI_THREADS = 64;
constexpr int WY_BLOCK = WY_THREADS + 32 + WY_EPI_THREADS;
constexpr int LDT = 68;                // padded f32 row stride of M / T (conflict-free float4 rows)
constexpr int R_QK = 0, R_V = 65536, R_Z = 81920, R_T = 147456, R_N = R_T + WC * LDT * 4, R_TB = 172032,
              R_P = 204800, R_SMALL = 221184;
static_assert(R_N + 6 * 256 * 4 <= R_TB, "prefill shared memory layout");
static_assert(R_P == R_TB + 32768, "the chunk tile set lands in one bulk copy");
static_assert(R_Z + 2 * 16384 <= R_T, "two silu(z) boxes");
constexpr int LDY = DV + 8;            // padded bf16 row stride of the y transpose (rows 272 B apart)
static_assert(WC * LDY * 2 <= WC * LDT * 4, "y transpose fits the T region");
constexpr int SMALL_FLOATS = 3 * 2 * 64 + 128;
constexpr int R_G = ((R_SMALL + SMALL_FLOATS * 4 + 192 + 1023) / 1024) * 1024;   // gate boxes [2][64 t][16 B]
constexpr int WY_SMEM = R_G + 2 * WC * 16;
static_assert(WY_SMEM <= 232448, "prefill shared memory budget");
constexpr uint32_t TM_S = 0, TM_U = 192, TM_W = 256, TM_QS = 320, TM_PD = 384;
// A operands of the sequential pass in tensor memory (row v = lane, two bf16 per column): S0 hi [128, 192) and lo
// [448, 512) from the state split until Q S0^T and D have read them, then D hi [128, 160), D lo [160, 192),
// Dd hi [448, 480), Dd lo [480, 512)
constexpr uint32_t TM_AH = 128, TM_AL = 448;
constexpr uint64_t WY_WAIT_NS = 2000000000ull;
constexpr uint32_t TILESET = WY_TILESET_BYTES;   // T beta hi, lo | T beta gamma hi, lo | P (.) QK hi, lo
static_assert(TILESET == 6 * 8192, "tile set layout");

// gdn_wy_chunk_kernel shared memory: two Q | K buffers (the next item's copies land in the other one; once the
// item's [Q; K] K^T has been taken, its buffer holds the warp groups' N blocks), per warp group M / T (f32), per
// v-head gates (up to 8 heads; beta and log g of the item and of the next one)
constexpr int A_QKB = 32768;                  // one Q | K buffer
constexpr int A_NB = 6 * 256 * 4;             // one warp group's N blocks
static_assert(2 * A_NB <= A_QKB, "both groups' N blocks fit a consumed Q | K buffer");
constexpr int A_TN = WC * LDT * 4;
constexpr int A_QK = 0, A_T = 2 * A_QKB, A_SMALL = A_T + 2 * A_TN;
constexpr int A_SMEM = A_SMALL + 7 * 8 * WC * 4 + 32;
static_assert(2 * (A_SMEM + 1024) <= 233472, "two chunk-pass CTAs per SM");
constexpr int WA_THREADS = 256;
constexpr int WP_THREADS = 1024;

__device__ __forceinline__ uint32_t pack_bf2(float lo_half, float hi_half) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo_half, hi_half);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// hi = bf16(x), lo = bf16(x - hi) for 8 consecutive values, packed as two 16-byte vectors.
__device__ __forceinline__ void split8(const float* x, uint4& hi, uint4& lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        h[i] = pack_bf2(x[2 * i], x[2 * i + 1]);
        l[i] = pack_bf2(x[2 * i] - __uint_as_float(h[i] << 16), x[2 * i + 1] - __uint_as_float(h[i] & 0xFFFF0000u));
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// split8 on f32 pairs (the same bits: hi and x - hi rounded per lane as the scalar form does).
__device__ __forceinline__ void split8_f2(const uint64_t* x, uint4& hi, uint4& lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        h[i] = f2_to_bf2(x[i]);
        l[i] = f2_to_bf2(f2_sub(x[i], bf2_to_f2(h[i])));
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}
__device__ __forceinline__ uint64_t f2_of(const uint32_t* r) { return f2_pack(__uint_as_float(r[0]), __uint_as_float(r[1])); }

// 16-byte vector at row r, column group c8 (8 columns) of a [rows][COLS] bf16 tile.
template <int COLS>
__device__ __forceinline__ void st_tile(uint8_t* base, int r, int c8, const uint4& v) {
    *reinterpret_cast<uint4*>(base + (r >> 3) * (COLS / 8) * 128 + c8 * 128 + (r & 7) * 16) = v;
}

// Rows [0, 64) of one 256-byte record field into a [64][128] tile; rows >= nv zero-filled.
// Eight consecutive lanes take eight consecutive rows of one 16-byte column group, so the
// shared-memory writes of a quarter-warp hit distinct banks and each row's 32-byte sector
// is read by one instruction.
__device__ __forceinline__ void load_field(uint32_t dst, const uint8_t* rec0, int field, int nv, int tid) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int idx = tid + i * WY_THREADS;
        const int t = (idx & 7) | ((idx >> 7) << 3), ch = (idx >> 3) & 15;
        const bool ok = t < nv;
        const uint8_t* src = rec0 + (ok ? (size_t)t * REC_BYTES + field + ch * 16 : 0);
        cp_async16(dst + umma_tile_off(t, ch * 8, 128), src, ok ? 16u : 0u);
    }
}

// beta and log g of the chunk's tokens (zero for rows >= nv).
__device__ __forceinline__ void load_gates(float* s_beta, float* s_lgr, const uint8_t* rec0, int nv, int tid) {
    if (tid < 2 * WC) {
        const int t = tid & (WC - 1);
        const bool ok = t < nv;
        float* dst = tid < WC ? s_beta + t : s_lgr + t;
        const uint8_t* src = rec0 + (ok ? (size_t)t * REC_BYTES + (tid < WC ? 1028 : 1032) : 0);
        cp_async4(smem_u32(dst), src, ok ? 4u : 0u);
    }
}

// Wait for the MMAs committed to `bar` (phase `ph`); false on timeout.
__device__ __forceinline__ bool wy_wait(uint64_t* bar, uint32_t& ph) {
    const bool ok = mbar_wait_bounded(bar, ph, WY_WAIT_NS);
    ph ^= 1u;
    tc_fence_after();
    return ok;
}

// Make generic-proxy shared-memory writes and TMEM stores of all threads visible to the
// next MMA issue, and every thread's earlier TMEM loads complete before it.
__device__ __forceinline__ void wy_sync_for_mma() {
    fence_async_shared();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
}

// Inclusive scan of one chunk's log g (log2 units), gamma_t = exp(lg_t) and exp(lg_last - lg_t) (one warp;
// lane holds tokens lane and 32 + lane).
__device__ __forceinline__ void wy_scan_core(float x0, float x1, float* lg, float* gam, float* tail, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float y0 = __shfl_up_sync(0xffffffffu, x0, o);
        const float y1 = __shfl_up_sync(0xffffffffu, x1, o);
        if (lane >= o) { x0 += y0; x1 += y1; }
    }
    x1 += __shfl_sync(0xffffffffu, x0, 31);
    const float kLog2e = 1.4426950408889634f;
    x0 *= kLog2e;
    x1 *= kLog2e;
    const float last = __shfl_sync(0xffffffffu, x1, 31);
    lg[lane] = x0;
    lg[32 + lane] = x1;
    gam[lane] = exp2f(x0);
    gam[32 + lane] = exp2f(x1);
    tail[lane] = exp2f(last - x0);
    tail[32 + lane] = exp2f(last - x1);
}

__device__ __forceinline__ void wy_scan(const float* lgr, float* lg, float* gam, float* tail, int lane) {
    wy_scan_core(lgr[lane], lgr[32 + lane], lg, gam, tail, lane);
}

// The same from a chunk's gate box (per token 16 bytes: g, beta, log g, pad); tokens >= nv count as log g = 0.
__device__ __forceinline__ void wy_scan_g4(const float* g4, int nv, float* lg, float* gam, float* tail, int lane) {
    wy_scan_core(lane < nv ? g4[lane * 4 + 2] : 0.0f, 32 + lane < nv ? g4[(32 + lane) * 4 + 2] : 0.0f, lg, gam, tail,
                 lane);
}

__device__ __forceinline__ bool wy_qualifies(const RecurArgs& a, int seq, int& t0, int& T, int& slot) {
    t0 = __ldg(a.cu_seqlens + seq);
    T = __ldg(a.cu_seqlens + seq + 1) - t0;
    slot = __ldg(a.slot_ids + seq);
    return slot >= 0 && slot < a.n_slots && T >= a.wy_min_t && t0 >= 0 && t0 + T <= a.n_tokens;
}


// 16-byte vector at row r, column group c8 of a [rows][COLS] bf16 tile in global memory (same layout).
template <int COLS>
__device__ __forceinline__ void st_tile_g(uint8_t* base, int r, int c8, const uint4& v) {
    *reinterpret_cast<uint4*>(base + (r >> 3) * (COLS / 8) * 128 + c8 * 128 + (r & 7) * 16) = v;
}

// ------------------------------------------------------------------ plan (one CTA)
// wy_cb[i] = number of 64-token chunks of the qualifying sequences before sequence i (exclusive prefix);
// wy_plan[0] = all chunks (or -1 when they exceed the scratch: error flagged, nothing runs), wy_plan[1] =
// qualifying sequences m, wy_plan[2 ..] = them ranked longest first (ties: call order) when m <= WY_SORT_CAP.
__global__ void __launch_bounds__(WP_THREADS, 1) gdn_wy_plan_kernel(const RecurArgs a) {
    __shared__ int s_warp[WP_THREADS / 32];
    __shared__ int s_run, s_cnt;
    __shared__ int l_seq[WY_SORT_CAP], l_len[WY_SORT_CAP];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // The chunk-parallel pass may launch now and set up.  It (and the sequential pass, which may launch while this
    // grid still runs) read the tables below only after their dependency wait, and with coherent loads (__ldcg):
    // the non-coherent path (__ldg) is only for data no running grid writes, and returned stale tables here.
    pdl_launch_dependents();
    pdl_wait();
    if (tid == 0) {
        s_run = 0;
        s_cnt = 0;
        *a.wy_counter = 0;
    }
    __syncthreads();
    for (int base = 0; base < a.n_seq; base += WP_THREADS) {
        const int i = base + tid;
        int t0 = 0, T = 0, slot = 0;
        const bool q = i < a.n_seq && wy_qualifies(a, i, t0, T, slot);
        const int nc = q ? (T + WC - 1) / WC : 0;
        if (q) {
            const int e = atomicAdd(&s_cnt, 1);
            if (e < WY_SORT_CAP) {
                l_seq[e] = i;
                l_len[e] = T;
            }
        }
        int x = nc;   // inclusive warp scan
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) s_warp[warp] = x;
        __syncthreads();
        if (warp == 0) {
            int w = s_warp[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o) w += y;
            }
            s_warp[lane] = w;   // inclusive over warps
        }
        __syncthreads();
        const int excl = s_run + (warp ? s_warp[warp - 1] : 0) + x - nc;
        if (i < a.n_seq) a.wy_cb[i] = excl;
        // the chunk table of the chunk-parallel pass: (first token row, tokens) of every chunk
        for (int c = 0; c < nc && excl + c < a.wy_cap_chunks; ++c)
            a.wy_chunks[excl + c] = make_int2(t0 + c * WC, (T - c * WC) < WC ? (T - c * WC) : WC);
        __syncthreads();
        if (tid == 0) s_run += s_warp[WP_THREADS / 32 - 1];
        __syncthreads();
    }
    const int m = s_cnt;
    if (m <= WY_SORT_CAP) {
        for (int e = tid; e < m; e += WP_THREADS) {
            const int le = l_len[e], se = l_seq[e];
            int r = 0;
            for (int f = 0; f < m; ++f) {
                const int lf = l_len[f];
                r += (lf > le) || (lf == le && l_seq[f] < se);
            }
            a.wy_plan[2 + r] = se;
        }
    }
    if (tid == 0) {
        const long long total = s_run;
        if (total > a.wy_cap_chunks) {
            atomicOr(a.err, ERR_BAD_SEQLENS);
            a.wy_plan[0] = -1;
        } else {
            a.wy_plan[0] = (int)total;
        }
        a.wy_plan[1] = m;
    }
}

// ------------------------------------------------------------------ chunk-parallel pass
// Per item (chunk, k-head): [QK; G] = [Q; K] K^T once, then the k-head's v-heads two at a time, one per
// warp group (warps 0-3 and 4-7; each group reaches all 128 TMEM lanes, one warp per lane quarter), each
// with its own M / T and N regions and group-local named barriers.
__device__ __forceinline__ void wa_head(const RecurArgs& a, uint8_t* out, float* fT, float* fN, const float* lgc,
                                        const float* gamc, const float* betc, uint32_t tcol, int gt, int bar_id) {
    const int gw = gt >> 5, lane = gt & 31;     // warp of the group = TMEM lane quarter
    const int L = gw * 32 + lane;
    // ---- lanes 0..63 hold QK row t -> P (.) QK hi/lo tiles; lanes 64..127 hold G row t -> M (f32)
    {
        const bool is_g = L >= WC;
        const int t = L & (WC - 1);
        const float lg_t = lgc[t];
        const float b_t = betc[t];
#pragma unroll 1
        for (int jj = 0; jj < 4; ++jj) {
            float x[16];
            tmem_ld16(tcol + jj * 16, x);
            if (is_g) {
                float mv[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const int s = jj * 16 + e;
                    mv[e] = s < t ? b_t * exp2f(lg_t - lgc[s]) * x[e] : 0.f;
                }
                float* mrow = fT + t * LDT + jj * 16;
#pragma unroll
                for (int e = 0; e < 16; e += 4)
                    *reinterpret_cast<float4*>(mrow + e) = make_float4(mv[e], mv[e + 1], mv[e + 2], mv[e + 3]);
            } else {
                float pv[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const int s = jj * 16 + e;
                    pv[e] = s <= t ? exp2f(lg_t - lgc[s]) * x[e] : 0.f;
                }
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    uint4 h4, l4;
                    split8(pv + 8 * u, h4, l4);
                    st_tile_g<64>(out + 32768, t, jj * 2 + u, h4);
                    st_tile_g<64>(out + 40960, t, jj * 2 + u, l4);
                }
            }
        }
    }
    named_bar_sync(bar_id, 128);
    // ---- T = (I + M)^-1 by 16 x 16 blocks, in place over M: the diagonal blocks by forward substitution
    // (warps 2, 3 of the group; lane: block 2 (gw - 2) + lane/16, column s)
    if (gw >= 2) {
        const int b = 2 * (gw - 2) + (lane >> 4), s = lane & 15;
        float* Mb = fT + 16 * b * LDT + 16 * b;
        float col[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) col[q] = q == s ? 1.f : 0.f;
#pragma unroll
        for (int t = 1; t < 16; ++t) {
            float a0 = 0.f, a1 = 0.f;
#pragma unroll
            for (int j4 = 0; j4 < t; j4 += 4) {
                const float4 mv = *reinterpret_cast<const float4*>(Mb + t * LDT + j4);
                a0 = fmaf(mv.x, col[j4], a0);
                a1 = fmaf(mv.y, col[j4 + 1], a1);
                a0 = fmaf(mv.z, col[j4 + 2], a0);
                a1 = fmaf(mv.w, col[j4 + 3], a1);
            }
            if (t > s) col[t] = -(a0 + a1);
        }
        __syncwarp();
#pragma unroll
        for (int q = 0; q < 16; ++q) Mb[q * LDT + s] = col[q];
    }
    named_bar_sync(bar_id, 128);
    // N_ik = T_ii M_ik for the six blocks below the diagonal (pair index i(i-1)/2 + k); each task is 4
    // consecutive outputs of one row: 384 tasks
    for (int task = gt; task < 6 * 64; task += 128) {
        const int pi = task >> 6, rem = task & 63;
        const int r = rem >> 2, c4 = (rem & 3) * 4;
        const int i = pi < 1 ? 1 : (pi < 3 ? 2 : 3);
        const int kk = pi - i * (i - 1) / 2;
        const float* Ti = fT + (16 * i + r) * LDT + 16 * i;
        const float* Mk = fT + 16 * i * LDT + 16 * kk + c4;
        uint64_t a01 = 0, a23 = 0;   // (x, y) and (z, w) of the four outputs, as f32 pairs (+0)
#pragma unroll
        for (int m4 = 0; m4 < 16; m4 += 4) {
            const float4 tr = *reinterpret_cast<const float4*>(Ti + m4);
            const float tv[4] = {tr.x, tr.y, tr.z, tr.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 mr = *reinterpret_cast<const float4*>(Mk + (m4 + q) * LDT);
                const uint64_t t2 = f2_pack(tv[q], tv[q]);
                a01 = f2_fma(t2, f2_pack(mr.x, mr.y), a01);
                a23 = f2_fma(t2, f2_pack(mr.z, mr.w), a23);
            }
        }
        float4 acc;
        f2_unpack(a01, acc.x, acc.y);
        f2_unpack(a23, acc.z, acc.w);
        *reinterpret_cast<float4*>(fN + pi * 256 + r * 16 + c4) = acc;
    }
    named_bar_sync(bar_id, 128);
    // block rows 1..3: T_ij = -sum_{k=j}^{i-1} N_ik T_kj (4 outputs per task)
#pragma unroll
    for (int i = 1; i < 4; ++i) {
        for (int task = gt; task < 64 * i; task += 128) {
            const int jb = task >> 6, rem = task & 63;
            const int r = rem >> 2, c4 = (rem & 3) * 4;
            uint64_t a01 = 0, a23 = 0;   // f32 pairs (+0)
            for (int kk = jb; kk < i; ++kk) {
                const float* Nr = fN + (i * (i - 1) / 2 + kk) * 256 + r * 16;
                const float* Tc = fT + 16 * kk * LDT + 16 * jb + c4;
#pragma unroll
                for (int m4 = 0; m4 < 16; m4 += 4) {
                    const float4 nr = *reinterpret_cast<const float4*>(Nr + m4);
                    const float nv4[4] = {nr.x, nr.y, nr.z, nr.w};
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float4 tr = *reinterpret_cast<const float4*>(Tc + (m4 + q) * LDT);
                        const uint64_t n2 = f2_pack(nv4[q], nv4[q]);
                        a01 = f2_fma(n2, f2_pack(tr.x, tr.y), a01);
                        a23 = f2_fma(n2, f2_pack(tr.z, tr.w), a23);
                    }
                }
            }
            float4 acc;
            f2_unpack(a01, acc.x, acc.y);
            f2_unpack(a23, acc.z, acc.w);
            *reinterpret_cast<float4*>(fT + (16 * i + r) * LDT + 16 * jb + c4) =
                make_float4(-acc.x, -acc.y, -acc.z, -acc.w);
        }
        named_bar_sync(bar_id, 128);
    }
    // ---- (T beta) and (T beta gamma) hi/lo tiles; thread (row t, columns [32 cq, +32))
    {
        const int t = gt & 63, cq = gt >> 6;
#pragma unroll 1
        for (int h16 = 0; h16 < 2; ++h16) {
            const int c0 = 32 * cq + 16 * h16;
            const float* Tr = fT + t * LDT + c0;
            float tb[16], tg[16];
#pragma unroll
            for (int e4 = 0; e4 < 16; e4 += 4) {
                const float4 x = *reinterpret_cast<const float4*>(Tr + e4);
                tb[e4] = x.x; tb[e4 + 1] = x.y; tb[e4 + 2] = x.z; tb[e4 + 3] = x.w;
            }
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const int s = c0 + e;
                const float x = s <= t ? tb[e] * betc[s] : 0.f;
                tb[e] = x;
                tg[e] = x * gamc[s];
            }
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                uint4 h4, l4;
                const int cg = c0 / 8 + u;
                split8(tb + 8 * u, h4, l4);
                st_tile_g<64>(out, t, cg, h4);
                st_tile_g<64>(out + 8192, t, cg, l4);
                split8(tg + 8 * u, h4, l4);
                st_tile_g<64>(out + 16384, t, cg, h4);
                st_tile_g<64>(out + 24576, t, cg, l4);
            }
        }
    }
    named_bar_sync(bar_id, 128);   // M / T region free for the group's next head
}

__global__ void __launch_bounds__(WA_THREADS, 2) gdn_wy_chunk_kernel(const RecurArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    float* s_beta2 = reinterpret_cast<float*>(smem + A_SMALL);   // [2 buffers][8][64]
    float* s_lgr2 = s_beta2 + 2 * 8 * WC;                        // [2 buffers][8][64] log g per token
    float* s_lg = s_lgr2 + 2 * 8 * WC;                           // [8][64] cumulative, log2 units
    float* s_gam = s_lg + 8 * WC;                                // [8][64] exp(lg_t)
    float* s_tail = s_gam + 8 * WC;                              // [8][64] (unused here)
    uint64_t* bar = reinterpret_cast<uint64_t*>(s_tail + 8 * WC);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
    volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int grp = warp >> 2, gt = tid & 127;                  // warp group, thread within it
    const uint32_t sb = smem_u32(smem);
    const int ratio = a.hv / a.hk;
    float* fT = reinterpret_cast<float*>(smem + A_T + grp * A_TN);

    if (tid == 0) {
        mbar_init(bar, 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(tmem_slot, 64);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tcol = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    uint32_t ph = 0;
    pdl_launch_dependents();   // the sequential pass may take SMs as this grid's CTAs leave them
    pdl_wait();
    const int total = __ldcg(a.wy_plan);   // the plan tables: coherent loads (see gdn_wy_plan_kernel)
    const int n_items = total > 0 ? total * a.hk : 0;

    // (first token row, tokens) of item `it`'s chunk from the plan's table; read an item ahead of its fetch
    auto chunk_of = [&](int it) { return it < n_items ? __ldcg(a.wy_chunks + it / a.hk) : make_int2(0, 0); };
    // Q, K and the gates of item `it` (chunk `chunk`) into buffer `buf` (cp.async, one commit group per thread and
    // item; an empty group past the last item keeps the group count uniform)
    auto fetch = [&](int it, int2 chunk, int buf) {
        if (it < n_items) {
            const int hk = it % a.hk;
            const uint8_t* recq = a.recs + ((long long)(hk * ratio) * a.rec_cap + chunk.x) * REC_BYTES;
            const uint32_t dq = sb + A_QK + buf * A_QKB;
            load_field(dq, recq, 0, chunk.y, tid);
            load_field(dq + 16384, recq, 256, chunk.y, tid);
            for (int j = 0; j < ratio; ++j)
                load_gates(s_beta2 + (buf * 8 + j) * WC, s_lgr2 + (buf * 8 + j) * WC,
                           a.recs + ((long long)(hk * ratio + j) * a.rec_cap + chunk.x) * REC_BYTES, chunk.y, tid);
        }
        cp_async_commit();
    };

    fetch(blockIdx.x, chunk_of(blockIdx.x), 0);
    int2 next_chunk = chunk_of(blockIdx.x + gridDim.x);
    int buf = 0;
    for (int it = blockIdx.x; it < n_items; it += gridDim.x, buf ^= 1) {
        const int g = it / a.hk, hk = it - g * a.hk;
        // the other buffer was released by the previous item's last barrier; the chunk after it is looked up now,
        // so its table read has an item's time to land
        const int2 nc = next_chunk;
        next_chunk = chunk_of(it + 2 * gridDim.x);
        fetch(it + gridDim.x, nc, buf ^ 1);
        cp_async_wait_group<1>();         // this item's group has landed (the next one may still be in flight)
        __syncthreads();
        const float* s_beta = s_beta2 + buf * 8 * WC;
        if (warp < ratio) wy_scan(s_lgr2 + (buf * 8 + warp) * WC, s_lg + warp * WC, s_gam + warp * WC, s_tail + warp * WC, lane);
        wy_sync_for_mma();
        // [QK; G] = [Q; K] K^T -> TMEM columns [0, 64) (rows 0..63 QK, rows 64..127 G)
        const uint32_t dq = sb + A_QK + buf * A_QKB;
        if (tid == 0) {
            const uint32_t id = umma_idesc_bf16(128, 64);
            const uint64_t da = umma_desc(dq, 128, 0), db = umma_desc(dq + 16384, 128, 0);
            for (int ks = 0; ks < 8; ++ks) umma_bf16(tmem, da + ks * KSTEP_K, db + ks * KSTEP_K, id, ks > 0);
            umma_commit(bar);
        }
        if (!wy_wait(bar, ph)) { atomicOr(a.err, ERR_TIMEOUT); *s_abort = 1; }
        __syncthreads();
        if (*s_abort) break;

        // the MMA has read Q and K: the buffer holds the N blocks of both groups until the item ends
        float* fN = reinterpret_cast<float*>(smem + A_QK + buf * A_QKB + grp * A_NB);
        for (int j0 = 0; j0 < ratio; j0 += 2) {
            const int j = j0 + grp;
            if (j < ratio) {
                const int hv = hk * ratio + j;
                uint8_t* out = a.wy_tiles + ((size_t)g * a.hv + hv) * TILESET;
                wa_head(a, out, fT, fN, s_lg + j * WC, s_gam + j * WC, s_beta + j * WC, tcol, gt, 1 + grp);
            }
        }
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    }
    cp_async_wait_all();   // no copy lands after the CTA ends (the prefetch of an item that an abort skipped)
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 64);
}

// ------------------------------------------------------------------ sequential pass

// bf16x2 helpers of the epilogue: (lo, hi) rounded to one bf16x2 word; a bf16x2 product rounded once.
__device__ __forceinline__ uint32_t bf2_pack(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;\n" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}
__device__ __forceinline__ uint32_t bf2_mul(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;\n" : "=r"(d) : "r"(a), "r"(b));
    return d;
}


// A compute warp's shared-memory and tensor-memory writes for the next MMA batch are done: one arrival per warp.
// Batch i of a chunk's MMAs (0: U/W, 1: Q S0^T, 2: D, 3: P D, 4: the state update) may go: the compute threads' shared-
// and tensor-memory writes for it are done.  A hardware named barrier of the 256 compute threads (arriving without
// waiting) and the issuing warp (waiting): it wakes the issuer within tens of cycles, where an mbarrier poll took
// hundreds.  Every compute thread arrives on each of the four once per chunk, and on batch 0's before leaving a
// chunk loop early, so the issuer never waits on one that does not come.
constexpr int WY_RDY_BAR = 3;   // named barriers 3..7 (1: compute warps, 2: epilogue warps)
__device__ __forceinline__ void ct_ready(int i) {
    fence_async_shared();
    tc_fence_before();
    named_bar_arrive(WY_RDY_BAR + i, WY_THREADS + 32);
}

// Q, K and V tiles of the sequential pass arrive by TMA token-major: element (t, f) of a [64 t][128 f] tile at
// (f / 8) * 1024 + t * 16 + (f % 8) * 2.  Read MN-major (K = t, M or N = f): 8-token groups 128 B apart (LBO),
// 8-feature groups 1024 B apart (SBO), a k-step of 16 tokens advances 256 B.  Read K-major (K = f, M or N = t):
// 8-feature groups 1024 B apart (LBO), 8-token groups 128 B apart (SBO), a k-step of 16 features advances 2048 B.
__device__ __forceinline__ uint64_t tok_desc_mn(uint32_t saddr) { return umma_desc_raw(saddr, 128u, 1024u); }
__device__ __forceinline__ uint64_t tok_desc_k(uint32_t saddr) { return umma_desc_raw(saddr, 1024u, 128u); }
constexpr uint64_t TOK_KSTEP_MN = 256u >> 4, TOK_KSTEP_K = 2048u >> 4;
__global__ void __launch_bounds__(WY_BLOCK, 1) gdn_wy_kernel(const RecurArgs a,
                                                                const __grid_constant__ CUtensorMap tm_rec,
                                                                const __grid_constant__ CUtensorMap tm_gate,
                                                                const __grid_constant__ CUtensorMap tm_z) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const float* s_g4 = reinterpret_cast<const float*>(smem + R_G);   // [2][64][4]: g, beta, log g, pad per token
    float* s_lg = reinterpret_cast<float*>(smem + R_SMALL);       // [2][64] cumulative, log2 units
    float* s_gam = s_lg + 2 * WC;                                 // [2][64] exp(lg_t)
    float* s_tail = s_gam + 2 * WC;                               // [2][64] exp(lg_last - lg_t)
    float* s_nw = s_tail + 2 * WC;                                // 128 floats of room; holds norm_w as bf16 pairs
    uint32_t* s_nw2 = reinterpret_cast<uint32_t*>(s_nw);          // [64] norm_w (2c, 2c+1) as a bf16x2 word
    uint64_t* bar = reinterpret_cast<uint64_t*>(s_nw + DV);       // MMA batches waited in order
    uint64_t* bar_qs = bar + 1;                                   // (Q S0^T)^T, issued early
    uint64_t* bar_s = bar + 2;                                    // state update, waited when S is next used
    uint64_t* bar_tb = bar + 3;   // the chunk's T beta / T beta gamma tiles (bulk copy; U and W wait for them)
    uint64_t* bar_in = bar + 4;                                   // [2] Q, K and gates of the chunk of that parity
    uint64_t* bar_v = bar + 6;                                    // V of the current / next chunk
    uint64_t* bar_w = bar + 7;     // W^T of the chunk (issued before U, so the -W^T tiles need not wait for U)
    // bar + 8 .. bar + 10: unused
    uint64_t* bar_fin = bar + 11;  // every MMA of the issuing warp complete (kernel exit)
    uint64_t* bar_z = bar + 12;    // [2] silu(z) box of the chunk of that parity
    uint64_t* epi_full = bar + 14;  // a chunk's y is transposed into s_yt (thread 0 of the compute warps)
    uint64_t* epi_free = bar + 15;  // the epilogue warps are done with s_yt and the chunk's z box
    uint64_t* bar_tp = bar + 16;    // the chunk's P (.) QK tiles (bulk copy; only P D waits for them)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 17);
    volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* s_ticket = s_abort + 1;
    uint16_t* s_yt = reinterpret_cast<uint16_t*>(smem + R_T);    // y [64 t][LDY] bf16, the epilogue's transpose

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quarter = warp & 3, hh = warp >> 2;   // TMEM lane quarter, column half
    const int L = quarter * 32 + lane;              // TMEM lane = MMA row owned by this thread
    const uint32_t sb = smem_u32(smem);
    const int ratio = a.hv / a.hk;

    if (tid == 0) {
        mbar_init(bar, 1);
        mbar_init(bar_qs, 1);
        mbar_init(bar_s, 1);
        mbar_init(bar_tb, 1);
        mbar_init(bar_in, 1);
        mbar_init(bar_in + 1, 1);
        mbar_init(bar_v, 1);
        mbar_init(bar_fin, 1);
        mbar_init(bar_z, 1);
        mbar_init(bar_z + 1, 1);
        mbar_init(epi_full, 1);
        mbar_init(bar_tp, 1);
        mbar_init(bar_w, 1);
        mbar_init(epi_free, WY_EPI_THREADS / 32);
        *s_abort = 0;
        fence_mbar_init();
    }
    for (int i = tid; i < DV / 2; i += WY_THREADS)
        s_nw2[i] = (uint32_t)a.norm_w[2 * i] | ((uint32_t)a.norm_w[2 * i + 1] << 16);
    if (warp == 0) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    uint32_t ph = 0, ph_qs = 0, ph_s = 0, ph_tb = 0, ph_v = 0;
    uint32_t ph_in = 0;        // bit b: the phase of bar_in[b] to wait for next
    uint32_t nb = 0;           // (issuing warp) completions of bar before the current chunk
    uint32_t ph_tp = 0;        // (issuing warp) the phase of bar_tp to wait for next
    // copies of the chunk inputs, issued by the MMA-issuing warp (bar_in[0], bar_in[1], bar_v, bar_tb: bits 0-3;
    // bar_tp: bit 6) and the z boxes by the epilogue warps (bar_z[0], bar_z[1]: bits 4-5): a phase issued on that
    // barrier / the parity of the next issue, for the bounded drain at the exit
    uint32_t cp_any = 0, cp_next = 0;
    uint32_t ph_z = 0;         // (epilogue warps) bit b: the phase of bar_z[b] to wait for next
    uint32_t ph_zc = 0;        // (compute warps) the same, for their SiLU of the raw z boxes
    uint32_t ph_w = 0;         // (compute warps) the phase of bar_w to wait for next
    uint32_t n_yt = 0;         // chunks whose y this CTA has handed to the epilogue warps (compute and epilogue)
    pdl_wait();

    const int total = __ldcg(a.wy_plan);   // the plan tables: coherent loads (see gdn_wy_plan_kernel)
    const int m_seq = __ldcg(a.wy_plan + 1);
    const bool ranked = m_seq <= WY_SORT_CAP;
    const int n_work = total < 0 ? 0 : (ranked ? m_seq : a.n_seq) * a.hv;

    for (;;) {
        if (tid == 0) *s_ticket = atomicAdd(a.wy_counter, 1);
        __syncthreads();
        const int k = *s_ticket;
        const bool stop = k >= n_work || *s_abort;
        __syncthreads();
        if (stop) break;
        const int si = k / a.hv;
        const int hv = k - si * a.hv;
        const int seq = ranked ? __ldcg(a.wy_plan + 2 + si) : si;
        int t0, T, slot;
        if (!wy_qualifies(a, seq, t0, T, slot)) continue;
        float* st = a.rec + ((size_t)slot * a.hv + hv) * (DV * DK);
        const float* st_in = (a.rec_in ? a.rec_in : a.rec) + ((size_t)slot * a.hv + hv) * (DV * DK);
        const uint8_t* tiles = a.wy_tiles + ((size_t)__ldcg(a.wy_cb + seq) * a.hv + hv) * TILESET;
        const size_t tile_step = (size_t)a.hv * TILESET;   // next chunk of the same head
        const int n_chunks = (T + WC - 1) / WC;

        // Copies of a chunk's inputs (one thread issues each; the compute warps wait for them).  Q, K and the gates
        // of chunk cc into buffer b and V: TMA boxes of 64 token rows from the records (record chunks 0-15 Q, 16-31
        // K, 32-47 V, 48-63 silu(z), 64 the gates), landing token-major with rows 16 bytes apart.  The tile set of
        // chunk cc (T beta, T beta gamma | P (.) QK) by two bulk copies on one barrier phase.
        auto note_copy = [&](int bit) {
            cp_any |= 1u << bit;
            cp_next ^= 1u << bit;
        };
        auto issue_qkg = [&](int cc, int b) {
            mbar_arrive_expect_tx(bar_in + b, 2 * 16384 + WC * 16);
            tma_load_4d(smem + R_QK + b * 32768, &tm_rec, 0, t0 + cc * WC, 0, hv, bar_in + b);
            tma_load_4d(smem + R_QK + b * 32768 + 16384, &tm_rec, 0, t0 + cc * WC, 16, hv, bar_in + b);
            tma_load_4d(smem + R_G + b * WC * 16, &tm_gate, 0, t0 + cc * WC, 64, hv, bar_in + b);
            note_copy(b);
        };
        auto issue_v = [&](int cc) {
            mbar_arrive_expect_tx(bar_v, 16384);
            tma_load_4d(smem + R_V, &tm_rec, 0, t0 + cc * WC, 32, hv, bar_v);
            note_copy(2);
        };
        auto issue_tiles_tb = [&](int cc) {   // T beta / T beta gamma: R_TB must be free
            mbar_arrive_expect_tx(bar_tb, R_P - R_TB);
            bulk_g2s(smem + R_TB, tiles + (size_t)cc * tile_step, R_P - R_TB, bar_tb);
            note_copy(3);
        };
        auto issue_tiles_p = [&](int cc) {    // P (.) QK: R_P must be free
            mbar_arrive_expect_tx(bar_tp, TILESET - (R_P - R_TB));
            bulk_g2s(smem + R_P, tiles + (size_t)cc * tile_step + (R_P - R_TB), TILESET - (R_P - R_TB), bar_tp);
            note_copy(6);
        };
        auto issue_z = [&](int cc) {          // z (or silu(z)) of chunk cc into buffer cc & 1
            mbar_arrive_expect_tx(bar_z + (cc & 1), 16384);
            if (a.z)   // the caller's z: token rows ld_z apart, v-head hv at 16-byte chunks [16 hv, 16 hv + 16)
                tma_load_4d(smem + R_Z + (cc & 1) * 16384, &tm_z, 0, t0 + cc * WC, 16 * hv, 0, bar_z + (cc & 1));
            else
                tma_load_4d(smem + R_Z + (cc & 1) * 16384, &tm_rec, 0, t0 + cc * WC, 48, hv, bar_z + (cc & 1));
            note_copy(4 + (cc & 1));
        };

        if (warp < WY_THREADS / 32) {
            // ---- state -> TMEM S (thread (v, half) owns row v, columns [64 half, 64 half + 64))
            {
                const float* src = st_in + (size_t)L * DK + hh * 64;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float v[16];
#pragma unroll
                    for (int e = 0; e < 16; e += 4) {
                        const float4 f = __ldcs(reinterpret_cast<const float4*>(src + j * 16 + e));
                        v[e] = f.x; v[e + 1] = f.y; v[e + 2] = f.z; v[e + 3] = f.w;
                    }
                    tmem_st16(tmem + lane_base + TM_S + hh * 64 + j * 16, v);
                }
                tmem_st_wait();
            }

            for (int c = 0; c < n_chunks; ++c) {
                const int kb = c & 1;
                const int nv = (T - c * WC) < WC ? (T - c * WC) : WC;
                const bool has_next = c + 1 < n_chunks;
                const int nv1 = has_next ? ((T - (c + 1) * WC) < WC ? (T - (c + 1) * WC) : WC) : 0;
                const float* gamc = s_gam + kb * WC;
                const float* tailc = s_tail + kb * WC;

                // ---- phase A: the previous state update is complete.  The chunk's inputs are read only by the MMAs,
                // and the issuing warp waits for them; the compute warps wait only where they touch them: to clear
                // the rows past a sequence's end and for the first chunk's decay scan (one completion per chunk on
                // each barrier, so the phase bits advance either way)
                if (nv < WC || c == 0) {
                    const bool ok_q = mbar_wait_bounded(bar_in + kb, (ph_in >> kb) & 1u, WY_WAIT_NS);
                    const bool ok_v = mbar_wait_bounded(bar_v, ph_v, WY_WAIT_NS);
                    if (!(ok_q && ok_v)) { atomicOr(a.err, ERR_TIMEOUT); *s_abort = 1; }
                }
                ph_in ^= 1u << kb;
                ph_v ^= 1u;
                if (c > 0) {
                    // the previous chunk's state update still reads the K buffer refilled below
                    if (!mbar_wait_bounded(bar_s, ph_s, WY_WAIT_NS)) { atomicOr(a.err, ERR_TIMEOUT); *s_abort = 1; }
                    ph_s ^= 1u;
                    tc_fence_after();
                }
                // (the issuing warp may raise the abort flag at any time: the decision is taken once, by barrier)
                if (named_bar_or(1, WY_THREADS, *s_abort != 0)) {
                    named_bar_arrive(WY_RDY_BAR, WY_THREADS + 32);   // the issuer waits for batch 0, then stops
                    break;
                }
                // a chunk that ends its sequence: the rows past the end hold the next sequence's tokens (or zeros);
                // K and V rows there are cleared so only exact zeros meet the zero rows of T beta and T beta gamma
                if (nv < WC) {
                    const int rows = WC - nv;
                    for (int idx = tid; idx < rows * 32; idx += WY_THREADS) {
                        const int tile = idx / (rows * 16), rem = idx - tile * rows * 16;
                        uint8_t* base = tile ? smem + R_V : smem + R_QK + kb * 32768 + 16384;
                        *reinterpret_cast<uint4*>(base + (rem & 15) * 1024 + (nv + (rem >> 4)) * 16) = make_uint4(0, 0, 0, 0);
                    }
                }
                if (c == 0 && warp == 0) wy_scan_g4(s_g4, nv, s_lg, s_gam, s_tail, lane);   // later chunks: during P D
                // ---- phase B (issuing warp): U^T = V^T (T beta)^T, W^T = K^T (T beta gamma)^T; they need only the
                // chunk's own inputs and overlap the state split below
                fence_async_shared();
                tc_fence_before();
                // the decays and the cleared rows visible to every compute thread (a full chunk after the first has
                // neither to publish: the barrier above suffices)
                if (c == 0 || nv < WC) named_bar_sync(1, WY_THREADS);
                named_bar_arrive(WY_RDY_BAR, WY_THREADS + 32);
                // ---- phase C: S0 hi/lo tiles [v][d]; S *= gamma_last in place
                {
                    const float g_last = gamc[WC - 1];
                    uint32_t sr[4][16];   // the thread's 64 state columns: four loads in flight, one wait
#pragma unroll
                    for (int j = 0; j < 4; ++j) tmem_ld16_async(tmem + lane_base + TM_S + hh * 64 + j * 16, sr[j]);
                    tmem_ld_wait();
                    const uint64_t g2 = f2_pack(g_last, g_last);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        uint64_t sp[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) sp[e] = f2_of(&sr[j][2 * e]);
                        uint4 hi0, lo0, hi1, lo1;
                        split8_f2(sp, hi0, lo0);
                        split8_f2(sp + 4, hi1, lo1);
                        tmem_st8(tmem + lane_base + TM_AH + hh * 32 + j * 8, hi0, hi1);
                        tmem_st8(tmem + lane_base + TM_AL + hh * 32 + j * 8, lo0, lo1);
                        float sv[16];
#pragma unroll
                        for (int e = 0; e < 8; ++e) f2_unpack(f2_mul(sp[e], g2), sv[2 * e], sv[2 * e + 1]);
                        tmem_st16(tmem + lane_base + TM_S + hh * 64 + j * 16, sv);
                    }
                    tmem_st_wait();
                }
                // (Q S0^T)^T = S0 Q^T -> QS by the issuing warp, off the critical path (read in H)
                ct_ready(1);
                // ---- phase E: -W^T hi/lo tiles [d][t]; then D^T = U^T - S0 W^T onto U.  W is issued (and committed)
                // before U: its split runs while U's MMAs do; the tiles overwrite U's T beta operand, so they are
                // stored once U / W's completion is seen as well
                if (!mbar_wait_bounded(bar_w, ph_w, WY_WAIT_NS)) { atomicOr(a.err, ERR_TIMEOUT); *s_abort = 1; }
                ph_w ^= 1u;
                tc_fence_after();
                uint32_t wr[2][16];
#pragma unroll
                for (int j = 0; j < 2; ++j) tmem_ld16_async(tmem + lane_base + TM_W + hh * 32 + j * 16, wr[j]);
                tmem_ld_wait();
                uint4 whi[2][2], wlo[2][2];
#pragma unroll
                for (int j = 0; j < 2; ++j) {
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        // split W, then negate both halves (bf16 rounding is symmetric: the bits of the split of -W)
                        uint64_t wp[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) wp[e] = f2_of(&wr[j][8 * u + 2 * e]);
                        uint4 hi, lo;
                        split8_f2(wp, hi, lo);
                        whi[j][u] = make_uint4(hi.x ^ 0x80008000u, hi.y ^ 0x80008000u, hi.z ^ 0x80008000u, hi.w ^ 0x80008000u);
                        wlo[j][u] = make_uint4(lo.x ^ 0x80008000u, lo.y ^ 0x80008000u, lo.z ^ 0x80008000u, lo.w ^ 0x80008000u);
                    }
                }
                if (!wy_wait(bar, ph)) { atomicOr(a.err, ERR_TIMEOUT); *s_abort = 1; }   // U / W complete
#pragma unroll
                for (int j = 0; j < 2; ++j)
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        st_tile<64>(smem + R_TB, L, hh * 4 + j * 2 + u, whi[j][u]);
                        st_tile<64>(smem + R_TB + 16384, L, hh * 4 + j * 2 + u, wlo[j][u]);
                    }
                ct_ready(2);   // D^T = U^T - S0 W^T onto U by the issuing warp
                // while D runs: this chunk's z box (the caller's raw z) becomes silu(z) in place, for the epilogue
                // warps, which read it after this chunk's y (the prefill tiles' fast SiLU, bf2_silu_fast)
                if (a.z) {
                    const int zb = c & 1;
                    if (mbar_wait_bounded(bar_z + zb, (ph_zc >> zb) & 1u, WY_WAIT_NS)) {
                        uint8_t* zbox = smem + R_Z + zb * 16384;
                        for (int u = tid; u < WC * 16; u += WY_THREADS) {   // unit u: feature chunk u / 64, token u % 64
                            if ((u & (WC - 1)) < nv) {
                                uint4* zp = reinterpret_cast<uint4*>(zbox + (u >> 6) * 1024 + (u & (WC - 1)) * 16);
                                uint4 zz = *zp;
                                zz.x = bf2_silu_fast(zz.x);
                                zz.y = bf2_silu_fast(zz.y);
                                zz.z = bf2_silu_fast(zz.z);
                                zz.w = bf2_silu_fast(zz.w);
                                *zp = zz;
                            }
                        }
                    } else {
                        atomicOr(a.err, ERR_TIMEOUT);
                        *s_abort = 1;
                    }
                    ph_zc ^= 1u << zb;
                }
                if (!wy_wait(bar, ph)) { atomicOr(a.err, ERR_TIMEOUT); *s_abort = 1; }
                if (!wy_wait(bar_qs, ph_qs)) { atomicOr(a.err, ERR_TIMEOUT); *s_abort = 1; }

                // ---- phase F: D^T and Dd^T = D^T diag(exp(lg_last - lg_s)) as hi/lo tiles [v][s]
                uint32_t dr[2][16];
#pragma unroll
                for (int j = 0; j < 2; ++j) tmem_ld16_async(tmem + lane_base + TM_U + hh * 32 + j * 16, dr[j]);
                tmem_ld_wait();
                uint64_t dp[2][8];
#pragma unroll
                for (int j = 0; j < 2; ++j) {
#pragma unroll
                    for (int e = 0; e < 8; ++e) dp[j][e] = f2_of(&dr[j][2 * e]);
                    uint4 hi0, lo0, hi1, lo1;
                    split8_f2(dp[j], hi0, lo0);
                    split8_f2(dp[j] + 4, hi1, lo1);
                    tmem_st8(tmem + lane_base + TM_AH + hh * 16 + j * 8, hi0, hi1);
                    tmem_st8(tmem + lane_base + TM_AH + 32 + hh * 16 + j * 8, lo0, lo1);
                }
                // ---- phase G (issuing warp): (P D)^T = D^T P^T -> PD (waited in H) as soon as D's hi / lo are in
                tmem_st_wait();
                ct_ready(3);
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const float2* tl2 = reinterpret_cast<const float2*>(tailc + hh * 32 + j * 16);
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const float2 tv = tl2[e];
                        dp[j][e] = f2_mul(dp[j][e], f2_pack(tv.x, tv.y));
                    }
                    uint4 hi0, lo0, hi1, lo1;
                    split8_f2(dp[j], hi0, lo0);
                    split8_f2(dp[j] + 4, hi1, lo1);
                    tmem_st8(tmem + lane_base + TM_AL + hh * 16 + j * 8, hi0, hi1);
                    tmem_st8(tmem + lane_base + TM_AL + 32 + hh * 16 + j * 8, lo0, lo1);
                }
                // ... then S += Dd^T K -> S (waited when the state or the K buffer is next touched)
                tmem_st_wait();
                ct_ready(4);
                if (has_next && warp == 7) {
                    // the next chunk's decay scan, from its gate box, while P D runs (its buffers are the other
                    // parity's; the barrier at the end of this chunk publishes them; the same barrier phase is
                    // waited again in phase A)
                    if (!mbar_wait_bounded(bar_in + (kb ^ 1), (ph_in >> (kb ^ 1)) & 1u, WY_WAIT_NS)) {
                        atomicOr(a.err, ERR_TIMEOUT);
                        *s_abort = 1;
                    }
                    wy_scan_g4(s_g4 + (kb ^ 1) * WC * 4, nv1, s_lg + (kb ^ 1) * WC, s_gam + (kb ^ 1) * WC,
                               s_tail + (kb ^ 1) * WC, lane);
                }
                // Q S0^T completed before phase F: its columns load while P D runs
                uint32_t qr[2][16], pr[2][16];
#pragma unroll
                for (int j = 0; j < 2; ++j) tmem_ld16_async(tmem + lane_base + TM_QS + hh * 32 + j * 16, qr[j]);
                if (!wy_wait(bar, ph)) { atomicOr(a.err, ERR_TIMEOUT); *s_abort = 1; }

                // ---- phase H: y^T[v][t] = gamma_t QS[v][t] + PD[v][t], rounded to bf16, transposed through smem for
                // the epilogue warps (gated RMSNorm per token), once they are done with the previous chunk's y
                if (n_yt > 0 && !mbar_wait_bounded(epi_free, (n_yt - 1) & 1u, WY_WAIT_NS)) {
                    atomicOr(a.err, ERR_TIMEOUT);
                    *s_abort = 1;
                }
                {
#pragma unroll
                    for (int j = 0; j < 2; ++j) tmem_ld16_async(tmem + lane_base + TM_PD + hh * 32 + j * 16, pr[j]);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 2; ++j)
#pragma unroll
                        for (int e = 0; e < 16; e += 2) {
                            const int t = hh * 32 + j * 16 + e;
                            const float2 g = *reinterpret_cast<const float2*>(gamc + t);
                            // gamma_t * QS + PD for tokens t, t + 1, each rounded once (an f32 FMA per lane)
                            const uint32_t yb = f2_to_bf2(f2_fma(f2_pack(g.x, g.y), f2_of(&qr[j][e]), f2_of(&pr[j][e])));
                            s_yt[t * LDY + L] = (uint16_t)(yb & 0xFFFFu);
                            s_yt[(t + 1) * LDY + L] = (uint16_t)(yb >> 16);
                        }
                }
                // y is in s_yt and every TMEM read of the chunk is complete: one barrier, then the epilogue warps
                tc_fence_before();
                named_bar_sync(1, WY_THREADS);
                tc_fence_after();
                if (tid == 0) mbar_arrive(epi_full);
                ++n_yt;
            }
            if (n_chunks > 0 && !*s_abort) {
                if (!mbar_wait_bounded(bar_s, ph_s, WY_WAIT_NS)) { atomicOr(a.err, ERR_TIMEOUT); *s_abort = 1; }
                ph_s ^= 1u;
                tc_fence_after();
            }

            // ---- state back to the pool (row v, columns [64 half, +64))
            {
                float* dst = st + (size_t)L * DK + hh * 64;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float v[16];
                    tmem_ld16(tmem + lane_base + TM_S + hh * 64 + j * 16, v);
#pragma unroll
                    for (int e = 0; e < 16; e += 4)
                        __stcs(reinterpret_cast<float4*>(dst + j * 16 + e), make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]));
                }
            }
            // ---- conv-state windows: the last K-1 rows of [old window; tokens]
            {
                uint16_t* cs = a.conv + (size_t)slot * (KC - 1) * a.D;
                const int hk = hv / ratio;
                for (int idx = tid; idx < DV + ((hv % ratio == 0) ? 2 * DK : 0); idx += WY_THREADS) {
                    const int ch = idx < DV ? 2 * a.hk * DK + hv * DV + idx
                                            : ((idx - DV) < DK ? hk * DK + (idx - DV) : a.hk * DK + hk * DK + (idx - DV - DK));
                    uint16_t w[KC - 1];
#pragma unroll
                    for (int j = 0; j < KC - 1; ++j) {
                        const int p = T + j;
                        w[j] = p < KC - 1 ? cs[(size_t)p * a.D + ch] : a.qkv[(long long)(t0 + p - (KC - 1)) * a.ld_qkv + ch];
                    }
#pragma unroll
                    for (int j = 0; j < KC - 1; ++j) cs[(size_t)j * a.D + ch] = w[j];
                }
            }
        } else if (warp == WY_ISSUER_WARP) {
            // ---- the issuing warp: each MMA batch once the compute warps report its operands written
            auto ready = [&](int i) -> bool {   // batch i's operands are written (false: the compute warps stopped)
                named_bar_sync(WY_RDY_BAR + i, WY_THREADS + 32);
                tc_fence_after();
                return i != 0 || *s_abort == 0;
            };
            // the item's first chunk inputs (every buffer's last reader, in the previous item, is complete)
            if (elect_one()) {
                issue_tiles_tb(0);
                issue_tiles_p(0);
                issue_qkg(0, 0);
                issue_v(0);
                if (n_chunks > 1) bulk_prefetch_l2(tiles + tile_step, TILESET);   // chunk 1's tile set into L2
            }
            __syncwarp();
            bool done = true;
            for (int c = 0; c < n_chunks; ++c) {
                const uint32_t sQ = sb + R_QK + (c & 1) * 32768;    // Q [64][128], then K [64][128] at +16384
                const uint32_t sK = sQ + 16384;
                const bool has_next = c + 1 < n_chunks;
                if (c > 0) {
                    // the previous chunk's state update, and so its P D, is complete: its K buffer and R_P are free
                    const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar_s, ph_s, WY_WAIT_NS));
                    if (!ok) {
                        if (lane == 0) { atomicOr(a.err, ERR_TIMEOUT); *s_abort = 1; }
                        done = false;
                        break;
                    }
                    ph_s ^= 1u;
                    if (elect_one()) issue_tiles_p(c);
                    __syncwarp();
                }
                if (has_next) {
                    if (elect_one()) issue_qkg(c + 1, (c + 1) & 1);
                    __syncwarp();
                }
                // U^T = V^T (T beta)^T -> U;  W^T = K^T (T beta gamma)^T -> W   (V, K read MN-major)
                if (!ready(0)) { done = false; break; }
                {   // the chunk's Q, K, V and T beta / T beta gamma tiles have landed
                    const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar_in + (c & 1), (ph_in >> (c & 1)) & 1u,
                                                                              WY_WAIT_NS) &&
                                                                mbar_wait_bounded(bar_v, ph_v, WY_WAIT_NS) &&
                                                                mbar_wait_bounded(bar_tb, ph_tb, WY_WAIT_NS));
                    if (!ok) {
                        if (lane == 0) { atomicOr(a.err, ERR_TIMEOUT); *s_abort = 1; }
                        done = false;
                        break;
                    }
                    ph_in ^= 1u << (c & 1);
                    ph_v ^= 1u;
                    ph_tb ^= 1u;
                }
                if (elect_one()) {
                    const uint32_t id = umma_idesc_bf16(128, 64, true, false);
                    const uint64_t dv = tok_desc_mn(sb + R_V), dk = tok_desc_mn(sK);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint64_t dt = umma_desc(sb + R_TB + 16384 + h * 8192, 64, 0);
#pragma unroll
                        for (int ks = 0; ks < 4; ++ks)
                            umma_bf16(tmem + TM_W, dk + ks * TOK_KSTEP_MN, dt + ks * KSTEP_K, id, (h | ks) != 0);
                    }
                    umma_commit(bar_w);   // W first: the compute warps' -W^T tiles wait only for it
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint64_t dt = umma_desc(sb + R_TB + h * 8192, 64, 0);
#pragma unroll
                        for (int ks = 0; ks < 4; ++ks)
                            umma_bf16(tmem + TM_U, dv + ks * TOK_KSTEP_MN, dt + ks * KSTEP_K, id, (h | ks) != 0);
                    }
                    umma_commit(bar);
                }
                __syncwarp();
                // (Q S0^T)^T = S0 Q^T -> QS
                if (!ready(1)) { done = false; break; }
                if (elect_one()) {
                    const uint32_t idq = umma_idesc_bf16(128, 64);
                    const uint64_t dq = tok_desc_k(sQ);
#pragma unroll
                    for (int h = 0; h < 2; ++h)
#pragma unroll
                        for (int ks = 0; ks < 8; ++ks)
                            umma_bf16_ta(tmem + TM_QS, tmem + (h ? TM_AL : TM_AH) + ks * 8, dq + ks * TOK_KSTEP_K, idq,
                                         (h | ks) != 0);
                    umma_commit(bar_qs);
                }
                __syncwarp();
                if (has_next) {   // U has read V: the next chunk's V streams in
                    const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar, nb & 1u, WY_WAIT_NS));
                    if (!ok) {
                        if (lane == 0) { atomicOr(a.err, ERR_TIMEOUT); *s_abort = 1; }
                        done = false;
                        break;
                    }
                    if (elect_one()) issue_v(c + 1);
                    __syncwarp();
                }
                // D^T = U^T - S0 W^T onto U (S0 and -W^T as hi/lo pairs, lo x lo dropped)
                if (!ready(2)) { done = false; break; }
                if (elect_one()) {
                    const uint32_t idd = umma_idesc_bf16(128, 64, false, true);
                    const uint32_t as0[3] = {TM_AH, TM_AL, TM_AH}, bw[3] = {R_TB, R_TB, R_TB + 16384};
                    constexpr uint64_t kmn = umma_kstep_mn(64);
#pragma unroll
                    for (int p = 0; p < 3; ++p) {
                        const uint64_t db = umma_desc_mn(sb + bw[p], 64, 0);
#pragma unroll
                        for (int ks = 0; ks < 8; ++ks)
                            umma_bf16_ta(tmem + TM_U, tmem + as0[p] + ks * 8, db + ks * kmn, idd, 1u);
                    }
                    umma_commit(bar);
                }
                __syncwarp();
                if (has_next) {
                    // D has read -W^T: the next chunk's T beta / T beta gamma tiles stream into R_TB as soon as it
                    // completes (U / W's phase of bar completed above, so this parity wait is for D's)
                    const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar, (nb + 1) & 1u, WY_WAIT_NS));
                    if (!ok) {
                        if (lane == 0) { atomicOr(a.err, ERR_TIMEOUT); *s_abort = 1; }
                        done = false;
                        break;
                    }
                    if (elect_one()) {
                        issue_tiles_tb(c + 1);
                        // the tile set after it into L2 now, so its copies hit L2 when they are issued (the
                        // T beta copy otherwise arrived late for U / W)
                        if (c + 2 < n_chunks) bulk_prefetch_l2(tiles + (size_t)(c + 2) * tile_step, TILESET);
                    }
                    __syncwarp();
                }
                // (P D)^T = D^T P^T -> PD once D's hi / lo are written and the P tiles landed
                if (!ready(3)) { done = false; break; }
                if (!__all_sync(0xffffffffu, mbar_wait_bounded(bar_tp, ph_tp, WY_WAIT_NS))) {
                    if (lane == 0) { atomicOr(a.err, ERR_TIMEOUT); *s_abort = 1; }
                    done = false;
                    break;
                }
                ph_tp ^= 1u;
                if (elect_one()) {
                    const uint32_t idp = umma_idesc_bf16(128, 64);
                    const uint32_t ad[3] = {TM_AH, TM_AH + 32, TM_AH}, bp[3] = {R_P, R_P, R_P + 8192};
#pragma unroll
                    for (int p = 0; p < 3; ++p) {
                        const uint64_t db = umma_desc(sb + bp[p], 64, 0);
#pragma unroll
                        for (int ks = 0; ks < 4; ++ks)
                            umma_bf16_ta(tmem + TM_PD, tmem + ad[p] + ks * 8, db + ks * KSTEP_K, idp, (p | ks) != 0);
                    }
                    umma_commit(bar);
                }
                __syncwarp();
                // S += Dd^T K once the compute warps have written Dd's hi / lo
                if (!ready(4)) { done = false; break; }
                if (elect_one()) {
                    const uint32_t ids = umma_idesc_bf16(128, 128, false, true);
                    const uint64_t dk = tok_desc_mn(sK);
#pragma unroll
                    for (int h = 0; h < 2; ++h)
#pragma unroll
                        for (int ks = 0; ks < 4; ++ks)
                            umma_bf16_ta(tmem + TM_S, tmem + TM_AL + h * 32 + ks * 8, dk + ks * TOK_KSTEP_MN, ids, 1u);   // K MN-major
                    umma_commit(bar_s);
                }
                __syncwarp();
                nb += 3;   // U/W, D and P D completed on bar this chunk
            }
            if (done && n_chunks > 0) ph_s ^= 1u;   // the last state update is waited for by the compute warps only
        } else {
            // ---- the epilogue warps: each chunk once its y is in s_yt (and its z box landed): per token, gated
            // RMSNorm over the 128 v of the row times silu(z), stored; one token row per thread.  The sum of
            // squares adds four quarter sums as the compute warps' epilogue did (same bits).
            const int et = tid - WY_EPI_WARP * 32;   // token row of the chunk
            if (warp == WY_EPI_WARP) {   // the first two chunks' z boxes (both buffers are free)
                if (elect_one()) {
                    issue_z(0);
                    if (n_chunks > 1) issue_z(1);
                }
                __syncwarp();
            }
            // Chunk cc's z box once it landed (with raw z the compute warps turn it into silu(z) during the chunk's
            // D, before they hand its y over)
            auto take_z = [&](int cc) -> bool {
                const int zb = cc & 1;
                const bool zok = mbar_wait_bounded(bar_z + zb, (ph_z >> zb) & 1u, WY_WAIT_NS);
                ph_z ^= 1u << zb;
                return zok;
            };
            bool z_ok = n_chunks > 0 ? take_z(0) : true;
            for (int c = 0; c < n_chunks; ++c) {
                const int nv = (T - c * WC) < WC ? (T - c * WC) : WC;
                const int zb = c & 1;
                const bool ok = z_ok && mbar_wait_bounded(epi_full, n_yt & 1u, WY_WAIT_NS);
                if (named_bar_or(2, WY_EPI_THREADS, !ok)) {   // one decision for both epilogue warps
                    if (et == 0) {
                        atomicOr(a.err, ERR_TIMEOUT);
                        *s_abort = 1;
                    }
                    break;
                }
                ++n_yt;
                if (et < nv) {
                    const uint4* yr = reinterpret_cast<const uint4*>(s_yt + et * LDY);
                    float part[4];
#pragma unroll
                    for (int qd = 0; qd < 4; ++qd) {
                        float ss = 0.f;
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const uint4 q = yr[qd * 4 + i];
                            const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const float y0 = __uint_as_float(w4[e] << 16), y1 = __uint_as_float(w4[e] & 0xFFFF0000u);
                                ss += y0 * y0 + y1 * y1;
                            }
                        }
                        part[qd] = ss;
                    }
                    const float ss = (part[0] + part[1]) + (part[2] + part[3]);
                    const float nrm = 1.0f / sqrtf(ss / (float)DV + a.eps);
                    uint16_t* dst = a.out + (long long)(t0 + c * WC + et) * a.ld_out + (long long)hv * DV;
                    const bool vec = (reinterpret_cast<uintptr_t>(dst) & 15u) == 0;
                    const uint8_t* zrow = smem + R_Z + zb * 16384 + et * 16;   // feature chunk i at i * 1024
#pragma unroll 4
                    for (int i = 0; i < 16; ++i) {   // columns v = 8 i .. 8 i + 7
                        const uint4 q = yr[i];
                        const uint4 zz = *reinterpret_cast<const uint4*>(zrow + i * 1024);
                        const uint32_t yw[4] = {q.x, q.y, q.z, q.w}, zw[4] = {zz.x, zz.y, zz.z, zz.w};
                        uint32_t o[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            // bf16(bf16(bf16(y * nrm) * w) * z), two columns at once: the product of two bf16 values
                            // is exact in f32, so one bf16x2 multiply rounds exactly as f32 then bf16 does
                            const uint32_t yn = bf2_pack(__uint_as_float(yw[e] << 16) * nrm,
                                                         __uint_as_float(yw[e] & 0xFFFF0000u) * nrm);
                            o[e] = bf2_mul(zw[e], bf2_mul(yn, s_nw2[i * 4 + e]));
                        }
                        if (vec) {
                            *reinterpret_cast<uint4*>(dst + i * 8) = make_uint4(o[0], o[1], o[2], o[3]);
                        } else {
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                dst[i * 8 + 2 * e] = (uint16_t)(o[e] & 0xFFFFu);
                                dst[i * 8 + 2 * e + 1] = (uint16_t)(o[e] >> 16);
                            }
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(epi_free);
                // both epilogue warps are done with chunk c's z box: chunk c + 2's streams into it
                named_bar_sync(2, WY_EPI_THREADS);
                if (warp == WY_EPI_WARP && c + 2 < n_chunks) {
                    if (elect_one()) issue_z(c + 2);
                    __syncwarp();
                }
                if (c + 1 < n_chunks) z_ok = take_z(c + 1);   // while the compute warps finish chunk c + 1's y
            }
        }
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    }

    if (warp == WY_ISSUER_WARP) {   // no MMA of the issuing warp is in flight when the CTA ends
        if (elect_one()) umma_commit(bar_fin);
        __syncwarp();
        mbar_wait_bounded(bar_fin, 0, WY_WAIT_NS);
    }
    // no copy lands after the CTA ends: each issuing thread waits (bounded) for the last phase it issued on each
    // barrier, which has long completed unless a wait gave up
    for (int bit = 0; bit < 7; ++bit)
        if ((cp_any >> bit) & 1u) {
            uint64_t* b = bit < 2    ? bar_in + bit
                          : bit == 2 ? bar_v
                          : bit == 3 ? bar_tb
                          : bit == 6 ? bar_tp
                                     : bar_z + (bit - 4);
            mbar_wait_bounded(b, ((cp_next >> bit) & 1u) ^ 1u, WY_WAIT_NS);
        }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 512);
}

static int g_wy_sms[64] = {0};

cudaError_t launch_wy(const RecurArgs& r, cudaStream_t stream) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!r.wy_counter || !r.wy_tiles || !r.wy_cb || !r.wy_plan || !r.wy_chunks) return cudaErrorInvalidValue;
    if (g_wy_sms[dev] == 0) {
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(gdn_wy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, WY_SMEM);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(gdn_wy_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, A_SMEM);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(gdn_wy_chunk_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 (int)cudaSharedmemCarveoutMaxShared);
        if (e != cudaSuccess) return e;
        g_wy_sms[dev] = sms;
    }
    const int n_items = r.n_seq * r.hv;
    if (n_items == 0) return cudaSuccess;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t c = {};
    c.stream = stream;
    c.attrs = attr;
    c.numAttrs = 1;
    c.gridDim = dim3(1, 1, 1);
    c.blockDim = dim3(WP_THREADS, 1, 1);
    e = cudaLaunchKernelEx(&c, gdn_wy_plan_kernel, r);
    if (e != cudaSuccess) return e;
    c.gridDim = dim3((unsigned)(2 * g_wy_sms[dev]), 1, 1);
    c.blockDim = dim3(WA_THREADS, 1, 1);
    c.dynamicSmemBytes = A_SMEM;
    e = cudaLaunchKernelEx(&c, gdn_wy_chunk_kernel, r);
    if (e != cudaSuccess) return e;
    // the sequential pass reads each chunk's Q, K, V and gates from the records by TMA, and z from the caller's
    // tensor (one "record" of ld_z elements per token, one head) when its rows are 16-byte aligned
    CUtensorMap tm_rec, tm_gate, tm_z;
    if (!tmap_records(&tm_rec, r.recs, r.n_tokens, r.rec_cap, r.hv, REC_BYTES, WC, 16) ||
        !tmap_records(&tm_gate, r.recs, r.n_tokens, r.rec_cap, r.hv, REC_BYTES, WC, 1))
        return cudaErrorNotSupported;
    if (r.z) {
        if (!wy_z_direct(r.z, r.ld_z) || r.ld_z < (long long)r.hv * DV ||
            !tmap_records(&tm_z, r.z, r.n_tokens, r.n_tokens, 1, (int)(r.ld_z * 2), WC, 16))
            return cudaErrorNotSupported;
    } else {
        tm_z = tm_rec;   // not read
    }
    c.gridDim = dim3((unsigned)(n_items < g_wy_sms[dev] ? n_items : g_wy_sms[dev]), 1, 1);
    c.blockDim = dim3(WY_BLOCK, 1, 1);
    c.dynamicSmemBytes = WY_SMEM;
    return cudaLaunchKernelEx(&c, gdn_wy_kernel, r, tm_rec, tm_gate, tm_z);
}

}  // namespace gdn
