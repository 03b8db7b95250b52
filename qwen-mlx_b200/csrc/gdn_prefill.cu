// gdn_prefill.cu -- chunked (WY) gated delta rule on tcgen05 tensor cores for the
// multi-token sequences of a packed step (sm_100a).
//
// The recurrence of metal_gdn.rs:37-62, S_t = g_t S_{t-1} + d_t k_t^T with
// d_t = beta_t (v_t - g_t S_{t-1} k_t) and y_t = S_t q_t, is evaluated 64 tokens
// at a time.  With lg_t = sum_{j<=t} log g_j inside the chunk, gamma_t = exp(lg_t)
// and S0 the state entering the chunk:
//   G = K K^T, QK = Q K^T                                (tensor cores, exact bf16 inputs)
//   M[t][s] = beta_t exp(lg_t - lg_s) G[t][s]  (s < t),  T = (I + M)^-1   (CUDA cores)
//   U = T diag(beta) V,  W = T diag(beta gamma) K          (tensor cores)
//   D = U - W S0^T                                        (the chunk's rank-1 update vectors)
//   Y = diag(gamma) Q S0^T + P (.) QK D,  P[t][s] = exp(lg_t - lg_s) (s <= t)
//   S_C = gamma_C S0 + D^T diag(exp(lg_C - lg_s)) K
// f32 operands (T, W, S0, D, P (.) QK) enter the bf16 MMAs as hi + lo bf16 pairs
// (hi = bf16(x), lo = bf16(x - hi)); products of two split operands drop lo*lo.
// The f32 state S lives in TMEM for the whole sequence: each chunk scales it by
// gamma_C in place and the state-update MMA accumulates onto it.  The epilogue
// rounds y to bf16 (metal_gdn.rs:54) and applies silu(z) * rms_norm(y, norm_w, eps)
// (qwen3_5.rs:660-665) on the row each thread owns.  Decays stay in log space, so
// long chunks of strong decay cannot underflow into 0/0.
//
// One CTA (128 threads, 4 warps) per (sequence, v-head) item at a time, persistent
// over the items whose segment has at least WY_MIN_T tokens; shorter segments stay
// on the token-sequential recurrence kernel.  Inputs are the prep kernel's records.
//
// Shared memory (bytes), K-major bf16 tiles in the layout of gdn_umma.cuh; regions are
// reused once their last reader (an MMA waited on, or a barrier) is done:
//   R_K   16K  K [64 t][128 d]            -> W_hi [64 t][128 d]
//   R_Q   16K  Q [64 t][128 d]
//   R_KT  16K  K^T [128 d][64 s]
//   R_VT  16K  V^T [128 v][64 s]          -> W_lo
//   R_M   16K  M f32 [64][64]             -> D^T hi [128 v][64 s]
//   R_T   16K  T f32 [64][64]             -> D^T lo
//   R_P   16K  (P(.)QK) hi, lo [64 t][64 s]
//   R_TB  32K  (T beta) hi, lo; (T beta gamma) hi, lo [64 t][64 s] -> Dd^T hi, lo [128 v][64 s]
//   R_S   64K  S0 hi, lo [128 v][128 d]
// TMEM (512 columns): S [0,128) (M=128 layout), A [128,256), B [256,384), C [384,512)
// (M=64 accumulators: row t in lane 32*(t/16) + t%16).
#include "gdn_device.cuh"
#include "gdn_internal.h"
#include "gdn_ptx.cuh"
#include "gdn_umma.cuh"

namespace gdn {

constexpr int WC = 64;                 // tokens per chunk
constexpr int WY_THREADS = 128;
constexpr int R_K = 0, R_Q = 16384, R_KT = 32768, R_VT = 49152, R_M = 65536, R_T = 81920, R_P = 98304,
              R_TB = 114688, R_S = 147456, R_SMALL = 212992;
constexpr int WY_SMEM = R_SMALL + 4 * 64 * 4 + 128 * 4 + 64;
static_assert(WY_SMEM <= 232448, "prefill shared memory budget");
constexpr uint32_t TM_S = 0, TM_A = 128, TM_B = 256, TM_C = 384;
constexpr uint64_t WY_WAIT_NS = 2000000000ull;

__device__ __forceinline__ void split_bf16(float x, uint16_t& hi, uint16_t& lo) {
    hi = f2bf(x);
    lo = f2bf(x - bf2f(hi));
}

__device__ __forceinline__ void st_bf16(uint8_t* base, uint32_t off, uint16_t v) {
    *reinterpret_cast<uint16_t*>(base + off) = v;
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

__global__ void __launch_bounds__(WY_THREADS, 1) gdn_wy_kernel(const RecurArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    float* s_beta = reinterpret_cast<float*>(smem + R_SMALL);
    float* s_lg = s_beta + 64;
    float* s_gam = s_lg + 64;      // exp(lg_t)
    float* s_tail = s_gam + 64;    // exp(lg_last - lg_t)
    float* s_nw = s_tail + 64;     // norm_w [128]
    uint64_t* bar = reinterpret_cast<uint64_t*>(s_nw + 128);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
    volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t sbase = smem_u32(smem);
    const int n_items = a.n_seq * a.hv;
    const int ratio = a.hv / a.hk;

    if (tid == 0) {
        mbar_init(bar, 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    for (int i = tid; i < DV; i += WY_THREADS) s_nw[i] = bf2f(a.norm_w[i]);
    if (warp == 0) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    uint32_t ph = 0;
    pdl_wait();

    // M=64 accumulator row owned by this thread (lanes 0..15 of each warp)
    const bool row_thread = lane < 16;
    const int trow = warp * 16 + (lane & 15);

    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int seq = item / a.hv;
        const int hv = item - seq * a.hv;
        const int t0 = __ldg(a.cu_seqlens + seq);
        const int T = __ldg(a.cu_seqlens + seq + 1) - t0;
        const int slot = __ldg(a.slot_ids + seq);
        if (slot < 0 || slot >= a.n_slots || T < a.wy_min_t || t0 < 0 || t0 + T > a.n_tokens) continue;
        if (*s_abort) break;
        float* st = a.rec + ((size_t)slot * a.hv + hv) * (DV * DK);
        const float* st_in = (a.rec_in ? a.rec_in : a.rec) + ((size_t)slot * a.hv + hv) * (DV * DK);

        // ---- state -> TMEM S (thread v owns row v)
        {
            const float* src = st_in + (size_t)tid * DK;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float v[16];
#pragma unroll
                for (int e = 0; e < 16; e += 4) {
                    const float4 f = __ldcs(reinterpret_cast<const float4*>(src + j * 16 + e));
                    v[e] = f.x; v[e + 1] = f.y; v[e + 2] = f.z; v[e + 3] = f.w;
                }
                tmem_st16(tmem + lane_base + TM_S + j * 16, v);
            }
            tmem_st_wait();
        }

        const int n_chunks = (T + WC - 1) / WC;
        for (int c = 0; c < n_chunks && !*s_abort; ++c) {
            const int n0 = t0 + c * WC;
            const int nv = (T - c * WC) < WC ? (T - c * WC) : WC;
            const uint8_t* rec0 = a.recs + ((long long)hv * a.rec_cap + n0) * REC_BYTES;

            // ---- phase A: the chunk's K, Q (K-major), K^T, V^T, beta, log-decay
            for (int i = tid; i < WC * 16; i += WY_THREADS) {
                const int t = i >> 4, ch = i & 15;
                uint4 qv = make_uint4(0, 0, 0, 0), kv = qv, vv = qv;
                if (t < nv) {
                    const uint8_t* r = rec0 + (size_t)t * REC_BYTES;
                    qv = *reinterpret_cast<const uint4*>(r + ch * 16);
                    kv = *reinterpret_cast<const uint4*>(r + 256 + ch * 16);
                    vv = *reinterpret_cast<const uint4*>(r + 512 + ch * 16);
                }
                *reinterpret_cast<uint4*>(smem + R_Q + umma_tile_off(t, ch * 8, 128)) = qv;
                *reinterpret_cast<uint4*>(smem + R_K + umma_tile_off(t, ch * 8, 128)) = kv;
                const uint16_t* k8 = reinterpret_cast<const uint16_t*>(&kv);
                const uint16_t* v8 = reinterpret_cast<const uint16_t*>(&vv);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    st_bf16(smem + R_KT, umma_tile_off(ch * 8 + e, t, 64), k8[e]);
                    st_bf16(smem + R_VT, umma_tile_off(ch * 8 + e, t, 64), v8[e]);
                }
            }
            if (tid < WC) {
                float b = 0.f, ld = 0.f;
                if (tid < nv) {
                    const float* gb = reinterpret_cast<const float*>(rec0 + (size_t)tid * REC_BYTES + 1024);
                    b = gb[1];
                    ld = gb[2];
                }
                s_beta[tid] = b;
                s_lg[tid] = ld;
            }
            __syncthreads();
            if (tid == 0) {
                float acc = 0.f;
                for (int t = 0; t < WC; ++t) {
                    acc += s_lg[t];
                    s_lg[t] = acc;
                }
            }
            __syncthreads();
            if (tid < WC) {
                s_gam[tid] = expf(s_lg[tid]);
                s_tail[tid] = expf(s_lg[WC - 1] - s_lg[tid]);
            }
            wy_sync_for_mma();

            // ---- phase B: G = K K^T -> A[0,64), QK = Q K^T -> A[64,128)
            if (tid == 0) {
                const uint32_t id = umma_idesc_bf16(64, 64);
                for (int ks = 0; ks < 8; ++ks)
                    umma_bf16(tmem + TM_A, umma_desc(sbase + R_K, 128, ks), umma_desc(sbase + R_K, 128, ks), id, ks > 0);
                for (int ks = 0; ks < 8; ++ks)
                    umma_bf16(tmem + TM_A + 64, umma_desc(sbase + R_Q, 128, ks), umma_desc(sbase + R_K, 128, ks), id,
                              ks > 0);
                umma_commit(bar);
            }
            if (!wy_wait(bar, ph)) { atomicOr(a.err, ERR_TIMEOUT); *s_abort = 1; }

            // ---- phase C1: M (f32) and P (.) QK (hi/lo) from this thread's row
            {
                float* fM = reinterpret_cast<float*>(smem + R_M);
                const float lg_t = s_lg[trow];
                const float b_t = s_beta[trow];
                for (int j = 0; j < 4; ++j) {
                    float gv[16], qv[16];
                    tmem_ld16(tmem + lane_base + TM_A + j * 16, gv);
                    tmem_ld16(tmem + lane_base + TM_A + 64 + j * 16, qv);
                    if (row_thread) {
#pragma unroll
                        for (int e = 0; e < 16; ++e) {
                            const int s = j * 16 + e;
                            const float dec = expf(lg_t - s_lg[s]);
                            fM[trow * 64 + s] = s < trow ? b_t * dec * gv[e] : 0.f;
                            uint16_t hi, lo;
                            split_bf16(s <= trow ? dec * qv[e] : 0.f, hi, lo);
                            st_bf16(smem + R_P, umma_tile_off(trow, s, 64), hi);
                            st_bf16(smem + R_P + 8192, umma_tile_off(trow, s, 64), lo);
                        }
                    }
                }
            }
            // ---- phase C2: S0 hi/lo from TMEM (row v = tid); S *= gamma_last in place
            {
                const float g_last = s_gam[WC - 1];
                for (int j = 0; j < 8; ++j) {
                    float sv[16];
                    tmem_ld16(tmem + lane_base + TM_S + j * 16, sv);
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        uint16_t hi, lo;
                        split_bf16(sv[e], hi, lo);
                        st_bf16(smem + R_S, umma_tile_off(tid, j * 16 + e, 128), hi);
                        st_bf16(smem + R_S + 32768, umma_tile_off(tid, j * 16 + e, 128), lo);
                        sv[e] *= g_last;
                    }
                    tmem_st16(tmem + lane_base + TM_S + j * 16, sv);
                }
                tmem_st_wait();
            }
            __syncthreads();

            // ---- phase C3: T = (I + M)^-1, column s by the lane pair (2s, 2s+1)
            {
                const float* fM = reinterpret_cast<const float*>(smem + R_M);
                float* fT = reinterpret_cast<float*>(smem + R_T);
                const int s = tid >> 1, p = tid & 1;
                if (p == 0) fT[s * 64 + s] = 1.f;
                __syncwarp();
                for (int t = 1; t < WC; ++t) {
                    float acc = 0.f;
                    if (t > s)
                        for (int j = s + p; j < t; j += 2) acc += fM[t * 64 + j] * fT[j * 64 + s];
                    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
                    if (t > s && p == 0) fT[t * 64 + s] = -acc;
                    __syncwarp();
                }
            }
            __syncthreads();
            // ---- phase C4: (T beta) and (T beta gamma) as hi/lo bf16 tiles
            {
                const float* fT = reinterpret_cast<const float*>(smem + R_T);
                for (int i = tid; i < WC * WC; i += WY_THREADS) {
                    const int t = i >> 6, s = i & 63;
                    const float x = s <= t ? fT[t * 64 + s] : 0.f;
                    const float tb = x * s_beta[s];
                    uint16_t hi, lo;
                    split_bf16(tb, hi, lo);
                    st_bf16(smem + R_TB, umma_tile_off(t, s, 64), hi);
                    st_bf16(smem + R_TB + 8192, umma_tile_off(t, s, 64), lo);
                    split_bf16(tb * s_gam[s], hi, lo);
                    st_bf16(smem + R_TB + 16384, umma_tile_off(t, s, 64), hi);
                    st_bf16(smem + R_TB + 24576, umma_tile_off(t, s, 64), lo);
                }
            }
            wy_sync_for_mma();

            // ---- phase D: U = (T beta) V -> B;  W = (T beta gamma) K -> C
            if (tid == 0) {
                const uint32_t id = umma_idesc_bf16(64, 128);
                for (int h = 0; h < 2; ++h)
                    for (int ks = 0; ks < 4; ++ks)
                        umma_bf16(tmem + TM_B, umma_desc(sbase + R_TB + h * 8192, 64, ks), umma_desc(sbase + R_VT, 64, ks),
                                  id, (h | ks) != 0);
                for (int h = 0; h < 2; ++h)
                    for (int ks = 0; ks < 4; ++ks)
                        umma_bf16(tmem + TM_C, umma_desc(sbase + R_TB + 16384 + h * 8192, 64, ks),
                                  umma_desc(sbase + R_KT, 64, ks), id, (h | ks) != 0);
                umma_commit(bar);
            }
            if (!wy_wait(bar, ph)) { atomicOr(a.err, ERR_TIMEOUT); *s_abort = 1; }

            // ---- phase E: W hi/lo tiles; then W S0^T -> A and Q S0^T -> C
            for (int j = 0; j < 8; ++j) {
                float wv[16];
                tmem_ld16(tmem + lane_base + TM_C + j * 16, wv);
                if (row_thread) {
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        uint16_t hi, lo;
                        split_bf16(wv[e], hi, lo);
                        st_bf16(smem + R_K, umma_tile_off(trow, j * 16 + e, 128), hi);
                        st_bf16(smem + R_VT, umma_tile_off(trow, j * 16 + e, 128), lo);
                    }
                }
            }
            wy_sync_for_mma();
            if (tid == 0) {
                const uint32_t id = umma_idesc_bf16(64, 128);
                const uint32_t aw[3] = {R_K, R_K, R_VT}, bs[3] = {R_S, R_S + 32768, R_S};
                for (int p = 0; p < 3; ++p)
                    for (int ks = 0; ks < 8; ++ks)
                        umma_bf16(tmem + TM_A, umma_desc(sbase + aw[p], 128, ks), umma_desc(sbase + bs[p], 128, ks), id,
                                  (p | ks) != 0);
                for (int h = 0; h < 2; ++h)
                    for (int ks = 0; ks < 8; ++ks)
                        umma_bf16(tmem + TM_C, umma_desc(sbase + R_Q, 128, ks), umma_desc(sbase + R_S + h * 32768, 128, ks),
                                  id, (h | ks) != 0);
                umma_commit(bar);
            }
            if (!wy_wait(bar, ph)) { atomicOr(a.err, ERR_TIMEOUT); *s_abort = 1; }

            // ---- phase F: D = U - W S0^T; D^T and Dd^T = D^T diag(exp(lg_last - lg_s)) as hi/lo tiles
            {
                const float tail = s_tail[trow];
                for (int j = 0; j < 8; ++j) {
                    float uv[16], wsv[16];
                    tmem_ld16(tmem + lane_base + TM_B + j * 16, uv);
                    tmem_ld16(tmem + lane_base + TM_A + j * 16, wsv);
                    if (row_thread) {
#pragma unroll
                        for (int e = 0; e < 16; ++e) {
                            const int v = j * 16 + e;
                            const float d = uv[e] - wsv[e];
                            uint16_t hi, lo;
                            split_bf16(d, hi, lo);
                            st_bf16(smem + R_M, umma_tile_off(v, trow, 64), hi);
                            st_bf16(smem + R_T, umma_tile_off(v, trow, 64), lo);
                            split_bf16(d * tail, hi, lo);
                            st_bf16(smem + R_TB, umma_tile_off(v, trow, 64), hi);
                            st_bf16(smem + R_TB + 16384, umma_tile_off(v, trow, 64), lo);
                        }
                    }
                }
            }
            wy_sync_for_mma();
            // ---- phase G: (P (.) QK) D -> B;  S += Dd^T K -> S
            if (tid == 0) {
                const uint32_t id64 = umma_idesc_bf16(64, 128);
                const uint32_t ap[3] = {R_P, R_P, R_P + 8192}, bd[3] = {R_M, R_T, R_M};
                for (int p = 0; p < 3; ++p)
                    for (int ks = 0; ks < 4; ++ks)
                        umma_bf16(tmem + TM_B, umma_desc(sbase + ap[p], 64, ks), umma_desc(sbase + bd[p], 64, ks), id64,
                                  (p | ks) != 0);
                const uint32_t id128 = umma_idesc_bf16(128, 128);
                for (int h = 0; h < 2; ++h)
                    for (int ks = 0; ks < 4; ++ks)
                        umma_bf16(tmem + TM_S, umma_desc(sbase + R_TB + h * 16384, 64, ks), umma_desc(sbase + R_KT, 64, ks),
                                  id128, 1u);
                umma_commit(bar);
            }
            if (!wy_wait(bar, ph)) { atomicOr(a.err, ERR_TIMEOUT); *s_abort = 1; }

            // ---- phase H: y = gamma_t Q S0^T + (P (.) QK) D, rounded to bf16; gated RMSNorm
            {
                const bool valid = row_thread && trow < nv;
                const float gam = s_gam[trow];
                float ss = 0.f;
                for (int j = 0; j < 8; ++j) {
                    float qs[16], pd[16];
                    tmem_ld16(tmem + lane_base + TM_C + j * 16, qs);
                    tmem_ld16(tmem + lane_base + TM_B + j * 16, pd);
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        const float y = rbf(gam * qs[e] + pd[e]);
                        ss += y * y;
                    }
                }
                const float nrm = 1.0f / sqrtf(ss / (float)DV + a.eps);
                const long long n = (long long)n0 + trow;
                const uint8_t* rec = rec0 + (size_t)trow * REC_BYTES;
                for (int j = 0; j < 8; ++j) {
                    float qs[16], pd[16];
                    tmem_ld16(tmem + lane_base + TM_C + j * 16, qs);
                    tmem_ld16(tmem + lane_base + TM_B + j * 16, pd);
                    if (valid) {
                        const uint4 z0 = *reinterpret_cast<const uint4*>(rec + 768 + j * 32);
                        const uint4 z1 = *reinterpret_cast<const uint4*>(rec + 768 + j * 32 + 16);
                        const uint16_t* zz0 = reinterpret_cast<const uint16_t*>(&z0);
                        const uint16_t* zz1 = reinterpret_cast<const uint16_t*>(&z1);
                        uint16_t o[16];
#pragma unroll
                        for (int e = 0; e < 16; ++e) {
                            const float y = rbf(gam * qs[e] + pd[e]);
                            const float yn = rbf(rbf(y * nrm) * s_nw[j * 16 + e]);
                            const float zs = bf2f(e < 8 ? zz0[e] : zz1[e - 8]);
                            o[e] = f2bf(zs * yn);
                        }
                        uint16_t* dst = a.out + n * a.ld_out + (long long)hv * DV + j * 16;
#pragma unroll
                        for (int e = 0; e < 16; ++e) dst[e] = o[e];
                    }
                }
            }
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
        }

        // ---- state back to the pool (row v = tid)
        {
            float* dst = st + (size_t)tid * DK;
            for (int j = 0; j < 8; ++j) {
                float v[16];
                tmem_ld16(tmem + lane_base + TM_S + j * 16, v);
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
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
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
    if (g_wy_sms[dev] == 0) {
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(gdn_wy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, WY_SMEM);
        if (e != cudaSuccess) return e;
        g_wy_sms[dev] = sms;
    }
    const int n_items = r.n_seq * r.hv;
    if (n_items == 0) return cudaSuccess;
    const int grid = n_items < g_wy_sms[dev] ? n_items : g_wy_sms[dev];
    gdn_wy_kernel<<<grid, WY_THREADS, WY_SMEM, stream>>>(r);
    return cudaGetLastError();
}

}  // namespace gdn
