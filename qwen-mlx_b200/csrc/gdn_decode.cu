// gdn_decode.cu -- the fused GDN layer step as two kernels chained with
// programmatic dependent launch (sm_100a).
//
// K1 gdn_prep_kernel (token-parallel, small; its tiled forms serve calls with multi-token
//    segments: gdn_prep_vec_kernel, 8 channels per lane, when rows allow 16-byte access, else
//    gdn_prep_tile_kernel, 2 channels per thread): for every packed token and
//    k-head group, the causal depthwise conv + SiLU of its q, k and v channels
//    (reference rounding: S=1 -> bf16 products and bf16 sum, qwen3_5.rs:602-610;
//    S>1 -> f32 conv1d, qwen3_5.rs:617-623), q/k RMSNorm with gains 1/dk and
//    bf16(dk^-1/2) (qwen3_5.rs:636-639), beta and g (compiled_ops.rs:30-43) and
//    silu(z) (qwen3_5.rs:664).  It writes one 1056-byte record per (v-head,
//    token) into the pool's scratch: q | k | v | silu(z) (bf16 x 128 each) |
//    g (f32) | beta (f32 holding the bf16 value) | log g (f32) | pad.  K1 reads
//    the conv state, and shifts the windows of one-token sequences in place.
// K2 gdn_recur_kernel (persistent, one CTA per SM): work item = (sequence,
//    v-head).  A producer warp streams each item's 64 KiB f32 state tile
//    ([dv][dk], metal_gdn.rs:25-26) and its token records into a 3-stage
//    shared-memory ring with bulk async copies completing on mbarriers; 8
//    consumer warps pull the tile into registers (warp w: rows 16w..16w+15,
//    lane l: columns 4l..4l+3), run the gated delta rule per token
//    (metal_gdn.rs:37-62), write the gated RMSNorm output silu(z) *
//    rms_norm(y, norm_w, eps) (qwen3_5.rs:660-665), store the tile back with
//    128-bit evict-first stores, and write the conv-state windows back (the
//    v channels of the item's head, and the q/k channels when the head is the
//    first of its k-head group).  K1 has completed before any K2 write
//    (griddepcontrol.wait), so no window is overwritten before it is read.
//
// PDL: K1 waits for its predecessor before touching memory, then lets K2
// launch; K2 starts streaming state tiles (which K1 never touches) before its
// own griddepcontrol.wait and only reads K1's records after it.
#include "gdn_device.cuh"
#include "gdn_internal.h"
#include "gdn_ptx.cuh"

namespace gdn {

constexpr int K2_CONSUMER_WARPS = 8;
constexpr int K2_CONSUMERS = K2_CONSUMER_WARPS * 32;
constexpr int K2_THREADS = K2_CONSUMERS + 32;
constexpr int NSTAGE = 3;
constexpr int TILE_BYTES = DV * DK * 4;                               // 65536
constexpr int STAGE_BYTES = TILE_BYTES + REC_PER_STAGE * REC_BYTES;   // 73856
constexpr int K2_SMEM = NSTAGE * STAGE_BYTES + 2 * NSTAGE * 8 + NSTAGE * 16 + 2 * DV * 4 + 4 * 4;
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;                     // 2 s bound on every wait
static_assert(STAGE_BYTES % 16 == 0, "stage alignment");
static_assert(K2_SMEM <= 232448, "shared memory budget");

// ------------------------------------------------------------------ K1

// Sequence owning packed token n: cu[i] <= n < cu[i+1] (binary search).  -1 if the tables do not cover n.
__device__ __forceinline__ int find_seq(const int32_t* __restrict__ cu, int n_seq, int n) {
    int lo = 0, hi = n_seq;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (__ldg(cu + mid) <= n) lo = mid; else hi = mid;
    }
    if (n_seq <= 0 || __ldg(cu + lo) > n || __ldg(cu + lo + 1) <= n) return -1;
    return lo;
}

__device__ __forceinline__ void unpack_w4(uint2 wu, float (&w)[4]) {
    w[0] = __uint_as_float(wu.x << 16);
    w[1] = __uint_as_float(wu.x & 0xffff0000u);
    w[2] = __uint_as_float(wu.y << 16);
    w[3] = __uint_as_float(wu.y & 0xffff0000u);
}

// nn::silu for the prefill tiles: sigmoid from the fast exponential and divide intrinsics (a few ulp in f32).
// The result is rounded to bf16, so it can differ from silu_bf only when the f32 value lies within a few ulp
// of a bf16 rounding boundary (about 1 output in 10^4, by one bf16 ulp).
__device__ __forceinline__ float silu_bf_fast(float x) { return rbf(x * __fdividef(1.0f, 1.0f + __expf(-x))); }

// silu(sum_j w[j] * x[j]) with the conv1d (f32) rounding, fast SiLU (prefill tiles).
__device__ __forceinline__ float conv_silu_fast(const float (&x)[4], const float (&w)[4]) {
    float acc = x[0] * w[0];
    acc = acc + x[1] * w[1];
    acc = acc + x[2] * w[2];
    acc = acc + x[3] * w[3];
    return silu_bf_fast(rbf(acc));
}

// silu(sum_j w[j] * x[j]) with the reference's decode (bf16 products + bf16 sum) or conv1d (f32) rounding.
__device__ __forceinline__ float conv_silu(const float (&x)[4], const float (&w)[4], bool decode) {
    float acc;
    if (decode) {
        acc = rbf(x[0] * w[0]);
        acc = acc + rbf(x[1] * w[1]);
        acc = acc + rbf(x[2] * w[2]);
        acc = acc + rbf(x[3] * w[3]);
    } else {
        acc = x[0] * w[0];
        acc = acc + x[1] * w[1];
        acc = acc + x[2] * w[2];
        acc = acc + x[3] * w[3];
    }
    return silu_bf(rbf(acc));
}

// Conv taps x[0..3] = padded[t..t+3] of channel ch, padded = [conv window (K-1 rows); tokens].
// x[3] (the current token) is passed in; the window rows come from `cs` or from earlier tokens.
__device__ __forceinline__ void load_taps(const PrepArgs& a, const uint16_t* cs, int ch, int t0, int t, float xcur,
                                          float (&x)[4]) {
#pragma unroll
    for (int j = 0; j < KC - 1; ++j) {
        const int p = t + j;
        x[j] = p < KC - 1 ? bf2f(cs[(size_t)p * a.D + ch]) : bf2f(a.qkv[(long long)(t0 + p - (KC - 1)) * a.ld_qkv + ch]);
    }
    x[KC - 1] = xcur;
}

// One CTA per (packed token, k-head); 256 threads = 128 q + 128 k channels, and the
// v channels / z columns of the k-head's v-heads (Hv/Hk * 128 of each).
// Loads are issued in two batches: everything indexed by the token (inputs, weights,
// and the routing entries of the sequence the token belongs to when each sequence
// has one token), then the slot's conv windows.  With a.tables_stable (the routing tables were
// complete before the preceding kernel started, and that kernel does not write this layer's conv
// state) the routing, weight and window loads are issued before the wait on the preceding kernel,
// which may still be running, and only the token inputs are read after it.
__global__ void __launch_bounds__(256) gdn_prep_kernel(const PrepArgs a) {
    const bool early = a.tables_stable != 0;
    if (!early) {
        pdl_wait();
        pdl_launch_dependents();
    }
    __shared__ float s_red[8];

    const int n = blockIdx.x;
    const int hk = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ratio = a.hv / a.hk;
    const bool low = tid < 128;
    const int c = tid & 127;
    const int qk_ch = (low ? 0 : a.hk * DK) + hk * DK + c;
    const int nv = ratio * DV;             // v channels of this k-head group
    const int v_idx0 = tid;                // first v channel handled by this thread (ratio <= 2: the only one)
    int v_ch = 0, v_hv = 0, v_c = 0;
    if (v_idx0 < nv) {
        v_hv = hk * ratio + v_idx0 / DV;
        v_c = v_idx0 % DV;
        v_ch = 2 * a.hk * DK + v_hv * DV + v_c;
    }

    // ---- batch 1: routing guess, weights (and, unless early, the token's inputs)
    const int guess = n < a.n_seq ? n : a.n_seq - 1;
    const int cu_g0 = __ldg(a.cu_seqlens + guess);
    const int cu_g1 = __ldg(a.cu_seqlens + guess + 1);
    const int slot_g = __ldg(a.slot_ids + guess);
    float w_qk[4];
    unpack_w4(__ldg(reinterpret_cast<const uint2*>(a.conv_w + (size_t)qk_ch * KC)), w_qk);
    float w_v[4] = {0.f, 0.f, 0.f, 0.f};
    if (v_idx0 < nv) unpack_w4(__ldg(reinterpret_cast<const uint2*>(a.conv_w + (size_t)v_ch * KC)), w_v);
    float gb_alog = 0.f, gb_dt = 0.f;
    if (tid < ratio) {
        gb_alog = a.A_log[hk * ratio + tid];
        gb_dt = a.dt_bias[hk * ratio + tid];
    }
    float x_qk = 0.f, x_v = 0.f, z_v = 0.f, gb_b = 0.f, gb_a = 0.f;
    auto load_inputs = [&]() {
        x_qk = bf2f(a.qkv[(long long)n * a.ld_qkv + qk_ch]);
        if (v_idx0 < nv) {
            x_v = bf2f(a.qkv[(long long)n * a.ld_qkv + v_ch]);
            z_v = bf2f(a.z[(long long)n * a.ld_z + (long long)v_hv * DV + v_c]);
        }
        if (tid < ratio) {
            const int hv = hk * ratio + tid;
            gb_b = bf2f(a.ab[(long long)n * a.ld_ab + hv]);
            gb_a = bf2f(a.ab[(long long)n * a.ld_ab + a.hv + hv]);
        }
    };
    if (!early) load_inputs();

    // ---- routing
    int seq, slot;
    if (cu_g0 <= n && n < cu_g1) {
        seq = guess;
        slot = slot_g;
    } else {
        seq = find_seq(a.cu_seqlens, a.n_seq, n);
        if (seq < 0) {
            if (tid == 0 && hk == 0) atomicOr(a.err, ERR_BAD_SEQLENS);
            return;
        }
        slot = __ldg(a.slot_ids + seq);
    }
    const int t0 = __ldg(a.cu_seqlens + seq);
    const int T = __ldg(a.cu_seqlens + seq + 1) - t0;
    if (slot < 0 || slot >= a.n_slots || t0 + T > a.n_tokens) {
        if (tid == 0 && hk == 0 && n == t0) atomicOr(a.err, slot < 0 || slot >= a.n_slots ? ERR_BAD_SLOT : ERR_BAD_SEQLENS);
        return;
    }
    const int t = n - t0;
    const bool decode = (T == 1);
    uint16_t* cs = a.conv + (size_t)slot * (KC - 1) * a.D;

    // ---- batch 2: conv windows (a one-token sequence's taps are its window rows and its input)
    float xq[4], xv[4] = {0.f, 0.f, 0.f, 0.f};
    if (decode) {
#pragma unroll
        for (int j = 0; j < KC - 1; ++j) xq[j] = bf2f(cs[(size_t)j * a.D + qk_ch]);
        if (v_idx0 < nv) {
#pragma unroll
            for (int j = 0; j < KC - 1; ++j) xv[j] = bf2f(cs[(size_t)j * a.D + v_ch]);
        }
    }
    if (early) {
        pdl_wait();
        pdl_launch_dependents();
        load_inputs();
    }
    if (decode) {
        xq[KC - 1] = x_qk;
        xv[KC - 1] = x_v;
    } else {
        load_taps(a, cs, qk_ch, t0, t, x_qk, xq);
        if (v_idx0 < nv) load_taps(a, cs, v_ch, t0, t, x_v, xv);
    }
    if (decode) {
        // A one-token sequence: this thread is the only reader of these windows in this call,
        // so it shifts them in place (new window = last K-1 rows of [old window; x]).
#pragma unroll
        for (int j = 0; j < KC - 1; ++j) cs[(size_t)j * a.D + qk_ch] = f2bf(xq[j + 1]);
        if (v_idx0 < nv) {
#pragma unroll
            for (int j = 0; j < KC - 1; ++j) cs[(size_t)j * a.D + v_ch] = f2bf(xv[j + 1]);
        }
    }

    // ---- q / k: conv, SiLU, RMSNorm with the scale folded into the gain
    const float o = conv_silu(xq, w_qk, decode);
    const float ss = warp_sum(o * o);
    if (lane == 0) s_red[warp] = ss;
    __syncthreads();
    const float tot = low ? (s_red[0] + s_red[1]) + (s_red[2] + s_red[3]) : (s_red[4] + s_red[5]) + (s_red[6] + s_red[7]);
    const float nrm = 1.0f / sqrtf(tot / (float)DK + 1e-6f);
    const float gain = low ? 0.0078125f : 0.08837890625f;  // bf16(1/128), bf16(128^-0.5)
    const uint16_t qk_val = f2bf(rbf(o * nrm) * gain);
    for (int j = 0; j < ratio; ++j) {
        uint8_t* rec = a.rec + ((long long)(hk * ratio + j) * a.rec_cap + n) * REC_BYTES;
        reinterpret_cast<uint16_t*>(rec)[(low ? 0 : 128) + c] = qk_val;
    }
    // ---- v and silu(z)
    if (v_idx0 < nv) {
        uint8_t* rec = a.rec + ((long long)v_hv * a.rec_cap + n) * REC_BYTES;
        reinterpret_cast<uint16_t*>(rec)[256 + v_c] = f2bf(conv_silu(xv, w_v, decode));
        reinterpret_cast<uint16_t*>(rec)[384 + v_c] = f2bf(silu_bf(z_v));
    }
    // groups wider than 256 v channels (Hv/Hk > 2): remaining channels, one pass each
    for (int idx = 256 + tid; idx < nv; idx += 256) {
        const int hv = hk * ratio + idx / DV;
        const int cv = idx % DV;
        const int ch = 2 * a.hk * DK + hv * DV + cv;
        float w4[4], x4[4];
        unpack_w4(__ldg(reinterpret_cast<const uint2*>(a.conv_w + (size_t)ch * KC)), w4);
        load_taps(a, cs, ch, t0, t, bf2f(a.qkv[(long long)n * a.ld_qkv + ch]), x4);
        if (decode) {
#pragma unroll
            for (int j = 0; j < KC - 1; ++j) cs[(size_t)j * a.D + ch] = f2bf(x4[j + 1]);
        }
        uint8_t* rec = a.rec + ((long long)hv * a.rec_cap + n) * REC_BYTES;
        reinterpret_cast<uint16_t*>(rec)[256 + cv] = f2bf(conv_silu(x4, w4, decode));
        reinterpret_cast<uint16_t*>(rec)[384 + cv] =
            f2bf(silu_bf(bf2f(a.z[(long long)n * a.ld_z + (long long)hv * DV + cv])));
    }
    // ---- gates (compiled_beta_g)
    if (tid < ratio) {
        const int hv = hk * ratio + tid;
        const float sp = gate_softplus(gb_a, gb_dt, a.dt_bf16);
        float* gb = reinterpret_cast<float*>(a.rec + ((long long)hv * a.rec_cap + n) * REC_BYTES + 1024);
        const float logdecay = -(expf(gb_alog) * sp);
        gb[0] = expf(logdecay);
        gb[1] = rbf(sigmoid_f32(gb_b));
        gb[2] = logdecay;  // log g, for the chunked prefill kernel
    }
}

// ------------------------------------------------------------------ K1, tiled

constexpr int PT_TOK = 16;  // packed tokens per tiled-prep CTA

__device__ __forceinline__ void unpack_pair(uint32_t u, float& lo, float& hi) {
    lo = __uint_as_float(u << 16);
    hi = __uint_as_float(u & 0xffff0000u);
}

__device__ __forceinline__ uint32_t pack_pair(float lo, float hi) {
    return (uint32_t)f2bf(lo) | ((uint32_t)f2bf(hi) << 16);
}

// Token loop of the tiled prep.  SIMPLE: every token of the tile sits at position >= 3 of a
// multi-token sequence, so no tap comes from the conv window and no token takes the decode
// rounding (nearly every prefill tile).
template <bool SIMPLE>
__device__ __forceinline__ void prep_tile_tokens(const PrepArgs& a, int ch, bool is_qk, bool has_pair, bool z_ok,
                                                 uint8_t* vrec, uint8_t* zrec, const float (&w)[2][4],
                                                 uint32_t (*s_x)[256], const uint32_t (*s_z)[128], const int* s_seq,
                                                 const int* s_t, const int* s_T, const int* s_slot,
                                                 float (*s_red)[PT_TOK]) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint32_t win[KC - 1] = {s_x[0][tid], s_x[1][tid], s_x[2][tid]};
#pragma unroll 1
    for (int j = 0; j < PT_TOK; ++j) {
        const uint32_t cur = s_x[j + KC - 1][tid];
        const bool valid = s_seq[j] >= 0;
        float o0 = 0.f, o1 = 0.f;
        if (valid) {
            if (has_pair) {
                uint32_t tap[KC] = {win[0], win[1], win[2], cur};
                bool decode = false;
                if (!SIMPLE) {
                    const int t = s_t[j];
                    decode = s_T[j] == 1;
                    uint16_t* cs = a.conv + (size_t)s_slot[j] * (KC - 1) * a.D;
#pragma unroll
                    for (int p = 0; p < KC - 1; ++p)
                        if (t + p < KC - 1) tap[p] = *reinterpret_cast<const uint32_t*>(cs + (size_t)(t + p) * a.D + ch);
                    if (decode) {
#pragma unroll
                        for (int p = 0; p < KC - 1; ++p)
                            *reinterpret_cast<uint32_t*>(cs + (size_t)p * a.D + ch) = tap[p + 1];
                    }
                }
                float x0[4], x1[4];
#pragma unroll
                for (int p = 0; p < KC; ++p) unpack_pair(tap[p], x0[p], x1[p]);
                if (SIMPLE) {
                    o0 = conv_silu_fast(x0, w[0]);
                    o1 = conv_silu_fast(x1, w[1]);
                } else {
                    o0 = conv_silu(x0, w[0], decode);
                    o1 = conv_silu(x1, w[1], decode);
                }
                if (!is_qk) *reinterpret_cast<uint32_t*>(vrec + (size_t)j * REC_BYTES) = pack_pair(o0, o1);
            }
            if (z_ok) {
                const uint32_t zp = s_z[j][tid >> 1];
                const float zv = __uint_as_float((tid & 1) ? (zp & 0xffff0000u) : (zp << 16));
                *reinterpret_cast<uint16_t*>(zrec + (size_t)j * REC_BYTES) = f2bf(SIMPLE ? silu_bf_fast(zv) : silu_bf(zv));
            }
        }
        if (is_qk) {
            // o0, o1 are bf16 values: park them exactly in this thread's spent row j
            s_x[j][tid] = pack_pair(o0, o1);
            const float ss = warp_sum(o0 * o0 + o1 * o1);
            if (lane == 0) s_red[warp][j] = ss;
        }
        win[0] = win[1];
        win[1] = win[2];
        win[2] = cur;
    }
}

// Tiled K1 for calls that carry multi-token segments: one CTA per (16 consecutive packed
// tokens, k-head), same records and rounding as gdn_prep_kernel.  Thread tid owns one bf16
// channel pair: threads 0..63 q pairs, 64..127 k pairs, 128..255 the v pairs of the k-head's
// v-heads (Hv/Hk <= 2); and z column tid of those heads.  The pair's 19 tap rows (3 before the
// tile) and the z pairs are fetched up front with cp.async into shared columns; a rolled
// token loop then slides a 3-row window through registers, so a tap row is read once per
// tile and the loop body stays small.  q / k outputs wait in the thread's own spent tap rows
// until the RMSNorm sums are known.  Needs qkv / z rows at 4-byte alignment.
__global__ void __launch_bounds__(256) gdn_prep_tile_kernel(const PrepArgs a) {
    pdl_wait();
    pdl_launch_dependents();
    __shared__ uint32_t s_x[PT_TOK + KC - 1][256];  // [row][thread]: rows n0-3 .. n0+15 of the pair
    __shared__ uint32_t s_z[PT_TOK][128];           // z pairs of the group, loaded by the v threads
    __shared__ int s_seq[PT_TOK], s_t[PT_TOK], s_T[PT_TOK], s_slot[PT_TOK];
    __shared__ float s_red[4][PT_TOK];

    const int n0 = blockIdx.x * PT_TOK;
    const int hk = blockIdx.y;
    const int tid = threadIdx.x;
    const int ratio = a.hv / a.hk;
    const bool is_qk = tid < 128, is_q = tid < 64;
    // this thread's channel pair
    int ch, v_hv = 0, v_c = 0;
    bool has_pair = true;
    if (is_qk) {
        ch = (is_q ? 0 : a.hk * DK) + hk * DK + 2 * (tid & 63);
    } else {
        const int vi = 2 * (tid - 128);
        has_pair = vi < ratio * DV;
        v_hv = hk * ratio + vi / DV;
        v_c = vi % DV;
        ch = 2 * a.hk * DK + v_hv * DV + v_c;
    }

    // ---- inputs of the pair: tap rows and z, asynchronously
    if (has_pair) {
#pragma unroll
        for (int r = 0; r < PT_TOK + KC - 1; ++r) {
            const int row = n0 - (KC - 1) + r;
            const bool ok = row >= 0 && row < a.n_tokens;
            cp_async4(smem_u32(&s_x[r][tid]), a.qkv + (ok ? (long long)row * a.ld_qkv + ch : 0), ok ? 4u : 0u);
        }
        if (!is_qk) {
#pragma unroll
            for (int j = 0; j < PT_TOK; ++j) {
                const bool ok = n0 + j < a.n_tokens;
                cp_async4(smem_u32(&s_z[j][tid - 128]),
                          a.z + (ok ? (long long)(n0 + j) * a.ld_z + (long long)v_hv * DV + v_c : 0), ok ? 4u : 0u);
            }
        }
    }
    cp_async_commit();

    // ---- routing of the tile's tokens (s_seq < 0: no such token, or a rejected sequence)
    bool simple_tok = true;
    if (tid < PT_TOK) {
        const int n = n0 + tid;
        int seq = -1, t = 0, T = 0, slot = -1;
        if (n < a.n_tokens) {
            const int guess = n < a.n_seq ? n : a.n_seq - 1;
            if (__ldg(a.cu_seqlens + guess) <= n && n < __ldg(a.cu_seqlens + guess + 1))
                seq = guess;
            else
                seq = find_seq(a.cu_seqlens, a.n_seq, n);
            if (seq < 0) {
                if (hk == 0) atomicOr(a.err, ERR_BAD_SEQLENS);
            } else {
                const int t0 = __ldg(a.cu_seqlens + seq);
                T = __ldg(a.cu_seqlens + seq + 1) - t0;
                slot = __ldg(a.slot_ids + seq);
                t = n - t0;
                if (slot < 0 || slot >= a.n_slots || t0 + T > a.n_tokens) {
                    if (hk == 0 && t == 0) atomicOr(a.err, slot < 0 || slot >= a.n_slots ? ERR_BAD_SLOT : ERR_BAD_SEQLENS);
                    seq = -1;
                }
            }
        }
        s_seq[tid] = seq;
        s_t[tid] = t;
        s_T[tid] = T;
        s_slot[tid] = slot;
        simple_tok = seq < 0 || (t >= KC - 1 && T > 1);
    }
    cp_async_wait_all();
    const bool simple = __syncthreads_and(simple_tok) != 0;

    float w[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    if (has_pair) {
        unpack_w4(__ldg(reinterpret_cast<const uint2*>(a.conv_w + (size_t)ch * KC)), w[0]);
        unpack_w4(__ldg(reinterpret_cast<const uint2*>(a.conv_w + (size_t)(ch + 1) * KC)), w[1]);
    }
    const bool z_ok = tid < ratio * DV;
    uint8_t* vrec = a.rec + ((long long)v_hv * a.rec_cap + n0) * REC_BYTES + 512 + 2 * v_c;
    uint8_t* zrec = a.rec + ((long long)(hk * ratio + tid / DV) * a.rec_cap + n0) * REC_BYTES + 768 + 2 * (tid % DV);

    // ---- conv + SiLU over the tile's tokens; v and silu(z) go straight to the records
    if (simple)
        prep_tile_tokens<true>(a, ch, is_qk, has_pair, z_ok, vrec, zrec, w, s_x, s_z, s_seq, s_t, s_T, s_slot, s_red);
    else
        prep_tile_tokens<false>(a, ch, is_qk, has_pair, z_ok, vrec, zrec, w, s_x, s_z, s_seq, s_t, s_T, s_slot, s_red);

    // ---- q / k RMSNorm with the scale folded into the gain
    if (is_qk) {
        named_bar_sync(1, 128);
        const float gain = is_q ? 0.0078125f : 0.08837890625f;  // bf16(1/128), bf16(128^-0.5)
        const int w0 = is_q ? 0 : 2;
        const int off = (is_q ? 0 : 256) + 4 * (tid & 63);
#pragma unroll 1
        for (int j = 0; j < PT_TOK; ++j) {
            if (s_seq[j] < 0) continue;
            const float tot = s_red[w0][j] + s_red[w0 + 1][j];
            const float nrm = 1.0f / sqrtf(tot / (float)DK + 1e-6f);
            float o0, o1;
            unpack_pair(s_x[j][tid], o0, o1);
            const uint32_t val = pack_pair(rbf(o0 * nrm) * gain, rbf(o1 * nrm) * gain);
            for (int r = 0; r < ratio; ++r) {
                uint8_t* rec = a.rec + ((long long)(hk * ratio + r) * a.rec_cap + n0 + j) * REC_BYTES;
                *reinterpret_cast<uint32_t*>(rec + off) = val;
            }
        }
    }
    // ---- gates (compiled_beta_g)
    for (int idx = tid; idx < PT_TOK * ratio; idx += 256) {
        const int j = idx / ratio;
        if (s_seq[j] < 0) continue;
        const int n = n0 + j;
        const int hv = hk * ratio + idx % ratio;
        const float b = bf2f(a.ab[(long long)n * a.ld_ab + hv]);
        const float av = bf2f(a.ab[(long long)n * a.ld_ab + a.hv + hv]);
        const float sp = gate_softplus(av, a.dt_bias[hv], a.dt_bf16);
        const float logdecay = -(expf(a.A_log[hv]) * sp);
        float* gb = reinterpret_cast<float*>(a.rec + ((long long)hv * a.rec_cap + n) * REC_BYTES + 1024);
        gb[0] = expf(logdecay);
        gb[1] = rbf(sigmoid_f32(b));
        gb[2] = logdecay;
    }
}

// ------------------------------------------------------------------ K1, 8-channel lanes

constexpr int PV_TOK = 16;                    // tokens per sub-tile (one sliding conv window per lane)
constexpr int PV_SUB = 1;                     // sub-tiles per CTA
constexpr int PV_RING = 4;                    // conv-window prefetch depth (tokens) of the general path
constexpr int PV_THREADS = PV_SUB * 96;       // per sub-tile: warp q | k, warp v, warp z
constexpr int PV_ROWS = PV_TOK + KC - 1;      // tap rows of a sub-tile (3 before it)
static_assert(PV_SUB * PV_TOK <= 32, "one warp routes the CTA's tokens");

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
    unpack_pair(u.x, f[0], f[1]);
    unpack_pair(u.y, f[2], f[3]);
    unpack_pair(u.z, f[4], f[5]);
    unpack_pair(u.w, f[6], f[7]);
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
    return make_uint4(pack_pair(f[0], f[1]), pack_pair(f[2], f[3]), pack_pair(f[4], f[5]), pack_pair(f[6], f[7]));
}

// Round 8 values to bf16 precision in place, two per conversion instruction (the conversions share the
// transcendental pipe with the SiLU's exponential and reciprocal, which bounds this kernel).
__device__ __forceinline__ void rbf8(float (&f)[8]) {
#pragma unroll
    for (int c = 0; c < 8; c += 2) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(f[c], f[c + 1]);
        const uint32_t u = *reinterpret_cast<const uint32_t*>(&h);
        f[c] = __uint_as_float(u << 16);
        f[c + 1] = __uint_as_float(u & 0xffff0000u);
    }
}

// Pack 8 values that are already bf16-exact (no rounding left to do): bit moves only.
__device__ __forceinline__ uint4 pack8_exact(const float (&f)[8]) {
    uint32_t u[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
        u[i] = (__float_as_uint(f[2 * i]) >> 16) | (__float_as_uint(f[2 * i + 1]) & 0xffff0000u);
    return make_uint4(u[0], u[1], u[2], u[3]);
}

// silu of 8 bf16-exact values (bf2_silu_fast, the same bits as the chunked pass's epilogue), rounded to bf16 in
// pairs.
__device__ __forceinline__ void silu8_fast(float (&f)[8]) {
#pragma unroll
    for (int c = 0; c < 8; c += 2) {
        const uint32_t w = bf2_silu_fast((__float_as_uint(f[c]) >> 16) | (__float_as_uint(f[c + 1]) & 0xFFFF0000u));
        f[c] = __uint_as_float(w << 16);
        f[c + 1] = __uint_as_float(w & 0xFFFF0000u);
    }
}

// The all-interior-token form of prep_vec_conv (every token at position >= 3 of a multi-token sequence: no
// window taps, no decode rounding), on f32 pairs: the conv as fma.rn.f32x2 in the scalar order (x0 w0 first,
// then + x1 w1, + x2 w2, + x3 w3), bf16 rounding and SiLU (bf2_silu_fast) per pair, the bf16 words stored as
// they come out.  QK: the RMSNorm sum of squares in channel order, normalise, round, gain, round, as before.
template <bool QK>
__device__ __forceinline__ void prep_vec_simple(const PrepArgs& a, bool active, int n0, int ratio, int hv0,
                                                int rec_off, const uint4* raw, const float (&w)[8][4],
                                                const int* s_seq) {
    const int lane = threadIdx.x & 31;
    uint64_t W[4][KC];   // [channel pair][tap]
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
        for (int k = 0; k < KC; ++k) W[p][k] = f2_pack(w[2 * p][k], w[2 * p + 1][k]);
    uint64_t xm[KC - 1][4];
#pragma unroll
    for (int r = 0; r < KC - 1; ++r) {
        const uint4 u = raw[r * 32];
        xm[r][0] = bf2_to_f2(u.x);
        xm[r][1] = bf2_to_f2(u.y);
        xm[r][2] = bf2_to_f2(u.z);
        xm[r][3] = bf2_to_f2(u.w);
    }
    const float gain = lane < 16 ? 0.0078125f : 0.08837890625f;  // bf16(1/128), bf16(128^-0.5)
    // unrolled by three, the window's length: the 3-row window rotates through registers without moves
    // (config 4: 43.9 -> 42.8 ms per step against an unroll of two; four measured 44.0)
#pragma unroll 3
    for (int j = 0; j < PV_TOK; ++j) {
        const uint4 u = raw[(j + KC - 1) * 32];
        const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
        uint64_t xc[4];
        uint32_t sw[4];   // silu(bf16(conv)) as bf16x2 words
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            xc[p] = bf2_to_f2(uw[p]);
            uint64_t acc = f2_mul(xm[0][p], W[p][0]);
            acc = f2_fma(xm[1][p], W[p][1], acc);
            acc = f2_fma(xm[2][p], W[p][2], acc);
            acc = f2_fma(xc[p], W[p][3], acc);
            sw[p] = bf2_silu_fast(f2_to_bf2(acc));
        }
        const bool valid = s_seq[j] >= 0;        // uniform over the warp
        if (QK) {
            float o[8];
#pragma unroll
            for (int p = 0; p < 4; ++p) {
                o[2 * p] = __uint_as_float(sw[p] << 16);
                o[2 * p + 1] = __uint_as_float(sw[p] & 0xFFFF0000u);
            }
            float ss = 0.f;
#pragma unroll
            for (int c = 0; c < 8; ++c) ss += o[c] * o[c];
#pragma unroll
            for (int m = 8; m > 0; m >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
            if (valid) {
                const float nrm = 1.0f / sqrtf(ss / (float)DK + 1e-6f);
                uint32_t vw[4];
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    const uint64_t v = bf2_to_f2(f2_to_bf2(f2_mul(f2_pack(o[2 * p], o[2 * p + 1]), f2_pack(nrm, nrm))));
                    vw[p] = f2_to_bf2(f2_mul(v, f2_pack(gain, gain)));
                }
                const uint4 val = make_uint4(vw[0], vw[1], vw[2], vw[3]);
                for (int r = 0; r < ratio; ++r)
                    *reinterpret_cast<uint4*>(a.rec + ((long long)(hv0 + r) * a.rec_cap + n0 + j) * REC_BYTES + rec_off) = val;
            }
        } else if (valid && active) {
            *reinterpret_cast<uint4*>(a.rec + ((long long)hv0 * a.rec_cap + n0 + j) * REC_BYTES + rec_off) =
                make_uint4(sw[0], sw[1], sw[2], sw[3]);
        }
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            xm[0][p] = xm[1][p];
            xm[1][p] = xm[2][p];
            xm[2][p] = xc[p];
        }
    }
}

// Conv + SiLU of one lane's 8 channels over the sub-tile's tokens.  raw[32 r] is tap row n0-3+r of the channels
// (r < 19, in the lane's shared-memory column).  QK: the lane's channels are q (lanes 0-15) or k (lanes 16-31) of
// the k-head; each token's RMSNorm sum is reduced over the 16 lanes of the half-warp and the normalised values go
// to the records of the k-head's v-heads.  Otherwise the channels are v channels of v-head `hv0` and go to that
// head's records.  SIMPLE: every token sits at position >= 3 of a multi-token sequence (no window taps, no decode
// rounding, fast SiLU), as in prep_tile_tokens.  Otherwise the conv-window rows of the tokens at positions < 3
// are fetched PV_RING tokens ahead into the lane's column of `ring` (PV_RING slots of 3 rows).
template <bool SIMPLE, bool QK>
__device__ __forceinline__ void prep_vec_conv(const PrepArgs& a, int ch, bool active, int n0, int ratio, int hv0,
                                              int rec_off, const uint4* raw, uint4* ring, const float (&w)[8][4],
                                              const int* s_seq, const int* s_t, const int* s_T, const int* s_slot) {
    const int lane = threadIdx.x & 31;
    // window rows of token jj (positions < 3 only) into ring slot jj % PV_RING; one commit group per token
    auto prefetch = [&](int jj) {
        if (jj < PV_TOK) {
            const int t = s_t[jj];
            if (s_seq[jj] >= 0 && active && t < KC - 1) {
                const uint16_t* cs = a.conv + (size_t)s_slot[jj] * (KC - 1) * a.D + ch;
#pragma unroll
                for (int p = 0; p < KC - 1; ++p)
                    if (t + p < KC - 1)
                        cp_async16(smem_u32(ring + ((jj % PV_RING) * (KC - 1) + p) * 32), cs + (size_t)(t + p) * a.D, 16u);
            }
        }
        cp_async_commit();
    };
    float xm[KC - 1][8];
    if (SIMPLE) {
#pragma unroll
        for (int p = 0; p < KC - 1; ++p) unpack8(raw[p * 32], xm[p]);
    } else {
#pragma unroll 1
        for (int jj = 0; jj < PV_RING; ++jj) prefetch(jj);
    }
#pragma unroll (SIMPLE ? 2 : 1)
    for (int j = 0; j < PV_TOK; ++j) {
        float xc[8];
        unpack8(raw[(j + KC - 1) * 32], xc);
        const bool valid = s_seq[j] >= 0;        // uniform over the warp
        float o[8];
        if (SIMPLE) {
            // conv_silu_fast for 8 channels, with the two bf16 roundings done in pairs
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                float acc = xm[0][c] * w[c][0];
                acc = acc + xm[1][c] * w[c][1];
                acc = acc + xm[2][c] * w[c][2];
                acc = acc + xc[c] * w[c][3];
                o[c] = acc;
            }
            rbf8(o);
            silu8_fast(o);
        } else {
            cp_async_wait_group<PV_RING - 1>();  // token j's window rows have landed
            const int t = s_t[j];
            const bool win = valid && active && t < KC - 1;
            const bool decode = valid && active && s_T[j] == 1;
            const uint4* rs = ring + (j % PV_RING) * (KC - 1) * 32;
            uint4 tap[KC - 1];
#pragma unroll
            for (int p = 0; p < KC - 1; ++p) tap[p] = win && t + p < KC - 1 ? rs[p * 32] : raw[(j + p) * 32];
            if (decode) {
                uint16_t* cs = a.conv + (size_t)s_slot[j] * (KC - 1) * a.D + ch;
                *reinterpret_cast<uint4*>(cs) = tap[1];
                *reinterpret_cast<uint4*>(cs + a.D) = tap[2];
                *reinterpret_cast<uint4*>(cs + 2 * (size_t)a.D) = raw[(j + KC - 1) * 32];
            }
            float x[KC - 1][8];
#pragma unroll
            for (int p = 0; p < KC - 1; ++p) unpack8(tap[p], x[p]);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const float x4[KC] = {x[0][c], x[1][c], x[2][c], xc[c]};
                o[c] = conv_silu(x4, w[c], decode);
            }
        }
        if (QK) {
            float ss = 0.f;
#pragma unroll
            for (int c = 0; c < 8; ++c) ss += o[c] * o[c];
#pragma unroll
            for (int m = 8; m > 0; m >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
            if (valid) {
                const float nrm = 1.0f / sqrtf(ss / (float)DK + 1e-6f);
                const float gain = lane < 16 ? 0.0078125f : 0.08837890625f;  // bf16(1/128), bf16(128^-0.5)
                float v[8];
#pragma unroll
                for (int c = 0; c < 8; ++c) v[c] = o[c] * nrm;
                rbf8(v);
#pragma unroll
                for (int c = 0; c < 8; ++c) v[c] *= gain;
                const uint4 val = pack8(v);
                for (int r = 0; r < ratio; ++r)
                    *reinterpret_cast<uint4*>(a.rec + ((long long)(hv0 + r) * a.rec_cap + n0 + j) * REC_BYTES + rec_off) = val;
            }
        } else if (valid && active) {
            *reinterpret_cast<uint4*>(a.rec + ((long long)hv0 * a.rec_cap + n0 + j) * REC_BYTES + rec_off) = pack8_exact(o);
        }
        if (SIMPLE) {
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                xm[0][c] = xm[1][c];
                xm[1][c] = xm[2][c];
                xm[2][c] = xc[c];
            }
        } else {
            prefetch(j + PV_RING);   // slot j % PV_RING was consumed above
        }
    }
    if (!SIMPLE) cp_async_wait_all();
}

// K1 for calls with multi-token segments when the inputs allow 16-byte access: same records, rounding and
// conv-window updates as gdn_prep_tile_kernel, with each lane owning 8 consecutive channels.  One CTA per
// (16 packed tokens, k-head): warp 0 takes the q channels (lanes 0-15) and k channels (lanes 16-31) of the
// k-head, warp 1 the v channels and warp 2 the z columns of its v-heads (lanes 16r .. 16r+15: v-head
// hk * Hv/Hk + r), and warp 2 also the gates.  A conv lane copies its 19 tap rows (16 bytes each) into its own
// shared-memory column up front and slides a 3-row window through a rolled token loop (an unrolled one
// overflows the instruction cache); a z lane loads its rows 8 at a time.
__global__ void __launch_bounds__(PV_THREADS, 6) gdn_prep_vec_kernel(const PrepArgs a) {
    pdl_wait();
    pdl_launch_dependents();
    __shared__ uint4 s_raw[PV_SUB][2][PV_ROWS][32];              // [sub-tile][q|k, v][tap row][lane]
    __shared__ uint4 s_ring[PV_SUB][2][PV_RING * (KC - 1)][32];  // conv-window rows of the general path
    __shared__ int s_seq[PV_SUB * PV_TOK], s_t[PV_SUB * PV_TOK], s_T[PV_SUB * PV_TOK], s_slot[PV_SUB * PV_TOK];
    __shared__ int s_simple[PV_SUB];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int sub = warp / 3, role = warp % 3;
    const int hk = blockIdx.y;
    const int ratio = a.hv / a.hk;
    const int nb = blockIdx.x * PV_SUB * PV_TOK;
    const int n0 = nb + sub * PV_TOK;
    const int half = lane >> 4, c8 = 8 * (lane & 15);
    const int hv0 = hk * ratio;
    const bool active = role == 0 || half < ratio;

    // ---- this lane's tap rows and weights, issued before the routing
    int ch = 0;
    float w[8][4];
    const uint4* col = &s_raw[sub][role < 2 ? role : 0][0][lane];
    uint4* ring = &s_ring[sub][role < 2 ? role : 0][0][lane];
    if (role < 2) {
        ch = role == 0 ? (half ? a.hk * DK : 0) + hk * DK + c8 : 2 * a.hk * DK + (hv0 + half) * DV + c8;
#pragma unroll
        for (int r = 0; r < PV_ROWS; ++r) {
            const int row = n0 - (KC - 1) + r;
            const bool ok = active && row >= 0 && row < a.n_tokens;
            cp_async16(smem_u32(col + r * 32), a.qkv + (ok ? (long long)row * a.ld_qkv + ch : 0), ok ? 16u : 0u);
        }
        cp_async_commit();
        const uint4* wp = reinterpret_cast<const uint4*>(a.conv_w + (size_t)ch * KC);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4 u = active ? __ldg(wp + i) : make_uint4(0u, 0u, 0u, 0u);
            unpack_w4(make_uint2(u.x, u.y), w[2 * i]);
            unpack_w4(make_uint2(u.z, u.w), w[2 * i + 1]);
        }
    }

    // ---- routing of the CTA's tokens (s_seq < 0: no such token, or a rejected sequence)
    if (warp == 0) {
        bool simple_tok = true;
        if (lane < PV_SUB * PV_TOK) {
            const int n = nb + lane;
            int seq = -1, t = 0, T = 0, slot = -1;
            if (n < a.n_tokens) {
                const int guess = n < a.n_seq ? n : a.n_seq - 1;
                if (__ldg(a.cu_seqlens + guess) <= n && n < __ldg(a.cu_seqlens + guess + 1))
                    seq = guess;
                else
                    seq = find_seq(a.cu_seqlens, a.n_seq, n);
                if (seq < 0) {
                    if (hk == 0) atomicOr(a.err, ERR_BAD_SEQLENS);
                } else {
                    const int t0 = __ldg(a.cu_seqlens + seq);
                    T = __ldg(a.cu_seqlens + seq + 1) - t0;
                    slot = __ldg(a.slot_ids + seq);
                    t = n - t0;
                    if (slot < 0 || slot >= a.n_slots || t0 + T > a.n_tokens) {
                        if (hk == 0 && t == 0)
                            atomicOr(a.err, slot < 0 || slot >= a.n_slots ? ERR_BAD_SLOT : ERR_BAD_SEQLENS);
                        seq = -1;
                    }
                }
            }
            s_seq[lane] = seq;
            s_t[lane] = t;
            s_T[lane] = T;
            s_slot[lane] = slot;
            simple_tok = seq < 0 || (t >= KC - 1 && T > 1);
        }
        const unsigned bits = __ballot_sync(0xffffffffu, simple_tok);
        if (lane < PV_SUB) s_simple[lane] = ((bits >> (lane * PV_TOK)) & 0xffffu) == 0xffffu;
    }
    __syncthreads();

    const int* q_seq = s_seq + sub * PV_TOK;
    const int* q_t = s_t + sub * PV_TOK;
    const int* q_T = s_T + sub * PV_TOK;
    const int* q_slot = s_slot + sub * PV_TOK;
    const bool simple = s_simple[sub] != 0;
    if (role < 2) cp_async_wait_all();       // the lane's own column: no barrier needed
    if (role == 0) {
        const int off = (half ? 256 : 0) + 2 * c8;
        if (simple)
            prep_vec_simple<true>(a, true, n0, ratio, hv0, off, col, w, q_seq);
        else
            prep_vec_conv<false, true>(a, ch, true, n0, ratio, hv0, off, col, ring, w, q_seq, q_t, q_T, q_slot);
    } else if (role == 1) {
        const int off = 512 + 2 * c8;
        if (simple)
            prep_vec_simple<false>(a, active, n0, ratio, hv0 + half, off, col, w, q_seq);
        else
            prep_vec_conv<false, false>(a, ch, active, n0, ratio, hv0 + half, off, col, ring, w, q_seq, q_t, q_T, q_slot);
    } else {
        // silu(z) of the lane's 8 columns, 8 rows at a time; none for the tokens of segments the chunked pass
        // takes when it reads z itself (z_skip_min_t)
        if (active) {
            const uint16_t* zp = a.z + (long long)n0 * a.ld_z + (hv0 + half) * DV + c8;
            const int skip_t = a.z_skip_min_t > 0 ? a.z_skip_min_t : 0x7fffffff;
#pragma unroll 1
            for (int jb = 0; jb < PV_TOK; jb += 8) {
                bool need[8];
                bool any = false;
#pragma unroll
                for (int r = 0; r < 8; ++r) {
                    need[r] = q_seq[jb + r] >= 0 && q_T[jb + r] < skip_t;   // routed tokens lie below n_tokens
                    any |= need[r];
                }
                if (!any) continue;   // uniform over the warp: the routing is per token
                uint4 zr[8];
#pragma unroll
                for (int r = 0; r < 8; ++r)
                    // coherent loads: z is the output of a projection that may release this kernel early
                    zr[r] = need[r] ? __ldcg(reinterpret_cast<const uint4*>(zp + (long long)(jb + r) * a.ld_z))
                                    : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
                for (int r = 0; r < 8; ++r) {
                    if (!need[r]) continue;
                    float zv[8];
                    unpack8(zr[r], zv);
                    if (simple) {
                        silu8_fast(zv);
                    } else {
#pragma unroll
                        for (int c = 0; c < 8; ++c) zv[c] = silu_bf(zv[c]);
                    }
                    *reinterpret_cast<uint4*>(a.rec + ((long long)(hv0 + half) * a.rec_cap + n0 + jb + r) * REC_BYTES +
                                              768 + 2 * c8) = pack8_exact(zv);
                }
            }
        }
        // gates (compiled_beta_g): lane = token (lane & 15) of v-head hv0 + half
        const int j = lane & 15;
        if (half < ratio && q_seq[j] >= 0) {
            const int n = n0 + j;
            const int hv = hv0 + half;
            const float b = bf2f(a.ab[(long long)n * a.ld_ab + hv]);
            const float av = bf2f(a.ab[(long long)n * a.ld_ab + a.hv + hv]);
            const float sp = gate_softplus(av, a.dt_bias[hv], a.dt_bf16);
            const float logdecay = -(expf(a.A_log[hv]) * sp);
            // the record's last sector whole (gates and zero padding): no partly written sector
            float4* gb = reinterpret_cast<float4*>(a.rec + ((long long)hv * a.rec_cap + n) * REC_BYTES + 1024);
            gb[0] = make_float4(expf(logdecay), rbf(sigmoid_f32(b)), logdecay, 0.f);
            gb[1] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
}

// ------------------------------------------------------------------ K2

// All 288 threads meet here.  Normally every issued copy was consumed; after a
// timed-out wait, thread 0 waits (bounded) for copies still in flight so the
// CTA never exits with an async write pending into its shared memory.
__device__ __forceinline__ void drain_and_exit(uint64_t* full, volatile int* s_issued, volatile int* s_consumed,
                                               int tid) {
    __syncwarp();
    named_bar_sync(2, K2_THREADS);
    if (tid == 0) {
        const int issued = *s_issued, consumed = *s_consumed;
        for (int k = consumed; k < issued; ++k)
            mbar_wait_bounded(&full[k % NSTAGE], (uint32_t)(k / NSTAGE) & 1u, WAIT_LIMIT_NS);
    }
}

// Per-stage header written by the producer before it arms the stage's full barrier.
struct StageHdr {
    int slot, hv, t0, T;  // T < 0: end of this CTA's work
};

__global__ void __launch_bounds__(K2_THREADS, 1) gdn_recur_kernel(const RecurArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + NSTAGE * STAGE_BYTES);
    uint64_t* empty = full + NSTAGE;
    StageHdr* hdr = reinterpret_cast<StageHdr*>(empty + NSTAGE);
    float* s_y = reinterpret_cast<float*>(hdr + NSTAGE);   // [2][DV], double-buffered per token
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_y + 2 * DV);
    volatile int* s_issued = s_abort + 1;    // items whose copies the producer issued
    volatile int* s_consumed = s_abort + 2;  // items the consumers took out of the ring

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n_items = a.n_seq * a.hv;
    const int ratio = a.hv / a.hk;

    if (tid == 0) {
        for (int s = 0; s < NSTAGE; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], K2_CONSUMER_WARPS);
        }
        *s_abort = 0;
        *s_issued = 0;
        *s_consumed = 0;
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == K2_CONSUMER_WARPS) {
        // ------------------------------------------------ producer (one lane)
        if (lane == 0) {
            const float* st_src = a.rec_in ? a.rec_in : a.rec;
            int k = 0;
            bool waited = false;
            int pend_stage[NSTAGE], pend_hv[NSTAGE], pend_t0[NSTAGE], pend_n[NSTAGE];
            int npend = 0;
            bool ok = true;
            // routing entries of the next item are loaded one iteration ahead
            int item = blockIdx.x;
            int nx_t0 = 0, nx_t1 = 0, nx_slot = 0;
            if (item < n_items) {
                const int sq = item / a.hv;
                nx_t0 = __ldg(a.cu_seqlens + sq);
                nx_t1 = __ldg(a.cu_seqlens + sq + 1);
                nx_slot = __ldg(a.slot_ids + sq);
            }
            for (; item < n_items && ok; item += gridDim.x) {
                const int hv = item % a.hv;
                const int t0 = nx_t0;
                const int T = nx_t1 - nx_t0;
                const int slot = nx_slot;
                const int next = item + gridDim.x;
                if (next < n_items) {
                    const int sq = next / a.hv;
                    nx_t0 = __ldg(a.cu_seqlens + sq);
                    nx_t1 = __ldg(a.cu_seqlens + sq + 1);
                    nx_slot = __ldg(a.slot_ids + sq);
                }
                const bool bad_slot = slot < 0 || slot >= a.n_slots;
                const bool bad_len = T < 0 || t0 < 0 || t0 + T > a.n_tokens;
                if (bad_slot || bad_len) {
                    if (hv == 0) atomicOr(a.err, (bad_slot ? ERR_BAD_SLOT : 0) | (bad_len ? ERR_BAD_SEQLENS : 0));
                    continue;
                }
                if (T == 0) continue;
                if (a.wy_min_t > 0 && T >= a.wy_min_t) continue;  // handled by the chunked prefill kernel
                const int s = k % NSTAGE;
                const uint32_t ph = (uint32_t)(k / NSTAGE) & 1u;
                if (k >= NSTAGE && !mbar_wait_bounded(&empty[s], ph ^ 1u, WAIT_LIMIT_NS)) {
                    atomicOr(a.err, ERR_TIMEOUT);
                    *s_abort = 1;
                    ok = false;
                    break;
                }
                const int nrec = T < REC_PER_STAGE ? T : REC_PER_STAGE;
                uint8_t* stage = smem + s * STAGE_BYTES;
                hdr[s].slot = slot;
                hdr[s].hv = hv;
                hdr[s].t0 = t0;
                hdr[s].T = T;
                mbar_arrive_expect_tx(&full[s], TILE_BYTES + nrec * REC_BYTES);
                bulk_g2s(stage, st_src + ((size_t)slot * a.hv + hv) * (DV * DK), TILE_BYTES, &full[s]);
                if (!waited) {
                    pend_stage[npend] = s; pend_hv[npend] = hv; pend_t0[npend] = t0; pend_n[npend] = nrec;
                    if (++npend == NSTAGE) {
                        pdl_wait();
                        waited = true;
                        for (int q = 0; q < npend; ++q)
                            bulk_g2s(smem + pend_stage[q] * STAGE_BYTES + TILE_BYTES,
                                     a.recs + ((long long)pend_hv[q] * a.rec_cap + pend_t0[q]) * REC_BYTES,
                                     pend_n[q] * REC_BYTES, &full[pend_stage[q]]);
                        npend = 0;
                    }
                } else {
                    bulk_g2s(stage + TILE_BYTES, a.recs + ((long long)hv * a.rec_cap + t0) * REC_BYTES,
                             nrec * REC_BYTES, &full[s]);
                }
                ++k;
            }
            if (!waited) {
                pdl_wait();
                for (int q = 0; q < npend; ++q)
                    bulk_g2s(smem + pend_stage[q] * STAGE_BYTES + TILE_BYTES,
                             a.recs + ((long long)pend_hv[q] * a.rec_cap + pend_t0[q]) * REC_BYTES,
                             pend_n[q] * REC_BYTES, &full[pend_stage[q]]);
            }
            *s_issued = k;
            if (ok) {
                // end-of-work marker in the next stage
                const int s = k % NSTAGE;
                const uint32_t ph = (uint32_t)(k / NSTAGE) & 1u;
                if (k < NSTAGE || mbar_wait_bounded(&empty[s], ph ^ 1u, WAIT_LIMIT_NS)) {
                    hdr[s].T = -1;
                    mbar_arrive(&full[s]);
                } else {
                    atomicOr(a.err, ERR_TIMEOUT);
                    *s_abort = 1;
                }
            }
        }
        drain_and_exit(full, s_issued, s_consumed, tid);
        return;
    }

    // ---------------------------------------------------- consumers (256 threads)
    pdl_wait();
    const int oc = warp * 16 + (lane & 15);          // output column of this lane in the epilogue
    const float nw = bf2f(a.norm_w[oc]);
    const int myrow = warp * RPW + (lane >> 1);
    int buf = 0;
    int k = 0;
    while (true) {
        const int s = k % NSTAGE;
        const uint32_t ph = (uint32_t)(k / NSTAGE) & 1u;
        if (!mbar_wait_bounded(&full[s], ph, WAIT_LIMIT_NS)) {
            atomicOr(a.err, ERR_TIMEOUT);
            *s_abort = 1;
        }
        if (*s_abort) break;
        const StageHdr h = hdr[s];
        if (h.T < 0) break;
        ++k;

        const uint8_t* stage = smem + s * STAGE_BYTES;
        const float* tile = reinterpret_cast<const float*>(stage);
        float4 S[RPW];
#pragma unroll
        for (int j = 0; j < RPW; ++j) S[j] = *reinterpret_cast<const float4*>(tile + (warp * RPW + j) * DK + lane * 4);

        for (int t = 0; t < h.T; ++t) {
            const uint8_t* rec = t < REC_PER_STAGE ? stage + TILE_BYTES + t * REC_BYTES
                                                   : a.recs + ((long long)h.hv * a.rec_cap + h.t0 + t) * REC_BYTES;
            const uint2 qu = *reinterpret_cast<const uint2*>(rec + lane * 8);
            const uint2 ku = *reinterpret_cast<const uint2*>(rec + 256 + lane * 8);
            const float vv = bf2f(reinterpret_cast<const uint16_t*>(rec)[256 + myrow]);
            const float zs = bf2f(reinterpret_cast<const uint16_t*>(rec)[384 + oc]);
            const float gt = reinterpret_cast<const float*>(rec + 1024)[0];
            const float bt = reinterpret_cast<const float*>(rec + 1024)[1];
            if (t == h.T - 1) {
                // every read of this stage is done: hand it back to the producer
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
            }
            const float4 q4 = make_float4(__uint_as_float(qu.x << 16), __uint_as_float(qu.x & 0xffff0000u),
                                          __uint_as_float(qu.y << 16), __uint_as_float(qu.y & 0xffff0000u));
            const float4 k4 = make_float4(__uint_as_float(ku.x << 16), __uint_as_float(ku.x & 0xffff0000u),
                                          __uint_as_float(ku.y << 16), __uint_as_float(ku.y & 0xffff0000u));
            float p[RPW];
#pragma unroll
            for (int j = 0; j < RPW; ++j) {
                S[j].x *= gt; S[j].y *= gt; S[j].z *= gt; S[j].w *= gt;
                p[j] = S[j].x * k4.x + S[j].y * k4.y + S[j].z * k4.z + S[j].w * k4.w;
            }
            const float kv = reduce_scatter16(p, lane);
            const float delta = (vv - kv) * bt;
#pragma unroll
            for (int j = 0; j < RPW; ++j) {
                const float d = __shfl_sync(0xffffffffu, delta, 2 * j);
                S[j].x += k4.x * d; S[j].y += k4.y * d; S[j].z += k4.z * d; S[j].w += k4.w * d;
                p[j] = S[j].x * q4.x + S[j].y * q4.y + S[j].z * q4.z + S[j].w * q4.w;
            }
            const float yv = reduce_scatter16(p, lane);
            float* sy = s_y + buf * DV;
            if (!(lane & 1)) sy[myrow] = rbf(yv);
            named_bar_sync(1, K2_CONSUMERS);
            // gated RMSNorm epilogue: every warp reduces all 128 y (same order, same result),
            // lanes 0..15 of warp w write output columns 16w..16w+15
            const float4 y4 = *reinterpret_cast<const float4*>(sy + lane * 4);
            const float ss = warp_sum(y4.x * y4.x + y4.y * y4.y + y4.z * y4.z + y4.w * y4.w);
            if (lane < 16) {
                const float nrm = 1.0f / sqrtf(ss / (float)DV + a.eps);
                const float yn = rbf(rbf(sy[oc] * nrm) * nw);
                a.out[(long long)(h.t0 + t) * a.ld_out + (long long)h.hv * DV + oc] = f2bf(zs * yn);
            }
            buf ^= 1;
        }

        // state tile back to the pool (evict-first: it is not re-read in this step)
        float* dst = a.rec + ((size_t)h.slot * a.hv + h.hv) * (DV * DK) + (warp * RPW) * DK + lane * 4;
#pragma unroll
        for (int j = 0; j < RPW; ++j) __stcs(reinterpret_cast<float4*>(dst + j * DK), S[j]);

        if (h.T > 1) {
            // conv-state windows of a multi-token sequence: the last K-1 rows of [old window; tokens]
            // (one-token sequences were shifted in place by the prep kernel)
            uint16_t* cs = a.conv + (size_t)h.slot * (KC - 1) * a.D;
            const int hk = h.hv / ratio;
            for (int idx = tid; idx < DV + ((h.hv % ratio == 0) ? 2 * DK : 0); idx += K2_CONSUMERS) {
                const int ch = idx < DV ? 2 * a.hk * DK + h.hv * DV + idx
                                        : ((idx - DV) < DK ? hk * DK + (idx - DV) : a.hk * DK + hk * DK + (idx - DV - DK));
                uint16_t w[KC - 1];
#pragma unroll
                for (int j = 0; j < KC - 1; ++j) {
                    const int p = h.T + j;
                    w[j] = p < KC - 1 ? cs[(size_t)p * a.D + ch]
                                      : a.qkv[(long long)(h.t0 + p - (KC - 1)) * a.ld_qkv + ch];
                }
#pragma unroll
                for (int j = 0; j < KC - 1; ++j) cs[(size_t)j * a.D + ch] = w[j];
            }
        }
    }
    if (tid == 0) *s_consumed = k;
    drain_and_exit(full, s_issued, s_consumed, tid);
}

static int g_num_sms[64] = {0};

int g_decode_kernel = 0;
SplitCtl g_split_ctl = {2000000000ull, -1};

cudaError_t launch_layer_step_v2(const PrepArgs& p, const RecurArgs& r, cudaStream_t stream) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (g_num_sms[dev] == 0) {
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(gdn_recur_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, K2_SMEM);
        if (e != cudaSuccess) return e;
        g_num_sms[dev] = sms;
    }
    if (p.n_tokens == 0 || r.n_seq == 0) return cudaSuccess;
    // One token per sequence on average: few sequences take the split kernel (4 CTAs per (sequence, v-head)
    // tile), many the fused one-kernel step ((sequence, k-head) items balance over the SMs there).
    if (p.n_tokens == p.n_seq && r.wy_min_t == 0) {
        const bool split_ok = r.hv % r.hk == 0 && r.hv / r.hk <= 2;
        const int mode = g_decode_kernel;
        if (split_ok && (mode == 1 || (mode == 0 && r.n_seq < SPLIT_MAX_SEQ)))
            return launch_decode_split(p, r, g_split_ctl, stream);
        if (mode == 2 || (mode == 0 && r.n_seq >= FUSED_MIN_SEQ)) return launch_decode_fused(p, r, stream);
    }

    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;

    // Calls with multi-token segments take the tiled prep when the bf16 pair loads are aligned.
    const bool pairs_aligned = ((reinterpret_cast<uintptr_t>(p.qkv) | reinterpret_cast<uintptr_t>(p.z)) & 3u) == 0 &&
                               (p.ld_qkv & 1) == 0 && (p.ld_z & 1) == 0;
    const bool tiled = p.n_tokens > p.n_seq && pairs_aligned && p.hv <= 2 * p.hk;
    // ... and the 8-channel form when every row, weight, window and record access can be 16 bytes wide.
    const bool vec = tiled &&
                     ((reinterpret_cast<uintptr_t>(p.qkv) | reinterpret_cast<uintptr_t>(p.z) |
                       reinterpret_cast<uintptr_t>(p.conv_w) | reinterpret_cast<uintptr_t>(p.conv) |
                       reinterpret_cast<uintptr_t>(p.rec)) & 15u) == 0 &&
                     (p.ld_qkv & 7) == 0 && (p.ld_z & 7) == 0 && (p.D & 7) == 0;
    cudaLaunchConfig_t c1 = {};
    if (vec) {
        constexpr int per_cta = PV_SUB * PV_TOK;
        c1.gridDim = dim3((unsigned)((p.n_tokens + per_cta - 1) / per_cta), (unsigned)p.hk, 1);
        c1.blockDim = dim3(PV_THREADS, 1, 1);
    } else {
        c1.gridDim = tiled ? dim3((unsigned)((p.n_tokens + PT_TOK - 1) / PT_TOK), (unsigned)p.hk, 1)
                           : dim3((unsigned)p.n_tokens, (unsigned)p.hk, 1);
        c1.blockDim = dim3(256, 1, 1);
    }
    c1.stream = stream;
    c1.attrs = attr;
    c1.numAttrs = 1;
    e = vec     ? cudaLaunchKernelEx(&c1, gdn_prep_vec_kernel, p)
        : tiled ? cudaLaunchKernelEx(&c1, gdn_prep_tile_kernel, p)
                : cudaLaunchKernelEx(&c1, gdn_prep_kernel, p);
    if (e != cudaSuccess) return e;

    const int n_items = r.n_seq * r.hv;
    cudaLaunchConfig_t c2 = {};
    c2.gridDim = dim3((unsigned)(n_items < g_num_sms[dev] ? n_items : g_num_sms[dev]), 1, 1);
    c2.blockDim = dim3(K2_THREADS, 1, 1);
    c2.dynamicSmemBytes = K2_SMEM;
    c2.stream = stream;
    c2.attrs = attr;
    c2.numAttrs = 1;
    return cudaLaunchKernelEx(&c2, gdn_recur_kernel, r);
}

}  // namespace gdn
