// gdn_fused.cu -- the decode layer step as ONE persistent kernel per layer (sm_100a), for calls
// whose sequences carry one token each on average (n_tokens == n_seq; any segment length is
// handled, long ones slowly).
//
// Work item = (sequence, k-head): the k-head's q/k channels and its Hv/Hk v-heads.  Per CTA
// (one per SM, 672 threads):
//   warps 0..15  consumers: per v-head, the state tile [dv][dk] in registers (warp w: rows
//                8w..8w+7, lane l: columns 4l..4l+3), the gated delta rule per token
//                (metal_gdn.rs:37-62) and the gated RMSNorm epilogue (qwen3_5.rs:660-665);
//                the updated tile goes back into its stage and one bulk async store returns it
//                to the pool while the warps move on;
//   warp 16      producer (one lane): the v-heads' 64 KiB f32 state tiles into a 3-stage ring
//                with bulk async copies completing on mbarriers;
//   warps 17..20 prep: conv + SiLU of the q, k and v channels (decode rounding for a one-token
//                segment, qwen3_5.rs:602-610; f32 conv1d otherwise, :617-623), q/k RMSNorm
//                (:636-639), silu(z), beta and g (compiled_ops.rs:30-43), written as token records
//                straight into the stage next to its state tile (tokens past the 4th of a segment
//                go to the pool's record scratch), then the conv-state windows: shifted in place
//                for a one-token segment, rewritten from the tokens otherwise.
// The item owns every reader of its conv windows, so the in-place shift needs no ordering with
// other CTAs.  Prep and the state copies overlap; a stage's full barrier completes when the
// tile has landed and the prep has arrived.  Compared with the two-kernel step (gdn_decode.cu)
// this removes the kernel boundary between prep and recurrence, and 16 consumer warps halve the
// per-token dependent chain.
//
// PDL: the kernel lets its dependents launch at once (their CTAs then start as these exit) and
// waits (griddepcontrol.wait) before touching global memory, so completions stay in stream order.
#include "gdn_device.cuh"
#include "gdn_internal.h"
#include "gdn_ptx.cuh"

namespace gdn {

constexpr int FD_CWARPS = 16;
constexpr int FD_CONSUMERS = FD_CWARPS * 32;              // 512
constexpr int FD_PWARP = FD_CWARPS;                       // producer warp
constexpr int FD_QWARP0 = FD_CWARPS + 1;                  // first prep warp
constexpr int FD_PREP = 4 * 32;                           // 128 prep threads
constexpr int FD_THREADS = FD_CONSUMERS + 32 + FD_PREP;   // 672
constexpr int FD_RPW = DV / FD_CWARPS;                    // 8 state rows per consumer warp
constexpr int FD_NSTAGE = 3;
constexpr int FD_TILE = DV * DK * 4;
constexpr int FD_STAGE = FD_TILE + REC_PER_STAGE * REC_BYTES;   // 69,696
constexpr int FD_OFF_BAR = FD_NSTAGE * FD_STAGE;
constexpr int FD_OFF_HDR = FD_OFF_BAR + 2 * FD_NSTAGE * 8;
constexpr int FD_OFF_Y = FD_OFF_HDR + FD_NSTAGE * 16;
constexpr int FD_OFF_QK = FD_OFF_Y + 2 * DV * 4;
constexpr int FD_OFF_RED = FD_OFF_QK + REC_PER_STAGE * FD_PREP * 4;
constexpr int FD_OFF_FLAGS = FD_OFF_RED + 2 * 4 * 4;
constexpr int FD_SMEM = FD_OFF_FLAGS + 16;
static_assert(FD_STAGE % 16 == 0, "stage alignment");
static_assert(FD_SMEM <= 232448, "shared memory budget");
constexpr uint64_t FD_WAIT_NS = 2000000000ull;
constexpr int FD_BAR_Y = 1, FD_BAR_PREP = 2, FD_BAR_DRAIN = 3, FD_BAR_STORE = 4;

struct FdHdr {
    int slot, hv, t0, T;  // T < 0: end of this CTA's work
};

// Routing entries of sequence seq.
struct FdRoute {
    int t0, T, slot;
};

__device__ __forceinline__ FdRoute fd_load_route(const RecurArgs& r, int seq) {
    FdRoute q;
    q.t0 = __ldg(r.cu_seqlens + seq);
    q.T = __ldg(r.cu_seqlens + seq + 1) - q.t0;
    q.slot = __ldg(r.slot_ids + seq);
    return q;
}

// False when the item has nothing to do here (a rejected sequence is reported once, by k-head 0).
__device__ __forceinline__ bool fd_route_ok(const RecurArgs& r, const FdRoute& q, int hk, bool report) {
    const bool bad_slot = q.slot < 0 || q.slot >= r.n_slots;
    const bool bad_len = q.T < 0 || q.t0 < 0 || q.t0 + q.T > r.n_tokens;
    if (bad_slot || bad_len) {
        if (report && hk == 0) atomicOr(r.err, (bad_slot ? ERR_BAD_SLOT : 0) | (bad_len ? ERR_BAD_SEQLENS : 0));
        return false;
    }
    if (q.T == 0) return false;
    if (r.wy_min_t > 0 && q.T >= r.wy_min_t) return false;
    return true;
}

// Conv taps of channel ch for token t of a segment starting at packed row t0: padded[t..t+3] with
// padded = [conv window (K-1 rows); tokens].
__device__ __forceinline__ void fd_taps(const PrepArgs& p, const uint16_t* cs, int ch, int t0, int t, float (&x)[4]) {
#pragma unroll
    for (int j = 0; j < KC; ++j) {
        const int q = t + j;
        x[j] = q < KC - 1 ? bf2f(cs[(size_t)q * p.D + ch]) : bf2f(p.qkv[(long long)(t0 + q - (KC - 1)) * p.ld_qkv + ch]);
    }
}

// The conv window of channel ch after a segment of T >= 2 tokens: the last K-1 rows of [window; tokens].
__device__ __forceinline__ void fd_window_writeback(const PrepArgs& p, uint16_t* cs, int ch, int t0, int T) {
    uint16_t w[KC - 1];
#pragma unroll
    for (int j = 0; j < KC - 1; ++j) {
        const int q = T + j;
        w[j] = q < KC - 1 ? cs[(size_t)q * p.D + ch] : p.qkv[(long long)(t0 + q - (KC - 1)) * p.ld_qkv + ch];
    }
#pragma unroll
    for (int j = 0; j < KC - 1; ++j) cs[(size_t)j * p.D + ch] = w[j];
}

// All threads meet; then thread 0 waits (bounded) for state copies issued but never consumed,
// so the CTA never exits with an async write pending into its shared memory.
__device__ __forceinline__ void fd_drain(uint64_t* full, volatile int* s_issued, volatile int* s_consumed, int tid) {
    __syncwarp();
    named_bar_sync(FD_BAR_DRAIN, FD_THREADS);
    if (tid == 0) {
        const int issued = *s_issued, consumed = *s_consumed;
        for (int k = consumed; k < issued; ++k)
            mbar_wait_bounded(&full[k % FD_NSTAGE], (uint32_t)(k / FD_NSTAGE) & 1u, FD_WAIT_NS);
    }
}

__global__ void __launch_bounds__(FD_THREADS, 1) gdn_decode_fused_kernel(const PrepArgs p, const RecurArgs r) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + FD_OFF_BAR);
    uint64_t* empty = full + FD_NSTAGE;
    FdHdr* hdr = reinterpret_cast<FdHdr*>(smem + FD_OFF_HDR);
    float* s_y = reinterpret_cast<float*>(smem + FD_OFF_Y);             // [2][DV]
    uint32_t* s_qk = reinterpret_cast<uint32_t*>(smem + FD_OFF_QK);     // [REC_PER_STAGE][128] q|k bf16 pairs
    float* s_red = reinterpret_cast<float*>(smem + FD_OFF_RED);         // [2][4] prep-warp sums of squares
    volatile int* s_abort = reinterpret_cast<volatile int*>(smem + FD_OFF_FLAGS);
    volatile int* s_issued = s_abort + 1;
    volatile int* s_consumed = s_abort + 2;
    volatile int* s_prep_issued = s_abort + 3;   // items whose prep loads are issued (gates the tile copies)

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ratio = r.hv / r.hk;
    const int n_groups = r.n_seq * r.hk;

    if (tid == 0) {
        for (int s = 0; s < FD_NSTAGE; ++s) {
            mbar_init(&full[s], 2);           // producer (with the tile's bytes) + prep
            mbar_init(&empty[s], 1);          // consumer thread 0, once the stage's state store has read it
        }
        *s_abort = 0;
        *s_issued = 0;
        *s_consumed = 0;
        *s_prep_issued = 0;
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == FD_PWARP) {
        // ------------------------------------------------ producer (one lane)
        if (lane == 0) {
            pdl_wait();
            const float* st_src = r.rec_in ? r.rec_in : r.rec;
            int k = 0, gi = 0;
            bool ok = true;
            FdRoute nx{};
            if (blockIdx.x < n_groups) nx = fd_load_route(r, blockIdx.x / r.hk);
            for (int g = blockIdx.x; g < n_groups && ok; g += gridDim.x) {
                const int seq = g / r.hk, hk = g - seq * r.hk;
                const FdRoute q = nx;
                if (g + (int)gridDim.x < n_groups) nx = fd_load_route(r, (g + gridDim.x) / r.hk);
                if (!fd_route_ok(r, q, hk, true)) continue;
                const int t0 = q.t0, T = q.T, slot = q.slot;
                // the first item's state copies go out after its prep loads, so those small loads reach
                // DRAM ahead of the CTA's first 128 KiB of bulk traffic; later items prefetch freely
                if (gi == 0) {
                    const uint64_t t_start = global_timer_ns();
                    while (*s_prep_issued <= gi) {
                        if (global_timer_ns() - t_start > FD_WAIT_NS) {
                            atomicOr(r.err, ERR_TIMEOUT);
                            *s_abort = 1;
                            ok = false;
                            break;
                        }
                    }
                    if (!ok) break;
                }
                ++gi;
                for (int j = 0; j < ratio; ++j) {
                    const int hv = hk * ratio + j;
                    const int s = k % FD_NSTAGE;
                    const uint32_t ph = (uint32_t)(k / FD_NSTAGE) & 1u;
                    if (k >= FD_NSTAGE && !mbar_wait_bounded(&empty[s], ph ^ 1u, FD_WAIT_NS)) {
                        atomicOr(r.err, ERR_TIMEOUT);
                        *s_abort = 1;
                        ok = false;
                        break;
                    }
                    hdr[s].slot = slot;
                    hdr[s].hv = hv;
                    hdr[s].t0 = t0;
                    hdr[s].T = T;
                    mbar_arrive_expect_tx(&full[s], FD_TILE);
                    bulk_g2s(smem + s * FD_STAGE, st_src + ((size_t)slot * r.hv + hv) * (DV * DK), FD_TILE, &full[s]);
                    ++k;
                }
            }
            *s_issued = k;
            if (ok) {
                const int s = k % FD_NSTAGE;
                const uint32_t ph = (uint32_t)(k / FD_NSTAGE) & 1u;
                if (k < FD_NSTAGE || mbar_wait_bounded(&empty[s], ph ^ 1u, FD_WAIT_NS)) {
                    hdr[s].T = -1;
                    mbar_arrive(&full[s]);
                } else {
                    atomicOr(r.err, ERR_TIMEOUT);
                    *s_abort = 1;
                }
            }
        }
        fd_drain(full, s_issued, s_consumed, tid);
        return;
    }

    if (warp >= FD_QWARP0) {
        // ------------------------------------------------ prep (128 threads)
        const int pt = tid - FD_QWARP0 * 32;
        const int pw = pt >> 5;
        const bool is_q = pt < 64;
        pdl_wait();
        int k = 0, gi = 0;
        int par = 0;
        bool ok = true;
        FdRoute nx{};
        if (blockIdx.x < n_groups) nx = fd_load_route(r, blockIdx.x / r.hk);
        for (int g = blockIdx.x; g < n_groups && ok; g += gridDim.x) {
            const int seq = g / r.hk, hk = g - seq * r.hk;
            const FdRoute rq = nx;
            if (g + (int)gridDim.x < n_groups) nx = fd_load_route(r, (g + gridDim.x) / r.hk);
            if (!fd_route_ok(r, rq, hk, false)) continue;
            const int t0 = rq.t0, T = rq.T, slot = rq.slot;
            uint16_t* cs = p.conv + (size_t)slot * (KC - 1) * p.D;
            const bool decode = T == 1;
            ++gi;
            if (decode && ratio <= 2) {
                // ---- one token, Hv/Hk <= 2: every load of the item at once, then compute, then records
                const long long n = t0;
                const int qk_ch = (is_q ? 0 : r.hk * DK) + hk * DK + 2 * (pt & 63);
                uint16_t xq[2][4], xv[2][4];
                float wq[2][4], wv[2][4], zz[2] = {0.f, 0.f};
#pragma unroll
                for (int e = 0; e < 2; ++e) {
#pragma unroll
                    for (int j = 0; j < KC - 1; ++j) xq[e][j] = cs[(size_t)j * p.D + qk_ch + e];
                    xq[e][KC - 1] = p.qkv[n * p.ld_qkv + qk_ch + e];
                    fd_unpack_w(p.conv_w, qk_ch + e, wq[e]);
                }
#pragma unroll
                for (int jj = 0; jj < 2; ++jj) {
                    if (jj < ratio) {
                        const int hv = hk * ratio + jj;
                        const int vch = 2 * r.hk * DK + hv * DV + pt;
#pragma unroll
                        for (int j = 0; j < KC - 1; ++j) xv[jj][j] = cs[(size_t)j * p.D + vch];
                        xv[jj][KC - 1] = p.qkv[n * p.ld_qkv + vch];
                        fd_unpack_w(p.conv_w, vch, wv[jj]);
                        zz[jj] = bf2f(p.z[n * p.ld_z + (long long)hv * DV + pt]);
                    }
                }
                float gb_b = 0.f, gb_a = 0.f, gb_alog = 0.f, gb_dt = 0.f;
                if (pt < ratio) {
                    const int hv = hk * ratio + pt;
                    gb_b = bf2f(p.ab[n * p.ld_ab + hv]);
                    gb_a = bf2f(p.ab[n * p.ld_ab + r.hv + hv]);
                    gb_alog = p.A_log[hv];
                    gb_dt = p.dt_bias[hv];
                }
                named_bar_sync(FD_BAR_PREP, FD_PREP);   // every prep load of the item is issued
                if (pt == 0) *s_prep_issued = gi;
                // the item is its windows' only reader in this call: shift them in place
#pragma unroll
                for (int j = 0; j < KC - 1; ++j) {
                    cs[(size_t)j * p.D + qk_ch] = xq[0][j + 1];
                    cs[(size_t)j * p.D + qk_ch + 1] = xq[1][j + 1];
                }
#pragma unroll
                for (int jj = 0; jj < 2; ++jj) {
                    if (jj < ratio) {
                        const int vch = 2 * r.hk * DK + (hk * ratio + jj) * DV + pt;
#pragma unroll
                        for (int j = 0; j < KC - 1; ++j) cs[(size_t)j * p.D + vch] = xv[jj][j + 1];
                    }
                }
                // q / k conv, SiLU, RMSNorm (gain folded), v conv, silu(z), gates
                float f0[4], f1[4];
#pragma unroll
                for (int j = 0; j < KC; ++j) {
                    f0[j] = bf2f(xq[0][j]);
                    f1[j] = bf2f(xq[1][j]);
                }
                const float o0 = fd_conv_silu(f0, wq[0], true);
                const float o1 = fd_conv_silu(f1, wq[1], true);
                const float ss = warp_sum(o0 * o0 + o1 * o1);
                if (lane == 0) s_red[par * 4 + pw] = ss;
                float vo[2] = {0.f, 0.f}, zs[2] = {0.f, 0.f};
#pragma unroll
                for (int jj = 0; jj < 2; ++jj) {
                    if (jj < ratio) {
                        float fv[4];
#pragma unroll
                        for (int j = 0; j < KC; ++j) fv[j] = bf2f(xv[jj][j]);
                        vo[jj] = fd_conv_silu(fv, wv[jj], true);
                        zs[jj] = silu_bf(zz[jj]);
                    }
                }
                float g_dec = 0.f, g_beta = 0.f, g_log = 0.f;
                if (pt < ratio) {
                    const float sp = gate_softplus(gb_a, gb_dt, p.dt_bf16);
                    g_log = -(expf(gb_alog) * sp);
                    g_dec = expf(g_log);
                    g_beta = rbf(sigmoid_f32(gb_b));
                }
                named_bar_sync(FD_BAR_PREP, FD_PREP);
                const float tot = s_red[par * 4 + (pw & 2)] + s_red[par * 4 + (pw & 2) + 1];
                par ^= 1;
                const float nrm = 1.0f / sqrtf(tot / (float)DK + 1e-6f);
                const float gain = is_q ? 0.0078125f : 0.08837890625f;  // bf16(1/128), bf16(128^-0.5)
                const uint32_t qkv_word =
                    (uint32_t)f2bf(rbf(o0 * nrm) * gain) | ((uint32_t)f2bf(rbf(o1 * nrm) * gain) << 16);
                // the heads' stages must be free before their records are written
                bool timed_out = false;
                for (int jj = 0; jj < ratio; ++jj) {
                    const int kk = k + jj;
                    if (kk >= FD_NSTAGE &&
                        !mbar_wait_bounded(&empty[kk % FD_NSTAGE], ((uint32_t)(kk / FD_NSTAGE) & 1u) ^ 1u, FD_WAIT_NS)) {
                        timed_out = true;
                        atomicOr(r.err, ERR_TIMEOUT);
                        *s_abort = 1;
                    }
                }
                if (named_bar_or(FD_BAR_PREP, FD_PREP, timed_out || *s_abort)) {
                    ok = false;
                    break;
                }
#pragma unroll
                for (int jj = 0; jj < 2; ++jj) {
                    if (jj < ratio) {
                        uint8_t* rec = smem + ((k + jj) % FD_NSTAGE) * FD_STAGE + FD_TILE;
                        reinterpret_cast<uint32_t*>(rec)[pt] = qkv_word;
                        reinterpret_cast<uint16_t*>(rec)[256 + pt] = f2bf(vo[jj]);
                        reinterpret_cast<uint16_t*>(rec)[384 + pt] = f2bf(zs[jj]);
                    }
                }
                if (pt < ratio) {
                    float* gb = reinterpret_cast<float*>(smem + ((k + pt) % FD_NSTAGE) * FD_STAGE + FD_TILE + 1024);
                    gb[0] = g_dec;
                    gb[1] = g_beta;
                    gb[2] = g_log;
                }
                named_bar_sync(FD_BAR_PREP, FD_PREP);   // every record of the item is written
                if (pt == 0)
                    for (int jj = 0; jj < ratio; ++jj) mbar_arrive(&full[(k + jj) % FD_NSTAGE]);
                k += ratio;
                continue;
            }
            if (pt == 0) *s_prep_issued = gi;
            // ---- q / k: channel pair (qk_ch, qk_ch + 1) of this thread, every token of the segment
            const int qk_ch = (is_q ? 0 : r.hk * DK) + hk * DK + 2 * (pt & 63);
            float wq[2][4];
            fd_unpack_w(p.conv_w, qk_ch, wq[0]);
            fd_unpack_w(p.conv_w, qk_ch + 1, wq[1]);
            const float gain = is_q ? 0.0078125f : 0.08837890625f;  // bf16(1/128), bf16(128^-0.5)
            for (int t = 0; t < T; ++t) {
                float x0[4], x1[4];
                fd_taps(p, cs, qk_ch, t0, t, x0);
                fd_taps(p, cs, qk_ch + 1, t0, t, x1);
                if (decode) {
                    // the item is the windows' only reader in this call: shift them in place
#pragma unroll
                    for (int j = 0; j < KC - 1; ++j) {
                        cs[(size_t)j * p.D + qk_ch] = f2bf(x0[j + 1]);
                        cs[(size_t)j * p.D + qk_ch + 1] = f2bf(x1[j + 1]);
                    }
                }
                const float o0 = fd_conv_silu(x0, wq[0], decode);
                const float o1 = fd_conv_silu(x1, wq[1], decode);
                const float ss = warp_sum(o0 * o0 + o1 * o1);
                if (lane == 0) s_red[par * 4 + pw] = ss;
                named_bar_sync(FD_BAR_PREP, FD_PREP);
                const float tot = s_red[par * 4 + (pw & 2)] + s_red[par * 4 + (pw & 2) + 1];
                par ^= 1;
                const float nrm = 1.0f / sqrtf(tot / (float)DK + 1e-6f);
                const uint32_t val = (uint32_t)f2bf(rbf(o0 * nrm) * gain) | ((uint32_t)f2bf(rbf(o1 * nrm) * gain) << 16);
                if (t < REC_PER_STAGE) {
                    s_qk[t * FD_PREP + pt] = val;
                } else {
                    for (int j = 0; j < ratio; ++j)
                        reinterpret_cast<uint32_t*>(p.rec + ((long long)(hk * ratio + j) * p.rec_cap + t0 + t) * REC_BYTES)[pt] = val;
                }
            }
            if (!decode) {
                fd_window_writeback(p, cs, qk_ch, t0, T);
                fd_window_writeback(p, cs, qk_ch + 1, t0, T);
            }
            // ---- each v-head: v channel pt, z column pt, gates; records into the head's stage
            for (int j = 0; j < ratio; ++j) {
                const int hv = hk * ratio + j;
                const int s = k % FD_NSTAGE;
                const uint32_t ph = (uint32_t)(k / FD_NSTAGE) & 1u;
                bool timed_out = false;
                if (k >= FD_NSTAGE && !mbar_wait_bounded(&empty[s], ph ^ 1u, FD_WAIT_NS)) {
                    timed_out = true;
                    atomicOr(r.err, ERR_TIMEOUT);
                    *s_abort = 1;
                }
                if (named_bar_or(FD_BAR_PREP, FD_PREP, timed_out || *s_abort)) {
                    ok = false;
                    break;
                }
                const int vch = 2 * r.hk * DK + hv * DV + pt;
                float wv[4];
                fd_unpack_w(p.conv_w, vch, wv);
                uint8_t* srec = smem + s * FD_STAGE + FD_TILE;
                for (int t = 0; t < T; ++t) {
                    float x[4];
                    fd_taps(p, cs, vch, t0, t, x);
                    if (decode) {
#pragma unroll
                        for (int q = 0; q < KC - 1; ++q) cs[(size_t)q * p.D + vch] = f2bf(x[q + 1]);
                    }
                    const float vo = fd_conv_silu(x, wv, decode);
                    const long long n = (long long)t0 + t;
                    const float zs = silu_bf(bf2f(p.z[n * p.ld_z + (long long)hv * DV + pt]));
                    uint8_t* rec = t < REC_PER_STAGE ? srec + t * REC_BYTES
                                                     : p.rec + ((long long)hv * p.rec_cap + n) * REC_BYTES;
                    reinterpret_cast<uint16_t*>(rec)[256 + pt] = f2bf(vo);
                    reinterpret_cast<uint16_t*>(rec)[384 + pt] = f2bf(zs);
                    if (t < REC_PER_STAGE) reinterpret_cast<uint32_t*>(rec)[pt] = s_qk[t * FD_PREP + pt];
                    if (pt == 0) {
                        const float b = bf2f(p.ab[n * p.ld_ab + hv]);
                        const float av = bf2f(p.ab[n * p.ld_ab + r.hv + hv]);
                        const float sp = gate_softplus(av, p.dt_bias[hv], p.dt_bf16);
                        const float logdecay = -(expf(p.A_log[hv]) * sp);
                        float* gb = reinterpret_cast<float*>(rec + 1024);
                        gb[0] = expf(logdecay);
                        gb[1] = rbf(sigmoid_f32(b));
                        gb[2] = logdecay;
                    }
                }
                if (!decode) fd_window_writeback(p, cs, vch, t0, T);
                named_bar_sync(FD_BAR_PREP, FD_PREP);   // every record of the head is written
                if (pt == 0) mbar_arrive(&full[s]);
                ++k;
            }
        }
        if (ok) {
            // end-of-work marker: the prep's arrival on the producer's sentinel stage
            const int s = k % FD_NSTAGE;
            const uint32_t ph = (uint32_t)(k / FD_NSTAGE) & 1u;
            bool timed_out = false;
            if (k >= FD_NSTAGE && !mbar_wait_bounded(&empty[s], ph ^ 1u, FD_WAIT_NS)) {
                timed_out = true;
                atomicOr(r.err, ERR_TIMEOUT);
                *s_abort = 1;
            }
            if (!named_bar_or(FD_BAR_PREP, FD_PREP, timed_out) && pt == 0) mbar_arrive(&full[s]);
        }
        fd_drain(full, s_issued, s_consumed, tid);
        return;
    }

    // ---------------------------------------------------- consumers (512 threads)
    pdl_wait();
    const int row0 = warp * FD_RPW;
    const int rr = (lane >> 2) & 7;                  // state row (within the warp) this lane's sums land on
    const int oc = warp * 8 + (lane & 7);           // output column written by lanes 0..7
    const float nw = bf2f(r.norm_w[oc]);
    int buf = 0;
    int k = 0;
    int pend_s = -1;   // (thread 0) stage whose state store may still be reading it
    while (true) {
        const int s = k % FD_NSTAGE;
        const uint32_t ph = (uint32_t)(k / FD_NSTAGE) & 1u;
        bool timed_out = false;
        if (!mbar_wait_bounded(&full[s], ph, FD_WAIT_NS)) {
            timed_out = true;
            atomicOr(r.err, ERR_TIMEOUT);
            *s_abort = 1;
        }
        if (named_bar_or(FD_BAR_Y, FD_CONSUMERS, timed_out || *s_abort)) break;
        const FdHdr h = hdr[s];
        if (h.T < 0) break;
        ++k;

        const uint8_t* stage = smem + s * FD_STAGE;
        const float* tile = reinterpret_cast<const float*>(stage);
        float4 S[FD_RPW];
#pragma unroll
        for (int j = 0; j < FD_RPW; ++j) S[j] = *reinterpret_cast<const float4*>(tile + (row0 + j) * DK + lane * 4);

        for (int t = 0; t < h.T; ++t) {
            const uint8_t* rec = t < REC_PER_STAGE ? stage + FD_TILE + t * REC_BYTES
                                                   : r.recs + ((long long)h.hv * r.rec_cap + h.t0 + t) * REC_BYTES;
            const uint2 qu = *reinterpret_cast<const uint2*>(rec + lane * 8);
            const uint2 ku = *reinterpret_cast<const uint2*>(rec + 256 + lane * 8);
            const float vv = bf2f(reinterpret_cast<const uint16_t*>(rec)[256 + row0 + rr]);
            const float zs = bf2f(reinterpret_cast<const uint16_t*>(rec)[384 + oc]);
            const float gt = reinterpret_cast<const float*>(rec + 1024)[0];
            const float bt = reinterpret_cast<const float*>(rec + 1024)[1];
            const float4 q4 = make_float4(__uint_as_float(qu.x << 16), __uint_as_float(qu.x & 0xffff0000u),
                                          __uint_as_float(qu.y << 16), __uint_as_float(qu.y & 0xffff0000u));
            const float4 k4 = make_float4(__uint_as_float(ku.x << 16), __uint_as_float(ku.x & 0xffff0000u),
                                          __uint_as_float(ku.y << 16), __uint_as_float(ku.y & 0xffff0000u));
            float pp[FD_RPW];
#pragma unroll
            for (int j = 0; j < FD_RPW; ++j) {
                S[j].x *= gt; S[j].y *= gt; S[j].z *= gt; S[j].w *= gt;
                pp[j] = S[j].x * k4.x + S[j].y * k4.y + S[j].z * k4.z + S[j].w * k4.w;
            }
            const float kv = reduce_scatter8(pp, lane);
            const float delta = (vv - kv) * bt;
#pragma unroll
            for (int j = 0; j < FD_RPW; ++j) {
                const float d = __shfl_sync(0xffffffffu, delta, 4 * j);
                S[j].x += k4.x * d; S[j].y += k4.y * d; S[j].z += k4.z * d; S[j].w += k4.w * d;
                pp[j] = S[j].x * q4.x + S[j].y * q4.y + S[j].z * q4.z + S[j].w * q4.w;
            }
            const float yv = reduce_scatter8(pp, lane);
            float* sy = s_y + buf * DV;
            if ((lane & 3) == 0) sy[row0 + rr] = rbf(yv);
            named_bar_sync(FD_BAR_Y, FD_CONSUMERS);
            // gated RMSNorm: every warp reduces all 128 y (same order, same result); lanes 0..7 of
            // warp w write output columns 8w..8w+7
            const float4 y4 = *reinterpret_cast<const float4*>(sy + lane * 4);
            const float ss = warp_sum(y4.x * y4.x + y4.y * y4.y + y4.z * y4.z + y4.w * y4.w);
            if (lane < 8) {
                const float nrm = 1.0f / sqrtf(ss / (float)DV + r.eps);
                const float yn = rbf(rbf(sy[oc] * nrm) * nw);
                r.out[(long long)(h.t0 + t) * r.ld_out + (long long)h.hv * DV + oc] = f2bf(zs * yn);
            }
            buf ^= 1;
        }

        // the previous item's state store has had this item's compute to read its stage: release it
        if (tid == 0 && pend_s >= 0) {
            bulk_wait_read_all();
            mbar_arrive(&empty[pend_s]);
            pend_s = -1;
        }
        // state tile back into its stage, then one bulk store to the pool (the copy engine drains it while
        // the consumers go on)
        float* tw = reinterpret_cast<float*>(smem + s * FD_STAGE);
#pragma unroll
        for (int j = 0; j < FD_RPW; ++j) *reinterpret_cast<float4*>(tw + (row0 + j) * DK + lane * 4) = S[j];
        fence_async_shared();
        named_bar_sync(FD_BAR_STORE, FD_CONSUMERS);
        if (tid == 0) {
            bulk_s2g(r.rec + ((size_t)h.slot * r.hv + h.hv) * (DV * DK), tw, FD_TILE);
            bulk_commit();
            pend_s = s;
        }
    }
    if (tid == 0) {
        if (pend_s >= 0) mbar_arrive(&empty[pend_s]);
        bulk_wait_all();   // every state store performed before the CTA ends
        *s_consumed = k;
    }
    fd_drain(full, s_issued, s_consumed, tid);
}

static int g_fd_sms[64] = {0};

cudaError_t launch_decode_fused(const PrepArgs& p, const RecurArgs& r, cudaStream_t stream) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (g_fd_sms[dev] == 0) {
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(gdn_decode_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, FD_SMEM);
        if (e != cudaSuccess) return e;
        g_fd_sms[dev] = sms;
    }
    const int n_groups = r.n_seq * r.hk;
    if (p.n_tokens == 0 || n_groups == 0) return cudaSuccess;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t c = {};
    c.gridDim = dim3((unsigned)(n_groups < g_fd_sms[dev] ? n_groups : g_fd_sms[dev]), 1, 1);
    c.blockDim = dim3(FD_THREADS, 1, 1);
    c.dynamicSmemBytes = FD_SMEM;
    c.stream = stream;
    c.attrs = attr;
    c.numAttrs = 1;
    return cudaLaunchKernelEx(&c, gdn_decode_fused_kernel, p, r);
}

}  // namespace gdn
