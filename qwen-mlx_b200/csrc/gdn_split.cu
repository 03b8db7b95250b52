// gdn_split.cu -- the decode layer step for calls of few sequences: each (sequence, v-head) state
// tile is split by dv rows over 4 CTAs of a thread-block cluster (sm_100a).
//
// A cluster of 4 * (Hv/Hk) CTAs serves one (sequence, k-head).  CTA rank c takes v-head
// hk * (Hv/Hk) + c / 4 and state rows [32 (c % 4), +32): a 16 KiB slice of the f32 tile [dv][dk]
// (metal_gdn.rs:25-26).  The reference's own grid splits dv the same way (one thread row per dv,
// metal_gdn.rs:154-155); here a small batch becomes 4x as many independent streams, so every SM has
// work and a slice's bytes move while others compute.  Per CTA (128 threads):
//   * every CTA repeats the k-head's q/k prep -- conv + SiLU of its 256 channels with the decode
//     rounding of a one-token segment (qwen3_5.rs:602-610; f32 conv1d for longer segments,
//     :617-623), RMSNorm with the gains bf16(1/dk) and bf16(dk^-1/2) (:636-639) -- cheaper than a
//     round of exchange; warp 0 does the v channels of its 32 rows, warp 1 silu(z) of those rows,
//     thread 64 beta and g (compiled_ops.rs:30-43);
//   * the gated delta rule on the slice (metal_gdn.rs:37-62): warp w rows 8w..8w+7, lane l columns
//     4l..4l+3, row sums by a reduce-scatter over the lanes;
//   * the gated RMSNorm (qwen3_5.rs:660-665) needs sum(y^2) over all 128 rows of the head: the 4 CTAs
//     of a head write their partial sums into each other's shared memory (distributed shared memory,
//     plain stores) and meet at a cluster barrier, one per token;
//   * the conv windows of the k-head's q/k channels are read by every CTA of the cluster and those of
//     a v-head by its 4 CTAs.  All reads happen before a CTA's first cluster-barrier arrival and all
//     in-place window updates after its wait, so no window is overwritten before every reader has
//     it; the updates are divided among the CTAs (32 of the q/k channels each, and the CTA's own 32 v
//     channels).
// The state slice arrives with one bulk async copy (non-tensor, no multicast) completing on an
// mbarrier and leaves with one bulk store.
//
// PDL.  With tables_stable the routing entries, the state slice, the conv windows and the weights are
// read before griddepcontrol.wait; the kernel releases its dependents right after the wait.  The next
// layer's CTAs (16.9 KiB of shared memory each) fit beside this layer's and stream their own slices
// while this layer computes.  This is safe because a grid passes griddepcontrol.wait only when every
// earlier kernel of the stream has completed, and the next grid launches only after all of this grid's
// CTAs have passed it, so everything that wrote the next layer's state has completed by then.
//
// Every wait is bounded: the mbarrier wait for the slice gives up after ctl.wait_ns (2 s in normal
// use), records 1 << 7 in the error word and skips the slice's update; the CTA still meets its
// cluster at every barrier, so its peers never wait for it.
#include "gdn_device.cuh"
#include "gdn_internal.h"
#include "gdn_ptx.cuh"

namespace gdn {

constexpr int SP_THREADS = 128;
constexpr int SP_ROWS = 32;                    // state rows (dv) per CTA
constexpr int SP_RPW = SP_ROWS / 4;            // 8 rows per warp
constexpr int SP_SLICE = SP_ROWS * DK * 4;     // 16 KiB
static_assert(SP_RPW == 8, "reduce_scatter8 covers 8 rows per warp");

__global__ void __launch_bounds__(SP_THREADS, 8) gdn_decode_split_kernel(const PrepArgs p, const RecurArgs r,
                                                                      const SplitCtl ctl) {
    __shared__ __align__(128) float s_tile[SP_ROWS * DK];   // the state slice [32][128]
    __shared__ __align__(16) float s_qn[DK];                // q after conv, SiLU, RMSNorm, gain (bf16 values)
    __shared__ __align__(16) float s_kn[DK];                // k, likewise
    __shared__ float s_v[SP_ROWS];                          // v of this CTA's rows
    __shared__ float s_z[SP_ROWS];                          // silu(z) of this CTA's rows
    __shared__ float s_y[SP_ROWS];                          // bf16(y) of this CTA's rows
    __shared__ float s_red[4];                              // q / k sums of squares per warp
    __shared__ float s_ss[4];                               // sum(y^2) per warp
    __shared__ float s_part[2][4];                          // sum(y^2) of the head's 4 CTAs (written by them)
    __shared__ float s_gate[2];                             // g, beta
    __shared__ __align__(8) uint64_t s_full;
    __shared__ int s_timeout;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ratio = r.hv / r.hk;
    const int csize = 4 * ratio;
    const int crank = (int)(blockIdx.x % (unsigned)csize);   // == %cluster_ctarank (1-D clusters of csize)
    const int grp = (int)(blockIdx.x / (unsigned)csize);
    const int seq = grp / r.hk, hk = grp - seq * r.hk;
    const int jh = crank >> 2, qd = crank & 3;
    const int hv = hk * ratio + jh;
    const int row0 = SP_ROWS * qd;
    const bool is_q = tid < 64;
    const int qk_ch = (is_q ? 0 : r.hk * DK) + hk * DK + 2 * (tid & 63);
    const int v_ch = 2 * r.hk * DK + hv * DV + row0 + lane;   // warp 0
    const uint64_t wait_ns = ctl.wait_ns;

    if (tid == 0) {
        mbar_init(&s_full, 1);
        s_timeout = 0;
        fence_mbar_init();
    }
    __syncthreads();
    // the cluster's CTAs must all be running before one stores into another's shared memory: this
    // arrival is waited for before the first such store
    cluster_arrive_relaxed();

    // ---- routing, state slice, windows, weights: before the PDL wait when the tables are stable
    int t0 = 0, T = 0, slot = 0;
    bool ok = false, copied = false;
    float xq0[KC], xq1[KC], xv[KC], wq0[KC], wq1[KC], wv[KC];
    float nw = 0.f, a_log = 0.f, dt_b = 0.f;
    auto fetch = [&]() {
        t0 = __ldg(r.cu_seqlens + seq);
        T = __ldg(r.cu_seqlens + seq + 1) - t0;
        slot = __ldg(r.slot_ids + seq);
        const bool bad_slot = slot < 0 || slot >= r.n_slots;
        const bool bad_len = T < 0 || t0 < 0 || t0 + T > r.n_tokens;
        if ((bad_slot || bad_len) && hk == 0 && crank == 0 && tid == 0)
            atomicOr(r.err, (bad_slot ? ERR_BAD_SLOT : 0) | (bad_len ? ERR_BAD_SEQLENS : 0));
        ok = !bad_slot && !bad_len && T > 0;
        if (!ok) return;
        if (tid == 0) {
            const float* src = (r.rec_in ? r.rec_in : r.rec) + (((size_t)slot * r.hv + hv) * DV + row0) * DK;
            mbar_arrive_expect_tx(&s_full, SP_SLICE);
            // ctl.skip_block (failure-detection tests only): the barrier is armed but that CTA's copy is
            // never issued, so its bounded wait runs out
            if ((int)blockIdx.x != ctl.skip_block) {
                bulk_g2s(s_tile, src, SP_SLICE, &s_full);
                copied = true;
            }
        }
        const uint16_t* cs = p.conv + (size_t)slot * (KC - 1) * p.D;
#pragma unroll
        for (int j = 0; j < KC - 1; ++j) {
            xq0[j] = bf2f(cs[(size_t)j * p.D + qk_ch]);
            xq1[j] = bf2f(cs[(size_t)j * p.D + qk_ch + 1]);
        }
        fd_unpack_w(p.conv_w, qk_ch, wq0);
        fd_unpack_w(p.conv_w, qk_ch + 1, wq1);
        if (warp == 0) {
#pragma unroll
            for (int j = 0; j < KC - 1; ++j) xv[j] = bf2f(cs[(size_t)j * p.D + v_ch]);
            fd_unpack_w(p.conv_w, v_ch, wv);
            nw = bf2f(r.norm_w[row0 + lane]);
        }
        if (tid == 64) {
            a_log = p.A_log[hv];
            dt_b = p.dt_bias[hv];
        }
    };
    if (p.tables_stable) fetch();
    pdl_wait();
    pdl_launch_dependents();
    if (!p.tables_stable) fetch();
    if (!ok) return;   // uniform over the cluster: every CTA of it serves the same sequence

    const float gain = is_q ? 0.0078125f : 0.08837890625f;   // bf16(1/128), bf16(128^-0.5)
    const bool decode = T == 1;
    float4 S[SP_RPW];
    bool have_state = false;
    const int rr = (lane >> 2) & 7;     // row (within the warp) whose sums this lane holds
    for (int t = 0; t < T; ++t) {
        const long long n = (long long)t0 + t;
        // ---- prep of token n: conv taps [window; tokens] roll through x*[0..3]
        xq0[KC - 1] = bf2f(p.qkv[n * p.ld_qkv + qk_ch]);
        xq1[KC - 1] = bf2f(p.qkv[n * p.ld_qkv + qk_ch + 1]);
        float zraw = 0.f, b_raw = 0.f, a_raw = 0.f;
        if (warp == 0) xv[KC - 1] = bf2f(p.qkv[n * p.ld_qkv + v_ch]);
        if (warp == 1) zraw = bf2f(p.z[n * p.ld_z + (long long)hv * DV + row0 + lane]);
        if (tid == 64) {
            b_raw = bf2f(p.ab[n * p.ld_ab + hv]);
            a_raw = bf2f(p.ab[n * p.ld_ab + r.hv + hv]);
        }
        const float o0 = fd_conv_silu(xq0, wq0, decode);
        const float o1 = fd_conv_silu(xq1, wq1, decode);
        const float ss = warp_sum(o0 * o0 + o1 * o1);
        if (lane == 0) s_red[warp] = ss;
        if (warp == 0) s_v[lane] = fd_conv_silu(xv, wv, decode);
        if (warp == 1) s_z[lane] = silu_bf(zraw);
        if (tid == 64) {
            const float sp = gate_softplus(a_raw, dt_b, p.dt_bf16);
            s_gate[0] = expf(-(expf(a_log) * sp));
            s_gate[1] = rbf(sigmoid_f32(b_raw));
        }
        __syncthreads();
        {
            const float tot = is_q ? s_red[0] + s_red[1] : s_red[2] + s_red[3];
            const float nrm = 1.0f / sqrtf(tot / (float)DK + 1e-6f);
            float* dst = (is_q ? s_qn : s_kn) + 2 * (tid & 63);
            dst[0] = bf2f(f2bf(rbf(o0 * nrm) * gain));
            dst[1] = bf2f(f2bf(rbf(o1 * nrm) * gain));
        }
#pragma unroll
        for (int j = 0; j < KC - 1; ++j) {   // the window after this token
            xq0[j] = xq0[j + 1];
            xq1[j] = xq1[j + 1];
            xv[j] = xv[j + 1];
        }
        if (t == 0) {
            // the state slice (bounded wait; a copy that never lands leaves this CTA's rows untouched)
            if (tid == 0 && !mbar_wait_bounded(&s_full, 0, wait_ns)) {
                s_timeout = 1;
                atomicOr(r.err, ERR_TIMEOUT);
            }
            __syncthreads();
            have_state = !s_timeout;
            if (have_state) {
#pragma unroll
                for (int j = 0; j < SP_RPW; ++j)
                    S[j] = *reinterpret_cast<const float4*>(s_tile + (warp * SP_RPW + j) * DK + lane * 4);
            }
        } else {
            __syncthreads();
        }

        // ---- gated delta rule on this CTA's 32 rows
        float yb = 0.f;
        if (have_state) {
            const float gt = s_gate[0], bt = s_gate[1];
            const float4 q4 = *reinterpret_cast<const float4*>(s_qn + lane * 4);
            const float4 k4 = *reinterpret_cast<const float4*>(s_kn + lane * 4);
            float pp[SP_RPW];
#pragma unroll
            for (int j = 0; j < SP_RPW; ++j) {
                S[j].x *= gt; S[j].y *= gt; S[j].z *= gt; S[j].w *= gt;
                pp[j] = S[j].x * k4.x + S[j].y * k4.y + S[j].z * k4.z + S[j].w * k4.w;
            }
            const float kv = reduce_scatter8(pp, lane);
            const float delta = (s_v[warp * SP_RPW + rr] - kv) * bt;
#pragma unroll
            for (int j = 0; j < SP_RPW; ++j) {
                const float d = __shfl_sync(0xffffffffu, delta, 4 * j);
                S[j].x += k4.x * d; S[j].y += k4.y * d; S[j].z += k4.z * d; S[j].w += k4.w * d;
                pp[j] = S[j].x * q4.x + S[j].y * q4.y + S[j].z * q4.z + S[j].w * q4.w;
            }
            yb = rbf(reduce_scatter8(pp, lane));
        }
        const bool row_lane = (lane & 3) == 0;
        if (row_lane) s_y[warp * SP_RPW + rr] = yb;
        const float ssy = warp_sum(row_lane ? yb * yb : 0.f);
        if (lane == 0) s_ss[warp] = ssy;
        __syncthreads();
        // ---- sum(y^2) over the head: this CTA's partial into slot [t & 1][qd] of the head's 4 CTAs
        if (t == 0) cluster_wait();   // every CTA of the cluster is running
        if (tid < 4) {
            const float part = s_ss[0] + s_ss[1] + s_ss[2] + s_ss[3];
            st_cluster_f32(&s_part[t & 1][qd], (uint32_t)(jh * 4 + tid), part);
        }
        cluster_arrive();
        cluster_wait();
        if (warp == 0) {
            const float* pt = s_part[t & 1];
            const float tot = pt[0] + pt[1] + pt[2] + pt[3];
            const float nrm = 1.0f / sqrtf(tot / (float)DV + r.eps);
            const float yn = rbf(rbf(s_y[lane] * nrm) * nw);
            if (have_state) r.out[n * r.ld_out + (long long)hv * DV + row0 + lane] = f2bf(s_z[lane] * yn);
        }
    }

    // ---- the slice back to the pool (one bulk store)
    if (have_state) {
#pragma unroll
        for (int j = 0; j < SP_RPW; ++j)
            *reinterpret_cast<float4*>(s_tile + (warp * SP_RPW + j) * DK + lane * 4) = S[j];
        fence_async_shared();
    }
    __syncthreads();
    if (tid == 0) {
        if (have_state) {
            bulk_s2g(r.rec + (((size_t)slot * r.hv + hv) * DV + row0) * DK, s_tile, SP_SLICE);
            bulk_commit();
        } else if (copied) {
            mbar_wait_bounded(&s_full, 0, wait_ns);   // a copy still in flight must land before the CTA ends
        }
    }
    // ---- conv windows: every reader of them in the cluster passed the first cluster barrier; this CTA
    // writes q/k channel pairs of threads [16 c, 16 c + 16) for the c with c % csize == crank, and its own
    // 32 v channels
    uint16_t* cs = p.conv + (size_t)slot * (KC - 1) * p.D;
    if (((tid >> 4) % csize) == crank) {
#pragma unroll
        for (int j = 0; j < KC - 1; ++j) {
            cs[(size_t)j * p.D + qk_ch] = f2bf(xq0[j]);
            cs[(size_t)j * p.D + qk_ch + 1] = f2bf(xq1[j]);
        }
    }
    if (warp == 0) {
#pragma unroll
        for (int j = 0; j < KC - 1; ++j) cs[(size_t)j * p.D + v_ch] = f2bf(xv[j]);
    }
    if (tid == 0 && have_state) bulk_wait_all();   // the slice is written before the CTA ends
}

static int g_sp_ready[64] = {0};

cudaError_t launch_decode_split(const PrepArgs& p, const RecurArgs& r, const SplitCtl& ctl, cudaStream_t stream) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (r.hk <= 0 || r.hv % r.hk || r.hv / r.hk > 2) return cudaErrorInvalidValue;
    if (!g_sp_ready[dev]) {
        e = cudaFuncSetAttribute(gdn_decode_split_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
        if (e != cudaSuccess) return e;
        g_sp_ready[dev] = 1;
    }
    if (p.n_tokens == 0 || r.n_seq == 0) return cudaSuccess;
    const int csize = 4 * (r.hv / r.hk);
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)csize;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cudaLaunchConfig_t c = {};
    c.gridDim = dim3((unsigned)(r.n_seq * r.hk * csize), 1, 1);
    c.blockDim = dim3(SP_THREADS, 1, 1);
    c.dynamicSmemBytes = 0;
    c.stream = stream;
    c.attrs = attr;
    c.numAttrs = 2;
    return cudaLaunchKernelEx(&c, gdn_decode_split_kernel, p, r, ctl);
}

}  // namespace gdn
