// gdn_step.cu -- the fused GDN layer step and the stand-alone recurrence (sm_100a).
//
// One CTA owns one (sequence, v-head) pair: its 128x128 f32 state tile
// (64 KiB, [dv][dk] with dk fastest, metal_gdn.rs:25-26) is streamed from the
// slot pool into registers once, carried through all of the sequence's tokens
// of this call, and written back once.  Warp w owns rows dv in [16w, 16w+16);
// lane l owns columns dk in [4l, 4l+4) of each of them, so every load and store
// of the tile is a coalesced 128-bit access (512 contiguous bytes per warp row).
//
// Per token, the fused mode computes in the CTA:
//   conv + SiLU for its q, k and v channels, with the reference's rounding
//     (S=1: bf16 products and bf16 sum, qwen3_5.rs:602-610; S>1: f32 conv1d,
//     qwen3_5.rs:617-623),
//   q/k RMSNorm with gains 1/dk and bf16(dk^-1/2) (qwen3_5.rs:636-639),
//   beta and g (compiled_ops.rs:30-43),
//   the gated delta rule (metal_gdn.rs:37-62) on the register tile,
//   and silu(z) * rms_norm(y, norm_w, eps) (qwen3_5.rs:660-665).
// The v-heads that share a k-head (Hv/Hk of them, metal_gdn.rs:14) form one
// thread-block cluster: they all read the q/k conv state of that k-head, and
// the cluster's rank-0 CTA writes it back only after a cluster barrier, so no
// CTA can overwrite a window another CTA has yet to read.
#include "gdn_device.cuh"
#include "gdn_internal.h"

namespace gdn {

// One conv tap window step for one channel: out = silu(sum_j w[j] * padded[t+j]).
__device__ __forceinline__ float conv_channel(const float (&win)[3], float x, const float (&w)[4], bool decode) {
    float acc;
    if (decode) {
        // padded.multiply(cw) -> bf16 products; sum_axis(1) -> f32 accumulate, bf16 result
        acc = rbf(win[0] * w[0]);
        acc = acc + rbf(win[1] * w[1]);
        acc = acc + rbf(win[2] * w[2]);
        acc = acc + rbf(x * w[3]);
    } else {
        // conv1d: f32 accumulate of exact bf16 x bf16 products, one rounding
        acc = win[0] * w[0];
        acc = acc + win[1] * w[1];
        acc = acc + win[2] * w[2];
        acc = acc + x * w[3];
    }
    return silu_bf(rbf(acc));
}

__device__ __forceinline__ void load_w4(const uint16_t* p, float (&w)[4]) {
    uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
    w[0] = __uint_as_float(u.x << 16);
    w[1] = __uint_as_float(u.x & 0xffff0000u);
    w[2] = __uint_as_float(u.y << 16);
    w[3] = __uint_as_float(u.y & 0xffff0000u);
}

template <bool FUSED>
__global__ void __launch_bounds__(NT, 2) gdn_step_kernel(const StepArgs a) {
    __shared__ __align__(16) float s_q[DK];
    __shared__ __align__(16) float s_k[DK];
    __shared__ float s_v[DV];
    __shared__ float s_z[DV];
    __shared__ float s_y[DV];
    __shared__ float s_red[2][NW];
    __shared__ float s_gb[2];

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int hv = blockIdx.x;
    const int seq = blockIdx.y;
    const int ratio = a.hv / a.hk;
    const int hk = hv / ratio;

    // ---- routing (uniform over the CTA and over its cluster)
    int t0, T;
    if (a.cu_seqlens) {
        t0 = __ldg(a.cu_seqlens + seq);
        T = __ldg(a.cu_seqlens + seq + 1) - t0;
    } else {
        t0 = seq * a.T_dense;
        T = a.T_dense;
    }
    const int slot = a.slot_ids ? __ldg(a.slot_ids + seq) : seq;
    const bool bad_slot = slot < 0 || slot >= a.n_slots;
    const bool bad_len = T < 0 || t0 < 0 || (long long)t0 + T > (long long)a.n_tokens;
    if (bad_slot || bad_len) {
        if (tid == 0 && hv == 0 && a.err) atomicOr(a.err, (bad_slot ? ERR_BAD_SLOT : 0) | (bad_len ? ERR_BAD_SEQLENS : 0));
        return;
    }
    if (T == 0) return;

    // ---- stream the state tile in (issued first; consumed after the prologue)
    const size_t tile = (size_t)DV * DK;
    const size_t tile_off = ((size_t)slot * a.hv + hv) * tile + (size_t)(warp * RPW) * DK + lane * 4;
    const float* st_in = (a.rec_in ? a.rec_in : a.rec) + tile_off;
    float* st_out = a.rec + tile_off;
    float4 S[RPW];
#pragma unroll
    for (int j = 0; j < RPW; ++j) S[j] = __ldcs(reinterpret_cast<const float4*>(st_in + (size_t)j * DK));

    // ---- conv channel ownership: low half = q channel (+ v channel), high half = k channel (+ z)
    const bool low = tid < 128;
    const int c = tid & 127;
    const int qkw = a.hk * DK;
    const int ch0 = low ? hk * DK + c : qkw + hk * DK + c;
    const int ch1 = 2 * qkw + hv * DV + c;
    uint16_t* cs = nullptr;
    float w0[4], w1[4], win0[3], win1[3];
    if constexpr (FUSED) {
        cs = a.conv + (size_t)slot * (KC - 1) * a.D;
        load_w4(a.conv_w + (size_t)ch0 * KC, w0);
#pragma unroll
        for (int j = 0; j < KC - 1; ++j) win0[j] = bf2f(cs[(size_t)j * a.D + ch0]);
        if (low) {
            load_w4(a.conv_w + (size_t)ch1 * KC, w1);
#pragma unroll
            for (int j = 0; j < KC - 1; ++j) win1[j] = bf2f(cs[(size_t)j * a.D + ch1]);
        } else {
#pragma unroll
            for (int j = 0; j < KC - 1; ++j) win1[j] = 0.0f;
#pragma unroll
            for (int j = 0; j < KC; ++j) w1[j] = 0.0f;
        }
        if (ratio > 1) cluster_arrive_release();  // this CTA has read the shared q/k windows
    }
    const bool decode = (T == 1);

    for (int t = 0; t < T; ++t) {
        const long long n = (long long)t0 + t;
        if constexpr (FUSED) {
            const float x0 = bf2f(a.qkv[n * a.ld_qkv + ch0]);
            const float o0 = conv_channel(win0, x0, w0, decode);
            win0[0] = win0[1]; win0[1] = win0[2]; win0[2] = x0;
            float o1 = 0.0f, zs = 0.0f;
            if (low) {
                const float x1 = bf2f(a.qkv[n * a.ld_qkv + ch1]);
                o1 = conv_channel(win1, x1, w1, decode);
                win1[0] = win1[1]; win1[1] = win1[2]; win1[2] = x1;
            } else {
                zs = silu_bf(bf2f(a.z[n * a.ld_z + (long long)hv * DV + c]));
            }
            const float ss = warp_sum(o0 * o0);
            if (lane == 0) s_red[0][warp] = ss;
            if (tid == 0) {
                const float b = bf2f(a.ab[n * a.ld_ab + hv]);
                const float av = bf2f(a.ab[n * a.ld_ab + a.hv + hv]);
                s_gb[1] = rbf(sigmoid_f32(b));
                const float sp = logf(expf(av + a.dt_bias[hv]) + 1.0f);
                s_gb[0] = expf(-(expf(a.A_log[hv]) * sp));
            }
            __syncthreads();
            const float tot = low ? (s_red[0][0] + s_red[0][1]) + (s_red[0][2] + s_red[0][3])
                                  : (s_red[0][4] + s_red[0][5]) + (s_red[0][6] + s_red[0][7]);
            const float nrm = 1.0f / sqrtf(tot / (float)DK + 1e-6f);
            const float gain = low ? 0.0078125f : 0.08837890625f;  // bf16(1/128), bf16(128^-0.5)
            const float nv = rbf(rbf(o0 * nrm) * gain);
            if (low) {
                s_q[c] = nv;
                s_v[c] = o1;
            } else {
                s_k[c] = nv;
                s_z[c] = zs;
            }
            __syncthreads();
        } else {
            if (low) {
                s_q[c] = bf2f(a.q[(n * a.hk + hk) * DK + c]);
                s_v[c] = bf2f(a.v[(n * a.hv + hv) * DV + c]);
            } else {
                s_k[c] = bf2f(a.k[(n * a.hk + hk) * DK + c]);
            }
            if (tid == 0) {
                s_gb[0] = a.g[n * a.hv + hv];
                s_gb[1] = bf2f(a.beta[n * a.hv + hv]);
            }
            __syncthreads();
        }

        // ---- gated delta rule on the register tile (metal_gdn.rs:38-55)
        const float4 k4 = *reinterpret_cast<const float4*>(&s_k[lane * 4]);
        const float4 q4 = *reinterpret_cast<const float4*>(&s_q[lane * 4]);
        const float gt = s_gb[0];
        const float bt = s_gb[1];
        float p[RPW];
#pragma unroll
        for (int j = 0; j < RPW; ++j) {
            S[j].x *= gt; S[j].y *= gt; S[j].z *= gt; S[j].w *= gt;
            p[j] = S[j].x * k4.x + S[j].y * k4.y + S[j].z * k4.z + S[j].w * k4.w;
        }
        const float kv = reduce_scatter16(p, lane);
        const int myrow = warp * RPW + (lane >> 1);
        const float delta = (s_v[myrow] - kv) * bt;
#pragma unroll
        for (int j = 0; j < RPW; ++j) {
            const float d = __shfl_sync(0xffffffffu, delta, 2 * j);
            S[j].x += k4.x * d; S[j].y += k4.y * d; S[j].z += k4.z * d; S[j].w += k4.w * d;
            p[j] = S[j].x * q4.x + S[j].y * q4.y + S[j].z * q4.z + S[j].w * q4.w;
        }
        const float yv = reduce_scatter16(p, lane);

        if constexpr (FUSED) {
            if (!(lane & 1)) s_y[myrow] = rbf(yv);
            __syncthreads();
            // ---- gated RMSNorm epilogue: silu(z) * rms_norm(y, norm_w, eps)
            if (low) {
                const float y1 = s_y[c];
                const float s2 = warp_sum(y1 * y1);
                if (lane == 0) s_red[1][warp] = s2;
            }
            __syncthreads();
            if (low) {
                const float tot = (s_red[1][0] + s_red[1][1]) + (s_red[1][2] + s_red[1][3]);
                const float nrm = 1.0f / sqrtf(tot / (float)DV + a.eps);
                const float yn = rbf(rbf(s_y[c] * nrm) * bf2f(a.norm_w[c]));
                a.out[n * a.ld_out + (long long)hv * DV + c] = f2bf(s_z[c] * yn);
            }
        } else {
            if (!(lane & 1)) a.y[(n * a.hv + hv) * DV + myrow] = f2bf(yv);
            __syncthreads();
        }
    }

    // ---- write the tile back once
#pragma unroll
    for (int j = 0; j < RPW; ++j) __stcs(reinterpret_cast<float4*>(st_out + (size_t)j * DK), S[j]);

    if constexpr (FUSED) {
        if (ratio > 1) cluster_wait_acquire();  // every CTA of the k-head group has read the old windows
        if (low) {
#pragma unroll
            for (int j = 0; j < KC - 1; ++j) cs[(size_t)j * a.D + ch1] = f2bf(win1[j]);
        }
        if (hv % ratio == 0) {
#pragma unroll
            for (int j = 0; j < KC - 1; ++j) cs[(size_t)j * a.D + ch0] = f2bf(win0[j]);
        }
    }
}

// beta = bf16(sigmoid(b)), g = exp(-exp(A_log) * softplus(a + dt_bias))   (compiled_ops.rs:30-43)
__global__ void beta_g_kernel(const uint16_t* __restrict__ ab, long long ld_ab, int n_tokens, int hv,
                              const float* __restrict__ A_log, const float* __restrict__ dt_bias,
                              uint16_t* __restrict__ beta, float* __restrict__ g) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)n_tokens * hv) return;
    const long long t = i / hv;
    const int h = (int)(i % hv);
    const float b = bf2f(ab[t * ld_ab + h]);
    const float av = bf2f(ab[t * ld_ab + hv + h]);
    beta[i] = f2bf(sigmoid_f32(b));
    const float sp = logf(expf(av + dt_bias[h]) + 1.0f);
    g[i] = expf(-(expf(A_log[h]) * sp));
}

static cudaError_t launch_step(const StepArgs& a, bool fused, cudaStream_t stream) {
    const int ratio = a.hv / a.hk;
    dim3 grid(a.hv, a.n_seq, 1);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(NT, 1, 1);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    cfg.attrs = attr;
    cfg.numAttrs = 0;
    if (fused && ratio > 1) {
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = ratio;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.numAttrs = 1;
    }
    if (fused) return cudaLaunchKernelEx(&cfg, gdn_step_kernel<true>, a);
    return cudaLaunchKernelEx(&cfg, gdn_step_kernel<false>, a);
}

cudaError_t launch_layer_step(const StepArgs& a, cudaStream_t stream) { return launch_step(a, true, stream); }
cudaError_t launch_recurrence(const StepArgs& a, cudaStream_t stream) { return launch_step(a, false, stream); }

cudaError_t launch_beta_g(const uint16_t* ab, long long ld_ab, int n_tokens, int hv, const float* A_log,
                          const float* dt_bias, uint16_t* beta, float* g, cudaStream_t stream) {
    const long long n = (long long)n_tokens * hv;
    if (n == 0) return cudaSuccess;
    const int threads = 256;
    const unsigned blocks = (unsigned)((n + threads - 1) / threads);
    beta_g_kernel<<<blocks, threads, 0, stream>>>(ab, ld_ab, n_tokens, hv, A_log, dt_bias, beta, g);
    return cudaGetLastError();
}

}  // namespace gdn
