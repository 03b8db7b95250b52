// gdn_step.cu -- the stand-alone gated delta recurrence (sm_100a): the drop-in
// for gated_delta_kernel (metal_gdn.rs:170-218), on pool slots or on dense
// reference-layout state arrays.
//
// One CTA owns one (sequence, v-head) pair: its 128x128 f32 state tile
// (64 KiB, [dv][dk] with dk fastest, metal_gdn.rs:25-26) is loaded into
// registers once, carried through all of the sequence's tokens of this call,
// and written back once.  Warp w owns rows dv in [16w, 16w+16); lane l owns
// columns dk in [4l, 4l+4) of each of them, so every load and store of the tile
// is a coalesced 128-bit access (512 contiguous bytes per warp row).  Per token
// the CTA stages q, k (its k-head, metal_gdn.rs:14), v, g and beta in shared
// memory and runs the rule of metal_gdn.rs:38-55 on the register tile; the row
// sums use a 16-shuffle reduce-scatter per warp.
#include "gdn_device.cuh"
#include "gdn_internal.h"

namespace gdn {

__global__ void __launch_bounds__(NT, 2) gdn_recurrence_kernel(const StepArgs a) {
    __shared__ __align__(16) float s_q[DK];
    __shared__ __align__(16) float s_k[DK];
    __shared__ float s_v[DV];
    __shared__ float s_gb[2];

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int hv = blockIdx.x;
    const int seq = blockIdx.y;
    const int ratio = a.hv / a.hk;
    const int hk = hv / ratio;

    // ---- routing (uniform over the CTA)
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

    // ---- the state tile: loads issued first, consumed after the first token's operands arrive
    const size_t tile = (size_t)DV * DK;
    const size_t tile_off = ((size_t)slot * a.hv + hv) * tile + (size_t)(warp * RPW) * DK + lane * 4;
    const float* st_in = (a.rec_in ? a.rec_in : a.rec) + tile_off;
    float* st_out = a.rec + tile_off;
    float4 S[RPW];
#pragma unroll
    for (int j = 0; j < RPW; ++j) S[j] = __ldcs(reinterpret_cast<const float4*>(st_in + (size_t)j * DK));

    const bool low = tid < 128;
    const int c = tid & 127;

    for (int t = 0; t < T; ++t) {
        const long long n = (long long)t0 + t;
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
        if (!(lane & 1)) a.y[(n * a.hv + hv) * DV + myrow] = f2bf(yv);
        __syncthreads();   // the staged operands are rewritten by the next token
    }

    // ---- write the tile back once
#pragma unroll
    for (int j = 0; j < RPW; ++j) __stcs(reinterpret_cast<float4*>(st_out + (size_t)j * DK), S[j]);
}

// beta = bf16(sigmoid(b)), g = exp(-exp(A_log) * softplus(a + dt_bias))   (compiled_ops.rs:30-43)
__global__ void beta_g_kernel(const uint16_t* __restrict__ ab, long long ld_ab, int n_tokens, int hv,
                              const float* __restrict__ A_log, const float* __restrict__ dt_bias, int dt_bf16,
                              uint16_t* __restrict__ beta, float* __restrict__ g) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)n_tokens * hv) return;
    const long long t = i / hv;
    const int h = (int)(i % hv);
    const float b = bf2f(ab[t * ld_ab + h]);
    const float av = bf2f(ab[t * ld_ab + hv + h]);
    beta[i] = f2bf(sigmoid_f32(b));
    const float sp = gate_softplus(av, dt_bias[h], dt_bf16 != 0);
    g[i] = expf(-(expf(A_log[h]) * sp));
}

cudaError_t launch_recurrence(const StepArgs& a, cudaStream_t stream) {
    gdn_recurrence_kernel<<<dim3(a.hv, a.n_seq, 1), NT, 0, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_beta_g(const uint16_t* ab, long long ld_ab, int n_tokens, int hv, const float* A_log,
                          const float* dt_bias, int dt_bf16, uint16_t* beta, float* g, cudaStream_t stream) {
    const long long n = (long long)n_tokens * hv;
    if (n == 0) return cudaSuccess;
    const int threads = 256;
    const unsigned blocks = (unsigned)((n + threads - 1) / threads);
    beta_g_kernel<<<blocks, threads, 0, stream>>>(ab, ld_ab, n_tokens, hv, A_log, dt_bias, dt_bf16, beta, g);
    return cudaGetLastError();
}

}  // namespace gdn
