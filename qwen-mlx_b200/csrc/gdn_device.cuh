// gdn_device.cuh -- device helpers shared by the GDN kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {

constexpr int DK = 128;        // head_k_dim (specialised)
constexpr int DV = 128;        // head_v_dim (specialised)
constexpr int KC = 4;          // conv taps (linear_conv_kernel_dim)
constexpr int NT = 256;        // threads per CTA of the recurrence kernel
constexpr int NW = NT / 32;    // warps per CTA
constexpr int RPW = DV / NW;   // state rows (dv) per warp = 16

// Error bits recorded in the pool's device error word (1 << GDN_E_*).
constexpr int ERR_BAD_SLOT = 1 << 3;
constexpr int ERR_BAD_SEQLENS = 1 << 4;
constexpr int ERR_TIMEOUT = 1 << 7;  // a bounded device wait gave up (GDN_E_DEVICE)

__device__ __forceinline__ float bf2f(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }
__device__ __forceinline__ uint16_t f2bf(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }
// Round an f32 value to bf16 precision (round-to-nearest-even) and widen back.
__device__ __forceinline__ float rbf(float f) { return bf2f(f2bf(f)); }

// 1 / (1 + exp(-x)); the correctly rounded reciprocal equals the correctly rounded quotient 1 / y.
__device__ __forceinline__ float sigmoid_f32(float x) { return __frcp_rn(1.0f + expf(-x)); }
// nn::silu on a bf16 value: computed in f32, rounded once to bf16.
__device__ __forceinline__ float silu_bf(float x) { return rbf(x * sigmoid_f32(x)); }

// softplus(a + dt_bias) of compiled_beta_g (compiled_ops.rs:36-40).  With an f32 dt_bias, MLX promotes
// a + dt_bias to f32; with a bf16 dt_bias (dt_bf16) the add and its exp are bf16 ops, each rounded to
// bf16, and the + 1 (an f32 constant) promotes back to f32.
__device__ __forceinline__ float gate_softplus(float a, float dt, bool dt_bf16) {
    if (dt_bf16) {
        const float s = rbf(a + dt);
        return logf(rbf(expf(s)) + 1.0f);
    }
    return logf(expf(a + dt) + 1.0f);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Reduce-scatter of 16 per-lane partials across the warp: returns the full
// 32-lane sum of row (lane >> 1).  Lanes 2r and 2r+1 both hold row r's sum.
// 16 shuffles instead of the 80 of 16 independent butterflies.
__device__ __forceinline__ float reduce_scatter16(const float (&p)[16], int lane) {
    float a8[8];
    const bool b4 = lane & 16;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        float send = b4 ? p[j] : p[j + 8];
        float keep = b4 ? p[j + 8] : p[j];
        a8[j] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
    float a4[4];
    const bool b3 = lane & 8;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float send = b3 ? a8[j] : a8[j + 4];
        float keep = b3 ? a8[j + 4] : a8[j];
        a4[j] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    float a2[2];
    const bool b2 = lane & 4;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        float send = b2 ? a4[j] : a4[j + 2];
        float keep = b2 ? a4[j + 2] : a4[j];
        a2[j] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    const bool b1 = lane & 2;
    float send = b1 ? a2[0] : a2[1];
    float keep = b1 ? a2[1] : a2[0];
    float a1 = keep + __shfl_xor_sync(0xffffffffu, send, 2);
    return a1 + __shfl_xor_sync(0xffffffffu, a1, 1);
}

// Reduce-scatter of 8 per-lane partials across the warp: returns the full 32-lane sum of
// partial r = (lane >> 2) & 7 (every lane of a group of 4 holds the same value).
__device__ __forceinline__ float reduce_scatter8(const float (&p)[8], int lane) {
    float a4[4];
    const bool b4 = lane & 16;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float send = b4 ? p[j] : p[j + 4];
        const float keep = b4 ? p[j + 4] : p[j];
        a4[j] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
    float a2[2];
    const bool b3 = lane & 8;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const float send = b3 ? a4[j] : a4[j + 2];
        const float keep = b3 ? a4[j + 2] : a4[j];
        a2[j] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    const bool b2 = lane & 4;
    const float send = b2 ? a2[0] : a2[1];
    float a1 = (b2 ? a2[1] : a2[0]) + __shfl_xor_sync(0xffffffffu, send, 4);
    a1 += __shfl_xor_sync(0xffffffffu, a1, 2);
    a1 += __shfl_xor_sync(0xffffffffu, a1, 1);
    return a1;
}

// The 4 conv taps of channel ch (conv weight [D][4] bf16, 8-byte aligned rows).
__device__ __forceinline__ void fd_unpack_w(const uint16_t* cw, int ch, float (&w)[4]) {
    const uint2 wu = __ldg(reinterpret_cast<const uint2*>(cw + (size_t)ch * KC));
    w[0] = __uint_as_float(wu.x << 16);
    w[1] = __uint_as_float(wu.x & 0xffff0000u);
    w[2] = __uint_as_float(wu.y << 16);
    w[3] = __uint_as_float(wu.y & 0xffff0000u);
}

// silu(sum w x) with the decode (bf16 products + bf16 sum) or conv1d (f32) rounding.
__device__ __forceinline__ float fd_conv_silu(const float (&x)[4], const float (&w)[4], bool decode) {
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

// ---- packed f32 pairs (sm_100 f32x2 arithmetic: each lane of the pair rounds as the scalar operation does)
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
// bf16x2 word (lo in the low half) -> f32 pair, exact
__device__ __forceinline__ uint64_t bf2_to_f2(uint32_t w) {
    return f2_pack(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}
// f32 pair -> bf16x2 word, each rounded to nearest even
__device__ __forceinline__ uint32_t f2_to_bf2(uint64_t v) {
    float lo, hi;
    f2_unpack(v, lo, hi);
    uint32_t d;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}
// silu(x) = x / (1 + e^-x) of a pair for the fast (prefill) paths: e^-x = 2^(-x log2 e) and the reciprocal from
// the PTX approximate instructions (ex2.approx, rcp.approx: a few ulp in f32); x -> -inf gives -0, x -> +inf x.
__device__ __forceinline__ uint64_t f2_silu_fast(uint64_t x) {
    const uint64_t t = f2_mul(x, f2_pack(-1.44269504088896341f, -1.44269504088896341f));
    float t0, t1, e0, e1;
    f2_unpack(t, t0, t1);
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(t0));
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(t1));
    const uint64_t d = f2_add(f2_pack(e0, e1), f2_pack(1.0f, 1.0f));
    float d0, d1, r0, r1;
    f2_unpack(d, d0, d1);
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r0) : "f"(d0));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r1) : "f"(d1));
    return f2_mul(x, f2_pack(r0, r1));
}
// silu of a bf16x2 word, rounded to bf16 as a pair
__device__ __forceinline__ uint32_t bf2_silu_fast(uint32_t w) { return f2_to_bf2(f2_silu_fast(bf2_to_f2(w))); }

}  // namespace gdn
