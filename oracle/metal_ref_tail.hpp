/*
 * metal_ref_tail.hpp -- grid driver and C entry point for the CPU-compiled
 * reference Metal kernel (see metal_ref_shim.hpp).  TEST INFRASTRUCTURE ONLY.
 *
 * mref_gated_delta_kernel has the argument meaning of gated_delta_kernel
 * (metal_gdn.rs:170-173): q,k [B,T,Hk,Dk] bf16, v [B,T,Hv,Dv] bf16,
 * g [B,T,Hv] f32, beta [B,T,Hv] bf16, state_in [B,Hv,Dv,Dk] f32 ->
 * y [B,T,Hv,Dv] bf16, state_out [B,Hv,Dv,Dk] f32 (a separate buffer; the
 * reference zero-initialises outputs, metal_gdn.rs:141).
 */
#pragma once

template <int Hk, int Hv, int Dk, int Dv>
static void gdn_grid(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* g, const uint16_t* beta,
                     const float* state_in, uint16_t* y, float* state_out, int B, int T) {
    using namespace mref;
    std::memset(y, 0, sizeof(uint16_t) * (size_t)B * T * Hv * Dv);
    std::memset(state_out, 0, sizeof(float) * (size_t)B * Hv * Dv * Dk);
    for (int n = 0; n < B * Hv; ++n)
        for (int dv = 0; dv < Dv; ++dv)
            gdn_simdgroup<Hk, Hv, Dk, Dv>(DevPtr<const bfloat>{(const bfloat*)q}, DevPtr<const bfloat>{(const bfloat*)k},
                                          DevPtr<const bfloat>{(const bfloat*)v}, DevPtr<const float>{g},
                                          DevPtr<const bfloat>{(const bfloat*)beta}, DevPtr<const float>{state_in},
                                          DevPtr<bfloat>{(bfloat*)y}, DevPtr<float>{state_out}, T, (uint32_t)dv,
                                          (uint32_t)n);
}

extern "C" int mref_gated_delta_kernel(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* g,
                                       const uint16_t* beta, const float* state_in, int T, int B, int hk, int hv,
                                       int dk, int dv, uint16_t* y, float* state_out) {
#define MREF_CASE(HK, HV, DK, DV)                                                        \
    if (hk == HK && hv == HV && dk == DK && dv == DV) {                                  \
        gdn_grid<HK, HV, DK, DV>(q, k, v, g, beta, state_in, y, state_out, B, T);        \
        return 0;                                                                        \
    }
    MREF_CASE(16, 32, 128, 128)
    MREF_CASE(2, 4, 128, 128)
    MREF_CASE(1, 2, 128, 128)
    MREF_CASE(2, 2, 128, 128)
    MREF_CASE(2, 2, 64, 32)
    MREF_CASE(4, 8, 32, 64)
#undef MREF_CASE
    return 1;
}
