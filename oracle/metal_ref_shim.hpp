/*
 * metal_ref_shim.hpp -- run the reference's Metal GDN kernel body on the CPU.
 *
 * TEST INFRASTRUCTURE ONLY (oracle pin).  build_ref.py reads the kernel
 * string GDN_KERNEL_SOURCE from src/models/metal_gdn.rs:10-67 of the
 * reference, wraps it in GDN_SIMDGROUP_SIGNATURE / GDN_PRELUDE and pipes the
 * result to g++ (nothing of the reference is written to disk).  The body is
 * Metal Shading Language, which is C++14 with a few built-ins; this header
 * supplies those built-ins so the body compiles unchanged as C++:
 *
 *   - one call of the body runs one SIMD-group: the 32 lanes execute in lock
 *     step, so every per-lane scalar (`float`, lane indices) becomes a
 *     32-wide value (Lanes<T>), and `simd_sum` is a pairwise tree over lanes;
 *   - device pointers become DevPtr<T>, whose operator[] gathers/scatters
 *     when indexed by a lane vector;
 *   - `bfloat` converts to float exactly and from float by round-to-nearest-even;
 *   - the template parameters InT, StT, T, Hk, Hv, Dk, Dv are supplied as in
 *     metal_gdn.rs:154-165 (grid (32, Dv, B*Hv), threadgroup (32, 4, 1)).
 *
 * The only divergent statement of the body is the lane-0 store of y
 * (metal_gdn.rs:53-55) of a value that simd_sum made uniform; `if` on a lane
 * mask therefore takes lane 0.
 */
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>

namespace mref {

constexpr int W = 32;

struct LF;

struct bfloat {
    uint16_t bits;
    bfloat() = default;
    operator float() const {
        uint32_t u = (uint32_t)bits << 16;
        float f;
        std::memcpy(&f, &u, 4);
        return f;
    }
    static uint16_t from_f32(float f) {
        uint32_t u;
        std::memcpy(&u, &f, 4);
        if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
        u += 0x7fffu + ((u >> 16) & 1u);
        return (uint16_t)(u >> 16);
    }
    explicit bfloat(const LF& v);
};

struct LU {
    uint32_t v[W];
};
struct LMask {
    bool v[W];
    explicit operator bool() const { return v[0]; }
};

struct LF {
    float v[W];
    LF() { for (int l = 0; l < W; ++l) v[l] = 0.0f; }
    LF(float s) { for (int l = 0; l < W; ++l) v[l] = s; }
    LF& operator+=(const LF& o) { for (int l = 0; l < W; ++l) v[l] = v[l] + o.v[l]; return *this; }
};

inline bfloat::bfloat(const LF& x) : bits(from_f32(x.v[0])) {}

inline LF operator+(const LF& a, const LF& b) { LF r; for (int l = 0; l < W; ++l) r.v[l] = a.v[l] + b.v[l]; return r; }
inline LF operator-(const LF& a, const LF& b) { LF r; for (int l = 0; l < W; ++l) r.v[l] = a.v[l] - b.v[l]; return r; }
inline LF operator*(const LF& a, const LF& b) { LF r; for (int l = 0; l < W; ++l) r.v[l] = a.v[l] * b.v[l]; return r; }
inline LF operator*(const LF& a, float s) { LF r; for (int l = 0; l < W; ++l) r.v[l] = a.v[l] * s; return r; }
inline LF operator*(float s, const LF& a) { LF r; for (int l = 0; l < W; ++l) r.v[l] = s * a.v[l]; return r; }
inline LF operator-(float s, const LF& a) { LF r; for (int l = 0; l < W; ++l) r.v[l] = s - a.v[l]; return r; }
inline LF operator-(const LF& a, float s) { LF r; for (int l = 0; l < W; ++l) r.v[l] = a.v[l] - s; return r; }
inline LF operator+(const LF& a, float s) { LF r; for (int l = 0; l < W; ++l) r.v[l] = a.v[l] + s; return r; }

inline LU operator*(int s, const LU& a) { LU r; for (int l = 0; l < W; ++l) r.v[l] = (uint32_t)s * a.v[l]; return r; }
inline LU operator+(const LU& a, int s) { LU r; for (int l = 0; l < W; ++l) r.v[l] = a.v[l] + (uint32_t)s; return r; }
inline LMask operator==(const LU& a, int s) { LMask m; for (int l = 0; l < W; ++l) m.v[l] = a.v[l] == (uint32_t)s; return m; }

/* simd_sum: pairwise tree over the 32 lanes, broadcast to all lanes. */
inline LF simd_sum(const LF& x) {
    float p[W];
    for (int l = 0; l < W; ++l) p[l] = x.v[l];
    for (int off = W / 2; off > 0; off >>= 1)
        for (int l = 0; l < off; ++l) p[l] = p[l] + p[l + off];
    return LF(p[0]);
}

template <class T>
struct LaneRef {
    T* p;
    LU idx;
    operator LF() const { LF r; for (int l = 0; l < W; ++l) r.v[l] = (float)p[idx.v[l]]; return r; }
    LaneRef& operator=(const LF& x) {
        for (int l = 0; l < W; ++l) p[idx.v[l]] = x.v[l];
        return *this;
    }
};

template <class T>
struct DevPtr {
    T* p;
    DevPtr operator+(long o) const { return DevPtr{p + o}; }
    DevPtr& operator+=(long o) { p += o; return *this; }
    T& operator[](long i) const { return p[i]; }
    LaneRef<T> operator[](const LU& i) const { return LaneRef<T>{p, i}; }
};

struct GridPos {
    LU x;
    uint32_t y, z;
};

}  // namespace mref

/*
 * One SIMD-group of the kernel: grid coordinates (y = dv row, z = b*Hv + hv).
 * The body refers to q, k, v, g, beta, state_in, y, state_out and to the
 * template parameters; all are supplied here with the reference's names.
 * build_ref.py emits:  GDN_SIMDGROUP_SIGNATURE { GDN_PRELUDE
 *                      #define float LF  <body>  #undef float }
 * and then includes metal_ref_tail.hpp.
 */
#define GDN_SIMDGROUP_SIGNATURE                                                                           \
    template <int Hk, int Hv, int Dk, int Dv>                                                             \
    static void gdn_simdgroup(mref::DevPtr<const mref::bfloat> q, mref::DevPtr<const mref::bfloat> k,     \
                              mref::DevPtr<const mref::bfloat> v, mref::DevPtr<const float> g,            \
                              mref::DevPtr<const mref::bfloat> beta, mref::DevPtr<const float> state_in,  \
                              mref::DevPtr<mref::bfloat> y, mref::DevPtr<float> state_out, int T,         \
                              uint32_t grid_y, uint32_t grid_z)

#define GDN_PRELUDE                                                                                       \
    using namespace mref;                                                                                 \
    using InT = bfloat;                                                                                   \
    using StT = LF;                                                                                       \
    GridPos thread_position_in_grid, thread_position_in_threadgroup;                                      \
    LU thread_index_in_simdgroup;                                                                         \
    for (int l = 0; l < W; ++l) {                                                                         \
        thread_position_in_grid.x.v[l] = (uint32_t)l;                                                     \
        thread_position_in_threadgroup.x.v[l] = (uint32_t)l;                                              \
        thread_index_in_simdgroup.v[l] = (uint32_t)l;                                                     \
    }                                                                                                     \
    thread_position_in_grid.y = grid_y;                                                                   \
    thread_position_in_grid.z = grid_z;                                                                   \
    thread_position_in_threadgroup.y = grid_y % 4u;                                                       \
    thread_position_in_threadgroup.z = 0u;                                                                \
    (void)thread_position_in_threadgroup;
