// gdn_attn.cu -- the full-attention layer body of the hybrid decoder (Qwen35Attention::forward_with_cache,
// src/models/qwen3_5.rs:377-459) over a continuously batched, ragged step with a slot-indexed KV cache.
//
// Three kernels per call, all HBM- or latency-bound (decode reads each cached key and value once per
// kv head; no GEMM-shaped work is left once the projections are done):
//   gdn_attn_prep_kernel     one CTA per (token, head of q | k | v): q/k RMSNorm (MLX fast::rms_norm
//                            rounding: x * rsqrt(mean x^2 + eps) rounded to bf16, times the gain, rounded),
//                            rotate-half RoPE on the first rotary_dim dims (f32, rounded once), q into the
//                            workspace, k and v into the cache row of the token's position;
//   gdn_attn_split_kernel    one CTA per (token, kv head, key split) with one warp per q head of the GQA
//                            group: the group shares every K / V row it streams; online softmax in f32
//                            (log2 domain) over the split's keys, partial (max, sum, acc) to the workspace;
//   gdn_attn_combine_kernel  one CTA per (token, q head): merges the splits, rounds the attention output to
//                            bf16 and applies the sigmoid output gate (qwen3_5.rs:455-456).
// Each token sees exactly the keys [0, its position] of its own slot, whatever the other sequences of the
// step hold (the reference's batched executor zero-pads ragged caches and runs SDPA unmasked,
// src/scheduler/mlx_executor.rs:57-86).  Splits past a token's context write max = -inf and the combine
// skips them, so a token's result does not depend on the split count the batch chose.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <vector>

#include "gdn.h"
#include "gdn_device.cuh"
#include "gdn_hybrid.h"
#include "gdn_internal.h"

namespace gdn {
namespace {

constexpr int AP_THREADS = 128;       // prep CTA: head_dim / 128 dims per thread
constexpr int SPLIT_KEYS_MIN = 256;   // keys per split CTA, at least
constexpr int MAX_SPLITS = 64;
constexpr float LOG2E = 1.4426950408889634f;

struct AttnArgs {
    const uint16_t* q_full; const uint16_t* k_in; const uint16_t* v_in;
    const uint16_t* qn_w; const uint16_t* kn_w;
    uint16_t* k_cache; uint16_t* v_cache;
    const int32_t* tok_slot;   // [N]
    const int32_t* tok_pos;    // [N] position of the token (its context is [0, pos])
    uint16_t* qbuf;            // [N][nh][hd] roped, normalised q
    float* part_m;             // [N][nh][ns] running max (log2 units)
    float* part_l;             // [N][nh][ns] running sum
    float* part_acc;           // [N][nh][ns][hd]
    uint16_t* out;             // [N][nh*hd]
    int n_tokens, nh, nkv, hd, rot, max_ctx, n_split, split_keys;
    float eps, log2_theta, scale_log2;
};

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Workspace carve-up shared by the size query and the step.
struct AttnLayout {
    size_t tok_slot, tok_pos, qbuf, part_m, part_l, part_acc, total;
};

AttnLayout attn_layout(int N, int nh, int hd, int ns) {
    AttnLayout L{};
    size_t o = 0;
    L.tok_slot = o;                                   // [slot x N | position x N]: one upload
    L.tok_pos = o + sizeof(int32_t) * N;
    o = align256(o + 2 * sizeof(int32_t) * N);
    L.qbuf = o;     o = align256(o + sizeof(uint16_t) * (size_t)N * nh * hd);
    L.part_m = o;   o = align256(o + sizeof(float) * (size_t)N * nh * ns);
    L.part_l = o;   o = align256(o + sizeof(float) * (size_t)N * nh * ns);
    L.part_acc = o; o = align256(o + sizeof(float) * (size_t)N * nh * ns * hd);
    L.total = o;
    return L;
}

// Splits of the key range: enough CTAs to cover the SMs a few times over at decode, one split when the
// (token, kv head) pairs already do (prefill), and never a split shorter than SPLIT_KEYS_MIN keys.
int attn_splits(int N, int nkv, int max_kv) {
    if (max_kv <= 0 || N <= 0) return 1;
    const int by_len = (max_kv + SPLIT_KEYS_MIN - 1) / SPLIT_KEYS_MIN;
    const int pairs = N * nkv;
    const int by_grid = pairs >= 4 * 148 ? 1 : (4 * 148 + pairs - 1) / pairs;
    int ns = by_len < by_grid ? by_len : by_grid;
    if (ns > MAX_SPLITS) ns = MAX_SPLITS;
    return ns < 1 ? 1 : ns;
}

__device__ __forceinline__ float block_sum128(float v, float* red) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    const float s = red[0] + red[1] + red[2] + red[3];
    __syncthreads();
    return s;
}

// blockIdx.x = token, blockIdx.y = head: [0, nh) q heads, [nh, nh + nkv) k heads, [nh + nkv, nh + 2 nkv) v heads.
__global__ void __launch_bounds__(AP_THREADS) gdn_attn_prep_kernel(const AttnArgs a) {
    __shared__ float s_y[256];
    __shared__ float red[4];
    const int t = blockIdx.x, head = blockIdx.y, tid = threadIdx.x;
    const int hd = a.hd;   // dims tid and tid + 128 of the head (hd 64 leaves half the CTA idle)
    const int slot = a.tok_slot[t], pos = a.tok_pos[t];
    const bool is_q = head < a.nh, is_k = !is_q && head < a.nh + a.nkv;
    const uint16_t* src;
    if (is_q) src = a.q_full + (size_t)t * (2 * a.nh * hd) + (size_t)head * 2 * hd;      // [q | gate] per head
    else if (is_k) src = a.k_in + (size_t)t * (a.nkv * hd) + (size_t)(head - a.nh) * hd;
    else src = a.v_in + (size_t)t * (a.nkv * hd) + (size_t)(head - a.nh - a.nkv) * hd;

    float x[2] = {0.f, 0.f};
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int d = tid + i * AP_THREADS;
        if (d < hd) {
            x[i] = bf2f(src[d]);
            ss += x[i] * x[i];
        }
    }
    if (!is_q && !is_k) {   // v: the projection output as is
        const int kvh = head - a.nh - a.nkv;
        uint16_t* dst = a.v_cache + (((size_t)slot * a.nkv + kvh) * a.max_ctx + pos) * hd;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int d = tid + i * AP_THREADS;
            if (d < hd) dst[d] = src[d];
        }
        return;
    }
    const float tot = block_sum128(ss, red);
    const float nrm = 1.0f / sqrtf(tot / (float)hd + a.eps);
    const uint16_t* gw = is_q ? a.qn_w : a.kn_w;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int d = tid + i * AP_THREADS;
        if (d < hd) s_y[d] = rbf(bf2f(gw[d]) * rbf(x[i] * nrm));
    }
    __syncthreads();
    uint16_t* dst;
    if (is_q) dst = a.qbuf + ((size_t)t * a.nh + head) * hd;
    else dst = a.k_cache + (((size_t)slot * a.nkv + (head - a.nh)) * a.max_ctx + pos) * hd;
    const int half = a.rot >> 1;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int d = tid + i * AP_THREADS;
        if (d >= hd) continue;
        float r = s_y[d];
        if (d < a.rot) {
            const int fi = d < half ? d : d - half;
            // angle = pos * theta^(-fi / half), as pos * 2^(-fi * log2(theta) / half)
            const float inv_freq = exp2f(-(float)fi * a.log2_theta / (float)half);
            float sn, cs;
            sincosf((float)pos * inv_freq, &sn, &cs);
            r = d < half ? s_y[d] * cs - s_y[d + half] * sn : s_y[d - half] * sn + s_y[d] * cs;
        }
        dst[d] = f2bf(r);
    }
}

// DPL consecutive bf16 of a row (DPL * 2 bytes, aligned to that size) widened to f32: one 16-, 8- or 4-byte load.
template <int DPL>
__device__ __forceinline__ void load_dims(const uint16_t* p, float (&x)[DPL]) {
    uint32_t w[DPL / 2];
    if constexpr (DPL == 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(p);
        w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    } else if constexpr (DPL == 4) {
        const uint2 v = *reinterpret_cast<const uint2*>(p);
        w[0] = v.x; w[1] = v.y;
    } else {
        w[0] = *reinterpret_cast<const uint32_t*>(p);
    }
#pragma unroll
    for (int i = 0; i < DPL / 2; ++i) {
        x[2 * i] = __uint_as_float(w[i] << 16);
        x[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
}

// blockIdx = (token, kv head, split); warp w = q head kvh * G + w.  Lane l holds dims [l * DPL, +DPL).
template <int HD>
__global__ void __launch_bounds__(512) gdn_attn_split_kernel(const AttnArgs a) {
    constexpr int DPL = HD / 32;
    const int t = blockIdx.x, kvh = blockIdx.y, sp = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = a.nh / a.nkv;
    const int h = kvh * G + warp;
    const int slot = a.tok_slot[t];
    const int ctx = a.tok_pos[t] + 1;
    const int k0 = sp * a.split_keys;
    const int k1 = min(ctx, k0 + a.split_keys);
    const size_t pi = ((size_t)t * a.nh + h) * a.n_split + sp;
    if (k0 >= k1) {
        if (lane == 0) {
            a.part_m[pi] = -INFINITY;
            a.part_l[pi] = 0.f;
        }
        return;
    }
    float q[DPL];
    load_dims<DPL>(a.qbuf + ((size_t)t * a.nh + h) * HD + lane * DPL, q);
#pragma unroll
    for (int i = 0; i < DPL; ++i) q[i] *= a.scale_log2;
    const size_t base = (((size_t)slot * a.nkv + kvh) * a.max_ctx) * HD + lane * DPL;
    const uint16_t* kb = a.k_cache + base;
    const uint16_t* vb = a.v_cache + base;
    float m = -INFINITY, l = 0.f, acc[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[i] = 0.f;

    constexpr int KB = 4;   // keys per step: their loads and reductions overlap
    for (int j0 = k0; j0 < k1; j0 += KB) {
        float kx[KB][DPL], vx[KB][DPL], s[KB];
#pragma unroll
        for (int u = 0; u < KB; ++u) {
            const int j = j0 + u;
            if (j < k1) {
                load_dims<DPL>(kb + (size_t)j * HD, kx[u]);
                load_dims<DPL>(vb + (size_t)j * HD, vx[u]);
            } else {
#pragma unroll
                for (int i = 0; i < DPL; ++i) { kx[u][i] = 0.f; vx[u][i] = 0.f; }
            }
        }
#pragma unroll
        for (int u = 0; u < KB; ++u) {
            float d = 0.f;
#pragma unroll
            for (int i = 0; i < DPL; ++i) d = fmaf(q[i], kx[u][i], d);
            s[u] = d;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
            for (int u = 0; u < KB; ++u) s[u] += __shfl_xor_sync(0xffffffffu, s[u], o);
        }
        float mn = m;
#pragma unroll
        for (int u = 0; u < KB; ++u) {
            if (j0 + u >= k1) s[u] = -INFINITY;
            mn = fmaxf(mn, s[u]);
        }
        const float alpha = exp2f(m - mn);   // m = -inf on the first step: alpha = 0 (acc, l are 0)
        l *= alpha;
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[i] *= alpha;
#pragma unroll
        for (int u = 0; u < KB; ++u) {
            const float p = exp2f(s[u] - mn);   // 0 for the keys past the split
            l += p;
#pragma unroll
            for (int i = 0; i < DPL; ++i) acc[i] = fmaf(p, vx[u][i], acc[i]);
        }
        m = mn;
    }
    if (lane == 0) {
        a.part_m[pi] = m;
        a.part_l[pi] = l;
    }
    float* pa = a.part_acc + pi * HD + lane * DPL;
#pragma unroll
    for (int i = 0; i < DPL; ++i) pa[i] = acc[i];
}

// blockIdx = (token, q head); thread d = one dim (blockDim = hd).
__global__ void __launch_bounds__(256) gdn_attn_combine_kernel(const AttnArgs a) {
    const int t = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
    const size_t p0 = ((size_t)t * a.nh + h) * a.n_split;
    float M = -INFINITY;
    for (int s = 0; s < a.n_split; ++s) M = fmaxf(M, a.part_m[p0 + s]);
    float L = 0.f, o = 0.f;
    for (int s = 0; s < a.n_split; ++s) {
        const float ms = a.part_m[p0 + s];
        if (ms == -INFINITY) continue;   // an empty split
        const float w = exp2f(ms - M);
        L = fmaf(w, a.part_l[p0 + s], L);
        o = fmaf(w, a.part_acc[(p0 + s) * a.hd + d], o);
    }
    const float attn = rbf(o / L);   // the SDPA output, bf16
    const float g = bf2f(a.q_full[(size_t)t * (2 * a.nh * a.hd) + (size_t)h * 2 * a.hd + a.hd + d]);
    const float sg = rbf(sigmoid_f32(g));   // nn::sigmoid on the bf16 gate
    a.out[((size_t)t * a.nh + h) * a.hd + d] = f2bf(attn * sg);
}

int attn_check(const gdn_attn_config* c) {
    char msg[256];
    if (!c) return record_error(GDN_E_INVALID, "attention config is NULL");
    if (c->n_heads <= 0 || c->n_kv_heads <= 0 || c->n_heads % c->n_kv_heads != 0) {
        snprintf(msg, sizeof msg, "n_heads (%d) must be a positive multiple of n_kv_heads (%d)", c->n_heads,
                 c->n_kv_heads);
        return record_error(GDN_E_INVALID, msg);
    }
    if (c->n_heads / c->n_kv_heads > 16) return record_error(GDN_E_UNSUPPORTED, "GQA groups above 16 q heads");
    if (c->head_dim != 64 && c->head_dim != 128 && c->head_dim != 256) {
        snprintf(msg, sizeof msg, "head_dim %d: only 64, 128 and 256 are specialised", c->head_dim);
        return record_error(GDN_E_UNSUPPORTED, msg);
    }
    if (c->rotary_dim < 0 || c->rotary_dim > c->head_dim || (c->rotary_dim & 1))
        return record_error(GDN_E_INVALID, "rotary_dim must be even and within [0, head_dim]");
    if (c->max_ctx <= 0) return record_error(GDN_E_INVALID, "max_ctx must be positive");
    if (!(c->rms_norm_eps >= 0.f) || !(c->rope_theta > 0.f))
        return record_error(GDN_E_INVALID, "rms_norm_eps must be >= 0 and rope_theta > 0");
    return GDN_OK;
}

}  // namespace
}  // namespace gdn

using namespace gdn;

extern "C" {

int gdn_attn_workspace_bytes(const gdn_attn_config* cfg, int32_t n_tokens, int32_t max_kv_len, int64_t* bytes) {
    int rc = attn_check(cfg);
    if (rc) return rc;
    if (!bytes || n_tokens < 0 || max_kv_len < 0) return record_error(GDN_E_INVALID, "bad workspace query");
    const int ns = attn_splits(n_tokens, cfg->n_kv_heads, max_kv_len);
    *bytes = (int64_t)attn_layout(n_tokens, cfg->n_heads, cfg->head_dim, ns).total;
    return record_ok();
}

int gdn_attn_step(const gdn_attn_config* cfg, const gdn_bf16* q_full, const gdn_bf16* k_in, const gdn_bf16* v_in,
                  const gdn_bf16* q_norm_w, const gdn_bf16* k_norm_w, gdn_bf16* k_cache, gdn_bf16* v_cache,
                  int32_t n_slots, const int32_t* slot_ids, const int32_t* cu_seqlens, const int32_t* positions,
                  int32_t n_seq, int32_t n_tokens, gdn_bf16* out, void* workspace, int64_t workspace_bytes,
                  void* stream) {
    int rc = attn_check(cfg);
    if (rc) return rc;
    char msg[256];
    if (n_seq < 0 || n_tokens < 0) return record_error(GDN_E_INVALID, "n_seq and n_tokens must be >= 0");
    if (n_tokens == 0) return record_ok();
    if (!q_full || !k_in || !v_in || !q_norm_w || !k_norm_w || !k_cache || !v_cache || !out || !workspace ||
        !slot_ids || !cu_seqlens || !positions)
        return record_error(GDN_E_INVALID, "a required pointer is NULL");
    if (n_slots <= 0) return record_error(GDN_E_INVALID, "n_slots must be positive");
    // host tables -> per-token (slot, position), with the checks of gdn_validate_tables plus the cache bound
    if (cu_seqlens[0] != 0 || cu_seqlens[n_seq] != n_tokens) {
        snprintf(msg, sizeof msg, "cu_seqlens must run from 0 to n_tokens (%d)", n_tokens);
        return record_error(GDN_E_BAD_SEQLENS, msg);
    }
    std::vector<int32_t> tab(2 * (size_t)n_tokens);
    std::vector<char> used(n_slots, 0);
    int max_kv = 0;
    for (int i = 0; i < n_seq; ++i) {
        const int s = slot_ids[i], b = cu_seqlens[i], e = cu_seqlens[i + 1];
        if (s < 0 || s >= n_slots || used[s]) {
            snprintf(msg, sizeof msg, "slot %d of sequence %d out of range [0,%d) or repeated", s, i, n_slots);
            return record_error(GDN_E_BAD_SLOT, msg);
        }
        used[s] = 1;
        if (e < b || e > n_tokens) return record_error(GDN_E_BAD_SEQLENS, "cu_seqlens decreasing or past n_tokens");
        if (positions[i] < 0 || (long long)positions[i] + (e - b) > cfg->max_ctx) {
            snprintf(msg, sizeof msg, "sequence %d: position %d + %d tokens exceeds the cache's %d", i, positions[i],
                     e - b, cfg->max_ctx);
            return record_error(GDN_E_INVALID, msg);
        }
        for (int j = b; j < e; ++j) {
            tab[j] = s;
            tab[n_tokens + j] = positions[i] + (j - b);
        }
        if (e > b && positions[i] + (e - b) > max_kv) max_kv = positions[i] + (e - b);
    }
    const int nh = cfg->n_heads, nkv = cfg->n_kv_heads, hd = cfg->head_dim;
    const int ns = attn_splits(n_tokens, nkv, max_kv);
    const AttnLayout L = attn_layout(n_tokens, nh, hd, ns);
    if (workspace_bytes < (int64_t)L.total) {
        snprintf(msg, sizeof msg, "workspace of %lld B is below the %zu B this call needs",
                 (long long)workspace_bytes, L.total);
        return record_error(GDN_E_INVALID, msg);
    }
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e =
        cudaMemcpyAsync(ws + L.tok_slot, tab.data(), 2 * sizeof(int32_t) * n_tokens, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) {
        snprintf(msg, sizeof msg, "routing table upload: %s", cudaGetErrorString(e));
        return record_error(GDN_E_CUDA, msg);
    }
    AttnArgs a{};
    a.q_full = q_full; a.k_in = k_in; a.v_in = v_in; a.qn_w = q_norm_w; a.kn_w = k_norm_w;
    a.k_cache = k_cache; a.v_cache = v_cache;
    a.tok_slot = reinterpret_cast<const int32_t*>(ws + L.tok_slot);
    a.tok_pos = reinterpret_cast<const int32_t*>(ws + L.tok_pos);
    a.qbuf = reinterpret_cast<uint16_t*>(ws + L.qbuf);
    a.part_m = reinterpret_cast<float*>(ws + L.part_m);
    a.part_l = reinterpret_cast<float*>(ws + L.part_l);
    a.part_acc = reinterpret_cast<float*>(ws + L.part_acc);
    a.out = out;
    a.n_tokens = n_tokens; a.nh = nh; a.nkv = nkv; a.hd = hd; a.rot = cfg->rotary_dim; a.max_ctx = cfg->max_ctx;
    a.n_split = ns;
    a.split_keys = (max_kv + ns - 1) / ns;
    a.eps = cfg->rms_norm_eps;
    a.log2_theta = (float)std::log2((double)cfg->rope_theta);
    a.scale_log2 = (1.0f / std::sqrt((float)hd)) * LOG2E;   // (hd as f32).sqrt().recip(), qwen3_5.rs:351

    gdn_attn_prep_kernel<<<dim3(n_tokens, nh + 2 * nkv), AP_THREADS, 0, st>>>(a);
    const dim3 grid(n_tokens, nkv, ns);
    const int threads = 32 * (nh / nkv);
    if (hd == 256) gdn_attn_split_kernel<256><<<grid, threads, 0, st>>>(a);
    else if (hd == 128) gdn_attn_split_kernel<128><<<grid, threads, 0, st>>>(a);
    else gdn_attn_split_kernel<64><<<grid, threads, 0, st>>>(a);
    gdn_attn_combine_kernel<<<dim3(n_tokens, nh), hd, 0, st>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess) {
        snprintf(msg, sizeof msg, "attention launch: %s", cudaGetErrorString(e));
        return record_error(GDN_E_CUDA, msg);
    }
    return record_ok();
}

}  // extern "C"
