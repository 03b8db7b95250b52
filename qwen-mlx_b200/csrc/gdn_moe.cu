// gdn_moe.cu -- the sparse MoE block of the hybrid decoder (SparseMoeBlock::forward,
// src/models/qwen3_5.rs:262-302) over a batch of tokens, with the checkpoint's MLX 4-bit experts.
//
// Expert-major, so that every expert weight row that any token needs is streamed from HBM once per
// call, however many tokens picked that expert (the reference's gather_qmm, qwen3_5.rs:142-152, is
// indexed per (token, expert) pair):
//   gdn_moe_route_kernel    one CTA per token: router logits (bf16), softmax, top-k by block argmax,
//                           renormalisation (qwen3_5.rs:268-284), and the shared-expert gate logit;
//   gdn_moe_bucket_kernel   one CTA: counting sort of the (token, k) pairs by expert, the shared expert
//                           taken as expert E with one pair per token, and the list of experts with pairs
//                           (the next two grids cover only those);
//   gdn_moe_up_kernel       CTA per (expert, 16 rows of gate|up, 32 of its pairs): 4-bit dequant of
//                           both rows in registers, dots with up to 8 staged token rows at a time,
//                           h = silu(gate x) * up x (compiled_ops.rs:99-143);
//   gdn_moe_down_kernel     CTA per (expert, 64 rows of down, 32 of its pairs): y = down h;
//   gdn_moe_combine_kernel  one CTA per token: sum_j w_j y_j + sigmoid(gate logit) * y_shared.
// All of it is weight-streaming integer/float work on the CUDA cores: at decode batch sizes a token
// group shares each dequantised row across its up-to-8 tokens, and the rows are read once.
#include <cuda_runtime.h>

#include <cstdio>

#include "gdn.h"
#include "gdn_device.cuh"
#include "gdn_hybrid.h"
#include "gdn_internal.h"

namespace gdn {
namespace {

constexpr int MR_THREADS = 1024;  // route: 32 warps share the router's rows
constexpr int MX_THREADS = 256;   // up / down: 8 warps x 2 rows
constexpr int MX_ROWS = 16;       // gate|up rows per CTA (many CTAs per expert: at decode an expert has few tokens)
constexpr int MD_ROWS = 64;       // down rows per CTA (a down row is short: moe_inter columns)
constexpr int MX_TG = 8;          // token rows staged together
constexpr int MX_TC = 32;         // pairs per CTA
constexpr int MAX_HIDDEN = 4096;
constexpr int MAX_INTER = 4096;
constexpr int MAX_EXPERTS = 1024;
constexpr int MAX_TOPK = 16;

struct MoeArgs {
    int N, H, E, K, I, Is, norm, do_route;
    const uint16_t* x;
    const uint16_t* router;
    gdn_q4_matrix gate, up, down, sh_gate, sh_up, sh_down;
    const uint16_t* shared_gate;
    uint16_t* logits;        // [N][E] or null
    int32_t* ids;            // [N][K]
    uint16_t* w;             // [N][K]
    float* sg;               // [N] shared-expert gate logit (bf16 value); null: not computed
    int32_t* off;            // [E + 2] pair offsets by expert (E = shared)
    int32_t* act;            // [E + 2]: act[0] = experts with pairs, act[1 ..] = their ids (ascending)
    int32_t* list;           // [P] pairs sorted by expert
    uint16_t* h;             // [P][Imax]
    uint16_t* y;             // [P][H]
    uint16_t* out;           // [N][H]
    int Imax;
};

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct MoeLayout {
    size_t ids, w, sg, off, act, list, h, y, total;
};

MoeLayout moe_layout(const gdn_moe_config* c, int N) {
    MoeLayout L{};
    const size_t P = (size_t)N * (c->top_k + 1);
    const int Imax = c->moe_inter > c->shared_inter ? c->moe_inter : c->shared_inter;
    size_t o = 0;
    L.ids = o;  o = align256(o + sizeof(int32_t) * (size_t)N * c->top_k);
    L.w = o;    o = align256(o + sizeof(uint16_t) * (size_t)N * c->top_k);
    L.sg = o;   o = align256(o + sizeof(float) * (size_t)N);
    L.off = o;  o = align256(o + sizeof(int32_t) * (size_t)(c->n_experts + 2));
    L.act = o;  o = align256(o + sizeof(int32_t) * (size_t)(c->n_experts + 2));
    L.list = o; o = align256(o + sizeof(int32_t) * P);
    L.h = o;    o = align256(o + sizeof(uint16_t) * P * Imax);
    L.y = o;    o = align256(o + sizeof(uint16_t) * P * c->hidden);
    L.total = o;
    return L;
}

// Dot of x (f32 in shared memory) with a bf16 row, over a warp: lane covers columns [8 lane + 256 i, +8).
__device__ __forceinline__ float warp_dot_bf16(const float* xs, const uint16_t* row, int H, int lane) {
    float acc = 0.f;
#pragma unroll 4
    for (int c = lane * 8; c < H; c += 256) {
        const uint4 v = *reinterpret_cast<const uint4*>(row + c);
        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            acc = fmaf(xs[c + 2 * i], __uint_as_float(wv[i] << 16), acc);
            acc = fmaf(xs[c + 2 * i + 1], __uint_as_float(wv[i] & 0xFFFF0000u), acc);
        }
    }
    return warp_sum(acc);
}

// blockIdx.x = token.  Dynamic shared memory: x as f32 [H], then probabilities [E].
__global__ void __launch_bounds__(MR_THREADS) gdn_moe_route_kernel(const MoeArgs a) {
    extern __shared__ float msm[];
    float* xs = msm;
    float* pr = msm + a.H;
    __shared__ float rv[MR_THREADS / 32];
    __shared__ int ri[MR_THREADS / 32];
    __shared__ float s_w[MAX_TOPK];
    __shared__ int s_id[MAX_TOPK];
    const int t = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    constexpr int NWARP = MR_THREADS / 32;
    for (int c = tid; c < a.H; c += MR_THREADS) xs[c] = bf2f(a.x[(size_t)t * a.H + c]);
    __syncthreads();
    // shared_expert_gate: Linear(hidden, 1), bf16 output (qwen3_5.rs:296)
    if (a.sg && warp == NWARP - 1) {
        const float d = warp_dot_bf16(xs, a.shared_gate, a.H, lane);
        if (lane == 0) a.sg[t] = rbf(d);
    }
    if (!a.do_route) return;
    for (int e = warp; e < a.E; e += NWARP) {
        const float d = rbf(warp_dot_bf16(xs, a.router + (size_t)e * a.H, a.H, lane));
        if (lane == 0) {
            pr[e] = d;
            if (a.logits) a.logits[(size_t)t * a.E + e] = f2bf(d);
        }
    }
    __syncthreads();
    // softmax over the bf16 logits in f32, each probability rounded once to bf16 (qwen3_5.rs:269)
    float mx = -INFINITY;
    for (int e = tid; e < a.E; e += MR_THREADS) mx = fmaxf(mx, pr[e]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) rv[warp] = mx;
    __syncthreads();
    mx = rv[0];
#pragma unroll
    for (int i = 1; i < NWARP; ++i) mx = fmaxf(mx, rv[i]);
    __syncthreads();
    float sum = 0.f;
    for (int e = tid; e < a.E; e += MR_THREADS) sum += expf(pr[e] - mx);
    sum = warp_sum(sum);
    if (lane == 0) rv[warp] = sum;
    __syncthreads();
    sum = 0.f;
#pragma unroll
    for (int i = 0; i < NWARP; ++i) sum += rv[i];
    for (int e = tid; e < a.E; e += MR_THREADS) pr[e] = rbf(expf(pr[e] - mx) / sum);
    __syncthreads();
    // top-k: k rounds of block argmax (larger p first, lower expert index among equal p)
    for (int j = 0; j < a.K; ++j) {
        float bv = -1.f;
        int bi = 0x7fffffff;
        for (int e = tid; e < a.E; e += MR_THREADS) {
            const float v = pr[e];
            if (v > bv || (v == bv && e < bi)) { bv = v; bi = e; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) { rv[warp] = bv; ri[warp] = bi; }
        __syncthreads();
        if (tid == 0) {
            for (int i = 1; i < NWARP; ++i)
                if (rv[i] > bv || (rv[i] == bv && ri[i] < bi)) { bv = rv[i]; bi = ri[i]; }
            s_w[j] = bv;
            s_id[j] = bi;
            pr[bi] = -2.f;   // below every probability: not picked again
        }
        __syncthreads();
    }
    if (tid == 0) {
        float den = 1.f;
        if (a.norm) {   // topk_weights / topk_weights.sum(-1) in bf16 (qwen3_5.rs:279-282)
            float s = 0.f;
            for (int j = 0; j < a.K; ++j) s += s_w[j];
            den = rbf(s);
        }
        for (int j = 0; j < a.K; ++j) {
            a.ids[(size_t)t * a.K + j] = s_id[j];
            a.w[(size_t)t * a.K + j] = f2bf(a.norm ? s_w[j] / den : s_w[j]);
        }
    }
}

// Expert of pair p: ids[p] for the routed pairs p < N K, the shared expert E for p = N K + token.
__device__ __forceinline__ int pair_expert(const MoeArgs& a, int p) {
    if (p >= a.N * a.K) return a.E;
    const int e = a.ids[p];
    return (e >= 0 && e < a.E) ? e : -1;   // an id out of range joins no expert; the combine skips it
}
__device__ __forceinline__ int pair_token(const MoeArgs& a, int p) {
    return p < a.N * a.K ? p / a.K : p - a.N * a.K;
}

__global__ void __launch_bounds__(1024) gdn_moe_bucket_kernel(const MoeArgs a) {
    __shared__ int cnt[MAX_EXPERTS + 2];
    const int tid = threadIdx.x;
    const int P = a.N * (a.K + 1);
    for (int e = tid; e <= a.E + 1; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int p = tid; p < P; p += blockDim.x) {
        const int e = pair_expert(a, p);
        if (e >= 0) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    if (tid == 0) {
        int run = 0, n_act = 0;
        for (int e = 0; e <= a.E; ++e) {
            const int c = cnt[e];
            cnt[e] = run;   // becomes the expert's cursor
            a.off[e] = run;
            run += c;
            if (c > 0) a.act[1 + n_act++] = e;
        }
        a.off[a.E + 1] = run;
        a.act[0] = n_act;
    }
    __syncthreads();
    for (int p = tid; p < P; p += blockDim.x) {
        const int e = pair_expert(a, p);
        if (e >= 0) a.list[atomicAdd(&cnt[e], 1)] = p;
    }
}

// One weight row of a 4-bit matrix: words [lane + 32 i] hold columns [8 w, +8), group w / 8 (64 columns).
// Dequantised values are rounded once to bf16, as MLX's quantized matmul writes its weight tile.
__device__ __forceinline__ void dequant8(uint32_t q, float s, float b, float (&wv)[8]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) wv[i] = rbf(fmaf(s, (float)((q >> (4 * i)) & 0xFu), b));
}

// Stage the input rows (x of the tokens, or h of the pairs) of pairs [g0, g0 + ng) into shared memory.
__device__ __forceinline__ void stage_rows(uint16_t* dst, const uint16_t* src, size_t ld_src, int cols, bool by_token,
                                           const MoeArgs& a, int g0, int ng) {
    const int v_per_row = cols / 8;
    for (int i = threadIdx.x; i < ng * v_per_row; i += blockDim.x) {
        const int r = i / v_per_row, c = i - r * v_per_row;
        const int p = a.list[g0 + r];
        const size_t row = by_token ? (size_t)pair_token(a, p) : (size_t)p;
        reinterpret_cast<uint4*>(dst + (size_t)r * cols)[c] = reinterpret_cast<const uint4*>(src + row * ld_src)[c];
    }
}

// blockIdx = (active expert, 16-row block of gate/up, 32-pair block of the expert's pairs).
__global__ void __launch_bounds__(MX_THREADS) gdn_moe_up_kernel(const MoeArgs a) {
    extern __shared__ __align__(16) uint16_t xs_up[];   // [MX_TG][H]
    if ((int)blockIdx.x >= a.act[0]) return;
    const int e = a.act[1 + blockIdx.x];
    const bool sh = e == a.E;
    const int I = sh ? a.Is : a.I;
    const int r0 = blockIdx.y * MX_ROWS;
    if (r0 >= I) return;
    const int beg = a.off[e] + blockIdx.z * MX_TC;
    const int end = min(a.off[e + 1], beg + MX_TC);
    if (beg >= end) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int H = a.H, wpr = H / 8, gpr = H / 64;
    const gdn_q4_matrix& G = sh ? a.sh_gate : a.gate;
    const gdn_q4_matrix& U = sh ? a.sh_up : a.up;
    const size_t erow = sh ? 0 : (size_t)e * a.I;   // first row of this expert in the stacked matrices
    for (int g0 = beg; g0 < end; g0 += MX_TG) {
        const int ng = min(MX_TG, end - g0);
        __syncthreads();
        stage_rows(xs_up, a.x, (size_t)H, H, true, a, g0, ng);
        __syncthreads();
        for (int rr = 0; rr < MX_ROWS / 8; ++rr) {
            const int r = r0 + warp * (MX_ROWS / 8) + rr;
            if (r >= I) break;
            const size_t row = erow + r;
            float ag[MX_TG], au[MX_TG];
#pragma unroll
            for (int k = 0; k < MX_TG; ++k) { ag[k] = 0.f; au[k] = 0.f; }
#pragma unroll 4
            for (int w = lane; w < wpr; w += 32) {
                const int grp = w >> 3;
                float wg[8], wu[8];
                dequant8(G.q[row * wpr + w], bf2f(G.scales[row * gpr + grp]), bf2f(G.biases[row * gpr + grp]), wg);
                dequant8(U.q[row * wpr + w], bf2f(U.scales[row * gpr + grp]), bf2f(U.biases[row * gpr + grp]), wu);
#pragma unroll
                for (int k = 0; k < MX_TG; ++k) {
                    if (k < ng) {
                        const uint4 v = reinterpret_cast<const uint4*>(xs_up + (size_t)k * H)[w];
                        const uint32_t xv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float x0 = __uint_as_float(xv[i] << 16), x1 = __uint_as_float(xv[i] & 0xFFFF0000u);
                            ag[k] = fmaf(wg[2 * i], x0, ag[k]);
                            ag[k] = fmaf(wg[2 * i + 1], x1, ag[k]);
                            au[k] = fmaf(wu[2 * i], x0, au[k]);
                            au[k] = fmaf(wu[2 * i + 1], x1, au[k]);
                        }
                    }
                }
            }
#pragma unroll
            for (int k = 0; k < MX_TG; ++k) {
                ag[k] = warp_sum(ag[k]);
                au[k] = warp_sum(au[k]);
                if (lane == k && k < ng) {
                    // gate and up outputs are bf16 (gather_qmm); silu(g) * u as two bf16 ops
                    const float hv = rbf(silu_bf(rbf(ag[k])) * rbf(au[k]));
                    a.h[(size_t)a.list[g0 + k] * a.Imax + r] = f2bf(hv);
                }
            }
        }
    }
}

// blockIdx = (active expert, 64-row block of down, 32-pair block of the expert's pairs).
__global__ void __launch_bounds__(MX_THREADS) gdn_moe_down_kernel(const MoeArgs a) {
    extern __shared__ __align__(16) uint16_t hs_dn[];   // [MX_TG][I]
    if ((int)blockIdx.x >= a.act[0]) return;
    const int e = a.act[1 + blockIdx.x];
    const bool sh = e == a.E;
    const int I = sh ? a.Is : a.I;
    const int r0 = blockIdx.y * MD_ROWS;
    const int beg = a.off[e] + blockIdx.z * MX_TC;
    const int end = min(a.off[e + 1], beg + MX_TC);
    if (beg >= end || r0 >= a.H) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wpr = I / 8, gpr = I / 64;
    const gdn_q4_matrix& D = sh ? a.sh_down : a.down;
    const size_t erow = sh ? 0 : (size_t)e * a.H;
    for (int g0 = beg; g0 < end; g0 += MX_TG) {
        const int ng = min(MX_TG, end - g0);
        __syncthreads();
        stage_rows(hs_dn, a.h, (size_t)a.Imax, I, false, a, g0, ng);
        __syncthreads();
        for (int rr = 0; rr < MD_ROWS / 8; ++rr) {
            const int r = r0 + warp * (MD_ROWS / 8) + rr;
            if (r >= a.H) break;
            const size_t row = erow + r;
            float ac[MX_TG];
#pragma unroll
            for (int k = 0; k < MX_TG; ++k) ac[k] = 0.f;
#pragma unroll 2
            for (int w = lane; w < wpr; w += 32) {
                const int grp = w >> 3;
                float wd[8];
                dequant8(D.q[row * wpr + w], bf2f(D.scales[row * gpr + grp]), bf2f(D.biases[row * gpr + grp]), wd);
#pragma unroll
                for (int k = 0; k < MX_TG; ++k) {
                    if (k < ng) {
                        const uint4 v = reinterpret_cast<const uint4*>(hs_dn + (size_t)k * I)[w];
                        const uint32_t hv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            ac[k] = fmaf(wd[2 * i], __uint_as_float(hv[i] << 16), ac[k]);
                            ac[k] = fmaf(wd[2 * i + 1], __uint_as_float(hv[i] & 0xFFFF0000u), ac[k]);
                        }
                    }
                }
            }
#pragma unroll
            for (int k = 0; k < MX_TG; ++k) {
                ac[k] = warp_sum(ac[k]);
                if (lane == k && k < ng) a.y[(size_t)a.list[g0 + k] * a.H + r] = f2bf(ac[k]);
            }
        }
    }
}

// blockIdx.x = token.  out = bf16(bf16(sum_j bf16(y_j w_j)) + bf16(bf16(sigmoid(sg)) y_shared))
// (qwen3_5.rs:287-300: the weighted experts summed over k, the gated shared expert added).
__global__ void __launch_bounds__(256) gdn_moe_combine_kernel(const MoeArgs a) {
    const int t = blockIdx.x;
    const float sig = rbf(sigmoid_f32(a.sg[t]));
    const size_t ps = (size_t)a.N * a.K + t;
    for (int d = threadIdx.x; d < a.H; d += blockDim.x) {
        float acc = 0.f;
        for (int j = 0; j < a.K; ++j) {
            const size_t p = (size_t)t * a.K + j;
            const int e = a.ids[p];
            if (e < 0 || e >= a.E) continue;
            acc += rbf(bf2f(a.y[p * a.H + d]) * bf2f(a.w[p]));
        }
        const float shg = rbf(sig * bf2f(a.y[ps * a.H + d]));
        a.out[(size_t)t * a.H + d] = f2bf(rbf(acc) + shg);
    }
}

int moe_check(const gdn_moe_config* c) {
    if (!c) return record_error(GDN_E_INVALID, "MoE config is NULL");
    if (c->hidden <= 0 || c->hidden % 64 || c->hidden > MAX_HIDDEN)
        return record_error(GDN_E_UNSUPPORTED, "hidden must be a positive multiple of 64, at most 4096");
    if (c->n_experts <= 0 || c->n_experts > MAX_EXPERTS)
        return record_error(GDN_E_UNSUPPORTED, "n_experts must be in [1, 1024]");
    if (c->top_k <= 0 || c->top_k > MAX_TOPK || c->top_k > c->n_experts)
        return record_error(GDN_E_UNSUPPORTED, "top_k must be in [1, min(16, n_experts)]");
    if (c->moe_inter <= 0 || c->moe_inter % 64 || c->moe_inter > MAX_INTER || c->shared_inter <= 0 ||
        c->shared_inter % 64 || c->shared_inter > MAX_INTER)
        return record_error(GDN_E_UNSUPPORTED, "moe_inter and shared_inter must be positive multiples of 64, <= 4096");
    return GDN_OK;
}

bool q4_ok(const gdn_q4_matrix& m) { return m.q && m.scales && m.biases; }

MoeArgs moe_args(const gdn_moe_config* c, const gdn_moe_weights* w, const gdn_bf16* x, int N) {
    MoeArgs a{};
    a.N = N; a.H = c->hidden; a.E = c->n_experts; a.K = c->top_k; a.I = c->moe_inter; a.Is = c->shared_inter;
    a.Imax = a.I > a.Is ? a.I : a.Is;
    a.norm = c->norm_topk_prob != 0;
    a.x = x;
    a.router = w->router;
    a.gate = w->gate; a.up = w->up; a.down = w->down;
    a.sh_gate = w->sh_gate; a.sh_up = w->sh_up; a.sh_down = w->sh_down;
    a.shared_gate = w->shared_gate;
    return a;
}

cudaError_t launch_route(const MoeArgs& a, cudaStream_t st) {
    const size_t smem = sizeof(float) * (size_t)(a.H + a.E);
    cudaError_t e = cudaFuncSetAttribute(gdn_moe_route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    gdn_moe_route_kernel<<<a.N, MR_THREADS, smem, st>>>(a);
    return cudaGetLastError();
}

}  // namespace
}  // namespace gdn

using namespace gdn;

extern "C" {

int gdn_moe_workspace_bytes(const gdn_moe_config* cfg, int32_t n_tokens, int64_t* bytes) {
    int rc = moe_check(cfg);
    if (rc) return rc;
    if (!bytes || n_tokens < 0) return record_error(GDN_E_INVALID, "bad workspace query");
    *bytes = (int64_t)moe_layout(cfg, n_tokens).total;
    return record_ok();
}

int gdn_moe_route(const gdn_moe_config* cfg, const gdn_moe_weights* w, const gdn_bf16* x, int32_t n_tokens,
                  gdn_bf16* logits, int32_t* ids, gdn_bf16* weights, void* stream) {
    int rc = moe_check(cfg);
    if (rc) return rc;
    if (n_tokens < 0) return record_error(GDN_E_INVALID, "n_tokens must be >= 0");
    if (n_tokens == 0) return record_ok();
    if (!w || !x || !ids || !weights || !w->router) return record_error(GDN_E_INVALID, "a required pointer is NULL");
    MoeArgs a = moe_args(cfg, w, x, n_tokens);
    a.do_route = 1;
    a.logits = logits; a.ids = ids; a.w = weights;   // a.sg stays NULL: no shared-expert gate here
    const cudaError_t e = launch_route(a, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) {
        char msg[256];
        snprintf(msg, sizeof msg, "MoE route launch: %s", cudaGetErrorString(e));
        return record_error(GDN_E_CUDA, msg);
    }
    return record_ok();
}

int gdn_moe_step(const gdn_moe_config* cfg, const gdn_moe_weights* w, const gdn_bf16* x, int32_t n_tokens,
                 const int32_t* route_ids, const gdn_bf16* route_weights, gdn_bf16* out, void* workspace,
                 int64_t workspace_bytes, void* stream) {
    int rc = moe_check(cfg);
    if (rc) return rc;
    char msg[256];
    if (n_tokens < 0) return record_error(GDN_E_INVALID, "n_tokens must be >= 0");
    if (n_tokens == 0) return record_ok();
    if (!w || !x || !out || !workspace || !w->shared_gate || !q4_ok(w->gate) || !q4_ok(w->up) || !q4_ok(w->down) ||
        !q4_ok(w->sh_gate) || !q4_ok(w->sh_up) || !q4_ok(w->sh_down))
        return record_error(GDN_E_INVALID, "a required pointer is NULL");
    if ((route_ids == nullptr) != (route_weights == nullptr))
        return record_error(GDN_E_INVALID, "route_ids and route_weights are given together or not at all");
    if (!route_ids && !w->router) return record_error(GDN_E_INVALID, "router weight is NULL and no routing given");
    const MoeLayout L = moe_layout(cfg, n_tokens);
    if (workspace_bytes < (int64_t)L.total) {
        snprintf(msg, sizeof msg, "workspace of %lld B is below the %zu B this call needs", (long long)workspace_bytes,
                 L.total);
        return record_error(GDN_E_INVALID, msg);
    }
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    MoeArgs a = moe_args(cfg, w, x, n_tokens);
    a.sg = reinterpret_cast<float*>(ws + L.sg);
    a.off = reinterpret_cast<int32_t*>(ws + L.off);
    a.act = reinterpret_cast<int32_t*>(ws + L.act);
    a.list = reinterpret_cast<int32_t*>(ws + L.list);
    a.h = reinterpret_cast<uint16_t*>(ws + L.h);
    a.y = reinterpret_cast<uint16_t*>(ws + L.y);
    a.out = out;
    if (route_ids) {
        a.ids = const_cast<int32_t*>(route_ids);
        a.w = const_cast<uint16_t*>(route_weights);
        a.do_route = 0;
    } else {
        a.ids = reinterpret_cast<int32_t*>(ws + L.ids);
        a.w = reinterpret_cast<uint16_t*>(ws + L.w);
        a.do_route = 1;
    }
    cudaError_t e = launch_route(a, st);   // routing (unless given) and the shared-expert gate logit
    if (e == cudaSuccess) {
        gdn_moe_bucket_kernel<<<1, 1024, 0, st>>>(a);
        // pairs of one expert: at most one per token from the router (its picks are distinct); a routing
        // given by the caller may repeat an expert within a token
        const int max_pairs = route_ids ? n_tokens * cfg->top_k : n_tokens;
        const int zb = (max_pairs + MX_TC - 1) / MX_TC;
        const size_t up_smem = sizeof(uint16_t) * MX_TG * (size_t)a.H;
        const size_t dn_smem = sizeof(uint16_t) * MX_TG * (size_t)a.Imax;
        e = cudaFuncSetAttribute(gdn_moe_up_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)up_smem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(gdn_moe_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dn_smem);
        if (e == cudaSuccess) {
            // experts with pairs: at most min(E, N K) routed ones plus the shared expert
            const long long routed = (long long)n_tokens * cfg->top_k;
            const int gx = (routed < a.E ? (int)routed : a.E) + 1;
            gdn_moe_up_kernel<<<dim3(gx, (a.Imax + MX_ROWS - 1) / MX_ROWS, zb), MX_THREADS, up_smem, st>>>(a);
            gdn_moe_down_kernel<<<dim3(gx, (a.H + MD_ROWS - 1) / MD_ROWS, zb), MX_THREADS, dn_smem, st>>>(a);
            gdn_moe_combine_kernel<<<n_tokens, 256, 0, st>>>(a);
            e = cudaGetLastError();
        }
    }
    if (e != cudaSuccess) {
        snprintf(msg, sizeof msg, "MoE launch: %s", cudaGetErrorString(e));
        return record_error(GDN_E_CUDA, msg);
    }
    return record_ok();
}

}  // extern "C"
