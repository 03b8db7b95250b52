/*
 * gdn_oracle.c -- CPU restatement of the reference GatedDeltaNet layer step.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker and the timed
 * CPU baseline ("port").  Only tests/, __graft_entry__.smoke() and bench.py
 * (its cpu_baseline leg and --impl reference) may load it.  The product
 * (qwen-mlx_b200/csrc) never links or calls it.
 *
 * Reference followed (paths inside emanueleDiVizio/qwen-mlx):
 *   src/models/qwen3_5.rs:559-669   GatedDeltaNet::forward_with_cache (layer order, dtypes)
 *   src/models/qwen3_5.rs:551-552   q/k RMSNorm gains bf16(1/dk), bf16(dk^-0.5)
 *   src/models/qwen3_5.rs:593-610   S=1 conv: bf16 products, bf16 sum, SiLU
 *   src/models/qwen3_5.rs:611-624   S>1 conv: conv1d groups=D, f32 accumulate
 *   src/models/qwen3_5.rs:1058-1066 conv weight [D,K,1] (used here as [D][K])
 *   src/models/compiled_ops.rs:12-49 beta = bf16(sigmoid(f32 b)); g = exp(-exp(A_log)*softplus(a+dt_bias))
 *   src/models/metal_gdn.rs:10-67   gated delta recurrence (state [b][hv][dv][dk] f32)
 *   src/models/metal_gdn.rs:14      GQA: hk = hv / (Hv/Hk)
 *   src/models/qwen3_5.rs:660-665   gated RMSNorm: silu(z) * rms_norm(y, w, eps)
 *   src/models/qwen3_5.rs:729-739   decoder pre-norm + residual (used to chain the stack)
 *
 * The arithmetic inside MLX ops (mlx-rs 0.25.3 / mlx-sys 0.2.0, not vendored)
 * is restated from MLX's published kernels, with these rounding points:
 *   - every MLX op computes in f32 and rounds once to its output dtype;
 *   - fast::rms_norm rounds twice: bf16(x * rsqrt(mean(x^2)+eps)), then bf16(w * that);
 *   - silu(x) = bf16(x * sigmoid(x)) computed in f32;
 *   - sums over the conv taps and GEMM dot products accumulate in f32.
 * The Metal kernel's simd_sum is a pairwise tree over the 32 lanes; each lane
 * first sums its own 4 consecutive dk terms in order (metal_gdn.rs:38-44).
 * Build with -ffp-contract=off so every multiply and add rounds separately.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_OK 0
#define ORC_EINVAL 1
#define ORC_ENOMEM 2

/* ------------------------------------------------------------ bf16 helpers */
static inline float bf(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}
static inline uint16_t tobf(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
static inline float rnd(float f) { return bf(tobf(f)); }

static inline float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }
/* nn::silu on a bf16 array (qwen3_5.rs:610, :623, :664): one rounding. */
static inline float silu_bf(float x) { return rnd(x * sigmoidf_(x)); }

typedef struct orc_cfg {
    int32_t hidden, hk, hv, dk, dv, conv_k;
    float eps;
} orc_cfg;

static inline int conv_dim(const orc_cfg* c) { return 2 * c->hk * c->dk + c->hv * c->dv; }

/* ------------------------------------------------------------ building blocks */

static inline float lane_tree_sum_fwd(float* p) {
    for (int off = 16; off > 0; off >>= 1)
        for (int l = 0; l < off; ++l) p[l] = p[l] + p[l + off];
    return p[0];
}

/* MLX fast::rms_norm over one row of n bf16 values; w == NULL means a constant gain. */
static void rms_norm_row(const uint16_t* x, const uint16_t* w, uint16_t w_const, int n, float eps,
                         uint16_t* out) {
    float acc = 0.0f;
    for (int i = 0; i < n; ++i) {
        float xi = bf(x[i]);
        acc += xi * xi;
    }
    float normalizer = 1.0f / sqrtf(acc / (float)n + eps);
    for (int i = 0; i < n; ++i) {
        float t = rnd(bf(x[i]) * normalizer);
        float wi = bf(w ? w[i] : w_const);
        out[i] = tobf(wi * t);
    }
}

void orc_rms_norm(const uint16_t* x, const uint16_t* w, int64_t rows, int32_t n, float eps, uint16_t* out) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) rms_norm_row(x + r * n, w, 0, n, eps, out + r * n);
}

/* Accumulation order of the f32 dot products in orc_linear.  The reference's GEMM
 * (MLX matmul / quantized_matmul, qwen3_5.rs:572-586, :668) accumulates in f32 in an
 * order the reference does not fix.  0: sequential over k (default).  1: 32
 * interleaved partial sums (k mod 32) combined by a pairwise tree -- a different,
 * equally valid order, used by the tests to measure how much the layer's output
 * depends on the order. */
static int g_linear_order = 0;
void orc_set_linear_order(int order) { g_linear_order = order; }

/* Linear without bias (nn::Linear / matmul): out[m][n] = bf16(sum_k x[m][k] w[n][k]) with f32 accumulation. */
void orc_linear(const uint16_t* x, const uint16_t* w, int64_t M, int32_t N, int32_t K, uint16_t* out) {
    float* wf = (float*)malloc(sizeof(float) * (size_t)N * K);
    float* xf = (float*)malloc(sizeof(float) * (size_t)M * K);
    if (!wf || !xf) { free(wf); free(xf); return; }
    const int order = g_linear_order;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)N * K; ++i) wf[i] = bf(w[i]);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < M * K; ++i) xf[i] = bf(x[i]);
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t m = 0; m < M; ++m)
        for (int32_t n = 0; n < N; ++n) {
            const float* xr = xf + m * K;
            const float* wr = wf + (int64_t)n * K;
            float acc = 0.0f;
            if (order == 1) {
                float part[32];
                for (int l = 0; l < 32; ++l) part[l] = 0.0f;
                for (int32_t k = 0; k < K; ++k) part[k & 31] += xr[k] * wr[k];
                acc = lane_tree_sum_fwd(part);
            } else if (order == 2) {
                for (int32_t k0 = 0; k0 < K; k0 += 16) {
                    float blk = 0.0f;
                    for (int32_t k = k0; k < k0 + 16 && k < K; ++k) blk += xr[k] * wr[k];
                    acc += blk;
                }
            } else if (order == 3) {
                for (int32_t k = K - 1; k >= 0; --k) acc += xr[k] * wr[k];
            } else {
                for (int32_t k = 0; k < K; ++k) acc += xr[k] * wr[k];
            }
            out[m * N + n] = tobf(acc);
        }
    free(wf);
    free(xf);
}

/* compiled_ops.rs:12-49.  ab row = [b (Hv) | a (Hv)] (merged order, qwen3_5.rs:583).
 * dt_bf16 != 0: the checkpoint stores dt_bias in bf16 (given here widened to f32).  MLX then computes
 * add(a_raw, dt_bias) and exp of it as bf16 ops (each rounded to bf16, :36-37); add(exp_sum, 1.0f)
 * promotes to f32 (:38-39).  With an f32 dt_bias the add promotes to f32 and everything after is f32. */
void orc_gates(const uint16_t* ab, int64_t ld_ab, int64_t n_tok, int32_t hv, const float* A_log,
               const float* dt_bias, int32_t dt_bf16, float* g, uint16_t* beta) {
    for (int64_t t = 0; t < n_tok; ++t)
        for (int32_t h = 0; h < hv; ++h) {
            float b = bf(ab[t * ld_ab + h]);
            float a = bf(ab[t * ld_ab + hv + h]);
            beta[t * hv + h] = tobf(sigmoidf_(b));
            float s = a + dt_bias[h];
            float es;
            if (dt_bf16) {
                s = rnd(s);
                es = rnd(expf(s));
            } else {
                es = expf(s);
            }
            float sp = logf(es + 1.0f);
            float e = expf(A_log[h]);
            g[t * hv + h] = expf(-(e * sp));
        }
}

/* Pairwise tree over 32 lane partials (the Metal simd_sum stand-in). */
static inline float lane_tree_sum(float* p) {
    for (int off = 16; off > 0; off >>= 1)
        for (int l = 0; l < off; ++l) p[l] = p[l] + p[l + off];
    return p[0];
}

/*
 * Gated delta recurrence for one (sequence, v-head): metal_gdn.rs:28-66.
 * st      [dv][dk] f32, updated in place
 * q,k     T tokens, stride ldqk elements between tokens, dk values each (bf16)
 * v       T tokens, stride ldv, dv values (bf16)
 * g,beta  T tokens, stride ldg (f32 / bf16)
 * y       T tokens, stride ldy, dv values (bf16)
 */
static void recur_head(float* st, int dk, int dv, int T, const uint16_t* q, const uint16_t* k, int64_t ldqk,
                       const uint16_t* v, int64_t ldv, const float* g, const uint16_t* beta, int64_t ldg,
                       uint16_t* y, int64_t ldy) {
    const int npt = dk / 32;
    float part[32];
    for (int t = 0; t < T; ++t) {
        const uint16_t* qt = q + t * ldqk;
        const uint16_t* kt = k + t * ldqk;
        float gt = g[t * ldg];
        float bt = bf(beta[t * ldg]);
        for (int r = 0; r < dv; ++r) {
            float* s = st + (int64_t)r * dk;
            for (int l = 0; l < 32; ++l) {
                float acc = 0.0f;
                for (int i = 0; i < npt; ++i) {
                    int idx = npt * l + i;
                    s[idx] = s[idx] * gt;
                    acc += s[idx] * bf(kt[idx]);
                }
                part[l] = acc;
            }
            float kv = lane_tree_sum(part);
            float delta = (bf(v[t * ldv + r]) - kv) * bt;
            for (int l = 0; l < 32; ++l) {
                float acc = 0.0f;
                for (int i = 0; i < npt; ++i) {
                    int idx = npt * l + i;
                    s[idx] = s[idx] + bf(kt[idx]) * delta;
                    acc += s[idx] * bf(qt[idx]);
                }
                part[l] = acc;
            }
            y[t * ldy + r] = tobf(lane_tree_sum(part));
        }
    }
}

/*
 * Reference-shaped recurrence (metal_gdn.rs:170-218): dense [B,T,...] inputs,
 * state [B,Hv,dv,dk] f32 updated in place (the reference returns it as a new array).
 */
int orc_recurrence(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* g, const uint16_t* beta,
                   float* state, int32_t T, int32_t B, int32_t hk, int32_t hv, int32_t dk, int32_t dv, uint16_t* y) {
    if (dk % 32 || hv % hk) return ORC_EINVAL;
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int32_t b = 0; b < B; ++b)
        for (int32_t h = 0; h < hv; ++h) {
            int32_t kh = h / (hv / hk);
            int64_t tok0 = (int64_t)b * T;
            recur_head(state + ((int64_t)b * hv + h) * dv * dk, dk, dv, T,
                       q + tok0 * hk * dk + (int64_t)kh * dk, k + tok0 * hk * dk + (int64_t)kh * dk, (int64_t)hk * dk,
                       v + tok0 * hv * dv + (int64_t)h * dv, (int64_t)hv * dv, g + tok0 * hv + h, beta + tok0 * hv + h,
                       hv, y + tok0 * hv * dv + (int64_t)h * dv, (int64_t)hv * dv);
        }
    return ORC_OK;
}

/*
 * Packed ragged recurrence over per-sequence dense states: sequence i owns
 * tokens [cu[i], cu[i+1]) and state[i].  Inputs are packed by token.
 */
int orc_recurrence_packed(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* g,
                          const uint16_t* beta, float* state, const int32_t* cu, int32_t n_seq, int32_t hk, int32_t hv,
                          int32_t dk, int32_t dv, uint16_t* y) {
    if (dk % 32 || hv % hk) return ORC_EINVAL;
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int32_t i = 0; i < n_seq; ++i)
        for (int32_t h = 0; h < hv; ++h) {
            int32_t kh = h / (hv / hk);
            int64_t tok0 = cu[i];
            int32_t T = cu[i + 1] - cu[i];
            recur_head(state + ((int64_t)i * hv + h) * dv * dk, dk, dv, T, q + tok0 * hk * dk + (int64_t)kh * dk,
                       k + tok0 * hk * dk + (int64_t)kh * dk, (int64_t)hk * dk, v + tok0 * hv * dv + (int64_t)h * dv,
                       (int64_t)hv * dv, g + tok0 * hv + h, beta + tok0 * hv + h, hv,
                       y + tok0 * hv * dv + (int64_t)h * dv, (int64_t)hv * dv);
        }
    return ORC_OK;
}

/*
 * Causal depthwise conv + SiLU for one sequence of T tokens (qwen3_5.rs:593-624).
 * xin   [T][ld_x] bf16 (first D columns are the qkv projection)
 * cs    [K-1][D] bf16 conv state, replaced by the last K-1 rows of [cs; x]
 * w     [D][K] bf16
 * out   [T][D] bf16 (post-SiLU)
 */
static void conv_seq(const orc_cfg* c, const uint16_t* xin, int64_t ld_x, int32_t T, uint16_t* cs, const uint16_t* w,
                     uint16_t* out) {
    const int D = conv_dim(c), K = c->conv_k;
    const int P = T + K - 1;
    uint16_t* pad = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)P * D);
    memcpy(pad, cs, sizeof(uint16_t) * (size_t)(K - 1) * D);
    for (int t = 0; t < T; ++t) memcpy(pad + (int64_t)(K - 1 + t) * D, xin + t * ld_x, sizeof(uint16_t) * D);
    for (int t = 0; t < T; ++t)
        for (int ch = 0; ch < D; ++ch) {
            float acc;
            if (T == 1) {
                /* padded.multiply(cw) -> bf16, sum_axis(1) -> bf16 (f32 accumulate) */
                acc = 0.0f;
                for (int j = 0; j < K; ++j) acc += rnd(bf(pad[(int64_t)(t + j) * D + ch]) * bf(w[(int64_t)ch * K + j]));
            } else {
                /* conv1d: f32 accumulate, one rounding */
                acc = 0.0f;
                for (int j = 0; j < K; ++j) acc += bf(pad[(int64_t)(t + j) * D + ch]) * bf(w[(int64_t)ch * K + j]);
            }
            out[(int64_t)t * D + ch] = tobf(silu_bf(rnd(acc)));
        }
    memcpy(cs, pad + (int64_t)T * D, sizeof(uint16_t) * (size_t)(K - 1) * D);
    free(pad);
}

/* Conv + SiLU alone over one sequence (KAT hook): state cs updated in place. */
int orc_conv(const orc_cfg* c, const uint16_t* x, int64_t ld_x, int32_t T, uint16_t* cs, const uint16_t* w,
             uint16_t* out) {
    if (T <= 0) return ORC_OK;
    conv_seq(c, x, ld_x, T, cs, w, out);
    return ORC_OK;
}

typedef struct orc_layer_w {
    const uint16_t* conv_w;  /* [D][K] */
    const float* A_log;      /* [Hv] */
    const float* dt_bias;    /* [Hv] */
    const uint16_t* norm_w;  /* [dv] */
    int32_t dt_bias_bf16;    /* dt_bias stored in bf16 by the checkpoint (see orc_gates) */
} orc_layer_w;

/*
 * One fused GDN layer step between the projections (qwen3_5.rs:588-665) over a
 * packed ragged batch.  Sequence i owns tokens [cu[i], cu[i+1]) and the dense
 * states conv_state[i] ([K-1][D] bf16) and rec_state[i] ([Hv][dv][dk] f32).
 *   qkv  [N][ld_qkv] bf16   z [N][ld_z] bf16   ab [N][ld_ab] bf16 (b | a)
 *   out  [N][Hv*dv] bf16    y (optional) [N][Hv*dv] bf16 recurrence output
 */
int orc_layer_step(const orc_cfg* c, const orc_layer_w* w, const uint16_t* qkv, int64_t ld_qkv, const uint16_t* z,
                   int64_t ld_z, const uint16_t* ab, int64_t ld_ab, uint16_t* conv_state, float* rec_state,
                   const int32_t* cu, int32_t n_seq, uint16_t* out, uint16_t* y_opt) {
    const int D = conv_dim(c), hk = c->hk, hv = c->hv, dk = c->dk, dv = c->dv, K = c->conv_k;
    if (dk % 32 || hv % hk || K < 2) return ORC_EINVAL;
    const int64_t N = cu[n_seq];
    uint16_t* conv_out = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(N > 0 ? N : 1) * D);
    uint16_t* qn = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(N > 0 ? N : 1) * hk * dk);
    uint16_t* kn = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(N > 0 ? N : 1) * hk * dk);
    uint16_t* vv = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(N > 0 ? N : 1) * hv * dv);
    uint16_t* y = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(N > 0 ? N : 1) * hv * dv);
    float* g = (float*)malloc(sizeof(float) * (size_t)(N > 0 ? N : 1) * hv);
    uint16_t* beta = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(N > 0 ? N : 1) * hv);
    if (!conv_out || !qn || !kn || !vv || !y || !g || !beta) {
        free(conv_out); free(qn); free(kn); free(vv); free(y); free(g); free(beta);
        return ORC_ENOMEM;
    }
    /* 1. conv + SiLU per sequence */
#pragma omp parallel for schedule(dynamic)
    for (int32_t i = 0; i < n_seq; ++i) {
        int32_t T = cu[i + 1] - cu[i];
        if (T <= 0) continue;
        conv_seq(c, qkv + (int64_t)cu[i] * ld_qkv, ld_qkv, T, conv_state + (int64_t)i * (K - 1) * D, w->conv_w,
                 conv_out + (int64_t)cu[i] * D);
    }
    /* 2. split + q/k RMSNorm with the scale baked into the gain (qwen3_5.rs:626-639) */
    const uint16_t qw = tobf(powf((float)dk, -1.0f));
    const uint16_t kw = tobf(powf((float)dk, -0.5f));
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < N; ++t) {
        const uint16_t* row = conv_out + t * D;
        for (int h = 0; h < hk; ++h) {
            rms_norm_row(row + h * dk, NULL, qw, dk, 1e-6f, qn + (t * hk + h) * dk);
            rms_norm_row(row + hk * dk + h * dk, NULL, kw, dk, 1e-6f, kn + (t * hk + h) * dk);
        }
        memcpy(vv + t * hv * dv, row + 2 * hk * dk, sizeof(uint16_t) * hv * dv);
    }
    /* 3. gates */
    orc_gates(ab, ld_ab, N, hv, w->A_log, w->dt_bias, w->dt_bias_bf16, g, beta);
    /* 4. recurrence */
    orc_recurrence_packed(qn, kn, vv, g, beta, rec_state, cu, n_seq, hk, hv, dk, dv, y);
    /* 5. gated RMSNorm: silu(z) * rms_norm(y, norm_w, eps) */
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < N; ++t) {
        uint16_t yn[512];
        for (int h = 0; h < hv; ++h) {
            rms_norm_row(y + (t * hv + h) * dv, w->norm_w, 0, dv, c->eps, yn);
            for (int r = 0; r < dv; ++r) {
                float zs = silu_bf(bf(z[t * ld_z + h * dv + r]));
                out[t * hv * dv + h * dv + r] = tobf(zs * bf(yn[r]));
            }
        }
    }
    if (y_opt) memcpy(y_opt, y, sizeof(uint16_t) * (size_t)N * hv * dv);
    free(conv_out); free(qn); free(kn); free(vv); free(y); free(g); free(beta);
    return ORC_OK;
}

typedef struct orc_mixer_w {
    orc_layer_w core;
    const uint16_t* w_qkv;  /* [D][H] */
    const uint16_t* w_z;    /* [Hv*dv][H] */
    const uint16_t* w_b;    /* [Hv][H] */
    const uint16_t* w_a;    /* [Hv][H] */
    const uint16_t* w_out;  /* [H][Hv*dv] */
    const uint16_t* pre_w;  /* [H] decoder input RMSNorm gain */
} orc_mixer_w;

/*
 * Whole mixer (qwen3_5.rs:559-669): x [N][H] -> mixer output [N][H], with the
 * unmerged bf16 projections (in_proj_qkv, in_proj_z, in_proj_a, in_proj_b).
 */
int orc_mixer_step(const orc_cfg* c, const orc_mixer_w* w, const uint16_t* x, uint16_t* conv_state, float* rec_state,
                   const int32_t* cu, int32_t n_seq, uint16_t* mix_out) {
    const int D = conv_dim(c), hv = c->hv, dv = c->dv, H = c->hidden;
    const int64_t N = cu[n_seq];
    const int64_t ldp = (int64_t)D + hv * dv + 2 * hv;
    uint16_t* proj = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(N > 0 ? N : 1) * ldp);
    uint16_t* tmp = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(N > 0 ? N : 1) * (D > hv * dv ? D : hv * dv));
    uint16_t* gated = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(N > 0 ? N : 1) * hv * dv);
    if (!proj || !tmp || !gated) { free(proj); free(tmp); free(gated); return ORC_ENOMEM; }
    /* qkv */
    orc_linear(x, w->w_qkv, N, D, H, tmp);
    for (int64_t t = 0; t < N; ++t) memcpy(proj + t * ldp, tmp + t * D, sizeof(uint16_t) * D);
    orc_linear(x, w->w_z, N, hv * dv, H, tmp);
    for (int64_t t = 0; t < N; ++t) memcpy(proj + t * ldp + D, tmp + t * hv * dv, sizeof(uint16_t) * hv * dv);
    orc_linear(x, w->w_b, N, hv, H, tmp);
    for (int64_t t = 0; t < N; ++t) memcpy(proj + t * ldp + D + hv * dv, tmp + t * hv, sizeof(uint16_t) * hv);
    orc_linear(x, w->w_a, N, hv, H, tmp);
    for (int64_t t = 0; t < N; ++t) memcpy(proj + t * ldp + D + hv * dv + hv, tmp + t * hv, sizeof(uint16_t) * hv);
    int rc = orc_layer_step(c, &w->core, proj, ldp, proj + D, ldp, proj + D + hv * dv, ldp, conv_state, rec_state, cu,
                            n_seq, gated, NULL);
    if (rc == ORC_OK) orc_linear(gated, w->w_out, N, H, hv * dv, mix_out);
    free(proj); free(tmp); free(gated);
    return rc;
}

/*
 * One decoder-style residual step per GDN layer (qwen3_5.rs:729-739 restricted
 * to the mixer): h <- h + mixer(rms_norm(h, pre_w, eps)), over `n_layers`
 * layers.  conv_state / rec_state hold [n_layers][n_seq][...].
 */
int orc_stack_step(const orc_cfg* c, const orc_mixer_w* ws, int32_t n_layers, uint16_t* h, uint16_t* conv_state,
                   float* rec_state, const int32_t* cu, int32_t n_seq) {
    const int D = conv_dim(c), H = c->hidden;
    const int64_t N = cu[n_seq];
    uint16_t* hn = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(N > 0 ? N : 1) * H);
    uint16_t* mo = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(N > 0 ? N : 1) * H);
    if (!hn || !mo) { free(hn); free(mo); return ORC_ENOMEM; }
    int rc = ORC_OK;
    for (int32_t l = 0; l < n_layers && rc == ORC_OK; ++l) {
        orc_rms_norm(h, ws[l].pre_w, N, H, c->eps, hn);
        rc = orc_mixer_step(c, &ws[l], hn, conv_state + (int64_t)l * n_seq * (c->conv_k - 1) * D,
                            rec_state + (int64_t)l * n_seq * c->hv * c->dv * c->dk, cu, n_seq, mo);
        for (int64_t i = 0; i < N * H; ++i) h[i] = tobf(bf(h[i]) + bf(mo[i]));
    }
    free(hn); free(mo);
    return rc;
}

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
