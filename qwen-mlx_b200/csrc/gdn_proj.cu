// gdn_proj.cu -- the pieces around the fused step that make a whole mixer layer
// and the residual stack:
//   * the in/out projections (qwen3_5.rs:572-586, :667-668) as bf16 GEMMs with f32
//     accumulation and a bf16 result, run by cuBLASLt (a library GEMM, declared as
//     such: these are plain matmuls, nn::Linear without bias);
//   * the decoder-layer input RMSNorm and residual add (qwen3_5.rs:729-739), fused
//     into one row kernel: h <- bf16(h + o); hn <- bf16(w * bf16(h * rsqrt(mean(h^2) + eps))).
#include <cublasLt.h>

#include <cstring>

#include "gdn_device.cuh"
#include "gdn_internal.h"
#include "gdn_ptx.cuh"

namespace gdn {

// ------------------------------------------------------------------ row kernel

// One CTA per row of H bf16 values.  If `o` is non-null the residual is added first
// (h_out = bf16(h_in + o)); then, unless `hn` is null, hn = MLX fast::rms_norm(h_out, w, eps):
// the normalised value is rounded to bf16 before the gain multiply, which rounds again.
// Launched as a programmatic dependent: it lets the next kernel (the in-projection, which streams its static
// weight before its own dependency wait) launch at once, then waits for the kernel that produced h and o.  h and
// o are read with coherent loads (__ldcg): the out-projection before it releases it early, and the non-coherent
// path is only for data no running grid writes.
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(const uint16_t* h_in, long long ld_h,
                                                          const uint16_t* o, long long ld_o,
                                                          uint16_t* h_out, const uint16_t* __restrict__ w,
                                                          uint16_t* __restrict__ hn, long long ld_hn, int H,
                                                          float eps) {
    __shared__ float s_red[8];
    pdl_launch_dependents();
    pdl_wait();
    const long long r = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float acc = 0.0f;
    // first pass: residual add (written back), sum of squares
    for (int c = tid; c < H; c += 256) {
        float v = bf2f(__ldcg(h_in + r * ld_h + c));
        if (o) {
            v = rbf(v + bf2f(__ldcg(o + r * ld_o + c)));
            h_out[r * ld_h + c] = f2bf(v);
        }
        acc += v * v;
    }
    if (!hn) return;  // residual add only
    acc = warp_sum(acc);
    if (lane == 0) s_red[warp] = acc;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += s_red[i];
    const float nrm = 1.0f / sqrtf(tot / (float)H + eps);
    for (int c = tid; c < H; c += 256) {
        const float v = o ? bf2f(h_out[r * ld_h + c]) : bf2f(__ldcg(h_in + r * ld_h + c));
        hn[r * ld_hn + c] = f2bf(bf2f(w[c]) * rbf(v * nrm));
    }
}

cudaError_t launch_add_rmsnorm(const uint16_t* h_in, long long ld_h, const uint16_t* o, long long ld_o,
                               uint16_t* h_out, const uint16_t* w, uint16_t* hn, long long ld_hn, int rows, int H,
                               float eps, cudaStream_t stream) {
    if (rows <= 0) return cudaSuccess;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t c = {};
    c.gridDim = dim3((unsigned)rows, 1, 1);
    c.blockDim = dim3(256, 1, 1);
    c.stream = stream;
    c.attrs = attr;
    c.numAttrs = 1;
    return cudaLaunchKernelEx(&c, add_rmsnorm_kernel, h_in, ld_h, o, ld_o, h_out, w, hn, ld_hn, H, eps);
}

// ------------------------------------------------------------------ GEMM (cuBLASLt)

// Per GEMM shape, the cuBLASLt algorithm that timed fastest among the heuristic's top candidates
// (chosen on the first call made outside stream capture; calls during capture take the top one).
struct GemmPlan {
    int M, N, K;
    long long ldx, ldo;
    cublasLtMatmulAlgo_t algo;
};

struct GemmCtx {
    cublasLtHandle_t handle = nullptr;
    void* workspace = nullptr;
    size_t ws_bytes = 0;
    GemmPlan plans[32];
    int n_plans = 0;
};

GemmCtx* gemm_create(void* workspace, size_t ws_bytes) {
    GemmCtx* g = new GemmCtx();
    if (cublasLtCreate(&g->handle) != CUBLAS_STATUS_SUCCESS) {
        delete g;
        return nullptr;
    }
    g->workspace = workspace;
    g->ws_bytes = ws_bytes;
    return g;
}

void gemm_destroy(GemmCtx* g) {
    if (!g) return;
    if (g->handle) cublasLtDestroy(g->handle);
    delete g;
}

// out[m][n] = bf16( sum_k x[m][k] * w[n][k] ), row-major x [M][K] (stride ldx), w [N][K]
// (stride K), out [M][N] (stride ldo); f32 accumulation.  In cuBLAS's column-major
// terms this is out^T (N x M) = w (stored K x N, transposed) * x^T (K x M).
int gemm_bf16_nt(GemmCtx* g, int M, int N, int K, const uint16_t* x, long long ldx, const uint16_t* w,
                 uint16_t* out, long long ldo, cudaStream_t stream) {
    if (M <= 0) return 0;
    cublasLtMatmulDesc_t op = nullptr;
    cublasLtMatrixLayout_t la = nullptr, lb = nullptr, lc = nullptr;
    cublasLtMatmulPreference_t pref = nullptr;
    int rc = 1;
    do {
        if (cublasLtMatmulDescCreate(&op, CUBLAS_COMPUTE_32F, CUDA_R_32F) != CUBLAS_STATUS_SUCCESS) break;
        const cublasOperation_t ta = CUBLAS_OP_T, tb = CUBLAS_OP_N;
        cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSA, &ta, sizeof ta);
        cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSB, &tb, sizeof tb);
        if (cublasLtMatrixLayoutCreate(&la, CUDA_R_16BF, K, N, K) != CUBLAS_STATUS_SUCCESS) break;
        if (cublasLtMatrixLayoutCreate(&lb, CUDA_R_16BF, K, M, ldx) != CUBLAS_STATUS_SUCCESS) break;
        if (cublasLtMatrixLayoutCreate(&lc, CUDA_R_16BF, N, M, ldo) != CUBLAS_STATUS_SUCCESS) break;
        const float alpha = 1.0f, beta = 0.0f;
        const GemmPlan* plan = nullptr;
        for (int i = 0; i < g->n_plans; ++i) {
            const GemmPlan& q = g->plans[i];
            if (q.M == M && q.N == N && q.K == K && q.ldx == ldx && q.ldo == ldo) plan = &q;
        }
        cublasLtMatmulAlgo_t algo;
        if (plan) {
            algo = plan->algo;
        } else {
            if (cublasLtMatmulPreferenceCreate(&pref) != CUBLAS_STATUS_SUCCESS) break;
            cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &g->ws_bytes,
                                                 sizeof g->ws_bytes);
            cublasLtMatmulHeuristicResult_t heur[8];
            int found = 0;
            if (cublasLtMatmulAlgoGetHeuristic(g->handle, op, la, lb, lc, lc, pref, 8, heur, &found) !=
                    CUBLAS_STATUS_SUCCESS ||
                found == 0)
                break;
            algo = heur[0].algo;
            cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
            cudaStreamIsCapturing(stream, &cap);
            if (cap == cudaStreamCaptureStatusNone && found > 1) {
                // time every candidate on this call's operands (3 runs each, after one warm-up run)
                cudaEvent_t e0, e1;
                cudaEventCreate(&e0);
                cudaEventCreate(&e1);
                float best = 1e30f;
                for (int i = 0; i < found; ++i) {
                    if (cublasLtMatmul(g->handle, op, &alpha, w, la, x, lb, &beta, out, lc, out, lc, &heur[i].algo,
                                       g->workspace, g->ws_bytes, stream) != CUBLAS_STATUS_SUCCESS)
                        continue;
                    cudaEventRecord(e0, stream);
                    for (int r = 0; r < 3; ++r)
                        cublasLtMatmul(g->handle, op, &alpha, w, la, x, lb, &beta, out, lc, out, lc, &heur[i].algo,
                                       g->workspace, g->ws_bytes, stream);
                    cudaEventRecord(e1, stream);
                    cudaEventSynchronize(e1);
                    float ms = 0.f;
                    cudaEventElapsedTime(&ms, e0, e1);
                    if (ms < best) {
                        best = ms;
                        algo = heur[i].algo;
                    }
                }
                cudaEventDestroy(e0);
                cudaEventDestroy(e1);
                if (g->n_plans < 32) g->plans[g->n_plans++] = GemmPlan{M, N, K, ldx, ldo, algo};
            }
        }
        if (cublasLtMatmul(g->handle, op, &alpha, w, la, x, lb, &beta, out, lc, out, lc, &algo, g->workspace,
                           g->ws_bytes, stream) != CUBLAS_STATUS_SUCCESS)
            break;
        rc = 0;
    } while (false);
    if (pref) cublasLtMatmulPreferenceDestroy(pref);
    if (lc) cublasLtMatrixLayoutDestroy(lc);
    if (lb) cublasLtMatrixLayoutDestroy(lb);
    if (la) cublasLtMatrixLayoutDestroy(la);
    if (op) cublasLtMatmulDescDestroy(op);
    return rc;
}

}  // namespace gdn
