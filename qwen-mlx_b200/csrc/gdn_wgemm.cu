// gdn_wgemm.cu -- weight-streaming projection GEMM (qwen3_5.rs:572-586 in_proj_*, :668 out_proj):
// y[m][n] = bf16(sum_k x[m][k] * w[n][k]) with f32 accumulation, for calls of at most 64 tokens
// per launch (longer calls run in blocks of 64 tokens; the mixer instead expands a 4-bit weight to bf16
// once, wq_untile_kernel, and runs one library GEMM for them).
//
// With few tokens the GEMM moves each weight once for 2*M flops: it is bound by streaming the weight
// out of HBM.  So the weight is stored once, at load, in the layout the tensor core reads ("tiled
// weight"), and every CTA streams its share with bulk async copies.  The unit of storage is a block
// of 8 rows (a row group) x 64 columns (a k-tile), blocks ordered k-tile major, row group minor, so
// any run of row groups of one k-tile is contiguous.  Two formats:
//
//   bf16: block (kt, rg) is 1 KB at (kt * NRG + rg) * 1024 (NRG = ceil(N/8)); element (8 rg + r8,
//     64 kt + 8 c + e) at c*128 + r8*16 + e*2 -- the K-major core-matrix layout with 128 B between the
//     8-column chunks and 1 KB between row groups; zero padding.
//   4-bit (MLX affine quantization, groups of 64 columns = one k-tile; w = scale * q + bias, q in
//     0..15): block (kt, rg) is 288 B at (kt * NRG + rg) * 288: word (c, r8) at c*32 + r8*4 holds the
//     codes of row 8 rg + r8, columns 64 kt + 8c .. +7 (column 8c+e in nibble e/2 for even e, 4 + e/2
//     for odd e), then the 8 row scales (bf16) at 256 and the 8 row biases at 272.  The loader warps
//     dequantize a unit into the bf16 layout above, each weight rounded once to bf16 (one bf16x2 FMA,
//     scale * q + bias), as MLX's quantized matmul tile loader does.
//
// Work: the rows are cut into NS slabs of at most 16 row groups (128 rows); unit (slab, kt) is one
// contiguous copy.  Units in (slab, kt) order are cut into G equal contiguous runs, one per CTA
// (G = min(#SMs, units)).  When the rows allow slabs of >= 64 rows on every SM (the in-projection),
// NS is a multiple of G and every CTA owns whole slabs: no partial sums at all.  Otherwise (the
// out-projection: 2048 rows) slabs are 128 rows, a CTA's run may cover part of a slab's k range,
// partial f32 sums go to a workspace, and the last CTA to finish a slab (per-slab arrival counter)
// adds them in CTA order: the sum order, and so the output, repeats bit for bit.
//
// MMA: tcgen05 kind::f16, the weight slab as A (M = 128; rows past the slab are ignored), the tokens
// as B (N = MP = 16/32/64 padded tokens, K-major, column-first: LBO MP*16 B, SBO 128 B); the f32
// accumulators [128 rows][MP tokens] (one set per issuer) live in TMEM, double-buffered.
//
// Roles: warp 0 streams the weight (bulk copies from several lanes; the first ring's worth is issued
// before the wait on the previous kernel, since the weight does not depend on it); warps 1 and 6 (lane
// 0) issue the MMAs of the even / odd units into two accumulator sets; warps 2-5 drain the accumulators
// (TMEM lane quarter w%4) and store; the loader warps (from warp 7: 4 groups of 1 warp for bf16; for
// 4-bit, 8 groups of 2 warps at 16 tokens, 4 of 2 at 32, 4 of 1 at 64; group g takes units g, g+NG, ...)
// copy each unit's token chunk into the stage with plain loads (and dequantize a 4-bit unit), fence the
// writes for the tensor core and signal.
// Every wait is bounded (2 s): a timeout sets ERR_TIMEOUT and the CTA winds down.
#include <cuda_runtime.h>

#include "gdn_device.cuh"
#include "gdn_internal.h"
#include "gdn_umma.cuh"

namespace gdn {

namespace {

constexpr int WG_ROWS = 128;                 // rows of one MMA (a slab holds at most this many)
constexpr int WG_K = 64;                     // columns of a k-tile (and of a 4-bit group)
constexpr int WG_BLK = 1024;                 // bf16 block: 8 rows x 64 columns
constexpr int WQ_BLK = 288;                  // 4-bit block: codes 256 B, scales 16 B, biases 16 B
constexpr int WG_TILE = 16 * WG_BLK;         // bf16 unit of a full slab (16 row groups)
constexpr int WQ_TILE = 16 * WQ_BLK;         // 4-bit unit of a full slab
constexpr uint64_t WG_WAIT_NS = 2000000000ull;

template <int MP, bool Q4>
struct WgShape {
    // Weight stream: PL lanes of warp 0 issue bulk copies side by side (lane l takes units l, l+PL, ...):
    // one thread's copies are accepted one at a time, so several lanes are needed to keep the HBM busy
    // with units of a few KB.  Loaders: NG groups of WPU warps; group g takes units g, g+NG, ..., its
    // warps split the unit's rows and token chunks.  Parity waits stay exact because nothing runs more
    // than one phase ahead on a barrier: NG <= NST (stage-free barriers), NQ % NG == 0 (4-bit staging:
    // unit i - NQ of a slot was the same group's), and the ring depth a multiple of PL (a lane's last
    // DEPTH/PL copies never share a slot, so its drain waits the right phases).
    static constexpr int PL = Q4 ? 8 : 4;
    static constexpr int NG = (Q4 && MP == 16) ? 8 : 4;
    static constexpr int WPU = (Q4 && MP < 64) ? 2 : 1;
    static constexpr int NL = NG * WPU;                     // loader warps
    static constexpr int THREADS = 32 * (7 + NL);           // + producer, 2 MMA issuers, 4 epilogue warps
    static constexpr int XB = MP * WG_K * 2;                // token chunk of one stage
    static constexpr int STG = WG_TILE + XB;                // one MMA stage (weight tile + tokens)
    static constexpr int SMEM_MAX = 227 * 1024 - 1024;      // rings + barriers
    static constexpr int NQ = Q4 ? 16 : 0;                 // 4-bit staging ring (a multiple of PL and NG)
    static constexpr int NST_FIT = (SMEM_MAX - 1024 - NQ * WQ_TILE) / STG;
    static constexpr int NST = Q4 ? (NST_FIT > 8 ? 8 : NST_FIT) / 2 * 2 : (NST_FIT > 12 ? 12 : NST_FIT) / PL * PL;
    // One tcgen05.commit (hundreds of cycles) frees a group of G consecutive stages: stage s's "free"
    // barrier is empty[s / G], completed once per pass over the ring.
    static constexpr int G = (NST % 4 == 0) ? 4 : 2;
    static constexpr int OFF_Q = NST * STG;
    static constexpr int OFF_BARS = OFF_Q + NQ * WQ_TILE;
    // wfull/xfull/empty [NST], qfull/qempty [NQ], acc full x2, acc empty x2, done x2
    static constexpr int N_BARS = 3 * NST + 2 * NQ + 6;
    static constexpr int SMEM = OFF_BARS + N_BARS * 8 + 16;
    // Two MMA issuers (units of even / odd index) accumulate into their own f32 set [128][MP]; one
    // accumulator buffer holds both sets, double-buffered: 64 / 128 / 256 TMEM columns.
    static constexpr int ACC_COLS = 2 * MP;
    static constexpr int TMEM_COLS = 2 * ACC_COLS < 32 ? 32 : 2 * ACC_COLS;
    static_assert(SMEM <= 227 * 1024, "shared memory");
    static_assert(!Q4 || NST >= 6, "4-bit stage ring too shallow");
    static_assert(NST >= 8 || Q4, "bf16 ring too shallow");
    static_assert(NG <= NST && (Q4 ? (NQ % NG == 0 && NQ % PL == 0) : (NST % PL == 0)), "ring sizes");
    static_assert(NST % G == 0 && G % 2 == 0, "stage groups (each issuer commits once per group)");
};

struct WgArgs {
    const uint8_t* tiles;
    const uint16_t* x;
    long long ldx;
    uint16_t* y;
    long long ldy;
    int M, N, K;
    int NRG, NS, KT;  // row groups, slabs, k-tiles
    int rot;          // every CTA owns whole slabs: each slab walks its k-tiles from a slab-dependent start
    int U;            // NS * KT units (U * G < 2^31)
    int G;
    float* ws;        // [2*G][128*MP] f32 partial sums
    int* cnt;         // [NS] arrival counters (zero between launches)
    int* err;
};

// Index math in 32 bits (the host checks U * G < 2^31): a 64-bit division costs hundreds of cycles.
__device__ __forceinline__ int wg_run_start(int c, int U, int G) { return (int)((unsigned)(c * U) / (unsigned)G); }
__device__ __forceinline__ int wg_slab_rg0(int slab, int NRG, int NS) {
    return (int)((unsigned)(slab * NRG) / (unsigned)NS);
}

// Walks a CTA's units (slab, j-th k-tile of the slab) without a division per unit.  With rotation the
// j-th k-tile of slab s is (j + 7 s) mod KT, so the CTAs read different token chunks at any moment
// (the order is fixed per slab, so the sums repeat bit for bit).
struct WgPos {
    int slab, j;       // current unit
    int rg0, nrg;      // row groups of the slab
    int rot;           // k-tile of j = 0
    __device__ __forceinline__ void set_slab(const WgArgs& a) {
        rg0 = wg_slab_rg0(slab, a.NRG, a.NS);
        nrg = wg_slab_rg0(slab + 1, a.NRG, a.NS) - rg0;
        rot = a.rot ? (int)((unsigned)(7 * slab) % (unsigned)a.KT) : 0;
    }
    __device__ __forceinline__ void start(int u, const WgArgs& a) {
        slab = (int)((unsigned)u / (unsigned)a.KT);
        j = u - slab * a.KT;
        set_slab(a);
    }
    __device__ __forceinline__ void advance(int step, const WgArgs& a) {
        j += step;
        if (j >= a.KT) {
            while (j >= a.KT) {
                j -= a.KT;
                ++slab;
            }
            set_slab(a);
        }
    }
    __device__ __forceinline__ int kt(int KT) const {
        const int k = j + rot;
        return k >= KT ? k - KT : k;
    }
};
// The CTA whose run holds tile-unit u: the largest c with floor(c*U/G) <= u.
__device__ __forceinline__ int wg_cta_of(int u, int U, int G) {
    return (int)((unsigned)((u + 1) * G + U - 1) / (unsigned)U) - 1;
}

// Bounded mbarrier wait: one plain test, then polls spaced by `sleep_ns` of __nanosleep, so waiting
// warps leave the schedulers to the warps on the critical path (the MMA issuer polls without sleeping).
__device__ __forceinline__ bool wg_wait(uint64_t* bar, uint32_t parity, uint32_t sleep_ns = 0) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (global_timer_ns() - t0 > WG_WAIT_NS) return false;
        if (sleep_ns) __nanosleep(sleep_ns);
    }
}

// The same wait for a whole warp: lane 0 polls, the warp gets its answer (one poller per warp keeps
// the barrier unit free for the copies and arrivals on the critical path).  Warp-uniform call.
__device__ __forceinline__ bool wg_wait_warp(uint64_t* bar, uint32_t parity, uint32_t sleep_ns) {
    bool ok = true;
    if ((threadIdx.x & 31) == 0) ok = wg_wait(bar, parity, sleep_ns);
    return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

__device__ __forceinline__ uint32_t bf16x2_fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.bf16x2 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Eight 4-bit codes (nibble order of the 4-bit tile) -> eight bf16 weights scale * q + bias, in
// column order.  (nib | 0x4300) is the bf16 of 128 + q exactly; subtracting 128 is exact.
__device__ __forceinline__ uint4 wq_dequant8(uint32_t w, uint32_t s2, uint32_t b2) {
    const uint32_t one2 = 0x3F803F80u, m128 = 0xC300C300u;
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t t = ((w >> (4 * j)) & 0x000F000Fu) | 0x43004300u;
        o[j] = bf16x2_fma(bf16x2_fma(t, one2, m128), s2, b2);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

}  // namespace

// ------------------------------------------------------------------ weight tiling (once, at load)

__global__ void __launch_bounds__(256) wg_tile_kernel(const uint16_t* __restrict__ w, int N, int K, int NRG,
                                                      uint8_t* __restrict__ tiles, long long n_chunks) {
    const long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // 16-byte chunk (kt, rg, c, r8)
    if (q >= n_chunks) return;
    const int r8 = (int)(q & 7), c = (int)((q >> 3) & 7);
    const long long blk = q >> 6;
    const int kt = (int)(blk / NRG), rg = (int)(blk % NRG);
    const long long n = (long long)rg * 8 + r8;
    const int k0 = kt * WG_K + c * 8;
    uint16_t v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = (n < N && k0 + j < K) ? w[n * K + k0 + j] : (uint16_t)0;
    uint4 o;
    o.x = v[0] | ((uint32_t)v[1] << 16);
    o.y = v[2] | ((uint32_t)v[3] << 16);
    o.z = v[4] | ((uint32_t)v[5] << 16);
    o.w = v[6] | ((uint32_t)v[7] << 16);
    *reinterpret_cast<uint4*>(tiles + q * 16) = o;
}

// MLX layout in: wq [N][K/8] uint32 (column k in bits 4*(k%8) of word k/8), scales / biases [N][K/64].
__global__ void __launch_bounds__(256) wq_tile_kernel(const uint32_t* __restrict__ wq,
                                                      const uint16_t* __restrict__ scales,
                                                      const uint16_t* __restrict__ biases, int N, int K, int NRG,
                                                      uint8_t* __restrict__ tiles, long long n_words) {
    const long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // word (kt, rg, c, r8)
    if (q >= n_words) return;
    const int r8 = (int)(q & 7), c = (int)((q >> 3) & 7);
    const long long blk = q >> 6;
    const int kt = (int)(blk / NRG), rg = (int)(blk % NRG);
    const long long n = (long long)rg * 8 + r8;
    uint32_t out = 0;
    uint16_t sc = 0, bi = 0;
    if (n < N) {
        const uint32_t in = wq[n * (K / 8) + kt * 8 + c];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int pos = (e & 1) ? 4 + (e >> 1) : (e >> 1);
            out |= ((in >> (4 * e)) & 0xFu) << (4 * pos);
        }
        sc = scales[n * (K / 64) + kt];
        bi = biases[n * (K / 64) + kt];
    }
    uint8_t* t = tiles + blk * WQ_BLK;
    *reinterpret_cast<uint32_t*>(t + c * 32 + r8 * 4) = out;
    if (c == 0) {
        *reinterpret_cast<uint16_t*>(t + 256 + r8 * 2) = sc;
        *reinterpret_cast<uint16_t*>(t + 272 + r8 * 2) = bi;
    }
}

// ------------------------------------------------------------------ the GEMM

template <int MP, bool Q4>
__global__ void __launch_bounds__(WgShape<MP, Q4>::THREADS, 1) wg_gemm_kernel(WgArgs a) {
    using S = WgShape<MP, Q4>;
    constexpr int BLK = Q4 ? WQ_BLK : WG_BLK;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + S::OFF_BARS);  // bf16: weight bytes landed
    uint64_t* xfull = wfull + S::NST;                                   // tokens (and 4-bit dequant) in
    uint64_t* empty = xfull + S::NST;                                   // MMAs of the stage done
    uint64_t* qfull = empty + S::NST;                                   // 4-bit: staged tile landed
    uint64_t* qempty = qfull + S::NQ;                                   // 4-bit: staged tile read
    uint64_t* accf = qempty + S::NQ;
    uint64_t* acce = accf + 2;
    uint64_t* done = acce + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 2);
    volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* s_last = s_abort + 1;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int cta = blockIdx.x;
    const int ua = wg_run_start(cta, a.U, a.G), ub = wg_run_start(cta + 1, a.U, a.G);
    const int n_units = ub - ua;
    const int KT = a.KT;

    if (tid == 0) {
        for (int s = 0; s < S::NST; ++s) {
            mbar_init(&wfull[s], 1);
            mbar_init(&xfull[s], S::WPU);
            if (s % S::G == 0) mbar_init(&empty[s / S::G], 2);  // one commit per issuer
        }
        for (int s = 0; s < S::NQ; ++s) {
            mbar_init(&qfull[s], 1);
            mbar_init(&qempty[s], S::WPU);
        }
        mbar_init(&accf[0], 2);
        mbar_init(&accf[1], 2);
        mbar_init(&acce[0], 128);
        mbar_init(&acce[1], 128);
        mbar_init(&done[0], 1);
        mbar_init(&done[1], 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, S::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------------------------------------------------------- weight stream
        if (lane < S::PL) {
            constexpr int DEPTH = Q4 ? S::NQ : S::NST;
            uint64_t* landed = Q4 ? qfull : wfull;
            uint64_t* freed = Q4 ? qempty : empty;
            WgPos pos;
            pos.start(ua + lane, a);
            int i = lane, last = -1;
            for (; i < (int)n_units; i += S::PL, pos.advance(S::PL, a)) {
                const int s = i % DEPTH;
                if (i >= DEPTH && !wg_wait(&freed[Q4 ? s : s / S::G], ((uint32_t)(i / DEPTH) & 1u) ^ 1u, 32)) {
                    atomicOr(a.err, ERR_TIMEOUT);
                    *s_abort = 1;
                }
                if (*s_abort) break;
                uint8_t* dst = Q4 ? smem + S::OFF_Q + s * WQ_TILE : smem + s * S::STG;
                const uint32_t bytes = (uint32_t)(pos.nrg * BLK);
                mbar_arrive_expect_tx(&landed[s], bytes);
                bulk_g2s(dst, a.tiles + ((long long)pos.kt(KT) * a.NRG + pos.rg0) * BLK, bytes, &landed[s]);
                last = i;
            }
            // No copy may still be landing when the CTA exits (only after a timeout can one be unconsumed):
            // this lane's last DEPTH/PL copies, whose slots no later copy has reused.
            for (int j = last; j >= 0 && j > last - DEPTH; j -= S::PL)
                wg_wait(&landed[j % DEPTH], (uint32_t)(j / DEPTH) & 1u, 64);
        }
        __syncwarp();
    } else if (warp == 1 || warp == 6) {
        // ---------------------------------------------------------------- MMA issue: issuer p takes the
        // units of index parity p (one thread's MMA issue and barrier tests cost more per unit than the
        // tensor core needs, so two issuers share the stream) into its own accumulator set.
        const int p = warp == 1 ? 0 : 1;
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_bf16(128, MP);
            int i = 0;
            int seg = 0;
            for (int u = ua; u < ub && !*s_abort; ++seg) {
                const int kt0 = u % KT;
                const int len = min(KT - kt0, ub - u);
                const int ab = seg & 1;
                if (seg >= 2 && !wg_wait(&acce[ab], (uint32_t)((seg >> 1) - 1) & 1u)) {
                    atomicOr(a.err, ERR_TIMEOUT);
                    *s_abort = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(ab * S::ACC_COLS + p * MP);
                bool bad = false, first = true;
                for (int j = 0; j < len; ++j, ++i) {
                    if ((i & 1) != p) continue;
                    const int s = i % S::NST;
                    const uint32_t ph = (uint32_t)(i / S::NST) & 1u;
                    if ((!Q4 && !wg_wait(&wfull[s], ph)) || !wg_wait(&xfull[s], ph)) {
                        bad = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sw = smem_u32(smem + s * S::STG);
                    const uint64_t ad = umma_desc_raw(sw, 128u, 1024u);  // 128 B per k chunk, 1 KB per row group
                    const uint64_t bd = umma_desc_raw(sw + WG_TILE, (uint32_t)(MP * 16), 128u);
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
                        umma_bf16(d, ad + (uint64_t)ks * (256u >> 4), bd + (uint64_t)ks * ((MP * 32u) >> 4), idesc,
                                  (!first || ks > 0) ? 1u : 0u);
                    first = false;
                    // this issuer's last unit of the stage group: its share of freeing the group
                    if (s % S::G == S::G - 2 + p) umma_commit(&empty[s / S::G]);
                }
                if (bad) {
                    atomicOr(a.err, ERR_TIMEOUT);
                    *s_abort = 1;
                    break;
                }
                umma_commit(&accf[ab]);
                u += len;
            }
            umma_commit(&done[p]);  // arrives once every MMA this issuer issued has completed
            if (!wg_wait(&done[p], 0)) atomicOr(a.err, ERR_TIMEOUT);
        }
        __syncwarp();
    } else if (warp < 6) {
        // ---------------------------------------------------------------- epilogue warps 2..5
        const int etid = tid - 64;
        const int quarter = warp & 3;
        const int r = 32 * quarter + lane;
        const int first_slab = ua / KT;
        const uint32_t trow = tmem + ((uint32_t)(32 * quarter) << 16);
        int seg = 0;
        for (int u = ua; u < ub; ++seg) {
            const int t = u / KT;  // slab
            const int rg0 = wg_slab_rg0(t, a.NRG, a.NS), rows = 8 * (wg_slab_rg0(t + 1, a.NRG, a.NS) - rg0);
            const int kt0 = (int)(u % KT);
            const int len = min(KT - kt0, ub - u);
            const int ab = seg & 1;
            const bool bad = !wg_wait_warp(&accf[ab], (uint32_t)(seg >> 1) & 1u, 256);
            if (bad) {
                atomicOr(a.err, ERR_TIMEOUT);
                *s_abort = 1;
            }
            if (named_bar_or(1, 128, bad || *s_abort)) break;
            tc_fence_after();
            // set p holds the units of index parity p; a one-unit segment has only one of them
            const int i0 = u - ua;
            const bool has0 = len >= 2 || (i0 & 1) == 0, has1 = len >= 2 || (i0 & 1) == 1;
            float acc[MP];
#pragma unroll
            for (int m = 0; m < MP; ++m) acc[m] = 0.0f;
#pragma unroll
            for (int p = 0; p < 2; ++p) {  // sets added in a fixed order
                if (p == 0 ? !has0 : !has1) continue;
#pragma unroll
                for (int j = 0; j < MP; j += 16) {
                    float v[16];
                    tmem_ld16(trow + (uint32_t)(ab * S::ACC_COLS + p * MP + j), v);
#pragma unroll
                    for (int e = 0; e < 16; ++e) acc[j + e] += v[e];
                }
            }
            tc_fence_before();
            mbar_arrive(&acce[ab]);
            const long long n = (long long)rg0 * 8 + r;
            const bool row_ok = r < rows && n < a.N;
            if (kt0 == 0 && len == KT) {
                if (row_ok) {
#pragma unroll
                    for (int m = 0; m < MP; ++m)
                        if (m < a.M) a.y[(long long)m * a.ldy + n] = f2bf(acc[m]);
                }
            } else {
                float4* mine = reinterpret_cast<float4*>(a.ws + (size_t)(2 * cta + (t == first_slab ? 0 : 1)) *
                                                                    (WG_ROWS * MP) + (size_t)r * MP);
#pragma unroll
                for (int m = 0; m < MP; m += 4) mine[m / 4] = make_float4(acc[m], acc[m + 1], acc[m + 2], acc[m + 3]);
                __threadfence();
                named_bar_sync(1, 128);
                const int c0 = wg_cta_of(t * KT, a.U, a.G), c1 = wg_cta_of(t * KT + KT - 1, a.U, a.G);
                if (etid == 0) *s_last = (atomicAdd(&a.cnt[t], 1) == c1 - c0) ? 1 : 0;
                named_bar_sync(1, 128);
                if (*s_last) {
                    __threadfence();
                    float sum[MP];
#pragma unroll
                    for (int m = 0; m < MP; ++m) sum[m] = 0.0f;
                    // in CTA order; this CTA's own partial is read back from where it was just stored.  Two
                    // contributors' loads are in flight at a time; the adds stay in CTA order.
                    auto part = [&](int c) {
                        const int cf = wg_run_start(c, a.U, a.G) / KT;
                        return reinterpret_cast<const float4*>(a.ws + (size_t)(2 * c + (t == cf ? 0 : 1)) *
                                                                          (WG_ROWS * MP) + (size_t)r * MP);
                    };
                    for (int c = c0; c <= c1; c += 2) {
                        const bool two = c + 1 <= c1;
                        const float4* p0 = part(c);
                        const float4* p1 = two ? part(c + 1) : p0;
                        float4 v0[MP / 4], v1[MP / 4];
#pragma unroll
                        for (int m = 0; m < MP / 4; ++m) {
                            v0[m] = __ldcg(p0 + m);
                            v1[m] = two ? __ldcg(p1 + m) : make_float4(0.f, 0.f, 0.f, 0.f);
                        }
#pragma unroll
                        for (int m = 0; m < MP / 4; ++m) {
                            sum[4 * m] += v0[m].x;
                            sum[4 * m + 1] += v0[m].y;
                            sum[4 * m + 2] += v0[m].z;
                            sum[4 * m + 3] += v0[m].w;
                        }
                        if (two) {
#pragma unroll
                            for (int m = 0; m < MP / 4; ++m) {
                                sum[4 * m] += v1[m].x;
                                sum[4 * m + 1] += v1[m].y;
                                sum[4 * m + 2] += v1[m].z;
                                sum[4 * m + 3] += v1[m].w;
                            }
                        }
                    }
                    if (row_ok) {
#pragma unroll
                        for (int m = 0; m < MP; ++m)
                            if (m < a.M) a.y[(long long)m * a.ldy + n] = f2bf(sum[m]);
                    }
                    if (etid == 0) a.cnt[t] = 0;  // every contributor has arrived: ready for the next launch
                }
            }
            u += len;
        }
    } else {
        // ---------------------------------------------------------------- loader warps
        const int lw = warp - 7, grp = lw / S::WPU, half = lw % S::WPU;
        pdl_wait();  // the tokens are the previous kernel's output
        constexpr int XPL = MP / (4 * S::WPU);  // 16-byte token chunks per lane per unit
        // token chunk of this warp's share of unit (k-tile kt), loaded into registers one unit ahead
        auto load_x = [&](int kt, uint4 (&xv)[XPL]) {
#pragma unroll
            for (int e = 0; e < XPL; ++e) {
                const int q = half * 32 + lane + 32 * S::WPU * e;
                const int m = q >> 3, c = q & 7;
                const int k0 = kt * WG_K + c * 8;
                xv[e] = make_uint4(0u, 0u, 0u, 0u);
                if (m < a.M && k0 < a.K) xv[e] = __ldcg(reinterpret_cast<const uint4*>(a.x + (long long)m * a.ldx + k0));
            }
        };
        WgPos pos;
        pos.start(ua + grp, a);
        uint4 xv[XPL];
        if (grp < n_units) load_x(pos.kt(KT), xv);
        for (int i = grp; i < n_units; i += S::NG, pos.advance(S::NG, a)) {
            const int s = i % S::NST;
            bool bad = false;
            if (i >= S::NST) bad = !wg_wait_warp(&empty[s / S::G], ((uint32_t)(i / S::NST) & 1u) ^ 1u, 64);
            if (bad) {
                atomicOr(a.err, ERR_TIMEOUT);
                *s_abort = 1;
            }
            if (__any_sync(0xffffffffu, bad || *s_abort)) break;
            uint8_t* stg = smem + s * S::STG;
            if constexpr (Q4) {
                const int qs = i % S::NQ;
                bad = !wg_wait_warp(&qfull[qs], (uint32_t)(i / S::NQ) & 1u, 64);
                if (bad) {
                    atomicOr(a.err, ERR_TIMEOUT);
                    *s_abort = 1;
                }
                if (__any_sync(0xffffffffu, bad || *s_abort)) break;
                const uint8_t* qt = smem + S::OFF_Q + qs * WQ_TILE;
                const int nrows = 8 * pos.nrg;
                // this warp owns rows [half * 128 / WPU, +128 / WPU); lane owns every 32nd, all 8 chunks of each
#pragma unroll
                for (int rr = 0; rr < 4 / S::WPU; ++rr) {
                    const int row = half * (128 / S::WPU) + lane + 32 * rr;
                    if (row < nrows) {
                        const uint8_t* blk = qt + (row >> 3) * WQ_BLK;
                        const int r8 = row & 7;
                        const uint32_t sb = *reinterpret_cast<const uint16_t*>(blk + 256 + r8 * 2);
                        const uint32_t bb = *reinterpret_cast<const uint16_t*>(blk + 272 + r8 * 2);
                        const uint32_t s2 = sb | (sb << 16), b2 = bb | (bb << 16);
                        uint32_t wv[8];
#pragma unroll
                        for (int c = 0; c < 8; ++c) wv[c] = *reinterpret_cast<const uint32_t*>(blk + c * 32 + r8 * 4);
                        uint8_t* dst = stg + (row >> 3) * WG_BLK + r8 * 16;
#pragma unroll
                        for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(dst + c * 128) = wq_dequant8(wv[c], s2, b2);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&qempty[qs]);  // staged tile consumed: the stream may refill it
            }
#pragma unroll
            for (int e = 0; e < XPL; ++e) {
                const int q = half * 32 + lane + 32 * S::WPU * e;
                const int m = q >> 3, c = q & 7;
                *reinterpret_cast<uint4*>(stg + WG_TILE + c * MP * 16 + m * 16) = xv[e];
            }
            if (i + S::NG < n_units) {  // next unit's tokens, in flight while this unit waits on the tensor core
                WgPos nxt = pos;
                nxt.advance(S::NG, a);
                load_x(nxt.kt(KT), xv);
            }
            fence_async_shared();  // these generic-proxy writes before the tensor core's reads
            __syncwarp();
            if (lane == 0) mbar_arrive(&xfull[s]);
        }
    }

    pdl_launch_dependents();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, S::TMEM_COLS);
}

// ------------------------------------------------------------------ host side

// 4-bit tiles -> row-major bf16 weight [N][K] (each weight scale * q + bias rounded once, as the loader warps
// stage it): calls of more than WG_MAX_M tokens expand the weight once and run one library GEMM instead of
// streaming the tiles once per 64-token block.  Thread = (row n, 8-column chunk).
__global__ void __launch_bounds__(256) wq_untile_kernel(const uint8_t* __restrict__ tiles, int N, int K, int NRG,
                                                        uint16_t* __restrict__ w, long long n_chunks) {
    const long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= n_chunks) return;
    const int kc = K / 8;
    const long long n = q / kc;
    const int c8 = (int)(q - n * kc);
    const int kt = c8 >> 3, c = c8 & 7, rg = (int)(n >> 3), r8 = (int)(n & 7);
    const uint8_t* blk = tiles + ((long long)kt * NRG + rg) * WQ_BLK;
    const uint32_t word = *reinterpret_cast<const uint32_t*>(blk + c * 32 + r8 * 4);
    const uint32_t sb = *reinterpret_cast<const uint16_t*>(blk + 256 + r8 * 2);
    const uint32_t bb = *reinterpret_cast<const uint16_t*>(blk + 272 + r8 * 2);
    *reinterpret_cast<uint4*>(w + n * K + c8 * 8) = wq_dequant8(word, sb | (sb << 16), bb | (bb << 16));
}

long long wg_tile_bytes(int N, int K) {
    const long long NRG = (N + 7) / 8, KT = (K + WG_K - 1) / WG_K;
    return NRG * KT * WG_BLK;
}

long long wq_tile_bytes(int N, int K) {
    const long long NRG = (N + 7) / 8, KT = K / WG_K;
    return NRG * KT * WQ_BLK;
}

cudaError_t launch_wg_tile(const uint16_t* w, int N, int K, uint8_t* tiles, cudaStream_t stream) {
    const long long NRG = (N + 7) / 8, KT = (K + WG_K - 1) / WG_K;
    const long long n_chunks = NRG * KT * 64;
    wg_tile_kernel<<<(unsigned)((n_chunks + 255) / 256), 256, 0, stream>>>(w, N, K, (int)NRG, tiles, n_chunks);
    return cudaGetLastError();
}

cudaError_t launch_wq_tile(const uint32_t* wq, const uint16_t* scales, const uint16_t* biases, int N, int K,
                           uint8_t* tiles, cudaStream_t stream) {
    if (K % WG_K != 0) return cudaErrorInvalidValue;
    const long long NRG = (N + 7) / 8, KT = K / WG_K;
    const long long n_words = NRG * KT * 64;
    wq_tile_kernel<<<(unsigned)((n_words + 255) / 256), 256, 0, stream>>>(wq, scales, biases, N, K, (int)NRG, tiles,
                                                                          n_words);
    return cudaGetLastError();
}

cudaError_t launch_wq_untile(const void* tiles, int N, int K, uint16_t* w, cudaStream_t stream) {
    if (K % WG_K != 0 || N <= 0) return cudaErrorInvalidValue;
    const long long NRG = (N + 7) / 8, n_chunks = (long long)N * (K / 8);
    wq_untile_kernel<<<(unsigned)((n_chunks + 255) / 256), 256, 0, stream>>>(
        reinterpret_cast<const uint8_t*>(tiles), N, K, (int)NRG, w, n_chunks);
    return cudaGetLastError();
}

long long wg_workspace_floats(int n_sm) { return 2LL * n_sm * WG_ROWS * WG_MAX_M; }

int wg_num_slabs(int NRG, int n_sm) {
    if (NRG >= 8 * n_sm) return n_sm * ((NRG + 16 * n_sm - 1) / (16 * n_sm));
    return (NRG + 15) / 16;
}

static bool g_wg_attr[6][64] = {};

template <int MP, bool Q4>
static cudaError_t launch_mp(const WgArgs& a, int dev, cudaStream_t stream) {
    using S = WgShape<MP, Q4>;
    const int which = (MP == 16 ? 0 : (MP == 32 ? 1 : 2)) + (Q4 ? 3 : 0);
    if (!g_wg_attr[which][dev]) {
        const cudaError_t e =
            cudaFuncSetAttribute(wg_gemm_kernel<MP, Q4>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM);
        if (e != cudaSuccess) return e;
        g_wg_attr[which][dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)a.G);
    cfg.blockDim = dim3(S::THREADS);
    cfg.dynamicSmemBytes = S::SMEM;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, wg_gemm_kernel<MP, Q4>, a);
}

cudaError_t launch_wg_gemm(const WgGemm& g, cudaStream_t stream) {
    if (g.M <= 0) return cudaSuccess;
    if (g.M > WG_MAX_M) return cudaErrorInvalidValue;
    if (g.q4 && g.K % WG_K != 0) return cudaErrorInvalidValue;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    WgArgs a;
    a.tiles = g.tiles;
    a.x = g.x;
    a.ldx = g.ldx;
    a.y = g.y;
    a.ldy = g.ldy;
    a.M = g.M;
    a.N = g.N;
    a.K = g.K;
    a.NRG = (g.N + 7) / 8;
    a.KT = (g.K + WG_K - 1) / WG_K;
    // Slabs of at most 16 row groups.  With >= 8 row groups per SM every CTA gets whole slabs (as many
    // as the others); otherwise slabs are full 128-row MMAs and the k range is split across CTAs.
    a.NS = wg_num_slabs(a.NRG, g.n_sm);
    if ((long long)a.NS * a.KT * (g.n_sm + 1) >= (1LL << 31)) return cudaErrorInvalidValue;  // 32-bit unit math
    a.U = a.NS * a.KT;
    a.G = (int)(a.U < g.n_sm ? a.U : g.n_sm);
    a.rot = (a.NS % a.G == 0) ? 1 : 0;  // whole slabs per CTA: no run splits a slab's k range
    a.ws = g.ws;
    a.cnt = g.cnt;
    a.err = g.err;
    if (g.q4) {
        if (g.M <= 16) return launch_mp<16, true>(a, dev, stream);
        if (g.M <= 32) return launch_mp<32, true>(a, dev, stream);
        return launch_mp<64, true>(a, dev, stream);
    }
    if (g.M <= 16) return launch_mp<16, false>(a, dev, stream);
    if (g.M <= 32) return launch_mp<32, false>(a, dev, stream);
    return launch_mp<64, false>(a, dev, stream);
}

}  // namespace gdn
