// gdn_wq16.cu -- the MLX 4-bit projection (quantized_matmul with transpose, bits 4, group 64;
// qwen3_5.rs:572-586 in_proj_*, :668 out_proj on the reference's quantized checkpoint) for calls of at
// most 16 tokens (decode), on tcgen05 tensor cores with the weight operand in tensor memory.
//
// y[m][n] = bf16(sum_k x[m][k] * w[n][k]), w = bf16(scale * q + bias) (one rounding per weight, as MLX's
// quantized-matmul tile loader writes it), f32 accumulation.
//
// A decode call moves each 4-bit weight once for 2 * M flops, so the kernel is a stream over the codes.  The
// dequantized weight goes into TENSOR MEMORY (tcgen05.st from the registers of the thread that decoded it) and
// the MMA reads its A operand from there (tcgen05.mma ... [a_tmem]); shared memory holds only the codes and the
// tokens.  A 128 x 16 x 16 MMA occupies the tensor core ~44 cycles whatever its operands, so a k-tile of 64
// columns costs at least 4 x 44 cycles: the issuer is written so that its own work stays close to that.
//
// Layout: the 4-bit tiles of gdn_weight_tile_q4 (block (kt, rg) = 8 rows x one 64-column group, 288 B at
// (kt * NRG + rg) * 288: code word (c, r) at c*32 + r*4, 8 scales at 256, 8 biases at 272).  A CTA owns a
// slab of at most 16 row groups (128 rows, one M = 128 MMA; rows past the slab are never written) and a range
// of k-tiles; per k-tile its blocks are one contiguous bulk copy.  When the row groups allow >= 8 per SM (the
// in-projection) every CTA takes a whole slab over all k-tiles; otherwise (the out-projection) 128-row slabs
// are split along k and the last CTA of a slab to finish adds the f32 partials in split order (per-slab
// arrival counter, one release/acquire atomic per CTA; the partials of all splits are loaded at once by 512
// threads), so the output repeats bit for bit.
//
// The tokens arrive by TMA: one 64-column x 16-row box per k-tile from a tensor map over x (rows >= M read as
// zero), 128-byte swizzled, the B operand's K-major SWIZZLE_128B layout.  Per-thread cp.async of the same
// bytes stalled the loading warps for thousands of cycles behind the code stream.
//
// Roles (576 threads): warp 0 streams the slab's codes (all lanes issue copies; before the dependency wait: the
// weight does not depend on earlier kernels); warp 1 allocates tensor memory, waits for the producer of x,
// issues the token loads and then the MMAs (the whole warp runs the loop so every operand is warp-uniform; one
// elected lane issues); warps 2-17 decode: warp 2 + 4p + q takes TMEM lane quarter q (rows 32q..32q+31, one row
// per lane) and the k-tiles i with i % 4 == p, each k-tile into one of 15 A buffers of 32 TMEM columns (64 bf16
// per row); warps 2-5 store the accumulator.  Every wait is bounded (2 s; ERR_TIMEOUT, the CTA winds down).
#include <cuda.h>
#include <cuda_runtime.h>

#include "gdn_device.cuh"
#include "gdn_internal.h"
#include "gdn_ptx.cuh"
#include "gdn_umma.cuh"

namespace gdn {

namespace {

constexpr int Q16_DECODE_WARPS = 16;     // 4 per TMEM lane quarter, k-tiles round-robin
constexpr int Q16_THREADS = 32 * (2 + Q16_DECODE_WARPS);
constexpr int Q16_BLK = 288;               // 4-bit block: 8 rows x 64 columns (codes, scales, biases)
constexpr int Q16_MP = 16;                 // tokens (MMA N); rows >= M of the box are zero
constexpr int Q16_XT = Q16_MP * 128;       // one k-tile of tokens in shared memory: 16 rows x 128 B
constexpr int Q16_NA = 15;                 // A buffers in TMEM (32 columns each)
constexpr uint32_t Q16_TM_D = 0;           // accumulator [128 rows][16 tokens] f32: columns [0, 16)
constexpr uint32_t Q16_TM_A = 32;          // A buffers: columns [32, 512)
constexpr uint32_t Q16_TM_COLS = 512;
constexpr uint64_t Q16_WAIT_NS = 2000000000ull;
constexpr int Q16_MAX_KT = 64;             // k-tiles a CTA holds at once (one barrier each)
constexpr int Q16_MAX_SPLITS = 8;          // k-splits of a slab (the reduction loads one partial per split at once)
constexpr int Q16_BARS = (Q16_MAX_KT + 2 * Q16_NA + 2) * 8 + 16;
constexpr int Q16_SMEM_MAX = 220 * 1024;

struct Q16Args {
    CUtensorMap tmx;      // x [M][K] bf16, box 64 x 16, SWIZZLE_128B
    const uint8_t* tiles;
    uint16_t* y;
    long long ldy;
    int M, N;
    int NRG, KT;          // row groups, k-tiles
    int NS, splits, ktc;  // slabs, k splits per slab, k-tiles per split
    int wbytes;           // shared-memory bytes of one k-tile's codes (nrg_max * 288)
    int xoff, boff;       // shared-memory offsets: tokens (1024-aligned), barriers
    float* ws;            // [NS][splits][128][16] f32 partial sums (splits > 1)
    int* cnt;             // [NS] arrival counters (zero between launches)
    int* err;
};

__device__ __forceinline__ uint32_t q16_bf16x2_fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.bf16x2 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// 32 consecutive 32-bit TMEM columns of this thread's lane (warp-collective).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
        "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
        "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}

__global__ void __launch_bounds__(Q16_THREADS, 1) gdn_wq16_kernel(const __grid_constant__ Q16Args a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int slab = (int)blockIdx.x / a.splits, split = (int)blockIdx.x - slab * a.splits;
    const int rg0 = (int)(((long long)slab * a.NRG) / a.NS), rg1 = (int)(((long long)(slab + 1) * a.NRG) / a.NS);
    const int nrg = rg1 - rg0;
    const int kt0 = split * a.ktc;
    const int nkt = (a.KT - kt0) < a.ktc ? (a.KT - kt0) : a.ktc;
    uint8_t* s_w = smem;                                      // [nkt][wbytes] codes
    uint8_t* s_x = smem + a.xoff;                             // [nkt][16 rows][128 B] tokens, 128-byte swizzled
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + a.boff);
    uint64_t* wfull = bars;                                   // [Q16_MAX_KT] codes of k-tile i landed
    uint64_t* afull = wfull + Q16_MAX_KT;                     // [NA] A buffer written (4 warps)
    uint64_t* afree = afull + Q16_NA;                         // [NA] A buffer read by its MMAs
    uint64_t* xfull = afree + Q16_NA;                         // tokens landed (tx bytes)
    uint64_t* dfull = xfull + 1;                              // accumulator complete
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dfull + 1);
    volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* s_last = s_abort + 1;

    if (tid == 0) {
        for (int i = 0; i < Q16_MAX_KT; ++i) mbar_init(wfull + i, 1);
        for (int i = 0; i < Q16_NA; ++i) {
            mbar_init(afull + i, 4);           // one arrival per decoding warp
            mbar_init(afree + i, 1);
        }
        mbar_init(xfull, 1);
        mbar_init(dfull, 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, Q16_TM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // The next kernel may launch once every CTA got here and run its own pre-wait part; it waits for this grid
    // to complete before it reads y, and reads y with coherent loads (TMA, cp.async.cg, __ldcg or plain loads):
    // the non-coherent path (__ldg) returned stale data to kernels released early.
    pdl_launch_dependents();

    if (warp == 0) {
        // ---- codes of the slab's k-tiles (static weight: before the dependency wait), one copy per k-tile,
        // issued side by side from all 32 lanes (one thread's bulk copies are accepted one at a time)
        const uint32_t bytes = (uint32_t)nrg * Q16_BLK;
        for (int i = lane; i < nkt; i += 32) {
            mbar_arrive_expect_tx(wfull + i, bytes);
            bulk_g2s(s_w + (size_t)i * a.wbytes, a.tiles + ((size_t)(kt0 + i) * a.NRG + rg0) * Q16_BLK, bytes,
                     wfull + i);
        }
    } else if (warp == 1) {
        // ---- tokens: after the producer of x, one TMA box per k-tile from the lanes side by side
        pdl_wait();
        if (lane == 0) mbar_arrive_expect_tx(xfull, (uint32_t)(nkt * Q16_XT));
        __syncwarp();
        for (int i = lane; i < nkt; i += 32) tma_load_2d(s_x + (size_t)i * Q16_XT, &a.tmx, (kt0 + i) * 64, 0, xfull);

        // ---- MMA issuer: the whole warp runs the loop, so every operand is warp-uniform, and one elected lane
        // issues; the loop is unrolled over the A-buffer ring, so TMEM addresses and descriptor offsets are
        // constants (a descriptor recomputed per MMA from a loop counter costs the issuer ~60 cycles per MMA)
        {
            const uint32_t idesc = umma_idesc_bf16(128, Q16_MP);
            bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(xfull, 0, Q16_WAIT_NS));
            uint64_t bdi = umma_desc_sw128(smem_u32(s_x));   // k-tile i0, first k-step
            uint32_t par = 0;
            for (int i0 = 0; ok && i0 < nkt; i0 += Q16_NA) {
#pragma unroll
                for (int b = 0; b < Q16_NA; ++b) {
                    if (ok && i0 + b < nkt) {
                        ok = __all_sync(0xffffffffu, mbar_wait_bounded(afull + b, par, Q16_WAIT_NS));
                        if (ok) {
                            tc_fence_after();
                            if (elect_one()) {
#pragma unroll
                                for (int s = 0; s < 4; ++s)
                                    umma_bf16_ta(tmem + Q16_TM_D, tmem + Q16_TM_A + b * 32 + s * 8,
                                                 bdi + (uint64_t)((b * Q16_XT + s * 32) >> 4), idesc,
                                                 (i0 + b + s) != 0);
                                umma_commit(afree + b);
                            }
                            __syncwarp();
                        }
                    }
                }
                par ^= 1u;
                bdi += (uint64_t)((Q16_NA * Q16_XT) >> 4);
            }
            if (!ok && lane == 0) {
                atomicOr(a.err, ERR_TIMEOUT);
                *s_abort = 1;
            }
            // dfull completes when every MMA issued above has: the epilogue reads the accumulator after it,
            // and after a timeout this warp waits for it so no MMA is in flight when the CTA ends
            if (elect_one()) umma_commit(dfull);
            __syncwarp();
            if (!ok) mbar_wait_bounded(dfull, 0, Q16_WAIT_NS);
        }
    } else {
        // ---- decode: quarter qd (rows 32 qd + lane), k-tiles i with i % 4 == par
        const int dw = warp - 2, qd = dw & 3, par = dw >> 2;
        const int r = 32 * qd + lane;                          // row within the slab
        const bool row_ok = r < nrg * 8;
        const int rg = r >> 3, r8 = r & 7;
        const uint32_t ta = tmem + ((uint32_t)(qd * 32) << 16) + Q16_TM_A;
        bool ok = true;
        for (int i = par; i < nkt; i += Q16_DECODE_WARPS / 4) {
            const int b = i % Q16_NA;
            bool w_ok = true;
            if (i >= Q16_NA) w_ok = mbar_wait_bounded(afree + b, (uint32_t)((i - Q16_NA) / Q16_NA) & 1u, Q16_WAIT_NS);
            w_ok = w_ok && mbar_wait_bounded(wfull + i, 0, Q16_WAIT_NS);
            if (!w_ok) { ok = false; break; }
            tc_fence_after();
            uint32_t v[32];
            if (row_ok) {
                const uint8_t* blk = s_w + (size_t)i * a.wbytes + rg * Q16_BLK;
                const uint16_t s1 = *reinterpret_cast<const uint16_t*>(blk + 256 + 2 * r8);
                const uint16_t b1 = *reinterpret_cast<const uint16_t*>(blk + 272 + 2 * r8);
                const uint32_t s2 = (uint32_t)s1 | ((uint32_t)s1 << 16), b2 = (uint32_t)b1 | ((uint32_t)b1 << 16);
                const uint32_t one2 = 0x3F803F80u, m128 = 0xC300C300u;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const uint32_t w = *reinterpret_cast<const uint32_t*>(blk + c * 32 + r8 * 4);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        // (nib | 0x4300) is the bf16 of 128 + q exactly; -128 is exact; then scale * q + bias
                        // rounded once: columns 8c + 2j, 8c + 2j + 1
                        const uint32_t t = ((w >> (4 * j)) & 0x000F000Fu) | 0x43004300u;
                        v[c * 4 + j] = q16_bf16x2_fma(q16_bf16x2_fma(t, one2, m128), s2, b2);
                    }
                }
            } else {
#pragma unroll
                for (int c = 0; c < 32; ++c) v[c] = 0u;
            }
            tmem_st32(ta + b * 32, v);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(afull + b);
        }
        if (!ok) {
            atomicOr(a.err, ERR_TIMEOUT);
            *s_abort = 1;
        }
        // ---- epilogue (warps 2-5): the accumulator rows of this quarter
        if (par == 0) {
            const bool d_ok = ok && mbar_wait_bounded(dfull, 0, Q16_WAIT_NS) && !*s_abort;
            tc_fence_after();
            float d[16];
#pragma unroll
            for (int m = 0; m < 16; ++m) d[m] = 0.f;
            if (d_ok) tmem_ld16(tmem + ((uint32_t)(qd * 32) << 16) + Q16_TM_D, d);
            const int n = rg0 * 8 + r;
            if (a.splits == 1) {
                if (d_ok && row_ok && n < a.N) {
#pragma unroll
                    for (int m = 0; m < Q16_MP; ++m)
                        if (m < a.M) a.y[(long long)m * a.ldy + n] = f2bf(d[m]);
                }
            } else {
                float* part = a.ws + (((size_t)slab * a.splits + split) * 128 + r) * Q16_MP;
#pragma unroll
                for (int m = 0; m < 16; m += 4)
                    __stcg(reinterpret_cast<float4*>(part + m), make_float4(d[m], d[m + 1], d[m + 2], d[m + 3]));
            }
        }
    }

    // ---- k-split partials: the last CTA of the slab to arrive adds all of them in split order.  The CTA barrier
    // orders this CTA's partial stores before thread 0's release; its acquire, then the barrier, order the
    // other CTAs' partials before the loads (which bypass L1).
    if (a.splits > 1) {
        __syncthreads();
        if (tid == 0) {
            int prev;
            asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;\n" : "=r"(prev) : "l"(a.cnt + slab) : "memory");
            *s_last = prev == a.splits - 1;
        }
        __syncthreads();
        if (*s_last) {
            if (tid < 128 * Q16_MP / 4) {
                const int r = tid >> 2, m0 = (tid & 3) * 4;
                const float* p = a.ws + ((size_t)slab * a.splits * 128 + r) * Q16_MP + m0;
                float4 v[Q16_MAX_SPLITS];
#pragma unroll
                for (int sp = 0; sp < Q16_MAX_SPLITS; ++sp)
                    if (sp < a.splits) v[sp] = __ldcg(reinterpret_cast<const float4*>(p + (size_t)sp * 128 * Q16_MP));
                float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int sp = 0; sp < Q16_MAX_SPLITS; ++sp)
                    if (sp < a.splits) {
                        acc.x += v[sp].x; acc.y += v[sp].y; acc.z += v[sp].z; acc.w += v[sp].w;
                    }
                const int n = rg0 * 8 + r;
                if (!*s_abort && r < nrg * 8 && n < a.N) {
                    const float o[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        if (m0 + j < a.M) a.y[(long long)(m0 + j) * a.ldy + n] = f2bf(o[j]);
                }
            }
            if (tid == 0) a.cnt[slab] = 0;   // zero at rest for the next launch
        }
    }

    // no code copy may land after the CTA ends: every k-tile's copy was waited for by its decoder unless a
    // wait gave up, in which case thread 0 waits (bounded) for the rest; the same for the token boxes
    __syncthreads();
    if (tid == 0 && *s_abort) {
        for (int i = 0; i < nkt; ++i) mbar_wait_bounded(wfull + i, 0, Q16_WAIT_NS);
        mbar_wait_bounded(xfull, 0, Q16_WAIT_NS);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, Q16_TM_COLS);
}

// ------------------------------------------------------------------ bf16 tiles, at most 16 tokens
// The same stream for a bf16 weight in the tiled layout of gdn_weight_tile (block (kt, rg) = 8 rows x 64 columns,
// 1 KB at (kt * NRG + rg) * 1024, K-major core matrices: chunk c of row r at c*128 + r*16).  A slab's k-tile is
// nrg consecutive blocks, i.e. a [8 nrg][64] operand tile in exactly the layout the MMA reads from shared memory
// (K-major, no swizzle: LBO 128 B, SBO 1 KB), so the weight goes by bulk copy straight into a ring of stages and
// the MMA takes its A operand from there (rows past the slab read whatever follows the stage; their accumulator
// rows are never stored).  Roles (192 threads): warp 0 streams the k-tiles into the ring (4 lanes side by side,
// each owning every 4th stage; before the dependency wait), warp 1 loads the tokens by TMA after the wait and
// issues 4 MMAs per k-tile, releasing the stage by tcgen05.commit; warps 2-5 store the accumulator (or the
// k-split partials, reduced as in gdn_wq16_kernel).  Every wait is bounded.
constexpr int B16_THREADS = 32 * 6;
constexpr int B16_BLK = 1024;
constexpr int B16_MAX_STAGES = 16;
constexpr int B16_LANES = 4;               // issuing lanes of warp 0 (stages are a multiple of it)
constexpr int B16_BARS = (2 * B16_MAX_STAGES + 2) * 8 + 16;

struct B16Args {
    CUtensorMap tmx;      // x [M][K] bf16, box 64 x 16, SWIZZLE_128B
    const uint8_t* tiles;
    uint16_t* y;
    long long ldy;
    int M, N;
    int NRG, KT;
    int NS, splits, ktc;
    int stages, sbytes;   // ring depth, bytes per stage (nrg_max KB)
    int xoff, boff;       // shared-memory offsets: tokens (1024-aligned), barriers
    float* ws;
    int* cnt;
    int* err;
};

__global__ void __launch_bounds__(B16_THREADS, 1) gdn_wb16_kernel(const __grid_constant__ B16Args a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int slab = (int)blockIdx.x / a.splits, split = (int)blockIdx.x - slab * a.splits;
    const int rg0 = (int)(((long long)slab * a.NRG) / a.NS), rg1 = (int)(((long long)(slab + 1) * a.NRG) / a.NS);
    const int nrg = rg1 - rg0;
    const int kt0 = split * a.ktc;
    const int nkt = (a.KT - kt0) < a.ktc ? (a.KT - kt0) : a.ktc;
    const int S = a.stages;
    uint8_t* s_w = smem;                                      // [S][sbytes] weight ring
    uint8_t* s_x = smem + a.xoff;                             // [nkt][16 rows][128 B] tokens, 128-byte swizzled
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + a.boff);
    uint64_t* sfull = bars;                                   // [S] stage landed
    uint64_t* sfree = sfull + B16_MAX_STAGES;                 // [S] stage read by its MMAs
    uint64_t* xfull = sfree + B16_MAX_STAGES;
    uint64_t* dfull = xfull + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dfull + 1);
    volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* s_last = s_abort + 1;

    if (tid == 0) {
        for (int i = 0; i < B16_MAX_STAGES; ++i) {
            mbar_init(sfull + i, 1);
            mbar_init(sfree + i, 1);
        }
        mbar_init(xfull, 1);
        mbar_init(dfull, 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, 32);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // the next kernel may launch once every CTA got here (it reads y only after its wait, with coherent loads)
    pdl_launch_dependents();

    if (warp == 0) {
        // ---- weight k-tiles into the ring (static weight: before the dependency wait); lane j < 4 owns the
        // stages s = j mod 4 and waits for each one's previous MMAs before reusing it (issuing from 4 lanes side
        // by side: one thread's bulk copies are accepted one at a time; a converged wait for 4 stages at a time,
        // then 4 copies in one instruction, measured 14.0 against 12.9 us for the in-projection)
        const uint32_t bytes = (uint32_t)nrg * B16_BLK;
        bool ok = true;
        if (lane < B16_LANES) {
            for (int i = lane; i < nkt; i += B16_LANES) {
                const int st = i % S, use = i / S;
                if (use > 0 && !mbar_wait_bounded(sfree + st, (uint32_t)(use - 1) & 1u, Q16_WAIT_NS)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(sfull + st, bytes);
                bulk_g2s(s_w + (size_t)st * a.sbytes, a.tiles + ((size_t)(kt0 + i) * a.NRG + rg0) * B16_BLK, bytes,
                         sfull + st);
            }
        }
        if (!ok) {
            atomicOr(a.err, ERR_TIMEOUT);
            *s_abort = 1;
        }
    } else if (warp == 1) {
        // ---- tokens after the producer of x, one TMA box per k-tile from the lanes side by side
        pdl_wait();
        if (lane == 0) mbar_arrive_expect_tx(xfull, (uint32_t)(nkt * Q16_XT));
        __syncwarp();
        for (int i = lane; i < nkt; i += 32) tma_load_2d(s_x + (size_t)i * Q16_XT, &a.tmx, (kt0 + i) * 64, 0, xfull);
        // ---- MMA issuer (the whole warp runs the loop; one elected lane issues)
        {
            const uint32_t idesc = umma_idesc_bf16(128, Q16_MP);
            bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(xfull, 0, Q16_WAIT_NS));
            const uint64_t ad0 = umma_desc(smem_u32(s_w), 64, 0);
            const uint64_t bd0 = umma_desc_sw128(smem_u32(s_x));
            uint32_t par = 0;
            for (int i0 = 0; ok && i0 < nkt; i0 += S) {
                for (int b = 0; b < S; ++b) {
                    const int i = i0 + b;
                    if (!ok || i >= nkt) break;
                    ok = __all_sync(0xffffffffu, mbar_wait_bounded(sfull + b, par, Q16_WAIT_NS));
                    if (ok) {
                        tc_fence_after();
                        if (elect_one()) {
                            const uint64_t ad = ad0 + (uint64_t)(((uint32_t)b * (uint32_t)a.sbytes) >> 4);
                            const uint64_t bd = bd0 + (uint64_t)(((uint32_t)i * Q16_XT) >> 4);
#pragma unroll
                            for (int s = 0; s < 4; ++s)
                                umma_bf16(tmem, ad + (uint64_t)s * KSTEP_K, bd + (uint64_t)((s * 32) >> 4), idesc,
                                          (i + s) != 0);
                            umma_commit(sfree + b);
                        }
                        __syncwarp();
                    }
                }
                par ^= 1u;
            }
            if (!ok && lane == 0) {
                atomicOr(a.err, ERR_TIMEOUT);
                *s_abort = 1;
            }
            if (elect_one()) umma_commit(dfull);
            __syncwarp();
            if (!ok) mbar_wait_bounded(dfull, 0, Q16_WAIT_NS);
        }
    } else {
        // ---- epilogue (warps 2-5): the accumulator rows of the warp's TMEM lane quarter (warp index mod 4)
        const int qd = warp & 3;
        const int r = 32 * qd + lane;
        const bool row_ok = r < nrg * 8;
        const bool d_ok = mbar_wait_bounded(dfull, 0, Q16_WAIT_NS) && !*s_abort;
        tc_fence_after();
        float d[16];
#pragma unroll
        for (int m = 0; m < 16; ++m) d[m] = 0.f;
        if (d_ok) tmem_ld16(tmem + ((uint32_t)(qd * 32) << 16), d);
        if (!d_ok && lane == 0) {
            atomicOr(a.err, ERR_TIMEOUT);
            *s_abort = 1;
        }
        const int n = rg0 * 8 + r;
        if (a.splits == 1) {
            if (d_ok && row_ok && n < a.N) {
#pragma unroll
                for (int m = 0; m < Q16_MP; ++m)
                    if (m < a.M) a.y[(long long)m * a.ldy + n] = f2bf(d[m]);
            }
        } else {
            float* part = a.ws + (((size_t)slab * a.splits + split) * 128 + r) * Q16_MP;
#pragma unroll
            for (int m = 0; m < 16; m += 4)
                __stcg(reinterpret_cast<float4*>(part + m), make_float4(d[m], d[m + 1], d[m + 2], d[m + 3]));
        }
    }

    // ---- k-split partials: the last CTA of the slab to arrive adds all of them in split order (as in
    // gdn_wq16_kernel)
    if (a.splits > 1) {
        __syncthreads();
        if (tid == 0) {
            int prev;
            asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;\n" : "=r"(prev) : "l"(a.cnt + slab) : "memory");
            *s_last = prev == a.splits - 1;
        }
        __syncthreads();
        if (*s_last) {
            for (int q = tid; q < 128 * Q16_MP / 4; q += B16_THREADS) {
                const int r = q >> 2, m0 = (q & 3) * 4;
                const float* p = a.ws + ((size_t)slab * a.splits * 128 + r) * Q16_MP + m0;
                float4 v[Q16_MAX_SPLITS];
#pragma unroll
                for (int sp = 0; sp < Q16_MAX_SPLITS; ++sp)
                    if (sp < a.splits) v[sp] = __ldcg(reinterpret_cast<const float4*>(p + (size_t)sp * 128 * Q16_MP));
                float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int sp = 0; sp < Q16_MAX_SPLITS; ++sp)
                    if (sp < a.splits) {
                        acc.x += v[sp].x; acc.y += v[sp].y; acc.z += v[sp].z; acc.w += v[sp].w;
                    }
                const int n = rg0 * 8 + r;
                if (!*s_abort && r < nrg * 8 && n < a.N) {
                    const float o[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        if (m0 + j < a.M) a.y[(long long)(m0 + j) * a.ldy + n] = f2bf(o[j]);
                }
            }
            if (tid == 0) a.cnt[slab] = 0;   // zero at rest for the next launch
        }
    }

    // no copy may land after the CTA ends: after a wait gave up, thread 0 waits (bounded) for every stage's last
    // copy and for the token boxes
    __syncthreads();
    if (tid == 0 && *s_abort) {
        for (int i = (nkt > S ? nkt - S : 0); i < nkt; ++i)
            mbar_wait_bounded(sfull + i % S, (uint32_t)(i / S) & 1u, Q16_WAIT_NS);
        mbar_wait_bounded(xfull, 0, Q16_WAIT_NS);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, 32);
}

static bool g_b16_attr[64] = {};

static bool g_q16_attr[64] = {};

// The tensor map of the last few token matrices (the stack reuses its buffers from step to step).
struct Q16Map {
    CUtensorMap map;
    const void* x;
    long long ldx;
    int M, K;
};
thread_local Q16Map g_q16_maps[8];
thread_local int g_q16_next = 0;

bool token_map(CUtensorMap* out, const uint16_t* x, long long ldx, int M, int K) {
    for (const Q16Map& m : g_q16_maps)
        if (m.x == x && m.ldx == ldx && m.M == M && m.K == K) {
            *out = m.map;
            return true;
        }
    Q16Map& slot = g_q16_maps[g_q16_next];
    if (!tmap_bf16_2d_sw128(&slot.map, x, (uint64_t)K, (uint64_t)M, (uint64_t)ldx * 2, 64, Q16_MP)) return false;
    slot.x = x;
    slot.ldx = ldx;
    slot.M = M;
    slot.K = K;
    g_q16_next = (g_q16_next + 1) % 8;
    *out = slot.map;
    return true;
}

}  // namespace

// Whether gdn_wq16_kernel serves a call: at most 16 tokens and K a multiple of 64 (x rows must also start on
// 16-byte boundaries, which every caller checks).  launch_wq16 answers cudaErrorNotSupported when K needs more
// k-splits than the reduction takes; the caller then streams the weight with gdn_wgemm's kernel.
bool wq16_supported(int M, int N, int K) { return M >= 1 && M <= Q16_MP && K % 64 == 0 && N > 0; }

cudaError_t launch_wq16(const WgGemm& g, cudaStream_t stream) {
    if (!wq16_supported(g.M, g.N, g.K) || ((uintptr_t)g.x & 15u) != 0 || g.ldx % 8 != 0 || g.ldx < g.K)
        return cudaErrorInvalidValue;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    Q16Args a;
    if (!token_map(&a.tmx, g.x, g.ldx, g.M, g.K)) return cudaErrorInvalidValue;
    a.tiles = g.tiles;
    a.y = g.y;
    a.ldy = g.ldy;
    a.M = g.M;
    a.N = g.N;
    a.NRG = (g.N + 7) / 8;
    a.KT = g.K / 64;
    if (a.NRG >= 8 * g.n_sm) {
        // whole slabs: one per SM when they stay within 16 row groups
        a.NS = g.n_sm * ((a.NRG + 16 * g.n_sm - 1) / (16 * g.n_sm));
        a.splits = 1;
    } else {
        // 128-row slabs split along k so that the CTAs cover the SMs
        a.NS = (a.NRG + 15) / 16;
        a.splits = g.n_sm / a.NS > 1 ? g.n_sm / a.NS : 1;
        if (a.splits > Q16_MAX_SPLITS) a.splits = Q16_MAX_SPLITS;
        if (a.splits > a.KT) a.splits = a.KT;
    }
    const int nrg_max = (a.NRG + a.NS - 1) / a.NS;
    a.wbytes = nrg_max * Q16_BLK;
    auto layout = [&](int ktc) {
        a.ktc = ktc;
        a.xoff = ((ktc * a.wbytes + 1023) / 1024) * 1024;
        a.boff = a.xoff + ktc * Q16_XT;
        return (size_t)a.boff + Q16_BARS;
    };
    size_t smem = layout((a.KT + a.splits - 1) / a.splits);
    // more splits while a split's codes and tokens exceed the shared-memory budget or the barrier count
    while (smem > (size_t)Q16_SMEM_MAX || a.ktc > Q16_MAX_KT) {
        if (++a.splits > Q16_MAX_SPLITS) return cudaErrorNotSupported;   // K too long for the reduction
        smem = layout((a.KT + a.splits - 1) / a.splits);
    }
    a.splits = (a.KT + a.ktc - 1) / a.ktc;   // no empty split
    if (a.NS * a.splits > 65535) return cudaErrorInvalidValue;
    if (a.splits > 1 && ((long long)a.NS * a.splits * 128 * Q16_MP > wg_workspace_floats(g.n_sm) || a.NS > 4096))
        return cudaErrorNotSupported;   // partials or arrival counters beyond the pool's workspace
    a.ws = g.ws;
    a.cnt = g.cnt;
    a.err = g.err;
    if (!g_q16_attr[dev]) {
        e = cudaFuncSetAttribute(gdn_wq16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        g_q16_attr[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(a.NS * a.splits));
    cfg.blockDim = dim3(Q16_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gdn_wq16_kernel, a);
}

bool wb16_supported(int M, int N, int K) { return M >= 1 && M <= Q16_MP && K % 64 == 0 && N > 0; }

cudaError_t launch_wb16(const WgGemm& g, cudaStream_t stream) {
    if (!wb16_supported(g.M, g.N, g.K) || g.q4 || ((uintptr_t)g.x & 15u) != 0 || g.ldx % 8 != 0 || g.ldx < g.K ||
        ((uintptr_t)g.tiles & 15u) != 0)
        return cudaErrorInvalidValue;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    B16Args a;
    if (!token_map(&a.tmx, g.x, g.ldx, g.M, g.K)) return cudaErrorInvalidValue;
    a.tiles = g.tiles;
    a.y = g.y;
    a.ldy = g.ldy;
    a.M = g.M;
    a.N = g.N;
    a.NRG = (g.N + 7) / 8;
    a.KT = g.K / 64;
    if (a.NRG >= 8 * g.n_sm) {
        a.NS = g.n_sm * ((a.NRG + 16 * g.n_sm - 1) / (16 * g.n_sm));   // whole slabs of <= 16 row groups
        a.splits = 1;
    } else {
        a.NS = (a.NRG + 15) / 16;                                      // 128-row slabs split along k
        a.splits = g.n_sm / a.NS > 1 ? g.n_sm / a.NS : 1;
        if (a.splits > Q16_MAX_SPLITS) a.splits = Q16_MAX_SPLITS;
        if (a.splits > a.KT) a.splits = a.KT;
    }
    a.ktc = (a.KT + a.splits - 1) / a.splits;
    a.splits = (a.KT + a.ktc - 1) / a.ktc;   // no empty split
    const int nrg_max = (a.NRG + a.NS - 1) / a.NS;
    a.sbytes = nrg_max * B16_BLK;
    // stages: a multiple of the issuing lanes, at most the split's k-tiles (rounded up) and the budget; the MMA of
    // the last stage reads 16 KB from its start, so the tokens start no earlier than that
    const size_t xbytes = (size_t)a.ktc * Q16_XT;
    int st = B16_MAX_STAGES;
    auto layout = [&](int stages) {
        a.stages = stages;
        size_t x0 = (size_t)stages * a.sbytes;
        const size_t reach = (size_t)(stages - 1) * a.sbytes + 16 * B16_BLK;
        if (x0 < reach) x0 = reach;
        a.xoff = (int)(((x0 + 1023) / 1024) * 1024);
        a.boff = a.xoff + (int)xbytes;
        return (size_t)a.boff + B16_BARS;
    };
    const int need = ((a.ktc + B16_LANES - 1) / B16_LANES) * B16_LANES;
    if (st > need) st = need;
    size_t smem = layout(st);
    while (smem > (size_t)Q16_SMEM_MAX && st > B16_LANES) smem = layout(st -= B16_LANES);
    if (smem > (size_t)Q16_SMEM_MAX) return cudaErrorNotSupported;   // the tokens of a split do not fit
    if (a.NS * a.splits > 65535) return cudaErrorInvalidValue;
    if (a.splits > 1 && ((long long)a.NS * a.splits * 128 * Q16_MP > wg_workspace_floats(g.n_sm) || a.NS > 4096))
        return cudaErrorNotSupported;
    a.ws = g.ws;
    a.cnt = g.cnt;
    a.err = g.err;
    if (!g_b16_attr[dev]) {
        e = cudaFuncSetAttribute(gdn_wb16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        g_b16_attr[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(a.NS * a.splits));
    cfg.blockDim = dim3(B16_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gdn_wb16_kernel, a);
}

}  // namespace gdn
