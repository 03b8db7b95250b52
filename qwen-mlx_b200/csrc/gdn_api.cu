// gdn_api.cu -- C ABI of include/gdn.h: slot-indexed state pool, routing
// validation, error reporting and the launch of the fused kernels.
#include <cstdarg>
#include <cstdio>
#include <cstdint>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "gdn.h"
#include "gdn_internal.h"

#define GDN_VERSION_STRING "gdn-b200 0.1.0 (sm_100a)"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int ok() {
    g_last_error.clear();
    return GDN_OK;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(GDN_E_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// Switches to `dev` for the lifetime of the guard and restores the caller's device.
struct DeviceGuard {
    int prev = -1;
    cudaError_t status = cudaSuccess;
    explicit DeviceGuard(int dev) {
        status = cudaGetDevice(&prev);
        if (status == cudaSuccess && prev != dev) status = cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

}  // namespace

namespace gdn {
int record_error(int code, const char* msg) { return fail(code, "%s", msg); }
int record_ok() { return ok(); }
}  // namespace gdn

struct gdn_pool {
    int device;
    gdn_config cfg;
    int32_t n_slots;
    int32_t D;
    size_t rec_slot_elems;   // Hv*dv*dk
    size_t conv_slot_elems;  // (K-1)*D
    float* rec;              // [n_layers][n_slots][Hv][dv][dk]
    uint16_t* conv;          // [n_layers][n_slots][K-1][D]
    int32_t* err;            // device words: [0] error flags, [1] chunked-kernel work ticket
    gdn::GemmCtx* gemm;      // cuBLASLt handle for the projections
    void* gemm_ws;           // its workspace
    int n_sm;                // multiprocessors of the pool's device
    int* wg_cnt;             // weight-streaming GEMM: per-row-tile arrival counters [kWgMaxTiles] (zero at rest)
    float* wg_ws;            // weight-streaming GEMM: partial sums [wg_workspace_floats(n_sm)]
    uint16_t* wdq;           // one projection weight expanded from 4-bit tiles to bf16 [wdq_elems]
    size_t wdq_elems;
    uint16_t* proj;          // scratch [rec_cap][D + Hv*dv + 2*Hv]: projection outputs
    uint16_t* gated;         // scratch [rec_cap][Hv*dv]: layer-step output (out_proj input)
    uint16_t* hn;            // scratch [rec_cap][hidden]: normed stack input
    uint16_t* mix;           // scratch [rec_cap][hidden]: mixer output
    uint8_t* recs;           // scratch: per-(v-head, token) records of the layer step [Hv][rec_cap][REC_BYTES]
    long long rec_cap;       // tokens per call the scratch holds
    uint8_t* wy_tiles;       // scratch: chunked-prefill tile sets [wy_cap][Hv][WY_TILESET_BYTES], then the chunk
                             // table [wy_cap] int2
    long long wy_cap;        // chunks the tile scratch holds (rec_cap / 32 + 1: segments of >= 32 tokens)
    int32_t* wy_cb;          // chunked-prefill plan: chunk prefix per sequence [65536] ...
    int32_t* wy_plan;        // ... and the chunk count, sequence count and ranking [WY_PLAN_INTS]
};

static constexpr int kDeviceWords = 16;  // one 64-byte allocation
static constexpr int kWgMaxTiles = 4096;  // arrival counters: weight-streaming GEMMs of up to 4096 row slabs

static long long proj_ld(const gdn_pool* p) { return (long long)p->D + p->cfg.n_v_heads * 128 + 2 * p->cfg.n_v_heads; }

static long long wy_chunks_for(long long tokens) { return tokens / gdn::WY_MIN_T + 1; }

static size_t wy_tile_bytes(const gdn_pool* p, long long tokens) {
    return (size_t)wy_chunks_for(tokens) * (p->cfg.n_v_heads * (size_t)gdn::WY_TILESET_BYTES + sizeof(int2));
}

static int reserve_records(gdn_pool* p, long long tokens) {
    if (tokens <= p->rec_cap) return GDN_OK;
    const size_t rec_bytes = (size_t)tokens * p->cfg.n_v_heads * gdn::REC_BYTES;
    const size_t proj_bytes = (size_t)tokens * proj_ld(p) * 2;
    const size_t gated_bytes = (size_t)tokens * p->cfg.n_v_heads * 128 * 2;
    const size_t hid_bytes = (size_t)tokens * p->cfg.hidden * 2;
    const size_t tile_bytes = wy_tile_bytes(p, tokens);
    uint8_t *buf = nullptr, *tiles = nullptr;
    uint16_t *proj = nullptr, *gated = nullptr, *hn = nullptr, *mix = nullptr;
    cudaError_t e = cudaMalloc(&buf, rec_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&proj, proj_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&gated, gated_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&hn, hid_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&mix, hid_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&tiles, tile_bytes);
    if (e != cudaSuccess) {
        cudaFree(buf); cudaFree(proj); cudaFree(gated); cudaFree(hn); cudaFree(mix); cudaFree(tiles);
        return fail(GDN_E_NOMEM, "cudaMalloc of step scratch for %lld tokens failed: %s", tokens, cudaGetErrorString(e));
    }
    if (p->recs) {
        cudaDeviceSynchronize();
        cudaFree(p->recs); cudaFree(p->proj); cudaFree(p->gated); cudaFree(p->hn); cudaFree(p->mix);
        cudaFree(p->wy_tiles);
    }
    p->recs = buf;
    p->proj = proj; p->gated = gated; p->hn = hn; p->mix = mix;
    p->wy_tiles = tiles;
    p->wy_cap = wy_chunks_for(tokens);
    p->rec_cap = tokens;
    return GDN_OK;
}

static int check_cfg(const gdn_config* c) {
    if (!c) return fail(GDN_E_INVALID, "config is NULL");
    if (c->n_k_heads <= 0 || c->n_v_heads <= 0 || c->n_layers <= 0 || c->hidden <= 0)
        return fail(GDN_E_INVALID, "config has a non-positive size (hk=%d hv=%d layers=%d hidden=%d)", c->n_k_heads,
                    c->n_v_heads, c->n_layers, c->hidden);
    if (c->n_v_heads % c->n_k_heads)
        return fail(GDN_E_INVALID, "n_v_heads (%d) must be a multiple of n_k_heads (%d)", c->n_v_heads, c->n_k_heads);
    if (c->head_k_dim != gdn::DK_ABI || c->head_v_dim != gdn::DV_ABI)
        return fail(GDN_E_UNSUPPORTED, "only head_k_dim = head_v_dim = 128 is specialised (got %d, %d)",
                    c->head_k_dim, c->head_v_dim);
    if (c->conv_kernel != 4) return fail(GDN_E_UNSUPPORTED, "only conv_kernel = 4 is specialised (got %d)", c->conv_kernel);
    if (c->n_v_heads / c->n_k_heads > 8)
        return fail(GDN_E_UNSUPPORTED, "n_v_heads / n_k_heads = %d exceeds the portable cluster size 8",
                    c->n_v_heads / c->n_k_heads);
    if (!(c->rms_norm_eps >= 0.0f)) return fail(GDN_E_INVALID, "rms_norm_eps must be >= 0");
    return GDN_OK;
}

extern "C" {

const char* gdn_last_error(void) { return g_last_error.c_str(); }

const char* gdn_version(void) { return GDN_VERSION_STRING; }

int gdn_pool_create(int device, const gdn_config* cfg, int32_t n_slots, gdn_pool** out) {
    if (!out) return fail(GDN_E_INVALID, "out is NULL");
    *out = nullptr;
    int rc = check_cfg(cfg);
    if (rc) return rc;
    if (n_slots <= 0) return fail(GDN_E_INVALID, "n_slots must be positive (got %d)", n_slots);
    int ndev = 0;
    cudaError_t e = cudaGetDeviceCount(&ndev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
    if (device < 0 || device >= ndev) return fail(GDN_E_INVALID, "device %d out of range [0,%d)", device, ndev);
    DeviceGuard g(device);
    if (g.status != cudaSuccess) return cuda_fail(g.status, "cudaSetDevice");

    gdn_pool* p = new (std::nothrow) gdn_pool();
    if (!p) return fail(GDN_E_NOMEM, "host allocation failed");
    p->device = device;
    p->cfg = *cfg;
    p->n_slots = n_slots;
    p->D = 2 * cfg->n_k_heads * cfg->head_k_dim + cfg->n_v_heads * cfg->head_v_dim;
    p->rec_slot_elems = (size_t)cfg->n_v_heads * cfg->head_v_dim * cfg->head_k_dim;
    p->conv_slot_elems = (size_t)(cfg->conv_kernel - 1) * p->D;
    const size_t rec_bytes = sizeof(float) * p->rec_slot_elems * n_slots * cfg->n_layers;
    const size_t conv_bytes = sizeof(uint16_t) * p->conv_slot_elems * n_slots * cfg->n_layers;
    e = cudaMalloc(&p->rec, rec_bytes);
    if (e != cudaSuccess) {
        delete p;
        return fail(GDN_E_NOMEM, "cudaMalloc of %zu B of recurrent state failed: %s", rec_bytes, cudaGetErrorString(e));
    }
    e = cudaMalloc(&p->conv, conv_bytes);
    if (e != cudaSuccess) {
        cudaFree(p->rec);
        delete p;
        return fail(GDN_E_NOMEM, "cudaMalloc of %zu B of conv state failed: %s", conv_bytes, cudaGetErrorString(e));
    }
    e = cudaMalloc(&p->err, kDeviceWords * sizeof(int32_t));
    if (e != cudaSuccess) {
        cudaFree(p->rec);
        cudaFree(p->conv);
        delete p;
        return fail(GDN_E_NOMEM, "cudaMalloc of the error word failed: %s", cudaGetErrorString(e));
    }
    e = cudaMemset(p->rec, 0, rec_bytes);
    if (e == cudaSuccess) e = cudaMemset(p->conv, 0, conv_bytes);
    if (e == cudaSuccess) e = cudaMemset(p->err, 0, kDeviceWords * sizeof(int32_t));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(p->rec);
        cudaFree(p->conv);
        cudaFree(p->err);
        delete p;
        return cuda_fail(e, "zeroing the pool");
    }
    p->recs = nullptr;
    p->proj = p->gated = p->hn = p->mix = nullptr;
    p->wy_tiles = nullptr;
    p->wy_cap = 0;
    p->rec_cap = 0;
    p->wy_cb = nullptr;
    p->wy_plan = nullptr;
    e = cudaMalloc(&p->wy_cb, (65536 + gdn::WY_PLAN_INTS) * sizeof(int32_t));
    if (e != cudaSuccess) {
        cudaFree(p->rec);
        cudaFree(p->conv);
        cudaFree(p->err);
        delete p;
        return fail(GDN_E_NOMEM, "cudaMalloc of the prefill plan failed: %s", cudaGetErrorString(e));
    }
    p->wy_plan = p->wy_cb + 65536;
    p->gemm = nullptr;
    p->gemm_ws = nullptr;
    p->wg_cnt = nullptr;
    p->wg_ws = nullptr;
    p->wdq = nullptr;
    p->wdq_elems = 0;
    p->n_sm = 0;
    rc = reserve_records(p, n_slots > 1024 ? n_slots : 1024);
    if (rc == GDN_OK) {
        const size_t ws = 32u << 20;
        e = cudaMalloc(&p->gemm_ws, ws);
        if (e == cudaSuccess) p->gemm = gdn::gemm_create(p->gemm_ws, ws);
        if (e != cudaSuccess || !p->gemm) rc = fail(GDN_E_NOMEM, "cuBLASLt handle / workspace creation failed");
    }
    if (rc == GDN_OK) {
        e = cudaDeviceGetAttribute(&p->n_sm, cudaDevAttrMultiProcessorCount, device);
        if (e == cudaSuccess) e = cudaMalloc(&p->wg_cnt, kWgMaxTiles * sizeof(int));
        if (e == cudaSuccess) e = cudaMalloc(&p->wg_ws, gdn::wg_workspace_floats(p->n_sm) * sizeof(float));
        if (e == cudaSuccess) e = cudaMemset(p->wg_cnt, 0, kWgMaxTiles * sizeof(int));
        if (e == cudaSuccess) {
            const size_t in_w = (size_t)proj_ld(p) * p->cfg.hidden, out_w = (size_t)p->cfg.hidden * p->cfg.n_v_heads * 128;
            p->wdq_elems = in_w > out_w ? in_w : out_w;
            e = cudaMalloc(&p->wdq, p->wdq_elems * sizeof(uint16_t));
        }
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e != cudaSuccess) rc = fail(GDN_E_NOMEM, "projection GEMM workspace: %s", cudaGetErrorString(e));
    }
    if (rc) {
        cudaFree(p->rec);
        cudaFree(p->conv);
        cudaFree(p->err);
        cudaFree(p->recs); cudaFree(p->proj); cudaFree(p->gated); cudaFree(p->hn); cudaFree(p->mix);
        cudaFree(p->wy_tiles); cudaFree(p->wy_cb);
        cudaFree(p->gemm_ws);
        cudaFree(p->wg_cnt);
        cudaFree(p->wg_ws);
        cudaFree(p->wdq);
        gdn::gemm_destroy(p->gemm);
        delete p;
        return rc;
    }
    *out = p;
    return ok();
}

int gdn_pool_reserve_tokens(gdn_pool* p, int32_t max_tokens) {
    if (!p) return fail(GDN_E_INVALID, "pool is NULL");
    if (max_tokens < 0) return fail(GDN_E_INVALID, "max_tokens must be >= 0");
    DeviceGuard g(p->device);
    if (g.status != cudaSuccess) return cuda_fail(g.status, "cudaSetDevice");
    int rc = reserve_records(p, max_tokens);
    return rc ? rc : ok();
}

int gdn_pool_destroy(gdn_pool* p) {
    if (!p) return ok();
    DeviceGuard g(p->device);
    cudaFree(p->rec);
    cudaFree(p->conv);
    cudaFree(p->err);
    cudaFree(p->recs);
    cudaFree(p->proj);
    cudaFree(p->gated);
    cudaFree(p->hn);
    cudaFree(p->mix);
    cudaFree(p->wy_tiles);
    cudaFree(p->wy_cb);
    gdn::gemm_destroy(p->gemm);
    cudaFree(p->gemm_ws);
    cudaFree(p->wg_cnt);
    cudaFree(p->wg_ws);
    cudaFree(p->wdq);
    delete p;
    return ok();
}

int gdn_pool_layer_state(gdn_pool* p, int32_t layer, float** rec, gdn_bf16** conv) {
    if (!p) return fail(GDN_E_INVALID, "pool is NULL");
    if (layer < 0 || layer >= p->cfg.n_layers)
        return fail(GDN_E_INVALID, "layer %d out of range [0,%d)", layer, p->cfg.n_layers);
    if (rec) *rec = p->rec + (size_t)layer * p->n_slots * p->rec_slot_elems;
    if (conv) *conv = p->conv + (size_t)layer * p->n_slots * p->conv_slot_elems;
    return ok();
}

int gdn_pool_bytes(const gdn_pool* p, size_t* bytes) {
    if (!p || !bytes) return fail(GDN_E_INVALID, "NULL argument");
    *bytes = (sizeof(float) * p->rec_slot_elems + sizeof(uint16_t) * p->conv_slot_elems) * (size_t)p->n_slots *
                 p->cfg.n_layers +
             sizeof(int32_t) + (size_t)p->rec_cap * p->cfg.n_v_heads * gdn::REC_BYTES +
             (size_t)p->rec_cap * 2 * (proj_ld(p) + p->cfg.n_v_heads * 128 + 2 * p->cfg.hidden) + (32u << 20) +
             kWgMaxTiles * sizeof(int) + (size_t)gdn::wg_workspace_floats(p->n_sm) * sizeof(float) +
             p->wdq_elems * sizeof(uint16_t) + wy_tile_bytes(p, p->rec_cap) +
             (65536 + gdn::WY_PLAN_INTS) * sizeof(int32_t);
    return ok();
}

int gdn_slot_reset(gdn_pool* p, const int32_t* slots, int32_t n, void* stream) {
    if (!p) return fail(GDN_E_INVALID, "pool is NULL");
    if (n < 0 || (n > 0 && !slots)) return fail(GDN_E_INVALID, "bad slot list");
    for (int32_t i = 0; i < n; ++i)
        if (slots[i] < 0 || slots[i] >= p->n_slots)
            return fail(GDN_E_BAD_SLOT, "slot %d out of range [0,%d)", slots[i], p->n_slots);
    DeviceGuard g(p->device);
    if (g.status != cudaSuccess) return cuda_fail(g.status, "cudaSetDevice");
    cudaStream_t s = (cudaStream_t)stream;
    for (int32_t l = 0; l < p->cfg.n_layers; ++l)
        for (int32_t i = 0; i < n; ++i) {
            const size_t idx = (size_t)l * p->n_slots + slots[i];
            cudaError_t e = cudaMemsetAsync(p->rec + idx * p->rec_slot_elems, 0, sizeof(float) * p->rec_slot_elems, s);
            if (e == cudaSuccess)
                e = cudaMemsetAsync(p->conv + idx * p->conv_slot_elems, 0, sizeof(uint16_t) * p->conv_slot_elems, s);
            if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync (slot reset)");
        }
    return ok();
}

static int slot_copy(gdn_pool* p, int32_t slot, int32_t layer, void* rec, void* conv, bool to_host) {
    if (!p) return fail(GDN_E_INVALID, "pool is NULL");
    if (slot < 0 || slot >= p->n_slots) return fail(GDN_E_BAD_SLOT, "slot %d out of range [0,%d)", slot, p->n_slots);
    if (layer < 0 || layer >= p->cfg.n_layers)
        return fail(GDN_E_INVALID, "layer %d out of range [0,%d)", layer, p->cfg.n_layers);
    DeviceGuard g(p->device);
    if (g.status != cudaSuccess) return cuda_fail(g.status, "cudaSetDevice");
    const size_t idx = (size_t)layer * p->n_slots + slot;
    cudaError_t e = cudaSuccess;
    if (rec) {
        float* d = p->rec + idx * p->rec_slot_elems;
        e = to_host ? cudaMemcpy(rec, d, sizeof(float) * p->rec_slot_elems, cudaMemcpyDeviceToHost)
                    : cudaMemcpy(d, rec, sizeof(float) * p->rec_slot_elems, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy (recurrent state)");
    }
    if (conv) {
        uint16_t* d = p->conv + idx * p->conv_slot_elems;
        e = to_host ? cudaMemcpy(conv, d, sizeof(uint16_t) * p->conv_slot_elems, cudaMemcpyDeviceToHost)
                    : cudaMemcpy(d, conv, sizeof(uint16_t) * p->conv_slot_elems, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy (conv state)");
    }
    return ok();
}

int gdn_slot_export(gdn_pool* p, int32_t slot, int32_t layer, float* rec, gdn_bf16* conv) {
    return slot_copy(p, slot, layer, rec, conv, true);
}

int gdn_slot_import(gdn_pool* p, int32_t slot, int32_t layer, const float* rec, const gdn_bf16* conv) {
    return slot_copy(p, slot, layer, const_cast<float*>(rec), const_cast<gdn_bf16*>(conv), false);
}

int gdn_validate_tables(int32_t n_slots, const int32_t* slot_ids, const int32_t* cu, int32_t n_seq,
                        int32_t n_tokens) {
    if (n_slots <= 0) return fail(GDN_E_INVALID, "n_slots must be positive (got %d)", n_slots);
    if (n_seq < 0 || n_tokens < 0) return fail(GDN_E_INVALID, "negative n_seq or n_tokens");
    if (n_seq > 0 && (!slot_ids || !cu)) return fail(GDN_E_INVALID, "NULL routing table");
    if (n_seq == 0) {
        if (n_tokens != 0) return fail(GDN_E_BAD_SEQLENS, "n_seq = 0 but n_tokens = %d", n_tokens);
        return ok();
    }
    if (cu[0] != 0) return fail(GDN_E_BAD_SEQLENS, "cu_seqlens[0] = %d, expected 0", cu[0]);
    for (int32_t i = 0; i < n_seq; ++i)
        if (cu[i + 1] < cu[i])
            return fail(GDN_E_BAD_SEQLENS, "cu_seqlens decreases at %d (%d -> %d)", i, cu[i], cu[i + 1]);
    if (cu[n_seq] != n_tokens)
        return fail(GDN_E_BAD_SEQLENS, "cu_seqlens[%d] = %d, expected n_tokens = %d", n_seq, cu[n_seq], n_tokens);
    std::vector<unsigned char> seen((size_t)n_slots, 0);
    for (int32_t i = 0; i < n_seq; ++i) {
        const int32_t s = slot_ids[i];
        if (s < 0 || s >= n_slots) return fail(GDN_E_BAD_SLOT, "slot_ids[%d] = %d out of range [0,%d)", i, s, n_slots);
        if (seen[s]) return fail(GDN_E_BAD_SLOT, "slot %d appears twice in one batch", s);
        seen[s] = 1;
    }
    return ok();
}

int gdn_validate_batch(const gdn_pool* p, const int32_t* slot_ids, const int32_t* cu, int32_t n_seq,
                       int32_t n_tokens) {
    if (!p) return fail(GDN_E_INVALID, "pool is NULL");
    return gdn_validate_tables(p->n_slots, slot_ids, cu, n_seq, n_tokens);
}

int gdn_pool_check(gdn_pool* p, int32_t* flags, int reset) {
    if (!p || !flags) return fail(GDN_E_INVALID, "NULL argument");
    DeviceGuard g(p->device);
    if (g.status != cudaSuccess) return cuda_fail(g.status, "cudaSetDevice");
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(flags, p->err, sizeof(int32_t), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && reset) e = cudaMemset(p->err, 0, sizeof(int32_t));
    if (e != cudaSuccess) return cuda_fail(e, "reading the error word");
    return ok();
}

static gdn::StepArgs base_args(gdn_pool* p, int32_t layer) {
    gdn::StepArgs a;
    std::memset(&a, 0, sizeof a);
    a.rec = p->rec + (size_t)layer * p->n_slots * p->rec_slot_elems;
    a.n_slots = p->n_slots;
    a.hk = p->cfg.n_k_heads;
    a.hv = p->cfg.n_v_heads;
    a.err = p->err;
    return a;
}

static int check_common(gdn_pool* p, int32_t layer, const int32_t* slot_ids, const int32_t* cu, int32_t n_seq,
                        int32_t n_tokens) {
    if (!p) return fail(GDN_E_INVALID, "pool is NULL");
    if (layer < 0 || layer >= p->cfg.n_layers)
        return fail(GDN_E_INVALID, "layer %d out of range [0,%d)", layer, p->cfg.n_layers);
    if (n_seq < 0 || n_tokens < 0) return fail(GDN_E_INVALID, "negative n_seq or n_tokens");
    if (n_seq > 65535) return fail(GDN_E_UNSUPPORTED, "n_seq %d exceeds 65535 per call", n_seq);
    if (n_seq > 0 && (!slot_ids || !cu)) return fail(GDN_E_INVALID, "NULL routing table");
    return GDN_OK;
}

static int layer_step(gdn_pool* p, int32_t layer, const gdn_layer_weights* w, const gdn_step_io* io,
                      const int32_t* slot_ids, const int32_t* cu, int32_t n_seq, int32_t n_tokens, uint32_t flags,
                      void* stream) {
    int rc = check_common(p, layer, slot_ids, cu, n_seq, n_tokens);
    if (rc) return rc;
    if (!w || !w->conv_w || !w->A_log || !w->dt_bias || !w->norm_w) return fail(GDN_E_INVALID, "NULL layer weight");
    if (!io || !io->qkv || !io->z || !io->ab || !io->out) return fail(GDN_E_INVALID, "NULL step buffer");
    if (((uintptr_t)w->conv_w & 7u) != 0) return fail(GDN_E_INVALID, "conv_w must be 8-byte aligned");
    if (io->ld_qkv < p->D || io->ld_z < (int64_t)p->cfg.n_v_heads * 128 || io->ld_ab < 2 * p->cfg.n_v_heads ||
        io->ld_out < (int64_t)p->cfg.n_v_heads * 128)
        return fail(GDN_E_INVALID, "row stride smaller than the row");
    if (n_tokens > p->rec_cap)
        return fail(GDN_E_INVALID, "n_tokens %d exceeds the pool's reserved %lld tokens per call (gdn_pool_reserve_tokens)",
                    n_tokens, p->rec_cap);
    if (n_seq == 0 || n_tokens == 0) return ok();
    DeviceGuard g(p->device);
    if (g.status != cudaSuccess) return cuda_fail(g.status, "cudaSetDevice");
    float* rec = p->rec + (size_t)layer * p->n_slots * p->rec_slot_elems;
    uint16_t* conv = p->conv + (size_t)layer * p->n_slots * p->conv_slot_elems;
    gdn::PrepArgs pa;
    std::memset(&pa, 0, sizeof pa);
    pa.qkv = io->qkv; pa.ld_qkv = io->ld_qkv;
    pa.z = io->z; pa.ld_z = io->ld_z;
    pa.ab = io->ab; pa.ld_ab = io->ld_ab;
    pa.conv = conv;
    pa.conv_w = w->conv_w;
    pa.A_log = w->A_log;
    pa.dt_bias = w->dt_bias;
    pa.slot_ids = slot_ids;
    pa.cu_seqlens = cu;
    pa.n_seq = n_seq; pa.n_slots = p->n_slots; pa.n_tokens = n_tokens;
    pa.hk = p->cfg.n_k_heads; pa.hv = p->cfg.n_v_heads; pa.D = p->D;
    pa.rec = p->recs;
    pa.rec_cap = p->rec_cap;
    pa.err = p->err;
    pa.tables_stable = (flags & GDN_STEP_TABLES_STABLE) ? 1 : 0;
    pa.dt_bf16 = w->dt_bias_bf16 ? 1 : 0;
    gdn::RecurArgs ra;
    std::memset(&ra, 0, sizeof ra);
    ra.rec = rec;
    ra.rec_in = nullptr;
    ra.conv = conv;
    ra.qkv = io->qkv; ra.ld_qkv = io->ld_qkv;
    ra.recs = p->recs;
    ra.rec_cap = p->rec_cap;
    ra.norm_w = w->norm_w;
    ra.eps = p->cfg.rms_norm_eps;
    ra.out = io->out; ra.ld_out = io->ld_out;
    ra.slot_ids = slot_ids;
    ra.cu_seqlens = cu;
    ra.n_seq = n_seq; ra.n_slots = p->n_slots; ra.n_tokens = n_tokens;
    ra.hk = p->cfg.n_k_heads; ra.hv = p->cfg.n_v_heads; ra.D = p->D;
    ra.err = p->err;
    // A call with more tokens than sequences has multi-token segments: the long ones run the
    // chunked tensor-core kernel after the streaming kernel has done the rest.
    const bool has_long = n_tokens > n_seq;
    ra.wy_min_t = has_long ? gdn::WY_MIN_T : 0;
    ra.wy_counter = p->err + 1;
    ra.wy_tiles = p->wy_tiles;
    ra.wy_cap_chunks = p->wy_cap;
    ra.wy_chunks = reinterpret_cast<int2*>(p->wy_tiles + (size_t)p->wy_cap * p->cfg.n_v_heads * gdn::WY_TILESET_BYTES);
    ra.wy_cb = p->wy_cb;
    ra.wy_plan = p->wy_plan;
    if (has_long && gdn::wy_z_direct(io->z, io->ld_z)) {   // z to the chunked kernel directly, not via the records
        ra.z = io->z;
        ra.ld_z = io->ld_z;
        pa.z_skip_min_t = gdn::WY_MIN_T;
    }
    cudaError_t e = gdn::launch_layer_step_v2(pa, ra, (cudaStream_t)stream);
    if (e == cudaSuccess && has_long) e = gdn::launch_wy(ra, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "gdn_layer_step launch");
    return ok();
}

int gdn_layer_step(gdn_pool* p, int32_t layer, const gdn_layer_weights* w, const gdn_step_io* io,
                   const int32_t* slot_ids, const int32_t* cu, int32_t n_seq, int32_t n_tokens, void* stream) {
    return layer_step(p, layer, w, io, slot_ids, cu, n_seq, n_tokens, 0u, stream);
}

int gdn_layer_step_ex(gdn_pool* p, int32_t layer, const gdn_layer_weights* w, const gdn_step_io* io,
                      const int32_t* slot_ids, const int32_t* cu, int32_t n_seq, int32_t n_tokens, uint32_t flags,
                      void* stream) {
    if (flags & ~(uint32_t)GDN_STEP_TABLES_STABLE) return fail(GDN_E_INVALID, "unknown flags 0x%x", flags);
    return layer_step(p, layer, w, io, slot_ids, cu, n_seq, n_tokens, flags, stream);
}

static bool mixer_weights_ok(const gdn_mixer_weights* w) {
    return w && (w->w_in || w->w_in_tiles || w->w_in_q4) && (w->w_out || w->w_out_tiles || w->w_out_q4) &&
           w->step.conv_w && w->step.A_log && w->step.dt_bias && w->step.norm_w;
}

// The weight-streaming kernel reads x rows that start on 16-byte boundaries, in whole 8-column chunks.
static bool wg_rows_ok(int K, const void* x, long long ldx, const void* tiles) {
    return K % 8 == 0 && ldx % 8 == 0 && ((uintptr_t)x & 15u) == 0 && ((uintptr_t)tiles & 15u) == 0;
}

// y = x w^T on the weight-streaming kernel, in token blocks of WG_MAX_M (each block streams the weight); a call of
// at most 16 tokens runs the 16-token kernels instead: 4-bit with the dequantized weight in tensor memory, bf16
// with the weight tiles streamed into shared-memory stages.
static int wg_run(gdn_pool* p, bool q4, int M, int N, int K, const uint16_t* x, long long ldx, const void* tiles,
                  uint16_t* y, long long ldy, cudaStream_t s, const char* what) {
    if (!q4 && gdn::wb16_supported(M, N, K)) {
        gdn::WgGemm g;
        g.tiles = reinterpret_cast<const uint8_t*>(tiles);
        g.q4 = false;
        g.x = x; g.ldx = ldx;
        g.y = y; g.ldy = ldy;
        g.M = M; g.N = N; g.K = K;
        g.n_sm = p->n_sm; g.ws = p->wg_ws; g.cnt = p->wg_cnt; g.err = p->err;
        const cudaError_t e = gdn::launch_wb16(g, s);
        if (e == cudaSuccess) return GDN_OK;
        if (e != cudaErrorNotSupported)
            return fail(GDN_E_CUDA, "%s: bf16 projection launch failed (M=%d N=%d K=%d): %s", what, M, N, K,
                        cudaGetErrorString(e));
        // a split's tokens do not fit in shared memory: stream the weight below
    }
    if (q4 && gdn::wq16_supported(M, N, K)) {
        gdn::WgGemm g;
        g.tiles = reinterpret_cast<const uint8_t*>(tiles);
        g.q4 = true;
        g.x = x; g.ldx = ldx;
        g.y = y; g.ldy = ldy;
        g.M = M; g.N = N; g.K = K;
        g.n_sm = p->n_sm; g.ws = p->wg_ws; g.cnt = p->wg_cnt; g.err = p->err;
        const cudaError_t e = gdn::launch_wq16(g, s);
        if (e == cudaSuccess) return GDN_OK;
        if (e != cudaErrorNotSupported)
            return fail(GDN_E_CUDA, "%s: 4-bit projection launch failed (M=%d N=%d K=%d): %s", what, M, N, K,
                        cudaGetErrorString(e));
        // K too long for the tensor-memory kernel's k-splits: stream the weight below
    }
    for (int m0 = 0; m0 < M; m0 += gdn::WG_MAX_M) {
        gdn::WgGemm g;
        g.tiles = reinterpret_cast<const uint8_t*>(tiles);
        g.q4 = q4;
        g.x = x + (long long)m0 * ldx; g.ldx = ldx;
        g.y = y + (long long)m0 * ldy; g.ldy = ldy;
        g.M = M - m0 < gdn::WG_MAX_M ? M - m0 : gdn::WG_MAX_M;
        g.N = N; g.K = K;
        g.n_sm = p->n_sm; g.ws = p->wg_ws; g.cnt = p->wg_cnt; g.err = p->err;
        const cudaError_t e = gdn::launch_wg_gemm(g, s);
        if (e != cudaSuccess)
            return fail(GDN_E_CUDA, "%s: weight-streaming GEMM launch failed (M=%d N=%d K=%d): %s", what, g.M, N, K,
                        cudaGetErrorString(e));
    }
    return GDN_OK;
}

// One projection y = x w^T: 4-bit tiles when given (calls of at most WG_MAX_M tokens on a weight with
// enough rows for whole slabs on every SM stream them; longer calls, and weights of fewer rows (the
// out-projection, where streaming needs split-k partial sums), expand the weight to bf16 once into the
// pool's scratch and run one cuBLASLt GEMM), else bf16 tiles for calls of at most WG_MAX_M tokens, else
// cuBLASLt on the row-major weight.
static int projection(gdn_pool* p, int M, int N, int K, const uint16_t* x, long long ldx, const uint16_t* w,
                      const void* w_tiles, const void* w_q4, uint16_t* y, long long ldy, cudaStream_t s,
                      const char* what) {
    if (w_q4) {
        if (!wg_rows_ok(K, x, ldx, w_q4) || K % 64 != 0)
            return fail(GDN_E_INVALID, "%s: 4-bit projection needs K %% 64 == 0 and 16-byte aligned rows", what);
        const bool whole_slabs = (N + 7) / 8 >= 8 * p->n_sm;
        const bool tmem_kernel = gdn::wq16_supported(M, N, K);   // <= 16 tokens: any row count
        if ((M > gdn::WG_MAX_M || (!whole_slabs && !tmem_kernel)) && (size_t)N * K <= p->wdq_elems) {
            const cudaError_t e = gdn::launch_wq_untile(w_q4, N, K, p->wdq, s);
            if (e != cudaSuccess) return cuda_fail(e, "4-bit weight expansion");
            if (gdn::gemm_bf16_nt(p->gemm, M, N, K, x, ldx, p->wdq, y, ldy, s))
                return fail(GDN_E_CUDA, "%s: cuBLASLt GEMM failed (M=%d N=%d K=%d)", what, M, N, K);
            return GDN_OK;
        }
        return wg_run(p, true, M, N, K, x, ldx, w_q4, y, ldy, s, what);
    }
    if (w_tiles && M <= gdn::WG_MAX_M && wg_rows_ok(K, x, ldx, w_tiles))
        return wg_run(p, false, M, N, K, x, ldx, w_tiles, y, ldy, s, what);
    if (!w)
        return fail(GDN_E_INVALID, "%s: M=%d tokens needs the row-major weight (tiled path: 1..%d tokens, "
                    "16-byte aligned rows)", what, M, gdn::WG_MAX_M);
    if (gdn::gemm_bf16_nt(p->gemm, M, N, K, x, ldx, w, y, ldy, s))
        return fail(GDN_E_CUDA, "%s: cuBLASLt GEMM failed (M=%d N=%d K=%d)", what, M, N, K);
    return GDN_OK;
}

// One mixer layer on the pool's scratch: x -> proj -> fused step -> gated -> y.
static int mixer_layer(gdn_pool* p, int32_t layer, const gdn_mixer_weights* w, const gdn_bf16* x, int64_t ld_x,
                       gdn_bf16* y, int64_t ld_y, const int32_t* slot_ids, const int32_t* cu, int32_t n_seq,
                       int32_t n_tokens, void* stream) {
    const int H = p->cfg.hidden;
    const int zd = p->cfg.n_v_heads * 128;
    const long long ldp = proj_ld(p);
    cudaStream_t s = (cudaStream_t)stream;
    int rc = projection(p, n_tokens, (int)ldp, H, x, ld_x, w->w_in, w->w_in_tiles, w->w_in_q4, p->proj, ldp, s,
                        "in-projection");
    if (rc) return rc;
    gdn_step_io io;
    io.qkv = p->proj; io.ld_qkv = ldp;
    io.z = p->proj + p->D; io.ld_z = ldp;
    io.ab = p->proj + p->D + zd; io.ld_ab = ldp;
    io.out = p->gated; io.ld_out = zd;
    // The in-projection kernel stands between the caller's kernels and the step, and lets the step start
    // only after everything before it has finished: the tables and this layer's conv state are settled.
    rc = layer_step(p, layer, &w->step, &io, slot_ids, cu, n_seq, n_tokens, GDN_STEP_TABLES_STABLE, stream);
    if (rc) return rc;
    return projection(p, n_tokens, H, zd, p->gated, zd, w->w_out, w->w_out_tiles, w->w_out_q4, y, ld_y, s,
                      "out-projection");
}

int gdn_linear(gdn_pool* p, int32_t n_tokens, int32_t n_out, int32_t n_in, const gdn_bf16* x, int64_t ld_x,
               const gdn_bf16* w, gdn_bf16* y, int64_t ld_y, void* stream) {
    if (!p) return fail(GDN_E_INVALID, "pool is NULL");
    if (n_tokens < 0 || n_out <= 0 || n_in <= 0 || ld_x < n_in || ld_y < n_out)
        return fail(GDN_E_INVALID, "bad GEMM shape (M=%d N=%d K=%d ld_x=%lld ld_y=%lld)", n_tokens, n_out, n_in,
                    (long long)ld_x, (long long)ld_y);
    if (n_tokens == 0) return ok();
    if (!x || !w || !y) return fail(GDN_E_INVALID, "NULL tensor");
    DeviceGuard g(p->device);
    if (g.status != cudaSuccess) return cuda_fail(g.status, "cudaSetDevice");
    if (gdn::gemm_bf16_nt(p->gemm, n_tokens, n_out, n_in, x, ld_x, w, y, ld_y, (cudaStream_t)stream))
        return fail(GDN_E_CUDA, "cuBLASLt GEMM failed (M=%d N=%d K=%d)", n_tokens, n_out, n_in);
    return ok();
}

int64_t gdn_weight_tile_bytes(int32_t n_out, int32_t n_in) {
    if (n_out <= 0 || n_in <= 0) return 0;
    return gdn::wg_tile_bytes(n_out, n_in);
}

int gdn_weight_tile(int32_t n_out, int32_t n_in, const gdn_bf16* w, void* tiles, void* stream) {
    if (n_out <= 0 || n_in <= 0) return fail(GDN_E_INVALID, "bad weight shape [%d][%d]", n_out, n_in);
    if (!w || !tiles) return fail(GDN_E_INVALID, "NULL tensor");
    if (((uintptr_t)tiles & 15u) != 0) return fail(GDN_E_INVALID, "tiled weight buffer must be 16-byte aligned");
    const cudaError_t e = gdn::launch_wg_tile(w, n_out, n_in, reinterpret_cast<uint8_t*>(tiles), (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "weight tiling kernel launch");
    return ok();
}

int64_t gdn_weight_tile_q4_bytes(int32_t n_out, int32_t n_in) {
    if (n_out <= 0 || n_in <= 0 || n_in % 64 != 0) return 0;
    return gdn::wq_tile_bytes(n_out, n_in);
}

int gdn_weight_tile_q4(int32_t n_out, int32_t n_in, const uint32_t* w_q, const gdn_bf16* scales,
                       const gdn_bf16* biases, void* tiles, void* stream) {
    if (n_out <= 0 || n_in <= 0 || n_in % 64 != 0)
        return fail(GDN_E_INVALID, "bad 4-bit weight shape [%d][%d] (n_in must be a multiple of the group, 64)",
                    n_out, n_in);
    if (!w_q || !scales || !biases || !tiles) return fail(GDN_E_INVALID, "NULL tensor");
    if (((uintptr_t)tiles & 15u) != 0) return fail(GDN_E_INVALID, "tiled weight buffer must be 16-byte aligned");
    const cudaError_t e = gdn::launch_wq_tile(w_q, scales, biases, n_out, n_in, reinterpret_cast<uint8_t*>(tiles),
                                              (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "4-bit weight tiling kernel launch");
    return ok();
}

static int linear_tiled_common(gdn_pool* p, bool q4, int32_t n_tokens, int32_t n_out, int32_t n_in,
                               const gdn_bf16* x, int64_t ld_x, const void* tiles, gdn_bf16* y, int64_t ld_y,
                               void* stream, const char* what) {
    if (!p) return fail(GDN_E_INVALID, "pool is NULL");
    if (n_tokens < 0 || n_out <= 0 || n_in <= 0 || ld_x < n_in || ld_y < n_out)
        return fail(GDN_E_INVALID, "bad GEMM shape (M=%d N=%d K=%d ld_x=%lld ld_y=%lld)", n_tokens, n_out, n_in,
                    (long long)ld_x, (long long)ld_y);
    if (n_tokens == 0) return ok();
    if (!x || !tiles || !y) return fail(GDN_E_INVALID, "NULL tensor");
    if (!wg_rows_ok(n_in, x, ld_x, tiles) || (q4 && n_in % 64 != 0))
        return fail(GDN_E_INVALID, "%s needs n_in %% %d == 0 and 16-byte aligned x rows and weight", what,
                    q4 ? 64 : 8);
    if (gdn::wg_num_slabs((n_out + 7) / 8, p->n_sm) > kWgMaxTiles)
        return fail(GDN_E_INVALID, "n_out %d: more row slabs than the pool's %d counters", n_out, kWgMaxTiles);
    DeviceGuard g(p->device);
    if (g.status != cudaSuccess) return cuda_fail(g.status, "cudaSetDevice");
    const int rc = wg_run(p, q4, n_tokens, n_out, n_in, x, ld_x, tiles, y, ld_y, (cudaStream_t)stream, what);
    return rc ? rc : ok();
}

int gdn_linear_tiled(gdn_pool* p, int32_t n_tokens, int32_t n_out, int32_t n_in, const gdn_bf16* x, int64_t ld_x,
                     const void* w_tiles, gdn_bf16* y, int64_t ld_y, void* stream) {
    return linear_tiled_common(p, false, n_tokens, n_out, n_in, x, ld_x, w_tiles, y, ld_y, stream,
                               "gdn_linear_tiled");
}

int gdn_linear_q4(gdn_pool* p, int32_t n_tokens, int32_t n_out, int32_t n_in, const gdn_bf16* x, int64_t ld_x,
                  const void* w_q4_tiles, gdn_bf16* y, int64_t ld_y, void* stream) {
    return linear_tiled_common(p, true, n_tokens, n_out, n_in, x, ld_x, w_q4_tiles, y, ld_y, stream, "gdn_linear_q4");
}

int gdn_mixer_step(gdn_pool* p, int32_t layer, const gdn_mixer_weights* w, const gdn_bf16* x, int64_t ld_x,
                   gdn_bf16* y, int64_t ld_y, const int32_t* slot_ids, const int32_t* cu, int32_t n_seq,
                   int32_t n_tokens, void* stream) {
    int rc = check_common(p, layer, slot_ids, cu, n_seq, n_tokens);
    if (rc) return rc;
    if (!mixer_weights_ok(w)) return fail(GDN_E_INVALID, "NULL mixer weight");
    if (!x || !y || ld_x < p->cfg.hidden || ld_y < p->cfg.hidden) return fail(GDN_E_INVALID, "bad x / y buffer");
    if (n_tokens > p->rec_cap)
        return fail(GDN_E_INVALID, "n_tokens %d exceeds the pool's reserved %lld tokens per call", n_tokens, p->rec_cap);
    if (n_seq == 0 || n_tokens == 0) return ok();
    DeviceGuard g(p->device);
    if (g.status != cudaSuccess) return cuda_fail(g.status, "cudaSetDevice");
    rc = mixer_layer(p, layer, w, x, ld_x, y, ld_y, slot_ids, cu, n_seq, n_tokens, stream);
    return rc ? rc : ok();
}

int gdn_stack_step(gdn_pool* p, const gdn_mixer_weights* layers, gdn_bf16* h, int64_t ld_h,
                   const int32_t* slot_ids, const int32_t* cu, int32_t n_seq, int32_t n_tokens, void* stream) {
    int rc = check_common(p, 0, slot_ids, cu, n_seq, n_tokens);
    if (rc) return rc;
    if (!layers || !h || ld_h < p->cfg.hidden) return fail(GDN_E_INVALID, "bad layers / h");
    for (int l = 0; l < p->cfg.n_layers; ++l)
        if (!mixer_weights_ok(&layers[l]) || !layers[l].pre_norm_w)
            return fail(GDN_E_INVALID, "NULL weight in layer %d", l);
    if (n_tokens > p->rec_cap)
        return fail(GDN_E_INVALID, "n_tokens %d exceeds the pool's reserved %lld tokens per call", n_tokens, p->rec_cap);
    if (n_seq == 0 || n_tokens == 0) return ok();
    DeviceGuard g(p->device);
    if (g.status != cudaSuccess) return cuda_fail(g.status, "cudaSetDevice");
    cudaStream_t s = (cudaStream_t)stream;
    const int H = p->cfg.hidden;
    const float eps = p->cfg.rms_norm_eps;
    for (int l = 0; l < p->cfg.n_layers; ++l) {
        // h <- h + mix_{l-1} (from layer 1 on), hn <- rms_norm(h, pre_norm_w[l])
        cudaError_t e = gdn::launch_add_rmsnorm(h, ld_h, l ? p->mix : nullptr, H, h, layers[l].pre_norm_w, p->hn, H,
                                                n_tokens, H, eps, s);
        if (e != cudaSuccess) return cuda_fail(e, "pre-norm launch");
        rc = mixer_layer(p, l, &layers[l], p->hn, H, p->mix, H, slot_ids, cu, n_seq, n_tokens, stream);
        if (rc) return rc;
    }
    cudaError_t e = gdn::launch_add_rmsnorm(h, ld_h, p->mix, H, h, layers[0].pre_norm_w, nullptr, H, n_tokens, H,
                                            eps, s);
    if (e != cudaSuccess) return cuda_fail(e, "residual launch");
    return ok();
}

int gdn_recurrence(gdn_pool* p, int32_t layer, const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v,
                   const float* g, const gdn_bf16* beta, const int32_t* slot_ids, const int32_t* cu, int32_t n_seq,
                   int32_t n_tokens, gdn_bf16* y, void* stream) {
    int rc = check_common(p, layer, slot_ids, cu, n_seq, n_tokens);
    if (rc) return rc;
    if (!q || !k || !v || !g || !beta || !y) return fail(GDN_E_INVALID, "NULL tensor");
    if (n_seq == 0) return ok();
    DeviceGuard dg(p->device);
    if (dg.status != cudaSuccess) return cuda_fail(dg.status, "cudaSetDevice");
    gdn::StepArgs a = base_args(p, layer);
    a.slot_ids = slot_ids;
    a.cu_seqlens = cu;
    a.n_seq = n_seq;
    a.n_tokens = n_tokens;
    a.q = q; a.k = k; a.v = v; a.g = g; a.beta = beta; a.y = y;
    cudaError_t e = gdn::launch_recurrence(a, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "gdn_recurrence launch");
    return ok();
}

int gdn_gated_delta_kernel(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v, const float* g,
                           const gdn_bf16* beta, const float* state_in, int32_t seq_len, int32_t batch, int32_t hk,
                           int32_t hv, int32_t dk, int32_t dv, gdn_bf16* y, float* state_out, void* stream) {
    if (!q || !k || !v || !g || !beta || !state_in || !y || !state_out) return fail(GDN_E_INVALID, "NULL tensor");
    if (seq_len < 0 || batch < 0 || hk <= 0 || hv <= 0 || hv % hk)
        return fail(GDN_E_INVALID, "bad shape (T=%d B=%d hk=%d hv=%d)", seq_len, batch, hk, hv);
    if (dk != 128 || dv != 128) return fail(GDN_E_UNSUPPORTED, "only dk = dv = 128 is specialised (got %d, %d)", dk, dv);
    if (batch > 65535) return fail(GDN_E_UNSUPPORTED, "batch %d exceeds 65535 per call", batch);
    if ((long long)batch * seq_len > 0x7fffffffLL) return fail(GDN_E_UNSUPPORTED, "B*T overflows int32");
    if ((((uintptr_t)state_in) | ((uintptr_t)state_out)) & 15u)
        return fail(GDN_E_INVALID, "state_in / state_out must be 16-byte aligned");
    if (batch == 0) return ok();
    gdn::StepArgs a;
    std::memset(&a, 0, sizeof a);
    a.rec = state_out;
    a.rec_in = (state_in == state_out) ? nullptr : state_in;
    a.n_seq = batch;
    a.n_slots = batch;
    a.T_dense = seq_len;
    a.n_tokens = batch * seq_len;
    a.hk = hk;
    a.hv = hv;
    a.q = q; a.k = k; a.v = v; a.g = g; a.beta = beta; a.y = y;
    cudaError_t e = gdn::launch_recurrence(a, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "gdn_gated_delta_kernel launch");
    return ok();
}

int gdn_set_decode_kernel(int mode) {
    if (mode < 0 || mode > 3) return fail(GDN_E_INVALID, "decode kernel mode %d not in 0..3", mode);
    gdn::g_decode_kernel = mode;
    return ok();
}

int gdn_test_set_wait_fault(int32_t skip_block, int64_t wait_ns) {
    if (wait_ns <= 0) return fail(GDN_E_INVALID, "wait_ns must be positive");
    gdn::g_split_ctl.skip_block = skip_block;
    gdn::g_split_ctl.wait_ns = (unsigned long long)wait_ns;
    return ok();
}

int gdn_beta_g_ex(const gdn_bf16* ab, int64_t ld_ab, int32_t n_tokens, int32_t hv, const float* A_log,
                  const float* dt_bias, int32_t dt_bias_bf16, gdn_bf16* beta, float* g, void* stream) {
    if (!ab || !A_log || !dt_bias || !beta || !g) return fail(GDN_E_INVALID, "NULL tensor");
    if (n_tokens < 0 || hv <= 0 || ld_ab < 2 * hv) return fail(GDN_E_INVALID, "bad shape");
    cudaError_t e = gdn::launch_beta_g(ab, ld_ab, n_tokens, hv, A_log, dt_bias, dt_bias_bf16 ? 1 : 0, beta, g,
                                       (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "gdn_beta_g launch");
    return ok();
}

int gdn_beta_g(const gdn_bf16* ab, int64_t ld_ab, int32_t n_tokens, int32_t hv, const float* A_log,
               const float* dt_bias, gdn_bf16* beta, float* g, void* stream) {
    return gdn_beta_g_ex(ab, ld_ab, n_tokens, hv, A_log, dt_bias, 0, beta, g, stream);
}

}  // extern "C"
