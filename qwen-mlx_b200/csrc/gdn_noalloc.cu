// gdn_noalloc.cu -- gdn_layer_step_noalloc: the fused GDN layer step for callers
// that cannot allocate device memory.
//
// Some callers may not call cudaMalloc: an engine that reserves one fixed device
// arena at start-up and forbids allocation afterwards (cudaMalloc can synchronise
// the device, fragments the arena and cannot run inside stream capture), or a
// host framework whose own caching allocator owns all device memory.  Such a
// caller keeps the recurrent and conv states in memory it already owns and
// passes them in; this entry point runs the same two kernels as gdn_layer_step
// (prep + streaming recurrence) and takes their scratch -- one 1056-byte record
// per (v-head, token) -- from the file-scope array below instead of a pool.
//
// The array is a fixed NOALLOC_MAX_RECORDS records (4,259,840 bytes) in every
// device that loads this library, held until the process exits.  A call may
// carry at most NOALLOC_MAX_RECORDS / Hv packed tokens (128 for Hv = 32).
// All calls on a device share the array and it keeps the last call's records,
// so calls that overlap on the GPU (different streams, or different host
// threads) race; serialise them.  Nothing in it has to start at zero: every
// record a call reads was written earlier in that same call.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "gdn.h"
#include "gdn_internal.h"

namespace {

constexpr long long NOALLOC_MAX_RECORDS = 4096;
constexpr size_t NOALLOC_RECORD_BYTES = (size_t)NOALLOC_MAX_RECORDS * gdn::REC_BYTES;

// records [Hv][n_tokens][REC_BYTES], then one int32 word the kernels' bounds checks may set
static __device__ __align__(256) uint8_t g_noalloc_scratch[NOALLOC_RECORD_BYTES + 256];

constexpr int MAX_DEVICES = 64;
std::mutex g_setup_mutex;
uint8_t* g_scratch_ptr[MAX_DEVICES] = {nullptr};

// Set-up, once per device, with that device current: the device address of the scratch array
// (the host-side symbol is not a device address; the kernels get this pointer), and a cleared
// error word.  The first call on a device does this, so make it before capturing any stream into
// a CUDA graph.
int scratch_of_current_device(uint8_t** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES)
        return gdn::record_error(GDN_E_CUDA, "cudaGetDevice failed or device index out of range");
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_ptr[dev]) {
        void* ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess || !ptr) return gdn::record_error(GDN_E_CUDA, "cudaGetSymbolAddress of the scratch failed");
        const int32_t zero = 0;
        e = cudaMemcpyToSymbol(g_noalloc_scratch, &zero, sizeof zero, NOALLOC_RECORD_BYTES, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return gdn::record_error(GDN_E_CUDA, "clearing the no-alloc error word failed");
        g_scratch_ptr[dev] = static_cast<uint8_t*>(ptr);
    }
    *out = g_scratch_ptr[dev];
    return GDN_OK;
}

}  // namespace

extern "C" {

int gdn_layer_step_noalloc(const gdn_config* cfg, int32_t n_slots, float* rec_state, gdn_bf16* conv_state,
                           const gdn_layer_weights* w, const gdn_step_io* io, const int32_t* slot_ids,
                           const int32_t* cu_seqlens, int32_t n_seq, int32_t n_tokens, void* stream) {
    using gdn::record_error;
    if (!cfg || !rec_state || !conv_state || !w || !io) return record_error(GDN_E_INVALID, "NULL argument");
    if (!w->conv_w || !w->A_log || !w->dt_bias || !w->norm_w) return record_error(GDN_E_INVALID, "NULL layer weight");
    if (!io->qkv || !io->z || !io->ab || !io->out) return record_error(GDN_E_INVALID, "NULL step buffer");
    if (cfg->head_k_dim != gdn::DK_ABI || cfg->head_v_dim != gdn::DV_ABI || cfg->conv_kernel != 4)
        return record_error(GDN_E_UNSUPPORTED, "only head_k_dim = head_v_dim = 128 and conv_kernel = 4 are specialised");
    if (cfg->n_k_heads <= 0 || cfg->n_v_heads <= 0 || cfg->n_v_heads % cfg->n_k_heads)
        return record_error(GDN_E_INVALID, "n_v_heads must be a positive multiple of n_k_heads");
    if (n_slots <= 0 || n_seq < 0 || n_tokens < 0 || n_seq > 65535)
        return record_error(GDN_E_INVALID, "bad n_slots / n_seq / n_tokens");
    if (n_seq > 0 && (!slot_ids || !cu_seqlens)) return record_error(GDN_E_INVALID, "NULL routing table");
    const int D = 2 * cfg->n_k_heads * cfg->head_k_dim + cfg->n_v_heads * cfg->head_v_dim;
    if (io->ld_qkv < D || io->ld_z < (int64_t)cfg->n_v_heads * 128 || io->ld_ab < 2 * cfg->n_v_heads ||
        io->ld_out < (int64_t)cfg->n_v_heads * 128)
        return record_error(GDN_E_INVALID, "row stride smaller than the row");
    if (((uintptr_t)rec_state & 15u) || ((uintptr_t)w->conv_w & 7u))
        return record_error(GDN_E_INVALID, "rec_state must be 16-byte and conv_w 8-byte aligned");
    // the fixed scratch bounds the tokens of one call: Hv records per token
    if ((long long)n_tokens * cfg->n_v_heads > NOALLOC_MAX_RECORDS)
        return record_error(GDN_E_INVALID,
                            "n_tokens * n_v_heads exceeds the fixed no-alloc scratch of 4096 records (128 tokens "
                            "per call at 32 v-heads); split the batch or use gdn_layer_step with a pool");
    if (n_seq == 0 || n_tokens == 0) return gdn::record_ok();

    uint8_t* scratch = nullptr;
    const int rc = scratch_of_current_device(&scratch);
    if (rc != GDN_OK) return rc;

    gdn::PrepArgs pa;
    std::memset(&pa, 0, sizeof pa);
    pa.qkv = io->qkv; pa.ld_qkv = io->ld_qkv;
    pa.z = io->z; pa.ld_z = io->ld_z;
    pa.ab = io->ab; pa.ld_ab = io->ld_ab;
    pa.conv = conv_state;
    pa.conv_w = w->conv_w;
    pa.A_log = w->A_log;
    pa.dt_bias = w->dt_bias;
    pa.dt_bf16 = w->dt_bias_bf16 ? 1 : 0;
    pa.slot_ids = slot_ids;
    pa.cu_seqlens = cu_seqlens;
    pa.n_seq = n_seq; pa.n_slots = n_slots; pa.n_tokens = n_tokens;
    pa.hk = cfg->n_k_heads; pa.hv = cfg->n_v_heads; pa.D = D;
    pa.rec = scratch;
    pa.rec_cap = n_tokens;
    pa.err = reinterpret_cast<int32_t*>(scratch + NOALLOC_RECORD_BYTES);

    gdn::RecurArgs ra;
    std::memset(&ra, 0, sizeof ra);
    ra.rec = rec_state;
    ra.rec_in = nullptr;
    ra.conv = conv_state;
    ra.qkv = io->qkv; ra.ld_qkv = io->ld_qkv;
    ra.recs = scratch;
    ra.rec_cap = n_tokens;
    ra.norm_w = w->norm_w;
    ra.eps = cfg->rms_norm_eps;
    ra.out = io->out; ra.ld_out = io->ld_out;
    ra.slot_ids = slot_ids;
    ra.cu_seqlens = cu_seqlens;
    ra.n_seq = n_seq; ra.n_slots = n_slots; ra.n_tokens = n_tokens;
    ra.hk = cfg->n_k_heads; ra.hv = cfg->n_v_heads; ra.D = D;
    ra.err = pa.err;

    const cudaError_t e = gdn::launch_layer_step_v2(pa, ra, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return record_error(GDN_E_CUDA, cudaGetErrorString(e));
    return gdn::record_ok();
}

// The device error word of the no-alloc step on the current device.  The kernels record a failed
// bounds check (1 << GDN_E_BAD_SLOT, 1 << GDN_E_BAD_SEQLENS) or a bounded wait that gave up (1 << 7)
// there; a call that set a bit returned GDN_OK but its outputs and the state it touched are not to be
// trusted.  Waits for the device, reads the word and clears it when `reset` is non-zero; allocates
// nothing.
int gdn_noalloc_check(int32_t* flags, int reset) {
    if (!flags) return gdn::record_error(GDN_E_INVALID, "flags is NULL");
    uint8_t* scratch = nullptr;
    const int rc = scratch_of_current_device(&scratch);
    if (rc != GDN_OK) return rc;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess)
        e = cudaMemcpyFromSymbol(flags, g_noalloc_scratch, sizeof(int32_t), NOALLOC_RECORD_BYTES, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && reset) {
        const int32_t zero = 0;
        e = cudaMemcpyToSymbol(g_noalloc_scratch, &zero, sizeof zero, NOALLOC_RECORD_BYTES, cudaMemcpyHostToDevice);
    }
    if (e != cudaSuccess) return gdn::record_error(GDN_E_CUDA, cudaGetErrorString(e));
    return gdn::record_ok();
}

}  // extern "C"
