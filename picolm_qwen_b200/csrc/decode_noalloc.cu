// decode_noalloc.cu -- picoattn_decode_noalloc: the decode step with its
// scratch memory in a fixed device array instead of a caller workspace.
//
// Who needs this: an embedder that sizes all of its memory once at start-up and
// must not allocate on the per-token path (the way the reference engine sizes
// RunState once in allocate_run_state), or a host whose device memory belongs
// to another allocator (a serving framework's pool) and that cannot hand this
// library a workspace.  Such a caller cannot call cudaMalloc itself, and
// cudaMalloc on the token path may also synchronise the device and stall
// decoding.  This entry point runs the same three decode kernels as
// picoattn_decode; only the place their scratch lives differs.
//
// The scratch is one file-scope device array, g_decode_scratch, of
// kNoAllocScratchBytes.  Every GPU that loads the library holds it until the
// process exits.  Its device address is looked up once per device
// (cudaGetSymbolAddress, with that device current) on the first call made with
// that device current; make that first call before any stream capture.  All
// calls share the array and it keeps the last call's contents: each call clears
// the status header it relies on before launching, and calls whose kernels
// overlap on the GPU (e.g. on two streams) race on the array.
#include <mutex>

#include "picoattn.h"
#include "picoattn_internal.h"

namespace picoattn {

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB per device
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
void* g_addr[kMaxDevices] = {};

// Device address of g_decode_scratch on the current device (host code cannot
// use the symbol itself: on the host it names a stand-in, not device memory).
cudaError_t scratch_address(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_decode_scratch);
        if (e != cudaSuccess) return e;
        g_addr[dev] = p;
    }
    *out = g_addr[dev];
    return cudaSuccess;
}

}  // namespace

}  // namespace picoattn

using namespace picoattn;

extern "C" int32_t picoattn_decode_noalloc(const picoattn_config_t* cfg, int32_t layer, int32_t n_seqs,
                                           int32_t max_ctx, const float* q, const float* k, const float* v,
                                           const float* q_norm_w, const float* k_norm_w, const float* rope_cos,
                                           const float* rope_sin, uint16_t* const* k_cache,
                                           uint16_t* const* v_cache, const int32_t* pos, float* out,
                                           picoattn_stream_t stream, uint32_t* status_out) {
    int32_t st = picoattn_config_check(cfg);
    if (st != PICOATTN_OK) return st;
    if (layer < 0 || layer >= cfg->n_layers || n_seqs <= 0) return PICOATTN_EINVAL;
    if (!q || !k || !v || !rope_cos || !rope_sin || !k_cache || !v_cache || !pos || !out) return PICOATTN_EINVAL;
    if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) & 15u) return PICOATTN_EINVAL;
    if ((q_norm_w == nullptr) != (k_norm_w == nullptr)) return PICOATTN_EINVAL;
    if (max_ctx <= 0 || max_ctx > cfg->max_seq_len) return PICOATTN_ERANGE;
    DecodePlan plan;
    if (!make_decode_plan(*cfg, n_seqs, max_ctx, &plan)) return PICOATTN_EUNSUPPORTED;
    if (plan.ws_total > kNoAllocScratchBytes) return PICOATTN_ENOSPACE;  // beyond the fixed 8 MiB scratch
    st = picoattn_device_check();
    if (st != PICOATTN_OK) return st;
    void* scratch = nullptr;
    st = cuda_status(scratch_address(&scratch));
    if (st != PICOATTN_OK) return st;
    cudaStream_t s = (cudaStream_t)stream;
    // the sticky status word must start each call at zero; everything else in
    // the scratch is written by the kernels before it is read
    st = cuda_status(cudaMemsetAsync(scratch, 0, kWsHeaderBytes, s));
    if (st != PICOATTN_OK) return st;

    uint8_t* w = static_cast<uint8_t*>(scratch);
    DecodeArgs a{};
    a.hq = cfg->n_heads;
    a.hkv = cfg->n_kv_heads;
    a.g = a.hq / a.hkv;
    a.hd = cfg->head_dim;
    a.kvd = a.hkv * a.hd;
    a.max_seq = cfg->max_seq_len;
    a.layer = layer;
    a.n_seqs = n_seqs;
    a.max_ctx = max_ctx;
    a.rope_mode = cfg->rope_mode;
    a.eps = cfg->qk_norm_eps;
    a.q = q, a.k = k, a.v = v, a.qn_w = q_norm_w, a.kn_w = k_norm_w, a.rope_cos = rope_cos, a.rope_sin = rope_sin;
    a.kc_ptrs = k_cache, a.vc_ptrs = v_cache, a.kc_one = nullptr, a.vc_one = nullptr;
    a.pos_dev = pos, a.pos_host = 0, a.out = out;
    a.status = reinterpret_cast<unsigned int*>(w);
    a.q_rot = reinterpret_cast<float*>(w + plan.ws_qrot);
    a.part_ml = reinterpret_cast<float*>(w + plan.ws_ml);
    a.part_o = reinterpret_cast<float*>(w + plan.ws_o);
    a.n_slots = plan.n_slots;
    a.prefix = reinterpret_cast<long long*>(w + plan.ws_prefix);
    a.row_offset = 0;
    a.local_rows = cfg->max_seq_len;
    a.shard_out = nullptr;
    a.tile_rows = plan.tile_rows;
    a.stages = plan.stages;
    a.warps_per_head = plan.warps_per_head;
    a.compute_warps = plan.compute_warps;
    st = cuda_status(launch_decode(a, plan, s, PICOATTN_STAGE_ALL));
    if (st != PICOATTN_OK) return st;
    if (status_out) {
        unsigned int dev_status = 0;
        cudaError_t e = cudaMemcpyAsync(&dev_status, scratch, sizeof dev_status, cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        st = cuda_status(e);
        if (st != PICOATTN_OK) return st;
        *status_out = dev_status;
        if (dev_status) return PICOATTN_EDEVSTATUS;
    }
    return PICOATTN_OK;
}
