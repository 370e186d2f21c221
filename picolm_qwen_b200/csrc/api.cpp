// api.cpp -- the extern "C" boundary declared in include/picoattn.h.
//
// Host-side argument checking, workspace carving, the RoPE table builder and
// dispatch to the CUDA launchers.  No allocation happens on the call paths.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <initializer_list>

#include <cuda_runtime.h>

#include "picoattn.h"
#include "picoattn_internal.h"

using namespace picoattn;

namespace {
thread_local cudaError_t g_last_cuda_error = cudaSuccess;
}  // namespace

int32_t picoattn::cuda_status(cudaError_t e) {
    if (e == cudaSuccess) return PICOATTN_OK;
    g_last_cuda_error = e;
    return PICOATTN_ECUDA;
}

namespace {

bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// The sm_100 check, once per device (cached; thread-safe).  A device of
// another architecture reads as cudaErrorNoKernelImageForDevice inside the
// cache and maps to PICOATTN_EDEVICE.
int32_t device_ok() {
    static PerDeviceOnce check;
    const cudaError_t e = check.run([] {
        int dev = 0, major = 0, minor = 0;
        cudaError_t r = cudaGetDevice(&dev);
        if (r == cudaSuccess) r = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
        if (r == cudaSuccess) r = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
        if (r != cudaSuccess) return r;
        return major == 10 && minor == 0 ? cudaSuccess : cudaErrorNoKernelImageForDevice;
    });
    if (e == cudaErrorNoKernelImageForDevice) return PICOATTN_EDEVICE;
    return cuda_status(e);
}

int32_t decode_common(const picoattn_config_t* cfg, int32_t layer, int32_t n_seqs, int32_t max_ctx,
                      const float* q, const float* k, const float* v, const float* qn, const float* kn,
                      const float* rc, const float* rs, uint16_t* const* kcp, uint16_t* const* vcp,
                      uint16_t* kc1, uint16_t* vc1, const int32_t* pos_dev, int32_t pos_host, float* out,
                      void* ws, size_t ws_bytes, cudaStream_t stream, uint32_t stages) {
    int32_t st = picoattn_config_check(cfg);
    if (stages == 0 || (stages & ~PICOATTN_STAGE_ALL)) return PICOATTN_EINVAL;
    if (st != PICOATTN_OK) return st;
    if (layer < 0 || layer >= cfg->n_layers || n_seqs <= 0) return PICOATTN_EINVAL;
    if (!q || !k || !v || !rc || !rs || !out || !ws) return PICOATTN_EINVAL;
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out)) return PICOATTN_EINVAL;
    if ((qn == nullptr) != (kn == nullptr)) return PICOATTN_EINVAL;
    if (kcp == nullptr && (kc1 == nullptr || vc1 == nullptr)) return PICOATTN_EINVAL;
    if (kcp != nullptr && vcp == nullptr) return PICOATTN_EINVAL;
    if (kc1 && (!aligned16(kc1) || !aligned16(vc1))) return PICOATTN_EINVAL;
    if (max_ctx <= 0 || max_ctx > cfg->max_seq_len) return PICOATTN_ERANGE;
    if (!pos_dev && (pos_host < 0 || pos_host >= cfg->max_seq_len)) return PICOATTN_ERANGE;
    DecodePlan plan;
    if (!make_decode_plan(*cfg, n_seqs, max_ctx, &plan)) return PICOATTN_EUNSUPPORTED;
    if (ws_bytes < plan.ws_total || !aligned16(ws)) return PICOATTN_ENOSPACE;
    st = device_ok();
    if (st != PICOATTN_OK) return st;

    uint8_t* w = static_cast<uint8_t*>(ws);
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
    a.q = q, a.k = k, a.v = v, a.qn_w = qn, a.kn_w = kn, a.rope_cos = rc, a.rope_sin = rs;
    a.kc_ptrs = kcp, a.vc_ptrs = vcp, a.kc_one = kc1, a.vc_one = vc1;
    a.pos_dev = pos_dev, a.pos_host = pos_host, a.out = out;
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
    return cuda_status(launch_decode(a, plan, stream, stages));
}

// Workspace of picoattn_decode_layer: the decode workspace first (its status
// header at offset 0), then q, k, v and the attention output, fp32.
struct LayerWs {
    size_t decode, q, k, v, attn, total;
};
bool layer_ws(const picoattn_config_t& cfg, int n_seqs, int max_ctx, LayerWs* l) {
    DecodePlan plan;
    if (!make_decode_plan(cfg, n_seqs, max_ctx, &plan)) return false;
    const size_t qd = (size_t)cfg.n_heads * cfg.head_dim, kvd = (size_t)cfg.n_kv_heads * cfg.head_dim;
    l->decode = 0;
    l->q = align_up(plan.ws_total, 256);
    l->k = align_up(l->q + (size_t)n_seqs * qd * 4, 256);
    l->v = align_up(l->k + (size_t)n_seqs * kvd * 4, 256);
    l->attn = align_up(l->v + (size_t)n_seqs * kvd * 4, 256);
    l->total = align_up(l->attn + (size_t)n_seqs * qd * 4, 256);
    return true;
}

}  // namespace

extern "C" {

int32_t picoattn_version(void) { return 100; }

const char* picoattn_strerror(int32_t s) {
    switch (s) {
        case PICOATTN_OK: return "ok";
        case PICOATTN_EINVAL: return "invalid argument";
        case PICOATTN_EUNSUPPORTED: return "unsupported shape";
        case PICOATTN_ERANGE: return "position out of range";
        case PICOATTN_ENOSPACE: return "workspace too small or misaligned";
        case PICOATTN_ECUDA: return "CUDA error";
        case PICOATTN_ENCCL: return "NCCL error";
        case PICOATTN_ETIMEOUT: return "timed out";
        case PICOATTN_EDEVICE: return "device is not sm_100";
        case PICOATTN_EDEVSTATUS: return "a kernel flagged bad input";
        case PICOATTN_EIO: return "file could not be opened, read or written";
        case PICOATTN_EFORMAT: return "not a KVCP or GGUF file of this shape";
        case PICOATTN_ENOENT: return "no such tensor in the model file";
        default: return "unknown status";
    }
}

const char* picoattn_last_cuda_error(void) {
    return g_last_cuda_error == cudaSuccess ? "no CUDA error" : cudaGetErrorString(g_last_cuda_error);
}

int32_t picoattn_config_check(const picoattn_config_t* c) {
    if (!c) return PICOATTN_EINVAL;
    if (c->n_layers <= 0 || c->n_heads <= 0 || c->n_kv_heads <= 0 || c->max_seq_len <= 0) return PICOATTN_EINVAL;
    if (c->n_heads % c->n_kv_heads != 0) return PICOATTN_EINVAL;
    if (c->head_dim <= 0 || c->head_dim % 2 != 0) return PICOATTN_EINVAL;
    if (c->rope_mode != PICOATTN_ROPE_NEOX && c->rope_mode != PICOATTN_ROPE_INTERLEAVED) return PICOATTN_EINVAL;
    if (!(c->qk_norm_eps >= 0.f) || !(c->rope_freq_base > 0.f)) return PICOATTN_EINVAL;
    if (c->head_dim != 64 && c->head_dim != 128) return PICOATTN_EUNSUPPORTED;
    const int hkv = c->n_kv_heads;
    if (!(hkv == 1 || hkv == 2 || hkv == 4 || hkv == 8)) return PICOATTN_EUNSUPPORTED;
    if (c->n_heads / hkv > 16) return PICOATTN_EUNSUPPORTED;
    return PICOATTN_OK;
}

int32_t picoattn_rope_table(const picoattn_config_t* c, float* cos_out, float* sin_out) {
    if (!c || !cos_out || !sin_out || c->max_seq_len <= 0 || c->head_dim <= 0 || c->head_dim % 2) return PICOATTN_EINVAL;
    const int half = c->head_dim / 2;
    const float base = c->rope_freq_base;
    // Same float expression as Model::allocate_run_state (cpp/model.hpp:1013):
    // powf, a float division and cosf/sinf from the C library.
    for (int p = 0; p < c->max_seq_len; p++) {
        for (int i = 0; i < half; i++) {
            const float theta = (float)p / powf(base, (float)(2 * i) / (float)c->head_dim);
            cos_out[(size_t)p * half + i] = cosf(theta);
            sin_out[(size_t)p * half + i] = sinf(theta);
        }
    }
    return PICOATTN_OK;
}

int32_t picoattn_device_check(void) { return device_ok(); }

int32_t picoattn_workspace_init(void* ws, size_t ws_bytes, picoattn_stream_t stream) {
    if (!ws || ws_bytes < kWsHeaderBytes) return PICOATTN_EINVAL;
    return cuda_status(cudaMemsetAsync(ws, 0, kWsHeaderBytes, (cudaStream_t)stream));
}

int32_t picoattn_workspace_status(void* ws, picoattn_stream_t stream, uint32_t* status_out) {
    if (!ws || !status_out) return PICOATTN_EINVAL;
    unsigned int v = 0;
    cudaError_t e = cudaMemcpyAsync(&v, ws, sizeof v, cudaMemcpyDeviceToHost, (cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(ws, 0, sizeof v, (cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
    *status_out = v;
    return cuda_status(e);
}

size_t picoattn_decode_workspace_size(const picoattn_config_t* cfg, int32_t n_seqs, int32_t max_ctx) {
    if (picoattn_config_check(cfg) != PICOATTN_OK || n_seqs <= 0 || max_ctx <= 0) return 0;
    DecodePlan plan;
    if (!make_decode_plan(*cfg, n_seqs, max_ctx, &plan)) return 0;
    return plan.ws_total;
}

int32_t picoattn_decode(const picoattn_config_t* cfg, int32_t layer, int32_t n_seqs, int32_t max_ctx,
                        const float* q, const float* k, const float* v, const float* q_norm_w,
                        const float* k_norm_w, const float* rope_cos, const float* rope_sin,
                        uint16_t* const* k_cache, uint16_t* const* v_cache, const int32_t* pos, float* out,
                        void* workspace, size_t workspace_bytes, picoattn_stream_t stream) {
    return picoattn_decode_staged(cfg, layer, n_seqs, max_ctx, q, k, v, q_norm_w, k_norm_w, rope_cos, rope_sin,
                                  k_cache, v_cache, pos, out, workspace, workspace_bytes, stream,
                                  PICOATTN_STAGE_ALL);
}

int32_t picoattn_decode_staged(const picoattn_config_t* cfg, int32_t layer, int32_t n_seqs, int32_t max_ctx,
                               const float* q, const float* k, const float* v, const float* q_norm_w,
                               const float* k_norm_w, const float* rope_cos, const float* rope_sin,
                               uint16_t* const* k_cache, uint16_t* const* v_cache, const int32_t* pos,
                               float* out, void* workspace, size_t workspace_bytes, picoattn_stream_t stream,
                               uint32_t stages) {
    if (!k_cache || !v_cache || !pos) return PICOATTN_EINVAL;
    return decode_common(cfg, layer, n_seqs, max_ctx, q, k, v, q_norm_w, k_norm_w, rope_cos, rope_sin, k_cache,
                         v_cache, nullptr, nullptr, pos, 0, out, workspace, workspace_bytes,
                         (cudaStream_t)stream, stages);
}

int32_t picoattn_decode_one(const picoattn_config_t* cfg, int32_t layer, int32_t pos, const float* q,
                            const float* k, const float* v, const float* q_norm_w, const float* k_norm_w,
                            const float* rope_cos, const float* rope_sin, uint16_t* k_cache, uint16_t* v_cache,
                            float* out, void* workspace, size_t workspace_bytes, picoattn_stream_t stream) {
    if (!k_cache || !v_cache) return PICOATTN_EINVAL;
    if (cfg && (pos < 0 || pos >= cfg->max_seq_len)) return PICOATTN_ERANGE;
    return decode_common(cfg, layer, 1, pos + 1, q, k, v, q_norm_w, k_norm_w, rope_cos, rope_sin, nullptr,
                         nullptr, k_cache, v_cache, nullptr, pos, out, workspace, workspace_bytes,
                         (cudaStream_t)stream, PICOATTN_STAGE_ALL);
}

int32_t picoattn_prefill_kernel(const picoattn_config_t* cfg) {
    const int32_t st = picoattn_config_check(cfg);
    if (st != PICOATTN_OK) return st;
    const int32_t d = device_ok();
    if (d != PICOATTN_OK) return d;
    const int v = prefill_kernel_variant(*cfg);
    return v < 0 ? PICOATTN_ECUDA : v;
}

size_t picoattn_prefill_workspace_size(const picoattn_config_t* cfg, int32_t n_tok) {
    if (picoattn_config_check(cfg) != PICOATTN_OK || n_tok <= 0) return 0;
    return prefill_workspace_bytes(*cfg, n_tok);
}

int32_t picoattn_prefill_staged(const picoattn_config_t* cfg, int32_t layer, int32_t n_tok, int32_t start_pos,
                                int32_t in_dtype, const void* q, const void* k, const void* v,
                                const float* q_norm_w, const float* k_norm_w, const float* rope_cos,
                                const float* rope_sin, uint16_t* k_cache, uint16_t* v_cache, float* out,
                                void* workspace, size_t workspace_bytes, picoattn_stream_t stream, uint32_t stages) {
    int32_t st = picoattn_config_check(cfg);
    if (st != PICOATTN_OK) return st;
    if (stages == 0 || (stages & ~(PICOATTN_STAGE_PREPARE | PICOATTN_STAGE_ATTEND))) return PICOATTN_EINVAL;
    if (layer < 0 || layer >= cfg->n_layers || n_tok <= 0) return PICOATTN_EINVAL;
    if (in_dtype != PICOATTN_DTYPE_F32 && in_dtype != PICOATTN_DTYPE_F16) return PICOATTN_EINVAL;
    if (!q || !k || !v || !rope_cos || !rope_sin || !k_cache || !v_cache || !out || !workspace)
        return PICOATTN_EINVAL;
    if ((q_norm_w == nullptr) != (k_norm_w == nullptr)) return PICOATTN_EINVAL;
    if (!aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out)) return PICOATTN_EINVAL;
    if (!aligned16(q) || !aligned16(k) || !aligned16(v)) return PICOATTN_EINVAL;
    if (start_pos < 0 || (int64_t)start_pos + n_tok > cfg->max_seq_len) return PICOATTN_ERANGE;
    if (workspace_bytes < prefill_workspace_bytes(*cfg, n_tok) || !aligned16(workspace)) return PICOATTN_ENOSPACE;
    st = device_ok();
    if (st != PICOATTN_OK) return st;
    uint8_t* w = static_cast<uint8_t*>(workspace);
    PrefillArgs a{};
    a.hq = cfg->n_heads;
    a.hkv = cfg->n_kv_heads;
    a.g = a.hq / a.hkv;
    a.hd = cfg->head_dim;
    a.kvd = a.hkv * a.hd;
    a.max_seq = cfg->max_seq_len;
    a.layer = layer;
    a.n_tok = n_tok;
    a.start = start_pos;
    a.n_qtiles = (n_tok + 127) / 128;
    a.rope_mode = cfg->rope_mode;
    a.in_dtype = in_dtype;
    a.eps = cfg->qk_norm_eps;
    a.q = q, a.k = k, a.v = v, a.qn_w = q_norm_w, a.kn_w = k_norm_w, a.rope_cos = rope_cos, a.rope_sin = rope_sin;
    a.k_cache = k_cache, a.v_cache = v_cache, a.out = out;
    a.status = reinterpret_cast<unsigned int*>(w);
    a.work_counter = reinterpret_cast<int*>(w + 64);
    a.q16 = reinterpret_cast<__half*>(w + kWsHeaderBytes);
    return cuda_status(launch_prefill(a, (cudaStream_t)stream, stages));
}

int32_t picoattn_prefill(const picoattn_config_t* cfg, int32_t layer, int32_t n_tok, int32_t start_pos,
                         int32_t in_dtype, const void* q, const void* k, const void* v, const float* q_norm_w,
                         const float* k_norm_w, const float* rope_cos, const float* rope_sin, uint16_t* k_cache,
                         uint16_t* v_cache, float* out, void* workspace, size_t workspace_bytes,
                         picoattn_stream_t stream) {
    return picoattn_prefill_staged(cfg, layer, n_tok, start_pos, in_dtype, q, k, v, q_norm_w, k_norm_w, rope_cos,
                                   rope_sin, k_cache, v_cache, out, workspace, workspace_bytes, stream,
                                   PICOATTN_STAGE_PREPARE | PICOATTN_STAGE_ATTEND);
}

size_t picoattn_weight_bytes(int32_t w_type, int32_t n_in, int32_t n_out) {
    const int be = weight_block_elems(w_type);
    if (be == 0 || n_in <= 0 || n_out <= 0 || n_in % be != 0) return 0;
    MatvecPart p;
    float dummy;
    if (!matvec_part(w_type, &dummy, nullptr, n_in, n_out, &dummy, 0, &p)) return 0;
    return p.row_bytes * (size_t)n_out;
}

int32_t picoattn_matvec(const void* w, int32_t w_type, const float* bias, int32_t n_in, int32_t n_out,
                        int32_t n_vec, const float* x, float* out, int32_t accumulate, picoattn_stream_t stream) {
    if (!w || !x || !out || n_vec <= 0 || n_in <= 0 || n_out <= 0) return PICOATTN_EINVAL;
    if (weight_block_elems(w_type) == 0) return PICOATTN_EUNSUPPORTED;
    if (!aligned16(x) || !aligned16(out) || ((uintptr_t)w & 3u)) return PICOATTN_EINVAL;
    MatvecArgs a{};
    if (!matvec_part(w_type, w, bias, n_in, n_out, out, (size_t)n_out, &a.part[0])) return PICOATTN_EINVAL;
    const int32_t st = device_ok();
    if (st != PICOATTN_OK) return st;
    a.n_parts = 1;
    a.n_in = n_in;
    a.n_vec = n_vec;
    a.rows_total = n_out;
    a.accumulate = accumulate ? 1 : 0;
    a.x = x;
    return cuda_status(launch_matvec(a, (cudaStream_t)stream));
}

size_t picoattn_decode_layer_workspace_size(const picoattn_config_t* cfg, int32_t dim, int32_t n_seqs,
                                            int32_t max_ctx) {
    if (picoattn_config_check(cfg) != PICOATTN_OK || dim <= 0 || n_seqs <= 0 || max_ctx <= 0) return 0;
    LayerWs l;
    return layer_ws(*cfg, n_seqs, max_ctx, &l) ? l.total : 0;
}

}  // extern "C"

namespace {

// A launch of the tensor-core mat-vec with x formed on the fly (fused norm or
// SwiGLU, MatvecArgs.x_norm_w / x_up); when that kernel does not take the
// launch, the separate kernel first (`unfused`), then the plain mat-vec.
template <class Unfused>
cudaError_t matvec_fused(MatvecArgs a, cudaStream_t s, Unfused&& unfused) {
    const cudaError_t e = launch_matvec_mma(a, s);
    if (e != cudaErrorNotSupported) return e;
    const float* x = nullptr;
    const cudaError_t u = unfused(&x);
    if (u != cudaSuccess) return u;
    a.x = x;
    a.x_norm_w = a.x_up = nullptr;
    return launch_matvec(a, s);
}

// picoattn_decode_layer.  qkv_after_own: the launch before it is this
// library's own (its weights may be read before that kernel finishes).
// attn_norm_w: xb is the raw residual, normalised inside the projection
// launch (or by a norm kernel into xb_scratch when that cannot be).
int32_t decode_layer_impl(const picoattn_config_t* cfg, int32_t layer, int32_t dim, int32_t n_seqs, int32_t max_ctx,
                          const float* xb, const picoattn_layer_weights_t* wt, const float* q_norm_w,
                          const float* k_norm_w, const float* rope_cos, const float* rope_sin,
                          uint16_t* const* k_cache, uint16_t* const* v_cache, const int32_t* pos, float* x,
                          void* workspace, size_t workspace_bytes, picoattn_stream_t stream, bool qkv_after_own,
                          const float* attn_norm_w = nullptr, float* xb_scratch = nullptr) {
    int32_t st = picoattn_config_check(cfg);
    if (st != PICOATTN_OK) return st;
    if (!wt || !xb || !x || !k_cache || !v_cache || !pos || !workspace || dim <= 0 || n_seqs <= 0)
        return PICOATTN_EINVAL;
    if (!aligned16(xb) || !aligned16(x) || !aligned16(workspace)) return PICOATTN_EINVAL;
    const int qd = cfg->n_heads * cfg->head_dim, kvd = cfg->n_kv_heads * cfg->head_dim;
    LayerWs l;
    if (max_ctx <= 0 || max_ctx > cfg->max_seq_len) return PICOATTN_ERANGE;
    if (!layer_ws(*cfg, n_seqs, max_ctx, &l)) return PICOATTN_EUNSUPPORTED;
    if (workspace_bytes < l.total) return PICOATTN_ENOSPACE;
    uint8_t* w = static_cast<uint8_t*>(workspace);
    float* q = reinterpret_cast<float*>(w + l.q);
    float* k = reinterpret_cast<float*>(w + l.k);
    float* v = reinterpret_cast<float*>(w + l.v);
    float* attn = reinterpret_cast<float*>(w + l.attn);
    for (int32_t t : {wt->wq_type, wt->wk_type, wt->wv_type, wt->wo_type})
        if (weight_block_elems(t) == 0) return PICOATTN_EUNSUPPORTED;
    MatvecArgs qkv{};
    if (!matvec_part(wt->wq_type, wt->wq, wt->bq, dim, qd, q, (size_t)qd, &qkv.part[0]) ||
        !matvec_part(wt->wk_type, wt->wk, wt->bk, dim, kvd, k, (size_t)kvd, &qkv.part[1]) ||
        !matvec_part(wt->wv_type, wt->wv, wt->bv, dim, kvd, v, (size_t)kvd, &qkv.part[2]))
        return PICOATTN_EINVAL;
    MatvecArgs o{};
    if (!matvec_part(wt->wo_type, wt->wo, wt->bo, qd, dim, x, (size_t)dim, &o.part[0])) return PICOATTN_EINVAL;
    st = device_ok();
    if (st != PICOATTN_OK) return st;
    const cudaStream_t s = (cudaStream_t)stream;
    qkv.n_parts = 3;
    qkv.n_in = dim;
    qkv.n_vec = n_seqs;
    qkv.rows_total = qd + 2 * kvd;
    qkv.x = xb;
    qkv.weights_ready = qkv_after_own ? 1 : 0;
    if (attn_norm_w) {
        qkv.x_norm_w = attn_norm_w;
        st = cuda_status(matvec_fused(qkv, s, [&](const float** xo) {
            *xo = xb_scratch;
            return launch_rmsnorm(xb, attn_norm_w, xb_scratch, dim, n_seqs, s);
        }));
    } else {
        st = cuda_status(launch_matvec(qkv, s));
    }
    if (st != PICOATTN_OK) return st;
    st = decode_common(cfg, layer, n_seqs, max_ctx, q, k, v, q_norm_w, k_norm_w, rope_cos, rope_sin, k_cache,
                       v_cache, nullptr, nullptr, pos, 0, attn, workspace, l.q, s, PICOATTN_STAGE_ALL);
    if (st != PICOATTN_OK) return st;
    o.n_parts = 1;
    o.n_in = qd;
    o.n_vec = n_seqs;
    o.rows_total = dim;
    o.accumulate = 1;
    o.x = attn;
    o.weights_ready = 1;  // after the decode kernels
    return cuda_status(launch_matvec(o, s));
}

}  // namespace

extern "C" {

int32_t picoattn_decode_layer(const picoattn_config_t* cfg, int32_t layer, int32_t dim, int32_t n_seqs,
                              int32_t max_ctx, const float* xb, const picoattn_layer_weights_t* wt,
                              const float* q_norm_w, const float* k_norm_w, const float* rope_cos,
                              const float* rope_sin, uint16_t* const* k_cache, uint16_t* const* v_cache,
                              const int32_t* pos, float* x, void* workspace, size_t workspace_bytes,
                              picoattn_stream_t stream) {
    return decode_layer_impl(cfg, layer, dim, n_seqs, max_ctx, xb, wt, q_norm_w, k_norm_w, rope_cos, rope_sin,
                             k_cache, v_cache, pos, x, workspace, workspace_bytes, stream, false);
}

size_t picoattn_ffn_workspace_size(int32_t dim, int32_t n_ffn, int32_t n_vec) {
    if (dim <= 0 || n_ffn <= 0 || n_vec <= 0) return 0;
    // xb [n_vec][dim], gate and up [n_vec][n_ffn], fp32; then the down
    // projection's x fragments (one vector, n_ffn a multiple of 256)
    return align_up((size_t)n_vec * dim * 4, 256) + 2 * align_up((size_t)n_vec * n_ffn * 4, 256) +
           align_up(xfrag_bytes(n_ffn), 256);
}

int32_t picoattn_rmsnorm(const float* x, const float* weight, float* out, int32_t dim, int32_t n_vec,
                         picoattn_stream_t stream) {
    if (!x || !weight || !out || dim <= 0 || n_vec <= 0) return PICOATTN_EINVAL;
    if (!aligned16(x) || !aligned16(out) || !aligned16(weight)) return PICOATTN_EINVAL;
    const int32_t st = device_ok();
    if (st != PICOATTN_OK) return st;
    return cuda_status(launch_rmsnorm(x, weight, out, dim, n_vec, (cudaStream_t)stream));
}

}  // extern "C"

namespace {

// picoattn_ffn; after_own: the launch before it is this library's own
int32_t ffn_impl(const picoattn_ffn_weights_t* w, const float* ffn_norm_w, int32_t dim, int32_t n_ffn, int32_t n_vec,
                 float* x, void* workspace, size_t workspace_bytes, picoattn_stream_t stream, bool after_own) {
    if (!w || !ffn_norm_w || !x || !workspace || dim <= 0 || n_ffn <= 0 || n_vec <= 0) return PICOATTN_EINVAL;
    if (!aligned16(x) || !aligned16(workspace) || !aligned16(ffn_norm_w)) return PICOATTN_EINVAL;
    for (int32_t t : {w->gate_type, w->up_type, w->down_type})
        if (weight_block_elems(t) == 0) return PICOATTN_EUNSUPPORTED;
    if (workspace_bytes < picoattn_ffn_workspace_size(dim, n_ffn, n_vec)) return PICOATTN_ENOSPACE;
    uint8_t* base = static_cast<uint8_t*>(workspace);
    float* xb = reinterpret_cast<float*>(base);
    float* gate = reinterpret_cast<float*>(base + align_up((size_t)n_vec * dim * 4, 256));
    float* up = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(gate) + align_up((size_t)n_vec * n_ffn * 4, 256));
    MatvecArgs gu{};
    if (!matvec_part(w->gate_type, w->w_gate, w->b_gate, dim, n_ffn, gate, (size_t)n_ffn, &gu.part[0]) ||
        !matvec_part(w->up_type, w->w_up, nullptr, dim, n_ffn, up, (size_t)n_ffn, &gu.part[1]))
        return PICOATTN_EINVAL;
    MatvecArgs dn{};
    if (!matvec_part(w->down_type, w->w_down, w->b_down, n_ffn, dim, x, (size_t)dim, &dn.part[0]))
        return PICOATTN_EINVAL;
    int32_t st = device_ok();
    if (st != PICOATTN_OK) return st;
    const cudaStream_t s = (cudaStream_t)stream;
    // norm, gate and up in one launch when the tensor-core kernel takes it
    gu.n_parts = 2;
    gu.n_in = dim;
    gu.n_vec = n_vec;
    gu.rows_total = 2 * n_ffn;
    gu.x = x;
    gu.x_norm_w = ffn_norm_w;
    gu.weights_ready = after_own ? 1 : 0;
    st = cuda_status(matvec_fused(gu, s, [&](const float** xo) {
        *xo = xb;
        return launch_rmsnorm(x, ffn_norm_w, xb, dim, n_vec, s);
    }));
    if (st != PICOATTN_OK) return st;
    // SwiGLU and the down projection: x's fragments made once by a small
    // kernel (each down block would otherwise prepare the whole n_ffn-long x),
    // else SwiGLU inside the down launch, else the separate kernels
    dn.n_parts = 1;
    dn.n_in = n_ffn;
    dn.n_vec = n_vec;
    dn.rows_total = dim;
    dn.accumulate = 1;
    dn.x = gate;
    dn.weights_ready = 1;  // after the gate/up launch
    uint32_t* xfrag = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(up) +
                                                  align_up((size_t)n_vec * n_ffn * 4, 256));
    if (n_vec == 1 && xfrag_bytes(n_ffn) > 0) {
        const bool pairs = w->down_type == PICOATTN_WT_Q4_K;
        MatvecArgs pre = dn;
        pre.xfrag = xfrag;
        pre.xfrag_pairs = pairs ? 1 : 0;
        const cudaError_t e = launch_xfrag(gate, up, n_ffn, pairs, xfrag, s);
        if (e != cudaErrorNotSupported) {
            if (e != cudaSuccess) return cuda_status(e);
            const cudaError_t m = launch_matvec_mma(pre, s);
            if (m != cudaErrorNotSupported) return cuda_status(m);
        }
    }
    dn.x_up = up;
    return cuda_status(matvec_fused(dn, s, [&](const float** xo) {
        *xo = gate;
        return launch_silu_mul(gate, up, (size_t)n_vec * n_ffn, s);
    }));
}

}  // namespace

extern "C" {

int32_t picoattn_ffn(const picoattn_ffn_weights_t* w, const float* ffn_norm_w, int32_t dim, int32_t n_ffn,
                     int32_t n_vec, float* x, void* workspace, size_t workspace_bytes, picoattn_stream_t stream) {
    return ffn_impl(w, ffn_norm_w, dim, n_ffn, n_vec, x, workspace, workspace_bytes, stream, false);
}

size_t picoattn_logits_workspace_size(int32_t dim, int32_t n_vec) {
    if (dim <= 0 || n_vec <= 0) return 0;
    return align_up((size_t)n_vec * dim * 4, 256);
}

int32_t picoattn_logits(const float* x, const float* output_norm_w, const void* w_out, int32_t w_type, int32_t dim,
                        int32_t vocab, int32_t n_vec, float* logits, void* workspace, size_t workspace_bytes,
                        picoattn_stream_t stream) {
    if (!x || !output_norm_w || !w_out || !logits || !workspace || dim <= 0 || vocab <= 0 || n_vec <= 0)
        return PICOATTN_EINVAL;
    if (!aligned16(x) || !aligned16(logits) || !aligned16(workspace) || !aligned16(output_norm_w))
        return PICOATTN_EINVAL;
    if (weight_block_elems(w_type) == 0) return PICOATTN_EUNSUPPORTED;
    if (workspace_bytes < picoattn_logits_workspace_size(dim, n_vec)) return PICOATTN_ENOSPACE;
    float* xb = static_cast<float*>(workspace);
    MatvecArgs a{};
    if (!matvec_part(w_type, w_out, nullptr, dim, vocab, logits, (size_t)vocab, &a.part[0])) return PICOATTN_EINVAL;
    int32_t st = device_ok();
    if (st != PICOATTN_OK) return st;
    const cudaStream_t s = (cudaStream_t)stream;
    a.n_parts = 1;
    a.n_in = dim;
    a.n_vec = n_vec;
    a.rows_total = vocab;
    a.x = x;
    a.x_norm_w = output_norm_w;  // the final norm inside the launch when it can be
    return cuda_status(matvec_fused(a, s, [&](const float** xo) {
        *xo = xb;
        return launch_rmsnorm(x, output_norm_w, xb, dim, n_vec, s);
    }));
}

// Workspace of picoattn_decode_block: the decode-layer workspace first (its
// status header at offset 0), then the normalised hidden state xb, then the
// FFN's workspace.
size_t picoattn_decode_block_workspace_size(const picoattn_config_t* cfg, int32_t dim, int32_t n_ffn,
                                            int32_t n_seqs, int32_t max_ctx) {
    const size_t l = picoattn_decode_layer_workspace_size(cfg, dim, n_seqs, max_ctx);
    const size_t f = picoattn_ffn_workspace_size(dim, n_ffn, n_seqs);
    if (l == 0 || f == 0) return 0;
    return align_up(l, 256) + align_up((size_t)n_seqs * dim * 4, 256) + f;
}

int32_t picoattn_decode_block(const picoattn_config_t* cfg, int32_t layer, int32_t dim, int32_t n_ffn,
                              int32_t n_seqs, int32_t max_ctx, const float* attn_norm_w,
                              const picoattn_layer_weights_t* attn_weights, const float* ffn_norm_w,
                              const picoattn_ffn_weights_t* ffn_weights, const float* q_norm_w,
                              const float* k_norm_w, const float* rope_cos, const float* rope_sin,
                              uint16_t* const* k_cache, uint16_t* const* v_cache, const int32_t* pos, float* x,
                              void* workspace, size_t workspace_bytes, picoattn_stream_t stream) {
    if (!attn_norm_w || !x || !workspace || dim <= 0 || n_seqs <= 0 || n_ffn <= 0) return PICOATTN_EINVAL;
    if (!aligned16(attn_norm_w) || !aligned16(x) || !aligned16(workspace)) return PICOATTN_EINVAL;
    const size_t l = picoattn_decode_layer_workspace_size(cfg, dim, n_seqs, max_ctx);
    if (l == 0) return picoattn_config_check(cfg) != PICOATTN_OK ? picoattn_config_check(cfg) : PICOATTN_EINVAL;
    const size_t total = picoattn_decode_block_workspace_size(cfg, dim, n_ffn, n_seqs, max_ctx);
    if (workspace_bytes < total) return PICOATTN_ENOSPACE;
    uint8_t* base = static_cast<uint8_t*>(workspace);
    float* xb = reinterpret_cast<float*>(base + align_up(l, 256));
    uint8_t* ffn_ws = base + align_up(l, 256) + align_up((size_t)n_seqs * dim * 4, 256);
    // the attention norm inside the q/k/v launch (into xb only when that
    // launch cannot take it), then the FFN after this call's own kernels
    int32_t st = decode_layer_impl(cfg, layer, dim, n_seqs, max_ctx, x, attn_weights, q_norm_w, k_norm_w, rope_cos,
                                   rope_sin, k_cache, v_cache, pos, x, workspace, l, stream, false, attn_norm_w, xb);
    if (st != PICOATTN_OK) return st;
    return ffn_impl(ffn_weights, ffn_norm_w, dim, n_ffn, n_seqs, x, ffn_ws,
                    picoattn_ffn_workspace_size(dim, n_ffn, n_seqs), stream, true);
}

}  // extern "C"
