// splitkv.cu -- decode over a shard of the cache rows, and the log-sum-exp
// combination of shard results (long-context decode split across GPUs).
//
// The reference attends rows 0..pos in one loop (cpp/model.hpp:378-413).  Split
// across G devices, device g holds absolute positions [row_offset,
// row_offset + local_rows) of every layer and computes, per q head, the softmax
// over its rows only: o_g = sum_t e^(s_t) v_t / sum_t e^(s_t) and
// lse_g = log2 sum_t 2^(s_t log2 e).  Any device then recovers the reference's
// result exactly as  sum_g 2^(lse_g - L) o_g,  L = log2 sum_g 2^lse_g.
#include <cmath>

#include "device_common.cuh"
#include "picoattn.h"
#include "picoattn_internal.h"

namespace picoattn {

namespace {

template <int HD>
__global__ void __launch_bounds__(HD) combine_shards_kernel(const float* __restrict__ parts, float* __restrict__ out,
                                                            int n_seqs, int hq, int n_shards) {
    const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
    const size_t stride_shard = (size_t)n_seqs * hq * (HD + 2);
    const float* p = parts + ((size_t)b * hq + h) * (HD + 2);
    float M = -INFINITY;
    for (int s = 0; s < n_shards; s++) M = fmaxf(M, p[s * stride_shard + HD]);
    float L = 0.f, acc = 0.f;
    for (int s = 0; s < n_shards; s++) {
        const float lse = p[s * stride_shard + HD];
        if (lse == -INFINITY) continue;  // a shard without rows of this sequence
        const float w = ex2(lse - M);
        L += w;
        acc += w * p[s * stride_shard + d];
    }
    out[((size_t)b * hq + h) * HD + d] = acc / L;
}

}  // namespace

cudaError_t launch_combine_shards(const float* parts, float* out, int n_seqs, int hq, int hd, int n_shards,
                                  cudaStream_t stream) {
    dim3 grid((unsigned)hq, (unsigned)n_seqs);
    if (hd == 64) combine_shards_kernel<64><<<grid, 64, 0, stream>>>(parts, out, n_seqs, hq, n_shards);
    else combine_shards_kernel<128><<<grid, 128, 0, stream>>>(parts, out, n_seqs, hq, n_shards);
    return cudaGetLastError();
}

int32_t decode_shard_impl(const picoattn_config_t* cfg, int32_t layer, int32_t n_seqs, int32_t max_ctx,
                          int32_t row_offset, int32_t local_rows, const float* q, const float* k, const float* v,
                          const float* qn, const float* kn, const float* rc, const float* rs,
                          uint16_t* const* kcp, uint16_t* const* vcp, const int32_t* pos, float* partial, void* ws,
                          size_t ws_bytes, cudaStream_t stream, const XchgArgs* x) {
    int32_t st = picoattn_config_check(cfg);
    if (st != PICOATTN_OK) return st;
    if (layer < 0 || layer >= cfg->n_layers || n_seqs <= 0) return PICOATTN_EINVAL;
    if (!q || !k || !v || !rc || !rs || !kcp || !vcp || !pos || !partial || !ws) return PICOATTN_EINVAL;
    if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)partial) & 15u) return PICOATTN_EINVAL;
    if ((qn == nullptr) != (kn == nullptr)) return PICOATTN_EINVAL;
    if (local_rows <= 0 || row_offset < 0 || (int64_t)row_offset + local_rows > cfg->max_seq_len)
        return PICOATTN_ERANGE;
    if (max_ctx <= 0 || max_ctx > local_rows) return PICOATTN_ERANGE;
    DecodePlan plan;
    if (!make_decode_plan(*cfg, n_seqs, max_ctx, &plan)) return PICOATTN_EUNSUPPORTED;
    if (ws_bytes < plan.ws_total || ((uintptr_t)ws & 15u)) return PICOATTN_ENOSPACE;
    st = picoattn_device_check();
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
    a.kc_ptrs = kcp, a.vc_ptrs = vcp, a.kc_one = nullptr, a.vc_one = nullptr;
    a.pos_dev = pos, a.pos_host = 0, a.out = nullptr;
    a.status = reinterpret_cast<unsigned int*>(w);
    a.q_rot = reinterpret_cast<float*>(w + plan.ws_qrot);
    a.part_ml = reinterpret_cast<float*>(w + plan.ws_ml);
    a.part_o = reinterpret_cast<float*>(w + plan.ws_o);
    a.n_slots = plan.n_slots;
    a.prefix = reinterpret_cast<long long*>(w + plan.ws_prefix);
    a.row_offset = row_offset;
    a.local_rows = local_rows;
    a.shard_out = partial;
    if (x) a.x = *x;
    a.tile_rows = plan.tile_rows;
    a.stages = plan.stages;
    a.warps_per_head = plan.warps_per_head;
    a.compute_warps = plan.compute_warps;
    return cuda_status(launch_decode(a, plan, stream, PICOATTN_STAGE_ALL));
}

}  // namespace picoattn

using namespace picoattn;

extern "C" {

size_t picoattn_shard_partial_bytes(const picoattn_config_t* cfg, int32_t n_seqs) {
    if (picoattn_config_check(cfg) != PICOATTN_OK || n_seqs <= 0) return 0;
    return (size_t)n_seqs * cfg->n_heads * (cfg->head_dim + 2) * sizeof(float);
}

int32_t picoattn_decode_shard(const picoattn_config_t* cfg, int32_t layer, int32_t n_seqs, int32_t max_ctx,
                              int32_t row_offset, int32_t local_rows, const float* q, const float* k, const float* v,
                              const float* q_norm_w, const float* k_norm_w, const float* rope_cos,
                              const float* rope_sin, uint16_t* const* k_cache, uint16_t* const* v_cache,
                              const int32_t* pos, float* partial, void* workspace, size_t workspace_bytes,
                              picoattn_stream_t stream) {
    return decode_shard_impl(cfg, layer, n_seqs, max_ctx, row_offset, local_rows, q, k, v, q_norm_w, k_norm_w,
                             rope_cos, rope_sin, k_cache, v_cache, pos, partial, workspace, workspace_bytes,
                             (cudaStream_t)stream, nullptr);
}

int32_t picoattn_combine_shards(const picoattn_config_t* cfg, int32_t n_seqs, int32_t n_shards,
                                const float* partials, float* out, picoattn_stream_t stream) {
    int32_t st = picoattn_config_check(cfg);
    if (st != PICOATTN_OK) return st;
    if (n_seqs <= 0 || n_shards <= 0 || !partials || !out) return PICOATTN_EINVAL;
    st = picoattn_device_check();
    if (st != PICOATTN_OK) return st;
    return cuda_status(
        launch_combine_shards(partials, out, n_seqs, cfg->n_heads, cfg->head_dim, n_shards, (cudaStream_t)stream));
}

}  // extern "C"
