// p2p_exchange.cu -- split-KV decode across the GPUs of one node with the
// shard-result exchange and the log-sum-exp combine done by the merge kernel
// over peer memory (NVLink stores and flags), instead of a library all-gather
// followed by a combine kernel.  The kernel side is exchange_slice
// (decode.cu); this file owns the exchange areas: each rank allocates one and
// exports it to the other ranks' processes by a CUDA IPC handle.  Layout
// (picoattn_internal.h, XchgArgs): per-slice slots of (value, sequence) words
// and call counters, plus the rank's local shard buffer.  The counters live in device memory, so
// a captured CUDA graph replays correctly.
#include <cstring>

#include <cuda_runtime.h>

#include "device_common.cuh"
#include "picoattn.h"
#include "picoattn_internal.h"

using namespace picoattn;

namespace {

constexpr int kMaxRanks = 8;

struct Layout {
    int n_ranks, n_seqs, hq, hd;
    size_t slots, counters, shard, total;
};

Layout make_layout(int n_ranks, int n_seqs, int hq, int hd) {
    Layout l{};
    l.n_ranks = n_ranks, l.n_seqs = n_seqs, l.hq = hq, l.hd = hd;
    const size_t rows = (size_t)n_seqs * hq * (hd / kXchgCols);  // exchanged slices
    l.slots = 0;
    l.counters = align_up(l.slots + 2ull * n_ranks * rows * kXchgWords * sizeof(uint64_t), 256);
    l.shard = align_up(l.counters + rows * sizeof(uint32_t), 256);
    l.total = align_up(l.shard + (size_t)n_seqs * hq * (hd + 2) * sizeof(float), 256);
    return l;
}

struct P2PComm {
    Layout lay;
    int rank = 0;
    uint8_t* local = nullptr;
    uint8_t* peer[kMaxRanks] = {};
    bool imported[kMaxRanks] = {};
    uint8_t** peers_dev = nullptr;
    bool open = false;
    int device = 0;
    unsigned long long timeout_ns = 2000000000ull;  // the exchange wait's bound
};

P2PComm* as_comm(void* c) { return static_cast<P2PComm*>(c); }

}  // namespace

extern "C" {

size_t picoattn_p2p_area_bytes(const picoattn_config_t* cfg, int32_t n_seqs, int32_t n_ranks) {
    if (picoattn_config_check(cfg) != PICOATTN_OK || n_seqs <= 0 || n_ranks <= 0 || n_ranks > kMaxRanks) return 0;
    return make_layout(n_ranks, n_seqs, cfg->n_heads, cfg->head_dim).total;
}

int32_t picoattn_p2p_create(const picoattn_config_t* cfg, int32_t n_seqs, int32_t n_ranks, int32_t rank,
                            void* ipc_handle_out, void** comm_out) {
    int32_t st = picoattn_config_check(cfg);
    if (st != PICOATTN_OK) return st;
    if (!ipc_handle_out || !comm_out || n_seqs <= 0 || n_ranks <= 0 || n_ranks > kMaxRanks || rank < 0 ||
        rank >= n_ranks)
        return PICOATTN_EINVAL;
    if (cfg->head_dim != 64 && cfg->head_dim != 128) return PICOATTN_EUNSUPPORTED;
    st = picoattn_device_check();
    if (st != PICOATTN_OK) return st;
    auto* c = new P2PComm();
    c->lay = make_layout(n_ranks, n_seqs, cfg->n_heads, cfg->head_dim);
    c->rank = rank;
    cudaGetDevice(&c->device);
    cudaIpcMemHandle_t h;
    if (cudaMalloc(&c->local, c->lay.total) != cudaSuccess || cudaMemset(c->local, 0, c->lay.total) != cudaSuccess ||
        cudaMalloc(&c->peers_dev, sizeof(uint8_t*) * kMaxRanks) != cudaSuccess ||
        cudaIpcGetMemHandle(&h, c->local) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        if (c->local) cudaFree(c->local);
        if (c->peers_dev) cudaFree(c->peers_dev);
        delete c;
        return PICOATTN_ECUDA;
    }
    static_assert(sizeof(cudaIpcMemHandle_t) <= PICOATTN_P2P_HANDLE_BYTES, "IPC handle size");
    std::memset(ipc_handle_out, 0, PICOATTN_P2P_HANDLE_BYTES);
    std::memcpy(ipc_handle_out, &h, sizeof h);
    *comm_out = c;
    return PICOATTN_OK;
}

int32_t picoattn_p2p_open(void* comm, const void* ipc_handles) {
    P2PComm* c = as_comm(comm);
    if (!c || !ipc_handles || c->open) return PICOATTN_EINVAL;
    const auto* hb = static_cast<const uint8_t*>(ipc_handles);
    for (int p = 0; p < c->lay.n_ranks; p++) {
        if (p == c->rank) {
            c->peer[p] = c->local;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, hb + (size_t)p * PICOATTN_P2P_HANDLE_BYTES, sizeof h);
        void* ptr = nullptr;
        if (cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return PICOATTN_ECUDA;
        c->peer[p] = static_cast<uint8_t*>(ptr);
        c->imported[p] = true;
    }
    if (cudaMemcpy(c->peers_dev, c->peer, sizeof(uint8_t*) * kMaxRanks, cudaMemcpyHostToDevice) != cudaSuccess)
        return PICOATTN_ECUDA;
    c->open = true;
    return PICOATTN_OK;
}

int32_t picoattn_p2p_set_timeout(void* comm, double timeout_s) {
    P2PComm* c = as_comm(comm);
    if (!c || !(timeout_s > 0.0) || timeout_s > 60.0) return PICOATTN_EINVAL;
    c->timeout_ns = (unsigned long long)(timeout_s * 1e9);
    return PICOATTN_OK;
}

int32_t picoattn_p2p_destroy(void* comm) {
    P2PComm* c = as_comm(comm);
    if (!c) return PICOATTN_EINVAL;
    cudaDeviceSynchronize();
    for (int p = 0; p < c->lay.n_ranks; p++)
        if (c->imported[p]) cudaIpcCloseMemHandle(c->peer[p]);
    cudaFree(c->peers_dev);
    cudaFree(c->local);
    delete c;
    return PICOATTN_OK;
}

int32_t picoattn_decode_splitkv_p2p(const picoattn_config_t* cfg, int32_t layer, int32_t n_seqs, int32_t max_ctx,
                                    int32_t row_offset, int32_t local_rows, const float* q, const float* k,
                                    const float* v, const float* q_norm_w, const float* k_norm_w,
                                    const float* rope_cos, const float* rope_sin, uint16_t* const* k_cache,
                                    uint16_t* const* v_cache, const int32_t* pos, float* out, void* workspace,
                                    size_t workspace_bytes, void* comm, picoattn_stream_t stream) {
    P2PComm* c = as_comm(comm);
    if (!c || !c->open || !out || ((uintptr_t)out & 15u)) return PICOATTN_EINVAL;
    if (cfg && (cfg->n_heads != c->lay.hq || cfg->head_dim != c->lay.hd || n_seqs != c->lay.n_seqs))
        return PICOATTN_EINVAL;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != c->device) return PICOATTN_EINVAL;
    XchgArgs x{};
    x.peers = c->peers_dev;
    x.slots = c->lay.slots;
    x.counters = c->lay.counters;
    x.rank = c->rank;
    x.n_ranks = c->lay.n_ranks;
    x.out = out;
    x.timeout_ns = c->timeout_ns;
    float* shard = reinterpret_cast<float*>(c->local + c->lay.shard);
    return decode_shard_impl(cfg, layer, n_seqs, max_ctx, row_offset, local_rows, q, k, v, q_norm_w, k_norm_w,
                             rope_cos, rope_sin, k_cache, v_cache, pos, shard, workspace, workspace_bytes,
                             static_cast<cudaStream_t>(stream), &x);
}

}  // extern "C"
