// nccl_comm.cpp -- NCCL plumbing for split-KV decode across GPUs.
//
// One process per GPU.  Communicators are created non-blocking
// (ncclCommInitRankConfig, blocking = 0) and polled with ncclCommGetAsyncError
// under a host deadline; a rank that never joins turns into PICOATTN_ETIMEOUT
// and an aborted communicator (ncclCommAbort), never a hang.
#include <chrono>
#include <cstring>
#include <thread>

#include <cuda_runtime.h>
#include <nccl.h>

#include "picoattn.h"
#include "picoattn_internal.h"

namespace picoattn {
cudaError_t launch_combine_shards(const float* parts, float* out, int n_seqs, int hq, int hd, int n_shards,
                                  cudaStream_t stream);
}  // namespace picoattn

using namespace picoattn;

namespace {

struct Comm {
    ncclComm_t comm = nullptr;
    int n_ranks = 0, rank = 0;
    double timeout_s = 60.0;
};

// Waits until the communicator's pending work has been enqueued (non-blocking
// communicators return ncclInProgress from calls that are not yet done).
int32_t settle(Comm* c, ncclResult_t r) {
    if (r != ncclSuccess && r != ncclInProgress) return PICOATTN_ENCCL;
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::duration<double>(c->timeout_s);
    ncclResult_t state = r;
    while (state == ncclInProgress) {
        if (ncclCommGetAsyncError(c->comm, &state) != ncclSuccess) return PICOATTN_ENCCL;
        if (state == ncclInProgress) {
            if (std::chrono::steady_clock::now() > deadline) {
                ncclCommAbort(c->comm);
                c->comm = nullptr;
                return PICOATTN_ETIMEOUT;
            }
            std::this_thread::sleep_for(std::chrono::microseconds(50));
        }
    }
    return state == ncclSuccess ? PICOATTN_OK : PICOATTN_ENCCL;
}

}  // namespace

extern "C" {

int32_t picoattn_nccl_unique_id(void* id_out) {
    if (!id_out) return PICOATTN_EINVAL;
    ncclUniqueId id;
    if (ncclGetUniqueId(&id) != ncclSuccess) return PICOATTN_ENCCL;
    std::memcpy(id_out, &id, sizeof id);
    return PICOATTN_OK;
}

int32_t picoattn_nccl_comm_create(int32_t n_ranks, const void* id, int32_t rank, double timeout_s, void** comm_out) {
    if (!id || !comm_out || n_ranks <= 0 || rank < 0 || rank >= n_ranks || !(timeout_s > 0)) return PICOATTN_EINVAL;
    auto* c = new Comm();
    c->n_ranks = n_ranks;
    c->rank = rank;
    c->timeout_s = timeout_s;
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof uid);
    ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
    config.blocking = 0;
    ncclResult_t r = ncclCommInitRankConfig(&c->comm, n_ranks, uid, rank, &config);
    int32_t st = settle(c, r);
    if (st != PICOATTN_OK) {
        if (c->comm) ncclCommAbort(c->comm);
        delete c;
        return st;
    }
    *comm_out = c;
    return PICOATTN_OK;
}

int32_t picoattn_nccl_comm_destroy(void* comm) {
    auto* c = static_cast<Comm*>(comm);
    if (!c) return PICOATTN_EINVAL;
    int32_t st = PICOATTN_OK;
    if (c->comm) {
        ncclResult_t r = ncclCommFinalize(c->comm);
        st = settle(c, r);
        if (c->comm) ncclCommDestroy(c->comm);
    }
    delete c;
    return st;
}

size_t picoattn_splitkv_gather_bytes(const picoattn_config_t* cfg, int32_t n_seqs, int32_t n_ranks) {
    if (picoattn_config_check(cfg) != PICOATTN_OK || n_seqs <= 0 || n_ranks <= 0) return 0;
    return (size_t)n_ranks * n_seqs * cfg->n_heads * (cfg->head_dim + 2) * sizeof(float);
}

int32_t picoattn_decode_splitkv_nccl(const picoattn_config_t* cfg, int32_t layer, int32_t n_seqs, int32_t max_ctx,
                                     int32_t row_offset, int32_t local_rows, const float* q, const float* k,
                                     const float* v, const float* q_norm_w, const float* k_norm_w,
                                     const float* rope_cos, const float* rope_sin, uint16_t* const* k_cache,
                                     uint16_t* const* v_cache, const int32_t* pos, float* gather, float* out,
                                     void* workspace, size_t workspace_bytes, void* comm, picoattn_stream_t stream) {
    auto* c = static_cast<Comm*>(comm);
    if (!c || !c->comm || !gather || !out) return PICOATTN_EINVAL;
    const size_t per = (size_t)n_seqs * cfg->n_heads * (cfg->head_dim + 2);
    float* mine = gather + per * c->rank;
    int32_t st = decode_shard_impl(cfg, layer, n_seqs, max_ctx, row_offset, local_rows, q, k, v, q_norm_w, k_norm_w,
                                   rope_cos, rope_sin, k_cache, v_cache, pos, mine, workspace, workspace_bytes,
                                   (cudaStream_t)stream, nullptr);
    if (st != PICOATTN_OK) return st;
    st = settle(c, ncclAllGather(mine, gather, per, ncclFloat, c->comm, (cudaStream_t)stream));
    if (st != PICOATTN_OK) return st;
    return launch_combine_shards(gather, out, n_seqs, cfg->n_heads, cfg->head_dim, c->n_ranks,
                                 (cudaStream_t)stream) == cudaSuccess
               ? PICOATTN_OK
               : PICOATTN_ECUDA;
}

}  // extern "C"
