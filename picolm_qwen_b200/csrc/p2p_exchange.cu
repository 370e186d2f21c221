// p2p_exchange.cu -- split-KV decode across the GPUs of one node with the
// shard-result exchange and the log-sum-exp combine in ONE kernel over peer
// memory (NVLink stores), instead of a library all-gather followed by a
// combine kernel.
//
// Each rank owns an exchange area, exported to the other ranks' processes by a
// CUDA IPC handle:
//   slots    [2 parities][n_ranks][n_seqs][hq][ROW] fp32   ROW = hd + 4: the
//            normalised shard output (hd), its log2-sum-exp, padding
//   flags    [2 parities][n_ranks][n_seqs][hq] u32      written by the source rank
//   counters [n_seqs][hq] u32                           calls so far, this rank only
//   shard    [n_seqs][hq][hd + 2] fp32                  this rank's decode result
// Per call, block (head h, sequence b) bumps its counter to `seq` (all ranks make
// the same calls, so their counters advance in lockstep), stores its shard row
// into slot [seq % 2][rank][b][h] of every rank's area, then -- after a
// system-scope fence -- sets flag [seq % 2][rank][b][h] = seq there; it then
// waits (bounded) until every rank's flag in its own area reads seq and combines
// the rows: out = sum_r 2^(lse_r - L) o_r, L = log2 sum_r 2^lse_r, exactly as
// picoattn_combine_shards.  Parity double-buffering makes slot reuse safe: a rank
// writes call n+2 into a slot only after its call n+1 saw every rank's call n+1
// flag, which each rank raised after finishing its call n.  The counters live in
// device memory, so a captured CUDA graph replays correctly.
#include <cstring>

#include <cuda_runtime.h>

#include "device_common.cuh"
#include "picoattn.h"
#include "picoattn_internal.h"

namespace picoattn {
int32_t decode_shard_impl(const picoattn_config_t* cfg, int32_t layer, int32_t n_seqs, int32_t max_ctx,
                          int32_t row_offset, int32_t local_rows, const float* q, const float* k, const float* v,
                          const float* qn, const float* kn, const float* rc, const float* rs,
                          uint16_t* const* kcp, uint16_t* const* vcp, const int32_t* pos, float* partial, void* ws,
                          size_t ws_bytes, cudaStream_t stream);
}  // namespace picoattn

using namespace picoattn;

namespace {

constexpr int kMaxRanks = 8;

struct Layout {
    int n_ranks, n_seqs, hq, hd, row;
    size_t slots, flags, counters, shard, total;
};

Layout make_layout(int n_ranks, int n_seqs, int hq, int hd) {
    Layout l{};
    l.n_ranks = n_ranks, l.n_seqs = n_seqs, l.hq = hq, l.hd = hd, l.row = hd + 4;
    const size_t rows = (size_t)n_seqs * hq;
    l.slots = 0;
    l.flags = align_up(l.slots + 2ull * n_ranks * rows * l.row * sizeof(float), 256);
    l.counters = align_up(l.flags + 2ull * n_ranks * rows * sizeof(uint32_t), 256);
    l.shard = align_up(l.counters + rows * sizeof(uint32_t), 256);
    l.total = align_up(l.shard + rows * (hd + 2) * sizeof(float), 256);
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
};

struct ExchangeArgs {
    uint8_t* const* peers;  // [n_ranks] exchange areas, this rank's own included
    const float* shard;     // [n_seqs][hq][hd+2] this rank's result
    float* out;             // [n_seqs][hq][hd]
    uint32_t* counters;     // [n_seqs][hq] in this rank's area
    unsigned int* status;   // sticky device status (decode workspace header)
    size_t slots, flags;
    int n_ranks, rank, n_seqs, hq;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

template <int HD>
__global__ void __launch_bounds__(128) exchange_combine_kernel(ExchangeArgs a) {
    constexpr int ROW = HD + 4, ROW4 = ROW / 4;
    const int h = blockIdx.x, b = blockIdx.y, t = threadIdx.x;
    const size_t rows = (size_t)a.n_seqs * a.hq, row_idx = (size_t)b * a.hq + h;
    __shared__ __align__(16) float s_row[ROW];
    __shared__ uint32_t s_seq;
    pdl_wait();  // the shard result comes from the kernel before
    pdl_trigger();
    if (t == 0) {
        const uint32_t c = a.counters[row_idx] + 1;
        a.counters[row_idx] = c;
        s_seq = c;
    }
    for (int i = t; i < ROW; i += blockDim.x) s_row[i] = i < HD + 2 ? a.shard[row_idx * (HD + 2) + i] : 0.f;
    __syncthreads();
    const uint32_t seq = s_seq, par = seq & 1u;
    // publish this rank's row into slot [par][rank][b][h] of every rank's area
    const size_t my_slot = ((size_t)par * a.n_ranks + a.rank) * rows + row_idx;
    for (int p = 0; p < a.n_ranks; p++) {
        float4* dst = reinterpret_cast<float4*>(a.peers[p] + a.slots) + my_slot * ROW4;
        for (int i = t; i < ROW4; i += blockDim.x) dst[i] = reinterpret_cast<const float4*>(s_row)[i];
    }
    __threadfence_system();
    __syncthreads();
    if (t < a.n_ranks) st_release_sys(reinterpret_cast<uint32_t*>(a.peers[t] + a.flags) + my_slot, seq);
    // wait for every rank's row in this rank's area (bounded)
    if (t < a.n_ranks) {
        const uint32_t* f =
            reinterpret_cast<const uint32_t*>(a.peers[a.rank] + a.flags) + ((size_t)par * a.n_ranks + t) * rows + row_idx;
        uint64_t t0 = 0;
        for (uint32_t it = 0; ld_acquire_sys(f) != seq; ++it) {
            if ((it & 255u) == 0u) {
                if (*reinterpret_cast<volatile unsigned int*>(a.status) & PICOATTN_DEV_TIMEOUT) break;
                const uint64_t now = global_timer_ns();
                if (it == 0u) t0 = now;
                else if (now - t0 > 2000000000ull) {
                    atomicOr(a.status, PICOATTN_DEV_TIMEOUT);
                    break;
                }
            }
        }
    }
    __syncthreads();
    // log-sum-exp combine of the n_ranks rows (read past L1: peers wrote them)
    const float* base = reinterpret_cast<const float*>(a.peers[a.rank] + a.slots);
    auto src = [&](int r) { return base + (((size_t)par * a.n_ranks + r) * rows + row_idx) * ROW; };
    float M = -INFINITY;
    for (int r = 0; r < a.n_ranks; r++) M = fmaxf(M, __ldcg(src(r) + HD));
    for (int d = t; d < HD; d += blockDim.x) {
        float L = 0.f, acc = 0.f;
        for (int r = 0; r < a.n_ranks; r++) {
            const float lse = __ldcg(src(r) + HD);
            if (lse == -INFINITY) continue;  // a rank without rows of this sequence
            const float w = ex2(lse - M);
            L += w;
            acc += w * __ldcg(src(r) + d);
        }
        a.out[row_idx * HD + d] = acc / L;
    }
}

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
    auto* s = static_cast<cudaStream_t>(stream);
    float* shard = reinterpret_cast<float*>(c->local + c->lay.shard);
    int32_t st = decode_shard_impl(cfg, layer, n_seqs, max_ctx, row_offset, local_rows, q, k, v, q_norm_w, k_norm_w,
                                   rope_cos, rope_sin, k_cache, v_cache, pos, shard, workspace, workspace_bytes, s);
    if (st != PICOATTN_OK) return st;
    ExchangeArgs a{};
    a.peers = c->peers_dev;
    a.shard = shard;
    a.out = out;
    a.counters = reinterpret_cast<uint32_t*>(c->local + c->lay.counters);
    a.status = static_cast<unsigned int*>(workspace);
    a.slots = c->lay.slots;
    a.flags = c->lay.flags;
    a.n_ranks = c->lay.n_ranks;
    a.rank = c->rank;
    a.n_seqs = n_seqs;
    a.hq = c->lay.hq;
    // programmatic stream serialisation: the blocks launch while the merge
    // kernel finishes and wait for it in pdl_wait
    cudaLaunchConfig_t lc{};
    lc.gridDim = dim3((unsigned)a.hq, (unsigned)n_seqs);
    lc.blockDim = dim3((unsigned)c->lay.hd);
    lc.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    const cudaError_t e = c->lay.hd == 64 ? cudaLaunchKernelEx(&lc, exchange_combine_kernel<64>, a)
                                          : cudaLaunchKernelEx(&lc, exchange_combine_kernel<128>, a);
    return e == cudaSuccess && cudaGetLastError() == cudaSuccess ? PICOATTN_OK : PICOATTN_ECUDA;
}

}  // extern "C"
