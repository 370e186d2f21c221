// picoattn_internal.h -- launch descriptors shared by the ABI layer and the kernels.
#pragma once

#include <cstddef>
#include <cstdint>
#include <mutex>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "picoattn.h"

namespace picoattn {

// Workspace header: the first 256 bytes of every workspace.
struct WsHeader {
    unsigned int status;  // sticky PICOATTN_DEV_* bits
    unsigned int pad[63];
};
constexpr size_t kWsHeaderBytes = 256;

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// One-time setup per CUDA device.  Kernel attributes (the dynamic shared-memory
// limit, the carveout) belong to a device, so a process that drives several
// GPUs sets them on each; run() calls setup() the first time it sees the
// current device and returns that result on every later call with the same
// device current.  Thread-safe.
class PerDeviceOnce {
  public:
    template <class F>
    cudaError_t run(F&& setup) {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        if (dev < 0 || dev >= kMaxDev) return cudaErrorInvalidDevice;
        std::lock_guard<std::mutex> lock(mu_);
        if (!done_[dev]) {
            err_[dev] = setup();
            done_[dev] = true;
        }
        return err_[dev];
    }

  private:
    static constexpr int kMaxDev = 64;
    std::mutex mu_;
    bool done_[kMaxDev] = {};
    cudaError_t err_[kMaxDev] = {};
};

// Records a CUDA error for picoattn_last_cuda_error() on the calling thread and
// maps it to a status: PICOATTN_OK for cudaSuccess, else PICOATTN_ECUDA.
int32_t cuda_status(cudaError_t e);

// Decode launch plan: how the cache rows of a sequence are cut into chunks
// (one CTA each), tiles (one pipeline stage each) and row groups (16 rows, one
// warp-level MMA step each).
struct DecodePlan {
    int compute_warps;    // 4 or 8
    int warps_per_head;   // compute_warps / n_kv_heads
    int tile_rows;        // rows per pipeline stage (multiple of 16*warps_per_head)
    int stages;           // pipeline depth
    int grid_ctas;        // persistent CTAs of the attention kernel
    int merge_blocks;     // one sequence: blocks of the merge kernel (one per q head, at most one per SM)
    int max_grid;         // upper bound on grid_ctas (sizes the partial slots)
    int n_slots;          // partial slots per head: (max_grid + n_seqs) * warps_per_head, rounded up to even
    int smem_bytes;       // dynamic shared memory per CTA
    size_t ws_prefix, ws_qrot, ws_ml, ws_o, ws_total;  // workspace offsets and size
};

// Split-KV decode over the GPUs of one node with the shard results exchanged
// through peer memory by the merge kernel: each (head, 32-column slice) block
// stores its slice and log2-sum-exp into every rank's exchange area and
// combines the ranks' slices from its own.  Every 8-byte word carries a value
// and the call's sequence number, written with one store, so a reader that
// sees the number sees the value: no fence or separate flag is needed.
// Area layout (per rank, offsets below):
//   slots    [2 parities][n_ranks][n_seqs * hq * hd/32][kXchgWords] u64 words
//   counters [n_seqs * hq * hd/32] u32   calls so far, this rank only
constexpr int kXchgCols = 32;
constexpr int kXchgWords = kXchgCols + 2;  // the slice, its log2-sum-exp, one word of padding
struct XchgArgs {
    uint8_t* const* peers;  // [n_ranks] exchange areas (device array), this rank's own included; null: no exchange
    size_t slots, counters;
    int rank, n_ranks;
    float* out;             // [n_seqs][hq][hd] the combined output
    unsigned long long timeout_ns;  // bound on the wait for the other ranks' words
};

struct DecodeArgs {
    int hq, hkv, g, hd, kvd, max_seq, layer, n_seqs, max_ctx;
    int rope_mode;
    float eps;
    const float* q;
    const float* k;
    const float* v;
    const float* qn_w;
    const float* kn_w;
    const float* rope_cos;
    const float* rope_sin;
    uint16_t* const* kc_ptrs;  // per-sequence cache bases (device array), or null
    uint16_t* const* vc_ptrs;
    uint16_t* kc_one;          // single-sequence base when kc_ptrs is null
    uint16_t* vc_one;
    const int* pos_dev;        // per-sequence positions (device), or null
    int pos_host;              // position when pos_dev is null
    float* out;
    unsigned int* status;
    float* q_rot;              // [n_seqs][hq][hd]
    long long* prefix;         // [n_seqs+1] exclusive prefix sums of attended lengths
    int row_offset;            // absolute position of local cache row 0 (0 unless the rows are sharded)
    int local_rows;            // cache rows per layer in the local slab (max_seq unless sharded)
    float* shard_out;          // non-null: write [n_seqs][hq][hd+2] = (acc/sum, log2-sum-exp) instead of out
    float* part_ml;            // [hq][n_slots][2]  (max, sum) in log2 units; slot = (cta + seq) * warps_per_head + warp
    float* part_o;             // [hq][n_slots][hd]  (a head's pieces are contiguous: the merge bulk-copies them)
    int n_slots;
    int tile_rows, stages, warps_per_head, compute_warps;
    int fused_append;          // one sequence, all stages: the attention kernel appends the new k/v row itself
    XchgArgs x;                // the merge kernel exchanges the shard results (x.peers non-null)
};

bool make_decode_plan(const picoattn_config_t& cfg, int n_seqs, int max_ctx, DecodePlan* plan);

// Decode over a slab of local cache rows (split-KV shard), all stages; the
// result goes to partial ([n_seqs][hq][hd+2]: normalised output, log2-sum-exp)
// or, with x, is exchanged with the other ranks and combined into x->out.
int32_t decode_shard_impl(const picoattn_config_t* cfg, int32_t layer, int32_t n_seqs, int32_t max_ctx,
                          int32_t row_offset, int32_t local_rows, const float* q, const float* k, const float* v,
                          const float* qn, const float* kn, const float* rc, const float* rs,
                          uint16_t* const* kcp, uint16_t* const* vcp, const int32_t* pos, float* partial, void* ws,
                          size_t ws_bytes, cudaStream_t stream, const XchgArgs* x);
cudaError_t launch_decode(const DecodeArgs& a, const DecodePlan& plan, cudaStream_t stream, unsigned stages);
int device_sm_count();

// Projections (matvec.cu): out[v * out_stride + row] = W[row] . x[v] (+ bias[row]),
// or added into out.  Up to three matrices that read the same x in one launch.
struct MatvecPart {
    const uint8_t* w;   // n_out rows of row_bytes, in the GGUF block layout of `type`
    const float* bias;  // [n_out] or null
    float* out;
    size_t out_stride, row_bytes;
    int type, n_out, block_bytes;
};
struct MatvecArgs {
    MatvecPart part[3];
    int n_parts, n_in, n_vec, rows_total, accumulate;
    const float* x;  // [n_vec][n_in], 16-byte aligned
    // 1: no kernel ahead of this launch in the stream writes the weight
    // matrices (a launch that follows one of this library's own kernels), so
    // the tensor-core kernel may read them before the programmatic-launch wait
    int weights_ready;
    // The tensor-core kernel only (launch_matvec_mma): x is formed on the fly
    // from the caller's vector.  x_norm_w: x = rmsnorm(x) with these weights
    // (the model-dimension norm, as launch_rmsnorm computes it); x_up: x =
    // silu(x) * x_up (the FFN gate).  Null: x as given.
    const float* x_norm_w;
    const float* x_up;
    // x's fragments made beforehand by launch_xfrag (x then unused), for the
    // position map of launches of Q4_K only (xfrag_pairs = 1) or the other one
    const uint32_t* xfrag;
    int xfrag_pairs;
};
int weight_block_elems(int type);  // weights per block of a PICOATTN_WT_* type (0: unsupported)
int weight_block_bytes(int type);
bool matvec_part(int type, const void* w, const float* bias, int n_in, int n_out, float* out, size_t out_stride,
                 MatvecPart* p);
cudaError_t launch_matvec(const MatvecArgs& a, cudaStream_t stream);
// One vector of Q4_K / Q6_K matrices on the integer tensor cores (matvec_mma.cu);
// cudaErrorNotSupported when the launch does not fit it.
cudaError_t launch_matvec_mma(const MatvecArgs& a, cudaStream_t stream);
// x's integer-digit fragments for the tensor-core mat-vec, made once (x =
// silu(x) * up when up is given): xfrag_bytes(n_in) bytes at out (0: n_in not
// a multiple of 256).  pairs: for launches of Q4_K matrices only.
size_t xfrag_bytes(int n_in);
cudaError_t launch_xfrag(const float* x, const float* up, int n_in, bool pairs, uint32_t* out, cudaStream_t stream);

// The rest of a decode layer (layer_ops.cu): model-dimension RMSNorm of n_vec
// vectors, and the FFN gate gate = silu(gate) * up over n elements.
cudaError_t launch_rmsnorm(const float* x, const float* w, float* out, int dim, int n_vec, cudaStream_t stream);
cudaError_t launch_silu_mul(float* gate, const float* up, size_t n, cudaStream_t stream);

struct PrefillArgs {
    int hq, hkv, g, hd, kvd, max_seq, layer, n_tok, start, n_qtiles;
    int rope_mode, in_dtype;
    float eps;
    const void* q;   // [n_tok][hq*hd]  fp32 or fp16
    const void* k;   // [n_tok][kvd]
    const void* v;
    const float* qn_w;
    const float* kn_w;
    const float* rope_cos;
    const float* rope_sin;
    uint16_t* k_cache;  // sequence cache base [n_layers][max_seq][kvd]
    uint16_t* v_cache;
    float* out;         // [n_tok][hq*hd]
    unsigned int* status;
    int* work_counter;  // workspace header: next work item of the persistent attention kernel
    __half* q16;        // workspace: rotated, scaled q [n_tok][hq][hd]
};

cudaError_t launch_prefill(const PrefillArgs& a, cudaStream_t stream, unsigned stages);
size_t prefill_workspace_bytes(const picoattn_config_t& cfg, int n_tok);
// attention kernel picoattn_prefill launches for this shape on the current device:
// 2 CTA pair, 1 head pair, 0 one head per CTA, -1 setup failed
int prefill_kernel_variant(const picoattn_config_t& cfg);

}  // namespace picoattn
