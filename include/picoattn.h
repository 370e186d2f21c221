/*
 * picoattn.h -- C ABI of the B200 (sm_100a) attention step.
 *
 * The reference engine (rain1201/picolm_qwen) runs its attention step inline in
 * the forward functions; it has no callable seam besides the RoPE function
 * pointer (RopeFn, cpp/model.hpp:176).  This ABI is the seam: the block
 *
 *     QK-RMSNorm  (cpp/model.hpp:326-333, 342-349)
 *     RoPE        (cpp/model.hpp:351-352 -> cpp/tensor.hpp:201-369)
 *     fp16 K/V store at row pos   (cpp/model.hpp:354-373)
 *     online-softmax GQA attention over rows 0..pos (cpp/model.hpp:375-418)
 *
 * of Model::forward (decode) and of Model::forward_batch (prefill,
 * cpp/model.hpp:507-593) becomes one call.  The caller keeps the reference's
 * data: q/k/v as produced by the projections, the per-layer FP16 KV cache in the
 * reference layout (uint16 [n_layers][max_seq_len][n_kv_heads*head_dim],
 * cpp/model.hpp:1003-1006), the host-built RoPE table ([max_seq_len][head_dim/2],
 * cpp/model.hpp:1008-1017) and the attention output xb [n_heads*head_dim].
 *
 * Conventions
 *   - Every pointer argument is device memory unless its comment says "host".
 *   - The caller owns every buffer (as RunState owns them in the reference,
 *     cpp/model.hpp:158-174); the library allocates nothing on these paths.
 *   - Every entry point returns PICOATTN_OK (0) or a negative status; none
 *     exits, throws or traps.  Errors that only the device can see (a position
 *     read from device memory that is out of range, a misaligned cache
 *     pointer) set a sticky bit in the workspace header, read back with
 *     picoattn_workspace_status().
 *   - Calls are asynchronous on `stream` and re-entrant per stream.
 *   - Kernels are built for sm_100a only; on any other device calls return
 *     PICOATTN_EDEVICE.
 */
#ifndef PICOATTN_H
#define PICOATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* A cudaStream_t; NULL is the legacy default stream. */
typedef struct CUstream_st* picoattn_stream_t;

/* Status codes. */
#define PICOATTN_OK            0
#define PICOATTN_EINVAL       -1  /* null pointer, bad count, inconsistent shape */
#define PICOATTN_EUNSUPPORTED -2  /* shape the kernels do not implement */
#define PICOATTN_ERANGE       -3  /* a position outside [0, max_seq_len) */
#define PICOATTN_ENOSPACE     -4  /* workspace smaller than the *_workspace_size() */
#define PICOATTN_ECUDA        -5  /* CUDA runtime error */
#define PICOATTN_ENCCL        -6  /* NCCL error */
#define PICOATTN_ETIMEOUT     -7  /* a bounded wait ran out */
#define PICOATTN_EDEVICE      -8  /* current device is not sm_100 */
#define PICOATTN_EDEVSTATUS   -9  /* a kernel flagged bad input (see workspace status) */
#define PICOATTN_EIO         -10  /* a file could not be opened, read or written */
#define PICOATTN_EFORMAT     -11  /* not a KVCP/GGUF file, or its shape does not match the config */
#define PICOATTN_ENOENT      -12  /* no such tensor in the model file */

/* Device-side sticky status bits (picoattn_workspace_status). */
#define PICOATTN_DEV_BAD_POS      0x1u  /* pos[b] < 0, >= max_seq_len or >= max_ctx */
#define PICOATTN_DEV_MISALIGNED   0x2u  /* a cache pointer not 16-byte aligned */
#define PICOATTN_DEV_TIMEOUT      0x4u  /* a bounded barrier wait gave up */

/* RoPE pairing.  NEOX = TensorOps::rope_qwen (cpp/tensor.hpp:201-283, element i
 * with i+hd/2).  INTERLEAVED = rope_llama's scalar definition (element 2i with
 * 2i+1, picolm/tensor.c:247-293).  The reference picks one from the model file
 * name (cpp/picolm.cpp:181-186); here it is explicit. */
#define PICOATTN_ROPE_NEOX        0
#define PICOATTN_ROPE_INTERLEAVED 1

/* Element type of q/k/v inputs. */
#define PICOATTN_DTYPE_F32 0
#define PICOATTN_DTYPE_F16 1

/* Model shape as the reference's config map holds it (cpp/model.hpp:33-47). */
typedef struct {
    int32_t n_layers;        /* cfg::N_LAYERS  */
    int32_t n_heads;         /* cfg::N_HEADS   */
    int32_t n_kv_heads;      /* cfg::N_KV_HEADS; n_heads % n_kv_heads == 0 */
    int32_t head_dim;        /* cfg::HEAD_DIM; 64 or 128 */
    int32_t max_seq_len;     /* cfg::MAX_SEQ_LEN: cache rows per layer */
    float   rope_freq_base;  /* cfg::ROPE_FREQ_BASE */
    int32_t rope_mode;       /* PICOATTN_ROPE_* */
    float   qk_norm_eps;     /* 1e-6 in the reference (cpp/tensor.hpp:162) */
} picoattn_config_t;

/* ---------------------------------------------------------------------- */
/* Host helpers                                                            */
/* ---------------------------------------------------------------------- */

/* Library version, major*10000 + minor*100 + patch. */
int32_t picoattn_version(void);

/* Text for a status code. */
const char* picoattn_strerror(int32_t status);

/* Text of the last CUDA runtime error behind a PICOATTN_ECUDA status on the
 * calling thread. */
const char* picoattn_last_cuda_error(void);

/* Validates a config; PICOATTN_OK, EINVAL or EUNSUPPORTED. */
int32_t picoattn_config_check(const picoattn_config_t* cfg);

/* Fills HOST arrays cos_out/sin_out [max_seq_len][head_dim/2] exactly as
 * Model::allocate_run_state does (cpp/model.hpp:1008-1017):
 *   theta = (float)pos / powf(base, (float)(2i)/(float)head_dim); cosf/sinf.
 * The kernels read this table instead of evaluating sin/cos on the device so
 * that positions up to 131071 rotate exactly as the reference rotates them. */
int32_t picoattn_rope_table(const picoattn_config_t* cfg, float* cos_out, float* sin_out);

/* Returns PICOATTN_OK when the current CUDA device is sm_100. */
int32_t picoattn_device_check(void);

/* Workspace header: zero the sticky device-status word.  Call once after
 * allocating a workspace (cudaMemset of the first 256 bytes also does). */
int32_t picoattn_workspace_init(void* workspace, size_t workspace_bytes, picoattn_stream_t stream);

/* Synchronises `stream`, reads the sticky device-status bits into *status_out
 * (host) and clears them. */
int32_t picoattn_workspace_status(void* workspace, picoattn_stream_t stream, uint32_t* status_out);

/* ---------------------------------------------------------------------- */
/* Decode (Model::forward, cpp/model.hpp:326-418)                          */
/* ---------------------------------------------------------------------- */

/* Workspace bytes for picoattn_decode with n_seqs sequences whose longest
 * attended length (pos+1) is at most max_ctx. */
size_t picoattn_decode_workspace_size(const picoattn_config_t* cfg, int32_t n_seqs, int32_t max_ctx);

/*
 * One decode step of layer `layer` for n_seqs independent sequences (n_seqs = 1
 * is the reference's single-sequence forward(token, pos)).
 *   q        [n_seqs][n_heads*head_dim]    fp32, projection output (state.q)
 *   k, v     [n_seqs][n_kv_heads*head_dim] fp32 (state.xb2 before each store)
 *   q_norm_w, k_norm_w  [head_dim] fp32 per-layer QK-RMSNorm weights, or both
 *            NULL when the layer has none (cpp/model.hpp:326-349)
 *   rope_cos, rope_sin  [max_seq_len][head_dim/2] fp32 (picoattn_rope_table);
 *            any 4-byte aligned address
 *   k_cache, v_cache    device array of n_seqs device pointers; entry b is
 *            sequence b's cache base, uint16 [n_layers][max_seq_len][kv_dim],
 *            16-byte aligned
 *   pos      [n_seqs] int32 device: the position of the new token; row pos of
 *            this layer is written and rows 0..pos are attended
 *   max_ctx  host upper bound on pos[b]+1 over the batch (sizes the launch)
 *   out      [n_seqs][n_heads*head_dim] fp32 attention output (state.xb)
 * Replaces cpp/model.hpp:326-418 (C engine: picolm/model.c:725-825).
 */
int32_t picoattn_decode(const picoattn_config_t* cfg, int32_t layer, int32_t n_seqs, int32_t max_ctx,
                        const float* q, const float* k, const float* v,
                        const float* q_norm_w, const float* k_norm_w,
                        const float* rope_cos, const float* rope_sin,
                        uint16_t* const* k_cache, uint16_t* const* v_cache,
                        const int32_t* pos, float* out,
                        void* workspace, size_t workspace_bytes, picoattn_stream_t stream);

/* Stage bits for picoattn_decode_staged. */
#define PICOATTN_STAGE_PREPARE 0x1u  /* QK-norm, RoPE, fp16 append of row pos, rotated q to workspace */
#define PICOATTN_STAGE_ATTEND  0x2u  /* split-KV attention partials into the workspace */
#define PICOATTN_STAGE_COMBINE 0x4u  /* log-sum-exp merge of the partials into out */
#define PICOATTN_STAGE_ALL     0x7u

/*
 * picoattn_decode split into its three kernels; `stages` selects which run
 * (in the order above).  Stages communicate through the workspace, so a call
 * with ATTEND must follow one with PREPARE on the same workspace and stream,
 * with the same arguments.  Lets a caller put events between the kernels or
 * overlap other work with them.  picoattn_decode == stages PICOATTN_STAGE_ALL.
 */
int32_t picoattn_decode_staged(const picoattn_config_t* cfg, int32_t layer, int32_t n_seqs, int32_t max_ctx,
                               const float* q, const float* k, const float* v,
                               const float* q_norm_w, const float* k_norm_w,
                               const float* rope_cos, const float* rope_sin,
                               uint16_t* const* k_cache, uint16_t* const* v_cache,
                               const int32_t* pos, float* out,
                               void* workspace, size_t workspace_bytes, picoattn_stream_t stream,
                               uint32_t stages);

/*
 * Single-sequence decode with a host position, the shape of the reference's
 * Model::forward(token, pos) call site (cpp/model.hpp:288): k_cache/v_cache are
 * the sequence's cache bases (device), pos is a host int.
 */
int32_t picoattn_decode_one(const picoattn_config_t* cfg, int32_t layer, int32_t pos,
                            const float* q, const float* k, const float* v,
                            const float* q_norm_w, const float* k_norm_w,
                            const float* rope_cos, const float* rope_sin,
                            uint16_t* k_cache, uint16_t* v_cache, float* out,
                            void* workspace, size_t workspace_bytes, picoattn_stream_t stream);

/*
 * picoattn_decode without a workspace argument: the call allocates nothing and
 * needs no caller-provided scratch.  No counterpart in the reference (whose CPU
 * engine needs no device scratch); it exists for callers that cannot allocate
 * device memory on their token path: engines that size all memory once at
 * start-up, and hosts whose device memory is owned by another allocator.
 *   Scratch: a fixed 8 MiB device array inside the library, held by every GPU
 *   that loads the library until the process exits.  Requests whose decode
 *   workspace (picoattn_decode_workspace_size) exceeds 8 MiB return
 *   PICOATTN_ENOSPACE; nothing is launched.
 *   The first call made with a given device current looks up the array's
 *   device address; make that first call before any stream capture.
 *   All calls share the array and it keeps the last call's contents: each call
 *   clears its status word first; calls whose kernels overlap on the GPU
 *   (different streams) race and must not be issued.
 *   status_out (host, optional): when non-NULL the call synchronises `stream`
 *   and stores the device status bits (PICOATTN_DEV_*) there; a non-zero value
 *   is also returned as PICOATTN_EDEVSTATUS.  This is the only way to observe
 *   them: with status_out NULL the bits stay in the shared array, which the
 *   next call clears, and no other entry point reads them.
 * Other arguments as for picoattn_decode.
 */
int32_t picoattn_decode_noalloc(const picoattn_config_t* cfg, int32_t layer, int32_t n_seqs, int32_t max_ctx,
                                const float* q, const float* k, const float* v,
                                const float* q_norm_w, const float* k_norm_w,
                                const float* rope_cos, const float* rope_sin,
                                uint16_t* const* k_cache, uint16_t* const* v_cache,
                                const int32_t* pos, float* out,
                                picoattn_stream_t stream, uint32_t* status_out);

/* ---------------------------------------------------------------------- */
/* Split-KV decode across GPUs (long context)                             */
/* ---------------------------------------------------------------------- */
/* The reference attends rows 0..pos in one loop (cpp/model.hpp:378-413); it
 * has no multi-device path.  Split across G devices, device g holds absolute
 * positions [row_offset, row_offset + local_rows) of every layer and of every
 * sequence, computes a per-head shard result (acc/sum over its rows and the
 * log2-sum-exp of its scores), and any device recovers the single-loop result
 * by a log-sum-exp combination. */

/* Bytes of one shard result: [n_seqs][n_heads][head_dim + 2] fp32. */
size_t picoattn_shard_partial_bytes(const picoattn_config_t* cfg, int32_t n_seqs);

/*
 * Decode step over this device's shard.  k_cache/v_cache entries are the local
 * slab bases, uint16 [n_layers][local_rows][kv_dim]; pos[] are absolute
 * positions (< max_seq_len; RoPE uses them); the new token's row is stored only
 * by the device whose shard holds pos.  max_ctx bounds the local rows attended
 * (<= local_rows).  partial receives [n_seqs][n_heads][head_dim+2]: the
 * normalised shard output and, at index head_dim, its log2-sum-exp (-inf when
 * the shard holds no row <= pos).  Workspace: picoattn_decode_workspace_size
 * (cfg, n_seqs, max_ctx).
 */
int32_t picoattn_decode_shard(const picoattn_config_t* cfg, int32_t layer, int32_t n_seqs, int32_t max_ctx,
                              int32_t row_offset, int32_t local_rows,
                              const float* q, const float* k, const float* v,
                              const float* q_norm_w, const float* k_norm_w,
                              const float* rope_cos, const float* rope_sin,
                              uint16_t* const* k_cache, uint16_t* const* v_cache,
                              const int32_t* pos, float* partial,
                              void* workspace, size_t workspace_bytes, picoattn_stream_t stream);

/* out[n_seqs][n_heads*head_dim] = log-sum-exp combination of n_shards shard
 * results laid out [n_shards][n_seqs][n_heads][head_dim+2] (device). */
int32_t picoattn_combine_shards(const picoattn_config_t* cfg, int32_t n_seqs, int32_t n_shards,
                                const float* partials, float* out, picoattn_stream_t stream);

/* NCCL: 128-byte unique id (host buffer) for picoattn_nccl_comm_create. */
int32_t picoattn_nccl_unique_id(void* id_out);
/* Non-blocking communicator creation; returns PICOATTN_ETIMEOUT (and aborts the
 * communicator) if the other ranks do not join within timeout_s seconds. */
int32_t picoattn_nccl_comm_create(int32_t n_ranks, const void* id, int32_t rank, double timeout_s, void** comm_out);
int32_t picoattn_nccl_comm_destroy(void* comm);
/* Bytes of the all-gather buffer of picoattn_decode_splitkv_nccl. */
size_t picoattn_splitkv_gather_bytes(const picoattn_config_t* cfg, int32_t n_seqs, int32_t n_ranks);
/* picoattn_decode_shard into this rank's slice of `gather`, an in-place NCCL
 * all-gather of the shard results, then picoattn_combine_shards into out
 * (every rank gets the full output, as the next layer's projections need). */
int32_t picoattn_decode_splitkv_nccl(const picoattn_config_t* cfg, int32_t layer, int32_t n_seqs, int32_t max_ctx,
                                     int32_t row_offset, int32_t local_rows,
                                     const float* q, const float* k, const float* v,
                                     const float* q_norm_w, const float* k_norm_w,
                                     const float* rope_cos, const float* rope_sin,
                                     uint16_t* const* k_cache, uint16_t* const* v_cache,
                                     const int32_t* pos, float* gather, float* out,
                                     void* workspace, size_t workspace_bytes, void* comm,
                                     picoattn_stream_t stream);

/* ---------------------------------------------------------------------- */
/* Prefill (Model::forward_batch, cpp/model.hpp:462-593)                   */
/* ---------------------------------------------------------------------- */

/* Workspace bytes for picoattn_prefill of up to n_tok tokens. */
size_t picoattn_prefill_workspace_size(const picoattn_config_t* cfg, int32_t n_tok);

/*
 * Attention step of one layer for a prompt of n_tok tokens at positions
 * start_pos .. start_pos+n_tok-1 of one sequence.  Token i runs the decode step
 * at pos = start_pos+i (cpp/model.hpp:493-593): its k/v row is stored and it
 * attends over rows 0..pos, i.e. causal attention over the cache.
 *   in_dtype  PICOATTN_DTYPE_F32 or PICOATTN_DTYPE_F16 for q, k, v
 *   q         [n_tok][n_heads*head_dim]    (pre-norm, pre-RoPE projection output)
 *   k, v      [n_tok][n_kv_heads*head_dim]
 *   q_norm_w, k_norm_w, rope_cos, rope_sin   as for picoattn_decode
 *   k_cache, v_cache   the sequence's cache bases (device, 16-byte aligned);
 *             rows 0..start_pos-1 of this layer must already hold the earlier
 *             tokens, rows start_pos..start_pos+n_tok-1 are written
 *   out       [n_tok][n_heads*head_dim] fp32
 * Requires start_pos + n_tok <= max_seq_len.
 */
int32_t picoattn_prefill(const picoattn_config_t* cfg, int32_t layer, int32_t n_tok, int32_t start_pos,
                         int32_t in_dtype, const void* q, const void* k, const void* v,
                         const float* q_norm_w, const float* k_norm_w,
                         const float* rope_cos, const float* rope_sin,
                         uint16_t* k_cache, uint16_t* v_cache, float* out,
                         void* workspace, size_t workspace_bytes, picoattn_stream_t stream);

/* picoattn_prefill split into its kernels (PICOATTN_STAGE_PREPARE: norm, RoPE,
 * cache append and fp16 q; PICOATTN_STAGE_ATTEND: causal attention into out).
 * Same contract as picoattn_decode_staged. */
int32_t picoattn_prefill_staged(const picoattn_config_t* cfg, int32_t layer, int32_t n_tok, int32_t start_pos,
                                int32_t in_dtype, const void* q, const void* k, const void* v,
                                const float* q_norm_w, const float* k_norm_w,
                                const float* rope_cos, const float* rope_sin,
                                uint16_t* k_cache, uint16_t* v_cache, float* out,
                                void* workspace, size_t workspace_bytes, picoattn_stream_t stream,
                                uint32_t stages);

/* ---- split-KV decode with the exchange over peer memory ----------------------
 * One process per GPU on one node.  Each rank creates its exchange area (device
 * memory, picoattn_p2p_area_bytes) and gets a CUDA IPC handle for it; the caller
 * moves the n_ranks handles between the processes (any transport) and opens the
 * communicator with all of them, in rank order.  picoattn_decode_splitkv_p2p
 * then runs the decode over this rank's rows (as picoattn_decode_shard), and
 * its merge kernel stores each head slice of the shard result, with its
 * log-sum-exp, into every rank's area over NVLink as (value, call number)
 * words, waits (bounded; PICOATTN_DEV_TIMEOUT in the workspace status) for every
 * rank's words of the same call in its own area and combines them by
 * log-sum-exp into out, on every rank.  Every rank must make the same sequence
 * of calls.  Destroy only after every rank's last call has completed (a
 * barrier).  No counterpart in the reference. */
#define PICOATTN_P2P_HANDLE_BYTES 64
size_t picoattn_p2p_area_bytes(const picoattn_config_t* cfg, int32_t n_seqs, int32_t n_ranks);
int32_t picoattn_p2p_create(const picoattn_config_t* cfg, int32_t n_seqs, int32_t n_ranks, int32_t rank,
                            void* ipc_handle_out, void** comm_out);
int32_t picoattn_p2p_open(void* comm, const void* ipc_handles);
int32_t picoattn_p2p_destroy(void* comm);
/* Bound on each wait for the other ranks' words, in seconds (0 < timeout_s <=
 * 60; 2 s after create).  A wait that runs out leaves NaN in the outputs it
 * was to combine and sets PICOATTN_DEV_TIMEOUT in the workspace status, so a
 * rank that stops calling costs the others one bounded wait, not a hang. */
int32_t picoattn_p2p_set_timeout(void* comm, double timeout_s);
int32_t picoattn_decode_splitkv_p2p(const picoattn_config_t* cfg, int32_t layer, int32_t n_seqs, int32_t max_ctx,
                                    int32_t row_offset, int32_t local_rows,
                                    const float* q, const float* k, const float* v,
                                    const float* q_norm_w, const float* k_norm_w,
                                    const float* rope_cos, const float* rope_sin,
                                    uint16_t* const* k_cache, uint16_t* const* v_cache,
                                    const int32_t* pos, float* out, void* workspace, size_t workspace_bytes,
                                    void* comm, picoattn_stream_t stream);

/* ---- KV-cache persistence in the C engine's KVCP file format ----------------
 * The reference saves a prompt's KV cache to skip its prefill next time
 * (picolm/model.c:870-983, kvcache_save / kvcache_load; magic "KVCP",
 * picolm/model.h:12).  File layout, little-endian:
 *   u32 magic 0x4B564350, u32 n_pos, u32 n_layers, u32 kv_dim,
 *   K rows 0..n_pos-1 of layer 0, of layer 1, ... (fp16, kv_dim each),
 *   V rows in the same order.
 * These entries read and write that format straight from and to a device
 * cache in the library's layout ([n_layers][max_seq_len][kv_dim] fp16, the
 * reference's own), so files are interchangeable with the reference's.
 *
 * picoattn_kvcp_bytes: size of the file for n_pos positions.
 * picoattn_kvcp_save: n_pos in [1, max_seq_len] (else PICOATTN_ERANGE); the
 *   device rows are copied out in stream order (the call returns when the file
 *   is written).
 * picoattn_kvcp_load: fills rows 0..n_pos-1 of every layer and returns n_pos;
 *   PICOATTN_EIO when the file cannot be read, PICOATTN_EFORMAT for a bad magic,
 *   a layer count or kv_dim other than the config's, n_pos outside
 *   [0, max_seq_len] or a short file (the reference reports all of these as 0
 *   cached positions); *n_pos_out = 0 on any error.
 * picoattn_kvcp_pack / _unpack: the same bytes in a caller buffer (host or
 *   device memory) instead of a file, stream-ordered (pack: dst_bytes >=
 *   picoattn_kvcp_bytes; unpack reads the header synchronously).
 * Not on the attention call path: save and load allocate pinned staging. */
#define PICOATTN_KVCP_MAGIC 0x4B564350u
size_t picoattn_kvcp_bytes(const picoattn_config_t* cfg, int32_t n_pos);
int32_t picoattn_kvcp_save(const picoattn_config_t* cfg, int32_t n_pos, const uint16_t* k_cache,
                           const uint16_t* v_cache, const char* path, picoattn_stream_t stream);
int32_t picoattn_kvcp_load(const picoattn_config_t* cfg, const char* path, uint16_t* k_cache, uint16_t* v_cache,
                           int32_t* n_pos_out, picoattn_stream_t stream);
int32_t picoattn_kvcp_pack(const picoattn_config_t* cfg, int32_t n_pos, const uint16_t* k_cache,
                           const uint16_t* v_cache, void* dst, size_t dst_bytes, picoattn_stream_t stream);
int32_t picoattn_kvcp_unpack(const picoattn_config_t* cfg, const void* src, size_t src_bytes, uint16_t* k_cache,
                             uint16_t* v_cache, int32_t* n_pos_out, picoattn_stream_t stream);

/* Which attention kernel picoattn_prefill launches for this shape on the
 * current device: PICOATTN_PREFILL_CTA_PAIR (head_dim 128, an even number of q
 * heads per KV head: two SMs per head pair, 2-CTA tensor-core instructions),
 * PICOATTN_PREFILL_HEAD_PAIR (one SM per head pair), PICOATTN_PREFILL_SINGLE
 * (one CTA per q head and tile); a negative status on error.  No counterpart in
 * the reference (diagnostic). */
#define PICOATTN_PREFILL_SINGLE 0
#define PICOATTN_PREFILL_HEAD_PAIR 1
#define PICOATTN_PREFILL_CTA_PAIR 2
int32_t picoattn_prefill_kernel(const picoattn_config_t* cfg);

/* ---- Projections around the attention step ---------------------------------
 *
 * The q/k/v projections with their biases (cpp/model.hpp:318-366) and the
 * output projection with its bias and the residual add (cpp/model.hpp:420-427)
 * on the GPU, for the weight formats TensorOps::matmul_bias multiplies with
 * (cpp/tensor.hpp:110-143, formats cpp/quant.hpp:16-74).  Weights stay in
 * their GGUF block layout, row-major as in the file (n_out rows of
 * picoattn_weight_bytes(type, n_in, 1) bytes); each is turned into fp32 with
 * the reference's dequantize_row_* arithmetic (bit-identical weights) and
 * multiplied in fp32 (sums in the GPU's order: results agree to rounding).
 * Biases are fp32 (the reference dequantises them once at load,
 * cpp/model.hpp:948-983).  Weight pointers: 4-byte aligned; x, out: 16.
 */
#define PICOATTN_WT_F32  1
#define PICOATTN_WT_F16  2
#define PICOATTN_WT_Q4_0 3
#define PICOATTN_WT_Q8_0 9
#define PICOATTN_WT_Q4_K 13
#define PICOATTN_WT_Q6_K 15

/* Bytes of n_out rows of n_in weights of a PICOATTN_WT_* type (gguf_type_row_size,
 * cpp/quant.hpp:170-175); 0 for an unsupported type or n_in not a multiple of
 * the type's block (32, or 256 for Q4_K and Q6_K). */
size_t picoattn_weight_bytes(int32_t w_type, int32_t n_in, int32_t n_out);

/* out[v*n_out + d] = W[d,:] . x[v*n_in : (v+1)*n_in] (+ bias[d]) for v < n_vec
 * (accumulate != 0: added to out, as vec_add does with the residual).
 * Replaces TensorOps::matmul_bias (cpp/tensor.hpp:110-143) on the device. */
int32_t picoattn_matvec(const void* w, int32_t w_type, const float* bias, int32_t n_in, int32_t n_out,
                        int32_t n_vec, const float* x, float* out, int32_t accumulate, picoattn_stream_t stream);

/* One layer's attention weights as the model file holds them. */
typedef struct {
    const void* wq;  /* [n_heads*head_dim][dim]   */
    const void* wk;  /* [n_kv_heads*head_dim][dim] */
    const void* wv;  /* [n_kv_heads*head_dim][dim] */
    const void* wo;  /* [dim][n_heads*head_dim]   */
    int32_t wq_type, wk_type, wv_type, wo_type;  /* PICOATTN_WT_* */
    const float* bq; /* fp32 biases, or NULL */
    const float* bk;
    const float* bv;
    const float* bo;
} picoattn_layer_weights_t;

size_t picoattn_decode_layer_workspace_size(const picoattn_config_t* cfg, int32_t dim, int32_t n_seqs,
                                            int32_t max_ctx);

/* The attention block of one layer for n_seqs sequences, from the normalised
 * hidden state xb [n_seqs][dim] to the residual x [n_seqs][dim]:
 *   q = Wq.xb + bq, k = Wk.xb + bk, v = Wv.xb + bv       (cpp/model.hpp:318-366)
 *   QK-norm, RoPE, cache append at pos, attention        (picoattn_decode)
 *   x += Wo.attn + bo                                    (cpp/model.hpp:420-427)
 * in one stream-ordered chain (three projections in one kernel, the decode
 * kernels, the output projection).  Caches, positions and norms as for
 * picoattn_decode.  The workspace begins with a decode workspace: initialise
 * it with picoattn_workspace_init; picoattn_workspace_status reads it. */
int32_t picoattn_decode_layer(const picoattn_config_t* cfg, int32_t layer, int32_t dim, int32_t n_seqs,
                              int32_t max_ctx, const float* xb, const picoattn_layer_weights_t* weights,
                              const float* q_norm_w, const float* k_norm_w, const float* rope_cos,
                              const float* rope_sin, uint16_t* const* k_cache, uint16_t* const* v_cache,
                              const int32_t* pos, float* x, void* workspace, size_t workspace_bytes,
                              picoattn_stream_t stream);

/* ---- The rest of the decode layer: norms, FFN, logits ------------------------
 *
 * With these the whole per-token forward of the C++ engine
 * (Model::forward, cpp/model.hpp:288-458) runs on the device: per layer
 * picoattn_decode_block (attention norm, picoattn_decode_layer, the FFN
 * block), then picoattn_logits.  Only the embedding row (a table lookup,
 * cpp/model.hpp:302-308) is the caller's.  Weights as for picoattn_matvec;
 * norm weights fp32 [dim] (the reference dequantises them once at load,
 * cpp/model.hpp:924-945).  The model-dimension norms add their squares in
 * the GPU's order (the reference: four SSE lanes), so they agree to fp32
 * rounding; eps is the reference's 1e-6. */

/* out[v] = x[v] / sqrt(mean(x[v]^2) + 1e-6) * weight for v < n_vec, dim
 * floats each (TensorOps::rmsnorm, cpp/tensor.hpp:146-176).  x, out 16-byte
 * aligned; out may equal x. */
int32_t picoattn_rmsnorm(const float* x, const float* weight, float* out, int32_t dim, int32_t n_vec,
                         picoattn_stream_t stream);

/* One layer's FFN weights as the model file holds them. */
typedef struct {
    const void* w_gate;  /* [n_ffn][dim] */
    const void* w_up;    /* [n_ffn][dim] */
    const void* w_down;  /* [dim][n_ffn] */
    int32_t gate_type, up_type, down_type;  /* PICOATTN_WT_* */
    const float* b_gate; /* fp32 [n_ffn] or NULL */
    const float* b_down; /* fp32 [dim] or NULL (the reference multiplies up without a bias) */
} picoattn_ffn_weights_t;

size_t picoattn_ffn_workspace_size(int32_t dim, int32_t n_ffn, int32_t n_vec);

/* The FFN block of one layer and its residual, in place on x [n_vec][dim]
 * (cpp/model.hpp:429-452):
 *   xb = rmsnorm(x, ffn_norm_w); h = silu(Wg.xb + bg) * (Wu.xb); x += Wd.h + bd
 * gate and up go out as one launch; silu (1/(1+e^-x), times x) and the
 * product in one kernel; the down projection adds into x. */
int32_t picoattn_ffn(const picoattn_ffn_weights_t* weights, const float* ffn_norm_w, int32_t dim, int32_t n_ffn,
                     int32_t n_vec, float* x, void* workspace, size_t workspace_bytes, picoattn_stream_t stream);

size_t picoattn_logits_workspace_size(int32_t dim, int32_t n_vec);

/* logits[v] = W_out . rmsnorm(x[v], output_norm_w) for v < n_vec, vocab each
 * (cpp/model.hpp:454-457). */
int32_t picoattn_logits(const float* x, const float* output_norm_w, const void* w_out, int32_t w_type, int32_t dim,
                        int32_t vocab, int32_t n_vec, float* logits, void* workspace, size_t workspace_bytes,
                        picoattn_stream_t stream);

size_t picoattn_decode_block_workspace_size(const picoattn_config_t* cfg, int32_t dim, int32_t n_ffn,
                                            int32_t n_seqs, int32_t max_ctx);

/* One whole transformer layer of the decode step for n_seqs sequences, on
 * the residual x [n_seqs][dim] in place (cpp/model.hpp:315-452):
 *   xb = rmsnorm(x, attn_norm_w); picoattn_decode_layer(xb -> x); picoattn_ffn(x)
 * Arguments as for those calls.  The workspace begins with a decode
 * workspace: initialise it with picoattn_workspace_init;
 * picoattn_workspace_status reads it. */
int32_t picoattn_decode_block(const picoattn_config_t* cfg, int32_t layer, int32_t dim, int32_t n_ffn,
                              int32_t n_seqs, int32_t max_ctx, const float* attn_norm_w,
                              const picoattn_layer_weights_t* attn_weights, const float* ffn_norm_w,
                              const picoattn_ffn_weights_t* ffn_weights, const float* q_norm_w,
                              const float* k_norm_w, const float* rope_cos, const float* rope_sin,
                              uint16_t* const* k_cache, uint16_t* const* v_cache, const int32_t* pos, float* x,
                              void* workspace, size_t workspace_bytes, picoattn_stream_t stream);

/* ---- GGUF model files to the device -------------------------------------------
 *
 * The C++ engine's loader (Model::parse_gguf, cpp/model.hpp:705-902) on the
 * host: the file is mapped read-only and parsed with the engine's rules (the
 * metadata keys it reads, by substring, cpp/gguf_metadata.hpp:241-275; its
 * defaults and its context cap: max_seq_len_override when smaller than the
 * file's context, else at most 2048; tensor types shifted by one into the
 * engine's numbering = PICOATTN_WT_*; tensors under the engine's keys:
 * layer -1 for token_embd, output_norm and output (output = token_embd when
 * the file has none), else blk.<layer>.<key> with ".weight" removed).
 * picoattn_gguf_upload copies every tensor into one caller-allocated device
 * arena (256-byte aligned) and adds fp32 copies of the norms and biases (the
 * arrays the engine dequantises at load, cpp/model.hpp:924-1000), so that
 * picoattn_gguf_arena_tensor hands picoattn_decode_block and picoattn_logits
 * their weights.  Not on the token path: open maps the file, upload copies
 * it and synchronises the stream. */
typedef struct picoattn_gguf picoattn_gguf_t;

/* The model shape as the engine reads it from the file. */
typedef struct {
    int32_t n_embd, n_ffn, n_heads, n_kv_heads, n_layers, vocab_size, max_seq_len, head_dim;
    float rope_freq_base;
    int32_t alignment;  /* general.alignment, 0 when absent (32 used) */
} picoattn_gguf_config_t;

/* PICOATTN_EIO (cannot open or map), PICOATTN_EFORMAT (not a GGUF v2/v3 file
 * the engine can read), else PICOATTN_OK and *out. */
int32_t picoattn_gguf_open(const char* path, int32_t max_seq_len_override, picoattn_gguf_t** out);
int32_t picoattn_gguf_close(picoattn_gguf_t* model);
int32_t picoattn_gguf_get_config(const picoattn_gguf_t* model, picoattn_gguf_config_t* cfg);
/* Type (PICOATTN_WT_*), byte count and file offset of a tensor by the engine's
 * key (layer -1: token_embd, output_norm, output); PICOATTN_ENOENT if absent. */
int32_t picoattn_gguf_find(const picoattn_gguf_t* model, int32_t layer, const char* key, int32_t* type,
                           size_t* bytes, size_t* file_offset);
/* Device bytes the arena needs. */
size_t picoattn_gguf_arena_bytes(const picoattn_gguf_t* model);
/* Copies the model into `arena` (device, 256-byte aligned) and synchronises
 * `stream`; norms and biases must be F32 or F16 (else PICOATTN_EUNSUPPORTED). */
int32_t picoattn_gguf_upload(const picoattn_gguf_t* model, void* arena, size_t arena_bytes,
                             picoattn_stream_t stream);
/* A tensor's device address in the arena and its type: the file's bytes, or
 * for norms and biases (keys attn_norm, ffn_norm, output_norm, attn_q_norm,
 * attn_k_norm, *_b) their fp32 copy (type PICOATTN_WT_F32). */
int32_t picoattn_gguf_arena_tensor(const picoattn_gguf_t* model, const void* arena, int32_t layer, const char* key,
                                   const void** dev_ptr, int32_t* type);

#ifdef __cplusplus
}
#endif
#endif /* PICOATTN_H */
