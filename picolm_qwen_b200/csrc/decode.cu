// decode.cu -- single-token (decode) attention step for sm_100a.
//
// Replaces the inline block of Model::forward, cpp/model.hpp:326-418
// (C engine: picolm/model.c:725-825), for a batch of independent sequences.
//
// Three kernels, in stream order:
//   prep   one warp per head vector: per-head QK-RMSNorm and RoPE in the
//          reference's exact fp32 operation order; the new k/v row rounded to
//          fp16 with the reference's rounding and stored at row pos of the
//          layer's cache slab; the rotated q kept in the workspace.  One extra
//          block scans the attended lengths (pos+1) into row prefix sums.
//   attn   persistent split-KV attention.  The rows of all sequences are
//          concatenated and cut into gridDim.x equal contiguous slices, one per
//          CTA, so every CTA streams the same number of bytes whatever the mix
//          of lengths.  A producer warp streams whole cache rows (all KV heads,
//          contiguous in the reference layout) into shared memory with TMA bulk
//          copies, running ahead across sequence boundaries; compute warps,
//          one per KV head (several per head when there are fewer than four
//          heads), run QK^T and PV for all q heads of that KV head as
//          tensor-core MMAs, so every q head of a GQA group shares each K/V
//          tile read from HBM.  Online softmax in fp32 (log2 domain).  A CTA
//          that covers a whole sequence writes its normalised output; pieces
//          of longer sequences go to partial slots.
//   merge  log-sum-exp combination of the pieces of each sequence that was
//          split across CTAs.
#include <cmath>
#include <cstdio>
#include <utility>

#include "device_common.cuh"
#include "picoattn_internal.h"
#include "prep_common.cuh"

namespace picoattn {

namespace {

__device__ __forceinline__ int seq_pos(const DecodeArgs& a, int b) {
    return a.pos_dev ? a.pos_dev[b] : a.pos_host;
}
__device__ __forceinline__ uint16_t* seq_kcache(const DecodeArgs& a, int b) {
    return a.kc_ptrs ? a.kc_ptrs[b] : a.kc_one;
}
__device__ __forceinline__ uint16_t* seq_vcache(const DecodeArgs& a, int b) {
    return a.vc_ptrs ? a.vc_ptrs[b] : a.vc_one;
}
// Rows of this sequence held in the local slab that the token at `pos` attends:
// the slab holds absolute positions [row_offset, row_offset + local_rows).
__device__ __forceinline__ int local_len(const DecodeArgs& a, int pos) {
    return max(0, min(pos + 1 - a.row_offset, a.local_rows));
}
__device__ __forceinline__ bool pos_ok(const DecodeArgs& a, int pos) {
    return pos >= 0 && pos < a.max_seq && local_len(a, pos) <= a.max_ctx;
}

// CTA i streams concatenated rows [slice_start(i), slice_start(i+1)).
__device__ __forceinline__ long long slice_start(long long i, long long R, long long G) { return i * R / G; }

// The CTA whose slice holds concatenated row x (0 <= x < R).
__device__ __forceinline__ int cta_of_row(long long x, long long R, int G) {
    long long i = x * G / R;
    while (i + 1 < G && slice_start(i + 1, R, G) <= x) i++;
    while (i > 0 && slice_start(i, R, G) > x) i--;
    return (int)i;
}

// ---------------------------------------------------------------------------
// prep
// ---------------------------------------------------------------------------

// Exclusive scan of the attended lengths (pos+1, or 0 for a rejected position)
// into prefix[0..n_seqs]; one block of NT threads.
template <int NT>
__device__ void scan_lengths(const DecodeArgs& a) {
    __shared__ long long warp_tot[NT / 32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int per = (a.n_seqs + NT - 1) / NT;
    const int b0 = min(tid * per, a.n_seqs), b1 = min(b0 + per, a.n_seqs);
    long long mine = 0;
    for (int b = b0; b < b1; b++) {
        const int p = seq_pos(a, b);
        mine += pos_ok(a, p) ? local_len(a, p) : 0;
    }
    long long incl = mine;
    for (int o = 1; o < 32; o <<= 1) {
        const long long v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    long long base = 0;
    for (int w = 0; w < warp; w++) base += warp_tot[w];
    long long run = base + incl - mine;
    for (int b = b0; b < b1; b++) {
        a.prefix[b] = run;
        const int p = seq_pos(a, b);
        run += pos_ok(a, p) ? local_len(a, p) : 0;
    }
    if (tid == NT - 1) a.prefix[a.n_seqs] = base + incl;
}

template <int HD>
__global__ void __launch_bounds__(256) decode_prep_kernel(DecodeArgs a) {
    // The attention kernel after this one may launch at once; it waits for this
    // kernel before it reads anything written here.
    pdl_trigger();
    // q/k/v may come from the kernel before, which may also still read the
    // workspace written here
    pdl_wait();
    if (blockIdx.y == (unsigned)a.n_seqs) {  // the extra block row: length prefix sums
        if (blockIdx.x == 0) scan_lengths<256>(a);
        return;
    }
    // 8 warps x 4 head vectors of one sequence per block (helpers: prep_common.cuh)
    constexpr int V = HD / 32;
    __shared__ float sq[8][4 * HD];
    const int b = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos = seq_pos(a, b);
    if (!pos_ok(a, pos)) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(a.status, PICOATTN_DEV_BAD_POS);
        return;
    }
    const int n_slots = a.hq + 2 * a.hkv;
    const int slot0 = (blockIdx.x * 8 + warp) * 4;
    if (slot0 >= n_slots) return;
    RopeLane<HD> rl;
    rope_lane_load<HD>(rl, a.rope_cos + (size_t)pos * (HD / 2), a.rope_sin + (size_t)pos * (HD / 2), a.rope_mode,
                       lane);
    float qw[V], kw[V];
    if (a.qn_w) {
#pragma unroll
        for (int j = 0; j < V; j++) qw[j] = a.qn_w[V * lane + j], kw[j] = a.kn_w[V * lane + j];
    }
    Vec<HD> x[4];
    int kind[4], head[4];
#pragma unroll
    for (int u = 0; u < 4; u++) {
        const int slot = slot0 + u;
        kind[u] = slot < a.hq ? 0 : (slot < a.hq + a.hkv ? 1 : (slot < n_slots ? 2 : 3));
        head[u] = kind[u] == 0 ? slot : (kind[u] == 1 ? slot - a.hq : slot - a.hq - a.hkv);
        if (kind[u] == 0) vec_load<HD>(x[u], a.q, ((size_t)b * a.hq + head[u]) * HD, PICOATTN_DTYPE_F32, lane);
        else if (kind[u] == 1) vec_load<HD>(x[u], a.k, ((size_t)b * a.hkv + head[u]) * HD, PICOATTN_DTYPE_F32, lane);
        else if (kind[u] == 2) vec_load<HD>(x[u], a.v, ((size_t)b * a.hkv + head[u]) * HD, PICOATTN_DTYPE_F32, lane);
    }
    const int lrow = pos - a.row_offset;  // the new row lives in this slab only if 0 <= lrow < local_rows
    const bool row_here = lrow >= 0 && lrow < a.local_rows;
    const size_t row = ((size_t)a.layer * a.local_rows + (row_here ? lrow : 0)) * a.kvd;
    if (a.qn_w) {  // QK-RMSNorm of the q and k vectors, four at a time
        float wsel[4][V];
        bool nrm[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            nrm[u] = kind[u] == 0 || kind[u] == 1;
#pragma unroll
            for (int j = 0; j < V; j++) wsel[u][j] = kind[u] == 0 ? qw[j] : kw[j];
        }
        vec_rmsnorm4<HD>(x, wsel, nrm, a.eps, sq[warp], lane);
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
        if (kind[u] == 3) break;
        if (kind[u] != 0 && !row_here) continue;
        if (kind[u] != 2) {
            vec_rope<HD>(x[u], rl, a.rope_mode, lane);
        }
        if (kind[u] == 0)
            vec_store_f32<HD>(x[u], a.q_rot + ((size_t)b * a.hq + head[u]) * HD, lane);
        else
            vec_store_ref16<HD>(x[u], (kind[u] == 1 ? seq_kcache(a, b) : seq_vcache(a, b)) + row +
                                          (size_t)head[u] * HD, lane);
    }
}

// ---------------------------------------------------------------------------
// merge: out = sum_p 2^(m_p - M) acc_p / sum_p 2^(m_p - M) l_p over the pieces
// ---------------------------------------------------------------------------

// Merges the partial (max, sum, acc) pieces of one (head, sequence) into its
// output columns [z*DS, z*DS+DS), with NT threads (tid < NT) and `sync` as
// their barrier.  The work is a chain of dependent steps, so it keeps to one
// round of loads after the position and prefix sums: at once, (max, sum) of
// every piece into shared memory (thread = piece) and the acc columns d..d+3 of
// every NG-th piece (thread = (group, 4 columns)), RPT rows each held in
// registers; then the block max M, the weights 2^(m - M), the block sum L of
// weight * sum, and the weighted acc rows summed over the groups.  The pieces
// are read from L2 (__ldcg), where the attention kernel just left them.
// Shared memory: m_s, l_s [kMergeMaxPieces], red [NT/32].
constexpr int kMergeMaxPieces = 1280;

// One exchange word: a value and the call's sequence number in one 8-byte
// store (single-copy atomic), so the reader needs no fence.
__device__ __forceinline__ void st_word(uint64_t* p, float v, uint32_t seq) {
    asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(__float_as_uint(v)), "r"(seq) : "memory");
}

__device__ __forceinline__ void ld_word(const uint64_t* p, float& v, uint32_t& seq) {
    uint32_t a, b;
    asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(a), "=r"(b) : "l"(p) : "memory");
    v = __uint_as_float(a);
    seq = b;
}

// Waits (bounded by timeout_ns) until, for every rank r < n, the words
// lse_src(r) and o_src(r) carry sequence number seq; their values go to lr[r],
// o[r].  Each pass loads every missing word at once, so the ranks' words
// arrive in parallel rather than one round trip after another.  A wait that
// gives up leaves NaN (and PICOATTN_DEV_TIMEOUT set).
template <class Src>
__device__ __forceinline__ void wait_words(int n, Src src, int col, uint32_t seq, float (&lr)[8], float (&o)[8],
                                           unsigned int* status, unsigned long long timeout_ns) {
    uint32_t done = 0u;
    const uint32_t all = (1u << n) - 1u;
    uint64_t t0 = 0;
    for (uint32_t it = 0;; ++it) {
#pragma unroll
        for (int r = 0; r < 8; r++) {
            if (r < n && !(done & (1u << r))) {
                float v0, v1;
                uint32_t s0, s1;
                ld_word(src(r) + kXchgCols, v0, s0);
                ld_word(src(r) + col, v1, s1);
                if (s0 == seq && s1 == seq) {
                    lr[r] = v0;
                    o[r] = v1;
                    done |= 1u << r;
                }
            }
        }
        if (done == all) return;
        if ((it & 63u) == 0u) {
            const uint64_t now = global_timer_ns();
            if (it == 0u) t0 = now;
            else if ((*reinterpret_cast<volatile unsigned int*>(status) & PICOATTN_DEV_TIMEOUT) ||
                     now - t0 > timeout_ns) {
                atomicOr(status, PICOATTN_DEV_TIMEOUT);
#pragma unroll
                for (int r = 0; r < 8; r++)
                    if (r < n && !(done & (1u << r))) lr[r] = o[r] = __int_as_float(0x7fc00000);
                return;
            }
        }
    }
}

// out = sum_r 2^(lse_r - Lm) o_r / sum_r 2^(lse_r - Lm), Lm = max_r lse_r, over
// the ranks with rows of the sequence (lse_r > -inf).
__device__ __forceinline__ float combine_ranks(int n, const float (&lr)[8], const float (&o)[8]) {
    float Lm = -INFINITY;
#pragma unroll
    for (int r = 0; r < 8; r++)
        if (r < n) Lm = fmaxf(Lm, lr[r]);
    float L = 0.f, acc = 0.f;
#pragma unroll
    for (int r = 0; r < 8; r++) {
        if (r < n && lr[r] != -INFINITY) {
            const float w = ex2(lr[r] - Lm);
            L += w;
            acc += w * o[r];
        }
    }
    return acc / L;
}

// Exchange of one (head, 32-column slice) of the shard result with the other
// ranks, by the threads of the merge block.  res (held by the threads with
// holder set, column col) and lse are this rank's values.  Per call the block
// bumps its slice counter to seq (every rank makes the same calls, so the
// counters advance in lockstep) and stores its slice row, as (value, seq)
// words, into slot [seq % 2][rank][slice] of every rank's area; each holder
// then waits (bounded) for its column's and the log2-sum-exp words of every
// rank in its own area and combines them:
//   out = sum_r 2^(lse_r - Lm) o_r / sum_r 2^(lse_r - Lm),  Lm = max_r lse_r,
// skipping ranks without rows of the sequence (lse_r = -inf), as
// picoattn_combine_shards does.  Parity double-buffering makes slot reuse
// safe: a rank writes call n+2 into a slot only after its call n+1 saw every
// rank's call n+1 words, written after that rank finished reading call n.
// sbuf: kXchgWords floats of shared memory.
template <int HD, class Sync>
__device__ __forceinline__ void exchange_slice(const DecodeArgs& a, int b, int h, int z, float res, float lse,
                                               bool holder, int col, float* sbuf, uint32_t* s_seq, int tid,
                                               Sync sync) {
    const XchgArgs& x = a.x;
    constexpr int NS = HD / kXchgCols;
    const size_t rows = (size_t)a.n_seqs * a.hq * NS, idx = ((size_t)b * a.hq + h) * NS + z;
    if (tid == 0) {
        uint32_t* ctr = reinterpret_cast<uint32_t*>(x.peers[x.rank] + x.counters) + idx;
        const uint32_t c = *ctr + 1;
        *ctr = c;
        *s_seq = c;
        sbuf[kXchgCols] = lse;
    }
    if (holder) sbuf[col] = res;
    sync();
    const uint32_t seq = *s_seq, par = seq & 1u;
    const size_t my_slot = ((size_t)par * x.n_ranks + x.rank) * rows + idx;
    constexpr int NW = kXchgCols + 1;  // words carrying data
    for (int i = tid; i < NW * x.n_ranks; i += blockDim.x)
        st_word(reinterpret_cast<uint64_t*>(x.peers[i / NW] + x.slots) + my_slot * kXchgWords + i % NW, sbuf[i % NW],
                seq);
    if (holder) {
        const uint64_t* base = reinterpret_cast<const uint64_t*>(x.peers[x.rank] + x.slots);
        auto src = [&](int r) { return base + (((size_t)par * x.n_ranks + r) * rows + idx) * kXchgWords; };
        float lr[8], o[8];  // n_ranks <= 8
        wait_words(x.n_ranks, src, col, seq, lr, o, a.status, x.timeout_ns);
        x.out[((size_t)b * a.hq + h) * HD + z * kXchgCols + col] = combine_ranks(x.n_ranks, lr, o);
    }
}

template <int HD, int DS, int NT, int RPT, class Sync>
__device__ __forceinline__ void merge_slice(const DecodeArgs& a, int G, int b, int h, int z, float* m_s, float* l_s,
                                            float* red, int tid, Sync sync) {
    constexpr int C4 = DS / 4, NG = NT / C4, TPC = NT / DS;
    static_assert(NG * DS <= kMergeMaxPieces, "group sums fit in l_s");
    float* part = l_s;
    const int lane = tid & 31, warp = tid >> 5;
    const size_t row_stride = a.shard_out ? (size_t)(HD + 2) : (size_t)HD;
    float* dst = (a.shard_out ? a.shard_out : a.out) + ((size_t)b * a.hq + h) * row_stride + z * DS;
    const bool lse_writer = z == 0 && tid == 0;
    // exchanging with the other ranks (32-column slices only): every block takes part
    const bool xchg = DS == kXchgCols && a.x.peers != nullptr;
    const int col = tid / TPC, j = tid % TPC;  // output column of this thread (holder: j == 0)
    const int pos = seq_pos(a, b);
    long long R, p0, p1;
    if (a.n_seqs == 1) {  // the attended rows follow from the position (no prefix pass may have run)
        R = p1 = pos_ok(a, pos) ? local_len(a, pos) : 0;
        p0 = 0;
    } else {
        R = a.prefix[a.n_seqs], p0 = a.prefix[b], p1 = a.prefix[b + 1];
    }
    float res, lse;  // this block's column value (holders) and log2-sum-exp
    if (!pos_ok(a, pos) || p0 == p1) {
        // a rejected position: NaN; no rows of this sequence in this shard: an empty partial
        res = pos_ok(a, pos) ? 0.f : __int_as_float(0x7fc00000);
        lse = pos_ok(a, pos) ? -INFINITY : __int_as_float(0x7fc00000);
    } else {
        // the CTAs whose slices hold this sequence's rows (the last row is always in
        // CTA G-1's slice; a sequence starting at row 0 starts in CTA 0's, which may
        // be empty when R < G: such pieces are skipped)
        const int i_lo = p0 == 0 ? 0 : cta_of_row(p0, R, G);
        const int i_hi = p1 == R ? G - 1 : cta_of_row(p1 - 1, R, G);
        const int W = a.warps_per_head, lw = __ffs(W) - 1;  // W is 1, 2, 4 or 8
        if (i_lo == i_hi && W == 1 && !xchg) return;  // written directly by the attention kernel
        const int n_pieces = (i_hi - i_lo + 1) * W;  // <= kMergeMaxPieces (checked on the host)
        // piece k = (CTA i_lo + k/W, warp k%W) -> slot (cta + seq, warp) of head h
        auto slot_of = [&](int k) -> uint32_t {
            return (uint32_t)h * (uint32_t)a.n_slots + (uint32_t)(((i_lo + (k >> lw) + b) << lw) | (k & (W - 1)));
        };
        for (int k = tid; k < n_pieces; k += NT) {
            const int i = i_lo + (k >> lw);
            float2 ml = make_float2(-INFINITY, 0.f);
            if (R >= G || slice_start(i, R, G) < slice_start(i + 1, R, G))
                ml = __ldcg(reinterpret_cast<const float2*>(a.part_ml + (size_t)slot_of(k) * 2));
            m_s[k] = ml.x;
            l_s[k] = ml.y;
        }
        const int c4 = tid % C4, grp = tid / C4;
        const float* po = a.part_o + z * DS + c4 * 4;
        float4 ov[RPT];
#pragma unroll
        for (int u = 0; u < RPT; u++) {
            const int k = grp + u * NG;
            ov[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (k < n_pieces) ov[u] = __ldcg(reinterpret_cast<const float4*>(po + (size_t)slot_of(k) * HD));
        }
        sync();
        float mloc = -INFINITY;
        for (int k = tid; k < n_pieces; k += NT) mloc = fmaxf(mloc, m_s[k]);
        for (int o = 16; o; o >>= 1) mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, o));
        if (lane == 0) red[warp] = mloc;
        sync();
        float M = red[0];
#pragma unroll
        for (int w = 1; w < NT / 32; w++) M = fmaxf(M, red[w]);
        float lloc = 0.f;
        for (int k = tid; k < n_pieces; k += NT) {
            const float m = m_s[k];
            const float wgt = m == -INFINITY ? 0.f : ex2(m - M);
            lloc += wgt * l_s[k];
            m_s[k] = wgt;
        }
        for (int o = 16; o; o >>= 1) lloc += __shfl_xor_sync(0xffffffffu, lloc, o);
        sync();  // every thread has read red[] for M; weights complete; l_s free
        if (lane == 0) red[warp] = lloc;
        // weighted acc rows (pieces of weight 0 may hold stale slots: skipped)
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < RPT; u++) {
            const int k = grp + u * NG;
            const float wgt = k < n_pieces ? m_s[k] : 0.f;
            if (wgt != 0.f)
                acc.x += wgt * ov[u].x, acc.y += wgt * ov[u].y, acc.z += wgt * ov[u].z, acc.w += wgt * ov[u].w;
        }
        for (int k = grp + RPT * NG; k < n_pieces; k += NG) {  // beyond RPT rows per thread
            const float wgt = m_s[k];
            if (wgt != 0.f) {
                const float4 v = __ldcg(reinterpret_cast<const float4*>(po + (size_t)slot_of(k) * HD));
                acc.x += wgt * v.x, acc.y += wgt * v.y, acc.z += wgt * v.z, acc.w += wgt * v.w;
            }
        }
        *reinterpret_cast<float4*>(part + grp * DS + c4 * 4) = acc;
        sync();
        float L = 0.f;
#pragma unroll
        for (int w = 0; w < NT / 32; w++) L += red[w];
        // the NG group sums of column col: TPC threads of one warp, NG / TPC each
        float o = 0.f;
#pragma unroll
        for (int g2 = j; g2 < NG; g2 += TPC) o += part[g2 * DS + col];
#pragma unroll
        for (int sh = TPC / 2; sh; sh >>= 1) o += __shfl_xor_sync(0xffffffffu, o, sh);
        res = o / L;
        lse = M + __log2f(L);
        sync();  // m_s, l_s and red may be reused
    }
    if (xchg) {
        exchange_slice<HD>(a, b, h, z, res, lse, j == 0, col, m_s, reinterpret_cast<uint32_t*>(red), tid, sync);
    } else {
        if (j == 0) dst[col] = res;
        if (a.shard_out && lse_writer) dst[HD] = lse;
    }
}

// Merge for one sequence: one block per q head (plan.merge_blocks), launched
// while the attention kernel runs (programmatic dependent launch); its blocks
// take SMs as attention CTAs exit and wait for the attention kernel to
// complete.  Block i takes heads i, i + gridDim.x, ...; a head's G*W pieces
// (acc rows, and their (max, sum) pairs) are contiguous in the partial slots.
// The merge's time is set by the round trips it makes: each chunk of up
// to MergeSeqShape::CK pieces (a whole head for one piece per attention CTA)
// arrives by one bulk copy (TMA: its cost is per copy, not per byte), and the
// block keeps kMergeSeqRing chunks, its whole share for a 16K-row shard, in
// flight.  Per chunk warp 0 folds the (max, sum) pairs into the running
// log2-sum-exp and writes each piece's weight to shared memory; then thread
// (column, group) adds the weighted acc rows of every NG-th piece (four
// independent sums, no branch), and the groups are added when the head is
// done.  Calls with a peer exchange take the column-slice merge instead.
constexpr int kMergeSeqThreads = 512;
constexpr int kMergeSeqRing = 3;
constexpr int kMergeSeqMaxUnits = 512;  // (head, 32-column slice) units of one block: hq <= 128

template <int HD>
struct MergeSeqShape {
    static constexpr int CK = HD == 128 ? 144 : 280;  // pieces per chunk slot (72 / 70 KB of acc rows)
    static constexpr int NG = kMergeSeqThreads / HD;
    static constexpr int off_bar = 0;
    static constexpr int off_seq = 32;
    static constexpr int off_w = off_seq + kMergeSeqMaxUnits * 4;  // [CK] weights, then keep, L, M
    static constexpr int off_ml = (off_w + (CK + 32) * 4 + 15) / 16 * 16;
    static constexpr int off_buf = (off_ml + kMergeSeqRing * (CK + 2) * 8 + 127) / 128 * 128;
    static constexpr int off_red = off_buf + kMergeSeqRing * CK * HD * 4;
    static constexpr int bytes = off_red + 2 * NG * HD * 4;  // group sums, double-buffered by head
    static_assert(bytes <= 227 * 1024, "one block per SM");
};

template <int HD>
__global__ void __launch_bounds__(kMergeSeqThreads, 1) decode_merge_seq_kernel(DecodeArgs a, int G) {
    pdl_trigger();
    using Sh = MergeSeqShape<HD>;
    constexpr int NG = Sh::NG, CK = Sh::CK, NR = kMergeSeqRing;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Sh::off_bar);
    float* w_s = reinterpret_cast<float*>(smem + Sh::off_w);
    float2* ml_s = reinterpret_cast<float2*>(smem + Sh::off_ml);
    float* buf = reinterpret_cast<float*>(smem + Sh::off_buf);
    float* red = reinterpret_cast<float*>(smem + Sh::off_red);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int col = tid % HD, grp = tid / HD;
    const int pos = seq_pos(a, 0);
    const bool ok = pos_ok(a, pos);
    const long long R = ok ? local_len(a, pos) : 0;
    const int W = a.warps_per_head, lw = __ffs(W) - 1;  // W is 1, 2, 4 or 8
    const bool empty = !ok || R == 0;  // a rejected position: NaN; no rows in this shard: an empty partial
    if (!empty && G == 1 && W == 1) {  // written directly by the attention kernel
        pdl_wait();
        return;
    }
    const int n_heads = (int)blockIdx.x < a.hq ? (a.hq - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int n_pieces = G * W;
    const int n_chunks = (n_pieces + CK - 1) / CK;
    const int cpc = ((n_pieces + n_chunks - 1) / n_chunks + 1) & ~1;  // pieces per chunk: even, <= CK
    const int n_steps = empty ? 0 : n_heads * n_chunks;
    auto head_of = [&](int hi) { return (int)blockIdx.x + hi * (int)gridDim.x; };
    // a finished head: threads tid < HD hold column tid (warp z = slice z)
    auto finish = [&](int hi, float res, float lse) {
        const int h = head_of(hi);
        {
            const size_t row_stride = a.shard_out ? (size_t)(HD + 2) : (size_t)HD;
            float* dst = (a.shard_out ? a.shard_out : a.out) + (size_t)h * row_stride;
            dst[tid] = res;
            if (a.shard_out && tid == 0) dst[HD] = lse;
        }
    };
    // step -> (head hi, chunk c) in ring slot step % NR, by thread 0: two bulk
    // copies (acc rows; the (max, sum) pairs rounded up to an even count, a
    // 16-byte multiple: the slot after a head's last piece exists, n_slots > G*W,
    // and chunk starts are even, n_slots even)
    auto issue = [&](int step) {
        const int hi = step / n_chunks, c = step % n_chunks, sl = step % NR;
        const int k0 = c * cpc, cnt = min(cpc, n_pieces - k0);
        const size_t first = (size_t)head_of(hi) * a.n_slots + k0;
        const uint32_t ob = (uint32_t)cnt * HD * 4u, mb = (uint32_t)((cnt + 1) & ~1) * 8u;
        mbar_arrive_expect_tx(&full[sl], ob + mb);
        bulk_g2s(buf + (size_t)sl * CK * HD, a.part_o + first * HD, ob, &full[sl]);
        bulk_g2s(ml_s + sl * (CK + 2), a.part_ml + first * 2, mb, &full[sl]);
    };
    // The position (read above: no kernel of this library writes it, and a
    // caller's kernel that does completes before this one starts) and the
    // barriers are set up before waiting for the attention kernel, whose
    // partials are read only after the wait.
    if (tid == 0) {
        for (int sl = 0; sl < NR; sl++) mbar_init(&full[sl], 1);
        fence_mbar_init();
    }
    pdl_wait();
    if (tid == 0)
        for (int j = 0; j < NR && j < n_steps; j++) issue(j);
    __syncthreads();
    if (empty && tid < HD)
        for (int hi = 0; hi < n_heads; hi++)
            finish(hi, ok ? 0.f : __int_as_float(0x7fc00000), ok ? -INFINITY : __int_as_float(0x7fc00000));
    float M = -INFINITY, L = 0.f;  // running log2-sum-exp of the head (warp 0)
    float acc = 0.f;               // this thread's group sum of column col
    bool live = true;              // the waits have not timed out
    for (int step = 0; step < n_steps; step++) {
        const int hi = step / n_chunks, c = step % n_chunks, sl = step % NR;
        const int k0 = c * cpc, cnt = min(cpc, n_pieces - k0);
        if (live) live = mbar_wait(&full[sl], (uint32_t)((step / NR) & 1), a.status);
        const float2* mls = ml_s + sl * (CK + 2);
        const float* bs = buf + (size_t)sl * CK * HD;
        if (warp == 0) {
            // pieces of CTAs with empty slices (R < G) hold stale slots: weight 0
            float cm = -INFINITY;
            for (int j = lane; j < cnt; j += 32) {
                const int i = (k0 + j) >> lw;
                if (R >= G || slice_start(i, R, G) < slice_start(i + 1, R, G)) cm = fmaxf(cm, mls[j].x);
            }
            for (int o = 16; o; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
            const float Mn = fmaxf(M, cm);
            const float keep = Mn == -INFINITY ? 1.f : ex2(M - Mn);  // 0 while M = -inf
            float ls = 0.f;
            for (int j = lane; j < cnt; j += 32) {
                const int i = (k0 + j) >> lw;
                const bool v = Mn != -INFINITY && (R >= G || slice_start(i, R, G) < slice_start(i + 1, R, G));
                const float wj = v ? ex2(mls[j].x - Mn) : 0.f;
                w_s[j] = wj;
                if (v) ls += wj * mls[j].y;
            }
            for (int o = 16; o; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
            L = L * keep + ls;
            M = Mn;
            if (lane == 0) w_s[CK] = keep, w_s[CK + 1] = L, w_s[CK + 2] = M;
        }
        __syncthreads();  // weights of this chunk
        // read now: warp 0 rewrites them in the next step, after the barrier below
        const float keep = w_s[CK], Lh = w_s[CK + 1], Mh = w_s[CK + 2];
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
        int j = grp;
        for (; j + 3 * NG < cnt; j += 4 * NG) {
            const float w0 = w_s[j], w1 = w_s[j + NG], w2 = w_s[j + 2 * NG], w3 = w_s[j + 3 * NG];
            const float v0 = bs[j * HD + col], v1 = bs[(j + NG) * HD + col];
            const float v2 = bs[(j + 2 * NG) * HD + col], v3 = bs[(j + 3 * NG) * HD + col];
            s0 += w0 != 0.f ? w0 * v0 : 0.f;  // weight 0: a stale slot may hold anything
            s1 += w1 != 0.f ? w1 * v1 : 0.f;
            s2 += w2 != 0.f ? w2 * v2 : 0.f;
            s3 += w3 != 0.f ? w3 * v3 : 0.f;
        }
        for (; j < cnt; j += NG) {
            const float w0 = w_s[j];
            s0 += w0 != 0.f ? w0 * bs[j * HD + col] : 0.f;
        }
        acc = acc * keep + ((s0 + s1) + (s2 + s3));
        const bool last = c == n_chunks - 1;
        float* rh = red + (hi & 1) * NG * HD;
        if (last) rh[grp * HD + col] = acc;
        __syncthreads();  // slot sl and the weights are read; group sums complete
        // the slot is free: the chunk NR steps ahead goes into it
        if (tid == 0 && step + NR < n_steps) issue(step + NR);
        if (last) {
            // the head is done: its group sums, in the half of red for its parity
            // (the next head's sums may be written while the column threads still
            // read these; the head after that writes here only after they passed
            // another barrier)
            if (tid < HD) {
                float o = 0.f;
#pragma unroll
                for (int g2 = 0; g2 < NG; g2++) o += rh[g2 * HD + tid];
                finish(hi, o / Lh, Mh + __log2f(Lh));
            }
            acc = 0.f;
            M = -INFINITY, L = 0.f;
        }
    }
}

// RPT: acc rows per thread held in registers, enough for one long sequence's
// pieces (one per attention CTA) with 32- or 64-column slices; the whole-row
// variant serves many short sequences of a few pieces each and keeps two.
template <int HD, int DS, int NT>
struct MergeRows {
    static constexpr int NG = NT / (DS / 4);
    static constexpr int value = DS == HD ? 2 : ((160 + NG - 1) / NG < 10 ? (160 + NG - 1) / NG : 10);
};

// The merge as its own kernel: block (head, sequence, column slice).  The next
// kernel may launch at once (pdl_trigger first); with 256 threads, at most 64
// registers and ~11 KB of shared memory a block fits on an SM beside an
// attention CTA of the next call.
template <int HD, int DS>
__global__ void __launch_bounds__(256, 4) decode_merge_kernel(DecodeArgs a, int G) {
    __shared__ float m_s[kMergeMaxPieces];
    __shared__ float l_s[kMergeMaxPieces];
    __shared__ float red[8];
    pdl_trigger();
    pdl_wait();
    merge_slice<HD, DS, 256, MergeRows<HD, DS, 256>::value>(a, G, blockIdx.y, blockIdx.x, blockIdx.z, m_s, l_s, red,
                                                            threadIdx.x, [] { __syncthreads(); });
}

// ---------------------------------------------------------------------------
// attn: persistent split-KV GQA attention
// ---------------------------------------------------------------------------

// Calls fn(b, row_begin, row_end, whole, seq_rows) for each sequence segment
// of this CTA's slice, in order (rows local to the sequence; seq_rows = the
// sequence's attended rows in this slab).
template <typename F>
__device__ __forceinline__ void for_each_segment(const DecodeArgs& a, const long long* prefix, long long R0,
                                                 long long R1, F&& fn) {
    // first sequence: the last b with prefix[b] <= R0 (binary search)
    int lo = 0, hi = a.n_seqs;  // prefix[lo] <= R0 < prefix[hi] for the answer lo
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (prefix[mid] <= R0) lo = mid;
        else hi = mid;
    }
    for (int b = lo; b < a.n_seqs; b++) {
        const long long p0 = prefix[b], p1 = prefix[b + 1];
        if (p0 >= R1) break;
        const long long s = max(R0, p0), e = min(R1, p1);
        if (e > s) fn(b, (int)(s - p0), (int)(e - p0), p0 == s && p1 == e, (int)(p1 - p0));
    }
}

// The A operand of the QK^T MMA for the G q heads of KV head kvh of sequence b
// (rows = heads, padded to 16 with zeros): per-head QK-RMSNorm and RoPE with
// the prep helpers (the reference's operation order, prep_common.cuh), scaled
// by log2(e)/sqrt(hd) so scores come out in log2 units (the reference divides by
// sqrtf(hd) and uses expf), rounded to fp16.  Four heads at a time pass through
// the warp's staging area sq (4*HD floats) into the lanes that hold their rows.
// The RoPE row of the position and the q-norm weights (QRot::load) are
// constants of the model, so a caller may load them before waiting for the
// kernel that writes q.
template <int HD>
struct QRot {
    RopeLane<HD> rl;
    float w[HD / 32];  // the q-norm weights of this lane's elements, shared by every head
    __device__ __forceinline__ void load(const DecodeArgs& a, int pos, int lane) {
        rope_lane_load<HD>(rl, a.rope_cos + (size_t)pos * (HD / 2), a.rope_sin + (size_t)pos * (HD / 2), a.rope_mode,
                           lane);
        if (a.qn_w) {
#pragma unroll
            for (int j = 0; j < HD / 32; j++) w[j] = a.qn_w[(HD / 32) * lane + j];
        }
    }
};

template <int HD>
__device__ __forceinline__ void q_fragments(const DecodeArgs& a, int b, const QRot<HD>& qr, int kvh, float* sq,
                                            int lane, uint32_t (&qa)[HD / 16][4]) {
    constexpr int V = HD / 32;
    const int G_q = a.g, gid = lane >> 2, tig = lane & 3;
    const float qscale = 1.4426950408889634f / sqrtf((float)HD);
#pragma unroll
    for (int kk = 0; kk < HD / 16; kk++) qa[kk][0] = qa[kk][1] = qa[kk][2] = qa[kk][3] = 0u;
    const float* qb = a.q + ((size_t)b * a.hq + (size_t)kvh * G_q) * HD;
    // four heads at a time; the next four heads' loads are issued before this
    // group's arithmetic, so their latency overlaps it
    Vec<HD> xn[4];
    auto load4 = [&](int u0) {
#pragma unroll
        for (int u = 0; u < 4; u++) {
            if (u0 + u < G_q) vec_load<HD>(xn[u], qb, (size_t)(u0 + u) * HD, PICOATTN_DTYPE_F32, lane);
            else
#pragma unroll
                for (int j = 0; j < V; j++) xn[u].x[j] = 0.f;
        }
    };
    load4(0);
    for (int u0 = 0; u0 < G_q; u0 += 4) {
        Vec<HD> x[4];
        bool live[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            x[u] = xn[u];
            live[u] = u0 + u < G_q;
        }
        if (u0 + 4 < G_q) load4(u0 + 4);
        if (a.qn_w) vec_rmsnorm4<HD>(x, qr.w, live, a.eps, sq, lane);
#pragma unroll
        for (int u = 0; u < 4; u++) {
            if (live[u]) {
                vec_rope<HD>(x[u], qr.rl, a.rope_mode, lane);
                vec_store_f32<HD>(x[u], sq + u * HD, lane);
            }
        }
        __syncwarp();
        const int ra = gid - u0, rb = gid + 8 - u0;  // staging rows of this lane's two fragment rows
        const bool ha = ra >= 0 && ra < 4 && gid < G_q, hb = rb >= 0 && rb < 4 && gid + 8 < G_q;
#pragma unroll
        for (int kk = 0; kk < HD / 16; kk++) {
            const int c0 = kk * 16 + 2 * tig, c1 = c0 + 8;
            if (ha) {
                qa[kk][0] = pack_half2(sq[ra * HD + c0] * qscale, sq[ra * HD + c0 + 1] * qscale);
                qa[kk][2] = pack_half2(sq[ra * HD + c1] * qscale, sq[ra * HD + c1 + 1] * qscale);
            }
            if (hb) {
                qa[kk][1] = pack_half2(sq[rb * HD + c0] * qscale, sq[rb * HD + c0 + 1] * qscale);
                qa[kk][3] = pack_half2(sq[rb * HD + c1] * qscale, sq[rb * HD + c1 + 1] * qscale);
            }
        }
        __syncwarp();  // sq is reused
    }
}

// The same A operand for a layer without q-norm, straight from the caller's q
// rows.  Lane (gid, tig) holds columns 16kk + 2tig + {0, 1, 8, 9} of heads gid
// and gid + 8, and both columns of every RoPE pair it needs are its own: the
// two columns of a float2 (interleaved), or columns c and c + HD/2, which is
// step kk + HD/32 (NeoX).  So each lane loads its values with float2 loads and
// rotates them in registers, with vec_rope's operations and roundings, then
// scales and rounds them as q_fragments does: the same fragments, without the
// staging through shared memory.  QRope holds the lane's RoPE factors, which
// depend on the position only (loaded before waiting for the kernel that
// writes q).
template <int HD>
struct QRope {
    float c[HD / 8], s[HD / 8];
    __device__ __forceinline__ void load(const DecodeArgs& a, int pos, int lane) {
        const int tig = lane & 3;
        const float* cr = a.rope_cos + (size_t)pos * (HD / 2);
        const float* sr = a.rope_sin + (size_t)pos * (HD / 2);
        if (a.rope_mode == PICOATTN_ROPE_NEOX) {  // factor 4kk + 2h + e: column 16kk + 2tig + 8h + e < HD/2
#pragma unroll
            for (int kk = 0; kk < HD / 32; kk++)
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const int col = 16 * kk + 2 * tig + 8 * h;  // 4-byte loads: the tables need only 4-byte alignment
                    c[4 * kk + 2 * h] = cr[col], c[4 * kk + 2 * h + 1] = cr[col + 1];
                    s[4 * kk + 2 * h] = sr[col], s[4 * kk + 2 * h + 1] = sr[col + 1];
                }
        } else {  // factor 2kk + h: the pair of columns 16kk + 2tig + 8h, +1
#pragma unroll
            for (int kk = 0; kk < HD / 16; kk++)
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const int i = 8 * kk + tig + 4 * h;
                    c[2 * kk + h] = cr[i];
                    s[2 * kk + h] = sr[i];
                }
        }
    }
};

template <int HD>
__device__ __forceinline__ void q_fragments_direct(const DecodeArgs& a, int b, const QRope<HD>& r, int kvh, int lane,
                                                   uint32_t (&qa)[HD / 16][4]) {
    constexpr int K = HD / 16, H = HD / 32;
    const int G_q = a.g, gid = lane >> 2, tig = lane & 3;
    const float qscale = 1.4426950408889634f / sqrtf((float)HD);
#pragma unroll
    for (int kk = 0; kk < K; kk++) qa[kk][0] = qa[kk][1] = qa[kk][2] = qa[kk][3] = 0u;
    const float* qb = a.q + ((size_t)b * a.hq + (size_t)kvh * G_q) * HD + 2 * tig;
#pragma unroll
    for (int half = 0; half < 2; half++) {
        const int row = gid + 8 * half;
        if (row >= G_q) continue;
        float2 x[K][2];
#pragma unroll
        for (int kk = 0; kk < K; kk++)
#pragma unroll
            for (int h = 0; h < 2; h++)
                x[kk][h] = *reinterpret_cast<const float2*>(qb + (size_t)row * HD + 16 * kk + 8 * h);
        float2 y[K][2];
        if (a.rope_mode == PICOATTN_ROPE_NEOX) {
#pragma unroll
            for (int kk = 0; kk < H; kk++)
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const int f = 4 * kk + 2 * h;
                    const float2 lo = x[kk][h], hi = x[kk + H][h];
                    y[kk][h].x = __fsub_rn(__fmul_rn(lo.x, r.c[f]), __fmul_rn(hi.x, r.s[f]));
                    y[kk][h].y = __fsub_rn(__fmul_rn(lo.y, r.c[f + 1]), __fmul_rn(hi.y, r.s[f + 1]));
                    y[kk + H][h].x = __fadd_rn(__fmul_rn(lo.x, r.s[f]), __fmul_rn(hi.x, r.c[f]));
                    y[kk + H][h].y = __fadd_rn(__fmul_rn(lo.y, r.s[f + 1]), __fmul_rn(hi.y, r.c[f + 1]));
                }
        } else {
#pragma unroll
            for (int kk = 0; kk < K; kk++)
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const int f = 2 * kk + h;
                    const float x0 = x[kk][h].x, x1 = x[kk][h].y;
                    y[kk][h].x = __fsub_rn(__fmul_rn(x0, r.c[f]), __fmul_rn(x1, r.s[f]));
                    y[kk][h].y = __fadd_rn(__fmul_rn(x0, r.s[f]), __fmul_rn(x1, r.c[f]));
                }
        }
#pragma unroll
        for (int kk = 0; kk < K; kk++) {
            qa[kk][half] = pack_half2(y[kk][0].x * qscale, y[kk][0].y * qscale);
            qa[kk][2 + half] = pack_half2(y[kk][1].x * qscale, y[kk][1].y * qscale);
        }
    }
}

// The same A operand from the q rows the prep kernel rotated (workspace q_rot).
template <int HD>
__device__ __forceinline__ void q_from_rot(const DecodeArgs& a, int b, int kvh, int lane, uint32_t (&qa)[HD / 16][4]) {
    const int G_q = a.g, gid = lane >> 2, tig = lane & 3;
    const float qscale = 1.4426950408889634f / sqrtf((float)HD);
    const float* qb = a.q_rot + ((size_t)b * a.hq + (size_t)kvh * G_q) * HD;
    const bool ra = gid < G_q, rb = gid + 8 < G_q;
#pragma unroll
    for (int kk = 0; kk < HD / 16; kk++) {
        const int c0 = kk * 16 + 2 * tig, c1 = c0 + 8;
        const float2 v0 = ra ? *reinterpret_cast<const float2*>(qb + gid * HD + c0) : make_float2(0.f, 0.f);
        const float2 v1 = rb ? *reinterpret_cast<const float2*>(qb + (gid + 8) * HD + c0) : make_float2(0.f, 0.f);
        const float2 v2 = ra ? *reinterpret_cast<const float2*>(qb + gid * HD + c1) : make_float2(0.f, 0.f);
        const float2 v3 = rb ? *reinterpret_cast<const float2*>(qb + (gid + 8) * HD + c1) : make_float2(0.f, 0.f);
        qa[kk][0] = pack_half2(v0.x * qscale, v0.y * qscale);
        qa[kk][1] = pack_half2(v1.x * qscale, v1.y * qscale);
        qa[kk][2] = pack_half2(v2.x * qscale, v2.y * qscale);
        qa[kk][3] = pack_half2(v3.x * qscale, v3.y * qscale);
    }
}

// The new k/v row of KV head kvh for one sequence at position pos: QK-RMSNorm
// and RoPE of k and the reference's fp16 rounding of both, the same helpers and
// order as the prep kernel, stored at row lrow of the slab's k and v caches.
template <int HD>
__device__ __forceinline__ void append_row(const DecodeArgs& a, int pos, int kvh, uint16_t* krow, uint16_t* vrow,
                                           float* sq, int lane) {
    constexpr int V = HD / 32;
    Vec<HD> xk, xv;
    vec_load<HD>(xk, a.k, (size_t)kvh * HD, PICOATTN_DTYPE_F32, lane);
    vec_load<HD>(xv, a.v, (size_t)kvh * HD, PICOATTN_DTYPE_F32, lane);
    RopeLane<HD> rl;
    rope_lane_load<HD>(rl, a.rope_cos + (size_t)pos * (HD / 2), a.rope_sin + (size_t)pos * (HD / 2), a.rope_mode,
                       lane);
    if (a.kn_w) {
        float w[V];
#pragma unroll
        for (int j = 0; j < V; j++) w[j] = a.kn_w[V * lane + j];
        vec_rmsnorm<HD>(xk, w, a.eps, sq, lane);
    }
    vec_rope<HD>(xk, rl, a.rope_mode, lane);
    vec_store_ref16<HD>(xk, krow + (size_t)kvh * HD, lane);
    vec_store_ref16<HD>(xv, vrow + (size_t)kvh * HD, lane);
}

// Dynamic shared memory of the attention kernel: a 128-byte header (stage
// barriers <= 48 B, then the single-sequence prefix, position, cache bases, the
// new-row barrier and the CTA's slice), the compute warps' q staging areas, the
// K/V tile stages.
constexpr int kAttnHdrBytes = 128;
constexpr int kAttnMaxSmem = 227 * 1024;
__host__ __device__ constexpr int attn_qstage_bytes(int compute_warps, int hd) { return compute_warps * 4 * hd * 4; }

template <int HD>
__global__ void __launch_bounds__(288, 1) decode_attn_kernel(DecodeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NW = a.compute_warps, W = a.warps_per_head, T = a.tile_rows;
    // The merge kernel may launch now: it waits for this grid to complete.
    pdl_trigger();
    const uint32_t row_bytes = (uint32_t)a.kvd * 2u;
    // A tile of T rows is 8 groups of Gr = T/8 consecutive rows, each group
    // padded by 16 bytes; an ldmatrix 8x8 matrix takes one row from each group
    // (rows Gr*q + u, q = 0..7), whose 16-byte pieces then fall in 8 different
    // bank quads (row_bytes is a multiple of 128), so it is conflict-free.
    // Key order within a tile: 16-key group rg holds u = 2rg (keys 0-7 of the
    // MMA) and u = 2rg + 1 (keys 8-15), q = the key's position in each half.
    const int Gr = T / 8;
    const uint32_t gstride = (uint32_t)Gr * row_bytes + 16u;
    const uint32_t stride = row_bytes + 16u;             // the tile's space: T padded rows
    const uint32_t tile_bytes = (uint32_t)T * stride;  // >= 8 * gstride
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + a.stages;
    long long* s_prefix = reinterpret_cast<long long*>(smem + 48);
    int* s_pos = reinterpret_cast<int*>(smem + 64);
    uint16_t** s_base = reinterpret_cast<uint16_t**>(smem + 72);
    uint64_t* row_ready = reinterpret_cast<uint64_t*>(smem + 88);  // fused append: the new row is in memory
    long long* s_slice = reinterpret_cast<long long*>(smem + 96);  // R, R0, R1 (below)
    float* qstage = reinterpret_cast<float*>(smem + kAttnHdrBytes);
    uint8_t* tiles = smem + kAttnHdrBytes + attn_qstage_bytes(NW, HD);
    const size_t slab = (size_t)a.layer * a.local_rows * a.kvd;

    // Programmatic dependent launch: this kernel may start while the kernels
    // before it still run.  With one sequence its attended rows follow from the
    // position alone, so the CTAs lay out their slices and stream the cache
    // rows that are already final at once; q, k and v are caller inputs that the
    // kernel before may still be writing, so the compute warps wait for it
    // before they read and rotate them.  The new k/v row comes from
    // the prep kernel (waited for before the tile that holds it) or, when all
    // stages run in one call (fused_append), from this kernel: the CTA whose
    // slice holds it computes and stores it first, and its producer waits for
    // those stores.  Results are written only after pdl_wait(), since the kernel
    // before may still read the partial slots.  With several sequences the CTAs
    // wait for the prep kernel's row prefix sums first.  Every CTA waits before
    // it exits, so this grid completes after the kernels before it.
    //
    // The producer warp sets the CTA up (position, cache bases, barriers, its
    // slice) and starts streaming at once; the compute warps of a fused call
    // wait for the kernel before, rotate q (they load the position themselves)
    // and meet the producer's setup at a named barrier.
    const long long* prefix = a.n_seqs == 1 ? s_prefix : a.prefix;
    if (a.n_seqs != 1) pdl_wait();
    uint32_t qa[HD / 16][4];  // the q rows of this compute warp's KV head (MMA A operand)
    constexpr int kSetupBar = 1;
    if (warp == NW) {
        if (a.n_seqs == 1) {
            if (lane == 0) {
                const int p = seq_pos(a, 0);
                s_pos[0] = p;
                s_prefix[0] = 0;
                s_prefix[1] = pos_ok(a, p) ? local_len(a, p) : 0;
                if (a.fused_append && !pos_ok(a, p) && blockIdx.x == 0) atomicOr(a.status, PICOATTN_DEV_BAD_POS);
            } else if (lane == 1) {  // the cache bases, loaded alongside the position
                s_base[0] = seq_kcache(a, 0);
                s_base[1] = seq_vcache(a, 0);
            }
            __syncwarp();
        }
        if (lane == 0) {
            for (int s = 0; s < a.stages; s++) {
                mbar_init(&full[s], 1);
                mbar_init(&empty[s], (uint32_t)NW);
            }
            mbar_init(row_ready, (uint32_t)a.hkv);  // one writer warp per KV head
            fence_mbar_init();
            // this CTA's slice [R0, R1) of the R concatenated rows, computed once
            const int G = (int)gridDim.x, cta = (int)blockIdx.x;
            const long long R = prefix[a.n_seqs];
            s_slice[0] = R;
            if ((unsigned long long)R * (unsigned)G < (1ull << 32)) {  // the same quotients in 32 bits
                const unsigned r = (unsigned)R, g = (unsigned)G, c = (unsigned)cta;
                s_slice[1] = c * r / g;
                s_slice[2] = (c + 1u) * r / g;
            } else {
                s_slice[1] = slice_start(cta, R, G);
                s_slice[2] = slice_start(cta + 1, R, G);
            }
        }
        __syncwarp();
        named_bar_arrive(kSetupBar, blockDim.x);
    } else {
        if (a.fused_append) {  // one sequence: q from the caller's buffer, rotated here
            // The position, its RoPE row and the q-norm weights are read at once
            // (no kernel of this library writes them, and a kernel of the caller's
            // that does has completed before this one starts: it makes no early
            // launch); q, k and v may come from the kernel before this one (a
            // projection that let this kernel launch early), so they are read only
            // after waiting for it.
            int p = 0;
            if (lane == 0) p = seq_pos(a, 0);
            p = __shfl_sync(0xffffffffu, p, 0);
            // a rejected position leaves no rows (the CTA exits below) and must not
            // index the RoPE table
            const bool p_ok = pos_ok(a, p);
            if (a.qn_w == nullptr) {
                QRope<HD> qr;
                if (p_ok) qr.load(a, p, lane);
                pdl_wait();
                if (p_ok) q_fragments_direct<HD>(a, 0, qr, warp / W, lane, qa);
            } else {
                QRot<HD> qr;
                if (p_ok) qr.load(a, p, lane);
                pdl_wait();
                if (p_ok) q_fragments<HD>(a, 0, qr, warp / W, qstage + warp * 4 * HD, lane, qa);
            }
        }
        named_bar_sync(kSetupBar, blockDim.x);
    }
    const long long R = s_slice[0], R0 = s_slice[1], R1 = s_slice[2];
    if (R0 >= R1) {
        pdl_wait();
        return;
    }
    // fused append: the new row (local row R-1 when it lies in this slab) is in
    // this CTA's slice
    const int new_lrow = a.fused_append ? s_pos[0] - a.row_offset : -1;
    const bool has_new = a.fused_append && new_lrow >= 0 && new_lrow < a.local_rows && new_lrow == R - 1 &&
                         R0 <= new_lrow && new_lrow < R1;

    if (warp == NW) {
        // ---------------- producer: TMA bulk copies of whole cache rows --------
        int t = 0;  // tile counter across segments
        bool ok = true, dep_done = a.n_seqs > 1;
        for_each_segment(a, prefix, R0, R1, [&](int b, int r0, int r1, bool, int seq_rows) {
            const uint16_t* kslab = (a.n_seqs == 1 ? s_base[0] : seq_kcache(a, b)) + slab;
            const uint16_t* vslab = (a.n_seqs == 1 ? s_base[1] : seq_vcache(a, b)) + slab;
            if (((uintptr_t)kslab | (uintptr_t)vslab) & 15u) {
                // flagged; the tiles still arrive (with zero-length copies avoided by
                // loading nothing and completing the barrier) so consumers stay in step
                if (lane == 0) atomicOr(a.status, PICOATTN_DEV_MISALIGNED);
                kslab = vslab = nullptr;
            }
            for (int row0 = r0; row0 < r1; row0 += T, t++) {
                const int s = t % a.stages, use = t / a.stages;
                if (ok && use > 0) ok = mbar_wait(&empty[s], (uint32_t)((use - 1) & 1), a.status);
                const int valid = min(T, r1 - row0);
                if (kslab == nullptr) {
                    if (lane == 0) mbar_arrive(&full[s]);
                    continue;
                }
                if (row0 + T >= r1 && r1 == seq_rows) {  // the tile holds the new row
                    if (has_new) {
                        if (ok) ok = mbar_wait(row_ready, 0u, a.status);
                    } else if (!dep_done && !a.fused_append) {
                        pdl_wait();
                        dep_done = true;
                    }
                }
                if (lane == 0) mbar_arrive_expect_tx(&full[s], 2u * (uint32_t)T * row_bytes);
                __syncwarp();
                uint8_t* kdst = tiles + (size_t)s * 2u * tile_bytes;
                // The tile's rows in 8 groups of Gr = T/8 consecutive rows, one bulk
                // copy per group (a copy's cost is per copy, not per byte).  A group
                // may reach past the segment into rows that are final and finite
                // (other slices' rows; their scores are masked) but never to a row
                // that is unwritten or still being written: the sequence's new row
                // only after this CTA waited for it (rows_ok).  Such a group, and
                // rows past the segment end, go row by row, rows past the end
                // repeating its last row: finite data, masked, so no stale shared
                // memory is ever used.
                const int rows_ok = (dep_done || has_new) ? seq_rows : seq_rows - 1;
                for (int i = lane; i < 16; i += 32) {
                    const int kv = i >> 3, q = i & 7;
                    const uint16_t* base = kv ? vslab : kslab;
                    uint8_t* dst = kdst + kv * tile_bytes + (uint32_t)q * gstride;
                    const int g0 = row0 + Gr * q;
                    if (g0 + Gr <= rows_ok) {
                        bulk_g2s(dst, base + (size_t)g0 * a.kvd, (uint32_t)Gr * row_bytes, &full[s]);
                    } else {
                        for (int u = 0; u < Gr; u++) {
                            const int src_row = row0 + min(Gr * q + u, valid - 1);
                            bulk_g2s(dst + (uint32_t)u * row_bytes, base + (size_t)src_row * a.kvd, row_bytes,
                                     &full[s]);
                        }
                    }
                }
                if (a.n_seqs == 1 && t == a.stages - 1) {
                    // One sequence: with the ring's first tiles requested, the rows
                    // after them (final rows only, up to ~40 MB over the grid) are
                    // requested into L2 at once, so the cache keeps streaming while
                    // the kernels before this one (the previous layer's merge and
                    // exchange) finish and the compute warps wait for q; the ring
                    // then reads them from L2.  A hint: nothing waits for it.
                    const int ahead = (int)((40u << 20) / gridDim.x / (2u * row_bytes));
                    const int p0 = row0 + T, p1 = min(min(r1, rows_ok), p0 + ahead);
                    if (p1 > p0) {
                        const int per = (p1 - p0 + 15) / 16;
                        const int c0 = p0 + (lane & 15) * per, c1 = min(p1, c0 + per);
                        if (c1 > c0)
                            bulk_prefetch_l2((lane >> 4 ? vslab : kslab) + (size_t)c0 * a.kvd,
                                             (uint32_t)(c1 - c0) * row_bytes);
                    }
                }
            }
        });
        return;
    }

    // ---------------- compute warps ----------------------------------------
    const int kvh = warp / W, wi = warp % W;
    const int gid = lane >> 2, tig = lane & 3;
    const int G_q = a.g;
    // ldmatrix row addresses (matrix lane >> 3, row lane & 7 = group q): K
    // matrices (keys 0-7 | dims 0-7, keys 0-7 | dims 8-15, keys 8-15 | ...),
    // V transposed (keys 0-7 | dims 0-7, keys 8-15 | dims 0-7, ...)
    const uint32_t k_lane = (uint32_t)(lane & 7) * gstride + (uint32_t)(lane >> 4) * row_bytes +
                            (uint32_t)(((lane >> 3) & 1) * 16);
    const uint32_t v_lane = (uint32_t)(lane & 7) * gstride + (uint32_t)((lane >> 3) & 1) * row_bytes +
                            (uint32_t)((lane >> 4) * 16);
    const uint32_t head_off = (uint32_t)kvh * HD * 2u;
    const uint32_t tiles_u32 = smem_u32(tiles);
    float* sq = qstage + warp * 4 * HD;
    int t = 0;
    bool dep_done = a.n_seqs > 1;
    if (has_new && wi == 0) {  // the new row of this warp's KV head, before anything else
        uint16_t* krow = s_base[0] + slab + (size_t)new_lrow * a.kvd;
        uint16_t* vrow = s_base[1] + slab + (size_t)new_lrow * a.kvd;
        append_row<HD>(a, s_pos[0], kvh, krow, vrow, sq, lane);
        fence_proxy_async_global();  // the producer's bulk copies read these rows
        __syncwarp();
        if (lane == 0) mbar_arrive(row_ready);
    }

    for_each_segment(a, prefix, R0, R1, [&](int b, int r0, int r1, bool whole, int) {
        if (!a.fused_append) {
            // q rotated by the prep kernel (finished: waited for above or before
            // the new row's tile, which every slice of one sequence reaches last)
            if (!dep_done) {
                pdl_wait();
                dep_done = true;
            }
            q_from_rot<HD>(a, b, kvh, lane, qa);
        }
        float m[2] = {-1e30f, -1e30f}, l[2] = {0.f, 0.f};
        float o[HD / 8][4];
#pragma unroll
        for (int i = 0; i < HD / 8; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

        for (int row0 = r0; row0 < r1; row0 += T, t++) {
            const int s = t % a.stages;
            mbar_wait(&full[s], (uint32_t)((t / a.stages) & 1), a.status);
            const int valid = min(T, r1 - row0);
            const uint32_t kbase = tiles_u32 + (uint32_t)s * 2u * tile_bytes + head_off;
            const uint32_t vbase = kbase + tile_bytes;
            for (int rg = wi; rg * 16 < T && 2 * rg < valid; rg += W) {
                const uint32_t goff = (uint32_t)(2 * rg) * row_bytes;
                float sc[2][4];
#pragma unroll
                for (int j = 0; j < 2; j++) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
                for (int kk = 0; kk < HD / 16; kk++) {
                    uint32_t bk[4];
                    ldsm_x4(bk, kbase + goff + k_lane + (uint32_t)kk * 32u);
                    mma_16816(sc[0], qa[kk], bk[0], bk[1]);
                    mma_16816(sc[1], qa[kk], bk[2], bk[3]);
                }
                // key (S column 2tig + (e & 1) of half j) = row Gr * column + 2rg + j
                if (Gr * 7 + 2 * rg + 1 >= valid) {
#pragma unroll
                    for (int j = 0; j < 2; j++)
#pragma unroll
                        for (int e = 0; e < 4; e++)
                            if (Gr * (2 * tig + (e & 1)) + 2 * rg + j >= valid) sc[j][e] = -INFINITY;
                }
                float mx0 = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
                float mx1 = fmaxf(fmaxf(sc[0][2], sc[0][3]), fmaxf(sc[1][2], sc[1][3]));
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
                const float mn0 = fmaxf(m[0], mx0), mn1 = fmaxf(m[1], mx1);
                const float c0 = ex2(m[0] - mn0), c1 = ex2(m[1] - mn1);
                m[0] = mn0;
                m[1] = mn1;
                float p[2][4];
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    p[j][0] = ex2(sc[j][0] - mn0);
                    p[j][1] = ex2(sc[j][1] - mn0);
                    p[j][2] = ex2(sc[j][2] - mn1);
                    p[j][3] = ex2(sc[j][3] - mn1);
                }
                l[0] = l[0] * c0 + ((p[0][0] + p[0][1]) + (p[1][0] + p[1][1]));
                l[1] = l[1] * c1 + ((p[0][2] + p[0][3]) + (p[1][2] + p[1][3]));
                if (__any_sync(0xffffffffu, c0 != 1.f || c1 != 1.f)) {
#pragma unroll
                    for (int i = 0; i < HD / 8; i++) {
                        o[i][0] *= c0;
                        o[i][1] *= c0;
                        o[i][2] *= c1;
                        o[i][3] *= c1;
                    }
                }
                const uint32_t pa[4] = {pack_half2(p[0][0], p[0][1]), pack_half2(p[0][2], p[0][3]),
                                        pack_half2(p[1][0], p[1][1]), pack_half2(p[1][2], p[1][3])};
#pragma unroll
                for (int dt = 0; dt < HD / 16; dt++) {
                    uint32_t bv[4];
                    ldsm_x4_t(bv, vbase + goff + v_lane + (uint32_t)dt * 32u);
                    mma_16816(o[2 * dt], pa, bv[0], bv[1]);
                    mma_16816(o[2 * dt + 1], pa, bv[2], bv[3]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }

        // flush this segment: normalised output if the CTA saw the whole
        // sequence (and one warp per head), else the (max, sum, acc) partial.
        // The kernel before may still read the partial slots and outputs.
        if (!dep_done) {
            pdl_wait();
            dep_done = true;
        }
        l[0] += __shfl_xor_sync(0xffffffffu, l[0], 1);
        l[0] += __shfl_xor_sync(0xffffffffu, l[0], 2);
        l[1] += __shfl_xor_sync(0xffffffffu, l[1], 1);
        l[1] += __shfl_xor_sync(0xffffffffu, l[1], 2);
        const bool direct = whole && W == 1 && a.x.peers == nullptr;
        const size_t slot = (size_t)(blockIdx.x + b) * W + wi;
#pragma unroll
        for (int half = 0; half < 2; half++) {
            const int r = gid + 8 * half;
            if (r < G_q) {
                const int h = kvh * G_q + r;
                if (direct) {
                    const float inv = 1.0f / l[half];
                    float* od = a.shard_out ? a.shard_out + ((size_t)b * a.hq + h) * (HD + 2) + 2 * tig
                                            : a.out + ((size_t)b * a.hq + h) * HD + 2 * tig;
#pragma unroll
                    for (int i = 0; i < HD / 8; i++)
                        *reinterpret_cast<float2*>(od + i * 8) =
                            make_float2(o[i][2 * half] * inv, o[i][2 * half + 1] * inv);
                    if (a.shard_out && tig == 0)  // log2-sum-exp of this shard's scores
                        a.shard_out[((size_t)b * a.hq + h) * (HD + 2) + HD] = m[half] + __log2f(l[half]);
                } else {
                    const size_t pi = (size_t)h * a.n_slots + slot;
                    float* od = a.part_o + pi * HD + 2 * tig;
#pragma unroll
                    for (int i = 0; i < HD / 8; i++)
                        *reinterpret_cast<float2*>(od + i * 8) = make_float2(o[i][2 * half], o[i][2 * half + 1]);
                    if (tig == 0)
                        *reinterpret_cast<float2*>(a.part_ml + pi * 2) = make_float2(m[half], l[half]);
                }
            }
        }
    });
}

// Launch with programmatic stream serialisation: the kernel may start while the
// one before it in the stream finishes (see pdl_wait / pdl_trigger).
template <typename... P, typename... A>
cudaError_t launch_pdl(void (*kernel)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, A&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<A>(args)...);
}

template <int HD>
cudaError_t launch_decode_hd(const DecodeArgs& a_in, const DecodePlan& plan, cudaStream_t stream, unsigned stages) {
    static PerDeviceOnce setup;
    const cudaError_t se = setup.run([] {
        // The small kernels ask for the largest shared-memory carveout, so that an
        // attention CTA launched early (programmatic dependent launch) fits on an
        // SM that still runs one of them.
        cudaError_t e = cudaFuncSetAttribute(decode_attn_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kAttnMaxSmem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(decode_prep_kernel<HD>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(decode_merge_kernel<HD, HD>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(decode_merge_kernel<HD, 64>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(decode_merge_kernel<HD, 32>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(decode_merge_seq_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     MergeSeqShape<HD>::bytes);
        return e;
    });
    if (se != cudaSuccess) return se;
    // One sequence with every stage in this call: the attention kernel appends
    // the new row itself and the merge derives the rows from the position, so
    // no prep kernel runs.
    DecodeArgs a = a_in;
    a.fused_append = (stages == PICOATTN_STAGE_ALL && a.n_seqs == 1) ? 1 : 0;
    cudaError_t e = cudaSuccess;
    if ((stages & PICOATTN_STAGE_PREPARE) && !a.fused_append)
        e = launch_pdl(decode_prep_kernel<HD>, dim3((unsigned)((a.hq + 2 * a.hkv + 31) / 32), (unsigned)a.n_seqs + 1),
                       dim3(256), 0, stream, a);
    if (e == cudaSuccess && (stages & PICOATTN_STAGE_ATTEND))
        e = launch_pdl(decode_attn_kernel<HD>, dim3((unsigned)plan.grid_ctas), dim3((plan.compute_warps + 1) * 32),
                       (size_t)plan.smem_bytes, stream, a);
    // One sequence: one block per q head fed by bulk copies, except with a
    // peer exchange, where the column-slice kernel below posts and combines
    // 32-column slices (measured on B200: the 8-GPU split-KV step at 16K rows
    // per rank 21,805 -> 22,956 GB/s with it, while a whole-model token step
    // on one GPU runs 341 tok/s with the per-head merge against 320).
    if (e == cudaSuccess && (stages & PICOATTN_STAGE_COMBINE) && a.n_seqs == 1 && a.x.peers == nullptr) {
        e = launch_pdl(decode_merge_seq_kernel<HD>, dim3((unsigned)plan.merge_blocks), dim3(kMergeSeqThreads),
                       (size_t)MergeSeqShape<HD>::bytes, stream, a, plan.grid_ctas);
    } else if (e == cudaSuccess && (stages & PICOATTN_STAGE_COMBINE)) {
        // column slices: the narrowest of 32 or 64 columns that keeps the grid
        // within one block per SM (a block beside each attention CTA of the next
        // call), else one block per (head, sequence)
        const long units = (long)a.hq * a.n_seqs;
        const int sms = plan.max_grid / 2;
        const dim3 blk(256);
        if (a.x.peers != nullptr || units * (HD / 32) <= sms)  // the exchange works on 32-column slices
            e = launch_pdl(decode_merge_kernel<HD, 32>, dim3((unsigned)a.hq, (unsigned)a.n_seqs, HD / 32), blk, 0,
                           stream, a, plan.grid_ctas);
        else if (HD > 64 && units * (HD / 64) <= sms)
            e = launch_pdl(decode_merge_kernel<HD, 64>, dim3((unsigned)a.hq, (unsigned)a.n_seqs, HD / 64), blk, 0,
                           stream, a, plan.grid_ctas);
        else if (units >= 2L * plan.max_grid)
            e = launch_pdl(decode_merge_kernel<HD, HD>, dim3((unsigned)a.hq, (unsigned)a.n_seqs, 1), blk, 0, stream,
                           a, plan.grid_ctas);
        else
            e = launch_pdl(decode_merge_kernel<HD, 32>, dim3((unsigned)a.hq, (unsigned)a.n_seqs, HD / 32), blk, 0,
                           stream, a, plan.grid_ctas);
    }
    return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace

int device_sm_count() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
    return n;
}

bool make_decode_plan(const picoattn_config_t& cfg, int n_seqs, int max_ctx, DecodePlan* plan) {
    const int hkv = cfg.n_kv_heads, hd = cfg.head_dim, hq = cfg.n_heads;
    if (!(hkv == 1 || hkv == 2 || hkv == 4 || hkv == 8)) return false;
    if (hd != 64 && hd != 128) return false;
    if (hq % hkv != 0 || hq / hkv > 16) return false;
    DecodePlan p{};
    p.compute_warps = hkv <= 4 ? 4 : 8;
    p.warps_per_head = p.compute_warps / hkv;
    const int kvd = hkv * hd;
    const int stride = kvd * 2 + 16;
    int R = 1;
    p.tile_rows = 16 * p.warps_per_head;
    while (2 * p.tile_rows * stride < 24 * 1024 && R < 4) {
        R *= 2;
        p.tile_rows = 16 * p.warps_per_head * R;
    }
    const int stage_bytes = 2 * p.tile_rows * stride;
    p.stages = 3 * stage_bytes <= 200 * 1024 ? 3 : 2;
    p.smem_bytes = kAttnHdrBytes + attn_qstage_bytes(p.compute_warps, hd) + p.stages * stage_bytes;
    if (p.smem_bytes > kAttnMaxSmem) return false;
    // Persistent grid: as many CTAs as fit at once (smem-limited), but no more
    // than one per 64 rows of the largest possible workload (a 16K-row shard of
    // one sequence still spreads over the SMs).
    const int sms = device_sm_count();
    const int per_sm = p.smem_bytes <= 113 * 1024 ? 2 : 1;
    const long long work_rows = (long long)n_seqs * max_ctx;
    // One sequence: the merge kernel takes one block per q head (up to one per
    // SM).  Its blocks become resident as attention CTAs exit and start the
    // moment the attention kernel completes, each with one head's pieces.  (The
    // next call's attention reads its q only after this merge completes, so
    // nothing is gained by reserving SMs for the merge to overlap it; measured
    // on B200, a head per block on every SM beats 4-16 blocks on reserved SMs at
    // every length: 128K rows 114 -> 93.5 us per layer, a 16K-row shard 25.2 ->
    // 22.0, 4K rows 14.4 -> 13.2.)
    p.merge_blocks = std::min(hq, sms);
    const int attn_sms = sms;
    long long g = std::min<long long>((long long)attn_sms * per_sm, (work_rows + 63) / 64);
    p.grid_ctas = (int)std::max<long long>(1, g);
    p.max_grid = sms * 2;
    // pieces per sequence <= grid_ctas * warps_per_head; the merge kernel holds
    // them in kMergeMaxPieces shared-memory slots
    if (p.max_grid * p.warps_per_head > kMergeMaxPieces) return false;
    p.n_slots = ((p.max_grid + n_seqs) * p.warps_per_head + 1) & ~1;
    const size_t slots = (size_t)p.n_slots;
    size_t off = kWsHeaderBytes;
    p.ws_prefix = off;
    off = align_up(off + (size_t)(n_seqs + 1) * 8, 256);
    p.ws_qrot = off;
    off = align_up(off + (size_t)n_seqs * hq * hd * 4, 256);
    p.ws_ml = off;
    off = align_up(off + slots * hq * 2 * 4, 256);
    p.ws_o = off;
    off = align_up(off + slots * hq * hd * 4, 256);
    p.ws_total = off;
    *plan = p;
    return true;
}

cudaError_t launch_decode(const DecodeArgs& a, const DecodePlan& plan, cudaStream_t stream, unsigned stages) {
    return a.hd == 64 ? launch_decode_hd<64>(a, plan, stream, stages) : launch_decode_hd<128>(a, plan, stream, stages);
}

}  // namespace picoattn
