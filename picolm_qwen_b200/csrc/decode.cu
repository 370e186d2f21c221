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
// into prefix[0..n_seqs]; one block of 256 threads.
__device__ void scan_lengths(const DecodeArgs& a) {
    __shared__ long long warp_tot[8];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int per = (a.n_seqs + 255) / 256;
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
    if (tid == 255) a.prefix[a.n_seqs] = base + incl;
}

template <int HD>
__global__ void __launch_bounds__(256) decode_prep_kernel(DecodeArgs a) {
    if (blockIdx.y == (unsigned)a.n_seqs) {  // the extra block row: length prefix sums
        if (blockIdx.x == 0) scan_lengths(a);
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
// attn: persistent split-KV GQA attention
// ---------------------------------------------------------------------------

// Calls fn(b, row_begin, row_end) for each sequence segment of this CTA's
// slice, in order (rows local to the sequence).
template <typename F>
__device__ __forceinline__ void for_each_segment(const DecodeArgs& a, long long R0, long long R1, F&& fn) {
    // first sequence: the last b with prefix[b] <= R0 (binary search)
    int lo = 0, hi = a.n_seqs;  // prefix[lo] <= R0 < prefix[hi] for the answer lo
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (a.prefix[mid] <= R0) lo = mid;
        else hi = mid;
    }
    for (int b = lo; b < a.n_seqs; b++) {
        const long long p0 = a.prefix[b], p1 = a.prefix[b + 1];
        if (p0 >= R1) break;
        const long long s = max(R0, p0), e = min(R1, p1);
        if (e > s) fn(b, (int)(s - p0), (int)(e - p0), p0 == s && p1 == e);
    }
}

template <int HD>
__global__ void __launch_bounds__(288, 1) decode_attn_kernel(DecodeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NW = a.compute_warps, W = a.warps_per_head, T = a.tile_rows;
    const int G = gridDim.x, cta = blockIdx.x;
    const long long R = a.prefix[a.n_seqs];
    const long long R0 = slice_start(cta, R, G), R1 = slice_start(cta + 1, R, G);
    if (R0 >= R1) return;

    const uint32_t row_bytes = (uint32_t)a.kvd * 2u;
    const uint32_t stride = row_bytes + 16u;  // padded rows: ldmatrix is conflict-free
    const uint32_t tile_bytes = (uint32_t)T * stride;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + a.stages;
    uint8_t* tiles = smem + 128;
    const size_t slab = (size_t)a.layer * a.local_rows * a.kvd;

    if (threadIdx.x == 0) {
        for (int s = 0; s < a.stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], (uint32_t)NW);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == NW) {
        // ---------------- producer: TMA bulk copies of whole cache rows --------
        int t = 0;  // tile counter across segments
        bool ok = true;
        for_each_segment(a, R0, R1, [&](int b, int r0, int r1, bool) {
            const uint16_t* kslab = seq_kcache(a, b) + slab;
            const uint16_t* vslab = seq_vcache(a, b) + slab;
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
                if (lane == 0) mbar_arrive_expect_tx(&full[s], 2u * (uint32_t)T * row_bytes);
                __syncwarp();
                uint8_t* kdst = tiles + (size_t)s * 2u * tile_bytes;
                // Rows past the end of the segment repeat its last row: finite data
                // whose scores are masked, so no stale shared memory is ever used.
                for (int i = lane; i < 2 * T; i += 32) {
                    const int kv = i >= T, r = kv ? i - T : i;
                    const int src_row = row0 + min(r, valid - 1);
                    const uint16_t* src = (kv ? vslab : kslab) + (size_t)src_row * a.kvd;
                    bulk_g2s(kdst + kv * tile_bytes + (uint32_t)r * stride, src, row_bytes, &full[s]);
                }
            }
        });
        return;
    }

    // ---------------- compute warps ----------------------------------------
    const int kvh = warp / W, wi = warp % W;
    const int gid = lane >> 2, tig = lane & 3;
    const int G_q = a.g;
    const float qscale = 1.4426950408889634f / sqrtf((float)HD);
    const uint32_t k_lane = (uint32_t)((lane & 7) + ((lane >> 4) << 3)) * stride + (uint32_t)(((lane >> 3) & 1) * 16);
    const uint32_t v_lane = (uint32_t)((lane & 7) + (((lane >> 3) & 1) << 3)) * stride + (uint32_t)((lane >> 4) * 16);
    const uint32_t head_off = (uint32_t)kvh * HD * 2u;
    const uint32_t tiles_u32 = smem_u32(tiles);
    int t = 0;

    for_each_segment(a, R0, R1, [&](int b, int r0, int r1, bool whole) {
        // q of the G heads of this KV head as the A operand (rows = heads, padded
        // to 16 with zeros), pre-scaled by log2(e)/sqrt(hd) so scores come out in
        // log2 units (the reference divides by sqrtf(hd) and uses expf).
        uint32_t qa[HD / 16][4];
        {
            const float* qb = a.q_rot + ((size_t)b * a.hq + (size_t)kvh * G_q) * HD;
            const bool ra = gid < G_q, rb = gid + 8 < G_q;
#pragma unroll
            for (int kk = 0; kk < HD / 16; kk++) {
                const int c0 = kk * 16 + 2 * tig, c1 = c0 + 8;
                float2 v0 = ra ? *reinterpret_cast<const float2*>(qb + gid * HD + c0) : make_float2(0.f, 0.f);
                float2 v1 = rb ? *reinterpret_cast<const float2*>(qb + (gid + 8) * HD + c0) : make_float2(0.f, 0.f);
                float2 v2 = ra ? *reinterpret_cast<const float2*>(qb + gid * HD + c1) : make_float2(0.f, 0.f);
                float2 v3 = rb ? *reinterpret_cast<const float2*>(qb + (gid + 8) * HD + c1) : make_float2(0.f, 0.f);
                qa[kk][0] = pack_half2(v0.x * qscale, v0.y * qscale);
                qa[kk][1] = pack_half2(v1.x * qscale, v1.y * qscale);
                qa[kk][2] = pack_half2(v2.x * qscale, v2.y * qscale);
                qa[kk][3] = pack_half2(v3.x * qscale, v3.y * qscale);
            }
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
            for (int rg = wi; rg * 16 < valid; rg += W) {
                const uint32_t goff = (uint32_t)(rg * 16) * stride;
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
                const int nvalid = valid - rg * 16;
                if (nvalid < 16) {
#pragma unroll
                    for (int j = 0; j < 2; j++)
#pragma unroll
                        for (int e = 0; e < 4; e++)
                            if (8 * j + 2 * tig + (e & 1) >= nvalid) sc[j][e] = -INFINITY;
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
        // sequence (and one warp per head), else the (max, sum, acc) partial
        l[0] += __shfl_xor_sync(0xffffffffu, l[0], 1);
        l[0] += __shfl_xor_sync(0xffffffffu, l[0], 2);
        l[1] += __shfl_xor_sync(0xffffffffu, l[1], 1);
        l[1] += __shfl_xor_sync(0xffffffffu, l[1], 2);
        const bool direct = whole && W == 1;
        const size_t pbase = ((size_t)(cta + b) * W + wi) * a.hq;
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
                    float* od = a.part_o + (pbase + h) * HD + 2 * tig;
#pragma unroll
                    for (int i = 0; i < HD / 8; i++)
                        *reinterpret_cast<float2*>(od + i * 8) = make_float2(o[i][2 * half], o[i][2 * half + 1]);
                    if (tig == 0)
                        *reinterpret_cast<float2*>(a.part_ml + (pbase + h) * 2) = make_float2(m[half], l[half]);
                }
            }
        }
    });
}

// ---------------------------------------------------------------------------
// merge: out = sum_p 2^(m_p - M) acc_p / sum_p 2^(m_p - M) l_p over the pieces
// ---------------------------------------------------------------------------

// Merges the partial (max, sum, acc) pieces of one (head, sequence) into its
// output; block z handles head-dim columns [z*DS, z*DS+DS), so that few long
// sequences still spread over many blocks.
template <int HD, int DS>
__global__ void __launch_bounds__(256) decode_merge_kernel(DecodeArgs a, int G) {
    // 256 threads: column d = z*DS + tid % DS, piece group = tid / DS; every group
    // sums its pieces with 4 independent accumulators so many loads are in flight
    constexpr int NT = 256, NG = NT / DS;
    __shared__ float w_s[2048];
    __shared__ float red[NT / 32];
    __shared__ float bc[2];
    __shared__ float part[NG][DS];
    const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int dl = tid % DS, grp = tid / DS, d = blockIdx.z * DS + dl;
    const bool lse_writer = blockIdx.z == 0 && dl == 0;
    const size_t row_stride = a.shard_out ? (size_t)(HD + 2) : (size_t)HD;
    float* dst = (a.shard_out ? a.shard_out : a.out) + ((size_t)b * a.hq + h) * row_stride + d;
    const int pos = seq_pos(a, b);
    if (!pos_ok(a, pos)) {
        if (grp == 0) {
            *dst = __int_as_float(0x7fc00000);
            if (a.shard_out && lse_writer) dst[HD - d] = __int_as_float(0x7fc00000);
        }
        return;
    }
    const long long R = a.prefix[a.n_seqs];
    const long long p0 = a.prefix[b], p1 = a.prefix[b + 1];
    if (p0 == p1) {  // no rows of this sequence in this shard: empty partial
        if (grp == 0) {
            *dst = 0.f;
            if (lse_writer) dst[HD] = -INFINITY;
        }
        return;
    }
    const int i_lo = cta_of_row(p0, R, G), i_hi = cta_of_row(p1 - 1, R, G);
    const int W = a.warps_per_head;
    if (i_lo == i_hi && W == 1) return;  // written directly by the attention kernel
    const int n_pieces = (i_hi - i_lo + 1) * W;  // <= 2048 (checked on the host)
    // piece k -> (cta i_lo + k/W, warp k%W); skipped if that CTA's slice is empty
    auto piece = [&](int k) -> size_t { return ((size_t)(i_lo + k / W + b) * W + k % W) * a.hq + h; };
    float mloc = -INFINITY;
    for (int k = tid; k < n_pieces; k += NT) {
        const int i = i_lo + k / W;
        float m = -INFINITY;
        if (slice_start(i, R, G) < slice_start(i + 1, R, G)) m = a.part_ml[piece(k) * 2];
        w_s[k] = m;
        mloc = fmaxf(mloc, m);
    }
    for (int o = 16; o; o >>= 1) mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, o));
    if (lane == 0) red[warp] = mloc;
    __syncthreads();
    if (tid == 0) {
        float M = red[0];
        for (int w = 1; w < NT / 32; w++) M = fmaxf(M, red[w]);
        bc[0] = M;
    }
    __syncthreads();
    const float M = bc[0];
    float lloc = 0.f;
    for (int k = tid; k < n_pieces; k += NT) {
        float wgt = 0.f;
        if (w_s[k] != -INFINITY) {
            wgt = ex2(w_s[k] - M);
            lloc += wgt * a.part_ml[piece(k) * 2 + 1];
        }
        w_s[k] = wgt;
    }
    for (int o = 16; o; o >>= 1) lloc += __shfl_xor_sync(0xffffffffu, lloc, o);
    __syncthreads();
    if (lane == 0) red[warp] = lloc;
    __syncthreads();
    if (tid == 0) {
        float L = 0.f;
        for (int w = 0; w < NT / 32; w++) L += red[w];
        bc[1] = L;
    }
    __syncthreads();
    // 8 independent accumulators: 8 loads of each thread in flight at once
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    int k = grp;
    for (; k + 7 * NG < n_pieces; k += 8 * NG) {
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const float wgt = w_s[k + u * NG];
            if (wgt != 0.f) acc[u] += wgt * a.part_o[piece(k + u * NG) * HD + d];
        }
    }
    for (; k < n_pieces; k += NG) {
        const float wgt = w_s[k];
        if (wgt != 0.f) acc[0] += wgt * a.part_o[piece(k) * HD + d];
    }
    part[grp][dl] = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
    __syncthreads();
    if (grp == 0) {
        float o = part[0][dl];
#pragma unroll
        for (int g2 = 1; g2 < NG; g2++) o += part[g2][dl];
        *dst = o / bc[1];
        if (a.shard_out && lse_writer) dst[HD] = M + __log2f(bc[1]);
    }
}

template <int HD>
cudaError_t launch_decode_hd(const DecodeArgs& a, const DecodePlan& plan, cudaStream_t stream, unsigned stages) {
    static bool attr_done = false;
    if (!attr_done) {
        cudaError_t e = cudaFuncSetAttribute(decode_attn_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             200 * 1024 + 256);
        if (e != cudaSuccess) return e;
        attr_done = true;
    }
    const int n_slots = a.hq + 2 * a.hkv;
    if (stages & PICOATTN_STAGE_PREPARE)
        decode_prep_kernel<HD><<<dim3((unsigned)((n_slots + 31) / 32), (unsigned)a.n_seqs + 1), 256, 0, stream>>>(a);
    if (stages & PICOATTN_STAGE_ATTEND)
        decode_attn_kernel<HD><<<plan.grid_ctas, (plan.compute_warps + 1) * 32, plan.smem_bytes, stream>>>(a);
    if (stages & PICOATTN_STAGE_COMBINE) {
        // one block per (head, sequence) when those fill the GPU twice over, else
        // each also split into HD/32 column slices
        if ((long)a.hq * a.n_seqs >= 2L * plan.max_grid)
            decode_merge_kernel<HD, HD><<<dim3((unsigned)a.hq, (unsigned)a.n_seqs, 1), 256, 0, stream>>>(
                a, plan.grid_ctas);
        else
            decode_merge_kernel<HD, 32><<<dim3((unsigned)a.hq, (unsigned)a.n_seqs, HD / 32), 256, 0, stream>>>(
                a, plan.grid_ctas);
    }
    return cudaGetLastError();
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
    p.smem_bytes = 128 + p.stages * stage_bytes;
    if (p.smem_bytes > 200 * 1024 + 256) return false;
    // Persistent grid: as many CTAs as fit at once (smem-limited), but no more
    // than one per 64 rows of the largest possible workload (a 16K-row shard of
    // one sequence still spreads over every SM).
    const int sms = device_sm_count();
    const int per_sm = p.smem_bytes <= 113 * 1024 ? 2 : 1;
    const long long work_rows = (long long)n_seqs * max_ctx;
    long long g = std::min<long long>((long long)sms * per_sm, (work_rows + 63) / 64);
    p.grid_ctas = (int)std::max<long long>(1, g);
    p.max_grid = sms * 2;
    // pieces per sequence <= grid_ctas * warps_per_head; the merge kernel holds
    // them in 2048 shared-memory slots
    if (p.max_grid * p.warps_per_head > 2048) return false;
    const size_t slots = (size_t)(p.max_grid + n_seqs) * p.warps_per_head;
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
