// decode.cu -- single-token (decode) attention step for sm_100a.
//
// Replaces the inline block of Model::forward, cpp/model.hpp:326-418
// (C engine: picolm/model.c:725-825), for a batch of independent sequences.
//
// Three kernels, in stream order:
//   prep   one CTA per sequence: per-head QK-RMSNorm and RoPE in the reference's
//          exact fp32 operation order, the new k/v row rounded to fp16 with the
//          reference's rounding and stored at row pos of the layer's cache slab,
//          the rotated q kept in the workspace.
//   attn   one CTA per (chunk of cache rows, sequence).  A producer warp streams
//          whole cache rows (all KV heads, contiguous in the reference layout)
//          into shared memory with TMA bulk copies; compute warps, one per KV
//          head (or several per head when there are fewer than four heads), run
//          QK^T and PV for all the q heads of that KV head as tensor-core MMAs,
//          so every q head of a GQA group shares each K/V tile read from HBM.
//          Online softmax in fp32 (log2 domain); each warp emits an
//          un-normalised (max, sum, acc[hd]) partial.
//   merge  log-sum-exp combination of the partials of each (sequence, q head)
//          into the normalised output acc/sum.
#include <cmath>
#include <cstdio>

#include "device_common.cuh"
#include "picoattn_internal.h"

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
__device__ __forceinline__ bool pos_ok(const DecodeArgs& a, int pos) {
    return pos >= 0 && pos < a.max_seq && pos < a.max_ctx;
}

// ---------------------------------------------------------------------------
// prep: norm + RoPE + fp16 append, one warp per head vector
// ---------------------------------------------------------------------------

// Per-head RMSNorm in the reference's order (cpp/tensor.hpp:146-176): element
// i is squared into lane i%4 of a 4-wide accumulator, lanes folded as
// (l0+l2)+(l1+l3), scale = 1/sqrt(ss/n + eps), out = (x*scale)*w.  Explicit
// _rn intrinsics keep every operation a single IEEE rounding (no FMA fusion).
template <int HD>
__device__ __forceinline__ void rmsnorm_ref(float* x, const float* w, float eps, int lane) {
    float part = 0.f;
    if (lane < 4) {
#pragma unroll 8
        for (int i = lane; i < HD; i += 4) part = __fadd_rn(part, __fmul_rn(x[i], x[i]));
    }
    const float l0 = __shfl_sync(0xffffffffu, part, 0);
    const float l1 = __shfl_sync(0xffffffffu, part, 1);
    const float l2 = __shfl_sync(0xffffffffu, part, 2);
    const float l3 = __shfl_sync(0xffffffffu, part, 3);
    const float ss = __fadd_rn(__fadd_rn(l0, l2), __fadd_rn(l1, l3));
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)HD), eps)));
    for (int i = lane; i < HD; i += 32) x[i] = __fmul_rn(__fmul_rn(x[i], scale), w[i]);
    __syncwarp();
}

// RoPE of one head (cpp/tensor.hpp:201-283 NeoX; picolm/tensor.c:247-293
// interleaved): (x0, x1) -> (x0*c - x1*s, x0*s + x1*c), each product and the
// sum rounded separately as in the reference's scalar/SSE code.
template <int HD>
__device__ __forceinline__ void rope_ref(float* x, const float* c, const float* s, int mode, int lane) {
    constexpr int half = HD / 2;
    for (int i = lane; i < half; i += 32) {
        const int i0 = mode == PICOATTN_ROPE_NEOX ? i : 2 * i;
        const int i1 = mode == PICOATTN_ROPE_NEOX ? i + half : 2 * i + 1;
        const float x0 = x[i0], x1 = x[i1], ci = c[i], si = s[i];
        x[i0] = __fsub_rn(__fmul_rn(x0, ci), __fmul_rn(x1, si));
        x[i1] = __fadd_rn(__fmul_rn(x0, si), __fmul_rn(x1, ci));
    }
    __syncwarp();
}

template <int HD>
__global__ void __launch_bounds__(128) decode_prep_kernel(DecodeArgs a) {
    __shared__ float buf[4][HD];
    const int b = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos = seq_pos(a, b);
    if (!pos_ok(a, pos)) {
        if (threadIdx.x == 0) atomicOr(a.status, PICOATTN_DEV_BAD_POS);
        return;
    }
    const size_t row = ((size_t)a.layer * a.max_seq + pos) * a.kvd;
    uint16_t* krow = seq_kcache(a, b) + row;
    uint16_t* vrow = seq_vcache(a, b) + row;
    const float* crow = a.rope_cos + (size_t)pos * (HD / 2);
    const float* srow = a.rope_sin + (size_t)pos * (HD / 2);
    float* x = buf[warp];
    const int n_slots = a.hq + 2 * a.hkv;
    for (int slot = warp; slot < n_slots; slot += 4) {
        int kind, h;  // 0 = q head, 1 = k head, 2 = v head
        const float* src;
        if (slot < a.hq) {
            kind = 0, h = slot, src = a.q + ((size_t)b * a.hq + h) * HD;
        } else if (slot < a.hq + a.hkv) {
            kind = 1, h = slot - a.hq, src = a.k + ((size_t)b * a.hkv + h) * HD;
        } else {
            kind = 2, h = slot - a.hq - a.hkv, src = a.v + ((size_t)b * a.hkv + h) * HD;
        }
        for (int i = lane; i < HD; i += 32) x[i] = src[i];
        __syncwarp();
        if (kind != 2) {
            const float* w = kind == 0 ? a.qn_w : a.kn_w;
            if (w) rmsnorm_ref<HD>(x, w, a.eps, lane);
            rope_ref<HD>(x, crow, srow, a.rope_mode, lane);
        }
        if (kind == 0) {
            float* dst = a.q_rot + ((size_t)b * a.hq + h) * HD;
            for (int i = lane; i < HD; i += 32) dst[i] = x[i];
        } else {
            uint16_t* dst = (kind == 1 ? krow : vrow) + (size_t)h * HD;
            for (int i = lane; i < HD; i += 32) dst[i] = f32_to_f16_ref(x[i]);
        }
        __syncwarp();
    }
}

// ---------------------------------------------------------------------------
// attn: split-KV GQA attention over one chunk of cache rows
// ---------------------------------------------------------------------------

template <int HD>
__global__ void __launch_bounds__(288, 1) decode_attn_kernel(DecodeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int chunk = blockIdx.x, b = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NW = a.compute_warps, W = a.warps_per_head, T = a.tile_rows;

    const int pos = seq_pos(a, b);
    if (!pos_ok(a, pos)) return;  // flagged by prep
    const int len = pos + 1;
    const int r0 = chunk * a.chunk_rows;
    if (r0 >= len) return;
    const int r1 = min(r0 + a.chunk_rows, len);
    const int n_tiles = (r1 - r0 + T - 1) / T;

    const size_t slab = (size_t)a.layer * a.max_seq * a.kvd;
    const uint16_t* kslab = seq_kcache(a, b) + slab;
    const uint16_t* vslab = seq_vcache(a, b) + slab;
    if (((uintptr_t)kslab | (uintptr_t)vslab) & 15u) {
        if (threadIdx.x == 0) atomicOr(a.status, PICOATTN_DEV_MISALIGNED);
        return;
    }

    const uint32_t row_bytes = (uint32_t)a.kvd * 2u;
    const uint32_t stride = row_bytes + 16u;  // padded rows: ldmatrix is conflict-free
    const uint32_t tile_bytes = (uint32_t)T * stride;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + a.stages;
    uint8_t* tiles = smem + 128;

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
        for (int t = 0; t < n_tiles; t++) {
            const int s = t % a.stages;
            const int use = t / a.stages;
            if (use > 0 && !mbar_wait(&empty[s], (uint32_t)((use - 1) & 1), a.status)) break;
            const int row0 = r0 + t * T;
            const int valid = min(T, r1 - row0);
            if (lane == 0) mbar_arrive_expect_tx(&full[s], 2u * (uint32_t)T * row_bytes);
            __syncwarp();
            uint8_t* kdst = tiles + (size_t)s * 2u * tile_bytes;
            // Rows past the end of the chunk repeat its last row: finite data
            // whose scores are masked, so no stale shared memory is ever used.
            for (int i = lane; i < 2 * T; i += 32) {
                const int kv = i >= T, r = kv ? i - T : i;
                const int src_row = row0 + min(r, valid - 1);
                const uint16_t* src = (kv ? vslab : kslab) + (size_t)src_row * a.kvd;
                bulk_g2s(kdst + kv * tile_bytes + (uint32_t)r * stride, src, row_bytes, &full[s]);
            }
        }
        return;
    }

    // ---------------- compute warps ----------------------------------------
    const int kvh = warp / W, wi = warp % W;
    const int gid = lane >> 2, tig = lane & 3;
    const int G = a.g;

    // q of the G heads of this KV head as the A operand (rows = heads, padded
    // to 16 with zeros), pre-scaled by log2(e)/sqrt(hd) so scores come out in
    // log2 units (the reference divides by sqrtf(hd) and uses expf).
    uint32_t qa[HD / 16][4];
    {
        const float qscale = 1.4426950408889634f / sqrtf((float)HD);
        const float* qb = a.q_rot + ((size_t)b * a.hq + (size_t)kvh * G) * HD;
#pragma unroll
        for (int kk = 0; kk < HD / 16; kk++) {
            const int c0 = kk * 16 + 2 * tig, c1 = c0 + 8;
            float v[8];
            const bool ra = gid < G, rb = gid + 8 < G;
            v[0] = ra ? qb[gid * HD + c0] : 0.f;
            v[1] = ra ? qb[gid * HD + c0 + 1] : 0.f;
            v[2] = rb ? qb[(gid + 8) * HD + c0] : 0.f;
            v[3] = rb ? qb[(gid + 8) * HD + c0 + 1] : 0.f;
            v[4] = ra ? qb[gid * HD + c1] : 0.f;
            v[5] = ra ? qb[gid * HD + c1 + 1] : 0.f;
            v[6] = rb ? qb[(gid + 8) * HD + c1] : 0.f;
            v[7] = rb ? qb[(gid + 8) * HD + c1 + 1] : 0.f;
            qa[kk][0] = pack_half2(v[0] * qscale, v[1] * qscale);
            qa[kk][1] = pack_half2(v[2] * qscale, v[3] * qscale);
            qa[kk][2] = pack_half2(v[4] * qscale, v[5] * qscale);
            qa[kk][3] = pack_half2(v[6] * qscale, v[7] * qscale);
        }
    }

    float m[2] = {-1e30f, -1e30f}, l[2] = {0.f, 0.f};
    float o[HD / 8][4];
#pragma unroll
    for (int i = 0; i < HD / 8; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

    // per-lane ldmatrix offsets inside a 16-row group of this head's columns
    const uint32_t k_lane = (uint32_t)((lane & 7) + ((lane >> 4) << 3)) * stride + (uint32_t)(((lane >> 3) & 1) * 16);
    const uint32_t v_lane = (uint32_t)((lane & 7) + (((lane >> 3) & 1) << 3)) * stride + (uint32_t)((lane >> 4) * 16);
    const uint32_t head_off = (uint32_t)kvh * HD * 2u;
    const uint32_t tiles_u32 = smem_u32(tiles);

    for (int t = 0; t < n_tiles; t++) {
        const int s = t % a.stages;
        mbar_wait(&full[s], (uint32_t)((t / a.stages) & 1), a.status);
        const int valid = min(T, r1 - (r0 + t * T));
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

    // partial (max, sum, acc) of this warp's rows
    l[0] += __shfl_xor_sync(0xffffffffu, l[0], 1);
    l[0] += __shfl_xor_sync(0xffffffffu, l[0], 2);
    l[1] += __shfl_xor_sync(0xffffffffu, l[1], 1);
    l[1] += __shfl_xor_sync(0xffffffffu, l[1], 2);
    const int part = chunk * W + wi;
    const size_t pbase = ((size_t)b * a.max_parts + part) * a.hq;
#pragma unroll
    for (int half = 0; half < 2; half++) {
        const int r = gid + 8 * half;
        if (r < G) {
            const int h = kvh * G + r;
            float* od = a.part_o + (pbase + h) * HD + 2 * tig;
#pragma unroll
            for (int i = 0; i < HD / 8; i++)
                *reinterpret_cast<float2*>(od + i * 8) = make_float2(o[i][2 * half], o[i][2 * half + 1]);
            if (tig == 0) *reinterpret_cast<float2*>(a.part_ml + (pbase + h) * 2) = make_float2(m[half], l[half]);
        }
    }
}

// ---------------------------------------------------------------------------
// merge: out = sum_p 2^(m_p - M) acc_p / sum_p 2^(m_p - M) l_p
// ---------------------------------------------------------------------------

template <int HD>
__global__ void __launch_bounds__(HD) decode_merge_kernel(DecodeArgs a) {
    const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
    float* dst = a.out + ((size_t)b * a.hq + h) * HD + d;
    const int pos = seq_pos(a, b);
    if (!pos_ok(a, pos)) {
        *dst = __int_as_float(0x7fc00000);
        return;
    }
    const int n_parts = ((pos + a.chunk_rows) / a.chunk_rows) * a.warps_per_head;
    const float* ml = a.part_ml + (size_t)b * a.max_parts * a.hq * 2;
    const float* po = a.part_o + (size_t)b * a.max_parts * a.hq * HD;
    float M = -INFINITY;
    for (int p = 0; p < n_parts; p++) M = fmaxf(M, ml[((size_t)p * a.hq + h) * 2]);
    float L = 0.f, acc = 0.f;
    for (int p = 0; p < n_parts; p++) {
        const float2 v = *reinterpret_cast<const float2*>(ml + ((size_t)p * a.hq + h) * 2);
        const float w = ex2(v.x - M);
        L += w * v.y;
        acc += w * po[((size_t)p * a.hq + h) * HD + d];
    }
    *dst = acc / L;
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
    if (stages & PICOATTN_STAGE_PREPARE) decode_prep_kernel<HD><<<a.n_seqs, 128, 0, stream>>>(a);
    if (stages & PICOATTN_STAGE_ATTEND) {
        dim3 grid((unsigned)plan.max_chunks, (unsigned)a.n_seqs);
        decode_attn_kernel<HD><<<grid, (plan.compute_warps + 1) * 32, plan.smem_bytes, stream>>>(a);
    }
    if (stages & PICOATTN_STAGE_COMBINE)
        decode_merge_kernel<HD><<<dim3((unsigned)a.hq, (unsigned)a.n_seqs), HD, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace

namespace {
constexpr long kTargetCtas = 148L * 8;
int decode_parts_capacity(int n_seqs, int warps_per_head) {
    const long per_seq = n_seqs >= kTargetCtas ? 1 : kTargetCtas / n_seqs;
    return (int)per_seq * warps_per_head;
}
}  // namespace

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
    // Chunks grow until the grid holds at most kTargetCtas CTAs (or one chunk
    // per sequence), so n_seqs * max_chunks <= max(n_seqs, kTargetCtas) for any
    // max_ctx and the partial buffers below have a size independent of it.
    p.chunk_rows = p.tile_rows;
    for (;;) {
        const long chunks = (max_ctx + p.chunk_rows - 1) / p.chunk_rows;
        if (chunks <= 1 || (long)n_seqs * chunks <= kTargetCtas) break;
        if (p.chunk_rows >= max_ctx) break;  // unreachable (chunks would be 1); keeps the doubling bounded
        p.chunk_rows *= 2;
    }
    p.max_chunks = (max_ctx + p.chunk_rows - 1) / p.chunk_rows;
    p.max_parts = decode_parts_capacity(n_seqs, p.warps_per_head);
    const size_t max_parts = (size_t)p.max_parts;
    size_t off = kWsHeaderBytes;
    p.ws_qrot = off;
    off = align_up(off + (size_t)n_seqs * hq * hd * 4, 256);
    p.ws_ml = off;
    off = align_up(off + (size_t)n_seqs * max_parts * hq * 2 * 4, 256);
    p.ws_o = off;
    off = align_up(off + (size_t)n_seqs * max_parts * hq * hd * 4, 256);
    p.ws_total = off;
    *plan = p;
    return true;
}

cudaError_t launch_decode(const DecodeArgs& a, const DecodePlan& plan, cudaStream_t stream, unsigned stages) {
    return a.hd == 64 ? launch_decode_hd<64>(a, plan, stream, stages) : launch_decode_hd<128>(a, plan, stream, stages);
}

}  // namespace picoattn
