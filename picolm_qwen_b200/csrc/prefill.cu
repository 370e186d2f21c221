// prefill.cu -- prompt (prefill) attention step for sm_100a.
//
// Replaces the per-token attention block of Model::forward_batch,
// cpp/model.hpp:507-593: token i of the prompt runs the decode step at
// pos = start_pos + i, so it attends causally over cache rows 0..pos.
//
// Two kernels:
//   prefill_prep   one CTA per token: QK-RMSNorm + RoPE in the reference's exact
//                  fp32 order, k/v rows rounded to fp16 with the reference's
//                  rounding into the cache, q pre-scaled by log2(e)/sqrt(hd)
//                  and stored as fp16 [n_tok][n_heads][hd] in the workspace.
//   prefill_attn   causal flash attention on the 5th-generation tensor cores.
//                  One CTA per (128-token q tile, q head); warp roles:
//                    warps 0-3  softmax: thread r owns q row r = TMEM lane r
//                    warp 4     TMA producer (Q once, K/V 128-row tiles)
//                    warp 5     MMA issuer and TMEM owner
//                  S = Q K^T goes to TMEM (two 128-column buffers so QK of
//                  tile j+1 overlaps the softmax of tile j); P (fp16) is written
//                  back over its S columns and fed to O += P V straight from
//                  TMEM; O (128 columns fp32) lives in TMEM until the epilogue.
//                  Online softmax in the log2 domain with a lazy rescale: O is
//                  rescaled only when a row maximum grows by more than 8
//                  (p <= 2^8 stays exact in fp16), which keeps the O round trip
//                  off the common path.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <mutex>

#include <cuda.h>

#include "device_common.cuh"
#include "picoattn_internal.h"
#include "prep_common.cuh"
#include "tcgen05.cuh"

namespace picoattn {

namespace {

constexpr int BM = 128;  // q rows per tile
constexpr int BN = 128;  // keys per tile
constexpr float kRescaleThreshold = 8.0f;
// largest p = 2^(s - stale max) the single-pass softmax keeps: 2^15 < 65504
// stays finite and exact in fp16
constexpr float kStaleMaxP = 32768.0f;

// ---------------------------------------------------------------------------
// prep (head-vector helpers in prep_common.cuh)
// ---------------------------------------------------------------------------

// fp16 input bits -> the reference's fp16 rounding of their fp32 value: the
// identity on every fp16 value except NaN, whose payload becomes the quiet bit
// (f32_to_f16_ref of the widened value); two halves per word.
__device__ __forceinline__ uint32_t h2_ref16(uint32_t w) {
    uint32_t r = 0;
#pragma unroll
    for (int k = 0; k < 2; k++) {
        uint32_t h = (w >> (16 * k)) & 0xFFFFu;
        if ((h & 0x7C00u) == 0x7C00u && (h & 0x3FFu)) h = (h & 0x8000u) | 0x7E00u;
        r |= h << (16 * k);
    }
    return r;
}

// A unit = up to 8 head vectors of ONE kind (q, k or v) of one token, so the
// three paths never run predicated inside each other.  Each lane holds V =
// HD/32 elements of each vector, both members of its RoPE pairs (prep_idx), so
// RoPE needs no exchange between lanes.
//
// The grid is one wave of blocks that stays resident (8 warps each); warp w of
// W takes units w, w+W, w+2W, ...  Each warp stages its units' inputs in a ring
// of kPrepStages shared-memory slots by cp.async (16 bytes per lane, L2 only),
// so the next units' loads are in flight while it works on the current one:
// the kernel streams at the memory's rate instead of waiting once per unit.
// A slot holds the unit's 8 rows, each HD * element bytes plus 16 bytes of
// padding (the padding puts the rows of the 8 vectors on different banks).
//
// RMSNorm: the reference accumulates the squares of elements i = c, c+4, c+8, ...
// into lane c = i % 4 in index order (cpp/tensor.hpp:146-176).  Lane 4u+c runs
// chain c of vector u straight from the staged row (elements c + 4m, m in
// order), all 32 lanes busy for 8 vectors; lane u then folds vector u's chains
// as (c0+c2)+(c1+c3) and computes its scale, as in vec_rmsnorm.
constexpr int kPrepUnit = 8;    // head vectors per unit
constexpr int kPrepStages = 2;  // staged units per warp
constexpr int kPrepWarps = 8;   // warps per block

__host__ __device__ constexpr int prep_row_bytes(int hd, int esize) { return hd * esize + 16; }
__host__ __device__ constexpr int prep_slot_bytes(int hd, int esize) {
    return kPrepUnit * prep_row_bytes(hd, esize);
}
__host__ __device__ constexpr int prep_smem_bytes(int hd, int esize) {
    return kPrepWarps * kPrepStages * prep_slot_bytes(hd, esize);
}

// Units are numbered kind-major: every token's q groups first (token-major),
// then every token's k groups, then the v groups, so the warps of an SM mostly
// run the same one of the three code paths at a time.
struct PrepUnit {
    int tok, kind, h0, nh;
};

__device__ __forceinline__ PrepUnit prep_unit(const PrefillArgs& a, int unit, int qg, int kg) {
    PrepUnit p;
    const int nq = a.n_tok * qg, nk = a.n_tok * kg;
    int g;
    if (unit < nq) {
        p.kind = 0, p.tok = unit / qg, g = unit - p.tok * qg;
    } else if (unit < nq + nk) {
        unit -= nq;
        p.kind = 1, p.tok = unit / kg, g = unit - p.tok * kg;
    } else {
        unit -= nq + nk;
        p.kind = 2, p.tok = unit / kg, g = unit - p.tok * kg;
    }
    p.h0 = g * kPrepUnit;
    p.nh = min(kPrepUnit, (p.kind == 0 ? a.hq : a.hkv) - p.h0);
    return p;
}

// This lane's share of the copy of one unit's rows into `slot`: 16-byte pieces,
// lane-strided, then one commit (an empty group when the unit does not exist,
// so every lane has committed the same number of groups).
template <int HD, int ES>
__device__ __forceinline__ void prep_stage(const PrefillArgs& a, int unit, int n_units, int qg, int kg,
                                           uint8_t* slot, int lane) {
    if (unit < n_units) {
        const PrepUnit p = prep_unit(a, unit, qg, kg);
        const void* base = p.kind == 0 ? a.q : (p.kind == 1 ? a.k : a.v);
        const int nheads = p.kind == 0 ? a.hq : a.hkv;
        const uint8_t* src = reinterpret_cast<const uint8_t*>(base) + ((size_t)p.tok * nheads + p.h0) * HD * ES;
        constexpr int PR = HD * ES / 16;  // 16-byte pieces per row (a power of two, 8..32)
#pragma unroll
        for (int it = 0; it < kPrepUnit * PR / 32; it++) {
            const int i = lane + 32 * it, u = i / PR, pc = i % PR;
            if (u < p.nh) cp_async16(slot + u * prep_row_bytes(HD, ES) + 16 * pc, src + (size_t)u * HD * ES + 16 * pc);
        }
    }
    cp_async_commit();
}

// Element e of a staged row as fp32 (fp16 rows widened exactly); elements e, e+1.
template <int ES>
__device__ __forceinline__ float prep_elem(const uint8_t* row, int e) {
    if constexpr (ES == 2) return __half2float(reinterpret_cast<const __half*>(row)[e]);
    else return reinterpret_cast<const float*>(row)[e];
}
template <int ES>
__device__ __forceinline__ float2 prep_elem2(const uint8_t* row, int e) {
    if constexpr (ES == 2) return __half22float2(*reinterpret_cast<const __half2*>(row + 2 * e));
    else return *reinterpret_cast<const float2*>(row + 4 * e);
}

// The elements of a head vector lane l holds, x[0..V-1], chosen so that both
// of its RoPE pairs stay inside the lane:
//   HD 128: 2l, 2l+1, 64+2l, 65+2l  (NeoX pairs (2l, 64+2l), (2l+1, 65+2l);
//           interleaved pairs (2l, 2l+1), (64+2l, 65+2l))
//   HD 64:  NeoX l, 32+l; interleaved 2l, 2l+1 (one pair)
template <int HD>
__device__ __forceinline__ int prep_idx(int lane, int j, bool neox) {
    if constexpr (HD == 128) return (j < 2 ? 2 * lane : 64 + 2 * lane) + (j & 1);
    else return neox ? lane + 32 * j : 2 * lane + j;
}

template <int HD, int ES>
__device__ __forceinline__ void prep_load(float (&x)[HD / 32], const uint8_t* row, int lane, bool neox) {
    if constexpr (HD == 128) {
        const float2 a = prep_elem2<ES>(row, 2 * lane), b = prep_elem2<ES>(row, 64 + 2 * lane);
        x[0] = a.x, x[1] = a.y, x[2] = b.x, x[3] = b.y;
    } else if (neox) {
        x[0] = prep_elem<ES>(row, lane), x[1] = prep_elem<ES>(row, 32 + lane);
    } else {
        const float2 a = prep_elem2<ES>(row, 2 * lane);
        x[0] = a.x, x[1] = a.y;
    }
}

// 16-bit results h[j] of x[j] to dst at this lane's element positions
template <int HD>
__device__ __forceinline__ void prep_store16(uint16_t* dst, const uint32_t (&hp)[HD / 64], int lane, bool neox) {
    if constexpr (HD == 128) {
        *reinterpret_cast<uint32_t*>(dst + 2 * lane) = hp[0];
        *reinterpret_cast<uint32_t*>(dst + 64 + 2 * lane) = hp[1];
    } else if (neox) {
        dst[lane] = (uint16_t)(hp[0] & 0xFFFFu);
        dst[32 + lane] = (uint16_t)(hp[0] >> 16);
    } else {
        *reinterpret_cast<uint32_t*>(dst + 2 * lane) = hp[0];
    }
}

// RoPE of one pair (products and sums rounded separately, as vec_rope):
// (x0, x1) -> (x0*c - x1*s, x0*s + x1*c).  Scalar intrinsics: a packed
// multiply followed by a packed subtract may be contracted into one fused
// multiply-add, which rounds differently from the reference.
__device__ __forceinline__ void prep_rot(float& x0, float& x1, float c, float s) {
    const float a = x0, b = x1;
    x0 = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    x1 = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
}

// RoPE of this lane's pairs.
template <int HD>
__device__ __forceinline__ void prep_rope(float (&x)[HD / 32], const float* crow, const float* srow, int lane,
                                          bool neox) {
    if constexpr (HD == 128) {
        if (neox) {  // table rows 2l, 2l+1; pairs (x0, x2), (x1, x3) (4-byte loads: the
                     // caller's table need only be 4-byte aligned)
            prep_rot(x[0], x[2], crow[2 * lane], srow[2 * lane]);
            prep_rot(x[1], x[3], crow[2 * lane + 1], srow[2 * lane + 1]);
        } else {     // table rows l, 32+l; pairs (x0, x1), (x2, x3)
            prep_rot(x[0], x[1], crow[lane], srow[lane]);
            prep_rot(x[2], x[3], crow[32 + lane], srow[32 + lane]);
        }
    } else {
        prep_rot(x[0], x[1], crow[lane], srow[lane]);
    }
}

// fp16 input bits -> the reference's fp16 rounding of their fp32 value (the
// identity except on NaN, h2_ref16): a half is NaN when its magnitude plus
// 0x3FF carries into bit 15, so one add tests both halves of a word.
__device__ __forceinline__ uint32_t h2_ref16_fast(uint32_t w) {
    return (((w & 0x7FFF7FFFu) + 0x03FF03FFu) & 0x80008000u) ? h2_ref16(w) : w;
}

// One unit whose rows are staged in `slot`.  Every row of the slot is read and
// processed whether or not the unit has that head (rows past nh hold stale
// data, and their results are never stored), so the arithmetic runs without
// per-head branches.
template <int HD, int ES>
__device__ __forceinline__ void prep_unit_run(const PrefillArgs& a, const PrepUnit& p, const uint8_t* slot, int lane) {
    constexpr int V = HD / 32;
    constexpr int U = kPrepUnit;
    constexpr int RB = prep_row_bytes(HD, ES);
    const int nh = p.nh;
    const int pos = a.start + p.tok;
    const size_t crow = ((size_t)a.layer * a.max_seq + pos) * a.kvd;
    const bool neox = a.rope_mode == PICOATTN_ROPE_NEOX;

    if (p.kind == 2) {  // v: stored as the reference's fp16 of the input
        uint16_t* dst = a.v_cache + crow + (size_t)p.h0 * HD;
#pragma unroll
        for (int u = 0; u < U; u++) {
            if constexpr (ES == 2) {  // the bits themselves, NaN payloads aside
                if constexpr (V == 4) {
                    uint2 w = *reinterpret_cast<const uint2*>(slot + u * RB + 8 * lane);
                    w.x = h2_ref16_fast(w.x), w.y = h2_ref16_fast(w.y);
                    if (u < nh) *reinterpret_cast<uint2*>(dst + u * HD + V * lane) = w;
                } else {
                    const uint32_t w = h2_ref16_fast(*reinterpret_cast<const uint32_t*>(slot + u * RB + 4 * lane));
                    if (u < nh) *reinterpret_cast<uint32_t*>(dst + u * HD + V * lane) = w;
                }
            } else {
                float x[V];
                prep_load<HD, ES>(x, slot + u * RB, lane, neox);
                uint32_t hp[V / 2];
#pragma unroll
                for (int j = 0; j < V / 2; j++) hp[j] = f32x2_to_f16_ref(x[2 * j], x[2 * j + 1]);
                if (u < nh) prep_store16<HD>(dst + u * HD, hp, lane, neox);
            }
        }
        return;
    }

    float x[U][V];
#pragma unroll
    for (int u = 0; u < U; u++) prep_load<HD, ES>(x[u], slot + u * RB, lane, neox);
    if (a.qn_w) {
        const float* wsrc = p.kind == 0 ? a.qn_w : a.kn_w;
        float w[V];
#pragma unroll
        for (int j = 0; j < V; j++) w[j] = wsrc[prep_idx<HD>(lane, j, neox)];
        // chain c = lane & 3 of vector lane >> 2: elements c, c+4, ..., in order
        constexpr int CH = HD / 4;
        float part = 0.f;
        const uint8_t* row = slot + (lane >> 2) * RB;
        const int c = lane & 3;
#pragma unroll
        for (int m = 0; m < CH; m++) {
            const float e = prep_elem<ES>(row, c + 4 * m);
            // the square of a widened fp16 value is exact in fp32 (at most 22
            // significant bits, no underflow), so one fused multiply-add rounds
            // exactly as the reference's rounded square plus rounded sum
            if constexpr (ES == 2) part = __fmaf_rn(e, e, part);
            else part = __fadd_rn(part, __fmul_rn(e, e));
        }
        const int s4 = (lane & 7) * 4;
        const float c0 = __shfl_sync(0xffffffffu, part, s4 + 0), c1 = __shfl_sync(0xffffffffu, part, s4 + 1);
        const float c2 = __shfl_sync(0xffffffffu, part, s4 + 2), c3 = __shfl_sync(0xffffffffu, part, s4 + 3);
        const float ss = __fadd_rn(__fadd_rn(c0, c2), __fadd_rn(c1, c3));
        // ss / HD: HD is a power of two, so the product with 1/HD is the same
        // correctly rounded quotient
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(ss, 1.0f / (float)HD), a.eps)));
        // (x * scale) * w, two roundings, as vec_rmsnorm
#pragma unroll
        for (int u = 0; u < U; u++) {
            const float su = __shfl_sync(0xffffffffu, scale, u);
            const uint64_t s2 = f2_pack(su, su);
#pragma unroll
            for (int j = 0; j < V; j += 2)
                f2_unpack(f2_mul(f2_mul(f2_pack(x[u][j], x[u][j + 1]), s2), f2_pack(w[j], w[j + 1])), x[u][j],
                          x[u][j + 1]);
        }
    }
    const float* rc = a.rope_cos + (size_t)pos * (HD / 2);
    const float* rs = a.rope_sin + (size_t)pos * (HD / 2);
    if (p.kind == 0) {
        const float qscale = 1.4426950408889634f / sqrtf((float)HD);
        const uint64_t qs2 = f2_pack(qscale, qscale);
        uint16_t* dst = reinterpret_cast<uint16_t*>(a.q16 + ((size_t)p.tok * a.hq + p.h0) * HD);
#pragma unroll
        for (int u = 0; u < U; u++) {
            prep_rope<HD>(x[u], rc, rs, lane, neox);
            uint32_t hp[V / 2];
#pragma unroll
            for (int j = 0; j < V / 2; j++) {
                float lo, hi;
                f2_unpack(f2_mul(f2_pack(x[u][2 * j], x[u][2 * j + 1]), qs2), lo, hi);
                hp[j] = pack_half2(lo, hi);
            }
            if (u < nh) prep_store16<HD>(dst + u * HD, hp, lane, neox);
        }
    } else {
        uint16_t* dst = a.k_cache + crow + (size_t)p.h0 * HD;
#pragma unroll
        for (int u = 0; u < U; u++) {
            prep_rope<HD>(x[u], rc, rs, lane, neox);
            uint32_t hp[V / 2];
#pragma unroll
            for (int j = 0; j < V / 2; j++) hp[j] = f32x2_to_f16_ref(x[u][2 * j], x[u][2 * j + 1]);
            if (u < nh) prep_store16<HD>(dst + u * HD, hp, lane, neox);
        }
    }
}

// Launched with programmatic stream serialisation after the previous layer's
// attention kernel: it waits for that kernel (which still reads the q operand
// and may still write the output) before it reads or writes anything, and lets
// the attention kernel after it launch only once its own stores are done, so
// that kernel's early CTAs do not take SMs the rest of this grid needs.
template <int HD, int ES>
__global__ void __launch_bounds__(kPrepWarps * 32) prefill_prep_kernel(PrefillArgs a) {
    extern __shared__ __align__(16) uint8_t prep_smem[];
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (blockIdx.x == 0 && threadIdx.x == 0) *a.work_counter = 0;  // attention work queue
    const int qg = (a.hq + kPrepUnit - 1) / kPrepUnit, kg = (a.hkv + kPrepUnit - 1) / kPrepUnit;
    const int n_units = a.n_tok * (qg + 2 * kg);
    const int W = gridDim.x * kPrepWarps;
    const int first = blockIdx.x * kPrepWarps + warp;
    uint8_t* ring = prep_smem + (size_t)warp * kPrepStages * prep_slot_bytes(HD, ES);
#pragma unroll
    for (int s = 0; s < kPrepStages; s++)
        prep_stage<HD, ES>(a, first + s * W, n_units, qg, kg, ring + s * prep_slot_bytes(HD, ES), lane);
    for (int k = 0, unit = first; unit < n_units; k++, unit += W) {
        uint8_t* slot = ring + (k % kPrepStages) * prep_slot_bytes(HD, ES);
        cp_async_wait<kPrepStages - 1>();  // this lane's pieces of the unit have landed
        __syncwarp();                      // and every other lane's
        prep_unit_run<HD, ES>(a, prep_unit(a, unit, qg, kg), slot, lane);
        __syncwarp();  // every lane has read the slot before it is refilled
        prep_stage<HD, ES>(a, unit + kPrepStages * W, n_units, qg, kg, slot, lane);
    }
    cp_async_wait<0>();
    pdl_trigger();
}

// ---------------------------------------------------------------------------
// attention (tcgen05 / TMEM)
// ---------------------------------------------------------------------------

// Writes a 32 x 32 block of a head's output, rows y..y+31 (lane i holds row y+i:
// the TMEM lane layout) and columns x..x+31, scaled by `inv`.  Stored from that
// layout, each lane's row sits hq*hd*4 bytes from its neighbour's and every warp
// store touches 32 lines; the SM's store path then limits the epilogue.  Instead
// the block goes into a 4 KB shared stage in the 128-byte-swizzled layout (16-byte
// unit g of row r at unit g ^ (r & 7): conflict-free for these row-wise writes)
// and leaves as one tiled TMA store; rows past the map's extent are not written.
// The stage is reused once the previous store has read it.  A block whose rows
// all lie past the map (y >= rows) is not stored at all.
__device__ __forceinline__ void stage_store_32x32(const uint32_t (&o)[32], float inv, float* stage,
                                                  const CUtensorMap* map, int x, int y, int rows, int lane) {
    if (y >= rows) return;
    if (lane == 0) bulk_wait_read_all();
    __syncwarp();
#pragma unroll
    for (int g = 0; g < 8; g++) {
        const float4 val = make_float4(__uint_as_float(o[4 * g]) * inv, __uint_as_float(o[4 * g + 1]) * inv,
                                       __uint_as_float(o[4 * g + 2]) * inv, __uint_as_float(o[4 * g + 3]) * inv);
        *reinterpret_cast<float4*>(stage + lane * 32 + ((g ^ (lane & 7)) * 4)) = val;
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
        tma_store_2d(map, stage, x, y);
        bulk_commit_group();
    }
}

template <int HD>
struct AttnSmem {
    static constexpr int kBoxBytes = BM * 128;              // one 128-row x 64-column fp16 box
    static constexpr int kTileBytes = (HD / 64) * kBoxBytes;  // 128 rows x HD columns
    static constexpr int NK = 2, NV = 2;
    static constexpr int kQ = 0;
    static constexpr int kK = kQ + kTileBytes;
    static constexpr int kV = kK + NK * kTileBytes;
    static constexpr int kStage = kV + NV * kTileBytes;  // epilogue: 32 x 32 fp32 per softmax warp
    static constexpr int kBars = kStage + 4 * 4096;
    static constexpr int kEnd = kBars + 256;
    static constexpr int kDynBytes = kEnd + 1024;  // slack to align the base to 1024
};

template <int HD>
__global__ void __launch_bounds__(192, 1)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                        PrefillArgs a) {
    using L = AttnSmem<HD>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const int qt = a.n_qtiles - 1 - (int)blockIdx.x;  // longest rows of the causal triangle first
    const int h = blockIdx.y;
    const int kvh = h / a.g;
    const int q0 = qt * BM;
    const int q_last = min(q0 + BM, a.n_tok) - 1;  // last real token of the tile
    const int n_kv = (a.start + q_last) / BN + 1;

    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBars);
    uint64_t* q_full = bars + 0;
    uint64_t* k_full = bars + 1;
    uint64_t* k_empty = k_full + L::NK;
    uint64_t* v_full = k_empty + L::NK;
    uint64_t* v_empty = v_full + L::NV;
    uint64_t* s_full = v_empty + L::NV;  // [2]
    uint64_t* p_full = s_full + 2;       // [2]
    uint64_t* pv_done = p_full + 2;      // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pv_done + 2);

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < L::NK; s++) mbar_init(&k_full[s], 1), mbar_init(&k_empty[s], 1);
        for (int s = 0; s < L::NV; s++) mbar_init(&v_full[s], 1), mbar_init(&v_empty[s], 1);
        for (int b = 0; b < 2; b++) mbar_init(&s_full[b], 1), mbar_init(&p_full[b], 4), mbar_init(&pv_done[b], 1);
        fence_mbar_init();
    }
    if (warp == 5) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tS0 = tmem, tO = tmem + 256;

    const uint32_t sQ = smem_u32(smem + L::kQ);
    const uint32_t sK = smem_u32(smem + L::kK);
    const uint32_t sV = smem_u32(smem + L::kV);

    if (warp == 4) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmV);
            mbar_arrive_expect_tx(q_full, L::kTileBytes);
            for (int c = 0; c < HD / 64; c++)
                tma_load_2d(smem + L::kQ + c * L::kBoxBytes, &tmQ, h * HD + 64 * c, q0, q_full);
            for (int j = 0; j < n_kv; j++) {
                const int sk = j % L::NK, uk = j / L::NK;
                if (uk > 0) mbar_wait(&k_empty[sk], (uint32_t)((uk - 1) & 1), a.status);
                mbar_arrive_expect_tx(&k_full[sk], L::kTileBytes);
                for (int c = 0; c < HD / 64; c++)
                    tma_load_2d(smem + L::kK + sk * L::kTileBytes + c * L::kBoxBytes, &tmK, kvh * HD + 64 * c, j * BN,
                                &k_full[sk]);
                const int sv = j % L::NV, uv = j / L::NV;
                if (uv > 0) mbar_wait(&v_empty[sv], (uint32_t)((uv - 1) & 1), a.status);
                mbar_arrive_expect_tx(&v_full[sv], L::kTileBytes);
                for (int c = 0; c < HD / 64; c++)
                    tma_load_2d(smem + L::kV + sv * L::kTileBytes + c * L::kBoxBytes, &tmV, kvh * HD + 64 * c, j * BN,
                                &v_full[sv]);
            }
        }
        __syncwarp();
    } else if (warp == 5) {
        // ---------------- MMA issuer ----------------
        constexpr uint32_t idesc_qk = idesc_f16_f32(BM, BN, false, false);
        constexpr uint32_t idesc_pv = idesc_f16_f32(BM, HD, false, true);
        const uint64_t dq = smem_desc_sw128(sQ, 16, 1024);
        const uint64_t dk = smem_desc_sw128(sK, 16, 1024);
        // B = V tile, MN-major: 64-column boxes LBO apart, 8-key groups SBO apart
        const uint64_t dv = smem_desc_sw128(sV, L::kBoxBytes, 1024);
        auto issue_pv = [&](int i) {
            const int b = i & 1, sv = i % L::NV;
            mbar_wait(&p_full[b], (uint32_t)((i >> 1) & 1), a.status);
            mbar_wait(&v_full[sv], (uint32_t)((i / L::NV) & 1), a.status);
            tc_fence_after();
            if (lane == 0) {
                const uint64_t vd = desc_advance(dv, sv * L::kTileBytes);
#pragma unroll
                for (int kk = 0; kk < BN / 16; kk++)
                    umma_ts(tO, tS0 + b * 128 + kk * 8, desc_advance(vd, kk * 16 * 128), idesc_pv,
                            (i > 0 || kk > 0) ? 1u : 0u);
                umma_commit(&v_empty[sv]);
                umma_commit(&pv_done[b]);
            }
            __syncwarp();
        };
        mbar_wait(q_full, 0, a.status);
        for (int j = 0; j < n_kv; j++) {
            const int b = j & 1, sk = j % L::NK;
            mbar_wait(&k_full[sk], (uint32_t)((j / L::NK) & 1), a.status);
            if (j >= 2) mbar_wait(&pv_done[b], (uint32_t)(((j - 2) >> 1) & 1), a.status);
            tc_fence_after();
            if (lane == 0) {
                const uint64_t kd = desc_advance(dk, sk * L::kTileBytes);
#pragma unroll
                for (int kk = 0; kk < HD / 16; kk++) {
                    const uint32_t koff = (kk >> 2) * L::kBoxBytes + (kk & 3) * 32;
                    umma_ss(tS0 + b * 128, desc_advance(dq, koff), desc_advance(kd, koff), idesc_qk, kk > 0 ? 1u : 0u);
                }
                umma_commit(&s_full[b]);
                umma_commit(&k_empty[sk]);
            }
            __syncwarp();
            if (j >= 1) issue_pv(j - 1);
        }
        issue_pv(n_kv - 1);
    } else {
        // ---------------- softmax warpgroup ----------------
        const int r = threadIdx.x;  // q row within the tile == TMEM lane
        const int qpos = a.start + q0 + r;
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        float m_run = -INFINITY, l_run = 0.f;
        for (int j = 0; j < n_kv; j++) {
            const int b = j & 1;
            mbar_wait(&s_full[b], (uint32_t)((j >> 1) & 1), a.status);
            tc_fence_after();
            uint32_t sr[BN];
            // four loads in flight, one wait
            tmem_ld32(tS0 + b * 128 + 0 + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
            tmem_ld32(tS0 + b * 128 + 32 + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
            tmem_ld32(tS0 + b * 128 + 64 + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&sr[64]));
            tmem_ld32(tS0 + b * 128 + 96 + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&sr[96]));
            tmem_ld_wait();
            float* s = reinterpret_cast<float*>(sr);
            const int kbase = j * BN;
            if (kbase + BN - 1 > a.start + q0) {  // tile crosses the diagonal of this q tile
#pragma unroll
                for (int c = 0; c < BN; c++)
                    if (kbase + c > qpos) s[c] = -INFINITY;
            }
            // row max with 8 independent chains
            float mx8[8];
#pragma unroll
            for (int e = 0; e < 8; e++) mx8[e] = s[e];
#pragma unroll
            for (int c = 8; c < BN; c += 8)
#pragma unroll
                for (int e = 0; e < 8; e++) mx8[e] = fmaxf(mx8[e], s[c + e]);
            const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                                   fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
            if (j == 0) {
                m_run = mx;
            } else if (__any_sync(0xffffffffu, mx > m_run + kRescaleThreshold)) {
                const float m_new = fmaxf(m_run, mx);
                const float corr = ex2(m_run - m_new);
                // O holds the sum through tile j-1: wait for that PV, then scale it in place
                mbar_wait(&pv_done[(j - 1) & 1], (uint32_t)(((j - 1) >> 1) & 1), a.status);
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < HD / 32; c++) {
                    uint32_t t[32];
                    tmem_ld32(tO + c * 32 + lane_off, t);
                    tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 32; e++) t[e] = __float_as_uint(__uint_as_float(t[e]) * corr);
                    tmem_st32(tO + c * 32 + lane_off, t);
                }
                tmem_st_wait();
                l_run *= corr;
                m_run = m_new;
            }
            float ls8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int c = 0; c < BN / 64; c++) {
                uint32_t t[32];
#pragma unroll
                for (int e = 0; e < 32; e++) {
                    const float p0 = ex2(s[c * 64 + 2 * e] - m_run);
                    const float p1 = ex2(s[c * 64 + 2 * e + 1] - m_run);
                    ls8[e & 7] += p0 + p1;
                    t[e] = pack_half2(p0, p1);
                }
                tmem_st32(tS0 + b * 128 + c * 32 + lane_off, t);
            }
            l_run += ((ls8[0] + ls8[1]) + (ls8[2] + ls8[3])) + ((ls8[4] + ls8[5]) + (ls8[6] + ls8[7]));
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[b]);
        }
        // epilogue: O / l -> out[token][h][:]
        mbar_wait(&pv_done[(n_kv - 1) & 1], (uint32_t)(((n_kv - 1) >> 1) & 1), a.status);
        tc_fence_after();
        const float inv = 1.0f / l_run;
        const int row0 = q0 + warp * 32;
        float* stage = reinterpret_cast<float*>(smem + L::kStage + warp * 4096);
#pragma unroll 1
        for (int c = 0; c < HD / 32; c++) {
            uint32_t t[32];
            tmem_ld32(tO + c * 32 + lane_off, t);
            tmem_ld_wait();
            stage_store_32x32(t, inv, stage, &tmO, h * HD + c * 32, row0, a.n_tok, lane);
        }
        if (lane == 0) bulk_wait_all();
        tc_fence_before();
    }
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ---------------------------------------------------------------------------
// attention, head-pair persistent variant (even GQA group size)
// ---------------------------------------------------------------------------
//
// Work item = (128-token q tile, two q heads h0, h0+1 of the same KV group);
// items are handed out longest-first by an atomic counter, so a persistent
// grid of one CTA per SM balances the causal triangle.  Both heads read the
// same K/V tiles: one TMA stream feeds two softmax warpgroups, each with its own
// S (128 TMEM columns, P written back over it) and O (128 columns):
//   TMEM  [0,128) S0   [128,256) S1   [256,384) O0   [384,512) O1
// Warps 0-3 / 4-7 softmax for head 0 / 1 (thread = q row = TMEM lane), warp 8
// TMA and work-queue fetch, warp 9 MMA issue.  Per KV tile t the MMA warp issues
// PV0(t), QK0(t+1), PV1(t), QK1(t+1), so each warpgroup's softmax overlaps the
// other head's tensor work.

// One KV tile of the online softmax for the q row of this thread (TMEM lane):
// reads S (128 fp32 columns at tS), writes P (fp16, over the first 64 columns
// of S), updates the running max m_run and sum l_run, and rescales O (at tO)
// when a row max grows past the stale-max margin.  wait_prev_pv() must return
// once the PV of the previous tile has completed (called only before O is
// rescaled).  Returns with the P stores complete (tcgen05.wait::st).
template <int HD, class WaitPrevPV>
__device__ __forceinline__ void softmax_tile(uint32_t tS, uint32_t tO, uint32_t lane_off, int j, int kbase, int qpos,
                                             bool diag, float& m_run, float& l_run, WaitPrevPV wait_prev_pv) {
    // Optimistic single pass: p = 2^(s - m_run) with the running max, kept
    // in registers.  p <= 2^15 is exact in fp16 and safe in the fp32 sums,
    // so unless some p of the tile exceeds 2^15 (a row max above m_run + 15;
    // checked on the packed fp16 values) P is stored as is.  On the first
    // tile of an item the running max starts as the max of the first 32
    // columns (column 0 is visible to every row).
    bool done = false;
    {
        uint32_t pk[BN / 2];
        uint64_t ls2[4] = {0ull, 0ull, 0ull, 0ull};  // packed (even, odd) column sums
        __half2 hm[4] = {__float2half2_rn(0.f), __float2half2_rn(0.f), __float2half2_rn(0.f),
                         __float2half2_rn(0.f)};
        uint32_t sbuf[2][32];
        tmem_ld32(tS + lane_off, sbuf[0]);
        if (j == 0) {
            tmem_ld_wait();
            float m0 = -INFINITY;
#pragma unroll
            for (int e = 0; e < 32; e++)
                if (!diag || kbase + e <= qpos) m0 = fmaxf(m0, __uint_as_float(sbuf[0][e]));
            m_run = m0;
        }
        const uint64_t mm2 = f2_pack(m_run, m_run);
#pragma unroll
        for (int c = 0; c < BN / 32; c++) {
            tmem_ld_wait();
            uint32_t (&sr)[32] = sbuf[c & 1];
            if (c + 1 < BN / 32) tmem_ld32(tS + (c + 1) * 32 + lane_off, sbuf[(c + 1) & 1]);
#pragma unroll
            for (int e = 0; e < 16; e++) {
                float s0 = __uint_as_float(sr[2 * e]), s1 = __uint_as_float(sr[2 * e + 1]);
                if (diag) {
                    if (kbase + c * 32 + 2 * e > qpos) s0 = -INFINITY;
                    if (kbase + c * 32 + 2 * e + 1 > qpos) s1 = -INFINITY;
                }
                float d0, d1;
                f2_unpack(f2_sub(f2_pack(s0, s1), mm2), d0, d1);
                const float p0 = ex2(d0), p1 = ex2(d1);
                ls2[e & 3] = f2_add(ls2[e & 3], f2_pack(p0, p1));
                const __half2 h = __floats2half2_rn(p0, p1);
                hm[e & 3] = __hmax2(hm[e & 3], h);
                pk[c * 16 + e] = *reinterpret_cast<const uint32_t*>(&h);
            }
        }
        const float2 hmax = __half22float2(__hmax2(__hmax2(hm[0], hm[1]), __hmax2(hm[2], hm[3])));
        const float pmax = fmaxf(hmax.x, hmax.y);
        if (!__any_sync(0xffffffffu, !(pmax <= kStaleMaxP))) {
            tmem_st32(tS + 0 + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&pk[0]));
            tmem_st32(tS + 32 + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&pk[32]));
            float a0, a1;
            f2_unpack(f2_add(f2_add(ls2[0], ls2[1]), f2_add(ls2[2], ls2[3])), a0, a1);
            l_run += a0 + a1;
            done = true;
        }
    }
    if (!done) {
        if (j == 0) {
            // first tile of the item: row max first (scores read twice)
            uint32_t sr[BN];
            tmem_ld32(tS + 0 + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
            tmem_ld32(tS + 32 + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
            tmem_ld32(tS + 64 + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&sr[64]));
            tmem_ld32(tS + 96 + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&sr[96]));
            tmem_ld_wait();
            float* sv = reinterpret_cast<float*>(sr);
            if (diag) {
#pragma unroll
                for (int c = 0; c < BN; c++)
                    if (kbase + c > qpos) sv[c] = -INFINITY;
            }
            float mx8[8];
#pragma unroll
            for (int e = 0; e < 8; e++) mx8[e] = sv[e];
#pragma unroll
            for (int c = 8; c < BN; c += 8)
#pragma unroll
                for (int e = 0; e < 8; e++) mx8[e] = fmaxf(mx8[e], sv[c + e]);
            m_run = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                          fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
        } else {
            // a row max jumped: rescale O (sum through tile j-1) to the new max
            float mx = -INFINITY;
#pragma unroll 1
            for (int c = 0; c < BN / 32; c++) {
                uint32_t sr[32];
                tmem_ld32(tS + c * 32 + lane_off, sr);
                tmem_ld_wait();
#pragma unroll
                for (int e = 0; e < 32; e++)
                    if (!diag || kbase + c * 32 + e <= qpos) mx = fmaxf(mx, __uint_as_float(sr[e]));
            }
            const float m_new = fmaxf(m_run, mx);
            const float corr = ex2(m_run - m_new);
            wait_prev_pv();
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < HD / 32; c++) {
                uint32_t o[32];
                tmem_ld32(tO + c * 32 + lane_off, o);
                tmem_ld_wait();
#pragma unroll
                for (int e = 0; e < 32; e++) o[e] = __float_as_uint(__uint_as_float(o[e]) * corr);
                tmem_st32(tO + c * 32 + lane_off, o);
            }
            tmem_st_wait();
            l_run *= corr;
            m_run = m_new;
        }
        // exact pass: 32 scores at a time -> p (fp16) over the S columns
        // already read: chunk c's P lands in columns [16c, 16c+16) < 32(c+1)
        float ls8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        uint32_t sbuf[2][32];
        tmem_ld32(tS + lane_off, sbuf[0]);
#pragma unroll
        for (int c = 0; c < BN / 32; c++) {
            tmem_ld_wait();
            uint32_t (&sr)[32] = sbuf[c & 1];
            if (c + 1 < BN / 32) tmem_ld32(tS + (c + 1) * 32 + lane_off, sbuf[(c + 1) & 1]);
            uint32_t pk[16];
#pragma unroll
            for (int e = 0; e < 16; e++) {
                float s0 = __uint_as_float(sr[2 * e]), s1 = __uint_as_float(sr[2 * e + 1]);
                if (diag) {
                    if (kbase + c * 32 + 2 * e > qpos) s0 = -INFINITY;
                    if (kbase + c * 32 + 2 * e + 1 > qpos) s1 = -INFINITY;
                }
                const float p0 = ex2(s0 - m_run);
                const float p1 = ex2(s1 - m_run);
                ls8[e & 7] += p0 + p1;
                pk[e] = pack_half2(p0, p1);
            }
            tmem_st16(tS + c * 16 + lane_off, pk);
        }
        l_run += ((ls8[0] + ls8[1]) + (ls8[2] + ls8[3])) + ((ls8[4] + ls8[5]) + (ls8[6] + ls8[7]));
    }
    tmem_st_wait();
}

template <int HD>
struct Attn2Smem {
    static constexpr int kBoxBytes = BM * 128;
    static constexpr int kTileBytes = (HD / 64) * kBoxBytes;
    static constexpr int NK = 2, NV = 2;
    static constexpr int kQ = 0;  // Q0, Q1
    static constexpr int kK = kQ + 2 * kTileBytes;
    static constexpr int kV = kK + NK * kTileBytes;
    // epilogue staging: one 32 x 32 fp32 block per softmax warp
    static constexpr int kStage = kV + NV * kTileBytes;
    static constexpr int kBars = kStage + 8 * 4096;
    static constexpr int kEnd = kBars + 512;
    static constexpr int kDynBytes = kEnd + 1024;
};

template <int HD>
__global__ void __maxnreg__(168)
    prefill_attn2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                         PrefillArgs a) {
    using L = Attn2Smem<HD>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_pairs = a.hq / 2;
    const int n_items = a.n_qtiles * n_pairs;

    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBars);
    uint64_t* item_full = bars + 0;     // [2]
    uint64_t* item_empty = bars + 2;    // [2]
    uint64_t* q_full = bars + 4;
    uint64_t* q_empty = bars + 5;
    uint64_t* k_full = bars + 6;        // [NK]
    uint64_t* k_empty = k_full + L::NK;
    uint64_t* v_full = k_empty + L::NK;
    uint64_t* v_empty = v_full + L::NV;
    uint64_t* s_full = v_empty + L::NV;  // [2] per head
    uint64_t* p_full = s_full + 2;       // [2]
    uint64_t* pv_done = p_full + 2;      // [2]
    uint64_t* o_free = pv_done + 2;      // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_free + 2);
    int* item_slot = reinterpret_cast<int*>(tmem_slot + 1);  // [2]

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; i++) mbar_init(&item_full[i], 1), mbar_init(&item_empty[i], 3);
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        for (int s = 0; s < L::NK; s++) mbar_init(&k_full[s], 1), mbar_init(&k_empty[s], 1);
        for (int s = 0; s < L::NV; s++) mbar_init(&v_full[s], 1), mbar_init(&v_empty[s], 1);
        for (int w = 0; w < 2; w++)
            mbar_init(&s_full[w], 1), mbar_init(&p_full[w], 4), mbar_init(&pv_done[w], 1), mbar_init(&o_free[w], 4);
        fence_mbar_init();
    }
    if (warp == 9) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t sQ = smem_u32(smem + L::kQ);
    const uint32_t sK = smem_u32(smem + L::kK);
    const uint32_t sV = smem_u32(smem + L::kV);

    auto n_kv_of = [&](int qt) {
        const int q_last = min(qt * BM + BM, a.n_tok) - 1;
        return (a.start + q_last) / BN + 1;
    };
    auto decode_item = [&](int it, int& qt, int& h0) {
        qt = a.n_qtiles - 1 - it / n_pairs;  // longest rows of the causal triangle first
        h0 = 2 * (it % n_pairs);
    };

    if (warp == 8) {
        // ---------------- work queue + TMA producer ----------------
        if (lane == 0) {
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmV);
            int t = 0;  // KV tile counter across items
            for (int k = 0;; k++) {
                const int slot = k & 1;
                if (k >= 2) mbar_wait(&item_empty[slot], (uint32_t)(((k >> 1) - 1) & 1), a.status);
                int it = atomicAdd(a.work_counter, 1);
                if (it >= n_items) it = -1;
                *reinterpret_cast<volatile int*>(&item_slot[slot]) = it;
                mbar_arrive(&item_full[slot]);  // release: the slot write is visible to waiters
                if (it < 0) break;
                int qt, h0;
                decode_item(it, qt, h0);
                const int kvh = h0 / a.g;
                if (k >= 1) mbar_wait(q_empty, (uint32_t)((k - 1) & 1), a.status);
                mbar_arrive_expect_tx(q_full, 2 * L::kTileBytes);
                for (int w = 0; w < 2; w++)
                    for (int c = 0; c < HD / 64; c++)
                        tma_load_2d(smem + L::kQ + w * L::kTileBytes + c * L::kBoxBytes, &tmQ, (h0 + w) * HD + 64 * c,
                                    qt * BM, q_full);
                const int n_kv = n_kv_of(qt);
                for (int j = 0; j < n_kv; j++, t++) {
                    const int sk = t % L::NK, uk = t / L::NK;
                    if (uk > 0) mbar_wait(&k_empty[sk], (uint32_t)((uk - 1) & 1), a.status);
                    mbar_arrive_expect_tx(&k_full[sk], L::kTileBytes);
                    for (int c = 0; c < HD / 64; c++)
                        tma_load_2d(smem + L::kK + sk * L::kTileBytes + c * L::kBoxBytes, &tmK, kvh * HD + 64 * c,
                                    j * BN, &k_full[sk]);
                    const int sv = t % L::NV, uv = t / L::NV;
                    if (uv > 0) mbar_wait(&v_empty[sv], (uint32_t)((uv - 1) & 1), a.status);
                    mbar_arrive_expect_tx(&v_full[sv], L::kTileBytes);
                    for (int c = 0; c < HD / 64; c++)
                        tma_load_2d(smem + L::kV + sv * L::kTileBytes + c * L::kBoxBytes, &tmV, kvh * HD + 64 * c,
                                    j * BN, &v_full[sv]);
                }
            }
        }
        __syncwarp();
    } else if (warp == 9) {
        // ---------------- MMA issuer (lane 0) ----------------
        // Per KV tile t two issue points of 16 MMAs each: [PV0(t), QK0(t+1)] and
        // [PV1(t), QK1(t+1)], each preceded by ONE batch of barrier probes.  S_w(t+1)
        // overwrites P_w(t), the A operand of the PV issued just before it:
        // tcgen05.mma operations of one thread execute in issue order, so no
        // completion wait is needed between the two.
        if (lane == 0) {
            constexpr uint32_t idesc_qk = idesc_f16_f32(BM, BN, false, false);
            constexpr uint32_t idesc_pv = idesc_f16_f32(BM, HD, false, true);
            const uint64_t dq = smem_desc_sw128(sQ, 16, 1024);            // Q0; Q1 one tile later
            const uint64_t dk = smem_desc_sw128(sK, 16, 1024);            // K stage 0
            const uint64_t dv = smem_desc_sw128(sV, L::kBoxBytes, 1024);  // V stage 0, MN-major
            auto mma_qk = [&](int w, int sk) {
                const uint64_t qd = desc_advance(dq, w * L::kTileBytes);
                const uint64_t kd = desc_advance(dk, sk * L::kTileBytes);
                const uint32_t dS = tmem + w * 128;
#pragma unroll
                for (int kk = 0; kk < HD / 16; kk++) {
                    const uint32_t koff = (kk >> 2) * L::kBoxBytes + (kk & 3) * 32;
                    umma_ss(dS, desc_advance(qd, koff), desc_advance(kd, koff), idesc_qk, kk > 0 ? 1u : 0u);
                }
                umma_commit(&s_full[w]);
            };
            auto mma_pv = [&](int w, int sv, bool first) {
                const uint64_t vd = desc_advance(dv, sv * L::kTileBytes);
                const uint32_t dS = tmem + w * 128, dO = tmem + 256 + w * 128;
#pragma unroll
                for (int kk = 0; kk < BN / 16; kk++)
                    umma_ts(dO, dS + kk * 8, desc_advance(vd, kk * 16 * 128), idesc_pv,
                            (!first || kk > 0) ? 1u : 0u);
                umma_commit(&pv_done[w]);
            };
            int t = 0;  // KV tile counter across items
            for (int k = 0;; k++) {
                const int slot = k & 1;
                mbar_wait(&item_full[slot], (uint32_t)((k >> 1) & 1), a.status);
                const int it = *reinterpret_cast<volatile int*>(&item_slot[slot]);
                mbar_arrive(&item_empty[slot]);
                if (it < 0) break;
                int qt, h0;
                decode_item(it, qt, h0);
                const int n_kv = n_kv_of(qt);
                const uint32_t po = (uint32_t)((k - 1) & 1);  // o_free phase of the previous item
                {   // prologue: QK of the first tile for both heads
                    const int sk = t % L::NK;
                    const uint32_t pk = (uint32_t)((t / L::NK) & 1);
                    if (!(mbar_test(q_full, (uint32_t)(k & 1)) & mbar_test(&k_full[sk], pk))) {
                        mbar_wait(q_full, (uint32_t)(k & 1), a.status);
                        mbar_wait(&k_full[sk], pk, a.status);
                    }
                    tc_fence_after();
                    mma_qk(0, sk);
                    mma_qk(1, sk);
                    umma_commit(&k_empty[sk]);
                    if (n_kv == 1) umma_commit(q_empty);
                }
                for (int j = 0; j < n_kv; j++, t++) {
                    const int sv = t % L::NV, skn = (t + 1) % L::NK;
                    const uint32_t pv = (uint32_t)((t / L::NV) & 1), pp = (uint32_t)(t & 1);
                    const uint32_t pkn = (uint32_t)(((t + 1) / L::NK) & 1);
                    const bool more = j + 1 < n_kv, first = j == 0, need_o = first && k >= 1;
                    // issue point 1: V(t), P0(t), O0 free (first tile), K(t+1)
                    bool ok = mbar_test(&v_full[sv], pv) & mbar_test(&p_full[0], pp);
                    if (need_o) ok &= mbar_test(&o_free[0], po);
                    if (more) ok &= mbar_test(&k_full[skn], pkn);
                    if (!ok) {
                        mbar_wait(&v_full[sv], pv, a.status);
                        mbar_wait(&p_full[0], pp, a.status);
                        if (need_o) mbar_wait(&o_free[0], po, a.status);
                        if (more) mbar_wait(&k_full[skn], pkn, a.status);
                    }
                    tc_fence_after();
                    mma_pv(0, sv, first);
                    if (more) mma_qk(0, skn);
                    // issue point 2: P1(t), O1 free (first tile)
                    ok = mbar_test(&p_full[1], pp);
                    if (need_o) ok &= mbar_test(&o_free[1], po);
                    if (!ok) {
                        mbar_wait(&p_full[1], pp, a.status);
                        if (need_o) mbar_wait(&o_free[1], po, a.status);
                    }
                    tc_fence_after();
                    mma_pv(1, sv, first);
                    umma_commit(&v_empty[sv]);
                    if (more) {
                        mma_qk(1, skn);
                        umma_commit(&k_empty[skn]);
                        if (j + 2 == n_kv) umma_commit(q_empty);
                    }
                }
            }
        }
        __syncwarp();
    } else {
        // ---------------- softmax warpgroups ----------------
        const int w = warp >> 2;           // head of the pair
        const int r = threadIdx.x & 127;   // q row == TMEM lane
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t tS = tmem + w * 128, tO = tmem + 256 + w * 128;
        int t = 0;
        for (int k = 0;; k++) {
            const int slot = k & 1;
            mbar_wait(&item_full[slot], (uint32_t)((k >> 1) & 1), a.status);
            const int it = *reinterpret_cast<volatile int*>(&item_slot[slot]);
            // one arrival per warpgroup, after all of its warps have read the slot
            asm volatile("bar.sync %0, 128;" ::"r"(1 + w) : "memory");
            if ((threadIdx.x & 127) == 0) mbar_arrive(&item_empty[slot]);
            if (it < 0) break;
            int qt, h0;
            decode_item(it, qt, h0);
            const int h = h0 + w;
            const int q0 = qt * BM;
            const int qpos = a.start + q0 + r;
            const int n_kv = n_kv_of(qt);
            float m_run = -INFINITY, l_run = 0.f;
            for (int j = 0; j < n_kv; j++, t++) {
                mbar_wait(&s_full[w], (uint32_t)(t & 1), a.status);
                tc_fence_after();
                const int kbase = j * BN;
                const bool diag = kbase + BN - 1 > a.start + q0;  // tile crosses this q tile's diagonal
                softmax_tile<HD>(tS, tO, lane_off, j, kbase, qpos, diag, m_run, l_run,
                                 [&] { mbar_wait(&pv_done[w], (uint32_t)((t - 1) & 1), a.status); });
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[w]);
            }
            // epilogue: O / l -> out[token][h][:], then hand O back to the MMA warp
            mbar_wait(&pv_done[w], (uint32_t)((t - 1) & 1), a.status);
            tc_fence_after();
            const float inv = 1.0f / l_run;
            const int row0 = q0 + (warp & 3) * 32;
            float* stage = reinterpret_cast<float*>(smem + L::kStage + warp * 4096);
#pragma unroll 1
            for (int c = 0; c < HD / 32; c++) {
                uint32_t o[32];
                tmem_ld32(tO + c * 32 + lane_off, o);
                tmem_ld_wait();
                if (c == HD / 32 - 1) {  // O is in registers: the MMA warp may overwrite it
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&o_free[w]);
                }
                stage_store_32x32(o, inv, stage, &tmO, h * HD + c * 32, row0, a.n_tok, lane);
            }
        }
        if (lane == 0) bulk_wait_all();  // the stage must outlive the stores reading it
    }
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ---------------------------------------------------------------------------
// attention, CTA-pair variant (even GQA group size, head_dim 128)
// ---------------------------------------------------------------------------
//
// A cluster of two CTAs on two SMs takes a work item (128-token q tile, heads
// h0, h0+1 of one KV group): CTA r holds head h0+r.  The leader CTA (rank 0)
// issues 2-CTA tensor-core instructions (M = 256: each CTA's 128 q rows) for
// both:
//   S = Q K^T   B = K tile split by keys: CTA r loads keys [64r, 64r+64)
//   O += P V    B = V tile split by columns: CTA r loads hd columns [64r, 64r+64)
// so each SM loads half of every K/V tile, and one thread issues the MMAs of
// two SMs.  TMEM: S_a, S_b, O_0, O_1 (4 x 128 columns).  S is double-buffered,
// so QK of tile t+1 runs while the softmax of tile t does and the softmax never
// waits for a PV; O alternates between items, so an item's output drains while
// the next item runs.  Per CTA: warps 0-3 and 4-7 softmax over key columns
// [0,64) and [64,128) of the same q rows (thread = q row, softmax_half), warp 8
// TMA, warp 9 MMA issue (leader only) and TMEM allocation, warps 10-13
// epilogue (O / l -> out by TMA stores).
// Cross-CTA signalling: the peer's TMA bytes complete on the leader's full
// barriers; MMA completions are committed to the same barrier in both CTAs; the
// peer's softmax and epilogue arrive on the leader's barriers through cluster
// addresses.  Items go to clusters statically, longest first, in serpentine
// order.
// One part (KP = BN/NP of the tile's key columns, part q) of a KV tile of the
// online softmax for the q row of this thread; the warps holding the other
// parts of the same 32 rows (NP in all, one sub-partition) run the same steps,
// and they agree through named barrier `bar` (their NP*32 threads) and the
// exchange area `xs` (SoftmaxXs<NP>::kFloats floats):
//   xs[0..31]            part 0's first-tile max estimate, per lane
//   xs[32 + 32q + lane]  part q's tile max on the exact path
//   flags after that     per-tile flags [tile parity][part]
// All parts keep the same running max m_run; l_run is this part's partial sum.
// P (fp16) of the part's keys goes to TMEM columns [KP*q, KP*q + KP/2) of the S
// buffer, which this part has already read.  On the first tile the running max
// starts as the max of the tile's first 32 columns (part 0's; column 0 is
// visible to every row).  If any p of any part would exceed 2^15 all take the
// exact path: shared new max, each rescales its columns of O and its partial
// sum, then recomputes P.
template <int NP>
struct SoftmaxXs {
    static constexpr int kFlags = 32 + 32 * NP;
    static constexpr int kFloats = kFlags + 2 * NP + (NP == 4 ? 0 : 4);  // a multiple of 4
};

template <int HD, int NP, class WaitPrevPV>
__device__ __forceinline__ void softmax_part(uint32_t tS, uint32_t tO, uint32_t lane_off, int part, int j, int t,
                                             int kbase, int qpos, bool diag, float& m_run, float& l_run, int bar,
                                             float* xs, int lane, WaitPrevPV wait_prev_pv) {
    constexpr int KP = BN / NP, NC = KP / 32;  // columns per part, 32-column chunks per part
    const int col0 = part * KP;
    // one 32-column chunk of this part's scores, masked beyond the diagonal
    auto load_chunk = [&](int c, uint32_t (&sr)[32]) {
        tmem_ld32(tS + col0 + c * 32 + lane_off, sr);
        tmem_ld_wait();
        if (diag) {
#pragma unroll
            for (int e = 0; e < 32; e++)
                if (kbase + col0 + c * 32 + e > qpos) sr[e] = __float_as_uint(-INFINITY);
        }
    };
    if (j == 0) {  // running max estimate from the tile's first 32 columns
        if (part == 0) {
            uint32_t sr[32];
            load_chunk(0, sr);
            float m0 = -INFINITY;
#pragma unroll
            for (int e = 0; e < 32; e++) m0 = fmaxf(m0, __uint_as_float(sr[e]));
            xs[lane] = m0;
        }
        named_bar_sync(bar, NP * 32);
        m_run = xs[lane];
    }
    uint32_t pk[KP / 2];
    // p = 2^(s - m_run) for the part's scores into pk; partial sum and max p.
    // With two chunks the second one's TMEM load is in flight while the first
    // is processed.
    auto p_pass = [&](float& psum, float& pmax) {
        const uint64_t mm2 = f2_pack(m_run, m_run);
        uint64_t ls2[4] = {0ull, 0ull, 0ull, 0ull};
        __half2 hm[2] = {__float2half2_rn(0.f), __float2half2_rn(0.f)};
        uint32_t sb[NC][32];
        tmem_ld32(tS + col0 + lane_off, sb[0]);
#pragma unroll
        for (int c = 0; c < NC; c++) {
            tmem_ld_wait();
            if (c + 1 < NC) tmem_ld32(tS + col0 + (c + 1) * 32 + lane_off, sb[c + 1]);
            uint32_t (&sr)[32] = sb[c];
            if (diag) {
#pragma unroll
                for (int e = 0; e < 32; e++)
                    if (kbase + col0 + c * 32 + e > qpos) sr[e] = __float_as_uint(-INFINITY);
            }
#pragma unroll
            for (int e = 0; e < 16; e++) {
                float d0, d1;
                f2_unpack(f2_sub(f2_pack(__uint_as_float(sr[2 * e]), __uint_as_float(sr[2 * e + 1])), mm2), d0, d1);
                const float p0 = ex2(d0), p1 = ex2(d1);
                ls2[e & 3] = f2_add(ls2[e & 3], f2_pack(p0, p1));
                const __half2 h = __floats2half2_rn(p0, p1);
                hm[e & 1] = __hmax2(hm[e & 1], h);
                pk[c * 16 + e] = *reinterpret_cast<const uint32_t*>(&h);
            }
        }
        float a0, a1;
        f2_unpack(f2_add(f2_add(ls2[0], ls2[1]), f2_add(ls2[2], ls2[3])), a0, a1);
        psum = a0 + a1;
        const float2 hmax = __half22float2(__hmax2(hm[0], hm[1]));
        pmax = fmaxf(hmax.x, hmax.y);
    };
    float psum, pmax;
    p_pass(psum, pmax);
    // every part must accept the stale max for these rows
    int* flags = reinterpret_cast<int*>(xs + SoftmaxXs<NP>::kFlags);
    const bool ok = __all_sync(0xffffffffu, pmax <= kStaleMaxP);
    if (lane == 0) flags[(t & 1) * NP + part] = ok ? 1 : 0;
    named_bar_sync(bar, NP * 32);
    bool ok_all = true;
#pragma unroll
    for (int q = 0; q < NP; q++) ok_all &= flags[(t & 1) * NP + q] != 0;
    if (!ok_all) {
        // exact path: the new row max over all parts
        float mx = -INFINITY;
#pragma unroll 1
        for (int c = 0; c < NC; c++) {
            uint32_t sr[32];
            load_chunk(c, sr);
#pragma unroll
            for (int e = 0; e < 32; e++) mx = fmaxf(mx, __uint_as_float(sr[e]));
        }
        xs[32 + part * 32 + lane] = mx;
        named_bar_sync(bar, NP * 32);
        float m_new = j == 0 ? -INFINITY : m_run;
#pragma unroll
        for (int q = 0; q < NP; q++) m_new = fmaxf(m_new, xs[32 + q * 32 + lane]);
        if (j > 0) {  // rescale this part's O columns (sum through tile j-1) and partial sum
            const float corr = ex2(m_run - m_new);
            wait_prev_pv();
            tc_fence_after();
            constexpr int OC = HD / NP;  // O columns of this part
#pragma unroll 1
            for (int c = 0; c < OC / 32; c++) {
                uint32_t o[32];
                tmem_ld32(tO + part * OC + c * 32 + lane_off, o);
                tmem_ld_wait();
#pragma unroll
                for (int e = 0; e < 32; e++) o[e] = __float_as_uint(__uint_as_float(o[e]) * corr);
                tmem_st32(tO + part * OC + c * 32 + lane_off, o);
            }
            tmem_st_wait();
            l_run *= corr;
        }
        m_run = m_new;
        p_pass(psum, pmax);
    }
    if constexpr (KP / 2 == 32) {
        tmem_st32(tS + col0 + lane_off, pk);
    } else {
        tmem_st16(tS + col0 + lane_off, pk);
    }
    l_run += psum;
    tmem_st_wait();
}

// Softmax parts per tile row in the CTA-pair kernel: four warps per
// sub-partition share its exponential unit (each 32 columns per row), so one
// warp's loads, stores and waits hide behind the others' exponentials.
constexpr int kPairParts = 4;
constexpr int kPairThreads = kPairParts * 128 + 64 + 128;  // softmax, TMA + MMA, epilogue

struct PairSmem {
    static constexpr int kQBytes = 2 * BM * 128;    // 128 rows x 128 hd columns (two 64-column boxes)
    static constexpr int kKBytes = 2 * 64 * 128;    // 64 keys x 128 hd columns (two boxes)
    static constexpr int kVBytes = 128 * 128;       // 128 keys x 64 hd columns (one box)
    static constexpr int NK = 3, NV = 3;
    static constexpr int kQ = 0;  // two Q slots: item k uses slot k % 2
    static constexpr int kK = kQ + 2 * kQBytes;
    static constexpr int kV = kK + NK * kKBytes;
    static constexpr int kStage = kV + NV * kVBytes;  // epilogue: 32 x 32 fp32 per epilogue warp
    static constexpr int kLsum = kStage + 4 * 4096;   // row sums handed to the epilogue [O buffer][part][128]
    static constexpr int kXch = kLsum + 2 * kPairParts * 128 * 4;  // softmax part exchange, per row group
    static constexpr int kBars = kXch + 4 * SoftmaxXs<kPairParts>::kFloats * 4;
    static constexpr int kEnd = kBars + 512;
    static constexpr int kDynBytes = kEnd + 1024;
};

// kPairThreads = 704 threads: 22 warps, six of them on two of the SM's
// sub-partitions, whose 16,384 registers then allow 80 per thread
__global__ void __launch_bounds__(kPairThreads, 1)
    prefill_attn_pair_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKh,
                             const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                             PrefillArgs a) {
    constexpr int HD = 128;
    using L = PairSmem;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int cluster = blockIdx.x >> 1, n_clusters = gridDim.x >> 1;
    const int n_pairs = a.hq / 2;
    const int n_items = a.n_qtiles * n_pairs;

    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBars);
    uint64_t* q_full = bars + 0;          // [2] leader: both Q tiles of the slot landed
    uint64_t* q_empty = bars + 2;         // [2] both: last QK reading the slot done
    uint64_t* k_full = bars + 4;          // [NK] leader
    uint64_t* k_empty = k_full + L::NK;   // [NK] both
    uint64_t* v_full = k_empty + L::NK;   // [NV] leader
    uint64_t* v_empty = v_full + L::NV;   // [NV] both
    uint64_t* s_full = v_empty + L::NV;   // [2] both, per S buffer
    uint64_t* p_full = s_full + 2;        // [2] leader, one arrival per softmax warp of both CTAs
    // PV(t) completes pv_done[t % 2]: with QK(t+1) issued before PV(t) a single
    // barrier could run two phases behind a waiter, which a parity wait cannot tell
    uint64_t* pv_done = p_full + 2;       // [2] both
    uint64_t* o_full = pv_done + 2;       // [2] both, per O buffer: the item's last PV done
    uint64_t* l_full = o_full + 2;        // [2] own, one arrival per softmax warp: row sums written
    uint64_t* o_free = l_full + 2;        // [2] leader, 8 arrivals (4 epilogue warps x 2 CTAs)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_free + 2);
    float* lsum = reinterpret_cast<float*>(smem + L::kLsum);
    float* xch = reinterpret_cast<float*>(smem + L::kXch);

    if (threadIdx.x == 0) {
        for (int b = 0; b < 2; b++) mbar_init(&q_full[b], 1), mbar_init(&q_empty[b], 1);
        for (int s = 0; s < L::NK; s++) mbar_init(&k_full[s], 1), mbar_init(&k_empty[s], 1);
        for (int s = 0; s < L::NV; s++) mbar_init(&v_full[s], 1), mbar_init(&v_empty[s], 1);
        for (int b = 0; b < 2; b++) {
            mbar_init(&s_full[b], 1), mbar_init(&p_full[b], 2 * 4 * kPairParts), mbar_init(&pv_done[b], 1);
            mbar_init(&o_full[b], 1), mbar_init(&l_full[b], 4 * kPairParts), mbar_init(&o_free[b], 8);
        }
        fence_mbar_init();
    }
    constexpr int W_TMA = 4 * kPairParts, W_MMA = W_TMA + 1, W_EPI = W_TMA + 2;
    // Programmatic dependent launch: the next kernel (the next layer's prep,
    // which waits for this one to complete) may launch now; this kernel set
    // itself up while the prep kernel before it finished, and waits for it
    // before its first load of q or the cache and its first store.
    pdl_trigger();
    if (warp == W_MMA) tmem_alloc_pair(tmem_slot, 512);
    tc_fence_before();
    cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated in both
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();

    // item r-th of this cluster: serpentine over the longest-first order
    auto item_of = [&](int r) {
        const int idx = r * n_clusters + ((r & 1) ? (n_clusters - 1 - cluster) : cluster);
        return idx < n_items ? idx : -1;
    };
    auto n_kv_of = [&](int qt) {
        const int q_last = min(qt * BM + BM, a.n_tok) - 1;
        return (a.start + q_last) / BN + 1;
    };

    if (warp == W_TMA) {
        // ---------------- TMA producer (both CTAs) ----------------
        if (lane == 0) {
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmKh);
            prefetch_tmap(&tmV);
            int t = 0, items = 0;
            for (int k = 0;; k++) {
                const int it = item_of(k);
                if (it < 0) break;
                const int qt = a.n_qtiles - 1 - it / n_pairs, h0 = 2 * (it % n_pairs);
                const int h = h0 + (int)rank, kvh = h0 / a.g;
                const int qs = k & 1;
                if (k >= 2) mbar_wait(&q_empty[qs], (uint32_t)(((k >> 1) - 1) & 1), a.status);
                if (rank == 0) mbar_arrive_expect_tx(&q_full[qs], 2 * L::kQBytes);
                for (int c = 0; c < 2; c++)
                    tma_load_2d_pair(smem + L::kQ + qs * L::kQBytes + c * BM * 128, &tmQ, h * HD + 64 * c, qt * BM,
                                     mapa_shared(&q_full[qs], 0));
                const int n_kv = n_kv_of(qt);
                for (int j = 0; j < n_kv; j++, t++) {
                    const int sk = t % L::NK, uk = t / L::NK;
                    if (uk > 0) mbar_wait(&k_empty[sk], (uint32_t)((uk - 1) & 1), a.status);
                    if (rank == 0) mbar_arrive_expect_tx(&k_full[sk], 2 * L::kKBytes);
                    const uint32_t kf = mapa_shared(&k_full[sk], 0);
                    for (int c = 0; c < 2; c++)
                        tma_load_2d_pair(smem + L::kK + sk * L::kKBytes + c * 64 * 128, &tmKh, kvh * HD + 64 * c,
                                         j * BN + 64 * (int)rank, kf);
                    const int sv = t % L::NV, uv = t / L::NV;
                    if (uv > 0) mbar_wait(&v_empty[sv], (uint32_t)((uv - 1) & 1), a.status);
                    if (rank == 0) mbar_arrive_expect_tx(&v_full[sv], 2 * L::kVBytes);
                    tma_load_2d_pair(smem + L::kV + sv * L::kVBytes, &tmV, kvh * HD + 64 * (int)rank, j * BN,
                                     mapa_shared(&v_full[sv], 0));
                }
                items = k + 1;
            }
            // tail: the leader's last commits to this CTA's empty barriers must have
            // landed before the CTA may exit
            for (int s = 0; s < L::NK && s < t; s++) {
                const int last = s + L::NK * ((t - 1 - s) / L::NK);
                mbar_wait(&k_empty[s], (uint32_t)((last / L::NK) & 1), a.status);
            }
            for (int s = 0; s < L::NV && s < t; s++) {
                const int last = s + L::NV * ((t - 1 - s) / L::NV);
                mbar_wait(&v_empty[s], (uint32_t)((last / L::NV) & 1), a.status);
            }
            for (int qs = 0; qs < 2 && qs < items; qs++) {
                const int last = qs + 2 * ((items - 1 - qs) / 2);
                mbar_wait(&q_empty[qs], (uint32_t)((last >> 1) & 1), a.status);
            }
        }
        __syncwarp();
    } else if (warp == W_MMA) {
        // ---------------- MMA issuer (leader lane 0) ----------------
        if (rank == 0 && lane == 0) {
            constexpr uint32_t idesc_qk = idesc_f16_f32(2 * BM, BN, false, false);
            constexpr uint32_t idesc_pv = idesc_f16_f32(2 * BM, HD, false, true);
            const uint64_t dq = smem_desc_sw128(smem_u32(smem + L::kQ), 16, 1024);
            const uint64_t dk = smem_desc_sw128(smem_u32(smem + L::kK), 16, 1024);
            const uint64_t dv = smem_desc_sw128(smem_u32(smem + L::kV), L::kVBytes, 1024);
            auto mma_qk = [&](int tt, int qs) {  // S[tt % 2] = Q(slot qs) K(tt)^T
                const int sk = tt % L::NK;
                const uint64_t kd = desc_advance(dk, sk * L::kKBytes);
                const uint64_t qd = desc_advance(dq, qs * L::kQBytes);
                const uint32_t dS = tmem + (uint32_t)((tt & 1) * 128);
#pragma unroll
                for (int kk = 0; kk < HD / 16; kk++) {
                    const uint32_t qoff = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
                    const uint32_t koff = (kk >> 2) * (64 * 128) + (kk & 3) * 32;
                    umma2_ss(dS, desc_advance(qd, qoff), desc_advance(kd, koff), idesc_qk, kk > 0 ? 1u : 0u);
                }
                umma2_commit_both(&s_full[tt & 1]);
                umma2_commit_both(&k_empty[sk]);
            };
            // QK of tile tt, the jj-th of item kk (n tiles): Q and K must have landed
            auto issue_qk = [&](int tt, int kk, int jj, int n) {
                const uint32_t pk = (uint32_t)((tt / L::NK) & 1);
                bool ok = mbar_test(&k_full[tt % L::NK], pk);
                if (jj == 0) ok &= mbar_test(&q_full[kk & 1], (uint32_t)((kk >> 1) & 1));
                if (!ok) {
                    if (jj == 0) mbar_wait(&q_full[kk & 1], (uint32_t)((kk >> 1) & 1), a.status);
                    mbar_wait(&k_full[tt % L::NK], pk, a.status);
                }
                tc_fence_after();
                mma_qk(tt, kk & 1);
                if (jj + 1 == n) umma2_commit_both(&q_empty[kk & 1]);  // the item's last QK: Q slot free
            };
            int it = item_of(0);
            int t = 0;
            if (it >= 0) {
                const int n0 = n_kv_of(a.n_qtiles - 1 - it / n_pairs);
                issue_qk(0, 0, 0, n0);
            }
            for (int k = 0; it >= 0; k++) {
                const int n_kv = n_kv_of(a.n_qtiles - 1 - it / n_pairs);
                const int it_next = item_of(k + 1);
                const int n_next = it_next >= 0 ? n_kv_of(a.n_qtiles - 1 - it_next / n_pairs) : 0;
                const int ob = k & 1;
                const uint32_t tO = tmem + 256 + (uint32_t)(ob * 128);
                for (int j = 0; j < n_kv; j++, t++) {
                    // S of the next tile into the other buffer, across the item boundary
                    if (j + 1 < n_kv) issue_qk(t + 1, k, j + 1, n_kv);
                    else if (n_next > 0) issue_qk(t + 1, k + 1, 0, n_next);
                    const int sv = t % L::NV;
                    const uint32_t pp = (uint32_t)((t >> 1) & 1), pv = (uint32_t)((t / L::NV) & 1);
                    // the first PV of item k overwrites O_(k%2): item k-2's epilogue must have read it
                    const bool first = j == 0, need_o = first && k >= 2;
                    const uint32_t po = (uint32_t)(((k >> 1) - 1) & 1);
                    bool ok = mbar_test(&p_full[t & 1], pp) & mbar_test(&v_full[sv], pv);
                    if (need_o) ok &= mbar_test(&o_free[ob], po);
                    if (!ok) {
                        mbar_wait(&p_full[t & 1], pp, a.status);
                        mbar_wait(&v_full[sv], pv, a.status);
                        if (need_o) mbar_wait(&o_free[ob], po, a.status);
                    }
                    tc_fence_after();
                    const uint64_t vd = desc_advance(dv, sv * L::kVBytes);
                    const uint32_t dS = tmem + (uint32_t)((t & 1) * 128);
                    // P of part q's keys (KP = BN/NP of them) in S columns [KP*q, KP*q + KP/2);
                    // K step kk covers keys [16kk, 16kk+16): 8 packed columns
                    constexpr int KP = BN / kPairParts;
#pragma unroll
                    for (int kk = 0; kk < BN / 16; kk++)
                        umma2_ts(tO, dS + (uint32_t)((kk * 16 / KP) * KP + (kk * 16 % KP) / 2),
                                 desc_advance(vd, kk * 16 * 128), idesc_pv, (!first || kk > 0) ? 1u : 0u);
                    umma2_commit_both(&pv_done[t & 1]);
                    umma2_commit_both(&v_empty[sv]);
                    if (j + 1 == n_kv) umma2_commit_both(&o_full[ob]);
                }
                it = it_next;
            }
        }
        __syncwarp();
    } else if (warp < W_TMA) {
        // ---------------- softmax (both CTAs): warps 4q..4q+3 take key columns [KP*q, KP*q + KP) ----------------
        const int part = warp >> 2;
        const int r = threadIdx.x & 127;  // q row == TMEM lane
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const int bar = 1 + (warp & 3);  // with the warps of the other parts over the same rows
        float* xs = xch + (warp & 3) * SoftmaxXs<kPairParts>::kFloats;
        const uint32_t p_full_l0 = mapa_shared(&p_full[0], 0), p_full_l1 = mapa_shared(&p_full[1], 0);
        int t = 0;
        for (int k = 0;; k++) {
            const int it = item_of(k);
            if (it < 0) break;
            const int qt = a.n_qtiles - 1 - it / n_pairs;
            const int q0 = qt * BM;
            const int qpos = a.start + q0 + r;
            const int n_kv = n_kv_of(qt);
            const uint32_t tO = tmem + 256 + (uint32_t)((k & 1) * 128);
            float m_run = -INFINITY, l_run = 0.f;
            for (int j = 0; j < n_kv; j++, t++) {
                if (!mbar_test(&s_full[t & 1], (uint32_t)((t >> 1) & 1)))
                    mbar_wait(&s_full[t & 1], (uint32_t)((t >> 1) & 1), a.status);
                tc_fence_after();
                const int kbase = j * BN;
                const bool diag = kbase + BN - 1 > a.start + q0;
                const uint32_t tS = tmem + (uint32_t)((t & 1) * 128);
                softmax_part<HD, kPairParts>(
                    tS, tO, lane_off, part, j, t, kbase, qpos, diag, m_run, l_run, bar, xs, lane,
                    [&] { mbar_wait(&pv_done[(t - 1) & 1], (uint32_t)(((t - 1) >> 1) & 1), a.status); });
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_remote((t & 1) ? p_full_l1 : p_full_l0);
            }
            // hand the partial row sums to the epilogue warps.  lsum[k % 2] is free
            // again: item k-2's epilogue read it before releasing O_(k%2), which
            // this item's first PV waited for
            lsum[((k & 1) * kPairParts + part) * 128 + r] = l_run;
            __syncwarp();
            if (lane == 0) mbar_arrive(&l_full[k & 1]);
        }
    } else if (warp >= W_EPI) {
        // ---------------- epilogue (both CTAs) ----------------
        const int sub = warp & 3;  // TMEM subpartition of this warp: rows 32*sub ..
        const uint32_t lane_off = (uint32_t)(sub * 32) << 16;
        float* stage = reinterpret_cast<float*>(smem + L::kStage + (warp - W_EPI) * 4096);
        int k = 0;
        for (;; k++) {
            const int it = item_of(k);
            if (it < 0) break;
            const int qt = a.n_qtiles - 1 - it / n_pairs, h = 2 * (it % n_pairs) + (int)rank;
            const int ob = k & 1;
            const uint32_t tO = tmem + 256 + (uint32_t)(ob * 128);
            mbar_wait(&o_full[ob], (uint32_t)((k >> 1) & 1), a.status);
            mbar_wait(&l_full[ob], (uint32_t)((k >> 1) & 1), a.status);
            tc_fence_after();
            float lsum_row = 0.f;
#pragma unroll
            for (int q = 0; q < kPairParts; q++) lsum_row += lsum[(ob * kPairParts + q) * 128 + sub * 32 + lane];
            const float inv = 1.0f / lsum_row;
            const int row0 = qt * BM + sub * 32;
#pragma unroll 1
            for (int c = 0; c < HD / 32; c++) {
                uint32_t o[32];
                tmem_ld32(tO + c * 32 + lane_off, o);
                tmem_ld_wait();
                if (c == HD / 32 - 1) {  // O and l are in registers: release the buffer
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_remote(mapa_shared(&o_free[ob], 0));
                }
                stage_store_32x32(o, inv, stage, &tmO, h * HD + c * 32, row0, a.n_tok, lane);
            }
        }
        if (lane == 0) bulk_wait_all();
    }
    tc_fence_before();
    cluster_sync_all();  // no CTA leaves while its peer may still signal it
    if (warp == W_MMA) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, 512);
    }
}

// ---------------------------------------------------------------------------
// host: tensor maps and launch
// ---------------------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// 2-D map over a row-major fp16 matrix [rows][inner] with row stride `stride_bytes`;
// 64-column x box_rows boxes with the 128-byte swizzle the UMMA descriptors above expect.
// Rows past `rows` read as zeros.
bool make_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint64_t stride_bytes,
              uint32_t box_rows = 128) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {stride_bytes};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D map over the fp32 output [n_tok][hq*hd] for the epilogue's stores: 32 x 32
// boxes (128-byte rows, 128-byte swizzle, matching stage_store_32x32's stage).
bool make_out_map(CUtensorMap* m, float* base, uint64_t inner, uint64_t rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {inner * 4};
    const cuuint32_t box[2] = {32, 32};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// One-time, per-device setup of the prefill kernels for one head_dim: their
// shared-memory limits, the prep kernel's resident blocks per SM (its grid is
// one wave), and whether the CTA-pair and head-pair kernels can be resident
// (the CTA pair needs kPairThreads threads x 80 registers and 2-CTA clusters).
struct PrefillSetup {
    bool done = false;
    cudaError_t err = cudaSuccess;
    int pair_clusters = 0;  // resident CTA-pair clusters, 0 if none
    bool pair_ok = false;   // head-pair kernel resident
    int sms = 148;
    int prep_blocks[2] = {1, 1};  // prep blocks per SM: fp16 inputs, fp32 inputs
};

// The prep kernel for one input element size: the largest shared-memory
// carveout (the attention kernel after it needs it too, so the SM need not
// change its split between the two) and its resident blocks per SM.
template <int HD, int ES>
cudaError_t prep_setup(int& blocks) {
    cudaError_t e = cudaFuncSetAttribute(prefill_prep_kernel<HD, ES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         prep_smem_bytes(HD, ES));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(prefill_prep_kernel<HD, ES>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e == cudaSuccess)
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, prefill_prep_kernel<HD, ES>, kPrepWarps * 32,
                                                          prep_smem_bytes(HD, ES));
    if (e == cudaSuccess && blocks < 1) e = cudaErrorInvalidConfiguration;
    return e;
}

template <int HD>
const PrefillSetup& prefill_setup() {
    static std::mutex mu;
    static PrefillSetup table[64];
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    PrefillSetup& st = table[dev & 63];
    if (st.done) return st;
    st.done = true;
    cudaDeviceGetAttribute(&st.sms, cudaDevAttrMultiProcessorCount, dev);
    st.err = prep_setup<HD, 2>(st.prep_blocks[0]);
    if (st.err != cudaSuccess) return st;
    st.err = prep_setup<HD, 4>(st.prep_blocks[1]);
    if (st.err != cudaSuccess) return st;
    st.err = cudaFuncSetAttribute(prefill_attn_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  AttnSmem<HD>::kDynBytes);
    if (st.err != cudaSuccess) return st;
    st.err = cudaFuncSetAttribute(prefill_attn2_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  Attn2Smem<HD>::kDynBytes);
    if (st.err != cudaSuccess) return st;
    int nb = 0;
    st.pair_ok = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, prefill_attn2_kernel<HD>, 320,
                                                               Attn2Smem<HD>::kDynBytes) == cudaSuccess &&
                 nb > 0;
    if (HD == 128 && cudaFuncSetAttribute(prefill_attn_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          PairSmem::kDynBytes) == cudaSuccess) {
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2, attr[0].val.clusterDim.y = 1, attr[0].val.clusterDim.z = 1;
        cfg.gridDim = dim3(2, 1, 1);
        cfg.blockDim = dim3(kPairThreads, 1, 1);
        cfg.dynamicSmemBytes = PairSmem::kDynBytes;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, prefill_attn_pair_kernel, &cfg) == cudaSuccess) st.pair_clusters = n;
    }
    cudaGetLastError();  // a refused query leaves the CTA pair off, not an error
    return st;
}

// 2: CTA pair, 1: head pair on one SM, 0: one head per CTA
template <int HD>
int prefill_variant(const PrefillSetup& st, int g) {
    if (HD == 128 && g % 2 == 0 && st.pair_clusters > 0) return 2;
    if (g % 2 == 0 && st.pair_ok) return 1;
    return 0;
}

template <int HD>
cudaError_t launch_prefill_hd(const PrefillArgs& a, cudaStream_t stream, unsigned stages) {
    if (stages & PICOATTN_STAGE_PREPARE) {
        // units of (token, kind, group of 8 heads); one wave of 8-warp blocks,
        // fewer when there are fewer units than warps
        const PrefillSetup& st = prefill_setup<HD>();
        if (st.err != cudaSuccess) return st.err;
        const bool f16 = a.in_dtype == PICOATTN_DTYPE_F16;
        const long units = (long)a.n_tok * ((a.hq + kPrepUnit - 1) / kPrepUnit + 2 * ((a.hkv + kPrepUnit - 1) / kPrepUnit));
        const long wave = (long)st.prep_blocks[f16 ? 0 : 1] * st.sms;
        const long blocks = std::min((units + kPrepWarps - 1) / kPrepWarps, wave);
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.gridDim = dim3((unsigned)blocks, 1, 1);
        cfg.blockDim = dim3(kPrepWarps * 32, 1, 1);
        cfg.dynamicSmemBytes = f16 ? prep_smem_bytes(HD, 2) : prep_smem_bytes(HD, 4);
        cfg.stream = stream;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        const cudaError_t e = f16 ? cudaLaunchKernelEx(&cfg, prefill_prep_kernel<HD, 2>, a)
                                  : cudaLaunchKernelEx(&cfg, prefill_prep_kernel<HD, 4>, a);
        if (e != cudaSuccess) return e;
    }
    if (stages & PICOATTN_STAGE_ATTEND) {
        const PrefillSetup& st = prefill_setup<HD>();
        if (st.err != cudaSuccess) return st.err;
        CUtensorMap mq, mk, mv, mo;
        const uint64_t kvd = (uint64_t)a.kvd;
        const size_t slab = (size_t)a.layer * a.max_seq * a.kvd;
        if (!make_map(&mq, a.q16, (uint64_t)a.hq * HD, (uint64_t)a.n_tok, (uint64_t)a.hq * HD * 2) ||
            !make_map(&mv, a.v_cache + slab, kvd, (uint64_t)(a.start + a.n_tok), kvd * 2) ||
            !make_out_map(&mo, a.out, (uint64_t)a.hq * HD, (uint64_t)a.n_tok))
            return cudaErrorInvalidValue;
        const int variant = prefill_variant<HD>(st, a.g);
        const int n_pair_items = a.n_qtiles * (a.hq / 2);
        if (variant == 2) {
            // CTA pairs (head_dim 128, heads in pairs of one KV group): clusters of 2;
            // K tiles come in halves of 64 keys
            if (!make_map(&mk, a.k_cache + slab, kvd, (uint64_t)(a.start + a.n_tok), kvd * 2, 64))
                return cudaErrorInvalidValue;
            const int clusters = n_pair_items < st.pair_clusters ? n_pair_items : st.pair_clusters;
            cudaLaunchConfig_t cfg = {};
            cudaLaunchAttribute attr[2];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = 2, attr[0].val.clusterDim.y = 1, attr[0].val.clusterDim.z = 1;
            attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[1].val.programmaticStreamSerializationAllowed = 1;
            cfg.gridDim = dim3((unsigned)(2 * clusters), 1, 1);
            cfg.blockDim = dim3(kPairThreads, 1, 1);
            cfg.dynamicSmemBytes = PairSmem::kDynBytes;
            cfg.stream = stream;
            cfg.attrs = attr;
            cfg.numAttrs = 2;
            cudaError_t e = cudaLaunchKernelEx(&cfg, prefill_attn_pair_kernel, mq, mk, mv, mo, a);
            if (e != cudaSuccess) return e;
            return cudaGetLastError();
        }
        if (!make_map(&mk, a.k_cache + slab, kvd, (uint64_t)(a.start + a.n_tok), kvd * 2))
            return cudaErrorInvalidValue;
        if (variant == 1) {
            // head pairs share a KV head: persistent grid, one CTA per SM
            const int grid = n_pair_items < st.sms ? n_pair_items : st.sms;
            prefill_attn2_kernel<HD><<<grid, 320, Attn2Smem<HD>::kDynBytes, stream>>>(mq, mk, mv, mo, a);
        } else {
            dim3 grid((unsigned)a.n_qtiles, (unsigned)a.hq);
            prefill_attn_kernel<HD><<<grid, 192, AttnSmem<HD>::kDynBytes, stream>>>(mq, mk, mv, mo, a);
        }
    }
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_prefill(const PrefillArgs& a, cudaStream_t stream, unsigned stages) {
    return a.hd == 64 ? launch_prefill_hd<64>(a, stream, stages) : launch_prefill_hd<128>(a, stream, stages);
}

int prefill_kernel_variant(const picoattn_config_t& cfg) {
    const int g = cfg.n_heads / cfg.n_kv_heads;
    if (cfg.head_dim == 64) {
        const PrefillSetup& st = prefill_setup<64>();
        return st.err != cudaSuccess ? -1 : prefill_variant<64>(st, g);
    }
    const PrefillSetup& st = prefill_setup<128>();
    return st.err != cudaSuccess ? -1 : prefill_variant<128>(st, g);
}

size_t prefill_workspace_bytes(const picoattn_config_t& cfg, int n_tok) {
    return kWsHeaderBytes + align_up((size_t)n_tok * cfg.n_heads * cfg.head_dim * 2, 256);
}

}  // namespace picoattn
