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
#include <cmath>
#include <cstdio>

#include <cuda.h>

#include "device_common.cuh"
#include "picoattn_internal.h"
#include "tcgen05.cuh"

namespace picoattn {

namespace {

constexpr int BM = 128;  // q rows per tile
constexpr int BN = 128;  // keys per tile
constexpr float kRescaleThreshold = 8.0f;

// ---------------------------------------------------------------------------
// prep
// ---------------------------------------------------------------------------

template <int HD>
__device__ __forceinline__ void rmsnorm_ref_p(float* x, const float* w, float eps, int lane) {
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

template <int HD>
__device__ __forceinline__ void rope_ref_p(float* x, const float* c, const float* s, int mode, int lane) {
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

__device__ __forceinline__ float load_in(const void* p, size_t i, int dtype) {
    return dtype == PICOATTN_DTYPE_F16 ? __half2float(reinterpret_cast<const __half*>(p)[i])
                                       : reinterpret_cast<const float*>(p)[i];
}

template <int HD>
__global__ void __launch_bounds__(256) prefill_prep_kernel(PrefillArgs a) {
    __shared__ float buf[8][HD];
    const int i = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos = a.start + i;
    const size_t row = ((size_t)a.layer * a.max_seq + pos) * a.kvd;
    const float* crow = a.rope_cos + (size_t)pos * (HD / 2);
    const float* srow = a.rope_sin + (size_t)pos * (HD / 2);
    const float qscale = 1.4426950408889634f / sqrtf((float)HD);
    float* x = buf[warp];
    const int n_slots = a.hq + 2 * a.hkv;
    {
        const int slot = blockIdx.x * 8 + warp;  // one warp per head vector
        if (slot >= n_slots) return;
        int kind, h;
        const void* src;
        size_t off;
        if (slot < a.hq) {
            kind = 0, h = slot, src = a.q, off = ((size_t)i * a.hq + h) * HD;
        } else if (slot < a.hq + a.hkv) {
            kind = 1, h = slot - a.hq, src = a.k, off = ((size_t)i * a.hkv + h) * HD;
        } else {
            kind = 2, h = slot - a.hq - a.hkv, src = a.v, off = ((size_t)i * a.hkv + h) * HD;
        }
        for (int d = lane; d < HD; d += 32) x[d] = load_in(src, off + d, a.in_dtype);
        __syncwarp();
        if (kind != 2) {
            const float* w = kind == 0 ? a.qn_w : a.kn_w;
            if (w) rmsnorm_ref_p<HD>(x, w, a.eps, lane);
            rope_ref_p<HD>(x, crow, srow, a.rope_mode, lane);
        }
        if (kind == 0) {
            __half* dst = a.q16 + ((size_t)i * a.hq + h) * HD;
            for (int d = lane; d < HD; d += 32) dst[d] = __float2half_rn(x[d] * qscale);
        } else {
            uint16_t* dst = (kind == 1 ? a.k_cache : a.v_cache) + row + (size_t)h * HD;
            for (int d = lane; d < HD; d += 32) dst[d] = f32_to_f16_ref(x[d]);
        }
        __syncwarp();
    }
}

// ---------------------------------------------------------------------------
// attention (tcgen05 / TMEM)
// ---------------------------------------------------------------------------

template <int HD>
struct AttnSmem {
    static constexpr int kBoxBytes = BM * 128;              // one 128-row x 64-column fp16 box
    static constexpr int kTileBytes = (HD / 64) * kBoxBytes;  // 128 rows x HD columns
    static constexpr int NK = 2, NV = 2;
    static constexpr int kQ = 0;
    static constexpr int kK = kQ + kTileBytes;
    static constexpr int kV = kK + NK * kTileBytes;
    static constexpr int kBars = kV + NV * kTileBytes;
    static constexpr int kEnd = kBars + 256;
    static constexpr int kDynBytes = kEnd + 1024;  // slack to align the base to 1024
};

template <int HD>
__global__ void __launch_bounds__(192, 1)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, PrefillArgs a) {
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
        auto issue_pv = [&](int i) {
            const int b = i & 1, sv = i % L::NV;
            mbar_wait(&p_full[b], (uint32_t)((i >> 1) & 1), a.status);
            mbar_wait(&v_full[sv], (uint32_t)((i / L::NV) & 1), a.status);
            tc_fence_after();
            if (lane == 0) {
                const uint32_t vbase = sV + sv * L::kTileBytes;
#pragma unroll
                for (int kk = 0; kk < BN / 16; kk++) {
                    // B = V tile, MN-major: 64-column boxes LBO apart, 8-key groups SBO apart
                    const uint64_t bdesc = smem_desc_sw128(vbase + kk * 16 * 128, L::kBoxBytes, 1024);
                    umma_ts(tO, tS0 + b * 128 + kk * 8, bdesc, idesc_pv, (i > 0 || kk > 0) ? 1u : 0u);
                }
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
                const uint32_t kbase = sK + sk * L::kTileBytes;
#pragma unroll
                for (int kk = 0; kk < HD / 16; kk++) {
                    const uint32_t koff = (kk >> 2) * L::kBoxBytes + (kk & 3) * 32;
                    const uint64_t adesc = smem_desc_sw128(sQ + koff, 16, 1024);
                    const uint64_t bdesc = smem_desc_sw128(kbase + koff, 16, 1024);
                    umma_ss(tS0 + b * 128, adesc, bdesc, idesc_qk, kk > 0 ? 1u : 0u);
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
            float s[BN];
#pragma unroll
            for (int c = 0; c < BN / 32; c++) {
                uint32_t t[32];
                tmem_ld32(tS0 + b * 128 + c * 32 + lane_off, t);
                tmem_ld_wait();
#pragma unroll
                for (int e = 0; e < 32; e++) s[c * 32 + e] = __uint_as_float(t[e]);
            }
            const int kbase = j * BN;
            if (kbase + BN - 1 > a.start + q0) {  // tile crosses the diagonal of this q tile
#pragma unroll
                for (int c = 0; c < BN; c++)
                    if (kbase + c > qpos) s[c] = -INFINITY;
            }
            float mx = s[0];
#pragma unroll
            for (int c = 1; c < BN; c++) mx = fmaxf(mx, s[c]);
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
            float lsum = 0.f;
#pragma unroll
            for (int c = 0; c < BN / 64; c++) {
                uint32_t t[32];
#pragma unroll
                for (int e = 0; e < 32; e++) {
                    const float p0 = ex2(s[c * 64 + 2 * e] - m_run);
                    const float p1 = ex2(s[c * 64 + 2 * e + 1] - m_run);
                    lsum += p0 + p1;
                    t[e] = pack_half2(p0, p1);
                }
                tmem_st32(tS0 + b * 128 + c * 32 + lane_off, t);
            }
            l_run += lsum;
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[b]);
        }
        // epilogue: O / l -> out[token][h][:]
        mbar_wait(&pv_done[(n_kv - 1) & 1], (uint32_t)(((n_kv - 1) >> 1) & 1), a.status);
        tc_fence_after();
        const int tok = q0 + r;
        const float inv = 1.0f / l_run;
        float* dst = a.out + ((size_t)tok * a.hq + h) * HD;
#pragma unroll
        for (int c = 0; c < HD / 32; c++) {
            uint32_t t[32];
            tmem_ld32(tO + c * 32 + lane_off, t);
            tmem_ld_wait();
            if (tok < a.n_tok) {
#pragma unroll
                for (int e = 0; e < 32; e += 4)
                    *reinterpret_cast<float4*>(dst + c * 32 + e) =
                        make_float4(__uint_as_float(t[e]) * inv, __uint_as_float(t[e + 1]) * inv,
                                    __uint_as_float(t[e + 2]) * inv, __uint_as_float(t[e + 3]) * inv);
            }
        }
        tc_fence_before();
    }
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
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
// 64 x 128 boxes with the 128-byte swizzle the UMMA descriptors above expect.
// Rows past `rows` read as zeros.
bool make_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint64_t stride_bytes) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {stride_bytes};
    const cuuint32_t box[2] = {64, 128};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int HD>
cudaError_t launch_prefill_hd(const PrefillArgs& a, cudaStream_t stream, unsigned stages) {
    if (stages & PICOATTN_STAGE_PREPARE) {
        const unsigned slot_blocks = (unsigned)((a.hq + 2 * a.hkv + 7) / 8);
        prefill_prep_kernel<HD><<<dim3(slot_blocks, (unsigned)a.n_tok), 256, 0, stream>>>(a);
    }
    if (stages & PICOATTN_STAGE_ATTEND) {
        static bool attr_done = false;
        if (!attr_done) {
            cudaError_t e = cudaFuncSetAttribute(prefill_attn_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 AttnSmem<HD>::kDynBytes);
            if (e != cudaSuccess) return e;
            attr_done = true;
        }
        CUtensorMap mq, mk, mv;
        const uint64_t kvd = (uint64_t)a.kvd;
        const size_t slab = (size_t)a.layer * a.max_seq * a.kvd;
        if (!make_map(&mq, a.q16, (uint64_t)a.hq * HD, (uint64_t)a.n_tok, (uint64_t)a.hq * HD * 2) ||
            !make_map(&mk, a.k_cache + slab, kvd, (uint64_t)(a.start + a.n_tok), kvd * 2) ||
            !make_map(&mv, a.v_cache + slab, kvd, (uint64_t)(a.start + a.n_tok), kvd * 2))
            return cudaErrorInvalidValue;
        dim3 grid((unsigned)a.n_qtiles, (unsigned)a.hq);
        prefill_attn_kernel<HD><<<grid, 192, AttnSmem<HD>::kDynBytes, stream>>>(mq, mk, mv, a);
    }
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_prefill(const PrefillArgs& a, cudaStream_t stream, unsigned stages) {
    return a.hd == 64 ? launch_prefill_hd<64>(a, stream, stages) : launch_prefill_hd<128>(a, stream, stages);
}

size_t prefill_workspace_bytes(const picoattn_config_t& cfg, int n_tok) {
    return kWsHeaderBytes + align_up((size_t)n_tok * cfg.n_heads * cfg.head_dim * 2, 256);
}

}  // namespace picoattn
