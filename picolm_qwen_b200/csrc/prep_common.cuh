// prep_common.cuh -- per-warp processing of one head vector (q, k or v of one
// token), shared by the decode and prefill prep kernels.
//
// Lane l owns elements [V*l, V*l + V), V = HD/32, so every load and store is one
// vector instruction per lane.  The arithmetic is the reference's, operation by
// operation, with every step a single IEEE rounding:
//   RMSNorm (cpp/tensor.hpp:146-176): squares rounded one by one, summed in four
//   interleaved lanes (element i into lane i%4) folded as (l0+l2)+(l1+l3),
//   scale = 1/sqrtf(ss/n + eps), out = (x*scale)*w;
//   RoPE (cpp/tensor.hpp:201-283 NeoX, picolm/tensor.c:247-293 interleaved):
//   (x0, x1) -> (x0*c - x1*s, x0*s + x1*c), products and sum rounded separately.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

#include "device_common.cuh"
#include "picoattn.h"

namespace picoattn {

template <int HD>
struct Vec {
    static constexpr int V = HD / 32;
    float x[V];
};

template <int HD>
__device__ __forceinline__ void vec_load(Vec<HD>& v, const void* src, size_t off, int dtype, int lane) {
    constexpr int V = HD / 32;
    if (dtype == PICOATTN_DTYPE_F16) {
        const __half* p = reinterpret_cast<const __half*>(src) + off + V * lane;
        if constexpr (V == 4) {
            const uint2 u = *reinterpret_cast<const uint2*>(p);
            const __half2 h0 = *reinterpret_cast<const __half2*>(&u.x), h1 = *reinterpret_cast<const __half2*>(&u.y);
            v.x[0] = __low2float(h0), v.x[1] = __high2float(h0), v.x[2] = __low2float(h1), v.x[3] = __high2float(h1);
        } else {
            const __half2 h0 = *reinterpret_cast<const __half2*>(p);
            v.x[0] = __low2float(h0), v.x[1] = __high2float(h0);
        }
    } else {
        const float* p = reinterpret_cast<const float*>(src) + off + V * lane;
        if constexpr (V == 4) {
            const float4 f = *reinterpret_cast<const float4*>(p);
            v.x[0] = f.x, v.x[1] = f.y, v.x[2] = f.z, v.x[3] = f.w;
        } else {
            const float2 f = *reinterpret_cast<const float2*>(p);
            v.x[0] = f.x, v.x[1] = f.y;
        }
    }
}

// The RoPE table entries this lane needs for row `pos` (one vector load each).
template <int HD>
struct RopeLane {
    float c[HD / 32], s[HD / 32];
};

template <int HD>
__device__ __forceinline__ void rope_lane_load(RopeLane<HD>& r, const float* crow, const float* srow, int mode,
                                               int lane) {
    constexpr int V = HD / 32;
    if (mode == PICOATTN_ROPE_NEOX) {
        // element e = V*lane + j pairs with e +- HD/2 (lane +- 16); pair index V*(lane & 15) + j
        const int i = V * (lane & 15);
#pragma unroll
        for (int j = 0; j < V; j++) r.c[j] = crow[i + j], r.s[j] = srow[i + j];
    } else {
        // elements (2i, 2i+1) are both in this lane: pair index V*lane/2 + jp
        const int i = V * lane / 2;
#pragma unroll
        for (int jp = 0; jp < V / 2; jp++) r.c[jp] = crow[i + jp], r.s[jp] = srow[i + jp];
    }
}

template <int HD>
__device__ __forceinline__ void vec_rmsnorm(Vec<HD>& v, const float (&w)[HD / 32], float eps, float* sq, int lane) {
    constexpr int V = HD / 32;
#pragma unroll
    for (int j = 0; j < V; j++) sq[V * lane + j] = __fmul_rn(v.x[j], v.x[j]);
    __syncwarp();
    float part = 0.f;
    if (lane < 4) {
#pragma unroll 8
        for (int d = lane; d < HD; d += 4) part = __fadd_rn(part, sq[d]);
    }
    const float l0 = __shfl_sync(0xffffffffu, part, 0), l1 = __shfl_sync(0xffffffffu, part, 1);
    const float l2 = __shfl_sync(0xffffffffu, part, 2), l3 = __shfl_sync(0xffffffffu, part, 3);
    const float ss = __fadd_rn(__fadd_rn(l0, l2), __fadd_rn(l1, l3));
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)HD), eps)));
#pragma unroll
    for (int j = 0; j < V; j++) v.x[j] = __fmul_rn(__fmul_rn(v.x[j], scale), w[j]);
    __syncwarp();  // sq is reused by the next vector
}

// RMSNorm of up to four vectors at once (norm[u] selects them; w[u] are this
// lane's weights for vector u).  Same arithmetic as vec_rmsnorm: lanes 4u..4u+3
// run the reference's four interleaved lane sums of vector u side by side, lane
// u folds them and computes vector u's scale, so one summation loop and one
// divide/sqrt sequence serve four vectors.  sq: 4*HD floats of shared memory.
// W is float[4][HD/32] (weights per vector) or float[HD/32] (one set for all).
template <int HD>
__device__ __forceinline__ float rms_w(const float (&w)[4][HD / 32], int u, int j) { return w[u][j]; }
template <int HD>
__device__ __forceinline__ float rms_w(const float (&w)[HD / 32], int, int j) { return w[j]; }

template <int HD, class Wt>
__device__ __forceinline__ void vec_rmsnorm4(Vec<HD> (&v)[4], const Wt& w, const bool (&norm)[4], float eps,
                                             float* sq, int lane) {
    constexpr int V = HD / 32;
#pragma unroll
    for (int u = 0; u < 4; u++)
#pragma unroll
        for (int j = 0; j < V; j++) sq[u * HD + V * lane + j] = __fmul_rn(v[u].x[j], v[u].x[j]);
    __syncwarp();
    float part = 0.f;
    if (lane < 16) {
        const float* s = sq + (lane >> 2) * HD;
#pragma unroll 8
        for (int d = lane & 3; d < HD; d += 4) part = __fadd_rn(part, s[d]);
    }
    // lane u < 4 gathers the four lane sums of vector u
    const int src = (lane & 3) * 4;
    const float l0 = __shfl_sync(0xffffffffu, part, src + 0), l1 = __shfl_sync(0xffffffffu, part, src + 1);
    const float l2 = __shfl_sync(0xffffffffu, part, src + 2), l3 = __shfl_sync(0xffffffffu, part, src + 3);
    const float ss = __fadd_rn(__fadd_rn(l0, l2), __fadd_rn(l1, l3));
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)HD), eps)));
#pragma unroll
    for (int u = 0; u < 4; u++) {
        const float su = __shfl_sync(0xffffffffu, scale, u);
        if (norm[u]) {
#pragma unroll
            for (int j = 0; j < V; j++) v[u].x[j] = __fmul_rn(__fmul_rn(v[u].x[j], su), rms_w<HD>(w, u, j));
        }
    }
    __syncwarp();  // sq is reused
}

template <int HD>
__device__ __forceinline__ void vec_rope(Vec<HD>& v, const RopeLane<HD>& r, int mode, int lane) {
    constexpr int V = HD / 32;
    if (mode == PICOATTN_ROPE_NEOX) {
        float p[V];
#pragma unroll
        for (int j = 0; j < V; j++) p[j] = __shfl_xor_sync(0xffffffffu, v.x[j], 16);
        if (lane < 16) {  // first half: x0 = own, x1 = partner
#pragma unroll
            for (int j = 0; j < V; j++) v.x[j] = __fsub_rn(__fmul_rn(v.x[j], r.c[j]), __fmul_rn(p[j], r.s[j]));
        } else {          // second half: x0 = partner, x1 = own
#pragma unroll
            for (int j = 0; j < V; j++) v.x[j] = __fadd_rn(__fmul_rn(p[j], r.s[j]), __fmul_rn(v.x[j], r.c[j]));
        }
    } else {
#pragma unroll
        for (int jp = 0; jp < V / 2; jp++) {
            const float x0 = v.x[2 * jp], x1 = v.x[2 * jp + 1];
            v.x[2 * jp] = __fsub_rn(__fmul_rn(x0, r.c[jp]), __fmul_rn(x1, r.s[jp]));
            v.x[2 * jp + 1] = __fadd_rn(__fmul_rn(x0, r.s[jp]), __fmul_rn(x1, r.c[jp]));
        }
    }
}

// Stores: fp32, fp16 (round to nearest even) scaled, or the reference's fp16 bits.
template <int HD>
__device__ __forceinline__ void vec_store_f32(const Vec<HD>& v, float* dst, int lane) {
    constexpr int V = HD / 32;
    if constexpr (V == 4) *reinterpret_cast<float4*>(dst + V * lane) = make_float4(v.x[0], v.x[1], v.x[2], v.x[3]);
    else *reinterpret_cast<float2*>(dst + V * lane) = make_float2(v.x[0], v.x[1]);
}

template <int HD>
__device__ __forceinline__ void vec_store_h16_scaled(const Vec<HD>& v, __half* dst, float scale, int lane) {
    constexpr int V = HD / 32;
    if constexpr (V == 4) {
        uint2 u;
        u.x = pack_half2(v.x[0] * scale, v.x[1] * scale);
        u.y = pack_half2(v.x[2] * scale, v.x[3] * scale);
        *reinterpret_cast<uint2*>(dst + V * lane) = u;
    } else {
        *reinterpret_cast<uint32_t*>(dst + V * lane) = pack_half2(v.x[0] * scale, v.x[1] * scale);
    }
}

template <int HD>
__device__ __forceinline__ void vec_store_ref16(const Vec<HD>& v, uint16_t* dst, int lane) {
    constexpr int V = HD / 32;
    if constexpr (V == 4) {
        uint2 u;
        u.x = (uint32_t)f32_to_f16_ref(v.x[0]) | ((uint32_t)f32_to_f16_ref(v.x[1]) << 16);
        u.y = (uint32_t)f32_to_f16_ref(v.x[2]) | ((uint32_t)f32_to_f16_ref(v.x[3]) << 16);
        *reinterpret_cast<uint2*>(dst + V * lane) = u;
    } else {
        *reinterpret_cast<uint32_t*>(dst + V * lane) =
            (uint32_t)f32_to_f16_ref(v.x[0]) | ((uint32_t)f32_to_f16_ref(v.x[1]) << 16);
    }
}

}  // namespace picoattn
