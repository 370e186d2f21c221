// matvec.cu -- the projections around the attention step on the GPU:
// out[v][d] = W[d, :] . x[v, :] (+ bias[d]) for the weight formats the C++
// engine multiplies with (TensorOps::matmul_bias, cpp/tensor.hpp:110-143;
// block layouts cpp/quant.hpp:33-74, dequantisation cpp/quant.hpp:175-295).
//
// One warp per output row.  The warp stages the bytes of 32 consecutive
// 32-weight units of its row into shared memory with coalesced 4-byte loads,
// then each lane turns one unit into 32 fp32 weights with the same float
// operations as the reference's dequantize_row_* (each product and difference
// rounded on its own: no contraction, so the weights are bit-identical) and
// accumulates their products with x in fp32.  The dot product's summation
// order is the GPU's own (the reference sums in SSE lanes), so results agree
// to rounding, not bit for bit.  Several matrices that read the same x (q, k
// and v) go out in one launch, their rows dealt to warps in one sequence.
// Bound by HBM: every weight byte is read once per group of NV vectors.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "device_common.cuh"
#include "picoattn_internal.h"

namespace picoattn {

namespace {

constexpr int kMvWarps = 8;           // warps per block
constexpr int kMvChunkWords = 1024;   // staged bytes per warp: 32 units of F32 = 4 KB

__device__ __forceinline__ float half_bits(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t lds16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }

// get_scale_min_k4, cpp/quant.hpp:210-218: the 6-bit scale and min of
// sub-block j of a Q4_K block.
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t* q, int& sc, int& mn) {
    if (j < 4) {
        sc = q[j] & 63;
        mn = q[j + 4] & 63;
    } else {
        sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// The 32 weights of unit `sub` of the block at `blk` (shared memory).
__device__ __forceinline__ void decode_unit(int type, const uint8_t* blk, int sub, float (&w)[32]) {
    switch (type) {
        case PICOATTN_WT_F32:
#pragma unroll
            for (int i = 0; i < 32; i++) w[i] = reinterpret_cast<const float*>(blk)[i];
            break;
        case PICOATTN_WT_F16:
#pragma unroll
            for (int i = 0; i < 32; i++) w[i] = half_bits(lds16(blk + 2 * i));
            break;
        case PICOATTN_WT_Q4_0: {  // dequantize_row_q4_0, cpp/quant.hpp:197-207
            const float d = half_bits(lds16(blk));
#pragma unroll
            for (int i = 0; i < 16; i++) {
                const int b = blk[2 + i];
                w[i] = __fmul_rn(d, (float)(b & 0xF) - 8.0f);
                w[i + 16] = __fmul_rn(d, (float)(b >> 4) - 8.0f);
            }
            break;
        }
        case PICOATTN_WT_Q8_0: {  // dequantize_row_q8_0, cpp/quant.hpp:187-195
            const float d = half_bits(lds16(blk));
#pragma unroll
            for (int i = 0; i < 32; i++) w[i] = __fmul_rn(d, (float)(int8_t)blk[2 + i]);
            break;
        }
        case PICOATTN_WT_Q4_K: {  // dequantize_row_q4_K, cpp/quant.hpp:220-251
            // unit sub = 2*j + h: pair j of 32 quant bytes, low (h = 0) or high nibbles
            const float d = half_bits(lds16(blk)), dmin = half_bits(lds16(blk + 2));
            int sc, mn;
            scale_min_k4(sub, blk + 4, sc, mn);
            const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)mn);
            const uint8_t* q = blk + 16 + 32 * (sub >> 1);
            const int sh = (sub & 1) * 4;
#pragma unroll
            for (int l = 0; l < 32; l++) w[l] = __fsub_rn(__fmul_rn(d1, (float)((q[l] >> sh) & 0xF)), m1);
            break;
        }
        case PICOATTN_WT_Q6_K: {  // dequantize_row_q6_K, cpp/quant.hpp:253-281
            // unit sub = 4*c + qq: chunk c of 128 weights, quarter qq
            const int c = sub >> 2, qq = sub & 3;
            const uint8_t* ql = blk + 64 * c + (qq & 1) * 32;
            const uint8_t* qh = blk + 128 + 32 * c;
            const int8_t* scl = reinterpret_cast<const int8_t*>(blk + 192) + 8 * c + 2 * qq;
            const float d = half_bits(lds16(blk + 208));
            const int lsh = (qq >> 1) * 4, hsh = 2 * qq;
#pragma unroll
            for (int l = 0; l < 32; l++) {
                const int q = (((ql[l] >> lsh) & 0xF) | (((qh[l] >> hsh) & 3) << 4)) - 32;
                w[l] = __fmul_rn(__fmul_rn(d, (float)scl[l / 16]), (float)q);
            }
            break;
        }
        default:
#pragma unroll
            for (int i = 0; i < 32; i++) w[i] = 0.f;
    }
}

__device__ __forceinline__ int units_per_block(int type) {
    return (type == PICOATTN_WT_Q4_K || type == PICOATTN_WT_Q6_K) ? 8 : 1;
}

// NV vectors per pass over a row: the weights are decoded once per pass.
template <int NV>
__global__ void __launch_bounds__(kMvWarps * 32, 2) matvec_kernel(MatvecArgs a) {
    __shared__ __align__(16) uint32_t stage[kMvWarps][kMvChunkWords + 4];
    // The next kernel may launch now; inputs are read after the kernel before
    // this one completed (every CTA waits before it exits, see pdl_wait).
    pdl_trigger();
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint32_t* st = stage[warp];
    const int n_units = a.n_in / 32;
    for (int r = blockIdx.x * kMvWarps + warp; r < a.rows_total; r += gridDim.x * kMvWarps) {
        // the matrix holding global row r (selected, not indexed: the parts stay
        // in the parameter space)
        int row = r;
        const bool in1 = a.n_parts > 1 && row >= a.part[0].n_out;
        if (in1) row -= a.part[0].n_out;
        const bool in2 = in1 && a.n_parts > 2 && row >= a.part[1].n_out;
        if (in2) row -= a.part[1].n_out;
        const MatvecPart P = in2 ? a.part[2] : (in1 ? a.part[1] : a.part[0]);
        const int type = P.type, upb = units_per_block(type), qsz = (int)(P.block_bytes);
        const uint8_t* rowp = P.w + (size_t)row * P.row_bytes;
        for (int v0 = 0; v0 < a.n_vec; v0 += NV) {
            float acc[NV];
#pragma unroll
            for (int v = 0; v < NV; v++) acc[v] = 0.f;
            for (int u0 = 0; u0 < n_units; u0 += 32) {
                // stage blocks [b0, b1) that hold units [u0, u0 + 32)
                const int b0 = u0 / upb, b1 = (min(n_units, u0 + 32) + upb - 1) / upb;
                const uintptr_t g0 = (uintptr_t)(rowp + (size_t)b0 * qsz), g1 = (uintptr_t)(rowp + (size_t)b1 * qsz);
                const uintptr_t a0 = g0 & ~(uintptr_t)3;
                const int nwords = (int)((g1 - a0) >> 2), tail = (int)((g1 - a0) & 3);
                __syncwarp();  // the previous chunk's reads are done
                for (int i = lane; i < nwords; i += 32) st[i] = __ldg(reinterpret_cast<const uint32_t*>(a0) + i);
                if (tail && lane == 0) {  // the last bytes of the matrix may end inside a word
                    uint32_t t = 0;
                    for (int k = 0; k < tail; k++) t |= (uint32_t)__ldg(reinterpret_cast<const uint8_t*>(a0) + 4 * nwords + k) << (8 * k);
                    st[nwords] = t;
                }
                __syncwarp();
                const int u = u0 + lane;
                if (u < n_units) {
                    const int k = u - b0 * upb;
                    float w[32];
                    decode_unit(type, reinterpret_cast<const uint8_t*>(st) + (g0 - a0) + (size_t)(k / upb) * qsz,
                                k % upb, w);
#pragma unroll
                    for (int v = 0; v < NV; v++) {
                        if (v0 + v < a.n_vec) {
                            const float4* xv = reinterpret_cast<const float4*>(a.x + (size_t)(v0 + v) * a.n_in + 32 * u);
#pragma unroll
                            for (int g = 0; g < 8; g++) {
                                const float4 xx = __ldg(xv + g);
                                acc[v] = fmaf(w[4 * g], xx.x, acc[v]);
                                acc[v] = fmaf(w[4 * g + 1], xx.y, acc[v]);
                                acc[v] = fmaf(w[4 * g + 2], xx.z, acc[v]);
                                acc[v] = fmaf(w[4 * g + 3], xx.w, acc[v]);
                            }
                        }
                    }
                }
            }
#pragma unroll
            for (int v = 0; v < NV; v++) {
#pragma unroll
                for (int o = 16; o; o >>= 1) acc[v] += __shfl_xor_sync(0xffffffffu, acc[v], o);
            }
            if (lane == 0) {
#pragma unroll
                for (int v = 0; v < NV; v++) {
                    if (v0 + v < a.n_vec) {
                        // matmul, then the bias added (vec_add), then the residual
                        float y = acc[v];
                        if (P.bias) y = __fadd_rn(y, P.bias[row]);
                        float* o = P.out + (size_t)(v0 + v) * P.out_stride + row;
                        *o = a.accumulate ? __fadd_rn(*o, y) : y;
                    }
                }
            }
        }
    }
}

}  // namespace

int weight_block_elems(int type) {
    switch (type) {
        case PICOATTN_WT_F32: case PICOATTN_WT_F16: return 32;
        case PICOATTN_WT_Q4_0: case PICOATTN_WT_Q8_0: return 32;
        case PICOATTN_WT_Q4_K: case PICOATTN_WT_Q6_K: return 256;
        default: return 0;
    }
}

int weight_block_bytes(int type) {
    switch (type) {
        case PICOATTN_WT_F32: return 128;  // 32 elements (the unit the kernel stages)
        case PICOATTN_WT_F16: return 64;
        case PICOATTN_WT_Q4_0: return 18;
        case PICOATTN_WT_Q8_0: return 34;
        case PICOATTN_WT_Q4_K: return 144;
        case PICOATTN_WT_Q6_K: return 210;
        default: return 0;
    }
}

bool matvec_part(int type, const void* w, const float* bias, int n_in, int n_out, float* out, size_t out_stride,
                 MatvecPart* p) {
    const int be = weight_block_elems(type);
    if (be == 0 || n_in <= 0 || n_in % be != 0 || n_out <= 0 || !w || !out) return false;
    if (((uintptr_t)w & 3u) != 0) return false;
    p->w = static_cast<const uint8_t*>(w);
    p->bias = bias;
    p->out = out;
    p->out_stride = out_stride;
    p->type = type;
    p->n_out = n_out;
    // the kernel's block: 32 elements for F32/F16 (units of its own), else the format's block
    p->block_bytes = weight_block_bytes(type);
    p->row_bytes = (size_t)(n_in / (type == PICOATTN_WT_Q4_K || type == PICOATTN_WT_Q6_K ? 256 : 32)) * p->block_bytes;
    return true;
}

cudaError_t launch_matvec(const MatvecArgs& a, cudaStream_t stream) {
    const int sms = device_sm_count();
    const long long want = ((long long)a.rows_total + kMvWarps - 1) / kMvWarps;
    const int grid = (int)std::min<long long>(want, (long long)sms * 8);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)std::max(1, grid));
    cfg.blockDim = dim3(kMvWarps * 32);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (a.n_vec == 1) return cudaLaunchKernelEx(&cfg, matvec_kernel<1>, a);
    if (a.n_vec == 2) return cudaLaunchKernelEx(&cfg, matvec_kernel<2>, a);
    return cudaLaunchKernelEx(&cfg, matvec_kernel<4>, a);
}

}  // namespace picoattn
