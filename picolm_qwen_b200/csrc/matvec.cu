// matvec.cu -- the projections around the attention step on the GPU:
// out[v][d] = W[d, :] . x[v, :] (+ bias[d]) for the weight formats the C++
// engine multiplies with (TensorOps::matmul_bias, cpp/tensor.hpp:110-143;
// block layouts cpp/quant.hpp:33-74, dequantisation cpp/quant.hpp:175-295).
//
// Work is cut into chunks: the bytes of 32 consecutive 32-weight units of one
// row, copied into a warp's shared-memory slot with asynchronous copies, a few
// chunks ahead of the one being used.  Each lane turns one unit into 32 fp32
// weights with the same float operations as the reference's dequantize_row_*
// (each product and difference rounded on its own: no contraction, so the
// weights are bit-identical) and accumulates their products with x in fp32.
// The dot product's summation order is the GPU's own (the reference sums in
// SSE lanes), so results agree to rounding, not bit for bit.  One vector of
// Q4_K, Q6_K or Q8_0 weights (the model formats that matter) goes to the
// streaming kernels below (matvecq_direct_kernel, matvecq_kernel: x in shared
// memory, the dequantisation factored per scale group); one vector of the
// other formats (matvec1_kernel): a block per group of four consecutive rows,
// its warps taking the group's chunk steps and holding their x values in
// registers for the four rows.  Several vectors, or F32 weights
// (matvec_kernel): a warp per row.  Several matrices that read the same x (q,
// k and v) go out in one launch.  Every weight byte is read once per pass over
// the vectors; the kernels are bound by instruction issue, not yet by HBM.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "device_common.cuh"
#include "picoattn_internal.h"

namespace picoattn {

namespace {

constexpr int kMvWarps = 8;           // warps per block
constexpr int kMvRingWords = 2064;    // per warp: DEPTH chunk slots of (2064 / DEPTH) words
constexpr size_t kMvSmem = (size_t)kMvWarps * kMvRingWords * 4;
// A chunk (32 units) of F32 weights is 4 KB, of F16 2 KB, of the block formats
// at most 1088 B: F32 gets two 4 KB slots, the rest four 2 KB slots (each slot
// with spare words for the 4-byte-boundary start and the unaligned reads).

// 4 bytes at any byte offset of a staged chunk (two aligned reads, a funnel
// shift; the buffer has a spare word at its end).
__device__ __forceinline__ uint32_t ld4(const uint8_t* p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~(uintptr_t)3);
    return __funnelshift_r(w[0], w[1], (uint32_t)(a & 3) * 8u);
}

__device__ __forceinline__ float half_at(const uint8_t* p, int hi) {
    const uint32_t v = ld4(p);
    return __half2float(__ushort_as_half((uint16_t)(hi ? v >> 16 : v & 0xFFFF)));
}

// Four bytes (0..255 each) of v as exact floats 2^23 + b, in two pairs; the
// caller subtracts 2^23 (+ an offset) with one packed subtraction per pair,
// which is exact, so the result is the integer (minus the offset) exactly,
// as the reference's (float) conversions give.
__device__ __forceinline__ void bytes_biased(uint32_t v, uint64_t& p01, uint64_t& p23) {
    p01 = f2_pack(__uint_as_float(__byte_perm(v, 0x4B000000u, 0x7540)),
                  __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7541)));
    p23 = f2_pack(__uint_as_float(__byte_perm(v, 0x4B000000u, 0x7542)),
                  __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7543)));
}

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

// acc[v] += w . x[v] over the 32 weights of unit `sub` of the block at `blk`
// (a staged chunk), whose x starts at xu.  The weights are the reference's
// dequantize_row_* values exactly: every product and difference rounded on its
// own (packed f32x2 operations round each lane like the scalar ones).
// xq(v, j): elements 4j..4j+3 of vector v's 32 x values for this unit.
template <int NV, class XQ>
__device__ __forceinline__ void unit_dot(int type, const uint8_t* blk, int sub, XQ xq, int nv, uint64_t (&acc)[NV]) {
    // fma4(j, ...): the weights 4j..4j+3 as two pairs
    auto fma4 = [&](int j, uint64_t w01, uint64_t w23) {
#pragma unroll
        for (int v = 0; v < NV; v++) {
            if (v < nv) {
                const float4 x = xq(v, j);
                acc[v] = f2_fma(w01, f2_pack(x.x, x.y), acc[v]);
                acc[v] = f2_fma(w23, f2_pack(x.z, x.w), acc[v]);
            }
        }
    };
    switch (type) {
        case PICOATTN_WT_F32:
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const float4 w = *reinterpret_cast<const float4*>(blk + 16 * j);
                fma4(j, f2_pack(w.x, w.y), f2_pack(w.z, w.w));
            }
            break;
        case PICOATTN_WT_F16:
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const uint32_t a = ld4(blk + 8 * j), b = ld4(blk + 8 * j + 4);
                const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&a));
                const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&b));
                fma4(j, f2_pack(f0.x, f0.y), f2_pack(f1.x, f1.y));
            }
            break;
        case PICOATTN_WT_Q4_0: {  // dequantize_row_q4_0, cpp/quant.hpp:197-207: d * ((float)nib - 8)
            const float d = half_at(blk, 0);
            const uint64_t dd = f2_pack(d, d), off = f2_pack(8388616.f, 8388616.f);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const uint32_t v = ld4(blk + 2 + 4 * j);
                uint64_t a, b;
                bytes_biased(v & 0x0F0F0F0Fu, a, b);  // weights 4j.. (low nibbles)
                fma4(j, f2_mul(dd, f2_sub(a, off)), f2_mul(dd, f2_sub(b, off)));
                bytes_biased((v >> 4) & 0x0F0F0F0Fu, a, b);  // weights 16+4j.. (high nibbles)
                fma4(4 + j, f2_mul(dd, f2_sub(a, off)), f2_mul(dd, f2_sub(b, off)));
            }
            break;
        }
        case PICOATTN_WT_Q8_0: {  // dequantize_row_q8_0, cpp/quant.hpp:187-195: d * (float)q
            const float d = half_at(blk, 0);
            const uint64_t dd = f2_pack(d, d), off = f2_pack(8388736.f, 8388736.f);  // 2^23 + 128
#pragma unroll
            for (int j = 0; j < 8; j++) {
                uint64_t a, b;
                bytes_biased(ld4(blk + 2 + 4 * j) ^ 0x80808080u, a, b);
                fma4(j, f2_mul(dd, f2_sub(a, off)), f2_mul(dd, f2_sub(b, off)));
            }
            break;
        }
        case PICOATTN_WT_Q4_K: {  // dequantize_row_q4_K, cpp/quant.hpp:220-251: d1 * q - m1
            // unit sub = 2*j + h: pair j of 32 quant bytes, low (h = 0) or high nibbles
            const uint32_t h = ld4(blk);
            const float d = __half2float(__ushort_as_half((uint16_t)(h & 0xFFFF)));
            const float dmin = __half2float(__ushort_as_half((uint16_t)(h >> 16)));
            int sc, mn;
            scale_min_k4(sub, blk + 4, sc, mn);
            const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)mn);
            const uint64_t dd = f2_pack(d1, d1), mm = f2_pack(m1, m1), off = f2_pack(8388608.f, 8388608.f);
            const uint8_t* q = blk + 16 + 32 * (sub >> 1);
            const uint32_t sh = (sub & 1) * 4;
            uint32_t qw[8];
            if ((reinterpret_cast<uintptr_t>(q) & 15u) == 0) {  // blocks 16-byte aligned: two 16-byte reads
                const uint4 q0 = *reinterpret_cast<const uint4*>(q), q1 = *reinterpret_cast<const uint4*>(q + 16);
                qw[0] = q0.x, qw[1] = q0.y, qw[2] = q0.z, qw[3] = q0.w;
                qw[4] = q1.x, qw[5] = q1.y, qw[6] = q1.z, qw[7] = q1.w;
            } else {
#pragma unroll
                for (int j = 0; j < 8; j++) qw[j] = ld4(q + 4 * j);
            }
#pragma unroll
            for (int j = 0; j < 8; j++) {
                uint64_t a, b;
                bytes_biased((qw[j] >> sh) & 0x0F0F0F0Fu, a, b);
                fma4(j, f2_sub(f2_mul(dd, f2_sub(a, off)), mm), f2_sub(f2_mul(dd, f2_sub(b, off)), mm));
            }
            break;
        }
        case PICOATTN_WT_Q6_K: {  // dequantize_row_q6_K, cpp/quant.hpp:253-281: d * sc * (q - 32)
            // unit sub = 4*c + qq: chunk c of 128 weights, quarter qq
            const int c = sub >> 2, qq = sub & 3;
            const uint8_t* ql = blk + 64 * c + (qq & 1) * 32;
            const uint8_t* qh = blk + 128 + 32 * c;
            const int8_t* scl = reinterpret_cast<const int8_t*>(blk + 192) + 8 * c + 2 * qq;
            const float d = half_at(blk + 208, 0);
            const float ds0 = __fmul_rn(d, (float)scl[0]), ds1 = __fmul_rn(d, (float)scl[1]);
            const uint32_t lsh = (qq >> 1) * 4, hsh = 2 * qq;
            const uint64_t off = f2_pack(8388640.f, 8388640.f);  // 2^23 + 32
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const uint32_t qv = ((ld4(ql + 4 * j) >> lsh) & 0x0F0F0F0Fu) | (((ld4(qh + 4 * j) >> hsh) & 0x03030303u) << 4);
                const float ds = j < 4 ? ds0 : ds1;  // weights 0..15 and 16..31
                const uint64_t dd = f2_pack(ds, ds);
                uint64_t a, b;
                bytes_biased(qv, a, b);
                fma4(j, f2_mul(dd, f2_sub(a, off)), f2_mul(dd, f2_sub(b, off)));
            }
            break;
        }
        default:
            break;
    }
}

// log2 of the 32-weight units per block (8 for Q4_K and Q6_K, else 1): the
// chunk arithmetic shifts and masks instead of dividing by a run-time value (a
// 32-bit division is a long instruction sequence)
__device__ __forceinline__ int units_per_block_log2(int type) {
    return (type == PICOATTN_WT_Q4_K || type == PICOATTN_WT_Q6_K) ? 3 : 0;
}

// The matrix (of up to three) that holds global row r, and r's row in it.
__device__ __forceinline__ MatvecPart part_of(const MatvecArgs& a, int r, int& row) {
    row = r;
    const bool in1 = a.n_parts > 1 && row >= a.part[0].n_out;
    if (in1) row -= a.part[0].n_out;
    const bool in2 = in1 && a.n_parts > 2 && row >= a.part[1].n_out;
    if (in2) row -= a.part[1].n_out;
    return in2 ? a.part[2] : (in1 ? a.part[1] : a.part[0]);
}

// Every warp walks its rows chunk by chunk (32 units of 32 weights); chunk j+1
// is copied into the warp's other buffer (cp.async, 4-byte words) while chunk j
// is decoded, so a row costs about one memory round trip, not one per chunk.
template <int NV, int DEPTH>
__global__ void __launch_bounds__(kMvWarps * 32, 2) matvec_kernel(MatvecArgs a) {
    constexpr int kSlotWords = kMvRingWords / DEPTH;  // 1032 or 516 words: 16-byte multiples
    static_assert(kSlotWords % 4 == 0, "16-byte aligned slots");
    extern __shared__ __align__(16) uint32_t mv_smem[];
    // The next kernel may launch now; inputs are read after the kernel before
    // this one completed (every CTA waits before it exits, see pdl_wait).
    pdl_trigger();
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint32_t* bufs = mv_smem + (size_t)warp * kMvRingWords;
    const int n_units = a.n_in / 32, cpr = (n_units + 31) / 32;  // chunks per row
    const int gw = blockIdx.x * kMvWarps + warp, nw = gridDim.x * kMvWarps;
    const int my_rows = gw < a.rows_total ? (a.rows_total - 1 - gw) / nw + 1 : 0;
    const int n_chunks = my_rows * cpr;
    // chunk j: row gw + (j / cpr) * nw, units from (j % cpr) * 32; its bytes
    // [g0, g1) staged from the 4-byte boundary a0 <= g0
    auto chunk = [&](int j, MatvecPart& P, int& row, int& b0, uintptr_t& g0, uintptr_t& a0, int& nwords,
                     int& tail) {
        P = part_of(a, gw + (j / cpr) * nw, row);
        const int lu = units_per_block_log2(P.type), u0 = (j % cpr) * 32;
        b0 = u0 >> lu;
        const int b1 = (min(n_units, u0 + 32) + (1 << lu) - 1) >> lu;
        const uint8_t* rowp = P.w + (size_t)row * P.row_bytes;
        g0 = reinterpret_cast<uintptr_t>(rowp + (size_t)b0 * P.block_bytes);
        const uintptr_t g1 = reinterpret_cast<uintptr_t>(rowp + (size_t)b1 * P.block_bytes);
        a0 = g0 & ~(uintptr_t)3;
        nwords = (int)((g1 - a0) >> 2);
        tail = (int)((g1 - a0) & 3);
    };
    auto issue = [&](int j) {
        if (j < n_chunks) {
            MatvecPart P;
            int row, b0, nwords, tail;
            uintptr_t g0, a0;
            chunk(j, P, row, b0, g0, a0, nwords, tail);
            uint32_t* dst = bufs + (j % DEPTH) * kSlotWords;
            for (int i = lane; i < nwords; i += 32) cp_async4(dst + i, reinterpret_cast<const uint32_t*>(a0) + i);
            if (tail && lane == 0) {  // the matrix may end inside a word: no read past it
                uint32_t t = 0;
                for (int k = 0; k < tail; k++)
                    t |= (uint32_t)__ldg(reinterpret_cast<const uint8_t*>(a0) + 4 * nwords + k) << (8 * k);
                dst[nwords] = t;
            }
        }
        cp_async_commit();
    };
    for (int v0 = 0; v0 < a.n_vec; v0 += NV) {
        const int nv = min(NV, a.n_vec - v0);
        uint64_t acc[NV];
#pragma unroll
        for (int v = 0; v < NV; v++) acc[v] = 0ull;
        for (int j = 0; j < DEPTH - 1; j++) issue(j);
        for (int j = 0; j < n_chunks; j++) {
            issue(j + DEPTH - 1);  // into the slot chunk j - 1 used
            cp_async_wait<DEPTH - 1>();
            __syncwarp();  // chunk j is in its slot (every lane's copies and the tail)
            MatvecPart P;
            int row, b0, nwords, tail;
            uintptr_t g0, a0;
            chunk(j, P, row, b0, g0, a0, nwords, tail);
            const int lu = units_per_block_log2(P.type), u = (j % cpr) * 32 + lane;
            if (u < n_units) {
                const int k = u - (b0 << lu);
                const uint8_t* blk = reinterpret_cast<const uint8_t*>(bufs + (j % DEPTH) * kSlotWords) + (g0 - a0) +
                                     (size_t)(k >> lu) * P.block_bytes;
                const float* xu = a.x + (size_t)v0 * a.n_in + 32 * u;
                unit_dot<NV>(P.type, blk, k & ((1 << lu) - 1),
                             [&](int v, int jj) {
                                 return __ldg(reinterpret_cast<const float4*>(xu + (size_t)v * a.n_in) + jj);
                             },
                             nv, acc);
            }
            __syncwarp();  // the slot is read before chunk j + DEPTH overwrites it
            if (j % cpr == cpr - 1) {  // the row is done
                float y[NV];
#pragma unroll
                for (int v = 0; v < NV; v++) {
                    float lo, hi;
                    f2_unpack(acc[v], lo, hi);
                    y[v] = lo + hi;
#pragma unroll
                    for (int o = 16; o; o >>= 1) y[v] += __shfl_xor_sync(0xffffffffu, y[v], o);
                    acc[v] = 0ull;
                }
                if (lane == 0) {
#pragma unroll
                    for (int v = 0; v < NV; v++) {
                        if (v < nv) {
                            // matmul, then the bias added (vec_add), then the residual
                            float yv = y[v];
                            if (P.bias) yv = __fadd_rn(yv, P.bias[row]);
                            float* o = P.out + (size_t)(v0 + v) * P.out_stride + row;
                            *o = a.accumulate ? __fadd_rn(*o, yv) : yv;
                        }
                    }
                }
            }
        }
        cp_async_wait<0>();
        __syncwarp();
    }
}

// One vector: a block takes a group of kMvRows consecutive rows (one matrix:
// the host checks that every matrix's row count is a multiple of kMvRows) and
// its warps take the group's chunk steps (32 units of 32 weights) in turn.  At
// each of its steps a warp loads its lanes' units of x into registers once and
// applies them to the group's rows (x traffic through L1 falls kMvRows-fold:
// in the row-at-a-time order it bounded the kernel); the warps' partial sums
// are added in warp order through shared memory, so results do not depend on
// timing.  Many warps per row keep enough copies in flight even for the
// 3,584-row matrices of a decode layer.  Chunk slots as in matvec_kernel
// (block formats and F16 only: F32 chunks need the larger slots).
constexpr int kMvRows = 4;
// warps per block of matvec1_kernel: at most four, so that the register bound
// below lets five or more blocks share an SM (more copies in flight)
constexpr int kMv1Warps = 4;

template <int DEPTH>
__global__ void __launch_bounds__(kMv1Warps * 32, 5) matvec1_kernel(MatvecArgs a) {
    constexpr int kSlotWords = kMvRingWords / DEPTH;
    extern __shared__ __align__(16) uint32_t mv_smem[];
    __shared__ float part_sums[kMv1Warps][kMvRows];
    pdl_trigger();
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwb = blockDim.x >> 5;
    uint32_t* bufs = mv_smem + (size_t)warp * kMvRingWords;
    const int n_units = a.n_in / 32, cpr = (n_units + 31) / 32;
    const int n_groups = a.rows_total / kMvRows;
    for (int grp = blockIdx.x; grp < n_groups; grp += gridDim.x) {
        int row0;
        const MatvecPart P = part_of(a, grp * kMvRows, row0);
        const int lu = units_per_block_log2(P.type), bb = P.block_bytes;
        const uint8_t* base = P.w + (size_t)row0 * P.row_bytes;
        // this warp's steps: warp, warp + nwb, ...; chunk c = (its k-th step, row c % kMvRows)
        const int my_steps = warp < cpr ? (cpr - 1 - warp) / nwb + 1 : 0;
        const int n_chunks = my_steps * kMvRows;
        auto span = [&](int c, int& b0, uintptr_t& g0, uintptr_t& a0, int& nwords, int& tail) {
            const int u0 = (warp + (c / kMvRows) * nwb) * 32;
            b0 = u0 >> lu;
            const int b1 = (min(n_units, u0 + 32) + (1 << lu) - 1) >> lu;
            const uint8_t* rowp = base + (size_t)(c % kMvRows) * P.row_bytes;
            g0 = reinterpret_cast<uintptr_t>(rowp + (size_t)b0 * bb);
            const uintptr_t g1 = reinterpret_cast<uintptr_t>(rowp + (size_t)b1 * bb);
            a0 = g0 & ~(uintptr_t)3;
            nwords = (int)((g1 - a0) >> 2);
            tail = (int)((g1 - a0) & 3);
        };
        auto issue = [&](int c) {
            if (c < n_chunks) {
                int b0, nwords, tail;
                uintptr_t g0, a0;
                span(c, b0, g0, a0, nwords, tail);
                uint32_t* dst = bufs + (c % DEPTH) * kSlotWords;
                // 16-byte copies where the chunk starts on a 16-byte boundary (the
                // slots do), 4-byte copies for the rest
                const int n16 = (a0 & 15u) == 0 ? nwords >> 2 : 0;
                for (int i = lane; i < n16; i += 32) cp_async16(dst + 4 * i, reinterpret_cast<const uint32_t*>(a0) + 4 * i);
                for (int i = 4 * n16 + lane; i < nwords; i += 32)
                    cp_async4(dst + i, reinterpret_cast<const uint32_t*>(a0) + i);
                if (tail && lane == 0) {  // the matrix may end inside a word: no read past it
                    uint32_t t = 0;
                    for (int k = 0; k < tail; k++)
                        t |= (uint32_t)__ldg(reinterpret_cast<const uint8_t*>(a0) + 4 * nwords + k) << (8 * k);
                    dst[nwords] = t;
                }
            }
            cp_async_commit();
        };
        // the group's row sums, rotated one place per row so that the current
        // row's is always acc[0]: the row loop stays rolled (one copy of the
        // decode in the instruction cache, not one per row) without indexing
        // registers at run time
        uint64_t acc[kMvRows];
#pragma unroll
        for (int r = 0; r < kMvRows; r++) acc[r] = 0ull;
        float4 xr[8];  // this lane's unit of x at the current step
        for (int c = 0; c < DEPTH - 1; c++) issue(c);
        for (int k = 0; k < my_steps; k++) {
            const int u = (warp + k * nwb) * 32 + lane;
            if (u < n_units) {
#pragma unroll
                for (int jj = 0; jj < 8; jj++) xr[jj] = __ldg(reinterpret_cast<const float4*>(a.x + 32 * u) + jj);
            }
#pragma unroll 1
            for (int r = 0; r < kMvRows; r++) {
                const int c = k * kMvRows + r;
                issue(c + DEPTH - 1);
                cp_async_wait<DEPTH - 1>();
                __syncwarp();  // chunk c is in its slot (every lane's copies and the tail)
                if (u < n_units) {
                    int b0, nwords, tail;
                    uintptr_t g0, a0;
                    span(c, b0, g0, a0, nwords, tail);
                    const int ku = u - (b0 << lu);
                    const uint8_t* blk = reinterpret_cast<const uint8_t*>(bufs + (c % DEPTH) * kSlotWords) +
                                         (g0 - a0) + (size_t)(ku >> lu) * bb;
                    uint64_t one[1] = {acc[0]};
                    unit_dot<1>(P.type, blk, ku & ((1 << lu) - 1), [&](int, int jj) { return xr[jj]; }, 1, one);
                    acc[0] = one[0];
                }
                const uint64_t t = acc[0];
#pragma unroll
                for (int q = 0; q + 1 < kMvRows; q++) acc[q] = acc[q + 1];
                acc[kMvRows - 1] = t;
                __syncwarp();  // the slot is read before chunk c + DEPTH overwrites it
            }
        }
        cp_async_wait<0>();
#pragma unroll
        for (int r = 0; r < kMvRows; r++) {
            float lo, hi;
            f2_unpack(acc[r], lo, hi);
            float y = lo + hi;
#pragma unroll
            for (int o = 16; o; o >>= 1) y += __shfl_xor_sync(0xffffffffu, y, o);
            if (lane == 0) part_sums[warp][r] = y;
        }
        __syncthreads();  // every warp's partial sums
        if (warp == 0 && lane < kMvRows) {
            float y = part_sums[0][lane];
            for (int w2 = 1; w2 < nwb; w2++) y += part_sums[w2][lane];
            // matmul, then the bias added (vec_add), then the residual
            const int row = row0 + lane;
            if (P.bias) y = __fadd_rn(y, P.bias[row]);
            float* o = P.out + row;
            *o = a.accumulate ? __fadd_rn(*o, y) : y;
        }
        __syncthreads();  // part_sums and the slots are free for the next group
    }
}

// ---------------------------------------------------------------------------
// One vector, block formats Q4_K, Q6_K and Q8_0: matvecq_kernel
// ---------------------------------------------------------------------------
//
// A warp takes a row at a time and the row's "items" 32 at a time (a round):
// a Q4_K block's 32-byte quant chunk = 64 weights, a Q6_K half block = 128
// weights, a pair of Q8_0 blocks = 64 weights; lane i decodes item i of the
// round.  The round's bytes (contiguous in the row) arrive in the warp's
// shared-memory buffer by 16-byte asynchronous copies, consecutive lanes on
// consecutive 16 bytes (whole sectors, whatever the format's alignment), one
// round ahead of the one being decoded.  x sits padded in shared memory (4
// floats after every 64, so the lanes' item rows of x fall on different banks)
// with its sums per 16 weights.  The arithmetic is the reference's
// dequantisation factored per scale group, in fp32:
//   Q4_K  w = d1*q - m1           sum_i w_i x_i = d1 * sum q x - m1 * sum x
//   Q6_K  w = (d*sc) * (q - 32)   = (d*sc) * (sum q x - 32 * sum x)
//   Q8_0  w = d * q               = d * sum q x
// with d1 = d*sc, m1 = dmin*mn and d*sc rounded as the reference rounds them
// (cpp/quant.hpp:187-281); a weight costs a byte permute (q as the float
// 2^23 + q), half a packed subtraction and half a packed FMA.  The products
// are the reference's, summed in another order: results agree to fp32
// rounding (the bar the chunked kernels meet).
constexpr int kMqBuf = 3424;  // per buffer: 16 Q6_K blocks (3360 B) + alignment slack + a spare word

__device__ __forceinline__ int xpad(int i) { return i + 4 * (i >> 6); }

// the 4 bytes at byte offset o of a shared buffer (o even; a spare word follows the data)
__device__ __forceinline__ uint32_t sm_u32(const uint8_t* buf, int o) {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(buf + (o & ~3));
    return __funnelshift_r(w[0], w[1], (uint32_t)(o & 3) * 8u);
}

// acc += (the 4 bytes of v as floats) . x[0..3] (x 16-byte aligned in shared memory),
// the bytes made exact floats by the 2^23 + b bit pattern and `off` subtracted
__device__ __forceinline__ void dot4(uint32_t v, const float* x, uint64_t off, uint64_t& acc) {
    uint64_t a, b;
    bytes_biased(v, a, b);
    const float4 xv = *reinterpret_cast<const float4*>(x);
    acc = f2_fma(f2_sub(a, off), f2_pack(xv.x, xv.y), acc);
    acc = f2_fma(f2_sub(b, off), f2_pack(xv.z, xv.w), acc);
}

__device__ __forceinline__ float f2_sum(uint64_t v) {
    float lo, hi;
    f2_unpack(v, lo, hi);
    return lo + hi;
}

// Q4_K item: block at byte o of buf, quant chunk j (weights 64j..64j+63 of the
// block; xs = their x, x16 = their 16-weight sums).  aligned16: o is a
// multiple of 16 (then whole 16-byte reads)
__device__ __forceinline__ float item_q4k(const uint8_t* buf, int o, int j, bool aligned16, const float* xs,
                                          const float* x16) {
    uint32_t hw[4], qw[8];
    if (aligned16) {
        const uint4 h = *reinterpret_cast<const uint4*>(buf + o);
        const uint4 q0 = *reinterpret_cast<const uint4*>(buf + o + 16 + 32 * j);
        const uint4 q1 = *reinterpret_cast<const uint4*>(buf + o + 32 + 32 * j);
        hw[0] = h.x, hw[1] = h.y, hw[2] = h.z, hw[3] = h.w;
        qw[0] = q0.x, qw[1] = q0.y, qw[2] = q0.z, qw[3] = q0.w, qw[4] = q1.x, qw[5] = q1.y, qw[6] = q1.z,
        qw[7] = q1.w;
    } else {
#pragma unroll
        for (int k = 0; k < 4; k++) hw[k] = sm_u32(buf, o + 4 * k);
#pragma unroll
        for (int k = 0; k < 8; k++) qw[k] = sm_u32(buf, o + 16 + 32 * j + 4 * k);
    }
    const float d = __half2float(__ushort_as_half((uint16_t)(hw[0] & 0xFFFF)));
    const float dmin = __half2float(__ushort_as_half((uint16_t)(hw[0] >> 16)));
    // byte k of the 12 scale bytes, without indexing memory
    auto sb = [&](int k) -> int { return (int)(((k < 4 ? hw[1] : (k < 8 ? hw[2] : hw[3])) >> (8 * (k & 3))) & 0xFFu); };
    // get_scale_min_k4, cpp/quant.hpp:210-218
    auto scale_min = [&](int jj, int& sc, int& mn) {
        if (jj < 4) {
            sc = sb(jj) & 63;
            mn = sb(jj + 4) & 63;
        } else {
            sc = (sb(jj + 4) & 0xF) | ((sb(jj - 4) >> 6) << 4);
            mn = (sb(jj + 4) >> 4) | ((sb(jj) >> 6) << 4);
        }
    };
    int sc0, mn0, sc1, mn1;
    scale_min(2 * j, sc0, mn0);
    scale_min(2 * j + 1, sc1, mn1);
    const float d1 = __fmul_rn(d, (float)sc0), m1 = __fmul_rn(dmin, (float)mn0);
    const float d2 = __fmul_rn(d, (float)sc1), m2 = __fmul_rn(dmin, (float)mn1);
    const uint64_t off = f2_pack(8388608.f, 8388608.f);
    uint64_t lo = 0ull, hi = 0ull;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        dot4(qw[k] & 0x0F0F0F0Fu, xs + 4 * k, off, lo);
        dot4((qw[k] >> 4) & 0x0F0F0F0Fu, xs + xpad(32 + 4 * k), off, hi);
    }
    const float xlo = x16[0] + x16[1], xhi = x16[2] + x16[3];
    return (d1 * f2_sum(lo) - m1 * xlo) + (d2 * f2_sum(hi) - m2 * xhi);
}

// Q6_K item: block at byte o of buf (even), half c (weights 128c..128c+127)
__device__ __forceinline__ float item_q6k(const uint8_t* buf, int o, int c, const float* xs, const float* x16) {
    const int ql = o + 64 * c, qh = o + 128 + 32 * c;
    const uint32_t sw0 = sm_u32(buf, o + 192 + 8 * c), sw1 = sm_u32(buf, o + 196 + 8 * c);
    const uint32_t dw = sm_u32(buf, o + 206);  // d in the high half
    const float d = __half2float(__ushort_as_half((uint16_t)(dw >> 16)));
    const uint64_t off = f2_pack(8388608.f, 8388608.f);
    float res = 0.f;
#pragma unroll
    for (int h = 0; h < 2; h++) {  // weights l = 16h..16h+15 of every quarter (one scale each)
        uint64_t s[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int l = 16 * h + 4 * k;
            const uint32_t a = sm_u32(buf, ql + l), b = sm_u32(buf, ql + 32 + l), hb = sm_u32(buf, qh + l);
            dot4((a & 0x0F0F0F0Fu) | ((hb << 4) & 0x30303030u), xs + l, off, s[0]);
            dot4((b & 0x0F0F0F0Fu) | ((hb << 2) & 0x30303030u), xs + xpad(32 + l), off, s[1]);
            dot4(((a >> 4) & 0x0F0F0F0Fu) | (hb & 0x30303030u), xs + xpad(64 + l), off, s[2]);
            dot4(((b >> 4) & 0x0F0F0F0Fu) | ((hb >> 2) & 0x30303030u), xs + xpad(96 + l), off, s[3]);
        }
#pragma unroll
        for (int qq = 0; qq < 4; qq++) {
            const int si = h + 2 * qq;  // the scale of these weights: sc[is + l/16 + 2qq]
            const int8_t sc = (int8_t)(((si < 4 ? sw0 : sw1) >> (8 * (si & 3))) & 0xFF);
            const float ds = __fmul_rn(d, (float)sc);
            res += ds * (f2_sum(s[qq]) - 32.f * x16[2 * qq + h]);
        }
    }
    return res;
}

// Q8_0 item: the 68 bytes of blocks 2p and 2p+1 at byte o of buf (even)
__device__ __forceinline__ float item_q80(const uint8_t* buf, int o, const float* xs) {
    uint32_t v[17];
#pragma unroll
    for (int k = 0; k < 17; k++) v[k] = sm_u32(buf, o + 4 * k) ^ 0x80808080u;  // signed bytes + 128
    const float d0 = __half2float(__ushort_as_half((uint16_t)((v[0] ^ 0x8080u) & 0xFFFF)));
    const float d1 = __half2float(__ushort_as_half((uint16_t)((v[8] ^ 0x80800000u) >> 16)));
    const uint64_t off = f2_pack(8388736.f, 8388736.f);  // 2^23 + 128
    uint64_t s0 = 0ull, s1 = 0ull;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        // block 0's quants start at byte 2: bytes 2+4k.. of the pair
        dot4(__byte_perm(v[k], v[k + 1], 0x5432), xs + 4 * k, off, s0);
        dot4(v[9 + k], xs + xpad(32 + 4 * k), off, s1);
    }
    return d0 * f2_sum(s0) + d1 * f2_sum(s1);
}

// Q4_K and Q8_0 read straight from global memory: Q4_K blocks (144 bytes) of a
// 16-byte aligned matrix start on 16-byte boundaries, so an item is three
// 16-byte loads; Q8_0 block pairs (68 bytes) are seventeen 4-byte loads.
__device__ __forceinline__ float item_q4k_g(const uint8_t* blk, int j, const float* xs, const float* x16) {
    const uint4 h = __ldg(reinterpret_cast<const uint4*>(blk));
    const uint4 q0 = __ldg(reinterpret_cast<const uint4*>(blk + 16 + 32 * j));
    const uint4 q1 = __ldg(reinterpret_cast<const uint4*>(blk + 32 + 32 * j));
    const uint32_t hw[4] = {h.x, h.y, h.z, h.w};
    const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    const float d = __half2float(__ushort_as_half((uint16_t)(hw[0] & 0xFFFF)));
    const float dmin = __half2float(__ushort_as_half((uint16_t)(hw[0] >> 16)));
    auto sb = [&](int k) -> int { return (int)(((k < 4 ? hw[1] : (k < 8 ? hw[2] : hw[3])) >> (8 * (k & 3))) & 0xFFu); };
    auto scale_min = [&](int jj, int& sc, int& mn) {  // get_scale_min_k4, cpp/quant.hpp:210-218
        if (jj < 4) {
            sc = sb(jj) & 63;
            mn = sb(jj + 4) & 63;
        } else {
            sc = (sb(jj + 4) & 0xF) | ((sb(jj - 4) >> 6) << 4);
            mn = (sb(jj + 4) >> 4) | ((sb(jj) >> 6) << 4);
        }
    };
    int sc0, mn0, sc1, mn1;
    scale_min(2 * j, sc0, mn0);
    scale_min(2 * j + 1, sc1, mn1);
    const float d1 = __fmul_rn(d, (float)sc0), m1 = __fmul_rn(dmin, (float)mn0);
    const float d2 = __fmul_rn(d, (float)sc1), m2 = __fmul_rn(dmin, (float)mn1);
    const uint64_t off = f2_pack(8388608.f, 8388608.f);
    uint64_t lo = 0ull, hi = 0ull;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        dot4(qw[k] & 0x0F0F0F0Fu, xs + 4 * k, off, lo);
        dot4((qw[k] >> 4) & 0x0F0F0F0Fu, xs + xpad(32 + 4 * k), off, hi);
    }
    const float xlo = x16[0] + x16[1], xhi = x16[2] + x16[3];
    return (d1 * f2_sum(lo) - m1 * xlo) + (d2 * f2_sum(hi) - m2 * xhi);
}

__device__ __forceinline__ float item_q80_g(const uint8_t* pr, const float* xs) {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(pr);
    uint32_t v[17];
#pragma unroll
    for (int k = 0; k < 17; k++) v[k] = __ldg(w + k) ^ 0x80808080u;  // signed bytes + 128
    const float d0 = __half2float(__ushort_as_half((uint16_t)((v[0] ^ 0x8080u) & 0xFFFF)));
    const float d1 = __half2float(__ushort_as_half((uint16_t)((v[8] ^ 0x80800000u) >> 16)));
    const uint64_t off = f2_pack(8388736.f, 8388736.f);  // 2^23 + 128
    uint64_t s0 = 0ull, s1 = 0ull;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        dot4(__byte_perm(v[k], v[k + 1], 0x5432), xs + 4 * k, off, s0);
        dot4(v[9 + k], xs + xpad(32 + 4 * k), off, s1);
    }
    return d0 * f2_sum(s0) + d1 * f2_sum(s1);
}

// x (padded) and its 16-weight sums into shared memory, by the whole block
__device__ __forceinline__ void stage_x(const float* x, int n_in, float* xs, float* x16) {
    for (int i = threadIdx.x; i < n_in / 4; i += blockDim.x)
        *reinterpret_cast<float4*>(xs + xpad(4 * i)) = __ldg(reinterpret_cast<const float4*>(x) + i);
    __syncthreads();
    for (int g = threadIdx.x; g < n_in / 16; g += blockDim.x) {
        float t = 0.f;
#pragma unroll
        for (int i = 0; i < 16; i++) t += xs[xpad(16 * g + i)];
        x16[g] = t;
    }
    __syncthreads();
}

// One warp per row (rows warp, warp + all warps, ...) of Q4_K or Q8_0 parts;
// lanes take the row's items in turn and the warp adds their sums in a fixed
// tree.
__global__ void __launch_bounds__(256) matvecq_direct_kernel(MatvecArgs a) {
    extern __shared__ __align__(16) uint8_t mq_smem[];
    pdl_trigger();
    pdl_wait();
    const int n_in = a.n_in;
    float* xs = reinterpret_cast<float*>(mq_smem);
    float* x16 = xs + xpad(n_in) + 4;
    stage_x(a.x, n_in, xs, x16);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwb = (int)(blockDim.x >> 5);
    const int nw = gridDim.x * nwb;
    for (int r = blockIdx.x * nwb + warp; r < a.rows_total; r += nw) {
        int row;
        const MatvecPart P = part_of(a, r, row);
        const uint8_t* rowp = P.w + (size_t)row * P.row_bytes;
        float acc = 0.f;
        if (P.type == PICOATTN_WT_Q4_K) {
            const int n_items = (n_in / 256) * 4;
            for (int it = lane; it < n_items; it += 32)
                acc += item_q4k_g(rowp + (size_t)(it >> 2) * 144, it & 3, xs + xpad(64 * it), x16 + 4 * it);
        } else {
            const int n_items = n_in / 64;
            for (int it = lane; it < n_items; it += 32) acc += item_q80_g(rowp + (size_t)it * 68, xs + xpad(64 * it));
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) {
            float y = acc;
            if (P.bias) y = __fadd_rn(y, P.bias[row]);
            float* op = P.out + row;
            *op = a.accumulate ? __fadd_rn(*op, y) : y;
        }
    }
}

// items per row, bytes per item step and items per block of a streamed format
struct MqFormat {
    int items_per_block, block_bytes;
};
__device__ __forceinline__ MqFormat mq_format(int type) {
    if (type == PICOATTN_WT_Q4_K) return {4, 144};
    if (type == PICOATTN_WT_Q6_K) return {2, 210};
    return {1, 68};  // Q8_0: a pair of blocks per item
}

__global__ void __launch_bounds__(512) matvecq_kernel(MatvecArgs a) {
    extern __shared__ __align__(16) uint8_t mq_smem[];
    pdl_trigger();
    pdl_wait();
    const int n_in = a.n_in, nwb = (int)(blockDim.x >> 5);
    float* xs = reinterpret_cast<float*>(mq_smem);  // x, padded: xpad(n_in) floats
    float* x16 = xs + xpad(n_in) + 4;                // sums of x per 16 weights
    uint8_t* bufs = mq_smem + (((size_t)xpad(n_in) + 4 + n_in / 16) * 4 + 15) / 16 * 16;
    stage_x(a.x, n_in, xs, x16);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nw = gridDim.x * nwb, gw = blockIdx.x * nwb + warp;
    uint8_t* wbuf = bufs + (size_t)warp * 2 * kMqBuf;
    // a task = (row, round); the warp's rows are gw, gw + nw, ...
    struct Task {
        int r, round;
    };
    auto rounds_of = [&](int r) {
        int row;
        const MatvecPart P = part_of(a, r, row);
        const MqFormat f = mq_format(P.type);
        const int n_items = P.type == PICOATTN_WT_Q8_0 ? n_in / 64 : (n_in / 256) * f.items_per_block;
        return (n_items + 31) / 32;
    };
    // the bytes of a task: [g0, g1) of the row; they land from the 16-byte
    // boundary at or below g0 (delta bytes in) in buffer k & 1
    auto span = [&](Task t, uintptr_t& g0, uintptr_t& g1, MatvecPart& P, int& row, int& n_items) {
        P = part_of(a, t.r, row);
        const MqFormat f = mq_format(P.type);
        n_items = P.type == PICOATTN_WT_Q8_0 ? n_in / 64 : (n_in / 256) * f.items_per_block;
        const int i0 = 32 * t.round, i1 = min(n_items, i0 + 32);
        const int ipb = f.items_per_block;
        const uint8_t* rowp = P.w + (size_t)row * P.row_bytes;
        g0 = reinterpret_cast<uintptr_t>(rowp + (size_t)(i0 / ipb) * f.block_bytes);
        g1 = reinterpret_cast<uintptr_t>(rowp + (size_t)((i1 + ipb - 1) / ipb) * f.block_bytes);
    };
    auto issue = [&](Task t, int slot) {
        if (t.r < a.rows_total) {
            uintptr_t g0, g1;
            MatvecPart P;
            int row, n_items;
            span(t, g0, g1, P, row, n_items);
            const uintptr_t a0 = g0 & ~(uintptr_t)15;
            const int n16 = (int)((g1 - a0 + 15) >> 4);
            uint8_t* dst = wbuf + slot * kMqBuf;
            for (int i = lane; i < n16; i += 32) {
                const uintptr_t src = a0 + 16 * (uintptr_t)i;
                // the last piece may run past the matrix: copy only the bytes before g1
                const uintptr_t left = g1 > src ? g1 - src : 0;
                const uint32_t n = left < 16 ? (uint32_t)left : 16u;
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst + 16 * i)),
                             "l"(src), "r"(n)
                             : "memory");
            }
        }
        cp_async_commit();
    };
    auto next = [&](Task t) {
        return t.round + 1 < rounds_of(t.r) ? Task{t.r, t.round + 1} : Task{t.r + nw, 0};
    };
    Task cur{gw, 0};
    Task nxt = cur.r < a.rows_total ? next(cur) : Task{a.rows_total, 0};
    issue(cur, 0);
    float acc = 0.f;
    for (int k = 0; cur.r < a.rows_total; k++) {
        issue(nxt, (k + 1) & 1);
        cp_async_wait<1>();
        __syncwarp();  // this task's bytes (every lane's copies) are in its buffer
        uintptr_t g0, g1;
        MatvecPart P;
        int row, n_items;
        span(cur, g0, g1, P, row, n_items);
        const uint8_t* buf = wbuf + (k & 1) * kMqBuf;
        const int delta = (int)(g0 & 15), it = 32 * cur.round + lane;
        if (it < n_items) {
            if (P.type == PICOATTN_WT_Q4_K) {
                const int b = (it >> 2) - (32 * cur.round >> 2), j = it & 3, w0 = 64 * it;
                acc += item_q4k(buf, delta + 144 * b, j, delta == 0, xs + xpad(w0), x16 + (w0 >> 4));
            } else if (P.type == PICOATTN_WT_Q6_K) {
                const int b = (it >> 1) - (32 * cur.round >> 1), c = it & 1, w0 = 128 * it;
                acc += item_q6k(buf, delta + 210 * b, c, xs + xpad(w0), x16 + (w0 >> 4));
            } else {
                acc += item_q80(buf, delta + 68 * (it - 32 * cur.round), xs + xpad(64 * it));
            }
        }
        if (cur.round + 1 == (n_items + 31) / 32) {  // the row is done
#pragma unroll
            for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
            if (lane == 0) {
                // matmul, then the bias added (vec_add), then the residual
                float y = acc;
                if (P.bias) y = __fadd_rn(y, P.bias[row]);
                float* op = P.out + row;
                *op = a.accumulate ? __fadd_rn(*op, y) : y;
            }
            acc = 0.f;
        }
        __syncwarp();  // the buffer is read before the task after next overwrites it
        cur = nxt;
        nxt = cur.r < a.rows_total ? next(cur) : Task{a.rows_total, 0};
    }
    cp_async_wait<0>();
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
    cfg.dynamicSmemBytes = kMvSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    static PerDeviceOnce setup;
    const cudaError_t se = setup.run([] {
        for (auto k : {matvec_kernel<1, 2>, matvec_kernel<2, 2>, matvec_kernel<4, 2>, matvec_kernel<1, 4>,
                       matvec_kernel<2, 4>, matvec_kernel<4, 4>, matvec1_kernel<4>}) {
            const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMvSmem);
            if (e != cudaSuccess) return e;
        }
        return cudaSuccess;
    });
    if (se != cudaSuccess) return se;
    // one vector of Q4_K / Q6_K weights: the tensor-core kernel
    const cudaError_t me = launch_matvec_mma(a, stream);
    if (me != cudaErrorNotSupported) return me;
    bool f32 = false;  // F32 chunks need the 4 KB slots
    for (int p = 0; p < a.n_parts; p++) f32 = f32 || a.part[p].type == PICOATTN_WT_F32;
    if (f32) {
        if (a.n_vec == 1) return cudaLaunchKernelEx(&cfg, matvec_kernel<1, 2>, a);
        if (a.n_vec == 2) return cudaLaunchKernelEx(&cfg, matvec_kernel<2, 2>, a);
        return cudaLaunchKernelEx(&cfg, matvec_kernel<4, 2>, a);
    }
    // one vector of Q4_K / Q6_K / Q8_0 weights (Q8_0 rows in whole block pairs):
    // the streaming kernel
    bool streamed = a.n_vec == 1 && a.n_in % 64 == 0;
    for (int p = 0; p < a.n_parts; p++) {
        const int t = a.part[p].type;
        // 16-byte aligned matrices: Q4_K items are 16-byte loads, and Q6_K round
        // copies start at a 16-byte boundary at or below the round's first byte,
        // which must not lie before the matrix
        streamed = streamed && (t == PICOATTN_WT_Q4_K || t == PICOATTN_WT_Q6_K || t == PICOATTN_WT_Q8_0) &&
                   ((uintptr_t)a.part[p].w & 15u) == 0;
    }
    // shared memory: x (padded) and its 16-weight sums; the staged kernel adds two
    // round buffers per warp
    const size_t mq_x = (((size_t)(a.n_in + 4 * (a.n_in >> 6)) + 4 + (size_t)a.n_in / 16) * 4 + 15) / 16 * 16;
    const int mq_warps = mq_x + 16 * 2 * (size_t)kMqBuf <= 220 * 1024 ? 16 : 8;
    const size_t mq_smem = mq_x + (size_t)mq_warps * 2 * kMqBuf;
    if (streamed && mq_smem <= 220 * 1024) {
        static PerDeviceOnce mq_setup;
        const cudaError_t e = mq_setup.run([] {
            cudaError_t r = cudaFuncSetAttribute(matvecq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
            if (r == cudaSuccess)
                r = cudaFuncSetAttribute(matvecq_direct_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
            return r;
        });
        if (e != cudaSuccess) return e;
        // Q6_K parts go to the staged kernel, Q4_K and Q8_0 parts to the direct one
        MatvecArgs st = a, dr = a;
        st.n_parts = dr.n_parts = 0;
        st.rows_total = dr.rows_total = 0;
        for (int p = 0; p < a.n_parts; p++) {
            MatvecArgs& g = a.part[p].type == PICOATTN_WT_Q6_K ? st : dr;
            g.part[g.n_parts++] = a.part[p];
            g.rows_total += a.part[p].n_out;
        }
        if (dr.n_parts > 0) {
            const long long want = ((long long)dr.rows_total + 7) / 8;
            const int per_sm = std::max(1, std::min(8, (int)((227 * 1024) / (mq_x + 1024))));
            cfg.gridDim = dim3((unsigned)std::max<long long>(1, std::min<long long>(want, (long long)sms * per_sm)));
            cfg.blockDim = dim3(256);
            cfg.dynamicSmemBytes = mq_x;
            const cudaError_t r = cudaLaunchKernelEx(&cfg, matvecq_direct_kernel, dr);
            if (r != cudaSuccess || st.n_parts == 0) return r;
        }
        const long long want = ((long long)st.rows_total + mq_warps - 1) / mq_warps;
        const int per_sm = std::max(1, (int)((227 * 1024) / (mq_smem + 1024)));
        cfg.gridDim = dim3((unsigned)std::max<long long>(1, std::min<long long>(want, (long long)sms * per_sm)));
        cfg.blockDim = dim3((unsigned)(32 * mq_warps));
        cfg.dynamicSmemBytes = mq_smem;
        return cudaLaunchKernelEx(&cfg, matvecq_kernel, st);
    }
    bool groups = a.n_vec == 1;  // row groups need every matrix's rows in whole groups
    for (int p = 0; p < a.n_parts; p++) groups = groups && a.part[p].n_out % kMvRows == 0;
    if (groups) {
        // a block per group of rows, a warp per chunk step (up to kMv1Warps;
        // with more steps each warp takes several in turn)
        const int cpr = (a.n_in / 32 + 31) / 32;
        const int nwb = std::min(kMv1Warps, cpr);
        const long long n_groups = a.rows_total / kMvRows;
        cfg.gridDim = dim3((unsigned)std::max<long long>(1, std::min<long long>(n_groups, (long long)sms * 16)));
        cfg.blockDim = dim3((unsigned)(nwb * 32));
        cfg.dynamicSmemBytes = (size_t)nwb * kMvRingWords * 4;
        return cudaLaunchKernelEx(&cfg, matvec1_kernel<4>, a);
    }
    if (a.n_vec == 2) return cudaLaunchKernelEx(&cfg, matvec_kernel<2, 4>, a);
    return cudaLaunchKernelEx(&cfg, matvec_kernel<4, 4>, a);
}

}  // namespace picoattn
