// matvec_mma.cu -- one vector times Q4_K / Q6_K matrices on the integer tensor
// cores (the projections of a decode step: TensorOps::matmul_bias,
// cpp/tensor.hpp:110-143, with the blocks of cpp/quant.hpp:60-74 dequantised
// as cpp/quant.hpp:220-281 does).
//
// The weights of a 256-weight super-block are integers times per-group scales:
//   Q4_K  w = (d*sc_s) * q - (dmin*mn_s)   q in 0..15, 8 groups s of 32
//   Q6_K  w = (d*sc_g) * (q - 32)          q in 0..63, 16 groups g of 16
// so a row's dot product with x is, per super-block,
//   d * sum_groups sc * (sum_k q_k x_k)  [- dmin * sum_s mn_s * X_s]
// with X_s the sum of x over group s.  x is written once per call as an
// integer per element: for super-block b, x_k = xi_k * 2^(E_b - 29) with
// 2^E_b <= max|x| < 2^(E_b+1) and |xi_k| < 2^30 (exact for every element
// within 2^6 of the block's largest; smaller ones round at 2^(E_b-30)).
// xi is split into four signed byte digits (xi = sum_j digit_j * 256^j), and
// the tensor cores compute sum_k q_k * digit_j(x_k) exactly
// (mma.sync m16n8k32, u8 or s8 weights times s8 digits, s32 accumulate):
//   A = 16 rows x 32 weights of a tile (nibbles / 6-bit codes expanded to
//       bytes in registers), k < 16 from one scale group and k >= 16 from
//       another;
//   B = 32 x 8: column n = (group half n/4, digit n%4), the digits of the x
//       elements of that half's group, zero elsewhere;
// so the 8 columns of C are (group, digit) sums for 16 rows.  The group
// scales multiply those exact integer sums (s32 multiply-add: exact), and
// each row ends as d * 2^(E_b-29) * sum_j 256^j T_j in fp32.  Products and
// sums of the super-block are exact; the result differs from the reference's
// fp32 loop by the rounding of its own summation (the same bar as the
// CUDA-core kernels).
//
// Work: a block takes T consecutive 16-row tiles; its S warps split the
// super-blocks of a row into S contiguous slices (S up to 16 when there are
// few tiles), each warp streaming its slice of every tile (two rows per lane,
// the mma fragment layout).  The S slice sums of a row are added in slice
// order through shared memory, so results do not depend on timing or grid
// size.  Each warp first turns its slice of x into the B fragments (shared
// memory, 1 KB per super-block).  The grid is one wave of the blocks that fit
// on the SMs.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <utility>

#include "device_common.cuh"
#include "picoattn_internal.h"

namespace picoattn {

namespace {

constexpr int kMmMaxSlices = 16;
constexpr int kMmMaxTiles = 32;

struct MmArgs {
    MatvecArgs a;
    int nsb, slices, tiles_per_block, n_tiles;
    int tile_start[4];  // first tile of each part; tile_start[n_parts] = n_tiles
};

// d = A(u8) . B(s8), exact s32 (c = 0 or the running sums)
__device__ __forceinline__ void imma_u8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                        const int (&c)[4]) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(c[0]), "r"(c[1]), "r"(c[2]),
          "r"(c[3]));
}
__device__ __forceinline__ void imma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

// prmt.b32 with a full selector: a nibble with its top bit set repeats the
// sign of the byte it names (a signed byte widened in one ALU instruction)
__device__ __forceinline__ uint32_t prmt(uint32_t x, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(x), "r"(sel));
    return r;
}

__device__ __forceinline__ uint32_t ldg32(const uint8_t* p) { return __ldg(reinterpret_cast<const uint32_t*>(p)); }

// 4 bytes at a 2-byte aligned address inside a Q6_K block (kMis: p is 2 mod 4):
// the aligned words around it, neither reaching outside the block
template <bool kMis>
__device__ __forceinline__ uint32_t ldg32_2(const uint8_t* p) {
    if constexpr (!kMis) return ldg32(p);
    return __byte_perm(ldg32(p - 2), ldg32(p + 2), 0x5432);
}

// A 6-bit code q in each byte, as the signed byte q - 32: q ^ 32 is q - 32 in
// 6-bit two's complement; bit 5 of it, times 6, fills bits 6 and 7.
__device__ __forceinline__ uint32_t q6_signed(uint32_t q) {
    const uint32_t r = q ^ 0x20202020u;
    return r + (r & 0x20202020u) * 6u;
}

// The words of one super-block of one row that a lane needs.
//   Q4_K: w[0..3] the block's 16-byte head (d, dmin, 12 scale bytes);
//         w[4+m] the code bytes of mma m (qs bytes 32(m/2) + 16(m%2) + 4t..+3, or
//         32(m/2) + 8t + 4(m%2)..+3 in launches of Q4_K only)
//   Q6_K: w[3(2c+h)+0..2] = ql[64c+16h+4t], ql[64c+32+16h+4t], qh[32c+16h+4t];
//         w[12..15] the 16 scale bytes; w[16] d (low half)
constexpr int kRawQ4K = 12, kRawQ6K = 17;

// kPairs (launches of Q4_K only): lane t takes bytes 8t..8t+7 of each 32-byte
// group (mma 2jg + h uses bytes 8t + 4h..+3), one 8-byte load per group, so an
// instruction's 8 rows x 32 bytes are whole sectors.  Otherwise the layout
// Q6_K shares: bytes 16h + 4t..+3 of the group.
template <bool kPairs, int kRaw>
__device__ __forceinline__ void load_q4k(const uint8_t* blk, int t, uint32_t (&w)[kRaw]) {
    const uint4 h = __ldg(reinterpret_cast<const uint4*>(blk));
    w[0] = h.x, w[1] = h.y, w[2] = h.z, w[3] = h.w;
    if constexpr (kPairs) {
#pragma unroll
        for (int jg = 0; jg < 4; jg++) {
            const uint2 v = __ldg(reinterpret_cast<const uint2*>(blk + 16 + 32 * jg + 8 * t));
            w[4 + 2 * jg] = v.x, w[5 + 2 * jg] = v.y;
        }
    } else {
#pragma unroll
        for (int m = 0; m < 8; m++) w[4 + m] = ldg32(blk + 16 + 32 * (m >> 1) + 16 * (m & 1) + 4 * t);
    }
}

template <bool kMis, int kRaw>
__device__ __forceinline__ void load_q6k_as(const uint8_t* blk, int t, uint32_t (&w)[kRaw]) {
#pragma unroll
    for (int ch = 0; ch < 4; ch++) {
        const int c = ch >> 1, h = ch & 1;
        w[3 * ch + 0] = ldg32_2<kMis>(blk + 64 * c + 16 * h + 4 * t);
        w[3 * ch + 1] = ldg32_2<kMis>(blk + 64 * c + 32 + 16 * h + 4 * t);
        w[3 * ch + 2] = ldg32_2<kMis>(blk + 128 + 32 * c + 16 * h + 4 * t);
    }
#pragma unroll
    for (int k = 0; k < 4; k++) w[12 + k] = ldg32_2<kMis>(blk + 192 + 4 * k);
    w[16] = __ldg(reinterpret_cast<const unsigned short*>(blk + 208));
}

// one branch per block (2 mod 4 or not): the same for every row of a matrix
// whose rows are a whole number of words long
template <int kRaw>
__device__ __forceinline__ void load_q6k(const uint8_t* blk, int t, uint32_t (&w)[kRaw]) {
    if ((reinterpret_cast<uintptr_t>(blk) & 2u) != 0)
        load_q6k_as<true>(blk, t, w);
    else
        load_q6k_as<false>(blk, t, w);
}

// One Q4_K super-block of rows g (w0) and g+8 (w1): adds its contribution
// to acc0 / acc1.  bf: this super-block's B fragments; r: 2^(E_b-29) * 256^j0;
// xs: the 8 group sums X_s of x.
template <int kRaw>
__device__ __forceinline__ void sb_q4k(const uint32_t (&w0)[kRaw], const uint32_t (&w1)[kRaw], const uint32_t* bf,
                                       uint32_t bmask, float r, const float* xs, int t, int lane, float& acc0,
                                       float& acc1) {
    const int u = t >> 1;  // this lane's C columns belong to group half u
    int T00 = 0, T01 = 0, T10 = 0, T11 = 0;
#pragma unroll
    for (int jg = 0; jg < 4; jg++) {
        int c[4] = {0, 0, 0, 0};
#pragma unroll
        for (int hh = 0; hh < 2; hh++) {
            const int m = 2 * jg + hh;
            const uint32_t bv = bf[m * 32 + lane];
            const uint32_t q0 = w0[4 + m], q1 = w1[4 + m];
            const uint32_t a[4] = {q0 & 0x0F0F0F0Fu, q1 & 0x0F0F0F0Fu, (q0 >> 4) & 0x0F0F0F0Fu,
                                   (q1 >> 4) & 0x0F0F0F0Fu};
            int d[4];
            imma_u8(d, a, bv & bmask, bv & ~bmask, c);
            c[0] = d[0], c[1] = d[1], c[2] = d[2], c[3] = d[3];
        }
        // the 6-bit scale of group s = 2jg + u (get_scale_min_k4, cpp/quant.hpp:210-218)
        const int s = 2 * jg + u;
        int sc0, sc1;
        if (jg < 2) {
            sc0 = (int)((w0[1] >> (8 * s)) & 63u);
            sc1 = (int)((w1[1] >> (8 * s)) & 63u);
        } else {
            const int sh = 8 * (s - 4);
            sc0 = (int)(((w0[3] >> sh) & 0xFu) | (((w0[1] >> sh) >> 6 & 3u) << 4));
            sc1 = (int)(((w1[3] >> sh) & 0xFu) | (((w1[1] >> sh) >> 6 & 3u) << 4));
        }
        T00 += sc0 * c[0], T01 += sc0 * c[1];
        T10 += sc1 * c[2], T11 += sc1 * c[3];
    }
    // the mins of groups t and t + 4
    const float xa = xs[t], xb = xs[t + 4];
    auto mins = [&](const uint32_t (&w)[kRaw]) {
        const int sh = 8 * t;
        const int ma = (int)((w[2] >> sh) & 63u);
        const int mb = (int)(((w[3] >> sh) >> 4 & 0xFu) | (((w[2] >> sh) >> 6 & 3u) << 4));
        return (float)ma * xa + (float)mb * xb;
    };
    const float M0 = mins(w0), M1 = mins(w1);
    const float d0 = __half2float(__ushort_as_half((uint16_t)(w0[0] & 0xFFFFu)));
    const float dm0 = __half2float(__ushort_as_half((uint16_t)(w0[0] >> 16)));
    const float d1 = __half2float(__ushort_as_half((uint16_t)(w1[0] & 0xFFFFu)));
    const float dm1 = __half2float(__ushort_as_half((uint16_t)(w1[0] >> 16)));
    const float F0 = (float)T00 + 256.f * (float)T01, F1 = (float)T10 + 256.f * (float)T11;
    acc0 = fmaf(d0 * F0, r, acc0) - dm0 * M0;
    acc1 = fmaf(d1 * F1, r, acc1) - dm1 * M1;
}

// One Q6_K super-block of rows g (w0) and g+8 (w1)
template <int kRaw>
__device__ __forceinline__ void sb_q6k(const uint32_t (&w0)[kRaw], const uint32_t (&w1)[kRaw], const uint32_t* bf,
                                       uint32_t bmask, float r, int t, int lane, float& acc0, float& acc1) {
    const int u = t >> 1;
    // byte h + 2u of a scale word, sign-extended
    uint32_t sext_sel[2];
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const uint32_t b = (uint32_t)(h + 2 * u);
        sext_sel[h] = b | ((8u | b) << 4) | ((8u | b) << 8) | ((8u | b) << 12);
    }
    int T00 = 0, T01 = 0, T10 = 0, T11 = 0;
#pragma unroll
    for (int m = 0; m < 8; m++) {
        const int jg = m >> 1, c = jg >> 1, odd = jg & 1, h = m & 1, ch = 2 * c + h;
        auto codes = [&](const uint32_t (&w)[kRaw], uint32_t& lo, uint32_t& hi) {
            const uint32_t qa = w[3 * ch], qb = w[3 * ch + 1], hb = w[3 * ch + 2];
            if (!odd) {
                lo = (qa & 0x0F0F0F0Fu) | ((hb << 4) & 0x30303030u);
                hi = (qb & 0x0F0F0F0Fu) | ((hb << 2) & 0x30303030u);
            } else {
                lo = ((qa >> 4) & 0x0F0F0F0Fu) | (hb & 0x30303030u);
                hi = ((qb >> 4) & 0x0F0F0F0Fu) | ((hb >> 2) & 0x30303030u);
            }
            lo = q6_signed(lo);
            hi = q6_signed(hi);
        };
        uint32_t l0, h0, l1, h1;
        codes(w0, l0, h0);
        codes(w1, l1, h1);
        const uint32_t a[4] = {l0, l1, h0, h1};
        const uint32_t bv = bf[m * 32 + lane];
        int d[4];
        imma_s8(d, a, bv & bmask, bv & ~bmask);
        // scale of this lane's group: sc[8c + h + 4odd + 2u], a signed byte
        const uint32_t sel = sext_sel[h];
        const int sc0 = (int)prmt(w0[12 + 2 * c + odd], sel);
        const int sc1 = (int)prmt(w1[12 + 2 * c + odd], sel);
        T00 += sc0 * d[0], T01 += sc0 * d[1];
        T10 += sc1 * d[2], T11 += sc1 * d[3];
    }
    const float d0 = __half2float(__ushort_as_half((uint16_t)(w0[16] & 0xFFFFu)));
    const float d1 = __half2float(__ushort_as_half((uint16_t)(w1[16] & 0xFFFFu)));
    const float F0 = (float)T00 + 256.f * (float)T01, F1 = (float)T10 + 256.f * (float)T11;
    acc0 = fmaf(d0 * F0, r, acc0);
    acc1 = fmaf(d1 * F1, r, acc1);
}

// x of super-blocks [b0, b1) into this warp's B fragments (bf, 256 words per
// super-block), scales (pw: 2^(E_b-29), a power of two down to 2^-149; 0 for
// blocks whose largest magnitude is below 2^-120, NaN for non-finite x) and
// group sums (xsum, 8 per super-block).  dig: 256 words of scratch.
// kFuse: 0 x as given, 1 x = (x * norm_s) * norm_w, 2 x = silu(x) * up
template <bool kPairs, int kFuse>
__device__ __forceinline__ void prep_x(const float* x, int b0, int b1, uint32_t* bf, float* pw, float* xsum,
                                       uint32_t* dig, int lane, const float* norm_w, float norm_s, const float* up) {
    const int g = lane >> 2, t = lane & 3;
    // the slice's x lands in its B-fragment area first (1 KB per super-block
    // either way), every piece in flight at once
    for (int i = lane; i < (b1 - b0) * 64; i += 32) cp_async16(bf + 4 * i, x + 256 * b0 + 4 * i);
    cp_async_commit();
    cp_async_wait<0>();
    __syncwarp();
    for (int b = b0; b < b1; b++) {
        const float* xb = reinterpret_cast<const float*>(bf + (b - b0) * 256);
        const float4 v0 = *reinterpret_cast<const float4*>(xb + 8 * lane);
        const float4 v1 = *reinterpret_cast<const float4*>(xb + 8 * lane + 4);
        float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        if constexpr (kFuse == 1) {  // (x * s) * w, the norm's two roundings
            const float4 w0 = __ldg(reinterpret_cast<const float4*>(norm_w + 256 * b + 8 * lane));
            const float4 w1 = __ldg(reinterpret_cast<const float4*>(norm_w + 256 * b + 8 * lane + 4));
            const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (int i = 0; i < 8; i++) v[i] = __fmul_rn(__fmul_rn(v[i], norm_s), w[i]);
        } else if constexpr (kFuse == 2) {  // silu(g) * up: the reciprocal of 1 + e^-g, times g, times up
            const float4 u0 = __ldg(reinterpret_cast<const float4*>(up + 256 * b + 8 * lane));
            const float4 u1 = __ldg(reinterpret_cast<const float4*>(up + 256 * b + 8 * lane + 4));
            const float u[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v[i])));
                v[i] = __fmul_rn(__fmul_rn(v[i], sig), u[i]);
            }
        }
        uint32_t mx = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) mx = max(mx, __float_as_uint(v[i]) & 0x7FFFFFFFu);
#pragma unroll
        for (int o = 16; o; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        // mx: the largest magnitude's bits (NaN / inf compare above every finite)
        const int e = (int)(mx >> 23) - 127;  // E_b
        const bool bad = mx >= 0x7F800000u, tiny = e < -120;
        // xi = x * 2^(29 - e) in two exact power-of-two steps (29 - e can pass 127)
        const int k = 29 - e;
        const int k1 = k > 120 ? 120 : k;
        const float s1 = __uint_as_float((uint32_t)(127 + k1) << 23);
        const float s2 = __uint_as_float((uint32_t)(127 + k - k1) << 23);
        float part = 0.f;
        uint32_t dw[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            part += v[i];
            const int xi = (bad || tiny) ? 0 : __float2int_rn((v[i] * s1) * s2);
            dw[i] = ((uint32_t)xi + 0x80808080u) ^ 0x80808080u;  // the four signed digits, low digit first
        }
        part += __shfl_xor_sync(0xffffffffu, part, 1);
        part += __shfl_xor_sync(0xffffffffu, part, 2);
        if (t == 0) xsum[8 * b + g] = part;  // lanes 4s..4s+3 hold group s
        if (lane == 0) {
            // 2^(e-29): a normal float's exponent field, or a denormal's single bit
            const int ex = e - 29 + 127;
            pw[b] = bad ? __uint_as_float(0x7FC00000u)
                        : (tiny ? 0.f : __uint_as_float(ex > 0 ? (uint32_t)ex << 23 : 1u << (22 + ex)));
        }
        __syncwarp();
        *reinterpret_cast<uint4*>(dig + 8 * lane) = make_uint4(dw[0], dw[1], dw[2], dw[3]);
        *reinterpret_cast<uint4*>(dig + 8 * lane + 4) = make_uint4(dw[4], dw[5], dw[6], dw[7]);
        __syncwarp();
        // lane (g, t), mma m: digit g%4 of x at 64(m/2) + 32(g/4) + 16(m%2) + 4t + 0..3
        // (kPairs: 64(m/2) + 32(g/4) + 8t + 4(m%2) + 0..3), the weights lane t
        // of the A fragment holds for k = 4t..4t+3 (g < 4) or 16 + 4t.. (g >= 4)
        const uint32_t j = (uint32_t)(g & 3);
        const uint32_t sel = j | ((4u + j) << 4);
#pragma unroll
        for (int m = 0; m < 8; m++) {
            const int p = 64 * (m >> 1) + 32 * (g >> 2) + (kPairs ? 8 * t + 4 * (m & 1) : 16 * (m & 1) + 4 * t);
            const uint4 q = *reinterpret_cast<const uint4*>(dig + p);
            const uint32_t lo = __byte_perm(q.x, q.y, sel), hi = __byte_perm(q.z, q.w, sel);
            bf[(b - b0) * 256 + m * 32 + lane] = __byte_perm(lo, hi, 0x5410);
        }
        __syncwarp();
    }
}

// kMode: 0 every matrix Q4_K, 1 every matrix Q6_K, 2 both (chosen per tile).
// kFuse: x as given (0), normalised on the fly (1: x_norm_w), silu(x) * x_up (2),
// fragments made beforehand by launch_xfrag (3: xfrag).
// The single-format kernels fit 64 registers, so two 16-warp blocks share an SM.
template <int kMode, int kFuse>
__global__ void __launch_bounds__(kMmMaxSlices * 32, kMode == 2 ? 1 : 2) matvec_mma_kernel(MmArgs p) {
    constexpr int kRaw = kMode == 0 ? kRawQ4K : kRawQ6K;
    extern __shared__ __align__(16) uint8_t mm_smem[];
    const MatvecArgs& a = p.a;
    pdl_trigger();
    // the weights may be read before the kernels ahead of this one finish only
    // when none of them writes them (weights_ready); x always after
    if (!a.weights_ready) pdl_wait();
    const int nsb = p.nsb, S = p.slices, T = p.tiles_per_block;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    // shared memory: B fragments of every super-block [nsb][8][32], digit
    // scratch [S][256], slice sums [T][S][16], group sums [nsb][8], scales [nsb]
    uint32_t* bf_all = reinterpret_cast<uint32_t*>(mm_smem);
    uint32_t* dig = bf_all + (size_t)nsb * 256 + warp * 256;
    float* partial = reinterpret_cast<float*>(bf_all + (size_t)nsb * 256 + (size_t)S * 256);
    float* xsum = partial + (size_t)T * S * 16;
    float* pw = xsum + 8 * nsb;
    float* red = pw + nsb;  // [S] per-warp sums of squares (fused norm)
    const int b0 = warp * nsb / S, b1 = (warp + 1) * nsb / S, ns = b1 - b0;
    const int tile0 = blockIdx.x * T;
    const int n_my = min(T, p.n_tiles - tile0);
    const int steps = n_my * ns;
    // rows g and g + 8 of a tile (clamped to its matrix) and their type
    auto tile_info = [&](int tl, const uint8_t*& r0, const uint8_t*& r1, int& type) {
        const int tile = tile0 + tl;
        int pi = 0;
        while (pi + 1 < a.n_parts && tile >= p.tile_start[pi + 1]) pi++;
        const MatvecPart& P = a.part[pi];
        const int row = (tile - p.tile_start[pi]) * 16 + g;
        const int ra = min(row, P.n_out - 1), rb = min(row + 8, P.n_out - 1);
        r0 = P.w + (size_t)ra * P.row_bytes;
        r1 = P.w + (size_t)rb * P.row_bytes;
        type = P.type;
    };
    auto load = [&](const uint8_t* r0, const uint8_t* r1, int type, int b, uint32_t (&w0)[kRaw],
                    uint32_t (&w1)[kRaw]) {
        if (kMode == 0 || (kMode == 2 && type == PICOATTN_WT_Q4_K)) {
            load_q4k<kMode == 0, kRaw>(r0 + (size_t)b * 144, t, w0);
            load_q4k<kMode == 0, kRaw>(r1 + (size_t)b * 144, t, w1);
        } else if constexpr (kMode != 0) {
            load_q6k<kRaw>(r0 + (size_t)b * 210, t, w0);
            load_q6k<kRaw>(r1 + (size_t)b * 210, t, w1);
        }
    };
    // the warp's (tile, super-block) steps: a step's words are loaded and used
    // at once, the many warps of an SM (small register footprint) keeping the
    // loads in flight; the first step's words are requested before x is
    // prepared
    const uint8_t *r0 = nullptr, *r1 = nullptr;
    int ty = 0;
    uint32_t w0[kRaw], w1[kRaw];
    if (steps > 0) {
        tile_info(0, r0, r1, ty);
        if (a.weights_ready && t == 0) {
            // the first tile's rows of this warp's slice into L2 while the kernel
            // before still runs: one bulk prefetch per row (rows g and g + 8),
            // between 16-byte boundaries inside the row's slice
            const size_t bb = ty == PICOATTN_WT_Q4_K ? 144 : 210;
            for (int k = 0; k < 2; k++) {
                const uint8_t* rp = k ? r1 : r0;
                const uintptr_t s0 = (reinterpret_cast<uintptr_t>(rp + b0 * bb) + 15) & ~(uintptr_t)15;
                const uintptr_t s1 = reinterpret_cast<uintptr_t>(rp + b1 * bb) & ~(uintptr_t)15;
                if (s1 > s0)
                    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(s0), "r"((uint32_t)(s1 - s0))
                                 : "memory");
            }
        }
        load(r0, r1, ty, b0, w0, w1);
    }
    if (a.weights_ready) pdl_wait();
    float norm_s = 1.f;
    if constexpr (kFuse == 1) {
        // the norm's scale 1 / sqrt(mean(x^2) + 1e-6) over the whole vector, by
        // every block alike (the same order of additions in each)
        float ss = 0.f;
        for (int i = threadIdx.x; i < a.n_in / 4; i += blockDim.x) {
            const float4 v = __ldg(reinterpret_cast<const float4*>(a.x) + i);
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        float tot = 0.f;
        for (int i = 0; i < S; i++) tot += red[i];
        norm_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)a.n_in), 1e-6f)));
    }
    if constexpr (kFuse == 3) {
        // x's fragments, scales and group sums made once by launch_xfrag
        // (a.xfrag: [nsb][256] words, then [nsb] scales, then [nsb][8] sums)
        const uint32_t* xf = a.xfrag;
        const float* xpw = reinterpret_cast<const float*>(xf + (size_t)nsb * 256);
        const float* xxs = xpw + nsb;
        for (int i = lane; i < ns * 64; i += 32) cp_async16(bf_all + (size_t)b0 * 256 + 4 * i, xf + (size_t)b0 * 256 + 4 * i);
        cp_async_commit();
        for (int i = lane; i < ns; i += 32) pw[b0 + i] = xpw[b0 + i];
        for (int i = lane; i < 8 * ns; i += 32) xsum[8 * b0 + i] = xxs[8 * b0 + i];
        cp_async_wait<0>();
    } else if (ns > 0) {
        prep_x<kMode == 0, kFuse>(a.x, b0, b1, bf_all + (size_t)b0 * 256, pw, xsum, dig, lane, a.x_norm_w, norm_s,
                                  a.x_up);
    }
    __syncwarp();
    const uint32_t bmask = g < 4 ? 0xFFFFFFFFu : 0u;  // B column g: low half (k < 16) or high half
    float acc0 = 0.f, acc1 = 0.f;
    int ctl = 0;
    for (int st = 0; st < steps; st++) {
        const int tl = st / ns, bi = st - tl * ns, b = b0 + bi;
        if (st > 0) {
            if (tl != ctl) tile_info(tl, r0, r1, ty), ctl = tl;
            load(r0, r1, ty, b, w0, w1);
        }
        const float r = pw[b] * ((t & 1) ? 65536.f : 1.f);
        const uint32_t* bf = bf_all + (size_t)b * 256;
        if (kMode == 0 || (kMode == 2 && ty == PICOATTN_WT_Q4_K))
            sb_q4k<kRaw>(w0, w1, bf, bmask, r, xsum + 8 * b, t, lane, acc0, acc1);
        else if constexpr (kMode != 0)
            sb_q6k<kRaw>(w0, w1, bf, bmask, r, t, lane, acc0, acc1);
        if (bi == ns - 1) {  // the tile's slice is done: the quad's four parts of each row
            acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
            acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
            acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
            acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
            if (t == 0) {
                partial[((size_t)tl * S + warp) * 16 + g] = acc0;
                partial[((size_t)tl * S + warp) * 16 + g + 8] = acc1;
            }
            acc0 = acc1 = 0.f;
        }
    }
    __syncthreads();
    // the rows: slice sums in slice order, then the bias (vec_add), then the residual
    for (int i = threadIdx.x; i < n_my * 16; i += blockDim.x) {
        const int tl = i >> 4, rr = i & 15, tile = tile0 + tl;
        int pi = 0;
        while (pi + 1 < a.n_parts && tile >= p.tile_start[pi + 1]) pi++;
        const MatvecPart& P = a.part[pi];
        const int row = (tile - p.tile_start[pi]) * 16 + rr;
        if (row >= P.n_out) continue;
        float y = 0.f;
        for (int w = 0; w < S; w++) y += partial[((size_t)tl * S + w) * 16 + rr];
        if (P.bias) y = __fadd_rn(y, P.bias[row]);
        float* op = P.out + row;
        *op = a.accumulate ? __fadd_rn(*op, y) : y;
    }
}

// x's fragments, scales and group sums once for a whole launch, one warp per
// 256-element block (the x preparation of matvec_mma_kernel, written to global
// memory: [nsb][256] words, [nsb] scales, [nsb][8] group sums).  kFuse 2:
// x = silu(x) * up.
template <bool kPairs, int kFuse>
__global__ void __launch_bounds__(256) xfrag_kernel(const float* x, const float* up, int nsb, uint32_t* out) {
    __shared__ __align__(16) uint32_t sm[8][512];  // per warp: fragments, digit scratch
    pdl_trigger();
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.x * 8 + warp;
    if (b >= nsb) return;
    float* pw = reinterpret_cast<float*>(out + (size_t)nsb * 256);
    float* xs = pw + nsb;
    prep_x<kPairs, kFuse>(x, b, b + 1, sm[warp], pw, xs, sm[warp] + 256, lane, nullptr, 1.f, up);
    __syncwarp();
    for (int i = lane; i < 64; i += 32)
        reinterpret_cast<uint4*>(out + (size_t)b * 256)[i] = reinterpret_cast<const uint4*>(sm[warp])[i];
}

}  // namespace

size_t xfrag_bytes(int n_in) { return n_in % 256 ? 0 : (size_t)(n_in / 256) * (1024 + 4 + 32); }

cudaError_t launch_xfrag(const float* x, const float* up, int n_in, bool pairs, uint32_t* out, cudaStream_t stream) {
    if (n_in % 256 != 0 || ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(up) |
                             reinterpret_cast<uintptr_t>(out)) & 15u))
        return cudaErrorNotSupported;
    const int nsb = n_in / 256;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)((nsb + 7) / 8));
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (up)
        return pairs ? cudaLaunchKernelEx(&cfg, xfrag_kernel<true, 2>, x, up, nsb, out)
                     : cudaLaunchKernelEx(&cfg, xfrag_kernel<false, 2>, x, up, nsb, out);
    return pairs ? cudaLaunchKernelEx(&cfg, xfrag_kernel<true, 0>, x, up, nsb, out)
                 : cudaLaunchKernelEx(&cfg, xfrag_kernel<false, 0>, x, up, nsb, out);
}

// One vector of Q4_K / Q6_K matrices: returns cudaErrorNotSupported when the
// launch does not fit this kernel (other formats, several vectors, rows of
// other lengths), so the caller takes the CUDA-core kernels.
cudaError_t launch_matvec_mma(const MatvecArgs& a, cudaStream_t stream) {
    if (a.n_vec != 1 || a.n_in % 256 != 0 || a.n_parts < 1 || a.n_parts > 3) return cudaErrorNotSupported;
    if ((reinterpret_cast<uintptr_t>(a.x) & 15u) != 0) return cudaErrorNotSupported;
    if ((reinterpret_cast<uintptr_t>(a.x_norm_w) | reinterpret_cast<uintptr_t>(a.x_up) |
         reinterpret_cast<uintptr_t>(a.xfrag)) & 15u)
        return cudaErrorNotSupported;
    // fragments made for another position map (launch_xfrag's pairs flag)
    if (a.xfrag) {
        int q4 = 0;
        for (int i = 0; i < a.n_parts; i++) q4 += a.part[i].type == PICOATTN_WT_Q4_K;
        if ((q4 == a.n_parts) != (a.xfrag_pairs != 0)) return cudaErrorNotSupported;
    }
    MmArgs p{};
    p.a = a;
    p.nsb = a.n_in / 256;
    int tiles = 0;
    for (int i = 0; i < a.n_parts; i++) {
        const MatvecPart& P = a.part[i];
        if (P.type != PICOATTN_WT_Q4_K && P.type != PICOATTN_WT_Q6_K) return cudaErrorNotSupported;
        // Q4_K heads are 16-byte loads (rows of 144-byte blocks stay on 16-byte
        // boundaries); Q6_K words are read as the aligned words around them
        if ((reinterpret_cast<uintptr_t>(P.w) & 15u) != 0) return cudaErrorNotSupported;
        p.tile_start[i] = tiles;
        tiles += (P.n_out + 15) / 16;
    }
    p.tile_start[a.n_parts] = tiles;
    p.n_tiles = tiles;
    int n4 = 0;
    for (int i = 0; i < a.n_parts; i++) n4 += a.part[i].type == PICOATTN_WT_Q4_K;
    using Kern = void (*)(MmArgs);
    static const Kern kernels[3][4] = {
        {matvec_mma_kernel<0, 0>, matvec_mma_kernel<0, 1>, matvec_mma_kernel<0, 2>, matvec_mma_kernel<0, 3>},
        {matvec_mma_kernel<1, 0>, matvec_mma_kernel<1, 1>, matvec_mma_kernel<1, 2>, matvec_mma_kernel<1, 3>},
        {matvec_mma_kernel<2, 0>, matvec_mma_kernel<2, 1>, matvec_mma_kernel<2, 2>, matvec_mma_kernel<2, 3>}};
    const int mode = n4 == a.n_parts ? 0 : (n4 == 0 ? 1 : 2);
    const int fuse = a.xfrag ? 3 : (a.x_norm_w ? 1 : (a.x_up ? 2 : 0));
    const Kern kfn = kernels[mode][fuse];
    const void* kern = (const void*)kfn;
    static PerDeviceOnce setup;
    const cudaError_t se = setup.run([] {
        for (const auto& row : kernels)
            for (Kern k : row) {
                const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
                if (e != cudaSuccess) return e;
            }
        return cudaSuccess;
    });
    if (se != cudaSuccess) return se;
    auto smem_for = [&](int sl, int tpb) {
        return (size_t)p.nsb * 256 * 4 + (size_t)sl * 1024 + (size_t)tpb * sl * 64 + (size_t)p.nsb * 32 +
               (size_t)p.nsb * 4 + (size_t)kMmMaxSlices * 4;
    };
    // the launch shape: S warps per row tile (each a contiguous slice of the
    // super-blocks; at most 15 % longer than the mean slice, or the most even),
    // T tiles per block, one wave of the blocks that fit.  Among the slice
    // counts, the one with the fewest steps per warp (T x slice length),
    // counting SMs left idle as lost time; the larger on ties.
    const int sms = device_sm_count();
    int dev = 0;
    cudaError_t de = cudaGetDevice(&dev);
    if (de != cudaSuccess) return de;
    const long long key = ((((long long)dev * 4 + mode) * 4 + fuse) * 4096 + p.nsb) * (1LL << 24) + tiles;
    static std::mutex shape_mu;
    static std::map<long long, std::pair<int, int>> shapes;  // key -> (slices, tiles per block)
    {
        std::lock_guard<std::mutex> lk(shape_mu);
        const auto it = shapes.find(key);
        if (it != shapes.end()) {
            p.slices = it->second.first;
            p.tiles_per_block = it->second.second;
        }
    }
    double best_cost = 1e30;
    int best_s = p.slices, best_t = p.tiles_per_block;
    for (int sl = best_s ? 0 : std::min(p.nsb, kMmMaxSlices); sl >= 1; sl--) {
        const int len = (p.nsb + sl - 1) / sl;
        if ((double)len * sl / p.nsb > 1.15 && sl != 1 && sl != std::min(p.nsb, kMmMaxSlices)) continue;
        int per_sm = 0;
        cudaError_t oe = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 32 * sl, smem_for(sl, 1));
        if (oe != cudaSuccess) return oe;
        if (per_sm < 1) continue;
        const long long slots = (long long)per_sm * sms;
        int tpb = (int)std::min<long long>(kMmMaxTiles, (tiles + slots - 1) / slots);
        // the slice sums of T tiles must fit beside the rest
        while (tpb > 1 && smem_for(sl, tpb) > 220 * 1024) tpb--;
        const long long blocks = (tiles + tpb - 1) / tpb;
        const long long waves = (blocks + slots - 1) / slots;
        const double busy = std::min(1.0, (double)blocks / sms);
        const double cost = (double)tpb * len * waves / busy;
        if (cost < best_cost - 1e-9) best_cost = cost, best_s = sl, best_t = tpb;
        if (sl <= 4 && best_s) break;
    }
    if (best_s == 0 || smem_for(best_s, best_t) > 220 * 1024) return cudaErrorNotSupported;
    p.slices = best_s;
    p.tiles_per_block = best_t;
    {
        std::lock_guard<std::mutex> lk(shape_mu);
        shapes[key] = {best_s, best_t};
    }
    const size_t smem = smem_for(best_s, best_t);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)((tiles + p.tiles_per_block - 1) / p.tiles_per_block));
    cfg.blockDim = dim3((unsigned)(32 * p.slices));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kfn, p);
}

}  // namespace picoattn
