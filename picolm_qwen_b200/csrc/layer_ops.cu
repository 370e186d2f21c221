// layer_ops.cu -- the rest of a decode layer around the attention block on the
// GPU: the model-dimension RMSNorm (TensorOps::rmsnorm, cpp/tensor.hpp:146-176,
// used before attention, before the FFN and before the logits,
// cpp/model.hpp:317, 430, 454) and the SwiGLU gate of the FFN
// (TensorOps::silu then elemwise_mul, cpp/tensor.hpp:371-408, as
// cpp/model.hpp:437-441 applies them).  The projections around them are
// picoattn_matvec's kernels (matvec.cu).
//
// Both kernels are launched with programmatic stream serialisation like the
// decode and projection kernels: each lets the next kernel launch at once and
// waits for the kernel before it to complete before it reads anything.
#include <algorithm>
#include <utility>

#include <cuda_runtime.h>

#include "device_common.cuh"
#include "picoattn_internal.h"

namespace picoattn {

namespace {

constexpr int kNormThreads = 256;

// out[v] = (x[v] * s) * w with s = 1 / sqrt(mean(x[v]^2) + 1e-6), one block per
// vector.  The reference accumulates the squares in four SSE lanes and adds
// them at the end; here the block adds per-thread partial sums in a tree, so
// the sum agrees to fp32 rounding, not bit for bit.  The scale and the two
// products are single IEEE roundings in the reference's order.
// out may be x: every element is read (twice) and written by the same thread,
// its second read before its write.
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const float* x, const float* __restrict__ w, float* out,
                                                               int dim) {
    __shared__ float red[kNormThreads / 32];
    pdl_trigger();
    pdl_wait();
    const float* xv = x + (size_t)blockIdx.x * dim;
    float* ov = out + (size_t)blockIdx.x * dim;
    float ss = 0.f;
    const bool vec4 = (dim & 3) == 0;
    if (vec4) {
        for (int i = threadIdx.x; i < dim / 4; i += kNormThreads) {
            const float4 t = reinterpret_cast<const float4*>(xv)[i];
            ss += t.x * t.x + t.y * t.y + t.z * t.z + t.w * t.w;
        }
    } else {
        for (int i = threadIdx.x; i < dim; i += kNormThreads) ss += xv[i] * xv[i];
    }
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kNormThreads / 32; i++) tot += red[i];
    const float s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)dim), 1e-6f)));
    if (vec4) {
        for (int i = threadIdx.x; i < dim / 4; i += kNormThreads) {
            const float4 t = reinterpret_cast<const float4*>(xv)[i];
            const float4 g = reinterpret_cast<const float4*>(w)[i];
            reinterpret_cast<float4*>(ov)[i] =
                make_float4(__fmul_rn(__fmul_rn(t.x, s), g.x), __fmul_rn(__fmul_rn(t.y, s), g.y),
                            __fmul_rn(__fmul_rn(t.z, s), g.z), __fmul_rn(__fmul_rn(t.w, s), g.w));
        }
    } else {
        for (int i = threadIdx.x; i < dim; i += kNormThreads) ov[i] = __fmul_rn(__fmul_rn(xv[i], s), w[i]);
    }
}

// gate[i] = (gate[i] * (1 / (1 + exp(-gate[i])))) * up[i]: silu in the
// reference's SSE order (the reciprocal of 1 + e^-x, then the product with x)
// and the elementwise product with the up projection.
__global__ void __launch_bounds__(256) silu_mul_kernel(float* __restrict__ gate, const float* __restrict__ up,
                                                       size_t n) {
    pdl_trigger();
    pdl_wait();
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float g = gate[i];
        const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
        gate[i] = __fmul_rn(__fmul_rn(g, sig), up[i]);
    }
}

template <typename... P, typename... A>
cudaError_t launch_pdl_kernel(void (*kernel)(P...), dim3 grid, dim3 block, cudaStream_t stream, A&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<A>(args)...);
}

}  // namespace

cudaError_t launch_rmsnorm(const float* x, const float* w, float* out, int dim, int n_vec, cudaStream_t stream) {
    return launch_pdl_kernel(rmsnorm_kernel, dim3((unsigned)n_vec), dim3(kNormThreads), stream, x, w, out, dim);
}

cudaError_t launch_silu_mul(float* gate, const float* up, size_t n, cudaStream_t stream) {
    const size_t blocks = std::min<size_t>((n + 255) / 256, (size_t)device_sm_count() * 8);
    return launch_pdl_kernel(silu_mul_kernel, dim3((unsigned)std::max<size_t>(1, blocks)), dim3(256), stream, gate,
                             up, n);
}

}  // namespace picoattn
