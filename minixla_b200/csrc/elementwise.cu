// Standalone element-wise kernels and the 3xTF32 operand split.
//
// add  : out[i] = a[i] + b[i % b_size]   -- tensor_add's rule (tensor.c:64-86):
//        b is either the same shape as a or a trailing suffix of it (a bias
//        row), so a plain modulo indexes it.
// relu : out[i] = x[i] > 0 ? x[i] : 0    -- tensor.c:110-120
// split: small = x - rne_tf32(x), the part of x a TF32 operand loses.  The
//        GEMM reads big = rne_tf32(x) from x itself through a rounding
//        (TFLOAT32) TMA map, so only the low part is materialised.
//
// All three are HBM-bound streams: 128-bit loads/stores, grid-stride loops
// over a grid sized as a multiple of the SM count.
#include <cuda_runtime.h>

#include "internal.h"

namespace mxb {

namespace {

constexpr int kBlock = 256;

int grid_for(long long work_items, int num_sms) {
    long long blocks = (work_items + kBlock - 1) / kBlock;
    const long long cap = static_cast<long long>(num_sms) * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return static_cast<int>(blocks);
}

__device__ __forceinline__ float relu1(float x) { return x > 0.0f ? x : 0.0f; }

__global__ void add_same_vec4(const float4* __restrict__ a, const float4* __restrict__ b,
                              float4* __restrict__ out, long long n4) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const float4 x = __ldcs(a + i), y = __ldcs(b + i);
        __stcs(out + i, make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w));
    }
}

// b_size % 4 == 0: four consecutive outputs use four consecutive b elements.
__global__ void add_bcast_vec4(const float4* __restrict__ a, const float* __restrict__ b, long long b_size,
                               float4* __restrict__ out, long long n4) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const float4 x = __ldcs(a + i);
        const float4 y = __ldg(reinterpret_cast<const float4*>(b + (4 * i) % b_size));
        __stcs(out + i, make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w));
    }
}

__global__ void add_scalar(const float* __restrict__ a, const float* __restrict__ b, long long b_size,
                           float* __restrict__ out, long long n) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        out[i] = a[i] + b[i % b_size];
}

__global__ void relu_vec4(const float4* __restrict__ x, float4* __restrict__ out, long long n4) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const float4 v = __ldcs(x + i);
        __stcs(out + i, make_float4(relu1(v.x), relu1(v.y), relu1(v.z), relu1(v.w)));
    }
}

__global__ void relu_scalar(const float* __restrict__ x, float* __restrict__ out, long long n) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        out[i] = relu1(x[i]);
}

// TF32 keeps the top 19 bits of an fp32 word (sign, 8 exponent, 10 mantissa).
// Round to nearest even at bit 13: add 0xFFF plus the kept LSB, clear the low
// 13 bits; acting on the magnitude bits makes it symmetric in sign.  This is
// the rounding TMA applies when it loads through a TFLOAT32 map, so
// x - rne_tf32(x) is exactly the part the GEMM's big operand leaves out (an
// exact fp32 difference: both values lie within one TF32 ulp).  Non-finite
// inputs, and values whose rounding overflows, give small = 0.
__device__ __forceinline__ float small_part(float x) {
    const uint32_t u = __float_as_uint(x);
    if ((u & 0x7F800000u) == 0x7F800000u) return 0.0f;
    const uint32_t big_bits = (u + 0x0FFFu + ((u >> 13) & 1u)) & 0xFFFFE000u;
    if ((big_bits & 0x7F800000u) == 0x7F800000u) return 0.0f;
    return x - __uint_as_float(big_bits);
}

__global__ void split_tf32_kernel(const float* __restrict__ x, long long rows, long long cols,
                                  long long ld_in, float* __restrict__ small, long long ld_out) {
    const long long n = rows * cols;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long r = i / cols, c = i - r * cols;
        small[r * ld_out + c] = small_part(x[r * ld_in + c]);
    }
}

__global__ void split_tf32_vec4(const float4* __restrict__ x, float4* __restrict__ small, long long n4) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const float4 v = __ldcs(x + i);
        small[i] = make_float4(small_part(v.x), small_part(v.y), small_part(v.z), small_part(v.w));
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

cudaError_t launch_add(const float* a, long long n, const float* b, long long b_size, float* out,
                       int num_sms, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    const bool al = aligned16(a) && aligned16(b) && aligned16(out) && n % 4 == 0;
    if (al && b_size == n) {
        add_same_vec4<<<grid_for(n / 4, num_sms), kBlock, 0, stream>>>(
            reinterpret_cast<const float4*>(a), reinterpret_cast<const float4*>(b),
            reinterpret_cast<float4*>(out), n / 4);
    } else if (al && b_size % 4 == 0) {
        add_bcast_vec4<<<grid_for(n / 4, num_sms), kBlock, 0, stream>>>(
            reinterpret_cast<const float4*>(a), b, b_size, reinterpret_cast<float4*>(out), n / 4);
    } else {
        add_scalar<<<grid_for(n, num_sms), kBlock, 0, stream>>>(a, b, b_size, out, n);
    }
    note_launch();
    return cudaGetLastError();
}

cudaError_t launch_relu(const float* x, long long n, float* out, int num_sms, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    if (aligned16(x) && aligned16(out) && n % 4 == 0) {
        relu_vec4<<<grid_for(n / 4, num_sms), kBlock, 0, stream>>>(reinterpret_cast<const float4*>(x),
                                                                  reinterpret_cast<float4*>(out), n / 4);
    } else {
        relu_scalar<<<grid_for(n, num_sms), kBlock, 0, stream>>>(x, out, n);
    }
    note_launch();
    return cudaGetLastError();
}

cudaError_t launch_split_tf32(const float* x, long long rows, long long cols, long long ld_in,
                              float* small, long long ld_out, int num_sms, cudaStream_t stream) {
    const long long n = rows * cols;
    if (n <= 0) return cudaSuccess;
    if (ld_in == cols && ld_out == cols && n % 4 == 0 && aligned16(x) && aligned16(small)) {
        split_tf32_vec4<<<grid_for(n / 4, num_sms), kBlock, 0, stream>>>(
            reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(small), n / 4);
    } else {
        split_tf32_kernel<<<grid_for(n, num_sms), kBlock, 0, stream>>>(x, rows, cols, ld_in, small, ld_out);
    }
    note_launch();
    return cudaGetLastError();
}

}  // namespace mxb
