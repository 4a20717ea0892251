// Skinny fused GEMM for few output rows (M <= 16): out = epi(A[M,K] @ B[K,N]).
// use_skinny_gemm routes up to 8 rows here in TF32 mode and up to 16 in
// 3xTF32 mode; 9 to 16 TF32 rows run faster on the tensor-core kernel with
// its K split.
//
// With one to a few rows the work is reading B (4*K*N bytes); a 128-row
// tensor-core tile would idle most of the MMA and cover too few SMs.  This
// path is HBM-bound CUDA-core fp32:
//   1. partial kernel: grid = column blocks x K splits, sized to ~4 CTAs per
//      SM.  Each CTA stages its rows of A for its k-range in shared memory;
//      each thread owns four consecutive columns, reads one float4 of each B
//      row (a warp reads 512 contiguous bytes per row) and accumulates
//      M x 4 sums in registers.  Partial sums go to pooled workspace
//      [splits][M][N].
//   2. reduce kernel: each CTA takes 32 consecutive outputs; warp g sums a
//      fixed group of splits for them (coalesced 128-byte rows), the eight
//      group sums are added in a fixed order (deterministic for a given
//      split plan), then the node's epilogue steps are applied in order and
//      each output is stored once.
// fp32 multiply-adds: at least as accurate as either precision mode.
//
// One-kernel form (whenever A's rows of a K slice fit in shared memory): a
// cluster of kSplits CTAs shares one 128-column block and splits K between
// its CTAs, and each CTA's eight warps split its slice again.  Each warp
// keeps M x 4 sums per thread; the CTA adds its warps' sums in warp order in
// shared memory, then CTA r of the cluster adds the kSplits CTAs' sums for
// columns 16r .. 16r+15 through distributed shared memory in rank order,
// applies the epilogue and stores.  No workspace, no second launch, and the
// summation order is fixed.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "internal.h"
#include "sm100_ptx.cuh"

namespace mxb {

namespace {

constexpr int kThreads = 256;
constexpr int kColsPerCta = kThreads * 4;
constexpr int kMaxSmemFloats = 12 * 1024;  // 48 KiB of staged A

template <int MR>
__global__ void __launch_bounds__(kThreads)
    skinny_partial_kernel(const float* __restrict__ A, long long lda, const float* __restrict__ B, long long ldb,
                          float* __restrict__ partial, int M, int N, int K, int k_per_split) {
    extern __shared__ float sA[];  // [M][k_per_split]
    const int k0 = blockIdx.y * k_per_split;
    const int k1 = min(K, k0 + k_per_split);
    const int kl = k1 - k0;
    for (int i = threadIdx.x; i < M * kl; i += kThreads) {
        const int m = i / kl, kk = i - m * kl;
        sA[m * k_per_split + kk] = A[static_cast<long long>(m) * lda + k0 + kk];
    }
    __syncthreads();
    const int col = (blockIdx.x * kThreads + threadIdx.x) * 4;
    if (col >= N) return;
    float acc[MR][4];
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0.0f;
    const bool vec = col + 3 < N && (ldb & 3) == 0 && (reinterpret_cast<uintptr_t>(B) & 15) == 0;
    const float* bp = B + static_cast<long long>(k0) * ldb + col;
    auto fma_row = [&](const float4& b, int k) {
#pragma unroll
        for (int m = 0; m < MR; ++m) {
            if (m < M) {
                const float a = sA[m * k_per_split + k];
                acc[m][0] = fmaf(a, b.x, acc[m][0]);
                acc[m][1] = fmaf(a, b.y, acc[m][1]);
                acc[m][2] = fmaf(a, b.z, acc[m][2]);
                acc[m][3] = fmaf(a, b.w, acc[m][3]);
            }
        }
    };
    int k = 0;
    if (vec) {
        // Eight independent row loads in flight per thread, then their FMAs in k order.
        for (; k + 8 <= kl; k += 8) {
            float4 b[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) b[u] = __ldcs(reinterpret_cast<const float4*>(bp + static_cast<long long>(u) * ldb));
            bp += 8 * ldb;
#pragma unroll
            for (int u = 0; u < 8; ++u) fma_row(b[u], k + u);
        }
        for (; k < kl; ++k, bp += ldb) fma_row(__ldcs(reinterpret_cast<const float4*>(bp)), k);
    } else {
        for (; k < kl; ++k, bp += ldb) {
            float4 b;
            b.x = bp[0];
            b.y = col + 1 < N ? bp[1] : 0.0f;
            b.z = col + 2 < N ? bp[2] : 0.0f;
            b.w = col + 3 < N ? bp[3] : 0.0f;
            fma_row(b, k);
        }
    }
#pragma unroll
    for (int m = 0; m < MR; ++m) {
        if (m >= M) break;
        float* dst = partial + (static_cast<long long>(blockIdx.y) * M + m) * N + col;
#pragma unroll
        for (int c = 0; c < 4; ++c)
            if (col + c < N) dst[c] = acc[m][c];
    }
}

struct SkinnyEpilogue {
    int n_steps;
    EpStepDev steps[MXB_MAX_EPILOGUE];
};

constexpr int kReduceGroups = kThreads / 32;

__global__ void __launch_bounds__(kThreads)
    skinny_reduce_kernel(const float* __restrict__ partial, int splits, float* __restrict__ out, long long ldo, int M,
                         int N, long long row_base, const __grid_constant__ SkinnyEpilogue epi) {
    __shared__ float group_sum[kReduceGroups][32];
    const long long total = static_cast<long long>(M) * N;
    const int lane = threadIdx.x & 31;
    const int g = threadIdx.x >> 5;
    const int per = (splits + kReduceGroups - 1) / kReduceGroups;
    const int s0 = g * per, s1 = min(splits, s0 + per);
    for (long long base = blockIdx.x * 32ll; base < total; base += static_cast<long long>(gridDim.x) * 32) {
        const long long idx = base + lane;
        float x = 0.0f;
        if (idx < total) {
            const int m = static_cast<int>(idx / N), n = static_cast<int>(idx - static_cast<long long>(m) * N);
            const float* p = partial + (static_cast<long long>(s0) * M + m) * N + n;
            const long long stride = static_cast<long long>(M) * N;
#pragma unroll 4
            for (int s = s0; s < s1; ++s, p += stride) x += *p;
        }
        group_sum[g][lane] = x;
        __syncthreads();
        if (g == 0 && idx < total) {
            const int m = static_cast<int>(idx / N), n = static_cast<int>(idx - static_cast<long long>(m) * N);
            float v = group_sum[0][lane];
#pragma unroll
            for (int q = 1; q < kReduceGroups; ++q) v += group_sum[q][lane];
            for (int i = 0; i < epi.n_steps; ++i) {
                const EpStepDev& st = epi.steps[i];
                if (st.kind == MXB_EP_ADD_FULL) {
                    v += st.ptr[static_cast<long long>(m) * st.ld_or_size + n];
                } else if (st.kind == MXB_EP_ADD_ROW) {
                    v += st.ptr[n];
                } else if (st.kind == MXB_EP_ADD_MOD) {
                    const unsigned long long flat =
                        static_cast<unsigned long long>(m + row_base) * static_cast<unsigned long long>(N) + n;
                    v += st.ptr[flat % static_cast<unsigned long long>(st.ld_or_size)];
                } else if (st.kind == MXB_EP_RELU) {
                    v = v > 0.0f ? v : 0.0f;
                } else if (st.kind == MXB_EP_SCALE) {
                    v = v * st.scale;
                }
            }
            out[static_cast<long long>(m) * ldo + n] = v;
        }
        __syncthreads();
    }
}

constexpr int kSplits = 8;           // CTAs of a cluster, one K slice each
constexpr int kClusterCols = 128;    // output columns of a cluster (32 lanes x float4)
constexpr int kMaxSliceFloats = 16 * 1024;  // A's rows of one K slice staged in shared memory

// Epilogue of one output element (row m, column n), eval_fused's step order.
__device__ __forceinline__ float skinny_epilogue(float v, int m, int n, int N, long long row_base,
                                                 const SkinnyEpilogue& epi) {
    for (int i = 0; i < epi.n_steps; ++i) {
        const EpStepDev& st = epi.steps[i];
        if (st.kind == MXB_EP_ADD_FULL) {
            v += st.ptr[static_cast<long long>(m) * st.ld_or_size + n];
        } else if (st.kind == MXB_EP_ADD_ROW) {
            v += st.ptr[n];
        } else if (st.kind == MXB_EP_ADD_MOD) {
            const unsigned long long flat =
                static_cast<unsigned long long>(m + row_base) * static_cast<unsigned long long>(N) + n;
            v += st.ptr[flat % static_cast<unsigned long long>(st.ld_or_size)];
        } else if (st.kind == MXB_EP_RELU) {
            v = v > 0.0f ? v : 0.0f;
        } else if (st.kind == MXB_EP_SCALE) {
            v = v * st.scale;
        }
    }
    return v;
}

template <int MR>
__global__ void __cluster_dims__(1, kSplits, 1) __launch_bounds__(kThreads, 2)
    skinny_cluster_kernel(const float* __restrict__ A, long long lda, const float* __restrict__ B, long long ldb,
                          float* __restrict__ out, long long ldo, int M, int N, int K, long long row_base,
                          const __grid_constant__ SkinnyEpilogue epi) {
    extern __shared__ float sm[];
    const int slice = (K + kSplits - 1) / kSplits;  // rows of K per CTA
    const int k0 = blockIdx.y * slice;
    const int k1 = min(K, k0 + slice);
    const int kl = max(0, k1 - k0);
    float* sA = sm;                                 // [M][slice] during the k-loop,
    float* part = sm;                               // then [8 warps][M][128] in the same bytes
    for (int i = threadIdx.x; i < M * kl; i += kThreads) {
        const int m = i / kl, kk = i - m * kl;
        sA[m * slice + kk] = A[static_cast<long long>(m) * lda + k0 + kk];
    }
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int col = blockIdx.x * kClusterCols + lane * 4;
    const int per_warp = (kl + 7) / 8;
    const int w0 = min(kl, warp * per_warp), w1 = min(kl, w0 + per_warp);
    float acc[MR][4];
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0.0f;
    auto fma_row = [&](const float4& b, int k) {
#pragma unroll
        for (int m = 0; m < MR; ++m) {
            if (m < M) {
                const float a = sA[m * slice + k];
                acc[m][0] = fmaf(a, b.x, acc[m][0]);
                acc[m][1] = fmaf(a, b.y, acc[m][1]);
                acc[m][2] = fmaf(a, b.z, acc[m][2]);
                acc[m][3] = fmaf(a, b.w, acc[m][3]);
            }
        }
    };
    if (col < N) {
        const float* bp = B + static_cast<long long>(k0 + w0) * ldb + col;
        int k = w0;
        if (col + 3 < N && (ldb & 3) == 0 && (reinterpret_cast<uintptr_t>(B) & 15) == 0) {
            // kBatch independent row loads in flight (16 while the sums need
            // few registers), then their FMAs in k order.
            constexpr int kBatch = MR <= 8 ? 16 : 8;
            for (; k + kBatch <= w1; k += kBatch) {
                float4 b[kBatch];
#pragma unroll
                for (int u = 0; u < kBatch; ++u)
                    b[u] = __ldcs(reinterpret_cast<const float4*>(bp + static_cast<long long>(u) * ldb));
                bp += kBatch * ldb;
#pragma unroll
                for (int u = 0; u < kBatch; ++u) fma_row(b[u], k + u);
            }
            for (; k < w1; ++k, bp += ldb) fma_row(__ldcs(reinterpret_cast<const float4*>(bp)), k);
        } else {
            for (; k < w1; ++k, bp += ldb) {
                float4 b;
                b.x = bp[0];
                b.y = col + 1 < N ? bp[1] : 0.0f;
                b.z = col + 2 < N ? bp[2] : 0.0f;
                b.w = col + 3 < N ? bp[3] : 0.0f;
                fma_row(b, k);
            }
        }
    }
    __syncthreads();  // every warp is done with sA before its bytes hold the sums
#pragma unroll
    for (int m = 0; m < MR; ++m) {
        if (m >= M) break;
#pragma unroll
        for (int c = 0; c < 4; ++c) part[(warp * M + m) * kClusterCols + lane * 4 + c] = acc[m][c];
    }
    __syncthreads();
    // This CTA's sums: warps added in order, into warp 0's rows.
    for (int e = threadIdx.x; e < M * kClusterCols; e += kThreads) {
        float v = part[e];
        for (int w = 1; w < 8; ++w) v += part[w * M * kClusterCols + e];
        part[e] = v;
    }
    cluster_sync();  // every CTA's sums are visible to the cluster
    // CTA r: columns 16r .. 16r+15 of the block, summed over the cluster's CTAs in rank order.
    const uint32_t rank = static_cast<uint32_t>(blockIdx.y % kSplits);
    constexpr int kColsPerRank = kClusterCols / kSplits;
    for (int e = threadIdx.x; e < M * kColsPerRank; e += kThreads) {
        const int m = e / kColsPerRank;
        const int j = static_cast<int>(rank) * kColsPerRank + (e - m * kColsPerRank);
        const uint32_t addr = static_cast<uint32_t>(__cvta_generic_to_shared(&part[m * kClusterCols + j]));
        float v = 0.0f;
#pragma unroll
        for (int q = 0; q < kSplits; ++q) v += ld_shared_cluster_f32(mapa_shared(addr, static_cast<uint32_t>(q)));
        const int n = blockIdx.x * kClusterCols + j;
        if (n < N) out[static_cast<long long>(m) * ldo + n] = skinny_epilogue(v, m, n, N, row_base, epi);
    }
    cluster_sync();  // no CTA leaves while the others may still read its shared memory
}

template <int MR>
cudaError_t launch_cluster(const float* A, long long lda, const float* B, long long ldb, float* out, long long ldo,
                           int M, int N, int K, long long row_base, const SkinnyEpilogue& epi, cudaStream_t stream) {
    auto kernel = skinny_cluster_kernel<MR>;
    const int slice = (K + kSplits - 1) / kSplits;
    const size_t smem = std::max<size_t>(static_cast<size_t>(M) * slice, 8ull * M * kClusterCols) * sizeof(float);
    static std::mutex mu;
    static uint64_t configured = 0;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (dev >= 64 || !(configured & (1ull << dev))) {
            e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(std::max(kMaxSliceFloats, 8 * 16 * kClusterCols) * sizeof(float)));
            if (e != cudaSuccess) return e;
            if (dev < 64) configured |= 1ull << dev;
        }
    }
    const dim3 grid((N + kClusterCols - 1) / kClusterCols, kSplits);
    kernel<<<grid, kThreads, smem, stream>>>(A, lda, B, ldb, out, ldo, M, N, K, row_base, epi);
    return cudaGetLastError();
}

template <int MR>
cudaError_t launch_partial(const SkinnyPlan& pl, const float* A, long long lda, const float* B, long long ldb,
                           float* partial, int M, int N, int K, cudaStream_t stream) {
    const dim3 grid(pl.col_blocks, pl.splits);
    const size_t smem = static_cast<size_t>(M) * pl.k_per_split * sizeof(float);
    skinny_partial_kernel<MR><<<grid, kThreads, smem, stream>>>(A, lda, B, ldb, partial, M, N, K, pl.k_per_split);
    return cudaGetLastError();
}

}  // namespace

SkinnyPlan plan_skinny(int M, int N, int K, int num_sms) {
    SkinnyPlan p;
    // One kernel whenever a K slice of A's rows fits in shared memory (no
    // workspace then).  Measured against the two-kernel form: (1, 4096,
    // 4096) 12.3 vs 19.2 us, (16, 4096, 4096) 29.6 vs 35.7, (1, 1000, 780)
    // 8.1 vs 13.2.  MINIXLA_SKINNY_FORM=split forces the two kernels.
    const long long slice = (K + kSplits - 1) / kSplits;
    const char* force = getenv("MINIXLA_SKINNY_FORM");
    if (static_cast<long long>(M) * slice <= kMaxSliceFloats && !(force && !strcmp(force, "split"))) {
        p.one_kernel = true;
        p.splits = 0;
        return p;
    }
    p.col_blocks = (N + kColsPerCta - 1) / kColsPerCta;
    // About four CTAs per SM, each streaming at least 32 rows of B.
    int splits = (4 * num_sms + p.col_blocks - 1) / p.col_blocks;
    splits = std::max(1, std::min(splits, (K + 31) / 32));
    int kps = (K + splits - 1) / splits;
    const int kps_cap = std::max(32, kMaxSmemFloats / std::max(1, M));
    if (kps > kps_cap) kps = kps_cap;
    p.k_per_split = kps;
    p.splits = (K + kps - 1) / kps;
    return p;
}

// ------------------------------------------------------------------ tiny problems
//
// Small dense problems in 3xTF32 mode (config 1's 128^3 and the like) are
// set by latency, not throughput: one launch of a plain CUDA-core kernel,
// fp32 FMAs (more accurate than 3xTF32), no tensor-map set-up and no split
// pre-pass.  Each CTA owns a 32 x 32 output tile; 256 threads hold 2 x 2
// outputs each; K runs in chunks of kTinyBK staged in shared memory (A
// transposed, so a thread's two rows are one broadcast read per k), all of
// a chunk's loads issued before its stores.

namespace {

constexpr int kTinyBK = 128;

__global__ void __launch_bounds__(256)
    tiny_gemm_kernel(const float* __restrict__ A, long long lda, const float* __restrict__ B, long long ldb,
                     float* __restrict__ out, long long ldo, int M, int N, int K, long long row_base,
                     const __grid_constant__ SkinnyEpilogue epi) {
    __shared__ float As[kTinyBK][33];  // As[k][m]
    __shared__ float Bs[kTinyBK][32];  // Bs[k][n]
    constexpr int kPer = 32 * kTinyBK / 256;  // elements of each operand a thread stages per chunk
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int m0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
    float acc[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};
    for (int k0 = 0; k0 < K; k0 += kTinyBK) {
        // All of the chunk's loads are issued before any store, so their latencies overlap.
        float ra[kPer], rb[kPer];
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int i = threadIdx.x + u * 256;
            const int r = i / kTinyBK, k = i - r * kTinyBK;  // A: consecutive threads along k
            ra[u] = (m0 + r < M && k0 + k < K) ? __ldg(A + static_cast<long long>(m0 + r) * lda + k0 + k) : 0.0f;
            const int kb = i >> 5, c = i & 31;                // B: consecutive threads along n
            rb[u] = (k0 + kb < K && n0 + c < N) ? __ldg(B + static_cast<long long>(k0 + kb) * ldb + n0 + c) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int i = threadIdx.x + u * 256;
            const int r = i / kTinyBK, k = i - r * kTinyBK;
            As[k][r] = ra[u];
            Bs[i >> 5][i & 31] = rb[u];
        }
        __syncthreads();
#pragma unroll 16
        for (int k = 0; k < kTinyBK; ++k) {
            const float a0 = As[k][2 * ty], a1 = As[k][2 * ty + 1];
            const float b0 = Bs[k][2 * tx], b1 = Bs[k][2 * tx + 1];
            acc[0][0] = fmaf(a0, b0, acc[0][0]);
            acc[0][1] = fmaf(a0, b1, acc[0][1]);
            acc[1][0] = fmaf(a1, b0, acc[1][0]);
            acc[1][1] = fmaf(a1, b1, acc[1][1]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int m = m0 + 2 * ty + i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int n = n0 + 2 * tx + j;
            if (n < N) out[static_cast<long long>(m) * ldo + n] = skinny_epilogue(acc[i][j], m, n, N, row_base, epi);
        }
    }
}

}  // namespace

// TF32 mode: up to 8 rows.  From 9 rows the tensor-core kernel with its K
// split streams B faster than the CUDA cores multiply it (K = N = 8192:
// M = 8 65 -> 54 us, 12 rows 90 -> 54 us, 16 rows 96 -> 56 us; M = 4 51 vs
// 54 us stays here).  3xTF32 mode: up to 16 rows, as the low-part pass over
// B alone costs more than the whole CUDA-core product (M = 16: 95 vs 200 us).
bool use_skinny_gemm(int M, int precision) {
    int limit = precision == GPU_PRECISION_3XTF32 ? kSkinnyMaxRows : 8;
    if (const char* v = getenv("MINIXLA_SKINNY_MAX_ROWS")) limit = std::min(kSkinnyMaxRows, std::max(0, atoi(v)));
    return M <= limit;
}

bool use_tiny_gemm(int M, int N, int K, int precision) {
    const long long mnk = static_cast<long long>(M) * N * K;
    if (const char* v = getenv("MINIXLA_TINY_MAX_MNK")) return mnk <= atoll(v);
    return mnk <= (precision == GPU_PRECISION_3XTF32 ? kTinyMaxMnk3x : kTinyMaxMnk);
}

cudaError_t launch_tiny_gemm(const float* A, long long lda, const float* B, long long ldb, float* out, long long ldo,
                             int M, int N, int K, long long row_base, const EpStepDev* steps, int n_steps,
                             cudaStream_t stream) {
    SkinnyEpilogue epi{};
    epi.n_steps = n_steps;
    for (int i = 0; i < n_steps; ++i) epi.steps[i] = steps[i];
    const dim3 grid((N + 31) / 32, (M + 31) / 32);
    tiny_gemm_kernel<<<grid, 256, 0, stream>>>(A, lda, B, ldb, out, ldo, M, N, K, row_base, epi);
    note_launch();
    return cudaGetLastError();
}

cudaError_t launch_skinny_gemm(const float* A, long long lda, const float* B, long long ldb, float* out, long long ldo,
                               int M, int N, int K, long long row_base, const EpStepDev* steps, int n_steps,
                               float* workspace, const SkinnyPlan& pl, int num_sms, cudaStream_t stream) {
    if (M < 1 || M > kSkinnyMaxRows) return cudaErrorInvalidValue;
    cudaError_t e;
    if (pl.one_kernel) {
        SkinnyEpilogue epi{};
        epi.n_steps = n_steps;
        for (int i = 0; i < n_steps; ++i) epi.steps[i] = steps[i];
        if (M == 1) e = launch_cluster<1>(A, lda, B, ldb, out, ldo, M, N, K, row_base, epi, stream);
        else if (M == 2) e = launch_cluster<2>(A, lda, B, ldb, out, ldo, M, N, K, row_base, epi, stream);
        else if (M <= 4) e = launch_cluster<4>(A, lda, B, ldb, out, ldo, M, N, K, row_base, epi, stream);
        else if (M <= 8) e = launch_cluster<8>(A, lda, B, ldb, out, ldo, M, N, K, row_base, epi, stream);
        else e = launch_cluster<16>(A, lda, B, ldb, out, ldo, M, N, K, row_base, epi, stream);
        note_launch();
        return e;
    }
    if (M == 1) e = launch_partial<1>(pl, A, lda, B, ldb, workspace, M, N, K, stream);
    else if (M == 2) e = launch_partial<2>(pl, A, lda, B, ldb, workspace, M, N, K, stream);
    else if (M <= 4) e = launch_partial<4>(pl, A, lda, B, ldb, workspace, M, N, K, stream);
    else if (M <= 8) e = launch_partial<8>(pl, A, lda, B, ldb, workspace, M, N, K, stream);
    else e = launch_partial<16>(pl, A, lda, B, ldb, workspace, M, N, K, stream);
    note_launch();
    if (e != cudaSuccess) return e;
    SkinnyEpilogue epi{};
    epi.n_steps = n_steps;
    for (int i = 0; i < n_steps; ++i) epi.steps[i] = steps[i];
    const long long total = static_cast<long long>(M) * N;
    long long blocks = (total + 31) / 32;
    if (blocks > 8ll * num_sms) blocks = 8ll * num_sms;
    skinny_reduce_kernel<<<static_cast<int>(blocks), kThreads, 0, stream>>>(workspace, pl.splits, out, ldo, M, N, row_base,
                                                                          epi);
    note_launch();
    return cudaGetLastError();
}

}  // namespace mxb
