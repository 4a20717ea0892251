// Fused GEMM + element-wise epilogue for sm_100a:  out = epi(A @ B), fp32 in/out.
//
// This is the kernel behind an OP_FUSED node (graph.c:32-52 builds the node,
// eval_fused at graph.c:64-115 defines its value).  Design:
//
//  * Persistent CTAs, one per SM (grid = min(tiles, SMs)), each walking a
//    grouped tile order so concurrently running tiles share A row-blocks and
//    B column-blocks in L2.
//  * Output tile 128 x BN.  k advances in blocks of 32 fp32 = one 128-byte
//    swizzle row, staged in a STAGES-deep shared-memory ring by TMA:
//      A box [128 rows][32 k]     K-major, SWIZZLE_128B  (16 KiB)
//      B boxes [32 k][32 n] x BN/32, MN-major, SWIZZLE_128B_ATOM_32B (4 KiB each)
//    B is consumed MN-major straight from its row-major [K, N] layout, so no
//    transpose pass exists anywhere.
//  * Warp roles (192 threads):
//      warp 0      one thread issues the TMA loads
//      warp 1      allocates TMEM; one thread issues tcgen05.mma (kind::tf32,
//                  M=128, N=BN, K=8) into an fp32 accumulator in TMEM
//      warps 2..5  epilogue: tcgen05.ld the accumulator (warp w reads TMEM
//                  lanes 32*(w%4)..+31, i.e. one output row per thread),
//                  apply the node's epilogue steps in order, store once.
//    TMEM holds two accumulators (2*BN columns) so the epilogue of tile i
//    overlaps the main loop of tile i+1.
//  * Every operand goes through a TFLOAT32 tensor map, so TMA rounds fp32 to
//    TF32 (round to nearest even) on its way into shared memory; fed raw
//    fp32, the tensor core would truncate instead.
//  * 3xTF32 mode: a pre-pass writes small = x - rne_tf32(x) for A and B; the
//    raw operands loaded through the rounding maps are exactly big =
//    rne_tf32(x).  Per k-step the MMA warp issues big*big + big*small +
//    small*big into the same accumulator.  The tensor core's fp32
//    accumulation truncates toward zero, a bias that grows with K, so this
//    mode accumulates K in segments of kSegKb k-blocks: each segment starts
//    a fresh TMEM accumulator and the epilogue sums the segments in fp32
//    registers with round-to-nearest.
//  * Every mbarrier wait is bounded (global-timer limit).  A wait that runs
//    out records an error bit in global memory, raises a CTA-wide abort flag,
//    waits (bounded) for its own copies / MMAs in flight, frees TMEM and
//    returns; the host reports MXB_E_TIMEOUT.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "internal.h"
#include "sm100_ptx.cuh"

namespace mxb {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 32;           // fp32 elements per 128-byte swizzle row
constexpr int kThreads = 192;
constexpr int kBoxBytes = 32 * 32 * 4;  // one B box: 32 k-rows x 128 bytes

constexpr int kSegKb = 8;           // k-blocks (of 32) per accumulation segment in 3xTF32 mode
// With at most this many k-blocks the main loop is short (K <= 1024), so the
// epilogue prefetches its rows of the ADD operands before the accumulator is
// ready; longer loops prefetch once it is (earlier lines would be evicted).
constexpr int kShortKb = 32;

struct FusedParams {
    float* out;
    long long ldo;
    int M, N, K;
    int n_steps;
    int tiles_m, tiles_n, num_tiles, num_kb;
    int group_m;
    int seg_kb;                     // k-blocks per accumulation segment (num_kb: one segment)
    long long row_base;             // global index of row 0 of this launch (modulo-rule operands)
    unsigned long long timeout_ns;
    int* err;
    EpStepDev steps[MXB_MAX_EPILOGUE];
};

template <int BN, int STAGES, bool SPLIT3>
struct Cfg {
    static constexpr int kABytes = kBM * kBK * 4;
    static constexpr int kBBytes = BN * kBK * 4;
    static constexpr int kOperandBytes = kABytes + kBBytes;
    static constexpr int kStageBytes = (SPLIT3 ? 2 : 1) * kOperandBytes;
    static constexpr int kTmemCols = 2 * BN;
    static constexpr int kBarOffset = STAGES * kStageBytes;
    static constexpr int kNumBars = 2 * STAGES + 5;
    static constexpr int kSmemBytes = 1024 + kBarOffset + kNumBars * 8 + 16;
    static_assert(kStageBytes % 1024 == 0, "stages must keep 1 KiB swizzle alignment");
    static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN");
    static_assert(kTmemCols == 64 || kTmemCols == 128 || kTmemCols == 256 || kTmemCols == 512,
                  "TMEM allocation must be a power of two >= 32 columns");
    static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

// Error bits written to the device error word.
enum : int { kErrProducer = 1, kErrMma = 2, kErrEpilogue = 4, kErrProbe = 8 };

__device__ __forceinline__ void tile_coords(int t, const FusedParams& p, int& mb, int& nb) {
    // Groups of group_m row-blocks; inside a group the row-block varies fastest,
    // so a wave of CTAs covers a compact group_m x (wave/group_m) patch.
    const int group_tiles = p.group_m * p.tiles_n;
    const int g = t / group_tiles;
    const int first_m = g * p.group_m;
    const int gm = min(p.tiles_m - first_m, p.group_m);
    const int r = t - g * group_tiles;
    mb = first_m + r % gm;
    nb = r / gm;
}

__device__ __forceinline__ void raise_error(const FusedParams& p, volatile int* abort_flag, int bit) {
    atomicOr(p.err, bit);
    *abort_flag = 1;
}

// Applies the node's epilogue steps, in order, to 32 consecutive outputs of
// one row (cols col..col+31), exactly as eval_fused does per cell
// (graph.c:98-109): ADD adds the operand element, RELU is x > 0 ? x : 0.
// `prod` (pair kernel, DUAL) holds this chunk of the second product, added
// at the MXB_EP_ADD_PRODUCT step.
// A row segment of W floats at an address that is 4-byte but not 16-byte
// aligned (odd row pitches): PRE scalars up to the next 16-byte boundary,
// float4s in the middle, scalars for the tail; PRE is the segment's
// misalignment, so every index is a compile-time constant.
template <int W, int PRE>
__device__ __forceinline__ void add_segment(float (&v)[W], const float* src) {
#pragma unroll
    for (int i = 0; i < PRE; ++i) v[i] += __ldcs(src + i);
    constexpr int kG = (W - PRE) / 4;
#pragma unroll
    for (int g = 0; g < kG; ++g) {
        const float4 c = __ldcs(reinterpret_cast<const float4*>(src + PRE) + g);
        v[PRE + 4 * g + 0] += c.x;
        v[PRE + 4 * g + 1] += c.y;
        v[PRE + 4 * g + 2] += c.z;
        v[PRE + 4 * g + 3] += c.w;
    }
#pragma unroll
    for (int i = PRE + 4 * kG; i < W; ++i) v[i] += __ldcs(src + i);
}

template <int W, int PRE>
__device__ __forceinline__ void store_segment(const float (&v)[W], float* dst) {
#pragma unroll
    for (int i = 0; i < PRE; ++i) __stcs(dst + i, v[i]);
    constexpr int kG = (W - PRE) / 4;
#pragma unroll
    for (int g = 0; g < kG; ++g)
        __stcs(reinterpret_cast<float4*>(dst + PRE) + g,
               make_float4(v[PRE + 4 * g], v[PRE + 4 * g + 1], v[PRE + 4 * g + 2], v[PRE + 4 * g + 3]));
#pragma unroll
    for (int i = PRE + 4 * kG; i < W; ++i) __stcs(dst + i, v[i]);
}

// Scalars before the first 16-byte boundary of a 4-byte aligned address.
__device__ __forceinline__ int lead_scalars(const float* p) {
    return static_cast<int>((4 - ((reinterpret_cast<uintptr_t>(p) >> 2) & 3)) & 3);
}

template <int W = 32>
__device__ __forceinline__ void apply_epilogue(float (&v)[W], int row, int col, bool row_ok,
                                               const FusedParams& p, const float* prod = nullptr) {
    static_assert(W % 4 == 0, "whole float4 groups");
    const bool full_cols = col + W <= p.N;
    for (int s = 0; s < p.n_steps; ++s) {
        const int kind = p.steps[s].kind;
        const float* ptr = p.steps[s].ptr;
        if (kind == MXB_EP_ADD_PRODUCT) {
            if (prod) {
#pragma unroll
                for (int i = 0; i < W; ++i) v[i] += prod[i];
            }
        } else if (kind == MXB_EP_RELU) {
#pragma unroll
            for (int i = 0; i < W; ++i) v[i] = v[i] > 0.0f ? v[i] : 0.0f;
        } else if (kind == MXB_EP_SCALE) {
            const float sc = p.steps[s].scale;
#pragma unroll
            for (int i = 0; i < W; ++i) v[i] = v[i] * sc;
        } else if (kind == MXB_EP_ADD_FULL) {
            if (!row_ok) continue;
            const long long ld = p.steps[s].ld_or_size;
            const float* src = ptr + static_cast<long long>(row) * ld + col;
            if (full_cols && (ld & 3) == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
                const float4* s4 = reinterpret_cast<const float4*>(src);
#pragma unroll
                for (int i = 0; i < W / 4; ++i) {
                    const float4 c = __ldcs(s4 + i);
                    v[4 * i + 0] += c.x;
                    v[4 * i + 1] += c.y;
                    v[4 * i + 2] += c.z;
                    v[4 * i + 3] += c.w;
                }
            } else if (full_cols) {
                switch (lead_scalars(src)) {
                    case 0: add_segment<W, 0>(v, src); break;
                    case 1: add_segment<W, 1>(v, src); break;
                    case 2: add_segment<W, 2>(v, src); break;
                    default: add_segment<W, 3>(v, src); break;
                }
            } else {
#pragma unroll
                for (int i = 0; i < W; ++i)
                    if (col + i < p.N) v[i] += __ldg(src + i);
            }
        } else if (kind == MXB_EP_ADD_ROW) {
            const float* src = ptr + col;
            if (full_cols && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
                const float4* s4 = reinterpret_cast<const float4*>(src);
#pragma unroll
                for (int i = 0; i < W / 4; ++i) {
                    const float4 c = __ldg(s4 + i);
                    v[4 * i + 0] += c.x;
                    v[4 * i + 1] += c.y;
                    v[4 * i + 2] += c.z;
                    v[4 * i + 3] += c.w;
                }
            } else {
#pragma unroll
                for (int i = 0; i < W; ++i)
                    if (col + i < p.N) v[i] += __ldg(src + i);
            }
        } else if (kind == MXB_EP_ADD_MOD) {
            if (!row_ok) continue;
            const unsigned long long size = static_cast<unsigned long long>(p.steps[s].ld_or_size);
            const unsigned long long base =
                static_cast<unsigned long long>(row + p.row_base) * static_cast<unsigned long long>(p.N) + col;
#pragma unroll
            for (int i = 0; i < W; ++i)
                if (col + i < p.N) v[i] += __ldg(ptr + (base + i) % size);
        }
    }
}

template <int W = 32>
__device__ __forceinline__ void store_row_chunk(const float (&v)[W], int row, int col,
                                                const FusedParams& p) {
    float* dst = p.out + static_cast<long long>(row) * p.ldo + col;
    if (col + W <= p.N && (p.ldo & 3) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
        for (int i = 0; i < W / 4; ++i)
            __stcs(d4 + i, make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]));
    } else if (col + W <= p.N) {
        // Odd row pitch: align each row's segment on its own.
        switch (lead_scalars(dst)) {
            case 0: store_segment<W, 0>(v, dst); break;
            case 1: store_segment<W, 1>(v, dst); break;
            case 2: store_segment<W, 2>(v, dst); break;
            default: store_segment<W, 3>(v, dst); break;
        }
    } else {
#pragma unroll
        for (int i = 0; i < W; ++i)
            if (col + i < p.N) dst[i] = v[i];
    }
}

// Pulls this thread's rows of every full-matrix ADD operand, columns
// col .. col + ncols, into L2 ahead of the epilogue's loads.
__device__ __forceinline__ void prefetch_full_operands(int row, int col, int ncols, const FusedParams& p) {
    for (int s = 0; s < p.n_steps; ++s) {
        if (p.steps[s].kind != MXB_EP_ADD_FULL) continue;
        const float* src = p.steps[s].ptr + static_cast<long long>(row) * p.steps[s].ld_or_size + col;
        for (int c = 0; c < ncols; c += 32)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<uint64_t>(src + c)));
    }
}

template <int BN, int STAGES, bool SPLIT3, bool SEG>
__global__ void __launch_bounds__(kThreads, 1)
    fused_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                      const __grid_constant__ FusedParams p) {
    using C = Cfg<BN, STAGES, SPLIT3>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOffset);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::kNumBars);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const uint32_t bar0 = smem_addr(bars);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
    auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
    auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + 2 + a); };
    const uint32_t drain_bar = bar0 + 8u * (2 * STAGES + 4);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull_bar(a), 1);
            mbar_init(tempty_bar(a), 128);
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        if (SPLIT3) {
            tma_prefetch_desc(&tmA2);
            tma_prefetch_desc(&tmB2);
        }
    }
    if (warp == 1) {
        tmem_alloc(smem_addr(tmem_slot), C::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            long long issued = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
                int mb, nb;
                tile_coords(t, p, mb, nb);
                const int m0 = mb * kBM, n0 = nb * BN;
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (*abort_flag) { ok = false; break; }
                    if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.timeout_ns)) {
                        raise_error(p, abort_flag, kErrProducer);
                        ok = false;
                        break;
                    }
                    uint8_t* st = smem + stage * C::kStageBytes;
                    const uint32_t fb = full_bar(stage);
                    mbar_arrive_expect_tx(fb, C::kStageBytes);
                    const int k0 = kb * kBK;
                    tma_load_2d(smem_addr(st), &tmA, fb, k0, m0);
#pragma unroll
                    for (int j = 0; j < BN / 32; ++j)
                        tma_load_2d(smem_addr(st + C::kABytes + j * kBoxBytes), &tmB, fb, n0 + 32 * j, k0);
                    if (SPLIT3) {
                        uint8_t* st2 = st + C::kOperandBytes;
                        tma_load_2d(smem_addr(st2), &tmA2, fb, k0, m0);
#pragma unroll
                        for (int j = 0; j < BN / 32; ++j)
                            tma_load_2d(smem_addr(st2 + C::kABytes + j * kBoxBytes), &tmB2, fb,
                                        n0 + 32 * j, k0);
                    }
                    ++issued;
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
            }
            if (!ok) {
                // Let the copies still in flight land before the CTA leaves.
                const long long n = issued < STAGES ? issued : STAGES;
                for (long long i = 1; i <= n; ++i) {
                    const long long idx = issued - i;
                    const int s = static_cast<int>(idx % STAGES);
                    const uint32_t ph = static_cast<uint32_t>((idx / STAGES) & 1);
                    mbar_wait(full_bar(s), ph, p.timeout_ns);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_tf32(kBM, BN);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
                for (int k_begin = 0; k_begin < p.num_kb && ok; k_begin += p.seg_kb) {
                    const int k_end = min(p.num_kb, k_begin + p.seg_kb);
                    if (*abort_flag) { ok = false; break; }
                    if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, p.timeout_ns)) {
                        raise_error(p, abort_flag, kErrMma);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                    for (int kb = k_begin; kb < k_end; ++kb) {
                        if (!mbar_wait(full_bar(stage), phase, p.timeout_ns)) {
                            raise_error(p, abort_flag, kErrMma);
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t a_addr = smem_addr(smem + stage * C::kStageBytes);
                        const uint32_t b_addr = a_addr + C::kABytes;
#pragma unroll
                        for (int kk = 0; kk < kBK / 8; ++kk) {
                            // A: K-major, advance 8 fp32 = 32 bytes inside the swizzled row.
                            const uint64_t da = smem_desc(a_addr + kk * 32, 16, 1024, kLayoutSW128);
                            // B: MN-major, advance 8 k-rows = 1 KiB; 4-row atoms 512 B apart,
                            // 32-column boxes 4 KiB apart.
                            const uint64_t db = smem_desc(b_addr + kk * 1024, kBoxBytes, 512, kLayoutSW128Base32B);
                            const uint32_t accumulate = (kb != k_begin || kk != 0) ? 1u : 0u;
                            if (SPLIT3) {
                                const uint64_t da2 =
                                    smem_desc(a_addr + C::kOperandBytes + kk * 32, 16, 1024, kLayoutSW128);
                                const uint64_t db2 = smem_desc(b_addr + C::kOperandBytes + kk * 1024, kBoxBytes,
                                                               512, kLayoutSW128Base32B);
                                // Small cross terms first, the dominant big*big product last.
                                mma_tf32(d_tmem, da, db2, idesc, accumulate);
                                mma_tf32(d_tmem, da2, db, idesc, 1u);
                                mma_tf32(d_tmem, da, db, idesc, 1u);
                            } else {
                                mma_tf32(d_tmem, da, db, idesc, accumulate);
                            }
                        }
                        mma_commit(empty_bar(stage));
                        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                    }
                    if (!ok) break;
                    mma_commit(tfull_bar(acc));
                    acc ^= 1;
                    if (acc == 0) acc_phase ^= 1u;
                }
            }
            // All MMAs issued by this thread must finish before TMEM is freed.
            mma_commit(drain_bar);
            if (!mbar_wait(drain_bar, 0, p.timeout_ns)) raise_error(p, abort_flag, kErrMma);
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const int quad = warp & 3;  // TMEM lane quadrant this warp may access
        const int row_in_tile = quad * 32 + lane;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
            int mb, nb;
            tile_coords(t, p, mb, nb);
            const int row = mb * kBM + row_in_tile;
            const bool row_ok = row < p.M;
            const int col0 = nb * BN;
            int chunks = (p.N - col0 + 31) / 32;
            if (chunks > BN / 32) chunks = BN / 32;
            const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
            bool failed = false;
            if (row_ok) {
                // Short k-loops: fetch C while the MMAs run; long ones: just before the drain.
                if (p.num_kb <= kShortKb) prefetch_full_operands(row, col0, min(BN, p.N - col0), p);
            }
            if (SEG) {
                // Sum the K segments in registers (fp32, round to nearest), 16
                // columns at a time.  After the last segment the totals go back
                // into that accumulator and the epilogue reads them from there,
                // with the registers free.
                float total[BN];
                for (int k_begin = 0; k_begin < p.num_kb; k_begin += p.seg_kb) {
                    const bool first = k_begin == 0;
                    const bool last = k_begin + p.seg_kb >= p.num_kb;
                    const bool stop = __any_sync(0xffffffffu, *abort_flag != 0);
                    const bool got = !stop && mbar_wait(tfull_bar(acc), acc_phase, p.timeout_ns);
                    if (!__all_sync(0xffffffffu, got)) {
                        if (lane == 0 && !stop) raise_error(p, abort_flag, kErrEpilogue);
                        failed = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t taddr = lane_base + static_cast<uint32_t>(acc * BN);
#pragma unroll
                    for (int g = 0; g < BN / 16; ++g) {
                        uint32_t r[16];
                        tmem_ld_32x32b_x16(taddr + 16 * g, r);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 16; ++i)
                            total[16 * g + i] = first ? __uint_as_float(r[i]) : total[16 * g + i] + __uint_as_float(r[i]);
                        if (last) {
#pragma unroll
                            for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(total[16 * g + i]);
                            tmem_st_32x32b_x16(taddr + 16 * g, r);
                        }
                    }
                    if (last) {
                        tmem_st_wait();
                        for (int c = 0; c < chunks; ++c) {
                            uint32_t r[32];
                            tmem_ld_32x32b_x32(taddr + 32 * c, r);
                            tmem_ld_wait();
                            float v[32];
#pragma unroll
                            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
                            const int col = col0 + 32 * c;
                            apply_epilogue(v, row, col, row_ok, p);
                            if (row_ok) store_row_chunk(v, row, col, p);
                        }
                    }
                    tc_fence_before();
                    mbar_arrive(tempty_bar(acc));
                    acc ^= 1;
                    if (acc == 0) acc_phase ^= 1u;
                }
                if (failed) break;
            } else {
                const bool stop = __any_sync(0xffffffffu, *abort_flag != 0);
                const bool got = !stop && mbar_wait(tfull_bar(acc), acc_phase, p.timeout_ns);
                if (!__all_sync(0xffffffffu, got)) {
                    if (lane == 0 && !stop) raise_error(p, abort_flag, kErrEpilogue);
                    break;
                }
                tc_fence_after();
                if (row_ok && p.num_kb > kShortKb) prefetch_full_operands(row, col0, min(BN, p.N - col0), p);
                const uint32_t taddr = lane_base + static_cast<uint32_t>(acc * BN);
                for (int c = 0; c < chunks; ++c) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(taddr + 32 * c, r);
                    tmem_ld_wait();
                    if (c == chunks - 1) {
                        // Accumulator fully read: hand it back to the MMA warp.
                        tc_fence_before();
                        mbar_arrive(tempty_bar(acc));
                    }
                    float v[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
                    const int col = col0 + 32 * c;
                    apply_epilogue(v, row, col, row_ok, p);
                    if (row_ok) store_row_chunk(v, row, col, p);
                }
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1u;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::kTmemCols);
    }
}

// ------------------------------------------------------------------ CTA-pair kernel (TF32)
//
// Pair tile 256 x BN on a 2-CTA cluster (the two SMs of a TPC).  CTA r owns
// output rows m0 + 128 r .. +128; per k-block it stages its 128 rows of A and
// B columns n0 + (BN/2) r .. +BN/2 (half of the tile's B).  The leader (rank
// 0) issues tcgen05.mma.cta_group::2 (M=256, N=BN, K=8), which reads the A
// and B halves from both CTAs' shared memory and leaves each CTA's 128 x BN
// accumulator in that CTA's TMEM.  Per SM that halves the B bytes staged and
// read per MMA: with BN = 256 a stage is 32 KiB and six stages fit.  With
// BN = 512 the leader issues two N = 256 MMAs per k step, each into its own
// 256 accumulator columns; CTA r stages, for MMA h, B columns
// nb*512 + 256 h + 128 r .. +128, so accumulator column c is output column
// nb*512 + c.  A stage is 48 KiB (four fit) and the 512 columns leave one
// TMEM buffer: the epilogue drains it before the next tile starts.
//
// DUAL: the node's epilogue holds one step that adds a second product
// A @ B2 with the same A (a bare matmul on the same left operand whose only
// consumer is this node: config 4's relu(h W2 + b2) + h W2').  Each k-block
// stages A once with the B and B2 halves; the MMA warp issues A.B into
// accumulator 0 and A.B2 into accumulator 1 next to it in TMEM; the epilogue
// reads both and adds the second where the step stands.  The second product
// never goes to HBM and A is read once for both.  With BN = 128 a stage holds
// the same 32 KiB as the BN = 256 single product (A 16 KiB + two 8 KiB B
// halves), and the two accumulators of both TMEM buffers fill the 512
// columns, so the epilogue still overlaps the next tile's k-loop.
//
// Barriers: full[s] lives in the leader and counts both CTAs' TMA bytes (the
// peer's loads signal it through its cluster address); empty[s] and tfull[a]
// live in both CTAs and receive the leader's multicast commits; tempty[a]
// lives in the leader and takes one arrival per epilogue warp of either CTA.

template <int STAGES, int BN, bool DUAL, int EPI = 4>
struct PairCfg {
    static_assert(EPI == 4 || EPI == 8, "epilogue warps: one or two per TMEM lane quadrant");
    static constexpr int kThreadsPerCta = 64 + 32 * EPI;         // TMA warp, MMA warp, epilogue warps
    static constexpr int kABytes = 128 * kBK * 4;                // 16 KiB: this CTA's A rows
    static constexpr int kBBytes = (BN / 2) * kBK * 4;           // this CTA's B columns (per product)
    static constexpr int kStageBytes = kABytes + (DUAL ? 2 : 1) * kBBytes;
    // One MMA covers at most N = 256: wider tiles issue BN / 256 of them per
    // k step, each on its own 256 accumulator columns.
    static constexpr int kSubN = BN < 256 ? BN : 256;
    static constexpr int kSubs = BN / kSubN;
    static constexpr int kSubBoxes = kSubN / 64;                 // 32-column B boxes per CTA per sub-MMA
    static constexpr int kAccCols = (DUAL ? 2 : 1) * BN;         // TMEM columns of one tile's accumulators
    static constexpr int kBufs = kAccCols <= 256 ? 2 : 1;        // accumulator buffers in TMEM
    static constexpr int kTmemCols = kBufs * kAccCols;
    static constexpr int kBarOffset = STAGES * kStageBytes;
    static constexpr int kNumBars = 2 * STAGES + 5;
    static constexpr int kSmemBytes = 1024 + kBarOffset + kNumBars * 8 + 16;
    static_assert(BN == 128 || BN == 256 || BN == 512, "pair tile width");
    static_assert(!(DUAL && BN == 512), "two products use 128- or 256-column tiles");
    static_assert(kStageBytes % 1024 == 0, "stages must keep 1 KiB swizzle alignment");
    static_assert(kTmemCols == 256 || kTmemCols == 512, "TMEM allocation");
    static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

template <int STAGES, int BN, bool DUAL, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PairCfg<STAGES, BN, DUAL, EPI>::kThreadsPerCta, 1)
    fused_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                           const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                           const __grid_constant__ FusedParams p) {
    using C = PairCfg<STAGES, BN, DUAL, EPI>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOffset);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::kNumBars);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const uint32_t bar0 = smem_addr(bars);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
    auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
    auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + 2 + a); };
    const uint32_t drain_bar = bar0 + 8u * (2 * STAGES + 4);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair = blockIdx.x >> 1;
    const int num_pairs = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull_bar(a), 1);
            mbar_init(tempty_bar(a), 2 * EPI);  // every epilogue warp of the two CTAs
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        if (DUAL) {
            tma_prefetch_desc(&tmA2);
            tma_prefetch_desc(&tmB2);
        }
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_addr(tmem_slot), C::kTmemCols);
        tmem_relinquish_pair();
    }
    __syncwarp();
    tc_fence_before();
    cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer (both CTAs)
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            long long issued = 0;
            bool ok = true;
            for (int t = pair; t < p.num_tiles && ok; t += num_pairs) {
                int mb, nb;
                tile_coords(t, p, mb, nb);
                const int m0 = mb * 256 + static_cast<int>(rank) * 128;
                // CTA r stages, for sub-MMA h, B columns nb*BN + h*kSubN + r*kSubN/2 ..
                // + kSubN/2, so accumulator column c is output column nb*BN + c.
                const int n0 = nb * BN + static_cast<int>(rank) * (C::kSubN / 2);
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (*abort_flag) { ok = false; break; }
                    if (!mbar_wait_cluster(empty_bar(stage), phase ^ 1u, p.timeout_ns)) {
                        raise_error(p, abort_flag, kErrProducer);
                        ok = false;
                        break;
                    }
                    uint8_t* st = smem + stage * C::kStageBytes;
                    if (rank == 0) mbar_arrive_expect_tx(full_bar(stage), 2 * C::kStageBytes);
                    const uint32_t fb = mapa_shared(full_bar(stage), 0);
                    const int k0 = kb * kBK;
                    tma_load_2d_pair(smem_addr(st), &tmA, fb, k0, m0);
#pragma unroll
                    for (int j = 0; j < BN / 64; ++j)
                        tma_load_2d_pair(smem_addr(st + C::kABytes + j * kBoxBytes), &tmB, fb,
                                         n0 + (j / C::kSubBoxes) * C::kSubN + 32 * (j % C::kSubBoxes), k0);
                    if (DUAL) {
#pragma unroll
                        for (int j = 0; j < BN / 64; ++j)
                            tma_load_2d_pair(smem_addr(st + C::kABytes + C::kBBytes + j * kBoxBytes), &tmB2, fb,
                                             n0 + 32 * j, k0);
                    }
                    ++issued;
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
            }
            if (!ok && rank == 0) {
                // The leader's full barriers count both CTAs' bytes: wait for the copies in flight.
                const long long n = issued < STAGES ? issued : STAGES;
                for (long long i = 1; i <= n; ++i) {
                    const long long idx = issued - i;
                    mbar_wait_cluster(full_bar(static_cast<int>(idx % STAGES)),
                                      static_cast<uint32_t>((idx / STAGES) & 1), p.timeout_ns);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer (leader only)
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = idesc_tf32(256, C::kSubN);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int t = pair; t < p.num_tiles && ok; t += num_pairs) {
                if (*abort_flag) break;
                if (!mbar_wait_cluster(tempty_bar(acc), acc_phase ^ 1u, p.timeout_ns)) {
                    raise_error(p, abort_flag, kErrMma);
                    break;
                }
                tc_fence_after();
                const uint32_t d_tile = tmem_base + static_cast<uint32_t>(acc * C::kAccCols);
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait_cluster(full_bar(stage), phase, p.timeout_ns)) {
                        raise_error(p, abort_flag, kErrMma);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_addr(smem + stage * C::kStageBytes);
                    const uint32_t b_addr = a_addr + C::kABytes;
#pragma unroll
                    for (int kk = 0; kk < kBK / 8; ++kk) {
                        const uint64_t da = smem_desc(a_addr + kk * 32, 16, 1024, kLayoutSW128);
                        const uint64_t db = smem_desc(b_addr + kk * 1024, kBoxBytes, 512, kLayoutSW128Base32B);
                        const uint32_t accumulate = (kb | kk) != 0 ? 1u : 0u;
                        mma_tf32_pair(d_tile, da, db, idesc, accumulate);
#pragma unroll
                        for (int h = 1; h < C::kSubs; ++h) {
                            const uint64_t dbh = smem_desc(b_addr + h * C::kSubBoxes * kBoxBytes + kk * 1024,
                                                           kBoxBytes, 512, kLayoutSW128Base32B);
                            mma_tf32_pair(d_tile + h * C::kSubN, da, dbh, idesc, accumulate);
                        }
                        if (DUAL) {
                            const uint64_t db2 =
                                smem_desc(b_addr + C::kBBytes + kk * 1024, kBoxBytes, 512, kLayoutSW128Base32B);
                            mma_tf32_pair(d_tile + BN, da, db2, idesc, accumulate);
                        }
                    }
                    mma_commit_pair(empty_bar(stage), 0x3);
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
                if (!ok) break;
                mma_commit_pair(tfull_bar(acc), 0x3);
                if (C::kBufs == 2) acc ^= 1;
                if (acc == 0) acc_phase ^= 1u;
            }
            mma_commit_pair(drain_bar, 0x1);
            if (!mbar_wait_cluster(drain_bar, 0, p.timeout_ns)) raise_error(p, abort_flag, kErrMma);
        }
    } else {
        // ------------------------------------------------------------ epilogue (both CTAs)
        // Warp w reads TMEM lane quadrant w % 4; with EPI = 8 the two warps of a
        // quadrant split the tile's columns in halves.
        const int quad = warp & 3;
        constexpr int kChunksPerWarp = BN / 32 / (EPI / 4);
        const int c_first = ((warp - 2) >> 2) * kChunksPerWarp;
        const int row_in_tile = static_cast<int>(rank) * 128 + quad * 32 + lane;
        const uint32_t tempty_leader0 = mapa_shared(tempty_bar(0), 0);
        const uint32_t tempty_leader1 = mapa_shared(tempty_bar(1), 0);
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int t = pair; t < p.num_tiles; t += num_pairs) {
            int mb, nb;
            tile_coords(t, p, mb, nb);
            const int row = mb * 256 + row_in_tile;
            const bool row_ok = row < p.M;
            const int col0 = nb * BN;
            int chunks = (p.N - col0 + 31) / 32;
            if (chunks > c_first + kChunksPerWarp) chunks = c_first + kChunksPerWarp;
            // C rows into L2: during the k-loop when it is short, else once the accumulator is ready.
            const bool fetch = row_ok && chunks > c_first;
            if (fetch && p.num_kb <= kShortKb)
                prefetch_full_operands(row, col0 + 32 * c_first, 32 * (chunks - c_first), p);
            const bool stop = __any_sync(0xffffffffu, *abort_flag != 0);
            const bool got = !stop && mbar_wait_cluster(tfull_bar(acc), acc_phase, p.timeout_ns);
            if (!__all_sync(0xffffffffu, got)) {
                if (lane == 0 && !stop) raise_error(p, abort_flag, kErrEpilogue);
                break;
            }
            tc_fence_after();
            if (fetch && p.num_kb > kShortKb)
                prefetch_full_operands(row, col0 + 32 * c_first, 32 * (chunks - c_first), p);
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                                   static_cast<uint32_t>(acc * C::kAccCols);
            if (chunks <= c_first) {
                // No columns of this tile for this warp: release the accumulator at once.
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(acc ? tempty_leader1 : tempty_leader0);
            }
            for (int c = c_first; c < chunks; ++c) {
                uint32_t r[32];
                float w[32];
                tmem_ld_32x32b_x32(taddr + 32 * c, r);
                if (DUAL) {
                    uint32_t r2[32];
                    tmem_ld_32x32b_x32(taddr + BN + 32 * c, r2);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; ++i) w[i] = __uint_as_float(r2[i]);
                } else {
                    tmem_ld_wait();
                }
                if (c == chunks - 1) {
                    // This warp is done with the accumulator: tell the leader's MMA warp.
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(acc ? tempty_leader1 : tempty_leader0);
                }
                float v[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
                const int col = col0 + 32 * c;
                if (DUAL)
                    apply_epilogue(v, row, col, row_ok, p, w);
                else
                    apply_epilogue(v, row, col, row_ok, p);
                if (row_ok) store_row_chunk(v, row, col, p);
            }
            if (C::kBufs == 2) acc ^= 1;
            if (acc == 0) acc_phase ^= 1u;
        }
    }

    __syncwarp();
    tc_fence_before();
    cluster_sync();  // no CTA leaves while its peer may still signal its barriers
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, C::kTmemCols);
    }
}

// ------------------------------------------------------------------ CTA-pair kernel (3xTF32)
//
// The exact-fp32 mode on the 256 x 256 pair tile.  Per k-block each CTA stages
// its 128 A rows and its 128 of the tile's B columns twice -- big through the
// rounding maps of A and B themselves, small (x - big) from the pre-pass --
// 64 KiB, three stages.  The leader issues big*small, small*big and big*big
// per 8-wide k step (M=256, N=256, cta_group::2) into one TMEM accumulator.
// As in the single-CTA kernel, K is accumulated in segments of kSegKb
// k-blocks, each in a fresh accumulator (two 256-column buffers), because
// the tensor core's fp32 accumulation truncates toward zero; eight epilogue
// warps sum the segments in fp32 registers with round-to-nearest: warp w
// reads TMEM lane quadrant w % 4 and column half (w - 2) / 4, so each thread
// keeps 128 running totals.  Per SM this stages the same A bytes as the
// single-CTA kernel for twice the columns.
//
// DUAL: a second product A @ B2 on the same A (the two-product form of the
// TF32 pair kernel).  The tile is 256 x 128 per product: a stage holds A's
// big and small parts with 64-column halves of B and B2 (64 KiB again), the
// leader issues the three MMAs (N=128) for each product, and each segment
// buffer holds both 128-column accumulators.  Warp w of column half h sums
// columns 64h .. 64h+63 of both products, so the epilogue finds A.B and
// A.B2 of the same output columns in one thread.

constexpr int kPair3Threads = 320;  // TMA warp, MMA warp, 8 epilogue warps

template <int STAGES, bool DUAL>
struct Pair3Cfg {
    static constexpr int kBN = DUAL ? 128 : 256;           // output columns of the pair tile
    static constexpr int kProducts = DUAL ? 2 : 1;
    static constexpr int kABytes = 128 * kBK * 4;          // 16 KiB: this CTA's A rows
    static constexpr int kBBytes = (kBN / 2) * kBK * 4;    // this CTA's B columns, per product
    static constexpr int kOperandBytes = kABytes + kProducts * kBBytes;
    static constexpr int kStageBytes = 2 * kOperandBytes;  // big parts, then small parts
    static constexpr int kTmemCols = 512;                  // two segment buffers of 256 columns
    static constexpr int kBarOffset = STAGES * kStageBytes;
    static constexpr int kNumBars = 2 * STAGES + 5;
    static constexpr int kSmemBytes = 1024 + kBarOffset + kNumBars * 8 + 16;
    static_assert(kProducts * kBN == 256, "a segment buffer is 256 columns");
    static_assert(kStageBytes % 1024 == 0, "stages must keep 1 KiB swizzle alignment");
    static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

template <int STAGES, bool DUAL>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPair3Threads, 1)
    fused_gemm_pair3_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                            const __grid_constant__ CUtensorMap tmAs, const __grid_constant__ CUtensorMap tmBs,
                            const __grid_constant__ CUtensorMap tmB2, const __grid_constant__ CUtensorMap tmB2s,
                            const __grid_constant__ FusedParams p) {
    using C = Pair3Cfg<STAGES, DUAL>;
    constexpr int BN = C::kBN;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOffset);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::kNumBars);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const uint32_t bar0 = smem_addr(bars);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
    auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
    auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + 2 + a); };
    const uint32_t drain_bar = bar0 + 8u * (2 * STAGES + 4);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair = blockIdx.x >> 1;
    const int num_pairs = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull_bar(a), 1);
            mbar_init(tempty_bar(a), 16);  // 8 epilogue warps in each of the two CTAs
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        tma_prefetch_desc(&tmAs);
        tma_prefetch_desc(&tmBs);
        if (DUAL) {
            tma_prefetch_desc(&tmB2);
            tma_prefetch_desc(&tmB2s);
        }
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_addr(tmem_slot), C::kTmemCols);
        tmem_relinquish_pair();
    }
    __syncwarp();
    tc_fence_before();
    cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer (both CTAs)
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            long long issued = 0;
            bool ok = true;
            for (int t = pair; t < p.num_tiles && ok; t += num_pairs) {
                int mb, nb;
                tile_coords(t, p, mb, nb);
                const int m0 = mb * 256 + static_cast<int>(rank) * 128;
                const int n0 = nb * BN + static_cast<int>(rank) * (BN / 2);
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (*abort_flag) { ok = false; break; }
                    if (!mbar_wait_cluster(empty_bar(stage), phase ^ 1u, p.timeout_ns)) {
                        raise_error(p, abort_flag, kErrProducer);
                        ok = false;
                        break;
                    }
                    uint8_t* st = smem + stage * C::kStageBytes;
                    uint8_t* st2 = st + C::kOperandBytes;
                    if (rank == 0) mbar_arrive_expect_tx(full_bar(stage), 2 * C::kStageBytes);
                    const uint32_t fb = mapa_shared(full_bar(stage), 0);
                    const int k0 = kb * kBK;
                    tma_load_2d_pair(smem_addr(st), &tmA, fb, k0, m0);
                    tma_load_2d_pair(smem_addr(st2), &tmAs, fb, k0, m0);
#pragma unroll
                    for (int j = 0; j < BN / 64; ++j) {
                        tma_load_2d_pair(smem_addr(st + C::kABytes + j * kBoxBytes), &tmB, fb, n0 + 32 * j, k0);
                        tma_load_2d_pair(smem_addr(st2 + C::kABytes + j * kBoxBytes), &tmBs, fb, n0 + 32 * j, k0);
                        if (DUAL) {
                            tma_load_2d_pair(smem_addr(st + C::kABytes + C::kBBytes + j * kBoxBytes), &tmB2, fb,
                                             n0 + 32 * j, k0);
                            tma_load_2d_pair(smem_addr(st2 + C::kABytes + C::kBBytes + j * kBoxBytes), &tmB2s, fb,
                                             n0 + 32 * j, k0);
                        }
                    }
                    ++issued;
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
            }
            if (!ok && rank == 0) {
                // The leader's full barriers count both CTAs' bytes: wait for the copies in flight.
                const long long n = issued < STAGES ? issued : STAGES;
                for (long long i = 1; i <= n; ++i) {
                    const long long idx = issued - i;
                    mbar_wait_cluster(full_bar(static_cast<int>(idx % STAGES)),
                                      static_cast<uint32_t>((idx / STAGES) & 1), p.timeout_ns);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer (leader only)
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = idesc_tf32(256, BN);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int t = pair; t < p.num_tiles && ok; t += num_pairs) {
                for (int k_begin = 0; k_begin < p.num_kb && ok; k_begin += p.seg_kb) {
                    const int k_end = min(p.num_kb, k_begin + p.seg_kb);
                    if (*abort_flag) { ok = false; break; }
                    if (!mbar_wait_cluster(tempty_bar(acc), acc_phase ^ 1u, p.timeout_ns)) {
                        raise_error(p, abort_flag, kErrMma);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * 256);
                    for (int kb = k_begin; kb < k_end; ++kb) {
                        if (!mbar_wait_cluster(full_bar(stage), phase, p.timeout_ns)) {
                            raise_error(p, abort_flag, kErrMma);
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t a_addr = smem_addr(smem + stage * C::kStageBytes);
#pragma unroll
                        for (int kk = 0; kk < kBK / 8; ++kk) {
                            const uint64_t da = smem_desc(a_addr + kk * 32, 16, 1024, kLayoutSW128);
                            const uint64_t das =
                                smem_desc(a_addr + C::kOperandBytes + kk * 32, 16, 1024, kLayoutSW128);
                            const uint32_t accumulate = (kb != k_begin || kk != 0) ? 1u : 0u;
#pragma unroll
                            for (int q = 0; q < C::kProducts; ++q) {
                                const uint32_t b_addr = a_addr + C::kABytes + q * C::kBBytes;
                                const uint64_t db =
                                    smem_desc(b_addr + kk * 1024, kBoxBytes, 512, kLayoutSW128Base32B);
                                const uint64_t dbs = smem_desc(b_addr + C::kOperandBytes + kk * 1024, kBoxBytes,
                                                               512, kLayoutSW128Base32B);
                                const uint32_t d = d_tmem + static_cast<uint32_t>(q * BN);
                                // Small cross terms first, the dominant big*big product last.
                                mma_tf32_pair(d, da, dbs, idesc, accumulate);
                                mma_tf32_pair(d, das, db, idesc, 1u);
                                mma_tf32_pair(d, da, db, idesc, 1u);
                            }
                        }
                        mma_commit_pair(empty_bar(stage), 0x3);
                        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                    }
                    if (!ok) break;
                    mma_commit_pair(tfull_bar(acc), 0x3);
                    acc ^= 1;
                    if (acc == 0) acc_phase ^= 1u;
                }
            }
            mma_commit_pair(drain_bar, 0x1);
            if (!mbar_wait_cluster(drain_bar, 0, p.timeout_ns)) raise_error(p, abort_flag, kErrMma);
        }
    } else {
        // ------------------------------------------------------------ epilogue (both CTAs, 8 warps)
        // Each thread sums 128 accumulator columns: columns 128h .. 128h+127
        // of the single product, or (DUAL) 64h .. 64h+63 of both products.
        const int quad = warp & 3;
        const int half = (warp - 2) >> 2;
        const int row_in_tile = static_cast<int>(rank) * 128 + quad * 32 + lane;
        const uint32_t tempty_leader0 = mapa_shared(tempty_bar(0), 0);
        const uint32_t tempty_leader1 = mapa_shared(tempty_bar(1), 0);
        const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
        // TMEM column of this thread's 16-column group g (0..7).
        auto group_col = [&](int g) -> uint32_t {
            return DUAL ? static_cast<uint32_t>((g >> 2) * BN + half * 64 + 16 * (g & 3))
                        : static_cast<uint32_t>(half * 128 + 16 * g);
        };
        int acc = 0;
        uint32_t acc_phase = 0;
        bool failed = false;
        for (int t = pair; t < p.num_tiles && !failed; t += num_pairs) {
            int mb, nb;
            tile_coords(t, p, mb, nb);
            const int row = mb * 256 + row_in_tile;
            const bool row_ok = row < p.M;
            const int col0 = nb * BN + half * (DUAL ? 64 : 128);  // first output column of this thread
            float total[128];
            for (int k_begin = 0; k_begin < p.num_kb; k_begin += p.seg_kb) {
                const bool first = k_begin == 0;
                const bool last = k_begin + p.seg_kb >= p.num_kb;
                const bool stop = __any_sync(0xffffffffu, *abort_flag != 0);
                const bool got = !stop && mbar_wait_cluster(tfull_bar(acc), acc_phase, p.timeout_ns);
                if (!__all_sync(0xffffffffu, got)) {
                    if (lane == 0 && !stop) raise_error(p, abort_flag, kErrEpilogue);
                    failed = true;
                    break;
                }
                tc_fence_after();
                const uint32_t taddr = lane_base + static_cast<uint32_t>(acc * 256);
                // 16 columns at a time: 128 totals + 16 loaded values stay in registers.
                // After the last segment the totals go back into this accumulator,
                // so the epilogue below runs with the registers free.
#pragma unroll
                for (int g = 0; g < 8; ++g) {
                    uint32_t r[16];
                    tmem_ld_32x32b_x16(taddr + group_col(g), r);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 16; ++i)
                        total[16 * g + i] = first ? __uint_as_float(r[i]) : total[16 * g + i] + __uint_as_float(r[i]);
                    if (last) {
#pragma unroll
                        for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(total[16 * g + i]);
                        tmem_st_32x32b_x16(taddr + group_col(g), r);
                    }
                }
                if (last) {
                    tmem_st_wait();
                    if (DUAL) {
                        // 16 columns of both products at a time.
                        for (int c = 0; c < 4; ++c) {
                            const int col = col0 + 16 * c;
                            if (col >= p.N) break;
                            uint32_t r[16], r2[16];
                            tmem_ld_32x32b_x16(taddr + group_col(c), r);
                            tmem_ld_32x32b_x16(taddr + group_col(4 + c), r2);
                            tmem_ld_wait();
                            float v[16], w[16];
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                v[i] = __uint_as_float(r[i]);
                                w[i] = __uint_as_float(r2[i]);
                            }
                            apply_epilogue<16>(v, row, col, row_ok, p, w);
                            if (row_ok) store_row_chunk<16>(v, row, col, p);
                        }
                    } else {
                        for (int c = 0; c < 4; ++c) {
                            const int col = col0 + 32 * c;
                            if (col >= p.N) break;
                            uint32_t r[32];
                            tmem_ld_32x32b_x32(taddr + group_col(2 * c), r);
                            tmem_ld_wait();
                            float v[32];
#pragma unroll
                            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
                            apply_epilogue(v, row, col, row_ok, p);
                            if (row_ok) store_row_chunk(v, row, col, p);
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(acc ? tempty_leader1 : tempty_leader0);
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1u;
            }
        }
    }

    __syncwarp();
    tc_fence_before();
    cluster_sync();  // no CTA leaves while its peer may still signal its barriers
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, C::kTmemCols);
    }
}

// ------------------------------------------------------------------ host side

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// Row-major [rows, cols] fp32 with row pitch `ld` elements; box [box_rows][box_cols].
bool make_map(CUtensorMap* map, const float* base, long long rows, long long cols, long long ld,
              int box_cols, int box_rows, CUtensorMapSwizzle swizzle) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 4};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    // TFLOAT32: TMA rounds each fp32 element to TF32 (nearest even) on load.
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_TFLOAT32, 2, const_cast<float*>(base), dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int BN, int STAGES, bool SPLIT3, bool SEG>
cudaError_t run_variant(const GemmLaunch& g, cudaStream_t stream) {
    using C = Cfg<BN, STAGES, SPLIT3>;
    auto kernel = fused_gemm_kernel<BN, STAGES, SPLIT3, SEG>;
    // The shared-memory opt-in is per device: remember which devices have it.
    static std::mutex mu;
    static uint64_t configured = 0;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (dev >= 64 || !(configured & (1ull << dev))) {
            e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
            if (e != cudaSuccess) return e;
            if (dev < 64) configured |= 1ull << dev;
        }
    }

    const float* a_hi = g.A;   // through the rounding map this is big = rne_tf32(A)
    const float* b_hi = g.B;
    CUtensorMap mA, mB, mA2, mB2;
    constexpr CUtensorMapSwizzle kSwA = CU_TENSOR_MAP_SWIZZLE_128B;
    constexpr CUtensorMapSwizzle kSwB = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
    if (!make_map(&mA, a_hi, g.M, g.K, g.lda, kBK, kBM, kSwA) || !make_map(&mB, b_hi, g.K, g.N, g.ldb, 32, kBK, kSwB))
        return cudaErrorInvalidValue;
    if (SPLIT3) {
        if (!make_map(&mA2, g.A_small, g.M, g.K, g.lda, kBK, kBM, kSwA) ||
            !make_map(&mB2, g.B_small, g.K, g.N, g.ldb, 32, kBK, kSwB))
            return cudaErrorInvalidValue;
    } else {
        mA2 = mA;
        mB2 = mB;
    }

    FusedParams p{};
    p.out = g.out;
    p.ldo = g.ldo;
    p.M = g.M;
    p.N = g.N;
    p.K = g.K;
    p.n_steps = g.n_steps;
    p.tiles_m = (g.M + kBM - 1) / kBM;
    p.tiles_n = (g.N + BN - 1) / BN;
    p.num_tiles = p.tiles_m * p.tiles_n;
    p.num_kb = (g.K + kBK - 1) / kBK;
    p.group_m = 16;
    p.seg_kb = SEG ? kSegKb : p.num_kb;
    p.row_base = g.row_base;
    p.timeout_ns = g.timeout_ns;
    p.err = g.err;
    for (int i = 0; i < g.n_steps; ++i) p.steps[i] = g.steps[i];

    const int grid = p.num_tiles < g.num_sms ? p.num_tiles : g.num_sms;
    kernel<<<grid, kThreads, C::kSmemBytes, stream>>>(mA, mB, mA2, mB2, p);
    note_launch();
    return cudaGetLastError();
}

template <int STAGES, int BN, bool DUAL, int EPI = 4>
cudaError_t run_pair_variant(const GemmLaunch& g, cudaStream_t stream) {
    using C = PairCfg<STAGES, BN, DUAL, EPI>;
    auto kernel = fused_gemm_pair_kernel<STAGES, BN, DUAL, EPI>;
    static std::mutex mu;
    static uint64_t configured = 0;
    static int max_clusters[64] = {0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    int clusters = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (dev >= 64 || !(configured & (1ull << dev))) {
            e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
            if (e != cudaSuccess) return e;
            // How many 2-CTA clusters fit at once with this much shared memory.
            cudaLaunchConfig_t cfg = {};
            cudaLaunchAttribute attr;
            attr.id = cudaLaunchAttributeClusterDimension;
            attr.val.clusterDim.x = 2;
            attr.val.clusterDim.y = 1;
            attr.val.clusterDim.z = 1;
            cfg.gridDim = dim3(2 * (g.num_sms / 2), 1, 1);
            cfg.blockDim = dim3(C::kThreadsPerCta, 1, 1);
            cfg.dynamicSmemBytes = C::kSmemBytes;
            cfg.attrs = &attr;
            cfg.numAttrs = 1;
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n < 1) {
                cudaGetLastError();
                n = g.num_sms / 2;
            }
            if (dev < 64) {
                max_clusters[dev] = n;
                configured |= 1ull << dev;
            }
            clusters = n;
        } else {
            clusters = max_clusters[dev];
        }
    }

    constexpr CUtensorMapSwizzle kSwA = CU_TENSOR_MAP_SWIZZLE_128B;
    constexpr CUtensorMapSwizzle kSwB = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
    CUtensorMap mA, mB, mA2, mB2;
    if (!make_map(&mA, g.A, g.M, g.K, g.lda, kBK, 128, kSwA) || !make_map(&mB, g.B, g.K, g.N, g.ldb, 32, kBK, kSwB))
        return cudaErrorInvalidValue;
    if (DUAL) {
        // The second product shares A (same rows, K and pitch); only B2 has a map of its own.
        if (g.A2 != g.A || g.K2 != g.K || g.lda2 != g.lda || !g.B2 ||
            !make_map(&mB2, g.B2, g.K, g.N, g.ldb2, 32, kBK, kSwB))
            return cudaErrorInvalidValue;
        mA2 = mA;
    } else {
        mA2 = mA;
        mB2 = mB;
    }

    FusedParams p{};
    p.out = g.out;
    p.ldo = g.ldo;
    p.M = g.M;
    p.N = g.N;
    p.K = g.K;
    p.n_steps = g.n_steps;
    p.tiles_m = (g.M + 255) / 256;
    p.tiles_n = (g.N + BN - 1) / BN;
    p.num_tiles = p.tiles_m * p.tiles_n;
    p.num_kb = (g.K + kBK - 1) / kBK;
    p.group_m = 8;
    p.seg_kb = p.num_kb;
    p.row_base = g.row_base;
    p.timeout_ns = g.timeout_ns;
    p.err = g.err;
    for (int i = 0; i < g.n_steps; ++i) p.steps[i] = g.steps[i];

    const int pairs = p.num_tiles < clusters ? p.num_tiles : clusters;
    kernel<<<2 * pairs, C::kThreadsPerCta, C::kSmemBytes, stream>>>(mA, mB, mA2, mB2, p);
    note_launch();
    return cudaGetLastError();
}

template <int STAGES, bool DUAL>
cudaError_t run_pair3_variant(const GemmLaunch& g, cudaStream_t stream) {
    using C = Pair3Cfg<STAGES, DUAL>;
    auto kernel = fused_gemm_pair3_kernel<STAGES, DUAL>;
    static std::mutex mu;
    static uint64_t configured = 0;
    static int max_clusters[64] = {0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    int clusters = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (dev >= 64 || !(configured & (1ull << dev))) {
            e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
            if (e != cudaSuccess) return e;
            cudaLaunchConfig_t cfg = {};
            cudaLaunchAttribute attr;
            attr.id = cudaLaunchAttributeClusterDimension;
            attr.val.clusterDim.x = 2;
            attr.val.clusterDim.y = 1;
            attr.val.clusterDim.z = 1;
            cfg.gridDim = dim3(2 * (g.num_sms / 2), 1, 1);
            cfg.blockDim = dim3(kPair3Threads, 1, 1);
            cfg.dynamicSmemBytes = C::kSmemBytes;
            cfg.attrs = &attr;
            cfg.numAttrs = 1;
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n < 1) {
                cudaGetLastError();
                n = g.num_sms / 2;
            }
            if (dev < 64) {
                max_clusters[dev] = n;
                configured |= 1ull << dev;
            }
            clusters = n;
        } else {
            clusters = max_clusters[dev];
        }
    }
    if (!g.A_small || !g.B_small) return cudaErrorInvalidValue;

    constexpr CUtensorMapSwizzle kSwA = CU_TENSOR_MAP_SWIZZLE_128B;
    constexpr CUtensorMapSwizzle kSwB = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
    CUtensorMap mA, mB, mAs, mBs, mB2, mB2s;
    if (!make_map(&mA, g.A, g.M, g.K, g.lda, kBK, 128, kSwA) || !make_map(&mB, g.B, g.K, g.N, g.ldb, 32, kBK, kSwB) ||
        !make_map(&mAs, g.A_small, g.M, g.K, g.lda, kBK, 128, kSwA) ||
        !make_map(&mBs, g.B_small, g.K, g.N, g.ldb, 32, kBK, kSwB))
        return cudaErrorInvalidValue;
    if (DUAL) {
        // The second product shares A (same rows, K and pitch); B2 and its low part have maps of their own.
        if (g.A2 != g.A || g.K2 != g.K || g.lda2 != g.lda || !g.B2 || !g.B2_small ||
            !make_map(&mB2, g.B2, g.K, g.N, g.ldb2, 32, kBK, kSwB) ||
            !make_map(&mB2s, g.B2_small, g.K, g.N, g.ldb2, 32, kBK, kSwB))
            return cudaErrorInvalidValue;
    } else {
        mB2 = mB;
        mB2s = mBs;
    }

    FusedParams p{};
    p.out = g.out;
    p.ldo = g.ldo;
    p.M = g.M;
    p.N = g.N;
    p.K = g.K;
    p.n_steps = g.n_steps;
    p.tiles_m = (g.M + 255) / 256;
    p.tiles_n = (g.N + C::kBN - 1) / C::kBN;
    p.num_tiles = p.tiles_m * p.tiles_n;
    p.num_kb = (g.K + kBK - 1) / kBK;
    p.group_m = 8;
    p.seg_kb = kSegKb;
    p.row_base = g.row_base;
    p.timeout_ns = g.timeout_ns;
    p.err = g.err;
    for (int i = 0; i < g.n_steps; ++i) p.steps[i] = g.steps[i];

    const int pairs = p.num_tiles < clusters ? p.num_tiles : clusters;
    kernel<<<2 * pairs, kPair3Threads, C::kSmemBytes, stream>>>(mA, mB, mAs, mBs, mB2, mB2s, p);
    note_launch();
    return cudaGetLastError();
}

// Which TF32 kernel: the CTA-pair kernel once there are enough 256 x 256
// tiles to occupy the SMs, else the single-CTA kernel (128 x 256 or 128 x 128
// tiles spread over more SMs).  MINIXLA_GEMM_VARIANT=pair|pair512|single
// overrides.
bool use_pair_kernel(const GemmLaunch& g) {
    if (const char* v = getenv("MINIXLA_GEMM_VARIANT")) {
        if (!strcmp(v, "pair") || !strcmp(v, "pair512")) return true;
        if (!strcmp(v, "single")) return false;
    }
    const long long pair_tiles = static_cast<long long>((g.M + 255) / 256) * ((g.N + 255) / 256);
    return g.M >= 256 && pair_tiles >= g.num_sms / 4;
}

// Tile width of the single-CTA kernels (128-row tiles): 256 once those tiles
// fill the GPU, else the widest of 128 / 64 / 32 that gives at least half
// the SMs a tile (32 when none does).  MINIXLA_SINGLE_BN forces one.
int single_cta_width(const GemmLaunch& g) {
    if (const char* v = getenv("MINIXLA_SINGLE_BN")) {
        const int w = atoi(v);
        if (w == 32 || w == 64 || w == 128 || w == 256) return w;
    }
    const long long tiles_m = (g.M + kBM - 1) / kBM;
    auto tiles = [&](int bn) { return tiles_m * ((g.N + bn - 1) / bn); };
    if (g.N > 128 && tiles(256) >= g.num_sms) return 256;
    for (int bn : {128, 64})
        if (tiles(bn) >= g.num_sms / 2) return bn;
    return 32;
}

// TF32 pair kernel with 256 x 512 tiles: per k-block each CTA stages 16 KiB
// of A and 32 KiB of B for eight 256 x 256 x 8 MMAs -- a quarter fewer bytes
// per MMA than the 256 x 256 tile, whose 32 KiB feed four.  The 512
// accumulator columns fill TMEM, so the epilogue no longer overlaps the next
// tile's k-loop (single buffer); it prefetches its rows of C into L2 first.
// Measured at 8192^3: 784 vs 712 TFLOP/s, and 693 vs 652 under the power
// cap.  (Eight epilogue warps instead of four drained no faster.)  Used once
// the wide tiles alone give every CTA pair a tile.
bool pair_wide_tiles(const GemmLaunch& g) {
    if (const char* v = getenv("MINIXLA_GEMM_VARIANT")) {
        if (!strcmp(v, "pair512")) return true;
        if (!strcmp(v, "pair")) return false;
    }
    const long long wide_tiles = static_cast<long long>((g.M + 255) / 256) * ((g.N + 511) / 512);
    return wide_tiles >= g.num_sms / 2;
}

}  // namespace

cudaError_t launch_fused_gemm(const GemmLaunch& g, cudaStream_t stream) {
    if (g.A2) {
        // Two products of one A in one kernel (callers run other cases as two launches).
        if (g.precision == GPU_PRECISION_3XTF32) return run_pair3_variant<3, true>(g, stream);
        // TF32: 256-column tiles put both accumulators in the 512 TMEM columns (one buffer,
        // 48 KiB stages); 128-column tiles keep two buffers for problems with few tiles.
        if (g.precision != GPU_PRECISION_TF32) return cudaErrorInvalidValue;
        const long long tiles256 = static_cast<long long>((g.M + 255) / 256) * ((g.N + 255) / 256);
        if (tiles256 >= g.num_sms / 2) return run_pair_variant<4, 256, true>(g, stream);
        return run_pair_variant<6, 128, true>(g, stream);
    }
    if (g.precision == GPU_PRECISION_3XTF32) {
        if (use_pair_kernel(g)) return run_pair3_variant<3, false>(g, stream);
        switch (single_cta_width(g)) {
            case 256:
            case 128: return run_variant<128, 3, true, true>(g, stream);
            case 64: return run_variant<64, 4, true, true>(g, stream);
            default: return run_variant<32, 5, true, true>(g, stream);
        }
    }
    if (use_pair_kernel(g)) {
        return pair_wide_tiles(g) ? run_pair_variant<4, 512, false>(g, stream)
                                  : run_pair_variant<6, 256, false>(g, stream);
    }
    // One TF32 product on one CTA.  Narrower tiles for problems with few
    // tiles, so more SMs share the k-loops and the epilogue.
    switch (single_cta_width(g)) {
        case 256: return run_variant<256, 4, false, false>(g, stream);
        case 128: return run_variant<128, 6, false, false>(g, stream);
        case 64: return run_variant<64, 8, false, false>(g, stream);
        default: return run_variant<32, 8, false, false>(g, stream);
    }
}

// ------------------------------------------------------------------ bounded-wait probe

namespace {
__global__ void wait_timeout_probe_kernel(int* err, unsigned long long timeout_ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(smem_addr(&bar), 1);
        fence_barrier_init();
        // Nothing ever arrives on this barrier: the wait must give up by itself.
        if (!mbar_wait(smem_addr(&bar), 0, timeout_ns)) atomicOr(err, kErrProbe);
    }
}
}  // namespace

cudaError_t launch_wait_timeout_probe(int* err, unsigned long long timeout_ns, cudaStream_t stream) {
    wait_timeout_probe_kernel<<<1, 32, 0, stream>>>(err, timeout_ns);
    note_launch();
    return cudaGetLastError();
}

// ------------------------------------------------------------------ timer hold
//
// Keeps the stream busy for about `ns` of global time (and at most 2^24
// polls), so that a start event recorded after it is stamped when the work
// behind it is already queued: kernel timers then measure the kernels, not
// the host's time to enqueue them.

namespace {
__global__ void hold_kernel(unsigned long long ns) {
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 0; it < (1u << 24); ++it)
        if (global_timer_ns() - t0 >= ns) break;
}
}  // namespace

cudaError_t launch_hold(unsigned long long ns, cudaStream_t stream) {
    hold_kernel<<<1, 1, 0, stream>>>(ns);
    return cudaGetLastError();
}

}  // namespace mxb
