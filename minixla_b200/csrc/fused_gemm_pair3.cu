// 3xTF32 CTA-pair kernels (cta_group::2): 256x256 tiles of one product and
// the two-product form on 256x128 tiles, K summed in segments.
#include "gemm_common.cuh"

namespace mxb {

namespace {

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

// The peer copies as a call of their own: this kernel runs at 168 registers
// a thread, and inlined they pushed the segment sums into local memory.
__device__ __noinline__ void push_rows_apart(const FusedParams& p, int row0, int c0, int c1) {
    push_rows<2>(p, row0, c0, c1);
}

// PUSH: after a tile's last segment each epilogue warp also copies its 32
// rows x 128 columns into the peers' copies (FusedParams::peer_out), with the
// accumulator already released; a separate instance keeps the others' code.
// BATCHED: p.batch products of one shape, A, B and their low parts as 3-D
// tensor maps (third coordinate: the product).
template <int STAGES, bool DUAL, bool PUSH = false, bool BATCHED = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPair3Threads, 1)
    fused_gemm_pair3_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                            const __grid_constant__ CUtensorMap tmAs, const __grid_constant__ CUtensorMap tmBs,
                            const __grid_constant__ CUtensorMap tmB2, const __grid_constant__ CUtensorMap tmB2s,
                            const __grid_constant__ FusedParams p) {
    using C = Pair3Cfg<STAGES, DUAL>;
    constexpr int BN = C::kBN;
    static_assert(!(PUSH && DUAL), "peer rows are written for one product");
    static_assert(!(BATCHED && (DUAL || PUSH)), "a batched launch has one product and no peer rows");
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
                int b = 0;
                if (BATCHED) {
                    b = t / p.tiles_per_batch;
                    tile_coords(t - b * p.tiles_per_batch, p, mb, nb);
                } else {
                    tile_coords(t, p, mb, nb);
                }
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
                    if (BATCHED) {
                        tma_load_3d_pair(smem_addr(st), &tmA, fb, k0, m0, b);
                        tma_load_3d_pair(smem_addr(st2), &tmAs, fb, k0, m0, b);
#pragma unroll
                        for (int j = 0; j < BN / 64; ++j) {
                            tma_load_3d_pair(smem_addr(st + C::kABytes + j * kBoxBytes), &tmB, fb, n0 + 32 * j, k0, b);
                            tma_load_3d_pair(smem_addr(st2 + C::kABytes + j * kBoxBytes), &tmBs, fb, n0 + 32 * j, k0,
                                             b);
                        }
                    } else {
                        tma_load_2d_pair(smem_addr(st), &tmA, fb, k0, m0);
                        tma_load_2d_pair(smem_addr(st2), &tmAs, fb, k0, m0);
#pragma unroll
                        for (int j = 0; j < BN / 64; ++j) {
                            tma_load_2d_pair(smem_addr(st + C::kABytes + j * kBoxBytes), &tmB, fb, n0 + 32 * j, k0);
                            tma_load_2d_pair(smem_addr(st2 + C::kABytes + j * kBoxBytes), &tmBs, fb, n0 + 32 * j,
                                             k0);
                            if (DUAL) {
                                tma_load_2d_pair(smem_addr(st + C::kABytes + C::kBBytes + j * kBoxBytes), &tmB2, fb,
                                                 n0 + 32 * j, k0);
                                tma_load_2d_pair(smem_addr(st2 + C::kABytes + C::kBBytes + j * kBoxBytes), &tmB2s,
                                                 fb, n0 + 32 * j, k0);
                            }
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
            int b = 0;
            if (BATCHED) {
                b = t / p.tiles_per_batch;
                tile_coords(t - b * p.tiles_per_batch, p, mb, nb);
            } else {
                tile_coords(t, p, mb, nb);
            }
            const long long out_off = BATCHED ? b * p.out_bstride : 0;
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
                            apply_epilogue(v, row, col, row_ok, p, nullptr, b);
                            if (row_ok) store_row_chunk(v, row, col, p, out_off);
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(acc ? tempty_leader1 : tempty_leader0);
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1u;
                if (PUSH && last) {
                    // Overlaps the next tile's MMAs: the accumulator is released.
                    const int c_end = col0 + 128 < p.N ? col0 + 128 : p.N;
                    push_rows_apart(p, mb * 256 + row_in_tile - lane, col0, c_end);
                }
            }
        }
        // Peer stores performed before the kernel counts as finished.
        if (PUSH) __threadfence_system();
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

template <int STAGES, bool DUAL, bool PUSH = false, bool BATCHED = false>
cudaError_t run_pair3_variant(const GemmLaunch& g, cudaStream_t stream) {
    using C = Pair3Cfg<STAGES, DUAL>;
    auto kernel = fused_gemm_pair3_kernel<STAGES, DUAL, PUSH, BATCHED>;
    if (BATCHED != (g.batch > 1)) return cudaErrorInvalidValue;
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
    if (BATCHED) {
        if (!make_map_3d(&mA, g.A, g.batch, g.M, g.K, g.lda, g.a_bstride, kBK, 128, kSwA) ||
            !make_map_3d(&mB, g.B, g.batch, g.K, g.N, g.ldb, g.b_bstride, 32, kBK, kSwB) ||
            !make_map_3d(&mAs, g.A_small, g.batch, g.M, g.K, g.lda, g.a_bstride, kBK, 128, kSwA) ||
            !make_map_3d(&mBs, g.B_small, g.batch, g.K, g.N, g.ldb, g.b_bstride, 32, kBK, kSwB))
            return cudaErrorInvalidValue;
    } else if (!make_map(&mA, g.A, g.M, g.K, g.lda, kBK, 128, kSwA) ||
               !make_map(&mB, g.B, g.K, g.N, g.ldb, 32, kBK, kSwB) ||
               !make_map(&mAs, g.A_small, g.M, g.K, g.lda, kBK, 128, kSwA) ||
               !make_map(&mBs, g.B_small, g.K, g.N, g.ldb, 32, kBK, kSwB)) {
        return cudaErrorInvalidValue;
    }
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
    if (PUSH != (g.n_peers > 0)) return cudaErrorInvalidValue;
    if (PUSH) {
        if (DUAL || g.n_peers > kMaxPeers || !g.peer_out) return cudaErrorInvalidValue;
        bool vec = (g.ldo & 3) == 0 && (reinterpret_cast<uintptr_t>(g.out) & 15) == 0;
        for (int i = 0; i < g.n_peers; ++i) {
            if (!g.peer_out[i]) return cudaErrorInvalidValue;
            p.peer_out[i] = g.peer_out[i];
            vec = vec && (reinterpret_cast<uintptr_t>(g.peer_out[i]) & 15) == 0;
        }
        p.n_peers = g.n_peers;
        p.push_vec = vec ? 1 : 0;
    }

    p.batch = 1;
    if (BATCHED) {
        const long long tiles = static_cast<long long>(p.num_tiles) * g.batch;
        if (tiles >= (1ll << 31) || !g.ep_bstride) return cudaErrorInvalidValue;
        p.batch = static_cast<int>(g.batch);
        p.tiles_per_batch = p.num_tiles;
        p.num_tiles = static_cast<int>(tiles);
        p.out_bstride = g.out_bstride;
        for (int i = 0; i < g.n_steps; ++i) p.ep_bstride[i] = g.ep_bstride[i];
    }

    const int pairs = p.num_tiles < clusters ? p.num_tiles : clusters;
    kernel<<<2 * pairs, kPair3Threads, C::kSmemBytes, stream>>>(mA, mB, mAs, mBs, mB2, mB2s, p);
    note_launch();
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_pair_3xtf32(const GemmLaunch& g, bool dual, cudaStream_t stream) {
    if (g.batch > 1) {
        if (dual || g.n_peers > 0) return cudaErrorInvalidValue;
        return run_pair3_variant<3, false, false, true>(g, stream);
    }
    if (g.n_peers > 0) return dual ? cudaErrorInvalidValue : run_pair3_variant<3, false, true>(g, stream);
    return dual ? run_pair3_variant<3, true>(g, stream) : run_pair3_variant<3, false>(g, stream);
}

}  // namespace mxb
