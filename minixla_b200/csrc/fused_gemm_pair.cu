// TF32 CTA-pair kernels (cta_group::2): 256x256 and 256x512 tiles of one
// product, and the two-product form on 128- or 256-wide tiles.
#include "gemm_common.cuh"

namespace mxb {

namespace {

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
// consumer is this node, as in the 3-layer MLP's relu(h W2 + b2) + h W2').  Each k-block
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
// lives in the leader and takes one arrival per epilogue warp of either CTA;
// so does tload, which tells the MMA warp that a stream-K tail's accumulator
// has been loaded back into TMEM.
//
// Stream-K (FusedParams::sk_q > 0, single-product instances): when the tiles
// are not a multiple of the CTA pairs, the last one to two waves' k-blocks are
// spread evenly over all pairs (pair_work); a tile split between two pairs
// is handed from the pair running its first k-blocks to the pair running the
// rest as the raw fp32 accumulator, through global memory, so the MMA chain
// of every output element is unchanged.

template <int STAGES, int BN, bool DUAL, int EPI = 4, bool PUSH = false>
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
    // Single-product tiles move C and the output through TMA boxes
    // (FusedParams::tma_c / tma_out; not in batched launches, whose C has a
    // third coordinate): two 32 x 32 boxes per epilogue warp, each with its
    // mbarrier for C loads.
    static constexpr bool kTmaC = !DUAL && !PUSH;
    static constexpr int kNumBars = 2 * STAGES + 6 + 2 * EPI;
    // PUSH: two 8-row x 128-column staging buffers per epilogue warp for the
    // TMA stores of the row all-gather; kTmaC: the two boxes (the same 8 KiB);
    // 1 KiB aligned after the barriers.
    static constexpr int kStagingOffset = (kBarOffset + kNumBars * 8 + 16 + 1023) / 1024 * 1024;
    static constexpr int kStagingPerWarp = 2 * kPushBoxRows * kPushBoxCols * 4;
    static_assert(kStagingPerWarp == 2 * 32 * 32 * 4, "a warp's staging holds two 32 x 32 boxes");
    static constexpr int kSmemBytes =
        1024 + ((PUSH || kTmaC) ? kStagingOffset + EPI * kStagingPerWarp : kBarOffset + kNumBars * 8 + 16);
    static_assert(BN == 128 || BN == 256 || BN == 512, "pair tile width");
    static_assert(!(DUAL && BN == 512), "two products use 128- or 256-column tiles");
    static_assert(kStageBytes % 1024 == 0, "stages must keep 1 KiB swizzle alignment");
    static_assert(kTmemCols == 256 || kTmemCols == 512, "TMEM allocation");
    static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

// The row all-gather of one warp's 32 finished rows, columns c0 .. c1, by
// TMA tile stores: the warp reads its rows back from L2 (one 512-byte row
// segment per instruction) into one of its two staging buffers (8 rows x 128
// columns) and lane 0 stores the buffer to every peer's copy with one TMA
// instruction per peer, starting at a different peer per warp.  The copy
// engine then drives the NVLink writes, so the warp's cost is the read-back
// and one store per peer per 4 KiB; a buffer is refilled once the stores
// issued from it two rounds earlier have read it.
__device__ __forceinline__ void push_rows_tma(const PeerMaps& pm, const FusedParams& p, float* staging, int row0,
                                              int c0, int c1, int& buf) {
    __syncwarp();
    const int lane = threadIdx.x & 31;
    const int rows = min(32, p.M - row0);
    if (rows <= 0 || c0 >= c1) return;
    const int q0 = (row0 >> 5) % p.n_peers;
    for (int rb = 0; rb < rows; rb += kPushBoxRows) {
        for (int cb = c0; cb < c1; cb += kPushBoxCols) {
            float* sb = staging + buf * (kPushBoxRows * kPushBoxCols);
            if (lane == 0) bulk_wait_group_read<1>();
            __syncwarp();
            const int col = cb + 4 * lane;
#pragma unroll
            for (int r = 0; r < kPushBoxRows; ++r) {
                const int row = row0 + rb + r;
                float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (row < p.M && col < c1) {
                    const float* src = p.out + static_cast<long long>(row) * p.ldo + col;
                    if (col + 4 <= c1) {
                        v = *reinterpret_cast<const float4*>(src);
                    } else {
                        v.x = src[0];
                        if (col + 1 < c1) v.y = src[1];
                        if (col + 2 < c1) v.z = src[2];
                    }
                }
                *reinterpret_cast<float4*>(sb + r * kPushBoxCols + 4 * lane) = v;
            }
            fence_proxy_async_shared();
            __syncwarp();
            if (lane == 0) {
                int q = q0;
                for (int j = 0; j < p.n_peers; ++j) {
                    tma_store_2d(&pm.m[q], smem_addr(sb), cb, row0 + rb);
                    q = q + 1 == p.n_peers ? 0 : q + 1;
                }
                bulk_commit_group();
            }
            buf ^= 1;
        }
    }
}

// PUSH: the epilogue also writes each tile's rows into the peers' copies
// (FusedParams::peer_out), a separate instance so the other launches keep
// their registers.
// BATCHED: p.batch products of one shape in one launch, A and B as 3-D tensor
// maps (third coordinate: the product), as in the single-CTA kernel.
template <int STAGES, int BN, bool DUAL, int EPI, bool PUSH, bool BATCHED = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PairCfg<STAGES, BN, DUAL, EPI>::kThreadsPerCta, 1)
    fused_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                           const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                           const __grid_constant__ FusedParams p, const __grid_constant__ PeerMaps pm,
                           const __grid_constant__ EpiMaps em) {
    using C = PairCfg<STAGES, BN, DUAL, EPI, PUSH>;
    constexpr bool kBoxes = C::kTmaC && !BATCHED;
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
    const uint32_t tload_bar = bar0 + 8u * (2 * STAGES + 5);
    // Epilogue warp w's boxes (kTmaC): barrier of box i's C load.
    auto cbox_bar = [&](int w, int i) { return bar0 + 8u * (2 * STAGES + 6 + 2 * (w - 2) + i); };

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
        mbar_init(tload_bar, 2 * EPI);  // every epilogue warp of the two CTAs, once per launch
        for (int i = 0; i < 2 * EPI; ++i) mbar_init(bar0 + 8u * (2 * STAGES + 6 + i), 1);
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        if (kBoxes && p.tma_c) tma_prefetch_desc(&em.c);
        if (kBoxes && p.tma_out) tma_prefetch_desc(&em.out);
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
            PairWork wk;
            for (int idx = 0; ok && pair_work(p, pair, num_pairs, idx, wk); ++idx) {
                const int t = wk.t;
                int mb, nb;
                int b = 0;
                if (BATCHED) {
                    b = t / p.tiles_per_batch;
                    tile_coords(t - b * p.tiles_per_batch, p, mb, nb);
                } else {
                    tile_coords(t, p, mb, nb);
                }
                const int m0 = mb * 256 + static_cast<int>(rank) * 128;
                // CTA r stages, for sub-MMA h, B columns nb*BN + h*kSubN + r*kSubN/2 ..
                // + kSubN/2, so accumulator column c is output column nb*BN + c.
                const int n0 = nb * BN + static_cast<int>(rank) * (C::kSubN / 2);
                for (int kb = wk.kb0; kb < wk.kb1; ++kb) {
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
                    if (BATCHED) {
                        tma_load_3d_pair(smem_addr(st), &tmA, fb, k0, m0, b);
#pragma unroll
                        for (int j = 0; j < BN / 64; ++j)
                            tma_load_3d_pair(smem_addr(st + C::kABytes + j * kBoxBytes), &tmB, fb,
                                             n0 + (j / C::kSubBoxes) * C::kSubN + 32 * (j % C::kSubBoxes), k0, b);
                    } else {
                        tma_load_2d_pair(smem_addr(st), &tmA, fb, k0, m0);
#pragma unroll
                        for (int j = 0; j < BN / 64; ++j)
                            tma_load_2d_pair(smem_addr(st + C::kABytes + j * kBoxBytes), &tmB, fb,
                                             n0 + (j / C::kSubBoxes) * C::kSubN + 32 * (j % C::kSubBoxes), k0);
                    }
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
            PairWork wk;
            for (int idx = 0; ok && pair_work(p, pair, num_pairs, idx, wk); ++idx) {
                if (*abort_flag) break;
                if (!mbar_wait_cluster(tempty_bar(acc), acc_phase ^ 1u, p.timeout_ns)) {
                    raise_error(p, abort_flag, kErrMma);
                    break;
                }
                // A stream-K tail starts from the accumulator its head pair
                // left, once the epilogue warps have loaded it into TMEM.
                if (wk.kind == kWorkTail && (*abort_flag || !mbar_wait_cluster(tload_bar, 0, p.timeout_ns))) {
                    raise_error(p, abort_flag, kErrMma);
                    break;
                }
                tc_fence_after();
                const uint32_t d_tile = tmem_base + static_cast<uint32_t>(acc * C::kAccCols);
                for (int kb = wk.kb0; kb < wk.kb1; ++kb) {
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
                        const uint32_t accumulate = (wk.kind == kWorkTail || kb != wk.kb0 || kk != 0) ? 1u : 0u;
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
        uint32_t cbox_phase = 0;    // bit i: parity of box i's next C load
        uint32_t cbox_pending = 0;  // bit i: a C load into box i not yet waited for
        bool cbox_failed = false;
        // Stream-K hand-off: this warp's rows of the tile (lane quadrant,
        // column range) in the head pair's slot and the flag it sets.
        const int sk_warp = (static_cast<int>(rank) * EPI + (warp - 2));
        float* push_staging = reinterpret_cast<float*>(smem + C::kStagingOffset + (warp - 2) * C::kStagingPerWarp);
        int push_buf = 0;
        PairWork wk;
        for (int idx = 0; pair_work(p, pair, num_pairs, idx, wk); ++idx) {
            const int t = wk.t;
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
            const int col0 = nb * BN;
            int chunks = (p.N - col0 + 31) / 32;
            if (chunks > c_first + kChunksPerWarp) chunks = c_first + kChunksPerWarp;
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                                   static_cast<uint32_t>(acc * C::kAccCols);
            const bool head = !BATCHED && !DUAL && wk.kind == kWorkHead;
            if (!BATCHED && !DUAL && wk.kind == kWorkTail) {
                // Load the head pair's accumulator into this (free) TMEM buffer,
                // then let the MMA warp continue the chain.
                const int src_pair = pair - 1;
                const bool ready = __all_sync(0xffffffffu, *abort_flag == 0) &&
                                   wait_flag_gpu(p.sk_flags + src_pair * 2 * EPI + sk_warp, 1, p.timeout_ns);
                if (!__all_sync(0xffffffffu, ready)) {
                    if (lane == 0) raise_error(p, abort_flag, kErrEpilogue);
                    break;
                }
                const float* src = p.sk_ws + (static_cast<long long>(src_pair) * 2 + rank) * (BN * 128) +
                                   (quad * 32 + lane) * 4;
                // Four chunks' loads in flight per round trip (the MMA warp
                // waits for this buffer meanwhile).
                for (int c0 = c_first; c0 < chunks; c0 += 4) {
                    uint32_t r[4][32];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        if (c0 + u < chunks) {
#pragma unroll
                            for (int j = 0; j < 8; ++j) {
                                const float4 x = ld_global_cg_v4(src + (8 * (c0 + u) + j) * 512);
                                r[u][4 * j + 0] = __float_as_uint(x.x);
                                r[u][4 * j + 1] = __float_as_uint(x.y);
                                r[u][4 * j + 2] = __float_as_uint(x.z);
                                r[u][4 * j + 3] = __float_as_uint(x.w);
                            }
                        }
                    }
#pragma unroll
                    for (int u = 0; u < 4; ++u)
                        if (c0 + u < chunks) tmem_st_32x32b_x32(taddr + 32 * (c0 + u), r[u]);
                }
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(mapa_shared(tload_bar, 0));
            }
            // C rows into L2: during the k-loop when it is short, else once the accumulator is ready.
            const bool fetch = !head && row_ok && chunks > c_first;
            if (fetch && p.prefetch_early)
                prefetch_full_operands(row, col0 + 32 * c_first, 32 * (chunks - c_first), p, b);
            const bool stop = __any_sync(0xffffffffu, *abort_flag != 0);
            const bool got = !stop && mbar_wait_cluster(tfull_bar(acc), acc_phase, p.timeout_ns);
            if (!__all_sync(0xffffffffu, got)) {
                if (lane == 0 && !stop) raise_error(p, abort_flag, kErrEpilogue);
                break;
            }
            tc_fence_after();
            if (fetch && !p.prefetch_early)
                prefetch_full_operands(row, col0 + 32 * c_first, 32 * (chunks - c_first), p, b);
            if (chunks <= c_first) {
                // No columns of this tile for this warp: release the accumulator at once.
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(acc ? tempty_leader1 : tempty_leader0);
            }
            if (head) {
                // A stream-K head: the raw accumulator goes to this pair's slot
                // ([column / 4][row][4], 512 contiguous bytes per instruction);
                // no epilogue.
                float* dst = p.sk_ws + (static_cast<long long>(pair) * 2 + rank) * (BN * 128) + (quad * 32 + lane) * 4;
                const uint64_t pol = l2_policy_evict_normal();
                for (int c = c_first; c < chunks; ++c) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(taddr + 32 * c, r);
                    tmem_ld_wait();
                    if (c == chunks - 1) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive_cluster(acc ? tempty_leader1 : tempty_leader0);
                    }
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        st_global_v4_hint(dst + (8 * c + j) * 512, __uint_as_float(r[4 * j]),
                                          __uint_as_float(r[4 * j + 1]), __uint_as_float(r[4 * j + 2]),
                                          __uint_as_float(r[4 * j + 3]), pol);
                }
                __threadfence();
                __syncwarp();
                if (lane == 0) st_release_gpu(p.sk_flags + pair * 2 * EPI + sk_warp, 1);
                if (C::kBufs == 2) acc ^= 1;
                if (acc == 0) acc_phase ^= 1u;
                continue;
            }
            // Single-product, unbatched tiles (kBoxes): C in (tma_c) and the
            // result out (tma_out) as 32 x 32 TMA boxes of this warp's 32 rows, through
            // two 128-byte swizzled boxes of shared memory per warp; each lane
            // reads and writes its own row there.  Box i holds C of chunk c,
            // then chunk c's result until its TMA store has read it, then C of
            // chunk c + 2.  Read and written by each lane from and to its own
            // row of global memory (32 rows per warp instruction), C and the
            // output kept the load/store unit busy for 37,000 of the 45,000
            // cycles a 256 x 512 tile's drain took, the MMA warp waiting for
            // the accumulator all along (256 x 256 tiles drain while the next
            // tile runs, except at the end of a launch).
            const int box_row0 = mb * 256 + static_cast<int>(rank) * 128 + quad * 32;
            const bool boxes = kBoxes && box_row0 < p.M;
            const bool cbox = boxes && p.tma_c;
            const bool obox = boxes && p.tma_out;
            uint8_t* const box_buf = smem + C::kStagingOffset + (warp - 2) * C::kStagingPerWarp;
            // Issued by lane 0; every lane keeps the pending bits.
            auto cbox_load = [&](int c) {
                const int i = (c - c_first) & 1;
                if (lane == 0) {
                    mbar_arrive_expect_tx(cbox_bar(warp, i), 32 * 32 * 4);
                    tma_load_2d(smem_addr(box_buf + i * 4096), &em.c, cbox_bar(warp, i), col0 + 32 * c, box_row0);
                }
                cbox_pending |= 1u << i;
            };
            // The previous tile's box stores have read both boxes (its last
            // chunk may have used either box), and its lanes' reads of them
            // come before the TMA writes below.
            if ((cbox || obox) && c_first < chunks && lane == 0) {
                if (obox) bulk_wait_group_read<0>();
                fence_proxy_async_shared();
            }
            if (cbox && c_first < chunks) {
                cbox_load(c_first);
                if (!obox && c_first + 1 < chunks) cbox_load(c_first + 1);
            }
            for (int c = c_first; c < chunks; ++c) {
                uint32_t r[32];
                float w[32];
                tmem_ld_32x32b_x32(taddr + 32 * c, r);
                const int i = (c - c_first) & 1;
                if (cbox && obox && c + 1 < chunks) {
                    // box i ^ 1 is free once chunk c - 1's store has read it
                    if (lane == 0) bulk_wait_group_read<0>();
                    cbox_load(c + 1);
                } else if (!cbox && obox && lane == 0) {
                    bulk_wait_group_read<1>();  // chunk c - 2's store has read box i
                }
                if (DUAL) {
                    uint32_t r2[32];
                    tmem_ld_32x32b_x32(taddr + BN + 32 * c, r2);
                    tmem_ld_wait();
#pragma unroll
                    for (int k = 0; k < 32; ++k) w[k] = __uint_as_float(r2[k]);
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
                for (int k = 0; k < 32; ++k) v[k] = __uint_as_float(r[k]);
                const int col = col0 + 32 * c;
                uint8_t* const rowp = box_buf + i * 4096 + lane * 128;
                if (cbox) {
                    const bool got = mbar_wait(cbox_bar(warp, i), (cbox_phase >> i) & 1u, p.timeout_ns);
                    if (!__all_sync(0xffffffffu, got)) {
                        if (lane == 0) raise_error(p, abort_flag, kErrEpilogue);
                        cbox_failed = true;
                        break;
                    }
                    cbox_phase ^= 1u << i;
                    cbox_pending &= ~(1u << i);
                    // Step 0 (v += C), the add the FULL step makes; columns
                    // past N read the box's zero fill and are never stored.
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const float4 x = *reinterpret_cast<const float4*>(rowp + ((j ^ (lane & 7)) << 4));
                        v[4 * j] += x.x;
                        v[4 * j + 1] += x.y;
                        v[4 * j + 2] += x.z;
                        v[4 * j + 3] += x.w;
                    }
                    if (!obox) {
                        __syncwarp();  // every lane has read box i: it may be refilled
                        if (c + 2 < chunks) {
                            if (lane == 0) fence_proxy_async_shared();  // those reads before the TMA write
                            cbox_load(c + 2);
                        }
                    }
                }
                if (DUAL)
                    apply_epilogue(v, row, col, row_ok, p, w);
                else
                    apply_epilogue(v, row, col, row_ok, p, nullptr, b, cbox);
                if (obox) {
                    // The result into box i (rows past M and columns past N are
                    // clipped by the store), then one TMA store of the box.
                    if (!cbox) __syncwarp();  // lane 0 waited for box i above
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        *reinterpret_cast<float4*>(rowp + ((j ^ (lane & 7)) << 4)) =
                            make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                    fence_proxy_async_shared();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&em.out, smem_addr(box_buf + i * 4096), col, box_row0);
                        bulk_commit_group();
                    }
                } else if (row_ok) {
                    store_row_chunk(v, row, col, p, out_off);
                }
            }
            if (PUSH) {
                // The accumulator is already released: these copies overlap the next tile's k-loop.
                const int c_end = col0 + 32 * chunks < p.N ? col0 + 32 * chunks : p.N;
                if (p.push_tma)
                    push_rows_tma(pm, p, push_staging, mb * 256 + row_in_tile - lane, col0 + 32 * c_first, c_end,
                                  push_buf);
                else
                    push_rows<8>(p, mb * 256 + row_in_tile - lane, col0 + 32 * c_first, c_end);
            }
            if (cbox_failed) break;
            if (C::kBufs == 2) acc ^= 1;
            if (acc == 0) acc_phase ^= 1u;
        }
        // A C box load that was not waited for (a wait that ran out above) must
        // land before the CTA leaves: wait for it once more, bounded.  The
        // boxes' stores complete before it leaves too.
        if (kBoxes) {
            for (int i = 0; i < 2; ++i)
                if (cbox_pending & (1u << i)) mbar_wait(cbox_bar(warp, i), (cbox_phase >> i) & 1u, p.timeout_ns);
            if (lane == 0) bulk_wait_group<0>();
            __syncwarp();
        }
        // Peer stores performed before the kernel counts as finished.
        if (PUSH) {
            if (lane == 0) bulk_wait_group<0>();
            __syncwarp();
            __threadfence_system();
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

// MINIXLA_GATHER_TMA=0: the row all-gather stores through the epilogue
// warps' own global stores instead of TMA tile stores.
bool gather_tma_enabled() {
    const char* v = getenv("MINIXLA_GATHER_TMA");
    return !(v && v[0] == '0');
}

template <int STAGES, int BN, bool DUAL, int EPI = 4, bool PUSH = false, bool BATCHED = false>
cudaError_t run_pair_variant(const GemmLaunch& g, cudaStream_t stream) {
    using C = PairCfg<STAGES, BN, DUAL, EPI, PUSH>;
    auto kernel = fused_gemm_pair_kernel<STAGES, BN, DUAL, EPI, PUSH, BATCHED>;
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
    if (BATCHED) {
        if (!make_map_3d(&mA, g.A, g.batch, g.M, g.K, g.lda, g.a_bstride, kBK, 128, kSwA) ||
            !make_map_3d(&mB, g.B, g.batch, g.K, g.N, g.ldb, g.b_bstride, 32, kBK, kSwB))
            return cudaErrorInvalidValue;
    } else if (!make_map(&mA, g.A, g.M, g.K, g.lda, kBK, 128, kSwA) ||
               !make_map(&mB, g.B, g.K, g.N, g.ldb, 32, kBK, kSwB)) {
        return cudaErrorInvalidValue;
    }
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
    p.prefetch_early = prefetch_early(g.M, g.N, g.K, g.batch > 1 ? g.batch : 1);
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
    PeerMaps pm;
    memset(&pm, 0, sizeof(pm));
    if (PUSH && p.push_vec && gather_tma_enabled() && g.M >= kPushBoxRows && g.N >= kPushBoxCols) {
        // This launch's rows in each peer's copy: the same [M, N] block at peer_out[i], pitch ldo.
        bool ok = true;
        for (int i = 0; i < g.n_peers && ok; ++i)
            ok = make_store_map(&pm.m[i], g.peer_out[i], g.M, g.N, g.ldo, kPushBoxCols, kPushBoxRows);
        p.push_tma = ok ? 1 : 0;
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
    if (!BATCHED && !DUAL && g.sk_ws && g.sk_flags && pairs <= g.sk_pairs && BN <= g.sk_cols) {
        // Stream-K over the last one to two waves when the tiles are not a
        // multiple of the pairs: every pair then gets the same number of
        // k-blocks (within one), where the last wave would leave some idle.
        const StreamKSplit sk = streamk_split(p.num_tiles, p.num_kb, pairs);
        if (sk.q > 0) {
            p.sk_dp_tiles = sk.dp_tiles;
            p.sk_q = sk.q;
            p.sk_extra = sk.extra;
            p.sk_ws = g.sk_ws;
            p.sk_flags = g.sk_flags;
            const cudaError_t e2 = cudaMemsetAsync(g.sk_flags, 0, sizeof(int) * pairs * 2 * EPI, stream);
            if (e2 != cudaSuccess) return e2;
        }
    }
    EpiMaps em;
    memset(&em, 0, sizeof(em));
    if (C::kTmaC && !BATCHED && epi_tma_enabled()) {
        if (g.n_steps > 0 && g.steps[0].kind == MXB_EP_ADD_FULL && (g.steps[0].ld_or_size & 3) == 0 &&
            (reinterpret_cast<uintptr_t>(g.steps[0].ptr) & 15) == 0)
            p.tma_c = make_epi_map(&em.c, g.steps[0].ptr, g.M, g.N, g.steps[0].ld_or_size) ? 1 : 0;
        if ((g.ldo & 3) == 0 && (reinterpret_cast<uintptr_t>(g.out) & 15) == 0)
            p.tma_out = make_epi_map(&em.out, g.out, g.M, g.N, g.ldo) ? 1 : 0;
    }
    kernel<<<2 * pairs, C::kThreadsPerCta, C::kSmemBytes, stream>>>(mA, mB, mA2, mB2, p, pm, em);
    note_launch();
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_pair_tf32(const GemmLaunch& g, bool wide_tiles, cudaStream_t stream) {
    if (g.batch > 1) {
        if (g.n_peers > 0 || g.A2) return cudaErrorInvalidValue;
        return run_pair_variant<6, 256, false, 4, false, true>(g, stream);
    }
    if (g.n_peers > 0)
        return wide_tiles ? run_pair_variant<4, 512, false, 4, true>(g, stream)
                          : run_pair_variant<6, 256, false, 4, true>(g, stream);
    return wide_tiles ? run_pair_variant<4, 512, false>(g, stream) : run_pair_variant<6, 256, false>(g, stream);
}

// 256-column tiles put both accumulators in the 512 TMEM columns (one buffer,
// 48 KiB stages); 128-column tiles keep two buffers for problems with few tiles
// (the choice is plan_fused_gemm's).
cudaError_t launch_pair_tf32_dual(const GemmLaunch& g, cudaStream_t stream) {
    if (plan_fused_gemm(g, 1).tile_cols == 256) return run_pair_variant<4, 256, true>(g, stream);
    return run_pair_variant<6, 128, true>(g, stream);
}

}  // namespace mxb
