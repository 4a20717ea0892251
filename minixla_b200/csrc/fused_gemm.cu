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
//
// This file holds the single-CTA kernels and the kernel choice.  The CTA-pair
// kernels (cta_group::2, 256-row tiles) live in fused_gemm_pair.cu (TF32) and
// fused_gemm_pair3.cu (3xTF32); all share the epilogue, the error reporting
// and the tensor-map encoder in gemm_common.cuh.
#include "gemm_common.cuh"

namespace mxb {

namespace {

template <int BN, int STAGES, bool SPLIT3>
struct Cfg {
    static constexpr int kABytes = kBM * kBK * 4;
    static constexpr int kBBytes = BN * kBK * 4;
    static constexpr int kOperandBytes = kABytes + kBBytes;
    static constexpr int kStageBytes = (SPLIT3 ? 2 : 1) * kOperandBytes;
    static constexpr int kTmemCols = 2 * BN;
    static constexpr int kBarOffset = STAGES * kStageBytes;
    // TF32 tiles move C and the output through TMA boxes: two 32 x 32 fp32
    // boxes per epilogue warp, 1 KiB aligned after the barriers, each with an
    // mbarrier for its C loads (the last 8 barriers).
    static constexpr bool kBoxRoom = !SPLIT3;
    static constexpr int kNumBars = 2 * STAGES + 5 + 8;
    static constexpr int kBoxOffset = (kBarOffset + kNumBars * 8 + 16 + 1023) / 1024 * 1024;
    static constexpr int kSmemBytes =
        1024 + (kBoxRoom ? kBoxOffset + 4 * 8192 : kBarOffset + kNumBars * 8 + 16);
    static_assert(kStageBytes % 1024 == 0, "stages must keep 1 KiB swizzle alignment");
    static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN");
    static_assert(kTmemCols == 64 || kTmemCols == 128 || kTmemCols == 256 || kTmemCols == 512,
                  "TMEM allocation must be a power of two >= 32 columns");
    static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

// KSPLIT: tile t is a K slice of output tile t / p.splits.  With
// p.ks_cluster (one tile per cluster of p.splits CTAs, one slice per CTA) the
// epilogue warps leave their slice raw in their own shared memory, the
// cluster synchronises, and each CTA sums its share of the tile's rows over
// the slices of every CTA of the cluster through distributed shared memory,
// in slice order, then applies the epilogue (ksplit_cluster_reduce).  Without
// it, the slices go raw to workspace and ksplit_reduce_kernel, launched next,
// sums them the same way.
//
// BATCHED: p.batch products of the same shape in one launch; A, B (and their
// low parts) are 3-D tensor maps whose third coordinate is the product, so a
// partial tile or k-block never reads the next product's rows.
// The raw slice of one K-split CTA in its shared memory: 128 rows x 128
// columns as float4s, row r's float4 f at r * 32 + (f ^ (r & 31)), so that a
// quarter-warp writing one float4 of eight rows, or reading eight float4s of
// one row, touches eight different 16-byte bank groups.
__device__ __forceinline__ uint32_t ks_slot(int row, int f) {
    return static_cast<uint32_t>(row * 32 + (f ^ (row & 31))) * 16u;
}

// Thread `row` (0..127) stores 32 raw accumulator columns, chunk c, into the slice buffer.
__device__ __forceinline__ void ks_dump_chunk(uint8_t* buf, int row, int c, const uint32_t (&r)[32]) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
        *reinterpret_cast<float4*>(buf + ks_slot(row, 8 * c + j)) =
            make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]), __uint_as_float(r[4 * j + 2]),
                        __uint_as_float(r[4 * j + 3]));
}

// After the cluster barrier: CTA `rank` of the tile's cluster sums rows
// [rank * R, (rank + 1) * R) of the slices of all S CTAs, in slice order
// (slice 0, + slice 1, ...: the same additions as ksplit_reduce_kernel),
// applies the node's epilogue and stores.  All six warps take part (the TMA
// and MMA warps are idle by then): warp w takes rows w, w + 6, ... (RPT of
// them), lane l the four columns 4l .. 4l + 3.  Every slice load of every row
// a thread owns is issued before the first add (S x RPT float4s in flight),
// so the sum waits on distributed shared memory once.  Issued four rows at a
// time by the four epilogue warps, each round waited for its loads and then
// its C loads, and the sum took 16,000 of (8191, 127, 3000)'s 52,000 cycles
// (28,000 in the k-loop).
template <int S, int RPT>
__device__ __forceinline__ void ksplit_cluster_reduce_t(const FusedParams& p, const uint8_t* buf, int mb, int nb,
                                                        int warp, int lane) {
    constexpr int kWarps = kThreads / 32;
    constexpr int kPer = (128 + S - 1) / S;
    static_assert(RPT * kWarps >= kPer, "rows per thread cover the CTA's share");
    const uint32_t rank = cluster_ctarank();
    const int r_lo = static_cast<int>(rank) * kPer, r_hi = min(128, r_lo + kPer);
    const int col = nb * 128 + 4 * lane;
    if (col >= p.N) return;
    const uint32_t base = smem_addr(buf);
    float v[RPT][4];
    int row[RPT];
    bool ok[RPT];
    float4 x[S][RPT];
#pragma unroll
    for (int u = 0; u < RPT; ++u) {
        const int r = r_lo + warp + kWarps * u;
        row[u] = mb * 128 + r;
        ok[u] = r < r_hi && row[u] < p.M;
    }
#pragma unroll
    for (int s = 0; s < S; ++s) {
        const uint32_t remote = mapa_shared(base, static_cast<uint32_t>(s));
#pragma unroll
        for (int u = 0; u < RPT; ++u)
            x[s][u] = ld_shared_cluster_v4(remote + ks_slot(ok[u] ? r_lo + warp + kWarps * u : r_lo, lane));
    }
#pragma unroll
    for (int u = 0; u < RPT; ++u) {
        v[u][0] = x[0][u].x;
        v[u][1] = x[0][u].y;
        v[u][2] = x[0][u].z;
        v[u][3] = x[0][u].w;
#pragma unroll
        for (int s = 1; s < S; ++s) {
            v[u][0] += x[s][u].x;
            v[u][1] += x[s][u].y;
            v[u][2] += x[s][u].z;
            v[u][3] += x[s][u].w;
        }
    }
    apply_epilogue_rows<RPT>(v, row, ok, col, p);
#pragma unroll
    for (int u = 0; u < RPT; ++u)
        if (ok[u]) store_row_chunk<4>(v[u], row[u], col, p);
}

// In-cluster sums come in 2, 3 or 4 slices (fused_gemm_ksplit_in_cluster).
__device__ __forceinline__ void ksplit_cluster_reduce(const FusedParams& p, const uint8_t* buf, int mb, int nb,
                                                      int warp, int lane) {
    switch (p.splits) {
        case 2: ksplit_cluster_reduce_t<2, 11>(p, buf, mb, nb, warp, lane); break;
        case 3: ksplit_cluster_reduce_t<3, 8>(p, buf, mb, nb, warp, lane); break;
        default: ksplit_cluster_reduce_t<4, 6>(p, buf, mb, nb, warp, lane); break;
    }
}

template <int BN, int STAGES, bool SPLIT3, bool SEG, bool KSPLIT = false, bool BATCHED = false>
__global__ void __launch_bounds__(kThreads, 1)
    fused_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                      const __grid_constant__ FusedParams p, const __grid_constant__ EpiMaps em) {
    using C = Cfg<BN, STAGES, SPLIT3>;
    // Plain TF32 tiles: the epilogue's C and output through TMA boxes
    // (FusedParams::tma_c / tma_out), as in the CTA-pair kernels.
    constexpr bool kBoxes = C::kBoxRoom && !KSPLIT && !BATCHED;
    static_assert(!KSPLIT || SPLIT3 == SEG, "K split: TF32, or 3xTF32 with segments");
    static_assert(!(KSPLIT && BATCHED), "a batched launch does not split K");
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
    auto cbox_bar = [&](int w, int i) { return bar0 + 8u * (2 * STAGES + 5 + 2 * (w - 2) + i); };

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // K split: the reduce kernel, launched next as a programmatic dependent,
    // may be scheduled now; it waits for this grid's completion itself.
    if (KSPLIT) asm volatile("griddepcontrol.launch_dependents;");

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
        for (int i = 0; i < 8; ++i) mbar_init(bar0 + 8u * (2 * STAGES + 5 + i), 1);
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        if (SPLIT3) {
            tma_prefetch_desc(&tmA2);
            tma_prefetch_desc(&tmB2);
        }
        if (kBoxes && p.tma_c) tma_prefetch_desc(&em.c);
        if (kBoxes && p.tma_out) tma_prefetch_desc(&em.out);
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
                int kb_lo = 0, kb_hi = p.num_kb;
                int b = 0;
                if (KSPLIT) {
                    tile_coords(t / p.splits, p, mb, nb);
                    kb_lo = (t % p.splits) * p.kb_per_split;
                    kb_hi = min(p.num_kb, kb_lo + p.kb_per_split);
                } else if (BATCHED) {
                    b = t / p.tiles_per_batch;
                    tile_coords(t - b * p.tiles_per_batch, p, mb, nb);
                } else {
                    tile_coords(t, p, mb, nb);
                }
                const int m0 = mb * kBM, n0 = nb * BN;
                for (int kb = kb_lo; kb < kb_hi; ++kb) {
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
                    if (BATCHED) {
                        tma_load_3d(smem_addr(st), &tmA, fb, k0, m0, b);
#pragma unroll
                        for (int j = 0; j < BN / 32; ++j)
                            tma_load_3d(smem_addr(st + C::kABytes + j * kBoxBytes), &tmB, fb, n0 + 32 * j, k0, b);
                        if (SPLIT3) {
                            uint8_t* st2 = st + C::kOperandBytes;
                            tma_load_3d(smem_addr(st2), &tmA2, fb, k0, m0, b);
#pragma unroll
                            for (int j = 0; j < BN / 32; ++j)
                                tma_load_3d(smem_addr(st2 + C::kABytes + j * kBoxBytes), &tmB2, fb,
                                            n0 + 32 * j, k0, b);
                        }
                    } else {
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
                int kb_lo = 0, kb_hi = p.num_kb;
                if (KSPLIT) {
                    kb_lo = (t % p.splits) * p.kb_per_split;
                    kb_hi = min(p.num_kb, kb_lo + p.kb_per_split);
                }
                for (int k_begin = kb_lo; k_begin < kb_hi && ok; k_begin += p.seg_kb) {
                    const int k_end = min(kb_hi, k_begin + p.seg_kb);
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
        uint32_t cbox_phase = 0;    // bit i: parity of box i's next C load
        uint32_t cbox_pending = 0;  // bit i: a C load into box i not yet waited for
        bool cbox_failed = false;
        const int row_in_tile = quad * 32 + lane;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
            int mb, nb;
            int b = 0;
            if (BATCHED) {
                b = t / p.tiles_per_batch;
                tile_coords(t - b * p.tiles_per_batch, p, mb, nb);
            } else {
                tile_coords(KSPLIT ? t / p.splits : t, p, mb, nb);
            }
            const long long out_off = BATCHED ? b * p.out_bstride : 0;
            const int row = mb * kBM + row_in_tile;
            const bool row_ok = row < p.M;
            const int col0 = nb * BN;
            int chunks = (p.N - col0 + 31) / 32;
            if (chunks > BN / 32) chunks = BN / 32;
            const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
            bool failed = false;
            if (!KSPLIT && row_ok) {
                // Short k-loops: fetch C while the MMAs run; long ones: just before the drain.
                if (p.prefetch_early) prefetch_full_operands(row, col0, min(BN, p.N - col0), p, b);
            }
            if (KSPLIT && row_ok) {
                // Fetch C into L2 for the reduce kernel while the MMAs run.
                prefetch_full_operands(row, col0, min(BN, p.N - col0), p);
            }
            if (KSPLIT && !SEG) {
                const bool stop = __any_sync(0xffffffffu, *abort_flag != 0);
                const bool got = !stop && mbar_wait(tfull_bar(acc), acc_phase, p.timeout_ns);
                if (!__all_sync(0xffffffffu, got)) {
                    if (lane == 0 && !stop) raise_error(p, abort_flag, kErrEpilogue);
                    break;
                }
                tc_fence_after();
                const uint32_t taddr = lane_base + static_cast<uint32_t>(acc * BN);
                float* slice = p.ks_cluster ? nullptr
                                            : p.ks_ws + static_cast<long long>(t % p.splits) * p.ks_stride +
                                                  static_cast<long long>(row) * p.ks_ld;
                for (int c = 0; c < chunks; ++c) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(taddr + 32 * c, r);
                    tmem_ld_wait();
                    if (c == chunks - 1) {
                        tc_fence_before();
                        mbar_arrive(tempty_bar(acc));
                    }
                    if (p.ks_cluster)
                        ks_dump_chunk(smem, row_in_tile, c, r);
                    else if (row_ok)
                        store_partial(r, slice + col0 + 32 * c, col0 + 32 * c, p.N);
                }
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1u;
            } else if (SEG) {
                // Sum the K segments in registers (fp32, round to nearest), 16
                // columns at a time.  After the last segment the totals go back
                // into that accumulator and the epilogue reads them from there,
                // with the registers free.
                // K split: this CTA's slice [kb_lo, kb_hi) in segments; its
                // total goes raw to the slice workspace for the reduce kernel.
                int kb_lo = 0, kb_hi = p.num_kb;
                if (KSPLIT) {
                    kb_lo = (t % p.splits) * p.kb_per_split;
                    kb_hi = min(p.num_kb, kb_lo + p.kb_per_split);
                }
                float total[BN];
                for (int k_begin = kb_lo; k_begin < kb_hi; k_begin += p.seg_kb) {
                    const bool first = k_begin == kb_lo;
                    const bool last = k_begin + p.seg_kb >= kb_hi;
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
                        float* slice = nullptr;
                        if (KSPLIT && !p.ks_cluster)
                            slice = p.ks_ws + static_cast<long long>(t % p.splits) * p.ks_stride +
                                    static_cast<long long>(row) * p.ks_ld;
                        for (int c = 0; c < chunks; ++c) {
                            uint32_t r[32];
                            tmem_ld_32x32b_x32(taddr + 32 * c, r);
                            tmem_ld_wait();
                            const int col = col0 + 32 * c;
                            if (KSPLIT) {
                                if (p.ks_cluster)
                                    ks_dump_chunk(smem, row_in_tile, c, r);
                                else if (row_ok)
                                    store_partial(r, slice + col, col, p.N);
                            } else {
                                float v[32];
#pragma unroll
                                for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
                                apply_epilogue(v, row, col, row_ok, p, nullptr, b);
                                if (row_ok) store_row_chunk(v, row, col, p, out_off);
                            }
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
                if (row_ok && !p.prefetch_early) prefetch_full_operands(row, col0, min(BN, p.N - col0), p, b);
                const uint32_t taddr = lane_base + static_cast<uint32_t>(acc * BN);
                // C in and the result out as 32 x 32 TMA boxes of this warp's
                // 32 rows through two shared-memory boxes, as the CTA-pair
                // kernels' epilogue does (fused_gemm_pair.cu): box i holds C
                // of chunk c, then chunk c's result until its store has read
                // it, then C of chunk c + 2.
                const int box_row0 = mb * kBM + quad * 32;
                const bool boxes = kBoxes && box_row0 < p.M;
                const bool cbox = boxes && p.tma_c;
                const bool obox = boxes && p.tma_out;
                uint8_t* const box_buf = smem + C::kBoxOffset + (warp - 2) * 8192;
                auto cbox_load = [&](int c) {
                    const int i = c & 1;
                    if (lane == 0) {
                        mbar_arrive_expect_tx(cbox_bar(warp, i), 32 * 32 * 4);
                        tma_load_2d(smem_addr(box_buf + i * 4096), &em.c, cbox_bar(warp, i), col0 + 32 * c, box_row0);
                    }
                    cbox_pending |= 1u << i;
                };
                // The previous tile's box stores have read both boxes, and its
                // lanes' reads of them come before the TMA writes below.
                if ((cbox || obox) && lane == 0) {
                    if (obox) bulk_wait_group_read<0>();
                    fence_proxy_async_shared();
                }
                if (cbox) {
                    cbox_load(0);
                    if (!obox && chunks > 1) cbox_load(1);
                }
                for (int c = 0; c < chunks; ++c) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(taddr + 32 * c, r);
                    const int i = c & 1;
                    if (cbox && obox && c + 1 < chunks) {
                        // box i ^ 1 is free once chunk c - 1's store has read it
                        if (lane == 0) bulk_wait_group_read<0>();
                        cbox_load(c + 1);
                    } else if (!cbox && obox && lane == 0) {
                        bulk_wait_group_read<1>();  // chunk c - 2's store has read box i
                    }
                    tmem_ld_wait();
                    if (c == chunks - 1) {
                        // Accumulator fully read: hand it back to the MMA warp.
                        tc_fence_before();
                        mbar_arrive(tempty_bar(acc));
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
                                if (lane == 0) fence_proxy_async_shared();
                                cbox_load(c + 2);
                            }
                        }
                    }
                    apply_epilogue(v, row, col, row_ok, p, nullptr, b, cbox);
                    if (obox) {
                        // The result into box i (rows past M and columns past N
                        // are clipped by the store), then one TMA store of it.
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
                if (cbox_failed) break;
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1u;
            }
        }
        // A C box load not waited for (a wait that ran out above) lands before
        // the CTA leaves, and so do the boxes' stores.
        if (kBoxes) {
            for (int i = 0; i < 2; ++i)
                if (cbox_pending & (1u << i)) mbar_wait(cbox_bar(warp, i), (cbox_phase >> i) & 1u, p.timeout_ns);
            if (lane == 0) bulk_wait_group<0>();
            __syncwarp();
        }
    }

    if (KSPLIT && p.ks_cluster) {
        // Every CTA of the tile's cluster reaches both barriers on every path
        // (a timed-out wait above only skips work), so neither can hang.
        __syncwarp();
        cluster_sync();  // each slice is in its CTA's shared memory
        {
            int mb, nb;
            tile_coords(static_cast<int>(blockIdx.x) / p.splits, p, mb, nb);
            ksplit_cluster_reduce(p, smem, mb, nb, warp, lane);
        }
        __syncwarp();
        cluster_sync();  // no CTA leaves while the others still read its slice
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::kTmemCols);
    }
}

// Second kernel of a K-split launch: the slices summed in slice order, then
// the node's epilogue.  Thread i takes four consecutive columns of one row,
// so a warp reads 512 contiguous bytes of a slice row; every SM takes part.
__global__ void __launch_bounds__(256) ksplit_reduce_kernel(const __grid_constant__ FusedParams p) {
    // Launched as a programmatic dependent of the split GEMM: its CTAs are
    // resident early, and this wait returns once that grid has finished and
    // its slices are visible.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int groups = (p.N + 3) / 4;
    const long long total = static_cast<long long>(p.M) * groups;
    for (long long i = blockIdx.x * 256ll + threadIdx.x; i < total; i += static_cast<long long>(gridDim.x) * 256) {
        const int row = static_cast<int>(i / groups);
        const int col = static_cast<int>(i - static_cast<long long>(row) * groups) * 4;
        float v[4];
        sum_slices4(v, p, row, col);
        apply_epilogue<4>(v, row, col, true, p);
        store_row_chunk<4>(v, row, col, p);
    }
}

// ------------------------------------------------------------------ host side

// The reduce kernel of a K split is launched as a programmatic dependent of
// the GEMM (it starts early and waits on griddepcontrol.wait);
// MINIXLA_KSPLIT_PDL=0 launches it in plain stream order.
// MINIXLA_BATCH_PAIR=0 keeps batched launches on the single-CTA kernel.
bool batch_pair_tiles() {
    const char* v = getenv("MINIXLA_BATCH_PAIR");
    return !(v && v[0] == '0');
}

// MINIXLA_BATCH_WIDE=0 keeps batched TF32 launches on 128-wide tiles.
bool batch_wide_tiles() {
    const char* v = getenv("MINIXLA_BATCH_WIDE");
    return !(v && v[0] == '0');
}

bool ksplit_pdl_enabled() {
    const char* v = getenv("MINIXLA_KSPLIT_PDL");
    return !(v && v[0] == '0');
}

// MINIXLA_KSPLIT_REDUCE=kernel: slices through workspace and the reduce
// kernel instead of summed inside the GEMM's clusters.
bool ksplit_cluster_enabled() {
    const char* v = getenv("MINIXLA_KSPLIT_REDUCE");
    return !(v && !strcmp(v, "kernel"));
}

template <int BN, int STAGES, bool SPLIT3, bool SEG, bool KSPLIT = false, bool BATCHED = false>
cudaError_t run_variant(const GemmLaunch& g, cudaStream_t stream) {
    using C = Cfg<BN, STAGES, SPLIT3>;
    auto kernel = fused_gemm_kernel<BN, STAGES, SPLIT3, SEG, KSPLIT, BATCHED>;
    if (BATCHED != (g.batch > 1)) return cudaErrorInvalidValue;
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
    if (BATCHED) {
        // Products stored back to back: A_b = A + b * a_bstride, B_b = B + b * b_bstride.
        if (!make_map_3d(&mA, a_hi, g.batch, g.M, g.K, g.lda, g.a_bstride, kBK, kBM, kSwA) ||
            !make_map_3d(&mB, b_hi, g.batch, g.K, g.N, g.ldb, g.b_bstride, 32, kBK, kSwB))
            return cudaErrorInvalidValue;
        if (SPLIT3 && (!make_map_3d(&mA2, g.A_small, g.batch, g.M, g.K, g.lda, g.a_bstride, kBK, kBM, kSwA) ||
                       !make_map_3d(&mB2, g.B_small, g.batch, g.K, g.N, g.ldb, g.b_bstride, 32, kBK, kSwB)))
            return cudaErrorInvalidValue;
    } else {
        if (!make_map(&mA, a_hi, g.M, g.K, g.lda, kBK, kBM, kSwA) ||
            !make_map(&mB, b_hi, g.K, g.N, g.ldb, 32, kBK, kSwB))
            return cudaErrorInvalidValue;
        if (SPLIT3 && (!make_map(&mA2, g.A_small, g.M, g.K, g.lda, kBK, kBM, kSwA) ||
                       !make_map(&mB2, g.B_small, g.K, g.N, g.ldb, 32, kBK, kSwB)))
            return cudaErrorInvalidValue;
    }
    if (!SPLIT3) {
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
    p.prefetch_early = prefetch_early(g.M, g.N, g.K, g.batch > 1 ? g.batch : 1);
    p.row_base = g.row_base;
    p.timeout_ns = g.timeout_ns;
    p.err = g.err;
    if (g.n_peers > 0) return cudaErrorInvalidValue;  // only the CTA-pair kernels write peer rows
    for (int i = 0; i < g.n_steps; ++i) p.steps[i] = g.steps[i];
    p.splits = 1;
    p.kb_per_split = p.num_kb;
    if (KSPLIT) {
        static_assert(!KSPLIT || (BN == kKsplitTileCols && kBM == kKsplitTileRows), "K-split tile");
        if (g.k_splits < 2) return cudaErrorInvalidValue;
        // Whole k-blocks per slice and no empty slice: splits <= k_splits.
        p.kb_per_split = (p.num_kb + g.k_splits - 1) / g.k_splits;
        p.splits = (p.num_kb + p.kb_per_split - 1) / p.kb_per_split;
        p.num_tiles *= p.splits;
        p.ks_cluster = fused_gemm_ksplit_in_cluster(g) ? 1 : 0;
        if (!p.ks_cluster && !g.ks_ws) return cudaErrorInvalidValue;
        p.ks_ws = g.ks_ws;
        p.ks_ld = (g.N + 3) / 4 * 4;
        p.ks_stride = static_cast<long long>(g.M) * p.ks_ld;
    } else if (g.k_splits > 1) {
        return cudaErrorInvalidValue;
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

    EpiMaps em;
    memset(&em, 0, sizeof(em));
    if (C::kBoxRoom && !KSPLIT && !BATCHED && epi_tma_enabled()) {
        if (g.n_steps > 0 && g.steps[0].kind == MXB_EP_ADD_FULL && (g.steps[0].ld_or_size & 3) == 0 &&
            (reinterpret_cast<uintptr_t>(g.steps[0].ptr) & 15) == 0)
            p.tma_c = make_epi_map(&em.c, g.steps[0].ptr, g.M, g.N, g.steps[0].ld_or_size) ? 1 : 0;
        if ((g.ldo & 3) == 0 && (reinterpret_cast<uintptr_t>(g.out) & 15) == 0)
            p.tma_out = make_epi_map(&em.out, g.out, g.M, g.N, g.ldo) ? 1 : 0;
    }
    const int grid = p.num_tiles < g.num_sms ? p.num_tiles : g.num_sms;
    if (KSPLIT && p.ks_cluster) {
        // One cluster of p.splits CTAs per tile, one slice per CTA; the slices
        // are summed inside the kernel.
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(static_cast<unsigned>(p.num_tiles));
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = C::kSmemBytes;
        cfg.stream = stream;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = static_cast<unsigned>(p.splits);
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, kernel, mA, mB, mA2, mB2, p, em);
        if (e != cudaSuccess) return e;
        note_launch();
        return cudaGetLastError();
    }
    kernel<<<grid, kThreads, C::kSmemBytes, stream>>>(mA, mB, mA2, mB2, p, em);
    note_launch();
    if (KSPLIT) {
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        const long long items = static_cast<long long>(g.M) * ((g.N + 3) / 4);
        const long long blocks = std::min<long long>((items + 255) / 256, 8ll * g.num_sms);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(static_cast<unsigned>(blocks));
        cfg.blockDim = dim3(256);
        cfg.stream = stream;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr.val.programmaticStreamSerializationAllowed = ksplit_pdl_enabled() ? 1 : 0;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, ksplit_reduce_kernel, p);
        if (e != cudaSuccess) return e;
        note_launch();
    }
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
// the wide tiles alone give every CTA pair a tile, unless they would end in a
// stream-K tail with a k-loop under kWideStreamKMinKb blocks: there the
// 256 x 256 tiles, twice as many and so in finer waves, ran faster
// (held-stream CUDA events, wide with its stream-K tail vs 256 x 256):
// (4096, 8192, 4096) 411.6 vs 378.9 us, (8192, 4096, 4096) 409.4 vs 380.9,
// (4096, 8192, 2048) 271.3 vs 212.0, (6144, 8192, 4096) 604.1 vs 594.0,
// (4096, 6144, 4096) 323.6 vs 319.5; at K = 8192 the two were even
// ((4096, 8192, 8192) 729.1 vs 732.2) and without a stream-K tail the wide
// tiles won ((6144)^3 609.3 vs 645.1, 8192^3 1385.5 vs 1492.8).
constexpr int kWideStreamKMinKb = 256;

bool pair_wide_tiles(const GemmLaunch& g) {
    if (const char* v = getenv("MINIXLA_GEMM_VARIANT")) {
        if (!strcmp(v, "pair512")) return true;
        if (!strcmp(v, "pair")) return false;
    }
    const long long wide_tiles = static_cast<long long>((g.M + 255) / 256) * ((g.N + 511) / 512);
    if (wide_tiles < g.num_sms / 2) return false;
    const int num_kb = (g.K + kBK - 1) / kBK;
    if (num_kb < kWideStreamKMinKb && wide_tiles < (1ll << 31) &&
        streamk_split(static_cast<int>(wide_tiles), num_kb, g.num_sms / 2).q > 0)
        return false;
    return true;
}

}  // namespace

// K split of the single-CTA kernels on 128 x 128 tiles (TF32, and 3xTF32
// with its segments inside each slice): when those tiles
// would fill at most half the SMs and K has at least 64 k-blocks,
// min(8, SMs / tiles, k-blocks / 16) CTAs share each tile's k-loop, and a
// reduce kernel sums the slices.  Measured against the unsplit 64- / 32-wide tiles (TF32, held-
// stream CUDA events): (8191, 127, 3000) 44.1 -> 41.5 us, (4096, 128, 2048)
// 27.4 -> 21.4, (1024, 1024, 4096) 48.0 -> 37.7, (640, 384, 4100) 45.9 ->
// 25.6, (2048, 256, 8192) 80.8 -> 37.3, (512, 512, 8192) 78.8 -> 33.8,
// (1024, 1024, 16384) 156.7 -> 97.2; with 32 k-blocks ((1000)^3) it lost
// (19.4 -> 21.4), hence kKsplitMinKb.  3xTF32: (4096, 128, 2048) 62.3 ->
// 42.0 us, (512, 512, 8192) 170.9 -> 70.5.  The count follows the node's full row
// count (choice_rows), so a node run in row chunks or shards gets the same
// sums.  MINIXLA_KSPLIT=0 turns it off, =n forces n ways (2..8);
// MINIXLA_SINGLE_BN alone leaves K unsplit.
constexpr int kKsplitMinKb = 64;  // K >= 2017

int fused_gemm_k_splits(const GemmLaunch& g) {
    if (g.A2 || g.n_peers > 0 || g.batch > 1 || use_pair_kernel(g)) return 1;
    const long long rows = g.choice_rows > 0 ? g.choice_rows : g.M;
    const long long tiles = ((rows + kKsplitTileRows - 1) / kKsplitTileRows) *
                            ((g.N + kKsplitTileCols - 1) / kKsplitTileCols);
    const int num_kb = (g.K + kBK - 1) / kBK;
    int s = 1;
    if (num_kb >= kKsplitMinKb && 2 * tiles <= g.num_sms)
        s = static_cast<int>(std::min<long long>({8, g.num_sms / tiles, num_kb / 16}));
    if (const char* v = getenv("MINIXLA_KSPLIT")) {
        const int f = atoi(v);
        if (f == 0 || f == 1) return 1;
        if (f >= 2 && f <= 8) return std::min(f, num_kb);
    }
    if (getenv("MINIXLA_SINGLE_BN")) return 1;  // a forced tile width runs unsplit
    return std::max(1, std::min(s, num_kb));
}

// Stream-K on the TF32 CTA-pair kernels (single products): the tiles of the
// last one to two waves are shared out by k-blocks over every pair when the
// tile count is not a multiple of the pairs (streamk_split), with a split
// tile's accumulator handed from one pair to the next through global memory.
// Reported for num_sms / 2 pairs; the launch uses the pairs that fit.
int fused_gemm_streamk_tiles(const GemmLaunch& g) {
    if (g.precision != GPU_PRECISION_TF32 || g.A2 || g.batch > 1) return 0;
    const GemmPlan pl = plan_fused_gemm(g, 1);
    if (pl.kernel != MXB_KERNEL_CTA_PAIR || pl.products != 1) return 0;
    const long long tiles = static_cast<long long>((g.M + 255) / 256) * ((g.N + pl.tile_cols - 1) / pl.tile_cols);
    if (tiles >= (1ll << 31)) return 0;
    const StreamKSplit sk = streamk_split(static_cast<int>(tiles), (g.K + kBK - 1) / kBK, g.num_sms / 2);
    return sk.q > 0 ? static_cast<int>(tiles) - sk.dp_tiles : 0;
}

// Whether a K-split launch of g sums its slices inside the GEMM (one cluster
// of `splits` CTAs per tile; every tile's cluster resident at once needs
// tiles x splits <= SMs, which fused_gemm_k_splits keeps unless a split count
// is forced).  Otherwise the slices need workspace and the reduce kernel.
// Clusters of up to four: eight-CTA clusters of these ~200 KB CTAs do not all
// fit at once (512 x 512 x 8192, 16 clusters of 8: 40.9 us against 25.5 us
// with the reduce kernel), while with two slices the in-cluster sum wins
// ((8191, 127, 3000): 31.7 vs 39.9 us; (640, 384, 4100), four: 20.4 vs 21.4 us).
bool fused_gemm_ksplit_in_cluster(const GemmLaunch& g) {
    if (g.k_splits < 2 || !ksplit_cluster_enabled()) return false;
    const int num_kb = (g.K + kBK - 1) / kBK;
    const int per = (num_kb + g.k_splits - 1) / g.k_splits;
    const int splits = (num_kb + per - 1) / per;
    const long long tiles = static_cast<long long>((g.M + kKsplitTileRows - 1) / kKsplitTileRows) *
                            ((g.N + kKsplitTileCols - 1) / kKsplitTileCols);
    return splits >= 2 && splits <= 4 && tiles * splits <= g.num_sms;
}

size_t fused_gemm_streamk_bytes(const GemmLaunch& g) {
    if (fused_gemm_streamk_tiles(g) == 0) return 0;
    const int pairs = g.num_sms / 2;
    const int cols = plan_fused_gemm(g, 1).tile_cols;
    // Raw accumulators (2 CTAs x 128 rows x tile columns per pair), then the flags.
    return static_cast<size_t>(pairs) * 2 * 128 * cols * sizeof(float) + static_cast<size_t>(pairs) * 2 * 8 * sizeof(int);
}

bool fused_gemm_pushes_rows(const GemmLaunch& g) {
    const char* v = getenv("MINIXLA_GATHER_PUSH");
    if (v && v[0] == '0') return false;
    return !g.A2 && g.batch <= 1 && use_pair_kernel(g);
}

GemmPlan plan_fused_gemm(const GemmLaunch& g, int k_splits) {
    GemmPlan pl{};
    pl.products = g.A2 ? 2 : 1;
    pl.k_splits = 1;
    if (g.A2 && g.batch <= 1) {
        // Two products of one A in one kernel (callers run other cases as two
        // launches): 3xTF32 on 256 x 128 pair tiles; TF32 on 256 x 256 tiles
        // once they give every CTA pair a tile, else 256 x 128.
        pl.kernel = MXB_KERNEL_CTA_PAIR;
        pl.tile_rows = 256;
        const long long tiles256 = static_cast<long long>((g.M + 255) / 256) * ((g.N + 255) / 256);
        pl.tile_cols = g.precision == GPU_PRECISION_TF32 && tiles256 >= g.num_sms / 2 ? 256 : 128;
        return pl;
    }
    if (g.batch <= 1 && use_pair_kernel(g)) {
        pl.kernel = MXB_KERNEL_CTA_PAIR;
        pl.tile_rows = 256;
        pl.tile_cols = g.precision == GPU_PRECISION_TF32 && pair_wide_tiles(g) ? 512 : 256;
        return pl;
    }
    pl.kernel = MXB_KERNEL_SINGLE_CTA;
    pl.tile_rows = kBM;
    if (g.batch > 1 && g.M >= 1024 && g.N >= 1024 && g.K >= 1024 && batch_pair_tiles()) {
        // Products from 1024^3 on 256 x 256 CTA-pair tiles once the batch
        // gives every CTA pair a tile (32 x 1024^3: TF32 162 -> 152 us, 3xTF32
        // 441 -> 411 us).  The single-CTA tiles stayed faster at 512^3 (84 vs
        // 88 us), on ragged 300-row products (21 vs 26 us) and with a short K
        // (8 x (1100, 1030, 300), 3xTF32: 108 vs 118 us).
        const long long pair_tiles = g.batch * ((g.M + 255) / 256) * ((g.N + 255) / 256);
        if (pair_tiles >= g.num_sms / 2) {
            pl.kernel = MXB_KERNEL_CTA_PAIR;
            pl.tile_rows = 256;
            pl.tile_cols = 256;
            return pl;
        }
    }
    if (g.batch > 1) {
        // All products in one launch (the caller batches only products too
        // small to fill the GPU alone): 128 x 256 tiles in TF32 mode from
        // N = 512 (32 x 1024^3: 197 -> 162 us; at N = 256 they were no
        // faster), else 128 x 128.
        pl.tile_cols = g.precision == GPU_PRECISION_TF32 && g.N >= 512 && batch_wide_tiles() ? 256 : 128;
        return pl;
    }
    if (k_splits > 1) {
        pl.k_splits = k_splits;
        pl.tile_cols = kKsplitTileCols;
        return pl;
    }
    // Narrower tiles for problems with few tiles, so more SMs share the
    // k-loops and the epilogue; 3xTF32 stages two operand pairs, so its
    // widest single-CTA tile is 128.
    const int w = single_cta_width(g);
    pl.tile_cols = g.precision == GPU_PRECISION_3XTF32 && w == 256 ? 128 : w;
    return pl;
}

cudaError_t launch_fused_gemm(const GemmLaunch& g, cudaStream_t stream) {
    if (g.precision != GPU_PRECISION_TF32 && g.precision != GPU_PRECISION_3XTF32) return cudaErrorInvalidValue;
    const bool x3 = g.precision == GPU_PRECISION_3XTF32;
    const GemmPlan pl = plan_fused_gemm(g, g.k_splits);
    if (pl.kernel == MXB_KERNEL_CTA_PAIR) {
        if (g.batch > 1) return x3 ? launch_pair_3xtf32(g, false, stream) : launch_pair_tf32(g, false, stream);
        if (pl.products == 2) return x3 ? launch_pair_3xtf32(g, true, stream) : launch_pair_tf32_dual(g, stream);
        return x3 ? launch_pair_3xtf32(g, false, stream) : launch_pair_tf32(g, pl.tile_cols == 512, stream);
    }
    if (g.batch > 1) {
        if (g.A2 || g.k_splits > 1 || g.n_peers > 0) return cudaErrorInvalidValue;
        if (x3) return run_variant<128, 3, true, true, false, true>(g, stream);
        return pl.tile_cols == 256 ? run_variant<256, 4, false, false, false, true>(g, stream)
                                   : run_variant<128, 6, false, false, false, true>(g, stream);
    }
    if (pl.k_splits > 1)
        return x3 ? run_variant<128, 3, true, true, true>(g, stream) : run_variant<128, 6, false, false, true>(g, stream);
    if (x3) {
        switch (pl.tile_cols) {
            case 128: return run_variant<128, 3, true, true>(g, stream);
            case 64: return run_variant<64, 4, true, true>(g, stream);
            default: return run_variant<32, 5, true, true>(g, stream);
        }
    }
    switch (pl.tile_cols) {
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
