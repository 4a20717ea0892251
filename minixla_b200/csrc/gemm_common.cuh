// Shared by the fused-GEMM translation units (fused_gemm.cu: single-CTA
// kernels and the dispatcher; fused_gemm_pair.cu: TF32 CTA-pair kernels;
// fused_gemm_pair3.cu: 3xTF32 CTA-pair kernels): tile constants, the kernel
// parameter block, tile order, bounded-wait error reporting, the fused
// epilogue in registers, and the TMA tensor-map encoder.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "internal.h"
#include "sm100_ptx.cuh"

namespace mxb {

// Launchers of the CTA-pair kernels (their translation units).
cudaError_t launch_pair_tf32(const GemmLaunch& g, bool wide_tiles, cudaStream_t stream);
cudaError_t launch_pair_tf32_dual(const GemmLaunch& g, cudaStream_t stream);
cudaError_t launch_pair_3xtf32(const GemmLaunch& g, bool dual, cudaStream_t stream);

namespace {

constexpr int kBM = 128;
constexpr int kBK = 32;           // fp32 elements per 128-byte swizzle row
constexpr int kThreads = 192;
constexpr int kBoxBytes = 32 * 32 * 4;  // one B box: 32 k-rows x 128 bytes

constexpr int kSegKb = 8;           // k-blocks (of 32) per accumulation segment in 3xTF32 mode
// With at most this many k-blocks the main loop is short (K <= 1024), so the
// epilogue prefetches its rows of the ADD operands before the accumulator is
// ready; longer loops prefetch once it is (earlier lines would be evicted) --
// unless the whole problem fits in a part of L2 (kEarlyPrefetchBytes of A, B,
// C and the output), where nothing evicts them.
constexpr int kShortKb = 32;
constexpr long long kEarlyPrefetchBytes = 64ll << 20;

inline int prefetch_early(long long M, long long N, long long K, long long batch = 1) {
    const long long bytes = 4 * batch * (M * K + K * N + 2 * M * N);
    return (K + 31) / 32 <= kShortKb || bytes <= kEarlyPrefetchBytes ? 1 : 0;
}

struct FusedParams {
    float* out;
    long long ldo;
    int M, N, K;
    int n_steps;
    int tiles_m, tiles_n, num_tiles, num_kb;
    int group_m;
    int seg_kb;                     // k-blocks per accumulation segment (num_kb: one segment)
    int prefetch_early;             // ADD operands into L2 during the k-loop (prefetch_early())
    long long row_base;             // global index of row 0 of this launch (modulo-rule operands)
    unsigned long long timeout_ns;
    int* err;
    EpStepDev steps[MXB_MAX_EPILOGUE];
    // Row all-gather (CTA-pair kernels only): the same rows of `out` in
    // each peer GPU's copy of the full output (same ldo), written by the
    // epilogue warps once their tile is stored locally.
    float* peer_out[kMaxPeers];
    int n_peers;
    int push_vec;                   // 16-byte aligned bases and ldo % 4 == 0: float4 copies
    int push_tma;                   // push_vec and PeerMaps valid: tile stores through TMA
    // Single-buffer CTA-pair tiles: the epilogue reads step 0's FULL operand
    // (tma_c, EpiMaps::c valid) and writes the output (tma_out, EpiMaps::out
    // valid) as 32 x 32 TMA boxes through shared memory.
    int tma_c;
    int tma_out;
    // K split (single-CTA TF32 kernel, KSPLIT instances): tile t is output
    // tile t / splits, k-blocks [s * kb_per_split, +kb_per_split) with
    // s = t % splits.  Slice s of the product goes raw to ks_ws + s * ks_stride
    // (row pitch ks_ld); a second kernel sums the slices and applies the epilogue.
    int splits;
    int kb_per_split;
    float* ks_ws;
    long long ks_stride, ks_ld;
    // K split summed inside the GEMM: the `splits` CTAs of a tile form one
    // cluster, leave their slices in shared memory and add them up through
    // distributed shared memory (no workspace, no second kernel).
    int ks_cluster;
    // Batched launch (single-CTA BATCHED instances): tile t is tile
    // t % tiles_per_batch of product b = t / tiles_per_batch; out and each
    // FULL operand step s advance by out_bstride / ep_bstride[s] elements per
    // product, and the modulo rule counts rows from row_base + b * M.
    int batch;
    int tiles_per_batch;
    long long out_bstride;
    long long ep_bstride[MXB_MAX_EPILOGUE];
    // Stream-K tail (TF32 CTA-pair kernels; sk_q == 0: off).  Tiles
    // [0, sk_dp_tiles) go one per pair in turn, a multiple of the pair count;
    // the k-blocks of the remaining tiles, taken as one run of
    // (num_tiles - sk_dp_tiles) * num_kb iterations, are dealt out in
    // contiguous ranges of sk_q (sk_q + 1 for the first sk_extra pairs).
    // sk_q >= num_kb, so a tile is shared by at most two pairs: the one that
    // runs its first k-blocks (the head, first on its list) stores the raw
    // accumulator to sk_ws and sets its flags; the other (the tail, last on
    // its list) loads that accumulator back into TMEM and continues
    // accumulating, so each output is the same chain of MMAs into one fp32
    // accumulator as without the split: the bits do not change.
    int sk_dp_tiles;
    int sk_q, sk_extra;
    float* sk_ws;                   // [pair][cta][BN / 4][128 rows][4]: raw accumulators of heads
    int* sk_flags;                  // [pair][cta][epilogue warp]: 1 once that warp's rows are stored
};

// Host side of the stream-K schedule: with `tiles` tiles of `num_kb`
// k-blocks on `pairs` pairs, whole waves but the last run one tile per pair
// (dp_tiles), and the remaining tiles (more than one wave, less than two) are
// shared out by k-blocks: q each, q + 1 for the first `extra` pairs.  q = 0
// when the tiles are a multiple of the pairs (or fewer), or when
// MINIXLA_STREAMK=0.
struct StreamKSplit {
    int dp_tiles = 0, q = 0, extra = 0;
};

inline bool streamk_enabled() {
    const char* v = getenv("MINIXLA_STREAMK");
    return !(v && v[0] == '0');
}

// Used when the idle share of the last wave is at least 1/kStreamKMinLoss of
// the job (one idle pair-tile in 25): below that the hand-offs cost about
// what they win back (8192^3: 6 idle pair-tiles in 512, no gain measured).
constexpr int kStreamKMinLoss = 25;
constexpr int kStreamKMinKb = 64;

inline StreamKSplit streamk_split(int tiles, int num_kb, int pairs) {
    StreamKSplit s;
    // At least two whole waves: the pairs run the first ones in step (tiles
    // that share rows of A or columns of B read the same k-blocks at the same
    // time, so L2 serves them once), and the stream-K part, whose pairs sit
    // at different k and read A and B several times over from HBM (4096^3,
    // all of it stream-K: 712 vs 293 MB of DRAM reads, L2 hits 51 vs 70%),
    // stays under half the work.
    // And k-loops of at least kStreamKMinKb blocks: with short ones the
    // hand-off costs more than the balance wins ((3300, 6001, 997): 229 vs
    // 217 us; (5120, 4096, 1024): even).
    if (!streamk_enabled() || pairs < 2 || tiles < 2 * pairs || tiles % pairs == 0 || num_kb < kStreamKMinKb)
        return s;
    const long long idle = static_cast<long long>(pairs - tiles % pairs);
    if (idle * kStreamKMinLoss < tiles) return s;
    s.dp_tiles = (tiles / pairs - 1) * pairs;
    const long long iters = static_cast<long long>(tiles - s.dp_tiles) * num_kb;
    s.q = static_cast<int>(iters / pairs);
    s.extra = static_cast<int>(iters % pairs);
    return s;
}

// Tensor maps of this launch's rows in every peer's copy of the output
// (FLOAT32, no rounding, no swizzle; box 8 rows x 128 columns), for the TMA
// stores of the row all-gather (FusedParams::push_tma).
constexpr int kPushBoxRows = 8, kPushBoxCols = 128;
struct PeerMaps {
    CUtensorMap m[kMaxPeers];
};

// MINIXLA_EPI_TMA=0: the TF32 kernels' epilogue reads C and writes the
// output row by row from global memory instead of through TMA boxes.
inline bool epi_tma_enabled() {
    const char* v = getenv("MINIXLA_EPI_TMA");
    return !(v && v[0] == '0');
}

// The epilogue's tensor maps (make_epi_map): step 0's FULL operand, [M, N],
// its own pitch (FusedParams::tma_c); the output, [M, N], pitch ldo (tma_out).
struct EpiMaps {
    CUtensorMap c;
    CUtensorMap out;
};

// One unit of a CTA pair's work: k-blocks [kb0, kb1) of tile t.
enum : int { kWorkFull = 0, kWorkHead = 1, kWorkTail = 2 };
struct PairWork {
    int t, kb0, kb1, kind;
};

// Item `idx` of pair `pair`'s list, in execution order: its whole tiles of
// the first waves (one per pair in turn, so the pairs keep step through them
// and share A and B in L2 as without stream-K), then its stream-K head (if
// any), the whole tiles inside its stream-K range, and its stream-K tail (if
// any), which comes last so that the neighbouring pair's head is long done.
// False past the end.
__host__ __device__ __forceinline__ bool pair_work(const FusedParams& p, int pair, int num_pairs, int idx,
                                                   PairWork& w) {
    const int nk = p.num_kb;
    if (p.sk_q == 0) {
        w.t = pair + idx * num_pairs;
        w.kb0 = 0;
        w.kb1 = nk;
        w.kind = kWorkFull;
        return w.t < p.num_tiles;
    }
    const long long s = static_cast<long long>(pair) * p.sk_q + (pair < p.sk_extra ? pair : p.sk_extra);
    const long long e = s + p.sk_q + (pair < p.sk_extra ? 1 : 0);
    const int tile_lo = static_cast<int>(s / nk), tile_hi = static_cast<int>((e - 1) / nk);
    const int tail_kb = static_cast<int>(s - static_cast<long long>(tile_lo) * nk);      // > 0: tail of tile_lo
    const int head_kb = static_cast<int>(e - static_cast<long long>(tile_hi) * nk);      // < nk: head of tile_hi
    const bool has_tail = tail_kb > 0, has_head = head_kb < nk;
    int i = idx;
    const int n_dp = p.sk_dp_tiles / num_pairs;
    if (i < n_dp) {
        w.t = pair + i * num_pairs;
        w.kb0 = 0;
        w.kb1 = nk;
        w.kind = kWorkFull;
        return true;
    }
    i -= n_dp;
    if (has_head) {
        if (i == 0) {
            w.t = p.sk_dp_tiles + tile_hi;
            w.kb0 = 0;
            w.kb1 = head_kb;
            w.kind = kWorkHead;
            return true;
        }
        --i;
    }
    const int f_lo = has_tail ? tile_lo + 1 : tile_lo, f_hi = has_head ? tile_hi - 1 : tile_hi;
    if (i <= f_hi - f_lo) {
        w.t = p.sk_dp_tiles + f_lo + i;
        w.kb0 = 0;
        w.kb1 = nk;
        w.kind = kWorkFull;
        return true;
    }
    i -= f_hi >= f_lo ? f_hi - f_lo + 1 : 0;
    if (has_tail && i == 0) {
        w.t = p.sk_dp_tiles + tile_lo;
        w.kb0 = tail_kb;
        w.kb1 = nk;
        w.kind = kWorkTail;
        return true;
    }
    return false;
}

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

// The node's steps for W columns of one row.  step0_applied: the caller has
// already added step 0's FULL operand (read from a TMA box).
template <int W = 32>
__device__ __forceinline__ void apply_epilogue(float (&v)[W], int row, int col, bool row_ok,
                                               const FusedParams& p, const float* prod = nullptr, int b = 0,
                                               bool step0_applied = false) {
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
            if (!row_ok || (s == 0 && step0_applied)) continue;
            const long long ld = p.steps[s].ld_or_size;
            const float* src = ptr + static_cast<long long>(row) * ld + col;
            if (b) src += b * p.ep_bstride[s];
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
                static_cast<unsigned long long>(row + p.row_base + static_cast<long long>(b) * p.M) *
                    static_cast<unsigned long long>(p.N) + col;
#pragma unroll
            for (int i = 0; i < W; ++i)
                if (col + i < p.N) v[i] += __ldg(ptr + (base + i) % size);
        }
    }
}

// The same steps for four columns col .. col + 3 of R rows at once
// (v[u] is row row[u]; rows with ok[u] false are left alone), step by step
// across the rows, so the loads of one step for all R rows are in flight
// together.  Bits as apply_epilogue<4> row by row.
template <int R>
__device__ __forceinline__ void apply_epilogue_rows(float (&v)[R][4], const int (&row)[R], const bool (&ok)[R],
                                                    int col, const FusedParams& p) {
    const bool full_cols = col + 4 <= p.N;
    for (int s = 0; s < p.n_steps; ++s) {
        const int kind = p.steps[s].kind;
        const float* ptr = p.steps[s].ptr;
        if (kind == MXB_EP_RELU) {
#pragma unroll
            for (int u = 0; u < R; ++u)
#pragma unroll
                for (int i = 0; i < 4; ++i) v[u][i] = v[u][i] > 0.0f ? v[u][i] : 0.0f;
        } else if (kind == MXB_EP_SCALE) {
            const float sc = p.steps[s].scale;
#pragma unroll
            for (int u = 0; u < R; ++u)
#pragma unroll
                for (int i = 0; i < 4; ++i) v[u][i] = v[u][i] * sc;
        } else if (kind == MXB_EP_ADD_FULL) {
            const long long ld = p.steps[s].ld_or_size;
            float add[R][4];
#pragma unroll
            for (int u = 0; u < R; ++u) {
#pragma unroll
                for (int i = 0; i < 4; ++i) add[u][i] = 0.0f;
                if (!ok[u]) continue;
                const float* src = ptr + static_cast<long long>(row[u]) * ld + col;
                if (full_cols && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
                    const float4 c = __ldcs(reinterpret_cast<const float4*>(src));
                    add[u][0] = c.x;
                    add[u][1] = c.y;
                    add[u][2] = c.z;
                    add[u][3] = c.w;
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        if (col + i < p.N) add[u][i] = __ldcs(src + i);
                }
            }
#pragma unroll
            for (int u = 0; u < R; ++u)
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    if (ok[u] && col + i < p.N) v[u][i] += add[u][i];
        } else if (kind == MXB_EP_ADD_ROW) {
            float add[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) add[i] = col + i < p.N ? __ldg(ptr + col + i) : 0.0f;
#pragma unroll
            for (int u = 0; u < R; ++u)
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    if (col + i < p.N) v[u][i] += add[i];
        } else if (kind == MXB_EP_ADD_MOD) {
            const unsigned long long size = static_cast<unsigned long long>(p.steps[s].ld_or_size);
#pragma unroll
            for (int u = 0; u < R; ++u) {
                if (!ok[u]) continue;
                const unsigned long long base =
                    static_cast<unsigned long long>(row[u] + p.row_base) * static_cast<unsigned long long>(p.N) + col;
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    if (col + i < p.N) v[u][i] += __ldg(ptr + (base + i) % size);
            }
        }
    }
}

template <int W = 32>
__device__ __forceinline__ void store_row_chunk(const float (&v)[W], int row, int col,
                                                const FusedParams& p, long long off = 0) {
    float* dst = p.out + off + static_cast<long long>(row) * p.ldo + col;
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

// Copies rows row0 .. row0 + 31 (those below M), columns c0 .. c1, of the
// output into every peer's copy.  The calling warp stored these rows just
// before (lane i row row0 + i), so __syncwarp orders those stores before the
// loads, which hit L2.  One instruction moves 512 contiguous bytes of a row;
// kU rows are in flight at a time.  The stores are plain global stores to
// peer addresses (NVLink), so this warp's cost is issue only while the link
// drains, and it runs while the MMA warp is already on the next tile.  Each
// warp starts its round of peers at a different one (by its 32-row block),
// so the warps of a GPU spread their stores over every peer's ingress at
// once instead of all writing to the same GPU first.
template <int kU = 4>
__device__ __forceinline__ void push_rows(const FusedParams& p, int row0, int c0, int c1) {
    __syncwarp();
    const int lane = threadIdx.x & 31;
    const int rows = min(32, p.M - row0);
    if (rows <= 0 || c0 >= c1) return;
    const int q0 = (row0 >> 5) % p.n_peers;
    if (p.push_vec) {
        // c0 is a multiple of 32, so every float4 below is 16-byte aligned.
        const int segs = (c1 - c0 + 127) / 128;  // 128-column segments per row
        const int items = rows * segs;
        for (int i0 = 0; i0 < items; i0 += kU) {
            float4 v[kU];
            long long off[kU];
            int col[kU];
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int i = i0 + u;
                const int r = i / segs;
                col[u] = c0 + (i - r * segs) * 128 + 4 * lane;
                if (i >= items) col[u] = c1;  // nothing to copy
                off[u] = static_cast<long long>(row0 + r) * p.ldo + col[u];
                if (col[u] + 4 <= c1) v[u] = *reinterpret_cast<const float4*>(p.out + off[u]);
            }
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                if (col[u] + 4 <= c1) {
                    int q = q0;
                    for (int j = 0; j < p.n_peers; ++j) {
                        *reinterpret_cast<float4*>(p.peer_out[q] + off[u]) = v[u];
                        q = q + 1 == p.n_peers ? 0 : q + 1;
                    }
                } else {
                    // Row tail when N % 4 != 0: at most three scalars.
                    for (int j = 0; col[u] + j < c1; ++j) {
                        const float x = p.out[off[u] + j];
                        for (int q = 0; q < p.n_peers; ++q) p.peer_out[q][off[u] + j] = x;
                    }
                }
            }
        }
    } else {
        for (int r = 0; r < rows; ++r) {
            const long long base = static_cast<long long>(row0 + r) * p.ldo;
            for (int c = c0 + lane; c < c1; c += 32) {
                const float x = p.out[base + c];
                for (int q = 0; q < p.n_peers; ++q) p.peer_out[q][base + c] = x;
            }
        }
    }
}

// Stores one row's 32 raw accumulator values (columns col .. col + 31, those
// below n) at dst, 16-byte aligned when the chunk is whole.
__device__ __forceinline__ void store_partial(const uint32_t (&r)[32], float* dst, int col, int n) {
    if (col + 32 <= n) {
        float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
        for (int i = 0; i < 8; ++i)
            __stcg(d4 + i, make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                                       __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3])));
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if (col + i < n) __stcg(dst + i, __uint_as_float(r[i]));
    }
}

// v = slice 0 + slice 1 + ... of row `row`, columns col .. col + 3 (zero past
// N), in slice order.
__device__ __forceinline__ void sum_slices4(float (&v)[4], const FusedParams& p, int row, int col) {
    const float* src = p.ks_ws + static_cast<long long>(row) * p.ks_ld + col;
    if (col + 4 <= p.N) {
        float4 x = __ldcg(reinterpret_cast<const float4*>(src));
        v[0] = x.x;
        v[1] = x.y;
        v[2] = x.z;
        v[3] = x.w;
        for (int s = 1; s < p.splits; ++s) {
            x = __ldcg(reinterpret_cast<const float4*>(src + s * p.ks_stride));
            v[0] += x.x;
            v[1] += x.y;
            v[2] += x.z;
            v[3] += x.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float x = 0.0f;
            if (col + i < p.N) {
                x = __ldcg(src + i);
                for (int s = 1; s < p.splits; ++s) x += __ldcg(src + s * p.ks_stride + i);
            }
            v[i] = x;
        }
    }
}

// Pulls this thread's rows of every full-matrix ADD operand, columns
// col .. col + ncols, into L2 ahead of the epilogue's loads.
__device__ __forceinline__ void prefetch_full_operands(int row, int col, int ncols, const FusedParams& p,
                                                       int b = 0) {
    for (int s = 0; s < p.n_steps; ++s) {
        if (p.steps[s].kind != MXB_EP_ADD_FULL) continue;
        const float* src = p.steps[s].ptr + static_cast<long long>(row) * p.steps[s].ld_or_size + col;
        if (b) src += b * p.ep_bstride[s];
        for (int c = 0; c < ncols; c += 32)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<uint64_t>(src + c)));
    }
}

// ------------------------------------------------------------------ tensor maps

// Encoders of the tensor maps the kernels read and write; all go through
// encode_tensor_map (tensor_maps.cu), which caches the descriptors.
// Row-major [rows, cols] fp32 with row pitch `ld` elements; box [box_rows][box_cols].
// TFLOAT32: TMA rounds each fp32 element to TF32 (nearest even) on load.
bool make_map(CUtensorMap* map, const float* base, long long rows, long long cols, long long ld,
              int box_cols, int box_rows, CUtensorMapSwizzle swizzle) {
    const unsigned long long dims[2] = {static_cast<unsigned long long>(cols), static_cast<unsigned long long>(rows)};
    const unsigned long long strides[1] = {static_cast<unsigned long long>(ld) * 4};
    const unsigned box[2] = {static_cast<unsigned>(box_cols), static_cast<unsigned>(box_rows)};
    return encode_tensor_map(map, CU_TENSOR_MAP_DATA_TYPE_TFLOAT32, 2, base, dims, strides, box, swizzle,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
}

// Row-major [rows, cols] fp32 destination of TMA tile stores (FLOAT32, no
// swizzle), row pitch `ld` elements; box [box_rows][box_cols].
bool make_store_map(CUtensorMap* map, const float* base, long long rows, long long cols, long long ld, int box_cols,
                    int box_rows) {
    const unsigned long long dims[2] = {static_cast<unsigned long long>(cols), static_cast<unsigned long long>(rows)};
    const unsigned long long strides[1] = {static_cast<unsigned long long>(ld) * 4};
    const unsigned box[2] = {static_cast<unsigned>(box_cols), static_cast<unsigned>(box_rows)};
    return encode_tensor_map(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE);
}

// Row-major [rows, cols] fp32 read or written by the epilogue as 32 x 32
// boxes (FLOAT32: no rounding), 128-byte swizzled in shared memory: row r's
// 16-byte chunk j sits at position j ^ (r % 8), so a warp whose lane r reads
// or writes one chunk of row r touches eight different bank groups.
bool make_epi_map(CUtensorMap* map, const float* base, long long rows, long long cols, long long ld) {
    const unsigned long long dims[2] = {static_cast<unsigned long long>(cols), static_cast<unsigned long long>(rows)};
    const unsigned long long strides[1] = {static_cast<unsigned long long>(ld) * 4};
    const unsigned box[2] = {32, 32};
    return encode_tensor_map(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B);
}

// `batch` row-major [rows, cols] fp32 matrices, `bstride` elements apart, row
// pitch `ld`; box [1][box_rows][box_cols].  Rows and columns past a matrix's
// edge read as zeros, never as the next matrix's.
bool make_map_3d(CUtensorMap* map, const float* base, long long batch, long long rows, long long cols,
                 long long ld, long long bstride, int box_cols, int box_rows, CUtensorMapSwizzle swizzle) {
    const unsigned long long dims[3] = {static_cast<unsigned long long>(cols), static_cast<unsigned long long>(rows),
                                        static_cast<unsigned long long>(batch)};
    const unsigned long long strides[2] = {static_cast<unsigned long long>(ld) * 4,
                                           static_cast<unsigned long long>(bstride) * 4};
    const unsigned box[3] = {static_cast<unsigned>(box_cols), static_cast<unsigned>(box_rows), 1};
    return encode_tensor_map(map, CU_TENSOR_MAP_DATA_TYPE_TFLOAT32, 3, base, dims, strides, box, swizzle,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
}

}  // namespace
}  // namespace mxb
