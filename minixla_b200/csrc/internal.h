// Internal declarations shared by the library's translation units.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>
#include <cstddef>

#include "../../include/minixla_b200.h"

namespace mxb {

// Device-side copy of one epilogue step; byte-identical to mxb_ep_step.
struct EpStepDev {
    int kind;
    int reserved;
    const float* ptr;
    long long ld_or_size;
    float scale;
    int reserved2;
};
static_assert(sizeof(EpStepDev) == sizeof(mxb_ep_step), "EpStepDev must mirror mxb_ep_step");

// Everything a fused-GEMM launch needs besides the tensor maps.
// Peer copies of a row all-gather that the TF32 CTA-pair kernel writes itself
// (one process per GPU on one NVLink domain: at most eight GPUs).
constexpr int kMaxPeers = MXB_MAX_PEERS;

struct GemmLaunch {
    const float* A; long long lda;     // M x K, lda % 4 == 0
    const float* B; long long ldb;     // K x N, ldb % 4 == 0
    const float* A_small;              // 3xTF32 only: x - rne_tf32(x), same pitches
    const float* B_small;
    const float* A2; long long lda2;   // optional second product A2[M,K2] @ B2[K2,N], added at the
    const float* B2; long long ldb2;   // MXB_EP_ADD_PRODUCT step; A2 == nullptr: none
    const float* B2_small;             // 3xTF32 only: low part of B2
    int K2;
    float* out; long long ldo;
    int M, N, K;
    long long row_base;                // global index of row 0 (rows of a larger matrix)
    const EpStepDev* steps; int n_steps;
    int precision;                     // GPU_PRECISION_TF32 / GPU_PRECISION_3XTF32
    int* err;                          // device error word
    unsigned long long timeout_ns;
    int num_sms;
    float* const* peer_out;            // n_peers > 0: also write the rows here (CTA-pair kernels only)
    int n_peers;
    int choice_rows;                   // rows the K split is chosen for (0: M)
    int k_splits;                      // > 1: single-CTA TF32 kernel with K split this many ways
    float* ks_ws;                      // k_splits * M * round4(N) floats
    // batch > 1: that many products of this shape in one launch, the b-th at
    // A + b * a_bstride, B + b * b_bstride (and the low parts likewise), out +
    // b * out_bstride; FULL epilogue step s reads b * ep_bstride[s] further on.
    long long batch;
    long long a_bstride, b_bstride, out_bstride;
    const long long* ep_bstride;
    // Stream-K workspace of the TF32 CTA-pair kernels (nullptr: none, every
    // tile whole on one pair): room for sk_pairs pairs' raw accumulators
    // (pairs x 2 x 128 x tile columns floats) and flags (pairs x 2 x 8 ints).
    float* sk_ws;
    int* sk_flags;
    int sk_pairs;
    int sk_cols;                       // tile columns sk_ws was sized for
};

// Stream-K workspace a launch of g needs (0: it runs no stream-K tail); the
// caller passes it as GemmLaunch::sk_ws / sk_flags with sk_pairs = num_sms / 2.
size_t fused_gemm_streamk_bytes(const GemmLaunch& g);
// Tiles of g run as stream-K work on num_sms / 2 pairs (0: none).
int fused_gemm_streamk_tiles(const GemmLaunch& g);

// Skinny GEMM (skinny_gemm.cu): few output rows, CUDA-core fp32, split over
// column blocks x K ranges; workspace holds splits * M * N floats.
constexpr int kSkinnyMaxRows = 16;
// Whether an M-row product (M: the node's full row count) runs on the skinny
// kernels: up to 8 rows in TF32 mode, 16 in 3xTF32 mode;
// MINIXLA_SKINNY_MAX_ROWS=n (0..16) sets the limit for both.
bool use_skinny_gemm(int M, int precision);
struct SkinnyPlan {
    bool one_kernel = false;  // cluster kernel: no workspace (splits == 0)
    int col_blocks = 1;
    int splits = 1;
    int k_per_split = 1;
};
SkinnyPlan plan_skinny(int M, int N, int K, int num_sms);
cudaError_t launch_skinny_gemm(const float* A, long long lda, const float* B, long long ldb, float* out, long long ldo,
                               int M, int N, int K, long long row_base, const EpStepDev* steps, int n_steps,
                               float* workspace, const SkinnyPlan& plan, int num_sms, cudaStream_t stream);

// Tiny dense problems in 3xTF32 mode (skinny_gemm.cu): one CUDA-core fp32
// kernel with 32 x 32 output tiles instead of two split kernels and the
// tensor-core GEMM, up to M*N*K <= kTinyMaxMnk3x (measured: 128^3 10.1 vs
// 19.4 us, 384^3 16.4 vs 25.5 us, 512^3 27.5 vs 25.5 us).  In TF32 mode the
// tensor-core kernels were as fast or faster at every size (128^3 9.1 vs
// 10.1 us), so kTinyMaxMnk is 0.  MINIXLA_TINY_MAX_MNK overrides both.
constexpr long long kTinyMaxMnk = 0;
constexpr long long kTinyMaxMnk3x = 1ll << 26;
bool use_tiny_gemm(int M, int N, int K, int precision);
cudaError_t launch_tiny_gemm(const float* A, long long lda, const float* B, long long ldb, float* out, long long ldo,
                             int M, int N, int K, long long row_base, const EpStepDev* steps, int n_steps,
                             cudaStream_t stream);

// Kernel launchers (fused_gemm.cu, elementwise.cu).  Return cudaError_t.
cudaError_t launch_fused_gemm(const GemmLaunch& g, cudaStream_t stream);
// Whether launch_fused_gemm(g) runs a CTA-pair kernel (TF32 or 3xTF32) for one
// product, the kernels that write peer rows themselves (MINIXLA_GATHER_PUSH=0:
// never).
bool fused_gemm_pushes_rows(const GemmLaunch& g);
// Kernel family (MXB_KERNEL_*), tile and K split that launch_fused_gemm runs
// for g when the caller provides workspace for `k_splits` slices (0 or 1:
// none); products = 2 for a shared-A second product in the same kernel.
struct GemmPlan {
    int kernel;
    int tile_rows, tile_cols;
    int k_splits;
    int products;
};
GemmPlan plan_fused_gemm(const GemmLaunch& g, int k_splits);
// How many ways launch_fused_gemm(g) splits K (1: none); the caller supplies
// the workspace a split needs (GemmLaunch::ks_ws).
int fused_gemm_k_splits(const GemmLaunch& g);
// Whether that split sums its slices inside the GEMM's clusters (no workspace).
bool fused_gemm_ksplit_in_cluster(const GemmLaunch& g);
constexpr int kKsplitTileRows = 128, kKsplitTileCols = 128;
cudaError_t launch_split_tf32(const float* x, long long rows, long long cols, long long ld_in,
                              float* small, long long ld_out, int num_sms, cudaStream_t stream);
cudaError_t launch_add(const float* a, long long n, const float* b, long long b_size, float* out,
                       int num_sms, cudaStream_t stream);
cudaError_t launch_relu(const float* x, long long n, float* out, int num_sms, cudaStream_t stream);
cudaError_t launch_wait_timeout_probe(int* err, unsigned long long timeout_ns, cudaStream_t stream);
cudaError_t launch_hold(unsigned long long ns, cudaStream_t stream);

// Host <-> device copies (hostcopy.cu): pageable host memory goes through a
// context's ring of pinned slots filled by several host threads; pinned
// memory and small copies go straight to cudaMemcpyAsync.  copy_d2h into
// pageable memory returns once the data has arrived.
class Stager;
Stager* stager_create();
void stager_destroy(Stager* s);
cudaError_t copy_h2d(Stager* s, void* dst, const void* src, size_t bytes, cudaStream_t stream);
cudaError_t copy_d2h(Stager* s, void* dst, const void* src, size_t bytes, cudaStream_t stream);
// Faults in fresh pageable host memory with the stager's copy threads (one
// write per page), ahead of downloads into it; nothing for pinned memory.
void prefault_host(Stager* s, void* dst, size_t bytes);

// cuTensorMapEncodeTiled through a per-process cache keyed by every argument
// (tensor_maps.cu): dtype / swizzle / l2_promotion are the CUtensorMap* enum
// values, dims and box have `rank` entries, strides rank - 1 (bytes).
// MINIXLA_TMAP_CACHE=0 encodes every time.  False when encoding fails.
bool encode_tensor_map(struct CUtensorMap_st* map, int dtype, int rank, const void* base,
                       const unsigned long long* dims, const unsigned long long* strides, const unsigned* box,
                       int swizzle, int l2_promotion);

// Process-wide count of kernel launches issued by this library.
void note_launch(unsigned n = 1);

// Records a failure message for mxb_last_error() and prints it to stderr.
void set_error(const char* fmt, ...);

}  // namespace mxb
