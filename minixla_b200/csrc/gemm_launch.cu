// GEMM dispatch for graph nodes: pitch padding for TMA, the skinny / single-CTA
// / CTA-pair choice with 3xTF32 workspace, epilogue steps from EpSteps, and
// the helpers every executor shares (finish, result tensors, ordering events).
#include <cuda_runtime.h>
#include <sys/mman.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "runtime_internal.h"

namespace mxb {

// ---------------------------------------------------------------- GEMM dispatch


// TMA needs 16-byte row pitches: a matrix whose width is not a multiple of 4
// is copied into a pitch-padded temporary (one strided device copy).
bool tma_operand(GpuCtx* ctx, const float* src, long long rows, long long cols, Operand& op,
                 cudaStream_t stream) {
    if (cols % 4 == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
        op.ptr = src;
        op.ld = cols;
        return true;
    }
    const long long ld = (cols + 3) / 4 * 4;
    float* tmp = static_cast<float*>(ctx->pool->alloc(static_cast<size_t>(rows * ld) * 4, stream));
    if (!tmp) return false;
    if (!cuda_ok(cudaMemcpy2DAsync(tmp, ld * 4, src, cols * 4, cols * 4, rows, cudaMemcpyDeviceToDevice,
                                   stream),
                 "pitch-padding copy")) {
        ctx->pool->release(tmp, stream);
        return false;
    }
    op.ptr = tmp;
    op.ld = ld;
    op.owned = tmp;
    return true;
}


// Whether launch_gemm runs a shared-A second product in the same kernel:
// TF32 always (M > 16); 3xTF32 when the 256 x 128 pair tiles occupy a
// quarter of the SMs (else two launches, on the single-CTA kernels).
static bool dual_in_one_kernel(const GpuCtx* ctx, const float* A, long long lda, int M, int N, int K,
                               const Product& prod, int precision) {
    if (M <= kSkinnyMaxRows || !dual_kernel_enabled() || prod.A != A || prod.lda != lda || prod.K != K) return false;
    if (precision == GPU_PRECISION_TF32) return true;
    const long long tiles = static_cast<long long>((M + 255) / 256) * ((N + 127) / 128);
    return M >= 256 && tiles >= ctx->num_sms / 4;
}

int launch_gemm(GpuCtx* ctx, const float* A, long long lda, const float* B, long long ldb, float* out,
                long long ldo, int M, int N, int K, const EpStepDev* steps, int n_steps, int precision,
                cudaStream_t stream, const float* B_small_pre, long long row_base,
                const Product* prod, int choice_rows, PeerRows* peers, const BatchSpec* batch) {
    const int rows_for_choice = choice_rows > 0 ? choice_rows : M;
    const long long nb = batch && batch->count > 1 ? batch->count : 1;
    if (nb > 1 && (prod || (peers && peers->n > 0) || !batch->ep_bstride)) return MXB_E_ARG;
    if (prod && !dual_in_one_kernel(ctx, A, lda, M, N, K, *prod, precision)) {
        // Two launches: the second product into pooled workspace, then the
        // node reading it as a full add at the same step.
        float* ws = static_cast<float*>(ctx->pool->alloc(static_cast<size_t>(M) * N * sizeof(float), stream));
        if (!ws) return MXB_E_NOMEM;
        int rc = launch_gemm(ctx, prod->A, prod->lda, prod->B, prod->ldb, ws, N, M, N, prod->K, nullptr, 0, precision,
                             stream, prod->B_small, 0, nullptr, rows_for_choice);
        if (rc == MXB_OK) {
            EpStepDev st2[MXB_MAX_EPILOGUE];
            for (int i = 0; i < n_steps; ++i) {
                st2[i] = steps[i];
                if (st2[i].kind == MXB_EP_ADD_PRODUCT) {
                    st2[i].kind = MXB_EP_ADD_FULL;
                    st2[i].ptr = ws;
                    st2[i].ld_or_size = N;
                }
            }
            rc = launch_gemm(ctx, A, lda, B, ldb, out, ldo, M, N, K, st2, n_steps, precision, stream, B_small_pre,
                             row_base, nullptr, rows_for_choice);
        }
        ctx->pool->release(ws, stream);
        return rc;
    }
    // A batch was routed here by batched_in_one_launch: tensor-core kernels only.
    const bool skinny = nb == 1 && use_skinny_gemm(rows_for_choice, precision);
    if (nb == 1 && !skinny && use_tiny_gemm(rows_for_choice, N, K, precision)) {
        // Small enough that one plain CUDA-core launch beats the set-up of the tensor-core kernels.
        return cuda_ok(launch_tiny_gemm(A, lda, B, ldb, out, ldo, M, N, K, row_base, steps, n_steps, stream),
                       "tiny GEMM launch")
                   ? MXB_OK
                   : MXB_E_CUDA;
    }
    if (skinny) {
        // Few rows: HBM-bound on B, CUDA-core fp32 split over columns and K.
        const SkinnyPlan pl = plan_skinny(M, N, K, ctx->num_sms);
        float* ws = nullptr;  // the one-kernel form needs no workspace
        if (!pl.one_kernel) {
            ws = static_cast<float*>(ctx->pool->alloc(static_cast<size_t>(pl.splits) * M * N * sizeof(float), stream));
            if (!ws) return MXB_E_NOMEM;
        }
        const int rc = cuda_ok(launch_skinny_gemm(A, lda, B, ldb, out, ldo, M, N, K, row_base, steps, n_steps, ws, pl,
                                                  ctx->num_sms, stream),
                               "skinny GEMM launch")
                           ? MXB_OK
                           : MXB_E_CUDA;
        ctx->pool->release(ws, stream);
        return rc;
    }
    GemmLaunch g{};
    g.row_base = row_base;
    g.A = A;
    g.lda = lda;
    g.B = B;
    g.ldb = ldb;
    g.out = out;
    g.ldo = ldo;
    g.M = M;
    g.N = N;
    g.K = K;
    g.steps = steps;
    g.n_steps = n_steps;
    g.precision = precision;
    if (prod) {
        g.A2 = prod->A;
        g.lda2 = prod->lda;
        g.B2 = prod->B;
        g.ldb2 = prod->ldb;
        g.K2 = prod->K;
    }
    g.err = ctx->d_err;
    g.timeout_ns = ctx->timeout_ns;
    g.num_sms = ctx->num_sms;
    if (peers && peers->n > 0 && !prod && fused_gemm_pushes_rows(g)) {
        g.peer_out = peers->out;
        g.n_peers = peers->n;
    }
    g.choice_rows = rows_for_choice;
    if (nb > 1) {
        g.batch = nb;
        g.a_bstride = static_cast<long long>(M) * lda;
        g.b_bstride = static_cast<long long>(K) * ldb;
        g.out_bstride = static_cast<long long>(M) * ldo;
        g.ep_bstride = batch->ep_bstride;
    }
    // 3xTF32 low parts of A, B, B2; K-split slices; stream-K accumulators and flags
    float* ws[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
    int rc = MXB_OK;
    g.k_splits = fused_gemm_k_splits(g);
    if (g.k_splits > 1 && !fused_gemm_ksplit_in_cluster(g)) {
        // Raw partial sums, one M x round4(N) slice per K slice.
        const size_t slice = static_cast<size_t>(M) * ((N + 3) / 4 * 4);
        ws[3] = static_cast<float*>(ctx->pool->alloc(g.k_splits * slice * sizeof(float), stream));
        if (!ws[3]) rc = MXB_E_NOMEM;
        g.ks_ws = ws[3];
    }
    if (const size_t skb = rc == MXB_OK ? fused_gemm_streamk_bytes(g) : 0) {
        // The CTA-pair kernel's stream-K hand-off: accumulators of the pairs
        // that run a split tile's first k-blocks, then one flag per epilogue warp.
        const int pairs = ctx->num_sms / 2;
        ws[4] = static_cast<float*>(ctx->pool->alloc(skb, stream));
        if (!ws[4]) rc = MXB_E_NOMEM;
        g.sk_ws = ws[4];
        g.sk_flags = ws[4] ? reinterpret_cast<int*>(ws[4] + (skb - static_cast<size_t>(pairs) * 16 * sizeof(int)) /
                                                                sizeof(float))
                           : nullptr;
        g.sk_pairs = pairs;
        g.sk_cols = plan_fused_gemm(g, 1).tile_cols;
    }
    if (rc == MXB_OK && precision == GPU_PRECISION_3XTF32) {
        // Low parts of every product of a batch (stored back to back like A and B).
        const size_t a_bytes = static_cast<size_t>(nb * M) * lda * 4, b_bytes = static_cast<size_t>(nb * K) * ldb * 4;
        const bool need_b2 = prod && !prod->B_small;
        ws[0] = static_cast<float*>(ctx->pool->alloc(a_bytes, stream));
        if (ws[0] && !B_small_pre) ws[1] = static_cast<float*>(ctx->pool->alloc(b_bytes, stream));
        if (ws[0] && need_b2)
            ws[2] = static_cast<float*>(ctx->pool->alloc(static_cast<size_t>(K) * prod->ldb * 4, stream));
        if (!ws[0] || (!B_small_pre && !ws[1]) || (need_b2 && !ws[2])) {
            rc = MXB_E_NOMEM;
        } else if (!cuda_ok(launch_split_tf32(A, nb * M, K, lda, ws[0], lda, ctx->num_sms, stream), "split A") ||
                   (!B_small_pre &&
                    !cuda_ok(launch_split_tf32(B, nb * K, N, ldb, ws[1], ldb, ctx->num_sms, stream), "split B")) ||
                   (need_b2 && !cuda_ok(launch_split_tf32(prod->B, K, N, prod->ldb, ws[2], prod->ldb, ctx->num_sms,
                                                          stream),
                                        "split B2"))) {
            rc = MXB_E_CUDA;
        } else {
            g.A_small = ws[0];
            g.B_small = B_small_pre ? B_small_pre : ws[1];
            if (prod) g.B2_small = prod->B_small ? prod->B_small : ws[2];
        }
    }
    if (rc == MXB_OK && !cuda_ok(launch_fused_gemm(g, stream), "fused GEMM launch")) rc = MXB_E_CUDA;
    if (rc == MXB_OK && g.n_peers > 0) peers->pushed = true;
    for (float* w : ws) ctx->pool->release(w, stream);
    return rc;
}

// Builds the device epilogue of an OP_FUSED node from its EpSteps
// (graph.h:17-18) for batch `bt` of `batch`.  eval_fused adds
// op[(bt*M*N + i*N + j) % size] (graph.c:100-105): an operand holding every
// batch (batch*M*N elements) is FULL at this batch's offset; one holding one
// M x N block is FULL for every batch; a [N] row is ROW; any other size
// keeps the modulo rule (MOD, rows counted from bt*M through row_base).
// RELU maps to RELU; other step ops are skipped, as eval_fused skips them.
int build_epilogue(const Node* n, int M, int N, long long batch, long long bt,
                   const std::unordered_map<const Node*, const float*>& dev_of,
                   const std::unordered_map<const Node*, long long>& size_of, EpStepDev* out,
                   const Node* absorbed) {
    const long long MN = static_cast<long long>(M) * N;
    int k = 0;
    for (int e = 0; e < n->n_epilogue; ++e) {
        const EpStep& s = n->epilogue[e];
        EpStepDev d{};
        if (s.op == OP_ADD && absorbed && s.operand == absorbed) {
            d.kind = MXB_EP_ADD_PRODUCT;  // the absorbed matmul, computed in the same kernel
        } else if (s.op == OP_ADD) {
            const long long sz = size_of.at(s.operand);
            d.ptr = dev_of.at(s.operand);
            if (sz == batch * MN) {
                d.kind = MXB_EP_ADD_FULL;
                d.ptr += bt * MN;
                d.ld_or_size = N;
            } else if (sz == MN) {
                d.kind = MXB_EP_ADD_FULL;
                d.ld_or_size = N;
            } else if (sz == N) {
                d.kind = MXB_EP_ADD_ROW;
                d.ld_or_size = N;
            } else {
                d.kind = MXB_EP_ADD_MOD;
                d.ld_or_size = sz;
            }
        } else if (s.op == OP_RELU) {
            d.kind = MXB_EP_RELU;
        } else {
            continue;
        }
        out[k++] = d;
    }
    return k;
}

// Batched (rank-3) nodes: products that leave most of the GPU idle one at a
// time run together in one launch of the single-CTA kernel (3-D tensor maps,
// the product index from the tile index).  Larger products keep their own
// launches on the kernels chosen for their shape, as do few-row products
// (skinny kernels) and, in 3xTF32 mode, batches small enough in total for the
// one-launch CUDA-core kernel.  MINIXLA_BATCH_LAUNCH=0 keeps one launch per
// product.
bool batched_in_one_launch(int num_sms, long long batch, int M, int N, int K, int precision) {
    if (batch < 2) return false;
    if (const char* v = getenv("MINIXLA_BATCH_LAUNCH"))
        if (v[0] == '0') return false;
    if (use_skinny_gemm(M, precision)) return false;
    const long long rows_total = batch * M;
    if (rows_total < (1ll << 31) && use_tiny_gemm(static_cast<int>(rows_total), N, K, precision)) return false;
    const long long tiles = static_cast<long long>((M + 127) / 128) * ((N + 127) / 128);
    return tiles < num_sms;
}

// Runs one matmul-anchored node on device buffers: `batch` products of
// A[M,K] @ B[K,N] stored back to back (batch = 1 for 2-D nodes).
int run_gemm_node(GpuCtx* ctx, const Node* n, const float* dA, int M, int K, const float* dB, int N,
                  float* dOut, const std::unordered_map<const Node*, const float*>& dev_of,
                  const std::unordered_map<const Node*, long long>& size_of, int precision,
                  cudaStream_t stream, long long batch, const Node* absorbed,
                  const Product* prod) {
    Operand a, b;
    int rc = MXB_OK;
    // Pitch padding treats the batches as one tall matrix (rows are contiguous).
    if (!tma_operand(ctx, dA, batch * M, K, a, stream) || !tma_operand(ctx, dB, batch * K, N, b, stream)) {
        rc = MXB_E_NOMEM;
    }
    if (rc == MXB_OK && !prod && batched_in_one_launch(ctx->num_sms, batch, M, N, K, precision)) {
        // Every product in one launch.  A FULL operand's step for product 1
        // differs from product 0's by its batch stride (M * N for an operand
        // holding every product, 0 for one M x N block); the modulo rule's
        // row count advances by M per product inside the kernel.
        EpStepDev steps[MXB_MAX_EPILOGUE], next[MXB_MAX_EPILOGUE];
        long long bstride[MXB_MAX_EPILOGUE] = {};
        int n_steps = 0;
        if (n->op == OP_FUSED) {
            n_steps = build_epilogue(n, M, N, batch, 0, dev_of, size_of, steps, absorbed);
            build_epilogue(n, M, N, batch, 1, dev_of, size_of, next, absorbed);
            for (int i = 0; i < n_steps; ++i)
                if (steps[i].kind == MXB_EP_ADD_FULL) bstride[i] = next[i].ptr - steps[i].ptr;
        }
        BatchSpec bs;
        bs.count = batch;
        bs.ep_bstride = bstride;
        rc = launch_gemm(ctx, a.ptr, a.ld, b.ptr, b.ld, dOut, N, M, N, K, steps, n_steps, precision, stream, nullptr,
                         0, nullptr, 0, nullptr, &bs);
        ctx->pool->release(a.owned, stream);
        ctx->pool->release(b.owned, stream);
        return rc;
    }
    for (long long bt = 0; bt < batch && rc == MXB_OK; ++bt) {
        EpStepDev steps[MXB_MAX_EPILOGUE];
        const int n_steps =
            n->op == OP_FUSED ? build_epilogue(n, M, N, batch, bt, dev_of, size_of, steps, absorbed) : 0;
        rc = launch_gemm(ctx, a.ptr + bt * M * a.ld, a.ld, b.ptr + bt * K * b.ld, b.ld,
                         dOut + bt * static_cast<long long>(M) * N, N, M, N, K, steps, n_steps, precision, stream,
                         nullptr, bt * M, prod);
    }
    ctx->pool->release(a.owned, stream);
    ctx->pool->release(b.owned, stream);
    return rc;
}

// Synchronises the context stream and folds a device-side error word into a code.
int finish(GpuCtx* ctx) {
    if (!cuda_ok(cudaStreamSynchronize(ctx->stream), "stream synchronize")) return MXB_E_CUDA;
    int err = 0;
    if (!cuda_ok(cudaMemcpy(&err, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost), "error word read"))
        return MXB_E_CUDA;
    if (err) {
        cudaMemset(ctx->d_err, 0, sizeof(int));
        set_error("a device-side wait ran out of time (error bits 0x%x); results discarded", err);
        return MXB_E_TIMEOUT;
    }
    return MXB_OK;
}

Tensor* new_host_tensor(const std::vector<int>& dims) {
    // Same allocation pattern as create_tensor (tensor.c:8-53), so the caller
    // releases the result with the reference's free_tensor.
    Tensor* t = static_cast<Tensor*>(calloc(1, sizeof(Tensor)));
    if (!t) return nullptr;
    t->ndim = static_cast<int>(dims.size());
    t->shape = static_cast<int*>(malloc(dims.size() * sizeof(int)));
    t->strides = static_cast<size_t*>(malloc(dims.size() * sizeof(size_t)));
    size_t size = 1;
    if (t->shape && t->strides) {
        for (int i = t->ndim - 1; i >= 0; --i) {
            t->shape[i] = dims[i];
            t->strides[i] = size;
            size *= static_cast<size_t>(dims[i]);
        }
    }
    t->size = size;
    // Large results: 2 MiB-aligned with transparent huge pages requested, so
    // the download into fresh memory takes one page fault per 2 MiB instead
    // of one per 4 KiB.  posix_memalign memory is released by free(), as
    // free_tensor does.
    const size_t bytes = size * sizeof(float);
    void* data = nullptr;
    if (bytes >= (8u << 20)) {
        if (posix_memalign(&data, 2u << 20, bytes) != 0) data = nullptr;
        if (data) madvise(data, bytes, MADV_HUGEPAGE);  // advice only: ignored where unsupported
    } else {
        data = malloc(bytes);
    }
    t->data = static_cast<float*>(data);
    if (!t->shape || !t->strides || !t->data) {
        free(t->data);
        free(t->shape);
        free(t->strides);
        free(t);
        return nullptr;
    }
    return t;
}

}  // namespace mxb
