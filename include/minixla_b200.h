/*
 * minixla_b200 -- a B200 (sm_100a) backend for MiniXLA's OP_FUSED hot path.
 *
 * libminixla_b200.so is a drop-in replacement for MiniXLA's gpu_exec.c +
 * runtime.c + ptx.c.  A MiniXLA program keeps building its graph with the
 * reference's own tensor.c / graph.c / optimizer.c and links this library in
 * place of those three GPU files; it can keep including the reference's
 * gpu_exec.h / runtime.h unchanged.  Include this header (after the
 * reference's headers, if both are used) only for the additive API below.
 *
 * Conventions kept from the reference (gpu_exec.c:63-69, 240-248, 547-549):
 * failures return NULL or -1.0 and print one line to stderr; nothing aborts;
 * every device buffer is released on every path; calls are synchronous
 * (the result is on the host when the call returns); a GpuCtx is used from
 * one host thread at a time for graph execution (gpu_execute and friends).
 * The device-pointer launches (mxb_fused_gemm, mxb_fused_gemm2, mxb_add,
 * mxb_relu) only touch the context's pool, which is locked, and may come
 * from several threads.
 */
#ifndef MINIXLA_B200_H
#define MINIXLA_B200_H

#include <stddef.h>

#if defined(__GNUC__)
#define MXB_API __attribute__((visibility("default")))
#else
#define MXB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------
 * Host data model.  These are the reference's layouts, restated byte for
 * byte because the library reads caller-built graphs in place:
 *   Tensor  -- tensor.h:6-12
 *   OpType  -- graph.h:6-15
 *   EpStep  -- graph.h:17-18
 *   Node    -- graph.h:20-31
 * If the reference's tensor.h / graph.h were included first, their
 * definitions are used instead (same include guards' presence is checked).
 * ---------------------------------------------------------------------- */
#if !defined(TENSOR_H) && !defined(MXB_TENSOR_DEFINED)
#define MXB_TENSOR_DEFINED
typedef struct {
    float*  data;      /* row-major fp32, `size` elements; malloc'd        */
    int*    shape;     /* ndim extents                                      */
    size_t* strides;   /* ndim element strides (row-major)                  */
    int     ndim;
    size_t  size;      /* product of shape                                  */
} Tensor;
#endif

#if !defined(GRAPH_H) && !defined(MXB_GRAPH_DEFINED)
#define MXB_GRAPH_DEFINED
typedef enum {
    OP_INPUT,
    OP_MATMUL,
    OP_ADD,
    OP_MUL,
    OP_RELU,
    OP_SOFTMAX,
    OP_TRANSPOSE,
    OP_FUSED
} OpType;

struct Node;
typedef struct { OpType op; struct Node* operand; } EpStep;

typedef struct Node {
    OpType        op;
    struct Node** inputs;      /* OP_FUSED: [A, B, ADD operands in step order] */
    int           n_inputs;
    Tensor*       output;      /* set on OP_INPUT leaves                       */
    int           owns_output;
    char          visited;
    int           uses;
    char          is_const;
    EpStep*       epilogue;    /* OP_FUSED only: ADD(operand) / RELU steps     */
    int           n_epilogue;
} Node;
#endif

/* ------------------------------------------------------------------------
 * The reference's GPU entry points, same signatures and ownership
 * (gpu_exec.h:7-42, runtime.h:9).  Behavioural differences of this backend:
 *  - kernels are hand-written sm_100a (tcgen05 / TMEM / TMA) CUDA, picked per
 *    node signature; no PTX is generated or JIT-compiled;
 *  - gpu_execute also accepts a bare OP_MATMUL, standalone OP_ADD / OP_RELU
 *    nodes, and ADD operands of any size (a [N] bias row, or any operand by
 *    eval_fused's modulo rule, graph.c:100-105), where the reference GPU path
 *    refused them (gpu_exec.c:472-482, 515-518);
 *  - precision: gpu_execute / gpu_time_kernel_ms / gpu_run_fused compute in
 *    the context's precision mode (default 3xTF32, fp32-faithful);
 *    gpu_run_tensorcore / gpu_time_kernel_tc_ms always use one TF32 product,
 *    as the reference's tensor-core path does (ptx.c:352-595).
 * ---------------------------------------------------------------------- */
#ifndef GPU_EXEC_H
typedef struct GpuCtx GpuCtx;

/* Context on device 0 (or on $MINIXLA_DEVICE) -- gpu_exec.h:12-13. */
MXB_API GpuCtx* gpu_ctx_create(void);
/* Releases the context's streams, pooled device memory and kernels -- gpu_exec.h:14. */
MXB_API void    gpu_ctx_destroy(GpuCtx* ctx);
/* Runs the optimized DAG; returns a fresh host tensor for the root (caller
 * frees it with free_tensor).  Does not modify the graph -- gpu_exec.h:16-20. */
MXB_API Tensor* gpu_execute(Node* root, GpuCtx* ctx);
/* Kernel-only timing of one OP_FUSED node: inputs uploaded once, `warmup`
 * launches, then the minimum over `reps` CUDA-event-timed launches, in ms;
 * -1.0 on failure -- gpu_exec.h:21-32.  Also times rank-3 (batched) nodes,
 * which the reference's timer refused: every product of the batch. */
MXB_API double  gpu_time_kernel_ms(Node* root, GpuCtx* ctx, int warmup, int reps);
/* One OP_FUSED node through a single TF32 tensor-core product -- gpu_exec.h:34-39. */
MXB_API Tensor* gpu_run_tensorcore(const Node* fused, GpuCtx* ctx);
/* Kernel-only timing of the TF32 path -- gpu_exec.h:41-42. */
MXB_API double  gpu_time_kernel_tc_ms(Node* root, GpuCtx* ctx, int warmup, int reps);
#endif

#ifndef RUNTIME_H
/* Self-contained single-node run -- runtime.h:9.  `ptx` is accepted for ABI
 * compatibility and ignored: the kernel is chosen from the node itself. */
MXB_API Tensor* gpu_run_fused(const Node* fused, const char* ptx);
#endif

/* ------------------------------------------------------------------------
 * Additive API (no counterpart in the reference).
 * ---------------------------------------------------------------------- */

/* Precision modes. */
#define GPU_PRECISION_TF32    1   /* one TF32 product per k, fp32 accumulate        */
#define GPU_PRECISION_3XTF32  3   /* x = big + small split, three TF32 products:
                                     fp32-faithful results                          */

/* Context on a given CUDA device (one process per GPU).  NULL on failure. */
MXB_API GpuCtx* gpu_ctx_create_on(int device);
/* One context driving GPUs 0..ngpu-1 from this thread (gpu_ctx_create does
 * the same when $MINIXLA_NGPU > 1).  gpu_execute then splits the rows of
 * every row-wise node over the GPUs: leaves read whole (B operands, bias
 * rows) are uploaded once and replicated by peer copies over NVLink, row
 * leaves are uploaded shard by shard, each GPU computes its rows, and result
 * rows go from each GPU straight into the host tensor; an NCCL all-gather
 * runs only when a later node reads an intermediate whole.  Graphs that are
 * not row-wise run on GPU 0.  All other entry points use GPU 0.  NULL on
 * failure. */
MXB_API GpuCtx* gpu_ctx_create_multi(int ngpu);
/* Number of GPUs a context drives (1 unless made by gpu_ctx_create_multi). */
MXB_API int     gpu_ctx_ngpu(const GpuCtx* ctx);
/* The row split a multi-GPU context uses: part p of `parts` gets rows
 * [r0, r1) of M, the first M % parts parts one row more.  0 or MXB_E_ARG. */
MXB_API int     mxb_shard_rows(long long M, int parts, int part, long long* r0, long long* r1);
/* Keeps a host tensor (typically a weight) in device memory: it is uploaded
 * now, to every GPU of the context, and every later gpu_execute /
 * gpu_execute_into on this context reads that copy instead of uploading the
 * leaf again.  The caller must not change the tensor's data while it is
 * resident (release it and keep it again after a change); a tensor whose
 * data pointer or size changed since is uploaded as usual.  Resident copies
 * are freed by gpu_ctx_release_resident or gpu_ctx_destroy.  0 or MXB_E_*. */
MXB_API int     gpu_ctx_keep_resident(GpuCtx* ctx, const Tensor* t);
/* Frees the resident copy of `t`, or of every resident tensor when t is NULL. */
MXB_API int     gpu_ctx_release_resident(GpuCtx* ctx, const Tensor* t);
/* Sets / reads the precision used by gpu_execute, gpu_time_kernel_ms and
 * gpu_run_fused.  The initial mode comes from $MINIXLA_PRECISION ("tf32" or
 * "3xtf32"), else 3xTF32.  Returns 0, or -1 for an unknown mode. */
MXB_API int     gpu_ctx_set_precision(GpuCtx* ctx, int mode);
MXB_API int     gpu_ctx_get_precision(const GpuCtx* ctx);
/* Device index of the context, or -1. */
MXB_API int     gpu_ctx_device(const GpuCtx* ctx);

/* ---- Device-pointer entry points ----------------------------------------
 * For callers that keep operands resident in HBM (benchmarks, frameworks):
 * no host copies.  All pointers are device pointers of the context's device;
 * `stream` is a cudaStream_t (NULL = the context's own stream).  Launches are
 * asynchronous on that stream.  Return 0 on success, a negative MXB_E* code
 * on failure (and one stderr line).
 */
enum {
    MXB_EP_ADD_FULL = 0,  /* x += operand[i*ld + j]      (M x N operand, row pitch ld) */
    MXB_EP_ADD_ROW  = 1,  /* x += operand[j]             ([N] bias row)                */
    MXB_EP_ADD_MOD  = 2,  /* x += operand[(i*N + j) % size]  (eval_fused's rule)       */
    MXB_EP_RELU     = 3,  /* x = x > 0 ? x : 0                                         */
    MXB_EP_SCALE    = 4,  /* x *= scale                                                */
    MXB_EP_ADD_PRODUCT = 5 /* x += (A2 @ B2)[i,j]  (mxb_fused_gemm2's second product)   */
};
#define MXB_MAX_EPILOGUE 16   /* the reference fuses at most 16 steps (optimizer.c:104-107) */

typedef struct {
    int          kind;       /* MXB_EP_*                                  */
    int          reserved;
    const float* operand;    /* ADD_*: device pointer                     */
    long long    ld_or_size; /* ADD_FULL: row pitch; ADD_MOD: element count */
    float        scale;      /* SCALE                                     */
    int          reserved2;
} mxb_ep_step;

enum {
    MXB_OK          = 0,
    MXB_E_ARG       = -1,   /* bad shape / pointer / pitch / mode          */
    MXB_E_CUDA      = -2,   /* a CUDA runtime call failed                  */
    MXB_E_NOMEM     = -3,   /* device allocation failed                    */
    MXB_E_TIMEOUT   = -4,   /* a bounded device-side wait ran out          */
    MXB_E_UNSUPPORTED = -5  /* node or shape outside what the backend runs */
};

/* Like gpu_execute, but downloads the root into a caller-provided host
 * tensor with the same element count (for example one backed by pinned
 * memory, so the download runs at full link speed).  0 or an MXB_E_* code. */
MXB_API int gpu_execute_into(Node* root, GpuCtx* ctx, Tensor* out);

/* out[M,N] = epi(A[M,K] @ B[K,N]).  Row pitches lda, ldb, ldo in elements.
 * A and B must be 16-byte aligned with lda % 4 == 0 and ldb % 4 == 0 (TMA);
 * other shapes go through gpu_execute, which pads.  precision is
 * GPU_PRECISION_TF32 or GPU_PRECISION_3XTF32 (3xTF32 uses pooled workspace
 * from the context).  n_steps <= MXB_MAX_EPILOGUE. */
MXB_API int mxb_fused_gemm(GpuCtx* ctx,
                   const float* A, long long lda,
                   const float* B, long long ldb,
                   float* out, long long ldo,
                   int M, int N, int K,
                   const mxb_ep_step* steps, int n_steps,
                   int precision, void* stream);

/* out[M,N] = epi(A[M,K] @ B[K,N]) where one MXB_EP_ADD_PRODUCT step adds a
 * second product A2[M,K2] @ B2[K2,N] at its place in the chain.  No
 * counterpart in the reference: there optimize() leaves a bare OP_MATMUL
 * feeding a fused node's ADD step as a node of its own (optimizer.c:94-132)
 * and eval_fused adds its stored result (graph.c:98-105); gpu_execute uses
 * this fusion for such a matmul when the fused node is its only consumer and
 * both share the left operand.  With A2 == A (same pointer, pitch and
 * K2 == K, M > 16; in 3xTF32 mode also enough 256 x 128 tiles to fill a
 * quarter of the SMs) both products accumulate side by side in TMEM in one
 * kernel that stages A once, and the second never goes to HBM; otherwise the
 * second product runs first into pooled workspace.  Values are the same
 * either way.  A2 and B2
 * follow mxb_fused_gemm's layout rules (lda2, ldb2 % 4 == 0); exactly one
 * ADD_PRODUCT step. */
MXB_API int mxb_fused_gemm2(GpuCtx* ctx,
                   const float* A, long long lda,
                   const float* B, long long ldb,
                   const float* A2, long long lda2,
                   const float* B2, long long ldb2, int K2,
                   float* out, long long ldo,
                   int M, int N, int K,
                   const mxb_ep_step* steps, int n_steps,
                   int precision, void* stream);

/* The 3xTF32 fused GEMM for callers that cannot allocate device memory.  No
 * counterpart in the reference.  Some callers must not call cudaMalloc: a
 * plugin inside a framework that owns the whole device-memory budget through
 * its own allocator, or a latency-critical serving loop, where cudaMalloc /
 * cudaFree synchronise the device.  This entry point allocates nothing and
 * needs no GpuCtx: the low parts of A and B live in a fixed 16 MiB device
 * array inside the library (held by every GPU that loads it until exit), so
 * M*lda + K*ldb must not exceed 4 Mi floats (else MXB_E_ARG).  Same operands,
 * layout rules and epilogue steps as mxb_fused_gemm; runs on the current
 * device and on `stream` (NULL = the legacy default stream), and returns once
 * the work on that stream is finished.  The first call on a device looks up
 * the array's device address; make it before any stream capture.  As every
 * call synchronises its stream, a call on a stream that is being captured is
 * refused with MXB_E_ARG.  Device-side waits are bounded by
 * $MINIXLA_WAIT_TIMEOUT_MS (else 5 s).  Calls share the array, so calls that
 * overlap on the GPU race and must be serialised. */
MXB_API int mxb_fused_gemm_noalloc(const float* A, long long lda,
                                   const float* B, long long ldb,
                                   float* out, long long ldo,
                                   int M, int N, int K,
                                   const mxb_ep_step* steps, int n_steps,
                                   void* stream);

/* ---- Row-sharded GEMM with the all-gather in the epilogue ---------------
 * No counterpart in the reference (its GPU path is single-device).  With one
 * process per GPU, GPU g owns rows r0..r1 of out = epi(A @ B); a consumer
 * that needs the whole [M, N] tensor on every GPU would otherwise run an
 * NCCL all-gather after the kernel.  mxb_fused_gemm_allgather computes this
 * GPU's rows like mxb_fused_gemm into `out` (its rows of its own copy of the
 * full output) and writes the same rows into every peer GPU's copy:
 * peer_out[i] is where those rows start in peer i's copy (same ldo), a
 * device pointer opened with mxb_ipc_open.  On the CTA-pair kernels (either
 * mode; M >= 256 with enough tiles to occupy the GPU) the epilogue warps
 * store each finished tile to the peers over NVLink while the tensor cores
 * run the next tile; every other kernel is followed by one strided copy per
 * peer on the same stream.  Values are identical either way.  Peer rows are
 * complete once the kernel has finished on the writing GPU: before reading
 * rows that peers wrote, or writing a buffer a peer may still read,
 * synchronise the ranks on the stream (for example a one-element NCCL
 * all-reduce).  n_peers <= MXB_MAX_PEERS.  MINIXLA_GATHER_PUSH=0 forces the
 * copy form. */
#define MXB_MAX_PEERS 7
#define MXB_IPC_HANDLE_BYTES 64
MXB_API int mxb_fused_gemm_allgather(GpuCtx* ctx,
                   const float* A, long long lda,
                   const float* B, long long ldb,
                   float* out, long long ldo,
                   float* const* peer_out, int n_peers,
                   int M, int N, int K,
                   const mxb_ep_step* steps, int n_steps,
                   int precision, void* stream);

/* Device buffers shared between processes (CUDA IPC, no multicast object).
 * mxb_ipc_alloc allocates `bytes` on `device` and returns the pointer and a
 * handle that another process passes to mxb_ipc_open to map the same memory
 * (peer access over NVLink).  Every process that opened a handle closes it
 * (mxb_ipc_close) before the owner frees it (mxb_ipc_free). */
MXB_API int mxb_ipc_alloc(int device, size_t bytes, void** dptr, unsigned char* handle);
MXB_API int mxb_ipc_open(int device, const unsigned char* handle, void** dptr);
MXB_API int mxb_ipc_close(int device, void* dptr);
MXB_API int mxb_ipc_free(int device, void* dptr);

/* Launches of mxb_fused_gemm_allgather whose kernel wrote the peer rows
 * itself (the rest used copies), in this process. */
MXB_API unsigned long long mxb_gather_push_count(void);

/* ---- Which kernel runs a product ---------------------------------------
 * No counterpart in the reference (its GPU path has one kernel per mode).
 * mxb_gemm_plan_for reports what mxb_fused_gemm / gpu_execute run for an
 * M x N x K product (M: the node's full row count) in `precision` on a GPU
 * with `num_sms` SMs, under the current MINIXLA_* settings: the kernel family,
 * its output tile and how many ways K is split across CTAs.  Host-only: it
 * touches no GPU.  0 or MXB_E_ARG. */
enum {
    MXB_KERNEL_SKINNY = 1,     /* CUDA-core fp32 over column blocks x K slices (few rows)     */
    MXB_KERNEL_TINY = 2,       /* CUDA-core fp32, 32 x 32 tiles, one launch (tiny problems)    */
    MXB_KERNEL_SINGLE_CTA = 3, /* tcgen05, one CTA per 128-row tile                           */
    MXB_KERNEL_CTA_PAIR = 4    /* tcgen05 cta_group::2, 256-row tiles on two SMs              */
};
typedef struct {
    int kernel;                /* MXB_KERNEL_*                                                */
    int tile_rows, tile_cols;  /* output tile of one CTA (pair: of the two CTAs)              */
    int k_splits;              /* CTAs sharing one tile's K range (1: none)                   */
    int products;              /* products per launch: 1, or the batch when a rank-3 node's  */
                               /* products all run in one launch                             */
    int streamk_tiles;         /* CTA pair (TF32): tiles whose k-blocks are shared out evenly */
                               /* over the pairs because they do not fill the last waves     */
                               /* (0: every tile runs whole on one pair)                     */
    int reserved[2];
} mxb_gemm_plan;
MXB_API int mxb_gemm_plan_for(int M, int N, int K, int precision, int num_sms, mxb_gemm_plan* plan);
/* The same for a rank-3 node of `batch` products of M x N x K (eval_fused's
 * batch loop, graph.c:80-113): products = batch when they all run in one
 * launch, else the single-product plan (one launch per product). */
MXB_API int mxb_gemm_plan_batch_for(long long batch, int M, int N, int K, int precision, int num_sms,
                                    mxb_gemm_plan* plan);

/* Standalone element-wise nodes (tensor.c:64-86 and 110-120 semantics):
 * out[i] = a[i] + b[i % b_size]  and  out[i] = x[i] > 0 ? x[i] : 0. */
MXB_API int mxb_add(GpuCtx* ctx, const float* a, long long n, const float* b, long long b_size,
            float* out, void* stream);
MXB_API int mxb_relu(GpuCtx* ctx, const float* x, long long n, float* out, void* stream);

/* Synchronises the context's device work and reports a device-side error
 * recorded by a kernel (MXB_E_TIMEOUT after a bounded wait ran out), then
 * clears it.  0 when clean. */
MXB_API int mxb_check_device_error(GpuCtx* ctx);

/* Test hook for the failure path: launches a kernel that waits, with a limit
 * of `timeout_ns`, on a barrier that nothing completes; the kernel records
 * MXB_E_TIMEOUT and returns, leaving the context usable.  Returns the status
 * the host read back (MXB_E_TIMEOUT expected). */
MXB_API int mxb_selftest_wait_timeout(GpuCtx* ctx, unsigned long long timeout_ns);

/* Number of kernels this library has launched in this process (all
 * contexts); used by benchmarks to report launches in a timed region. */
MXB_API unsigned long long mxb_launch_count(void);

/* Short description of the last failure on this thread ("" if none). */
MXB_API const char* mxb_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* MINIXLA_B200_H */
