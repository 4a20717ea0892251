// Host runtime behind the C ABI: errors and counters, GpuCtx create / destroy,
// resident operands, the single-node entry points and the kernel-only
// timers, and every extern "C" function.  The device pool and GpuCtx are in
// runtime_internal.h; graph analysis in graph_plan.cu; GEMM dispatch in
// gemm_launch.cu; the executors in exec_graph.cu (one stream + side
// streams), exec_streamed.cu (row chunks) and exec_sharded.cu (multi-GPU).
//
// Replaces gpu_exec.c / runtime.c of gouthamk16/miniXLA:
//  - gpu_exec.c:57-93   GpuCtx create/destroy  -> gpu_ctx_create_on /
//                       gpu_ctx_destroy (runtime API, non-blocking streams,
//                       device pool, error word)
//  - gpu_exec.c:34-53   PTX-string module cache -> none needed: kernels are
//                       compiled sm_100a code, chosen by node signature
//  - gpu_exec.c:419-551 gpu_execute -> execute_graph() (exec_graph.cu):
//                       topological order, last-use release into the pool
//                       (not cuMemFree), all work stream-ordered, one
//                       synchronise before download
//  - gpu_exec.c:327-410, 251-323 kernel-only timers -> time_fused()
//  - runtime.c:16-128   gpu_run_fused -> run_single()
#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <mutex>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "internal.h"
#include "runtime_internal.h"

// ---------------------------------------------------------------- ABI checks
// The library reads caller-built Tensor / Node / EpStep structs in place, so
// their layout must be the reference's (tensor.h:6-12, graph.h:17-31) on LP64.
static_assert(sizeof(Tensor) == 40, "Tensor layout");
static_assert(offsetof(Tensor, data) == 0 && offsetof(Tensor, shape) == 8 &&
                  offsetof(Tensor, strides) == 16 && offsetof(Tensor, ndim) == 24 &&
                  offsetof(Tensor, size) == 32,
              "Tensor field offsets");
static_assert(sizeof(EpStep) == 16 && offsetof(EpStep, operand) == 8, "EpStep layout");
static_assert(sizeof(Node) == 64, "Node layout");
static_assert(offsetof(Node, inputs) == 8 && offsetof(Node, n_inputs) == 16 &&
                  offsetof(Node, output) == 24 && offsetof(Node, owns_output) == 32 &&
                  offsetof(Node, visited) == 36 && offsetof(Node, uses) == 40 &&
                  offsetof(Node, is_const) == 44 && offsetof(Node, epilogue) == 48 &&
                  offsetof(Node, n_epilogue) == 56,
              "Node field offsets");

namespace mxb {

// ---------------------------------------------------------------- errors, counters

static std::atomic<unsigned long long> g_launches{0};
static std::atomic<unsigned long long> g_gather_pushes{0};  // all-gathers written by the kernel itself
static thread_local std::string t_last_error;

void note_launch(unsigned n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

void set_error(const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
    fprintf(stderr, "minixla_b200: %s\n", buf);
}


}  // namespace mxb

using mxb::cuda_ok;
using mxb::set_error;

namespace mxb {

// ---------------------------------------------------------------- single-node paths

// Device copies of one fused node's operands, taken from the host tensors
// hanging off its inputs (runtime.c:17-84 and gpu_exec.c:339-362 do the same).
struct SingleNode {
    int M = 0, N = 0, K = 0;
    long long batch = 1;  // rank-3 and higher nodes (kernel timers only): products stored back to back
    float *dA = nullptr, *dB = nullptr, *dOut = nullptr;
    std::vector<float*> ops;
    std::unordered_map<const Node*, const float*> dev_of;
    std::unordered_map<const Node*, long long> size_of;

    void release(GpuCtx* ctx) {
        ctx->pool->release(dA, ctx->stream);
        ctx->pool->release(dB, ctx->stream);
        ctx->pool->release(dOut, ctx->stream);
        for (float* p : ops) ctx->pool->release(p, ctx->stream);
        dA = dB = dOut = nullptr;
        ops.clear();
    }
};

static float* upload(GpuCtx* ctx, const Tensor* t) {
    float* d = static_cast<float*>(ctx->pool->alloc(t->size * 4, ctx->stream));
    if (!d) return nullptr;
    if (!cuda_ok(copy_h2d(ctx->stager, d, t->data, t->size * 4, ctx->stream), "upload")) {
        ctx->pool->release(d, ctx->stream);
        return nullptr;
    }
    return d;
}

static int prepare_single(const Node* fused, GpuCtx* ctx, const char* who, SingleNode& s,
                          bool allow_batch = false) {
    if (!fused || !ctx) {
        set_error("%s: NULL node or context", who);
        return MXB_E_ARG;
    }
    if (fused->op != OP_FUSED && fused->op != OP_MATMUL) {
        set_error("%s: node is not OP_FUSED", who);
        return MXB_E_ARG;
    }
    const Tensor* a = fused->n_inputs >= 2 && fused->inputs[0] ? fused->inputs[0]->output : nullptr;
    const Tensor* b = fused->n_inputs >= 2 && fused->inputs[1] ? fused->inputs[1]->output : nullptr;
    if (!a || !b) {
        set_error("%s: matmul operands need host tensors", who);
        return MXB_E_ARG;
    }
    if (a->ndim != b->ndim || a->ndim < 2 || (a->ndim > 2 && !allow_batch)) {
        set_error("%s: only 2D tensors supported", who);
        return MXB_E_UNSUPPORTED;
    }
    const int r = a->ndim;
    if (a->shape[r - 1] != b->shape[r - 2]) {
        set_error("%s: incompatible matmul operand shapes", who);
        return MXB_E_ARG;
    }
    for (int d = 0; d < r - 2; ++d) {
        if (a->shape[d] != b->shape[d]) {  // eval_fused's rule (graph.c:71-76)
            set_error("%s: matmul batch dimension %d mismatch", who, d);
            return MXB_E_ARG;
        }
    }
    if (fused->op == OP_FUSED && fused->n_epilogue > MXB_MAX_EPILOGUE) {
        set_error("%s: too many epilogue steps", who);
        return MXB_E_UNSUPPORTED;
    }
    s.M = a->shape[r - 2];
    s.K = a->shape[r - 1];
    s.N = b->shape[r - 1];
    s.batch = static_cast<long long>(a->size) / (static_cast<long long>(s.M) * s.K);
    if (!(s.dA = upload(ctx, a)) || !(s.dB = upload(ctx, b))) return MXB_E_NOMEM;
    if (fused->op == OP_FUSED) {
        for (int e = 0; e < fused->n_epilogue; ++e) {
            const EpStep& st = fused->epilogue[e];
            if (st.op != OP_ADD) continue;
            const Tensor* t = st.operand ? st.operand->output : nullptr;
            if (!t || !t->data) {
                set_error("%s: ADD epilogue operand needs a host tensor", who);
                return MXB_E_ARG;
            }
            if (s.dev_of.count(st.operand)) continue;
            float* d = upload(ctx, t);
            if (!d) return MXB_E_NOMEM;
            s.ops.push_back(d);
            s.dev_of[st.operand] = d;
            s.size_of[st.operand] = static_cast<long long>(t->size);
        }
    }
    s.dOut = static_cast<float*>(ctx->pool->alloc(static_cast<size_t>(s.batch * s.M) * s.N * 4, ctx->stream));
    return s.dOut ? MXB_OK : MXB_E_NOMEM;
}

static Tensor* run_single(const Node* fused, GpuCtx* ctx, int precision, const char* who) {
    DeviceScope scope(ctx ? ctx->device : 0);
    SingleNode s;
    Tensor* result = nullptr;
    int rc = prepare_single(fused, ctx, who, s);
    if (rc == MXB_OK)
        rc = run_gemm_node(ctx, fused, s.dA, s.M, s.K, s.dB, s.N, s.dOut, s.dev_of, s.size_of, precision,
                           ctx->stream);
    if (rc == MXB_OK) rc = finish(ctx);
    if (rc == MXB_OK) {
        result = new_host_tensor({s.M, s.N});
        if (!result ||
            !cuda_ok(copy_d2h(ctx->stager, result->data, s.dOut, static_cast<size_t>(s.M) * s.N * 4, ctx->stream),
                     "result download") ||
            !cuda_ok(cudaStreamSynchronize(ctx->stream), "download synchronize")) {
            if (result) {
                free(result->data);
                free(result->shape);
                free(result->strides);
                free(result);
            }
            result = nullptr;
        }
    }
    if (ctx) {
        s.release(ctx);
        cudaStreamSynchronize(ctx->stream);
    }
    return result;
}

// Kernel-only timing (gpu_exec.c:327-410): operands uploaded once, `warmup`
// untimed launches each followed by a synchronise, then the minimum over
// `reps` CUDA-event-timed launches on the context stream.  In 3xTF32 mode a
// launch includes the operand split, which is part of that mode's work.
static double time_fused(Node* root, GpuCtx* ctx, int warmup, int reps, int precision, const char* who) {
    if (!root || !ctx || root->op != OP_FUSED) return -1.0;
    if (root->n_inputs < 2 || !root->inputs[0]->output || !root->inputs[1]->output) return -1.0;
    if (reps < 1) return -1.0;
    DeviceScope scope(ctx->device);
    SingleNode s;
    double best = -1.0;
    int rc = prepare_single(root, ctx, who, s, /*allow_batch=*/true);
    if (rc == MXB_OK) {
        for (int w = 0; w < warmup && rc == MXB_OK; ++w) {
            rc = run_gemm_node(ctx, root, s.dA, s.M, s.K, s.dB, s.N, s.dOut, s.dev_of, s.size_of, precision,
                               ctx->stream, s.batch);
            if (rc == MXB_OK) rc = finish(ctx);
        }
        double lo = 1e30;
        for (int r = 0; r < reps && rc == MXB_OK; ++r) {
            // The stream is held busy while the launch is prepared and queued,
            // so the events bracket the kernels alone (gpu_exec.c:380-398 times
            // its kernel launch between two events the same way).
            if (!cuda_ok(launch_hold(50000, ctx->stream), "timer hold launch")) {
                rc = MXB_E_CUDA;
                break;
            }
            cudaEventRecord(ctx->ev0, ctx->stream);
            rc = run_gemm_node(ctx, root, s.dA, s.M, s.K, s.dB, s.N, s.dOut, s.dev_of, s.size_of, precision,
                               ctx->stream, s.batch);
            cudaEventRecord(ctx->ev1, ctx->stream);
            if (rc == MXB_OK && cuda_ok(cudaEventSynchronize(ctx->ev1), "event synchronize")) {
                float ms = 0.f;
                cudaEventElapsedTime(&ms, ctx->ev0, ctx->ev1);
                lo = std::min(lo, static_cast<double>(ms));
            } else if (rc == MXB_OK) {
                rc = MXB_E_CUDA;
            }
        }
        if (rc == MXB_OK) rc = finish(ctx);
        if (rc == MXB_OK) best = lo;
    }
    s.release(ctx);
    cudaStreamSynchronize(ctx->stream);
    return best;
}

static int precision_from_env() {
    const char* p = getenv("MINIXLA_PRECISION");
    if (!p) return GPU_PRECISION_3XTF32;
    if (!strcmp(p, "tf32") || !strcmp(p, "TF32")) return GPU_PRECISION_TF32;
    return GPU_PRECISION_3XTF32;
}

static bool valid_precision(int p) { return p == GPU_PRECISION_TF32 || p == GPU_PRECISION_3XTF32; }

}  // namespace mxb

// ================================================================== C ABI

extern "C" {

GpuCtx* gpu_ctx_create_on(int device) {
    int count = 0;
    if (!cuda_ok(cudaGetDeviceCount(&count), "cudaGetDeviceCount")) return nullptr;
    if (device < 0 || device >= count) {
        set_error("gpu_ctx_create: device %d out of range (%d devices)", device, count);
        return nullptr;
    }
    mxb::DeviceScope scope(device);
    cudaDeviceProp prop;
    if (!cuda_ok(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties")) return nullptr;
    if (prop.major != 10) {
        set_error("gpu_ctx_create: device %d is sm_%d%d; this library carries sm_100a code only", device,
                  prop.major, prop.minor);
        return nullptr;
    }
    GpuCtx* g = new (std::nothrow) GpuCtx();
    if (!g) return nullptr;
    g->device = device;
    g->num_sms = prop.multiProcessorCount;
    g->precision = mxb::precision_from_env();
    if (const char* t = getenv("MINIXLA_WAIT_TIMEOUT_MS")) {
        const long long ms = atoll(t);
        if (ms > 0) g->timeout_ns = static_cast<unsigned long long>(ms) * 1000000ull;
    }
    bool ok = cuda_ok(cudaFree(nullptr), "context init") &&
              cuda_ok(cudaStreamCreateWithFlags(&g->stream, cudaStreamNonBlocking), "stream create") &&
              cuda_ok(cudaStreamCreateWithFlags(&g->h2d, cudaStreamNonBlocking), "stream create") &&
              cuda_ok(cudaStreamCreateWithFlags(&g->d2h, cudaStreamNonBlocking), "stream create") &&
              cuda_ok(cudaMalloc(&g->d_err, sizeof(int)), "error word alloc") &&
              cuda_ok(cudaMemset(g->d_err, 0, sizeof(int)), "error word clear") &&
              cuda_ok(cudaEventCreate(&g->ev0), "event create") && cuda_ok(cudaEventCreate(&g->ev1), "event create");
    if (ok) g->pool = new (std::nothrow) mxb::DevicePool(device);
    if (ok) g->stager = mxb::stager_create();  // its pinned slots are made on first use
    if (ok) g->stager_dl = mxb::stager_create();
    if (!ok || !g->pool || !g->stager || !g->stager_dl) {
        gpu_ctx_destroy(g);
        return nullptr;
    }
    return g;
}

GpuCtx* gpu_ctx_create_multi(int ngpu) {
    int count = 0;
    if (!cuda_ok(cudaGetDeviceCount(&count), "cudaGetDeviceCount")) return nullptr;
    if (ngpu < 1 || ngpu > count) {
        set_error("gpu_ctx_create_multi: %d GPUs requested, %d present", ngpu, count);
        return nullptr;
    }
    GpuCtx* g = gpu_ctx_create_on(0);
    if (!g) return nullptr;
    for (int d = 1; d < ngpu; ++d) {
        GpuCtx* p = gpu_ctx_create_on(d);
        if (!p) {
            gpu_ctx_destroy(g);
            return nullptr;
        }
        g->peers.push_back(p);
    }
    // Peer access lets replication copies run device to device over NVLink.
    for (int a = 0; a < ngpu; ++a) {
        mxb::DeviceScope scope(a);
        for (int b = 0; b < ngpu; ++b) {
            int can = 0;
            if (a == b || cudaDeviceCanAccessPeer(&can, a, b) != cudaSuccess || !can) continue;
            const cudaError_t e = cudaDeviceEnablePeerAccess(b, 0);
            if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) {
                set_error("gpu_ctx_create_multi: peer access %d -> %d: %s", a, b, cudaGetErrorString(e));
            }
            cudaGetLastError();
        }
    }
    return g;
}

GpuCtx* gpu_ctx_create(void) {
    if (const char* n = getenv("MINIXLA_NGPU")) {
        const int ngpu = atoi(n);
        if (ngpu > 1) return gpu_ctx_create_multi(ngpu);
    }
    int dev = 0;
    if (const char* d = getenv("MINIXLA_DEVICE")) dev = atoi(d);
    return gpu_ctx_create_on(dev);
}

int gpu_ctx_ngpu(const GpuCtx* ctx) { return ctx ? 1 + static_cast<int>(ctx->peers.size()) : 0; }

static void free_resident(GpuCtx* ctx, GpuCtx::Resident& r) {
    for (size_t d = 0; d < r.dev.size(); ++d) {
        GpuCtx* c = d == 0 ? ctx : ctx->peers[d - 1];
        mxb::DeviceScope scope(c->device);
        cudaStreamSynchronize(c->stream);
        if (r.dev[d]) cudaFree(r.dev[d]);
    }
    r.dev.clear();
}

int gpu_ctx_keep_resident(GpuCtx* ctx, const Tensor* t) {
    if (!ctx || !t || !t->data || t->size == 0) {
        set_error("gpu_ctx_keep_resident: NULL context or empty tensor");
        return MXB_E_ARG;
    }
    gpu_ctx_release_resident(ctx, t);
    GpuCtx::Resident r{t->data, t->size, {}};
    const size_t bytes = t->size * sizeof(float);
    const size_t ndev = 1 + ctx->peers.size();
    for (size_t d = 0; d < ndev; ++d) {
        GpuCtx* c = d == 0 ? ctx : ctx->peers[d - 1];
        mxb::DeviceScope scope(c->device);
        float* p = nullptr;
        if (cudaMalloc(&p, bytes) != cudaSuccess) {
            cudaGetLastError();
            c->pool->trim();
            if (cudaMalloc(&p, bytes) != cudaSuccess) {
                cudaGetLastError();
                set_error("gpu_ctx_keep_resident: device allocation of %zu bytes failed", bytes);
                free_resident(ctx, r);
                return MXB_E_NOMEM;
            }
        }
        r.dev.push_back(p);
        if (!cuda_ok(mxb::copy_h2d(c->stager, p, t->data, bytes, c->stream), "resident upload") ||
            !cuda_ok(cudaStreamSynchronize(c->stream), "resident upload synchronize")) {
            free_resident(ctx, r);
            return MXB_E_CUDA;
        }
    }
    ctx->resident[t] = std::move(r);
    return MXB_OK;
}

int gpu_ctx_release_resident(GpuCtx* ctx, const Tensor* t) {
    if (!ctx) return MXB_E_ARG;
    if (!t) {
        for (auto& kv : ctx->resident) free_resident(ctx, kv.second);
        ctx->resident.clear();
        return MXB_OK;
    }
    auto it = ctx->resident.find(t);
    if (it == ctx->resident.end()) return MXB_OK;
    free_resident(ctx, it->second);
    ctx->resident.erase(it);
    return MXB_OK;
}

int mxb_shard_rows(long long M, int parts, int part, long long* r0, long long* r1) {
    if (M < 0 || parts < 1 || part < 0 || part >= parts || !r0 || !r1) return MXB_E_ARG;
    mxb::shard_range(M, parts, part, *r0, *r1);
    return MXB_OK;
}

void gpu_ctx_destroy(GpuCtx* g) {
    if (!g) return;
    gpu_ctx_release_resident(g, nullptr);
    if (!g->comms.empty() && mxb::nccl().ok) {
        for (ncclComm_t c : g->comms)
            if (c) mxb::nccl().comm_destroy(c);
    }
    for (GpuCtx* p : g->peers) gpu_ctx_destroy(p);
    {
        mxb::DeviceScope scope(g->device);
        if (g->stream) cudaStreamSynchronize(g->stream);
        mxb::stager_destroy(g->stager);
        mxb::stager_destroy(g->stager_dl);
        delete g->pool;
        if (g->d_err) cudaFree(g->d_err);
        if (g->ev0) cudaEventDestroy(g->ev0);
        if (g->ev1) cudaEventDestroy(g->ev1);
        for (cudaEvent_t e : g->sync_events) cudaEventDestroy(e);
        for (cudaStream_t st : g->side) cudaStreamDestroy(st);
        if (g->h2d) cudaStreamDestroy(g->h2d);
        if (g->d2h) cudaStreamDestroy(g->d2h);
        if (g->stream) cudaStreamDestroy(g->stream);
    }
    delete g;
}

int gpu_ctx_set_precision(GpuCtx* ctx, int mode) {
    if (!ctx || !mxb::valid_precision(mode)) {
        set_error("gpu_ctx_set_precision: unknown mode %d", mode);
        return -1;
    }
    ctx->precision = mode;
    return 0;
}

int gpu_ctx_get_precision(const GpuCtx* ctx) { return ctx ? ctx->precision : -1; }

int gpu_ctx_device(const GpuCtx* ctx) { return ctx ? ctx->device : -1; }

Tensor* gpu_execute(Node* root, GpuCtx* ctx) {
    Tensor* out = nullptr;
    return mxb::execute_graph(root, ctx, nullptr, &out) == MXB_OK ? out : nullptr;
}

int gpu_execute_into(Node* root, GpuCtx* ctx, Tensor* out) {
    if (!out) {
        set_error("gpu_execute_into: NULL destination");
        return MXB_E_ARG;
    }
    return mxb::execute_graph(root, ctx, out, nullptr);
}

double gpu_time_kernel_ms(Node* root, GpuCtx* ctx, int warmup, int reps) {
    return mxb::time_fused(root, ctx, warmup, reps, ctx ? ctx->precision : 0, "gpu_time_kernel_ms");
}

double gpu_time_kernel_tc_ms(Node* root, GpuCtx* ctx, int warmup, int reps) {
    return mxb::time_fused(root, ctx, warmup, reps, GPU_PRECISION_TF32, "gpu_time_kernel_tc_ms");
}

Tensor* gpu_run_tensorcore(const Node* fused, GpuCtx* ctx) {
    if (!ctx) {
        set_error("gpu_run_tensorcore: NULL context");
        return nullptr;
    }
    return mxb::run_single(fused, ctx, GPU_PRECISION_TF32, "gpu_run_tensorcore");
}

Tensor* gpu_run_fused(const Node* fused, const char* ptx) {
    (void)ptx;  // kernels are compiled sm_100a code chosen from the node itself
    GpuCtx* ctx = gpu_ctx_create();
    if (!ctx) return nullptr;
    Tensor* r = mxb::run_single(fused, ctx, ctx->precision, "gpu_run_fused");
    gpu_ctx_destroy(ctx);
    return r;
}

// Argument checks shared by mxb_fused_gemm and mxb_fused_gemm_allgather, then
// the launch (with peer rows when `peers` is given).
static int fused_gemm_checked(const char* fn, GpuCtx* ctx, const float* A, long long lda, const float* B,
                              long long ldb, float* out, long long ldo, int M, int N, int K, const mxb_ep_step* steps,
                              int n_steps, int precision, void* stream, mxb::PeerRows* peers) {
    if (!ctx || !A || !B || !out || M < 1 || N < 1 || K < 1 || lda < K || ldb < N || ldo < N ||
        n_steps < 0 || n_steps > MXB_MAX_EPILOGUE || (n_steps > 0 && !steps) || !mxb::valid_precision(precision)) {
        set_error("%s: invalid arguments", fn);
        return MXB_E_ARG;
    }
    if (lda % 4 || ldb % 4 || (reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15)) {
        set_error("%s: A and B need 16-byte aligned bases and row pitches (lda %% 4 == 0, ldb %% 4 == 0)", fn);
        return MXB_E_ARG;
    }
    mxb::EpStepDev dev_steps[MXB_MAX_EPILOGUE];
    for (int i = 0; i < n_steps; ++i) {
        const mxb_ep_step& s = steps[i];
        const bool is_add = s.kind == MXB_EP_ADD_FULL || s.kind == MXB_EP_ADD_ROW || s.kind == MXB_EP_ADD_MOD;
        if (s.kind < MXB_EP_ADD_FULL || s.kind > MXB_EP_SCALE || (is_add && !s.operand) ||
            (s.kind == MXB_EP_ADD_FULL && s.ld_or_size < N) || (s.kind == MXB_EP_ADD_MOD && s.ld_or_size < 1)) {
            set_error("%s: invalid epilogue step %d", fn, i);
            return MXB_E_ARG;
        }
        memcpy(&dev_steps[i], &s, sizeof(s));
    }
    mxb::DeviceScope scope(ctx->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    return mxb::launch_gemm(ctx, A, lda, B, ldb, out, ldo, M, N, K, dev_steps, n_steps, precision, st, nullptr, 0,
                            nullptr, 0, peers);
}

int mxb_fused_gemm(GpuCtx* ctx, const float* A, long long lda, const float* B, long long ldb, float* out,
                   long long ldo, int M, int N, int K, const mxb_ep_step* steps, int n_steps, int precision,
                   void* stream) {
    return fused_gemm_checked("mxb_fused_gemm", ctx, A, lda, B, ldb, out, ldo, M, N, K, steps, n_steps, precision,
                              stream, nullptr);
}

int mxb_gemm_plan_batch_for(long long batch, int M, int N, int K, int precision, int num_sms, mxb_gemm_plan* plan) {
    if (!plan || batch < 1 || M < 1 || N < 1 || K < 1 || num_sms < 2 || !mxb::valid_precision(precision)) {
        set_error("mxb_gemm_plan_batch_for: invalid arguments");
        return MXB_E_ARG;
    }
    if (!mxb::batched_in_one_launch(num_sms, batch, M, N, K, precision)) return mxb_gemm_plan_for(M, N, K, precision, num_sms, plan);
    memset(plan, 0, sizeof(*plan));
    mxb::GemmLaunch g{};
    g.M = M;
    g.N = N;
    g.K = K;
    g.precision = precision;
    g.num_sms = num_sms;
    g.choice_rows = M;
    g.batch = batch;
    const mxb::GemmPlan pl = mxb::plan_fused_gemm(g, 1);
    plan->kernel = pl.kernel;
    plan->tile_rows = pl.tile_rows;
    plan->tile_cols = pl.tile_cols;
    plan->k_splits = 1;
    plan->products = static_cast<int>(std::min<long long>(batch, 1ll << 30));
    return MXB_OK;
}

int mxb_gemm_plan_for(int M, int N, int K, int precision, int num_sms, mxb_gemm_plan* plan) {
    if (!plan || M < 1 || N < 1 || K < 1 || num_sms < 2 || !mxb::valid_precision(precision)) {
        set_error("mxb_gemm_plan_for: invalid arguments");
        return MXB_E_ARG;
    }
    memset(plan, 0, sizeof(*plan));
    plan->products = 1;
    plan->k_splits = 1;
    // The same order as launch_gemm: skinny, tiny, then the tensor-core plan.
    if (mxb::use_skinny_gemm(M, precision)) {
        const mxb::SkinnyPlan sp = mxb::plan_skinny(M, N, K, num_sms);
        plan->kernel = MXB_KERNEL_SKINNY;
        plan->tile_rows = M;
        plan->tile_cols = sp.one_kernel ? 128 : (N + sp.col_blocks - 1) / sp.col_blocks;
        plan->k_splits = sp.one_kernel ? 8 : sp.splits;
        return MXB_OK;
    }
    if (mxb::use_tiny_gemm(M, N, K, precision)) {
        plan->kernel = MXB_KERNEL_TINY;
        plan->tile_rows = plan->tile_cols = 32;
        return MXB_OK;
    }
    mxb::GemmLaunch g{};
    g.M = M;
    g.N = N;
    g.K = K;
    g.precision = precision;
    g.num_sms = num_sms;
    g.choice_rows = M;
    const mxb::GemmPlan pl = mxb::plan_fused_gemm(g, mxb::fused_gemm_k_splits(g));
    plan->kernel = pl.kernel;
    plan->tile_rows = pl.tile_rows;
    plan->tile_cols = pl.tile_cols;
    plan->k_splits = pl.k_splits;
    plan->streamk_tiles = mxb::fused_gemm_streamk_tiles(g);
    return MXB_OK;
}

int mxb_fused_gemm_allgather(GpuCtx* ctx, const float* A, long long lda, const float* B, long long ldb, float* out,
                             long long ldo, float* const* peer_out, int n_peers, int M, int N, int K,
                             const mxb_ep_step* steps, int n_steps, int precision, void* stream) {
    if (n_peers < 0 || n_peers > MXB_MAX_PEERS || (n_peers > 0 && !peer_out)) {
        set_error("mxb_fused_gemm_allgather: n_peers must be 0..%d with a pointer per peer", MXB_MAX_PEERS);
        return MXB_E_ARG;
    }
    for (int i = 0; i < n_peers; ++i) {
        if (!peer_out[i] || peer_out[i] == out) {
            set_error("mxb_fused_gemm_allgather: peer_out[%d] is null or the local output", i);
            return MXB_E_ARG;
        }
    }
    mxb::PeerRows peers;
    peers.out = peer_out;
    peers.n = n_peers;
    int rc = fused_gemm_checked("mxb_fused_gemm_allgather", ctx, A, lda, B, ldb, out, ldo, M, N, K, steps, n_steps,
                                precision, stream, &peers);
    if (rc != MXB_OK || n_peers == 0) return rc;
    if (peers.pushed) {
        mxb::g_gather_pushes.fetch_add(1, std::memory_order_relaxed);
        return MXB_OK;
    }
    // The kernel wrote only local rows: one strided copy per peer (copy
    // engines over NVLink), ordered after it on the same stream.
    mxb::DeviceScope scope(ctx->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    for (int i = 0; i < n_peers; ++i) {
        if (!mxb::cuda_ok(cudaMemcpy2DAsync(peer_out[i], ldo * 4, out, ldo * 4, static_cast<size_t>(N) * 4, M,
                                            cudaMemcpyDeviceToDevice, st),
                          "peer row copy"))
            return MXB_E_CUDA;
    }
    return MXB_OK;
}

int mxb_fused_gemm2(GpuCtx* ctx, const float* A, long long lda, const float* B, long long ldb, const float* A2,
                    long long lda2, const float* B2, long long ldb2, int K2, float* out, long long ldo, int M, int N,
                    int K, const mxb_ep_step* steps, int n_steps, int precision, void* stream) {
    if (!ctx || !A || !B || !A2 || !B2 || !out || M < 1 || N < 1 || K < 1 || K2 < 1 || lda < K || ldb < N ||
        lda2 < K2 || ldb2 < N || ldo < N || n_steps < 1 || n_steps > MXB_MAX_EPILOGUE || !steps ||
        !mxb::valid_precision(precision)) {
        set_error("mxb_fused_gemm2: invalid arguments");
        return MXB_E_ARG;
    }
    if (lda % 4 || ldb % 4 || lda2 % 4 || ldb2 % 4 || (reinterpret_cast<uintptr_t>(A) & 15) ||
        (reinterpret_cast<uintptr_t>(B) & 15) || (reinterpret_cast<uintptr_t>(A2) & 15) ||
        (reinterpret_cast<uintptr_t>(B2) & 15)) {
        set_error("mxb_fused_gemm2: A, B, A2 and B2 need 16-byte aligned bases and row pitches (multiples of 4)");
        return MXB_E_ARG;
    }
    mxb::EpStepDev dev_steps[MXB_MAX_EPILOGUE];
    int n_prod = 0;
    for (int i = 0; i < n_steps; ++i) {
        const mxb_ep_step& s = steps[i];
        const bool is_add = s.kind == MXB_EP_ADD_FULL || s.kind == MXB_EP_ADD_ROW || s.kind == MXB_EP_ADD_MOD;
        if (s.kind < MXB_EP_ADD_FULL || s.kind > MXB_EP_ADD_PRODUCT || (is_add && !s.operand) ||
            (s.kind == MXB_EP_ADD_FULL && s.ld_or_size < N) || (s.kind == MXB_EP_ADD_MOD && s.ld_or_size < 1)) {
            set_error("mxb_fused_gemm2: invalid epilogue step %d", i);
            return MXB_E_ARG;
        }
        n_prod += s.kind == MXB_EP_ADD_PRODUCT;
        memcpy(&dev_steps[i], &s, sizeof(s));
    }
    if (n_prod != 1) {
        set_error("mxb_fused_gemm2: exactly one MXB_EP_ADD_PRODUCT step required (got %d)", n_prod);
        return MXB_E_ARG;
    }
    mxb::DeviceScope scope(ctx->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    const mxb::Product prod{A2, lda2, B2, ldb2, K2};
    return mxb::launch_gemm(ctx, A, lda, B, ldb, out, ldo, M, N, K, dev_steps, n_steps, precision, st, nullptr, 0,
                            &prod);
}

int mxb_add(GpuCtx* ctx, const float* a, long long n, const float* b, long long b_size, float* out, void* stream) {
    if (!ctx || !a || !b || !out || n < 0 || b_size < 1) {
        set_error("mxb_add: invalid arguments");
        return MXB_E_ARG;
    }
    mxb::DeviceScope scope(ctx->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    return cuda_ok(mxb::launch_add(a, n, b, b_size, out, ctx->num_sms, st), "add launch") ? MXB_OK : MXB_E_CUDA;
}

int mxb_relu(GpuCtx* ctx, const float* x, long long n, float* out, void* stream) {
    if (!ctx || !x || !out || n < 0) {
        set_error("mxb_relu: invalid arguments");
        return MXB_E_ARG;
    }
    mxb::DeviceScope scope(ctx->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    return cuda_ok(mxb::launch_relu(x, n, out, ctx->num_sms, st), "relu launch") ? MXB_OK : MXB_E_CUDA;
}

int mxb_check_device_error(GpuCtx* ctx) {
    if (!ctx) return MXB_E_ARG;
    mxb::DeviceScope scope(ctx->device);
    if (!cuda_ok(cudaDeviceSynchronize(), "device synchronize")) return MXB_E_CUDA;
    return mxb::finish(ctx);
}

int mxb_selftest_wait_timeout(GpuCtx* ctx, unsigned long long timeout_ns) {
    if (!ctx) return MXB_E_ARG;
    mxb::DeviceScope scope(ctx->device);
    if (!cuda_ok(mxb::launch_wait_timeout_probe(ctx->d_err, timeout_ns, ctx->stream), "probe launch"))
        return MXB_E_CUDA;
    return mxb::finish(ctx);
}

unsigned long long mxb_launch_count(void) { return mxb::g_launches.load(); }

unsigned long long mxb_gather_push_count(void) { return mxb::g_gather_pushes.load(); }

const char* mxb_last_error(void) { return mxb::t_last_error.c_str(); }

}  // extern "C"
