// Host runtime behind the C ABI: GpuCtx, a caching device pool, the DAG
// executor (gpu_execute) and the kernel-only timers.
//
// Replaces gpu_exec.c / runtime.c of gouthamk16/miniXLA:
//  - gpu_exec.c:57-93   GpuCtx create/destroy  -> GpuCtx below (runtime API,
//                       one non-blocking stream, device pool, error word)
//  - gpu_exec.c:34-53   PTX-string module cache -> none needed: kernels are
//                       compiled sm_100a code, chosen by node signature
//  - gpu_exec.c:419-551 gpu_execute -> execute_graph(): topological order,
//                       last-use release into the pool (not cuMemFree), all
//                       work stream-ordered, one synchronise before download
//  - gpu_exec.c:327-410, 251-323 kernel-only timers -> time_fused()
//  - runtime.c:16-128   gpu_run_fused -> run_single()
#include <cuda_runtime.h>
#include <dlfcn.h>
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

static bool cuda_ok(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return true;
    set_error("%s: %s", what, cudaGetErrorString(e));
    return false;
}

// ---------------------------------------------------------------- device pool
//
// Size-class free lists.  A released block carries an event recorded on the
// stream that last used it; handing it to a different stream makes that
// stream wait on the event, so reuse is always stream-ordered.  A failed
// cudaMalloc first returns every cached block to the driver and retries.
// MINIXLA_FAIL_ALLOC_AT=n makes the n-th pool allocation of the process fail
// (host-side fault injection for the out-of-memory path).  A mutex guards the
// lists, so host threads may share a context's pool (the reference API
// itself is single-threaded; the device-pointer entry points need not be).

static std::atomic<long long> g_alloc_calls{0};

class DevicePool {
  public:
    explicit DevicePool(int device) : device_(device) {}
    ~DevicePool() {
        trim_locked();
        for (auto& kv : live_) cudaFree(kv.first);
        for (cudaEvent_t e : spare_events_) cudaEventDestroy(e);
    }

    void* alloc(size_t bytes, cudaStream_t stream) {
        std::lock_guard<std::mutex> lock(mu_);
        const long long call = g_alloc_calls.fetch_add(1) + 1;
        if (const char* fail = getenv("MINIXLA_FAIL_ALLOC_AT")) {
            if (atoll(fail) == call) {
                set_error("device allocation of %zu bytes failed (injected by MINIXLA_FAIL_ALLOC_AT)", bytes);
                return nullptr;
            }
        }
        const size_t cls = size_class(bytes);
        auto it = free_.find(cls);
        if (it != free_.end() && !it->second.empty()) {
            Cached c = it->second.back();
            it->second.pop_back();
            cached_bytes_ -= cls;
            if (c.stream != stream) cudaStreamWaitEvent(stream, c.ready, 0);
            spare_events_.push_back(c.ready);
            live_[c.ptr] = cls;
            return c.ptr;
        }
        void* p = nullptr;
        if (cudaMalloc(&p, cls) != cudaSuccess) {
            cudaGetLastError();
            trim_locked();
            if (cudaMalloc(&p, cls) != cudaSuccess) {
                cudaGetLastError();
                set_error("device allocation of %zu bytes failed", cls);
                return nullptr;
            }
        }
        live_[p] = cls;
        return p;
    }

    void release(void* p, cudaStream_t stream) {
        if (!p) return;
        std::lock_guard<std::mutex> lock(mu_);
        auto it = live_.find(p);
        if (it == live_.end()) return;
        const size_t cls = it->second;
        live_.erase(it);
        cudaEvent_t ev = take_event();
        if (ev) cudaEventRecord(ev, stream);
        free_[cls].push_back(Cached{p, stream, ev});
        cached_bytes_ += cls;
        if (!ev) {  // could not make an event: fall back to a full sync before reuse
            cudaStreamSynchronize(stream);
        }
    }

    void trim() {
        std::lock_guard<std::mutex> lock(mu_);
        trim_locked();
    }

    size_t live_bytes() {
        std::lock_guard<std::mutex> lock(mu_);
        size_t s = 0;
        for (auto& kv : live_) s += kv.second;
        return s;
    }
    size_t cached_bytes() {
        std::lock_guard<std::mutex> lock(mu_);
        return cached_bytes_;
    }

  private:
    void trim_locked() {
        for (auto& kv : free_) {
            for (Cached& c : kv.second) {
                if (c.ready) {
                    cudaEventSynchronize(c.ready);
                    spare_events_.push_back(c.ready);
                }
                cudaFree(c.ptr);
            }
            kv.second.clear();
        }
        cached_bytes_ = 0;
    }

    struct Cached {
        void* ptr;
        cudaStream_t stream;
        cudaEvent_t ready;
    };

    static size_t size_class(size_t bytes) {
        if (bytes == 0) bytes = 1;
        if (bytes <= (1u << 20)) return (bytes + 511) & ~static_cast<size_t>(511);
        const size_t mb2 = static_cast<size_t>(2) << 20;
        return (bytes + mb2 - 1) / mb2 * mb2;
    }

    cudaEvent_t take_event() {
        if (!spare_events_.empty()) {
            cudaEvent_t e = spare_events_.back();
            spare_events_.pop_back();
            return e;
        }
        cudaEvent_t e = nullptr;
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        return e;
    }

    int device_;
    std::mutex mu_;
    std::unordered_map<size_t, std::vector<Cached>> free_;
    std::unordered_map<void*, size_t> live_;
    std::vector<cudaEvent_t> spare_events_;
    size_t cached_bytes_ = 0;
};

// Keeps the caller's current device and restores it on scope exit.
struct DeviceScope {
    int prev = -1;
    explicit DeviceScope(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) {
            cudaGetLastError();
            prev = -1;
        }
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceScope() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

}  // namespace mxb

using mxb::cuda_ok;
using mxb::set_error;

struct GpuCtx {
    int device = 0;
    int num_sms = 148;
    int precision = GPU_PRECISION_3XTF32;
    unsigned long long timeout_ns = 5ull * 1000 * 1000 * 1000;
    cudaStream_t stream = nullptr;   // kernels
    cudaStream_t h2d = nullptr;      // host-to-device copies of the row-streamed executor
    cudaStream_t d2h = nullptr;      // device-to-host copies of the row-streamed executor
    std::vector<cudaStream_t> side;  // extra compute streams for independent DAG nodes (made on first use)
    int* d_err = nullptr;
    mxb::DevicePool* pool = nullptr;
    mxb::Stager* stager = nullptr;   // pinned slots for copies from / to pageable host memory
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    std::vector<cudaEvent_t> sync_events;  // reusable ordering events (no timing)
    std::vector<GpuCtx*> peers;            // devices 1..n-1 of a multi-GPU context
    std::vector<ncclComm_t> comms;         // one per device, made on the first all-gather
    struct Resident {
        const float* data;                 // host data pointer when kept
        size_t size;                       // element count when kept
        std::vector<float*> dev;           // one copy per device (this context, then its peers)
    };
    std::unordered_map<const Tensor*, Resident> resident;  // gpu_ctx_keep_resident
};

namespace mxb {

// ---------------------------------------------------------------- graph analysis

struct Info {
    const Node* node = nullptr;
    std::vector<int> dims;        // logical output shape
    long long size = 0;           // element count
    int last_use = -1;            // index of the last consumer in topo order
    float* dev = nullptr;         // device buffer (compact, row-major)
    bool borrowed = false;        // dev is a resident copy, not this call's to release
};

// Device copy of a resident leaf on device `d` of `ctx` (0 = ctx itself,
// then its peers), or nullptr when the tensor is not resident or its data
// pointer / size changed since it was kept.
static float* resident_copy(const GpuCtx* ctx, const Node* n, size_t d) {
    if (n->op != OP_INPUT || !n->output) return nullptr;
    auto it = ctx->resident.find(n->output);
    if (it == ctx->resident.end()) return nullptr;
    const GpuCtx::Resident& r = it->second;
    if (r.data != n->output->data || r.size != n->output->size || d >= r.dev.size()) return nullptr;
    return r.dev[d];
}

// Post-order DFS over inputs: every node after all of its inputs
// (graph.c:171-190 defines the same order; this copy does not touch the
// nodes' `visited` flags, so the caller's graph is never written).
static std::vector<const Node*> topo_order(const Node* root) {
    std::vector<const Node*> order;
    std::unordered_set<const Node*> seen;
    std::vector<std::pair<const Node*, int>> stack;
    stack.push_back({root, 0});
    seen.insert(root);
    while (!stack.empty()) {
        auto& top = stack.back();
        const Node* n = top.first;
        if (top.second < n->n_inputs) {
            const Node* in = n->inputs[top.second++];
            if (in && seen.insert(in).second) stack.push_back({in, 0});
        } else {
            order.push_back(n);
            stack.pop_back();
        }
    }
    return order;
}

static bool same_dims(const std::vector<int>& a, const std::vector<int>& b) { return a == b; }

// tensor_add's broadcast rule (tensor.c:57-63): b's shape is a trailing suffix of a's.
static bool trailing_suffix(const std::vector<int>& a, const std::vector<int>& b) {
    if (b.size() > a.size()) return false;
    for (size_t i = 0; i < b.size(); ++i)
        if (b[i] != a[a.size() - b.size() + i]) return false;
    return true;
}

static long long product(const std::vector<int>& d) {
    long long s = 1;
    for (int x : d) s *= x;
    return s;
}

// Fills dims/size for every node; false (with a message) for anything this
// backend cannot run.
static bool infer_shapes(const std::vector<const Node*>& order,
                         std::unordered_map<const Node*, int>& index, std::vector<Info>& info) {
    info.resize(order.size());
    for (size_t i = 0; i < order.size(); ++i) {
        const Node* n = order[i];
        index[n] = static_cast<int>(i);
        Info& f = info[i];
        f.node = n;
        switch (n->op) {
            case OP_INPUT: {
                const Tensor* t = n->output;
                if (!t || !t->data || t->ndim <= 0 || !t->shape) {
                    set_error("gpu_execute: OP_INPUT node without a host tensor");
                    return false;
                }
                f.dims.assign(t->shape, t->shape + t->ndim);
                f.size = static_cast<long long>(t->size);
                if (f.size != product(f.dims)) {
                    set_error("gpu_execute: input tensor size does not match its shape");
                    return false;
                }
                break;
            }
            case OP_FUSED:
            case OP_MATMUL: {
                if (n->n_inputs < 2 || !n->inputs[0] || !n->inputs[1]) {
                    set_error("gpu_execute: matmul node needs two inputs");
                    return false;
                }
                const Info& a = info[index.at(n->inputs[0])];
                const Info& b = info[index.at(n->inputs[1])];
                // eval_fused's rule (graph.c:67-77): same rank >= 2, equal batch
                // dimensions, inner dimensions agree; batches run one after another.
                const size_t r = a.dims.size();
                if (r < 2 || b.dims.size() != r || a.dims[r - 1] != b.dims[r - 2]) {
                    set_error("gpu_execute: incompatible matmul operand shapes (ranks %zu and %zu)", r,
                              b.dims.size());
                    return false;
                }
                for (size_t d = 0; d + 2 < r; ++d) {
                    if (a.dims[d] != b.dims[d]) {
                        set_error("gpu_execute: matmul batch dimension %zu mismatch", d);
                        return false;
                    }
                }
                f.dims = a.dims;
                f.dims[r - 1] = b.dims[r - 1];
                f.size = product(f.dims);
                if (n->op == OP_FUSED) {
                    if (n->n_epilogue > MXB_MAX_EPILOGUE) {
                        set_error("gpu_execute: %d epilogue steps exceed the limit of %d", n->n_epilogue,
                                  MXB_MAX_EPILOGUE);
                        return false;
                    }
                    for (int e = 0; e < n->n_epilogue; ++e) {
                        const EpStep& s = n->epilogue[e];
                        if (s.op == OP_ADD && (!s.operand || !index.count(s.operand))) {
                            set_error("gpu_execute: ADD epilogue operand is not an input of its fused node");
                            return false;
                        }
                    }
                }
                break;
            }
            case OP_ADD: {
                if (n->n_inputs != 2) {
                    set_error("gpu_execute: add node needs two inputs");
                    return false;
                }
                const Info& a = info[index.at(n->inputs[0])];
                const Info& b = info[index.at(n->inputs[1])];
                if (!same_dims(a.dims, b.dims) && !trailing_suffix(a.dims, b.dims)) {
                    set_error("gpu_execute: add operand shape must match, or be a trailing suffix of, the first");
                    return false;
                }
                f.dims = a.dims;
                f.size = a.size;
                break;
            }
            case OP_RELU: {
                if (n->n_inputs != 1) {
                    set_error("gpu_execute: relu node needs one input");
                    return false;
                }
                const Info& a = info[index.at(n->inputs[0])];
                f.dims = a.dims;
                f.size = a.size;
                break;
            }
            default:
                set_error("gpu_execute: op %d is not supported on the GPU (supported: input, fused, matmul, "
                          "add, relu)",
                          static_cast<int>(n->op));
                return false;
        }
    }
    for (size_t j = 0; j < order.size(); ++j) {
        const Node* n = order[j];
        for (int a = 0; a < n->n_inputs; ++a) {
            auto it = index.find(n->inputs[a]);
            if (it != index.end() && static_cast<int>(j) > info[it->second].last_use)
                info[it->second].last_use = static_cast<int>(j);
        }
    }
    return true;
}

// ---------------------------------------------------------------- product fusion

// MINIXLA_DUAL_GEMM=0 runs every second product as its own launch (the two
// forms give the same values; tests compare them).
static bool dual_kernel_enabled() {
    const char* v = getenv("MINIXLA_DUAL_GEMM");
    return !(v && v[0] == '0');
}
//
// optimize() never fuses a bare matmul (optimizer.c:94-132), so a matmul that
// feeds a fused node's ADD step stays a node of its own and eval_fused adds
// its stored result (graph.c:98-105) -- config 4's F2 = relu(h W2 + b2) +
// h W2'.  When that fused node is the matmul's only reader and both products
// share the left operand, they run in one kernel (the pair kernels' DUAL
// forms, TF32 and 3xTF32): A is staged once for both and the matmul's value
// never goes to HBM.  Conditions: the matmul is 2-D, not the root, read once
// (by one ADD step), has the fused node's A node as its A, and is shaped like
// the fused node's 2-D output with more than 16 rows; the row pitches are
// multiples of 4 (no padding copies).  launch_gemm still runs the two
// products as two launches where the one-kernel form does not apply.
// Returns, per node, the index of the matmul it absorbs (-1 for none).
static std::vector<int> plan_products(const std::vector<const Node*>& order,
                                      const std::unordered_map<const Node*, int>& index,
                                      const std::vector<Info>& info, int precision) {
    const size_t n = order.size();
    std::vector<int> absorb(n, -1);
    if (!dual_kernel_enabled()) return absorb;
    std::vector<int> refs(n, 0);
    for (size_t i = 0; i < n; ++i)
        for (int a = 0; a < order[i]->n_inputs; ++a) refs[index.at(order[i]->inputs[a])]++;
    auto two_d = [&](int k) { return info[k].dims.size() == 2; };
    for (size_t i = 0; i < n; ++i) {
        const Node* f = order[i];
        if (f->op != OP_FUSED || !two_d(static_cast<int>(i)) || info[i].dims[0] <= kSkinnyMaxRows) continue;
        const int fa = index.at(f->inputs[0]), fb = index.at(f->inputs[1]);
        if (info[fa].dims[1] % 4 || info[fb].dims[1] % 4) continue;
        for (int e = 0; e < f->n_epilogue && absorb[i] < 0; ++e) {
            if (f->epilogue[e].op != OP_ADD) continue;
            const int j = index.at(f->epilogue[e].operand);
            const Node* m = order[j];
            if (m->op != OP_MATMUL || j == static_cast<int>(n) - 1 || refs[j] != 1 || !two_d(j) ||
                info[j].dims != info[i].dims)
                continue;
            if (m->inputs[0] != f->inputs[0]) continue;
            const int mb = index.at(m->inputs[1]);
            if (!two_d(mb) || info[mb].dims[1] % 4) continue;
            absorb[i] = j;
        }
    }
    return absorb;
}

// ---------------------------------------------------------------- GEMM dispatch

// Device operand of a fused GEMM, with its row pitch; `owned` buffers are
// temporaries to hand back to the pool after the launch.
struct Operand {
    const float* ptr = nullptr;
    long long ld = 0;
    float* owned = nullptr;
};

// TMA needs 16-byte row pitches: a matrix whose width is not a multiple of 4
// is copied into a pitch-padded temporary (one strided device copy).
static bool tma_operand(GpuCtx* ctx, const float* src, long long rows, long long cols, Operand& op,
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

// Launches epi(A @ B) with already-validated, TMA-ready operands.  For
// 3xTF32 the low parts of A and B (x - rne_tf32(x)) go to pooled workspace first.
// A second product A[M,K] @ B[K,N] that a fused node's MXB_EP_ADD_PRODUCT
// step adds (a bare matmul absorbed into its only consumer).
struct Product {
    const float* A;
    long long lda;
    const float* B;
    long long ldb;
    int K;
    const float* B_small = nullptr;  // 3xTF32: low part of B made beforehand (else split here)
};

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

static int launch_gemm(GpuCtx* ctx, const float* A, long long lda, const float* B, long long ldb, float* out,
                       long long ldo, int M, int N, int K, const EpStepDev* steps, int n_steps, int precision,
                       cudaStream_t stream, const float* B_small_pre = nullptr, long long row_base = 0,
                       const Product* prod = nullptr) {
    if (prod && !dual_in_one_kernel(ctx, A, lda, M, N, K, *prod, precision)) {
        // Two launches: the second product into pooled workspace, then the
        // node reading it as a full add at the same step.
        float* ws = static_cast<float*>(ctx->pool->alloc(static_cast<size_t>(M) * N * sizeof(float), stream));
        if (!ws) return MXB_E_NOMEM;
        int rc = launch_gemm(ctx, prod->A, prod->lda, prod->B, prod->ldb, ws, N, M, N, prod->K, nullptr, 0, precision,
                             stream, prod->B_small);
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
                             row_base);
        }
        ctx->pool->release(ws, stream);
        return rc;
    }
    if (M <= kSkinnyMaxRows) {
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
    float* ws[3] = {nullptr, nullptr, nullptr};
    int rc = MXB_OK;
    if (precision == GPU_PRECISION_3XTF32) {
        const size_t a_bytes = static_cast<size_t>(M) * lda * 4, b_bytes = static_cast<size_t>(K) * ldb * 4;
        const bool need_b2 = prod && !prod->B_small;
        ws[0] = static_cast<float*>(ctx->pool->alloc(a_bytes, stream));
        if (ws[0] && !B_small_pre) ws[1] = static_cast<float*>(ctx->pool->alloc(b_bytes, stream));
        if (ws[0] && need_b2)
            ws[2] = static_cast<float*>(ctx->pool->alloc(static_cast<size_t>(K) * prod->ldb * 4, stream));
        if (!ws[0] || (!B_small_pre && !ws[1]) || (need_b2 && !ws[2])) {
            rc = MXB_E_NOMEM;
        } else if (!cuda_ok(launch_split_tf32(A, M, K, lda, ws[0], lda, ctx->num_sms, stream), "split A") ||
                   (!B_small_pre &&
                    !cuda_ok(launch_split_tf32(B, K, N, ldb, ws[1], ldb, ctx->num_sms, stream), "split B")) ||
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
static int build_epilogue(const Node* n, int M, int N, long long batch, long long bt,
                          const std::unordered_map<const Node*, const float*>& dev_of,
                          const std::unordered_map<const Node*, long long>& size_of, EpStepDev* out,
                          const Node* absorbed = nullptr) {
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

// Runs one matmul-anchored node on device buffers: `batch` products of
// A[M,K] @ B[K,N] stored back to back (batch = 1 for 2-D nodes).
static int run_gemm_node(GpuCtx* ctx, const Node* n, const float* dA, int M, int K, const float* dB, int N,
                         float* dOut, const std::unordered_map<const Node*, const float*>& dev_of,
                         const std::unordered_map<const Node*, long long>& size_of, int precision,
                         cudaStream_t stream, long long batch = 1, const Node* absorbed = nullptr,
                         const Product* prod = nullptr) {
    Operand a, b;
    int rc = MXB_OK;
    // Pitch padding treats the batches as one tall matrix (rows are contiguous).
    if (!tma_operand(ctx, dA, batch * M, K, a, stream) || !tma_operand(ctx, dB, batch * K, N, b, stream)) {
        rc = MXB_E_NOMEM;
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
static int finish(GpuCtx* ctx) {
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

static Tensor* new_host_tensor(const std::vector<int>& dims) {
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
    t->data = static_cast<float*>(malloc(size * sizeof(float)));
    if (!t->shape || !t->strides || !t->data) {
        free(t->data);
        free(t->shape);
        free(t->strides);
        free(t);
        return nullptr;
    }
    return t;
}

// ---------------------------------------------------------------- row streaming
//
// When every computed node is row-wise in one row count M -- a GEMM's output
// rows follow the rows of its A operand (B is needed whole), add / relu rows
// follow their inputs -- the graph runs in row chunks.  Leaves needed whole
// (B operands, bias rows) are uploaded first; leaves whose rows follow M are
// uploaded chunk by chunk on a copy stream, each chunk's kernels start on the
// compute stream as soon as its rows have landed, and each chunk's result rows
// go back on a second copy stream, so copies in both directions overlap the
// arithmetic.  Graphs that need an intermediate whole (as a B operand, or
// through eval_fused's modulo rule) keep the one-stream executor.

struct RowStreamPlan {
    bool ok = false;
    int M = 0;
    std::vector<char> chunked;  // per node (leaves only): upload by row chunks
};

static bool rows_follow(const Info& f, int M) { return f.dims.size() == 2 && f.dims[0] == M; }

static RowStreamPlan plan_row_stream(const std::vector<const Node*>& order,
                                     const std::unordered_map<const Node*, int>& index,
                                     const std::vector<Info>& info) {
    RowStreamPlan plan;
    const size_t n = order.size();
    if (order.back()->op == OP_INPUT || info.back().dims.size() != 2) return plan;
    const int M = info.back().dims[0];
    std::vector<char> whole(n, 0), rowwise(n, 0);
    auto row_source = [&](int i) { return order[i]->op == OP_INPUT ? rows_follow(info[i], M) : rowwise[i] != 0; };
    for (size_t i = 0; i < n; ++i) {
        const Node* nd = order[i];
        const Info& f = info[i];
        if (nd->op == OP_INPUT) continue;
        if (!rows_follow(f, M)) return plan;
        if (nd->op == OP_FUSED || nd->op == OP_MATMUL) {
            const int ia = index.at(nd->inputs[0]), ib = index.at(nd->inputs[1]);
            whole[ib] = 1;
            if (!row_source(ia) || info[ia].dims[1] % 4 || info[ib].dims[1] % 4) return plan;
            if (nd->op == OP_FUSED) {
                for (int e = 0; e < nd->n_epilogue; ++e) {
                    if (nd->epilogue[e].op != OP_ADD) continue;
                    const int io = index.at(nd->epilogue[e].operand);
                    if (info[io].size == f.size) {
                        if (!(row_source(io) && info[io].dims == f.dims)) return plan;
                    } else {
                        whole[io] = 1;  // bias row, or an operand read by eval_fused's modulo rule
                    }
                }
            }
        } else if (nd->op == OP_ADD) {
            const int ia = index.at(nd->inputs[0]), ib = index.at(nd->inputs[1]);
            if (!row_source(ia)) return plan;
            if (info[ib].size == f.size) {
                if (!row_source(ib)) return plan;
            } else {
                whole[ib] = 1;  // trailing-suffix row of length dims[1]
            }
        } else if (nd->op == OP_RELU) {
            if (!row_source(index.at(nd->inputs[0]))) return plan;
        } else {
            return plan;
        }
        rowwise[i] = 1;
    }
    plan.chunked.assign(n, 0);
    for (size_t i = 0; i < n; ++i) {
        if (order[i]->op != OP_INPUT) {
            if (whole[i]) return plan;
        } else if (!whole[i] && rows_follow(info[i], M)) {
            plan.chunked[i] = 1;
        }
    }
    plan.ok = true;
    plan.M = M;
    return plan;
}

constexpr int kSideStreams = 3;

static cudaEvent_t sync_event(GpuCtx* ctx, size_t k) {
    while (ctx->sync_events.size() <= k) {
        cudaEvent_t e = nullptr;
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        ctx->sync_events.push_back(e);
    }
    return ctx->sync_events[k];
}

// Runs a graph that plan_row_stream accepted; the root's rows are written to
// `host_dst` (root.size floats).
static int execute_streamed(GpuCtx* ctx, const std::vector<const Node*>& order,
                            const std::unordered_map<const Node*, int>& index, std::vector<Info>& info,
                            const RowStreamPlan& plan, int chunks, float* host_dst) {
    cudaStream_t cs = ctx->stream, hs = ctx->h2d, ds = ctx->d2h;
    const int M = plan.M;
    const int rows_per = std::max(128, (M + chunks - 1) / chunks);
    const int n_chunks = (M + rows_per - 1) / rows_per;
    const size_t n = order.size();
    std::vector<float*> b_small(n, nullptr), b2_small(n, nullptr);
    size_t next_event = 0;
    int rc = MXB_OK;
    auto order_after = [&](cudaStream_t waiter, cudaStream_t signaller) {
        cudaEvent_t e = sync_event(ctx, next_event++);
        if (!e || cudaEventRecord(e, signaller) != cudaSuccess || cudaStreamWaitEvent(waiter, e, 0) != cudaSuccess) {
            set_error("row streaming: event ordering failed");
            return false;
        }
        return true;
    };

    std::vector<char> chunked = plan.chunked;
    const std::vector<int> absorb = plan_products(order, index, info, ctx->precision);
    std::vector<char> absorbed(n, 0);
    for (size_t i = 0; i < n; ++i)
        if (absorb[i] >= 0) absorbed[absorb[i]] = 1;
    for (size_t i = 0; i < n && rc == MXB_OK; ++i) {
        if (absorbed[i]) continue;  // computed inside its consumer's kernel, chunk by chunk
        if (float* res = resident_copy(ctx, order[i], 0)) {
            info[i].dev = res;
            info[i].borrowed = true;
            chunked[i] = 0;
            continue;
        }
        info[i].dev = static_cast<float*>(ctx->pool->alloc(static_cast<size_t>(info[i].size) * 4, cs));
        if (!info[i].dev) rc = MXB_E_NOMEM;
    }
    // Uploads may touch pooled blocks only after the compute stream's earlier work on them.
    if (rc == MXB_OK && !order_after(hs, cs)) rc = MXB_E_CUDA;
    for (size_t i = 0; i < n && rc == MXB_OK; ++i) {
        if (order[i]->op == OP_INPUT && !chunked[i] && !info[i].borrowed &&
            !cuda_ok(copy_h2d(ctx->stager, info[i].dev, order[i]->output->data,
                              static_cast<size_t>(info[i].size) * 4, hs),
                     "input upload"))
            rc = MXB_E_CUDA;
    }
    if (rc == MXB_OK && !order_after(cs, hs)) rc = MXB_E_CUDA;
    // 3xTF32: the low part of every B operand, once for all chunks.
    for (size_t i = 0; i < n && rc == MXB_OK; ++i) {
        const Node* nd = order[i];
        if (ctx->precision != GPU_PRECISION_3XTF32 || (nd->op != OP_FUSED && nd->op != OP_MATMUL) || absorbed[i])
            continue;
        const Info& b = info[index.at(nd->inputs[1])];
        b_small[i] = static_cast<float*>(ctx->pool->alloc(static_cast<size_t>(b.size) * 4, cs));
        if (!b_small[i]) {
            rc = MXB_E_NOMEM;
        } else if (!cuda_ok(launch_split_tf32(b.dev, b.dims[0], b.dims[1], b.dims[1], b_small[i], b.dims[1],
                                              ctx->num_sms, cs),
                            "split B")) {
            rc = MXB_E_CUDA;
        }
        if (rc == MXB_OK && absorb[i] >= 0) {
            // The absorbed matmul's B: its low part once for all chunks too.
            const Info& b2 = info[index.at(order[absorb[i]]->inputs[1])];
            b2_small[i] = static_cast<float*>(ctx->pool->alloc(static_cast<size_t>(b2.size) * 4, cs));
            if (!b2_small[i]) {
                rc = MXB_E_NOMEM;
            } else if (!cuda_ok(launch_split_tf32(b2.dev, b2.dims[0], b2.dims[1], b2.dims[1], b2_small[i],
                                                  b2.dims[1], ctx->num_sms, cs),
                                "split B2")) {
                rc = MXB_E_CUDA;
            }
        }
    }
    std::vector<cudaEvent_t> computed(n_chunks, nullptr);
    for (int c = 0; c < n_chunks && rc == MXB_OK; ++c) {
        const long long r0 = static_cast<long long>(c) * rows_per;
        const long long r1 = std::min<long long>(M, r0 + rows_per);
        for (size_t i = 0; i < n && rc == MXB_OK; ++i) {
            if (!chunked[i]) continue;
            const long long cols = info[i].size / M;
            if (!cuda_ok(copy_h2d(ctx->stager, info[i].dev + r0 * cols, order[i]->output->data + r0 * cols,
                                  static_cast<size_t>((r1 - r0) * cols) * 4, hs),
                         "chunk upload"))
                rc = MXB_E_CUDA;
        }
        if (rc == MXB_OK && !order_after(cs, hs)) rc = MXB_E_CUDA;
        for (size_t i = 0; i < n && rc == MXB_OK; ++i) {
            const Node* nd = order[i];
            const Info& f = info[i];
            const long long cols = f.dims.size() == 2 ? f.dims[1] : 0;
            if (absorbed[i]) continue;
            if (nd->op == OP_FUSED || nd->op == OP_MATMUL) {
                const Info& a = info[index.at(nd->inputs[0])];
                const Info& b = info[index.at(nd->inputs[1])];
                const int K = a.dims[1], N = b.dims[1];
                EpStepDev steps[MXB_MAX_EPILOGUE];
                int n_steps = 0;
                for (int e = 0; nd->op == OP_FUSED && e < nd->n_epilogue; ++e) {
                    const EpStep& st = nd->epilogue[e];
                    EpStepDev d{};
                    if (st.op == OP_ADD && absorb[i] >= 0 && st.operand == order[absorb[i]]) {
                        d.kind = MXB_EP_ADD_PRODUCT;
                    } else if (st.op == OP_ADD) {
                        const Info& o = info[index.at(st.operand)];
                        d.kind = o.size == f.size ? MXB_EP_ADD_FULL
                                                  : (o.size == N ? MXB_EP_ADD_ROW : MXB_EP_ADD_MOD);
                        d.ptr = o.size == f.size ? o.dev + r0 * N : o.dev;
                        d.ld_or_size = d.kind == MXB_EP_ADD_MOD ? o.size : N;
                    } else if (st.op == OP_RELU) {
                        d.kind = MXB_EP_RELU;
                    } else {
                        continue;
                    }
                    steps[n_steps++] = d;
                }
                Product prod{};
                if (absorb[i] >= 0) {
                    const Node* m = order[absorb[i]];
                    const Info& a2 = info[index.at(m->inputs[0])];
                    const Info& b2 = info[index.at(m->inputs[1])];
                    const int K2 = a2.dims[1];
                    prod = Product{a2.dev + r0 * K2, K2, b2.dev, N, K2, b2_small[i]};
                }
                rc = launch_gemm(ctx, a.dev + r0 * K, K, b.dev, N, f.dev + r0 * N, N, static_cast<int>(r1 - r0), N, K,
                                 steps, n_steps, ctx->precision, cs, b_small[i], r0, absorb[i] >= 0 ? &prod : nullptr);
            } else if (nd->op == OP_ADD) {
                const Info& a = info[index.at(nd->inputs[0])];
                const Info& b = info[index.at(nd->inputs[1])];
                const bool same = b.size == f.size;
                if (!cuda_ok(launch_add(a.dev + r0 * cols, (r1 - r0) * cols, same ? b.dev + r0 * cols : b.dev,
                                        same ? (r1 - r0) * cols : b.size, f.dev + r0 * cols, ctx->num_sms, cs),
                             "add launch"))
                    rc = MXB_E_CUDA;
            } else if (nd->op == OP_RELU) {
                const Info& a = info[index.at(nd->inputs[0])];
                if (!cuda_ok(launch_relu(a.dev + r0 * cols, (r1 - r0) * cols, f.dev + r0 * cols, ctx->num_sms, cs),
                             "relu launch"))
                    rc = MXB_E_CUDA;
            }
        }
        if (rc == MXB_OK) {
            computed[c] = sync_event(ctx, next_event++);
            if (!computed[c] || cudaEventRecord(computed[c], cs) != cudaSuccess) rc = MXB_E_CUDA;
        }
    }
    // Downloads are enqueued after all uploads and kernels: with a pageable
    // destination each copy blocks the host until it is done.
    const Info& root = info.back();
    const long long out_cols = root.size / M;
    for (int c = 0; c < n_chunks && rc == MXB_OK; ++c) {
        const long long r0 = static_cast<long long>(c) * rows_per;
        const long long r1 = std::min<long long>(M, r0 + rows_per);
        if (cudaStreamWaitEvent(ds, computed[c], 0) != cudaSuccess ||
            !cuda_ok(copy_d2h(ctx->stager, host_dst + r0 * out_cols, root.dev + r0 * out_cols,
                              static_cast<size_t>((r1 - r0) * out_cols) * 4, ds),
                     "chunk download"))
            rc = MXB_E_CUDA;
    }
    // The pool reuses blocks in compute-stream order: join both copy streams first.
    order_after(cs, ds);
    order_after(cs, hs);
    for (size_t i = 0; i < n; ++i) {
        if (!info[i].borrowed) ctx->pool->release(info[i].dev, cs);
        ctx->pool->release(b_small[i], cs);
        ctx->pool->release(b2_small[i], cs);
        info[i].dev = nullptr;
    }
    cudaStreamSynchronize(ds);
    cudaStreamSynchronize(hs);
    const int done = finish(ctx);
    return rc != MXB_OK ? rc : done;
}

static int stream_chunks() {
    const char* c = getenv("MINIXLA_STREAM_CHUNKS");
    return c ? atoi(c) : 8;
}

// ---------------------------------------------------------------- multi-GPU row sharding
//
// A context made by gpu_ctx_create_multi(n) drives n GPUs from one host
// thread.  The rows of every row-wise node are split over the devices
// (shard_range); each device uploads and computes only its rows.  Leaves
// that are read whole -- B operands, bias rows -- go up to device 0 once and
// are replicated to the others by peer copies over NVLink.  Result rows go
// from each device straight into the host tensor, so the output is never
// gathered.  Only when a later node reads an intermediate whole (as its B
// operand, say) do the devices exchange that intermediate's row shards:
// NCCL broadcasts of each shard, grouped into one all-gather.

static void shard_range(long long M, int parts, int part, long long& r0, long long& r1) {
    const long long base = M / parts, extra = M % parts;
    r0 = part * base + std::min<long long>(part, extra);
    r1 = r0 + base + (part < extra ? 1 : 0);
}

struct NcclApi {
    bool ok = false;
    decltype(&ncclCommInitAll) comm_init_all = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    decltype(&ncclBroadcast) broadcast = nullptr;
    decltype(&ncclGroupStart) group_start = nullptr;
    decltype(&ncclGroupEnd) group_end = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
};

// NCCL is loaded on first use (the copy already in the process if there is
// one), so the library itself loads where NCCL is absent.
static const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) return;
        api.comm_init_all = reinterpret_cast<decltype(api.comm_init_all)>(dlsym(h, "ncclCommInitAll"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        api.broadcast = reinterpret_cast<decltype(api.broadcast)>(dlsym(h, "ncclBroadcast"));
        api.group_start = reinterpret_cast<decltype(api.group_start)>(dlsym(h, "ncclGroupStart"));
        api.group_end = reinterpret_cast<decltype(api.group_end)>(dlsym(h, "ncclGroupEnd"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
        api.ok = api.comm_init_all && api.comm_destroy && api.broadcast && api.group_start && api.group_end &&
                 api.error_string;
    });
    return api;
}

struct ShardPlan {
    bool ok = false;
    int M = 0;
    std::vector<char> whole;  // needed whole on every device (replicated / all-gathered)
    std::vector<char> full;   // stored full-size on every device (whole, or not row-aligned)
};

static ShardPlan plan_shards(const std::vector<const Node*>& order, const std::unordered_map<const Node*, int>& index,
                             const std::vector<Info>& info) {
    ShardPlan plan;
    const size_t n = order.size();
    if (order.back()->op == OP_INPUT || info.back().dims.size() != 2) return plan;
    const int M = info.back().dims[0];
    std::vector<char> whole(n, 0), rowwise(n, 0);
    auto row_source = [&](int i) { return order[i]->op == OP_INPUT ? rows_follow(info[i], M) : rowwise[i] != 0; };
    for (size_t i = 0; i < n; ++i) {
        const Node* nd = order[i];
        const Info& f = info[i];
        if (nd->op == OP_INPUT) continue;
        if (!rows_follow(f, M)) return plan;
        if (nd->op == OP_FUSED || nd->op == OP_MATMUL) {
            const int ia = index.at(nd->inputs[0]), ib = index.at(nd->inputs[1]);
            whole[ib] = 1;
            if (!row_source(ia) || info[ia].dims[1] % 4 || info[ib].dims[1] % 4) return plan;
            for (int e = 0; nd->op == OP_FUSED && e < nd->n_epilogue; ++e) {
                if (nd->epilogue[e].op != OP_ADD) continue;
                const int io = index.at(nd->epilogue[e].operand);
                if (info[io].size == f.size) {
                    if (!(row_source(io) && info[io].dims == f.dims)) return plan;
                } else {
                    whole[io] = 1;
                }
            }
        } else if (nd->op == OP_ADD) {
            const int ia = index.at(nd->inputs[0]), ib = index.at(nd->inputs[1]);
            if (!row_source(ia)) return plan;
            if (info[ib].size == f.size) {
                if (!row_source(ib)) return plan;
            } else {
                whole[ib] = 1;
            }
        } else if (nd->op == OP_RELU) {
            if (!row_source(index.at(nd->inputs[0]))) return plan;
        } else {
            return plan;
        }
        rowwise[i] = 1;
    }
    plan.full.assign(n, 0);
    for (size_t i = 0; i < n; ++i)
        plan.full[i] = whole[i] || (order[i]->op == OP_INPUT && !rows_follow(info[i], M));
    plan.whole = whole;
    plan.ok = true;
    plan.M = M;
    return plan;
}

static int nccl_check(ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return MXB_OK;
    set_error("%s: %s", what, nccl().error_string ? nccl().error_string(r) : "NCCL error");
    return MXB_E_CUDA;
}

static int execute_sharded(GpuCtx* ctx0, const std::vector<const Node*>& order,
                           const std::unordered_map<const Node*, int>& index, std::vector<Info>& info,
                           const ShardPlan& plan, float* host_dst) {
    std::vector<GpuCtx*> ctxs{ctx0};
    ctxs.insert(ctxs.end(), ctx0->peers.begin(), ctx0->peers.end());
    const int P = static_cast<int>(ctxs.size());
    const size_t n = order.size();
    const int M = plan.M;
    std::vector<long long> r0(P), r1(P);
    for (int d = 0; d < P; ++d) shard_range(M, P, d, r0[d], r1[d]);
    std::vector<std::vector<float*>> ptr(P, std::vector<float*>(n, nullptr));
    // Resident leaves are whole on every device already.
    std::vector<char> full = plan.full, borrowed(n, 0);
    for (size_t i = 0; i < n; ++i) {
        if (!resident_copy(ctx0, order[i], 0) || !resident_copy(ctx0, order[i], P - 1)) continue;
        borrowed[i] = full[i] = 1;
        for (int d = 0; d < P; ++d) ptr[d][i] = resident_copy(ctx0, order[i], d);
    }
    auto cols_of = [&](size_t i) { return info[i].dims.size() == 2 ? static_cast<long long>(info[i].dims[1]) : 0ll; };
    // Rows [r0, r1) of node i on device d.
    auto rows = [&](int d, size_t i) { return full[i] ? ptr[d][i] + r0[d] * cols_of(i) : ptr[d][i]; };
    int rc = MXB_OK;

    for (int d = 0; d < P && rc == MXB_OK; ++d) {
        DeviceScope scope(ctxs[d]->device);
        for (size_t i = 0; i < n && rc == MXB_OK; ++i) {
            if (borrowed[i]) continue;
            const long long elems = full[i] ? info[i].size : (r1[d] - r0[d]) * cols_of(i);
            if (elems <= 0) continue;
            ptr[d][i] = static_cast<float*>(ctxs[d]->pool->alloc(static_cast<size_t>(elems) * 4, ctxs[d]->stream));
            if (!ptr[d][i]) rc = MXB_E_NOMEM;
        }
    }
    // Leaves: row shards straight from the host; whole leaves once to device 0, then peer copies.
    size_t ev_k = 0;
    for (size_t i = 0; i < n && rc == MXB_OK; ++i) {
        if (order[i]->op != OP_INPUT || borrowed[i]) continue;
        const float* host = order[i]->output->data;
        if (!full[i]) {
            for (int d = 0; d < P && rc == MXB_OK; ++d) {
                if (!ptr[d][i]) continue;
                DeviceScope scope(ctxs[d]->device);
                const long long c = cols_of(i);
                if (!cuda_ok(copy_h2d(ctxs[d]->stager, ptr[d][i], host + r0[d] * c,
                                      static_cast<size_t>((r1[d] - r0[d]) * c) * 4, ctxs[d]->stream),
                             "shard upload"))
                    rc = MXB_E_CUDA;
            }
            continue;
        }
        const size_t bytes = static_cast<size_t>(info[i].size) * 4;
        {
            DeviceScope scope(ctx0->device);
            if (!cuda_ok(copy_h2d(ctx0->stager, ptr[0][i], host, bytes, ctx0->stream), "upload"))
                rc = MXB_E_CUDA;
        }
        cudaEvent_t e = nullptr;
        if (rc == MXB_OK && P > 1) {
            DeviceScope scope(ctx0->device);
            e = sync_event(ctx0, ev_k++);
            if (!e || cudaEventRecord(e, ctx0->stream) != cudaSuccess) rc = MXB_E_CUDA;
        }
        for (int d = 1; d < P && rc == MXB_OK; ++d) {
            DeviceScope scope(ctxs[d]->device);
            if (cudaStreamWaitEvent(ctxs[d]->stream, e, 0) != cudaSuccess ||
                !cuda_ok(cudaMemcpyPeerAsync(ptr[d][i], ctxs[d]->device, ptr[0][i], ctx0->device, bytes,
                                             ctxs[d]->stream),
                         "peer replication"))
                rc = MXB_E_CUDA;
        }
    }
    // Computed nodes, each device on its own rows.
    for (size_t i = 0; i < n && rc == MXB_OK; ++i) {
        const Node* nd = order[i];
        if (nd->op == OP_INPUT) continue;
        const Info& f = info[i];
        const long long cols = cols_of(i);
        for (int d = 0; d < P && rc == MXB_OK; ++d) {
            const long long m = r1[d] - r0[d];
            if (m <= 0) continue;
            GpuCtx* c = ctxs[d];
            DeviceScope scope(c->device);
            if (nd->op == OP_FUSED || nd->op == OP_MATMUL) {
                const size_t ia = index.at(nd->inputs[0]), ib = index.at(nd->inputs[1]);
                const int K = info[ia].dims[1], N = info[ib].dims[1];
                EpStepDev steps[MXB_MAX_EPILOGUE];
                int n_steps = 0;
                for (int e = 0; nd->op == OP_FUSED && e < nd->n_epilogue; ++e) {
                    const EpStep& st = nd->epilogue[e];
                    EpStepDev s{};
                    if (st.op == OP_ADD) {
                        const size_t io = index.at(st.operand);
                        const Info& o = info[io];
                        s.kind = o.size == f.size ? MXB_EP_ADD_FULL : (o.size == N ? MXB_EP_ADD_ROW : MXB_EP_ADD_MOD);
                        s.ptr = s.kind == MXB_EP_ADD_FULL ? rows(d, io) : ptr[d][io];
                        s.ld_or_size = s.kind == MXB_EP_ADD_MOD ? o.size : N;
                    } else if (st.op == OP_RELU) {
                        s.kind = MXB_EP_RELU;
                    } else {
                        continue;
                    }
                    steps[n_steps++] = s;
                }
                rc = launch_gemm(c, rows(d, ia), K, ptr[d][ib], N, rows(d, i), N, static_cast<int>(m), N, K, steps,
                                 n_steps, ctx0->precision, c->stream, nullptr, r0[d]);
            } else if (nd->op == OP_ADD) {
                const size_t ia = index.at(nd->inputs[0]), ib = index.at(nd->inputs[1]);
                const bool same = info[ib].size == f.size;
                if (!cuda_ok(launch_add(rows(d, ia), m * cols, same ? rows(d, ib) : ptr[d][ib],
                                        same ? m * cols : info[ib].size, rows(d, i), c->num_sms, c->stream),
                             "add launch"))
                    rc = MXB_E_CUDA;
            } else if (nd->op == OP_RELU) {
                const size_t ia = index.at(nd->inputs[0]);
                if (!cuda_ok(launch_relu(rows(d, ia), m * cols, rows(d, i), c->num_sms, c->stream), "relu launch"))
                    rc = MXB_E_CUDA;
            }
        }
        if (rc != MXB_OK || !plan.whole[i] || P == 1) continue;
        // A later node reads this intermediate whole: all-gather its row shards.
        const NcclApi& api = nccl();
        if (!api.ok) {
            set_error("multi-GPU all-gather needs NCCL (libnccl.so.2), which could not be loaded");
            rc = MXB_E_UNSUPPORTED;
            break;
        }
        if (ctx0->comms.empty()) {
            std::vector<int> devs(P);
            for (int d = 0; d < P; ++d) devs[d] = ctxs[d]->device;
            ctx0->comms.assign(P, nullptr);
            rc = nccl_check(api.comm_init_all(ctx0->comms.data(), P, devs.data()), "ncclCommInitAll");
            if (rc != MXB_OK) {
                ctx0->comms.clear();
                break;
            }
        }
        rc = nccl_check(api.group_start(), "ncclGroupStart");
        for (int root = 0; root < P && rc == MXB_OK; ++root) {
            const long long count = (r1[root] - r0[root]) * cols;
            if (count <= 0) continue;
            for (int d = 0; d < P && rc == MXB_OK; ++d) {
                rc = nccl_check(api.broadcast(rows(root, i), ptr[d][i] + r0[root] * cols, static_cast<size_t>(count),
                                              ncclFloat, root, ctx0->comms[d], ctxs[d]->stream),
                                "ncclBroadcast");
            }
        }
        const int end = nccl_check(api.group_end(), "ncclGroupEnd");
        if (rc == MXB_OK) rc = end;
    }
    // Result rows from every device into the host tensor.
    const size_t root_i = n - 1;
    const long long out_cols = cols_of(root_i);
    for (int d = 0; d < P && rc == MXB_OK; ++d) {
        const long long m = r1[d] - r0[d];
        if (m <= 0) continue;
        DeviceScope scope(ctxs[d]->device);
        if (!cuda_ok(copy_d2h(ctxs[d]->stager, host_dst + r0[d] * out_cols, rows(d, root_i),
                              static_cast<size_t>(m * out_cols) * 4, ctxs[d]->stream),
                     "shard download"))
            rc = MXB_E_CUDA;
    }
    for (int d = 0; d < P; ++d) {
        DeviceScope scope(ctxs[d]->device);
        const int done = finish(ctxs[d]);
        if (rc == MXB_OK) rc = done;
        for (size_t i = 0; i < n; ++i)
            if (!borrowed[i]) ctxs[d]->pool->release(ptr[d][i], ctxs[d]->stream);
    }
    return rc;
}

// The DAG executor behind gpu_execute / gpu_execute_into.  When `dst` is
// given the root is downloaded into it (its size must match), otherwise a
// new host tensor is returned through *result.
static int execute_graph(Node* root, GpuCtx* ctx, Tensor* dst, Tensor** result) {
    if (!root || !ctx) {
        set_error("gpu_execute: NULL root or context");
        return MXB_E_ARG;
    }
    DeviceScope scope(ctx->device);
    cudaStream_t stream = ctx->stream;
    const std::vector<const Node*> order = topo_order(root);
    std::unordered_map<const Node*, int> index;
    std::vector<Info> info;
    if (!infer_shapes(order, index, info)) return MXB_E_UNSUPPORTED;

    if (!ctx->peers.empty()) {
        const ShardPlan plan = plan_shards(order, index, info);
        if (plan.ok) {
            if (dst && (!dst->data || static_cast<long long>(dst->size) != info.back().size)) {
                set_error("gpu_execute_into: destination holds %zu elements, result has %lld",
                          static_cast<size_t>(dst->size), info.back().size);
                return MXB_E_ARG;
            }
            Tensor* t = dst ? nullptr : new_host_tensor(info.back().dims);
            if (!dst && !t) {
                set_error("gpu_execute: host allocation of the result failed");
                return MXB_E_NOMEM;
            }
            const int rc = execute_sharded(ctx, order, index, info, plan, dst ? dst->data : t->data);
            if (rc != MXB_OK) {
                if (t) {
                    free(t->data);
                    free(t->shape);
                    free(t->strides);
                    free(t);
                }
                return rc;
            }
            if (t) *result = t;
            return MXB_OK;
        }
        // Not row-shardable: the whole graph runs on device 0.
    }

    const int chunks = stream_chunks();
    if (chunks > 1 && info.back().dims.size() == 2 && info.back().dims[0] >= 2 * 128) {
        const RowStreamPlan plan = plan_row_stream(order, index, info);
        if (plan.ok) {
            if (dst) {
                if (!dst->data || static_cast<long long>(dst->size) != info.back().size) {
                    set_error("gpu_execute_into: destination holds %zu elements, result has %lld",
                              static_cast<size_t>(dst->size), info.back().size);
                    return MXB_E_ARG;
                }
                return execute_streamed(ctx, order, index, info, plan, chunks, dst->data);
            }
            Tensor* t = new_host_tensor(info.back().dims);
            if (!t) {
                set_error("gpu_execute: host allocation of the result failed");
                return MXB_E_NOMEM;
            }
            const int rc = execute_streamed(ctx, order, index, info, plan, chunks, t->data);
            if (rc != MXB_OK) {
                free(t->data);
                free(t->shape);
                free(t->strides);
                free(t);
                return rc;
            }
            *result = t;
            return MXB_OK;
        }
    }

    // Independent nodes run on different streams (up to 1 + kSideStreams): a
    // computed node continues the stream of an input whose chain it extends,
    // else it takes the stream whose last node is oldest.  Inputs made on
    // another stream are waited on by event, and a buffer goes back to the
    // pool only after every consumer's stream has passed it.
    const size_t n_nodes = order.size();
    if (ctx->side.empty()) {
        for (int k = 0; k < kSideStreams; ++k) {
            cudaStream_t st = nullptr;
            if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) {
                cudaGetLastError();
                break;
            }
            ctx->side.push_back(st);
        }
    }
    std::vector<cudaStream_t> streams{stream};
    streams.insert(streams.end(), ctx->side.begin(), ctx->side.end());
    const int n_streams = static_cast<int>(streams.size());
    std::vector<int> stream_of(n_nodes, 0), last_on(n_streams, -1);
    std::vector<cudaEvent_t> done(n_nodes, nullptr);
    std::vector<std::vector<int>> inputs_of(n_nodes), consumers(n_nodes);
    // A matmul absorbed into its consumer is never materialised: its inputs
    // become inputs of the consumer and live until the consumer has run.
    const std::vector<int> absorb = plan_products(order, index, info, ctx->precision);
    std::vector<char> absorbed(n_nodes, 0);
    for (size_t i = 0; i < n_nodes; ++i)
        if (absorb[i] >= 0) absorbed[absorb[i]] = 1;
    for (size_t i = 0; i < n_nodes; ++i) {
        if (absorbed[i]) continue;
        auto add_input = [&](const Node* in) {
            const int j = index.at(in);
            if (std::find(inputs_of[i].begin(), inputs_of[i].end(), j) != inputs_of[i].end()) return;
            inputs_of[i].push_back(j);
            consumers[j].push_back(static_cast<int>(i));
        };
        for (int a = 0; a < order[i]->n_inputs; ++a) {
            const Node* in = order[i]->inputs[a];
            if (absorb[i] >= 0 && in == order[absorb[i]]) {
                for (int b = 0; b < in->n_inputs; ++b) add_input(in->inputs[b]);
            } else {
                add_input(in);
            }
        }
    }
    for (size_t i = 0; i < n_nodes; ++i) info[i].last_use = -1;
    for (size_t i = 0; i < n_nodes; ++i)
        for (int j : inputs_of[i]) info[j].last_use = std::max(info[j].last_use, static_cast<int>(i));
    size_t next_event = 0;

    std::unordered_map<const Node*, const float*> dev_of;
    std::unordered_map<const Node*, long long> size_of;
    int rc = MXB_OK;
    for (size_t i = 0; i < n_nodes && rc == MXB_OK; ++i) {
        const Node* n = order[i];
        Info& f = info[i];
        if (absorbed[i]) continue;  // computed inside its consumer's kernel
        int sidx = -1;
        if (n->op == OP_INPUT) {
            sidx = 0;
        } else {
            for (int j : inputs_of[i])
                if (order[j]->op != OP_INPUT && last_on[stream_of[j]] == j) {
                    sidx = stream_of[j];
                    break;
                }
            if (sidx < 0) {
                sidx = 0;
                for (int k = 1; k < n_streams; ++k)
                    if (last_on[k] < last_on[sidx]) sidx = k;
            }
        }
        stream_of[i] = sidx;
        const cudaStream_t st = streams[sidx];
        for (int j : inputs_of[i])
            if (stream_of[j] != sidx && done[j]) cudaStreamWaitEvent(st, done[j], 0);
        if (float* res = resident_copy(ctx, n, 0)) {
            f.dev = res;
            f.borrowed = true;
        } else {
            f.dev = static_cast<float*>(ctx->pool->alloc(static_cast<size_t>(f.size) * 4, st));
        }
        if (!f.dev) {
            rc = MXB_E_NOMEM;
            break;
        }
        dev_of[n] = f.dev;
        size_of[n] = f.size;
        switch (n->op) {
            case OP_INPUT:
                if (!f.borrowed && !cuda_ok(copy_h2d(ctx->stager, f.dev, n->output->data,
                                                     static_cast<size_t>(f.size) * 4, st),
                                            "input upload"))
                    rc = MXB_E_CUDA;
                break;
            case OP_FUSED:
            case OP_MATMUL: {
                const Info& a = info[index.at(n->inputs[0])];
                const Info& b = info[index.at(n->inputs[1])];
                const size_t r = a.dims.size();
                const long long batch = a.size / (static_cast<long long>(a.dims[r - 2]) * a.dims[r - 1]);
                if (absorb[i] >= 0) {
                    const Node* m = order[absorb[i]];
                    const Info& a2 = info[index.at(m->inputs[0])];
                    const Info& b2 = info[index.at(m->inputs[1])];
                    const Product prod{a2.dev, a2.dims[1], b2.dev, b2.dims[1], a2.dims[1]};
                    rc = run_gemm_node(ctx, n, a.dev, a.dims[0], a.dims[1], b.dev, b.dims[1], f.dev, dev_of, size_of,
                                       ctx->precision, st, 1, m, &prod);
                } else {
                    rc = run_gemm_node(ctx, n, a.dev, a.dims[r - 2], a.dims[r - 1], b.dev, b.dims[r - 1], f.dev,
                                       dev_of, size_of, ctx->precision, st, batch);
                }
                break;
            }
            case OP_ADD: {
                const Info& a = info[index.at(n->inputs[0])];
                const Info& b = info[index.at(n->inputs[1])];
                if (!cuda_ok(launch_add(a.dev, a.size, b.dev, b.size, f.dev, ctx->num_sms, st), "add launch"))
                    rc = MXB_E_CUDA;
                break;
            }
            case OP_RELU: {
                const Info& a = info[index.at(n->inputs[0])];
                if (!cuda_ok(launch_relu(a.dev, a.size, f.dev, ctx->num_sms, st), "relu launch"))
                    rc = MXB_E_CUDA;
                break;
            }
            default:
                rc = MXB_E_UNSUPPORTED;
        }
        if (rc != MXB_OK) break;
        done[i] = sync_event(ctx, next_event++);
        if (!done[i] || cudaEventRecord(done[i], st) != cudaSuccess) {
            set_error("gpu_execute: event record failed");
            rc = MXB_E_CUDA;
            break;
        }
        last_on[sidx] = static_cast<int>(i);
        // Last-use release (gpu_exec.c:520-528), stream-ordered into the pool
        // after every consumer of the buffer.
        for (int j : inputs_of[i]) {
            Info& in = info[j];
            if (in.last_use != static_cast<int>(i) || !in.dev) continue;
            if (!in.borrowed) {
                for (int c : consumers[j])
                    if (stream_of[c] != sidx && done[c]) cudaStreamWaitEvent(st, done[c], 0);
                ctx->pool->release(in.dev, st);
            }
            in.dev = nullptr;
        }
    }
    // Everything joins the main stream before the result is read.
    for (int k = 1; k < n_streams; ++k)
        if (last_on[k] >= 0) cudaStreamWaitEvent(stream, done[last_on[k]], 0);

    Info& r = info.back();  // the root is last in post-order
    if (rc == MXB_OK) rc = finish(ctx);
    if (rc == MXB_OK) {
        if (dst) {
            if (!dst->data || static_cast<long long>(dst->size) != r.size) {
                set_error("gpu_execute_into: destination holds %zu elements, result has %lld",
                          dst ? static_cast<size_t>(dst->size) : 0, r.size);
                rc = MXB_E_ARG;
            } else if (!cuda_ok(copy_d2h(ctx->stager, dst->data, r.dev, static_cast<size_t>(r.size) * 4, stream),
                                "result download") ||
                       !cuda_ok(cudaStreamSynchronize(stream), "download synchronize")) {
                rc = MXB_E_CUDA;
            }
        } else {
            Tensor* t = new_host_tensor(r.dims);
            if (!t) {
                set_error("gpu_execute: host allocation of the result failed");
                rc = MXB_E_NOMEM;
            } else if (!cuda_ok(copy_d2h(ctx->stager, t->data, r.dev, static_cast<size_t>(r.size) * 4, stream),
                                "result download") ||
                       !cuda_ok(cudaStreamSynchronize(stream), "download synchronize")) {
                free(t->data);
                free(t->shape);
                free(t->strides);
                free(t);
                rc = MXB_E_CUDA;
            } else {
                *result = t;
            }
        }
    }
    for (Info& f : info) {
        if (f.dev && !f.borrowed) ctx->pool->release(f.dev, stream);
        f.dev = nullptr;
    }
    if (rc != MXB_OK) cudaStreamSynchronize(stream);
    return rc;
}

// ---------------------------------------------------------------- single-node paths

// Device copies of one fused node's operands, taken from the host tensors
// hanging off its inputs (runtime.c:17-84 and gpu_exec.c:339-362 do the same).
struct SingleNode {
    int M = 0, N = 0, K = 0;
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

static int prepare_single(const Node* fused, GpuCtx* ctx, const char* who, SingleNode& s) {
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
    if (a->ndim != 2 || b->ndim != 2) {
        set_error("%s: only 2D tensors supported", who);
        return MXB_E_UNSUPPORTED;
    }
    if (a->shape[1] != b->shape[0]) {
        set_error("%s: incompatible matmul operand shapes", who);
        return MXB_E_ARG;
    }
    if (fused->op == OP_FUSED && fused->n_epilogue > MXB_MAX_EPILOGUE) {
        set_error("%s: too many epilogue steps", who);
        return MXB_E_UNSUPPORTED;
    }
    s.M = a->shape[0];
    s.K = a->shape[1];
    s.N = b->shape[1];
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
    s.dOut = static_cast<float*>(ctx->pool->alloc(static_cast<size_t>(s.M) * s.N * 4, ctx->stream));
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
    int rc = prepare_single(root, ctx, who, s);
    if (rc == MXB_OK) {
        for (int w = 0; w < warmup && rc == MXB_OK; ++w) {
            rc = run_gemm_node(ctx, root, s.dA, s.M, s.K, s.dB, s.N, s.dOut, s.dev_of, s.size_of, precision,
                               ctx->stream);
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
                               ctx->stream);
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
    if (!ok || !g->pool || !g->stager) {
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

int mxb_fused_gemm(GpuCtx* ctx, const float* A, long long lda, const float* B, long long ldb, float* out,
                   long long ldo, int M, int N, int K, const mxb_ep_step* steps, int n_steps, int precision,
                   void* stream) {
    if (!ctx || !A || !B || !out || M < 1 || N < 1 || K < 1 || lda < K || ldb < N || ldo < N ||
        n_steps < 0 || n_steps > MXB_MAX_EPILOGUE || (n_steps > 0 && !steps) || !mxb::valid_precision(precision)) {
        set_error("mxb_fused_gemm: invalid arguments");
        return MXB_E_ARG;
    }
    if (lda % 4 || ldb % 4 || (reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15)) {
        set_error("mxb_fused_gemm: A and B need 16-byte aligned bases and row pitches (lda %% 4 == 0, ldb %% 4 == 0)");
        return MXB_E_ARG;
    }
    mxb::EpStepDev dev_steps[MXB_MAX_EPILOGUE];
    for (int i = 0; i < n_steps; ++i) {
        const mxb_ep_step& s = steps[i];
        const bool is_add = s.kind == MXB_EP_ADD_FULL || s.kind == MXB_EP_ADD_ROW || s.kind == MXB_EP_ADD_MOD;
        if (s.kind < MXB_EP_ADD_FULL || s.kind > MXB_EP_SCALE || (is_add && !s.operand) ||
            (s.kind == MXB_EP_ADD_FULL && s.ld_or_size < N) || (s.kind == MXB_EP_ADD_MOD && s.ld_or_size < 1)) {
            set_error("mxb_fused_gemm: invalid epilogue step %d", i);
            return MXB_E_ARG;
        }
        memcpy(&dev_steps[i], &s, sizeof(s));
    }
    mxb::DeviceScope scope(ctx->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    return mxb::launch_gemm(ctx, A, lda, B, ldb, out, ldo, M, N, K, dev_steps, n_steps, precision, st);
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

const char* mxb_last_error(void) { return mxb::t_last_error.c_str(); }

}  // extern "C"
