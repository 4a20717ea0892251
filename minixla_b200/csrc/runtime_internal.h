// Declarations shared by the host runtime's translation units: the device
// pool, GpuCtx, the per-node bookkeeping of an execution, and the functions
// that plan a graph, launch its GEMMs and run it with one of the executors
// (one stream + side streams, row-streamed, multi-GPU row shards).
#pragma once

#include <cuda_runtime.h>
#include <nccl.h>

#include <atomic>
#include <cstddef>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "internal.h"

namespace mxb {

inline bool cuda_ok(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return true;
    set_error("%s: %s", what, cudaGetErrorString(e));
    return false;
}

// Process-wide count of pool allocations (MINIXLA_FAIL_ALLOC_AT counts them).
inline std::atomic<long long>& alloc_calls() {
    static std::atomic<long long> n{0};
    return n;
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
        const long long call = alloc_calls().fetch_add(1) + 1;
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
    mxb::Stager* stager_dl = nullptr;  // a second ring for downloads that run beside uploads
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

struct Info {
    const Node* node = nullptr;
    std::vector<int> dims;        // logical output shape
    long long size = 0;           // element count
    int last_use = -1;            // index of the last consumer in topo order
    float* dev = nullptr;         // device buffer (compact, row-major)
    bool borrowed = false;        // dev is a resident copy, not this call's to release
};

// Device operand of a fused GEMM, with its row pitch; `owned` buffers are
// temporaries to hand back to the pool after the launch.
struct Operand {
    const float* ptr = nullptr;
    long long ld = 0;
    float* owned = nullptr;
};

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

struct RowStreamPlan {
    bool ok = false;
    int M = 0;
    std::vector<char> chunked;  // per node (leaves only): upload by row chunks
};

struct NcclApi {
    bool ok = false;
    decltype(&ncclCommInitAll) comm_init_all = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    decltype(&ncclBroadcast) broadcast = nullptr;
    decltype(&ncclGroupStart) group_start = nullptr;
    decltype(&ncclGroupEnd) group_end = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
};

struct ShardPlan {
    bool ok = false;
    int M = 0;
    std::vector<char> whole;  // needed whole on every device (replicated / all-gathered)
    std::vector<char> full;   // stored full-size on every device (whole, or not row-aligned)
};

constexpr int kSideStreams = 3;  // side streams of the one-stream executor

// A 2-D node whose rows are the M rows of the graph's root (row sharding and streaming).
inline bool rows_follow(const Info& f, int M) { return f.dims.size() == 2 && f.dims[0] == M; }

// graph_plan.cu
float* resident_copy(const GpuCtx* ctx, const Node* n, size_t d);
std::vector<const Node*> topo_order(const Node* root);
bool infer_shapes(const std::vector<const Node*>& order, std::unordered_map<const Node*, int>& index,
                  std::vector<Info>& info);
bool dual_kernel_enabled();
std::vector<int> plan_products(const std::vector<const Node*>& order, const std::unordered_map<const Node*, int>& index,
                               const std::vector<Info>& info, int precision);

// gemm_launch.cu
bool tma_operand(GpuCtx* ctx, const float* src, long long rows, long long cols, Operand& op, cudaStream_t stream);
// choice_rows (0: M) is the row count the kernel family is chosen for: the
// row-streamed and sharded executors pass the node's full row count, so a
// node gets the same arithmetic (tensor-core or CUDA-core fp32) however its
// rows are split.
// `peers` (mxb_fused_gemm_allgather): peer copies of the output rows, handed
// to the kernel when it is one that writes them itself (`pushed` set).
struct PeerRows {
    float* const* out = nullptr;
    int n = 0;
    bool pushed = false;
};
// `batch` (run_gemm_node): count > 1 products of this shape stored back to
// back (A every M * lda, B every K * ldb, out every M * ldo floats) in one
// launch of the single-CTA kernel; FULL step s advances ep_bstride[s] floats
// per product.  The caller passes it only for shapes that launch_gemm would
// run on the tensor-core kernels.
struct BatchSpec {
    long long count = 1;
    const long long* ep_bstride = nullptr;
};
int launch_gemm(GpuCtx* ctx, const float* A, long long lda, const float* B, long long ldb, float* out, long long ldo,
                int M, int N, int K, const EpStepDev* steps, int n_steps, int precision, cudaStream_t stream,
                const float* B_small_pre = nullptr, long long row_base = 0, const Product* prod = nullptr,
                int choice_rows = 0, PeerRows* peers = nullptr, const BatchSpec* batch = nullptr);
// Whether run_gemm_node runs `batch` products of M x N x K in one launch.
bool batched_in_one_launch(int num_sms, long long batch, int M, int N, int K, int precision);
int build_epilogue(const Node* n, int M, int N, long long batch, long long bt,
                   const std::unordered_map<const Node*, const float*>& dev_of,
                   const std::unordered_map<const Node*, long long>& size_of, EpStepDev* out,
                   const Node* absorbed = nullptr);
int run_gemm_node(GpuCtx* ctx, const Node* n, const float* dA, int M, int K, const float* dB, int N, float* dOut,
                  const std::unordered_map<const Node*, const float*>& dev_of,
                  const std::unordered_map<const Node*, long long>& size_of, int precision, cudaStream_t stream,
                  long long batch = 1, const Node* absorbed = nullptr, const Product* prod = nullptr);
int finish(GpuCtx* ctx);
Tensor* new_host_tensor(const std::vector<int>& dims);

// exec_streamed.cu
RowStreamPlan plan_row_stream(const std::vector<const Node*>& order, const std::unordered_map<const Node*, int>& index,
                              const std::vector<Info>& info);
int execute_streamed(GpuCtx* ctx, const std::vector<const Node*>& order,
                     const std::unordered_map<const Node*, int>& index, std::vector<Info>& info,
                     const RowStreamPlan& plan, int chunks, float* host_dst, bool fresh_dst = false);
// Row chunks for a root of `root_bytes`: $MINIXLA_STREAM_CHUNKS, else 16 from
// 128 MiB of result (finer pipelining of the copies), else 8.
int stream_chunks(long long root_bytes);
cudaEvent_t sync_event(GpuCtx* ctx, size_t k);  // the context's k-th reusable ordering event

// exec_sharded.cu
void shard_range(long long M, int parts, int part, long long& r0, long long& r1);
const NcclApi& nccl();
ShardPlan plan_shards(const std::vector<const Node*>& order, const std::unordered_map<const Node*, int>& index,
                      const std::vector<Info>& info);
int execute_sharded(GpuCtx* ctx0, const std::vector<const Node*>& order,
                    const std::unordered_map<const Node*, int>& index, std::vector<Info>& info, const ShardPlan& plan,
                    float* host_dst);

// exec_graph.cu
int execute_graph(Node* root, GpuCtx* ctx, Tensor* dst, Tensor** result);

}  // namespace mxb
