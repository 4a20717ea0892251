// mxb_fused_gemm_noalloc: the 3xTF32 fused GEMM for callers that must not
// allocate device memory.
//
// Who needs it: code that runs where cudaMalloc / cudaFree are off limits --
// a plugin inside a host framework that owns the whole device-memory budget
// through its own allocator (a direct cudaMalloc would escape its accounting,
// or fail once the budget is reserved), and latency-critical serving loops,
// where cudaMalloc / cudaFree synchronise the device and take unbounded time.
// Such callers pass inputs and outputs they already own; the only other memory
// the computation needs -- the low parts x - rne_tf32(x) of A and B -- lives
// here in a fixed device array that every GPU loading this library holds
// until the process exits.
//
// Set-up: the first call on each device looks up the device addresses of the
// array and of an error word (cudaGetSymbolAddress, with that device current)
// and caches them; make that first call before any stream capture.  Every
// call reads the error word back and synchronises its stream before it
// returns, so a call on a stream that is being captured is refused
// (MXB_E_ARG) before anything is enqueued.  Calls share the array: calls that
// overlap on the GPU (other host threads, other streams) race on it and must
// be serialised by the caller.  Device-side waits are bounded by
// $MINIXLA_WAIT_TIMEOUT_MS (read once per process, as gpu_ctx_create reads
// it), else 5 s.
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "internal.h"

namespace mxb {

namespace {

// 16 MiB of fp32: room for the low parts of A (M x lda) and B (K x ldb).
constexpr long long kNoAllocScratchFloats = 4ll << 20;

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];
static __device__ int g_noalloc_err;

struct DeviceSlots {
    bool ready = false;
    float* scratch = nullptr;   // device address of g_noalloc_scratch
    int* err = nullptr;         // device address of g_noalloc_err
    int num_sms = 0;
};

constexpr int kMaxDevices = 64;
std::mutex g_slots_mu;
DeviceSlots g_slots[kMaxDevices];

// The bound on every device-side wait: $MINIXLA_WAIT_TIMEOUT_MS, else 5 s.
unsigned long long wait_timeout_ns() {
    static const unsigned long long ns = [] {
        unsigned long long v = 5ull * 1000 * 1000 * 1000;
        if (const char* t = getenv("MINIXLA_WAIT_TIMEOUT_MS")) {
            const long long ms = atoll(t);
            if (ms > 0) v = static_cast<unsigned long long>(ms) * 1000000ull;
        }
        return v;
    }();
    return ns;
}

// Once per device, with that device current.
int device_slots(int dev, DeviceSlots& out) {
    if (dev < 0 || dev >= kMaxDevices) {
        set_error("mxb_fused_gemm_noalloc: device %d outside the supported range", dev);
        return MXB_E_ARG;
    }
    std::lock_guard<std::mutex> lock(g_slots_mu);
    DeviceSlots& s = g_slots[dev];
    if (!s.ready) {
        int major = 0;
        cudaError_t e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
        if (e == cudaSuccess && major != 10) {
            set_error("mxb_fused_gemm_noalloc: device %d is not sm_100", dev);
            return MXB_E_UNSUPPORTED;
        }
        if (e == cudaSuccess) e = cudaGetSymbolAddress(reinterpret_cast<void**>(&s.scratch), g_noalloc_scratch);
        if (e == cudaSuccess) e = cudaGetSymbolAddress(reinterpret_cast<void**>(&s.err), g_noalloc_err);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&s.num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) {
            set_error("mxb_fused_gemm_noalloc: set-up on device %d failed: %s", dev, cudaGetErrorString(e));
            s = DeviceSlots{};
            return MXB_E_CUDA;
        }
        s.ready = true;
    }
    out = s;
    return MXB_OK;
}

}  // namespace

}  // namespace mxb

extern "C" int mxb_fused_gemm_noalloc(const float* A, long long lda, const float* B, long long ldb, float* out,
                                      long long ldo, int M, int N, int K, const mxb_ep_step* steps, int n_steps,
                                      void* stream) {
    using namespace mxb;
    if (!A || !B || !out || M < 1 || N < 1 || K < 1 || lda < K || ldb < N || ldo < N || n_steps < 0 ||
        n_steps > MXB_MAX_EPILOGUE || (n_steps > 0 && !steps)) {
        set_error("mxb_fused_gemm_noalloc: invalid arguments");
        return MXB_E_ARG;
    }
    if (lda % 4 || ldb % 4 || (reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15)) {
        set_error("mxb_fused_gemm_noalloc: A and B need 16-byte aligned bases and row pitches "
                  "(lda %% 4 == 0, ldb %% 4 == 0)");
        return MXB_E_ARG;
    }
    const long long need = static_cast<long long>(M) * lda + static_cast<long long>(K) * ldb;
    if (need > kNoAllocScratchFloats) {
        set_error("mxb_fused_gemm_noalloc: M*lda + K*ldb = %lld floats of scratch needed, the fixed array "
                  "holds %lld (16 MiB); use mxb_fused_gemm for larger problems",
                  need, kNoAllocScratchFloats);
        return MXB_E_ARG;
    }
    EpStepDev dev_steps[MXB_MAX_EPILOGUE];
    for (int i = 0; i < n_steps; ++i) {
        const mxb_ep_step& s = steps[i];
        const bool is_add = s.kind == MXB_EP_ADD_FULL || s.kind == MXB_EP_ADD_ROW || s.kind == MXB_EP_ADD_MOD;
        if (s.kind < MXB_EP_ADD_FULL || s.kind > MXB_EP_SCALE || (is_add && !s.operand) ||
            (s.kind == MXB_EP_ADD_FULL && s.ld_or_size < N) || (s.kind == MXB_EP_ADD_MOD && s.ld_or_size < 1)) {
            set_error("mxb_fused_gemm_noalloc: invalid epilogue step %d", i);
            return MXB_E_ARG;
        }
        memcpy(&dev_steps[i], &s, sizeof(s));
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        set_error("mxb_fused_gemm_noalloc: no current CUDA device");
        return MXB_E_CUDA;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaStreamCaptureStatus capturing = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &capturing) != cudaSuccess || capturing != cudaStreamCaptureStatusNone) {
        set_error("mxb_fused_gemm_noalloc: the stream is being captured (or cannot be queried); this call reads "
                  "its error word back and synchronises the stream, which a capture does not allow");
        return MXB_E_ARG;
    }
    DeviceSlots slots;
    int rc = device_slots(dev, slots);
    if (rc != MXB_OK) return rc;

    float* a_small = slots.scratch;
    float* b_small = slots.scratch + static_cast<long long>(M) * lda;  // lda % 4 == 0 keeps 16-byte alignment
    cudaError_t e = cudaMemsetAsync(slots.err, 0, sizeof(int), st);
    if (e == cudaSuccess) e = launch_split_tf32(A, M, K, lda, a_small, lda, slots.num_sms, st);
    if (e == cudaSuccess) e = launch_split_tf32(B, K, N, ldb, b_small, ldb, slots.num_sms, st);
    if (e == cudaSuccess) {
        GemmLaunch g{};
        g.A = A;
        g.lda = lda;
        g.B = B;
        g.ldb = ldb;
        g.A_small = a_small;
        g.B_small = b_small;
        g.out = out;
        g.ldo = ldo;
        g.M = M;
        g.N = N;
        g.K = K;
        g.steps = dev_steps;
        g.n_steps = n_steps;
        g.precision = GPU_PRECISION_3XTF32;
        g.err = slots.err;
        g.timeout_ns = wait_timeout_ns();
        g.num_sms = slots.num_sms;
        e = launch_fused_gemm(g, st);
    }
    int err_word = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&err_word, slots.err, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        set_error("mxb_fused_gemm_noalloc: %s", cudaGetErrorString(e));
        return MXB_E_CUDA;
    }
    if (err_word) {
        set_error("mxb_fused_gemm_noalloc: a device-side wait ran out of time (error bits 0x%x)", err_word);
        return MXB_E_TIMEOUT;
    }
    return MXB_OK;
}
