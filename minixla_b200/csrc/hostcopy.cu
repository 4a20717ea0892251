// Host <-> device copies for pageable host memory.
//
// MiniXLA's tensors live in malloc'd (pageable) host memory (create_tensor,
// tensor.c:8-53).  The driver copies such memory through its own small
// pinned bounce buffer, one piece after another, at about 10-12 GB/s on the
// B200 hosts -- a fifth of what PCIe 5 x16 moves from pinned memory.  Here a
// context keeps a ring of pinned slots; a few host threads fill a slot with
// memcpy while the DMA engine drains the previous one, so the copy runs at
// the lower of the parallel memcpy rate and the link rate.  Pinned (or
// registered) host memory and small copies go straight to cudaMemcpyAsync.
#include <cuda_runtime.h>

#include <algorithm>
#include <condition_variable>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "internal.h"

namespace mxb {

namespace {

constexpr size_t kStageMinBytes = 2u << 20;  // smaller copies: the driver's own path

// A small pool of host threads that split one memcpy between them (one
// thread moves about 10 GB/s).  One copy at a time; the caller takes part 0.
// Each Stager owns one, so uploads and downloads staged at the same time (on
// two host threads) do not queue behind each other.
class CopyThreads {
  public:
    CopyThreads() = default;
    // Starts the helpers (once): half the cores, at most seven, even though
    // an upload ring and a download ring may both run (8192^3 through
    // gpu_execute on 16 cores: 25.5 ms a step with seven helpers per ring
    // against 27.8 ms with four; slots of 16 or 32 MiB were slower);
    // $MINIXLA_STAGE_THREADS (0..15) sets the number of helpers instead.
    void start() {
        if (started_) return;
        started_ = true;
        const unsigned hw = std::thread::hardware_concurrency();
        unsigned n = hw >= 4 ? std::min(7u, hw / 2) : 0;
        if (const char* v = getenv("MINIXLA_STAGE_THREADS")) {
            const int k = atoi(v);
            if (k >= 0 && k <= 15) n = static_cast<unsigned>(k);
        }
        for (unsigned i = 0; i < n; ++i) workers_.emplace_back([this, i] { run(i + 1); });
    }
    CopyThreads(const CopyThreads&) = delete;
    CopyThreads& operator=(const CopyThreads&) = delete;

    void copy(void* dst, const void* src, size_t bytes) { split(static_cast<char*>(dst), static_cast<const char*>(src), bytes); }

    // Writes one byte per 4 KiB page of fresh memory, so the page faults
    // (and the kernel's zeroing of the pages) are taken by several threads
    // ahead of the copies into it.
    void touch(void* dst, size_t bytes) { split(static_cast<char*>(dst), nullptr, bytes); }

    ~CopyThreads() {
        {
            std::lock_guard<std::mutex> lk(mu_);
            stop_ = true;
            ++gen_;
        }
        cv_.notify_all();
        for (std::thread& t : workers_) t.join();
    }

  private:
    static void part_job(char* d, const char* s, size_t n) {
        if (s) {
            memcpy(d, s, n);
        } else {
            for (size_t off = 0; off < n; off += 4096) reinterpret_cast<volatile char*>(d)[off] = 0;
        }
    }

    // Splits one job (a copy, or a touch when src is null) between the caller and the helpers.
    void split(char* dst, const char* src, size_t bytes) {
        if (workers_.empty() || bytes < (1u << 20)) {
            part_job(dst, src, bytes);
            return;
        }
        std::lock_guard<std::mutex> job(job_mu_);
        const size_t parts = workers_.size() + 1;
        const size_t per = ((bytes + parts - 1) / parts + 4095) & ~static_cast<size_t>(4095);
        {
            std::lock_guard<std::mutex> lk(mu_);
            dst_ = dst;
            src_ = src;
            bytes_ = bytes;
            per_ = per;
            pending_ = workers_.size();
            ++gen_;
        }
        cv_.notify_all();
        part_job(dst, src, std::min(per, bytes));
        std::unique_lock<std::mutex> lk(mu_);
        done_.wait(lk, [&] { return pending_ == 0; });
    }

    void run(size_t part) {
        uint64_t seen = 0;
        for (;;) {
            char* d;
            const char* s;
            size_t b, per;
            {
                std::unique_lock<std::mutex> lk(mu_);
                cv_.wait(lk, [&] { return gen_ != seen; });
                seen = gen_;
                if (stop_) return;
                d = dst_;
                s = src_;
                b = bytes_;
                per = per_;
            }
            const size_t off = part * per;
            if (off < b) part_job(d + off, s ? s + off : nullptr, std::min(per, b - off));
            std::lock_guard<std::mutex> lk(mu_);
            if (--pending_ == 0) done_.notify_one();
        }
    }

    std::vector<std::thread> workers_;
    std::mutex job_mu_, mu_;
    std::condition_variable cv_, done_;
    char* dst_ = nullptr;
    const char* src_ = nullptr;
    size_t bytes_ = 0, per_ = 0, pending_ = 0;
    uint64_t gen_ = 0;
    bool stop_ = false;
    bool started_ = false;
};

bool host_pinned(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

bool staging_enabled() {
    const char* v = getenv("MINIXLA_STAGED_COPY");
    return !(v && v[0] == '0');
}

}  // namespace

// A ring of pinned slots owned by one context; each slot carries the event
// of the last copy that used it.
class Stager {
  public:
    static constexpr int kSlots = 4;
    // Slot size: 8 MiB, or $MINIXLA_STAGE_SLOT_MB (1..64) read when the ring
    // is made; bigger slots mean fewer hand-offs to the copy threads per
    // copy, at kSlots times the pinned memory.
    size_t slot_bytes_ = 8u << 20;

    ~Stager() {
        for (cudaEvent_t& e : ev_) {
            if (e) {
                cudaEventSynchronize(e);
                cudaEventDestroy(e);
            }
        }
        if (buf_) cudaFreeHost(buf_);
    }

    bool ready() {
        if (buf_) return true;
        if (failed_) return false;
        if (const char* v = getenv("MINIXLA_STAGE_SLOT_MB")) {
            const int mb = atoi(v);
            if (mb >= 1 && mb <= 64) slot_bytes_ = static_cast<size_t>(mb) << 20;
        }
        void* b = nullptr;
        if (cudaHostAlloc(&b, kSlots * slot_bytes_, cudaHostAllocDefault) != cudaSuccess) {
            cudaGetLastError();
            failed_ = true;
            return false;
        }
        for (cudaEvent_t& e : ev_) {
            if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) {
                cudaGetLastError();
                failed_ = true;
                cudaFreeHost(b);
                return false;
            }
        }
        buf_ = static_cast<char*>(b);
        copier_.start();
        return true;
    }

    cudaError_t to_device(char* dst, const char* src, size_t bytes, cudaStream_t st) {
        for (size_t off = 0; off < bytes; off += slot_bytes_) {
            const size_t n = std::min(slot_bytes_, bytes - off);
            const int s = take_slot();
            cudaError_t e = cudaEventSynchronize(ev_[s]);  // the slot's previous copy has left it
            if (e != cudaSuccess) return e;
            copier_.copy(slot(s), src + off, n);
            if ((e = cudaMemcpyAsync(dst + off, slot(s), n, cudaMemcpyHostToDevice, st)) != cudaSuccess) return e;
            if ((e = cudaEventRecord(ev_[s], st)) != cudaSuccess) return e;
        }
        return cudaSuccess;
    }

    // Faults in fresh pageable memory that downloads will fill (see touch).
    void prefault(char* dst, size_t bytes) {
        if (ready()) copier_.touch(dst, bytes);
    }

    // Returns when the data is in `dst` (as a copy to pageable memory does).
    cudaError_t to_host(char* dst, const char* src, size_t bytes, cudaStream_t st) {
        const size_t pieces = (bytes + slot_bytes_ - 1) / slot_bytes_;
        std::vector<int> slot_of(pieces, -1);
        auto issue = [&](size_t i) -> cudaError_t {
            const size_t off = i * slot_bytes_, n = std::min(slot_bytes_, bytes - off);
            const int s = take_slot();
            slot_of[i] = s;
            cudaError_t e = cudaEventSynchronize(ev_[s]);
            if (e != cudaSuccess) return e;
            if ((e = cudaMemcpyAsync(slot(s), src + off, n, cudaMemcpyDeviceToHost, st)) != cudaSuccess) return e;
            return cudaEventRecord(ev_[s], st);
        };
        size_t issued = 0;
        cudaError_t e = cudaSuccess;
        for (; issued < pieces && issued < static_cast<size_t>(kSlots) && e == cudaSuccess; ++issued) e = issue(issued);
        for (size_t i = 0; i < pieces && e == cudaSuccess; ++i) {
            const int s = slot_of[i];
            if ((e = cudaEventSynchronize(ev_[s])) != cudaSuccess) break;
            const size_t off = i * slot_bytes_;
            copier_.copy(dst + off, slot(s), std::min(slot_bytes_, bytes - off));
            if (issued < pieces) e = issue(issued++);  // reuses the slot just emptied
        }
        return e;
    }

  private:
    char* slot(int s) { return buf_ + static_cast<size_t>(s) * slot_bytes_; }
    int take_slot() {
        const int s = next_;
        next_ = (next_ + 1) % kSlots;
        return s;
    }

    char* buf_ = nullptr;
    cudaEvent_t ev_[kSlots] = {};
    int next_ = 0;
    bool failed_ = false;
    CopyThreads copier_;
};

Stager* stager_create() { return new (std::nothrow) Stager(); }
void stager_destroy(Stager* s) { delete s; }

cudaError_t copy_h2d(Stager* s, void* dst, const void* src, size_t bytes, cudaStream_t st) {
    if (!s || bytes < kStageMinBytes || !staging_enabled() || host_pinned(src) || !s->ready())
        return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, st);
    return s->to_device(static_cast<char*>(dst), static_cast<const char*>(src), bytes, st);
}

void prefault_host(Stager* s, void* dst, size_t bytes) {
    if (s && bytes >= kStageMinBytes && staging_enabled() && !host_pinned(dst)) s->prefault(static_cast<char*>(dst), bytes);
}

cudaError_t copy_d2h(Stager* s, void* dst, const void* src, size_t bytes, cudaStream_t st) {
    if (!s || bytes < kStageMinBytes || !staging_enabled() || host_pinned(dst) || !s->ready())
        return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, st);
    return s->to_host(static_cast<char*>(dst), static_cast<const char*>(src), bytes, st);
}

}  // namespace mxb
