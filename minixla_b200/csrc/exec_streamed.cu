// The row-streamed executor: uploads, kernels and downloads pipelined by row
// chunks over three streams.
#include <cuda_runtime.h>

#include <algorithm>
#include <condition_variable>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "runtime_internal.h"

namespace mxb {

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



RowStreamPlan plan_row_stream(const std::vector<const Node*>& order,
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


cudaEvent_t sync_event(GpuCtx* ctx, size_t k) {
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
int execute_streamed(GpuCtx* ctx, const std::vector<const Node*>& order,
                     const std::unordered_map<const Node*, int>& index, std::vector<Info>& info,
                     const RowStreamPlan& plan, int chunks, float* host_dst, bool fresh_dst) {
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
        // Nodes on the CUDA-core kernels (few rows, tiny problems) need no low parts.
        if (use_skinny_gemm(M, ctx->precision) || use_tiny_gemm(M, b.dims[1], b.dims[0], ctx->precision)) continue;
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
    // Result rows come back on their own host thread (with their own pinned
    // ring), chunk by chunk as soon as each chunk's kernels are enqueued, so
    // a pageable destination is filled while later chunks are still being
    // staged up: the two directions of the link and of the host copies run
    // side by side.
    const Info& root = info.back();
    const long long out_cols = root.size / M;
    std::mutex dl_mu;
    std::condition_variable dl_cv;
    int enqueued = 0;        // chunks whose computed event is recorded
    bool abandon = false;    // the main thread stopped early
    int dl_rc = MXB_OK;
    auto download_all = [&] {
        if (!cuda_ok(cudaSetDevice(ctx->device), "download thread device")) {
            dl_rc = MXB_E_CUDA;
            return;
        }
        // A fresh destination (gpu_execute's new result tensor): take its page
        // faults now, while the inputs are still going up.
        if (fresh_dst) prefault_host(ctx->stager_dl, host_dst, static_cast<size_t>(root.size) * 4);
        for (int c = 0; c < n_chunks; ++c) {
            {
                std::unique_lock<std::mutex> lk(dl_mu);
                dl_cv.wait(lk, [&] { return enqueued > c || abandon; });
                if (enqueued <= c) return;
            }
            const long long r0 = static_cast<long long>(c) * rows_per;
            const long long r1 = std::min<long long>(M, r0 + rows_per);
            if (cudaStreamWaitEvent(ds, computed[c], 0) != cudaSuccess ||
                !cuda_ok(copy_d2h(ctx->stager_dl, host_dst + r0 * out_cols, root.dev + r0 * out_cols,
                                  static_cast<size_t>((r1 - r0) * out_cols) * 4, ds),
                         "chunk download")) {
                dl_rc = MXB_E_CUDA;
                return;
            }
        }
    };
    // Without a thread (creation refused), the same downloads run after the
    // uploads and kernels are enqueued, on this thread.
    std::thread downloader;
    try {
        downloader = std::thread(download_all);
    } catch (...) {
    }
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
                                 steps, n_steps, ctx->precision, cs, b_small[i], r0, absorb[i] >= 0 ? &prod : nullptr,
                                 M);
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
            // computed[] is filled before the download thread may read it
            // (sync_event grows ctx->sync_events only on this thread).
            cudaEvent_t e = sync_event(ctx, next_event++);
            if (!e || cudaEventRecord(e, cs) != cudaSuccess) {
                rc = MXB_E_CUDA;
            } else {
                std::lock_guard<std::mutex> lk(dl_mu);
                computed[c] = e;
                enqueued = c + 1;
            }
            dl_cv.notify_one();
        }
    }
    {
        std::lock_guard<std::mutex> lk(dl_mu);
        abandon = true;
    }
    dl_cv.notify_one();
    if (downloader.joinable())
        downloader.join();
    else
        download_all();
    if (rc == MXB_OK && dl_rc != MXB_OK) {
        set_error("row streaming: a result download failed");
        rc = dl_rc;
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

int stream_chunks(long long root_bytes) {
    if (const char* c = getenv("MINIXLA_STREAM_CHUNKS")) return atoi(c);
    return root_bytes >= (128ll << 20) ? 16 : 8;
}

}  // namespace mxb
