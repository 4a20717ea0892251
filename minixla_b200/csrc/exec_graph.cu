// gpu_execute's entry: picks the multi-GPU, row-streamed or one-stream
// executor; the one-stream executor schedules independent nodes over up to
// four streams.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "runtime_internal.h"

namespace mxb {

// The DAG executor behind gpu_execute / gpu_execute_into.  When `dst` is
// given the root is downloaded into it (its size must match), otherwise a
// new host tensor is returned through *result.
int execute_graph(Node* root, GpuCtx* ctx, Tensor* dst, Tensor** result) {
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

    const int chunks = stream_chunks(info.back().size * 4);
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
            const int rc = execute_streamed(ctx, order, index, info, plan, chunks, t->data, true);
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

}  // namespace mxb
