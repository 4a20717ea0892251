// The multi-GPU executor of a gpu_ctx_create_multi context: row shards per
// device, whole-read leaves replicated over NVLink, NCCL all-gathers only
// where a later node reads an intermediate whole.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include <dlfcn.h>

#include "runtime_internal.h"

namespace mxb {

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

void shard_range(long long M, int parts, int part, long long& r0, long long& r1) {
    const long long base = M / parts, extra = M % parts;
    r0 = part * base + std::min<long long>(part, extra);
    r1 = r0 + base + (part < extra ? 1 : 0);
}


// NCCL is loaded on first use (the copy already in the process if there is
// one), so the library itself loads where NCCL is absent.
const NcclApi& nccl() {
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


ShardPlan plan_shards(const std::vector<const Node*>& order, const std::unordered_map<const Node*, int>& index,
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

// Runs fn(d) for every device d = 0 .. P-1 at the same time, on P host
// threads (d = 0 on the caller's), each with its device current; returns the
// first failure's code and carries its message over to the calling thread.
// Used for the staged host copies, whose cost is host memcpy into each
// device's pinned ring: one thread per device runs those side by side.
template <typename Fn>
static int for_each_device(int P, const std::vector<GpuCtx*>& ctxs, Fn fn) {
    std::vector<int> rc(P, MXB_OK);
    std::vector<std::string> msg(P);
    auto run = [&](int d) {
        DeviceScope scope(ctxs[d]->device);
        rc[d] = fn(d);
        if (rc[d] != MXB_OK) msg[d] = mxb_last_error();
    };
    std::vector<std::thread> threads;
    std::vector<int> inline_devices;  // devices whose thread could not be made: run here
    for (int d = 1; d < P; ++d) {
        try {
            threads.emplace_back(run, d);
        } catch (...) {
            inline_devices.push_back(d);
        }
    }
    run(0);
    for (int d : inline_devices) run(d);
    for (std::thread& t : threads) t.join();
    for (int d = 0; d < P; ++d) {
        if (rc[d] != MXB_OK) {
            if (d > 0) set_error("%s", msg[d].c_str());
            return rc[d];
        }
    }
    return MXB_OK;
}

static int nccl_check(ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return MXB_OK;
    set_error("%s: %s", what, nccl().error_string ? nccl().error_string(r) : "NCCL error");
    return MXB_E_CUDA;
}

int execute_sharded(GpuCtx* ctx0, const std::vector<const Node*>& order,
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
    // Leaves: whole leaves once to device 0, then peer copies (this thread);
    // then every device's row shards straight from the host, one host thread
    // per device.
    size_t ev_k = 0;
    for (size_t i = 0; i < n && rc == MXB_OK; ++i) {
        if (order[i]->op != OP_INPUT || borrowed[i] || !full[i]) continue;
        const float* host = order[i]->output->data;
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
    if (rc == MXB_OK) {
        rc = for_each_device(P, ctxs, [&](int d) {
            for (size_t i = 0; i < n; ++i) {
                if (order[i]->op != OP_INPUT || borrowed[i] || full[i] || !ptr[d][i]) continue;
                const long long c = cols_of(i);
                if (!cuda_ok(copy_h2d(ctxs[d]->stager, ptr[d][i], order[i]->output->data + r0[d] * c,
                                      static_cast<size_t>((r1[d] - r0[d]) * c) * 4, ctxs[d]->stream),
                             "shard upload"))
                    return MXB_E_CUDA;
            }
            return MXB_OK;
        });
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
                                 n_steps, ctx0->precision, c->stream, nullptr, r0[d], nullptr, plan.M);
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
    // Result rows from every device into the host tensor, one host thread per device.
    const size_t root_i = n - 1;
    const long long out_cols = cols_of(root_i);
    if (rc == MXB_OK) {
        rc = for_each_device(P, ctxs, [&](int d) {
            const long long m = r1[d] - r0[d];
            if (m <= 0) return MXB_OK;
            return cuda_ok(copy_d2h(ctxs[d]->stager, host_dst + r0[d] * out_cols, rows(d, root_i),
                                    static_cast<size_t>(m * out_cols) * 4, ctxs[d]->stream),
                           "shard download")
                       ? MXB_OK
                       : MXB_E_CUDA;
        });
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

}  // namespace mxb
