// Graph analysis for the executors: post-order, shapes and last uses,
// resident leaves, and which bare matmuls are absorbed into their consumer.
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

// ---------------------------------------------------------------- graph analysis


// Device copy of a resident leaf on device `d` of `ctx` (0 = ctx itself,
// then its peers), or nullptr when the tensor is not resident or its data
// pointer / size changed since it was kept.
float* resident_copy(const GpuCtx* ctx, const Node* n, size_t d) {
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
std::vector<const Node*> topo_order(const Node* root) {
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
bool infer_shapes(const std::vector<const Node*>& order,
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
bool dual_kernel_enabled() {
    const char* v = getenv("MINIXLA_DUAL_GEMM");
    return !(v && v[0] == '0');
}
//
// optimize() never fuses a bare matmul (optimizer.c:94-132), so a matmul that
// feeds a fused node's ADD step stays a node of its own and eval_fused adds
// its stored result (graph.c:98-105) -- the 3-layer MLP's F2 = relu(h W2 + b2) +
// h W2'.  When that fused node is the matmul's only reader and both products
// share the left operand, they run in one kernel (the pair kernels' DUAL
// forms, TF32 and 3xTF32): A is staged once for both and the matmul's value
// never goes to HBM.  Conditions: the matmul is 2-D, not the root, read once
// (by one ADD step), has the fused node's A node as its A, and is shaped like
// the fused node's 2-D output with more than 16 rows; the row pitches are
// multiples of 4 (no padding copies).  launch_gemm still runs the two
// products as two launches where the one-kernel form does not apply.
// Returns, per node, the index of the matmul it absorbs (-1 for none).
std::vector<int> plan_products(const std::vector<const Node*>& order,
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

}  // namespace mxb
