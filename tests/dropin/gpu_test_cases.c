/* MiniXLA's own GPU test suite (gpu_test.c), compiled unmodified against
 * libminixla_b200.so: the file is included verbatim with its main() renamed,
 * so this program can run its cases one at a time by name
 * (`gpu_test_cases <case>`), each in its own process, and report which one
 * fails instead of stopping at the first assert.
 *
 * One case is replaced: test_broadcast_bias_rejected_on_gpu (gpu_test.c:48-73)
 * asserts that both GPU entry points REFUSE a fused node whose ADD operand is
 * a [N] bias row, because the reference's PTX emitter could not broadcast it.
 * This backend runs that node (eval_fused's modulo rule, graph.c:100-105), so
 * `broadcast_bias_runs_on_gpu` builds the same graph and checks both entry
 * points against execute() instead.
 *
 * Built by oracle/Makefile (target `dropin`) with -I pointing at the
 * reference sources; links the reference's tensor.c, graph.c, optimizer.c and
 * ptx.c (emit_ptx: gpu_run_fused takes a PTX string it ignores here). */
#define main minixla_reference_gpu_test_main
#include "gpu_test.c"
#undef main

#include <string.h>

static void broadcast_bias_runs_on_gpu(void) {
    Tensor* a = create_tensor((float[]){1, 2, 3, 4, 5, 6}, (int[]){2, 3}, 2);
    Tensor* b = create_tensor((float[]){1, 2, 3, 4, 5, 6}, (int[]){3, 2}, 2);
    Tensor* bias = create_tensor((float[]){-30, -60}, (int[]){2}, 1);
    Node* root = optimize(g_relu(g_add(g_matmul(input_node(a), input_node(b)), input_node(bias))));
    assert(root->op == OP_FUSED);
    Tensor* cpu_out = execute(root);
    assert(cpu_out);
    char* ptx = emit_ptx(root);
    Tensor* via_runtime = gpu_run_fused(root, ptx);
    free(ptx);
    assert(via_runtime && approx_tensors(cpu_out, via_runtime, 1e-4f));
    GpuCtx* ctx = gpu_ctx_create();
    assert(ctx);
    Tensor* via_exec = gpu_execute(root, ctx);
    gpu_ctx_destroy(ctx);
    assert(via_exec && approx_tensors(cpu_out, via_exec, 1e-4f));
    free_tensor(via_runtime); free_tensor(via_exec);
    free_graph(root);
    free_tensor(a); free_tensor(b); free_tensor(bias);
    printf("broadcast_bias_runs_on_gpu PASS\n");
}

static const struct { const char* name; void (*run)(void); } kCases[] = {
    {"test_single_fused", test_single_fused},
    {"broadcast_bias_runs_on_gpu", broadcast_bias_runs_on_gpu},
    {"test_diamond_shared_input", test_diamond_shared_input},
    {"test_two_layer", test_two_layer},
    {"test_deep_chain", test_deep_chain},
    {"test_module_cache", test_module_cache},
    {"bench_large_matmul", bench_large_matmul},
    {"test_tensorcore_correctness", test_tensorcore_correctness},
    {"test_tensorcore_epilogue", test_tensorcore_epilogue},
};

int main(int argc, char** argv) {
    const int n = (int)(sizeof(kCases) / sizeof(kCases[0]));
    if (argc < 2) {
        for (int i = 0; i < n; ++i) printf("%s\n", kCases[i].name);
        return 0;
    }
    for (int i = 0; i < n; ++i)
        if (strcmp(argv[1], kCases[i].name) == 0) {
            kCases[i].run();
            return 0;
        }
    fprintf(stderr, "unknown case %s\n", argv[1]);
    return 64;
}
