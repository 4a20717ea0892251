/* A MiniXLA C program as a user writes it: the reference's own headers and
 * graph code (tensor.c, graph.c, optimizer.c), linked against
 * libminixla_b200.so in place of gpu_exec.c / runtime.c / ptx.c.  Prints OK
 * when gpu_execute gives the answer of tests.c's fused-node case
 * (relu(A.B + C) = {0, 28, 49, 0}); exits 2 when no GPU context exists. */
#include <stdio.h>
#include "gpu_exec.h"
#include "optimizer.h"
int main(void) {
    Tensor* a = create_tensor((float[]){1, 2, 3, 4, 5, 6}, (int[]){2, 3}, 2);
    Tensor* b = create_tensor((float[]){1, 2, 3, 4, 5, 6}, (int[]){3, 2}, 2);
    Tensor* c = create_tensor((float[]){-100, 0, 0, -100}, (int[]){2, 2}, 2);
    Node* root = optimize(g_relu(g_add(g_matmul(input_node(a), input_node(b)), input_node(c))));
    GpuCtx* ctx = gpu_ctx_create();
    if (!ctx) { printf("no GPU context\n"); return 2; }
    Tensor* out = gpu_execute(root, ctx);
    int ok = out && out->data[0] == 0 && out->data[1] == 28 && out->data[2] == 49 && out->data[3] == 0;
    printf("%s\n", ok ? "OK" : "MISMATCH");
    free_tensor(out); gpu_ctx_destroy(ctx); free_graph(root);
    free_tensor(a); free_tensor(b); free_tensor(c);
    return ok ? 0 : 1;
}
