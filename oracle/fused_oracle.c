/*
 * CPU oracle for the OP_FUSED hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * This file is the checker, never the product: only tests/, the package's
 * smoke() and bench.py's CPU-baseline leg load it.  The CUDA library never
 * links or calls it, and nothing on the product path falls back to it.
 *
 * It restates MiniXLA's CPU evaluation of a fused node, eval_fused
 * (graph.c:64-115 of gouthamk16/miniXLA), for one 2-D problem:
 *
 *   for each output cell (i, j):
 *       x = 0.0f;  for k in 0..K-1:  x += A[i*K+k] * B[k*N+j]     (graph.c:96-97)
 *       for each epilogue step e in order:                          (graph.c:98-109)
 *           ADD : x += op[(i*N + j) % op_size]   (full matrix, [N] bias, or any
 *                                                 operand, by the same modulo rule)
 *           RELU: x = x > 0 ? x : 0
 *       out[i*N+j] = x                                              (graph.c:110)
 *
 * Bit-exactness with the reference: each output cell sees the same fp32
 * operations in the same order as eval_fused (one fp32 multiply rounded to
 * float, then one fp32 add, k ascending).  The loops here run i-k-j so the
 * inner loop vectorises over j, which changes nothing per cell.  The file
 * must be compiled with -ffp-contract=off so no multiply-add is fused.
 *
 * SCALE (x *= s) is an extra epilogue step of the new backend; the reference
 * has no such op (its eval_fused ignores unknown steps, graph.c:98-109), so
 * SCALE is checked only against the float64 path here.
 *
 * Pinned against: the known answers of the reference's own tests
 * (tests.c:92-107 -> {0,28,49,0}; tests.c:48-65 -> {0,0,19,4};
 * tests.c:191-220 -> {5,4,11,10}) and, bit for bit, against the reference's
 * execute() compiled from its own sources by oracle/Makefile.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

enum { ORACLE_ADD = 0, ORACLE_RELU = 1, ORACLE_SCALE = 2 };

typedef struct {
    int kind;            /* ORACLE_ADD / ORACLE_RELU / ORACLE_SCALE        */
    const float* op;     /* ADD operand, flat row-major                    */
    long long op_size;   /* its element count (the modulo of graph.c:105)  */
    float scale;         /* SCALE factor                                   */
} oracle_step;

/* Rows [r0, r1) of out = epi(A[M,K] @ B[K,N]), fp32 exactly as eval_fused.
 * A_rows points at row r0 of A (so callers can pass a row sample). */
static void fused_rows_f32(const float* A_rows, const float* B, float* out_rows,
                           long long N, long long K, long long r0, long long r1,
                           const oracle_step* steps, int n_steps, float* acc) {
    for (long long i = r0; i < r1; i++) {
        const float* a = A_rows + (i - r0) * K;
        for (long long j = 0; j < N; j++) acc[j] = 0.0f;
        for (long long k = 0; k < K; k++) {
            const float aik = a[k];
            const float* b = B + k * N;
            for (long long j = 0; j < N; j++) {
                float p = aik * b[j];
                acc[j] = acc[j] + p;
            }
        }
        float* o = out_rows + (i - r0) * N;
        for (long long j = 0; j < N; j++) {
            float x = acc[j];
            for (int e = 0; e < n_steps; e++) {
                const oracle_step* s = &steps[e];
                if (s->kind == ORACLE_ADD) {
                    x += s->op[(unsigned long long)(i * N + j) % (unsigned long long)s->op_size];
                } else if (s->kind == ORACLE_RELU) {
                    x = x > 0 ? x : 0;
                } else if (s->kind == ORACLE_SCALE) {
                    x = x * s->scale;
                }
            }
            o[j] = x;
        }
    }
}

/* Same rows in float64 (products and sums in double, epilogue in double),
 * used to measure how far the fp32 oracle itself is from the exact value. */
static void fused_rows_f64(const float* A_rows, const float* B, double* out_rows,
                           long long N, long long K, long long r0, long long r1,
                           const oracle_step* steps, int n_steps, double* acc) {
    for (long long i = r0; i < r1; i++) {
        const float* a = A_rows + (i - r0) * K;
        for (long long j = 0; j < N; j++) acc[j] = 0.0;
        for (long long k = 0; k < K; k++) {
            const double aik = a[k];
            const float* b = B + k * N;
            for (long long j = 0; j < N; j++) acc[j] += aik * (double)b[j];
        }
        double* o = out_rows + (i - r0) * N;
        for (long long j = 0; j < N; j++) {
            double x = acc[j];
            for (int e = 0; e < n_steps; e++) {
                const oracle_step* s = &steps[e];
                if (s->kind == ORACLE_ADD) {
                    x += (double)s->op[(unsigned long long)(i * N + j) % (unsigned long long)s->op_size];
                } else if (s->kind == ORACLE_RELU) {
                    x = x > 0 ? x : 0;
                } else if (s->kind == ORACLE_SCALE) {
                    x = x * (double)s->scale;
                }
            }
            o[j] = x;
        }
    }
}

typedef struct {
    const float* A; const float* B; void* out;
    long long N, K;
    const long long* rows; long long n_rows;     /* explicit row list    */
    long long begin, end;                        /* slice of that list   */
    const oracle_step* steps; int n_steps;
    int f64; int ok;
} worker_arg;

static void* worker(void* p) {
    worker_arg* w = (worker_arg*)p;
    void* acc = malloc((size_t)w->N * (w->f64 ? sizeof(double) : sizeof(float)));
    if (!acc) { w->ok = 0; return NULL; }
    for (long long t = w->begin; t < w->end; t++) {
        long long i = w->rows[t];
        if (w->f64)
            fused_rows_f64(w->A + i * w->K, w->B, (double*)w->out + t * w->N,
                           w->N, w->K, i, i + 1, w->steps, w->n_steps, (double*)acc);
        else
            fused_rows_f32(w->A + i * w->K, w->B, (float*)w->out + t * w->N,
                           w->N, w->K, i, i + 1, w->steps, w->n_steps, (float*)acc);
    }
    free(acc);
    w->ok = 1;
    return NULL;
}

/*
 * Evaluate the listed output rows of epi(A @ B): out is [n_rows, N] (float or
 * double, per f64), row t of out holding output row rows[t].  Rows are
 * independent in eval_fused (graph.c:94-112), so a row sample is exact for
 * the rows it holds.  Work is split over n_threads host threads.
 * Returns 0 on success, -1 on allocation or thread failure.
 */
int oracle_fused_rows(const float* A, const float* B, void* out,
                      long long M, long long N, long long K,
                      const long long* rows, long long n_rows,
                      const oracle_step* steps, int n_steps,
                      int f64, int n_threads) {
    (void)M;
    if (n_threads < 1) n_threads = 1;
    if (n_threads > n_rows) n_threads = (int)(n_rows > 0 ? n_rows : 1);
    pthread_t* th = (pthread_t*)calloc((size_t)n_threads, sizeof(pthread_t));
    worker_arg* args = (worker_arg*)calloc((size_t)n_threads, sizeof(worker_arg));
    if (!th || !args) { free(th); free(args); return -1; }
    int rc = 0, started = 0;
    for (int t = 0; t < n_threads; t++) {
        args[t] = (worker_arg){A, B, out, N, K, rows, n_rows,
                               n_rows * t / n_threads, n_rows * (t + 1) / n_threads,
                               steps, n_steps, f64, 0};
        if (pthread_create(&th[t], NULL, worker, &args[t]) != 0) { rc = -1; break; }
        started++;
    }
    for (int t = 0; t < started; t++) {
        pthread_join(th[t], NULL);
        if (!args[t].ok) rc = -1;
    }
    free(th); free(args);
    return rc;
}

/* Whole-matrix convenience wrapper: every row, fp32, n_threads threads. */
int oracle_fused(const float* A, const float* B, float* out,
                 long long M, long long N, long long K,
                 const oracle_step* steps, int n_steps, int n_threads) {
    long long* rows = (long long*)malloc((size_t)(M > 0 ? M : 1) * sizeof(long long));
    if (!rows) return -1;
    for (long long i = 0; i < M; i++) rows[i] = i;
    int rc = oracle_fused_rows(A, B, out, M, N, K, rows, M, steps, n_steps, 0, n_threads);
    free(rows);
    return rc;
}

/*
 * Standalone element-wise nodes, restating tensor.c:
 *   tensor_add (tensor.c:64-86): out[i] = a[i] + b[i % b_size]
 *   relu       (tensor.c:110-120): out[i] = x[i] > 0 ? x[i] : 0
 */
void oracle_add(const float* a, long long a_size, const float* b, long long b_size, float* out) {
    for (long long i = 0; i < a_size; i++) out[i] = a[i] + b[i % b_size];
}

void oracle_relu(const float* x, long long n, float* out) {
    for (long long i = 0; i < n; i++) out[i] = x[i] > 0 ? x[i] : 0;
}
