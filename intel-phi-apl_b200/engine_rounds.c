/* engine_rounds.c: a sequence of product rounds run the way the reference engine's generated code
 * runs them, in C against the C ABI of include/rt_b200.h (librt_b200.so). It is the caller's side
 * of the boundary, not part of the library: bench.py times the end-to-end decode step through it,
 * so the measurement includes the C ABI calls and host<->device crossings of an engine and nothing
 * of Python's.
 *
 * A round, as src/apl/compiler/em.apl:1014-1046 emits it: queue the round's product(s)
 * (rt_gemv_q / rt_gemm_q / rt_gemm_silu_q, em.apl:601-617), rt_gemv_open before the wait for the
 * host, then x crosses the link (here rt_b200_pull from host memory: link_pull,
 * src/card/link.c:86-118), rt_gemv_go runs the round, and y crosses back (rt_b200_push:
 * link_push), which returns once y is on the host, with the round's error status. */
#include <stddef.h>

#include "rt_b200.h"

struct eng_round {
    int kind;  /* 0: a product of t tokens (rt_gemv_q at t = 1, else rt_gemm_q); 1: a SwiGLU pair */
    int open;  /* 1: rt_gemv_open before x is pulled (the round's weights stream meanwhile) */
    const void *w, *w2;
    long rows, cols, t;
    float *x_dev;
    const float *x_host;
    size_t x_bytes;
    float *y_dev;
    float *y_host;
    size_t y_bytes;
};

/* Runs rounds r[0..n) `steps` times in order; 0, or the first error code a push returned. */
int eng_run_rounds(struct rt *R, const struct eng_round *r, int n, int steps)
{
    for (int s = 0; s < steps; s++)
        for (int i = 0; i < n; i++) {
            const struct eng_round *q = &r[i];
            if (q->kind == 1)
                rt_gemm_silu_q(R, q->w, q->w2, q->rows, q->cols, q->x_dev, q->t, q->y_dev);
            else if (q->t == 1)
                rt_gemv_q(R, q->w, q->rows, q->cols, q->x_dev, q->y_dev);
            else
                rt_gemm_q(R, q->w, q->rows, q->cols, q->x_dev, q->t, q->y_dev);
            if (q->open)
                rt_gemv_open(R);
            int rc = rt_b200_pull(R, q->x_dev, q->x_host, q->x_bytes);
            if (rc)
                return rc;
            rt_gemv_go(R);
            rc = rt_b200_push(R, q->y_host, q->y_dev, q->y_bytes);
            if (rc)
                return rc;
        }
    return 0;
}
