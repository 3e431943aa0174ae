/* ref_harness.c: TEST INFRASTRUCTURE ONLY. A thin C harness around the reference's own host-side
 * implementation of the Q8_0 products: gemv_i_repack, gemv_i_thread and gemm_i_thread
 * (src/card/gemv.c:23-40, 168-181; src/card/gemm.c:271-294) over the lane-exact host model of
 * src/card/knc.h:148-298, run on the reference's thread team (src/card/team.c:90-129).
 * oracle/Makefile compiles it together with those reference sources, where they lie in the
 * read-only reference tree, into oracle/_ref/libq8ref.so; nothing of the reference is copied.
 *
 * Used by tests/golden/make_golden.py (golden vectors), tests (parity of the restatement) and
 * bench.py's CPU baseline. Every product runs with no tile chain, the path on which "y is the
 * same bits at any thread count" (src/card/gemv.h:38-41): the reference's canonical order. */
#define _GNU_SOURCE
#include <sched.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "gemm.h"
#include "gemv.h"
#include "team.h"

static struct team *g_team;
static int g_threads;

/* A team of n threads pinned to CPUs 0..n-1 (the bench's KNC CPU map does not apply on a normal
 * host). Replaces any earlier team. Returns n, or -1. */
int refh_team(int n)
{
    if (n < 1)
        n = 1;
    if (g_team && g_threads == n)
        return n;
    if (g_team) {
        team_destroy(g_team);
        g_team = NULL;
    }
    int *cpus = malloc(sizeof(int) * (size_t)n);
    if (!cpus)
        return -1;
    cpu_set_t allowed;
    int have = 0;
    if (sched_getaffinity(0, sizeof allowed, &allowed) == 0) {
        for (int c = 0; c < CPU_SETSIZE && have < n; c++)
            if (CPU_ISSET(c, &allowed))
                cpus[have++] = c;
    }
    for (int i = have; i < n; i++)
        cpus[i] = i;
    g_team = team_create(cpus, n, have >= n);
    free(cpus);
    if (!g_team)
        return -1;
    g_threads = n;
    return n;
}

/* Form I bytes of a GGUF Q8_0 matrix (rows % 16 == 0, cols % 32 == 0), repacked by the
 * reference's own gemv_i_repack. */
long refh_form_i_bytes(long rows, long cols) { return gemv_i_bytes(rows, cols); }

void refh_repack(const uint8_t *q8, long rows, long cols, void *form_i) { gemv_i_repack(q8, rows, cols, form_i); }

/* y = W x over a form I matrix, the team's whole-group split */
void refh_gemv(const void *form_i, long rows, long cols, const float *x, float *y)
{
    if (!g_team && refh_team(1) < 0)
        return;
    struct gemv_job j;
    memset(&j, 0, sizeof j);
    j.w = form_i;
    j.rows = rows;
    j.cols = cols;
    j.x = x;
    j.y = y;
    team_run(g_team, gemv_i_thread, &j);
}

/* Y [t rows] = X [t cols] W^T over a form I matrix, one pass over the weights for t tokens */
void refh_gemm(const void *form_i, long rows, long cols, const float *x, long t, float *y)
{
    if (!g_team && refh_team(1) < 0)
        return;
    struct gemm_job j;
    memset(&j, 0, sizeof j);
    j.w = form_i;
    j.rows = rows;
    j.cols = cols;
    j.t = t;
    j.x = x;
    j.x_stride = cols;
    j.y = y;
    team_run(g_team, gemm_i_thread, &j);
}
