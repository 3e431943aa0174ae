/* prims_oracle.c: TEST INFRASTRUCTURE ONLY. A CPU restatement of the reference's host-half
 * primitives next to the weight products (Lasimeri/Intel-Phi-APL, src/host/rt_host.c:128-279):
 * the inner products over an attention head's history and the delta rule's state products, in
 * the reference's rounding order. Used by tests/ and bench.py's CPU leg as the checker only.
 *
 * The order, from the reference's AVX2 code:
 *   - a dot product runs 8 lanes: lane j keeps acc_j = fma(row[k+j], v[k+j], acc_j) for
 *     k = 0, 8, 16, ... (c a multiple of 8), from +0; the lanes are then summed as
 *     ((l0+l4) + (l2+l6)) + ((l1+l5) + (l3+l7)) (hsum8, src/host/vec8.h:49-55);
 *   - rt_ip21_kv (rt_host.c:135-162): z[h*t + s] = dot(kv[s][l[h]][:], b[h][:]), kv as
 *     [t][n1][c];
 *   - rt_ip12_kv (rt_host.c:164-189): z[h][k] = fma(a[h][s], kv[s][l[h]][k], z[h][k]) over
 *     s = 0..t-1 in order, from +0;
 *   - rt_ip21 (rt_host.c:200-247): z[h][i] = dot(a[h][i][:], b[h][:]) (the 8-row groups and
 *     the tail rows use the same per-row lanes);
 *   - rt_scale_outer (rt_host.c:261-279): z[i][q] = fma(g, s[i][q], a[i] * b[q]), the product
 *     rounded first. */
#include <math.h>

#include "q8_oracle.h"

static float hsum8(const float l[8])
{
    const float s0 = l[0] + l[4], s1 = l[1] + l[5], s2 = l[2] + l[6], s3 = l[3] + l[7];
    return (s0 + s2) + (s1 + s3);
}

static float dot8(const float *row, const float *v, long c)
{
    float l[8] = {0};
    for (long k = 0; k < c; k += 8)
        for (int j = 0; j < 8; j++)
            l[j] = fmaf(row[k + j], v[k + j], l[j]);
    return hsum8(l);
}

void q8o_ip21_kv(float *z, const float *kv, long n1, long c, const long *l, long h, long t, const float *b)
{
    for (long i = 0; i < h * t; i++) {
        const long hh = i / t, s = i % t;
        z[i] = dot8(kv + s * n1 * c + l[hh] * c, b + hh * c, c);
    }
}

void q8o_ip12_kv(float *z, const float *a, const float *kv, long n1, long c, const long *l, long h, long t)
{
    for (long hh = 0; hh < h; hh++) {
        float *zh = z + hh * c;
        for (long k = 0; k < c; k++)
            zh[k] = 0.0f;
        for (long s = 0; s < t; s++) {
            const float w = a[hh * t + s], *row = kv + s * n1 * c + l[hh] * c;
            for (long k = 0; k < c; k++)
                zh[k] = fmaf(w, row[k], zh[k]);
        }
    }
}

void q8o_ip21(float *z, const float *a, long h, long r, long c, const float *b)
{
    for (long hh = 0; hh < h; hh++)
        for (long i = 0; i < r; i++)
            z[hh * r + i] = dot8(a + (hh * r + i) * c, b + hh * c, c);
}

void q8o_scale_outer(float *z, const float *s, float g, const float *a, const float *b, long m, long k)
{
    for (long i = 0; i < m; i++)
        for (long q = 0; q < k; q++) {
            const float p = a[i] * b[q];
            z[i * k + q] = fmaf(g, s[i * k + q], p);
        }
}
