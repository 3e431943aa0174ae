// host_prims.cu: the primitives that sit between a decode step's weight products where the
// reference's placement gives them to its host worker (src/host/rt_host.c:128-279): the inner
// products over an attention head's history (rt_ip21_kv, rt_ip12_kv), the delta rule's state
// products (rt_ip21) and its fused state update (rt_scale_outer). Each keeps the reference's
// rounding order exactly:
//   - a dot product is 8 lanes of fma chains (lane j takes columns j, j+8, j+16, ... from +0),
//     summed as ((l0+l4) + (l2+l6)) + ((l1+l5) + (l3+l7)) (the AVX2 hsum8, src/host/vec8.h:49-55).
//     Here 8 threads make one output, one lane each, and combine by shuffles in that order;
//   - rt_ip12_kv's z[h][k] is one fma chain over the history in order (rt_host.c:164-180): it
//     cannot be split, so each thread keeps one chain per query head it serves while the key
//     slice streams through shared memory, shared by the query heads of one kv head;
//   - rt_scale_outer is z = fma(g, s, a*b) with the product rounded first (rt_host.c:261-279).
#include "q8_kernels.h"
#include "q8_ptx.cuh"

namespace q8 {
namespace {

// ---------------------------------------------------------------- dot products (ip21, ip21_kv)
// Thread 8*o + j holds lane j of output o.
__device__ __forceinline__ float lanes_sum(float l) {
    // each 8-thread group is 8-aligned in its warp: xor 4, then 2, then 1 stays inside it
    const float s = l + __shfl_xor_sync(0xffffffffu, l, 4);  // l0+l4 .. l3+l7 (and mirrored)
    const float u = s + __shfl_xor_sync(0xffffffffu, s, 2);  // (l0+l4)+(l2+l6), (l1+l5)+(l3+l7)
    return u + __shfl_xor_sync(0xffffffffu, u, 1);           // their sum
}

template <bool KV>
__global__ void __launch_bounds__(256) dot8_kernel(float *z, const float *a, const float *b, long long n_out, long long per_h,
                                                   long long c, long long n1, PrimHeads heads) {
    const long long g = (long long)blockIdx.x * (blockDim.x / 8) + threadIdx.x / 8;
    const int j = threadIdx.x % 8;
    const bool live = g < n_out;
    const long long o = live ? g : 0;
    const long long hh = o / per_h, i = o - hh * per_h;
    // ip21: row o of a, b's row hh; ip21_kv: history row i of kv head l[hh], b's row hh
    const float *row = KV ? a + (i * n1 + heads.l[hh]) * c : a + o * c;
    const float *v = b + hh * c;
    float acc = 0.0f;
    if (live) {
        long long k = j;
#pragma unroll 4
        for (; k < c; k += 8)
            acc = __fmaf_rn(__ldg(row + k), __ldg(v + k), acc);
    }
    const float r = lanes_sum(acc);
    if (live && j == 0)
        z[o] = r;
}

// One thread per output, the 8 lanes in registers, 16-byte loads: for calls with outputs enough
// to fill the GPU this way (more loads in flight per thread than one lane per thread gives).
template <bool KV>
__global__ void __launch_bounds__(256) dot8_wide_kernel(float *z, const float *a, const float *b, long long n_out,
                                                        long long per_h, long long c, long long n1, PrimHeads heads) {
    const long long o = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (o >= n_out)
        return;
    const long long hh = o / per_h, i = o - hh * per_h;
    const float4 *row = reinterpret_cast<const float4 *>(KV ? a + (i * n1 + heads.l[hh]) * c : a + o * c);
    const float4 *v = reinterpret_cast<const float4 *>(b + hh * c);
    float l[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (long long k = 0; k < c / 4; k += 2) {
        const float4 r0 = __ldg(row + k), r1 = __ldg(row + k + 1), v0 = __ldg(v + k), v1 = __ldg(v + k + 1);
        l[0] = __fmaf_rn(r0.x, v0.x, l[0]);
        l[1] = __fmaf_rn(r0.y, v0.y, l[1]);
        l[2] = __fmaf_rn(r0.z, v0.z, l[2]);
        l[3] = __fmaf_rn(r0.w, v0.w, l[3]);
        l[4] = __fmaf_rn(r1.x, v1.x, l[4]);
        l[5] = __fmaf_rn(r1.y, v1.y, l[5]);
        l[6] = __fmaf_rn(r1.z, v1.z, l[6]);
        l[7] = __fmaf_rn(r1.w, v1.w, l[7]);
    }
    z[o] = __fadd_rn(__fadd_rn(__fadd_rn(l[0], l[4]), __fadd_rn(l[2], l[6])), __fadd_rn(__fadd_rn(l[1], l[5]), __fadd_rn(l[3], l[7])));
}

// Outputs from which one thread per output fills the GPU (148 SMs x 256 threads x 2). Below it
// the lane-per-thread form wins: 65,536 outputs over a 16 MB history took 12.8 us that way
// against 21.1 us one thread per output.
constexpr long long DOT_WIDE_MIN = 148ll * 256 * 2;

// ---------------------------------------------------------------- ip12_kv
// A CTA: one kv head's group of query heads (one warp each) and a 32-column slice of c. The
// slice of every history row, [t][32] floats, streams through a ring of SLOTS stages of ROWS rows
// (cp.async, 16 bytes per thread and copy); each thread keeps z[h][k] for its head and column as
// one fma chain over the rows in order.
// 768 history rows in flight (6 stages of 128): at one row every few cycles per chain, enough to
// cover DRAM latency (4 stages of 64 rows measured 56 us on a 4096-row history, 6 of 128: below).
constexpr int IP12_ROWS = 128, IP12_SLOTS = 6, IP12_K = 32;
__host__ __device__ constexpr size_t ip12_smem(int nh) { return size_t(IP12_SLOTS) * IP12_ROWS * (IP12_K + nh) * 4; }

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, bool ok) {
    const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    const int n = ok ? 16 : 0; // (a zero-size copy fills zeros: rows past t, columns past c)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n) : "memory");
}

__global__ void __launch_bounds__(32 * MAX_PRIM_GROUP) ip12_kv_kernel(float *z, const float *a, const float *kv,
                                                                      long long n1, long long c, long long t,
                                                                      PrimGroups groups) {
    // dynamic: [SLOTS][ROWS][K] of history, then [SLOTS][nmax][ROWS] of a (nmax: the launch's
    // largest group, blockDim.x / 32)
    extern __shared__ __align__(16) float dyn[];
    float(*ring)[IP12_ROWS][IP12_K] = reinterpret_cast<float(*)[IP12_ROWS][IP12_K]>(dyn);
    const int nmax = blockDim.x / 32;
    float *wbase = dyn + size_t(IP12_SLOTS) * IP12_ROWS * IP12_K;
    const int gi = blockIdx.y, warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int first = groups.first[gi], nh = groups.first[gi + 1] - first;
    const long long kvh = groups.kv[gi];
    const long long k0 = (long long)blockIdx.x * IP12_K;
    // stage s: rows [s*ROWS, +ROWS) of the slice (8 copies of 16 bytes per row) and the same
    // rows of a for each head of the group (16 copies of 16 bytes per head; a's rows are 4-byte
    // aligned only, so a is copied 4 bytes at a time unless t is a multiple of 4 and a 16-aligned)
    const bool a16 = (t % 4) == 0 && (reinterpret_cast<uintptr_t>(a) & 15) == 0;
    auto issue = [&](long long stage) {
        float(*slot)[IP12_K] = ring[stage % IP12_SLOTS];
        for (int e = threadIdx.x; e < IP12_ROWS * 8; e += blockDim.x) {
            const int rr = e / 8, q = e % 8;
            const long long row = stage * IP12_ROWS + rr, col = k0 + 4 * q;
            const bool ok = row < t && col < c;
            cp_async16(&slot[rr][4 * q], ok ? kv + (row * n1 + kvh) * c + col : kv, ok);
        }
        float(*ws)[IP12_ROWS] = reinterpret_cast<float(*)[IP12_ROWS]>(wbase + size_t(stage % IP12_SLOTS) * nmax * IP12_ROWS);
        const long long r0 = stage * IP12_ROWS;
        if (a16) {
            for (int e = threadIdx.x; e < nh * (IP12_ROWS / 4); e += blockDim.x) {
                const int hi = e / (IP12_ROWS / 4), q = e % (IP12_ROWS / 4);
                const long long row = r0 + 4 * q;
                const bool ok = row < t;
                cp_async16(&ws[hi][4 * q], ok ? a + (long long)groups.head[first + hi] * t + row : a, ok);
            }
        } else {
            for (int e = threadIdx.x; e < nh * IP12_ROWS; e += blockDim.x) {
                const int hi = e / IP12_ROWS, q = e % IP12_ROWS;
                const long long row = r0 + q;
                ws[hi][q] = row < t ? __ldg(a + (long long)groups.head[first + hi] * t + row) : 0.0f;
            }
        }
    };
    const long long nstages = (t + IP12_ROWS - 1) / IP12_ROWS;
    for (int s = 0; s < IP12_SLOTS - 1; ++s) {
        if (s < nstages)
            issue(s);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    const bool mine = warp < nh && k0 + lane < c;
    const long long hh = warp < nh ? groups.head[first + warp] : 0;
    float acc = 0.0f;
    for (long long st = 0; st < nstages; ++st) {
        asm volatile("cp.async.wait_group %0;" ::"n"(IP12_SLOTS - 2) : "memory");
        __syncthreads(); // stage st landed for every thread; slot (st - 1) % SLOTS is free again
        if (st + IP12_SLOTS - 1 < nstages)
            issue(st + IP12_SLOTS - 1);
        asm volatile("cp.async.commit_group;" ::: "memory");
        const float(*slot)[IP12_K] = ring[st % IP12_SLOTS];
        const float *ws = wbase + (size_t(st % IP12_SLOTS) * nmax + (warp < nh ? warp : 0)) * IP12_ROWS;
        const long long r0 = st * IP12_ROWS;
        const int nr = int(t - r0 < IP12_ROWS ? t - r0 : IP12_ROWS);
        if (mine) {
            int rr = 0;
            for (; rr + 16 <= nr; rr += 16) { // the operands of 16 steps first, then the chain
                float w[16], x[16];
#pragma unroll
                for (int q = 0; q < 16; ++q) {
                    w[q] = ws[rr + q];
                    x[q] = slot[rr + q][lane];
                }
#pragma unroll
                for (int q = 0; q < 16; ++q)
                    acc = __fmaf_rn(w[q], x[q], acc);
            }
            for (; rr < nr; ++rr)
                acc = __fmaf_rn(ws[rr], slot[rr][lane], acc);
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    if (mine)
        z[hh * c + k0 + lane] = acc;
}

// ---------------------------------------------------------------- scale_outer
__global__ void scale_outer_kernel(float *z, const float *s, float g, const float *a, const float *b, long long m,
                                   long long k) {
    const long long n = m * k;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
        const long long i = e / k, q = e - i * k;
        z[e] = __fmaf_rn(g, __ldg(s + e), __fmul_rn(__ldg(a + i), __ldg(b + q)));
    }
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

unsigned grid_of(long long threads, int block) {
    long long g = (threads + block - 1) / block;
    return unsigned(g < 1 ? 1 : (g > (1ll << 30) ? (1ll << 30) : g));
}

} // namespace

cudaError_t launch_ip21(float *z, const float *a, long long h, long long r, long long c, const float *b,
                        cudaStream_t stream) {
    const long long n = h * r;
    PrimHeads none = {};
    if (n >= DOT_WIDE_MIN && aligned16(a) && aligned16(b))
        dot8_wide_kernel<false><<<grid_of(n, 256), 256, 0, stream>>>(z, a, b, n, r, c, 0, none);
    else
        dot8_kernel<false><<<grid_of(n * 8, 256), 256, 0, stream>>>(z, a, b, n, r, c, 0, none);
    return cudaGetLastError();
}

cudaError_t launch_ip21_kv(float *z, const float *kv, long long n1, long long c, const PrimHeads &heads, long long h,
                           long long t, const float *b, cudaStream_t stream) {
    const long long n = h * t;
    if (n >= DOT_WIDE_MIN && aligned16(kv) && aligned16(b))
        dot8_wide_kernel<true><<<grid_of(n, 256), 256, 0, stream>>>(z, kv, b, n, t, c, n1, heads);
    else
        dot8_kernel<true><<<grid_of(n * 8, 256), 256, 0, stream>>>(z, kv, b, n, t, c, n1, heads);
    return cudaGetLastError();
}

cudaError_t launch_ip12_kv(float *z, const float *a, const float *kv, long long n1, long long c, const PrimGroups &groups,
                           long long t, cudaStream_t stream) {
    if (groups.n < 1 || groups.n > MAX_PRIM_HEADS)
        return cudaErrorInvalidValue;
    int most = 0;
    for (int g = 0; g < groups.n; ++g)
        most = groups.first[g + 1] - groups.first[g] > most ? groups.first[g + 1] - groups.first[g] : most;
    if (most < 1 || most > MAX_PRIM_GROUP)
        return cudaErrorInvalidValue;
    const dim3 grid(unsigned((c + IP12_K - 1) / IP12_K), unsigned(groups.n));
    ip12_kv_kernel<<<grid, 32 * most, ip12_smem(most), stream>>>(z, a, kv, n1, c, t, groups);
    return cudaGetLastError();
}

cudaError_t launch_scale_outer(float *z, const float *s, float g, const float *a, const float *b, long long m,
                               long long k, cudaStream_t stream) {
    const long long n = m * k;
    unsigned grid = grid_of(n, 256);
    grid = grid > 148u * 16 ? 148u * 16 : grid;
    scale_outer_kernel<<<grid, 256, 0, stream>>>(z, s, g, a, b, m, k);
    return cudaGetLastError();
}

cudaError_t preload_prims() {
    cudaFuncAttributes at;
    cudaError_t e;
    if ((e = cudaFuncGetAttributes(&at, dot8_kernel<false>)) != cudaSuccess ||
        (e = cudaFuncGetAttributes(&at, dot8_kernel<true>)) != cudaSuccess ||
        (e = cudaFuncGetAttributes(&at, dot8_wide_kernel<false>)) != cudaSuccess ||
        (e = cudaFuncGetAttributes(&at, dot8_wide_kernel<true>)) != cudaSuccess ||
        (e = cudaFuncSetAttribute(ip12_kv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  int(ip12_smem(MAX_PRIM_GROUP)))) != cudaSuccess)
        return e;
    return cudaFuncGetAttributes(&at, scale_outer_kernel);
}

} // namespace q8
