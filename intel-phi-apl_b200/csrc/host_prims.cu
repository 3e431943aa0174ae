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
#include <cuda.h>

#include <cstring>

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

// Output o of a launch: ip21 computes z[o] (row o of a against b's row o / per_h); ip21_kv runs
// its outputs history-row-major with the query heads in kv-head order within a row, so the heads
// that share a kv head read the same row at the same time (one load for the group).
struct DotOut {
    long long hh, i;
};
template <bool KV>
__device__ __forceinline__ DotOut dot_out(long long o, long long per_h, long long h, const PrimHeads &heads) {
    if (KV) {
        const long long i = o / h;
        return {heads.ord[o - i * h], i};
    }
    const long long hh = o / per_h;
    return {hh, o - hh * per_h};
}

// Thread 8*g + j holds lane j of output g. 16 steps' loads are issued before their fmas.
template <bool KV>
__global__ void __launch_bounds__(256, 4) dot8_kernel(float *z, const float *a, const float *b, long long n_out, long long per_h,
                                                   long long c, long long n1, long long h, PrimHeads heads) {
    const long long g = (long long)blockIdx.x * (blockDim.x / 8) + threadIdx.x / 8;
    const int j = threadIdx.x % 8;
    const bool live = g < n_out;
    const DotOut d = dot_out<KV>(live ? g : 0, per_h, h, heads);
    // ip21: row o of a, b's row hh; ip21_kv: history row i of kv head l[hh], b's row hh
    const float *row = KV ? a + (d.i * n1 + heads.l[d.hh]) * c : a + (d.hh * per_h + d.i) * c;
    const float *v = b + d.hh * c;
    float acc = 0.0f;
    if (live) {
        long long k = j;
        for (; k + 8 * 15 < c; k += 8 * 16) {
            float r[16], q[16];
#pragma unroll
            for (int s = 0; s < 16; ++s) {
                r[s] = __ldg(row + k + 8 * s);
                q[s] = __ldg(v + k + 8 * s);
            }
#pragma unroll
            for (int s = 0; s < 16; ++s)
                acc = __fmaf_rn(r[s], q[s], acc);
        }
        for (; k < c; k += 8)
            acc = __fmaf_rn(__ldg(row + k), __ldg(v + k), acc);
    }
    const float r = lanes_sum(acc);
    if (live && j == 0)
        z[d.hh * per_h + d.i] = r;
}

// One thread per output, the 8 lanes in registers, 16-byte loads: for calls with outputs enough
// to fill the GPU this way (more loads in flight per thread than one lane per thread gives).
template <bool KV>
__global__ void __launch_bounds__(256) dot8_wide_kernel(float *z, const float *a, const float *b, long long n_out,
                                                        long long per_h, long long c, long long n1, long long h,
                                                        PrimHeads heads) {
    const long long o = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (o >= n_out)
        return;
    const DotOut d = dot_out<KV>(o, per_h, h, heads);
    const float4 *row = reinterpret_cast<const float4 *>(KV ? a + (d.i * n1 + heads.l[d.hh]) * c : a + o * c);
    const float4 *v = reinterpret_cast<const float4 *>(b + d.hh * c);
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
    z[d.hh * per_h + d.i] = __fadd_rn(__fadd_rn(__fadd_rn(l[0], l[4]), __fadd_rn(l[2], l[6])),
                                      __fadd_rn(__fadd_rn(l[1], l[5]), __fadd_rn(l[3], l[7])));
}

// Outputs from which one thread per output fills the GPU (148 SMs x 256 threads x 2). Below it
// the lane-per-thread form wins: 65,536 outputs over a 16 MB history took 12.8 us that way
// against 21.1 us one thread per output.
constexpr long long DOT_WIDE_MIN = 148ll * 256 * 2;

// ---------------------------------------------------------------- ip12_kv
// A CTA: one kv head's group of query heads and a W-column slice of c (W = 32 where c allows,
// else 8); thread W*hi + j keeps z[h][k] for head hi of the group and column j of the slice as
// one fma chain over the history rows in order. The slice streams through a ring of SLOTS stages
// of ROWS rows, one 2-D tensor copy per stage (a W x ROWS box of the history seen as [t][n1*c],
// rows past t filled with zeros) issued by thread 0 and counted on the slot's barrier; the
// group's weights for the same rows come by per-thread cp.async. A warp runs alone on its
// scheduler and its chain takes one dependent fma per row, so the rest of a row's work has to
// fit in the fma's latency: the operands of the next 16 rows are loaded while the current 16
// chain (two register sets in turn, nothing copied between them), and four rows' weights come in
// one 16-byte load (weight rows padded by 16 bytes so that four heads' reads fall into different
// banks). Every wait is bounded: a slice that never lands sets ERR_TIMEOUT_FULL, the CTA stops
// issuing, thread 0 waits (bounded) for the copies it issued, and z is left unwritten.
constexpr int IP12_ROWS = 128, IP12_SLOTS = 8, IP12_WS = IP12_ROWS + 4;
__host__ __device__ constexpr size_t ip12_smem(int w, int nh) {
    return size_t(IP12_SLOTS) * (size_t(IP12_ROWS) * w + size_t(nh) * IP12_WS) * 4;
}

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, bool ok) {
    const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    const int n = ok ? 16 : 0; // (a zero-size copy fills zeros: rows past t)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async4(void *smem, const void *gmem, bool ok) {
    const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    const int n = ok ? 4 : 0;
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(s), "l"(gmem), "r"(n) : "memory");
}
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *tm, int c0, int c1, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(tm), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

template <int W>
__global__ void __launch_bounds__(W * MAX_PRIM_GROUP, 1) ip12_kv_kernel(float *z, const float *a, long long c, long long t,
                                                                        PrimGroups groups,
                                                                        const __grid_constant__ CUtensorMap tkv,
                                                                        unsigned *err) {
    // dynamic: [SLOTS][ROWS][W] of history, then [SLOTS][nmax][WS] of a (nmax = blockDim.x / W,
    // at least the launch's largest group)
    extern __shared__ __align__(128) float dyn[];
    __shared__ __align__(8) uint64_t full[IP12_SLOTS];
    __shared__ int s_bad;
    float(*ring)[IP12_ROWS][W] = reinterpret_cast<float(*)[IP12_ROWS][W]>(dyn);
    const int nmax = blockDim.x / W;
    float *wbase = dyn + size_t(IP12_SLOTS) * IP12_ROWS * W;
    const int gi = blockIdx.y, hi = threadIdx.x / W, j = threadIdx.x % W;
    const int first = groups.first[gi], nh = groups.first[gi + 1] - first;
    const long long k0 = (long long)blockIdx.x * W;     // c % W == 0: the slice is whole
    const int kx = int(groups.kv[gi] * c + k0);         // the slice's first column in [t][n1*c]
    const bool a16 = (t % 4) == 0 && (reinterpret_cast<uintptr_t>(a) & 15) == 0;
    if (threadIdx.x == 0) {
        for (int s = 0; s < IP12_SLOTS; ++s)
            mbar_init(&full[s], 1);
        fence_barrier_init();
        s_bad = 0;
    }
    __syncthreads();
    long long issued = 0, landed0 = 0; // (thread 0: stages issued, stages whose slice it saw land)
    auto issue = [&](long long stage) {
        const int sl = int(stage % IP12_SLOTS);
        const long long r0 = stage * IP12_ROWS;
        if (threadIdx.x == 0) {
            mbar_arrive_expect_tx(&full[sl], uint32_t(IP12_ROWS * W * 4));
            tma_load_2d(&ring[sl][0][0], &tkv, kx, int(r0), &full[sl]);
            issued = stage + 1;
        }
        float *ws = wbase + size_t(sl) * nmax * IP12_WS;
        if (a16) {
            for (int e = threadIdx.x; e < nh * (IP12_ROWS / 4); e += blockDim.x) {
                const int h2 = e / (IP12_ROWS / 4), q = e % (IP12_ROWS / 4);
                const long long row = r0 + 4 * q;
                const bool ok = row < t;
                cp_async16(ws + h2 * IP12_WS + 4 * q, ok ? a + (long long)groups.head[first + h2] * t + row : a, ok);
            }
        } else {
            for (int e = threadIdx.x; e < nh * IP12_ROWS; e += blockDim.x) {
                const int h2 = e / IP12_ROWS, q = e % IP12_ROWS;
                const long long row = r0 + q;
                const bool ok = row < t;
                cp_async4(ws + h2 * IP12_WS + q, ok ? a + (long long)groups.head[first + h2] * t + row : a, ok);
            }
        }
    };
    const long long nstages = (t + IP12_ROWS - 1) / IP12_ROWS;
    for (int s = 0; s < IP12_SLOTS - 1; ++s) {
        if (s < nstages)
            issue(s);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    const bool mine = hi < nh;
    float acc = 0.0f;
    for (long long st = 0; st < nstages; ++st) {
        asm volatile("cp.async.wait_group %0;" ::"n"(IP12_SLOTS - 2) : "memory");
        __syncthreads(); // stage st's weights landed for every thread; slot (st - 1) % SLOTS is free again
        if (*reinterpret_cast<volatile int *>(&s_bad))
            break; // (read by every thread after the same barrier: all leave together)
        if (st + IP12_SLOTS - 1 < nstages)
            issue(st + IP12_SLOTS - 1);
        asm volatile("cp.async.commit_group;" ::: "memory");
        const int sl = int(st % IP12_SLOTS);
        if (!mbar_wait(&full[sl], uint32_t((st / IP12_SLOTS) & 1))) {
            report(err, ERR_TIMEOUT_FULL);
            *reinterpret_cast<volatile int *>(&s_bad) = 1;
            continue;
        }
        if (threadIdx.x == 0)
            landed0 = st + 1;
        const float(*slot)[W] = ring[sl];
        const float *ws = wbase + (size_t(sl) * nmax + (mine ? hi : 0)) * IP12_WS;
        const int nr = int(t - st * IP12_ROWS < IP12_ROWS ? t - st * IP12_ROWS : IP12_ROWS);
        if (!mine)
            continue;
        if (nr == IP12_ROWS) {
            const float4 *w4 = reinterpret_cast<const float4 *>(ws);
            float4 wa[4], wb[4];
            float xa[16], xb[16];
            auto load = [&](float4 *w, float *x, int g) {
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    w[q] = w4[4 * g + q];
#pragma unroll
                for (int q = 0; q < 16; ++q)
                    x[q] = slot[16 * g + q][j];
            };
            auto chain = [&](const float4 *w, const float *x) {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    acc = __fmaf_rn(w[q].x, x[4 * q + 0], acc);
                    acc = __fmaf_rn(w[q].y, x[4 * q + 1], acc);
                    acc = __fmaf_rn(w[q].z, x[4 * q + 2], acc);
                    acc = __fmaf_rn(w[q].w, x[4 * q + 3], acc);
                }
            };
            load(wa, xa, 0);
#pragma unroll
            for (int g = 0; g < IP12_ROWS / 16; g += 2) {
                load(wb, xb, g + 1);
                chain(wa, xa);
                if (g + 2 < IP12_ROWS / 16)
                    load(wa, xa, g + 2);
                chain(wb, xb);
            }
        } else {
            for (int rr = 0; rr < nr; ++rr)
                acc = __fmaf_rn(ws[rr], slot[rr][j], acc);
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    if (threadIdx.x == 0) // copies thread 0 issued and did not see land (only after a timeout)
        for (long long s = landed0; s < issued; ++s)
            if (!mbar_wait(&full[s % IP12_SLOTS], uint32_t((s / IP12_SLOTS) & 1)))
                break;
    if (mine && !*reinterpret_cast<volatile int *>(&s_bad))
        z[(long long)groups.head[first + hi] * c + k0 + j] = acc;
}

// ---------------------------------------------------------------- scale_outer
// One element per thread, or four in 16-byte accesses (vec: k % 4 == 0, z, s and b 16-aligned,
// m * k < 2^31), the row and column from 32-bit index arithmetic where the size allows.
__global__ void __launch_bounds__(256) scale_outer_kernel(float *z, const float *s, float g, const float *a, const float *b,
                                                          long long m, long long k, int vec) {
    if (vec) {
        const int nq4 = int(k / 4), n4 = int(m) * nq4;
        const float4 *s4 = reinterpret_cast<const float4 *>(s), *b4 = reinterpret_cast<const float4 *>(b);
        float4 *z4 = reinterpret_cast<float4 *>(z);
        for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < n4; e += gridDim.x * blockDim.x) {
            const int i = e / nq4, q = e - i * nq4;
            const float ai = __ldg(a + i);
            const float4 sv = __ldg(s4 + e), bv = __ldg(b4 + q);
            float4 r;
            r.x = __fmaf_rn(g, sv.x, __fmul_rn(ai, bv.x));
            r.y = __fmaf_rn(g, sv.y, __fmul_rn(ai, bv.y));
            r.z = __fmaf_rn(g, sv.z, __fmul_rn(ai, bv.z));
            r.w = __fmaf_rn(g, sv.w, __fmul_rn(ai, bv.w));
            z4[e] = r;
        }
        return;
    }
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
        dot8_wide_kernel<false><<<grid_of(n, 256), 256, 0, stream>>>(z, a, b, n, r, c, 0, h, none);
    else
        dot8_kernel<false><<<grid_of(n * 8, 256), 256, 0, stream>>>(z, a, b, n, r, c, 0, h, none);
    return cudaGetLastError();
}

cudaError_t launch_ip21_kv(float *z, const float *kv, long long n1, long long c, const PrimHeads &heads, long long h,
                           long long t, const float *b, cudaStream_t stream) {
    const long long n = h * t;
    if (n >= DOT_WIDE_MIN && aligned16(kv) && aligned16(b))
        dot8_wide_kernel<true><<<grid_of(n, 256), 256, 0, stream>>>(z, kv, b, n, t, c, n1, h, heads);
    else
        dot8_kernel<true><<<grid_of(n * 8, 256), 256, 0, stream>>>(z, kv, b, n, t, c, n1, h, heads);
    return cudaGetLastError();
}

cudaError_t launch_ip12_kv(float *z, const float *a, const float *kv, long long n1, long long c, const PrimGroups &groups,
                           long long t, unsigned *err, cudaStream_t stream) {
    if (groups.n < 1 || groups.n > MAX_PRIM_HEADS || c < 8 || c % 8 || n1 * c >= (1ll << 31))
        return cudaErrorInvalidValue;
    int most = 0;
    for (int g = 0; g < groups.n; ++g)
        most = groups.first[g + 1] - groups.first[g] > most ? groups.first[g + 1] - groups.first[g] : most;
    if (most < 1 || most > MAX_PRIM_GROUP)
        return cudaErrorInvalidValue;
    // 32-column slices (128-byte history pieces) where c allows: measured faster than 8 on the
    // attention shapes, with four warps of one head each per CTA
    const int w = c % 32 == 0 ? 32 : 8;
    alignas(64) CUtensorMap tkv;
    memset(&tkv, 0, sizeof tkv);
    if (t > 0 && !map_f32_2d(&tkv, kv, uint64_t(n1 * c), uint64_t(t), uint64_t(n1 * c) * 4, uint32_t(w),
                             uint32_t(IP12_ROWS)))
        return cudaErrorInvalidValue;
    if (w == 32) {
        const int threads = 32 * most;
        ip12_kv_kernel<32><<<dim3(unsigned(c / 32), unsigned(groups.n)), threads, ip12_smem(32, most), stream>>>(
            z, a, c, t, groups, tkv, err);
    } else {
        const int threads = (8 * most + 31) / 32 * 32;
        ip12_kv_kernel<8><<<dim3(unsigned(c / 8), unsigned(groups.n)), threads, ip12_smem(8, threads / 8), stream>>>(
            z, a, c, t, groups, tkv, err);
    }
    return cudaGetLastError();
}

cudaError_t launch_scale_outer(float *z, const float *s, float g, const float *a, const float *b, long long m,
                               long long k, cudaStream_t stream) {
    const long long n = m * k;
    const int vec = k % 4 == 0 && n < (1ll << 31) && aligned16(z) && aligned16(s) && aligned16(b);
    unsigned grid = grid_of(vec ? n / 4 : n, 256);
    grid = grid > 148u * 16 ? 148u * 16 : grid;
    scale_outer_kernel<<<grid, 256, 0, stream>>>(z, s, g, a, b, m, k, vec);
    return cudaGetLastError();
}

cudaError_t preload_prims() {
    cudaFuncAttributes at;
    cudaError_t e;
    if ((e = cudaFuncGetAttributes(&at, dot8_kernel<false>)) != cudaSuccess ||
        (e = cudaFuncGetAttributes(&at, dot8_kernel<true>)) != cudaSuccess ||
        (e = cudaFuncGetAttributes(&at, dot8_wide_kernel<false>)) != cudaSuccess ||
        (e = cudaFuncGetAttributes(&at, dot8_wide_kernel<true>)) != cudaSuccess ||
        (e = cudaFuncSetAttribute(ip12_kv_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  int(ip12_smem(32, MAX_PRIM_GROUP)))) != cudaSuccess ||
        (e = cudaFuncSetAttribute(ip12_kv_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  int(ip12_smem(8, MAX_PRIM_GROUP)))) != cudaSuccess)
        return e;
    return cudaFuncGetAttributes(&at, scale_outer_kernel);
}

} // namespace q8
