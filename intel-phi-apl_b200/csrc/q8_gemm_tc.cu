// q8_gemm_tc.cu: the Q8_0 product for t >= 16 tokens on the 5th-generation tensor cores.
//
// Y[t][o] = sum_k fp16(q[o][k] * d[o][k/32]) * fp16(x[t][k]), fp32 sums in TMEM.
//
// At 16+ tokens the product is a dense contraction (the reference batches prompts of 16 and
// verify passes of K+1 tokens through the same weight pass, src/card/gemm.c:271-294). The
// per-(row, 32-column) fp16 scale d cannot be factored out of a K contraction, so each weight tile
// is dequantised to fp16 in shared memory first: q is exact in fp16, and fl16(q*d) rounds once.
// x is rounded to fp16 once per call (a pre-pass into scratch). fp16 rather than bf16: the same
// tcgen05 kind::f16 rate with 3 more mantissa bits, which is what holds the product within the
// stated 2e-3 (bf16 tiles measure ~1e-2 on the BASELINE shapes).
//
// A CTA (persistent, one per SM: it owns all 512 TMEM columns) runs 128-row x BN-token tiles:
//   warp 8      TMA: per 64-column stage, the quant box (128 rows x 64 B, 64B swizzle), the scale
//               box (128 rows x 8 scales) and the fp16 x box (BN rows x 128 B, 128B swizzle);
//   warps 4-7   dequant: thread i turns row i's 64 quants and 2 scales into 64 fp16 weights,
//               written into the A tile in the UMMA 128B-swizzled K-major layout;
//   warp 9      MMA: 4 x tcgen05.mma (M=128, N=BN, K=16) per stage into one of two TMEM
//               accumulators; tcgen05.commit frees the stage, and at a tile's end the accumulator;
//   warps 0-3   epilogue: tcgen05.ld of TMEM lanes 32*(warp%4).. -> y (or silu(g)*u for a pair).
// Every wait is bounded (error word on timeout); every TMA load is a plain single-CTA load.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>
#include <unordered_map>

#include "q8_kernels.h"
#include "q8_layout.h"
#include "q8_ptx.cuh"

namespace q8 {
namespace {

constexpr int BM = 128;          // weight rows per tile (MMA M)
constexpr int BK = 64;           // columns per stage
constexpr int MAX_BN = 256;      // tokens per tile (MMA N)
constexpr int MAX_STAGES = 6;
constexpr int NT = 320;          // 10 warps
constexpr int EPI_WARP0 = 0, DQ_WARP0 = 4, TMA_WARP = 8, MMA_WARP = 9;
constexpr int TMEM_COLS = 512;   // two accumulators of up to 256 columns
constexpr int OFF_Q = 0, OFF_D = 8192, OFF_A = 10240, OFF_X = 26624; // within a stage (1024-aligned)
constexpr size_t SMEM_LIMIT = 200 * 1024;

__host__ __device__ constexpr int stage_bytes(int bn) { return (OFF_X + bn * 128 + 1023) / 1024 * 1024; }

struct TcJobDev {
    CUtensorMap tq, td, tq2, td2; // quants and scales of W (and of the SwiGLU up matrix)
    float *y;
    long long rows, ldy;
    int cols, t, pair, n_pass, tiles, unit0; // tiles: row tiles; units = tiles * n_pass
};

struct TcParams {
    CUtensorMap tx[8];   // fp16 x per job
    TcJobDev job[8];
    int njobs, total_units, bn, stages;
    unsigned *err;
};

// The fp16 copy of x is written by the conversion kernel just before this one on the stream: the
// producer waits for it (a no-op without programmatic launch) before its first x load.

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *tm, int c0, int c1, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(tm), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(acc));
}

// UMMA shared-memory descriptor of a K-major tile in the 128B-swizzled canonical layout: rows of
// 128 B, 8-row groups 1024 B apart (SBO), leading offset 1 (unused when swizzled), version 1.
__device__ __forceinline__ uint64_t sw128_desc(const void *tile) {
    const uint64_t a = smem_u32(tile);
    return ((a & 0x3FFFF) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// kind::f16 instruction descriptor: fp32 accumulator, fp16 A and B, both K-major, M = 128, N = bn.
__device__ __forceinline__ uint32_t idesc_f16(int bn) {
    return (1u << 4) | (uint32_t(bn >> 3) << 17) | (uint32_t(BM >> 4) << 24);
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ int find_job(const TcParams &p, int u) {
    int j = 0;
    while (j + 1 < p.njobs && u >= p.job[j + 1].unit0)
        ++j;
    return j;
}

// A unit of work: row tile `rt` and token pass `np` of job `j`; a SwiGLU pair unit is two MMA
// tiles (gate, then up) sharing the x tiles and the two accumulators.
struct Unit {
    int j, rt, np, ntile; // ntile: MMA tiles in the unit (1 or 2)
};

__device__ __forceinline__ Unit unit_of(const TcParams &p, int u) {
    Unit w;
    w.j = find_job(p, u);
    const TcJobDev &J = p.job[w.j];
    const int lu = u - J.unit0;
    w.rt = lu / J.n_pass;
    w.np = lu - w.rt * J.n_pass;
    w.ntile = J.pair ? 2 : 1;
    return w;
}

__global__ void __launch_bounds__(NT, 1) gemm_tc_kernel(const __grid_constant__ TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int S = p.stages, BN = p.bn, SB = stage_bytes(BN);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + size_t(S) * SB);
    uint64_t *empty = full + MAX_STAGES;
    uint64_t *afull = empty + MAX_STAGES;
    uint64_t *accfull = afull + MAX_STAGES; // [2]
    uint64_t *accempty = accfull + 2;       // [2]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accempty + 2);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            mbar_init(&afull[s], 128);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&accfull[b], 1);
            mbar_init(&accempty[b], 128);
        }
        fence_barrier_init();
    }
    if (warp == MMA_WARP) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (threadIdx.x == 0)
        grid_launch_dependents();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    grid_wait(); // x (fp16) and the y buffers belong to the kernels before this one
    const int nk = 0; // per job (cols differ): computed in the loops
    (void)nk;

    if (warp == TMA_WARP) {
        // ---------------------------------------------------------------- producer
        if (lane == 0) {
            int s = 0, use = 0; // running stage counter
            bool ok = true;
            for (int u = blockIdx.x; u < p.total_units && ok; u += gridDim.x) {
                const Unit w = unit_of(p, u);
                const TcJobDev &J = p.job[w.j];
                const int nks = (J.cols + BK - 1) / BK;
                for (int ti = 0; ti < w.ntile && ok; ++ti) {
                    const CUtensorMap *tq = ti ? &J.tq2 : &J.tq, *td = ti ? &J.td2 : &J.td;
                    for (int kb = 0; kb < nks; ++kb, ++s) {
                        const int slot = s % S;
                        const int k = s / S;
                        if (k > 0 && !mbar_wait(&empty[slot], (k - 1) & 1)) {
                            report(p.err, ERR_TIMEOUT_MMA);
                            ok = false;
                            break;
                        }
                        uint8_t *st = smem + size_t(slot) * SB;
                        mbar_arrive_expect_tx(&full[slot], uint32_t(BM * 64 + BM * 16 + BN * 128));
                        const int k0 = kb * BK;
                        tma_load_2d(st + OFF_Q, tq, k0, w.rt * BM, &full[slot]);
                        tma_load_2d(st + OFF_D, td, (k0 / Q8_QK) & ~7, w.rt * BM, &full[slot]);
                        tma_load_2d(st + OFF_X, &p.tx[w.j], k0, w.np * BN, &full[slot]);
                        ++use;
                    }
                }
            }
            // leave no copy in flight: wait for the most recent fill of every slot
            for (int q = max(0, s - S); q < s; ++q)
                if (!mbar_wait(&full[q % S], (q / S) & 1))
                    report(p.err, ERR_TIMEOUT_DRAIN);
        }
    } else if (warp >= DQ_WARP0 && warp < DQ_WARP0 + 4) {
        // ---------------------------------------------------------------- dequant
        const int i = threadIdx.x - DQ_WARP0 * 32; // tile row
        int s = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < p.total_units && ok; u += gridDim.x) {
            const Unit w = unit_of(p, u);
            const TcJobDev &J = p.job[w.j];
            const int nks = (J.cols + BK - 1) / BK;
            for (int ti = 0; ti < w.ntile && ok; ++ti) {
                for (int kb = 0; kb < nks; ++kb, ++s) {
                    const int slot = s % S, k = s / S;
                    if (!mbar_wait(&full[slot], k & 1)) {
                        report(p.err, ERR_TIMEOUT_FULL);
                        ok = false;
                        break;
                    }
                    // the A tile of this slot is free once the MMAs of its previous use are done
                    if (k > 0 && !mbar_wait(&empty[slot], (k - 1) & 1)) {
                        report(p.err, ERR_TIMEOUT_MMA);
                        ok = false;
                        break;
                    }
                    uint8_t *st = smem + size_t(slot) * SB;
                    // the two scales of this 64-column stage, from the 8 the scale box holds
                    const int e0 = (kb * 2) & 7;
                    const uint32_t dd = *reinterpret_cast<const uint32_t *>(st + OFF_D + i * 16 + e0 * 2);
                    const __half2 d0 = __half2half2(__ushort_as_half(uint16_t(dd & 0xffff)));
                    const __half2 d1 = __half2half2(__ushort_as_half(uint16_t(dd >> 16)));
                    const __half2 bias = __half2half2(__ushort_as_half(uint16_t(0x6480))); // 1152
                    uint8_t *arow = st + OFF_A + i * 128;
#pragma unroll
                    for (int c = 0; c < 4; ++c) { // 16 quants per chunk; chunks 0,1 block 0; 2,3 block 1
                        const uint4 qv =
                            *reinterpret_cast<const uint4 *>(st + OFF_Q + i * 64 + ((c ^ ((i >> 1) & 3)) << 4));
                        const uint32_t wq[4] = {qv.x ^ 0x80808080u, qv.y ^ 0x80808080u, qv.z ^ 0x80808080u,
                                                qv.w ^ 0x80808080u};
                        const __half2 dd2 = c < 2 ? d0 : d1;
                        uint32_t outw[8];
#pragma unroll
                        for (int v = 0; v < 4; ++v) {
                            // (q+128) as the low byte of fp16 1024+(q+128): exact; minus 1152 -> q
                            const uint32_t lo = __byte_perm(wq[v], 0x64646464u, 0x4140u);
                            const uint32_t hi = __byte_perm(wq[v], 0x64646464u, 0x4342u);
                            __half2 a = __hsub2(*reinterpret_cast<const __half2 *>(&lo), bias);
                            __half2 b = __hsub2(*reinterpret_cast<const __half2 *>(&hi), bias);
                            a = __hmul2(a, dd2);
                            b = __hmul2(b, dd2);
                            outw[2 * v] = *reinterpret_cast<uint32_t *>(&a);
                            outw[2 * v + 1] = *reinterpret_cast<uint32_t *>(&b);
                        }
                        // 16 fp16 = two 16-byte chunks (2c, 2c+1) of the 128-byte row, swizzled
                        const int c0 = (2 * c) ^ (i & 7), c1 = (2 * c + 1) ^ (i & 7);
                        *reinterpret_cast<uint4 *>(arow + (c0 << 4)) = make_uint4(outw[0], outw[1], outw[2], outw[3]);
                        *reinterpret_cast<uint4 *>(arow + (c1 << 4)) = make_uint4(outw[4], outw[5], outw[6], outw[7]);
                    }
                    fence_proxy_async_shared(); // generic-proxy writes -> visible to the tensor core
                    mbar_arrive(&afull[slot]);
                }
            }
        }
    } else if (warp == MMA_WARP) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = idesc_f16(BN);
            int s = 0, tcount = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < p.total_units && ok; u += gridDim.x) {
                const Unit w = unit_of(p, u);
                const TcJobDev &J = p.job[w.j];
                const int nks = (J.cols + BK - 1) / BK;
                for (int ti = 0; ti < w.ntile && ok; ++ti, ++tcount) {
                    const int b = tcount & 1, bu = tcount >> 1;
                    if (bu > 0 && !mbar_wait(&accempty[b], (bu - 1) & 1)) {
                        report(p.err, ERR_TIMEOUT_MMA);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t tacc = tmem + uint32_t(b * 256);
                    for (int kb = 0; kb < nks; ++kb, ++s) {
                        const int slot = s % S, k = s / S;
                        if (!mbar_wait(&afull[slot], k & 1) || !mbar_wait(&full[slot], k & 1)) {
                            report(p.err, ERR_TIMEOUT_MMA);
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        uint8_t *st = smem + size_t(slot) * SB;
                        const uint64_t da = sw128_desc(st + OFF_A), db = sw128_desc(st + OFF_X);
#pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk) // +32 bytes along K per step
                            tc_mma(tacc, da + uint64_t(2 * kk), db + uint64_t(2 * kk), idesc, (kb | kk) ? 1u : 0u);
                        tc_commit(&empty[slot]);
                    }
                    if (ok)
                        tc_commit(&accfull[b]);
                }
            }
            // drain: the MMAs of the last use of every slot
            for (int q = max(0, s - S); q < s; ++q)
                if (!mbar_wait(&empty[q % S], (q / S) & 1))
                    report(p.err, ERR_TIMEOUT_DRAIN);
        }
    } else {
        // ---------------------------------------------------------------- epilogue (warps 0-3)
        const int e = warp & 3; // TMEM lanes 32e..32e+31 = tile rows
        int tcount = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < p.total_units && ok; u += gridDim.x) {
            const Unit w = unit_of(p, u);
            const TcJobDev &J = p.job[w.j];
            const int b0 = tcount & 1;
            bool got = true;
            for (int ti = 0; ti < w.ntile; ++ti) {
                const int b = (tcount + ti) & 1, bu = (tcount + ti) >> 1;
                got = got && mbar_wait(&accfull[b], bu & 1);
            }
            if (!got) {
                report(p.err, ERR_TIMEOUT_MMA);
                ok = false;
                break;
            }
            tc_fence_after();
            const long long row = (long long)w.rt * BM + 32 * e + lane;
            const int n0 = w.np * BN;
            for (int c0 = 0; c0 < BN; c0 += 16) {
                uint32_t r[16], r2[16];
                tmem_ld16(tmem + (uint32_t(32 * e) << 16) + uint32_t(b0 * 256 + c0), r);
                if (w.ntile == 2)
                    tmem_ld16(tmem + (uint32_t(32 * e) << 16) + uint32_t((b0 ^ 1) * 256 + c0), r2);
                tmem_wait_ld();
                if (row < J.rows) {
#pragma unroll
                    for (int c = 0; c < 16; ++c) {
                        const int tok = n0 + c0 + c;
                        if (tok < J.t) {
                            float v = __uint_as_float(r[c]);
                            if (w.ntile == 2) {
                                const float up = __uint_as_float(r2[c]);
                                v = v / (1.0f + expf(-v)) * up;
                            }
                            J.y[(long long)tok * J.ldy + row] = v;
                        }
                    }
                }
            }
            tc_fence_before();
            for (int ti = 0; ti < w.ntile; ++ti)
                mbar_arrive(&accempty[(tcount + ti) & 1]);
            tcount += w.ntile;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == MMA_WARP)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
}

__global__ void x_to_half_kernel(const float *x, long long ldx, int cols, int t, __half *xh) {
    const long long n = (long long)t * cols;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / cols, c = i - r * cols;
        xh[i] = __float2half_rn(x[r * ldx + c]);
    }
}

// ---------------------------------------------------------------- host: tensor maps
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void *f = nullptr;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return fn;
}

bool make_map(CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t d0, uint64_t d1, uint64_t stride1,
              uint32_t b0, uint32_t b1, CUtensorMapSwizzle sw) {
    auto fn = encode_fn();
    if (!fn)
        return false;
    const cuuint64_t dims[2] = {d0, d1}, strides[1] = {stride1};
    const cuuint32_t box[2] = {b0, b1}, es[2] = {1, 1};
    return fn(m, dt, 2, const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The quant and scale maps of a row-split matrix (rows x cols): quants are a 2-D uint8 array of
// cols bytes per row, rows q8s_row_bytes apart; scales a uint16 array at +cols of the same rows.
bool weight_maps(const uint8_t *w, long long rows, int cols, CUtensorMap *tq, CUtensorMap *td) {
    const uint64_t rb = uint64_t(q8s_row_bytes(cols));
    return make_map(tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, uint64_t(cols), uint64_t(rows), rb, 64, BM,
                    CU_TENSOR_MAP_SWIZZLE_64B) &&
           make_map(td, CU_TENSOR_MAP_DATA_TYPE_UINT16, w + cols, uint64_t(q8s_scale_stride(cols)), uint64_t(rows), rb, 8,
                    BM, CU_TENSOR_MAP_SWIZZLE_NONE);
}

} // namespace

size_t gemm_tc_scratch_bytes(const GemmJob *jobs, int n) {
    size_t s = 0;
    for (int j = 0; j < n; ++j)
        s += (size_t(jobs[j].t) * jobs[j].cols * sizeof(__half) + 255) / 256 * 256;
    return s;
}

cudaError_t launch_gemm_tc(const GemmJob *jobs, int n, void *scratch, size_t scratch_bytes, int num_sms,
                           unsigned *err, cudaStream_t stream, bool pdl) {
    if (n < 1 || n > 8)
        return cudaErrorInvalidValue;
    if (gemm_tc_scratch_bytes(jobs, n) > scratch_bytes || !scratch)
        return cudaErrorInvalidValue;
    // tokens per tile: the largest t split into passes of <= 256, rounded up to 16
    int tmax = 0;
    for (int j = 0; j < n; ++j)
        tmax = jobs[j].t > tmax ? jobs[j].t : tmax;
    const int npass_max = (tmax + MAX_BN - 1) / MAX_BN;
    int bn = ((tmax + npass_max - 1) / npass_max + 15) / 16 * 16;
    if (bn < 16)
        bn = 16;
    TcParams p;
    memset(&p, 0, sizeof p);
    p.njobs = n;
    p.bn = bn;
    p.err = err;
    const int sb = stage_bytes(bn);
    p.stages = int(SMEM_LIMIT / size_t(sb));
    if (p.stages > MAX_STAGES)
        p.stages = MAX_STAGES;
    if (p.stages < 2)
        return cudaErrorInvalidValue;
    uint8_t *sc = static_cast<uint8_t *>(scratch);
    int units = 0;
    for (int j = 0; j < n; ++j) {
        const GemmJob &G = jobs[j];
        if (G.cols < Q8_QK || G.cols % Q8_QK || G.t < 1 || G.rows < 1)
            return cudaErrorInvalidValue;
        __half *xh = reinterpret_cast<__half *>(sc);
        sc += (size_t(G.t) * G.cols * sizeof(__half) + 255) / 256 * 256;
        const long long nconv = (long long)G.t * G.cols;
        int grid = int((nconv + 255) / 256);
        grid = grid > 4096 ? 4096 : grid;
        x_to_half_kernel<<<grid, 256, 0, stream>>>(G.x, G.ldx, G.cols, G.t, xh);
        if (!make_map(&p.tx[j], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xh, uint64_t(G.cols), uint64_t(G.t),
                      uint64_t(G.cols) * 2, 64, uint32_t(bn), CU_TENSOR_MAP_SWIZZLE_128B))
            return cudaErrorInvalidValue;
        TcJobDev &J = p.job[j];
        if (!weight_maps(G.w, G.rows, G.cols, &J.tq, &J.td))
            return cudaErrorInvalidValue;
        J.pair = G.w2 != nullptr;
        if (J.pair && !weight_maps(G.w2, G.rows, G.cols, &J.tq2, &J.td2))
            return cudaErrorInvalidValue;
        J.y = G.y;
        J.rows = G.rows;
        J.ldy = G.ldy;
        J.cols = G.cols;
        J.t = G.t;
        J.n_pass = (G.t + bn - 1) / bn;
        J.tiles = int((G.rows + BM - 1) / BM);
        J.unit0 = units;
        units += J.tiles * J.n_pass;
    }
    p.total_units = units;
    const size_t smem = size_t(p.stages) * sb + 6 * 8 * MAX_STAGES + 64 + 1024;
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             int(SMEM_LIMIT + 4096));
        if (e != cudaSuccess)
            return e;
        attr = true;
    }
    int grid = num_sms > 0 ? num_sms : 148;
    if (grid > units)
        grid = units;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(NT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute lattr[1];
    lattr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    lattr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = lattr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemm_tc_kernel, p);
}

} // namespace q8
