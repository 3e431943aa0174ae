// q8_gemv.cu: the exact Q8_0 product on CUDA cores, for t = 1..4 tokens per pass. Behind
// rt_gemv / rt_gemv_q / rt_gemm(_q) at t < 16, the fused SwiGLU pair and the row gather.
//
// Arithmetic. Output row o of token t is the reference's exact rounding sequence
// (src/card/gemv.c:93-111, gemm.c keeps every token on it: src/card/gemm.h:6-7):
//     acc = +0; for each 32-column block b in order:
//         t_b = +0; for i = 0..31: t_b = fma(q_i, x_i, t_b);   acc = fma(t_b, fp16 d_b, acc)
// int8 -> fp32 and fp16 -> fp32 are exact, every fma is IEEE fp32 with one rounding, so each y is
// the reference host model's value bit for bit.
//
// Mapping. A row tile is R = 8 rows x all cols; it is streamed through shared memory in stages of
// 8 rows x 4096 columns by 1-D bulk copies (one per row, or two where a row is longer than a
// stage). Four compute warps (128 threads) own one 32-column block each: thread j keeps that
// block's 32 x values (per token) in registers and runs the 32-fma chain t_b for each of the 8
// rows, so the weight bytes are read once from shared memory and x never is. The t_b and the
// block scales go to a small partial-sum buffer; a fifth warp, which also issues the bulk copies,
// runs the serial chain acc = fma(t_b, d_b, acc) with one lane per (token, row) and writes y.
//
// Pipeline: 4 stage slots (full barriers completed by the copies' byte counts), 2 partial-sum
// buffers (tfull: compute -> chain, tempty: chain -> compute). Every wait is bounded; a timeout
// sets a bit in the context's error word and the CTA leaves.
#include <cuda_fp16.h>

#include "q8_kernels.h"
#include "q8_layout.h"
#include "q8_ptx.cuh"

namespace q8 {
namespace {

constexpr int R = 8;             // rows per tile / stage
constexpr int KC = 4096;         // columns per stage
constexpr int NBK = KC / Q8_QK;  // blocks per stage: 128
constexpr int STAGES = 4;
constexpr int NC = 128;          // compute threads: one block column each
constexpr int NT = NC + 32;      // + the chain / copy warp
constexpr int ROWB = KC + NBK * 2; // a row's slot: quants then scales, 4352 B
constexpr int SLOT = R * ROWB;
constexpr int TPAD = NBK + 1;    // partial-sum row stride (floats): conflict-free per lane = row
static_assert(NC == NBK, "one compute thread per block column of a stage");
static_assert(ROWB % 16 == 0 && SLOT % 16 == 0, "bulk copy destinations are 16-byte aligned");

template <int MT>
constexpr size_t smem_bytes() {
    return size_t(STAGES) * SLOT + size_t(2) * MT * R * TPAD * 4 + size_t(2) * R * TPAD * 4 + (STAGES + 4) * 8;
}

__device__ __forceinline__ int find_job(const GemvParams &p, int g) {
    int j = 0;
    while (j + 1 < p.njobs && g >= p.job[j + 1].tile0)
        ++j;
    return j;
}

// The CTA's sequence of stages: tiles blockIdx.x, +gridDim.x, ..., each in ceil(cols/KC) chunks.
// Every role walks its own copy of it.
struct StageIter {
    int g, c, job, nchunk;
    __device__ void start(const GemvParams &p) {
        g = blockIdx.x;
        c = 0;
        set(p);
    }
    __device__ void set(const GemvParams &p) {
        if (g < p.total_tiles) {
            job = find_job(p, g);
            nchunk = (p.job[job].cols + KC - 1) / KC;
        }
    }
    __device__ bool valid(const GemvParams &p) const { return g < p.total_tiles; }
    __device__ void next(const GemvParams &p) {
        if (++c == nchunk) {
            c = 0;
            g += gridDim.x;
            set(p);
        }
    }
};

// Row r (0..R-1) of a stage: its output index o, the matrix row it reads, whether it exists
// (valid) and whether it is read (load: a gather index outside the matrix is not).
struct StageRow {
    long long o, src;
    const uint8_t *mat;
    bool valid, load;
};

__device__ __forceinline__ StageRow stage_row(const GemvJob &J, int lt, int r) {
    const int rpt = J.w2 ? R / 2 : R; // output rows per tile
    StageRow s;
    s.o = (long long)lt * rpt + (r % rpt);
    s.mat = (J.w2 && r >= rpt) ? J.w2 : J.w;
    s.valid = s.o < J.rows;
    s.src = s.valid && J.idx ? (long long)J.idx[s.o] : s.o;
    s.load = s.valid && s.src >= 0 && s.src < J.src_rows;
    return s;
}

__device__ __forceinline__ void issue_stage(const GemvParams &p, const StageIter &it, uint8_t *slot_base,
                                            uint64_t *bar, uint64_t pol) {
    const GemvJob &J = p.job[it.job];
    const int lt = it.g - J.tile0;
    const long long rb = q8s_row_bytes(J.cols);
    const int c0 = it.c * KC;
    const int nbk = min(KC, J.cols - c0) / Q8_QK;
    const uint32_t qbytes = uint32_t(nbk) * Q8_QK, dbytes = (uint32_t(nbk) * 2u + 15u) & ~15u;
    const bool whole = J.cols == KC; // a row is exactly one slot row: one copy
    uint32_t total = 0;
    for (int r = 0; r < R; ++r)
        if (stage_row(J, lt, r).load)
            total += whole ? uint32_t(rb) : qbytes + dbytes;
    mbar_arrive_expect_tx(bar, total);
    for (int r = 0; r < R; ++r) {
        const StageRow sr = stage_row(J, lt, r);
        if (!sr.load)
            continue;
        const uint8_t *src = sr.mat + sr.src * rb;
        uint8_t *dst = slot_base + r * ROWB;
        if (whole) {
            bulk_g2s(dst, src, uint32_t(rb), bar, pol);
        } else {
            bulk_g2s(dst, src + c0, qbytes, bar, pol);
            bulk_g2s(dst + KC, src + J.cols + (c0 / Q8_QK) * 2, dbytes, bar, pol);
        }
    }
}

template <int MT>
__global__ void __launch_bounds__(NT, 1) gemv_exact_kernel(const __grid_constant__ GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *slots = smem;
    float *T = reinterpret_cast<float *>(smem + size_t(STAGES) * SLOT); // [2][MT][R][TPAD]
    float *TD = T + 2 * MT * R * TPAD;                                   // [2][R][TPAD]
    uint64_t *full = reinterpret_cast<uint64_t *>(TD + 2 * R * TPAD);    // [STAGES]
    uint64_t *tfull = full + STAGES;                                     // [2]
    uint64_t *tempty = tfull + 2;                                        // [2]
    const int tid = threadIdx.x;

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s)
            mbar_init(&full[s], 1);
        mbar_init(&tfull[0], NC);
        mbar_init(&tfull[1], NC);
        mbar_init(&tempty[0], 1);
        mbar_init(&tempty[1], 1);
        fence_barrier_init();
    }
    __syncthreads();

    if (tid < NC) {
        // ---------------------------------------------------------------- compute threads
        float xr[MT][Q8_QK];
        int xjob = -1, xc = -1, xb = -1;
        StageIter it;
        it.start(p);
        for (int s = 0; it.valid(p); it.next(p), ++s) {
            const int slot = s % STAGES;
            if (!mbar_wait(&full[slot], (s / STAGES) & 1)) {
                report(p.err, ERR_TIMEOUT_FULL);
                break;
            }
            const int tb = s & 1;
            if (s >= 2 && !mbar_wait(&tempty[tb], ((s >> 1) - 1) & 1)) {
                report(p.err, ERR_TIMEOUT_TEMPTY);
                break;
            }
            const GemvJob &J = p.job[it.job];
            const int lt = it.g - J.tile0;
            const int c0 = it.c * KC;
            const int nbk = min(KC, J.cols - c0) / Q8_QK;
            const uint8_t *sb = slots + size_t(slot) * SLOT;
            float *Tb = T + tb * MT * R * TPAD;
            float *TDb = TD + tb * R * TPAD;
            for (int u = tid; u < R * nbk; u += NC) {
                const int r = u / nbk, b = u - r * nbk;
                if (!stage_row(J, lt, r).load)
                    continue;
                if (b != xb || it.c != xc || it.job != xjob) {
                    xb = b;
                    xc = it.c;
                    xjob = it.job;
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        const float4 *xp = reinterpret_cast<const float4 *>(J.x + mt * J.ldx + c0 + b * Q8_QK);
#pragma unroll
                        for (int v = 0; v < 8; ++v) {
                            const float4 f = __ldg(xp + v);
                            xr[mt][4 * v + 0] = f.x;
                            xr[mt][4 * v + 1] = f.y;
                            xr[mt][4 * v + 2] = f.z;
                            xr[mt][4 * v + 3] = f.w;
                        }
                    }
                }
                const uint8_t *qp = sb + r * ROWB + b * Q8_QK;
                const uint4 q0 = *reinterpret_cast<const uint4 *>(qp);
                const uint4 q1 = *reinterpret_cast<const uint4 *>(qp + 16);
                const uint32_t wq[8] = {q0.x ^ 0x80808080u, q0.y ^ 0x80808080u, q0.z ^ 0x80808080u,
                                        q0.w ^ 0x80808080u, q1.x ^ 0x80808080u, q1.y ^ 0x80808080u,
                                        q1.z ^ 0x80808080u, q1.w ^ 0x80808080u};
                float t[MT];
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
                    t[mt] = 0.0f;
#pragma unroll
                for (int i = 0; i < Q8_QK; ++i) {
                    const float qf = q_to_f32(wq[i >> 2], i & 3);
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt)
                        t[mt] = __fmaf_rn(qf, xr[mt][i], t[mt]);
                }
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
                    Tb[(mt * R + r) * TPAD + b] = t[mt];
                const __half dh = *reinterpret_cast<const __half *>(sb + r * ROWB + KC + 2 * b);
                TDb[r * TPAD + b] = __half2float(dh);
            }
            mbar_arrive(&tfull[tb]);
        }
    } else {
        // ---------------------------------------------------------------- chain + copy warp
        const int lane = tid - NC;
        const uint64_t pol = policy_evict_first();
        StageIter pit, cit;
        pit.start(p);
        cit.start(p);
        int issued = 0;
        if (lane == 0) {
            for (; issued < STAGES - 1 && pit.valid(p); ++issued, pit.next(p))
                issue_stage(p, pit, slots + size_t(issued % STAGES) * SLOT, &full[issued % STAGES], pol);
        }
        const int mt = lane / R, r = lane % R;
        float acc = 0.0f;
        bool ok = true;
        for (int s = 0; cit.valid(p); cit.next(p), ++s) {
            if (lane == 0 && pit.valid(p)) {
                const int ns = s + STAGES - 1; // its slot last held stage s-1, consumed already
                issue_stage(p, pit, slots + size_t(ns % STAGES) * SLOT, &full[ns % STAGES], pol);
                pit.next(p);
                ++issued;
            }
            __syncwarp();
            const int tb = s & 1;
            if (!mbar_wait(&tfull[tb], (s >> 1) & 1)) {
                report(p.err, ERR_TIMEOUT_TFULL);
                ok = false;
                break;
            }
            const GemvJob &J = p.job[cit.job];
            const int lt = cit.g - J.tile0;
            const int nbk = min(KC, J.cols - cit.c * KC) / Q8_QK;
            const StageRow sr = stage_row(J, lt, r);
            const bool mine = mt < J.m && sr.load;
            if (cit.c == 0)
                acc = 0.0f;
            if (mine) {
                const float *tp = T + tb * MT * R * TPAD + (mt * R + r) * TPAD;
                const float *dp = TD + tb * R * TPAD + r * TPAD;
#pragma unroll 8
                for (int b = 0; b < nbk; ++b)
                    acc = __fmaf_rn(tp[b], dp[b], acc);
            }
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&tempty[tb]);
            if (cit.c == cit.nchunk - 1) {
                if (J.w2) {
                    const float up = __shfl_down_sync(0xffffffffu, acc, R / 2);
                    if (mine && r < R / 2) {
                        const float silu = acc / (1.0f + expf(-acc));
                        J.y[mt * J.ldy + sr.o] = silu * up;
                    }
                } else if (mine) {
                    J.y[mt * J.ldy + sr.o] = acc;
                } else if (mt < J.m && sr.valid) { // a gather index outside the matrix
                    J.y[mt * J.ldy + sr.o] = __int_as_float(0x7fc00000);
                    report(p.err, ERR_BAD_JOB);
                }
            }
        }
        // Leave no bulk copy in flight: on the normal path every issued stage was consumed; after
        // a timeout, wait (bounded) for the most recent use of each slot.
        if (!ok && lane == 0) {
            for (int k = max(0, issued - STAGES); k < issued; ++k)
                if (!mbar_wait(&full[k % STAGES], (k / STAGES) & 1))
                    report(p.err, ERR_TIMEOUT_DRAIN);
        }
    }
}

template <int MT>
cudaError_t launch_mt(const GemvParams &p, int grid, cudaStream_t stream) {
    const size_t smem = smem_bytes<MT>();
    static bool attr_set = false; // per process; the attribute is per function
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(gemv_exact_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        if (e != cudaSuccess)
            return e;
        attr_set = true;
    }
    gemv_exact_kernel<MT><<<grid, NT, smem, stream>>>(p);
    return cudaGetLastError();
}

} // namespace

cudaError_t launch_gemv(GemvParams &p, int num_sms, int grid_limit, cudaStream_t stream) {
    if (p.njobs < 1 || p.njobs > MAX_JOBS)
        return cudaErrorInvalidValue;
    const int m = p.job[0].m;
    int tiles = 0;
    for (int j = 0; j < p.njobs; ++j) {
        GemvJob &J = p.job[j];
        if (J.m != m || J.m < 1 || J.m > GEMV_MAX_T || J.cols < Q8_QK || J.cols % Q8_QK || J.rows < 1)
            return cudaErrorInvalidValue;
        const long long rpt = J.w2 ? R / 2 : R;
        J.tiles = int((J.rows + rpt - 1) / rpt);
        J.tile0 = tiles;
        tiles += J.tiles;
    }
    p.total_tiles = tiles;
    int grid = num_sms > 0 ? num_sms : 148;
    if (grid_limit > 0 && grid > grid_limit)
        grid = grid_limit;
    if (grid > tiles)
        grid = tiles;
    switch (m) {
    case 1: return launch_mt<1>(p, grid, stream);
    case 2: return launch_mt<2>(p, grid, stream);
    case 3: return launch_mt<3>(p, grid, stream);
    default: return launch_mt<4>(p, grid, stream);
    }
}

} // namespace q8
