// q8_gemv.cu: the exact Q8_0 product on CUDA cores, for t = 1..4 tokens per pass. Behind
// rt_gemv / rt_gemv_q / rt_gemm(_q) at t < 16, the fused SwiGLU pair and the row gather.
//
// Arithmetic. Output row o of token t is the reference's exact rounding sequence
// (src/card/gemv.c:93-111, gemm.c keeps every token on it: src/card/gemm.h:6-7):
//     acc = +0; for each 32-column block b in order:
//         t_b = +0; for i = 0..31: t_b = fma(q_i, x_i, t_b);   acc = fma(t_b, fp16 d_b, acc)
// int8 -> fp32 and fp16 -> fp32 are exact and every fma is one IEEE fp32 rounding (the packed
// f32x2 forms round each lane alone), so each y is the reference host model's value, bit for bit.
//
// Mapping. A row tile is R = 8 rows x all cols, streamed through shared memory in stages of
// 8 rows x 4096 columns by 1-D bulk copies (one per row, two where a row is longer than a stage).
//   warps 0-7  compute: thread j owns 32-column block j % 128 and row half j / 128 of the stage;
//              it keeps that block's x in registers, pulls its 4 rows' 32 quants and scales out
//              of the slot (then frees the slot) and runs the 4 rows' 32-fma chains side by side
//              (packed in row pairs); the t_b and fp32 scales go to a partial-sum buffer. Two
//              warps per SM sub-partition, each on a ~5 KB loop body, keep the issue slots busy;
//   warp 8     chain: one lane per (token, row) runs acc = fma(t_b, d_b, acc) in block order
//              and writes y (for a SwiGLU pair: silu(gate) * up);
//   warp 9     copies: issues a stage's bulk copies as soon as its slot is free.
// Barriers: full (copies landed), empty (slot read), tfull/tempty (partial sums). Every wait is
// bounded: a timeout sets a bit in the context's error word and the CTA leaves.
#include <cuda_fp16.h>

#include "q8_kernels.h"
#include "q8_layout.h"
#include "q8_ptx.cuh"

namespace q8 {
namespace {

constexpr int R = 8;               // rows per tile / stage
constexpr int KC = 4096;           // columns per stage
constexpr int NBK = KC / Q8_QK;    // blocks per stage: 128
constexpr int STAGES = 4;
constexpr int TBUF = 4;            // partial-sum buffers: compute may run this far ahead of the chain
constexpr int NC = 256;            // compute threads: (block column, row half) each
constexpr int NH = R / 2;          // rows per compute thread
constexpr int CHAIN_WARP = NC / 32, COPY_WARP = CHAIN_WARP + 1;
constexpr int NT = NC + 64;
constexpr int ROWB = KC + NBK * 2; // a row's slot: quants then scales, 4352 B
constexpr int SLOT = R * ROWB;
constexpr int TPAD = NBK + 1;      // partial-sum row stride (floats): conflict-free per lane = row
static_assert(NC == 2 * NBK, "two compute threads (row halves) per block column of a stage");
static_assert(ROWB % 16 == 0 && SLOT % 16 == 0, "bulk copy destinations are 16-byte aligned");

template <int MT>
constexpr size_t smem_bytes() {
    return size_t(STAGES) * SLOT + size_t(TBUF) * (MT + 1) * R * TPAD * 4 + (STAGES * 2 + TBUF * 2) * 8;
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
    StageRow sr[R];
    uint32_t total = 0;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        sr[r] = stage_row(J, lt, r);
        if (sr[r].load)
            total += whole ? uint32_t(rb) : qbytes + dbytes;
    }
    mbar_arrive_expect_tx(bar, total);
#pragma unroll
    for (int r = 0; r < R; ++r) {
        if (!sr[r].load)
            continue;
        const uint8_t *src = sr[r].mat + sr[r].src * rb;
        uint8_t *dst = slot_base + r * ROWB;
        if (whole) {
            bulk_g2s(dst, src, uint32_t(rb), bar, pol);
        } else {
            bulk_g2s(dst, src + c0, qbytes, bar, pol);
            bulk_g2s(dst + KC, src + J.cols + (c0 / Q8_QK) * 2, dbytes, bar, pol);
        }
    }
}

// Rows processed side by side by one compute thread: its 4 for one or two tokens; 2 at a time
// for three or four (the x registers grow with the tokens).
template <int MT>
constexpr int row_group() { return MT <= 2 ? NH : NH / 2; }

// The RG rows' 32-step chains of one block for MT tokens. MT == 1: rows in packed pairs
// (fma.rn.f32x2 and add.rn.f32x2: two independent IEEE operations). MT > 1: scalar.
template <int MT, int RG>
__device__ __forceinline__ void block_chains(const uint32_t (&wq)[RG][8], const float (&xr)[MT][Q8_QK],
                                             float (&t)[MT][RG]) {
    if constexpr (MT == 1) {
        float2 tp[RG / 2];
#pragma unroll
        for (int p = 0; p < RG / 2; ++p)
            tp[p] = make_float2(0.0f, 0.0f);
        const float2 bias = make_float2(-8388736.0f, -8388736.0f);
#pragma unroll
        for (int i = 0; i < Q8_QK; ++i) {
            const float2 xx = make_float2(xr[0][i], xr[0][i]);
#pragma unroll
            for (int p = 0; p < RG / 2; ++p) {
                // 2^23 + (q + 128) for the two rows, then minus 2^23 + 128: exact q
                const float2 m =
                    make_float2(__uint_as_float(__byte_perm(wq[2 * p][i >> 2], 0x4B000000u, 0x7650u + (i & 3))),
                                __uint_as_float(__byte_perm(wq[2 * p + 1][i >> 2], 0x4B000000u, 0x7650u + (i & 3))));
                tp[p] = __ffma2_rn(__fadd2_rn(m, bias), xx, tp[p]);
            }
        }
#pragma unroll
        for (int p = 0; p < RG / 2; ++p) {
            t[0][2 * p] = tp[p].x;
            t[0][2 * p + 1] = tp[p].y;
        }
    } else {
#pragma unroll
        for (int r = 0; r < RG; ++r)
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
                t[mt][r] = 0.0f;
#pragma unroll
        for (int i = 0; i < Q8_QK; ++i)
#pragma unroll
            for (int r = 0; r < RG; ++r) {
                const float qf = q_to_f32(wq[r][i >> 2], i & 3);
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
                    t[mt][r] = __fmaf_rn(qf, xr[mt][i], t[mt][r]);
            }
    }
}

template <int MT>
__global__ void __launch_bounds__(NT, 1) gemv_exact_kernel(const __grid_constant__ GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *slots = smem;
    float *T = reinterpret_cast<float *>(smem + size_t(STAGES) * SLOT); // [TBUF][MT][R][TPAD]
    float *TD = T + TBUF * MT * R * TPAD;                                 // [TBUF][R][TPAD]
    uint64_t *full = reinterpret_cast<uint64_t *>(TD + TBUF * R * TPAD);  // [STAGES]
    uint64_t *empty = full + STAGES;                                      // [STAGES]
    uint64_t *tfull = empty + STAGES;                                     // [TBUF]
    uint64_t *tempty = tfull + TBUF;                                      // [TBUF]
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NC);
        }
        for (int b = 0; b < TBUF; ++b) {
            mbar_init(&tfull[b], NC);
            mbar_init(&tempty[b], 1);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp < CHAIN_WARP) {
        // ---------------------------------------------------------------- compute threads
        float xr[MT][Q8_QK];
        int xjob = -1, xc = -1;
        StageIter it;
        it.start(p);
        for (int s = 0; it.valid(p); it.next(p), ++s) {
            const int slot = s % STAGES, tb = s % TBUF;
            if (!mbar_wait(&full[slot], (s / STAGES) & 1)) {
                report(p.err, ERR_TIMEOUT_FULL);
                break;
            }
            const GemvJob &J = p.job[it.job];
            const int c0 = it.c * KC;
            const int nbk = min(KC, J.cols - c0) / Q8_QK;
            const int b = tid % NBK, half = tid / NBK;
            const bool active = b < nbk;
            if (active && (it.c != xc || it.job != xjob)) {
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
            constexpr int RG = row_group<MT>();
            const uint8_t *qbase = slots + size_t(slot) * SLOT + b * Q8_QK; // row r's block b: + r*ROWB
            const uint8_t *dbase = slots + size_t(slot) * SLOT + KC + 2 * b; // row r's scale b: + r*ROWB
            float *Tb = T + tb * MT * R * TPAD;
            float *TDb = TD + tb * R * TPAD;
            bool ok = true;
#pragma unroll
            for (int g = 0; g < NH / RG; ++g) {
                uint32_t wq[RG][8];
                float dv[RG];
                if (active) {
#pragma unroll
                    for (int k = 0; k < RG; ++k) {
                        const int r = half * NH + g * RG + k;
                        const uint4 q0 = *reinterpret_cast<const uint4 *>(qbase + r * ROWB);
                        const uint4 q1 = *reinterpret_cast<const uint4 *>(qbase + r * ROWB + 16);
                        wq[k][0] = q0.x ^ 0x80808080u;
                        wq[k][1] = q0.y ^ 0x80808080u;
                        wq[k][2] = q0.z ^ 0x80808080u;
                        wq[k][3] = q0.w ^ 0x80808080u;
                        wq[k][4] = q1.x ^ 0x80808080u;
                        wq[k][5] = q1.y ^ 0x80808080u;
                        wq[k][6] = q1.z ^ 0x80808080u;
                        wq[k][7] = q1.w ^ 0x80808080u;
                        dv[k] = __half2float(*reinterpret_cast<const __half *>(dbase + r * ROWB));
                    }
                }
                if (g == NH / RG - 1)
                    mbar_arrive(&empty[slot]); // the slot's bytes are in registers: refill it
                if (g == 0 && s >= TBUF && !mbar_wait(&tempty[tb], ((s / TBUF) - 1) & 1)) {
                    report(p.err, ERR_TIMEOUT_TEMPTY);
                    ok = false;
                    break;
                }
                if (active) {
                    float t[MT][RG];
                    block_chains<MT, RG>(wq, xr, t);
#pragma unroll
                    for (int k = 0; k < RG; ++k) {
                        const int r = half * NH + g * RG + k;
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt)
                            Tb[(mt * R + r) * TPAD + b] = t[mt][k];
                        TDb[r * TPAD + b] = dv[k];
                    }
                }
            }
            if (!ok)
                break;
            mbar_arrive(&tfull[tb]);
        }
    } else if (warp == CHAIN_WARP) {
        // ---------------------------------------------------------------- chain warp
        const int mt = lane / R, r = lane % R;
        float acc = 0.0f;
        StageIter it;
        it.start(p);
        for (int s = 0; it.valid(p); it.next(p), ++s) {
            const int tb = s % TBUF;
            if (!mbar_wait(&tfull[tb], (s / TBUF) & 1)) {
                report(p.err, ERR_TIMEOUT_TFULL);
                break;
            }
            const GemvJob &J = p.job[it.job];
            const int lt = it.g - J.tile0;
            const int nbk = min(KC, J.cols - it.c * KC) / Q8_QK;
            const StageRow sr = stage_row(J, lt, r);
            const bool mine = mt < J.m && sr.load;
            if (it.c == 0)
                acc = 0.0f;
            if (mine) {
                const float *tp = T + tb * MT * R * TPAD + (mt * R + r) * TPAD;
                const float *dp = TD + tb * R * TPAD + r * TPAD;
                int b = 0;
                for (; b + 16 <= nbk; b += 16) { // loads first, then the 16 dependent fmas
                    float tv[16], dd[16];
#pragma unroll
                    for (int k = 0; k < 16; ++k) {
                        tv[k] = tp[b + k];
                        dd[k] = dp[b + k];
                    }
#pragma unroll
                    for (int k = 0; k < 16; ++k)
                        acc = __fmaf_rn(tv[k], dd[k], acc);
                }
                for (; b < nbk; ++b)
                    acc = __fmaf_rn(tp[b], dp[b], acc);
            }
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&tempty[tb]);
            if (it.c == it.nchunk - 1) {
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
    } else if (lane == 0) {
        // ---------------------------------------------------------------- copy issuer
        const uint64_t pol = policy_evict_first();
        StageIter it;
        it.start(p);
        int s = 0;
        bool ok = true;
        for (; it.valid(p); it.next(p), ++s) {
            const int slot = s % STAGES;
            if (s >= STAGES && !mbar_wait(&empty[slot], ((s / STAGES) - 1) & 1)) {
                report(p.err, ERR_TIMEOUT_FULL);
                ok = false;
                break;
            }
            issue_stage(p, it, slots + size_t(slot) * SLOT, &full[slot], pol);
        }
        // Leave no bulk copy in flight: on the normal path the compute threads consumed every
        // stage; after a timeout, wait (bounded) for the most recent fill of each slot.
        if (!ok)
            for (int k = max(0, s - STAGES); k < s; ++k)
                if (!mbar_wait(&full[k % STAGES], (k / STAGES) & 1))
                    report(p.err, ERR_TIMEOUT_DRAIN);
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
