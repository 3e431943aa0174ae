// q8_gemm_tc.cu: the Q8_0 product for t >= 16 tokens on the 5th-generation tensor cores.
//
// Y[t][o] = sum_k fp16(q[o][k] * d[o][k/32]) * fp16(x[t][k]), fp32 sums in TMEM.
//
// At 16+ tokens the product is a dense contraction (the reference batches prompts of 16 and
// verify passes of K+1 tokens through the same weight pass, src/card/gemm.c:271-294). The
// per-(row, 32-column) fp16 scale d cannot be factored out of a K contraction, so each weight tile
// is dequantised to fp16 first, into tensor memory as the MMA's A operand: q is exact in fp16, and
// fl16(q*d) rounds once.
// x is rounded to fp16 once per call (a pre-pass into scratch). fp16 rather than bf16: the same
// tcgen05 kind::f16 rate with 3 more mantissa bits, which is what holds the product within the
// stated 2e-3 (bf16 tiles measure ~1e-2 on the BASELINE shapes).
// fp16's range is narrow (normal from 2^-14, finite below 65504) while the reference takes any
// fp32 x and any fp16 scale (src/card/gemm.c:271-294). So both operands are scaled by powers of
// two into the middle of that range before rounding: token t's x by 2^s_t, with |x| <= 2^15 at
// its largest entry, and row o's weights by 2^r_o, with 127 * (the row's largest scale) in
// [2^14, 2^15). The accumulator then holds y * 2^(r_o + s_t), and the epilogue multiplies by
// 2^-r_o and 2^-s_t, which is exact. Where nothing under- or overflowed the fp16 operands are the
// unscaled ones' bits with a shifted exponent, so the product rounds exactly as it did unscaled.
// The pre-pass that rounds x also finds the factors (tc_prep_kernel).
//
// A CTA (persistent; one per SM owning all 512 TMEM columns, or two per SM with 256 each for
// tiles of up to 64 tokens: TcShape below) runs 128-row x BN-token tiles (a SwiGLU pair's tile:
// 64 rows of the gate matrix and the same 64 rows of the up matrix). The roles, for one CTA per SM:
//   warp 12     TMA: per 64-column stage, the quant box (128 rows x 64 B, 64B swizzle), the scale
//               box (128 rows x 8 scales) and the fp16 x box (BN rows x 128 B, 128B swizzle), into
//               a ring of S <= 8 shared-memory stages;
//   warps 4-11  dequant: thread (i, h) turns row i's 32 quants of block h and its scale into 32
//               fp16 weights and stores them (tcgen05.st) into TMEM lane i of the A ring, one A
//               slot per shared stage;
//   warp 13     MMA: 4 x tcgen05.mma (M=128, N=BN, K=16, A from TMEM, B = the x box) per stage;
//               one tcgen05.commit per stage frees the shared stage and with it the A slot, and at
//               a tile's end another frees the accumulator;
//   warps 0-3,  epilogue: tcgen05.ld of TMEM lanes 32*(warp%4).. -> y (or silu(g)*u for a pair);
//   14-25       four warps per lane quarter, each on a quarter of the tile's token columns.
// A pair's tile interleaves its two matrices by TMEM lane: lanes 32e..32e+15 hold gate rows
// 16e..16e+15 and lanes 32e+16..32e+31 the same up rows, so one warp holds both factors of its
// 16 output rows and combines them with a lane exchange (shfl.xor 16).
// A stays out of shared memory: the stage's traffic there is the bulk copies in, the dequant's
// quant reads and the tensor core's reads of x (writing A to shared memory and reading it back
// made the kernel shared-memory bound at ~1000 cycles per 64-column stage).
// The MMA thread is the critical issuer: a barrier wait stalls it ~200 cycles and a commit ~70
// (measured), with only about four MMAs queued behind it. So it waits once per stage, on the A
// slot's barrier only: the dequant threads arrive there after waiting for the stage's copies, so
// the stage's x box has landed too; and the A slot needs no barrier of its own, because the
// producer refills a shared stage only after its MMAs completed, and the dequant writes the slot
// only after that refill landed.
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
constexpr int PAIR_ROWS = BM / 2; // output rows per tile of a SwiGLU pair
constexpr int MAX_STAGES = 8;
// Tensor memory (128 lanes x 512 columns of 32 bits per SM): the accumulators first, then the
// dequantised A tiles in a ring of one 32-column slot per shared stage (a 128 x 64 fp16 tile:
// lane = row, column j = k 2j and 2j+1). How the columns are shared out: TcShape.
constexpr int A_COLS = BK / 2;

// The CTA's shape: CPS CTAs per SM, each owning 512 / CPS TMEM columns.
//   CPS = 1 (tiles of up to 256 tokens): 26 warps, 8 dequant (two per SM sub-partition, each on
//     one 32-column block of a stage), 16 epilogue (four per TMEM lane quarter, each on a quarter
//     of the tile's columns: the drain holds the next tile's MMAs, and a SwiGLU pair's exchange
//     and SiLU make it longer); accumulators in columns [0, 256) (two of 128 columns, double-
//     buffered, for tiles of <= 128 tokens, else one of 256), up to 8 A slots from 256.
//   CPS = 2 (tiles of up to 64 tokens): 10 warps, 4 dequant (each thread both blocks of its row),
//     4 epilogue; accumulators at columns 0 and 32 (tiles of <= 32 tokens) or 0 and 64, the A
//     slots from the next 32-column boundary (6 of them for tiles of <= 32 tokens, else 4: the
//     ring's depth is what bounds these small tiles, whose stages wait on DRAM latency). Two CTAs
//     share an SM and
//     its tensor core: at N <= 64 an MMA instruction takes ~46 cycles while each wait in the
//     issuing thread stalls it ~200, so a second issuer keeps the pipe fed.
constexpr int MAX_BN_TWO_CTAS = 64; // the two-CTA shape's tiles: two accumulators of up to 64 columns

template <int CPS>
struct TcShape {
    static constexpr int EPQ = CPS == 1 ? 4 : 1; // epilogue warps per TMEM lane quarter
    static constexpr int NDQ = 8 / CPS, EPI_WARPS = 4 * EPQ;
    static constexpr int DQ_WARP0 = 4, TMA_WARP = DQ_WARP0 + NDQ, MMA_WARP = TMA_WARP + 1;
    static constexpr int NT = 32 * (MMA_WARP + 1 + EPI_WARPS - 4); // epilogue: warps 0-3 (+ after MMA_WARP)
    static constexpr int TMEM_COLS = 512 / CPS, ACC_COLS = 256 / CPS;
    static constexpr int BLOCKS_PER_THREAD = 2 / (NDQ / 4); // 32-column blocks per dequant thread per stage
};
// Shared memory per stage (1024-aligned): the quant box (128 rows x 64 B, 64B swizzle), the scale
// box (128 rows x 8 fp16), the fp16 x box (bn rows x 128 B, 128B swizzle).
constexpr int OFF_Q = 0, OFF_D = 8192, OFF_X = 10240;
constexpr size_t SMEM_LIMIT = 224 * 1024;   // one CTA per SM: stages + barriers (the launch adds 1 KB of alignment)
constexpr size_t SMEM_LIMIT_2 = 110 * 1024; // two CTAs per SM

__host__ __device__ constexpr int stage_bytes(int bn) { return (OFF_X + bn * 128 + 1023) / 1024 * 1024; }
__host__ __device__ constexpr int n_acc(int bn, int cps) { return bn <= 128 / cps ? 2 : 1; }

struct TcJobDev {
    CUtensorMap tq, td, tq2, td2; // quants and scales of W (and of the SwiGLU up matrix)
    const int8_t *rexp;           // r_o per row: W's rows, then (a pair) the up matrix's rows
    const float *tokf;            // 2^-s_t per token
    float *y;
    float *part;                  // split-K partial sums as [plane][t][rows]: plane = (up ? ks : 0) + K part
    long long rows, ldy;
    int cols, t, pair, n_pass, tiles, unit0; // tiles: row tiles (of BM rows, PAIR_ROWS for a pair); units = tiles * n_pass * ks
    int ks;                                  // K parts (1: no split, the epilogue writes y)
};

struct TcParams {
    CUtensorMap tx[8];   // fp16 x per job
    TcJobDev job[8];
    int njobs, total_units, bn, stages;
    int a_base;     // TMEM column of the first A slot (after the accumulators)
    int acc_stride; // TMEM columns from the first accumulator to the second
    unsigned *err;
};

// The fp16 copy of x is written by the conversion kernel just before this one on the stream: every
// thread waits for it (griddepcontrol.wait, a no-op without programmatic launch) before the roles
// start.

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

// D[tmem] (+)= A[tmem] * B[smem descriptor]: M = 128, N from idesc, K = 16.
__device__ __forceinline__ void tc_mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(db), "r"(idesc), "r"(acc));
}

// 16 consecutive 32-bit columns of this thread's TMEM lane (the warp's 32-lane quarter).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

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

// A unit: row tile `rt`, token pass `np` and K part `kp` (64-column blocks kb0..kb1-1) of job `j`:
// one MMA tile.
struct Unit {
    int j, rt, np, kp, kb0, kb1;
};

__device__ __forceinline__ Unit unit_of(const TcParams &p, int u) {
    Unit w;
    w.j = find_job(p, u);
    const TcJobDev &J = p.job[w.j];
    const int lu = u - J.unit0;
    const int per_rt = J.n_pass * J.ks;
    w.rt = lu / per_rt;
    const int rem = lu - w.rt * per_rt;
    w.np = rem / J.ks;
    w.kp = rem - w.np * J.ks;
    const int nks = (J.cols + BK - 1) / BK;
    w.kb0 = int((long long)w.kp * nks / J.ks);
    w.kb1 = int((long long)(w.kp + 1) * nks / J.ks);
    return w;
}

// A role's position in the stage ring: slot and the parity of its current use.
struct Ring {
    int slot = 0;
    uint32_t phase = 0;
    __device__ __forceinline__ void next(int S) {
        if (++slot == S) {
            slot = 0;
            phase ^= 1u;
        }
    }
};

// 2^k as a float, for k in [-126, 127] (a normal number: exact).
__device__ __forceinline__ float pow2i(int k) { return __int_as_float((127 + k) << 23); }

// The fp16 scale of a row for its weights: 127 * dmax * 2^r in [2^14, 2^15), r in [-9, 31] for
// every finite nonzero fp16 dmax (given as its bits without the sign); 0 for a zero or
// non-finite maximum (an inf or NaN scale then propagates as in the reference).
__device__ __forceinline__ int row_exponent(unsigned dmax_bits) {
    if (dmax_bits == 0 || dmax_bits >= 0x7c00u)
        return 0;
    int e;
    frexpf(127.0f * __half2float(__ushort_as_half(uint16_t(dmax_bits))), &e); // value in [2^(e-1), 2^e)
    return 15 - e;
}

template <int CPS>
__global__ void __launch_bounds__(TcShape<CPS>::NT, CPS) gemm_tc_kernel(const __grid_constant__ TcParams p) {
    using Sh = TcShape<CPS>;
    constexpr int NDQ = Sh::NDQ, EPI_WARPS = Sh::EPI_WARPS, DQ_WARP0 = Sh::DQ_WARP0, TMA_WARP = Sh::TMA_WARP,
                  MMA_WARP = Sh::MMA_WARP, TMEM_COLS = Sh::TMEM_COLS;
    const int A_BASE = p.a_base;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int S = p.stages, BN = p.bn, SB = stage_bytes(BN), NACC = n_acc(BN, CPS), ACC_STRIDE = p.acc_stride;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + size_t(S) * SB); // [S]: TMA landed
    uint64_t *empty = full + MAX_STAGES;                                   // [S]: the stage's MMAs done
    uint64_t *afull = empty + MAX_STAGES;                                  // [S]: the stage's A slot in TMEM
    uint64_t *accfull = afull + MAX_STAGES;                                // [2]
    uint64_t *accempty = accfull + 2;                                      // [2]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accempty + 2);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            mbar_init(&afull[s], 32 * NDQ);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&accfull[b], 1);
            mbar_init(&accempty[b], 32 * EPI_WARPS);
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

    if (warp == TMA_WARP) {
        // ---------------------------------------------------------------- producer
        if (lane == 0) {
            int s = 0;
            Ring ring;
            bool ok = true;
            for (int u = blockIdx.x; u < p.total_units && ok; u += gridDim.x) {
                const Unit w = unit_of(p, u);
                const TcJobDev &J = p.job[w.j];
                for (int kb = w.kb0; kb < w.kb1; ++kb, ++s, ring.next(S)) {
                    const int slot = ring.slot;
                    if (s >= S && !mbar_wait(&empty[slot], ring.phase ^ 1)) {
                        report(p.err, ERR_TIMEOUT_MMA);
                        ok = false;
                        break;
                    }
                    uint8_t *st = smem + size_t(slot) * SB;
                    mbar_arrive_expect_tx(&full[slot], uint32_t(BM * 64 + BM * 16 + BN * 128));
                    const int k0 = kb * BK, ks0 = (k0 / Q8_QK) & ~7;
                    if (J.pair) { // 64 gate rows, then the same 64 up rows (maps of 64-row boxes)
                        tma_load_2d(st + OFF_Q, &J.tq, k0, w.rt * PAIR_ROWS, &full[slot]);
                        tma_load_2d(st + OFF_Q + PAIR_ROWS * 64, &J.tq2, k0, w.rt * PAIR_ROWS, &full[slot]);
                        tma_load_2d(st + OFF_D, &J.td, ks0, w.rt * PAIR_ROWS, &full[slot]);
                        tma_load_2d(st + OFF_D + PAIR_ROWS * 16, &J.td2, ks0, w.rt * PAIR_ROWS, &full[slot]);
                    } else {
                        tma_load_2d(st + OFF_Q, &J.tq, k0, w.rt * BM, &full[slot]);
                        tma_load_2d(st + OFF_D, &J.td, ks0, w.rt * BM, &full[slot]);
                    }
                    tma_load_2d(st + OFF_X, &p.tx[w.j], k0, w.np * BN, &full[slot]);
                }
            }
            // leave no copy in flight: wait for the most recent fill of every slot
            for (int q = max(0, s - S); q < s; ++q)
                if (!mbar_wait(&full[q % S], (q / S) & 1))
                    report(p.err, ERR_TIMEOUT_DRAIN);
        }
    } else if (warp >= DQ_WARP0 && warp < DQ_WARP0 + NDQ) {
        // ---------------------------------------------------------------- dequant -> TMEM
        const int i = (threadIdx.x - DQ_WARP0 * 32) % BM; // tile row = this thread's TMEM lane
        const int h0 = (threadIdx.x - DQ_WARP0 * 32) / BM * Sh::BLOCKS_PER_THREAD; // its first 32-column block
        const uint32_t lane_base = uint32_t(32 * (warp % 4)) << 16;
        const __half2 bias = __half2half2(__ushort_as_half(uint16_t(0x6480))); // 1152
        Ring ring;
        bool ok = true;
        // a pair's tile: lane 32e+l reads shared row 16e+l (gate, l < 16) or 64+16e+l-16 (up)
        const int ipair = (i & 16) ? PAIR_ROWS + 16 * (i >> 5) + (i & 15) : 16 * (i >> 5) + (i & 15);
        // this lane's weight row exponent r_o, loaded one unit ahead (its latency then hides
        // behind a unit's stages)
        auto row_exp = [&](int u) -> int {
            if (u >= p.total_units)
                return 0;
            const Unit w = unit_of(p, u);
            const TcJobDev &J = p.job[w.j];
            const long long row = J.pair ? (long long)w.rt * PAIR_ROWS + 16 * (i >> 5) + (i & 15)
                                         : (long long)w.rt * BM + i;
            if (row >= J.rows)
                return 0; // a tail tile's missing rows: zeros from the copy
            return J.rexp[(J.pair && (i & 16)) ? J.rows + row : row];
        };
        int rx_next = row_exp(blockIdx.x);
        for (int u = blockIdx.x; u < p.total_units && ok; u += gridDim.x) {
            const Unit w = unit_of(p, u);
            const int r = p.job[w.j].pair ? ipair : i; // the shared-memory row behind this lane
            const float rowf = pow2i(rx_next);
            rx_next = row_exp(u + gridDim.x);
            for (int kb = w.kb0; kb < w.kb1; ++kb, ring.next(S)) {
                const int slot = ring.slot; // also the A slot
                if (!mbar_wait(&full[slot], ring.phase)) {
                    report(p.err, ERR_TIMEOUT_FULL);
                    ok = false;
                    break;
                }
                const uint8_t *st = smem + size_t(slot) * SB;
                // the A slot is free: the MMAs of its previous use completed before the producer
                // refilled this shared stage, whose copies have landed
                tc_fence_after();
#pragma unroll
                for (int hb = 0; hb < Sh::BLOCKS_PER_THREAD; ++hb) {
                    const int h = h0 + hb;
                    // this block's scale (one of the 8 the scale box holds) times 2^r_o (exact
                    // while the result is a normal fp16), and its 32 quants
                    const __half2 dd2 = __half2half2(__float2half_rn(
                        __half2float(*reinterpret_cast<const __half *>(st + OFF_D + r * 16 + ((kb * 2 + h) & 7) * 2)) *
                        rowf));
                    uint32_t outw[16];
#pragma unroll
                    for (int cc = 0; cc < 2; ++cc) { // 16 quants per chunk; chunks 2h, 2h+1
                        const int c = 2 * h + cc;
                        const uint4 qv =
                            *reinterpret_cast<const uint4 *>(st + OFF_Q + r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
                        const uint32_t wq[4] = {qv.x ^ 0x80808080u, qv.y ^ 0x80808080u, qv.z ^ 0x80808080u,
                                                qv.w ^ 0x80808080u};
#pragma unroll
                        for (int v = 0; v < 4; ++v) {
                            // (q+128) as the low byte of fp16 1024+(q+128): exact; minus 1152 -> q
                            const uint32_t lo = __byte_perm(wq[v], 0x64646464u, 0x4140u);
                            const uint32_t hi = __byte_perm(wq[v], 0x64646464u, 0x4342u);
                            __half2 a = __hmul2(__hsub2(*reinterpret_cast<const __half2 *>(&lo), bias), dd2);
                            __half2 b = __hmul2(__hsub2(*reinterpret_cast<const __half2 *>(&hi), bias), dd2);
                            outw[8 * cc + 2 * v] = *reinterpret_cast<uint32_t *>(&a);
                            outw[8 * cc + 2 * v + 1] = *reinterpret_cast<uint32_t *>(&b);
                        }
                    }
                    tmem_st16(tmem + lane_base + uint32_t(A_BASE + slot * A_COLS + 16 * h), outw);
                }
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(&afull[slot]);
            }
        }
    } else if (warp == MMA_WARP) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = idesc_f16(BN);
            int s = 0, tcount = 0;
            Ring ring;
            // descriptors of slot 0's x box and A slot; slot k adds k stages / k A slots
            const uint64_t db0 = sw128_desc(smem + OFF_X);
            const uint32_t ta0 = tmem + uint32_t(A_BASE);
            bool ok = true;
            for (int u = blockIdx.x; u < p.total_units && ok; u += gridDim.x, ++tcount) {
                const Unit w = unit_of(p, u);
                const int b = tcount % NACC, bu = tcount / NACC;
                if (bu > 0 && !mbar_wait(&accempty[b], (bu - 1) & 1)) {
                    report(p.err, ERR_TIMEOUT_MMA);
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t tacc = tmem + uint32_t(b * ACC_STRIDE);
                for (int kb = w.kb0; kb < w.kb1; ++kb, ++s, ring.next(S)) {
                    const int slot = ring.slot;
                    // the dequant threads arrive after waiting for the stage's copies: the x box has
                    // landed too
                    if (!mbar_wait(&afull[slot], ring.phase)) {
                        report(p.err, ERR_TIMEOUT_MMA);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t db = db0 + uint64_t(slot * (SB >> 4)); // start address field, 16-byte units
                    const uint32_t ta = ta0 + uint32_t(slot * A_COLS);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) // K = 16 per MMA: 8 TMEM columns of A, 32 B of B
                        tc_mma_ts(tacc, ta + uint32_t(8 * kk), db + uint64_t(2 * kk), idesc,
                                  (kb != w.kb0 || kk) ? 1u : 0u);
                    tc_commit(&empty[slot]); // frees the shared stage and its A slot
                }
                if (ok)
                    tc_commit(&accfull[b]);
            }
            // drain: the MMAs of the last use of every slot
            for (int q = max(0, s - S); q < s; ++q)
                if (!mbar_wait(&empty[q % S], (q / S) & 1))
                    report(p.err, ERR_TIMEOUT_DRAIN);
        }
    } else {
        // ---------------------------------------------------------------- epilogue
        // Warp e (e = warp % 4) reads TMEM lanes 32e.. (rows 32e..32e+31 of the tile), 16 token
        // columns at a time; the quarter's EPQ warps share the tile's columns in whole 16-column
        // chunks. Each lane stores its row's values with plain stores (for each token the warp
        // writes 32 consecutive floats, one 128-byte segment); this measured faster here than
        // bulk tensor stores through shared-memory staging boxes, which queue behind the loads.
        // The accumulator is handed back as soon as a warp's last columns are in registers.
        // Each value is multiplied back by 2^-r_o (its row) and 2^-s_t (its token) first.
        const int e = warp & 3, eh = warp > MMA_WARP ? 1 + (warp - MMA_WARP - 1) / 4 : 0; // column share
        int tcount = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < p.total_units && ok; u += gridDim.x, ++tcount) {
            const Unit w = unit_of(p, u);
            const TcJobDev &J = p.job[w.j];
            const int b = tcount % NACC;
            // this lane's row exponent, loaded before the wait for the accumulator
            const bool up_lane = J.pair && (lane & 16);
            const long long orow = J.pair ? (long long)w.rt * PAIR_ROWS + 16 * e + (lane & 15)
                                          : (long long)w.rt * BM + 32 * e + lane;
            const float rinv = orow < J.rows ? pow2i(-int(J.rexp[up_lane ? J.rows + orow : orow])) : 1.0f;
            if (!mbar_wait(&accfull[b], (tcount / NACC) & 1)) {
                report(p.err, ERR_TIMEOUT_MMA);
                ok = false;
                break;
            }
            tc_fence_after();
            // this warp's columns: [cbeg, cend), whole 16-column chunks shared out over the
            // quarter's warps (a warp left without one only hands the accumulator back)
            constexpr int EPQ = Sh::EPQ;
            const int nch = BN / 16; // 16-column chunks, split as evenly as they go over the quarter's warps
            const int cbeg = 16 * (nch * eh / EPQ), cend = 16 * (nch * (eh + 1) / EPQ);
            if (cbeg >= cend) {
                tc_fence_before();
                mbar_arrive(&accempty[b]);
            }
            const uint32_t tacc = tmem + (uint32_t(32 * e) << 16) + uint32_t(b * ACC_STRIDE);
            const int n0 = w.np * BN;
            const long long nrows = J.rows;
            const int ntok = J.t;
            const bool split = J.ks > 1; // partial sums to the split-K planes, reduced afterwards
            // this lane's output row (for a pair: lanes l and l+16 hold gate and up of one row)
            const bool up = J.pair && (lane & 16);
            const long long row = J.pair ? (long long)w.rt * PAIR_ROWS + 16 * e + (lane & 15)
                                         : (long long)w.rt * BM + 32 * e + lane;
            for (int c0 = cbeg; c0 < cend; c0 += 16) {
                // the 16 tokens' factors 2^-s_t (1 past the last token: those columns are zero)
                float tf[16];
#pragma unroll
                for (int c = 0; c < 16; ++c)
                    tf[c] = n0 + c0 + c < ntok ? __ldg(J.tokf + n0 + c0 + c) : 1.0f;
                uint32_t r[16];
                tmem_ld16(tacc + uint32_t(c0), r);
                tmem_wait_ld();
                if (c0 + 16 >= cend) { // this warp's share of the accumulator is in registers
                    tc_fence_before();
                    mbar_arrive(&accempty[b]);
                }
                float v[16];
#pragma unroll
                for (int c = 0; c < 16; ++c)
                    v[c] = __uint_as_float(r[c]) * rinv * tf[c];
                if (J.pair && !split) {
                    // y = silu(g) * u: the gate lane finishes tokens c0..c0+7 of its row, the up
                    // lane tokens c0+8..c0+15, each taking the other factor from its partner
                    float g[8], uv[8];
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const float give = up ? v[k] : v[8 + k];
                        const float got = __shfl_xor_sync(0xffffffffu, give, 16);
                        g[k] = up ? got : v[k];
                        uv[k] = up ? v[8 + k] : got;
                    }
                    const int tk0 = n0 + c0 + (up ? 8 : 0);
                    if (row < nrows) {
                        float *yp = J.y + (long long)tk0 * J.ldy + row;
#pragma unroll
                        for (int k = 0; k < 8; ++k)
                            if (tk0 + k < ntok)
                                yp[(long long)k * J.ldy] = g[k] / (1.0f + expf(-g[k])) * uv[k];
                    }
                } else if (row < nrows) {
                    float *yp;
                    long long ld;
                    if (split) { // a pair's gate lanes to the gate planes, its up lanes to the up planes
                        const int plane = (up ? J.ks : 0) + w.kp;
                        yp = J.part + ((long long)plane * ntok + n0 + c0) * nrows + row;
                        ld = nrows;
                    } else {
                        yp = J.y + (long long)(n0 + c0) * J.ldy + row;
                        ld = J.ldy;
                    }
#pragma unroll
                    for (int c = 0; c < 16; ++c)
                        if (n0 + c0 + c < ntok)
                            yp[(long long)c * ld] = v[c];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == MMA_WARP)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
}

// The pre-pass of a job, before its product on the stream. Blocks [0, t): one token each: the
// largest |x| of the token gives s_t (|x| * 2^s_t <= 2^15 at that entry; s_t <= 126), then
// xh = fp16(x * 2^s_t) and tokf[t] = 2^-s_t. Blocks from t: the matrix rows (W's rows, then a
// pair's up rows), a half-warp per row: the row's largest scale gives r_o (row_exponent) into rexp.
constexpr int PREP_THREADS = 256;

// RPB rows per half-warp and batch: 8 where the matrix has rows enough to give every SM a block
// of 16-row warps, else 1 (a few deep blocks on a small matrix leave most SMs idle).
template <int RPB, int HELD>
__global__ void __launch_bounds__(PREP_THREADS) tc_prep_kernel(const float *x, long long ldx, int cols, int t,
                                                               __half *xh, float *tokf, const uint8_t *w,
                                                               const uint8_t *w2, long long rows, int8_t *rexp) {
    // Under programmatic launch the product may start its prologue now; this pass waits for the
    // kernel before it (x is its output, and the scratch written here may still be read by the
    // previous product).
    if (threadIdx.x == 0)
        grid_launch_dependents();
    grid_wait();
    if (blockIdx.x < unsigned(t)) {
        __shared__ float part[PREP_THREADS / 32];
        __shared__ int s_sh;
        const float *xt = x + (long long)blockIdx.x * ldx;
        __half *ht = xh + (long long)blockIdx.x * cols;
        // 16-byte pieces where the row allows, the whole row held in registers between the scan
        // and the conversion (rows of up to HELD * 4 * PREP_THREADS columns; HELD = 4 for rows of
        // 4096 columns or fewer, so that the blocks' registers leave room for more blocks per SM)
        const bool vec = cols % 4 == 0 && (reinterpret_cast<uintptr_t>(xt) & 15) == 0 &&
                         cols <= HELD * 4 * PREP_THREADS;
        float4 v[HELD];
        float amax = 0.0f;
        if (vec) {
            const float4 *x4 = reinterpret_cast<const float4 *>(xt);
#pragma unroll
            for (int q = 0; q < HELD; ++q) {
                const int c = threadIdx.x + q * PREP_THREADS;
                v[q] = c < cols / 4 ? __ldg(x4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int q = 0; q < HELD; ++q)
                amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[q].x), fabsf(v[q].y)), fmaxf(fabsf(v[q].z), fabsf(v[q].w))));
        } else {
            for (int c = threadIdx.x; c < cols; c += PREP_THREADS)
                amax = fmaxf(amax, fabsf(xt[c]));
        }
        for (int o = 16; o; o >>= 1)
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        if (threadIdx.x % 32 == 0)
            part[threadIdx.x / 32] = amax;
        __syncthreads();
        if (threadIdx.x == 0) {
            float m = part[0];
            for (int k = 1; k < PREP_THREADS / 32; ++k)
                m = fmaxf(m, part[k]);
            int sx = 0;
            if (m > 0.0f && m <= 3.4028234663852886e38f) {
                int e;
                frexpf(m, &e); // m in [2^(e-1), 2^e)
                sx = 15 - e;   // m * 2^sx in [2^14, 2^15)
                sx = sx > 126 ? 126 : sx;
            }
            s_sh = sx;
            tokf[blockIdx.x] = pow2i(-sx);
        }
        __syncthreads();
        const float f = pow2i(s_sh);
        if (vec) {
#pragma unroll
            for (int q = 0; q < HELD; ++q) {
                const int c = threadIdx.x + q * PREP_THREADS;
                if (c < cols / 4) {
                    const __half2 lo = __halves2half2(__float2half_rn(v[q].x * f), __float2half_rn(v[q].y * f));
                    const __half2 hi = __halves2half2(__float2half_rn(v[q].z * f), __float2half_rn(v[q].w * f));
                    uint2 u;
                    u.x = *reinterpret_cast<const unsigned *>(&lo);
                    u.y = *reinterpret_cast<const unsigned *>(&hi);
                    *reinterpret_cast<uint2 *>(ht + 4 * c) = u; // (cols % 4 == 0: 8-byte aligned)
                }
            }
        } else {
            for (int c = threadIdx.x; c < cols; c += PREP_THREADS)
                ht[c] = __float2half_rn(xt[c] * f);
        }
        return;
    }
    // The row exponents: a half-warp per row, 16-byte chunks of the row's scales, RPB rows per
    // half-warp at a time so that RPB loads per lane are in flight (a warp per row with one load
    // in flight left this pass latency-bound on large matrices: 28 us on the 151936-row head).
    const long long nrows = w2 ? 2 * rows : rows;
    const long long rb = q8s_row_bytes(cols), nsc16 = q8s_scale_stride(cols) / 8; // 16-byte scale chunks
    const int lane = threadIdx.x % 32, half = lane >> 4, hl = lane & 15;
    const long long wstep = (long long)(gridDim.x - t) * (PREP_THREADS / 32) * (2 * RPB);
    for (long long base = ((long long)(blockIdx.x - t) * (PREP_THREADS / 32) + threadIdx.x / 32) * (2 * RPB); base < nrows;
         base += wstep) {
        unsigned mb[RPB];
#pragma unroll
        for (int j = 0; j < RPB; ++j)
            mb[j] = 0;
#pragma unroll 4
        for (long long k = hl; k < nsc16; k += 16) {
            uint4 v[RPB];
#pragma unroll
            for (int j = 0; j < RPB; ++j) {
                const long long o = base + 2 * j + half;
                v[j] = make_uint4(0, 0, 0, 0);
                if (o < nrows)
                    v[j] = __ldg(reinterpret_cast<const uint4 *>((o < rows ? w + o * rb : w2 + (o - rows) * rb) + cols) + k);
            }
#pragma unroll
            for (int j = 0; j < RPB; ++j) {
                const unsigned a4[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    mb[j] = max(mb[j], max(a4[q] & 0x7fffu, (a4[q] >> 16) & 0x7fffu));
            }
        }
#pragma unroll
        for (int j = 0; j < RPB; ++j) {
            for (int off = 8; off; off >>= 1)
                mb[j] = max(mb[j], __shfl_xor_sync(0xffffffffu, mb[j], off));
            const long long o = base + 2 * j + half;
            if (hl == 0 && o < nrows)
                rexp[o] = int8_t(row_exponent(mb[j]));
        }
    }
}

// y[tok][row] = sum over K parts k (in order) of part[k][tok][row]; for a SwiGLU pair the gate
// planes come first, then the up planes, and y = silu(gate sum) * (up sum). Tokens on the grid's
// y dimension; four rows per thread in 16-byte loads and stores where rows and ldy are multiples
// of 4 and y is 16-aligned (vec), else one row per thread.
__device__ __forceinline__ float reduce_one(const float *p, long long plane, int ks, int pair) {
    float g = p[0];
#pragma unroll 1
    for (int k = 1; k < ks; ++k)
        g += p[k * plane];
    if (pair) {
        float u = p[ks * plane];
#pragma unroll 1
        for (int k = 1; k < ks; ++k)
            u += p[(ks + k) * plane];
        g = g / (1.0f + expf(-g)) * u;
    }
    return g;
}

// Parts [0, ks) of four rows added in K order; all loads of a batch of up to B parts are issued
// before their sums.
template <int B>
__device__ __forceinline__ float4 sum_parts(const float4 *p, long long pl4, int ks) {
    float4 g = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k0 = 0; k0 < ks; k0 += B) {
        float4 q[B];
#pragma unroll
        for (int k = 0; k < B; ++k)
            if (k0 + k < ks)
                q[k] = p[(k0 + k) * pl4];
#pragma unroll
        for (int k = 0; k < B; ++k)
            if (k0 + k < ks) {
                if (k0 + k == 0) {
                    g = q[0];
                } else {
                    g.x += q[k].x;
                    g.y += q[k].y;
                    g.z += q[k].z;
                    g.w += q[k].w;
                }
            }
    }
    return g;
}

template <bool PAIR>
__global__ void __launch_bounds__(128, PAIR ? 4 : 8) splitk_reduce_kernel(const float *part, int ks, long long rows, int t,
                                                                          float *y, long long ldy, int vec) {
    const int pair = PAIR;
    if (threadIdx.x == 0)
        grid_launch_dependents();
    grid_wait(); // the product's partial planes
    const long long plane = (long long)t * rows;
    for (long long tok = blockIdx.y; tok < t; tok += gridDim.y) {
        const float *pt = part + tok * rows;
        float *yt = y + tok * ldy;
        if (vec) {
            for (long long r4 = (long long)blockIdx.x * blockDim.x + threadIdx.x; r4 < rows / 4;
                 r4 += (long long)gridDim.x * blockDim.x) {
                const float4 *p4 = reinterpret_cast<const float4 *>(pt) + r4;
                const long long pl4 = plane / 4;
                float4 g = sum_parts<PAIR ? 8 : 4>(p4, pl4, ks);
                if (pair) {
                    const float4 u = sum_parts<8>(p4 + ks * pl4, pl4, ks);
                    g.x = g.x / (1.0f + expf(-g.x)) * u.x;
                    g.y = g.y / (1.0f + expf(-g.y)) * u.y;
                    g.z = g.z / (1.0f + expf(-g.z)) * u.z;
                    g.w = g.w / (1.0f + expf(-g.w)) * u.w;
                }
                reinterpret_cast<float4 *>(yt)[r4] = g;
            }
        } else {
            for (long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += (long long)gridDim.x * blockDim.x)
                yt[r] = reduce_one(pt + r, plane, ks, pair);
        }
    }
}

// A small kernel of the product's launch sequence, with programmatic dependent launch when pdl.
template <class... KArgs, class... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), unsigned grid, unsigned block, cudaStream_t stream, bool pdl,
                       Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// The reduce pass on a 2-D grid (row groups x tokens), programmatic when pdl.
cudaError_t launch_reduce(dim3 grid, cudaStream_t stream, bool pdl, const float *part, int ks, int pair, long long rows,
                          int t, float *y, long long ldy, int vec) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(128);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return pair ? cudaLaunchKernelEx(&cfg, splitk_reduce_kernel<true>, part, ks, rows, t, y, ldy, vec)
                : cudaLaunchKernelEx(&cfg, splitk_reduce_kernel<false>, part, ks, rows, t, y, ldy, vec);
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
// Boxes of box_rows rows (BM, or PAIR_ROWS for the two matrices of a SwiGLU pair).
bool weight_maps(const uint8_t *w, long long rows, int cols, uint32_t box_rows, CUtensorMap *tq, CUtensorMap *td) {
    const uint64_t rb = uint64_t(q8s_row_bytes(cols));
    return make_map(tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, uint64_t(cols), uint64_t(rows), rb, 64, box_rows,
                    CU_TENSOR_MAP_SWIZZLE_64B) &&
           make_map(td, CU_TENSOR_MAP_DATA_TYPE_UINT16, w + cols, uint64_t(q8s_scale_stride(cols)), uint64_t(rows), rb, 8,
                    box_rows, CU_TENSOR_MAP_SWIZZLE_NONE);
}

// Row tiles of a job: BM rows, or PAIR_ROWS output rows for a SwiGLU pair.
long long row_tiles(const GemmJob &G) {
    const long long tr = G.w2 ? PAIR_ROWS : BM;
    return (G.rows + tr - 1) / tr;
}

} // namespace

namespace {

// Tokens per tile: the largest t split into passes of <= MAX_BN, rounded up to 16.
// CTAs per SM for a tile of bn tokens: two issuers per tensor core up to 64 tokens.
int cps_of(int bn) { return bn <= MAX_BN_TWO_CTAS ? 2 : 1; }

int choose_bn(const GemmJob *jobs, int n) {
    int tmax = 0;
    for (int j = 0; j < n; ++j)
        tmax = jobs[j].t > tmax ? jobs[j].t : tmax;
    const int npass_max = (tmax + MAX_BN - 1) / MAX_BN;
    const int bn = ((tmax + npass_max - 1) / npass_max + 15) / 16 * 16;
    return bn < 16 ? 16 : bn;
}

// K parts per job, from a cost model of the launch measured on B200: units run in waves of one
// per CTA slot (one or two per SM); a unit costs its 64-column stages (~0.52 us each at 16 tokens: the two-CTA shape's
// ring waits on weight latency; ~0.55 us at 256: the tensor pipe) plus its
// pipeline fill (~2 us) and epilogue drain (~7 us for a 128 x 256 fp32 tile, in proportion for
// fewer tokens); a split job adds the reduce pass (a launch plus its partial planes read once and
// y written, ~5 TB/s). The model picks the number of parts (1..16, each at least 4 stages long)
// with the least estimated time; a part count must save 3% to beat a smaller one.
void choose_splits(const GemmJob *jobs, int n, int bn, int num_sms, bool allow, int *ks) {
    const int sms = (num_sms > 0 ? num_sms : 148) * cps_of(bn);
    auto kmax_of = [](const GemmJob &G) {
        const int nks = (G.cols + BK - 1) / BK;
        return nks / 4 > 1 ? nks / 4 : 1;
    };
    int best = 1;
    if (allow) {
        const double ts = 0.52 + 0.03 * bn / 256.0, fill = 2.0 + 7.0 * bn / 256.0;
        double best_t = 0.0;
        for (int k = 1; k <= 16; ++k) {
            long long units = 0;
            int maxst = 0;
            double red = 0.0;
            for (int j = 0; j < n; ++j) {
                const GemmJob &G = jobs[j];
                const int kj = k < kmax_of(G) ? k : kmax_of(G);
                const int nks = (G.cols + BK - 1) / BK;
                units += row_tiles(G) * ((G.t + bn - 1) / bn) * kj;
                const int st = (nks + kj - 1) / kj;
                maxst = st > maxst ? st : maxst;
                if (kj > 1)
                    red += double(kj + (G.w2 ? 2 : 1)) * (G.w2 ? 2 : 1) * G.t * double(G.rows) * 4.0;
            }
            const long long waves = (units + sms - 1) / sms;
            const double t = double(waves) * (maxst * ts + fill) + (red > 0 ? 2.0 + red / 5e6 : 0.0);
            if (k == 1 || t < best_t * 0.97) {
                best_t = t;
                best = k;
            }
        }
    }
    for (int j = 0; j < n; ++j)
        ks[j] = best < kmax_of(jobs[j]) ? best : kmax_of(jobs[j]);
}

size_t part_bytes(const GemmJob &G, int ks) {
    return ks > 1 ? (size_t(G.w2 ? 2 : 1) * ks * G.t * G.rows * sizeof(float) + 255) / 256 * 256 : 0;
}

// A job's pre-pass output: fp16 x, 2^-s_t per token and r_o per weight row, each 256-aligned.
size_t xh_bytes(const GemmJob &G) { return (size_t(G.t) * G.cols * sizeof(__half) + 255) / 256 * 256; }
size_t tokf_bytes(const GemmJob &G) { return (size_t(G.t) * sizeof(float) + 255) / 256 * 256; }
size_t rexp_bytes(const GemmJob &G) { return (size_t(G.rows) * (G.w2 ? 2 : 1) + 255) / 256 * 256; }
size_t x_bytes(const GemmJob &G) { return xh_bytes(G) + tokf_bytes(G) + rexp_bytes(G); }

// The shape's kernel on the current device: loaded, and its shared-memory limit set to the SM's
// per-CTA limit (preload_gemm_tc does it for both shapes at rt_init).
template <int CPS>
cudaError_t setup_shape() {
    return cudaFuncSetAttribute(gemm_tc_kernel<CPS>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
}

// One launch of the CPS-per-SM shape. With CPS = 1 the CTA allocates all 512 TMEM columns, so a
// second CTA on the SM would only wait in its allocation: more than half the SM's shared memory
// keeps it off. With CPS = 2 two CTAs fit (256 columns and at most ~113 KB each).
template <int CPS>
cudaError_t launch_shape(const TcParams &p, size_t smem, int units, int num_sms, cudaStream_t stream, bool pdl) {
    if (CPS == 1 && smem < 116 * 1024)
        smem = 116 * 1024;
    if (smem > (CPS == 1 ? 227 * 1024 : 113 * 1024))
        return cudaErrorInvalidValue;
    static bool attr = false;
    if (!attr) {
        cudaError_t e = setup_shape<CPS>();
        if (e != cudaSuccess)
            return e;
        attr = true;
    }
    int grid = (num_sms > 0 ? num_sms : 148) * CPS;
    if (grid > units)
        grid = units;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(TcShape<CPS>::NT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute lattr[1];
    lattr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    lattr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = lattr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemm_tc_kernel<CPS>, p);
}

} // namespace

cudaError_t preload_gemm_tc() {
    cudaError_t e;
    if ((e = setup_shape<1>()) != cudaSuccess || (e = setup_shape<2>()) != cudaSuccess)
        return e;
    cudaFuncAttributes a;
    if ((e = cudaFuncGetAttributes(&a, tc_prep_kernel<1, 4>)) != cudaSuccess ||
        (e = cudaFuncGetAttributes(&a, tc_prep_kernel<1, 16>)) != cudaSuccess ||
        (e = cudaFuncGetAttributes(&a, tc_prep_kernel<8, 4>)) != cudaSuccess ||
        (e = cudaFuncGetAttributes(&a, tc_prep_kernel<8, 16>)) != cudaSuccess)
        return e;
    if ((e = cudaFuncGetAttributes(&a, splitk_reduce_kernel<true>)) != cudaSuccess)
        return e;
    return cudaFuncGetAttributes(&a, splitk_reduce_kernel<false>);
}

size_t gemm_tc_scratch_bytes(const GemmJob *jobs, int n, int num_sms, bool split_k) {
    if (n < 1 || n > 8)
        return 0;
    int ks[8];
    choose_splits(jobs, n, choose_bn(jobs, n), num_sms, split_k, ks);
    size_t s = 0;
    for (int j = 0; j < n; ++j)
        s += x_bytes(jobs[j]) + part_bytes(jobs[j], ks[j]);
    return s;
}

cudaError_t launch_gemm_tc(const GemmJob *jobs, int n, void *scratch, size_t scratch_bytes, int num_sms,
                           unsigned *err, cudaStream_t stream, bool pdl, bool split_k) {
    if (n < 1 || n > 8)
        return cudaErrorInvalidValue;
    if (gemm_tc_scratch_bytes(jobs, n, num_sms, split_k) > scratch_bytes || !scratch)
        return cudaErrorInvalidValue;
    const int bn = choose_bn(jobs, n);
    int ks[8];
    choose_splits(jobs, n, bn, num_sms, split_k, ks);
    TcParams p;
    memset(&p, 0, sizeof p);
    p.njobs = n;
    p.bn = bn;
    p.err = err;
    const int sb = stage_bytes(bn), cps = cps_of(bn);
    const size_t smem_limit = cps == 1 ? SMEM_LIMIT : SMEM_LIMIT_2;
    // the A slots follow the accumulators (at columns 0 and ACC_COLS / 2 when double-buffered; two
    // CTAs per SM with tiles of <= 32 tokens: at 0 and 32), on a 32-column boundary
    const int acc_stride = cps == 2 && bn <= 32 ? 32 : (cps == 1 ? TcShape<1>::ACC_COLS : TcShape<2>::ACC_COLS) / n_acc(bn, cps);
    p.acc_stride = acc_stride;
    const int acc_end = (n_acc(bn, cps) - 1) * acc_stride + bn;
    p.a_base = cps == 1 ? TcShape<1>::ACC_COLS : (acc_end + A_COLS - 1) / A_COLS * A_COLS;
    const int tmem_cols = cps == 1 ? TcShape<1>::TMEM_COLS : TcShape<2>::TMEM_COLS;
    int max_s = (tmem_cols - p.a_base) / A_COLS;
    max_s = max_s < MAX_STAGES ? max_s : MAX_STAGES;
    p.stages = int((smem_limit - 512) / size_t(sb));
    if (p.stages > max_s)
        p.stages = max_s;
    if (p.stages < 2)
        return cudaErrorInvalidValue;
    uint8_t *sc = static_cast<uint8_t *>(scratch);
    int units = 0;
    for (int j = 0; j < n; ++j) {
        const GemmJob &G = jobs[j];
        if (G.cols < Q8_QK || G.cols % Q8_QK || G.t < 1 || G.rows < 1)
            return cudaErrorInvalidValue;
        __half *xh = reinterpret_cast<__half *>(sc);
        float *tokf = reinterpret_cast<float *>(sc + xh_bytes(G));
        int8_t *rexp = reinterpret_cast<int8_t *>(sc + xh_bytes(G) + tokf_bytes(G));
        sc += x_bytes(G);
        {
            const long long nrows = G.rows * (G.w2 ? 2 : 1);
            const int sms = num_sms > 0 ? num_sms : 148;
            const bool deep = nrows >= (long long)sms * (PREP_THREADS / 32) * 16;
            const long long rows_per_block = (PREP_THREADS / 32) * 2 * (deep ? 8 : 1);
            long long rblocks = (nrows + rows_per_block - 1) / rows_per_block;
            rblocks = rblocks > 1184 ? 1184 : rblocks;
            const bool narrow = G.cols <= 4 * 4 * PREP_THREADS;
            auto kern = deep ? (narrow ? tc_prep_kernel<8, 4> : tc_prep_kernel<8, 16>)
                             : (narrow ? tc_prep_kernel<1, 4> : tc_prep_kernel<1, 16>);
            cudaError_t e = launch_pdl(kern, unsigned(G.t + rblocks), PREP_THREADS, stream, pdl, G.x, G.ldx, G.cols, G.t,
                                       xh, tokf, G.w, G.w2, G.rows, rexp);
            if (e != cudaSuccess)
                return e;
        }
        if (!make_map(&p.tx[j], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xh, uint64_t(G.cols), uint64_t(G.t),
                      uint64_t(G.cols) * 2, 64, uint32_t(bn), CU_TENSOR_MAP_SWIZZLE_128B))
            return cudaErrorInvalidValue;
        TcJobDev &J = p.job[j];
        J.pair = G.w2 != nullptr;
        J.rexp = rexp;
        J.tokf = tokf;
        const uint32_t box_rows = J.pair ? PAIR_ROWS : BM;
        if (!weight_maps(G.w, G.rows, G.cols, box_rows, &J.tq, &J.td))
            return cudaErrorInvalidValue;
        if (J.pair && !weight_maps(G.w2, G.rows, G.cols, box_rows, &J.tq2, &J.td2))
            return cudaErrorInvalidValue;
        J.y = G.y;
        J.rows = G.rows;
        J.ldy = G.ldy;
        J.ks = ks[j];
        J.part = nullptr;
        if (J.ks > 1) {
            J.part = reinterpret_cast<float *>(sc);
            sc += part_bytes(G, J.ks);
        }
        J.cols = G.cols;
        J.t = G.t;
        J.n_pass = (G.t + bn - 1) / bn;
        J.tiles = int(row_tiles(G));
        J.unit0 = units;
        units += J.tiles * J.n_pass * J.ks;
    }
    p.total_units = units;
    size_t smem = size_t(p.stages) * sb + 8 * (3 * MAX_STAGES + 4) + 64 + 1024;
    cudaError_t e = cps == 1 ? launch_shape<1>(p, smem, units, num_sms, stream, pdl)
                             : launch_shape<2>(p, smem, units, num_sms, stream, pdl);
    if (e != cudaSuccess)
        return e;
    // the split jobs' partial sums, added in K order (stream order after the product)
    for (int j = 0; j < n; ++j) {
        const TcJobDev &J = p.job[j];
        if (J.ks < 2)
            continue;
        const int vec = J.rows % 4 == 0 && J.ldy % 4 == 0 && (reinterpret_cast<uintptr_t>(J.y) & 15) == 0;
        const long long per_tok = vec ? J.rows / 4 : J.rows;
        long long gx = (per_tok + 127) / 128;
        gx = gx > 1024 ? 1024 : gx;
        const dim3 grid(unsigned(gx), unsigned(J.t < 65535 ? J.t : 65535));
        if ((e = launch_reduce(grid, stream, pdl, static_cast<const float *>(J.part), J.ks, int(J.pair), J.rows, J.t, J.y,
                               J.ldy, vec)) != cudaSuccess)
            return e;
    }
    return cudaSuccess;
}

bool map_f32_2d(void *map, const float *base, uint64_t inner, uint64_t outer, uint64_t stride_bytes,
                uint32_t box_inner, uint32_t box_outer) {
    return make_map(static_cast<CUtensorMap *>(map), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, base, inner, outer, stride_bytes,
                    box_inner, box_outer, CU_TENSOR_MAP_SWIZZLE_NONE);
}

} // namespace q8
