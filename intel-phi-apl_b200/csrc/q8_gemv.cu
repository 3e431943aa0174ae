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
//              (packed in row pairs); the t_b and fp32 scales go to a partial-sum buffer;
//   chain      one or two warps (Cfg): one lane per (token, row) runs acc = fma(t_b, d_b, acc) in
//              block order and writes y (for a SwiGLU pair: silu(gate) * up). The chain is serial
//              per row, so the CTA's tiles alternate between the chain warps (a tile's chunks
//              stay on one);
//   last warp  copies: issues a stage's bulk copies as soon as its slot is free.
// One token runs two CTAs per SM, more tokens one (Cfg).
// Barriers: full (copies landed), empty (slot read), tfull/tempty (partial sums; tfull one set per
// chain warp: see the chain warps' loop). Every wait is
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
constexpr int NC = 256;            // compute threads: (block column, row half) each
constexpr int NH = R / 2;          // rows per compute thread
constexpr int CHAIN_WARP = NC / 32; // the first chain warp; the copy warp follows the chain warps

// The CTA's shape: CTAS CTAs per SM.
//   CTAS = 2 (one token, long launches): 320 threads, <= 102 registers and ~104 KB of shared
//   memory each, with a 2-stage ring, 4 partial-sum buffers and one chain warp. The SM holds 4
//   stages in flight as with one CTA, and the two CTAs' load and chain phases interleave instead
//   of every compute warp of the SM waiting on the same stage (the output head streams ~10%
//   faster). A CTA that finishes frees half an SM for the next kernel on the stream.
//   CTAS = 1: a 4-stage ring, two chain warps, and 8 partial-sum buffers for one token (they
//   absorb the chain's jitter), 4 for more (their partial sums fill the space). Launches of a
//   few stages per SM run faster so: each CTA has more stages in flight and chain warps.
template <int MT, int CTAS_>
struct Cfg {
    static_assert(CTAS_ == 1 || (CTAS_ == 2 && MT == 1), "two CTAs per SM for one token only");
    static constexpr int CTAS = CTAS_;
    static constexpr int STAGES = CTAS == 2 ? 2 : 4;                  // weight slots
    static constexpr int TBUF = CTAS == 2 ? 4 : (MT == 1 ? 8 : 4);    // partial-sum buffers
    static constexpr int NCHAIN = CTAS == 2 ? 1 : 2;                  // tile i of the CTA -> chain warp i % NCHAIN
    static constexpr int COPY_WARP = CHAIN_WARP + NCHAIN;
    static constexpr int NT = NC + 32 * NCHAIN + 32;                  // threads
    // tiles visited chunk-major together in a launch with rows of several chunks (one at a time in
    // the two-CTA form: its register budget has no room for the group's running sums)
    static constexpr int GROUP = CTAS == 2 ? 1 : 4;
};
// One-token launches with at least this many stages per SM run two CTAs per SM.
constexpr int TWO_CTA_MIN_STAGES_PER_SM = 12;
// A row's slot: quants, scales, then 16 bytes of padding (4368 B). The padding puts neighbouring
// rows 16 bytes apart in the bank space, so a warp reading two rows at once (lanes with b & 4 read
// the other row of a pair) touches eight distinct 16-byte bank groups per quarter-warp.
constexpr int ROWB = KC + NBK * 2 + 16;
constexpr int SLOT = R * ROWB;
constexpr int TPAD = NBK + 4;      // partial-sum row stride (floats): 16-byte rows, conflict-free per lane = row
static_assert(NC == 2 * NBK, "two compute threads (row halves) per block column of a stage");
static_assert(ROWB % 16 == 0 && SLOT % 16 == 0, "bulk copy destinations are 16-byte aligned");
static_assert(ROWB % 128 == 16, "a row pair's two rows sit in different bank groups");

// Per-stage row flags (row loaded or not), written by the copy warp, read by the chain warp. When
// the copy warp fills stage s, compute has released stage s-STAGES, so it has finished stage
// s-STAGES-1, whose partial-sum wait means the chain finished stage s-STAGES-1-TBUF: a ring of
// 16 entries is never overwritten while read.
constexpr int FRING = 16;

template <int MT, int CTAS>
constexpr size_t smem_bytes() {
    using C = Cfg<MT, CTAS>;
    static_assert(FRING >= C::STAGES + C::TBUF + 2, "row-flag ring");
    return size_t(C::STAGES) * SLOT + size_t(C::TBUF) * (MT + 1) * R * TPAD * 4 +
           (C::STAGES * 2 + C::TBUF * (C::NCHAIN + 1) + 1) * 8 + FRING * R;
}

// One job's fields, cached in registers by every role when its stage sequence enters the job:
// the per-stage work then touches no kernel parameter.
struct JobView {
    const uint8_t *w, *w2;
    const int32_t *idx;
    const float *x;
    float *y;
    unsigned *done_ctr;
    int nwait; // the waits themselves stay in the kernel parameters (read once per job)
    int x_written;
    long long rows, src_rows, ldx, ldy, rb;
    int cols, m, tile0, tiles, rpt, nchunk;
    __device__ __forceinline__ void load(const GemvJob &J) {
        done_ctr = J.done_ctr;
        nwait = J.nwait;
        x_written = J.x_written;
        w = J.w;
        w2 = J.w2;
        idx = J.idx;
        x = J.x;
        y = J.y;
        rows = J.rows;
        src_rows = J.src_rows;
        ldx = J.ldx;
        ldy = J.ldy;
        cols = J.cols;
        m = J.m;
        tile0 = J.tile0;
        tiles = J.tiles;
        rb = q8s_row_bytes(cols);
        rpt = w2 ? R / 2 : R; // output rows per tile
        nchunk = (cols + KC - 1) / KC;
    }
};

// The CTA's sequence of stages. Its tiles are blockIdx.x, +gridDim.x, ..., each ceil(cols/KC)
// chunks long. A row of several chunks is visited chunk-major over a group of up to GROUP tiles
// of the CTA (chunk 0 of each tile of the group, then chunk 1, ...): the compute warps then load
// each x chunk once per group instead of once per stage, and each row still runs its blocks in
// order (the chain warps keep a running sum per tile of the group). A gather's tiles go one at a
// time (its row index is loaded per tile). Every role walks its own copy; tiles only grow, so the
// job index only moves forward. k: the CTA's count of the current tile (its chain warp is
// k % NCHAIN); i: the tile's place in its group (its running-sum slot is i / NCHAIN).
template <int GROUP>
struct StageIter {
    int g, c, job;
    int gfirst, gsize, i, kbase, k;
    JobView J;
    template <class P>
    __device__ __forceinline__ void start(const P &p) {
        job = -1;
        kbase = 0;
        gfirst = blockIdx.x;
        if (gfirst < p.total_tiles)
            group(p);
        else
            g = gfirst;
    }
    template <class P>
    __device__ __forceinline__ void set(const P &p) {
        int j = job < 0 ? 0 : job;
        while (j + 1 < p.njobs && g >= p.job[j + 1].tile0)
            ++j;
        if (j != job) {
            job = j;
            J.load(p.job[j]);
        }
    }
    // a new group from tile gfirst
    template <class P>
    __device__ __forceinline__ void group(const P &p) {
        g = gfirst;
        set(p);
        gsize = 1;
        if (GROUP > 1 && J.nchunk > 1 && !J.idx) {
            const int left = 1 + (J.tile0 + J.tiles - 1 - gfirst) / int(gridDim.x); // this CTA's tiles left in the job
            gsize = left < GROUP ? left : GROUP;
        }
        i = 0;
        c = 0;
        k = kbase;
    }
    template <class P>
    __device__ __forceinline__ bool valid(const P &p) const { return g < p.total_tiles; }
    template <class P>
    __device__ __forceinline__ void next(const P &p) {
        if (++i == gsize) {
            i = 0;
            if (++c == J.nchunk) {
                kbase += gsize;
                gfirst += gsize * int(gridDim.x);
                if (gfirst < p.total_tiles)
                    group(p);
                else
                    g = gfirst;
                return;
            }
        }
        g = gfirst + i * int(gridDim.x);
        k = kbase + i;
    }
    // stage row r: the output index and the matrix it reads
    __device__ __forceinline__ long long out_row(int r) const { return (long long)(g - J.tile0) * J.rpt + (r % J.rpt); }
    __device__ __forceinline__ const uint8_t *matrix(int r) const { return (J.w2 && r >= J.rpt) ? J.w2 : J.w; }
};

// Rows processed side by side by one compute thread. Two at a time for one token: the second
// pair's shared-memory reads then overlap the first pair's chains in the other warps (all eight
// compute warps wait on the same stage, so one load phase per stage would leave the ALUs idle
// while shared memory serves every warp). All 4 for two tokens (the pair of tokens already
// gives each quant two uses); 2 at a time for three or four (the x registers grow).
template <int MT>
constexpr int row_group() { return MT == 2 ? NH : NH / 2; }

// The RG rows' 32-step chains of one block for MT tokens, rows in packed pairs (fma.rn.f32x2 and
// add.rn.f32x2: two independent IEEE operations per instruction). A pair's converted weights serve
// every token, so a weight costs one byte permute, half a packed add and MT halves of a packed fma.
template <int MT, int RG>
__device__ __forceinline__ void block_chains(const uint32_t (&wq)[RG][8], const float (&xr)[MT][Q8_QK],
                                             float (&t)[MT][RG]) {
    static_assert(RG % 2 == 0, "rows in pairs");
    float2 tp[MT][RG / 2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int p = 0; p < RG / 2; ++p)
            tp[mt][p] = make_float2(0.0f, 0.0f);
    const float2 bias = make_float2(-8388736.0f, -8388736.0f);
#pragma unroll
    for (int i = 0; i < Q8_QK; ++i) {
#pragma unroll
        for (int p = 0; p < RG / 2; ++p) {
            // 2^23 + (q + 128) for the two rows, then minus 2^23 + 128: exact q
            const float2 m = __fadd2_rn(
                make_float2(__uint_as_float(__byte_perm(wq[2 * p][i >> 2], 0x4B000000u, 0x7650u + (i & 3))),
                            __uint_as_float(__byte_perm(wq[2 * p + 1][i >> 2], 0x4B000000u, 0x7650u + (i & 3)))),
                bias);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
                tp[mt][p] = __ffma2_rn(m, make_float2(xr[mt][i], xr[mt][i]), tp[mt][p]);
        }
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int p = 0; p < RG / 2; ++p) {
            t[mt][2 * p] = tp[mt][p].x;
            t[mt][2 * p + 1] = tp[mt][p].y;
        }
}

// Waits until *ctr >= target (an acquire at GPU scope), bounded like every wait here.
__device__ __noinline__ bool wait_count(const unsigned *ctr, unsigned target) {
    const long long t0 = clock64();
    for (;;) {
        unsigned v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
        if (v >= target)
            return true;
        const long long dt = clock64() - t0;
        if (dt > WAIT_LIMIT_CYCLES)
            return false;
        if (dt > 20000) // past ~10 us, poll less often
            __nanosleep(200);
    }
}

// Waits until the gate word has reached `value` (modulo 2^32: the host counts rounds), read at
// system scope: the link stream's write-value operation sets it after the round's copies.
__device__ __noinline__ bool wait_gate(const unsigned *gate, unsigned value) {
    const long long t0 = clock64();
    for (;;) {
        unsigned v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(gate) : "memory");
        if (int(v - value) >= 0)
            return true;
        const long long dt = clock64() - t0;
        if (dt > WAIT_LIMIT_CYCLES)
            return false;
        if (dt > 20000)
            __nanosleep(200);
    }
}

// The failure path's self-test: one thread waits on a device counter that nothing advances, then
// on an mbarrier that nothing arrives on. Each wait gives up after WAIT_LIMIT_CYCLES (about a
// second) and reports its bit, as a stuck wait in a product kernel does; the kernel then returns.
__global__ void wait_probe_kernel(const unsigned *ctr, unsigned *err) {
    __shared__ uint64_t bar;
    if (threadIdx.x != 0)
        return;
    if (!wait_count(ctr, 1u))
        report(err, ERR_TIMEOUT_ROUND);
    mbar_init(&bar, 1);
    if (!mbar_wait(&bar, 0))
        report(err, ERR_TIMEOUT_FULL);
}

// GROUPED: some job of the launch has rows of several chunks (the instance without it carries no
// group bookkeeping, which the one-chunk rows would pay for in every stage).
template <int MT, int CTAS, class P, bool GROUPED>
__global__ void __launch_bounds__(Cfg<MT, CTAS>::NT, CTAS) gemv_exact_kernel(const __grid_constant__ P p) {
    using C = Cfg<MT, CTAS>;
    constexpr int GROUP = GROUPED ? C::GROUP : 1;
    constexpr int STAGES = C::STAGES, TBUF = C::TBUF, NCHAIN = C::NCHAIN, COPY_WARP = C::COPY_WARP;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *slots = smem;
    float *T = reinterpret_cast<float *>(smem + size_t(STAGES) * SLOT); // [TBUF][MT][R][TPAD]
    float *TD = T + TBUF * MT * R * TPAD;                                 // [TBUF][R][TPAD]
    uint64_t *full = reinterpret_cast<uint64_t *>(TD + TBUF * R * TPAD);  // [STAGES]
    uint64_t *empty = full + STAGES;                                      // [STAGES]
    uint64_t *tfull = empty + STAGES;                                     // [NCHAIN][TBUF]
    uint64_t *tempty = tfull + NCHAIN * TBUF;                             // [TBUF]
    uint64_t *depbar = tempty + TBUF;                                     // a chained round's dependency met
    uint8_t *rowflag = reinterpret_cast<uint8_t *>(depbar + 1);           // [FRING][R]: row was loaded
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NC);
        }
        for (int b = 0; b < TBUF; ++b) {
            for (int w = 0; w < NCHAIN; ++w)
                mbar_init(&tfull[w * TBUF + b], NC);
            mbar_init(&tempty[b], 1);
        }
        mbar_init(depbar, 1);
        fence_barrier_init();
        grid_launch_dependents();
    }
    __syncthreads();

    if (warp < CHAIN_WARP) {
        // ---------------------------------------------------------------- compute threads
        float xr[MT][Q8_QK];
        int xjob = -1, xc = -1, wjob = -1, ndep = 0;
        const int b = tid % NBK, half = tid / NBK;
        grid_wait(); // x comes from the previous kernel on the stream
        if (p.gate) {
            // an opened round: x lands after the launch. Compute thread 0 polls the gate and
            // passes it on through the CTA barrier (its first phase), as for a chained round.
            if (tid == 0) {
                if (!wait_gate(p.gate, p.gate_value))
                    report(p.err, ERR_TIMEOUT_GATE);
                mbar_arrive(depbar);
            } else if (lane == 0 && !mbar_wait(depbar, 0)) {
                report(p.err, ERR_TIMEOUT_GATE);
            }
            ndep = 1;
            __syncwarp();
        }
        StageIter<GROUP> it;
        it.start(p);
        for (int s = 0; it.valid(p); it.next(p), ++s) {
            const int slot = s % STAGES, tb = s % TBUF;
            if (!mbar_wait(&full[slot], (s / STAGES) & 1)) {
                report(p.err, ERR_TIMEOUT_FULL);
                break;
            }
            const int c0 = it.c * KC;
            const int nbk = min(KC, it.J.cols - c0) / Q8_QK;
            const bool active = b < nbk;
            if (it.job != wjob) {
                // A chained job that depends on earlier rounds of this launch: its x may be their
                // output (read after write), its y may overwrite their x (write after read) or
                // their y (write after write). Compute thread 0 alone polls those rounds' tile
                // counters (bounded, acquires at GPU scope) and passes the result on through a
                // CTA barrier that the other compute warps wait on, bounded like every wait here.
                // The tile's y is written by the chain warps only after these warps computed it,
                // so the one wait here orders the writes too.
                wjob = it.job;
                if (it.J.nwait) {
                    if (tid == 0) {
                        const GemvJob &PJ = p.job[it.job];
                        for (int k = 0; k < it.J.nwait; ++k)
                            if (!wait_count(PJ.wait_ctr[k], PJ.wait_target[k]))
                                report(p.err, ERR_TIMEOUT_ROUND);
                        mbar_arrive(depbar);
                    } else if (lane == 0 && !mbar_wait(depbar, ndep & 1)) {
                        report(p.err, ERR_TIMEOUT_ROUND);
                    }
                    ++ndep;
                    __syncwarp();
                }
            }
            if (active && (it.c != xc || it.job != xjob)) {
                xc = it.c;
                xjob = it.job;
                const bool coherent = it.J.x_written != 0; // x written earlier in this launch: not via L1
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    const float4 *xp = reinterpret_cast<const float4 *>(it.J.x + mt * it.J.ldx + c0 + b * Q8_QK);
#pragma unroll
                    for (int v = 0; v < 8; ++v) {
                        const float4 f = coherent ? __ldcg(xp + v) : __ldg(xp + v);
                        xr[mt][4 * v + 0] = f.x;
                        xr[mt][4 * v + 1] = f.y;
                        xr[mt][4 * v + 2] = f.z;
                        xr[mt][4 * v + 3] = f.w;
                    }
                }
            }
            constexpr int RG = row_group<MT>();
            static_assert(RG % 2 == 0, "row pairs stay inside one row group");
            const uint8_t *qbase = slots + size_t(slot) * SLOT + b * Q8_QK; // row r's block b: + r*ROWB
            const uint8_t *dbase = slots + size_t(slot) * SLOT + KC + 2 * b; // row r's scale b: + r*ROWB
            // Lanes with b & 4 take each row pair in the other order (register k holds row k ^ 1):
            // their 32-byte blocks would otherwise share banks with lanes b - 4 of the same row.
            const int rot = (b >> 2) & 1;
            const uint8_t *qeven = qbase + rot * ROWB, *qodd = qbase - rot * ROWB;
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
                        const uint8_t *qr = ((k & 1) ? qodd : qeven) + r * ROWB; // row r ^ rot
                        const uint4 q0 = *reinterpret_cast<const uint4 *>(qr);
                        const uint4 q1 = *reinterpret_cast<const uint4 *>(qr + 16);
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
                            Tb[(mt * R + r) * TPAD + b] = rot ? t[mt][k ^ 1] : t[mt][k];
                        TDb[r * TPAD + b] = dv[k];
                    }
                }
            }
            if (!ok)
                break;
            mbar_arrive(&tfull[(it.k % NCHAIN) * TBUF + tb]); // the tile's chain warp
        }
    } else if (warp < COPY_WARP) {
        // ---------------------------------------------------------------- chain warps
        const int mt = lane / R, r = lane % R, cw = warp - CHAIN_WARP;
        constexpr int ACCS = (GROUP + NCHAIN - 1) / NCHAIN;
        float accs[ACCS]; // the running sums of this warp's tiles of the current group
#pragma unroll
        for (int a = 0; a < ACCS; ++a)
            accs[a] = 0.0f;
        // A row-sharded launch also stores each output into every peer's staging image of the
        // round being produced ([t][rows_total]).
        const PeerOut &po = p.peer;
        unsigned long long stage_off = 0;
        if (po.on) {
            // the previous launch on the stream (the last round's gather) has completed: under
            // programmatic launch this kernel may start before it does
            grid_wait();
            const unsigned long long round0 =
                *reinterpret_cast<const volatile unsigned long long *>(po.region[po.rank] + PEER_PRODUCED);
            stage_off = peer_image(round0 + 1);
        }
        float *const yh = p.y_host;
        auto put = [&](float *y, long long ldy, long long o, float v) {
            y[mt * ldy + o] = v;
            if (yh)
                yh[mt * ldy + o] = v; // the round's only job: y's own layout, in host memory
            if (po.on) {
                const long long gi = mt * po.rows_total + po.row0 + o;
                for (int w = 0; w < po.world; ++w)
                    if (w != po.rank)
                        reinterpret_cast<float *>(po.region[w] + stage_off)[gi] = v;
            }
        };
        // The chain warps take the CTA's tiles in turn, so a chain warp skips the other's tiles:
        // after a tile of at least TBUF chunks it would wait on a shared barrier more than one
        // phase ahead, which a parity wait cannot tell from the phase before. So each chain
        // warp has its own TBUF barriers, which advance only on its own stages, and keeps their
        // parities here (bit b: buffer b).
        uint32_t tpar = 0;
        StageIter<GROUP> it;
        it.start(p);
        for (int s = 0; it.valid(p); ++s) {
            const bool own = it.k % NCHAIN == cw;
            const int tb = s % TBUF;
            const bool last_chunk = it.c == it.J.nchunk - 1;
            if (own) {
                if (!mbar_wait(&tfull[cw * TBUF + tb], (tpar >> tb) & 1u)) {
                    report(p.err, ERR_TIMEOUT_TFULL);
                    break;
                }
                tpar ^= 1u << tb;
                const int nbk = min(KC, it.J.cols - it.c * KC) / Q8_QK;
                const long long o = it.out_row(r);
                const bool valid = o < it.J.rows;
                const bool loaded = rowflag[(s % FRING) * R + r] != 0;
                const bool mine = mt < it.J.m && loaded;
                const int slot = it.i / NCHAIN;
                float acc = 0.0f; // (selected from registers: no local-memory indexing)
#pragma unroll
                for (int a = 0; a < ACCS; ++a)
                    if (a == slot && it.c > 0)
                        acc = accs[a];
                if (mine) {
                    const float *tp = T + tb * MT * R * TPAD + (mt * R + r) * TPAD;
                    const float *dp = TD + tb * R * TPAD + r * TPAD;
                    int b = 0;
                    for (; b + 16 <= nbk; b += 16) { // 128-bit loads first, then 16 dependent fmas
                        float4 tv[4], dd[4];
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            tv[k] = *reinterpret_cast<const float4 *>(tp + b + 4 * k);
                            dd[k] = *reinterpret_cast<const float4 *>(dp + b + 4 * k);
                        }
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            acc = __fmaf_rn(tv[k].x, dd[k].x, acc);
                            acc = __fmaf_rn(tv[k].y, dd[k].y, acc);
                            acc = __fmaf_rn(tv[k].z, dd[k].z, acc);
                            acc = __fmaf_rn(tv[k].w, dd[k].w, acc);
                        }
                    }
                    for (; b < nbk; ++b)
                        acc = __fmaf_rn(tp[b], dp[b], acc);
                }
#pragma unroll
                for (int a = 0; a < ACCS; ++a)
                    if (a == slot)
                        accs[a] = acc;
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(&tempty[tb]);
                if (last_chunk) {
                    if (it.J.w2) {
                        const float up = __shfl_down_sync(0xffffffffu, acc, R / 2);
                        if (mine && r < R / 2) {
                            const float silu = acc / (1.0f + expf(-acc));
                            put(it.J.y, it.J.ldy, o, silu * up);
                        }
                    } else if (mine) {
                        put(it.J.y, it.J.ldy, o, acc);
                    } else if (mt < it.J.m && valid) { // a gather index outside the matrix
                        put(it.J.y, it.J.ldy, o, __int_as_float(0x7fc00000));
                        report(p.err, ERR_BAD_JOB);
                    }
                    if (it.J.done_ctr) { // chained: the tile's outputs, then its count (release)
                        __threadfence();
                        __syncwarp();
                        if (lane == 0)
                            atomicAdd(it.J.done_ctr, 1u);
                    }
                }
            }
            it.next(p);
        }
    } else {
        // ---------------------------------------------------------------- copy issuer (one warp:
        // lane r < R owns stage row r; a gather's row index is loaded one stage ahead)
        const uint64_t pol = policy_evict_first();
        bool gathers = false;
        for (int j = 0; j < p.njobs; ++j)
            gathers |= p.job[j].idx != nullptr;
        if (!p.early || gathers)
            grid_wait(); // weights (unless the caller vouches for them) and row lists may be outputs of it
        if (gathers && p.gate) { // an opened round's row lists may land with its x
            if (lane == 0 && !wait_gate(p.gate, p.gate_value))
                report(p.err, ERR_TIMEOUT_GATE);
            __syncwarp();
        }
        StageIter<GROUP> it;
        it.start(p);
        long long src = -1; // this lane's source row for the current stage (gathers: prefetched)
        if (it.valid(p) && lane < R && it.J.idx) {
            const long long o = it.out_row(lane);
            src = o < it.J.rows ? (long long)__ldg(it.J.idx + o) : -1;
        }
        int s = 0;
        bool ok = true;
        for (; it.valid(p); ++s) {
            const int slot = s % STAGES;
            if (s >= STAGES && !mbar_wait(&empty[slot], ((s / STAGES) - 1) & 1)) {
                report(p.err, ERR_TIMEOUT_FULL);
                ok = false;
                break;
            }
            const int c0 = it.c * KC;
            const int nbk = min(KC, it.J.cols - c0) / Q8_QK;
            const uint32_t qbytes = uint32_t(nbk) * Q8_QK, dbytes = (uint32_t(nbk) * 2u + 15u) & ~15u;
            const bool whole = it.J.cols == KC; // a row is exactly one slot row: one copy
            const long long o = it.out_row(lane);
            const bool valid = lane < R && o < it.J.rows;
            const long long srow = it.J.idx ? src : o;
            const bool load = valid && srow >= 0 && srow < it.J.src_rows;
            const uint8_t *mat = it.matrix(lane);
            const uint32_t bytes = load ? (whole ? uint32_t(it.J.rb) : qbytes + dbytes) : 0u;
            const uint32_t total = __reduce_add_sync(0xffffffffu, bytes);
            if (lane < R)
                rowflag[(s % FRING) * R + lane] = load ? 1 : 0;
            const int cur_c = it.c;
            const int cur_cols = it.J.cols;
            // the next stage's gather index, loaded now so its latency overlaps this stage
            it.next(p);
            if (it.valid(p) && lane < R && it.J.idx) {
                if (it.c == 0) {
                    const long long on = it.out_row(lane);
                    src = on < it.J.rows ? (long long)__ldg(it.J.idx + on) : -1;
                } // a later chunk of the same tile keeps the same row
            }
            __syncwarp();
            if (lane == 0)
                mbar_arrive_expect_tx(&full[slot], total);
            __syncwarp();
            if (load) {
                const uint8_t *row = mat + srow * (long long)q8s_row_bytes(cur_cols);
                uint8_t *dst = slots + size_t(slot) * SLOT + lane * ROWB;
                if (whole) {
                    bulk_g2s(dst, row, bytes, &full[slot], pol);
                } else {
                    bulk_g2s(dst, row + cur_c * KC, qbytes, &full[slot], pol);
                    bulk_g2s(dst + KC, row + cur_cols + (cur_c * KC / Q8_QK) * 2, dbytes, &full[slot], pol);
                }
            }
        }
        // Leave no bulk copy in flight: on the normal path the compute threads consumed every
        // stage; after a timeout, wait (bounded) for the most recent fill of each slot.
        if (!ok && lane == 0)
            for (int k = max(0, s - STAGES); k < s; ++k)
                if (!mbar_wait(&full[k % STAGES], (k / STAGES) & 1))
                    report(p.err, ERR_TIMEOUT_DRAIN);
    }

    if (p.peer.on) {
        // The last CTA to finish advances the round count (every CTA has read it by then: its
        // chain warps read it before the CTA's barrier below). The gather kernel on the side
        // stream publishes the round, after this kernel has completed.
        __syncthreads();
        if (tid == 0) {
            unsigned char *mine = p.peer.region[p.peer.rank];
            unsigned *done = reinterpret_cast<unsigned *>(mine + PEER_PCTAS);
            if (atomicAdd(done, 1u) == gridDim.x - 1) {
                unsigned long long *round = reinterpret_cast<unsigned long long *>(mine + PEER_PRODUCED);
                *round = *round + 1;
                *done = 0;
            }
        }
    }
    if (p.y_host) {
        // The last CTA to finish tells the host: each CTA's host stores are ordered (barrier, then
        // one system-scope fence) before its count, the last count before the flag.
        __syncthreads();
        if (tid == 0) {
            __threadfence_system();
            if (atomicAdd(p.host_ctr, 1u) == gridDim.x - 1) {
                *p.host_ctr = 0;
                const unsigned seq = p.host_ctr[1] + 1; // (only this CTA writes it)
                p.host_ctr[1] = seq;
                __threadfence_system();
                asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p.host_flag), "r"(seq) : "memory");
            }
        }
    }
}

// One kernel instance's set-up on the current device: its shared-memory attribute and the CTAs
// that fit on an SM (kept per process). Done for every instance by preload_gemv at rt_init, so no
// launch loads a kernel or sets an attribute first (that can wait for the GPU, which an opened
// round's gated kernel holds).
template <int MT, int CTAS, class P, bool GROUPED>
cudaError_t setup_mt(int *per_sm_out) {
    using C = Cfg<MT, CTAS>;
    const size_t smem = smem_bytes<MT, CTAS>();
    static int per_sm = 0;
    if (per_sm == 0 || !per_sm_out) {
        cudaError_t e = cudaFuncSetAttribute(gemv_exact_kernel<MT, CTAS, P, GROUPED>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             int(smem));
        if (e != cudaSuccess)
            return e;
        int n = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gemv_exact_kernel<MT, CTAS, P, GROUPED>, C::NT, smem);
        if (e != cudaSuccess)
            return e;
        if (n < 1)
            return cudaErrorInvalidConfiguration;
        per_sm = n < CTAS ? n : CTAS;
    }
    if (per_sm_out)
        *per_sm_out = per_sm;
    return cudaSuccess;
}

template <int MT, int CTAS, class P, bool GROUPED>
cudaError_t launch_mt_g(const P &p, int num_sms, int grid_limit, cudaStream_t stream, bool pdl, bool coop) {
    using C = Cfg<MT, CTAS>;
    const size_t smem = smem_bytes<MT, CTAS>();
    int per_sm = 0;
    cudaError_t es = setup_mt<MT, CTAS, P, GROUPED>(&per_sm);
    if (es != cudaSuccess)
        return es;
    int grid = per_sm * (num_sms > 0 ? num_sms : 148);
    if (grid_limit > 0 && grid > grid_limit)
        grid = grid_limit;
    if (grid > p.total_tiles && !coop)
        grid = p.total_tiles;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(C::NT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (coop) {
        // every CTA resident at once: a chained round waits on other CTAs' tiles
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
    } else {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
    }
    cfg.attrs = attr;
    cfg.numAttrs = (pdl || coop) ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemv_exact_kernel<MT, CTAS, P, GROUPED>, p);
}

// rows of several chunks (not gathered) somewhere in the launch
template <class P>
bool any_grouped(const P &p) {
    for (int j = 0; j < p.njobs; ++j)
        if (p.job[j].cols > KC && !p.job[j].idx)
            return true;
    return false;
}

template <int MT, int CTAS, class P = GemvParams>
cudaError_t launch_mt(const P &p, int num_sms, int grid_limit, cudaStream_t stream, bool pdl, bool coop = false) {
    if constexpr (CTAS == 1)
        if (any_grouped(p))
            return launch_mt_g<MT, CTAS, P, true>(p, num_sms, grid_limit, stream, pdl, coop);
    return launch_mt_g<MT, CTAS, P, false>(p, num_sms, grid_limit, stream, pdl, coop);
}

template <int MT, int CTAS, class P>
cudaError_t setup_both() {
    cudaError_t e = setup_mt<MT, CTAS, P, false>(nullptr);
    if constexpr (CTAS == 1)
        if (e == cudaSuccess)
            e = setup_mt<MT, CTAS, P, true>(nullptr);
    return e;
}

} // namespace

// Tile bookkeeping shared by both launchers: checks the jobs, fills tiles / tile0 / total_tiles,
// and returns the stages (tile x chunk) of the launch (-1 for an invalid job list).
template <class P>
long long plan_tiles(P &p, int max_jobs) {
    if (p.njobs < 1 || p.njobs > max_jobs)
        return -1;
    const int m = p.job[0].m;
    int tiles = 0;
    long long stages = 0;
    for (int j = 0; j < p.njobs; ++j) {
        GemvJob &J = p.job[j];
        if (J.m != m || J.m < 1 || J.m > GEMV_MAX_T || J.cols < Q8_QK || J.cols % Q8_QK || J.rows < 1)
            return -1;
        const long long rpt = J.w2 ? R / 2 : R;
        J.tiles = int((J.rows + rpt - 1) / rpt);
        J.tile0 = tiles;
        tiles += J.tiles;
        stages += (long long)J.tiles * ((J.cols + KC - 1) / KC);
    }
    p.total_tiles = tiles;
    return stages;
}

cudaError_t launch_gemv(GemvParams &p, int num_sms, int grid_limit, cudaStream_t stream, bool pdl) {
    const long long stages = plan_tiles(p, MAX_JOBS);
    if (stages < 0)
        return cudaErrorInvalidValue;
    const int sms = num_sms > 0 ? num_sms : 148;
    switch (p.job[0].m) {
    case 1:
        return stages >= (long long)TWO_CTA_MIN_STAGES_PER_SM * sms ? launch_mt<1, 2>(p, num_sms, grid_limit, stream, pdl)
                                                                    : launch_mt<1, 1>(p, num_sms, grid_limit, stream, pdl);
    case 2: return launch_mt<2, 1>(p, num_sms, grid_limit, stream, pdl);
    case 3: return launch_mt<3, 1>(p, num_sms, grid_limit, stream, pdl);
    default: return launch_mt<4, 1>(p, num_sms, grid_limit, stream, pdl);
    }
}

cudaError_t preload_gemv() {
    cudaError_t e;
    if ((e = setup_both<1, 1, GemvParams>()) != cudaSuccess || (e = setup_both<1, 2, GemvParams>()) != cudaSuccess ||
        (e = setup_both<2, 1, GemvParams>()) != cudaSuccess || (e = setup_both<3, 1, GemvParams>()) != cudaSuccess ||
        (e = setup_both<4, 1, GemvParams>()) != cudaSuccess || (e = setup_both<1, 1, ChainParams>()) != cudaSuccess ||
        (e = setup_both<2, 1, ChainParams>()) != cudaSuccess || (e = setup_both<3, 1, ChainParams>()) != cudaSuccess ||
        (e = setup_both<4, 1, ChainParams>()) != cudaSuccess)
        return e;
    cudaFuncAttributes a;
    return cudaFuncGetAttributes(&a, wait_probe_kernel);
}

cudaError_t launch_wait_probe(const unsigned *ctr, unsigned *err, cudaStream_t stream) {
    if (!ctr || !err)
        return cudaErrorInvalidValue;
    wait_probe_kernel<<<1, 32, 0, stream>>>(ctr, err);
    return cudaGetLastError();
}

cudaError_t launch_gemv_chain(ChainParams &p, int num_sms, cudaStream_t stream) {
    if (plan_tiles(p, MAX_CHAIN_JOBS) < 0)
        return cudaErrorInvalidValue;
    switch (p.job[0].m) {
    case 1: return launch_mt<1, 1, ChainParams>(p, num_sms, 0, stream, false, true);
    case 2: return launch_mt<2, 1, ChainParams>(p, num_sms, 0, stream, false, true);
    case 3: return launch_mt<3, 1, ChainParams>(p, num_sms, 0, stream, false, true);
    default: return launch_mt<4, 1, ChainParams>(p, num_sms, 0, stream, false, true);
    }
}

} // namespace q8
