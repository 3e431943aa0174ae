// q8_kernels.h: what the host shim (rt_b200.cu) sees of the kernels: the job tables and the
// launchers. Plain pointers and integers; every pointer is device memory.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace q8 {

constexpr int MAX_JOBS = 16;  // products one launch serves (a round: the reference queues <= 8)
constexpr int GEMV_MAX_T = 4; // tokens per pass of the CUDA-core kernel (larger t: several passes)
constexpr int MAX_WAITS = 4;  // earlier rounds a chained round can wait on (more: a new launch)

// One product of the CUDA-core kernel: y[t][o] = sum_k W[row(o)][k] * x[t][k] for o < rows,
// t < m, in the reference's rounding order. row(o) = idx ? idx[o] : o. With w2 set the job is a
// fused SwiGLU pair: y[t][o] = silu((Wg x)[o]) * (Wu x)[o], w = Wg, w2 = Wu.
struct GemvJob {
    const uint8_t *w;   // row-split layout (q8_layout.h)
    const uint8_t *w2;  // the up matrix of a SwiGLU pair, or null
    const int32_t *idx; // row gather list, or null
    const float *x;     // [m][ldx]
    float *y;           // [m][ldy]
    long long rows;     // outputs per token
    long long src_rows; // rows of w (a gather's indices are checked against it)
    long long ldx, ldy;
    int cols;           // a multiple of 32
    int m;              // tokens, 1..GEMV_MAX_T
    int tiles;          // row tiles of this job (filled by the launcher)
    int tile0;          // its first tile in the launch (filled by the launcher)
    // Chained launches (launch_gemv_chain): the job's round counts its finished row tiles into
    // done_ctr; the job starts its tiles (reads x, and later writes y) only once
    // *wait_ctr[i] >= wait_target[i] for every i < nwait: the tile counts of the earlier rounds it
    // depends on. Null / 0 in plain launches.
    unsigned *done_ctr;
    const unsigned *wait_ctr[MAX_WAITS];
    unsigned wait_target[MAX_WAITS];
    int nwait;
    int x_written;      // chained: x overlaps a y written earlier in the launch (read it past L1)
};
// Chained launches' round counters sit one per 128-byte line (pollers and the tile counts of
// other rounds do not share it).
constexpr int ROUND_CTR_STRIDE = 32;

// ---- the all-gather of a row-sharded product over NVLink (one job per launch)
// Each rank owns a peer region, mapped by every other rank (CUDA IPC):
//   [0, 64)     flags[w]: uint64, the last round rank w has published (w's gather kernel writes it)
//   [64, 128)   reads[w]: uint64, the last round rank w has copied out of its own staging
//   [128, 132)  uint32, the product kernel's finished CTAs (local use)
//   [132, 136)  uint32, the gather kernel's finished CTAs (local use)
//   [136, 144)  uint64, rounds produced by this rank (advanced by the product kernel's last CTA)
//   [144, 152)  uint64, rounds gathered by this rank (advanced by the gather kernel's last CTA)
//   [PEER_HDR, +PEER_IMAGES*PEER_STAGE_BYTES)  staging images of y, [t][rows] fp32, round r in
//               image r % PEER_IMAGES.
// Round r: the product kernel (R's stream) stores each output into its local y and into image r
// of every peer (NVLink stores), and its last CTA advances the round count; nothing else, so the
// next product follows at once (with its programmatic early start). The rounds are gathered in
// batches of up to GATHER_BATCH: after a batch's last product (an event), a small gather kernel on
// a side stream publishes the batch (a system-scope fence, then its last round as its flag in
// every peer's region), waits (bounded) for every peer's flag, copies the peers' rows of each
// round from its own images into that round's y, tells every peer it has read the batch, and
// waits (bounded) until every peer has read it too. A product whose image was last used by round
// q waits (on R's stream, an event) for the gather of the batch holding q: with 16 images and
// batches of 8 that batch is long done. Batches, not rounds: an event between two products costs
// the second one its early start, ~3.6 us a round on 2 GPUs (products alone 1.41 ms a step, with
// an event pair per round 1.88, with a gather per round 2.14). No product kernel ever waits on
// another GPU: the cross-GPU waits are all in the gather kernels.
constexpr int MAX_PEERS = 8;
constexpr size_t PEER_HDR = 256;
constexpr int PEER_IMAGES = 16;
constexpr int GATHER_BATCH = 8;
constexpr size_t PEER_STAGE_BYTES = size_t(8) << 20; // t * rows * 4 bytes at most (the head at t = 4: 2.4 MB)
constexpr size_t PEER_REGION_BYTES = PEER_HDR + PEER_IMAGES * PEER_STAGE_BYTES;
constexpr size_t PEER_FLAGS = 0, PEER_READS = 64, PEER_PCTAS = 128, PEER_GCTAS = 132, PEER_PRODUCED = 136,
                 PEER_GATHERED = 144;
__host__ __device__ constexpr size_t peer_image(unsigned long long round) {
    return PEER_HDR + size_t(round % PEER_IMAGES) * PEER_STAGE_BYTES;
}

struct PeerOut {
    unsigned char *region[MAX_PEERS]; // every rank's region as mapped on this GPU (own: local)
    long long row0, rows_total;       // this rank's first output row; the product's rows
    int rank, world, on;              // on = 0: an unsharded launch
};

template <int NJ>
struct GemvParamsT {
    GemvJob job[NJ];
    int njobs;
    int total_tiles;
    int early;     // 1: weights may stream in before the previous kernel on the stream completes
    unsigned *err; // the context's device error word
    PeerOut peer;  // peer.on: one job, row-sharded; y is gathered through the peers' staging
    // An opened round (rt_gemv_open): the kernel is launched before its x has landed. It streams
    // its weights at once, but reads x (and row lists) only once *gate has reached gate_value
    // (written by the link stream after the round's pulls, at rt_gemv_go), bounded like every
    // wait. Null: no gate.
    const unsigned *gate;
    unsigned gate_value;
    // A round whose y also goes straight to the host (rt_b200_push of a held round, one job):
    // every output is stored at y_host[the same index] as well (mapped pinned host memory, the
    // device's address of it), and the last CTA to finish advances host_ctr[1] (the direct
    // rounds so far, device memory) and writes its new value into *host_flag (mapped host memory,
    // which the host polls) after a system-scope fence, so that the host sees y whole once it
    // sees the flag. host_ctr[0] counts the finished CTAs (left at 0). The parameters hold no
    // per-launch value, so a CUDA graph of the round can be launched again as it is.
    // Null y_host: none of it.
    float *y_host;
    unsigned *host_flag;
    unsigned *host_ctr;
};
using GemvParams = GemvParamsT<MAX_JOBS>;

// A chain: a sequence of rounds (each one or more jobs, all with the same m) in ONE persistent,
// cooperative launch. Weights stream across round boundaries without a launch in between; a
// round that depends on an earlier one waits on the device for that round's tiles (bounded)
// before it reads x. 160 jobs fit the kernel parameters (one decode step is 129 rounds).
constexpr int MAX_CHAIN_JOBS = 160;
using ChainParams = GemvParamsT<MAX_CHAIN_JOBS>;
// Fills the tile fields (the done/wait fields are the caller's). One CTA shape for the chain.
cudaError_t launch_gemv_chain(ChainParams &p, int num_sms, cudaStream_t stream);
// The bounded waits' self-test (rt_b200_wait_probe): *ctr must be 0 and stay 0.
cudaError_t launch_wait_probe(const unsigned *ctr, unsigned *err, cudaStream_t stream);

// ---- the host-half primitives beside the products (host_prims.cu)
constexpr int MAX_PRIM_HEADS = 128; // query heads of one call
constexpr int MAX_PRIM_GROUP = 16;  // query heads of one kv head in one ip12_kv CTA (8 threads each)
struct PrimHeads {
    long long l[MAX_PRIM_HEADS]; // the kv head of each query head
    int ord[MAX_PRIM_HEADS];     // the query heads sorted by kv head (stable): neighbours share rows
};
// The query heads grouped by kv head, each group <= MAX_PRIM_GROUP heads: group g is heads
// head[first[g] .. first[g+1]) of kv head kv[g].
struct PrimGroups {
    int n;
    int first[MAX_PRIM_HEADS + 1];
    int head[MAX_PRIM_HEADS];
    long long kv[MAX_PRIM_HEADS];
};
cudaError_t launch_ip21(float *z, const float *a, long long h, long long r, long long c, const float *b,
                        cudaStream_t stream);
cudaError_t launch_ip21_kv(float *z, const float *kv, long long n1, long long c, const PrimHeads &heads, long long h,
                           long long t, const float *b, cudaStream_t stream);
cudaError_t launch_ip12_kv(float *z, const float *a, const float *kv, long long n1, long long c, const PrimGroups &groups,
                           long long t, unsigned *err, cudaStream_t stream);
// A 2-D fp32 tensor map (no swizzle, zero fill) into `map` (a CUtensorMap, 64-byte aligned):
// `outer` rows of `inner` floats, `stride_bytes` apart, boxes of box_inner x box_outer.
bool map_f32_2d(void *map, const float *base, uint64_t inner, uint64_t outer, uint64_t stride_bytes,
                uint32_t box_inner, uint32_t box_outer);
cudaError_t launch_scale_outer(float *z, const float *s, float g, const float *a, const float *b, long long m,
                               long long k, cudaStream_t stream);
cudaError_t preload_prims();

// A batch of consecutive peer-gathered rounds (the protocol above), gathered on the side stream
// after the batch's last product: round i's y is [t[i]][rows[i]], its own rows in place.
struct GatherBatch {
    float *y[GATHER_BATCH];
    long long rows[GATHER_BATCH];
    int t[GATHER_BATCH];
    int n;
};
cudaError_t launch_peer_gather(const PeerOut &po, const GatherBatch &b, unsigned *err, cudaStream_t stream);

// Launches the exact CUDA-core product over p.job[0..njobs) (all with the same m). Fills the
// tile fields. grid_limit 0 = one CTA per SM. pdl: launch with programmatic stream serialization
// (the kernel overlaps the previous one's tail and waits for it before reading x or idx).
cudaError_t launch_gemv(GemvParams &p, int num_sms, int grid_limit, cudaStream_t stream, bool pdl);

// ---- the tensor-core gemm (t >= 16): y[t][o] = sum_k fp16(W)[o][k] * fp16(x)[t][k], fp32 sums
struct GemmJob {
    const uint8_t *w;   // row-split layout
    const uint8_t *w2;  // SwiGLU up matrix, or null
    const float *x;     // [t][ldx] fp32 (rounded to fp16 into scratch by the launcher)
    float *y;           // [t][ldy]
    long long rows;
    long long ldx, ldy;
    int cols;
    int t;
};

// Scratch (device bytes) launch_gemm_tc needs for these jobs: their x in fp16, and with split_k
// the fp32 partial sums of jobs whose K is split (launches with fewer row-tile units than SMs).
size_t gemm_tc_scratch_bytes(const GemmJob *jobs, int n, int num_sms, bool split_k);
// Up to 8 jobs in one persistent launch (plus one fp16 conversion of each x, and with split_k one
// reduce pass per split job).
cudaError_t launch_gemm_tc(const GemmJob *jobs, int n, void *scratch, size_t scratch_bytes, int num_sms,
                           unsigned *err, cudaStream_t stream, bool pdl, bool split_k);

// Each kernel file's kernels loaded and their attributes set on the current device (rt_init calls
// these, so that no later launch does it first: under lazy module loading the first launch of a
// kernel may have to wait for the GPU, which a gated kernel of an opened round holds until go).
cudaError_t preload_gemv();
cudaError_t preload_gemm_tc();
cudaError_t preload_peer();

// ---- utilities
// The repack stages a whole GGUF row in shared memory (what makes it safe in place): rows of at
// most this many GGUF bytes, i.e. cols <= 192,736.
constexpr long long REPACK_MAX_ROW_BYTES = 200 * 1024;
cudaError_t launch_repack(const uint8_t *gguf, long long rows, int cols, uint8_t *out, cudaStream_t stream);
cudaError_t launch_synth_q8(uint8_t *out_split, long long row0, long long rows, int cols, uint64_t seed,
                            uint64_t stream_id, float sigma, cudaStream_t stream);
cudaError_t launch_synth_f32(float *out, long long n, uint64_t seed, uint64_t stream_id, float sigma,
                             cudaStream_t stream);
cudaError_t launch_q8_row(const uint8_t *w, int cols, long long row, float *z, cudaStream_t stream);

}  // namespace q8
