/* rt_b200.h: the C ABI of the B200 Q8_0 weight products (librt_b200.so).
 *
 * It keeps the reference runtime's product entry points (Lasimeri/Intel-Phi-APL, src/card/rt.h)
 * with their prototypes unchanged, so the code the APL compiler generates for every Q8_0 product
 * (src/apl/compiler/em.apl:601-617) links against this library as it is. What changes is where
 * the data lives and who computes:
 *
 *   - w, x, y (and z, idx) are DEVICE pointers in HBM on the calling thread's current CUDA device;
 *   - w is a matrix in the row-split Q8_0 layout (gemv_s_bytes / gemv_s_repack below), not the
 *     reference's form I;
 *   - the products run as sm_100a CUDA kernels; y is bit-identical to the reference's host model
 *     for t < 16 tokens (fp32, same rounding order) and within 2e-3 (relative, rms floor) for the
 *     tensor-core path at t >= 16 (fp16 operands, fp32 sums);
 *   - by default every product call returns with its results in y (the reference's team_run is
 *     blocking too); rt_b200_set_async makes them stream-ordered instead.
 *
 * Preconditions, as the reference states them (src/card/rt.h:5-8, src/card/gemv.h:1): cols a
 * multiple of 32. Unlike the reference, rows need not be a multiple of 16 and every argument is
 * checked: a call that cannot run does nothing and records an error for rt_b200_last_error(). The
 * reference's functions are void and check nothing (src/card/rt.c:205-285).
 *
 * Thread safety: one calling thread per struct rt, as in the reference (its queue is static
 * state, src/card/rt.c:217-226); different struct rt may be used from different threads. */
#ifndef RT_B200_H
#define RT_B200_H
#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define RTB_API __attribute__((visibility("default")))
#else
#define RTB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

struct team;
struct gemm_chain;

/* The reference's runtime state, field for field (src/card/rt.h:19-26), so generated code that
 * declares one compiles unchanged. Here `chain` holds this library's device context (stream,
 * queue, error word, scratch); team and gemm_chain stay NULL; threads is stored, not used. */
struct rt {
    struct team *team;
    char *frame;
    void *chain;
    struct gemm_chain *gemm_chain;
    int threads;
    int last;
};

/* ---------------------------------------------------------------- the reference's products */

/* src/card/rt.h:39 (rt.c:179-203). Binds R to the current CUDA device: creates its stream, error
 * word and queue. 0, or -1 (no device, no memory). `threads` is kept in R->threads only. */
RTB_API int rt_init(struct rt *R, int threads);

/* src/card/rt.h:62 (rt.c:205-214). y[rows] = W x, W rows x cols Q8_0 (row-split), x[cols]. */
RTB_API void rt_gemv(struct rt *R, const void *w, long rows, long cols, const float *x, float *y);

/* src/card/rt.h:65-69 (rt.c:217-285). The round: queue up to RT_BATCH products that do not read
 * each other's results, then rt_gemv_go runs all of them in one launch per kind and clears the
 * queue.
 * rt_gemv_open opens the round before its x has landed, as the reference does (rt.c:267-285: its
 * threads read ahead until go). Here the round's CUDA-core products (t < 16) are launched at once:
 * they stream their weights while the host still prepares x, and wait on the GPU (bounded, about a
 * second) for go before they read x or a row list. Between open and go the host may pull the
 * round's inputs (rt_b200_pull then copies on a link stream of R's, which first waits for the work
 * already on R's stream); rt_gemv_go releases the round after those copies and launches the rest.
 * As in the reference (src/card/team.h:21-24), nothing else may use R between open and go: a
 * product or push on R's stream would wait for the opened round, whose wait for go then gives up
 * and reports RTB_EKERNEL. rt_b200_sync closes an open round without releasing it (its kernel gives
 * up and the error is returned). Open does nothing (go runs everything) for tensor-core products,
 * row-sharded runtimes, chains, and while R's stream is being captured into a graph. */
#define RT_BATCH 8
RTB_API void rt_gemv_q(struct rt *R, const void *w, long rows, long cols, const float *x, float *y);
RTB_API void rt_gemv_open(struct rt *R);
RTB_API void rt_gemv_go(struct rt *R);

/* src/card/rt.h:71-72 (rt.c:244-265). Y = X W^T for t tokens: x [t cols], y [t rows], rows
 * contiguous. One pass over the weights serves up to 4 tokens on CUDA cores (t < 16, exact); from
 * t = 16 the tensor cores take the whole product in one pass. */
RTB_API void rt_gemm(struct rt *R, const void *w, long rows, long cols, const float *x, long t, float *y);
RTB_API void rt_gemm_q(struct rt *R, const void *w, long rows, long cols, const float *x, long t, float *y);

/* src/card/rt.h:85 (rt.c:484-501). z[cols] = row `row` of W dequantised: z[i] = (float)q * d. */
RTB_API void rt_q8_row(const void *w, long cols, long row, float *z);

/* ---- The host-half primitives beside the products: the inner products over an attention head's
 * history and the delta rule's state products, which the reference runs on its host worker
 * (src/host/rt_host.c:128-279, prototypes src/card/rt.h:73-82). Here they run on the GPU, on R's
 * stream (blocking unless async, as the products), with device pointers and the reference's
 * rounding order bit for bit: a dot product is 8 lanes of fma chains over columns j, j+8, ...
 * summed ((l0+l4)+(l2+l6))+((l1+l5)+(l3+l7)) (src/host/vec8.h:49-55). c is a multiple of 8;
 * l (host memory, h <= 128 entries) gives each query head's kv head, in [0, n1); kv is
 * [t][n1][c] and 16-byte aligned. Not inside a chain. */
/* z[h*t + s] = dot(kv[s][l[h]][:], b[h][:]) (src/host/rt_host.c:135-162) */
RTB_API void rt_ip21_kv(struct rt *R, float *z, const float *kv, long n1, long c, const long *l, long h, long t,
                        const float *b);
/* z[h][k] = fma(a[h][s], kv[s][l[h]][k], z[h][k]) over s = 0..t-1 in order, from 0
 * (src/host/rt_host.c:164-189) */
RTB_API void rt_ip12_kv(struct rt *R, float *z, const float *a, const float *kv, long n1, long c, const long *l, long h,
                        long t);
/* z[h][i] = dot(a[h][i][:], b[h][:]), a as [h][r][c] (src/host/rt_host.c:200-247) */
RTB_API void rt_ip21(struct rt *R, float *z, const float *a, long h, long r, long c, const float *b);
/* z[i][q] = fma(g, s[i][q], a[i] * b[q]), the product rounded first, m x k (src/host/rt_host.c:261-279;
 * any k here, a multiple of 8 there) */
RTB_API void rt_scale_outer(struct rt *R, float *z, const float *s, float g, const float *a, const float *b, long m,
                            long k);

/* ---------------------------------------------------------------- load side */

/* Bytes of a rows x cols matrix in the row-split layout: each row holds its cols int8 quants
 * (16-byte aligned) then its cols/32 fp16 scales padded to a multiple of 8. Equals the GGUF size
 * rows*cols*34/32 when cols is a multiple of 256. Replaces gemv_i_bytes (src/card/gemv.h:51). */
RTB_API long gemv_s_bytes(long rows, long cols);

/* GGUF Q8_0 rows (per 32 columns: fp16 d, 32 int8 q) -> the row-split layout, on the device.
 * q8 and out are device pointers; out == q8 (in place) is allowed when cols % 256 == 0, as the
 * reference repacks in place at load (src/card/gemv.c:42-52, src/card/engine.c:303-316).
 * cols <= 192,736 (a GGUF row of at most 200 KiB, staged whole in shared memory).
 * Returns 0 or an RTB_E* code. Replaces gemv_i_repack (src/card/gemv.h:55). */
RTB_API int gemv_s_repack(const void *q8, long rows, long cols, void *out);

/* The reference's load-side names (src/card/gemv.h:51-67), so the engine's load site
 * (src/card/engine.c:295-316) links unchanged: they produce this library's row-split layout
 * under the old names. gemv_i_bytes = gemv_s_bytes. gemv_i_repack = gemv_s_repack (void, as in
 * the reference; a failure is recorded for rt_b200_last_error(NULL)). gemv_i_repack_thread is a
 * team body, as the engine runs it (team_run(R.team, gemv_i_repack_thread, &job) on n threads):
 * thread 0 repacks the whole matrix in place on the GPU (job->w a device pointer, cols % 256 == 0,
 * so a row keeps its length) and returns when it is done; the other threads return at once, and
 * job->tmp (the reference's per-thread scratch) is not used. */
struct gemv_repack_job {
    void *w;
    long rows, cols;
    void *tmp;
};
RTB_API long gemv_i_bytes(long rows, long cols);
RTB_API void gemv_i_repack(const uint8_t *q8, long rows, long cols, void *out);
RTB_API void gemv_i_repack_thread(void *arg, int tid, int n);

/* ---------------------------------------------------------------- fused products
 * The reference runs these as separate queued gemvs plus host work (src/apl/qwen35.apl:124-126,
 * 170-172; src/apl/compiler/em.apl:820-840). Here each is one pass in the queued round. */

/* h[t][rows] = silu(Wg x)[t] * (Wu x)[t]: the SwiGLU gate and up products fused, each product in
 * the reference's exact order before the fp32 silu(g)*u = g/(1+exp(-g))*u. t >= 1. */
RTB_API void rt_gemm_silu_q(struct rt *R, const void *w_gate, const void *w_up, long rows, long cols, const float *x,
                    long t, float *h);
RTB_API void rt_gemm_silu(struct rt *R, const void *w_gate, const void *w_up, long rows, long cols, const float *x, long t,
                  float *h);

/* y[i] = row idx[i] of W times x, i < n: the draft head's product over a subset of the output
 * matrix's rows (DraftLogits, src/apl/qwen35.apl:170-172; the reference takes a row prefix,
 * this takes any list). W has w_rows rows; idx is a device array of n int32 row numbers. An index
 * outside [0, w_rows) is not read: its y is NaN and the call reports RTB_EKERNEL. */
RTB_API void rt_gemv_rows_q(struct rt *R, const void *w, long w_rows, const int32_t *idx, long n, long cols,
                            const float *x, float *y);
RTB_API void rt_gemv_rows(struct rt *R, const void *w, long w_rows, const int32_t *idx, long n, long cols,
                          const float *x, float *y);

/* No counterpart in the reference. The tensor-core product of rt_gemm (t >= 16 tokens, same kernel
 * and same results) for callers that cannot allocate device memory: engines that reserve all of
 * HBM up front or forbid allocation while serving. It needs no rt_init, and its scratch (the fp16
 * copy of x) is a fixed 8 MiB device array inside this library, so t * cols must be <= 4,194,304;
 * larger calls return RTB_EINVAL. Runs on `stream` (a cudaStream_t; NULL is the legacy default
 * stream) and returns after the product is in y: RTB_OK, or RTB_EINVAL / RTB_ECUDA / RTB_EKERNEL.
 * The first call on a device looks up that array's device address: make it before any stream
 * capture. All calls share the array, so calls that overlap on the GPU (two threads or two
 * streams at once) race and must not be made. */
RTB_API int rt_gemm_static(const void *w, long rows, long cols, const float *x, long t, float *y, void *stream);

/* ---------------------------------------------------------------- B200 runtime controls */

enum {
    RTB_OK = 0,
    RTB_EINVAL = 1,   /* an argument the products cannot take (size, alignment, null) */
    RTB_ECUDA = 2,    /* a CUDA runtime call failed */
    RTB_EKERNEL = 3,  /* a kernel reported through its error word: a bounded wait that gave up, or a
                         gather index outside the matrix */
    RTB_ENOMEM = 4,   /* device memory */
    RTB_ENOTINIT = 5, /* R was not initialised by rt_init */
    RTB_EQUEUE = 6,   /* more than RT_BATCH*2 queued products */
    RTB_ENCCL = 7,    /* a collective failed */
};

/* The first error since the last call (0 if none), for R (or, with R NULL, for the calling
 * thread's calls that take no R: rt_q8_row, gemv_s_repack); reading it clears it. If msg is not
 * NULL, up to n bytes of a description are written there. */
RTB_API int rt_b200_last_error(struct rt *R, char *msg, size_t n);

/* 0: every product call returns after its results are in y (default). 1: calls only enqueue on
 * R's stream; rt_b200_sync waits and returns the first error. */
RTB_API void rt_b200_set_async(struct rt *R, int on);
RTB_API int rt_b200_sync(struct rt *R);

/* The link crossing of a round, where the engine keeps x and y in host memory (the reference's
 * link_pull / link_push, src/card/link.c:86-118). pull enqueues a host -> device copy of `bytes`
 * on R's stream (on its link stream while a round is open) and returns; push enqueues the
 * device -> host copy, waits for R's stream (the bytes are on the host at return, and a kernel's
 * error word is read) and returns 0 or the first error. Pinned host memory keeps the copies
 * asynchronous. A round: queue the product, rt_gemv_open, pull x, rt_gemv_go (async mode), push y. */
RTB_API int rt_b200_pull(struct rt *R, void *dev, const void *host, size_t bytes);
RTB_API int rt_b200_push(struct rt *R, void *host, const void *dev, size_t bytes);

/* 1: the caller vouches that no kernel between products writes the weight matrices (model
 * weights are read-only after load). Each product kernel is then launched with programmatic
 * dependent launch and streams its weights while the previous kernel on the stream finishes; it
 * still waits for that kernel before reading x or a row list and before writing y. 0 (default):
 * products start after the previous kernel completes, as plain stream order. */
RTB_API void rt_b200_set_overlap(struct rt *R, int on);

/* No counterpart in the reference (its link_push is a DMA copy, src/card/link.c:105-118). 1: a
 * round's y may come back from its own product kernel. In async mode rt_gemv_go then holds back a
 * round of one CUDA-core product (t <= 4, one GPU, no chain, R's stream not being captured)
 * instead of launching it, and the next call on R launches it. When that call is rt_b200_push of
 * exactly that product's y (dev = y, bytes = t * rows * 4) into pinned host memory the GPU can
 * write (cudaHostAlloc, or cudaHostRegister'd and mapped: on 64-bit systems with unified
 * addressing any pinned memory), the kernel also stores each output there and its last CTA raises
 * a flag in mapped host memory; push returns once the host sees the flag (y is then whole on the
 * host) with the round's error status, without a device-to-host copy or a stream synchronization.
 * Any other call on R, or a push of anything else, launches the held round first as rt_gemv_go
 * would have. The held product runs as a CUDA graph, captured the first time that round (same
 * product, same y) comes and launched as it is when it comes again (an engine's rounds repeat
 * every token; at most 4096 graphs are kept). The caller vouches that between rt_gemv_go and its
 * next call on R it enqueues nothing of its own on R's stream that needs the held product.
 * 0 (default): go launches at once. */
RTB_API void rt_b200_set_push_direct(struct rt *R, int on);

/* R's CUDA stream (a cudaStream_t); set_stream makes R use the caller's stream instead (NULL:
 * back to R's own; the legacy default stream is cudaStreamLegacy, not NULL). */
RTB_API void *rt_b200_stream(struct rt *R);
RTB_API void rt_b200_set_stream(struct rt *R, void *stream);

/* Frees what rt_init made. R can be initialised again. */
RTB_API void rt_b200_free(struct rt *R);

/* ---------------------------------------------------------------- row sharding over GPUs
 * One process per GPU. With world > 1, every product's w is this rank's row shard (rows/world
 * consecutive rows, rank-major, rows % world == 0) while rows, y and t keep the whole product's
 * meaning: each rank computes its rows and y is filled on every rank over NVLink.
 * - A single product of <= 4 tokens (rt_gemv, rt_gemm, rt_gemm_silu) gathers y over NVLink
 *   without NCCL: the product kernel also stores every output into each peer's staging buffer
 *   (CUDA IPC mappings set up by rt_b200_shard), and a small gather kernel on a side stream of
 *   R's, once per 8 such products, publishes them, waits (bounded) for the peers', and copies
 *   their rows into each product's y. R's stream goes on with the next product at once; it waits
 *   for a gather only where it must: a product whose x or y overlaps a y still being gathered,
 *   the product 16 rounds later (the staging buffers' reuse), and whatever else runs, pulls or
 *   pushes on R, or R synchronized or flushed. So in async mode y is whole, on R's stream, for what follows; blocking calls return
 *   with y whole. A sequence captured into a CUDA graph must end with rt_b200_flush, which joins
 *   the side stream back into the capture.
 * - Queued rounds, t > 4 and the tensor-core path all-gather y with NCCL.
 * All ranks must issue the same products in the same order. nccl_id is the 128-byte ncclUniqueId
 * from rt_b200_nccl_id on rank 0, passed to every rank by the caller. 0 or an RTB_E* code.
 * The environment variable RTB_NO_PEER_GATHER (set before rt_b200_shard) keeps every round on
 * NCCL. rt_b200_peer_gather: 1 when the in-kernel gather is set up, else 0. */
RTB_API int rt_b200_nccl_id(void *out128);
RTB_API int rt_b200_shard(struct rt *R, int rank, int world, const void *nccl_id);
RTB_API int rt_b200_peer_gather(struct rt *R);

/* Enqueues the kernel that finishes a row-sharded product's pending gather, if one is pending (a
 * no-op otherwise, and with one GPU). Can be captured into a graph. 0 or an RTB_E* code. */
RTB_API int rt_b200_flush(struct rt *R);

/* The rows of a rows-row matrix that rank `rank` of `world` holds and computes, as the products
 * split them: *row0 and *n (rows / world consecutive rows, rank-major). Host only, no device: an
 * engine loads each matrix's shard with it. 0, or RTB_EINVAL (rows % world != 0, bad rank). */
RTB_API int rt_b200_shard_rows(long rows, int rank, int world, long *row0, long *n);

/* A self-test of the failure path: one kernel on R's stream waits, bounded, on a device counter
 * that nothing advances and then on an mbarrier that nothing arrives on, the two kinds of wait the
 * product kernels make. Each gives up after about a second and reports through the error word, as
 * a stuck wait in a product does. Returns RTB_EKERNEL (also recorded for rt_b200_last_error, whose
 * message names both waits) after about two seconds; R stays usable. No GPU fault is involved. */
RTB_API int rt_b200_wait_probe(struct rt *R);

/* ---------------------------------------------------------------- chains: rounds in one launch
 * Between rt_b200_chain_begin and rt_b200_chain_end, products (rt_gemv, rt_gemm, rt_gemm_silu,
 * rt_gemv_rows) and queued rounds (rt_gemv_go) are recorded, not run: each call or go is one round.
 * rt_b200_chain_end runs them in order as ONE persistent launch per 160 products (one decode step
 * is 129 rounds): weights stream across round boundaries with no launch in between, and a round
 * that depends on earlier rounds waits for them on the GPU before it reads x or writes y.
 * serial != 0 makes every round wait for the one before (a decode step's dependency chain);
 * serial == 0 makes a round wait for every earlier round it conflicts with: its x overlaps their
 * y (read after write), or its y overlaps their x (write after read) or their y (write after
 * write). A round with more than four such rounds not already covered by each other's waits
 * starts a new launch. Rounds that cannot chain (t > 4, the tensor-core path, several GPUs) run
 * as separate launches in the same order. Blocking mode waits at rt_b200_chain_end. 0 or an
 * RTB_E* code. */
RTB_API int rt_b200_chain_begin(struct rt *R);
RTB_API int rt_b200_chain_end(struct rt *R, int serial);

/* ---------------------------------------------------------------- the weight loader
 * A GGUF file into device memory, its Q8_0 matrices repacked in place into the row-split layout
 * (the engine's load step: src/card/engine.c:268-330, src/card/stream.c:77-104).
 * rtb_gguf_info parses the header only (host): the tensor table and the file size. A header whose
 * sizes cannot be right (dims whose product wraps or exceeds 2^50 elements, a tensor running past
 * the file's end, rows that are not whole blocks, an alignment that is not a power of two) is
 * refused with RTB_EINVAL by both calls, before anything is read into the arena.
 * rt_b200_load_gguf reads the whole file into `arena` (device, >= the file size rounded up to 8,
 * 256-byte aligned) through page-aligned O_DIRECT reads into pinned buffers (buffered reads where
 * the file system refuses O_DIRECT), each slot's copy to the GPU overlapping the next read; then
 * computes the file's position-weighted sum (sum of word_i * (2i+1) mod 2^64 over 8-byte words,
 * src/bench/arena.h:26-44) on the GPU, and repacks every Q8_0 matrix whose rows keep their length
 * (cols % 256 == 0) in place, each distinct offset once. Tensor i is at arena + out[i].offset
 * (out[i].dev). Other types are left as they are in the file. 0 or an RTB_E* code;
 * rtb_load_error() tells what failed. */
typedef struct rtb_tensor {
    char name[96];
    int type;                  /* GGML type: 0 F32, 1 F16, 8 Q8_0, 30 BF16 */
    int n_dims;
    long long dim[4];          /* dim[0]: the fastest (columns) */
    unsigned long long offset; /* from the start of the file */
    unsigned long long bytes;
    void *dev;                 /* rt_b200_load_gguf: the tensor in the arena */
    int repacked;              /* 1: a Q8_0 matrix now in the row-split layout */
    int pad_;
} rtb_tensor;

typedef struct rtb_load_stats {
    unsigned long long file_bytes;
    unsigned long long file_sum; /* the position-weighted sum of the file */
    double seconds;              /* open to the end of the repack */
    double seconds_repack;       /* the sum and the repacks on the GPU, after the last copy */
    int direct;                  /* 1: the reads bypassed the page cache (O_DIRECT) */
    int q8_matrices;             /* Q8_0 matrices repacked */
} rtb_load_stats;

RTB_API int rtb_gguf_info(const char *path, rtb_tensor *out, int cap, int *n, unsigned long long *file_bytes);
RTB_API int rt_b200_load_gguf(struct rt *R, const char *path, void *arena, unsigned long long arena_bytes,
                              rtb_tensor *out, int cap, int *n, rtb_load_stats *stats);
RTB_API const char *rtb_load_error(void);

/* ---------------------------------------------------------------- synthetic inputs (benchmarks, tests)
 * Rows [row0, row0+rows) of a seeded Q8_0 matrix with w ~ sigma*N(0,1), written in the row-split
 * layout to dst (device); and n seeded fp32 values ~ sigma*N(0,1). The values are the same bits
 * the CPU generator of the tests produces for the same (seed, stream, index). 0 or RTB_E*. */
RTB_API int rtb_synth_q8_0(void *dst, long row0, long rows, long cols, uint64_t seed, uint64_t stream, float sigma);
RTB_API int rtb_synth_f32(float *dst, long n, uint64_t seed, uint64_t stream, float sigma);

#ifdef __cplusplus
}
#endif
#endif
