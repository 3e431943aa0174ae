// rt_b200.cu: the C ABI of include/rt_b200.h. Host code only: argument checks, the queued round,
// the split of a product into kernel launches, row sharding with an NCCL all-gather, and the
// error state. The reference's counterparts are src/card/rt.c:179-285 (products) and 484-501
// (rt_q8_row); there the work runs on a thread team, here on the GPU.
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <atomic>
#include <bitset>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <new>
#include <vector>

#include "../../include/rt_b200.h"
#include "q8_kernels.h"
#include "q8_layout.h"

// NCCL is resolved at run time, on first use (rt_b200_shard, rt_b200_nccl_id): loading this library
// loads no NCCL, and a process that already holds one (PyTorch bundles its own) shares it.
namespace {
struct Nccl {
    bool tried = false, ok = false;
    decltype(&ncclGetUniqueId) GetUniqueId = nullptr;
    decltype(&ncclCommInitRank) CommInitRank = nullptr;
    decltype(&ncclCommDestroy) CommDestroy = nullptr;
    decltype(&ncclAllGather) AllGather = nullptr;
    decltype(&ncclAllReduce) AllReduce = nullptr;
    decltype(&ncclGroupStart) GroupStart = nullptr;
    decltype(&ncclGroupEnd) GroupEnd = nullptr;
    decltype(&ncclGetErrorString) GetErrorString = nullptr;
};

Nccl &nccl() {
    static Nccl n;
    static std::once_flag once;
    std::call_once(once, [] {
        n.tried = true;
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h)
            h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h)
            return;
        n.GetUniqueId = reinterpret_cast<decltype(n.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
        n.CommInitRank = reinterpret_cast<decltype(n.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
        n.CommDestroy = reinterpret_cast<decltype(n.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
        n.AllGather = reinterpret_cast<decltype(n.AllGather)>(dlsym(h, "ncclAllGather"));
        n.AllReduce = reinterpret_cast<decltype(n.AllReduce)>(dlsym(h, "ncclAllReduce"));
        n.GroupStart = reinterpret_cast<decltype(n.GroupStart)>(dlsym(h, "ncclGroupStart"));
        n.GroupEnd = reinterpret_cast<decltype(n.GroupEnd)>(dlsym(h, "ncclGroupEnd"));
        n.GetErrorString = reinterpret_cast<decltype(n.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
        n.ok = n.GetUniqueId && n.CommInitRank && n.CommDestroy && n.AllGather && n.AllReduce && n.GroupStart &&
               n.GroupEnd && n.GetErrorString;
    });
    return n;
}
} // namespace

namespace {

constexpr int TC_MIN_T = 16; // from this many tokens the product is a dense contraction: tensor cores

enum Kind { K_GEMM, K_SILU, K_ROWS };

struct Item {
    Kind kind;
    const uint8_t *w, *w2;
    const int32_t *idx;
    const float *x;
    float *y;
    long long rows, cols, t;
    long long src_rows; // rows of w (a gather's bound)
};

struct Ctx {
    int device = 0, num_sms = 148;
    cudaStream_t own_stream = nullptr, stream = nullptr;
    bool async = false;
    bool overlap = false; // weights are read-only between products: prefetch them early (PDL)
    unsigned *d_err = nullptr;        // the error word (q8_ptx.cuh: bits, then the mirror's address)
    volatile unsigned *h_err = nullptr; // its mirror in mapped host memory: nonzero once a kernel reported
    bool synced = true;               // own stream, nothing enqueued on it since its last synchronize
    int status = RTB_OK;
    char msg[256] = {0};
    std::vector<Item> queue;
    int rank = 0, world = 1;
    ncclComm_t comm = nullptr;
    // the fused all-gather (q8_kernels.h, PeerOut): this rank's peer region and every rank's
    // mapping of it here; peer_ok false means rounds all-gather through NCCL instead
    unsigned char *peer_local = nullptr;
    unsigned char *peer_map[q8::MAX_PEERS] = {};
    bool peer_ok = false;
    // the row-sharded products' gathers (q8_kernels.h), in batches on a side stream: the stream;
    // the open batch (rounds launched, their gather not yet); the batches launched whose gathers
    // R's stream has not waited for (each with its last round, its events' slot: the batch's last
    // product done on R's stream, its gather done on the side stream, and the capture it was
    // recorded in, 0: none); the rounds issued and those R's stream has waited for; and the y of
    // the rounds not waited for (the hazards of later products)
    static constexpr int NSLOT = 4;
    cudaStream_t gside = nullptr;
    cudaEvent_t ev_prod[NSLOT] = {}, ev_gath[NSLOT] = {};
    q8::GatherBatch open_b = {};
    unsigned long long open_first = 0;
    struct Issued {
        unsigned long long last, cap;
        int slot;
    };
    std::vector<Issued> issued;
    int next_slot = 0;
    unsigned long long prounds = 0, waited = 0;
    struct PendingY {
        const float *y;
        size_t bytes;
        unsigned long long round;
    };
    std::vector<PendingY> pending;
    void *scratch = nullptr; // grows on demand (the tensor-core path's fp16 x)
    size_t scratch_bytes = 0;
    // chains (rt_b200_chain_begin .. rt_b200_chain_end): recorded rounds, and the device counters
    // of their finished tiles (one per round of a launch)
    bool chaining = false;
    std::vector<std::vector<Item>> chain;
    unsigned *d_round = nullptr;
    // opened rounds (rt_gemv_open .. rt_gemv_go): the gate word the pre-launched kernel waits on,
    // the rounds counted so far, and the link stream that carries the round's pulls and then the
    // gate's new value
    unsigned *d_gate = nullptr;
    unsigned gate_seq = 0;
    cudaStream_t link = nullptr;
    cudaEvent_t ev_before = nullptr, ev_link = nullptr;
    bool round_open = false;
    // direct pushes (rt_b200_set_push_direct): a round of one CUDA-core product that rt_gemv_go
    // held back instead of launching, its launch left to the next call on R; the host word the
    // product's last CTA raises (mapped, beside the error mirror), its device address, the
    // device counters behind it (finished CTAs, direct rounds) and the direct rounds launched so
    // far; the rounds' kernels as CUDA graphs (captured once on a private stream, launched as
    // they are for a round seen before)
    bool direct = false;
    bool held = false;
    Item held_item;
    volatile unsigned *h_flag = nullptr;
    unsigned *h_flag_dev = nullptr;
    unsigned *d_hctr = nullptr;
    unsigned host_seq = 0;
    cudaStream_t cap = nullptr;
    std::unordered_map<std::string, cudaGraphExec_t> graphs;
};

// cuStreamWriteValue32 (the driver's stream memory operation: executed by the GPU's front end in
// stream order, it needs no SM, so it cannot queue behind the gated kernel it releases), looked up
// through the runtime; null where the driver lacks it (rt_gemv_open then does nothing).
using WriteValue32 = CUresult (*)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);
WriteValue32 write_value32() {
    static WriteValue32 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void *f = nullptr;
        if (cudaGetDriverEntryPointByVersion("cuStreamWriteValue32", &f, 11070, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<WriteValue32>(f);
    });
    return fn;
}

bool flush_pending(Ctx *c);
bool overlaps(const void *a, size_t na, const void *b, size_t nb);
bool launch_held(Ctx *c);

// Errors of the calls that take no struct rt.
thread_local int t_status = RTB_OK;
thread_local char t_msg[256];

void set_err(int *status, char *msg, int code, const char *fmt, va_list ap) {
    if (*status != RTB_OK)
        return; // keep the first
    *status = code;
    vsnprintf(msg, 256, fmt, ap);
}

void ctx_err(Ctx *c, int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    set_err(&c->status, c->msg, code, fmt, ap);
    va_end(ap);
}

void thread_err(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    set_err(&t_status, t_msg, code, fmt, ap);
    va_end(ap);
}

Ctx *ctx_raw(struct rt *R) {
    if (!R || !R->chain) {
        thread_err(RTB_ENOTINIT, "struct rt not initialised by rt_init");
        return nullptr;
    }
    return static_cast<Ctx *>(R->chain);
}

// R's context for an entry point, after launching a round rt_gemv_go held back (every call on R but
// rt_b200_push, which may launch it with y going straight to the host, comes after that launch).
Ctx *ctx_of(struct rt *R) {
    Ctx *c = ctx_raw(R);
    if (c && c->held)
        launch_held(c);
    return c;
}

bool cuda_ok(Ctx *c, cudaError_t e, const char *what) {
    if (e == cudaSuccess)
        return true;
    ctx_err(c, e == cudaErrorMemoryAllocation ? RTB_ENOMEM : RTB_ECUDA, "%s: %s", what, cudaGetErrorString(e));
    return false;
}

bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

bool check_product(Ctx *c, const char *fn, const void *w, long long rows, long long cols, const float *x, long long t,
                   const float *y) {
    if (!w || !x || !y) {
        ctx_err(c, RTB_EINVAL, "%s: null pointer", fn);
        return false;
    }
    if (rows < 1 || cols < Q8_QK || cols % Q8_QK || t < 1 || cols > (1ll << 30) || rows > (1ll << 40) ||
        (t >= TC_MIN_T && (rows > (1ll << 31) || t > (1 << 20)))) {
        ctx_err(c, RTB_EINVAL, "%s: rows %lld cols %lld t %lld (cols a multiple of 32, all >= 1)", fn, rows, cols, t);
        return false;
    }
    if (!aligned(w, 16) || !aligned(x, 16) || !aligned(y, 4)) {
        ctx_err(c, RTB_EINVAL, "%s: w and x must be 16-byte aligned, y 4-byte aligned", fn);
        return false;
    }
    if (c->world > 1 && rows % c->world) {
        ctx_err(c, RTB_EINVAL, "%s: rows %lld not divisible by the %d shards", fn, rows, c->world);
        return false;
    }
    return true;
}

// The error word's bits (q8_ptx.cuh), named for the message.
void error_word_text(unsigned h, char *out, size_t n) {
    static const char *const names[] = {
        "a stage's bulk copy never completed",
        "a stage's partial sums never arrived",
        "the chain never released a partial-sum buffer",
        "a tensor-core stage never completed",
        "copies in flight at exit never completed",
        "a gather index outside the matrix (its y is NaN)",
        "a peer GPU's flag never arrived",
        "a chained round's dependency never completed",
        "an opened round's x never landed (rt_gemv_open without rt_gemv_go)",
    };
    size_t used = 0;
    out[0] = 0;
    for (unsigned b = 0; b < sizeof names / sizeof names[0] && used + 1 < n; ++b)
        if (h & (1u << b)) {
            const int k = snprintf(out + used, n - used, "%s%s", used ? "; " : "", names[b]);
            used = k < 0 ? n : used + size_t(k) < n ? used + size_t(k) : n - 1;
        }
}

// Waits for R's stream and reads the kernels' error word: its host mirror first (no copy), the
// bits only when it is set.
bool read_error_word(Ctx *c) {
    if (!cuda_ok(c, cudaStreamSynchronize(c->stream), "synchronize"))
        return false;
    c->synced = c->stream == c->own_stream;
    if (!*c->h_err)
        return true;
    unsigned h = 0;
    if (!cuda_ok(c, cudaMemcpy(&h, c->d_err, sizeof h, cudaMemcpyDeviceToHost), "read error word"))
        return false;
    *c->h_err = 0;
    if (h) {
        char what[200];
        error_word_text(h, what, sizeof what);
        ctx_err(c, RTB_EKERNEL, "kernel error word 0x%x: %s", h, what);
        cuda_ok(c, cudaMemsetAsync(c->d_err, 0, sizeof(unsigned), c->stream), "clear error word");
        c->synced = false;
        return false;
    }
    return true;
}

bool finish(Ctx *c) {
    if (c->async)
        return true;
    return flush_pending(c) && read_error_word(c); // a blocking call returns with y whole
}

// The output rows rank `rank` of `world` computes of a product with `rows` rows, and where they
// start: rows / world consecutive rows, rank-major (rows % world == 0, checked by the callers).
void split_rows(long long rows, int rank, int world, long long *lr, long long *r0) {
    *lr = rows / world;
    *r0 = (long long)rank * *lr;
}

void shard_rows(const Ctx *c, long long rows, long long *lr, long long *r0) { split_rows(rows, c->rank, c->world, lr, r0); }

// One CUDA-core launch per group of jobs with the same token count.
bool flush_gemv(Ctx *c, std::vector<q8::GemvJob> &jobs) {
    while (!jobs.empty()) {
        const int m = jobs[0].m;
        q8::GemvParams p;
        memset(&p, 0, sizeof p);
        p.err = c->d_err;
        p.early = c->overlap ? 1 : 0;
        std::vector<q8::GemvJob> rest;
        for (const q8::GemvJob &j : jobs) {
            if (j.m == m && p.njobs < q8::MAX_JOBS)
                p.job[p.njobs++] = j;
            else
                rest.push_back(j);
        }
        if (!cuda_ok(c, q8::launch_gemv(p, c->num_sms, 0, c->stream, c->overlap), "gemv launch"))
            return false;
        jobs.swap(rest);
    }
    return true;
}

bool ensure_scratch(Ctx *c, size_t bytes) {
    if (bytes <= c->scratch_bytes)
        return true;
    if (c->scratch && !cuda_ok(c, cudaStreamSynchronize(c->stream), "synchronize before scratch growth"))
        return false;
    cudaFree(c->scratch);
    c->scratch = nullptr;
    c->scratch_bytes = 0;
    if (!cuda_ok(c, cudaMalloc(&c->scratch, bytes), "scratch"))
        return false;
    c->scratch_bytes = bytes;
    return true;
}

// One tensor-core launch per 8 jobs (t >= TC_MIN_T), their x converted into the scratch.
bool flush_tc(Ctx *c, std::vector<q8::GemmJob> &jobs) {
    for (size_t i = 0; i < jobs.size(); i += 8) {
        const int n = int(jobs.size() - i < 8 ? jobs.size() - i : 8);
        const size_t need = q8::gemm_tc_scratch_bytes(&jobs[i], n, c->num_sms, true);
        if (!ensure_scratch(c, need))
            return false;
        if (!cuda_ok(c, q8::launch_gemm_tc(&jobs[i], n, c->scratch, c->scratch_bytes, c->num_sms, c->d_err, c->stream,
                                           c->overlap, true),
                     "tensor-core gemm launch"))
            return false;
    }
    jobs.clear();
    return true;
}

// One row-sharded product of <= 4 tokens on CUDA cores, its y gathered through the peers' staging
// images (the product's stores, then a batched gather kernel on the side stream), instead of an
// NCCL all-gather.
bool peer_gatherable(const Ctx *c, const std::vector<Item> &items) {
    if (c->world < 2 || !c->peer_ok || items.size() != 1)
        return false;
    const Item &it = items[0];
    return it.kind != K_ROWS && it.t <= q8::GEMV_MAX_T &&
           size_t(it.t) * size_t(it.rows) * sizeof(float) <= q8::PEER_STAGE_BYTES;
}

q8::PeerOut peer_out(const Ctx *c) {
    q8::PeerOut po;
    memset(&po, 0, sizeof po);
    for (int w = 0; w < c->world; ++w)
        po.region[w] = c->peer_map[w];
    po.rank = c->rank;
    po.world = c->world;
    return po;
}

// The capture R's stream is in (its id), or 0.
unsigned long long capture_id(cudaStream_t s) {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    unsigned long long id = 0;
    if (cudaStreamGetCaptureInfo(s, &st, &id) != cudaSuccess || st != cudaStreamCaptureStatusActive)
        return 0;
    return id;
}

// The open batch's gather, on the side stream after the batch's last product.
bool issue_batch(Ctx *c) {
    if (c->open_b.n == 0)
        return true;
    if (int(c->issued.size()) == Ctx::NSLOT) { // (every slot in use: the oldest batch first)
        const Ctx::Issued o = c->issued.front();
        if (o.cap == capture_id(c->stream) &&
            !cuda_ok(c, cudaStreamWaitEvent(c->stream, c->ev_gath[o.slot], 0), "wait for a gather"))
            return false;
        c->issued.erase(c->issued.begin());
        c->waited = o.last;
    }
    const int slot = c->next_slot;
    c->next_slot = (c->next_slot + 1) % Ctx::NSLOT;
    q8::PeerOut po = peer_out(c);
    po.on = 1;
    const q8::GatherBatch b = c->open_b;
    c->open_b.n = 0;
    if (!cuda_ok(c, cudaEventRecord(c->ev_prod[slot], c->stream), "gather: event") ||
        !cuda_ok(c, cudaStreamWaitEvent(c->gside, c->ev_prod[slot], 0), "gather: stream wait") ||
        !cuda_ok(c, q8::launch_peer_gather(po, b, c->d_err, c->gside), "peer gather") ||
        !cuda_ok(c, cudaEventRecord(c->ev_gath[slot], c->gside), "gather: event"))
        return false;
    c->issued.push_back({c->open_first + b.n - 1, capture_id(c->stream), slot});
    return true;
}

// R's stream waits until the rounds up to r are gathered (a batch's gather waits for the peers'
// reads of the whole batch, and the batches run in order). An event recorded in another capture
// context (or none, while capturing) cannot be waited on: work from before a capture must have
// been synchronised, as graphs need anyway.
bool wait_upto(Ctx *c, unsigned long long r) {
    if (r <= c->waited)
        return true;
    if (r >= c->open_first && c->open_b.n && !issue_batch(c)) // r not launched for gathering yet
        return false;
    const unsigned long long cap = capture_id(c->stream);
    while (!c->issued.empty() && c->waited < r) {
        const Ctx::Issued o = c->issued.front();
        c->issued.erase(c->issued.begin());
        if (o.last >= r && o.cap == cap &&
            !cuda_ok(c, cudaStreamWaitEvent(c->stream, c->ev_gath[o.slot], 0), "wait for a gather"))
            return false;
        c->waited = o.last;
    }
    std::vector<Ctx::PendingY> keep;
    for (const Ctx::PendingY &q : c->pending)
        if (q.round > c->waited)
            keep.push_back(q);
    c->pending.swap(keep);
    return true;
}

// R's stream waits for every round's gather: y is whole on R's stream from here on.
bool flush_pending(Ctx *c) {
    if (c->prounds <= c->waited)
        return true;
    return issue_batch(c) && wait_upto(c, c->prounds);
}

// One row-sharded product: the product kernel on R's stream (its rows into y and into the peers'
// staging), its round added to the open batch (gathered on the side stream once the batch is
// full, or when something needs it). A product whose x overlaps a y not yet gathered, or whose y
// overlaps one other than its own (the same buffer and shape: its own rows, which the gathers
// leave alone), waits for that gather first; so does one whose staging image was last used
// PEER_IMAGES rounds ago (the images' reuse, q8_kernels.h).
bool run_peer_gathered(Ctx *c, const Item &it) {
    long long lr, r0;
    shard_rows(c, it.rows, &lr, &r0);
    const size_t xb = size_t(it.t * it.cols) * 4, yb = size_t(it.t * it.rows) * 4;
    unsigned long long need = 0;
    for (const Ctx::PendingY &q : c->pending)
        if (overlaps(it.x, xb, q.y, q.bytes) || (overlaps(it.y, yb, q.y, q.bytes) && !(it.y == q.y && yb == q.bytes)))
            need = q.round > need ? q.round : need;
    const unsigned long long r = ++c->prounds;
    if (r > (unsigned long long)q8::PEER_IMAGES && r - q8::PEER_IMAGES > need)
        need = r - q8::PEER_IMAGES;
    if (need && !wait_upto(c, need))
        return false;
    q8::GemvParams p;
    memset(&p, 0, sizeof p);
    p.err = c->d_err;
    p.early = c->overlap ? 1 : 0;
    p.njobs = 1;
    q8::GemvJob &j = p.job[0];
    j.w = it.w;
    j.w2 = it.kind == K_SILU ? it.w2 : nullptr;
    j.x = it.x;
    j.ldx = it.cols;
    j.ldy = it.rows;
    j.y = it.y + r0;
    j.rows = lr;
    j.src_rows = lr;
    j.cols = int(it.cols);
    j.m = int(it.t);
    q8::PeerOut &po = p.peer;
    po = peer_out(c);
    po.row0 = r0;
    po.rows_total = it.rows;
    po.on = 1;
    if (!cuda_ok(c, q8::launch_gemv(p, c->num_sms, 0, c->stream, c->overlap), "gemv launch"))
        return false;
    if (c->open_b.n == 0)
        c->open_first = r;
    const int i = c->open_b.n++;
    c->open_b.y[i] = it.y;
    c->open_b.rows[i] = it.rows;
    c->open_b.t[i] = int(it.t);
    c->pending.push_back({it.y, yb, r});
    return c->open_b.n < q8::GATHER_BATCH || issue_batch(c);
}

// The CUDA-core job of tokens [k, k + 4) of a product (rows lr from r0 on this rank).
q8::GemvJob cuda_core_job(const Item &it, long long k, long long lr, long long r0) {
    q8::GemvJob j;
    memset(&j, 0, sizeof j);
    j.w = it.w;
    j.w2 = it.kind == K_SILU ? it.w2 : nullptr;
    j.idx = it.kind == K_ROWS ? it.idx : nullptr;
    j.x = it.x + k * it.cols;
    j.ldx = it.cols;
    j.ldy = it.rows;
    j.y = it.y + k * it.rows + r0;
    j.rows = lr;
    j.src_rows = it.kind == K_ROWS ? it.src_rows : lr;
    j.cols = int(it.cols);
    j.m = int(it.t - k < q8::GEMV_MAX_T ? it.t - k : q8::GEMV_MAX_T);
    return j;
}

// Splits the items into kernel jobs (t >= 16: one tensor-core job; else passes of <= 4 tokens on
// CUDA cores), launches them, then all-gathers the sharded outputs.
bool run_items(Ctx *c, const std::vector<Item> &items) {
    c->synced = false;
    if (peer_gatherable(c, items))
        return run_peer_gathered(c, items[0]);
    if (!flush_pending(c))
        return false;
    std::vector<q8::GemvJob> jobs;
    std::vector<q8::GemmJob> tc;
    for (const Item &it : items) {
        long long lr = it.rows, r0 = 0;
        if (it.kind != K_ROWS)
            shard_rows(c, it.rows, &lr, &r0);
        if (it.kind != K_ROWS && it.t >= TC_MIN_T) {
            q8::GemmJob g;
            memset(&g, 0, sizeof g);
            g.w = it.w;
            g.w2 = it.kind == K_SILU ? it.w2 : nullptr;
            g.x = it.x;
            g.ldx = it.cols;
            g.y = it.y + r0;
            g.ldy = it.rows;
            g.rows = lr;
            g.cols = int(it.cols);
            g.t = int(it.t);
            tc.push_back(g);
            continue;
        }
        for (long long k = 0; k < it.t; k += q8::GEMV_MAX_T)
            jobs.push_back(cuda_core_job(it, k, lr, r0));
    }
    if (!flush_gemv(c, jobs) || !flush_tc(c, tc))
        return false;
    if (c->world > 1) {
        if (nccl().GroupStart() != ncclSuccess) {
            ctx_err(c, RTB_ENCCL, "ncclGroupStart");
            return false;
        }
        for (const Item &it : items) {
            if (it.kind == K_ROWS)
                continue; // the gather list is not sharded
            long long lr, r0;
            shard_rows(c, it.rows, &lr, &r0);
            for (long long k = 0; k < it.t; ++k) {
                float *yt = it.y + k * it.rows;
                ncclResult_t e = nccl().AllGather(yt + r0, yt, size_t(lr), ncclFloat32, c->comm, c->stream);
                if (e != ncclSuccess) {
                    nccl().GroupEnd();
                    ctx_err(c, RTB_ENCCL, "ncclAllGather: %s", nccl().GetErrorString(e));
                    return false;
                }
            }
        }
        ncclResult_t e = nccl().GroupEnd();
        if (e != ncclSuccess) {
            ctx_err(c, RTB_ENCCL, "ncclGroupEnd: %s", nccl().GetErrorString(e));
            return false;
        }
    }
    return true;
}

bool run_now(Ctx *c, const Item &it) {
    std::vector<Item> one(1, it);
    if (c->chaining) {
        c->chain.push_back(one);
        return true;
    }
    return run_items(c, one) && finish(c);
}

// ---------------------------------------------------------------- direct pushes

// A round rt_gemv_go may hold back for a direct push: direct pushes on, async, one GPU, no chain,
// and one CUDA-core product of one pass (<= 4 tokens); never while the stream is being captured
// (a held launch could then miss the graph).
bool holdable(Ctx *c, const std::vector<Item> &items) {
    if (!c->direct || !c->async || c->chaining || c->world > 1 || items.size() != 1 || items[0].t > q8::GEMV_MAX_T)
        return false;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    return cudaStreamIsCapturing(c->stream, &cs) == cudaSuccess && cs == cudaStreamCaptureStatusNone;
}

bool launch_held(Ctx *c) {
    if (!c->held)
        return true;
    c->held = false;
    std::vector<Item> one(1, c->held_item);
    return run_items(c, one);
}

// The device's address of host memory the GPU can write (pinned and mapped), else null.
float *mapped(const void *host) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, host) != cudaSuccess) {
        cudaGetLastError(); // (an unregistered pointer: not an error of R's)
        return nullptr;
    }
    return a.type == cudaMemoryTypeHost ? static_cast<float *>(a.devicePointer) : nullptr;
}

// The held round, launched with the product's y also stored into host memory (the device address
// yh) and a host flag raised by its last CTA; returns once the flag is up (y is on the host) or the
// launch ended without it. The kernel runs as a CUDA graph, captured the first time this round
// (same product, same y) comes and launched as it is afterwards: an engine repeats its rounds
// every token, and the graph's launch skips the kernel's 2.4 KB of parameters. (The round's pull
// stays a copy of its own, issued at rt_b200_pull: as a node of the graph it measured 6.6 us a
// round against 2.5.) The host polls the flag and, now and then, whether the stream has finished:
// a kernel that faulted raises no flag, and the wait then ends through the stream's error.
int push_direct(Ctx *c, const Item &it, float *yh) {
    q8::GemvParams p;
    memset(&p, 0, sizeof p);
    p.err = c->d_err;
    p.njobs = 1;
    p.job[0] = cuda_core_job(it, 0, it.rows, 0);
    p.y_host = yh;
    p.host_flag = c->h_flag_dev;
    p.host_ctr = c->d_hctr;
    const std::string key(reinterpret_cast<const char *>(&p), sizeof p);
    c->synced = false;
    cudaGraphExec_t exec = nullptr;
    auto found = c->graphs.find(key);
    if (found != c->graphs.end()) {
        exec = found->second;
    } else {
        if (c->graphs.size() >= 4096) { // (a bound on what a changing engine could pile up)
            for (auto &g : c->graphs)
                cudaGraphExecDestroy(g.second);
            c->graphs.clear();
        }
        cudaGraph_t g = nullptr;
        bool ok = cuda_ok(c, cudaStreamBeginCapture(c->cap, cudaStreamCaptureModeThreadLocal), "capture a round");
        if (ok) {
            ok = cuda_ok(c, q8::launch_gemv(p, c->num_sms, 0, c->cap, false), "gemv launch");
            const cudaError_t e = cudaStreamEndCapture(c->cap, &g);
            ok = ok && cuda_ok(c, e, "capture a round");
        }
        ok = ok && cuda_ok(c, cudaGraphInstantiate(&exec, g, 0), "instantiate a round");
        if (g)
            cudaGraphDestroy(g);
        if (!ok)
            return c->status;
        c->graphs.emplace(key, exec);
    }
    if (!cuda_ok(c, cudaGraphLaunch(exec, c->stream), "launch a round"))
        return c->status;
    const unsigned seq = ++c->host_seq; // the kernel's count of direct rounds, one ahead now
    bool up = false;
    for (unsigned long i = 1;; ++i) {
        if (*c->h_flag == seq) {
            up = true;
            break;
        }
        if ((i & 4095) == 0) {
            const cudaError_t q = cudaStreamQuery(c->stream);
            if (q != cudaErrorNotReady) {
                up = *c->h_flag == seq;
                break;
            }
        }
#if defined(__x86_64__)
        __builtin_ia32_pause();
#endif
    }
    std::atomic_thread_fence(std::memory_order_acquire);
    if (*c->h_err || !up) { // a kernel reported (or the launch failed): synchronize and read why
        if (read_error_word(c) && !up)
            ctx_err(c, RTB_ECUDA, "rt_b200_push: the product ended without its completion flag");
    }
    return c->status;
}

// ---------------------------------------------------------------- chains

bool overlaps(const void *a, size_t na, const void *b, size_t nb) {
    const uintptr_t a0 = reinterpret_cast<uintptr_t>(a), b0 = reinterpret_cast<uintptr_t>(b);
    return a0 < b0 + nb && b0 < a0 + na;
}

// Whether the recorded rounds can run as chained launches: every product on CUDA cores with the
// same number of tokens (<= 4), one GPU, and no gather list written inside the chain.
bool chainable(const Ctx *c) {
    if (c->world > 1 || c->chain.empty())
        return false;
    const long long t = c->chain[0][0].t;
    for (size_t r = 0; r < c->chain.size(); ++r)
        for (const Item &it : c->chain[r]) {
            if (it.t != t || it.t > q8::GEMV_MAX_T)
                return false;
            if (it.idx)
                for (size_t q = 0; q < c->chain.size(); ++q)
                    for (const Item &o : c->chain[q])
                        if (overlaps(it.idx, size_t(it.rows) * 4, o.y, size_t(o.rows * o.t) * 4))
                            return false;
        }
    return true;
}

long long item_tiles(const Item &it) { return (it.rows + (it.kind == K_SILU ? 3 : 7)) / (it.kind == K_SILU ? 4 : 8); }

// Whether round b (later) must wait for round a (earlier): b reads what a writes (x over a's y),
// or b writes what a reads or writes (y over a's x or y).
bool round_conflict(const std::vector<Item> &a, const std::vector<Item> &b) {
    for (const Item &o : a)
        for (const Item &it : b) {
            const size_t xb = size_t(it.t * it.cols) * 4, yb = size_t(it.t * it.rows) * 4;
            const size_t oxb = size_t(o.t * o.cols) * 4, oyb = size_t(o.t * o.rows) * 4;
            if (overlaps(it.x, xb, o.y, oyb) || overlaps(it.y, yb, o.x, oxb) || overlaps(it.y, yb, o.y, oyb))
                return true;
        }
    return false;
}

// One chained launch per <= MAX_CHAIN_JOBS jobs. Round r's jobs count their tiles into d_round[r]
// and wait (before their first tile) for the earlier rounds of the same launch they conflict
// with (round_conflict), or with `serial` simply for the previous round. A round finished means
// its own waits were met, so a wait on round q also covers everything q waited on: the list keeps
// only the rounds not already covered that way. A round that would still need more than
// MAX_WAITS waits starts a new launch. Rounds in different launches are ordered by the stream.
bool run_chain(Ctx *c, bool serial) {
    using Bits = std::bitset<q8::MAX_CHAIN_JOBS>;
    c->synced = false;
    const size_t nr = c->chain.size();
    size_t r = 0;
    while (r < nr) {
        q8::ChainParams p;
        memset(&p, 0, sizeof p);
        p.err = c->d_err;
        const size_t r0 = r;
        std::vector<long long> round_tiles;
        std::vector<Bits> covered; // per round of this launch: the rounds its finish implies
        for (; r < nr && p.njobs + int(c->chain[r].size()) <= q8::MAX_CHAIN_JOBS; ++r) {
            const size_t lr = r - r0; // round index inside this launch
            std::vector<int> deps;     // latest first
            for (size_t q = lr; q-- > 0;)
                if (serial ? q + 1 == lr : round_conflict(c->chain[r0 + q], c->chain[r]))
                    deps.push_back(int(q));
            std::vector<int> waits;
            Bits cov;
            for (int q : deps) { // a later round's finish covers the earlier ones it waited on
                if (cov[size_t(q)])
                    continue;
                waits.push_back(q);
                cov |= covered[size_t(q)];
                cov.set(size_t(q));
            }
            if (waits.size() > size_t(q8::MAX_WAITS))
                break; // this round opens the next launch, after every round before it
            long long tiles = 0;
            for (const Item &it : c->chain[r])
                tiles += item_tiles(it);
            for (const Item &it : c->chain[r]) {
                q8::GemvJob &j = p.job[p.njobs++];
                j.w = it.w;
                j.w2 = it.kind == K_SILU ? it.w2 : nullptr;
                j.idx = it.kind == K_ROWS ? it.idx : nullptr;
                j.x = it.x;
                j.ldx = it.cols;
                j.ldy = it.rows;
                j.y = it.y;
                j.rows = it.rows;
                j.src_rows = it.kind == K_ROWS ? it.src_rows : it.rows;
                j.cols = int(it.cols);
                j.m = int(it.t);
                j.done_ctr = c->d_round + q8::ROUND_CTR_STRIDE * lr;
                j.nwait = int(waits.size());
                for (size_t k = 0; k < waits.size(); ++k) {
                    j.wait_ctr[k] = c->d_round + q8::ROUND_CTR_STRIDE * size_t(waits[k]);
                    j.wait_target[k] = unsigned(round_tiles[size_t(waits[k])]);
                }
                j.x_written = 0;
                for (size_t q = 0; q < r && !j.x_written; ++q) // any earlier round of the chain
                    for (const Item &o : c->chain[q])
                        if (overlaps(it.x, size_t(it.t * it.cols) * 4, o.y, size_t(o.t * o.rows) * 4))
                            j.x_written = 1;
            }
            round_tiles.push_back(tiles);
            covered.push_back(cov);
        }
        if (r == r0) {
            ctx_err(c, RTB_EINVAL, "chain: a round of more than %d products", q8::MAX_CHAIN_JOBS);
            return false;
        }
        if (!cuda_ok(c, cudaMemsetAsync(c->d_round, 0, sizeof(unsigned) * q8::ROUND_CTR_STRIDE * (r - r0), c->stream),
                     "round counters") ||
            !cuda_ok(c, q8::launch_gemv_chain(p, c->num_sms, c->stream), "chained launch"))
            return false;
    }
    return true;
}

bool enqueue(Ctx *c, const Item &it) {
    if (c->queue.size() >= size_t(2 * RT_BATCH)) {
        ctx_err(c, RTB_EQUEUE, "more than %d products queued before rt_gemv_go", 2 * RT_BATCH);
        return false;
    }
    c->queue.push_back(it);
    return true;
}

Item make_item(Kind k, const void *w, const void *w2, const int32_t *idx, long long rows, long long cols,
               const float *x, long long t, float *y) {
    Item it;
    it.kind = k;
    it.w = static_cast<const uint8_t *>(w);
    it.w2 = static_cast<const uint8_t *>(w2);
    it.idx = idx;
    it.x = x;
    it.y = y;
    it.rows = rows;
    it.cols = cols;
    it.t = t;
    it.src_rows = rows;
    return it;
}

// rt_gemv_open: launches the queued round's CUDA-core products now, gated: their weights stream in
// while the host still prepares x, and their compute waits on the device for the gate to reach this
// round's number. The link stream first waits for everything already on R's stream (the round's
// pulls must not overwrite an x an earlier product still reads). Tensor-core products (their
// pre-pass reads x at once), several GPUs, chains and stream capture (the gate value would be
// frozen into the graph) keep the plain round: open then does nothing and go runs everything.
void open_round(Ctx *c) {
    if (c->round_open || c->chaining || c->world > 1 || c->queue.empty() || !write_value32())
        return;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(c->stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone)
        return;
    std::vector<q8::GemvJob> jobs;
    std::vector<Item> rest;
    for (const Item &it : c->queue) {
        if (it.t >= TC_MIN_T) {
            rest.push_back(it);
            continue;
        }
        for (long long k = 0; k < it.t; k += q8::GEMV_MAX_T) {
            q8::GemvJob j;
            memset(&j, 0, sizeof j);
            j.w = it.w;
            j.w2 = it.kind == K_SILU ? it.w2 : nullptr;
            j.idx = it.kind == K_ROWS ? it.idx : nullptr;
            j.x = it.x + k * it.cols;
            j.ldx = it.cols;
            j.ldy = it.rows;
            j.y = it.y + k * it.rows;
            j.rows = it.rows;
            j.src_rows = it.kind == K_ROWS ? it.src_rows : it.rows;
            j.cols = int(it.cols);
            j.m = int(it.t - k < q8::GEMV_MAX_T ? it.t - k : q8::GEMV_MAX_T);
            j.x_written = 1; // x lands during the kernel: read it past L1
            jobs.push_back(j);
        }
    }
    if (jobs.empty())
        return;
    // The tensor-core products left for go get their scratch now: growing it at go would allocate
    // (and may synchronize) while the gated kernel holds the GPU waiting for go.
    if (!rest.empty()) {
        size_t need = 0;
        std::vector<q8::GemmJob> tc;
        for (const Item &it : rest) {
            q8::GemmJob g;
            memset(&g, 0, sizeof g);
            g.w = it.w;
            g.w2 = it.kind == K_SILU ? it.w2 : nullptr;
            g.x = it.x;
            g.ldx = it.cols;
            g.y = it.y;
            g.ldy = it.rows;
            g.rows = it.rows;
            g.cols = int(it.cols);
            g.t = int(it.t);
            tc.push_back(g);
        }
        for (size_t i = 0; i < tc.size(); i += 8) {
            const int n = int(tc.size() - i < 8 ? tc.size() - i : 8);
            const size_t b = q8::gemm_tc_scratch_bytes(&tc[i], n, c->num_sms, true);
            need = b > need ? b : need;
        }
        if (!ensure_scratch(c, need))
            return;
    }
    // (R's own stream, synchronized since its last work: nothing there can still read an x)
    if (!c->synced && (!cuda_ok(c, cudaEventRecord(c->ev_before, c->stream), "open: event") ||
                       !cuda_ok(c, cudaStreamWaitEvent(c->link, c->ev_before, 0), "open: link stream wait")))
        return;
    c->synced = false;
    const unsigned value = c->gate_seq + 1;
    while (!jobs.empty()) { // one gated launch per token count, as flush_gemv groups them
        const int m = jobs[0].m;
        q8::GemvParams p;
        memset(&p, 0, sizeof p);
        p.err = c->d_err;
        p.early = c->overlap ? 1 : 0;
        p.gate = c->d_gate;
        p.gate_value = value;
        std::vector<q8::GemvJob> later;
        for (const q8::GemvJob &j : jobs) {
            if (j.m == m && p.njobs < q8::MAX_JOBS)
                p.job[p.njobs++] = j;
            else
                later.push_back(j);
        }
        if (!cuda_ok(c, q8::launch_gemv(p, c->num_sms, 0, c->stream, c->overlap), "open: gated launch")) {
            // the kernels already launched wait for this value: release them now
            c->gate_seq = value;
            write_value32()(reinterpret_cast<CUstream>(c->link), reinterpret_cast<CUdeviceptr>(c->d_gate), value, 0);
            return;
        }
        jobs.swap(later);
    }
    c->gate_seq = value;
    c->queue.swap(rest);
    c->round_open = true;
}

// rt_gemv_go of an opened round: after the round's pulls on the link stream, the gate takes the
// round's number (the write is fenced after the copies); R's stream then also waits for the link
// stream, so whatever follows on it sees the pulled data.
bool release_gate(Ctx *c, bool more) {
    c->round_open = false;
    const CUresult r = write_value32()(reinterpret_cast<CUstream>(c->link), reinterpret_cast<CUdeviceptr>(c->d_gate),
                                       c->gate_seq, 0);
    if (r != CUDA_SUCCESS) {
        ctx_err(c, RTB_ECUDA, "rt_gemv_go: cuStreamWriteValue32 failed (%d)", int(r));
        return false;
    }
    // With nothing more to launch, what follows on R's stream comes after the gated kernel, which
    // read x only after the gate, itself written after the pulls: R needs no wait of its own.
    return !more || (cuda_ok(c, cudaEventRecord(c->ev_link, c->link), "go: event") &&
                     cuda_ok(c, cudaStreamWaitEvent(c->stream, c->ev_link, 0), "go: stream wait"));
}

} // namespace

namespace {

void drop_peers(Ctx *c) {
    if (c->gside) {
        cudaStreamSynchronize(c->gside);
        cudaStreamDestroy(c->gside);
        c->gside = nullptr;
        for (int i = 0; i < Ctx::NSLOT; ++i) {
            cudaEventDestroy(c->ev_prod[i]);
            cudaEventDestroy(c->ev_gath[i]);
            c->ev_prod[i] = c->ev_gath[i] = nullptr;
        }
    }
    c->pending.clear();
    c->issued.clear();
    c->open_b.n = 0;
    c->next_slot = 0;
    c->prounds = c->waited = 0;
    for (int w = 0; w < q8::MAX_PEERS; ++w) {
        if (c->peer_map[w] && c->peer_map[w] != c->peer_local)
            cudaIpcCloseMemHandle(c->peer_map[w]);
        c->peer_map[w] = nullptr;
    }
    cudaFree(c->peer_local);
    c->peer_local = nullptr;
    c->peer_ok = false;
}

// Maps every rank's peer region on this GPU: each rank allocates and zeroes its own, the CUDA IPC
// handles travel through one NCCL all-gather, and each rank opens the others'. Any failure leaves
// the fused gather off (rounds then all-gather through NCCL).
void setup_peers(Ctx *c) {
    drop_peers(c);
    if (c->world < 2 || c->world > q8::MAX_PEERS)
        return;
    if (cudaMalloc(&c->peer_local, q8::PEER_REGION_BYTES) != cudaSuccess) {
        c->peer_local = nullptr;
        return;
    }
    bool evs = cudaStreamCreateWithFlags(&c->gside, cudaStreamNonBlocking) == cudaSuccess;
    for (int i = 0; evs && i < Ctx::NSLOT; ++i)
        evs = cudaEventCreateWithFlags(&c->ev_prod[i], cudaEventDisableTiming) == cudaSuccess &&
              cudaEventCreateWithFlags(&c->ev_gath[i], cudaEventDisableTiming) == cudaSuccess;
    cudaIpcMemHandle_t mine;
    void *d_handles = nullptr;
    std::vector<cudaIpcMemHandle_t> all(size_t(c->world));
    bool ok = evs && cudaMemset(c->peer_local, 0, q8::PEER_HDR) == cudaSuccess &&
              cudaIpcGetMemHandle(&mine, c->peer_local) == cudaSuccess &&
              cudaMalloc(&d_handles, sizeof(cudaIpcMemHandle_t) * size_t(c->world)) == cudaSuccess;
    if (ok) {
        unsigned char *slot = static_cast<unsigned char *>(d_handles) + sizeof mine * size_t(c->rank);
        ok = cudaMemcpyAsync(slot, &mine, sizeof mine, cudaMemcpyHostToDevice, c->stream) == cudaSuccess &&
             nccl().AllGather(slot, d_handles, sizeof mine, ncclUint8, c->comm, c->stream) == ncclSuccess &&
             cudaMemcpyAsync(all.data(), d_handles, sizeof mine * size_t(c->world), cudaMemcpyDeviceToHost, c->stream) ==
                 cudaSuccess &&
             cudaStreamSynchronize(c->stream) == cudaSuccess;
    }
    cudaFree(d_handles);
    for (int w = 0; ok && w < c->world; ++w) {
        if (w == c->rank) {
            c->peer_map[w] = c->peer_local;
            continue;
        }
        void *p = nullptr;
        ok = cudaIpcOpenMemHandle(&p, all[size_t(w)], cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
        c->peer_map[w] = static_cast<unsigned char *>(p);
    }
    // every rank's region is zeroed and mapped before any rank's first product can write to it
    int flag = ok ? 1 : 0, *d_flag = nullptr;
    if (cudaMalloc(&d_flag, sizeof(int)) == cudaSuccess) {
        if (cudaMemcpyAsync(d_flag, &flag, sizeof flag, cudaMemcpyHostToDevice, c->stream) != cudaSuccess ||
            nccl().AllReduce(d_flag, d_flag, 1, ncclInt32, ncclMin, c->comm, c->stream) != ncclSuccess ||
            cudaMemcpyAsync(&flag, d_flag, sizeof flag, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess ||
            cudaStreamSynchronize(c->stream) != cudaSuccess)
            flag = 0;
        cudaFree(d_flag);
    } else {
        flag = 0;
    }
    cudaGetLastError(); // a failed IPC open is not the caller's error: the NCCL path stands in
    if (flag)
        c->peer_ok = true;
    else
        drop_peers(c);
}

} // namespace

extern "C" {

int rt_init(struct rt *R, int threads) {
    if (!R)
        return -1;
    Ctx *c = new (std::nothrow) Ctx();
    if (!c)
        return -1;
    if (cudaGetDevice(&c->device) != cudaSuccess ||
        cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, c->device) != cudaSuccess ||
        cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking) != cudaSuccess) {
        delete c;
        return -1;
    }
    c->stream = c->own_stream;
    // mapped host words: the error mirror at 0, the direct pushes' flag 128 bytes on
    unsigned *h_err = nullptr, *h_err_dev = nullptr;
    if (q8::preload_gemv() != cudaSuccess || q8::preload_gemm_tc() != cudaSuccess || q8::preload_peer() != cudaSuccess ||
        q8::preload_prims() != cudaSuccess ||
        cudaHostAlloc(&h_err, 256, cudaHostAllocMapped) != cudaSuccess ||
        cudaHostGetDevicePointer(&h_err_dev, h_err, 0) != cudaSuccess) {
        if (h_err)
            cudaFreeHost(h_err);
        cudaStreamDestroy(c->own_stream);
        delete c;
        return -1;
    }
    memset(h_err, 0, 256);
    c->h_err = h_err;
    c->h_flag = h_err + 32;
    c->h_flag_dev = h_err_dev + 32;
    if (cudaMalloc(&c->d_err, 16) != cudaSuccess || cudaMemset(c->d_err, 0, 16) != cudaSuccess ||
        cudaMemcpy(c->d_err + 2, &h_err_dev, sizeof h_err_dev, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMalloc(&c->d_round, sizeof(unsigned) * q8::ROUND_CTR_STRIDE * q8::MAX_CHAIN_JOBS) != cudaSuccess ||
        cudaMalloc(&c->d_gate, sizeof(unsigned)) != cudaSuccess || cudaMemset(c->d_gate, 0, sizeof(unsigned)) != cudaSuccess ||
        cudaMalloc(&c->d_hctr, 2 * sizeof(unsigned)) != cudaSuccess || cudaMemset(c->d_hctr, 0, 2 * sizeof(unsigned)) != cudaSuccess ||
        cudaStreamCreateWithFlags(&c->cap, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&c->link, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&c->ev_before, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&c->ev_link, cudaEventDisableTiming) != cudaSuccess) {
        // (the chains' round counters: allocated here, so a chain can be captured in a graph)
        cudaFree(c->d_err);
        cudaFree(c->d_round);
        cudaFree(c->d_gate);
        cudaFree(c->d_hctr);
        if (c->cap)
            cudaStreamDestroy(c->cap);
        if (c->link)
            cudaStreamDestroy(c->link);
        if (c->ev_before)
            cudaEventDestroy(c->ev_before);
        if (c->ev_link)
            cudaEventDestroy(c->ev_link);
        cudaFreeHost(h_err);
        cudaStreamDestroy(c->own_stream);
        delete c;
        return -1;
    }
    c->queue.reserve(2 * RT_BATCH);
    R->team = nullptr;
    R->chain = c;
    R->gemm_chain = nullptr;
    R->threads = threads;
    return 0;
}

void rt_b200_free(struct rt *R) {
    if (!R || !R->chain)
        return;
    Ctx *c = static_cast<Ctx *>(R->chain);
    launch_held(c);
    if (c->round_open) // release the pre-launched kernel: its results are not wanted
        release_gate(c, false);
    flush_pending(c);
    cudaStreamSynchronize(c->stream);
    cudaStreamSynchronize(c->link);
    drop_peers(c);
    if (c->comm)
        nccl().CommDestroy(c->comm);
    cudaFree(c->d_round);
    cudaFree(c->d_gate);
    cudaFree(c->d_hctr);
    for (auto &g : c->graphs)
        cudaGraphExecDestroy(g.second);
    c->graphs.clear();
    cudaStreamDestroy(c->cap);
    cudaFree(c->scratch);
    cudaFree(c->d_err);
    cudaEventDestroy(c->ev_before);
    cudaEventDestroy(c->ev_link);
    cudaStreamDestroy(c->link);
    cudaStreamDestroy(c->own_stream);
    cudaFreeHost(const_cast<unsigned *>(c->h_err));
    delete c;
    R->chain = nullptr;
}

void rt_gemv(struct rt *R, const void *w, long rows, long cols, const float *x, float *y) {
    Ctx *c = ctx_of(R);
    if (c && check_product(c, "rt_gemv", w, rows, cols, x, 1, y))
        run_now(c, make_item(K_GEMM, w, nullptr, nullptr, rows, cols, x, 1, y));
}

void rt_gemm(struct rt *R, const void *w, long rows, long cols, const float *x, long t, float *y) {
    Ctx *c = ctx_of(R);
    if (c && check_product(c, "rt_gemm", w, rows, cols, x, t, y))
        run_now(c, make_item(K_GEMM, w, nullptr, nullptr, rows, cols, x, t, y));
}

void rt_gemv_q(struct rt *R, const void *w, long rows, long cols, const float *x, float *y) {
    Ctx *c = ctx_of(R);
    if (c && check_product(c, "rt_gemv_q", w, rows, cols, x, 1, y))
        enqueue(c, make_item(K_GEMM, w, nullptr, nullptr, rows, cols, x, 1, y));
}

void rt_gemm_q(struct rt *R, const void *w, long rows, long cols, const float *x, long t, float *y) {
    Ctx *c = ctx_of(R);
    if (c && check_product(c, "rt_gemm_q", w, rows, cols, x, t, y))
        enqueue(c, make_item(K_GEMM, w, nullptr, nullptr, rows, cols, x, t, y));
}

void rt_gemv_open(struct rt *R) {
    Ctx *c = ctx_of(R);
    if (c)
        open_round(c);
}

void rt_gemv_go(struct rt *R) {
    Ctx *c = ctx_raw(R);
    if (!c)
        return;
    if (c->held) // a round held before goes first
        launch_held(c);
    std::vector<Item> items;
    items.swap(c->queue);
    bool ok = true;
    const bool was_open = c->round_open;
    if (c->round_open) {
        ok = release_gate(c, !items.empty());
    } else if (items.empty()) {
        return;
    }
    if (c->chaining) {
        if (!items.empty())
            c->chain.push_back(items);
        return;
    }
    if (ok && !items.empty() && !was_open && holdable(c, items)) {
        c->held = true; // launched by the next call on R: a direct push, or any other call
        c->held_item = items[0];
        return;
    }
    if (ok && (items.empty() || run_items(c, items)))
        finish(c);
}

void rt_gemm_silu_q(struct rt *R, const void *w_gate, const void *w_up, long rows, long cols, const float *x, long t,
                    float *h) {
    Ctx *c = ctx_of(R);
    if (!c)
        return;
    if (!w_up) {
        ctx_err(c, RTB_EINVAL, "rt_gemm_silu_q: null w_up");
        return;
    }
    if (!aligned(w_up, 16)) {
        ctx_err(c, RTB_EINVAL, "rt_gemm_silu_q: w_up must be 16-byte aligned");
        return;
    }
    if (check_product(c, "rt_gemm_silu_q", w_gate, rows, cols, x, t, h))
        enqueue(c, make_item(K_SILU, w_gate, w_up, nullptr, rows, cols, x, t, h));
}

void rt_gemm_silu(struct rt *R, const void *w_gate, const void *w_up, long rows, long cols, const float *x, long t,
                  float *h) {
    Ctx *c = ctx_of(R);
    if (!c)
        return;
    if (!w_up || !aligned(w_up, 16)) {
        ctx_err(c, RTB_EINVAL, "rt_gemm_silu: w_up null or not 16-byte aligned");
        return;
    }
    if (check_product(c, "rt_gemm_silu", w_gate, rows, cols, x, t, h))
        run_now(c, make_item(K_SILU, w_gate, w_up, nullptr, rows, cols, x, t, h));
}

static bool check_rows(Ctx *c, const char *fn, long w_rows, const int32_t *idx, long n) {
    if (!idx || n < 1 || w_rows < 1) {
        ctx_err(c, RTB_EINVAL, "%s: null idx, n < 1 or w_rows < 1", fn);
        return false;
    }
    if (!aligned(idx, 4)) {
        ctx_err(c, RTB_EINVAL, "%s: idx must be 4-byte aligned", fn);
        return false;
    }
    return true;
}

void rt_gemv_rows_q(struct rt *R, const void *w, long w_rows, const int32_t *idx, long n, long cols, const float *x,
                    float *y) {
    Ctx *c = ctx_of(R);
    if (!c || !check_rows(c, "rt_gemv_rows_q", w_rows, idx, n))
        return;
    const int world = c->world;
    c->world = 1; // a gather list is not sharded: check as a plain product
    const bool ok = check_product(c, "rt_gemv_rows_q", w, n, cols, x, 1, y);
    c->world = world;
    if (ok) {
        Item it = make_item(K_ROWS, w, nullptr, idx, n, cols, x, 1, y);
        it.src_rows = w_rows;
        enqueue(c, it);
    }
}

void rt_gemv_rows(struct rt *R, const void *w, long w_rows, const int32_t *idx, long n, long cols, const float *x,
                  float *y) {
    Ctx *c = ctx_of(R);
    if (!c || !check_rows(c, "rt_gemv_rows", w_rows, idx, n))
        return;
    const int world = c->world;
    c->world = 1;
    const bool ok = check_product(c, "rt_gemv_rows", w, n, cols, x, 1, y);
    c->world = world;
    if (ok) {
        Item it = make_item(K_ROWS, w, nullptr, idx, n, cols, x, 1, y);
        it.src_rows = w_rows;
        run_now(c, it);
    }
}

// ---------------------------------------------------------------- host-half primitives
// (src/host/rt_host.c:128-279; the kernels in host_prims.cu). On R's stream, device pointers;
// blocking unless async, as the products.

// The common checks; false (and R's error set) if the call cannot run.
static bool prim_ok(Ctx *c, const char *fn, bool ptrs, long h, long c_cols) {
    if (c->chaining) {
        ctx_err(c, RTB_EINVAL, "%s: not inside a chain (rt_b200_chain_begin .. end)", fn);
        return false;
    }
    if (!ptrs) {
        ctx_err(c, RTB_EINVAL, "%s: null or misaligned pointer (4 bytes; kv 16)", fn);
        return false;
    }
    if (h < 1 || h > q8::MAX_PRIM_HEADS) {
        ctx_err(c, RTB_EINVAL, "%s: h = %ld outside [1, %d]", fn, h, q8::MAX_PRIM_HEADS);
        return false;
    }
    if (c_cols < 8 || c_cols % 8) {
        ctx_err(c, RTB_EINVAL, "%s: c = %ld is not a positive multiple of 8", fn, c_cols);
        return false;
    }
    return flush_pending(c);
}

static bool heads_ok(Ctx *c, const char *fn, const long *l, long h, long n1) {
    if (!l || n1 < 1) {
        ctx_err(c, RTB_EINVAL, "%s: null l or n1 < 1", fn);
        return false;
    }
    for (long i = 0; i < h; ++i)
        if (l[i] < 0 || l[i] >= n1) {
            ctx_err(c, RTB_EINVAL, "%s: l[%ld] = %ld outside [0, n1 = %ld)", fn, i, l[i], n1);
            return false;
        }
    return true;
}

void rt_ip21(struct rt *R, float *z, const float *a, long h, long r, long c_cols, const float *b) {
    Ctx *c = ctx_of(R);
    if (!c || !prim_ok(c, "rt_ip21", z && b && (r == 0 || a) && aligned(z, 4) && aligned(a, 4) && aligned(b, 4), h, c_cols))
        return;
    if (r < 0) {
        ctx_err(c, RTB_EINVAL, "rt_ip21: r < 0");
        return;
    }
    c->synced = false;
    if (cuda_ok(c, q8::launch_ip21(z, a, h, r, c_cols, b, c->stream), "rt_ip21"))
        finish(c);
}

void rt_ip21_kv(struct rt *R, float *z, const float *kv, long n1, long c_cols, const long *l, long h, long t,
                const float *b) {
    Ctx *c = ctx_of(R);
    // (an empty history reads no kv: a null kv is then fine)
    const bool kv_ok = t == 0 || (kv && aligned(kv, 16));
    if (!c || !prim_ok(c, "rt_ip21_kv", z && b && kv_ok && aligned(z, 4) && aligned(b, 4), h, c_cols) ||
        !heads_ok(c, "rt_ip21_kv", l, h, n1))
        return;
    if (t < 0) {
        ctx_err(c, RTB_EINVAL, "rt_ip21_kv: t < 0");
        return;
    }
    q8::PrimHeads heads;
    memset(&heads, 0, sizeof heads);
    for (long i = 0; i < h; ++i) {
        heads.l[i] = l[i];
        heads.ord[i] = int(i);
    }
    // the heads that share a kv head side by side: their threads then read each row together
    std::stable_sort(heads.ord, heads.ord + h, [&](int x, int y) { return l[x] < l[y]; });
    c->synced = false;
    if (cuda_ok(c, q8::launch_ip21_kv(z, kv, n1, c_cols, heads, h, t, b, c->stream), "rt_ip21_kv"))
        finish(c);
}

void rt_ip12_kv(struct rt *R, float *z, const float *a, const float *kv, long n1, long c_cols, const long *l, long h,
                long t) {
    Ctx *c = ctx_of(R);
    const bool in_ok = t == 0 || (a && kv && aligned(a, 4) && aligned(kv, 16)); // (t = 0: z = 0, nothing read)
    if (!c || !prim_ok(c, "rt_ip12_kv", z && in_ok && aligned(z, 4), h, c_cols) ||
        !heads_ok(c, "rt_ip12_kv", l, h, n1))
        return;
    if (t < 0) {
        ctx_err(c, RTB_EINVAL, "rt_ip12_kv: t < 0");
        return;
    }
    // the query heads grouped by kv head (the groups share each streamed history slice), split
    // into groups of at most MAX_PRIM_GROUP
    q8::PrimGroups g;
    memset(&g, 0, sizeof g);
    std::vector<char> done(size_t(h), 0);
    int nh = 0;
    for (long i = 0; i < h; ++i) {
        if (done[size_t(i)])
            continue;
        g.first[g.n] = nh;
        g.kv[g.n] = l[i];
        for (long j = i; j < h; ++j)
            if (!done[size_t(j)] && l[j] == l[i]) {
                if (nh - g.first[g.n] == q8::MAX_PRIM_GROUP) { // a full group: the next one, same kv head
                    ++g.n;
                    g.first[g.n] = nh;
                    g.kv[g.n] = l[i];
                }
                g.head[nh++] = int(j);
                done[size_t(j)] = 1;
            }
        ++g.n;
    }
    g.first[g.n] = nh;
    c->synced = false;
    if (cuda_ok(c, q8::launch_ip12_kv(z, a, kv, n1, c_cols, g, t, c->d_err, c->stream), "rt_ip12_kv"))
        finish(c);
}

void rt_scale_outer(struct rt *R, float *z, const float *s, float g, const float *a, const float *b, long m, long k) {
    Ctx *c = ctx_of(R);
    if (!c)
        return;
    if (c->chaining) {
        ctx_err(c, RTB_EINVAL, "rt_scale_outer: not inside a chain (rt_b200_chain_begin .. end)");
        return;
    }
    if (!z || !s || !a || !b || !aligned(z, 4) || !aligned(s, 4) || !aligned(a, 4) || !aligned(b, 4) || m < 0 || k < 0) {
        ctx_err(c, RTB_EINVAL, "rt_scale_outer: null or misaligned pointer, or m, k < 0");
        return;
    }
    if (!flush_pending(c))
        return;
    if (m == 0 || k == 0)
        return;
    c->synced = false;
    if (cuda_ok(c, q8::launch_scale_outer(z, s, g, a, b, m, k, c->stream), "rt_scale_outer"))
        finish(c);
}

void rt_q8_row(const void *w, long cols, long row, float *z) {
    if (!w || !z || cols < Q8_QK || cols % Q8_QK || row < 0 || !aligned(w, 16)) {
        thread_err(RTB_EINVAL, "rt_q8_row: bad argument (cols %ld row %ld)", cols, row);
        return;
    }
    cudaError_t e = q8::launch_q8_row(static_cast<const uint8_t *>(w), int(cols), row, z, 0);
    if (e == cudaSuccess)
        e = cudaStreamSynchronize(0);
    if (e != cudaSuccess)
        thread_err(RTB_ECUDA, "rt_q8_row: %s", cudaGetErrorString(e));
}

long gemv_s_bytes(long rows, long cols) {
    if (rows < 0 || cols < 0 || cols % Q8_QK)
        return -1;
    return long(q8s_bytes(rows, cols));
}

int gemv_s_repack(const void *q8, long rows, long cols, void *out) {
    if (!q8 || !out || rows < 1 || cols < Q8_QK || cols % Q8_QK) {
        thread_err(RTB_EINVAL, "gemv_s_repack: bad argument");
        return RTB_EINVAL;
    }
    if (q8_gguf_row_bytes(cols) > q8::REPACK_MAX_ROW_BYTES) {
        thread_err(RTB_EINVAL, "gemv_s_repack: cols %ld above the repack's %lld", cols,
                   q8::REPACK_MAX_ROW_BYTES / Q8_GGUF_BLOCK * Q8_QK);
        return RTB_EINVAL;
    }
    if (q8 == out && q8s_row_bytes(cols) != q8_gguf_row_bytes(cols)) {
        thread_err(RTB_EINVAL, "gemv_s_repack: in place needs cols %% 256 == 0");
        return RTB_EINVAL;
    }
    if (q8 != out) { // the two must not overlap
        const uintptr_t a = reinterpret_cast<uintptr_t>(q8), b = reinterpret_cast<uintptr_t>(out);
        const uintptr_t an = uintptr_t(rows * q8_gguf_row_bytes(cols)), bn = uintptr_t(q8s_bytes(rows, cols));
        if (a < b + bn && b < a + an) {
            thread_err(RTB_EINVAL, "gemv_s_repack: input and output overlap (not in place)");
            return RTB_EINVAL;
        }
    }
    if (!aligned(out, 16)) {
        thread_err(RTB_EINVAL, "gemv_s_repack: out must be 16-byte aligned");
        return RTB_EINVAL;
    }
    cudaError_t e = q8::launch_repack(static_cast<const uint8_t *>(q8), rows, int(cols), static_cast<uint8_t *>(out), 0);
    if (e == cudaSuccess)
        e = cudaStreamSynchronize(0);
    if (e != cudaSuccess) {
        thread_err(RTB_ECUDA, "gemv_s_repack: %s", cudaGetErrorString(e));
        return RTB_ECUDA;
    }
    return RTB_OK;
}

long gemv_i_bytes(long rows, long cols) { return gemv_s_bytes(rows, cols); }

void gemv_i_repack(const uint8_t *q8, long rows, long cols, void *out) { (void)gemv_s_repack(q8, rows, cols, out); }

void gemv_i_repack_thread(void *arg, int tid, int n) {
    (void)n;
    if (tid != 0)
        return;
    const gemv_repack_job *j = static_cast<const gemv_repack_job *>(arg);
    if (!j) {
        thread_err(RTB_EINVAL, "gemv_i_repack_thread: null job");
        return;
    }
    (void)gemv_s_repack(j->w, j->rows, j->cols, j->w);
}

int rt_b200_last_error(struct rt *R, char *msg, size_t n) {
    int *status = &t_status;
    char *m = t_msg;
    if (R && R->chain) {
        Ctx *c = static_cast<Ctx *>(R->chain);
        status = &c->status;
        m = c->msg;
    }
    const int s = *status;
    if (msg && n) {
        strncpy(msg, s ? m : "", n - 1);
        msg[n - 1] = 0;
    }
    *status = RTB_OK;
    m[0] = 0;
    return s;
}

void rt_b200_set_overlap(struct rt *R, int on) {
    Ctx *c = ctx_of(R);
    if (c)
        c->overlap = on != 0;
}

void rt_b200_set_async(struct rt *R, int on) {
    Ctx *c = ctx_of(R);
    if (c)
        c->async = on != 0;
}

int rt_b200_sync(struct rt *R) {
    Ctx *c = ctx_of(R);
    if (!c)
        return RTB_ENOTINIT;
    // An open round whose go never came: its kernel gives up on the gate (about a second) and
    // reports it through the error word; the round is closed either way.
    c->round_open = false;
    flush_pending(c);
    read_error_word(c);
    cuda_ok(c, cudaStreamSynchronize(c->link), "synchronize the link stream");
    return c->status;
}

int rt_b200_pull(struct rt *R, void *dev, const void *host, size_t bytes) {
    Ctx *c = ctx_of(R);
    if (!c)
        return RTB_ENOTINIT;
    if ((!dev || !host) && bytes) {
        ctx_err(c, RTB_EINVAL, "rt_b200_pull: null pointer");
        return RTB_EINVAL;
    }
    // while a round is open its kernel is already on R's stream, waiting for this x: the copy goes
    // on the link stream, which rt_gemv_go then orders before the gate's release
    if (!c->round_open && !flush_pending(c)) // (a pending gather must not land on what this copies)
        return c->status;
    cudaStream_t s = c->round_open ? c->link : c->stream;
    if (!c->round_open)
        c->synced = false;
    if (bytes && !cuda_ok(c, cudaMemcpyAsync(dev, host, bytes, cudaMemcpyHostToDevice, s), "rt_b200_pull"))
        return c->status;
    return RTB_OK;
}

int rt_b200_push(struct rt *R, void *host, const void *dev, size_t bytes) {
    Ctx *c = ctx_raw(R);
    if (!c)
        return RTB_ENOTINIT;
    if ((!dev || !host) && bytes) {
        launch_held(c);
        ctx_err(c, RTB_EINVAL, "rt_b200_push: null pointer");
        return RTB_EINVAL;
    }
    if (c->held) {
        // the held round's y, whole, into host memory the GPU can write: the product stores it
        // there itself and raises the host flag; anything else launches the round as usual
        const Item it = c->held_item;
        c->held = false;
        float *yh = nullptr;
        if (dev == it.y && bytes == size_t(it.t * it.rows) * sizeof(float) && aligned(host, 4) &&
            (yh = mapped(host)) != nullptr)
            return push_direct(c, it, yh);
        std::vector<Item> one(1, it);
        if (!run_items(c, one))
            return c->status;
    }
    if (!flush_pending(c)) // y whole before it crosses
        return c->status;
    if (bytes && !cuda_ok(c, cudaMemcpyAsync(host, dev, bytes, cudaMemcpyDeviceToHost, c->stream), "rt_b200_push"))
        return c->status;
    read_error_word(c); // waits for the stream: the bytes have landed, kernel errors surface here
    return c->status;
}

void *rt_b200_stream(struct rt *R) {
    Ctx *c = ctx_of(R);
    return c ? static_cast<void *>(c->stream) : nullptr;
}

void rt_b200_set_stream(struct rt *R, void *stream) {
    Ctx *c = ctx_of(R);
    if (c) {
        flush_pending(c); // on the stream it was left on
        c->stream = stream ? static_cast<cudaStream_t>(stream) : c->own_stream;
        c->synced = false;
    }
}

void rt_b200_set_push_direct(struct rt *R, int on) {
    Ctx *c = ctx_of(R);
    if (c)
        c->direct = on != 0;
}

int rt_b200_flush(struct rt *R) {
    Ctx *c = ctx_of(R);
    if (!c)
        return RTB_ENOTINIT;
    flush_pending(c);
    return c->status;
}

int rt_b200_nccl_id(void *out128) {
    if (!out128)
        return RTB_EINVAL;
    ncclUniqueId id;
    if (!nccl().ok || nccl().GetUniqueId(&id) != ncclSuccess)
        return RTB_ENCCL;
    static_assert(sizeof(id) == 128, "ncclUniqueId is 128 bytes");
    memcpy(out128, &id, sizeof id);
    return RTB_OK;
}

int rt_b200_shard(struct rt *R, int rank, int world, const void *nccl_id) {
    Ctx *c = ctx_of(R);
    if (!c)
        return RTB_ENOTINIT;
    if (world < 1 || rank < 0 || rank >= world || (world > 1 && !nccl_id)) {
        ctx_err(c, RTB_EINVAL, "rt_b200_shard: rank %d world %d", rank, world);
        return RTB_EINVAL;
    }
    flush_pending(c);
    cudaStreamSynchronize(c->stream);
    drop_peers(c);
    if (c->comm) {
        nccl().CommDestroy(c->comm);
        c->comm = nullptr;
    }
    c->rank = rank;
    c->world = world;
    if (world == 1)
        return RTB_OK;
    if (!nccl().ok) {
        c->world = 1;
        c->rank = 0;
        ctx_err(c, RTB_ENCCL, "rt_b200_shard: libnccl.so.2 not found");
        return RTB_ENCCL;
    }
    ncclUniqueId id;
    memcpy(&id, nccl_id, sizeof id);
    ncclResult_t e = nccl().CommInitRank(&c->comm, world, id, rank);
    if (e != ncclSuccess) {
        c->comm = nullptr;
        c->world = 1;
        c->rank = 0;
        ctx_err(c, RTB_ENCCL, "ncclCommInitRank: %s", nccl().GetErrorString(e));
        return RTB_ENCCL;
    }
    if (!getenv("RTB_NO_PEER_GATHER"))
        setup_peers(c);
    return RTB_OK;
}

int rt_b200_chain_begin(struct rt *R) {
    Ctx *c = ctx_of(R);
    if (!c)
        return RTB_ENOTINIT;
    if (c->chaining || !c->queue.empty()) {
        ctx_err(c, RTB_EINVAL, "rt_b200_chain_begin: a chain or a queued round is open");
        return RTB_EINVAL;
    }
    c->chaining = true;
    c->chain.clear();
    return RTB_OK;
}

int rt_b200_chain_end(struct rt *R, int serial) {
    Ctx *c = ctx_of(R);
    if (!c)
        return RTB_ENOTINIT;
    if (!c->chaining) {
        ctx_err(c, RTB_EINVAL, "rt_b200_chain_end without rt_b200_chain_begin");
        return RTB_EINVAL;
    }
    c->chaining = false;
    std::vector<std::vector<Item>> rounds;
    rounds.swap(c->chain);
    if (rounds.empty())
        return RTB_OK;
    bool ok;
    c->chain.swap(rounds);
    if (chainable(c)) {
        ok = run_chain(c, serial != 0);
        c->chain.clear();
    } else { // not chainable: the rounds run one launch (and gather) each, in order
        rounds.swap(c->chain);
        ok = true;
        for (size_t r = 0; ok && r < rounds.size(); ++r)
            ok = run_items(c, rounds[r]);
    }
    if (ok)
        ok = finish(c);
    return ok ? RTB_OK : (c->status != RTB_OK ? c->status : RTB_ECUDA);
}

int rt_b200_wait_probe(struct rt *R) {
    Ctx *c = ctx_of(R);
    if (!c)
        return RTB_ENOTINIT;
    unsigned *ctr = nullptr; // a counter that nothing advances
    if (!cuda_ok(c, cudaMalloc(&ctr, sizeof(unsigned)), "wait probe"))
        return c->status;
    if (cuda_ok(c, cudaMemsetAsync(ctr, 0, sizeof(unsigned), c->stream), "wait probe") &&
        cuda_ok(c, q8::launch_wait_probe(ctr, c->d_err, c->stream), "wait probe launch"))
        read_error_word(c); // waits for the kernel: RTB_EKERNEL with the two waits' bits
    cudaStreamSynchronize(c->stream);
    cudaFree(ctr);
    return c->status;
}

int rt_b200_shard_rows(long rows, int rank, int world, long *row0, long *n) {
    if (!row0 || !n || world < 1 || rank < 0 || rank >= world || rows < 1 || rows % world) {
        thread_err(RTB_EINVAL, "rt_b200_shard_rows: rows %ld rank %d world %d", rows, rank, world);
        return RTB_EINVAL;
    }
    long long lr, r0;
    split_rows(rows, rank, world, &lr, &r0);
    *row0 = long(r0);
    *n = long(lr);
    return RTB_OK;
}

int rt_b200_peer_gather(struct rt *R) {
    Ctx *c = ctx_of(R);
    return c && c->peer_ok ? 1 : 0;
}

int rtb_synth_q8_0(void *dst, long row0, long rows, long cols, uint64_t seed, uint64_t stream, float sigma) {
    if (!dst || rows < 1 || row0 < 0 || cols < Q8_QK || cols % Q8_QK || !aligned(dst, 16))
        return RTB_EINVAL;
    cudaError_t e = q8::launch_synth_q8(static_cast<uint8_t *>(dst), row0, rows, int(cols), seed, stream, sigma, 0);
    if (e == cudaSuccess)
        e = cudaStreamSynchronize(0);
    return e == cudaSuccess ? RTB_OK : RTB_ECUDA;
}

int rtb_synth_f32(float *dst, long n, uint64_t seed, uint64_t stream, float sigma) {
    if (!dst || n < 1)
        return RTB_EINVAL;
    cudaError_t e = q8::launch_synth_f32(dst, n, seed, stream, sigma, 0);
    if (e == cudaSuccess)
        e = cudaStreamSynchronize(0);
    return e == cudaSuccess ? RTB_OK : RTB_ECUDA;
}

} // extern "C"
