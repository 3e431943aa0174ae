// gguf_load.cu: the weight loader. A GGUF file goes from disk into HBM and its Q8_0 matrices into
// the row-split layout, as the reference engine brings a model onto the card:
//   - the file is read in page-aligned slots with O_DIRECT (src/card/stream.c:77-104 reads its
//     O_DIRECT slots the same way), here by four reader threads into pinned host buffers, each
//     slot's host-to-device copy overlapping the next read (buffered reads where the file system
//     refuses O_DIRECT);
//   - the file's position-weighted sum, sum of word_i * (2i + 1) mod 2^64 over its 8-byte words
//     (src/bench/arena.h:26-44, printed by src/card/engine.c:280-285), is computed on the GPU over
//     the device image: exact, whatever the split;
//   - every Q8_0 matrix is repacked in place on the GPU, once per distinct offset (a tied output
//     shares the embedding's), as src/card/engine.c:303-316 repacks on its team.
// The GGUF header is parsed on the host (the fields src/host/gguf_reader.c:166-218 reads: keys,
// the general.alignment key, tensor names, dims, types and offsets).
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/rt_b200.h"
#include "q8_kernels.h"
#include "q8_layout.h"

namespace {

// ---------------------------------------------------------------- GGUF header
enum : uint32_t { GT_F32 = 0, GT_F16 = 1, GT_Q8_0 = 8, GT_BF16 = 30 };

// bytes per block and elements per block of the tensor types this loader sizes
bool type_size(uint32_t type, uint64_t *bytes, uint64_t *elems) {
    switch (type) {
    case GT_F32: *bytes = 4; *elems = 1; return true;
    case GT_F16: *bytes = 2; *elems = 1; return true;
    case GT_BF16: *bytes = 2; *elems = 1; return true;
    case GT_Q8_0: *bytes = Q8_GGUF_BLOCK; *elems = Q8_QK; return true;
    default: return false;
    }
}

struct Reader {
    FILE *f = nullptr;
    std::string err;
    bool ok = true;
    bool get(void *p, size_t n) {
        if (ok && fread(p, 1, n, f) != n) {
            ok = false;
            err = "truncated header";
        }
        return ok;
    }
    uint32_t u32() {
        uint32_t v = 0;
        get(&v, 4);
        return v;
    }
    uint64_t u64() {
        uint64_t v = 0;
        get(&v, 8);
        return v;
    }
    std::string str() {
        const uint64_t n = u64();
        if (!ok || n > (1u << 20)) {
            ok = false;
            err = "bad string length";
            return {};
        }
        std::string s(size_t(n), '\0');
        get(&s[0], size_t(n));
        return s;
    }
    bool skip(uint64_t n) {
        if (ok && fseeko(f, off_t(n), SEEK_CUR) != 0) {
            ok = false;
            err = "truncated header";
        }
        return ok;
    }
};

// GGUF metadata value types and their fixed sizes (0 for strings and arrays)
uint64_t scalar_bytes(uint32_t vt) {
    switch (vt) {
    case 0: case 1: case 7: return 1;  // u8, i8, bool
    case 2: case 3: return 2;          // u16, i16
    case 4: case 5: case 6: return 4;  // u32, i32, f32
    case 10: case 11: case 12: return 8; // u64, i64, f64
    default: return 0;
    }
}

// Reads one metadata value; returns its integer value for integer types (alignment).
bool read_value(Reader &r, uint32_t vt, uint64_t *ival, int depth = 0) {
    *ival = 0;
    if (vt == 8) { // string
        r.str();
        return r.ok;
    }
    if (vt == 9) { // array: element type, count, elements
        const uint32_t et = r.u32();
        const uint64_t n = r.u64();
        if (depth > 2 || n > (1ull << 32)) {
            r.ok = false;
            r.err = "bad array";
            return false;
        }
        const uint64_t eb = scalar_bytes(et);
        if (eb)
            return r.skip(eb * n);
        for (uint64_t i = 0; i < n && r.ok; ++i) {
            uint64_t dummy;
            read_value(r, et, &dummy, depth + 1);
        }
        return r.ok;
    }
    const uint64_t b = scalar_bytes(vt);
    if (!b) {
        r.ok = false;
        r.err = "unknown metadata type";
        return false;
    }
    uint64_t v = 0;
    r.get(&v, size_t(b));
    *ival = v;
    return r.ok;
}

struct Table {
    std::vector<rtb_tensor> t;
    uint64_t file_bytes = 0, data_start = 0;
    std::string err;
};

bool parse(const char *path, Table *tab) {
    Reader r;
    r.f = fopen(path, "rb");
    if (!r.f) {
        tab->err = std::string(path) + ": " + strerror(errno);
        return false;
    }
    struct stat st;
    if (fstat(fileno(r.f), &st) != 0 || st.st_size < 0) {
        tab->err = std::string(path) + ": " + strerror(errno);
        fclose(r.f);
        return false;
    }
    tab->file_bytes = uint64_t(st.st_size);
    char magic[4] = {0};
    r.get(magic, 4);
    if (r.ok && memcmp(magic, "GGUF", 4) != 0) {
        r.ok = false;
        r.err = "not a GGUF file";
    }
    const uint32_t version = r.u32();
    if (r.ok && (version < 2 || version > 3)) {
        r.ok = false;
        r.err = "GGUF version " + std::to_string(version) + " (2 or 3 supported)";
    }
    const uint64_t n_tensors = r.u64(), n_kv = r.u64();
    if (r.ok && (n_tensors > (1u << 20) || n_kv > (1u << 20))) {
        r.ok = false;
        r.err = "implausible header counts";
    }
    uint64_t alignment = 32;
    for (uint64_t i = 0; i < n_kv && r.ok; ++i) {
        const std::string key = r.str();
        const uint32_t vt = r.u32();
        uint64_t v = 0;
        read_value(r, vt, &v);
        if (r.ok && key == "general.alignment") {
            if (v == 0 || (v & (v - 1)) || v > (1u << 20)) { // GGUF: a power of two
                r.ok = false;
                r.err = "general.alignment " + std::to_string(v) + " is not a power of two <= 1 MiB";
                break;
            }
            alignment = v;
        }
    }
    for (uint64_t i = 0; i < n_tensors && r.ok; ++i) {
        rtb_tensor t;
        memset(&t, 0, sizeof t);
        const std::string name = r.str();
        snprintf(t.name, sizeof t.name, "%s", name.c_str());
        t.n_dims = int(r.u32());
        if (r.ok && (t.n_dims < 1 || t.n_dims > 4)) {
            r.ok = false;
            r.err = "tensor " + name + ": dims";
            break;
        }
        // every size below stays far from 2^63, so no later sum or product of them wraps
        uint64_t ne = 1;
        bool dims_ok = true;
        for (int d = 0; d < t.n_dims; ++d) {
            const uint64_t v = r.u64();
            t.dim[d] = (long long)v;
            dims_ok = dims_ok && v <= (1ull << 40) && !__builtin_mul_overflow(ne, v, &ne) && ne <= (1ull << 50);
        }
        if (r.ok && !dims_ok) {
            r.ok = false;
            r.err = "tensor " + name + ": implausible dims";
            break;
        }
        t.type = int(r.u32());
        t.offset = r.u64();
        uint64_t bb = 0, be = 1;
        if (r.ok && !type_size(uint32_t(t.type), &bb, &be)) {
            r.ok = false;
            r.err = "tensor " + name + ": unsupported type " + std::to_string(t.type);
            break;
        }
        if (r.ok && (ne % be || uint64_t(t.dim[0]) % be)) { // GGUF: every row is whole blocks
            r.ok = false;
            r.err = "tensor " + name + ": rows not a whole number of blocks";
            break;
        }
        t.bytes = ne / be * bb;
        tab->t.push_back(t);
    }
    const uint64_t header_end = r.ok ? uint64_t(ftello(r.f)) : 0;
    fclose(r.f);
    if (!r.ok) {
        tab->err = std::string(path) + ": " + r.err;
        return false;
    }
    tab->data_start = (header_end + alignment - 1) / alignment * alignment;
    const uint64_t fb = tab->file_bytes; // < 2^63 (an off_t), so data_start + offset below cannot wrap
    for (rtb_tensor &t : tab->t) {
        if (t.offset > fb || t.bytes > fb || tab->data_start > fb || tab->data_start + t.offset > fb - t.bytes) {
            tab->err = std::string(path) + ": tensor " + t.name + " runs past the end of the file";
            return false;
        }
        t.offset += tab->data_start;
    }
    return true;
}

// ---------------------------------------------------------------- the file's sum
__global__ void file_sum_kernel(const unsigned long long *w, long long words, unsigned long long *out) {
    unsigned long long s = 0;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < words; i += (long long)gridDim.x * blockDim.x)
        s += w[i] * (2ull * (unsigned long long)i + 1ull); // mod 2^64
    for (int o = 16; o; o >>= 1)
        s += __shfl_down_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0)
        atomicAdd(out, s);
}

thread_local char t_load_msg[256];

// Whether the load repacks tensor t in place (a Q8_0 matrix whose rows keep their length:
// cols % 256 == 0, rows narrow enough for the repack's staging, 16-byte aligned), and its shape.
bool repackable(const rtb_tensor &t, long long *rows_out, long long *cols_out) {
    if (t.type != GT_Q8_0 || t.n_dims < 2)
        return false;
    const long long cols = t.dim[0];
    long long rows = 1;
    for (int d = 1; d < t.n_dims; ++d)
        rows *= t.dim[d];
    if (rows < 1 || q8_gguf_row_bytes(cols) > q8::REPACK_MAX_ROW_BYTES || q8s_row_bytes(cols) != q8_gguf_row_bytes(cols) ||
        t.offset % 16)
        return false; // empty, wider than the repack stages, or a row would change length: left in GGUF layout
    *rows_out = rows;
    *cols_out = cols;
    return true;
}

// An in-place repack rewrites its tensor's bytes, so no other tensor may share any of them,
// except a tied copy of the same matrix (same offset, type and dims: repacked once, both marked
// repacked). A table with any other overlap (a crafted or mis-tied file) is refused before
// anything is read.
bool check_repack_overlaps(const Table &tab, std::string *why) {
    for (size_t i = 0; i < tab.t.size(); ++i) {
        const rtb_tensor &a = tab.t[i];
        long long rows, cols;
        if (!repackable(a, &rows, &cols))
            continue;
        for (size_t j = 0; j < tab.t.size(); ++j) {
            const rtb_tensor &b = tab.t[j];
            if (j == i || b.bytes == 0 || !(a.offset < b.offset + b.bytes && b.offset < a.offset + a.bytes))
                continue;
            bool tie = a.offset == b.offset && a.type == b.type && a.n_dims == b.n_dims && a.bytes == b.bytes;
            for (int d = 0; tie && d < a.n_dims; ++d)
                tie = a.dim[d] == b.dim[d];
            if (!tie) {
                *why = std::string("tensors ") + a.name + " and " + b.name +
                       " share bytes but are not the same matrix (the in-place repack would corrupt one)";
                return false;
            }
        }
    }
    return true;
}

int fail(int code, const std::string &msg) {
    snprintf(t_load_msg, sizeof t_load_msg, "%s", msg.c_str());
    return code;
}

} // namespace

extern "C" {

RTB_API int rtb_gguf_info(const char *path, rtb_tensor *out, int cap, int *n, unsigned long long *file_bytes) {
    if (!path || !n)
        return fail(RTB_EINVAL, "rtb_gguf_info: null argument");
    Table tab;
    if (!parse(path, &tab))
        return fail(RTB_EINVAL, tab.err);
    *n = int(tab.t.size());
    if (file_bytes)
        *file_bytes = tab.file_bytes;
    for (int i = 0; out && i < cap && i < *n; ++i)
        out[i] = tab.t[size_t(i)];
    return RTB_OK;
}

RTB_API const char *rtb_load_error(void) { return t_load_msg; }

RTB_API int rt_b200_load_gguf(struct rt *R, const char *path, void *arena, unsigned long long arena_bytes,
                              rtb_tensor *out, int cap, int *n, rtb_load_stats *stats) {
    (void)R; // the load runs on a stream of its own; R is the engine it is for
    if (!path || !arena || !n)
        return fail(RTB_EINVAL, "rt_b200_load_gguf: null argument");
    if (reinterpret_cast<uintptr_t>(arena) % 256)
        return fail(RTB_EINVAL, "rt_b200_load_gguf: the arena must be 256-byte aligned");
    Table tab;
    if (!parse(path, &tab))
        return fail(RTB_EINVAL, tab.err);
    const uint64_t fb = tab.file_bytes;
    if (arena_bytes < (fb + 7) / 8 * 8)
        return fail(RTB_EINVAL, "rt_b200_load_gguf: arena smaller than the file");
    {
        std::string why;
        if (!check_repack_overlaps(tab, &why))
            return fail(RTB_EINVAL, "rt_b200_load_gguf: " + why);
    }
    if (out && cap < int(tab.t.size()))
        return fail(RTB_EINVAL, "rt_b200_load_gguf: tensor table too small");

    const auto t0 = std::chrono::steady_clock::now();
    bool direct = true;
    int fd = open(path, O_RDONLY | O_DIRECT);
    if (fd < 0) { // e.g. tmpfs: buffered reads
        direct = false;
        fd = open(path, O_RDONLY);
    }
    if (fd < 0)
        return fail(RTB_EINVAL, std::string(path) + ": " + strerror(errno));

    // Reader threads: thread k reads slots k, k+T, ... into its own pinned buffers and copies
    // each to the GPU on its own stream, the copy of one slot overlapping the read of the next;
    // several threads keep several reads in flight on the device.
    constexpr size_t CHUNK = size_t(32) << 20, PAGE = 4096;
    constexpr int T = 4, NBUF = 2;
    cudaStream_t s = nullptr;
    cudaStream_t ts[T] = {};
    void *buf[T][NBUF] = {};
    cudaEvent_t ev[T][NBUF] = {}, tdone[T] = {}, e_read = nullptr, e_done = nullptr;
    unsigned long long *d_sum = nullptr;
    int rc = RTB_OK;
    std::mutex mu;
    auto cuda = [&](cudaError_t e, const char *what) {
        if (e != cudaSuccess) {
            std::lock_guard<std::mutex> lock(mu);
            if (rc == RTB_OK)
                rc = fail(RTB_ECUDA, std::string("rt_b200_load_gguf: ") + what + ": " + cudaGetErrorString(e));
        }
        return e == cudaSuccess;
    };
    bool ok = cuda(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "stream") &&
              cuda(cudaMalloc(&d_sum, sizeof *d_sum), "sum") && cuda(cudaMemsetAsync(d_sum, 0, sizeof *d_sum, s), "sum") &&
              cuda(cudaEventCreate(&e_read), "event") && cuda(cudaEventCreate(&e_done), "event");
    for (int k = 0; ok && k < T; ++k) {
        ok = cuda(cudaStreamCreateWithFlags(&ts[k], cudaStreamNonBlocking), "stream") &&
             cuda(cudaEventCreateWithFlags(&tdone[k], cudaEventDisableTiming), "event");
        for (int b = 0; ok && b < NBUF; ++b)
            ok = cuda(cudaHostAlloc(&buf[k][b], CHUNK, cudaHostAllocDefault), "pinned buffer") &&
                 cuda(cudaEventCreateWithFlags(&ev[k][b], cudaEventDisableTiming), "event");
    }
    const uint64_t nslots = (fb + CHUNK - 1) / CHUNK;
    int device = 0;
    ok = ok && cuda(cudaGetDevice(&device), "device");
    std::vector<std::thread> readers;
    std::vector<int> read_ok(T, 1);
    for (int k = 0; ok && k < T; ++k)
        readers.emplace_back([&, k] {
            if (!cuda(cudaSetDevice(device), "device")) { // the current device is per thread
                read_ok[size_t(k)] = 0;
                return;
            }
            bool used[NBUF] = {};
            for (uint64_t i = uint64_t(k), n = 0; i < nslots; i += T, ++n) {
                const int b = int(n % NBUF);
                if (used[b] && !cuda(cudaEventSynchronize(ev[k][b]), "copy wait")) {
                    read_ok[size_t(k)] = 0;
                    return;
                }
                const uint64_t off = i * CHUNK;
                const size_t want = size_t(fb - off < CHUNK ? fb - off : CHUNK);
                const size_t len = direct ? (want + PAGE - 1) / PAGE * PAGE : want; // whole pages for O_DIRECT
                size_t got = 0;
                while (got < want) {
                    const ssize_t r = pread(fd, static_cast<char *>(buf[k][b]) + got, len - got, off_t(off + got));
                    if (r <= 0)
                        break;
                    got += size_t(r);
                }
                if (got < want) {
                    std::lock_guard<std::mutex> lock(mu);
                    if (rc == RTB_OK)
                        rc = fail(RTB_EINVAL, std::string(path) + ": short read at offset " + std::to_string(off + got));
                    read_ok[size_t(k)] = 0;
                    return;
                }
                if (!cuda(cudaMemcpyAsync(static_cast<char *>(arena) + off, buf[k][b], want, cudaMemcpyHostToDevice, ts[k]),
                          "copy") ||
                    !cuda(cudaEventRecord(ev[k][b], ts[k]), "event")) {
                    read_ok[size_t(k)] = 0;
                    return;
                }
                used[b] = true;
            }
        });
    for (std::thread &th : readers)
        th.join();
    for (int k = 0; ok && k < T; ++k)
        ok = read_ok[size_t(k)] && cuda(cudaEventRecord(tdone[k], ts[k]), "event") &&
             cuda(cudaStreamWaitEvent(s, tdone[k], 0), "join");
    close(fd);
    if (ok && fb % 8) // the sum is over whole words: the tail word counts with zeros
        ok = cuda(cudaMemsetAsync(static_cast<char *>(arena) + fb, 0, size_t(8 - fb % 8), s), "pad");
    if (ok)
        ok = cuda(cudaEventRecord(e_read, s), "event");
    // the file's sum over the device image
    const long long words = (long long)((fb + 7) / 8);
    if (ok && words > 0) {
        file_sum_kernel<<<4 * 148, 256, 0, s>>>(static_cast<const unsigned long long *>(arena), words, d_sum);
        ok = cuda(cudaGetLastError(), "sum kernel");
    }
    // Q8_0 matrices into the row-split layout, in place, each distinct offset once
    int repacked = 0;
    std::vector<uint64_t> done;
    for (size_t i = 0; ok && i < tab.t.size(); ++i) {
        rtb_tensor &t = tab.t[i];
        t.dev = static_cast<char *>(arena) + t.offset;
        long long rows, cols;
        if (!repackable(t, &rows, &cols))
            continue;
        bool seen = false; // a tied copy (same offset, type and dims: check_repack_overlaps)
        for (uint64_t o : done)
            seen |= o == t.offset;
        t.repacked = 1;
        if (seen)
            continue;
        done.push_back(t.offset);
        ok = cuda(q8::launch_repack(static_cast<const uint8_t *>(t.dev), rows, int(cols), static_cast<uint8_t *>(t.dev), s),
                  "repack");
        ++repacked;
    }
    unsigned long long sum = 0;
    if (ok)
        ok = cuda(cudaEventRecord(e_done, s), "event") &&
             cuda(cudaMemcpyAsync(&sum, d_sum, sizeof sum, cudaMemcpyDeviceToHost, s), "sum") &&
             cuda(cudaStreamSynchronize(s), "load");
    const auto t1 = std::chrono::steady_clock::now();
    float ms_repack = 0;
    if (ok)
        cudaEventElapsedTime(&ms_repack, e_read, e_done);
    for (int k = 0; k < T; ++k) {
        for (int b = 0; b < NBUF; ++b) {
            if (ev[k][b])
                cudaEventDestroy(ev[k][b]);
            if (buf[k][b])
                cudaFreeHost(buf[k][b]);
        }
        if (tdone[k])
            cudaEventDestroy(tdone[k]);
        if (ts[k])
            cudaStreamDestroy(ts[k]);
    }
    if (e_read)
        cudaEventDestroy(e_read);
    if (e_done)
        cudaEventDestroy(e_done);
    cudaFree(d_sum);
    if (s)
        cudaStreamDestroy(s);
    if (!ok)
        return rc != RTB_OK ? rc : RTB_ECUDA;
    *n = int(tab.t.size());
    for (int i = 0; out && i < *n; ++i)
        out[i] = tab.t[size_t(i)];
    if (stats) {
        memset(stats, 0, sizeof *stats);
        stats->file_bytes = fb;
        stats->file_sum = sum;
        stats->seconds = std::chrono::duration<double>(t1 - t0).count();
        stats->seconds_repack = double(ms_repack) / 1e3;
        stats->direct = direct ? 1 : 0;
        stats->q8_matrices = repacked;
    }
    return RTB_OK;
}

} // extern "C"
