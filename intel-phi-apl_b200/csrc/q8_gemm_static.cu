// q8_gemm_static.cu: rt_gemm_static, the tensor-core Q8_0 product for callers that cannot
// allocate device memory.
//
// Some hosts of these products own every device allocation themselves: an engine that carves its
// whole HBM budget up front, a runtime that forbids allocation on the serving path, or a caller
// holding a fixed memory pool. Such a caller can't let the library cudaMalloc a scratch buffer,
// as rt_gemm's tensor-core path does for its fp16 copy of x.
// This entry point runs the same kernel with its scratch in a file-scope device array of fixed
// size instead. The caller passes only inputs and outputs. Nothing here calls cudaMalloc,
// cudaFree or an allocating library routine.
//
//   - Limits: the fp16 copy of x must fit STATIC_X_BYTES = 8 MiB, so t * cols <= 4,194,304
//     (e.g. 512 tokens of 8192 columns), and the per-row scale exponents STATIC_ROW_BYTES, so
//     rows <= 1,048,576. Larger calls are rejected with RTB_EINVAL.
//   - Every GPU that loads the library holds the array (9.5 MiB + 256 bytes) until the process
//     exits.
//   - All calls share the one array. Calls that overlap on the GPU (from two host threads, or on
//     two streams) race on it and must not be issued.
//   - The first call on a device looks up the array's device address on that device (the name
//     of the array in host code is only a stand-in, not a device address). Make that first call
//     before any stream capture. A later call repeats the look-up only if the device's context
//     changed (after cudaDeviceReset, say).
//   - Each call waits for `stream` before it returns: it reads the kernel's error word back.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "../../include/rt_b200.h"
#include "q8_kernels.h"
#include "q8_layout.h"

namespace {

constexpr size_t STATIC_HEADER = 256;             // the kernel's error word, then padding
constexpr size_t STATIC_X_BYTES = 8ull << 20;     // the fp16 copy of x
constexpr size_t STATIC_TOKEN_BYTES = 512ull << 10; // 2^-s_t per token: t <= 131,072 (t * cols <= 4 Mi, cols >= 32)
constexpr size_t STATIC_ROW_BYTES = 1ull << 20;   // r_o per weight row: rows <= 1,048,576
constexpr size_t STATIC_SCRATCH = STATIC_X_BYTES + STATIC_TOKEN_BYTES + STATIC_ROW_BYTES;
constexpr int MAX_DEVICES = 64;

static __device__ __align__(256) unsigned char g_static_scratch[STATIC_HEADER + STATIC_SCRATCH];

struct DeviceScratch {
    bool ready = false;
    void *ctx = nullptr;           // the device's context when the address was looked up
    unsigned char *base = nullptr; // device address of g_static_scratch on this device
    int num_sms = 0;
};

std::mutex g_setup_mutex;
DeviceScratch g_devices[MAX_DEVICES];

// The calling thread's current context (the driver's cuCtxGetCurrent, looked up through the
// runtime), or null.
void *current_context() {
    static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void *f = nullptr;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f, 4000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(f);
    });
    CUcontext c = nullptr;
    if (!fn || fn(&c) != CUDA_SUCCESS)
        return nullptr;
    return c;
}

// Once per device (again if its context changed), with that device current: the array's device
// address and the SM count.
int device_scratch(DeviceScratch **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES)
        return RTB_ECUDA;
    void *ctx = current_context(); // null before this thread's first CUDA work on the device
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    DeviceScratch &d = g_devices[dev];
    if (!d.ready || !ctx || d.ctx != ctx) {
        d.ready = false;
        void *p = nullptr;
        // (the look-up also makes the device's primary context current when none was)
        if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || !p)
            return RTB_ECUDA;
        if (cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return RTB_ECUDA;
        d.base = static_cast<unsigned char *>(p);
        d.ctx = current_context();
        d.ready = true;
    }
    *out = &d;
    return RTB_OK;
}

bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

} // namespace

extern "C" RTB_API int rt_gemm_static(const void *w, long rows, long cols, const float *x, long t, float *y,
                                      void *stream) {
    if (!w || !x || !y || rows < 1 || rows > (1l << 31) || cols < Q8_QK || cols % Q8_QK || t < 16 ||
        t > (1l << 20) || !aligned(w, 16) || !aligned(x, 16) || !aligned(y, 4))
        return RTB_EINVAL;
    const size_t xh_bytes = (size_t(t) * size_t(cols) * 2 + 255) / 256 * 256;
    if (xh_bytes > STATIC_X_BYTES || size_t(rows) > STATIC_ROW_BYTES)
        return RTB_EINVAL; // beyond the static scratch: use rt_gemm
    DeviceScratch *d = nullptr;
    const int rc = device_scratch(&d);
    if (rc != RTB_OK)
        return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned *err = reinterpret_cast<unsigned *>(d->base);
    // the array keeps the last call's contents: the error word must start at zero
    if (cudaMemsetAsync(err, 0, sizeof(unsigned), s) != cudaSuccess)
        return RTB_ECUDA;
    q8::GemmJob job = {};
    job.w = static_cast<const uint8_t *>(w);
    job.w2 = nullptr;
    job.x = x;
    job.ldx = cols;
    job.y = y;
    job.ldy = rows;
    job.rows = rows;
    job.cols = int(cols);
    job.t = int(t);
    if (q8::gemm_tc_scratch_bytes(&job, 1, d->num_sms, false) > STATIC_SCRATCH)
        return RTB_EINVAL;
    if (q8::launch_gemm_tc(&job, 1, d->base + STATIC_HEADER, STATIC_SCRATCH, d->num_sms, err, s, false, false) !=
        cudaSuccess)
        return RTB_ECUDA;
    unsigned h = 0;
    if (cudaMemcpyAsync(&h, err, sizeof h, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return RTB_ECUDA;
    return h ? RTB_EKERNEL : RTB_OK;
}
