// q8_peer.cu: the receiving half of the fused all-gather of a row-sharded product (the sending
// half is in the product kernel: q8_gemv.cu). The layout of a rank's peer region is in
// q8_kernels.h.
#include <cuda_runtime.h>

#include "q8_kernels.h"
#include "q8_ptx.cuh"

namespace q8 {
namespace {

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Every CTA waits for the peers' flags (one thread per peer, bounded), then copies its share of
// the peers' rows out of the staging image of this round.
__global__ void peer_finish_kernel(const PeerOut po, float *y, long long ldy, int t, unsigned *err) {
    // Under programmatic launch the next product may start now (it prefetches its weights and
    // waits for this kernel before reading x); this kernel waits for the product before it.
    if (threadIdx.x == 0)
        grid_launch_dependents();
    grid_wait();
    const unsigned char *mine = po.region[po.rank];
    const unsigned long long round =
        *reinterpret_cast<const volatile unsigned long long *>(mine + 72); // advanced by the product kernel
    __shared__ int ok;
    if (threadIdx.x == 0)
        ok = 1;
    __syncthreads();
    if (threadIdx.x < unsigned(po.world) && int(threadIdx.x) != po.rank) {
        const unsigned long long *flag = reinterpret_cast<const unsigned long long *>(mine) + threadIdx.x;
        const long long t0 = clock64();
        while (ld_acquire_sys(flag) < round) {
            if (clock64() - t0 > WAIT_LIMIT_CYCLES) {
                report(err, ERR_TIMEOUT_PEER);
                ok = 0;
                break;
            }
        }
    }
    __syncthreads();
    if (!ok)
        return;
    const float *stage = reinterpret_cast<const float *>(mine + peer_image(round));
    const long long rows = po.rows_total, lr = rows / po.world, own0 = (long long)po.rank * lr;
    const long long n = (long long)t * rows;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const long long tok = i / rows, row = i - tok * rows;
        if (row < own0 || row >= own0 + lr)
            y[tok * ldy + row] = stage[i];
    }
}

} // namespace

cudaError_t preload_peer() {
    cudaFuncAttributes a;
    return cudaFuncGetAttributes(&a, peer_finish_kernel);
}

cudaError_t launch_peer_finish(const PeerOut &po, float *y, long long ldy, int t, unsigned *err, cudaStream_t stream,
                               bool pdl) {
    if (!po.on || po.world < 2 || po.world > MAX_PEERS || t < 1 ||
        size_t(t) * size_t(po.rows_total) * sizeof(float) > PEER_STAGE_BYTES)
        return cudaErrorInvalidValue;
    const long long n = (long long)t * po.rows_total;
    int grid = int((n + 1023) / 1024);
    grid = grid < 1 ? 1 : (grid > 64 ? 64 : grid);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, peer_finish_kernel, po, y, ldy, t, err);
}

} // namespace q8
