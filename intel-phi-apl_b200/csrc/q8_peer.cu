// q8_peer.cu: the gather kernel of a row-sharded product's round (the protocol and the region's
// layout are in q8_kernels.h; the stores into the peers' staging images are in the product
// kernel, q8_gemv.cu). It runs on a side stream after the product, so the next product on R's
// stream does not wait for it.
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

__device__ __forceinline__ void st_release_sys(unsigned long long *p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Waits (bounded, about a second) until every peer's word at `off` in this rank's region has
// reached `value`; false if one never did.
__device__ bool wait_peers(const PeerOut &po, size_t off, unsigned long long value) {
    const unsigned char *mine = po.region[po.rank];
    for (int w = 0; w < po.world; ++w) {
        if (w == po.rank)
            continue;
        const unsigned long long *word = reinterpret_cast<const unsigned long long *>(mine + off) + w;
        const long long t0 = clock64();
        while (ld_acquire_sys(word) < value) {
            const long long dt = clock64() - t0;
            if (dt > WAIT_LIMIT_CYCLES)
                return false;
            if (dt > 20000)
                __nanosleep(64);
        }
    }
    return true;
}

constexpr int GATHER_THREADS = 128; // small, so its CTAs fit beside a product's on any SM

// Round r = the rounds gathered so far + 1 (gathers run in order on their stream, one per
// peer-gathered product). Every CTA: wait for the peers' flags of round r (CTA 0 first publishes
// this rank's), copy its share of the peers' rows out of this GPU's image r into y; the last CTA
// then tells the peers it has read round r, waits until every peer has read round r - 1 (so the
// product of round r + 2, which waits for this kernel, may overwrite their images of round
// r - 1), and advances the gathered count.
__global__ void __launch_bounds__(GATHER_THREADS) peer_gather_kernel(const PeerOut po, float *y, int t, unsigned *err) {
    __shared__ int ok;
    __shared__ unsigned long long round_sh;
    unsigned char *mine = po.region[po.rank];
    if (threadIdx.x == 0) {
        const unsigned long long r = *reinterpret_cast<const volatile unsigned long long *>(mine + PEER_GATHERED) + 1;
        round_sh = r;
        if (blockIdx.x == 0) {
            // the product of round r has completed (this kernel follows it): its stores into the
            // peers' images are made visible to them before the flag
            __threadfence_system();
            for (int w = 0; w < po.world; ++w)
                if (w != po.rank)
                    st_release_sys(reinterpret_cast<unsigned long long *>(po.region[w] + PEER_FLAGS) + po.rank, r);
        }
        ok = wait_peers(po, PEER_FLAGS, r) ? 1 : 0;
        if (!ok)
            report(err, ERR_TIMEOUT_PEER);
    }
    __syncthreads();
    const unsigned long long r = round_sh;
    if (ok) {
        const float *stage = reinterpret_cast<const float *>(mine + peer_image(r));
        const long long rows = po.rows_total, lr = rows / po.world, own0 = (long long)po.rank * lr;
        const long long n = (long long)t * rows;
        for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
            const long long tok = e / rows, row = e - tok * rows;
            if (row < own0 || row >= own0 + lr)
                y[tok * rows + row] = __ldcg(stage + e);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned *done = reinterpret_cast<unsigned *>(mine + PEER_GCTAS);
        __threadfence(); // this CTA's reads of the image are done before its count
        if (atomicAdd(done, 1u) == gridDim.x - 1) {
            *done = 0;
            __threadfence();
            for (int w = 0; w < po.world; ++w)
                if (w != po.rank)
                    st_release_sys(reinterpret_cast<unsigned long long *>(po.region[w] + PEER_READS) + po.rank, r);
            if (!wait_peers(po, PEER_READS, r - 1))
                report(err, ERR_TIMEOUT_PEER);
            *reinterpret_cast<volatile unsigned long long *>(mine + PEER_GATHERED) = r;
        }
    }
}

} // namespace

cudaError_t preload_peer() {
    cudaFuncAttributes a;
    return cudaFuncGetAttributes(&a, peer_gather_kernel);
}

cudaError_t launch_peer_gather(const PeerOut &po, float *y, int t, unsigned *err, cudaStream_t stream) {
    if (!po.on || po.world < 2 || po.world > MAX_PEERS || t < 1 ||
        size_t(t) * size_t(po.rows_total) * sizeof(float) > PEER_STAGE_BYTES)
        return cudaErrorInvalidValue;
    const long long n = (long long)t * po.rows_total;
    long long grid = (n + GATHER_THREADS * 16 - 1) / (GATHER_THREADS * 16); // ~16 outputs per thread
    grid = grid < 1 ? 1 : (grid > 64 ? 64 : grid);
    peer_gather_kernel<<<unsigned(grid), GATHER_THREADS, 0, stream>>>(po, y, t, err);
    return cudaGetLastError();
}

} // namespace q8
