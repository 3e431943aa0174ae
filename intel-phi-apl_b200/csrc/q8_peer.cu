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

// Rounds r0 .. r1 (r0 = the rounds gathered so far + 1: batches run in order on their stream).
// Every CTA: wait for the peers' flags of round r1 (CTA 0 first publishes this rank's), copy its
// share of the peers' rows of every round out of this GPU's images into the rounds' y; the last
// CTA then tells the peers it has read up to r1, waits until every peer has too (the products
// that wait for this kernel may then overwrite those images), and advances the gathered count.
__global__ void __launch_bounds__(GATHER_THREADS) peer_gather_kernel(const PeerOut po, const GatherBatch b, unsigned *err) {
    __shared__ int ok;
    __shared__ unsigned long long r0_sh;
    unsigned char *mine = po.region[po.rank];
    if (threadIdx.x == 0) {
        const unsigned long long r0 = *reinterpret_cast<const volatile unsigned long long *>(mine + PEER_GATHERED) + 1;
        const unsigned long long r1 = r0 + b.n - 1;
        r0_sh = r0;
        if (blockIdx.x == 0) {
            // the batch's products have completed (this kernel follows the last): their stores
            // into the peers' images are made visible to them before the flag
            __threadfence_system();
            for (int w = 0; w < po.world; ++w)
                if (w != po.rank)
                    st_release_sys(reinterpret_cast<unsigned long long *>(po.region[w] + PEER_FLAGS) + po.rank, r1);
        }
        ok = wait_peers(po, PEER_FLAGS, r1) ? 1 : 0;
        if (!ok)
            report(err, ERR_TIMEOUT_PEER);
    }
    __syncthreads();
    const unsigned long long r0 = r0_sh, r1 = r0 + b.n - 1;
    if (ok) {
        for (int i = 0; i < b.n; ++i) {
            const float *stage = reinterpret_cast<const float *>(mine + peer_image(r0 + i));
            const long long rows = b.rows[i], lr = rows / po.world, own0 = (long long)po.rank * lr;
            const long long n = (long long)b.t[i] * rows;
            float *y = b.y[i];
            for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
                const long long tok = e / rows, row = e - tok * rows;
                if (row < own0 || row >= own0 + lr)
                    y[tok * rows + row] = __ldcg(stage + e);
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned *done = reinterpret_cast<unsigned *>(mine + PEER_GCTAS);
        __threadfence(); // this CTA's reads of the images are done before its count
        if (atomicAdd(done, 1u) == gridDim.x - 1) {
            *done = 0;
            __threadfence();
            for (int w = 0; w < po.world; ++w)
                if (w != po.rank)
                    st_release_sys(reinterpret_cast<unsigned long long *>(po.region[w] + PEER_READS) + po.rank, r1);
            if (!wait_peers(po, PEER_READS, r1))
                report(err, ERR_TIMEOUT_PEER);
            *reinterpret_cast<volatile unsigned long long *>(mine + PEER_GATHERED) = r1;
        }
    }
}

} // namespace

cudaError_t preload_peer() {
    cudaFuncAttributes a;
    return cudaFuncGetAttributes(&a, peer_gather_kernel);
}

cudaError_t launch_peer_gather(const PeerOut &po, const GatherBatch &b, unsigned *err, cudaStream_t stream) {
    if (!po.on || po.world < 2 || po.world > MAX_PEERS || b.n < 1 || b.n > GATHER_BATCH)
        return cudaErrorInvalidValue;
    long long n = 0;
    for (int i = 0; i < b.n; ++i) {
        if (b.t[i] < 1 || size_t(b.t[i]) * size_t(b.rows[i]) * sizeof(float) > PEER_STAGE_BYTES)
            return cudaErrorInvalidValue;
        n += (long long)b.t[i] * b.rows[i];
    }
    long long grid = (n + GATHER_THREADS * 16 - 1) / (GATHER_THREADS * 16); // ~16 outputs per thread
    grid = grid < 1 ? 1 : (grid > 64 ? 64 : grid);
    peer_gather_kernel<<<unsigned(grid), GATHER_THREADS, 0, stream>>>(po, b, err);
    return cudaGetLastError();
}

} // namespace q8
