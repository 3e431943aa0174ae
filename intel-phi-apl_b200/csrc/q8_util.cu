// q8_util.cu: the load-side and support kernels.
//   - repack: GGUF Q8_0 rows -> the row-split layout (q8_layout.h), the device counterpart of the
//     reference's load-time repack (src/card/gemv.c:23-52, called at src/card/engine.c:303-316);
//     in place when a row keeps its length (cols a multiple of 256), as the reference repacks;
//   - q8_row: one dequantised row, z[i] = (float)q * (float)d in one fp32 rounding, as
//     rt_q8_row does (src/card/rt.c:484-501);
//   - synth: the seeded synthetic weights and activations, bit-identical to the CPU generator
//     (an Irwin-Hall sum of 12 uniforms per value from splitmix64 words; Q8_0 quantised with
//     d = amax/127 stored fp16 and q = round(w / d)).
#include <cuda_fp16.h>

#include "q8_kernels.h"
#include "q8_layout.h"

namespace q8 {
namespace {

// ---------------------------------------------------------------- repack
// One CTA per row: the whole GGUF row is read into shared memory before any byte is written, so
// out == gguf is safe when the two row lengths agree.
__global__ void repack_kernel(const uint8_t *gguf, long long rows, int cols, uint8_t *out) {
    extern __shared__ __align__(16) uint8_t row[];
    const int nb = cols / Q8_QK;
    const long long gb = q8_gguf_row_bytes(cols), sb = q8s_row_bytes(cols);
    const int ss = int(q8s_scale_stride(cols));
    for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
        const uint8_t *src = gguf + r * gb;
        for (long long i = threadIdx.x; i < gb; i += blockDim.x)
            row[i] = src[i];
        __syncthreads();
        uint8_t *dst = out + r * sb;
        for (int i = threadIdx.x; i < cols; i += blockDim.x) // quants
            dst[i] = row[(i / Q8_QK) * Q8_GGUF_BLOCK + 2 + (i % Q8_QK)];
        for (int b = threadIdx.x; b < ss; b += blockDim.x) { // scales, zero pad
            const uint16_t d = b < nb ? uint16_t(row[b * Q8_GGUF_BLOCK] | row[b * Q8_GGUF_BLOCK + 1] << 8) : 0;
            dst[cols + 2 * b] = uint8_t(d & 0xff);
            dst[cols + 2 * b + 1] = uint8_t(d >> 8);
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------- dequantised row
__global__ void q8_row_kernel(const uint8_t *w, int cols, long long row, float *z) {
    const uint8_t *p = w + row * q8s_row_bytes(cols);
    const __half *d = reinterpret_cast<const __half *>(p + cols);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < cols; i += gridDim.x * blockDim.x)
        z[i] = __fmul_rn(float(int8_t(p[i])), __half2float(d[i / Q8_QK]));
}

// ---------------------------------------------------------------- synthetic inputs
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ float normal_at(uint64_t base, uint64_t index) {
    uint32_t s = 0;
#pragma unroll
    for (uint64_t k = 0; k < 3; ++k) {
        const uint64_t z = mix64(base + (index * 3 + k + 1) * 0x9E3779B97F4A7C15ull);
        s += uint32_t(z & 0xffff) + uint32_t((z >> 16) & 0xffff) + uint32_t((z >> 32) & 0xffff) + uint32_t(z >> 48);
    }
    return __fsub_rn(__fmul_rn(float(2 * s + 12), 1.0f / 131072.0f), 6.0f);
}

// One thread per (row, block): 32 values, quantised, written into the split layout.
__global__ void synth_q8_kernel(uint8_t *out, long long row0, long long rows, int cols, uint64_t seed, uint64_t sid,
                                float sigma) {
    const uint64_t base = mix64(seed + 0x9E3779B97F4A7C15ull * (sid + 1));
    const int nb = cols / Q8_QK, ss = int(q8s_scale_stride(cols));
    const long long rb = q8s_row_bytes(cols);
    const long long n = rows * ss;
    for (long long u = blockIdx.x * (long long)blockDim.x + threadIdx.x; u < n; u += (long long)gridDim.x * blockDim.x) {
        const long long r = u / ss;
        const int b = int(u - r * ss);
        uint8_t *row = out + r * rb;
        if (b >= nb) { // scale padding
            reinterpret_cast<uint16_t *>(row + cols)[b] = 0;
            continue;
        }
        float w[Q8_QK], amax = 0.0f;
        const uint64_t e0 = uint64_t(row0 + r) * uint64_t(cols) + uint64_t(b) * Q8_QK;
#pragma unroll
        for (int i = 0; i < Q8_QK; ++i) {
            w[i] = __fmul_rn(normal_at(base, e0 + i), sigma);
            amax = fmaxf(amax, fabsf(w[i]));
        }
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        const __half dh = __float2half_rn(d);
        reinterpret_cast<__half *>(row + cols)[b] = dh;
        uint32_t packed[Q8_QK / 4];
#pragma unroll
        for (int i = 0; i < Q8_QK; i += 4) {
            uint32_t v = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                float q = roundf(__fmul_rn(w[i + k], id));
                q = fminf(127.0f, fmaxf(-127.0f, q));
                v |= uint32_t(uint8_t(int8_t(q))) << (8 * k);
            }
            packed[i / 4] = v;
        }
        uint4 *dst = reinterpret_cast<uint4 *>(row + b * Q8_QK);
        dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
        dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
    }
}

__global__ void synth_f32_kernel(float *out, long long n, uint64_t seed, uint64_t sid, float sigma) {
    const uint64_t base = mix64(seed + 0x9E3779B97F4A7C15ull * (sid + 1));
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        out[i] = __fmul_rn(normal_at(base, uint64_t(i)), sigma);
}

int grid_for(long long n, int block) {
    long long g = (n + block - 1) / block;
    return int(g < 1 ? 1 : g > 65535 * 16 ? 65535 * 16 : g);
}

} // namespace

cudaError_t launch_repack(const uint8_t *gguf, long long rows, int cols, uint8_t *out, cudaStream_t stream) {
    if (rows < 1 || cols < Q8_QK || cols % Q8_QK)
        return cudaErrorInvalidValue;
    const long long gb = q8_gguf_row_bytes(cols);
    if (gb > REPACK_MAX_ROW_BYTES)
        return cudaErrorInvalidValue;
    if (gb > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(repack_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(gb));
        if (e != cudaSuccess)
            return e;
    }
    const int grid = int(rows < 65536 ? rows : 65536);
    repack_kernel<<<grid, 256, size_t(gb), stream>>>(gguf, rows, cols, out);
    return cudaGetLastError();
}

cudaError_t launch_synth_q8(uint8_t *out, long long row0, long long rows, int cols, uint64_t seed, uint64_t sid,
                            float sigma, cudaStream_t stream) {
    if (rows < 1 || cols < Q8_QK || cols % Q8_QK)
        return cudaErrorInvalidValue;
    const long long n = rows * q8s_scale_stride(cols);
    synth_q8_kernel<<<grid_for(n, 128), 128, 0, stream>>>(out, row0, rows, cols, seed, sid, sigma);
    return cudaGetLastError();
}

cudaError_t launch_synth_f32(float *out, long long n, uint64_t seed, uint64_t sid, float sigma, cudaStream_t stream) {
    if (n < 1)
        return cudaErrorInvalidValue;
    synth_f32_kernel<<<grid_for(n, 256), 256, 0, stream>>>(out, n, seed, sid, sigma);
    return cudaGetLastError();
}

cudaError_t launch_q8_row(const uint8_t *w, int cols, long long row, float *z, cudaStream_t stream) {
    if (cols < Q8_QK || cols % Q8_QK || row < 0)
        return cudaErrorInvalidValue;
    q8_row_kernel<<<(cols + 255) / 256, 256, 0, stream>>>(w, cols, row, z);
    return cudaGetLastError();
}

} // namespace q8
