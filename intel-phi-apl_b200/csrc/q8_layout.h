// q8_layout.h: the split Q8_0 layout in HBM, shared by the kernels and the host shim.
//
// The reference stores Q8_0 weights as GGUF blocks (per row, per 32 columns: an fp16 scale d then
// 32 int8 q, 34 bytes; src/host/gguf_reader.c:21) and repacks them for its card into "form I"
// tiles (src/card/gemv.h:7-11). This library repacks them instead into a row-split form:
//
//   row r of a rows x cols matrix starts at  w + r * row_bytes(cols), and holds
//     [ cols int8 quants | S fp16 scales ]   S = cols/32 rounded up to a multiple of 8 (pad 0)
//
// so every row's quants start 16-byte aligned (coalesced 128-bit and bulk loads), the scales sit
// apart from the quants, and a row is self-contained: a row gather or rt_q8_row needs only the
// row index. With cols a multiple of 256 a row is exactly as long as its GGUF row (cols*34/32
// bytes), so the repack can run in place, row by row.
#pragma once
#include <stdint.h>

#ifdef __CUDACC__
#define Q8_HD __host__ __device__
#else
#define Q8_HD
#endif

#define Q8_QK 32
#define Q8_GGUF_BLOCK 34

static inline Q8_HD long long q8s_scale_stride(long long cols) { return (cols / Q8_QK + 7) / 8 * 8; }
static inline Q8_HD long long q8s_row_bytes(long long cols) { return cols + 2 * q8s_scale_stride(cols); }
static inline Q8_HD long long q8s_bytes(long long rows, long long cols) { return rows * q8s_row_bytes(cols); }
static inline Q8_HD long long q8_gguf_row_bytes(long long cols) { return cols / Q8_QK * Q8_GGUF_BLOCK; }
