// Shared definitions for the FlashDiffusion sm_100a library (libfd_sm100.so).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/fd_sm100.h"

namespace fd {

// Set the thread-local error message returned by fd_last_error() and return `code`.
int set_error(int code, const char* fmt, ...);

#define FD_CHECK_ARG(cond, ...)                                                 \
    do {                                                                       \
        if (!(cond)) return ::fd::set_error(FD_ERR_ARG, __VA_ARGS__);          \
    } while (0)

#define FD_CUDA_TRY(expr)                                                      \
    do {                                                                       \
        cudaError_t _e = (expr);                                               \
        if (_e != cudaSuccess)                                                 \
            return ::fd::set_error(FD_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,  \
                                   cudaGetErrorString(_e), __FILE__, __LINE__); \
    } while (0)

#define FD_TRY(expr)                                                           \
    do {                                                                       \
        int _s = (expr);                                                       \
        if (_s != FD_OK) return _s;                                            \
    } while (0)

__host__ __device__ static inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
__host__ __device__ static inline int64_t round_up(int64_t a, int64_t b) { return cdiv(a, b) * b; }
static inline size_t align256(size_t a) { return (a + 255) & ~size_t(255); }

// Load element i of a typed input array as fp32 (inputs arrive as f32/f16/bf16/f64).
__device__ __forceinline__ double load_as_f64(const void* p, int dtype, int64_t i) {
    switch (dtype) {
        case FD_DTYPE_F16: return (double)__half2float(((const __half*)p)[i]);
        case FD_DTYPE_BF16: return (double)__bfloat162float(((const __nv_bfloat16*)p)[i]);
        case FD_DTYPE_F64: return ((const double*)p)[i];
        default: return (double)((const float*)p)[i];
    }
}

// ---- operand formats -------------------------------------------------------
// 16-bit tile operand (FD_TILE_F16 / FD_TILE_BF16): row-major [n][kd] of
// fp16 / bf16 with s = sqrt(2*beta*log2(e)) and a^ = round16(s*(x-shift)):
//   query row  q~ = [ a^ (d) | 1 1 1 | split3(n) | 0 pad ]
//   key   row  k~ = [ a^ (d) | split3(n) | 1 1 1 | 0 pad ]
// n = -||a^||^2 / 2 of the row's own rounded values (split3 = three 16-bit
// parts summing to n to ~2^-24 relative).  Then q~.k~ = -(1/2)||a^_q - a^_k||^2
// = -beta*log2(e)*||a_q - a_k||^2 exactly for the rounded points a = a^/s:
// one MMA accumulator element is the whole base-2 exponent of a pair, and
// both sides round identically, so K(i,j) = K(j,i) for Q = K.
// kd = round_up(d + 6, 16).
//
// FD_TILE_F32 operand: row-major [n][dp] fp32 centred points scaled by
// sqrt(beta), dp = round_up(d,4), followed by n fp32 squared norms of the
// stored values (so the tile kernel evaluates exp(-||a-b||^2)).
static inline int kd_bf16(int d) { return (int)round_up(d + 6, 16); }
// FD_TILE_F16X3 operand: query row [a_hi | a_hi | a_lo | 1 1 1 | split3(n)], key row
// [b_hi | b_lo | b_hi | split3(n) | 1 1 1]: the three products a_hi b_hi +
// a_hi b_lo + a_lo b_hi carry the fp32 value of a.b to ~2^-22.
static inline int kd_f16x3(int d) { return (int)round_up(3 * d + 6, 16); }
static inline int kd_tile(int tile, int d) { return tile == FD_TILE_F16X3 ? kd_f16x3(d) : kd_bf16(d); }
static inline int dp_f32(int d) { return (int)round_up(d, 4); }

}  // namespace fd
