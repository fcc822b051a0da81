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
// FD_TILE_BF16 operand ("packed bf16 row"): row-major [n][kd] bf16 with
//   query row  q~ = [ c*(x-shift) rounded to bf16 (d) | 1 1 1 | split3(nq) | 0 pad ]
//   key   row  k~ = [ (x-shift) rounded to bf16 (d)   | split3(nk) | 1 1 1 | 0 pad ]
// with c = 2*beta*log2(e), nq = -||q^||^2/(2c) ... so that q~.k~ equals the
// base-2 exponent -beta*log2(e)*||a-b||^2 of the two rounded points (a = q^/c, b).
// kd = round_up(d + 6, 16).  Everything else (norms, bias) is folded in.
//
// FD_TILE_F32 operand: row-major [n][dp] fp32 centred points scaled by
// sqrt(beta), dp = round_up(d,4), followed by n fp32 squared norms of the
// stored values (so the tile kernel evaluates exp(-||a-b||^2)).
static inline int kd_bf16(int d) { return (int)round_up(d + 6, 16); }
static inline int dp_f32(int d) { return (int)round_up(d, 4); }

}  // namespace fd
