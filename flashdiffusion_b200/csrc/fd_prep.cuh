// Launchers for the O(N) helper kernels (fd_prep.cu) and the tile kernels.
#pragma once
#include <algorithm>
#include "fd_common.cuh"

namespace fd {

int launch_sq_norms(const void* X, int dtype, int64_t n, int d, float* sq, cudaStream_t s);
int launch_mean_rows(const void* X, int dtype, int64_t n, int d, float* shift, cudaStream_t s);
int launch_pack(const void* X, int dtype, int64_t n, int d, const float* shift, float beta, int side,
                int tile, void* op, cudaStream_t s);
int launch_rhs_f32(const void* V, int v_dtype, int64_t nk, int64_t nk_pad, int ldv, int c0, int rc,
                   const float* cs, const float* ch, float* u, cudaStream_t s);
int launch_rhs_bf16t(const void* V, int v_dtype, int64_t nk, int64_t ld, int ldv, int c0, int rc,
                     const float* cs, const float* ch, __nv_bfloat16* ut, cudaStream_t s);
int launch_rhs_f16t(const void* V, int v_dtype, int64_t nk, int64_t ld, int ldv, int c0, int rc, int rp,
                    const float* cs, const float* ch, unsigned* colmax, __half* ut, float* colscale, cudaStream_t s);
int launch_dmap_weights(const float* D, int64_t n, float alpha, float* w, cudaStream_t s);
int launch_dmap_rscale(const float* Kw, const float* w, int64_t n, float* Da, float* rs, cudaStream_t s);

// Epilogue description shared by the tile kernels: out[i*ldo + c0 + c] =
// acc[i][c] * row_scale[i] / row_div[i], stored as fp32 or fp64.
struct RowEpilogue {
    const float* row_scale;  // may be null
    const float* row_div;    // may be null
    void* out;
    int out_dtype;           // FD_DTYPE_F32 or FD_DTYPE_F64
    int64_t ldo;             // row stride of out, in elements
    int c0;                  // first output column of this launch
};

__device__ __forceinline__ void store_out(const RowEpilogue& ep, int64_t i, int c, double v) {
    if (ep.row_scale) v *= (double)ep.row_scale[i];
    if (ep.row_div) v /= (double)ep.row_div[i];
    const int64_t idx = i * ep.ldo + ep.c0 + c;
    if (ep.out_dtype == FD_DTYPE_F64) ((double*)ep.out)[idx] = v;
    else ((float*)ep.out)[idx] = (float)v;
}

// out rows [0, nq) x rc columns <- 0 (empty key set).
int launch_zero_rows(int64_t nq, int rc, const RowEpilogue& ep, cudaStream_t s);

// fp32 SIMT tiles (FD_TILE_F32).  u: (nk_pad, rc) fp32 prepared rhs.
size_t simt_workspace_bytes(int64_t nq, int64_t nk, int rc);
int launch_simt(const float* qpts, const float* qsq, int64_t nq, const float* kpts, const float* ksq,
                int64_t nk, int d, const float* u, int rc, float beta, const RowEpilogue& ep,
                void* ws, size_t ws_bytes, cudaStream_t s);

// 16-bit tcgen05 tiles (FD_TILE_F16 / FD_TILE_BF16).
size_t tc_workspace_bytes(int64_t nq, int64_t nk, int rc);
int launch_tc(const void* qop, int64_t nq, const void* kop, int64_t nk, int d, int tile,
              const void* rhs, int rc, const RowEpilogue& ep, void* ws, size_t ws_bytes, cudaStream_t s);

// 16-bit tcgen05 tiles with a block right-hand side (up to 64 columns per launch).
int block_rp(int rc);
int block_max_cols(int d);
size_t tc_block_workspace_bytes(int rp);
int launch_tc_block(const void* qop, int64_t nq, const void* kop, int64_t nk, int d, int tile, const void* ut,
                    int64_t ld, const float* colscale, int rc, const RowEpilogue& ep, void* ws, size_t ws_bytes,
                    cudaStream_t s);

int read_and_clear_status(cudaStream_t s, int* status);
// Device address of the library's status word (bounded-wait timeouts, fp16 range).
int status_word(int** ptr);
static inline bool is_tc_tile(int tile) {
    return tile == FD_TILE_BF16 || tile == FD_TILE_F16 || tile == FD_TILE_F16X3;
}

}  // namespace fd
