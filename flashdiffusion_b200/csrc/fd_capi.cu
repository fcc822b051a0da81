// extern "C" entry points of libfd_sm100.so (declared in include/fd_sm100.h).
// Validation happens here, before any launch; kernels live in fd_prep.cu,
// fd_simt.cu and fd_tc.cu.
#include <cstdarg>
#include <cstdio>

#include "fd_prep.cuh"

namespace fd {

static thread_local char g_err[512] = "no error";

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

__global__ void zero_rows_kernel(int64_t nq, int rc, RowEpilogue ep) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < nq * rc;
         e += (int64_t)gridDim.x * blockDim.x)
        store_out(ep, e / rc, (int)(e % rc), 0.0);
}

int launch_zero_rows(int64_t nq, int rc, const RowEpilogue& ep, cudaStream_t s) {
    if (nq * rc == 0) return FD_OK;
    zero_rows_kernel<<<(int)std::min<int64_t>(cdiv(nq * rc, 256), 148 * 8), 256, 0, s>>>(nq, rc, ep);
    FD_CUDA_TRY(cudaGetLastError());
    return FD_OK;
}

static bool valid_dtype(int t) { return t == FD_DTYPE_F32 || t == FD_DTYPE_F16 || t == FD_DTYPE_BF16 || t == FD_DTYPE_F64; }
static bool valid_tile(int t) {
    return t == FD_TILE_BF16 || t == FD_TILE_F32 || t == FD_TILE_F16 || t == FD_TILE_F16X3;
}

// columns of V handled per tile-kernel launch (an upper bound over d: operands
// wider than the block kernel's limit take one column per launch, which needs
// less)
static int cols_per_launch(int tile, int r) {
    if (tile == FD_TILE_F32) return 64;
    return r == 1 ? 1 : block_max_cols(0);
}

// prepared right-hand side: fp32 u (r = 1 tensor-core and fp32 paths) or the
// transposed, column-scaled fp16 block plus 2 x 64 column words (block path)
static size_t rhs_bytes(int64_t nk, int r, int tile) {
    const int rc = std::min(r, cols_per_launch(tile, r));
    const int64_t nk_pad = round_up(std::max<int64_t>(nk, 1), 128);
    if (is_tc_tile(tile) && r > 1)
        return align256(sizeof(__half) * 2 * (size_t)nk_pad * block_rp(rc)) + align256(sizeof(float) * 128);
    return align256(sizeof(float) * (size_t)nk_pad * rc);
}

static size_t kernel_ws_bytes(int64_t nq, int64_t nk, int r, int tile) {
    const int rc = std::min(r, cols_per_launch(tile, r));
    if (tile == FD_TILE_F32) return simt_workspace_bytes(nq, nk, rc);
    if (r > 1) return tc_block_workspace_bytes(block_rp(rc));
    return tc_workspace_bytes(nq, nk, rc);
}

}  // namespace fd

using namespace fd;

extern "C" {

const char* fd_last_error(void) { return g_err; }

int fd_version(void) { return 100; }

int fd_device_supported(int device) {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return 0;
    return prop.major == 10 ? 1 : 0;
}

int fd_check_status(void* stream) {
    int st = 0;
    FD_TRY(read_and_clear_status((cudaStream_t)stream, &st));
    if (st != FD_OK) return set_error(st, "a bounded device-side wait gave up (status %d)", st);
    return FD_OK;
}

int fd_compute_sq_norms(const void* X, int dtype, int64_t n, int d, float* sq, void* stream) {
    FD_CHECK_ARG(n >= 0 && d >= 1, "bad shape n=%lld d=%d", (long long)n, d);
    FD_CHECK_ARG(valid_dtype(dtype), "bad dtype %d", dtype);
    FD_CHECK_ARG(n == 0 || (X && sq), "null pointer");
    return launch_sq_norms(X, dtype, n, d, sq, (cudaStream_t)stream);
}

size_t fd_operand_bytes(int64_t n, int d, int tile) {
    if (n < 0 || d < 1) return 0;
    if (tile == FD_TILE_F32)
        return align256(sizeof(float) * (size_t)n * dp_f32(d)) + align256(sizeof(float) * (size_t)n);
    return align256(2 * (size_t)n * kd_tile(tile, d));
}

int fd_mean_rows(const void* X, int dtype, int64_t n, int d, float* shift, void* stream) {
    FD_CHECK_ARG(n >= 0 && d >= 1, "bad shape n=%lld d=%d", (long long)n, d);
    FD_CHECK_ARG(valid_dtype(dtype), "bad dtype %d", dtype);
    FD_CHECK_ARG(shift && (n == 0 || X), "null pointer");
    return launch_mean_rows(X, dtype, n, d, shift, (cudaStream_t)stream);
}

int fd_pack_operand(const void* X, int dtype, int64_t n, int d, const float* shift, float beta, int side,
                    int tile, void* operand, void* stream) {
    FD_CHECK_ARG(n >= 0 && d >= 1, "bad shape n=%lld d=%d", (long long)n, d);
    FD_CHECK_ARG(valid_dtype(dtype), "bad dtype %d", dtype);
    FD_CHECK_ARG(valid_tile(tile), "bad tile %d", tile);
    FD_CHECK_ARG(side == FD_SIDE_QUERY || side == FD_SIDE_KEY, "bad side %d", side);
    FD_CHECK_ARG(beta > 0.f, "beta must be positive (got %g)", (double)beta);
    FD_CHECK_ARG(kd_tile(tile, d) <= 416 || tile == FD_TILE_F32,
                 "tensor-core tiles support operand rows of up to 416 columns (d <= %d for this tile)",
                 tile == FD_TILE_F16X3 ? 136 : 410);
    FD_CHECK_ARG(n == 0 || (X && operand), "null pointer");
    FD_CHECK_ARG(((uintptr_t)operand & 255) == 0, "operand must be 256-byte aligned");
    return launch_pack(X, dtype, n, d, shift, beta, side, tile, operand, (cudaStream_t)stream);
}

size_t fd_apply_workspace_bytes(int64_t nq, int64_t nk, int r, int tile) {
    if (nq < 0 || nk < 0 || r < 1 || !valid_tile(tile)) return 0;
    return rhs_bytes(nk, r, tile) + kernel_ws_bytes(nq, nk, r, tile);
}

int fd_apply(const void* Qop, int64_t nq, const void* Kop, int64_t nk, int d, int tile, const void* V,
             int v_dtype, int r, const float* col_scale, const float* col_h, const float* row_scale,
             const float* row_div, void* out, int out_dtype, void* workspace, size_t workspace_bytes,
             void* stream) {
    cudaStream_t s = (cudaStream_t)stream;
    FD_CHECK_ARG(nq >= 0 && nk >= 0 && d >= 1 && r >= 1, "bad shape nq=%lld nk=%lld d=%d r=%d",
                 (long long)nq, (long long)nk, d, r);
    FD_CHECK_ARG(valid_tile(tile), "bad tile %d", tile);
    FD_CHECK_ARG(v_dtype == FD_DTYPE_F32 || v_dtype == FD_DTYPE_F64, "V must be fp32 or fp64");
    FD_CHECK_ARG(out_dtype == FD_DTYPE_F32 || out_dtype == FD_DTYPE_F64, "out must be fp32 or fp64");
    FD_CHECK_ARG(nq == 0 || out, "null out");
    FD_CHECK_ARG(nq == 0 || nk == 0 || (Qop && Kop), "null operand");
    const size_t need = fd_apply_workspace_bytes(nq, nk, r, tile);
    if (workspace_bytes < need)
        return set_error(FD_ERR_WORKSPACE, "workspace %zu B < required %zu B", workspace_bytes, need);
    FD_CHECK_ARG(need == 0 || (workspace && ((uintptr_t)workspace & 255) == 0),
                 "workspace must be non-null and 256-byte aligned");
    if (nq == 0) return FD_OK;

    // (the workspace query is sized for block_max_cols columns, an upper bound for any d)
    // block tensor-core path for every r > 1 (operand rows of up to 416 columns;
    // above 208 the key tiles stream through the ring as single boxes)
    const bool block = is_tc_tile(tile) && r > 1;
    const int cpl = block ? block_max_cols(d) : cols_per_launch(tile, r);
    const int64_t nk_pad = round_up(std::max<int64_t>(nk, 1), 128);
    uint8_t* ws = (uint8_t*)workspace;
    float* u = (float*)ws;
    uint8_t* kws = ws + rhs_bytes(nk, r, tile);
    const size_t kws_bytes = workspace_bytes - rhs_bytes(nk, r, tile);
    for (int c0 = 0; c0 < r; c0 += cpl) {
        const int rc = std::min(cpl, r - c0);
        RowEpilogue ep{row_scale, row_div, out, out_dtype, (int64_t)r, c0};
        if (nk == 0) { FD_TRY(launch_zero_rows(nq, rc, ep, s)); continue; }
        if (block) {
            const int rp = block_rp(rc);
            __half* ut = (__half*)ws;
            float* colscale = (float*)(ws + align256(sizeof(__half) * 2 * (size_t)nk_pad * rp));
            unsigned* colmax = (unsigned*)(colscale + 64);
            FD_TRY(launch_rhs_f16t(V, v_dtype, nk, nk_pad, r, c0, rc, rp, col_scale, col_h, colmax, ut, colscale, s));
            FD_TRY(launch_tc_block(Qop, nq, Kop, nk, d, tile, ut, nk_pad, colscale, rc, ep, kws, kws_bytes, s));
            continue;
        }
        FD_TRY(launch_rhs_f32(V, v_dtype, nk, nk_pad, r, c0, rc, col_scale, col_h, u, s));
        if (tile == FD_TILE_F32) {
            const float* qp = (const float*)Qop;
            const float* qsq = (const float*)((const uint8_t*)Qop + align256(sizeof(float) * (size_t)nq * dp_f32(d)));
            const float* kp = (const float*)Kop;
            const float* ksq = (const float*)((const uint8_t*)Kop + align256(sizeof(float) * (size_t)nk * dp_f32(d)));
            // the fp32 operands carry sqrt(beta) in their coordinates
            FD_TRY(launch_simt(qp, qsq, nq, kp, ksq, nk, d, u, rc, 1.0f, ep, kws, kws_bytes, s));
        } else {
            FD_TRY(launch_tc(Qop, nq, Kop, nk, d, tile, u, rc, ep, kws, kws_bytes, s));
        }
    }
    return FD_OK;
}

size_t fd_workspace_bytes(int64_t nq, int64_t nk, int d, int r, int tile) {
    if (nq < 0 || nk < 0 || d < 1 || r < 1 || !valid_tile(tile)) return 0;
    return align256(sizeof(float) * (size_t)d) + fd_operand_bytes(nq, d, tile) + fd_operand_bytes(nk, d, tile) +
           fd_apply_workspace_bytes(nq, nk, r, tile);
}

int fd_flash_diffusion(const void* Q, const void* K, int dtype, int64_t nq, int64_t nk, int d, const float* V,
                       int r, float beta, const float* rscale_q, const float* rscale_k, const float* h,
                       const float* row_div, int tile, float* out, void* workspace, size_t workspace_bytes,
                       void* stream) {
    cudaStream_t s = (cudaStream_t)stream;
    FD_CHECK_ARG(nq >= 0 && nk >= 0 && d >= 1 && r >= 1, "bad shape nq=%lld nk=%lld d=%d r=%d",
                 (long long)nq, (long long)nk, d, r);
    FD_CHECK_ARG(valid_dtype(dtype), "bad dtype %d", dtype);
    FD_CHECK_ARG(valid_tile(tile), "bad tile %d", tile);
    FD_CHECK_ARG(beta > 0.f, "beta must be positive (got %g)", (double)beta);
    const size_t need = fd_workspace_bytes(nq, nk, d, r, tile);
    if (workspace_bytes < need)
        return set_error(FD_ERR_WORKSPACE, "workspace %zu B < required %zu B", workspace_bytes, need);
    FD_CHECK_ARG(workspace && ((uintptr_t)workspace & 255) == 0, "workspace must be non-null and 256-byte aligned");
    FD_CHECK_ARG(nq == 0 || nk == 0 || (Q && K && out), "null pointer");
    if (nq == 0) return FD_OK;
    uint8_t* ws = (uint8_t*)workspace;
    float* shift = (float*)ws;
    ws += align256(sizeof(float) * (size_t)d);
    void* qop = ws;
    ws += fd_operand_bytes(nq, d, tile);
    void* kop = ws;
    ws += fd_operand_bytes(nk, d, tile);
    const size_t rest = workspace_bytes - (size_t)(ws - (uint8_t*)workspace);
    if (nk > 0) {
        FD_TRY(launch_mean_rows(K, dtype, nk, d, shift, s));
        FD_TRY(launch_pack(Q, dtype, nq, d, shift, beta, FD_SIDE_QUERY, tile, qop, s));
        FD_TRY(launch_pack(K, dtype, nk, d, shift, beta, FD_SIDE_KEY, tile, kop, s));
    }
    return fd_apply(qop, nq, kop, nk, d, tile, V, FD_DTYPE_F32, r, rscale_k, h, rscale_q, row_div, out,
                    FD_DTYPE_F32, ws, rest, stream);
}

int fd_prepass(const void* X, int dtype, int64_t n, int d, const float* w, float beta, int tile, float* D,
               void* workspace, size_t workspace_bytes, void* stream) {
    // w == NULL means unit weights (the first Coifman-Lafon pass)
    return fd_flash_diffusion(X, X, dtype, n, n, d, w, 1, beta, nullptr, nullptr, nullptr, nullptr, tile, D,
                              workspace, workspace_bytes, stream);
}

int fd_matvec(const void* X, int dtype, int64_t n, int d, const float* v, const float* rscale, float beta,
              int tile, float* out, void* workspace, size_t workspace_bytes, void* stream) {
    FD_CHECK_ARG(rscale || n == 0, "null rscale");
    return fd_flash_diffusion(X, X, dtype, n, n, d, v, 1, beta, rscale, rscale, nullptr, nullptr, tile, out,
                              workspace, workspace_bytes, stream);
}

int fd_dmap_weights(const float* D, int64_t n, float alpha, float* w, void* stream) {
    FD_CHECK_ARG(n >= 0 && (n == 0 || (D && w)), "bad arguments");
    return launch_dmap_weights(D, n, alpha, w, (cudaStream_t)stream);
}

int fd_dmap_rscale(const float* Kw, const float* w, int64_t n, float* D_alpha, float* rscale, void* stream) {
    FD_CHECK_ARG(n >= 0 && (n == 0 || (Kw && w && rscale)), "bad arguments");
    return launch_dmap_rscale(Kw, w, n, D_alpha, rscale, (cudaStream_t)stream);
}

}  // extern "C"
