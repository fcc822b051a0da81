/*
 * fd_sm100.h — C ABI of libfd_sm100.so, the B200 (sm_100a) FlashDiffusion operator.
 *
 * The operator never materialises the kernel matrix:
 *
 *     K(i,j) = exp(-beta * ||q_i - k_j||^2)
 *     out_i  = row_scale_i / row_div_i * sum_j K(i,j) * col_scale_j * h_j * V_j
 *
 * Reference interfaces each entry point replaces are cited as file:line of
 * sparsetrace/FlashDiffusion (FD/ = src/flashdiffusion/).
 *
 * Conventions
 *  - Every pointer is a DEVICE pointer unless stated otherwise; the caller owns
 *    every buffer (inputs, outputs and workspace).  Nothing here allocates
 *    device memory: sizes of caller-provided workspaces come from the *_bytes()
 *    queries.
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *    All work is enqueued on it; nothing synchronises the host.
 *  - Return value: FD_OK (0) or an FD_ERR_* code; fd_last_error() gives a
 *    human-readable message for the calling host thread.  Argument errors are
 *    detected before any launch (the reference raises RuntimeError through
 *    TORCH_CHECK in the same situations, FD/csrc/flash_diffusion_sm100.cu:98-110).
 *  - Device-side pipeline waits are bounded; a wait that gives up records
 *    FD_ERR_TIMEOUT in a device status word that fd_check_status() reads.
 */
#ifndef FD_SM100_H
#define FD_SM100_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define FD_OK 0
#define FD_ERR_ARG 1          /* bad argument (shape, null pointer, alignment, size) */
#define FD_ERR_CUDA 2         /* CUDA runtime / driver error                          */
#define FD_ERR_UNSUPPORTED 3  /* device is not sm_100-family or shape unsupported     */
#define FD_ERR_TIMEOUT 4      /* a bounded device-side wait gave up                   */
#define FD_ERR_WORKSPACE 5    /* caller workspace too small                           */
#define FD_ERR_RANGE 6        /* fp16 tile operand would overflow (use FD_TILE_BF16)   */

/* element types of caller inputs */
#define FD_DTYPE_F32 0
#define FD_DTYPE_F16 1
#define FD_DTYPE_BF16 2
#define FD_DTYPE_F64 3

/* tile precision of the distance GEMM */
#define FD_TILE_BF16 0  /* tcgen05 16-bit tiles, bf16 operands (wide range), fp32 accumulation */
#define FD_TILE_F32 1   /* fp32 SIMT tiles (matvec rel. L2 <= 1e-5)                           */
#define FD_TILE_F16 2   /* tcgen05 16-bit tiles, fp16 operands, fp32 accumulation: same speed
                           as bf16 with 8x finer rounding (matvec rel. L2 <= 2e-3); packing
                           records FD_ERR_RANGE in the status word when a row would overflow */
#define FD_TILE_F16X3 3 /* tcgen05 tiles of fp32-class accuracy (rel. L2 <= 1e-5): each
                           coordinate split into fp16 hi + lo and three products
                           (hi.hi + hi.lo + lo.hi) per pair; d <= 136 */

/* operand side for fd_pack_operand */
#define FD_SIDE_QUERY 0
#define FD_SIDE_KEY 1

/* Message for the last error on this host thread (never NULL). */
const char* fd_last_error(void);

/* Library version (major*10000 + minor*100 + patch). */
int fd_version(void);

/* 1 if `device` is a compute-capability 10.x (B200-class) GPU, else 0. */
int fd_device_supported(int device);

/* Read and clear the device status word written by bounded waits and by
 * fp16 packing (FD_OK, FD_ERR_TIMEOUT or FD_ERR_RANGE).  Synchronises `stream`. */
int fd_check_status(void* stream);

/* ---------------------------------------------------------------------------
 * Reference-compatible trio.  Replaces the pybind module flash_diffusion_sm100
 * (FD/csrc/flash_diffusion_sm100.cu:571-588) as used by FD/kernel_cuda_sm100.py:67-119.
 * X is (n, d) row-major of dtype FD_DTYPE_*.  `tile` selects FD_TILE_F16,
 * FD_TILE_BF16 or FD_TILE_F32.  Workspace: fd_workspace_bytes(n, n, d, 1, tile).
 * ------------------------------------------------------------------------- */

/* sq[i] = sum_k X[i,k]^2 in fp32.  Replaces compute_sq_norms
 * (FD/csrc/flash_diffusion_sm100.cu:456-476). */
int fd_compute_sq_norms(const void* X, int dtype, int64_t n, int d, float* sq, void* stream);

/* D[i] = sum_j exp(-beta ||x_i - x_j||^2) * w[j]  (w may be NULL = all ones).
 * Replaces prepass (FD/csrc/flash_diffusion_sm100.cu:478-518) and
 * prepass_rowsum (FD/kernel.py:141-182).  The reference binding also takes
 * sq_X; here squared norms are derived from the rounded tile operands so
 * that distances stay consistent, hence no sq argument. */
int fd_prepass(const void* X, int dtype, int64_t n, int d, const float* w, float beta, int tile,
               float* D, void* workspace, size_t workspace_bytes, void* stream);

/* out[i] = rscale[i] * sum_j exp(-beta ||x_i-x_j||^2) * rscale[j] * v[j].
 * Replaces matvec (FD/csrc/flash_diffusion_sm100.cu:520-569) and
 * DiffusionMap.matvec (FD/dmap.py:119-136). */
int fd_matvec(const void* X, int dtype, int64_t n, int d, const float* v, const float* rscale,
              float beta, int tile, float* out, void* workspace, size_t workspace_bytes, void* stream);

/* Workspace for fd_prepass / fd_matvec / fd_flash_diffusion. */
size_t fd_workspace_bytes(int64_t nq, int64_t nk, int d, int r, int tile);

/* General primitive FlashDiffusion(Q, K, V, beta, rscale_q, rscale_k, h)
 * (FD/kernel.py:189-257), plus an optional row divisor (the Doob row
 * normaliser Ph of FD/dmap.py:249-261).  Q (nq,d), K (nk,d) of `dtype`;
 * V (nk, r) fp32 row-major (NULL = all ones); out (nq, r) fp32.  Any of rscale_q, rscale_k, h,
 * row_div may be NULL (= ones).  The coordinates of Q and K are shifted by
 * the mean of K before rounding (the kernel is translation invariant). */
int fd_flash_diffusion(const void* Q, const void* K, int dtype, int64_t nq, int64_t nk, int d,
                       const float* V, int r, float beta, const float* rscale_q, const float* rscale_k,
                       const float* h, const float* row_div, int tile, float* out, void* workspace,
                       size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Resident-operand API: pack once, apply every solver iteration.  This is the
 * device-resident form of CUDAStateSM100 (FD/kernel_cuda_sm100.py:52-64).
 * ------------------------------------------------------------------------- */

/* Bytes of one packed operand of n points in d dims for `tile`. */
size_t fd_operand_bytes(int64_t n, int d, int tile);

/* Mean of the rows of X (n, d) into shift (d floats, device).  Used as the
 * common translation of both operands. */
int fd_mean_rows(const void* X, int dtype, int64_t n, int d, float* shift, void* stream);

/* Pack X (n,d) into a tile operand (fd_operand_bytes(n,d,tile) bytes, 256-byte
 * aligned).  `shift` (d floats, may be NULL) is subtracted first.  `side` is
 * FD_SIDE_QUERY or FD_SIDE_KEY; a query operand must be applied against a key
 * operand packed with the same beta, shift and tile. */
int fd_pack_operand(const void* X, int dtype, int64_t n, int d, const float* shift, float beta,
                    int side, int tile, void* operand, void* stream);

/* Workspace for fd_apply. */
size_t fd_apply_workspace_bytes(int64_t nq, int64_t nk, int r, int tile);

/* out = diag(row_scale / row_div) K(Q,K) diag(col_scale * col_h) V.
 * V is (nk, r) of v_dtype (FD_DTYPE_F32 or FD_DTYPE_F64; NULL = all ones), out is (nq, r) of
 * out_dtype (F32 or F64).  col_scale, col_h, row_scale, row_div may be NULL.
 * Modes of the reference map onto the pointers: prepass (V = w, rest NULL),
 * DMAP (row_scale = col_scale = rscale), AMAP (rscale_q, rscale_k), Doob
 * (col_h = h, row_div = Ph). */
int fd_apply(const void* Qop, int64_t nq, const void* Kop, int64_t nk, int d, int tile,
             const void* V, int v_dtype, int r, const float* col_scale, const float* col_h,
             const float* row_scale, const float* row_div, void* out, int out_dtype,
             void* workspace, size_t workspace_bytes, void* stream);

/* fd_apply without a workspace argument.  No counterpart in the reference.
 *
 * For callers that cannot allocate device memory or cannot pass this library
 * a device buffer: plugin / FFI hosts with no device allocator to hand over,
 * processes whose device memory belongs entirely to a fixed pool, and loops
 * that must avoid the implicit synchronisation of cudaMalloc/cudaFree.  The
 * scratch lives in one static device array of FD_NOALLOC_SCRATCH_BYTES (8 MiB)
 * inside the library, held on every GPU that loads the library until the
 * process exits.  Inputs, operands and the output are still the caller's.
 *
 * Limits: 16-bit tiles only (FD_TILE_F16 / FD_TILE_BF16) and
 * fd_apply_workspace_bytes(nq, nk, r, tile) <= FD_NOALLOC_SCRATCH_BYTES, which
 * on a 148-SM B200 means: r = 1 up to about 1.9 million keys; r = 2..16 up to
 * about 55,000 keys (the block path's cross-CTA partial sums take 4.6 MiB
 * whatever nk is); r >= 17 not supported (those partial sums alone exceed the
 * array).  Larger sizes return FD_ERR_WORKSPACE with a message naming nk, r
 * and the bytes needed, before any launch.
 * The first call on a device looks the array's device address up
 * (cudaGetSymbolAddress); make that first call before any stream capture.
 * All calls share the one array, so calls that overlap on the GPU (other
 * streams, other host threads) race on it; serialise them.  Nothing in the
 * scratch needs to start at zero.  No allocation of any kind is made. */
#define FD_NOALLOC_SCRATCH_BYTES (8u << 20)
int fd_apply_noalloc(const void* Qop, int64_t nq, const void* Kop, int64_t nk, int d, int tile,
                     const void* V, int v_dtype, int r, const float* col_scale, const float* col_h,
                     const float* row_scale, const float* row_div, void* out, int out_dtype,
                     void* stream);

/* ---------------------------------------------------------------------------
 * Lanczos vector operations (fp64, device).  Replace the host-side fp64
 * reorthogonalisation inside ARPACK that lanczos_eigsh (FD/eigensolver.py:33-85)
 * relies on; FD/eigensolver.py:17-20 states the fp64 basis requirement.
 * ------------------------------------------------------------------------- */

/* Workspace for fd_lanczos_reorth with n entries and `rows` basis rows. */
size_t fd_lanczos_workspace_bytes(int64_t n, int rows);

/* One Lanczos step's full reorthogonalisation.  V is a row-major fp64 basis
 * (row i at V + i*ldv, n entries, rows orthonormal), w the operator output
 * (overwritten).  Classical Gram-Schmidt applied twice against rows [0, rows):
 * coef[0..rows) = V w + V w1 (the projected-matrix column), coef[rows] = beta
 * = ||w2||, out (n entries; may be row `rows` of V) = w2 / beta, or zeros if
 * beta <= 1e-300 (the caller then restarts from a fresh vector).  Three passes
 * over V, fixed-order reductions (bit-reproducible), no host synchronisation.
 * 1 <= rows <= 96. */
int fd_lanczos_reorth(const double* V, int64_t ldv, int rows, int64_t n, double* w, double* out,
                      double* coef, void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Multi-GPU collective of the row-sharded operator (no counterpart in the
 * reference, which has no distributed code).  One process per GPU; rank r
 * owns contiguous row shards of Q and holds all of K; after its tile pass it
 * all-gathers the output shards over NVLink so every rank holds the whole
 * product.  NCCL is opened at run time (libnccl.so.2); without it these
 * return FD_ERR_UNSUPPORTED and the rest of the library is unaffected.
 * ------------------------------------------------------------------------- */

/* Size of the opaque rendezvous id (NCCL unique id), in bytes. */
size_t fd_comm_id_bytes(void);

/* Make a new rendezvous id on one rank (host memory of fd_comm_id_bytes());
 * the caller hands it to every rank by its own means. */
int fd_comm_get_id(void* id);

/* Join communicator `rank` of `nranks` on the current device (blocking until
 * every rank joined).  *comm receives an opaque handle. */
int fd_comm_init(void** comm, const void* id, int nranks, int rank);

/* recv[rank * bytes_per_rank ...] <- every rank's send (bytes_per_rank bytes
 * each; send may be recv's own chunk, in place), ordered on `stream`. */
int fd_comm_allgather(void* comm, const void* send, void* recv, size_t bytes_per_rank, void* stream);

/* FD_OK, or FD_ERR_CUDA if the communicator recorded an asynchronous error
 * (a peer that left, a network fault). */
int fd_comm_check(void* comm);

/* Abort (unblocks collectives in flight; for failure paths) or destroy. */
int fd_comm_abort(void* comm);
int fd_comm_destroy(void* comm);

/* ---------------------------------------------------------------------------
 * Bandwidth selection (FD/utils.py:16-52), fp32 row-major inputs, fp32 CUDA-core
 * arithmetic on coordinate differences.
 * ------------------------------------------------------------------------- */

/* out[i][0..k) = the k smallest squared distances from query row i to the key
 * rows, ascending (a query that is also a key finds itself at 0).  Replaces the
 * dense sort of knn_bandwidth, FD/utils.py:31-52 (sigma_i = sqrt(out[i][k]) with
 * k+1 columns).  1 <= k <= 64, k <= nk, 1 <= d <= 1024. */
int fd_knn_sqdist(const float* Q, int64_t nq, const float* K, int64_t nk, int d, int k, float* out,
                  void* stream);

/* Same result as fd_knn_sqdist on the tensor cores: every (query, key) pair is
 * screened with the fp32-class split operands (tcgen05, the C = k + 8 or more
 * best keys per row and key split kept), then the candidates' squared
 * distances are recomputed exactly as fd_knn_sqdist computes them (fp32
 * coordinate differences) and the k smallest written ascending.  Replaces the
 * dense sort of knn_bandwidth, FD/utils.py:31-52.  1 <= d <= 66, 1 <= k <= 24,
 * k <= nk; workspace fd_knn_tc_workspace_bytes(nq, nk, d, k) (packed operands
 * and candidates).  Synchronises `stream` once (the packing scale comes from
 * the data's largest centred norm). */
size_t fd_knn_tc_workspace_bytes(int64_t nq, int64_t nk, int d, int k);
int fd_knn_sqdist_tc(const float* Q, int64_t nq, const float* K, int64_t nk, int d, int k, float* out,
                     void* workspace, size_t workspace_bytes, void* stream);

/* out[i][j] = ||x_i - x_j||^2 for a sample of m <= 65535 rows (the median
 * heuristic, median_bandwidth, FD/utils.py:16-28). */
int fd_pairwise_sqdist(const float* X, int64_t m, int d, float* out, void* stream);

/* ---------------------------------------------------------------------------
 * RoPE-DMAP preprocessing (FD/ROPE.py:31-106,231-345).
 * ------------------------------------------------------------------------- */

/* Y (K x L*D fp32) = K windows of L samples of D features, each centred
 * ((x - mu[j]) / sigma[j], fp64), with coordinate pairs (2p, 2p+1) rotated by
 * pos * pos_scale * freqs[p] (fp64 sin/cos).  Window T, sample c, feature j is
 * read at F[T*sT + c*sC + j] and its position at pos[T*pT + c*pC]: a time series
 * (N x D) gives its K = N - (L-1) step Hankel windows with sT = D, sC = step*D,
 * pT = 1, pC = step, without copying them; a (B, L, D) window array has
 * sT = L*D, sC = D.  window_mode 0 rotates each sample by its own position;
 * window_mode 1 rotates the flattened window once by the position of sample c_w.
 * Pairs p >= n_freqs do not rotate; an odd last coordinate is copied.  Replaces
 * the host make_hankel_windows / _transform_windows chain of FD/ROPE.py. */
int fd_rope_windows(const double* F, int64_t sT, int64_t sC, const double* pos, int64_t pT, int64_t pC, int64_t K,
                    int D, int L, int window_mode, int c_w, double pos_scale, const double* freqs, int n_freqs,
                    const double* mu, const double* sigma, float* Y, void* stream);

/* Failure-path self-test (no counterpart in the reference): launches one bounded
 * device wait on a barrier that nothing arrives at, with a limit of limit_ns
 * (1e6..2e9).  The wait gives up and records FD_ERR_TIMEOUT in the status word
 * exactly as a stalled kernel pipeline would; the next fd_check_status on the
 * stream returns FD_ERR_TIMEOUT and clears it, and the context stays usable. */
int fd_selftest_wait_timeout(int64_t limit_ns, void* stream);

/* Options of the block (r > 1) tensor-core path, process-wide, for the next
 * launches (no counterpart in the reference, whose GPU path has no block
 * product).  group_tiles: key tiles summed in one tensor-core accumulator
 * before the sum moves to fp32 registers (1..64; 0 = default: 8 for the 16-bit
 * tiles, 1 for FD_TILE_F16X3).  The tensor-core accumulation rounds toward
 * zero, so fewer tiles per group give a smaller bias (about 7.5e-7 per tile of
 * group) at some speed.  products: 3 (default, P and U both split hi/lo) or 2
 * (16-bit tiles only: P rounded once to fp16; faster, 2^-12 noise per kernel
 * value).  0 restores the default.  Not thread-safe against concurrent
 * launches from other host threads. */
int fd_set_block_options(int group_tiles, int products);

/* Share of the exponentials of the 16-bit r = 1 tile kernels that runs on the
 * FMA pipe as a degree-4 polynomial (relative error below 3.7e-6) instead of
 * MUFU ex2, in columns per 16: 0, 2, 4, 6 or 8; -1 restores the default (4;
 * the fp32-class tiles always use MUFU).  Process-wide, for the next launches
 * (no counterpart in the reference, whose kernel calls expf). */
int fd_set_exp2_fma_cols(int cols);

/* Self-test of the FMA-pipe exponential (no counterpart in the reference):
 * y[i] = 2^x[i] computed exactly as the tile epilogues compute their
 * polynomial share (x clamped at -125), fp32 device arrays of length n. */
int fd_selftest_exp2_poly(const float* x, int64_t n, float* y, void* stream);

/* ---------------------------------------------------------------------------
 * Coifman-Lafon normalisation helpers (FD/dmap.py:108-115,
 * FD/kernel_cuda_sm100.py:89-98), fp32 vectors of length n.
 * ------------------------------------------------------------------------- */

/* w = D^-alpha. */
int fd_dmap_weights(const float* D, int64_t n, float alpha, float* w, void* stream);

/* D_alpha = Kw * w;  rscale = D_alpha^-1/2 * w  (Kw = prepass with weights w). */
int fd_dmap_rscale(const float* Kw, const float* w, int64_t n, float* D_alpha, float* rscale,
                   void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FD_SM100_H */
