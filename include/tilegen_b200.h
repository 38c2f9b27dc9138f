/*
 * tilegen_b200 C ABI: the int8_convrot hot path as prebuilt sm_100a kernels.
 *
 * Plain pointers and sizes only.  Every compute entry point
 *   - takes device pointers and a cudaStream_t passed as `void *stream`
 *     (NULL = the legacy default stream) and only enqueues work on it: no host
 *     synchronisation, no allocation;
 *   - returns a tg_status; nothing is launched when it is not TG_OK.
 * tg_rotate_quant, tg_quantize_act, tg_int8_gemm_dequant,
 * tg_int8_gemm_dequant_splitk and tg_int8_gemv_dequant work only on buffers
 * the caller owns, so they can be captured in CUDA graphs.
 * Device-side failures (a bounded wait that gave up) are recorded in a device
 * status word that tg_device_status() reads.
 *
 * The Python package binds these with ctypes (tilegen_b200/_lib.py).
 */
#ifndef TILEGEN_B200_H
#define TILEGEN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  TG_OK = 0,
  TG_ERR_INVALID_ARG = 1,   /* null pointer, negative size, bad dtype code */
  TG_ERR_UNSUPPORTED = 2,   /* shape/group outside what the kernel handles */
  TG_ERR_MISALIGNED = 3,    /* a pointer is not 16-byte aligned */
  TG_ERR_CUDA = 4,          /* a CUDA runtime/driver call failed (launch etc.) */
  TG_ERR_DEVICE_TIMEOUT = 5 /* tg_device_status(): a kernel's bounded wait expired */
} tg_status;

typedef enum { TG_DT_F32 = 0, TG_DT_F16 = 1, TG_DT_BF16 = 2 } tg_dtype;

/* Input activations tg_quantize_act applies before quantising (the names of
 * the reference's `input_act`, tilegen/comfyui/backend.py:174,201-204). */
typedef enum { TG_ACT_NONE = 0, TG_ACT_GELU_TANH = 1, TG_ACT_GELU = 2 } tg_act;

/* OR'ed into tg_quantize_act's `act`: evaluate the rotation in the reference
 * kernel's butterfly order (bit-identical to it) instead of the default short
 * order (see tg_rotate_quant). */
#define TG_QUANT_REFERENCE_ORDER 0x100

/* Library version, (major << 16) | minor. */
int tg_version(void);

/* Human-readable name of a tg_status value. */
const char *tg_status_string(int status);

/*
 * Fused group-Hadamard rotation + row-wise symmetric int8 quantisation.
 *
 * Replaces the reference's NVRTC kernel launch `quantize_convrot_native`
 * (tilegen/kernels/int8_convrot.py:196-230; kernel `fht_quant` at :47-104), and
 * also serves the weight side `quantize_convrot_weight`
 * (tilegen/quant/weight.py:14-39), which is the same operation on W rows.
 *
 *   x      [M, K] row-major, dtype x_dtype (TG_DT_F16 or TG_DT_BF16), 16-B aligned
 *   group  4, 16, 64 or 256 (a power of four, as tilegen/kernels/hadamard.py:18-22);
 *          K must be a multiple of 256 and at most tg_rotate_quant_max_k()
 *   q      [M, K] int8 out: clamp(rint(rot * 1/(sqrt(G)*scale)), -128, 127)
 *   scale  [M] fp32 out:   max(absmax(rot_unnormalised) / (127*sqrt(G)), 1e-30)
 * The rotation is evaluated in fp32 in a short butterfly order (each output
 * S - 2*a_i with S the sum of the butterfly's four inputs, one fma) and, for
 * rows whose rotated values are all finite, rint(rot * inv) as one fma: codes
 * may differ from the reference kernel's by one at rounding ties (about 1e-6
 * of them on DiT activations), scales by a few ulps.  tg_quantize_act with
 * TG_QUANT_REFERENCE_ORDER gives the reference kernel's bits.  bf16 is read
 * directly (the reference first casts bf16 to fp16, int8_convrot.py:204-206).
 * M == 0 is a no-op.
 */
int tg_rotate_quant(const void *x, int x_dtype, int64_t M, int64_t K, int group, int8_t *q, float *scale,
                    void *stream);

/* Largest K tg_rotate_quant and tg_quantize_act accept (a multiple of 256). */
int64_t tg_rotate_quant_max_k(void);

/*
 * tg_rotate_quant with the production wrapper's two other options fused into
 * the same pass over x (tilegen/comfyui/backend.py:166-244):
 *
 *   act    TG_ACT_NONE, TG_ACT_GELU_TANH or TG_ACT_GELU: the input activation
 *          of backend.py:201-204, applied first.  Evaluated in fp32 as torch's
 *          CUDA GELU kernels do (gelu_tanh: 0.5x(1+tanh(sqrt(2/pi)(x+0.044715x^3))),
 *          gelu: 0.5x(1+erf(x/sqrt(2)))) and rounded to x_dtype, exactly what
 *          the separate activation op would have stored for the quantiser.
 *   group  4, 16, 64 or 256: as tg_rotate_quant on act(x) (K % 256 == 0);
 *          1: no rotation, the row-wise branch of backend.py:230-232 (K % 64 == 0):
 *            scale[m] = max(absmax_m * fp32(1/127), 1e-30)   (NaN propagates)
 *            q[m,k]   = int8(clamp(rint(dtype(y[m,k] / dtype(scale[m]))), -128, 127))
 *          with y = act(x), the division in IEEE fp32, dtype() rounding to
 *          x_dtype, and NaN codes (0/0 when dtype(scale) underflows to 0 in
 *          fp16) stored as 0 -- torch's evaluation of those two lines on CUDA.
 *
 * tg_quantize_act(x, dt, M, K, G, TG_ACT_NONE, q, scale, s) runs the same
 * kernel as tg_rotate_quant(x, dt, M, K, G, q, scale, s) for G > 1.
 * TG_ERR_INVALID_ARG for an unknown act.  M == 0 is a no-op.
 */
int tg_quantize_act(const void *x, int x_dtype, int64_t M, int64_t K, int group, int act, int8_t *q, float *scale,
                    void *stream);

/*
 * The rotated quantiser with the DiT block's normalisation in front of it, in
 * the same pass over x: for row m and v = m / mod_rows,
 *   y[m,:] = LayerNorm(x[m,:]) * (1 + mod_scale[v,:]) + mod_shift[v,:]
 * (LayerNorm without affine, epsilon `eps`), then tg_rotate_quant on y.  The
 * normalised row, the product and the sum are each rounded to x_dtype, as the
 * separate torch ops would store them; the row mean and variance are fp32 sums
 * in a fixed order, rstd = 1 / sqrt(var + eps).  The reference's path starts at
 * int8_linear's input, so this has no reference counterpart: it removes the
 * write and re-read of the modulated activations between the block's
 * normalisation and its projection.
 *
 *   x                   [M, K] fp16/bf16, 16-B aligned; K % 256 == 0
 *   group               4, 16, 64 or 256 (rotated; the short butterfly order)
 *   mod_scale/mod_shift [ceil(M / mod_rows), K] of x_dtype, 16-B aligned
 *   mod_rows            rows per modulation vector (>= 1; M for one vector)
 *   q, scale            as tg_rotate_quant
 * TG_ERR_INVALID_ARG for eps < 0, NaN or inf, mod_rows < 1; M == 0 is a no-op.
 */
int tg_quantize_ln_mod(const void *x, int x_dtype, int64_t M, int64_t K, int group, float eps,
                       const void *mod_scale, const void *mod_shift, int64_t mod_rows, int8_t *q, float *scale,
                       void *stream);

/*
 * INT8 GEMM with the dequantisation fused into the epilogue (tcgen05 kind::i8,
 * int32 accumulators in tensor memory).
 *
 * Replaces `int8_matmul_dequant_chunked` (tilegen/quant/int8_ops.py:22-70):
 *   acc[m,n] = sum_k xq[m,k] * wq[n,k]                    (exact int32)
 *   out[m,n] = ((float(acc) * xscale[m]) * wscale[n]) + bias[n]
 * in fp32 with one rounding per operation (no FMA), stored as out_dtype with
 * round-to-nearest-even: bit-identical to the reference's torch sequence.
 *
 *   xq [M, K] int8, wq [N, K] int8 (both K-major, 16-B aligned; K % 16 == 0)
 *   xscale [M] fp32; wscale fp32 of wscale_numel = 1 (broadcast) or N
 *   bias [N] of bias_dtype (TG_DT_F32/F16/BF16) or NULL
 *   out [M, N] of out_dtype (TG_DT_F32/F16/BF16); N*sizeof(out) % 16 == 0
 * M == 0 is a no-op.  No temporary memory is used, so the reference's chunking
 * argument has nothing to bound.
 */
int tg_int8_gemm_dequant(const int8_t *xq, const float *xscale, const int8_t *wq, const float *wscale,
                         int64_t wscale_numel, const void *bias, int bias_dtype, int64_t M, int64_t N,
                         int64_t K, int out_dtype, void *out, void *stream);

/*
 * The same GEMM + dequantisation for few activation rows (1 <= M <= 128, decode
 * and preview steps), bit-identical to tg_int8_gemm_dequant.  Also replaces
 * `int8_matmul_dequant_chunked` (tilegen/quant/int8_ops.py:22-70), whose GEMM
 * at small M is whatever torch._int_mm does.  The weight streams through all
 * SMs: K is split across the CTAs of each 128-column tile, whose exact int32
 * partial sums are added either in shared memory (the tile's CTAs run as one
 * thread-block cluster: K split at most 8 ways; the workspace is then not
 * touched) or in the workspace, where the last CTA of the tile dequantises
 * (tg_int8_gemm_dequant_splitk_config tells which).
 *
 * Arguments as tg_int8_gemm_dequant (M > 128 gives TG_ERR_UNSUPPORTED), plus:
 *   workspace  tg_int8_gemm_dequant_splitk_workspace(M, N) bytes, 256-byte
 *              aligned, ZERO-FILLED before its first use; every call leaves it
 *              zero again (also one whose wait expired), so it needs no
 *              clearing between calls.  Calls that share a workspace must not
 *              overlap on the GPU.
 */
int tg_int8_gemm_dequant_splitk(const int8_t *xq, const float *xscale, const int8_t *wq, const float *wscale,
                                int64_t wscale_numel, const void *bias, int bias_dtype, int64_t M, int64_t N,
                                int64_t K, int out_dtype, void *out, void *workspace, size_t workspace_bytes,
                                void *stream);

/* Workspace bytes tg_int8_gemm_dequant_splitk needs for an M x N output. */
size_t tg_int8_gemm_dequant_splitk_workspace(int64_t M, int64_t N);

/* Largest M tg_int8_gemm_dequant_splitk accepts (128). */
int64_t tg_int8_gemm_dequant_splitk_max_m(void);

/*
 * How tg_int8_gemm_dequant_splitk runs an M x N x K problem with this output
 * dtype and bias presence on the current device: *slices = CTAs that split the
 * K of each 128-column tile; *cluster = 1 when they run as one thread-block
 * cluster and reduce in shared memory, 0 when they reduce through the
 * workspace.  No reference counterpart (for tests and tuning).
 */
int tg_int8_gemm_dequant_splitk_config(int64_t M, int64_t N, int64_t K, int out_dtype, int has_bias, int *slices,
                                       int *cluster);

/* Largest M tg_int8_gemv_dequant accepts. */
#define TG_GEMV_MAX_M 4

/*
 * The same GEMM + dequantisation for one to four activation rows, on the CUDA
 * cores: each warp streams four weight rows (over one part of K) with 128-bit
 * loads and sums exact int32 dp4a products; a quarter of the weight is asked
 * into L2 before the wait for the kernel that wrote xq, so the weight stream
 * starts while that kernel runs.
 * Bit-identical to tg_int8_gemm_dequant.  Replaces the reference's
 * `int8_matmul_dequant_chunked` (tilegen/quant/int8_ops.py:22-70) at these M,
 * where its GEMM is torch._int_mm's.  No workspace and no allocation.
 *
 * Arguments as tg_int8_gemm_dequant; TG_ERR_UNSUPPORTED for M > TG_GEMV_MAX_M.
 */
int tg_int8_gemv_dequant(const int8_t *xq, const float *xscale, const int8_t *wq, const float *wscale,
                         int64_t wscale_numel, const void *bias, int bias_dtype, int64_t M, int64_t N, int64_t K,
                         int out_dtype, void *out, void *stream);

/*
 * How tg_int8_gemv_dequant runs an N x K weight on the current device:
 * *parts = warps that split the K of each group of four weight rows (1, 2, 4
 * or 8), *ctas = its grid.  No reference counterpart (for tests and tuning).
 */
int tg_int8_gemv_dequant_config(int64_t N, int64_t K, int *parts, int *ctas);

/*
 * tg_int8_gemm_dequant_splitk for callers that cannot allocate device memory:
 * a plugin running inside a host application that owns all GPU memory through
 * its own allocator, or a serving process whose memory is fully reserved up
 * front, where a cudaMalloc would fail or stall the device.  It takes no
 * workspace: its scratch is a fixed array inside the library (4 MiB + 2 KiB on
 * every GPU that loads it, held until the process exits).  No counterpart in
 * the reference.
 *
 * Arguments and result as tg_int8_gemm_dequant_splitk without the workspace;
 * TG_ERR_UNSUPPORTED unless M <= 64, N <= 65536 and M * N <= 1048576.
 * The first call on a device looks up the array's device address (set-up, once
 * per device); make that first call before any stream capture.  When the
 * kernel sums through the array (tg_int8_gemm_dequant_splitk_config reports
 * cluster == 0), the call first zeroes the part of the array it uses (a memset
 * on `stream`); the cluster form sums in shared memory and leaves the array
 * alone.  All calls share the one array, so calls that overlap on the GPU
 * (different streams, or concurrent host threads) race and corrupt each
 * other's results: serialise them.
 */
int tg_int8_gemm_dequant_splitk_noalloc(const int8_t *xq, const float *xscale, const int8_t *wq,
                                        const float *wscale, int64_t wscale_numel, const void *bias, int bias_dtype,
                                        int64_t M, int64_t N, int64_t K, int out_dtype, void *out, void *stream);

/*
 * The tile shape tg_int8_gemm_dequant uses for an M x N problem on the
 * current device: *bn = tile width (UMMA N: 256, 224, 192, 160 or 128) and
 * *pair = 1 when the tile is 256 rows computed by a pair of SMs (tcgen05
 * cta_group::2), 0 for 128-row single-SM tiles.  The width minimises
 * (persistent waves) x (tile cost).  No reference counterpart (cuBLASLt chose
 * its own tiles).
 */
int tg_gemm_config(int64_t M, int64_t N, int *bn, int *pair);

/*
 * Force the GEMM tile shape for every later call in this process: bn 0 or one
 * of the widths above, pair -1 (automatic), 0 or 1.  For tests and tuning;
 * TG_ERR_INVALID_ARG for anything else.
 */
int tg_set_gemm_config(int bn, int pair);

/*
 * Cap the SMs the persistent kernels (tg_rotate_quant / tg_quantize_act and
 * tg_int8_gemm_dequant) size their grids for, in every later call of this
 * process: sms = 0 lifts the cap.  They normally take every SM, so a kernel
 * running at the same time on another stream (an NCCL collective, say) that
 * holds even one SM keeps part of their grid from starting until it ends;
 * with the SMs that kernel needs left out, both run at once.  No reference
 * counterpart.  TG_ERR_INVALID_ARG for sms < 0.
 */
int tg_set_sm_budget(int sms);

/* The current cap (0 = none). */
int tg_sm_budget(void);

/*
 * Read (and optionally clear) the device status word of `device`, which
 * kernels set when a bounded wait expires.  Synchronises the device.
 * *bits receives the raw word (0 = healthy); returns TG_ERR_DEVICE_TIMEOUT when
 * it is non-zero, TG_OK otherwise.
 */
int tg_device_status(int device, uint32_t *bits, int clear);

/*
 * Peer memory for the optional output all-gather of a row-sharded linear (one
 * process per GPU on one node).  No reference counterpart: the reference runs
 * on one GPU.
 *
 * tg_peer_alloc: `bytes` of device memory on the current device (cudaMalloc)
 *   and its interprocess handle, tg_peer_handle_bytes() bytes written to
 *   `handle`; free with tg_peer_free.
 * tg_peer_open: map another process's buffer from its handle into the current
 *   device's address space (peer access enabled on demand); *ptr is usable as
 *   a device pointer in copies.  A process cannot open its own handles.  Unmap
 *   with tg_peer_close.
 * tg_copy_async: enqueue a copy of `bytes` between device pointers (local or
 *   mapped peer memory) on `stream`; between GPUs it runs on a copy engine over
 *   NVLink and uses no SMs.
 */
size_t tg_peer_handle_bytes(void);
int tg_peer_alloc(size_t bytes, void **ptr, void *handle);
int tg_peer_free(void *ptr);
int tg_peer_open(const void *handle, void **ptr);
int tg_peer_close(void *ptr);
int tg_copy_async(void *dst, const void *src, size_t bytes, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* TILEGEN_B200_H */
