/*
 * qwantize_b200.h -- C ABI of the B200 (sm_100a) block-scale quantization
 * library libqwantize_b200.so.
 *
 * The reference (qwantize v0.1.2) is a pure-Python package with no FFI; each
 * entry point below replaces the functions of its Python API named beside it
 * (paths relative to the qwantize project root).  The Python package
 * qwantize_b200 binds them with ctypes and keeps the reference's function
 * names, keyword arguments, returned tuples and AssertionError behaviour.
 *
 * Conventions
 *   - Pointers are device pointers unless stated otherwise.  Inputs are never
 *     modified.  A NULL output pointer means "do not write it".
 *   - Every call is asynchronous on `stream` (a cudaStream_t; NULL = legacy
 *     default stream) and returns a status code; qz_last_error() returns a
 *     message for the last non-zero status of the calling thread.
 *   - Blocked layout: `n_blocks` contiguous blocks of `block_size` (16 or 32)
 *     elements, i.e. the reference's W.movedim(dim, -1).reshape(-1, bs).
 *   - Naive and SSE results are bit-identical to the reference's pure-PyTorch
 *     CPU path for bf16 and fp16 inputs (signed zeros and NaN bit patterns
 *     included).
 */
#ifndef QWANTIZE_B200_H
#define QWANTIZE_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define QZ_API __attribute__((visibility("default")))
#else
#define QZ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define QZ_OK 0
#define QZ_ERR_INVALID 1     /* bad argument (Python raises AssertionError / ValueError) */
#define QZ_ERR_CUDA 2        /* CUDA runtime / driver error */
#define QZ_ERR_TIMEOUT 3     /* a bounded device-side wait gave up */
#define QZ_ERR_UNSUPPORTED 4 /* device is not sm_100 */

/* element types */
#define QZ_DTYPE_F32 0
#define QZ_DTYPE_BF16 1
#define QZ_DTYPE_F16 2

/* formats */
#define QZ_FMT_NVFP4 0 /* E2M1 codes, FP8-E4M3 scale per block (126 positive values) */
#define QZ_FMT_MXFP4 1 /* E2M1 codes, UE8M0 power-of-two scale per block (254 values) */
/* 2 is the caller-supplied scale table of qz_quantize_table */
#define QZ_FMT_NVINT4 3 /* int codes in [-7, 7], FP8-E4M3 scale per block; block 16 or 32
                           (nvint4/reference.py:55-308) */
#define QZ_FMT_INT8 4   /* int codes in [-127, 127], scale = E4M3 value / 127; block 32, 64,
                           128 or 256 (int8/reference.py:87-389) */

/* scale-selection methods */
#define QZ_METHOD_NAIVE 0        /* nvfp4/reference.py:89-126, mxfp4/reference.py:89-129 */
#define QZ_METHOD_SSE 1          /* nvfp4/reference.py:129-239, mxfp4/reference.py:132-238 */
#define QZ_METHOD_HESSIAN 2      /* nvfp4/reference.py:266-407, mxfp4/reference.py:241-374 */
#define QZ_METHOD_NAIVE_ARGMIN 3 /* mxfp4/kernels.py:267-314 mxfp4_naive_torch */
#define QZ_METHOD_TWO_ARGMIN 4   /* mxfp4/kernels.py:317-377 mxfp4_optimal_torch */

/* Gram modes */
#define QZ_GRAM_FULL 0      /* H = X^T X, (K, K) fp32, symmetric */
#define QZ_GRAM_BLOCKDIAG 1 /* H_j = X_j^T X_j, (K/bs, bs, bs) fp32 */
#define QZ_GRAM_FULL_UPPER_TILES 2 /* the 256 x 256 tiles of X^T X on and above the diagonal, packed */

/*
 * qz_quantize -- per-block scale selection + E2M1 quantization in one pass.
 * Replaces nvfp4_naive / nvfp4_optimal / nvfp4_optimal_hessian and the
 * *_triton variants (nvfp4/reference.py:89-407, nvfp4/kernels.py:248-427),
 * mxfp4_naive / mxfp4_optimal / mxfp4_optimal_hessian / *_triton / *_torch
 * (mxfp4/reference.py:89-374, mxfp4/kernels.py:164-377).
 *   x           n_blocks*block_size elements of x_dtype, 16-byte aligned
 *   h_blocks    (n_col_blocks, bs, bs) fp32 block Hessians for
 *               QZ_METHOD_HESSIAN (block b uses h_blocks[b % n_col_blocks])
 *   scales      (n_blocks) fp32 chosen scales (the reference's `scales`)
 *   quants      (n_blocks*bs) fp32 signed codebook values (`quants`)
 *   dq          (n_blocks*bs) fp32 quants*scales (the dequant)
 *   scale_codes (n_blocks) E4M3 byte (NVFP4) or UE8M0 biased exponent (MXFP4)
 *   packed      (n_blocks*bs/2) E2M1 nibbles; element 2i in the low nibble of
 *               byte i, bit 3 = sign (the layout fp4.py:117-282 decodes)
 *   dq_bf16     (n_blocks*bs) bf16 dequant (exact: dequant values fit bf16)
 * The integer formats (QZ_FMT_NVINT4, QZ_FMT_INT8; methods NAIVE, SSE and
 * HESSIAN) write `quants` as the integer values, `scale_codes` as the E4M3
 * byte of the scale (NVINT4) or of 127 * scale (INT8), `packed` as two's
 * complement nibbles, element 2i in the low nibble of byte i (NVINT4,
 * n_blocks*bs/2 bytes) or one int8 per element (INT8, n_blocks*bs bytes), with
 * 0x8 / 0x80 marking a NaN quant, and `dq_bf16` rounded to nearest (INT8
 * dequant values need not fit bf16).  Their quants / dq / dq_bf16 and packed
 * outputs must be 16-byte aligned (NVINT4 at block 16: packed 8-byte aligned).
 */
QZ_API int qz_quantize(const void* x, int x_dtype, int64_t n_blocks, int block_size, int format,
                int method, const float* h_blocks, int64_t n_col_blocks, float* scales,
                float* quants, float* dq, uint8_t* scale_codes, uint8_t* packed,
                uint16_t* dq_bf16, void* stream);

/*
 * qz_quantize_grouped -- qz_quantize (NVFP4 / MXFP4, methods NAIVE and SSE)
 * over many inputs in one persistent launch per 256 inputs.  Replaces the
 * reference's row-chunked caller loops, which call one quantization function
 * per matrix or row range (experiments/quant_bench.py:107-117,
 * bench/full_bench.py:54-89): the chunks of 32 blocks of all inputs form one
 * work list, so small inputs (one GPU's row shard of a k_proj, say) share the
 * GPU instead of each launch filling a fraction of a wave.
 *   items    host array of n_items descriptors (read during the call only);
 *            each input and its outputs follow qz_quantize's rules (x and the
 *            fp32 / bf16 outputs 16-byte aligned, packed 8 / 16-byte aligned,
 *            NULL outputs skipped); all items share dtype, block size, format
 *            and method.  Results are bit-identical to one qz_quantize per item.
 */
typedef struct QzQuantItem {
  const void* x;
  int64_t n_blocks;
  float* scales;
  float* quants;
  float* dq;
  uint8_t* scale_codes;
  uint8_t* packed;
  uint16_t* dq_bf16;
} QzQuantItem;

QZ_API int qz_quantize_grouped(const QzQuantItem* items, int n_items, int x_dtype, int block_size, int format,
                               int method, void* stream);

/*
 * qz_quantize_table -- qz_quantize with a caller-supplied scale grid: `table`
 * is a device array of n_table (2..256) ascending positive fp32 scales, e.g.
 * the unsigned 8-bit UE4M4 / UE5M3 grids of exotic_scales.py:17-57.  Follows
 * the exotic-grid experiment (experiments/quant_exotic_scales.py:48-182): the
 * naive scale is snap_to_table(max|x| / 6) (exotic_scales.py:60-74), the
 * searches run over the table with the NVFP4 rules.  scale_codes receive the
 * table index.  Methods: naive, SSE, Hessian.
 */
QZ_API int qz_quantize_table(const void* x, int x_dtype, int64_t n_blocks, int block_size, int method,
                             const float* table, int n_table, const float* h_blocks, int64_t n_col_blocks,
                             float* scales, float* quants, float* dq, uint8_t* scale_codes, uint8_t* packed,
                             uint16_t* dq_bf16, void* stream);

/*
 * qz_admm -- ADMM refinement of NVFP4 codes and scales under block Hessians.
 * Replaces the iteration of nvfp4_admm (nvfp4/reference.py:466-534): from the
 * naive E4M3 scale, n_outer rounds of (n_inner ADMM steps projecting onto the
 * E2M1 codebook, then s = E4M3(x^T H q / q^T H q)).  The caller supplies, per
 * column block j, H_j, H_j / lambda_max(H_j) and inv(H_j / lambda_max + rho I)
 * (each (n_col_blocks, bs, bs) fp32; block b uses j = b % n_col_blocks).
 * quants / packed hold the ADMM codes; outputs as in qz_quantize.
 */
QZ_API int qz_admm(const void* x, int x_dtype, int64_t n_blocks, int block_size, const float* h_blocks,
                   const float* hn_blocks, const float* minv_blocks, int64_t n_col_blocks, int n_outer,
                   int n_inner, float rho, float* scales, float* quants, float* dq, uint8_t* scale_codes,
                   uint8_t* packed, uint16_t* dq_bf16, void* stream);

/*
 * qz_dequantize -- out = quants * scales per block.  Replaces nvfp4_dequantize
 * (nvfp4/reference.py:537-549) and mxfp4_dequantize (mxfp4/reference.py:377-389)
 * in the blocked layout.
 */
QZ_API int qz_dequantize(const float* scales, const float* quants, int64_t n_blocks, int block_size,
                  float* out, void* stream);

/*
 * qz_dequantize_packed -- packed E2M1 nibbles + scale bytes -> fp32 and/or
 * bf16.  Native-storage counterpart of qz_dequantize (the reference keeps fp32
 * only; its byte scales are s.to(float8_e4m3fn) in
 * bench/nvfp4_scale_distance.py:20-22 and scales_to_ue8m0_exponent in
 * mxfp4/reference.py:392-403).
 */
QZ_API int qz_dequantize_packed(const uint8_t* packed, const uint8_t* scale_codes, int64_t n_blocks,
                         int block_size, int format, float* out_f32, uint16_t* out_bf16,
                         void* stream);

/*
 * qz_fp4_unpack -- packed nibbles -> int8 values of the doubled codebook
 * {0,1,2,3,4,6,8,12} with sign.  Replaces fp4_unpack (fp4.py:257-282);
 * n_bytes must be a multiple of 4 (fp4.py:273).
 */
QZ_API int qz_fp4_unpack(const uint8_t* packed, int64_t n_bytes, int8_t* out, void* stream);

/*
 * qz_gram -- H = X^T X in fp32 from bf16 X (T, K) row-major, on the tcgen05
 * tensor cores.  Replaces the block-Hessian build of nvfp4/reference.py:304-317
 * (also nvfp4/kernels.py:386-397, mxfp4/reference.py:271-284).
 * QZ_GRAM_FULL writes the symmetric (K, K) matrix; QZ_GRAM_BLOCKDIAG writes
 * (K/bs, bs, bs).  accumulate != 0 adds into H instead of overwriting it.
 * QZ_GRAM_FULL_UPPER_TILES writes only the t(t+1)/2 tiles of 256 x 256 on and
 * above the diagonal (t = ceil(K / 256)) into H, t(t+1)/2 * 65536 floats:
 * tile (mi, nj >= mi) at index mi*t - mi*(mi-1)/2 + (nj - mi), each tile
 * column-major (element (r, c) at c*256 + r), entries beyond K zero.  It is
 * about half of the full matrix, so a token-sharded Gram all-reduces it and
 * expands it with qz_gram_unpack (same sums, bit for bit, as QZ_GRAM_FULL).
 */
QZ_API int qz_gram(const uint16_t* X, int64_t T, int64_t K, int mode, int block_size, int accumulate,
            float* H, void* stream);

/*
 * qz_gram_unpack -- the symmetric (K, K) H from the packed upper tiles of
 * qz_gram (QZ_GRAM_FULL_UPPER_TILES).  Added beside the reference's Hessian
 * build (nvfp4/reference.py:304-317) for the token-sharded all-reduce.
 */
QZ_API int qz_gram_unpack(const float* packed, int64_t K, float* H, void* stream);

/*
 * qz_gram_full_noalloc -- the full Gram H = X^T X of qz_gram (QZ_GRAM_FULL),
 * for callers that must not allocate device memory during the call, e.g. code
 * running inside a framework's own memory pool or allocator hook, or a host
 * program that has handed all device memory to another component.  qz_gram
 * allocates a small per-call counter buffer (cudaMallocAsync); this entry point
 * keeps those counters in a fixed 256 KB device array inside the library
 * instead, so it calls no allocator at all.  No counterpart in the reference.
 *   - Limit: at most 65,536 output tiles of 256 x 256, i.e. K <= 92416; larger
 *     K is rejected with QZ_ERR_INVALID before any device work.
 *   - The first call on each device looks up the array's device address
 *     (cudaGetSymbolAddress); make that first call before any stream capture.
 *   - All calls share the one array (zeroed at the start of each call): calls
 *     that can overlap on the GPU, on any stream, race and must be serialised.
 *   - Every GPU that loads the library keeps the array until the process exits.
 */
QZ_API int qz_gram_full_noalloc(const uint16_t* X, int64_t T, int64_t K, int accumulate, float* H,
                                void* stream);

/*
 * qz_gptq -- GPTQ error compensation over all column blocks (replaces the
 * loop of gptq_strided, experiments/quant_gptq_strided.py:49-135; the damped
 * inverse Hessian Hi of :72-85 is the caller's input).  Column groups of
 * group_cols (32, 64 or 128) columns run left to right: one kernel carries
 * every row through the group's blocks (scale search by `method` as in
 * qz_quantize on fp32 input, error d / Hi_cc, in-group update), then a
 * tcgen05 GEMM subtracts E @ Hi[group, later columns] from the later columns,
 * at fp32 accuracy (tf32 high / low operand pairs, three products).
 *   Wb        (K/bs, M, bs) fp32 working weight, column-block-major, updated
 *   Qb        (K/bs, M, bs) fp32 dequantized result
 *   Hi        (K, K) fp32 damped inverse Hessian; Hi_split 2*K*K fp32 scratch
 *   h_blocks  (K/bs, bs, bs) block Hessians for QZ_METHOD_HESSIAN, else NULL
 *   E         M * 2 * group_cols fp32 scratch
 *   loss      ceil(K / group_cols) * ceil(M / 8) doubles: sum of d^2 / Hi_cc
 *             per (group, 8-row slice); the reference's loss is their sum / M
 */
QZ_API int qz_gptq(float* Wb, float* Qb, const float* Hi, float* Hi_split, const float* h_blocks, int64_t M,
                   int64_t K, int block_size, int format, int method, int group_cols, float* E, double* loss,
                   void* stream);

/*
 * qz_spd_inverse -- in-place inverse of a symmetric positive definite fp32
 * matrix A (n x n, row-major, n a multiple of 32): the damped inverse Hessian
 * of GPTQ (experiments/quant_gptq_strided.py:72-85 takes it through
 * torch.linalg.cholesky + cholesky_inverse).  Recursive 2 x 2 blocking on
 * Schur complements; every product on the tensor cores at fp32 accuracy (tf32
 * high / low operand pairs), blocks of at most 128 inverted in double
 * precision.  work: 11 * n * n floats of scratch.  *status (device int) is set
 * to 1 if a pivot was not positive (A not positive definite; the result is
 * then not an inverse), else 0.
 */
QZ_API int qz_spd_inverse(float* A, int64_t n, float* work, int* status, void* stream);

/*
 * qz_weight_error_sums -- sums[0] += sum (W_dq - W)^2, sums[1] += sum W^2 in
 * double (metrics.py:23-27).  W and W_dq are n elements of w_dtype / dq_dtype.
 */
QZ_API int qz_weight_error_sums(const void* W, int w_dtype, const void* W_dq, int dq_dtype, int64_t n,
                         double* sums, void* stream);

/*
 * qz_output_error_sums -- sums[0] += sum ((X W_dq^T) - (X W^T))^2 and
 * sums[1] += sum (X W^T)^2 (metrics.py:29-50), one tcgen05 GEMM pass over
 * bf16 X (T, K) against bf16 W and W_dq (M, K) with the reduction fused into
 * the epilogue (the T x M products are never written).
 */
QZ_API int qz_output_error_sums(const uint16_t* X, int64_t T, int64_t K, const uint16_t* W,
                         const uint16_t* W_dq, int64_t M, double* sums, void* stream);

/*
 * qz_poll_device_error -- reads (and with clear != 0 resets) the flags that
 * bounded device-side waits set when they give up (bit 0: bulk-load wait,
 * bit 1: tensor-core pipeline wait, bit 2: epilogue wait).  Synchronous.
 * Returns QZ_ERR_TIMEOUT if any flag was set.  (No counterpart in the
 * reference, whose kernels have no device-side waits.)
 */
QZ_API int qz_poll_device_error(int clear, unsigned* flags_out);

/*
 * qz_selftest_wait -- exercises the bounded device-side wait that every kernel
 * of this library uses: one warp waits on an mbarrier that nothing arrives
 * on, gives up after limit_ns (at most 1e9), records bit 0 of the device error
 * flags and returns.  Afterwards qz_poll_device_error reports QZ_ERR_TIMEOUT
 * and the context stays usable.  For tests of the failure path; no
 * counterpart in the reference, whose kernels have no device-side waits.
 */
QZ_API int qz_selftest_wait(uint64_t limit_ns, void* stream);

/* Host helpers. */
QZ_API int qz_scale_table(int format, float* out_host, int* n_out); /* 126 / 254 ascending values */
QZ_API const char* qz_last_error(void);
QZ_API int qz_version(void);
QZ_API int qz_device_ok(void); /* QZ_OK if the current device is sm_100 */

#ifdef __cplusplus
}
#endif

#endif /* QWANTIZE_B200_H */
