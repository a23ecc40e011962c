// qz_abi.cu -- the extern "C" entry points declared in include/qwantize_b200.h:
// argument validation, status codes, per-thread error messages, dispatch.
#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/qwantize_b200.h"
#include "qz_kernels.h"

namespace qz {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return QZ_OK;
  return fail(QZ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// SM count of the current device (cached per device).
int current_sms(int* sms) {
  static int cache[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(QZ_ERR_INVALID, "device index %d out of range", dev);
  if (cache[dev] == 0) {
    int major = 0, n = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (major != 10) return fail(QZ_ERR_UNSUPPORTED, "device %d is sm_%d0, this library targets sm_100a", dev, major);
    cache[dev] = n;
  }
  *sms = cache[dev];
  return QZ_OK;
}

static bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

}  // namespace qz

using namespace qz;

extern "C" {

const char* qz_last_error(void) { return g_last_error.c_str(); }

int qz_version(void) { return 100; }

int qz_poll_device_error(int clear, unsigned* flags_out) {
  unsigned f = 0, g = 0;
  int st = cuda_status(read_device_error_quantize(&f, clear != 0), "qz_poll_device_error");
  if (st == QZ_OK) st = cuda_status(read_device_error_gemm(&g, clear != 0), "qz_poll_device_error");
  f |= g;
  g = 0;
  if (st == QZ_OK) st = cuda_status(read_device_error_int(&g, clear != 0), "qz_poll_device_error");
  f |= g;
  if (flags_out) *flags_out = f;
  if (st != QZ_OK) return st;
  if (f) return fail(QZ_ERR_TIMEOUT, "a device-side wait gave up (flags 0x%x)", f);
  return QZ_OK;
}

int qz_selftest_wait(uint64_t limit_ns, void* stream) {
  if (limit_ns > 1000000000ull) return fail(QZ_ERR_INVALID, "limit_ns must be at most 1e9 (one second)");
  int sms = 0;
  int st = current_sms(&sms);
  if (st != QZ_OK) return st;
  return cuda_status(launch_wait_selftest(limit_ns, static_cast<cudaStream_t>(stream)), "qz_selftest_wait launch");
}

int qz_device_ok(void) {
  int sms = 0;
  return current_sms(&sms);
}

int qz_scale_table(int format, float* out_host, int* n_out) {
  if (!out_host || !n_out) return fail(QZ_ERR_INVALID, "qz_scale_table: NULL output");
  if (format == QZ_FMT_NVFP4 || format == QZ_FMT_NVINT4 || format == QZ_FMT_INT8) {
    int n = 0;
    for (int c = 1; c < 0x7f; ++c) {
      int e = c >> 3, m = c & 7;
      const float v = e == 0 ? (float)m / 512.0f : ldexpf(1.0f + m / 8.0f, e - 7);
      // INT8: the effective scales E4M3 / 127 (int8/reference.py:151-152), IEEE division
      out_host[n++] = format == QZ_FMT_INT8 ? v / 127.0f : v;
    }
    *n_out = n;
    return QZ_OK;
  }
  if (format == QZ_FMT_MXFP4) {
    for (int e = 1; e <= 254; ++e) out_host[e - 1] = ldexpf(1.0f, e - 127);
    *n_out = 254;
    return QZ_OK;
  }
  return fail(QZ_ERR_INVALID, "qz_scale_table: unknown format %d", format);
}

// NVINT4 / INT8 (qz_int.cu): validation and launch.
static int quantize_int(const void* x, int x_dtype, int64_t n_blocks, int block_size, int format, int method,
                        const float* h_blocks, int64_t n_col_blocks, float* scales, float* quants, float* dq,
                        uint8_t* scale_codes, uint8_t* packed, uint16_t* dq_bf16, void* stream) {
  if (format == QZ_FMT_NVINT4 && block_size != 16 && block_size != 32)
    return fail(QZ_ERR_INVALID, "block_size=%d, expected one of (16, 32)", block_size);
  if (format == QZ_FMT_INT8 && block_size != 32 && block_size != 64 && block_size != 128 && block_size != 256)
    return fail(QZ_ERR_INVALID, "block_size=%d, expected one of (32, 64, 128, 256)", block_size);
  if (method != QZ_METHOD_NAIVE && method != QZ_METHOD_SSE && method != QZ_METHOD_HESSIAN)
    return fail(QZ_ERR_INVALID, "the integer formats support the naive, SSE and Hessian methods, got %d", method);
  if (x_dtype != QZ_DTYPE_F32 && x_dtype != QZ_DTYPE_BF16 && x_dtype != QZ_DTYPE_F16)
    return fail(QZ_ERR_INVALID, "unknown dtype %d", x_dtype);
  if (n_blocks < 0) return fail(QZ_ERR_INVALID, "n_blocks must be >= 0");
  if (n_blocks == 0) return QZ_OK;
  if (!x || !aligned(x, 16)) return fail(QZ_ERR_INVALID, "x must be non-NULL and 16-byte aligned");
  if ((quants && !aligned(quants, 16)) || (dq && !aligned(dq, 16)) || (dq_bf16 && !aligned(dq_bf16, 16)) ||
      (packed && !aligned(packed, format == QZ_FMT_NVINT4 && block_size == 16 ? 8 : 16)))
    return fail(QZ_ERR_INVALID, "quants/dq/dq_bf16 must be 16-byte aligned, packed 8/16-byte aligned");
  if (method == QZ_METHOD_HESSIAN) {
    if (!h_blocks) return fail(QZ_ERR_INVALID, "X or H_blocks required");
    if (n_col_blocks <= 0 || n_blocks % n_col_blocks != 0 || n_col_blocks > 2147483647LL)
      return fail(QZ_ERR_INVALID, "n_blocks (%lld) must be a multiple of n_col_blocks (%lld)",
                  (long long)n_blocks, (long long)n_col_blocks);
    if (!aligned(h_blocks, 16)) return fail(QZ_ERR_INVALID, "h_blocks must be 16-byte aligned");
  }
  int sms = 0;
  int st = current_sms(&sms);
  if (st != QZ_OK) return st;
  QuantArgs p{x, n_blocks, h_blocks, n_col_blocks, scales, quants, dq, scale_codes, packed, dq_bf16};
  return cuda_status(launch_quantize_int(p, x_dtype, block_size, format, method, sms,
                                         static_cast<cudaStream_t>(stream)),
                     "qz_quantize launch (integer format)");
}

int qz_quantize(const void* x, int x_dtype, int64_t n_blocks, int block_size, int format,
                int method, const float* h_blocks, int64_t n_col_blocks, float* scales,
                float* quants, float* dq, uint8_t* scale_codes, uint8_t* packed,
                uint16_t* dq_bf16, void* stream) {
  if (format == QZ_FMT_NVINT4 || format == QZ_FMT_INT8)
    return quantize_int(x, x_dtype, n_blocks, block_size, format, method, h_blocks, n_col_blocks, scales, quants,
                        dq, scale_codes, packed, dq_bf16, stream);
  if (block_size != 16 && block_size != 32)
    return fail(QZ_ERR_INVALID, "block_size must be 16 or 32, got %d", block_size);
  if (format != QZ_FMT_NVFP4 && format != QZ_FMT_MXFP4)
    return fail(QZ_ERR_INVALID, "unknown format %d", format);
  if (method < QZ_METHOD_NAIVE || method > QZ_METHOD_TWO_ARGMIN)
    return fail(QZ_ERR_INVALID, "unknown method %d", method);
  if (method >= QZ_METHOD_NAIVE_ARGMIN && format != QZ_FMT_MXFP4)
    return fail(QZ_ERR_INVALID, "the argmin methods (mxfp4_*_torch) are MXFP4 only");
  if (x_dtype != QZ_DTYPE_F32 && x_dtype != QZ_DTYPE_BF16 && x_dtype != QZ_DTYPE_F16)
    return fail(QZ_ERR_INVALID, "unknown dtype %d", x_dtype);
  if (n_blocks < 0) return fail(QZ_ERR_INVALID, "n_blocks must be >= 0");
  if (n_blocks == 0) return QZ_OK;
  if (!x) return fail(QZ_ERR_INVALID, "x is NULL");
  if (!aligned(x, 16)) return fail(QZ_ERR_INVALID, "x must be 16-byte aligned");
  if ((quants && !aligned(quants, 16)) || (dq && !aligned(dq, 16)) ||
      (dq_bf16 && !aligned(dq_bf16, 16)) || (packed && !aligned(packed, block_size == 16 ? 8 : 16)))
    return fail(QZ_ERR_INVALID, "quants/dq/dq_bf16 must be 16-byte aligned, packed 8/16-byte aligned");
  if (method == QZ_METHOD_HESSIAN) {
    if (!h_blocks) return fail(QZ_ERR_INVALID, "X or H_blocks required");
    if (n_col_blocks <= 0 || n_blocks % n_col_blocks != 0)
      return fail(QZ_ERR_INVALID, "n_blocks (%lld) must be a multiple of n_col_blocks (%lld)",
                  (long long)n_blocks, (long long)n_col_blocks);
    if (n_col_blocks > 2147483647LL) return fail(QZ_ERR_INVALID, "too many column blocks");
    if (!aligned(h_blocks, 16)) return fail(QZ_ERR_INVALID, "h_blocks must be 16-byte aligned");
  }
  int sms = 0;
  int st = current_sms(&sms);
  if (st != QZ_OK) return st;
  QuantArgs p{x, n_blocks, h_blocks, n_col_blocks, scales, quants, dq, scale_codes, packed, dq_bf16};
  return cuda_status(launch_quantize(p, x_dtype, block_size, format, method, sms,
                                     static_cast<cudaStream_t>(stream)),
                     "qz_quantize launch");
}

int qz_quantize_grouped(const QzQuantItem* items, int n_items, int x_dtype, int block_size, int format,
                        int method, void* stream) {
  if (block_size != 16 && block_size != 32)
    return fail(QZ_ERR_INVALID, "block_size must be 16 or 32, got %d", block_size);
  if (format != QZ_FMT_NVFP4 && format != QZ_FMT_MXFP4)
    return fail(QZ_ERR_INVALID, "qz_quantize_grouped supports NVFP4 and MXFP4, got format %d", format);
  if (method != QZ_METHOD_NAIVE && method != QZ_METHOD_SSE)
    return fail(QZ_ERR_INVALID, "qz_quantize_grouped supports the naive and SSE methods, got %d", method);
  if (x_dtype != QZ_DTYPE_F32 && x_dtype != QZ_DTYPE_BF16 && x_dtype != QZ_DTYPE_F16)
    return fail(QZ_ERR_INVALID, "unknown dtype %d", x_dtype);
  if (n_items < 0) return fail(QZ_ERR_INVALID, "n_items must be >= 0");
  if (n_items == 0) return QZ_OK;
  if (!items) return fail(QZ_ERR_INVALID, "items is NULL");
  for (int i = 0; i < n_items; ++i) {
    const QzQuantItem& it = items[i];
    if (it.n_blocks < 0) return fail(QZ_ERR_INVALID, "item %d: n_blocks must be >= 0", i);
    if (it.n_blocks == 0) continue;
    if (!it.x || !aligned(it.x, 16)) return fail(QZ_ERR_INVALID, "item %d: x must be non-NULL and 16-byte aligned", i);
    if ((it.quants && !aligned(it.quants, 16)) || (it.dq && !aligned(it.dq, 16)) ||
        (it.dq_bf16 && !aligned(it.dq_bf16, 16)) || (it.packed && !aligned(it.packed, block_size == 16 ? 8 : 16)))
      return fail(QZ_ERR_INVALID, "item %d: quants/dq/dq_bf16 must be 16-byte aligned, packed 8/16-byte aligned", i);
  }
  int sms = 0;
  int st = current_sms(&sms);
  if (st != QZ_OK) return st;
  // Launches of up to kMaxGroupItems inputs; the descriptors travel as the
  // kernel's parameter.
  static thread_local GroupArgs g;
  for (int i0 = 0; i0 < n_items; i0 += kMaxGroupItems) {
    const int n = n_items - i0 < kMaxGroupItems ? n_items - i0 : kMaxGroupItems;
    int64_t chunks = 0;
    int m = 0;
    for (int i = i0; i < i0 + n; ++i) {
      const QzQuantItem& it = items[i];
      if (it.n_blocks == 0) continue;
      g.item[m] = GroupItem{it.x, it.n_blocks, chunks, it.scales, it.quants, it.dq, it.scale_codes, it.packed,
                            it.dq_bf16};
      chunks += (it.n_blocks + 31) / 32;
      ++m;
    }
    g.n_items = m;
    g.n_chunks = chunks;
    st = cuda_status(launch_quantize_grouped(g, x_dtype, block_size, format, method, sms,
                                             static_cast<cudaStream_t>(stream)),
                     "qz_quantize_grouped launch");
    if (st != QZ_OK) return st;
  }
  return QZ_OK;
}

int qz_admm(const void* x, int x_dtype, int64_t n_blocks, int block_size, const float* h_blocks,
            const float* hn_blocks, const float* minv_blocks, int64_t n_col_blocks, int n_outer, int n_inner,
            float rho, float* scales, float* quants, float* dq, uint8_t* scale_codes, uint8_t* packed,
            uint16_t* dq_bf16, void* stream) {
  if (block_size != 16 && block_size != 32)
    return fail(QZ_ERR_INVALID, "block_size must be 16 or 32, got %d", block_size);
  if (x_dtype != QZ_DTYPE_F32 && x_dtype != QZ_DTYPE_BF16 && x_dtype != QZ_DTYPE_F16)
    return fail(QZ_ERR_INVALID, "unknown dtype %d", x_dtype);
  if (n_blocks < 0 || n_outer < 0 || n_inner < 0) return fail(QZ_ERR_INVALID, "negative size or iteration count");
  if (n_blocks == 0) return QZ_OK;
  if (!x || !h_blocks || !hn_blocks || !minv_blocks) return fail(QZ_ERR_INVALID, "NULL input");
  if (n_col_blocks <= 0 || n_blocks % n_col_blocks != 0 || n_col_blocks > 2147483647LL)
    return fail(QZ_ERR_INVALID, "n_blocks (%lld) must be a multiple of n_col_blocks (%lld)", (long long)n_blocks,
                (long long)n_col_blocks);
  if (!aligned(x, 16) || (quants && !aligned(quants, 16)) || (dq && !aligned(dq, 16)))
    return fail(QZ_ERR_INVALID, "x, quants and dq must be 16-byte aligned");
  int sms = 0;
  int st = current_sms(&sms);
  if (st != QZ_OK) return st;
  QuantArgs p{x, n_blocks, h_blocks, n_col_blocks, scales, quants, dq, scale_codes, packed, dq_bf16};
  return cuda_status(launch_admm(p, h_blocks, hn_blocks, minv_blocks, n_outer, n_inner, rho, x_dtype, block_size,
                                 sms, static_cast<cudaStream_t>(stream)),
                     "qz_admm launch");
}

int qz_quantize_table(const void* x, int x_dtype, int64_t n_blocks, int block_size, int method,
                      const float* table, int n_table, const float* h_blocks, int64_t n_col_blocks,
                      float* scales, float* quants, float* dq, uint8_t* scale_codes, uint8_t* packed,
                      uint16_t* dq_bf16, void* stream) {
  if (block_size != 16 && block_size != 32)
    return fail(QZ_ERR_INVALID, "block_size must be 16 or 32, got %d", block_size);
  if (method != QZ_METHOD_NAIVE && method != QZ_METHOD_SSE && method != QZ_METHOD_HESSIAN)
    return fail(QZ_ERR_INVALID, "table formats support the naive, SSE and Hessian methods, got %d", method);
  if (x_dtype != QZ_DTYPE_F32 && x_dtype != QZ_DTYPE_BF16 && x_dtype != QZ_DTYPE_F16)
    return fail(QZ_ERR_INVALID, "unknown dtype %d", x_dtype);
  if (!table || n_table < 2 || n_table > 256)
    return fail(QZ_ERR_INVALID, "table must hold 2..256 sorted positive scales, got %d", n_table);
  if (n_blocks < 0) return fail(QZ_ERR_INVALID, "n_blocks must be >= 0");
  if (n_blocks == 0) return QZ_OK;
  if (!x || !aligned(x, 16)) return fail(QZ_ERR_INVALID, "x must be non-NULL and 16-byte aligned");
  if ((quants && !aligned(quants, 16)) || (dq && !aligned(dq, 16)) || (dq_bf16 && !aligned(dq_bf16, 16)) ||
      (packed && !aligned(packed, block_size == 16 ? 8 : 16)))
    return fail(QZ_ERR_INVALID, "quants/dq/dq_bf16 must be 16-byte aligned, packed 8/16-byte aligned");
  if (method == QZ_METHOD_HESSIAN) {
    if (!h_blocks) return fail(QZ_ERR_INVALID, "X or H_blocks required");
    if (n_col_blocks <= 0 || n_blocks % n_col_blocks != 0 || n_col_blocks > 2147483647LL)
      return fail(QZ_ERR_INVALID, "n_blocks (%lld) must be a multiple of n_col_blocks (%lld)",
                  (long long)n_blocks, (long long)n_col_blocks);
  }
  int sms = 0;
  int st = current_sms(&sms);
  if (st != QZ_OK) return st;
  QuantArgs p{x, n_blocks, h_blocks, n_col_blocks, scales, quants, dq, scale_codes, packed, dq_bf16, table, n_table};
  return cuda_status(launch_quantize_table(p, x_dtype, block_size, method, sms, static_cast<cudaStream_t>(stream)),
                     "qz_quantize_table launch");
}

int qz_dequantize(const float* scales, const float* quants, int64_t n_blocks, int block_size,
                  float* out, void* stream) {
  if (block_size != 16 && block_size != 32 && block_size != 64 && block_size != 128 && block_size != 256)
    return fail(QZ_ERR_INVALID, "block_size must be 16, 32, 64, 128 or 256, got %d", block_size);
  if (n_blocks < 0) return fail(QZ_ERR_INVALID, "n_blocks must be >= 0");
  if (n_blocks == 0) return QZ_OK;
  if (!scales || !quants || !out) return fail(QZ_ERR_INVALID, "NULL pointer");
  if (!aligned(quants, 16) || !aligned(out, 16))
    return fail(QZ_ERR_INVALID, "quants and out must be 16-byte aligned");
  int sms = 0;
  int st = current_sms(&sms);
  if (st != QZ_OK) return st;
  return cuda_status(launch_dequantize(scales, quants, n_blocks, block_size, out, sms,
                                       static_cast<cudaStream_t>(stream)),
                     "qz_dequantize launch");
}

int qz_dequantize_packed(const uint8_t* packed, const uint8_t* scale_codes, int64_t n_blocks,
                         int block_size, int format, float* out_f32, uint16_t* out_bf16,
                         void* stream) {
  if (block_size != 16 && block_size != 32)
    return fail(QZ_ERR_INVALID, "block_size must be 16 or 32, got %d", block_size);
  if (format != QZ_FMT_NVFP4 && format != QZ_FMT_MXFP4)
    return fail(QZ_ERR_INVALID, "unknown format %d", format);
  if (n_blocks < 0) return fail(QZ_ERR_INVALID, "n_blocks must be >= 0");
  if (n_blocks == 0) return QZ_OK;
  if (!packed || !scale_codes) return fail(QZ_ERR_INVALID, "NULL input");
  if (!aligned(packed, 4) || (out_f32 && !aligned(out_f32, 16)) || (out_bf16 && !aligned(out_bf16, 16)))
    return fail(QZ_ERR_INVALID, "packed must be 4-byte aligned, outputs 16-byte aligned");
  int sms = 0;
  int st = current_sms(&sms);
  if (st != QZ_OK) return st;
  return cuda_status(launch_dequantize_packed(packed, scale_codes, n_blocks, block_size, format,
                                              out_f32, out_bf16, sms,
                                              static_cast<cudaStream_t>(stream)),
                     "qz_dequantize_packed launch");
}

int qz_fp4_unpack(const uint8_t* packed, int64_t n_bytes, int8_t* out, void* stream) {
  if (n_bytes < 0 || n_bytes % 4 != 0)
    return fail(QZ_ERR_INVALID, "Input size must be a multiple of 4 bytes");
  if (n_bytes == 0) return QZ_OK;
  if (!packed || !out) return fail(QZ_ERR_INVALID, "NULL pointer");
  if (!aligned(packed, 4) || !aligned(out, 8))
    return fail(QZ_ERR_INVALID, "packed must be 4-byte aligned, out 8-byte aligned");
  int sms = 0;
  int st = current_sms(&sms);
  if (st != QZ_OK) return st;
  return cuda_status(launch_unpack(packed, n_bytes, out, sms, static_cast<cudaStream_t>(stream)),
                     "qz_fp4_unpack launch");
}

int qz_weight_error_sums(const void* W, int w_dtype, const void* W_dq, int dq_dtype, int64_t n,
                         double* sums, void* stream) {
  if (w_dtype < 0 || w_dtype > 2 || dq_dtype < 0 || dq_dtype > 2)
    return fail(QZ_ERR_INVALID, "unknown dtype");
  if (n < 0) return fail(QZ_ERR_INVALID, "n must be >= 0");
  if (n == 0) return QZ_OK;
  if (!W || !W_dq || !sums) return fail(QZ_ERR_INVALID, "NULL pointer");
  int sms = 0;
  int st = current_sms(&sms);
  if (st != QZ_OK) return st;
  return cuda_status(launch_weight_sums(W, w_dtype, W_dq, dq_dtype, n, sums, sms,
                                        static_cast<cudaStream_t>(stream)),
                     "qz_weight_error_sums launch");
}

}  // extern "C"
