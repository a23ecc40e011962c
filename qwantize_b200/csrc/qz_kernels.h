// qz_kernels.h -- internal launch interface between the C ABI (qz_abi.cu) and
// the kernel translation units.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace qz {

struct QuantArgs {
  const void* x;
  int64_t n_blocks;
  const float* h_blocks;
  int64_t n_col_blocks;
  float* scales;
  float* quants;
  float* dq;
  uint8_t* scale_codes;
  uint8_t* packed;
  uint16_t* dq_bf16;
  const float* table;  // kTable format: sorted positive scale values (device), n_table of them
  int n_table;
};

// One input of a grouped launch (qz_quantize_grouped): its blocks, outputs
// and the index of its first chunk of 32 blocks in the launch's chunk space.
struct GroupItem {
  const void* x;
  int64_t n_blocks;
  int64_t chunk0;
  float* scales;
  float* quants;
  float* dq;
  uint8_t* scale_codes;
  uint8_t* packed;
  uint16_t* dq_bf16;
};

// Inputs per grouped launch: the descriptors travel as a kernel parameter
// (256 x 72 bytes, inside the 32 KB parameter space), so no device memory is
// needed for them.
constexpr int kMaxGroupItems = 256;

struct GroupArgs {
  int n_items;
  int64_t n_chunks;
  GroupItem item[kMaxGroupItems];
};

// One column group of GPTQ (qz_gptq): quantize its column blocks left to
// right for every row, propagating each block's scaled error into the rest of
// the group; write the dequantized blocks, the scaled errors for the update
// of the later columns, and per-CTA loss partials.
struct GptqGroupArgs {
  float* Wb;              // (nblk, M, bs) working weight, column-block-major
  float* Qb;              // (nblk, M, bs) dequantized result
  const float* Hi;        // (K, K) damped inverse Hessian
  const float* h_blocks;  // (nblk, bs, bs) block Hessians (Hessian method) or NULL
  float* E;               // (M, 2 * gk): tf32 high parts of the scaled errors, then the low parts; or NULL
  double* loss;           // one partial per CTA
  int64_t M, K;
  int g0, gb, gk;         // first column block, blocks in this group, group width in columns (E stride)
};

constexpr int kGptqRows = 8;  // rows (one warp each) per CTA of the group kernel

cudaError_t launch_gptq_group(const GptqGroupArgs& a, int bs, int fmt, int method, cudaStream_t st);
cudaError_t launch_split_tf32(const float* src, float* hi, float* lo, int64_t n, int num_sms, cudaStream_t st);

cudaError_t launch_spd_block_inverse(float* V, float* S, int64_t ld, int64_t lo, int s, int* bad, cudaStream_t st);

cudaError_t launch_quantize_grouped(const GroupArgs& g, int dtype, int bs, int fmt, int method, int num_sms,
                                    cudaStream_t st);
cudaError_t launch_quantize_nvint4(const QuantArgs& p, int dtype, int bs, int method, int num_sms,
                                   cudaStream_t st);
cudaError_t launch_quantize_int8_bs32(const QuantArgs& p, int dtype, int method, int num_sms, cudaStream_t st);
cudaError_t launch_quantize_int(const QuantArgs& p, int dtype, int bs, int fmt, int method, int num_sms,
                                cudaStream_t st);
cudaError_t launch_quantize_table(const QuantArgs& p, int dtype, int bs, int method, int num_sms, cudaStream_t st);
cudaError_t launch_quantize(const QuantArgs& p, int dtype, int bs, int fmt, int method,
                            int num_sms, cudaStream_t st);
cudaError_t launch_admm(const QuantArgs& qa, const float* h, const float* hn, const float* minv, int n_outer,
                        int n_inner, float rho, int dtype, int bs, int num_sms, cudaStream_t st);
cudaError_t launch_dequantize(const float* scales, const float* quants, int64_t n_blocks, int bs,
                              float* out, int num_sms, cudaStream_t st);
cudaError_t launch_dequantize_packed(const uint8_t* packed, const uint8_t* codes, int64_t n_blocks,
                                     int bs, int fmt, float* out_f32, uint16_t* out_bf16,
                                     int num_sms, cudaStream_t st);
cudaError_t launch_unpack(const uint8_t* packed, int64_t n_bytes, int8_t* out, int num_sms,
                          cudaStream_t st);
cudaError_t launch_weight_sums(const void* W, int wdt, const void* Wdq, int ddt, int64_t n,
                               double* sums, int num_sms, cudaStream_t st);

cudaError_t launch_wait_selftest(uint64_t limit_ns, cudaStream_t st);

cudaError_t read_device_error_quantize(unsigned* out, bool clear);
cudaError_t read_device_error_gemm(unsigned* out, bool clear);
cudaError_t read_device_error_int(unsigned* out, bool clear);

}  // namespace qz
