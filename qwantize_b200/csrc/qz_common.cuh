// qz_common.cuh -- device helpers shared by the quantization kernels.
//
// The arithmetic restates the reference's pure-PyTorch CPU evaluation order
// exactly (qwantize v0.1.2, nvfp4/reference.py and mxfp4/reference.py):
//   * sum(-1) over a 16/32-element fp32 row = eight interleaved accumulators,
//     acc[k] = v[k] + v[k+8] (+ v[k+16] + v[k+24]), then acc0 + acc1 + ... + acc7
//     in sequence;
//   * cumsum = sequential double accumulation, each prefix rounded to fp32;
//   * every multiply / add / divide / sqrt is a separately rounded IEEE op
//     (the translation units using this are compiled with -fmad=false and use
//     the __f*_rn intrinsics).
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace qz {

constexpr int kDtF32 = 0, kDtBF16 = 1, kDtF16 = 2;
constexpr int kNVFP4 = 0, kMXFP4 = 1, kTable = 2;  // kTable: caller-supplied sorted scale table
constexpr int kNVINT4 = 3, kInt8 = 4;              // symmetric integer grids (qz_int.cu)
constexpr int kNaive = 0, kSSE = 1, kHessian = 2, kNaiveArgmin = 3, kTwoArgmin = 4;

// NaN bit patterns the reference produces for a NaN scale: the E4M3 NaN code
// 0x7f widened to fp32 (NVFP4) and torch CPU log2/pow's all-ones NaN (MXFP4).
constexpr uint32_t kNvNanBits = 0x7ff00000u;
constexpr uint32_t kMxNanBits = 0xffffffffu;

// E2M1 decision boundaries and codebook (nvfp4/reference.py:14-16).
__device__ __forceinline__ constexpr float bnd(int k) {
  return k == 0 ? 0.25f : k == 1 ? 0.75f : k == 2 ? 1.25f : k == 3 ? 1.75f
       : k == 4 ? 2.5f : k == 5 ? 3.5f : 5.0f;
}
__device__ __forceinline__ constexpr float cbv(int k) {
  return k == 0 ? 0.0f : k == 1 ? 0.5f : k == 2 ? 1.0f : k == 3 ? 1.5f
       : k == 4 ? 2.0f : k == 5 ? 3.0f : k == 6 ? 4.0f : 6.0f;
}

// fl32(a / s) > B_k without dividing, for a >= 0 and a finite s > 0:
// the boundaries have at most 3 significant bits, so the fp32 midpoint just
// above B_k is B_k + ulp(B_k) / 2 and a tie there rounds (to even) down to
// B_k; hence fl(a / s) > B_k  <=>  a / s > B_k + ulp / 2  <=>  a > s * (B_k +
// ulp / 2), a product that is exact in double (<= 24 + 24 significant bits)
// and, for fp32 a, the same test as a > RD_fp32(that product).
__device__ __forceinline__ constexpr double bnd_mid(int k) {
  return k == 0 ? 0.25 + 0x1p-26 : k == 1 ? 0.75 + 0x1p-25 : k == 2 ? 1.25 + 0x1p-24 : k == 3 ? 1.75 + 0x1p-24
       : k == 4 ? 2.5 + 0x1p-23 : k == 5 ? 3.5 + 0x1p-23 : 5.0 + 0x1p-22;
}
__device__ __forceinline__ float div_threshold(float s, int k) {
  return __double2float_rd(__dmul_rn((double)s, bnd_mid(k)));
}

// Codebook value of a runtime index 0..7 without a table or branches:
// for c >= 2 the E2M1 value 2^((c>>1)-1) * (1 + (c&1)/2) has fp32 bits
// (c << 22) + 0x3f000000; c = 1 is 0.5 and c = 0 is 0.
__device__ __forceinline__ float cb_rt(uint32_t c) {
  float v = __uint_as_float((c << 22) + 0x3f000000u);
  v = c == 1u ? 0.5f : v;
  return c == 0u ? 0.0f : v;
}

// Hardware E2M1 rounding (sm_100a).  For an input with at most 11 significant
// bits (bf16 / fp16) and any E4M3 or UE8M0 scale s > 0, rounding
// y' = |x| * RN(RN(1/s) * (1 - 2^-13)) to nearest-even never meets a tie and
// equals the reference's bucketize(|x| / s) (ties to the smaller entry):
// proved exhaustively over all such inputs and scales by
// tests/test_rounding_cpu.py.  Inf saturates to the largest code.
constexpr float kBiasDown = 0.9998779296875f;  // 1 - 2^-13

// Two magnitude codes in one byte: lo -> bits 0..3, hi -> bits 4..7.
__device__ __forceinline__ uint32_t e2m1x2_rn(float lo, float hi) {
  uint32_t out;
  asm("{\n .reg .b8 b;\n cvt.rn.satfinite.e2m1x2.f32 b, %1, %2;\n cvt.u32.u8 %0, b;\n}\n"
      : "=r"(out)
      : "f"(hi), "f"(lo));
  return out;
}

// Decode a byte of two (signed) E2M1 codes to fp32 values (exact).
__device__ __forceinline__ float2 e2m1x2_to_float2(uint32_t byte) {
  uint32_t h2;
  asm("{\n .reg .b8 b;\n cvt.u8.u32 b, %1;\n cvt.rn.f16x2.e2m1x2 %0, b;\n}\n" : "=r"(h2) : "r"(byte));
  __half2 h = *reinterpret_cast<__half2*>(&h2);
  return __half22float2(h);
}

__device__ __forceinline__ bool is_nan_bits(uint32_t abs_bits) { return abs_bits > 0x7f800000u; }

// x.to(float8_e4m3fn).to(float32) for x >= 0 or NaN: round to nearest even,
// subnormal step 2^-9, values above 464 (which round past 448) become NaN.
__device__ __forceinline__ float e4m3_snap_nonneg(float a) {
  if (!(a <= 464.0f)) return __uint_as_float(kNvNanBits);
  if (a < 0.015625f) return __fmul_rn(rintf(__fmul_rn(a, 512.0f)), 0.001953125f);
  uint32_t u = __float_as_uint(a);
  u += 0x7ffffu + ((u >> 20) & 1u);
  return __uint_as_float(u & 0xfff00000u);
}

// E4M3 code of a non-negative value on the E4M3 grid (NaN -> 0x7f).
__device__ __forceinline__ uint32_t e4m3_code(float s) {
  uint32_t u = __float_as_uint(s);
  if (is_nan_bits(u & 0x7fffffffu)) return 0x7f;
  if (s == 0.0f) return 0;
  if (s < 0.015625f) return (uint32_t)__float2int_rn(__fmul_rn(s, 512.0f));
  uint32_t e = ((u >> 23) & 0xff) - 120;
  return (e << 3) | ((u >> 20) & 7);
}

// Value of positive E4M3 code c (1..126).
__device__ __forceinline__ float e4m3_value(int c) {
  if (c < 8) return __fmul_rn((float)c, 0.001953125f);
  return __uint_as_float(((uint32_t)c << 20) + (120u << 23));
}

// Largest code whose value is <= v (0 if none); v >= 0 and not NaN.
__device__ __forceinline__ int e4m3_floor_code(float v) {
  if (v >= 448.0f) return 126;
  if (v < 0.001953125f) return 0;
  if (v < 0.015625f) return (int)floorf(__fmul_rn(v, 512.0f));
  uint32_t u = __float_as_uint(v);
  return (int)(((((u >> 23) & 0xff) - 120) << 3) | ((u >> 20) & 7));
}

// Smallest code whose value is >= v (127 if none); v >= 0 and not NaN.
__device__ __forceinline__ int e4m3_ceil_code(float v) {
  if (v <= 0.001953125f) return 1;
  if (v > 448.0f) return 127;
  int f = e4m3_floor_code(v);
  return e4m3_value(f) == v ? f : f + 1;
}

// MXFP4 naive exponent (mxfp4/reference.py:114-118):
// clamp(floor(log2(max(amax, 1e-30))) - 2 + 127, 1, 254), with the exact
// floor(log2) from the bits (torch's fp32 log2 path gives the same for every
// bf16/fp16 input).  NaN is handled by the caller.
__device__ __forceinline__ int ue8m0_naive_exp(uint32_t amax_bits) {
  if (amax_bits >= 0x7f800000u) return 254;   // inf
  if (amax_bits < 0x0da24260u) return 25;     // below 1e-30f: log2(1e-30) = -99.66
  int e = (int)(amax_bits >> 23) - 2;         // floor(log2) - 2 + 127
  return e > 254 ? 254 : e;
}

__device__ __forceinline__ float pow2f(int e) {  // 2^e for -126 <= e <= 127
  return __uint_as_float((uint32_t)(e + 127) << 23);
}

// sum(-1) of a BS-element row in torch's CPU order.
template <int BS>
__device__ __forceinline__ float sum8(const float (&v)[BS]) {
  float acc[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) acc[k] = v[k];
#pragma unroll
  for (int i = 8; i < BS; i += 8)
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] = __fadd_rn(acc[k], v[i + k]);
  float r = acc[0];
#pragma unroll
  for (int k = 1; k < 8; ++k) r = __fadd_rn(r, acc[k]);
  return r;
}

// In-register ascending sort of non-negative float bit patterns (NaN patterns
// compare above inf, so they sort last, like torch.sort): Batcher odd-even
// merge networks, 63 compare-exchanges for 16 inputs and 191 for 32.
#define QZ_CE(i, j)                   \
  {                                   \
    const uint32_t a_ = v[i], b_ = v[j]; \
    v[i] = min(a_, b_);               \
    v[j] = max(a_, b_);               \
  }
template <int N>
__device__ __forceinline__ void sort_u32(uint32_t (&v)[N]) {
  if constexpr (N == 16) {
    QZ_CE(0, 1); QZ_CE(2, 3); QZ_CE(0, 2); QZ_CE(1, 3); QZ_CE(1, 2); QZ_CE(4, 5);
    QZ_CE(6, 7); QZ_CE(4, 6); QZ_CE(5, 7); QZ_CE(5, 6); QZ_CE(0, 4); QZ_CE(2, 6);
    QZ_CE(2, 4); QZ_CE(1, 5); QZ_CE(3, 7); QZ_CE(3, 5); QZ_CE(1, 2); QZ_CE(3, 4);
    QZ_CE(5, 6); QZ_CE(8, 9); QZ_CE(10, 11); QZ_CE(8, 10); QZ_CE(9, 11); QZ_CE(9, 10);
    QZ_CE(12, 13); QZ_CE(14, 15); QZ_CE(12, 14); QZ_CE(13, 15); QZ_CE(13, 14); QZ_CE(8, 12);
    QZ_CE(10, 14); QZ_CE(10, 12); QZ_CE(9, 13); QZ_CE(11, 15); QZ_CE(11, 13); QZ_CE(9, 10);
    QZ_CE(11, 12); QZ_CE(13, 14); QZ_CE(0, 8); QZ_CE(4, 12); QZ_CE(4, 8); QZ_CE(2, 10);
    QZ_CE(6, 14); QZ_CE(6, 10); QZ_CE(2, 4); QZ_CE(6, 8); QZ_CE(10, 12); QZ_CE(1, 9);
    QZ_CE(5, 13); QZ_CE(5, 9); QZ_CE(3, 11); QZ_CE(7, 15); QZ_CE(7, 11); QZ_CE(3, 5);
    QZ_CE(7, 9); QZ_CE(11, 13); QZ_CE(1, 2); QZ_CE(3, 4); QZ_CE(5, 6); QZ_CE(7, 8);
    QZ_CE(9, 10); QZ_CE(11, 12); QZ_CE(13, 14);
  } else {
    QZ_CE(0, 1); QZ_CE(2, 3); QZ_CE(0, 2); QZ_CE(1, 3); QZ_CE(1, 2); QZ_CE(4, 5);
    QZ_CE(6, 7); QZ_CE(4, 6); QZ_CE(5, 7); QZ_CE(5, 6); QZ_CE(0, 4); QZ_CE(2, 6);
    QZ_CE(2, 4); QZ_CE(1, 5); QZ_CE(3, 7); QZ_CE(3, 5); QZ_CE(1, 2); QZ_CE(3, 4);
    QZ_CE(5, 6); QZ_CE(8, 9); QZ_CE(10, 11); QZ_CE(8, 10); QZ_CE(9, 11); QZ_CE(9, 10);
    QZ_CE(12, 13); QZ_CE(14, 15); QZ_CE(12, 14); QZ_CE(13, 15); QZ_CE(13, 14); QZ_CE(8, 12);
    QZ_CE(10, 14); QZ_CE(10, 12); QZ_CE(9, 13); QZ_CE(11, 15); QZ_CE(11, 13); QZ_CE(9, 10);
    QZ_CE(11, 12); QZ_CE(13, 14); QZ_CE(0, 8); QZ_CE(4, 12); QZ_CE(4, 8); QZ_CE(2, 10);
    QZ_CE(6, 14); QZ_CE(6, 10); QZ_CE(2, 4); QZ_CE(6, 8); QZ_CE(10, 12); QZ_CE(1, 9);
    QZ_CE(5, 13); QZ_CE(5, 9); QZ_CE(3, 11); QZ_CE(7, 15); QZ_CE(7, 11); QZ_CE(3, 5);
    QZ_CE(7, 9); QZ_CE(11, 13); QZ_CE(1, 2); QZ_CE(3, 4); QZ_CE(5, 6); QZ_CE(7, 8);
    QZ_CE(9, 10); QZ_CE(11, 12); QZ_CE(13, 14); QZ_CE(16, 17); QZ_CE(18, 19); QZ_CE(16, 18);
    QZ_CE(17, 19); QZ_CE(17, 18); QZ_CE(20, 21); QZ_CE(22, 23); QZ_CE(20, 22); QZ_CE(21, 23);
    QZ_CE(21, 22); QZ_CE(16, 20); QZ_CE(18, 22); QZ_CE(18, 20); QZ_CE(17, 21); QZ_CE(19, 23);
    QZ_CE(19, 21); QZ_CE(17, 18); QZ_CE(19, 20); QZ_CE(21, 22); QZ_CE(24, 25); QZ_CE(26, 27);
    QZ_CE(24, 26); QZ_CE(25, 27); QZ_CE(25, 26); QZ_CE(28, 29); QZ_CE(30, 31); QZ_CE(28, 30);
    QZ_CE(29, 31); QZ_CE(29, 30); QZ_CE(24, 28); QZ_CE(26, 30); QZ_CE(26, 28); QZ_CE(25, 29);
    QZ_CE(27, 31); QZ_CE(27, 29); QZ_CE(25, 26); QZ_CE(27, 28); QZ_CE(29, 30); QZ_CE(16, 24);
    QZ_CE(20, 28); QZ_CE(20, 24); QZ_CE(18, 26); QZ_CE(22, 30); QZ_CE(22, 26); QZ_CE(18, 20);
    QZ_CE(22, 24); QZ_CE(26, 28); QZ_CE(17, 25); QZ_CE(21, 29); QZ_CE(21, 25); QZ_CE(19, 27);
    QZ_CE(23, 31); QZ_CE(23, 27); QZ_CE(19, 21); QZ_CE(23, 25); QZ_CE(27, 29); QZ_CE(17, 18);
    QZ_CE(19, 20); QZ_CE(21, 22); QZ_CE(23, 24); QZ_CE(25, 26); QZ_CE(27, 28); QZ_CE(29, 30);
    QZ_CE(0, 16); QZ_CE(8, 24); QZ_CE(8, 16); QZ_CE(4, 20); QZ_CE(12, 28); QZ_CE(12, 20);
    QZ_CE(4, 8); QZ_CE(12, 16); QZ_CE(20, 24); QZ_CE(2, 18); QZ_CE(10, 26); QZ_CE(10, 18);
    QZ_CE(6, 22); QZ_CE(14, 30); QZ_CE(14, 22); QZ_CE(6, 10); QZ_CE(14, 18); QZ_CE(22, 26);
    QZ_CE(2, 4); QZ_CE(6, 8); QZ_CE(10, 12); QZ_CE(14, 16); QZ_CE(18, 20); QZ_CE(22, 24);
    QZ_CE(26, 28); QZ_CE(1, 17); QZ_CE(9, 25); QZ_CE(9, 17); QZ_CE(5, 21); QZ_CE(13, 29);
    QZ_CE(13, 21); QZ_CE(5, 9); QZ_CE(13, 17); QZ_CE(21, 25); QZ_CE(3, 19); QZ_CE(11, 27);
    QZ_CE(11, 19); QZ_CE(7, 23); QZ_CE(15, 31); QZ_CE(15, 23); QZ_CE(7, 11); QZ_CE(15, 19);
    QZ_CE(23, 27); QZ_CE(3, 5); QZ_CE(7, 9); QZ_CE(11, 13); QZ_CE(15, 17); QZ_CE(19, 21);
    QZ_CE(23, 25); QZ_CE(27, 29); QZ_CE(1, 2); QZ_CE(3, 4); QZ_CE(5, 6); QZ_CE(7, 8);
    QZ_CE(9, 10); QZ_CE(11, 12); QZ_CE(13, 14); QZ_CE(15, 16); QZ_CE(17, 18); QZ_CE(19, 20);
    QZ_CE(21, 22); QZ_CE(23, 24); QZ_CE(25, 26); QZ_CE(27, 28); QZ_CE(29, 30);
  }
}
#undef QZ_CE

template <int DT>
struct Elem { static constexpr int kSize = DT == kDtF32 ? 4 : 2; };

__device__ __forceinline__ float bf16_bits_to_float(uint32_t h) { return __uint_as_float(h << 16); }
__device__ __forceinline__ float f16_bits_to_float(uint32_t h) {
  return __half2float(__ushort_as_half((unsigned short)h));
}

// Load one block of BS elements (16-byte aligned) as fp32.
template <int BS, int DT>
__device__ __forceinline__ void load_block(const void* base, int64_t blk, float (&x)[BS]) {
  const uint4* p = reinterpret_cast<const uint4*>(
      static_cast<const char*>(base) + blk * (int64_t)(BS * Elem<DT>::kSize));
  constexpr int kVec = BS * Elem<DT>::kSize / 16;
#pragma unroll
  for (int v = 0; v < kVec; ++v) {
    uint4 w = __ldg(p + v);
    uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (DT == kDtF32) {
        x[v * 4 + k] = __uint_as_float(ww[k]);
      } else if (DT == kDtBF16) {
        x[v * 8 + 2 * k] = bf16_bits_to_float(ww[k] & 0xffffu);
        x[v * 8 + 2 * k + 1] = bf16_bits_to_float(ww[k] >> 16);
      } else {
        x[v * 8 + 2 * k] = f16_bits_to_float(ww[k] & 0xffffu);
        x[v * 8 + 2 * k + 1] = f16_bits_to_float(ww[k] >> 16);
      }
    }
  }
}

}  // namespace qz
