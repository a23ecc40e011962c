// qz_quantize.cu -- fused per-block scale search + E2M1 quantization for sm_100a.
//
// Layout of the work.  Blocks (16 or 32 contiguous elements) are grouped in
// chunks of 32, one chunk per warp at a time.  Every warp runs its own bulk-copy
// (TMA) pipeline: lane 0 keeps kStages chunk loads in flight into the warp's
// shared-memory ring, completion tracked by one mbarrier per stage, so HBM reads
// are large contiguous transfers and warps never wait for each other.
//   * Lane L owns block L of the chunk: amax, naive scale, search bounds, final
//     quantization and all stores of that block.
//   * SSE search: the (block, candidate) pairs of the whole chunk are spread
//     evenly over the 32 lanes (a block's candidates are data dependent, 0..39),
//     each lane evaluates its pairs against |x| rows kept in shared memory, and
//     the winner per block is the minimum of the 64-bit key (SSE bits, index).
//     This equals the reference's ascending loop with strict '<' updates: the
//     first (lowest) scale achieving the minimum SSE, kept only if below the
//     naive error.  (The reference's clipping fast-fail never changes that
//     winner: a candidate's clipping error is a partial sum, in the same order,
//     of its SSE's non-negative terms.)
//   * Hessian search keeps the reference's sequential semantics (its fast-fail
//     does change results) in a CTA-per-column-block kernel with H_j in smem.
// Semantics follow qwantize v0.1.2:
//   naive   nvfp4/reference.py:89-126, mxfp4/reference.py:89-129
//   SSE     nvfp4/reference.py:129-239, mxfp4/reference.py:132-238
//   Hessian nvfp4/reference.py:266-407, mxfp4/reference.py:241-374 (the shipped
//           MXFP4 function crashes; this is its intended algorithm)
//   argmin  mxfp4/kernels.py:267-377 (mxfp4_naive_torch / mxfp4_optimal_torch)
// Compiled with -fmad=false: every product and sum is separately rounded, in
// the order torch's CPU kernels use, so results are bit-identical.
#include <cuda_bf16.h>

#include "qz_common.cuh"
#include "qz_kernels.h"
#include "qz_ptx.cuh"

namespace qz {

// How bucketize(|x| / s) is evaluated exactly:
//   NVFP4, bf16/fp16 input: count thresholds B_k*s that |x| exceeds (|x| has
//     <= 11 significant bits and B_k*s <= 7, so |x|/s rounds onto a boundary
//     only when it equals it; B_k*s <= 5*448 never overflows);
//   NVFP4, fp32 input: the IEEE quotient;
//   MXFP4: |x| times the exact reciprocal 2^-e (identical to the quotient).
enum RoundMode { kCmp = 0, kDiv = 1, kRcp = 2 };
template <int FMT, int DT>
struct Mode { static constexpr int v = FMT == kMXFP4 ? kRcp : ((DT == kDtF32 || FMT == kTable) ? kDiv : kCmp); };

// Dequant magnitude t = q*s for a = |x| and a finite scale s >= 0.
template <int MODE>
struct FastQ {
  float T[7], V[7], s, r;
  __device__ __forceinline__ explicit FastQ(float s_) : s(s_) {
#pragma unroll
    for (int k = 0; k < 7; ++k) {
      if (MODE == kCmp) T[k] = __fmul_rn(bnd(k), s_);
      // the IEEE quotient's decisions as thresholds (s = 0 gives thresholds 0:
      // every decision fails for a = 0 or NaN, passes for a > 0 -- dequant 0
      // either way, as with the quotient)
      if (MODE == kDiv) T[k] = div_threshold(s_, k);
      V[k] = __fmul_rn(cbv(k + 1), s_);
    }
    r = MODE == kRcp ? __frcp_rn(s_) : 0.0f;
  }
  __device__ __forceinline__ float operator()(float a) const {
    float t = 0.0f;
    if (MODE == kCmp || MODE == kDiv) {
#pragma unroll
      for (int k = 0; k < 7; ++k) t = (a > T[k]) ? V[k] : t;
    } else {
      float y = __fmul_rn(a, r);
#pragma unroll
      for (int k = 0; k < 7; ++k) t = (y > bnd(k)) ? V[k] : t;
    }
    return t;
  }
};

// bucketize index for any scale (0, NaN included): #{k : !(y <= B_k)}.
template <int MODE>
__device__ __forceinline__ int fp4_index(float a, float s) {
  int idx = 0;
  if (MODE == kCmp) {
#pragma unroll
    for (int k = 0; k < 7; ++k) idx += (a <= __fmul_rn(bnd(k), s)) ? 0 : 1;
  } else if (MODE == kDiv && s > 0.0f && __float_as_uint(s) < 0x7f800000u && a == a) {
#pragma unroll
    for (int k = 0; k < 7; ++k) idx += (a > div_threshold(s, k)) ? 1 : 0;
  } else {
    float y = MODE == kDiv ? __fdiv_rn(a, s) : __fmul_rn(a, __frcp_rn(s));
#pragma unroll
    for (int k = 0; k < 7; ++k) idx += (y <= bnd(k)) ? 0 : 1;
  }
  return idx;
}

// Block SSE (compute_block_sse, nvfp4/reference.py:72-86) for finite s >= 0.
template <int BS, int MODE>
__device__ __forceinline__ float block_sse(const float (&a)[BS], float s) {
  FastQ<MODE> q(s);
  float d2[BS];
#pragma unroll
  for (int i = 0; i < BS; ++i) {
    float d = __fsub_rn(a[i], q(a[i]));
    d2[i] = __fmul_rn(d, d);
  }
  return sum8<BS>(d2);
}

// Packed fp32 pairs (sm_100a f32x2 arithmetic): two independent IEEE
// round-to-nearest operations per instruction, the same results as two scalar
// __f*_rn operations.
__device__ __forceinline__ uint64_t pk2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 up2(uint64_t v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return make_float2(lo, hi);
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// sum8 over squared pairs: acc lanes (k, k+1) are one packed pair, so the
// element pair (i, i+1) with i even adds into pair (i % 8) / 2.
template <int BS>
__device__ __forceinline__ float sum8_pairs(const uint64_t (&sq)[BS / 2]) {
  uint64_t acc[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) acc[k] = sq[k];
#pragma unroll
  for (int i = 4; i < BS / 2; ++i) acc[i & 3] = add2(acc[i & 3], sq[i]);
  const float2 p0 = up2(acc[0]), p1 = up2(acc[1]), p2 = up2(acc[2]), p3 = up2(acc[3]);
  float r = __fadd_rn(p0.x, p0.y);
  r = __fadd_rn(r, p1.x);
  r = __fadd_rn(r, p1.y);
  r = __fadd_rn(r, p2.x);
  r = __fadd_rn(r, p2.y);
  r = __fadd_rn(r, p3.x);
  return __fadd_rn(r, p3.y);
}

// Block SSE with hardware rounding: bf16/fp16 inputs, finite s > 0, with
// c = RN(RN(1/s) * (1 - 2^-13)) precomputed.  d = a - q*s is one FMA: q*s is
// exact in fp32 (q has <= 2 significant bits, s <= 4, and a UE8M0 product that
// overflows is infinite in both forms), so the single rounding of the FMA equals
// the reference's rounding of a - dq.
template <int BS>
__device__ __forceinline__ float block_sse_hw(const float (&a)[BS], float s, float c) {
  uint64_t sq[BS / 2];
  const uint64_t c2 = pk2(c, c), ms2 = pk2(-s, -s);
#pragma unroll
  for (int i = 0; i < BS; i += 2) {
    // y = a*c, q = E2M1(y) decoded through f16, d = a - q*s, d*d: one chain,
    // the code byte never leaves its 8-bit register
    uint64_t r;
    asm("{\n .reg .b64 a2, y, q2, d;\n .reg .f32 y0, y1, q0, q1;\n .reg .b8 b;\n .reg .b32 h;\n"
        " .reg .b16 lo, hi;\n"
        " mov.b64 a2, {%1, %2};\n mul.rn.f32x2 y, a2, %3;\n mov.b64 {y0, y1}, y;\n"
        " cvt.rn.satfinite.e2m1x2.f32 b, y1, y0;\n cvt.rn.f16x2.e2m1x2 h, b;\n mov.b32 {lo, hi}, h;\n"
        " cvt.f32.f16 q0, lo;\n cvt.f32.f16 q1, hi;\n mov.b64 q2, {q0, q1};\n"
        " fma.rn.f32x2 d, q2, %4, a2;\n mul.rn.f32x2 %0, d, d;\n}\n"
        : "=l"(r) : "f"(a[i]), "f"(a[i + 1]), "l"(c2), "l"(ms2));
    sq[i / 2] = r;
  }
  return sum8_pairs<BS>(sq);
}

// NVFP4 variant: the decoded codes stay in f16 and feed a mixed-precision FMA
// (f16 x f16 + f32 -> f32): d = RN(a - q*s) with -s held exactly in f16 (every
// E4M3 value is a normal f16), saving the f16 -> f32 conversions.
template <int BS>
__device__ __forceinline__ float block_sse_hw_nv(const float (&a)[BS], uint32_t neg_s_h, float c) {
  uint64_t sq[BS / 2];
  const uint64_t c2 = pk2(c, c);
  const unsigned short ns = (unsigned short)neg_s_h;
#pragma unroll
  for (int i = 0; i < BS; i += 2) {
    uint64_t r;
    asm("{\n .reg .b64 a2, y, d;\n .reg .f32 y0, y1, d0, d1;\n .reg .b8 b;\n .reg .b32 h;\n"
        " .reg .b16 lo, hi;\n"
        " mov.b64 a2, {%1, %2};\n mul.rn.f32x2 y, a2, %3;\n mov.b64 {y0, y1}, y;\n"
        " cvt.rn.satfinite.e2m1x2.f32 b, y1, y0;\n cvt.rn.f16x2.e2m1x2 h, b;\n mov.b32 {lo, hi}, h;\n"
        " fma.rn.f32.f16 d0, lo, %4, %1;\n fma.rn.f32.f16 d1, hi, %4, %2;\n"
        " mov.b64 d, {d0, d1};\n mul.rn.f32x2 %0, d, d;\n}\n"
        : "=l"(r) : "f"(a[i]), "f"(a[i + 1]), "l"(c2), "h"(ns));
    sq[i / 2] = r;
  }
  return sum8_pairs<BS>(sq);
}

// Per-CTA table of candidate scales and their biased reciprocals, indexed by
// E4M3 code (1..126) or UE8M0 biased exponent (1..254).
struct CandTable {
  float val[256];
  uint2 cn[256];         // x: bits of the biased reciprocal c; y: f16 bits of -val (NVFP4)
  float mid[256];       // kTable: midpoints (t[i] + t[i+1]) * 0.5 of snap_to_table
  int n;                // number of candidate codes (kTable: table length)
};

// One per CTA of every kernel that uses it (file-scope shared variable).
__shared__ CandTable s_ctab;

template <int FMT>
__device__ __forceinline__ void fill_cand_table(CandTable& t, const float* table = nullptr, int n_table = 0) {
  if constexpr (FMT == kTable) {
    // exotic_scales.py:60-74 snap_to_table: nearest entry via bucketize over
    // midpoints computed in fp32; the candidates are the table itself
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
      const float v = i < n_table ? table[i] : 1.0f;
      t.val[i] = v;
      t.cn[i] = make_uint2(0u, 0u);
      t.mid[i] = i + 1 < n_table ? __fmul_rn(__fadd_rn(table[i], table[i + 1]), 0.5f) : 0.0f;
    }
    if (threadIdx.x == 0) t.n = n_table;
    return;
  }
  if constexpr (FMT == kInt8) {
    // int8/reference.py:151-152: the effective scales E4M3 / 127, indexed by E4M3 code
    // (index 0: scale 0, never a candidate)
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
      const float v = i == 0 ? 0.0f : (i <= 126 ? __fdiv_rn(e4m3_value(i), 127.0f) : 3.0e38f);
      t.val[i] = v;
      t.cn[i] = make_uint2(__float_as_uint(__frcp_rn(v)), 0u);
    }
    if (threadIdx.x == 0) t.n = 127;
    return;
  }
  constexpr bool kE4 = FMT == kNVFP4 || FMT == kNVINT4;
  if (threadIdx.x == 0) t.n = kE4 ? 127 : 255;
  for (int i = threadIdx.x; i < 256; i += blockDim.x) {
    const bool ok = kE4 ? (i >= 1 && i <= 126) : (i >= 1 && i <= 254);
    const float v = ok ? (kE4 ? e4m3_value(i) : pow2f(i - 127)) : 1.0f;
    t.val[i] = v;
    // NVINT4 rounds with the unbiased RN(1/s); the E2M1 formats with the biased one
    t.cn[i] = make_uint2(__float_as_uint(FMT == kNVINT4 ? __frcp_rn(v) : __fmul_rn(__frcp_rn(v), kBiasDown)),
                         FMT == kNVFP4 ? (uint32_t)__half_as_ushort(__float2half_rn(-v)) : 0u);
  }
}

// clamp(round(x / s), -7, 7), round half to even (int4_quantize,
// nvint4/reference.py:29-41).  fast (16-bit input, finite s > 0, rc = RN(1/s)):
// rint(x * rc), exact except at a tie |x - q s| == s/2 (q s exact), where an
// odd q moves to its even neighbour.  Otherwise the IEEE quotient with the
// reference's x86 NaN payloads: x's NaN, else s's, 0 / 0 the default NaN.
__device__ __forceinline__ float int4_q(float xv, float s, float rc, bool fast, bool snan) {
  float q;
  if (fast) {
    q = rintf(__fmul_rn(xv, rc));
    if (fabsf(q) <= 8.0f) {
      const float e = __fmaf_rn(-q, s, xv);
      if (fabsf(e) == __fmul_rn(0.5f, s) && (__float2int_rz(q) & 1)) q = __fadd_rn(q, e > 0.0f ? 1.0f : -1.0f);
    }
    return fminf(fmaxf(q, -7.0f), 7.0f);  // keeps -0.0
  }
  const uint32_t xb = __float_as_uint(xv);
  if (is_nan_bits(xb & 0x7fffffffu)) return __uint_as_float(xb | 0x00400000u);
  if (snan) return s;
  if (s == 0.0f && xv == 0.0f) return __uint_as_float(0xffc00000u);
  q = rintf(__fdiv_rn(xv, s));
  return q < -7.0f ? -7.0f : (q > 7.0f ? 7.0f : q);
}

// NVINT4 block SSE on |x| = a (nvint4/reference.py:49-56): 16-bit inputs and a
// finite s > 0 round a * RN(1/s) (exact except at half-integer ties, which
// leave the same |d| = s/2 either way; q s is exact, so d is one FMA);
// otherwise the IEEE quotient, with s = 0 and NaN propagating as in torch.
template <int BS, int DT>
__device__ __forceinline__ float int4_sse(const float (&a)[BS], float s, float rc) {
  const uint32_t sb = __float_as_uint(s);
  if (DT != kDtF32 && sb > 0u && sb < 0x7f800000u) {
    uint64_t sq[BS / 2];
    const uint64_t c2 = pk2(rc, rc), ms2 = pk2(-s, -s);
    const uint64_t kMagic2 = pk2(12582912.0f, 12582912.0f), kNegMagic2 = pk2(-12582912.0f, -12582912.0f);
#pragma unroll
    for (int i = 0; i < BS; i += 2) {
      const uint64_t a2 = pk2(a[i], a[i + 1]);
      // round half to even of y >= 0 on the FMA pipe: (y + 1.5*2^23) - 1.5*2^23
      // (exact below 2^22; above it the result still clamps to 7)
      const float2 y = up2(add2(add2(mul2(a2, c2), kMagic2), kNegMagic2));
      const uint64_t q2 = pk2(fminf(y.x, 7.0f), fminf(y.y, 7.0f));
      const uint64_t d = fma2(q2, ms2, a2);
      sq[i / 2] = mul2(d, d);
    }
    return sum8_pairs<BS>(sq);
  }
  float d2[BS];
#pragma unroll
  for (int i = 0; i < BS; ++i) {
    float q = rintf(__fdiv_rn(a[i], s));
    q = q > 7.0f ? 7.0f : q;  // keeps NaN
    const float d = __fsub_rn(a[i], __fmul_rn(q, s));
    d2[i] = __fmul_rn(d, d);
  }
  return sum8<BS>(d2);
}

// INT8 block SSE on |x| = a (int8/reference.py:65-83): q = round(a / s) (the
// scales E4M3 / 127 carry full fp32 mantissas: the IEEE quotient decides near
// half integers), rounded half to even by the 1.5 * 2^23 add / subtract,
// clamped to 127 (NaN propagates); d = a - fl(q s) rounds twice, as in the
// reference.  rc = RN(1/s).
// round(a / s) by IEEE division; out of line: the search calls it rarely
__device__ __noinline__ float int8_round_div(float a, float s) {
  return __fadd_rn(__fadd_rn(__fdiv_rn(a, s), 12582912.0f), -12582912.0f);
}
template <int BS>
__device__ __forceinline__ float int8_sse(const float (&a)[BS], float s, float rc) {
  float d2[BS];
#pragma unroll
  for (int i = 0; i < BS; ++i) {
    // a * RN(1/s) is within 2^-15.4 of fl(a / s) below 128, so its rounding
    // agrees unless it lies within 2^-14 of a half integer: then the quotient
    // decides (s = 0 gives inf / NaN either way; above 128 both clamp)
    const float y = __fmul_rn(a[i], rc);
    float q = __fadd_rn(__fadd_rn(y, 12582912.0f), -12582912.0f);
    if (fabsf(fabsf(__fsub_rn(y, q)) - 0.5f) <= 0x1p-14f) q = int8_round_div(a[i], s);
    q = q > 127.0f ? 127.0f : q;
    const float d = __fsub_rn(a[i], __fmul_rn(q, s));
    d2[i] = __fmul_rn(d, d);
  }
  return sum8<BS>(d2);
}

// The same SSE for the candidate-parallel search, where the block's |x| row
// also sits in shared memory (row).  The loop is branch-free: it rounds
// y = a * RN(1/s) and only records the largest |y - round(y)|; a lane whose
// block has an element within 2^-14 of a half integer (rare) recomputes the
// whole block from the row with IEEE quotients, out of line.  Short straight
// code matters here: with a branch and a call site per element the kernel
// stalled on instruction fetch.
template <int BS>
__device__ __noinline__ float int8_sse_exact(const float* row, float s) {
  float acc[8];
#pragma unroll 1
  for (int i = 0; i < BS; i += 8) {  // torch's CPU row-sum order (sum8)
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float a = row[i + k];
      float q = __fadd_rn(__fadd_rn(__fdiv_rn(a, s), 12582912.0f), -12582912.0f);
      q = q > 127.0f ? 127.0f : q;
      const float d = __fsub_rn(a, __fmul_rn(q, s));
      const float d2 = __fmul_rn(d, d);
      acc[k] = i == 0 ? d2 : __fadd_rn(acc[k], d2);
    }
  }
  float r = acc[0];
#pragma unroll
  for (int k = 1; k < 8; ++k) r = __fadd_rn(r, acc[k]);
  return r;
}
template <int BS>
__device__ __forceinline__ float int8_sse_row(const float (&a)[BS], float s, float rc, const float* row) {
  float d2[BS];
  float far = 0.0f;  // largest |y - round(y)|; NaN (s = 0) is ignored, as the quotient path agrees there
#pragma unroll
  for (int i = 0; i < BS; ++i) {
    const float y = __fmul_rn(a[i], rc);
    float q = __fadd_rn(__fadd_rn(y, 12582912.0f), -12582912.0f);
    far = fmaxf(far, fabsf(__fsub_rn(y, q)));
    q = q > 127.0f ? 127.0f : q;
    const float d = __fsub_rn(a[i], __fmul_rn(q, s));
    d2[i] = __fmul_rn(d, d);
  }
  const float E = sum8<BS>(d2);
  return far >= 0.5f - 0x1p-14f ? int8_sse_exact<BS>(row, s) : E;
}

// Candidate SSE: the hardware path for 16-bit inputs, IEEE division for fp32.
template <int BS, int MODE, int DT, int FMT>
__device__ __forceinline__ float cand_sse(const float (&a)[BS], const CandTable& t, int code) {
  if constexpr (FMT == kNVINT4) return int4_sse<BS, DT>(a, t.val[code], __uint_as_float(t.cn[code].x));
  else if constexpr (FMT == kInt8) return int8_sse<BS>(a, t.val[code], __uint_as_float(t.cn[code].x));
  else
  if constexpr (DT != kDtF32 && FMT == kNVFP4) {
    const uint2 e = t.cn[code];
    return block_sse_hw_nv<BS>(a, e.y, __uint_as_float(e.x));
  } else if constexpr (DT != kDtF32 && FMT == kMXFP4) {
    return block_sse_hw<BS>(a, t.val[code], __uint_as_float(t.cn[code].x));
  }
  else return block_sse<BS, MODE>(a, t.val[code]);
}

// SSE of the naive scale s0 (finite, >= 0): the hardware path when s0 > 0 and
// the input is 16-bit; s0 = 0 (NVFP4 blocks below 6 * 2^-10) takes the generic one.
template <int BS, int MODE, int DT, int FMT>
__device__ __forceinline__ float base_sse(const float (&a)[BS], float s) {
  if constexpr (FMT == kInt8) return int8_sse<BS>(a, s, __frcp_rn(s));
  if constexpr (FMT == kNVINT4) {
    const uint32_t sb = __float_as_uint(s);
    return int4_sse<BS, DT>(a, s, sb > 0u && sb < 0x7f800000u ? __frcp_rn(s) : 0.0f);
  }
  if constexpr (DT != kDtF32 && FMT != kTable) {
    if (s > 0.0f) return block_sse_hw<BS>(a, s, __fmul_rn(__frcp_rn(s), kBiasDown));
  }
  return block_sse<BS, MODE>(a, s);
}

// Clipping error sum(clamp(|x| - Q s, 0)^2) (nvfp4/reference.py:209; Q = 7 for
// NVINT4, nvint4/reference.py:258).
template <int BS, int FMT = kNVFP4>
__device__ __forceinline__ float block_clip(const float (&a)[BS], float s) {
  float t = __fmul_rn(FMT == kInt8 ? 127.0f : (FMT == kNVINT4 ? 7.0f : 6.0f), s), v[BS];
#pragma unroll
  for (int i = 0; i < BS; ++i) {
    float c = __fsub_rn(a[i], t);
    c = c < 0.0f ? 0.0f : c;
    v[i] = __fmul_rn(c, c);
  }
  return sum8<BS>(v);
}

// r^T H r with r = x - dq: Hr_a = fma chain over b ascending, then the torch
// sum order over r_a * Hr_a.  Hj is in shared memory (broadcast reads).
template <int BS, int MODE>
__device__ __forceinline__ float block_hess(const float (&x)[BS], const float (&a)[BS], float s,
                                            const float* __restrict__ Hj) {
  FastQ<MODE> q(s);
  float r[BS];
#pragma unroll
  for (int i = 0; i < BS; ++i) {
    float t = q(a[i]);
    float dq = x[i] > 0.0f ? t : (x[i] < 0.0f ? -t : 0.0f);
    r[i] = __fsub_rn(x[i], dq);
  }
  float acc8[8];
#pragma unroll 1
  for (int ra = 0; ra < BS; ++ra) {
    const float4* h4 = reinterpret_cast<const float4*>(Hj + ra * BS);
    float acc = 0.0f;
#pragma unroll
    for (int b4 = 0; b4 < BS / 4; ++b4) {
      float4 h = h4[b4];
      acc = __fmaf_rn(h.x, r[4 * b4 + 0], acc);
      acc = __fmaf_rn(h.y, r[4 * b4 + 1], acc);
      acc = __fmaf_rn(h.z, r[4 * b4 + 2], acc);
      acc = __fmaf_rn(h.w, r[4 * b4 + 3], acc);
    }
    // r[ra] with a runtime index would spill r to local memory: select instead
    float rr = 0.0f;
#pragma unroll
    for (int i = 0; i < BS; ++i) rr = (i == ra) ? r[i] : rr;
    float pa = __fmul_rn(rr, acc);
    // torch sum order: acc8[k] = p[k] + p[k+8] (+ p[k+16] + p[k+24])
    int k = ra & 7;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j == k) acc8[j] = ra < 8 ? pa : __fadd_rn(acc8[j], pa);
  }
  float res = acc8[0];
#pragma unroll
  for (int k = 1; k < 8; ++k) res = __fadd_rn(res, acc8[k]);
  return res;
}

// Shared-memory float4 load the compiler may not hoist: H_j is loop-invariant
// across candidates, and keeping all of it in registers (bs*bs floats) spills.
__device__ __forceinline__ float4 lds_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}

// r^T H r as block_hess computes it (each row of H r is a sequential FMA chain
// over b ascending, then the torch sum order over a of r_a * (H r)_a), with the
// rows' chains interleaved for instruction-level parallelism.  Ht is H_j
// transposed in shared memory (Ht[b*BS + a] = H_j[a][b]), so one broadcast
// float4 load feeds four chains.  For bf16/fp16 inputs and s > 0 the residual
// uses the hardware rounding: r = x - sign(x) q s = +-RN(|x| - q s) with the
// sign of x applied by flipping the sign bit, bit-identical to the generic path
// (q s is exact).
template <int BS, int MODE, int DT, int FMT = kNVFP4>
__device__ __forceinline__ float block_hess_ilp(const float (&x)[BS], const float (&a)[BS], float s,
                                                const float* __restrict__ Ht) {
  float r[BS];
  if constexpr (FMT == kNVINT4) {  // r = x - dq with the exact int4 rounding (dq: the scale's NaN first)
    const uint32_t sb = __float_as_uint(s);
    const bool fast = DT != kDtF32 && sb > 0u && sb < 0x7f800000u, snan = is_nan_bits(sb & 0x7fffffffu);
    const float rc = fast ? __frcp_rn(s) : 0.0f;
#pragma unroll
    for (int i = 0; i < BS; ++i) {
      const float q = int4_q(x[i], s, rc, fast, snan);
      const float dq = snan ? s : (is_nan_bits(__float_as_uint(q) & 0x7fffffffu) ? q : __fmul_rn(q, s));
      r[i] = __fsub_rn(x[i], dq);
    }
  } else if constexpr (FMT == kInt8) {  // r = x - fl(q s), q = clamp(round(x / s)) with the reference's NaNs
    const bool snan = is_nan_bits(__float_as_uint(s) & 0x7fffffffu);
#pragma unroll
    for (int i = 0; i < BS; ++i) {
      const uint32_t xb = __float_as_uint(x[i]);
      float q;
      if (is_nan_bits(xb & 0x7fffffffu)) q = __uint_as_float(xb | 0x00400000u);
      else if (snan) q = s;
      else if (s == 0.0f && x[i] == 0.0f) q = __uint_as_float(0xffc00000u);
      else {
        q = rintf(__fdiv_rn(x[i], s));
        q = q < -127.0f ? -127.0f : (q > 127.0f ? 127.0f : q);
      }
      const float dq = snan ? s : (is_nan_bits(__float_as_uint(q) & 0x7fffffffu) ? q : __fmul_rn(q, s));
      r[i] = __fsub_rn(x[i], dq);
    }
} else if (MODE != kDiv && s > 0.0f) {  // 16-bit input with an E4M3 / UE8M0 scale
    const float c = __fmul_rn(__frcp_rn(s), kBiasDown);
#pragma unroll
    for (int i = 0; i < BS; i += 2) {
      const float2 q = e2m1x2_to_float2(e2m1x2_rn(__fmul_rn(a[i], c), __fmul_rn(a[i + 1], c)));
      // x - sign(x) q s = sign(x) * (|x| - q s): flip by x's sign bit (keeps -0.0)
      r[i] = __uint_as_float(__float_as_uint(__fmaf_rn(-q.x, s, a[i])) ^ (__float_as_uint(x[i]) & 0x80000000u));
      r[i + 1] = __uint_as_float(__float_as_uint(__fmaf_rn(-q.y, s, a[i + 1])) ^
                                 (__float_as_uint(x[i + 1]) & 0x80000000u));
    }
  } else {
    FastQ<MODE> q(s);
#pragma unroll
    for (int i = 0; i < BS; ++i) {
      const float t = q(a[i]);
      const float dq = x[i] > 0.0f ? t : (x[i] < 0.0f ? -t : 0.0f);
      r[i] = __fsub_rn(x[i], dq);
    }
  }
  float acc8[8];
#pragma unroll
  for (int g = 0; g < BS; g += 16) {
    // rows (g + 2k, g + 2k + 1) as one packed pair: fma.rn.f32x2 is two
    // independent single-rounding FMAs, the scalar chains bit for bit
    uint64_t acc2[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) acc2[k] = 0ull;
#pragma unroll
    for (int b = 0; b < BS; ++b) {
      const uint32_t hrow = smem_u32(Ht + b * BS + g);
      const uint64_t rb = pk2(r[b], r[b]);
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        const float4 h = lds_f4(hrow + 16 * q4);
        acc2[2 * q4 + 0] = fma2(pk2(h.x, h.y), rb, acc2[2 * q4 + 0]);
        acc2[2 * q4 + 1] = fma2(pk2(h.z, h.w), rb, acc2[2 * q4 + 1]);
      }
    }
    float acc[16];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float2 v = up2(acc2[k]);
      acc[2 * k] = v.x;
      acc[2 * k + 1] = v.y;
    }
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const int ai = g + k;
      const float pa = __fmul_rn(r[ai], acc[k]);
      acc8[ai & 7] = ai < 8 ? pa : __fadd_rn(acc8[ai & 7], pa);
    }
  }
  float res = acc8[0];
#pragma unroll
  for (int k = 1; k < 8; ++k) res = __fadd_rn(res, acc8[k]);
  return res;
}

// Number of table entries below v (strict) / at or below v; v not NaN.
__device__ __forceinline__ int table_count_below(float v, bool inclusive) {
  int lo = 0, hi = s_ctab.n;
  while (lo < hi) {
    const int m = (lo + hi) >> 1;
    const float t = s_ctab.val[m];
    if (inclusive ? (t <= v) : (t < v)) lo = m + 1; else hi = m;
  }
  return lo;
}

// Naive scale for FMT from amax bits (NaN propagates with the reference's bits).
template <int FMT>
__device__ __forceinline__ float naive_scale(uint32_t amax_bits) {
  if constexpr (FMT == kTable) {
    // snap_to_table((amax / 6).clamp(min=1e-12)) (exotic_scales.py:60-74):
    // bucketize over the midpoints (right=False; NaN -> last entry)
    float c = __fdiv_rn(__uint_as_float(amax_bits), 6.0f);
    c = c < 1e-12f ? 1e-12f : c;
    int lo = 0, hi = s_ctab.n - 1;
    if (is_nan_bits(amax_bits)) lo = hi;
    while (lo < hi) {
      const int m = (lo + hi) >> 1;
      if (s_ctab.mid[m] < c) lo = m + 1; else hi = m;
    }
    return s_ctab.val[lo];
  }
  if (is_nan_bits(amax_bits)) return __uint_as_float(FMT == kMXFP4 ? kMxNanBits : kNvNanBits);
  float amax = __uint_as_float(amax_bits);
  if constexpr (FMT == kInt8) {  // e4m3(max(amax, 1e-12)) / 127 (int8/reference.py:112-114)
    const float v = e4m3_snap_nonneg(amax < 1e-12f ? 1e-12f : amax);
    return is_nan_bits(__float_as_uint(v)) ? v : __fdiv_rn(v, 127.0f);
  }
  if (FMT == kNVFP4 || FMT == kNVINT4) {
    // (amax / Q_MAX).clamp(min=1e-12): Q_MAX 6 (nvfp4/reference.py:114), 7 (nvint4/reference.py:76)
    float c = __fdiv_rn(amax, FMT == kNVINT4 ? 7.0f : 6.0f);
    c = c < 1e-12f ? 1e-12f : c;
    return e4m3_snap_nonneg(c);
  }
  return pow2f(ue8m0_naive_exp(amax_bits) - 127);
}

// Bounds of the bounded search (nvfp4/reference.py:171-189).  Produces the
// inclusive range [lo, hi] of candidate indices (E4M3 codes / UE8M0 biased
// exponents); lo > hi when there is nothing to search.
template <int BS, int FMT>
__device__ __forceinline__ void search_range(const float (&x)[BS], const float (&a)[BS],
                                             float amax, float E0, int& lo, int& hi) {
  lo = 1;
  hi = 0;
  uint64_t sq[BS / 2];  // x.pow(2).sum(-1), packed pairs (x*x == |x|*|x| bit for bit)
#pragma unroll
  for (int i = 0; i < BS; i += 2) {
    const uint64_t a2 = pk2(a[i], a[i + 1]);
    sq[i / 2] = mul2(a2, a2);
  }
  bool noise = sum8_pairs<BS>(sq) <= E0;
  constexpr float kQ = FMT == kInt8 ? 127.0f : (FMT == kNVINT4 ? 7.0f : 6.0f);
  constexpr float kD0 = (FMT == kNVINT4 || FMT == kInt8) ? 0.5f : 0.25f;
  float s_min = __fdiv_rn(__fsub_rn(amax, __fsqrt_rn(E0)), kQ);
  s_min = s_min < 0.0f ? 0.0f : s_min;
  uint32_t srt[BS];
#pragma unroll
  for (int i = 0; i < BS; ++i) srt[i] = __float_as_uint(a[i]);
  sort_u32<BS>(srt);
  double c = 0.0;
  int k_star = 0;
#pragma unroll
  for (int i = 0; i < BS; ++i) {
    float v = __uint_as_float(srt[i]);
    c = __dadd_rn(c, (double)__fmul_rn(v, v));
    k_star += (__double2float_rn(c) <= E0) ? 1 : 0;
  }
  if (k_star >= BS) noise = true;
  int kidx = k_star < BS - 1 ? k_star : BS - 1;
  float y = 0.0f;
#pragma unroll
  for (int i = 0; i < BS; ++i) y = (i == kidx) ? __uint_as_float(srt[i]) : y;
  float s_max = __fdiv_rn(y, kD0);
  if (noise || !(s_min <= s_max)) return;
  if (FMT == kTable || FMT == kInt8) {
    lo = table_count_below(s_min, false);
    hi = table_count_below(s_max, true) - 1;
    if (FMT == kInt8 && lo < 1) lo = 1;  // index 0 (scale 0) is not a candidate
  } else if (FMT == kNVFP4 || FMT == kNVINT4) {
    lo = e4m3_ceil_code(s_min);
    hi = e4m3_floor_code(s_max);
  } else {
    uint32_t bmin = __float_as_uint(s_min), bmax = __float_as_uint(s_max);
    if (bmin >= 0x7f800000u) return;
    lo = bmin <= 0x00800000u ? 1 : (int)(bmin >> 23) + ((bmin & 0x7fffffu) ? 1 : 0);
    hi = bmax < 0x00800000u ? 0 : (bmax >= 0x7f800000u ? 254 : (int)(bmax >> 23));
    hi = hi > 254 ? 254 : hi;
  }
}

template <int FMT>
__device__ __forceinline__ float cand_value(int c) {
  if constexpr (FMT == kTable || FMT == kInt8) return s_ctab.val[c];
  return (FMT == kNVFP4 || FMT == kNVINT4) ? e4m3_value(c) : pow2f(c - 127);
}

// Signed codebook of mxfp4/kernels.py:284-287 (entry 8 is +0.0).
__device__ __forceinline__ float cb16(int k) {
  float m = cb_rt((uint32_t)k & 7u);
  return k < 8 ? m : -m;  // (k = 8 gives -0.0: same deltas as the table's +0.0)
}
// The table entry itself, as stored in the output (entry 8 is +0.0).
__device__ __forceinline__ float cb16_entry(int k) { return k == 8 ? 0.0f : cb16(k); }

// argmin_k |x - s*cb16[k]| with torch.argmin semantics (the first NaN wins,
// else the first minimum).
__device__ __forceinline__ int argmin_index(float x, float s) {
  int best = 0;
  float bd = 0.0f;
  bool found_nan = false;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    float d = fabsf(__fsub_rn(x, __fmul_rn(s, cb16(k))));
    bool isn = d != d;
    if (!found_nan) {
      if (isn) { best = k; found_nan = true; }
      else if (k == 0 || d < bd) { bd = d; best = k; }
    }
  }
  return best;
}

template <int BS>
__device__ __forceinline__ float block_sse_argmin(const float (&x)[BS], float s) {
  float d2[BS];
#pragma unroll
  for (int i = 0; i < BS; ++i) {
    float d = __fsub_rn(x[i], __fmul_rn(s, cb16(argmin_index(x[i], s))));
    d2[i] = __fmul_rn(d, d);
  }
  return sum8<BS>(d2);
}

// Final quantization with scale s (any value, NaN included) and all outputs.

// Eight signed E2M1 codes of y[0..7] (hardware RN, saturating), element k in
// nibble k of the result (the packed storage order).
__device__ __forceinline__ uint32_t e2m1x8_rn(const float (&y)[8]) {
  uint32_t w;
  asm("{\n .reg .b8 b0, b1, b2, b3;\n"
      " cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n"
      " cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n"
      " mov.b32 %0, {b0, b1, b2, b3};\n}\n"
      : "=r"(w)
      : "f"(y[0]), "f"(y[1]), "f"(y[2]), "f"(y[3]), "f"(y[4]), "f"(y[5]), "f"(y[6]), "f"(y[7]));
  return w;
}

// Byte k of w (two codes) decoded to f16x2 bits (exact, signs kept).
template <int K>
__device__ __forceinline__ uint32_t e2m1x2_byte_to_h2(uint32_t w) {
  uint32_t h2;
  asm("{\n .reg .b8 b;\n .reg .b32 t;\n shr.b32 t, %1, %2;\n cvt.u8.u32 b, t;\n"
      " cvt.rn.f16x2.e2m1x2 %0, b;\n}\n"
      : "=r"(h2) : "r"(w), "n"(8 * K));
  return h2;
}

// q * s for both halves of a decoded f16x2 pair, s given as f16 bits (exact:
// E2M1 x E4M3 products have <= 6 significant bits and lie in [2^-10, 2688]);
// the -0 addend keeps the sign of a zero product (-0 * s = -0, as in torch).
__device__ __forceinline__ float2 h2_times_s(uint32_t q_h2, uint32_t s_h) {
  float d0, d1;
  asm("{\n .reg .b16 lo, hi, s;\n mov.b32 {lo, hi}, %2;\n cvt.u16.u32 s, %3;\n"
      " fma.rn.f32.f16 %0, lo, s, 0f80000000;\n fma.rn.f32.f16 %1, hi, s, 0f80000000;\n}\n"
      : "=f"(d0), "=f"(d1) : "r"(q_h2), "r"(s_h));
  return make_float2(d0, d1);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {  // exact inputs
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Outputs of one block from its packed codes (hardware path: finite s > 0).
template <int BS, int FMT>
__device__ __forceinline__ void write_outputs_hw(const QuantArgs& p, int64_t b, const uint32_t (&codes)[BS / 8],
                                                 float s) {
  if (p.scales) p.scales[b] = s;
  if (p.scale_codes) p.scale_codes[b] = (uint8_t)(FMT == kNVFP4 ? e4m3_code(s) : (__float_as_uint(s) >> 23));
  if (p.packed) {
    if constexpr (BS == 16) *reinterpret_cast<uint2*>(p.packed + b * 8) = make_uint2(codes[0], codes[1]);
    else *reinterpret_cast<uint4*>(p.packed + b * 16) = make_uint4(codes[0], codes[1], codes[2], codes[3]);
  }
  const uint32_t s_h = FMT == kNVFP4 ? (uint32_t)__half_as_ushort(__float2half_rn(s)) : 0u;
#pragma unroll
  for (int w = 0; w < BS / 8; ++w) {  // eight elements per step, stored as they are made
    float dq[8], q[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t h2;
      if (k == 0) h2 = e2m1x2_byte_to_h2<0>(codes[w]);
      else if (k == 1) h2 = e2m1x2_byte_to_h2<1>(codes[w]);
      else if (k == 2) h2 = e2m1x2_byte_to_h2<2>(codes[w]);
      else h2 = e2m1x2_byte_to_h2<3>(codes[w]);
      if (p.quants || FMT != kNVFP4) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h2));
        q[2 * k] = f.x;
        q[2 * k + 1] = f.y;
      }
      if constexpr (FMT == kNVFP4) {
        const float2 d = h2_times_s(h2, s_h);
        dq[2 * k] = d.x;
        dq[2 * k + 1] = d.y;
      } else {
        dq[2 * k] = __fmul_rn(q[2 * k], s);
        dq[2 * k + 1] = __fmul_rn(q[2 * k + 1], s);
      }
    }
    if (p.dq_bf16)
      reinterpret_cast<uint4*>(p.dq_bf16 + b * BS)[w] =
          make_uint4(pack_bf16x2(dq[0], dq[1]), pack_bf16x2(dq[2], dq[3]), pack_bf16x2(dq[4], dq[5]),
                     pack_bf16x2(dq[6], dq[7]));
    if (p.quants) {
      float4* o = reinterpret_cast<float4*>(p.quants + b * BS + 8 * w);
      o[0] = make_float4(q[0], q[1], q[2], q[3]);
      o[1] = make_float4(q[4], q[5], q[6], q[7]);
    }
    if (p.dq) {
      float4* o = reinterpret_cast<float4*>(p.dq + b * BS + 8 * w);
      o[0] = make_float4(dq[0], dq[1], dq[2], dq[3]);
      o[1] = make_float4(dq[4], dq[5], dq[6], dq[7]);
    }
  }
}

// NVINT4 outputs of one block (nvint4/reference.py:29-46): quants =
// clamp(round(x / s), -7, 7) with round half to even, dequant q * s.  For
// 16-bit input and a finite s > 0, q = rint(x * RN(1/s)) except at an exact
// tie |x - q s| == s/2 (q s exact), where an odd q moves to its even
// neighbour.  Otherwise the IEEE quotient with the reference's x86 NaN
// payloads: x's NaN, else s's, 0 / 0 the default NaN; the dequant takes the
// scale's NaN first.  packed: two's complement nibbles, element 2i low, 0x8
// for a NaN quant; scale code: the E4M3 byte of s.
template <int BS, int DT>
__device__ __forceinline__ void write_block_int4(const QuantArgs& p, int64_t b, const float (&x)[BS], float s) {
  const uint32_t sb = __float_as_uint(s);
  const bool fast = DT != kDtF32 && sb > 0u && sb < 0x7f800000u;
  const bool snan = is_nan_bits(sb & 0x7fffffffu);
  const float rc = fast ? __frcp_rn(s) : 0.0f;
  uint32_t words[BS / 8];
#pragma unroll
  for (int w = 0; w < BS / 8; ++w) {  // eight elements per step, stored as 16-byte vectors
    float q8[8], d8[8];
    uint32_t word = 0u;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float q = int4_q(x[8 * w + k], s, rc, fast, snan);
      const bool qn = is_nan_bits(__float_as_uint(q) & 0x7fffffffu);
      q8[k] = q;
      d8[k] = snan ? s : (qn ? q : __fmul_rn(q, s));
      word |= (qn ? 0x8u : ((uint32_t)__float2int_rn(q) & 0xfu)) << (4 * k);
    }
    words[w] = word;
    if (p.dq_bf16) {  // exact: the dequant has <= 7 significant bits
      uint32_t h[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        h[k] = (__float_as_uint(d8[2 * k]) >> 16) | (__float_as_uint(d8[2 * k + 1]) & 0xffff0000u);
      reinterpret_cast<uint4*>(p.dq_bf16 + b * BS)[w] = make_uint4(h[0], h[1], h[2], h[3]);
    }
    if (p.quants) {
      float4* o = reinterpret_cast<float4*>(p.quants + b * BS + 8 * w);
      o[0] = make_float4(q8[0], q8[1], q8[2], q8[3]);
      o[1] = make_float4(q8[4], q8[5], q8[6], q8[7]);
    }
    if (p.dq) {
      float4* o = reinterpret_cast<float4*>(p.dq + b * BS + 8 * w);
      o[0] = make_float4(d8[0], d8[1], d8[2], d8[3]);
      o[1] = make_float4(d8[4], d8[5], d8[6], d8[7]);
    }
  }
  if (p.scales) p.scales[b] = s;
  if (p.scale_codes) p.scale_codes[b] = (uint8_t)e4m3_code(s);
  if (p.packed) {
    if constexpr (BS == 16) *reinterpret_cast<uint2*>(p.packed + b * 8) = make_uint2(words[0], words[1]);
    else *reinterpret_cast<uint4*>(p.packed + b * 16) = make_uint4(words[0], words[1], words[2], words[3]);
  }
}

// INT8 outputs of one block (int8/reference.py:36-62): quants =
// clamp(round(x / s), -127, 127) by IEEE division with the reference's x86 NaN
// payloads, dequant fl(q s) (the scale's NaN first).  packed: one int8 per
// element (0x80 for a NaN quant); scale code: the E4M3 byte of 127 s (its
// index in the candidate table); dq_bf16 rounded to nearest.
template <int BS, int DT>
__device__ __forceinline__ void write_block_int8(const QuantArgs& p, int64_t b, const float (&x)[BS], float s) {
  const bool snan = is_nan_bits(__float_as_uint(s) & 0x7fffffffu);
#pragma unroll
  for (int w = 0; w < BS / 8; ++w) {  // eight elements per step, 16-byte / 8-byte stores
    float q8[8], d8[8];
    uint32_t bytes[2] = {0u, 0u};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float xv = x[8 * w + k];
      const uint32_t xb = __float_as_uint(xv);
      float q;
      if (is_nan_bits(xb & 0x7fffffffu)) q = __uint_as_float(xb | 0x00400000u);
      else if (snan) q = s;
      else if (s == 0.0f && xv == 0.0f) q = __uint_as_float(0xffc00000u);
      else {
        q = rintf(__fdiv_rn(xv, s));
        q = q < -127.0f ? -127.0f : (q > 127.0f ? 127.0f : q);
      }
      const bool qn = is_nan_bits(__float_as_uint(q) & 0x7fffffffu);
      q8[k] = q;
      d8[k] = snan ? s : (qn ? q : __fmul_rn(q, s));
      bytes[k / 4] |= (qn ? 0x80u : ((uint32_t)__float2int_rn(q) & 0xffu)) << (8 * (k % 4));
    }
    if (p.packed) reinterpret_cast<uint2*>(p.packed + b * BS)[w] = make_uint2(bytes[0], bytes[1]);
    if (p.dq_bf16) {
      uint32_t h[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        h[k] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(d8[2 * k])) |
               ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(d8[2 * k + 1])) << 16);
      reinterpret_cast<uint4*>(p.dq_bf16 + b * BS)[w] = make_uint4(h[0], h[1], h[2], h[3]);
    }
    if (p.quants) {
      float4* o = reinterpret_cast<float4*>(p.quants + b * BS + 8 * w);
      o[0] = make_float4(q8[0], q8[1], q8[2], q8[3]);
      o[1] = make_float4(q8[4], q8[5], q8[6], q8[7]);
    }
    if (p.dq) {
      float4* o = reinterpret_cast<float4*>(p.dq + b * BS + 8 * w);
      o[0] = make_float4(d8[0], d8[1], d8[2], d8[3]);
      o[1] = make_float4(d8[4], d8[5], d8[6], d8[7]);
    }
  }
  if (p.scales) p.scales[b] = s;
  if (p.scale_codes) p.scale_codes[b] = snan ? (uint8_t)0x7f : (uint8_t)table_count_below(s, false);
}

template <int BS, int FMT, int METHOD, int DT>
__device__ __forceinline__ void write_block(const QuantArgs& p, int64_t b, const float (&x)[BS], float s) {
  if constexpr (FMT == kNVINT4) {
    write_block_int4<BS, DT>(p, b, x, s);
    return;
  }
  if constexpr (FMT == kInt8) {
    write_block_int8<BS, DT>(p, b, x, s);
    return;
  }
  constexpr int MODE = Mode<FMT, DT>::v;
  float quant[BS];
  uint32_t nib[BS];
  const bool argmin = METHOD == kNaiveArgmin || METHOD == kTwoArgmin;
  const uint32_t sb = __float_as_uint(s);
  // hardware rounding: 16-bit input, finite s > 0, no NaN element (a NaN
  // element makes amax, hence s, NaN)
  if (!argmin && DT != kDtF32 && FMT != kTable && sb > 0u && sb < 0x7f800000u) {
    // Packed path: y = RN(x * c) + 0 makes -0 quantize to +0 (torch.sign(-0)
    // is 0) while a negative value that rounds to zero keeps code 8 (-0), the
    // reference's sign * 0; the hardware conversion gives sign and magnitude.
    const float c = __fmul_rn(__frcp_rn(s), kBiasDown);
    const uint64_t c2 = pk2(c, c), z2 = pk2(0.0f, 0.0f);
    uint32_t codes[BS / 8];
#pragma unroll
    for (int w = 0; w < BS / 8; ++w) {
      float y[8];
#pragma unroll
      for (int k = 0; k < 8; k += 2) {
        const float2 t = up2(fma2(pk2(x[8 * w + k], x[8 * w + k + 1]), c2, z2));
        y[k] = t.x;
        y[k + 1] = t.y;
      }
      codes[w] = e2m1x8_rn(y);
    }
    write_outputs_hw<BS, FMT>(p, b, codes, s);
    return;
  }
#pragma unroll
  for (int i = 0; i < BS; ++i) {
    if (argmin) {
      int k = argmin_index(x[i], s);
      quant[i] = cb16_entry(k);
      nib[i] = k < 8 ? k : (k == 8 ? 0 : 8 + (k - 8));
    } else {
      int idx = fp4_index<MODE>(fabsf(x[i]), s);
      float q = cb_rt((uint32_t)idx);
      quant[i] = x[i] > 0.0f ? q : (x[i] < 0.0f ? -q : 0.0f);  // torch.sign semantics
      nib[i] = (x[i] < 0.0f ? 8u : 0u) | ((x[i] > 0.0f || x[i] < 0.0f) ? (uint32_t)idx : 0u);
    }
  }
  const bool snan = is_nan_bits(__float_as_uint(s) & 0x7fffffffu);
  if (p.scales) p.scales[b] = s;
  if (p.scale_codes) {
    uint32_t code = FMT == kTable ? (uint32_t)table_count_below(s, false)
                    : (FMT == kNVFP4 ? e4m3_code(s) : (snan ? 0xffu : (__float_as_uint(s) >> 23)));
    p.scale_codes[b] = (uint8_t)code;
  }
  float dq[BS];
#pragma unroll
  for (int i = 0; i < BS; ++i) dq[i] = snan ? s : __fmul_rn(quant[i], s);
  if (p.quants) {
    float4* o = reinterpret_cast<float4*>(p.quants + b * BS);
#pragma unroll
    for (int v = 0; v < BS / 4; ++v)
      o[v] = make_float4(quant[4 * v], quant[4 * v + 1], quant[4 * v + 2], quant[4 * v + 3]);
  }
  if (p.dq) {
    float4* o = reinterpret_cast<float4*>(p.dq + b * BS);
#pragma unroll
    for (int v = 0; v < BS / 4; ++v)
      o[v] = make_float4(dq[4 * v], dq[4 * v + 1], dq[4 * v + 2], dq[4 * v + 3]);
  }
  if (p.dq_bf16) {
    uint4* o = reinterpret_cast<uint4*>(p.dq_bf16 + b * BS);
#pragma unroll
    for (int v = 0; v < BS / 8; ++v) {
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        w[k] = (__float_as_uint(dq[8 * v + 2 * k]) >> 16) |
               (__float_as_uint(dq[8 * v + 2 * k + 1]) & 0xffff0000u);
      o[v] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  if (p.packed) {
    uint32_t w[BS / 8];
#pragma unroll
    for (int v = 0; v < BS / 8; ++v) {
      uint32_t acc = 0;
#pragma unroll
      for (int k = 0; k < 8; ++k) acc |= nib[8 * v + k] << (4 * k);
      w[v] = acc;
    }
    if constexpr (BS == 16) {
      *reinterpret_cast<uint2*>(p.packed + b * 8) = make_uint2(w[0], w[1]);
    } else {
      *reinterpret_cast<uint4*>(p.packed + b * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

template <int BS>
__device__ __forceinline__ uint32_t abs_and_amax(const float (&x)[BS], float (&a)[BS]) {
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < BS; ++i) {
    uint32_t u = __float_as_uint(x[i]) & 0x7fffffffu;
    a[i] = __uint_as_float(u);
    m = max(m, u);  // NaN patterns compare above inf: NaN propagates like torch amax
  }
  return m;
}

// Largest magnitude of one block of 16-bit values, as raw 16-bit bits
// (unsigned compare of sign-cleared bits orders finite values, then inf, then
// NaN patterns: NaN propagates like torch amax).
template <int BS>
__device__ __forceinline__ uint32_t raw_amax16(const unsigned char* raw) {
  const uint4* p = reinterpret_cast<const uint4*>(raw);
  uint32_t m2 = 0;
#pragma unroll
  for (int v = 0; v < BS / 8; ++v) {
    const uint4 w = p[v];
    m2 = __vmaxu2(m2, w.x & 0x7fff7fffu);
    m2 = __vmaxu2(m2, w.y & 0x7fff7fffu);
    m2 = __vmaxu2(m2, w.z & 0x7fff7fffu);
    m2 = __vmaxu2(m2, w.w & 0x7fff7fffu);
  }
  return max(m2 & 0xffffu, m2 >> 16);
}

// Convert one block from raw shared memory to fp32.
template <int BS, int DT>
__device__ __forceinline__ void smem_block(const unsigned char* raw, float (&x)[BS]) {
  const uint4* p = reinterpret_cast<const uint4*>(raw);
  constexpr int kVec = BS * Elem<DT>::kSize / 16;
#pragma unroll
  for (int v = 0; v < kVec; ++v) {
    uint4 w = p[v];
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

// ---------------------------------------------------------------------------
// Per-warp geometry
// ---------------------------------------------------------------------------
constexpr int kWarps = 8;             // warps per CTA
constexpr int kThreads = kWarps * 32;

template <int BS, int FMT, int DT, int METHOD>
struct WarpGeom {
  static constexpr int kChunkBytes = 32 * BS * Elem<DT>::kSize;  // 1-4 KB
  static constexpr int kStages = kChunkBytes <= 2048 ? 4 : 2;
  static constexpr bool kCoop = METHOD == kSSE && FMT != kMXFP4;
  static constexpr int kCpi = 3;  // candidate codes per cooperative work item
  static constexpr int kRowBytes = kCoop ? 32 * BS * 4 : 0;     // |x| rows for cooperation
  static constexpr int kBytes = kStages * kChunkBytes + kRowBytes + (kCoop ? 32 * 8 + 64 * 4 : 0) +
                                kStages * 8;
  static constexpr int kBytesAligned = (kBytes + 127) / 128 * 128;
};

// Minimum resident CTAs per SM (register caps), chosen by measurement.
template <int BS, int FMT, int METHOD>
struct MinCtas {
  static constexpr int v = METHOD != kSSE ? 1 : (BS == 16 ? ((FMT == kNVFP4 || FMT == kNVINT4) ? 3 : 4) : 2);
};

// Where a warp's chunks come from.  A chunk is 32 consecutive blocks of one
// input; locate() maps a chunk index to its input bytes, its block count (32
// except at the end of an input) and its first block, advancing `cur`, an
// item cursor that only moves forward (a warp visits chunks in ascending
// order); outputs() gives the output pointers of item `cur`.
//   SingleSrc: one input (qz_quantize).
//   GroupSrc:  many inputs in one launch (qz_quantize_grouped), chunks
//              numbered item after item.
struct SingleSrc {
  const QuantArgs& p;
  __device__ __forceinline__ int64_t n_chunks() const { return (p.n_blocks + 31) / 32; }
  template <int CHUNK_BYTES>
  __device__ __forceinline__ void locate(int64_t ch, int& cur, const char*& x, int& nb, int64_t& blk0) const {
    (void)cur;
    x = static_cast<const char*>(p.x) + ch * (int64_t)CHUNK_BYTES;
    const int64_t left = p.n_blocks - ch * 32;
    nb = left < 32 ? (int)left : 32;
    blk0 = ch * 32;
  }
  __device__ __forceinline__ const QuantArgs& outputs(int) const { return p; }
};

struct GroupSrc {
  const GroupArgs& g;
  __device__ __forceinline__ int64_t n_chunks() const { return g.n_chunks; }
  template <int CHUNK_BYTES>
  __device__ __forceinline__ void locate(int64_t ch, int& cur, const char*& x, int& nb, int64_t& blk0) const {
    while (cur + 1 < g.n_items && ch >= g.item[cur + 1].chunk0) ++cur;
    const GroupItem& it = g.item[cur];
    const int64_t local = ch - it.chunk0;
    x = static_cast<const char*>(it.x) + local * (int64_t)CHUNK_BYTES;
    const int64_t left = it.n_blocks - local * 32;
    nb = left < 32 ? (int)left : 32;
    blk0 = local * 32;
  }
  __device__ __forceinline__ QuantArgs outputs(int cur) const {
    const GroupItem& it = g.item[cur];
    QuantArgs q{};
    q.x = it.x;
    q.n_blocks = it.n_blocks;
    q.scales = it.scales;
    q.quants = it.quants;
    q.dq = it.dq;
    q.scale_codes = it.scale_codes;
    q.packed = it.packed;
    q.dq_bf16 = it.dq_bf16;
    return q;
  }
};

// Naive / SSE / argmin methods: the work of one CTA.
template <int BS, int FMT, int METHOD, int DT, class Src>
__device__ __forceinline__ void quantize_cta(const Src& src, const float* table, int n_table) {
  using G = WarpGeom<BS, FMT, DT, METHOD>;
  constexpr int MODE = Mode<FMT, DT>::v;
  constexpr int S = G::kStages;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  CandTable& ctab = s_ctab;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (METHOD == kSSE || FMT == kTable || FMT == kInt8) {
    fill_cand_table<FMT>(ctab, table, n_table);
    __syncthreads();
  }
  unsigned char* wbase = smem_raw + warp * G::kBytesAligned;
  unsigned char* stage = wbase;                                  // S x chunk
  float* rows = reinterpret_cast<float*>(wbase + S * G::kChunkBytes);  // 32 x BS |x|
  unsigned long long* best = reinterpret_cast<unsigned long long*>(
      wbase + S * G::kChunkBytes + G::kRowBytes);                 // 32 keys
  int* incl = reinterpret_cast<int*>(best + (G::kCoop ? 32 : 0)); // 32 inclusive sums
  int* lo_s = incl + (G::kCoop ? 32 : 0);                         // 32 lows
  uint64_t* bar = reinterpret_cast<uint64_t*>(
      wbase + S * G::kChunkBytes + G::kRowBytes + (G::kCoop ? 32 * 8 + 64 * 4 : 0));

  const int64_t n_chunks = src.n_chunks();
  const int64_t gwarp = (int64_t)blockIdx.x * kWarps + warp;
  const int64_t nwarps = (int64_t)gridDim.x * kWarps;
  int issue_cur = 0, work_cur = 0;  // item cursors of the loads and of the work

  auto issue = [&](int64_t i) {  // lane 0 only
    int64_t ch = gwarp + i * nwarps;
    if (ch >= n_chunks) return;
    const char* xs;
    int nb;
    int64_t blk0;
    src.template locate<G::kChunkBytes>(ch, issue_cur, xs, nb, blk0);
    uint32_t bytes = (uint32_t)(nb * BS * Elem<DT>::kSize);
    uint64_t* b = bar + (i % S);
    mbar_arrive_expect_tx(b, bytes);
    bulk_load(stage + (i % S) * G::kChunkBytes, xs, bytes, b);
  };

  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(bar + s, 1);
    fence_barrier_init();
    for (int s = 0; s < S; ++s) issue(s);
  }
  __syncwarp();

  for (int64_t i = 0;; ++i) {
    const int64_t ch = gwarp + i * nwarps;
    if (ch >= n_chunks) break;
    const bool landed = mbar_wait_bounded(bar + (i % S), (uint32_t)((i / S) & 1), kDevErrLoadTimeout);
    if (!__all_sync(0xffffffffu, landed)) {  // the whole warp leaves together
      // a copy never landed: wait (bounded) for this warp's copies still in
      // flight, that one included, so none lands after the CTA has exited
      if (lane == 0)
        for (int64_t k = i; k < i + S && gwarp + k * nwarps < n_chunks; ++k)
          mbar_wait_bounded(bar + (k % S), (uint32_t)((k / S) & 1), kDevErrLoadTimeout);
      return;
    }
    const char* xs;
    int nbc;
    int64_t blk0;
    src.template locate<G::kChunkBytes>(ch, work_cur, xs, nbc, blk0);
    const auto& p = src.outputs(work_cur);
    const int64_t blk = blk0 + lane;
    const bool valid = lane < nbc;
    float x[BS];
    uint32_t amax16 = 0;  // 16-bit inputs: amax of the raw magnitudes, two per word
    if (valid) {
      const unsigned char* raw = stage + (i % S) * G::kChunkBytes + lane * BS * Elem<DT>::kSize;
      smem_block<BS, DT>(raw, x);
      if constexpr (DT != kDtF32) amax16 = raw_amax16<BS>(raw);
    } else {
#pragma unroll
      for (int k = 0; k < BS; ++k) x[k] = 0.0f;
    }
    __syncwarp();
    if (lane == 0) {
      fence_proxy_async_smem();
      issue(i + S);
    }

    float a[BS];
    uint32_t amax_bits;
    if constexpr (DT == kDtF32) {
      amax_bits = abs_and_amax<BS>(x, a);
    } else {
#pragma unroll
      for (int k = 0; k < BS; ++k) a[k] = fabsf(x[k]);
      amax_bits = DT == kDtBF16 ? amax16 << 16 : __float_as_uint(f16_bits_to_float(amax16));
    }
    float s = naive_scale<FMT>(amax_bits);
    const bool s_nan = is_nan_bits(__float_as_uint(s) & 0x7fffffffu);

    if constexpr (METHOD == kSSE && !G::kCoop) {
      // MXFP4: 1-4 power-of-two candidates per block; each lane walks its own
      // (the ascending loop with strict '<', clipping fast-fail omitted as above).
      if (valid && !s_nan) {
        const float E0 = base_sse<BS, MODE, DT, FMT>(a, s);
        int lo, hi;
        search_range<BS, FMT>(x, a, __uint_as_float(amax_bits), E0, lo, hi);
        float best_E = E0;
#pragma unroll 1
        for (int c = lo; c <= hi; ++c) {
          const float E = cand_sse<BS, MODE, DT, FMT>(a, ctab, c);
          if (E < best_E) { best_E = E; s = ctab.val[c]; }
        }
      }
    } else if constexpr (METHOD == kSSE) {
      // A NaN naive scale (NaN amax, or NVFP4 amax/6 > 464) makes the
      // reference's E0 and bounds NaN: no candidate is ever in range.
      int lo = 1, hi = 0;
      float E0 = 0.0f;
      float4* row = reinterpret_cast<float4*>(rows + lane * BS);
#pragma unroll
      for (int v = 0; v < BS / 4; ++v) row[v] = make_float4(a[4 * v], a[4 * v + 1], a[4 * v + 2], a[4 * v + 3]);
      if (valid && !s_nan) {
        if constexpr (FMT == kInt8) E0 = int8_sse_row<BS>(a, s, __frcp_rn(s), rows + lane * BS);
        else E0 = base_sse<BS, MODE, DT, FMT>(a, s);
        search_range<BS, FMT>(x, a, __uint_as_float(amax_bits), E0, lo, hi);
      }
      // Work items of CPI consecutive candidates of one block: the lookup, the
      // row reload and the atomic are paid once per item (the last item of a
      // block repeats its highest candidate, which cannot change the minimum).
      // The naive scale's own code is dropped when it is an end of [lo, hi]
      // (its SSE is E0 bit for bit and E0's key wins ties); it usually is lo.
      constexpr int CPI = G::kCpi;
      if (hi >= lo) {
        const int cn = (FMT == kTable || FMT == kInt8) ? table_count_below(s, false) : (int)e4m3_code(s);
        if (cn == lo) ++lo;
        else if (cn == hi) --hi;
      }
      const int n = hi >= lo ? hi - lo + 1 : 0;
      const int n_items = (n + CPI - 1) / CPI;

      int sc = n_items;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        int t = __shfl_up_sync(0xffffffffu, sc, o);
        if (lane >= o) sc += t;
      }
      incl[lane] = sc;
      lo_s[lane] = lo | (hi << 16);
      best[lane] = (unsigned long long)__float_as_uint(E0) << 32;
      const int total = __shfl_sync(0xffffffffu, sc, 31);
      __syncwarp();
      int bb = 0;
#pragma unroll 1
      for (int it = lane; it < total; it += 32) {
        while (it >= incl[bb]) ++bb;
        const int lh = lo_s[bb];
        const int c0 = (lh & 0xffff) + CPI * (it - (bb ? incl[bb - 1] : 0));
        const int ch = lh >> 16;
        float ar[BS];
        const float4* r4 = reinterpret_cast<const float4*>(rows + bb * BS);
#pragma unroll
        for (int v = 0; v < BS / 4; ++v) {
          float4 t = r4[v];
          ar[4 * v] = t.x; ar[4 * v + 1] = t.y; ar[4 * v + 2] = t.z; ar[4 * v + 3] = t.w;
        }
        unsigned long long key = ~0ull;
        if constexpr (FMT == kInt8) {
          // one copy of the 32-element body (instruction fetch, see int8_sse_row)
#pragma unroll 1
          for (int k = 0; k < CPI; ++k) {
            const int c = c0 + k <= ch ? c0 + k : ch;
            const float E = int8_sse_row<BS>(ar, ctab.val[c], __uint_as_float(ctab.cn[c].x), rows + bb * BS);
            const unsigned long long kk = ((unsigned long long)__float_as_uint(E) << 32) | (unsigned)(c + 1);
            key = kk < key ? kk : key;
          }
        } else {
#pragma unroll
          for (int k = 0; k < CPI; ++k) {
            const int c = c0 + k <= ch ? c0 + k : ch;
            const float E = cand_sse<BS, MODE, DT, FMT>(ar, ctab, c);
            // low word c + 1: 0 stays the naive scale, which wins ties
            const unsigned long long kk = ((unsigned long long)__float_as_uint(E) << 32) | (unsigned)(c + 1);
            key = kk < key ? kk : key;
          }
        }
        atomicMin(best + bb, key);
      }
      __syncwarp();
      const unsigned win = (unsigned)(best[lane] & 0xffffffffu);
      if (win != 0) s = ctab.val[win - 1];
      __syncwarp();  // rows/best are rewritten by the next chunk
    } else if constexpr (METHOD == kTwoArgmin) {
      if (valid && !s_nan) {
        int e0 = ue8m0_naive_exp(amax_bits);
        int e1 = e0 + 1 > 254 ? 254 : e0 + 1;
        float s1 = pow2f(e1 - 127);
        if (block_sse_argmin<BS>(x, s1) < block_sse_argmin<BS>(x, s)) s = s1;
      }
    }
    if (valid) write_block<BS, FMT, METHOD, DT>(p, blk, x, s);
  }
}

template <int BS, int FMT, int METHOD, int DT>
__global__ void __launch_bounds__(kThreads, MinCtas<BS, FMT, METHOD>::v) quantize_kernel(QuantArgs p) {
  quantize_cta<BS, FMT, METHOD, DT>(SingleSrc{p}, p.table, p.n_table);
}

// Many inputs in one persistent launch (NVFP4 / MXFP4, naive and SSE).
template <int BS, int FMT, int METHOD, int DT>
__global__ void __launch_bounds__(kThreads, MinCtas<BS, FMT, METHOD>::v)
    quantize_grouped_kernel(const __grid_constant__ GroupArgs g) {
  quantize_cta<BS, FMT, METHOD, DT>(GroupSrc{g}, nullptr, 0);
}

// Hessian method: CTA (j, row chunk); the CTA's H_j lives (transposed) in
// shared memory.  Each thread walks its block's candidates in ascending order
// with the reference's fast-fail rule, which does depend on the running best.
template <int BS, int FMT, int DT>
__global__ void __launch_bounds__(128, BS == 32 ? 3 : 1) hessian_kernel(QuantArgs p) {
  constexpr int MODE = Mode<FMT, DT>::v;
  __shared__ __align__(16) float Ht[BS * BS];
  const int64_t j = blockIdx.x;
  const float* Hg = p.h_blocks + j * (BS * BS);
  for (int i = threadIdx.x; i < BS * BS; i += blockDim.x) Ht[(i % BS) * BS + i / BS] = Hg[i];
  if (FMT == kTable || FMT == kInt8) fill_cand_table<FMT>(s_ctab, p.table, p.n_table);
  __syncthreads();
  const int64_t M = p.n_blocks / p.n_col_blocks;
  for (int64_t m = (int64_t)blockIdx.y * blockDim.x + threadIdx.x; m < M;
       m += (int64_t)gridDim.y * blockDim.x) {
    const int64_t b = m * p.n_col_blocks + j;
    float x[BS], a[BS];
    load_block<BS, DT>(p.x, b, x);
    uint32_t amax_bits = abs_and_amax<BS>(x, a);
    float s = naive_scale<FMT>(amax_bits);
    if (!is_nan_bits(__float_as_uint(s) & 0x7fffffffu)) {
      const float E0 = base_sse<BS, MODE, DT, FMT>(a, s);
      float best_E = block_hess_ilp<BS, MODE, DT, FMT>(x, a, s, Ht);
      int lo, hi;
      search_range<BS, FMT>(x, a, __uint_as_float(amax_bits), E0, lo, hi);
#pragma unroll 1
      for (int c = lo; c <= hi; ++c) {
        const float sc = cand_value<FMT>(c);
        const float Hc = block_clip<BS, FMT>(a, sc);
        // NVFP4 fast-fail: 10x the running Hessian best (nvfp4/reference.py:377);
        // MXFP4: the baseline SSE (mxfp4/reference.py:346).
        // (the exotic-grid experiment uses the NVFP4 rule: quant_exotic_scales.py:157)
        const bool pass = FMT != kMXFP4 ? (Hc < __fmul_rn(best_E, 10.0f)) : (Hc < E0);
        if (!pass) continue;
        const float E = block_hess_ilp<BS, MODE, DT, FMT>(x, a, sc, Ht);
        if (E < best_E) { best_E = E; s = sc; }
      }
    }
    write_block<BS, FMT, kHessian, DT>(p, b, x, s);
  }
}

// ---------------------------------------------------------------------------
// ADMM refinement (nvfp4/reference.py:410-534): one thread per block, CTA per
// column block j with H_j, H_j / lambda_max and inv(H_j / lambda_max + rho I)
// transposed in shared memory.  The reference stops all blocks once no scale
// changed; a block whose scale did not change reproduces itself exactly on
// another pass, so each block stops on its own (same results).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float quant_unit(float v) {  // fp4_quantize(v, 1)
  const float a = fabsf(v);
  int idx = 0;
#pragma unroll
  for (int k = 0; k < 7; ++k) idx += (a <= bnd(k)) ? 0 : 1;
  const float q = cb_rt((uint32_t)idx);
  return v > 0.0f ? q : (v < 0.0f ? -q : 0.0f);
}

// y = A v with A^T in shared memory (At[b*BS + a] = A[a][b]); every y[a] is a
// sequential FMA chain over b ascending.
// The chains of (y[2k], y[2k+1]) run as one packed fma.rn.f32x2 pair (two
// single-rounding FMAs: the scalar chains bit for bit).
template <int BS>
__device__ __forceinline__ void matvec_t(const float* __restrict__ At, const float (&v)[BS], float (&y)[BS]) {
  uint64_t y2[BS / 2];
#pragma unroll
  for (int k = 0; k < BS / 2; ++k) y2[k] = 0ull;
#pragma unroll
  for (int b = 0; b < BS; ++b) {
    const uint32_t row = smem_u32(At + b * BS);
    const uint64_t vb = pk2(v[b], v[b]);
#pragma unroll
    for (int q4 = 0; q4 < BS / 4; ++q4) {
      const float4 h = lds_f4(row + 16 * q4);
      y2[2 * q4 + 0] = fma2(pk2(h.x, h.y), vb, y2[2 * q4 + 0]);
      y2[2 * q4 + 1] = fma2(pk2(h.z, h.w), vb, y2[2 * q4 + 1]);
    }
  }
#pragma unroll
  for (int k = 0; k < BS / 2; ++k) {
    const float2 t = up2(y2[k]);
    y[2 * k] = t.x;
    y[2 * k + 1] = t.y;
  }
}

struct AdmmArgs {
  QuantArgs q;
  const float* h;     // (J, bs, bs)
  const float* hn;    // (J, bs, bs)
  const float* minv;  // (J, bs, bs)
  int n_outer, n_inner;
  float rho;
};

template <int BS, int DT>
__global__ void __launch_bounds__(64) admm_kernel(AdmmArgs A) {
  const QuantArgs& p = A.q;
  __shared__ __align__(16) float Ht[BS * BS], Hnt[BS * BS], Mt[BS * BS];
  const int64_t j = blockIdx.x;
  for (int i = threadIdx.x; i < BS * BS; i += blockDim.x) {
    const int t = (i % BS) * BS + i / BS;
    Ht[t] = A.h[j * BS * BS + i];
    Hnt[t] = A.hn[j * BS * BS + i];
    Mt[t] = A.minv[j * BS * BS + i];
  }
  __syncthreads();
  const int64_t M = p.n_blocks / p.n_col_blocks;
  for (int64_t m = (int64_t)blockIdx.y * blockDim.x + threadIdx.x; m < M; m += (int64_t)gridDim.y * blockDim.x) {
    const int64_t b = m * p.n_col_blocks + j;
    float x[BS], a[BS];
    load_block<BS, DT>(p.x, b, x);
    const uint32_t amax_bits = abs_and_amax<BS>(x, a);
    float s = naive_scale<kNVFP4>(amax_bits);
    float z[BS], u[BS], hw[BS], v[BS];
#pragma unroll
    for (int i = 0; i < BS; ++i) z[i] = 0.0f;
#pragma unroll 1
    for (int t = 0; t < A.n_outer; ++t) {
#pragma unroll
      for (int i = 0; i < BS; ++i) {
        v[i] = __fdiv_rn(x[i], s);  // w = x / s
        z[i] = quant_unit(v[i]);
        u[i] = 0.0f;
      }
      matvec_t<BS>(Hnt, v, hw);  // Hw = H_norm w
#pragma unroll 1
      for (int k = 0; k < A.n_inner; ++k) {
#pragma unroll
        for (int i = 0; i < BS; ++i) v[i] = __fadd_rn(hw[i], __fmul_rn(A.rho, __fsub_rn(z[i], u[i])));
        float q[BS];
        matvec_t<BS>(Mt, v, q);  // q = M_inv rhs
#pragma unroll
        for (int i = 0; i < BS; ++i) {
          z[i] = quant_unit(__fadd_rn(q[i], u[i]));
          u[i] = __fsub_rn(__fadd_rn(u[i], q[i]), z[i]);
        }
      }
      // scale update: s = E4M3(x^T H q* / q*^T H q*) where valid
      matvec_t<BS>(Ht, z, v);  // Hq
      float pn[BS], pd[BS];
#pragma unroll
      for (int i = 0; i < BS; ++i) {
        pn[i] = __fmul_rn(x[i], v[i]);
        pd[i] = __fmul_rn(z[i], v[i]);
      }
      const float numer = sum8<BS>(pn), denom = sum8<BS>(pd);
      const bool valid = numer > 0.0f && denom > 1e-12f;
      float sc = __fdiv_rn(numer, denom < 1e-12f ? 1e-12f : denom);
      sc = sc < 1e-12f ? 1e-12f : sc;
      const float s_new = valid ? e4m3_snap_nonneg(sc) : s;
      if (s_new == s) break;
      s = s_new;
    }
    // outputs: quants are the ADMM codes z (not a re-quantization of x)
    const bool snan = is_nan_bits(__float_as_uint(s) & 0x7fffffffu);
    if (p.scales) p.scales[b] = s;
    if (p.scale_codes) p.scale_codes[b] = (uint8_t)e4m3_code(s);
    float dq[BS];
    uint32_t nib[BS];
#pragma unroll
    for (int i = 0; i < BS; ++i) {
      dq[i] = snan ? s : __fmul_rn(z[i], s);
      const uint32_t zb = __float_as_uint(z[i]), mag = zb & 0x7fffffffu;
      const uint32_t idx = mag == 0u ? 0u : (mag == 0x3f000000u ? 1u : ((mag - 0x3f000000u) >> 22));
      nib[i] = ((zb >> 31) << 3) | idx;
    }
    if (p.quants) {
      float4* o = reinterpret_cast<float4*>(p.quants + b * BS);
#pragma unroll
      for (int k = 0; k < BS / 4; ++k) o[k] = make_float4(z[4 * k], z[4 * k + 1], z[4 * k + 2], z[4 * k + 3]);
    }
    if (p.dq) {
      float4* o = reinterpret_cast<float4*>(p.dq + b * BS);
#pragma unroll
      for (int k = 0; k < BS / 4; ++k) o[k] = make_float4(dq[4 * k], dq[4 * k + 1], dq[4 * k + 2], dq[4 * k + 3]);
    }
    if (p.dq_bf16) {
#pragma unroll
      for (int i = 0; i < BS; ++i) p.dq_bf16[b * BS + i] = (uint16_t)(__float_as_uint(dq[i]) >> 16);
    }
    if (p.packed) {
#pragma unroll
      for (int i = 0; i < BS; i += 2) p.packed[b * (BS / 2) + i / 2] = (uint8_t)(nib[i] | (nib[i + 1] << 4));
    }
  }
}

cudaError_t launch_admm(const QuantArgs& qa, const float* h, const float* hn, const float* minv, int n_outer,
                        int n_inner, float rho, int dtype, int bs, int num_sms, cudaStream_t st) {
  if (qa.n_blocks == 0) return cudaSuccess;
  AdmmArgs A{qa, h, hn, minv, n_outer, n_inner, rho};
  const int64_t M = qa.n_blocks / qa.n_col_blocks;
  int64_t gy = (M + 63) / 64;
  const int64_t per_j = ((int64_t)num_sms * 16 + qa.n_col_blocks - 1) / qa.n_col_blocks;
  gy = gy < per_j ? gy : per_j;
  gy = gy < 1 ? 1 : (gy > 65535 ? 65535 : gy);
  dim3 grid((unsigned)qa.n_col_blocks, (unsigned)gy);
  if (bs == 16) {
    if (dtype == kDtBF16) admm_kernel<16, kDtBF16><<<grid, 64, 0, st>>>(A);
    else if (dtype == kDtF16) admm_kernel<16, kDtF16><<<grid, 64, 0, st>>>(A);
    else admm_kernel<16, kDtF32><<<grid, 64, 0, st>>>(A);
  } else {
    if (dtype == kDtBF16) admm_kernel<32, kDtBF16><<<grid, 64, 0, st>>>(A);
    else if (dtype == kDtF16) admm_kernel<32, kDtF16><<<grid, 64, 0, st>>>(A);
    else admm_kernel<32, kDtF32><<<grid, 64, 0, st>>>(A);
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// GPTQ column group (experiments/quant_gptq_strided.py:49-135, gptq_strided).
// Rows are independent in GPTQ -- a row's later columns depend only on its own
// earlier errors and the shared inverse Hessian -- so each warp carries one
// row through the whole group: the row's group columns sit in shared memory,
// Hi's group block (and, for the Hessian method, the group's H_j) beside them
// for the CTA's kGptqRows warps.  For every column block, left to right:
//   scale search with the lanes spread over the candidates (each lane scores
//   candidates lo + lane, lo + lane + 32, ... with the same device code and
//   arithmetic as qz_quantize on fp32 input; SSE: minimum of the
//   (error, index) keys over the warp; Hessian: the reference's sequential
//   fast-fail scan over the precomputed values), dequantize, d = w - q,
//   err = d / Hi_cc, loss += d^2 / Hi_cc, then with the lanes over columns
//   W[later columns of the group] -= err @ Hi[block rows, those columns].
// The scaled errors leave as tf32 high / low pairs for the tensor-core update
// of the columns after the group (qz_gemm.cu).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

__device__ __forceinline__ unsigned long long warp_min_u64(unsigned long long k) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, k, o);
    k = t < k ? t : k;
  }
  return k;
}

// Scale of one fp32 block (every lane holds the block), chosen exactly as
// quantize_kernel (naive, SSE) and hessian_kernel (Hessian; Ht = H_j
// transposed in shared memory) choose it, with the candidates spread over the
// warp's lanes.
template <int BS, int FMT, int METHOD>
__device__ __forceinline__ float choose_scale_warp(const float (&x)[BS], const float* Ht, int lane) {
  constexpr int MODE = Mode<FMT, kDtF32>::v;
  float a[BS];
  const uint32_t amax_bits = abs_and_amax<BS>(x, a);
  float s = naive_scale<FMT>(amax_bits);
  if (METHOD == kNaive || is_nan_bits(__float_as_uint(s) & 0x7fffffffu)) return s;
  const float E0 = base_sse<BS, MODE, kDtF32, FMT>(a, s);
  int lo, hi;
  search_range<BS, FMT>(x, a, __uint_as_float(amax_bits), E0, lo, hi);
  if constexpr (METHOD == kSSE) {
    // first minimum of the error over [lo, hi], kept only below E0: the
    // reference's ascending loop with strict '<' (its clipping fast-fail never
    // changes the winner)
    unsigned long long key = (unsigned long long)__float_as_uint(E0) << 32;
    for (int c = lo + lane; c <= hi; c += 32) {
      const float E = cand_sse<BS, MODE, kDtF32, FMT>(a, s_ctab, c);
      const unsigned long long k = ((unsigned long long)__float_as_uint(E) << 32) | (unsigned)(c + 1);
      key = k < key ? k : key;
    }
    key = warp_min_u64(key);
    const unsigned win = (unsigned)(key & 0xffffffffu);
    return win ? s_ctab.val[win - 1] : s;
  } else {
    float best = block_hess_ilp<BS, MODE, kDtF32, FMT>(x, a, s, Ht);
    for (int base = lo; base <= hi; base += 32) {
      const int c = base + lane;
      float Hc = 0.0f, E = 0.0f;
      if (c <= hi) {
        const float sc = cand_value<FMT>(c);
        Hc = block_clip<BS, FMT>(a, sc);
        E = block_hess_ilp<BS, MODE, kDtF32, FMT>(x, a, sc, Ht);
      }
      const int n = hi - base + 1 < 32 ? hi - base + 1 : 32;
      for (int k = 0; k < n; ++k) {  // the reference's sequential scan (nvfp4/reference.py:367-393)
        const float hk = __shfl_sync(0xffffffffu, Hc, k), ek = __shfl_sync(0xffffffffu, E, k);
        const bool pass = FMT != kMXFP4 ? (hk < __fmul_rn(best, 10.0f)) : (hk < E0);
        if (pass && ek < best) { best = ek; s = cand_value<FMT>(base + k); }
      }
    }
    return s;
  }
}

template <int BS, int FMT, int METHOD>
__global__ void __launch_bounds__(kGptqRows * 32) gptq_group_kernel(GptqGroupArgs A) {
  constexpr int MODE = Mode<FMT, kDtF32>::v;
  extern __shared__ __align__(16) float gsm[];
  const int gc = A.gb * BS;  // columns of this group
  const int64_t c0 = (int64_t)A.g0 * BS;
  float* Hg = gsm;                    // gc x gc: Hi[c0 + r][c0 + c]
  float* hd = Hg + gc * gc;           // gc: Hi diagonal
  float* Hts = hd + gc;               // gb x BS x BS: H_j transposed (Hessian method)
  float* Wr = Hts + (METHOD == kHessian ? A.gb * BS * BS : 0);  // kGptqRows x gc: the warps' rows
  __shared__ double red[kGptqRows];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (METHOD != kNaive) fill_cand_table<FMT>(s_ctab);
  for (int i = threadIdx.x; i < gc * gc; i += blockDim.x) Hg[i] = A.Hi[(c0 + i / gc) * A.K + c0 + i % gc];
  for (int i = threadIdx.x; i < gc; i += blockDim.x) hd[i] = A.Hi[(c0 + i) * A.K + c0 + i];
  if (METHOD == kHessian)
    for (int i = threadIdx.x; i < A.gb * BS * BS; i += blockDim.x) {
      const int jj = i / (BS * BS), e = i % (BS * BS);
      Hts[jj * BS * BS + (e % BS) * BS + e / BS] = A.h_blocks[((int64_t)A.g0 + jj) * BS * BS + e];
    }
  const int64_t m = (int64_t)blockIdx.x * kGptqRows + warp;
  const bool valid = m < A.M;
  float* row = Wr + warp * gc;
  for (int c = lane; c < gc; c += 32)
    row[c] = valid ? A.Wb[(((int64_t)A.g0 + c / BS) * A.M + m) * BS + c % BS] : 0.0f;
  __syncthreads();
  double loss = 0.0;
  for (int jj = 0; jj < A.gb; ++jj) {
    float x[BS];
#pragma unroll
    for (int i = 0; i < BS; ++i) x[i] = row[jj * BS + i];
    const float s = choose_scale_warp<BS, FMT, METHOD>(x, Hts + jj * BS * BS, lane);
    const bool snan = is_nan_bits(__float_as_uint(s) & 0x7fffffffu);
    float err[BS];
    float dq_own = 0.0f, e_own = 0.0f;
#pragma unroll
    for (int i = 0; i < BS; ++i) {
      // fp4_quantize * s (the generic path of write_block for fp32 input)
      const float q = cb_rt((uint32_t)fp4_index<MODE>(fabsf(x[i]), s));
      const float qs = x[i] > 0.0f ? q : (x[i] < 0.0f ? -q : 0.0f);
      const float dq = snan ? s : __fmul_rn(qs, s);
      const float d = __fsub_rn(x[i], dq);
      const float h = hd[jj * BS + i];
      err[i] = __fdiv_rn(d, h);
      loss += (double)__fdiv_rn(__fmul_rn(d, d), h);
      if (i == lane) { dq_own = dq; e_own = err[i]; }
    }
    if (valid && lane < BS) {
      A.Qb[(((int64_t)A.g0 + jj) * A.M + m) * BS + lane] = dq_own;
      if (A.E) {
        float* e = A.E + m * 2 * A.gk + jj * BS + lane;
        const float hi = tf32_rna(e_own);
        e[0] = hi;
        e[A.gk] = tf32_rna(__fsub_rn(e_own, hi));
      }
    }
    // the rest of the group: W[c] -= sum_i err_i * Hi[block row i][c]
    for (int c = (jj + 1) * BS + lane; c < gc; c += 32) {
      float acc = 0.0f;
#pragma unroll
      for (int i = 0; i < BS; ++i) acc = __fmaf_rn(err[i], Hg[(jj * BS + i) * gc + c], acc);
      row[c] = __fsub_rn(row[c], acc);
    }
    __syncwarp();
  }
  if (lane == 0) red[warp] = valid ? loss : 0.0;
  __syncthreads();
  if (threadIdx.x == 0) {
    double sum = 0.0;
    for (int w = 0; w < kGptqRows; ++w) sum += red[w];
    A.loss[blockIdx.x] = sum;
  }
}

template <int BS, int FMT, int METHOD>
static cudaError_t launch_gptq_t(const GptqGroupArgs& a, cudaStream_t st) {
  const int gc = a.gb * BS;
  const size_t smem = ((size_t)gc * gc + gc + (METHOD == kHessian ? (size_t)a.gb * BS * BS : 0) +
                       (size_t)kGptqRows * gc) * 4;
  cudaError_t e = cudaFuncSetAttribute(gptq_group_kernel<BS, FMT, METHOD>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const unsigned grid = (unsigned)((a.M + kGptqRows - 1) / kGptqRows);
  gptq_group_kernel<BS, FMT, METHOD><<<grid, kGptqRows * 32, smem, st>>>(a);
  return cudaGetLastError();
}

template <int BS, int FMT>
static cudaError_t launch_gptq_m(const GptqGroupArgs& a, int method, cudaStream_t st) {
  if (method == kNaive) return launch_gptq_t<BS, FMT, kNaive>(a, st);
  if (method == kSSE) return launch_gptq_t<BS, FMT, kSSE>(a, st);
  if (method == kHessian) return launch_gptq_t<BS, FMT, kHessian>(a, st);
  return cudaErrorInvalidValue;
}

cudaError_t launch_gptq_group(const GptqGroupArgs& a, int bs, int fmt, int method, cudaStream_t st) {
  if (a.M == 0 || a.gb == 0) return cudaSuccess;
  if (bs == 16)
    return fmt == kNVFP4 ? launch_gptq_m<16, kNVFP4>(a, method, st) : launch_gptq_m<16, kMXFP4>(a, method, st);
  return fmt == kNVFP4 ? launch_gptq_m<32, kNVFP4>(a, method, st) : launch_gptq_m<32, kMXFP4>(a, method, st);
}

// ---------------------------------------------------------------------------
// host-side launch
// ---------------------------------------------------------------------------
template <int BS, int FMT, int METHOD, int DT>
static cudaError_t launch_q(const QuantArgs& p, int num_sms, cudaStream_t st) {
  using G = WarpGeom<BS, FMT, DT, METHOD>;
  const int smem = kWarps * G::kBytesAligned;
  // Set up once per instantiation and device (a benign race: every thread
  // computes the same values).
  static int s_per_sm[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  int per_sm = dev < 64 ? s_per_sm[dev] : 0;
  if (per_sm == 0) {
    e = cudaFuncSetAttribute(quantize_kernel<BS, FMT, METHOD, DT>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, quantize_kernel<BS, FMT, METHOD, DT>, kThreads,
                                                      smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    if (dev < 64) s_per_sm[dev] = per_sm;
  }
  const int64_t n_chunks = (p.n_blocks + 31) / 32;
  int64_t want = (n_chunks + kWarps - 1) / kWarps;
  int64_t cap = (int64_t)num_sms * per_sm;
  unsigned grid = (unsigned)(want < cap ? want : cap);
  quantize_kernel<BS, FMT, METHOD, DT><<<grid, kThreads, smem, st>>>(p);
  return cudaGetLastError();
}

template <int BS, int FMT, int METHOD, int DT>
static cudaError_t launch_g(const GroupArgs& g, int num_sms, cudaStream_t st) {
  using G = WarpGeom<BS, FMT, DT, METHOD>;
  const int smem = kWarps * G::kBytesAligned;
  static int s_per_sm[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  int per_sm = dev < 64 ? s_per_sm[dev] : 0;
  if (per_sm == 0) {
    e = cudaFuncSetAttribute(quantize_grouped_kernel<BS, FMT, METHOD, DT>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, quantize_grouped_kernel<BS, FMT, METHOD, DT>,
                                                      kThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    if (dev < 64) s_per_sm[dev] = per_sm;
  }
  const int64_t want = (g.n_chunks + kWarps - 1) / kWarps;
  const int64_t cap = (int64_t)num_sms * per_sm;
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  quantize_grouped_kernel<BS, FMT, METHOD, DT><<<grid, kThreads, smem, st>>>(g);
  return cudaGetLastError();
}

template <int BS, int FMT, int DT>
static cudaError_t launch_g_method(const GroupArgs& g, int method, int num_sms, cudaStream_t st) {
  if (method == kNaive) return launch_g<BS, FMT, kNaive, DT>(g, num_sms, st);
  if (method == kSSE) return launch_g<BS, FMT, kSSE, DT>(g, num_sms, st);
  return cudaErrorInvalidValue;
}

template <int BS, int FMT>
static cudaError_t launch_g_dtype(const GroupArgs& g, int dtype, int method, int num_sms, cudaStream_t st) {
  if (dtype == kDtBF16) return launch_g_method<BS, FMT, kDtBF16>(g, method, num_sms, st);
  if (dtype == kDtF16) return launch_g_method<BS, FMT, kDtF16>(g, method, num_sms, st);
  return launch_g_method<BS, FMT, kDtF32>(g, method, num_sms, st);
}

cudaError_t launch_quantize_grouped(const GroupArgs& g, int dtype, int bs, int fmt, int method, int num_sms,
                                    cudaStream_t st) {
  if (g.n_chunks == 0) return cudaSuccess;
  if (bs == 16)
    return fmt == kNVFP4 ? launch_g_dtype<16, kNVFP4>(g, dtype, method, num_sms, st)
                         : launch_g_dtype<16, kMXFP4>(g, dtype, method, num_sms, st);
  return fmt == kNVFP4 ? launch_g_dtype<32, kNVFP4>(g, dtype, method, num_sms, st)
                       : launch_g_dtype<32, kMXFP4>(g, dtype, method, num_sms, st);
}

template <int BS, int FMT, int DT>
static cudaError_t launch_fmt_dt(const QuantArgs& p, int method, int num_sms, cudaStream_t st) {
  if (method == kHessian) {
    const int64_t M = p.n_blocks / p.n_col_blocks;
    int64_t gy = (M + 127) / 128;
    int64_t want = (int64_t)num_sms * 16;
    int64_t per_j = (want + p.n_col_blocks - 1) / p.n_col_blocks;
    gy = gy < per_j ? gy : per_j;
    if (gy < 1) gy = 1;
    if (gy > 65535) gy = 65535;
    dim3 grid((unsigned)p.n_col_blocks, (unsigned)gy);
    hessian_kernel<BS, FMT, DT><<<grid, 128, 0, st>>>(p);
    return cudaGetLastError();
  }
  switch (method) {
    case kNaive: return launch_q<BS, FMT, kNaive, DT>(p, num_sms, st);
    case kSSE: return launch_q<BS, FMT, kSSE, DT>(p, num_sms, st);
    case kNaiveArgmin:
      if constexpr (FMT == kMXFP4) return launch_q<BS, FMT, kNaiveArgmin, DT>(p, num_sms, st);
      return cudaErrorInvalidValue;
    case kTwoArgmin:
      if constexpr (FMT == kMXFP4) return launch_q<BS, FMT, kTwoArgmin, DT>(p, num_sms, st);
      return cudaErrorInvalidValue;
    default: return cudaErrorInvalidValue;
  }
}

template <int BS, int FMT>
static cudaError_t launch_fmt(const QuantArgs& p, int dtype, int method, int sms, cudaStream_t st) {
  switch (dtype) {
    case kDtBF16: return launch_fmt_dt<BS, FMT, kDtBF16>(p, method, sms, st);
    case kDtF16: return launch_fmt_dt<BS, FMT, kDtF16>(p, method, sms, st);
    default: return launch_fmt_dt<BS, FMT, kDtF32>(p, method, sms, st);
  }
}

cudaError_t launch_quantize_table(const QuantArgs& p, int dtype, int bs, int method, int num_sms,
                                  cudaStream_t st) {
  if (p.n_blocks == 0) return cudaSuccess;
  return bs == 16 ? launch_fmt<16, kTable>(p, dtype, method, num_sms, st)
                  : launch_fmt<32, kTable>(p, dtype, method, num_sms, st);
}

template <int BS, int DT>
static cudaError_t launch_hessian_nvint4(const QuantArgs& p, int num_sms, cudaStream_t st) {
  const int64_t M = p.n_blocks / p.n_col_blocks;
  int64_t gy = (M + 127) / 128;
  const int64_t want = (int64_t)num_sms * 16;
  const int64_t per_j = (want + p.n_col_blocks - 1) / p.n_col_blocks;
  gy = gy < per_j ? gy : per_j;
  if (gy < 1) gy = 1;
  if (gy > 65535) gy = 65535;
  hessian_kernel<BS, kNVINT4, DT><<<dim3((unsigned)p.n_col_blocks, (unsigned)gy), 128, 0, st>>>(p);
  return cudaGetLastError();
}

// NVINT4 on the per-thread-block kernels (INT8 runs in qz_int.cu).
template <int BS>
static cudaError_t launch_nvint4_bs(const QuantArgs& p, int dtype, int method, int sms, cudaStream_t st) {
  if (method == kHessian) {
    if (dtype == kDtBF16) return launch_hessian_nvint4<BS, kDtBF16>(p, sms, st);
    if (dtype == kDtF16) return launch_hessian_nvint4<BS, kDtF16>(p, sms, st);
    return launch_hessian_nvint4<BS, kDtF32>(p, sms, st);
  }
  if (method == kNaive) {
    if (dtype == kDtBF16) return launch_q<BS, kNVINT4, kNaive, kDtBF16>(p, sms, st);
    if (dtype == kDtF16) return launch_q<BS, kNVINT4, kNaive, kDtF16>(p, sms, st);
    return launch_q<BS, kNVINT4, kNaive, kDtF32>(p, sms, st);
  }
  if (method == kSSE) {
    if (dtype == kDtBF16) return launch_q<BS, kNVINT4, kSSE, kDtBF16>(p, sms, st);
    if (dtype == kDtF16) return launch_q<BS, kNVINT4, kSSE, kDtF16>(p, sms, st);
    return launch_q<BS, kNVINT4, kSSE, kDtF32>(p, sms, st);
  }
  return cudaErrorInvalidValue;
}

// INT8 at block 32 on the per-thread-block kernels (larger blocks run in qz_int.cu).
template <int DT>
static cudaError_t launch_hessian_int8_bs32(const QuantArgs& p, int num_sms, cudaStream_t st) {
  const int64_t M = p.n_blocks / p.n_col_blocks;
  int64_t gy = (M + 127) / 128;
  const int64_t want = (int64_t)num_sms * 16;
  const int64_t per_j = (want + p.n_col_blocks - 1) / p.n_col_blocks;
  gy = gy < per_j ? gy : per_j;
  if (gy < 1) gy = 1;
  if (gy > 65535) gy = 65535;
  hessian_kernel<32, kInt8, DT><<<dim3((unsigned)p.n_col_blocks, (unsigned)gy), 128, 0, st>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_quantize_int8_bs32(const QuantArgs& p, int dtype, int method, int num_sms, cudaStream_t st) {
  if (p.n_blocks == 0) return cudaSuccess;
  if (method == kHessian) {
    if (dtype == kDtBF16) return launch_hessian_int8_bs32<kDtBF16>(p, num_sms, st);
    if (dtype == kDtF16) return launch_hessian_int8_bs32<kDtF16>(p, num_sms, st);
    return launch_hessian_int8_bs32<kDtF32>(p, num_sms, st);
  }
  if (method == kNaive) {
    if (dtype == kDtBF16) return launch_q<32, kInt8, kNaive, kDtBF16>(p, num_sms, st);
    if (dtype == kDtF16) return launch_q<32, kInt8, kNaive, kDtF16>(p, num_sms, st);
    return launch_q<32, kInt8, kNaive, kDtF32>(p, num_sms, st);
  }
  if (method == kSSE) {
    if (dtype == kDtBF16) return launch_q<32, kInt8, kSSE, kDtBF16>(p, num_sms, st);
    if (dtype == kDtF16) return launch_q<32, kInt8, kSSE, kDtF16>(p, num_sms, st);
    return launch_q<32, kInt8, kSSE, kDtF32>(p, num_sms, st);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_quantize_nvint4(const QuantArgs& p, int dtype, int bs, int method, int num_sms, cudaStream_t st) {
  if (p.n_blocks == 0) return cudaSuccess;
  return bs == 16 ? launch_nvint4_bs<16>(p, dtype, method, num_sms, st)
                  : launch_nvint4_bs<32>(p, dtype, method, num_sms, st);
}

cudaError_t launch_quantize(const QuantArgs& p, int dtype, int bs, int fmt, int method,
                            int num_sms, cudaStream_t st) {
  if (p.n_blocks == 0) return cudaSuccess;
  if (bs == 16)
    return fmt == kNVFP4 ? launch_fmt<16, kNVFP4>(p, dtype, method, num_sms, st)
                         : launch_fmt<16, kMXFP4>(p, dtype, method, num_sms, st);
  return fmt == kNVFP4 ? launch_fmt<32, kNVFP4>(p, dtype, method, num_sms, st)
                       : launch_fmt<32, kMXFP4>(p, dtype, method, num_sms, st);
}

// Self-test of the bounded wait: one warp waits on an mbarrier that nothing
// ever arrives on.  The wait gives up after limit_ns, sets kDevErrLoadTimeout
// in this unit's error flag and the kernel returns normally; no copy or
// tensor-core operation is in flight, so the context stays usable.
__global__ void __launch_bounds__(32) wait_selftest_kernel(uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncwarp();
  mbar_wait_bounded(&bar, 0u, kDevErrLoadTimeout, limit_ns);  // phase 0 never completes
}

cudaError_t launch_wait_selftest(uint64_t limit_ns, cudaStream_t st) {
  wait_selftest_kernel<<<1, 32, 0, st>>>(limit_ns);
  return cudaGetLastError();
}

cudaError_t read_device_error_quantize(unsigned* out, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(out, qz_device_error, sizeof(unsigned));
  if (e != cudaSuccess || !clear) return e;
  unsigned zero = 0;
  return cudaMemcpyToSymbol(qz_device_error, &zero, sizeof(unsigned));
}

}  // namespace qz
