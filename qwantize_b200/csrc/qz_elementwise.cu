// qz_elementwise.cu -- HBM-bound kernels: dequantize (fp32 and packed storage),
// fp4 nibble unpack, and the weight-error sums of compute_metrics.
// Grid-stride loops over 16-byte vectors, grids sized to a multiple of the SM
// count.
#include "qz_common.cuh"
#include "qz_kernels.h"

namespace qz {

// quants * scales with the NaN payload the reference's CPU
// `quants * scales.unsqueeze(dim)` returns: the scale's NaN if the scale is NaN,
// else the quant's (quieted); torch's multiply kernel puts its second operand
// first (measured for broadcast and contiguous operands).
__device__ __forceinline__ float mul_x86(float q, float s) {
  float r = __fmul_rn(q, s);
  if (r != r) {
    uint32_t qb = __float_as_uint(q), sb = __float_as_uint(s);
    if (is_nan_bits(sb & 0x7fffffffu)) return __uint_as_float(sb | 0x00400000u);
    if (is_nan_bits(qb & 0x7fffffffu)) return __uint_as_float(qb | 0x00400000u);
    return __uint_as_float(0xffc00000u);  // inf * 0: x86 default NaN
  }
  return r;
}

// nvfp4/reference.py:537-549, blocked layout; one float4 per thread step.
__global__ void dequantize_kernel(const float* __restrict__ scales, const float4* __restrict__ q,
                                  int64_t n_vec, int shift_vec_per_block, float4* __restrict__ out) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_vec; i += stride) {
    float s = __ldg(scales + (i >> shift_vec_per_block));
    float4 v = __ldg(q + i);
    out[i] = make_float4(mul_x86(v.x, s), mul_x86(v.y, s), mul_x86(v.z, s), mul_x86(v.w, s));
  }
}

__device__ __forceinline__ float e2m1_value(uint32_t nib) {
  float m = cb_rt(nib & 7u);
  return (nib & 8u) ? -m : m;
}

__device__ __forceinline__ float code_to_scale(uint32_t c, int fmt) {
  if (fmt == kNVFP4) {
    uint32_t m = c & 0x7fu;
    if (m == 0x7fu) return __uint_as_float(kNvNanBits);
    float v = m == 0 ? 0.0f : e4m3_value((int)m);
    return (c & 0x80u) ? -v : v;
  }
  if (c == 0xffu) return __uint_as_float(kMxNanBits);
  if (c == 0) return __uint_as_float(0x00400000u);  // 2^-127 (subnormal fp32)
  return pow2f((int)c - 127);
}

// One thread per 8 elements (4 packed bytes).
__global__ void dequantize_packed_kernel(const uint32_t* __restrict__ packed,
                                         const uint8_t* __restrict__ codes, int64_t n_words,
                                         int words_per_block_shift, int fmt,
                                         float4* __restrict__ out_f32, uint4* __restrict__ out_bf16) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_words; i += stride) {
    float s = code_to_scale(__ldg(codes + (i >> words_per_block_shift)), fmt);
    uint32_t w = __ldg(packed + i);
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float q = e2m1_value((w >> (4 * k)) & 0xfu);
      v[k] = (s != s) ? s : __fmul_rn(q, s);
    }
    if (out_f32) {
      out_f32[2 * i] = make_float4(v[0], v[1], v[2], v[3]);
      out_f32[2 * i + 1] = make_float4(v[4], v[5], v[6], v[7]);
    }
    if (out_bf16) {
      uint32_t h[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        h[k] = (__float_as_uint(v[2 * k]) >> 16) | (__float_as_uint(v[2 * k + 1]) & 0xffff0000u);
      out_bf16[i] = make_uint4(h[0], h[1], h[2], h[3]);
    }
  }
}

// fp4.py:117-254: nibble bits 0-2 index {0,1,2,3,4,6,8,12}, bit 3 = sign.
__global__ void unpack_kernel(const uint32_t* __restrict__ in, int64_t n_words,
                              uint2* __restrict__ out) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_words; i += stride) {
    uint32_t w = __ldg(in + i), o[2] = {0, 0};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      uint32_t nib = (w >> (4 * k)) & 0xfu;
      uint32_t mag = (0xC8643210u >> (4 * (nib & 7u))) & 0xfu;
      uint32_t v = (nib & 8u) ? ((0u - mag) & 0xffu) : mag;
      o[k >> 2] |= v << (8 * (k & 3));
    }
    out[i] = make_uint2(o[0], o[1]);
  }
}

template <int DT>
__device__ __forceinline__ float load1(const void* p, int64_t i) {
  if (DT == kDtF32) return __ldg(static_cast<const float*>(p) + i);
  uint32_t h = __ldg(static_cast<const unsigned short*>(p) + i);
  return DT == kDtBF16 ? bf16_bits_to_float(h) : f16_bits_to_float(h);
}

// sums[0] += sum (dq - w)^2, sums[1] += sum w^2 (double), metrics.py:23-27.
template <int WDT, int DDT>
__global__ void weight_sums_kernel(const void* __restrict__ W, const void* __restrict__ Wdq, int64_t n,
                                   double* __restrict__ sums) {
  double e = 0.0, w2 = 0.0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    double w = load1<WDT>(W, i), d = (double)load1<DDT>(Wdq, i) - w;
    e += d * d;
    w2 += w * w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    e += __shfl_xor_sync(0xffffffffu, e, o);
    w2 += __shfl_xor_sync(0xffffffffu, w2, o);
  }
  __shared__ double red[2][32];
  int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) { red[0][wid] = e; red[1][wid] = w2; }
  __syncthreads();
  if (threadIdx.x == 0) {
    double a = 0, b = 0;
    for (int k = 0; k < (int)(blockDim.x >> 5); ++k) { a += red[0][k]; b += red[1][k]; }
    atomicAdd(sums, a);
    atomicAdd(sums + 1, b);
  }
}

static unsigned grid_for(int64_t n_items, int threads, int num_sms, int per_sm = 8) {
  int64_t g = (n_items + threads - 1) / threads, cap = (int64_t)num_sms * per_sm;
  return (unsigned)(g < cap ? (g < 1 ? 1 : g) : cap);
}

cudaError_t launch_dequantize(const float* scales, const float* quants, int64_t n_blocks, int bs,
                              float* out, int num_sms, cudaStream_t st) {
  int64_t n_vec = n_blocks * bs / 4;
  if (n_vec == 0) return cudaSuccess;
  dequantize_kernel<<<grid_for(n_vec, 256, num_sms), 256, 0, st>>>(
      scales, reinterpret_cast<const float4*>(quants), n_vec, __builtin_ctz((unsigned)bs) - 2,
      reinterpret_cast<float4*>(out));
  return cudaGetLastError();
}

cudaError_t launch_dequantize_packed(const uint8_t* packed, const uint8_t* codes, int64_t n_blocks,
                                     int bs, int fmt, float* out_f32, uint16_t* out_bf16,
                                     int num_sms, cudaStream_t st) {
  int64_t n_words = n_blocks * bs / 8;
  if (n_words == 0) return cudaSuccess;
  dequantize_packed_kernel<<<grid_for(n_words, 256, num_sms), 256, 0, st>>>(
      reinterpret_cast<const uint32_t*>(packed), codes, n_words, bs == 16 ? 1 : 2, fmt,
      reinterpret_cast<float4*>(out_f32), reinterpret_cast<uint4*>(out_bf16));
  return cudaGetLastError();
}

cudaError_t launch_unpack(const uint8_t* packed, int64_t n_bytes, int8_t* out, int num_sms,
                          cudaStream_t st) {
  int64_t n_words = n_bytes / 4;
  if (n_words == 0) return cudaSuccess;
  unpack_kernel<<<grid_for(n_words, 256, num_sms), 256, 0, st>>>(
      reinterpret_cast<const uint32_t*>(packed), n_words, reinterpret_cast<uint2*>(out));
  return cudaGetLastError();
}

template <int WDT>
static void launch_ws(const void* W, const void* Wdq, int ddt, int64_t n, double* sums,
                      unsigned g, cudaStream_t st) {
  if (ddt == kDtF32) weight_sums_kernel<WDT, kDtF32><<<g, 256, 0, st>>>(W, Wdq, n, sums);
  else if (ddt == kDtBF16) weight_sums_kernel<WDT, kDtBF16><<<g, 256, 0, st>>>(W, Wdq, n, sums);
  else weight_sums_kernel<WDT, kDtF16><<<g, 256, 0, st>>>(W, Wdq, n, sums);
}

cudaError_t launch_weight_sums(const void* W, int wdt, const void* Wdq, int ddt, int64_t n,
                               double* sums, int num_sms, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  unsigned g = grid_for(n, 256, num_sms, 4);
  if (wdt == kDtF32) launch_ws<kDtF32>(W, Wdq, ddt, n, sums, g, st);
  else if (wdt == kDtBF16) launch_ws<kDtBF16>(W, Wdq, ddt, n, sums, g, st);
  else launch_ws<kDtF16>(W, Wdq, ddt, n, sums, g, st);
  return cudaGetLastError();
}

// x = hi + lo with hi = tf32(x) (round to nearest, ties away) and lo = tf32(x -
// hi): the operand split of the three-product tf32 GEMM (hi*hi + hi*lo +
// lo*hi) that keeps GPTQ's error update at fp32 accuracy on the tensor cores.
__global__ void split_tf32_kernel(const float4* __restrict__ src, float4* __restrict__ hi, float4* __restrict__ lo,
                                  int64_t n4) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 v = src[i];
    float in[4] = {v.x, v.y, v.z, v.w}, h[4], l[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t r;
      asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(in[k]));
      h[k] = __uint_as_float(r);
      asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(__fsub_rn(in[k], h[k])));
      l[k] = __uint_as_float(r);
    }
    hi[i] = make_float4(h[0], h[1], h[2], h[3]);
    lo[i] = make_float4(l[0], l[1], l[2], l[3]);
  }
}

cudaError_t launch_split_tf32(const float* src, float* hi, float* lo, int64_t n, int num_sms, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  split_tf32_kernel<<<(unsigned)(num_sms * 8), 256, 0, st>>>(reinterpret_cast<const float4*>(src),
                                                            reinterpret_cast<float4*>(hi),
                                                            reinterpret_cast<float4*>(lo), n / 4);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Pieces of the symmetric-positive-definite inverse (qz_spd_inverse).  Every
// matrix is fp32 row-major with leading dimension ld; its tf32 high / low
// split lives in a stacked buffer (high part at S[i], low part at S[i + lo]).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void store_split(float* S, int64_t i, int64_t lo, float v) {
  uint32_t h, l;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(v));
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(l) : "f"(__fsub_rn(v, __uint_as_float(h))));
  S[i] = __uint_as_float(h);
  S[i + lo] = __uint_as_float(l);
}

// In-place inverse of one s x s diagonal block (s <= 96, a multiple of 32)
// by the symmetric Gauss-Jordan sweep without pivoting, in double precision (a
// symmetric positive definite matrix needs no pivoting; a pivot <= 0 means the
// input is not positive definite: *bad is set).
//
// After the pivots of a set P are swept, the matrix is [A_PP^-1, A_PP^-1 A_PQ;
// -A_QP A_PP^-1, Schur complement] (Q the rest): the P x P and Q x Q blocks are
// symmetric and the P x Q block is minus the transpose of the Q x P block.  So
// only the upper triangle is kept and updated, and the pivot's row and column
// both come from its "cross" u (u[k] = U[p][k] for k >= p, U[k][p] for k < p):
// column p is u, row p is u with the swept entries (k < p) negated.
//
// The block lives in a D x D frame (D = 64 or 96, the smallest >= s;
// identity outside s) over 16 x 16 threads, each holding the (D/16)^2 elements
// (rows ty + 16a, columns tx + 16b) in registers; per pivot only its cross
// passes through shared memory (two buffers, so one barrier per pivot).
// Double precision is slow on this part (a pivot costs about 1 us, mostly the
// latency of its dependent double operations), so frames follow s, only the
// upper triangle's elements are updated, and the recursion stops at 96.
template <int D>
__global__ void __launch_bounds__(256) spd_block_inverse_kernel(float* V, float* S, int64_t ld, int64_t lo, int s,
                                                                int* bad) {
  constexpr int E = D / 16;
  __shared__ double cross[2][D];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  double A[E][E];
#pragma unroll
  for (int a = 0; a < E; ++a)
#pragma unroll
    for (int b = 0; b < E; ++b) {
      const int i = ty + 16 * a, j = tx + 16 * b;
      A[a][b] = (i < s && j < s) ? (double)V[i * ld + j] : (i == j ? 1.0 : 0.0);
    }
  for (int p = 0; p < s; ++p) {
    const int buf = p & 1, pa = p >> 4, pr = p & 15;
    if (ty == pr) {  // row p: the cross at k >= p
#pragma unroll
      for (int b = 0; b < E; ++b) {
        double v = 0.0;
#pragma unroll
        for (int a = 0; a < E; ++a) v = a == pa ? A[a][b] : v;
        if (tx + 16 * b >= p) cross[buf][tx + 16 * b] = v;
      }
    }
    if (tx == pr) {  // column p: the cross at k < p
#pragma unroll
      for (int a = 0; a < E; ++a) {
        double v = 0.0;
#pragma unroll
        for (int b = 0; b < E; ++b) v = b == pa ? A[a][b] : v;
        if (ty + 16 * a < p) cross[buf][ty + 16 * a] = v;
      }
    }
    __syncthreads();
    const double piv = cross[buf][p];
    if (threadIdx.x == 0 && !(piv > 0.0)) atomicExch(bad, 1);
    const double d = 1.0 / piv;
    double ui[E], uj[E], fi[E], rj[E];
#pragma unroll
    for (int a = 0; a < E; ++a) {
      ui[a] = cross[buf][ty + 16 * a];
      fi[a] = ui[a] * d;  // column p, scaled
    }
#pragma unroll
    for (int b = 0; b < E; ++b) {
      uj[b] = cross[buf][tx + 16 * b];
      rj[b] = tx + 16 * b < p ? -uj[b] : uj[b];  // row p
    }
#pragma unroll
    for (int a = 0; a < E; ++a)
#pragma unroll
      for (int b = a + 1; b < E; ++b) A[a][b] = fma(-fi[a], rj[b], A[a][b]);
    if (ty <= tx) {
#pragma unroll
      for (int a = 0; a < E; ++a) A[a][a] = fma(-fi[a], rj[a], A[a][a]);
    }
    // row p (k > p): u d; column p (k < p): -u d; the pivot: d
    if (ty == pr) {
#pragma unroll
      for (int a = 0; a < E; ++a)
        if (a == pa)
#pragma unroll
          for (int b = 0; b < E; ++b) {
            const int j = tx + 16 * b;
            if (j > p) A[a][b] = uj[b] * d;
            else if (j == p) A[a][b] = d;
          }
    }
    if (tx == pr) {
#pragma unroll
      for (int b = 0; b < E; ++b)
        if (b == pa)
#pragma unroll
          for (int a = 0; a < E; ++a)
            if (ty + 16 * a < p) A[a][b] = -ui[a] * d;
    }
  }
  // the upper triangle is the inverse; write it and its mirror (through a
  // shared-memory transpose, so the stores stay row-contiguous)
  extern __shared__ float tr[];  // D x (D + 1)
#pragma unroll
  for (int a = 0; a < E; ++a)
#pragma unroll
    for (int b = 0; b < E; ++b) tr[(ty + 16 * a) * (D + 1) + tx + 16 * b] = (float)A[a][b];
  __syncthreads();
#pragma unroll
  for (int a = 0; a < E; ++a)
#pragma unroll
    for (int b = 0; b < E; ++b) {
      const int i = ty + 16 * a, j = tx + 16 * b;
      if (i < s && j < s) {
        const float v = i <= j ? tr[i * (D + 1) + j] : tr[j * (D + 1) + i];
        V[i * ld + j] = v;
        store_split(S, i * ld + j, lo, v);
      }
    }
}

template <int D>
static cudaError_t spd_block_launch(float* V, float* S, int64_t ld, int64_t lo, int s, int* bad, cudaStream_t st) {
  const int smem = D * (D + 1) * 4;
  cudaError_t e = cudaFuncSetAttribute(spd_block_inverse_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  spd_block_inverse_kernel<D><<<1, 256, smem, st>>>(V, S, ld, lo, s, bad);
  return cudaGetLastError();
}

cudaError_t launch_spd_block_inverse(float* V, float* S, int64_t ld, int64_t lo, int s, int* bad, cudaStream_t st) {
  if (s <= 64) return spd_block_launch<64>(V, S, ld, lo, s, bad, st);
  if (s <= 96) return spd_block_launch<96>(V, S, ld, lo, s, bad, st);
  return cudaErrorInvalidValue;
}


}  // namespace qz
