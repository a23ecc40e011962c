// qz_int.cu -- INT8 block quantization for blocks of 64, 128 and 256
// (int8/reference.py): q = clamp(round(x / s), -127, 127), round half to even,
// s = e4m3(max(amax, 1e-12)) / 127, candidates E4M3 / 127, on the search
// skeleton of NVFP4 (naive scale, SSE bounds, bounded exhaustive search,
// Hessian variant).  NVINT4 and INT8 at block 32 fit one lane per block and run
// on the per-thread-block kernels of qz_quantize.cu.
//
// Layout: eight lanes per block (a warp holds four consecutive blocks); lane
// g of a group holds elements g, g+8, g+16, ...  With that layout torch's CPU
// row-sum order for rows of >= 32 (32 accumulators at stride 32, combined as
// ((acc[m] + acc[m+8]) + acc[m+16]) + acc[m+24], then a left fold) is local to
// each lane, followed by one left fold over the eight lanes.  The bounds need
// |x| sorted: a bitonic network in shared memory, then the sequential fp64
// prefix (torch.cumsum) with early exit (the prefix sums are non-decreasing).
// Candidates are visited in ascending order with a strict '<' per block, so no
// atomics are needed; the loop runs warp-uniform (shuffles need the whole
// warp), groups with fewer candidates mask theirs.
//
// Rounding: INT8 scales carry full fp32 mantissas, so quotients are IEEE
// divisions; the searches round them half to even with the 1.5 * 2^23 add /
// subtract on the FMA pipe.  NaN payloads follow the reference on x86: x / s
// returns x's NaN, else s's NaN, 0 / 0 the default NaN 0xffc00000; dequant
// returns the scale's NaN first.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "qz_common.cuh"
#include "qz_kernels.h"
#include "qz_ptx.cuh"

namespace qz {
namespace {

constexpr int kIWarps = 8;
constexpr int kIThreads = kIWarps * 32;
constexpr uint32_t kDefaultNaN = 0xffc00000u;

template <int FMT>
struct IntQ { static constexpr float v = FMT == kNVINT4 ? 7.0f : 127.0f; };

__shared__ float s_itab[128];  // candidate scales, ascending (126 used)
__shared__ float s_irc[128];   // RN(1 / candidate)

// torch row-sum order, the part local to one lane (elements g + 8j).
template <int BS>
__device__ __forceinline__ float lane_sum(const float (&v)[BS / 8]) {
  if constexpr (BS == 16) {
    return __fadd_rn(v[0], v[1]);
  } else {
    float A[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      A[t] = v[t];
#pragma unroll
      for (int jj = 1; jj < BS / 32; ++jj) A[t] = __fadd_rn(A[t], v[t + 4 * jj]);
    }
    return __fadd_rn(__fadd_rn(__fadd_rn(A[0], A[1]), A[2]), A[3]);
  }
}

// ((a0 + a1) + a2) + ... + a7 over the eight lanes of the group; every lane of
// the warp must call it (full-warp shuffles).
__device__ __forceinline__ float group_fold(float a8) {
  const int base = threadIdx.x & 24;
  float r = __shfl_sync(0xffffffffu, a8, base);
#pragma unroll
  for (int m = 1; m < 8; ++m) r = __fadd_rn(r, __shfl_sync(0xffffffffu, a8, base + m));
  return r;
}

template <int BS>
__device__ __forceinline__ float group_sum(const float (&v)[BS / 8]) {
  return group_fold(lane_sum<BS>(v));
}

// clamp(round(x / s), -Q, Q) with the reference's NaN payloads (exact RNE).
template <int FMT, int DT>
__device__ __forceinline__ float int_q_exact(float x, float s, float rc, bool fast) {
  constexpr float Q = IntQ<FMT>::v;
  const uint32_t xb = __float_as_uint(x), sb = __float_as_uint(s);
  if (is_nan_bits(xb & 0x7fffffffu)) return __uint_as_float(xb | 0x00400000u);
  if (is_nan_bits(sb & 0x7fffffffu)) return s;
  if (s == 0.0f && x == 0.0f) return __uint_as_float(kDefaultNaN);
  const float q = rintf(__fdiv_rn(x, s));
  return q < -Q ? -Q : (q > Q ? Q : q);
}

__device__ __forceinline__ float int_dq(float q, float s) {
  if (is_nan_bits(__float_as_uint(s) & 0x7fffffffu)) return s;
  if (is_nan_bits(__float_as_uint(q) & 0x7fffffffu)) return q;
  return __fmul_rn(q, s);
}

// Block SSE for a finite scale s >= 0 or NaN (compute_block_sse,
// nvint4/reference.py:50-56, int8/reference.py:68-83).
template <int BS, int FMT, int DT>
__device__ __forceinline__ float int_sse(const float (&x)[BS / 8], float s, float rc, bool fast) {
  float d2[BS / 8];
#pragma unroll
  for (int j = 0; j < BS / 8; ++j) {  // on |x| (the SSE is sign-symmetric); NaN propagates
    const float a = fabsf(x[j]);
    const float q = __fadd_rn(__fadd_rn(__fdiv_rn(a, s), 12582912.0f), -12582912.0f);
    const float qc = q > IntQ<FMT>::v ? IntQ<FMT>::v : q;
    const float d = __fsub_rn(a, __fmul_rn(qc, s));
    d2[j] = __fmul_rn(d, d);
  }
  return group_sum<BS>(d2);
}

// sum(clamp(|x| - Q s, 0)^2) (nvint4/reference.py:144, int8/reference.py:200).
template <int BS, int FMT>
__device__ __forceinline__ float int_clip(const float (&x)[BS / 8], float s) {
  const float t = __fmul_rn(IntQ<FMT>::v, s);
  float v[BS / 8];
#pragma unroll
  for (int j = 0; j < BS / 8; ++j) {
    float c = __fsub_rn(fabsf(x[j]), t);
    c = c < 0.0f ? 0.0f : c;
    v[j] = __fmul_rn(c, c);
  }
  return group_sum<BS>(v);
}

// r^T H_j r: rows of H r as FMA chains over b ascending, then the torch row
// sum of r_a * (H r)_a.  rbuf: the group's BS floats of shared memory.
template <int BS, int FMT, int DT>
__device__ __forceinline__ float int_hess(const float (&x)[BS / 8], float s, float rc, bool fast,
                                          const float* __restrict__ Hj, float* rbuf) {
  const int g = threadIdx.x & 7;
  float r[BS / 8];
#pragma unroll
  for (int j = 0; j < BS / 8; ++j) {
    const float q = int_q_exact<FMT, DT>(x[j], s, rc, fast);
    r[j] = __fsub_rn(x[j], int_dq(q, s));
    rbuf[g + 8 * j] = r[j];
  }
  __syncwarp();
  float p[BS / 8];
#pragma unroll
  for (int j = 0; j < BS / 8; ++j) {
    const float4* h4 = reinterpret_cast<const float4*>(Hj + (size_t)(g + 8 * j) * BS);
    float acc = 0.0f;
#pragma unroll 4
    for (int b4 = 0; b4 < BS / 4; ++b4) {
      const float4 h = __ldg(h4 + b4);
      const float4 rv = *reinterpret_cast<const float4*>(rbuf + 4 * b4);
      acc = __fmaf_rn(h.x, rv.x, acc);
      acc = __fmaf_rn(h.y, rv.y, acc);
      acc = __fmaf_rn(h.z, rv.z, acc);
      acc = __fmaf_rn(h.w, rv.w, acc);
    }
    p[j] = acc;
  }
#pragma unroll
  for (int j = 0; j < BS / 8; ++j) p[j] = __fmul_rn(r[j], p[j]);
  __syncwarp();  // rbuf is rewritten by the next evaluation
  return group_sum<BS>(p);
}

template <int DT>
__device__ __forceinline__ float raw_elem(const unsigned char* raw, int i) {
  if constexpr (DT == kDtF32) return reinterpret_cast<const float*>(raw)[i];
  const uint32_t h = reinterpret_cast<const uint16_t*>(raw)[i];
  return DT == kDtBF16 ? bf16_bits_to_float(h) : f16_bits_to_float(h);
}

// Per-warp shared memory: a ring of kStages bulk-copy stages of kTiles tiles
// (four blocks each, raw input), then two areas of one padded row per group
// (sort keys; |x| for the SSE search or the residual of the Hessian), then the
// stages' mbarriers.
template <int BS, int DT>
struct IGeom {
  static constexpr int kTile = 4 * BS * Elem<DT>::kSize;
  static constexpr int kTiles = kTile >= 2048 ? 1 : 2048 / kTile;
  static constexpr int kStage = kTiles * kTile;
  static constexpr int kStages = kStage < 2048 ? 4 : 2;  // two for 2 KB stages: two CTAs per SM at bs 256
  static constexpr int kRing = kStages * kStage;
  static constexpr int kRow = BS + 4;  // padded per-group row (floats): no bank conflicts across groups
  static constexpr int kArea = 4 * kRow * 4;
  static constexpr int kBytes = kRing + 2 * kArea + kStages * 8;
};

template <int BS, int FMT, int METHOD, int DT>
__global__ void __launch_bounds__(kIThreads) int_kernel(QuantArgs p) {
  using G = IGeom<BS, DT>;
  constexpr int NE = BS / 8;
  constexpr float Q = IntQ<FMT>::v;
  extern __shared__ __align__(16) unsigned char ismem[];
  for (int i = threadIdx.x; i < 128; i += blockDim.x) {
    float v = i < 126 ? e4m3_value(i + 1) : 3.0e38f;
    if (FMT == kInt8 && i < 126) v = __fdiv_rn(v, 127.0f);
    s_itab[i] = v;
    s_irc[i] = __frcp_rn(v);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, grp = lane >> 3, g = lane & 7;
  unsigned char* wbase = ismem + warp * G::kBytes;
  uint32_t* wsort = reinterpret_cast<uint32_t*>(wbase + G::kRing) + grp * G::kRow;
  float* wr = reinterpret_cast<float*>(wbase + G::kRing + G::kArea) + grp * G::kRow;
  uint64_t* bar = reinterpret_cast<uint64_t*>(wbase + G::kRing + 2 * G::kArea);

  const int64_t blocks_per_chunk = (int64_t)G::kTiles * 4;
  const int64_t n_chunks = (p.n_blocks + blocks_per_chunk - 1) / blocks_per_chunk;
  const int64_t gwarp = (int64_t)blockIdx.x * kIWarps + warp, nwarps = (int64_t)gridDim.x * kIWarps;
  const char* src = static_cast<const char*>(p.x);
  auto issue = [&](int64_t i) {  // lane 0: chunk i of this warp into stage i % kStages
    const int64_t ch = gwarp + i * nwarps;
    if (ch >= n_chunks) return;
    const int64_t nb = p.n_blocks - ch * blocks_per_chunk < blocks_per_chunk ? p.n_blocks - ch * blocks_per_chunk
                                                                          : blocks_per_chunk;
    const uint32_t bytes = (uint32_t)(nb * BS * Elem<DT>::kSize);
    uint64_t* bb = bar + (i % G::kStages);
    mbar_arrive_expect_tx(bb, bytes);
    bulk_load(wbase + (i % G::kStages) * G::kStage, src + ch * blocks_per_chunk * BS * Elem<DT>::kSize, bytes, bb);
  };
  if (lane == 0) {
    for (int k = 0; k < G::kStages; ++k) mbar_init(bar + k, 1);
    fence_barrier_init();
    for (int k = 0; k < G::kStages; ++k) issue(k);
  }
  __syncwarp();

  for (int64_t ci = 0;; ++ci) {
   const int64_t ch = gwarp + ci * nwarps;
   if (ch >= n_chunks) break;
   const bool landed = mbar_wait_bounded(bar + (ci % G::kStages), (uint32_t)((ci / G::kStages) & 1),
                                         kDevErrLoadTimeout);
   if (!__all_sync(0xffffffffu, landed)) {  // the whole warp leaves together
     // a copy never landed: drain what this warp still has in flight (bounded), then stop
     for (int64_t k = ci + 1; k < ci + G::kStages && gwarp + k * nwarps < n_chunks; ++k)
       mbar_wait_bounded(bar + (k % G::kStages), (uint32_t)((k / G::kStages) & 1), kDevErrLoadTimeout);
     return;
   }
   const unsigned char* stage = wbase + (ci % G::kStages) * G::kStage;
   for (int tt = 0; tt < G::kTiles; ++tt) {
    const int64_t b0 = (ch * G::kTiles + tt) * 4;
    if (b0 >= p.n_blocks) break;
    const int nb = (int)(p.n_blocks - b0 < 4 ? p.n_blocks - b0 : 4);
    const unsigned char* wraw = stage + tt * G::kTile;
    const bool valid = grp < nb;
    const int64_t b = b0 + grp;
    float x[NE];
#pragma unroll
    for (int j = 0; j < NE; ++j) x[j] = valid ? raw_elem<DT>(wraw + grp * BS * Elem<DT>::kSize, g + 8 * j) : 0.0f;

    // amax (NaN patterns order above inf: NaN propagates)
    uint32_t m = 0;
#pragma unroll
    for (int j = 0; j < NE; ++j) m = max(m, __float_as_uint(x[j]) & 0x7fffffffu);
    m = max(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = max(m, __shfl_xor_sync(0xffffffffu, m, 2));
    m = max(m, __shfl_xor_sync(0xffffffffu, m, 4));
    const float amax = __uint_as_float(m);

    // naive scale (nvint4/reference.py:76-78; int8/reference.py:112-114) and
    // the E4M3 code of the stored value (NVINT4: s; INT8: 127 s)
    float s;
    int code;
    if (is_nan_bits(m)) {
      s = __uint_as_float(kNvNanBits);
      code = 0x7f;
    } else {
      const float v = e4m3_snap_nonneg(amax < 1e-12f ? 1e-12f : amax);
      code = (int)e4m3_code(v);
      s = is_nan_bits(__float_as_uint(v)) ? v : __fdiv_rn(v, 127.0f);
    }
    const bool s_fin = __float_as_uint(s) > 0u && __float_as_uint(s) < 0x7f800000u;
    float rc = s_fin ? __frcp_rn(s) : 0.0f;

    if constexpr (METHOD != kNaive) {
      // bounds (nvint4/reference.py:111-133; int8/reference.py:160-186)
      const float E0 = int_sse<BS, FMT, DT>(x, s, rc, s_fin);
      float sq[NE];
#pragma unroll
      for (int j = 0; j < NE; ++j) sq[j] = __fmul_rn(x[j], x[j]);
      bool noise = group_sum<BS>(sq) <= E0;
      float s_min = __fdiv_rn(__fsub_rn(amax, __fsqrt_rn(E0)), Q);
      s_min = s_min < 0.0f ? 0.0f : s_min;
#pragma unroll
      for (int j = 0; j < NE; ++j) wsort[g + 8 * j] = __float_as_uint(x[j]) & 0x7fffffffu;
      __syncwarp();
      for (int k = 2; k <= BS; k <<= 1) {  // bitonic sort, ascending (NaN patterns last)
        for (int jj = k >> 1; jj > 0; jj >>= 1) {
          for (int i = g; i < BS; i += 8) {
            const int ix = i ^ jj;
            if (ix > i) {
              const uint32_t u = wsort[i], v = wsort[ix];
              if ((u > v) == ((i & k) == 0)) { wsort[i] = v; wsort[ix] = u; }
            }
          }
          __syncwarp();
        }
      }
      int k_star = 0;  // torch.cumsum: sequential fp64, each prefix rounded to fp32
      double acc = 0.0;
      for (int i = 0; i < BS; ++i) {
        const float v = __uint_as_float(wsort[i]);
        acc = __dadd_rn(acc, (double)__fmul_rn(v, v));
        if (__double2float_rn(acc) <= E0) ++k_star; else break;
      }
      if (k_star >= BS) noise = true;
      const float y = __uint_as_float(wsort[k_star < BS - 1 ? k_star : BS - 1]);
      __syncwarp();
      const float s_max = __fdiv_rn(y, 0.5f);
      int lo = 0, hi = -1;
      if (valid && !noise && s_min <= s_max) {
        int a = 0, c = 126;  // first index with scale >= s_min
        while (a < c) { const int mm = (a + c) >> 1; if (s_itab[mm] < s_min) a = mm + 1; else c = mm; }
        lo = a;
        a = 0; c = 126;      // first index with scale > s_max
        while (a < c) { const int mm = (a + c) >> 1; if (s_itab[mm] <= s_max) a = mm + 1; else c = mm; }
        hi = a - 1;
      }
      const int n = hi >= lo ? hi - lo + 1 : 0;
      const int n_max = __reduce_max_sync(0xffffffffu, (unsigned)n);
      const float* Hj = METHOD == kHessian ? p.h_blocks + (size_t)(valid ? b % p.n_col_blocks : 0) * BS * BS
                                           : nullptr;
      float best_E = METHOD == kSSE ? E0 : int_hess<BS, FMT, DT>(x, s, rc, s_fin, Hj, wr);
      int best_c = -1;
#pragma unroll 1
      for (int it = 0; it < n_max; ++it) {
        const bool act = it < n;
        const int ci = act ? lo + it : 0;
        const float sc = s_itab[ci], rcc = s_irc[ci];
        float E;
        if constexpr (METHOD == kSSE) {
          E = int_sse<BS, FMT, DT>(x, sc, rcc, true);
        } else {
          // fast-fail: 10x the running Hessian best (nvint4/reference.py:259, int8/reference.py:334)
          const float hc = int_clip<BS, FMT>(x, sc);  // every lane: the fold shuffles the whole warp
          const bool pass = act && hc < __fmul_rn(best_E, 10.0f);
          if (!__any_sync(0xffffffffu, pass)) continue;
          E = int_hess<BS, FMT, DT>(x, sc, rcc, true, Hj, wr);
          if (!pass) continue;
        }
        if (act && E < best_E) { best_E = E; best_c = ci; }
      }
      if (best_c >= 0) {
        s = s_itab[best_c];
        rc = s_irc[best_c];
        code = best_c + 1;
      }
    }

    // outputs
    const bool fast = __float_as_uint(s) > 0u && __float_as_uint(s) < 0x7f800000u;
    uint32_t nib[NE];
#pragma unroll
    for (int j = 0; j < NE; ++j) {
      const float q = int_q_exact<FMT, DT>(x[j], s, rc, fast);
      const float d = int_dq(q, s);
      const int64_t e = b * BS + g + 8 * j;
      const bool qn = is_nan_bits(__float_as_uint(q) & 0x7fffffffu);
      nib[j] = qn ? 0x80u : ((uint32_t)__float2int_rn(q) & 0xffu);
      if (valid) {
        if (p.quants) p.quants[e] = q;
        if (p.dq) p.dq[e] = d;
        if (p.dq_bf16) p.dq_bf16[e] = __bfloat16_as_ushort(__float2bfloat16_rn(d));
        if (p.packed) p.packed[e] = (uint8_t)nib[j];
      }
    }
    if (valid && g == 0) {
      if (p.scales) p.scales[b] = s;
      if (p.scale_codes) p.scale_codes[b] = (uint8_t)code;
    }
   }
   __syncwarp();  // the stage is refilled below
   if (lane == 0) {
     fence_proxy_async_smem();
     issue(ci + G::kStages);
   }
  }
}

template <int BS, int FMT, int METHOD, int DT>
cudaError_t launch_int_k(const QuantArgs& p, int num_sms, cudaStream_t st) {
  using G = IGeom<BS, DT>;
  const int smem = kIWarps * G::kBytes;
  static int s_per_sm[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  int per_sm = dev < 64 ? s_per_sm[dev] : 0;
  if (per_sm == 0) {
    e = cudaFuncSetAttribute(int_kernel<BS, FMT, METHOD, DT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, int_kernel<BS, FMT, METHOD, DT>, kIThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    if (dev < 64) s_per_sm[dev] = per_sm;
  }
  const int64_t n_chunks = (p.n_blocks + G::kTiles * 4 - 1) / (G::kTiles * 4);
  const int64_t want = (n_chunks + kIWarps - 1) / kIWarps;
  const int64_t cap = (int64_t)num_sms * per_sm;
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  int_kernel<BS, FMT, METHOD, DT><<<grid, kIThreads, smem, st>>>(p);
  return cudaGetLastError();
}

template <int BS, int FMT, int DT>
cudaError_t launch_int_m(const QuantArgs& p, int method, int num_sms, cudaStream_t st) {
  switch (method) {
    case kNaive: return launch_int_k<BS, FMT, kNaive, DT>(p, num_sms, st);
    case kSSE: return launch_int_k<BS, FMT, kSSE, DT>(p, num_sms, st);
    case kHessian: return launch_int_k<BS, FMT, kHessian, DT>(p, num_sms, st);
    default: return cudaErrorInvalidValue;
  }
}

template <int BS, int FMT>
cudaError_t launch_int_d(const QuantArgs& p, int dtype, int method, int num_sms, cudaStream_t st) {
  switch (dtype) {
    case kDtBF16: return launch_int_m<BS, FMT, kDtBF16>(p, method, num_sms, st);
    case kDtF16: return launch_int_m<BS, FMT, kDtF16>(p, method, num_sms, st);
    default: return launch_int_m<BS, FMT, kDtF32>(p, method, num_sms, st);
  }
}

}  // namespace

cudaError_t read_device_error_int(unsigned* out, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(out, qz_device_error, sizeof(unsigned));
  if (e != cudaSuccess || !clear) return e;
  unsigned zero = 0;
  return cudaMemcpyToSymbol(qz_device_error, &zero, sizeof(unsigned));
}

cudaError_t launch_quantize_int(const QuantArgs& p, int dtype, int bs, int fmt, int method, int num_sms,
                                cudaStream_t st) {
  if (fmt == kNVINT4) {
    return launch_quantize_nvint4(p, dtype, bs, method, num_sms, st);  // qz_quantize.cu
  }
  if (fmt == kInt8) {
    if (bs == 32) return launch_quantize_int8_bs32(p, dtype, method, num_sms, st);  // qz_quantize.cu
    switch (bs) {
      case 64: return launch_int_d<64, kInt8>(p, dtype, method, num_sms, st);
      case 128: return launch_int_d<128, kInt8>(p, dtype, method, num_sms, st);
      case 256: return launch_int_d<256, kInt8>(p, dtype, method, num_sms, st);
      default: return cudaErrorInvalidValue;
    }
  }
  return cudaErrorInvalidValue;
}

}  // namespace qz
