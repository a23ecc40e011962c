// qz_gemm.cu -- the two dense contractions of the path on the 5th-generation
// tensor cores (tcgen05 + TMEM + TMA), bf16 operands, fp32 accumulation:
//
//   Gram      H = X^T X for X (T, K) row-major (the Hessian build of
//             nvfp4/reference.py:304-317).  Both operands are column panels of
//             X read straight from its row-major layout as MN-major tiles (no
//             transpose pass).  Only tiles touching the upper triangle are
//             computed; the epilogue writes each (i, j >= i) and its mirror, so
//             H is exactly symmetric.  The block-diagonal mode runs only the
//             tiles on the diagonal and writes (K/bs, bs, bs).
//   Metrics   sum((X W_dq^T - X W^T)^2) and sum((X W^T)^2) (metrics.py:29-50):
//             one GEMM of X against [W_tile; W_dq_tile] (N = 128 + 128), the
//             squared-difference reduction done from TMEM in the epilogue, the
//             T x M products never written.
//
// Kernel structure (one persistent CTA per SM, 192 threads; full Gram and
// metrics 320):
//   warp 0   TMA producer: a ring of operand stages (4 x 48 KB; full Gram and
//            metrics 3 x 64 KB)
//   warp 1   TMEM allocator + MMA issuer (one thread issues tcgen05.mma,
//            tcgen05.commit frees a smem stage / publishes an accumulator)
//   warps 2-5 epilogue: tcgen05.ld of the 128 x N fp32 accumulator
//   Two accumulators (2 x 256 TMEM columns) let the epilogue of one tile overlap
//   the main loop of the next.  The 256-row tiles of the full Gram and the
//   metrics use both as one (rows 0-127 and 128-255) and drain them with 8
//   epilogue warps (2-9); their units are long (hundreds to thousands of
//   K-steps), so the unoverlapped epilogue costs 1-2%.  Every mbarrier wait is
//   bounded (2 s): on timeout the kernel records an error flag, all roles stop,
//   TMEM is freed, and the
//   host reports QZ_ERR_TIMEOUT.  No TMA multicast anywhere.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "../../include/qwantize_b200.h"
#include "qz_kernels.h"
#include "qz_ptx.cuh"

namespace qz {

int fail(int code, const char* fmt, ...);
int cuda_status(cudaError_t e, const char* what);
int current_sms(int* sms);

constexpr int kBM = 128, kBK = 64;  // tile rows, K-step (64 bf16 = one 128-byte swizzle row)

enum GemmMode { kGramFull = 0, kGramDiag = 1, kMetrics = 2, kGptq = 3, kTf3 = 4 };

// The fp32-accuracy modes: tf32 tensor-core products of high / low operand
// pairs (kGptq: GPTQ's error update; kTf3: C = beta C + alpha A B for the
// symmetric-positive-definite inverse).
__host__ __device__ constexpr bool tf_mode(int mode) { return mode == kGptq || mode == kTf3; }
// The modes whose 256-row output tile is two M = 128 MMAs sharing one B panel.
__host__ __device__ constexpr bool wide_mode(int mode) { return mode == kGramFull || mode == kMetrics; }

// Per-mode geometry.  Full Gram: 256 x 256 tiles, A 32 KB + B 32 KB per stage
// (a diagonal tile loads one panel for both), 3 stages; each stage feeds two
// M = 128 MMAs that share the B panel, so a stage is 1024 tensor cycles for 64
// KB of operands (two thirds of the L2 -> shared traffic per flop of a 128 x
// 256 tile).  Metrics: likewise 256 token rows x [128 rows of W; 128 of W_dq],
// A 32 KB + B 32 KB per stage, 3 stages.
// Block-diagonal Gram: 128 x 128 diagonal tiles whose A and B panels are the
// same columns of X, so one 16 KB panel per stage feeds both operands; 8 stages.
// GPTQ update: 128 x 128 tiles of fp32 operands as tf32 high / low pairs; a
// stage holds 32 columns of K (128 bytes per row) of A_hi, A_lo, B_hi, B_lo.
template <int MODE>
struct Geo {
  static constexpr int BM = wide_mode(MODE) ? 256 : kBM;  // output tile rows
  static constexpr int BN = (MODE == kGramDiag || tf_mode(MODE)) ? 128 : 256;
  static constexpr int kABytes = tf_mode(MODE) ? 2 * kBM * 128 : BM * kBK * 2;
  static constexpr int kBBytes = MODE == kGramDiag ? 0 : (tf_mode(MODE) ? 2 * BN * 128 : BN * kBK * 2);
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = MODE == kGramDiag ? 8 : ((tf_mode(MODE) || wide_mode(MODE)) ? 3 : 4);
  static constexpr int kTmemCols = 2 * BN;
  // Full Gram: one 256 x 256 tile is two M = 128 accumulators (all 512 TMEM
  // columns, no double buffer) drained by 8 epilogue warps; other modes keep
  // two accumulators, 4 epilogue warps
  static constexpr int kAccs = wide_mode(MODE) ? 1 : 2;
  static constexpr int kEpiThreads = wide_mode(MODE) ? 256 : 128;
  static constexpr int kThreads = 64 + kEpiThreads;
  static constexpr int kSmem = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
};

struct GemmParams {
  int64_t T, K, M;      // Gram: X is (T, K); Metrics: X (T, K), W (M, K)
  int bs;               // block size for kGramDiag
  int accumulate;       // add into H instead of storing
  int64_t tiles_m, tiles_n, n_tiles;
  int64_t splits, split_rows;  // kGramDiag: T is cut into `splits` ranges of split_rows
  int64_t seg_rows, band;      // kGramFull: token rows per segment, tile rows per band
  int* seq;                    // kGramFull: per-tile count of segments already added
  int64_t tiles_per_seg;       // kGramFull: tiles in one segment (units = tiles x segments)
  // kGramFull, last wave: units from tail_start on are the last tail_tiles
  // tiles of the last segment (first tile tail_tile0, rows from tail_r0), each
  // cut into pieces of tail_piece_rows token rows that count as further
  // segments (last_seg, last_seg + 1, ...) of their tile
  int64_t tail_start, tail_tiles, tail_tile0, tail_r0, tail_piece_rows, last_seg;
  float* H;
  float* packed;        // kGramFull: when set, the upper 256 x 256 tiles instead of H (column-major tiles)
  float* partials;      // kGramDiag: splits-1 partial (K/bs, bs, bs) buffers
  double* sums;
  uint32_t lbo, sbo;    // MN-major descriptor offsets (bytes)
  // kGptq: W -= E @ Hi[group rows, columns c1..K) written into the
  // column-block-major working weight Wb (nblk, M, bs)
  float* Wb;
  int64_t g0c, c1, gk;  // group's first column, first column after the group, group width
  // tf32 modes: the operand tiles of output tile (mi, nj) at K step ks come
  // from map_a at (a_x0 + 32 ks, a_y0 + 128 mi) (high parts) and (+ a_lo_dx,
  // + a_lo_dy) (low parts), and likewise from map_b with 128 nj
  int a_x0, a_y0, a_lo_dx, a_lo_dy, b_x0, b_y0, b_lo_dx, b_lo_dy;
  // kTf3 output: rows m < p.M, columns n < p.N of C (value, leading dimension
  // ldc) = alpha acc (+ C if beta); with Cs, its tf32 high part at Cs[i] and
  // low part at Cs[i + cs_lo]
  int64_t N, ldc, cs_lo;
  float* C;
  float* Cs;
  float alpha;
  int beta;
  // kTf3 extra copies of the result: D1 = d1_sign * C at the same position,
  // D2 = d2_sign * C^T (value and split each, same leading dimension)
  float *D1, *D1s, *D2, *D2s;
  float d1_sign, d2_sign;
};

// ---------------------------------------------------------------------------
// PTX wrappers specific to the tensor-core pipeline
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 inputs, fp32 accumulate).
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::tf32 (fp32 containers, tf32
// products, fp32 accumulate).
__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every tcgen05.mma issued so far by this thread is done.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 bits, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor (tcgen05), 128-byte swizzle.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3fffu);
  d |= (uint64_t)((lbo >> 4) & 0x3fffu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3fffu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::f16: bf16 x bf16 -> fp32, M x N.
__host__ __device__ constexpr uint32_t instr_desc(int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4)                       // D format: f32
         | (1u << 7)                     // A format: bf16
         | (1u << 10)                    // B format: bf16
         | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Instruction descriptor for kind::tf32: tf32 x tf32 -> fp32, both K-major.
__host__ __device__ constexpr uint32_t instr_desc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---------------------------------------------------------------------------
// tile enumeration
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tile_coords(const GemmParams& p, int mode, int64_t t, int64_t& mi, int64_t& nj) {
  if (mode == kGramDiag) {  // unit t = (split, tile): tile = t % tiles_m
    mi = t % p.tiles_m;
    nj = t / p.tiles_m;     // the split index
    return;
  }
  if (mode == kMetrics || tf_mode(mode)) {
    mi = t / p.tiles_n;
    nj = t % p.tiles_n;
    return;
  }
  // kGramFull: 256 x 256 tiles (mi, nj) with nj >= mi, enumerated in bands of
  // p.band tile rows, column by column inside a band, so the ~148 tiles in
  // flight share few column panels of X (L2 reuse).
  int64_t r = t;
  for (int64_t b0 = 0; b0 < p.tiles_m; b0 += p.band) {
    const int64_t rows_end = b0 + p.band < p.tiles_m ? b0 + p.band : p.tiles_m;
    for (int64_t n = b0; n < p.tiles_n; ++n) {
      const int64_t hi = rows_end < n + 1 ? rows_end : n + 1;  // rows with mi <= n
      const int64_t cnt = hi - b0;
      if (r < cnt) { mi = b0 + r; nj = n; return; }
      r -= cnt;
    }
  }
  mi = nj = 0;
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
// A work unit: output tile (mi, nj), the rows [r0, r0 + 64*steps) of X it
// reduces over (Gram) or its K-steps (metrics), and for the full Gram the tile
// id and segment (units run segment-major: every segment's tiles, in order).
struct Unit {
  int64_t mi, nj, r0, steps, tile, seg;
};

template <int MODE>
__device__ __forceinline__ Unit unit_of(const GemmParams& p, int64_t t) {
  Unit u{};
  if (MODE == kMetrics) {
    tile_coords(p, MODE, t, u.mi, u.nj);
    u.steps = (p.K + kBK - 1) / kBK;
    return u;
  }
  if (tf_mode(MODE)) {
    tile_coords(p, MODE, t, u.mi, u.nj);
    u.steps = p.gk / 32;  // 32 fp32 columns (128 bytes) per stage
    return u;
  }
  if (MODE == kGramDiag) {
    tile_coords(p, MODE, t, u.mi, u.nj);  // nj = split index
    u.r0 = u.nj * p.split_rows;
  } else if (t < p.tail_start) {
    u.seg = t / p.tiles_per_seg;
    u.tile = t % p.tiles_per_seg;
    tile_coords(p, MODE, u.tile, u.mi, u.nj);
    u.r0 = u.seg * p.seg_rows;
  } else {
    const int64_t q = t - p.tail_start, piece = q / p.tail_tiles;
    u.tile = p.tail_tile0 + q % p.tail_tiles;
    u.seg = p.last_seg + piece;
    tile_coords(p, MODE, u.tile, u.mi, u.nj);
    u.r0 = p.tail_r0 + piece * p.tail_piece_rows;
    const int64_t r1 = u.r0 + p.tail_piece_rows < p.T ? u.r0 + p.tail_piece_rows : p.T;
    u.steps = (r1 - u.r0 + kBK - 1) / kBK;
    return u;
  }
  const int64_t rows = MODE == kGramDiag ? p.split_rows : p.seg_rows;
  const int64_t r1 = u.r0 + rows < p.T ? u.r0 + rows : p.T;
  u.steps = (r1 - u.r0 + kBK - 1) / kBK;
  return u;
}

template <int MODE>
__global__ void __launch_bounds__(Geo<MODE>::kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                const __grid_constant__ CUtensorMap map_c, GemmParams p) {
  using G = Geo<MODE>;
  constexpr int BN = G::BN;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + G::kStages * G::kStageBytes);
  uint64_t* empty = full + G::kStages;
  uint64_t* tfull = empty + G::kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;  // the MMA issuer's final commit (all its MMAs retired)
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_s = reinterpret_cast<volatile int*>(tmem_base_s + 1);
  volatile int* go_s = abort_s + 1;  // full Gram: the segment-order verdict of this tile

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < G::kStages; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 1); }
    for (int a = 0; a < 2; ++a) { mbar_init(tfull + a, 1); mbar_init(tempty + a, G::kEpiThreads); }
    mbar_init(mma_done, 1);
    *abort_s = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_base_s, G::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_s;

  auto wait = [&](uint64_t* bar, uint32_t parity, unsigned err) -> bool {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity)) {
      if (*abort_s) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        atomicOr(&qz_device_error, err);
        *abort_s = 1;
        return false;
      }
    }
    return true;
  };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t it = 0;
      for (int64_t t = blockIdx.x; t < p.n_tiles; t += gridDim.x) {
        const Unit u = unit_of<MODE>(p, t);
        const int64_t mi = u.mi, nj = u.nj, r0 = u.r0, k_steps = u.steps;
        for (int64_t ks = 0; ks < k_steps; ++ks, ++it) {
          const int s = it % G::kStages;
          if (!wait(empty + s, ((it / G::kStages) & 1) ^ 1, kDevErrLoadTimeout)) goto producer_done;
          unsigned char* sa = smem + s * G::kStageBytes;
          unsigned char* sb = sa + G::kABytes;
          // a diagonal full-Gram tile reads one panel for both operands
          const bool one_panel = MODE == kGramFull && mi == nj;
          mbar_arrive_expect_tx(full + s, one_panel ? G::kABytes : G::kStageBytes);
          if (tf_mode(MODE)) {
            // high and low parts of a 128 x 32 tile of A and of B^T (K-major)
            const int kx = (int)(ks * 32), ay = p.a_y0 + (int)(mi * kBM), by = p.b_y0 + (int)(nj * 128);
            tma_load_2d(sa, &map_a, p.a_x0 + kx, ay, full + s);
            tma_load_2d(sa + 16384, &map_a, p.a_x0 + p.a_lo_dx + kx, ay + p.a_lo_dy, full + s);
            tma_load_2d(sb, &map_b, p.b_x0 + kx, by, full + s);
            tma_load_2d(sb + 16384, &map_b, p.b_x0 + p.b_lo_dx + kx, by + p.b_lo_dy, full + s);
          } else if (MODE == kMetrics) {
            const int kx = (int)(ks * kBK);
            tma_load_2d(sa, &map_a, kx, (int)(mi * G::BM), full + s);               // X rows (t)
            tma_load_2d(sb, &map_b, kx, (int)(nj * 128), full + s);                 // W rows
            tma_load_2d(sb + 128 * kBK * 2, &map_c, kx, (int)(nj * 128), full + s);  // W_dq rows
          } else {
            const int ty = (int)(r0 + ks * kBK);
            const int i0 = (int)(mi * G::BM);
#pragma unroll
            for (int q = 0; q < G::BM / 64; ++q) tma_load_2d(sa + 8192 * q, &map_a, i0 + 64 * q, ty, full + s);
            if (MODE == kGramFull && !one_panel) {
              const int j0 = (int)(nj * BN);
#pragma unroll
              for (int q = 0; q < 4; ++q) tma_load_2d(sb + 8192 * q, &map_a, j0 + 64 * q, ty, full + s);
            }
          }
        }
      }
    producer_done:
      // Before the CTA can exit, every load issued must have landed (after an
      // abort the MMA issuer stops consuming): wait, bounded, on the phase of
      // the last load issued into each stage.  In a normal run these phases
      // have long completed and each wait returns at once.
      for (uint32_t k = it > (uint32_t)G::kStages ? it - G::kStages : 0u; k < it; ++k)
        mbar_wait_bounded(full + (k % G::kStages), (k / G::kStages) & 1, kDevErrLoadTimeout);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr bool mn = MODE != kMetrics && !tf_mode(MODE);
      constexpr uint32_t idesc = tf_mode(MODE) ? instr_desc_tf32(kBM, BN) : instr_desc(kBM, BN, mn, mn);
      uint32_t it = 0, lt = 0;
      for (int64_t t = blockIdx.x; t < p.n_tiles; t += gridDim.x, ++lt) {
        const Unit u = unit_of<MODE>(p, t);
        const int64_t k_steps = u.steps;
        const uint32_t acc = G::kAccs == 2 ? (lt & 1) : 0u;
        const uint32_t phase = G::kAccs == 2 ? ((lt >> 1) & 1) : (lt & 1);
        if (!wait(tempty + acc, phase ^ 1, kDevErrMmaTimeout)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int64_t ks = 0; ks < k_steps; ++ks, ++it) {
          const int s = it % G::kStages;
          if (!wait(full + s, (it / G::kStages) & 1, kDevErrMmaTimeout)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * G::kStageBytes);
          const uint32_t sb = (MODE == kGramDiag || (MODE == kGramFull && u.mi == u.nj)) ? sa : sa + G::kABytes;
          if constexpr (tf_mode(MODE)) {
            // D += A_hi B_hi + A_hi B_lo + A_lo B_hi, 8 tf32 (32 bytes) of K per MMA
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ah = smem_desc(sa + kk * 32, 16, 1024), al = smem_desc(sa + 16384 + kk * 32, 16, 1024);
              const uint64_t bh = smem_desc(sb + kk * 32, 16, 1024), bl = smem_desc(sb + 16384 + kk * 32, 16, 1024);
              umma_tf32(d_tmem, al, bh, idesc, (ks > 0 || kk > 0) ? 1u : 0u);
              umma_tf32(d_tmem, ah, bl, idesc, 1u);
              umma_tf32(d_tmem, ah, bh, idesc, 1u);
            }
          } else if constexpr (MODE == kMetrics) {
            // X rows 0-127 and 128-255 of the tile against the same [W; W_dq]
            // panel (K-major: row 128 starts 16 KB into the A panel)
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) {
              const uint64_t bd = smem_desc(sb + kk * 32, 16, 1024);
              const uint32_t accum = (ks > 0 || kk > 0) ? 1u : 0u;
              umma_bf16(d_tmem, smem_desc(sa + kk * 32, 16, 1024), bd, idesc, accum);
              umma_bf16(d_tmem + BN, smem_desc(sa + 16384 + kk * 32, 16, 1024), bd, idesc, accum);
            }
          } else if constexpr (MODE == kGramFull) {
            // rows 0-127 and 128-255 of the tile against the same 256 columns
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) {
              const uint64_t bd = smem_desc(sb + kk * 2048, p.lbo, p.sbo);
              const uint32_t accum = (ks > 0 || kk > 0) ? 1u : 0u;
              umma_bf16(d_tmem, smem_desc(sa + kk * 2048, p.lbo, p.sbo), bd, idesc, accum);
              umma_bf16(d_tmem + BN, smem_desc(sa + 16384 + kk * 2048, p.lbo, p.sbo), bd, idesc, accum);
            }
          } else {
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) {
              uint64_t ad, bd;
              if (mn) {  // MN-major: a 16-row K step is two 8-row swizzle atoms (2 KB)
                ad = smem_desc(sa + kk * 2048, p.lbo, p.sbo);
                bd = smem_desc(sb + kk * 2048, p.lbo, p.sbo);
              } else {   // K-major: 16 elements = 32 bytes inside the 128-byte swizzle row
                ad = smem_desc(sa + kk * 32, 16, 1024);
                bd = smem_desc(sb + kk * 32, 16, 1024);
              }
              umma_bf16(d_tmem, ad, bd, idesc, (ks > 0 || kk > 0) ? 1u : 0u);
            }
          }
          umma_commit(empty + s);
        }
        if (!ok) break;
        umma_commit(tfull + acc);
      }
      // the MMAs issued must retire before TMEM is freed (also after an abort)
      umma_commit(mma_done);
      mbar_wait_bounded(mma_done, 0u, kDevErrMmaTimeout);
    }
  } else {
    // ---------------- epilogue (warps 2..5, full Gram 2..9) ----------------
    const int quarter = warp & 3;            // TMEM lanes 32*quarter .. +31
    const int row = quarter * 32 + lane;     // accumulator row of this thread
    const int half = (warp - 2) >> 2;        // full Gram: which M = 128 accumulator
    uint32_t lt = 0;
    double part0 = 0.0, part1 = 0.0;
    for (int64_t t = blockIdx.x; t < p.n_tiles; t += gridDim.x, ++lt) {
      const Unit u = unit_of<MODE>(p, t);
      const int64_t mi = u.mi, nj = u.nj;
      const uint32_t acc = G::kAccs == 2 ? (lt & 1) : 0u;
      const uint32_t phase = G::kAccs == 2 ? ((lt >> 1) & 1) : (lt & 1);
      if (!wait(tfull + acc, phase, kDevErrEpilogueTimeout)) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + ((uint32_t)(quarter * 32) << 16) + (wide_mode(MODE) ? half : acc) * BN;
      if (MODE == kMetrics) {
        const int64_t trow = mi * G::BM + half * 128 + row;
        float e = 0.0f, r2 = 0.0f;
#pragma unroll 1
        for (int c = 0; c < 128; c += 16) {
          float ref[16], dq[16];
          tmem_ld16(taddr + c, ref);
          tmem_ld16(taddr + 128 + c, dq);
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const float d = dq[q] - ref[q];
            e = fmaf(d, d, e);
            r2 = fmaf(ref[q], ref[q], r2);
          }
        }
        if (trow < p.T) { part0 += (double)e; part1 += (double)r2; }
      } else if (MODE == kGptq) {
        // W[m, c] -= D for the tile's columns c = c1 + 128 nj + ..., written
        // into the column-block-major working weight (16 consecutive columns
        // of one row are 64 contiguous bytes of one block row)
        const int64_t m = mi * kBM + row;
        const int bs = p.bs;
#pragma unroll 1
        for (int c = 0; c < BN; c += 16) {
          float v[16];
          tmem_ld16(taddr + c, v);
          const int64_t col = p.c1 + nj * BN + c;
          if (m >= p.M || col >= p.K) continue;
          float4* d4 = reinterpret_cast<float4*>(p.Wb + ((col / bs) * p.M + m) * bs + col % bs);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float4 w = d4[q];
            w.x -= v[4 * q]; w.y -= v[4 * q + 1]; w.z -= v[4 * q + 2]; w.w -= v[4 * q + 3];
            d4[q] = w;
          }
        }
      } else if (MODE == kTf3) {
        // C = alpha acc (+ C), and its tf32 high / low split when requested;
        // 16 consecutive columns per chunk (M, N, ldc and the block offsets
        // are multiples of 32, so chunks are whole and 16-byte aligned)
        const int64_t r = mi * kBM + row;
#pragma unroll 1
        for (int c = 0; c < BN; c += 16) {
          float v[16];
          tmem_ld16(taddr + c, v);
          const int64_t c0 = nj * BN + c;
          if (r >= p.M || c0 >= p.N) continue;
          float4* cp = reinterpret_cast<float4*>(p.C + r * p.ldc + c0);
          float o[16];
          if (p.beta) {
            float4 t[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) t[q] = cp[q];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              o[4 * q] = fmaf(p.alpha, v[4 * q], t[q].x);
              o[4 * q + 1] = fmaf(p.alpha, v[4 * q + 1], t[q].y);
              o[4 * q + 2] = fmaf(p.alpha, v[4 * q + 2], t[q].z);
              o[4 * q + 3] = fmaf(p.alpha, v[4 * q + 3], t[q].w);
            }
          } else {
#pragma unroll
            for (int q = 0; q < 16; ++q) o[q] = p.alpha * v[q];
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) cp[q] = make_float4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
          float hi[16], lo[16];
#pragma unroll
          for (int q = 0; q < 16; ++q) {  // tf32 split (round to nearest; odd: split(-v) = -split(v))
            uint32_t h, l;
            asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(o[q]));
            hi[q] = __uint_as_float(h);
            asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(l) : "f"(o[q] - hi[q]));
            lo[q] = __uint_as_float(l);
          }
          if (p.Cs) {
            float4* hp = reinterpret_cast<float4*>(p.Cs + r * p.ldc + c0);
            float4* lp = reinterpret_cast<float4*>(p.Cs + p.cs_lo + r * p.ldc + c0);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              hp[q] = make_float4(hi[4 * q], hi[4 * q + 1], hi[4 * q + 2], hi[4 * q + 3]);
              lp[q] = make_float4(lo[4 * q], lo[4 * q + 1], lo[4 * q + 2], lo[4 * q + 3]);
            }
          }
          if (p.D1) {
            const float g = p.d1_sign;
            float4* vp = reinterpret_cast<float4*>(p.D1 + r * p.ldc + c0);
            float4* hp = reinterpret_cast<float4*>(p.D1s + r * p.ldc + c0);
            float4* lp = reinterpret_cast<float4*>(p.D1s + p.cs_lo + r * p.ldc + c0);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              vp[q] = make_float4(g * o[4 * q], g * o[4 * q + 1], g * o[4 * q + 2], g * o[4 * q + 3]);
              hp[q] = make_float4(g * hi[4 * q], g * hi[4 * q + 1], g * hi[4 * q + 2], g * hi[4 * q + 3]);
              lp[q] = make_float4(g * lo[4 * q], g * lo[4 * q + 1], g * lo[4 * q + 2], g * lo[4 * q + 3]);
            }
          }
          if (p.D2) {  // transposed: lanes (consecutive rows r) write consecutive addresses
            const float g = p.d2_sign;
#pragma unroll
            for (int q = 0; q < 16; ++q) {
              const int64_t ti = (c0 + q) * p.ldc + r;
              p.D2[ti] = g * o[q];
              p.D2s[ti] = g * hi[q];
              p.D2s[ti + p.cs_lo] = g * lo[q];
            }
          }
        }
      } else if (MODE == kGramDiag && p.bs > 32) {
        // bs 64 / 128: the rows of this warp belong to one block, whose bs
        // columns start at cb inside the 128-wide tile (loads are warp-wide)
        const int bs = p.bs;
        const int cb = (quarter * 32 / bs) * bs;
        const int64_t i = mi * kBM + row;
        float* dst = (nj == 0 ? p.H : p.partials + (nj - 1) * p.K * bs) + (i / bs) * bs * bs + (i % bs) * bs;
        const bool add = nj == 0 && p.accumulate;
#pragma unroll 1
        for (int c = 0; c < bs; c += 16) {
          float v[16];
          tmem_ld16(taddr + cb + c, v);
          if (i < p.K) {
#pragma unroll
            for (int q = 0; q < 16; q += 4) {
              float4 w = make_float4(v[q], v[q + 1], v[q + 2], v[q + 3]);
              float4* d4 = reinterpret_cast<float4*>(dst + c + q);
              if (add) {
                const float4 o = *d4;
                w.x += o.x; w.y += o.y; w.z += o.z; w.w += o.w;
              }
              *d4 = w;
            }
          }
        }
      } else if (MODE == kGramDiag) {
        // this warp's rows 32q..32q+31 meet the diagonal in columns 32q..32q+31
        float v[32];
        float* v0 = v;
        tmem_ld16(taddr + quarter * 32, *reinterpret_cast<float(*)[16]>(v0));
        tmem_ld16(taddr + quarter * 32 + 16, *reinterpret_cast<float(*)[16]>(v0 + 16));
        const int64_t i = mi * kBM + row;
        if (i < p.K) {
          const int bs = p.bs;
          const bool hi = bs == 16 && lane >= 16;  // bs 16: the second 16-column block
          float* dst = (nj == 0 ? p.H : p.partials + (nj - 1) * p.K * bs) + (i / bs) * bs * bs + (i % bs) * bs;
          const bool add = nj == 0 && p.accumulate;
#pragma unroll
          for (int q = 0; q < 32; q += 4) {
            if (q >= bs) break;
            float4 w = hi ? make_float4(v[16 + (q & 15)], v[17 + (q & 15)], v[18 + (q & 15)], v[19 + (q & 15)])
                          : make_float4(v[q], v[q + 1], v[q + 2], v[q + 3]);
            float4* d4 = reinterpret_cast<float4*>(dst + q);
            if (add) {
              float4 o = *d4;
              w.x += o.x; w.y += o.y; w.z += o.z; w.w += o.w;
            }
            *d4 = w;
          }
        }
      } else {
        // segments of one tile are added in order: one thread waits until the
        // previous segment of this tile has been written (bounded) and hands
        // its verdict to all epilogue warps through shared memory, so they
        // all continue or all stop; add, then publish
        bool go = true;
        if (warp == 2 && lane == 0) {
          const volatile int* sq = p.seq + u.tile;
          if (*sq < u.seg) {
            const uint64_t t0 = globaltimer_ns();
            while (*sq < u.seg) {
              if (*abort_s) { go = false; break; }
              if (globaltimer_ns() - t0 > kWaitLimitNs) {
                atomicOr(&qz_device_error, kDevErrEpilogueTimeout);
                *abort_s = 1;
                go = false;
                break;
              }
              __nanosleep(256);
            }
          }
          *go_s = go ? 1 : 0;
        }
        asm volatile("bar.sync 1, %0;" ::"n"(G::kEpiThreads) : "memory");
        go = *go_s != 0;
        if (!go) break;
        __threadfence();
        const bool add = u.seg > 0 || p.accumulate;
        const int64_t i = mi * G::BM + half * 128 + row;
        const int64_t j0 = nj * BN;
        // packed upper tiles: tile (mi, nj) at its upper-triangle index, element
        // (r, c) at c * 256 + r, so the lanes (consecutive rows) store together
        float* tile = p.packed ? p.packed + (mi * p.tiles_n - mi * (mi - 1) / 2 + (nj - mi)) * 65536 +
                                     half * 128 + row
                               : nullptr;
#pragma unroll 1
        for (int c = 0; tile && c < BN; c += 16) {
          float v[16];
          tmem_ld16(taddr + c, v);
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            float* d = tile + (int64_t)(c + q) * 256;
            *d = add ? v[q] + *d : v[q];
          }
        }
#pragma unroll 1
        for (int c = 0; !tile && c < BN; c += 16) {
          float v[16];
          tmem_ld16(taddr + c, v);
          if (i >= p.K) continue;
          const int64_t jc = j0 + c;
          if (jc >= i + 1 && jc + 16 <= p.K) {
            // whole chunk strictly right of the diagonal: vector row stores
            float4* up = reinterpret_cast<float4*>(p.H + i * p.K + jc);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              float4 w = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
              if (add) {
                float4 o = up[q];
                w.x += o.x; w.y += o.y; w.z += o.z; w.w += o.w;
              }
              up[q] = w;
              v[4 * q] = w.x; v[4 * q + 1] = w.y; v[4 * q + 2] = w.z; v[4 * q + 3] = w.w;
            }
#pragma unroll
            for (int q = 0; q < 16; ++q) p.H[(jc + q) * p.K + i] = v[q];  // mirror: coalesced over lanes
          } else {
#pragma unroll
            for (int q = 0; q < 16; ++q) {
              const int64_t j = jc + q;
              if (j >= p.K || j < i) continue;
              float* up = p.H + i * p.K + j;
              const float val = add ? v[q] + *up : v[q];
              *up = val;
              if (j > i) p.H[j * p.K + i] = val;
            }
          }
        }
      }
      if (MODE == kGramFull) {
        __threadfence();
        asm volatile("bar.sync 1, %0;" ::"n"(G::kEpiThreads) : "memory");  // the epilogue warps
        if (warp == 2 && lane == 0) atomicExch(p.seq + u.tile, (int)(u.seg + 1));
      }
      tc_fence_before();
      mbar_arrive(tempty + acc);
    }
    if (MODE == kMetrics) {
      // warp reduce, one atomic pair per warp
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        part0 += __shfl_xor_sync(0xffffffffu, part0, o);
        part1 += __shfl_xor_sync(0xffffffffu, part1, o);
      }
      if (lane == 0) {
        atomicAdd(p.sums, part0);
        atomicAdd(p.sums + 1, part1);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, G::kTmemCols);
  }
}

// H += partials[0] + partials[1] + ... in a fixed order (deterministic).
__global__ void add_partials_kernel(float4* __restrict__ H, const float4* __restrict__ parts, int64_t n4,
                                    int64_t n_parts) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 h = H[i];
    for (int64_t k = 0; k < n_parts; ++k) {
      float4 q = parts[k * n4 + i];
      h.x += q.x; h.y += q.y; h.z += q.z; h.w += q.w;
    }
    H[i] = h;
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D bf16 tensor map: rows of `inner` elements, `outer` rows, box inner x outer.
static int make_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint32_t box_inner,
                    uint32_t box_outer, bool f32 = false) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(QZ_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * (f32 ? 4 : 2)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(QZ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return QZ_OK;
}

template <int MODE>
static int launch_gemm(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& c, GemmParams p,
                       cudaStream_t st) {
  int sms = 0;
  int s = current_sms(&sms);
  if (s != QZ_OK) return s;
  static bool attr_set[64] = {false};  // per device (a benign race: every thread sets the same value)
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    e = cudaFuncSetAttribute(gemm_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, Geo<MODE>::kSmem);
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute");
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const int64_t grid = p.n_tiles < sms ? p.n_tiles : sms;
  if (grid <= 0) return QZ_OK;
  gemm_kernel<MODE><<<(unsigned)grid, Geo<MODE>::kThreads, Geo<MODE>::kSmem, st>>>(a, b, c, p);
  return cuda_status(cudaGetLastError(), "gemm launch");
}


// Full Gram: token rows per segment (a multiple of 64), the cost of one unit's
// epilogue in rows of its main loop, and tile rows per band.
constexpr int64_t kGramSegmentRows = 262144, kGramEpilogueRows = 1024;
// Block-diagonal Gram: a unit's fixed cost (pipeline fill, epilogue) in rows.
constexpr int64_t kDiagUnitRows = 256;
constexpr int64_t kGramBand = 4;
// MN-major descriptor offsets: 8 KB between 64-element swizzle atoms along M / N,
// 1 KB between 8-row groups along K.
constexpr uint32_t kMnLbo = 8192, kMnSbo = 1024;

// ---------------------------------------------------------------------------
// Fixed scratch for qz_gram_full_noalloc: the full Gram's per-tile segment
// counters live in this file-scope device array instead of memory the call
// allocates.  Every device that loads the library holds it (256 KB) until exit.
// ---------------------------------------------------------------------------
constexpr int64_t kNoAllocMaxTiles = 65536;
static __device__ __align__(256) int g_noalloc_tile_counters[kNoAllocMaxTiles];

// Device address of the array for the current device.  In host code the
// array's name is only a stand-in, so the address is looked up (with that
// device current) and cached.  The cache is keyed on the current CUDA context
// as well: after cudaDeviceReset the module is loaded again, possibly at
// another address, and the next call looks the address up afresh.
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

static int noalloc_counters(int** out) {
  static std::mutex mu;
  static int* addr[64] = {nullptr};
  static CUcontext ctx_of[64] = {nullptr};
  static CtxGetCurrentFn get_ctx = nullptr;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(QZ_ERR_INVALID, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!get_ctx) {
    void* fp = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fp, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return fail(QZ_ERR_CUDA, "cuCtxGetCurrent unavailable");
    get_ctx = reinterpret_cast<CtxGetCurrentFn>(fp);
  }
  CUcontext ctx = nullptr;  // NULL until the runtime has made a context current
  if (get_ctx(&ctx) != CUDA_SUCCESS) return fail(QZ_ERR_CUDA, "cuCtxGetCurrent failed");
  if (!addr[dev] || !ctx || ctx_of[dev] != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_tile_counters);  // also makes the primary context current
    if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress (no-alloc scratch)");
    if (get_ctx(&ctx) != CUDA_SUCCESS) return fail(QZ_ERR_CUDA, "cuCtxGetCurrent failed");
    addr[dev] = static_cast<int*>(p);
    ctx_of[dev] = ctx;
  }
  *out = addr[dev];
  return QZ_OK;
}

cudaError_t read_device_error_gemm(unsigned* out, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(out, qz_device_error, sizeof(unsigned));
  if (e != cudaSuccess || !clear) return e;
  unsigned zero = 0;
  return cudaMemcpyToSymbol(qz_device_error, &zero, sizeof(unsigned));
}

// Full Gram geometry: 256 x 256 tiles on and above the diagonal, per segment.
static int64_t full_gram_tiles(int64_t K) {
  const int64_t t = (K + 255) / 256;
  return t * (t + 1) / 2;
}

// Units run segment-major, one (tile, segment) unit per CTA at a time, so when
// the unit count leaves a partial last wave of r units (r <= tiles), those
// units -- the last r tiles of the last segment -- are cut into m row pieces
// each and the r*m pieces share the wave's idle SMs.  The pieces of a tile add
// into H in order (further segments of that tile), so the result stays
// deterministic; the order costs m epilogues in a row, so m balances the
// piece length against m epilogues (about kGramEpilogueRows rows each).
// H (K x K) from the packed upper tiles: one 64 x 64 block of H per CTA, read
// as the block U(min, max) of the upper triangle, which lies in one packed
// tile (coalesced along the tile's columns), and written row-major,
// transposed below the diagonal through shared memory.
__global__ void __launch_bounds__(256) gram_unpack_kernel(const float* __restrict__ P, int64_t K, int64_t t,
                                                          float* __restrict__ H) {
  __shared__ float sb[64][65];
  const int64_t bi = blockIdx.y, bj = blockIdx.x;
  const int64_t ur = bi < bj ? bi : bj, uc = bi < bj ? bj : bi;
  const int tx = threadIdx.x & 63, ty = threadIdx.x >> 6;
  const int64_t mi = ur >> 2, nj = uc >> 2;  // four 64-blocks per 256-tile
  const float* tile = P + (mi * t - mi * (mi - 1) / 2 + (nj - mi)) * 65536 + (ur & 3) * 64 + tx;
  const int64_t a = ur * 64 + tx;
#pragma unroll 4
  for (int cc = ty; cc < 64; cc += 4) {
    const int64_t b = uc * 64 + cc;
    sb[tx][cc] = (a < K && b < K) ? tile[((uc & 3) * 64 + cc) * 256] : 0.0f;
  }
  __syncthreads();
  const int64_t j = bj * 64 + tx;
#pragma unroll 4
  for (int r = ty; r < 64; r += 4) {
    const int64_t i = bi * 64 + r;
    if (i < K && j < K) H[i * K + j] = i <= j ? sb[r][tx] : sb[tx][r];
  }
}

static void full_gram_params(GemmParams& p, int64_t T, int64_t K, int sms) {
  p.tiles_m = p.tiles_n = (K + 255) / 256;
  const int64_t n = full_gram_tiles(K);
  p.tiles_per_seg = n;
  p.seg_rows = kGramSegmentRows;
  const int64_t segs = (T + p.seg_rows - 1) / p.seg_rows;
  p.n_tiles = n * segs;
  p.band = kGramBand;
  p.tail_start = p.n_tiles;
  p.tail_tiles = 1;
  const int64_t r = p.n_tiles % sms;
  if (r == 0 || r > n || sms < 2) return;
  const int64_t last_r0 = (segs - 1) * p.seg_rows, last_rows = T - last_r0;
  int64_t m = (int64_t)(sqrt((double)last_rows / kGramEpilogueRows) + 0.5);
  if (m > sms / r) m = sms / r;
  if (m < 2) return;
  int64_t piece = ((last_rows + m - 1) / m + kBK - 1) / kBK * kBK;
  m = (last_rows + piece - 1) / piece;  // every piece non-empty
  if (m < 2) return;
  p.tail_start = p.n_tiles - r;
  p.tail_tiles = r;
  p.tail_tile0 = n - r;
  p.tail_r0 = last_r0;
  p.tail_piece_rows = piece;
  p.last_seg = segs - 1;
  p.n_tiles = p.tail_start + r * m;
}

}  // namespace qz

using namespace qz;

extern "C" int qz_gram(const uint16_t* X, int64_t T, int64_t K, int mode, int block_size, int accumulate,
                       float* H, void* stream) {
  if (mode != QZ_GRAM_FULL && mode != QZ_GRAM_BLOCKDIAG && mode != QZ_GRAM_FULL_UPPER_TILES)
    return fail(QZ_ERR_INVALID, "unknown gram mode %d", mode);
  if (T < 0 || K <= 0) return fail(QZ_ERR_INVALID, "need T >= 0 and K > 0");
  if (K % 8 != 0) return fail(QZ_ERR_INVALID, "K must be a multiple of 8 (16-byte rows for TMA)");
  if (mode == QZ_GRAM_BLOCKDIAG &&
      ((block_size != 16 && block_size != 32 && block_size != 64 && block_size != 128) || K % block_size != 0))
    return fail(QZ_ERR_INVALID, "block_size must be 16, 32, 64 or 128 and divide K");
  if (K > 2147483647LL || T > 2147483647LL) return fail(QZ_ERR_INVALID, "T and K must fit in int32");
  if (!H) return fail(QZ_ERR_INVALID, "H is NULL");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t n_out = mode == QZ_GRAM_FULL ? K * K
                        : mode == QZ_GRAM_FULL_UPPER_TILES ? full_gram_tiles(K) * 65536 : K * block_size;
  if (T == 0) {
    if (accumulate) return QZ_OK;
    return cuda_status(cudaMemsetAsync(H, 0, (size_t)n_out * 4, st), "cudaMemsetAsync");
  }
  if (!X) return fail(QZ_ERR_INVALID, "X is NULL");
  if (reinterpret_cast<uintptr_t>(X) % 16) return fail(QZ_ERR_INVALID, "X must be 16-byte aligned");
  GemmParams p{};
  p.K = K; p.M = 0; p.bs = block_size; p.H = H;
  p.lbo = kMnLbo;
  p.sbo = kMnSbo;
  p.tiles_m = (K + kBM - 1) / kBM;
  int sms = 0;
  int s = current_sms(&sms);
  if (s != QZ_OK) return s;
  if (mode == QZ_GRAM_FULL || mode == QZ_GRAM_FULL_UPPER_TILES) {
    if (mode == QZ_GRAM_FULL_UPPER_TILES) p.packed = H;
    // One persistent launch over (segment, tile) units, segment-major: all CTAs
    // sweep the same token rows at about the same time, so the column panels
    // they share stay in L2.  A tile's segments are added in segment order
    // (per-tile counters in scratch), so H is deterministic and exactly symmetric.
    full_gram_params(p, T, K, sms);
    const int64_t n = p.tiles_per_seg;
    p.T = T;
    p.accumulate = accumulate;
    CUtensorMap map;
    s = make_map(&map, X, (uint64_t)K, (uint64_t)T, 64, 64);
    if (s != QZ_OK) return s;
    int* seq = nullptr;
    cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&seq), (size_t)n * sizeof(int), st);
    if (e != cudaSuccess) return cuda_status(e, "cudaMallocAsync (gram tile counters)");
    e = cudaMemsetAsync(seq, 0, (size_t)n * sizeof(int), st);
    p.seq = seq;
    s = e == cudaSuccess ? launch_gemm<kGramFull>(map, map, map, p, st) : cuda_status(e, "cudaMemsetAsync");
    cudaFreeAsync(seq, st);
    return s;
  }
  // Block-diagonal: (split, diagonal tile) units; split 0 writes H, the others
  // write scratch partials that one more pass adds in split order.
  CUtensorMap map;
  s = make_map(&map, X, (uint64_t)K, (uint64_t)T, 64, 64);
  if (s != QZ_OK) return s;
  p.T = T;
  p.accumulate = accumulate;
  p.tiles_n = 1;
  // Token splits: every CTA runs whole (tile, split) units, so the count is
  // chosen to minimise waves x (rows per unit + a unit's fixed cost in rows),
  // with at least 4096 rows per unit (tiles x splits a multiple of the SM
  // count fills every wave).
  int64_t splits = 1;
  {
    const int64_t max_splits = T / 4096 < 1024 ? T / 4096 : 1024;
    int64_t best = -1;
    for (int64_t S = 1; S <= (max_splits > 1 ? max_splits : 1); ++S) {
      const int64_t rows = ((T + S - 1) / S + kBK - 1) / kBK * kBK;
      const int64_t units = p.tiles_m * ((T + rows - 1) / rows);
      const int64_t cost = (units + sms - 1) / sms * (rows + kDiagUnitRows);
      if (best < 0 || cost < best) { best = cost; splits = S; }
    }
  }
  p.split_rows = ((T + splits - 1) / splits + kBK - 1) / kBK * kBK;
  splits = (T + p.split_rows - 1) / p.split_rows;
  p.splits = splits;
  p.n_tiles = p.tiles_m * splits;
  const size_t part_elems = (size_t)K * block_size;
  float* parts = nullptr;
  if (splits > 1) {
    cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&parts), (splits - 1) * part_elems * 4, st);
    if (e != cudaSuccess) return cuda_status(e, "cudaMallocAsync (gram partials)");
  }
  p.partials = parts;
  s = launch_gemm<kGramDiag>(map, map, map, p, st);
  if (s == QZ_OK && splits > 1) {
    const int64_t n4 = (int64_t)part_elems / 4;
    add_partials_kernel<<<(unsigned)(sms * 4), 256, 0, st>>>(reinterpret_cast<float4*>(H),
                                                              reinterpret_cast<const float4*>(parts), n4,
                                                              splits - 1);
    s = cuda_status(cudaGetLastError(), "add_partials launch");
  }
  if (parts) cudaFreeAsync(parts, st);
  return s;
}

extern "C" int qz_output_error_sums(const uint16_t* X, int64_t T, int64_t K, const uint16_t* W,
                                    const uint16_t* W_dq, int64_t M, double* sums, void* stream) {
  if (T < 0 || K <= 0 || M <= 0) return fail(QZ_ERR_INVALID, "need T >= 0, K > 0, M > 0");
  if (K % 8 != 0) return fail(QZ_ERR_INVALID, "K must be a multiple of 8 (16-byte rows for TMA)");
  if (K > 2147483647LL || T > 2147483647LL || M > 2147483647LL)
    return fail(QZ_ERR_INVALID, "T, K and M must fit in int32");
  if (!X || !W || !W_dq || !sums) return fail(QZ_ERR_INVALID, "NULL pointer");
  if ((reinterpret_cast<uintptr_t>(X) | reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(W_dq)) % 16)
    return fail(QZ_ERR_INVALID, "X, W and W_dq must be 16-byte aligned");
  if (T == 0) return QZ_OK;
  CUtensorMap mx, mw, mq;
  int s = make_map(&mx, X, (uint64_t)K, (uint64_t)T, 64, 256);
  if (s == QZ_OK) s = make_map(&mw, W, (uint64_t)K, (uint64_t)M, 64, 128);
  if (s == QZ_OK) s = make_map(&mq, W_dq, (uint64_t)K, (uint64_t)M, 64, 128);
  if (s != QZ_OK) return s;
  GemmParams p{};
  p.T = T; p.K = K; p.M = M; p.sums = sums;
  p.tiles_m = (T + Geo<kMetrics>::BM - 1) / Geo<kMetrics>::BM;
  p.tiles_n = (M + 127) / 128;
  p.n_tiles = p.tiles_m * p.tiles_n;
  return launch_gemm<kMetrics>(mx, mw, mq, p, static_cast<cudaStream_t>(stream));
}

extern "C" int qz_gram_unpack(const float* packed, int64_t K, float* H, void* stream) {
  if (K <= 0 || (K + 63) / 64 > 65535) return fail(QZ_ERR_INVALID, "need 0 < K <= 4194240, got %lld", (long long)K);
  if (!packed || !H) return fail(QZ_ERR_INVALID, "NULL pointer");
  const unsigned nb = (unsigned)((K + 63) / 64);
  gram_unpack_kernel<<<dim3(nb, nb), 256, 0, static_cast<cudaStream_t>(stream)>>>(packed, K, (K + 255) / 256, H);
  return cuda_status(cudaGetLastError(), "gram unpack launch");
}

extern "C" int qz_gram_full_noalloc(const uint16_t* X, int64_t T, int64_t K, int accumulate, float* H,
                                    void* stream) {
  if (T < 0 || K <= 0) return fail(QZ_ERR_INVALID, "need T >= 0 and K > 0");
  if (K % 8 != 0) return fail(QZ_ERR_INVALID, "K must be a multiple of 8 (16-byte rows for TMA)");
  if (K > 2147483647LL || T > 2147483647LL) return fail(QZ_ERR_INVALID, "T and K must fit in int32");
  if (!H) return fail(QZ_ERR_INVALID, "H is NULL");
  GemmParams p{};
  const int64_t n = full_gram_tiles(K);
  if (n > kNoAllocMaxTiles)
    return fail(QZ_ERR_INVALID,
                "qz_gram_full_noalloc: K = %lld needs %lld output tiles; the fixed scratch holds %lld "
                "(K <= 92416); use qz_gram",
                (long long)K, (long long)n, (long long)kNoAllocMaxTiles);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (T == 0) {
    if (accumulate) return QZ_OK;
    return cuda_status(cudaMemsetAsync(H, 0, (size_t)K * K * 4, st), "cudaMemsetAsync");
  }
  if (!X) return fail(QZ_ERR_INVALID, "X is NULL");
  if (reinterpret_cast<uintptr_t>(X) % 16) return fail(QZ_ERR_INVALID, "X must be 16-byte aligned");
  int* counters = nullptr;
  int s = noalloc_counters(&counters);
  if (s != QZ_OK) return s;
  // the counters must start at zero; the previous call left them non-zero
  s = cuda_status(cudaMemsetAsync(counters, 0, (size_t)n * sizeof(int), st), "cudaMemsetAsync (counters)");
  if (s != QZ_OK) return s;
  p.K = K; p.M = 0; p.bs = 16; p.H = H; p.T = T; p.accumulate = accumulate;
  p.lbo = kMnLbo;
  p.sbo = kMnSbo;
  int sms = 0;
  s = current_sms(&sms);
  if (s != QZ_OK) return s;
  full_gram_params(p, T, K, sms);
  p.seq = counters;
  CUtensorMap map;
  s = make_map(&map, X, (uint64_t)K, (uint64_t)T, 64, 64);
  if (s != QZ_OK) return s;
  return launch_gemm<kGramFull>(map, map, map, p, st);
}

extern "C" int qz_gptq(float* Wb, float* Qb, const float* Hi, float* Hi_split, const float* h_blocks, int64_t M,
                       int64_t K, int block_size, int format, int method, int group_cols, float* E, double* loss,
                       void* stream) {
  const int bs = block_size;
  if (bs != 16 && bs != 32) return fail(QZ_ERR_INVALID, "block_size must be 16 or 32, got %d", bs);
  if (format != QZ_FMT_NVFP4 && format != QZ_FMT_MXFP4) return fail(QZ_ERR_INVALID, "unknown format %d", format);
  if (method != QZ_METHOD_NAIVE && method != QZ_METHOD_SSE && method != QZ_METHOD_HESSIAN)
    return fail(QZ_ERR_INVALID, "qz_gptq supports the naive, SSE and Hessian methods, got %d", method);
  if (group_cols != 32 && group_cols != 64 && group_cols != 128)
    return fail(QZ_ERR_INVALID, "group_cols must be 32, 64 or 128, got %d", group_cols);
  if (group_cols % bs) return fail(QZ_ERR_INVALID, "group_cols must be a multiple of block_size");
  if (M < 0 || K <= 0 || K % bs) return fail(QZ_ERR_INVALID, "need M >= 0 and K a positive multiple of block_size");
  if (K > 1073741823LL || M > 2147483647LL) return fail(QZ_ERR_INVALID, "M and K too large");
  if (M == 0) return QZ_OK;
  if (!Wb || !Qb || !Hi || !Hi_split || !E || !loss) return fail(QZ_ERR_INVALID, "NULL pointer");
  if (method == QZ_METHOD_HESSIAN && !h_blocks) return fail(QZ_ERR_INVALID, "h_blocks required");
  const uintptr_t al = reinterpret_cast<uintptr_t>(Wb) | reinterpret_cast<uintptr_t>(Qb) |
                       reinterpret_cast<uintptr_t>(Hi) | reinterpret_cast<uintptr_t>(Hi_split) |
                       reinterpret_cast<uintptr_t>(E) | reinterpret_cast<uintptr_t>(h_blocks);
  if (al % 16) return fail(QZ_ERR_INVALID, "all buffers must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int sms = 0;
  int s = current_sms(&sms);
  if (s != QZ_OK) return s;
  s = cuda_status(launch_split_tf32(Hi, Hi_split, Hi_split + K * K, K * K, sms, st), "split_tf32 launch");
  if (s != QZ_OK) return s;
  CUtensorMap map_e, map_h;
  s = make_map(&map_e, E, (uint64_t)(2 * group_cols), (uint64_t)M, 32, 128, true);
  if (s == QZ_OK) s = make_map(&map_h, Hi_split, (uint64_t)K, (uint64_t)(2 * K), 32, 128, true);
  if (s != QZ_OK) return s;
  const int64_t nblk = K / bs, gb = group_cols / bs;
  const int64_t ctas = (M + kGptqRows - 1) / kGptqRows;
  int64_t gi = 0;
  for (int64_t g0 = 0; g0 < nblk; g0 += gb, ++gi) {
    const int64_t gbn = nblk - g0 < gb ? nblk - g0 : gb;
    const bool last = g0 + gbn >= nblk;
    GptqGroupArgs a{Wb, Qb, Hi, h_blocks, last ? nullptr : E, loss + gi * ctas, M, K, (int)g0, (int)gbn,
                    group_cols};
    s = cuda_status(launch_gptq_group(a, bs, format == QZ_FMT_NVFP4 ? 0 : 1, method, st), "gptq group launch");
    if (s != QZ_OK || last) break;
    GemmParams p{};
    p.M = M; p.K = K; p.bs = bs; p.Wb = Wb;
    p.g0c = g0 * bs; p.c1 = (g0 + gbn) * bs; p.gk = group_cols;
    // A: the scaled errors (high parts in columns [0, gk), low parts after);
    // B^T: rows c1 + n of Hi's split copy (high parts; low parts K rows
    // further), the group's columns (Hi is symmetric)
    p.a_x0 = 0; p.a_y0 = 0; p.a_lo_dx = group_cols; p.a_lo_dy = 0;
    p.b_x0 = (int)p.g0c; p.b_y0 = (int)p.c1; p.b_lo_dx = 0; p.b_lo_dy = (int)K;
    p.tiles_m = (M + kBM - 1) / kBM;
    p.tiles_n = (K - p.c1 + 127) / 128;
    p.n_tiles = p.tiles_m * p.tiles_n;
    s = launch_gemm<kGptq>(map_e, map_h, map_h, p, st);
    if (s != QZ_OK) break;
  }
  return s;
}

// ---------------------------------------------------------------------------
// Inverse of a symmetric positive definite matrix by recursive 2 x 2 blocking
// (Schur complements), every product on the tensor cores at fp32 accuracy
// (tf32 high / low pairs, three products).  For A = [A11 A12; A21 A22]:
//   X11 = inv(A11); T = X11 A12; S = A22 - T^T A12; Y = inv(S);
//   U = T Y; inv(A) = [X11 + U T^T, -U; -U^T, Y].
// Blocks are multiples of 32 (the K step of the GEMM); blocks of at most 128
// are inverted directly (Gauss-Jordan in double precision in shared memory).
// ---------------------------------------------------------------------------
namespace qz {

struct SpdWork {
  float* V;    // the matrix (n x n): input, then the inverse
  float* S;    // its split (2n x n): high part rows [0, n), low part rows [n, 2n)
  float *T, *Ts, *Tt, *Tts, *U, *Us;  // workspaces: values (n x n) and splits (2n x n)
  int64_t n;
  int* bad;
  CUtensorMap mS, mTs, mTts, mUs;
  cudaStream_t st;
};

// C (value at C, split at Cs) = alpha A B (+ C): A = rows [ay, ay + m), columns
// [ax, ax + k) of the split buffer behind map_a; B^T = rows [by, by + nn),
// columns [bx, bx + k) of the split buffer behind map_b.
static int tf3_gemm(const SpdWork& w, const CUtensorMap& ma, int ax, int ay, const CUtensorMap& mb, int bx, int by,
                    int64_t m, int64_t nn, int64_t k, float* C, float* Cs, float alpha, int beta,
                    const GemmParams& extra) {
  GemmParams p{};
  p.D1 = extra.D1; p.D1s = extra.D1s; p.d1_sign = extra.d1_sign;
  p.D2 = extra.D2; p.D2s = extra.D2s; p.d2_sign = extra.d2_sign;
  p.M = m; p.N = nn; p.gk = k; p.K = w.n;
  p.a_x0 = ax; p.a_y0 = ay; p.a_lo_dx = 0; p.a_lo_dy = (int)w.n;
  p.b_x0 = bx; p.b_y0 = by; p.b_lo_dx = 0; p.b_lo_dy = (int)w.n;
  p.C = C; p.Cs = Cs; p.ldc = w.n; p.cs_lo = w.n * w.n; p.alpha = alpha; p.beta = beta;
  p.tiles_m = (m + kBM - 1) / kBM;
  p.tiles_n = (nn + 127) / 128;
  p.n_tiles = p.tiles_m * p.tiles_n;
  return launch_gemm<kTf3>(ma, mb, mb, p, w.st);
}

static int spd_inverse_rec(const SpdWork& w, int64_t off, int64_t s) {
  const int64_t n = w.n;
  if (s <= 96)
    return cuda_status(launch_spd_block_inverse(w.V + off * n + off, w.S + off * n + off, n, n * n, (int)s, w.bad,
                                                w.st), "spd block inverse");
  const int64_t s1 = (s / 32 + 1) / 2 * 32, s2 = s - s1, o2 = off + s1;
  // T, T^T and U of this node live in their workspaces at this node's A12 /
  // A21 positions, which no node below it touches (the first child is done
  // before T exists; the second child works at rows and columns >= o2)
  const int64_t p12 = off * n + o2, p21 = o2 * n + off;
  int r = spd_inverse_rec(w, off, s1);  // X11
  if (r != QZ_OK) return r;
  // T = X11 A12  (B^T = A12^T = A21: rows o2.., columns off..); its epilogue
  // also writes T^T
  GemmParams e{};
  e.D2 = w.Tt + p21; e.D2s = w.Tts + p21; e.d2_sign = 1.0f;
  r = tf3_gemm(w, w.mS, (int)off, (int)off, w.mS, (int)off, (int)o2, s1, s2, s1, w.T + p12, w.Ts + p12, 1.0f, 0, e);
  if (r != QZ_OK) return r;
  // S = A22 - T^T A12  (A = T^T: s2 x s1; B^T = A21)
  r = tf3_gemm(w, w.mTts, (int)off, (int)o2, w.mS, (int)off, (int)o2, s2, s2, s1, w.V + o2 * n + o2,
               w.S + o2 * n + o2, -1.0f, 1, GemmParams{});
  if (r != QZ_OK) return r;
  r = spd_inverse_rec(w, o2, s2);  // Y
  if (r != QZ_OK) return r;
  // U = T Y  (B^T = Y, symmetric); its epilogue also writes X12 = -U and X21 = -U^T
  GemmParams u{};
  u.D1 = w.V + p12; u.D1s = w.S + p12; u.d1_sign = -1.0f;
  u.D2 = w.V + p21; u.D2s = w.S + p21; u.d2_sign = -1.0f;
  r = tf3_gemm(w, w.mTs, (int)o2, (int)off, w.mS, (int)o2, (int)o2, s1, s2, s2, w.U + p12, w.Us + p12, 1.0f, 0, u);
  if (r != QZ_OK) return r;
  // X11 += U T^T  (B^T = T)
  return tf3_gemm(w, w.mUs, (int)o2, (int)off, w.mTs, (int)o2, (int)off, s1, s1, s2, w.V + off * n + off,
                  w.S + off * n + off, 1.0f, 1, GemmParams{});
}

}  // namespace qz

extern "C" int qz_spd_inverse(float* A, int64_t n, float* work, int* status, void* stream) {
  if (n <= 0 || n % 32) return fail(QZ_ERR_INVALID, "n must be a positive multiple of 32, got %lld", (long long)n);
  if (n > 46336) return fail(QZ_ERR_INVALID, "n too large (%lld)", (long long)n);
  if (!A || !work || !status) return fail(QZ_ERR_INVALID, "NULL pointer");
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(work)) % 16)
    return fail(QZ_ERR_INVALID, "A and work must be 16-byte aligned");
  int sms = 0;
  int r = current_sms(&sms);
  if (r != QZ_OK) return r;
  SpdWork w{};
  w.n = n; w.V = A; w.bad = status; w.st = static_cast<cudaStream_t>(stream);
  const int64_t nn = n * n;
  w.S = work;
  w.T = work + 2 * nn; w.Ts = w.T + nn;
  w.Tt = w.Ts + 2 * nn; w.Tts = w.Tt + nn;
  w.U = w.Tts + 2 * nn; w.Us = w.U + nn;
  r = cuda_status(cudaMemsetAsync(status, 0, sizeof(int), w.st), "cudaMemsetAsync");
  if (r != QZ_OK) return r;
  r = cuda_status(launch_split_tf32(A, w.S, w.S + nn, nn, sms, w.st), "split_tf32 launch");
  if (r != QZ_OK) return r;
  r = make_map(&w.mS, w.S, (uint64_t)n, (uint64_t)(2 * n), 32, 128, true);
  if (r == QZ_OK) r = make_map(&w.mTs, w.Ts, (uint64_t)n, (uint64_t)(2 * n), 32, 128, true);
  if (r == QZ_OK) r = make_map(&w.mTts, w.Tts, (uint64_t)n, (uint64_t)(2 * n), 32, 128, true);
  if (r == QZ_OK) r = make_map(&w.mUs, w.Us, (uint64_t)n, (uint64_t)(2 * n), 32, 128, true);
  if (r != QZ_OK) return r;
  return spd_inverse_rec(w, 0, n);
}
