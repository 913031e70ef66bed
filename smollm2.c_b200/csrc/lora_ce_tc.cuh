// lora_ce_tc.cuh — the two GEMM passes with their rank sums on the tensor
// cores (ranks 8 to 64).
//
// The epilogues of lce_gemm_kernel form the rank sums of the step with r
// multiply-adds per logit:
//   pass 1  q[t][:]  = sum_v e^(z[t][v] - m_t) * B[:, v]       (for dU)
//   pass 2  dB[v][:] = sum_t p[t][v] * s*U[t][:]                 (the p part of dB)
// Both are products of the probability tile with a skinny matrix.  Here the
// epilogue only turns each logit tile into probabilities, stored as f16 in
// TMEM, and the MMA warp multiplies that tile (A operand in TMEM) with the
// matching rows of B or s*U (B operand in shared memory, loaded by TMA) into
// a third TMEM accumulator that lives for the whole resident block.  TMEM
// layouts (512 columns):
//   ranks <= 32: [0, 192), [192, 384): logit tiles (double buffered); the
//                probabilities overwrite the tile's own logit columns;
//                [384, 384 + 2R): rank accumulator (hi | lo halves).  The
//                logits of tile i+2 wait for tile i's rank MMAs.
//   rank 64:     [0, 128), [128, 256): logit tiles; [256, 384): a separate
//                probability tile; [384, 512): rank accumulator.  The logits
//                of tile i+1 go into tile i-1's buffer once the epilogue has
//                read it, without waiting for tile i-1's rank MMAs.
//
// Precision: both factors are split x = x_hi + x_lo into f16 pairs.  The
// probability tile is stored as [P_hi (8 cols) | P_lo (8 cols)] per 16
// columns, and the rank operand as 2R rows [X_hi ; X_lo] (the pair's CTAs
// hold the hi and lo rows), so the two MMAs per K-step accumulate
// (P_hi + P_lo) . [X_hi | X_lo] and the rank sum is acc[:, j] + acc[:, R + j]:
// the product to about 2^-22 relative, like the f32 sums it replaces.
// Scaling keeps P in the normal f16 range: pass 1 stores 16 e^(z - m)
// (at most 16 e^8 with the lazy max), pass 2 stores 2^14 p (p <= 1).
//
// Pass 1 needs one max per tile for a row before any probability of the
// tile is written (P cannot be rescaled once in TMEM): the epilogue reads
// the tile twice, first for the max (shared by the two column halves of a
// row through shared memory), then for e^(z - m).  When the max moves past
// the lazy threshold, the row's part of the rank accumulator is rescaled in
// TMEM after the previous tile's rank MMAs have completed.
#pragma once
#include "lora_ce_kernels.cuh"

namespace lce {

// Streamed rows per tile.  Up to rank 32 the probabilities overwrite the
// logit columns they came from (the tile's rank MMAs finish before the next
// logits go into that buffer), so two 192-column logit tiles and the rank
// accumulator fit in TMEM; rank 64 keeps a separate 128-column probability
// tile beside two 128-column logit tiles.
__host__ __device__ constexpr int tc_bn(int R) { return R <= 32 ? 192 : 128; }
__host__ __device__ constexpr bool tc_in_place(int R) { return R <= 32; }
constexpr int kMaxBNT = 192;
constexpr int kMaxStT = 8;
constexpr int kEpiWarpsT = 8;                  // two per TMEM lane quarter
constexpr int kThreadsT = 32 * (kEpiWarpsT + 3);
constexpr int kXWarpT = 2 + kEpiWarpsT;        // rank-operand loader
constexpr uint32_t kPColT = 256;               // separate probability tile (rank 64)
constexpr uint32_t kQColT = 384;               // rank accumulator column
constexpr float kP1Exp = 4.0f;                 // pass 1 stores 2^4 e^(z - m)
constexpr float kP2Exp = 14.0f;                // pass 2 stores 2^14 p
constexpr float kLazyT = 8.0f;                 // pass 1 moves its max only past this
// Smallest rank whose handles use these passes by default.
#ifndef LCE_TC_MIN_RANK
#define LCE_TC_MIN_RANK 16
#endif

enum : int {
  kTFull = 0,
  kTEmpty = kTFull + kMaxStT,
  kTAFull = kTEmpty + kMaxStT,
  kTAEmpty,
  kTZFull,                     // logit tile in TMEM (2 buffers)
  kTPFull = kTZFull + 2,       // probability tile written (the logit buffer read)
  kTPEmpty,                    // rank MMAs done with the probability tile
  kTXFull,                     // rank operand tile loaded (2 buffers)
  kTXEmpty = kTXFull + 2,
  kTQFull = kTXEmpty + 2,      // the block's rank accumulator is complete
  kTQEmpty,                    // ... and has been read
  kTDrain,
  kTAccEmpty,                  // in place: the tile's rank MMAs are done (2 buffers)
  kTNumBars = kTAccEmpty + 2
};

// Dynamic shared memory: [resident K-blocks | ring | rank operand (xbufs
// buffers x 2 K-blocks of R rows) | max exchange (2 x 2 x 128 floats) |
// barriers | TMEM slot].  Rank 64 keeps one rank-operand buffer, so that
// its ring still has 4 stages beside 11 resident K-blocks.
struct TcLayout {
  static __host__ __device__ constexpr int xbufs(int R) { return R >= 64 ? 1 : 2; }
  // streamed K-block of one CTA (tc_bn / 2 rows of 128 B): one ring stage
  static __host__ __device__ constexpr int stage_bytes(int R) { return tc_bn(R) / 2 * kBK * 2; }
  static __host__ __device__ constexpr int ring_off(int kblocks) { return kblocks * kAKBytes; }
  static __host__ __device__ constexpr int x_off(int kblocks, int stages, int R) {
    return ring_off(kblocks) + stages * stage_bytes(R);
  }
  static __host__ __device__ constexpr int x_kblock_bytes(int R) { return R * 128; }
  static __host__ __device__ constexpr int x_buf_bytes(int R) {
    return tc_bn(R) / kBK * x_kblock_bytes(R);
  }
  static __host__ __device__ constexpr int xch_off(int kblocks, int stages, int R) {
    return x_off(kblocks, stages, R) + xbufs(R) * x_buf_bytes(R);
  }
  static __host__ __device__ constexpr int bar_off(int kblocks, int stages, int R) {
    return xch_off(kblocks, stages, R) + 2 * 2 * kBM * 4;
  }
  static __host__ __device__ constexpr int bytes(int kblocks, int stages, int R) {
    return bar_off(kblocks, stages, R) + kTNumBars * 8 + 16;
  }
  // the most ring stages that fit beside the rest
  static __host__ __device__ constexpr int stages(int kblocks, int R) {
    return (kMaxDynSmem - bytes(kblocks, 0, R)) / stage_bytes(R) < kMaxStT
               ? (kMaxDynSmem - bytes(kblocks, 0, R)) / stage_bytes(R)
               : kMaxStT;
  }
};

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ float2 unpack_f16x2(uint32_t u) {
  __half2 h;
  memcpy(&h, &u, 4);
  return __half22float2(h);
}
// x = hi + lo for a column pair: hi = f16(x), lo = f16(x - hi).
__device__ __forceinline__ void split_f16x2(float2 x, uint32_t& hi, uint32_t& lo) {
  hi = pack_f16x2(x.x, x.y);
  const float2 b = unpack_f16x2(hi);
  const float2 r = __ffma2_rn(b, make_float2(-1.f, -1.f), x);  // exact
  lo = pack_f16x2(r.x, r.y);
}

// The streamed tile of linear tile x (in resident row a): each row's tiles
// are rotated so that the cluster owning the row's first tile takes
// streamed tile k mod n_b as its k-th tile.  All clusters then sweep the
// streamed operand (W in pass 1, h in pass 2) in phase, which keeps the
// window of it that they read at one time small in L2.  A rotation of a
// whole row is a permutation of its tiles, so every tile is still taken
// exactly once, and every role of the kernel uses the same mapping.
__device__ __forceinline__ int tc_tile_b(long long x, int a, int n_b, long long total, int G) {
  const long long row0 = (long long)a * n_b;
  const long long start = tile_start(tile_owner(row0, total, G), total, G);  // <= row0
  return (int)((x - start) % n_b);
}

// Rank accumulator of this thread's row: Q[j] = acc[j] + acc[R + j] for
// ranks [j0, j0 + 16) (or all R < 16).  Waits for its own TMEM loads.
template <int R>
__device__ __forceinline__ void read_rank_acc(uint32_t q_addr, int j0, float (&q)[R < 16 ? R : 16]) {
  constexpr int W = R < 16 ? R : 16;
  float a[W], b[W];
  tmem_ld<W>(q_addr + (uint32_t)j0, a);
  tmem_ld<W>(q_addr + (uint32_t)(R + j0), b);
  tmem_ld_wait<W>(a);
  tmem_ld_wait<W>(b);
#pragma unroll
  for (int i = 0; i < W; ++i) q[i] = a[i] + b[i];
}

// kPass 1: resident = positions (h), streamed = vocab rows (W), rank
//          operand = B^T [hi ; lo] (xv, 2R x Vpad);
// kPass 2: resident = vocab rows (W), streamed = positions (h), rank
//          operand = (s*U)^T [hi ; lo] (xt, 2R x Tcap).
// CTA pairs only (cta_group::2, M = 256).  Partial slots as lce_gemm_kernel:
// pass 1 writes per (segment, column half) max / sum / q with q's ranks
// split between the halves (zeros elsewhere); pass 2 writes one dB slot per
// segment, the halves taking half of the ranks each.
template <int kPass, int R>
__global__ void __launch_bounds__(kThreadsT, 1)
    lce_gemm_tc(const __grid_constant__ CUtensorMap map_res,
                const __grid_constant__ CUtensorMap map_str,
                const __grid_constant__ CUtensorMap map_res_aug,
                const __grid_constant__ CUtensorMap map_str_aug,
                const __grid_constant__ CUtensorMap map_x, const GemmArgs g) {
  static_assert(R >= 8 && R <= 64 && R % 8 == 0, "tensor-core rank sums: ranks 8..64");
  constexpr int kXKB = TcLayout::x_kblock_bytes(R);
  constexpr int kXBuf = TcLayout::x_buf_bytes(R);
  constexpr int kXN = TcLayout::xbufs(R);
  constexpr int kBNT = tc_bn(R);
  constexpr bool kInPlace = tc_in_place(R);
  constexpr int kStRowsT = kBNT / 2;
  constexpr int kStBytesT = TcLayout::stage_bytes(R);
  constexpr int kXBlocksT = kBNT / kBK;
  constexpr int kResRows = 2 * kBM;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const int kSt = g.stages;
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  {
    uint32_t dyn_bytes;
    asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn_bytes));
    if (kSt < 2 || kSt > kMaxStT ||
        pad + (uint32_t)TcLayout::bytes(g.kblocks, kSt, R) > dyn_bytes) {
      if (threadIdx.x == 0) atomicCAS(g.err, 0, kErrSmemAlign);
      return;
    }
  }
  uint8_t* smem = smem_raw + pad;
  uint8_t* sA = smem;
  uint8_t* sB = smem + TcLayout::ring_off(g.kblocks);
  uint8_t* sX = smem + TcLayout::x_off(g.kblocks, kSt, R);
  float* xch = reinterpret_cast<float*>(smem + TcLayout::xch_off(g.kblocks, kSt, R));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TcLayout::bar_off(g.kblocks, kSt, R));
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kTNumBars);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const long long total = (long long)g.n_a * g.n_b;
  const int G = gridDim.x / 2;
  const int unit = blockIdx.x / 2;
  const long long x_begin = tile_start(unit, total, G);
  const long long x_end = tile_start(unit + 1, total, G);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kSt; ++i) {
      mbar_init(&bars[kTFull + i], 1);
      mbar_init(&bars[kTEmpty + i], 1);
    }
    mbar_init(&bars[kTAFull], 1);
    mbar_init(&bars[kTAEmpty], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[kTZFull + i], 1);
      mbar_init(&bars[kTXFull + i], 1);
      mbar_init(&bars[kTXEmpty + i], 1);
    }
    mbar_init(&bars[kTPFull], 2 * kEpiWarpsT);
    mbar_init(&bars[kTPEmpty], 1);
    mbar_init(&bars[kTQFull], 1);
    mbar_init(&bars[kTQEmpty], 2 * kEpiWarpsT);
    mbar_init(&bars[kTDrain], 1);
    mbar_init(&bars[kTAccEmpty], 1);
    mbar_init(&bars[kTAccEmpty + 1], 1);
    fence_mbar_init();
    prefetch_tmap(&map_res);
    prefetch_tmap(&map_str);
    prefetch_tmap(&map_x);
    if (g.kblocks > g.kmain) {
      prefetch_tmap(&map_res_aug);
      prefetch_tmap(&map_str_aug);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // peer barriers initialised before any signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int cur_a = -1;
      uint32_t a_uses = 0;
      int issued_parity[kMaxStT];
      for (int i = 0; i < kMaxStT; ++i) issued_parity[i] = -1;
      bool ok = true;
      for (long long x = x_begin; x < x_end && ok; ++x) {
        const int a = (int)(x / g.n_b);
        const int b = tc_tile_b(x, a, g.n_b, total, G);
        if (a != cur_a) {
          if (a_uses > 0 &&
              !mbar_wait(&bars[kTAEmpty], (a_uses - 1) & 1, g.err, kErrWaitProducer)) {
            ok = false;
            break;
          }
          if (leader) mbar_expect_tx(&bars[kTAFull], (uint32_t)(2 * g.kblocks * kAKBytes));
          const int row0 = (g.a0 + a) * kResRows + (int)rank * kBM;
          for (int kb = 0; kb < g.kblocks; ++kb) {
            const CUtensorMap* m = kb < g.kmain ? &map_res : &map_res_aug;
            const int kx = (kb < g.kmain ? kb : kb - g.kmain) * kBK;
            tma_load_2d_pair(sA + kb * kAKBytes, m, mapa_shared(smem_u32(&bars[kTAFull]), 0), kx,
                             row0);
          }
          cur_a = a;
          ++a_uses;
        }
        const int srow0 = b * kBNT + (int)rank * kStRowsT;
        for (int kb = 0; kb < g.kstr; ++kb) {
          if (!mbar_wait(&bars[kTEmpty + stage], phase ^ 1, g.err, kErrWaitProducer)) {
            ok = false;
            break;
          }
          if (leader) mbar_expect_tx(&bars[kTFull + stage], (uint32_t)(2 * kStBytesT));
          const CUtensorMap* m = kb < g.kmain ? &map_str : &map_str_aug;
          const int kx = (kb < g.kmain ? kb : kb - g.kmain) * kBK;
          tma_load_2d_pair(sB + stage * kStBytesT, m,
                           mapa_shared(smem_u32(&bars[kTFull + stage]), 0), kx, srow0);
          issued_parity[stage] = (int)phase;
          if (++stage == kSt) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (leader) {
        for (int i = 0; i < kSt; ++i)
          if (issued_parity[i] >= 0)
            mbar_drain_wait(&bars[kTFull + i], (uint32_t)issued_parity[i], g.err);
        if (a_uses > 0) mbar_drain_wait(&bars[kTAFull], (a_uses - 1) & 1, g.err);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer (leader CTA)
    // Order on the tensor pipe: logits(i), rank(i-1), logits(i+1), rank(i),
    // ...  The logits of tile i+1 go into the buffer of tile i-1, which the
    // epilogue has finished reading before it signalled tile i-1's
    // probabilities (waited for by rank(i-1), issued earlier).
    if (lane == 0 && leader) {
      constexpr uint32_t kIdesc = idesc_f16_f32(kResRows, kBNT);
      constexpr uint32_t kIdescX = idesc_f16_f32(kResRows, 2 * R);
      const uint32_t q_tmem = tmem_base + kQColT;
      const uint32_t p_tmem = tmem_base + kPColT;
      int stage = 0;
      uint32_t phase = 0;
      int cur_a = -1;
      uint32_t a_uses = 0;
      int blk = -1;
      long long li = 0;
      bool ok = true;
      bool have_prev = false, prev_first = false, prev_last = false;
      int prev_blk = 0;
      long long prev_li = 0;
      auto rank_mmas = [&]() -> bool {
        const int xb = (int)(prev_li % kXN);
        if (!mbar_wait(&bars[kTPFull], (uint32_t)(prev_li & 1), g.err, kErrWaitMma)) return false;
        if (!mbar_wait(&bars[kTXFull + xb], (uint32_t)((prev_li / kXN) & 1), g.err, kErrWaitMma))
          return false;
        if (prev_first && prev_blk > 0 &&
            !mbar_wait(&bars[kTQEmpty], (uint32_t)((prev_blk - 1) & 1), g.err, kErrWaitMma))
          return false;
        tc_fence_after();
        const uint8_t* xs = sX + xb * kXBuf;
        const uint32_t p_src = kInPlace ? tmem_base + (uint32_t)((prev_li & 1) * kBNT) : p_tmem;
#pragma unroll
        for (int k = 0; k < kBNT / 16; ++k) {
          const uint64_t bdesc =
              sw128_kmajor_desc(smem_u32(xs + (k >> 2) * kXKB)) + (uint64_t)(2 * (k & 3));
          umma_f16_ts_pair(q_tmem, p_src + (uint32_t)(16 * k), bdesc, kIdescX,
                           (prev_first && k == 0) ? 0u : 1u);
          umma_f16_ts_pair(q_tmem, p_src + (uint32_t)(16 * k + 8), bdesc, kIdescX, 1u);
        }
        umma_commit_pair(&bars[kTXEmpty + xb], 0x3);
        if constexpr (kInPlace) umma_commit_pair(&bars[kTAccEmpty + (int)(prev_li & 1)], 0x3);
        else umma_commit_pair(&bars[kTPEmpty], 0x3);
        if (prev_last) umma_commit_pair(&bars[kTQFull], 0x3);
        return true;
      };
      for (long long x = x_begin; x < x_end && ok; ++x, ++li) {
        const int a = (int)(x / g.n_b);
        const bool first = a != cur_a;
        if (first) {
          if (!mbar_wait(&bars[kTAFull], a_uses & 1, g.err, kErrWaitMma)) break;
          ++a_uses;
          cur_a = a;
          ++blk;
        }
        const int buf = (int)(li & 1);
        // in place, tile li-2's probabilities sit in this buffer until its
        // rank MMAs are done
        if (kInPlace && !mbar_wait(&bars[kTAccEmpty + buf], (uint32_t)(((li >> 1) & 1) ^ 1), g.err,
                                   kErrWaitMma))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(buf * kBNT);
        for (int kb = 0; kb < g.kmain; ++kb) {
          if (!mbar_wait(&bars[kTFull + stage], phase, g.err, kErrWaitMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = sw128_kmajor_desc(smem_u32(sA + kb * kAKBytes));
          const uint64_t bdesc = sw128_kmajor_desc(smem_u32(sB + stage * kStBytesT));
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_f16_pair(d_tmem, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), kIdesc,
                          (kb | k) != 0 ? 1u : 0u);
          umma_commit_pair(&bars[kTEmpty + stage], 0x3);
          if (++stage == kSt) {
            stage = 0;
            phase ^= 1;
          }
        }
        const int n_str_aug = g.kstr - g.kmain;
        int aug_stage[2] = {0, 0};
        for (int i = 0; i < n_str_aug && ok; ++i) {
          if (!mbar_wait(&bars[kTFull + stage], phase, g.err, kErrWaitMma)) {
            ok = false;
            break;
          }
          aug_stage[i] = stage;
          if (++stage == kSt) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        if (n_str_aug > 0) {
          tc_fence_after();
          for (int sidx = 0; sidx < g.n_aug; ++sidx) {
            const int ia = g.aug_a[sidx], ib = g.aug_b[sidx];
            const uint64_t adesc =
                sw128_kmajor_desc(smem_u32(sA + (g.kmain + (ia >> 2)) * kAKBytes)) +
                (uint64_t)(2 * (ia & 3));
            const uint64_t bdesc =
                sw128_kmajor_desc(smem_u32(sB + aug_stage[ib >> 2] * kStBytesT)) +
                (uint64_t)(2 * (ib & 3));
            umma_f16_pair(d_tmem, adesc, bdesc, kIdesc, 1u);
          }
          for (int i = 0; i < n_str_aug; ++i) umma_commit_pair(&bars[kTEmpty + aug_stage[i]], 0x3);
        }
        const bool last_of_a = x + 1 == x_end || (int)((x + 1) / g.n_b) != a;
        umma_commit_pair(&bars[kTZFull + buf], 0x3);
        if (last_of_a) umma_commit_pair(&bars[kTAEmpty], 0x3);
        if (have_prev && !rank_mmas()) {
          ok = false;
          break;
        }
        have_prev = true;
        prev_first = first;
        prev_last = last_of_a;
        prev_li = li;
        prev_blk = blk;
      }
      if (ok && have_prev) rank_mmas();
      // All MMAs issued by this thread complete before TMEM is released.
      umma_commit_pair(&bars[kTDrain], 0x1);
      mbar_drain_wait(&bars[kTDrain], 0, g.err);
    }
  } else if (warp < kXWarpT) {
    // ------------------------------------------------ epilogue (warps 2..9)
    const int e = warp - 2;
    const int quarter = warp & 3;
    const int half = e >> 2;  // column half of every tile (64 columns)
    const int row = quarter * 32 + lane;
    const uint32_t lane_addr = tmem_base + ((uint32_t)(quarter * 32) << 16);
    const uint32_t q_addr = lane_addr + kQColT;
    const uint32_t p_addr = lane_addr + kPColT + (uint32_t)(half * (kBNT / 2));
    constexpr int kHalfCols = kBNT / 2;
    constexpr int NCH = kHalfCols / 16;
    constexpr int kQW = R < 16 ? R : 16;
    const float2 L2 = make_float2(kLog2e, kLog2e);
    int cur_a = -1, blk = -1;
    long long li = 0;
    bool failed = false, first_tile = false;
    // this thread's resident row: pass 1 position t / pass 2 vocab row v
    int rr = 0;
    bool valid = false;
    int tgt = -1;                         // pass 1
    float m = -INFINITY, mL = -INFINITY;  // pass 1 lazy max
    float2 s2 = make_float2(0.f, 0.f);    // pass 1 sum of 16 e^(z - m), even / odd columns

    // The rank accumulator of the finished block: pass 1 q (this half's
    // ranks, zeros for the other half's), pass 2 dB (this half's ranks).
    auto flush_block = [&](int a_done, int blk_done) {
      const int seg = unit - tile_owner((long long)a_done * g.n_b, total, G);
      if (!failed && !mbar_wait(&bars[kTQFull], (uint32_t)(blk_done & 1), g.err, kErrWaitEpilogue))
        failed = true;
      tc_fence_after();
      if (!failed) {
        if constexpr (kPass == 1) {
          const long long o = (long long)(2 * seg + half) * g.Tcap + rr;
          if (valid) {
            g.p_max[o] = m;
            g.p_sum[o] = (s2.x + s2.y) * (1.0f / 16.0f);
          }
#pragma unroll 1
          for (int j0 = 0; j0 < R; j0 += kQW) {
            float q[kQW];
            read_rank_acc<R>(q_addr, j0, q);
            if (valid) {
#pragma unroll
              for (int i = 0; i < kQW; ++i) {
                const int j = j0 + i;
                g.p_q[o * R + j] = (j < R / 2) == (half == 0) ? q[i] * (1.0f / 16.0f) : 0.f;
              }
            }
          }
        } else {
          float* o = g.gBp + (long long)seg * g.Vpad * R;
#pragma unroll 1
          for (int j0 = 0; j0 < R; j0 += kQW) {
            float q[kQW];
            read_rank_acc<R>(q_addr, j0, q);
            if (valid) {
#pragma unroll
              for (int i = 0; i < kQW; ++i) {
                const int j = j0 + i;
                if ((j < R / 2) == (half == 0)) o[bidx(rr, j, R)] = q[i] * (1.0f / 16384.0f);
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&bars[kTQEmpty]), 0));
    };

    for (long long x = x_begin; x < x_end; ++x, ++li) {
      const int a = (int)(x / g.n_b);
      const int b = tc_tile_b(x, a, g.n_b, total, G);
      if (a != cur_a) {
        if (cur_a >= 0) flush_block(cur_a, blk);
        rr = (g.a0 + a) * kResRows + (int)rank * kBM + row;
        if constexpr (kPass == 1) {
          valid = rr < g.T;
          tgt = valid ? __float_as_int(g.tok[tidx(rr, g.rank_total + 2, g.rank_total)]) : -1;
          m = -INFINITY;
          mL = -INFINITY;
          s2 = make_float2(0.f, 0.f);
        } else {
          valid = rr < g.V;
        }
        cur_a = a;
        ++blk;
        first_tile = true;
      }
      const int buf = (int)(li & 1);
      if (!failed && !mbar_wait(&bars[kTZFull + buf], (uint32_t)((li >> 1) & 1), g.err,
                                kErrWaitEpilogue))
        failed = true;
      tc_fence_after();
      const uint32_t zb = lane_addr + (uint32_t)(buf * kBNT + half * kHalfCols);
      const int gcol = b * kBNT + half * kHalfCols;
      const int limit = kPass == 1 ? g.V : g.T;
      const bool tail = gcol + kHalfCols > limit;
      // Probabilities: in place over this tile's logits, or in the separate
      // buffer once tile li-1's rank MMAs are done with it.  Either way a
      // rescale of the rank accumulator waits for those rank MMAs.
      const uint32_t pb = kInPlace ? zb : p_addr;
      bool p_free = kInPlace || li == 0;
      auto wait_p_free = [&]() {
        if (!p_free && !failed &&
            !mbar_wait(&bars[kTPEmpty], (uint32_t)((li - 1) & 1), g.err, kErrWaitEpilogue))
          failed = true;
        p_free = true;
        tc_fence_after();
      };
      auto wait_prev_rank = [&]() {
        if constexpr (kInPlace) {
          if (li > 0 && !failed &&
              !mbar_wait(&bars[kTAccEmpty + (int)((li - 1) & 1)], (uint32_t)(((li - 1) >> 1) & 1),
                         g.err, kErrWaitEpilogue))
            failed = true;
          tc_fence_after();
        } else {
          wait_p_free();
        }
      };
      if constexpr (kPass == 1) {
        // (a) the row's max over the tile; the two halves of a row meet in
        // shared memory (a 64-thread barrier per lane quarter, passed by both
        // warps on every tile, failed or not)
        float cm = -INFINITY;
        if (!failed) {
          constexpr int NL = kHalfCols / 32;
          float zz[NL][32];
#pragma unroll
          for (int l = 0; l < NL; ++l) tmem_ld<32>(zb + (uint32_t)(32 * l), zz[l]);
#pragma unroll
          for (int l = 0; l < NL; ++l) tmem_ld_wait<32>(zz[l]);
          if (tail) {
#pragma unroll
            for (int l = 0; l < NL; ++l)
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (gcol + 32 * l + i >= g.V) zz[l][i] = -INFINITY;
          }
          float mx[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            mx[i] = fmaxf(fmaxf(zz[0][i], zz[0][i + 8]), fmaxf(zz[0][i + 16], zz[0][i + 24]));
#pragma unroll
            for (int l = 1; l < NL; ++l)
              mx[i] = fmaxf(mx[i], fmaxf(fmaxf(zz[l][i], zz[l][i + 8]),
                                         fmaxf(zz[l][i + 16], zz[l][i + 24])));
          }
          cm = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                     fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
        }
        float* xb = xch + (li & 1) * 2 * kBM;
        xb[half * kBM + row] = cm;
        named_bar_sync(1 + quarter, 64);
        cm = fmaxf(cm, xb[(half ^ 1) * kBM + row]);
        if (cm > m + kLazyT) {
          const float f = ex2f((m - cm) * kLog2e);  // 0 when m = -inf
          s2 = __fmul2_rn(s2, make_float2(f, f));
          if (!first_tile) {
            // rescale this half's columns of the rank accumulator once the
            // previous tile's rank MMAs have landed
            wait_prev_rank();
            if (!failed) {
#pragma unroll 1
              for (int j0 = 0; j0 < R; j0 += kQW) {
                float q[kQW];
                uint32_t u[kQW];
                const uint32_t qa = q_addr + (uint32_t)(half * R + j0);
                tmem_ld<kQW>(qa, q);
                tmem_ld_wait<kQW>(q);
#pragma unroll
                for (int i = 0; i < kQW; ++i) u[i] = __float_as_uint(q[i] * f);
                tmem_st<kQW>(qa, u);
              }
            }
          }
          m = cm;
          mL = cm * kLog2e;
        }
        // (b) P = 2^4 e^(z - m) as f16 hi/lo, the sum, the target logit
        const float2 nmL2 = make_float2(kP1Exp - mL, kP1Exp - mL);
        if (!failed) {
          float za[16], zc[16];
          auto chunk = [&](int c, float (&z)[16]) {
            const int v0 = gcol + 16 * c;
            if (tail) {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                if (v0 + i >= g.V) z[i] = -INFINITY;
            }
            uint32_t hi[8], lo[8];
#pragma unroll
            for (int p = 0; p < 8; ++p) {
              const float2 x2 = __ffma2_rn(make_float2(z[2 * p], z[2 * p + 1]), L2, nmL2);
              const float2 e2 = make_float2(ex2f(x2.x), ex2f(x2.y));
              s2 = __fadd2_rn(s2, e2);
              split_f16x2(e2, hi[p], lo[p]);
            }
            if (valid && (unsigned)(tgt - v0) < 16u) {
              float zt = 0.f;
              const int k = tgt - v0;
#pragma unroll
              for (int i = 0; i < 16; ++i)
                asm("{\n\t.reg .pred p;\n\tsetp.eq.s32 p, %2, %3;\n\tselp.f32 %0, %1, %0, p;\n\t}"
                    : "+f"(zt)
                    : "f"(z[i]), "r"(k), "r"(i));
              g.z_tgt[rr] = zt;
            }
            if (c == 0) wait_p_free();
            tmem_st<8>(pb + (uint32_t)(16 * c), hi);
            tmem_st<8>(pb + (uint32_t)(16 * c + 8), lo);
          };
          tmem_ld<16>(zb, za);
          tmem_ld_wait<16>(za);
#pragma unroll
          for (int c = 0; c < NCH; c += 2) {
            tmem_ld<16>(zb + (uint32_t)(16 * (c + 1)), zc);
            chunk(c, za);
            tmem_ld_wait<16>(zc);
            if (c + 2 < NCH) tmem_ld<16>(zb + (uint32_t)(16 * (c + 2)), za);
            chunk(c + 1, zc);
            if (c + 2 < NCH) tmem_ld_wait<16>(za);
          }
        }
      } else {
        // P = 2^14 p = 2^(z log2 e + nml[t]) as f16 hi/lo; positions >= T
        // (tail tiles) contribute nothing
        if (!failed) {
          float za[16], zc[16], na[16], nc[16];
          auto chunk = [&](int c, const float (&z)[16], const float (&nm)[16]) {
            const int t0 = gcol + 16 * c;
            uint32_t hi[8], lo[8];
#pragma unroll
            for (int p = 0; p < 8; ++p) {
              const float2 x2 = __ffma2_rn(make_float2(z[2 * p], z[2 * p + 1]), L2,
                                           make_float2(nm[2 * p], nm[2 * p + 1]));
              float2 e2 = make_float2(ex2f(x2.x), ex2f(x2.y));
              if (tail) {
                if (t0 + 2 * p >= g.T) e2.x = 0.f;
                if (t0 + 2 * p + 1 >= g.T) e2.y = 0.f;
              }
              split_f16x2(e2, hi[p], lo[p]);
            }
            if (c == 0) wait_p_free();
            tmem_st<8>(pb + (uint32_t)(16 * c), hi);
            tmem_st<8>(pb + (uint32_t)(16 * c + 8), lo);
          };
          tmem_ld<16>(zb, za);
          ld_vec<16>(g.nml + gcol, na);
          tmem_ld_wait<16>(za);
#pragma unroll
          for (int c = 0; c < NCH; c += 2) {
            tmem_ld<16>(zb + (uint32_t)(16 * (c + 1)), zc);
            ld_vec<16>(g.nml + gcol + 16 * (c + 1), nc);
            chunk(c, za, na);
            tmem_ld_wait<16>(zc);
            if (c + 2 < NCH) {
              tmem_ld<16>(zb + (uint32_t)(16 * (c + 2)), za);
              ld_vec<16>(g.nml + gcol + 16 * (c + 2), na);
            }
            chunk(c + 1, zc, nc);
            if (c + 2 < NCH) tmem_ld_wait<16>(za);
          }
        }
      }
      if (!p_free) wait_p_free();  // a failed tile still keeps the barrier phases in step
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&bars[kTPFull]), 0));
      first_tile = false;
    }
    if (cur_a >= 0) flush_block(cur_a, blk);
  } else if (warp == kXWarpT) {
    // ------------------------------------------------ rank-operand loader (both CTAs)
    // Tile li's columns of [X_hi ; X_lo] go to buffer li % kXN: this CTA
    // loads its R rows (the leader the hi rows, the peer the lo rows) once
    // tile li-kXN's rank MMAs are done with that buffer.
    if (lane == 0) {
      long long li = 0;
      for (long long x = x_begin; x < x_end; ++x, ++li) {
        const int b = tc_tile_b(x, (int)(x / g.n_b), g.n_b, total, G);
        const int xb = (int)(li % kXN);
        const long long use = li / kXN;
        if (use >= 1 && !mbar_wait(&bars[kTXEmpty + xb], (uint32_t)((use - 1) & 1), g.err,
                                   kErrWaitProducer))
          break;
        if (leader) mbar_expect_tx(&bars[kTXFull + xb], (uint32_t)(2 * kXBuf));
        for (int kb = 0; kb < kXBlocksT; ++kb)
          tma_load_2d_pair(sX + xb * kXBuf + kb * kXKB, &map_x,
                           mapa_shared(smem_u32(&bars[kTXFull + xb]), 0), b * kBNT + kb * kBK,
                           (int)rank * R);
      }
      if (leader)
        for (long long k = li - kXN < 0 ? 0 : li - kXN; k < li; ++k)
          mbar_drain_wait(&bars[kTXFull + (int)(k % kXN)], (uint32_t)((k / kXN) & 1), g.err);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

// Pass 1's rank operand: xv[j][v] = f16(B[j][v]), xv[R + j][v] = f16(B[j][v] - hi)
// for v < V (TMA fills the columns past V with zeros).
template <int R>
__global__ void lce_xt_vocab(int V, long long ld, const float* __restrict__ Bt,
                             __half* __restrict__ xv) {
  const long long n = (long long)V * R;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long k = (long long)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += stride) {
    const int j = (int)(k / V), v = (int)(k % V);
    const float x = Bt[bidx(v, j, R)];
    const __half hi = __float2half_rn(x);
    xv[(long long)j * ld + v] = hi;
    xv[(long long)(R + j) * ld + v] = __float2half_rn(x - __half2float(hi));
  }
}

// Pass 2's rank operand and per-position scalar from the position records:
// xt[j][t] = f16(sU[t][j]) hi / lo, nml[t] = -M*log2(e) + log2(1/S) + 14.
template <int R>
__global__ void lce_xt_pos(int T, long long ld, const float* __restrict__ tok,
                           __half* __restrict__ xt, float* __restrict__ nml) {
  const long long n = (long long)T * R;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long k = (long long)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += stride) {
    const int j = (int)(k / T), t = (int)(k % T);
    const float x = tok[tidx(t, j, R)];
    const __half hi = __float2half_rn(x);
    xt[(long long)j * ld + t] = hi;
    xt[(long long)(R + j) * ld + t] = __float2half_rn(x - __half2float(hi));
    if (j == 0) nml[t] = tok[tidx(t, R, R)] + log2f(tok[tidx(t, R + 1, R)]) + kP2Exp;
  }
}

}  // namespace lce
