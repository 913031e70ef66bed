// lora_ce_kernels.cuh — device code of the LoRA-on-lm_head step.
//
// HBM layout (all device buffers owned by the handle; T = positions of this
// rank, R = LoRA rank, Vpad = V rounded up to 256):
//   W    [V][d]        f16   tied lm_head, uploaded once (K-major operand)
//   h16  [Tcap][d]     f16   hidden states converted by lce_prep
//   Bt   [Vpad][R]     f32   LoRA B, vocab-major (rows >= V are zero)
//   A    [d][R]        f32   LoRA A, reference layout
//   tok  [Tpad][R+4]   f32   per position: s*U[0..R), M, 1/S, target, 0
//   P1 partials        f32   per (segment, position): max, sum, q[R]
//   gBp  [seg][Vpad][R] f32  pass-2 partial dB per CTA segment
//   G    [d*R + V*R + 2]     packed gradient sums | loss sum | n_pred,
//                            the one buffer NCCL all-reduces
//
// The two GEMM passes share one warp-specialised mainloop: a 128-row
// operand tile stays resident in shared memory for a run of consecutive
// tiles while 256-row tiles of the other operand stream through a TMA ring;
// tcgen05.mma accumulates each 128x256 fp32 tile into one of two TMEM
// buffers so the epilogue of tile i overlaps the MMAs of tile i+1.
//   pass 1: resident = 128 positions of h, streamed = 256 vocab rows of W.
//           Each epilogue thread owns one position and keeps an online
//           max / sum(exp) / sum(exp * B[:,v]) over its vocab range.
//   pass 2: resident = 128 vocab rows of W, streamed = 256 positions of h.
//           Each epilogue thread owns one vocab row and accumulates
//           dB[v][:] = sum_t sU[t][:] * (p[t][v] - onehot) over its run of
//           positions.
// Neither epilogue needs a reduction across threads, and the T x V logits
// never leave TMEM/registers.
#pragma once
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include "sm100.cuh"

namespace lce {

constexpr int kBM = 128;               // resident rows per tile (TMEM lanes)
constexpr int kBN = 256;               // streamed rows per tile (TMEM columns)
constexpr int kBK = 64;                // K elements per 128-byte swizzle row
constexpr int kStages = 2;             // streamed-operand ring depth
constexpr int kAKBytes = kBM * kBK * 2;   // 16 KB per resident K-block
constexpr int kBStageBytes = kBN * kBK * 2;  // 32 KB per streamed stage
constexpr int kEpiWarps = 8;           // two per TMEM lane quarter
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr int kThreads = 64 + kEpiThreads;  // warp0 TMA, warp1 MMA, warps 2.. epilogue
constexpr float kLog2e = 1.4426950408889634f;
constexpr uint32_t kTmemCols = 512;    // two 256-column fp32 accumulators
constexpr int kMaxKBlocks = 10;        // d <= 640

__host__ __device__ constexpr int tok_stride(int R) { return R + 4; }

// CTA c of G processes the linear tile range [start(c), start(c+1)),
// start(c) = floor(c * total / G); tiles are numbered a * n_b + b so the
// resident operand changes rarely.  owner(x) is the CTA holding tile x.
__host__ __device__ inline long long tile_start(int c, long long total, int G) {
  return (long long)c * total / G;
}
__host__ __device__ inline int tile_owner(long long x, long long total, int G) {
  return (int)(((x + 1) * (long long)G - 1) / total);
}

struct GemmArgs {
  int n_a, n_b;      // resident-tile count, streamed-tile count
  int kblocks;       // d / 64
  int T, V, R;
  long long Tcap;    // partial-buffer row stride (positions)
  long long Vpad;    // rows of Bt / gBp
  int* err;
  // pass 1
  const float* tok;   // [Tpad][R+4]
  const float* Bt;    // [Vpad][R]
  float* p_max;       // [seg][Tcap]
  float* p_sum;       // [seg][Tcap]
  float* p_q;         // [seg][Tcap][R]
  float* z_tgt;       // [Tcap]
  // pass 2
  float* gBp;         // [seg][Vpad][R]
};

// Dynamic shared memory: [resident K-blocks | streamed ring | staged
// column records (2 x kBN x rec floats, optional) | barriers].
struct SmemLayout {
  static __host__ __device__ constexpr int a_off() { return 0; }
  static __host__ __device__ constexpr int b_off(int kblocks) { return kblocks * kAKBytes; }
  static __host__ __device__ constexpr int rec_off(int kblocks) {
    return b_off(kblocks) + kStages * kBStageBytes;
  }
  static __host__ __device__ constexpr int rec_bytes(int rec_floats) {
    return 2 * kBN * rec_floats * 4;
  }
  static __host__ __device__ constexpr int bar_off(int kblocks, int rec_floats) {
    return rec_off(kblocks) + rec_bytes(rec_floats);
  }
  static __host__ __device__ constexpr int bytes(int kblocks, int rec_floats) {
    return 1024 /*align slack*/ + bar_off(kblocks, rec_floats) + 256;
  }
};
constexpr int kMaxDynSmem = 232448;  // 227 KB opt-in per CTA on sm_100

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// N floats (N % 4 == 0) through 16-byte loads from global or shared memory.
template <int N>
__device__ __forceinline__ void ld_vec(const float* p, float (&v)[N]) {
#pragma unroll
  for (int j = 0; j < N; j += 4) {
    const float4 x = *reinterpret_cast<const float4*>(p + j);
    v[j] = x.x; v[j + 1] = x.y; v[j + 2] = x.z; v[j + 3] = x.w;
  }
}
template <int N>
__device__ __forceinline__ void st_vec(float* p, const float (&v)[N]) {
#pragma unroll
  for (int j = 0; j < N; j += 4)
    *reinterpret_cast<float4*>(p + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
}

// Barrier indices inside the barrier block.
enum : int {
  kBarFull = 0,                    // [kStages] stage loaded
  kBarEmpty = kBarFull + kStages,  // [kStages] stage consumed by MMA
  kBarAFull = kBarEmpty + kStages, // resident tile loaded
  kBarAEmpty,                      // resident tile no longer read
  kBarAccFull,                     // [2] accumulator ready
  kBarAccEmpty = kBarAccFull + 2,  // [2] accumulator drained
  kBarDrain = kBarAccEmpty + 2,    // end-of-kernel MMA drain
  kNumBars
};

// Wait that ignores the shared error flag (used only to drain copies and
// MMAs still in flight before the CTA exits).
__device__ __forceinline__ void mbar_drain_wait(uint64_t* bar, uint32_t parity, int* err) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kWaitTimeoutNs) {
      atomicCAS(err, 0, kErrDrain);
      return;
    }
  }
}

// ------------------------------------------------------------- epilogues
// Each epilogue struct owns one TMEM lane (a resident row) and consumes the
// columns of the streamed tile in chunks of kCW.  Per column it needs a
// small record (kRec floats): the mainloop stages the records of a whole
// tile in shared memory (or points at them in global memory, where the
// layout is the same).

// Pass 1: the thread owns position t; columns are vocab ids; the record of
// column v is B[:, v] (R floats).
template <int R>
struct EpiLse {
  static constexpr int kRec = R;
  static constexpr int kCW = 16;
  static constexpr float kLazy = 8.0f;   // move the reference max only past this
  static constexpr float kRedo = 80.0f;  // re-sum a chunk that jumped this far
  int t;
  bool valid;
  int tgt;
  float sU[R];
  float m, mL, s;  // reference max, m*log2(e), sum of e^(z-m)
  float q[R];      // sum of e^(z-m) * B[:, v]

  __device__ static const float* global_recs(const GemmArgs& g, int b) {
    return g.Bt + (long long)b * kBN * R;
  }
  __device__ static void load_rec(const GemmArgs& g, int b, int c, float (&r)[kRec]) {
    ld_vec<R>(g.Bt + ((long long)b * kBN + c) * R, r);
  }

  __device__ void begin(const GemmArgs& g, int a, int row) {
    t = a * kBM + row;
    valid = t < g.T;
    const float* tk = g.tok + (long long)(valid ? t : 0) * tok_stride(R);
    ld_vec<R>(tk, sU);
    tgt = valid ? __float_as_int(tk[R + 2]) : -1;
    m = -INFINITY;
    mL = -INFINITY;
    s = 0.f;
#pragma unroll
    for (int j = 0; j < R; ++j) q[j] = 0.f;
  }

  // One pass per column: z = acc + sU.B[:,v], e = e^(z - m), s += e,
  // q += e*B[:,v], where m only moves (and s, q are rescaled) when the
  // chunk max exceeds it by more than kLazy, so terms up to e^kLazy are
  // summed at full precision; a chunk more than kRedo above m (the first
  // chunk, or a jump that could have overflowed) is summed again.
  __device__ __forceinline__ void chunk(const GemmArgs& g, int v0, float (&acc)[kCW],
                                        const float* recs) {
    if (v0 >= g.V) return;
    const float s_old = s;
    float q_old[R];
#pragma unroll
    for (int j = 0; j < R; ++j) q_old[j] = q[j];
    const bool tail = v0 + kCW > g.V;
    float cm = -INFINITY;
#pragma unroll
    for (int i = 0; i < kCW; ++i) {
      float bv[R];
      ld_vec<R>(recs + i * R, bv);
      float z = acc[i];
#pragma unroll
      for (int j = 0; j < R; ++j) z = fmaf(sU[j], bv[j], z);
      if (tail && v0 + i >= g.V) z = -INFINITY;
      acc[i] = z;
      cm = fmaxf(cm, z);
      const float e = ex2f(fmaf(z, kLog2e, -mL));
      s += e;
#pragma unroll
      for (int j = 0; j < R; ++j) q[j] = fmaf(e, bv[j], q[j]);
    }
    if (cm > m + kLazy) {
      if (cm - m <= kRedo) {
        const float f = ex2f((m - cm) * kLog2e);
        s *= f;
#pragma unroll
        for (int j = 0; j < R; ++j) q[j] *= f;
      } else {
        const float f = ex2f((m - cm) * kLog2e);  // 0 when m = -inf
        const float cmL = cm * kLog2e;
        s = s_old * f;
#pragma unroll
        for (int j = 0; j < R; ++j) q[j] = q_old[j] * f;
        const volatile float* vr = recs;  // fresh loads: keeps the first loop's rows dead
#pragma unroll
        for (int i = 0; i < kCW; ++i) {
          const float e = ex2f(fmaf(acc[i], kLog2e, -cmL));
          s += e;
#pragma unroll
          for (int j = 0; j < R; ++j) q[j] = fmaf(e, vr[i * R + j], q[j]);
        }
      }
      m = cm;
      mL = cm * kLog2e;
    }
    if (valid && (unsigned)(tgt - v0) < (unsigned)kCW) {
      // Opaque selects keep acc[] in registers (a plain acc[tgt - v0] would
      // move the whole array to local memory).
      float zt = 0.f;
      const int k = tgt - v0;
#pragma unroll
      for (int i = 0; i < kCW; ++i)
        asm("{\n\t.reg .pred p;\n\tsetp.eq.s32 p, %2, %3;\n\tselp.f32 %0, %1, %0, p;\n\t}"
            : "+f"(zt)
            : "f"(acc[i]), "r"(k), "r"(i));
      g.z_tgt[t] = zt;
    }
  }

  __device__ void flush(const GemmArgs& g, int slot) {
    if (!valid) return;
    const long long o = (long long)slot * g.Tcap + t;
    g.p_max[o] = m;
    g.p_sum[o] = s;
#pragma unroll
    for (int j = 0; j < R; ++j) g.p_q[o * R + j] = q[j];
  }
};

// Pass 2: the thread owns vocab row v; columns are positions; the record
// of position t is {sU[0..R), M*log2(e), 1/S, target, 0}.
template <int R>
struct EpiGrad {
  static constexpr int kRec = R + 4;
  static constexpr int kCW = 16;
  int v;
  bool valid;
  float bv[R];
  float gacc[R];

  __device__ static const float* global_recs(const GemmArgs& g, int b) {
    return g.tok + (long long)b * kBN * kRec;
  }
  __device__ static void load_rec(const GemmArgs& g, int b, int c, float (&r)[kRec]) {
    ld_vec<kRec>(g.tok + ((long long)b * kBN + c) * kRec, r);
  }

  __device__ void begin(const GemmArgs& g, int a, int row) {
    v = a * kBM + row;
    valid = v < g.V;
    ld_vec<R>(g.Bt + (long long)(valid ? v : 0) * R, bv);
#pragma unroll
    for (int j = 0; j < R; ++j) gacc[j] = 0.f;
  }

  // p = e^(z - M) / S = 2^(z*log2(e) - M*log2(e)) * (1/S); dl = p - onehot;
  // dB[v][:] += sU[t][:] * dl.
  __device__ __forceinline__ void chunk(const GemmArgs& g, int t0, float (&acc)[kCW],
                                        const float* recs) {
    if (t0 >= g.T) return;  // padded positions contribute nothing
#pragma unroll
    for (int i = 0; i < kCW; ++i) {
      float su[R];
      ld_vec<R>(recs + i * kRec, su);
      const float4 mi = *reinterpret_cast<const float4*>(recs + i * kRec + R);
      float z = acc[i];
#pragma unroll
      for (int j = 0; j < R; ++j) z = fmaf(bv[j], su[j], z);
      float p = ex2f(fmaf(z, kLog2e, -mi.x)) * mi.y;
      if (__float_as_int(mi.z) == v) p -= 1.0f;
#pragma unroll
      for (int j = 0; j < R; ++j) gacc[j] = fmaf(su[j], p, gacc[j]);
    }
  }

  __device__ void flush(const GemmArgs& g, int slot) {
    if (!valid) return;
    float* o = g.gBp + ((long long)slot * g.Vpad + v) * R;
#pragma unroll
    for (int j = 0; j < R; ++j) o[j] = gacc[j];
  }
};

// ------------------------------------------------------------- mainloop
// kStage: stage the column records of each tile in shared memory (double
// buffered, prefetched one tile ahead); otherwise read them from global.
template <class Epi, bool kStage>
__global__ void __launch_bounds__(kThreads, 1)
    lce_gemm_kernel(const __grid_constant__ CUtensorMap map_res,
                    const __grid_constant__ CUtensorMap map_str, const GemmArgs g) {
  constexpr int kRecF = kStage ? Epi::kRec : 0;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem + SmemLayout::a_off();
  uint8_t* sB = smem + SmemLayout::b_off(g.kblocks);
  float* srec = reinterpret_cast<float*>(smem + SmemLayout::rec_off(g.kblocks));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SmemLayout::bar_off(g.kblocks, kRecF));
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long total = (long long)g.n_a * g.n_b;
  const int G = gridDim.x;
  const long long x_begin = tile_start(blockIdx.x, total, G);
  const long long x_end = tile_start(blockIdx.x + 1, total, G);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&bars[kBarFull + i], 1);
      mbar_init(&bars[kBarEmpty + i], 1);
    }
    mbar_init(&bars[kBarAFull], 1);
    mbar_init(&bars[kBarAEmpty], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[kBarAccFull + i], 1);
      mbar_init(&bars[kBarAccEmpty + i], kEpiThreads / 32);
    }
    mbar_init(&bars[kBarDrain], 1);
    fence_mbar_init();
    prefetch_tmap(&map_res);
    prefetch_tmap(&map_str);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int cur_a = -1;
      uint32_t a_uses = 0;
      int issued_parity[kStages];
      for (int i = 0; i < kStages; ++i) issued_parity[i] = -1;
      bool ok = true;
      for (long long x = x_begin; x < x_end && ok; ++x) {
        const int a = (int)(x / g.n_b);
        const int b = (int)(x % g.n_b);
        if (a != cur_a) {
          if (a_uses > 0 &&
              !mbar_wait(&bars[kBarAEmpty], (a_uses - 1) & 1, g.err, kErrWaitProducer)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&bars[kBarAFull], (uint32_t)(g.kblocks * kAKBytes));
          for (int kb = 0; kb < g.kblocks; ++kb)
            tma_load_2d(sA + kb * kAKBytes, &map_res, &bars[kBarAFull], kb * kBK, a * kBM);
          cur_a = a;
          ++a_uses;
        }
        for (int kb = 0; kb < g.kblocks; ++kb) {
          if (!mbar_wait(&bars[kBarEmpty + stage], phase ^ 1, g.err, kErrWaitProducer)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&bars[kBarFull + stage], (uint32_t)kBStageBytes);
          tma_load_2d(sB + stage * kBStageBytes, &map_str, &bars[kBarFull + stage], kb * kBK,
                      b * kBN);
          issued_parity[stage] = (int)phase;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Never leave the CTA with bulk copies still landing in its smem.
      for (int i = 0; i < kStages; ++i)
        if (issued_parity[i] >= 0) mbar_drain_wait(&bars[kBarFull + i], (uint32_t)issued_parity[i], g.err);
      if (a_uses > 0) mbar_drain_wait(&bars[kBarAFull], (a_uses - 1) & 1, g.err);
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdesc = idesc_f16_f32(kBM, kBN);
      int stage = 0;
      uint32_t phase = 0;
      int cur_a = -1;
      uint32_t a_uses = 0;
      long long li = 0;
      bool ok = true;
      for (long long x = x_begin; x < x_end && ok; ++x, ++li) {
        const int a = (int)(x / g.n_b);
        if (a != cur_a) {
          if (!mbar_wait(&bars[kBarAFull], a_uses & 1, g.err, kErrWaitMma)) break;
          ++a_uses;
          cur_a = a;
        }
        const int buf = (int)(li & 1);
        const uint32_t use = (uint32_t)(li >> 1);
        if (!mbar_wait(&bars[kBarAccEmpty + buf], (use & 1) ^ 1, g.err, kErrWaitMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(buf * kBN);
        for (int kb = 0; kb < g.kblocks; ++kb) {
          if (!mbar_wait(&bars[kBarFull + stage], phase, g.err, kErrWaitMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = sw128_kmajor_desc(smem_u32(sA + kb * kAKBytes));
          const uint64_t bdesc = sw128_kmajor_desc(smem_u32(sB + stage * kBStageBytes));
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_f16(d_tmem, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), kIdesc,
                     (kb | k) != 0 ? 1u : 0u);
          umma_commit(&bars[kBarEmpty + stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&bars[kBarAccFull + buf]);
        if (x + 1 == x_end || (int)((x + 1) / g.n_b) != a) umma_commit(&bars[kBarAEmpty]);
      }
      // All MMAs issued by this thread complete before TMEM is released.
      umma_commit(&bars[kBarDrain]);
      mbar_drain_wait(&bars[kBarDrain], 0, g.err);
    }
  } else {
    // ------------------------------------------------ epilogue (warps 2..9)
    // Warp w reads TMEM lanes 32*(w%4)..+31; warps 2-5 take columns
    // 0..127 of each tile, warps 6-9 columns 128..255, so every resident
    // row has two partial states, flushed to slots 2*segment + half.
    const int e = warp - 2;
    const int quarter = warp & 3;
    const int half = e >> 2;
    const int row = quarter * 32 + lane;
    const int ct = e * 32 + lane;  // the column this thread stages
    const uint32_t lane_addr = tmem_base + ((uint32_t)(quarter * 32) << 16);
    constexpr int CW = Epi::kCW;
    constexpr int NCH = (kBN / 2) / CW;
    Epi epi;
    int cur_a = -1;
    long long li = 0;
    bool failed = false;
    float rec[Epi::kRec];
    if (kStage && x_begin < x_end) Epi::load_rec(g, (int)(x_begin % g.n_b), ct, rec);
    for (long long x = x_begin; x < x_end; ++x, ++li) {
      const int a = (int)(x / g.n_b);
      const int b = (int)(x % g.n_b);
      if (a != cur_a) {
        if (cur_a >= 0 && !failed)
          epi.flush(g, 2 * (blockIdx.x - tile_owner((long long)cur_a * g.n_b, total, G)) + half);
        epi.begin(g, a, row);
        cur_a = a;
      }
      const float* recs;
      if constexpr (kStage) {
        // Every epilogue thread reaches this barrier once per tile, also
        // after a failed wait, so the barrier count always matches.
        float* buf = srec + (li & 1) * (kBN * Epi::kRec);
        st_vec<Epi::kRec>(buf + ct * Epi::kRec, rec);
        named_bar_sync(1, kEpiThreads);
        if (x + 1 < x_end) Epi::load_rec(g, (int)((x + 1) % g.n_b), ct, rec);
        recs = buf;
      } else {
        recs = Epi::global_recs(g, b);
      }
      if (failed) continue;
      const int buf = (int)(li & 1);
      const uint32_t use = (uint32_t)(li >> 1);
      if (!mbar_wait(&bars[kBarAccFull + buf], use & 1, g.err, kErrWaitEpilogue)) {
        failed = true;
        continue;
      }
      tc_fence_after();
      {
        // Two register buffers: the TMEM load of chunk c+1 is in flight
        // while chunk c is processed.
        const int col0 = half * (kBN / 2);
        const uint32_t base = lane_addr + (uint32_t)(buf * kBN + col0);
        const float* rb = recs + col0 * Epi::kRec;
        const int gcol = b * kBN + col0;
        float ca[CW], cb[CW];
        tmem_ld<CW>(base, ca);
        tmem_ld_wait<CW>(ca);
#pragma unroll 1
        for (int c = 0; c < NCH; c += 2) {
          tmem_ld<CW>(base + (uint32_t)((c + 1) * CW), cb);
          epi.chunk(g, gcol + c * CW, ca, rb + c * CW * Epi::kRec);
          tmem_ld_wait<CW>(cb);
          if (c + 2 < NCH) tmem_ld<CW>(base + (uint32_t)((c + 2) * CW), ca);
          epi.chunk(g, gcol + (c + 1) * CW, cb, rb + (c + 1) * CW * Epi::kRec);
          if (c + 2 < NCH) tmem_ld_wait<CW>(ca);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kBarAccEmpty + buf]);
    }
    if (cur_a >= 0 && !failed)
      epi.flush(g, 2 * (blockIdx.x - tile_owner((long long)cur_a * g.n_b, total, G)) + half);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ------------------------------------------------------------- small kernels
// h (bf16 / f16 / f32) -> f16 rows; s*U = s*(h16 . A); per-position record
// {sU[0..R), M, 1/S, target, 0} (M, 1/S filled by lce_combine).  One warp
// per position; positions in [T, Tpad) get an all-zero record with target
// -1 so that pass 2 can read whole tiles.
template <int R>
__global__ void lce_prep(const void* __restrict__ H, int dtype, int T, int Tpad, int d,
                         const float* __restrict__ A, float scale,
                         const int32_t* __restrict__ targets, int V,
                         __half* __restrict__ h16, float* __restrict__ tok, int* err) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= Tpad) return;
  float* rec = tok + (long long)w * tok_stride(R);
  if (w >= T) {
    for (int j = lane; j < tok_stride(R); j += 32) rec[j] = 0.f;
    if (lane == 0) rec[R + 2] = __int_as_float(-1);
    return;
  }
  float u[R];
#pragma unroll
  for (int j = 0; j < R; ++j) u[j] = 0.f;
  for (int i = lane; i < d; i += 32) {
    const long long o = (long long)w * d + i;
    float x;
    if (dtype == 0) x = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(H)[o]);
    else if (dtype == 1) x = __half2float(reinterpret_cast<const __half*>(H)[o]);
    else x = reinterpret_cast<const float*>(H)[o];
    const __half hv = __float2half_rn(x);
    h16[o] = hv;
    const float hf = __half2float(hv);
#pragma unroll
    for (int j = 0; j < R; ++j) u[j] = fmaf(hf, A[i * R + j], u[j]);
  }
#pragma unroll
  for (int j = 0; j < R; ++j) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) u[j] += __shfl_xor_sync(0xffffffffu, u[j], off);
  }
  if (lane == 0) {
    int tg = targets[w];
    if (tg < 0 || tg >= V) {
      atomicCAS(err, 0, kErrTarget);
      tg = 0;
    }
#pragma unroll
    for (int j = 0; j < R; ++j) rec[j] = scale * u[j];
    rec[R] = 0.f;
    rec[R + 1] = 0.f;
    rec[R + 2] = __int_as_float(tg);
    rec[R + 3] = 0.f;
  }
}

// Merge the pass-1 partials of each position (two slots per CTA segment,
// one per column half): M = max, S = sum e^(z-M), Q = sum e^(z-M) B[:,v];
// then p_t, loss_t = -log(p_t + 1e-12) and dU_t = s * (Q/S - B[:,target])
// (the reference's d_mid, src/train.c:161-168).  The record of t gets
// M*log2(e) and 1/S for pass 2.
template <int R>
__global__ void lce_combine(int T, int n_b1, int G1, long long Tcap, const float* __restrict__ p_max,
                            const float* __restrict__ p_sum, const float* __restrict__ p_q,
                            const float* __restrict__ z_tgt, const float* __restrict__ Bt,
                            float scale, float* __restrict__ tok, float* __restrict__ dU,
                            float* __restrict__ loss_tok) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  const int a = t / kBM;
  const long long total = (long long)((T + kBM - 1) / kBM) * n_b1;
  const int s0 = tile_owner((long long)a * n_b1, total, G1);
  const int s1 = tile_owner((long long)a * n_b1 + n_b1 - 1, total, G1);
  const int nslot = 2 * (s1 - s0 + 1);
  float M = -INFINITY;
  for (int k = 0; k < nslot; ++k) M = fmaxf(M, p_max[(long long)k * Tcap + t]);
  float S = 0.f, Q[R];
#pragma unroll
  for (int j = 0; j < R; ++j) Q[j] = 0.f;
  for (int k = 0; k < nslot; ++k) {
    const long long o = (long long)k * Tcap + t;
    const float pm = p_max[o];
    if (pm == -INFINITY) continue;  // a half that saw no valid column
    const float f = expf(pm - M);
    S = fmaf(p_sum[o], f, S);
#pragma unroll
    for (int j = 0; j < R; ++j) Q[j] = fmaf(p_q[o * R + j], f, Q[j]);
  }
  const float inv = 1.0f / S;
  float* rec = tok + (long long)t * tok_stride(R);
  const int tg = __float_as_int(rec[R + 2]);
  const float pt = expf(z_tgt[t] - M) * inv;
  loss_tok[t] = -logf(pt + 1e-12f);
  rec[R] = M * kLog2e;
  rec[R + 1] = inv;
#pragma unroll
  for (int j = 0; j < R; ++j) dU[(long long)t * R + j] = scale * (Q[j] * inv - Bt[(long long)tg * R + j]);
}

// dA partials: gAp[c][i][j] = sum over the kDAChunk positions of chunk c
// of h16[t][i] * dU[t][j].
constexpr int kDAChunk = 64;
template <int R>
__global__ void lce_dA_partial(int T, int d, const __half* __restrict__ h16,
                               const float* __restrict__ dU, float* __restrict__ gAp) {
  __shared__ float sdU[kDAChunk * R];
  const int c = blockIdx.x;
  const int t0 = c * kDAChunk;
  const int nt = min(kDAChunk, T - t0);
  for (int k = threadIdx.x; k < nt * R; k += blockDim.x) sdU[k] = dU[(long long)t0 * R + k];
  __syncthreads();
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    float acc[R];
#pragma unroll
    for (int j = 0; j < R; ++j) acc[j] = 0.f;
    for (int tt = 0; tt < nt; ++tt) {
      const float hv = __half2float(h16[(long long)(t0 + tt) * d + i]);
#pragma unroll
      for (int j = 0; j < R; ++j) acc[j] = fmaf(hv, sdU[tt * R + j], acc[j]);
    }
#pragma unroll
    for (int j = 0; j < R; ++j) gAp[((long long)c * d + i) * R + j] = acc[j];
  }
}

// Pack the step's gradient sums: G = [dA (d*R) | dB (V*R, vocab-major) |
// sum of losses | n_pred].  Every output element is summed in a fixed
// order, so the step is deterministic.
template <int R>
__global__ void lce_finalize(int T, int d, int V, long long Vpad, int n_chunks,
                             const float* __restrict__ gAp, int n_b2, int G2,
                             const float* __restrict__ gBp, const float* __restrict__ loss_tok,
                             float* __restrict__ Gbuf) {
  const long long nA = (long long)d * R;
  const long long nB = (long long)V * R;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const int n_a2 = (V + kBM - 1) / kBM;
  const long long total2 = (long long)n_a2 * n_b2;
  for (long long k = (long long)blockIdx.x * blockDim.x + threadIdx.x; k < nA + nB; k += stride) {
    float s = 0.f;
    if (k < nA) {
      for (int c = 0; c < n_chunks; ++c) s += gAp[(long long)c * nA + k];
    } else {
      const long long e = k - nA;
      const int v = (int)(e / R);
      const int a = v / kBM;
      const int s0 = tile_owner((long long)a * n_b2, total2, G2);
      const int s1 = tile_owner((long long)a * n_b2 + n_b2 - 1, total2, G2);
      for (int q = 0; q < 2 * (s1 - s0 + 1); ++q) s += gBp[(long long)q * Vpad * R + e];
    }
    Gbuf[k] = s;
  }
  if (blockIdx.x == 0) {
    __shared__ float red[256];
    float s = 0.f;
    for (int t = threadIdx.x; t < T; t += blockDim.x) s += loss_tok[t];
    red[threadIdx.x] = s;
    __syncthreads();
    for (int w = blockDim.x / 2; w > 0; w >>= 1) {
      if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
      __syncthreads();
    }
    if (threadIdx.x == 0) {
      Gbuf[nA + nB] = red[0];
      Gbuf[nA + nB + 1] = (float)T;
    }
  }
}

// Sum of squares of the mean gradient, per block (global-norm clip).
__global__ void lce_sqnorm(long long n, const float* __restrict__ Gbuf, double* __restrict__ part) {
  __shared__ double red[256];
  const float inv = 1.0f / Gbuf[n + 1];
  double s = 0.0;
  for (long long k = (long long)blockIdx.x * blockDim.x + threadIdx.x; k < n;
       k += (long long)gridDim.x * blockDim.x) {
    const float g = Gbuf[k] * inv;
    s += (double)g * (double)g;
  }
  red[threadIdx.x] = s;
  __syncthreads();
  for (int w = blockDim.x / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) part[blockIdx.x] = red[0];
}

struct AdamArgs {
  long long n;       // d*R + V*R parameters
  float lr, b1, b2, c1, c2, eps, wd;  // c1 = 1 - b1, c2 = 1 - b2 (in f32)
  float b1t, b2t;    // 1 - b^step, computed on the host with powf
  float clip;
  int n_norm_parts;
};

// g = G / n_pred (x clip coefficient); decoupled decay; Adam update
// (src/train.c:175-196), written with explicitly rounded operations so the
// update is the reference's f32 arithmetic, op for op.
__global__ void lce_adam(AdamArgs a, float* __restrict__ params, float* __restrict__ mom1,
                         float* __restrict__ mom2, const float* __restrict__ Gbuf,
                         float* __restrict__ gmean, const double* __restrict__ norm_parts,
                         float* __restrict__ loss_out) {
  const float n_pred = Gbuf[a.n + 1];
  const float inv = __fdiv_rn(1.0f, n_pred);
  float coef = 1.0f;
  if (a.clip > 0.f) {
    double ss = 0.0;
    for (int i = 0; i < a.n_norm_parts; ++i) ss += norm_parts[i];
    const float norm = (float)sqrt(ss);
    const float c = __fdiv_rn(a.clip, __fadd_rn(norm, 1e-6f));
    if (c < 1.0f) coef = c;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && loss_out) *loss_out = __fmul_rn(Gbuf[a.n], inv);
  for (long long k = (long long)blockIdx.x * blockDim.x + threadIdx.x; k < a.n;
       k += (long long)gridDim.x * blockDim.x) {
    float g = __fmul_rn(Gbuf[k], inv);
    if (coef != 1.0f) g = __fmul_rn(g, coef);
    gmean[k] = g;
    float p = params[k];
    if (a.wd > 0.f) p = __fsub_rn(p, __fmul_rn(__fmul_rn(a.lr, a.wd), p));
    const float m = __fadd_rn(__fmul_rn(a.b1, mom1[k]), __fmul_rn(a.c1, g));
    const float v = __fadd_rn(__fmul_rn(a.b2, mom2[k]), __fmul_rn(__fmul_rn(a.c2, g), g));
    mom1[k] = m;
    mom2[k] = v;
    const float mhat = __fdiv_rn(m, a.b1t);
    const float vhat = __fdiv_rn(v, a.b2t);
    p = __fsub_rn(p, __fdiv_rn(__fmul_rn(a.lr, mhat), __fadd_rn(__fsqrt_rn(vhat), a.eps)));
    params[k] = p;
  }
}

}  // namespace lce
