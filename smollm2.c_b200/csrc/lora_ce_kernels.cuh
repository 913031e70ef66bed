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
//
// Rank augmentation (ranks 8 to 64): the LoRA term of the logits,
// s*U[t].B[:,v], joins the tensor-core product as extra K-blocks, with
// x_hi = f16(x), x_lo = f16(x - x_hi):
//   layout 1 (ranks 8, 16; one 64-wide block)
//     haug[t] = [sU_hi | sU_hi | sU_lo | 0],  waug[v] = [B_hi | B_lo | B_hi | 0]
//   layout 2 (ranks 32, 64; 2R columns)
//     haug[t] = [sU_hi | sU_lo],  waug[v] = [B_hi | B_lo]
//     with K-steps pairing the hi.hi, hi.lo and lo.hi column slices
//     (GemmArgs::aug_a / aug_b).
// Either way the accumulator holds h.W + sU_hi.B_hi + sU_hi.B_lo +
// sU_lo.B_hi: the rank term to about 2^-22 relative (only lo.lo is dropped),
// and the epilogues skip r multiply-adds per logit.  At rank 4 the extra
// K-block (11% more MMA work) costs more than the four multiply-adds it
// saves, so rank 4 keeps the term in the epilogue.  Ranks 32 and 64 run each
// pass once per 16-rank chunk of the epilogue sums (GemmArgs::rank_off).
#pragma once
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include "sm100.cuh"

namespace lce {

constexpr int kBM = 128;               // resident rows per tile (TMEM lanes)
constexpr int kBN = 256;               // streamed rows per tile (TMEM columns)
constexpr int kBK = 64;                // K elements per 128-byte swizzle row
constexpr int kRingBytes = 65536;      // streamed-operand ring (2 x 32 KB, or 4 x 16 KB per CTA in pairs)
constexpr int kMaxStages = 4;
constexpr int kAKBytes = kBM * kBK * 2;   // 16 KB per resident K-block
// Per-CTA streamed rows per tile and stage geometry for 1-CTA (kPair 1) and
// CTA-pair (kPair 2, cta_group::2) tiles.
__host__ __device__ constexpr int str_rows(int pair) { return kBN / pair; }
__host__ __device__ constexpr int stage_bytes(int pair) { return str_rows(pair) * kBK * 2; }
__host__ __device__ constexpr int num_stages(int pair) { return kRingBytes / stage_bytes(pair); }
// In CTA pairs a pass runs the ring of its epilogue (Epi::kRing, at least
// two 16 KB stages), smaller beside many resident K-blocks to leave room for
// staged records; single CTAs use kRingBytes.
template <class Epi, bool kStage, int kPair>
__host__ __device__ constexpr int ring_bytes() {
  return kPair == 2 ? Epi::kRing : kRingBytes;
}
// Warp roles: warp 0 TMA producer, warp 1 MMA issuer, then kEpiWarps
// epilogue warps (4 or 2 per TMEM lane quarter, set per epilogue by its
// register needs), then one record-loader warp.
__host__ __device__ constexpr int epi_threads(int epi_warps) { return 32 * epi_warps; }
__host__ __device__ constexpr int col_parts(int epi_warps) { return epi_warps / 4; }
__host__ __device__ constexpr int block_threads(int epi_warps) { return 32 * (epi_warps + 3); }
constexpr float kLog2e = 1.4426950408889634f;
constexpr uint32_t kTmemCols = 512;    // two 256-column fp32 accumulators
constexpr int kMaxKBlocks = 12;        // resident K-blocks: d/64 plus rank augmentation
// Smallest rank whose LoRA term joins the MMA as an extra K-block.
#ifndef LCE_AUG_MIN_RANK
#define LCE_AUG_MIN_RANK 8
#endif

// Pair-interleaved layouts.  B (vocab-major) and the per-position records
// keep the same field of two consecutive columns side by side, so one
// 16-byte load yields float2 operands for a column pair:
//   B:   bidx(v, j)    = (v/2)*2R + 2j + v%2               (j < R)
//   tok: tidx(t, f)    = (t/2)*2(R+4) + 2f + t%2, fields f:
//        0..R-1 s*U[t][:], R: -M*log2(e), R+1: 1/S, R+2: target (int bits), R+3: 0
// A whole 256-column tile is one contiguous block in either layout.
__host__ __device__ constexpr int tok_stride(int R) { return R + 4; }
// A rank chunk's pass-2 record of position t: fields 0..15 sU of the
// chunk's 16 ranks, 16: -M*log2(e), 17: 1/S, pair-interleaved like tidx.
constexpr int kChunkRec = 18;
__host__ __device__ inline long long crec_idx(long long t, int f) {
  return (t >> 1) * 2 * kChunkRec + 2 * f + (t & 1);
}
__host__ __device__ inline long long bidx(long long v, int j, int R) {
  return (v >> 1) * 2 * R + 2 * j + (v & 1);
}
__host__ __device__ inline long long tidx(long long t, int f, int R) {
  return (t >> 1) * 2 * (R + 4) + 2 * f + (t & 1);
}

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
  int kblocks;       // resident K-blocks: kmain, plus the rank-augmentation blocks
  int kstr;          // streamed K-blocks per tile: kmain, plus the rank-augmentation blocks
  int kmain;         // d / 64 K-blocks of h / W
  int a0;            // first resident block of this launch (pass 1 runs per chunk of positions)
  // Rank augmentation: after the kmain K-blocks, MMA K-step s (16 wide)
  // pairs column slice aug_a[s] of the resident augmentation blocks with
  // slice aug_b[s] of the streamed ones (slice i = block i/4, columns
  // 16*(i%4) ..), so that hi/lo products can be formed from any layout.
  int n_aug;
  uint8_t aug_a[16], aug_b[16];
  // Ranks: the epilogue handles ranks [rank_off, rank_off + R) of a rank
  // of rank_total (larger ranks run as chunks of 16, one launch each).
  int rank_total, rank_off;
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
  // tensor-core rank sums (lce_gemm_tc)
  int stages;         // streamed-operand ring stages
  const float* nml;   // pass 2: per position -M*log2(e) + log2(1/S) + 14
};

// Dynamic shared memory: [resident K-blocks | streamed ring (ring bytes) | staged
// column records (2 x kBN x rec floats, optional) | barriers].
struct SmemLayout {
  static __host__ __device__ constexpr int a_off() { return 0; }
  static __host__ __device__ constexpr int b_off(int kblocks) { return kblocks * kAKBytes; }
  static __host__ __device__ constexpr int rec_off(int kblocks, int ring) {
    return b_off(kblocks) + ring;
  }
  // rec_floats: floats per column summed over the record buffers
  static __host__ __device__ constexpr int rec_bytes(int rec_floats) {
    return kBN * rec_floats * 4;
  }
  static __host__ __device__ constexpr int bar_off(int kblocks, int rec_floats, int ring) {
    return rec_off(kblocks, ring) + rec_bytes(rec_floats);
  }
  // The dynamic shared array is declared 1024-byte aligned, so no slack is
  // reserved for aligning it; the kernel checks the alignment it got.
  static __host__ __device__ constexpr int bytes(int kblocks, int rec_floats, int ring) {
    return bar_off(kblocks, rec_floats, ring) + 256;
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
  kBarFull = 0,                       // [kMaxStages] stage loaded
  kBarEmpty = kBarFull + kMaxStages,  // [kMaxStages] stage consumed by MMA
  kBarAFull = kBarEmpty + kMaxStages, // resident tile loaded
  kBarAEmpty,                      // resident tile no longer read
  kBarAccFull,                     // [2] accumulator ready
  kBarAccEmpty = kBarAccFull + 2,  // [2] accumulator drained
  kBarDrain = kBarAccEmpty + 2,    // end-of-kernel MMA drain
  kBarRecFull,                     // [2] tile records loaded
  kBarRecEmpty = kBarRecFull + 2,  // [2] tile records no longer read
  kNumBars = kBarRecEmpty + 2
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

__device__ __forceinline__ float2 f2(float x, float y) { return make_float2(x, y); }

// Pass 1: the thread owns position t; columns are vocab ids; the records of
// a column pair are B[:, v], B[:, v+1] interleaved (2R floats).
template <int R, bool kAug_ = (R >= LCE_AUG_MIN_RANK), bool kChunk = false>
struct EpiLse {
  static constexpr bool kAug = kAug_;  // rank term in the accumulator
  static constexpr int kRec = R;  // floats per column
  // ring (CTA pairs): 3 stages beside 10 resident K-blocks at rank 8, 2 at
  // rank 16 and in rank chunks (up to 11 resident K-blocks)
  static constexpr int kRing = !kAug ? kRingBytes : (R >= 16 || kChunk) ? 32768 : 49152;
  // staged record buffers (tile i+1 loads during tile i); a rank chunk
  // beside 11 resident K-blocks has room for one
  static constexpr int kRecBufs = kChunk ? 1 : 2;
  static constexpr int kWarps = R == 4 ? 16 : 8;  // 16 at rank 8 would spill
  static constexpr int kCW = (R >= 16 || kWarps == 16) ? 8 : 16;
  static constexpr float kLazy = 8.0f;   // move the reference max only past this
  static constexpr float kRedo = 80.0f;  // re-sum a chunk that jumped this far
  int t;
  bool valid;
  int tgt;
  float2 sU2[R];  // (s*U[t][j], s*U[t][j])
  float m, mL;    // reference max, m*log2(e)
  float2 s2;      // sum of e^(z-m) over even / odd columns
  float2 q2[R];   // sum of e^(z-m) * B[j][v] over even / odd columns

  __device__ static const float* global_recs(const GemmArgs& g, int b) {
    return g.Bt + (long long)b * kBN * R;
  }
  __device__ static int limit(const GemmArgs& g) { return g.V; }

  __device__ void begin(const GemmArgs& g, int abs_row) {
    t = abs_row;
    valid = t < g.T;
    const long long tt = valid ? t : 0;
    if constexpr (!kAug) {
#pragma unroll
      for (int j = 0; j < R; ++j) {
        const float u = g.tok[tidx(tt, j, R)];
        sU2[j] = f2(u, u);
      }
    }
    tgt = valid ? __float_as_int(g.tok[tidx(tt, g.rank_total + 2, g.rank_total)]) : -1;
    m = -INFINITY;
    mL = -INFINITY;
    s2 = f2(0.f, 0.f);
#pragma unroll
    for (int j = 0; j < R; ++j) q2[j] = f2(0.f, 0.f);
  }

  // Per column: z = acc + sU.B[:,v], e = e^(z - m), s += e, q += e*B[:,v],
  // two columns per f32x2 instruction.  m only moves (and s, q are
  // rescaled) when the chunk max exceeds it by more than kLazy, so terms up
  // to e^kLazy are summed at full precision; a chunk more than kRedo above
  // m (the first chunk, or a jump that could have overflowed) is summed
  // again against its own max.
  template <bool kTail>
  __device__ __forceinline__ void chunk(const GemmArgs& g, int v0, float (&acc)[kCW],
                                        const float* recs) {
    if (kTail && v0 >= g.V) return;
    const float2 s_old = s2;
    float2 q_old[R];
#pragma unroll
    for (int j = 0; j < R; ++j) q_old[j] = q2[j];
    const float2 L2 = f2(kLog2e, kLog2e);
    const float2 nmL2 = f2(-mL, -mL);
    float cm = -INFINITY;
#pragma unroll
    for (int p = 0; p < kCW / 2; ++p) {
      float b[2 * R];
      ld_vec<2 * R>(recs + p * 2 * R, b);
      float2 z2 = f2(acc[2 * p], acc[2 * p + 1]);
      if constexpr (!kAug) {
#pragma unroll
        for (int j = 0; j < R; ++j) z2 = __ffma2_rn(sU2[j], f2(b[2 * j], b[2 * j + 1]), z2);
      }
      if (kTail) {
        if (v0 + 2 * p >= g.V) z2.x = -INFINITY;
        if (v0 + 2 * p + 1 >= g.V) z2.y = -INFINITY;
      }
      acc[2 * p] = z2.x;
      acc[2 * p + 1] = z2.y;
      cm = fmaxf(cm, fmaxf(z2.x, z2.y));
      const float2 x2 = __ffma2_rn(z2, L2, nmL2);
      const float2 e2 = f2(ex2f(x2.x), ex2f(x2.y));
      s2 = __fadd2_rn(s2, e2);
#pragma unroll
      for (int j = 0; j < R; ++j) q2[j] = __ffma2_rn(e2, f2(b[2 * j], b[2 * j + 1]), q2[j]);
    }
    if (cm > m + kLazy) {
      const float f = ex2f((m - cm) * kLog2e);  // 0 when m = -inf
      const float2 ff = f2(f, f);
      if (cm - m <= kRedo) {
        s2 = __fmul2_rn(s2, ff);
#pragma unroll
        for (int j = 0; j < R; ++j) q2[j] = __fmul2_rn(q2[j], ff);
      } else {
        s2 = __fmul2_rn(s_old, ff);
#pragma unroll
        for (int j = 0; j < R; ++j) q2[j] = __fmul2_rn(q_old[j], ff);
        const float2 ncmL2 = f2(-cm * kLog2e, -cm * kLog2e);
        const volatile float* vr = recs;  // fresh loads: keeps the first loop's rows dead
#pragma unroll
        for (int p = 0; p < kCW / 2; ++p) {
          const float2 x2 = __ffma2_rn(f2(acc[2 * p], acc[2 * p + 1]), L2, ncmL2);
          const float2 e2 = f2(ex2f(x2.x), ex2f(x2.y));
          s2 = __fadd2_rn(s2, e2);
#pragma unroll
          for (int j = 0; j < R; ++j)
            q2[j] = __ffma2_rn(e2, f2(vr[p * 2 * R + 2 * j], vr[p * 2 * R + 2 * j + 1]), q2[j]);
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
    g.p_sum[o] = s2.x + s2.y;
#pragma unroll
    for (int j = 0; j < R; ++j) g.p_q[o * g.rank_total + g.rank_off + j] = q2[j].x + q2[j].y;
  }
};

// Pass 2: the thread owns vocab row v; columns are positions; the records
// of a position pair are tok[] fields interleaved (2(R+4) floats).  This
// pass accumulates the p part of dl = p - onehot; lce_onehot adds the
// onehot part.
template <int R, bool kAug_ = (R >= LCE_AUG_MIN_RANK), bool kChunk = false>
struct EpiGrad {
  static constexpr bool kAug = kAug_;  // rank term in the accumulator
  // rank chunks read their own records {sU[0..16), -M log2 e, 1/S}
  // (crec_idx), the others the position records tok[] (tidx)
  static constexpr int kRec = kChunk ? R + 2 : R + 4;
  // 2 stages beside 10 or 11 resident K-blocks
  static constexpr int kRing = !kAug ? kRingBytes : 32768;
  // rank 16 (and rank chunks) stage one record buffer: 2 x 20 KB do not fit
  // beside 10 resident K-blocks; the loader then waits for the previous
  // tile's release
  static constexpr int kRecBufs = (kAug && R >= 16) ? 1 : 2;
  static constexpr int kWarps = R <= 8 ? 16 : 8;
  static constexpr int kCW = (R >= 16 || kWarps == 16) ? 8 : 16;
  int v;
  bool valid;
  float2 bv2[R];  // (B[j][v], B[j][v])
  float2 g2[R];   // dB[v][j] over even / odd positions

  __device__ static const float* global_recs(const GemmArgs& g, int b) {
    return g.tok + (long long)b * kBN * kRec;
  }
  __device__ static int limit(const GemmArgs& g) { return g.T; }

  __device__ void begin(const GemmArgs& g, int abs_row) {
    v = abs_row;
    valid = v < g.V;
    const long long vv = valid ? v : 0;
#pragma unroll
    for (int j = 0; j < R; ++j) {
      if constexpr (!kAug) {
        const float b = g.Bt[bidx(vv, j, R)];
        bv2[j] = f2(b, b);
      }
      g2[j] = f2(0.f, 0.f);
    }
  }

  // p = e^(z - M) / S = 2^(z*log2(e) - M*log2(e)) * (1/S); dB[v][:] += sU * p.
  template <bool kTail>
  __device__ __forceinline__ void chunk(const GemmArgs& g, int t0, float (&acc)[kCW],
                                        const float* recs) {
    if (kTail && t0 >= g.T) return;  // fully padded chunk (zero records) adds nothing
    const float2 L2 = f2(kLog2e, kLog2e);
#pragma unroll
    for (int p = 0; p < kCW / 2; ++p) {
      const float* rp = recs + p * 2 * kRec;
      float su[2 * R];
      ld_vec<2 * R>(rp, su);
      const float4 mi = *reinterpret_cast<const float4*>(rp + 2 * R);  // -ML pair, 1/S pair
      float2 z2 = f2(acc[2 * p], acc[2 * p + 1]);
      if constexpr (!kAug) {
#pragma unroll
        for (int j = 0; j < R; ++j) z2 = __ffma2_rn(bv2[j], f2(su[2 * j], su[2 * j + 1]), z2);
      }
      const float2 x2 = __ffma2_rn(z2, L2, f2(mi.x, mi.y));
      const float2 p2 = __fmul2_rn(f2(ex2f(x2.x), ex2f(x2.y)), f2(mi.z, mi.w));
#pragma unroll
      for (int j = 0; j < R; ++j) g2[j] = __ffma2_rn(f2(su[2 * j], su[2 * j + 1]), p2, g2[j]);
    }
  }

  __device__ void flush(const GemmArgs& g, int slot) {
    if (!valid) return;
    const int rt = g.rank_total;
    float* o = g.gBp + (long long)slot * g.Vpad * rt;
#pragma unroll
    for (int j = 0; j < R; ++j) o[bidx(v, g.rank_off + j, rt)] = g2[j].x + g2[j].y;
  }
};

// Chunk dispatch: the masked variant only for tiles that reach past the
// last column.
template <class Epi>
__device__ __forceinline__ void run_chunk(Epi& epi, const GemmArgs& g, bool tail, int col,
                                          float (&acc)[Epi::kCW], const float* recs) {
  if (tail) epi.template chunk<true>(g, col, acc, recs);
  else epi.template chunk<false>(g, col, acc, recs);
}

// ------------------------------------------------------------- mainloop
// One CTA (kPair 1) or a CTA pair launched as a 2-CTA cluster (kPair 2)
// owns a run of consecutive tiles.  A tile is (kBM * kPair) resident rows x
// kBN streamed rows; in a pair each CTA holds 128 resident rows and loads
// kBN/2 of the streamed rows, and the leader CTA (rank 0) issues
// tcgen05.mma.cta_group::2 over both CTAs' shared memory, so every W / h
// byte a CTA streams serves 256 resident rows.  Barrier ownership in a
// pair: `full`, `a_full`, `acc_empty` and `drain` live in the leader
// (both CTAs' copies signal them); `empty`, `a_empty`, `acc_full` live in
// both CTAs (the leader's commit reaches both).
// kStage: stage the column records of each tile in shared memory (double
// buffered, prefetched one tile ahead); otherwise read them from global.
template <class Epi, bool kStage, int kPair>
__global__ void __launch_bounds__(block_threads(Epi::kWarps), 1)
    lce_gemm_kernel(const __grid_constant__ CUtensorMap map_res,
                    const __grid_constant__ CUtensorMap map_str,
                    const __grid_constant__ CUtensorMap map_res_aug,
                    const __grid_constant__ CUtensorMap map_str_aug, const GemmArgs g) {
  constexpr int kEpiWarps = Epi::kWarps;
  constexpr int kEpiThreads = epi_threads(kEpiWarps);
  constexpr int kColParts = col_parts(kEpiWarps);
  constexpr int kRecWarp = 2 + kEpiWarps;
  constexpr int kRecF = kStage ? Epi::kRec * Epi::kRecBufs : 0;
  constexpr int kRB = Epi::kRecBufs;
  constexpr int kRingB = ring_bytes<Epi, kStage, kPair>();
  constexpr int kStBytes = stage_bytes(kPair);
  constexpr int kSt = kRingB / kStBytes;
  static_assert(kSt >= 2 && kSt <= kMaxStages, "ring stages");
  constexpr int kStRows = str_rows(kPair);
  constexpr int kResRows = kBM * kPair;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment by index arithmetic on the shared array, so that
  // pointers derived from it stay in the shared address space.  The array is
  // declared aligned and the layout reserves no slack: a base that arrived
  // misaligned by more than the launch's spare bytes is reported, not used
  // (both CTAs of a pair see the same base and return together).
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  {
    uint32_t dyn_bytes;
    asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn_bytes));
    if (pad + (uint32_t)SmemLayout::bytes(g.kblocks, kRecF, kRingB) > dyn_bytes) {
      if (threadIdx.x == 0) atomicCAS(g.err, 0, kErrSmemAlign);
      return;
    }
  }
  uint8_t* smem = smem_raw + pad;
  uint8_t* sA = smem + SmemLayout::a_off();
  uint8_t* sB = smem + SmemLayout::b_off(g.kblocks);
  float* srec = reinterpret_cast<float*>(smem + SmemLayout::rec_off(g.kblocks, kRingB));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SmemLayout::bar_off(g.kblocks, kRecF, kRingB));
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = kPair == 2 ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const long long total = (long long)g.n_a * g.n_b;
  const int G = gridDim.x / kPair;              // tile-range owners (CTAs or pairs)
  const int unit = blockIdx.x / kPair;
  const long long x_begin = tile_start(unit, total, G);
  const long long x_end = tile_start(unit + 1, total, G);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kSt; ++i) {
      mbar_init(&bars[kBarFull + i], 1);
      mbar_init(&bars[kBarEmpty + i], 1);
    }
    mbar_init(&bars[kBarAFull], 1);
    mbar_init(&bars[kBarAEmpty], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[kBarAccFull + i], 1);
      mbar_init(&bars[kBarAccEmpty + i], kPair * kEpiThreads / 32);
    }
    mbar_init(&bars[kBarDrain], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[kBarRecFull + i], 1);
      mbar_init(&bars[kBarRecEmpty + i], kEpiThreads / 32);
    }
    fence_mbar_init();
    prefetch_tmap(&map_res);
    prefetch_tmap(&map_str);
    if (g.kblocks > g.kmain) {
      prefetch_tmap(&map_res_aug);
      prefetch_tmap(&map_str_aug);
    }
  }
  if (warp == 1) {
    if constexpr (kPair == 2) {
      tmem_alloc_pair(tmem_slot, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (kPair == 2) cluster_sync();  // peer barriers initialised before any signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int cur_a = -1;
      uint32_t a_uses = 0;
      int issued_parity[kMaxStages];
      for (int i = 0; i < kMaxStages; ++i) issued_parity[i] = -1;
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
          if (leader)
            mbar_expect_tx(&bars[kBarAFull], (uint32_t)(kPair * g.kblocks * kAKBytes));
          const int row0 = (g.a0 + a) * kResRows + (int)rank * kBM;
          for (int kb = 0; kb < g.kblocks; ++kb) {
            // K-blocks past kmain come from the rank-augmentation map, at x = 0
            const CUtensorMap* m = kb < g.kmain ? &map_res : &map_res_aug;
            const int kx = (kb < g.kmain ? kb : kb - g.kmain) * kBK;
            if constexpr (kPair == 2)
              tma_load_2d_pair(sA + kb * kAKBytes, m,
                               mapa_shared(smem_u32(&bars[kBarAFull]), 0), kx, row0);
            else
              tma_load_2d(sA + kb * kAKBytes, m, &bars[kBarAFull], kx, row0);
          }
          cur_a = a;
          ++a_uses;
        }
        const int srow0 = b * kBN + (int)rank * kStRows;
        for (int kb = 0; kb < g.kstr; ++kb) {
          if (!mbar_wait(&bars[kBarEmpty + stage], phase ^ 1, g.err, kErrWaitProducer)) {
            ok = false;
            break;
          }
          if (leader) mbar_expect_tx(&bars[kBarFull + stage], (uint32_t)(kPair * kStBytes));
          const CUtensorMap* m = kb < g.kmain ? &map_str : &map_str_aug;
          const int kx = (kb < g.kmain ? kb : kb - g.kmain) * kBK;
          if constexpr (kPair == 2)
            tma_load_2d_pair(sB + stage * kStBytes, m,
                             mapa_shared(smem_u32(&bars[kBarFull + stage]), 0), kx, srow0);
          else
            tma_load_2d(sB + stage * kStBytes, m, &bars[kBarFull + stage], kx, srow0);
          issued_parity[stage] = (int)phase;
          if (++stage == kSt) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Never leave with bulk copies still landing: the leader's full
      // barriers count both CTAs' bytes, so the leader drains them (the
      // closing cluster barrier keeps the peer resident meanwhile).
      if (leader) {
        for (int i = 0; i < kSt; ++i)
          if (issued_parity[i] >= 0)
            mbar_drain_wait(&bars[kBarFull + i], (uint32_t)issued_parity[i], g.err);
        if (a_uses > 0) mbar_drain_wait(&bars[kBarAFull], (a_uses - 1) & 1, g.err);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer (leader CTA)
    if (lane == 0 && leader) {
      constexpr uint32_t kIdesc = idesc_f16_f32(kResRows, kBN);
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
        auto mma = [&](uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
          if constexpr (kPair == 2) umma_f16_pair(d_tmem, adesc, bdesc, kIdesc, accumulate);
          else umma_f16(d_tmem, adesc, bdesc, kIdesc, accumulate);
        };
        auto release = [&](int st_) {
          if constexpr (kPair == 2) umma_commit_pair(&bars[kBarEmpty + st_], 0x3);
          else umma_commit(&bars[kBarEmpty + st_]);
        };
        for (int kb = 0; kb < g.kmain; ++kb) {
          if (!mbar_wait(&bars[kBarFull + stage], phase, g.err, kErrWaitMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = sw128_kmajor_desc(smem_u32(sA + kb * kAKBytes));
          const uint64_t bdesc = sw128_kmajor_desc(smem_u32(sB + stage * kStBytes));
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            mma(adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), (kb | k) != 0 ? 1u : 0u);
          release(stage);
          if (++stage == kSt) {
            stage = 0;
            phase ^= 1;
          }
        }
        // rank augmentation: all of this tile's streamed augmentation stages
        // (one or two; the ring has at least two) in the ring at once, then
        // the scheduled K-steps, then their release
        const int n_str_aug = g.kstr - g.kmain;
        int aug_stage[2] = {0, 0};
        for (int i = 0; i < n_str_aug && ok; ++i) {
          if (!mbar_wait(&bars[kBarFull + stage], phase, g.err, kErrWaitMma)) {
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
                sw128_kmajor_desc(smem_u32(sB + aug_stage[ib >> 2] * kStBytes)) +
                (uint64_t)(2 * (ib & 3));
            mma(adesc, bdesc, 1u);
          }
          for (int i = 0; i < n_str_aug; ++i) release(aug_stage[i]);
        }
        if (!ok) break;
        const bool last_of_a = x + 1 == x_end || (int)((x + 1) / g.n_b) != a;
        if constexpr (kPair == 2) {
          umma_commit_pair(&bars[kBarAccFull + buf], 0x3);
          if (last_of_a) umma_commit_pair(&bars[kBarAEmpty], 0x3);
        } else {
          umma_commit(&bars[kBarAccFull + buf]);
          if (last_of_a) umma_commit(&bars[kBarAEmpty]);
        }
      }
      // All MMAs issued by this thread complete before TMEM is released.
      if constexpr (kPair == 2) umma_commit_pair(&bars[kBarDrain], 0x1);
      else umma_commit(&bars[kBarDrain]);
      mbar_drain_wait(&bars[kBarDrain], 0, g.err);
    }
  } else if (warp < kRecWarp) {
    // ------------------------------------------------ epilogue (warps 2..kRecWarp-1)
    // Warp w reads TMEM lanes 32*(w%4)..+31; the four warps of a lane
    // quarter take 64-column slices of each tile, so every resident row has
    // kColParts partial states, flushed to slots kColParts*segment + part.
    const int e = warp - 2;
    const int quarter = warp & 3;
    const int half = e >> 2;  // column slice index
    const int row = quarter * 32 + lane;
    const uint32_t lane_addr = tmem_base + ((uint32_t)(quarter * 32) << 16);
    constexpr int CW = Epi::kCW;
    constexpr int NCH = (kBN / kColParts) / CW;
    Epi epi;
    int cur_a = -1;
    long long li = 0;
    bool failed = false;
    for (long long x = x_begin; x < x_end; ++x, ++li) {
      const int a = (int)(x / g.n_b);
      const int b = (int)(x % g.n_b);
      if (a != cur_a) {
        if (cur_a >= 0 && !failed)
          epi.flush(g, kColParts * (unit - tile_owner((long long)cur_a * g.n_b, total, G)) + half);
        epi.begin(g, (g.a0 + a) * kResRows + (int)rank * kBM + row);
        cur_a = a;
      }
      const int rbuf = (int)(li % kRB);
      const uint32_t ruse = (uint32_t)(li / kRB);
      const float* recs = kStage ? srec + rbuf * (kBN * Epi::kRec) : Epi::global_recs(g, b);
      if (failed) continue;
      const int buf = (int)(li & 1);
      const uint32_t use = (uint32_t)(li >> 1);
      if (!mbar_wait(&bars[kBarAccFull + buf], use & 1, g.err, kErrWaitEpilogue) ||
          (kStage && !mbar_wait(&bars[kBarRecFull + rbuf], ruse & 1, g.err, kErrWaitEpilogue))) {
        failed = true;
        continue;
      }
      tc_fence_after();
      {
        // Two register buffers: the TMEM load of chunk c+1 is in flight
        // while chunk c is processed.
        const int col0 = half * (kBN / kColParts);
        const uint32_t base = lane_addr + (uint32_t)(buf * kBN + col0);
        const float* rb = recs + col0 * Epi::kRec;
        const int gcol = b * kBN + col0;
        // Only a tile that reaches past the last vocab id / position needs
        // the masked chunk variant.
        const bool tail = gcol + kBN / kColParts > Epi::limit(g);
        float ca[CW], cb[CW];
        // Records read from global memory (not staged): the lanes prefetch
        // into L1 the lines of chunk c+2's records while chunk c runs.
        constexpr int kRecLine = 32;  // floats per 128-byte line
        constexpr int kChunkLines = (CW * Epi::kRec + kRecLine - 1) / kRecLine;
        auto prefetch_recs = [&](int c) {
          if constexpr (!kStage) {
            if (c < NCH && lane < kChunkLines)
              asm volatile("prefetch.L1 [%0];" ::"l"(rb + c * CW * Epi::kRec + lane * kRecLine));
          }
        };
        prefetch_recs(0);
        prefetch_recs(1);
        tmem_ld<CW>(base, ca);
        tmem_ld_wait<CW>(ca);
#pragma unroll 1
        for (int c = 0; c < NCH; c += 2) {
          prefetch_recs(c + 2);
          prefetch_recs(c + 3);
          tmem_ld<CW>(base + (uint32_t)((c + 1) * CW), cb);
          run_chunk<Epi>(epi, g, tail, gcol + c * CW, ca, rb + c * CW * Epi::kRec);
          tmem_ld_wait<CW>(cb);
          if (c + 2 < NCH) tmem_ld<CW>(base + (uint32_t)((c + 2) * CW), ca);
          run_chunk<Epi>(epi, g, tail, gcol + (c + 1) * CW, cb,
                                 rb + (c + 1) * CW * Epi::kRec);
          if (c + 2 < NCH) tmem_ld_wait<CW>(ca);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (kStage) mbar_arrive(&bars[kBarRecEmpty + rbuf]);
        if constexpr (kPair == 2)
          mbar_arrive_cluster(mapa_shared(smem_u32(&bars[kBarAccEmpty + buf]), 0));
        else
          mbar_arrive(&bars[kBarAccEmpty + buf]);
      }
    }
    if (cur_a >= 0 && !failed)
      epi.flush(g, kColParts * (unit - tile_owner((long long)cur_a * g.n_b, total, G)) + half);
  } else if (warp == kRecWarp) {
    // ------------------------------------------------ record loader (both CTAs)
    // The records of tile li (256 columns, one contiguous block in global)
    // go to buffer li % kRB once the epilogue has released tile li - kRB.
    if (kStage && lane == 0) {
      constexpr uint32_t kBytes = (uint32_t)(kBN * Epi::kRec * 4);
      long long li = 0;
      int issued = 0;
      for (long long x = x_begin; x < x_end; ++x, ++li) {
        const int b = (int)(x % g.n_b);
        const int buf = (int)(li % kRB);
        const uint32_t use = (uint32_t)(li / kRB);
        if (use > 0 &&
            !mbar_wait(&bars[kBarRecEmpty + buf], (use - 1) & 1, g.err, kErrWaitProducer))
          break;
        mbar_expect_tx(&bars[kBarRecFull + buf], kBytes);
        bulk_load(srec + buf * (kBN * Epi::kRec), Epi::global_recs(g, b), kBytes,
                  &bars[kBarRecFull + buf]);
        ++issued;
      }
      // drain: the last load into each buffer has landed
      for (int k = issued - kRB < 0 ? 0 : issued - kRB; k < issued; ++k)
        mbar_drain_wait(&bars[kBarRecFull + (k % kRB)], (uint32_t)((k / kRB) & 1), g.err);
    }
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (kPair == 2) cluster_sync();  // peer done with the leader's barriers / MMAs done
  if (warp == 1) {
    tc_fence_after();
    if constexpr (kPair == 2) tmem_dealloc_pair(tmem_base, kTmemCols);
    else tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ------------------------------------------------------------- small kernels
// h (bf16 / f16 / f32) -> f16 rows; s*U = s*(h16 . A); per-position record
// {sU[0..R), M, 1/S, target, 0} (M, 1/S filled by lce_combine).  One warp
// per position (grid-stride), lane l converting elements 2l, 2l+1 of each
// 64-element slice, so global accesses are coalesced and the A rows read
// from shared memory are contiguous across lanes.  Positions in [T, Tpad)
// get an all-zero record with target -1 so pass 2 can read whole tiles.
template <int R>
__global__ void lce_prep(const void* __restrict__ H, int dtype, int t_lo, int t_hi, int T, int d,
                         const float* __restrict__ A, float scale,
                         const int32_t* __restrict__ targets, int V,
                         __half* __restrict__ h16, float* __restrict__ tok, int* err,
                         __half* __restrict__ haug, int aug_layout, int aug_width,
                         float* __restrict__ tokc, long long tokc_stride) {
  extern __shared__ __align__(16) float sA[];  // [d][R]
  for (int k = threadIdx.x; k < d * R; k += blockDim.x) sA[k] = A[k];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  for (int w = t_lo + ((blockIdx.x * blockDim.x + threadIdx.x) >> 5); w < t_hi; w += nw) {
    if (w >= T) {  // padding position: all fields zero, target -1
      for (int f = lane; f < tok_stride(R); f += 32)
        tok[tidx(w, f, R)] = f == R + 2 ? __int_as_float(-1) : 0.f;
      if (haug)
        for (int cc = 2 * lane; cc < aug_width; cc += 64)
          *reinterpret_cast<__half2*>(haug + (long long)w * aug_width + cc) =
              __floats2half2_rn(0.f, 0.f);
      if (tokc)  // chunk records of a padding position: all zero
        for (int c = 0; c < R / 16; ++c)
          for (int f = lane; f < kChunkRec; f += 32) tokc[c * tokc_stride + crec_idx(w, f)] = 0.f;
      continue;
    }
    float u[R];
#pragma unroll
    for (int j = 0; j < R; ++j) u[j] = 0.f;
    for (int i = 2 * lane; i < d; i += 64) {
      const long long o = (long long)w * d + i;
      float2 x;
      if (dtype == 0) x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(
                          reinterpret_cast<const __nv_bfloat16*>(H) + o));
      else if (dtype == 1) x = __half22float2(*reinterpret_cast<const __half2*>(
                               reinterpret_cast<const __half*>(H) + o));
      else x = *reinterpret_cast<const float2*>(reinterpret_cast<const float*>(H) + o);
      const __half2 hv = __floats2half2_rn(x.x, x.y);
      *reinterpret_cast<__half2*>(h16 + o) = hv;
      const float2 hf = __half22float2(hv);
      float a0[R], a1[R];
      ld_vec<R>(sA + i * R, a0);
      ld_vec<R>(sA + (i + 1) * R, a1);
#pragma unroll
      for (int j = 0; j < R; ++j) u[j] = fmaf(hf.y, a1[j], fmaf(hf.x, a0[j], u[j]));
    }
#pragma unroll
    for (int j = 0; j < R; ++j) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) u[j] += __shfl_xor_sync(0xffffffffu, u[j], off);
    }
    if (haug) {
      // columns of the augmentation row: layout 1 [sU_hi | sU_hi | sU_lo | 0]
      // (ranks <= 21, one 64-wide block), layout 2 [sU_hi | sU_lo] (ranks 32,
      // 64); lane l writes columns 2l, 2l+1 of each 64-column block
      for (int cb = 0; cb < aug_width; cb += 64) {
        __half hv2[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const int c = cb + 2 * lane + k, part = c / R, jc = c - part * R;
          float su = 0.f;
#pragma unroll
          for (int j = 0; j < R; ++j) su = (j == jc) ? scale * u[j] : su;
          const __half hi = __float2half_rn(su);
          const __half lo = __float2half_rn(su - __half2float(hi));
          const bool is_lo = aug_layout == 1 ? part == 2 : part == 1;
          const bool used = aug_layout == 1 ? part < 3 : part < 2;
          hv2[k] = !used ? __float2half_rn(0.f) : is_lo ? lo : hi;
        }
        *reinterpret_cast<__half2*>(haug + (long long)w * aug_width + cb + 2 * lane) =
            __halves2half2(hv2[0], hv2[1]);
      }
    }
    if (tokc) {
      // rank chunks of 16: sU of the chunk; M, 1/S come from lce_combine
      for (int c = 0; c < R / 16; ++c)
        for (int f = lane; f < kChunkRec; f += 32) {
          float val = 0.f;
#pragma unroll
          for (int j = 0; j < R; ++j) val = (f < 16 && j == 16 * c + f) ? scale * u[j] : val;
          tokc[c * tokc_stride + crec_idx(w, f)] = val;
        }
    }
    if (lane == 0) {
      int tg = targets[w];
      if (tg < 0 || tg >= V) {
        atomicCAS(err, 0, kErrTarget);
        tg = 0;
      }
#pragma unroll
      for (int j = 0; j < R; ++j) tok[tidx(w, j, R)] = scale * u[j];
      tok[tidx(w, R, R)] = 0.f;
      tok[tidx(w, R + 1, R)] = 0.f;
      tok[tidx(w, R + 2, R)] = __int_as_float(tg);
      tok[tidx(w, R + 3, R)] = 0.f;
    }
  }
}

// lce_prep for ranks 16..64: the same outputs, computed with lanes over
// ranks instead of over d (the d-strided reads of A rows conflict on
// every shared-memory bank once a row is 64 B or more, and the warp-wide
// reduction of R sums costs 5R shuffles).  A warp takes kPrepQ * 64/R
// positions at a time: it converts their h rows (f16 out, the f16 values
// kept as f32 in shared memory), then lane (g, jp) accumulates
// U[g*kPrepQ + q][2jp, 2jp+1] for its kPrepQ positions, reading A[i][2jp..]
// (consecutive across lanes) and h[.][i..i+3] (one row per lane group).
constexpr int kPrepQ = 4;
constexpr int kPrepMaxWarps = 8;
__host__ __device__ constexpr int prep_wide_rows(int R) { return kPrepQ * 64 / R; }
// Warps per block: as many as fit beside A in shared memory, up to 8.
__host__ __device__ constexpr int prep_wide_warps(int R, int d) {
  return (kMaxDynSmem - d * R * 4) / (prep_wide_rows(R) * (d + 4) * 4) < kPrepMaxWarps
             ? (kMaxDynSmem - d * R * 4) / (prep_wide_rows(R) * (d + 4) * 4)
             : kPrepMaxWarps;
}
__host__ __device__ constexpr int prep_wide_smem(int R, int d) {
  return d * R * 4 + prep_wide_warps(R, d) * prep_wide_rows(R) * (d + 4) * 4;
}
template <int R>
__global__ void __launch_bounds__(32 * kPrepMaxWarps)
    lce_prep_wide(const void* __restrict__ H, int dtype, int t_lo, int t_hi, int T, int d,
                  const float* __restrict__ A, float scale, const int32_t* __restrict__ targets,
                  int V, __half* __restrict__ h16, float* __restrict__ tok, int* err,
                  __half* __restrict__ haug, int aug_layout, int aug_width,
                  float* __restrict__ tokc, long long tokc_stride) {
  static_assert(R >= 16 && R <= 64, "wide prep: ranks 16..64");
  constexpr int NP = prep_wide_rows(R);  // positions per warp batch
  constexpr int kLanesPer = R / 2;       // lanes per position group
  extern __shared__ __align__(16) float smem_f[];
  float* sA = smem_f;  // [d][R]
  const int ldh = d + 4;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* sh = smem_f + d * R + warp * NP * ldh;  // [NP][d + 4]
  for (int k = threadIdx.x; k < d * R; k += blockDim.x) sA[k] = A[k];
  __syncthreads();
  const int g = lane / kLanesPer, jp = lane % kLanesPer;
  const int warps_blk = blockDim.x >> 5;
  const int nwarps = gridDim.x * warps_blk;
  for (int w0 = t_lo + (blockIdx.x * warps_blk + warp) * NP; w0 < t_hi; w0 += nwarps * NP) {
    // convert this batch's rows (positions >= T read as zero rows); the NP
    // rows' loads of one column pair are issued together
    for (int i = 2 * lane; i < d; i += 64) {
      float2 x[NP];
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        const int w = w0 + p;
        x[p] = make_float2(0.f, 0.f);
        if (w < T && w < t_hi) {
          const long long o = (long long)w * d + i;
          if (dtype == 0) x[p] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(
                              reinterpret_cast<const __nv_bfloat16*>(H) + o));
          else if (dtype == 1) x[p] = __half22float2(*reinterpret_cast<const __half2*>(
                                   reinterpret_cast<const __half*>(H) + o));
          else x[p] = *reinterpret_cast<const float2*>(reinterpret_cast<const float*>(H) + o);
        }
      }
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        const int w = w0 + p;
        const __half2 hv = __floats2half2_rn(x[p].x, x[p].y);
        if (w < T && w < t_hi)
          *reinterpret_cast<__half2*>(h16 + (long long)w * d + i) = hv;
        *reinterpret_cast<float2*>(sh + p * ldh + i) = __half22float2(hv);
      }
    }
    __syncwarp();
    float2 acc[kPrepQ];
#pragma unroll
    for (int q = 0; q < kPrepQ; ++q) acc[q] = make_float2(0.f, 0.f);
    const float* hrow = sh + g * kPrepQ * ldh;
#pragma unroll 2
    for (int i = 0; i < d; i += 4) {
      float2 a[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) a[k] = *reinterpret_cast<const float2*>(sA + (i + k) * R + 2 * jp);
#pragma unroll
      for (int q = 0; q < kPrepQ; ++q) {
        const float4 hv = *reinterpret_cast<const float4*>(hrow + q * ldh + i);
        acc[q].x = fmaf(hv.x, a[0].x, acc[q].x);
        acc[q].y = fmaf(hv.x, a[0].y, acc[q].y);
        acc[q].x = fmaf(hv.y, a[1].x, acc[q].x);
        acc[q].y = fmaf(hv.y, a[1].y, acc[q].y);
        acc[q].x = fmaf(hv.z, a[2].x, acc[q].x);
        acc[q].y = fmaf(hv.z, a[2].y, acc[q].y);
        acc[q].x = fmaf(hv.w, a[3].x, acc[q].x);
        acc[q].y = fmaf(hv.w, a[3].y, acc[q].y);
      }
    }
    __syncwarp();  // the batch's rows are read before the next batch overwrites them
#pragma unroll
    for (int q = 0; q < kPrepQ; ++q) {
      const int w = w0 + g * kPrepQ + q;
      if (w >= t_hi) continue;
      const bool pad = w >= T;
      const int j0 = 2 * jp;
      const float su0 = pad ? 0.f : scale * acc[q].x, su1 = pad ? 0.f : scale * acc[q].y;
      tok[tidx(w, j0, R)] = su0;
      tok[tidx(w, j0 + 1, R)] = su1;
      if (jp == 0) {
        int tg = -1;
        if (!pad) {
          tg = targets[w];
          if (tg < 0 || tg >= V) {
            atomicCAS(err, 0, kErrTarget);
            tg = 0;
          }
        }
        tok[tidx(w, R, R)] = 0.f;
        tok[tidx(w, R + 1, R)] = 0.f;
        tok[tidx(w, R + 2, R)] = __int_as_float(tg);
        tok[tidx(w, R + 3, R)] = 0.f;
      }
      if (haug) {
        const __half h0 = __float2half_rn(su0), h1 = __float2half_rn(su1);
        const __half2 hi = __halves2half2(h0, h1);
        const __half2 lo = __floats2half2_rn(su0 - __half2float(h0), su1 - __half2float(h1));
        __half* row = haug + (long long)w * aug_width;
        if (aug_layout == 1) {  // [sU_hi | sU_hi | sU_lo | 0]
          *reinterpret_cast<__half2*>(row + j0) = hi;
          *reinterpret_cast<__half2*>(row + R + j0) = hi;
          *reinterpret_cast<__half2*>(row + 2 * R + j0) = lo;
          for (int c = 3 * R + j0; c < aug_width; c += R)
            *reinterpret_cast<__half2*>(row + c) = __floats2half2_rn(0.f, 0.f);
        } else {  // [sU_hi | sU_lo | 0]
          *reinterpret_cast<__half2*>(row + j0) = hi;
          *reinterpret_cast<__half2*>(row + R + j0) = lo;
          for (int c = 2 * R + j0; c < aug_width; c += R)
            *reinterpret_cast<__half2*>(row + c) = __floats2half2_rn(0.f, 0.f);
        }
      }
      if (tokc) {  // rank chunks of 16: sU of the chunk; M, 1/S come from lce_combine
        const int c = j0 / 16, f = j0 % 16;
        tokc[c * tokc_stride + crec_idx(w, f)] = su0;
        tokc[c * tokc_stride + crec_idx(w, f + 1)] = su1;
        if (jp < R / 16) {
          tokc[jp * tokc_stride + crec_idx(w, 16)] = 0.f;
          tokc[jp * tokc_stride + crec_idx(w, 17)] = 0.f;
        }
      }
    }
  }
}

// The vocabulary side of rank augmentation, rebuilt at the start of every
// step from the current B (rows >= V are zero like B): layout 1
// waug[v] = [B_hi | B_lo | B_hi | 0] (ranks <= 21, one 64-wide block),
// layout 2 waug[v] = [B_hi | B_lo] (ranks 32, 64).  One thread per 8
// columns of a row (16-byte stores).  With Bc, also B's rank chunks of 16,
// each in the pair-interleaved layout of rank 16 (pass 1's column records).
template <int R>
__global__ void lce_aug_b(const float* __restrict__ Bt, long long Vpad, __half* __restrict__ waug,
                          int aug_layout, int aug_width, float* __restrict__ Bc,
                          long long Bc_stride) {
  static_assert(3 * R <= 64 || R % 16 == 0, "layout 1 fits one block; larger ranks use layout 2");
  const int groups = aug_width / 8;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < Vpad * groups;
       i += (long long)gridDim.x * blockDim.x) {
    const long long v = i / groups;
    const int c0 = (int)(i - v * groups) * 8;
    __align__(16) __half o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int c = c0 + e, part = c / R, j = c - part * R;
      const bool used = aug_layout == 1 ? part < 3 : part < 2;
      const bool is_lo = part == 1;  // [hi | lo | hi] and [hi | lo] alike
      const float b = used ? Bt[bidx(v, j, R)] : 0.f;
      const __half hi = __float2half_rn(b);
      const __half lo = __float2half_rn(b - __half2float(hi));
      o[e] = is_lo ? lo : hi;  // unused columns: b = 0, hi = 0
    }
    *reinterpret_cast<uint4*>(waug + v * aug_width + c0) = *reinterpret_cast<const uint4*>(o);
  }
  if (Bc) {  // rank chunks of 16 in their own pair-interleaved arrays
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < Vpad * R;
         i += (long long)gridDim.x * blockDim.x) {
      const long long v = i / R;
      const int j = (int)(i - v * R);
      Bc[(j / 16) * Bc_stride + bidx(v, j % 16, 16)] = Bt[bidx(v, j, R)];
    }
  }
}

// Merge the pass-1 partials of each position (two slots per CTA segment,
// one per column half): M = max, S = sum e^(z-M), Q = sum e^(z-M) B[:,v];
// then p_t, loss_t = -log(p_t + 1e-12) and dU_t = s * (Q/S - B[:,target])
// (the reference's d_mid, src/train.c:161-168).  The record of t gets
// M*log2(e) and 1/S for pass 2.
template <int R>
__global__ void lce_combine(int T, int cparts, int res_rows, int n_b1, int units1, int chunks,
                            long long Tcap,
                            const float* __restrict__ p_max,
                            const float* __restrict__ p_sum, const float* __restrict__ p_q,
                            const float* __restrict__ z_tgt, const float* __restrict__ Bt,
                            float scale, float* __restrict__ tok, float* __restrict__ dU,
                            float* __restrict__ loss_tok, float* __restrict__ tokc,
                            long long tokc_stride) {
  // one warp per position; lane k merges slots k, k+32, ... (fixed order)
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  // Pass 1 ran as `chunks` launches over even splits of the n_a position
  // blocks (chunk c: blocks [start(c), start(c+1))), each with its own tile
  // ranges over min(units1, tiles of the chunk) owners.
  const int n_a = (T + res_rows - 1) / res_rows;
  const int ab = t / res_rows;
  const int c = tile_owner(ab, n_a, chunks);
  const int a_lo = (int)tile_start(c, n_a, chunks), a_hi = (int)tile_start(c + 1, n_a, chunks);
  const int a = ab - a_lo;
  const long long total = (long long)(a_hi - a_lo) * n_b1;
  const int G1 = (int)(total < units1 ? total : units1);
  const int s0 = tile_owner((long long)a * n_b1, total, G1);
  const int s1 = tile_owner((long long)a * n_b1 + n_b1 - 1, total, G1);
  const int nslot = cparts * (s1 - s0 + 1);
  float M = -INFINITY;
  for (int k = lane; k < nslot; k += 32) M = fmaxf(M, p_max[(long long)k * Tcap + t]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  float S = 0.f, Q[R];
#pragma unroll
  for (int j = 0; j < R; ++j) Q[j] = 0.f;
  for (int k = lane; k < nslot; k += 32) {
    const long long o = (long long)k * Tcap + t;
    const float pm = p_max[o];
    if (pm == -INFINITY) continue;  // a slice that saw no valid column
    const float f = expf(pm - M);
    S = fmaf(p_sum[o], f, S);
#pragma unroll
    for (int j = 0; j < R; ++j) Q[j] = fmaf(p_q[o * R + j], f, Q[j]);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    S += __shfl_xor_sync(0xffffffffu, S, off);
#pragma unroll
    for (int j = 0; j < R; ++j) Q[j] += __shfl_xor_sync(0xffffffffu, Q[j], off);
  }
  if (lane != 0) return;
  const float inv = 1.0f / S;
  const int tg = __float_as_int(tok[tidx(t, R + 2, R)]);
  const float pt = expf(z_tgt[t] - M) * inv;
  loss_tok[t] = -logf(pt + 1e-12f);
  tok[tidx(t, R, R)] = -(M * kLog2e);
  tok[tidx(t, R + 1, R)] = inv;
  if (tokc)  // the rank chunks' records of position t (pass 2 of each chunk)
    for (int c = 0; c < R / 16; ++c) {
      tokc[c * tokc_stride + crec_idx(t, 16)] = -(M * kLog2e);
      tokc[c * tokc_stride + crec_idx(t, 17)] = inv;
    }
#pragma unroll
  for (int j = 0; j < R; ++j) dU[(long long)t * R + j] = scale * (Q[j] * inv - Bt[bidx(tg, j, R)]);
}

// lce_combine for ranks 16..64, lanes over ranks: every lane walks the few
// partial slots of its position (the max and the sum are the same in every
// lane), and lane l merges q and writes dU for ranks l, l + 32 (< R), so no
// warp reduction of R sums is needed and the dU row is written by all lanes.
template <int R>
__global__ void lce_combine_wide(int T, int cparts, int res_rows, int n_b1, int units1, int chunks,
                                 long long Tcap, const float* __restrict__ p_max,
                                 const float* __restrict__ p_sum, const float* __restrict__ p_q,
                                 const float* __restrict__ z_tgt, const float* __restrict__ Bt,
                                 float scale, float* __restrict__ tok, float* __restrict__ dU,
                                 float* __restrict__ loss_tok, float* __restrict__ tokc,
                                 long long tokc_stride) {
  static_assert(R >= 16 && R <= 64, "wide combine: ranks 16..64");
  constexpr int kPer = (R + 31) / 32;  // ranks per lane
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  const int n_a = (T + res_rows - 1) / res_rows;
  const int ab = t / res_rows;
  const int c = tile_owner(ab, n_a, chunks);
  const int a_lo = (int)tile_start(c, n_a, chunks), a_hi = (int)tile_start(c + 1, n_a, chunks);
  const int a = ab - a_lo;
  const long long total = (long long)(a_hi - a_lo) * n_b1;
  const int G1 = (int)(total < units1 ? total : units1);
  const int s0 = tile_owner((long long)a * n_b1, total, G1);
  const int s1 = tile_owner((long long)a * n_b1 + n_b1 - 1, total, G1);
  const int nslot = cparts * (s1 - s0 + 1);
  float M = -INFINITY;
  for (int k = 0; k < nslot; ++k) M = fmaxf(M, p_max[(long long)k * Tcap + t]);
  float S = 0.f, Q[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) Q[i] = 0.f;
  for (int k = 0; k < nslot; ++k) {
    const long long o = (long long)k * Tcap + t;
    const float pm = p_max[o];
    if (pm == -INFINITY) continue;  // a slice that saw no valid column
    const float f = expf(pm - M);
    S = fmaf(p_sum[o], f, S);
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int j = lane + 32 * i;
      if (j < R) Q[i] = fmaf(p_q[o * R + j], f, Q[i]);
    }
  }
  const float inv = 1.0f / S;
  const int tg = __float_as_int(tok[tidx(t, R + 2, R)]);
  if (lane == 0) {
    const float pt = expf(z_tgt[t] - M) * inv;
    loss_tok[t] = -logf(pt + 1e-12f);
    tok[tidx(t, R, R)] = -(M * kLog2e);
    tok[tidx(t, R + 1, R)] = inv;
    if (tokc)  // the rank chunks' records of position t (pass 2 of each chunk)
      for (int cc = 0; cc < R / 16; ++cc) {
        tokc[cc * tokc_stride + crec_idx(t, 16)] = -(M * kLog2e);
        tokc[cc * tokc_stride + crec_idx(t, 17)] = inv;
      }
  }
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int j = lane + 32 * i;
    if (j < R) dU[(long long)t * R + j] = scale * (Q[i] * inv - Bt[bidx(tg, j, R)]);
  }
}

// The onehot part of dl = p - onehot for dB: corr[v][j] = -(sum of
// s*U[t][j] over the positions t whose target is v).  Each term is rounded
// to a 64-bit fixed-point number (2^-30 resolution) and added with integer
// atomics: integer sums do not depend on the order of the additions, so the
// result is deterministic however the (Zipf-skewed) targets collide, and
// the one final rounding to f32 (in lce_finalize) is at least as accurate
// as a sequential f32 sum.  |s*U| must stay below 2^17 per position.
constexpr float kFixScale = 1073741824.0f;  // 2^30
constexpr double kFixInv = 1.0 / 1073741824.0;
template <int R>
__global__ void lce_onehot(int T, const float* __restrict__ tok,
                           unsigned long long* __restrict__ corr_fx, int* err) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const int lane = threadIdx.x & 31;
  const bool valid = t < T;
  const int tg = valid ? __float_as_int(tok[tidx(t, R + 2, R)]) : -1;
  long long q[R];
#pragma unroll
  for (int j = 0; j < R; ++j) {
    const float u = valid ? tok[tidx(t, j, R)] : 0.f;
    if (!(fabsf(u) < 131072.0f)) atomicCAS(err, 0, kErrRange);
    q[j] = __float2ll_rn(u * kFixScale);
  }
  // Positions of one warp that share a target are added up first (integer
  // sums, so the grouping does not change the result) and the lowest lane
  // of each group issues the atomics: Zipf-skewed targets collide often.
  long long sum[R];
#pragma unroll
  for (int j = 0; j < R; ++j) sum[j] = 0;
  for (int k = 0; k < 32; ++k) {
    const int tk = __shfl_sync(0xffffffffu, tg, k);
#pragma unroll
    for (int j = 0; j < R; ++j) {
      const long long qk = __shfl_sync(0xffffffffu, q[j], k);
      if (tk == tg) sum[j] += qk;
    }
  }
  const unsigned peers = __match_any_sync(0xffffffffu, tg);
  if (valid && lane == __ffs(peers) - 1) {
#pragma unroll
    for (int j = 0; j < R; ++j) atomicAdd(&corr_fx[bidx(tg, j, R)], (unsigned long long)sum[j]);
  }
}

// dA partials: gAp[c][i][j] = sum over the kDAChunk positions of chunk c
// of h16[t][i] * dU[t][j].  Grid (chunks, d / 64); a block of 32 x Y
// threads: thread (x, y) sums columns 2x, 2x+1 of its 64-column slice over
// every Y-th position of the chunk, then the Y partial sums are added in a
// fixed order.
constexpr int kDAChunk = 256;
__host__ __device__ constexpr int da_rows(int R) { return R <= 8 ? 16 : 4; }
template <int R>
__global__ void __launch_bounds__(32 * da_rows(R)) lce_dA_partial(int T, int d,
                                                                  const __half* __restrict__ h16,
                                                                  const float* __restrict__ dU,
                                                                  float* __restrict__ gAp,
                                                                  int rank_total, int rank_off) {
  constexpr int Y = da_rows(R);
  constexpr int NT = 32 * Y;
  __shared__ __align__(16) float sdU[kDAChunk * R];
  __shared__ float sred[Y][64 * R];
  const int c = blockIdx.x;
  const int t0 = c * kDAChunk;
  const int nt = min(kDAChunk, T - t0);
  const int tid = threadIdx.y * 32 + threadIdx.x;
  for (int k = tid; k < nt * R; k += NT)
    sdU[k] = dU[(long long)(t0 + k / R) * rank_total + rank_off + k % R];
  __syncthreads();
  const int i = blockIdx.y * 64 + 2 * threadIdx.x;
  // a0 / a1: columns i / i+1, ranks in pairs (j, j+1) per f32x2 fma, whose
  // lanes are the same fmas in the same position order as scalar ones
  static_assert(R % 4 == 0, "ranks in float4 groups");
  float2 a0[R / 2], a1[R / 2];
#pragma unroll
  for (int j = 0; j < R / 2; ++j) a0[j] = a1[j] = make_float2(0.f, 0.f);
  if (i < d) {
    const __half* hp = h16 + (long long)t0 * d + i;
#pragma unroll 4
    for (int tt = threadIdx.y; tt < nt; tt += Y) {
      const float2 hv = __half22float2(*reinterpret_cast<const __half2*>(hp + (long long)tt * d));
      const float2 hx = make_float2(hv.x, hv.x), hy = make_float2(hv.y, hv.y);
#pragma unroll
      for (int j = 0; j < R; j += 4) {
        const float4 u = *reinterpret_cast<const float4*>(&sdU[tt * R + j]);
        const float2 u01 = make_float2(u.x, u.y), u23 = make_float2(u.z, u.w);
        a0[j / 2] = __ffma2_rn(hx, u01, a0[j / 2]);
        a0[j / 2 + 1] = __ffma2_rn(hx, u23, a0[j / 2 + 1]);
        a1[j / 2] = __ffma2_rn(hy, u01, a1[j / 2]);
        a1[j / 2 + 1] = __ffma2_rn(hy, u23, a1[j / 2 + 1]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < R / 2; ++j) {
    sred[threadIdx.y][(2 * threadIdx.x) * R + 2 * j] = a0[j].x;
    sred[threadIdx.y][(2 * threadIdx.x) * R + 2 * j + 1] = a0[j].y;
    sred[threadIdx.y][(2 * threadIdx.x + 1) * R + 2 * j] = a1[j].x;
    sred[threadIdx.y][(2 * threadIdx.x + 1) * R + 2 * j + 1] = a1[j].y;
  }
  __syncthreads();
  for (int k = tid; k < 64 * R; k += NT) {
    float v = 0.f;
#pragma unroll
    for (int y = 0; y < Y; ++y) v += sred[y][k];
    const int ii = blockIdx.y * 64 + k / R;
    if (ii < d) gAp[((long long)c * d + ii) * rank_total + rank_off + (k % R)] = v;
  }
}

struct AdamArgs {
  long long n;       // d*R + V*R parameters
  float lr, b1, b2, c1, c2, eps, wd;  // c1 = 1 - b1, c2 = 1 - b2 (in f32)
  float b1t, b2t;    // 1 - b^step, computed on the host with powf
  float clip;
  int n_norm_parts;
};

// The optimizer update of one parameter from its mean gradient g: decoupled
// decay, then the Adam update (src/train.c:175-196), written with
// explicitly rounded operations so that it is the reference's f32
// arithmetic, op for op.
__device__ __forceinline__ void adam_element(const AdamArgs& a, long long k, float g,
                                             float* __restrict__ params,
                                             float* __restrict__ mom1,
                                             float* __restrict__ mom2) {
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

// Pack the step's gradient sums: G = [dA (d*R) | dB (V*R, vocab-major) |
// sum of losses | n_pred].  Every output element is summed in a fixed
// order, so the step is deterministic.  Modes (template kMode):
//   kFinG:     G only (a collective and/or the clip follow);
//   kFinNorm:  G and, per block, the sum of squares of g = G / n_pred (the
//              clip's global norm without a separate pass; no collective);
//   kFinAdam:  G, then g = G / n_pred and the whole optimizer update of the
//              element in the same pass (no collective, no clip): the
//              finalize, norm and Adam kernels of a step fused into one.
// Without a collective n_pred is this step's T.
enum : int { kFinG = 0, kFinNorm = 1, kFinAdam = 2 };
template <int R, int kMode>
__global__ void __launch_bounds__(256) lce_finalize(
    AdamArgs aa, int T, int cparts, int d, int V, long long Vpad, int n_chunks,
    const float* __restrict__ gAp, int res_rows, int n_b2, int G2, const float* __restrict__ gBp,
    unsigned long long* __restrict__ corr_fx, const float* __restrict__ loss_tok,
    float* __restrict__ Gbuf, float* __restrict__ params, float* __restrict__ mom1,
    float* __restrict__ mom2, float* __restrict__ gmean, double* __restrict__ norm_parts,
    float* __restrict__ loss_out) {
  const long long nA = (long long)d * R;
  const long long nB = Vpad * R;  // pair layout, entries of vocab ids >= V stay zero
  const long long stride = (long long)gridDim.x * blockDim.x;
  const int n_a2 = (V + res_rows - 1) / res_rows;
  const long long total2 = (long long)n_a2 * n_b2;
  const float inv = __fdiv_rn(1.0f, (float)T);
  double ss = 0.0;
  for (long long k = (long long)blockIdx.x * blockDim.x + threadIdx.x; k < nA + nB; k += stride) {
    float s = 0.f;
    if (k < nA) {
      for (int c = 0; c < n_chunks; ++c) s += gAp[(long long)c * nA + k];
    } else {
      const long long e = k - nA;
      const int v = (int)(2 * (e / (2 * R)) + (e & 1));
      if (v < V) {
        const int a = v / res_rows;
        const int s0 = tile_owner((long long)a * n_b2, total2, G2);
        const int s1 = tile_owner((long long)a * n_b2 + n_b2 - 1, total2, G2);
        for (int q = 0; q < cparts * (s1 - s0 + 1); ++q) s += gBp[(long long)q * Vpad * R + e];
        const long long c = (long long)corr_fx[e];
        if (c != 0) {
          s -= (float)((double)c * kFixInv);
          corr_fx[e] = 0ull;  // ready for the next step
        }
      }
    }
    Gbuf[k] = s;
    if constexpr (kMode == kFinNorm) {
      const float g = s * inv;
      ss += (double)g * (double)g;
    } else if constexpr (kMode == kFinAdam) {
      const float g = __fmul_rn(s, inv);
      gmean[k] = g;
      adam_element(aa, k, g, params, mom1, mom2);
    }
  }
  __shared__ float red[256];
  __shared__ double dred[256];
  if constexpr (kMode == kFinNorm) {
    dred[threadIdx.x] = ss;
    __syncthreads();
    for (int w = blockDim.x / 2; w > 0; w >>= 1) {
      if (threadIdx.x < w) dred[threadIdx.x] += dred[threadIdx.x + w];
      __syncthreads();
    }
    if (threadIdx.x == 0) norm_parts[blockIdx.x] = dred[0];
  }
  if (blockIdx.x == 0) {
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
      if (kMode == kFinAdam && loss_out) *loss_out = __fmul_rn(red[0], inv);
    }
  }
}

// Sum of squares of the mean gradient, per block (global-norm clip).
static __global__ void lce_sqnorm(long long n, const float* __restrict__ Gbuf, double* __restrict__ part) {
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

// g = G / n_pred (x clip coefficient); decoupled decay; Adam update
// (src/train.c:175-196), written with explicitly rounded operations so the
// update is the reference's f32 arithmetic, op for op.
static __global__ void lce_adam(AdamArgs a, float* __restrict__ params, float* __restrict__ mom1,
                         float* __restrict__ mom2, const float* __restrict__ Gbuf,
                         float* __restrict__ gmean, const double* __restrict__ norm_parts,
                         float* __restrict__ loss_out) {
  const float n_pred = Gbuf[a.n + 1];
  const float inv = __fdiv_rn(1.0f, n_pred);
  float coef = 1.0f;
  if (a.clip > 0.f) {
    // every block reduces the norm partials the same way (strided sums, then
    // a fixed tree), so every block gets the identical coefficient
    __shared__ double red[256];
    double ss = 0.0;
    for (int i = threadIdx.x; i < a.n_norm_parts; i += blockDim.x) ss += norm_parts[i];
    red[threadIdx.x] = ss;
    __syncthreads();
    for (int w = blockDim.x / 2; w > 0; w >>= 1) {
      if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
      __syncthreads();
    }
    const float norm = (float)sqrt(red[0]);
    const float c = __fdiv_rn(a.clip, __fadd_rn(norm, 1e-6f));
    if (c < 1.0f) coef = c;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && loss_out) *loss_out = __fmul_rn(Gbuf[a.n], inv);
  for (long long k = (long long)blockIdx.x * blockDim.x + threadIdx.x; k < a.n;
       k += (long long)gridDim.x * blockDim.x) {
    float g = __fmul_rn(Gbuf[k], inv);
    if (coef != 1.0f) g = __fmul_rn(g, coef);
    gmean[k] = g;
    adam_element(a, k, g, params, mom1, mom2);
  }
}

}  // namespace lce
