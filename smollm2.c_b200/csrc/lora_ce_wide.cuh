// lora_ce_wide.cuh — the training step for adapter ranks 65..256 (kernel
// ranks 128 and 256), the range the reference accepts above the fused
// passes' 64 (LORA_MAX_RANK 256, src/train.c:20, 156-160).
//
// The fused passes keep the full-rank logit term s*U*B inside the MMA as
// 2R extra resident K-columns; from rank 128 those no longer fit in shared
// memory beside the streamed ring, and the rank accumulator no longer fits
// in TMEM beside the logit tiles.  This path instead materialises the logit
// rows of a block of positions in HBM and runs the reference's per-position
// arithmetic (lora_accum, src/train.c:144-173) as whole-block products:
//
//   sU    = s * (h16 . A)                      [T][R]
//   Z     = h16 . W^T + sU . B                 [P][V]   per position block
//   Z    <- softmax(Z) - onehot(target)        (ce_loss_and_grad, :107-121)
//   dB   += sU^T . Z                           [R][V]
//   dU    = s * (Z . B^T)                      [P][R]
//   dA    = h16^T . dU                         [d][R]   over all positions
//
// then packs G = [dA | dB | sum of losses | n_pred] in the layout the
// fused path's finalize writes, so the all-reduce, the clip and Adam are
// the same kernels.  The products are fp32 CUDA-core GEMMs (f16 operands
// widen exactly), so every sum is an fp32 sum like the reference's, in a
// different order.  It is a slower path than the fused passes: it reads and
// writes each logit row several times instead of keeping it on chip.
#pragma once

#include <cuda_fp16.h>

#include <type_traits>

#include "lora_ce_kernels.cuh"

namespace lce {

constexpr int kWTile = 128;     // output rows and columns per block
constexpr int kWK = 16;         // K elements per shared-memory stage
constexpr int kWThreads = 256;  // 16 x 16 threads, 8 x 8 outputs each
constexpr int kWMaxSplit = 32;  // K splits of the dU and dA products

// Element (m, k) of a GEMM operand stored with K contiguous (p[m*ld + k])
// or with M contiguous (p[k*ld + m]); T is float or __half.
template <class T, bool kKC>
struct WideOp {
  const T* p;
  long long ld;
  static constexpr bool kKContig = kKC;
  __device__ __forceinline__ float at(int m, int k) const {
    const long long o = kKC ? (long long)m * ld + k : (long long)k * ld + m;
    if constexpr (std::is_same<T, __half>::value)
      return __half2float(p[o]);
    else
      return p[o];
  }
};

// c[m][n] = alpha * v
struct WideStore {
  float* c;
  long long ld;
  float alpha;
  __device__ __forceinline__ void operator()(int m, int n, int, float v) const {
    c[(long long)m * ld + n] = alpha * v;
  }
};

// c[m][n] += v (each element owned by one thread of one block)
struct WideAdd {
  float* c;
  long long ld;
  __device__ __forceinline__ void operator()(int m, int n, int, float v) const {
    c[(long long)m * ld + n] += v;
  }
};

// c[split][m][n] = v (split-K partials, summed later in split order)
struct WideSplit {
  float* c;
  long long ld, split_stride;
  __device__ __forceinline__ void operator()(int m, int n, int z, float v) const {
    c[(long long)z * split_stride + (long long)m * ld + n] = v;
  }
};

// The 8 elements of a 128 x 16 operand tile that thread `tid` moves: for
// K-contiguous operands 16 consecutive threads read one row's 16 k, for
// M-contiguous ones 128 consecutive threads read one k's 128 rows.
template <class Op>
__device__ __forceinline__ void wide_fetch(const Op& op, int r0, int rows, int k0, int k_hi,
                                           int tid, float (&reg)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = tid + i * kWThreads;
    const int r = Op::kKContig ? e / kWK : e % kWTile;
    const int k = Op::kKContig ? e % kWK : e / kWTile;
    const int gr = r0 + r, gk = k0 + k;
    reg[i] = (gr < rows && gk < k_hi) ? op.at(gr, gk) : 0.f;
  }
}

template <class Op>
__device__ __forceinline__ void wide_stash(const float (&reg)[8], int tid,
                                           float (*s)[kWTile + 4]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = tid + i * kWThreads;
    const int r = Op::kKContig ? e / kWK : e % kWTile;
    const int k = Op::kKContig ? e % kWK : e / kWTile;
    s[k][r] = reg[i];
  }
}

// C[m][n] = sum over this block's K range of A(m, k) * B(n, k), handed to
// the epilogue element by element.  blockIdx = (n tile, m tile, K split);
// split z covers k in [z*k_split, (z+1)*k_split).  Two shared-memory
// stages: the next stage is read into registers while the current one is
// multiplied, and written to the other stage after it (one barrier per
// stage).  The multiply-adds run two columns per f32x2 instruction, each
// lane of it an ordinary fp32 fma.
template <class OA, class OB, class Ep>
__global__ void __launch_bounds__(kWThreads, 2) lw_gemm(int M, int N, int K, int k_split, OA oa,
                                                     OB ob, Ep ep) {
  __shared__ __align__(16) float sa[2][kWK][kWTile + 4];
  __shared__ __align__(16) float sb[2][kWK][kWTile + 4];
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int m0 = blockIdx.y * kWTile, n0 = blockIdx.x * kWTile;
  const int k_lo = blockIdx.z * k_split;
  const int k_hi = min(K, k_lo + k_split);
  float2 acc[8][4];  // [row][column pair]
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = make_float2(0.f, 0.f);
  if (k_lo < k_hi) {
    float ra[8], rb[8];
    wide_fetch(oa, m0, M, k_lo, k_hi, tid, ra);
    wide_fetch(ob, n0, N, k_lo, k_hi, tid, rb);
    wide_stash<OA>(ra, tid, sa[0]);
    wide_stash<OB>(rb, tid, sb[0]);
    __syncthreads();
    int buf = 0;
    for (int k0 = k_lo; k0 < k_hi; k0 += kWK) {
      const bool more = k0 + kWK < k_hi;
      if (more) {
        wide_fetch(oa, m0, M, k0 + kWK, k_hi, tid, ra);
        wide_fetch(ob, n0, N, k0 + kWK, k_hi, tid, rb);
      }
#pragma unroll
      for (int k = 0; k < kWK; ++k) {
        float a[8], b[8];
        *reinterpret_cast<float4*>(&a[0]) = *reinterpret_cast<const float4*>(&sa[buf][k][ty * 4]);
        *reinterpret_cast<float4*>(&a[4]) =
            *reinterpret_cast<const float4*>(&sa[buf][k][64 + ty * 4]);
        *reinterpret_cast<float4*>(&b[0]) = *reinterpret_cast<const float4*>(&sb[buf][k][tx * 4]);
        *reinterpret_cast<float4*>(&b[4]) =
            *reinterpret_cast<const float4*>(&sb[buf][k][64 + tx * 4]);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float2 ai = make_float2(a[i], a[i]);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            acc[i][j] = __ffma2_rn(ai, make_float2(b[2 * j], b[2 * j + 1]), acc[i][j]);
        }
      }
      if (more) {
        wide_stash<OA>(ra, tid, sa[buf ^ 1]);
        wide_stash<OB>(rb, tid, sb[buf ^ 1]);
        __syncthreads();
        buf ^= 1;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
      if (n < N) ep(m, n, (int)blockIdx.z, (j & 1) ? acc[i][j >> 1].y : acc[i][j >> 1].x);
    }
  }
}

// h (bf16 / f16 / f32) -> f16 rows, round to nearest (the fused path's
// lce_prep conversion).
static __global__ void lw_convert(const void* __restrict__ H, int dtype, long long n,
                                  __half* __restrict__ h16) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    float x;
    if (dtype == 0)
      x = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(H)[i]);
    else if (dtype == 1)
      x = __half2float(reinterpret_cast<const __half*>(H)[i]);
    else
      x = reinterpret_cast<const float*>(H)[i];
    h16[i] = __float2half_rn(x);
  }
}

// B (pair-interleaved in params, bidx) -> plain [R][Vpad], zero past V.
static __global__ void lw_b_plain(const float* __restrict__ Bt, int R, int V, long long Vpad,
                                  float* __restrict__ Bp) {
  const long long n = (long long)R * Vpad;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const int j = (int)(i / Vpad);
    const long long v = i - (long long)j * Vpad;
    Bp[i] = v < V ? Bt[bidx(v, j, R)] : 0.f;
  }
}

__device__ __forceinline__ float lw_block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float r = red[0];
  for (int i = 1; i < nw; ++i) r = fmaxf(r, red[i]);
  return r;
}

__device__ __forceinline__ float lw_block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float r = red[0];
  for (int i = 1; i < nw; ++i) r += red[i];
  return r;
}

// One position per block (src/train.c:107-121): max, sum of e^(z - max),
// loss = -log(p_target + 1e-12), then the row becomes p - onehot(target).
// A target outside [0, V) sets the error flag and is read as 0.
constexpr int kWSoftThreads = 512;
static __global__ void __launch_bounds__(kWSoftThreads)
    lw_softmax(float* __restrict__ Z, long long ldz, int V, const int32_t* __restrict__ targets,
               int t0, float* __restrict__ loss_tok, int* err) {
  __shared__ float red[kWSoftThreads / 32];
  float* z = Z + (long long)blockIdx.x * ldz;
  float mx = -INFINITY;
  for (int v = threadIdx.x; v < V; v += blockDim.x) mx = fmaxf(mx, z[v]);
  mx = lw_block_max(mx, red);
  float s = 0.f;
  for (int v = threadIdx.x; v < V; v += blockDim.x) s += expf(z[v] - mx);
  s = lw_block_sum(s, red);
  const float inv = 1.0f / s;
  int tg = targets[t0 + blockIdx.x];
  if (tg < 0 || tg >= V) {
    if (threadIdx.x == 0) atomicCAS(err, 0, kErrTarget);
    tg = 0;
  }
  const float pt = expf(z[tg] - mx) * inv;
  __syncthreads();  // every thread has read z[tg] before the row is overwritten
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    const float p = expf(z[v] - mx) * inv;
    z[v] = v == tg ? p - 1.0f : p;
  }
  if (threadIdx.x == 0) loss_tok[t0 + blockIdx.x] = -logf(pt + 1e-12f);
}

// dU[p][j] = s * sum over the K splits (in split order) of the partials.
static __global__ void lw_reduce_du(int P, int R, int splits, const float* __restrict__ part,
                                    float scale, float* __restrict__ dU) {
  const long long n = (long long)P * R;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int z = 0; z < splits; ++z) s += part[(long long)z * n + i];
    dU[i] = scale * s;
  }
}

// G = [dA (d x R) | dB (bidx layout) | sum of losses | n_pred = T]: dA from
// its split partials (split order), dB from the accumulated [R][Vpad]
// product, the loss sum over positions in a fixed order.
static __global__ void __launch_bounds__(256)
    lw_pack(int d, int R, int V, long long Vpad, int T, int a_splits,
            const float* __restrict__ dA_part, const float* __restrict__ dBacc,
            const float* __restrict__ loss_tok, float* __restrict__ G) {
  const long long nA = (long long)d * R, nB = Vpad * R;
  for (long long k = (long long)blockIdx.x * blockDim.x + threadIdx.x; k < nA + nB;
       k += (long long)gridDim.x * blockDim.x) {
    float s = 0.f;
    if (k < nA) {
      for (int z = 0; z < a_splits; ++z) s += dA_part[(long long)z * nA + k];
    } else {
      const long long e = k - nA;
      const long long v = 2 * (e / (2 * R)) + (e & 1);
      const int j = (int)((e % (2 * R)) >> 1);
      if (v < V) s = dBacc[(long long)j * Vpad + v];
    }
    G[k] = s;
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
      G[nA + nB] = red[0];
      G[nA + nB + 1] = (float)T;
    }
  }
}

}  // namespace lce
