// lora_body.cu — the SmolLM2 body forward on the GPU for every position of
// a batch of sequences at once (C ABI: include/lora_body.h).  The reference
// computes the same hidden states one position at a time on the CPU
// (forward_prefill / forward_decode, src/forward.c:935-1093, 1129-1256).
//
// Exactness.  The integer parts are exact: int8 weights (per-row scales)
// and int8 activations (per-tensor scales) are quantised with the
// reference's own rounding rules and summed in int32, so each matmul output
// is bit-identical given bit-identical inputs.  The float parts follow the
// reference's operation order with explicitly rounded operations (no
// contraction, as the reference's -std=c99 build has none): RoPE from f32
// cos / sin tables computed on the host with the same libm calls, the
// attention dot products and weighted sums in the reference's order, the
// residual adds, the RMSNorm's f64 sum of squares in index order.  One
// thing differs: e^x (softmax, sigmoid) comes from a double-precision exp
// rounded to f32 (exp_ref), which differs from glibc's expf in the last bit
// for a small fraction of arguments; such a difference can move an int8
// activation of the next matmul by one step now and then, which the tests
// bound.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "lora_body.h"

namespace {

thread_local std::string g_body_error;

int bfail(int code, const std::string& msg) {
  g_body_error = msg;
  return code;
}

#define BD_CUDA(call)                                                                   \
  do {                                                                                  \
    cudaError_t e_ = (call);                                                            \
    if (e_ != cudaSuccess)                                                              \
      return bfail(LORA_CE_ECUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)

constexpr int kHd = 64;          // head dimension (the reference's attention rows)
constexpr int kMaxSeqBody = 4096;

// ------------------------------------------------------------------ kernels

// e^x rounded to f32 from CUDA's double-precision exp: the correctly rounded
// result except where the exact value lies within a double-precision error
// of a float rounding boundary.  The reference calls glibc's expf, which
// agrees with this on all but 0.008% of the floats in [-100, 80] (a sweep of
// 1.4e9 of them on the build host); CUDA's own expf has a 2-ulp bound, and
// every last-bit difference in a softmax weight or a sigmoid can move an
// int8 activation of the next matmul by one step.
__device__ __forceinline__ float exp_ref(float x) { return (float)exp((double)x); }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// quantize_f16_rows_to_q8_perrow (src/forward.c:441-462): per row, scale =
// amax / 127, q = (int)(v * (127 / amax) + 0.5) clamped to [-127, 127].
__global__ void bd_quant_rows(const __half* __restrict__ W, int rows, int cols,
                              int8_t* __restrict__ q, float* __restrict__ scale) {
  const int r = blockIdx.x;
  if (r >= rows) return;
  const __half* w = W + (size_t)r * cols;
  float amax = 0.f;
  for (int i = threadIdx.x; i < cols; i += blockDim.x) amax = fmaxf(amax, fabsf(__half2float(w[i])));
  __shared__ float red[32];
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_max(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  amax = red[0];
  const float inv = amax > 0.f ? __fdiv_rn(127.0f, amax) : 0.f;
  for (int i = threadIdx.x; i < cols; i += blockDim.x) {
    int v = __float2int_rz(__fadd_rn(__fmul_rn(__half2float(w[i]), inv), 0.5f));
    v = v > 127 ? 127 : v < -127 ? -127 : v;
    q[(size_t)r * cols + i] = (int8_t)v;
  }
  if (threadIdx.x == 0) scale[r] = amax > 0.f ? __fdiv_rn(amax, 127.0f) : 1.0f;
}

// x[t] = token_embd[tokens[t]] in f32 (exact); an id out of range reads row
// 0 and sets the error flag.
__global__ void bd_embed(const int32_t* __restrict__ tokens, int T, int d, int V,
                         const __half* __restrict__ embd, float* __restrict__ x, int* err) {
  const long long n = (long long)T * d;
  for (long long k = (long long)blockIdx.x * blockDim.x + threadIdx.x; k < n;
       k += (long long)gridDim.x * blockDim.x) {
    const int t = (int)(k / d), i = (int)(k % d);
    int tok = tokens[t];
    if (tok < 0 || tok >= V) {
      if (i == 0) atomicExch(err, 1);
      tok = 0;
    }
    x[k] = __half2float(embd[(size_t)tok * d + i]);
  }
}

// Per-tensor int8 quantisation of one row (the x86 branch of
// quantize_row_to_q8_tensor, src/forward.c:157-166): scale = amax / 127,
// q = (int)roundf(v * (127 / amax)) clamped to [-127, 127].  One warp.
__device__ __forceinline__ void quant_row_warp(const float* __restrict__ src, int n,
                                               int8_t* __restrict__ dst, float* scale_out,
                                               int lane) {
  float amax = 0.f;
  for (int i = lane; i < n; i += 32) amax = fmaxf(amax, fabsf(src[i]));
  amax = warp_max(amax);
  const float inv = amax > 0.f ? __fdiv_rn(127.0f, amax) : 0.f;
  for (int i = lane; i < n; i += 32) {
    int v = (int)roundf(__fmul_rn(src[i], inv));
    v = v > 127 ? 127 : v < -127 ? -127 : v;
    dst[i] = (int8_t)v;
  }
  if (lane == 0) *scale_out = amax > 0.f ? __fdiv_rn(amax, 127.0f) : 1.0f;
}

// rmsnorm (the x86 branch, src/forward.c:366-371): f64 sum of squares,
// inv = 1 / sqrtf(ss / n + eps), out = x * inv * w.  One warp per row: the
// lanes square the row into shared memory (each square of an f32 is exact
// in f64), lane 0 adds them in index order as the reference does, then the
// normalised row goes to `xn` (scratch) and on to int8 + scale (quantised)
// or to the final hidden state in out_dtype.
constexpr int kNormWarps = 4;
__global__ void __launch_bounds__(32 * kNormWarps)
    bd_norm(const float* __restrict__ x, const float* __restrict__ w, int T, int d, float eps,
            float* __restrict__ xn, int8_t* __restrict__ xq, float* __restrict__ xs,
            void* __restrict__ out, int out_dtype) {
  extern __shared__ double sq_all[];
  const int wib = threadIdx.x >> 5;
  const int warp = blockIdx.x * kNormWarps + wib;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  double* sq = sq_all + (size_t)wib * d;
  const float* xr = x + (size_t)warp * d;
  for (int i = lane; i < d; i += 32) sq[i] = (double)xr[i] * (double)xr[i];
  __syncwarp();
  double ss = 0.0;
  if (lane == 0) {
    int i = 0;
    for (; i + 8 <= d; i += 8) {
      const double a0 = sq[i], a1 = sq[i + 1], a2 = sq[i + 2], a3 = sq[i + 3];
      const double a4 = sq[i + 4], a5 = sq[i + 5], a6 = sq[i + 6], a7 = sq[i + 7];
      ss += a0; ss += a1; ss += a2; ss += a3; ss += a4; ss += a5; ss += a6; ss += a7;
    }
    for (; i < d; ++i) ss += sq[i];
  }
  ss = __shfl_sync(0xffffffffu, ss, 0);
  ss /= d;
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)ss, eps)));
  float* nr = xn + (size_t)warp * d;
  for (int i = lane; i < d; i += 32) nr[i] = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
  __syncwarp();
  if (xq) {
    quant_row_warp(nr, d, xq + (size_t)warp * d, xs + warp, lane);
  } else {
    for (int i = lane; i < d; i += 32) {
      const float v = nr[i];
      const size_t k = (size_t)warp * d + i;
      if (out_dtype == LORA_CE_F32)
        static_cast<float*>(out)[k] = v;
      else if (out_dtype == LORA_CE_BF16)
        static_cast<__nv_bfloat16*>(out)[k] = __float2bfloat16_rn(v);
      else
        static_cast<__half*>(out)[k] = __float2half_rn(v);
    }
  }
}

// Per-tensor int8 quantisation of rows of n floats, one warp per row.
__global__ void bd_quant_act(const float* __restrict__ src, int T, int n, int8_t* __restrict__ q,
                             float* __restrict__ s) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  quant_row_warp(src + (size_t)warp * n, n, q + (size_t)warp * n, s + warp, lane);
}

// SwiGLU then int8: a = g * (1 / (1 + e^-g)) * u (src/forward.c:1239-1242),
// quantised over the row (per-tensor, as quant_row_warp).  gu is [T][2*ffn]
// (gate | up); one 256-thread block per row.
__global__ void __launch_bounds__(256) bd_act_quant(const float* __restrict__ gu, int T, int ffn,
                                                    float* __restrict__ a, int8_t* __restrict__ q,
                                                    float* __restrict__ s) {
  const int row = blockIdx.x;
  if (row >= T) return;
  const float* g = gu + (size_t)row * 2 * ffn;
  float* ar = a + (size_t)row * ffn;
  float amax = 0.f;
  for (int i = threadIdx.x; i < ffn; i += blockDim.x) {
    const float gv = g[i];
    const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_ref(-gv)));
    const float v = __fmul_rn(__fmul_rn(gv, sig), g[ffn + i]);
    ar[i] = v;
    amax = fmaxf(amax, fabsf(v));
  }
  __shared__ float red[32];
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_max(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  amax = red[0];
  const float inv = amax > 0.f ? __fdiv_rn(127.0f, amax) : 0.f;
  for (int i = threadIdx.x; i < ffn; i += blockDim.x) {
    int v = (int)roundf(__fmul_rn(ar[i], inv));
    v = v > 127 ? 127 : v < -127 ? -127 : v;
    q[(size_t)row * ffn + i] = (int8_t)v;
  }
  if (threadIdx.x == 0) s[row] = amax > 0.f ? __fdiv_rn(amax, 127.0f) : 1.0f;
}

// Y[t][n] (+)= (float)(sum_k X[t][k] * W[n][k]) * xs[t] * ws[n]: the
// reference's matmul_q8_dot_perrow (src/forward.c:470-511, int32 sums, two
// rounded multiplies), with `accumulate` adding it to Y as the residual
// add does.  Tiles of 8*MR positions x 64 outputs (MR = 4 for the wide
// gate/up GEMM, 2 for the narrower ones, whose 32-position tiles left SMs
// idle), 128 threads of MR x 4 outputs, K in 64-byte steps (K % 64 == 0)
// with the next step's tile loaded into registers while the current one is
// multiplied (dp4a; the int32 sums are exact in any order, so the tiling
// does not change any result).
constexpr int kGemmTN = 64;
template <int MR>
__global__ void __launch_bounds__(128) bd_gemm_q8(const int8_t* __restrict__ X,
                                                  const float* __restrict__ xs, int T, int K,
                                                  const int8_t* __restrict__ W,
                                                  const float* __restrict__ ws, int N,
                                                  float* __restrict__ Y, int ldy, int accumulate) {
  constexpr int TM = 8 * MR;
  __shared__ int sX[TM][17];
  __shared__ int sW[kGemmTN][17];
  const int t0 = blockIdx.y * TM, n0 = blockIdx.x * kGemmTN;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;  // 16 x 8 threads
  int acc[MR][4];
#pragma unroll
  for (int m = 0; m < MR; ++m)
#pragma unroll
    for (int n = 0; n < 4; ++n) acc[m][n] = 0;
  // this thread's share of a K-step: MR words of X, 8 of W
  int rx[MR], rw[8];
  auto load = [&](int k0) {
#pragma unroll
    for (int u = 0; u < MR; ++u) {
      const int i = threadIdx.x + 128 * u, r = i >> 4, c = i & 15;
      const int tr = t0 + r;
      rx[u] = tr < T ? __ldg(reinterpret_cast<const int*>(X + (size_t)tr * K + k0 + 4 * c)) : 0;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = threadIdx.x + 128 * u, r = i >> 4, c = i & 15;
      const int nr = n0 + r;
      rw[u] = nr < N ? __ldg(reinterpret_cast<const int*>(W + (size_t)nr * K + k0 + 4 * c)) : 0;
    }
  };
  load(0);
  for (int k0 = 0; k0 < K; k0 += 64) {
#pragma unroll
    for (int u = 0; u < MR; ++u) {
      const int i = threadIdx.x + 128 * u;
      sX[i >> 4][i & 15] = rx[u];
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = threadIdx.x + 128 * u;
      sW[i >> 4][i & 15] = rw[u];
    }
    __syncthreads();
    if (k0 + 64 < K) load(k0 + 64);
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      int av[MR], bv[4];
#pragma unroll
      for (int m = 0; m < MR; ++m) av[m] = sX[ty * MR + m][c];
#pragma unroll
      for (int n = 0; n < 4; ++n) bv[n] = sW[tx * 4 + n][c];
#pragma unroll
      for (int m = 0; m < MR; ++m)
#pragma unroll
        for (int n = 0; n < 4; ++n) acc[m][n] = __dp4a(av[m], bv[n], acc[m][n]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    const int t = t0 + ty * MR + m;
    if (t >= T) continue;
    const float sx = xs[t];
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      const int o = n0 + tx * 4 + n;
      if (o >= N) continue;
      const float y = __fmul_rn(__fmul_rn(__int2float_rn(acc[m][n]), sx), ws[o]);
      float* dst = Y + (size_t)t * ldy + o;
      *dst = accumulate ? __fadd_rn(*dst, y) : y;
    }
  }
}

// RoPE from the f32 tables (rope_llama_table, src/forward.c:552-565) on q
// (heads 0..nh-1 of the qkv row) and k (the next nkv heads) at each
// position's place in its sequence.
__global__ void bd_rope(float* __restrict__ qkv, int T, int ld, int n_rot_heads,
                        const int32_t* __restrict__ pos, const float* __restrict__ cosT,
                        const float* __restrict__ sinT) {
  constexpr int half = kHd / 2;
  const long long n = (long long)T * n_rot_heads * half;
  for (long long k = (long long)blockIdx.x * blockDim.x + threadIdx.x; k < n;
       k += (long long)gridDim.x * blockDim.x) {
    const int i = (int)(k % half);
    const int hh = (int)((k / half) % n_rot_heads);
    const int t = (int)(k / ((long long)half * n_rot_heads));
    float* v = qkv + (size_t)t * ld + hh * kHd;
    const float c = cosT[(size_t)pos[t] * half + i], s = sinT[(size_t)pos[t] * half + i];
    const float a = v[2 * i], b = v[2 * i + 1];
    v[2 * i] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    v[2 * i + 1] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
  }
}

// Causal GQA attention in the reference's order (src/forward.c:1186-1229),
// one warp per (position, query head) item: scores q.k / 8 (each lane one
// key, the 64-term sum in index order), max, e = e^(s - max), the sum of e
// in key order (lane 0), then out[i] = sum over keys of (e * (1/sum)) * v[i]
// in key order (lanes over i).  Keys from seq_start + s_start(window) to t.
// One block per (tile of kAttnTile positions, KV head) first copies that
// head's K and V rows for the tile's key range into shared memory (rows
// padded to kAttnRowF floats, so the lanes' row-strided float4 reads fall in
// different banks): every key row is read from global memory once per
// block instead of once per item.  A block whose key range has more rows
// than `stage_cap` reads them from global memory.  The loads are vectorised
// and the key loops unrolled so that they are in flight ahead of the ordered
// additions.
constexpr int kAttnTile = 8;
constexpr int kAttnTWarps = 12;
constexpr int kAttnRowF = kHd + 4;
// dynamic shared memory of bd_attn_tile: the warps' score rows, then the
// staged K and V rows
inline size_t attn_tile_smem(int max_seq, int stage_cap) {
  return (size_t)kAttnTWarps * max_seq * 4 + 2 * (size_t)stage_cap * kAttnRowF * 4;
}
__global__ void __launch_bounds__(32 * kAttnTWarps)
    bd_attn_tile(const float* __restrict__ qkv, int T, int ld, int nh, int nkv, int dim,
                 const int32_t* __restrict__ pos, int window, float* __restrict__ out, int max_seq,
                 int stage_cap) {
  extern __shared__ __align__(16) float att_smem[];
  __shared__ int s_lo;
  const int wib = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * kAttnTile;
  const int t1 = min(T, t0 + kAttnTile);
  const int kvh = blockIdx.y;
  const int gsz = nh / nkv;  // query heads of this KV head: h * nkv / nh == kvh
  auto first_key = [&](int t) {
    const int p = pos[t];
    int lo = 0;
    if (window > 0) {
      lo = p + 1 - window;
      if (lo < 0) lo = 0;
      if (lo > p) lo = p;
    }
    return t - p + lo;
  };
  if (threadIdx.x == 0) {
    int m = t0;
    for (int t = t0; t < t1; ++t) m = min(m, first_key(t));
    s_lo = m;
  }
  __syncthreads();
  const int kv_lo = s_lo;
  const int n_rows = t1 - kv_lo;
  const bool staged = n_rows <= stage_cap;
  float* sc_all = att_smem;                        // [kAttnTWarps][max_seq] scores
  float* sK = att_smem + (size_t)kAttnTWarps * max_seq;
  float* sV = sK + (size_t)stage_cap * kAttnRowF;
  const float* gK = qkv + dim + kvh * kHd;
  const float* gV = qkv + dim + nkv * kHd + kvh * kHd;
  if (staged) {
    // 16 float4 per row; each thread moves up to 8 (row, float4) slices of
    // K and V per round, all loads of a round in flight before its stores
    constexpr int kQ = kHd / 4, kU = 8;
    const int n4 = n_rows * kQ;
    for (int k0 = 0; k0 < n4; k0 += kU * (int)blockDim.x) {
      float4 kv4[kU], vv4[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int k = k0 + u * (int)blockDim.x + (int)threadIdx.x;
        if (k < n4) {
          const size_t go = (size_t)(kv_lo + k / kQ) * ld;
          kv4[u] = __ldg(reinterpret_cast<const float4*>(gK + go) + k % kQ);
          vv4[u] = __ldg(reinterpret_cast<const float4*>(gV + go) + k % kQ);
        }
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int k = k0 + u * (int)blockDim.x + (int)threadIdx.x;
        if (k < n4) {
          const size_t so = (size_t)(k / kQ) * kAttnRowF + 4 * (k % kQ);
          *reinterpret_cast<float4*>(sK + so) = kv4[u];
          *reinterpret_cast<float4*>(sV + so) = vv4[u];
        }
      }
    }
  }
  __syncthreads();
  // row r of K / V: base + (r - row0) * stride
  const float* kb = staged ? sK : gK;
  const float* vb = staged ? sV : gV;
  const long long kst = staged ? kAttnRowF : ld;
  const int row0 = staged ? kv_lo : 0;
  float* sc = sc_all + (size_t)wib * max_seq;
  const int n_items = (t1 - t0) * gsz;
  for (int it = wib; it < n_items; it += kAttnTWarps) {
    const int t = t0 + it / gsz, h = kvh * gsz + it % gsz;
    const int first = first_key(t);
    const int n_keys = t - first + 1;
    float qv[kHd];
    {
      const float4* q4 = reinterpret_cast<const float4*>(qkv + (size_t)t * ld + h * kHd);
#pragma unroll
      for (int i = 0; i < kHd / 4; ++i) {
        const float4 v = __ldg(q4 + i);
        qv[4 * i] = v.x; qv[4 * i + 1] = v.y; qv[4 * i + 2] = v.z; qv[4 * i + 3] = v.w;
      }
    }
    float mx = -INFINITY;
    for (int j = lane; j < n_keys; j += 32) {
      const float4* k4 = reinterpret_cast<const float4*>(kb + (long long)(first + j - row0) * kst);
      float kv[kHd];
#pragma unroll
      for (int i = 0; i < kHd / 4; ++i) {
        const float4 v = k4[i];
        kv[4 * i] = v.x; kv[4 * i + 1] = v.y; kv[4 * i + 2] = v.z; kv[4 * i + 3] = v.w;
      }
      float dd = 0.f;
#pragma unroll
      for (int i = 0; i < kHd; ++i) dd = __fadd_rn(dd, __fmul_rn(qv[i], kv[i]));
      dd = __fmul_rn(dd, 0.125f);  // 1 / sqrtf(64)
      sc[j] = dd;
      mx = fmaxf(mx, dd);
    }
    mx = warp_max(mx);
    __syncwarp();
    for (int j = lane; j < n_keys; j += 32) sc[j] = exp_ref(__fsub_rn(sc[j], mx));
    __syncwarp();
    float sum = 0.f;
    if (lane == 0) {
      int j = 0;
      for (; j + 8 <= n_keys; j += 8) {
        const float e0 = sc[j], e1 = sc[j + 1], e2 = sc[j + 2], e3 = sc[j + 3];
        const float e4 = sc[j + 4], e5 = sc[j + 5], e6 = sc[j + 6], e7 = sc[j + 7];
        sum = __fadd_rn(sum, e0); sum = __fadd_rn(sum, e1); sum = __fadd_rn(sum, e2);
        sum = __fadd_rn(sum, e3); sum = __fadd_rn(sum, e4); sum = __fadd_rn(sum, e5);
        sum = __fadd_rn(sum, e6); sum = __fadd_rn(sum, e7);
      }
      for (; j < n_keys; ++j) sum = __fadd_rn(sum, sc[j]);
    }
    sum = __shfl_sync(0xffffffffu, sum, 0);
    const float inv_sum = sum > 0.f ? __fdiv_rn(1.0f, sum) : 0.f;
    float o0 = 0.f, o1 = 0.f;
    int j = 0;
    for (; j + 8 <= n_keys; j += 8) {
      float va[8], vb2[8], wg[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float* vr = vb + (long long)(first + j + u - row0) * kst;
        va[u] = vr[lane];
        vb2[u] = vr[lane + 32];
        wg[u] = __fmul_rn(sc[j + u], inv_sum);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        o0 = __fadd_rn(o0, __fmul_rn(wg[u], va[u]));
        o1 = __fadd_rn(o1, __fmul_rn(wg[u], vb2[u]));
      }
    }
    for (; j < n_keys; ++j) {
      const float wgt = __fmul_rn(sc[j], inv_sum);
      const float* vr = vb + (long long)(first + j - row0) * kst;
      o0 = __fadd_rn(o0, __fmul_rn(wgt, vr[lane]));
      o1 = __fadd_rn(o1, __fmul_rn(wgt, vr[lane + 32]));
    }
    float* orow = out + (size_t)t * dim + h * kHd;
    orow[lane] = o0;
    orow[lane + 32] = o1;
    __syncwarp();  // sc is reused by this warp's next item
  }
}

}  // namespace

struct lora_body_handle {
  lora_body_config cfg{};
  int d = 0, ffn = 0, kvdim = 0, nqkv = 0, Tcap = 0;
  int attn_cap = 0;  // K / V rows bd_attn_tile stages per block
  int num_sms = 0;
  cudaStream_t stream = nullptr;
  // weights (int8 per-row) and scales, per layer
  struct Layer {
    int8_t* wqkv = nullptr;  // [q | k | v] rows, each [d]
    float* sqkv = nullptr;
    int8_t* wo = nullptr;
    float* so = nullptr;
    int8_t* wgu = nullptr;   // [gate | up] rows, each [d]
    float* sgu = nullptr;
    int8_t* wd = nullptr;    // [d] rows of [ffn]
    float* sd = nullptr;
    float* attn_norm = nullptr;
    float* ffn_norm = nullptr;
    int window = 0;
    bool set = false;
  };
  std::vector<Layer> layers;
  __half* embd = nullptr;
  float* out_norm = nullptr;
  bool have_embd = false;
  float* rope_cos = nullptr;
  float* rope_sin = nullptr;
  // activations
  float* x = nullptr;     // [Tcap][d] residual stream
  float* xn = nullptr;    // [Tcap][max(d, ffn)] scratch (normalised rows, SwiGLU output)
  int8_t* xq = nullptr;   // [Tcap][max(d, ffn)]
  float* xs = nullptr;    // [Tcap]
  float* qkv = nullptr;   // [Tcap][nqkv]
  float* att = nullptr;   // [Tcap][d]
  float* gu = nullptr;    // [Tcap][2 ffn]
  int32_t* pos = nullptr;
  int32_t* tok = nullptr;  // staging for host tokens
  float* hout = nullptr;   // staging for host output
  int32_t* pos_host = nullptr;  // pinned
  int* err = nullptr;
  int32_t* tgt = nullptr;  // staging for host targets (lora_body_train_step)
  float* loss = nullptr;   // [loss, spare]
  // the forward as a CUDA graph, for the last (T, tokens, output, dtype)
  bool use_graph = true;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t gexec = nullptr;
  int gT = -1, gdtype = 0;
  const int32_t* gtok = nullptr;
  void* gout = nullptr;
};

namespace {

template <class T>
int balloc(T** p, size_t count) {
  if (cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T) + 16) != cudaSuccess) {
    *p = nullptr;
    cudaGetLastError();
    return bfail(LORA_CE_ENOMEM, "cudaMalloc failed");
  }
  return 0;
}

void drop_body_graph(lora_body_handle* h);

void free_body(lora_body_handle* h) {
  drop_body_graph(h);
  for (auto& L : h->layers) {
    void* ps[] = {L.wqkv, L.sqkv, L.wo, L.so, L.wgu, L.sgu, L.wd, L.sd, L.attn_norm, L.ffn_norm};
    for (void* p : ps)
      if (p) cudaFree(p);
  }
  void* ps[] = {h->embd, h->out_norm, h->rope_cos, h->rope_sin, h->x,   h->xn,  h->xq,
                h->xs,   h->qkv,      h->att,      h->gu,       h->pos, h->tok, h->hout,
                h->err,  h->tgt,      h->loss};
  for (void* p : ps)
    if (p) cudaFree(p);
  if (h->pos_host) cudaFreeHost(h->pos_host);
  if (h->stream) cudaStreamDestroy(h->stream);
}

// Upload f16 rows, quantise them to int8 rows at q (rows x cols) with scales.
int upload_quant(lora_body_handle* h, const uint16_t* src, int rows, int cols, int8_t* q,
                 float* scale, __half* tmp) {
  BD_CUDA(cudaMemcpyAsync(tmp, src, (size_t)rows * cols * 2, cudaMemcpyHostToDevice, h->stream));
  bd_quant_rows<<<rows, 256, 0, h->stream>>>(tmp, rows, cols, q, scale);
  BD_CUDA(cudaGetLastError());
  return 0;
}

int check_offsets(lora_body_handle* h, const int32_t* offsets, int n_seqs, int* T_out) {
  if (!offsets || n_seqs < 1) return bfail(LORA_CE_EINVAL, "need at least one sequence");
  if (offsets[0] != 0) return bfail(LORA_CE_EINVAL, "offsets[0] must be 0");
  for (int i = 0; i < n_seqs; ++i) {
    const int len = offsets[i + 1] - offsets[i];
    if (len < 1 || len > h->cfg.max_seq)
      return bfail(LORA_CE_EINVAL, "every sequence needs 1..max_seq positions");
  }
  const int T = offsets[n_seqs];
  if (T > h->Tcap) return bfail(LORA_CE_EINVAL, "more positions than max_tokens");
  *T_out = T;
  return 0;
}

// The whole forward on the handle's stream: d_tok [T] -> out [T][d].
// The forward's kernels (capturable: no host work, no copies).
int enqueue_body(lora_body_handle* h, const int32_t* d_tok, int T, void* out, int out_dtype) {
  cudaStream_t st = h->stream;
  const int d = h->d, ffn = h->ffn, nh = h->cfg.n_heads, nkv = h->cfg.n_kv_heads;
  const int eb = (int)std::min<long long>(((long long)T * d + 255) / 256, 4096);
  bd_embed<<<eb, 256, 0, st>>>(d_tok, T, d, h->cfg.vocab, h->embd, h->x, h->err);
  const int rows_blocks = (T * 32 + 255) / 256;  // one warp per row, 8 per block
  const int norm_blocks = (T + kNormWarps - 1) / kNormWarps;
  const size_t norm_smem = (size_t)kNormWarps * d * sizeof(double);
  // int8 GEMM Y (+)= X . W^T over N outputs: tiles of 32 positions, or of
  // 16 where 32-position tiles would leave SMs without a block
  auto gemm = [&](const int8_t* W, const float* ws, int K, int N, float* Y, int ldy, int acc) {
    const int nb = (N + kGemmTN - 1) / kGemmTN;
    if ((long long)nb * ((T + 31) / 32) < h->num_sms)
      bd_gemm_q8<2><<<dim3(nb, (T + 15) / 16), 128, 0, st>>>(h->xq, h->xs, T, K, W, ws, N, Y,
                                                            ldy, acc);
    else
      bd_gemm_q8<4><<<dim3(nb, (T + 31) / 32), 128, 0, st>>>(h->xq, h->xs, T, K, W, ws, N, Y,
                                                            ldy, acc);
  };
  const int max_seq = h->cfg.max_seq;
  const size_t attn_smem = attn_tile_smem(max_seq, h->attn_cap);
  const dim3 g_att((unsigned)((T + kAttnTile - 1) / kAttnTile), (unsigned)nkv);
  const int rope_blocks = (int)std::min<long long>(((long long)T * (nh + nkv) * 32 + 255) / 256, 8192);
  for (int L = 0; L < h->cfg.n_layers; ++L) {
    const auto& ly = h->layers[L];
    bd_norm<<<norm_blocks, 32 * kNormWarps, norm_smem, st>>>(h->x, ly.attn_norm, T, d, h->cfg.rms_eps, h->xn, h->xq,
                                         h->xs, nullptr, 0);
    gemm(ly.wqkv, ly.sqkv, d, h->nqkv, h->qkv, h->nqkv, 0);
    bd_rope<<<rope_blocks, 256, 0, st>>>(h->qkv, T, h->nqkv, nh + nkv, h->pos, h->rope_cos,
                                         h->rope_sin);
    bd_attn_tile<<<g_att, 32 * kAttnTWarps, attn_smem, st>>>(
        h->qkv, T, h->nqkv, nh, nkv, d, h->pos, ly.window, h->att, max_seq, h->attn_cap);
    bd_quant_act<<<rows_blocks, 256, 0, st>>>(h->att, T, d, h->xq, h->xs);
    gemm(ly.wo, ly.so, d, d, h->x, d, 1);
    bd_norm<<<norm_blocks, 32 * kNormWarps, norm_smem, st>>>(h->x, ly.ffn_norm, T, d, h->cfg.rms_eps, h->xn, h->xq,
                                         h->xs, nullptr, 0);
    gemm(ly.wgu, ly.sgu, d, 2 * ffn, h->gu, 2 * ffn, 0);
    bd_act_quant<<<T, 256, 0, st>>>(h->gu, T, ffn, h->xn, h->xq, h->xs);
    gemm(ly.wd, ly.sd, ffn, d, h->x, d, 1);
  }
  bd_norm<<<norm_blocks, 32 * kNormWarps, norm_smem, st>>>(h->x, h->out_norm, T, d, h->cfg.rms_eps, h->xn, nullptr,
                                       nullptr, out, out_dtype);
  BD_CUDA(cudaGetLastError());
  return 0;
}

void drop_body_graph(lora_body_handle* h) {
  if (h->gexec) cudaGraphExecDestroy(h->gexec);
  if (h->graph) cudaGraphDestroy(h->graph);
  h->gexec = nullptr;
  h->graph = nullptr;
  h->gT = -1;
}

// Positions of the tokens within their sequences (uploaded every call), then
// the forward: a CUDA graph of its ~8 launches per layer, captured on first
// use and replayed while (T, tokens, output, dtype) repeat.
int run_body(lora_body_handle* h, const int32_t* d_tok, const int32_t* offsets, int n_seqs,
             int T, void* out, int out_dtype) {
  cudaStream_t st = h->stream;
  for (int i = 0; i < n_seqs; ++i)
    for (int t = offsets[i]; t < offsets[i + 1]; ++t) h->pos_host[t] = t - offsets[i];
  BD_CUDA(cudaMemcpyAsync(h->pos, h->pos_host, (size_t)T * 4, cudaMemcpyHostToDevice, st));
  if (!h->use_graph) return enqueue_body(h, d_tok, T, out, out_dtype);
  if (!(h->gexec && h->gT == T && h->gtok == d_tok && h->gout == out && h->gdtype == out_dtype)) {
    drop_body_graph(h);
    cudaGraph_t graph = nullptr;
    if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
      cudaGetLastError();
      h->use_graph = false;
      return enqueue_body(h, d_tok, T, out, out_dtype);
    }
    const int rc = enqueue_body(h, d_tok, T, out, out_dtype);
    const cudaError_t ce = cudaStreamEndCapture(st, &graph);
    cudaGraphExec_t exec = nullptr;
    if (rc || ce != cudaSuccess || !graph || cudaGraphInstantiate(&exec, graph, 0) != cudaSuccess) {
      if (graph) cudaGraphDestroy(graph);
      cudaGetLastError();
      h->use_graph = false;  // launch directly from now on
      return rc ? rc : enqueue_body(h, d_tok, T, out, out_dtype);
    }
    h->graph = graph;
    h->gexec = exec;
    h->gT = T;
    h->gtok = d_tok;
    h->gout = out;
    h->gdtype = out_dtype;
  }
  BD_CUDA(cudaGraphLaunch(h->gexec, st));
  return 0;
}

int body_check_error(lora_body_handle* h) {
  int e = 0;
  BD_CUDA(cudaMemcpyAsync(&e, h->err, 4, cudaMemcpyDeviceToHost, h->stream));
  BD_CUDA(cudaStreamSynchronize(h->stream));
  if (e) {
    BD_CUDA(cudaMemset(h->err, 0, 4));
    return bfail(LORA_CE_EDEVICE, "token id out of range");
  }
  return 0;
}

}  // namespace

extern "C" {

const char* lora_body_last_error(void) { return g_body_error.c_str(); }

int lora_body_create(const lora_body_config* c, lora_body_handle** out) {
  if (!out) return bfail(LORA_CE_EINVAL, "null output pointer");
  *out = nullptr;
  if (!c) return bfail(LORA_CE_EINVAL, "null config");
  if (c->n_layers < 1 || c->dim < 64 || c->dim % 64 || c->dim > 4096 || c->n_heads < 1 ||
      c->n_kv_heads < 1 || c->n_heads % c->n_kv_heads || c->dim / c->n_heads != kHd ||
      c->dim % c->n_heads || c->ffn_hidden < 64 || c->ffn_hidden % 64 || c->vocab < 1 ||
      c->max_seq < 1 || c->max_seq > kMaxSeqBody || c->max_tokens < 1 ||
      c->max_tokens > (1 << 22) || !(c->rms_eps > 0.f) || !(c->rope_theta > 0.f))
    return bfail(LORA_CE_EINVAL, "bad body configuration (head_dim must be 64)");
  BD_CUDA(cudaSetDevice(c->device));
  lora_body_handle* h = new (std::nothrow) lora_body_handle();
  if (!h) return bfail(LORA_CE_ENOMEM, "host allocation failed");
  h->cfg = *c;
  h->d = c->dim;
  h->ffn = c->ffn_hidden;
  h->kvdim = c->n_kv_heads * kHd;
  h->nqkv = h->d + 2 * h->kvdim;
  h->Tcap = c->max_tokens;
  h->layers.resize(c->n_layers);
  if (cudaDeviceGetAttribute(&h->num_sms, cudaDevAttrMultiProcessorCount, c->device) !=
      cudaSuccess) {
    delete h;
    return bfail(LORA_CE_ECUDA, "cudaDeviceGetAttribute failed");
  }
  {
    const char* e = getenv("LORA_BODY_GRAPHS");  // "0": launch the kernels directly
    h->use_graph = !(e && e[0] == '0');
  }
  const size_t T = (size_t)h->Tcap, d = h->d, ffn = h->ffn, wide = std::max(d, ffn);
  int rc = 0;
  if (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess)
    rc = bfail(LORA_CE_ECUDA, "cudaStreamCreate failed");
  for (auto& L : h->layers) {
    if (!rc) rc = balloc(&L.wqkv, (size_t)h->nqkv * d);
    if (!rc) rc = balloc(&L.sqkv, (size_t)h->nqkv);
    if (!rc) rc = balloc(&L.wo, d * d);
    if (!rc) rc = balloc(&L.so, d);
    if (!rc) rc = balloc(&L.wgu, 2 * ffn * d);
    if (!rc) rc = balloc(&L.sgu, 2 * ffn);
    if (!rc) rc = balloc(&L.wd, d * ffn);
    if (!rc) rc = balloc(&L.sd, d);
    if (!rc) rc = balloc(&L.attn_norm, d);
    if (!rc) rc = balloc(&L.ffn_norm, d);
  }
  if (!rc) rc = balloc(&h->embd, (size_t)c->vocab * d);
  if (!rc) rc = balloc(&h->out_norm, d);
  if (!rc) rc = balloc(&h->rope_cos, (size_t)c->max_seq * (kHd / 2));
  if (!rc) rc = balloc(&h->rope_sin, (size_t)c->max_seq * (kHd / 2));
  if (!rc) rc = balloc(&h->x, T * d);
  if (!rc) rc = balloc(&h->xn, T * wide);
  if (!rc) rc = balloc(&h->xq, T * wide);
  if (!rc) rc = balloc(&h->xs, T);
  if (!rc) rc = balloc(&h->qkv, T * h->nqkv);
  if (!rc) rc = balloc(&h->att, T * d);
  if (!rc) rc = balloc(&h->gu, T * 2 * ffn);
  if (!rc) rc = balloc(&h->pos, T);
  if (!rc) rc = balloc(&h->tok, T);
  if (!rc) rc = balloc(&h->hout, T * d);
  if (!rc) rc = balloc(&h->err, 1);
  if (!rc) rc = balloc(&h->tgt, T);
  if (!rc) rc = balloc(&h->loss, 2);
  if (!rc && cudaMallocHost(reinterpret_cast<void**>(&h->pos_host), T * 4) != cudaSuccess) {
    h->pos_host = nullptr;
    rc = bfail(LORA_CE_ENOMEM, "cudaMallocHost failed");
  }
  if (!rc && cudaMemset(h->err, 0, 4) != cudaSuccess) rc = bfail(LORA_CE_ECUDA, "cudaMemset failed");
  if (!rc) {
    // stage a whole tile's key range up to a 200 KB block (the usual case:
    // max_seq 256 needs 263 rows, 143 KB); longer ranges read global memory
    const long long want = kAttnTile + (long long)c->max_seq - 1;
    const long long fit =
        (200LL * 1024 - (long long)kAttnTWarps * c->max_seq * 4) / (2LL * kAttnRowF * 4);
    h->attn_cap = (int)std::max<long long>(0, std::min(want, fit));
    if (cudaFuncSetAttribute(bd_attn_tile, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)attn_tile_smem(c->max_seq, h->attn_cap)) != cudaSuccess)
      rc = bfail(LORA_CE_ECUDA, "attention shared memory");
  }
  if (!rc && cudaFuncSetAttribute(bd_norm, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)(kNormWarps * c->dim * sizeof(double))) != cudaSuccess)
    rc = bfail(LORA_CE_ECUDA, "norm shared memory");
  if (!rc) {
    // RoPE tables exactly as forward_load builds them (src/forward.c:889-899)
    const int half = kHd / 2;
    std::vector<float> cs((size_t)c->max_seq * half), sn(cs.size());
    for (int p = 0; p < c->max_seq; ++p)
      for (int i = 0; i < half; ++i) {
        const float freq = 1.0f / powf(c->rope_theta, (2.0f * (float)i) / (float)kHd);
        const float angle = (float)p * freq;
        cs[(size_t)p * half + i] = cosf(angle);
        sn[(size_t)p * half + i] = sinf(angle);
      }
    if (cudaMemcpy(h->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(h->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
      rc = bfail(LORA_CE_ECUDA, "RoPE table upload failed");
  }
  if (rc) {
    free_body(h);
    delete h;
    return rc;
  }
  *out = h;
  return 0;
}

int lora_body_destroy(lora_body_handle* h) {
  if (!h) return 0;
  cudaSetDevice(h->cfg.device);
  if (h->stream) cudaStreamSynchronize(h->stream);
  free_body(h);
  delete h;
  return 0;
}

int lora_body_set_embedding(lora_body_handle* h, const uint16_t* token_embd,
                            const float* output_norm) {
  if (!h || !token_embd || !output_norm) return bfail(LORA_CE_EINVAL, "null argument");
  BD_CUDA(cudaSetDevice(h->cfg.device));
  BD_CUDA(cudaMemcpyAsync(h->embd, token_embd, (size_t)h->cfg.vocab * h->d * 2,
                          cudaMemcpyHostToDevice, h->stream));
  BD_CUDA(cudaMemcpyAsync(h->out_norm, output_norm, (size_t)h->d * 4, cudaMemcpyHostToDevice,
                          h->stream));
  BD_CUDA(cudaStreamSynchronize(h->stream));
  h->have_embd = true;
  return 0;
}

int lora_body_set_layer(lora_body_handle* h, int32_t layer, const float* attn_norm,
                        const uint16_t* wq, const uint16_t* wk, const uint16_t* wv,
                        const uint16_t* wo, const float* ffn_norm, const uint16_t* w_gate,
                        const uint16_t* w_up, const uint16_t* w_down) {
  if (!h || layer < 0 || layer >= h->cfg.n_layers || !attn_norm || !wq || !wk || !wv || !wo ||
      !ffn_norm || !w_gate || !w_up || !w_down)
    return bfail(LORA_CE_EINVAL, "bad argument");
  BD_CUDA(cudaSetDevice(h->cfg.device));
  auto& L = h->layers[layer];
  const int d = h->d, ffn = h->ffn, kv = h->kvdim;
  __half* tmp = nullptr;
  if (cudaMalloc(&tmp, (size_t)std::max(ffn, d) * d * 2) != cudaSuccess) {
    cudaGetLastError();
    return bfail(LORA_CE_ENOMEM, "cudaMalloc failed");
  }
  int rc = 0;
  // each upload waits for the previous quantisation (same stream) before
  // the staging buffer is overwritten
  if (!rc) rc = upload_quant(h, wq, d, d, L.wqkv, L.sqkv, tmp);
  if (!rc) rc = upload_quant(h, wk, kv, d, L.wqkv + (size_t)d * d, L.sqkv + d, tmp);
  if (!rc) rc = upload_quant(h, wv, kv, d, L.wqkv + (size_t)(d + kv) * d, L.sqkv + d + kv, tmp);
  if (!rc) rc = upload_quant(h, wo, d, d, L.wo, L.so, tmp);
  if (!rc) rc = upload_quant(h, w_gate, ffn, d, L.wgu, L.sgu, tmp);
  if (!rc) rc = upload_quant(h, w_up, ffn, d, L.wgu + (size_t)ffn * d, L.sgu + ffn, tmp);
  if (!rc) rc = upload_quant(h, w_down, d, ffn, L.wd, L.sd, tmp);
  if (!rc && (cudaMemcpyAsync(L.attn_norm, attn_norm, (size_t)d * 4, cudaMemcpyHostToDevice,
                              h->stream) != cudaSuccess ||
              cudaMemcpyAsync(L.ffn_norm, ffn_norm, (size_t)d * 4, cudaMemcpyHostToDevice,
                              h->stream) != cudaSuccess))
    rc = bfail(LORA_CE_ECUDA, "norm upload failed");
  if (cudaStreamSynchronize(h->stream) != cudaSuccess && !rc)
    rc = bfail(LORA_CE_ECUDA, "layer upload failed");
  cudaFree(tmp);
  if (!rc) L.set = true;
  return rc;
}

int lora_body_set_window(lora_body_handle* h, int32_t layer, int32_t window) {
  if (!h || layer < 0 || layer >= h->cfg.n_layers || window < 0)
    return bfail(LORA_CE_EINVAL, "bad argument");
  if (h->layers[layer].window != window) drop_body_graph(h);  // captured with the old one
  h->layers[layer].window = window;
  return 0;
}

static int ready(lora_body_handle* h) {
  if (!h) return bfail(LORA_CE_EINVAL, "null handle");
  if (!h->have_embd) return bfail(LORA_CE_ESTATE, "lora_body_set_embedding not called");
  for (const auto& L : h->layers)
    if (!L.set) return bfail(LORA_CE_ESTATE, "a layer has no weights (lora_body_set_layer)");
  return 0;
}

int lora_body_hidden(lora_body_handle* h, const int32_t* tokens, const int32_t* offsets,
                     int32_t n_seqs, float* H_out) {
  int rc = ready(h);
  if (rc) return rc;
  if (!tokens || !H_out) return bfail(LORA_CE_EINVAL, "null argument");
  int T = 0;
  if ((rc = check_offsets(h, offsets, n_seqs, &T))) return rc;
  for (int t = 0; t < T; ++t)
    if (tokens[t] < 0 || tokens[t] >= h->cfg.vocab) return bfail(LORA_CE_EINVAL, "token id out of range");
  BD_CUDA(cudaSetDevice(h->cfg.device));
  BD_CUDA(cudaMemcpyAsync(h->tok, tokens, (size_t)T * 4, cudaMemcpyHostToDevice, h->stream));
  if ((rc = run_body(h, h->tok, offsets, n_seqs, T, h->hout, LORA_CE_F32))) return rc;
  BD_CUDA(cudaMemcpyAsync(H_out, h->hout, (size_t)T * h->d * 4, cudaMemcpyDeviceToHost, h->stream));
  return body_check_error(h);
}

int lora_body_hidden_device(lora_body_handle* h, const int32_t* d_tokens, const int32_t* offsets,
                            int32_t n_seqs, void* d_H, int32_t h_dtype) {
  int rc = ready(h);
  if (rc) return rc;
  if (!d_tokens || !d_H) return bfail(LORA_CE_EINVAL, "null argument");
  if (h_dtype < LORA_CE_BF16 || h_dtype > LORA_CE_F32) return bfail(LORA_CE_EINVAL, "bad dtype");
  if ((reinterpret_cast<uintptr_t>(d_H) & 15) != 0)
    return bfail(LORA_CE_EINVAL, "d_H must be 16-byte aligned");
  int T = 0;
  if ((rc = check_offsets(h, offsets, n_seqs, &T))) return rc;
  BD_CUDA(cudaSetDevice(h->cfg.device));
  // the previous call's positions may still be in flight from pos_host
  BD_CUDA(cudaStreamSynchronize(h->stream));
  return run_body(h, d_tokens, offsets, n_seqs, T, d_H, h_dtype);
}

int lora_body_train_step(lora_body_handle* h, lora_ce_handle* ce, const int32_t* tokens,
                         const int32_t* offsets, int32_t n_seqs, const int32_t* targets,
                         float* loss_out) {
  int rc = ready(h);
  if (rc) return rc;
  if (!ce || !tokens || !targets || !loss_out) return bfail(LORA_CE_EINVAL, "null argument");
  int T = 0;
  if ((rc = check_offsets(h, offsets, n_seqs, &T))) return rc;
  for (int t = 0; t < T; ++t)
    if (tokens[t] < 0 || tokens[t] >= h->cfg.vocab || targets[t] < 0 ||
        targets[t] >= h->cfg.vocab)
      return bfail(LORA_CE_EINVAL, "token or target id out of range");
  BD_CUDA(cudaSetDevice(h->cfg.device));
  BD_CUDA(cudaMemcpyAsync(h->tok, tokens, (size_t)T * 4, cudaMemcpyHostToDevice, h->stream));
  BD_CUDA(cudaMemcpyAsync(h->tgt, targets, (size_t)T * 4, cudaMemcpyHostToDevice, h->stream));
  if ((rc = run_body(h, h->tok, offsets, n_seqs, T, h->hout, LORA_CE_F32))) return rc;
  if ((rc = body_check_error(h))) return rc;  // waits: the step's inputs are ready
  rc = lora_ce_step_device(ce, h->hout, LORA_CE_F32, T, h->tgt, h->loss);
  if (!rc) rc = lora_ce_sync(ce);
  if (rc) return bfail(rc, std::string("lora_ce step: ") + lora_ce_last_error());
  BD_CUDA(cudaMemcpy(loss_out, h->loss, 4, cudaMemcpyDeviceToHost));
  return 0;
}

int lora_body_sync(lora_body_handle* h) {
  if (!h) return bfail(LORA_CE_EINVAL, "null handle");
  BD_CUDA(cudaSetDevice(h->cfg.device));
  return body_check_error(h);
}

void* lora_body_stream(lora_body_handle* h) { return h ? (void*)h->stream : nullptr; }

}  // extern "C"
