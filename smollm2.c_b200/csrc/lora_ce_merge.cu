// lora_ce_merge.cu — LoRA merge into the tied lm_head:
//   W'[v][i] = f16trunc(f32(W[v][i]) + scale * sum_k A[i][k] * B[k][v])
// with the reference's exact arithmetic (src/train.c:393-460): the rank sum
// in k order with separately rounded multiplies and adds, the merge path's
// own f16 -> f32 conversion (which halves f16 subnormals and maps exponent
// 31 to 2^16 * 1.f) and its f32 -> f16 conversion (below).  HBM-bound:
// 2 bytes read + 2 bytes written per weight.
#include <cuda_runtime.h>

#include <algorithm>
#include <string>

#include "lora_ce.h"

namespace {

thread_local std::string g_merge_error;

int merge_fail(int code, const char* msg) {
  g_merge_error = msg;
  return code;
}

// The merge path's f32 -> f16 conversion, as the reference writes it
// (src/train.c:392-407).  Its normal-range branch adds 0x0C800000 (not the
// 0xC8000000 that rebiases the exponent) and its subnormal branch shifts the
// 24-bit mantissa by too little, so both intermediate results exceed 16 bits
// and the reference's (uint16_t) cast keeps the low 16.  The & 0xffff here is
// that cast; without it the extra bits would spill into the neighbouring
// packed half-word.
__device__ __forceinline__ uint32_t merge_f32_to_f16_bits(float f) {
  const uint32_t x = __float_as_uint(f);
  const uint32_t sign = (x & 0x80000000u) >> 16;
  const uint32_t em = x & 0x7fffffffu;
  if (em >= 0x47800000u) return sign | (em > 0x7f800000u ? 0x7e00u : 0x7c00u);
  if (em < 0x38800000u) {
    if (em < 0x33000000u) return sign;
    const uint32_t sh = 113u - (em >> 23);
    const uint32_t mant = (em & 0x7fffffu) | 0x800000u;
    return (sign | (mant >> sh)) & 0xffffu;
  }
  return (sign | ((em + 0xc800000u) >> 13)) & 0xffffu;
}

// Tiled merge.  A CTA owns column tile blockIdx.y (CT = 8 * blockDim.x
// columns) and walks row tiles of VT = kRB * blockDim.y rows.  Thread
// (tx, ty) accumulates rows v0 + ty*kRB + j, columns col0 + tx*8 + e, one
// separately rounded multiply and add per k in ascending k (the reference's
// order), then merges 8 weights per row with 16-byte accesses.
//   A_s[kk][h][c*4 + q] = A[col0 + c*8 + 4h + q][k0 + kk]  (h = 0, 1)
//   B_s[kk][j]          = B[k0 + kk][v0 + j]
// Resident form (kResident): A^T for the whole rank stays in shared memory;
// the next tile's B and W are copied into the other half of double-buffered
// B_s / W_s by cp.async while this tile computes, so a tile costs one
// barrier and no exposed load latency.  Each thread copies and later reads
// its own W segments; B_s is read by all, after the barrier.
//   W_s[buf][j][c*8 .. c*8+7] = W[v0 + j][col0 + c*8 ..]  Chunked form: k chunks of KC staged per tile (large
// ranks, where the arithmetic dominates).
constexpr int kRB = 4;
constexpr int kBPer = 4;  // B values of a tile per thread at most (resident form)

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// The rank sum uses scalar __fmul_rn / __fadd_rn: a paired f32x2 multiply
// feeding a paired add comes out FMA-rounded on sm_100a even when both carry
// an explicit .rn (measured: on random workload-scaled inputs every one of
// the 1.41 M of 8.39 M results where the separately rounded and the fused
// results differ took the fused value), and the reference rounds the
// product and the sum separately.

// The merge path's f16 -> f32 conversion (src/train.c:433-454): exact for
// exponent 1..30, exponent 31 (inf / NaN) becomes 2^16 * 1.f, and a
// subnormal mant * 2^-24 becomes mant * 2^-25 (its normalisation loop starts
// from exponent 0).  Written without a branch: for exponent 1..31,
// ((h & 0x7fff) << 13) + (112 << 23) is (exp + 112) << 23 | mant << 13 (no
// carry: exp + 112 <= 143).  For exponent 0 the same bits are
// 2^-15 * (1 + mant * 2^-10) = 2^-15 + mant * 2^-25, so subtracting 2^-15
// (exact: the difference is representable) leaves mant * 2^-25, which is
// what the merge path's conversion yields there (+0 for mant 0).  The sign
// is applied last, so -0 stays -0.
__device__ __forceinline__ float merge_in(uint32_t h) {
  const float fa = __uint_as_float(((h & 0x7fffu) << 13) + 0x38000000u);
  const float a = (h & 0x7c00u) ? fa : __fsub_rn(fa, 3.0517578125e-05f /* 2^-15 */);
  return __uint_as_float(__float_as_uint(a) | ((h & 0x8000u) << 16));
}

// merge_f32_to_f16_bits with the range tests ordered for the common case.
__device__ __forceinline__ uint32_t merge_out(float f) {
  const uint32_t x = __float_as_uint(f);
  const uint32_t em = x & 0x7fffffffu;
  if (__builtin_expect(em - 0x38800000u < 0x0f000000u, 1))
    return (((x >> 16) & 0x8000u) | ((em + 0xc800000u) >> 13)) & 0xffffu;
  return merge_f32_to_f16_bits(f);
}

__device__ __forceinline__ uint32_t merge_one(uint32_t hb, float s, float scale) {
  return merge_out(__fadd_rn(merge_in(hb), __fmul_rn(scale, s)));
}

template <bool kResident>
__global__ void __launch_bounds__(512) lce_merge(const uint16_t* __restrict__ W,
                                                 const float* __restrict__ A,
                                                 const float* __restrict__ B, int d, int R, int V,
                                                 float scale, int KC, uint16_t* __restrict__ out) {
  extern __shared__ float4 merge_smem4[];
  float* smem = reinterpret_cast<float*>(merge_smem4);
  const int CG = blockDim.x, CT = CG * 8, VT = kRB * blockDim.y;
  const int tx = threadIdx.x, ty = threadIdx.y, tid = ty * CG + tx, nthr = CG * blockDim.y;
  const int col0 = blockIdx.y * CT;
  const int ncol = min(CT, d - col0);
  float* A_s = smem;             // [KC][CT]
  float* B_s = smem + KC * CT;   // [2][KC][VT] resident, [KC][VT] chunked
  const bool col_ok = tx * 8 < ncol;
  const int ntiles = (V + VT - 1) / VT;

  auto stage_A = [&](int k0, int kc) {
    for (int t = tid; t < ncol * kc; t += nthr) {
      const int i = t / kc, kk = t - i * kc;
      const int c = i >> 3, h = (i >> 2) & 1, q = i & 3;
      A_s[kk * CT + h * (CT / 2) + c * 4 + q] = A[(long long)(col0 + i) * R + k0 + kk];
    }
  };
  auto load_w = [&](int tile, uint4 (&wv)[kRB]) {
#pragma unroll
    for (int j = 0; j < kRB; ++j) {
      const int v = tile * VT + ty * kRB + j;
      wv[j] = (col_ok && v < V)
                  ? *reinterpret_cast<const uint4*>(W + (long long)v * d + col0 + tx * 8)
                  : make_uint4(0, 0, 0, 0);
    }
  };
  auto compute = [&](const float* Bt, int kc, float (&acc)[kRB][8], int astride) {
    for (int kk = 0; kk < kc; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(A_s + kk * astride + tx * 4);
      const float4 a1 = *reinterpret_cast<const float4*>(A_s + kk * astride + CT / 2 + tx * 4);
      const float4 b = *reinterpret_cast<const float4*>(Bt + kk * VT + ty * kRB);
      const float bj[kRB] = {b.x, b.y, b.z, b.w};
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
      for (int j = 0; j < kRB; ++j)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[j][e] = __fadd_rn(acc[j][e], __fmul_rn(av[e], bj[j]));
    }
  };
  auto epilogue = [&](int tile, const uint4 (&wv)[kRB], const float (&acc)[kRB][8]) {
    if (!col_ok) return;
#pragma unroll
    for (int j = 0; j < kRB; ++j) {
      const int v = tile * VT + ty * kRB + j;
      if (v >= V) continue;
      const uint32_t w32[4] = {wv[j].x, wv[j].y, wv[j].z, wv[j].w};
      uint32_t o32[4];
#pragma unroll
      for (int p = 0; p < 4; ++p)
        o32[p] = merge_one(w32[p] & 0xffffu, acc[j][2 * p], scale) |
                 (merge_one(w32[p] >> 16, acc[j][2 * p + 1], scale) << 16);
      *reinterpret_cast<uint4*>(out + (long long)v * d + col0 + tx * 8) =
          make_uint4(o32[0], o32[1], o32[2], o32[3]);
    }
  };

  int tile = blockIdx.x;
  if constexpr (kResident) {
    // KC == R, R * VT <= kBPer * nthr (checked by the launcher)
    const int nb = R * VT;
    uint16_t* W_s = reinterpret_cast<uint16_t*>(B_s + 2 * nb);  // [2][VT][CT]
    // this thread's B copies: element t = tid + q*nthr of a tile, at
    // B[kk][v0 + j] with t = kk*VT + j (tile independent apart from v0)
    int b_kk[kBPer], b_j[kBPer];
#pragma unroll
    for (int q = 0; q < kBPer; ++q) {
      const int t = tid + q * nthr;
      b_kk[q] = t < nb ? t / VT : -1;
      b_j[q] = t < nb ? t - (t / VT) * VT : 0;
    }
    auto issue = [&](int t_, int b_) {
#pragma unroll
      for (int j = 0; j < kRB; ++j) {
        const int row = ty * kRB + j, v = t_ * VT + row;
        if (col_ok && v < V)
          cp_async16(W_s + ((size_t)b_ * VT + row) * CT + tx * 8, W + (long long)v * d + col0 + tx * 8);
      }
#pragma unroll
      for (int q = 0; q < kBPer; ++q) {
        if (b_kk[q] >= 0) {
          const int v = t_ * VT + b_j[q];
          float* dst = B_s + b_ * nb + tid + q * nthr;
          if (v < V) cp_async4(dst, B + (long long)b_kk[q] * V + v);
          else *dst = 0.0f;
        }
      }
      cp_async_commit();
    };
    stage_A(0, R);
    issue(tile, 0);
    int buf = 0;
    for (; tile < ntiles; tile += gridDim.x) {
      cp_async_wait_all();
      __syncthreads();  // this tile's B_s visible; the other buffers no longer read
      const int nt = tile + gridDim.x;
      if (nt < ntiles) issue(nt, buf ^ 1);
      float acc[kRB][8];
#pragma unroll
      for (int j = 0; j < kRB; ++j)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[j][e] = 0.0f;
      compute(B_s + buf * nb, R, acc, CT);
      uint4 wv[kRB];
#pragma unroll
      for (int j = 0; j < kRB; ++j)
        wv[j] = *reinterpret_cast<const uint4*>(W_s + ((size_t)buf * VT + ty * kRB + j) * CT + tx * 8);
      epilogue(tile, wv, acc);
      buf ^= 1;
    }
  } else {
    for (; tile < ntiles; tile += gridDim.x) {
      uint4 wv[kRB];
      load_w(tile, wv);
      const int v0 = tile * VT;
      float acc[kRB][8];
#pragma unroll
      for (int j = 0; j < kRB; ++j)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[j][e] = 0.0f;
      for (int k0 = 0; k0 < R; k0 += KC) {
        const int kc = min(KC, R - k0);
        __syncthreads();  // previous readers of A_s / B_s are done
        stage_A(k0, kc);
        for (int t = tid; t < kc * VT; t += nthr) {
          const int kk = t / VT, j = t - kk * VT;
          B_s[t] = (v0 + j < V) ? B[(long long)(k0 + kk) * V + v0 + j] : 0.0f;
        }
        __syncthreads();
        compute(B_s, kc, acc, CT);
      }
      epilogue(tile, wv, acc);
    }
  }
}

int check_merge_args(const void* W, const void* A, const void* B, int dim, int rank, int vocab,
                     const void* out) {
  if (!W || !A || !B || !out) return merge_fail(LORA_CE_EINVAL, "null pointer");
  if (dim < 8 || dim % 8 != 0) return merge_fail(LORA_CE_EINVAL, "dim must be a multiple of 8");
  if (rank < 1 || rank > 256) return merge_fail(LORA_CE_EINVAL, "rank must be in [1, 256]");
  if (vocab < 1) return merge_fail(LORA_CE_EINVAL, "vocab must be positive");
  return 0;
}

}  // namespace

extern "C" int lora_ce_merge_weight_device(const uint16_t* d_W, const float* d_A,
                                           const float* d_B, int32_t dim, int32_t rank,
                                           int32_t vocab, float scale, uint16_t* d_out,
                                           void* stream) {
  int rc = check_merge_args(d_W, d_A, d_B, dim, rank, vocab, d_out);
  if (rc) return rc;
  if (((reinterpret_cast<uintptr_t>(d_W) | reinterpret_cast<uintptr_t>(d_out)) & 15) != 0)
    return merge_fail(LORA_CE_EINVAL, "W and out must be 16-byte aligned");
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // column groups of 8 per CTA (a whole row up to d = 1024), row sub-tiles so
  // that a CTA has 256..512 threads
  const int groups = dim / 8;
  const int CG = std::min(groups, 128);
  const int RS = std::max(1, std::min(512 / CG, (256 + CG - 1) / CG));
  const int CT = CG * 8, VT = kRB * RS;
  // Resident form when A^T for the whole rank, two B tiles and two W tiles
  // fit in 220 KB (rank 64 at d = 576: 191 KB) and a tile's B is at most
  // kBPer values per thread; otherwise k chunks of about 64 KB.
  const int nthr = CG * RS;
  const size_t res_smem = (size_t)rank * (CT + 2 * VT) * sizeof(float) + (size_t)2 * VT * CT * 2;
  const bool resident = res_smem <= 220u * 1024u && rank * VT <= kBPer * nthr;
  const size_t per_k = (size_t)(CT + VT) * sizeof(float);
  const int KC = resident ? rank : std::max(1, std::min(rank, (int)((64u * 1024u) / per_k)));
  const size_t smem = resident ? res_smem : (size_t)KC * per_k;
  auto kern = resident ? lce_merge<true> : lce_merge<false>;
  static thread_local int s_optin_dev = -1;
  if (s_optin_dev != dev) {
    if (cudaFuncSetAttribute(lce_merge<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             227 * 1024) != cudaSuccess ||
        cudaFuncSetAttribute(lce_merge<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             227 * 1024) != cudaSuccess)
      return merge_fail(LORA_CE_ECUDA, "cudaFuncSetAttribute failed");
    s_optin_dev = dev;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, nthr, smem) != cudaSuccess ||
      per_sm < 1)
    return merge_fail(LORA_CE_ECUDA, "merge kernel does not fit on the device");
  const int ntiles = (vocab + VT - 1) / VT;
  const dim3 grid((unsigned)std::min(ntiles, per_sm * sms), (unsigned)((groups + CG - 1) / CG));
  kern<<<grid, dim3(CG, RS), smem, reinterpret_cast<cudaStream_t>(stream)>>>(
      d_W, d_A, d_B, dim, rank, vocab, scale, KC, d_out);
  if (cudaGetLastError() != cudaSuccess) return merge_fail(LORA_CE_ECUDA, "merge launch failed");
  return 0;
}

extern "C" int lora_ce_merge_weight(const uint16_t* W, const float* A, const float* B,
                                    int32_t dim, int32_t rank, int32_t vocab, float scale,
                                    uint16_t* out, int32_t device) {
  int rc = check_merge_args(W, A, B, dim, rank, vocab, out);
  if (rc) return rc;
  if (cudaSetDevice(device) != cudaSuccess) return merge_fail(LORA_CE_ECUDA, "cudaSetDevice failed");
  const size_t nw = (size_t)vocab * dim * 2, na = (size_t)dim * rank * 4, nb = (size_t)rank * vocab * 4;
  void *dW = nullptr, *dA = nullptr, *dB = nullptr, *dO = nullptr;
  rc = 0;
  if (cudaMalloc(&dW, nw) != cudaSuccess || cudaMalloc(&dA, na) != cudaSuccess ||
      cudaMalloc(&dB, nb) != cudaSuccess || cudaMalloc(&dO, nw) != cudaSuccess)
    rc = merge_fail(LORA_CE_ENOMEM, "cudaMalloc failed");
  if (!rc && (cudaMemcpy(dW, W, nw, cudaMemcpyHostToDevice) != cudaSuccess ||
              cudaMemcpy(dA, A, na, cudaMemcpyHostToDevice) != cudaSuccess ||
              cudaMemcpy(dB, B, nb, cudaMemcpyHostToDevice) != cudaSuccess))
    rc = merge_fail(LORA_CE_ECUDA, "upload failed");
  if (!rc)
    rc = lora_ce_merge_weight_device((const uint16_t*)dW, (const float*)dA, (const float*)dB, dim,
                                     rank, vocab, scale, (uint16_t*)dO, nullptr);
  if (!rc && cudaMemcpy(out, dO, nw, cudaMemcpyDeviceToHost) != cudaSuccess)
    rc = merge_fail(LORA_CE_ECUDA, "download failed");
  cudaFree(dW);
  cudaFree(dA);
  cudaFree(dB);
  cudaFree(dO);
  return rc;
}

extern "C" const char* lora_ce_merge_last_error(void) { return g_merge_error.c_str(); }
