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

__device__ __forceinline__ float merge_f16_bits_to_f32(uint32_t h) {
  const uint32_t sign = (h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1fu;
  const uint32_t mant = h & 0x3ffu;
  if (exp == 0) {
    const float f = mant ? __fmul_rn((float)mant, 2.98023223876953125e-8f /* 2^-25 */) : 0.0f;
    return __uint_as_float(__float_as_uint(f) | sign);
  }
  return __uint_as_float(sign | ((exp + 112u) << 23) | (mant << 13));
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
// columns) and walks row tiles of VT = kRB * blockDim.y rows.  A^T for the
// tile's columns is staged in shared memory in k chunks of KC (once per CTA
// when the whole rank fits, KC == R), B[k0..k0+KC)[v0..v0+VT) per row tile.
// Thread (tx, ty) accumulates rows v0 + ty*kRB + j, columns col0 + tx*8 + e,
// one separately rounded multiply and add per k in ascending k
// (the reference's order), then merges 8 weights per row with 16-byte
// accesses; its W values are loaded before the k loop so the HBM reads
// overlap the arithmetic.
//   A_s[kk][h][c*4 + q] = A[col0 + c*8 + 4h + q][k0 + kk]  (h = 0, 1)
//   B_s[kk][j]          = B[k0 + kk][v0 + j]
constexpr int kRB = 4;

// The rank sum uses scalar __fmul_rn / __fadd_rn: a paired f32x2 multiply
// feeding a paired add comes out FMA-rounded on sm_100a even when both carry
// an explicit .rn (measured: on random workload-scaled inputs every one of
// the 1.41 M of 8.39 M results where the separately rounded and the fused
// results differ took the fused value), and the reference rounds the
// product and the sum separately.

__device__ __forceinline__ uint32_t merge_one(uint32_t hb, float s, float scale) {
  return merge_f32_to_f16_bits(__fadd_rn(merge_f16_bits_to_f32(hb), __fmul_rn(scale, s)));
}

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
  float* B_s = smem + KC * CT;   // [KC][VT]
  const bool single = KC >= R;
  const bool col_ok = tx * 8 < ncol;
  auto stage_A = [&](int k0, int kc) {
    for (int t = tid; t < ncol * kc; t += nthr) {
      const int i = t / kc, kk = t - i * kc;
      const int c = i >> 3, h = (i >> 2) & 1, q = i & 3;
      A_s[kk * CT + h * (CT / 2) + c * 4 + q] = A[(long long)(col0 + i) * R + k0 + kk];
    }
  };
  if (single) {
    stage_A(0, R);
  }
  const int ntiles = (V + VT - 1) / VT;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int v0 = tile * VT;
    uint4 wv[kRB];
#pragma unroll
    for (int j = 0; j < kRB; ++j) {
      const int v = v0 + ty * kRB + j;
      wv[j] = (col_ok && v < V)
                  ? *reinterpret_cast<const uint4*>(W + (long long)v * d + col0 + tx * 8)
                  : make_uint4(0, 0, 0, 0);
    }
    float acc[kRB][8];
#pragma unroll
    for (int j = 0; j < kRB; ++j)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[j][e] = 0.0f;
    for (int k0 = 0; k0 < R; k0 += KC) {
      const int kc = min(KC, R - k0);
      __syncthreads();  // previous readers of A_s / B_s are done
      if (!single) stage_A(k0, kc);
      for (int t = tid; t < kc * VT; t += nthr) {
        const int kk = t / VT, j = t - kk * VT;
        B_s[kk * VT + j] = (v0 + j < V) ? B[(long long)(k0 + kk) * V + v0 + j] : 0.0f;
      }
      __syncthreads();
      for (int kk = 0; kk < kc; ++kk) {
        const float4 a0 = *reinterpret_cast<const float4*>(A_s + kk * CT + tx * 4);
        const float4 a1 = *reinterpret_cast<const float4*>(A_s + kk * CT + CT / 2 + tx * 4);
        const float4 b = *reinterpret_cast<const float4*>(B_s + kk * VT + ty * kRB);
        const float bj[kRB] = {b.x, b.y, b.z, b.w};
        const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
        for (int j = 0; j < kRB; ++j)
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[j][e] = __fadd_rn(acc[j][e], __fmul_rn(av[e], bj[j]));
      }
    }
    if (col_ok) {
#pragma unroll
      for (int j = 0; j < kRB; ++j) {
        const int v = v0 + ty * kRB + j;
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
  // the whole rank staged once per CTA when A^T for the column tile fits in
  // 200 KB (rank 64 at d = 576 takes 147 KB); otherwise 64 KB k chunks
  const size_t per_k = (size_t)(CT + VT) * sizeof(float);
  const int KC = (size_t)rank * per_k <= 200u * 1024u
                     ? rank
                     : std::max(1, (int)((64u * 1024u) / per_k));
  const size_t smem = (size_t)KC * per_k;
  static thread_local int s_optin_dev = -1;
  if (s_optin_dev != dev) {
    if (cudaFuncSetAttribute(lce_merge, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) !=
        cudaSuccess)
      return merge_fail(LORA_CE_ECUDA, "cudaFuncSetAttribute failed");
    s_optin_dev = dev;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, lce_merge, CG * RS, smem) !=
          cudaSuccess || per_sm < 1)
    return merge_fail(LORA_CE_ECUDA, "merge kernel does not fit on the device");
  const int ntiles = (vocab + VT - 1) / VT;
  const dim3 grid((unsigned)std::min(ntiles, per_sm * sms), (unsigned)((groups + CG - 1) / CG));
  lce_merge<<<grid, dim3(CG, RS), smem, reinterpret_cast<cudaStream_t>(stream)>>>(
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
