// lora_ce_q4k.cu — Q4_K (GGUF / ggml type 12) dequantisation for the QLoRA
// lm_head: 144-byte super-blocks of 256 weights over the flattened [V][d]
// tensor, f16 d, f16 dmin, twelve bytes of 6-bit (scale, min) pairs for the
// eight 32-weight sub-blocks and 128 bytes of 4-bit quants.
//   y = (d * sc) * q - (dmin * m), each product and the difference rounded
//   separately (ggml's scalar order without contraction)
// HBM-bound: 144 bytes in and 512 (f16) or 1024 (f32) bytes out per block.
// Lane l of a block's warp produces weights 8l .. 8l+7 (run c = l / 8 of
// 64, low nibbles for the first 32 of a run, high nibbles for the second)
// from one 8-byte quant load and the block's 16-byte header, which all
// lanes read (a broadcast), and writes them with 16- or 32-byte stores.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <string>

#include "lora_ce.h"

namespace {

thread_local std::string g_q4k_error;

int q4k_fail(int code, const char* msg) {
  g_q4k_error = msg;
  return code;
}

// One warp per block; lane l makes weights 8l .. 8l+7 of the block.
// * Decoding: each quant nibble q becomes the f32 with bits 0x4B0000qq,
//   2^23 + q, by one byte permute, and subtracting 2^23 is exact. The
//   6-bit (scale, min) pair of sub-block j comes from the three 32-bit
//   words of scales[] with one shift by 8 * (j % 4).
// * Arithmetic: (d * sc) * q - dmin * m, each step rounded separately, as
//   written above.
template <bool kF16>
__global__ void __launch_bounds__(256) lce_q4k_dequant(const uint8_t* __restrict__ blocks,
                                                        long long n_blocks, void* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  const int c = lane >> 3;          // run of 64
  const int hi = (lane >> 2) & 1;   // high nibbles: second 32 of the run
  const int o = (lane & 3) * 8;     // offset in the run's 32 quant bytes
  const int j = 2 * c + hi;         // sub-block
  const int sh = 8 * (j & 3);
  auto decode = [&](long long b, const uint4& hdr, const uint2& qv) {
    const uint32_t s0 = hdr.y >> sh, s1 = hdr.z >> sh, s2 = hdr.w >> sh;  // scales[k], [k+4], [k+8]
    uint32_t sc, m;
    if (j < 4) {
      sc = s0 & 63u;
      m = s1 & 63u;
    } else {
      sc = (s2 & 15u) | ((s0 & 0xC0u) >> 2);
      m = ((s2 >> 4) & 15u) | ((s1 & 0xC0u) >> 2);
    }
    const float d = __half2float(__ushort_as_half((unsigned short)(hdr.x & 0xffffu)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(hdr.x >> 16)));
    const float dsc = __fmul_rn(d, (float)sc);
    const float mm = __fmul_rn(dmin, (float)m);
    // the eight nibbles as bytes 0..7 of n0, n1
    const uint32_t n0 = hi ? (qv.x >> 4) & 0x0F0F0F0Fu : qv.x & 0x0F0F0F0Fu;
    const uint32_t n1 = hi ? (qv.y >> 4) & 0x0F0F0F0Fu : qv.y & 0x0F0F0F0Fu;
    float y[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      // bits 0x4B0000qq: byte e%4 of the nibble word, then 00 00 4B
      const uint32_t bits = __byte_perm(e < 4 ? n0 : n1, 0x4B000000u, (e & 3) | 0x7540u);
      const float q = __fsub_rn(__uint_as_float(bits), 8388608.0f);  // exact
      y[e] = __fsub_rn(__fmul_rn(dsc, q), mm);
    }
    const long long w0 = b * 256 + 64 * c + 32 * hi + o;
    if constexpr (kF16) {
      uint32_t p[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {  // two round-to-nearest conversions per instruction
        const __half2 v = __float22half2_rn(make_float2(y[2 * k], y[2 * k + 1]));
        p[k] = *reinterpret_cast<const uint32_t*>(&v);
      }
      *reinterpret_cast<uint4*>(static_cast<uint16_t*>(out) + w0) = make_uint4(p[0], p[1], p[2], p[3]);
    } else {
      float4* dst = reinterpret_cast<float4*>(static_cast<float*>(out) + w0);
      dst[0] = make_float4(y[0], y[1], y[2], y[3]);
      dst[1] = make_float4(y[4], y[5], y[6], y[7]);
    }
  };
  auto qoff = [&](long long b) { return blocks + b * 144 + 16 + 32 * c + o; };
  // kInFlight blocks per iteration: all their loads are issued before any
  // is decoded, so a warp keeps several global loads outstanding
  constexpr int kInFlight = 4;
  for (long long b = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < n_blocks;
       b += kInFlight * warps) {
    uint4 hd[kInFlight];
    uint2 qd[kInFlight];
#pragma unroll
    for (int u = 0; u < kInFlight; ++u) {
      const long long bu = b + u * warps;
      hd[u] = make_uint4(0, 0, 0, 0);
      qd[u] = make_uint2(0, 0);
      if (bu < n_blocks) {
        hd[u] = *reinterpret_cast<const uint4*>(blocks + bu * 144);  // d, dmin | scales
        qd[u] = *reinterpret_cast<const uint2*>(qoff(bu));
      }
    }
#pragma unroll
    for (int u = 0; u < kInFlight; ++u)
      if (b + u * warps < n_blocks) decode(b + u * warps, hd[u], qd[u]);
  }
}

}  // namespace

extern "C" int lora_ce_q4k_dequant_device(const void* d_blocks, int64_t n_blocks, void* d_out,
                                          int32_t out_dtype, void* stream) {
  if (!d_blocks || !d_out || n_blocks < 1) return q4k_fail(LORA_CE_EINVAL, "bad argument");
  if (out_dtype != LORA_CE_F16 && out_dtype != LORA_CE_F32)
    return q4k_fail(LORA_CE_EINVAL, "out_dtype must be LORA_CE_F16 or LORA_CE_F32");
  if (((reinterpret_cast<uintptr_t>(d_blocks) | reinterpret_cast<uintptr_t>(d_out)) & 15) != 0)
    return q4k_fail(LORA_CE_EINVAL, "blocks and out must be 16-byte aligned");
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long grid = std::min<long long>((n_blocks + 7) / 8, 8LL * sms);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  const auto* src = static_cast<const uint8_t*>(d_blocks);
  if (out_dtype == LORA_CE_F16)
    lce_q4k_dequant<true><<<(unsigned)grid, 256, 0, s>>>(src, n_blocks, d_out);
  else
    lce_q4k_dequant<false><<<(unsigned)grid, 256, 0, s>>>(src, n_blocks, d_out);
  if (cudaGetLastError() != cudaSuccess) return q4k_fail(LORA_CE_ECUDA, "dequant launch failed");
  return 0;
}

extern "C" int lora_ce_q4k_dequant(const void* blocks, int64_t n_blocks, void* out,
                                   int32_t out_dtype, int32_t device) {
  if (!blocks || !out || n_blocks < 1) return q4k_fail(LORA_CE_EINVAL, "bad argument");
  if (out_dtype != LORA_CE_F16 && out_dtype != LORA_CE_F32)
    return q4k_fail(LORA_CE_EINVAL, "out_dtype must be LORA_CE_F16 or LORA_CE_F32");
  if (cudaSetDevice(device) != cudaSuccess) return q4k_fail(LORA_CE_ECUDA, "cudaSetDevice failed");
  const size_t nin = (size_t)n_blocks * 144;
  const size_t nout = (size_t)n_blocks * 256 * (out_dtype == LORA_CE_F16 ? 2 : 4);
  void *din = nullptr, *dout = nullptr;
  int rc = 0;
  if (cudaMalloc(&din, nin) != cudaSuccess || cudaMalloc(&dout, nout) != cudaSuccess)
    rc = q4k_fail(LORA_CE_ENOMEM, "cudaMalloc failed");
  if (!rc && cudaMemcpy(din, blocks, nin, cudaMemcpyHostToDevice) != cudaSuccess)
    rc = q4k_fail(LORA_CE_ECUDA, "upload failed");
  if (!rc) rc = lora_ce_q4k_dequant_device(din, n_blocks, dout, out_dtype, nullptr);
  if (!rc && cudaMemcpy(out, dout, nout, cudaMemcpyDeviceToHost) != cudaSuccess)
    rc = q4k_fail(LORA_CE_ECUDA, "download failed");
  cudaFree(din);
  cudaFree(dout);
  return rc;
}

extern "C" const char* lora_ce_q4k_last_error(void) { return g_q4k_error.c_str(); }
