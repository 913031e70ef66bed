// lora_ce_q4k.cu — Q4_K (GGUF / ggml type 12) dequantisation for the QLoRA
// lm_head: 144-byte super-blocks of 256 weights over the flattened [V][d]
// tensor, f16 d, f16 dmin, twelve bytes of 6-bit (scale, min) pairs for the
// eight 32-weight sub-blocks and 128 bytes of 4-bit quants.
//   y = (d * sc) * q - (dmin * m), each product and the difference rounded
//   separately (ggml's scalar order without contraction)
// HBM-bound: 144 bytes in and 512 (f16) or 1024 (f32) bytes out per block.
// One warp per block; lane l produces weights 8l .. 8l+7 (run c = l / 8 of
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

__device__ __forceinline__ uint32_t byte_of(const uint4& v, int i) {
  const uint32_t w = i < 4 ? v.x : i < 8 ? v.y : i < 12 ? v.z : v.w;
  return (w >> (8 * (i & 3))) & 0xffu;
}

template <bool kF16>
__global__ void __launch_bounds__(256) lce_q4k_dequant(const uint8_t* __restrict__ blocks,
                                                        long long n_blocks, void* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long b = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < n_blocks;
       b += warps) {
    const uint8_t* blk = blocks + b * 144;
    const uint4 hdr = *reinterpret_cast<const uint4*>(blk);  // d, dmin, scales[12]
    const int c = lane >> 3;                   // run of 64
    const int hi = (lane >> 2) & 1;            // high nibbles: second 32 of the run
    const int o = (lane & 3) * 8;              // offset in the run's 32 quant bytes
    const int j = 2 * c + hi;                  // sub-block
    const uint2 qv = *reinterpret_cast<const uint2*>(blk + 16 + 32 * c + o);
    // scales[k] is header byte 4 + k
    int sc, m;
    if (j < 4) {
      sc = byte_of(hdr, 4 + j) & 63;
      m = byte_of(hdr, 8 + j) & 63;
    } else {
      sc = (byte_of(hdr, 8 + j) & 15) | ((byte_of(hdr, j) >> 6) << 4);
      m = (byte_of(hdr, 8 + j) >> 4) | ((byte_of(hdr, 4 + j) >> 6) << 4);
    }
    const float d = __half2float(__ushort_as_half((unsigned short)(hdr.x & 0xffffu)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(hdr.x >> 16)));
    const float dsc = __fmul_rn(d, (float)sc);
    const float mm = __fmul_rn(dmin, (float)m);
    float y[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t byte = ((e < 4 ? qv.x : qv.y) >> (8 * (e & 3))) & 0xffu;
      const uint32_t q = hi ? (byte >> 4) : (byte & 15u);
      y[e] = __fsub_rn(__fmul_rn(dsc, (float)q), mm);
    }
    const long long w0 = b * 256 + 64 * c + 32 * hi + o;
    if constexpr (kF16) {
      uint32_t p[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        p[k] = (uint32_t)__half_as_ushort(__float2half_rn(y[2 * k])) |
               ((uint32_t)__half_as_ushort(__float2half_rn(y[2 * k + 1])) << 16);
      *reinterpret_cast<uint4*>(static_cast<uint16_t*>(out) + w0) = make_uint4(p[0], p[1], p[2], p[3]);
    } else {
      float4* dst = reinterpret_cast<float4*>(static_cast<float*>(out) + w0);
      dst[0] = make_float4(y[0], y[1], y[2], y[3]);
      dst[1] = make_float4(y[4], y[5], y[6], y[7]);
    }
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
