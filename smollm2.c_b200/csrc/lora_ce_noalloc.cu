// lora_ce_noalloc.cu — per-position LoRA lm_head cross-entropy loss that
// allocates no memory at all.
//
// Who needs it: callers that cannot call cudaMalloc on the hot path — an
// evaluation loop running inside a serving process whose GPU memory is
// fully reserved up front by its own pool, or a runtime that forbids
// allocation after start-up so that it can never fail (or stall on an
// implicit device synchronisation) mid-request.  Such a caller gets the same
// loss the training step computes, on its own stream and device buffers,
// with every scratch buffer the kernels need living in this file's
// statically sized device arrays instead.
//
// The call only enqueues work on the caller's stream and returns; host-side
// argument errors come back as return codes, while a device-side error (a
// target id outside [0, V)) turns every output loss into NaN, since reading
// an error flag back to the host would need a host buffer.
//
// Limits (checked, with a clear error): rank 4, positions T <= 4096,
// vocabulary V <= 49152, hidden size d a multiple of 64 up to 576.  The
// arrays below take about 8.9 MB on every GPU that loads the library, until
// the process exits.  All calls share them and they keep the last call's
// contents: calls that can overlap on the GPU (different streams, or
// different host threads on one device) race and must be serialised by the
// caller.  The first call on a device resolves the arrays' device addresses
// (cudaGetSymbolAddress); make that first call before any stream capture.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "lora_ce.h"
#include "lora_ce_kernels.cuh"

using namespace lce;

namespace {

constexpr int kNaRank = 4;
constexpr int kNaMaxT = 4096;
constexpr int kNaMaxV = 49152;
constexpr int kNaMaxD = 576;
constexpr long long kNaP1Cap = 131072;  // pass-1 partial slots x positions (worst case 100,352)

// Scratch: one set per process, shared by all calls on a device.
static __device__ __align__(256) __half g_h16[(size_t)kNaMaxT * kNaMaxD];
static __device__ __align__(256) float g_tok[(size_t)kNaMaxT * (kNaRank + 4)];
static __device__ __align__(256) float g_params[(size_t)kNaMaxD * kNaRank + (size_t)kNaMaxV * kNaRank];
static __device__ __align__(256) float g_pmax[kNaP1Cap];
static __device__ __align__(256) float g_psum[kNaP1Cap];
static __device__ __align__(256) float g_pq[kNaP1Cap * kNaRank];
static __device__ __align__(256) float g_ztgt[kNaMaxT];
static __device__ __align__(256) float g_dU[(size_t)kNaMaxT * kNaRank];
static __device__ __align__(256) int g_err[4];

struct DeviceScratch {
  bool ready = false;
  __half* h16 = nullptr;
  float* tok = nullptr;
  float* params = nullptr;
  float* pmax = nullptr;
  float* psum = nullptr;
  float* pq = nullptr;
  float* ztgt = nullptr;
  float* dU = nullptr;
  int* err = nullptr;
  int units = 0;  // co-resident 2-CTA clusters of the pass-1 kernel
};

constexpr int kMaxDevices = 64;
DeviceScratch g_dev[kMaxDevices];
std::mutex g_dev_mutex;

thread_local std::string g_na_error;

int na_fail(int code, const char* msg) {
  g_na_error = msg;
  return code;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

bool na_map(CUtensorMap* m, const void* base, long long rows, int d, int box_rows) {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return false;
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  cuuint64_t dims[2] = {(cuuint64_t)d, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)d * 2};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

template <class P, class S>
bool symbol_ptr(P** out, const S& sym) {
  return cudaGetSymbolAddress(reinterpret_cast<void**>(out), sym) == cudaSuccess && *out;
}

// Once per device, with that device current: the device addresses of the
// scratch arrays (the host-side names are only stand-ins) and the number of
// co-resident pass-1 clusters.  No allocation happens here either.
int setup_device(int dev, DeviceScratch** out) {
  std::lock_guard<std::mutex> lock(g_dev_mutex);
  DeviceScratch& s = g_dev[dev];
  if (!s.ready) {
    if (!symbol_ptr(&s.h16, g_h16) || !symbol_ptr(&s.tok, g_tok) ||
        !symbol_ptr(&s.params, g_params) || !symbol_ptr(&s.pmax, g_pmax) ||
        !symbol_ptr(&s.psum, g_psum) || !symbol_ptr(&s.pq, g_pq) ||
        !symbol_ptr(&s.ztgt, g_ztgt) || !symbol_ptr(&s.dU, g_dU) ||
        !symbol_ptr(&s.err, g_err))
      return na_fail(LORA_CE_ECUDA, "cudaGetSymbolAddress failed for the scratch arrays");
    auto kern = lce_gemm_kernel<EpiLse<kNaRank>, true, 2>;
    const int kblocks_max = kNaMaxD / kBK;
    using Epi = EpiLse<kNaRank>;
    const int smem = SmemLayout::bytes(kblocks_max, Epi::kRec * Epi::kRecBufs, Epi::kRing);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess)
      return na_fail(LORA_CE_ECUDA, "cudaFuncSetAttribute failed");
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess)
      return na_fail(LORA_CE_ECUDA, "cudaGetDeviceProperties failed");
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned)prop.multiProcessorCount);
    lc.blockDim = dim3(block_threads(EpiLse<kNaRank>::kWarps));
    lc.dynamicSmemBytes = (size_t)smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &lc) != cudaSuccess || n < 1)
      return na_fail(LORA_CE_ECUDA, "pass-1 kernel cannot be made resident");
    s.units = n;
    s.ready = true;
  }
  *out = &s;
  return 0;
}

// B [R][V] (reference layout) -> the pair-interleaved layout the kernels
// read; rows V..Vpad-1 zero.
__global__ void na_pack_B(const float* __restrict__ B, int V, long long Vpad, float* __restrict__ Bp) {
  const long long n = Vpad * kNaRank;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (long long)gridDim.x * blockDim.x) {
    const long long v = 2 * (e / (2 * kNaRank)) + (e & 1);
    const int j = (int)((e % (2 * kNaRank)) / 2);
    Bp[e] = v < V ? B[(long long)j * V + v] : 0.f;
  }
}

// A device-side error of this call (flag set by lce_prep) poisons the output.
__global__ void na_poison(const int* __restrict__ err, float* __restrict__ loss, int T) {
  if (*(volatile const int*)err == 0) return;
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < T; t += gridDim.x * blockDim.x)
    loss[t] = __int_as_float(0x7fc00000);
}

int max_seg(int n_a, int n_b, int G) {
  const long long total = (long long)n_a * n_b;
  int best = 1;
  for (int a = 0; a < n_a; ++a) {
    const int s0 = tile_owner((long long)a * n_b, total, G);
    const int s1 = tile_owner((long long)a * n_b + n_b - 1, total, G);
    if (s1 - s0 + 1 > best) best = s1 - s0 + 1;
  }
  return best;
}

}  // namespace

extern "C" int lora_ce_token_loss_noalloc(const uint16_t* d_W, int32_t vocab, int32_t dim,
                                          const float* d_A, const float* d_B, float scale,
                                          const void* d_H, int32_t h_dtype, int32_t T,
                                          const int32_t* d_targets, float* d_loss,
                                          void* stream) {
  if (!d_W || !d_A || !d_B || !d_H || !d_targets || !d_loss)
    return na_fail(LORA_CE_EINVAL, "null device pointer");
  if (h_dtype < LORA_CE_BF16 || h_dtype > LORA_CE_F32)
    return na_fail(LORA_CE_EINVAL, "bad hidden-state dtype");
  if (T < 1 || T > kNaMaxT) return na_fail(LORA_CE_EINVAL, "T must be in [1, 4096]");
  if (vocab < 1 || vocab > kNaMaxV) return na_fail(LORA_CE_EINVAL, "vocab must be in [1, 49152]");
  if (dim < 64 || dim % 64 != 0 || dim > kNaMaxD)
    return na_fail(LORA_CE_EINVAL, "dim must be a multiple of 64 in [64, 576]");
  // every argument check comes before anything is enqueued or set up, so a
  // rejected call leaves the stream and the shared scratch untouched
  if ((reinterpret_cast<uintptr_t>(d_H) & 15) != 0)
    return na_fail(LORA_CE_EINVAL, "hidden states must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(d_W) & 15) != 0)
    return na_fail(LORA_CE_EINVAL, "W must be 16-byte aligned (TMA operand)");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return na_fail(LORA_CE_ECUDA, "cudaGetDevice failed");
  DeviceScratch* s = nullptr;
  int rc = setup_device(dev, &s);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int R = kNaRank, d = dim, V = vocab;
  const long long Vpad = (V + kBN - 1) / kBN * kBN;
  const long long Tpad = (T + kBN - 1) / kBN * kBN;
  const int kblocks = d / kBK;
  const int res_rows = 2 * kBM;
  const int n_a1 = (T + res_rows - 1) / res_rows, n_b1 = (int)(Vpad / kBN);
  const long long total1 = (long long)n_a1 * n_b1;
  const int G1 = (int)(total1 < s->units ? total1 : s->units);
  const long long stride1 = (long long)n_a1 * res_rows;
  const int cp1 = col_parts(EpiLse<R>::kWarps);
  if ((long long)cp1 * max_seg(n_a1, n_b1, G1) * stride1 > kNaP1Cap)
    return na_fail(LORA_CE_ESTATE, "pass-1 partials exceed the static scratch");
  CUtensorMap mapH, mapW;
  if (!na_map(&mapH, s->h16, T, d, kBM) || !na_map(&mapW, d_W, V, d, kBM))
    return na_fail(LORA_CE_ECUDA, "cuTensorMapEncodeTiled failed");

  if (cudaMemsetAsync(s->err, 0, sizeof(int), st) != cudaSuccess)
    return na_fail(LORA_CE_ECUDA, "cudaMemsetAsync failed");
  // A [d][R] and the packed B share one buffer, as in the training step
  if (cudaMemcpyAsync(s->params, d_A, (size_t)d * R * 4, cudaMemcpyDeviceToDevice, st) !=
      cudaSuccess)
    return na_fail(LORA_CE_ECUDA, "cudaMemcpyAsync failed");
  float* Bp = s->params + (size_t)d * R;
  na_pack_B<<<256, 256, 0, st>>>(d_B, V, Vpad, Bp);
  lce_prep<R><<<(int)std::min<long long>((Tpad + 7) / 8, 592), 256, (size_t)d * R * 4, st>>>(
      d_H, h_dtype, 0, (int)Tpad, T, d, s->params, scale, d_targets, V, s->h16, s->tok, s->err,
      nullptr, 0, 0, nullptr, 0);
  GemmArgs g{};
  g.kblocks = kblocks;
  g.kstr = kblocks;
  g.kmain = kblocks;
  g.rank_total = R;
  g.rank_off = 0;
  g.T = T;
  g.V = V;
  g.R = R;
  g.Vpad = Vpad;
  g.err = s->err;
  g.tok = s->tok;
  g.Bt = Bp;
  g.p_max = s->pmax;
  g.p_sum = s->psum;
  g.p_q = s->pq;
  g.z_tgt = s->ztgt;
  g.gBp = nullptr;
  g.n_a = n_a1;
  g.n_b = n_b1;
  g.Tcap = stride1;
  {
    using Epi = EpiLse<R>;
    const int smem = SmemLayout::bytes(kblocks, Epi::kRec * Epi::kRecBufs, Epi::kRing);
    auto kern = lce_gemm_kernel<EpiLse<R>, true, 2>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess)
      return na_fail(LORA_CE_ECUDA, "cudaFuncSetAttribute failed");
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned)(G1 * 2));
    lc.blockDim = dim3(block_threads(EpiLse<kNaRank>::kWarps));
    lc.dynamicSmemBytes = (size_t)smem;
    lc.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    if (cudaLaunchKernelEx(&lc, kern, mapH, mapW, mapH, mapW, g) != cudaSuccess)
      return na_fail(LORA_CE_ECUDA, "pass-1 launch failed");
  }
  lce_combine<R><<<(T + 7) / 8, 256, 0, st>>>(T, cp1, res_rows, n_b1, s->units, 1, stride1,
                                                  s->pmax,
                                                  s->psum, s->pq, s->ztgt, Bp, scale, s->tok,
                                                  s->dU, d_loss, nullptr, 0);
  na_poison<<<(T + 255) / 256, 256, 0, st>>>(s->err, d_loss, T);
  if (cudaGetLastError() != cudaSuccess) return na_fail(LORA_CE_ECUDA, "kernel launch failed");
  return 0;
}

extern "C" const char* lora_ce_noalloc_last_error(void) { return g_na_error.c_str(); }
