// lora_ce_api.cu — host side of the C ABI declared in include/lora_ce.h:
// handle lifetime, uploads, the per-step launch sequence and the optional
// NCCL all-reduce.  No CPU compute path exists: every step runs on the GPU
// or fails with an error code.
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <thread>
#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <string>
#include <type_traits>
#include <vector>

#include "lora_ce.h"
#include "lora_ce_kernels.cuh"
#include "lora_ce_tc.cuh"
#include "lora_ce_wide.cuh"

using namespace lce;

namespace {

// Phases of one step, in launch order (lora_ce_phase_name).
enum Phase { kPhPrep, kPhPass1, kPhCombine, kPhPass2, kPhDA, kPhFinalize, kPhAllReduce,
             kPhNorm, kPhAdam, kNumPhases };
const char* const kPhaseNames[kNumPhases] = {"prep", "pass1_lse", "combine", "pass2_grad",
                                             "dA_partial", "finalize", "allreduce",
                                             "sqnorm", "adam"};

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

#define LCE_CUDA(call)                                                                  \
  do {                                                                                  \
    cudaError_t e_ = (call);                                                            \
    if (e_ != cudaSuccess)                                                              \
      return fail(LORA_CE_ECUDA, std::string(#call) + ": " + cudaGetErrorString(e_));  \
  } while (0)

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// [rows][d] f16 row-major, read in boxes of 64 x box_rows with 128 B swizzle.
bool make_map(CUtensorMap* m, const void* base, long long rows, int d, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)d, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)d * 2};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

// [rows][width] f16 with a row stride of ld elements (ld % 8 == 0), read in
// boxes of 64 x box_rows with 128 B swizzle; columns past width read as 0.
bool make_map_ld(CUtensorMap* m, const void* base, long long rows, long long width, long long ld,
                 int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)width, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

long long round_up(long long x, long long m) { return (x + m - 1) / m * m; }

// NCCL is loaded on first use (a communicator is only needed for
// multi-GPU runs), preferring a libnccl already loaded in the process (for
// example PyTorch's) so that two different NCCL builds never meet in one
// process; otherwise the system libnccl.so.2.  Communicators are
// non-blocking: every NCCL call returns at once, its completion (and any
// asynchronous error) is polled against a host deadline, and a collective
// that does not finish in time is aborted (ncclCommAbort ends NCCL's
// kernels) and reported as LORA_CE_ENCCL.
struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  bool ok = false;
};

const NcclApi& nccl() {
  static NcclApi api;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!lib) lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (lib) {
      auto sym = [lib](auto& fn, const char* name) {
        fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(lib, name));
      };
      sym(api.GetUniqueId, "ncclGetUniqueId");
      sym(api.CommInitRankConfig, "ncclCommInitRankConfig");
      sym(api.AllReduce, "ncclAllReduce");
      sym(api.CommGetAsyncError, "ncclCommGetAsyncError");
      sym(api.CommFinalize, "ncclCommFinalize");
      sym(api.CommDestroy, "ncclCommDestroy");
      sym(api.CommAbort, "ncclCommAbort");
      sym(api.GetErrorString, "ncclGetErrorString");
      api.ok = api.GetUniqueId && api.CommInitRankConfig && api.AllReduce &&
               api.CommGetAsyncError && api.CommFinalize && api.CommDestroy && api.CommAbort;
    }
  }
  return api;
}

using Clock = std::chrono::steady_clock;

double ms_since(Clock::time_point t0) {
  return std::chrono::duration<double, std::milli>(Clock::now() - t0).count();
}

// Poll a non-blocking communicator until its last call has completed
// (ncclSuccess), failed, or `timeout_ms` passed (ncclInProgress returned).
ncclResult_t nccl_settle(ncclComm_t comm, double timeout_ms) {
  const Clock::time_point t0 = Clock::now();
  for (;;) {
    ncclResult_t st = ncclInProgress;
    if (nccl().CommGetAsyncError(comm, &st) != ncclSuccess) return ncclInternalError;
    if (st != ncclInProgress) return st;
    if (ms_since(t0) > timeout_ms) return ncclInProgress;
    std::this_thread::yield();
  }
}

const char* nccl_str(ncclResult_t r) {
  return nccl().GetErrorString ? nccl().GetErrorString(r) : "NCCL error";
}

// Largest T a handle may be created for (the planning loops below and the
// position-indexed buffers are sized from it).
constexpr int kMaxTokens = 1 << 24;

// Largest number of CTA segments any resident tile's run of n_b tiles is
// split into, for n_a x n_b tiles over G CTAs.
int max_segments(int n_a, int n_b, int G) {
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

namespace {
// Chunks of a host-input step: pass 1 runs once per chunk of position blocks
// so that the copy of the next chunk overlaps it.  Chunks of at least 8
// blocks keep each launch's tile ranges long.
constexpr int kMaxChunks = 4;
int step_chunks(int n_a1) { return n_a1 >= 32 ? 4 : n_a1 >= 16 ? 2 : 1; }
}  // namespace

struct lora_ce_handle {
  lora_ce_config cfg{};
  // r: the adapter's rank; R: the rank the kernels run at, r rounded up to
  // 4, 8, 16, 32 or 64.  The extra columns of A and rows of B are zero and stay
  // zero (their U, dU, dA and dB terms are exactly 0, so Adam leaves them at
  // 0), which makes a rank-r step identical to the reference's.
  int r = 0, R = 0, d = 0, V = 0;
  long long Vpad = 0, Tcap = 0;
  int num_sms = 0;
  int pair = 2;             // 2: CTA-pair (cta_group::2) GEMM tiles; 1: single-CTA tiles
  int units1 = 0, units2 = 0;  // co-resident tile-range owners of pass 1 / pass 2
  // ranks 8..64 in CTA pairs: both passes with their rank sums on the tensor
  // cores (lce_gemm_tc, 192-column streamed tiles)
  bool tc = false;
  int units1t = 0, units2t = 0;
  cudaStream_t stream = nullptr;
  // host-input steps copy h in chunks on `cstream` while the compute stream
  // converts and runs pass 1 on the chunks that have arrived
  cudaStream_t cstream = nullptr;
  cudaEvent_t ev_start = nullptr;
  cudaEvent_t ev_chunk[kMaxChunks] = {};
  // CUDA graphs of whole steps, replayed while (T, dtype, input pointers)
  // repeat; only Adam's bias corrections change between replays
  struct StepGraph {
    bool valid = false;
    bool host = false;  // lora_ce_step (copies + read-back) or lora_ce_step_device
    int T = 0, dtype = 0;
    const void* H = nullptr;
    const int32_t* tgt = nullptr;
    float* d_loss = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    cudaGraphNode_t adam = nullptr;  // the node that takes the Adam arguments
    cudaKernelNodeParams adam_p{};
    int adam_nargs = 0;
    long long nparam = 0;
    int launches = 0;
    unsigned long long last_use = 0;
  };
  static constexpr int kGraphs = 4;
  StepGraph graphs[kGraphs];
  unsigned long long graph_clock = 0;
  bool use_graphs = true;
  float* res_host = nullptr;  // pinned [loss, error code] read back by lora_ce_step
  bool poisoned = false;
  bool have_weight = false;
  int32_t step = 0;
  int32_t launches = 0;
  int last_T = 0;
  // device buffers
  __half* W = nullptr;
  __half* h16 = nullptr;
  float* tok = nullptr;
  float* params = nullptr;  // [A (d*R) | B (Vpad*R, pair-interleaved: bidx)]
  float* mom1 = nullptr;
  float* mom2 = nullptr;
  float* Gbuf = nullptr;    // [dA | dB (bidx layout) | loss | n_pred]
  float* gmean = nullptr;
  float* p_max = nullptr;
  float* p_sum = nullptr;
  float* p_q = nullptr;
  long long p1_cap = 0;     // floats per p_max / p_sum
  float* z_tgt = nullptr;
  float* loss_tok = nullptr;
  float* dU = nullptr;
  float* gAp = nullptr;
  float* gBp = nullptr;
  unsigned long long* corr_fx = nullptr;  // onehot part of dB, fixed point [Vpad*R]
  int gbp_segs = 0;
  double* norm_parts = nullptr;
  int* err = nullptr;       // device error flag
  float* d_loss = nullptr;  // [loss, err-as-int] result pair
  void* in_H = nullptr;     // staging for host inputs
  int32_t* in_tgt = nullptr;
  CUtensorMap mapW_res{}, mapW_str{};
  // rank augmentation (R >= 8): waug [Vpad][64], haug [Tcap][64] f16
  __half* w_aug = nullptr;
  __half* h_aug = nullptr;
  // ranks 32, 64: per 16-rank chunk, pass 1's column records (B, rank-16
  // layout) and pass 2's position records (sU, -M log2 e, 1/S)
  float* Bc = nullptr;
  float* tokc = nullptr;
  CUtensorMap mapWa_res{}, mapWa_str{};
  // tensor-core rank sums: pass 1's B^T [hi ; lo] (2R x Vpad), pass 2's
  // (s*U)^T [hi ; lo] (2R x Tcap) and per-position exponent offsets
  __half* xv = nullptr;
  __half* xt = nullptr;
  float* nml = nullptr;
  CUtensorMap mapW_strT{}, mapWa_strT{}, mapXv{};
  // ranks 65..256 (kernel ranks 128, 256): position blocks of `wide_p`
  // positions with materialised logit rows (lora_ce_wide.cuh)
  bool wide = false;
  int wide_p = 0;
  float* w_sU = nullptr;     // [Tcap][R] s*U
  float* w_Z = nullptr;      // [wide_p][Vpad] logits, then p - onehot
  float* w_Bp = nullptr;     // [R][Vpad] B, plain
  float* w_dB = nullptr;     // [R][Vpad] dB sums
  float* w_dUp = nullptr;    // [kWMaxSplit][wide_p][R] split partials of dU
  float* w_dAp = nullptr;    // [kWMaxSplit][d][R] split partials of dA
  ncclComm_t comm = nullptr;
  int nranks = 1, rank = 0;
  double comm_timeout_ms = 60000.0;  // bound on any wait that involves a collective
  bool stuck = false;  // streams still busy after an aborted collective
  // optional per-phase timing (events on the handle's stream)
  bool prof = false;
  cudaEvent_t ev[kNumPhases + 1] = {};
  // optional timing of host-input steps (events captured into the step's
  // graph): [0] compute stream at step start, [1] copy stream before the
  // first chunk, [2 .. 2+chunks) after each chunk, [kMaxChunks + 2] result
  // read back; plus the host's own time inside the last lora_ce_step
  bool ctime = false;
  cudaEvent_t tev[kMaxChunks + 3] = {};
  int ctime_chunks = 0;
  float host_us[2] = {0.f, 0.f};  // enqueue (or graph launch), wait for the result
};

namespace {

void drop_graphs(lora_ce_handle* h);

template <class T>
int dalloc(T** p, size_t count) {
  if (cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T) + 16) != cudaSuccess) {
    *p = nullptr;
    cudaGetLastError();  // not sticky: clear it so later launch checks do not see it
    return fail(LORA_CE_ENOMEM, "cudaMalloc failed");
  }
  if (cudaMemset(*p, 0, count * sizeof(T) + 16) != cudaSuccess)
    return fail(LORA_CE_ECUDA, "cudaMemset failed");
  return 0;
}

void free_streams(lora_ce_handle* h) {
  if (h->res_host) cudaFreeHost(h->res_host);
  for (cudaEvent_t e : h->ev_chunk)
    if (e) cudaEventDestroy(e);
  if (h->ev_start) cudaEventDestroy(h->ev_start);
  if (h->cstream) cudaStreamDestroy(h->cstream);
  if (h->stream) cudaStreamDestroy(h->stream);
}

void free_all(lora_ce_handle* h) {
  void* ptrs[] = {h->W,     h->h16,   h->tok,      h->params, h->mom1,  h->mom2,
                  h->Gbuf,  h->gmean, h->p_max,    h->p_sum,  h->p_q,   h->z_tgt,
                  h->loss_tok, h->dU, h->gAp,      h->gBp,    h->norm_parts, h->err, h->corr_fx,
                  h->d_loss, h->in_H, h->in_tgt, h->w_aug, h->h_aug, h->Bc, h->tokc,
                  h->xv, h->xt, h->nml, h->w_sU, h->w_Z, h->w_Bp, h->w_dB, h->w_dUp,
                  h->w_dAp};
  for (void* p : ptrs)
    if (p) cudaFree(p);
}

// The rank the kernels run at: the adapter's rank rounded up.
int kernel_rank(int r) {
  return r <= 4 ? 4 : r <= 8 ? 8 : r <= 16 ? 16 : r <= 32 ? 32 : r <= 64 ? 64 : r <= 128 ? 128 : 256;
}

// Largest rank of the fused passes; ranks above it take the wide-rank path.
constexpr int kMaxFusedRank = 64;
constexpr int kMaxRank = 256;  // LORA_MAX_RANK (src/train.c:20)

// The same decisions at run time, for sizing a handle's buffers.
int aug_width_of(int R) {
  if (R < LCE_AUG_MIN_RANK) return 0;
  return R <= 16 ? 64 : (2 * R + 63) / 64 * 64;
}

int check_cfg(const lora_ce_config* c) {
  if (!c) return fail(LORA_CE_EINVAL, "null config");
  if (c->dim < 64 || c->dim % 64 != 0 || c->dim > 64 * kMaxKBlocks)
    return fail(LORA_CE_EINVAL, "dim must be a multiple of 64 in [64, 640]");
  if (c->vocab < 1) return fail(LORA_CE_EINVAL, "vocab must be positive");
  if (c->rank < 1 || c->rank > kMaxRank) return fail(LORA_CE_EINVAL, "rank must be in [1, 256]");
  if (c->rank <= kMaxFusedRank &&
      c->dim / 64 + aug_width_of(kernel_rank(c->rank)) / 64 > kMaxKBlocks)
    return fail(LORA_CE_EINVAL, "dim too large for this rank (resident K-blocks)");
  if (c->max_tokens < 1 || c->max_tokens > kMaxTokens)
    return fail(LORA_CE_EINVAL, "max_tokens must be in [1, 2^24]");
  if (!(c->lr >= 0.f) || !(c->eps > 0.f) || !(c->beta1 >= 0.f && c->beta1 < 1.f) ||
      !(c->beta2 >= 0.f && c->beta2 < 1.f) || !(c->weight_decay >= 0.f) ||
      !(c->clip_norm >= 0.f) || !std::isfinite(c->scale))
    return fail(LORA_CE_EINVAL, "bad optimizer hyper-parameters");
  return 0;
}

// The finalize kernel blocks (a grid-stride pass over the parameters) and
// the norm partials they may write.
constexpr int kFinBlocksMax = 2048;
// Parameter counts of the two kernels whose AdamArgs a graph replay updates.
constexpr int kAdamArgs = 8;
constexpr int kFinalizeArgs = 21;

const void* fused_finalize_fn(int R) {
  switch (R) {
    case 4: return reinterpret_cast<const void*>(lce_finalize<4, kFinAdam>);
    case 8: return reinterpret_cast<const void*>(lce_finalize<8, kFinAdam>);
    case 16: return reinterpret_cast<const void*>(lce_finalize<16, kFinAdam>);
    case 32: return reinterpret_cast<const void*>(lce_finalize<32, kFinAdam>);
    default: return reinterpret_cast<const void*>(lce_finalize<64, kFinAdam>);
  }
}

using GemmKernel = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap,
                           const CUtensorMap, const GemmArgs);

// Adam's arguments for step `step` (the bias corrections 1 - beta^step are
// computed on the host with powf, as src/train.c:178-179 does).
AdamArgs adam_args(const lora_ce_handle* h, long long nparam, int32_t step) {
  AdamArgs aa{};
  aa.n = nparam;
  aa.lr = h->cfg.lr;
  aa.b1 = h->cfg.beta1;
  aa.b2 = h->cfg.beta2;
  aa.c1 = 1.0f - h->cfg.beta1;
  aa.c2 = 1.0f - h->cfg.beta2;
  aa.eps = h->cfg.eps;
  aa.wd = h->cfg.weight_decay;
  aa.clip = h->cfg.clip_norm;
  aa.b1t = 1.0f - powf(h->cfg.beta1, (float)step);
  aa.b2t = 1.0f - powf(h->cfg.beta2, (float)step);
  aa.n_norm_parts = aa.clip > 0.f ? 256 : 0;
  return aa;
}


// Everything a kernel rank decides.  Ranks up to 16 run each pass once;
// ranks 32 and 64 run each pass once per chunk of 16 ranks (the epilogue's
// accumulators for 16 ranks are what fits in registers), with the full-rank
// logit term in the MMA either way.
//   augmentation layout 0: none (rank 4: the term is epilogue FMAs)
//   layout 1: one 64-wide block, [sU_hi | sU_hi | sU_lo] . [B_hi | B_lo | B_hi]
//   layout 2: [sU_hi | sU_lo] . [B_hi | B_lo], 2R columns, K-steps pairing
//             hi.hi, hi.lo and lo.hi slices
template <int R>
struct RankPlan {
  static constexpr bool kChunked = R > 16;
  static constexpr int kRC = kChunked ? 16 : R;  // ranks per pass
  using EL = std::conditional_t<kChunked, EpiLse<16, true, true>, EpiLse<R>>;
  using EG = std::conditional_t<kChunked, EpiGrad<16, true, true>, EpiGrad<R>>;
  static constexpr bool kAug = EL::kAug;
  static constexpr int kLayout = !kAug ? 0 : kChunked ? 2 : 1;
  static constexpr int kAugWidth = kLayout == 2 ? (2 * R + 63) / 64 * 64 : kLayout == 1 ? 64 : 0;
  static constexpr int kAugBlocks = kAugWidth / 64;
  static_assert(EG::kAug == kAug, "both passes augment the rank term or neither");
  static void schedule(GemmArgs& g) {
    g.n_aug = 0;
    if constexpr (kLayout == 1) {
      for (int s = 0; s < (3 * R + 15) / 16; ++s) {
        g.aug_a[g.n_aug] = (uint8_t)s;
        g.aug_b[g.n_aug++] = (uint8_t)s;
      }
    } else if constexpr (kLayout == 2) {
      constexpr int q = R / 16;
      for (int k = 0; k < q; ++k) {
        const uint8_t pa[3] = {(uint8_t)k, (uint8_t)k, (uint8_t)(q + k)};
        const uint8_t pb[3] = {(uint8_t)k, (uint8_t)(q + k), (uint8_t)k};
        for (int m = 0; m < 3; ++m) {
          g.aug_a[g.n_aug] = pa[m];
          g.aug_b[g.n_aug++] = pb[m];
        }
      }
    }
  }
};

template <class Epi>
GemmKernel gemm_kernel(int pair, int kblocks, int* smem_out) {
  const int smem_staged = SmemLayout::bytes(kblocks, Epi::kRec * Epi::kRecBufs,
                                            pair == 2 ? Epi::kRing : kRingBytes);
  const bool staged = smem_staged <= kMaxDynSmem;
  *smem_out = staged ? smem_staged
                     : SmemLayout::bytes(kblocks, 0, pair == 2 ? Epi::kRing : kRingBytes);
  if (pair == 2) return staged ? lce_gemm_kernel<Epi, true, 2> : lce_gemm_kernel<Epi, false, 2>;
  return staged ? lce_gemm_kernel<Epi, true, 1> : lce_gemm_kernel<Epi, false, 1>;
}

template <int R>
void plan_units(lora_ce_handle* h, int* u1, int* u2);

// How many tile-range owners (CTAs, or 2-CTA clusters) of this GEMM pass
// can be resident at once: the persistent split assumes all of them are.
template <class Epi>
int resident_units(int pair, int kblocks, int num_sms) {
  int smem = 0;
  auto kern = gemm_kernel<Epi>(pair, kblocks, &smem);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return 0;
  if (pair == 1) return num_sms;
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3((unsigned)num_sms);
  lc.blockDim = dim3(block_threads(Epi::kWarps));
  lc.dynamicSmemBytes = (size_t)smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &lc) != cudaSuccess) return 0;
  return n;
}

// The tensor-core rank-sum passes (CTA pairs, ranks 8..64).
template <int kPass, int R>
int tc_smem(int kblocks) {
  return TcLayout::bytes(kblocks, TcLayout::stages(kblocks, R), R);
}

template <int kPass, int R>
int resident_units_tc(int kblocks, int num_sms) {
  const int smem = tc_smem<kPass, R>(kblocks);
  if (TcLayout::stages(kblocks, R) < 2 || smem > kMaxDynSmem) return 0;
  auto kern = lce_gemm_tc<kPass, R>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return 0;
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3((unsigned)num_sms);
  lc.blockDim = dim3(kThreadsT);
  lc.dynamicSmemBytes = (size_t)smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &lc) != cudaSuccess) return 0;
  return n;
}

template <int kPass, int R>
int launch_gemm_tc(const CUtensorMap& map_res, const CUtensorMap& map_str,
                   const CUtensorMap& map_res_aug, const CUtensorMap& map_str_aug,
                   const CUtensorMap& map_x, const GemmArgs& g, int units, cudaStream_t st) {
  const int smem = tc_smem<kPass, R>(g.kblocks);
  auto kern = lce_gemm_tc<kPass, R>;
  LCE_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3((unsigned)(units * 2));
  lc.blockDim = dim3(kThreadsT);
  lc.dynamicSmemBytes = (size_t)smem;
  lc.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  LCE_CUDA(cudaLaunchKernelEx(&lc, kern, map_res, map_str, map_res_aug, map_str_aug, map_x, g));
  return 0;
}

// Co-resident units of a rank's two passes; also lets lce_prep of large
// ranks use its d*R floats of dynamic shared memory.
template <int R>
void plan_units(lora_ce_handle* h, int* u1, int* u2) {
  using Plan = RankPlan<R>;
  const int kb = h->d / kBK + Plan::kAugBlocks;
  *u1 = resident_units<typename Plan::EL>(h->pair, kb, h->num_sms);
  *u2 = resident_units<typename Plan::EG>(h->pair, kb, h->num_sms);
  if constexpr (R >= 8) {
    if (h->tc) {
      h->units1t = resident_units_tc<1, R>(kb, h->num_sms);
      h->units2t = resident_units_tc<2, R>(kb, h->num_sms);
      if (h->units1t < 1 || h->units2t < 1) h->tc = false;  // the per-logit epilogues instead
    }
  }
  const int prep_smem = h->d * R * 4;
  if (prep_smem > 48 * 1024 &&
      cudaFuncSetAttribute(lce_prep<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, prep_smem) !=
          cudaSuccess)
    *u1 = 0;
  if constexpr (R >= 16) {
    if (cudaFuncSetAttribute(lce_prep_wide<R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             prep_wide_smem(R, h->d)) != cudaSuccess)
      *u1 = 0;
  }
}

// Launch one GEMM pass: `units` tile-range owners (CTAs, or 2-CTA clusters).
template <class Epi>
int launch_gemm(const CUtensorMap& map_res, const CUtensorMap& map_str,
                const CUtensorMap& map_res_aug, const CUtensorMap& map_str_aug, const GemmArgs& g,
                int units, int pair, int kblocks, cudaStream_t st) {
  int smem = 0;
  auto kern = gemm_kernel<Epi>(pair, kblocks, &smem);
  LCE_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3((unsigned)(units * pair));
  lc.blockDim = dim3(block_threads(Epi::kWarps));
  lc.dynamicSmemBytes = (size_t)smem;
  lc.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)pair;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  lc.attrs = attr;
  lc.numAttrs = pair == 2 ? 1 : 0;
  LCE_CUDA(cudaLaunchKernelEx(&lc, kern, map_res, map_str, map_res_aug, map_str_aug, g));
  return 0;
}

inline void mark(lora_ce_handle* h, int phase) {
  if (h->prof) cudaEventRecord(h->ev[phase], h->stream);
}

template <int R>
int run_step(lora_ce_handle* h, const void* dH, int dtype, int T, const int32_t* dtg,
             float* d_loss_out, int chunks, const cudaEvent_t* chunk_ready) {
  using Plan = RankPlan<R>;
  using EL = typename Plan::EL;
  using EG = typename Plan::EG;
  constexpr bool kAug = Plan::kAug;
  constexpr int kRC = Plan::kRC;
  cudaStream_t st = h->stream;
  const int d = h->d, V = h->V;
  const int kmain = d / kBK;
  const int kblocks = kmain + Plan::kAugBlocks;  // resident and streamed K-blocks alike
  const long long Tpad = round_up(T, kBN);
  int launches = 0;
  // ranks 8..64: rank sums on the tensor cores (one launch per pass at every rank)
  const bool tc = R >= 8 && h->tc;
  const bool rank_chunks = Plan::kChunked && !tc;
  if (rank_chunks) chunks = 1;  // rank chunks: one launch per chunk of ranks instead

  CUtensorMap mapH_res, mapH_str;
  if (!make_map(&mapH_res, h->h16, T, d, kBM) || !make_map(&mapH_str, h->h16, T, d, kBN))
    return fail(LORA_CE_ECUDA, "cuTensorMapEncodeTiled failed for h");
  CUtensorMap mapHa_res = mapH_res, mapHa_str = mapH_str;  // unused unless kAug
  if (kAug && (!make_map(&mapHa_res, h->h_aug, T, Plan::kAugWidth, kBM) ||
               !make_map(&mapHa_str, h->h_aug, T, Plan::kAugWidth, kBN)))
    return fail(LORA_CE_ECUDA, "cuTensorMapEncodeTiled failed for the rank augmentation");

  const int pair = h->pair;
  const int res_rows = kBM * pair;
  const int n_a1 = (T + res_rows - 1) / res_rows;
  const int n_b1 = tc ? (V + tc_bn(R) - 1) / tc_bn(R) : (int)(h->Vpad / kBN);
  const int units1 = tc ? h->units1t : h->units1;
  chunks = std::max(1, std::min(chunks, n_a1));
  const int cp1 = tc ? col_parts(kEpiWarpsT) : col_parts(EL::kWarps);
  const int cp2 = tc ? 1 : col_parts(EG::kWarps);
  int seg1 = 0;
  for (int c = 0; c < chunks; ++c) {
    const int na = (int)(tile_start(c + 1, n_a1, chunks) - tile_start(c, n_a1, chunks));
    const long long tot = (long long)na * n_b1;
    seg1 = std::max(seg1, cp1 * max_segments(na, n_b1, (int)std::min<long long>(units1, tot)));
  }
  const long long stride1 = (long long)n_a1 * res_rows;
  if ((long long)seg1 * stride1 > h->p1_cap)
    return fail(LORA_CE_ESTATE, "pass-1 partial buffer too small");
  GemmArgs g{};
  g.kblocks = kblocks;
  g.kstr = kblocks;
  g.kmain = kmain;
  Plan::schedule(g);
  g.rank_total = R;
  g.rank_off = 0;
  g.T = T;
  g.V = V;
  g.R = kRC;
  g.Vpad = h->Vpad;
  g.err = h->err;
  g.tok = h->tok;
  g.Bt = h->params + (long long)d * R;
  g.p_max = h->p_max;
  g.p_sum = h->p_sum;
  g.p_q = h->p_q;
  g.z_tgt = h->z_tgt;
  g.gBp = h->gBp;
  g.Tcap = stride1;
  g.stages = tc ? TcLayout::stages(kblocks, R) : 0;
  g.nml = h->nml;

  mark(h, kPhPrep);
  float* const Bfull = h->params + (long long)d * R;
  const long long tokc_stride = h->Tcap * kChunkRec, Bc_stride = h->Vpad * 16;
  if constexpr (kAug) {  // the vocabulary side of the augmentation, from the current B
    const int groups = Plan::kAugWidth / 8;
    const int blocks = (int)std::min<long long>((h->Vpad * groups + 255) / 256, 8LL * h->num_sms);
    lce_aug_b<R><<<blocks, 256, 0, st>>>(Bfull, h->Vpad, h->w_aug, Plan::kLayout, Plan::kAugWidth,
                                         rank_chunks ? h->Bc : nullptr, Bc_stride);
    ++launches;
  }
  if constexpr (R >= 8) {
    if (tc) {  // pass 1's rank operand B^T [hi ; lo]
      const int blocks = (int)std::min<long long>(((long long)V * R + 255) / 256, 8LL * h->num_sms);
      lce_xt_vocab<R><<<blocks, 256, 0, st>>>(V, h->Vpad, Bfull, h->xv);
      ++launches;
    }
  }
  // 1. per chunk of position blocks: convert h, U = h.A, per-position
  //    records; 2. pass 1 on those positions (per-position max / sum / q)
  for (int c = 0; c < chunks; ++c) {
    const int a_lo = (int)tile_start(c, n_a1, chunks), a_hi = (int)tile_start(c + 1, n_a1, chunks);
    const int t_lo = a_lo * res_rows;
    const int t_hi = c + 1 == chunks ? (int)Tpad : a_hi * res_rows;  // last chunk pads to Tpad
    if (chunk_ready) LCE_CUDA(cudaStreamWaitEvent(st, chunk_ready[c], 0));
    if constexpr (R >= 16) {  // lanes over ranks, one block per SM
      const int warps_blk = prep_wide_warps(R, d);
      const int per_block = warps_blk * prep_wide_rows(R);
      const int blocks = (int)std::min<long long>((t_hi - t_lo + per_block - 1) / per_block,
                                                  h->num_sms);
      lce_prep_wide<R><<<blocks, 32 * warps_blk, (size_t)prep_wide_smem(R, d), st>>>(
          dH, dtype, t_lo, t_hi, T, d, h->params, h->cfg.scale, dtg, V, h->h16, h->tok, h->err,
          kAug ? h->h_aug : nullptr, Plan::kLayout, Plan::kAugWidth,
          rank_chunks ? h->tokc : nullptr, tokc_stride);
      ++launches;
    } else {
      const int threads = 256;  // 8 warps per block, grid-stride over positions
      const int blocks = (int)std::min<long long>((t_hi - t_lo + 7) / 8, 4LL * h->num_sms);
      lce_prep<R><<<blocks, threads, (size_t)d * R * 4, st>>>(
          dH, dtype, t_lo, t_hi, T, d, h->params, h->cfg.scale, dtg, V, h->h16, h->tok, h->err,
          kAug ? h->h_aug : nullptr, Plan::kLayout, Plan::kAugWidth,
          rank_chunks ? h->tokc : nullptr, tokc_stride);
      ++launches;
    }
    if (c == 0) mark(h, kPhPass1);
    g.a0 = a_lo;
    g.n_a = a_hi - a_lo;
    g.n_b = n_b1;
    const long long tot = (long long)g.n_a * n_b1;
    const int Gc = (int)std::min<long long>(units1, tot);
    if constexpr (R >= 8) {
      if (tc) {
        int rc = launch_gemm_tc<1, R>(mapH_res, h->mapW_strT, mapHa_res, h->mapWa_strT, h->mapXv,
                                      g, Gc, st);
        if (rc) return rc;
        ++launches;
        continue;
      }
    }
    for (int rc0 = 0; rc0 < R; rc0 += kRC) {  // rank chunks (one pass below rank 32)
      g.rank_off = rc0;
      g.Bt = Plan::kChunked ? h->Bc + (rc0 / 16) * Bc_stride : Bfull;
      int rc = launch_gemm<EL>(mapH_res, pair == 2 ? h->mapW_res : h->mapW_str, mapHa_res,
                               pair == 2 ? h->mapWa_res : h->mapWa_str, g, Gc, pair, kblocks, st);
      if (rc) return rc;
      ++launches;
    }
  }
  g.a0 = 0;
  g.rank_off = 0;
  g.Bt = Bfull;
  // 3. merge partials -> M, 1/S, loss_t, dU
  mark(h, kPhCombine);
  if constexpr (R >= 16)  // lanes over ranks
    lce_combine_wide<R><<<(T + 7) / 8, 256, 0, st>>>(
        T, cp1, res_rows, n_b1, units1, chunks, stride1, h->p_max, h->p_sum, h->p_q, h->z_tgt,
        Bfull, h->cfg.scale, h->tok, h->dU, h->loss_tok, rank_chunks ? h->tokc : nullptr,
        tokc_stride);
  else
    lce_combine<R><<<(T + 7) / 8, 256, 0, st>>>(T, cp1, res_rows, n_b1, units1, chunks, stride1,
                                                h->p_max, h->p_sum, h->p_q, h->z_tgt, Bfull,
                                                h->cfg.scale, h->tok, h->dU, h->loss_tok,
                                                rank_chunks ? h->tokc : nullptr, tokc_stride);
  ++launches;
  // onehot part of dB (order-independent fixed-point sums)
  lce_onehot<R><<<(T + 63) / 64, 64, 0, st>>>(T, h->tok, h->corr_fx, h->err);
  ++launches;
  // 4. pass 2: dB per vocab row
  const int n_a2 = (V + res_rows - 1) / res_rows;
  const int n_b2 = tc ? (T + tc_bn(R) - 1) / tc_bn(R) : (int)(Tpad / kBN);
  const long long total2 = (long long)n_a2 * n_b2;
  const int G2 = (int)std::min<long long>(tc ? h->units2t : h->units2, total2);
  if (cp2 * max_segments(n_a2, n_b2, G2) > h->gbp_segs)
    return fail(LORA_CE_ESTATE, "pass-2 partial buffer too small");
  if constexpr (R >= 8) {
    if (tc) {  // pass 2's rank operand (s*U)^T [hi ; lo] and exponent offsets
      const int blocks = (int)std::min<long long>(((long long)T * R + 255) / 256, 8LL * h->num_sms);
      lce_xt_pos<R><<<blocks, 256, 0, st>>>(T, h->Tcap, h->tok, h->xt, h->nml);
      ++launches;
    }
  }
  mark(h, kPhPass2);
  g.n_a = n_a2;
  g.n_b = n_b2;
  if constexpr (R >= 8) {
    if (tc) {
      CUtensorMap mapH_strT, mapHa_strT, mapXt;
      if (!make_map(&mapH_strT, h->h16, T, d, tc_bn(R) / 2) ||
          !make_map(&mapHa_strT, h->h_aug, T, Plan::kAugWidth, tc_bn(R) / 2) ||
          !make_map_ld(&mapXt, h->xt, 2 * R, T, h->Tcap, R))
        return fail(LORA_CE_ECUDA, "cuTensorMapEncodeTiled failed for pass 2");
      int rc = launch_gemm_tc<2, R>(h->mapW_res, mapH_strT, h->mapWa_res, mapHa_strT, mapXt, g,
                                    G2, st);
      if (rc) return rc;
      ++launches;
    }
  }
  for (int rc0 = 0; rc0 < R && !tc; rc0 += kRC) {  // rank chunks: their own position records
    g.rank_off = rc0;
    g.tok = rank_chunks ? h->tokc + (rc0 / 16) * tokc_stride : h->tok;
    int rc = launch_gemm<EG>(h->mapW_res, pair == 2 ? mapH_res : mapH_str, h->mapWa_res,
                             pair == 2 ? mapHa_res : mapHa_str, g, G2, pair, kblocks, st);
    if (rc) return rc;
    ++launches;
  }
  g.tok = h->tok;
  // 5. dA partials, 6. pack gradient sums
  const int n_chunks = (T + kDAChunk - 1) / kDAChunk;
  mark(h, kPhDA);
  for (int rc0 = 0; rc0 < R; rc0 += kRC) {
    lce_dA_partial<kRC><<<dim3(n_chunks, (d + 63) / 64), dim3(32, da_rows(kRC)), 0, st>>>(
        T, d, h->h16, h->dU, h->gAp, R, rc0);
    ++launches;
  }
  const long long nparam = (long long)d * R + h->Vpad * R;
  const int32_t next_step = h->step + 1;
  AdamArgs aa = adam_args(h, nparam, next_step);
  // Without a collective the optimizer fuses into the finalize pass: the
  // whole update (no clip) or the clip's norm partials (clip).  With one,
  // the all-reduce has to sit between the gradient sums and the update.
  const int fin_blocks = (int)std::min<long long>((nparam + 255) / 256, kFinBlocksMax);
  const int fin_mode = h->comm ? kFinG : aa.clip > 0.f ? kFinNorm : kFinAdam;
  if (fin_mode == kFinNorm) aa.n_norm_parts = fin_blocks;
  mark(h, kPhFinalize);
  {
    auto fin = fin_mode == kFinAdam ? lce_finalize<R, kFinAdam>
               : fin_mode == kFinNorm ? lce_finalize<R, kFinNorm> : lce_finalize<R, kFinG>;
    fin<<<fin_blocks, 256, 0, st>>>(aa, T, cp2, d, V, h->Vpad, n_chunks, h->gAp, res_rows, n_b2,
                                    G2, h->gBp, h->corr_fx, h->loss_tok, h->Gbuf, h->params,
                                    h->mom1, h->mom2, h->gmean, h->norm_parts, d_loss_out);
    ++launches;
  }
  // 7. data-parallel sum over ranks
  mark(h, kPhAllReduce);
  if (h->comm) {
    ncclResult_t r = nccl().AllReduce(h->Gbuf, h->Gbuf, (size_t)(nparam + 2), ncclFloat, ncclSum,
                                      h->comm, st);
    if (r == ncclInProgress) r = nccl_settle(h->comm, h->comm_timeout_ms);
    if (r != ncclSuccess)
      return fail(LORA_CE_ENCCL, std::string("ncclAllReduce: ") + nccl_str(r));
  }
  // 8. clip norm (optional), 9. Adam
  mark(h, kPhNorm);
  if (fin_mode == kFinG && aa.clip > 0.f) {
    lce_sqnorm<<<256, 256, 0, st>>>(nparam, h->Gbuf, h->norm_parts);
    ++launches;
  }
  mark(h, kPhAdam);
  if (fin_mode != kFinAdam) {
    const int blocks = (int)std::min<long long>((nparam + 255) / 256, 8LL * h->num_sms);
    lce_adam<<<blocks, 256, 0, st>>>(aa, h->params, h->mom1, h->mom2, h->Gbuf, h->gmean,
                                     h->norm_parts, d_loss_out);
    ++launches;
  }
  mark(h, kNumPhases);
  LCE_CUDA(cudaGetLastError());
  h->step = next_step;
  h->launches = launches;
  h->last_T = T;
  return 0;
}

// K splits of a split-K product whose output has `tiles` 128 x 128 tiles:
// enough blocks for two per SM, each split a multiple of kWK long.
void wide_splits(long long K, long long tiles, int num_sms, int* splits, int* k_split) {
  long long s = (2LL * num_sms + tiles - 1) / tiles;
  s = std::max(1LL, std::min<long long>(s, kWMaxSplit));
  const long long ks = round_up((K + s - 1) / s, kWK);
  *k_split = (int)ks;
  *splits = (int)((K + ks - 1) / ks);
}

// The step for ranks 65..256 (kernel ranks 128 and 256), lora_ce_wide.cuh:
// per block of wide_p positions the logit rows are materialised, turned
// into p - onehot, and multiplied into dB and dU; dA follows over all
// positions; G is packed in the fused path's layout, and the all-reduce,
// clip and Adam are the fused path's kernels.
int run_step_wide(lora_ce_handle* h, const void* dH, int dtype, int T, const int32_t* dtg,
                  float* d_loss_out, int chunks, const cudaEvent_t* chunk_ready) {
  cudaStream_t st = h->stream;
  const int d = h->d, V = h->V, R = h->R;
  const long long Vpad = h->Vpad;
  const float scale = h->cfg.scale;
  const int grid_ew = 8 * h->num_sms;  // grid-stride element-wise kernels
  const unsigned rt = (unsigned)((R + kWTile - 1) / kWTile);
  int launches = 0;
  mark(h, kPhPrep);
  for (int c = 0; chunk_ready && c < chunks; ++c)
    LCE_CUDA(cudaStreamWaitEvent(st, chunk_ready[c], 0));
  lw_convert<<<grid_ew, 256, 0, st>>>(dH, dtype, (long long)T * d, h->h16);
  float* const Bt = h->params + (long long)d * R;
  lw_b_plain<<<grid_ew, 256, 0, st>>>(Bt, R, V, Vpad, h->w_Bp);
  LCE_CUDA(cudaMemsetAsync(h->w_dB, 0, (size_t)R * Vpad * 4, st));
  launches += 2;
  mark(h, kPhPass1);
  const unsigned vt = (unsigned)((V + kWTile - 1) / kWTile);
  for (int p0 = 0; p0 < T; p0 += h->wide_p) {
    const int Pb = std::min(h->wide_p, T - p0);
    const unsigned mt = (unsigned)((Pb + kWTile - 1) / kWTile);  // <= 4096: wide_p <= 2^19
    float* const sU = h->w_sU + (long long)p0 * R;
    // sU = s * (h16 . A)
    lw_gemm<<<dim3(rt, mt, 1), kWThreads, 0, st>>>(
        Pb, R, d, d, WideOp<__half, true>{h->h16 + (long long)p0 * d, d},
        WideOp<float, false>{h->params, R}, WideStore{sU, R, scale});
    // Z = h16 . W^T + sU . B
    lw_gemm<<<dim3(vt, mt, 1), kWThreads, 0, st>>>(
        Pb, V, d, d, WideOp<__half, true>{h->h16 + (long long)p0 * d, d},
        WideOp<__half, true>{h->W, d}, WideStore{h->w_Z, Vpad, 1.0f});
    lw_gemm<<<dim3(vt, mt, 1), kWThreads, 0, st>>>(Pb, V, R, R, WideOp<float, true>{sU, R},
                                                   WideOp<float, false>{h->w_Bp, Vpad},
                                                   WideAdd{h->w_Z, Vpad});
    // loss per position; Z <- p - onehot
    lw_softmax<<<Pb, kWSoftThreads, 0, st>>>(h->w_Z, Vpad, V, dtg, p0, h->loss_tok, h->err);
    // dB += sU^T . Z
    lw_gemm<<<dim3(vt, rt, 1), kWThreads, 0, st>>>(R, V, Pb, Pb, WideOp<float, false>{sU, R},
                                                   WideOp<float, false>{h->w_Z, Vpad},
                                                   WideAdd{h->w_dB, Vpad});
    // dU = s * (Z . B^T), split over the vocabulary
    int splits = 1, k_split = V;
    wide_splits(V, (long long)mt * rt, h->num_sms, &splits, &k_split);
    lw_gemm<<<dim3(rt, mt, (unsigned)splits), kWThreads, 0, st>>>(
        Pb, R, V, k_split, WideOp<float, true>{h->w_Z, Vpad}, WideOp<float, true>{h->w_Bp, Vpad},
        WideSplit{h->w_dUp, R, (long long)Pb * R});
    lw_reduce_du<<<grid_ew, 256, 0, st>>>(Pb, R, splits, h->w_dUp, scale,
                                          h->dU + (long long)p0 * R);
    launches += 7;
  }
  mark(h, kPhCombine);
  mark(h, kPhPass2);
  mark(h, kPhDA);
  // dA = h16^T . dU over all positions, split over positions
  int a_splits = 1, a_k = T;
  const unsigned dt = (unsigned)((d + kWTile - 1) / kWTile);
  wide_splits(T, (long long)dt * rt, h->num_sms, &a_splits, &a_k);
  lw_gemm<<<dim3(rt, dt, (unsigned)a_splits), kWThreads, 0, st>>>(
      d, R, T, a_k, WideOp<__half, false>{h->h16, d}, WideOp<float, false>{h->dU, R},
      WideSplit{h->w_dAp, R, (long long)d * R});
  ++launches;
  const long long nparam = (long long)d * R + Vpad * R;
  const int32_t next_step = h->step + 1;
  const AdamArgs aa = adam_args(h, nparam, next_step);
  mark(h, kPhFinalize);
  lw_pack<<<(int)std::min<long long>((nparam + 255) / 256, kFinBlocksMax), 256, 0, st>>>(
      d, R, V, Vpad, T, a_splits, h->w_dAp, h->w_dB, h->loss_tok, h->Gbuf);
  ++launches;
  mark(h, kPhAllReduce);
  if (h->comm) {
    ncclResult_t r = nccl().AllReduce(h->Gbuf, h->Gbuf, (size_t)(nparam + 2), ncclFloat, ncclSum,
                                      h->comm, st);
    if (r == ncclInProgress) r = nccl_settle(h->comm, h->comm_timeout_ms);
    if (r != ncclSuccess)
      return fail(LORA_CE_ENCCL, std::string("ncclAllReduce: ") + nccl_str(r));
  }
  mark(h, kPhNorm);
  if (aa.clip > 0.f) {
    lce_sqnorm<<<256, 256, 0, st>>>(nparam, h->Gbuf, h->norm_parts);
    ++launches;
  }
  mark(h, kPhAdam);
  lce_adam<<<(int)std::min<long long>((nparam + 255) / 256, 8LL * h->num_sms), 256, 0, st>>>(
      aa, h->params, h->mom1, h->mom2, h->Gbuf, h->gmean, h->norm_parts, d_loss_out);
  ++launches;
  mark(h, kNumPhases);
  LCE_CUDA(cudaGetLastError());
  h->step = next_step;
  h->launches = launches;
  h->last_T = T;
  return 0;
}

int dispatch_step(lora_ce_handle* h, const void* dH, int dtype, int T, const int32_t* dtg,
                  float* d_loss, int chunks = 1, const cudaEvent_t* chunk_ready = nullptr) {
  if (h->wide) return run_step_wide(h, dH, dtype, T, dtg, d_loss, chunks, chunk_ready);
  switch (h->R) {
    case 4: return run_step<4>(h, dH, dtype, T, dtg, d_loss, chunks, chunk_ready);
    case 8: return run_step<8>(h, dH, dtype, T, dtg, d_loss, chunks, chunk_ready);
    case 16: return run_step<16>(h, dH, dtype, T, dtg, d_loss, chunks, chunk_ready);
    case 32: return run_step<32>(h, dH, dtype, T, dtg, d_loss, chunks, chunk_ready);
    case 64: return run_step<64>(h, dH, dtype, T, dtg, d_loss, chunks, chunk_ready);
  }
  return fail(LORA_CE_EINVAL, "unsupported rank");
}

int check_step_args(lora_ce_handle* h, const void* H, int dtype, int T, const int32_t* tg) {
  if (!h) return fail(LORA_CE_EINVAL, "null handle");
  if (h->poisoned) return fail(LORA_CE_ESTATE, "handle poisoned by an earlier error");
  if (!h->have_weight) return fail(LORA_CE_ESTATE, "lora_ce_set_weight_f16 not called");
  if (!H || !tg) return fail(LORA_CE_EINVAL, "null input");
  if (dtype < 0 || dtype > 2) return fail(LORA_CE_EINVAL, "bad hidden-state dtype");
  if (T < 1 || T > h->cfg.max_tokens) return fail(LORA_CE_EINVAL, "T out of range");
  if ((reinterpret_cast<uintptr_t>(H) & 15) != 0)
    return fail(LORA_CE_EINVAL, "hidden states must be 16-byte aligned");
  return 0;
}

int elt_size(int dtype) { return dtype == LORA_CE_F32 ? 4 : 2; }

// Abort the communicator after a failed or expired collective: NCCL's
// kernels end, the handle's streams drain, the graphs (which hold the
// communicator's calls) are dropped and the handle is poisoned.
int abort_comm(lora_ce_handle* h, const std::string& why) {
  nccl().CommAbort(h->comm);
  h->comm = nullptr;
  h->poisoned = true;
  // the streams should drain once NCCL's kernels have ended; the wait for
  // that is bounded too, and streams that do not drain are left alone (the
  // handle then keeps its device memory at destroy rather than block)
  const Clock::time_point t0 = Clock::now();
  while (cudaStreamQuery(h->stream) == cudaErrorNotReady ||
         cudaStreamQuery(h->cstream) == cudaErrorNotReady) {
    if (ms_since(t0) > h->comm_timeout_ms) {
      h->stuck = true;
      return fail(LORA_CE_ENCCL, why + "; the handle's streams did not drain after the abort");
    }
    std::this_thread::yield();
  }
  cudaGetLastError();
  drop_graphs(h);
  return fail(LORA_CE_ENCCL, why);
}

// Wait for the handle's stream.  With a communicator the wait is bounded:
// the stream is polled together with the communicator's asynchronous
// error, and a collective that has not completed within comm_timeout_ms
// (a peer that left, a failed link) is aborted.
int wait_stream(lora_ce_handle* h) {
  if (!h->comm) {
    LCE_CUDA(cudaStreamSynchronize(h->stream));
    return 0;
  }
  const Clock::time_point t0 = Clock::now();
  for (;;) {
    const cudaError_t q = cudaStreamQuery(h->stream);
    if (q == cudaSuccess) return 0;
    if (q != cudaErrorNotReady) return fail(LORA_CE_ECUDA, cudaGetErrorString(q));
    ncclResult_t ae = ncclSuccess;
    nccl().CommGetAsyncError(h->comm, &ae);
    if (ae != ncclSuccess && ae != ncclInProgress)
      return abort_comm(h, std::string("NCCL asynchronous error: ") + nccl_str(ae));
    if (ms_since(t0) > h->comm_timeout_ms)
      return abort_comm(h, "collective timed out (a peer rank did not take part); "
                           "communicator aborted, handle poisoned");
    std::this_thread::yield();
  }
}

int check_device_error(lora_ce_handle* h) {
  int e = 0;
  LCE_CUDA(cudaMemcpyAsync(&e, h->err, sizeof(int), cudaMemcpyDeviceToHost, h->stream));
  if (int rc = wait_stream(h)) return rc;
  if (e != 0) {
    h->poisoned = true;
    char buf[96];
    snprintf(buf, sizeof buf, "device error %d (%s)", e,
             e == kErrTarget      ? "target id out of range"
             : e == kErrRange     ? "s*U out of the supported range"
             : e == kErrSmemAlign ? "shared memory base not 1024-byte aligned"
                                  : "bounded wait expired");
    return fail(LORA_CE_EDEVICE, buf);
  }
  return 0;
}

}  // namespace

namespace {

void drop_graph(lora_ce_handle::StepGraph& gph) {
  if (gph.exec) cudaGraphExecDestroy(gph.exec);
  if (gph.graph) cudaGraphDestroy(gph.graph);
  gph = lora_ce_handle::StepGraph{};
}

void drop_graphs(lora_ce_handle* h) {
  for (auto& gph : h->graphs) drop_graph(gph);
}

// Everything one step enqueues on the handle's streams.  Host-input steps
// (H, targets in host memory) copy them in (h in chunks on the copy stream,
// see run_step) and read [loss, error code] back into res_host;
// device-input steps write the loss to d_loss.
int enqueue_step(lora_ce_handle* h, bool host, const void* H, int dtype, int T,
                 const int32_t* targets, float* d_loss) {
  if (!host) return dispatch_step(h, H, dtype, T, targets, d_loss);
  if (h->ctime) LCE_CUDA(cudaEventRecord(h->tev[0], h->stream));
  LCE_CUDA(cudaMemcpyAsync(h->in_tgt, targets, (size_t)T * 4, cudaMemcpyHostToDevice, h->stream));
  const int res_rows = kBM * h->pair;
  const int n_a1 = (T + res_rows - 1) / res_rows;
  const int chunks = h->prof ? 1 : step_chunks(n_a1);
  const size_t row_bytes = (size_t)h->d * elt_size(dtype);
  LCE_CUDA(cudaEventRecord(h->ev_start, h->stream));  // the previous step is done with in_H
  LCE_CUDA(cudaStreamWaitEvent(h->cstream, h->ev_start, 0));
  if (h->ctime) LCE_CUDA(cudaEventRecord(h->tev[1], h->cstream));
  for (int c = 0; c < chunks; ++c) {
    const long long t_lo = tile_start(c, n_a1, chunks) * res_rows;
    const long long t_hi = std::min<long long>(T, tile_start(c + 1, n_a1, chunks) * res_rows);
    LCE_CUDA(cudaMemcpyAsync(static_cast<char*>(h->in_H) + t_lo * row_bytes,
                             static_cast<const char*>(H) + t_lo * row_bytes,
                             (size_t)(t_hi - t_lo) * row_bytes, cudaMemcpyHostToDevice, h->cstream));
    LCE_CUDA(cudaEventRecord(h->ev_chunk[c], h->cstream));
    if (h->ctime) LCE_CUDA(cudaEventRecord(h->tev[2 + c], h->cstream));
  }
  h->ctime_chunks = chunks;
  int rc = dispatch_step(h, h->in_H, dtype, T, h->in_tgt, h->d_loss, chunks, h->ev_chunk);
  if (rc) return rc;
  LCE_CUDA(cudaMemcpyAsync(h->d_loss + 1, h->err, 4, cudaMemcpyDeviceToDevice, h->stream));
  LCE_CUDA(cudaMemcpyAsync(h->res_host, h->d_loss, 8, cudaMemcpyDeviceToHost, h->stream));
  if (h->ctime) LCE_CUDA(cudaEventRecord(h->tev[kMaxChunks + 2], h->stream));
  return 0;
}

// The cached graph for these arguments, captured on first use; nullptr when
// capture is not possible (the caller then launches the step directly).
lora_ce_handle::StepGraph* step_graph(lora_ce_handle* h, bool host, const void* H, int dtype,
                                      int T, const int32_t* targets, float* d_loss) {
  for (auto& gph : h->graphs)
    if (gph.valid && gph.host == host && gph.T == T && gph.dtype == dtype && gph.H == H &&
        gph.tgt == targets && gph.d_loss == d_loss) {
      gph.last_use = ++h->graph_clock;
      return &gph;
    }
  lora_ce_handle::StepGraph* slot = &h->graphs[0];
  for (auto& gph : h->graphs)
    if (!gph.valid || gph.last_use < slot->last_use) slot = &gph;
  drop_graph(*slot);
  // capturing enqueues nothing: restore the host-side step bookkeeping after
  const int32_t step = h->step, launches = h->launches;
  const int last_T = h->last_T;
  if (cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeRelaxed) != cudaSuccess) return nullptr;
  const int rc = enqueue_step(h, host, H, dtype, T, targets, d_loss);
  const int new_launches = h->launches;
  h->step = step;
  h->launches = launches;
  h->last_T = last_T;
  cudaGraph_t graph = nullptr;
  const cudaError_t ce = cudaStreamEndCapture(h->stream, &graph);
  if (rc || ce != cudaSuccess || !graph) {
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();
    return nullptr;
  }
  cudaGraphExec_t exec = nullptr;
  if (cudaGraphInstantiate(&exec, graph, 0) != cudaSuccess) {
    cudaGraphDestroy(graph);
    cudaGetLastError();
    return nullptr;
  }
  // the Adam node, whose bias corrections change every step
  size_t n = 0;
  cudaGraphGetNodes(graph, nullptr, &n);
  std::vector<cudaGraphNode_t> nodes(n);
  cudaGraphGetNodes(graph, nodes.data(), &n);
  // (lce_adam, or the finalize kernel with the update fused in; both take
  // the AdamArgs as their first parameter)
  cudaGraphNode_t adam = nullptr;
  cudaKernelNodeParams ap{};
  int nargs = 0;
  const void* fused = fused_finalize_fn(h->R);
  for (cudaGraphNode_t nd : nodes) {
    cudaGraphNodeType ty;
    if (cudaGraphNodeGetType(nd, &ty) != cudaSuccess || ty != cudaGraphNodeTypeKernel) continue;
    cudaKernelNodeParams p{};
    if (cudaGraphKernelNodeGetParams(nd, &p) != cudaSuccess) continue;
    if (p.func == reinterpret_cast<void*>(lce_adam) || p.func == fused) {
      adam = nd;
      ap = p;
      nargs = p.func == fused ? kFinalizeArgs : kAdamArgs;
    }
  }
  if (!adam || !ap.kernelParams) {
    cudaGraphExecDestroy(exec);
    cudaGraphDestroy(graph);
    return nullptr;
  }
  slot->valid = true;
  slot->host = host;
  slot->T = T;
  slot->dtype = dtype;
  slot->H = H;
  slot->tgt = targets;
  slot->d_loss = d_loss;
  slot->graph = graph;
  slot->exec = exec;
  slot->adam = adam;
  slot->adam_p = ap;
  slot->adam_nargs = nargs;
  slot->nparam = (long long)h->d * h->R + h->Vpad * h->R;
  slot->launches = new_launches;
  slot->last_use = ++h->graph_clock;
  return slot;
}

// Replay: set this step's Adam arguments, launch the graph.
int launch_step_graph(lora_ce_handle* h, lora_ce_handle::StepGraph* gph, int T) {
  // the captured AdamArgs with this step's bias corrections; every other
  // argument keeps its captured value
  AdamArgs aa = *static_cast<const AdamArgs*>(gph->adam_p.kernelParams[0]);
  const AdamArgs fresh = adam_args(h, gph->nparam, h->step + 1);
  aa.b1t = fresh.b1t;
  aa.b2t = fresh.b2t;
  void* args[kFinalizeArgs];
  args[0] = &aa;
  for (int i = 1; i < gph->adam_nargs; ++i) args[i] = gph->adam_p.kernelParams[i];
  cudaKernelNodeParams p = gph->adam_p;
  p.kernelParams = args;
  p.extra = nullptr;
  LCE_CUDA(cudaGraphExecKernelNodeSetParams(gph->exec, gph->adam, &p));
  LCE_CUDA(cudaGraphLaunch(gph->exec, h->stream));
  h->step += 1;
  h->launches = gph->launches;
  h->last_T = T;
  return 0;
}

int run_or_replay(lora_ce_handle* h, bool host, const void* H, int dtype, int T,
                  const int32_t* targets, float* d_loss) {
  // timed host-input steps launch directly (their events are plain records)
  if (h->use_graphs && !h->prof && !(host && h->ctime)) {
    lora_ce_handle::StepGraph* gph = step_graph(h, host, H, dtype, T, targets, d_loss);
    if (gph) return launch_step_graph(h, gph, T);
    h->use_graphs = false;  // capture failed: launch directly from now on
  }
  return enqueue_step(h, host, H, dtype, T, targets, d_loss);
}

}  // namespace

namespace {

// Buffers and streams of a wide-rank handle (ranks 65..256).  The logit
// rows of one position block take at most 512 MB.
int create_wide(lora_ce_handle* h) {
  h->wide = true;
  h->tc = false;
  h->units1 = h->units2 = 1;
  const int R = h->R, d = h->d;
  const long long V = h->V, Vpad = h->Vpad, Tcap = h->Tcap;
  const long long rows = (512LL << 20) / (Vpad * 4) / kWTile * kWTile;
  h->wide_p = (int)std::max<long long>(kWTile, std::min<long long>(rows, Tcap));
  const long long P = h->wide_p;
  const long long nparam = (long long)d * R + Vpad * R;
  // dU split partials: the most (K splits x block positions) any block can
  // use, over block sizes 1..P (the splits depend on its 128-row tiles)
  long long dup = 0;
  {
    const long long rt = (R + kWTile - 1) / kWTile;
    for (long long mt = 1; (mt - 1) * kWTile < P; ++mt) {
      int splits = 1, k_split = 0;
      wide_splits(V, mt * rt, h->num_sms, &splits, &k_split);
      dup = std::max(dup, (long long)splits * std::min(P, mt * kWTile));
    }
  }
  int rc = 0;
  if (!rc) rc = dalloc(&h->W, (size_t)V * d);
  if (!rc) rc = dalloc(&h->h16, (size_t)Tcap * d);
  if (!rc) rc = dalloc(&h->params, (size_t)nparam);
  if (!rc) rc = dalloc(&h->mom1, (size_t)nparam);
  if (!rc) rc = dalloc(&h->mom2, (size_t)nparam);
  if (!rc) rc = dalloc(&h->Gbuf, (size_t)nparam + 2);
  if (!rc) rc = dalloc(&h->gmean, (size_t)nparam);
  if (!rc) rc = dalloc(&h->loss_tok, (size_t)Tcap);
  if (!rc) rc = dalloc(&h->dU, (size_t)Tcap * R);
  if (!rc) rc = dalloc(&h->norm_parts, kFinBlocksMax);
  if (!rc) rc = dalloc(&h->err, 1);
  if (!rc) rc = dalloc(&h->d_loss, 2);
  if (!rc) rc = dalloc(reinterpret_cast<char**>(&h->in_H), (size_t)Tcap * d * 4);
  if (!rc) rc = dalloc(&h->in_tgt, (size_t)Tcap);
  if (!rc) rc = dalloc(&h->w_sU, (size_t)Tcap * R);
  if (!rc) rc = dalloc(&h->w_Z, (size_t)P * Vpad);
  if (!rc) rc = dalloc(&h->w_Bp, (size_t)R * Vpad);
  if (!rc) rc = dalloc(&h->w_dB, (size_t)R * Vpad);
  if (!rc) rc = dalloc(&h->w_dUp, (size_t)dup * R);
  if (!rc) rc = dalloc(&h->w_dAp, (size_t)kWMaxSplit * d * R);
  if (!rc && (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess ||
              cudaStreamCreateWithFlags(&h->cstream, cudaStreamNonBlocking) != cudaSuccess))
    rc = fail(LORA_CE_ECUDA, "cudaStreamCreate failed");
  if (!rc && cudaMallocHost(reinterpret_cast<void**>(&h->res_host), 16) != cudaSuccess)
    rc = fail(LORA_CE_ENOMEM, "cudaMallocHost failed");
  if (!rc && cudaEventCreateWithFlags(&h->ev_start, cudaEventDisableTiming) != cudaSuccess)
    rc = fail(LORA_CE_ECUDA, "cudaEventCreate failed");
  for (int c = 0; c < kMaxChunks && !rc; ++c)
    if (cudaEventCreateWithFlags(&h->ev_chunk[c], cudaEventDisableTiming) != cudaSuccess)
      rc = fail(LORA_CE_ECUDA, "cudaEventCreate failed");
  return rc;
}

}  // namespace

extern "C" {

void lora_ce_default_config(lora_ce_config* c, int32_t dim, int32_t vocab, int32_t rank,
                            int32_t max_tokens) {
  if (!c) return;
  memset(c, 0, sizeof(*c));
  c->dim = dim;
  c->vocab = vocab;
  c->rank = rank;
  c->scale = rank > 0 ? 16.0f / (float)rank : 0.f;
  c->lr = 1e-4f;
  c->beta1 = 0.9f;
  c->beta2 = 0.999f;
  c->eps = 1e-8f;
  c->weight_decay = 0.f;
  c->clip_norm = 0.f;
  c->max_tokens = max_tokens;
  c->device = 0;
}

const char* lora_ce_last_error(void) { return g_last_error.c_str(); }

int lora_ce_create(const lora_ce_config* cfg, lora_ce_handle** out) {
  if (!out) return fail(LORA_CE_EINVAL, "null output pointer");
  *out = nullptr;
  int rc = check_cfg(cfg);
  if (rc) return rc;
  LCE_CUDA(cudaSetDevice(cfg->device));
  cudaDeviceProp prop;
  LCE_CUDA(cudaGetDeviceProperties(&prop, cfg->device));
  if (prop.major != 10) return fail(LORA_CE_ECUDA, "this library runs on sm_100 (B200) only");
  if (!encode_fn()) return fail(LORA_CE_ECUDA, "cuTensorMapEncodeTiled unavailable");
  lora_ce_handle* h = new (std::nothrow) lora_ce_handle();
  if (!h) return fail(LORA_CE_ENOMEM, "host allocation failed");
  h->cfg = *cfg;
  h->r = cfg->rank;
  h->R = kernel_rank(cfg->rank);
  h->d = cfg->dim;
  h->V = cfg->vocab;
  h->Vpad = round_up(cfg->vocab, kBN);
  h->Tcap = round_up(cfg->max_tokens, kBN);
  h->num_sms = prop.multiProcessorCount;
  {
    const char* e = getenv("LORA_CE_CTA_PAIR");  // "1": single-CTA tiles (comparison runs)
    h->pair = (e && e[0] == '1') ? 1 : 2;
    const char* gr = getenv("LORA_CE_GRAPHS");  // "0": launch every step directly
    h->use_graphs = !(gr && gr[0] == '0');
    // Tensor-core rank sums from rank LCE_TC_MIN_RANK up (below it the
    // per-logit epilogues are faster); LORA_CE_TC=0 turns them off, =1
    // turns them on from rank 8 (comparison and parity runs).
    const char* tc = getenv("LORA_CE_TC");
    const int tc_min = tc && tc[0] == '1' ? 8 : LCE_TC_MIN_RANK;
    h->tc = h->pair == 2 && h->R >= tc_min && !(tc && tc[0] == '0');
  }
  if (h->R > kMaxFusedRank) {
    rc = create_wide(h);
    if (rc) {
      free_all(h);
      free_streams(h);
      delete h;
      return rc;
    }
    *out = h;
    return 0;
  }
  const int R = h->R, d = h->d;
  const int res_rows = kBM * h->pair;
  {
    int u1 = 0, u2 = 0;
    switch (R) {
      case 4: plan_units<4>(h, &u1, &u2); break;
      case 8: plan_units<8>(h, &u1, &u2); break;
      case 16: plan_units<16>(h, &u1, &u2); break;
      case 32: plan_units<32>(h, &u1, &u2); break;
      default: plan_units<64>(h, &u1, &u2); break;
    }
    if (u1 < 1 || u2 < 1) {
      delete h;
      return fail(LORA_CE_ECUDA, "GEMM kernels cannot be made resident on this device");
    }
    h->units1 = u1;
    h->units2 = u2;
  }
  const long long V = h->V, Vpad = h->Vpad, Tcap = h->Tcap;
  // worst-case partial-buffer sizes over every T <= max_tokens
  long long p1 = 0;
  int s2 = 1;
  const int n_b1 = (int)(Vpad / kBN), n_a2 = (int)((V + res_rows - 1) / res_rows);
  for (int n_a1 = 1; (long long)n_a1 * res_rows < Tcap + res_rows; ++n_a1) {
    // one pass-1 launch (device-input steps) or the chunked launches of a
    // host-input step: slots per position are the most over the chunks
    int seg = 0;
    for (int chunks : {1, step_chunks(n_a1)}) {
      for (int c = 0; c < chunks; ++c) {
        const int na = (int)(tile_start(c + 1, n_a1, chunks) - tile_start(c, n_a1, chunks));
        const long long total = (long long)na * n_b1;
        const int G = (int)std::min<long long>(h->units1, total);
        seg = std::max(seg, max_segments(na, n_b1, G));
      }
    }
    p1 = std::max<long long>(p1, (long long)col_parts(16) * seg * n_a1 * res_rows);
    if (h->tc) {  // 192-column vocab tiles
      const int n_b1t = (int)((V + tc_bn(R) - 1) / tc_bn(R));
      int segt = 0;
      for (int chunks : {1, step_chunks(n_a1)}) {
        for (int c = 0; c < chunks; ++c) {
          const int na = (int)(tile_start(c + 1, n_a1, chunks) - tile_start(c, n_a1, chunks));
          const long long total = (long long)na * n_b1t;
          const int G = (int)std::min<long long>(h->units1t, total);
          segt = std::max(segt, max_segments(na, n_b1t, G));
        }
      }
      p1 = std::max<long long>(p1, (long long)col_parts(kEpiWarpsT) * segt * n_a1 * res_rows);
    }
  }
  for (int n_b2 = 1; (long long)n_b2 * kBN <= Tcap; ++n_b2) {
    const long long total = (long long)n_a2 * n_b2;
    const int G = (int)std::min<long long>(h->units2, total);
    s2 = std::max(s2, col_parts(16) * max_segments(n_a2, n_b2, G));
  }
  if (h->tc) {  // 192-column position tiles, one slot per segment
    for (int n_b2 = 1; (long long)(n_b2 - 1) * tc_bn(R) < Tcap; ++n_b2) {
      const long long total = (long long)n_a2 * n_b2;
      const int G = (int)std::min<long long>(h->units2t, total);
      s2 = std::max(s2, max_segments(n_a2, n_b2, G));
    }
  }
  h->p1_cap = p1;
  h->gbp_segs = s2;
  const long long nparam_pad = (long long)d * R + Vpad * R;
  const long long nparam = nparam_pad;
  rc = 0;
  if (!rc) rc = dalloc(&h->W, (size_t)V * d);
  if (!rc) rc = dalloc(&h->h16, (size_t)Tcap * d);
  if (!rc) rc = dalloc(&h->tok, (size_t)Tcap * tok_stride(R));
  if (!rc) rc = dalloc(&h->params, (size_t)nparam_pad);
  if (!rc) rc = dalloc(&h->mom1, (size_t)nparam_pad);
  if (!rc) rc = dalloc(&h->mom2, (size_t)nparam_pad);
  if (!rc) rc = dalloc(&h->Gbuf, (size_t)nparam + 2);
  if (!rc) rc = dalloc(&h->gmean, (size_t)nparam);
  if (!rc) rc = dalloc(&h->p_max, (size_t)p1);
  if (!rc) rc = dalloc(&h->p_sum, (size_t)p1);
  if (!rc) rc = dalloc(&h->p_q, (size_t)p1 * R);
  if (!rc) rc = dalloc(&h->z_tgt, (size_t)Tcap);
  if (!rc) rc = dalloc(&h->loss_tok, (size_t)Tcap);
  if (!rc) rc = dalloc(&h->dU, (size_t)Tcap * R);
  if (!rc) rc = dalloc(&h->gAp, (size_t)((Tcap + kDAChunk - 1) / kDAChunk) * d * R);
  if (!rc) rc = dalloc(&h->gBp, (size_t)s2 * Vpad * R);
  if (!rc) rc = dalloc(&h->corr_fx, (size_t)Vpad * R);
  if (!rc) rc = dalloc(&h->norm_parts, kFinBlocksMax);
  if (!rc) rc = dalloc(&h->err, 1);
  if (!rc) rc = dalloc(&h->d_loss, 2);
  if (!rc) rc = dalloc(reinterpret_cast<char**>(&h->in_H), (size_t)Tcap * d * 4);
  if (!rc) rc = dalloc(&h->in_tgt, (size_t)Tcap);
  const int aug_width = aug_width_of(R);
  const bool aug = aug_width > 0;
  if (!rc && aug) rc = dalloc(&h->w_aug, (size_t)Vpad * aug_width);
  if (!rc && aug) rc = dalloc(&h->h_aug, (size_t)Tcap * aug_width);
  if (!rc && R > 16 && !h->tc) rc = dalloc(&h->Bc, (size_t)(R / 16) * Vpad * 16);
  if (!rc && R > 16 && !h->tc) rc = dalloc(&h->tokc, (size_t)(R / 16) * Tcap * kChunkRec);
  if (!rc && h->tc) rc = dalloc(&h->xv, (size_t)2 * R * Vpad);
  if (!rc && h->tc) rc = dalloc(&h->xt, (size_t)2 * R * Tcap);
  if (!rc && h->tc) rc = dalloc(&h->nml, (size_t)Tcap + kMaxBNT);
  if (!rc && (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess ||
              cudaStreamCreateWithFlags(&h->cstream, cudaStreamNonBlocking) != cudaSuccess))
    rc = fail(LORA_CE_ECUDA, "cudaStreamCreate failed");
  if (!rc && cudaMallocHost(reinterpret_cast<void**>(&h->res_host), 16) != cudaSuccess)
    rc = fail(LORA_CE_ENOMEM, "cudaMallocHost failed");
  if (!rc && cudaEventCreateWithFlags(&h->ev_start, cudaEventDisableTiming) != cudaSuccess)
    rc = fail(LORA_CE_ECUDA, "cudaEventCreate failed");
  for (int c = 0; c < kMaxChunks && !rc; ++c)
    if (cudaEventCreateWithFlags(&h->ev_chunk[c], cudaEventDisableTiming) != cudaSuccess)
      rc = fail(LORA_CE_ECUDA, "cudaEventCreate failed");
  if (!rc && !(make_map(&h->mapW_res, h->W, V, d, kBM) && make_map(&h->mapW_str, h->W, V, d, kBN)))
    rc = fail(LORA_CE_ECUDA, "cuTensorMapEncodeTiled failed for W");
  if (!rc && aug && !(make_map(&h->mapWa_res, h->w_aug, V, aug_width, kBM) &&
                       make_map(&h->mapWa_str, h->w_aug, V, aug_width, kBN)))
    rc = fail(LORA_CE_ECUDA, "cuTensorMapEncodeTiled failed for the rank augmentation");
  if (!rc && h->tc &&
      !(make_map(&h->mapW_strT, h->W, V, d, tc_bn(R) / 2) &&
        make_map(&h->mapWa_strT, h->w_aug, V, aug_width, tc_bn(R) / 2) &&
        make_map_ld(&h->mapXv, h->xv, 2 * R, V, Vpad, R)))
    rc = fail(LORA_CE_ECUDA, "cuTensorMapEncodeTiled failed for the tensor-core rank sums");
  if (!aug) {  // never read without augmentation; any valid map fills the kernel parameter
    h->mapWa_res = h->mapW_res;
    h->mapWa_str = h->mapW_str;
  }
  if (rc) {
    free_all(h);
    free_streams(h);
    delete h;
    return rc;
  }
  *out = h;
  return 0;
}

int lora_ce_destroy(lora_ce_handle* h) {
  if (!h) return 0;
  cudaSetDevice(h->cfg.device);
  if (h->stuck) {  // never block on streams an aborted collective left busy
    delete h;
    return fail(LORA_CE_ENCCL, "handle destroyed with busy streams; its device memory is kept");
  }
  if (h->stream) cudaStreamSynchronize(h->stream);
  if (h->cstream) cudaStreamSynchronize(h->cstream);
  drop_graphs(h);  // graphs holding NCCL calls go before the communicator
  if (h->comm) {
    // finalize (flush), bounded; a communicator that does not settle is aborted
    ncclResult_t r = nccl().CommFinalize(h->comm);
    if (r == ncclInProgress) r = nccl_settle(h->comm, h->comm_timeout_ms);
    if (r == ncclSuccess)
      nccl().CommDestroy(h->comm);
    else
      nccl().CommAbort(h->comm);
    h->comm = nullptr;
  }
  for (cudaEvent_t e : h->ev)
    if (e) cudaEventDestroy(e);
  for (cudaEvent_t e : h->tev)
    if (e) cudaEventDestroy(e);
  free_all(h);
  free_streams(h);
  delete h;
  return 0;
}

int lora_ce_set_weight_f16(lora_ce_handle* h, const uint16_t* W) {
  if (!h || !W) return fail(LORA_CE_EINVAL, "null argument");
  LCE_CUDA(cudaSetDevice(h->cfg.device));
  LCE_CUDA(cudaMemcpyAsync(h->W, W, (size_t)h->V * h->d * 2, cudaMemcpyHostToDevice, h->stream));
  LCE_CUDA(cudaStreamSynchronize(h->stream));
  h->have_weight = true;
  return 0;
}

int lora_ce_set_weight_q4k(lora_ce_handle* h, const void* blocks) {
  if (!h || !blocks) return fail(LORA_CE_EINVAL, "bad argument");
  const long long n = (long long)h->V * h->d;
  if (n % 256 != 0) return fail(LORA_CE_EINVAL, "vocab*dim must be a multiple of 256 for Q4_K");
  LCE_CUDA(cudaSetDevice(h->cfg.device));
  void* tmp = nullptr;
  if (cudaMalloc(&tmp, (size_t)(n / 256) * 144) != cudaSuccess)
    return fail(LORA_CE_ENOMEM, "cudaMalloc failed");
  int rc = 0;
  if (cudaMemcpyAsync(tmp, blocks, (size_t)(n / 256) * 144, cudaMemcpyHostToDevice, h->stream) !=
      cudaSuccess)
    rc = fail(LORA_CE_ECUDA, "Q4_K upload failed");
  if (!rc) {
    rc = lora_ce_q4k_dequant_device(tmp, n / 256, h->W, LORA_CE_F16, h->stream);
    if (rc) fail(rc, lora_ce_q4k_last_error());
  }
  if (cudaStreamSynchronize(h->stream) != cudaSuccess && !rc)
    rc = fail(LORA_CE_ECUDA, "Q4_K dequantisation failed");
  cudaFree(tmp);
  if (!rc) h->have_weight = true;
  return rc;
}

int lora_ce_set_adapter(lora_ce_handle* h, const float* A, const float* B, int32_t step) {
  if (!h || !A || !B || step < 0) return fail(LORA_CE_EINVAL, "bad argument");
  LCE_CUDA(cudaSetDevice(h->cfg.device));
  const int r = h->r, R = h->R, d = h->d, V = h->V;
  std::vector<float> Bt((size_t)h->Vpad * R, 0.f);
  for (int j = 0; j < r; ++j)
    for (int v = 0; v < V; ++v) Bt[(size_t)bidx(v, j, R)] = B[(size_t)j * V + v];
  const size_t nA = (size_t)d * R;
  std::vector<float> Ap(nA, 0.f);
  for (int i = 0; i < d; ++i)
    for (int j = 0; j < r; ++j) Ap[(size_t)i * R + j] = A[(size_t)i * r + j];
  LCE_CUDA(cudaMemcpyAsync(h->params, Ap.data(), nA * 4, cudaMemcpyHostToDevice, h->stream));
  LCE_CUDA(cudaMemcpyAsync(h->params + nA, Bt.data(), Bt.size() * 4, cudaMemcpyHostToDevice,
                           h->stream));
  const size_t np = nA + Bt.size();
  LCE_CUDA(cudaMemsetAsync(h->mom1, 0, np * 4, h->stream));
  LCE_CUDA(cudaMemsetAsync(h->mom2, 0, np * 4, h->stream));
  LCE_CUDA(cudaStreamSynchronize(h->stream));
  h->step = step;
  return 0;
}

int lora_ce_set_scale(lora_ce_handle* h, float scale) {
  if (!h || !std::isfinite(scale)) return fail(LORA_CE_EINVAL, "bad argument");
  if (scale != h->cfg.scale) drop_graphs(h);  // captured steps carry the scale
  h->cfg.scale = scale;
  return 0;
}

int lora_ce_get_adapter(lora_ce_handle* h, float* A, float* B, int32_t* step) {
  if (!h) return fail(LORA_CE_EINVAL, "null handle");
  LCE_CUDA(cudaSetDevice(h->cfg.device));
  int rc = check_device_error(h);
  if (rc) return rc;
  const int r = h->r, R = h->R, d = h->d, V = h->V;
  if (A) {
    std::vector<float> Ap((size_t)d * R);
    LCE_CUDA(cudaMemcpy(Ap.data(), h->params, Ap.size() * 4, cudaMemcpyDeviceToHost));
    for (int i = 0; i < d; ++i)
      for (int j = 0; j < r; ++j) A[(size_t)i * r + j] = Ap[(size_t)i * R + j];
  }
  if (B) {
    std::vector<float> Bt((size_t)h->Vpad * R);
    LCE_CUDA(cudaMemcpy(Bt.data(), h->params + (size_t)d * R, Bt.size() * 4,
                        cudaMemcpyDeviceToHost));
    for (int j = 0; j < r; ++j)
      for (int v = 0; v < V; ++v) B[(size_t)j * V + v] = Bt[(size_t)bidx(v, j, R)];
  }
  if (step) *step = h->step;
  return 0;
}

int lora_ce_get_grads(lora_ce_handle* h, float* gA, float* gB, float* loss_sum, float* n_pred) {
  if (!h) return fail(LORA_CE_EINVAL, "null handle");
  LCE_CUDA(cudaSetDevice(h->cfg.device));
  int rc = check_device_error(h);
  if (rc) return rc;
  const int r = h->r, R = h->R, d = h->d, V = h->V;
  if (gA) {
    std::vector<float> t((size_t)d * R);
    LCE_CUDA(cudaMemcpy(t.data(), h->gmean, t.size() * 4, cudaMemcpyDeviceToHost));
    for (int i = 0; i < d; ++i)
      for (int j = 0; j < r; ++j) gA[(size_t)i * r + j] = t[(size_t)i * R + j];
  }
  if (gB) {
    std::vector<float> t((size_t)h->Vpad * R);
    LCE_CUDA(cudaMemcpy(t.data(), h->gmean + (size_t)d * R, t.size() * 4, cudaMemcpyDeviceToHost));
    for (int j = 0; j < r; ++j)
      for (int v = 0; v < V; ++v) gB[(size_t)j * V + v] = t[(size_t)bidx(v, j, R)];
  }
  const long long nparam = (long long)d * R + h->Vpad * R;
  float tail[2];
  LCE_CUDA(cudaMemcpy(tail, h->Gbuf + nparam, 8, cudaMemcpyDeviceToHost));
  if (loss_sum) *loss_sum = tail[0];
  if (n_pred) *n_pred = tail[1];
  return 0;
}

int lora_ce_get_token_loss(lora_ce_handle* h, float* loss_t, int32_t T) {
  if (!h || !loss_t || T < 0 || T > h->last_T) return fail(LORA_CE_EINVAL, "bad argument");
  LCE_CUDA(cudaSetDevice(h->cfg.device));
  int rc = check_device_error(h);
  if (rc) return rc;
  LCE_CUDA(cudaMemcpy(loss_t, h->loss_tok, (size_t)T * 4, cudaMemcpyDeviceToHost));
  return 0;
}


int lora_ce_step_device(lora_ce_handle* h, const void* dH, int32_t dtype, int32_t T,
                        const int32_t* dtg, float* d_loss) {
  int rc = check_step_args(h, dH, dtype, T, dtg);
  if (rc) return rc;
  LCE_CUDA(cudaSetDevice(h->cfg.device));
  rc = run_or_replay(h, false, dH, dtype, T, dtg, d_loss ? d_loss : h->d_loss);
  if (rc) h->poisoned = true;
  return rc;
}

int lora_ce_step(lora_ce_handle* h, const void* H, int32_t dtype, int32_t T,
                 const int32_t* targets, float* loss_out) {
  using clk = std::chrono::steady_clock;
  const auto t0 = clk::now();
  int rc = check_step_args(h, H, dtype, T, targets);
  if (rc) return rc;
  LCE_CUDA(cudaSetDevice(h->cfg.device));
  rc = run_or_replay(h, true, H, dtype, T, targets, nullptr);
  if (rc) {
    h->poisoned = true;
    return rc;
  }
  const auto t1 = clk::now();
  if ((rc = wait_stream(h))) return rc;
  const auto t2 = clk::now();
  h->host_us[0] = std::chrono::duration<float, std::micro>(t1 - t0).count();
  h->host_us[1] = std::chrono::duration<float, std::micro>(t2 - t1).count();
  float res[2];
  memcpy(res, h->res_host, 8);
  int e;
  memcpy(&e, &res[1], 4);
  if (e != 0) {
    h->poisoned = true;
    return fail(LORA_CE_EDEVICE, e == kErrTarget      ? "target id out of range"
                                 : e == kErrRange     ? "s*U out of the supported range"
                                 : e == kErrSmemAlign ? "shared memory base not 1024-byte aligned"
                                                      : "device pipeline error (bounded wait expired)");
  }
  if (loss_out) *loss_out = res[0];
  return 0;
}

int lora_ce_apply_grads(lora_ce_handle* h, const float* gA, const float* gB, float n_pred) {
  if (!h || !gA || !gB || !(n_pred > 0.f)) return fail(LORA_CE_EINVAL, "bad argument");
  if (h->poisoned) return fail(LORA_CE_ESTATE, "handle poisoned by an earlier error");
  LCE_CUDA(cudaSetDevice(h->cfg.device));
  const int r = h->r, R = h->R, d = h->d, V = h->V;
  const long long nA = (long long)d * R, nparam = nA + h->Vpad * R;
  // G in the kernels' layout: [dA (d x R) | dB (pair-interleaved) | loss | n_pred]
  std::vector<float> G((size_t)nparam + 2, 0.f);
  for (int i = 0; i < d; ++i)
    for (int j = 0; j < r; ++j) G[(size_t)i * R + j] = gA[(size_t)i * r + j];
  for (int j = 0; j < r; ++j)
    for (int v = 0; v < V; ++v) G[(size_t)(nA + bidx(v, j, R))] = gB[(size_t)j * V + v];
  G[(size_t)nparam + 1] = n_pred;
  LCE_CUDA(cudaMemcpyAsync(h->Gbuf, G.data(), G.size() * 4, cudaMemcpyHostToDevice, h->stream));
  const int32_t next_step = h->step + 1;
  AdamArgs aa = adam_args(h, nparam, next_step);
  if (aa.clip > 0.f) lce_sqnorm<<<256, 256, 0, h->stream>>>(nparam, h->Gbuf, h->norm_parts);
  const int blocks = (int)std::min<long long>((nparam + 255) / 256, 8LL * h->num_sms);
  lce_adam<<<blocks, 256, 0, h->stream>>>(aa, h->params, h->mom1, h->mom2, h->Gbuf, h->gmean,
                                           h->norm_parts, nullptr);
  LCE_CUDA(cudaGetLastError());
  LCE_CUDA(cudaStreamSynchronize(h->stream));
  h->step = next_step;
  return 0;
}

int lora_ce_sync(lora_ce_handle* h) {
  if (!h) return fail(LORA_CE_EINVAL, "null handle");
  LCE_CUDA(cudaSetDevice(h->cfg.device));
  return check_device_error(h);
}

int lora_ce_nccl_unique_id(void* id128) {
  if (!id128) return fail(LORA_CE_EINVAL, "null id buffer");
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
  if (!nccl().ok) return fail(LORA_CE_ENCCL, "libnccl.so.2 could not be loaded");
  ncclUniqueId id;
  if (nccl().GetUniqueId(&id) != ncclSuccess) return fail(LORA_CE_ENCCL, "ncclGetUniqueId failed");
  memcpy(id128, &id, 128);
  return 0;
}

int lora_ce_comm_init(lora_ce_handle* h, int32_t nranks, int32_t rank, const void* id128) {
  if (!h || !id128 || nranks < 1 || rank < 0 || rank >= nranks)
    return fail(LORA_CE_EINVAL, "bad communicator arguments");
  if (h->comm) return fail(LORA_CE_ESTATE, "communicator already initialised");
  LCE_CUDA(cudaSetDevice(h->cfg.device));
  if (!nccl().ok) return fail(LORA_CE_ENCCL, "libnccl.so.2 could not be loaded");
  ncclUniqueId id;
  memcpy(&id, id128, 128);
  drop_graphs(h);  // steps captured without the all-reduce
  ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
  config.blocking = 0;
  ncclComm_t comm = nullptr;
  ncclResult_t r = nccl().CommInitRankConfig(&comm, nranks, id, rank, &config);
  if (r == ncclInProgress) r = nccl_settle(comm, h->comm_timeout_ms);
  if (r != ncclSuccess) {
    if (comm) nccl().CommAbort(comm);
    return fail(LORA_CE_ENCCL, std::string("ncclCommInitRankConfig: ") +
                                   (r == ncclInProgress ? "timed out" : nccl_str(r)));
  }
  h->comm = comm;
  h->nranks = nranks;
  h->rank = rank;
  return 0;
}

int lora_ce_set_comm_timeout(lora_ce_handle* h, int32_t timeout_ms) {
  if (!h || timeout_ms < 1) return fail(LORA_CE_EINVAL, "bad argument");
  h->comm_timeout_ms = (double)timeout_ms;
  return 0;
}

int lora_ce_set_profiling(lora_ce_handle* h, int32_t enable) {
  if (!h) return fail(LORA_CE_EINVAL, "null handle");
  LCE_CUDA(cudaSetDevice(h->cfg.device));
  if (enable && !h->ev[0])
    for (cudaEvent_t& e : h->ev) LCE_CUDA(cudaEventCreate(&e));
  h->prof = enable != 0;
  return 0;
}

int32_t lora_ce_phase_times(lora_ce_handle* h, float* ms, int32_t cap) {
  if (!h || !ms || !h->prof) return fail(LORA_CE_EINVAL, "profiling not enabled");
  if (cudaSetDevice(h->cfg.device) != cudaSuccess ||
      cudaEventSynchronize(h->ev[kNumPhases]) != cudaSuccess)
    return fail(LORA_CE_ECUDA, "cudaEventSynchronize failed");
  const int n = cap < kNumPhases ? cap : kNumPhases;
  for (int i = 0; i < n; ++i)
    if (cudaEventElapsedTime(&ms[i], h->ev[i], h->ev[i + 1]) != cudaSuccess)
      return fail(LORA_CE_ECUDA, "cudaEventElapsedTime failed");
  return n;
}

int lora_ce_set_copy_timing(lora_ce_handle* h, int32_t enable) {
  if (!h) return fail(LORA_CE_EINVAL, "null handle");
  LCE_CUDA(cudaSetDevice(h->cfg.device));
  if (enable && !h->tev[0])
    for (cudaEvent_t& e : h->tev) LCE_CUDA(cudaEventCreate(&e));
  h->ctime = enable != 0;
  return 0;
}

int32_t lora_ce_copy_times(lora_ce_handle* h, float* out, int32_t cap) {
  if (!h || !out || cap < 1) return fail(LORA_CE_EINVAL, "bad argument");
  if (!h->ctime) {  // the host's own times of the last lora_ce_step only
    out[0] = h->host_us[0];
    if (cap > 1) out[1] = h->host_us[1];
    return cap > 1 ? 2 : 1;
  }
  if (h->ctime_chunks < 1) return fail(LORA_CE_EINVAL, "no host-input step yet");
  if (cudaSetDevice(h->cfg.device) != cudaSuccess ||
      cudaEventSynchronize(h->tev[kMaxChunks + 2]) != cudaSuccess)
    return fail(LORA_CE_ECUDA, "cudaEventSynchronize failed");
  const int nc = h->ctime_chunks;
  float v[4 + kMaxChunks + 1];
  int n = 0;
  v[n++] = h->host_us[0];
  v[n++] = h->host_us[1];
  float ms = 0.f;
  if (cudaEventElapsedTime(&ms, h->tev[0], h->tev[1]) != cudaSuccess)
    return fail(LORA_CE_ECUDA, "cudaEventElapsedTime failed");
  v[n++] = ms;
  for (int c = 0; c < nc; ++c) {
    if (cudaEventElapsedTime(&ms, h->tev[1 + c], h->tev[2 + c]) != cudaSuccess)
      return fail(LORA_CE_ECUDA, "cudaEventElapsedTime failed");
    v[n++] = ms;
  }
  if (cudaEventElapsedTime(&ms, h->tev[0], h->tev[kMaxChunks + 2]) != cudaSuccess)
    return fail(LORA_CE_ECUDA, "cudaEventElapsedTime failed");
  v[n++] = ms;
  const int m = cap < n ? cap : n;
  for (int i = 0; i < m; ++i) out[i] = v[i];
  return m;
}

const char* lora_ce_phase_name(int32_t i) {
  return (i >= 0 && i < kNumPhases) ? kPhaseNames[i] : "";
}

void* lora_ce_stream(lora_ce_handle* h) { return h ? (void*)h->stream : nullptr; }

int32_t lora_ce_last_launches(lora_ce_handle* h) { return h ? h->launches : 0; }

}  // extern "C"
