/*
 * lora_ce.h — C ABI of the B200 LoRA-on-lm_head training step.
 *
 * One handle drives one GPU.  A step takes the hidden states h [T][d] of T
 * positions and the id each position predicts, and runs
 *
 *   z      = h.W^T + scale.(h.A).B          (W tied lm_head [V][d], f16)
 *   loss_t = -log(softmax(z_t)[target_t] + 1e-12)
 *   dA, dB = analytic gradients of sum_t loss_t
 *   g      = (dA, dB) / n_pred              (n_pred summed over all ranks)
 *   Adam(W) update of A, B                  (optional decoupled weight decay
 *                                            and global-norm clip)
 *
 * which is the part of the reference's train_step that follows the body
 * forward (src/train.c:198-242: lora_accum per position, the mean over
 * n_pred, adam_update).  The adapter uses the reference layouts: A is
 * [d][r] (A[i*r + j]) and B is [r][V] (B[j*V + v]) (src/train.c:35-36).
 *
 * Conventions, as in the reference's C API (src/train.h): every call
 * returns 0 on success or a negative LORA_CE_E* code; nothing aborts or
 * exits.  lora_ce_last_error() returns a message for the last failure on
 * the calling thread.  A handle is not thread-safe; use one per GPU/rank.
 * Host buffers passed in are only borrowed for the duration of the call.
 */
#ifndef LORA_CE_H
#define LORA_CE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LORA_CE_OK 0
#define LORA_CE_EINVAL (-1)   /* bad argument (sizes, null pointers, ids) */
#define LORA_CE_ENOMEM (-2)   /* device or host allocation failed */
#define LORA_CE_ECUDA (-3)    /* CUDA runtime / driver error */
#define LORA_CE_ENCCL (-4)    /* NCCL error or collective timeout */
#define LORA_CE_EDEVICE (-5)  /* a kernel reported an error (bounded wait
                                 expired, target id out of range) */
#define LORA_CE_ESTATE (-6)   /* handle poisoned by an earlier error, or a
                                 call made in the wrong order */

/* Element type of the hidden states passed to a step. */
#define LORA_CE_BF16 0
#define LORA_CE_F16 1
#define LORA_CE_F32 2

typedef struct lora_ce_config {
    int32_t dim;        /* d: hidden size, multiple of 64, <= 640 (576) */
    int32_t vocab;      /* V: vocabulary size (49152) */
    int32_t rank;       /* r: 1..256, LORA_MAX_RANK (src/train.c:20).  Run
                           at 4, 8, 16, 32, 64, 128 or 256 with zero
                           padding, which leaves every result unchanged;
                           ranks above 64 take a slower path that keeps the
                           logit rows of a block of positions in HBM */
    float scale;        /* alpha / r (train_create: src/train.c:62-63) */
    float lr;           /* learning rate */
    float beta1;        /* 0.9   (ADAM_B1, src/train.c:23) */
    float beta2;        /* 0.999 (ADAM_B2, src/train.c:24) */
    float eps;          /* 1e-8  (ADAM_EPS, src/train.c:25) */
    float weight_decay; /* decoupled (AdamW); 0 = the reference's Adam */
    float clip_norm;    /* global L2 clip of the mean gradient; 0 = off */
    int32_t max_tokens; /* largest T a step on this handle will be given */
    int32_t device;     /* CUDA device ordinal */
} lora_ce_config;

typedef struct lora_ce_handle lora_ce_handle;

/* Fill *cfg with the reference defaults for the given shape
 * (beta1/beta2/eps from src/train.c:23-25, lr 1e-4 and alpha 16 from
 * cmd_train src/studio.c:150-154, no weight decay, no clip). */
void lora_ce_default_config(lora_ce_config* cfg, int32_t dim, int32_t vocab,
                            int32_t rank, int32_t max_tokens);

/* Replaces train_create's allocation of the adapter/optimizer state
 * (src/train.c:53-81).  The adapter starts at A = 0, B = 0 and the Adam
 * step at 0; load it with lora_ce_set_adapter. */
int lora_ce_create(const lora_ce_config* cfg, lora_ce_handle** out);

/* Replaces train_free (src/train.c:98-104). */
int lora_ce_destroy(lora_ce_handle* h);

/* Upload the tied lm_head / token_embd weight, [V][d] f16 bit patterns as
 * stored in the GGUF (dims[0] = d innermost; src/train.c:498-516). */
int lora_ce_set_weight_f16(lora_ce_handle* h, const uint16_t* W);

/* Upload the lm_head weight as Q4_K (GGUF / ggml type 12) super-blocks:
 * V*d/256 blocks of 144 bytes over the flattened [V][d] tensor (V*d must
 * be a multiple of 256).  The weight is dequantised once on the GPU into
 * the f16 operand of the logits GEMM (it is frozen during LoRA training), so
 * a QLoRA step costs what an f16 step costs.  No counterpart in the
 * reference (QLoRA is refused, src/studio.c:187-191). */
int lora_ce_set_weight_q4k(lora_ce_handle* h, const void* blocks);

/* Q4_K super-blocks -> weights, y = (d*sc)*q - (dmin*m) with each product
 * and the difference rounded separately; out_dtype LORA_CE_F32 gives y,
 * LORA_CE_F16 gives y rounded to nearest f16.  Host buffers (device
 * `device`), or device pointers (16-byte aligned) enqueued on `stream`. */
int lora_ce_q4k_dequant(const void* blocks, int64_t n_blocks, void* out,
                        int32_t out_dtype, int32_t device);
int lora_ce_q4k_dequant_device(const void* d_blocks, int64_t n_blocks,
                               void* d_out, int32_t out_dtype, void* stream);
const char* lora_ce_q4k_last_error(void);

/* Load an adapter (reference layouts) and the Adam step counter; resets
 * the Adam moments, as train_load does (src/train.c:261-283: LORA0001
 * carries no optimizer state). */
int lora_ce_set_adapter(lora_ce_handle* h, const float* A_dxr,
                        const float* B_rxv, int32_t step);

/* Set the LoRA scale alpha/r used by the following steps (train_load takes
 * the scale stored in the LORA0001 file, src/train.c:278). */
int lora_ce_set_scale(lora_ce_handle* h, float scale);

/* Read the adapter back in the reference layouts (what train_save writes,
 * src/train.c:244-259).  Any pointer may be NULL. */
int lora_ce_get_adapter(lora_ce_handle* h, float* A_dxr, float* B_rxv,
                        int32_t* step);

/* One training step from HOST buffers: H [T][d] of type h_dtype, targets
 * [T] int32 in [0, V).  Copies in, runs the step, and writes the mean loss
 * over all ranks' positions to *loss_out (train_step's return value).
 * Replaces the per-position lora_accum loop, the mean and adam_update of
 * train_step (src/train.c:213-241). */
int lora_ce_step(lora_ce_handle* h, const void* H, int32_t h_dtype,
                 int32_t T, const int32_t* targets, float* loss_out);

/* Same step on DEVICE buffers of the handle's device (no host copies; the
 * mean loss is left on the device at d_loss, which may be NULL). */
int lora_ce_step_device(lora_ce_handle* h, const void* d_H, int32_t h_dtype,
                        int32_t T, const int32_t* d_targets, float* d_loss);

/* The mean gradients (dA [d][r], dB [r][V]) applied by the last step, the
 * summed loss and n_pred over all ranks.  Any pointer may be NULL. */
int lora_ce_get_grads(lora_ce_handle* h, float* gA_dxr, float* gB_rxv,
                      float* loss_sum, float* n_pred);

/* Per-position loss of the last step on this rank (T floats). */
int lora_ce_get_token_loss(lora_ce_handle* h, float* loss_t, int32_t T);

/* One optimizer step from caller-supplied gradient SUMS over n_pred
 * positions (gA [d][r], gB [r][V], reference layouts, host buffers):
 * g = sum * (1/n_pred), then the optional clip and weight decay, then the
 * Adam update, advancing the step counter.  This is the mean and
 * adam_update of train_step (src/train.c:230-239 and 175-196) with the
 * gradients supplied by the caller instead of lora_accum (for example
 * sums accumulated over several micro-batches). */
int lora_ce_apply_grads(lora_ce_handle* h, const float* gA_dxr, const float* gB_rxv,
                        float n_pred);

/* Data-parallel token sharding: every rank runs the same steps on its own
 * positions; one NCCL sum all-reduce of [dA | dB | loss | n_pred] runs
 * between the gradient and the Adam kernels.  lora_ce_nccl_unique_id fills
 * 128 bytes on one rank, which the caller distributes to all ranks. */
int lora_ce_nccl_unique_id(void* id128);
int lora_ce_comm_init(lora_ce_handle* h, int32_t nranks, int32_t rank,
                      const void* id128);

/* Bound, in ms (default 60000), on every wait that involves the
 * communicator: its initialisation, an all-reduce's enqueue and a step's
 * completion.  The communicator is non-blocking: a collective that does not
 * complete in time (a peer rank that left) or that reports an asynchronous
 * error is aborted (ncclCommAbort), the call returns LORA_CE_ENCCL and the
 * handle is poisoned, so every rank sees an error instead of a hang. */
int lora_ce_set_comm_timeout(lora_ce_handle* h, int32_t timeout_ms);

/* Wait for the handle's stream and report a device-side error of the steps
 * launched since the last check (lora_ce_step_device does not wait). */
int lora_ce_sync(lora_ce_handle* h);

/* Per-phase timing with CUDA events on the handle's stream.  When enabled,
 * every step records an event before each phase; lora_ce_phase_times waits
 * for the last step and writes the duration in ms of up to cap phases (in
 * launch order: prep, pass1_lse, combine, pass2_grad, dA_partial, finalize,
 * allreduce, sqnorm, adam) and returns how many it wrote. */
int lora_ce_set_profiling(lora_ce_handle* h, int32_t enable);
int32_t lora_ce_phase_times(lora_ce_handle* h, float* ms, int32_t cap);
const char* lora_ce_phase_name(int32_t i);

/* Timing of host-input steps (lora_ce_step), to see where the time of a
 * step that starts from host memory goes.  While enabled, host-input steps
 * launch their kernels and copies directly (not as a replayed CUDA graph)
 * with timing events between them; lora_ce_copy_times waits for the last
 * host-input step and writes: [0] host us inside lora_ce_step before the
 * wait (argument checks, graph launch), [1] host us waiting for the
 * result, [2] ms from the step's start on the compute stream to the start
 * of the copies, [3 .. 3+c) ms of each of the c chunk copies of h, [3+c]
 * ms from the step's start to the result read-back.  Returns how many
 * values it wrote (at most cap).  With timing off it writes only [0] and
 * [1] of the last lora_ce_step (graph replays included) and returns 2. */
int lora_ce_set_copy_timing(lora_ce_handle* h, int32_t enable);
int32_t lora_ce_copy_times(lora_ce_handle* h, float* out, int32_t cap);

/* The CUDA stream the handle launches on (a cudaStream_t). */
void* lora_ce_stream(lora_ce_handle* h);

/* Number of kernel launches the last step issued. */
int32_t lora_ce_last_launches(lora_ce_handle* h);

const char* lora_ce_last_error(void);

/* LoRA merge into the tied lm_head, replacing lora_patched_weight
 * (src/train.c:415-460, called by train_merge :465-542):
 * out[v][i] = f16trunc(f32(W[v][i]) + scale * sum_k A[i][k] * B[k][v]) with
 * the reference's exact arithmetic, including its merge-path f16 -> f32
 * conversion (f16 subnormals halved) and its f32 -> f16 conversion, which
 * keeps the low 16 bits of a mis-rebiased intermediate (src/train.c:392-407)
 * and so differs from IEEE f16 for almost every weight: the output is
 * bit-identical to the reference's merged tensor, defect included.
 * Host buffers (W, out [V][d] f16
 * bits; A [d][r], B [r][V]); rank <= 256 as LORA_MAX_RANK; d a multiple
 * of 8.  The _device variant takes device pointers (W and out 16-byte
 * aligned) and enqueues on `stream` without waiting. */
int lora_ce_merge_weight(const uint16_t* W, const float* A_dxr, const float* B_rxv,
                         int32_t dim, int32_t rank, int32_t vocab, float scale,
                         uint16_t* out, int32_t device);
int lora_ce_merge_weight_device(const uint16_t* d_W, const float* d_A,
                                const float* d_B, int32_t dim, int32_t rank,
                                int32_t vocab, float scale, uint16_t* d_out,
                                void* stream);
const char* lora_ce_merge_last_error(void);

/* Per-position loss -log(softmax(h.W^T + scale.(h.A).B)[target] + 1e-12)
 * for callers that cannot allocate GPU memory at call time (a serving or
 * evaluation process whose memory is reserved up front, or a runtime that
 * must never fail or stall in an allocation mid-request).  No counterpart
 * in the reference.  It allocates nothing: all scratch lives in statically
 * sized device arrays (about 8.9 MB per GPU that loads the library, held
 * until exit), and every argument is a device pointer on the current
 * device: W [V][d] f16 bits, A [d][4], B [4][V] (reference layouts),
 * H [T][d] of h_dtype, targets [T], loss out [T].  Work is enqueued on
 * `stream` (a cudaStream_t; NULL = legacy default stream) and the call
 * returns without waiting.  Limits: rank 4, T <= 4096, V <= 49152, d a
 * multiple of 64 up to 576; larger sizes return LORA_CE_EINVAL.  A target
 * outside [0, V) makes every output loss NaN.  All calls share the scratch
 * arrays, so calls that can overlap on the GPU race and must be serialised
 * by the caller; the first call on a device resolves the arrays' device
 * addresses, so make it before any stream capture.  Errors are described
 * by lora_ce_noalloc_last_error(). */
int lora_ce_token_loss_noalloc(const uint16_t* d_W, int32_t vocab, int32_t dim,
                               const float* d_A, const float* d_B, float scale,
                               const void* d_H, int32_t h_dtype, int32_t T,
                               const int32_t* d_targets, float* d_loss,
                               void* stream);
const char* lora_ce_noalloc_last_error(void);

#ifdef __cplusplus
}
#endif
#endif /* LORA_CE_H */
