/*
 * lora_body.h — C ABI of the B200 body forward of the SmolLM2 architecture:
 * the hidden state h of every position of a batch of token sequences, the
 * input of the LoRA-on-lm_head step (include/lora_ce.h).
 *
 * The reference produces h one position at a time: train_step
 * (src/train.c:198-229) runs forward_prefill for position 0 and
 * forward_decode for every following position and reads
 * forward_last_hidden (src/forward.c:935-1093, 1129-1256, 1099-1101).  Per
 * position both compute the same thing, which this library computes for
 * all positions of all sequences at once (teacher forcing):
 *
 *   x = token_embd[tok]                                  (f16 -> f32)
 *   per layer:  xn = rmsnorm(x, attn_norm)   (f64 sum of squares)
 *               q, k, v = int8(xn) . int8 W  (per-tensor activations,
 *                                             per-row weights, int32 sums)
 *               rope(q, k) at the position within its sequence (f32
 *                                             cos / sin tables)
 *               causal GQA attention over the sequence's earlier positions
 *               x += int8(attn) . int8 Wo
 *               xn = rmsnorm(x, ffn_norm)
 *               g, u = int8(xn) . int8 Wgate, Wup
 *               x += int8(g * sigmoid(g) * u) . int8 Wdown
 *   h = rmsnorm(x, output_norm)
 *
 * with the reference's quantisation rules (weights: src/forward.c:441-462,
 * activations: the x86 branch of :157-166), its operation order and its
 * f32 KV cache and f32 RoPE tables (the default modes).  Weights are passed
 * as stored in the GGUF (f16 matrices with dims[0] = inputs innermost, f32
 * norms) and quantised on the GPU at upload.
 *
 * Conventions as lora_ce.h: 0 or a negative LORA_CE_E* code, never abort;
 * lora_body_last_error() describes the last failure on the calling thread.
 * One handle per GPU, not thread-safe.
 */
#ifndef LORA_BODY_H
#define LORA_BODY_H

#include <stdint.h>

#include "lora_ce.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct lora_body_config {
    int32_t n_layers;    /* 30 */
    int32_t dim;         /* 576, a multiple of 64, <= 4096 */
    int32_t n_heads;     /* 9 */
    int32_t n_kv_heads;  /* 3 (n_heads a multiple of it) */
    int32_t ffn_hidden;  /* 1536, a multiple of 64 */
    int32_t vocab;       /* 49152 */
    float rms_eps;       /* 1e-5 */
    float rope_theta;    /* 1e5 */
    int32_t max_seq;     /* longest sequence a call may contain (<= 4096) */
    int32_t max_tokens;  /* most positions over all sequences of one call */
    int32_t device;      /* CUDA device ordinal */
} lora_body_config;

typedef struct lora_body_handle lora_body_handle;

/* Replaces forward_load's allocations (src/forward.c:671-880); the head
 * dimension is dim / n_heads and must be 64 (the reference's attention
 * reads 64-float rows, src/forward.c:1013). */
int lora_body_create(const lora_body_config* cfg, lora_body_handle** out);
int lora_body_destroy(lora_body_handle* h);

/* token_embd.weight [vocab][dim] f16 bits and output_norm.weight [dim]. */
int lora_body_set_embedding(lora_body_handle* h, const uint16_t* token_embd,
                            const float* output_norm);

/* One layer's tensors as stored in the GGUF: the norms [dim] f32; wq
 * [dim][dim], wk and wv [kv_dim][dim], wo [dim][dim], gate and up
 * [ffn][dim], down [dim][ffn], all f16 bits with rows = outputs.  Host
 * buffers; quantised to int8 per row on the GPU as forward_load does
 * (quantize_f16_rows_to_q8_perrow, src/forward.c:441-462). */
int lora_body_set_layer(lora_body_handle* h, int32_t layer, const float* attn_norm,
                        const uint16_t* wq, const uint16_t* wk, const uint16_t* wv,
                        const uint16_t* wo, const float* ffn_norm, const uint16_t* w_gate,
                        const uint16_t* w_up, const uint16_t* w_down);

/* A sliding window for one layer (attn_registry's SWA type, src/
 * attn_registry.c:80-85): position t attends to the last `window`
 * positions of its sequence; 0 (the default) = dense. */
int lora_body_set_window(lora_body_handle* h, int32_t layer, int32_t window);

/* Hidden states of every position: sequence i is tokens[offsets[i] ..
 * offsets[i+1]) (offsets has n_seqs + 1 entries, offsets[0] = 0, host
 * memory), its positions numbered from 0.  H_out [T][dim] f32 (host), T =
 * offsets[n_seqs]: row t is forward_last_hidden after the reference's
 * forward has consumed tokens[..t] of that sequence.  A token id outside
 * [0, vocab) fails with LORA_CE_EINVAL before anything runs. */
int lora_body_hidden(lora_body_handle* h, const int32_t* tokens, const int32_t* offsets,
                     int32_t n_seqs, float* H_out);

/* The same on device memory: d_tokens [T] on the handle's device, offsets
 * on the host, d_H [T][dim] of h_dtype (LORA_CE_F32, LORA_CE_BF16 or
 * LORA_CE_F16; 16-byte aligned).  Enqueued on the handle's stream; returns
 * without waiting for this call's work (it does wait for the previous
 * call's, whose position table it reuses).  Token ids are range-checked on
 * the GPU: an id outside
 * [0, vocab) is read as 0 and reported by the next lora_body_sync as
 * LORA_CE_EDEVICE. */
int lora_body_hidden_device(lora_body_handle* h, const int32_t* d_tokens,
                            const int32_t* offsets, int32_t n_seqs, void* d_H,
                            int32_t h_dtype);

/* One training step whose hidden states come from this body: the
 * positions of n_seqs packed samples (tokens and offsets as
 * lora_body_hidden; the hidden state of position t feeds the prediction of
 * targets[t]), run through the body into the body's own device buffer, then
 * lora_ce_step_device on `ce` (same device), waited for; *loss_out gets the
 * step's mean loss.  This is train_step with its per-position
 * forward_prefill / forward_decode loop (src/train.c:210-229) replaced by
 * one batched body forward; host buffers in. */
int lora_body_train_step(lora_body_handle* h, lora_ce_handle* ce, const int32_t* tokens,
                         const int32_t* offsets, int32_t n_seqs, const int32_t* targets,
                         float* loss_out);

/* Wait for the handle's stream; report a device-side error. */
int lora_body_sync(lora_body_handle* h);

/* The CUDA stream the handle launches on (a cudaStream_t). */
void* lora_body_stream(lora_body_handle* h);

const char* lora_body_last_error(void);

#ifdef __cplusplus
}
#endif
#endif /* LORA_BODY_H */
