/*
 * lora_train.h — what the GPU trainer (smollm2.c_b200/host/lora_train.c)
 * adds to the reference's trainer API of src/train.h.  The seven functions
 * of src/train.h:27-42 keep their signatures and come from lora_train.c;
 * this header declares the one thing the GPU step needs that forward_ctx
 * does not expose: the f16 lm_head (tied token_embd.weight) weight.
 *
 * Include after the reference's "train.h" and "gguf.h".
 */
#ifndef LORA_TRAIN_H
#define LORA_TRAIN_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Upload the lm_head weight, [vocab][dim] f16 bits, to the trainer's GPU.
 * No counterpart in the reference (its train_step reads base logits from
 * forward_decode).  Returns 0 or -1; train_step returns -1.0f until it has
 * succeeded once. */
int lora_train_set_lm_head(train_state* t, const uint16_t* w_f16);

/* Same, taking token_embd.weight (dims {dim, vocab}) from a loaded model:
 * the call cmd_train adds after train_create (src/studio.c:234).  F16, or
 * Q4_K (GGUF type 12, super-blocks over the flattened tensor) for QLoRA,
 * which is dequantised once on the GPU; the reference itself refuses
 * QLoRA (src/studio.c:187-191). */
int lora_train_set_lm_head_gguf(train_state* t, const gguf_ctx* g);

/* Run the body forward on the GPU too (include/lora_body.h), from the
 * model's own tensors: train_step and train_run then compute the hidden
 * states of all of a step's positions in one batched forward instead of
 * forward_prefill / forward_decode per position (src/train.c:210-229).  The
 * int8 rules, the order of the float operations and the KV / RoPE modes are
 * the reference's defaults (f32 KV cache, f32 RoPE tables); e^x comes from a
 * double-precision exp, so hidden states can differ from the CPU body's in
 * the last bits.  Opt-in; returns 0 or -1.  No counterpart in the
 * reference. */
int lora_train_set_body_gguf(train_state* t, const gguf_ctx* g);

#ifdef __cplusplus
}
#endif

#endif  /* LORA_TRAIN_H */
