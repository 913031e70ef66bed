/*
 * studio_env.c — test infrastructure for the GPU trainer
 * (smollm2.c_b200/host/lora_train.c): the body-forward functions the trainer
 * calls (src/forward.h: forward_dim, forward_vocab_size, forward_reset,
 * forward_prefill, forward_decode, forward_last_hidden), serving
 * caller-provided hidden rows instead of running the transformer.  Linked
 * by oracle/Makefile with the reference's own gguf.c, gguf_write.c and
 * hw_probe.c into oracle/_ref/libstudio_env.so, so that train_run and
 * train_merge run against the reference's file handling.  Never part of
 * the product.
 *
 * The base logits the reference's forward writes are not used by the GPU
 * trainer; this forward writes zeros there and counts the calls so a test
 * can check the prefill / decode sequence of train_step
 * (src/train.c:207-226).
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "gguf.h"

struct forward_ctx {
    int dim, vocab, n_pos, pos;
    const float* H; /* [n_pos][dim], borrowed */
    int n_prefill, n_decode, bad_calls;
};
typedef struct forward_ctx forward_ctx;

forward_ctx* env_forward_create(int dim, int vocab, const float* H, int n_pos) {
    forward_ctx* f = calloc(1, sizeof(*f));
    if (!f) return NULL;
    f->dim = dim;
    f->vocab = vocab;
    f->H = H;
    f->n_pos = n_pos;
    return f;
}

void env_forward_free(forward_ctx* f) { free(f); }

/* calls[0] prefills, calls[1] decodes, calls[2] out-of-order calls */
void env_forward_calls(const forward_ctx* f, int* calls) {
    calls[0] = f->n_prefill;
    calls[1] = f->n_decode;
    calls[2] = f->bad_calls;
}

int forward_dim(const forward_ctx* f) { return f->dim; }
int forward_vocab_size(const forward_ctx* f) { return f->vocab; }
void forward_reset(forward_ctx* f) { f->pos = -1; }

int forward_prefill(forward_ctx* f, const int* tokens, int n_tokens, float* logits_out) {
    (void)tokens;
    if (n_tokens != 1 || f->n_pos < 1) return -1;
    if (f->pos != -1) f->bad_calls++;
    f->pos = 0;
    f->n_prefill++;
    memset(logits_out, 0, (size_t)f->vocab * sizeof(float));
    return 0;
}

int forward_decode(forward_ctx* f, int token, int pos, float* logits_out) {
    (void)token;
    if (pos < 0 || pos >= f->n_pos) return -1;
    if (pos != f->pos + 1) f->bad_calls++;
    f->pos = pos;
    f->n_decode++;
    memset(logits_out, 0, (size_t)f->vocab * sizeof(float));
    return 0;
}

const float* forward_last_hidden(const forward_ctx* f) {
    if (f->pos < 0 || f->pos >= f->n_pos) return NULL;
    return f->H + (size_t)f->pos * f->dim;
}

/* A model file opened with the reference's gguf_load, for tests that hand a
 * gguf_ctx to the trainer (lora_train_set_lm_head_gguf). */
gguf_ctx* env_gguf_open(const char* path) {
    gguf_ctx* g = calloc(1, sizeof(*g));
    if (!g) return NULL;
    if (gguf_load(path, g) < 0) {
        free(g);
        return NULL;
    }
    return g;
}

void env_gguf_close(gguf_ctx* g) {
    if (!g) return;
    gguf_free(g);
    free(g);
}

/* dims[0..1], dtype and the first `n` bytes of tensor `name`; 0 or -1. */
int env_gguf_tensor(const char* path, const char* name, uint64_t* dims, int* dtype, void* out,
                    size_t n) {
    gguf_ctx g;
    if (gguf_load(path, &g) < 0) return -1;
    const gguf_tensor_info* t = gguf_tensor_get(&g, name);
    int rc = -1;
    if (t) {
        dims[0] = t->dims[0];
        dims[1] = t->n_dims > 1 ? t->dims[1] : 1;
        *dtype = (int)t->dtype;
        const void* d = gguf_tensor_data(&g, t);
        if (d) {
            memcpy(out, d, n);
            rc = 0;
        }
    }
    gguf_free(&g);
    return rc;
}
