/*
 * body_ref.c — test infrastructure: the reference's own body forward
 * (src/forward.c, compiled unmodified from the reference tree by
 * oracle/Makefile into oracle/_ref/libref_body.so) driven the way
 * train_step drives it (src/train.c:210-229): forward_prefill on the first
 * token of a sequence, then forward_decode position by position, reading
 * forward_last_hidden after each.  The rows are the hidden states the GPU
 * body forward must reproduce.  Never part of the product.
 */
#define _POSIX_C_SOURCE 199309L
#include "forward.h"
#include "gguf.h"

#include <stdlib.h>
#include <string.h>
#include <time.h>

static gguf_ctx g_model;
static forward_ctx* g_fwd = NULL;
static int g_vocab = 0, g_dim = 0;

/* Load a model file for the calls below (max_seq positions per sequence). */
int ref_body_load(const char* path, int max_seq) {
    if (g_fwd) { forward_free(g_fwd); gguf_free(&g_model); g_fwd = NULL; }
    if (gguf_load(path, &g_model) < 0) return -1;
    if (forward_load(&g_fwd, &g_model, max_seq) < 0) { gguf_free(&g_model); return -1; }
    g_vocab = forward_vocab_size(g_fwd);
    g_dim = forward_dim(g_fwd);
    return 0;
}

/* Hidden state of every position of one sequence: H_out [n][dim]; returns
 * the seconds spent in the reference's forward, or -1. */
double ref_body_hidden(const int* tokens, int n, float* H_out) {
    if (!g_fwd || n < 1) return -1.0;
    float* logits = (float*)malloc((size_t)g_vocab * sizeof(float));
    if (!logits) return -1.0;
    struct timespec t0, t1;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    forward_reset(g_fwd);
    int rc = forward_prefill(g_fwd, tokens, 1, logits);
    if (rc == 0) memcpy(H_out, forward_last_hidden(g_fwd), (size_t)g_dim * sizeof(float));
    for (int pos = 1; pos < n && rc == 0; pos++) {
        rc = forward_decode(g_fwd, tokens[pos], pos, logits);
        if (rc == 0)
            memcpy(H_out + (size_t)pos * g_dim, forward_last_hidden(g_fwd),
                   (size_t)g_dim * sizeof(float));
    }
    clock_gettime(CLOCK_MONOTONIC, &t1);
    free(logits);
    if (rc != 0) return -1.0;
    return (double)(t1.tv_sec - t0.tv_sec) + 1e-9 * (double)(t1.tv_nsec - t0.tv_nsec);
}

void ref_body_free(void) {
    if (g_fwd) { forward_free(g_fwd); gguf_free(&g_model); g_fwd = NULL; }
}
