/*
 * ref_harness.c — runs the reference's OWN src/train.c (compiled from the
 * reference tree, unmodified, by oracle/Makefile into oracle/_ref/) on
 * seeded inputs, to pin the restatement in lora_oracle.c.  Test
 * infrastructure only.
 *
 * train.c is #included so that its static lora_accum/adam_update and the
 * fields of struct train_state (gA, gB, A, B) are reachable.  The body
 * forward is replaced by this file's forward_* functions, which serve
 * caller-provided hidden states and compute the base logits from the f16
 * lm_head in fp32 with fp64 accumulation, as the reference's own x86
 * matmul_f32 does (src/forward.c:396-403).
 */
#include "train.c"   /* found through -I<reference>/src */
#include "backward.h"

struct forward_ctx {
    int dim, vocab;
    const uint16_t* W; /* [vocab][dim] f16 bits */
    const float* H;    /* [positions][dim] */
    int n_pos;
    int pos;
    float* wrow;
};

static float h_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)(h & 0x8000u)) << 16;
    int exp = (h >> 10) & 0x1f, mant = h & 0x3ff;
    uint32_t u;
    float f;
    if (exp == 0) {
        if (mant == 0) { u = sign; memcpy(&f, &u, 4); return f; }
        f = ldexpf((float)mant, -24);
        return sign ? -f : f;
    }
    if (exp == 0x1f) u = sign | 0x7f800000u | ((uint32_t)mant << 13);
    else u = sign | ((uint32_t)(exp + 127 - 15) << 23) | ((uint32_t)mant << 13);
    memcpy(&f, &u, 4);
    return f;
}

static void h_logits(forward_ctx* f, float* out) {
    const float* x = f->H + (size_t)f->pos * f->dim;
    for (int o = 0; o < f->vocab; o++) {
        const uint16_t* w16 = f->W + (size_t)o * f->dim;
        for (int i = 0; i < f->dim; i++) f->wrow[i] = h_f16_to_f32(w16[i]);
        double acc = 0.0;
        for (int i = 0; i < f->dim; i++) acc += (double)f->wrow[i] * (double)x[i];
        out[o] = (float)acc;
    }
}

int forward_dim(const forward_ctx* f) { return f->dim; }
int forward_vocab_size(const forward_ctx* f) { return f->vocab; }
void forward_reset(forward_ctx* f) { f->pos = 0; }
int forward_prefill(forward_ctx* f, const int* tokens, int n_tokens, float* logits_out) {
    (void)tokens;
    if (n_tokens != 1) return -1;
    f->pos = 0;
    h_logits(f, logits_out);
    return 0;
}
int forward_decode(forward_ctx* f, int token, int pos, float* logits_out) {
    (void)token;
    if (pos < 0 || pos >= f->n_pos) return -1;
    f->pos = pos;
    h_logits(f, logits_out);
    return 0;
}
const float* forward_last_hidden(const forward_ctx* f) {
    return f->H + (size_t)f->pos * f->dim;
}

/*
 * Run n_steps reference train_step calls on the same sample.
 * tokens has n_tokens ids; H has one hidden row per position (n_tokens-1
 * rows are used).  If A_io/B_io are non-NULL and init_from_io != 0 the
 * adapter starts from them (layouts [d][r] and [r][V]); otherwise the
 * reference's train_create init (Kaiming A from seed, B = 0) is used.
 * On return A_io/B_io hold the updated adapter, gA/gB the mean gradient
 * of the last step (the reference keeps it in t->gA/t->gB), losses[k] the
 * loss of step k.  Returns 0 or -1.
 */
int ref_train_steps(int d, int V, int rank, int alpha, float lr, int seq_max,
                    int seed, const uint16_t* W, const float* H,
                    const int* tokens, int n_tokens, int n_steps,
                    int init_from_io, float* A_io, float* B_io, float* gA,
                    float* gB, float* losses, int* step_out) {
    forward_ctx f = {d, V, W, H, n_tokens, 0, NULL};
    f.wrow = (float*)malloc((size_t)d * sizeof(float));
    train_params p;
    memset(&p, 0, sizeof(p));
    p.mode = TRAIN_LORA;
    p.lora_rank = rank;
    p.lora_alpha = alpha;
    p.seq_max = seq_max;
    p.batch = 1;
    p.lr = lr;
    p.epochs = 1;
    p.seed = seed;
    train_state* t = train_create(&f, &p);
    if (!t) { free(f.wrow); return -1; }
    size_t a_sz = (size_t)d * rank, b_sz = (size_t)rank * V;
    if (init_from_io) {
        memcpy(t->A, A_io, a_sz * sizeof(float));
        memcpy(t->B, B_io, b_sz * sizeof(float));
    }
    int rc = 0;
    for (int k = 0; k < n_steps; k++) {
        losses[k] = train_step(t, tokens, n_tokens);
        if (losses[k] < 0) { rc = -1; break; }
    }
    if (A_io) memcpy(A_io, t->A, a_sz * sizeof(float));
    if (B_io) memcpy(B_io, t->B, b_sz * sizeof(float));
    if (gA) memcpy(gA, t->gA, a_sz * sizeof(float));
    if (gB) memcpy(gB, t->gB, b_sz * sizeof(float));
    if (step_out) *step_out = t->step;
    train_free(t);
    free(f.wrow);
    return rc;
}

/* The reference's own LORA0001 writer, for format pinning. */
int ref_save_adapter(int d, int V, int rank, int alpha, int step,
                     const float* A, const float* B, const char* path) {
    forward_ctx f = {d, V, NULL, NULL, 0, 0, NULL};
    train_params p;
    memset(&p, 0, sizeof(p));
    p.lora_rank = rank;
    p.lora_alpha = alpha;
    train_state* t = train_create(&f, &p);
    if (!t) return -1;
    memcpy(t->A, A, (size_t)d * rank * sizeof(float));
    memcpy(t->B, B, (size_t)rank * V * sizeof(float));
    t->step = step;
    int rc = train_save(t, path);
    train_free(t);
    return rc;
}

/* The reference's softmax-CE finite-difference check (src/backward.c). */
float ref_grad_check_softmax_ce(int vocab, float eps) {
    return grad_check_softmax_ce(vocab, eps);
}

/* The reference's own merge arithmetic (lora_patched_weight, src/train.c:
 * 415-460, with its truncating f32 -> f16 conversion), for pinning the
 * oracle's restatement and the GPU merge kernel. */
int ref_merge_weight(const uint16_t* W, const float* A, const float* B, int dim,
                     int rank, int vocab, float scale, uint16_t* out) {
    uint16_t* p = lora_patched_weight(W, A, B, dim, rank, vocab, scale, "token_embd.weight");
    if (!p) return -1;
    memcpy(out, p, (size_t)vocab * dim * sizeof(uint16_t));
    free(p);
    return 0;
}

/* The reference's own train_run (src/train.c:295-389) over a packed dataset,
 * every sample's hidden rows served from H by position, with the adapter
 * from train_create (seeded Kaiming A, B = 0).  Returns train_run's rc. */
int ref_train_run_mem(int d, int V, int rank, int alpha, float lr, int seq_max, int seed,
                      int epochs, int max_steps, int checkpoint_every, const uint16_t* W,
                      const float* H, int n_pos, const char* packed, const char* out_dir,
                      long simulate_mem_kb);

int ref_train_run(int d, int V, int rank, int alpha, float lr, int seq_max, int seed,
                  int epochs, int max_steps, int checkpoint_every, const uint16_t* W,
                  const float* H, int n_pos, const char* packed, const char* out_dir) {
    return ref_train_run_mem(d, V, rank, alpha, lr, seq_max, seed, epochs, max_steps,
                             checkpoint_every, W, H, n_pos, packed, out_dir, 0);
}

/* ref_train_run with train_params.simulate_mem_kb set: the memory figure
 * train_run's watchdog compares with its emergency threshold
 * (src/train.c:355-369). */
int ref_train_run_mem(int d, int V, int rank, int alpha, float lr, int seq_max, int seed,
                      int epochs, int max_steps, int checkpoint_every, const uint16_t* W,
                      const float* H, int n_pos, const char* packed, const char* out_dir,
                      long simulate_mem_kb) {
    forward_ctx f = {d, V, W, H, n_pos, 0, NULL};
    f.wrow = (float*)malloc((size_t)d * sizeof(float));
    train_params p;
    memset(&p, 0, sizeof(p));
    p.mode = TRAIN_LORA;
    p.lora_rank = rank;
    p.lora_alpha = alpha;
    p.seq_max = seq_max;
    p.batch = 1;
    p.lr = lr;
    p.epochs = epochs;
    p.max_steps = max_steps;
    p.checkpoint_every = checkpoint_every;
    p.seed = seed;
    p.simulate_mem_kb = simulate_mem_kb;
    train_state* t = train_create(&f, &p);
    int rc = t ? train_run(t, packed, &p, out_dir) : -1;
    fflush(stdout);
    if (t) train_free(t);
    free(f.wrow);
    return rc;
}

/* The reference's own train_merge (src/train.c:465-542). */
int ref_train_merge(const char* base_gguf, const char* adapter, const char* out_gguf) {
    int rc = train_merge(base_gguf, adapter, out_gguf);
    fflush(stdout);
    return rc;
}

/* The reference's own gradient mean and adam_update (src/train.c:230-239,
 * 175-196) on caller-supplied gradient sums: n_steps updates of one
 * train_state, update k taking gA_sums[k] [d][r], gB_sums[k] [r][V] and
 * n_pred[k], the Adam step counter starting at step0 and the moments at
 * zero (carried from update to update).  A_io/B_io hold the adapter in and
 * out.  Pins the GPU Adam kernel bit for bit. */
int ref_adam_steps(int d, int V, int rank, float lr, int step0, int n_steps,
                   const float* gA_sums, const float* gB_sums, const int* n_pred,
                   float* A_io, float* B_io) {
    forward_ctx f = {d, V, NULL, NULL, 0, 0, NULL};
    train_params p;
    memset(&p, 0, sizeof(p));
    p.mode = TRAIN_LORA;
    p.lora_rank = rank;
    p.lora_alpha = 2 * rank;
    p.lr = lr;
    train_state* t = train_create(&f, &p);
    if (!t) return -1;
    const size_t a_sz = (size_t)d * rank, b_sz = (size_t)rank * V;
    memcpy(t->A, A_io, a_sz * sizeof(float));
    memcpy(t->B, B_io, b_sz * sizeof(float));
    t->step = step0;
    for (int k = 0; k < n_steps; k++) {
        memcpy(t->gA, gA_sums + (size_t)k * a_sz, a_sz * sizeof(float));
        memcpy(t->gB, gB_sums + (size_t)k * b_sz, b_sz * sizeof(float));
        /* train_step's mean (src/train.c:233-237) */
        float inv = 1.0f / (float)n_pred[k];
        for (size_t i = 0; i < a_sz; i++) t->gA[i] *= inv;
        for (size_t i = 0; i < b_sz; i++) t->gB[i] *= inv;
        adam_update(t);
    }
    memcpy(A_io, t->A, a_sz * sizeof(float));
    memcpy(B_io, t->B, b_sz * sizeof(float));
    train_free(t);
    return 0;
}
