/*
 * lora_train.c — the trainer API of src/train.h (train_create, train_free,
 * train_step, train_save, train_load, train_run, train_merge) with the
 * LoRA-on-lm_head step on a B200 through the lora_ce C ABI.  It replaces
 * src/train.c in the reference's build: compiled against the reference's
 * own headers (train.h, forward.h, gguf.h, gguf_write.h, hw_probe.h, data.h)
 * and linked with its forward / gguf / hw_probe objects, it keeps every
 * signature, return convention and printed line of the trainer.
 *
 * What moves to the GPU is the step of src/train.c:198-242: instead of
 * lora_accum + adam_update per position on the CPU, train_step gathers the
 * hidden state of every predicted position from the body forward (which
 * stays on the CPU, forward_prefill / forward_decode as before), then runs
 * one lora_ce_step over all of them (logits, softmax CE, dA, dB, mean,
 * Adam).  The merge of train_merge runs as lora_ce_merge_weight.
 *
 * One addition, because forward_ctx does not expose the lm_head weight:
 * lora_train_set_lm_head / lora_train_set_lm_head_gguf hand the f16
 * token_embd.weight to the trainer (cmd_train has the gguf_ctx in scope);
 * train_step returns -1.0f until one of them has been called.
 *
 * Optional settings the reference's train_params has no field for, read
 * once in train_create from the environment:
 *   LORA_CE_DEVICE        CUDA device ordinal (default 0)
 *   LORA_CE_WEIGHT_DECAY  decoupled weight decay (default 0: the reference's Adam)
 *   LORA_CE_CLIP_NORM     global gradient-norm clip (default 0: off)
 *   LORA_TRAIN_PACK       "1": train_run packs train_params.batch samples into
 *                         each step (one Adam update over all their predicted
 *                         positions).  The reference parses --batch but trains
 *                         one sample per step (src/train.c:340-351); that stays
 *                         the default.
 */
#include "train.h"
#include "gguf.h"
#include "gguf_write.h"
#include "hw_probe.h"
#include "data.h"

#include "lora_body.h"
#include "lora_ce.h"
#include "lora_train.h"

#include <errno.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>

enum { kMaxRank = 256, kSampleCap = 2048 };
static const char kAdapterMagic[8] = {'L', 'O', 'R', 'A', '0', '0', '0', '1'};

struct train_state {
    forward_ctx* f;
    train_params p;
    int dim, vocab, rank;
    float scale;
    int step;
    float last_loss;
    lora_ce_handle* gpu;
    int have_weight;
    int max_pred;     /* positions of one sample: seq_max - 1 */
    int pack;         /* samples per step in train_run (1 unless LORA_TRAIN_PACK) */
    float* H;         /* [pack * max_pred][dim] hidden rows of the current step */
    int32_t* targets; /* [pack * max_pred] */
    float* logits;    /* [vocab]: the body forward writes base logits here */
    /* the GPU body forward (lora_train_set_body_gguf), when set: the step's
     * input tokens and sample offsets instead of hidden rows */
    lora_body_handle* body;
    int32_t* tokens_in;  /* [pack * max_pred] */
    int32_t offsets[kSampleCap + 1];
    int n_samples;
};

static double env_double(const char* name, double def) {
    const char* s = getenv(name);
    if (!s || !*s) return def;
    char* end = NULL;
    double v = strtod(s, &end);
    return (end && *end == '\0') ? v : def;
}

/* A ~ N(0, 2/dim) by Box-Muller on glibc rand() after srand(seed or 42),
 * B = 0: the initial adapter of src/train.c:79-90, drawn on the host so
 * that it is bit-identical to the reference's. */
static void kaiming_init(float* A, size_t n, int dim, int seed) {
    srand((unsigned)(seed ? seed : 42));
    const float sd = sqrtf(2.0f / (float)dim);
    for (size_t i = 0; i < n; i++) {
        const float u1 = ((float)rand() + 1.0f) / ((float)RAND_MAX + 1.0f);
        const float u2 = ((float)rand() + 1.0f) / ((float)RAND_MAX + 1.0f);
        A[i] = sqrtf(-2.0f * logf(u1)) * cosf(6.28318530718f * u2) * sd;
    }
}

static void report(const char* where, int rc) {
    fprintf(stderr, "%s: lora_ce error %d: %s\n", where, rc, lora_ce_last_error());
}

train_state* train_create(forward_ctx* f, const train_params* p) {
    if (!f || !p) return NULL;
    train_state* t = calloc(1, sizeof(*t));
    if (!t) return NULL;
    t->f = f;
    t->p = *p;
    t->dim = forward_dim(f);
    t->vocab = forward_vocab_size(f);
    t->rank = p->lora_rank > 0 ? p->lora_rank : 8;
    const int alpha = p->lora_alpha > 0 ? p->lora_alpha : 2 * t->rank;
    t->scale = (float)alpha / (float)t->rank;
    t->max_pred = p->seq_max > 1 ? p->seq_max - 1 : 1;
    t->pack = (env_double("LORA_TRAIN_PACK", 0.0) != 0.0 && p->batch > 1) ? p->batch : 1;

    lora_ce_config cfg;
    lora_ce_default_config(&cfg, t->dim, t->vocab, t->rank, t->max_pred * t->pack);
    cfg.scale = t->scale;
    cfg.lr = p->lr;
    cfg.weight_decay = (float)env_double("LORA_CE_WEIGHT_DECAY", 0.0);
    cfg.clip_norm = (float)env_double("LORA_CE_CLIP_NORM", 0.0);
    cfg.device = (int32_t)env_double("LORA_CE_DEVICE", 0.0);
    int rc = lora_ce_create(&cfg, &t->gpu);
    if (rc != LORA_CE_OK) {
        report("train_create", rc);
        free(t);
        return NULL;
    }

    const size_t na = (size_t)t->dim * t->rank, nb = (size_t)t->rank * t->vocab;
    float* A = malloc(na * sizeof(float));
    float* B = calloc(nb, sizeof(float));
    t->H = malloc((size_t)t->pack * t->max_pred * t->dim * sizeof(float));
    t->targets = malloc((size_t)t->pack * t->max_pred * sizeof(int32_t));
    t->logits = malloc((size_t)t->vocab * sizeof(float));
    if (!A || !B || !t->H || !t->targets || !t->logits) {
        free(A);
        free(B);
        train_free(t);
        return NULL;
    }
    kaiming_init(A, na, t->dim, p->seed);
    rc = lora_ce_set_adapter(t->gpu, A, B, 0);
    free(A);
    free(B);
    if (rc != LORA_CE_OK) {
        report("train_create", rc);
        train_free(t);
        return NULL;
    }
    return t;
}

void train_free(train_state* t) {
    if (!t) return;
    if (t->body) lora_body_destroy(t->body);
    free(t->tokens_in);
    if (t->gpu) lora_ce_destroy(t->gpu);
    free(t->H);
    free(t->targets);
    free(t->logits);
    free(t);
}

int lora_train_set_lm_head(train_state* t, const uint16_t* w_f16) {
    if (!t || !w_f16) return -1;
    const int rc = lora_ce_set_weight_f16(t->gpu, w_f16);
    if (rc != LORA_CE_OK) {
        report("lora_train_set_lm_head", rc);
        return -1;
    }
    t->have_weight = 1;
    return 0;
}

int lora_train_set_lm_head_gguf(train_state* t, const gguf_ctx* g) {
    if (!t || !g) return -1;
    const gguf_tensor_info* ti = gguf_tensor_get(g, "token_embd.weight");
    const int shape_ok = ti && (int)ti->dims[0] == t->dim && (int)ti->dims[1] == t->vocab;
    if (!shape_ok || (ti->dtype != GGUF_DT_F16 && ti->dtype != GGUF_DT_Q4_K)) {
        fprintf(stderr,
                "lora_train: no F16 or Q4_K token_embd.weight of [%d x %d] in the model\n",
                t->vocab, t->dim);
        return -1;
    }
    const void* data = gguf_tensor_data(g, ti);
    if (ti->dtype == GGUF_DT_F16) return lora_train_set_lm_head(t, (const uint16_t*)data);
    /* QLoRA: Q4_K super-blocks over the flattened tensor, dequantised once
     * on the GPU into the f16 operand of the step */
    const int rc = lora_ce_set_weight_q4k(t->gpu, data);
    if (rc != LORA_CE_OK) {
        report("lora_train_set_lm_head_gguf", rc);
        return -1;
    }
    t->have_weight = 1;
    return 0;
}

int lora_train_set_body_gguf(train_state* t, const gguf_ctx* g) {
    if (!t || !g || t->body) return -1;
    lora_body_config c;
    memset(&c, 0, sizeof(c));
    c.n_layers = (int)gguf_kv_i64(g, "llama.block_count", -1);
    c.n_heads = (int)gguf_kv_i64(g, "llama.attention.head_count", -1);
    c.n_kv_heads = (int)gguf_kv_i64(g, "llama.attention.head_count_kv", -1);
    c.ffn_hidden = (int)gguf_kv_i64(g, "llama.feed_forward_length", -1);
    c.rms_eps = gguf_kv_f32(g, "llama.attention.layer_norm_rms_epsilon", 1e-5f);
    c.rope_theta = gguf_kv_f32(g, "llama.rope.freq_base", 10000.0f);
    c.dim = t->dim;
    c.vocab = t->vocab;
    c.max_seq = t->max_pred;
    c.max_tokens = t->max_pred * t->pack;
    c.device = (int32_t)env_double("LORA_CE_DEVICE", 0.0);
    lora_body_handle* b = NULL;
    int rc = lora_body_create(&c, &b);
    const gguf_tensor_info* e = gguf_tensor_get(g, "token_embd.weight");
    const gguf_tensor_info* on = gguf_tensor_get(g, "output_norm.weight");
    if (!rc && (!e || e->dtype != GGUF_DT_F16 || !on || on->dtype != GGUF_DT_F32)) rc = -1;
    if (!rc) rc = lora_body_set_embedding(b, (const uint16_t*)gguf_tensor_data(g, e),
                                          (const float*)gguf_tensor_data(g, on));
    static const char* const names[9] = {"attn_norm", "attn_q", "attn_k", "attn_v",
                                         "attn_output", "ffn_norm", "ffn_gate", "ffn_up",
                                         "ffn_down"};
    for (int L = 0; L < c.n_layers && !rc; L++) {
        const void* d[9];
        for (int k = 0; k < 9 && !rc; k++) {
            char name[96];
            snprintf(name, sizeof(name), "blk.%d.%s.weight", L, names[k]);
            const gguf_tensor_info* ti = gguf_tensor_get(g, name);
            const gguf_dtype want = (k == 0 || k == 5) ? GGUF_DT_F32 : GGUF_DT_F16;
            if (!ti || ti->dtype != want) rc = -1;
            else d[k] = gguf_tensor_data(g, ti);
        }
        if (!rc)
            rc = lora_body_set_layer(b, L, (const float*)d[0], (const uint16_t*)d[1],
                                     (const uint16_t*)d[2], (const uint16_t*)d[3],
                                     (const uint16_t*)d[4], (const float*)d[5],
                                     (const uint16_t*)d[6], (const uint16_t*)d[7],
                                     (const uint16_t*)d[8]);
    }
    int32_t* tok = rc ? NULL : malloc((size_t)c.max_tokens * sizeof(int32_t));
    if (rc || !tok) {
        fprintf(stderr, "lora_train_set_body_gguf: %s\n",
                rc > 0 || rc == -1 ? "model tensors missing or of an unsupported type"
                                   : lora_body_last_error());
        if (b) lora_body_destroy(b);
        free(tok);
        return -1;
    }
    t->body = b;
    t->tokens_in = tok;
    return 0;
}

/* The predicted positions of one sample (src/train.c:198-229): positions
 * 0 .. use_n-2 with use_n = min(n_tokens, seq_max), position pos predicting
 * tokens[pos+1], hidden rows from one prefill and use_n-2 decodes of the
 * body forward, stored from row `at` of the step buffers.  Returns the
 * number of positions, or -1. */
static int gather_sample(train_state* t, const int* tokens, int n_tokens, int at) {
    if (!tokens || n_tokens < 2) return -1;
    const int use_n = n_tokens < t->p.seq_max ? n_tokens : t->p.seq_max;
    if (use_n < 2) return -1;
    const int n_pred = use_n - 1;
    for (int pos = 0; pos < n_pred; pos++) {
        const int tgt = tokens[pos + 1];
        if (tgt < 0 || tgt >= t->vocab) return -1;
        t->targets[at + pos] = tgt;
    }
    if (t->body) {  /* the GPU body runs over the whole step at once */
        if (at == 0) t->n_samples = 0;
        for (int pos = 0; pos < n_pred; pos++) {
            if (tokens[pos] < 0 || tokens[pos] >= t->vocab) return -1;
            t->tokens_in[at + pos] = tokens[pos];
        }
        t->offsets[t->n_samples] = at;
        t->offsets[++t->n_samples] = at + n_pred;
        return n_pred;
    }
    forward_reset(t->f);
    if (forward_prefill(t->f, tokens, 1, t->logits) < 0) return -1;
    for (int pos = 0; pos < n_pred; pos++) {
        const float* h = forward_last_hidden(t->f);
        if (!h) return -1;
        memcpy(t->H + (size_t)(at + pos) * t->dim, h, (size_t)t->dim * sizeof(float));
        if (pos + 1 < n_pred && forward_decode(t->f, tokens[pos + 1], pos + 1, t->logits) < 0)
            return -1;
    }
    return n_pred;
}

/* One GPU step over the n gathered positions: the mean loss, or -1.0f. */
static float step_positions(train_state* t, int n, const char* where) {
    float loss = -1.0f;
    int rc;
    if (t->body) {
        rc = lora_body_train_step(t->body, t->gpu, t->tokens_in, t->offsets, t->n_samples,
                                  t->targets, &loss);
        if (rc != LORA_CE_OK) {
            fprintf(stderr, "%s: lora_body error %d: %s\n", where, rc, lora_body_last_error());
            return -1.0f;
        }
        t->step++;
        t->last_loss = loss;
        return loss;
    }
    rc = lora_ce_step(t->gpu, t->H, LORA_CE_F32, n, t->targets, &loss);
    if (rc != LORA_CE_OK) {
        report(where, rc);
        return -1.0f;
    }
    t->step++;
    t->last_loss = loss;
    return loss;
}

/* src/train.c:198-242: the mean loss over the sample's predicted positions,
 * or -1.0f on any failure. */
float train_step(train_state* t, const int* tokens, int n_tokens) {
    if (!t || !tokens || n_tokens < 2) return -1.0f;
    if (!t->have_weight) {
        fprintf(stderr, "train_step: lm_head weight not set (lora_train_set_lm_head)\n");
        return -1.0f;
    }
    const int n = gather_sample(t, tokens, n_tokens, 0);
    if (n < 1) return -1.0f;
    return step_positions(t, n, "train_step");
}

/* LORA0001 (src/train.c:244-258): magic, int32 {dim, vocab, rank, step},
 * f32 scale, f32 A [dim][rank], f32 B [rank][vocab]. */
int train_save(const train_state* t, const char* path) {
    if (!t || !path) return -1;
    const size_t na = (size_t)t->dim * t->rank, nb = (size_t)t->rank * t->vocab;
    float* buf = malloc((na + nb) * sizeof(float));
    if (!buf) return -1;
    int32_t step = 0;
    if (lora_ce_get_adapter(t->gpu, buf, buf + na, &step) != LORA_CE_OK) {
        report("train_save", -1);
        free(buf);
        return -1;
    }
    FILE* f = fopen(path, "wb");
    if (!f) {
        perror("train_save");
        free(buf);
        return -1;
    }
    const int32_t hdr[4] = {t->dim, t->vocab, t->rank, step};
    const float scale = t->scale;
    fwrite(kAdapterMagic, 1, sizeof(kAdapterMagic), f);
    fwrite(hdr, sizeof(int32_t), 4, f);
    fwrite(&scale, sizeof(float), 1, f);
    fwrite(buf, sizeof(float), na + nb, f);
    fclose(f);
    free(buf);
    return 0;
}

/* Reads a LORA0001 file of the same dim / vocab / rank (src/train.c:
 * 260-283): the step counter and the scale come from the file. */
int train_load(train_state* t, const char* path) {
    if (!t || !path) return -1;
    FILE* f = fopen(path, "rb");
    if (!f) return -1;
    char magic[8];
    int32_t hdr[4];
    float scale;
    if (fread(magic, 1, 8, f) != 8 || memcmp(magic, kAdapterMagic, 8) != 0 ||
        fread(hdr, sizeof(int32_t), 4, f) != 4) {
        fclose(f);
        return -1;
    }
    if (hdr[0] != t->dim || hdr[1] != t->vocab || hdr[2] != t->rank) {
        fprintf(stderr, "train_load: shape mismatch\n");
        fclose(f);
        return -1;
    }
    const size_t na = (size_t)t->dim * t->rank, nb = (size_t)t->rank * t->vocab;
    float* buf = malloc((na + nb) * sizeof(float));
    if (!buf || fread(&scale, sizeof(float), 1, f) != 1 ||
        fread(buf, sizeof(float), na + nb, f) != na + nb) {
        free(buf);
        fclose(f);
        return -1;
    }
    fclose(f);
    int rc = lora_ce_set_adapter(t->gpu, buf, buf + na, hdr[3]);
    if (rc == LORA_CE_OK) rc = lora_ce_set_scale(t->gpu, scale);
    free(buf);
    if (rc != LORA_CE_OK) {
        report("train_load", rc);
        return -1;
    }
    t->step = hdr[3];
    t->scale = scale;
    return 0;
}

/* ---------------------------------------------------------------- train_run
 * The packed dataset of src/data.c: <packed>.idx holds n sample_idx records
 * followed by a 20-byte trailer {int32 n, int32 total, int32 fmt,
 * char magic[8] = "STUDIO.."}; <packed> holds the int32 token ids. */
typedef struct {
    sample_idx* samples;
    int n;
    FILE* tokens;
} packed_set;

static int packed_open(packed_set* ps, const char* packed_path) {
    char idx_path[1024];
    snprintf(idx_path, sizeof(idx_path), "%s.idx", packed_path);
    FILE* idx = fopen(idx_path, "rb");
    if (!idx) {
        perror("train_run open idx");
        return -1;
    }
    int32_t trailer[3];
    char magic[8];
    if (fseek(idx, -20, SEEK_END) != 0 || fread(trailer, sizeof(int32_t), 3, idx) != 3 ||
        fread(magic, 1, 8, idx) != 8) {
        fclose(idx);
        return -1;
    }
    if (memcmp(magic, "STUDIO", 6) != 0) {
        fprintf(stderr, "train_run: bad packed magic\n");
        fclose(idx);
        return -1;
    }
    ps->n = trailer[0];
    if (ps->n <= 0) {
        fclose(idx);
        return -1;
    }
    ps->samples = malloc((size_t)ps->n * sizeof(sample_idx));
    if (!ps->samples) {
        fclose(idx);
        return -1;
    }
    rewind(idx);
    const size_t got = fread(ps->samples, sizeof(sample_idx), (size_t)ps->n, idx);
    fclose(idx);
    if (got != (size_t)ps->n) {
        free(ps->samples);
        return -1;
    }
    ps->tokens = fopen(packed_path, "rb");
    if (!ps->tokens) {
        perror("train_run open packed");
        free(ps->samples);
        return -1;
    }
    return 0;
}

static void packed_close(packed_set* ps) {
    free(ps->samples);
    fclose(ps->tokens);
}

/* Tokens of sample s (at most cap of them), or -1. */
static int packed_read(const packed_set* ps, int s, int* out, int cap) {
    int n = ps->samples[s].n_tokens;
    if (n > cap) n = cap;
    if (fseek(ps->tokens, ps->samples[s].offset, SEEK_SET) != 0) return -1;
    return (int)fread(out, sizeof(int), (size_t)n, ps->tokens);
}

int train_run(train_state* t, const char* packed_path, const train_params* p,
              const char* out_dir) {
    if (!t || !packed_path || !p || !out_dir) return -1;
    packed_set ps;
    if (packed_open(&ps, packed_path) != 0) return -1;
    mkdir(out_dir, 0755);

    const int max_steps = p->max_steps > 0 ? p->max_steps : ps.n * p->epochs;
    static int tokens[kSampleCap];
    char path[1024];
    int step = 0;
    float first_loss = -1.0f;
    /* packing (LORA_TRAIN_PACK): samples gathered for the next step */
    int packed = 0, packed_pos = 0, packed_first = 0;
    const int last_epoch = p->epochs - 1;
    for (int epoch = 0; epoch < p->epochs && step < max_steps; epoch++) {
        for (int s = 0; s < ps.n && step < max_steps; s++) {
            const int n = packed_read(&ps, s, tokens, kSampleCap);
            const int final_sample = epoch == last_epoch && s == ps.n - 1;
            float loss = -1.0f;
            int sample = s;
            if (t->pack == 1) {
                if (n < 2) continue;
                loss = train_step(t, tokens, n);
            } else {
                const int k = (n >= 2 && t->have_weight) ? gather_sample(t, tokens, n, packed_pos) : -1;
                if (k > 0) {
                    if (packed == 0) packed_first = s;
                    packed_pos += k;
                    ++packed;
                }
                if (packed == 0 || (packed < t->pack && !final_sample)) continue;
                loss = step_positions(t, packed_pos, "train_run");
                sample = packed_first;
                packed = packed_pos = 0;
            }
            if (loss < 0) continue;
            if (first_loss < 0) first_loss = loss;
            step++;
            printf("step=%d epoch=%d sample=%d loss=%.4f\n", step, epoch, sample, loss);
            fflush(stdout);

            /* memory watchdog (src/train.c:354-368) */
            hw_caps caps;
            hw_probe(&caps);
            if (p->simulate_mem_kb > 0) caps.mem_avail_kb = p->simulate_mem_kb;
            if (caps.mem_avail_kb < (long)MEM_EMERGENCY_MB * 1024) {
                snprintf(path, sizeof(path), "%s/emergency_%d.bin", out_dir, step);
                train_save(t, path);
                fprintf(stderr,
                        "train: emergency save at step %d (mem_avail=%ld MB, threshold=%d MB)\n",
                        step, caps.mem_avail_kb / 1024, MEM_EMERGENCY_MB);
                packed_close(&ps);
                return 0;
            }
            if (p->checkpoint_every > 0 && step % p->checkpoint_every == 0) {
                snprintf(path, sizeof(path), "%s/lora_%d.bin", out_dir, step);
                train_save(t, path);
            }
        }
    }
    snprintf(path, sizeof(path), "%s/lora_final.bin", out_dir);
    train_save(t, path);
    printf("train: done steps=%d first_loss=%.4f last_loss=%.4f adapter=%s\n", step, first_loss,
           t->last_loss, path);
    packed_close(&ps);
    return 0;
}

/* -------------------------------------------------------------- train_merge
 * src/train.c:465-542: read the adapter, patch token_embd.weight of the base
 * GGUF with W + scale * (A.B)^T and write the result with
 * gguf_patch_tensor.  The patched tensor comes from lora_ce_merge_weight,
 * bit-identical to the reference's lora_patched_weight. */
typedef struct {
    int dim, vocab, rank, step;
    float scale;
    float* A;
    float* B;
} adapter_file;

static int adapter_read(adapter_file* a, const char* path) {
    memset(a, 0, sizeof(*a));
    FILE* f = fopen(path, "rb");
    if (!f) {
        perror("train_merge adapter");
        return -1;
    }
    char magic[8];
    int32_t hdr[4];
    if (fread(magic, 1, 8, f) != 8 || memcmp(magic, kAdapterMagic, 8) != 0) {
        fprintf(stderr, "train_merge: bad adapter magic\n");
        fclose(f);
        return -1;
    }
    if (fread(hdr, sizeof(int32_t), 4, f) != 4 || fread(&a->scale, sizeof(float), 1, f) != 1) {
        fclose(f);
        return -1;
    }
    a->dim = hdr[0];
    a->vocab = hdr[1];
    a->rank = hdr[2];
    a->step = hdr[3];
    if (a->rank > kMaxRank) {
        fprintf(stderr, "train_merge: adapter rank %d > %d\n", a->rank, kMaxRank);
        fclose(f);
        return -1;
    }
    const size_t na = (size_t)a->dim * a->rank, nb = (size_t)a->rank * a->vocab;
    a->A = malloc(na * sizeof(float));
    a->B = malloc(nb * sizeof(float));
    const int ok = a->A && a->B && fread(a->A, sizeof(float), na, f) == na &&
                   fread(a->B, sizeof(float), nb, f) == nb;
    fclose(f);
    if (!ok) {
        free(a->A);
        free(a->B);
        return -1;
    }
    return 0;
}

int train_merge(const char* base_gguf, const char* adapter_path, const char* out_gguf) {
    if (!base_gguf || !adapter_path || !out_gguf) return -1;
    adapter_file a;
    if (adapter_read(&a, adapter_path) != 0) return -1;

    gguf_ctx g;
    if (gguf_load(base_gguf, &g) < 0) {
        free(a.A);
        free(a.B);
        return -1;
    }
    const char* name = "token_embd.weight";
    const gguf_tensor_info* ti = gguf_tensor_get(&g, name);
    const uint16_t* base = NULL;
    int rc = -1;
    if (!ti) {
        fprintf(stderr, "train_merge: token_embd.weight not found in base\n");
    } else if (ti->dtype != GGUF_DT_F16) {
        fprintf(stderr, "train_merge: expected F16 token_embd.weight, got dtype=%d\n", ti->dtype);
    } else if ((int)ti->dims[1] != a.vocab || (int)ti->dims[0] != a.dim) {
        fprintf(stderr, "train_merge: shape mismatch adapter[%d,%d] vs tensor[%d,%d]\n", a.dim,
                a.vocab, (int)ti->dims[0], (int)ti->dims[1]);
    } else if (!(base = (const uint16_t*)gguf_tensor_data(&g, ti))) {
        fprintf(stderr, "train_merge: tensor_data null\n");
    } else {
        rc = 0;
    }
    const size_t bytes = (size_t)a.vocab * a.dim * sizeof(uint16_t);
    uint16_t* patched = rc == 0 ? malloc(bytes) : NULL;
    if (rc == 0 && !patched) rc = -1;
    if (rc == 0) {
        const int device = (int)env_double("LORA_CE_DEVICE", 0.0);
        const int mrc = lora_ce_merge_weight(base, a.A, a.B, a.dim, a.rank, a.vocab, a.scale,
                                             patched, device);
        if (mrc != LORA_CE_OK) {
            fprintf(stderr, "train_merge: lora_ce_merge_weight error %d: %s\n", mrc,
                    lora_ce_merge_last_error());
            rc = -1;
        }
    }
    gguf_free(&g);
    free(a.A);
    free(a.B);
    if (rc != 0) {
        free(patched);
        return -1;
    }
    rc = gguf_patch_tensor(base_gguf, out_gguf, name, patched, bytes);
    free(patched);
    if (rc < 0) {
        fprintf(stderr, "train_merge: gguf_patch_tensor failed\n");
        return -1;
    }
    printf("train_merge: patched token_embd.weight (step=%d rank=%d scale=%.4f) into %s (%zu "
           "bytes)\n",
           a.step, a.rank, a.scale, out_gguf, bytes);
    return 0;
}
