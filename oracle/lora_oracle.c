/*
 * lora_oracle.c — CPU restatement of smollm2.c's LoRA-on-lm_head training
 * step, used ONLY as test infrastructure (the parity checker for the CUDA
 * path, and the timed CPU baseline in bench.py).  Nothing in the product
 * library links or calls this file.
 *
 * Every function follows one reference function, op for op, so that with
 * one thread the results are bit-identical to the reference built from its
 * own sources (checked by tests/test_oracle.py against oracle/_ref and the
 * committed fixtures in tests/golden/):
 *
 *   oracle_base_logits   src/forward.c:396-403   (x86 matmul_f32: fp64 acc.)
 *   f16 -> f32           src/forward.c:256-286   (f16_to_f32, exact)
 *   per-token step       src/train.c:124-173     (matmul_hA, matmul_midB,
 *                                                 lora_accum)
 *   softmax-CE           src/train.c:107-121     (ce_loss_and_grad)
 *   mean over n_pred     src/train.c:230-237
 *   Adam                 src/train.c:175-196     (adam_update)
 *   target indexing      src/train.c:198-229     (targets = tokens[pos+1])
 *   Kaiming A init       src/train.c:83-93       (glibc rand, Box-Muller)
 *   softmax-CE gradcheck src/backward.c:450-503  (grad_check_softmax_ce)
 *   merge                src/train.c:393-460     (lora_patched_weight)
 *   Q4_K dequantisation  not in the reference (src/gguf.h:43 only names
 *                        GGUF_DT_Q4_K = 12; src/gguf.c:323 gives it size 0);
 *                        restated from the public GGUF / ggml format, so
 *                        its parity is unpinned by the reference
 *
 * Extensions that the reference does not have (weight decay, grad-clip) are
 * applied after the mean exactly where an AdamW implementation applies
 * them; with wd = 0 and clip = 0 they are no-ops, so the reference path is
 * unchanged.  Their "on" settings are parity-unpinned by the reference.
 *
 * Build: gcc -std=c99 -O2 -ffp-contract=off (no -march=native, no fast-math:
 * the reference's own -std=c99 build does not contract a*b+c either).
 * With nthreads > 1 the per-token gradient sums are accumulated per
 * contiguous token block and the blocks are added in block order: the
 * result is deterministic but no longer bit-identical to the reference's
 * single running sum (it differs by fp32 re-association only).
 */
#define _GNU_SOURCE
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_B1 0.9f
#define ORACLE_B2 0.999f
#define ORACLE_EPS 1e-8f
#define ORACLE_MAX_RANK 256

/* f16 bits -> f32, exact (src/forward.c:256-286). */
float oracle_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)(h & 0x8000u)) << 16;
    int exp = (h >> 10) & 0x1f;
    int mant = h & 0x3ff;
    float f;
    uint32_t u;
    if (exp == 0) {
        if (mant == 0) { u = sign; memcpy(&f, &u, 4); return f; }
        f = ldexpf((float)mant, -24);
        return sign ? -f : f;
    }
    if (exp == 0x1f) {
        u = sign | 0x7f800000u | ((uint32_t)mant << 13);
        memcpy(&f, &u, 4);
        return f;
    }
    u = sign | ((uint32_t)(exp + 127 - 15) << 23) | ((uint32_t)mant << 13);
    memcpy(&f, &u, 4);
    return f;
}

/* Base logits of one position: fp64 accumulation over the hidden dim, then
 * rounded to f32 (src/forward.c:396-403, the x86 branch of matmul_f32 that
 * the reference uses for the tied lm_head).  Wf is W converted to f32
 * (exact).  Eight rows are interleaved so the eight running sums pipeline;
 * each row is still summed in index order, so every logit is bit-identical
 * to the reference's one-row loop (the f16 x f32 products are exact in
 * fp64). */
static void base_logits_f32w(const float* Wf, const float* h, int d, int V,
                             float* out) {
    int o = 0;
    for (; o + 8 <= V; o += 8) {
        const float* w = Wf + (size_t)o * d;
        double a0 = 0, a1 = 0, a2 = 0, a3 = 0, a4 = 0, a5 = 0, a6 = 0, a7 = 0;
        for (int i = 0; i < d; i++) {
            double x = (double)h[i];
            a0 += (double)w[i] * x;
            a1 += (double)w[(size_t)d + i] * x;
            a2 += (double)w[(size_t)2 * d + i] * x;
            a3 += (double)w[(size_t)3 * d + i] * x;
            a4 += (double)w[(size_t)4 * d + i] * x;
            a5 += (double)w[(size_t)5 * d + i] * x;
            a6 += (double)w[(size_t)6 * d + i] * x;
            a7 += (double)w[(size_t)7 * d + i] * x;
        }
        out[o] = (float)a0; out[o + 1] = (float)a1; out[o + 2] = (float)a2;
        out[o + 3] = (float)a3; out[o + 4] = (float)a4; out[o + 5] = (float)a5;
        out[o + 6] = (float)a6; out[o + 7] = (float)a7;
    }
    for (; o < V; o++) {
        const float* w = Wf + (size_t)o * d;
        double acc = 0.0;
        for (int i = 0; i < d; i++) acc += (double)w[i] * (double)h[i];
        out[o] = (float)acc;
    }
}

static float* convert_weight(const uint16_t* W, int d, int V) {
    float* Wf = (float*)malloc((size_t)V * d * sizeof(float));
    if (!Wf) return NULL;
    for (size_t i = 0; i < (size_t)V * d; i++) Wf[i] = oracle_f16_to_f32(W[i]);
    return Wf;
}

void oracle_base_logits(const uint16_t* W, const float* h, int d, int V,
                        float* out) {
    float* Wf = convert_weight(W, d, V);
    if (!Wf) return;
    base_logits_f32w(Wf, h, d, V, out);
    free(Wf);
}

/* Softmax-CE on one row, in place: logits -> p - onehot; returns the loss
 * (src/train.c:107-121). */
static float ce_row(float* logits, int V, int target, float* dl) {
    float mx = logits[0];
    for (int i = 1; i < V; i++) if (logits[i] > mx) mx = logits[i];
    float sum = 0.0f;
    for (int i = 0; i < V; i++) {
        dl[i] = expf(logits[i] - mx);
        sum += dl[i];
    }
    float inv = 1.0f / sum;
    for (int i = 0; i < V; i++) dl[i] *= inv;
    float loss = -logf(dl[target] + 1e-12f);
    dl[target] -= 1.0f;
    return loss;
}

typedef struct {
    int d, V, r;
    float scale;
    const float* Wf;    /* [V][d] f32 copy of the f16 weight */
    const float* A;     /* [d][r] */
    const float* B;     /* [r][V] */
    const float* H;     /* [T][d] */
    const int32_t* tgt; /* [T]    */
    int t0, t1;         /* token block [t0, t1) */
    float* gA;          /* [d][r] partial (zeroed by caller) */
    float* gB;          /* [r][V] partial (zeroed by caller) */
    float* loss;        /* per-token loss [T] */
    int status;
} block_job;

/* Base logits of OB_P positions at once.  Every logit is the same
 * sequential fp64 sum over the hidden index as base_logits_f32w: each f16 x
 * f32 product is exact in fp64, so only the order of the adds matters (and
 * a fused multiply-add of an exact product rounds like the separate add).
 * The position block only lets one pass over W serve OB_P positions, which
 * makes the checker fast enough for full-size workloads.  hT is [d][OB_P]
 * (position-minor, zero rows past the block), out [OB_P][V]. */
#define OB_P 16
#include <immintrin.h>

__attribute__((target("avx2,fma")))
static void base_logits_blk_fma(const float* Wf, const double* hT, int d, int V,
                                float* out) {
    int o = 0;
    for (; o + 2 <= V; o += 2) {
        const float* w0 = Wf + (size_t)o * d;
        const float* w1 = w0 + d;
        __m256d a0 = _mm256_setzero_pd(), a1 = a0, a2 = a0, a3 = a0;
        __m256d b0 = a0, b1 = a0, b2 = a0, b3 = a0;
        for (int i = 0; i < d; i++) {
            const double* hp = hT + (size_t)i * OB_P;
            const __m256d h0 = _mm256_loadu_pd(hp), h1 = _mm256_loadu_pd(hp + 4);
            const __m256d h2 = _mm256_loadu_pd(hp + 8), h3 = _mm256_loadu_pd(hp + 12);
            const __m256d x0 = _mm256_set1_pd((double)w0[i]);
            const __m256d x1 = _mm256_set1_pd((double)w1[i]);
            a0 = _mm256_fmadd_pd(x0, h0, a0);
            a1 = _mm256_fmadd_pd(x0, h1, a1);
            a2 = _mm256_fmadd_pd(x0, h2, a2);
            a3 = _mm256_fmadd_pd(x0, h3, a3);
            b0 = _mm256_fmadd_pd(x1, h0, b0);
            b1 = _mm256_fmadd_pd(x1, h1, b1);
            b2 = _mm256_fmadd_pd(x1, h2, b2);
            b3 = _mm256_fmadd_pd(x1, h3, b3);
        }
        double ra[OB_P], rb[OB_P];
        _mm256_storeu_pd(ra, a0); _mm256_storeu_pd(ra + 4, a1);
        _mm256_storeu_pd(ra + 8, a2); _mm256_storeu_pd(ra + 12, a3);
        _mm256_storeu_pd(rb, b0); _mm256_storeu_pd(rb + 4, b1);
        _mm256_storeu_pd(rb + 8, b2); _mm256_storeu_pd(rb + 12, b3);
        for (int p = 0; p < OB_P; p++) {
            out[(size_t)p * V + o] = (float)ra[p];
            out[(size_t)p * V + o + 1] = (float)rb[p];
        }
    }
    for (; o < V; o++) {
        const float* w = Wf + (size_t)o * d;
        for (int p = 0; p < OB_P; p++) {
            double acc = 0.0;
            for (int i = 0; i < d; i++) acc += (double)w[i] * hT[(size_t)i * OB_P + p];
            out[(size_t)p * V + o] = (float)acc;
        }
    }
}

static void base_logits_blk_plain(const float* Wf, const double* hT, int d, int V,
                                  float* out) {
    for (int o = 0; o < V; o++) {
        const float* w = Wf + (size_t)o * d;
        double acc[OB_P];
        for (int p = 0; p < OB_P; p++) acc[p] = 0.0;
        for (int i = 0; i < d; i++) {
            const double x = (double)w[i];
            for (int p = 0; p < OB_P; p++) acc[p] += x * hT[(size_t)i * OB_P + p];
        }
        for (int p = 0; p < OB_P; p++) out[(size_t)p * V + o] = (float)acc[p];
    }
}

static void base_logits_blk(const float* Wf, const double* hT, int d, int V, float* out) {
    static int have_fma = -1;
    if (have_fma < 0) {
        __builtin_cpu_init();
        have_fma = __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
    }
    if (have_fma) base_logits_blk_fma(Wf, hT, d, V, out);
    else base_logits_blk_plain(Wf, hT, d, V, out);
}

/* lora_accum (src/train.c:144-173) for the tokens of one block, OB_P
 * positions at a time.  Every running sum of the reference keeps its own
 * order: matmul_hA sums over d, matmul_midB over r, the dU sum over v, and
 * the gA / gB accumulators take the positions in increasing order.  The
 * loops only interleave independent sums (positions, ranks or vocabulary
 * columns side by side), so each value is bit-identical to the reference's
 * one-position loops. */
#define OB_VT 2048
static void* run_block(void* arg) {
    block_job* j = (block_job*)arg;
    const int d = j->d, V = j->V, R = j->r;
    const float sc = j->scale;
    float* logits = (float*)malloc((size_t)OB_P * V * sizeof(float));
    float* delta = (float*)malloc((size_t)OB_P * V * sizeof(float));
    float* dlT = (float*)malloc((size_t)OB_P * V * sizeof(float));
    double* hT = (double*)malloc((size_t)d * OB_P * sizeof(double));
    float* mid = (float*)malloc((size_t)OB_P * R * sizeof(float));
    float* d_mid = (float*)malloc((size_t)OB_P * R * sizeof(float));
    if (!logits || !delta || !dlT || !hT || !mid || !d_mid) {
        j->status = -1;
        free(logits); free(delta); free(dlT); free(hT); free(mid); free(d_mid);
        return NULL;
    }
    for (int t0 = j->t0; t0 < j->t1; t0 += OB_P) {
        const int np = j->t1 - t0 < OB_P ? j->t1 - t0 : OB_P;
        const float* Hb = j->H + (size_t)t0 * d;
        for (int i = 0; i < d; i++)
            for (int p = 0; p < OB_P; p++)
                hT[(size_t)i * OB_P + p] = p < np ? (double)Hb[(size_t)p * d + i] : 0.0;
        base_logits_blk(j->Wf, hT, d, V, logits);
        /* matmul_hA: mid[r] = sum over i in index order */
        for (int p = 0; p < np; p++) {
            const float* restrict h = Hb + (size_t)p * d;
            float* restrict m = mid + (size_t)p * R;
            for (int r = 0; r < R; r++) m[r] = 0.0f;
            for (int i = 0; i < d; i++) {
                const float hi = h[i];
                const float* restrict Ai = j->A + (size_t)i * R;
                for (int r = 0; r < R; r++) m[r] += hi * Ai[r];
            }
        }
        /* matmul_midB: delta[v] = sum over r in rank order (vocabulary
         * tiles, so each tile of B is read once per position block) */
        for (int v0 = 0; v0 < V; v0 += OB_VT) {
            const int n = V - v0 < OB_VT ? V - v0 : OB_VT;
            for (int p = 0; p < np; p++) memset(delta + (size_t)p * V + v0, 0, (size_t)n * 4);
            for (int r = 0; r < R; r++) {
                const float* restrict Br = j->B + (size_t)r * V + v0;
                for (int p = 0; p < np; p++) {
                    const float mr = mid[(size_t)p * R + r];
                    float* restrict dp = delta + (size_t)p * V + v0;
                    for (int v = 0; v < n; v++) dp[v] += mr * Br[v];
                }
            }
        }
        /* z += s.delta, softmax-CE; delta becomes dlogits (reused, as the
         * reference does) */
        for (int p = 0; p < np; p++) {
            float* restrict lg = logits + (size_t)p * V;
            float* restrict dp = delta + (size_t)p * V;
            for (int v = 0; v < V; v++) lg[v] += sc * dp[v];
            j->loss[t0 + p] = ce_row(lg, V, j->tgt[t0 + p], dp);
        }
        /* dlogits transposed [v][OB_P] (zero past the block) for the dU sums */
        for (int v = 0; v < V; v++)
            for (int p = 0; p < OB_P; p++)
                dlT[(size_t)v * OB_P + p] = p < np ? delta[(size_t)p * V + v] : 0.0f;
        for (int r = 0; r < R; r++) {
            /* gB[r][v] += (s.mid[r]).dl[v], positions in order */
            float* restrict g = j->gB + (size_t)r * V;
            for (int p = 0; p < np; p++) {
                const float c = sc * mid[(size_t)p * R + r];
                const float* restrict dp = delta + (size_t)p * V;
                for (int v = 0; v < V; v++) g[v] += c * dp[v];
            }
            /* dU[r] = s . sum over v in index order, one chain per position */
            const float* restrict Br = j->B + (size_t)r * V;
            float sacc[OB_P];
            for (int p = 0; p < OB_P; p++) sacc[p] = 0.0f;
            for (int v = 0; v < V; v++) {
                const float bv = Br[v];
                const float* restrict x = dlT + (size_t)v * OB_P;
                for (int p = 0; p < OB_P; p++) sacc[p] += bv * x[p];
            }
            for (int p = 0; p < np; p++) d_mid[(size_t)p * R + r] = sc * sacc[p];
        }
        /* gA[i][r] += h[i].dU[r], positions in order */
        for (int i = 0; i < d; i++) {
            float* restrict gAi = j->gA + (size_t)i * R;
            for (int p = 0; p < np; p++) {
                const float hi = Hb[(size_t)p * d + i];
                const float* restrict dm = d_mid + (size_t)p * R;
                for (int r = 0; r < R; r++) gAi[r] += hi * dm[r];
            }
        }
    }
    free(logits); free(delta); free(dlT); free(hT); free(mid); free(d_mid);
    j->status = 0;
    return NULL;
}

/*
 * Gradient of one step: accumulated gA/gB over T positions (not yet
 * divided by n_pred) and the per-position loss.  targets[t] is the id the
 * position predicts.  Returns 0, or -1 on bad arguments (rank above the
 * reference's LORA_MAX_RANK, target out of range).
 */
int oracle_accumulate(int d, int V, int r, float scale, const uint16_t* W,
                      const float* A, const float* B, const float* H,
                      const int32_t* targets, int T, int nthreads,
                      float* gA_sum, float* gB_sum, float* loss_tok) {
    if (r < 1 || r > ORACLE_MAX_RANK || T < 1 || d < 1 || V < 1) return -1;
    for (int t = 0; t < T; t++)
        if (targets[t] < 0 || targets[t] >= V) return -1;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > T) nthreads = T;
    size_t a_sz = (size_t)d * r, b_sz = (size_t)r * V;
    memset(gA_sum, 0, a_sz * sizeof(float));
    memset(gB_sum, 0, b_sz * sizeof(float));
    block_job* jobs = (block_job*)calloc((size_t)nthreads, sizeof(block_job));
    pthread_t* th = (pthread_t*)calloc((size_t)nthreads, sizeof(pthread_t));
    if (!jobs || !th) { free(jobs); free(th); return -1; }
    float* Wf = convert_weight(W, d, V);
    int rc = Wf ? 0 : -1;
    for (int k = 0; k < nthreads; k++) {
        block_job* j = &jobs[k];
        j->d = d; j->V = V; j->r = r; j->scale = scale;
        j->Wf = Wf; j->A = A; j->B = B; j->H = H; j->tgt = targets;
        j->t0 = (int)((long long)T * k / nthreads);
        j->t1 = (int)((long long)T * (k + 1) / nthreads);
        j->loss = loss_tok;
        if (k == 0) { j->gA = gA_sum; j->gB = gB_sum; }
        else {
            j->gA = (float*)calloc(a_sz, sizeof(float));
            j->gB = (float*)calloc(b_sz, sizeof(float));
            if (!j->gA || !j->gB) rc = -1;
        }
    }
    if (rc == 0) {
        if (nthreads == 1) run_block(&jobs[0]);
        else {
            for (int k = 0; k < nthreads; k++) pthread_create(&th[k], NULL, run_block, &jobs[k]);
            for (int k = 0; k < nthreads; k++) pthread_join(th[k], NULL);
        }
        for (int k = 0; k < nthreads; k++) if (jobs[k].status != 0) rc = -1;
        for (int k = 1; k < nthreads && rc == 0; k++) {
            for (size_t i = 0; i < a_sz; i++) gA_sum[i] += jobs[k].gA[i];
            for (size_t i = 0; i < b_sz; i++) gB_sum[i] += jobs[k].gB[i];
        }
    }
    for (int k = 1; k < nthreads; k++) { free(jobs[k].gA); free(jobs[k].gB); }
    free(Wf);
    free(jobs);
    free(th);
    return rc;
}

/*
 * Optimizer part of train_step: g *= 1/n_pred (src/train.c:233-237), then
 * the extensions (global-norm clip, decoupled weight decay; no-ops at 0),
 * then adam_update (src/train.c:175-196).  *step is the Adam step counter
 * (incremented here, as the reference does).  gA/gB are overwritten with
 * the mean gradient actually applied.
 */
void oracle_adam(int d, int V, int r, float lr, float wd, float clip,
                 int n_pred, int* step, float* A, float* B, float* gA,
                 float* gB, float* mA, float* vA, float* mB, float* vB) {
    size_t a_sz = (size_t)d * r, b_sz = (size_t)r * V;
    float inv = 1.0f / (float)n_pred;
    for (size_t i = 0; i < a_sz; i++) gA[i] *= inv;
    for (size_t i = 0; i < b_sz; i++) gB[i] *= inv;
    if (clip > 0.0f) {
        double ss = 0.0;
        for (size_t i = 0; i < a_sz; i++) ss += (double)gA[i] * gA[i];
        for (size_t i = 0; i < b_sz; i++) ss += (double)gB[i] * gB[i];
        float norm = (float)sqrt(ss);
        float c = clip / (norm + 1e-6f);
        if (c < 1.0f) {
            for (size_t i = 0; i < a_sz; i++) gA[i] *= c;
            for (size_t i = 0; i < b_sz; i++) gB[i] *= c;
        }
    }
    (*step)++;
    float b1t = 1.0f - powf(ORACLE_B1, (float)*step);
    float b2t = 1.0f - powf(ORACLE_B2, (float)*step);
    for (size_t i = 0; i < a_sz; i++) {
        if (wd > 0.0f) A[i] -= lr * wd * A[i];
        mA[i] = ORACLE_B1 * mA[i] + (1 - ORACLE_B1) * gA[i];
        vA[i] = ORACLE_B2 * vA[i] + (1 - ORACLE_B2) * gA[i] * gA[i];
        float mhat = mA[i] / b1t;
        float vhat = vA[i] / b2t;
        A[i] -= lr * mhat / (sqrtf(vhat) + ORACLE_EPS);
    }
    for (size_t i = 0; i < b_sz; i++) {
        if (wd > 0.0f) B[i] -= lr * wd * B[i];
        mB[i] = ORACLE_B1 * mB[i] + (1 - ORACLE_B1) * gB[i];
        vB[i] = ORACLE_B2 * vB[i] + (1 - ORACLE_B2) * gB[i] * gB[i];
        float mhat = mB[i] / b1t;
        float vhat = vB[i] / b2t;
        B[i] -= lr * mhat / (sqrtf(vhat) + ORACLE_EPS);
    }
}

/*
 * Full step over one packed sample, as train_step does it
 * (src/train.c:198-242): use_n = min(n_tokens, seq_max); positions
 * 0..use_n-2 predict tokens[pos+1]; H holds the hidden state of each
 * position (row pos).  Returns the mean loss, or -1.0f on error.
 * gA/gB receive the mean gradient that was applied.
 */
float oracle_train_step(int d, int V, int r, float scale, float lr, float wd,
                        float clip, int seq_max, const uint16_t* W,
                        const float* H, const int32_t* tokens, int n_tokens,
                        int nthreads, int* step, float* A, float* B,
                        float* gA, float* gB, float* mA, float* vA,
                        float* mB, float* vB) {
    if (!tokens || n_tokens < 2) return -1.0f;
    int use_n = n_tokens;
    if (use_n > seq_max) use_n = seq_max;
    if (use_n < 2) return -1.0f;
    int n_pred = use_n - 1;
    float* loss = (float*)malloc((size_t)n_pred * sizeof(float));
    if (!loss) return -1.0f;
    if (oracle_accumulate(d, V, r, scale, W, A, B, H, tokens + 1, n_pred,
                          nthreads, gA, gB, loss) != 0) {
        free(loss);
        return -1.0f;
    }
    float total = 0.0f;
    for (int t = 0; t < n_pred; t++) total += loss[t];
    free(loss);
    oracle_adam(d, V, r, lr, wd, clip, n_pred, step, A, B, gA, gB, mA, vA, mB, vB);
    float inv = 1.0f / (float)n_pred;
    return total * inv;
}

/* Kaiming init of A via Box-Muller on glibc rand() (src/train.c:83-93);
 * B starts at zero. */
void oracle_kaiming_init(int seed, int d, int r, float* A) {
    srand((unsigned)(seed ? seed : 42));
    float std_a = sqrtf(2.0f / (float)d);
    size_t a_sz = (size_t)d * r;
    for (size_t i = 0; i < a_sz; i++) {
        float u1 = ((float)rand() + 1.0f) / ((float)RAND_MAX + 1.0f);
        float u2 = ((float)rand() + 1.0f) / ((float)RAND_MAX + 1.0f);
        float z = sqrtf(-2.0f * logf(u1)) * cosf(6.28318530718f * u2);
        A[i] = z * std_a;
    }
}

/* Softmax-CE finite-difference check (src/backward.c:450-503): vocab-sized
 * logits from srand(42) / randf()*0.5, target vocab/2; returns the max abs
 * difference between p - onehot and the centred fp64 difference. */
static float gc_randf(void) { return ((float)rand() / 2147483647.0f) - 0.5f; }

static double ce_fwd_d(const float* logits, int vocab, int target) {
    double mx = logits[0];
    for (int i = 1; i < vocab; i++) if (logits[i] > mx) mx = logits[i];
    double sum = 0;
    for (int i = 0; i < vocab; i++) sum += exp((double)logits[i] - mx);
    double pt = exp((double)logits[target] - mx) / sum;
    return -log(pt + 1e-20);
}

float oracle_grad_check_softmax_ce(int vocab, float eps) {
    srand(42u);
    float* logits = (float*)malloc((size_t)vocab * sizeof(float));
    float* probs = (float*)malloc((size_t)vocab * sizeof(float));
    float* g_num = (float*)malloc((size_t)vocab * sizeof(float));
    if (!logits || !probs || !g_num) { free(logits); free(probs); free(g_num); return -1.0f; }
    for (int i = 0; i < vocab; i++) logits[i] = gc_randf() * 0.5f;
    int target = vocab / 2;
    float mx = logits[0];
    for (int i = 1; i < vocab; i++) if (logits[i] > mx) mx = logits[i];
    float sum = 0;
    for (int i = 0; i < vocab; i++) { probs[i] = expf(logits[i] - mx); sum += probs[i]; }
    float inv = 1.0f / sum;
    for (int i = 0; i < vocab; i++) probs[i] *= inv;
    probs[target] -= 1.0f; /* analytic p - onehot */
    for (int i = 0; i < vocab; i++) {
        float o = logits[i];
        logits[i] = o + eps; double lp = ce_fwd_d(logits, vocab, target);
        logits[i] = o - eps; double lm = ce_fwd_d(logits, vocab, target);
        logits[i] = o;
        g_num[i] = (float)((lp - lm) / (2.0 * eps));
    }
    float err = 0.0f;
    for (int i = 0; i < vocab; i++) {
        float e = fabsf(probs[i] - g_num[i]);
        if (e > err) err = e;
    }
    free(logits); free(probs); free(g_num);
    return err;
}

/* Truncating f32 -> f16 of the merge path (src/train.c:393-409). */
/* The merge path's f32 -> f16 conversion (src/train.c:392-407), restated
 * as written: the normal branch adds 0x0C800000 and the subnormal branch
 * shifts too little, so the intermediate exceeds 16 bits and the return
 * type keeps the low 16 (the reference's own (uint16_t) cast).  The result
 * differs from an IEEE conversion for almost every finite input; the
 * forward path's converter (src/forward.c:250-258) does not have this. */
uint16_t oracle_merge_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x & 0x80000000u) >> 16;
    uint32_t em = x & 0x7fffffffu;
    if (em >= 0x47800000u) {
        if (em > 0x7f800000u) return (uint16_t)(sign | 0x7e00);
        return (uint16_t)(sign | 0x7c00);
    }
    if (em < 0x38800000u) {
        if (em < 0x33000000u) return (uint16_t)sign;
        uint32_t sh = 113 - (em >> 23);
        uint32_t mant = (em & 0x7fffff) | 0x800000;
        return (uint16_t)(sign | (mant >> sh));
    }
    return (uint16_t)(sign | ((em + 0xc800000) >> 13));
}

/* f16 -> f32 as the merge path converts it (src/train.c:433-454): exact for
 * normal values, but an f16 subnormal m * 2^-24 comes out as m * 2^-25,
 * because that normalisation loop starts from exponent 0 rather than 1.
 * Reproduced here because the merged weights must match the reference's. */
static float merge_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t mant = h & 0x3ffu;
    float f;
    if (exp == 0) {
        f = mant ? ldexpf((float)mant, -25) : 0.0f;
        uint32_t u;
        memcpy(&u, &f, 4);
        u |= sign;
        memcpy(&f, &u, 4);
        return f;
    }
    /* exponent 31 (f16 inf / NaN) maps to 2^16 * 1.f, as the same formula does there */
    uint32_t u = sign | ((exp + 112u) << 23) | (mant << 13);
    memcpy(&f, &u, 4);
    return f;
}

/* W' = f16trunc(f32(W) + scale * (A.B)^T), row v, col i (src/train.c:415-460). */
void oracle_merge(const uint16_t* W, const float* A, const float* B, int d,
                  int r, int V, float scale, uint16_t* out) {
    for (int v = 0; v < V; v++) {
        for (int i = 0; i < d; i++) {
            const float* arow = A + (size_t)i * r;
            float s = 0.0f;
            for (int k = 0; k < r; k++) s += arow[k] * B[(size_t)k * V + v];
            float delta = scale * s;
            float base = merge_f16_to_f32(W[(size_t)v * d + i]);
            out[(size_t)v * d + i] = oracle_merge_f32_to_f16(base + delta);
        }
    }
}

/* ------------------------------------------------------------------ Q4_K
 * The ggml / GGUF Q4_K super-block (type 12), 144 bytes per 256 weights:
 *   f16 d, f16 dmin, uint8 scales[12], uint8 qs[128].
 * scales packs eight 6-bit (scale, min) pairs, one per 32-weight sub-block j:
 *   j < 4:  sc = scales[j] & 63,  m = scales[j+4] & 63
 *   j >= 4: sc = (scales[j+4] & 15) | ((scales[j-4] >> 6) << 4)
 *           m  = (scales[j+4] >> 4) | ((scales[j]   >> 6) << 4)
 * The 256 weights are four runs of 64; run c reads qs[32c .. 32c+31]: the
 * low nibbles are sub-block 2c, the high nibbles sub-block 2c+1, and
 *   y = (d * sc) * q - (dmin * m)
 * with d, dmin converted exactly from f16 and every product and the
 * difference rounded separately (ggml's scalar order, no contraction).
 * Blocks run over the flattened tensor (for W [V][d], d = 576, a block can
 * span two rows).  This restatement is the parity anchor of the GPU
 * dequantisation. */
static void q4k_scale_min(int j, const uint8_t* q, int* sc, int* m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 15) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

void oracle_q4k_dequant(const uint8_t* blocks, int64_t n_blocks, float* out) {
    for (int64_t b = 0; b < n_blocks; b++) {
        const uint8_t* blk = blocks + b * 144;
        uint16_t dh, mh;
        memcpy(&dh, blk, 2);
        memcpy(&mh, blk + 2, 2);
        const float d = oracle_f16_to_f32(dh), dmin = oracle_f16_to_f32(mh);
        const uint8_t* scales = blk + 4;
        const uint8_t* qs = blk + 16;
        float* y = out + b * 256;
        for (int c = 0; c < 4; c++) {
            int sc, m;
            q4k_scale_min(2 * c, scales, &sc, &m);
            const float d1 = d * (float)sc, m1 = dmin * (float)m;
            q4k_scale_min(2 * c + 1, scales, &sc, &m);
            const float d2 = d * (float)sc, m2 = dmin * (float)m;
            for (int l = 0; l < 32; l++) {
                const float p1 = d1 * (float)(qs[32 * c + l] & 15);
                y[64 * c + l] = p1 - m1;
            }
            for (int l = 0; l < 32; l++) {
                const float p2 = d2 * (float)(qs[32 * c + l] >> 4);
                y[64 * c + 32 + l] = p2 - m2;
            }
        }
    }
}
