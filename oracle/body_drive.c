/*
 * body_drive.c — test infrastructure: the training command of the
 * reference's studio (src/studio.c:224-241, cmd_train) as a small program.
 * It loads the model, runs the reference's own body forward (src/forward.c),
 * then the trainer's train_run over a packed dataset.  oracle/Makefile
 * builds it twice:
 *   _ref/train_body_ref  with the reference's src/train.c (its CPU trainer)
 *   _ref/train_body_gpu  with smollm2.c_b200/liblora_train.so (the GPU
 *                        trainer; -DWITH_LORA_TRAIN adds the one call that
 *                        hands it token_embd.weight)
 *   _ref/train_body_gpubody  the same with -DWITH_GPU_BODY: the trainer
 *                        also runs the body forward on the GPU
 *                        (lora_train_set_body_gguf)
 * so a test can run both on the same model and data.  Never part of the
 * product.
 *
 *   train_body_* MODEL PACKED OUT_DIR RANK ALPHA SEQ LR MAX_STEPS SEED
 */
#include "train.h"
#include "gguf.h"
#ifdef WITH_LORA_TRAIN
#include "lora_train.h"
#endif

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

int main(int argc, char** argv) {
    if (argc != 10) {
        fprintf(stderr, "usage: %s MODEL PACKED OUT_DIR RANK ALPHA SEQ LR MAX_STEPS SEED\n",
                argv[0]);
        return 2;
    }
    train_params p;
    memset(&p, 0, sizeof(p));
    p.mode = TRAIN_LORA;
    p.lora_rank = atoi(argv[4]);
    p.lora_alpha = atoi(argv[5]);
    p.seq_max = atoi(argv[6]);
    p.batch = 1;
    p.lr = (float)atof(argv[7]);
    p.epochs = 1;
    p.checkpoint_every = 0;
    p.max_steps = atoi(argv[8]);
    p.seed = atoi(argv[9]);

    gguf_ctx g;
    if (gguf_load(argv[1], &g) < 0) {
        fprintf(stderr, "body_drive: cannot load model %s\n", argv[1]);
        return 1;
    }
    forward_ctx* f = NULL;
    if (forward_load(&f, &g, p.seq_max + 8) < 0) {
        fprintf(stderr, "body_drive: forward_load failed\n");
        gguf_free(&g);
        return 1;
    }
    train_state* t = train_create(f, &p);
    int rc = 1;
    if (!t) {
        fprintf(stderr, "body_drive: train_create failed\n");
    } else {
#ifdef WITH_LORA_TRAIN
        if (lora_train_set_lm_head_gguf(t, &g) != 0
#ifdef WITH_GPU_BODY
            || lora_train_set_body_gguf(t, &g) != 0
#endif
        ) {
            train_free(t);
            forward_free(f);
            gguf_free(&g);
            return 1;
        }
#endif
        rc = train_run(t, argv[2], &p, argv[3]) < 0 ? 1 : 0;
        train_free(t);
    }
    forward_free(f);
    gguf_free(&g);
    return rc;
}
