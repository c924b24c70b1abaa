/* A C host driving the engine through include/engine_cuda.h the way
 * distcomp's local run drives its CPU engine (src/shard.c:470-505 and the
 * prompt feed of src/shard.c:911-917): the GGUF image read into memory
 * whole, EMBED / LAYERS / HEAD stages, every prompt token through the three
 * stages, then greedy decoding with the token fed back through the host.
 *
 *   shard_local [--full] [--device N] model.gguf n_gen tok0 tok1 ...
 *
 * --full: one FULL context instead (embed + layers + head on the device),
 * the prompt through ecu_prefill.  Prints the n_gen generated tokens on one
 * line; exit status 1 with the library's message on any error. */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "engine_cuda.h"

static int fail(const char *what, const char *msg)
{
    fprintf(stderr, "shard_local: %s: %s\n", what, msg && msg[0] ? msg : ecu_last_error());
    return 1;
}

int main(int argc, char **argv)
{
    int full = 0, device = 0, a = 1;
    while (a < argc && strncmp(argv[a], "--", 2) == 0) {
        if (strcmp(argv[a], "--full") == 0) full = 1;
        else if (strcmp(argv[a], "--device") == 0 && a + 1 < argc) device = atoi(argv[++a]);
        else return fail("usage", "shard_local [--full] [--device N] model.gguf n_gen tokens...");
        a++;
    }
    if (argc - a < 3) return fail("usage", "shard_local [--full] [--device N] model.gguf n_gen tokens...");
    const char *path = argv[a];
    const int   n_gen = atoi(argv[a + 1]);
    const int   n_prompt = argc - a - 2;
    int        *prompt = malloc(sizeof(int) * (size_t)n_prompt);
    int        *gen = malloc(sizeof(int) * (size_t)(n_gen > 0 ? n_gen : 1));
    for (int i = 0; i < n_prompt; i++) prompt[i] = atoi(argv[a + 2 + i]);

    /* the whole file in memory, as llm_open_file does (src/shard.c:84-104) */
    FILE *f = fopen(path, "rb");
    if (!f) return fail("open", path);
    fseek(f, 0, SEEK_END);
    const long size = ftell(f);
    fseek(f, 0, SEEK_SET);
    unsigned char *img = malloc((size_t)size);
    if (!img || fread(img, 1, (size_t)size, f) != (size_t)size) return fail("read", path);
    fclose(f);

    char       err[256] = {0};
    ecu_model *m = NULL;
    if (ecu_model_open(&m, img, (size_t)size, err, sizeof err) != 0) return fail("ecu_model_open", err);

    if (full) {
        ecu_ctx *c = NULL;
        if (ecu_ctx_open(&c, m, ECU_STAGE_FULL, 0, 0, 0, device, err, sizeof err) != 0)
            return fail("ecu_ctx_open FULL", err);
        ecu_info info;
        ecu_ctx_info(c, &info);
        float *out = calloc((size_t)info.n_embd + 1, sizeof(float));
        if (ecu_prefill(c, prompt, n_prompt, out) != 0) return fail("ecu_prefill", NULL);
        int tok = (int)out[info.n_embd];
        for (int i = 0; i < n_gen; i++) {
            gen[i] = tok;
            if (i + 1 == n_gen) break;
            if (ecu_forward(c, tok, out) != 0) return fail("ecu_forward", NULL);
            tok = (int)out[info.n_embd];
        }
        free(out);
        ecu_ctx_close(c);
    } else {
        ecu_ctx *emb = NULL, *lay = NULL, *head = NULL;
        if (ecu_ctx_open(&emb, m, ECU_STAGE_EMBED, 0, 0, 0, device, err, sizeof err) != 0)
            return fail("ecu_ctx_open EMBED", err);
        ecu_info info;
        ecu_ctx_info(emb, &info);
        if (ecu_ctx_open(&lay, m, ECU_STAGE_LAYERS, 0, info.n_layer - 1, 0, device, err, sizeof err) != 0)
            return fail("ecu_ctx_open LAYERS", err);
        if (ecu_ctx_open(&head, m, ECU_STAGE_HEAD, 0, 0, 0, device, err, sizeof err) != 0)
            return fail("ecu_ctx_open HEAD", err);
        /* EMBED writes n_embd floats, HEAD n_embd + 1 (normed state, token) */
        float *st = calloc((size_t)info.n_embd + 8, sizeof(float));
        int    tok = -1;
        for (int i = 0; i < n_prompt + n_gen - 1; i++) {
            const int t = i < n_prompt ? prompt[i] : tok;
            if (ecu_forward(emb, t, st) != 0 || ecu_forward(lay, t, st) != 0 || ecu_forward(head, t, st) != 0)
                return fail("ecu_forward", NULL);
            tok = (int)st[info.n_embd];
            if (i >= n_prompt - 1) gen[i - (n_prompt - 1)] = tok;
        }
        free(st);
        ecu_ctx_close(head);
        ecu_ctx_close(lay);
        ecu_ctx_close(emb);
    }
    for (int i = 0; i < n_gen; i++) printf(i ? " %d" : "%d", gen[i]);
    printf("\n");
    ecu_model_close(m);
    free(img);
    free(prompt);
    free(gen);
    return 0;
}
