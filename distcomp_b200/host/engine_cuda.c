/*
 * engine_cuda.c -- the reference engine's API (src/engine.h:72-101:
 * llm_ctx_floats, llm_ctx_open, llm_forward, llm_reset, llm_layer_once,
 * llm_step_layers, llm_pick) implemented over this library's C ABI
 * (include/engine_cuda.h).  Linking a reference program (dcd, dcctl, the
 * reference's tests) with this file instead of src/engine.c puts its stage on
 * the GPU with no other change to the program: the dcd shard role
 * (src/daemon.c:942-1111, shard_shape / shard_gen) opens its stage through
 * llm_ctx_open and steps it through llm_forward / llm_pick, and the wire
 * format, planner and scheduler stay the reference's.
 *
 * The stage lives on CUDA device DC_CUDA_DEVICE (default 0).  The caller's
 * layer store and float arena are not used (weights, work buffers and KV
 * cache are device memory); the llm_ctx keeps the geometry fields the
 * callers read (stage, first, last, n_* , pos) and, for a HEAD stage, a host
 * copy of the last logits in `logits` (src/engine.h:67: [n_vocab], HEAD
 * only), refreshed by every llm_forward.  A caller that sets `pos` itself
 * (the reference's engine_stages test rewinds lay.pos between tokens) is
 * honoured: the stage's position follows the field before each step.  The
 * engine handle of each llm_ctx is kept in a small table keyed by the
 * llm_ctx's address; opening the same llm_ctx again closes its previous
 * stage first.
 */
#include "engine.h"

#include "engine_cuda.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define DCB_MAX_CTX 64

static struct {
    const llm_ctx *key;
    ecu_model     *m;
    ecu_ctx       *c;
    float         *logits;     /* HEAD: the host copy the llm_ctx points at */
} g_tab[DCB_MAX_CTX];

static int slot_of(const llm_ctx *c)
{
    for (int i = 0; i < DCB_MAX_CTX; i++)
        if (g_tab[i].key == c) return i;
    return -1;
}

static ecu_ctx *ctx_of(const llm_ctx *c)
{
    const int i = slot_of(c);
    return i < 0 ? NULL : g_tab[i].c;
}

static void drop(int i)
{
    if (i < 0) return;
    if (g_tab[i].c) ecu_ctx_close(g_tab[i].c);
    if (g_tab[i].m) ecu_model_close(g_tab[i].m);
    free(g_tab[i].logits);
    g_tab[i].key = NULL;
    g_tab[i].c = NULL;
    g_tab[i].m = NULL;
    g_tab[i].logits = NULL;
}

/* The caller may have set c->pos (the reference's callers rewind a LAYERS
 * stage that way): the device stage follows before the next step. */
static void follow_pos(llm_ctx *c, ecu_ctx *e)
{
    ecu_info in;
    if (ecu_ctx_info(e, &in) == 0 && in.pos != c->pos) ecu_set_pos(e, c->pos);
}

/* A HEAD stage's logits into the llm_ctx's host copy. */
static void pull_logits(llm_ctx *c, int slot)
{
    if (slot >= 0 && g_tab[slot].logits && c->n_vocab > 0)
        ecu_get_logits(g_tab[slot].c, g_tab[slot].logits, (size_t)c->n_vocab);
}

static int device_id(void)
{
    const char *d = getenv("DC_CUDA_DEVICE");
    return d ? atoi(d) : 0;
}

/* The reference's parsed file as this library's model: the metadata values
 * (numbers as u32 or f32 by their GGUF type, strings) and every tensor's
 * borrowed bytes. */
static ecu_model *model_from(const gguf_file *g)
{
    ecu_model *m = ecu_model_new();
    if (!m) return NULL;
    for (size_t i = 0; i < g->n_meta; i++) {
        const gguf_meta *k = &g->meta[i];
        if (!k->key) continue;
        switch (k->type) {
        case 8:  /* string */
            if (k->str) ecu_model_set_str(m, k->key, k->str);
            break;
        case 6:  /* f32 */
        case 12: /* f64 */
            ecu_model_set_f32(m, k->key, (float)k->num);
            break;
        case 9:  /* array: the engine reads none */
            break;
        default: /* integers and bool */
            ecu_model_set_u32(m, k->key, (unsigned long)k->num);
            break;
        }
    }
    for (size_t i = 0; i < g->n_tensors; i++) {
        const gguf_tensor *t = &g->tensors[i];
        uint64_t dims[4] = {1, 1, 1, 1};
        for (unsigned d = 0; d < t->n_dims && d < 4; d++) dims[d] = (uint64_t)t->dims[d];
        if (ecu_model_add_tensor(m, t->name, t->n_dims, dims, t->type, t->data, t->nbytes) != 0) {
            ecu_model_close(m);
            return NULL;
        }
    }
    return m;
}

static void copy_info(llm_ctx *c, ecu_ctx *e)
{
    ecu_info in;
    if (ecu_ctx_info(e, &in) != 0) return;
    c->n_layer = in.n_layer;
    c->n_embd = in.n_embd;
    c->n_head = in.n_head;
    c->n_head_kv = in.n_head_kv;
    c->n_ff = in.n_ff;
    c->head_dim = in.head_dim;
    c->n_vocab = in.n_vocab;
    c->n_rep = in.n_rep;
    c->rms_eps = in.rms_eps;
    c->rope_base = in.rope_base;
    c->n_ctx = in.n_ctx;
    c->stage = in.stage;
    c->first = in.first;
    c->last = in.last;
    c->pos = in.pos;
}

size_t llm_ctx_floats(const gguf_file *g, int stage, int first, int last, int n_ctx)
{
    /* what the stage needs, counted in floats like the reference's arena:
     * here it is device memory */
    ecu_model *m = model_from(g);
    if (!m) return 0;
    const size_t b = ecu_ctx_bytes(m, stage, first, last, n_ctx);
    ecu_model_close(m);
    return (b + sizeof(float) - 1) / sizeof(float);
}

int llm_ctx_open(llm_ctx *c, const gguf_file *g, int stage, int first, int last, int n_ctx,
                 llm_layer *layer_store, float *arena, size_t arena_floats, char *err, size_t errlen)
{
    (void)layer_store;
    (void)arena;
    (void)arena_floats;
    if (!c || !g) {
        if (err && errlen) snprintf(err, errlen, "null argument");
        return -1;
    }
    drop(slot_of(c));
    int i = slot_of(NULL);
    if (i < 0) {
        if (err && errlen) snprintf(err, errlen, "more than %d open GPU stages", DCB_MAX_CTX);
        return -1;
    }
    ecu_model *m = model_from(g);
    if (!m) {
        if (err && errlen) snprintf(err, errlen, "%s", ecu_last_error());
        return -1;
    }
    ecu_ctx *e = NULL;
    if (ecu_ctx_open(&e, m, stage, first, last, n_ctx, device_id(), err, errlen) != 0) {
        ecu_model_close(m);
        return -1;
    }
    memset(c, 0, sizeof *c);
    g_tab[i].key = c;
    g_tab[i].m = m;
    g_tab[i].c = e;
    copy_info(c, e);
    if (stage == LLM_STAGE_HEAD && c->n_vocab > 0) {
        g_tab[i].logits = calloc((size_t)c->n_vocab, sizeof(float));
        if (!g_tab[i].logits) {
            if (err && errlen) snprintf(err, errlen, "out of host memory for the logits");
            drop(i);
            return -1;
        }
        c->logits = g_tab[i].logits;
    }
    return 0;
}

int llm_forward(llm_ctx *c, int token, float *out)
{
    const int slot = slot_of(c);
    ecu_ctx  *e = slot < 0 ? NULL : g_tab[slot].c;
    if (!e) return -1;
    follow_pos(c, e);
    const int rc = ecu_forward(e, token, out);
    copy_info(c, e);
    if (rc == 0) pull_logits(c, slot);
    return rc;
}

void llm_reset(llm_ctx *c)
{
    ecu_ctx *e = ctx_of(c);
    if (!e) return;
    ecu_reset(e);
    copy_info(c, e);
}

int llm_layer_once(llm_ctx *c, int layer_idx, float *out)
{
    ecu_ctx *e = ctx_of(c);
    if (!e) return -1;
    follow_pos(c, e);
    return ecu_layer_once(e, layer_idx, out);
}

int llm_step_layers(llm_ctx *c, int n, float *out)
{
    ecu_ctx *e = ctx_of(c);
    if (!e) return -1;
    follow_pos(c, e);
    const int rc = ecu_step_layers(e, n, out);
    copy_info(c, e);
    return rc;
}

int llm_pick(const llm_ctx *c)
{
    ecu_ctx *e = ctx_of(c);
    return e ? ecu_pick(e) : 0;
}
