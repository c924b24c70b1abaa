/*
 * ref_shim.c -- thin ctypes-friendly wrapper around the REFERENCE engine.
 *
 * TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together
 * with the reference's own src/engine.c, src/gguf.c, src/thread.c and
 * src/util.c (read in place, never copied) into oracle/_ref/libdcref.so.
 * It owns the gguf_file / llm_ctx structs and the float arenas so that
 * Python can drive llm_ctx_open / llm_forward / llm_pick without knowing
 * their layouts.  Used to pin the oracle restatement and as the CPU
 * baseline that bench.py --impl reference times.
 */
#include "engine.h"
#include "gguf.h"
#include "thread.h"

#include <stdlib.h>
#include <string.h>

typedef struct {
    llm_ctx c;
    float  *arena;
} refw_ctx;

void *refw_model_open(const void *buf, size_t size, char *err, size_t errlen)
{
    gguf_file *g = calloc(1, sizeof *g);
    if (gguf_open(g, buf, size, err, errlen) != 0) { free(g); return NULL; }
    return g;
}

void refw_model_close(void *g)
{
    if (!g) return;
    gguf_close(g);
    free(g);
}

void *refw_ctx_open(void *g, int stage, int first, int last, int n_ctx, char *err, size_t errlen)
{
    refw_ctx *r = calloc(1, sizeof *r);
    size_t    n = llm_ctx_floats(g, stage, first, last, n_ctx);
    r->arena = calloc(n ? n : 1, sizeof(float));
    if (!r->arena ||
        llm_ctx_open(&r->c, g, stage, first, last, n_ctx, NULL, r->arena, n, err, errlen) != 0) {
        free(r->arena);
        free(r);
        return NULL;
    }
    return r;
}

void refw_ctx_close(void *p)
{
    refw_ctx *r = p;
    if (!r) return;
    free(r->c.layers);      /* xcalloc'd by llm_ctx_open when layer_store is NULL */
    free(r->arena);
    free(r);
}

int refw_forward(void *p, int token, float *out) { return llm_forward(&((refw_ctx *)p)->c, token, out); }
int refw_layer_once(void *p, int i, float *out) { return llm_layer_once(&((refw_ctx *)p)->c, i, out); }
int refw_step_layers(void *p, int n, float *out) { return llm_step_layers(&((refw_ctx *)p)->c, n, out); }
int refw_pick(void *p) { return llm_pick(&((refw_ctx *)p)->c); }
void refw_reset(void *p) { llm_reset(&((refw_ctx *)p)->c); }
void refw_set_pos(void *p, int pos) { ((refw_ctx *)p)->c.pos = pos; }
const float *refw_logits(void *p) { return ((refw_ctx *)p)->c.logits; }
size_t refw_ctx_floats(void *g, int stage, int first, int last, int n_ctx)
{
    return llm_ctx_floats(g, stage, first, last, n_ctx);
}

/* gguf_dequant over a bare block buffer of `total` elements */
int refw_dequant(unsigned type, const void *raw, size_t total, size_t off, size_t n, float *dst)
{
    gguf_tensor t;
    memset(&t, 0, sizeof t);
    t.type = type;
    t.n_dims = 1;
    t.dims[0] = total;
    t.data = raw;
    return gguf_dequant(&t, dst, off, n);
}

void refw_set_threads(int n) { tp_set(n); }
int  refw_threads(void) { return tp_threads(); }
