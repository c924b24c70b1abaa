/*
 * dc_oracle.h -- CPU oracle for the distcomp llama token loop.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the reference
 * engine's arithmetic (src/gguf.c:464-786 block dequant, src/engine.c:256-526
 * forward pass), written so that the CUDA path in distcomp_b200 can be checked
 * against it.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg may load it.  The product path never links or calls it.
 *
 * Every function keeps the reference's order of floating-point operations
 * (sequential fp32 accumulation, double sum of squares, separate roundings
 * of products) so that on x86-64 built with -O2 and no FMA it reproduces the
 * reference bit for bit.  tests/test_oracle_pins.py pins it against the
 * golden vectors of the reference's own tests and against the reference
 * engine compiled from its sources (oracle/_ref).
 */
#ifndef DC_ORACLE_H
#define DC_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_STAGE_EMBED = 0, ORC_STAGE_LAYERS = 1, ORC_STAGE_HEAD = 2 };

typedef struct orc_model orc_model;
typedef struct orc_ctx   orc_ctx;

/* IEEE binary16 -> binary32, exact (src/gguf.c:464-486 rd_f16). */
float  orc_f16(uint16_t h);

/* Bytes taken by `n_elems` elements of ggml type `type`; 0 for an unknown
 * type (src/gguf.c:149-174 tensor_nbytes). */
size_t orc_type_bytes(unsigned type, size_t n_elems);

/* Dequantise elements [off, off+n) of a tensor of `total` elements whose raw
 * blocks start at `raw`.  Returns 0, or -1 with the reference's rejection
 * rules: range, block alignment of `off`, unsupported type
 * (src/gguf.c:733-786 gguf_dequant). */
int    orc_dequant(unsigned type, const uint8_t *raw, size_t total, size_t off, size_t n,
                   float *dst);

/* y[o] = sum_i W[i + o*n_in] x[i] with the reference's accumulation order:
 * one fp32 accumulator per row, block by block (src/engine.c:287-343
 * matvec_range).  Rows whose n_in is not a multiple of the block give 0. */
void   orc_matvec(unsigned type, const uint8_t *raw, int n_in, int n_out, const float *x,
                  float *y);

/* The same product accumulated in double from the dequantised weights, as
 * the "exact" yardstick of the GEMV tolerance checks. */
void   orc_matvec_f64(unsigned type, const uint8_t *raw, int n_in, int n_out, const float *x,
                      double *y);

/* GGUF v2/v3 view over a caller-owned file image (src/gguf.c:233-336).
 * Returns NULL and fills err on a malformed file. */
orc_model *orc_model_open(const void *file, size_t size, char *err, size_t errlen);
void       orc_model_close(orc_model *m);
/* Look a tensor up by name; returns 0 and fills the outputs, or -1. */
int        orc_model_tensor(const orc_model *m, const char *name, unsigned *type,
                            unsigned *n_dims, uint64_t dims[4], const uint8_t **data,
                            size_t *nbytes);

/* Engine stage over a model (src/engine.c:145-246 llm_ctx_open).  n_ctx 0
 * takes the model's context length.  Returns NULL and fills err. */
orc_ctx *orc_ctx_open(const orc_model *m, int stage, int first, int last, int n_ctx,
                      char *err, size_t errlen);
void     orc_ctx_close(orc_ctx *c);
int      orc_forward(orc_ctx *c, int token, float *out);        /* engine.c:468 */
int      orc_layer_once(orc_ctx *c, int layer_idx, float *out);  /* engine.c:499 */
int      orc_step_layers(orc_ctx *c, int n, float *out);         /* engine.c:507 */
int      orc_pick(const orc_ctx *c);                             /* engine.c:517 */
void     orc_reset(orc_ctx *c);                                  /* engine.c:248 */
void     orc_set_pos(orc_ctx *c, int pos);
const float *orc_logits(const orc_ctx *c);
/* n_layer, n_embd, n_head, n_head_kv, n_ff, head_dim, n_vocab, n_ctx, pos,
 * stage, first, last -> out[0..11]; rms_eps, rope_base -> fout[0..1]. */
void     orc_geom(const orc_ctx *c, int out[12], float fout[2]);

#ifdef __cplusplus
}
#endif
#endif
