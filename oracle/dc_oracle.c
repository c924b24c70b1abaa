/*
 * dc_oracle.c -- CPU oracle (test infrastructure; see dc_oracle.h).
 *
 * A restatement of the reference path written for checking, not speed:
 *   - GGUF v2/v3 header walk            src/gguf.c:233-336
 *   - per-format block dequant           src/gguf.c:464-786
 *   - engine stages, matvec, RMSNorm,
 *     NeoX RoPE, KV cache, attention,
 *     SwiGLU, argmax                     src/engine.c:55-526
 * Build flags must match the reference's (-O2, no -ffast-math, no FMA
 * contraction on x86-64) for the bit-for-bit pins to hold; oracle/Makefile
 * sets them.
 */
#include "dc_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------ fp16 ---- */

float orc_f16(uint16_t h)
{
    /* binary16: 1 sign, 5 exponent (bias 15), 10 mantissa bits */
    uint32_t sign = (uint32_t)(h >> 15) & 1u;
    uint32_t e    = (uint32_t)(h >> 10) & 0x1Fu;
    uint32_t man  = (uint32_t)h & 0x3FFu;
    uint32_t bits;
    if (e == 0x1F) {
        bits = (sign << 31) | 0x7F800000u | (man << 13);        /* inf / NaN */
    } else if (e != 0) {
        bits = (sign << 31) | ((e + 112u) << 23) | (man << 13);  /* normal */
    } else if (man == 0) {
        bits = sign << 31;                                      /* +-0 */
    } else {
        /* subnormal: renormalise the mantissa, lowering the exponent */
        int shift = 0;
        while (!(man & 0x400u)) { man <<= 1; shift++; }
        man &= 0x3FFu;
        bits = (sign << 31) | ((uint32_t)(113 - shift) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

static float f16le(const uint8_t *p) { return orc_f16((uint16_t)(p[0] | (p[1] << 8))); }

/* ------------------------------------------------------- block sizes ---- */

/* elements per block and bytes per block; 0 bytes = not a block format */
static void blk_geom(unsigned type, size_t *elems, size_t *bytes)
{
    static const struct { unsigned t; unsigned short e, b; } tab[] = {
        { 2, 32, 18 }, { 3, 32, 20 }, { 6, 32, 22 }, { 7, 32, 24 }, { 8, 32, 34 },
        { 9, 32, 36 }, { 10, 256, 84 }, { 11, 256, 110 }, { 12, 256, 144 },
        { 13, 256, 176 }, { 14, 256, 210 }, { 15, 256, 292 },
    };
    for (size_t i = 0; i < sizeof tab / sizeof tab[0]; i++)
        if (tab[i].t == type) { *elems = tab[i].e; *bytes = tab[i].b; return; }
    *elems = 0;
    *bytes = 0;
}

size_t orc_type_bytes(unsigned type, size_t n)
{
    if (type == 0) return n * 4;
    if (type == 1) return n * 2;
    if (type == 16) return n / 32 * 2;   /* the reference sizes IQ4_NL this way (gguf.c:171) */
    size_t e, b;
    blk_geom(type, &e, &b);
    return e ? n / e * b : 0;
}

/* ------------------------------------------------------ block decoders ---- */
/* One function per format; each writes one whole block of `out`.  The
 * arithmetic (operand order, separate roundings) follows gguf.c exactly. */

static void dq_q4_0(const uint8_t *b, float *y)          /* gguf.c:662-671 */
{
    const float d = f16le(b);
    for (int i = 0; i < 16; i++) {
        int lo = b[2 + i] & 0x0F, hi = b[2 + i] >> 4;
        y[i]      = (float)(lo - 8) * d;
        y[i + 16] = (float)(hi - 8) * d;
    }
}

static void dq_q4_1(const uint8_t *b, float *y)          /* gguf.c:673-682 */
{
    const float d = f16le(b), m = f16le(b + 2);
    for (int i = 0; i < 16; i++) {
        float lo = (float)(b[4 + i] & 0x0F), hi = (float)(b[4 + i] >> 4);
        float plo = lo * d, phi = hi * d;
        y[i]      = plo + m;
        y[i + 16] = phi + m;
    }
}

static uint32_t le32(const uint8_t *p)
{
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) |
           ((uint32_t)p[3] << 24);
}

static void dq_q5_0(const uint8_t *b, float *y)          /* gguf.c:684-697 */
{
    const float    d  = f16le(b);
    const uint32_t hb = le32(b + 2);
    for (int i = 0; i < 16; i++) {
        int lo = (b[6 + i] & 0x0F) | (int)(((hb >> i) & 1u) << 4);
        int hi = (b[6 + i] >> 4) | (int)(((hb >> (i + 16)) & 1u) << 4);
        y[i]      = (float)(lo - 16) * d;
        y[i + 16] = (float)(hi - 16) * d;
    }
}

static void dq_q5_1(const uint8_t *b, float *y)          /* gguf.c:699-712 */
{
    const float    d = f16le(b), m = f16le(b + 2);
    const uint32_t hb = le32(b + 4);
    for (int i = 0; i < 16; i++) {
        int   lo = (b[8 + i] & 0x0F) | (int)(((hb >> i) & 1u) << 4);
        int   hi = (b[8 + i] >> 4) | (int)(((hb >> (i + 16)) & 1u) << 4);
        float plo = (float)lo * d, phi = (float)hi * d;
        y[i]      = plo + m;
        y[i + 16] = phi + m;
    }
}

static void dq_q8_0(const uint8_t *b, float *y)          /* gguf.c:714-720 */
{
    const float d = f16le(b);
    for (int i = 0; i < 32; i++) y[i] = d * (float)(int8_t)b[2 + i];
}

static void dq_q2_K(const uint8_t *b, float *y)          /* gguf.c:497-510 */
{
    const uint8_t *sc = b, *qs = b + 16;
    const float    d = f16le(b + 80), dmin = f16le(b + 82);
    for (int g = 0; g < 16; g++) {
        const uint8_t *q   = qs + (g >> 3) * 32 + (g & 1) * 16;
        const int      sh  = 2 * ((g >> 1) & 3);
        const float    dl  = d * (float)(sc[g] & 0x0F);
        const float    ml  = dmin * (float)(sc[g] >> 4);
        for (int k = 0; k < 16; k++) {
            float p = dl * (float)((q[k] >> sh) & 3);
            y[g * 16 + k] = p - ml;
        }
    }
}

static void dq_q3_K(const uint8_t *b, float *y)          /* gguf.c:527-554 */
{
    const uint8_t *hmask = b, *qs = b + 32, *sc = b + 96;
    const float    d = f16le(b + 108);
    for (int j = 0; j < 16; j++) {
        int   s6 = ((sc[j & 7] >> (4 * (j >> 3))) & 0x0F) |
                   (((sc[8 + (j & 3)] >> (2 * (j >> 2))) & 0x03) << 4);
        float dl = d * (float)(s6 - 32);
        const uint8_t *q = qs + (j >> 3) * 32 + (j & 1) * 16;
        const uint8_t *h = hmask + (j & 1) * 16;
        int   sh = 2 * ((j >> 1) & 3);
        for (int l = 0; l < 16; l++) {
            int low2 = (q[l] >> sh) & 3;
            int neg4 = (((h[l] >> (j >> 1)) & 1) ^ 1) << 2;
            y[j * 16 + l] = dl * (float)(low2 - neg4);
        }
    }
}

/* 6-bit scale/min pair j of a K-quant scale array (gguf.c:558-567) */
static void k_scale_min(int j, const uint8_t *s, int *sc, int *mn)
{
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        *mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

static void dq_q4_K(const uint8_t *b, float *y)          /* gguf.c:569-589 */
{
    const float    d = f16le(b), dmin = f16le(b + 2);
    const uint8_t *s = b + 4, *qs = b + 16;
    for (int c = 0; c < 4; c++) {
        int   sa, ma, sb, mb;
        k_scale_min(2 * c, s, &sa, &ma);
        k_scale_min(2 * c + 1, s, &sb, &mb);
        float da = d * (float)sa, mina = dmin * (float)ma;
        float db = d * (float)sb, minb = dmin * (float)mb;
        const uint8_t *q = qs + 32 * c;
        for (int l = 0; l < 32; l++) {
            float pa = da * (float)(q[l] & 0x0F);
            float pb = db * (float)(q[l] >> 4);
            y[64 * c + l]      = pa - mina;
            y[64 * c + 32 + l] = pb - minb;
        }
    }
}

/* The reference reads the same 32 qh bytes with shifts 0 and 2 for every
 * 64-weight chunk (gguf.c:592-615).  That is not ggml's Q5_K, but it is the
 * reference's, and the reference is what this oracle restates. */
static void dq_q5_K(const uint8_t *b, float *y)
{
    const float    d = f16le(b), dmin = f16le(b + 2);
    const uint8_t *s = b + 4, *qh = b + 16, *qs = b + 48;
    for (int c = 0; c < 4; c++) {
        int   sa, ma, sb, mb;
        k_scale_min(2 * c, s, &sa, &ma);
        k_scale_min(2 * c + 1, s, &sb, &mb);
        float da = d * (float)sa, mina = dmin * (float)ma;
        float db = d * (float)sb, minb = dmin * (float)mb;
        const uint8_t *q = qs + 32 * c;
        for (int l = 0; l < 32; l++) {
            int   va = (int)((q[l] & 0x0F) | ((qh[l] & 3) << 4)) - 16;
            int   vb = (int)((q[l] >> 4) | (((qh[l] >> 2) & 3) << 4)) - 16;
            float pa = da * (float)va, pb = db * (float)vb;
            y[64 * c + l]      = pa - mina;
            y[64 * c + 32 + l] = pb - minb;
        }
    }
}

static void dq_q6_K(const uint8_t *b, float *y)          /* gguf.c:631-647 */
{
    const uint8_t *ql = b, *qh = b + 128;
    const int8_t  *sc = (const int8_t *)(b + 192);
    const float    d  = f16le(b + 208);
    for (int idx = 0; idx < 256; idx++) {
        int r = idx >> 5, col = idx & 31;
        int lo = (ql[(r >> 2) * 64 + (r & 1) * 32 + col] >> (4 * ((r >> 1) & 1))) & 0x0F;
        int hi = (qh[(r >> 2) * 32 + col] >> (2 * (r & 3))) & 0x03;
        float ds = d * (float)sc[idx >> 4];
        y[idx] = ds * (float)((lo | (hi << 4)) - 32);
    }
}

static void dq_q8_K(const uint8_t *b, float *y)          /* gguf.c:650-659 */
{
    for (int g = 0; g < 32; g++) {
        float d = f16le(b + 256 + 2 * g);
        for (int k = 0; k < 8; k++) y[8 * g + k] = d * (float)(int8_t)b[8 * g + k];
    }
}

typedef void (*dq_fn)(const uint8_t *, float *);

static dq_fn dq_for(unsigned type)
{
    switch (type) {
    case 2:  return dq_q4_0;
    case 3:  return dq_q4_1;
    case 6:  return dq_q5_0;
    case 7:  return dq_q5_1;
    case 8:  return dq_q8_0;
    case 10: return dq_q2_K;
    case 11: return dq_q3_K;
    case 12: return dq_q4_K;
    case 13: return dq_q5_K;
    case 14: return dq_q6_K;
    case 15: return dq_q8_K;
    default: return NULL;   /* Q8_1, IQ*: rejected like gguf.c:765 */
    }
}

int orc_dequant(unsigned type, const uint8_t *raw, size_t total, size_t off, size_t n, float *dst)
{
    if (!raw || !dst) return -1;
    if (off > total || n > total - off) return -1;
    if (n == 0) return 0;
    if (type == 0) {
        memcpy(dst, raw + off * 4, n * 4);
        return 0;
    }
    if (type == 1) {
        for (size_t i = 0; i < n; i++) dst[i] = f16le(raw + 2 * (off + i));
        return 0;
    }
    dq_fn fn = dq_for(type);
    if (!fn) return -1;
    size_t be, bb;
    blk_geom(type, &be, &bb);
    if (off % be) return -1;
    size_t nblk = (n + be - 1) / be;
    if (off / be + nblk > total / be) return -1;
    float tmp[256];
    const uint8_t *p = raw + (off / be) * bb;
    for (size_t k = 0; k < nblk; k++, p += bb) {
        size_t take = n - k * be < be ? n - k * be : be;
        if (take == be) {
            fn(p, dst + k * be);
        } else {
            fn(p, tmp);                 /* last, partial block */
            memcpy(dst + k * be, tmp, take * sizeof(float));
        }
    }
    return 0;
}

/* ------------------------------------------------------------- matvec ---- */

/* `total` is the element count of the whole tensor, which bounds the block
 * reads exactly as gguf_dequant's range check does */
static void matvec_t(unsigned type, const uint8_t *raw, size_t total, int n_in, int n_out,
                     const float *x, float *y)
{
    if (n_out <= 0) return;
    if (type == 0 || type == 1) {
        for (int o = 0; o < n_out; o++) {
            float acc = 0.0f;
            if (type == 0) {
                const float *w = (const float *)(const void *)raw + (size_t)o * (size_t)n_in;
                for (int i = 0; i < n_in; i++) acc += w[i] * x[i];
            } else {
                const uint8_t *w = raw + (size_t)o * (size_t)n_in * 2;
                for (int i = 0; i < n_in; i++) acc += f16le(w + 2 * i) * x[i];
            }
            y[o] = acc;
        }
        return;
    }
    /* engine.c:316 picks 256 for types 10..15 and 32 for everything else */
    size_t blk = (type >= 10 && type <= 15) ? 256 : 32;
    if ((size_t)n_in % blk) {
        for (int o = 0; o < n_out; o++) y[o] = 0.0f;
        return;
    }
    float  w[256];
    for (int o = 0; o < n_out; o++) {
        float acc = 0.0f;
        for (size_t b = 0; b < (size_t)n_in / blk; b++) {
            if (orc_dequant(type, raw, total, (size_t)o * n_in + b * blk, blk, w) != 0) {
                for (int k = o; k < n_out; k++) y[k] = 0.0f;   /* engine.c:332-337 */
                return;
            }
            const float *xs = x + b * blk;
            for (size_t k = 0; k < blk; k++) acc += w[k] * xs[k];
        }
        y[o] = acc;
    }
}

void orc_matvec(unsigned type, const uint8_t *raw, int n_in, int n_out, const float *x, float *y)
{
    matvec_t(type, raw, (size_t)n_in * (size_t)(n_out > 0 ? n_out : 0), n_in, n_out, x, y);
}

void orc_matvec_f64(unsigned type, const uint8_t *raw, int n_in, int n_out, const float *x,
                    double *y)
{
    size_t total = (size_t)n_in * (size_t)n_out;
    float *row = (float *)malloc(sizeof(float) * (size_t)(n_in + 256));
    for (int o = 0; o < n_out; o++) {
        double acc = 0.0;
        if (orc_dequant(type, raw, total, (size_t)o * n_in, (size_t)n_in, row) == 0)
            for (int i = 0; i < n_in; i++) acc += (double)row[i] * (double)x[i];
        y[o] = acc;
    }
    free(row);
}

/* ------------------------------------------------------------- GGUF ---- */

typedef struct {
    char    *key;
    unsigned type;
    double   num;
    char    *str;
} orc_kv;

typedef struct {
    char          *name;
    unsigned       n_dims;
    uint64_t       dims[4];
    unsigned       type;
    uint64_t       off;
    size_t         nbytes;
    const uint8_t *data;
} orc_tensor;

struct orc_model {
    orc_kv     *kv;
    size_t      n_kv;
    orc_tensor *t;
    size_t      n_t;
    unsigned    alignment;
};

typedef struct {
    const uint8_t *base, *p;
    size_t         size;
    int            bad;
} cursor;

static size_t left(const cursor *c) { return c->size - (size_t)(c->p - c->base); }

static uint64_t rdn(cursor *c, int nbytes)
{
    if (c->bad || left(c) < (size_t)nbytes) { c->bad = 1; return 0; }
    uint64_t v = 0;
    for (int i = 0; i < nbytes; i++) v |= (uint64_t)c->p[i] << (8 * i);
    c->p += nbytes;
    return v;
}

static char *rdstr(cursor *c)
{
    uint64_t n = rdn(c, 8);
    if (c->bad || n > left(c)) { c->bad = 1; return NULL; }
    char *s = (char *)malloc((size_t)n + 1);
    memcpy(s, c->p, (size_t)n);
    s[n] = '\0';
    c->p += n;
    return s;
}

/* scalar metadata value of GGUF type `t` as a double (gguf.c:112-129).
 * FLOAT64 consumes two 8-byte words and joins them with a 32-bit shift,
 * exactly as the reference does (gguf.c:125-126). */
static double rdnum(cursor *c, unsigned t)
{
    uint64_t v;
    switch (t) {
    case 0:  return (double)rdn(c, 1);
    case 1:  return (double)(int8_t)rdn(c, 1);
    case 2:  return (double)rdn(c, 2);
    case 3:  return (double)(int16_t)rdn(c, 2);
    case 4:  return (double)rdn(c, 4);
    case 5:  return (double)(int32_t)rdn(c, 4);
    case 6: { uint32_t u = (uint32_t)rdn(c, 4); float f; memcpy(&f, &u, 4); return f; }
    case 7:  return rdn(c, 1) ? 1.0 : 0.0;
    case 10: return (double)rdn(c, 8);
    case 11: { v = rdn(c, 8); int64_t s; memcpy(&s, &v, 8); return (double)s; }
    case 12: { uint64_t lo = rdn(c, 8), hi = rdn(c, 8); v = lo | (hi << 32);
               double dd; memcpy(&dd, &v, 8); return dd; }
    default: c->bad = 1; return 0;
    }
}

static size_t scalar_size(unsigned t)
{
    switch (t) {
    case 0: case 1: case 7: return 1;
    case 2: case 3:         return 2;
    case 4: case 5: case 6: return 4;
    case 10: case 11: case 12: return 8;
    default: return 0;
    }
}

void orc_model_close(orc_model *m)
{
    if (!m) return;
    for (size_t i = 0; i < m->n_kv; i++) { free(m->kv[i].key); free(m->kv[i].str); }
    for (size_t i = 0; i < m->n_t; i++) free(m->t[i].name);
    free(m->kv);
    free(m->t);
    free(m);
}

#define FAIL(...) do { snprintf(err, errlen, __VA_ARGS__); orc_model_close(m); return NULL; } while (0)

orc_model *orc_model_open(const void *file, size_t size, char *err, size_t errlen)
{
    orc_model *m = (orc_model *)calloc(1, sizeof *m);
    cursor     c = { (const uint8_t *)file, (const uint8_t *)file, size, 0 };
    m->alignment = 32;
    if (size < 24) FAIL("file too small for GGUF (%zu bytes)", size);
    if (rdn(&c, 4) != 0x46554747u) FAIL("bad magic");
    unsigned version = (unsigned)rdn(&c, 4);
    if (version < 2 || version > 3) FAIL("GGUF version %u unsupported", version);
    uint64_t nt = rdn(&c, 8), nkv = rdn(&c, 8);
    if (nt > size || nkv > size) FAIL("count larger than the file");
    if (nt == 0 || nt > 4096 || nkv > 4096) FAIL("implausible tensor/key counts");
    m->kv = (orc_kv *)calloc(nkv ? nkv : 1, sizeof *m->kv);
    m->t  = (orc_tensor *)calloc(nt, sizeof *m->t);
    for (uint64_t i = 0; i < nkv; i++) {
        orc_kv *kv = &m->kv[m->n_kv];
        kv->key  = rdstr(&c);
        kv->type = (unsigned)rdn(&c, 4);
        m->n_kv++;
        if (c.bad) FAIL("truncated metadata");
        if (kv->type > 12) FAIL("metadata key %s has unknown type %u", kv->key, kv->type);
        if (kv->type == 8) {
            kv->str = rdstr(&c);
        } else if (kv->type == 9) {
            unsigned at = (unsigned)rdn(&c, 4);
            uint64_t an = rdn(&c, 8);
            if (c.bad || an > left(&c)) FAIL("bad array");
            if (at == 8) {
                for (uint64_t k = 0; k < an && !c.bad; k++) free(rdstr(&c));
            } else {
                size_t step = scalar_size(at);
                if (!step || an * step > size) FAIL("bad array in metadata");
                for (uint64_t k = 0; k < an && !c.bad; k++) (void)rdnum(&c, at);
            }
        } else {
            kv->num = rdnum(&c, kv->type);
        }
        if (c.bad) FAIL("truncated metadata");
    }
    for (uint64_t i = 0; i < nt; i++) {
        orc_tensor *t = &m->t[m->n_t];
        t->name = rdstr(&c);
        m->n_t++;
        t->n_dims = (unsigned)rdn(&c, 4);
        if (c.bad) FAIL("truncated tensor table");
        if (t->n_dims > 4) FAIL("tensor with more than 4 dims");
        size_t total = 1;
        for (unsigned d = 0; d < t->n_dims; d++) {
            t->dims[d] = rdn(&c, 8);
            if (!t->dims[d]) FAIL("zero tensor dimension");
            total *= (size_t)t->dims[d];
        }
        t->type   = (unsigned)rdn(&c, 4);
        t->off    = rdn(&c, 8);
        if (c.bad) FAIL("truncated tensor table");
        t->nbytes = orc_type_bytes(t->type, total);
    }
    for (size_t i = 0; i < m->n_kv; i++)
        if (strcmp(m->kv[i].key, "general.alignment") == 0 && m->kv[i].num >= 1 &&
            m->kv[i].num <= 65536)
            m->alignment = (unsigned)m->kv[i].num;
    size_t base = (size_t)(c.p - c.base);
    base = (base + m->alignment - 1) / m->alignment * m->alignment;
    for (size_t i = 0; i < m->n_t; i++) {
        orc_tensor *t = &m->t[i];
        if (t->off > size || base + t->off + t->nbytes > size)
            FAIL("tensor %s lies outside the file", t->name);
        t->data = (const uint8_t *)file + base + t->off;
    }
    return m;
}
#undef FAIL

static const orc_kv *kv_find(const orc_model *m, const char *key)
{
    for (size_t i = 0; i < m->n_kv; i++)
        if (strcmp(m->kv[i].key, key) == 0) return &m->kv[i];
    return NULL;
}

/* arch-prefixed lookup first, then the bare key (gguf.c:390-400) */
static const orc_kv *kv_arch(const orc_model *m, const char *key, const char *arch)
{
    const orc_kv *kv = NULL;
    if (arch && *arch) {
        char full[160];
        snprintf(full, sizeof full, "%s.%s", arch, key);
        kv = kv_find(m, full);
    }
    return kv ? kv : kv_find(m, key);
}

static int get_u(const orc_model *m, const char *key, const char *arch, unsigned long *out)
{
    const orc_kv *kv = kv_arch(m, key, arch);
    if (!kv || kv->type == 8 || kv->type == 9) return -1;
    *out = (unsigned long)kv->num;
    return 0;
}

static int get_f(const orc_model *m, const char *key, const char *arch, float *out)
{
    const orc_kv *kv = kv_arch(m, key, arch);
    if (!kv || kv->type == 8 || kv->type == 9) return -1;
    *out = (float)kv->num;
    return 0;
}

static const orc_tensor *t_find(const orc_model *m, const char *name)
{
    for (size_t i = 0; i < m->n_t; i++)
        if (strcmp(m->t[i].name, name) == 0) return &m->t[i];
    return NULL;
}

int orc_model_tensor(const orc_model *m, const char *name, unsigned *type, unsigned *n_dims,
                     uint64_t dims[4], const uint8_t **data, size_t *nbytes)
{
    const orc_tensor *t = t_find(m, name);
    if (!t) return -1;
    *type = t->type;
    *n_dims = t->n_dims;
    for (int i = 0; i < 4; i++) dims[i] = i < (int)t->n_dims ? t->dims[i] : 1;
    *data = t->data;
    *nbytes = t->nbytes;
    return 0;
}

static size_t t_elems(const orc_tensor *t)
{
    size_t n = 1;
    for (unsigned i = 0; i < t->n_dims; i++) n *= (size_t)t->dims[i];
    return n;
}

/* ------------------------------------------------------------ engine ---- */

typedef struct {
    const orc_tensor *attn_norm, *wq, *wk, *wv, *wo, *ffn_norm, *wg, *wu, *wd;
    const orc_tensor *bq, *bk, *bv;
} orc_layer;

struct orc_ctx {
    int   n_layer, n_embd, n_head, n_head_kv, n_ff, head_dim, n_vocab, n_rep, n_ctx;
    float eps, rope_base;
    int   stage, first, last, pos;
    const orc_tensor *emb, *out_norm, *out_w;
    orc_layer *layers;
    float *xb, *xb2, *xb3, *wn, *q, *k, *v, *att, *bias, *qh, *scores, *logits, *kc, *vc;
};

/* dequantise the head of a tensor; zeros when that fails (engine.c:360-364) */
static void to_float(const orc_tensor *t, float *dst, size_t off, size_t n)
{
    if (orc_dequant(t->type, t->data, t_elems(t), off, n, dst) != 0)
        for (size_t i = 0; i < n; i++) dst[i] = 0.0f;
}

static void mv(float *y, const orc_tensor *w, const float *x, int n_in, int n_out)
{
    matvec_t(w->type, w->data, t_elems(w), n_in, n_out, x, y);
}

#define CERR(...) do { snprintf(err, errlen, __VA_ARGS__); orc_ctx_close(c); return NULL; } while (0)

orc_ctx *orc_ctx_open(const orc_model *m, int stage, int first, int last, int n_ctx, char *err,
                      size_t errlen)
{
    orc_ctx *c = (orc_ctx *)calloc(1, sizeof *c);
    const orc_kv *a = kv_find(m, "general.architecture");
    const char *arch = a ? a->str : NULL;
    if (!arch || !*arch) CERR("model has no general.architecture");
    if (strcmp(arch, "llama") != 0 && strcmp(arch, "qwen2") != 0)
        CERR("architecture %s is not supported", arch);

    /* geometry, engine.c:55-109 */
    unsigned long v;
    if (get_u(m, "block_count", arch, &v)) CERR("missing %s.block_count", arch);
    c->n_layer = (int)v;
    if (get_u(m, "embedding_length", arch, &v)) CERR("missing %s.embedding_length", arch);
    c->n_embd = (int)v;
    if (get_u(m, "feed_forward_length", arch, &v)) CERR("missing %s.feed_forward_length", arch);
    c->n_ff = (int)v;
    if (get_u(m, "attention.head_count", arch, &v)) CERR("missing %s.attention.head_count", arch);
    c->n_head = (int)v;
    c->n_head_kv = get_u(m, "attention.head_count_kv", arch, &v) ? c->n_head : (int)v;
    unsigned long ctxlen = 512;
    get_u(m, "context_length", arch, &ctxlen);
    c->n_ctx = (int)ctxlen;
    float eps = 1e-5f;
    if (get_f(m, "attention.layer_norm_rms_epsilon", arch, &eps) &&
        get_f(m, "attention.layer_norm_epsilon", arch, &eps))
        eps = 1e-5f;
    c->eps = eps;
    float rope = 10000.0f;
    get_f(m, "rope.freq_base", arch, &rope);
    c->rope_base = rope > 0 ? rope : 10000.0f;
    if (c->n_head <= 0 || c->n_embd % c->n_head) CERR("n_embd %d not divisible by n_head %d", c->n_embd, c->n_head);
    c->head_dim = c->n_embd / c->n_head;
    if (c->n_head_kv <= 0 || c->n_head % c->n_head_kv) CERR("n_head %d not divisible by n_head_kv %d", c->n_head, c->n_head_kv);
    c->n_rep = c->n_head / c->n_head_kv;
    unsigned long rd = 0;
    if (get_u(m, "rope.dimension_count", arch, &rd) == 0 && rd > 0) c->head_dim = (int)rd;
    const orc_tensor *te = t_find(m, "token_embd.weight");
    if (te) {
        if (te->n_dims != 2) CERR("token_embd.weight: expected 2 dims");
        c->n_vocab = (int)te->dims[1];
    } else if (get_u(m, "vocab_size", arch, &v) == 0) {
        c->n_vocab = (int)v;
    }
    if (c->n_ctx <= 0) c->n_ctx = 512;
    if (n_ctx > 0) c->n_ctx = n_ctx;

    if (stage == ORC_STAGE_LAYERS && (last < first || last >= c->n_layer))
        CERR("layers %d..%d outside the model (%d layers)", first, last, c->n_layer);
    c->stage = stage;
    c->first = first;
    c->last = last;
    if ((stage == ORC_STAGE_EMBED || stage == ORC_STAGE_HEAD) && c->n_vocab <= 0)
        CERR("cannot determine n_vocab for stage %d", stage);

    if (stage == ORC_STAGE_EMBED) {
        if (!(c->emb = te)) CERR("missing token_embd.weight");
    } else if (stage == ORC_STAGE_HEAD) {
        if (!(c->out_norm = t_find(m, "output_norm.weight"))) CERR("missing output_norm.weight");
        c->out_w = t_find(m, "output.weight");
        if (!c->out_w && !(c->out_w = te)) CERR("missing output.weight and token_embd.weight");
    } else {
        int n = last - first + 1;
        c->layers = (orc_layer *)calloc((size_t)n, sizeof *c->layers);
        static const char *sfx[9] = { "attn_norm.weight", "attn_q.weight", "attn_k.weight",
                                      "attn_v.weight", "attn_output.weight", "ffn_norm.weight",
                                      "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight" };
        for (int i = 0; i < n; i++) {
            orc_layer *L = &c->layers[i];
            const orc_tensor **slot[9] = { &L->attn_norm, &L->wq, &L->wk, &L->wv, &L->wo,
                                           &L->ffn_norm, &L->wg, &L->wu, &L->wd };
            char name[128];
            for (int k = 0; k < 9; k++) {
                snprintf(name, sizeof name, "blk.%d.%s", first + i, sfx[k]);
                if (!(*slot[k] = t_find(m, name))) CERR("missing tensor %s", name);
            }
            snprintf(name, sizeof name, "blk.%d.attn_q.bias", first + i); L->bq = t_find(m, name);
            snprintf(name, sizeof name, "blk.%d.attn_k.bias", first + i); L->bk = t_find(m, name);
            snprintf(name, sizeof name, "blk.%d.attn_v.bias", first + i); L->bv = t_find(m, name);
        }
    }

    int    wide = c->n_ff > c->n_embd ? c->n_ff : c->n_embd;
    size_t qd = (size_t)c->n_head * c->head_dim, kvd = (size_t)c->n_head_kv * c->head_dim;
    c->xb = (float *)calloc((size_t)c->n_embd, 4);
    c->xb2 = (float *)calloc((size_t)wide, 4);
    c->xb3 = (float *)calloc((size_t)c->n_ff, 4);
    c->wn = (float *)calloc((size_t)c->n_embd, 4);
    c->q = (float *)calloc(qd, 4);
    c->att = (float *)calloc(qd, 4);
    c->k = (float *)calloc(kvd, 4);
    c->v = (float *)calloc(kvd, 4);
    c->bias = (float *)calloc(qd > kvd ? qd : kvd, 4);
    c->qh = (float *)calloc((size_t)c->head_dim, 4);
    c->scores = (float *)calloc((size_t)c->n_ctx, 4);
    if (stage == ORC_STAGE_HEAD) c->logits = (float *)calloc((size_t)c->n_vocab, 4);
    if (stage == ORC_STAGE_LAYERS) {
        size_t per = (size_t)c->n_ctx * kvd * (size_t)(last - first + 1);
        c->kc = (float *)calloc(per, 4);
        c->vc = (float *)calloc(per, 4);
        if (!c->kc || !c->vc) CERR("out of memory for the KV cache");
    }
    return c;
}
#undef CERR

void orc_ctx_close(orc_ctx *c)
{
    if (!c) return;
    free(c->layers); free(c->xb); free(c->xb2); free(c->xb3); free(c->wn); free(c->q);
    free(c->att); free(c->k); free(c->v); free(c->bias); free(c->qh); free(c->scores);
    free(c->logits); free(c->kc); free(c->vc);
    free(c);
}

void orc_reset(orc_ctx *c) { if (c) c->pos = 0; }
void orc_set_pos(orc_ctx *c, int pos) { if (c) c->pos = pos; }
const float *orc_logits(const orc_ctx *c) { return c ? c->logits : NULL; }

void orc_geom(const orc_ctx *c, int out[12], float fout[2])
{
    int g[12] = { c->n_layer, c->n_embd, c->n_head, c->n_head_kv, c->n_ff, c->head_dim,
                  c->n_vocab, c->n_ctx, c->pos, c->stage, c->first, c->last };
    memcpy(out, g, sizeof g);
    fout[0] = c->eps;
    fout[1] = c->rope_base;
}

static void rmsnorm(float *dst, const float *x, const float *w, int n, float eps)
{
    double ss = 0.0;
    for (int i = 0; i < n; i++) ss += (double)x[i] * x[i];
    const float scale = 1.0f / sqrtf((float)(ss / n) + eps);
    for (int i = 0; i < n; i++) {
        float t = x[i] * scale;
        dst[i] = t * w[i];
    }
}

/* NeoX half-split rotation of (v[i], v[i + n/2]) (engine.c:367-378) */
static void rope(float *v, int n, int pos, float base)
{
    const int half = n / 2;
    for (int i = 0; i < half; i++) {
        float theta = (float)pos * powf(base, -2.0f * (float)i / (float)n);
        float cs = cosf(theta), sn = sinf(theta);
        float a = v[i], b = v[half + i];
        float ac = a * cs, bs = b * sn, bc = b * cs, as = a * sn;
        v[i]        = ac - bs;
        v[half + i] = bc + as;
    }
}

static void layer(orc_ctx *c, const orc_layer *L, int li, float *x)
{
    const int    ne = c->n_embd, hd = c->head_dim, nh = c->n_head, nkv = c->n_head_kv;
    const size_t kvd = (size_t)nkv * hd, plane = (size_t)c->n_ctx * kvd;

    to_float(L->attn_norm, c->wn, 0, (size_t)ne);
    rmsnorm(c->xb, x, c->wn, ne, c->eps);
    mv(c->q, L->wq, c->xb, ne, nh * hd);
    mv(c->k, L->wk, c->xb, ne, nkv * hd);
    mv(c->v, L->wv, c->xb, ne, nkv * hd);
    if (L->bq) { to_float(L->bq, c->bias, 0, (size_t)nh * hd); for (int i = 0; i < nh * hd; i++) c->q[i] += c->bias[i]; }
    if (L->bk) { to_float(L->bk, c->bias, 0, kvd); for (size_t i = 0; i < kvd; i++) c->k[i] += c->bias[i]; }
    if (L->bv) { to_float(L->bv, c->bias, 0, kvd); for (size_t i = 0; i < kvd; i++) c->v[i] += c->bias[i]; }

    float *kl = c->kc + (size_t)li * plane, *vl = c->vc + (size_t)li * plane;
    float *krow = kl + (size_t)c->pos * kvd, *vrow = vl + (size_t)c->pos * kvd;
    memcpy(krow, c->k, kvd * sizeof(float));
    memcpy(vrow, c->v, kvd * sizeof(float));
    for (int j = 0; j < nkv; j++) rope(krow + (size_t)j * hd, hd, c->pos, c->rope_base);

    const int   npos = c->pos + 1;
    const float kscale = 1.0f / sqrtf((float)hd);
    for (int h = 0; h < nh; h++) {
        const size_t koff = (size_t)(h / c->n_rep) * hd;
        memcpy(c->qh, c->q + (size_t)h * hd, (size_t)hd * sizeof(float));
        rope(c->qh, hd, c->pos, c->rope_base);
        float mx = -3.4e38f;
        for (int t = 0; t < npos; t++) {
            const float *kk = kl + (size_t)t * kvd + koff;
            float dot = 0.0f;
            for (int j = 0; j < hd; j++) dot += c->qh[j] * kk[j];
            dot *= kscale;
            c->scores[t] = dot;
            if (dot > mx) mx = dot;
        }
        float sum = 0.0f;
        for (int t = 0; t < npos; t++) {
            float e = expf(c->scores[t] - mx);
            c->scores[t] = e;
            sum += e;
        }
        float *acc = c->att + (size_t)h * hd;
        for (int j = 0; j < hd; j++) acc[j] = 0.0f;
        const float inv = sum > 0 ? 1.0f / sum : 0.0f;
        for (int t = 0; t < npos; t++) {
            const float *vv = vl + (size_t)t * kvd + koff;
            const float wgt = c->scores[t] * inv;
            for (int j = 0; j < hd; j++) acc[j] += vv[j] * wgt;
        }
    }

    mv(c->xb2, L->wo, c->att, nh * hd, ne);
    for (int i = 0; i < ne; i++) x[i] += c->xb2[i];

    to_float(L->ffn_norm, c->wn, 0, (size_t)ne);
    rmsnorm(c->xb, x, c->wn, ne, c->eps);
    mv(c->xb2, L->wg, c->xb, ne, c->n_ff);
    mv(c->xb3, L->wu, c->xb, ne, c->n_ff);
    for (int j = 0; j < c->n_ff; j++) {
        const float g = c->xb2[j];
        c->xb2[j] = (g / (1.0f + expf(-g))) * c->xb3[j];
    }
    mv(c->xb, L->wd, c->xb2, c->n_ff, ne);
    for (int i = 0; i < ne; i++) x[i] += c->xb[i];
}

int orc_pick(const orc_ctx *c)
{
    if (!c || !c->logits) return 0;
    int   best = 0;
    float bv = c->logits[0];
    for (int i = 1; i < c->n_vocab; i++)
        if (c->logits[i] > bv) { bv = c->logits[i]; best = i; }
    return best;
}

int orc_layer_once(orc_ctx *c, int idx, float *out)
{
    if (!c || c->stage != ORC_STAGE_LAYERS || !out) return -1;
    if (idx < 0 || idx > c->last - c->first) return -1;
    layer(c, &c->layers[idx], idx, out);
    return 0;
}

int orc_step_layers(orc_ctx *c, int n, float *out)
{
    if (!c || c->stage != ORC_STAGE_LAYERS || !out) return -1;
    if (n <= 0) n = c->last - c->first + 1;
    if (c->pos >= c->n_ctx) return -1;
    for (int i = 0; i < n; i++) layer(c, &c->layers[i], i, out);
    c->pos++;
    return 0;
}

int orc_forward(orc_ctx *c, int token, float *out)
{
    if (!c || !out) return -1;
    if (c->stage == ORC_STAGE_EMBED) {
        int rows = c->emb->n_dims == 2 ? (int)c->emb->dims[1] : c->n_vocab;
        if (token < 0 || token >= rows) return -1;
        to_float(c->emb, out, (size_t)token * (size_t)c->n_embd, (size_t)c->n_embd);
        return 0;
    }
    if (c->stage == ORC_STAGE_LAYERS) return orc_step_layers(c, 0, out);
    to_float(c->out_norm, c->wn, 0, (size_t)c->n_embd);
    rmsnorm(c->xb, out, c->wn, c->n_embd, c->eps);
    mv(c->logits, c->out_w, c->xb, c->n_embd, c->n_vocab);
    memcpy(out, c->xb, sizeof(float) * (size_t)c->n_embd);
    out[c->n_embd] = (float)orc_pick(c);
    return 0;
}
