// ecu_model.cpp -- host GGUF view (v2/v3) for the C ABI.
//
// Follows the reference reader's rules (src/gguf.c:233-336): magic, version
// 2..3, uint64 counts checked against the file size, <= 4096 tensors and
// keys, metadata value types 0..12, <= 4 non-zero dims, tensor byte sizes
// from the block table, data base aligned to general.alignment (default
// 32, accepted in 1..65536), every tensor inside the file.  One deliberate
// difference: a FLOAT64 metadata value is read as 8 bytes (the GGUF
// definition); the reference consumes 16 (src/gguf.c:125), which only
// matters for files it cannot read correctly anyway.
#include "ecu_model.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>

static thread_local std::string t_err;

void ecu_set_error(char *err, size_t errlen, const char *fmt, ...)
{
    char    buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_err = buf;
    if (err && errlen) snprintf(err, errlen, "%s", buf);
}

const char *ecu_get_error() { return t_err.c_str(); }

size_t ecu_type_nbytes(unsigned t, size_t n)
{
    switch (t) {
    case 0: return n * 4;
    case 1: return n * 2;
    case 2: return n / 32 * 18;
    case 3: return n / 32 * 20;
    case 6: return n / 32 * 22;
    case 7: return n / 32 * 24;
    case 8: return n / 32 * 34;
    case 9: return n / 32 * 36;
    case 10: return n / 256 * 84;
    case 11: return n / 256 * 110;
    case 12: return n / 256 * 144;
    case 13: return n / 256 * 176;
    case 14: return n / 256 * 210;
    case 15: return n / 256 * 292;
    case 16: return n / 32 * 2;
    default: return 0;
    }
}

namespace {
struct Reader {
    const uint8_t *base, *p;
    size_t         size;
    bool           bad = false;
    size_t left() const { return size - (size_t)(p - base); }
    uint64_t num(int nb)
    {
        if (bad || left() < (size_t)nb) { bad = true; return 0; }
        uint64_t v = 0;
        for (int i = 0; i < nb; i++) v |= (uint64_t)p[i] << (8 * i);
        p += nb;
        return v;
    }
    bool str(std::string &out)
    {
        uint64_t n = num(8);
        if (bad || n > left()) { bad = true; return false; }
        out.assign((const char *)p, (size_t)n);
        p += n;
        return true;
    }
};

size_t scalar_bytes(unsigned t)
{
    switch (t) {
    case 0: case 1: case 7: return 1;
    case 2: case 3: return 2;
    case 4: case 5: case 6: return 4;
    case 10: case 11: case 12: return 8;
    default: return 0;
    }
}

double scalar_value(Reader &r, unsigned t)
{
    uint64_t v;
    switch (t) {
    case 0: return (double)r.num(1);
    case 1: return (double)(int8_t)r.num(1);
    case 2: return (double)r.num(2);
    case 3: return (double)(int16_t)r.num(2);
    case 4: return (double)r.num(4);
    case 5: return (double)(int32_t)r.num(4);
    case 6: { uint32_t u = (uint32_t)r.num(4); float f; memcpy(&f, &u, 4); return f; }
    case 7: return r.num(1) ? 1.0 : 0.0;
    case 10: return (double)r.num(8);
    case 11: { v = r.num(8); int64_t s; memcpy(&s, &v, 8); return (double)s; }
    case 12: { v = r.num(8); double d; memcpy(&d, &v, 8); return d; }
    default: r.bad = true; return 0;
    }
}
}  // namespace

int ecu_model_parse(ecu_model *m, const void *file, size_t size, char *err, size_t errlen)
{
    Reader r{(const uint8_t *)file, (const uint8_t *)file, size};
    if (size < 24) { ecu_set_error(err, errlen, "file too small for GGUF (%zu bytes)", size); return -1; }
    uint32_t magic = (uint32_t)r.num(4);
    if (magic != 0x46554747u) {
        ecu_set_error(err, errlen, "not GGUF: magic 0x%08X (expected 0x46554747 'GGUF')", magic);
        return -1;
    }
    unsigned version = (unsigned)r.num(4);
    if (version < 2 || version > 3) { ecu_set_error(err, errlen, "GGUF version %u not supported (need 2 or 3)", version); return -1; }
    uint64_t nt = r.num(8), nkv = r.num(8);
    if (r.bad || nt > size || nkv > size) { ecu_set_error(err, errlen, "GGUF: count larger than the file"); return -1; }
    if (nt == 0 || nt > 4096 || nkv > 4096) {
        ecu_set_error(err, errlen, "GGUF: implausible number of tensors (%llu) or keys (%llu)",
                      (unsigned long long)nt, (unsigned long long)nkv);
        return -1;
    }
    m->version = version;
    for (uint64_t i = 0; i < nkv; i++) {
        EcuKv kv;
        if (!r.str(kv.key)) { ecu_set_error(err, errlen, "GGUF: truncated metadata"); return -1; }
        kv.type = (unsigned)r.num(4);
        if (r.bad) { ecu_set_error(err, errlen, "GGUF: truncated metadata"); return -1; }
        if (kv.type > 12) {
            ecu_set_error(err, errlen, "metadata: key \"%s\" has unknown value type %u", kv.key.c_str(), kv.type);
            return -1;
        }
        if (kv.type == 8) {
            if (!r.str(kv.str)) { ecu_set_error(err, errlen, "GGUF: truncated string"); return -1; }
        } else if (kv.type == 9) {
            unsigned at = (unsigned)r.num(4);
            uint64_t an = r.num(8);
            if (r.bad || an > r.left()) { ecu_set_error(err, errlen, "GGUF: array longer than the file"); return -1; }
            if (at == 8) {
                std::string s;
                for (uint64_t k = 0; k < an; k++)
                    if (!r.str(s)) { ecu_set_error(err, errlen, "GGUF: truncated string array"); return -1; }
            } else {
                size_t step = scalar_bytes(at);
                if (!step || an * step > size) { ecu_set_error(err, errlen, "GGUF: bad array in metadata"); return -1; }
                for (uint64_t k = 0; k < an && !r.bad; k++) (void)scalar_value(r, at);
            }
        } else {
            kv.num = scalar_value(r, kv.type);
        }
        if (r.bad) { ecu_set_error(err, errlen, "GGUF: truncated metadata"); return -1; }
        m->kv.push_back(std::move(kv));
    }
    for (uint64_t i = 0; i < nt; i++) {
        EcuTensor t;
        if (!r.str(t.name)) { ecu_set_error(err, errlen, "GGUF: truncated tensor table"); return -1; }
        t.n_dims = (unsigned)r.num(4);
        if (r.bad) { ecu_set_error(err, errlen, "GGUF: truncated tensor table"); return -1; }
        if (t.n_dims > 4) { ecu_set_error(err, errlen, "tensor %s has more than 4 dims", t.name.c_str()); return -1; }
        size_t total = 1;
        for (unsigned d = 0; d < t.n_dims; d++) {
            t.dims[d] = r.num(8);
            if (!r.bad && !t.dims[d]) { ecu_set_error(err, errlen, "tensor %s has a zero dimension", t.name.c_str()); return -1; }
            total *= (size_t)t.dims[d];
        }
        t.type = (unsigned)r.num(4);
        uint64_t off = r.num(8);
        if (r.bad) { ecu_set_error(err, errlen, "GGUF: truncated tensor table"); return -1; }
        t.nbytes = ecu_type_nbytes(t.type, total);
        t.off = off;
        m->t.push_back(std::move(t));
    }
    unsigned align = 32;
    for (auto &kv : m->kv)
        if (kv.key == "general.alignment" && kv.num >= 1 && kv.num <= 65536) align = (unsigned)kv.num;
    size_t base = (size_t)(r.p - r.base);
    base = (base + align - 1) / align * align;
    for (auto &t : m->t) {
        if (t.off > size || base + t.off + t.nbytes > size) {
            ecu_set_error(err, errlen, "tensor %s lies outside the file", t.name.c_str());
            return -1;
        }
        t.data = (const uint8_t *)file + base + t.off;
    }
    m->alignment = align;
    m->index();
    return 0;
}

ecu_model::~ecu_model()
{
    if (map) munmap(map, map_len);
}

void ecu_model::index()
{
    by_name.clear();
    for (size_t i = 0; i < t.size(); i++) by_name.emplace(t[i].name, i);   // first wins
}

const EcuTensor *ecu_model::find(const std::string &name) const
{
    auto it = by_name.find(name);
    return it == by_name.end() ? nullptr : &t[it->second];
}

const EcuKv *ecu_model::kv_find(const std::string &key) const
{
    for (auto &k : kv)
        if (k.key == key) return &k;
    return nullptr;
}

const EcuKv *ecu_model::kv_arch(const char *key, const char *arch) const
{
    const EcuKv *k = nullptr;
    if (arch && *arch) k = kv_find(std::string(arch) + "." + key);
    return k ? k : kv_find(key);
}

int ecu_model::get_u(const char *key, const char *arch, unsigned long *out) const
{
    const EcuKv *k = kv_arch(key, arch);
    if (!k || k->type == 8 || k->type == 9) return -1;
    *out = (unsigned long)k->num;
    return 0;
}

int ecu_model::get_f(const char *key, const char *arch, float *out) const
{
    const EcuKv *k = kv_arch(key, arch);
    if (!k || k->type == 8 || k->type == 9) return -1;
    *out = (float)k->num;
    return 0;
}

const char *ecu_model::get_s(const char *key) const
{
    const EcuKv *k = kv_find(key);
    return (k && k->type == 8) ? k->str.c_str() : nullptr;
}

// Geometry (src/engine.c:55-109 read_shape plus the arch check of
// engine.c:150-159).
int ecu_read_geom(const ecu_model *m, EcuGeom *g, char *err, size_t errlen)
{
    const char *arch = m->get_s("general.architecture");
    if (!arch || !*arch) { ecu_set_error(err, errlen, "model has no general.architecture"); return -1; }
    if (strcmp(arch, "llama") != 0 && strcmp(arch, "qwen2") != 0) {
        ecu_set_error(err, errlen, "architecture \"%s\" is not supported: the engine runs llama (LLaMA, Mistral) and qwen2", arch);
        return -1;
    }
    unsigned long v;
    if (m->get_u("block_count", arch, &v)) { ecu_set_error(err, errlen, "model has no %s.block_count", arch); return -1; }
    g->n_layer = (int)v;
    if (m->get_u("embedding_length", arch, &v)) { ecu_set_error(err, errlen, "model has no %s.embedding_length", arch); return -1; }
    g->n_embd = (int)v;
    if (m->get_u("feed_forward_length", arch, &v)) { ecu_set_error(err, errlen, "model has no %s.feed_forward_length", arch); return -1; }
    g->n_ff = (int)v;
    if (m->get_u("attention.head_count", arch, &v)) { ecu_set_error(err, errlen, "model has no %s.attention.head_count", arch); return -1; }
    g->n_head = (int)v;
    g->n_head_kv = m->get_u("attention.head_count_kv", arch, &v) ? g->n_head : (int)v;
    unsigned long ctx = 512;
    m->get_u("context_length", arch, &ctx);
    g->n_ctx = (int)ctx;
    float eps = 1e-5f;
    if (m->get_f("attention.layer_norm_rms_epsilon", arch, &eps) &&
        m->get_f("attention.layer_norm_epsilon", arch, &eps))
        eps = 1e-5f;
    g->eps = eps;
    float rope = 10000.0f;
    m->get_f("rope.freq_base", arch, &rope);
    g->rope_base = rope > 0 ? rope : 10000.0f;
    if (g->n_head <= 0 || g->n_embd % g->n_head) {
        ecu_set_error(err, errlen, "n_embd %d is not divisible by n_head %d", g->n_embd, g->n_head);
        return -1;
    }
    if (g->n_embd > 32768) {      // the RMSNorm kernels' partial buffers (RMS_MAX_W warps of 128)
        ecu_set_error(err, errlen, "n_embd %d above the supported 32768", g->n_embd);
        return -1;
    }
    g->head_dim = g->n_embd / g->n_head;
    if (g->n_head_kv <= 0 || g->n_head % g->n_head_kv) {
        ecu_set_error(err, errlen, "n_head %d is not divisible by n_head_kv %d", g->n_head, g->n_head_kv);
        return -1;
    }
    g->n_rep = g->n_head / g->n_head_kv;
    unsigned long rd = 0;
    if (m->get_u("rope.dimension_count", arch, &rd) == 0 && rd > 0) g->head_dim = (int)rd;
    const EcuTensor *emb = m->find("token_embd.weight");
    if (emb) {
        if (emb->n_dims != 2) { ecu_set_error(err, errlen, "token_embd.weight: expected 2 dims"); return -1; }
        g->n_vocab = (int)emb->dims[1];
    } else if (m->get_u("vocab_size", arch, &v) == 0) {
        g->n_vocab = (int)v;
    } else {
        g->n_vocab = 0;
    }
    if (g->n_ctx <= 0) g->n_ctx = 512;
    return 0;
}
