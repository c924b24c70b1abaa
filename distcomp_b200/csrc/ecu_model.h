// ecu_model.h -- host-side GGUF view shared by the engine translation units.
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

struct EcuKv {
    std::string key;
    unsigned    type = 0;      // GGUF metadata value type
    double      num = 0;
    std::string str;
};

struct EcuTensor {
    std::string    name;
    unsigned       n_dims = 0;
    uint64_t       dims[4] = {1, 1, 1, 1};
    unsigned       type = 0;   // ggml type
    uint64_t       off = 0;
    size_t         nbytes = 0;
    const uint8_t *data = nullptr;   // borrowed (caller's buffer)
    size_t elems() const
    {
        size_t n = 1;
        for (unsigned i = 0; i < n_dims; i++) n *= (size_t)dims[i];
        return n;
    }
};

struct ecu_model {
    std::vector<EcuKv>     kv;
    std::vector<EcuTensor> t;
    unsigned               version = 3, alignment = 32;
    std::unordered_map<std::string, size_t> by_name;
    void                  *map = nullptr;   // ecu_model_open_file: the read-only file mapping the tensors borrow
    size_t                 map_len = 0;
    ~ecu_model();

    void             index();
    const EcuTensor *find(const std::string &name) const;
    const EcuKv     *kv_find(const std::string &key) const;
    const EcuKv     *kv_arch(const char *key, const char *arch) const;
    int              get_u(const char *key, const char *arch, unsigned long *out) const;
    int              get_f(const char *key, const char *arch, float *out) const;
    const char      *get_s(const char *key) const;
};

// Model geometry as the reference derives it (src/engine.c:55-109).
struct EcuGeom {
    int   n_layer = 0, n_embd = 0, n_head = 0, n_head_kv = 0, n_ff = 0, head_dim = 0;
    int   n_vocab = 0, n_rep = 0, n_ctx = 0;
    float eps = 1e-5f, rope_base = 10000.0f;
};

int         ecu_model_parse(ecu_model *m, const void *file, size_t size, char *err, size_t errlen);
int         ecu_read_geom(const ecu_model *m, EcuGeom *g, char *err, size_t errlen);
size_t      ecu_type_nbytes(unsigned t, size_t n);
void        ecu_set_error(char *err, size_t errlen, const char *fmt, ...);
const char *ecu_get_error();
