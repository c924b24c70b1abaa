// ecu_misc.cuh -- small kernels: embedding row, dequant materialisation,
// weight repack, step bookkeeping.
#pragma once
#include "ecu_dequant.cuh"

// out[i] = element token*n + i of the embedding tensor (src/engine.c:472-484:
// row_to_float(t, out, token*ne, ne)).  The token comes from device state so
// that a graph replay picks up the argmax of the previous step.
static __global__ void k_embed(DevMat emb, StepState *st, float *out, int n)
{
    pdl_wait();
    pdl_trigger();
    // the token may come from device memory (another stage's argmax, a
    // receive): one outside the vocabulary flags the step instead of reading
    // past the table
    const int tok = st->token;
    if (tok < 0 || tok >= emb.n_out) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(&st->status, ECU_STATUS_BADTOKEN);
        return;
    }
    const size_t base = (size_t)tok * (size_t)n;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const size_t a = base + (size_t)i;
        out[i] = mat_elem(emb, (int)(a / (size_t)emb.n_in), (int)(a % (size_t)emb.n_in));
    }
}

// dst[e] = element off+e of a raw GGUF block stream of type t (bit-exact).
static __global__ void k_dequant_raw(int t, const uint8_t *raw, size_t off, size_t n, float *dst)
{
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += stride) {
        const size_t a = off + e;
        float v;
        if (t == GT_F32) {
            v = reinterpret_cast<const float *>(raw)[a];
        } else if (t == GT_F16) {
            v = f16x(raw + 2 * a);
        } else {
            const size_t be = (size_t)blk_elems(t);
            v = dq_elem(t, raw + (a / be) * (size_t)blk_bytes(t), (int)(a % be));
        }
        dst[e] = v;
    }
}

// dst[e] = element off+e of a device matrix, read back through its layout;
// `row_map` lets fused matrices expose one source tensor: source row r lives
// at device row row0 + r*rstride.
static __global__ void k_dequant_mat(DevMat m, int row0, int rstride, int n_in, size_t off, size_t n,
                              float *dst)
{
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += stride) {
        const size_t a = off + e;
        const int    r = (int)(a / (size_t)n_in), k = (int)(a % (size_t)n_in);
        dst[e] = mat_elem(m, row0 + r * rstride, k);
    }
}

// Q4_0 rows (18-byte blocks) -> SPLIT4 rows.  Source row r goes to device
// row row0 + r*rstride.  One thread per block.
static __global__ void k_repack_q4_0(const uint8_t *src, int nb, int n_rows, uint8_t *dst,
                              size_t dst_row_bytes, int row0, int rstride)
{
    const size_t total = (size_t)nb * n_rows;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const size_t   r = i / nb, b = i % nb;
        const uint8_t *s = src + i * 18;
        uint8_t       *d = dst + (size_t)(row0 + r * rstride) * dst_row_bytes;
        for (int k = 0; k < 16; k++) d[b * 16 + k] = s[2 + k];
        d[(size_t)nb * 16 + 2 * b] = s[0];
        d[(size_t)nb * 16 + 2 * b + 1] = s[1];
    }
}

// Q8_0 rows (34-byte blocks) -> SPLIT8 rows.
static __global__ void k_repack_q8_0(const uint8_t *src, int nb, int n_rows, uint8_t *dst,
                              size_t dst_row_bytes, int row0, int rstride)
{
    const size_t total = (size_t)nb * n_rows;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const size_t   r = i / nb, b = i % nb;
        const uint8_t *s = src + i * 34;
        uint8_t       *d = dst + (size_t)(row0 + r * rstride) * dst_row_bytes;
        for (int k = 0; k < 16; k++) {
            d[b * 16 + k] = s[2 + k];
            d[((size_t)nb + b) * 16 + k] = s[18 + k];
        }
        d[(size_t)nb * 32 + 2 * b] = s[0];
        d[(size_t)nb * 32 + 2 * b + 1] = s[1];
    }
}

// Q4_K rows (144-byte super-blocks) -> SPLITK4 rows.  Chunk c of a
// super-block (code bytes 32c..32c+31) holds sub-block 2c in its low nibbles
// and 2c+1 in its high ones (gguf.c:569-589); out byte t of sub-block 2c+h is
// nibble h of code bytes t and t+16.  One thread per super-block.
static __global__ void k_repack_q4_k(const uint8_t *src, int nsb, int n_rows, uint8_t *dst,
                                     size_t dst_row_bytes, int row0, int rstride)
{
    const size_t total = (size_t)nsb * n_rows;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const size_t   r = i / nsb, b = i % nsb;
        const uint8_t *s = src + i * 144;
        uint8_t       *d = dst + (size_t)(row0 + r * rstride) * dst_row_bytes;
        for (int c = 0; c < 4; c++)
            for (int t = 0; t < 16; t++) {
                const uint8_t lo = s[16 + 32 * c + t], hi = s[16 + 32 * c + 16 + t];
                d[(b * 8 + 2 * c) * 16 + t] = (uint8_t)((lo & 0x0F) | (hi << 4));
                d[(b * 8 + 2 * c + 1) * 16 + t] = (uint8_t)((lo >> 4) | (hi & 0xF0));
            }
        uint8_t *h = d + (size_t)nsb * 128 + b * 16;
        for (int k = 0; k < 16; k++) h[k] = s[k];
    }
}

// Raw rows copied to device row row0 + r*rstride (formats kept as is).
static __global__ void k_copy_rows(const uint8_t *src, size_t src_row_bytes, int n_rows, uint8_t *dst,
                            size_t dst_row_bytes, int row0, int rstride)
{
    const size_t total = src_row_bytes * (size_t)n_rows;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / src_row_bytes, c = i % src_row_bytes;
        dst[(size_t)(row0 + r * rstride) * dst_row_bytes + c] = src[i];
    }
}

// LAYERS-only stages advance the position at the end of a step.
static __global__ void k_step_advance(StepState *st)
{
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x == 0 && blockIdx.x == 0) st->pos = st->pos + 1;
}
