// ecu_dequant.cuh -- bit-exact per-element block decoders.
//
// Each decoder returns element i of one GGUF block and performs the same
// floating-point operations, in the same order and with the same separate
// roundings, as the reference's block dequant (src/gguf.c:464-720); the
// __fmul_rn/__fadd_rn/__fsub_rn intrinsics keep nvcc from contracting a
// product and a sum into one FMA, which would round differently.
#pragma once
#include "ecu_common.cuh"

// IEEE binary16 bits -> binary32, exact for every input including NaN
// payloads (src/gguf.c:464-486 rd_f16 gives the same bits).
__device__ __forceinline__ float f16_exact(uint32_t h)
{
    uint32_t sign = (h >> 15) & 1u, e = (h >> 10) & 0x1Fu, man = h & 0x3FFu, bits;
    if (e == 0x1F) {
        bits = (sign << 31) | 0x7F800000u | (man << 13);
    } else if (e != 0) {
        bits = (sign << 31) | ((e + 112u) << 23) | (man << 13);
    } else if (man == 0) {
        bits = sign << 31;
    } else {
        int lz = __clz(man) - 21;          // shifts to bring bit 10 up: man < 0x400
        man = (man << lz) & 0x3FFu;
        bits = (sign << 31) | ((uint32_t)(113 - lz) << 23) | (man << 13);
    }
    return __uint_as_float(bits);
}

__device__ __forceinline__ float f16x(const uint8_t *p)
{
    return f16_exact((uint32_t)p[0] | ((uint32_t)p[1] << 8));
}

// 6-bit scale / min pair j of a K-quant block (src/gguf.c:558-567).
__device__ __forceinline__ void kq_scale_min(int j, const uint8_t *s, int &sc, int &mn)
{
    if (j < 4) {
        sc = s[j] & 63;
        mn = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

// Element i of a block of type t starting at b.
__device__ __forceinline__ float dq_elem(int t, const uint8_t *b, int i)
{
    switch (t) {
    case GT_Q4_0: {                                           // gguf.c:662-671
        int j = i & 15;
        int q = i < 16 ? (b[2 + j] & 0x0F) : (b[2 + j] >> 4);
        return __fmul_rn((float)(q - 8), f16x(b));
    }
    case GT_Q4_1: {                                           // gguf.c:673-682
        int j = i & 15;
        int q = i < 16 ? (b[4 + j] & 0x0F) : (b[4 + j] >> 4);
        return __fadd_rn(__fmul_rn((float)q, f16x(b)), f16x(b + 2));
    }
    case GT_Q5_0: {                                           // gguf.c:684-697
        int      j = i & 15;
        uint32_t hb = ld_u32_bytes(b + 2);
        int q = i < 16 ? ((b[6 + j] & 0x0F) | (int)(((hb >> j) & 1u) << 4))
                       : ((b[6 + j] >> 4) | (int)(((hb >> (j + 16)) & 1u) << 4));
        return __fmul_rn((float)(q - 16), f16x(b));
    }
    case GT_Q5_1: {                                           // gguf.c:699-712
        int      j = i & 15;
        uint32_t hb = ld_u32_bytes(b + 4);
        int q = i < 16 ? ((b[8 + j] & 0x0F) | (int)(((hb >> j) & 1u) << 4))
                       : ((b[8 + j] >> 4) | (int)(((hb >> (j + 16)) & 1u) << 4));
        return __fadd_rn(__fmul_rn((float)q, f16x(b)), f16x(b + 2));
    }
    case GT_Q8_0:                                             // gguf.c:714-720
        return __fmul_rn(f16x(b), (float)(int8_t)b[2 + i]);
    case GT_Q2_K: {                                           // gguf.c:497-510
        int g = i >> 4, k = i & 15;
        const uint8_t *q = b + 16 + (g >> 3) * 32 + (g & 1) * 16;
        int   sh = 2 * ((g >> 1) & 3);
        float dl = __fmul_rn(f16x(b + 80), (float)(b[g] & 0x0F));
        float ml = __fmul_rn(f16x(b + 82), (float)(b[g] >> 4));
        return __fsub_rn(__fmul_rn(dl, (float)((q[k] >> sh) & 3)), ml);
    }
    case GT_Q3_K: {                                           // gguf.c:527-554
        int j = i >> 4, l = i & 15;
        const uint8_t *sc = b + 96;
        int   s6 = ((sc[j & 7] >> (4 * (j >> 3))) & 0x0F) |
                   (((sc[8 + (j & 3)] >> (2 * (j >> 2))) & 0x03) << 4);
        float dl = __fmul_rn(f16x(b + 108), (float)(s6 - 32));
        const uint8_t *q = b + 32 + (j >> 3) * 32 + (j & 1) * 16;
        const uint8_t *h = b + (j & 1) * 16;
        int low2 = (q[l] >> (2 * ((j >> 1) & 3))) & 3;
        int neg4 = (((h[l] >> (j >> 1)) & 1) ^ 1) << 2;
        return __fmul_rn(dl, (float)(low2 - neg4));
    }
    case GT_Q4_K: {                                           // gguf.c:569-589
        int c = i >> 6, r = i & 63, hi = r >> 5, l = r & 31;
        int sc, mn;
        kq_scale_min(2 * c + hi, b + 4, sc, mn);
        float dd = __fmul_rn(f16x(b), (float)sc), mm = __fmul_rn(f16x(b + 2), (float)mn);
        int   q = hi ? (b[16 + 32 * c + l] >> 4) : (b[16 + 32 * c + l] & 0x0F);
        return __fsub_rn(__fmul_rn(dd, (float)q), mm);
    }
    case GT_Q5_K: {   // gguf.c:592-615 (the reference's qh reading, kept as is)
        int c = i >> 6, r = i & 63, hi = r >> 5, l = r & 31;
        int sc, mn;
        kq_scale_min(2 * c + hi, b + 4, sc, mn);
        float dd = __fmul_rn(f16x(b), (float)sc), mm = __fmul_rn(f16x(b + 2), (float)mn);
        uint8_t qs = b[48 + 32 * c + l], qh = b[16 + l];
        int v = hi ? (int)((qs >> 4) | (((qh >> 2) & 3) << 4)) - 16
                   : (int)((qs & 0x0F) | ((qh & 3) << 4)) - 16;
        return __fsub_rn(__fmul_rn(dd, (float)v), mm);
    }
    case GT_Q6_K: {                                           // gguf.c:631-647
        int r = i >> 5, col = i & 31;
        int lo = (b[(r >> 2) * 64 + (r & 1) * 32 + col] >> (4 * ((r >> 1) & 1))) & 0x0F;
        int hi = (b[128 + (r >> 2) * 32 + col] >> (2 * (r & 3))) & 0x03;
        float ds = __fmul_rn(f16x(b + 208), (float)(int8_t)b[192 + (i >> 4)]);
        return __fmul_rn(ds, (float)((lo | (hi << 4)) - 32));
    }
    case GT_Q8_K:                                             // gguf.c:650-659
        return __fmul_rn(f16x(b + 256 + 2 * (i >> 3)), (float)(int8_t)b[i]);
    default:
        return 0.0f;
    }
}

// Element (row, k) of a device matrix in any layout.
__device__ __forceinline__ float mat_elem(const DevMat &m, int row, int k)
{
    const uint8_t *r = m.data + (size_t)row * m.row_bytes;
    int n_in = m.n_in;
    if (m.nseg > 1) {                                // column segment of k
        n_in /= m.nseg;
        r += (size_t)(k / n_in) * m.seg_bytes;
        k %= n_in;
    }
    if (m.type == GT_F32) return reinterpret_cast<const float *>(r)[k];
    if (m.type == GT_F16) return f16x(r + 2 * (size_t)k);
    if (m.layout == LAY_SPLITK4) {                   // Q4_K sub-block codes | headers
        const int      nb = n_in / 32, sb = k / 32, i = k % 32;
        const uint8_t *q = r + (size_t)sb * 16, *h = r + (size_t)nb * 16 + (size_t)(sb >> 3) * 16;
        const int      qq = i < 16 ? (q[i] & 0x0F) : (q[i - 16] >> 4);
        int sc, mn;
        kq_scale_min(sb & 7, h + 4, sc, mn);         // gguf.c:569-589 arithmetic
        const float dd = __fmul_rn(f16x(h), (float)sc), mm = __fmul_rn(f16x(h + 2), (float)mn);
        return __fsub_rn(__fmul_rn(dd, (float)qq), mm);
    }
    const int be = blk_elems(m.type), bi = k / be, i = k % be;
    if (m.layout == LAY_SPLIT4) {                    // Q4_0 codes | scales
        const int nb = n_in / 32;
        const uint8_t *q = r + (size_t)bi * 16;
        int qq = i < 16 ? (q[i] & 0x0F) : (q[i - 16] >> 4);
        return __fmul_rn((float)(qq - 8), f16x(r + (size_t)nb * 16 + 2 * bi));
    }
    if (m.layout == LAY_SPLIT8) {    // Q8_0 codes 0..15 | codes 16..31 | scales
        const int nb = n_in / 32;
        const uint8_t c = i < 16 ? r[(size_t)bi * 16 + i] : r[(size_t)(nb + bi) * 16 + i - 16];
        return __fmul_rn(f16x(r + (size_t)nb * 32 + 2 * bi), (float)(int8_t)c);
    }
    return dq_elem(m.type, r + (size_t)bi * blk_bytes(m.type), i);
}
