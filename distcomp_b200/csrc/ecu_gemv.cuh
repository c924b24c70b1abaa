// ecu_gemv.cuh -- fused dequant + GEMV kernels (batch-1 decode).
//
// y[o] = sum_i W[i + o*n_in] * x[i] over GGUF-quantised W (the quantised
// matvec of src/engine.c:287-357), with the neighbours of each matvec in the
// reference's layer loop fused in:
//   prologue  RMSNorm of x (src/engine.c:256-262), recomputed per CTA
//   epilogues y = acc | y += acc (residual, engine.c:453,465) |
//             SwiGLU on interleaved gate/up rows (engine.c:458-463) |
//             logits + argmax (engine.c:491-496, 517-526)
//
// Two paths:
//  * k_gemv_fast: Q4_0 / Q8_0 in the SPLIT layouts with n_in a multiple of
//    1024.  One CTA per SM streams its contiguous run of rows through a
//    4-stage shared-memory ring filled by bulk async copies (one producer
//    thread, mbarriers), so each SM keeps ~70 KB of weights in flight.  The
//    input vector is held in registers as three exact int8 "digit planes"
//    per 32-element block (x = s*(d0 + d1/128 + d2/16384), s a power of 2),
//    so one 4-bit or 8-bit code block costs 24 dp4a instead of 32 int->float
//    conversions and FMAs.  Each lane owns one block column; warps split the
//    row's 32-block groups and their partial sums meet in shared memory.
//  * k_gemv_generic: any supported format/layout, one warp per row, with
//    the bit-exact per-element decoder; used for F32/F16, K-quants, and
//    shapes the fast path does not take.
#pragma once
#include "ecu_dequant.cuh"
#include "ecu_pipe.cuh"

enum Epi : int { EPI_STORE = 0, EPI_ADD = 1, EPI_SWIGLU = 2, EPI_ARGMAX = 3 };

// Inputs of a GEMV launch (both paths).
struct GemvArgs {
    DevMat       m;
    const float *x;            // input vector, n_in floats
    const float *norm_w;       // RMSNorm weights (n_in) when the prologue is on
    float        eps;
    float       *y;            // output (STORE/ADD/ARGMAX: n_out; SWIGLU: n_out/2)
    float       *xn_out;       // optional: CTA 0 stores the normed input here
    float       *xn_dst;       // argmax: the last CTA copies xn_out here (n_in floats) once every
                               // CTA has read x (the normed state may replace x in place)
    // argmax epilogue
    float       *part_val;     // [gridDim.x]
    int         *part_idx;     // [gridDim.x]
    unsigned    *counter;      // zero between launches
    StepState   *st;           // token <- argmax; pos advanced if advance_pos
    int         *tok_hist;     // tok_hist[pos] <- argmax (nullable)
    float       *tok_out;      // *tok_out <- (float)argmax (nullable)
    int          advance_pos;
    int         *status;
    // fast-path geometry (set by the host planner)
    int          rows_per_cta;
    int          stage_rows;
    // L2 prefetch of the next GEMV's weights: CTA i warms
    // [pf_ptr + i*pf_stride, + pf_bytes), clipped to pf_end
    const uint8_t *pf_ptr;
    const uint8_t *pf_end;
    size_t       pf_stride;
    uint32_t     pf_bytes;
};

// ---------------------------------------------------------------- RMSNorm --
// 1/sqrt(mean(x^2)+eps) with the sum of squares in double (src/engine.c:258-
// 260).  The double sum has one fixed order, whatever the block size, so
// every kernel that normalises a vector gets the same bits:
//
//   P[q] = ((x[4q]^2 + x[4q+1]^2) + x[4q+2]^2) + x[4q+3]^2  (elements >= n: 0)
//          for q < Q = ceil(n/4) rounded up to a multiple of 32;
//   W[w] = bfly32(P[32w .. 32w+31]),  w < nW = Q/32;
//   L[l] = ((0 + W[l]) + W[l+32]) + ...  (l < 32);     sum = bfly32(L[0..31]),
//
// bfly32 being the xor butterfly v_l += v_{l^o} for o = 16, 8, 4, 2, 1 (every
// lane ends with the same bits: each pair adds the same two values).  A warp
// computes a W from 32 consecutive float4s held one per lane, so a kernel
// that holds its input in registers needs no shared-memory pass before it.
// nW <= 256 (n <= 32768; the model loader enforces it).
#define RMS_MAX_W 256

__device__ __forceinline__ double rms_sq4(float4 v)
{
    double p = (double)v.x * (double)v.x;
    p += (double)v.y * (double)v.y;
    p += (double)v.z * (double)v.z;
    p += (double)v.w * (double)v.w;
    return p;
}

__device__ __forceinline__ double rms_bfly32(double v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Number of W terms for an n-element vector.
__device__ __forceinline__ int rms_nw(int n) { return ((n + 3) / 4 + 31) / 32; }

// sum = bfly32 of the per-lane sequential sums of W[0..nW) (one warp).
__device__ __forceinline__ double rms_total_w(const double *W, int nW, int lane)
{
    double l = 0.0;
    for (int w = lane; w < nW; w += 32) l += W[w];
    return rms_bfly32(l);
}

__device__ __forceinline__ float rms_from_sum(double ss, int n, float eps)
{
    const float ms = (float)(ss / (double)n);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
}

// The scale of x[0..n) by threads [0, nthreads) (a multiple of 32), which
// must all call it; `bar` synchronises them.  dsum: RMS_MAX_W + 1 doubles.
// x is read through L2 (ld.global.cg).
template <class Bar>
__device__ float rms_scale(const float *x, int n, float eps, double *dsum, int tid, int nthreads, Bar bar)
{
    const int nW = rms_nw(n), lane = tid & 31, warp = tid >> 5, nwarps = nthreads >> 5;
    for (int w = warp; w < nW; w += nwarps) {
        const int q = 32 * w + lane;
        double p = 0.0;
        if ((n & 3) == 0) {
            if (4 * q < n) p = rms_sq4(__ldcg(reinterpret_cast<const float4 *>(x) + q));
        } else {
            for (int i = 4 * q; i < min(n, 4 * q + 4); i++) {
                const double e = (double)__ldcg(x + i);
                p = i == 4 * q ? e * e : p + e * e;
            }
        }
        p = rms_bfly32(p);
        if (lane == 0) dsum[w] = p;
    }
    bar();
    if (warp == 0) {
        const double t = rms_total_w(dsum, nW, lane);
        if (lane == 0) dsum[RMS_MAX_W] = t;
    }
    bar();
    return rms_from_sum(dsum[RMS_MAX_W], n, eps);
}

// ----------------------------------------------------------- argmax tail --
// First maximum in index order, NaN never selected, and the reference's
// fallback to 0 when logits[0] is NaN or nothing beats -inf
// (src/engine.c:517-526 scans with a strict >).
struct ArgBest {
    float v;
    int   i;
};

__device__ __forceinline__ ArgBest arg_better(ArgBest a, ArgBest b)
{
    if (b.i >= 0 && (b.v > a.v || (b.v == a.v && (a.i < 0 || b.i < a.i)))) return b;
    return a;
}

// Block-wide argmax of (v, i) pairs; every thread of the block calls it.
static __device__ ArgBest block_argmax(ArgBest mine, ArgBest *sh)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ArgBest other;
        other.v = __shfl_xor_sync(0xffffffffu, mine.v, o);
        other.i = __shfl_xor_sync(0xffffffffu, mine.i, o);
        mine = arg_better(mine, other);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) sh[warp] = mine;
    __syncthreads();
    if (threadIdx.x == 0) {
        ArgBest b = sh[0];
        for (int w = 1; w < nw; w++) b = arg_better(b, sh[w]);
        sh[0] = b;
    }
    __syncthreads();
    return sh[0];
}

// Per-CTA partial -> last CTA reduces all partials in CTA order and publishes.
static __device__ void argmax_finish(const GemvArgs &a, ArgBest cta_best, ArgBest *sh)
{
    __shared__ unsigned s_last;
    if (threadIdx.x == 0) {
        a.part_val[blockIdx.x] = cta_best.v;
        a.part_idx[blockIdx.x] = cta_best.i;
        __threadfence();
        unsigned t = atomicAdd(a.counter, 1u);
        s_last = (t == gridDim.x - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (a.xn_out && a.xn_dst)
        for (int i = threadIdx.x; i < a.m.n_in; i += blockDim.x) a.xn_dst[i] = __ldcg(a.xn_out + i);
    if (threadIdx.x == 0) {
        ArgBest b{-INFINITY, -1};
        for (unsigned c = 0; c < gridDim.x; c++) {
            ArgBest p{((volatile float *)a.part_val)[c], ((volatile int *)a.part_idx)[c]};
            b = arg_better(b, p);
        }
        const float l0 = ((volatile float *)a.y)[0];
        const int   tok = (b.i < 0 || isnan(l0)) ? 0 : b.i;
        if (a.st) {
            if (a.tok_hist) a.tok_hist[a.st->pos] = tok;
            a.st->token = tok;
            if (a.advance_pos) a.st->pos = a.st->pos + 1;
        }
        if (a.tok_out) *a.tok_out = (float)tok;
        *a.counter = 0u;
    }
}

__device__ __forceinline__ float silu_mul(float g, float u)
{
    // (g / (1 + expf(-g))) * u with IEEE division, as src/engine.c:462
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

// ============================================================ generic =====

// Warp per output row; lanes stride the row's elements / blocks.
template <int EPI>
__global__ void __launch_bounds__(256) k_gemv_generic(GemvArgs a)
{
    pdl_wait();
    pdl_trigger();
    const DevMat &m = a.m;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    __shared__ ArgBest sh[32];
    ArgBest best{-INFINITY, -1};
    for (int row = warp; row < m.n_out; row += nwarps) {
        float acc = 0.0f;
        if (!m.zero) {
            const uint8_t *r = m.data + (size_t)row * m.row_bytes;
            if (m.type == GT_F32) {
                const float *w = reinterpret_cast<const float *>(r);
                for (int k = lane; k < m.n_in; k += 32) acc = fmaf(w[k], a.x[k], acc);
            } else if (m.type == GT_F16) {
                for (int k = lane; k < m.n_in; k += 32) acc = fmaf(f16x(r + 2 * k), a.x[k], acc);
            } else {
                const int be = blk_elems(m.type), bb = blk_bytes(m.type), nb = m.n_in / be;
                for (int b = lane; b < nb; b += 32) {
                    const uint8_t *blk = r + (size_t)b * bb;
                    const float   *xs = a.x + (size_t)b * be;
                    float part = 0.0f;
                    for (int i = 0; i < be; i++) part = fmaf(dq_elem(m.type, blk, i), xs[i], part);
                    acc += part;
                }
            }
            acc = warp_sum(acc);
        }
        if (lane == 0) {
            if (EPI == EPI_ADD) a.y[row] = a.y[row] + acc;
            else a.y[row] = acc;
        }
        if (EPI == EPI_ARGMAX && lane == 0) best = arg_better(best, ArgBest{acc, row});
    }
    if (EPI == EPI_ARGMAX) {
        ArgBest b = block_argmax(best, sh);
        argmax_finish(a, b, sh);
    }
}

// Standalone RMSNorm (generic path and HEAD's normed-state output):
// out[i] = x[i] * scale * w[i], single CTA.
static __global__ void __launch_bounds__(256) k_rmsnorm(const float *x, const float *w, int n,
                                                 float eps, float *out)
{
    pdl_wait();
    pdl_trigger();
    __shared__ double dsum[RMS_MAX_W + 1];
    const float s = rms_scale(x, n, eps, dsum, threadIdx.x, blockDim.x, [] { __syncthreads(); });
    for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = __fmul_rn(__fmul_rn(x[i], s), w[i]);
}

// h[j] = silu(g[j]) * u[j] for the unfused gate/up path.
static __global__ void k_swiglu(const float *g, const float *u, float *h, int n)
{
    pdl_wait();
    pdl_trigger();
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x)
        h[j] = silu_mul(g[j], u[j]);
}

// =============================================================== fast =====

#define FAST_STAGES 4
#define FAST_MAX_THREADS 640    // nkg * rowpar <= 19 consumer warps + 1 producer
#define FAST_MAX_NKG 19         // n_in <= 19 * 1024 on the fast path
#define FAST_RB 4               // rows per consumer-warp batch

// 1.5 * 2^23: for |v| <= 2^22, v + M rounds v to the nearest integer (ties to
// even) and that integer, two's complement, sits in the low bits of the sum.
#define RND_MAGIC 12582912.0f

// Low bytes of four words -> one word [a.b0, b.b0, c.b0, d.b0].
__device__ __forceinline__ uint32_t pack_lo_bytes(uint32_t a, uint32_t b, uint32_t c, uint32_t d)
{
    return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// Exact three-plane int8 decomposition of one 32-element block of x:
// x = s * (d0 + d1/128 + d2/16384) + r, s = 2^k, |r| <= s / 32768, each
// digit in [-127, 127] (d0) or [-64, 64] (d1, d2).  No float->int
// conversions: each digit is the low byte of v + RND_MAGIC.
// FMT 4: word j<4 packs elements 4j..4j+3 (low nibbles of Q4_0 code word j),
//        word 4+j packs 16+4j..16+4j+3 (its high nibbles).
// FMT 8: word j packs elements 4j..4j+3.
// FMT 12 (Q4_K in SPLITK4 rows): FMT 4's order.
// off[p] = -8 * (sum of plane p's digits) for Q4_0 (the code offset), the
// plain sum for Q4_K (the sub-block minimum multiplies it), else 0.
template <int FMT>
__device__ __forceinline__ void make_digits(const float *xv, int (&xw)[3][8], int (&off)[3],
                                            float &sxs)
{
    float amax = 0.0f;
    bool  nan = false;
#pragma unroll
    for (int k = 0; k < 32; k++) {
        amax = fmaxf(amax, fabsf(xv[k]));
        nan |= xv[k] != xv[k];
    }
    int   e = 0;
    float inv = 0.0f;
    if (nan || !(amax < INFINITY)) {
        sxs = __int_as_float(0x7fc00000);   // inf/NaN in x: let the row come out NaN
    } else if (amax > 1e-30f) {
        frexpf(amax, &e);                   // amax < 2^e
        if (amax >= ldexpf(127.5f, e - 7)) e += 1;
        inv = ldexpf(1.0f, 7 - e);          // |x * inv| <= 127.5: d0 fits int8
        sxs = ldexpf(1.0f, e - 7 - 14);
    } else {
        sxs = 0.0f;                         // all-zero (or negligible) block
    }
    int sum[3] = {0, 0, 0};
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int base = (FMT == 4 || FMT == 12) ? ((j < 4) ? 4 * j : 16 + 4 * (j - 4)) : 4 * j;
        uint32_t b[3][4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float v  = __fmul_rn(xv[base + i], inv);            // exact
            const float t0 = __fadd_rn(v, RND_MAGIC);
            const float r0 = __fmul_rn(__fsub_rn(v, __fsub_rn(t0, RND_MAGIC)), 128.0f);
            const float t1 = __fadd_rn(r0, RND_MAGIC);
            const float r1 = __fmul_rn(__fsub_rn(r0, __fsub_rn(t1, RND_MAGIC)), 128.0f);
            const float t2 = __fadd_rn(r1, RND_MAGIC);
            b[0][i] = __float_as_uint(t0);
            b[1][i] = __float_as_uint(t1);
            b[2][i] = __float_as_uint(t2);
        }
#pragma unroll
        for (int p = 0; p < 3; p++) {
            xw[p][j] = (int)pack_lo_bytes(b[p][0], b[p][1], b[p][2], b[p][3]);
            sum[p] = __dp4a(xw[p][j], 0x01010101, sum[p]);
        }
    }
#pragma unroll
    for (int p = 0; p < 3; p++) off[p] = (FMT == 4) ? -8 * sum[p] : (FMT == 12) ? sum[p] : 0;
}

// Sub-block j (0..7) of a Q4_K super-block from its 16-byte header h (d,
// dmin, scales[12] as four little-endian words): dl = d*sc and ml = dmin*m,
// the reference's two products (gguf.c:558-590).  Byte k of the scales is
// s[k]; with jj = j & 3 the pair needs s[jj], s[4+jj] and s[8+jj] only.
// Sub-blocks 4-7 take their low 4 bits from s[8+jj] and the top 2 from bits
// 6-7 of s[jj] / s[4+jj]: with lane-constant shift and masks both cases are
// sc = ((A >> sA) & mA) | (C & mC), m = ((B >> sA) & mA) | ((C >> 4) & mC).
__device__ __forceinline__ void k4_scale_min(uint4 h, int j, float &dl, float &ml)
{
    const int      sh = 8 * (j & 3);
    const bool     up = j >= 4;
    const uint32_t sA = up ? 2u : 0u, mA = up ? 0x30u : 0x3Fu, mC = up ? 0x0Fu : 0u;
    const uint32_t A = (h.y >> sh) & 0xFFu, B = (h.z >> sh) & 0xFFu, C = (h.w >> sh) & 0xFFu;
    const uint32_t sc = ((A >> sA) & mA) | (C & mC);
    const uint32_t mn = ((B >> sA) & mA) | ((C >> 4) & mC);
    const float    d = __half2float(__ushort_as_half((unsigned short)(h.x & 0xFFFFu)));
    const float    dmin = __half2float(__ushort_as_half((unsigned short)(h.x >> 16)));
    dl = __fmul_rn(d, (float)sc);
    ml = __fmul_rn(dmin, (float)mn);
}

// One Q4_K sub-block's dot from its merged digit sums: t = sum of code*digit,
// sx = sum of digits (both x 2^14, 2^7, 1 per plane): dl*t - ml*sx, scaled.
__device__ __forceinline__ float k4_finish(int t, int sx, float dl, float ml, float sxs)
{
    return fmaf(dl, (float)t, -(ml * (float)sx)) * sxs;
}

// Dot of the lane's block in `row` (shared memory) with its digit planes.
template <int FMT>
__device__ __forceinline__ float block_dot(const uint8_t *row, int nb, int b,
                                           const int (&xw)[3][8], const int (&off)[3], float sxs)
{
    if (FMT == 4) {
        const uint4 q = *reinterpret_cast<const uint4 *>(row + (size_t)b * 16);
        const float d = __half2float(*reinterpret_cast<const __half *>(row + (size_t)nb * 16 + 2 * b));
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
        int a0 = off[0], a1 = off[1], a2 = off[2];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int lo = (int)(w[j] & 0x0F0F0F0Fu), hi = (int)((w[j] >> 4) & 0x0F0F0F0Fu);
            a0 = __dp4a(lo, xw[0][j], a0);
            a0 = __dp4a(hi, xw[0][4 + j], a0);
            a1 = __dp4a(lo, xw[1][j], a1);
            a1 = __dp4a(hi, xw[1][4 + j], a1);
            a2 = __dp4a(lo, xw[2][j], a2);
            a2 = __dp4a(hi, xw[2][4 + j], a2);
        }
        // |a0| <= 32*8*127, |a1|,|a2| <= 32*8*64: the merged value fits int32
        const int t = a0 * 16384 + a1 * 128 + a2;
        return (float)t * (d * sxs);
    } else if (FMT == 12) {
        // codes 0..15: |a0| <= 32*15*127, the merged value still fits int32
        const uint4 q = *reinterpret_cast<const uint4 *>(row + (size_t)b * 16);
        const uint4 h = *reinterpret_cast<const uint4 *>(row + (size_t)nb * 16 + (size_t)(b >> 3) * 16);
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
        int a0 = 0, a1 = 0, a2 = 0;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int lo = (int)(w[j] & 0x0F0F0F0Fu), hi = (int)((w[j] >> 4) & 0x0F0F0F0Fu);
            a0 = __dp4a(lo, xw[0][j], a0);
            a0 = __dp4a(hi, xw[0][4 + j], a0);
            a1 = __dp4a(lo, xw[1][j], a1);
            a1 = __dp4a(hi, xw[1][4 + j], a1);
            a2 = __dp4a(lo, xw[2][j], a2);
            a2 = __dp4a(hi, xw[2][4 + j], a2);
        }
        float dl, ml;
        k4_scale_min(h, b & 7, dl, ml);
        return k4_finish(a0 * 16384 + a1 * 128 + a2, off[0] * 16384 + off[1] * 128 + off[2], dl, ml, sxs);
    } else {
        // SPLIT8 rows keep the first and second 16 code bytes of every block
        // in two separate runs, so both 16-byte loads are conflict-free
        const uint4 q0 = *reinterpret_cast<const uint4 *>(row + (size_t)b * 16);
        const uint4 q1 = *reinterpret_cast<const uint4 *>(row + (size_t)(nb + b) * 16);
        const float d = __half2float(*reinterpret_cast<const __half *>(row + (size_t)nb * 32 + 2 * b));
        const int w[8] = {(int)q0.x, (int)q0.y, (int)q0.z, (int)q0.w,
                          (int)q1.x, (int)q1.y, (int)q1.z, (int)q1.w};
        int a0 = 0, a1 = 0, a2 = 0;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            a0 = __dp4a(w[j], xw[0][j], a0);
            a1 = __dp4a(w[j], xw[1][j], a1);
            a2 = __dp4a(w[j], xw[2][j], a2);
        }
        const float t = fmaf((float)a1, 128.0f, (float)a2);
        return fmaf((float)a0, 16384.0f, t) * (d * sxs);
    }
}

// Four per-lane row partials -> four row sums: afterwards lane l holds the
// sum of row (l >> 3) & 3 (a transposed butterfly: 6 shuffles for 4 rows).
__device__ __forceinline__ float warp_sum4(float v0, float v1, float v2, float v3, int lane)
{
    const bool up = lane & 16;
    float a0 = up ? v2 : v0, a1 = up ? v3 : v1;
    const float b0 = up ? v0 : v2, b1 = up ? v1 : v3;
    a0 += __shfl_xor_sync(0xffffffffu, b0, 16);
    a1 += __shfl_xor_sync(0xffffffffu, b1, 16);
    const bool mid = lane & 8;
    float c = mid ? a1 : a0;
    const float dd = mid ? a0 : a1;
    c += __shfl_xor_sync(0xffffffffu, dd, 8);
    c += __shfl_xor_sync(0xffffffffu, c, 4);
    c += __shfl_xor_sync(0xffffffffu, c, 2);
    c += __shfl_xor_sync(0xffffffffu, c, 1);
    return c;
}

// Shared-memory plan of one fast launch (host and device agree on it).
struct FastSmem {
    size_t stage_bytes, ring, bars, red, dig, dsum, argsh, total;
};

__host__ __device__ inline FastSmem fast_smem_plan(size_t row_bytes, int stage_rows,
                                                   int rows_per_cta, int nkg, int rowpar)
{
    FastSmem p;
    p.stage_bytes = ((size_t)stage_rows * row_bytes + 127) & ~(size_t)127;
    p.ring = 0;
    p.bars = p.ring + FAST_STAGES * p.stage_bytes;
    p.red = p.bars + 2 * FAST_STAGES * sizeof(uint64_t);
    p.dig = (p.red + (size_t)rows_per_cta * nkg * sizeof(float) + 15) & ~(size_t)15;
    // digit planes shared by the rowpar warps of a k-group: 28 words per block
    const size_t dig_bytes = rowpar > 1 ? (size_t)nkg * 32 * 28 * sizeof(int) : 0;
    p.dsum = p.dig + dig_bytes;
    p.argsh = p.dsum + (RMS_MAX_W + 2) * sizeof(double);
    p.total = p.argsh + 32 * sizeof(ArgBest);
    return p;
}

// L2 prefetch (no shared memory, no completion to wait for).
__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes)
{
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// blockDim = 32 * (nkg * rowpar + 1): consumer warps first, producer last.
// Consumer warp w serves k-group g = w % nkg (32 blocks = 1024 inputs of
// every row) and takes the stage's rows rp, rp + rowpar, ... (rp = w / nkg)
// four at a time.
template <int FMT, bool NORM, int EPI>
__global__ void __launch_bounds__(FAST_MAX_THREADS, 1) k_gemv_fast(GemvArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    const DevMat &m = a.m;
    const int nb = m.n_in / 32, nkg = nb / 32;
    const int nw = blockDim.x >> 5, ncw = nw - 1, rowpar = ncw / nkg;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = blockIdx.x * a.rows_per_cta;
    const int nrows = max(0, min(m.n_out, r0 + a.rows_per_cta) - r0);
    const int SR = a.stage_rows;
    const int nstages = (nrows + SR - 1) / SR;
    const FastSmem P = fast_smem_plan(m.row_bytes, SR, a.rows_per_cta, nkg, rowpar);
    uint8_t  *ring = smem + P.ring;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + P.bars);
    uint64_t *empty = full + FAST_STAGES;
    float    *red = reinterpret_cast<float *>(smem + P.red);
    int      *dig = reinterpret_cast<int *>(smem + P.dig);
    double   *dsum = reinterpret_cast<double *>(smem + P.dsum);
    ArgBest  *argsh = reinterpret_cast<ArgBest *>(smem + P.argsh);

    if (threadIdx.x == 0) {
        for (int s = 0; s < FAST_STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], ncw);
        }
        mbar_init_fence();
    }
    __syncthreads();

    if (warp == ncw) {
        // ---- producer: stream this CTA's rows through the ring ----------
        if (lane == 0) {
            const uint8_t *src = m.data + (size_t)r0 * m.row_bytes;
            for (int s = 0; s < nstages; s++) {
                const int slot = s % FAST_STAGES;
                if (s >= FAST_STAGES &&
                    !mbar_wait(&empty[slot], ((s / FAST_STAGES) - 1) & 1, a.status))
                    break;
                const int      rows = min(SR, nrows - s * SR);
                const uint32_t bytes = (uint32_t)(rows * m.row_bytes);
                mbar_expect_tx(&full[slot], bytes);
                bulk_g2s(ring + (size_t)slot * P.stage_bytes, src + (size_t)s * SR * m.row_bytes,
                         bytes, &full[slot]);
                if (s == FAST_STAGES - 1 || s == nstages - 1) pdl_trigger();
            }
            if (nstages == 0) pdl_trigger();
            // warm L2 with the start of the next GEMV's weights
            if (a.pf_ptr && a.pf_bytes) {
                const uint8_t *p = a.pf_ptr + (size_t)blockIdx.x * a.pf_stride;
                for (uint32_t o = 0; o < a.pf_bytes && p + o < a.pf_end; o += 32768) {
                    const uint32_t sz =
                        (uint32_t)min((size_t)min(32768u, a.pf_bytes - o), (size_t)(a.pf_end - (p + o))) & ~15u;
                    if (sz >= 16) prefetch_l2(p + o, sz);
                }
            }
        }
        pdl_wait();                       // before this warp joins the epilogue writes
    } else {
        // ---- consumers ---------------------------------------------------
        const int nct = ncw * 32, ctid = threadIdx.x;
        const int g = warp % nkg, rp = warp / nkg;
        pdl_wait();                       // x comes from the previous kernel
        // RMSNorm: the digit planes are those of x * w; the scale (one fp32
        // factor for the whole vector) multiplies each row's sum in the
        // epilogue, the order the persistent step uses (it knows the scale
        // only once every input block has arrived)
        float scale = 1.0f;
        if (NORM)
            scale = rms_scale(a.x, m.n_in, a.eps, dsum, ctid, nct, [nct] { named_bar(1, nct); });
        const int b = g * 32 + lane;      // this lane's block column
        int   xw[3][8], off[3];
        float sxs;
        if (rp == 0) {
            float xv[32];
            const float4 *x4 = reinterpret_cast<const float4 *>(a.x + (size_t)b * 32);
#pragma unroll
            for (int k = 0; k < 8; k++) {
                float4 t = x4[k];
                xv[4 * k] = t.x; xv[4 * k + 1] = t.y; xv[4 * k + 2] = t.z; xv[4 * k + 3] = t.w;
            }
            if (NORM) {
                const float4 *w4 = reinterpret_cast<const float4 *>(a.norm_w + (size_t)b * 32);
                float4 *o4 = (a.xn_out && blockIdx.x == 0) ? reinterpret_cast<float4 *>(a.xn_out + (size_t)b * 32)
                                                            : nullptr;
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    float4 t = w4[k];
                    // the normed input the stage outputs: (x * scale) * w, the
                    // reference's rounding (src/engine.c:261)
                    if (o4)
                        o4[k] = make_float4(__fmul_rn(__fmul_rn(xv[4 * k], scale), t.x),
                                            __fmul_rn(__fmul_rn(xv[4 * k + 1], scale), t.y),
                                            __fmul_rn(__fmul_rn(xv[4 * k + 2], scale), t.z),
                                            __fmul_rn(__fmul_rn(xv[4 * k + 3], scale), t.w));
                    xv[4 * k]     = __fmul_rn(xv[4 * k], t.x);
                    xv[4 * k + 1] = __fmul_rn(xv[4 * k + 1], t.y);
                    xv[4 * k + 2] = __fmul_rn(xv[4 * k + 2], t.z);
                    xv[4 * k + 3] = __fmul_rn(xv[4 * k + 3], t.w);
                }
            }
            make_digits<FMT>(xv, xw, off, sxs);
            if (rowpar > 1) {
                int4 *d4 = reinterpret_cast<int4 *>(dig + (size_t)b * 28);
#pragma unroll
                for (int p = 0; p < 3; p++) {
                    d4[2 * p] = make_int4(xw[p][0], xw[p][1], xw[p][2], xw[p][3]);
                    d4[2 * p + 1] = make_int4(xw[p][4], xw[p][5], xw[p][6], xw[p][7]);
                }
                d4[6] = make_int4(off[0], off[1], off[2], __float_as_int(sxs));
            }
        }
        if (rowpar > 1) {
            named_bar(1, nct);
            if (rp != 0) {
                const int4 *d4 = reinterpret_cast<const int4 *>(dig + (size_t)b * 28);
#pragma unroll
                for (int p = 0; p < 3; p++) {
                    const int4 u = d4[2 * p], v = d4[2 * p + 1];
                    xw[p][0] = u.x; xw[p][1] = u.y; xw[p][2] = u.z; xw[p][3] = u.w;
                    xw[p][4] = v.x; xw[p][5] = v.y; xw[p][6] = v.z; xw[p][7] = v.w;
                }
                const int4 t = d4[6];
                off[0] = t.x; off[1] = t.y; off[2] = t.z;
                sxs = __int_as_float(t.w);
            }
        }
        for (int s = 0; s < nstages; s++) {
            const int slot = s % FAST_STAGES;
            if (!mbar_wait(&full[slot], (s / FAST_STAGES) & 1, a.status)) break;
            const uint8_t *stage = ring + (size_t)slot * P.stage_bytes;
            const int      rows = min(SR, nrows - s * SR);
            for (int i0 = rp; i0 < rows; i0 += FAST_RB * rowpar) {
                float v[FAST_RB];
#pragma unroll
                for (int k = 0; k < FAST_RB; k++) {
                    const int i = i0 + k * rowpar;
                    v[k] = i < rows ? block_dot<FMT>(stage + (size_t)i * m.row_bytes, nb, b, xw, off, sxs)
                                    : 0.0f;
                }
                const float sum = warp_sum4(v[0], v[1], v[2], v[3], lane);
                const int   k = (lane >> 3) & 3, i = i0 + k * rowpar;
                if ((lane & 7) == 0 && i < rows) red[(s * SR + i) * nkg + g] = sum;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
    }
    __syncthreads();

    // ---- epilogue ----------------------------------------------------------
    const int nthr = blockDim.x;
    ArgBest   best{-INFINITY, -1};
    // the RMSNorm scale (written by rms_scale before the barrier above)
    const float rscale = NORM ? rms_from_sum(dsum[RMS_MAX_W], m.n_in, a.eps) : 1.0f;
    if (EPI == EPI_SWIGLU) {
        for (int j = threadIdx.x; j < nrows / 2; j += nthr) {
            float gsum = 0.0f, usum = 0.0f;
            for (int q = 0; q < nkg; q++) {
                gsum += red[(2 * j) * nkg + q];
                usum += red[(2 * j + 1) * nkg + q];
            }
            if (NORM) {
                gsum = __fmul_rn(gsum, rscale);
                usum = __fmul_rn(usum, rscale);
            }
            a.y[r0 / 2 + j] = silu_mul(gsum, usum);
        }
    } else {
        for (int r = threadIdx.x; r < nrows; r += nthr) {
            float acc = 0.0f;
            for (int q = 0; q < nkg; q++) acc += red[r * nkg + q];
            if (NORM) acc = __fmul_rn(acc, rscale);
            if (EPI == EPI_ADD) a.y[r0 + r] = a.y[r0 + r] + acc;
            else a.y[r0 + r] = acc;
            if (EPI == EPI_ARGMAX) best = arg_better(best, ArgBest{acc, r0 + r});
        }
    }
    if (EPI == EPI_ARGMAX) {
        ArgBest bb = block_argmax(best, argsh);
        argmax_finish(a, bb, argsh);
    }
}
