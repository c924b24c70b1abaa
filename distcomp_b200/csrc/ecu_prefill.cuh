// ecu_prefill.cuh -- the prompt of a FULL context as one batch per layer.
//
// The reference feeds a prompt token by token (src/shard.c:911-917); every
// projection is then a matrix-vector product.  Here the n prompt tokens of a
// layer go through each projection together, as one GEMM on the tensor
// cores, so every weight is read once per layer instead of n times:
//
//   embed rows -> per layer: RMSNorm -> QKV GEMM -> RoPE + KV append ->
//   causal attention (each token over the cache up to its own position) ->
//   O GEMM + residual -> RMSNorm -> gate/up GEMM -> SwiGLU -> down GEMM +
//   residual;  then the last token through the decode step's head.
//
// Precision: each GEMM operand is split into two fp16 parts, v = hi + lo
// (hi = fp16(v), lo = fp16(v - hi)), and the product is accumulated in fp32
// as hi*hi + hi*lo + lo*hi, which keeps about 22 bits of every factor --
// the error of the fp32 matvec the reference runs, not fp16's.  The
// dequantised weights (exact in fp32: code * fp16 scale) are split once per
// layer into a scratch matrix; the activations are split as they are
// produced.  The GEMM runs on tcgen05 (k_pf_gemm_tc: fp32 accumulators in
// tensor memory); k_pf_gemm, the same product with mma.sync m16n8k16, stays
// as the reference point (ECU_PF_TC=0).  Sums run in another order than the per-token path, so the
// prompt's activations and logits agree with it within the 1e-3 bar, not
// bit for bit.
#pragma once
#include "ecu_attn.cuh"
#include "ecu_common.cuh"
#include "ecu_dequant.cuh"
#include "ecu_gemv.cuh"
#include "ecu_pipe.cuh"

#include <cuda_fp16.h>

// Embedding rows of the n prompt tokens (any type of the raw matrix).
static __global__ void k_pf_embed(DevMat emb, const int *tok, int n, float *X, int E)
{
    const size_t total = (size_t)n * E;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
        const int    t = (int)(e / (size_t)E), i = (int)(e % (size_t)E);
        const size_t a = (size_t)tok[t] * (size_t)E + (size_t)i;
        X[e] = mat_elem(emb, (int)(a / (size_t)emb.n_in), (int)(a % (size_t)emb.n_in));
    }
}

__device__ __forceinline__ void pf_split(float v, __half &hi, __half &lo)
{
    hi = __float2half_rn(v);
    lo = __float2half_rn(__fsub_rn(v, __half2float(hi)));
}

// Row t of X, RMS-normalised with weights w exactly as the decode step does
// (rms_scale's summation order, the same two roundings per element), split
// into fp16 hi/lo.  One CTA (256 threads) per row.
static __global__ void __launch_bounds__(256) k_pf_norm_split(const float *X, const float *w, int E, float eps,
                                                               __half *hi, __half *lo)
{
    __shared__ double dsum[RMS_MAX_W + 1];
    const float *x = X + (size_t)blockIdx.x * E;
    const float  s = rms_scale(x, E, eps, dsum, threadIdx.x, blockDim.x, [] { __syncthreads(); });
    for (int i = threadIdx.x; i < E; i += blockDim.x) {
        const float v = __fmul_rn(__fmul_rn(__ldcg(x + i), s), w[i]);
        pf_split(v, hi[(size_t)blockIdx.x * E + i], lo[(size_t)blockIdx.x * E + i]);
    }
}

static __global__ void k_pf_split(const float *X, size_t count, __half *hi, __half *lo)
{
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < count; e += (size_t)gridDim.x * blockDim.x)
        pf_split(X[e], hi[e], lo[e]);
}

// Q4_0 (SPLIT4), Q8_0 (SPLIT8) or Q4_K (SPLITK4) rows, column segments
// included, dequantised and split, one thread per 32-element block: the
// values mat_elem gives, 64-byte stores.
static __global__ void k_pf_wsplit_fast(DevMat m, __half *hi, __half *lo)
{
    const int    nbt = m.n_in / 32, nb = nbt / m.nseg;     // blocks of a row, of a segment row
    const size_t total = (size_t)m.n_out * nbt;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
        const size_t   row = e / (size_t)nbt;
        const int      bt = (int)(e % (size_t)nbt), b = bt % nb;
        const uint8_t *r = m.data + (size_t)(bt / nb) * m.seg_bytes + row * m.row_bytes;
        float          v[32];
        if (m.layout == LAY_SPLITK4) {
            const uint4 q = *reinterpret_cast<const uint4 *>(r + (size_t)b * 16);
            const uint4 h = *reinterpret_cast<const uint4 *>(r + (size_t)nb * 16 + (size_t)(b >> 3) * 16);
            float dl, ml;
            k4_scale_min(h, b & 7, dl, ml);
            const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const uint32_t byte = (w[j >> 2] >> (8 * (j & 3))) & 0xFFu;
                v[j] = __fsub_rn(__fmul_rn(dl, (float)(byte & 0x0F)), ml);
                v[j + 16] = __fsub_rn(__fmul_rn(dl, (float)(byte >> 4)), ml);
            }
        } else if (m.layout == LAY_SPLIT4) {
            const uint4 q = *reinterpret_cast<const uint4 *>(r + (size_t)b * 16);
            const float d = f16x(r + (size_t)nb * 16 + 2 * b);
            const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const uint32_t byte = (w[j >> 2] >> (8 * (j & 3))) & 0xFFu;
                v[j] = __fmul_rn((float)((int)(byte & 0x0F) - 8), d);
                v[j + 16] = __fmul_rn((float)((int)(byte >> 4) - 8), d);
            }
        } else {
            const uint4 q0 = *reinterpret_cast<const uint4 *>(r + (size_t)b * 16);
            const uint4 q1 = *reinterpret_cast<const uint4 *>(r + (size_t)(nb + b) * 16);
            const float d = f16x(r + (size_t)nb * 32 + 2 * b);
            const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
            for (int j = 0; j < 32; j++) v[j] = __fmul_rn(d, (float)(int8_t)((w[j >> 2] >> (8 * (j & 3))) & 0xFFu));
        }
        __align__(16) __half h[32], l[32];
#pragma unroll
        for (int j = 0; j < 32; j++) pf_split(v[j], h[j], l[j]);
        uint4 *ho = reinterpret_cast<uint4 *>(hi + row * m.n_in + (size_t)bt * 32);
        uint4 *lo4 = reinterpret_cast<uint4 *>(lo + row * m.n_in + (size_t)bt * 32);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            ho[j] = reinterpret_cast<const uint4 *>(h)[j];
            lo4[j] = reinterpret_cast<const uint4 *>(l)[j];
        }
    }
}

// A device weight matrix (any layout) dequantised and split: rows x n_in.
static __global__ void k_pf_wsplit(DevMat m, __half *hi, __half *lo)
{
    const size_t total = (size_t)m.n_out * m.n_in;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x)
        pf_split(mat_elem(m, (int)(e / (size_t)m.n_in), (int)(e % (size_t)m.n_in)), hi[e], lo[e]);
}

// ----------------------------------------------------------------- GEMM ---
// C[M x N] (+)= A[M x K] * B[N x K]^T, A and B each given as fp16 hi/lo row-
// major with K contiguous (K % 8 == 0); C fp32 row-major with stride ldc; R
// (may equal C) added when non-null.  CTA tile 128 x 128, K step 32, two
// cp.async stages; 8 warps as 2 (M) x 4 (N), 64 x 32 each; rows past M or N
// load as zeros and are not stored.
#define PF_BM 128
#define PF_BN 128
#define PF_BK 32
#define PF_LDS 40            // halves per shared row: 80 B, conflict-free ldmatrix
#define PF_TILE (PF_BM * PF_LDS)

__host__ __device__ constexpr size_t pf_gemm_smem() { return (size_t)2 * 4 * PF_TILE * sizeof(__half); }

__device__ __forceinline__ void pf_cp16(void *dst, const void *src, bool ok)
{
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    const int      n = ok ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(n) : "memory");
}

__device__ __forceinline__ void pf_ldm4(unsigned (&r)[4], const __half *p)
{
    const unsigned a = (unsigned)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(a));
}

__device__ __forceinline__ void pf_mma(float (&c)[4], const unsigned (&a)[4], unsigned b0, unsigned b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
                 "{%8, %9}, {%0, %1, %2, %3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

static __global__ void __launch_bounds__(256) k_pf_gemm(const __half *Ahi, const __half *Alo, const __half *Bhi,
                                                         const __half *Blo, float *C, int M, int N, int K, int ldc,
                                                         const float *R)
{
    extern __shared__ __align__(16) __half pf_sm[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.y * PF_BM, n0 = blockIdx.x * PF_BN;
    const int wm = (warp >> 2) * 64, wn = (warp & 3) * 32;
    // stage s, operand o (0 A hi, 1 A lo, 2 B hi, 3 B lo)
    auto tile = [&](int s, int o) { return pf_sm + ((size_t)s * 4 + o) * PF_TILE; };
    const __half *src[4] = {Ahi, Alo, Bhi, Blo};

    auto load = [&](int s, int k0) {
        // 4 tiles of 128 rows x 32 halves = 512 16-byte chunks each
#pragma unroll
        for (int o = 0; o < 4; o++) {
            const int lim = o < 2 ? M : N, base = o < 2 ? m0 : n0;
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const int  ch = tid + j * 256, r = ch >> 2, c = (ch & 3) * 8;
                const bool ok = base + r < lim && k0 + c < K;
                const __half *g = src[o] + (ok ? (size_t)(base + r) * K + k0 + c : 0);
                pf_cp16(tile(s, o) + r * PF_LDS + c, g, ok);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };

    float acc[4][4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int q = 0; q < 4; q++) acc[i][j][q] = 0.0f;

    const int nk = (K + PF_BK - 1) / PF_BK;
    load(0, 0);
    for (int kt = 0; kt < nk; kt++) {
        const int s = kt & 1;
        if (kt + 1 < nk) {
            load(s ^ 1, (kt + 1) * PF_BK);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < PF_BK; kk += 16) {
            unsigned ah[4][4], al[4][4], bh[2][4], bl[2][4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int off = (wm + i * 16 + (lane & 15)) * PF_LDS + kk + (lane >> 4) * 8;
                pf_ldm4(ah[i], tile(s, 0) + off);
                pf_ldm4(al[i], tile(s, 1) + off);
            }
#pragma unroll
            for (int j = 0; j < 2; j++) {
                // matrices: (n 0-7, k 0-7), (n 0-7, k 8-15), (n 8-15, k 0-7), (n 8-15, k 8-15)
                const int off = (wn + j * 16 + (lane & 7) + ((lane >> 4) << 3)) * PF_LDS + kk + ((lane >> 3) & 1) * 8;
                pf_ldm4(bh[j], tile(s, 2) + off);
                pf_ldm4(bl[j], tile(s, 3) + off);
            }
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int jj = j >> 1, h = (j & 1) * 2;
                    pf_mma(acc[i][j], ah[i], bh[jj][h], bh[jj][h + 1]);
                    pf_mma(acc[i][j], ah[i], bl[jj][h], bl[jj][h + 1]);
                    pf_mma(acc[i][j], al[i], bh[jj][h], bh[jj][h + 1]);
                }
        }
        __syncthreads();                  // the stage is refilled next iteration
    }
    // C fragment: c0, c1 at (row g, cols 2t, 2t+1), c2, c3 at row g + 8
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int row = m0 + wm + i * 16 + g + h * 8;
                if (row >= M) continue;
#pragma unroll
                for (int q = 0; q < 2; q++) {
                    const int col = n0 + wn + j * 8 + 2 * t + q;
                    if (col >= N) continue;
                    const size_t e = (size_t)row * ldc + col;
                    const float  v = acc[i][j][h * 2 + q];
                    C[e] = R ? __fadd_rn(R[e], v) : v;
                }
            }
}

// ------------------------------------------------ GEMM on tcgen05 (TMEM) ---
// The same product on the 5th-generation tensor cores: one elected thread
// issues tcgen05.mma (kind::f16, M = 128 tokens, N = 128 weight rows, K = 16
// per instruction) on operands in shared memory, the fp32 accumulator lives
// in tensor memory (128 columns) and is read back with tcgen05.ld for the
// epilogue.  Operand tiles are 128 rows x 64 halves (one 128-byte swizzle
// atom per row: 16-byte chunk c of row r sits at chunk c ^ (r & 7)), loaded
// with cp.async, three stages; tcgen05.commit on a per-stage mbarrier tells
// the loaders when a stage's MMAs have read it.  Same interface and limits
// as k_pf_gemm (K % 8 == 0).
#define PF_TC_BK 64
#define PF_TC_STAGES 3
#define PF_TC_TILE (128 * PF_TC_BK * 2)      // bytes of one operand tile

__host__ __device__ constexpr size_t pf_tc_smem() { return (size_t)PF_TC_STAGES * 4 * PF_TC_TILE + 1024; }

// K-major, 128-byte-swizzled operand: rows 128 B apart, 8-row groups 1024 B
// apart (SBO), leading offset 1 (unused within one swizzle atom), version 1.
__device__ __forceinline__ uint64_t pf_sdesc(uint32_t saddr)
{
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void pf_tc_mma(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc)
{
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
                 :
                 : "r"(tmem), "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
                 : "memory");
}

static __global__ void __launch_bounds__(128, 1) k_pf_gemm_tc(const __half *Ahi, const __half *Alo,
                                                               const __half *Bhi, const __half *Blo, float *C,
                                                               int M, int N, int K, int ldc, const float *R,
                                                               int *status)
{
    extern __shared__ uint8_t pf_tc_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>(((uintptr_t)pf_tc_raw + 1023) & ~(uintptr_t)1023);
    __shared__ __align__(8) uint64_t mbar[PF_TC_STAGES];
    __shared__ uint32_t tmem_s;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.y * 128, n0 = blockIdx.x * 128;
    auto tile = [&](int s, int o) { return sm + ((size_t)s * 4 + o) * PF_TC_TILE; };
    const __half *src[4] = {Ahi, Alo, Bhi, Blo};

    if (warp == 0) {
        const uint32_t dst = (uint32_t)__cvta_generic_to_shared(&tmem_s);
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 128;" ::"r"(dst) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int s = 0; s < PF_TC_STAGES; s++) mbar_init(&mbar[s], 1);
        mbar_init_fence();
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_s;

    auto load = [&](int s, int k0) {
        // 4 tiles x 128 rows x 8 chunks of 16 bytes
        for (int q = tid; q < 4 * 128 * 8; q += 128) {
            const int  o = q >> 10, r = (q >> 3) & 127, c = q & 7;
            const int  lim = o < 2 ? M : N, row = (o < 2 ? m0 : n0) + r;
            const bool ok = row < lim && k0 + c * 8 < K;
            const __half *g = src[o] + (ok ? (size_t)row * K + k0 + c * 8 : 0);
            pf_cp16(tile(s, o) + r * 128 + ((c ^ (r & 7)) << 4), g, ok);
        }
    };
    const int nk = (K + PF_TC_BK - 1) / PF_TC_BK;
    // instruction descriptor: fp32 accumulate, fp16 A and B, both K-major,
    // N = 128 (>> 3), M = 128 (>> 4)
    const uint32_t idesc = (1u << 4) | ((128u >> 3) << 17) | ((128u >> 4) << 24);
    for (int s = 0; s < PF_TC_STAGES - 1; s++) {
        if (s < nk) load(s, s * PF_TC_BK);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    // ok: every wait so far succeeded (the same value in every thread: it is
    // combined by the loop's barrier).  A wait that gives up stops the
    // pipeline: no further stage loads (the stage may still be an operand of
    // MMAs in flight), no further MMAs and no C stores; the MMAs already
    // committed are drained below before the accumulator is freed.
    bool ok = true;
    int  last_commit = -1;
    for (int kt = 0; kt < nk; kt++) {
        const int s = kt % PF_TC_STAGES, nxt = kt + PF_TC_STAGES - 1;
        bool mine = true;
        if (nxt < nk) {
            // the stage nxt reuses was read by iteration kt - 1's MMAs
            if (kt >= 1)
                mine = mbar_wait<true>(&mbar[(kt - 1) % PF_TC_STAGES], (unsigned)((kt - 1) / PF_TC_STAGES) & 1u,
                                       status);
            if (mine) load(nxt % PF_TC_STAGES, nxt * PF_TC_BK);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_group %0;" ::"n"(PF_TC_STAGES - 1) : "memory");
        // this thread's copies into stage s are done: hand them to the
        // tensor core's (async) proxy, then to the issuing thread
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        ok = __syncthreads_and(mine) != 0;
        if (!ok) break;
        last_commit = kt;
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t a_hi = (uint32_t)__cvta_generic_to_shared(tile(s, 0));
            const uint32_t a_lo = (uint32_t)__cvta_generic_to_shared(tile(s, 1));
            const uint32_t b_hi = (uint32_t)__cvta_generic_to_shared(tile(s, 2));
            const uint32_t b_lo = (uint32_t)__cvta_generic_to_shared(tile(s, 3));
#pragma unroll
            for (int k = 0; k < PF_TC_BK / 16; k++) {
                // K = 16 halves = 32 bytes further along the swizzle atom
                const uint32_t off = (uint32_t)k * 32;
                pf_tc_mma(tmem, pf_sdesc(a_hi + off), pf_sdesc(b_hi + off), idesc, (kt | k) ? 1u : 0u);
                pf_tc_mma(tmem, pf_sdesc(a_hi + off), pf_sdesc(b_lo + off), idesc, 1u);
                pf_tc_mma(tmem, pf_sdesc(a_lo + off), pf_sdesc(b_hi + off), idesc, 1u);
            }
            const uint32_t bar = (uint32_t)__cvta_generic_to_shared(&mbar[s]);
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                         : "memory");
        }
        __syncwarp();
    }
    // the last commit covers every MMA issued before it; drained whatever the
    // status word says (bounded), so that no MMA is in flight when the
    // accumulator is read or freed
    asm volatile("cp.async.wait_all;" ::: "memory");
    if (last_commit >= 0) {
        const bool done = mbar_drain(&mbar[last_commit % PF_TC_STAGES],
                                     (unsigned)(last_commit / PF_TC_STAGES) & 1u, wait_limit_ns());
        if (!done && status) atomicOr(status, ECU_STATUS_TIMEOUT);
        ok = __syncthreads_and(ok && done) != 0;
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    // warp w reads accumulator lanes 32w..32w+31 (tile rows), 32 columns at a time
    const int row = m0 + warp * 32 + lane;
    for (int ch = 0; ch < 4 && ok; ch++) {
        uint32_t v[32];
        const uint32_t ta = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(ch * 32);
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
                     "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
                     "%30, %31}, [%32];"
                     : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                       "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
                       "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]),
                       "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]),
                       "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
                     : "r"(ta)
                     : "memory");
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (row < M) {
#pragma unroll
            for (int j = 0; j < 32; j++) {
                const int col = n0 + ch * 32 + j;
                if (col < N) {
                    const size_t e = (size_t)row * ldc + col;
                    const float  x = __uint_as_float(v[j]);
                    C[e] = R ? __fadd_rn(R[e], x) : x;
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 128;" ::"r"(tmem) : "memory");
}

// --------------------------------------------------------- RoPE, KV, attn --
// Row t of QKV (q | k | v of one token): biases, RoPE of q and k at position
// pos0 + t (src/engine.c:367-378), q rotated in place, k and v appended to
// this layer's cache planes [n_kv][n_ctx][hd].
static __global__ void k_pf_rope_kv(float *QKV, int ld, int n_head, int n_kv, int hd, int pos0, const float *cs,
                                    const float *bq, const float *bk, const float *bv, float *kc, float *vc, int n_ctx)
{
    const int t = blockIdx.x, pos = pos0 + t, half = hd / 2;
    float    *q = QKV + (size_t)t * ld, *k = q + (size_t)n_head * hd, *v = k + (size_t)n_kv * hd;
    const float *c = cs + (size_t)pos * hd;
    for (int i = threadIdx.x; i < n_head * half; i += blockDim.x) {
        const int h = i / half, j = i % half;
        float     x0 = q[h * hd + j], x1 = q[h * hd + j + half];
        if (bq) { x0 = __fadd_rn(x0, bq[h * hd + j]); x1 = __fadd_rn(x1, bq[h * hd + j + half]); }
        rope_pair(x0, x1, c[2 * j], c[2 * j + 1]);
        q[h * hd + j] = x0;
        q[h * hd + j + half] = x1;
    }
    for (int i = threadIdx.x; i < n_kv * half; i += blockDim.x) {
        const int g = i / half, j = i % half;
        float     k0 = k[g * hd + j], k1 = k[g * hd + j + half];
        float     v0 = v[g * hd + j], v1 = v[g * hd + j + half];
        if (bk) { k0 = __fadd_rn(k0, bk[g * hd + j]); k1 = __fadd_rn(k1, bk[g * hd + j + half]); }
        if (bv) { v0 = __fadd_rn(v0, bv[g * hd + j]); v1 = __fadd_rn(v1, bv[g * hd + j + half]); }
        rope_pair(k0, k1, c[2 * j], c[2 * j + 1]);
        float *kr = kc + ((size_t)g * n_ctx + pos) * hd, *vr = vc + ((size_t)g * n_ctx + pos) * hd;
        kr[j] = k0;
        kr[j + half] = k1;
        vr[j] = v0;
        vr[j + half] = v1;
    }
}

// Attention of token t, query head h (one CTA of HD threads): scores over
// cache positions 0..pos0+t in shared memory, exact max, expf, weights
// divided by their sum once, out = sum of weighted V rows.
#define PF_ATT_MAXPOS 8192
template <int HD>
static __global__ void __launch_bounds__(HD) k_pf_attn(const float *QKV, int ld, int n_head, int n_rep, int pos0,
                                                        const float *kc, const float *vc, int n_ctx, float kscale,
                                                        float *att)
{
    __shared__ float sc[PF_ATT_MAXPOS];
    __shared__ __align__(16) float qs[HD];
    __shared__ float red[HD / 32];
    const int t = blockIdx.y, h = blockIdx.x, g = h / n_rep, np = pos0 + t + 1;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    qs[tid] = QKV[(size_t)t * ld + (size_t)h * HD + tid];
    __syncthreads();
    const float *kb = kc + (size_t)g * n_ctx * HD, *vb = vc + (size_t)g * n_ctx * HD;
    // scores: warp w takes positions w, w + HD/32, ...; lanes over dims
    for (int p = warp; p < np; p += HD / 32) {
        const float *kr = kb + (size_t)p * HD;
        float        d = 0.0f;
        for (int j = lane; j < HD; j += 32) d = fmaf(qs[j], kr[j], d);
        d = warp_sum(d);
        if (lane == 0) sc[p] = d * kscale;
    }
    __syncthreads();
    float m = -INFINITY;
    for (int p = tid; p < np; p += HD) m = fmaxf(m, sc[p]);
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = red[0];
    for (int w = 1; w < HD / 32; w++) m = fmaxf(m, red[w]);
    __syncthreads();
    float l = 0.0f;
    for (int p = tid; p < np; p += HD) {
        const float e = expf(sc[p] - m);
        sc[p] = e;
        l += e;
    }
    l = warp_sum(l);
    if (lane == 0) red[warp] = l;
    __syncthreads();
    l = 0.0f;
    for (int w = 0; w < HD / 32; w++) l += red[w];
    float o = 0.0f;                               // dim tid
    for (int p = 0; p < np; p++) o = fmaf(sc[p], vb[(size_t)p * HD + tid], o);
    att[(size_t)t * n_head * HD + (size_t)h * HD + tid] = o / l;
}

// The same attention tiled over tokens: a CTA (256 threads) takes KV head g
// and 64 / n_rep consecutive tokens, i.e. 64 query vectors (query qi = token
// qi / n_rep, head g*n_rep + qi % n_rep), and walks the cache 32 positions
// at a time through shared memory, so every K/V row is read once per 64
// queries instead of once per query.  Thread tid serves the query pair
// 2*(tid/8), 2*(tid/8)+1: its 4 scores per query of a chunk (positions
// tid % 8 + 8j), a running max and sum per query shared by the pair's 8
// threads, and the HD/8 contiguous output dims of eighth tid % 8 for both
// queries, so every K and V float4 read from shared memory feeds two
// queries.  Q and K rows are padded to HD + 4 floats, V rows carry 4 floats
// of padding after every eighth: the rows (eighths) a warp reads start in
// distinct bank quads.  K/V rows arrive by cp.async (one buffer: two CTAs
// of this kernel share an SM, each one's copies overlap the other's
// arithmetic).  Softmax as k_pf_attn: scores * kscale, expf against the
// running max, one division by the sum at the end.
#define PF_QB 64
#define PF_KC 32
template <int HD>
struct PfAttnGeom {
    static constexpr int QS = HD + 4;                 // Q / K row stride (floats)
    static constexpr int DE = HD / 8;                 // output dims of an eighth
    static constexpr int VE = DE + 4;                 // V eighth stride
    static constexpr int VS = 8 * VE;                 // V row stride
};

template <int HD>
__host__ __device__ constexpr size_t pf_attn2_smem()
{
    return ((size_t)PF_QB * PfAttnGeom<HD>::QS + (size_t)PF_KC * PfAttnGeom<HD>::QS +
            (size_t)PF_KC * PfAttnGeom<HD>::VS + (size_t)PF_QB * (PF_KC + 1)) *
           sizeof(float);
}

template <int HD>
static __global__ void __launch_bounds__(256) k_pf_attn2(const float *QKV, int ld, int n, int n_head, int n_rep,
                                                          int pos0, const float *kc, const float *vc, int n_ctx,
                                                          float kscale, float *att)
{
    using Gm = PfAttnGeom<HD>;
    constexpr int QS = Gm::QS, DE = Gm::DE, VE = Gm::VE, VS = Gm::VS, C4 = HD / 4, NP = PF_KC / 8;
    static_assert(DE % 4 == 0, "head_dim a multiple of 32");
    extern __shared__ __align__(16) float pf_att_sm[];
    float *QSm = pf_att_sm;                         // [64][QS]
    float *KSm = QSm + PF_QB * QS;                  // [32][QS]
    float *VSm = KSm + PF_KC * QS;                  // [32][VS]
    float *PS = VSm + PF_KC * VS;                   // [64][33]
    const int tid = threadIdx.x, g = blockIdx.x, tb = PF_QB / n_rep, t0 = blockIdx.y * tb;
    const int qa = 2 * (tid >> 3), qb = qa + 1, sub = tid & 7;
    const int ta = t0 + qa / n_rep, ha = g * n_rep + qa % n_rep;
    const int tq = t0 + qb / n_rep, hb = g * n_rep + qb % n_rep;
    const bool va = ta < n, vbq = tq < n;
    for (int i = tid; i < PF_QB * HD; i += 256) {
        const int q = i / HD, d = i % HD, tt = t0 + q / n_rep, hq = g * n_rep + q % n_rep;
        QSm[q * QS + d] = tt < n ? QKV[(size_t)tt * ld + (size_t)hq * HD + d] : 0.0f;
    }
    const int   last = pos0 + min(n, t0 + tb) - 1;      // last key position any query sees
    const int   pa = pos0 + ta, pb = pos0 + tq;          // the queries' own positions
    const float *kb = kc + (size_t)g * n_ctx * HD, *vb = vc + (size_t)g * n_ctx * HD;
    float ma = -INFINITY, la = 0.0f, mb = -INFINITY, lb = 0.0f, oa[DE], ob[DE];
#pragma unroll
    for (int j = 0; j < DE; j++) oa[j] = ob[j] = 0.0f;
    const float4 *qa4 = reinterpret_cast<const float4 *>(QSm + qa * QS);
    const float4 *qb4 = reinterpret_cast<const float4 *>(QSm + qb * QS);
    // K and V rows of the chunk at c: 16-byte pieces, zero past the last
    // position any query sees
    auto load = [&](int c) {
        float *K = KSm, *V = VSm;
        for (int i = tid; i < PF_KC * C4; i += 256) {
            const int  p = i / C4, d = 4 * (i % C4), kp = c + p;
            const bool ok = kp <= last;
            const size_t src = ok ? (size_t)kp * HD + d : 0;
            pf_cp16(K + p * QS + d, kb + src, ok);
            pf_cp16(V + p * VS + (d / DE) * VE + d % DE, vb + src, ok);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    for (int c0 = 0; c0 <= last; c0 += PF_KC) {
        __syncthreads();                                 // Q stored / previous chunk consumed
        load(c0);
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncthreads();
        float sa[NP], sb[NP];
#pragma unroll
        for (int j = 0; j < NP; j++) sa[j] = sb[j] = 0.0f;
#pragma unroll 4
        for (int c = 0; c < C4; c++) {
            const float4 x = qa4[c], y = qb4[c];
#pragma unroll
            for (int j = 0; j < NP; j++) {
                const float4 kv = reinterpret_cast<const float4 *>(KSm + (sub + 8 * j) * QS)[c];
                sa[j] = fmaf(x.x, kv.x, fmaf(x.y, kv.y, fmaf(x.z, kv.z, fmaf(x.w, kv.w, sa[j]))));
                sb[j] = fmaf(y.x, kv.x, fmaf(y.y, kv.y, fmaf(y.z, kv.z, fmaf(y.w, kv.w, sb[j]))));
            }
        }
        float cma = -INFINITY, cmb = -INFINITY;
#pragma unroll
        for (int j = 0; j < NP; j++) {
            const int kp = c0 + sub + 8 * j;
            sa[j] = (va && kp <= pa) ? sa[j] * kscale : -INFINITY;
            sb[j] = (vbq && kp <= pb) ? sb[j] * kscale : -INFINITY;
            cma = fmaxf(cma, sa[j]);
            cmb = fmaxf(cmb, sb[j]);
        }
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            cma = fmaxf(cma, __shfl_xor_sync(0xffffffffu, cma, o));
            cmb = fmaxf(cmb, __shfl_xor_sync(0xffffffffu, cmb, o));
        }
        const float mna = fmaxf(ma, cma), mnb = fmaxf(mb, cmb);
        const float fa = mna == -INFINITY ? 1.0f : expf(ma - mna);
        const float fb = mnb == -INFINITY ? 1.0f : expf(mb - mnb);
        float lsa = 0.0f, lsb = 0.0f;
#pragma unroll
        for (int j = 0; j < NP; j++) {
            const float ea = sa[j] == -INFINITY ? 0.0f : expf(sa[j] - mna);
            const float eb = sb[j] == -INFINITY ? 0.0f : expf(sb[j] - mnb);
            PS[qa * (PF_KC + 1) + sub + 8 * j] = ea;
            PS[qb * (PF_KC + 1) + sub + 8 * j] = eb;
            lsa += ea;
            lsb += eb;
        }
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            lsa += __shfl_xor_sync(0xffffffffu, lsa, o);
            lsb += __shfl_xor_sync(0xffffffffu, lsb, o);
        }
        la = la * fa + lsa;
        lb = lb * fb + lsb;
        ma = mna;
        mb = mnb;
        __syncwarp();
#pragma unroll
        for (int j = 0; j < DE; j++) {
            oa[j] *= fa;
            ob[j] *= fb;
        }
        for (int p = 0; p < PF_KC; p++) {
            const float   ea = PS[qa * (PF_KC + 1) + p], eb = PS[qb * (PF_KC + 1) + p];
            const float4 *vr = reinterpret_cast<const float4 *>(VSm + p * VS + sub * VE);
#pragma unroll
            for (int c = 0; c < DE / 4; c++) {
                const float4 v = vr[c];
                oa[4 * c] = fmaf(ea, v.x, oa[4 * c]);
                oa[4 * c + 1] = fmaf(ea, v.y, oa[4 * c + 1]);
                oa[4 * c + 2] = fmaf(ea, v.z, oa[4 * c + 2]);
                oa[4 * c + 3] = fmaf(ea, v.w, oa[4 * c + 3]);
                ob[4 * c] = fmaf(eb, v.x, ob[4 * c]);
                ob[4 * c + 1] = fmaf(eb, v.y, ob[4 * c + 1]);
                ob[4 * c + 2] = fmaf(eb, v.z, ob[4 * c + 2]);
                ob[4 * c + 3] = fmaf(eb, v.w, ob[4 * c + 3]);
            }
        }
    }
    if (va) {
        float4 *dst = reinterpret_cast<float4 *>(att + (size_t)ta * n_head * HD + (size_t)ha * HD + sub * DE);
#pragma unroll
        for (int c = 0; c < DE / 4; c++)
            dst[c] = make_float4(oa[4 * c] / la, oa[4 * c + 1] / la, oa[4 * c + 2] / la, oa[4 * c + 3] / la);
    }
    if (vbq) {
        float4 *dst = reinterpret_cast<float4 *>(att + (size_t)tq * n_head * HD + (size_t)hb * HD + sub * DE);
#pragma unroll
        for (int c = 0; c < DE / 4; c++)
            dst[c] = make_float4(ob[4 * c] / lb, ob[4 * c + 1] / lb, ob[4 * c + 2] / lb, ob[4 * c + 3] / lb);
    }
}

// h[t][j] = silu(gate) * up from the interleaved gate/up rows (2j, 2j+1).
static __global__ void k_pf_swiglu(const float *GU, size_t n_rows, int ff, float *H)
{
    const size_t total = n_rows * (size_t)ff;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
        const size_t t = e / (size_t)ff, j = e % (size_t)ff;
        H[e] = silu_mul(GU[t * 2 * ff + 2 * j], GU[t * 2 * ff + 2 * j + 1]);
    }
}
