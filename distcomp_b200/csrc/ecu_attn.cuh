// ecu_attn.cuh -- decode attention with the Q/K/V bias, NeoX RoPE and the
// KV-cache append of the current position fused in (src/engine.c:392-450).
//
// Grid (n_head_kv, n_split).  CTA (g, s) owns KV head g and a contiguous
// slice of positions [0, pos].  Its K and V rows are one contiguous run each
// in the head-major cache, so they arrive in shared memory as bulk async
// copies, 32 positions per buffer, double-buffered; the first copies are
// issued before the kernel waits for the Q/K/V projection (cache rows below
// the current position were written by earlier steps).  The CTA ropes the
// n_rep query heads of the group once, scores its slice against each of them
// (each K row read once for the whole group), and keeps an exact-max softmax
// partial (m, l, acc) per query head in shared memory.  The n_split CTAs of a
// head form one thread-block cluster; each pushes its partial into rank 0's
// shared memory (distributed shared memory stores), and after a cluster
// barrier rank 0 merges them in split order (deterministic).  CTA
// (g, 0) writes the roped K row and the raw V row of the current position
// into the cache; the CTA whose slice holds the current position uses its own
// copy, so no CTA reads a row another CTA writes.
//
// Cache layout: [layer][kv head][n_ctx][head_dim] fp32.
#pragma once
#include "ecu_common.cuh"
#include "ecu_pipe.cuh"

#include <cooperative_groups.h>
namespace cg = cooperative_groups;

struct AttnArgs {
    const float *qkv;        // q [n_head*hd] | k [nkv*hd] | v [nkv*hd], pre-bias, pre-RoPE
    const float *bq, *bk, *bv;   // biases or null
    const float *rope_cs;    // [n_ctx][hd/2][2] cos, sin
    float       *kc, *vc;    // this layer's cache, [nkv][n_ctx][hd]
    float       *att;        // out [n_head*hd]
    const StepState *st;
    int         *status;
    int          n_head, n_kv, n_rep, n_ctx, n_split;
    float        kscale;     // 1/sqrtf(hd), computed on the host as the reference does
};

// (a*c - b*s, b*c + a*s) with separate roundings (src/engine.c:375-376)
__device__ __forceinline__ void rope_pair(float &a, float &b, float c, float s)
{
    const float na = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    const float nb = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
    a = na;
    b = nb;
}

#define ATT_THREADS 128
#define ATT_SUB 32        // positions per shared-memory buffer (one per lane)
#define ATT_MAX_SPLIT 16  // one cluster per KV head

// K/V rows sit in shared memory with a 16-byte pad, so that the 32 lanes of
// a warp reading the same column of 32 different rows hit distinct banks.
template <int HD>
__host__ __device__ constexpr int attn_row_stride()
{
    return HD + 4;
}

template <int HD>
__host__ __device__ constexpr size_t attn_smem_bytes()
{
    return (size_t)2 * 2 * ATT_SUB * attn_row_stride<HD>() * sizeof(float);   // 2 buffers x (K, V)
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// HD = head_dim (16, 32, 64 or 128), NREP = query heads per KV head.
// Launched with clusters of n_split CTAs along y (one cluster per KV head):
// the split partials meet in rank 0's shared memory.
// Work split inside a CTA: warp w owns query heads w, w+4, ...; for scores a
// lane owns a position, for the V accumulation a lane owns 4 dimensions.
template <int HD, int NREP>
__global__ void __launch_bounds__(ATT_THREADS) k_attention(AttnArgs a)
{
    constexpr int NW = ATT_THREADS / 32;
    constexpr int RS = attn_row_stride<HD>();
    constexpr int LPR = HD / 4;                 // lanes per V row (float4 each)
    constexpr int RPW = 32 / LPR;               // V rows per warp pass
    constexpr int HPW = (NREP + NW - 1) / NW;   // query heads per warp
    extern __shared__ __align__(128) float kvbuf[];   // [2][K|V][ATT_SUB][RS]
    __shared__ __align__(16) float q_s[NREP][HD];
    __shared__ __align__(16) float knew[HD], vnew[HD];
    __shared__ float cs_s[HD];
    // this CTA's (acc[HD], m, l) per head; rows padded to a 16-byte multiple
    // for the float4 stores
    __shared__ __align__(16) float part_s[NREP][HD + 4];
    __shared__ float wsplit[NREP][ATT_MAX_SPLIT];
    __shared__ float invl[NREP];
    __shared__ __align__(8) uint64_t bar[2];

    cg::cluster_group cluster = cg::this_cluster();
    const int g = blockIdx.x, split = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // the position is stable for the whole step (set before the graph runs)
    const int pos = a.st->pos, npos = pos + 1;
    const int chunk = (npos + a.n_split - 1) / a.n_split;
    const int t0 = min(npos, split * chunk), t1 = min(npos, t0 + chunk);
    const int nsub = (t1 - t0 + ATT_SUB - 1) / ATT_SUB;
    float *kbase = a.kc + (size_t)g * a.n_ctx * HD;
    float *vbase = a.vc + (size_t)g * a.n_ctx * HD;

    // rows [c0, c0+ATT_SUB) of the slice below the current position, one row
    // per lane of warp 0, into padded rows; lane 0 first announces the bytes
    auto issue = [&](int sb) {
        const int c0 = t0 + sb * ATT_SUB;
        const int c1 = min(min(t1, c0 + ATT_SUB), pos);
        const int nr = c1 > c0 ? c1 - c0 : 0;
        float *kb = kvbuf + (size_t)(sb & 1) * 2 * ATT_SUB * RS;
        if (lane == 0) mbar_expect_tx(&bar[sb & 1], (uint32_t)(2 * nr * HD * sizeof(float)));
        __syncwarp();
        if (lane < nr) {
            bulk_g2s(kb + lane * RS, kbase + (size_t)(c0 + lane) * HD, HD * sizeof(float), &bar[sb & 1]);
            bulk_g2s(kb + ATT_SUB * RS + lane * RS, vbase + (size_t)(c0 + lane) * HD, HD * sizeof(float),
                     &bar[sb & 1]);
        }
    };
    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        mbar_init_fence();
    }
    __syncthreads();
    if (warp == 0 && nsub > 0) issue(0);
    // the RoPE row depends only on the position: fetch it before waiting
    for (int j = tid; j < HD; j += ATT_THREADS) cs_s[j] = a.rope_cs[(size_t)pos * HD + j];
    pdl_wait();
    pdl_trigger();
    __syncthreads();
    const int qdim = a.n_head * HD, kvdim = a.n_kv * HD;

    // queries of this group, biased and roped; the new K (roped) and V
    for (int i = tid; i < NREP * (HD / 2); i += ATT_THREADS) {
        const int h = i / (HD / 2), j = i % (HD / 2), row = (g * NREP + h) * HD;
        float x0 = a.qkv[row + j], x1 = a.qkv[row + j + HD / 2];
        if (a.bq) { x0 = __fadd_rn(x0, a.bq[row + j]); x1 = __fadd_rn(x1, a.bq[row + j + HD / 2]); }
        rope_pair(x0, x1, cs_s[2 * j], cs_s[2 * j + 1]);
        q_s[h][j] = x0;
        q_s[h][j + HD / 2] = x1;
    }
    for (int j = tid; j < HD / 2; j += ATT_THREADS) {
        const int kr = qdim + g * HD, vr = qdim + kvdim + g * HD;
        float k0 = a.qkv[kr + j], k1 = a.qkv[kr + j + HD / 2];
        float v0 = a.qkv[vr + j], v1 = a.qkv[vr + j + HD / 2];
        if (a.bk) { k0 = __fadd_rn(k0, a.bk[g * HD + j]); k1 = __fadd_rn(k1, a.bk[g * HD + j + HD / 2]); }
        if (a.bv) { v0 = __fadd_rn(v0, a.bv[g * HD + j]); v1 = __fadd_rn(v1, a.bv[g * HD + j + HD / 2]); }
        rope_pair(k0, k1, cs_s[2 * j], cs_s[2 * j + 1]);
        knew[j] = k0; knew[j + HD / 2] = k1;
        vnew[j] = v0; vnew[j + HD / 2] = v1;
    }
    __syncthreads();
    if (split == 0)
        for (int j = tid; j < HD; j += ATT_THREADS) {
            kbase[(size_t)pos * HD + j] = knew[j];
            vbase[(size_t)pos * HD + j] = vnew[j];
        }

    // running softmax state of this warp's heads (identical in all lanes)
    float  m_run[HPW], l_run[HPW];
    float4 acc[HPW];      // dims [4*(lane%LPR), +4) over this lane's V rows
#pragma unroll
    for (int k = 0; k < HPW; k++) {
        m_run[k] = -INFINITY;
        l_run[k] = 0.0f;
        acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (int sb = 0; sb < nsub; sb++) {
        if (warp == 0 && sb + 1 < nsub) issue(sb + 1);   // that buffer was released below
        // on a timeout the status word is set and the stale buffer is used;
        // the host then reports the step as failed
        mbar_wait(&bar[sb & 1], (sb >> 1) & 1, a.status);
        const float *kb = kvbuf + (size_t)(sb & 1) * 2 * ATT_SUB * RS;
        const float *vb = kb + ATT_SUB * RS;
        const int    c0 = t0 + sb * ATT_SUB, cn = min(ATT_SUB, t1 - c0);
        const float *krow = (c0 + lane == pos) ? knew : kb + lane * RS;
#pragma unroll
        for (int k = 0; k < HPW; k++) {
            const int h = warp + k * NW;
            if (h >= NREP) break;
            // score of position c0 + lane against head h
            float s = -INFINITY;
            if (lane < cn) {
                const float4 *k4 = reinterpret_cast<const float4 *>(krow);
                const float4 *q4 = reinterpret_cast<const float4 *>(q_s[h]);
                float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll 8
                for (int j = 0; j < HD / 4; j++) {
                    const float4 kv = k4[j], qv = q4[j];
                    d0 = fmaf(qv.x, kv.x, d0);
                    d1 = fmaf(qv.y, kv.y, d1);
                    d2 = fmaf(qv.z, kv.z, d2);
                    d3 = fmaf(qv.w, kv.w, d3);
                }
                s = ((d0 + d1) + (d2 + d3)) * a.kscale;
            }
            const float mnew = fmaxf(m_run[k], warp_max(s));
            const float f = expf(m_run[k] - mnew);          // 0 while m_run is -inf
            const float e = lane < cn ? expf(s - mnew) : 0.0f;
            l_run[k] = l_run[k] * f + warp_sum(e);
            m_run[k] = mnew;
            acc[k].x *= f; acc[k].y *= f; acc[k].z *= f; acc[k].w *= f;
            // the same trip count in every lane: the shuffle needs all 32
            const int dq = lane % LPR;
            for (int pb = 0; pb < cn; pb += RPW) {
                const int   p = pb + lane / LPR;
                const float ep = __shfl_sync(0xffffffffu, e, p & 31);
                if (p < cn) {
                    const float4 vv = (c0 + p == pos) ? reinterpret_cast<const float4 *>(vnew)[dq]
                                                      : reinterpret_cast<const float4 *>(vb + p * RS)[dq];
                    acc[k].x = fmaf(ep, vv.x, acc[k].x);
                    acc[k].y = fmaf(ep, vv.y, acc[k].y);
                    acc[k].z = fmaf(ep, vv.z, acc[k].z);
                    acc[k].w = fmaf(ep, vv.w, acc[k].w);
                }
            }
        }
        __syncthreads();      // buffer sb&1 is free for sub-chunk sb+2
    }
    // this CTA's partial per head: acc summed over the RPW row groups
#pragma unroll
    for (int k = 0; k < HPW; k++) {
        const int h = warp + k * NW;
        if (h >= NREP) break;
#pragma unroll
        for (int o = LPR; o < 32; o <<= 1) {
            acc[k].x += __shfl_xor_sync(0xffffffffu, acc[k].x, o);
            acc[k].y += __shfl_xor_sync(0xffffffffu, acc[k].y, o);
            acc[k].z += __shfl_xor_sync(0xffffffffu, acc[k].z, o);
            acc[k].w += __shfl_xor_sync(0xffffffffu, acc[k].w, o);
        }
        if (lane < LPR) reinterpret_cast<float4 *>(part_s[h])[lane] = acc[k];
        if (lane == 0) {
            part_s[h][HD] = m_run[k];
            part_s[h][HD + 1] = l_run[k];
        }
    }
    // ---- merge: every CTA pushes its partial into rank 0's K/V buffer -----
    // (rank 0's buffer is free once every CTA of the cluster is past its
    // loop), then rank 0 merges from local shared memory in split order.
    constexpr int PER = NREP * (HD + 4);        // floats of one partial
    const int ns = a.n_split;
    cluster.sync();                             // all CTAs done with their K/V buffers
    __syncthreads();
    {
        float *dst = cluster.map_shared_rank(kvbuf, 0) + (size_t)split * PER;
        const float4 *src4 = reinterpret_cast<const float4 *>(&part_s[0][0]);
        float4 *dst4 = reinterpret_cast<float4 *>(dst);
        for (int i = tid; i < PER / 4; i += ATT_THREADS) dst4[i] = src4[i];
    }
    cluster.sync();                             // the pushes are visible to rank 0
    if (cluster.block_rank() != 0) return;
    const float *gath = kvbuf;                  // [ns][NREP][HD + 4]
    if (tid < NREP) {
        const int h = tid;
        float M = -INFINITY;
        for (int r = 0; r < ns; r++) M = fmaxf(M, gath[r * PER + h * (HD + 4) + HD]);
        float L = 0.0f;
        for (int r = 0; r < ns; r++) {
            const float ms = gath[r * PER + h * (HD + 4) + HD];
            const float w = ms > -INFINITY ? expf(ms - M) : 0.0f;
            wsplit[h][r] = w;
            L += gath[r * PER + h * (HD + 4) + HD + 1] * w;
        }
        invl[h] = L > 0.0f ? 1.0f / L : 0.0f;
    }
    __syncthreads();
    for (int i = tid; i < NREP * HD; i += ATT_THREADS) {
        const int h = i / HD, d = i % HD;
        float o = 0.0f;
        for (int r = 0; r < ns; r++) o = fmaf(gath[r * PER + h * (HD + 4) + d], wsplit[h][r], o);
        a.att[(g * NREP + h) * HD + d] = o * invl[h];
    }
}
