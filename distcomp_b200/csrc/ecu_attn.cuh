// ecu_attn.cuh -- decode attention with the Q/K/V bias, NeoX RoPE and the
// KV-cache append of the current position fused in (src/engine.c:392-450).
//
// Grid (n_head_kv, n_split).  CTA (g, s) owns KV head g and a contiguous
// slice of positions [0, pos]; it ropes the n_rep query heads of the group
// once, scores its slice against each of them (the K row is loaded once and
// shared by the group), and keeps an exact-max softmax partial (m, l, acc)
// per query head.  The last CTA of a head to finish (atomic ticket, no
// waiting) merges the partials in split order, so results are deterministic.
// CTA (g, 0) writes the roped K row and the raw V row of the current
// position into the cache; the CTA whose slice holds the current position
// uses its own copy, so no CTA reads a row another CTA is writing.
//
// Cache layout: [layer][kv head][n_ctx][head_dim] fp32 (head-major, so a
// head's positions are one contiguous run).
#pragma once
#include "ecu_common.cuh"

struct AttnArgs {
    const float *qkv;        // q [n_head*hd] | k [nkv*hd] | v [nkv*hd], pre-bias, pre-RoPE
    const float *bq, *bk, *bv;   // biases or null
    const float *rope_cs;    // [n_ctx][hd/2][2] cos, sin
    float       *kc, *vc;    // this layer's cache, [nkv][n_ctx][hd]
    float       *att;        // out [n_head*hd]
    float       *part;       // scratch [nkv][n_split][n_rep][hd + 2]
    unsigned    *counter;    // [nkv], zero between launches
    const StepState *st;
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
#define ATT_CHUNK 64      // positions scored per pass

// HD = head_dim (16, 32, 64 or 128), NREP = query heads per KV head.
template <int HD, int NREP>
__global__ void __launch_bounds__(ATT_THREADS) k_attention(AttnArgs a)
{
    constexpr int LPP = HD / 4;              // lanes per position (float4 each)
    constexpr int PPW = 32 / LPP;            // positions per warp pass
    constexpr int NW = ATT_THREADS / 32;
    constexpr int nrep = NREP;
    __shared__ __align__(16) float q_s[NREP][HD];
    __shared__ __align__(16) float knew[HD], vnew[HD];
    __shared__ float sc[NREP][ATT_CHUNK];
    __shared__ __align__(16) float acc_s[NW][NREP][HD];
    __shared__ unsigned s_last;

    pdl_wait();
    pdl_trigger();
    const int g = blockIdx.x, split = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int pos = a.st->pos, npos = pos + 1;
    const int chunk = (npos + a.n_split - 1) / a.n_split;
    const int t0 = min(npos, split * chunk), t1 = min(npos, t0 + chunk);
    const float *cs = a.rope_cs + (size_t)pos * HD;   // HD/2 (cos, sin) pairs
    const int qdim = a.n_head * HD, kvdim = a.n_kv * HD;

    // queries of this group, biased and roped; the new K (roped) and V
    for (int i = tid; i < nrep * (HD / 2); i += ATT_THREADS) {
        const int h = i / (HD / 2), j = i % (HD / 2), row = (g * nrep + h) * HD;
        float x0 = a.qkv[row + j], x1 = a.qkv[row + j + HD / 2];
        if (a.bq) { x0 = __fadd_rn(x0, a.bq[row + j]); x1 = __fadd_rn(x1, a.bq[row + j + HD / 2]); }
        rope_pair(x0, x1, cs[2 * j], cs[2 * j + 1]);
        q_s[h][j] = x0;
        q_s[h][j + HD / 2] = x1;
    }
    for (int j = tid; j < HD / 2; j += ATT_THREADS) {
        const int kr = qdim + g * HD, vr = qdim + kvdim + g * HD;
        float k0 = a.qkv[kr + j], k1 = a.qkv[kr + j + HD / 2];
        float v0 = a.qkv[vr + j], v1 = a.qkv[vr + j + HD / 2];
        if (a.bk) { k0 = __fadd_rn(k0, a.bk[g * HD + j]); k1 = __fadd_rn(k1, a.bk[g * HD + j + HD / 2]); }
        if (a.bv) { v0 = __fadd_rn(v0, a.bv[g * HD + j]); v1 = __fadd_rn(v1, a.bv[g * HD + j + HD / 2]); }
        rope_pair(k0, k1, cs[2 * j], cs[2 * j + 1]);
        knew[j] = k0; knew[j + HD / 2] = k1;
        vnew[j] = v0; vnew[j + HD / 2] = v1;
    }
    __syncthreads();
    float *krow_base = a.kc + (size_t)g * a.n_ctx * HD;
    float *vrow_base = a.vc + (size_t)g * a.n_ctx * HD;
    if (split == 0)
        for (int j = tid; j < HD; j += ATT_THREADS) {
            krow_base[(size_t)pos * HD + j] = knew[j];
            vrow_base[(size_t)pos * HD + j] = vnew[j];
        }

    // running per-head softmax state of this CTA (exact max over its slice)
    float m_run[NREP], l_run[NREP];
    // lane's accumulator: dims [4*(lane%LPP), +4) for positions of its sub-slot
    float4 acc[NREP];
#pragma unroll
    for (int h = 0; h < NREP; h++) {
        m_run[h] = -INFINITY;
        l_run[h] = 0.0f;
        acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const int sub = lane / LPP, dl = lane % LPP;   // position sub-slot, dim quad
    for (int c0 = t0; c0 < t1; c0 += ATT_CHUNK) {
        const int cn = min(ATT_CHUNK, t1 - c0);
        // scores: warp w handles positions c0 + w*PPW + sub, stride NW*PPW
        for (int p = warp * PPW + sub; p < ((cn + PPW - 1) / PPW) * PPW; p += NW * PPW) {
            const bool ok = p < cn;
            const int  t = c0 + (ok ? p : 0);
            float4 kv;
            if (t == pos) kv = reinterpret_cast<const float4 *>(knew)[dl];
            else kv = reinterpret_cast<const float4 *>(krow_base + (size_t)t * HD)[dl];
#pragma unroll
            for (int h = 0; h < nrep; h++) {
                const float4 qv = reinterpret_cast<const float4 *>(q_s[h])[dl];
                float d = qv.x * kv.x;
                d = fmaf(qv.y, kv.y, d);
                d = fmaf(qv.z, kv.z, d);
                d = fmaf(qv.w, kv.w, d);
#pragma unroll
                for (int o = LPP / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
                if (ok && dl == 0) sc[h][p] = d * a.kscale;
            }
        }
        __syncthreads();
        // chunk max per head, rescale running state
#pragma unroll
        for (int h = 0; h < nrep; h++) {
            float mx = -INFINITY;
            for (int p = 0; p < cn; p++) mx = fmaxf(mx, sc[h][p]);
            const float mnew = fmaxf(m_run[h], mx);
            const float f = expf(m_run[h] - mnew);   // 0 when m_run was -inf
            l_run[h] *= f;
            acc[h].x *= f; acc[h].y *= f; acc[h].z *= f; acc[h].w *= f;
            m_run[h] = mnew;
        }
        // e = exp(s - m); l += e; acc += e * v
        for (int p = warp * PPW + sub; p < cn; p += NW * PPW) {
            const int    t = c0 + p;
            const float4 vv = (t == pos) ? reinterpret_cast<const float4 *>(vnew)[dl]
                                         : reinterpret_cast<const float4 *>(vrow_base + (size_t)t * HD)[dl];
#pragma unroll
            for (int h = 0; h < nrep; h++) {
                const float e = expf(sc[h][p] - m_run[h]);
                l_run[h] += e;
                acc[h].x = fmaf(e, vv.x, acc[h].x);
                acc[h].y = fmaf(e, vv.y, acc[h].y);
                acc[h].z = fmaf(e, vv.z, acc[h].z);
                acc[h].w = fmaf(e, vv.w, acc[h].w);
            }
        }
        __syncthreads();
    }
    // l_run counts e over the positions this lane visited; reduce everything
    // over (sub-slots, warps) into one partial per head
#pragma unroll
    for (int h = 0; h < nrep; h++) {
        float l = l_run[h];
        for (int o = LPP; o < 32; o <<= 1) {
            l += __shfl_xor_sync(0xffffffffu, l, o);
            acc[h].x += __shfl_xor_sync(0xffffffffu, acc[h].x, o);
            acc[h].y += __shfl_xor_sync(0xffffffffu, acc[h].y, o);
            acc[h].z += __shfl_xor_sync(0xffffffffu, acc[h].z, o);
            acc[h].w += __shfl_xor_sync(0xffffffffu, acc[h].w, o);
        }
        l_run[h] = l;
        if (sub == 0) reinterpret_cast<float4 *>(acc_s[warp][h])[dl] = acc[h];
        if (lane == 0) sc[h][warp] = l;     // reuse sc as per-warp l scratch
    }
    __syncthreads();
    float *mypart = a.part + ((size_t)g * a.n_split + split) * nrep * (HD + 2);
    for (int i = tid; i < nrep * HD; i += ATT_THREADS) {
        const int h = i / HD, d = i % HD;
        float s = 0.0f;
        for (int w = 0; w < NW; w++) s += acc_s[w][h][d];
        mypart[h * (HD + 2) + d] = s;
    }
    if (tid == 0) {
#pragma unroll
        for (int h = 0; h < nrep; h++) {
            float l = 0.0f;
            for (int w = 0; w < NW; w++) l += sc[h][w];
            mypart[h * (HD + 2) + HD] = m_run[h];
            mypart[h * (HD + 2) + HD + 1] = l;
        }
    }
    // ---- the last CTA of this head merges the n_split partials ----------
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(&a.counter[g], 1u) == (unsigned)a.n_split - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const volatile float *hp = a.part + (size_t)g * a.n_split * nrep * (HD + 2);
    for (int h = 0; h < nrep; h++) {
        float M = -INFINITY;
        for (int s = 0; s < a.n_split; s++) M = fmaxf(M, hp[(s * nrep + h) * (HD + 2) + HD]);
        float L = 0.0f;
        for (int s = 0; s < a.n_split; s++) {
            const float ms = hp[(s * nrep + h) * (HD + 2) + HD];
            if (ms > -INFINITY) L += hp[(s * nrep + h) * (HD + 2) + HD + 1] * expf(ms - M);
        }
        const float inv = L > 0.0f ? 1.0f / L : 0.0f;
        for (int d = tid; d < HD; d += ATT_THREADS) {
            float o = 0.0f;
            for (int s = 0; s < a.n_split; s++) {
                const float ms = hp[(s * nrep + h) * (HD + 2) + HD];
                if (ms > -INFINITY) o += hp[(s * nrep + h) * (HD + 2) + d] * expf(ms - M);
            }
            a.att[(g * nrep + h) * HD + d] = o * inv;
        }
    }
    if (tid == 0) a.counter[g] = 0u;
}
