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
// partial (m, l, acc) per query head.  The last CTA of a head to finish
// (atomic ticket, no waiting) merges the partials in split order, so results
// are deterministic.  CTA (g, 0) writes the roped K row and the raw V row of
// the current position into the cache; the CTA whose slice holds the current
// position uses its own copy, so no CTA reads a row another CTA writes.
//
// Cache layout: [layer][kv head][n_ctx][head_dim] fp32.
#pragma once
#include "ecu_common.cuh"
#include "ecu_pipe.cuh"

struct AttnArgs {
    const float *qkv;        // q [n_head*hd] | k [nkv*hd] | v [nkv*hd], pre-bias, pre-RoPE
    const float *bq, *bk, *bv;   // biases or null
    const float *rope_cs;    // [n_ctx][hd/2][2] cos, sin
    float       *kc, *vc;    // this layer's cache, [nkv][n_ctx][hd]
    float       *att;        // out [n_head*hd]
    float       *part;       // scratch [nkv][n_split][n_rep][hd + 2]
    unsigned    *counter;    // [nkv], zero between launches
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
#define ATT_SUB 32        // positions per shared-memory buffer
#define ATT_MAX_SPLIT 64

template <int HD>
__host__ __device__ constexpr size_t attn_smem_bytes()
{
    return (size_t)2 * 2 * ATT_SUB * HD * sizeof(float);   // 2 buffers x (K, V)
}

// HD = head_dim (16, 32, 64 or 128), NREP = query heads per KV head.
// Needs n_split <= ATT_MAX_SPLIT and n_split*NREP*(HD+2) floats to fit the
// K/V buffers (the merge reuses them); the host planner guarantees both.
template <int HD, int NREP>
__global__ void __launch_bounds__(ATT_THREADS) k_attention(AttnArgs a)
{
    constexpr int LPP = HD / 4;              // lanes per position (float4 each)
    constexpr int PPW = 32 / LPP;            // positions per warp pass
    constexpr int NW = ATT_THREADS / 32;
    extern __shared__ __align__(128) float kvbuf[];   // [2][K|V][ATT_SUB][HD]
    __shared__ __align__(16) float q_s[NREP][HD];
    __shared__ __align__(16) float knew[HD], vnew[HD];
    __shared__ float sc[NREP][ATT_SUB];
    __shared__ __align__(16) float acc_s[NW][NREP][HD];
    __shared__ float wsplit[NREP][ATT_MAX_SPLIT];
    __shared__ __align__(8) uint64_t bar[2];
    __shared__ unsigned s_last;

    const int g = blockIdx.x, split = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // the position is stable for the whole step (set before the graph runs)
    const int pos = a.st->pos, npos = pos + 1;
    const int chunk = (npos + a.n_split - 1) / a.n_split;
    const int t0 = min(npos, split * chunk), t1 = min(npos, t0 + chunk);
    const int nsub = (t1 - t0 + ATT_SUB - 1) / ATT_SUB;
    float *kbase = a.kc + (size_t)g * a.n_ctx * HD;
    float *vbase = a.vc + (size_t)g * a.n_ctx * HD;

    // rows [c0, c0+ATT_SUB) of the slice that lie below the current position
    auto issue = [&](int sb) {
        const int c0 = t0 + sb * ATT_SUB;
        const int c1 = min(min(t1, c0 + ATT_SUB), pos);
        const uint32_t bytes = c1 > c0 ? (uint32_t)((c1 - c0) * HD * sizeof(float)) : 0u;
        float *kb = kvbuf + (size_t)(sb & 1) * 2 * ATT_SUB * HD;
        mbar_expect_tx(&bar[sb & 1], 2 * bytes);
        if (bytes) {
            bulk_g2s(kb, kbase + (size_t)c0 * HD, bytes, &bar[sb & 1]);
            bulk_g2s(kb + ATT_SUB * HD, vbase + (size_t)c0 * HD, bytes, &bar[sb & 1]);
        }
    };
    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        mbar_init_fence();
        if (nsub > 0) issue(0);
    }
    pdl_wait();
    pdl_trigger();
    const float *cs = a.rope_cs + (size_t)pos * HD;   // HD/2 (cos, sin) pairs
    const int qdim = a.n_head * HD, kvdim = a.n_kv * HD;

    // queries of this group, biased and roped; the new K (roped) and V
    for (int i = tid; i < NREP * (HD / 2); i += ATT_THREADS) {
        const int h = i / (HD / 2), j = i % (HD / 2), row = (g * NREP + h) * HD;
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
    if (split == 0)
        for (int j = tid; j < HD; j += ATT_THREADS) {
            kbase[(size_t)pos * HD + j] = knew[j];
            vbase[(size_t)pos * HD + j] = vnew[j];
        }

    float  m_run[NREP], l_run[NREP];
    float4 acc[NREP];     // dims [4*(lane%LPP), +4) of this lane's positions
#pragma unroll
    for (int h = 0; h < NREP; h++) {
        m_run[h] = -INFINITY;
        l_run[h] = 0.0f;
        acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const int sub_slot = lane / LPP, dl = lane % LPP;
    for (int sb = 0; sb < nsub; sb++) {
        if (tid == 0 && sb + 1 < nsub) issue(sb + 1);   // that buffer was released below
        // on a timeout the status word is set and the stale buffer is used;
        // the step's result is then reported as an error by the host
        mbar_wait(&bar[sb & 1], (sb >> 1) & 1, a.status);
        const float *kb = kvbuf + (size_t)(sb & 1) * 2 * ATT_SUB * HD;
        const float *vb = kb + ATT_SUB * HD;
        const int    c0 = t0 + sb * ATT_SUB, cn = min(ATT_SUB, t1 - c0);
        // scores: warp w handles positions w*PPW + sub_slot, stride NW*PPW
        for (int p = warp * PPW + sub_slot; p < ((cn + PPW - 1) / PPW) * PPW; p += NW * PPW) {
            const bool   ok = p < cn;
            const int    pp = ok ? p : 0;
            const float4 kv = (c0 + pp == pos) ? reinterpret_cast<const float4 *>(knew)[dl]
                                               : reinterpret_cast<const float4 *>(kb + pp * HD)[dl];
#pragma unroll
            for (int h = 0; h < NREP; h++) {
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
#pragma unroll
        for (int h = 0; h < NREP; h++) {
            float mx = -INFINITY;
            for (int p = 0; p < cn; p++) mx = fmaxf(mx, sc[h][p]);
            const float mnew = fmaxf(m_run[h], mx);
            const float f = expf(m_run[h] - mnew);   // 0 when m_run was -inf
            l_run[h] *= f;
            acc[h].x *= f; acc[h].y *= f; acc[h].z *= f; acc[h].w *= f;
            m_run[h] = mnew;
        }
        for (int p = warp * PPW + sub_slot; p < cn; p += NW * PPW) {
            const float4 vv = (c0 + p == pos) ? reinterpret_cast<const float4 *>(vnew)[dl]
                                              : reinterpret_cast<const float4 *>(vb + p * HD)[dl];
#pragma unroll
            for (int h = 0; h < NREP; h++) {
                const float e = expf(sc[h][p] - m_run[h]);
                l_run[h] += e;
                acc[h].x = fmaf(e, vv.x, acc[h].x);
                acc[h].y = fmaf(e, vv.y, acc[h].y);
                acc[h].z = fmaf(e, vv.z, acc[h].z);
                acc[h].w = fmaf(e, vv.w, acc[h].w);
            }
        }
        __syncthreads();      // buffer sb&1 is free for sub-chunk sb+2
    }
    // reduce over sub-slots (shuffles) and warps (shared memory)
#pragma unroll
    for (int h = 0; h < NREP; h++) {
        float l = l_run[h];
        for (int o = LPP; o < 32; o <<= 1) {
            l += __shfl_xor_sync(0xffffffffu, l, o);
            acc[h].x += __shfl_xor_sync(0xffffffffu, acc[h].x, o);
            acc[h].y += __shfl_xor_sync(0xffffffffu, acc[h].y, o);
            acc[h].z += __shfl_xor_sync(0xffffffffu, acc[h].z, o);
            acc[h].w += __shfl_xor_sync(0xffffffffu, acc[h].w, o);
        }
        if (sub_slot == 0) reinterpret_cast<float4 *>(acc_s[warp][h])[dl] = acc[h];
        if (lane == 0) sc[h][warp] = l;       // per-warp l
    }
    __syncthreads();
    float *mypart = a.part + ((size_t)g * a.n_split + split) * NREP * (HD + 2);
    for (int i = tid; i < NREP * HD; i += ATT_THREADS) {
        const int h = i / HD, d = i % HD;
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; w++) s += acc_s[w][h][d];
        mypart[h * (HD + 2) + d] = s;
    }
    if (tid < NREP) {
        float l = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; w++) l += sc[tid][w];
        mypart[tid * (HD + 2) + HD] = m_run[tid];
        mypart[tid * (HD + 2) + HD + 1] = l;
    }
    // ---- the last CTA of this head merges the n_split partials ----------
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(&a.counter[g], 1u) == (unsigned)a.n_split - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float *hp = a.part + (size_t)g * a.n_split * NREP * (HD + 2);
    const int    per = NREP * (HD + 2), total = a.n_split * per;
    float       *pm = kvbuf;                  // reuse the K/V buffers
    for (int i = tid; i < total; i += ATT_THREADS) pm[i] = __ldcg(hp + i);
    __syncthreads();
    if (tid < NREP) {
        const int h = tid;
        float M = -INFINITY;
        for (int s = 0; s < a.n_split; s++) M = fmaxf(M, pm[s * per + h * (HD + 2) + HD]);
        float L = 0.0f;
        for (int s = 0; s < a.n_split; s++) {
            const float ms = pm[s * per + h * (HD + 2) + HD];
            const float w = ms > -INFINITY ? expf(ms - M) : 0.0f;
            wsplit[h][s] = w;
            L += pm[s * per + h * (HD + 2) + HD + 1] * w;
        }
        sc[h][0] = L > 0.0f ? 1.0f / L : 0.0f;
    }
    __syncthreads();
    for (int i = tid; i < NREP * HD; i += ATT_THREADS) {
        const int h = i / HD, d = i % HD;
        float o = 0.0f;
        for (int s = 0; s < a.n_split; s++) o = fmaf(pm[s * per + h * (HD + 2) + d], wsplit[h][s], o);
        a.att[(g * NREP + h) * HD + d] = o * sc[h][0];
    }
    if (tid == 0) a.counter[g] = 0u;
}
