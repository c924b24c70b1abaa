// ecu_mega.cuh -- one decode step of a LAYERS or FULL stage as one persistent
// kernel.
//
// The step is a list of phases (built on the host from the stage's layers):
//
//   [embed]  per layer: Q/K/V GEMV (RMSNorm prologue) | attention over
//   (KV head, position split) items | merge of the splits per query head |
//   O GEMV (+ residual) | gate/up GEMV (RMSNorm prologue, SwiGLU epilogue) |
//   down GEMV (+ residual);  [head: RMSNorm + logits GEMV + argmax]
//
// -- the order of src/engine.c:380-497.  One CTA per SM, all resident
// (cooperative launch).  There is no grid barrier: the vectors that cross
// CTAs (residual stream, Q/K/V, attention output, SwiGLU output) are
// epoch-tagged words (ll_put), and each phase starts on its input as soon as
// the words it reads carry the epoch of the phase that writes them.  Every
// weight row this CTA multiplies during the whole step streams through a
// shared-memory ring of bulk async copies in phase order; the warp that
// releases a ring stage last issues the copy that refills it with the next
// chunk of the list, so there is no producer warp (16 warps of 128 registers
// rather than 17 of 96).  Weights do not depend on activations, so the
// weight stream runs ahead of the phase boundaries: while a CTA waits for
// its next input, that phase's rows are already landing.
// The GEMV arithmetic is the one of k_gemv_fast (int8 digit planes of the
// input, dp4a, the same row partials added in the same order), so its
// results are the same bits.
//
// The phase loop holds one copy of each phase body (the GEMV for Q4_0 and
// for Q8_0 rows, attention, merge, embed), whatever the layer count.
#pragma once
#include "ecu_attn.cuh"
#include "ecu_gemv.cuh"

#define MEGA_NCW 16                      // warps (all of them consume the ring)
#define MEGA_THREADS (32 * MEGA_NCW)
#define MEGA_RING_BYTES (128 * 1024)    // default weight ring, split into nst stages
#define MEGA_ATT_SUB 24                  // K/V rows per buffer (4 buffers: K and V of two halves), one slot
#define MEGA_MAX_STAGES 8
#define MEGA_MAX_NB 512                  // input blocks of a GEMV (n_in <= 16384)
#define MEGA_MAX_SPLIT 64                // position splits per KV head
#define MEGA_RED4_MAX 6600               // floats of 4-lane row partials a GEMV phase may keep
#ifndef ECU_MAX_TP
#define ECU_MAX_TP 8                     // tensor-parallel ranks
#endif

enum MegaKind : int { PH_EMBED = 0, PH_GEMV = 1, PH_ATTN = 2 };

// One phase of the step.
struct MegaPhase {
    int            kind;
    int            fmt;        // GEMV: 4 = Q4_0 SPLIT4 rows, 8 = Q8_0 SPLIT8 rows, 12 = Q4_K SPLITK4 rows
    int            norm;       // GEMV: RMSNorm of x (weights norm_w) first
    int            epi;        // GEMV: Epi
    const uint8_t *w;
    unsigned       row_bytes;
    int            n_in, n_out;
    int            rpc;        // rows per CTA (even for SwiGLU)
    int            sr;         // rows per ring stage
    int            nkg;        // n_in / 1024
    int            rowpar;     // consumer warps per k-group
    int            red4;       // row partials kept per lane pair of an 8-lane group (4 per row and k-group)
    const float   *x;
    const float   *norm_w;
    float         *y;
    float         *xn;         // GEMV with norm: CTA 0 stores the normed input here
    float         *kc, *vc;    // ATTN: this layer's cache planes [nkv][n_ctx][hd]; the Q/K/V GEMV
                               // before it: the same planes (its early K/V copies)
    const float   *bq, *bk, *bv;
    int            next_attn;  // the next phase is attention
    // epoch-tagged vectors (see ll_put): the phase that wrote this phase's
    // input (in_ep) and, for a residual add, the residual (y_ep); -1 = the
    // plain kernel input.  out_plain: also store the output as plain floats
    int            in_ep, y_ep, out_plain;
    const unsigned long long *x_ll;    // input vector, tagged
    unsigned long long       *y_ll;    // output vector, tagged
    int            out_base;   // index of this rank's first output element in y_ll (tensor parallel)
    int            bcast;      // outputs go to every rank's copy of y_ll
    int            pad_[2];
};
static_assert(sizeof(MegaPhase) % 16 == 0, "phase descriptors are copied in 16-byte pieces");

struct MegaArgs {
    const MegaPhase *ph;
    int              n_ph;
    const uint4     *tab;           // per phase, the ring cursor's view (mega_tab_entry); copied to shared memory
    DevMat           emb;           // PH_EMBED: the RAW embedding matrix
    float           *state;         // residual stream, n_embd (+1: token as float)
    float           *qkv, *att;
    unsigned long long *apart_ll;   // attention partials, tagged: [n_kv][n_split][NREP][HD + 2]
    float           *xn_tmp;        // head: normed state, copied to state at the end
    float           *part_val;      // argmax: per-CTA best
    int             *part_idx;
    unsigned        *ticket;        // argmax ticket, zero between steps
    unsigned        *bar;           // [1]: CTAs done with the launch, [3]: launches so far
    unsigned long long *x_ll, *qkv_ll, *att_ll, *h_ll;   // tagged activation vectors
    unsigned        *att_ticket;    // per KV head: splits done, zero between phases
    StepState       *st;
    int             *tok_hist;
    int             *status;
    const float     *rope_cs;
    unsigned long long *phase_ns;   // optional: CTA 0's time at the end of each phase
    unsigned long long *phase_clk;  // optional, with phase_ns: CTA 0's SM clock at the same points
    unsigned long long *phase_detail; // optional, [n_ph][4]: CTA 0's SM clock after the prologue,
                                    // after the main loop, after the epilogue; [3]: GEMV: ns its
                                    // warp 0 waited for ring stages, attention: when head 0 merged
    int              advance_pos;   // argmax epilogue advances st->pos (FULL)
    int              layers_advance;// LAYERS: st->pos++ once the last phase is done
    int              n_embd, n_head, n_kv, n_ctx, n_split;   // n_head, n_kv: this rank's heads
    int              tp_rank, tp_world;
    unsigned long long *ll_block;   // this rank's tagged vectors (x_ll ... the argmax slots)
    unsigned long long *peer[ECU_MAX_TP];   // every rank's block (IPC mappings), this one's included
    unsigned long long *arg_ll;     // argmax exchange: value and index word per rank
    int              vocab_base;    // first vocabulary row of this rank's head slice
    int              red_floats;    // row-partial floats the largest GEMV phase keeps
    unsigned         union_bytes;   // digit planes | attention K/V buffers
    int              nst;           // ring stages (<= MEGA_MAX_STAGES)
    int              pf_stages;     // chunks warmed in L2 ahead of the ring
    unsigned         stage_bytes;   // bytes per ring stage (multiple of 128)
    int              att_sub;       // attention: K/V rows per buffer (even, <= 32)
    int              att_nsl;       // attention: buffer slots (1, or 2: a round's copies overlap the previous round)
    int              att_l2;        // warm the next attention's K/V rows in L2: 2 at the start of the GEMV
                                    // before it, 1 at its end, 0 not
    int              att_early;     // the Q/K/V phase issues the attention's first nsl rounds of K/V copies
    int              stall_phase;   // failure-path testing: this GEMV phase waits for an input epoch that
                                    // no phase writes, so its bounded waits run out (-1: none)
    unsigned         kv_off;        // byte offset of the attention K/V buffers in the union (above the
                                    // Q/K/V phase's digit planes when att_early)
    // pipeline links (contexts on consecutive GPUs, one per stage): tagged
    // words with link_epoch(position) written into the next stage's memory
    unsigned long long *link_x;     // the stage's output state -> the next stage's x_ll (or null)
    unsigned long long *link_tok;   // the head's argmax -> the first stage's token word (or null)
    unsigned long long *tok_ll;     // this context's token word (a linked embedding reads it)
    int              link_in;       // the embedding waits for its token in tok_ll
    unsigned long long *cta_ns;     // optional, [n_ph + 1][grid]: every CTA's time at the start and at
                                    // the end of each phase (the skew between CTAs at phase boundaries)
    float            eps, kscale;
};

// ------------------------------------------------------- tagged vectors --
// The phases hand vectors to each other without grid barriers: every element
// is one 8-byte word {float, epoch of the phase that wrote it}, stored and
// loaded whole (aligned 64-bit relaxed accesses are single-copy atomic; GPU
// scope, or system scope in the instantiation for tensor-parallel ranks,
// which write into each other's memory over NVLink), so a reader that sees
// the epoch it expects also sees the value.  A reader spins on words that still carry an
// older epoch.  Epoch = (launch number mod 2^20) << 12 | (phase + 1): unique
// within a launch and against the previous one, which wrote every word.
// Every phase's input depends on all CTAs' output of an earlier phase, so
// these waits also order each buffer's reuse one layer later.

__device__ __forceinline__ unsigned ll_epoch(unsigned launch, int phase)
{
    return ((launch & 0xFFFFFu) << 12) | (unsigned)(phase + 1);
}

// A pipeline link: the words one stage's step writes into the next stage's
// memory (another GPU's) carry the token position and the low 12 bits all
// ones, which no phase epoch has (phase + 1 < 4095): the receiver knows the
// position of its step, and a stage writes position p + 1 only after the
// receiver's step p is over (the token has gone round the ring of stages).
// Phase inputs marked MEGA_EP_LINK read those words (system scope: another
// GPU wrote them); MEGA_EP_PLAIN inputs read the plain state.
#define MEGA_EP_PLAIN (-1)
#define MEGA_EP_LINK  (-2)
__device__ __forceinline__ unsigned link_epoch(int pos)
{
    return (((unsigned)pos & 0xFFFFFu) << 12) | 0xFFFu;
}

// SYS: system scope (tensor-parallel ranks read and write each other's
// words over NVLink); otherwise GPU scope.
template <bool SYS>
__device__ __forceinline__ void ll_put(unsigned long long *p, float v, unsigned e)
{
    const unsigned long long w = ((unsigned long long)e << 32) | __float_as_uint(v);
    if constexpr (SYS)
        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
    else
        asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

// A phase output element: into this rank's vector, or (bcast) into every
// rank's copy at the same offset.
template <bool SYS>
__device__ __forceinline__ void ll_put_out(const MegaArgs &a, bool bcast, unsigned long long *p, float v, unsigned e)
{
    if (!bcast) {
        ll_put<SYS>(p, v, e);
        return;
    }
    const size_t off = (size_t)(p - a.ll_block);
    for (int k = 0; k < a.tp_world; k++) ll_put<SYS>(a.peer[k] + off, v, e);
}

template <bool SYS>
__device__ __forceinline__ unsigned long long ll_word(const unsigned long long *p)
{
    unsigned long long w;
    if constexpr (SYS)
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    else
        asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

template <bool SYS>
__device__ __forceinline__ ulonglong2 ll_word2(const unsigned long long *p)
{
    ulonglong2 w;
    if constexpr (SYS)
        asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(w.x), "=l"(w.y) : "l"(p) : "memory");
    else
        asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(w.x), "=l"(w.y) : "l"(p) : "memory");
    return w;
}

// The same with the scope chosen at run time (system scope for words that
// another GPU writes).
__device__ __forceinline__ ulonglong2 ll_word2_rt(const unsigned long long *p, bool sys)
{
    ulonglong2 w;
    if (sys)
        asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(w.x), "=l"(w.y) : "l"(p) : "memory");
    else
        asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(w.x), "=l"(w.y) : "l"(p) : "memory");
    return w;
}

// Spin helper: true while waiting is still allowed (bounded; gives up at
// once when the step is already flagged as failed).
__device__ __forceinline__ bool ll_keep_waiting(unsigned it, uint64_t &t0, int *status)
{
    if ((it & 255u) != 0) return true;
    if (it == 256) t0 = globaltimer_ns();
    if (*reinterpret_cast<volatile int *>(status) != 0) return false;
    if (globaltimer_ns() - t0 > wait_limit_ns()) {
        atomicOr(status, ECU_STATUS_TIMEOUT);
        return false;
    }
    return true;
}

template <bool SYS>
__device__ __forceinline__ float ll_get(const unsigned long long *p, unsigned e, int *status)
{
    unsigned long long w = ll_word<SYS>(p);
    uint64_t t0 = 0;
    for (unsigned it = 1; (unsigned)(w >> 32) != e && ll_keep_waiting(it, t0, status); it++) w = ll_word<SYS>(p);
    return __uint_as_float((unsigned)w);
}

// Four tagged words (two 16-byte loads) all carrying epoch e.
__device__ __forceinline__ bool ll_tags4(const ulonglong2 (&w)[2], unsigned e)
{
    return (unsigned)(w[0].x >> 32) == e && (unsigned)(w[0].y >> 32) == e && (unsigned)(w[1].x >> 32) == e &&
           (unsigned)(w[1].y >> 32) == e;
}

// Float4s t = t0 + k*stride (k < K, t < nq) of a phase input: tagged (phase
// in_ep of this launch) or the plain kernel input.  Every load is issued
// before the first wait, so the K fetches cost one L2 round trip, not K.
template <int K, bool SYS>
__device__ __forceinline__ void input_batch(const MegaArgs &a, const MegaPhase &ph, int t0, int stride, int nq,
                                            unsigned ein, float4 (&v)[K])
{
    if (ph.in_ep != MEGA_EP_PLAIN) {
        // (a pipeline link's words come from another GPU: system scope)
        const bool sys = SYS || ph.in_ep == MEGA_EP_LINK;
        ulonglong2 w[K][2];
#pragma unroll
        for (int k = 0; k < K; k++) {
            const int t = t0 + k * stride;
            if (t < nq) {
                w[k][0] = ll_word2_rt(ph.x_ll + 4 * (size_t)t, sys);
                w[k][1] = ll_word2_rt(ph.x_ll + 4 * (size_t)t + 2, sys);
            }
        }
#pragma unroll
        for (int k = 0; k < K; k++) {
            const int t = t0 + k * stride;
            if (t < nq) {
                uint64_t tw = 0;
                for (unsigned it = 1; !ll_tags4(w[k], ein) && ll_keep_waiting(it, tw, a.status); it++) {
                    w[k][0] = ll_word2_rt(ph.x_ll + 4 * (size_t)t, sys);
                    w[k][1] = ll_word2_rt(ph.x_ll + 4 * (size_t)t + 2, sys);
                }
                v[k] = make_float4(__uint_as_float((unsigned)w[k][0].x), __uint_as_float((unsigned)w[k][0].y),
                                   __uint_as_float((unsigned)w[k][1].x), __uint_as_float((unsigned)w[k][1].y));
            }
        }
    } else {
#pragma unroll
        for (int k = 0; k < K; k++) {
            const int t = t0 + k * stride;
            if (t < nq) v[k] = __ldcg(reinterpret_cast<const float4 *>(ph.x) + t);
        }
    }
}

// A tagged word already loaded into w: re-polled until it carries epoch e.
template <bool SYS>
__device__ __forceinline__ float ll_settle(const unsigned long long *p, unsigned long long w, unsigned e, int *status)
{
    uint64_t t0 = 0;
    for (unsigned it = 1; (unsigned)(w >> 32) != e && ll_keep_waiting(it, t0, status); it++) w = ll_word<SYS>(p);
    return __uint_as_float((unsigned)w);
}

// ------------------------------------------------------------ smem layout --

struct MegaSmem {
    size_t ring, bars, abar, red, un, dsum, argsh, tab, total;
};

// One phase as the ring cursor sees it, 16 bytes: the weight pointer (0 for
// a phase without weight rows), row bytes (< 2^20) | rows per stage << 20,
// rows (< 2^17) | rows per CTA (< 2^15) << 17.
__host__ __device__ inline uint4 mega_tab_entry(const uint8_t *w, unsigned row_bytes, int sr, int n_out, int rpc)
{
    const unsigned long long pw = (unsigned long long)(uintptr_t)w;
    return make_uint4((unsigned)(pw & 0xFFFFFFFFull), (unsigned)(pw >> 32), row_bytes | ((unsigned)sr << 20),
                      (unsigned)n_out | ((unsigned)rpc << 17));
}

__host__ __device__ inline MegaSmem mega_smem_plan(int red_floats, unsigned ring_bytes, unsigned union_bytes,
                                                   int n_ph)
{
    MegaSmem p;
    p.ring = 0;
    p.bars = p.ring + (size_t)ring_bytes;
    p.abar = p.bars + MEGA_MAX_STAGES * sizeof(uint64_t);
    p.red = (p.abar + 8 * sizeof(uint64_t) + 15) & ~(size_t)15;    // K/V halves of 2 slots, partial gather
    p.un = (p.red + (size_t)red_floats * sizeof(float) + 127) & ~(size_t)127;
    // union: digit planes (and the RMSNorm staging) of a GEMV input | the
    // attention K/V buffers and split-partial gather
    p.dsum = p.un + (((size_t)union_bytes + 15) & ~(size_t)15);
    p.argsh = p.dsum + (RMS_MAX_W + 8) * sizeof(double);   // W terms + the total
    p.tab = (p.argsh + 32 * sizeof(ArgBest) + 15) & ~(size_t)15;
    p.total = p.tab + (size_t)n_ph * sizeof(uint4);
    return p;
}

// ---------------------------------------------------------------- digits ---

// The digit planes of make_digits, computed by 8 lanes per 32-element block:
// lane q of the group holds elements 4q..4q+3 (x4), which are word q of each
// plane in both the Q4_0 and the Q8_0 word order.  The block maximum is one
// 8-lane reduction of |x| as integer bits (for non-negative floats the bit
// order is the value order, and inf/NaN bits sort above every finite value),
// and frexpf/ldexpf are read off the exponent field: e = E - 126 for a normal
// amax with biased exponent E, e + 1 when its mantissa is >= 127/128 (amax >=
// 127.5 * 2^(e-7)), inv = 2^(7-e), sxs = 2^(e-21) -- the same values
// make_digits computes.  The Q4_0 code offsets are left to the consumer
// (digit_offsets).  All 32 lanes of the warp must call it.
__device__ __forceinline__ void digits_quad(float4 x4, int (&w)[3], float &sxs)
{
    unsigned ab = max(max(__float_as_uint(x4.x) & 0x7fffffffu, __float_as_uint(x4.y) & 0x7fffffffu),
                      max(__float_as_uint(x4.z) & 0x7fffffffu, __float_as_uint(x4.w) & 0x7fffffffu));
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) ab = max(ab, __shfl_xor_sync(0xffffffffu, ab, o));
    float inv = 0.0f;
    if (ab >= 0x7f800000u) {                         // inf or NaN in the block
        sxs = __int_as_float(0x7fc00000);
    } else if (__uint_as_float(ab) > 1e-30f) {
        int e = (int)(ab >> 23) - 126;
        if ((ab & 0x7fffffu) >= 0x7f0000u) e += 1;
        inv = __int_as_float((127 + 7 - e) << 23);
        sxs = __int_as_float((127 + e - 21) << 23);
    } else {
        sxs = 0.0f;
    }
    const float xv[4] = {x4.x, x4.y, x4.z, x4.w};
    uint32_t    b[3][4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float v  = __fmul_rn(xv[i], inv);
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
    for (int p = 0; p < 3; p++) w[p] = (int)pack_lo_bytes(b[p][0], b[p][1], b[p][2], b[p][3]);
}

// -8 * (sum of the block's digits of plane p): the Q4_0 code offset
// (codes are stored as c = q + 8), from the lane's own digit words.
__device__ __forceinline__ void digit_offsets(const int (&xw)[3][8], int (&off)[3])
{
#pragma unroll
    for (int p = 0; p < 3; p++) {
        int s = 0;
#pragma unroll
        for (int j = 0; j < 8; j++) s = __dp4a(xw[p][j], 0x01010101, s);
        off[p] = -8 * s;
    }
}

// The plain sums of the block's digits per plane (block_dot<12> multiplies
// them by the Q4_K sub-block minimum).
__device__ __forceinline__ void digit_sums(const int (&xw)[3][8], int (&off)[3])
{
#pragma unroll
    for (int p = 0; p < 3; p++) {
        int s = 0;
#pragma unroll
        for (int j = 0; j < 8; j++) s = __dp4a(xw[p][j], 0x01010101, s);
        off[p] = s;
    }
}

// ---------------------------------------------------------------- phases ---

// The ring's refill cursor: the next chunk to copy (phase, row offset) and
// how many chunks were issued; per slot, the warps done with it.
// A position in this CTA's list of weight chunks (phase order), with the
// current GEMV phase's rows cached so that moving on reads global memory
// only at a phase change.
struct ChunkCursor {
    int            p, i;
    const uint8_t *w;           // first row of this CTA in phase p
    unsigned       row_bytes;
    int            nrows, sr;
};

// The ring's cursors -- the next chunk to copy and, pf_stages chunks
// further on, the next chunk to warm in L2 -- the chunks issued, and per
// slot the warps done with it.
struct MegaRing {
    ChunkCursor cp, pf;
    int         issued;
    unsigned    done[MEGA_MAX_STAGES];
};

// The ring slot this CTA's consumers read next, and its barrier parity.
struct RingPos {
    int      slot;
    unsigned par;
};

struct MegaShared {
    int       pos;         // cache position of this step (read once at kernel start)
    unsigned  launch;      // launch number (epochs of the tagged vectors)
    uint8_t  *ring;
    MegaRing *rc;
    uint64_t *full, *abar;
    float    *red;
    int      *dig;
    float    *kvbuf;
    float    *cs;          // RoPE (cos, sin) row of the current position, staged a phase early
    uint64_t *dbar;        // completes when the next phase's descriptor has arrived
    double   *dsum;
    ArgBest  *argsh;
    const uint4 *tab;      // the phase table (shared memory)
    int       n_ph;
};

// Load phase p's geometry for this CTA into the ring cursor (from the
// shared-memory phase table: no global-memory round trip on the refill path).
__device__ __forceinline__ void cursor_load_phase(const MegaShared &S, ChunkCursor *c, int p)
{
    c->p = p;
    c->i = 0;
    c->nrows = 0;
    if (p >= S.n_ph) return;
    const uint4 t = S.tab[p];
    const uint8_t *w = reinterpret_cast<const uint8_t *>((uintptr_t)(((unsigned long long)t.y << 32) | t.x));
    if (!w) return;
    const int n_out = (int)(t.w & 0x1FFFFu), rpc = (int)(t.w >> 17);
    const int r0 = blockIdx.x * rpc;
    c->nrows = max(0, min(n_out, r0 + rpc) - r0);
    c->row_bytes = t.z & 0xFFFFFu;
    c->w = w + (size_t)r0 * c->row_bytes;
    c->sr = (int)(t.z >> 20);
}

// The chunk at the cursor (its first row, rows, row bytes), and advance it;
// false at the end of the list.
__device__ __forceinline__ bool cursor_next(const MegaShared &S, ChunkCursor *c, const uint8_t *&src, int &rows,
                                            unsigned &row_bytes)
{
    while (c->p < S.n_ph && c->i >= c->nrows) cursor_load_phase(S, c, c->p + 1);
    if (c->p >= S.n_ph) return false;
    rows = min(c->sr, c->nrows - c->i);
    row_bytes = c->row_bytes;
    src = c->w + (size_t)c->i * c->row_bytes;
    c->i += c->sr;
    return true;
}

// Copy the next chunk of this CTA's weight rows (phase order) into ring
// slot `slot`, and warm the chunk pf_stages further on in L2 (one thread;
// refills are serialised).
__device__ __forceinline__ void ring_issue(const MegaArgs &a, const MegaShared &S, int slot, bool warm = true)
{
    MegaRing      *rc = S.rc;
    const uint8_t *src;
    int            rows;
    unsigned       rb;
    if (!cursor_next(S, &rc->cp, src, rows, rb)) return;
    const uint32_t bytes = (uint32_t)rows * rb;
    mbar_expect_tx(&S.full[slot], bytes);
    bulk_g2s(S.ring + (size_t)slot * a.stage_bytes, src, bytes, &S.full[slot]);
    rc->issued++;
    if (warm && a.pf_stages > 0 && cursor_next(S, &rc->pf, src, rows, rb)) prefetch_l2(src, (uint32_t)rows * rb);
}

// Lane 0 of a warp that is done with ring slot `slot` (after __syncwarp).
// The arrivals count up forever; the warp whose arrival makes a multiple of
// MEGA_NCW is the last reader of this use of the slot and refills it.  Every
// arrival is a release; the refilling warp's acquire fence then orders every
// warp's reads of the slot (and the previous refill's cursor update) before
// the refill, and the proxy fence orders them before the bulk copy's writes.
// Refills happen in chunk order: the last release of slot s+1 comes after
// every warp's release of slot s.
__device__ __forceinline__ void ring_release(const MegaArgs &a, const MegaShared &S, int slot)
{
    unsigned old;
    asm volatile("atom.release.cta.shared::cta.add.u32 %0, [%1], 1;"
                 : "=r"(old)
                 : "r"(smem_addr(&S.rc->done[slot]))
                 : "memory");
    if ((old + 1) % MEGA_NCW == 0) {
        asm volatile("fence.acq_rel.cta;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        ring_issue(a, S, slot);
    }
}

// The first two levels of warp_sum4: lane l then holds the partial of row
// (l >> 3) & 3 over lanes {l, l^8, l^16, l^24}; the 8 partials of an 8-lane
// group added as ((p0+p4)+(p2+p6)) + ((p1+p5)+(p3+p7)) give the value
// warp_sum4 returns (its last three levels add in exactly that order).
__device__ __forceinline__ float warp_sum4_part(float v0, float v1, float v2, float v3, int lane)
{
    const bool up = lane & 16;
    float a0 = up ? v2 : v0, a1 = up ? v3 : v1;
    const float b0 = up ? v0 : v2, b1 = up ? v1 : v3;
    a0 += __shfl_xor_sync(0xffffffffu, b0, 16);
    a1 += __shfl_xor_sync(0xffffffffu, b1, 16);
    const bool mid = lane & 8;
    const float c = mid ? a1 : a0;
    const float dd = mid ? a0 : a1;
    return c + __shfl_xor_sync(0xffffffffu, dd, 8);
}

// The last two levels of warp_sum4 over the four pair sums q_j = p_j + p_{j+4}
// (j < 4) of an 8-lane group: ((p0+p4)+(p2+p6)) + ((p1+p5)+(p3+p7)), the
// value warp_sum4's last three levels give.
__device__ __forceinline__ float sum4_tree(const float *q)
{
    return (q[0] + q[2]) + (q[1] + q[3]);
}

// block_dot for four rows (row0 + k*stride) at once: all loads first, then
// the integer sums with each plane's low and high nibbles in separate chains
// (24 independent chains of 4 dp4a instead of 12 of 8).  Integer addition is
// exact, so every row gets block_dot's bits.
template <int FMT>
__device__ __forceinline__ void block_dot4(const uint8_t *row0, size_t stride, int nb, int b, const int (&xw)[3][8],
                                           const int (&off)[3], float sxs, float (&v)[4])
{
    if (FMT == 4) {
        uint4 q[4];
        float d[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            q[k] = *reinterpret_cast<const uint4 *>(row0 + k * stride + (size_t)b * 16);
            d[k] = __half2float(*reinterpret_cast<const __half *>(row0 + k * stride + (size_t)nb * 16 + 2 * b));
        }
        int acc[4][6];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            acc[k][0] = off[0]; acc[k][1] = off[1]; acc[k][2] = off[2];
            acc[k][3] = 0; acc[k][4] = 0; acc[k][5] = 0;
        }
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const uint32_t w = j == 0 ? q[k].x : j == 1 ? q[k].y : j == 2 ? q[k].z : q[k].w;
                const int lo = (int)(w & 0x0F0F0F0Fu), hi = (int)((w >> 4) & 0x0F0F0F0Fu);
                acc[k][0] = __dp4a(lo, xw[0][j], acc[k][0]);
                acc[k][3] = __dp4a(hi, xw[0][4 + j], acc[k][3]);
                acc[k][1] = __dp4a(lo, xw[1][j], acc[k][1]);
                acc[k][4] = __dp4a(hi, xw[1][4 + j], acc[k][4]);
                acc[k][2] = __dp4a(lo, xw[2][j], acc[k][2]);
                acc[k][5] = __dp4a(hi, xw[2][4 + j], acc[k][5]);
            }
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int t = (acc[k][0] + acc[k][3]) * 16384 + (acc[k][1] + acc[k][4]) * 128 + (acc[k][2] + acc[k][5]);
            v[k] = (float)t * (d[k] * sxs);
        }
    } else if (FMT == 12) {
        // Q4_K (SPLITK4): the same split chains on plain codes (off holds the
        // digit sums), then each row's sub-block scale and minimum
        uint4 q[4], hd[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            q[k] = *reinterpret_cast<const uint4 *>(row0 + k * stride + (size_t)b * 16);
            hd[k] = *reinterpret_cast<const uint4 *>(row0 + k * stride + (size_t)nb * 16 + (size_t)(b >> 3) * 16);
        }
        int acc[4][6];
#pragma unroll
        for (int k = 0; k < 4; k++)
#pragma unroll
            for (int i = 0; i < 6; i++) acc[k][i] = 0;
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const uint32_t w = j == 0 ? q[k].x : j == 1 ? q[k].y : j == 2 ? q[k].z : q[k].w;
                const int lo = (int)(w & 0x0F0F0F0Fu), hi = (int)((w >> 4) & 0x0F0F0F0Fu);
                acc[k][0] = __dp4a(lo, xw[0][j], acc[k][0]);
                acc[k][3] = __dp4a(hi, xw[0][4 + j], acc[k][3]);
                acc[k][1] = __dp4a(lo, xw[1][j], acc[k][1]);
                acc[k][4] = __dp4a(hi, xw[1][4 + j], acc[k][4]);
                acc[k][2] = __dp4a(lo, xw[2][j], acc[k][2]);
                acc[k][5] = __dp4a(hi, xw[2][4 + j], acc[k][5]);
            }
        const int sx = off[0] * 16384 + off[1] * 128 + off[2];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int t = (acc[k][0] + acc[k][3]) * 16384 + (acc[k][1] + acc[k][4]) * 128 + (acc[k][2] + acc[k][5]);
            float dl, ml;
            k4_scale_min(hd[k], b & 7, dl, ml);
            v[k] = k4_finish(t, sx, dl, ml, sxs);
        }
    } else {
#pragma unroll
        for (int k = 0; k < 4; k++) v[k] = block_dot<FMT>(row0 + k * stride, nb, b, xw, off, sxs);
    }
}

// Rows [0, rows) of one ring stage against this lane's block column: warp
// (g, rp) takes rows rp, rp + rowpar, ... four at a time.  Row partials of
// k-group g land in red[row * nkg + g], or with RED4 (the last two levels of
// the warp reduction left to the epilogue's sum4_tree) in
// red[row * (4 * nkg + 1) + 4 * g + lane % 4]: the odd row stride keeps the
// epilogue, one thread per row, free of bank conflicts.
template <int FMT, bool RED4>
__device__ __forceinline__ void mega_stage_rows(const uint8_t *stage, int rows, unsigned row_bytes, int nb,
                                                int b, int g, int rp, int rowpar, int nkg, int lane,
                                                const int (&xw)[3][8], const int (&off)[3], float sxs,
                                                float *red)
{
    static_assert(FAST_RB == 4, "four rows per warp batch");
    for (int i0 = rp; i0 < rows; i0 += FAST_RB * rowpar) {
        float v[FAST_RB];
        if (i0 + (FAST_RB - 1) * rowpar < rows) {
            block_dot4<FMT>(stage + (size_t)i0 * row_bytes, (size_t)rowpar * row_bytes, nb, b, xw, off, sxs, v);
        } else {
#pragma unroll
            for (int k = 0; k < FAST_RB; k++) {
                const int ii = i0 + k * rowpar;
                v[k] = ii < rows ? block_dot<FMT>(stage + (size_t)ii * row_bytes, nb, b, xw, off, sxs) : 0.0f;
            }
        }
        const int k = (lane >> 3) & 3, ii = i0 + k * rowpar;
        if (RED4) {
            const float part = warp_sum4_part(v[0], v[1], v[2], v[3], lane);
            const float pair = part + __shfl_xor_sync(0xffffffffu, part, 4);
            if (ii < rows && (lane & 4) == 0) red[ii * (4 * nkg + 1) + 4 * g + (lane & 3)] = pair;
        } else {
            const float sum = warp_sum4(v[0], v[1], v[2], v[3], lane);
            if ((lane & 7) == 0 && ii < rows) red[ii * nkg + g] = sum;
        }
    }
}

// Sum of row r's k-group partials, in k-group order.
__device__ __forceinline__ float row_total(const float *red, int r, int nkg, bool red4)
{
    float acc = 0.0f;
    if (red4)
        for (int q = 0; q < nkg; q++) acc += sum4_tree(red + (size_t)r * (4 * nkg + 1) + 4 * q);
    else
        for (int q = 0; q < nkg; q++) acc += red[r * nkg + q];
    return acc;
}

// Digit planes of the digit store for the input block of 8 lanes (t = b*8 + q).
__device__ __forceinline__ void store_digits(const MegaShared &S, int t, float4 v)
{
    int   w[3];
    float sxs;
    digits_quad(v, w, sxs);
    const int b = t >> 3, q = t & 7;
    int *d = S.dig + (size_t)b * 28;
    d[q] = w[0];
    d[8 + q] = w[1];
    d[16 + q] = w[2];
    if (q == 0) d[27] = __float_as_int(sxs);
}

__device__ __forceinline__ void attn_prefetch(const MegaArgs &a, const MegaPhase &ph, int pos, int hd);

// This CTA's attention item: KV head g, position split sp, positions
// [t0, t1) below or at pos, in rounds of 2 * att_sub positions.
struct AttItem {
    bool has;
    int  g, sp, t0, t1, nround;
};

__device__ __forceinline__ AttItem att_item(const MegaArgs &a, int pos)
{
    AttItem it;
    const int item = blockIdx.x;
    it.has = item < a.n_kv * a.n_split;
    it.g = it.has ? item / a.n_split : 0;
    it.sp = it.has ? item % a.n_split : 0;
    const int npos = pos + 1, chunk = (npos + a.n_split - 1) / a.n_split;
    it.t0 = min(npos, it.sp * chunk);
    it.t1 = it.has ? min(npos, it.t0 + chunk) : it.t0;
    it.nround = (it.t1 - it.t0 + 2 * a.att_sub - 1) / (2 * a.att_sub);
    return it;
}

// Half hf (att_sub rows) of round r of the item's K/V rows below the
// current position (contiguous in the head-major cache) into slot r % nsl:
// one bulk copy for K, one for V, completing on abar[slot * 2 + hf].  The
// proxy fence orders earlier generic accesses of those bytes before the
// copy's writes.
template <int HD>
__device__ __forceinline__ void att_issue(const MegaArgs &a, const MegaShared &S, const float *kc, const float *vc,
                                          const AttItem &it, int pos, int r, int hf)
{
    const int sub = a.att_sub, nsl = a.att_nsl, s_ = r % nsl;
    const int c0 = it.t0 + r * 2 * sub + hf * sub;
    const int c1 = min(min(it.t1, c0 + sub), pos);
    const int nr = c1 > c0 ? c1 - c0 : 0;
    const uint32_t bytes = (uint32_t)(nr * HD * sizeof(float));
    uint64_t *bar = &S.abar[s_ * 2 + hf];
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_expect_tx(bar, 2 * bytes);
    if (nr > 0) {
        const size_t base = (size_t)it.g * a.n_ctx * HD + (size_t)c0 * HD;
        bulk_g2s(S.kvbuf + (size_t)((s_ * 2 + 0) * 2 + hf) * sub * HD, kc + base, bytes, bar);
        bulk_g2s(S.kvbuf + (size_t)((s_ * 2 + 1) * 2 + hf) * sub * HD, vc + base, bytes, bar);
    }
}

// One GEMV phase on the consumer side: digit planes of the (normed) input
// into shared memory, this CTA's ring stages of the matrix (rp_: the next
// slot to read, carried over the whole step), the epilogue.  One body for
// both row formats: only the innermost loop depends on it.
// next: the following phase's descriptor when it is attention (its K/V rows
// are warmed in L2 and the RoPE row staged once the main loop is done).
template <bool SYS>
__device__ void mega_gemv(const MegaArgs &a, const MegaPhase &ph, const MegaShared &S, RingPos &rp_, int p_idx,
                          const MegaPhase *next, int hd)
{
    unsigned long long *det = (a.phase_detail && blockIdx.x == 0 && threadIdx.x == 0)
                                  ? a.phase_detail + (size_t)p_idx * 4 : nullptr;
    unsigned long long waited = 0;
    const bool q4 = ph.fmt == 4, k4 = ph.fmt == 12, red4 = q4 && ph.red4;
    const int nct = MEGA_NCW * 32, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nkg = ph.nkg, rowpar = ph.rowpar, nb = ph.n_in / 32;
    const int r0 = blockIdx.x * ph.rpc;
    const int nrows = max(0, min(ph.n_out, r0 + ph.rpc) - r0);
    const unsigned row_bytes = ph.row_bytes;
    const int epi = ph.epi;

    // the residual this CTA's rows add to (its own rows: no other CTA writes
    // them in this phase; nrows <= MEGA_THREADS for EPI_ADD): requested now,
    // settled after the prologue
    const bool has_res = epi == EPI_ADD && tid < nrows;
    // the RoPE row the next phase (attention) needs, requested now so that
    // its latency hides behind this phase (hd <= MEGA_THREADS)
    float cs_next = 0.0f;
    if (ph.next_attn && tid < hd) cs_next = __ldg(a.rope_cs + (size_t)S.pos * hd + tid);
    // the next attention's K/V rows into L2 while this phase streams its
    // weights (this phase's kc / vc are the next attention's cache planes)
    if (ph.next_attn && a.att_l2 == 2 && tid == 0) attn_prefetch(a, ph, S.pos, hd);
    unsigned long long yw = 0;
    if (has_res && ph.y_ep >= 0) yw = ll_word<SYS>(a.x_ll + ph.out_base + r0 + tid);
    if (has_res && ph.y_ep == MEGA_EP_LINK) yw = ll_word<true>(a.x_ll + r0 + tid);
    // the next attention's first K/V rounds (rows of earlier positions: no
    // dependence on this step) start streaming into their buffers now, above
    // this phase's digit planes
    if (ph.next_attn && a.att_early && (tid & 31) == 0 && tid < 64) {
        const AttItem it = att_item(a, S.pos);
        for (int r = 0; r < min(a.att_nsl, it.nround); r++)
            if (hd == 128) att_issue<128>(a, S, ph.kc, ph.vc, it, S.pos, r, tid >> 5);
            else att_issue<64>(a, S, ph.kc, ph.vc, it, S.pos, r, tid >> 5);
    }

    // ---- prologue: this warp's share of its k-group's input -------------------
    // k-group g (inputs [1024 g, 1024 g + 1024): 32 blocks, 8 passes of four
    // blocks) is prepared by its rowpar warps: warp rp takes passes rp,
    // rp + rowpar, ...  A pass is one float4 a lane (lane q of an 8-lane
    // group holds elements 4q..4q+3 of one block): the warp waits only for
    // those tagged words, adds their squares into one W term of the RMSNorm
    // sum (128 inputs; rms_scale's order) and stores the digit planes of x
    // (times the norm weights) in shared memory.  The group's warps then
    // meet at the group's own named barrier, so no warp waits for another
    // k-group's input; the RMSNorm scale, which needs every W term,
    // multiplies the row sums in the epilogue.
    // A CTA without rows reads no input: nothing it writes would tell a later
    // phase that it is done with the vector (the tagged vectors are reused
    // one layer later, ordered only by what each phase reads).
    // (an injected stall: the epoch of phase -1 of the next launch, which no
    // word carries)
    const unsigned ein = p_idx == a.stall_phase         ? ll_epoch(S.launch + 1u, -1)
                         : ph.in_ep == MEGA_EP_LINK      ? link_epoch(S.pos)
                                                         : ll_epoch(S.launch, ph.in_ep);
    const bool active = nrows > 0 && warp < nkg * rowpar;
    const int  g = active ? warp % nkg : 0, rp = active ? warp / nkg : 0;
    if (active) {
        const int     tg = g * 256 + lane;               // the group's first float4, this lane
        const float4 *w4 = reinterpret_cast<const float4 *>(ph.norm_w);
        for (int k0 = rp; k0 < 8; k0 += 2 * rowpar) {
            float4 v[2], wv[2];
            if (ph.norm)
#pragma unroll
                for (int k = 0; k < 2; k++)
                    if (k0 + k * rowpar < 8) wv[k] = __ldg(w4 + tg + 32 * (k0 + k * rowpar));
            input_batch<2, SYS>(a, ph, tg + 32 * k0, 32 * rowpar, g * 256 + 256, ein, v);
#pragma unroll
            for (int k = 0; k < 2; k++) {
                const int kk = k0 + k * rowpar;
                if (kk < 8) {
                    const int t = tg + 32 * kk;
                    float4    x4 = v[k];
                    if (ph.norm) {
                        const double sq = rms_bfly32(rms_sq4(x4));
                        if (lane == 0) S.dsum[t >> 5] = sq;
                        x4.x = __fmul_rn(x4.x, wv[k].x);
                        x4.y = __fmul_rn(x4.y, wv[k].y);
                        x4.z = __fmul_rn(x4.z, wv[k].z);
                        x4.w = __fmul_rn(x4.w, wv[k].w);
                    }
                    store_digits(S, t, x4);
                }
            }
        }
        if (rowpar > 1) named_bar(2 + g, 32 * rowpar);
        else __syncwarp();
    }
    float yprev = 0.0f;
    if (has_res)
        yprev = ph.y_ep >= 0 ? ll_settle<SYS>(a.x_ll + ph.out_base + r0 + tid, yw, ll_epoch(S.launch, ph.y_ep), a.status)
                : ph.y_ep == MEGA_EP_LINK ? ll_settle<true>(a.x_ll + r0 + tid, yw, link_epoch(S.pos), a.status)
                                          : __ldcg(ph.y + r0 + tid);

    if (det) det[0] = clock64();
    // ---- main loop ------------------------------------------------------------
    const int  b = g * 32 + lane;
    int   xw[3][8], off[3];
    float sxs = 0.0f;
    if (active) {
        const int4 *d4 = reinterpret_cast<const int4 *>(S.dig + (size_t)b * 28);
#pragma unroll
        for (int p = 0; p < 3; p++) {
            const int4 u = d4[2 * p], v = d4[2 * p + 1];
            xw[p][0] = u.x; xw[p][1] = u.y; xw[p][2] = u.z; xw[p][3] = u.w;
            xw[p][4] = v.x; xw[p][5] = v.y; xw[p][6] = v.z; xw[p][7] = v.w;
        }
        sxs = __int_as_float(S.dig[(size_t)b * 28 + 27]);
        if (q4) digit_offsets(xw, off);
        else if (k4) digit_sums(xw, off);
        else off[0] = off[1] = off[2] = 0;
    }
    const int sr = ph.sr;
    for (int i = 0; i < nrows; i += sr) {
        const int      slot = rp_.slot;
        const unsigned par = rp_.par;
        if (det && !mbar_test(&S.full[slot], par)) {
            const unsigned long long t0 = globaltimer_ns();
            mbar_wait<true>(&S.full[slot], par, a.status);
            waited += globaltimer_ns() - t0;
        } else {
            mbar_wait<true>(&S.full[slot], par, a.status);
        }
        const uint8_t *stage = S.ring + (size_t)slot * a.stage_bytes;
        const int      rows = min(sr, nrows - i);
        if (active) {
            if (q4 && red4)
                mega_stage_rows<4, true>(stage, rows, row_bytes, nb, b, g, rp, rowpar, nkg, lane, xw, off, sxs,
                                         S.red + (size_t)i * (4 * nkg + 1));
            else if (q4)
                mega_stage_rows<4, false>(stage, rows, row_bytes, nb, b, g, rp, rowpar, nkg, lane, xw, off, sxs,
                                          S.red + (size_t)i * nkg);
            else if (k4)
                mega_stage_rows<12, false>(stage, rows, row_bytes, nb, b, g, rp, rowpar, nkg, lane, xw, off, sxs,
                                           S.red + (size_t)i * nkg);
            else
                mega_stage_rows<8, false>(stage, rows, row_bytes, nb, b, g, rp, rowpar, nkg, lane, xw, off, sxs,
                                          S.red + (size_t)i * nkg);
        }
        __syncwarp();
        if (lane == 0) ring_release(a, S, slot);
        if (++rp_.slot == a.nst) {
            rp_.slot = 0;
            rp_.par ^= 1u;
        }
    }
    // the digit planes share bytes with the attention K/V buffers, which bulk
    // copies (the async proxy) fill later: order these generic accesses first
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    named_bar(1, nct);
    if (det) {
        det[1] = clock64();
        det[3] = waited;
    }
    if (next) {
        // next phase's descriptor: its copy was issued at this phase's start
        mbar_wait<true>(S.dbar, (unsigned)p_idx & 1u, a.status);
        if (tid == 0 && a.att_l2 == 1) attn_prefetch(a, *next, S.pos, hd);
        if (tid < hd) S.cs[tid] = cs_next;
    }

    // ---- epilogue over this CTA's rows --------------------------------------
    float         *y = ph.y;
    const unsigned eout = ll_epoch(S.launch, p_idx);
    // the RMSNorm scale: every warp adds the W terms in rms_scale's order
    // (the same bits in every warp, so no further barrier)
    float rscale = 1.0f;
    if (ph.norm && nrows > 0) rscale = rms_from_sum(rms_total_w(S.dsum, nkg * 8, lane), ph.n_in, a.eps);
    if (epi == EPI_SWIGLU) {
        for (int j = tid; j < nrows / 2; j += nct) {
            float gs = row_total(S.red, 2 * j, nkg, red4), us = row_total(S.red, 2 * j + 1, nkg, red4);
            if (ph.norm) {
                gs = __fmul_rn(gs, rscale);
                us = __fmul_rn(us, rscale);
            }
            ll_put_out<SYS>(a, ph.bcast, ph.y_ll + ph.out_base + r0 / 2 + j, silu_mul(gs, us), eout);
        }
        if (det) det[2] = clock64();
        return;
    }
    if (ph.xn && ph.norm && blockIdx.x == 0 && nrows > 0) {
        // the normed input the stage outputs, (x * scale) * w with the
        // reference's two roundings (src/engine.c:261); the tagged words
        // already carry the epoch (this CTA read them all in the prologue)
        const float4 *w4 = reinterpret_cast<const float4 *>(ph.norm_w);
        float4       *xn4 = reinterpret_cast<float4 *>(ph.xn);
        for (int t = tid; t < nb * 8; t += nct) {
            float4 v[1];
            input_batch<1, SYS>(a, ph, t, 0, nb * 8, ein, v);
            const float4 w = __ldg(w4 + t);
            xn4[t] = make_float4(__fmul_rn(__fmul_rn(v[0].x, rscale), w.x), __fmul_rn(__fmul_rn(v[0].y, rscale), w.y),
                                 __fmul_rn(__fmul_rn(v[0].z, rscale), w.z), __fmul_rn(__fmul_rn(v[0].w, rscale), w.w));
        }
    }
    ArgBest best{-INFINITY, -1};
    for (int r = tid; r < nrows; r += nct) {
        float acc = row_total(S.red, r, nkg, red4);
        if (ph.norm) acc = __fmul_rn(acc, rscale);
        if (epi == EPI_ADD) {
            const float out = yprev + acc;         // r == tid: nrows <= MEGA_THREADS
            ll_put_out<SYS>(a, ph.bcast, ph.y_ll + ph.out_base + r0 + r, out, eout);
            if (ph.out_plain) {
                y[r0 + r] = out;
                // the stage's output state, also into the next stage's input
                if (a.link_x) ll_put<true>(a.link_x + r0 + r, out, link_epoch(S.pos));
            }
        } else if (epi == EPI_STORE) {
            ll_put_out<SYS>(a, ph.bcast, ph.y_ll + ph.out_base + r0 + r, acc, eout);
        } else {
            y[r0 + r] = acc;                       // logits (argmax reads them after its ticket)
        }
        if (epi == EPI_ARGMAX) best = arg_better(best, ArgBest{acc, r0 + r});
    }
    if (det) det[2] = clock64();
    if (epi != EPI_ARGMAX) return;
    // per-CTA best -> the CTA that takes the last ticket reduces in CTA order
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ArgBest other;
        other.v = __shfl_xor_sync(0xffffffffu, best.v, o);
        other.i = __shfl_xor_sync(0xffffffffu, best.i, o);
        best = arg_better(best, other);
    }
    if (lane == 0) S.argsh[warp] = best;
    named_bar(1, nct);
    __shared__ unsigned s_last;
    if (tid == 0) {
        ArgBest bb = S.argsh[0];
        for (int w = 1; w < MEGA_NCW; w++) bb = arg_better(bb, S.argsh[w]);
        a.part_val[blockIdx.x] = bb.v;
        a.part_idx[blockIdx.x] = bb.i;
        __threadfence();
        s_last = atomicAdd(a.ticket, 1u) == gridDim.x - 1;
    }
    named_bar(1, nct);
    if (!s_last) return;
    __threadfence();
    // every CTA is past its prologue: the normed state may replace the
    // residual stream (the stage's output, src/engine.c:489)
    if (a.xn_tmp)
        for (int i = tid; i < a.n_embd; i += nct) a.state[i] = __ldcg(a.xn_tmp + i);
    if (tid == 0) {
        ArgBest bb{-INFINITY, -1};
        for (unsigned c = 0; c < gridDim.x; c++)
            bb = arg_better(bb, ArgBest{__ldcg(a.part_val + c), __ldcg(a.part_idx + c)});
        if (bb.i >= 0) bb.i += a.vocab_base;
        // a NaN first logit selects token 0 (the reference's rule): as an
        // infinite logit at index 0 it wins every comparison below
        if (a.tp_rank == 0 && isnan(__ldcg(y))) bb = ArgBest{INFINITY, 0};
        if (a.tp_world > 1) {
            // every rank's best to every rank, combined in rank order: all
            // ranks pick the same token
            const unsigned e = ll_epoch(S.launch, p_idx);
            const size_t   off = (size_t)(a.arg_ll - a.ll_block) + 2 * (size_t)a.tp_rank;
            for (int k = 0; k < a.tp_world; k++) {
                ll_put<SYS>(a.peer[k] + off, bb.v, e);
                ll_put<SYS>(a.peer[k] + off + 1, __int_as_float(bb.i), e);
            }
            ArgBest all{-INFINITY, -1};
            for (int k = 0; k < a.tp_world; k++)
                all = arg_better(all, ArgBest{ll_get<SYS>(a.arg_ll + 2 * k, e, a.status),
                                              __float_as_int(ll_get<SYS>(a.arg_ll + 2 * k + 1, e, a.status))});
            bb = all;
        }
        const int tok = bb.i < 0 ? 0 : bb.i;
        const int   pos = S.pos;
        if (a.tok_hist) a.tok_hist[pos] = tok;
        a.st->token = tok;
        // the first stage's next input (position pos + 1) on its GPU
        if (a.link_tok) ll_put<true>(a.link_tok, __int_as_float(tok), link_epoch(pos + 1));
        if (a.advance_pos) a.st->pos = pos + 1;
        a.state[a.n_embd] = (float)tok;
        *a.ticket = 0u;
    }
}

// Attention work item (KV head g, position split sp) = this CTA's index;
// query head h of the group on warp h.  Same arithmetic per split as
// k_attention; partials go to global memory for the merge phase.
template <int HD, int NREP, bool SYS>
__device__ void mega_attention(const MegaArgs &a, const MegaPhase &ph, const MegaShared &S, int &att_sb0,
                               int &att_sb1, int &merges, int p_idx)
{
    // profiling (CTA 0): after the Q/K/V prologue, after the position loop,
    // after the split ticket; and when KV head 0's merge ended
    unsigned long long *det = (a.phase_detail && blockIdx.x == 0 && threadIdx.x == 0)
                                  ? a.phase_detail + (size_t)p_idx * 4 : nullptr;
    // K/V rows sit unpadded in shared memory (one bulk copy per sub-chunk
    // and matrix); the score loop reads a row's float4 columns in an order
    // rotated by the lane, so the 32 lanes' rows still spread over the banks
    constexpr int RS = HD;
    constexpr int NC4 = HD / 4;
    static_assert((NC4 & (NC4 - 1)) == 0, "head_dim / 4 a power of two");
    __shared__ __align__(16) float q_s[NREP * HD];
    __shared__ __align__(16) float knew[HD], vnew[HD];
    const int nct = MEGA_NCW * 32, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const AttItem it = att_item(a, S.pos);
    const bool has = it.has;
    const int g = it.g, sp = it.sp, t0 = it.t0, t1 = it.t1, nround = it.nround;
    const int pos = S.pos;
    const int sub = a.att_sub, nsl = a.att_nsl;
    float *kbase = ph.kc + (size_t)g * a.n_ctx * HD;
    float *vbase = ph.vc + (size_t)g * a.n_ctx * HD;
    // buffer (slot s, matrix m: 0 = K, 1 = V, half hf) of sub rows
    auto buf = [&](int s_, int m, int hf) { return S.kvbuf + (size_t)((s_ * 2 + m) * 2 + hf) * sub * RS; };
    // the first nsl rounds' copies: issued by the Q/K/V phase (att_early),
    // else now; a slot is refilled after the barrier that ends the round
    // which read it
    if (!a.att_early && (tid & 31) == 0 && tid < 64)
        for (int r = 0; r < min(nsl, nround); r++) att_issue<HD>(a, S, ph.kc, ph.vc, it, pos, r, tid >> 5);
    const float *cs_s = S.cs;
    const unsigned ein = ll_epoch(S.launch, ph.in_ep);
    const int qdim = a.n_head * HD, kvdim = a.n_kv * HD;
    // a CTA without a work item reads nothing (see the GEMV prologue).
    // Items [0, NREP*HD/2): a query (head, rotation pair); then HD/2 K/V
    // pairs; each thread's words are all requested before it waits on one
    constexpr int NQP = NREP * (HD / 2);
    for (int i = has ? tid : nct; i < NQP + HD / 2; i += nct) {
        if (i < NQP) {
            const int h = i / (HD / 2), j = i % (HD / 2), row = (g * NREP + h) * HD;
            const unsigned long long *p0 = a.qkv_ll + row + j, *p1 = p0 + HD / 2;
            const unsigned long long w0 = ll_word<SYS>(p0), w1 = ll_word<SYS>(p1);
            float x0 = ll_settle<SYS>(p0, w0, ein, a.status), x1 = ll_settle<SYS>(p1, w1, ein, a.status);
            if (ph.bq) { x0 = __fadd_rn(x0, ph.bq[row + j]); x1 = __fadd_rn(x1, ph.bq[row + j + HD / 2]); }
            rope_pair(x0, x1, cs_s[2 * j], cs_s[2 * j + 1]);
            q_s[h * HD + j] = x0;
            q_s[h * HD + j + HD / 2] = x1;
        } else {
            const int j = i - NQP, kr = qdim + g * HD, vr = qdim + kvdim + g * HD;
            const unsigned long long *pk0 = a.qkv_ll + kr + j, *pk1 = pk0 + HD / 2;
            const unsigned long long *pv0 = a.qkv_ll + vr + j, *pv1 = pv0 + HD / 2;
            const unsigned long long wk0 = ll_word<SYS>(pk0), wk1 = ll_word<SYS>(pk1), wv0 = ll_word<SYS>(pv0),
                                     wv1 = ll_word<SYS>(pv1);
            float k0 = ll_settle<SYS>(pk0, wk0, ein, a.status), k1 = ll_settle<SYS>(pk1, wk1, ein, a.status);
            float v0 = ll_settle<SYS>(pv0, wv0, ein, a.status), v1 = ll_settle<SYS>(pv1, wv1, ein, a.status);
            if (ph.bk) { k0 = __fadd_rn(k0, ph.bk[g * HD + j]); k1 = __fadd_rn(k1, ph.bk[g * HD + j + HD / 2]); }
            if (ph.bv) { v0 = __fadd_rn(v0, ph.bv[g * HD + j]); v1 = __fadd_rn(v1, ph.bv[g * HD + j + HD / 2]); }
            rope_pair(k0, k1, cs_s[2 * j], cs_s[2 * j + 1]);
            knew[j] = k0; knew[j + HD / 2] = k1;
            vnew[j] = v0; vnew[j + HD / 2] = v1;
        }
    }
    named_bar(1, nct);
    if (det) det[0] = clock64();
    if (has && sp == 0)
        for (int j = tid; j < HD; j += nct) {
            kbase[(size_t)pos * HD + j] = knew[j];
            vbase[(size_t)pos * HD + j] = vnew[j];
        }
    // Each round (2*sub positions) in three steps, every K and V row read
    // from shared memory once for all NREP query heads of the KV head:
    //  scores: 8 threads per position, thread ds holding float4 columns ds,
    //          ds+8, ... (8 distinct bank quads per wavefront) against the
    //          NREP queries (broadcast reads), the 8 slices added by a
    //          butterfly; sc[h][p] = dot * kscale (-inf past the slice);
    //  softmax: warp h takes head h's positions, a running max over rounds:
    //          f = exp(m_old - m_new), e = exp(s - m_new), l = l*f + sum e;
    //  values: thread (float4 column c, position group pg) rescales its NREP
    //          accumulators by f and adds e[h][p] * V[p][c] over its group's
    //          positions.
    // After the last round the position groups' accumulators are added in
    // group order through shared memory into the split's partial.
    constexpr int C4 = HD / 4, PG = MEGA_THREADS / C4, NSL8 = 8;
    static_assert(C4 % NSL8 == 0 && NREP <= 8 && NREP <= MEGA_NCW, "attention thread layout");
    const int P = 2 * sub;                                 // <= 64: 8 threads a position cover 512
    float *sc = S.red;                                     // [NREP][64] scores
    float *es = sc + NREP * 64;                            // [64][NREP] weights
    float *fs = es + 64 * NREP;                            // [NREP] rescale factors
    float  m_run = -INFINITY, l_run = 0.0f;                // warp h < NREP: head h's
    float4 acc[NREP];
#pragma unroll
    for (int hh = 0; hh < NREP; hh++) acc[hh] = make_float4(0.f, 0.f, 0.f, 0.f);
    const int qp = tid >> 3, ds = tid & 7;                 // scores: position, column slice
    const int vc = tid % C4, pg = tid / C4;                // values: float4 column, position group
    for (int r = 0; r < nround; r++) {
        const int s_ = r % nsl, cb = t0 + r * P;           // this round's first position
        const int cn = min(P, t1 - cb);
        const unsigned par = (unsigned)((s_ ? att_sb1 : att_sb0) + r / nsl) & 1u;
        mbar_wait<true>(&S.abar[s_ * 2], par, a.status);
        if (cn > sub) mbar_wait<true>(&S.abar[s_ * 2 + 1], par, a.status);
        // ---- scores
        if (qp < P) {
            float d[NREP];
#pragma unroll
            for (int hh = 0; hh < NREP; hh++) d[hh] = 0.0f;
            if (qp < cn) {
                const float4 *k4 = (cb + qp == pos) ? reinterpret_cast<const float4 *>(knew)
                                                   : reinterpret_cast<const float4 *>(buf(s_, 0, qp / sub) +
                                                                                      (size_t)(qp % sub) * RS);
#pragma unroll 1
                for (int jj = 0; jj < C4 / NSL8; jj++) {
                    const int    j = ds + NSL8 * jj;
                    const float4 kv = k4[j];
#pragma unroll
                    for (int hh = 0; hh < NREP; hh++) {
                        const float4 qv = reinterpret_cast<const float4 *>(q_s + hh * HD)[j];
                        d[hh] = fmaf(qv.x, kv.x, fmaf(qv.y, kv.y, fmaf(qv.z, kv.z, fmaf(qv.w, kv.w, d[hh]))));
                    }
                }
            }
#pragma unroll
            for (int o = 1; o < NSL8; o <<= 1)
#pragma unroll
                for (int hh = 0; hh < NREP; hh++) d[hh] += __shfl_xor_sync(0xffffffffu, d[hh], o);
#pragma unroll
            for (int hh = 0; hh < NREP; hh++)
                if (ds == hh) sc[hh * 64 + qp] = qp < cn ? d[hh] * a.kscale : -INFINITY;
        }
        named_bar(1, nct);
        // ---- softmax (running max over the rounds)
        if (warp < NREP) {
            const float s0 = lane < P ? sc[warp * 64 + lane] : -INFINITY;
            const float s1 = lane + 32 < P ? sc[warp * 64 + lane + 32] : -INFINITY;
            const float mnew = fmaxf(m_run, warp_max(fmaxf(s0, s1)));
            const float f = expf(m_run - mnew);
            const float e0 = s0 == -INFINITY ? 0.0f : expf(s0 - mnew);
            const float e1 = s1 == -INFINITY ? 0.0f : expf(s1 - mnew);
            if (lane < P) es[lane * NREP + warp] = e0;
            if (lane + 32 < P) es[(lane + 32) * NREP + warp] = e1;
            l_run = l_run * f + warp_sum(e0 + e1);
            m_run = mnew;
            if (lane == 0) fs[warp] = f;
        }
        named_bar(1, nct);
        // ---- values
        {
#pragma unroll
            for (int hh = 0; hh < NREP; hh++) {
                const float f = fs[hh];
                acc[hh].x *= f; acc[hh].y *= f; acc[hh].z *= f; acc[hh].w *= f;
            }
            for (int pp = pg; pp < cn; pp += PG) {
                const float4 vv = (cb + pp == pos) ? reinterpret_cast<const float4 *>(vnew)[vc]
                                                   : reinterpret_cast<const float4 *>(buf(s_, 1, pp / sub) +
                                                                                      (size_t)(pp % sub) * RS)[vc];
                const float *ep = es + pp * NREP;
#pragma unroll
                for (int hh = 0; hh < NREP; hh++) {
                    const float e = ep[hh];
                    acc[hh].x = fmaf(e, vv.x, acc[hh].x);
                    acc[hh].y = fmaf(e, vv.y, acc[hh].y);
                    acc[hh].z = fmaf(e, vv.z, acc[hh].z);
                    acc[hh].w = fmaf(e, vv.w, acc[hh].w);
                }
            }
        }
        named_bar(1, nct);                          // both halves of slot s_ are free
        if (r + nsl < nround && (tid & 31) == 0 && tid < 64) att_issue<HD>(a, S, ph.kc, ph.vc, it, pos, r + nsl, tid >> 5);
    }
    // one phase of each of a slot's half barriers per round that used it
    // (a round with at most sub positions still completes both halves: its
    // second half's copy is empty)
    att_sb0 += (nround + nsl - 1) / nsl;
    att_sb1 += nsl > 1 ? nround / nsl : 0;
    if (det) det[1] = clock64();
    // the position groups' accumulators into the K/V buffers (free now: every
    // round's copies have landed), added in group order into this split's
    // partial, published as tagged words: per query head the HD unnormalised
    // sums, the running max and the weight sum
    const unsigned eout = ll_epoch(S.launch, p_idx);
    constexpr int  PW = HD + 2;                       // words of one head's partial
    const int      ns = a.n_split;
    {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        float4 *gsum = reinterpret_cast<float4 *>(S.dig);    // [PG][NREP][C4], the union's base
#pragma unroll
        for (int hh = 0; hh < NREP; hh++) gsum[((size_t)pg * NREP + hh) * C4 + vc] = acc[hh];
        named_bar(1, nct);
        unsigned long long *dst0 = a.apart_ll + (size_t)(g * ns + sp) * NREP * PW;
        if (has)
            for (int i = tid; i < NREP * C4; i += nct) {
                const int hh = i / C4, c = i % C4;
                float4    o4 = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int q = 0; q < PG; q++) {
                    const float4 v = gsum[((size_t)q * NREP + hh) * C4 + c];
                    o4.x += v.x; o4.y += v.y; o4.z += v.z; o4.w += v.w;
                }
                unsigned long long *dst = dst0 + (size_t)hh * PW + 4 * c;
                ll_put<SYS>(dst, o4.x, eout);
                ll_put<SYS>(dst + 1, o4.y, eout);
                ll_put<SYS>(dst + 2, o4.z, eout);
                ll_put<SYS>(dst + 3, o4.w, eout);
            }
        if (has && warp < NREP && lane == 0) {
            ll_put<SYS>(dst0 + (size_t)warp * PW + HD, m_run, eout);
            ll_put<SYS>(dst0 + (size_t)warp * PW + HD + 1, l_run, eout);
        }
    }
    // the K/V buffers were filled by the async proxy and read here; the next
    // phase writes the same bytes with ordinary stores
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (det) det[2] = clock64();

    // ---- merge, without tickets or fences: the KV head's NREP x HD outputs
    // are T = NREP * HD / 32 tasks of 32 dimensions of one query head; task j
    // runs on the CTA of split j % ns.  Every warp requests the splits' maxima
    // and weight sums (lane r: split r) and its own splits' sums (warp w:
    // splits w, w + 16, ...; lane = dimension) at once, waits until each word
    // carries this phase's epoch, and adds exp(m_r - M) acc_r in split order;
    // the 16 warp sums are added in warp order through shared memory:
    // out = sum_r exp(m_r - M) acc_r / sum_r exp(m_r - M) l_r.
    constexpr int T = NREP * (HD / 32);
    float *msum = S.red;                              // [MEGA_NCW][32], free after the rounds
    for (int j = sp; j < T; j += ns) {
        if (!has) break;
        const int hh = j / (HD / 32), d = (j % (HD / 32)) * 32 + lane;
        const unsigned long long *base = a.apart_ll + (size_t)g * ns * NREP * PW + (size_t)hh * PW;
        const size_t              rs = (size_t)NREP * PW;          // words between splits
        unsigned long long wm0 = 0, wl0 = 0, wm1 = 0, wl1 = 0, wa[4];
        if (lane < ns) { wm0 = ll_word<SYS>(base + lane * rs + HD); wl0 = ll_word<SYS>(base + lane * rs + HD + 1); }
        if (lane + 32 < ns) {
            wm1 = ll_word<SYS>(base + (lane + 32) * rs + HD);
            wl1 = ll_word<SYS>(base + (lane + 32) * rs + HD + 1);
        }
#pragma unroll
        for (int k = 0; k < 4; k++)
            if (warp + k * MEGA_NCW < ns) wa[k] = ll_word<SYS>(base + (warp + k * MEGA_NCW) * rs + d);
        float m0 = -INFINITY, l0 = 0.f, m1 = -INFINITY, l1 = 0.f;
        if (lane < ns) {
            m0 = ll_settle<SYS>(base + lane * rs + HD, wm0, eout, a.status);
            l0 = ll_settle<SYS>(base + lane * rs + HD + 1, wl0, eout, a.status);
        }
        if (lane + 32 < ns) {
            m1 = ll_settle<SYS>(base + (lane + 32) * rs + HD, wm1, eout, a.status);
            l1 = ll_settle<SYS>(base + (lane + 32) * rs + HD + 1, wl1, eout, a.status);
        }
        const float M = warp_max(fmaxf(m0, m1));
        const float w0 = m0 > -INFINITY ? expf(m0 - M) : 0.0f, w1 = m1 > -INFINITY ? expf(m1 - M) : 0.0f;
        float o = 0.0f;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int r = warp + k * MEGA_NCW;                   // warp-uniform
            const float wr = __shfl_sync(0xffffffffu, r < 32 ? w0 : w1, r & 31);
            if (r < ns) o = fmaf(ll_settle<SYS>(base + r * rs + d, wa[k], eout, a.status), wr, o);
        }
        msum[warp * 32 + lane] = o;
        named_bar(1, nct);
        if (warp == 0) {
            const float L = warp_sum(l0 * w0 + l1 * w1);
            const float invl = L > 0.0f ? 1.0f / L : 0.0f;
            float t = 0.0f;
            for (int w = 0; w < MEGA_NCW; w++) t += msum[w * 32 + lane];
            ll_put_out<SYS>(a, ph.bcast, ph.y_ll + (g * NREP + hh) * HD + d, t * invl, eout);
        }
        named_bar(1, nct);
    }
    // profiling: when KV head 0's merge was done (the CTA of split 0)
    if (a.phase_detail && has && g == 0 && sp == 0 && tid == 0)
        a.phase_detail[(size_t)p_idx * 4 + 3] = globaltimer_ns();
}

// L2 prefetch of the K and V rows this CTA's attention item will read (the
// positions below the current one of its split), issued a phase early.
__device__ __forceinline__ void attn_prefetch(const MegaArgs &a, const MegaPhase &ph, int pos, int hd)
{
    const int item = blockIdx.x;
    if (item >= a.n_kv * a.n_split) return;
    const int g = item / a.n_split, sp = item % a.n_split;
    const int npos = pos + 1;
    const int chunk = (npos + a.n_split - 1) / a.n_split;
    const int t0 = min(npos, sp * chunk), t1 = min(min(npos, t0 + chunk), pos);
    if (t1 <= t0) return;
    const size_t   off = ((size_t)g * a.n_ctx + t0) * hd;
    const uint32_t bytes = (uint32_t)((t1 - t0) * hd * sizeof(float));
    prefetch_l2(ph.kc + off, bytes);
    prefetch_l2(ph.vc + off, bytes);
}

template <bool SYS>
__device__ void mega_embed(const MegaArgs &a, const MegaShared &S, int p_idx)
{
    const unsigned eout = ll_epoch(S.launch, p_idx);
    const int    nct = MEGA_NCW * 32, n = a.n_embd;
    // a linked first stage waits for the token the last stage picked
    const int    tok = a.link_in ? __float_as_int(ll_get<true>(a.tok_ll, link_epoch(S.pos), a.status)) : a.st->token;
    if (tok < 0 || tok >= a.emb.n_out) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(&a.st->status, ECU_STATUS_BADTOKEN);
        return;
    }
    const size_t base = (size_t)tok * (size_t)n;
    for (int i = blockIdx.x * nct + threadIdx.x; i < n; i += gridDim.x * nct) {
        const size_t e = base + (size_t)i;
        ll_put<SYS>(a.x_ll + i, mat_elem(a.emb, (int)(e / (size_t)a.emb.n_in), (int)(e % (size_t)a.emb.n_in)), eout);
    }
}

template <int HD, int NREP, bool SYS>
__global__ void __launch_bounds__(MEGA_THREADS, 1) k_decode_mega(MegaArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    const int      nct = MEGA_NCW * 32, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const MegaSmem P = mega_smem_plan(a.red_floats, a.nst * a.stage_bytes, a.union_bytes, a.n_ph);
    MegaShared S;
    S.ring = smem + P.ring;
    S.full = reinterpret_cast<uint64_t *>(smem + P.bars);
    S.abar = reinterpret_cast<uint64_t *>(smem + P.abar);
    S.red = reinterpret_cast<float *>(smem + P.red);
    S.dig = reinterpret_cast<int *>(smem + P.un);
    S.kvbuf = reinterpret_cast<float *>(smem + P.un + a.kv_off);
    S.dsum = reinterpret_cast<double *>(smem + P.dsum);
    S.argsh = reinterpret_cast<ArgBest *>(smem + P.argsh);
    S.tab = reinterpret_cast<const uint4 *>(smem + P.tab);
    S.n_ph = a.n_ph;
    __shared__ MegaRing ring_state;
    __shared__ int pos_s;
    __shared__ unsigned launch_s;
    __shared__ __align__(16) MegaPhase ph_s[2];
    __shared__ __align__(8) uint64_t desc_bar;
    __shared__ __align__(16) float cs_row[HD];
    S.rc = &ring_state;
    S.cs = cs_row;
    S.dbar = &desc_bar;

    // the phase table into shared memory (the ring cursor reads only it)
    for (int i = threadIdx.x; i < a.n_ph; i += nct) reinterpret_cast<uint4 *>(smem + P.tab)[i] = __ldg(a.tab + i);
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int s = 0; s < a.nst; s++) mbar_init(&S.full[s], 1);
        for (int k = 0; k < 5; k++) mbar_init(&S.abar[k], 1);
        mbar_init(&desc_bar, 1);
        mbar_init_fence();
        pos_s = a.st->pos;            // stable for the whole step
        launch_s = a.bar[3];
        ph_s[0] = a.ph[0];
        S.rc->issued = 0;
        cursor_load_phase(S, &S.rc->cp, 0);
        for (int s = 0; s < a.nst; s++) S.rc->done[s] = 0u;
        for (int s = 0; s < a.nst; s++) ring_issue(a, S, s, false);     // the first chunks
        // the prefetch cursor starts where the copies are and runs
        // pf_stages chunks ahead of them
        S.rc->pf = S.rc->cp;
        const uint8_t *src;
        int            rows;
        unsigned       rb;
        for (int s = 0; s < a.pf_stages && cursor_next(S, &S.rc->pf, src, rows, rb); s++)
            prefetch_l2(src, (uint32_t)rows * rb);
    }
    __syncthreads();
    S.pos = pos_s;
    S.launch = launch_s;

    // ---- consumers -------------------------------------------------------------
    if (a.phase_ns && blockIdx.x == 0 && threadIdx.x == 0) {
        a.phase_ns[0] = globaltimer_ns();
        a.phase_clk[0] = clock64();
    }
    if (a.cta_ns && threadIdx.x == 0) a.cta_ns[blockIdx.x] = globaltimer_ns();
    RingPos rpos{0, 0u};
    int att_sb0 = 0, att_sb1 = 0, merges = 0;
    for (int p = 0; p < a.n_ph; p++) {
        // descriptors live in shared memory: phase p's arrived by a bulk
        // copy issued at the start of phase p-1, and phase p+1's is issued
        // now, so no phase starts with a global-memory round trip
        if (p > 0) mbar_wait<true>(&desc_bar, (unsigned)(p - 1) & 1u, a.status);
        const MegaPhase &ph = ph_s[p & 1];
        if (threadIdx.x == 0 && p + 1 < a.n_ph) {
            // the reads of that buffer (phase p-1's descriptor) are done:
            // every thread has passed the end of phase p-1
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_expect_tx(&desc_bar, (uint32_t)sizeof(MegaPhase));
            bulk_g2s(&ph_s[(p + 1) & 1], a.ph + p + 1, (uint32_t)sizeof(MegaPhase), &desc_bar);
        }
        const int kind = ph.kind;
        if (kind == PH_GEMV) {
            mega_gemv<SYS>(a, ph, S, rpos, p, ph.next_attn ? &ph_s[(p + 1) & 1] : nullptr, HD);
        } else if (kind == PH_ATTN) {
            mega_attention<HD, NREP, SYS>(a, ph, S, att_sb0, att_sb1, merges, p);
        } else {
            mega_embed<SYS>(a, S, p);
        }
        // the CTA's warps leave a phase together: shared buffers (row
        // partials, digit planes / K/V rows, the descriptor double buffer)
        // change hands only here
        named_bar(1, nct);
        if (a.phase_ns && blockIdx.x == 0 && threadIdx.x == 0) {
            a.phase_ns[p + 1] = globaltimer_ns();
            a.phase_clk[p + 1] = clock64();
        }
        if (a.cta_ns && threadIdx.x == 0) a.cta_ns[(size_t)(p + 1) * gridDim.x + blockIdx.x] = globaltimer_ns();
    }
    // ring and K/V copies still in flight (none, unless a wait gave up) land
    // before this CTA may exit
    named_bar(1, nct);
    if (threadIdx.x == 0) {
        const int n = S.rc->issued;
        for (int j = max(0, n - a.nst); j < n; j++)
            mbar_drain(&S.full[j % a.nst], (unsigned)(j / a.nst) & 1u, wait_limit_ns());
        for (int k = 0; k < 4; k++) {
            const int n_used = k < 2 ? att_sb0 : att_sb1;
            if (n_used > 0) mbar_drain(&S.abar[k], (unsigned)(n_used - 1) & 1u, wait_limit_ns());
        }
    }
    // a LAYERS stage advances its position once every phase is done; no
    // CTA reads it after the last attention phase
    if (a.layers_advance && blockIdx.x == 0 && threadIdx.x == 0) a.st->pos = S.pos + 1;
    if (a.phase_ns && blockIdx.x == 0 && threadIdx.x == 0) {
        a.phase_ns[a.n_ph] = globaltimer_ns();
        a.phase_clk[a.n_ph] = clock64();
    }
    // the last CTA out rewinds the exit counter and numbers the next launch
    // (the epochs of its tagged words differ from every word of this one)
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(a.bar + 1, 1u) == gridDim.x - 1) {
            a.bar[1] = 0u;
            a.bar[3] = a.bar[3] + 1u;
            __threadfence();
        }
    }
}
