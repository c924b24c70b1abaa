// ecu_engine.cu -- the llama token loop on one B200, behind engine_cuda.h.
//
// One context = one stage (EMBED / a LAYERS range / HEAD, src/engine.h:23-27)
// or the whole model (FULL) resident on one device.  A step is a fixed
// sequence of kernels on the context's stream, launched with programmatic
// dependent launch so that each GEMV starts streaming its weights while the
// previous kernel drains, and captured once into a CUDA graph that every
// later token replays.  Per-token inputs (token, position) live in device
// StepState, so the graph is position independent.
#include "../../include/engine_cuda.h"
#include "ecu_attn.cuh"
#include "ecu_gemv.cuh"
#include "ecu_mega.cuh"
#include "ecu_misc.cuh"
#include "ecu_model.h"
#include "ecu_prefill.cuh"

#include <atomic>
#include <mutex>
#include <cerrno>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <thread>
#include <vector>

static std::atomic<uint64_t> g_launches{0};

#define CK(call)                                                                        \
    do {                                                                                \
        cudaError_t e_ = (call);                                                        \
        if (e_ != cudaSuccess) {                                                        \
            ecu_set_error(nullptr, 0, "%s failed: %s", #call, cudaGetErrorString(e_)); \
            return -1;                                                                  \
        }                                                                               \
    } while (0)

// ------------------------------------------------------------ launching --

// One timed launch of the profiling replay.
struct ProfRec {
    const char *kind;
    double      bytes;
    cudaEvent_t e0, e1;
};

struct Launcher {
    cudaStream_t stream = nullptr;
    bool         pdl = true;
    int          count = 0;       // kernels enqueued since the last reset
    cudaError_t  err = cudaSuccess;
    // Profiling replay: events around every launch, tagged with the kind
    // and algorithmic bytes the enqueue code sets just before the launch.
    std::vector<ProfRec> *prof = nullptr;
    const char *kind = "kernel";
    double      bytes = 0;
    unsigned    cluster_y = 1;   // next launch: thread-block clusters of (1, cluster_y, 1)
    // The first kernel of a sequence follows host copies, not a kernel, so
    // it never gets a programmatic (early-start) dependency.

    template <typename... KArgs, typename... Args>
    void operator()(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, Args &&...args)
    {
        cudaLaunchConfig_t   cfg = {};
        cudaLaunchAttribute  attr[2];
        cfg.gridDim = grid;
        cfg.blockDim = block;
        cfg.dynamicSmemBytes = smem;
        cfg.stream = stream;
        unsigned na = 0;
        if (pdl && count > 0 && !prof) {
            attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[na].val.programmaticStreamSerializationAllowed = 1;
            na++;
        }
        if (cluster_y > 1) {
            attr[na].id = cudaLaunchAttributeClusterDimension;
            attr[na].val.clusterDim.x = 1;
            attr[na].val.clusterDim.y = cluster_y;
            attr[na].val.clusterDim.z = 1;
            na++;
        }
        cfg.attrs = attr;
        cfg.numAttrs = na;
        ProfRec r{kind, bytes, nullptr, nullptr};
        if (prof) {
            cudaEventCreate(&r.e0);
            cudaEventCreate(&r.e1);
            cudaEventRecord(r.e0, stream);
        }
        cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
        if (e != cudaSuccess && err == cudaSuccess) err = e;
        if (prof) {
            cudaEventRecord(r.e1, stream);
            prof->push_back(r);
        }
        kind = "kernel";
        bytes = 0;
        cluster_y = 1;
        count++;
    }
};

static int num_sms(int dev)
{
    static int cache[64] = {0};
    if (dev >= 0 && dev < 64 && cache[dev]) return cache[dev];
    int n = 148;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (dev >= 0 && dev < 64) cache[dev] = n;
    return n;
}

// ------------------------------------------------------------- GEMV plan --

static bool fast_ok(const DevMat &m)
{
    return !m.zero && m.nseg == 1 && (m.layout == LAY_SPLIT4 || m.layout == LAY_SPLIT8 || m.layout == LAY_SPLITK4) &&
           m.n_in % 1024 == 0 && m.n_in / 1024 <= FAST_MAX_NKG;
}

// Inputs of one column segment at most: the persistent step's digit planes
// hold this many.
#define SEG_MAX_IN (MEGA_MAX_NB * 32)

// Column segment s of m as a matrix of its own.
static DevMat seg_view(const DevMat &m, int s)
{
    DevMat v = m;
    v.nseg = 1;
    v.seg_bytes = 0;
    v.n_in = m.n_in / m.nseg;
    v.total = (size_t)v.n_in * m.n_out;
    if (m.data) v.data = m.data + (size_t)s * m.seg_bytes;
    return v;
}

// Largest dynamic shared memory a fast-GEMV launch may ask for: the
// opt-in per-block limit minus the kernel's own static shared memory.
static size_t g_fast_smem_max = 0;

template <int FMT, bool NORM, int EPI>
static void fast_attr_once()
{
    static std::atomic<uint64_t> done{0};     // one bit per device
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (!(done.load() & bit)) {
        int optin = 0;
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        cudaFuncAttributes fa;
        cudaFuncGetAttributes(&fa, k_gemv_fast<FMT, NORM, EPI>);
        const size_t dyn = (size_t)optin - fa.sharedSizeBytes;
        cudaFuncSetAttribute(k_gemv_fast<FMT, NORM, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)dyn);
        if (g_fast_smem_max == 0 || dyn < g_fast_smem_max) g_fast_smem_max = dyn;
        done |= bit;
    }
}

struct FastPlan {
    int    grid, threads, rows_per_cta, stage_rows;
    size_t smem;
};

static FastPlan plan_fast(const DevMat &m, int epi, int sms)
{
    FastPlan p;
    const int nkg = m.n_in / 1024;
    int rowpar = 16 / nkg;
    if (rowpar < 1) rowpar = 1;
    if (rowpar > 4) rowpar = 4;
    while (rowpar > 1 && 32 * (nkg * rowpar + 1) > FAST_MAX_THREADS) rowpar--;
    p.threads = 32 * (nkg * rowpar + 1);
    int grid = sms;
    for (;;) {
        int rpc = (m.n_out + grid - 1) / grid;
        if (epi == EPI_SWIGLU) rpc = (rpc + 1) & ~1;
        if ((size_t)rpc * nkg * sizeof(float) <= 48 * 1024 || grid >= m.n_out) {
            p.rows_per_cta = rpc;
            break;
        }
        grid += sms;
    }
    p.grid = (m.n_out + p.rows_per_cta - 1) / p.rows_per_cta;
    // ~40 KB stages, a whole number of row groups (one row per consumer warp)
    int sr = (int)(40960 / m.row_bytes);
    sr -= sr % rowpar;
    if (sr < rowpar) sr = rowpar;
    const int cap = ((p.rows_per_cta + rowpar - 1) / rowpar) * rowpar;
    if (sr > cap) sr = cap;
    p.stage_rows = sr;
    p.smem = fast_smem_plan(m.row_bytes, sr, p.rows_per_cta, nkg, rowpar).total;
    return p;
}

template <int HD, int R>
static void attn_attr()
{
    cudaFuncSetAttribute(k_attention<HD, R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)attn_smem_bytes<HD>());
    cudaFuncSetAttribute(k_attention<HD, R>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
}

// Largest cluster (= number of position splits per KV head, <= 16) of which
// n_kv can be resident at once.
template <int HD, int R>
static int attn_cluster_for(int n_kv, int max_split)
{
    for (int cs = ATT_MAX_SPLIT; cs >= 1; cs >>= 1) {
        if (cs > max_split) continue;
        cudaLaunchConfig_t  cfg = {};
        cudaLaunchAttribute at;
        cfg.gridDim = dim3(n_kv, cs);
        cfg.blockDim = dim3(ATT_THREADS);
        cfg.dynamicSmemBytes = attn_smem_bytes<HD>();
        at.id = cudaLaunchAttributeClusterDimension;
        at.val.clusterDim.x = 1;
        at.val.clusterDim.y = cs;
        at.val.clusterDim.z = 1;
        cfg.attrs = &at;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, k_attention<HD, R>, &cfg) == cudaSuccess && n >= n_kv)
            return cs;
        cudaGetLastError();
    }
    return 1;
}

static int attn_cluster(int hd, int rep, int n_kv, int max_split)
{
#define CL(HD_, R_) if (hd == HD_ && rep == R_) return attn_cluster_for<HD_, R_>(n_kv, max_split);
    CL(128, 1) CL(128, 2) CL(128, 4) CL(128, 8) CL(64, 1) CL(64, 2) CL(64, 4) CL(64, 8)
    CL(32, 1) CL(32, 2) CL(32, 4) CL(32, 8) CL(16, 1) CL(16, 2) CL(16, 4) CL(16, 8)
#undef CL
    return 1;
}

static void attn_attrs_all()
{
    attn_attr<128, 1>(); attn_attr<128, 2>(); attn_attr<128, 4>(); attn_attr<128, 8>();
    attn_attr<64, 1>(); attn_attr<64, 2>(); attn_attr<64, 4>(); attn_attr<64, 8>();
    attn_attr<32, 1>(); attn_attr<32, 2>(); attn_attr<32, 4>(); attn_attr<32, 8>();
    attn_attr<16, 1>(); attn_attr<16, 2>(); attn_attr<16, 4>(); attn_attr<16, 8>();
}

static void fast_attrs_all()
{
    fast_attr_once<4, false, EPI_STORE>(); fast_attr_once<4, false, EPI_ADD>();
    fast_attr_once<4, false, EPI_SWIGLU>(); fast_attr_once<4, false, EPI_ARGMAX>();
    fast_attr_once<4, true, EPI_STORE>(); fast_attr_once<4, true, EPI_ADD>();
    fast_attr_once<4, true, EPI_SWIGLU>(); fast_attr_once<4, true, EPI_ARGMAX>();
    fast_attr_once<8, false, EPI_STORE>(); fast_attr_once<8, false, EPI_ADD>();
    fast_attr_once<8, false, EPI_SWIGLU>(); fast_attr_once<8, false, EPI_ARGMAX>();
    fast_attr_once<8, true, EPI_STORE>(); fast_attr_once<8, true, EPI_ADD>();
    fast_attr_once<8, true, EPI_SWIGLU>(); fast_attr_once<8, true, EPI_ARGMAX>();
    fast_attr_once<12, false, EPI_STORE>(); fast_attr_once<12, false, EPI_ADD>();
    fast_attr_once<12, false, EPI_SWIGLU>(); fast_attr_once<12, false, EPI_ARGMAX>();
    fast_attr_once<12, true, EPI_STORE>(); fast_attr_once<12, true, EPI_ADD>();
    fast_attr_once<12, true, EPI_SWIGLU>(); fast_attr_once<12, true, EPI_ARGMAX>();
}

template <int FMT, bool NORM, int EPI>
static void launch_fast_t(Launcher &L, const GemvArgs &a, const FastPlan &p)
{
    fast_attr_once<FMT, NORM, EPI>();
    L(k_gemv_fast<FMT, NORM, EPI>, dim3(p.grid), dim3(p.threads), p.smem, a);
}

template <int FMT, bool NORM>
static void launch_fast_e(Launcher &L, const GemvArgs &a, const FastPlan &p, int epi)
{
    switch (epi) {
    case EPI_STORE:  launch_fast_t<FMT, NORM, EPI_STORE>(L, a, p); break;
    case EPI_ADD:    launch_fast_t<FMT, NORM, EPI_ADD>(L, a, p); break;
    case EPI_SWIGLU: launch_fast_t<FMT, NORM, EPI_SWIGLU>(L, a, p); break;
    default:         launch_fast_t<FMT, NORM, EPI_ARGMAX>(L, a, p); break;
    }
}

// Algorithmic bytes of y = W x: W as stored in the file, x read, y written.
static double gemv_bytes(const DevMat &m, int epi)
{
    const double w = m.zero ? 0.0 : (double)ecu_type_nbytes(m.type, (size_t)m.n_in * m.n_out);
    const double y = epi == EPI_SWIGLU ? m.n_out / 2 : (epi == EPI_ADD ? 2.0 * m.n_out : m.n_out);
    return w + 4.0 * m.n_in + 4.0 * y;
}

// Scratch a GEMV launch may need (argmax partials/counter, normed input).
struct GemvScratch {
    float    *xn = nullptr;        // >= max n_in floats (generic-path RMSNorm)
    float    *part_val = nullptr;  // >= grid
    int      *part_idx = nullptr;
    unsigned *counter = nullptr;
    int      *status = nullptr;
};

// y (epi) W * rmsnorm?(x).  norm_w null = no prologue.  For the argmax
// epilogue `a` carries the extra outputs.
static void enqueue_gemv(Launcher &L, int sms, const DevMat &m, const float *x, const float *norm_w,
                         float eps, float *y, int epi, const GemvScratch &s, GemvArgs a,
                         const DevMat *next = nullptr, int next_epi = EPI_STORE)
{
    if (m.nseg > 1) {
        // column segments (EPI_STORE / EPI_ADD without a norm prologue): the
        // first stores or adds W_0 x_0, the others add W_s x_s
        const char *kind = L.kind;
        for (int si = 0; si < m.nseg; si++) {
            const DevMat v = seg_view(m, si);
            const DevMat vn = si + 1 < m.nseg ? seg_view(m, si + 1) : DevMat{};
            const bool   last = si + 1 == m.nseg;
            L.kind = kind;
            enqueue_gemv(L, sms, v, x + (size_t)si * v.n_in, nullptr, eps, y, si == 0 ? epi : EPI_ADD, s, a,
                         last ? next : &vn, last ? next_epi : EPI_ADD);
        }
        return;
    }
    DevMat nv;
    if (next && next->nseg > 1) {
        nv = seg_view(*next, 0);
        next = &nv;
    }
    if (next && fast_ok(*next) && next->data) {
        const FastPlan np = plan_fast(*next, next_epi, sms);
        a.pf_ptr = next->data;
        a.pf_end = next->data + (size_t)next->n_out * next->row_bytes;
        a.pf_stride = (size_t)np.rows_per_cta * next->row_bytes;
        const size_t per = a.pf_stride < (size_t)65536 ? a.pf_stride : (size_t)65536;
        a.pf_bytes = (uint32_t)(per & ~(size_t)15);
    }
    if (L.bytes == 0) L.bytes = gemv_bytes(m, epi);
    a.m = m;
    a.eps = eps;
    a.y = y;
    a.part_val = s.part_val;
    a.part_idx = s.part_idx;
    a.counter = s.counter;
    a.status = s.status;
    FastPlan p{};
    if (fast_ok(m) && (epi != EPI_SWIGLU || m.n_out % 2 == 0)) p = plan_fast(m, epi, sms);
    if (p.grid > 0 && p.grid <= 4096 && p.smem <= g_fast_smem_max) {
        a.x = x;
        a.norm_w = norm_w;
        a.rows_per_cta = p.rows_per_cta;
        a.stage_rows = p.stage_rows;
        const bool norm = norm_w != nullptr;
        if (m.layout == LAY_SPLIT4) {
            if (norm) launch_fast_e<4, true>(L, a, p, epi);
            else launch_fast_e<4, false>(L, a, p, epi);
        } else if (m.layout == LAY_SPLITK4) {
            if (norm) launch_fast_e<12, true>(L, a, p, epi);
            else launch_fast_e<12, false>(L, a, p, epi);
        } else {
            if (norm) launch_fast_e<8, true>(L, a, p, epi);
            else launch_fast_e<8, false>(L, a, p, epi);
        }
        return;
    }
    const float *in = x;
    if (norm_w) {
        const char *k = L.kind;
        const double b = L.bytes;
        L.kind = "rmsnorm";
        L.bytes = 12.0 * m.n_in;
        L(k_rmsnorm, dim3(1), dim3(256), 0, x, norm_w, m.n_in, eps, s.xn);
        L.kind = k;
        L.bytes = b;
        in = s.xn;
    }
    a.x = in;
    const int warps = 8, grid = (m.n_out + warps - 1) / warps;
    const int g = grid < 4 * sms ? grid : 4 * sms;
    switch (epi) {
    case EPI_STORE: L(k_gemv_generic<EPI_STORE>, dim3(g), dim3(32 * warps), 0, a); break;
    case EPI_ADD:   L(k_gemv_generic<EPI_ADD>, dim3(g), dim3(32 * warps), 0, a); break;
    default:        L(k_gemv_generic<EPI_ARGMAX>, dim3(g), dim3(32 * warps), 0, a); break;
    }
}

// ------------------------------------------------------------- context --

struct LayerDev {
    // attention projections: one fused matrix (rows q|k|v) or three
    std::vector<DevMat> qkv;       // each writes rows [qkv_off[i], ...) of the qkv buffer
    std::vector<int>    qkv_off;
    DevMat              o;
    bool                gu_fused = false;
    DevMat              gu, g, u;  // fused: interleaved rows (gate j = 2j, up j = 2j+1)
    DevMat              d;
    float *attn_norm = nullptr, *ffn_norm = nullptr;
    float *bq = nullptr, *bk = nullptr, *bv = nullptr;
    // the layer's attention half (Q/K/V, attention, attn_output) and FFN
    // half (gate/up, down) on this context: a span may start at a layer's
    // FFN half or end at its attention half
    bool ha = true, hf = true;
    // source tensors, for ecu_dequant_tensor
    struct Src { std::string name; const DevMat *m; int row0, rstride, n_in; size_t elems; };
};

// Device allocations shared by a context and its forks (weights, norms, the
// RoPE table): freed when the last context holding them closes.
struct SharedAllocs {
    int                 device = 0;
    std::vector<void *> p;
    ~SharedAllocs()
    {
        if (p.empty()) return;
        cudaSetDevice(device);
        for (void *q : p) cudaFree(q);
    }
};

// Tensor-parallel slice of a FULL context: rank `rank` of `world` owns
// query heads [rank*nh, ..), KV heads [rank*nkv, ..), rows [rank*ne, ..) of
// attn_output and ffn_down, FFN channels [rank*ff, ..) and vocabulary rows
// [v0, v1); every projection keeps its whole input (no split reductions).
struct TpSlice {
    int rank = 0, world = 1;
    int nh = 0, nkv = 0, ne = 0, ff = 0, v0 = 0, v1 = 0;
};

struct ecu_ctx {
    int         device = 0, sms = 148;
    int         stage = 0, first = 0, last = 0, pos = 0;
    unsigned    span = 0;                 // ECU_SPAN_* of an ECU_STAGE_SPAN context
    EcuGeom     g;
    TpSlice     tp;
    std::vector<void *> tp_peers;         // IPC mappings of the other ranks' tagged vectors

    // batched prompt (ecu_prefill): activations of `rows` tokens, fp16 hi/lo
    // operands, one dequantised weight matrix; allocated on first use
    struct Prefill {
        int     rows = 0;
        size_t  wcap = 0;
        float  *X = nullptr, *QKV = nullptr, *ATT = nullptr, *GU = nullptr, *H = nullptr;
        __half *ah = nullptr, *al = nullptr, *wh = nullptr, *wl = nullptr;
        int    *tok = nullptr;
    } pf;
    cudaStream_t stream = nullptr;
    bool        pdl = true, use_graph = true;
    std::vector<void *> allocs;           // this context's own buffers
    std::shared_ptr<SharedAllocs> shared; // read-only tensors, shared with forks
    struct Uploader *up = nullptr;        // while opening: pinned double-buffered weight staging
    bool        to_shared = false;        // dalloc target while uploading weights
    size_t      bytes = 0;

    std::vector<LayerDev> layers;
    DevMat   emb, out;            // EMBED/FULL: emb; HEAD/FULL: out (logits matrix)
    float   *out_norm = nullptr;
    float   *rope_cs = nullptr;
    float   *kc = nullptr, *vc = nullptr;   // [layers][nkv][n_ctx][hd]
    float   *state = nullptr;     // n_embd + 1
    float   *qkv = nullptr, *att = nullptr, *h = nullptr, *gtmp = nullptr, *utmp = nullptr;
    float   *logits = nullptr;
    int      n_split = 1;
    GemvScratch scr;
    StepState *st = nullptr;      // device
    StepState *h_st = nullptr;    // pinned host slots, one per position: an
                                  // async copy may still be reading slot p
                                  // while the host fills slot p+1; slot
                                  // n_hslots receives the device state
    int        n_hslots = 0;
    float    *h_state = nullptr;  // pinned host staging, n_embd + 1
    int      *tok_hist = nullptr; // device [n_ctx]
    bool      have_logits = false;
    int       last_pick = 0;

    cudaGraphExec_t graph = nullptr;   // the full step
    int             graph_kernels = 0;

    // persistent whole-step kernel (LAYERS / FULL stages that qualify)
    bool        mega = false;
    std::string path = "kernels";         // which step implementation runs, and why
    void      (*mega_fn)(MegaArgs) = nullptr;
    MegaArgs    margs{};
    int         mega_grid = 0;
    size_t      mega_smem = 0;
    unsigned long long *mega_ll = nullptr;   // the tagged activation vectors, one block
    size_t      mega_ll_words = 0;
    int         stall_next = -1;          // ecu_inject_wait_timeout: the phase the next launch stalls
    std::vector<MegaPhase> mega_ph;       // host copy of the phase list (pipeline links patch inputs)
    cudaEvent_t ev_step = nullptr;        // ecu_step_dev on a caller's stream: ordering with the own stream
    void       *link_peer = nullptr;      // IPC mapping of the next stage's tagged vectors
    bool        linked_in = false;        // the step's input arrives over a pipeline link
    std::vector<const char *> ph_kind;    // per phase, for the profile
    std::vector<int> ph_in_ep;            // per phase: GEMV input's writer phase (-1: plain input or not a GEMV)
    std::vector<double>       ph_bytes;

    struct SrcRef { std::string name; DevMat m; int row0, rstride; size_t elems; int n_in; };
    std::vector<SrcRef> srcs;

    template <class T> T *dalloc(size_t n)
    {
        // 256 bytes of zeroed slack: the reference's Q8_K decoder reads its
        // 32 scales 28 bytes past a 292-byte block (src/gguf.c:655), so a
        // device copy of a Q8_K tensor must be readable that far past its end
        void *p = nullptr;
        if (cudaMalloc(&p, n * sizeof(T) + 256) != cudaSuccess) return nullptr;
        cudaMemset((uint8_t *)p + n * sizeof(T), 0, 256);
        if (to_shared) shared->p.push_back(p);
        else allocs.push_back(p);
        bytes += n * sizeof(T);
        return (T *)p;
    }
};

static size_t align16(size_t v) { return (v + 15) & ~(size_t)15; }

// Device row length of a matrix of type t with n_in inputs in `layout`.
static size_t dev_row_bytes(int t, int n_in, int layout)
{
    if (layout == LAY_SPLIT4 || layout == LAY_SPLITK4) return align16((size_t)n_in / 32 * 18);
    if (layout == LAY_SPLIT8) return align16((size_t)n_in / 32 * 34);
    if (t == GT_F32) return (size_t)n_in * 4;
    if (t == GT_F16) return (size_t)n_in * 2;
    return (size_t)(n_in / blk_elems(t)) * blk_bytes(t);
}

static int choose_layout(int t, int n_in)
{
    if (n_in % 1024 == 0 && n_in / 1024 <= FAST_MAX_NKG) {
        if (t == GT_Q4_0) return LAY_SPLIT4;
        if (t == GT_Q8_0) return LAY_SPLIT8;
        if (t == GT_Q4_K) return LAY_SPLITK4;
    }
    return LAY_RAW;
}

// Device shape of a matrix: its layout, column segments (allow_seg: a matrix
// wider than SEG_MAX_IN inputs is cut into equal segments of whole 1024-input
// groups when its segments take a fast layout) and a segment's row bytes.
struct MatShape {
    int    layout, nseg;
    size_t row_bytes;
};

static MatShape mat_shape(int t, int n_in, bool allow_split, bool allow_seg)
{
    MatShape s{allow_split ? choose_layout(t, n_in) : LAY_RAW, 1, 0};
    if (allow_split && allow_seg && n_in > SEG_MAX_IN) {
        const int ns = (n_in + SEG_MAX_IN - 1) / SEG_MAX_IN;
        if (n_in % (1024 * ns) == 0 && choose_layout(t, n_in / ns) != LAY_RAW) {
            s.nseg = ns;
            s.layout = choose_layout(t, n_in / ns);
        }
    }
    s.row_bytes = dev_row_bytes(t, n_in / s.nseg, s.layout);
    return s;
}

// Zero-output rule of the reference matvec: a quantised tensor whose n_in
// is not a multiple of its block (engine.c:317-320) or a type gguf_dequant
// rejects (engine.c:332-337) contributes zeros.
static bool zero_rule(int t, int n_in)
{
    if (t == GT_F32 || t == GT_F16) return false;
    if (n_in % blk_elems(t)) return true;
    return !dq_supported(t);
}

// Weight staging while a context opens: the host copies chunk i of a
// tensor's rows into pinned buffer i % 2 (several threads), one async copy
// moves it to device buffer i % 2 and the repack kernel lays it out, while
// the host already fills the other pinned buffer; an event per buffer says
// when it may be refilled.  The source is the caller's GGUF image or a file
// mapping (ecu_model_open_file: only the stage's tensors are paged in).
struct Uploader {
    uint8_t    *pin[2] = {nullptr, nullptr}, *dev[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    size_t      cap = 0;
    int         next = 0;
};

static void uploader_free(Uploader *u)
{
    if (!u) return;
    for (int b = 0; b < 2; b++) {
        if (u->ev[b]) cudaEventSynchronize(u->ev[b]), cudaEventDestroy(u->ev[b]);
        if (u->pin[b]) cudaFreeHost(u->pin[b]);
        if (u->dev[b]) cudaFree(u->dev[b]);
    }
    delete u;
}

static Uploader *uploader_new(size_t cap)
{
    Uploader *u = new Uploader();
    u->cap = cap;
    for (int b = 0; b < 2; b++)
        if (cudaMallocHost(&u->pin[b], cap) != cudaSuccess || cudaMalloc(&u->dev[b], cap + 256) != cudaSuccess ||
            cudaEventCreateWithFlags(&u->ev[b], cudaEventDisableTiming) != cudaSuccess) {
            cudaGetLastError();
            uploader_free(u);
            return nullptr;
        }
    return u;
}

// rows of `len` bytes, `stride` apart, packed into dst -- split over threads
static void host_pack_rows(uint8_t *dst, const uint8_t *src, size_t len, size_t stride, size_t rows)
{
    const size_t total = len * rows;
    const int    nt = total >= ((size_t)32 << 20) ? 8 : total >= ((size_t)4 << 20) ? 4 : 1;
    auto part = [&](size_t r0, size_t r1) {
        if (len == stride) memcpy(dst + r0 * len, src + r0 * stride, (r1 - r0) * len);
        else
            for (size_t r = r0; r < r1; r++) memcpy(dst + r * len, src + r * stride, len);
    };
    if (nt == 1) { part(0, rows); return; }
    std::vector<std::thread> th;
    for (int k = 0; k < nt; k++) th.emplace_back(part, rows * k / nt, rows * (k + 1) / nt);
    for (auto &t : th) t.join();
}

static void launch_repack(const ecu_ctx *c, const DevMat &m, const uint8_t *stage, int si, int rows, uint8_t *dst,
                          int row0, int rstride, size_t seg_src)
{
    const int grid = 4 * c->sms, blk = 256;
    if (m.layout == LAY_SPLIT4)
        k_repack_q4_0<<<grid, blk, 0, c->stream>>>(stage, si / 32, rows, dst, m.row_bytes, row0, rstride);
    else if (m.layout == LAY_SPLIT8)
        k_repack_q8_0<<<grid, blk, 0, c->stream>>>(stage, si / 32, rows, dst, m.row_bytes, row0, rstride);
    else if (m.layout == LAY_SPLITK4)
        k_repack_q4_k<<<grid, blk, 0, c->stream>>>(stage, si / 256, rows, dst, m.row_bytes, row0, rstride);
    else
        k_copy_rows<<<grid, blk, 0, c->stream>>>(stage, seg_src, rows, dst, m.row_bytes, row0, rstride);
}

// Upload rows [src_row0, src_row0 + rows) of tensor `src` (n_in inputs
// each) into device matrix `m` at rows row0, row0+rstride, ...  `stage` is a
// device staging buffer (used when no Uploader is active).
static int upload_rows(ecu_ctx *c, const EcuTensor *src, int n_in, int rows, DevMat &m, int row0,
                       int rstride, uint8_t *stage, size_t src_row0 = 0)
{
    if (m.zero) return 0;
    const size_t src_row = (size_t)ecu_type_nbytes(src->type, (size_t)n_in);
    const int    si = n_in / m.nseg;                          // inputs of a segment
    const size_t seg_src = (size_t)ecu_type_nbytes(src->type, (size_t)si);
    const int    grid = 4 * c->sms, blk = 256;
    if (Uploader *u = c->up) {
        const size_t per = std::max<size_t>(1, u->cap / std::max<size_t>(1, seg_src));
        if (seg_src > u->cap) { ecu_set_error(nullptr, 0, "a weight row exceeds the upload chunk"); return -1; }
        for (int sg = 0; sg < m.nseg; sg++) {
            const uint8_t *from = src->data + src_row0 * src_row + (size_t)sg * seg_src;
            uint8_t       *dst = const_cast<uint8_t *>(m.data) + (size_t)sg * m.seg_bytes;
            for (size_t r = 0; r < (size_t)rows; r += per) {
                const size_t nr = std::min(per, (size_t)rows - r);
                const int    b = u->next;
                u->next ^= 1;
                CK(cudaEventSynchronize(u->ev[b]));        // the chunk before last is done with buffer b
                host_pack_rows(u->pin[b], from + r * src_row, seg_src, src_row, nr);
                CK(cudaMemcpyAsync(u->dev[b], u->pin[b], nr * seg_src, cudaMemcpyHostToDevice, c->stream));
                launch_repack(c, m, u->dev[b], si, (int)nr, dst, row0 + (int)r * rstride, rstride, seg_src);
                CK(cudaGetLastError());
                CK(cudaEventRecord(u->ev[b], c->stream));
            }
        }
        return 0;
    }
    for (int sg = 0; sg < m.nseg; sg++) {
        // segment sg's part of every source row, packed rows of seg_src bytes
        const uint8_t *from = src->data + src_row0 * src_row + (size_t)sg * seg_src;
        if (m.nseg == 1)
            CK(cudaMemcpyAsync(stage, from, src_row * (size_t)rows, cudaMemcpyHostToDevice, c->stream));
        else
            CK(cudaMemcpy2DAsync(stage, seg_src, from, src_row, seg_src, (size_t)rows, cudaMemcpyHostToDevice,
                                 c->stream));
        uint8_t *dst = const_cast<uint8_t *>(m.data) + (size_t)sg * m.seg_bytes;
        launch_repack(c, m, stage, si, rows, dst, row0, rstride, seg_src);
        (void)grid;
        (void)blk;
        CK(cudaGetLastError());
        CK(cudaStreamSynchronize(c->stream));   // the staging buffer is reused
    }
    return 0;
}

static DevMat make_mat(ecu_ctx *c, int type, int n_in, int n_out, bool allow_split, bool allow_seg = false)
{
    DevMat m;
    m.type = type;
    m.n_in = n_in;
    m.n_out = n_out;
    m.zero = zero_rule(type, n_in);
    const MatShape sh = mat_shape(type, n_in, allow_split, allow_seg && !m.zero);
    m.layout = sh.layout;
    m.nseg = sh.nseg;
    m.row_bytes = sh.row_bytes;
    m.seg_bytes = m.row_bytes * (size_t)n_out;
    m.total = (size_t)n_in * n_out;
    if (!m.zero) m.data = c->dalloc<uint8_t>(m.seg_bytes * (size_t)m.nseg);
    return m;
}

// fp32 copy of the first n elements of a small tensor (norms, biases);
// zeros when the reference's row_to_float would fail (engine.c:360-364).
static float *upload_vec(ecu_ctx *c, const EcuTensor *t, size_t n, uint8_t *stage)
{
    float *d = c->dalloc<float>(n);
    if (!d) return nullptr;
    cudaMemsetAsync(d, 0, n * sizeof(float), c->stream);
    const int   ty = (int)t->type;
    const size_t total = t->elems();
    const bool  ok = dq_supported(ty) && n <= total &&
                    (ty == GT_F32 || ty == GT_F16 || (n + blk_elems(ty) - 1) / blk_elems(ty) <= total / blk_elems(ty));
    if (ok && n > 0) {
        size_t nbytes = (ty == GT_F32 || ty == GT_F16)
                            ? ecu_type_nbytes(ty, n)
                            : ((n + blk_elems(ty) - 1) / blk_elems(ty)) * blk_bytes(ty);
        cudaMemcpyAsync(stage, t->data, nbytes, cudaMemcpyHostToDevice, c->stream);
        k_dequant_raw<<<64, 256, 0, c->stream>>>(ty, stage, 0, n, d);
    }
    cudaStreamSynchronize(c->stream);
    return d;
}

static void ctx_free(ecu_ctx *c)
{
    if (!c) return;
    if (c->device >= 0) cudaSetDevice(c->device);
    uploader_free(c->up);
    if (c->graph) cudaGraphExecDestroy(c->graph);
    for (void *p : c->tp_peers)
        if (p) cudaIpcCloseMemHandle(p);
    if (c->link_peer) cudaIpcCloseMemHandle(c->link_peer);
    if (c->ev_step) cudaEventDestroy(c->ev_step);
    for (void *p : {(void *)c->pf.X, (void *)c->pf.QKV, (void *)c->pf.ATT, (void *)c->pf.GU, (void *)c->pf.H,
                    (void *)c->pf.ah, (void *)c->pf.al, (void *)c->pf.wh, (void *)c->pf.wl, (void *)c->pf.tok})
        if (p) cudaFree(p);
    for (void *p : c->allocs) cudaFree(p);
    if (c->h_st) cudaFreeHost(c->h_st);
    if (c->h_state) cudaFreeHost(c->h_state);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

// What a context's step does, by stage: EMBED (embedding row), LAYERS,
// HEAD, FULL (all three), SPAN (a layer range, first > last for none, with
// the embedding and/or the head by its flags).
static bool r_emb(const ecu_ctx *c)
{
    return c->stage == ECU_STAGE_EMBED || c->stage == ECU_STAGE_FULL ||
           (c->stage == ECU_STAGE_SPAN && (c->span & ECU_SPAN_EMBED));
}
static bool r_lay(const ecu_ctx *c)
{
    return c->stage == ECU_STAGE_LAYERS || c->stage == ECU_STAGE_FULL ||
           (c->stage == ECU_STAGE_SPAN && c->first <= c->last);
}
static bool r_head(const ecu_ctx *c)
{
    return c->stage == ECU_STAGE_HEAD || c->stage == ECU_STAGE_FULL ||
           (c->stage == ECU_STAGE_SPAN && (c->span & ECU_SPAN_HEAD));
}
// the step advances the position (a HEAD or EMBED stage keeps none)
static bool r_pos(const ecu_ctx *c) { return r_lay(c) || c->stage == ECU_STAGE_SPAN; }

// ------------------------------------------------------------- the step --

// First weight matrix the step touches after layer li's down projection.
static const DevMat *after_layer(const ecu_ctx *c, int li, int nl)
{
    if (li + 1 < nl) return &c->layers[li + 1].qkv[0];
    if (r_head(c)) return &c->out;
    return nullptr;
}

static void enqueue_layer(ecu_ctx *c, Launcher &L, int li, int nl = -1)
{
    if (nl < 0) nl = (int)c->layers.size();
    LayerDev   &ly = c->layers[li];
    const DevMat *gu_first = ly.gu_fused ? &ly.gu : &ly.g;
    const EcuGeom &g = c->g;
    const int   hd = g.head_dim, qdim = g.n_head * hd, kvdim = g.n_head_kv * hd;
    GemvArgs    a = {};
    a.st = c->st;

    if (ly.ha) {
        // (1) RMSNorm + Q/K/V projections
        if (ly.qkv.size() == 1) {
            L.kind = "gemv_qkv";
            enqueue_gemv(L, c->sms, ly.qkv[0], c->state, ly.attn_norm, g.eps, c->qkv, EPI_STORE, c->scr, a,
                         &ly.o, EPI_ADD);
        } else {
            L.kind = "rmsnorm";
            L.bytes = 12.0 * g.n_embd;
            L(k_rmsnorm, dim3(1), dim3(256), 0, (const float *)c->state, (const float *)ly.attn_norm,
              g.n_embd, g.eps, c->scr.xn);
            for (size_t i = 0; i < ly.qkv.size(); i++) {
                L.kind = "gemv_qkv";
                enqueue_gemv(L, c->sms, ly.qkv[i], c->scr.xn, nullptr, g.eps, c->qkv + ly.qkv_off[i],
                             EPI_STORE, c->scr, a);
            }
        }
        // (2) bias + RoPE + KV append + attention
        AttnArgs aa;
        aa.qkv = c->qkv;
        aa.bq = ly.bq;
        aa.bk = ly.bk;
        aa.bv = ly.bv;
        aa.rope_cs = c->rope_cs;
        const size_t plane = (size_t)g.n_head_kv * g.n_ctx * hd;
        aa.kc = c->kc + (size_t)li * plane;
        aa.vc = c->vc + (size_t)li * plane;
        aa.att = c->att;
        aa.st = c->st;
        aa.status = &c->st->status;
        aa.n_head = g.n_head;
        aa.n_kv = g.n_head_kv;
        aa.n_rep = g.n_rep;
        aa.n_ctx = g.n_ctx;
        aa.n_split = c->n_split;
        aa.kscale = 1.0f / sqrtf((float)hd);
        dim3 ag(g.n_head_kv, c->n_split);
        L.kind = "attention";
        L.cluster_y = (unsigned)c->n_split;
        // K and V rows of positions 0..pos read, one row of each written, q/att
        L.bytes = 2.0 * 4.0 * kvdim * (c->pos + 2) + 8.0 * qdim + 4.0 * (qdim + 2 * kvdim);
#define ATT_CASE(HD_, R_) \
        if (hd == HD_ && g.n_rep == R_) { L(k_attention<HD_, R_>, ag, dim3(ATT_THREADS), attn_smem_bytes<HD_>(), aa); } else
        ATT_CASE(128, 1) ATT_CASE(128, 2) ATT_CASE(128, 4) ATT_CASE(128, 8)
        ATT_CASE(64, 1) ATT_CASE(64, 2) ATT_CASE(64, 4) ATT_CASE(64, 8)
        ATT_CASE(32, 1) ATT_CASE(32, 2) ATT_CASE(32, 4) ATT_CASE(32, 8)
        ATT_CASE(16, 1) ATT_CASE(16, 2) ATT_CASE(16, 4) ATT_CASE(16, 8) {}
#undef ATT_CASE
        (void)qdim;
        (void)kvdim;
        // (3) x += Wo * att
        L.kind = "gemv_o";
        // (the next weights: this layer's gate/up, or with the attention half
        // only, what follows the layer)
        const DevMat *ox = ly.hf ? gu_first : after_layer(c, li, nl);
        const int     oe = ly.hf ? (ly.gu_fused ? EPI_SWIGLU : EPI_STORE) : (ox == &c->out ? EPI_ARGMAX : EPI_STORE);
        enqueue_gemv(L, c->sms, ly.o, c->att, nullptr, g.eps, c->state, EPI_ADD, c->scr, a, ox, oe);
    }
    if (ly.hf) {
        // (4) RMSNorm + gate/up + SwiGLU
        if (ly.gu_fused) {
            L.kind = "gemv_gate_up";
            enqueue_gemv(L, c->sms, ly.gu, c->state, ly.ffn_norm, g.eps, c->h, EPI_SWIGLU, c->scr, a, &ly.d,
                         EPI_ADD);
        } else {
            L.kind = "rmsnorm";
            L.bytes = 12.0 * g.n_embd;
            L(k_rmsnorm, dim3(1), dim3(256), 0, (const float *)c->state, (const float *)ly.ffn_norm,
              g.n_embd, g.eps, c->scr.xn);
            L.kind = "gemv_gate";
            enqueue_gemv(L, c->sms, ly.g, c->scr.xn, nullptr, g.eps, c->gtmp, EPI_STORE, c->scr, a);
            L.kind = "gemv_up";
            enqueue_gemv(L, c->sms, ly.u, c->scr.xn, nullptr, g.eps, c->utmp, EPI_STORE, c->scr, a);
            L.kind = "swiglu";
            L.bytes = 12.0 * g.n_ff;
            L(k_swiglu, dim3((g.n_ff + 255) / 256), dim3(256), 0, (const float *)c->gtmp,
              (const float *)c->utmp, c->h, g.n_ff);
        }
        // (5) x += Wd * h
        L.kind = "gemv_down";
        const DevMat *nx = after_layer(c, li, nl);
        enqueue_gemv(L, c->sms, ly.d, c->h, nullptr, g.eps, c->state, EPI_ADD, c->scr, a, nx,
                     nx == &c->out ? EPI_ARGMAX : EPI_STORE);
    }
}

static void enqueue_head(ecu_ctx *c, Launcher &L, bool advance)
{
    const EcuGeom &g = c->g;
    // RMSNorm fused into the head GEMV (the arithmetic of the persistent
    // step's head phase): the normed state goes to scratch, and the CTA that
    // finishes the argmax copies it over the state, HEAD's out[0..n_embd)
    GemvArgs a = {};
    a.st = c->st;
    a.tok_hist = c->tok_hist;
    a.tok_out = c->state + g.n_embd;
    a.advance_pos = advance ? 1 : 0;
    a.xn_out = c->scr.xn;
    a.xn_dst = c->state;
    L.kind = "gemv_head_argmax";
    // the next token of a context with layers starts with its first layer's
    // Q/K/V projection (or gate/up, for a span that starts at an FFN half)
    const DevMat *nx = nullptr;
    if (!c->layers.empty())
        nx = c->layers[0].ha ? &c->layers[0].qkv[0] : (c->layers[0].gu_fused ? &c->layers[0].gu : &c->layers[0].g);
    enqueue_gemv(L, c->sms, c->out, c->state, c->out_norm, g.eps, c->logits, EPI_ARGMAX, c->scr, a, nx,
                 EPI_STORE);
}

// Kernels of one step of the stage: nl layers (LAYERS/FULL) from layer 0.
static void enqueue_step(ecu_ctx *c, Launcher &L, int nl)
{
    if (r_emb(c)) {
        L.kind = "embed";
        L.bytes = 8.0 * c->g.n_embd + (double)ecu_type_nbytes(c->emb.type, (size_t)c->g.n_embd);
        L(k_embed, dim3(8), dim3(256), 0, c->emb, c->st, c->state, c->g.n_embd);
    }
    if (r_lay(c))
        for (int i = 0; i < nl; i++) enqueue_layer(c, L, i, nl);
    if (r_pos(c) && !r_head(c)) {
        L.kind = "step_advance";
        L(k_step_advance, dim3(1), dim3(32), 0, c->st);
    }
    if (r_head(c)) enqueue_head(c, L, r_pos(c));
}

static int n_stage_layers(const ecu_ctx *c)
{
    return r_lay(c) ? c->last - c->first + 1 : 0;
}

static int mega_launch(ecu_ctx *c, cudaStream_t s, unsigned long long *phase_ns,
                       unsigned long long *detail = nullptr);

// Enqueue one full step: the persistent kernel when the stage has one, else
// a graph replay when enabled (captured on first use).
static int run_step(ecu_ctx *c)
{
    if (c->mega) {
        if (mega_launch(c, c->stream, nullptr) != 0) return -1;
        g_launches += 1;
        return 0;
    }
    if (c->use_graph) {
        if (!c->graph) {
            cudaGraph_t gr;
            CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
            Launcher L{c->stream, c->pdl};
            enqueue_step(c, L, n_stage_layers(c));
            cudaError_t e = cudaStreamEndCapture(c->stream, &gr);
            if (L.err != cudaSuccess || e != cudaSuccess) {
                ecu_set_error(nullptr, 0, "graph capture failed: %s",
                              cudaGetErrorString(L.err != cudaSuccess ? L.err : e));
                if (e == cudaSuccess) cudaGraphDestroy(gr);
                return -1;
            }
            e = cudaGraphInstantiate(&c->graph, gr, 0);
            cudaGraphDestroy(gr);
            if (e != cudaSuccess) {
                ecu_set_error(nullptr, 0, "graph instantiate failed: %s", cudaGetErrorString(e));
                c->graph = nullptr;
                return -1;
            }
            c->graph_kernels = L.count;
        }
        CK(cudaGraphLaunch(c->graph, c->stream));
        g_launches += (uint64_t)c->graph_kernels;
        return 0;
    }
    Launcher L{c->stream, c->pdl};
    enqueue_step(c, L, n_stage_layers(c));
    g_launches += (uint64_t)L.count;
    if (L.err != cudaSuccess) {
        ecu_set_error(nullptr, 0, "kernel launch failed: %s", cudaGetErrorString(L.err));
        return -1;
    }
    return 0;
}

static int check_status(ecu_ctx *c)
{
    // the step state comes back with the step's other results: one async
    // copy into the pinned slot past the position slots, one synchronisation
    StepState *hs = c->h_st + c->n_hslots;
    CK(cudaMemcpyAsync(hs, c->st, sizeof(StepState), cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    const StepState s = *hs;
    if (s.status) {
        if (c->mega) {
            // counters and launch number restart at zero: the tagged vectors
            // must not hold words of an earlier launch with the same number
            CK(cudaMemset(c->margs.bar, 0, (4 + (size_t)c->g.n_head_kv) * sizeof(unsigned)));
            CK(cudaMemset(c->mega_ll, 0, c->mega_ll_words * sizeof(unsigned long long)));
        }
        if (s.status & ECU_STATUS_BADTOKEN)
            ecu_set_error(nullptr, 0, "the device-resident token is outside the vocabulary (%d)", c->g.n_vocab);
        else
            ecu_set_error(nullptr, 0, "a kernel gave up on a bounded wait (status %d)", s.status);
        CK(cudaMemset(&c->st->status, 0, sizeof(int)));
        return -1;
    }
    return 0;
}

// Run `enq` on the context's stream ordered after the caller's stream s, and
// order s after it.
template <class F> static int on_stream(ecu_ctx *c, void *stream, F enq)
{
    cudaStream_t s = stream ? (cudaStream_t)stream : c->stream;
    if (s == c->stream) return enq();
    cudaEvent_t ev;
    CK(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    CK(cudaEventRecord(ev, s));
    CK(cudaStreamWaitEvent(c->stream, ev, 0));
    if (enq() != 0) { cudaEventDestroy(ev); return -1; }
    CK(cudaEventRecord(ev, c->stream));
    CK(cudaStreamWaitEvent(s, ev, 0));
    cudaEventDestroy(ev);
    return 0;
}

// ------------------------------------------------ persistent step kernel --

typedef void (*MegaFn)(MegaArgs);

// sys: the tagged words cross GPUs (tensor-parallel ranks): system scope
static MegaFn mega_lookup(int hd, int rep, bool sys)
{
    if (hd == 128 && rep == 4) return sys ? k_decode_mega<128, 4, true> : k_decode_mega<128, 4, false>;
    if (hd == 128 && rep == 8) return sys ? k_decode_mega<128, 8, true> : k_decode_mega<128, 8, false>;
    if (hd == 64 && rep == 4) return sys ? k_decode_mega<64, 4, true> : k_decode_mega<64, 4, false>;
    return nullptr;
}

static size_t mega_smem_total(int red_floats, unsigned ring_bytes, unsigned union_bytes, int n_ph)
{
    return mega_smem_plan(red_floats, ring_bytes, union_bytes, n_ph).total;
}

// Q4_0 rows in SPLIT4, Q8_0 rows in SPLIT8 or Q4_K rows in SPLITK4, n_in
// (of a column segment) a multiple of 1024.
static bool mega_mat_ok(const DevMat &m)
{
    const DevMat v = m.nseg > 1 ? seg_view(m, 0) : m;
    return fast_ok(v) && v.n_in / 32 <= MEGA_MAX_NB && v.row_bytes <= MEGA_RING_BYTES / 2 &&
           ((v.type == GT_Q4_0 && v.layout == LAY_SPLIT4) || (v.type == GT_Q8_0 && v.layout == LAY_SPLIT8) ||
            (v.type == GT_Q4_K && v.layout == LAY_SPLITK4));
}

static MegaPhase mega_gemv_phase(const DevMat &m, int grid, unsigned stage_bytes, int norm, int epi,
                                 const float *x, const float *norm_w, float *y, float *xn)
{
    MegaPhase p = {};
    p.kind = PH_GEMV;
    p.fmt = m.layout == LAY_SPLIT4 ? 4 : m.layout == LAY_SPLITK4 ? 12 : 8;
    p.norm = norm;
    p.epi = epi;
    p.in_ep = p.y_ep = -1;                           // plain input / residual unless set
    p.w = m.data;
    p.row_bytes = (unsigned)m.row_bytes;
    p.n_in = m.n_in;
    p.n_out = m.n_out;
    int rpc = (m.n_out + grid - 1) / grid;
    if (epi == EPI_SWIGLU && (rpc & 1)) rpc++;        // whole gate/up pairs per CTA
    p.rpc = rpc;
    p.nkg = m.n_in / 1024;
    p.rowpar = std::max(1, MEGA_NCW / p.nkg);
    // rows per stage: as many as the stage holds (bytes in flight matter more
    // than a partly empty last batch of 4 rows)
    p.sr = (int)std::min<size_t>((size_t)rpc, stage_bytes / m.row_bytes);
    p.x = x;
    p.norm_w = norm_w;
    p.y = y;
    p.xn = xn;
    return p;
}

// Build the phase list and buffers of the persistent kernel when the stage
// qualifies (every projection fused and in a fast layout, an instantiated
// head geometry, cooperative launch, the shared-memory plan fits).  Leaves
// c->mega false otherwise: the per-kernel step serves the stage.
static int mega_setup(ecu_ctx *c)
{
    c->mega = false;
    auto no = [c](const char *why) {
        c->path = std::string("kernels: ") + why;
        return 0;
    };
    // ECU_MEGA=0 selects the per-kernel step
    const char *env = getenv("ECU_MEGA");
    if (env && env[0] == '0') return no("ECU_MEGA=0");
    // a stage with layers, or a span of the head alone
    if (!(r_lay(c) && !c->layers.empty()) && !(c->stage == ECU_STAGE_SPAN && r_head(c)))
        return no("stage without layers");
    const EcuGeom &g = c->g;
    const TpSlice &tp = c->tp;
    // this rank's query and KV heads (all of them without tensor parallelism)
    const int hd = g.head_dim, qdim = g.n_head * hd, qd_l = tp.nh * hd, kvd_l = tp.nkv * hd;
    const bool bcast = tp.world > 1;          // outputs every rank reads go to every rank
    MegaFn fn = mega_lookup(hd, g.n_rep, bcast);
    if (!fn) return no("head_dim / query heads per KV head not instantiated");
    // the weight matrices of a layer's halves on this context
    auto layer_mats = [](const LayerDev &ly) {
        std::vector<const DevMat *> v;
        if (ly.ha) { v.push_back(&ly.qkv[0]); v.push_back(&ly.o); }
        if (ly.hf) { v.push_back(&ly.gu); v.push_back(&ly.d); }
        return v;
    };
    for (auto &ly : c->layers) {
        if ((ly.ha && ly.qkv.size() != 1) || (ly.hf && !ly.gu_fused))
            return no("a layer's Q/K/V or gate/up are not fused");
        for (const DevMat *m : layer_mats(ly))
            if (!mega_mat_ok(*m)) return no("a layer matrix is not Q4_0/Q8_0/Q4_K in a fast layout");
    }
    const bool emb = r_emb(c), full = r_head(c);        // (full: the step ends with the head)
    if (full && !mega_mat_ok(c->out)) return no("output head not Q4_0/Q8_0/Q4_K in a fast layout");
    int coop = 0;
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, c->device);
    if (!coop) return no("no cooperative launch");
    const int grid = c->sms;
    // ring geometry: ECU_MEGA_RING stages (default 2) over ECU_MEGA_RING_KB
    // KB (default MEGA_RING_BYTES)
    int nst = 2;
    if (const char *r = getenv("ECU_MEGA_RING")) nst = std::max(2, std::min(MEGA_MAX_STAGES, atoi(r)));
    size_t ring_total = MEGA_RING_BYTES;
    if (const char *r = getenv("ECU_MEGA_RING_KB")) ring_total = (size_t)std::max(32, std::min(200, atoi(r))) * 1024;
    if (nst > MEGA_MAX_STAGES) return no("too many ring stages");
    unsigned stage_bytes = (unsigned)(ring_total / nst) & ~127u;
    // (row_bytes and n_in / nseg are those of a column segment)
    for (auto &ly : c->layers)
        for (const DevMat *m : layer_mats(ly))
            if (m->row_bytes > stage_bytes) return no("a weight row does not fit a ring stage");
    if (full && c->out.row_bytes > stage_bytes) return no("a head row does not fit a ring stage");
    // the shared-memory union: the digit planes of the widest GEMV input, or
    // the attention K/V buffers; the split partials of a head group, which
    // the merge gathers there, set the position splits per KV head (one
    // item per CTA at most)
    size_t un = (size_t)g.n_embd / 32 * 28 * sizeof(int);
    for (auto &ly : c->layers)
        for (const DevMat *m : layer_mats(ly))
            un = std::max(un, (size_t)(m->n_in / m->nseg) / 32 * 28 * sizeof(int));
    if (full) un = std::max(un, (size_t)c->out.n_in / 32 * 28 * sizeof(int));
    // attention K/V buffers: two slots (each round's copies overlap the
    // previous round's arithmetic) when the GEMV side of the union already
    // holds two slots of >= 20 rows a buffer, else one slot of MEGA_ATT_SUB
    // rows (ECU_MEGA_ATT=1 / 2 forces one / two slots)
    const size_t row4 = (size_t)4 * hd * sizeof(float);      // a row in each of a slot's 4 buffers
    int att_nsl = 1, att_sub = MEGA_ATT_SUB;
    const int sub2 = (int)std::min<size_t>(32, un / (2 * row4)) & ~1;
    const char *ae = getenv("ECU_MEGA_ATT");
    if (ae && ae[0] == '2') {
        att_nsl = 2;
        att_sub = std::max(sub2, MEGA_ATT_SUB);
    } else if (!(ae && ae[0] == '1') && sub2 >= 20) {
        att_nsl = 2;
        att_sub = sub2;
    }
    // ECU_MEGA_KV_EARLY=1: the first attention rounds' K/V copies are issued
    // by the Q/K/V phase before it, into buffers above the widest Q/K/V digit
    // planes (measured on the 8B shape: the attention phase gains less than
    // the Q/K/V phase loses to the extra copies in its stream, so by default
    // the attention phase issues them itself)
    const char *ke = getenv("ECU_MEGA_KV_EARLY");
    const bool  kv_early = ke && ke[0] == '1';
    size_t qkv_dig = 0;
    for (auto &ly : c->layers)
        if (ly.ha) qkv_dig = std::max(qkv_dig, (size_t)ly.qkv[0].n_in / 32 * 28 * sizeof(int));
    const size_t kv_off = kv_early ? ((qkv_dig + 127) & ~(size_t)127) : 0;
    un = std::max(un, kv_off + (size_t)att_nsl * att_sub * row4);
    // the attention's position-group sums (at the union's base): [512 / (hd/4)][n_rep][hd] floats
    un = std::max(un, (size_t)(MEGA_THREADS / (hd / 4)) * g.n_rep * hd * sizeof(float));
    // (counted over all KV heads of the model, so that a tensor-parallel
    // rank splits each head's positions exactly as one GPU does: the merge
    // then adds the same partials in the same order, bit for bit)
    int n_split = std::min(MEGA_MAX_SPLIT, grid / g.n_head_kv);
    if (const char *se = getenv("ECU_MEGA_SPLIT")) n_split = std::max(1, std::min(n_split, atoi(se)));
    n_split = std::max(1, std::min(n_split, g.n_ctx));

    std::vector<MegaPhase> ph;
    c->ph_kind.clear();
    c->ph_bytes.clear();
    auto add = [&](const MegaPhase &p, const char *kind, double bytes) {
        ph.push_back(p);
        c->ph_kind.push_back(kind);
        c->ph_bytes.push_back(bytes);
    };
    c->to_shared = false;
    float *xn_tmp = full ? c->dalloc<float>((size_t)g.n_embd + 4) : nullptr;
    // tagged vectors: residual stream, fused Q/K/V, attention output, SwiGLU
    // output; 4-word padded so every vector starts 32-byte aligned
    // (+ the argmax exchange of tensor-parallel ranks: a value and an index
    // word per rank); the same layout on every rank
    auto pad4 = [](size_t n) { return (n + 7) & ~(size_t)3; };
    // (+ this rank's attention split partials: per KV head, split and query
    // head the hd unnormalised sums, the running max and the weight sum)
    const size_t w_x = pad4(g.n_embd), w_qkv = pad4((size_t)qd_l + 2 * kvd_l), w_att = pad4(qdim),
                 w_h = pad4(g.n_ff), w_arg = pad4(2 * ECU_MAX_TP),
                 w_apart = pad4((size_t)tp.nkv * n_split * g.n_rep * (hd + 2));
    // (+ the token word a pipeline link delivers, right after the residual
    // stream: at the same offset in every context of the model)
    const size_t w_tok = 4;
    c->mega_ll_words = w_x + w_tok + w_qkv + w_att + w_h + w_arg + w_apart;
    c->mega_ll = c->dalloc<unsigned long long>(c->mega_ll_words);
    if (!c->mega_ll) return -1;
    CK(cudaMemset(c->mega_ll, 0, c->mega_ll_words * sizeof(unsigned long long)));
    unsigned long long *x_ll = c->mega_ll, *tok_ll = x_ll + w_x, *qkv_ll = tok_ll + w_tok, *att_ll = qkv_ll + w_qkv,
                       *h_ll = att_ll + w_att, *arg_ll = h_ll + w_h, *apart_ll = arg_ll + w_arg;
    // x_w: the phase that last wrote the residual stream (-1: the plain
    // input state of a LAYERS stage)
    int x_w = -1;
    if (emb) {
        MegaPhase p = {};
        p.kind = PH_EMBED;
        p.y_ll = x_ll;
        x_w = (int)ph.size();
        add(p, "embed", 8.0 * g.n_embd + (double)ecu_type_nbytes(c->emb.type, (size_t)g.n_embd));
    }
    // a residual-adding GEMV (attn_output, ffn_down): one phase per column
    // segment, each adding its W_s x_s to the residual the previous one wrote
    auto add_resid = [&](const DevMat &m, const char *kind, const float *x, unsigned long long *xin, int in_ep,
                         int out_plain) {
        for (int si = 0; si < m.nseg; si++) {
            const DevMat v = m.nseg > 1 ? seg_view(m, si) : m;
            MegaPhase    p = mega_gemv_phase(v, grid, stage_bytes, 0, EPI_ADD, x + (size_t)si * v.n_in, nullptr,
                                             c->state, nullptr);
            p.in_ep = in_ep;
            p.x_ll = xin + (size_t)si * v.n_in;
            p.y_ep = x_w;
            p.y_ll = x_ll;
            p.out_base = tp.rank * tp.ne;
            p.bcast = bcast;
            p.out_plain = si + 1 == m.nseg ? out_plain : 0;
            x_w = (int)ph.size();
            add(p, kind, gemv_bytes(v, EPI_ADD));
        }
    };
    const size_t plane = (size_t)tp.nkv * g.n_ctx * hd;
    for (size_t li = 0; li < c->layers.size(); li++) {
        LayerDev &ly = c->layers[li];
        if (ly.ha) {
            MegaPhase q = mega_gemv_phase(ly.qkv[0], grid, stage_bytes, 1, EPI_STORE, c->state, ly.attn_norm, c->qkv,
                                          nullptr);
            q.kc = c->kc + li * plane;              // the next attention's cache planes (early K/V copies)
            q.vc = c->vc + li * plane;
            q.in_ep = x_w;
            q.x_ll = x_ll;
            q.y_ll = qkv_ll;
            const int p_qkv = (int)ph.size();
            add(q, "gemv_qkv", gemv_bytes(ly.qkv[0], EPI_STORE));
            MegaPhase at = {};
            at.kind = PH_ATTN;
            at.kc = c->kc + li * plane;
            at.vc = c->vc + li * plane;
            at.bq = ly.bq;
            at.bk = ly.bk;
            at.bv = ly.bv;
            at.in_ep = p_qkv;
            at.y_ll = att_ll + (size_t)tp.rank * qd_l;   // this rank's heads of the whole vector
            at.bcast = bcast;
            const int p_at = (int)ph.size();
            add(at, "attention", -1.0);             // position dependent: filled in by the profile
            add_resid(ly.o, "gemv_o", c->att, att_ll, p_at, 0);
        }
        if (ly.hf) {
            MegaPhase gu = mega_gemv_phase(ly.gu, grid, stage_bytes, 1, EPI_SWIGLU, c->state, ly.ffn_norm, c->h,
                                           nullptr);
            gu.in_ep = x_w;
            gu.x_ll = x_ll;
            gu.y_ll = h_ll;
            gu.out_base = tp.rank * tp.ff;
            gu.bcast = bcast;
            const int p_gu = (int)ph.size();
            add(gu, "gemv_gate_up", gemv_bytes(ly.gu, EPI_SWIGLU));
            add_resid(ly.d, "gemv_down", c->h, h_ll, p_gu, 0);
        }
    }
    // without the head, the last residual phase also writes the stage's
    // output state in plain floats
    if (!full)
        for (size_t i = ph.size(); i-- > 0;)
            if (ph[i].kind == PH_GEMV && ph[i].epi == EPI_ADD) {
                ph[i].out_plain = 1;
                break;
            }
    if (full) {
        MegaPhase hp = mega_gemv_phase(c->out, grid, stage_bytes, 1, EPI_ARGMAX, c->state, c->out_norm, c->logits, xn_tmp);
        hp.in_ep = x_w;
        hp.x_ll = x_ll;
        add(hp, "gemv_head_argmax", gemv_bytes(c->out, EPI_ARGMAX) + 4.0 * g.n_embd);
    }
    if (ph.size() >= 4095) return no("more phases than the tagged vectors' epochs count");
    c->ph_in_ep.clear();
    for (const MegaPhase &q : ph) c->ph_in_ep.push_back(q.kind == PH_GEMV ? q.in_ep : -1);
    for (size_t i = 0; i + 1 < ph.size(); i++) ph[i].next_attn = ph[i + 1].kind == PH_ATTN ? 1 : 0;
    // row partials of a whole phase (Q4_0 phases keep 4 per row and k-group
    // when they fit); attention keeps its position groups' partials there
    const char *r4 = getenv("ECU_MEGA_RED4");
    const bool use_red4 = !(r4 && r4[0] == '0');
    int red = MEGA_NCW * (hd + 4);
    for (auto &p : ph)
        if (p.kind == PH_GEMV) {
            p.red4 = (use_red4 && p.fmt == 4 && p.rpc * (p.nkg * 4 + 1) <= MEGA_RED4_MAX) ? 1 : 0;
            red = std::max(red, p.red4 ? p.rpc * (p.nkg * 4 + 1) : p.rpc * p.nkg);
            if (p.epi == EPI_ADD && p.rpc > MEGA_THREADS) return no("residual rows per CTA above the thread count");
        }
    cudaFuncAttributes fa;
    int optin = 0;
    if (cudaFuncGetAttributes(&fa, fn) == cudaSuccess &&
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, c->device) == cudaSuccess &&
        mega_smem_total(red, (unsigned)nst * stage_bytes, (unsigned)un, (int)ph.size()) + fa.sharedSizeBytes > (size_t)optin) {
        // a wide model's digit planes, norm staging and row partials leave
        // less room: shrink the ring stages (1 KB at a time) while every
        // GEMV row still fits one, and refit the phases' rows per stage
        unsigned max_row = 0;
        for (auto &p : ph)
            if (p.kind == PH_GEMV) max_row = std::max(max_row, p.row_bytes);
        while (stage_bytes >= max_row + 1024 &&
               mega_smem_total(red, (unsigned)nst * stage_bytes, (unsigned)un, (int)ph.size()) + fa.sharedSizeBytes > (size_t)optin)
            stage_bytes -= 1024;
        for (auto &p : ph)
            if (p.kind == PH_GEMV) p.sr = (int)std::min<size_t>((size_t)p.rpc, stage_bytes / p.row_bytes);
    }
    cudaGetLastError();
    const size_t smem = mega_smem_total(red, (unsigned)nst * stage_bytes, (unsigned)un, (int)ph.size());
    // the attribute belongs to the kernel function, which every context of
    // the same head geometry shares (stages of different depths need
    // different amounts: the phase table): allow the device's whole opt-in
    // size, so that no context's setting cuts another's launches short
    if (optin == 0 || smem + fa.sharedSizeBytes > (size_t)optin ||
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             optin - (int)fa.sharedSizeBytes) != cudaSuccess) {
        cudaGetLastError();
        static char buf[160];
        snprintf(buf, sizeof buf, "shared memory %zu + %zu B over the %d B limit", smem,
                 (size_t)fa.sharedSizeBytes, optin);
        return no(buf);
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, MEGA_THREADS, smem) != cudaSuccess ||
        per_sm < 1) {
        cudaGetLastError();
        return no("no SM can hold one CTA of the persistent kernel");
    }
    // the ring cursor's phase table (copied into shared memory at launch)
    std::vector<uint4> tab(ph.size());
    for (size_t i = 0; i < ph.size(); i++) {
        const MegaPhase &q = ph[i];
        if (q.kind == PH_GEMV) {
            if (q.row_bytes >= (1u << 20) || q.sr >= (1 << 12) || q.n_out >= (1 << 17) || q.rpc >= (1 << 15))
                return no("a GEMV phase's geometry does not fit the phase table");
            tab[i] = mega_tab_entry(q.w, q.row_bytes, q.sr, q.n_out, q.rpc);
        } else {
            tab[i] = make_uint4(0u, 0u, 0u, 0u);
        }
    }
    uint4 *d_tab = c->dalloc<uint4>(ph.size());
    if (!d_tab) return -1;
    CK(cudaMemcpy(d_tab, tab.data(), tab.size() * sizeof(uint4), cudaMemcpyHostToDevice));
    MegaPhase *d_ph = c->dalloc<MegaPhase>(ph.size());
    float *pval = c->dalloc<float>((size_t)grid);
    int *pidx = c->dalloc<int>((size_t)grid);
    unsigned *ctr = c->dalloc<unsigned>(4 + (size_t)g.n_head_kv);
    if (!d_ph || !pval || !pidx || !ctr || (full && !xn_tmp)) return -1;
    CK(cudaMemcpy(d_ph, ph.data(), ph.size() * sizeof(MegaPhase), cudaMemcpyHostToDevice));
    CK(cudaMemset(ctr, 0, (4 + (size_t)g.n_head_kv) * sizeof(unsigned)));
    c->mega_ph = ph;
    MegaArgs &a = c->margs;
    a = MegaArgs{};
    a.ph = d_ph;
    a.n_ph = (int)ph.size();
    a.tab = d_tab;
    a.emb = c->emb;
    a.state = c->state;
    a.qkv = c->qkv;
    a.att = c->att;
    a.apart_ll = apart_ll;
    a.xn_tmp = xn_tmp;
    a.part_val = pval;
    a.part_idx = pidx;
    a.bar = ctr;
    a.x_ll = x_ll;
    a.qkv_ll = qkv_ll;
    a.att_ll = att_ll;
    a.h_ll = h_ll;
    a.ticket = ctr + 2;
    a.att_ticket = ctr + 4;
    a.st = c->st;
    a.tok_hist = c->tok_hist;
    a.status = &c->st->status;
    a.rope_cs = c->rope_cs;
    a.phase_ns = nullptr;
    a.phase_clk = nullptr;
    a.phase_detail = nullptr;
    a.advance_pos = (full && r_pos(c)) ? 1 : 0;
    a.layers_advance = (!full && r_pos(c)) ? 1 : 0;
    a.n_embd = g.n_embd;
    a.n_head = tp.nh;
    a.n_kv = tp.nkv;
    a.tp_rank = tp.rank;
    a.tp_world = tp.world;
    a.ll_block = c->mega_ll;
    for (int k = 0; k < ECU_MAX_TP; k++) a.peer[k] = k == tp.rank ? c->mega_ll : nullptr;
    a.arg_ll = arg_ll;
    a.vocab_base = tp.v0;
    a.n_ctx = g.n_ctx;
    a.n_split = n_split;
    a.red_floats = red;
    a.union_bytes = (unsigned)un;
    a.nst = nst;
    const char *pfe = getenv("ECU_MEGA_PF");
    a.pf_stages = pfe ? std::max(0, atoi(pfe)) : 0;
    a.stage_bytes = stage_bytes;
    a.att_sub = att_sub;
    a.att_nsl = att_nsl;
    // ECU_MEGA_ATT_L2: 0 no L2 warm-up of the K/V rows, 1 at the end of the
    // Q/K/V phase, 2 (default) at its start
    const char *al2 = getenv("ECU_MEGA_ATT_L2");
    a.att_l2 = (al2 && (al2[0] == '0' || al2[0] == '1')) ? al2[0] - '0' : 2;
    a.att_early = kv_early ? 1 : 0;
    a.stall_phase = -1;
    a.kv_off = (unsigned)kv_off;
    a.tok_ll = tok_ll;
    a.eps = g.eps;
    a.kscale = 1.0f / sqrtf((float)hd);
    c->mega_fn = fn;
    c->mega_grid = grid;
    c->mega_smem = smem;
    c->mega = true;
    c->path = "persistent";
    return 0;
}

// One step: a cooperative launch of the whole-step kernel on s.
// Persistent steps of one device run one after another, whatever stream
// they are enqueued on: the CTAs of a step wait for each other's words, so
// two steps whose CTAs shared the SMs (neither wholly resident) could only
// end by their bounded waits running out.  Each launch waits for the
// device's previous one (an event; free when both are on one stream).
static std::mutex  g_mega_mu;
static cudaEvent_t g_mega_ev[64] = {};

static cudaError_t mega_launch_serial(int device, const cudaLaunchConfig_t &cfg, MegaFn fn, const MegaArgs &a)
{
    std::lock_guard<std::mutex> lk(g_mega_mu);
    cudaEvent_t *ev = (device >= 0 && device < 64) ? &g_mega_ev[device] : nullptr;
    if (ev && !*ev && cudaEventCreateWithFlags(ev, cudaEventDisableTiming) != cudaSuccess) *ev = nullptr;
    if (ev && *ev) {
        const cudaError_t w = cudaStreamWaitEvent(cfg.stream, *ev, 0);
        if (w != cudaSuccess) return w;
    }
    const cudaError_t e = cudaLaunchKernelEx(&cfg, fn, a);
    if (e == cudaSuccess && ev && *ev) return cudaEventRecord(*ev, cfg.stream);
    return e;
}

static int mega_launch(ecu_ctx *c, cudaStream_t s, unsigned long long *phase_ns, unsigned long long *detail)
{
    if (c->tp.world > 1 && (int)c->tp_peers.size() != c->tp.world - 1) {
        ecu_set_error(nullptr, 0, "tensor-parallel rank %d is not connected to its peers (ecu_tp_connect)", c->tp.rank);
        return -1;
    }
    MegaArgs a = c->margs;
    a.stall_phase = c->stall_next;          // one launch only
    c->stall_next = -1;
    a.phase_ns = phase_ns;
    a.phase_clk = phase_ns ? phase_ns + a.n_ph + 1 : nullptr;   // the profile buffer's second row
    a.phase_detail = detail;
    cudaLaunchConfig_t  cfg = {};
    cudaLaunchAttribute at;
    cfg.gridDim = dim3((unsigned)c->mega_grid);
    cfg.blockDim = dim3(MEGA_THREADS);
    cfg.dynamicSmemBytes = c->mega_smem;
    cfg.stream = s;
    at.id = cudaLaunchAttributeCooperative;
    at.val.cooperative = 1;
    cfg.attrs = &at;
    cfg.numAttrs = 1;
    cudaError_t e = mega_launch_serial(c->device, cfg, c->mega_fn, a);
    if (e != cudaSuccess) {
        ecu_set_error(nullptr, 0, "persistent step launch failed: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

// Profiling replay of the persistent kernel: CUDA events around each launch
// ("decode_step") and CTA 0's exit time of every grid barrier, attributed to
// the phase that ended there.
static int mega_profile(ecu_ctx *c, int n_steps, ecu_kprof *out, int max_kinds)
{
    const int np = c->margs.n_ph;
    unsigned long long *d_ns = nullptr;
    // [np + 1] global ns, [np + 1] CTA 0's SM clock at the same points, [np][4] detail
    const size_t nbuf = 2 * ((size_t)np + 1) + 4 * (size_t)np;
    CK(cudaMalloc(&d_ns, sizeof(unsigned long long) * nbuf));
    CK(cudaMemset(d_ns, 0, sizeof(unsigned long long) * nbuf));
    std::vector<unsigned long long> ns(nbuf);
    unsigned long long *d_det = d_ns + 2 * (np + 1);
    int nk = 0;
    auto slot = [&](const char *kind, double bytes) -> ecu_kprof * {
        int k = 0;
        while (k < nk && strncmp(out[k].kind, kind, sizeof out[k].kind) != 0) k++;
        if (k == nk) {
            if (nk == max_kinds) return nullptr;
            memset(&out[k], 0, sizeof out[k]);
            snprintf(out[k].kind, sizeof out[k].kind, "%s", kind);
            out[k].bytes_per_launch = bytes;
            nk++;
        }
        return &out[k];
    };
    const EcuGeom &g = c->g;
    const int kvdim = g.n_head_kv * g.head_dim, qdim = g.n_head * g.head_dim;
    int rc = 0;
    for (int i = 0; i < n_steps && rc == 0; i++) {
        cudaEvent_t e0, e1;
        cudaEventCreate(&e0);
        cudaEventCreate(&e1);
        cudaEventRecord(e0, c->stream);
        rc = mega_launch(c, c->stream, d_ns, d_det);
        cudaEventRecord(e1, c->stream);
        g_launches += 1;
        if (rc == 0 && check_status(c) != 0) rc = -1;
        float ms = 0;
        cudaEventElapsedTime(&ms, e0, e1);
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        if (rc != 0) break;
        cudaMemcpy(ns.data(), d_ns, ns.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
        const double att_bytes = 2.0 * 4.0 * kvdim * (c->pos + 2) + 8.0 * qdim + 4.0 * (qdim + 2 * kvdim);
        double step_bytes = 0;
        for (int p = 0; p < np; p++) {
            const double b = c->ph_bytes[p] < 0 ? att_bytes : c->ph_bytes[p];
            step_bytes += b;
            if (ecu_kprof *k = slot(c->ph_kind[p], b)) {
                k->launches++;
                k->total_ms += (double)(ns[p + 1] - ns[p]) * 1e-6;
                if (c->ph_bytes[p] < 0) k->bytes_per_launch = b;
            }
            // GEMV phases: where CTA 0 spent the phase (barrier + prologue,
            // main loop, waiting for ring stages inside it, epilogue)
            const unsigned long long *dt = ns.data() + 2 * ((size_t)np + 1) + 4 * (size_t)p;
            const unsigned long long *clk = ns.data() + np + 1;
            // CTA 0's SM cycles per ns over this launch
            const double f = (double)(clk[np] - clk[0]) / (double)std::max<unsigned long long>(1, ns[np] - ns[0]);
            if (dt[0] && dt[1] && dt[2]) {
                // attention phases: [3] is when KV head 0's merge ended
                const bool att = c->ph_bytes[p] < 0;
                const char *part[4] = {"prologue", "main", "epilogue", att ? "merged" : "ring_wait"};
                const double v[4] = {(double)(dt[0] - clk[p]) / f, (double)(dt[1] - dt[0]) / f,
                                     (double)(dt[2] - dt[1]) / f,
                                     att ? (dt[3] > ns[p] ? (double)(dt[3] - ns[p]) : 0.0) : (double)dt[3]};
                for (int q = 0; q < 4; q++) {
                    char nm[32];
                    snprintf(nm, sizeof nm, "%.20s:%s", c->ph_kind[p], part[q]);
                    if (ecu_kprof *k = slot(nm, 0.0)) {
                        k->launches++;
                        k->total_ms += v[q] * 1e-6;
                    }
                }
            }
        }
        if (ecu_kprof *k = slot("decode_step", step_bytes)) {
            k->launches++;
            k->total_ms += ms;
            k->bytes_per_launch = step_bytes;
        }
        c->pos++;
    }
    cudaFree(d_ns);
    return rc == 0 ? nk : -1;
}

// ----------------------------------------------------------------- C ABI --

extern "C" {

const char *ecu_last_error(void) { return ecu_get_error(); }
uint64_t    ecu_kernel_launches(void) { return g_launches.load(); }
const char *ecu_version(void) { return "distcomp-b200 0.1 (sm_100a)"; }

int ecu_model_open(ecu_model **out, const void *file, size_t size, char *err, size_t errlen)
{
    if (!out || !file) { ecu_set_error(err, errlen, "null argument"); return -1; }
    ecu_model *m = new ecu_model();
    if (ecu_model_parse(m, file, size, err, errlen) != 0) {
        delete m;
        *out = nullptr;
        return -1;
    }
    *out = m;
    return 0;
}

int ecu_model_open_file(ecu_model **out, const char *path, char *err, size_t errlen)
{
    if (!out || !path) { ecu_set_error(err, errlen, "null argument"); return -1; }
    *out = nullptr;
    const int fd = open(path, O_RDONLY);
    if (fd < 0) { ecu_set_error(err, errlen, "cannot open %s: %s", path, strerror(errno)); return -1; }
    struct stat sb;
    if (fstat(fd, &sb) != 0 || sb.st_size <= 0) {
        ecu_set_error(err, errlen, "cannot size %s", path);
        close(fd);
        return -1;
    }
    const size_t len = (size_t)sb.st_size;
    void *p = mmap(nullptr, len, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (p == MAP_FAILED) { ecu_set_error(err, errlen, "cannot map %s: %s", path, strerror(errno)); return -1; }
    ecu_model *m = new ecu_model();
    m->map = p;
    m->map_len = len;
    if (ecu_model_parse(m, p, len, err, errlen) != 0) {
        delete m;
        return -1;
    }
    *out = m;
    return 0;
}

ecu_model *ecu_model_new(void) { return new ecu_model(); }

static int set_kv(ecu_model *m, const char *key, unsigned type, double num, const char *str)
{
    if (!m || !key) return -1;
    for (auto &k : m->kv)
        if (k.key == key) { k.type = type; k.num = num; k.str = str ? str : ""; return 0; }
    EcuKv k;
    k.key = key;
    k.type = type;
    k.num = num;
    if (str) k.str = str;
    m->kv.push_back(k);
    return 0;
}

int ecu_model_set_str(ecu_model *m, const char *key, const char *val) { return set_kv(m, key, 8, 0, val); }
int ecu_model_set_u32(ecu_model *m, const char *key, unsigned long v) { return set_kv(m, key, 4, (double)v, nullptr); }
int ecu_model_set_f32(ecu_model *m, const char *key, float v) { return set_kv(m, key, 6, (double)v, nullptr); }

int ecu_model_add_tensor(ecu_model *m, const char *name, unsigned n_dims, const uint64_t *dims,
                         unsigned ggml_type, const void *data, size_t nbytes)
{
    if (!m || !name || n_dims > 4 || (n_dims && !dims)) {
        ecu_set_error(nullptr, 0, "ecu_model_add_tensor: bad arguments");
        return -1;
    }
    EcuTensor t;
    t.name = name;
    t.n_dims = n_dims;
    for (unsigned i = 0; i < n_dims; i++) t.dims[i] = dims[i];
    t.type = ggml_type;
    t.data = (const uint8_t *)data;
    t.nbytes = nbytes;
    size_t want = ecu_type_nbytes(ggml_type, t.elems());
    if (want && nbytes < want) {
        ecu_set_error(nullptr, 0, "tensor %s: %zu bytes given, %zu needed", name, nbytes, want);
        return -1;
    }
    m->t.push_back(t);
    m->index();
    return 0;
}

void ecu_model_close(ecu_model *m) { delete m; }
size_t ecu_model_n_tensors(const ecu_model *m) { return m ? m->t.size() : 0; }

int ecu_model_tensor(const ecu_model *m, const char *name, unsigned *type, unsigned *n_dims,
                     uint64_t dims[4], const void **data, size_t *nbytes)
{
    const EcuTensor *t = m ? m->find(name) : nullptr;
    if (!t) return -1;
    if (type) *type = t->type;
    if (n_dims) *n_dims = t->n_dims;
    if (dims) for (int i = 0; i < 4; i++) dims[i] = t->dims[i];
    if (data) *data = t->data;
    if (nbytes) *nbytes = t->nbytes;
    return 0;
}

// Tensors a stage needs and their check (src/engine.c:169-213).
struct StageTensors {
    const EcuTensor *emb = nullptr, *out_norm = nullptr, *out = nullptr;
    struct L { const EcuTensor *an, *q, *k, *v, *o, *fn, *g, *u, *d, *bq, *bk, *bv; bool ha, hf; };
    std::vector<L> layers;
};

static int stage_tensors(const ecu_model *m, const EcuGeom &g, int stage, int first, int last,
                         StageTensors *st, char *err, size_t errlen, unsigned span = 0)
{
    const bool sp = stage == ECU_STAGE_SPAN;
    const bool emb = stage == ECU_STAGE_EMBED || stage == ECU_STAGE_FULL || (sp && (span & ECU_SPAN_EMBED));
    const bool head = stage == ECU_STAGE_HEAD || stage == ECU_STAGE_FULL || (sp && (span & ECU_SPAN_HEAD));
    const bool lay = stage == ECU_STAGE_LAYERS || stage == ECU_STAGE_FULL || (sp && first <= last);
    if (sp && (span & ~(ECU_SPAN_EMBED | ECU_SPAN_HEAD | ECU_SPAN_FFN_FIRST | ECU_SPAN_ATTN_LAST))) {
        ecu_set_error(err, errlen, "unknown span flags 0x%x", span);
        return -1;
    }
    if (sp && !lay && !emb && !head) {
        ecu_set_error(err, errlen, "a span of no layers needs the embedding or the head");
        return -1;
    }
    if (lay && (last < first || last >= g.n_layer || first < 0)) {
        ecu_set_error(err, errlen, "layers %d..%d outside the model: it has %d layers", first, last, g.n_layer);
        return -1;
    }
    if ((emb || head) && g.n_vocab <= 0) {
        ecu_set_error(err, errlen, "cannot determine the vocabulary size (n_vocab) for stage %d", stage);
        return -1;
    }
    if (emb) {
        st->emb = m->find("token_embd.weight");
        if (!st->emb) { ecu_set_error(err, errlen, "model has no token_embd.weight"); return -1; }
    }
    if (head) {
        st->out_norm = m->find("output_norm.weight");
        if (!st->out_norm) { ecu_set_error(err, errlen, "model has no output_norm.weight"); return -1; }
        st->out = m->find("output.weight");
        if (!st->out) st->out = m->find("token_embd.weight");
        if (!st->out) { ecu_set_error(err, errlen, "model has neither output.weight nor token_embd.weight"); return -1; }
    }
    if (lay) {
        static const char *sfx[9] = {"attn_norm.weight", "attn_q.weight", "attn_k.weight",
                                     "attn_v.weight", "attn_output.weight", "ffn_norm.weight",
                                     "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight"};
        for (int i = first; i <= last; i++) {
            StageTensors::L l{};
            l.ha = !(sp && i == first && (span & ECU_SPAN_FFN_FIRST));
            l.hf = !(sp && i == last && (span & ECU_SPAN_ATTN_LAST));
            if (!l.ha && !l.hf) {
                ecu_set_error(err, errlen, "layer %d would hold neither its attention nor its FFN half", i);
                return -1;
            }
            const EcuTensor **slot[9] = {&l.an, &l.q, &l.k, &l.v, &l.o, &l.fn, &l.g, &l.u, &l.d};
            char name[160];
            for (int k = 0; k < 9; k++) {
                if ((k < 5 && !l.ha) || (k >= 5 && !l.hf)) continue;      // the half this span leaves out
                snprintf(name, sizeof name, "blk.%d.%s", i, sfx[k]);
                if (!(*slot[k] = m->find(name))) { ecu_set_error(err, errlen, "model has no tensor %s", name); return -1; }
            }
            if (l.ha) {
                snprintf(name, sizeof name, "blk.%d.attn_q.bias", i); l.bq = m->find(name);
                snprintf(name, sizeof name, "blk.%d.attn_k.bias", i); l.bk = m->find(name);
                snprintf(name, sizeof name, "blk.%d.attn_v.bias", i); l.bv = m->find(name);
            }
            st->layers.push_back(l);
        }
    }
    return 0;
}

// The weight matrices must have the shapes the layer loop multiplies by
// (the reference trusts the file; a mismatch there reads past the tensor).
static int check_shape(const EcuTensor *t, int n_in, int n_out, char *err, size_t errlen)
{
    const uint64_t rows = t->n_dims >= 2 ? t->elems() / t->dims[0] : 1;
    if ((int64_t)t->dims[0] != n_in || (int64_t)rows < n_out) {
        ecu_set_error(err, errlen, "tensor %s is %llux%llu, the layer needs %dx%d", t->name.c_str(),
                      (unsigned long long)t->dims[0], (unsigned long long)rows, n_in, n_out);
        return -1;
    }
    return 0;
}

static int attn_supported(int hd, int rep)
{
    return (hd == 16 || hd == 32 || hd == 64 || hd == 128) && (rep == 1 || rep == 2 || rep == 4 || rep == 8);
}

size_t ecu_ctx_bytes(const ecu_model *m, int stage, int first, int last, int n_ctx)
{
    if (!m) return 0;
    EcuGeom g;
    if (ecu_read_geom(m, &g, nullptr, 0) != 0) return 0;
    if (n_ctx > 0) g.n_ctx = n_ctx;
    StageTensors st;
    if (stage_tensors(m, g, stage, first, last, &st, nullptr, 0) != 0) return 0;
    size_t b = 0;
    auto mat = [&](const EcuTensor *t, int n_in, int n_out, bool seg = false) {
        const MatShape sh = mat_shape((int)t->type, n_in, true, seg);
        b += sh.row_bytes * (size_t)n_out * (size_t)sh.nseg;
    };
    const int hd = g.head_dim, qd = g.n_head * hd, kvd = g.n_head_kv * hd;
    for (auto &l : st.layers) {
        mat(l.q, g.n_embd, qd); mat(l.k, g.n_embd, kvd); mat(l.v, g.n_embd, kvd);
        mat(l.o, qd, g.n_embd, true); mat(l.g, g.n_embd, g.n_ff); mat(l.u, g.n_embd, g.n_ff);
        mat(l.d, g.n_ff, g.n_embd, true);
        b += (size_t)(2 * g.n_embd + qd + 2 * kvd) * 4;
    }
    b += 2 * st.layers.size() * (size_t)g.n_ctx * kvd * 4;          // KV cache
    if (st.emb) b += dev_row_bytes((int)st.emb->type, g.n_embd, LAY_RAW) * (size_t)g.n_vocab;
    if (st.out) mat(st.out, g.n_embd, g.n_vocab);
    b += (size_t)g.n_ctx * hd * 4;                                    // RoPE table
    b += (size_t)(4 * g.n_embd + 4 * g.n_ff + 2 * qd + 2 * kvd + g.n_vocab + g.n_ctx) * 4;
    return b;
}

// A context's own device buffers: step state, token history, GEMV scratch,
// pinned host staging, and with layers the activations and the KV cache,
// with a head the logits.  Returns what failed, or nullptr.
static const char *alloc_buffers(ecu_ctx *c, bool layers, bool head)
{
    const EcuGeom &g = c->g;
    const int wide = g.n_ff > g.n_embd ? g.n_ff : g.n_embd;
    const int hd = g.head_dim, qd = g.n_head * hd;
    // this rank's query / KV heads (all of them without tensor parallelism)
    const int qd_l = c->tp.nh * hd, kvd_l = c->tp.nkv * hd;
    c->state = c->dalloc<float>((size_t)g.n_embd + 4);
    c->st = c->dalloc<StepState>(1);
    c->tok_hist = c->dalloc<int>((size_t)g.n_ctx + 1);
    c->scr.xn = c->dalloc<float>((size_t)wide + 4);
    c->scr.part_val = c->dalloc<float>(4096);
    c->scr.part_idx = c->dalloc<int>(4096);
    c->scr.counter = c->dalloc<unsigned>(4);
    c->scr.status = c->st ? &c->st->status : nullptr;
    if (!c->state || !c->st || !c->tok_hist || !c->scr.xn || !c->scr.part_val || !c->scr.part_idx || !c->scr.counter)
        return "work buffers";
    cudaMemset(c->st, 0, sizeof(StepState));
    cudaMemset(c->scr.counter, 0, 4 * sizeof(unsigned));
    cudaMemset(c->state, 0, ((size_t)g.n_embd + 4) * sizeof(float));
    c->n_hslots = g.n_ctx + 1;
    if (cudaMallocHost(&c->h_st, sizeof(StepState) * ((size_t)c->n_hslots + 1)) != cudaSuccess ||
        cudaMallocHost(&c->h_state, ((size_t)g.n_embd + 4) * sizeof(float)) != cudaSuccess)
        return "pinned host staging";
    memset(c->h_st, 0, sizeof(StepState) * ((size_t)c->n_hslots + 1));
    if (head) {
        c->logits = c->dalloc<float>((size_t)(c->tp.v1 - c->tp.v0) + 4);
        if (!c->logits) return "logits";
    }
    if (layers) {
        const size_t nl = (size_t)(c->last - c->first + 1);
        c->qkv = c->dalloc<float>((size_t)qd_l + 2 * kvd_l + 4);
        c->att = c->dalloc<float>((size_t)qd + 4);
        c->h = c->dalloc<float>((size_t)g.n_ff + 4);
        c->gtmp = c->dalloc<float>((size_t)g.n_ff + 4);
        c->utmp = c->dalloc<float>((size_t)g.n_ff + 4);
        const size_t plane = (size_t)c->tp.nkv * g.n_ctx * hd;
        c->kc = c->dalloc<float>(plane * nl);
        c->vc = c->dalloc<float>(plane * nl);
        if (!c->qkv || !c->att || !c->h || !c->gtmp || !c->utmp || !c->kc || !c->vc)
            return "KV cache and layer buffers";
    }
    return nullptr;
}

static int ctx_open_impl(ecu_ctx **out, const ecu_model *m, int stage, int first, int last, int n_ctx,
                         int device, int tp_rank, int tp_world, char *err, size_t errlen, unsigned span = 0);

int ecu_ctx_open(ecu_ctx **out, const ecu_model *m, int stage, int first, int last, int n_ctx,
                 int device, char *err, size_t errlen)
{
    if (err && errlen) err[0] = '\0';
    const int rc = ctx_open_impl(out, m, stage, first, last, n_ctx, device, 0, 1, err, errlen);
    // CUDA failures deep in the upload only set the thread's last error
    if (rc != 0 && err && errlen && !err[0]) snprintf(err, errlen, "%s", ecu_get_error());
    return rc;
}

int ecu_ctx_open_span(ecu_ctx **out, const ecu_model *m, int first, int last, unsigned flags, int n_ctx,
                      int device, char *err, size_t errlen)
{
    if (err && errlen) err[0] = '\0';
    const int rc = ctx_open_impl(out, m, ECU_STAGE_SPAN, first, last, n_ctx, device, 0, 1, err, errlen, flags);
    if (rc != 0 && err && errlen && !err[0]) snprintf(err, errlen, "%s", ecu_get_error());
    return rc;
}

int ecu_ctx_open_tp(ecu_ctx **out, const ecu_model *m, int n_ctx, int device, int tp_rank, int tp_world,
                    char *err, size_t errlen)
{
    if (err && errlen) err[0] = '\0';
    const int rc = ctx_open_impl(out, m, ECU_STAGE_FULL, 0, 0, n_ctx, device, tp_rank, tp_world, err, errlen);
    if (rc != 0 && err && errlen && !err[0]) snprintf(err, errlen, "%s", ecu_get_error());
    return rc;
}

static int ctx_open_impl(ecu_ctx **out, const ecu_model *m, int stage, int first, int last, int n_ctx,
                         int device, int tp_rank, int tp_world, char *err, size_t errlen, unsigned span)
{
    if (!out || !m) { ecu_set_error(err, errlen, "null argument"); return -1; }
    *out = nullptr;
    if (stage < ECU_STAGE_EMBED || stage > ECU_STAGE_SPAN) { ecu_set_error(err, errlen, "unknown stage %d", stage); return -1; }
    EcuGeom g;
    if (ecu_read_geom(m, &g, err, errlen) != 0) return -1;
    if (n_ctx > 0) g.n_ctx = n_ctx;
    if (stage == ECU_STAGE_FULL) { first = 0; last = g.n_layer - 1; }
    if (stage == ECU_STAGE_EMBED || stage == ECU_STAGE_HEAD) { first = 0; last = 0; }
    if (stage == ECU_STAGE_SPAN && first > last) { first = g.n_layer; last = g.n_layer - 1; }   // no layers
    StageTensors st;
    if (stage_tensors(m, g, stage, first, last, &st, err, errlen, span) != 0) return -1;
    const int hd = g.head_dim, qd = g.n_head * hd, kvd = g.n_head_kv * hd;
    if (!st.layers.empty()) {
        if (!attn_supported(hd, g.n_rep)) {
            ecu_set_error(err, errlen, "head_dim %d with %d query heads per KV head is not built", hd, g.n_rep);
            return -1;
        }
        if (hd % 2) { ecu_set_error(err, errlen, "odd head_dim %d", hd); return -1; }
        for (auto &l : st.layers) {
            if (l.ha && (check_shape(l.q, g.n_embd, qd, err, errlen) || check_shape(l.k, g.n_embd, kvd, err, errlen) ||
                         check_shape(l.v, g.n_embd, kvd, err, errlen) || check_shape(l.o, qd, g.n_embd, err, errlen)))
                return -1;
            if (l.hf && (check_shape(l.g, g.n_embd, g.n_ff, err, errlen) ||
                         check_shape(l.u, g.n_embd, g.n_ff, err, errlen) ||
                         check_shape(l.d, g.n_ff, g.n_embd, err, errlen)))
                return -1;
        }
    }
    if (st.out && check_shape(st.out, g.n_embd, g.n_vocab, err, errlen)) return -1;
    TpSlice tp;
    tp.rank = tp_rank;
    tp.world = tp_world;
    if (tp_world < 1 || tp_world > ECU_MAX_TP || tp_rank < 0 || tp_rank >= tp_world) {
        ecu_set_error(err, errlen, "tensor-parallel rank %d of %d", tp_rank, tp_world);
        return -1;
    }
    if (tp_world > 1 && (stage != ECU_STAGE_FULL || g.n_head_kv % tp_world || g.n_ff % tp_world ||
                         g.n_embd % tp_world)) {
        ecu_set_error(err, errlen, "tensor parallelism over %d ranks needs a FULL stage with KV heads, FFN "
                      "width and n_embd divisible by it", tp_world);
        return -1;
    }
    tp.nh = g.n_head / tp_world;
    tp.nkv = g.n_head_kv / tp_world;
    tp.ne = g.n_embd / tp_world;
    tp.ff = g.n_ff / tp_world;
    {
        const int vs = (g.n_vocab + tp_world - 1) / tp_world;
        tp.v0 = std::min(g.n_vocab, tp_rank * vs);
        tp.v1 = std::min(g.n_vocab, tp.v0 + vs);
    }
    if (st.emb && (st.emb->dims[0] != (uint64_t)g.n_embd)) {
        ecu_set_error(err, errlen, "token_embd.weight has %llu inputs, n_embd is %d",
                      (unsigned long long)st.emb->dims[0], g.n_embd);
        return -1;
    }
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
        ecu_set_error(err, errlen, "CUDA device %d not available (%d devices)", device, ndev);
        return -1;
    }
    if (cudaSetDevice(device) != cudaSuccess) { ecu_set_error(err, errlen, "cudaSetDevice(%d) failed", device); return -1; }
    fast_attrs_all();
    attn_attrs_all();
    {
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) { ecu_set_error(err, errlen, "kernel attribute setup failed: %s", cudaGetErrorString(e)); return -1; }
    }

    std::unique_ptr<ecu_ctx, void (*)(ecu_ctx *)> c(new ecu_ctx(), ctx_free);
    c->device = device;
    c->tp = tp;
    c->sms = num_sms(device);
    c->stage = stage;
    c->span = stage == ECU_STAGE_SPAN ? span : 0u;
    c->first = first;
    c->last = last;
    c->g = g;
    const char *e = getenv("ECU_PDL");
    c->pdl = !(e && e[0] == '0');
    e = getenv("ECU_GRAPH");
    c->use_graph = !(e && e[0] == '0');
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&c->ev_step, cudaEventDisableTiming) != cudaSuccess) {
        ecu_set_error(err, errlen, "cudaStreamCreate failed");
        return -1;
    }

    // weight matrices go through pinned double-buffered chunks (ECU_UPLOAD_MB,
    // default 64 MB per buffer); without them (no pinned memory), one
    // pageable copy per tensor into a staging buffer as large as the largest
    size_t up_mb = 64;
    if (const char *ue = getenv("ECU_UPLOAD_MB")) up_mb = (size_t)std::max(1, std::min(1024, atoi(ue)));
    c->up = uploader_new(up_mb << 20);
    size_t stage_bytes = 1 << 20;
    auto need = [&](const EcuTensor *t) { if (t && t->nbytes > stage_bytes) stage_bytes = t->nbytes; };
    need(st.out_norm);
    for (auto &l : st.layers) { need(l.an); need(l.fn); need(l.bq); need(l.bk); need(l.bv); }
    if (!c->up) {
        need(st.emb); need(st.out);
        for (auto &l : st.layers) { need(l.q); need(l.k); need(l.v); need(l.o); need(l.g); need(l.u); need(l.d); }
    }
    uint8_t *stage_buf = nullptr;
    if (cudaMalloc(&stage_buf, stage_bytes + 256) != cudaSuccess ||
        cudaMemset(stage_buf, 0, stage_bytes + 256) != cudaSuccess) {
        ecu_set_error(err, errlen, "out of device memory for a %zu-byte staging buffer", stage_bytes);
        return -1;
    }
    struct Freer { uint8_t *p; ~Freer() { cudaFree(p); } } freer{stage_buf};

    auto fail_oom = [&](const char *what) {
        ecu_set_error(err, errlen, "out of device memory (%s) after %zu bytes", what, c->bytes);
        return -1;
    };
    if (const char *what = alloc_buffers(c.get(), !st.layers.empty(), st.out != nullptr)) return fail_oom(what);
    c->shared = std::make_shared<SharedAllocs>();
    c->shared->device = device;
    c->to_shared = true;

    if (st.emb) {
        c->emb = make_mat(c.get(), (int)st.emb->type, g.n_embd, g.n_vocab, false);
        if (!c->emb.zero && !c->emb.data) return fail_oom("token_embd");
        if (upload_rows(c.get(), st.emb, g.n_embd, g.n_vocab, c->emb, 0, 1, stage_buf)) return -1;
        c->srcs.push_back({"token_embd.weight", c->emb, 0, 1, (size_t)g.n_embd * g.n_vocab, g.n_embd});
    }
    const bool whole = tp.world == 1;    // tensor-parallel ranks hold row slices
    if (st.out) {
        const int nv = tp.v1 - tp.v0;
        c->out = make_mat(c.get(), (int)st.out->type, g.n_embd, nv, true);
        if (!c->out.zero && !c->out.data) return fail_oom("output");
        if (upload_rows(c.get(), st.out, g.n_embd, nv, c->out, 0, 1, stage_buf, (size_t)tp.v0)) return -1;
        c->out_norm = upload_vec(c.get(), st.out_norm, (size_t)g.n_embd, stage_buf);
        if (!c->out_norm) return fail_oom("head buffers");
        if (whole && (st.out->name == "output.weight" || !st.emb))
            c->srcs.push_back({st.out->name, c->out, 0, 1, (size_t)g.n_embd * g.n_vocab, g.n_embd});
    }
    if (!st.layers.empty()) {
        const size_t nl = st.layers.size();
        // position splits per KV head = the cluster size (<= 16, <= one
        // CTA per SM over all heads, all clusters resident at once)
        int max_split = c->sms / g.n_head_kv;
        if (max_split > g.n_ctx) max_split = g.n_ctx;
        if (max_split < 1) max_split = 1;
        c->n_split = attn_cluster(hd, g.n_rep, g.n_head_kv, max_split);
        cudaGetLastError();
        c->rope_cs = c->dalloc<float>((size_t)g.n_ctx * hd);
        if (!c->rope_cs) return fail_oom("RoPE table");
        // RoPE table with the host libm, exactly as src/engine.c:371-373
        {
            std::vector<float> cs((size_t)g.n_ctx * hd);
            const int half = hd / 2;
            for (int p = 0; p < g.n_ctx; p++)
                for (int i = 0; i < half; i++) {
                    float freq = powf(g.rope_base, -2.0f * (float)i / (float)hd);
                    float ang = (float)p * freq;
                    cs[((size_t)p * half + i) * 2] = cosf(ang);
                    cs[((size_t)p * half + i) * 2 + 1] = sinf(ang);
                }
            cudaMemcpy(c->rope_cs, cs.data(), cs.size() * sizeof(float), cudaMemcpyHostToDevice);
        }
        c->layers.resize(nl);
        for (size_t i = 0; i < nl; i++) {
            const auto &l = st.layers[i];
            LayerDev   &ly = c->layers[i];
            char        nm[160];
            const int   li = first + (int)i;
            ly.ha = l.ha;
            ly.hf = l.hf;
            const int  qd_l = tp.nh * hd, kvd_l = tp.nkv * hd;
            if (l.ha) {
                // Q/K/V: fused when all three share a fast layout (a tensor-
                // parallel rank: its heads' rows of each)
                const int lq = choose_layout((int)l.q->type, g.n_embd);
                const bool fuse_qkv = lq != LAY_RAW && l.k->type == l.q->type && l.v->type == l.q->type;
                if (!fuse_qkv && !whole) {
                    ecu_set_error(err, errlen, "tensor parallelism needs Q/K/V of one fast type");
                    return -1;
                }
                if (fuse_qkv) {
                    DevMat mq = make_mat(c.get(), (int)l.q->type, g.n_embd, qd_l + 2 * kvd_l, true);
                    if (!mq.data) return fail_oom("attn_qkv");
                    if (upload_rows(c.get(), l.q, g.n_embd, qd_l, mq, 0, 1, stage_buf, (size_t)tp.rank * qd_l) ||
                        upload_rows(c.get(), l.k, g.n_embd, kvd_l, mq, qd_l, 1, stage_buf, (size_t)tp.rank * kvd_l) ||
                        upload_rows(c.get(), l.v, g.n_embd, kvd_l, mq, qd_l + kvd_l, 1, stage_buf,
                                    (size_t)tp.rank * kvd_l))
                        return -1;
                    ly.qkv.push_back(mq);
                    ly.qkv_off.push_back(0);
                    if (whole) {
                        snprintf(nm, sizeof nm, "blk.%d.attn_q.weight", li); c->srcs.push_back({nm, mq, 0, 1, (size_t)g.n_embd * qd, g.n_embd});
                        snprintf(nm, sizeof nm, "blk.%d.attn_k.weight", li); c->srcs.push_back({nm, mq, qd, 1, (size_t)g.n_embd * kvd, g.n_embd});
                        snprintf(nm, sizeof nm, "blk.%d.attn_v.weight", li); c->srcs.push_back({nm, mq, qd + kvd, 1, (size_t)g.n_embd * kvd, g.n_embd});
                    }
                } else {
                    const EcuTensor *ts[3] = {l.q, l.k, l.v};
                    const int        rows[3] = {qd, kvd, kvd}, offs[3] = {0, qd, qd + kvd};
                    const char      *sf[3] = {"attn_q", "attn_k", "attn_v"};
                    for (int k = 0; k < 3; k++) {
                        DevMat mm = make_mat(c.get(), (int)ts[k]->type, g.n_embd, rows[k], true);
                        if (!mm.zero && !mm.data) return fail_oom("attn_q/k/v");
                        if (upload_rows(c.get(), ts[k], g.n_embd, rows[k], mm, 0, 1, stage_buf)) return -1;
                        ly.qkv.push_back(mm);
                        ly.qkv_off.push_back(offs[k]);
                        snprintf(nm, sizeof nm, "blk.%d.%s.weight", li, sf[k]);
                        c->srcs.push_back({nm, mm, 0, 1, (size_t)g.n_embd * rows[k], g.n_embd});
                    }
                }
                ly.o = make_mat(c.get(), (int)l.o->type, qd, tp.ne, true, true);
                if (!ly.o.zero && !ly.o.data) return fail_oom("attn_output");
                if (upload_rows(c.get(), l.o, qd, tp.ne, ly.o, 0, 1, stage_buf, (size_t)tp.rank * tp.ne)) return -1;
                snprintf(nm, sizeof nm, "blk.%d.attn_output.weight", li);
                if (whole) c->srcs.push_back({nm, ly.o, 0, 1, (size_t)qd * g.n_embd, qd});
                ly.attn_norm = upload_vec(c.get(), l.an, (size_t)g.n_embd, stage_buf);
                // biases whole; a tensor-parallel rank points at its heads' part
                if (l.bq) ly.bq = upload_vec(c.get(), l.bq, (size_t)qd, stage_buf);
                if (l.bk) ly.bk = upload_vec(c.get(), l.bk, (size_t)kvd, stage_buf);
                if (l.bv) ly.bv = upload_vec(c.get(), l.bv, (size_t)kvd, stage_buf);
                if (ly.bq) ly.bq += (size_t)tp.rank * qd_l;
                if (ly.bk) ly.bk += (size_t)tp.rank * kvd_l;
                if (ly.bv) ly.bv += (size_t)tp.rank * kvd_l;
                if (!ly.attn_norm) return fail_oom("norm weights");
            }
            if (l.hf) {
                const int lg = choose_layout((int)l.g->type, g.n_embd);
                ly.gu_fused = lg != LAY_RAW && l.u->type == l.g->type;
                if (!ly.gu_fused && !whole) {
                    ecu_set_error(err, errlen, "tensor parallelism needs gate/up of one fast type");
                    return -1;
                }
                if (ly.gu_fused) {
                    ly.gu = make_mat(c.get(), (int)l.g->type, g.n_embd, 2 * tp.ff, true);
                    if (!ly.gu.data) return fail_oom("ffn_gate/up");
                    if (upload_rows(c.get(), l.g, g.n_embd, tp.ff, ly.gu, 0, 2, stage_buf, (size_t)tp.rank * tp.ff) ||
                        upload_rows(c.get(), l.u, g.n_embd, tp.ff, ly.gu, 1, 2, stage_buf, (size_t)tp.rank * tp.ff))
                        return -1;
                    if (whole) {
                        snprintf(nm, sizeof nm, "blk.%d.ffn_gate.weight", li); c->srcs.push_back({nm, ly.gu, 0, 2, (size_t)g.n_embd * g.n_ff, g.n_embd});
                        snprintf(nm, sizeof nm, "blk.%d.ffn_up.weight", li); c->srcs.push_back({nm, ly.gu, 1, 2, (size_t)g.n_embd * g.n_ff, g.n_embd});
                    }
                } else {
                    ly.g = make_mat(c.get(), (int)l.g->type, g.n_embd, g.n_ff, true);
                    ly.u = make_mat(c.get(), (int)l.u->type, g.n_embd, g.n_ff, true);
                    if ((!ly.g.zero && !ly.g.data) || (!ly.u.zero && !ly.u.data)) return fail_oom("ffn_gate/up");
                    if (upload_rows(c.get(), l.g, g.n_embd, g.n_ff, ly.g, 0, 1, stage_buf) ||
                        upload_rows(c.get(), l.u, g.n_embd, g.n_ff, ly.u, 0, 1, stage_buf))
                        return -1;
                    snprintf(nm, sizeof nm, "blk.%d.ffn_gate.weight", li); c->srcs.push_back({nm, ly.g, 0, 1, (size_t)g.n_embd * g.n_ff, g.n_embd});
                    snprintf(nm, sizeof nm, "blk.%d.ffn_up.weight", li); c->srcs.push_back({nm, ly.u, 0, 1, (size_t)g.n_embd * g.n_ff, g.n_embd});
                }
                ly.d = make_mat(c.get(), (int)l.d->type, g.n_ff, tp.ne, true, true);
                if (!ly.d.zero && !ly.d.data) return fail_oom("ffn_down");
                if (upload_rows(c.get(), l.d, g.n_ff, tp.ne, ly.d, 0, 1, stage_buf, (size_t)tp.rank * tp.ne)) return -1;
                snprintf(nm, sizeof nm, "blk.%d.ffn_down.weight", li);
                if (whole) c->srcs.push_back({nm, ly.d, 0, 1, (size_t)g.n_ff * g.n_embd, g.n_ff});
                ly.ffn_norm = upload_vec(c.get(), l.fn, (size_t)g.n_embd, stage_buf);
                if (!ly.ffn_norm) return fail_oom("norm weights");
            }
        }
    }
    // every chunk uploaded: the pinned staging goes back
    if (c->up) {
        if (cudaStreamSynchronize(c->stream) != cudaSuccess) {
            ecu_set_error(err, errlen, "upload failed: %s", cudaGetErrorString(cudaGetLastError()));
            return -1;
        }
        uploader_free(c->up);
        c->up = nullptr;
    }
    if (mega_setup(c.get()) != 0) return fail_oom("persistent step buffers");
    if (!whole && !c->mega) {
        ecu_set_error(err, errlen, "tensor parallelism runs the persistent step only (%s)", c->path.c_str());
        return -1;
    }
    // setup memsets/copies ran on the legacy stream, which does not order
    // against the context's non-blocking stream: finish them all here
    if (cudaDeviceSynchronize() != cudaSuccess || cudaGetLastError() != cudaSuccess) {
        ecu_set_error(err, errlen, "upload failed: %s", cudaGetErrorString(cudaGetLastError()));
        return -1;
    }
    *out = c.release();
    return 0;
}

void ecu_ctx_close(ecu_ctx *c) { ctx_free(c); }

int ecu_ctx_info(const ecu_ctx *c, ecu_info *i)
{
    if (!c || !i) return -1;
    i->n_layer = c->g.n_layer; i->n_embd = c->g.n_embd; i->n_head = c->g.n_head;
    i->n_head_kv = c->g.n_head_kv; i->n_ff = c->g.n_ff; i->head_dim = c->g.head_dim;
    i->n_vocab = c->g.n_vocab; i->n_rep = c->g.n_rep; i->n_ctx = c->g.n_ctx;
    i->stage = c->stage; i->first = c->first; i->last = c->last; i->pos = c->pos;
    i->device = c->device; i->rms_eps = c->g.eps; i->rope_base = c->g.rope_base;
    i->device_bytes = c->bytes;
    return 0;
}

void ecu_reset(ecu_ctx *c)
{
    if (!c) return;
    c->pos = 0;
    // a linked context's tagged words start over: no word a link wrote for
    // a position of the previous run may look like this run's input
    if (c->mega_ll && (c->linked_in || c->margs.link_x || c->margs.link_tok)) {
        cudaSetDevice(c->device);
        cudaMemsetAsync(c->mega_ll, 0, c->mega_ll_words * sizeof(unsigned long long), c->stream);
        cudaStreamSynchronize(c->stream);
    }
}

int ecu_set_pos(ecu_ctx *c, int pos)
{
    if (!c || pos < 0 || pos > c->g.n_ctx) return -1;
    c->pos = pos;
    return 0;
}

float *ecu_state_ptr(ecu_ctx *c) { return c ? c->state : nullptr; }
const char *ecu_ctx_path(const ecu_ctx *c) { return c ? c->path.c_str() : ""; }
void  *ecu_stream(ecu_ctx *c) { return c ? (void *)c->stream : nullptr; }

// Host-side checks of llm_forward (src/engine.c:468-515) before enqueueing.
static int step_check(ecu_ctx *c, int token)
{
    if (r_emb(c)) {
        if (token < 0 || token >= c->g.n_vocab) {
            ecu_set_error(nullptr, 0, "token %d outside the vocabulary (%d)", token, c->g.n_vocab);
            return -1;
        }
    }
    if (r_pos(c) && c->pos >= c->g.n_ctx) {
        ecu_set_error(nullptr, 0, "context exhausted (%d positions)", c->g.n_ctx);
        return -1;
    }
    return 0;
}

// Enqueue input state + one step on `stream` (the context's own stream).
static int enqueue_forward(ecu_ctx *c, int token)
{
    StepState *slot = c->h_st + (c->pos % c->n_hslots);
    slot->pos = c->pos;
    slot->token = token;
    CK(cudaMemcpyAsync(c->st, slot, 2 * sizeof(int), cudaMemcpyHostToDevice, c->stream));
    if (run_step(c) != 0) return -1;
    if (r_pos(c)) c->pos++;
    if (r_head(c)) c->have_logits = true;
    return 0;
}

int ecu_forward(ecu_ctx *c, int token, float *out)
{
    if (!c || !out) return -1;
    if (c->linked_in) { ecu_set_error(nullptr, 0, "a linked context takes its input over the link (ecu_step_dev)"); return -1; }
    cudaSetDevice(c->device);
    if (step_check(c, token) != 0) return -1;
    const size_t ne = (size_t)c->g.n_embd;
    if (!r_emb(c)) {
        memcpy(c->h_state, out, ne * sizeof(float));
        CK(cudaMemcpyAsync(c->state, c->h_state, ne * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    }
    if (enqueue_forward(c, token) != 0) return -1;
    const size_t nout = r_head(c) ? ne + 1 : ne;
    CK(cudaMemcpyAsync(c->h_state, c->state, nout * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    if (check_status(c) != 0) return -1;
    memcpy(out, c->h_state, nout * sizeof(float));
    if (nout == ne + 1) c->last_pick = (int)c->h_state[ne];
    return 0;
}

int ecu_forward_dev(ecu_ctx *c, int token, void *stream)
{
    if (!c) return -1;
    cudaSetDevice(c->device);
    if (step_check(c, token) != 0) return -1;
    return on_stream(c, stream, [&] { return enqueue_forward(c, token); });
}

int *ecu_token_ptr(ecu_ctx *c) { return c && c->st ? &c->st->token : nullptr; }

int ecu_step_dev(ecu_ctx *c, void *stream)
{
    if (!c) return -1;
    cudaSetDevice(c->device);
    if (r_pos(c) && c->pos >= c->g.n_ctx) {
        ecu_set_error(nullptr, 0, "context exhausted (%d positions)", c->g.n_ctx);
        return -1;
    }
    cudaStream_t s = stream ? (cudaStream_t)stream : c->stream;
    if (c->mega && s != c->stream) {
        // the persistent step straight on the caller's stream (a pipeline
        // stage's steps of every sequence share one): ordered after the
        // context's own stream only when that has work left, and the
        // context's stream ordered after the step for whatever follows there
        if (cudaStreamQuery(c->stream) != cudaSuccess) {
            cudaGetLastError();
            CK(cudaEventRecord(c->ev_step, c->stream));
            CK(cudaStreamWaitEvent(s, c->ev_step, 0));
        }
        StepState *slot = c->h_st + (c->pos % c->n_hslots);
        slot->pos = c->pos;
        CK(cudaMemcpyAsync(&c->st->pos, &slot->pos, sizeof(int), cudaMemcpyHostToDevice, s));
        if (mega_launch(c, s, nullptr) != 0) return -1;
        g_launches += 1;
        CK(cudaEventRecord(c->ev_step, s));
        CK(cudaStreamWaitEvent(c->stream, c->ev_step, 0));
        if (r_pos(c)) c->pos++;
        if (r_head(c)) c->have_logits = true;
        return 0;
    }
    return on_stream(c, stream, [&] {
        // the position comes from the host; the token stays where the
        // previous step (or the caller) left it in device memory
        StepState *slot = c->h_st + (c->pos % c->n_hslots);
        slot->pos = c->pos;
        CK(cudaMemcpyAsync(&c->st->pos, &slot->pos, sizeof(int), cudaMemcpyHostToDevice, c->stream));
        if (run_step(c) != 0) return -1;
        if (r_pos(c)) c->pos++;
        if (r_head(c)) c->have_logits = true;
        return 0;
    });
}

int ecu_ctx_fork(ecu_ctx **out, ecu_ctx *base, char *err, size_t errlen)
{
    if (err && errlen) err[0] = '\0';
    if (!out || !base) { ecu_set_error(err, errlen, "null argument"); return -1; }
    *out = nullptr;
    if (base->tp.world > 1) { ecu_set_error(err, errlen, "a tensor-parallel context is not forked"); return -1; }
    if (cudaSetDevice(base->device) != cudaSuccess) { ecu_set_error(err, errlen, "cudaSetDevice(%d) failed", base->device); return -1; }
    std::unique_ptr<ecu_ctx, void (*)(ecu_ctx *)> c(new ecu_ctx(), ctx_free);
    c->device = base->device;
    c->sms = base->sms;
    c->stage = base->stage;
    c->span = base->span;
    c->first = base->first;
    c->last = base->last;
    c->g = base->g;
    c->tp = base->tp;
    c->pdl = base->pdl;
    c->use_graph = base->use_graph;
    c->shared = base->shared;
    c->layers = base->layers;
    c->emb = base->emb;
    c->out = base->out;
    c->out_norm = base->out_norm;
    c->rope_cs = base->rope_cs;
    c->n_split = base->n_split;
    c->srcs = base->srcs;
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&c->ev_step, cudaEventDisableTiming) != cudaSuccess) {
        ecu_set_error(err, errlen, "cudaStreamCreate failed");
        return -1;
    }
    const bool layers = !c->layers.empty();
    const bool head = r_head(c.get());
    if (const char *what = alloc_buffers(c.get(), layers, head)) {
        ecu_set_error(err, errlen, "out of device memory (%s) after %zu bytes", what, c->bytes);
        return -1;
    }
    if (mega_setup(c.get()) != 0) {
        ecu_set_error(err, errlen, "out of device memory (persistent step buffers)");
        return -1;
    }
    if (cudaDeviceSynchronize() != cudaSuccess || cudaGetLastError() != cudaSuccess) {
        ecu_set_error(err, errlen, "fork failed: %s", cudaGetErrorString(cudaGetLastError()));
        return -1;
    }
    *out = c.release();
    return 0;
}

// Eager (non-graph) run of an explicit layer list; pos unchanged.
static int run_layers_eager(ecu_ctx *c, int from, int to, float *out)
{
    const size_t ne = (size_t)c->g.n_embd;
    memcpy(c->h_state, out, ne * sizeof(float));
    CK(cudaMemcpyAsync(c->state, c->h_state, ne * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    StepState *slot = c->h_st + (c->pos % c->n_hslots);
    slot->pos = c->pos;
    slot->token = 0;
    CK(cudaMemcpyAsync(c->st, slot, 2 * sizeof(int), cudaMemcpyHostToDevice, c->stream));
    Launcher L{c->stream, c->pdl};
    for (int i = from; i < to; i++) enqueue_layer(c, L, i);
    g_launches += (uint64_t)L.count;
    if (L.err != cudaSuccess) { ecu_set_error(nullptr, 0, "kernel launch failed: %s", cudaGetErrorString(L.err)); return -1; }
    CK(cudaMemcpyAsync(c->h_state, c->state, ne * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    if (check_status(c) != 0) return -1;
    memcpy(out, c->h_state, ne * sizeof(float));
    return 0;
}

int ecu_layer_once(ecu_ctx *c, int idx, float *out)
{
    if (!c || c->stage != ECU_STAGE_LAYERS || !out) return -1;
    if (idx < 0 || idx > c->last - c->first) return -1;
    if (c->pos >= c->g.n_ctx) { ecu_set_error(nullptr, 0, "position %d outside the cache", c->pos); return -1; }
    cudaSetDevice(c->device);
    return run_layers_eager(c, idx, idx + 1, out);
}

int ecu_step_layers(ecu_ctx *c, int n, float *out)
{
    if (!c || c->stage != ECU_STAGE_LAYERS || !out) return -1;
    const int all = c->last - c->first + 1;
    if (n <= 0) n = all;
    if (n > all) n = all;
    if (c->pos >= c->g.n_ctx) { ecu_set_error(nullptr, 0, "context exhausted (%d positions)", c->g.n_ctx); return -1; }
    cudaSetDevice(c->device);
    if (n == all) return ecu_forward(c, 0, out);
    if (run_layers_eager(c, 0, n, out) != 0) return -1;
    c->pos++;
    return 0;
}

int ecu_pick(const ecu_ctx *c)
{
    if (!c || !c->have_logits) return 0;
    return c->last_pick;
}

int ecu_get_logits(const ecu_ctx *c, float *out, size_t n)
{
    if (!c || !out || !c->logits || n > (size_t)(c->tp.v1 - c->tp.v0)) return -1;
    cudaSetDevice(c->device);
    CK(cudaStreamSynchronize(c->stream));
    CK(cudaMemcpy(out, c->logits, n * sizeof(float), cudaMemcpyDeviceToHost));
    return 0;
}

int ecu_sync(ecu_ctx *c)
{
    if (!c) return -1;
    cudaSetDevice(c->device);
    if (check_status(c) != 0) return -1;
    // the device-side loop leaves the argmax in state[n_embd]
    if (r_head(c)) {
        float t;
        CK(cudaMemcpy(&t, c->state + c->g.n_embd, sizeof t, cudaMemcpyDeviceToHost));
        c->last_pick = (int)t;
    }
    return 0;
}

int ecu_decode_async(ecu_ctx *c, int n_steps)
{
    if (!c || c->stage != ECU_STAGE_FULL || n_steps < 0) return -1;
    if (c->pos + n_steps > c->g.n_ctx) { ecu_set_error(nullptr, 0, "context exhausted"); return -1; }
    cudaSetDevice(c->device);
    for (int i = 0; i < n_steps; i++) {
        if (run_step(c) != 0) return -1;
        c->pos++;
    }
    c->have_logits = c->have_logits || n_steps > 0;
    return 0;
}

int ecu_generate(ecu_ctx *c, const int *prompt, int n_prompt, int n_gen, int *out_tokens)
{
    if (!c || c->stage != ECU_STAGE_FULL || n_prompt < 1 || n_gen < 0 || !prompt) return -1;
    if (c->pos + n_prompt + n_gen > c->g.n_ctx + 1) {
        ecu_set_error(nullptr, 0, "prompt + generation exceed the context (%d)", c->g.n_ctx);
        return -1;
    }
    for (int i = 0; i < n_prompt; i++)
        if (prompt[i] < 0 || prompt[i] >= c->g.n_vocab) {
            ecu_set_error(nullptr, 0, "prompt token %d outside the vocabulary", prompt[i]);
            return -1;
        }
    cudaSetDevice(c->device);
    // prompt tokens: host-fed, no sync between them
    for (int i = 0; i < n_prompt; i++)
        if (enqueue_forward(c, prompt[i]) != 0) return -1;
    // the last prompt step's argmax is generated token 0; each later step
    // consumes the previous argmax from device state
    const int start = c->pos;      // tok_hist[start - 1] = first generated token
    const int more = n_gen > 0 ? n_gen - 1 : 0;
    if (ecu_decode_async(c, more) != 0) return -1;
    if (check_status(c) != 0) return -1;
    if (n_gen > 0) {
        CK(cudaMemcpy(out_tokens, c->tok_hist + (start - 1), (size_t)n_gen * sizeof(int),
                      cudaMemcpyDeviceToHost));
        c->last_pick = out_tokens[n_gen - 1];
    }
    // state[n_embd] holds the last argmax for ecu_forward-style readers
    return 0;
}

int ecu_profile_cta_ns(ecu_ctx *c, unsigned long long *out, size_t n_words, int *grid, char *kinds, size_t kinds_len)
{
    if (!c || !out) return -1;
    if (grid) *grid = c->mega_grid;
    if (!c->mega) { ecu_set_error(nullptr, 0, "per-CTA phase times need the persistent step"); return -1; }
    const size_t np = (size_t)c->margs.n_ph, need = (np + 1) * (size_t)c->mega_grid;
    if (n_words < need) {
        ecu_set_error(nullptr, 0, "ecu_profile_cta_ns: %zu words needed", need);
        return -1;
    }
    if (c->pos >= c->g.n_ctx) { ecu_set_error(nullptr, 0, "context exhausted"); return -1; }
    cudaSetDevice(c->device);
    unsigned long long *d = nullptr;
    CK(cudaMalloc(&d, need * sizeof(unsigned long long)));
    StepState *slot = c->h_st + (c->pos % c->n_hslots);
    slot->pos = c->pos;
    cudaError_t e = cudaMemcpyAsync(&c->st->pos, &slot->pos, sizeof(int), cudaMemcpyHostToDevice, c->stream);
    c->margs.cta_ns = d;
    const int rc = e == cudaSuccess ? mega_launch(c, c->stream, nullptr) : -1;
    c->margs.cta_ns = nullptr;
    g_launches += 1;
    if (rc == 0) {
        if (r_pos(c)) c->pos++;
        if (r_head(c)) c->have_logits = true;
    }
    const int st = rc == 0 ? check_status(c) : -1;
    if (st == 0) e = cudaMemcpy(out, d, need * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
    cudaFree(d);
    if (st != 0 || e != cudaSuccess) return -1;
    if (kinds && kinds_len) {
        std::string k;
        for (size_t i = 0; i < c->ph_kind.size(); i++) k += (i ? "," : "") + std::string(c->ph_kind[i]);
        snprintf(kinds, kinds_len, "%s", k.c_str());
    }
    return (int)np;
}

int ecu_profile_steps(ecu_ctx *c, int n_steps, ecu_kprof *out, int max_kinds)
{
    if (!c || n_steps < 1 || !out || max_kinds < 1) return -1;
    if (!r_lay(c) && !c->mega) return -1;
    if (c->pos + n_steps > c->g.n_ctx) { ecu_set_error(nullptr, 0, "context exhausted"); return -1; }
    cudaSetDevice(c->device);
    if (c->mega) return mega_profile(c, n_steps, out, max_kinds);
    std::vector<ProfRec> recs;
    for (int i = 0; i < n_steps; i++) {
        Launcher L{c->stream, false};
        L.prof = &recs;
        enqueue_step(c, L, n_stage_layers(c));
        g_launches += (uint64_t)L.count;
        if (L.err != cudaSuccess) { ecu_set_error(nullptr, 0, "launch failed: %s", cudaGetErrorString(L.err)); return -1; }
        c->pos++;
    }
    if (check_status(c) != 0) return -1;
    int nk = 0;
    for (auto &r : recs) {
        float ms = 0;
        cudaEventElapsedTime(&ms, r.e0, r.e1);
        cudaEventDestroy(r.e0);
        cudaEventDestroy(r.e1);
        int k = 0;
        while (k < nk && strncmp(out[k].kind, r.kind, sizeof out[k].kind) != 0) k++;
        if (k == nk) {
            if (nk == max_kinds) continue;
            memset(&out[k], 0, sizeof out[k]);
            snprintf(out[k].kind, sizeof out[k].kind, "%s", r.kind);
            out[k].bytes_per_launch = r.bytes;
            nk++;
        }
        out[k].launches++;
        out[k].total_ms += ms;
    }
    return nk;
}

int ecu_dequant(unsigned type, const void *raw, size_t total, size_t off, size_t n, float *dst,
                int device)
{
    if (!raw || !dst) return -1;
    if (off > total || n > total - off) { ecu_set_error(nullptr, 0, "range outside the tensor"); return -1; }
    if (n == 0) return 0;
    const int t = (int)type;
    if (!dq_supported(t)) { ecu_set_error(nullptr, 0, "type %u not supported", type); return -1; }
    size_t first_byte, nbytes, rel_off;
    if (t == GT_F32 || t == GT_F16) {
        const size_t es = t == GT_F32 ? 4 : 2;
        first_byte = off * es;
        nbytes = n * es;
        rel_off = 0;
    } else {
        const size_t be = (size_t)blk_elems(t), bb = (size_t)blk_bytes(t);
        if (off % be) { ecu_set_error(nullptr, 0, "offset %zu not on a block boundary", off); return -1; }
        const size_t nblk = (n + be - 1) / be;
        if (off / be + nblk > total / be) { ecu_set_error(nullptr, 0, "blocks outside the tensor"); return -1; }
        first_byte = off / be * bb;
        nbytes = nblk * bb;
        rel_off = 0;
    }
    CK(cudaSetDevice(device));
    // bytes the decoder may touch past the last block (Q8_K, see dalloc):
    // the following bytes of the caller's tensor where there are any, zeros
    // after its end
    const size_t valid = ecu_type_nbytes(type, total);
    size_t tail = valid > first_byte + nbytes ? valid - first_byte - nbytes : 0;
    if (tail > 64) tail = 64;
    uint8_t *d_raw = nullptr;
    float   *d_out = nullptr;
    CK(cudaMalloc(&d_raw, nbytes + 256));
    if (cudaMalloc(&d_out, n * sizeof(float)) != cudaSuccess) { cudaFree(d_raw); ecu_set_error(nullptr, 0, "out of memory"); return -1; }
    int rc = 0;
    if (cudaMemset(d_raw, 0, nbytes + 256) != cudaSuccess ||
        cudaMemcpy(d_raw, (const uint8_t *)raw + first_byte, nbytes + tail, cudaMemcpyHostToDevice) != cudaSuccess)
        rc = -1;
    if (!rc) {
        k_dequant_raw<<<256, 256>>>(t, d_raw, rel_off, n, d_out);
        g_launches++;
        if (cudaDeviceSynchronize() != cudaSuccess ||
            cudaMemcpy(dst, d_out, n * sizeof(float), cudaMemcpyDeviceToHost) != cudaSuccess)
            rc = -1;
    }
    cudaFree(d_raw);
    cudaFree(d_out);
    if (rc) ecu_set_error(nullptr, 0, "ecu_dequant: CUDA error %s", cudaGetErrorString(cudaGetLastError()));
    return rc;
}

int ecu_dequant_tensor(ecu_ctx *c, const char *name, size_t off, size_t n, float *dst)
{
    if (!c || !name || !dst) return -1;
    for (auto &s : c->srcs) {
        if (s.name != name) continue;
        if (off > s.elems || n > s.elems - off) return -1;
        if (s.m.zero) { ecu_set_error(nullptr, 0, "tensor %s is not resident (zero rule)", name); return -1; }
        cudaSetDevice(c->device);
        float *d = nullptr;
        CK(cudaMalloc(&d, n * sizeof(float) + 256));
        k_dequant_mat<<<256, 256, 0, c->stream>>>(s.m, s.row0, s.rstride, s.n_in, off, n, d);
        g_launches++;
        int rc = 0;
        if (cudaStreamSynchronize(c->stream) != cudaSuccess ||
            cudaMemcpy(dst, d, n * sizeof(float), cudaMemcpyDeviceToHost) != cudaSuccess)
            rc = -1;
        cudaFree(d);
        return rc;
    }
    ecu_set_error(nullptr, 0, "no resident tensor named %s", name);
    return -1;
}

int ecu_matvec(unsigned type, const void *w_raw, int n_in, int n_out, const float *x, float *y,
               int device)
{
    if (!w_raw || !x || !y || n_in <= 0 || n_out <= 0) return -1;
    CK(cudaSetDevice(device));
    fast_attrs_all();
    CK(cudaGetLastError());
    ecu_ctx tmp;               // borrow the allocator/stream helpers
    tmp.device = device;
    tmp.sms = num_sms(device);
    CK(cudaStreamCreateWithFlags(&tmp.stream, cudaStreamNonBlocking));
    struct Cleanup {
        ecu_ctx *c;
        ~Cleanup()
        {
            for (void *p : c->allocs) cudaFree(p);
            c->allocs.clear();
            cudaStreamDestroy(c->stream);
            c->stream = nullptr;
        }
    } cleanup{&tmp};
    EcuTensor t;
    t.type = type;
    t.n_dims = 2;
    t.dims[0] = (uint64_t)n_in;
    t.dims[1] = (uint64_t)n_out;
    t.data = (const uint8_t *)w_raw;
    t.nbytes = ecu_type_nbytes(type, (size_t)n_in * n_out);
    DevMat m = make_mat(&tmp, (int)type, n_in, n_out, true, true);
    uint8_t *stage = tmp.dalloc<uint8_t>(t.nbytes + 16);
    float   *dx = tmp.dalloc<float>((size_t)n_in + 4);
    float   *dy = tmp.dalloc<float>((size_t)n_out + 4);
    GemvScratch s;
    s.xn = tmp.dalloc<float>((size_t)n_in + 4);
    s.part_val = tmp.dalloc<float>(4096);
    s.part_idx = tmp.dalloc<int>(4096);
    s.counter = tmp.dalloc<unsigned>(4);
    s.status = tmp.dalloc<int>(4);
    if ((!m.zero && !m.data) || !stage || !dx || !dy || !s.xn) { ecu_set_error(nullptr, 0, "out of memory"); return -1; }
    cudaMemset(s.status, 0, 4 * sizeof(int));
    cudaMemset(s.counter, 0, 4 * sizeof(unsigned));
    CK(cudaDeviceSynchronize());     // legacy-stream memsets before the non-blocking stream
    if (!m.zero && t.nbytes && upload_rows(&tmp, &t, n_in, n_out, m, 0, 1, stage) != 0) return -1;
    CK(cudaMemcpy(dx, x, (size_t)n_in * sizeof(float), cudaMemcpyHostToDevice));
    Launcher L{tmp.stream, false};
    GemvArgs a = {};
    enqueue_gemv(L, tmp.sms, m, dx, nullptr, 0.0f, dy, EPI_STORE, s, a);
    g_launches += (uint64_t)L.count;
    if (L.err != cudaSuccess) { ecu_set_error(nullptr, 0, "launch failed: %s", cudaGetErrorString(L.err)); return -1; }
    CK(cudaStreamSynchronize(tmp.stream));
    int st = 0;
    CK(cudaMemcpy(&st, s.status, sizeof st, cudaMemcpyDeviceToHost));
    if (st) { ecu_set_error(nullptr, 0, "bounded wait expired in the GEMV"); return -1; }
    CK(cudaMemcpy(y, dy, (size_t)n_out * sizeof(float), cudaMemcpyDeviceToHost));
    return 0;
}

int ecu_matvec_stream_bench(unsigned type, const void *w_raw, int n_in, int n_out, const float *x, float *y,
                            int device, int copies, int rounds, double *ms_per_matvec)
{
    if (!w_raw || !x || !y || !ms_per_matvec || n_in <= 0 || n_out <= 0 || copies < 1 || rounds < 1) {
        ecu_set_error(nullptr, 0, "ecu_matvec_stream_bench: bad arguments");
        return -1;
    }
    CK(cudaSetDevice(device));
    ecu_ctx tmp;
    tmp.device = device;
    tmp.sms = num_sms(device);
    CK(cudaStreamCreateWithFlags(&tmp.stream, cudaStreamNonBlocking));
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    struct Cleanup {
        ecu_ctx *c;
        cudaEvent_t *e0, *e1;
        ~Cleanup()
        {
            if (*e0) cudaEventDestroy(*e0);
            if (*e1) cudaEventDestroy(*e1);
            for (void *q : c->allocs) cudaFree(q);
            c->allocs.clear();
            cudaStreamDestroy(c->stream);
            c->stream = nullptr;
        }
    } cleanup{&tmp, &e0, &e1};
    MegaFn fn = mega_lookup(128, 4, false);
    EcuTensor t;
    t.type = type;
    t.n_dims = 2;
    t.dims[0] = (uint64_t)n_in;
    t.dims[1] = (uint64_t)n_out;
    t.data = (const uint8_t *)w_raw;
    t.nbytes = ecu_type_nbytes(type, (size_t)n_in * n_out);
    uint8_t *stage = tmp.dalloc<uint8_t>(t.nbytes + 16);
    if (!stage || !fn) { ecu_set_error(nullptr, 0, "out of memory"); return -1; }
    // the phase list: one GEMV (plain input x, tagged output) per copy
    const int grid = tmp.sms;
    const unsigned stage_bytes = (MEGA_RING_BYTES / 2) & ~127u;
    std::vector<MegaPhase> ph;
    std::vector<uint4> tab;
    int red = MEGA_NCW * (128 + 4);
    const size_t w_y = ((size_t)n_out + 7) & ~(size_t)3;
    float *dx = tmp.dalloc<float>((size_t)n_in + 4);
    unsigned long long *yll = tmp.dalloc<unsigned long long>(w_y + 64);
    unsigned *ctr = tmp.dalloc<unsigned>(16);
    StepState *st = tmp.dalloc<StepState>(1);
    if (!dx || !yll || !ctr || !st) { ecu_set_error(nullptr, 0, "out of memory"); return -1; }
    for (int k = 0; k < copies; k++) {
        DevMat m = make_mat(&tmp, (int)type, n_in, n_out, true, false);
        if (!m.data) { ecu_set_error(nullptr, 0, "out of memory for copy %d", k); return -1; }
        if (!mega_mat_ok(m)) {
            ecu_set_error(nullptr, 0, "ecu_matvec_stream_bench: the matrix has no fast layout (Q4_0/Q8_0/Q4_K, "
                                      "n_in a multiple of 1024)");
            return -1;
        }
        if (upload_rows(&tmp, &t, n_in, n_out, m, 0, 1, stage) != 0) return -1;
        if (m.row_bytes > stage_bytes) { ecu_set_error(nullptr, 0, "a row does not fit a ring stage"); return -1; }
        MegaPhase q = mega_gemv_phase(m, grid, stage_bytes, 0, EPI_STORE, dx, nullptr, nullptr, nullptr);
        q.y_ll = yll;
        q.red4 = (q.fmt == 4 && q.rpc * (q.nkg * 4 + 1) <= MEGA_RED4_MAX) ? 1 : 0;
        red = std::max(red, q.red4 ? q.rpc * (q.nkg * 4 + 1) : q.rpc * q.nkg);
        ph.push_back(q);
        tab.push_back(mega_tab_entry(q.w, q.row_bytes, q.sr, q.n_out, q.rpc));
    }
    const size_t un = (size_t)n_in / 32 * 28 * sizeof(int);
    const size_t smem = mega_smem_total(red, 2 * stage_bytes, (unsigned)un, (int)ph.size());
    cudaFuncAttributes fa;
    int optin = 0;
    CK(cudaFuncGetAttributes(&fa, fn));
    CK(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
    if (smem + fa.sharedSizeBytes > (size_t)optin) {
        ecu_set_error(nullptr, 0, "ecu_matvec_stream_bench: shared memory plan too large");
        return -1;
    }
    CK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes));
    MegaPhase *d_ph = tmp.dalloc<MegaPhase>(ph.size());
    uint4 *d_tab = tmp.dalloc<uint4>(tab.size());
    if (!d_ph || !d_tab) { ecu_set_error(nullptr, 0, "out of memory"); return -1; }
    CK(cudaMemcpy(d_ph, ph.data(), ph.size() * sizeof(MegaPhase), cudaMemcpyHostToDevice));
    CK(cudaMemcpy(d_tab, tab.data(), tab.size() * sizeof(uint4), cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dx, x, sizeof(float) * (size_t)n_in, cudaMemcpyHostToDevice));
    CK(cudaMemset(yll, 0, sizeof(unsigned long long) * (w_y + 64)));
    CK(cudaMemset(ctr, 0, 16 * sizeof(unsigned)));
    CK(cudaMemset(st, 0, sizeof(StepState)));
    MegaArgs a = {};
    a.ph = d_ph;
    a.n_ph = (int)ph.size();
    a.tab = d_tab;
    a.bar = ctr;
    a.ticket = ctr + 2;
    a.att_ticket = ctr + 4;
    a.st = st;
    a.status = &st->status;
    a.x_ll = a.qkv_ll = a.att_ll = a.h_ll = yll;
    a.ll_block = yll;
    a.peer[0] = yll;
    a.n_embd = n_in;
    a.n_head = 1;
    a.n_kv = 1;
    a.n_ctx = 1;
    a.n_split = 1;
    a.tp_world = 1;
    a.red_floats = red;
    a.union_bytes = (unsigned)un;
    a.nst = 2;
    a.stage_bytes = stage_bytes;
    a.att_sub = MEGA_ATT_SUB;
    a.att_nsl = 1;
    a.stall_phase = -1;
    a.eps = 1e-5f;
    a.kscale = 1.0f;
    CK(cudaDeviceSynchronize());
    cudaLaunchConfig_t  cfg = {};
    cudaLaunchAttribute at;
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(MEGA_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = tmp.stream;
    at.id = cudaLaunchAttributeCooperative;
    at.val.cooperative = 1;
    cfg.attrs = &at;
    cfg.numAttrs = 1;
    for (int r = 0; r < 2; r++) CK(mega_launch_serial(device, cfg, fn, a));     // warm-up
    CK(cudaStreamSynchronize(tmp.stream));
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    CK(cudaEventRecord(e0, tmp.stream));
    for (int r = 0; r < rounds; r++) CK(mega_launch_serial(device, cfg, fn, a));
    CK(cudaEventRecord(e1, tmp.stream));
    CK(cudaStreamSynchronize(tmp.stream));
    g_launches += (uint64_t)(rounds + 2);
    float ms = 0.0f;
    CK(cudaEventElapsedTime(&ms, e0, e1));
    *ms_per_matvec = (double)ms / ((double)rounds * copies);
    StepState hs;
    CK(cudaMemcpy(&hs, st, sizeof hs, cudaMemcpyDeviceToHost));
    if (hs.status) { ecu_set_error(nullptr, 0, "a bounded wait expired in the streamed GEMV"); return -1; }
    std::vector<unsigned long long> w((size_t)n_out);
    CK(cudaMemcpy(w.data(), yll, sizeof(unsigned long long) * (size_t)n_out, cudaMemcpyDeviceToHost));
    for (int i = 0; i < n_out; i++) {
        const unsigned u = (unsigned)(w[(size_t)i] & 0xFFFFFFFFull);
        memcpy(&y[i], &u, sizeof u);
    }
    return 0;
}

int ecu_set_wait_ns(int device, unsigned long long ns)
{
    if (ns == 0) {
        ecu_set_error(nullptr, 0, "ecu_set_wait_ns: the limit must be positive");
        return -1;
    }
    CK(cudaSetDevice(device));
    CK(cudaMemcpyToSymbol(g_wait_ns, &ns, sizeof ns));
    return 0;
}

int ecu_inject_wait_timeout(ecu_ctx *c)
{
    if (!c || !c->mega) {
        ecu_set_error(nullptr, 0, "ecu_inject_wait_timeout: only a context on the persistent step");
        return -1;
    }
    // the first GEMV phase whose input is a tagged vector (written by an
    // earlier phase of the same launch)
    for (int p = 0; p < (int)c->ph_in_ep.size(); p++)
        if (c->ph_in_ep[p] >= 0) {
            c->stall_next = p;
            return 0;
        }
    ecu_set_error(nullptr, 0, "ecu_inject_wait_timeout: no phase reads a tagged input");
    return -1;
}

int ecu_matvec_bench(unsigned type, const void *w_raw, int n_in, int n_out, const float *x, float *y, int device,
                     int copies, int rounds, double *ms_per_launch)
{
    if (!w_raw || !x || !y || !ms_per_launch || n_in <= 0 || n_out <= 0 || copies < 1 || rounds < 1) {
        ecu_set_error(nullptr, 0, "ecu_matvec_bench: bad arguments");
        return -1;
    }
    CK(cudaSetDevice(device));
    fast_attrs_all();
    CK(cudaGetLastError());
    ecu_ctx tmp;
    tmp.device = device;
    tmp.sms = num_sms(device);
    CK(cudaStreamCreateWithFlags(&tmp.stream, cudaStreamNonBlocking));
    cudaGraph_t     gr = nullptr;
    cudaGraphExec_t gx = nullptr;
    cudaEvent_t     e0 = nullptr, e1 = nullptr;
    struct Cleanup {
        ecu_ctx *c;
        cudaGraphExec_t *gx;
        cudaEvent_t *e0, *e1;
        ~Cleanup()
        {
            if (*gx) cudaGraphExecDestroy(*gx);
            if (*e0) cudaEventDestroy(*e0);
            if (*e1) cudaEventDestroy(*e1);
            for (void *p : c->allocs) cudaFree(p);
            c->allocs.clear();
            cudaStreamDestroy(c->stream);
            c->stream = nullptr;
        }
    } cleanup{&tmp, &gx, &e0, &e1};
    EcuTensor t;
    t.type = type;
    t.n_dims = 2;
    t.dims[0] = (uint64_t)n_in;
    t.dims[1] = (uint64_t)n_out;
    t.data = (const uint8_t *)w_raw;
    t.nbytes = ecu_type_nbytes(type, (size_t)n_in * n_out);
    // `copies` independent device copies in the layout the engine keeps
    // (fast SPLIT layouts where they apply), so that a rotation over them
    // streams from HBM rather than from L2
    std::vector<DevMat> mats;
    uint8_t *stage = tmp.dalloc<uint8_t>(t.nbytes + 16);
    if (!stage) { ecu_set_error(nullptr, 0, "out of memory"); return -1; }
    for (int k = 0; k < copies; k++) {
        DevMat m = make_mat(&tmp, (int)type, n_in, n_out, true, true);
        if (!m.zero && !m.data) { ecu_set_error(nullptr, 0, "out of memory for copy %d", k); return -1; }
        if (!m.zero && t.nbytes && upload_rows(&tmp, &t, n_in, n_out, m, 0, 1, stage) != 0) return -1;
        mats.push_back(m);
    }
    float *dx = tmp.dalloc<float>((size_t)n_in + 4);
    float *dy = tmp.dalloc<float>((size_t)n_out + 4);
    GemvScratch s;
    s.xn = tmp.dalloc<float>((size_t)n_in + 4);
    s.part_val = tmp.dalloc<float>(4096);
    s.part_idx = tmp.dalloc<int>(4096);
    s.counter = tmp.dalloc<unsigned>(4);
    s.status = tmp.dalloc<int>(4);
    if (!dx || !dy || !s.xn || !s.part_val || !s.part_idx || !s.counter || !s.status) {
        ecu_set_error(nullptr, 0, "out of memory");
        return -1;
    }
    CK(cudaMemset(s.status, 0, 4 * sizeof(int)));
    CK(cudaMemset(s.counter, 0, 4 * sizeof(unsigned)));
    CK(cudaMemcpy(dx, x, (size_t)n_in * sizeof(float), cudaMemcpyHostToDevice));
    CK(cudaDeviceSynchronize());
    // one graph: a launch per copy, back to back with programmatic dependent
    // launch, each warming the next copy's first rows in L2 (what the decode
    // step does between consecutive matrices)
    CK(cudaStreamBeginCapture(tmp.stream, cudaStreamCaptureModeThreadLocal));
    Launcher L{tmp.stream, true};
    for (int k = 0; k < copies; k++) {
        GemvArgs a = {};
        enqueue_gemv(L, tmp.sms, mats[k], dx, nullptr, 0.0f, dy, EPI_STORE, s, a, &mats[(k + 1) % copies]);
    }
    cudaError_t e = cudaStreamEndCapture(tmp.stream, &gr);
    if (e != cudaSuccess || L.err != cudaSuccess) {
        ecu_set_error(nullptr, 0, "ecu_matvec_bench: capture failed: %s",
                      cudaGetErrorString(e != cudaSuccess ? e : L.err));
        if (gr) cudaGraphDestroy(gr);
        return -1;
    }
    e = cudaGraphInstantiate(&gx, gr, 0);
    cudaGraphDestroy(gr);
    if (e != cudaSuccess) {
        ecu_set_error(nullptr, 0, "ecu_matvec_bench: graph instantiate failed: %s", cudaGetErrorString(e));
        return -1;
    }
    const int per_round = L.count;
    // warm-up: two rounds (first-touch of every copy, instruction cache)
    for (int r = 0; r < 2; r++) CK(cudaGraphLaunch(gx, tmp.stream));
    CK(cudaStreamSynchronize(tmp.stream));
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    CK(cudaEventRecord(e0, tmp.stream));
    for (int r = 0; r < rounds; r++) CK(cudaGraphLaunch(gx, tmp.stream));
    CK(cudaEventRecord(e1, tmp.stream));
    CK(cudaStreamSynchronize(tmp.stream));
    g_launches += (uint64_t)per_round * (uint64_t)(rounds + 2);
    float ms = 0.0f;
    CK(cudaEventElapsedTime(&ms, e0, e1));
    *ms_per_launch = (double)ms / ((double)rounds * copies);
    int st = 0;
    CK(cudaMemcpy(&st, s.status, sizeof st, cudaMemcpyDeviceToHost));
    if (st) { ecu_set_error(nullptr, 0, "bounded wait expired in the GEMV"); return -1; }
    CK(cudaMemcpy(y, dy, (size_t)n_out * sizeof(float), cudaMemcpyDeviceToHost));
    return 0;
}

}  // extern "C"

// ------------------------------------------------------ tensor parallel --

int ecu_tp_slice(const ecu_ctx *c, int *out4)
{
    if (!c || !out4) return -1;
    out4[0] = c->tp.rank;
    out4[1] = c->tp.world;
    out4[2] = c->tp.v0;
    out4[3] = c->tp.v1;
    return 0;
}

int ecu_tp_handle(ecu_ctx *c, unsigned char *out)
{
    if (!c || !out || !c->mega || !c->mega_ll) {
        ecu_set_error(nullptr, 0, "no persistent step to share");
        return -1;
    }
    cudaSetDevice(c->device);
    cudaIpcMemHandle_t h;
    CK(cudaIpcGetMemHandle(&h, c->mega_ll));
    static_assert(sizeof h == ECU_TP_HANDLE_BYTES, "IPC handle size");
    memcpy(out, &h, sizeof h);
    return 0;
}

int ecu_tp_connect(ecu_ctx *c, const unsigned char *handles)
{
    if (!c || !handles || !c->mega || c->tp.world < 2) {
        ecu_set_error(nullptr, 0, "not a tensor-parallel context");
        return -1;
    }
    if (!c->tp_peers.empty()) {
        ecu_set_error(nullptr, 0, "tensor-parallel ranks already connected");
        return -1;
    }
    cudaSetDevice(c->device);
    for (int k = 0; k < c->tp.world; k++) {
        if (k == c->tp.rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, handles + (size_t)k * ECU_TP_HANDLE_BYTES, sizeof h);
        void *p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            ecu_set_error(nullptr, 0, "opening rank %d's tagged vectors failed: %s", k, cudaGetErrorString(e));
            return -1;
        }
        c->tp_peers.push_back(p);
        c->margs.peer[k] = reinterpret_cast<unsigned long long *>(p);
    }
    char buf[64];
    snprintf(buf, sizeof buf, "persistent, tensor parallel %d/%d", c->tp.rank, c->tp.world);
    c->path = buf;
    return 0;
}

// ------------------------------------------------------ pipeline links -----

// The token word of a linked first stage, from the host (the prompt's last
// token before the first linked step), tagged for the position `epoch`
// encodes.
__global__ void k_link_feed(unsigned long long *w, int token, unsigned epoch)
{
    const unsigned long long v = ((unsigned long long)epoch << 32) | (unsigned)token;
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(w), "l"(v) : "memory");
}

static unsigned host_link_epoch(int pos) { return (((unsigned)pos & 0xFFFFFu) << 12) | 0xFFFu; }

static int link_check(ecu_ctx *c, const char *what)
{
    if (!c) return -1;
    if (!c->mega || !c->mega_ll) {
        ecu_set_error(nullptr, 0, "%s: pipeline links need the persistent step (%s)", what, c->path.c_str());
        return -1;
    }
    if (c->tp.world > 1) {
        ecu_set_error(nullptr, 0, "%s: a tensor-parallel context is not linked", what);
        return -1;
    }
    return 0;
}

int ecu_link_handle(ecu_ctx *c, unsigned char *out)
{
    if (link_check(c, "ecu_link_handle") != 0 || !out) return -1;
    cudaSetDevice(c->device);
    cudaIpcMemHandle_t h;
    CK(cudaIpcGetMemHandle(&h, c->mega_ll));
    static_assert(sizeof h == ECU_LINK_HANDLE_BYTES, "IPC handle size");
    memcpy(out, &h, sizeof h);
    return 0;
}

// The next stage's tagged block at `peer`: a stage with the head sends its
// argmax to the token word (right after the residual stream), any other
// stage its output state to the residual stream's words.
static void link_to(ecu_ctx *c, unsigned long long *peer)
{
    if (r_head(c)) {
        c->margs.link_tok = peer + (((size_t)c->g.n_embd + 7) & ~(size_t)3);
        c->margs.link_x = nullptr;
    } else {
        c->margs.link_x = peer;
        c->margs.link_tok = nullptr;
    }
}

int ecu_link_next(ecu_ctx *c, const unsigned char *handle)
{
    if (link_check(c, "ecu_link_next") != 0 || !handle) return -1;
    if (c->link_peer) { ecu_set_error(nullptr, 0, "ecu_link_next: already linked"); return -1; }
    cudaSetDevice(c->device);
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof h);
    void *p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        ecu_set_error(nullptr, 0, "opening the next stage's tagged vectors failed: %s", cudaGetErrorString(e));
        return -1;
    }
    c->link_peer = p;
    link_to(c, reinterpret_cast<unsigned long long *>(p));
    return 0;
}

int ecu_link_next_local(ecu_ctx *c, ecu_ctx *next)
{
    if (link_check(c, "ecu_link_next_local") != 0 || link_check(next, "ecu_link_next_local") != 0) return -1;
    if (next->g.n_embd != c->g.n_embd) { ecu_set_error(nullptr, 0, "ecu_link_next_local: different models"); return -1; }
    link_to(c, next->mega_ll);
    return 0;
}

int ecu_link_input(ecu_ctx *c)
{
    if (link_check(c, "ecu_link_input") != 0) return -1;
    if (c->linked_in) return 0;
    cudaSetDevice(c->device);
    if (r_emb(c)) {
        c->margs.link_in = 1;             // the embedding waits for the token word
    } else {
        // the phases that read the stage's input state read the link's words
        for (MegaPhase &q : c->mega_ph) {
            if (q.kind == PH_GEMV && q.in_ep == MEGA_EP_PLAIN) q.in_ep = MEGA_EP_LINK;
            if (q.kind == PH_GEMV && q.epi == EPI_ADD && q.y_ep == MEGA_EP_PLAIN) q.y_ep = MEGA_EP_LINK;
        }
        CK(cudaMemcpy(const_cast<MegaPhase *>(c->margs.ph), c->mega_ph.data(), c->mega_ph.size() * sizeof(MegaPhase),
                      cudaMemcpyHostToDevice));
    }
    c->linked_in = true;
    return 0;
}

int ecu_link_feed(ecu_ctx *c, int token, void *stream)
{
    if (link_check(c, "ecu_link_feed") != 0) return -1;
    if (!c->linked_in || !r_emb(c)) {
        ecu_set_error(nullptr, 0, "ecu_link_feed: not a linked first stage");
        return -1;
    }
    if (token < 0 || token >= c->g.n_vocab) {
        ecu_set_error(nullptr, 0, "token %d outside the vocabulary (%d)", token, c->g.n_vocab);
        return -1;
    }
    cudaSetDevice(c->device);
    cudaStream_t s = stream ? (cudaStream_t)stream : c->stream;
    k_link_feed<<<1, 1, 0, s>>>(c->margs.tok_ll, token, host_link_epoch(c->pos));
    CK(cudaGetLastError());
    g_launches += 1;
    return 0;
}

// ----------------------------------------------------------- prefill -----

static int pf_reserve(ecu_ctx *c, int n)
{
    ecu_ctx::Prefill &P = c->pf;
    const EcuGeom &g = c->g;
    const size_t hd = (size_t)g.head_dim, qd = (size_t)g.n_head * hd, kvd = (size_t)g.n_head_kv * hd;
    size_t wmax = 0;
    for (auto &ly : c->layers) {
        if (ly.ha)
            for (const DevMat *m : {&ly.qkv[0], &ly.o}) wmax = std::max(wmax, (size_t)m->n_out * m->n_in);
        if (ly.hf)
            for (const DevMat *m : {&ly.gu, &ly.d}) wmax = std::max(wmax, (size_t)m->n_out * m->n_in);
    }
    if (n > P.rows) {
        for (void *p : {(void *)P.X, (void *)P.QKV, (void *)P.ATT, (void *)P.GU, (void *)P.H, (void *)P.ah,
                        (void *)P.al, (void *)P.tok})
            if (p) cudaFree(p);
        P = ecu_ctx::Prefill{0, P.wcap, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, P.wh, P.wl,
                             nullptr};
        const size_t wide = std::max(std::max((size_t)g.n_embd, qd), (size_t)g.n_ff);
        bool ok = cudaMalloc(&P.X, sizeof(float) * n * (size_t)g.n_embd) == cudaSuccess &&
                  cudaMalloc(&P.QKV, sizeof(float) * n * (qd + 2 * kvd)) == cudaSuccess &&
                  cudaMalloc(&P.ATT, sizeof(float) * n * qd) == cudaSuccess &&
                  cudaMalloc(&P.GU, sizeof(float) * n * 2 * (size_t)g.n_ff) == cudaSuccess &&
                  cudaMalloc(&P.H, sizeof(float) * n * (size_t)g.n_ff) == cudaSuccess &&
                  cudaMalloc(&P.ah, sizeof(__half) * n * wide) == cudaSuccess &&
                  cudaMalloc(&P.al, sizeof(__half) * n * wide) == cudaSuccess &&
                  cudaMalloc(&P.tok, sizeof(int) * n) == cudaSuccess;
        if (!ok) {
            cudaGetLastError();
            ecu_set_error(nullptr, 0, "out of device memory for a %d-token prefill", n);
            return -1;
        }
        P.rows = n;
    }
    if (wmax > P.wcap) {
        if (P.wh) cudaFree(P.wh);
        if (P.wl) cudaFree(P.wl);
        P.wh = P.wl = nullptr;
        P.wcap = 0;
        if (cudaMalloc(&P.wh, sizeof(__half) * wmax) != cudaSuccess ||
            cudaMalloc(&P.wl, sizeof(__half) * wmax) != cudaSuccess) {
            cudaGetLastError();
            ecu_set_error(nullptr, 0, "out of device memory for the prefill weight operands");
            return -1;
        }
        P.wcap = wmax;
    }
    return 0;
}

// GEMM of the prefill: C[n x m.n_out] (+R) = A[n x m.n_in] * W^T, W split
// first; tcgen05 (ECU_PF_TC=0: the mma.sync kernel).
static int pf_gemm(ecu_ctx *c, const DevMat &m, int n, float *C, const float *R)
{
    ecu_ctx::Prefill &P = c->pf;
    if ((m.layout == LAY_SPLIT4 || m.layout == LAY_SPLIT8 || m.layout == LAY_SPLITK4) && m.n_in % 32 == 0)
        k_pf_wsplit_fast<<<8 * c->sms, 128, 0, c->stream>>>(m, P.wh, P.wl);
    else
        k_pf_wsplit<<<8 * c->sms, 256, 0, c->stream>>>(m, P.wh, P.wl);
    dim3 grid((unsigned)((m.n_out + PF_BN - 1) / PF_BN), (unsigned)((n + PF_BM - 1) / PF_BM));
    const char *e = getenv("ECU_PF_TC");
    if (!(e && e[0] == '0'))
        k_pf_gemm_tc<<<grid, 128, pf_tc_smem(), c->stream>>>(P.ah, P.al, P.wh, P.wl, C, n, m.n_out, m.n_in, m.n_out,
                                                              R, &c->st->status);
    else
        k_pf_gemm<<<grid, 256, pf_gemm_smem(), c->stream>>>(P.ah, P.al, P.wh, P.wl, C, n, m.n_out, m.n_in, m.n_out, R);
    CK(cudaGetLastError());
    return 0;
}

// Can the batched kernels run this context's prompt (else: token by token)?
static bool pf_batched(const ecu_ctx *c, bool &attn2)
{
    const EcuGeom &g = c->g;
    // the token-tiled attention (k_pf_attn2) has no position limit; the
    // one-query-per-CTA kernel keeps its scores in a PF_ATT_MAXPOS array
    const char *ae = getenv("ECU_PF_ATTN");
    attn2 = PF_QB % g.n_rep == 0 && !(ae && ae[0] == '0');
    bool batched = c->tp.world == 1 && (attn2 || g.n_ctx <= PF_ATT_MAXPOS) && (g.head_dim == 64 || g.head_dim == 128) &&
                   g.n_embd % 8 == 0 && g.n_ff % 8 == 0;
    for (auto &ly : c->layers) batched = batched && (!ly.ha || ly.qkv.size() == 1) && (!ly.hf || ly.gu_fused);
    return batched;
}

static int pf_attrs(const ecu_ctx *c)
{
    static std::atomic<unsigned> attr_done{0};            // per device (bit d), set once
    if (c->device >= 32 || !(attr_done.load() & (1u << c->device))) {
        CK(cudaFuncSetAttribute(k_pf_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pf_gemm_smem()));
        CK(cudaFuncSetAttribute(k_pf_gemm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pf_tc_smem()));
        CK(cudaFuncSetAttribute(k_pf_attn2<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pf_attn2_smem<128>()));
        CK(cudaFuncSetAttribute(k_pf_attn2<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pf_attn2_smem<64>()));
        if (c->device < 32) attr_done.fetch_or(1u << c->device);
    }
    return 0;
}

// The context's layers over the n rows of P.X (positions pos0..pos0+n-1):
// the KV cache filled, P.X holding the last layer's output rows.
static int pf_layers(ecu_ctx *c, int n, int pos0, bool attn2)
{
    ecu_ctx::Prefill &P = c->pf;
    const EcuGeom &g = c->g;
    const int hd = g.head_dim, qd = g.n_head * hd, kvd = g.n_head_kv * hd, E = g.n_embd;
    const int ldq = qd + 2 * kvd;
    const size_t plane = (size_t)g.n_head_kv * g.n_ctx * hd;
    const float kscale = 1.0f / sqrtf((float)hd);
    for (size_t li = 0; li < c->layers.size(); li++) {
        LayerDev &ly = c->layers[li];
        if (ly.ha) {
            k_pf_norm_split<<<n, 256, 0, c->stream>>>(P.X, ly.attn_norm, E, g.eps, P.ah, P.al);
            if (pf_gemm(c, ly.qkv[0], n, P.QKV, nullptr)) return -1;
            k_pf_rope_kv<<<n, 128, 0, c->stream>>>(P.QKV, ldq, g.n_head, g.n_head_kv, hd, pos0, c->rope_cs, ly.bq, ly.bk,
                                                   ly.bv, c->kc + li * plane, c->vc + li * plane, g.n_ctx);
            if (attn2) {
                // tiled over tokens: 64 query vectors a CTA
                dim3 ag((unsigned)g.n_head_kv, (unsigned)((n + PF_QB / g.n_rep - 1) / (PF_QB / g.n_rep)));
                if (hd == 128)
                    k_pf_attn2<128><<<ag, 256, pf_attn2_smem<128>(), c->stream>>>(P.QKV, ldq, n, g.n_head, g.n_rep, pos0,
                                                                                  c->kc + li * plane, c->vc + li * plane,
                                                                                  g.n_ctx, kscale, P.ATT);
                else
                    k_pf_attn2<64><<<ag, 256, pf_attn2_smem<64>(), c->stream>>>(P.QKV, ldq, n, g.n_head, g.n_rep, pos0,
                                                                                c->kc + li * plane, c->vc + li * plane,
                                                                                g.n_ctx, kscale, P.ATT);
            } else {
                dim3 ag((unsigned)g.n_head, (unsigned)n);
                if (hd == 128)
                    k_pf_attn<128><<<ag, 128, 0, c->stream>>>(P.QKV, ldq, g.n_head, g.n_rep, pos0, c->kc + li * plane,
                                                              c->vc + li * plane, g.n_ctx, kscale, P.ATT);
                else
                    k_pf_attn<64><<<ag, 64, 0, c->stream>>>(P.QKV, ldq, g.n_head, g.n_rep, pos0, c->kc + li * plane,
                                                            c->vc + li * plane, g.n_ctx, kscale, P.ATT);
            }
            k_pf_split<<<4 * c->sms, 256, 0, c->stream>>>(P.ATT, (size_t)n * qd, P.ah, P.al);
            if (pf_gemm(c, ly.o, n, P.X, P.X)) return -1;
        }
        if (ly.hf) {
            k_pf_norm_split<<<n, 256, 0, c->stream>>>(P.X, ly.ffn_norm, E, g.eps, P.ah, P.al);
            if (pf_gemm(c, ly.gu, n, P.GU, nullptr)) return -1;
            k_pf_swiglu<<<4 * c->sms, 256, 0, c->stream>>>(P.GU, (size_t)n, g.n_ff, P.H);
            k_pf_split<<<4 * c->sms, 256, 0, c->stream>>>(P.H, (size_t)n * g.n_ff, P.ah, P.al);
            if (pf_gemm(c, ly.d, n, P.X, P.X)) return -1;
        }
        CK(cudaGetLastError());
    }
    g_launches += 15 * c->layers.size();
    return 0;
}

// Row `row` of the device rows x as the head's input: the decode step's head
// (norm, logits, argmax) at position pos, the result (normed state + token)
// copied to out.
static int pf_head(ecu_ctx *c, const float *x_row, int pos, int token, float *out)
{
    const EcuGeom &g = c->g;
    const size_t   ne = (size_t)g.n_embd;
    CK(cudaMemcpyAsync(c->state, x_row, sizeof(float) * ne, cudaMemcpyDeviceToDevice, c->stream));
    StepState *slot = c->h_st + (pos % c->n_hslots);
    slot->pos = pos;
    slot->token = token;
    CK(cudaMemcpyAsync(c->st, slot, 2 * sizeof(int), cudaMemcpyHostToDevice, c->stream));
    Launcher L{c->stream, false};
    enqueue_head(c, L, true);
    g_launches += (uint64_t)L.count;
    if (L.err != cudaSuccess) {
        ecu_set_error(nullptr, 0, "kernel launch failed: %s", cudaGetErrorString(L.err));
        return -1;
    }
    c->pos = pos + 1;
    c->have_logits = true;
    CK(cudaMemcpyAsync(c->h_state, c->state, (ne + 1) * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    if (check_status(c) != 0) return -1;
    memcpy(out, c->h_state, (ne + 1) * sizeof(float));
    c->last_pick = (int)c->h_state[ne];
    return 0;
}

// A span's prompt rows: the embedding rows of the tokens (ECU_SPAN_EMBED),
// the layers in place (batched), then the head on the last row
// (ECU_SPAN_HEAD); the position advances by n.
static int span_prefill_rows(ecu_ctx *c, const int *tokens, int n, float *x, float *out)
{
    const EcuGeom &g = c->g;
    const size_t   rows_bytes = sizeof(float) * (size_t)n * g.n_embd;
    const int      pos0 = c->pos;
    if (pos0 + n > g.n_ctx) {
        ecu_set_error(nullptr, 0, "prompt of %d tokens at position %d exceeds the context (%d)", n, pos0, g.n_ctx);
        return -1;
    }
    if (r_head(c) && !out) { ecu_set_error(nullptr, 0, "a span with the head needs the output buffer"); return -1; }
    if (r_emb(c)) {
        if (!tokens) { ecu_set_error(nullptr, 0, "a span with the embedding needs the prompt tokens"); return -1; }
        for (int i = 0; i < n; i++)
            if (tokens[i] < 0 || tokens[i] >= g.n_vocab) {
                ecu_set_error(nullptr, 0, "token %d outside the vocabulary (%d)", tokens[i], g.n_vocab);
                return -1;
            }
        int *tok = nullptr;
        CK(cudaMallocAsync((void **)&tok, sizeof(int) * n, c->stream));
        CK(cudaMemcpyAsync(tok, tokens, sizeof(int) * n, cudaMemcpyHostToDevice, c->stream));
        k_pf_embed<<<4 * c->sms, 256, 0, c->stream>>>(c->emb, tok, n, x, g.n_embd);
        CK(cudaGetLastError());
        CK(cudaFreeAsync(tok, c->stream));
        g_launches += 1;
    }
    if (!c->layers.empty()) {
        bool attn2 = false;
        if (!pf_batched(c, attn2)) {
            ecu_set_error(nullptr, 0, "the batched prompt kernels do not cover this span's shapes");
            return -1;
        }
        if (pf_attrs(c) != 0 || pf_reserve(c, n) != 0) return -1;
        CK(cudaMemcpyAsync(c->pf.X, x, rows_bytes, cudaMemcpyDeviceToDevice, c->stream));
        if (pf_layers(c, n, pos0, attn2) != 0) return -1;
        CK(cudaMemcpyAsync(x, c->pf.X, rows_bytes, cudaMemcpyDeviceToDevice, c->stream));
    }
    if (r_head(c)) return pf_head(c, x + (size_t)(n - 1) * g.n_embd, pos0 + n - 1, tokens ? tokens[n - 1] : 0, out);
    c->pos = pos0 + n;
    CK(cudaMemcpyAsync(c->state, x + (size_t)(n - 1) * g.n_embd, sizeof(float) * g.n_embd, cudaMemcpyDeviceToDevice,
                       c->stream));
    StepState *slot = c->h_st + (c->pos % c->n_hslots);
    slot->pos = c->pos;
    slot->token = 0;
    CK(cudaMemcpyAsync(c->st, slot, 2 * sizeof(int), cudaMemcpyHostToDevice, c->stream));
    return check_status(c);
}

int ecu_prefill_rows(ecu_ctx *c, const int *tokens, int n, float *x, float *out)
{
    if (!c || n < 1 || !x) { ecu_set_error(nullptr, 0, "null argument or empty prompt"); return -1; }
    cudaSetDevice(c->device);
    const EcuGeom &g = c->g;
    const size_t   rows_bytes = sizeof(float) * (size_t)n * g.n_embd;
    if (c->stage == ECU_STAGE_FULL) { ecu_set_error(nullptr, 0, "a FULL context prefills with ecu_prefill"); return -1; }
    if (c->stage == ECU_STAGE_SPAN) return span_prefill_rows(c, tokens, n, x, out);
    if (c->stage == ECU_STAGE_EMBED) {
        if (!tokens) { ecu_set_error(nullptr, 0, "EMBED needs the prompt tokens"); return -1; }
        for (int i = 0; i < n; i++)
            if (tokens[i] < 0 || tokens[i] >= g.n_vocab) {
                ecu_set_error(nullptr, 0, "token %d outside the vocabulary (%d)", tokens[i], g.n_vocab);
                return -1;
            }
        int *tok = nullptr;
        CK(cudaMallocAsync((void **)&tok, sizeof(int) * n, c->stream));
        CK(cudaMemcpyAsync(tok, tokens, sizeof(int) * n, cudaMemcpyHostToDevice, c->stream));
        k_pf_embed<<<4 * c->sms, 256, 0, c->stream>>>(c->emb, tok, n, x, g.n_embd);
        CK(cudaGetLastError());
        CK(cudaFreeAsync(tok, c->stream));
        g_launches += 1;
        c->pos += n;
        CK(cudaStreamSynchronize(c->stream));
        return 0;
    }
    if (c->stage == ECU_STAGE_HEAD) {
        if (!out) { ecu_set_error(nullptr, 0, "HEAD needs the output buffer"); return -1; }
        const int pos = c->pos + n - 1;
        return pf_head(c, x + (size_t)(n - 1) * g.n_embd, pos, tokens ? tokens[n - 1] : 0, out);
    }
    // LAYERS
    if (c->pos + n > g.n_ctx) {
        ecu_set_error(nullptr, 0, "prompt of %d tokens at position %d exceeds the context (%d)", n, c->pos, g.n_ctx);
        return -1;
    }
    bool attn2 = false;
    if (!pf_batched(c, attn2)) {
        // the per-token step, row by row
        std::vector<float> h((size_t)g.n_embd + 8);
        for (int i = 0; i < n; i++) {
            CK(cudaMemcpy(h.data(), x + (size_t)i * g.n_embd, sizeof(float) * g.n_embd, cudaMemcpyDeviceToHost));
            if (ecu_forward(c, 0, h.data()) != 0) return -1;
            CK(cudaMemcpy(x + (size_t)i * g.n_embd, h.data(), sizeof(float) * g.n_embd, cudaMemcpyHostToDevice));
        }
        return 0;
    }
    if (pf_attrs(c) != 0 || pf_reserve(c, n) != 0) return -1;
    const int pos0 = c->pos;
    CK(cudaMemcpyAsync(c->pf.X, x, rows_bytes, cudaMemcpyDeviceToDevice, c->stream));
    if (pf_layers(c, n, pos0, attn2) != 0) return -1;
    CK(cudaMemcpyAsync(x, c->pf.X, rows_bytes, cudaMemcpyDeviceToDevice, c->stream));
    c->pos = pos0 + n;
    // the stage's state: the last row (what a LAYERS forward outputs)
    CK(cudaMemcpyAsync(c->state, c->pf.X + (size_t)(n - 1) * g.n_embd, sizeof(float) * g.n_embd,
                       cudaMemcpyDeviceToDevice, c->stream));
    StepState *slot = c->h_st + (c->pos % c->n_hslots);
    slot->pos = c->pos;
    slot->token = 0;
    CK(cudaMemcpyAsync(c->st, slot, 2 * sizeof(int), cudaMemcpyHostToDevice, c->stream));
    return check_status(c);
}

int ecu_prefill(ecu_ctx *c, const int *tokens, int n, float *out)
{
    if (!c || !tokens || !out || n < 1) { ecu_set_error(nullptr, 0, "null argument or empty prompt"); return -1; }
    cudaSetDevice(c->device);
    const EcuGeom &g = c->g;
    for (int i = 0; i < n; i++)
        if (tokens[i] < 0 || tokens[i] >= g.n_vocab) {
            ecu_set_error(nullptr, 0, "token %d outside the vocabulary (%d)", tokens[i], g.n_vocab);
            return -1;
        }
    if (c->stage != ECU_STAGE_FULL) { ecu_set_error(nullptr, 0, "prefill runs FULL contexts"); return -1; }
    if (c->pos + n > g.n_ctx) {
        ecu_set_error(nullptr, 0, "prompt of %d tokens at position %d exceeds the context (%d)", n, c->pos, g.n_ctx);
        return -1;
    }
    bool attn2 = false;
    if (!pf_batched(c, attn2)) {
        // shapes the batched kernels do not cover (and tensor-parallel ranks,
        // which step together): the per-token step, prompt token by token
        for (int i = 0; i < n; i++)
            if (ecu_forward(c, tokens[i], out) != 0) return -1;
        return 0;
    }
    if (pf_attrs(c) != 0 || pf_reserve(c, n) != 0) return -1;
    ecu_ctx::Prefill &P = c->pf;
    const int E = g.n_embd, pos0 = c->pos;
    CK(cudaMemcpyAsync(P.tok, tokens, sizeof(int) * n, cudaMemcpyHostToDevice, c->stream));
    k_pf_embed<<<4 * c->sms, 256, 0, c->stream>>>(c->emb, P.tok, n, P.X, E);
    g_launches += 1;
    if (pf_layers(c, n, pos0, attn2) != 0) return -1;
    return pf_head(c, P.X + (size_t)(n - 1) * E, pos0 + n - 1, tokens[n - 1], out);
}
