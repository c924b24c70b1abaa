// ecu_noalloc.cu -- logits + argmax over caller-owned device memory with no
// device allocation anywhere on the call path.
//
// Why it exists: some hosts of this engine cannot call cudaMalloc.  A dcd
// shard node sizes all of its memory up front from --pool-bytes and must
// not grow behind that budget; a host that hands out device memory from its
// own allocator or a fixed pool has no way to track cudaMalloc blocks taken
// inside a library; and cudaMalloc/cudaFree may synchronise the device,
// which a host pacing several streams cannot accept in the middle of a
// step.  ecu_matvec_argmax_noalloc gives those callers the HEAD stage's core
// step -- y = W x over raw GGUF blocks plus the reference's argmax -- on
// buffers they already own.
//
// The only memory the computation needs beyond the caller's inputs and
// outputs is the argmax scratch (one partial per CTA, a ticket counter and
// a status word).  It lives in the file-scope array below, 16 KiB that every
// device which loads the library holds until the process exits.
#include "../../include/engine_cuda.h"
#include "ecu_gemv.cuh"
#include "ecu_model.h"

#include <cstddef>

#define NOALLOC_ROWS_PER_CTA 256
#define NOALLOC_MAX_CTAS 2048
#define NOALLOC_MAX_ROWS (NOALLOC_ROWS_PER_CTA * NOALLOC_MAX_CTAS)   // 524288

struct NoallocScratch {
    float     part_val[NOALLOC_MAX_CTAS];
    int       part_idx[NOALLOC_MAX_CTAS];
    StepState st;            // pos stays 0: the argmax lands in tok_hist[0]
    unsigned  counter;       // argmax ticket, must be 0 at launch
    unsigned  pad;
};

// The scratch.  In host code this name is only a stand-in for the device
// symbol: its address must come from cudaGetSymbolAddress on each device.
static __device__ __align__(256) uint8_t g_noalloc_scratch[sizeof(NoallocScratch)];

// Device address of g_noalloc_scratch on the current device.  Looked up on
// every call (cudaGetSymbolAddress allocates nothing and is cheap): a cached
// address would go stale if the caller tore the context down and created it
// again (cudaDeviceReset), which reloads the module and may move the symbol.
static NoallocScratch *scratch_for_current_device(int dev)
{
    void *addr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&addr, g_noalloc_scratch);
    if (e != cudaSuccess || !addr) {
        ecu_set_error(nullptr, 0, "ecu_matvec_argmax_noalloc: cudaGetSymbolAddress failed on device %d: %s",
                      dev, cudaGetErrorString(e));
        return nullptr;
    }
    return (NoallocScratch *)addr;
}

extern "C" int ecu_matvec_argmax_noalloc(unsigned ggml_type, const void *d_w, int n_in, int n_out,
                                         const float *d_x, float *d_y, int *d_token, void *stream)
{
    if (!d_w || !d_x || !d_y || !d_token || n_in <= 0 || n_out <= 0) {
        ecu_set_error(nullptr, 0, "ecu_matvec_argmax_noalloc: null pointer or empty shape");
        return -1;
    }
    if (n_out > NOALLOC_MAX_ROWS) {
        ecu_set_error(nullptr, 0,
                      "ecu_matvec_argmax_noalloc: n_out %d exceeds the no-allocation limit of %d rows "
                      "(%d CTAs x %d rows of argmax scratch)",
                      n_out, NOALLOC_MAX_ROWS, NOALLOC_MAX_CTAS, NOALLOC_ROWS_PER_CTA);
        return -1;
    }
    const int t = (int)ggml_type;
    if (t != GT_F32 && t != GT_F16 && blk_bytes(t) == 0 && t != GT_IQ4_NL) {
        ecu_set_error(nullptr, 0, "ecu_matvec_argmax_noalloc: unknown ggml type %u", ggml_type);
        return -1;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) {
        ecu_set_error(nullptr, 0, "ecu_matvec_argmax_noalloc: no usable current device");
        return -1;
    }
    NoallocScratch *s = scratch_for_current_device(dev);
    if (!s) return -1;
    cudaStream_t st = (cudaStream_t)stream;
    // the array keeps the previous call's contents: zero the state the
    // kernel expects to start at zero (position, status, ticket counter)
    if (cudaMemsetAsync(&s->st, 0, sizeof(StepState) + 2 * sizeof(unsigned), st) != cudaSuccess) {
        ecu_set_error(nullptr, 0, "ecu_matvec_argmax_noalloc: clearing the scratch failed: %s",
                      cudaGetErrorString(cudaGetLastError()));
        return -1;
    }
    GemvArgs a = {};
    a.m.type = t;
    a.m.layout = LAY_RAW;
    a.m.n_in = n_in;
    a.m.n_out = n_out;
    a.m.zero = (t != GT_F32 && t != GT_F16) && (n_in % blk_elems(t) != 0 || !dq_supported(t));
    a.m.row_bytes = t == GT_F32 ? (size_t)n_in * 4 : t == GT_F16 ? (size_t)n_in * 2
                  : (a.m.zero ? 0 : (size_t)(n_in / blk_elems(t)) * blk_bytes(t));
    a.m.total = (size_t)n_in * n_out;
    a.m.data = (const uint8_t *)d_w;
    a.x = d_x;
    a.y = d_y;
    a.part_val = s->part_val;
    a.part_idx = s->part_idx;
    a.counter = &s->counter;
    a.st = &s->st;
    a.tok_hist = d_token;
    a.status = &s->st.status;
    const int grid = (n_out + NOALLOC_ROWS_PER_CTA - 1) / NOALLOC_ROWS_PER_CTA;
    k_gemv_generic<EPI_ARGMAX><<<grid, 256, 0, st>>>(a);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        ecu_set_error(nullptr, 0, "ecu_matvec_argmax_noalloc: launch failed: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}
