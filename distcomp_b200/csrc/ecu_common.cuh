// ecu_common.cuh -- shared definitions of the sm_100a engine.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stddef.h>

// ggml tensor types as stored in GGUF (src/gguf.c:149-174 lists the sizes).
enum GgmlType : int {
    GT_F32 = 0, GT_F16 = 1, GT_Q4_0 = 2, GT_Q4_1 = 3, GT_Q5_0 = 6, GT_Q5_1 = 7,
    GT_Q8_0 = 8, GT_Q8_1 = 9, GT_Q2_K = 10, GT_Q3_K = 11, GT_Q4_K = 12, GT_Q5_K = 13,
    GT_Q6_K = 14, GT_Q8_K = 15, GT_IQ4_NL = 16
};

// Device layouts of a weight matrix.  RAW keeps the GGUF block stream;
// SPLIT4/SPLIT8 move the fp16 block scales of Q4_0/Q8_0 out of the 18/34-byte
// blocks so that codes load as aligned 16-byte runs:
//   SPLIT4 row: [16 code bytes of block 0..nb-1][nb fp16 scales][pad to 16 B]
//   SPLIT8 row: [code bytes 0..15 of block 0..nb-1][code bytes 16..31 of
//                block 0..nb-1][nb fp16 scales][pad to 16 B]
// SPLITK4 does the same for Q4_K (256-weight super-blocks of 144 bytes:
// d, dmin, 12 bytes of 6-bit scales/mins, 128 code bytes): every 32-weight
// sub-block gets 16 code bytes in the Q4_0 nibble order (byte l: weight l in
// the low nibble, weight l+16 in the high one), then the 16-byte headers:
//   SPLITK4 row: [16 code bytes of sub-block 0..nb-1][nb/8 headers (d, dmin,
//                scales[12])]
// Values are untouched; only the byte order within a row changes.
enum Layout : int { LAY_RAW = 0, LAY_SPLIT4 = 1, LAY_SPLIT8 = 2, LAY_SPLITK4 = 3 };

__host__ __device__ inline int blk_elems(int t)
{
    return (t >= GT_Q2_K && t <= GT_Q8_K) ? 256 : 32;
}

__host__ __device__ inline int blk_bytes(int t)
{
    switch (t) {
    case GT_Q4_0: return 18;  case GT_Q4_1: return 20;  case GT_Q5_0: return 22;
    case GT_Q5_1: return 24;  case GT_Q8_0: return 34;  case GT_Q8_1: return 36;
    case GT_Q2_K: return 84;  case GT_Q3_K: return 110; case GT_Q4_K: return 144;
    case GT_Q5_K: return 176; case GT_Q6_K: return 210; case GT_Q8_K: return 292;
    default: return 0;
    }
}

// Types the block decoder understands (the reference rejects the rest,
// src/gguf.c:765-766).
__host__ __device__ inline bool dq_supported(int t)
{
    return t == GT_F32 || t == GT_F16 || t == GT_Q4_0 || t == GT_Q4_1 || t == GT_Q5_0 ||
           t == GT_Q5_1 || t == GT_Q8_0 || (t >= GT_Q2_K && t <= GT_Q8_K);
}

// Bytes of n elements (src/gguf.c:149-174 tensor_nbytes); 0 for unknown types.
inline size_t type_nbytes(int t, size_t n)
{
    if (t == GT_F32) return n * 4;
    if (t == GT_F16) return n * 2;
    if (t == GT_IQ4_NL) return n / 32 * 2;
    int b = blk_bytes(t);
    return b ? n / (size_t)blk_elems(t) * (size_t)b : 0;
}

// A weight matrix resident on the device: n_out rows of n_in inputs.  A
// wide matrix is kept as nseg column segments (inputs [s*n_in/nseg, ..)),
// each a complete matrix of its own, back to back seg_bytes apart; row_bytes
// is then a segment's row.
struct DevMat {
    int            type = -1;
    int            layout = LAY_RAW;
    int            n_in = 0, n_out = 0;
    size_t         row_bytes = 0;      // bytes between consecutive rows
    size_t         total = 0;          // elements of the source tensor
    const uint8_t *data = nullptr;     // device
    bool           zero = false;       // matvec yields zeros (engine.c:317-320 rule)
    int            nseg = 1;
    size_t         seg_bytes = 0;
};

// Per-step device state shared by the kernels of one context.
struct StepState {
    int pos;        // cache position of the current token
    int token;      // current input token
    int status;     // nonzero: a kernel gave up on a bounded wait, or read a bad token
    int pad;
};

#define ECU_STATUS_TIMEOUT 1
#define ECU_STATUS_BADTOKEN 2

// -------------------------------------------------------------- helpers ----

__device__ __forceinline__ float ld_f16(const uint8_t *p)
{
    // byte loads: GGUF blocks are not 2-byte aligned in general
    unsigned short h = (unsigned short)(p[0] | (p[1] << 8));
    return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ uint32_t ld_u32_bytes(const uint8_t *p)
{
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) |
           ((uint32_t)p[3] << 24);
}

// Programmatic dependent launch: wait for the producing grid's memory, and
// let the next grid start its prologue.  Both are no-ops when the launch
// carries no programmatic dependency.
__device__ __forceinline__ void pdl_wait()
{
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void pdl_trigger()
{
    asm volatile("griddepcontrol.launch_dependents;" :::);
}
