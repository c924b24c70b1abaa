/*
 * engine_cuda.h -- C ABI of the B200 (sm_100a) llama token loop.
 *
 * Drop-in for distcomp's CPU engine (src/engine.h:74-101) and its GGUF block
 * dequant (src/gguf.h:86).  Plain C types only: no CUDA or torch types cross
 * this boundary; streams are passed as `void *` (a cudaStream_t, or NULL for
 * the context's own stream).
 *
 * Contract kept from the reference:
 *   - errors are int 0 / -1; open functions write a message into err[errlen]
 *     (src/engine.c:23-27), ecu_last_error() returns the last one per thread;
 *   - a context serves one stage: EMBED, a contiguous LAYERS range or HEAD
 *     (src/engine.h:23-27); ECU_STAGE_FULL is an addition that runs all three
 *     back to back on one device;
 *   - ecu_forward has llm_forward's `out` contract (src/engine.h:83-88):
 *       EMBED  out[0..n_embd)  = embedding row of `token`
 *       LAYERS out in and out  = the state after this stage's layers
 *       HEAD   out[0..n_embd)  = normed state, out[n_embd] = argmax token
 *       FULL   as HEAD, from `token` alone;
 *   - a context is single-threaded, like llm_ctx.
 * Weights are uploaded (and repacked for coalesced loads, values unchanged)
 * once at open; the caller's file buffer may be released afterwards.
 */
#ifndef DC_ENGINE_CUDA_H
#define DC_ENGINE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    ECU_STAGE_EMBED  = 0,   /* src/engine.h:24 LLM_STAGE_EMBED  */
    ECU_STAGE_LAYERS = 1,   /* src/engine.h:25 LLM_STAGE_LAYERS */
    ECU_STAGE_HEAD   = 2,   /* src/engine.h:26 LLM_STAGE_HEAD   */
    ECU_STAGE_FULL   = 3,   /* new: embed + all layers + head on one device */
    ECU_STAGE_SPAN   = 4    /* new: a layer range with the embedding and/or the
                               head folded in (ecu_ctx_open_span) */
};

/* ecu_ctx_open_span flags */
#define ECU_SPAN_EMBED 1u   /* the step starts from a token: embedding row first */
#define ECU_SPAN_HEAD  2u   /* the step ends with the output head: argmax token */
#define ECU_SPAN_FFN_FIRST 4u   /* layer `first` contributes its FFN half only (RMSNorm,
                                   gate/up, SwiGLU, down + residual) */
#define ECU_SPAN_ATTN_LAST 8u   /* layer `last` contributes its attention half only
                                   (RMSNorm, Q/K/V, attention, attn_output + residual):
                                   a pipeline may cut a layer between its halves */

typedef struct ecu_model ecu_model;   /* host view of a GGUF file (borrowed bytes) */
typedef struct ecu_ctx   ecu_ctx;     /* one stage resident on one device           */

/* Geometry of an open context (the fields of llm_ctx, src/engine.h:46-70). */
typedef struct {
    int   n_layer, n_embd, n_head, n_head_kv, n_ff, head_dim, n_vocab, n_rep, n_ctx;
    int   stage, first, last, pos, device;
    float rms_eps, rope_base;
    size_t device_bytes;      /* weights + KV cache + work buffers on the device */
} ecu_info;

/* ---- GGUF view --------------------------------------------------------- */

/* Parse a GGUF v2/v3 image held by the caller (replaces gguf_open,
 * src/gguf.h:52).  Tensor data stay in `file` until a context is opened. */
int  ecu_model_open(ecu_model **out, const void *file, size_t size, char *err, size_t errlen);

/* Assemble a model from tensor views and metadata instead of a file image,
 * as dcd's shard role does when it builds a gguf_file from received tensors
 * (src/daemon.c:963-1019). */
/* The same from a GGUF file on disk: mapped read-only, so that a context
 * opened from it reads (pages in) only its stage's tensors, and the model
 * owns the mapping until ecu_model_close.  Replaces the reference's whole-
 * file fread (src/shard.c:84-104, llm_open_file) for stage nodes. */
int  ecu_model_open_file(ecu_model **out, const char *path, char *err, size_t errlen);

ecu_model *ecu_model_new(void);
int  ecu_model_set_str(ecu_model *m, const char *key, const char *val);
int  ecu_model_set_u32(ecu_model *m, const char *key, unsigned long val);
int  ecu_model_set_f32(ecu_model *m, const char *key, float val);
int  ecu_model_add_tensor(ecu_model *m, const char *name, unsigned n_dims, const uint64_t *dims,
                          unsigned ggml_type, const void *data, size_t nbytes);
void ecu_model_close(ecu_model *m);
/* Number of tensors, and lookup by name (gguf_tensor_find, src/gguf.h:72). */
size_t ecu_model_n_tensors(const ecu_model *m);
int  ecu_model_tensor(const ecu_model *m, const char *name, unsigned *ggml_type,
                      unsigned *n_dims, uint64_t dims[4], const void **data, size_t *nbytes);

/* ---- engine (src/engine.h:72-101) -------------------------------------- */

/* Device bytes a stage needs at context length n_ctx (0 = the model's);
 * the device counterpart of llm_ctx_floats (src/engine.h:74).  0 on error. */
size_t ecu_ctx_bytes(const ecu_model *m, int stage, int first, int last, int n_ctx);

/* Open a stage on CUDA device `device` (replaces llm_ctx_open,
 * src/engine.h:79).  The same geometry and error rules as the reference. */
int  ecu_ctx_open(ecu_ctx **out, const ecu_model *m, int stage, int first, int last, int n_ctx,
                  int device, char *err, size_t errlen);
/* A pipeline stage that folds the reference's EMBED / LAYERS / HEAD stages
 * of one node into one context (src/shard.c:358-437 gives a node's layer
 * range; its entry node also embeds, its exit node also runs the head):
 * layers first..last (first > last: none) plus the embedding and/or the
 * head by `flags`; with ECU_SPAN_FFN_FIRST / ECU_SPAN_ATTN_LAST the range
 * starts at layer first's FFN half / ends with layer last's attention half
 * (a layer cut between two GPUs: the residual stream is all that crosses).
 * One persistent step per token runs all of it.  Forward
 * contract: input a token with ECU_SPAN_EMBED, else a state in out;
 * output the state, plus out[n_embd] = the argmax with ECU_SPAN_HEAD.  The
 * position advances every step.  ecu_ctx_info reports ECU_STAGE_SPAN. */
int  ecu_ctx_open_span(ecu_ctx **out, const ecu_model *m, int first, int last, unsigned flags, int n_ctx,
                       int device, char *err, size_t errlen);
void ecu_ctx_close(ecu_ctx *c);
int  ecu_ctx_info(const ecu_ctx *c, ecu_info *info);
/* How the context runs a step: "persistent" (one cooperative kernel per
 * token, every phase of the stage inside it) or "kernels: <reason>" (one
 * kernel per operation, and why the persistent kernel does not apply).
 * No reference counterpart (the CPU engine has one implementation). */
const char *ecu_ctx_path(const ecu_ctx *c);

/* One token through the stage, host `out` (replaces llm_forward,
 * src/engine.h:88).  -1 for a token outside the vocabulary (EMBED/FULL) or
 * an exhausted context (LAYERS/FULL). */
int  ecu_forward(ecu_ctx *c, int token, float *out);
/* Rewind the KV cache (replaces llm_reset, src/engine.h:90). */
void ecu_reset(ecu_ctx *c);
/* Exactly one layer at the current position, position unchanged
 * (replaces llm_layer_once, src/engine.h:94). */
int  ecu_layer_once(ecu_ctx *c, int layer_idx, float *out);
/* The first n layers of the stage (0 = all), then pos++ (replaces
 * llm_step_layers, src/engine.h:98). */
int  ecu_step_layers(ecu_ctx *c, int n, float *out);
/* Argmax of the last HEAD/FULL logits, lowest index on ties (replaces
 * llm_pick, src/engine.h:101). */
int  ecu_pick(const ecu_ctx *c);
/* Copy the last logits to host memory (n floats, n <= n_vocab). */
int  ecu_get_logits(const ecu_ctx *c, float *out, size_t n);
/* Set the cache position directly (what engine_stages.c does with lay.pos). */
int  ecu_set_pos(ecu_ctx *c, int pos);

/* ---- device-resident chaining (no host hop between stages) ------------- */

/* Device pointer of the stage's state buffer (n_embd + 1 floats).  LAYERS
 * and HEAD read their input there; every stage leaves its output there. */
float *ecu_state_ptr(ecu_ctx *c);
/* ecu_forward without host copies: input/output in ecu_state_ptr(c),
 * enqueued on `stream` (NULL = the context's stream), not synchronised.
 * The token is read from host memory at enqueue time. */
int  ecu_forward_dev(ecu_ctx *c, int token, void *stream);
/* Device address of the context's current token (one int).  EMBED and FULL
 * steps read their input token there; HEAD and FULL steps write their argmax
 * there.  A pipeline hands the token from the last stage to the first by
 * writing this address (a device copy or an NCCL receive), the way the
 * reference's shard.c sends the argmax back to the entry node. */
int *ecu_token_ptr(ecu_ctx *c);
/* One step from device-resident input only: the token at ecu_token_ptr(c)
 * (EMBED/FULL) or the state at ecu_state_ptr(c) (LAYERS/HEAD), output left
 * in the state buffer (and the token word for HEAD/FULL), position advanced.
 * Enqueued on `stream` (NULL = the context's stream), not synchronised; a
 * token outside the vocabulary is reported by the next ecu_sync.  -1 when
 * the context is exhausted. */
int  ecu_step_dev(ecu_ctx *c, void *stream);
/* A second context of the same stage on the same device that shares the
 * first one's uploaded weights and keeps its own KV cache, position, work
 * buffers and stream: one per concurrent sequence (the reference keeps one
 * llm_ctx per process, src/daemon.c:757; a GPU stage serving several
 * interleaved sequences needs one cache each).  The weights are freed when
 * the last context holding them closes. */
int  ecu_ctx_fork(ecu_ctx **out, ecu_ctx *base, char *err, size_t errlen);

/* ---- tensor parallelism (the alternative partition to shard.c's layer
 * ranges, src/shard.c:358-437): one FULL context per GPU, rank r of w owns
 * query/KV heads [r*n/w, ..), the matching rows of the fused Q/K/V, rows
 * [r*n_embd/w, ..) of attn_output and ffn_down, FFN channels [r*n_ff/w, ..)
 * and a vocabulary slice of the head.  Every projection keeps its whole
 * input, so each output element is computed by one rank with the one-GPU
 * arithmetic (bit-identical results); the ranks exchange outputs inside the
 * persistent step through each other's memory (NVLink peer stores).  Steps
 * must be issued on every rank in the same order (ecu_forward / decode);
 * a rank that falls more than ~2 s behind makes the others' step fail with
 * a timeout status. */
#define ECU_TP_HANDLE_BYTES 64
int  ecu_ctx_open_tp(ecu_ctx **out, const ecu_model *m, int n_ctx, int device, int tp_rank, int tp_world,
                     char *err, size_t errlen);
/* This rank's shareable handle (ECU_TP_HANDLE_BYTES) for the other ranks. */
int  ecu_tp_handle(ecu_ctx *c, unsigned char *out);
/* Map every rank's handle (world * ECU_TP_HANDLE_BYTES, rank order; this
 * rank's own entry is ignored).  Call once, on every rank, before a step. */
int  ecu_tp_connect(ecu_ctx *c, const unsigned char *handles);
/* out4 = {rank, world, first vocabulary row, end row} of this context's head
 * slice (ecu_get_logits returns that slice). */
int  ecu_tp_slice(const ecu_ctx *c, int *out4);
/* ---- pipeline links: the stages of a layer pipeline (one context per GPU
 * and sequence, typically spans) hand the state and the token to each
 * other inside their persistent steps, as tagged words written straight
 * into the next stage's memory over NVLink, instead of a host or NCCL hop
 * between steps (the reference sends them over UDP, src/shard.c:664-723).
 * Each stage's step then only needs launching, in the same sequence order
 * on every GPU: a step waits (bounded, ~2 s, then the status reports a
 * timeout) until its input has arrived.  Contexts with the persistent step
 * only, not tensor-parallel ones; every stage of a pipeline opened from the
 * same model.  Use ecu_step_dev on linked contexts. */
#define ECU_LINK_HANDLE_BYTES 64
/* This context's shareable handle (ECU_LINK_HANDLE_BYTES), for the stage
 * before it (another process: CUDA IPC). */
int  ecu_link_handle(ecu_ctx *c, unsigned char *out);
/* Send this context's output to the stage whose handle this is: its output
 * state, or with the head its argmax token (to the first stage). */
int  ecu_link_next(ecu_ctx *c, const unsigned char *handle);
/* The same for a context of this process (next may be on the same device;
 * then its steps must follow this one's on one stream). */
int  ecu_link_next_local(ecu_ctx *c, ecu_ctx *next);
/* This context's input arrives over a link: the state for a stage without
 * the embedding, else the token.  Once set, ecu_forward is refused. */
int  ecu_link_input(ecu_ctx *c);
/* A linked first stage's input token for its next step from the host (the
 * token the prompt's last position picked), enqueued on `stream` (NULL =
 * the context's stream) before that step. */
int  ecu_link_feed(ecu_ctx *c, int token, void *stream);

/* Greedy decode on a FULL context without host round trips: feeds
 * prompt[0..n_prompt) token by token, then generates n_gen tokens, each one
 * fed back on the device.  out_tokens receives the n_gen generated ids.
 * Returns 0, or -1 when the context runs out. */
int  ecu_generate(ecu_ctx *c, const int *prompt, int n_prompt, int n_gen, int *out_tokens);
/* A prompt of n tokens through a FULL context at once (the reference feeds
 * prompts token by token, src/shard.c:911-917, one llm_forward each): every
 * layer runs its n tokens as one batch (GEMMs on the tensor cores with
 * split-fp16 operands, about fp32 accuracy; causal attention over the
 * cache), the cache gets the n positions, and the last token goes through
 * the head: out = normed state (n_embd) + the picked token, as ecu_forward's
 * out for that token, and the context's position advances by n.  Results
 * agree with the token-by-token path within the 1e-3 bar, not bit for bit.
 * Shapes the batched kernels do not cover (unfused projections, head_dim
 * other than 64/128, n_ctx > 8192) and tensor-parallel ranks run the
 * per-token step instead.  Scratch for the batch is allocated on first use
 * and grows with the longest prompt. */
int  ecu_prefill(ecu_ctx *c, const int *tokens, int n, float *out);

/* The batched prompt for one stage of a layer pipeline (src/shard.c:358-437
 * splits the model into EMBED, LAYERS ranges and HEAD; the reference feeds
 * the prompt through them token by token, src/shard.c:911-917).  x: device
 * memory the caller owns, n rows of n_embd floats (the n prompt positions).
 * EMBED: x = the embedding rows of tokens[0..n).  LAYERS: x goes through the
 * stage's layers in place (ecu_prefill's kernels), the stage's KV cache
 * gets positions pos..pos+n-1 and its position advances by n.  HEAD: the
 * last row of x through the head, out = normed state + picked token as
 * ecu_forward's (tokens may be NULL).  SPAN: those of its parts in that
 * order, the position advancing by n.  Every stage's rows agree bit for bit
 * with a FULL context's ecu_prefill of the same prompt.  Synchronises the
 * context's stream before returning. */
int  ecu_prefill_rows(ecu_ctx *c, const int *tokens, int n, float *x, float *out);
/* Decode steps on a FULL context continuing from the token in the state
 * buffer, on the context's stream, without synchronising; used to time the
 * device-side loop.  Returns 0 or -1. */
int  ecu_decode_async(ecu_ctx *c, int n_steps);
/* Wait for the context's stream; returns -1 if a kernel reported an error. */
int  ecu_sync(ecu_ctx *c);
/* The context's CUDA stream (as void *). */
void *ecu_stream(ecu_ctx *c);

/* ---- block dequant on the device (replaces gguf_dequant, src/gguf.h:86) - */

/* Dequantise elements [off, off+n) of a tensor of `total` elements and ggml
 * type `ggml_type` whose raw GGUF blocks are at host pointer `raw`, on
 * device `device`, into host `dst`.  Same rejection rules as the reference
 * (range, block-aligned off, supported types).  Bit-exact with it. */
int  ecu_dequant(unsigned ggml_type, const void *raw, size_t total, size_t off, size_t n,
                 float *dst, int device);
/* The same from a context's uploaded (repacked) copy of tensor `name`,
 * proving the device layout holds the file's values. */
int  ecu_dequant_tensor(ecu_ctx *c, const char *name, size_t off, size_t n, float *dst);

/* ---- single-GEMV entry point (the quantised matvec of src/engine.c:348) - */

/* y[o] = sum_i W[i + o*n_in] x[i] for a raw GGUF weight at host pointer
 * `w_raw` on `device`; x and y are host arrays.  Uploads per call: for
 * tests and one-off use, not the token loop. */
int  ecu_matvec(unsigned ggml_type, const void *w_raw, int n_in, int n_out, const float *x,
                float *y, int device);

/* ---- without device allocation ------------------------------------------ */

/* y = W x over raw GGUF blocks already in device memory (n_out rows of
 * n_in inputs, the file's block order), and *d_token = the first maximum of
 * y with llm_pick's rules, enqueued on `stream` (NULL = the legacy default
 * stream) without synchronising.  All pointers are device pointers the
 * caller owns.  No counterpart in the reference: it is for callers that
 * cannot allocate device memory -- a shard node held to a fixed memory
 * budget, a host that hands out device memory from its own pool, a loop
 * that cannot take cudaMalloc's device synchronisation.  It allocates
 * nothing: its scratch is one fixed 16 KiB array inside the library, which
 * limits n_out to 524288 rows (more returns -1 with a message).  Every
 * call looks that array's device address up with cudaGetSymbolAddress
 * (which allocates nothing), so the address stays right across a context
 * torn down and created again; make the first call on a device before any
 * stream capture.  Every call shares the array, so calls that may overlap
 * on the GPU (two streams, two threads) race: serialise them. */
int  ecu_matvec_argmax_noalloc(unsigned ggml_type, const void *d_w, int n_in, int n_out,
                               const float *d_x, float *d_y, int *d_token, void *stream);

/* ---- failure-path testing ------------------------------------------------ */

/* No counterpart in the reference, whose failure paths are host retries and
 * aborts (src/shard.c:533-545).  Every wait inside the engine's kernels (a
 * tagged word from another CTA or rank, a bulk copy's barrier) is bounded:
 * after the limit it sets the context's status word and lets the kernel run
 * to its end, and the step returns -1.  ecu_set_wait_ns sets that limit on
 * `device` (default 2 s; between launches).  ecu_inject_wait_timeout makes
 * the next persistent step of `c` wait, in its first GEMV phase with a
 * tagged input, for an input word that no phase writes: its waits run out,
 * that step returns -1 with the timeout in ecu_last_error, and the context
 * steps normally again afterwards (reset it: that step's cache row is not
 * valid).  -1 for a context on the per-kernel step. */
int  ecu_set_wait_ns(int device, unsigned long long ns);
int  ecu_inject_wait_timeout(ecu_ctx *c);

/* ---- measurement --------------------------------------------------------- */

/* Quantised-matvec microbenchmark (the reference's matvec,
 * src/engine.c:277-357, timed on the device): `copies` device copies of one
 * n_out x n_in matrix of raw GGUF blocks (host array w_raw, repacked into
 * the layouts the engine keeps), then `rounds` replays of a CUDA graph of
 * one launch of y = W_c x per copy, back to back; *ms_per_launch = CUDA
 * event time / launches.  Enough copies to exceed the L2 make every launch
 * stream its matrix from HBM.  y (host) = the last launch's output. */
int  ecu_matvec_bench(unsigned ggml_type, const void *w_raw, int n_in, int n_out, const float *x,
                      float *y, int device, int copies, int rounds, double *ms_per_launch);

/* The same matrices streamed through the persistent step's GEMV phases: one
 * cooperative launch runs one phase per copy (y = W_c x, plain x, each CTA's
 * rows through its shared-memory ring, the next copy's rows already in
 * flight while a phase ends), `rounds` launches timed with CUDA events;
 * *ms_per_matvec = time / (rounds * copies).  The decode step consumes its
 * weight matrices this way.  Q4_0 / Q8_0 / Q4_K with n_in a multiple of
 * 1024 (the fast layouts); -1 otherwise. */
int  ecu_matvec_stream_bench(unsigned ggml_type, const void *w_raw, int n_in, int n_out, const float *x,
                             float *y, int device, int copies, int rounds, double *ms_per_matvec);

/* Per-kernel-kind totals of a profiling replay. */
typedef struct {
    char   kind[32];          /* "gemv_gate_up", "attention", ...               */
    int    launches;
    double total_ms;          /* sum of CUDA-event durations of those launches  */
    double bytes_per_launch;  /* algorithmic bytes: weights as stored in the
                                 file + vectors read and written                 */
} ecu_kprof;

/* One persistent step with every CTA's time (globaltimer ns) at the start
 * and at the end of each phase: out[(p + 1) * grid + cta] = the end of
 * phase p, out[cta] = the start; n_words >= (phases + 1) * grid (*grid =
 * the CTA count, the SM count).  kinds (optional) receives the phases'
 * names, comma-separated.  Returns the number of phases, or -1.  The
 * position advances as in a step.  For measuring the CTAs' skew at phase
 * boundaries. */
int  ecu_profile_cta_ns(ecu_ctx *c, unsigned long long *out, size_t n_words, int *grid, char *kinds,
                        size_t kinds_len);
/* Run n_steps decode steps of a FULL (or LAYERS) context without the graph,
 * with a pair of CUDA events around every kernel on the context's stream,
 * and aggregate the durations per kernel kind into out[0..max_kinds).  The
 * steps are real decode steps (the position advances).  Returns the number
 * of kinds written, or -1. */
int  ecu_profile_steps(ecu_ctx *c, int n_steps, ecu_kprof *out, int max_kinds);

/* ---- misc -------------------------------------------------------------- */

const char *ecu_last_error(void);
/* Number of kernels this process has launched through the engine. */
uint64_t ecu_kernel_launches(void);
/* Library version string. */
const char *ecu_version(void);

#ifdef __cplusplus
}
#endif
#endif
