/* libquillm_cuda -- the C-ABI shim between quillm's C11 host layer and the hand-written sm_100a kernels.
 *
 * Plain C types only: device pointers are `void *` / typed C pointers into device memory, streams are
 * `void *` (a cudaStream_t, NULL = the library's per-device stream).  Every entry point returns an int
 * status (QMC_OK = 0, negative on error) and never aborts; qmc_last_error() gives the text of the
 * calling thread's last error.  Nothing here allocates on the decode path: model objects allocate all
 * device state when they are created.
 *
 * Reference interfaces replaced (paths relative to the reference project root):
 *   qmc_quantize_rows / qmc_dequantize_rows   src/qm_base.h:39-44   qm_quantize_row_q8/q4, dequantize
 *   qmc_matvec                                src/ops.h:23-25       qm_matvec (Q8_0/Q4_0/f32 weights)
 *   qmc_matmul_nt / qmc_matmul_nt_q           src/ops.h:26-27       qm_matmul_nt (f32), + quantized-W prefill
 *   qmc_rmsnorm/softmax/rope/swiglu           src/ops.h:29-34
 *   qmc_argmax                                src/sampler.h (qm_argmax, src/sampler.c:27-32)
 *   qmc_dot                                   src/kernels.h:9-15    qm_kernels.dot_f32/dot_q8/dot_q4
 *   qmc_model_*                               src/model.h:33-36     qm_model_load/free/forward
 */
#ifndef QUILLM_CUDA_H
#define QUILLM_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#pragma GCC visibility push(default)

enum {
    QMC_OK = 0,
    QMC_EINVAL = -1,   /* bad argument (shape, dtype, alignment, token/pos range) */
    QMC_ECUDA = -2,    /* a CUDA runtime call failed */
    QMC_ENOMEM = -3,   /* device or pinned-host allocation failed */
    QMC_ENCCL = -4,    /* an NCCL call failed */
    QMC_ETIMEOUT = -5, /* a device-side bounded wait expired; the kernel returned early */
    QMC_ESTATE = -6,   /* call out of order (e.g. forward before every tensor was uploaded) */
};

/* tensor dtypes: the .qlm / qm_dtype values (src/qm_base.h:11-15) */
enum { QMC_F32 = 0, QMC_F16 = 1 /* KV cache only */, QMC_Q8_0 = 2, QMC_Q4_0 = 3 };

const char *qmc_last_error(void);
int qmc_device_count(int *count);
/* makes `device` current for the calling thread and creates its stream on first use */
int qmc_set_device(int device);
int qmc_get_device(int *device);
/* the library's stream for the current device (a cudaStream_t) */
int qmc_stream(void **stream);
int qmc_sync(void);
/* reads and clears the device error word set by bounded waits; returns QMC_ETIMEOUT if it was set */
int qmc_check_device_error(void);
/* failure-detection self-test: runs ONE device-side bounded wait that nothing satisfies and returns once
 * the kernel has given up (after the wait limit, ~2 s).  kind 0: the grid-barrier counter poll of the
 * decode step; kind 1: an mbarrier wait of the weight pipeline, after one real bulk copy has landed.
 * The error word is left set, so the next qmc_check_device_error() returns QMC_ETIMEOUT (and clears it);
 * no fault is raised and the context stays usable.  *ms (may be NULL) receives the kernel's duration. */
int qmc_wait_selftest(int kind, float *ms);

/* ---- device buffers (for host layers that own no CUDA code) ---- */
/* page-lock [ptr, ptr + bytes) of host memory (read-only mappings allowed, e.g. a mapped .qlm) so that
 * qmc_model_upload / qmc_upload_tensor copy from it by DMA without a staging copy; undo with
 * qmc_host_unregister before the memory goes away.  The loaders in libquillm do this around their
 * uploads (replaces the reference's mmap-only load, src/qlm_file.c:152-172). */
int qmc_host_register(const void *ptr, size_t bytes);
int qmc_host_unregister(const void *ptr);
int qmc_malloc(void **dptr, size_t bytes);
int qmc_free(void *dptr);
int qmc_memcpy_h2d(void *dst, const void *src, size_t bytes, void *stream);
int qmc_memcpy_d2h(void *dst, const void *src, size_t bytes, void *stream);
int qmc_host_alloc(void **hptr, size_t bytes); /* pinned */
int qmc_host_free(void *hptr);

/* ---- row-wise quantization (bit-exact with the reference quantizer, src/quant.c:33-84) ---- */
/* x[rows][cols] f32 -> rows of Q8_0 / Q4_0 blocks (row bytes = ceil(cols/32) * 34 / 18) */
int qmc_quantize_rows(int dtype, const float *x, void *out, int64_t rows, int64_t cols, void *stream);
int qmc_dequantize_rows(int dtype, const void *in, float *y, int64_t rows, int64_t cols, void *stream);

/* ---- decode matvec: y[rows] = W[rows, cols] . x  (src/ops.c:57-61) ----
 * Quantized W: x is quantized to Q8_0 first (bit-exact); if xq != NULL the ceil(cols/32) Q8_0 blocks
 * are also written there, as the reference's caller-owned scratch receives them.  W must be 16-byte
 * aligned (the TMA staging reads whole 16-byte lines inside [W, W + rows*row_bytes)). */
int qmc_matvec(int dtype, const void *W, int64_t rows, int64_t cols, const float *x, float *y, void *xq,
               void *stream);

/* ---- prefill ----
 * f32 contract of qm_matmul_nt: C[M,N] = A[M,K] . B[N,K]^T  (src/ops.c:81-91) */
int qmc_matmul_nt(const float *A, const float *B, float *C, int64_t M, int64_t N, int64_t K, void *stream);
/* quantized W: row t of C[T,N] equals qmc_matvec(W, A[t]) (A rows quantized to Q8_0) */
int qmc_matmul_nt_q(int dtype, const void *W, const float *A, float *C, int64_t T, int64_t N, int64_t K,
                    void *stream);

/* Same result as qmc_matmul_nt_q, for callers that cannot call cudaMalloc -- code running while a CUDA
 * graph is being captured, or a host application that owns all device memory through its own allocator
 * and forbids a library from allocating.  No counterpart in the reference.  Allocates nothing: the
 * Q8_0-quantized rows of A go to one fixed 8 MiB array in the library's static device memory (held by
 * every GPU that loads the library until the process exits), so T * ceil(K/32) * 36 bytes must fit in
 * 8 MiB (e.g. T = 512 at K = 11008); larger calls return QMC_EINVAL.  The first call on a device looks
 * the array's address up (cudaGetSymbolAddress) and should come before any stream capture.  All calls
 * on a device share the array and each call overwrites it before reading it: two calls whose executions
 * overlap on the GPU (for example on two unsynchronised streams) race.  stream NULL means the CUDA
 * default stream. */
int qmc_matmul_nt_q_noalloc(int dtype, const void *W, const float *A, float *C, int64_t T, int64_t N, int64_t K,
                            void *stream);

/* Split-row weight layout: each row is its ceil(K/32) fp16 block scales (padded to a 16-byte multiple)
 * followed by the blocks' quant bytes (32 per Q8_0 block, 16 per Q4_0 block), so every payload is
 * 16-byte aligned; same numbers as the file's blocks, regrouped.  qmc_split_row_bytes gives the row
 * size; qmc_repack_split writes rows x that many bytes to dst from a .qlm-layout (AoS) matrix. */
int64_t qmc_split_row_bytes(int dtype, int64_t K);
int qmc_repack_split(int dtype, const void *W, int64_t rows, int64_t K, void *dst, void *stream);
/* qmc_matmul_nt_q on the tensor cores (tcgen05.mma kind::i8: one MMA per 32-element block gives the
 * exact int32 block dots, the epilogue applies the block scales in the reference's order), for a
 * split-row weight: the same C bit for bit.  The model's batched prompt forward uses it. */
int qmc_matmul_split_q(int dtype, const void *Wsplit, const float *A, float *C, int64_t T, int64_t N, int64_t K,
                       void *stream);

/* ---- elementwise, in place on device buffers (src/ops.c:93-133) ---- */
int qmc_rmsnorm(float *out, const float *x, const float *w, int64_t n, float eps, void *stream);
int qmc_softmax(float *x, int64_t n, void *stream);
int qmc_rope(float *v, int64_t n_heads, int64_t head_dim, int64_t pos, float theta, void *stream);
int qmc_swiglu(float *gate, const float *up, int64_t n, void *stream);
/* first index of the maximum (src/sampler.c:27-32) into *out_index (device int) */
int qmc_argmax(const float *x, int32_t n, int32_t *out_index, void *stream);
/* one dot of a weight row with Q8_0 activations (dtype Q8_0/Q4_0) or of two f32 vectors (dtype F32,
 * `xq` then holds the second f32 vector); result written to the device float *out */
int qmc_dot(int dtype, const void *w, const void *xq, int64_t n, float *out, void *stream);

/* ---- whole model, one decode step per call (src/model.c:158-191) ---- */
typedef struct qmc_model qmc_model;

typedef struct {
    int32_t dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, max_seq;
    float rope_theta, norm_eps;
} qmc_config;

/* tensor kinds for qmc_model_upload; layer is ignored for the three model-level tensors */
enum {
    QMC_T_TOK_EMBD = 0, QMC_T_NORM = 1, QMC_T_OUTPUT = 2,
    QMC_T_ATTN_NORM = 3, QMC_T_WQ = 4, QMC_T_WK = 5, QMC_T_WV = 6, QMC_T_WO = 7,
    QMC_T_FFN_NORM = 8, QMC_T_W1 = 9, QMC_T_W2 = 10, QMC_T_W3 = 11,
};

/* tp_size 1: single GPU (nccl_id ignored).  tp_size > 1: tensor-parallel rank tp_rank of tp_size, one
 * process per GPU; nccl_id is the 128-byte NCCL unique id made by rank 0 with qmc_nccl_unique_id and
 * shared with the other ranks by the caller.  The current device is used. */
int qmc_model_create(const qmc_config *cfg, int tp_rank, int tp_size, const void *nccl_id, qmc_model **out);
int qmc_nccl_unique_id(void *id128);
/* upload one full (unsharded) tensor from host memory in its .qlm layout; under tensor parallelism each
 * rank keeps only its shard.  rows x cols as in the file (cols = 0 for 1-D norm vectors). */
int qmc_model_upload(qmc_model *m, int kind, int layer, int dtype, int64_t rows, int64_t cols, const void *host);
/* fill every tensor on the device with the seeded N(0, std) generator (norm vectors = 1.0), quantized
 * to `dtype`; produces the same bytes as the oracle's .qlm synthesiser for the same (seed, std). */
int qmc_model_synthesize(qmc_model *m, int dtype, uint64_t seed, double std);
/* one decode step for (token, pos).  logits_host (optional, vocab floats) receives the logits;
 * next_token (optional) receives the greedy argmax.  Returns QMC_EINVAL on a bad token or pos. */
int qmc_model_forward(qmc_model *m, int32_t token, int32_t pos, float *logits_host, int32_t *next_token);
/* batched prompt forward: tokens[0..n) at positions pos0 .. pos0+n-1 through every layer together (each
 * matrix applied once to all n rows), filling those KV-cache slots; logits_host / next_token receive the
 * last token's logits and greedy argmax, as qmc_model_forward at pos0+n-1 would after feeding the prompt
 * one token at a time.  Replaces the reference's token-at-a-time prompt loop (src/main.c:129).  Under
 * tensor parallelism every rank calls it with the same tokens (collective: the wo / w2 partial sums are
 * all-reduced, the logits all-gathered).  Row buffers for n tokens are allocated on the first call that
 * needs them. */
int qmc_model_prefill(qmc_model *m, const int32_t *tokens, int32_t n, int32_t pos0, float *logits_host,
                      int32_t *next_token);
/* greedy generation kept on the device: feeds prompt[0..n_prompt) one token per step from position 0,
 * then appends n_gen greedy tokens; one host synchronisation at the end.  out_tokens gets n_gen ids. */
int qmc_model_generate(qmc_model *m, const int32_t *prompt, int32_t n_prompt, int32_t n_gen, int32_t *out_tokens);
/* enqueue `steps` decode steps that continue greedily from (token, pos) without any host copy: the
 * device-resident loop the bench times; no synchronisation (use qmc_sync).  token < 0 continues from
 * the device's current token and position (the state the previous steps left). */
int qmc_model_enqueue_decode(qmc_model *m, int32_t token, int32_t pos, int32_t steps);
/* synchronise and read the device's next input token and position */
int qmc_model_state(qmc_model *m, int32_t *token, int32_t *pos);
/* device logits buffer (vocab floats, valid after a step) and config */
int qmc_model_logits(qmc_model *m, const float **dev_logits);
int qmc_model_config(const qmc_model *m, qmc_config *cfg);
/* device bytes read per decode step at position pos (weights + KV), for roofline accounting */
int qmc_model_step_bytes(const qmc_model *m, int32_t pos, double *bytes);
/* how a decode step runs, fixed by the first step: *launches = kernel launches per step (1 for the
 * single-launch persistent path: one GPU, Q8_0/Q4_0 matrices; otherwise one per operation), *persistent =
 * 1 for that path.  Before the first step both are 0. */
int qmc_model_decode_info(const qmc_model *m, int32_t *launches, int32_t *persistent);
/* element type of the KV cache: QMC_F32 (default; the reference's fp32 cache, src/model.c:96) or
 * QMC_F16 (each K after RoPE and each V rounded to nearest-even fp16 when stored: half the cache bytes
 * and half the attention reads, numerics beyond the reference's contract).  Only before the model's
 * first step (QMC_ESTATE after it); the cache is reallocated and zeroed. */
int qmc_model_set_kv_dtype(qmc_model *m, int dtype);
int qmc_model_kv_dtype(const qmc_model *m, int *dtype);
int qmc_model_free(qmc_model *m);

/* ---- device-side sampler: temperature / top-k / top-p with the reference's xorshift64* stream
 * (src/sampler.c qm_sampler_init / qm_sample / qm_rng_uniform), drawing from logits in device memory so
 * a decode loop copies back one token instead of the vocab's logits.  Same candidate ranking, nucleus
 * and draw as the reference; probabilities use the device expf and sums run in another order, so a draw
 * can differ only where u falls within rounding of a cumulative-mass boundary. */
typedef struct qmc_sampler qmc_sampler;
/* settings normalised as qm_sampler_init (src/sampler.c:6-16): temperature < 0 -> 0 (greedy), top_k < 0
 * -> 0 (off), top_p outside (0, 1] -> 1 (off), seed 0 -> the reference's fixed default; allocates its
 * state and n_vocab floats of scratch on the current device */
int qmc_sampler_create(int32_t n_vocab, float temperature, int32_t top_k, float top_p, uint64_t seed,
                       qmc_sampler **out);
/* one draw from dev_logits[n_vocab] into *dev_token, enqueued on `stream` (NULL: the thread's stream);
 * the RNG state advances on the device in stream order */
int qmc_sampler_enqueue(qmc_sampler *s, const float *dev_logits, int32_t *dev_token, void *stream);
/* one draw, synchronously, into *token (host) */
int qmc_sampler_sample(qmc_sampler *s, const float *dev_logits, int32_t *token);
/* the current xorshift64* state (synchronises the device) */
int qmc_sampler_rng(qmc_sampler *s, uint64_t *state);
int qmc_sampler_free(qmc_sampler *s);
/* one decode step for (token, pos) whose next token is drawn by the sampler on the device: only the
 * 4-byte token comes back (qm_model_forward + qm_sample of src/main.c without the logits copy) */
int qmc_model_forward_sample(qmc_model *m, int32_t token, int32_t pos, qmc_sampler *s, int32_t *next_token);

#pragma GCC visibility pop
#ifdef __cplusplus
}
#endif
#endif
