/* quillm-b200 Llama-style decoder: drop-in for the reference's src/model.h:1-38.
 *
 * qm_model keeps the reference's public fields that callers read (cfg, file, tensor views, arena,
 * logits, pool, n_threads).  The activations, K/V caches and weights live in HBM, owned by the
 * libquillm_cuda model object `gpu`; the tokenizer (not on the decode path) is not part of this build.
 */
#ifndef QM_MODEL_H
#define QM_MODEL_H

#include "qlm_file.h"
#include "quillm_cuda.h"

#pragma GCC visibility push(default)

typedef struct {
    int32_t dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, max_seq;
    float rope_theta, norm_eps;
} qm_config;

typedef struct {
    const qm_tensor *attn_norm, *wq, *wk, *wv, *wo, *ffn_norm, *w1, *w2, *w3;
} qm_layer;

typedef struct {
    qm_config cfg;
    qlm_file file;
    const qm_tensor *tok_embd, *norm, *output;
    qm_layer *layers;
    qm_arena arena;  /* host: logits */
    float *logits;   /* [vocab], filled by every qm_model_forward */
    qm_pool *pool;
    int n_threads;
    qmc_model *gpu;  /* device state (weights, KV cache, activations, captured decode graph) */
} qm_model;

/* max_seq <= 0 keeps the file's value.  Uploads every tensor to the current CUDA device.  0 on success,
 * -1 with a message in err otherwise (src/model.h:33). */
int qm_model_load(qm_model *m, const char *path, int n_threads, int max_seq, char *err, size_t errlen);
/* tensor-parallel load: this process is rank tp_rank of tp_size (one process per GPU); nccl_id is the
 * 128-byte id from qmc_nccl_unique_id on rank 0, shared by the caller */
int qm_model_load_tp(qm_model *m, const char *path, int max_seq, int tp_rank, int tp_size, const void *nccl_id,
                     char *err, size_t errlen);
void qm_model_free(qm_model *m);
/* one decode step; returns the model-owned logits[vocab] or NULL for a bad token/pos or a GPU error */
float *qm_model_forward(qm_model *m, int32_t token, int32_t pos);
/* batched prompt forward: tokens[0..n) at positions pos0 .. pos0+n-1 in one pass through every layer;
 * returns the model-owned logits of the last token (as qm_model_forward at pos0+n-1 after feeding the
 * prompt token by token, src/main.c:129) or NULL on bad arguments or a GPU error; under tensor
 * parallelism every rank calls it with the same tokens */
float *qm_model_prefill(qm_model *m, const int32_t *tokens, int32_t n, int32_t pos0);
/* greedy generation kept on the device (prompt fed one token per step, then n_gen argmax tokens);
 * 0 on success */
int qm_model_generate(qm_model *m, const int32_t *prompt, int32_t n_prompt, int32_t n_gen, int32_t *out_tokens);
/* KV cache element type after load and before the first step: 0 = fp32 (the reference's cache, the
 * default), 1 = fp16 (half the cache bytes and attention reads; its own tolerance).  0 on success, -1
 * otherwise (bad dtype, or the model has already run a step). */
int qm_model_set_kv_dtype(qm_model *m, int dtype);

#pragma GCC visibility pop
#endif
