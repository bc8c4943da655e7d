/* quillm-b200 model driver: the reference's qm_model_* API (src/model.h:33-36) over libquillm_cuda.
 * Load = the reference's metadata and shape checks (src/model.c:35-90) + one upload of every tensor to
 * HBM; forward = one replay of the captured decode graph, logits copied back into m->logits. */
#include "model.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "hostgpu.h"

static int meta_u32(const qlm_file *f, const char *key, int32_t *out, char *err, size_t errlen) {
    const qlm_kv *kv = qlm_find_kv(f, key);
    if (!kv || kv->type != QLM_KV_U32 || kv->u32 == 0 || kv->u32 > (1u << 24)) {
        snprintf(err, errlen, "missing/invalid metadata '%s'", key);
        return -1;
    }
    *out = (int32_t)kv->u32;
    return 0;
}

static float meta_f32(const qlm_file *f, const char *key, float fallback) {
    const qlm_kv *kv = qlm_find_kv(f, key);
    return (kv && kv->type == QLM_KV_F32) ? kv->f32 : fallback;
}

/* tensor `name` with shape (d0) [f32 vector] or (d0, d1) */
static const qm_tensor *find_shaped(const qlm_file *f, const char *name, int64_t d0, int64_t d1, char *err,
                                    size_t errlen) {
    const qm_tensor *t = qlm_find_tensor(f, name);
    int ok = 0;
    if (t && d1 == 0) ok = t->ndim == 1 && t->ne[0] == d0 && t->type == QM_F32;
    else if (t) ok = t->ndim == 2 && t->ne[0] == d0 && t->ne[1] == d1;
    if (!ok) {
        snprintf(err, errlen, "missing or mis-shaped tensor '%s'", name);
        return NULL;
    }
    return t;
}

static int upload(qm_model *m, int kind, int layer, const qm_tensor *t, char *err, size_t errlen) {
    const int64_t rows = t->ne[0], cols = t->ndim == 2 ? t->ne[1] : 0;
    if (qmc_model_upload(m->gpu, kind, layer, (int)t->type, rows, cols, t->data) != QMC_OK) {
        snprintf(err, errlen, "upload of '%s' failed: %s", t->name, qmc_last_error());
        return -1;
    }
    return 0;
}

static int load_common(qm_model *m, const char *path, int n_threads, int max_seq, int tp_rank, int tp_size,
                       const void *nccl_id, char *err, size_t errlen) {
    memset(m, 0, sizeof *m);
    if (qlm_open(&m->file, path, err, errlen) != 0) return -1;
    const qlm_file *f = &m->file;
    qm_config *c = &m->cfg;
    if (meta_u32(f, "llama.dim", &c->dim, err, errlen) || meta_u32(f, "llama.hidden_dim", &c->hidden_dim, err, errlen) ||
        meta_u32(f, "llama.n_layers", &c->n_layers, err, errlen) ||
        meta_u32(f, "llama.n_heads", &c->n_heads, err, errlen) ||
        meta_u32(f, "llama.n_kv_heads", &c->n_kv_heads, err, errlen) ||
        meta_u32(f, "llama.vocab_size", &c->vocab_size, err, errlen) ||
        meta_u32(f, "llama.max_seq", &c->max_seq, err, errlen))
        goto fail;
    c->rope_theta = meta_f32(f, "llama.rope_theta", 10000.0f);
    c->norm_eps = meta_f32(f, "llama.norm_eps", 1e-5f);
    if (c->dim % c->n_heads || c->n_heads % c->n_kv_heads || (c->dim / c->n_heads) % 2 || c->n_layers > 1024) {
        snprintf(err, errlen, "inconsistent head configuration");
        goto fail;
    }
    if (max_seq > 0 && max_seq < c->max_seq) c->max_seq = max_seq;
    const int64_t D = c->dim, H = c->hidden_dim, KV = (int64_t)c->dim / c->n_heads * c->n_kv_heads, V = c->vocab_size;
    if (!(m->tok_embd = find_shaped(f, "tok_embd", V, D, err, errlen)) ||
        !(m->norm = find_shaped(f, "norm", D, 0, err, errlen)) ||
        !(m->output = find_shaped(f, "output", V, D, err, errlen)))
        goto fail;
    m->layers = calloc((size_t)c->n_layers, sizeof(qm_layer));
    if (!m->layers) {
        snprintf(err, errlen, "out of memory");
        goto fail;
    }
    static const char *names[9] = {"attn_norm", "wq", "wk", "wv", "wo", "ffn_norm", "w1", "w2", "w3"};
    for (int l = 0; l < c->n_layers; l++) {
        const int64_t shp[9][2] = {{D, 0}, {D, D}, {KV, D}, {KV, D}, {D, D}, {D, 0}, {H, D}, {D, H}, {H, D}};
        const qm_tensor **slot[9] = {&m->layers[l].attn_norm, &m->layers[l].wq, &m->layers[l].wk,
                                     &m->layers[l].wv,        &m->layers[l].wo, &m->layers[l].ffn_norm,
                                     &m->layers[l].w1,        &m->layers[l].w2, &m->layers[l].w3};
        for (int k = 0; k < 9; k++) {
            char nm[64];
            snprintf(nm, sizeof nm, "layers.%d.%s", l, names[k]);
            if (!(*slot[k] = find_shaped(f, nm, shp[k][0], shp[k][1], err, errlen))) goto fail;
        }
    }
    if (qh_begin() != 0) {
        snprintf(err, errlen, "%s", qm_last_error());
        goto fail;
    }
    qh_end();
    qmc_config qc = {c->dim, c->hidden_dim, c->n_layers, c->n_heads, c->n_kv_heads, c->vocab_size, c->max_seq,
                     c->rope_theta, c->norm_eps};
    if (qmc_model_create(&qc, tp_rank, tp_size, nccl_id, &m->gpu) != QMC_OK) {
        snprintf(err, errlen, "device model: %s", qmc_last_error());
        goto fail;
    }
    /* page-lock the mapped file for the uploads so every tensor goes to HBM by DMA straight from the
     * mapping (no staging copy); without it (registration refused) the uploads still work, slower */
    const int pinned = qmc_host_register(f->map, f->map_size) == QMC_OK;
    if (!pinned) qmc_last_error();
    int up_rc = upload(m, QMC_T_TOK_EMBD, -1, m->tok_embd, err, errlen) || upload(m, QMC_T_NORM, -1, m->norm, err, errlen) ||
                upload(m, QMC_T_OUTPUT, -1, m->output, err, errlen);
    static const int kinds[9] = {QMC_T_ATTN_NORM, QMC_T_WQ, QMC_T_WK, QMC_T_WV, QMC_T_WO,
                                 QMC_T_FFN_NORM,  QMC_T_W1, QMC_T_W2, QMC_T_W3};
    for (int l = 0; l < c->n_layers && !up_rc; l++) {
        const qm_tensor *ts[9] = {m->layers[l].attn_norm, m->layers[l].wq, m->layers[l].wk,
                                  m->layers[l].wv,        m->layers[l].wo, m->layers[l].ffn_norm,
                                  m->layers[l].w1,        m->layers[l].w2, m->layers[l].w3};
        for (int k = 0; k < 9 && !up_rc; k++) up_rc = upload(m, kinds[k], l, ts[k], err, errlen);
    }
    if (pinned) qmc_host_unregister(f->map);
    if (up_rc) goto fail;
    if (qm_arena_init(&m->arena, (size_t)V * 4 + QM_ALIGN) != 0 || !(m->logits = qm_arena_alloc(&m->arena, (size_t)V * 4))) {
        snprintf(err, errlen, "out of memory for runtime state");
        goto fail;
    }
    m->n_threads = n_threads < 1 ? 1 : n_threads;
    m->pool = qm_pool_create(m->n_threads);
    return 0;
fail:
    qm_model_free(m);
    return -1;
}

int qm_model_load(qm_model *m, const char *path, int n_threads, int max_seq, char *err, size_t errlen) {
    return load_common(m, path, n_threads, max_seq, 0, 1, NULL, err, errlen);
}

int qm_model_load_tp(qm_model *m, const char *path, int max_seq, int tp_rank, int tp_size, const void *nccl_id,
                     char *err, size_t errlen) {
    return load_common(m, path, 1, max_seq, tp_rank, tp_size, nccl_id, err, errlen);
}

void qm_model_free(qm_model *m) {
    if (m->gpu) qmc_model_free(m->gpu);
    qm_pool_destroy(m->pool);
    if (m->arena.base) qm_arena_free(&m->arena);
    free(m->layers);
    qlm_close(&m->file);
    memset(m, 0, sizeof *m);
}

float *qm_model_forward(qm_model *m, int32_t token, int32_t pos) {
    const qm_config *c = &m->cfg;
    if (token < 0 || token >= c->vocab_size || pos < 0 || pos >= c->max_seq) return NULL;
    if (qmc_model_forward(m->gpu, token, pos, m->logits, NULL) != QMC_OK) {
        qh_fail("qm_model_forward");
        return NULL;
    }
    return m->logits;
}

float *qm_model_prefill(qm_model *m, const int32_t *tokens, int32_t n, int32_t pos0) {
    if (!tokens || n < 1 || pos0 < 0 || (int64_t)pos0 + n > m->cfg.max_seq) return NULL;
    if (qmc_model_prefill(m->gpu, tokens, n, pos0, m->logits, NULL) != QMC_OK) {
        qh_fail("qm_model_prefill");
        return NULL;
    }
    return m->logits;
}

int qm_model_set_kv_dtype(qm_model *m, int dtype) {
    if (qmc_model_set_kv_dtype(m->gpu, dtype) != QMC_OK) {
        qh_fail("qm_model_set_kv_dtype");
        return -1;
    }
    return 0;
}

int qm_model_generate(qm_model *m, const int32_t *prompt, int32_t n_prompt, int32_t n_gen, int32_t *out_tokens) {
    if (qmc_model_generate(m->gpu, prompt, n_prompt, n_gen, out_tokens) != QMC_OK) {
        qh_fail("qm_model_generate");
        return -1;
    }
    return 0;
}
