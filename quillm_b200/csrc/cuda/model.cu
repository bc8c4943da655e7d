// Whole-model decode on the device (src/model.c:158-191), one CUDA graph per model.
//
// HBM layout (per GPU; with tensor parallelism each rank holds its shard):
//   wqkv  [Dl + 2*KVl rows][row_bytes(D)]   wq, wk, wv row shards stacked (bytes unchanged from the file)
//   wo    [D rows][row_bytes(Dl)]            K-shard (this rank's heads' input columns)
//   w1,w3 [Hl rows][row_bytes(D)], w2 [D rows][row_bytes(Hl)] (K-shard), output [Vl rows][row_bytes(D)]
//   tok_embd full, norms full (f32)
//   K/V caches f32 [L][max_seq][KVl], RoPE table f32x2 [max_seq][hd/2]
// Step (graph): embed -> L x { qkv GEMV (rmsnorm+quant prologue, RoPE + cache-store epilogue),
//   attention, wo GEMV (+residual), [all-reduce], w1/w3 GEMV (rmsnorm prologue, SwiGLU epilogue),
//   w2 GEMV (+residual), [all-reduce] } -> output GEMV (final rmsnorm) [all-gather] -> argmax/advance.
// Every kernel is launched with programmatic dependent launch so a GEMV's weight prefetch starts while
// the previous kernel drains.  Residual + all-reduce: rank 0 adds its partial product into x, other
// ranks store theirs, then one in-place sum all-reduce of D floats gives x + sum of partials everywhere.
#include <nccl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <thread>
#include <vector>

#include "attention.cuh"
#include "decode.cuh"
#include "elementwise.cuh"
#include "gemv.cuh"
#include "matmul.cuh"
#include "matmul_tc.cuh"
#include "prefill.cuh"
#include "synth.cuh"

using namespace qmc;

namespace {
struct Layer {
    float *attn_norm = nullptr, *ffn_norm = nullptr;
    uint8_t *wqkv = nullptr, *wo = nullptr, *w1 = nullptr, *w3 = nullptr, *w2 = nullptr;
    uint8_t *sqkv = nullptr, *swo = nullptr, *s13 = nullptr, *sw2 = nullptr;  // split-row copies (persistent path)
    // whole-row split copies for the tensor-core prefill: the same buffers as above, or, for a matrix
    // split along K, a second copy with whole rows
    uint8_t *pqkv = nullptr, *pwo = nullptr, *p13 = nullptr, *pw2 = nullptr;
    bool pstale = true;  // the whole-row copies of K-split matrices predate the decode copies' last refill
    int dt[12];          // dtype per uploaded kind (indices QMC_T_*), -1 = missing
    unsigned dirty = 0;  // kinds (bit QMC_T_*) uploaded since the split-row copies were last refilled
    // blocks per K-chunk of the split copies (>= the row's blocks: whole rows), chosen with the ring plan
    int kb_qkv = 1 << 30, kb_wo = 1 << 30, kb_13 = 1 << 30, kb_w2 = 1 << 30;
};
}  // namespace

struct qmc_model {
    qmc_config cfg;
    int dev = 0, rank = 0, tp = 1;
    ncclComm_t comm = nullptr;
    cudaStream_t stream = nullptr;
    int D, H, L, NH, NKV, V, S, hd, KVD;  // full model
    int NHl, NKVl, Dl, KVl, Hl, Vl;       // this rank
    int dt_tok = -1, dt_out = -1;
    uint8_t *tok = nullptr, *out = nullptr;
    float *norm = nullptr;
    std::vector<Layer> layers;
    std::vector<void *> allocs;
    float *x = nullptr, *xb = nullptr, *q = nullptr, *h = nullptr, *logits_l = nullptr, *logits = nullptr;
    void *kc = nullptr, *vc = nullptr;  // [L][max_seq][KVl] of float, or of __half when kv16
    int kv16 = 0;
    float *attn_part = nullptr;
    float2 *rope = nullptr;
    int *state = nullptr;  // [0] token  [1] pos  [2] step  [3] prompt length  [8] sampled token
    int *forced = nullptr, *gen = nullptr, *attn_cnt = nullptr;
    unsigned long long *amax = nullptr;  // [0] argmax key, [1] low 32 bits: CTA ticket (fused output argmax)
    int *h_state = nullptr;
    float *h_logits = nullptr;
    AttnPlan ap;
    cudaGraphExec_t graph = nullptr;
    bool have_tok = false, have_norm = false, have_out = false;
    // persistent decode path (tp 1, quantized matrices): split-row weights, phase list, barrier state
    bool mega = false, mega_checked = false, repacked = false, out_dirty = true;
    bool chunked = false;     // some matrix is split along K: its copy is not the tensor-core prefill's layout
    int kb_out = 1 << 30;
    DecodePlan plan;
    std::vector<DecodePhase> phases;
    DecodePhase *d_phases = nullptr;
    uint8_t *sout = nullptr;
    unsigned *gbar = nullptr;
    float *apart = nullptr;
    int maxseg = 1, gsplit = 1;
    // batched prompt forward: row buffers for up to pf_cap tokens (allocated on first use, grown on demand)
    int pf_cap = 0;
    int *pf_tok = nullptr;
    float *pf_x = nullptr, *pf_xn = nullptr, *pf_qkv = nullptr, *pf_att = nullptr, *pf_c = nullptr, *pf_h = nullptr,
          *pf_h3 = nullptr, *pf_ad = nullptr, *pf_adT = nullptr;
    int8_t *pf_aq = nullptr;
    // weight upload: pinned staging buffers (allocated on the first large upload)
    uint8_t *stage[2] = {nullptr, nullptr};
    // tensor parallelism on the persistent path: this rank's exchange block and every rank's, mapped
    uint8_t *xblk = nullptr;
    uint8_t *xpeer[kDecodeMaxTp] = {};
    int64_t xlog_off = 0;
    cudaEvent_t stage_ev[2] = {nullptr, nullptr};
};

namespace {

int64_t rbytes(int dt, int64_t cols) { return row_bytes(dt, cols); }

// layer l's slice of a KV cache
size_t kv_layer_bytes(const qmc_model *m) { return (size_t)m->S * m->KVl * (m->kv16 ? 2 : 4); }
void *kv_layer(const qmc_model *m, void *base, int l) { return (uint8_t *)base + (size_t)l * kv_layer_bytes(m); }

int dalloc(qmc_model *m, void **p, size_t bytes) {
    cudaError_t e = cudaMalloc(p, bytes + 256);  // slack: 16-byte line reads past a tensor's end stay inside
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(model)");
    m->allocs.push_back(*p);
    return QMC_OK;
}

// release one model buffer (no kernel may still use it: the caller synchronised the stream)
template <typename T>
int dfree(qmc_model *m, T **p) {
    if (!*p) return QMC_OK;
    for (size_t i = 0; i < m->allocs.size(); i++)
        if (m->allocs[i] == (void *)*p) {
            m->allocs.erase(m->allocs.begin() + (long)i);
            break;
        }
    QMC_CUDA(cudaFree((void *)*p));
    *p = nullptr;
    return QMC_OK;
}

bool valid_dt(int dt) { return dt == QMC_F32 || dt == QMC_Q8_0 || dt == QMC_Q4_0; }

// shard plan of one tensor kind on this rank: rows [r0, r0+nr) and columns [c0, c0+nc) of the full
// tensor, plus the destination and the row offset inside a stacked buffer
struct Shard {
    int64_t rows, cols, r0, nr, c0, nc;
};

Shard shard_of(const qmc_model *m, int kind) {
    const int64_t D = m->D, H = m->H, KV = m->KVD, V = m->V;
    Shard s{};
    auto rowsplit = [&](int64_t R, int64_t C, int64_t Rl) { s = Shard{R, C, m->rank * Rl, Rl, 0, C}; };
    auto colsplit = [&](int64_t R, int64_t C, int64_t Cl) { s = Shard{R, C, 0, R, m->rank * Cl, Cl}; };
    switch (kind) {
    case QMC_T_TOK_EMBD: s = Shard{V, D, 0, V, 0, D}; break;
    case QMC_T_NORM: case QMC_T_ATTN_NORM: case QMC_T_FFN_NORM: s = Shard{D, 0, 0, D, 0, 0}; break;
    case QMC_T_OUTPUT: rowsplit(V, D, m->Vl); break;
    case QMC_T_WQ: rowsplit(D, D, m->Dl); break;
    case QMC_T_WK: case QMC_T_WV: rowsplit(KV, D, m->KVl); break;
    case QMC_T_WO: colsplit(D, D, m->Dl); break;
    case QMC_T_W1: case QMC_T_W3: rowsplit(H, D, m->Hl); break;
    case QMC_T_W2: colsplit(D, H, m->Hl); break;
    }
    return s;
}

// destination buffer for (kind, layer, dtype), allocating it on first use
int dest_of(qmc_model *m, int kind, int layer, int dt, uint8_t **dst) {
    Layer *Ly = (layer >= 0 && layer < m->L) ? &m->layers[layer] : nullptr;
    const Shard s = shard_of(m, kind);
    int rc = QMC_OK;
    auto need = [&](uint8_t **buf, size_t bytes) -> int {
        if (!*buf) rc = dalloc(m, (void **)buf, bytes);
        return rc;
    };
    switch (kind) {
    case QMC_T_TOK_EMBD:
        if (m->tok && m->dt_tok != dt) return set_error(QMC_EINVAL, "tok_embd dtype changed");
        m->dt_tok = dt;
        if (need(&m->tok, (size_t)(s.nr * rbytes(dt, s.nc)))) return rc;
        *dst = m->tok;
        return QMC_OK;
    case QMC_T_OUTPUT:
        if (m->out && m->dt_out != dt) return set_error(QMC_EINVAL, "output dtype changed");
        m->dt_out = dt;
        if (need(&m->out, (size_t)(s.nr * rbytes(dt, s.nc)))) return rc;
        *dst = m->out;
        return QMC_OK;
    case QMC_T_NORM:
        if (need((uint8_t **)&m->norm, (size_t)m->D * 4)) return rc;
        *dst = (uint8_t *)m->norm;
        return QMC_OK;
    default: break;
    }
    if (!Ly) return set_error(QMC_EINVAL, "layer %d out of range", layer);
    // grouped tensors must share a dtype (they are streamed by one kernel)
    auto group_dt = [&](std::initializer_list<int> kinds) -> int {
        for (int k : kinds)
            if (Ly->dt[k] >= 0 && Ly->dt[k] != dt) return set_error(QMC_EINVAL, "layer %d: mixed dtypes in a fused group", layer);
        return QMC_OK;
    };
    switch (kind) {
    case QMC_T_ATTN_NORM:
        if (need((uint8_t **)&Ly->attn_norm, (size_t)m->D * 4)) return rc;
        *dst = (uint8_t *)Ly->attn_norm;
        return QMC_OK;
    case QMC_T_FFN_NORM:
        if (need((uint8_t **)&Ly->ffn_norm, (size_t)m->D * 4)) return rc;
        *dst = (uint8_t *)Ly->ffn_norm;
        return QMC_OK;
    case QMC_T_WQ: case QMC_T_WK: case QMC_T_WV: {
        if ((rc = group_dt({QMC_T_WQ, QMC_T_WK, QMC_T_WV}))) return rc;
        const int64_t rb = rbytes(dt, m->D);
        if (need(&Ly->wqkv, (size_t)((m->Dl + 2 * m->KVl) * rb))) return rc;
        const int64_t off = kind == QMC_T_WQ ? 0 : (kind == QMC_T_WK ? m->Dl : m->Dl + m->KVl);
        *dst = Ly->wqkv + off * rb;
        return QMC_OK;
    }
    case QMC_T_WO:
        if (need(&Ly->wo, (size_t)(m->D * rbytes(dt, m->Dl)))) return rc;
        *dst = Ly->wo;
        return QMC_OK;
    case QMC_T_W1: case QMC_T_W3:
        if ((rc = group_dt({QMC_T_W1, QMC_T_W3}))) return rc;
        if (need(kind == QMC_T_W1 ? &Ly->w1 : &Ly->w3, (size_t)(m->Hl * rbytes(dt, m->D)))) return rc;
        *dst = kind == QMC_T_W1 ? Ly->w1 : Ly->w3;
        return QMC_OK;
    case QMC_T_W2:
        if (need(&Ly->w2, (size_t)(m->D * rbytes(dt, m->Hl)))) return rc;
        *dst = Ly->w2;
        return QMC_OK;
    }
    return set_error(QMC_EINVAL, "unknown tensor kind %d", kind);
}

void mark(qmc_model *m, int kind, int layer, int dt) {
    if (kind == QMC_T_TOK_EMBD) m->have_tok = true;
    else if (kind == QMC_T_NORM) m->have_norm = true;
    else if (kind == QMC_T_OUTPUT) m->have_out = true, m->out_dirty = true;
    else m->layers[layer].dt[kind] = dt, m->layers[layer].dirty |= 1u << kind;
}

bool complete(const qmc_model *m) {
    if (!m->have_tok || !m->have_norm || !m->have_out) return false;
    for (const Layer &l : m->layers)
        for (int k = QMC_T_ATTN_NORM; k <= QMC_T_W3; k++)
            if (l.dt[k] < 0) return false;
    return true;
}

#define RC(x)                                                                                                          \
    do {                                                                                                               \
        int rc_ = (x);                                                                                                 \
        if (rc_) return rc_;                                                                                           \
    } while (0)

int nccl_check(ncclResult_t r, const char *what) {
    if (r == ncclSuccess) return QMC_OK;
    return set_error(QMC_ENCCL, "%s: %s", what, ncclGetErrorString(r));
}

// ---------------------------------------------------------------- persistent decode path
// Eligible when one GPU holds the model, every matrix is Q8_0/Q4_0 and the ring plan fits shared memory.
int setup_exchange(qmc_model *m);

bool decode_eligible(qmc_model *m, DevCtx *c) {
    if (m->tp > kDecodeMaxTp || m->hd > 128) return false;
    auto q = [](int dt) { return dt == QMC_Q8_0 || dt == QMC_Q4_0; };
    if (!q(m->dt_out)) return false;
    int nbmax = (int)nblocks(m->D);
    for (const Layer &l : m->layers)
        if (!q(l.dt[QMC_T_WQ]) || !q(l.dt[QMC_T_WO]) || !q(l.dt[QMC_T_W1]) || !q(l.dt[QMC_T_W2])) return false;
    nbmax = std::max(nbmax, (int)std::max(nblocks(m->Dl), nblocks(m->Hl)));
    const int group = m->NH / m->NKV, grid = c->num_sms;
    // Every matrix streams through ring slots: a unit (row / row pair) longer than a slot is split along K
    // into chunks of the most blocks that fit.  The chunk partial sums need shared
    // memory, which shrinks the slots: iterate until the chunking no longer grows.
    struct Mat { int dt; int64_t K; int urows; int64_t units; int *kb; };
    std::vector<Mat> mats;
    for (Layer &l : m->layers) {
        mats.push_back({l.dt[QMC_T_WQ], m->D, 2, (m->Dl + 2 * m->KVl) / 2, &l.kb_qkv});
        mats.push_back({l.dt[QMC_T_WO], m->Dl, 1, m->D, &l.kb_wo});
        mats.push_back({l.dt[QMC_T_W1], m->D, 2, m->Hl, &l.kb_13});
        mats.push_back({l.dt[QMC_T_W2], m->Hl, 1, m->D, &l.kb_w2});
    }
    mats.push_back({m->dt_out, m->D, 1, m->Vl, &m->kb_out});
    // whole rows when the largest unit fits a ring with at least two slots per consumer warp (33 or 22
    // slots): with one slot per warp (11) a warp's next stage cannot be in flight while it computes, and
    // K-chunks cut to the 22-slot ring decode faster (Llama-7B-shaped Q8_0: 407.9 against 386.1 tok/s)
    int64_t umax = 0;
    for (const Mat &x : mats) umax = std::max(umax, (int64_t)x.urows * split_row_bytes(x.dt, x.K));
    m->chunked = false;
    if (plan_decode(umax, nbmax, m->hd, group, c->max_smem_optin, &m->plan) && m->plan.nslots >= 2 * kDecodeWarps)
        return m->tp == 1 || setup_exchange(m) == QMC_OK;
    int64_t part = 0, stage_max = 0;
    for (int it = 0; it < 4; it++) {  // otherwise split every unit longer than a slot of the 22-slot ring
        const int64_t slot = decode_slot_bytes(nbmax, m->hd, group, c->max_smem_optin, part);
        int64_t need = 0;
        stage_max = 0;
        m->chunked = false;
        for (const Mat &x : mats) {
            const int64_t nb = nblocks(x.K);
            int64_t kb = nb;
            if ((int64_t)x.urows * split_row_bytes(x.dt, x.K) > slot) {
                kb = 0;
                while (kb + 1 < nb && (int64_t)x.urows * chunk_row_bytes(x.dt, kb + 1) <= slot) kb++;
                if (kb < 1) return false;
                m->chunked = true;
                const int64_t C = (nb + kb - 1) / kb;
                need = std::max(need, (x.units + grid - 1) / grid * C * x.urows * 4);
            }
            *x.kb = (int)kb;
            stage_max = std::max(stage_max, (int64_t)x.urows * chunk_row_bytes(x.dt, kb));
        }
        if (need <= part) break;
        part = need;
    }
    if (!plan_decode(stage_max, nbmax, m->hd, group, c->max_smem_optin, &m->plan, part)) return false;
    // tensor parallelism: every rank maps every rank's exchange block (CUDA IPC over NVLink); where that is
    // not possible the model keeps the per-operation graph with NCCL all-reduces.  Every rank takes the
    // same collective steps here, so the outcome is agreed before anyone returns.
    return m->tp == 1 || setup_exchange(m) == QMC_OK;
}

// The exchange block of this rank (zeroed: tag 0 means empty), its IPC handle all-gathered over the
// model's NCCL communicator, and every peer's block opened.  All ranks then agree (NCCL min) on whether
// every rank succeeded.
int setup_exchange(qmc_model *m) {
    const size_t bytes = (size_t)kXchSync + (size_t)16 * m->tp * m->D + (size_t)4 * m->V;
    m->xlog_off = (int64_t)kXchSync + (int64_t)16 * m->tp * m->D;
    int ok = 1;
    cudaIpcMemHandle_t h{};
    if (dalloc(m, (void **)&m->xblk, bytes) != QMC_OK || cudaMemset(m->xblk, 0, bytes + 256) != cudaSuccess ||
        cudaIpcGetMemHandle(&h, m->xblk) != cudaSuccess)
        ok = 0;
    cudaGetLastError();
    char *dh = nullptr;
    int *dok = nullptr;
    RC(dalloc(m, (void **)&dh, (size_t)64 * m->tp));
    RC(dalloc(m, (void **)&dok, 4));
    QMC_CUDA(cudaMemcpy(dh + 64 * m->rank, &h, 64, cudaMemcpyHostToDevice));
    QMC_CUDA(cudaMemcpy(dok, &ok, 4, cudaMemcpyHostToDevice));
    RC(nccl_check(ncclAllGather(dh + 64 * m->rank, dh, 64, ncclChar, m->comm, m->stream), "all-gather(ipc handles)"));
    RC(nccl_check(ncclAllReduce(dok, dok, 1, ncclInt, ncclMin, m->comm, m->stream), "all-reduce(ipc ok)"));
    QMC_CUDA(cudaStreamSynchronize(m->stream));
    std::vector<char> hh((size_t)64 * m->tp);
    QMC_CUDA(cudaMemcpy(hh.data(), dh, hh.size(), cudaMemcpyDeviceToHost));
    QMC_CUDA(cudaMemcpy(&ok, dok, 4, cudaMemcpyDeviceToHost));
    for (int r = 0; r < m->tp && ok; r++) {
        if (r == m->rank) {
            m->xpeer[r] = m->xblk;
            continue;
        }
        cudaIpcMemHandle_t ph;
        memcpy(&ph, hh.data() + 64 * r, 64);
        void *ptr = nullptr;
        if (cudaIpcOpenMemHandle(&ptr, ph, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            ok = 0;
            break;
        }
        m->xpeer[r] = (uint8_t *)ptr;
    }
    QMC_CUDA(cudaMemcpy(dok, &ok, 4, cudaMemcpyHostToDevice));
    RC(nccl_check(ncclAllReduce(dok, dok, 1, ncclInt, ncclMin, m->comm, m->stream), "all-reduce(ipc open)"));
    QMC_CUDA(cudaStreamSynchronize(m->stream));
    QMC_CUDA(cudaMemcpy(&ok, dok, 4, cudaMemcpyDeviceToHost));
    if (!ok) {
        for (int r = 0; r < m->tp; r++)
            if (m->xpeer[r] && r != m->rank) cudaIpcCloseMemHandle(m->xpeer[r]);
        for (int r = 0; r < m->tp; r++) m->xpeer[r] = nullptr;
        return set_error(QMC_ECUDA, "exchange blocks could not be mapped on every rank");
    }
    m->logits = (float *)(m->xblk + m->xlog_off);  // every rank's shard lands in every rank's logits
    return QMC_OK;
}

// split-row copies of every matrix (allocated once); FFN rows interleaved w1[0], w3[0], w1[1], ... so one
// copy streams both rows of a SwiGLU unit; rows longer than a ring slot split along K (decode.cuh).  Only
// the kinds uploaded since the last refill are repacked, layer by layer, and each layer's file-layout
// copies are released right after: the persistent path reads only the split-row copies (and the
// tensor-core prefill the same), so the model holds its weights once.  A later upload of one tensor
// allocates its file-layout buffer again, and only its rows are repacked.  A matrix split along K for
// decode gets a whole-row copy for the tensor-core prefill only when a batched prompt forward first
// runs (prefill_copies), and the output matrix keeps its file-layout copy (the batched prompt forward's
// final GEMV reads it).
int repack_weights(qmc_model *m) {
    cudaStream_t s = m->stream;
    for (Layer &l : m->layers) {
        const int dq = l.dt[QMC_T_WQ], dw = l.dt[QMC_T_WO], d1 = l.dt[QMC_T_W1], d2 = l.dt[QMC_T_W2];
        const int64_t nq = m->Dl + 2 * m->KVl, aq = rbytes(dq, m->D);
        const int64_t uq = chunked_unit_bytes(dq, m->D, l.kb_qkv, 2), uo = chunked_unit_bytes(dw, m->Dl, l.kb_wo, 1),
                      u13 = chunked_unit_bytes(d1, m->D, l.kb_13, 2), u2 = chunked_unit_bytes(d2, m->Hl, l.kb_w2, 1);
        if (!l.sqkv && (dalloc(m, (void **)&l.sqkv, (size_t)(nq / 2 * uq)) || dalloc(m, (void **)&l.swo, (size_t)(m->D * uo)) ||
                        dalloc(m, (void **)&l.s13, (size_t)(m->Hl * u13)) || dalloc(m, (void **)&l.sw2, (size_t)(m->D * u2))))
            return QMC_ENOMEM;

        const unsigned d = l.dirty;
        if (!d) continue;
        // wq | wk | wv row ranges of the stacked matrix (pairs of consecutive rows are units)
        const int64_t q0[3] = {0, m->Dl, m->Dl + m->KVl}, qn[3] = {m->Dl, m->KVl, m->KVl};
        const int qk[3] = {QMC_T_WQ, QMC_T_WK, QMC_T_WV};
        for (int j = 0; j < 3; j++)
            if (d & (1u << qk[j]))
                RC(launch_repack_chunked(dq, l.wqkv + q0[j] * aq, q0[j], qn[j], m->D, l.kb_qkv, 2, 2, 0, l.sqkv, s));
        if (d & (1u << QMC_T_WO)) RC(launch_repack_chunked(dw, l.wo, 0, m->D, m->Dl, l.kb_wo, 1, 1, 0, l.swo, s));
        if (d & (1u << QMC_T_W1)) RC(launch_repack_chunked(d1, l.w1, 0, m->Hl, m->D, l.kb_13, 2, 1, 0, l.s13, s));
        if (d & (1u << QMC_T_W3)) RC(launch_repack_chunked(d1, l.w3, 0, m->Hl, m->D, l.kb_13, 2, 1, 1, l.s13, s));
        if (d & (1u << QMC_T_W2)) RC(launch_repack_chunked(d2, l.w2, 0, m->D, m->Hl, l.kb_w2, 1, 1, 0, l.sw2, s));
        l.pstale = true;
        QMC_CUDA(cudaStreamSynchronize(s));
        RC(dfree(m, &l.wqkv));
        RC(dfree(m, &l.wo));
        RC(dfree(m, &l.w1));
        RC(dfree(m, &l.w3));
        RC(dfree(m, &l.w2));
        l.dirty = 0;
    }
    const int64_t uout = chunked_unit_bytes(m->dt_out, m->D, m->kb_out, 1);
    if (!m->sout && dalloc(m, (void **)&m->sout, (size_t)(m->Vl * uout))) return QMC_ENOMEM;
    if (m->out_dirty) RC(launch_repack_chunked(m->dt_out, m->out, 0, m->Vl, m->D, m->kb_out, 1, 1, 0, m->sout, s));
    m->out_dirty = false;
    QMC_CUDA(cudaStreamSynchronize(s));
    m->repacked = true;
    return QMC_OK;
}

// The whole-row split copies the tensor-core prefill reads: a matrix decoded from whole rows shares its
// decode copy; a K-split one gets a second copy, relaid out on the device from its chunks, allocated at
// the first batched prompt forward and refreshed after any upload (a decode-only model never holds it).
int prefill_copies(qmc_model *m) {
    cudaStream_t s = m->stream;
    const int big = 1 << 30;
    for (Layer &l : m->layers) {
        const int dq = l.dt[QMC_T_WQ], dw = l.dt[QMC_T_WO], d1 = l.dt[QMC_T_W1], d2 = l.dt[QMC_T_W2];
        const int64_t nq = m->Dl + 2 * m->KVl;
        const bool sq = l.kb_qkv < nblocks(m->D), so = l.kb_wo < nblocks(m->Dl), s1 = l.kb_13 < nblocks(m->D),
                   s2 = l.kb_w2 < nblocks(m->Hl);
        if (!sq) l.pqkv = l.sqkv;
        if (!so) l.pwo = l.swo;
        if (!s1) l.p13 = l.s13;
        if (!s2) l.pw2 = l.sw2;
        if (!l.pstale) continue;
        if (sq && !l.pqkv) RC(dalloc(m, (void **)&l.pqkv, (size_t)(nq * split_row_bytes(dq, m->D))));
        if (so && !l.pwo) RC(dalloc(m, (void **)&l.pwo, (size_t)(m->D * split_row_bytes(dw, m->Dl))));
        if (s1 && !l.p13) RC(dalloc(m, (void **)&l.p13, (size_t)(2 * m->Hl * split_row_bytes(d1, m->D))));
        if (s2 && !l.pw2) RC(dalloc(m, (void **)&l.pw2, (size_t)(m->D * split_row_bytes(d2, m->Hl))));
        if (sq) RC(launch_relayout_chunked(dq, l.sqkv, l.kb_qkv, l.pqkv, big, nq, m->D, 2, 2, 0, s));
        if (so) RC(launch_relayout_chunked(dw, l.swo, l.kb_wo, l.pwo, big, m->D, m->Dl, 1, 1, 0, s));
        if (s1) {
            RC(launch_relayout_chunked(d1, l.s13, l.kb_13, l.p13, big, m->Hl, m->D, 2, 1, 0, s));
            RC(launch_relayout_chunked(d1, l.s13, l.kb_13, l.p13, big, m->Hl, m->D, 2, 1, 1, s));
        }
        if (s2) RC(launch_relayout_chunked(d2, l.sw2, l.kb_w2, l.pw2, big, m->D, m->Hl, 1, 1, 0, s));
        l.pstale = false;
    }
    QMC_CUDA(cudaStreamSynchronize(s));
    return QMC_OK;
}

DecodePhase matrix_phase(const qmc_model *m, int grid, int kind, int dt, const uint8_t *W, int64_t units, int64_t K,
                         int urows, const float *in, const float *norm_w, float *out, int kb) {
    DecodePhase ph{};
    ph.xex = -1;
    ph.kb = (int)std::min<int64_t>(kb, nblocks(K));
    ph.C = (int)((nblocks(K) + ph.kb - 1) / ph.kb);
    ph.kind = kind;
    ph.dtype = dt;
    ph.W = W;
    ph.units = units;
    ph.K = (int)K;
    ph.nb = (int)nblocks(K);
    ph.urows = urows;
    ph.rbytes = (int)split_row_bytes(dt, K);
    ph.sbytes = (int)split_scale_bytes(K);
    // units per stage: the most a slot holds (more bytes in flight per warp) unless fewer evens out the
    // busiest warp's share of the busiest CTA's units by more than ~15 %
    const int64_t rmax = std::max<int64_t>(1, m->plan.slot_bytes / ((int64_t)urows * ph.rbytes));
    const int64_t per_cta = (units + grid - 1) / grid;
    auto load = [&](int64_t r) {  // units of the busiest warp
        const int64_t stages = (per_cta + r - 1) / r;
        return r * ((stages + m->plan.groups - 1) / m->plan.groups);
    };
    int64_t best = INT64_MAX;
    for (int64_t r = 1; r <= rmax; r++) best = std::min(best, load(r));
    for (int64_t r = rmax; r >= 1; r--)
        if (load(r) * 100 <= best * 115) {
            ph.R = (int)r;
            break;
        }
    if (ph.C > 1) ph.R = 1;  // a stage is one chunk of one unit
    ph.in = in;
    ph.norm_w = norm_w;
    ph.out = out;
    return ph;
}

int prepare_decode(qmc_model *m, DevCtx *c) {
    if (!m->mega_checked) {
        m->mega_checked = true;
        m->mega = decode_eligible(m, c);
        if (!m->mega) return QMC_OK;
        RC(repack_weights(m));  // allocates the split-row copies the phase list points at
        for (int l = 0; l < m->L; l++) {
            Layer &Ly = m->layers[l];
            void *kcl = kv_layer(m, m->kc, l), *vcl = kv_layer(m, m->vc, l);
            DecodePhase qkv = matrix_phase(m, c->num_sms, PH_QKV, Ly.dt[QMC_T_WQ], Ly.sqkv, (m->Dl + 2 * m->KVl) / 2, m->D, 2, m->x,
                                           Ly.attn_norm, nullptr, Ly.kb_qkv);
            qkv.embed = l == 0;
            qkv.kc = kcl, qkv.vc = vcl;
            DecodePhase at{};
            at.xex = -1;
            at.kind = PH_ATTN;
            at.kc = kcl, at.vc = vcl;
            m->phases.push_back(qkv);
            m->phases.push_back(at);
            DecodePhase wo = matrix_phase(m, c->num_sms, PH_WO, Ly.dt[QMC_T_WO], Ly.swo, m->D, m->Dl, 1, m->xb, nullptr, m->x, Ly.kb_wo);
            DecodePhase w2 = matrix_phase(m, c->num_sms, PH_W2, Ly.dt[QMC_T_W2], Ly.sw2, m->D, m->Hl, 1, m->h, nullptr, m->x, Ly.kb_w2);
            wo.xex = m->tp > 1 ? 2 * l : -1;  // tensor parallelism: partial rows, exchanged across the ranks
            w2.xex = m->tp > 1 ? 2 * l + 1 : -1;
            m->phases.push_back(wo);
            m->phases.push_back(matrix_phase(m, c->num_sms, PH_FFN, Ly.dt[QMC_T_W1], Ly.s13, m->Hl, m->D, 2, m->x, Ly.ffn_norm, m->h, Ly.kb_13));
            m->phases.push_back(w2);
        }
        m->phases.push_back(matrix_phase(m, c->num_sms, PH_OUT, m->dt_out, m->sout, m->Vl, m->D, 1, m->x, m->norm, m->logits, m->kb_out));
        const int group = m->NH / m->NKV;
        m->gsplit = (group + kDecodeHeadsPerUnit - 1) / kDecodeHeadsPerUnit;
        // at most kDecodeFastSegs segments per head: the wo prologue then merges them with every load in
        // flight (with few KV heads per GPU, e.g. under tensor parallelism, more would take its slow path)
        m->maxseg = std::max(1, std::min(kDecodeFastSegs, c->num_sms / (m->NKVl * m->gsplit)));
        const size_t units = (size_t)m->NKVl * m->gsplit;
        RC(dalloc(m, (void **)&m->d_phases, m->phases.size() * sizeof(DecodePhase)));
        RC(dalloc(m, (void **)&m->gbar, 64));
        RC(dalloc(m, (void **)&m->apart, units * m->maxseg * kDecodeHeadsPerUnit * (m->hd + kDecodePartHead) * 4));
        QMC_CUDA(cudaMemcpy(m->d_phases, m->phases.data(), m->phases.size() * sizeof(DecodePhase), cudaMemcpyHostToDevice));
        QMC_CUDA(cudaMemset(m->gbar, 0, 64));
        return QMC_OK;
    }
    if (m->mega && !m->repacked) RC(repack_weights(m));
    return QMC_OK;
}

int launch_decode_step(qmc_model *m, DevCtx *c) {
    DecodeParams p{};
    p.ph = m->d_phases;
    p.nph = (int)m->phases.size();
    p.D = m->D, p.Dq = m->Dl, p.KVl = m->KVl, p.hd = m->hd, p.nkv = m->NKVl, p.group = m->NH / m->NKV;
    p.gsplit = m->gsplit;
    p.eps = m->cfg.norm_eps;
    p.scale = 1.0f / sqrtf((float)m->hd);
    p.tok = m->tok;
    p.dt_tok = m->dt_tok;
    p.x = m->x, p.q = m->q, p.logits = m->logits;
    p.rope = m->rope;
    p.state = m->state, p.forced = m->forced, p.gen = m->gen, p.gen_cap = m->S;
    p.vocab = m->V;
    p.amax_key = m->amax;
    p.amax_ctr = (int *)(m->amax + 1);
    p.gbar = m->gbar;
    p.apart = m->apart, p.maxseg = m->maxseg;
    p.kv16 = m->kv16;
    p.err = c->err;
    p.nslots = m->plan.nslots, p.slot_bytes = m->plan.slot_bytes, p.off_part = m->plan.off_part;
    p.tp = m->tp, p.rank = m->rank, p.xph = 2 * m->L, p.xlog_off = m->xlog_off;
    for (int r = 0; r < kDecodeMaxTp; r++) p.peers.blk[r] = m->xpeer[r];
    p.off_bars = m->plan.off_bars, p.off_xq = m->plan.off_xq, p.off_xds = m->plan.off_xds, p.off_red = m->plan.off_red;
    return launch_decode(p, m->plan, c->num_sms, m->stream);
}

// after a device-side timeout the barrier words and tickets may be mid-count: clear them
int step_status(qmc_model *m) {
    const int rc = qmc_check_device_error();
    if (rc && m->mega) {
        cudaMemset(m->gbar, 0, 64);
        cudaMemset(m->amax, 0, 16);
    }
    return rc;
}

// per-token calls: the error word comes back with the step's own copies (one synchronisation); only a
// set word takes the slow path that reads, clears and resets
int enqueue_err_read(qmc_model *m) {
    DevCtx *c = ctx();
    if (!c) return QMC_ECUDA;
    QMC_CUDA(cudaMemcpyAsync(m->h_state + 15, c->err, 4, cudaMemcpyDeviceToHost, m->stream));
    return QMC_OK;
}
int step_status_read(qmc_model *m) { return m->h_state[15] ? step_status(m) : QMC_OK; }

// enqueue one decode step on m->stream (captured into the graph)
int enqueue_step(qmc_model *m) {
    cudaStream_t s = m->stream;
    DevCtx *c = ctx();
    if (m->mega) return launch_decode_step(m, c);
    const int *pos = m->state + 1;
    RC(launch_embed(m->dt_tok, m->tok, m->D, m->state, m->x, s, true));
    for (int l = 0; l < m->L; l++) {
        Layer &Ly = m->layers[l];
        void *kcl = kv_layer(m, m->kc, l), *vcl = kv_layer(m, m->vc, l);
        GemvArgs a;
        a.dtype = Ly.dt[QMC_T_WQ];
        a.W0 = Ly.wqkv;
        a.rows = m->Dl + 2 * m->KVl;
        a.K = m->D;
        a.x = m->x;
        a.norm_w = Ly.attn_norm;
        a.eps = m->cfg.norm_eps;
        a.epi = EPI_QKV;
        a.q = m->q;
        a.kcache = kcl;
        a.vcache = vcl;
        a.kv16 = m->kv16;
        a.Dq = m->Dl;
        a.KVl = m->KVl;
        a.hd = m->hd;
        a.rope = m->rope;
        a.pos = pos;
        a.err = c->err;
        RC(launch_gemv(a, s, true));
        RC(launch_attention(m->ap, m->q, kcl, vcl, m->kv16 != 0, m->xb, m->attn_part, m->attn_cnt, pos, m->NKVl, m->NH / m->NKV,
                            m->hd, m->KVl, s, true));
        GemvArgs o;
        o.dtype = Ly.dt[QMC_T_WO];
        o.W0 = Ly.wo;
        o.rows = m->D;
        o.K = m->Dl;
        o.x = m->xb;
        o.epi = m->rank == 0 ? EPI_ADD : EPI_STORE;
        o.y = m->x;
        o.err = c->err;
        RC(launch_gemv(o, s, true));
        if (m->tp > 1) RC(nccl_check(ncclAllReduce(m->x, m->x, m->D, ncclFloat, ncclSum, m->comm, s), "all-reduce(wo)"));
        GemvArgs f;
        f.dtype = Ly.dt[QMC_T_W1];
        f.W0 = Ly.w1;
        f.W1 = Ly.w3;
        f.rows = m->Hl;
        f.K = m->D;
        f.x = m->x;
        f.norm_w = Ly.ffn_norm;
        f.eps = m->cfg.norm_eps;
        f.epi = EPI_SWIGLU;
        f.y = m->h;
        f.err = c->err;
        RC(launch_gemv(f, s, true));
        GemvArgs d;
        d.dtype = Ly.dt[QMC_T_W2];
        d.W0 = Ly.w2;
        d.rows = m->D;
        d.K = m->Hl;
        d.x = m->h;
        d.epi = m->rank == 0 ? EPI_ADD : EPI_STORE;
        d.y = m->x;
        d.err = c->err;
        RC(launch_gemv(d, s, true));
        if (m->tp > 1) RC(nccl_check(ncclAllReduce(m->x, m->x, m->D, ncclFloat, ncclSum, m->comm, s), "all-reduce(w2)"));
    }
    GemvArgs g;
    g.dtype = m->dt_out;
    g.W0 = m->out;
    g.rows = m->Vl;
    g.K = m->D;
    g.x = m->x;
    g.norm_w = m->norm;
    g.eps = m->cfg.norm_eps;
    g.y = m->logits_l;
    g.err = c->err;
    const bool fused = m->tp == 1 && m->dt_out != QMC_F32;
    g.epi = fused ? EPI_LOGITS : EPI_STORE;
    if (fused) {  // greedy argmax + state advance in the output GEMV's last CTA
        g.amax_key = m->amax;
        g.amax_ctr = (int *)(m->amax + 1);
        g.state = m->state;
        g.forced = m->forced;
        g.gen = m->gen;
        g.gen_cap = m->S;
    }
    RC(launch_gemv(g, s, true));
    if (m->tp > 1)
        RC(nccl_check(ncclAllGather(m->logits_l, m->logits, m->Vl, ncclFloat, m->comm, s), "all-gather(logits)"));
    if (!fused)
        RC(launch_argmax(m->logits, m->V, m->state, s, true, m->state + 1, m->forced, m->state + 3, m->state + 2,
                         m->gen, m->S));
    return QMC_OK;
}

int build_graph(qmc_model *m) {
    if (m->graph) return m->mega && !m->repacked ? repack_weights(m) : QMC_OK;
    if (!complete(m)) return set_error(QMC_ESTATE, "model: not every tensor has been uploaded");
    RC(prepare_decode(m, ctx()));
    cudaGraph_t g = nullptr;
    QMC_CUDA(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    int rc = enqueue_step(m);
    cudaError_t e = cudaStreamEndCapture(m->stream, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
    e = cudaGraphInstantiate(&m->graph, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGraphInstantiate");
    return QMC_OK;
}

int check_dev(const qmc_model *m) {
    int d = -1;
    QMC_CUDA(cudaGetDevice(&d));
    if (d != m->dev) QMC_CUDA(cudaSetDevice(m->dev));
    return QMC_OK;
}

}  // namespace

extern "C" {

int qmc_nccl_unique_id(void *id128) {
    ncclUniqueId id;
    RC(nccl_check(ncclGetUniqueId(&id), "ncclGetUniqueId"));
    memcpy(id128, &id, sizeof id);
    return QMC_OK;
}

int qmc_model_create(const qmc_config *cfg, int tp_rank, int tp_size, const void *nccl_id, qmc_model **out) {
    if (!cfg || !out) return set_error(QMC_EINVAL, "model_create: null argument");
    *out = nullptr;
    DevCtx *c = ctx();
    if (!c) return QMC_ECUDA;
    const qmc_config &k = *cfg;
    if (k.dim <= 0 || k.hidden_dim <= 0 || k.n_layers <= 0 || k.n_heads <= 0 || k.n_kv_heads <= 0 || k.vocab_size <= 0 ||
        k.max_seq <= 0 || k.dim % k.n_heads || k.n_heads % k.n_kv_heads || (k.dim / k.n_heads) % 2)
        return set_error(QMC_EINVAL, "model_create: inconsistent configuration");
    if (tp_size < 1 || tp_rank < 0 || tp_rank >= tp_size) return set_error(QMC_EINVAL, "model_create: bad tp rank/size");
    const int hd = k.dim / k.n_heads;
    if (hd / 2 > kMaxRopeHalf) return set_error(QMC_EINVAL, "model_create: head_dim > 256");
    if (tp_size > 1 && (k.n_kv_heads % tp_size || k.vocab_size % tp_size || (k.dim / tp_size) % 32 ||
                        k.hidden_dim % (32 * tp_size)))
        return set_error(QMC_EINVAL, "model_create: shapes do not shard %d ways on 32-element block boundaries", tp_size);
    qmc_model *m = new qmc_model();
    m->cfg = k;
    m->rank = tp_rank;
    m->tp = tp_size;
    cudaGetDevice(&m->dev);
    m->stream = c->stream;
    m->D = k.dim, m->H = k.hidden_dim, m->L = k.n_layers, m->NH = k.n_heads, m->NKV = k.n_kv_heads;
    m->V = k.vocab_size, m->S = k.max_seq, m->hd = hd, m->KVD = hd * k.n_kv_heads;
    m->NHl = m->NH / tp_size, m->NKVl = m->NKV / tp_size, m->Dl = m->NHl * hd, m->KVl = m->NKVl * hd;
    m->Hl = m->H / tp_size, m->Vl = m->V / tp_size;
    m->layers.resize(m->L);
    for (Layer &l : m->layers)
        for (int i = 0; i < 12; i++) l.dt[i] = -1;
    int rc = QMC_OK;
    auto fail = [&](int r) {
        qmc_model_free(m);
        return r;
    };
    if (tp_size > 1) {
        if (!nccl_id) return fail(set_error(QMC_EINVAL, "model_create: tp_size > 1 needs an NCCL id"));
        ncclUniqueId id;
        memcpy(&id, nccl_id, sizeof id);
        if ((rc = nccl_check(ncclCommInitRank(&m->comm, tp_size, id, tp_rank), "ncclCommInitRank"))) return fail(rc);
    }
    m->ap = plan_attention(m->NKVl, m->NH / m->NKV, hd, m->S, c->num_sms);
    const size_t kvbytes = (size_t)m->L * m->S * m->KVl * 4;
    if ((rc = dalloc(m, (void **)&m->x, (size_t)m->D * 4)) || (rc = dalloc(m, (void **)&m->xb, (size_t)m->Dl * 4)) ||
        (rc = dalloc(m, (void **)&m->q, (size_t)m->Dl * 4)) || (rc = dalloc(m, (void **)&m->h, (size_t)m->Hl * 4)) ||
        (rc = dalloc(m, (void **)&m->logits, (size_t)m->V * 4)) || (rc = dalloc(m, (void **)&m->kc, kvbytes)) ||
        (rc = dalloc(m, (void **)&m->vc, kvbytes)) || (rc = dalloc(m, (void **)&m->attn_part, m->ap.part_floats * 4)) ||
        (rc = dalloc(m, (void **)&m->attn_cnt, (size_t)m->NKVl * 4)) ||
        (rc = dalloc(m, (void **)&m->rope, (size_t)m->S * (hd / 2) * 8)) || (rc = dalloc(m, (void **)&m->state, 64)) ||
        (rc = dalloc(m, (void **)&m->forced, (size_t)m->S * 4)) || (rc = dalloc(m, (void **)&m->gen, (size_t)m->S * 4)) ||
        (rc = dalloc(m, (void **)&m->amax, 16)))
        return fail(rc);
    m->logits_l = tp_size > 1 ? nullptr : m->logits;
    if (tp_size > 1 && (rc = dalloc(m, (void **)&m->logits_l, (size_t)m->Vl * 4))) return fail(rc);
    if (cudaMallocHost(&m->h_state, 64) != cudaSuccess || cudaMallocHost(&m->h_logits, (size_t)m->V * 4) != cudaSuccess)
        return fail(set_error(QMC_ENOMEM, "pinned host buffers"));
    // zeroed caches/counters, RoPE table from the reference's double expressions
    if (cudaMemsetAsync(m->kc, 0, kvbytes, m->stream) || cudaMemsetAsync(m->vc, 0, kvbytes, m->stream) ||
        cudaMemsetAsync(m->attn_cnt, 0, (size_t)m->NKVl * 4, m->stream) || cudaMemsetAsync(m->state, 0, 16, m->stream) ||
        cudaMemsetAsync(m->amax, 0, 16, m->stream))
        return fail(set_error(QMC_ECUDA, "memset"));
    std::vector<float> tab((size_t)m->S * hd);
    for (int p = 0; p < m->S; p++) rope_row_host(p, hd, k.rope_theta, tab.data() + (size_t)p * hd);
    if (cudaMemcpy(m->rope, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
        return fail(set_error(QMC_ECUDA, "rope table upload"));
    *out = m;
    return QMC_OK;
}

namespace {
constexpr int64_t kStageBytes = 32ll << 20;  // per pinned staging buffer
constexpr int kStageThreads = 8;             // host threads filling one chunk

// copy `rows` pieces of `piece` bytes, src_stride apart in host memory, to dst contiguously, returning
// once the device holds the data (the caller may release `src`):
//  - page-locked or registered source (qmc_host_register, e.g. a loader's mapped .qlm): DMA straight
//    from it;
//  - pageable contiguous source: the driver's copy (measured 19.8 GB/s for 3.8 GB of 7B weights,
//    against 15.1 through our own pinned staging, whose extra host memcpy is the bottleneck);
//  - pageable strided source (a column shard under tensor parallelism): chunks of the destination
//    gathered into two pinned buffers in turn by up to kStageThreads host threads while the previous
//    chunk's DMA runs.
int staged_upload(qmc_model *m, uint8_t *dst, const uint8_t *src, int64_t rows, int64_t piece, int64_t src_stride) {
    const int64_t total = rows * piece;
    cudaPointerAttributes pa{};
    const bool locked = cudaPointerGetAttributes(&pa, src) == cudaSuccess && pa.type == cudaMemoryTypeHost;
    cudaGetLastError();  // a pageable pointer may leave an error code behind on older drivers
    if (locked || total < (4ll << 20) || src_stride == piece) {
        if (src_stride == piece)
            QMC_CUDA(cudaMemcpyAsync(dst, src, (size_t)total, cudaMemcpyHostToDevice, m->stream));
        else
            QMC_CUDA(cudaMemcpy2DAsync(dst, (size_t)piece, src, (size_t)src_stride, (size_t)piece, (size_t)rows,
                                       cudaMemcpyHostToDevice, m->stream));
        QMC_CUDA(cudaStreamSynchronize(m->stream));
        return QMC_OK;
    }
    for (int b = 0; b < 2; b++) {
        if (!m->stage[b]) QMC_CUDA(cudaMallocHost(&m->stage[b], (size_t)kStageBytes));
        if (!m->stage_ev[b]) QMC_CUDA(cudaEventCreateWithFlags(&m->stage_ev[b], cudaEventDisableTiming));
    }
    auto fill = [&](uint8_t *buf, int64_t off, int64_t n) {  // destination bytes [off, off + n)
        auto part = [&](int64_t a, int64_t e) {
            while (a < e) {
                const int64_t r = a / piece, c = a % piece, len = std::min(e - a, piece - c);
                memcpy(buf + (a - off), src + r * src_stride + c, (size_t)len);
                a += len;
            }
        };
        const int nt = (int)std::min<int64_t>(kStageThreads, std::max<int64_t>(1, n >> 22));
        std::vector<std::thread> th;
        for (int i = 1; i < nt; i++) th.emplace_back(part, off + n * i / nt, off + n * (i + 1) / nt);
        part(off, off + n / nt);
        for (auto &x : th) x.join();
    };
    int b = 0;
    for (int64_t off = 0; off < total; off += kStageBytes, b ^= 1) {
        const int64_t n = std::min(kStageBytes, total - off);
        QMC_CUDA(cudaEventSynchronize(m->stage_ev[b]));  // the DMA that last read this buffer is done
        fill(m->stage[b], off, n);
        QMC_CUDA(cudaMemcpyAsync(dst + off, m->stage[b], (size_t)n, cudaMemcpyHostToDevice, m->stream));
        QMC_CUDA(cudaEventRecord(m->stage_ev[b], m->stream));
    }
    QMC_CUDA(cudaStreamSynchronize(m->stream));
    return QMC_OK;
}
}  // namespace

int qmc_model_upload(qmc_model *m, int kind, int layer, int dtype, int64_t rows, int64_t cols, const void *host) {
    if (!m || !host) return set_error(QMC_EINVAL, "upload: null argument");
    RC(check_dev(m));
    if (kind < 0 || kind > QMC_T_W3) return set_error(QMC_EINVAL, "upload: bad kind");
    if (!valid_dt(dtype)) return set_error(QMC_EINVAL, "upload: bad dtype %d", dtype);
    const bool vec = kind == QMC_T_NORM || kind == QMC_T_ATTN_NORM || kind == QMC_T_FFN_NORM;
    const Shard s = shard_of(m, kind);
    if (vec ? (dtype != QMC_F32 || rows != s.rows || cols != 0) : (rows != s.rows || cols != s.cols))
        return set_error(QMC_EINVAL, "upload: kind %d layer %d has shape %lldx%lld, expected %lldx%lld", kind, layer,
                         (long long)rows, (long long)cols, (long long)s.rows, (long long)s.cols);
    uint8_t *dst = nullptr;
    RC(dest_of(m, kind, layer, dtype, &dst));
    const uint8_t *src = (const uint8_t *)host;
    if (vec) {
        QMC_CUDA(cudaMemcpy(dst, src, (size_t)rows * 4, cudaMemcpyHostToDevice));
    } else if (s.c0 == 0 && s.nc == s.cols) {  // row shard: contiguous
        const int64_t rb = rbytes(dtype, cols);
        RC(staged_upload(m, dst, src + s.r0 * rb, 1, s.nr * rb, s.nr * rb));
    } else {  // column shard: each row's block range, gathered into the staging buffers
        const int64_t rb = rbytes(dtype, cols), rbl = rbytes(dtype, s.nc), off = rbytes(dtype, s.c0);
        RC(staged_upload(m, dst, src + s.r0 * rb + off, s.nr, rbl, rb));
    }
    mark(m, kind, layer, dtype);
    m->repacked = false;  // split-row copies are refilled before the next step
    return QMC_OK;
}

int qmc_model_synthesize(qmc_model *m, int dtype, uint64_t seed, double stdv) {
    if (!m) return set_error(QMC_EINVAL, "synthesize: null model");
    RC(check_dev(m));
    if (!valid_dt(dtype)) return set_error(QMC_EINVAL, "synthesize: bad dtype");
    const int L = m->L;
    for (int t = 0; t < 3 + 9 * L; t++) {
        int kind, layer = -1;
        if (t == 0) kind = QMC_T_TOK_EMBD;
        else if (t == 1 + 9 * L) kind = QMC_T_NORM;
        else if (t == 2 + 9 * L) kind = QMC_T_OUTPUT;
        else {
            static const int order[9] = {QMC_T_ATTN_NORM, QMC_T_WQ, QMC_T_WK, QMC_T_WV, QMC_T_WO,
                                         QMC_T_FFN_NORM,  QMC_T_W1, QMC_T_W2, QMC_T_W3};
            layer = (t - 1) / 9;
            kind = order[(t - 1) % 9];
        }
        const bool vec = kind == QMC_T_NORM || kind == QMC_T_ATTN_NORM || kind == QMC_T_FFN_NORM;
        const int dt = vec ? QMC_F32 : dtype;
        uint8_t *dst = nullptr;
        RC(dest_of(m, kind, layer, dt, &dst));
        const Shard s = shard_of(m, kind);
        if (vec) RC(launch_fill((float *)dst, m->D, 1.0f, m->stream));
        else RC(launch_synth(seed, (uint64_t)t, dt, s.cols, s.r0, s.nr, s.c0, s.nc, stdv, dst, m->stream));
        mark(m, kind, layer, dt);
    }
    m->repacked = false;
    QMC_CUDA(cudaStreamSynchronize(m->stream));
    return QMC_OK;
}

int qmc_model_forward(qmc_model *m, int32_t token, int32_t pos, float *logits_host, int32_t *next_token) {
    if (!m) return set_error(QMC_EINVAL, "forward: null model");
    if (token < 0 || token >= m->V || pos < 0 || pos >= m->S)
        return set_error(QMC_EINVAL, "forward: token %d / pos %d out of range", token, pos);
    RC(check_dev(m));
    RC(build_graph(m));
    m->h_state[0] = token, m->h_state[1] = pos, m->h_state[2] = 0, m->h_state[3] = 0;
    QMC_CUDA(cudaMemcpyAsync(m->state, m->h_state, 16, cudaMemcpyHostToDevice, m->stream));
    QMC_CUDA(cudaGraphLaunch(m->graph, m->stream));
    if (logits_host) QMC_CUDA(cudaMemcpyAsync(m->h_logits, m->logits, (size_t)m->V * 4, cudaMemcpyDeviceToHost, m->stream));
    QMC_CUDA(cudaMemcpyAsync(m->h_state + 4, m->state, 4, cudaMemcpyDeviceToHost, m->stream));
    RC(enqueue_err_read(m));
    QMC_CUDA(cudaStreamSynchronize(m->stream));
    RC(step_status_read(m));
    if (logits_host) memcpy(logits_host, m->h_logits, (size_t)m->V * 4);
    if (next_token) *next_token = m->h_state[4];
    return QMC_OK;
}

namespace {
// row buffers for T prompt tokens (old buffers stay allocated until the model is freed)
int prefill_buffers(qmc_model *m, int T) {
    if (T <= m->pf_cap) return QMC_OK;
    const int cap = std::min(m->S, std::max(T, ((T + 63) / 64) * 64));
    const int64_t wide = std::max<int64_t>(m->D, std::max<int64_t>(m->Hl, m->Dl + 2 * m->KVl));
    const int64_t nbk = nblocks(std::max<int64_t>(m->D, std::max<int64_t>(m->Hl, m->Dl)));
    int rc;
    if ((rc = dalloc(m, (void **)&m->pf_tok, (size_t)cap * 4)) || (rc = dalloc(m, (void **)&m->pf_x, (size_t)cap * m->D * 4)) ||
        (rc = dalloc(m, (void **)&m->pf_xn, (size_t)cap * m->D * 4)) ||
        (rc = dalloc(m, (void **)&m->pf_qkv, (size_t)cap * (m->Dl + 2 * m->KVl) * 4)) ||
        (rc = dalloc(m, (void **)&m->pf_att, (size_t)cap * m->Dl * 4)) || (rc = dalloc(m, (void **)&m->pf_c, (size_t)cap * wide * 4)) ||
        (rc = dalloc(m, (void **)&m->pf_h, (size_t)cap * m->Hl * 4)) || (rc = dalloc(m, (void **)&m->pf_h3, (size_t)cap * m->Hl * 4)) ||
        (rc = dalloc(m, (void **)&m->pf_aq, (size_t)cap * nbk * 32)) || (rc = dalloc(m, (void **)&m->pf_ad, (size_t)cap * nbk * 4)) ||
        (rc = dalloc(m, (void **)&m->pf_adT, (size_t)matmul_tc_scale_ld(cap) * nbk * 4)))
        return rc;
    m->pf_cap = cap;
    return QMC_OK;
}

// C[T][N] = A[T][K] . W^T: quantized W through per-row Q8_0 activations (row t = the matvec of A[t],
// src/ops.c:57-61), f32 W as the f32 contraction
int prefill_proj(qmc_model *m, int dt, const void *W, const float *A, int T, int64_t N, int64_t K, float *C) {
    if (dt == QMC_F32) return launch_gemm_f32(A, (const float *)W, C, T, N, K, m->stream);
    RC(launch_quantize_act(A, T, K, m->pf_aq, m->pf_ad, m->stream));
    return launch_matmul_q(dt, W, m->pf_aq, m->pf_ad, C, T, N, K, m->stream);
}
// the same on the tensor cores, from the split-row copy the decode kernel streams (C2: an interleaved
// w1/w3 matrix's rows 2i / 2i + 1 go to C / C2)
// A null: the activation blocks are already in pf_aq / pf_adT (rmsnorm fused with the quantization)
int prefill_proj_tc(qmc_model *m, int dt, const uint8_t *Ws, const float *A, int T, int64_t N, int64_t K, float *C,
                    float *C2) {
    if (A) RC(launch_quantize_act(A, T, K, m->pf_aq, m->pf_ad, m->stream, m->pf_adT, matmul_tc_scale_ld(T)));
    return launch_matmul_q_tc(dt, Ws, split_row_bytes(dt, K), m->pf_aq, m->pf_adT, C, C2, T, N, K, ctx()->err, m->stream);
}
// tensor parallelism: the wo / w2 contraction of a rank covers its column shard (its heads, its hidden
// rows), so pf_c holds a partial sum of every row; the ranks' partials are summed in place (NCCL) before
// the residual add, as the decode step adds them after its wo / w2 epilogues
int prefill_all_reduce(qmc_model *m, int T, const char *what) {
    if (m->tp == 1) return QMC_OK;
    return nccl_check(ncclAllReduce(m->pf_c, m->pf_c, (size_t)T * m->D, ncclFloat, ncclSum, m->comm, m->stream), what);
}
// x += add (when given), then rmsnorm(x) * w straight into the activation blocks of the next tensor-core
// contraction
int prefill_norm_quant(qmc_model *m, const float *add, const float *w, int T) {
    return launch_rmsnorm_quant_rows(m->pf_x, add, w, T, m->D, m->cfg.norm_eps, m->pf_aq, m->pf_ad, m->pf_adT,
                                     matmul_tc_scale_ld(T), m->stream);
}
}  // namespace

int qmc_model_prefill(qmc_model *m, const int32_t *tokens, int32_t n, int32_t pos0, float *logits_host,
                      int32_t *next_token) {
    if (!m || !tokens || n < 1 || pos0 < 0 || (int64_t)pos0 + n > m->S)
        return set_error(QMC_EINVAL, "prefill: bad arguments (n %d, pos0 %d, max_seq %d)", n, pos0, m ? m->S : 0);
    for (int i = 0; i < n; i++)
        if (tokens[i] < 0 || tokens[i] >= m->V) return set_error(QMC_EINVAL, "prefill: token %d out of range", tokens[i]);
    RC(check_dev(m));
    RC(prefill_buffers(m, n));
    cudaStream_t s = m->stream;
    DevCtx *c = ctx();
    if (!complete(m)) return set_error(QMC_ESTATE, "prefill: model incomplete");
    RC(prepare_decode(m, c));  // quantized models on the single-launch path: the split-row copies the tensor cores read
    const bool tc = m->mega;  // the tensor-core contraction reads the whole-row split copies
    if (tc) RC(prefill_copies(m));
    const int D = m->D, Dq = m->Dl, KVl = m->KVl, H = m->Hl, NQKV = Dq + 2 * KVl;
    const float eps = m->cfg.norm_eps;
    QMC_CUDA(cudaMemcpyAsync(m->pf_tok, tokens, (size_t)n * 4, cudaMemcpyHostToDevice, s));
    RC(launch_embed_rows(m->dt_tok, m->tok, D, m->pf_tok, n, m->pf_x, s));
    for (int l = 0; l < m->L; l++) {
        Layer &Ly = m->layers[l];
        void *kcl = kv_layer(m, m->kc, l), *vcl = kv_layer(m, m->vc, l);
        if (tc) {  // the previous layer's w2 residual is added here, fused with the norm
            RC(prefill_norm_quant(m, l > 0 ? m->pf_c : nullptr, Ly.attn_norm, n));
            RC(prefill_proj_tc(m, Ly.dt[QMC_T_WQ], Ly.pqkv, nullptr, n, NQKV, D, m->pf_qkv, nullptr));
        } else {
            RC(launch_rmsnorm_rows(m->pf_x, Ly.attn_norm, m->pf_xn, n, D, eps, s));
            RC(prefill_proj(m, Ly.dt[QMC_T_WQ], Ly.wqkv, m->pf_xn, n, NQKV, D, m->pf_qkv));
        }
        RC(launch_rope_kv_rows(m->pf_qkv, n, Dq, KVl, m->hd, pos0, m->rope, kcl, vcl, m->kv16 != 0, s));
        RC(launch_attn_prefill(m->pf_qkv, n, NQKV, m->NHl, m->NH / m->NKV, m->hd, KVl, pos0, 1.0f / sqrtf((float)m->hd), kcl,
                               vcl, m->kv16 != 0, m->pf_att, s));
        if (tc) RC(prefill_proj_tc(m, Ly.dt[QMC_T_WO], Ly.pwo, m->pf_att, n, D, Dq, m->pf_c, nullptr));
        else RC(prefill_proj(m, Ly.dt[QMC_T_WO], Ly.wo, m->pf_att, n, D, Dq, m->pf_c));
        RC(prefill_all_reduce(m, n, "all-reduce(prefill wo)"));
        if (tc) {  // wo residual fused with the norm
            RC(prefill_norm_quant(m, m->pf_c, Ly.ffn_norm, n));
            RC(prefill_proj_tc(m, Ly.dt[QMC_T_W1], Ly.p13, nullptr, n, 2 * (int64_t)H, D, m->pf_h, m->pf_h3));
        } else {
            RC(launch_add(m->pf_x, m->pf_c, (int64_t)n * D, s));
            RC(launch_rmsnorm_rows(m->pf_x, Ly.ffn_norm, m->pf_xn, n, D, eps, s));
            RC(prefill_proj(m, Ly.dt[QMC_T_W1], Ly.w1, m->pf_xn, n, H, D, m->pf_h));
            RC(prefill_proj(m, Ly.dt[QMC_T_W3], Ly.w3, m->pf_xn, n, H, D, m->pf_h3));
        }
        if (tc) {  // SwiGLU straight into the w2 contraction's activation blocks
            RC(launch_swiglu_quant_rows(m->pf_h, m->pf_h3, n, H, m->pf_aq, m->pf_ad, m->pf_adT, matmul_tc_scale_ld(n), s));
            RC(prefill_proj_tc(m, Ly.dt[QMC_T_W2], Ly.pw2, nullptr, n, D, H, m->pf_c, nullptr));
        } else {
            RC(launch_swiglu(m->pf_h, m->pf_h3, (int64_t)n * H, s));
            RC(prefill_proj(m, Ly.dt[QMC_T_W2], Ly.w2, m->pf_h, n, D, H, m->pf_c));
        }
        RC(prefill_all_reduce(m, n, "all-reduce(prefill w2)"));
        // w2 residual: on the tensor-core path the next layer's norm adds it, except after the last layer
        if (!tc || l == m->L - 1) RC(launch_add(m->pf_x, m->pf_c, (int64_t)n * D, s));
    }
    // logits of the last token: the output GEMV with the final rmsnorm fused, as a decode step's
    GemvArgs g;
    g.dtype = m->dt_out;
    g.W0 = m->out;
    g.rows = m->Vl;
    g.K = D;
    g.x = m->pf_x + (int64_t)(n - 1) * D;
    g.norm_w = m->norm;
    g.eps = eps;
    g.y = m->logits_l;
    g.epi = EPI_STORE;
    g.err = c->err;
    RC(launch_gemv(g, s, false));
    if (m->tp > 1)
        RC(nccl_check(ncclAllGather(m->logits_l, m->logits, m->Vl, ncclFloat, m->comm, s), "all-gather(prefill logits)"));
    QMC_CUDA(cudaMemcpyAsync(m->h_logits, m->logits, (size_t)m->V * 4, cudaMemcpyDeviceToHost, s));
    QMC_CUDA(cudaStreamSynchronize(s));
    RC(qmc_check_device_error());
    if (logits_host) memcpy(logits_host, m->h_logits, (size_t)m->V * 4);
    if (next_token) {  // first maximum; a NaN in slot 0 is never replaced (src/sampler.c:27-32)
        int bi = 0;
        float bv = m->h_logits[0];
        for (int i = 1; i < m->V; i++)
            if (m->h_logits[i] > bv) bv = m->h_logits[i], bi = i;
        *next_token = bi;
    }
    return QMC_OK;
}

int qmc_model_forward_sample(qmc_model *m, int32_t token, int32_t pos, qmc_sampler *s, int32_t *next_token) {
    if (!m || !s || !next_token) return set_error(QMC_EINVAL, "forward_sample: null argument");
    if (token < 0 || token >= m->V || pos < 0 || pos >= m->S)
        return set_error(QMC_EINVAL, "forward_sample: token %d / pos %d out of range", token, pos);
    RC(check_dev(m));
    RC(build_graph(m));
    m->h_state[0] = token, m->h_state[1] = pos, m->h_state[2] = 0, m->h_state[3] = 0;
    QMC_CUDA(cudaMemcpyAsync(m->state, m->h_state, 16, cudaMemcpyHostToDevice, m->stream));
    QMC_CUDA(cudaGraphLaunch(m->graph, m->stream));
    RC(qmc_sampler_enqueue(s, m->logits, m->state + 8, m->stream));
    QMC_CUDA(cudaMemcpyAsync(m->h_state + 4, m->state + 8, 4, cudaMemcpyDeviceToHost, m->stream));
    RC(enqueue_err_read(m));
    QMC_CUDA(cudaStreamSynchronize(m->stream));
    RC(step_status_read(m));
    *next_token = m->h_state[4];
    return QMC_OK;
}

int qmc_model_generate(qmc_model *m, const int32_t *prompt, int32_t n_prompt, int32_t n_gen, int32_t *out_tokens) {
    if (!m || !prompt || n_prompt < 1 || n_gen < 0 || (n_gen && !out_tokens))
        return set_error(QMC_EINVAL, "generate: bad arguments");
    if (n_prompt + n_gen - 1 > m->S) return set_error(QMC_EINVAL, "generate: %d positions exceed max_seq %d", n_prompt + n_gen - 1, m->S);
    for (int i = 0; i < n_prompt; i++)
        if (prompt[i] < 0 || prompt[i] >= m->V) return set_error(QMC_EINVAL, "generate: prompt token out of range");
    if (n_gen == 0) return QMC_OK;
    RC(check_dev(m));
    RC(build_graph(m));
    QMC_CUDA(cudaMemcpyAsync(m->forced, prompt, (size_t)n_prompt * 4, cudaMemcpyHostToDevice, m->stream));
    m->h_state[0] = prompt[0], m->h_state[1] = 0, m->h_state[2] = 0, m->h_state[3] = n_prompt;
    QMC_CUDA(cudaMemcpyAsync(m->state, m->h_state, 16, cudaMemcpyHostToDevice, m->stream));
    const int steps = n_prompt + n_gen - 1;
    for (int i = 0; i < steps; i++) QMC_CUDA(cudaGraphLaunch(m->graph, m->stream));
    QMC_CUDA(cudaMemcpyAsync(out_tokens, m->gen, (size_t)n_gen * 4, cudaMemcpyDeviceToHost, m->stream));
    QMC_CUDA(cudaStreamSynchronize(m->stream));
    return step_status(m);
}

int qmc_model_enqueue_decode(qmc_model *m, int32_t token, int32_t pos, int32_t steps) {
    if (!m || token >= m->V || steps < 0 || (token >= 0 && (pos < 0 || pos + steps > m->S)))
        return set_error(QMC_EINVAL, "enqueue_decode: bad arguments");
    RC(check_dev(m));
    RC(build_graph(m));
    if (token >= 0) {  // token < 0: continue from the device's current (token, pos)
        m->h_state[8] = token, m->h_state[9] = pos, m->h_state[10] = 0, m->h_state[11] = 1;
        QMC_CUDA(cudaMemcpyAsync(m->forced, m->h_state + 8, 4, cudaMemcpyHostToDevice, m->stream));
        QMC_CUDA(cudaMemcpyAsync(m->state, m->h_state + 8, 16, cudaMemcpyHostToDevice, m->stream));
    }
    for (int i = 0; i < steps; i++) QMC_CUDA(cudaGraphLaunch(m->graph, m->stream));
    return QMC_OK;
}

int qmc_model_state(qmc_model *m, int32_t *token, int32_t *pos) {
    if (!m) return set_error(QMC_EINVAL, "state: null model");
    RC(check_dev(m));
    QMC_CUDA(cudaMemcpyAsync(m->h_state + 12, m->state, 8, cudaMemcpyDeviceToHost, m->stream));
    QMC_CUDA(cudaStreamSynchronize(m->stream));
    if (token) *token = m->h_state[12];
    if (pos) *pos = m->h_state[13];
    return step_status(m);
}

int qmc_model_logits(qmc_model *m, const float **dev_logits) {
    if (!m || !dev_logits) return set_error(QMC_EINVAL, "logits: null argument");
    *dev_logits = m->logits;
    return QMC_OK;
}

int qmc_model_config(const qmc_model *m, qmc_config *cfg) {
    if (!m || !cfg) return set_error(QMC_EINVAL, "config: null argument");
    *cfg = m->cfg;
    return QMC_OK;
}

int qmc_model_step_bytes(const qmc_model *m, int32_t pos, double *bytes) {
    if (!m || !bytes) return set_error(QMC_EINVAL, "step_bytes: null argument");
    if (!complete(m)) return set_error(QMC_ESTATE, "step_bytes: model incomplete");
    double b = 0.0;
    for (const Layer &l : m->layers) {
        b += (double)(m->Dl + 2 * m->KVl) * rbytes(l.dt[QMC_T_WQ], m->D);
        b += (double)m->D * rbytes(l.dt[QMC_T_WO], m->Dl);
        b += 2.0 * m->Hl * rbytes(l.dt[QMC_T_W1], m->D);
        b += (double)m->D * rbytes(l.dt[QMC_T_W2], m->Hl);
        b += 2.0 * (pos + 1) * m->KVl * (m->kv16 ? 2.0 : 4.0);  // K and V reads
    }
    b += (double)m->Vl * rbytes(m->dt_out, m->D);
    *bytes = b;
    return QMC_OK;
}

int qmc_model_decode_info(const qmc_model *m, int32_t *launches, int32_t *persistent) {
    if (!m || !launches || !persistent) return set_error(QMC_EINVAL, "decode_info: null argument");
    *persistent = m->mega ? 1 : 0;
    if (!m->graph) *launches = 0;
    else if (m->mega) *launches = 1;
    else {  // embed + per layer {qkv, attention, wo, w1/w3, w2} + output (+ argmax when not fused)
        const bool fused = m->tp == 1 && m->dt_out != QMC_F32;
        *launches = 2 + 5 * m->L + (fused ? 0 : 1);
    }
    return QMC_OK;
}

int qmc_model_set_kv_dtype(qmc_model *m, int dtype) {
    if (!m) return set_error(QMC_EINVAL, "set_kv_dtype: null model");
    if (dtype != QMC_F32 && dtype != QMC_F16)
        return set_error(QMC_EINVAL, "set_kv_dtype: dtype %d is not QMC_F32 or QMC_F16", dtype);
    if (m->graph || m->mega_checked || m->pf_cap)
        return set_error(QMC_ESTATE, "set_kv_dtype: call it before the model's first step");
    RC(check_dev(m));
    if ((dtype == QMC_F16) == (m->kv16 != 0)) return QMC_OK;
    for (void **buf : {&m->kc, &m->vc}) {  // release the old caches (they hold no positions yet)
        for (size_t i = 0; i < m->allocs.size(); i++)
            if (m->allocs[i] == *buf) {
                m->allocs.erase(m->allocs.begin() + (long)i);
                break;
            }
        QMC_CUDA(cudaFree(*buf));
        *buf = nullptr;
    }
    m->kv16 = dtype == QMC_F16;
    const size_t bytes = (size_t)m->L * kv_layer_bytes(m);
    RC(dalloc(m, &m->kc, bytes));
    RC(dalloc(m, &m->vc, bytes));
    QMC_CUDA(cudaMemsetAsync(m->kc, 0, bytes, m->stream));
    QMC_CUDA(cudaMemsetAsync(m->vc, 0, bytes, m->stream));
    QMC_CUDA(cudaStreamSynchronize(m->stream));
    return QMC_OK;
}

int qmc_model_kv_dtype(const qmc_model *m, int *dtype) {
    if (!m || !dtype) return set_error(QMC_EINVAL, "kv_dtype: null argument");
    *dtype = m->kv16 ? QMC_F16 : QMC_F32;
    return QMC_OK;
}

int qmc_model_free(qmc_model *m) {
    if (!m) return QMC_OK;
    cudaSetDevice(m->dev);
    if (m->stream) cudaStreamSynchronize(m->stream);
    if (m->graph) cudaGraphExecDestroy(m->graph);
    for (int r = 0; r < kDecodeMaxTp; r++)
        if (m->xpeer[r] && m->xpeer[r] != m->xblk) cudaIpcCloseMemHandle(m->xpeer[r]);
    for (void *p : m->allocs) cudaFree(p);
    if (m->h_state) cudaFreeHost(m->h_state);
    if (m->h_logits) cudaFreeHost(m->h_logits);
    for (int b = 0; b < 2; b++) {
        if (m->stage[b]) cudaFreeHost(m->stage[b]);
        if (m->stage_ev[b]) cudaEventDestroy(m->stage_ev[b]);
    }
    if (m->comm) ncclCommDestroy(m->comm);
    delete m;
    return QMC_OK;
}

}  // extern "C"
