// Persistent whole-step decode kernel: one launch runs every matvec, attention and the greedy argmax
// of a decode step (tensor-parallel size 1, Q8_0 / Q4_0 weights in the split-row layout below).
#pragma once
#include "common.cuh"

namespace qmc {

// Split-row layout of a quantized matrix: each row is its ceil(K/32) fp16 block scales (padded to a
// 16-byte multiple) followed by the blocks' quant bytes (16 per Q4_0 block, 32 per Q8_0 block), so every
// row and every block payload is 16-byte aligned.  Same numbers as the file's AoS blocks, regrouped.
__host__ __device__ inline int64_t split_scale_bytes(int64_t K) { return ((nblocks(K) * 2 + 15) / 16) * 16; }
__host__ __device__ inline int64_t split_row_bytes(int dtype, int64_t K) {
    return split_scale_bytes(K) + nblocks(K) * (dtype == QMC_Q8_0 ? 32 : 16);
}
// AoS rows (file layout) -> split rows; row r goes to dst + r * dst_stride
int launch_repack_split(int dtype, const void *aos, int64_t rows, int64_t K, void *dst, int64_t dst_stride,
                        cudaStream_t s);

constexpr int kDecodeHeadsPerUnit = 4;  // query heads per attention work unit
constexpr int kDecodeWarps = 11;        // consumer warps per CTA (a ring has a multiple of this many slots)
constexpr int kDecodePartHead = 4;      // floats before acc[] in an attention segment partial
constexpr int kDecodeFastSegs = 4;      // position segments per head the wo prologue merges with all loads in flight

enum DecodePhaseKind : int { PH_QKV = 0, PH_ATTN = 1, PH_WO = 2, PH_FFN = 3, PH_W2 = 4, PH_OUT = 5 };

struct DecodePhase {
    int kind;             // DecodePhaseKind
    int dtype;            // weights: QMC_Q8_0 / QMC_Q4_0
    const uint8_t *W;     // split-row matrix; QKV rows q|k|v, FFN rows w1[0], w3[0], w1[1], ...
    int64_t units;        // units: rows (WO, W2, OUT) or row pairs (QKV RoPE pairs, FFN w1/w3 pairs)
    int K, nb, urows;     // columns, blocks per row, rows per unit
    int rbytes, sbytes;   // split-row bytes per row, scale bytes per row
    int R;                // units per ring stage
    int embed;            // input is the current token's embedding row (first phase)
    const float *in;      // input vector (x, SwiGLU output; WO merges the attention partials instead)
    const float *norm_w;  // fused rmsnorm weight or null
    float *out;           // WO/W2: x (+=), FFN: h, OUT: logits
    void *kc, *vc;        // QKV / ATTN: this layer's caches [max_seq][KVl] (float or __half: kv16)
    // tensor parallelism: exchange xex (2 x layer + {0: after wo, 1: after w2}) of the step, or -1.  The
    // row sums are this rank's partials: they go to slot xex % 2 of every rank, tagged, and each CTA then
    // adds the ranks' partials of its own rows to x
    int xex;
    // rows split along K (rows too long for a ring slot): C chunks of kb blocks (the last one shorter),
    // each a stage; a unit's chunks are consecutive, a row's chunk = its scales (padded to 16 bytes) and
    // quants.  C = 1: whole units, R per stage
    int C, kb;
    int pad_[1];
};

constexpr int kDecodeMaxTp = 8;
// per-rank exchange block (one allocation, mapped by every rank of a tensor-parallel group):
//   [0, 256)                   sync words: u32 key counter at 16, u32 epoch at 32, u64 argmax keys
//                              [kDecodeMaxTp] at 64
//   [256, 256 + 16 * tp * D)   partial rows [2 slots][tp ranks][D] as 64-bit (float bits, tag) words
//   then                       the full logits [V] floats (every rank writes its shard into every rank's)
constexpr int kXchSync = 256;
constexpr int kXchKeyCtr = 16, kXchEpoch = 32, kXchKeys = 64;
struct DecodePeers {
    uint8_t *blk[kDecodeMaxTp];  // every rank's exchange block (this rank's own at [rank])
};

struct DecodeParams {
    const DecodePhase *ph;
    int nph;
    int D, Dq, KVl, hd, nkv, group, gsplit;  // attention geometry (gsplit: CTAs per KV head's query group)
    float eps, scale;
    const uint8_t *tok;  // embedding table (file layout)
    int dt_tok;
    float *x;  // residual stream
    float *q;
    float *logits;
    const float2 *rope;
    int *state;  // [token, pos, step, prompt length]
    int vocab;   // valid tokens [0, vocab)
    const int *forced;
    int *gen;
    int gen_cap;
    unsigned long long *amax_key;
    int *amax_ctr;
    unsigned *gbar;  // grid barrier arrival counter (zero between steps)
    float *apart;    // attention segment partials [nkv * gsplit][maxseg][4][4 + hd]
    int maxseg;
    int kv16;  // the KV cache holds fp16 (else fp32)
    int tp, rank;      // tensor-parallel group (tp 1: a single GPU)
    int xph;           // cross-rank exchanges per step (2 x layers)
    int64_t xlog_off;  // byte offset of the logits in an exchange block
    DecodePeers peers;
    int *err;
    int nslots, slot_bytes;
    int off_bars, off_xq, off_xds, off_red, off_part;
};

// bytes of one row's chunk of kb blocks in the K-split layout (kb = all blocks: a split row)
__host__ __device__ inline int64_t chunk_row_bytes(int dtype, int64_t kb) {
    return ((kb * 2 + 15) / 16) * 16 + kb * (dtype == QMC_Q8_0 ? 32 : 16);
}
// K-split layout of a matrix: source row r (file layout) goes to unit r / per, position r % per + pos0,
// of units of urows rows cut in chunks of kb blocks (kb >= ceil(K/32): the split-row layout above)
// (row0: the global index of the first source row, so that a row range of a stacked matrix lands in its
// own units)
int launch_repack_chunked(int dtype, const void *aos, int64_t row0, int64_t rows, int64_t K, int kb, int urows, int per,
                          int pos0, void *dst, cudaStream_t s);
// the same matrix (rows [0, rows), same unit mapping) from chunks of kb_src blocks to chunks of kb_dst
int launch_relayout_chunked(int dtype, const void *src, int kb_src, void *dst, int kb_dst, int64_t rows, int64_t K,
                            int urows, int per, int pos0, cudaStream_t s);
// bytes of a unit of urows rows split into chunks of kb blocks
__host__ __device__ inline int64_t chunked_unit_bytes(int dtype, int64_t K, int64_t kb, int urows) {
    const int64_t nb = (K + 31) / 32, k = kb < nb ? kb : nb, C = (nb + k - 1) / k;
    return urows * ((C - 1) * chunk_row_bytes(dtype, k) + chunk_row_bytes(dtype, nb - (C - 1) * k));
}

struct DecodePlan {
    int nslots = 0, slot_bytes = 0, off_bars = 0, off_xq = 0, off_xds = 0, off_red = 0, off_part = 0;
    int groups = 0;  // stage groups (consumer warps that each take every groups-th stage)
    size_t smem = 0;
};
// ring / shared-memory plan for the largest unit and activation length of the model; false if the
// model does not fit (then the per-kernel path is used)
// part_bytes: shared memory for the chunk partial sums of K-split phases
bool plan_decode(int64_t max_unit_bytes, int nb_max, int hd, int group, size_t smem_optin, DecodePlan *out,
                 int64_t part_bytes = 0);
// the slot size of plan_decode's 22-slot ring (what K-split chunks are cut to)
int64_t decode_slot_bytes(int nb_max, int hd, int group, size_t smem_optin, int64_t part_bytes);
// one CTA per SM, cooperative (all CTAs co-resident for the grid barriers)
int launch_decode(const DecodeParams &p, const DecodePlan &plan, int grid, cudaStream_t s);

}  // namespace qmc
