// Device-side sampler: temperature / top-k / top-p over logits already in HBM, with the reference's
// xorshift64* stream (src/sampler.c), so a decode loop needs no 128 KB logits copy per token.
//
// The reference (src/sampler.c:50-106) ranks the candidates by (probability desc, index asc) with a heap,
// keeps the first top_k, takes the shortest prefix whose cumulative mass reaches top_p, draws
// u = rng() * mass and walks the prefix until the cumulative mass exceeds u.  Only three positions of
// that ranking matter: the top-k boundary, the top-p boundary and the element u lands on.  One CTA finds
// each with radix selection over the probability bits (non-negative floats order like their bit
// patterns), 8 bits per pass from the top, using counts for the top-k rank and probability mass for the
// other two; ties (equal probabilities) are resolved by index in closed form and a second selection
// over the index bits.  Masses are summed in double as the reference does, in a different order.
#include <math.h>

#include "sampler.cuh"

namespace qmc {
namespace {

constexpr int kST = 1024;  // threads of the sampling CTA

struct SampleArgs {
    const float *logits;
    int n;
    float temperature;
    int top_k;
    float top_p;
    uint64_t *rng;
    float *p;  // [n] probabilities (scratch)
    int32_t *out;
};

// xorshift64* draw in [0, 1) (src/sampler.c:18-25)
__device__ __forceinline__ float rng_uniform(uint64_t *state) {
    uint64_t x = *state;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *state = x;
    return (float)((x * 0x2545F4914F6CDD1DULL) >> 40) / 16777216.0f;
}

__device__ __forceinline__ uint32_t keyof(float v) { return __float_as_uint(v); }

// shared scratch of the selections
constexpr int kDigit = 11, kBins = 1 << kDigit;  // key bits per selection pass, bins per pass
struct SelShared {
    int cnt[kBins];
    double mass[kBins];
    uint32_t lo, hi;  // smallest / largest key in the set
    uint32_t prefix;
    int found;
    double rem;
    int irem;
};

// Radix selection over the keys of the elements in set S, descending.  mode 0: the element of rank
// `target` (1-based count); mode 1: the first element at which the cumulative mass reaches `target`
// (cum >= target); mode 2: the first element at which it exceeds `target` (cum > target).  Returns the
// key; *rest receives what is left of the target inside that key's group (count, or mass), *found
// whether any element qualifies.
template <typename InS>
__device__ uint32_t select_key(const float *p, int n, InS in_s, int mode, double target, double *rest, bool *found,
                               SelShared &sh) {
    const int t = threadIdx.x;
    if (t == 0) sh.lo = 0xffffffffu, sh.hi = 0u, sh.found = 1, sh.rem = target;
    __syncthreads();
    // The bits that every key of S shares need no pass: the passes start at the highest bit where the
    // smallest and largest keys differ.  (Nearly flat distributions share their top 10-20 bits; a pass
    // over them would send every element to one bin, every update an atomic on the same address.)
    {
        uint32_t lo = 0xffffffffu, hi = 0u;
        for (int i = t; i < n; i += kST) {
            const float v = p[i];
            if (in_s(i, v)) lo = min(lo, keyof(v)), hi = max(hi, keyof(v));
        }
        lo = __reduce_min_sync(0xffffffffu, lo);
        hi = __reduce_max_sync(0xffffffffu, hi);
        if ((t & 31) == 0) atomicMin(&sh.lo, lo), atomicMax(&sh.hi, hi);
    }
    __syncthreads();
    const uint32_t lo = sh.lo, hi = sh.hi;
    int bits = 0;  // low bits still to resolve (at least one pass: it checks the target against S's total)
    uint32_t pmask = 0;
    if (lo <= hi) {
        bits = lo == hi ? 1 : 32 - __clz(lo ^ hi);
        pmask = bits == 32 ? 0u : ~((1u << bits) - 1u);
    } else if (t == 0) {
        sh.found = 0;  // S is empty
    }
    if (t == 0) sh.prefix = lo & pmask;
    __syncthreads();
    while (bits > 0) {
        const int w = bits < kDigit ? bits : kDigit, shift = bits - w, nbin = 1 << w;
        for (int d = t; d < nbin; d += kST) sh.cnt[d] = 0, sh.mass[d] = 0.0;
        __syncthreads();
        const uint32_t prefix = sh.prefix;
        for (int i = t; i < n; i += kST) {
            const float v = p[i];
            const uint32_t k = keyof(v);
            if ((k & pmask) == prefix && in_s(i, v)) {
                const int d = (k >> shift) & (nbin - 1);
                if (mode == 0) atomicAdd(&sh.cnt[d], 1);
                else atomicAdd(&sh.mass[d], (double)v);
            }
        }
        __syncthreads();
        // the bin where the descending cumulative weight reaches the target: warp 0, lane l summing bins
        // nbin-1-l*c .. down (c = nbin/32), a warp scan of the lane sums, then the first lane whose range
        // holds the target walks its bins
        if (t < 32 && sh.found) {
            const int c = nbin >= 32 ? nbin / 32 : 1, top = nbin - 1 - t * c;
            double tot = 0.0;
            if (top >= 0)
                for (int e = 0; e < c; e++) tot += mode == 0 ? (double)sh.cnt[top - e] : sh.mass[top - e];
            double incl = tot;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const double y = __shfl_up_sync(0xffffffffu, incl, o);
                if (t >= o) incl += y;
            }
            const double rem = sh.rem - (incl - tot);  // what is left of the target when this range starts
            const bool here = top >= 0 && tot > 0.0 && (mode == 2 ? rem < tot : rem <= tot);
            const unsigned hit = __ballot_sync(0xffffffffu, here);
            if (hit == 0) {
                if (t == 0) sh.found = 0;
            } else if (t == __ffs(hit) - 1) {
                // the walk subtracts bin by bin, which need not reproduce `tot`'s rounding: if it runs
                // off the range's end, the pick stays the last bin that holds weight (with what was
                // left of the target clamped into it), never an empty bin
                double r = rem, last_w = 0.0;
                int pick = top, last = top;
                bool hit_bin = false;
                for (int e = 0; e < c && !hit_bin; e++) {
                    const double wd = mode == 0 ? (double)sh.cnt[top - e] : sh.mass[top - e];
                    if (wd > 0.0) {
                        if (mode == 2 ? r < wd : r <= wd) {
                            pick = top - e;
                            hit_bin = true;
                        } else {
                            last = top - e, last_w = wd;
                            r -= wd;
                        }
                    }
                }
                if (!hit_bin) {  // ran off the end: the last bin with weight, the target at its far edge
                    pick = last;
                    r = mode == 2 ? nextafter(last_w, 0.0) : last_w;
                }
                sh.prefix = prefix | ((uint32_t)pick << shift), sh.rem = r;
            }
        }
        __syncthreads();
        if (!sh.found) break;
        pmask |= (uint32_t)(nbin - 1) << shift;
        bits = shift;
    }
    *rest = sh.rem;
    *found = sh.found != 0;
    const uint32_t key = sh.prefix;
    __syncthreads();
    return key;
}

// the j-th smallest index (1-based) among the elements of S with key `key`
template <typename InS>
__device__ int select_tie(const float *p, int n, InS in_s, uint32_t key, int j, SelShared &sh) {
    const int t = threadIdx.x;
    if (t == 0) sh.prefix = 0, sh.irem = j;
    __syncthreads();
    uint32_t pmask = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int d = t; d < 256; d += kST) sh.cnt[d] = 0;
        __syncthreads();
        const uint32_t prefix = sh.prefix;
        for (int i = t; i < n; i += kST) {
            const float v = p[i];
            if (keyof(v) == key && ((uint32_t)i & pmask) == prefix && in_s(i, v)) atomicAdd(&sh.cnt[(i >> shift) & 255], 1);
        }
        __syncthreads();
        if (t == 0) {
            int rem = sh.irem, pick = 255;
            for (int d = 0; d < 256; d++) {
                if (rem <= sh.cnt[d]) {
                    pick = d;
                    break;
                }
                rem -= sh.cnt[d];
            }
            sh.prefix = prefix | ((uint32_t)pick << shift), sh.irem = rem;
        }
        __syncthreads();
        pmask |= 255u << shift;
    }
    const int idx = (int)sh.prefix;
    __syncthreads();
    return idx;
}

template <typename T>
__device__ T block_sum(T v, T *red) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int t = threadIdx.x;
    __syncthreads();
    if ((t & 31) == 0) red[t >> 5] = v;
    __syncthreads();
    if (t == 0) {
        T s = 0;
        for (int w = 0; w < kST / 32; w++) s += red[w];
        red[0] = s;
    }
    __syncthreads();
    const T s = red[0];
    __syncthreads();
    return s;
}

__global__ void __launch_bounds__(kST, 1) sample_kernel(SampleArgs a) {
    __shared__ SelShared sh;
    __shared__ double redd[kST / 32];
    __shared__ int redi[kST / 32];
    __shared__ unsigned long long best_s;
    const int t = threadIdx.x, n = a.n;
    const float *lg = a.logits;
    // greedy: first maximum, NaN in slot 0 never replaced (src/sampler.c:27-32, :52)
    if (a.temperature == 0.0f || a.top_k == 1) {
        if (t == 0) best_s = 0;
        __syncthreads();
        unsigned long long best = 0;
        for (int i = t; i < n; i += kST) {
            const float v = lg[i];
            if (v == v) best = max(best, argmax_key(v, i));
        }
        atomicMax(&best_s, best);
        __syncthreads();
        if (t == 0) *a.out = (lg[0] != lg[0] || best_s == 0) ? 0 : argmax_index(best_s);
        return;
    }
    // softmax(logits / T): max, e = expf((x - max) / T), double sum, p = (float)(e / sum)
    float mx = -INFINITY;
    for (int i = t; i < n; i += kST) mx = fmaxf(mx, lg[i]);
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    __shared__ float redf[kST / 32];
    if ((t & 31) == 0) redf[t >> 5] = mx;
    __syncthreads();
    if (t == 0) {
        float m = redf[0];
        for (int w = 1; w < kST / 32; w++) m = fmaxf(m, redf[w]);
        redf[0] = m;
    }
    __syncthreads();
    mx = redf[0];
    double sum = 0.0;
    for (int i = t; i < n; i += kST) {
        const float e = expf(__fdiv_rn(__fsub_rn(lg[i], mx), a.temperature));
        a.p[i] = e;
        sum += (double)e;
    }
    sum = block_sum(sum, redd);
    for (int i = t; i < n; i += kST) a.p[i] = (float)((double)a.p[i] / sum);
    __syncthreads();
    const float *p = a.p;
    // candidates: the top-p prefilter (a token with p < (1 - top_p) / (n - 1) can never be in the
    // nucleus), or all when it is off or removes everything (src/sampler.c:62-71)
    float cut = -1.0f;
    if (a.top_k == 0 && a.top_p < 1.0f && n > 1) {
        cut = __fdiv_rn(__fsub_rn(1.0f, a.top_p), (float)(n - 1));
        int c = 0;
        for (int i = t; i < n; i += kST) c += p[i] >= cut;
        if (block_sum(c, redi) == 0) cut = -1.0f;
    }
    int nc = n;
    if (cut >= 0.0f) {
        int c = 0;
        for (int i = t; i < n; i += kST) c += p[i] >= cut;
        nc = block_sum(c, redi);
    }
    auto cand = [&](int i, float v) { (void)i; return v >= cut; };  // cut < 0: every element
    const int k = (a.top_k > 0 && a.top_k < nc) ? a.top_k : nc;
    // top-k boundary (key tk, last tie index ik): the first k of the ranking
    double rest;
    bool found;
    uint32_t tk = 0;
    int ik = n;
    if (k < nc) {
        tk = select_key(p, n, cand, 0, (double)k, &rest, &found, sh);
        ik = select_tie(p, n, cand, tk, (int)rest, sh);
    }
    auto topk = [&](int i, float v) {
        if (!cand(i, v)) return false;
        if (k >= nc) return true;
        const uint32_t kv = keyof(v);
        return kv > tk || (kv == tk && i <= ik);
    };
    // nucleus: the shortest prefix of the top-k ranking whose cumulative mass reaches top_p, else all
    // of it (src/sampler.c:84-93)
    uint32_t tp = keyof(0.0f);
    int ip = -1;
    bool nuc_all = true;
    {
        const uint32_t key = select_key(p, n, topk, 1, (double)a.top_p, &rest, &found, sh);
        if (found) {
            nuc_all = false;
            tp = key;
            const double pt = (double)__uint_as_float(key);
            int ties = 0;
            for (int i = t; i < n; i += kST) ties += keyof(p[i]) == key && topk(i, p[i]);
            ties = block_sum(ties, redi);
            int j = pt > 0.0 ? (int)ceil(rest / pt) : 1;
            j = min(max(j, 1), ties);
            ip = select_tie(p, n, topk, key, j, sh);
        }
    }
    auto nucleus = [&](int i, float v) {
        if (!topk(i, v)) return false;
        if (nuc_all) return true;
        const uint32_t kv = keyof(v);
        return kv > tp || (kv == tp && i <= ip);
    };
    // draw, and the element where the cumulative mass first exceeds u (src/sampler.c:94-105)
    double mass = 0.0;
    for (int i = t; i < n; i += kST)
        if (nucleus(i, p[i])) mass += (double)p[i];
    mass = block_sum(mass, redd);
    __shared__ double u_s;
    if (t == 0) u_s = (double)rng_uniform(a.rng) * mass;
    __syncthreads();
    const double u = u_s;
    const uint32_t key = select_key(p, n, nucleus, 2, u, &rest, &found, sh);
    int pick;
    if (found) {
        const double pt = (double)__uint_as_float(key);
        int ties = 0;
        for (int i = t; i < n; i += kST) ties += keyof(p[i]) == key && nucleus(i, p[i]);
        ties = block_sum(ties, redi);
        int j = pt > 0.0 ? (int)floor(rest / pt) + 1 : 1;
        j = min(max(j, 1), ties);
        pick = select_tie(p, n, nucleus, key, j, sh);
    } else {  // rounding left u at or past the total: the last element of the prefix
        uint32_t lastk;
        if (!nuc_all) {
            lastk = tp;
            pick = ip;
        } else {
            // the lowest-ranked nucleus element: smallest key, then the largest index among its ties
            int cnt = 0;
            for (int i = t; i < n; i += kST) cnt += nucleus(i, p[i]);
            cnt = block_sum(cnt, redi);
            lastk = select_key(p, n, nucleus, 0, (double)cnt, &rest, &found, sh);
            pick = select_tie(p, n, nucleus, lastk, (int)rest, sh);
        }
        (void)lastk;
    }
    if (t == 0) *a.out = pick;
}

}  // namespace

int launch_sample(const float *logits, int n, float temperature, int top_k, float top_p, uint64_t *rng, float *p,
                  int32_t *out, cudaStream_t s) {
    SampleArgs a{logits, n, temperature, top_k, top_p, rng, p, out};
    sample_kernel<<<1, kST, 0, s>>>(a);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

}  // namespace qmc

// ---------------------------------------------------------------- C ABI
struct qmc_sampler {
    int dev = 0, n = 0, top_k = 0;
    float temperature = 0.0f, top_p = 1.0f;
    uint64_t *rng = nullptr;  // device
    float *p = nullptr;       // device scratch [n]
    int32_t *out = nullptr;   // device
    int32_t *h_out = nullptr; // pinned
};

namespace {
// make the sampler's device current: its buffers live there, and a kernel launched on another device
// would read and write them through peer addresses (or fault without peer access)
int sampler_device(const qmc_sampler *s) {
    int d = -1;
    QMC_CUDA(cudaGetDevice(&d));
    if (d != s->dev) QMC_CUDA(cudaSetDevice(s->dev));
    return QMC_OK;
}
}  // namespace

extern "C" {

int qmc_sampler_create(int32_t n_vocab, float temperature, int32_t top_k, float top_p, uint64_t seed,
                       qmc_sampler **out) {
    using namespace qmc;
    if (!out || n_vocab < 1) return set_error(QMC_EINVAL, "sampler_create: bad arguments");
    *out = nullptr;
    int dev = -1;
    QMC_CUDA(cudaGetDevice(&dev));
    qmc_sampler *s = new qmc_sampler();
    s->dev = dev;
    s->n = n_vocab;
    // the reference's normalisation of the settings (src/sampler.c:8-11)
    s->temperature = temperature < 0 ? 0 : temperature;
    s->top_k = top_k < 0 ? 0 : top_k;
    s->top_p = (top_p <= 0 || top_p > 1) ? 1.0f : top_p;
    const uint64_t st = seed ? seed : 0x9e3779b97f4a7c15ULL;
    cudaError_t e = cudaMalloc(&s->rng, 8);
    if (e == cudaSuccess) e = cudaMalloc(&s->p, (size_t)n_vocab * 4);
    if (e == cudaSuccess) e = cudaMalloc(&s->out, 4);
    if (e == cudaSuccess) e = cudaMallocHost(&s->h_out, 4);
    if (e == cudaSuccess) e = cudaMemcpy(s->rng, &st, 8, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        qmc_sampler_free(s);
        return cuda_fail(e, "sampler_create");
    }
    *out = s;
    return QMC_OK;
}

int qmc_sampler_enqueue(qmc_sampler *s, const float *dev_logits, int32_t *dev_token, void *stream) {
    using namespace qmc;
    if (!s || !dev_logits || !dev_token) return set_error(QMC_EINVAL, "sampler_enqueue: null argument");
    if (const int rc = sampler_device(s)) return rc;
    return launch_sample(dev_logits, s->n, s->temperature, s->top_k, s->top_p, s->rng, s->p, dev_token,
                         pick_stream(stream));
}

int qmc_sampler_sample(qmc_sampler *s, const float *dev_logits, int32_t *token) {
    using namespace qmc;
    if (!s || !dev_logits || !token) return set_error(QMC_EINVAL, "sampler_sample: null argument");
    if (const int rc = sampler_device(s)) return rc;
    cudaStream_t st = pick_stream(nullptr);
    const int rc = launch_sample(dev_logits, s->n, s->temperature, s->top_k, s->top_p, s->rng, s->p, s->out, st);
    if (rc) return rc;
    QMC_CUDA(cudaMemcpyAsync(s->h_out, s->out, 4, cudaMemcpyDeviceToHost, st));
    QMC_CUDA(cudaStreamSynchronize(st));
    *token = *s->h_out;
    return QMC_OK;
}

int qmc_sampler_rng(qmc_sampler *s, uint64_t *state) {
    using namespace qmc;
    if (!s || !state) return set_error(QMC_EINVAL, "sampler_rng: null argument");
    if (const int rc = sampler_device(s)) return rc;
    QMC_CUDA(cudaDeviceSynchronize());
    QMC_CUDA(cudaMemcpy(state, s->rng, 8, cudaMemcpyDeviceToHost));
    return QMC_OK;
}

int qmc_sampler_free(qmc_sampler *s) {
    if (!s) return QMC_OK;
    cudaSetDevice(s->dev);
    cudaFree(s->rng);
    cudaFree(s->p);
    cudaFree(s->out);
    if (s->h_out) cudaFreeHost(s->h_out);
    delete s;
    return QMC_OK;
}

}  // extern "C"
