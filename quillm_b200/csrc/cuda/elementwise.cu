// Quantize / dequantize, embedding lookup, argmax and the stand-alone elementwise ops of src/ops.c.
#include "elementwise.cuh"

namespace qmc {
namespace {

// ---------------------------------------------------------------- row quantization (warp per block)
__global__ void quantize_rows_kernel(int dtype, const float *__restrict__ x, uint8_t *__restrict__ out, int64_t rows,
                                     int64_t cols) {
    const int lane = threadIdx.x & 31;
    const int64_t nb = nblocks(cols), rb = row_bytes(dtype, cols);
    const int64_t w0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t blk = w0; blk < rows * nb; blk += nw) {
        const int64_t r = blk / nb, b = blk % nb, c = b * 32 + lane;
        const float v = c < cols ? x[r * cols + c] : 0.0f;
        float dd;
        uint32_t dh;
        if (dtype == QMC_Q8_0) {
            const int q = quant_lane(v, 127.0f, -127, 127, &dd, &dh);
            uint8_t *o = out + r * rb + b * kQ8Bytes;
            o[2 + lane] = (uint8_t)(int8_t)q;
            if (lane == 0) o[0] = (uint8_t)dh, o[1] = (uint8_t)(dh >> 8);
        } else {
            const int q = quant_lane(v, 7.0f, -8, 7, &dd, &dh) + 8;
            const int hi = __shfl_down_sync(0xffffffffu, q, 1);
            uint8_t *o = out + r * rb + b * kQ4Bytes;
            if (!(lane & 1)) o[2 + lane / 2] = (uint8_t)(q | (hi << 4));
            if (lane == 0) o[0] = (uint8_t)dh, o[1] = (uint8_t)(dh >> 8);
        }
    }
}

__global__ void dequantize_rows_kernel(int dtype, const uint8_t *__restrict__ in, float *__restrict__ y, int64_t rows,
                                       int64_t cols) {
    const int64_t rb = row_bytes(dtype, cols);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows * cols; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = deq_elem(dtype, in + (i / cols) * rb, i % cols);
}

// x = row `*token` of the embedding table (src/model.c:162)
__global__ void embed_kernel(int dtype, const uint8_t *__restrict__ table, int64_t cols, int64_t c0,
                             const int *__restrict__ token, float *__restrict__ x) {
    pdl_wait();
    const int64_t rb = row_bytes(dtype, cols);
    const uint8_t *row = table + (int64_t)(*token) * rb;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) x[c] = deq_elem(dtype, row, c);
    (void)c0;
    pdl_launch_dependents();
}

// ---------------------------------------------------------------- argmax (first maximum, src/sampler.c:27-32)
__device__ __forceinline__ void better(float &bv, int &bi, float v, int i) {
    // strictly greater wins; equal values keep the lower index
    if (v > bv || (v == bv && i < bi)) bv = v, bi = i;
}

__global__ void argmax_kernel(const float *__restrict__ x, int n, int *__restrict__ out, int *__restrict__ advance_pos,
                              const int *__restrict__ forced, const int *__restrict__ forced_n_ptr,
                              int *__restrict__ step_ctr, int *__restrict__ tokens_out, int tokens_cap) {
    pdl_wait();
    __shared__ float sv[32];
    __shared__ int si[32];
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = t; i < n; i += blockDim.x) {
        const float v = x[i];
        if (v == v) better(bv, bi, v, i);  // NaN never wins (the reference's `>` is false for NaN)
    }
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        better(bv, bi, ov, oi);
    }
    if (lane == 0) sv[warp] = bv, si[warp] = bi;
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x >> 5;
        bv = lane < nw ? sv[lane] : -INFINITY;
        bi = lane < nw ? si[lane] : 0x7fffffff;
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            better(bv, bi, ov, oi);
        }
        if (lane == 0) {
            int best = bi == 0x7fffffff ? 0 : bi;
            if (x[0] != x[0]) best = 0;  // a NaN in slot 0 is never replaced by the reference
            if (step_ctr) {
                // device-resident generation: state = {token, pos, step, prompt length}
                advance_state(best, out, forced, tokens_out, tokens_cap);
            } else {
                *out = best;
            }
            if (advance_pos && !step_ctr) *advance_pos += 1;
        }
    }
}

// ---------------------------------------------------------------- elementwise (src/ops.c:93-133)
__global__ void rmsnorm_kernel(float *out, const float *x, const float *w, int64_t n, float eps) {
    __shared__ double red[32];
    __shared__ float sinv;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    double ss = 0.0;
    for (int64_t i = t; i < n; i += blockDim.x) ss += (double)x[i] * (double)x[i];
    ss = warp_sum_d(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (t == 0) {
        double s = 0.0;
        for (int i = 0; i < (int)(blockDim.x >> 5); i++) s += red[i];
        sinv = (float)(1.0 / sqrt(s / (double)n + (double)eps));
    }
    __syncthreads();
    const float inv = sinv;
    for (int64_t i = t; i < n; i += blockDim.x) out[i] = __fmul_rn(__fmul_rn(x[i], inv), w[i]);
}

__global__ void softmax_kernel(float *x, int64_t n) {
    __shared__ float fred[32];
    __shared__ double dred[32];
    __shared__ float smx, sinv;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5, nw = blockDim.x >> 5;
    float mx = -INFINITY;
    for (int64_t i = t; i < n; i += blockDim.x) mx = fmaxf(mx, x[i]);
    mx = warp_max(mx);
    if (lane == 0) fred[warp] = mx;
    __syncthreads();
    if (t == 0) {
        float m = x[0];
        for (int i = 0; i < nw; i++) m = fred[i] > m ? fred[i] : m;
        smx = m;
    }
    __syncthreads();
    double s = 0.0;
    for (int64_t i = t; i < n; i += blockDim.x) {
        const float e = expf(x[i] - smx);
        x[i] = e;
        s += e;
    }
    s = warp_sum_d(s);
    if (lane == 0) dred[warp] = s;
    __syncthreads();
    if (t == 0) {
        double a = 0.0;
        for (int i = 0; i < nw; i++) a += dred[i];
        sinv = (float)(1.0 / a);
    }
    __syncthreads();
    for (int64_t i = t; i < n; i += blockDim.x) x[i] = __fmul_rn(x[i], sinv);
}

__global__ void rope_kernel(float *v, int64_t n_heads, int64_t hd, RopeRow cs) {
    const int64_t half = hd / 2;
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n_heads * half; j += (int64_t)gridDim.x * blockDim.x) {
        const int64_t h = j / half, i = j % half;
        float *p = v + h * hd + 2 * i;
        const float a = p[0], b = p[1], c = cs.v[2 * i], s = cs.v[2 * i + 1];
        p[0] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        p[1] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
    }
}

__global__ void swiglu_kernel(float *g, const float *u, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        g[i] = __fmul_rn(__fdiv_rn(g[i], __fadd_rn(1.0f, expf(-g[i]))), u[i]);
}

// one weight row against Q8_0 activations, or two f32 vectors: thread per block, then a tree sum
__global__ void dot_kernel(int dtype, const uint8_t *w, const uint8_t *xq, int64_t n, float *out) {
    __shared__ float red[32];
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    float s = 0.0f;
    if (dtype == QMC_F32) {
        for (int64_t i = t; i < n; i += blockDim.x) s = fmaf(((const float *)w)[i], ((const float *)xq)[i], s);
    } else {
        for (int64_t b = t; b < nblocks(n); b += blockDim.x) {
            const uint8_t *xb = xq + b * kQ8Bytes;
            int acc = 0;
            float dw;
            if (dtype == QMC_Q8_0) {
                const uint8_t *wb = w + b * kQ8Bytes;
                for (int i = 0; i < 32; i++) acc += (int)(int8_t)wb[2 + i] * (int)(int8_t)xb[2 + i];
                dw = h2f(wb[0] | (wb[1] << 8));
            } else {
                const uint8_t *wb = w + b * kQ4Bytes;
                for (int j = 0; j < 16; j++)
                    acc += ((wb[2 + j] & 15) - 8) * (int)(int8_t)xb[2 + 2 * j] +
                           ((wb[2 + j] >> 4) - 8) * (int)(int8_t)xb[3 + 2 * j];
                dw = h2f(wb[0] | (wb[1] << 8));
            }
            s += (float)acc * (dw * h2f(xb[0] | (xb[1] << 8)));
        }
    }
    s = warp_sum(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (t == 0) {
        float a = 0.0f;
        for (int i = 0; i < (int)(blockDim.x >> 5); i++) a += red[i];
        *out = a;
    }
}

inline cudaLaunchConfig_t cfg1(dim3 g, dim3 b, cudaStream_t s, bool pdl, cudaLaunchAttribute *attr) {
    cudaLaunchConfig_t c = {};
    c.gridDim = g;
    c.blockDim = b;
    c.stream = s;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    c.attrs = pdl ? attr : nullptr;
    c.numAttrs = pdl ? 1 : 0;
    return c;
}

}  // namespace

int launch_quantize_rows(int dtype, const float *x, void *out, int64_t rows, int64_t cols, cudaStream_t s) {
    if (dtype != QMC_Q8_0 && dtype != QMC_Q4_0) return set_error(QMC_EINVAL, "quantize: dtype must be Q8_0 or Q4_0");
    if (rows <= 0 || cols <= 0) return QMC_OK;
    const int64_t warps = rows * nblocks(cols);
    const int grid = (int)(warps * 32 + 255) / 256 < 65535 * 8 ? (int)((warps * 32 + 255) / 256) : 65535 * 8;
    quantize_rows_kernel<<<grid, 256, 0, s>>>(dtype, x, (uint8_t *)out, rows, cols);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

int launch_dequantize_rows(int dtype, const void *in, float *y, int64_t rows, int64_t cols, cudaStream_t s) {
    if (rows <= 0 || cols <= 0) return QMC_OK;
    const int64_t n = rows * cols;
    const int grid = (int)((n + 255) / 256 < 65535 * 16 ? (n + 255) / 256 : 65535 * 16);
    dequantize_rows_kernel<<<grid, 256, 0, s>>>(dtype, (const uint8_t *)in, y, rows, cols);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

int launch_embed(int dtype, const void *table, int64_t cols, const int *token, float *x, cudaStream_t s, bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t c = cfg1(dim3(1), dim3(1024), s, pdl, attr);
    QMC_CUDA(cudaLaunchKernelEx(&c, embed_kernel, dtype, (const uint8_t *)table, cols, (int64_t)0, token, x));
    return QMC_OK;
}

int launch_argmax(const float *x, int n, int *out, cudaStream_t s, bool pdl, int *advance_pos, const int *forced,
                  const int *forced_n, int *step_ctr, int *tokens_out, int tokens_cap) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t c = cfg1(dim3(1), dim3(1024), s, pdl, attr);
    QMC_CUDA(cudaLaunchKernelEx(&c, argmax_kernel, x, n, out, advance_pos, forced, forced_n, step_ctr, tokens_out,
                                tokens_cap));
    return QMC_OK;
}

int launch_rmsnorm(float *out, const float *x, const float *w, int64_t n, float eps, cudaStream_t s) {
    rmsnorm_kernel<<<1, 1024, 0, s>>>(out, x, w, n, eps);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

int launch_softmax(float *x, int64_t n, cudaStream_t s) {
    if (n <= 0) return QMC_OK;
    softmax_kernel<<<1, 1024, 0, s>>>(x, n);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

int launch_rope(float *v, int64_t n_heads, int64_t hd, const RopeRow &cs, cudaStream_t s) {
    const int64_t n = n_heads * (hd / 2);
    if (n <= 0) return QMC_OK;
    const int grid = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    rope_kernel<<<grid, 256, 0, s>>>(v, n_heads, hd, cs);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

int launch_swiglu(float *g, const float *u, int64_t n, cudaStream_t s) {
    if (n <= 0) return QMC_OK;
    const int grid = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    swiglu_kernel<<<grid, 256, 0, s>>>(g, u, n);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

int launch_dot(int dtype, const void *w, const void *xq, int64_t n, float *out, cudaStream_t s) {
    dot_kernel<<<1, 256, 0, s>>>(dtype, (const uint8_t *)w, (const uint8_t *)xq, n, out);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

}  // namespace qmc
