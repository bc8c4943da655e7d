// Seeded synthetic weights generated directly in HBM (the benchmark's N(0, std) random models).
//
// Definition (shared with the CPU writer used for the reference's .qlm files, which must produce the
// same bytes): element (r, c) of 2-D tensor number `tid` is (float)(std * z) where z is the inverse
// normal CDF of u = ((h >> 11) + 0.5) * 2^-53, h = fmix(fmix(seed ^ fmix(tid + C0)) + idx * C1),
// idx = r * cols + c, fmix = the splitmix64 finaliser.  The inverse CDF is Acklam's rational
// approximation (P. J. Acklam, 2003) with an atanh-series natural log.  Every double operation is an
// explicitly rounded intrinsic, so no FMA contraction can change a bit.  Quantized tensors are
// quantized per row with the bit-exact block quantizer.
#include "synth.cuh"

namespace qmc {
namespace {

__device__ __forceinline__ uint64_t fmix(uint64_t z) {
    z ^= z >> 30;
    z *= 0xbf58476d1ce4e5b9ULL;
    z ^= z >> 27;
    z *= 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

__device__ double syn_log(double x) {
    uint64_t b = (uint64_t)__double_as_longlong(x);
    int e = (int)((b >> 52) & 0x7ff) - 1023;
    b = (b & 0x000fffffffffffffULL) | 0x3ff0000000000000ULL;
    double m = __longlong_as_double((long long)b);
    if (m > 1.4142135623730951) {
        m = __dmul_rn(m, 0.5);
        e += 1;
    }
    const double s = __ddiv_rn(__dadd_rn(m, -1.0), __dadd_rn(m, 1.0));
    const double s2 = __dmul_rn(s, s);
    double p = __ddiv_rn(1.0, 25.0);
    for (int k = 11; k >= 0; k--) p = __dadd_rn(__ddiv_rn(1.0, (double)(2 * k + 1)), __dmul_rn(s2, p));
    return __dadd_rn(__dmul_rn((double)e, 0.6931471805599453), __dmul_rn(__dmul_rn(2.0, s), p));
}

__device__ __forceinline__ double hpoly(const double *c, int n, double x) {  // ((c0 x + c1) x + ...) + c_{n-1}
    double v = c[0];
    for (int i = 1; i < n; i++) v = __dadd_rn(__dmul_rn(v, x), c[i]);
    return v;
}

__device__ double syn_probit(double u) {
    const double a[6] = {-3.969683028665376e+01, 2.209460984245205e+02, -2.759285104469687e+02,
                         1.383577518672690e+02, -3.066479806614716e+01, 2.506628277459239e+00};
    const double b[6] = {-5.447609879822406e+01, 1.615858368580409e+02, -1.556989798598866e+02,
                         6.680131188771972e+01, -1.328068155288572e+01, 1.0};
    const double c[6] = {-7.784894002430293e-03, -3.223964580411365e-01, -2.400758277161838e+00,
                         -2.549732539343734e+00, 4.374664141464968e+00, 2.938163982698783e+00};
    const double d[5] = {7.784695709041462e-03, 3.224671290700398e-01, 2.445134137142996e+00,
                         3.754408661907416e+00, 1.0};
    if (u < 0.02425 || u > 0.97575) {
        const double t = __dsqrt_rn(__dmul_rn(-2.0, syn_log(u < 0.5 ? u : __dadd_rn(1.0, -u))));
        const double q = __ddiv_rn(hpoly(c, 6, t), hpoly(d, 5, t));
        return u < 0.5 ? q : -q;
    }
    const double q = __dadd_rn(u, -0.5), r = __dmul_rn(q, q);
    return __ddiv_rn(__dmul_rn(hpoly(a, 6, r), q), hpoly(b, 6, r));
}

__device__ __forceinline__ float syn_value(uint64_t key, uint64_t idx, double stdv) {
    const uint64_t h = fmix(key + idx * 0x9e3779b97f4a7c15ULL);
    const double u = __dmul_rn(__dadd_rn((double)(h >> 11), 0.5), 1.0 / 9007199254740992.0);
    return __double2float_rn(__dmul_rn(stdv, syn_probit(u)));
}

// rows [r0, r0+nr) and columns [c0, c0+nc) of a rows x cols tensor, written as a dense nr x nc tensor
// in `dtype` layout (c0 and nc multiples of 32 for quantized output, or nc = cols - c0)
__global__ void synth_kernel(uint64_t key, int dtype, int64_t cols, int64_t r0, int64_t nr, int64_t c0, int64_t nc,
                             double stdv, uint8_t *out) {
    const int lane = threadIdx.x & 31;
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5, nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int64_t nb = nblocks(nc), rb = row_bytes(dtype, nc);
    for (int64_t blk = gw; blk < nr * nb; blk += nwarps) {
        const int64_t r = blk / nb, b = blk % nb, cl = b * 32 + lane;
        const float v = cl < nc ? syn_value(key, (uint64_t)((r0 + r) * cols + c0 + cl), stdv) : 0.0f;
        if (dtype == QMC_F32) {
            if (cl < nc) ((float *)(out + r * rb))[cl] = v;
            continue;
        }
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

__global__ void fill_kernel(float *p, int64_t n, float v) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) p[i] = v;
}

uint64_t hfmix(uint64_t z) {
    z ^= z >> 30;
    z *= 0xbf58476d1ce4e5b9ULL;
    z ^= z >> 27;
    z *= 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

}  // namespace

int launch_synth(uint64_t seed, uint64_t tid, int dtype, int64_t cols, int64_t r0, int64_t nr, int64_t c0, int64_t nc,
                 double stdv, void *out, cudaStream_t s) {
    if (nr <= 0 || nc <= 0) return QMC_OK;
    if (dtype != QMC_F32 && (c0 % 32)) return set_error(QMC_EINVAL, "synth: column slice not block aligned");
    const uint64_t key = hfmix(seed ^ hfmix(tid + 0x632be59bd9b4e019ULL));
    const int64_t warps = nr * nblocks(nc);
    const int64_t grid = (warps * 32 + 255) / 256;
    synth_kernel<<<(int)(grid < 148 * 64 ? grid : 148 * 64), 256, 0, s>>>(key, dtype, cols, r0, nr, c0, nc, stdv,
                                                                        (uint8_t *)out);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

int launch_fill(float *p, int64_t n, float v, cudaStream_t s) {
    if (n <= 0) return QMC_OK;
    fill_kernel<<<(int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096), 256, 0, s>>>(p, n, v);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

}  // namespace qmc
