// C-ABI entry points of libquillm_cuda (include/quillm_cuda.h): error state, per-device context and the
// operator-level calls.  Model-level calls live in model.cu.
#include <math.h>
#include <stdint.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "attention.cuh"
#include "elementwise.cuh"
#include "gemv.cuh"
#include "decode.cuh"
#include "matmul.cuh"
#include "matmul_tc.cuh"

namespace qmc {

static thread_local char g_err[512] = "";

int set_error(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return code;
}

int cuda_fail(cudaError_t e, const char *what) {
    return set_error(e == cudaErrorMemoryAllocation ? QMC_ENOMEM : QMC_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

namespace {
constexpr int kMaxDev = 64;
DevCtx g_ctx[kMaxDev];
std::mutex g_mu;
}  // namespace

DevCtx *ctx() {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= kMaxDev) {
        set_error(QMC_ECUDA, "no CUDA device");
        return nullptr;
    }
    DevCtx *c = &g_ctx[d];
    if (c->device == d) return c;
    std::lock_guard<std::mutex> lk(g_mu);
    if (c->device == d) return c;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, d) != cudaSuccess) {
        set_error(QMC_ECUDA, "cudaGetDeviceProperties failed");
        return nullptr;
    }
    if (prop.major < 10) {
        set_error(QMC_ECUDA, "device %d is sm_%d%d; libquillm_cuda is built for sm_100a", d, prop.major, prop.minor);
        return nullptr;
    }
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&c->err, sizeof(int)) != cudaSuccess || cudaMemset(c->err, 0, sizeof(int)) != cudaSuccess) {
        set_error(QMC_ECUDA, "device context setup failed");
        return nullptr;
    }
    c->num_sms = prop.multiProcessorCount;
    c->max_smem_optin = prop.sharedMemPerBlockOptin;
    c->device = d;
    return c;
}

// host (cos, sin) table row: same double expressions as src/ops.c:116-118, rounded to float
void rope_row_host(int64_t pos, int64_t hd, float theta, float *out_cs) {
    for (int64_t i = 0; i < hd / 2; i++) {
        const double freq = pow((double)theta, -2.0 * (double)i / (double)hd);
        const double ang = (double)pos * freq;
        out_cs[2 * i] = (float)cos(ang);
        out_cs[2 * i + 1] = (float)sin(ang);
    }
}

// scratch that grows on demand (operator-level prefill only; models own their buffers)
static int ensure_scratch(DevCtx *c, size_t bytes, void **out) {
    static thread_local void *buf[kMaxDev];
    static thread_local size_t cap[kMaxDev];
    const int d = c->device;
    if (cap[d] < bytes) {
        if (buf[d]) {
            cudaStreamSynchronize(c->stream);
            cudaFree(buf[d]);
            buf[d] = nullptr;
            cap[d] = 0;
        }
        QMC_CUDA(cudaMalloc(&buf[d], bytes));
        cap[d] = bytes;
    }
    *out = buf[d];
    return QMC_OK;
}

}  // namespace qmc

using namespace qmc;

#define CTX_OR_FAIL()                                                                                                  \
    DevCtx *c_ = ctx();                                                                                                \
    if (!c_) return QMC_ECUDA;                                                                                         \
    (void)c_

namespace qmc {
// One bounded wait that nothing satisfies, written with the helpers the decode and matvec kernels wait
// with: kind 0 polls a grid-barrier counter no CTA raises; kind 1 lands one real bulk copy on an
// mbarrier (phase 0) and then waits for a phase 1 that no copy completes.  The kernel gives up after the
// wait limit, ORs its code into the error word and returns; nothing faults and the context stays usable.
__global__ void wait_selftest_kernel(int kind, const unsigned *ctr, const uint8_t *src, int *err) {
    __shared__ __align__(128) uint8_t buf[256];
    __shared__ uint64_t bar;
    if (threadIdx.x != 0) return;
    if (kind == 0) {
        if (!counter_wait(ctr, 1u)) raise_error(err, kErrFlagTimeout);
        return;
    }
    mbar_init(&bar, 1);
    fence_mbar_init();
    mbar_arrive_tx(&bar, sizeof buf);
    bulk_g2s(buf, src, sizeof buf, &bar);
    if (!mbar_wait(&bar, 0)) {  // the copy itself did not land
        raise_error(err, kErrMbarTimeout);
        return;
    }
    if (!mbar_wait(&bar, 1)) raise_error(err, kErrMbarTimeout);
}
}  // namespace qmc

extern "C" {

const char *qmc_last_error(void) { return g_err; }

int qmc_device_count(int *count) {
    if (!count) return set_error(QMC_EINVAL, "null count");
    QMC_CUDA(cudaGetDeviceCount(count));
    return QMC_OK;
}

int qmc_set_device(int device) {
    QMC_CUDA(cudaSetDevice(device));
    return ctx() ? QMC_OK : QMC_ECUDA;
}

int qmc_get_device(int *device) {
    QMC_CUDA(cudaGetDevice(device));
    return QMC_OK;
}

int qmc_stream(void **stream) {
    CTX_OR_FAIL();
    *stream = (void *)c_->stream;
    return QMC_OK;
}

int qmc_sync(void) {
    CTX_OR_FAIL();
    QMC_CUDA(cudaStreamSynchronize(c_->stream));
    return qmc_check_device_error();
}

int qmc_check_device_error(void) {
    CTX_OR_FAIL();
    int v = 0;
    QMC_CUDA(cudaMemcpy(&v, c_->err, sizeof v, cudaMemcpyDeviceToHost));
    if (v) {
        QMC_CUDA(cudaMemset(c_->err, 0, sizeof(int)));
        if (v & kErrBadState)
            return set_error(QMC_EINVAL, "a decode step found its device position or token out of range (code %d)", v);
        return set_error(QMC_ETIMEOUT, "a device-side bounded wait expired (code %d)", v);
    }
    return QMC_OK;
}

int qmc_wait_selftest(int kind, float *ms) {
    CTX_OR_FAIL();
    if (kind != 0 && kind != 1) return set_error(QMC_EINVAL, "wait_selftest: kind %d is not 0 or 1", kind);
    uint8_t *buf = nullptr;  // [0, 4): the counter (0); [256, 512): the copy's source
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    int rc = QMC_OK;
    cudaError_t e = cudaMalloc(&buf, 512);
    if (e == cudaSuccess) e = cudaMemsetAsync(buf, 0, 512, c_->stream);
    if (e == cudaSuccess) e = cudaEventCreate(&e0);
    if (e == cudaSuccess) e = cudaEventCreate(&e1);
    if (e == cudaSuccess) e = cudaEventRecord(e0, c_->stream);
    if (e == cudaSuccess) {
        wait_selftest_kernel<<<1, 32, 0, c_->stream>>>(kind, (const unsigned *)buf, buf + 256, c_->err);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaEventRecord(e1, c_->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c_->stream);
    float t = 0.0f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&t, e0, e1);
    if (e != cudaSuccess) rc = cuda_fail(e, "wait_selftest");
    else if (ms) *ms = t;
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (buf) cudaFree(buf);
    return rc;
}

int qmc_host_register(const void *ptr, size_t bytes) {
    if (!ptr || !bytes) return set_error(QMC_EINVAL, "host_register: null range");
    // read-only and portable: a loader's read-only file mapping qualifies, every device may DMA from it
    QMC_CUDA(cudaHostRegister(const_cast<void *>(ptr), bytes, cudaHostRegisterReadOnly | cudaHostRegisterPortable));
    return QMC_OK;
}

int qmc_host_unregister(const void *ptr) {
    if (!ptr) return set_error(QMC_EINVAL, "host_unregister: null pointer");
    QMC_CUDA(cudaHostUnregister(const_cast<void *>(ptr)));
    return QMC_OK;
}

int qmc_malloc(void **dptr, size_t bytes) {
    CTX_OR_FAIL();
    QMC_CUDA(cudaMalloc(dptr, bytes ? bytes : 1));
    return QMC_OK;
}
int qmc_free(void *dptr) {
    QMC_CUDA(cudaFree(dptr));
    return QMC_OK;
}
int qmc_memcpy_h2d(void *dst, const void *src, size_t bytes, void *stream) {
    CTX_OR_FAIL();
    QMC_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, pick_stream(stream)));
    return QMC_OK;
}
int qmc_memcpy_d2h(void *dst, const void *src, size_t bytes, void *stream) {
    CTX_OR_FAIL();
    QMC_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, pick_stream(stream)));
    return QMC_OK;
}
int qmc_host_alloc(void **hptr, size_t bytes) {
    QMC_CUDA(cudaMallocHost(hptr, bytes ? bytes : 1));
    return QMC_OK;
}
int qmc_host_free(void *hptr) {
    QMC_CUDA(cudaFreeHost(hptr));
    return QMC_OK;
}

int qmc_quantize_rows(int dtype, const float *x, void *out, int64_t rows, int64_t cols, void *stream) {
    CTX_OR_FAIL();
    return launch_quantize_rows(dtype, x, out, rows, cols, pick_stream(stream));
}

int qmc_dequantize_rows(int dtype, const void *in, float *y, int64_t rows, int64_t cols, void *stream) {
    CTX_OR_FAIL();
    if (dtype != QMC_F32 && dtype != QMC_Q8_0 && dtype != QMC_Q4_0) return set_error(QMC_EINVAL, "bad dtype");
    return launch_dequantize_rows(dtype, in, y, rows, cols, pick_stream(stream));
}

int qmc_matvec(int dtype, const void *W, int64_t rows, int64_t cols, const float *x, float *y, void *xq,
               void *stream) {
    CTX_OR_FAIL();
    if (!W || !x || !y) return set_error(QMC_EINVAL, "matvec: null pointer");
    if (rows <= 0 || cols <= 0) return QMC_OK;
    GemvArgs a;
    a.dtype = dtype;
    a.W0 = W;
    a.rows = rows;
    a.K = cols;
    a.x = x;
    a.y = y;
    a.epi = EPI_STORE;
    a.xq_out = dtype == QMC_F32 ? nullptr : xq;
    return launch_gemv(a, pick_stream(stream), false);
}

int qmc_matmul_nt(const float *A, const float *B, float *C, int64_t M, int64_t N, int64_t K, void *stream) {
    CTX_OR_FAIL();
    if (M <= 0 || N <= 0) return QMC_OK;
    if (!A || !B || !C || K < 0) return set_error(QMC_EINVAL, "matmul_nt: bad arguments");
    return launch_gemm_f32(A, B, C, M, N, K, pick_stream(stream));
}

int qmc_matmul_nt_q(int dtype, const void *W, const float *A, float *C, int64_t T, int64_t N, int64_t K,
                    void *stream) {
    CTX_OR_FAIL();
    if (T <= 0 || N <= 0) return QMC_OK;
    if (!W || !A || !C || K <= 0) return set_error(QMC_EINVAL, "matmul_nt_q: bad arguments");
    if (dtype == QMC_F32) return launch_gemm_f32(A, (const float *)W, C, T, N, K, pick_stream(stream));
    const int64_t nb = nblocks(K);
    void *scr = nullptr;
    const size_t qbytes = (size_t)(T * nb * 32 + 255) / 256 * 256;
    int rc = ensure_scratch(c_, qbytes + (size_t)T * nb * 4, &scr);
    if (rc) return rc;
    int8_t *aq = (int8_t *)scr;
    float *ad = (float *)((uint8_t *)scr + qbytes);
    cudaStream_t s = pick_stream(stream);
    if ((rc = launch_quantize_act(A, T, K, aq, ad, s))) return rc;
    return launch_matmul_q(dtype, W, aq, ad, C, T, N, K, s);
}

int64_t qmc_split_row_bytes(int dtype, int64_t K) {
    if ((dtype != QMC_Q8_0 && dtype != QMC_Q4_0) || K <= 0) return 0;
    return split_row_bytes(dtype, K);
}

int qmc_repack_split(int dtype, const void *W, int64_t rows, int64_t K, void *dst, void *stream) {
    CTX_OR_FAIL();
    if (!W || !dst || K <= 0 || rows < 0) return set_error(QMC_EINVAL, "repack_split: bad arguments");
    return launch_repack_split(dtype, W, rows, K, dst, split_row_bytes(dtype, K), pick_stream(stream));
}

int qmc_matmul_split_q(int dtype, const void *Wsplit, const float *A, float *C, int64_t T, int64_t N, int64_t K,
                       void *stream) {
    CTX_OR_FAIL();
    if (T <= 0 || N <= 0) return QMC_OK;
    if (!Wsplit || !A || !C || K <= 0) return set_error(QMC_EINVAL, "matmul_split_q: bad arguments");
    if (dtype != QMC_Q8_0 && dtype != QMC_Q4_0) return set_error(QMC_EINVAL, "matmul_split_q: bad dtype %d", dtype);
    const int64_t nb = nblocks(K), ld = matmul_tc_scale_ld(T);
    void *scr = nullptr;
    const size_t qbytes = (size_t)(T * nb * 32 + 255) / 256 * 256, dbytes = (size_t)(T * nb * 4 + 255) / 256 * 256;
    int rc = ensure_scratch(c_, qbytes + dbytes + (size_t)(nb * ld * 4), &scr);
    if (rc) return rc;
    int8_t *aq = (int8_t *)scr;
    float *ad = (float *)((uint8_t *)scr + qbytes), *adT = (float *)((uint8_t *)scr + qbytes + dbytes);
    cudaStream_t s = pick_stream(stream);
    if ((rc = launch_quantize_act(A, T, K, aq, ad, s, adT, ld))) return rc;
    return launch_matmul_q_tc(dtype, Wsplit, split_row_bytes(dtype, K), aq, adT, C, nullptr, T, N, K, c_->err, s);
}

}  // extern "C"

// ---------------------------------------------------------------- allocation-free prefill
// qmc_matmul_nt_q needs T * ceil(K/32) * 36 bytes of device scratch for the Q8_0-quantized rows of A
// and grows a cudaMalloc'd buffer for them.  The variant below takes that scratch from one fixed array
// in the library's static device memory instead, for callers that must not allocate (see the header).
namespace {
constexpr size_t kNoAllocScratchBytes = (size_t)8 << 20;  // 8 MiB on every GPU that loads the library
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
void *g_noalloc_addr[64];
std::mutex g_noalloc_mu;

// device address of g_noalloc_scratch on the current device, looked up once per device (the array's
// host-side name is only a stand-in; a kernel must be given this address)
int noalloc_scratch(void **out) {
    int d = 0;
    QMC_CUDA(cudaGetDevice(&d));
    if (d < 0 || d >= 64) return set_error(QMC_EINVAL, "device %d out of range", d);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_addr[d]) {
        void *p = nullptr;
        QMC_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
        g_noalloc_addr[d] = p;
    }
    *out = g_noalloc_addr[d];
    return QMC_OK;
}
}  // namespace

extern "C" {

int qmc_matmul_nt_q_noalloc(int dtype, const void *W, const float *A, float *C, int64_t T, int64_t N, int64_t K,
                            void *stream) {
    if (T <= 0 || N <= 0) return QMC_OK;
    if (!W || !A || !C || K <= 0) return set_error(QMC_EINVAL, "matmul_nt_q_noalloc: bad arguments");
    cudaStream_t s = (cudaStream_t)stream;  // NULL: the CUDA default stream (no library stream is created)
    if (dtype == QMC_F32) return launch_gemm_f32(A, (const float *)W, C, T, N, K, s);
    if (dtype != QMC_Q8_0 && dtype != QMC_Q4_0) return set_error(QMC_EINVAL, "matmul_nt_q_noalloc: bad dtype %d", dtype);
    const int64_t nb = nblocks(K);
    // T * nb * 36 must fit the array; compare by division first, so a huge T or K cannot wrap the
    // products below into a small value that passes
    const bool too_big = T > (int64_t)(kNoAllocScratchBytes / 36) / nb;
    const size_t qbytes = too_big ? 0 : (size_t)(T * nb * 32 + 255) / 256 * 256;
    const size_t need = too_big ? SIZE_MAX : qbytes + (size_t)T * nb * 4;
    if (need > kNoAllocScratchBytes)
        return set_error(QMC_EINVAL,
                         "matmul_nt_q_noalloc: T=%lld x K=%lld needs %zu bytes of scratch, above the fixed %zu "
                         "(T * ceil(K/32) * 36 must stay within it; split T or use qmc_matmul_nt_q)",
                         (long long)T, (long long)K, need, kNoAllocScratchBytes);
    void *scr = nullptr;
    int rc = noalloc_scratch(&scr);
    if (rc) return rc;
    int8_t *aq = (int8_t *)scr;
    float *ad = (float *)((uint8_t *)scr + qbytes);
    if ((rc = launch_quantize_act(A, T, K, aq, ad, s))) return rc;  // overwrites every byte it reads later
    return launch_matmul_q(dtype, W, aq, ad, C, T, N, K, s);
}

int qmc_rmsnorm(float *out, const float *x, const float *w, int64_t n, float eps, void *stream) {
    CTX_OR_FAIL();
    if (n <= 0) return QMC_OK;
    return launch_rmsnorm(out, x, w, n, eps, pick_stream(stream));
}

int qmc_softmax(float *x, int64_t n, void *stream) {
    CTX_OR_FAIL();
    return launch_softmax(x, n, pick_stream(stream));
}

int qmc_rope(float *v, int64_t n_heads, int64_t head_dim, int64_t pos, float theta, void *stream) {
    CTX_OR_FAIL();
    if (head_dim / 2 > kMaxRopeHalf) return set_error(QMC_EINVAL, "rope: head_dim > %d", 2 * kMaxRopeHalf);
    RopeRow cs;
    rope_row_host(pos, head_dim, theta, cs.v);
    return launch_rope(v, n_heads, head_dim, cs, pick_stream(stream));
}

int qmc_swiglu(float *gate, const float *up, int64_t n, void *stream) {
    CTX_OR_FAIL();
    return launch_swiglu(gate, up, n, pick_stream(stream));
}

int qmc_argmax(const float *x, int32_t n, int32_t *out_index, void *stream) {
    CTX_OR_FAIL();
    if (n <= 0 || !x || !out_index) return set_error(QMC_EINVAL, "argmax: bad arguments");
    return launch_argmax(x, n, out_index, pick_stream(stream), false);
}

int qmc_dot(int dtype, const void *w, const void *xq, int64_t n, float *out, void *stream) {
    CTX_OR_FAIL();
    if (dtype != QMC_F32 && dtype != QMC_Q8_0 && dtype != QMC_Q4_0) return set_error(QMC_EINVAL, "bad dtype");
    return launch_dot(dtype, w, xq, n, out, pick_stream(stream));
}

}  // extern "C"
