// tvq_abi.cu -- the exported C ABI (include/tvq.h): argument checks with the
// reference's error behaviour (ValueError -> TVQ_ERR_SIZE), host-buffer
// staging for the tvq_* entry points, and the asynchronous tvq_dev_* forms.
#include <cstring>
#include <cstdlib>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "tvq_common.cuh"
#include "tvq_kernels.h"

namespace tvq {

// ---------------------------------------------------------------- errors
namespace {
thread_local std::string g_last_error;
}

void set_error(int code, const std::string& msg) { g_last_error = "tvq error " + std::to_string(code) + ": " + msg; }

int cuda_fail(cudaError_t e, const char* what) {
    set_error(TVQ_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
    return TVQ_ERR_CUDA;
}

// ---------------------------------------------------------------- devices
namespace {
constexpr int kMaxDev = 64;
DeviceState g_dev[kMaxDev];
std::mutex g_dev_mu;

// Grow-only device scratch for the host-buffer entry points, one pool and
// one stream per device; the pool mutex serialises host-buffer calls.
struct HostCtx {
    std::mutex mu;
    cudaStream_t stream = nullptr;
    std::vector<std::pair<void*, size_t>> slots;
};
HostCtx g_host[kMaxDev];
}  // namespace

bool pdl_enabled() {
    static const bool on = [] {
        const char* e = getenv("TVQ_PDL");
        return !(e && atoi(e) == 0);
    }();
    return on;
}

DeviceState* device_state(int* rc) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) { *rc = cuda_fail(e, "cudaGetDevice"); return nullptr; }
    if (dev < 0 || dev >= kMaxDev) { set_error(TVQ_ERR_UNSUPPORTED, "device ordinal too large"); *rc = TVQ_ERR_UNSUPPORTED; return nullptr; }
    DeviceState& d = g_dev[dev];
    if (d.sm_count == 0) {
        std::lock_guard<std::mutex> lk(g_dev_mu);
        if (d.sm_count == 0) {
            int sms = 0, maj = 0, mnr = 0;
            if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess ||
                (e = cudaDeviceGetAttribute(&maj, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess ||
                (e = cudaDeviceGetAttribute(&mnr, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess) {
                *rc = cuda_fail(e, "cudaDeviceGetAttribute");
                return nullptr;
            }
            int* err = nullptr;
            if ((e = cudaMalloc(&err, sizeof(int))) != cudaSuccess || (e = cudaMemset(err, 0, sizeof(int))) != cudaSuccess) {
                *rc = cuda_fail(e, "device error word");
                return nullptr;
            }
            // per-call scratch (cudaMallocAsync) stays in the device's default
            // pool between calls, up to 1 GiB, instead of being unmapped at
            // every synchronisation
            cudaMemPool_t pool = nullptr;
            if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
                uint64_t keep = 1ull << 30;
                cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
            }
            d.cc_major = maj;
            d.cc_minor = mnr;
            d.d_error = err;
            d.sm_count = sms;  // published last
        }
    }
    *rc = TVQ_OK;
    return &d;
}

int check_device_error(cudaStream_t st) {
    int rc = 0;
    DeviceState* d = device_state(&rc);
    if (!d) return rc;
    TVQ_CUDA(cudaStreamSynchronize(st));
    int h = 0;
    TVQ_CUDA(cudaMemcpy(&h, d->d_error, sizeof(int), cudaMemcpyDeviceToHost));
    if (h != 0) {
        TVQ_CUDA(cudaMemset(d->d_error, 0, sizeof(int)));
        if (h == DEVERR_FIX_FULL) {
            set_error(TVQ_ERR_SIZE, "more undecided int8 attention rows than the exact fix-up lists hold");
            return TVQ_ERR_SIZE;
        }
        if (h == DEVERR_BAD_INDEX) {
            set_error(TVQ_ERR_INVALID, "index out of range (a permutation entry outside [0, cols))");
            return TVQ_ERR_INVALID;
        }
        set_error(TVQ_ERR_TIMEOUT, "device-side wait timed out (code " + std::to_string(h) + ")");
        return TVQ_ERR_TIMEOUT;
    }
    return TVQ_OK;
}

namespace {

// RAII context of one host-buffer call.
struct Host {
    HostCtx* ctx = nullptr;
    std::unique_lock<std::mutex> lk;
    int rc = TVQ_OK;
    Host() {
        DeviceState* d = device_state(&rc);
        if (!d) return;
        int dev = 0;
        cudaGetDevice(&dev);
        ctx = &g_host[dev];
        lk = std::unique_lock<std::mutex>(ctx->mu);
        if (!ctx->stream) {
            cudaError_t e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
            if (e != cudaSuccess) rc = cuda_fail(e, "cudaStreamCreate");
        }
    }
    cudaStream_t st() const { return ctx->stream; }
    // device buffer of at least `bytes` in slot i (contents not preserved)
    void* buf(size_t i, size_t bytes) {
        if (rc) return nullptr;
        if (ctx->slots.size() <= i) ctx->slots.resize(i + 1, {nullptr, 0});
        auto& s = ctx->slots[i];
        if (s.second < bytes || !s.first) {
            if (s.first) cudaFree(s.first);
            s.first = nullptr;
            s.second = 0;
            size_t want = bytes < 256 ? 256 : bytes;
            cudaError_t e = cudaMalloc(&s.first, want);
            if (e != cudaSuccess) { rc = cuda_fail(e, "cudaMalloc (scratch)"); return nullptr; }
            s.second = want;
        }
        return s.first;
    }
    int h2d(void* d, const void* h, size_t bytes) {
        if (rc || bytes == 0) return rc;
        cudaError_t e = cudaMemcpyAsync(d, h, bytes, cudaMemcpyHostToDevice, st());
        if (e != cudaSuccess) rc = cuda_fail(e, "cudaMemcpyAsync H2D");
        return rc;
    }
    int d2h(void* h, const void* d, size_t bytes) {
        if (rc || bytes == 0) return rc;
        cudaError_t e = cudaMemcpyAsync(h, d, bytes, cudaMemcpyDeviceToHost, st());
        if (e != cudaSuccess) rc = cuda_fail(e, "cudaMemcpyAsync D2H");
        return rc;
    }
    int finish() {
        if (rc) return rc;
        return check_device_error(st());
    }
};

#define TVQ_TRY try {
#define TVQ_CATCH                                                              \
    }                                                                          \
    catch (const std::bad_alloc&) {                                            \
        ::tvq::set_error(TVQ_ERR_CUDA, "host allocation failed");              \
        return TVQ_ERR_CUDA;                                                   \
    }                                                                          \
    catch (...) {                                                              \
        ::tvq::set_error(TVQ_ERR_INVALID, "unexpected exception");             \
        return TVQ_ERR_INVALID;                                                \
    }

#define HOST_BEGIN          \
    ::tvq::Host H;          \
    if (H.rc) return H.rc;

#define STEP(expr)                  \
    do {                            \
        int r__ = (expr);           \
        if (r__) return r__;        \
    } while (0)

template <typename T>
T* dev(Host& H, size_t slot, size_t count) {
    return static_cast<T*>(H.buf(slot, count * sizeof(T)));
}

// shared tail of the host GEMM entry points
int host_gemm(int kind, const void* A, const void* W, size_t elem_bytes_ignored, const float* bias, int64_t n_bias,
              float* Y, int64_t m, int64_t n, int64_t k, float scale_a, const float* scales_w, int64_t n_scales,
              int per_channel, int act) {
    (void)elem_bytes_ignored;
    TVQ_CHECK(m >= 0 && n >= 0 && k >= 0 && n_bias >= 0, TVQ_ERR_INVALID, "negative size");
    if (m == 0 || n == 0) return TVQ_OK;
    TVQ_CHECK(Y && (k == 0 || (A && W)), TVQ_ERR_INVALID, "null buffer");
    TVQ_CHECK(n_bias == 0 || n_bias >= n, TVQ_ERR_SIZE, "bias smaller than N");
    TVQ_CHECK(n_bias == 0 || bias, TVQ_ERR_INVALID, "null bias");
    if (per_channel) TVQ_CHECK(scales_w && n_scales >= n, TVQ_ERR_SIZE, "scales_w smaller than N");
    HOST_BEGIN
    const int64_t kp = (k + 15) / 16 * 16;  // TMA row pitch: pad K with zeros
    uint8_t* dA = dev<uint8_t>(H, 0, static_cast<size_t>(m * kp));
    uint8_t* dW = dev<uint8_t>(H, 1, static_cast<size_t>(n * kp));
    float* dY = dev<float>(H, 2, static_cast<size_t>(m * n));
    float* dB = dev<float>(H, 3, static_cast<size_t>(n_bias > 0 ? n : 1));
    float* dS = dev<float>(H, 4, static_cast<size_t>(n + 4));  // scale_a, pad, scales_w at +16 B
    if (H.rc) return H.rc;
    if (kp == k) {
        STEP(H.h2d(dA, A, static_cast<size_t>(m * k)));
        STEP(H.h2d(dW, W, static_cast<size_t>(n * k)));
    } else if (k > 0) {
        TVQ_CUDA(cudaMemsetAsync(dA, 0, static_cast<size_t>(m * kp), H.st()));
        TVQ_CUDA(cudaMemsetAsync(dW, 0, static_cast<size_t>(n * kp), H.st()));
        TVQ_CUDA(cudaMemcpy2DAsync(dA, kp, A, k, k, m, cudaMemcpyHostToDevice, H.st()));
        TVQ_CUDA(cudaMemcpy2DAsync(dW, kp, W, k, k, n, cudaMemcpyHostToDevice, H.st()));
    }
    if (n_bias > 0) STEP(H.h2d(dB, bias, static_cast<size_t>(n) * 4));
    STEP(H.h2d(dS, &scale_a, 4));
    if (per_channel) STEP(H.h2d(dS + 4, scales_w, static_cast<size_t>(n) * 4));
    else STEP(H.h2d(dS + 4, scales_w, 4));
    GemmArgs g;
    g.kind = kind;
    g.A = dA;
    g.W = dW;
    g.bias = n_bias > 0 ? dB : nullptr;
    g.Y = dY;
    g.m = m;
    g.n = n;
    g.k = kp;
    g.scale_a = dS;
    g.scales_w = dS + 4;
    g.per_channel = per_channel;
    g.act = act;
    STEP(launch_gemm(g, H.st()));
    STEP(H.d2h(Y, dY, static_cast<size_t>(m * n) * 4));
    return H.finish();
}

// matmul_int8_asymmetric on host buffers: the INT8 GEMM with its zero-point
// epilogue, the row sums of A and W computed on the device first
int host_gemm_asym(const int8_t* A, const int8_t* W, const float* bias, int64_t n_bias, float* Y, int64_t m, int64_t n,
                   int64_t k, float scale_a, int64_t zp_a, float scale_w, int64_t zp_w) {
    TVQ_CHECK(m >= 0 && n >= 0 && k >= 0 && n_bias >= 0, TVQ_ERR_INVALID, "negative size");
    if (m == 0 || n == 0) return TVQ_OK;
    TVQ_CHECK(Y && (k == 0 || (A && W)), TVQ_ERR_INVALID, "null buffer");
    TVQ_CHECK(n_bias == 0 || n_bias >= n, TVQ_ERR_SIZE, "bias smaller than N");
    TVQ_CHECK(n_bias == 0 || bias, TVQ_ERR_INVALID, "null bias");
    HOST_BEGIN
    const int64_t kp = (k + 15) / 16 * 16;
    uint8_t* dA = dev<uint8_t>(H, 0, static_cast<size_t>(std::max<int64_t>(m * kp, 1)));
    uint8_t* dW = dev<uint8_t>(H, 1, static_cast<size_t>(std::max<int64_t>(n * kp, 1)));
    float* dY = dev<float>(H, 2, static_cast<size_t>(m * n));
    float* dB = dev<float>(H, 3, static_cast<size_t>(n_bias > 0 ? n : 1));
    float* dS = dev<float>(H, 4, 8);
    int* dR = dev<int>(H, 5, static_cast<size_t>(m + n));
    if (H.rc) return H.rc;
    if (kp == k) {
        STEP(H.h2d(dA, A, static_cast<size_t>(m * k)));
        STEP(H.h2d(dW, W, static_cast<size_t>(n * k)));
    } else if (k > 0) {
        TVQ_CUDA(cudaMemsetAsync(dA, 0, static_cast<size_t>(m * kp), H.st()));
        TVQ_CUDA(cudaMemsetAsync(dW, 0, static_cast<size_t>(n * kp), H.st()));
        TVQ_CUDA(cudaMemcpy2DAsync(dA, kp, A, k, k, m, cudaMemcpyHostToDevice, H.st()));
        TVQ_CUDA(cudaMemcpy2DAsync(dW, kp, W, k, k, n, cudaMemcpyHostToDevice, H.st()));
    }
    if (n_bias > 0) STEP(H.h2d(dB, bias, static_cast<size_t>(n) * 4));
    const float sc[8] = {scale_a, 0.0f, 0.0f, 0.0f, scale_w, 0.0f, 0.0f, 0.0f};
    STEP(H.h2d(dS, sc, sizeof(sc)));
    STEP(launch_row_sums_i8(reinterpret_cast<const int8_t*>(dA), m, kp, dR, H.st()));
    STEP(launch_row_sums_i8(reinterpret_cast<const int8_t*>(dW), n, kp, dR + m, H.st()));
    GemmArgs g;
    g.kind = GEMM_I8;
    g.A = dA;
    g.W = dW;
    g.bias = n_bias > 0 ? dB : nullptr;
    g.Y = dY;
    g.m = m;
    g.n = n;
    g.k = kp;
    g.scale_a = dS;
    g.scales_w = dS + 4;
    g.per_channel = 0;
    g.zp_rows = dR;
    g.zp_cols = dR + m;
    g.zp_a = zp_a;
    g.zp_w = zp_w;
    g.zp_k = k;
    STEP(launch_gemm(g, H.st()));
    STEP(H.d2h(Y, dY, static_cast<size_t>(m * n) * 4));
    return H.finish();
}

// matmul_fp16 on host buffers: fp16 A [m, k] and W [n, k] (bit patterns), k
// padded with zeros to a multiple of 8 (the TMA row pitch)
int host_gemm_f16(const uint16_t* A, const uint16_t* W, const float* bias, int64_t n_bias, float* Y, int64_t m,
                  int64_t n, int64_t k) {
    TVQ_CHECK(m >= 0 && n >= 0 && k >= 0 && n_bias >= 0, TVQ_ERR_INVALID, "negative size");
    if (m == 0 || n == 0) return TVQ_OK;
    TVQ_CHECK(Y && (k == 0 || (A && W)), TVQ_ERR_INVALID, "null buffer");
    TVQ_CHECK(n_bias == 0 || n_bias >= n, TVQ_ERR_SIZE, "bias smaller than N");
    TVQ_CHECK(n_bias == 0 || bias, TVQ_ERR_INVALID, "null bias");
    HOST_BEGIN
    const int64_t kp = (k + 7) / 8 * 8;
    uint16_t* dA = dev<uint16_t>(H, 0, static_cast<size_t>(std::max<int64_t>(m * kp, 1)));
    uint16_t* dW = dev<uint16_t>(H, 1, static_cast<size_t>(std::max<int64_t>(n * kp, 1)));
    float* dY = dev<float>(H, 2, static_cast<size_t>(m * n));
    float* dB = dev<float>(H, 3, static_cast<size_t>(n_bias > 0 ? n : 1));
    if (H.rc) return H.rc;
    if (kp == k) {
        STEP(H.h2d(dA, A, static_cast<size_t>(m * k) * 2));
        STEP(H.h2d(dW, W, static_cast<size_t>(n * k) * 2));
    } else if (k > 0) {
        TVQ_CUDA(cudaMemsetAsync(dA, 0, static_cast<size_t>(m * kp) * 2, H.st()));
        TVQ_CUDA(cudaMemsetAsync(dW, 0, static_cast<size_t>(n * kp) * 2, H.st()));
        TVQ_CUDA(cudaMemcpy2DAsync(dA, kp * 2, A, k * 2, k * 2, m, cudaMemcpyHostToDevice, H.st()));
        TVQ_CUDA(cudaMemcpy2DAsync(dW, kp * 2, W, k * 2, k * 2, n, cudaMemcpyHostToDevice, H.st()));
    }
    if (n_bias > 0) STEP(H.h2d(dB, bias, static_cast<size_t>(n) * 4));
    GemmArgs g;
    g.kind = GEMM_F16X3;  // without low parts: the plain fp16 product
    g.A = dA;
    g.W = dW;
    g.bias = n_bias > 0 ? dB : nullptr;
    g.Y = dY;
    g.m = m;
    g.n = n;
    g.k = kp;
    STEP(launch_gemm(g, H.st()));
    STEP(H.d2h(Y, dY, static_cast<size_t>(m * n) * 4));
    return H.finish();
}

// A bounded wait on an mbarrier that nothing ever arrives at: the
// failure-detection path of every tensor-core kernel (record a code in the
// device error word, return), made to run out on purpose with a short
// limit.  The CTA exits normally, so the context stays usable.
__global__ void wait_selftest_kernel(int* err, uint64_t limit_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    __syncwarp();
    if (threadIdx.x == 0) mbar_wait_for(&bar, 0, err, DEVERR_TIMEOUT_TEST, limit_ns);
    __syncwarp();
}

}  // namespace
}  // namespace tvq

using namespace tvq;

extern "C" {

int tvq_version(void) { return 10000; }

int tvq_last_error(char* buf, int64_t len) {
    if (!buf || len <= 0) return TVQ_ERR_INVALID;
    const std::string& s = g_last_error;
    const size_t n = std::min<size_t>(s.size(), static_cast<size_t>(len - 1));
    memcpy(buf, s.data(), n);
    buf[n] = 0;
    return TVQ_OK;
}

int tvq_device_count(int* n) {
    TVQ_CHECK(n, TVQ_ERR_INVALID, "null out pointer");
    int c = 0;
    cudaError_t e = cudaGetDeviceCount(&c);
    if (e != cudaSuccess) { *n = 0; return cuda_fail(e, "cudaGetDeviceCount"); }
    *n = c;
    return TVQ_OK;
}

int tvq_device_error(void* stream) { return check_device_error(static_cast<cudaStream_t>(stream)); }

int tvq_selftest_wait_timeout(int64_t limit_us, void* stream) {
    TVQ_CHECK(limit_us >= 1 && limit_us <= 1000000, TVQ_ERR_INVALID, "limit must be 1 us .. 1 s");
    int rc = 0;
    DeviceState* d = device_state(&rc);
    if (!d) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    wait_selftest_kernel<<<1, 32, 0, st>>>(d->d_error, static_cast<uint64_t>(limit_us) * 1000u);
    TVQ_CUDA(cudaGetLastError());
    return check_device_error(st);
}

// ================================================================ host: engine.tkv

static int calibrate_common(const float* const* batches, const int64_t* sizes, int64_t nb, int symmetric,
                            float* scale, int64_t* zp, float* mn, float* mx) {
    TVQ_CHECK(nb >= 0 && batches && sizes, TVQ_ERR_INVALID, "null batch list");
    int64_t total = 0;
    for (int64_t b = 0; b < nb; b++) {
        TVQ_CHECK(sizes[b] >= 0 && (sizes[b] == 0 || batches[b]), TVQ_ERR_INVALID, "bad batch");
        total += sizes[b];
    }
    if (total == 0) {  // _quant_identity, engine.tkv:9-10
        if (scale) *scale = 1.0f;
        if (zp) *zp = 0;
        if (mn) *mn = -3.4028234663852886e38f;
        if (mx) *mx = 3.4028234663852886e38f;
        return TVQ_OK;
    }
    TVQ_TRY
    HOST_BEGIN
    int64_t biggest = 0;
    for (int64_t b = 0; b < nb; b++) biggest = std::max(biggest, sizes[b]);
    float* dx = dev<float>(H, 0, static_cast<size_t>(biggest));
    uint32_t* dmm = dev<uint32_t>(H, 1, 2);
    float* dfirst = dev<float>(H, 2, 1);
    float* dp = dev<float>(H, 3, 4);
    if (H.rc) return H.rc;
    STEP(launch_minmax_reset(dmm, H.st()));
    bool first = true;
    for (int64_t b = 0; b < nb; b++) {
        if (sizes[b] == 0) continue;
        STEP(H.h2d(dx, batches[b], static_cast<size_t>(sizes[b]) * 4));
        STEP(launch_minmax_accumulate(dx, sizes[b], dmm, first ? dfirst : nullptr, H.st()));
        first = false;
    }
    STEP(launch_minmax_finalize(dmm, dfirst, symmetric, dp, H.st()));
    float hp[4];
    STEP(H.d2h(hp, dp, sizeof(hp)));
    STEP(H.finish());
    if (scale) *scale = hp[0];
    if (zp) *zp = static_cast<int64_t>(hp[1]);
    if (mn) *mn = hp[2];
    if (mx) *mx = hp[3];
    return TVQ_OK;
    TVQ_CATCH
}

int tvq_calibrate_minmax(const float* data, int64_t n, int symmetric, float* scale, int64_t* zero_point,
                         float* min_val, float* max_val) {
    TVQ_CHECK(n >= 0 && (n == 0 || data), TVQ_ERR_INVALID, "null data");
    const float* b[1] = {data};
    int64_t s[1] = {n};
    return calibrate_common(b, s, 1, symmetric, scale, zero_point, min_val, max_val);
}

int tvq_calibrate_minmax_batches(const float* const* batches, const int64_t* sizes, int64_t n_batches, int symmetric,
                                 float* scale, int64_t* zero_point, float* min_val, float* max_val) {
    return calibrate_common(batches, sizes, n_batches, symmetric, scale, zero_point, min_val, max_val);
}

int tvq_calibrate_per_channel_minmax(const float* data, int64_t len, int64_t rows, int64_t cols, float* scales,
                                     int64_t n_scales) {
    // engine.tkv:203-206
    TVQ_CHECK(rows > 0 && cols > 0, TVQ_ERR_INVALID, "rows/cols must be > 0");
    TVQ_CHECK(len >= rows * cols, TVQ_ERR_SIZE, "data smaller than rows*cols");
    TVQ_CHECK(data && scales, TVQ_ERR_INVALID, "null buffer");
    TVQ_CHECK(n_scales >= rows, TVQ_ERR_SIZE, "scales smaller than rows");
    TVQ_TRY
    HOST_BEGIN
    float* dx = dev<float>(H, 0, static_cast<size_t>(rows * cols));
    int8_t* dq = dev<int8_t>(H, 1, static_cast<size_t>(rows * cols));
    float* ds = dev<float>(H, 2, static_cast<size_t>(rows));
    if (H.rc) return H.rc;
    STEP(H.h2d(dx, data, static_cast<size_t>(rows * cols) * 4));
    STEP(launch_rowwise(0, dx, dq, ds, rows, cols, H.st()));
    STEP(H.d2h(scales, ds, static_cast<size_t>(rows) * 4));
    return H.finish();
    TVQ_CATCH
}

int tvq_calibrate_per_channel_params(const float* data, int64_t len, int64_t rows, int64_t cols, int symmetric,
                                     float* scales, int64_t* zero_points, float* min_vals, float* max_vals,
                                     int64_t n) {
    // engine.tkv:203-206
    TVQ_CHECK(rows > 0 && cols > 0, TVQ_ERR_INVALID, "rows/cols must be > 0");
    TVQ_CHECK(len >= rows * cols, TVQ_ERR_SIZE, "data smaller than rows*cols");
    TVQ_CHECK(data && scales && zero_points && min_vals && max_vals, TVQ_ERR_INVALID, "null buffer");
    TVQ_CHECK(n >= rows, TVQ_ERR_SIZE, "output lists smaller than rows");
    TVQ_TRY
    HOST_BEGIN
    float* dx = dev<float>(H, 0, static_cast<size_t>(rows * cols));
    float* dp = dev<float>(H, 1, static_cast<size_t>(rows) * 5 + 2);  // scale, min, max, then i64 zero points
    if (H.rc) return H.rc;
    int64_t* dz = reinterpret_cast<int64_t*>(dp + 3 * rows + (rows & 1));
    STEP(H.h2d(dx, data, static_cast<size_t>(rows * cols) * 4));
    STEP(launch_rowwise_params(dx, rows, cols, symmetric ? 1 : 0, dp, dz, dp + rows, dp + 2 * rows, H.st()));
    STEP(H.d2h(scales, dp, static_cast<size_t>(rows) * 4));
    STEP(H.d2h(min_vals, dp + rows, static_cast<size_t>(rows) * 4));
    STEP(H.d2h(max_vals, dp + 2 * rows, static_cast<size_t>(rows) * 4));
    STEP(H.d2h(zero_points, dz, static_cast<size_t>(rows) * 8));
    return H.finish();
    TVQ_CATCH
}

int tvq_quantize_int8_symmetric(const float* src, int64_t n, int8_t* dst, int64_t dst_len, float scale) {
    TVQ_CHECK(n >= 0 && dst_len >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(dst_len >= n, TVQ_ERR_SIZE, "dst too small");  // engine.tkv:217-218
    if (n == 0) return TVQ_OK;
    TVQ_CHECK(src && dst, TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    HOST_BEGIN
    float* dx = dev<float>(H, 0, static_cast<size_t>(n));
    int8_t* dq = dev<int8_t>(H, 1, static_cast<size_t>(n));
    float* ds = dev<float>(H, 2, 1);
    if (H.rc) return H.rc;
    STEP(H.h2d(dx, src, static_cast<size_t>(n) * 4));
    STEP(H.h2d(ds, &scale, 4));
    STEP(launch_quantize_i8(dx, dq, n, ds, H.st()));
    STEP(H.d2h(dst, dq, static_cast<size_t>(n)));
    return H.finish();
    TVQ_CATCH
}

int tvq_dequantize_int8_symmetric(const int8_t* src, int64_t n, float* dst, int64_t dst_len, float scale) {
    TVQ_CHECK(n >= 0 && dst_len >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(dst_len >= n, TVQ_ERR_SIZE, "dst too small");  // engine.tkv:230-231
    if (n == 0) return TVQ_OK;
    TVQ_CHECK(src && dst, TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    HOST_BEGIN
    int8_t* dq = dev<int8_t>(H, 0, static_cast<size_t>(n));
    float* dy = dev<float>(H, 1, static_cast<size_t>(n));
    float* ds = dev<float>(H, 2, 1);
    if (H.rc) return H.rc;
    STEP(H.h2d(dq, src, static_cast<size_t>(n)));
    STEP(H.h2d(ds, &scale, 4));
    STEP(launch_dequantize_i8(dq, dy, 1, n, ds, 0, H.st()));
    STEP(H.d2h(dst, dy, static_cast<size_t>(n) * 4));
    return H.finish();
    TVQ_CATCH
}

int tvq_quantize_int8_per_channel(const float* src, int64_t src_len, int8_t* dst, int64_t dst_len, int64_t rows,
                                  int64_t cols, const float* scales, int64_t n_scales) {
    TVQ_CHECK(rows >= 0 && cols >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(dst_len >= rows * cols && src_len >= rows * cols, TVQ_ERR_SIZE, "span too small");  // :238-239
    TVQ_CHECK(n_scales >= rows, TVQ_ERR_SIZE, "scales smaller than rows");                       // :240-241
    if (rows * cols == 0) return TVQ_OK;
    TVQ_CHECK(src && dst && scales, TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    HOST_BEGIN
    float* dx = dev<float>(H, 0, static_cast<size_t>(rows * cols));
    int8_t* dq = dev<int8_t>(H, 1, static_cast<size_t>(rows * cols));
    float* ds = dev<float>(H, 2, static_cast<size_t>(rows));
    if (H.rc) return H.rc;
    STEP(H.h2d(dx, src, static_cast<size_t>(rows * cols) * 4));
    STEP(H.h2d(ds, scales, static_cast<size_t>(rows) * 4));
    STEP(launch_rowwise(1, dx, dq, ds, rows, cols, H.st()));
    STEP(H.d2h(dst, dq, static_cast<size_t>(rows * cols)));
    return H.finish();
    TVQ_CATCH
}

int tvq_dequantize_int8_per_channel(const int8_t* src, int64_t src_len, float* dst, int64_t dst_len, int64_t rows,
                                    int64_t cols, const float* scales, int64_t n_scales) {
    TVQ_CHECK(rows >= 0 && cols >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(dst_len >= rows * cols && src_len >= rows * cols, TVQ_ERR_SIZE, "span too small");
    TVQ_CHECK(n_scales >= rows, TVQ_ERR_SIZE, "scales smaller than rows");
    if (rows * cols == 0) return TVQ_OK;
    TVQ_CHECK(src && dst && scales, TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    HOST_BEGIN
    int8_t* dq = dev<int8_t>(H, 0, static_cast<size_t>(rows * cols));
    float* dy = dev<float>(H, 1, static_cast<size_t>(rows * cols));
    float* ds = dev<float>(H, 2, static_cast<size_t>(rows));
    if (H.rc) return H.rc;
    STEP(H.h2d(dq, src, static_cast<size_t>(rows * cols)));
    STEP(H.h2d(ds, scales, static_cast<size_t>(rows) * 4));
    STEP(launch_dequantize_i8(dq, dy, rows, cols, ds, 1, H.st()));
    STEP(H.d2h(dst, dy, static_cast<size_t>(rows * cols) * 4));
    return H.finish();
    TVQ_CATCH
}

int tvq_quantize_dynamic_int8_rowwise(const float* src, int64_t src_len, int8_t* dst, int64_t dst_len, int64_t rows,
                                      int64_t cols, float* scales_out, int64_t n_scales) {
    TVQ_CHECK(rows >= 0 && cols >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(dst_len >= rows * cols && src_len >= rows * cols, TVQ_ERR_SIZE, "span too small");  // :267-268
    TVQ_CHECK(n_scales >= rows, TVQ_ERR_SIZE, "scales_out smaller than rows");                   // :269-270
    if (rows == 0) return TVQ_OK;
    TVQ_CHECK(scales_out && (cols == 0 || (src && dst)), TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    HOST_BEGIN
    float* dx = dev<float>(H, 0, static_cast<size_t>(std::max<int64_t>(rows * cols, 1)));
    int8_t* dq = dev<int8_t>(H, 1, static_cast<size_t>(std::max<int64_t>(rows * cols, 1)));
    float* ds = dev<float>(H, 2, static_cast<size_t>(rows));
    if (H.rc) return H.rc;
    if (cols == 0) {
        // am = 0 -> 1e-8 -> scale fl32(1e-8/127) for every row
        std::vector<float> s(static_cast<size_t>(rows), static_cast<float>(0.00000001 / 127.0));
        memcpy(scales_out, s.data(), s.size() * 4);
        return TVQ_OK;
    }
    STEP(H.h2d(dx, src, static_cast<size_t>(rows * cols) * 4));
    STEP(launch_rowwise(2, dx, dq, ds, rows, cols, H.st()));
    STEP(H.d2h(dst, dq, static_cast<size_t>(rows * cols)));
    STEP(H.d2h(scales_out, ds, static_cast<size_t>(rows) * 4));
    return H.finish();
    TVQ_CATCH
}

// ================================================================ host: matmul.tkv

int tvq_matmul_int8_per_channel(const int8_t* A, const int8_t* W, const float* bias, int64_t n_bias, float* Y,
                                int64_t m, int64_t n, int64_t k, float scale_a, const float* scales_w,
                                int64_t n_scales, int act) {
    TVQ_TRY
    return host_gemm(GEMM_I8, A, W, 1, bias, n_bias, Y, m, n, k, scale_a, scales_w, n_scales, 1, act);
    TVQ_CATCH
}

int tvq_matmul_int8_symmetric(const int8_t* A, const int8_t* W, const float* bias, int64_t n_bias, float* Y,
                              int64_t m, int64_t n, int64_t k, float scale_a, float scale_w, int act) {
    TVQ_TRY
    return host_gemm(GEMM_I8, A, W, 1, bias, n_bias, Y, m, n, k, scale_a, &scale_w, 1, 0, act);
    TVQ_CATCH
}

int tvq_gemm_i8_acc(const int8_t* A, const int8_t* W, int32_t* acc, int64_t m, int64_t n, int64_t k) {
    TVQ_CHECK(m >= 0 && n >= 0 && k >= 0, TVQ_ERR_INVALID, "negative size");
    if (m == 0 || n == 0) return TVQ_OK;
    TVQ_CHECK(acc && (k == 0 || (A && W)), TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    HOST_BEGIN
    const int64_t kp = (k + 15) / 16 * 16;
    uint8_t* dA = dev<uint8_t>(H, 0, static_cast<size_t>(std::max<int64_t>(m * kp, 1)));
    uint8_t* dW = dev<uint8_t>(H, 1, static_cast<size_t>(std::max<int64_t>(n * kp, 1)));
    int32_t* dC = dev<int32_t>(H, 2, static_cast<size_t>(m * n));
    float* dS = dev<float>(H, 3, 2);
    if (H.rc) return H.rc;
    if (k > 0) {
        TVQ_CUDA(cudaMemsetAsync(dA, 0, static_cast<size_t>(m * kp), H.st()));
        TVQ_CUDA(cudaMemsetAsync(dW, 0, static_cast<size_t>(n * kp), H.st()));
        TVQ_CUDA(cudaMemcpy2DAsync(dA, kp, A, k, k, m, cudaMemcpyHostToDevice, H.st()));
        TVQ_CUDA(cudaMemcpy2DAsync(dW, kp, W, k, k, n, cudaMemcpyHostToDevice, H.st()));
    }
    const float one[2] = {1.0f, 1.0f};
    STEP(H.h2d(dS, one, 8));
    GemmArgs g;
    g.kind = GEMM_I8;
    g.A = dA;
    g.W = dW;
    g.acc_out = dC;
    g.m = m;
    g.n = n;
    g.k = kp;
    g.scale_a = dS;
    g.scales_w = dS + 1;
    g.per_channel = 0;
    STEP(launch_gemm(g, H.st()));
    STEP(H.d2h(acc, dC, static_cast<size_t>(m * n) * 4));
    return H.finish();
    TVQ_CATCH
}

int tvq_quantize_fp8_e4m3(const float* src, int64_t n, uint8_t* dst, int64_t dst_len, int mode) {
    TVQ_CHECK(n >= 0 && dst_len >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(dst_len >= n, TVQ_ERR_SIZE, "dst too small");  // matmul.tkv:61-62
    TVQ_CHECK(mode == TVQ_FP8_REF || mode == TVQ_FP8_HW, TVQ_ERR_INVALID, "bad FP8 mode");
    if (n == 0) return TVQ_OK;
    TVQ_CHECK(src && dst, TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    HOST_BEGIN
    float* dx = dev<float>(H, 0, static_cast<size_t>(n));
    uint8_t* dq = dev<uint8_t>(H, 1, static_cast<size_t>(n));
    if (H.rc) return H.rc;
    STEP(H.h2d(dx, src, static_cast<size_t>(n) * 4));
    STEP(launch_fp8_encode(dx, dq, 1, n, nullptr, 0, mode, H.st()));
    STEP(H.d2h(dst, dq, static_cast<size_t>(n)));
    return H.finish();
    TVQ_CATCH
}

int tvq_quantize_fp8_e4m3_scaled(const float* src, int64_t rows, int64_t cols, uint8_t* dst, const float* scales,
                                 int64_t n_scales, int per_row, int mode) {
    TVQ_CHECK(rows >= 0 && cols >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(mode == TVQ_FP8_REF || mode == TVQ_FP8_HW, TVQ_ERR_INVALID, "bad FP8 mode");
    TVQ_CHECK(n_scales >= (per_row ? rows : 1), TVQ_ERR_SIZE, "scales smaller than rows");
    if (rows * cols == 0) return TVQ_OK;
    TVQ_CHECK(src && dst && scales, TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    HOST_BEGIN
    float* dx = dev<float>(H, 0, static_cast<size_t>(rows * cols));
    uint8_t* dq = dev<uint8_t>(H, 1, static_cast<size_t>(rows * cols));
    float* ds = dev<float>(H, 2, static_cast<size_t>(per_row ? rows : 1));
    if (H.rc) return H.rc;
    STEP(H.h2d(dx, src, static_cast<size_t>(rows * cols) * 4));
    STEP(H.h2d(ds, scales, static_cast<size_t>(per_row ? rows : 1) * 4));
    STEP(launch_fp8_encode(dx, dq, rows, cols, ds, per_row ? 2 : 1, mode, H.st()));
    STEP(H.d2h(dst, dq, static_cast<size_t>(rows * cols)));
    return H.finish();
    TVQ_CATCH
}

int tvq_dequantize_fp8_e4m3(const uint8_t* src, int64_t n, float* dst, int64_t dst_len) {
    TVQ_CHECK(n >= 0 && dst_len >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(dst_len >= n, TVQ_ERR_SIZE, "dst too small");  // matmul.tkv:69-70
    if (n == 0) return TVQ_OK;
    TVQ_CHECK(src && dst, TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    HOST_BEGIN
    uint8_t* dq = dev<uint8_t>(H, 0, static_cast<size_t>(n));
    float* dy = dev<float>(H, 1, static_cast<size_t>(n));
    if (H.rc) return H.rc;
    STEP(H.h2d(dq, src, static_cast<size_t>(n)));
    STEP(launch_fp8_decode(dq, dy, n, H.st()));
    STEP(H.d2h(dst, dy, static_cast<size_t>(n) * 4));
    return H.finish();
    TVQ_CATCH
}

int tvq_matmul_fp8_e4m3(const uint8_t* A, const uint8_t* W, const float* bias, int64_t n_bias, float* Y, int64_t m,
                        int64_t n, int64_t k, float scale_a, const float* scales_w, int act) {
    TVQ_TRY
    if (scales_w) return host_gemm(GEMM_F8, A, W, 1, bias, n_bias, Y, m, n, k, scale_a, scales_w, n, 1, act);
    const float one = 1.0f;  // unscaled reference form: acc * (scale_a * 1) + bias
    return host_gemm(GEMM_F8, A, W, 1, bias, n_bias, Y, m, n, k, scale_a, &one, 1, 0, act);
    TVQ_CATCH
}

// ---- list[i32] compatibility forms
int tvq_quantize_int8_symmetric_i32(const float* src, int64_t n, int32_t* dst, int64_t dst_len, float scale) {
    TVQ_CHECK(n >= 0 && dst_len >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(dst_len >= n, TVQ_ERR_SIZE, "dst too small");
    if (n == 0) return TVQ_OK;
    TVQ_CHECK(src && dst, TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    HOST_BEGIN
    float* dx = dev<float>(H, 0, static_cast<size_t>(n));
    int8_t* dq = dev<int8_t>(H, 1, static_cast<size_t>(n));
    float* ds = dev<float>(H, 2, 1);
    int32_t* dw = dev<int32_t>(H, 3, static_cast<size_t>(n));
    if (H.rc) return H.rc;
    STEP(H.h2d(dx, src, static_cast<size_t>(n) * 4));
    STEP(H.h2d(ds, &scale, 4));
    STEP(launch_quantize_i8(dx, dq, n, ds, H.st()));
    STEP(launch_widen(dq, dw, n, 0, 0, H.st()));
    STEP(H.d2h(dst, dw, static_cast<size_t>(n) * 4));
    return H.finish();
    TVQ_CATCH
}

static int narrow_to_host_bytes(const int32_t* src, int64_t n, int32_t off, std::vector<uint8_t>& out) {
    // The list[i32] values are narrowed on the host: this is boundary
    // conversion of the caller's storage format, not computation.
    out.resize(static_cast<size_t>(n));
    for (int64_t i = 0; i < n; i++) out[static_cast<size_t>(i)] = static_cast<uint8_t>((src[i] + off) & 0xFF);
    return TVQ_OK;
}

int tvq_matmul_int8_per_channel_i32(const int32_t* A, const int32_t* W, const float* bias, int64_t n_bias, float* Y,
                                    int64_t m, int64_t n, int64_t k, float scale_a, const float* scales_w,
                                    int64_t n_scales) {
    TVQ_CHECK(m >= 0 && n >= 0 && k >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(n_scales >= n, TVQ_ERR_SIZE, "scales_w smaller than N");  // matmul.tkv:18-19
    if (m == 0 || n == 0) return TVQ_OK;
    TVQ_CHECK(k == 0 || (A && W), TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    std::vector<uint8_t> a8, w8;
    narrow_to_host_bytes(A, m * k, 0, a8);
    narrow_to_host_bytes(W, n * k, 0, w8);
    return host_gemm(GEMM_I8, a8.data(), w8.data(), 1, bias, n_bias, Y, m, n, k, scale_a, scales_w, n_scales, 1,
                     TVQ_ACT_NONE);
    TVQ_CATCH
}

int tvq_quantize_fp8_e4m3_i32(const float* src, int64_t n, int32_t* dst, int64_t dst_len) {
    TVQ_CHECK(n >= 0 && dst_len >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(dst_len >= n, TVQ_ERR_SIZE, "dst too small");
    if (n == 0) return TVQ_OK;
    TVQ_CHECK(src && dst, TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    HOST_BEGIN
    float* dx = dev<float>(H, 0, static_cast<size_t>(n));
    uint8_t* dq = dev<uint8_t>(H, 1, static_cast<size_t>(n));
    int32_t* dw = dev<int32_t>(H, 2, static_cast<size_t>(n));
    if (H.rc) return H.rc;
    STEP(H.h2d(dx, src, static_cast<size_t>(n) * 4));
    STEP(launch_fp8_encode(dx, dq, 1, n, nullptr, 0, 0, H.st()));
    STEP(launch_widen(dq, dw, n, 1, -128, H.st()));  // byte - 128, matmul.tkv:65
    STEP(H.d2h(dst, dw, static_cast<size_t>(n) * 4));
    return H.finish();
    TVQ_CATCH
}

int tvq_matmul_fp8_e4m3_i32(const int32_t* A, const int32_t* W, const float* bias, int64_t n_bias, float* Y,
                            int64_t m, int64_t n, int64_t k) {
    TVQ_CHECK(m >= 0 && n >= 0 && k >= 0, TVQ_ERR_INVALID, "negative size");
    if (m == 0 || n == 0) return TVQ_OK;
    TVQ_CHECK(k == 0 || (A && W), TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    std::vector<uint8_t> a8, w8;
    narrow_to_host_bytes(A, m * k, 128, a8);  // _fp8_decode(v) reads byte v + 128, matmul.tkv:76
    narrow_to_host_bytes(W, n * k, 128, w8);
    const float one = 1.0f;
    return host_gemm(GEMM_F8, a8.data(), w8.data(), 1, bias, n_bias, Y, m, n, k, 1.0f, &one, 1, 0, TVQ_ACT_NONE);
    TVQ_CATCH
}

int tvq_matmul_int8_asymmetric(const int8_t* A, const int8_t* W, const float* bias, int64_t n_bias, float* Y,
                               int64_t m, int64_t n, int64_t k, float scale_a, int64_t zp_a, float scale_w,
                               int64_t zp_w) {
    TVQ_TRY
    return host_gemm_asym(A, W, bias, n_bias, Y, m, n, k, scale_a, zp_a, scale_w, zp_w);
    TVQ_CATCH
}

int tvq_matmul_int8_asymmetric_i32(const int32_t* A, const int32_t* W, const float* bias, int64_t n_bias, float* Y,
                                   int64_t m, int64_t n, int64_t k, float scale_a, int64_t zp_a, float scale_w,
                                   int64_t zp_w) {
    TVQ_CHECK(m >= 0 && n >= 0 && k >= 0, TVQ_ERR_INVALID, "negative size");
    if (m == 0 || n == 0) return TVQ_OK;
    TVQ_CHECK(k == 0 || (A && W), TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    std::vector<uint8_t> a8, w8;
    narrow_to_host_bytes(A, m * k, 0, a8);
    narrow_to_host_bytes(W, n * k, 0, w8);
    return host_gemm_asym(reinterpret_cast<const int8_t*>(a8.data()), reinterpret_cast<const int8_t*>(w8.data()), bias,
                          n_bias, Y, m, n, k, scale_a, zp_a, scale_w, zp_w);
    TVQ_CATCH
}

int tvq_matmul_fp16(const uint16_t* A, const uint16_t* W, const float* bias, int64_t n_bias, float* Y, int64_t m,
                    int64_t n, int64_t k) {
    TVQ_TRY
    return host_gemm_f16(A, W, bias, n_bias, Y, m, n, k);
    TVQ_CATCH
}

int tvq_matmul_fp16_i32(const int32_t* A, const int32_t* W, const float* bias, int64_t n_bias, float* Y, int64_t m,
                        int64_t n, int64_t k) {
    TVQ_CHECK(m >= 0 && n >= 0 && k >= 0, TVQ_ERR_INVALID, "negative size");
    if (m == 0 || n == 0) return TVQ_OK;
    TVQ_CHECK(k == 0 || (A && W), TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    // two list entries per element, low byte first (& 255 each, matmul.tkv:84-87)
    std::vector<uint8_t> a8, w8;
    narrow_to_host_bytes(A, 2 * m * k, 0, a8);
    narrow_to_host_bytes(W, 2 * n * k, 0, w8);
    return host_gemm_f16(reinterpret_cast<const uint16_t*>(a8.data()), reinterpret_cast<const uint16_t*>(w8.data()),
                         bias, n_bias, Y, m, n, k);
    TVQ_CATCH
}

int tvq_quantize_fp16(const float* src, int64_t n, uint16_t* dst, int64_t dst_len) {
    TVQ_CHECK(n >= 0 && dst_len >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(dst_len >= n, TVQ_ERR_SIZE, "dst too small");
    if (n == 0) return TVQ_OK;
    TVQ_CHECK(src && dst, TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    HOST_BEGIN
    float* dx = dev<float>(H, 0, static_cast<size_t>(n));
    uint16_t* dq = dev<uint16_t>(H, 1, static_cast<size_t>(n));
    if (H.rc) return H.rc;
    STEP(H.h2d(dx, src, static_cast<size_t>(n) * 4));
    STEP(launch_f16_encode(dx, dq, n, H.st()));
    STEP(H.d2h(dst, dq, static_cast<size_t>(n) * 2));
    return H.finish();
    TVQ_CATCH
}

int tvq_quantize_fp16_i32(const float* src, int64_t n, int32_t* dst, int64_t dst_len) {
    TVQ_CHECK(n >= 0 && dst_len >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(dst_len >= 2 * n, TVQ_ERR_SIZE, "dst too small (need 2 bytes/elem)");  // matmul.tkv:107-108
    if (n == 0) return TVQ_OK;
    TVQ_CHECK(src && dst, TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    HOST_BEGIN
    float* dx = dev<float>(H, 0, static_cast<size_t>(n));
    uint16_t* dq = dev<uint16_t>(H, 1, static_cast<size_t>(n));
    int32_t* dw = dev<int32_t>(H, 2, static_cast<size_t>(2 * n));
    if (H.rc) return H.rc;
    STEP(H.h2d(dx, src, static_cast<size_t>(n) * 4));
    STEP(launch_f16_encode(dx, dq, n, H.st()));
    // each byte as a signed value (_to_sbyte, matmul.tkv:98-103), low byte first
    STEP(launch_widen(dq, dw, 2 * n, 0, 0, H.st()));
    STEP(H.d2h(dst, dw, static_cast<size_t>(2 * n) * 4));
    return H.finish();
    TVQ_CATCH
}

// ================================================================ device buffers

int tvq_dev_minmax_reset(uint32_t* minmax_dev, void* stream) {
    TVQ_CHECK(minmax_dev, TVQ_ERR_INVALID, "null buffer");
    return launch_minmax_reset(minmax_dev, static_cast<cudaStream_t>(stream));
}

int tvq_dev_minmax_accumulate(const float* x, int64_t n, uint32_t* minmax_dev, float* first_dev, void* stream) {
    TVQ_CHECK(n >= 0 && minmax_dev && (n == 0 || x), TVQ_ERR_INVALID, "null buffer");
    return launch_minmax_accumulate(x, n, minmax_dev, first_dev, static_cast<cudaStream_t>(stream));
}

int tvq_dev_minmax_finalize(const uint32_t* minmax_dev, const float* first_dev, int symmetric, float* params_dev,
                            void* stream) {
    TVQ_CHECK(minmax_dev && params_dev, TVQ_ERR_INVALID, "null buffer");
    return launch_minmax_finalize(minmax_dev, first_dev, symmetric, params_dev, static_cast<cudaStream_t>(stream));
}

int tvq_dev_quantize_int8(const float* x, int8_t* q, int64_t n, const float* scale_dev, void* stream) {
    TVQ_CHECK(n >= 0 && (n == 0 || (x && q && scale_dev)), TVQ_ERR_INVALID, "null buffer");
    return launch_quantize_i8(x, q, n, scale_dev, static_cast<cudaStream_t>(stream));
}

int tvq_dev_quantize_fp16(const float* x, uint16_t* q, int64_t n, void* stream) {
    TVQ_CHECK(n >= 0 && (n == 0 || (x && q)), TVQ_ERR_INVALID, "null buffer");
    return launch_f16_encode(x, q, n, static_cast<cudaStream_t>(stream));
}

int tvq_dev_matmul_fp16(const uint16_t* A, const uint16_t* W, const float* bias, float* Y, int64_t m, int64_t n,
                        int64_t k, void* stream) {
    TVQ_CHECK(m >= 0 && n >= 0 && k >= 0, TVQ_ERR_INVALID, "negative size");
    if (m == 0 || n == 0) return TVQ_OK;
    TVQ_CHECK(Y && (k == 0 || (A && W)), TVQ_ERR_INVALID, "null buffer");
    GemmArgs g;
    g.kind = GEMM_F16X3;  // without low parts: the plain fp16 product
    g.A = A;
    g.W = W;
    g.bias = bias;
    g.Y = Y;
    g.m = m;
    g.n = n;
    g.k = k;
    return launch_gemm(g, static_cast<cudaStream_t>(stream));
}

int tvq_dev_matmul_int8_asymmetric(const int8_t* A, const int8_t* W, const float* bias, float* Y, int64_t m, int64_t n,
                                   int64_t k, const float* scale_a_dev, int64_t zp_a, const float* scale_w_dev,
                                   int64_t zp_w, void* stream) {
    TVQ_CHECK(m >= 0 && n >= 0 && k >= 0, TVQ_ERR_INVALID, "negative size");
    if (m == 0 || n == 0) return TVQ_OK;
    TVQ_CHECK(Y && scale_a_dev && scale_w_dev && (k == 0 || (A && W)), TVQ_ERR_INVALID, "null buffer");
    TVQ_CHECK(m < (1ll << 31) && n < (1ll << 31), TVQ_ERR_UNSUPPORTED, "size out of range");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int* sums = nullptr;  // stream-ordered scratch: [m] + [n] row sums
    TVQ_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&sums), sizeof(int) * static_cast<size_t>(m + n), st));
    int rc = launch_row_sums_i8(A, m, k, sums, st);
    if (!rc) rc = launch_row_sums_i8(W, n, k, sums + m, st);
    if (!rc) {
        GemmArgs g;
        g.kind = GEMM_I8;
        g.A = A;
        g.W = W;
        g.bias = bias;
        g.Y = Y;
        g.m = m;
        g.n = n;
        g.k = k;
        g.scale_a = scale_a_dev;
        g.scales_w = scale_w_dev;
        g.per_channel = 0;
        g.zp_rows = sums;
        g.zp_cols = sums + m;
        g.zp_a = zp_a;
        g.zp_w = zp_w;
        g.zp_k = k;
        rc = launch_gemm(g, st);
    }
    cudaError_t e = cudaFreeAsync(sums, st);
    if (!rc && e != cudaSuccess) return cuda_fail(e, "cudaFreeAsync");
    return rc;
}

int tvq_dev_calibrate_quantize_per_channel(const float* w, int8_t* q, float* scales_dev, int64_t rows, int64_t cols,
                                           void* stream) {
    TVQ_CHECK(rows >= 0 && cols >= 0 && (rows * cols == 0 || (w && q && scales_dev)), TVQ_ERR_INVALID, "bad args");
    return launch_rowwise(0, w, q, scales_dev, rows, cols, static_cast<cudaStream_t>(stream));
}

int tvq_dev_quantize_int8_per_channel(const float* w, int8_t* q, const float* scales_dev, int64_t rows, int64_t cols,
                                      void* stream) {
    TVQ_CHECK(rows >= 0 && cols >= 0 && (rows * cols == 0 || (w && q && scales_dev)), TVQ_ERR_INVALID, "bad args");
    return launch_rowwise(1, w, q, const_cast<float*>(scales_dev), rows, cols, static_cast<cudaStream_t>(stream));
}

int tvq_dev_quantize_dynamic_rowwise(const float* x, int8_t* q, float* scales_dev, int64_t rows, int64_t cols,
                                     void* stream) {
    TVQ_CHECK(rows >= 0 && cols >= 0 && (rows * cols == 0 || (x && q && scales_dev)), TVQ_ERR_INVALID, "bad args");
    return launch_rowwise(2, x, q, scales_dev, rows, cols, static_cast<cudaStream_t>(stream));
}

int tvq_dev_quantize_fp8(const float* x, uint8_t* q, int64_t rows, int64_t cols, const float* scales_dev,
                         int scale_mode, int mode, void* stream) {
    TVQ_CHECK(rows >= 0 && cols >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(scale_mode >= 0 && scale_mode <= 2 && (scale_mode == 0 || scales_dev), TVQ_ERR_INVALID, "bad scale mode");
    TVQ_CHECK(mode == TVQ_FP8_REF || mode == TVQ_FP8_HW, TVQ_ERR_INVALID, "bad FP8 mode");
    return launch_fp8_encode(x, q, rows, cols, scales_dev, scale_mode, mode, static_cast<cudaStream_t>(stream));
}

int tvq_dev_dequantize_fp8(const uint8_t* q, float* y, int64_t n, void* stream) {
    TVQ_CHECK(n >= 0 && (n == 0 || (q && y)), TVQ_ERR_INVALID, "null buffer");
    return launch_fp8_decode(q, y, n, static_cast<cudaStream_t>(stream));
}

int tvq_dev_gemm(int kind, const void* A, const void* W, const float* bias, const float* residual, float* Y,
                 int8_t* Yq, int64_t m, int64_t n, int64_t k, const float* scale_a_dev, const float* scales_w_dev,
                 int per_channel, int act, const float* scale_out_dev, uint32_t* amax_dev, void* stream) {
    TVQ_CHECK(kind == GEMM_I8 || kind == GEMM_F8, TVQ_ERR_INVALID, "bad GEMM kind");
    TVQ_CHECK(act == TVQ_ACT_NONE || act == TVQ_ACT_RELU || act == TVQ_ACT_GELU_TANH || act == TVQ_ACT_GELU_ERF,
              TVQ_ERR_INVALID, "bad activation");
    TVQ_CHECK(Y || Yq || amax_dev, TVQ_ERR_INVALID, "no output");
    GemmArgs g;
    g.kind = kind;
    g.A = A;
    g.W = W;
    g.bias = bias;
    g.residual = residual;
    g.Y = Y;
    g.Yq = Yq;
    g.m = m;
    g.n = n;
    g.k = k;
    g.scale_a = scale_a_dev;
    g.scales_w = scales_w_dev;
    g.per_channel = per_channel;
    g.act = act;
    g.scale_out = scale_out_dev;
    g.amax = amax_dev;
    TVQ_TRY
    return launch_gemm(g, static_cast<cudaStream_t>(stream));
    TVQ_CATCH
}

int tvq_dev_split_tf32(const float* x, float* hi, float* lo, int64_t n, void* stream) {
    TVQ_CHECK(n >= 0 && (n == 0 || (x && hi && lo)), TVQ_ERR_INVALID, "null buffer");
    return launch_split_tf32(x, hi, lo, n, static_cast<cudaStream_t>(stream));
}

int tvq_dev_gemm_f32x3(const float* A_hi, const float* A_lo, const float* W_hi, const float* W_lo, float* Y, int64_t m,
                       int64_t n, int64_t k, void* stream) {
    TVQ_CHECK(Y && A_hi && A_lo && W_hi && W_lo, TVQ_ERR_INVALID, "null buffer");
    GemmArgs g;
    g.kind = GEMM_TF32X3;
    g.A = A_hi;
    g.A2 = A_lo;
    g.W = W_hi;
    g.W2 = W_lo;
    g.Y = Y;
    g.m = m;
    g.n = n;
    g.k = k;
    g.per_channel = 0;  // this kind reads no scales: Y is the accumulator
    TVQ_TRY
    return launch_gemm(g, static_cast<cudaStream_t>(stream));
    TVQ_CATCH
}

int tvq_dev_split_f16_rows(const float* x, void* hi, void* lo, float* rscale, int64_t rows, int64_t k, void* stream) {
    TVQ_CHECK(rows >= 0 && k >= 0, TVQ_ERR_INVALID, "negative size");
    if (rows == 0) return TVQ_OK;
    TVQ_CHECK(rscale && (k == 0 || (x && hi && lo)), TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    return launch_split_f16_rows(x, hi, lo, rscale, rows, k, static_cast<cudaStream_t>(stream));
    TVQ_CATCH
}

int tvq_dev_gemm_f16x3(const void* A_hi, const void* A_lo, const float* A_rscale, const void* W_hi, const void* W_lo,
                       const float* W_rscale, float* Y, int64_t m, int64_t n, int64_t k, void* stream) {
    TVQ_CHECK(Y && A_hi && A_lo && A_rscale && W_hi && W_lo && W_rscale, TVQ_ERR_INVALID, "null buffer");
    GemmArgs g;
    g.kind = GEMM_F16X3;
    g.A = A_hi;
    g.A2 = A_lo;
    g.W = W_hi;
    g.W2 = W_lo;
    g.scale_a = A_rscale;
    g.scales_w = W_rscale;
    g.Y = Y;
    g.m = m;
    g.n = n;
    g.k = k;
    TVQ_TRY
    return launch_gemm(g, static_cast<cudaStream_t>(stream));
    TVQ_CATCH
}

}  // extern "C"

// ---------------------------------------------------------------- ONNX QDQ operators
// (tv/runtime/session.tkv:1896-2071, 2789-2905)

extern "C" {

int tvq_dev_quantize_linear(const float* x, int8_t* y, int64_t outer, int64_t dim, int64_t inner,
                            const float* scales_dev, int64_t n_scales, int64_t zero_point, void* stream) {
    TVQ_CHECK(outer >= 0 && dim >= 0 && inner >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(outer * dim * inner == 0 || (x && y && scales_dev), TVQ_ERR_INVALID, "null buffer");
    return launch_quantize_linear(x, y, outer, dim, inner, scales_dev, n_scales, zero_point,
                                  static_cast<cudaStream_t>(stream));
}

int tvq_dev_dequantize_linear(const int8_t* x, float* y, int64_t outer, int64_t dim, int64_t inner,
                              const float* scales_dev, int64_t n_scales, int64_t zero_point, void* stream) {
    TVQ_CHECK(outer >= 0 && dim >= 0 && inner >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(outer * dim * inner == 0 || (x && y && scales_dev), TVQ_ERR_INVALID, "null buffer");
    return launch_dequantize_linear(x, y, outer, dim, inner, scales_dev, n_scales, zero_point,
                                    static_cast<cudaStream_t>(stream));
}

int tvq_dev_matmul_integer(const int8_t* a, const int8_t* b, int32_t* y, int64_t m, int64_t k, int64_t n,
                           void* stream) {
    TVQ_CHECK(m * n == 0 || (y && (k == 0 || (a && b))), TVQ_ERR_INVALID, "null buffer");
    return launch_matmul_integer(a, b, y, m, k, n, static_cast<cudaStream_t>(stream));
}

int tvq_dev_qlinear_matmul(const int8_t* a, float scale_a, int64_t zp_a, const int8_t* b, float scale_b,
                           int64_t zp_b, float scale_y, int64_t zp_y, int8_t* y, int64_t m, int64_t k, int64_t n,
                           void* stream) {
    TVQ_CHECK(m * n == 0 || (y && (k == 0 || (a && b))), TVQ_ERR_INVALID, "null buffer");
    return launch_qlinear_matmul(a, scale_a, zp_a, b, scale_b, zp_b, scale_y, zp_y, y, m, k, n,
                                 static_cast<cudaStream_t>(stream));
}

int tvq_dev_dynamic_quantize_linear(const float* x, int64_t n, int8_t* y, float* y_scale_dev, float* y_zp_dev,
                                    void* stream) {
    TVQ_CHECK(n >= 1, TVQ_ERR_SIZE, "DynamicQuantizeLinear needs at least one element");
    TVQ_CHECK(x && y && y_scale_dev && y_zp_dev, TVQ_ERR_INVALID, "null buffer");
    return launch_dynamic_quantize_linear(x, n, y, y_scale_dev, y_zp_dev, static_cast<cudaStream_t>(stream));
}

int tvq_quantize_linear(const float* x, int8_t* y, int64_t outer, int64_t dim, int64_t inner, const float* scales,
                        int64_t n_scales, int64_t zero_point) {
    TVQ_CHECK(outer >= 0 && dim >= 0 && inner >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(n_scales == 1 || n_scales == dim, TVQ_ERR_SIZE, "need one scale or one per channel of the axis");
    const int64_t n = outer * dim * inner;
    if (n == 0) return TVQ_OK;
    TVQ_CHECK(x && y && scales, TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    HOST_BEGIN
    float* dx = dev<float>(H, 0, static_cast<size_t>(n));
    int8_t* dy = dev<int8_t>(H, 1, static_cast<size_t>(n));
    float* ds = dev<float>(H, 2, static_cast<size_t>(n_scales));
    if (H.rc) return H.rc;
    STEP(H.h2d(dx, x, static_cast<size_t>(n) * 4));
    STEP(H.h2d(ds, scales, static_cast<size_t>(n_scales) * 4));
    STEP(launch_quantize_linear(dx, dy, outer, dim, inner, ds, n_scales, zero_point, H.st()));
    STEP(H.d2h(y, dy, static_cast<size_t>(n)));
    return H.finish();
    TVQ_CATCH
}

int tvq_dequantize_linear(const int8_t* x, float* y, int64_t outer, int64_t dim, int64_t inner, const float* scales,
                          int64_t n_scales, int64_t zero_point) {
    TVQ_CHECK(outer >= 0 && dim >= 0 && inner >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(n_scales == 1 || n_scales == dim, TVQ_ERR_SIZE, "need one scale or one per channel of the axis");
    const int64_t n = outer * dim * inner;
    if (n == 0) return TVQ_OK;
    TVQ_CHECK(x && y && scales, TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    HOST_BEGIN
    int8_t* dx = dev<int8_t>(H, 0, static_cast<size_t>(n));
    float* dy = dev<float>(H, 1, static_cast<size_t>(n));
    float* ds = dev<float>(H, 2, static_cast<size_t>(n_scales));
    if (H.rc) return H.rc;
    STEP(H.h2d(dx, x, static_cast<size_t>(n)));
    STEP(H.h2d(ds, scales, static_cast<size_t>(n_scales) * 4));
    STEP(launch_dequantize_linear(dx, dy, outer, dim, inner, ds, n_scales, zero_point, H.st()));
    STEP(H.d2h(y, dy, static_cast<size_t>(n) * 4));
    return H.finish();
    TVQ_CATCH
}

int tvq_matmul_integer(const int8_t* a, const int8_t* b, int32_t* y, int64_t m, int64_t k, int64_t n) {
    TVQ_CHECK(m >= 0 && k >= 0 && n >= 0, TVQ_ERR_INVALID, "negative size");
    if (m == 0 || n == 0) return TVQ_OK;
    TVQ_CHECK(y && (k == 0 || (a && b)), TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    HOST_BEGIN
    int8_t* da = dev<int8_t>(H, 0, static_cast<size_t>(std::max<int64_t>(m * k, 1)));
    int8_t* db = dev<int8_t>(H, 1, static_cast<size_t>(std::max<int64_t>(k * n, 1)));
    int32_t* dy = dev<int32_t>(H, 2, static_cast<size_t>(m * n));
    if (H.rc) return H.rc;
    if (k > 0) {
        STEP(H.h2d(da, a, static_cast<size_t>(m * k)));
        STEP(H.h2d(db, b, static_cast<size_t>(k * n)));
    }
    STEP(launch_matmul_integer(da, db, dy, m, k, n, H.st()));
    STEP(H.d2h(y, dy, static_cast<size_t>(m * n) * 4));
    return H.finish();
    TVQ_CATCH
}

int tvq_qlinear_matmul(const int8_t* a, float scale_a, int64_t zp_a, const int8_t* b, float scale_b, int64_t zp_b,
                       float scale_y, int64_t zp_y, int8_t* y, int64_t m, int64_t k, int64_t n) {
    TVQ_CHECK(m >= 0 && k >= 0 && n >= 0, TVQ_ERR_INVALID, "negative size");
    if (m == 0 || n == 0) return TVQ_OK;
    TVQ_CHECK(y && (k == 0 || (a && b)), TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    HOST_BEGIN
    int8_t* da = dev<int8_t>(H, 0, static_cast<size_t>(std::max<int64_t>(m * k, 1)));
    int8_t* db = dev<int8_t>(H, 1, static_cast<size_t>(std::max<int64_t>(k * n, 1)));
    int8_t* dy = dev<int8_t>(H, 2, static_cast<size_t>(m * n));
    if (H.rc) return H.rc;
    if (k > 0) {
        STEP(H.h2d(da, a, static_cast<size_t>(m * k)));
        STEP(H.h2d(db, b, static_cast<size_t>(k * n)));
    }
    STEP(launch_qlinear_matmul(da, scale_a, zp_a, db, scale_b, zp_b, scale_y, zp_y, dy, m, k, n, H.st()));
    STEP(H.d2h(y, dy, static_cast<size_t>(m * n)));
    return H.finish();
    TVQ_CATCH
}

int tvq_dynamic_quantize_linear(const float* x, int64_t n, int8_t* y, float* y_scale, float* y_zero_point) {
    TVQ_CHECK(n >= 1, TVQ_ERR_SIZE, "DynamicQuantizeLinear needs at least one element");
    TVQ_CHECK(x && y && y_scale && y_zero_point, TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    HOST_BEGIN
    float* dx = dev<float>(H, 0, static_cast<size_t>(n));
    int8_t* dy = dev<int8_t>(H, 1, static_cast<size_t>(n));
    float* dsz = dev<float>(H, 2, 2);
    if (H.rc) return H.rc;
    STEP(H.h2d(dx, x, static_cast<size_t>(n) * 4));
    STEP(launch_dynamic_quantize_linear(dx, n, dy, dsz, dsz + 1, H.st()));
    STEP(H.d2h(y, dy, static_cast<size_t>(n)));
    STEP(H.d2h(y_scale, dsz, 4));
    STEP(H.d2h(y_zero_point, dsz + 1, 4));
    return H.finish();
    TVQ_CATCH
}

}  // extern "C"

// ---------------------------------------------------------------- calibration methods
// calibrate_kl / _percentile / _mse, tv/quantization/engine.tkv:42-197.

namespace {

int calib_identity(float* scale, int64_t* zp, float* mn, float* mx) {
    // _quant_identity, engine.tkv:9-10
    *scale = 1.0f;
    *zp = 0;
    *mn = -3.4028234663852886e38f;
    *mx = 3.4028234663852886e38f;
    return TVQ_OK;
}

// run one device calibration on a host array; method 0 KL, 1 percentile, 2 MSE
int host_calibrate(int method, const float* data, int64_t n, int a0, int a1, float pct, float* scale, int64_t* zp,
                   float* mn, float* mx) {
    TVQ_CHECK(scale && zp && mn && mx, TVQ_ERR_INVALID, "null output");
    if (n == 0) return calib_identity(scale, zp, mn, mx);  // the empty check comes first in all three
    TVQ_CHECK(n > 0 && data, TVQ_ERR_INVALID, "null data");
    int fallback = 0;
    {
        TVQ_TRY
        HOST_BEGIN
        float* dx = dev<float>(H, 0, static_cast<size_t>(n));
        float* d4 = dev<float>(H, 1, 4);
        if (H.rc) return H.rc;
        STEP(H.h2d(dx, data, static_cast<size_t>(n) * 4));
        if (method == 0) STEP(launch_calibrate_kl(dx, n, a0, a1, d4, &fallback, H.st()));
        else if (method == 1) STEP(launch_calibrate_percentile(dx, n, pct, a0, d4, H.st()));
        else STEP(launch_calibrate_mse(dx, n, a0, d4, nullptr, &fallback, H.st()));
        float o[4] = {0, 0, 0, 0};
        if (!fallback) STEP(H.d2h(o, d4, 16));
        const int rc = H.finish();
        if (rc) return rc;
        if (!fallback) {
            *scale = o[0];
            *zp = static_cast<int64_t>(o[1]);
            *mn = o[2];
            *mx = o[3];
        }
        TVQ_CATCH
    }
    if (fallback) return tvq_calibrate_minmax(data, n, 1, scale, zp, mn, mx);  // max |x| < 1e-8
    return TVQ_OK;
}

}  // namespace

extern "C" {

int tvq_calibrate_kl(const float* data, int64_t n, int64_t num_bins, int64_t target_bins, float* scale,
                     int64_t* zero_point, float* min_val, float* max_val) {
    TVQ_CHECK(n >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(num_bins >= 1 && num_bins <= 4096 && target_bins >= 1, TVQ_ERR_UNSUPPORTED,
              "num_bins must be in [1, 4096] and target_bins >= 1");
    return host_calibrate(0, data, n, static_cast<int>(num_bins), static_cast<int>(target_bins), 0.0f, scale,
                          zero_point, min_val, max_val);
}

int tvq_calibrate_percentile(const float* data, int64_t n, float percentile, int symmetric, float* scale,
                             int64_t* zero_point, float* min_val, float* max_val) {
    TVQ_CHECK(n >= 0, TVQ_ERR_INVALID, "negative size");
    if (n > 0) TVQ_CHECK(percentile > 0.0f && percentile <= 100.0f, TVQ_ERR_SIZE, "percentile must be in (0, 100]");
    return host_calibrate(1, data, n, symmetric, 0, percentile, scale, zero_point, min_val, max_val);
}

int tvq_calibrate_mse(const float* data, int64_t n, int64_t num_candidates, float* scale, int64_t* zero_point,
                      float* min_val, float* max_val) {
    TVQ_CHECK(n >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(num_candidates <= 65535, TVQ_ERR_UNSUPPORTED, "too many candidates");
    return host_calibrate(2, data, n, static_cast<int>(num_candidates), 0, 0.0f, scale, zero_point, min_val,
                          max_val);
}

int tvq_dev_calibrate_mse_curve(const float* x, int64_t n, int64_t num_candidates, double* curve_dev,
                                float* out4_dev, int* fallback, void* stream) {
    TVQ_CHECK(n >= 1 && x && curve_dev && out4_dev && fallback, TVQ_ERR_INVALID, "bad arguments");
    TVQ_CHECK(num_candidates >= 4 && num_candidates <= 65535, TVQ_ERR_UNSUPPORTED, "4..65535 candidates");
    return launch_calibrate_mse(x, n, static_cast<int>(num_candidates), out4_dev, curve_dev, fallback,
                                static_cast<cudaStream_t>(stream));
}


// ---------------------------------------------------------------- group-wise INT4 (int4.tkv)

int tvq_dev_quantize_int4_grouped(const float* src, int64_t rows, int64_t cols, int64_t group_size, uint8_t* packed,
                                  float* scales, int64_t* zps, void* stream) {
    TVQ_CHECK(rows >= 0 && cols >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(rows * cols == 0 || (src && packed && scales), TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    return launch_int4_quantize(src, rows, cols, group_size, packed, scales, zps, static_cast<cudaStream_t>(stream));
    TVQ_CATCH
}

int tvq_dev_dequantize_int4_grouped(const uint8_t* packed, float* dst, int64_t rows, int64_t cols, int64_t group_size,
                                    const float* scales, const int64_t* zps, void* stream) {
    TVQ_CHECK(rows >= 0 && cols >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(rows * cols == 0 || (packed && dst && scales), TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    return launch_int4_dequantize(packed, dst, rows, cols, group_size, scales, zps, static_cast<cudaStream_t>(stream));
    TVQ_CATCH
}

int tvq_dev_permute_cols(const float* src, float* dst, int64_t rows, int64_t cols, const int64_t* perm, int inverse,
                         void* stream) {
    TVQ_CHECK(rows >= 0 && cols >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(rows * cols == 0 || (src && dst && perm), TVQ_ERR_INVALID, "null buffer");
    TVQ_CHECK(src != dst, TVQ_ERR_INVALID, "permute_cols cannot run in place");
    TVQ_TRY
    return launch_permute_cols(src, dst, rows, cols, perm, inverse, static_cast<cudaStream_t>(stream));
    TVQ_CATCH
}

int tvq_dev_matmul_int4_grouped(const float* A, const uint8_t* packed_w, const float* bias, float* Y, int64_t m,
                                int64_t n, int64_t k, int64_t group_size, const float* scales_w, const int64_t* perm,
                                void* stream) {
    TVQ_CHECK(m >= 0 && n >= 0 && k >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(group_size > 0 && k % group_size == 0 && k % 2 == 0, TVQ_ERR_SIZE,
              "k must be an even multiple of group_size");
    if (m == 0 || n == 0) return TVQ_OK;
    TVQ_CHECK(Y && (k == 0 || (A && packed_w && scales_w)), TVQ_ERR_INVALID, "null buffer");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    TVQ_TRY
    GemmArgs g;
    g.kind = GEMM_W4;
    g.bias = bias;
    g.Y = Y;
    g.m = m;
    g.n = n;
    g.k = k;
    g.group_size = group_size;
    g.scales_w = scales_w;
    if (k == 0) {
        g.scale_a = scales_w;  // unread
        return launch_gemm(g, st);
    }
    // scratch (stream-ordered): A hi / lo fp16 [m, k], its row scales, W as fp16 integers [n, k]
    const size_t ak = (static_cast<size_t>(m) * k * 2 + 15) & ~size_t(15);
    const size_t wk = (static_cast<size_t>(n) * k * 2 + 15) & ~size_t(15);
    uint8_t* buf = nullptr;
    TVQ_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&buf), 2 * ak + wk + sizeof(float) * m, st));
    float* ra = reinterpret_cast<float*>(buf + 2 * ak + wk);
    int r = launch_split_f16_rows(A, buf, buf + ak, ra, m, k, st, perm);
    if (!r) r = launch_int4_unpack_f16(packed_w, buf + 2 * ak, n, k, st);
    if (!r) {
        g.A = buf;
        g.A2 = buf + ak;
        g.W = buf + 2 * ak;
        g.scale_a = ra;
        r = launch_gemm(g, st);
    }
    cudaError_t e = cudaFreeAsync(buf, st);
    if (!r && e != cudaSuccess) return cuda_fail(e, "cudaFreeAsync");
    return r;
    TVQ_CATCH
}

// host-buffer forms (synchronous), the reference's signatures
int tvq_quantize_int4_grouped(const float* src, int64_t rows, int64_t cols, int64_t group_size, uint8_t* packed_out,
                              float* scales_out, int64_t* zps_out) {
    TVQ_CHECK(rows >= 0 && cols >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(group_size > 0 && cols % group_size == 0 && cols % 2 == 0, TVQ_ERR_SIZE,
              "cols must be a multiple of group_size and even");
    if (rows * cols == 0) return TVQ_OK;
    TVQ_CHECK(src && packed_out && scales_out, TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    HOST_BEGIN
    const int64_t ng = cols / group_size;
    float* ds = dev<float>(H, 0, static_cast<size_t>(rows * cols));
    uint8_t* dp = dev<uint8_t>(H, 1, static_cast<size_t>(rows * cols / 2));
    float* dsc = dev<float>(H, 2, static_cast<size_t>(rows * ng));
    int64_t* dz = zps_out ? dev<int64_t>(H, 3, static_cast<size_t>(rows * ng)) : nullptr;
    if (H.rc) return H.rc;
    TVQ_CUDA(cudaMemcpyAsync(ds, src, sizeof(float) * rows * cols, cudaMemcpyHostToDevice, H.st()));
    STEP(launch_int4_quantize(ds, rows, cols, group_size, dp, dsc, dz, H.st()));
    TVQ_CUDA(cudaMemcpyAsync(packed_out, dp, static_cast<size_t>(rows * cols / 2), cudaMemcpyDeviceToHost, H.st()));
    TVQ_CUDA(cudaMemcpyAsync(scales_out, dsc, sizeof(float) * rows * ng, cudaMemcpyDeviceToHost, H.st()));
    if (dz) TVQ_CUDA(cudaMemcpyAsync(zps_out, dz, sizeof(int64_t) * rows * ng, cudaMemcpyDeviceToHost, H.st()));
    return check_device_error(H.st());
    TVQ_CATCH
}

int tvq_dequantize_int4_grouped(const uint8_t* packed, float* dst, int64_t rows, int64_t cols, int64_t group_size,
                                const float* scales, int64_t n_scales, const int64_t* zps) {
    TVQ_CHECK(rows >= 0 && cols >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(group_size > 0 && cols % group_size == 0 && cols % 2 == 0, TVQ_ERR_SIZE,
              "cols must be a multiple of group_size and even");
    TVQ_CHECK(n_scales >= rows * (cols / group_size), TVQ_ERR_SIZE, "scales smaller than rows*num_groups");  // :53-54
    if (rows * cols == 0) return TVQ_OK;
    TVQ_CHECK(packed && dst && scales, TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    HOST_BEGIN
    const int64_t ng = cols / group_size;
    uint8_t* dp = dev<uint8_t>(H, 0, static_cast<size_t>(rows * cols / 2));
    float* dd = dev<float>(H, 1, static_cast<size_t>(rows * cols));
    float* dsc = dev<float>(H, 2, static_cast<size_t>(rows * ng));
    int64_t* dz = zps ? dev<int64_t>(H, 3, static_cast<size_t>(rows * ng)) : nullptr;
    if (H.rc) return H.rc;
    TVQ_CUDA(cudaMemcpyAsync(dp, packed, static_cast<size_t>(rows * cols / 2), cudaMemcpyHostToDevice, H.st()));
    TVQ_CUDA(cudaMemcpyAsync(dsc, scales, sizeof(float) * rows * ng, cudaMemcpyHostToDevice, H.st()));
    if (dz) TVQ_CUDA(cudaMemcpyAsync(dz, zps, sizeof(int64_t) * rows * ng, cudaMemcpyHostToDevice, H.st()));
    STEP(launch_int4_dequantize(dp, dd, rows, cols, group_size, dsc, dz, H.st()));
    TVQ_CUDA(cudaMemcpyAsync(dst, dd, sizeof(float) * rows * cols, cudaMemcpyDeviceToHost, H.st()));
    return check_device_error(H.st());
    TVQ_CATCH
}

int tvq_permute_cols(const float* src, float* dst, int64_t rows, int64_t cols, const int64_t* perm, int64_t n_perm,
                     int inverse) {
    TVQ_CHECK(rows >= 0 && cols >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(n_perm == cols, TVQ_ERR_SIZE, "perm length must equal cols");  // int4.tkv:170-171
    if (rows * cols == 0) return TVQ_OK;
    TVQ_CHECK(src && dst && perm, TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    HOST_BEGIN
    float* ds = dev<float>(H, 0, static_cast<size_t>(rows * cols));
    float* dd = dev<float>(H, 1, static_cast<size_t>(rows * cols));
    int64_t* dpm = dev<int64_t>(H, 2, static_cast<size_t>(cols));
    if (H.rc) return H.rc;
    TVQ_CUDA(cudaMemcpyAsync(ds, src, sizeof(float) * rows * cols, cudaMemcpyHostToDevice, H.st()));
    TVQ_CUDA(cudaMemcpyAsync(dpm, perm, sizeof(int64_t) * cols, cudaMemcpyHostToDevice, H.st()));
    if (inverse) TVQ_CUDA(cudaMemsetAsync(dd, 0, sizeof(float) * rows * cols, H.st()));
    STEP(launch_permute_cols(ds, dd, rows, cols, dpm, inverse, H.st()));
    TVQ_CUDA(cudaMemcpyAsync(dst, dd, sizeof(float) * rows * cols, cudaMemcpyDeviceToHost, H.st()));
    return check_device_error(H.st());
    TVQ_CATCH
}

int tvq_matmul_int4_grouped(const float* A, const uint8_t* packed_w, const float* bias, int64_t n_bias, float* Y,
                            int64_t m, int64_t n, int64_t k, int64_t group_size, const float* scales_w,
                            int64_t n_scales, const int64_t* perm) {
    TVQ_CHECK(m >= 0 && n >= 0 && k >= 0 && n_bias >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(group_size > 0 && k % group_size == 0 && k % 2 == 0, TVQ_ERR_SIZE,
              "k must be an even multiple of group_size");
    TVQ_CHECK(n_scales >= n * (k / group_size), TVQ_ERR_SIZE, "scales_w smaller than N*num_groups");  // int4.tkv:215-216
    TVQ_CHECK(n_bias == 0 || n_bias >= n, TVQ_ERR_SIZE, "bias smaller than N");
    if (m == 0 || n == 0) return TVQ_OK;
    TVQ_CHECK(Y && (k == 0 || (A && packed_w && scales_w)) && (n_bias == 0 || bias), TVQ_ERR_INVALID, "null buffer");
    TVQ_TRY
    HOST_BEGIN
    const int64_t ng = k / group_size;
    float* dA = dev<float>(H, 0, static_cast<size_t>(std::max<int64_t>(m * k, 1)));
    uint8_t* dW = dev<uint8_t>(H, 1, static_cast<size_t>(std::max<int64_t>(n * k / 2, 1)));
    float* dS = dev<float>(H, 2, static_cast<size_t>(std::max<int64_t>(n * ng, 1)));
    float* dB = n_bias ? dev<float>(H, 3, static_cast<size_t>(n)) : nullptr;
    float* dY = dev<float>(H, 4, static_cast<size_t>(m * n));
    int64_t* dP = perm ? dev<int64_t>(H, 5, static_cast<size_t>(std::max<int64_t>(k, 1))) : nullptr;
    if (H.rc) return H.rc;
    if (k) {
        TVQ_CUDA(cudaMemcpyAsync(dA, A, sizeof(float) * m * k, cudaMemcpyHostToDevice, H.st()));
        TVQ_CUDA(cudaMemcpyAsync(dW, packed_w, static_cast<size_t>(n * k / 2), cudaMemcpyHostToDevice, H.st()));
        TVQ_CUDA(cudaMemcpyAsync(dS, scales_w, sizeof(float) * n * ng, cudaMemcpyHostToDevice, H.st()));
        if (dP) TVQ_CUDA(cudaMemcpyAsync(dP, perm, sizeof(int64_t) * k, cudaMemcpyHostToDevice, H.st()));
    }
    if (dB) TVQ_CUDA(cudaMemcpyAsync(dB, bias, sizeof(float) * n, cudaMemcpyHostToDevice, H.st()));
    STEP(tvq_dev_matmul_int4_grouped(dA, dW, dB, dY, m, n, k, group_size, dS, dP, H.st()));
    TVQ_CUDA(cudaMemcpyAsync(Y, dY, sizeof(float) * m * n, cudaMemcpyDeviceToHost, H.st()));
    return check_device_error(H.st());
    TVQ_CATCH
}

}  // extern "C"
