// tvq_noalloc.cu -- the causal-attention entry point that allocates nothing.
//
// tvq_dev_attention needs a small device scratch (the list of 64-row query
// tiles it schedules) that the caller passes in.  Some callers cannot
// allocate device memory when they call: a host runtime whose device memory
// is all handed to its own fixed pool, or a latency-critical serving loop
// that must not allocate because cudaMalloc can synchronise the device.  For
// them, tvq_dev_attention_noalloc keeps that scratch in a file-scope device
// array of fixed size instead.
//
// The array is a host-side symbol in this file; the device address used by
// the kernel comes from cudaGetSymbolAddress, taken once per device (with
// that device current) on the first call there.  Every call shares the same
// array and overwrites the part it uses before reading it, so nothing needs
// clearing; calls that overlap on the GPU (other streams, other threads)
// race on it and must be serialised by the caller.
//
// The tile list is built on the host and copied into the array with
// pageable cudaMemcpyAsync calls from a stack buffer, so a call blocks the
// calling thread until the work already queued on its stream has finished
// and the last copy has been staged.  It always runs the fp32 SIMT
// attention kernel (head dims 16, 32, 48 and 64): the tensor-core kernel
// that tvq_dev_attention uses at head dim 64 needs fp16 operand copies of
// the whole qkv tensor as scratch, far beyond a modest fixed array.
#include <atomic>
#include <mutex>

#include "tvq_common.cuh"
#include "tvq_glue.h"

namespace tvq {
namespace {

// 32768 query tiles x 16 bytes = 512 KiB on every GPU that loads the library:
// enough for 2,097,152 tokens per call (64 tokens per tile per sequence).
constexpr int64_t kNoallocMaxTiles = 32768;
__device__ __align__(256) int4 g_noalloc_tiles[kNoallocMaxTiles];

constexpr int kMaxDevices = 64;
std::atomic<int4*> g_tiles_dev[kMaxDevices] = {};
std::mutex g_setup_mu;

// Device address of g_noalloc_tiles on the current device (set-up on first use).
int tiles_address(int4** out) {
    int dev = 0;
    TVQ_CUDA(cudaGetDevice(&dev));
    TVQ_CHECK(dev >= 0 && dev < kMaxDevices, TVQ_ERR_UNSUPPORTED, "device ordinal too large");
    int4* ptr = g_tiles_dev[dev].load(std::memory_order_acquire);
    if (!ptr) {
        std::lock_guard<std::mutex> lk(g_setup_mu);
        ptr = g_tiles_dev[dev].load(std::memory_order_relaxed);
        if (!ptr) {
            void* p = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_tiles);
            if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress (no-allocation attention scratch)");
            ptr = static_cast<int4*>(p);
            g_tiles_dev[dev].store(ptr, std::memory_order_release);
        }
    }
    *out = ptr;
    return TVQ_OK;
}

}  // namespace
}  // namespace tvq

using namespace tvq;

extern "C" int tvq_dev_attention_noalloc(const float* qkv, const int64_t* seg, int64_t n_seg, int64_t d,
                                         int64_t n_heads, float* out, int8_t* outq, const float* qscale_dev,
                                         uint32_t* amax_dev, void* stream) {
    TVQ_CHECK(qkv && seg && n_seg >= 1 && (out || outq || amax_dev), TVQ_ERR_INVALID, "bad arguments");
    TVQ_CHECK(!outq || qscale_dev, TVQ_ERR_INVALID, "int8 output needs a scale");
    // every size check comes before any copy or launch
    TVQ_CHECK(n_heads > 0 && d > 0 && n_heads <= d && d % n_heads == 0 && d < (1LL << 29), TVQ_ERR_INVALID,
              "d must be a positive multiple of the head count");
    const int64_t hd = d / n_heads;
    TVQ_CHECK(hd == 16 || hd == 32 || hd == 48 || hd == 64, TVQ_ERR_UNSUPPORTED, "head dim must be 16, 32, 48 or 64");
    TVQ_CHECK(seg[0] >= 0, TVQ_ERR_INVALID, "segment offsets must be non-negative");
    int64_t ntiles = 0;
    for (int64_t s = 0; s < n_seg; s++) {
        TVQ_CHECK(seg[s + 1] >= seg[s], TVQ_ERR_INVALID, "segments must be non-decreasing");
        ntiles += (seg[s + 1] - seg[s] + 63) / 64;
    }
    TVQ_CHECK(ntiles <= kNoallocMaxTiles, TVQ_ERR_SIZE,
              "too many 64-token query tiles for the no-allocation scratch (maximum 32768 per call)");
    TVQ_CHECK(seg[n_seg] < (1LL << 31), TVQ_ERR_SIZE, "too many tokens");
    int4* tiles = nullptr;
    int rc = tiles_address(&tiles);
    if (rc) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // Fill the scratch from a fixed stack buffer: a pageable cudaMemcpyAsync
    // returns once the source has been staged, so the buffer can be refilled.
    int4 buf[256];
    int nb = 0;
    int64_t done = 0;
    for (int64_t s = 0; s < n_seg; s++) {
        for (int64_t q0 = seg[s]; q0 < seg[s + 1]; q0 += 64) {
            buf[nb++] = make_int4(static_cast<int>(q0), static_cast<int>(seg[s]), static_cast<int>(seg[s + 1]), 0);
            if (nb == 256) {
                TVQ_CUDA(cudaMemcpyAsync(tiles + done, buf, sizeof(buf), cudaMemcpyHostToDevice, st));
                done += nb;
                nb = 0;
            }
        }
    }
    if (nb) TVQ_CUDA(cudaMemcpyAsync(tiles + done, buf, sizeof(int4) * nb, cudaMemcpyHostToDevice, st));
    TVQ_CUDA(cudaStreamSynchronize(st));  // staging of the last chunk is complete before buf goes away
    return launch_attention(qkv, tiles, static_cast<int>(ntiles), static_cast<int>(seg[n_seg]), static_cast<int>(d),
                            static_cast<int>(n_heads), out, outq, qscale_dev, amax_dev, st);
}
