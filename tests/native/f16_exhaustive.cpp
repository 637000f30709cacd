// Checks the kernels' 32-bit FP16 encoder (tvq_f16.h: f16_encode_fast)
// against the step-by-step restatement in the same header for every one of
// the 2^32 binary32 bit patterns, and against the CPU oracle's encoder
// (tvo_f16_encode, oracle/tvq_oracle.c) on every STRIDE-th pattern.
//   f16_exhaustive <path to liboracle.so> <stride>
// Prints the mismatch counts; exit status 0 iff both are zero.
#include <dlfcn.h>

#include <cinttypes>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "../../tokenvector/inference_b200/csrc/tvq_f16.h"

int main(int argc, char** argv) {
    if (argc < 3) return 2;
    void* h = dlopen(argv[1], RTLD_NOW);
    if (!h) { std::fprintf(stderr, "dlopen: %s\n", dlerror()); return 2; }
    auto oracle = reinterpret_cast<int (*)(float)>(dlsym(h, "tvo_f16_encode"));
    if (!oracle) return 2;
    const uint64_t stride = std::strtoull(argv[2], nullptr, 10);
    uint64_t bad_ref = 0, bad_oracle = 0, checked_oracle = 0;
#pragma omp parallel for reduction(+ : bad_ref, bad_oracle, checked_oracle) schedule(static)
    for (int64_t hi = 0; hi < 65536; hi++) {
        for (uint32_t lo = 0; lo < 65536; lo++) {
            const uint32_t b = (static_cast<uint32_t>(hi) << 16) | lo;
            const uint16_t f = tvq::f16_encode_fast(b);
            bad_ref += (f != tvq::f16_encode_ref(b));
            if (static_cast<uint64_t>(b) % stride == 0) {
                float x;
                std::memcpy(&x, &b, 4);
                checked_oracle++;
                bad_oracle += (f != static_cast<uint16_t>(oracle(x)));
            }
        }
    }
    std::printf("all 2^32 patterns: %" PRIu64 " differ from the step-by-step form; %" PRIu64
                " oracle checks: %" PRIu64 " differ\n", bad_ref, checked_oracle, bad_oracle);
    return (bad_ref == 0 && bad_oracle == 0) ? 0 : 1;
}
