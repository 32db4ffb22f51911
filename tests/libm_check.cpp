// Compares the restated expf/tanhf (gemma4-rs_b200/csrc/libm_glibc.cuh, host
// instantiation) with this machine's C library on a strided sweep of float
// bit patterns: argv[1] = stride. Prints "<mismatches> <checked>".
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "../gemma4-rs_b200/csrc/libm_glibc.cuh"

extern "C" float expf(float);
extern "C" float tanhf(float);

int main(int argc, char **argv) {
    const unsigned long long stride = argc > 1 ? strtoull(argv[1], nullptr, 10) : 4099;
    long bad = 0, checked = 0;
    for (unsigned long long u = 0; u < (1ull << 32); u += stride) {
        float x;
        const unsigned v = (unsigned)u;
        std::memcpy(&x, &v, 4);
        const float e0 = ::expf(x), e1 = g4a::glibc::expf(x);
        const float t0 = ::tanhf(x), t1 = g4a::glibc::tanhf(x);
        if (std::memcmp(&e0, &e1, 4) && !(std::isnan(e0) && std::isnan(e1))) bad++;
        if (std::memcmp(&t0, &t1, 4) && !(std::isnan(t0) && std::isnan(t1))) bad++;
        checked += 2;
    }
    std::printf("%ld %ld\n", bad, checked);
    return bad != 0;
}
