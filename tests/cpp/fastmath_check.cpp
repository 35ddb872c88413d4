// Host build of the device exponential core (emel.rs_b200/csrc/fastmath.cuh):
// sweeps binary32 inputs with a stride and counts results that differ from
// binary64 libm rounded once to binary32.  Prints "n diffs_exp diffs_expm1
// diffs_tanh max_ulp".
#include <climits>
#include <cstdio>
#include <cstdlib>

#include "fastmath.cuh"

static long long ord(float f) {
    int i;
    std::memcpy(&i, &f, 4);
    return i < 0 ? (long long)INT_MIN - i : i;
}

int main(int argc, char** argv) {
    const unsigned stride = argc > 1 ? (unsigned)std::strtoul(argv[1], nullptr, 10) : 9973u;
    long n = 0, diffs[3] = {0, 0, 0};
    long long worst = 0;
    for (unsigned long long u = 0; u <= 0xffffffffull; u += stride) {
        const unsigned w = (unsigned)u;
        float x;
        std::memcpy(&x, &w, 4);
        if (!(std::fabs(x) <= 90.0f)) continue;
        ++n;
        const float got[3] = {emel::fast_expf(x), emel::fast_expm1f(x), emel::fast_tanhf(x)};
        const float want[3] = {(float)std::exp((double)x), (float)std::expm1((double)x), (float)std::tanh((double)x)};
        for (int k = 0; k < 3; ++k) {
            const long long d = llabs(ord(got[k]) - ord(want[k]));
            if (d) {
                ++diffs[k];
                if (d > worst) worst = d;
            }
        }
    }
    std::printf("%ld %ld %ld %ld %lld\n", n, diffs[0], diffs[1], diffs[2], worst);
    return 0;
}
