// Host build of the device exponential core (emel.rs_b200/csrc/fastmath.cuh):
// sweeps binary32 inputs with a stride (every sign and exponent: saturation,
// infinities and NaNs included) and counts results that differ from binary64
// libm rounded once to binary32.  Prints "n diffs_exp diffs_expm1
// diffs_tanh max_ulp".
#include <climits>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "fastmath.cuh"

static long long ord(float f) {
    int i;
    std::memcpy(&i, &f, 4);
    return i < 0 ? (long long)INT_MIN - i : i;
}

static long n = 0, diffs[3] = {0, 0, 0};
static long long worst = 0;

static void check(float x) {
        ++n;
        const float got[3] = {emel::fast_expf(x), emel::fast_expm1f(x), emel::fast_tanhf(x)};
        const float want[3] = {(float)std::exp((double)x), (float)std::expm1((double)x), (float)std::tanh((double)x)};
        for (int k = 0; k < 3; ++k) {
            if (std::isnan(want[k]) || std::isnan(got[k])) {  // NaN in, NaN out (payload is the caller's business)
                if (!(std::isnan(want[k]) && std::isnan(got[k]))) {
                    ++diffs[k];
                    worst = LLONG_MAX;
                }
                continue;
            }
            const long long d = llabs(ord(got[k]) - ord(want[k]));
            if (d) {
                ++diffs[k];
                if (d > worst) worst = d;
            }
        }
}

static void check_window(float lo, float hi) {  // every binary32 in [lo, hi], lo < hi, same sign
    for (float x = lo; x <= hi; x = std::nextafter(x, INFINITY)) check(x);
}

// "edges": every binary32 in windows around the saturation thresholds (exp
// 89 / -104, expm1 -18, tanh +-10) and around zero; otherwise a stride over
// all 2^32 bit patterns.
int main(int argc, char** argv) {
    if (argc > 1 && std::string(argv[1]) == "edges") {
        const float w[][2] = {{88.0f, 90.0f}, {-105.0f, -103.0f}, {-19.0f, -17.0f}, {9.0f, 11.0f},
                              {-11.0f, -9.0f}, {-1e-38f, 1e-38f}, {-20.0f, -19.0f}};
        for (const auto& r : w) check_window(r[0], r[1]);
    } else {
        const unsigned stride = argc > 1 ? (unsigned)std::strtoul(argv[1], nullptr, 10) : 9973u;
        for (unsigned long long u = 0; u <= 0xffffffffull; u += stride) {
            const unsigned b = (unsigned)u;
            float x;
            std::memcpy(&x, &b, 4);
            check(x);
        }
    }
    std::printf("%ld %ld %ld %ld %lld\n", n, diffs[0], diffs[1], diffs[2], worst);
    return 0;
}
