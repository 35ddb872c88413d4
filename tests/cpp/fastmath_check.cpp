// Host build of the device exponential cores (emel.rs_b200/csrc/fastmath.cuh).
//   (default) / "edges": the binary64 core; sweeps binary32 inputs with a
//     stride (every sign and exponent: saturation, infinities and NaNs
//     included) and counts results that differ from binary64 libm rounded
//     once to binary32.  Prints "n diffs_exp diffs_expm1 diffs_tanh max_ulp".
//   "b32 <stride>": the binary32 core over the same strided sweep; prints
//     "n max_ulp_exp max_ulp_expm1 max_ulp_tanh nan_mismatches" against
//     binary64 libm rounded once.
//   "gelu": the reference's GELU (binary16 round trips, unary.rs:533-539)
//     with the binary32 tanh against the same formula with glibc's tanhf,
//     for every binary16 input; prints "inputs max_binary16_steps".
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
static void b32_sweep(unsigned stride) {
    long long n32 = 0, worst32[3] = {0, 0, 0}, nan_bad = 0;
    for (unsigned long long u = 0; u <= 0xffffffffull; u += stride) {
        const unsigned b = (unsigned)u;
        float x;
        std::memcpy(&x, &b, 4);
        ++n32;
        const float got[3] = {emel::exp32(x), emel::expm1_32(x), emel::tanh32(x)};
        const float want[3] = {(float)std::exp((double)x), (float)std::expm1((double)x), (float)std::tanh((double)x)};
        for (int k = 0; k < 3; ++k) {
            if (std::isnan(want[k]) || std::isnan(got[k])) {
                if (!(std::isnan(want[k]) && std::isnan(got[k]))) ++nan_bad;
                continue;
            }
            const long long d = llabs(ord(got[k]) - ord(want[k]));
            if (d > worst32[k]) worst32[k] = d;
        }
    }
    std::printf("%lld %lld %lld %lld %lld\n", n32, worst32[0], worst32[1], worst32[2], nan_bad);
}

static float round_half(float v) { return (float)(_Float16)v; }

static int half_ord(float v) {
    const _Float16 h = (_Float16)v;
    short s;
    std::memcpy(&s, &h, 2);
    return s < 0 ? -(s & 0x7fff) : s;
}

template <typename T>
static float gelu_ref(float v, T tanh_fn) {
    if (v <= -10.0f) return 0.0f;
    if (v >= 10.0f) return v;
    const float q = round_half(v);
    const float cube = 0.044715f * q * q * q;
    const float inner = 0.7978846f * (q + cube);
    return round_half((0.5f * q) * (1.0f + tanh_fn(inner)));
}

static void gelu_steps() {
    int worst = 0, inputs = 0;
    for (int h = 0; h < 65536; ++h) {
        const unsigned short hb = (unsigned short)h;
        _Float16 hv;
        std::memcpy(&hv, &hb, 2);
        const float v = (float)hv;
        if (std::isnan(v)) continue;
        ++inputs;
        const float want = gelu_ref(v, [](float x) { return tanhf(x); });
        const float got = gelu_ref(v, [](float x) { return emel::tanh32(x); });
        const int d = std::abs(half_ord(got) - half_ord(want));
        if (d > worst) worst = d;
    }
    std::printf("%d %d\n", inputs, worst);
}

// "gate <stride>": sigmoid 1 / (1 + e) and silu x / (1 + e) with e the
// device's gate exponential (exp32_gate(-x)) against the same formulas on
// binary64 exp rounded once, every stride-th binary32 input plus every input
// of the band -x in [15, 104] where 1 + e rounds; prints
// "n max_ulp_sigmoid max_ulp_silu".
static void gate_sweep(unsigned stride) {
    long n = 0;
    long long worst[2] = {0, 0};
    auto one = [&](float x) {
        if (std::isnan(x)) return;
        ++n;
        const float e = emel::exp32_gate(-x), ec = (float)std::exp(-(double)x);
        const float got[2] = {1.0f / (1.0f + e), x / (1.0f + e)};
        const float want[2] = {1.0f / (1.0f + ec), x / (1.0f + ec)};
        for (int k = 0; k < 2; ++k) {
            if (std::isnan(got[k]) || std::isnan(want[k])) {
                if (std::isnan(got[k]) != std::isnan(want[k])) worst[k] = LLONG_MAX;
                continue;
            }
            const long long d = std::llabs(ord(got[k]) - ord(want[k]));
            if (d > worst[k]) worst[k] = d;
        }
    };
    for (unsigned long long u = 0; u < (1ull << 32); u += stride) {
        const unsigned b = (unsigned)u;
        float x;
        std::memcpy(&x, &b, 4);
        one(x);
    }
    for (unsigned b = 0xc1700000u; b <= 0xc2d00000u; ++b) {  // -15 .. -104
        float x;
        std::memcpy(&x, &b, 4);
        one(x);
    }
    std::printf("%ld %lld %lld\n", n, worst[0], worst[1]);
}

int main(int argc, char** argv) {
    if (argc > 1 && std::string(argv[1]) == "gate") {
        gate_sweep(argc > 2 ? (unsigned)std::strtoul(argv[2], nullptr, 10) : 61u);
        return 0;
    }
    if (argc > 1 && std::string(argv[1]) == "b32") {
        b32_sweep(argc > 2 ? (unsigned)std::strtoul(argv[2], nullptr, 10) : 61u);
        return 0;
    }
    if (argc > 1 && std::string(argv[1]) == "gelu") {
        gelu_steps();
        return 0;
    }
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
