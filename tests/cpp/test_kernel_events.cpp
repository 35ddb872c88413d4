// C++ mirror of the reference's own unit tests, run through the device op
// table: each case restates a known answer from
// crates/emel-kernels/tests/any/{binary_ops,broadcast_ops,normalization_ops,
// reductions,softmax_ops,flash_attn_ops}.rs with the same inputs, events and
// expected values.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <vector>

#include "emel_kernels_cuda.hpp"

using namespace emel_kernels::cuda;

static int failures = 0;
#define CHECK(cond, what)                                           \
    do {                                                            \
        if (!(cond)) {                                              \
            std::printf("FAIL %s (%s:%d)\n", what, __FILE__, __LINE__); \
            ++failures;                                             \
        }                                                           \
    } while (0)

static Layout contiguous(std::array<uint64_t, 4> ne) { return *Layout::contiguous(DType::F32, ne); }

struct Buf {
    Buf(Kernel& k, std::vector<float> v) : host(std::move(v)), dev(k, host.size() * 4) { dev.upload(host.data(), host.size() * 4); }
    std::vector<float> read() {
        std::vector<float> out(host.size());
        dev.download(out.data(), out.size() * 4);
        return out;
    }
    TensorView view(Layout l) const { return dev.view(l); }
    std::vector<float> host;
    DeviceBuffer dev;
};

static bool same(const std::vector<float>& a, const std::vector<float>& b) {
    return a.size() == b.size() && std::memcmp(a.data(), b.data(), a.size() * 4) == 0;
}

// binary_ops.rs:18-61: dense formulas
static void binary_formulas(Kernel& k) {
    Buf lhs(k, {1, 2, 3, 4}), rhs(k, {10, 20, 30, 40}), out(k, {0, 0, 0, 0});
    Layout l = contiguous({4, 1, 1, 1});
    CHECK(k.process_event(OpAdd(lhs.view(l), rhs.view(l), out.view(l))).is_ok(), "add ok");
    CHECK(same(out.read(), {11, 22, 33, 44}), "add values");
    CHECK(k.process_event(OpSub(lhs.view(l), rhs.view(l), out.view(l))).is_ok(), "sub ok");
    CHECK(same(out.read(), {-9, -18, -27, -36}), "sub values");
    CHECK(k.process_event(OpMul(lhs.view(l), rhs.view(l), out.view(l))).is_ok(), "mul ok");
    CHECK(same(out.read(), {10, 40, 90, 160}), "mul values");
    CHECK(k.process_event(OpDiv(lhs.view(l), rhs.view(l), out.view(l))).is_ok(), "div ok");
    CHECK(same(out.read(), {0.1f, 0.1f, 0.1f, 0.1f}), "div values");
}

// binary_ops.rs:167: a count mismatch is rejected without writing
static void binary_rejection_does_not_mutate(Kernel& k) {
    Buf lhs(k, {1, 2, 3, 4}), rhs(k, {10, 20, 30, 40}), out(k, {9, 9, 9});
    Result r = k.process_event(OpDiv(lhs.view(contiguous({4, 1, 1, 1})), rhs.view(contiguous({4, 1, 1, 1})),
                                     out.view(contiguous({3, 1, 1, 1}))));
    CHECK(!r.is_ok() && r.error() == BinaryError::ShapeMismatch, "shape mismatch");
    CHECK(same(out.read(), {9, 9, 9}), "untouched");
}

// broadcast_ops.rs:19-62
static void row_broadcast(Kernel& k) {
    Buf src(k, {1, 2, 3, 4, 5, 6}), row(k, {10, 20, 30}), out(k, std::vector<float>(6, 0.0f));
    CHECK(k.process_event(OpAddBroadcastRow(src.view(contiguous({3, 2, 1, 1})), row.view(contiguous({3, 1, 1, 1})),
                                            out.view(contiguous({3, 2, 1, 1})))).is_ok(), "row add ok");
    CHECK(same(out.read(), {11, 22, 33, 14, 25, 36}), "row add values");
    CHECK(k.process_event(OpMulBroadcastRow(src.view(contiguous({3, 2, 1, 1})), row.view(contiguous({3, 1, 1, 1})),
                                            out.view(contiguous({3, 2, 1, 1})))).is_ok(), "row mul ok");
    CHECK(same(out.read(), {10, 40, 90, 40, 100, 180}), "row mul values");
    Buf bad(k, {2, 2});
    Result r = k.process_event(OpAddBroadcastRow(src.view(contiguous({3, 2, 1, 1})), bad.view(contiguous({2, 1, 1, 1})),
                                                 out.view(contiguous({3, 2, 1, 1}))));
    CHECK(!r.is_ok() && r.error() == BroadcastError::ShapeMismatch, "bad row rejected");
}

// normalization_ops.rs:29-73
static void normalization_known_answers(Kernel& k) {
    Buf in(k, {1, 2, 4, 2, 5, 8}), out(k, std::vector<float>(6, 0.0f));
    CHECK(k.process_event(OpNorm(in.view(contiguous({3, 2, 1, 1})), out.view(contiguous({3, 2, 1, 1})), 1.0f)).is_ok(),
          "norm ok");
    CHECK(same(out.read(), {-0.83405757f, -0.20851436f, 1.0425721f, -1.1338935f, 0.0f, 1.1338935f}), "norm values");
    Buf in2(k, {3, 4, 0, 2}), out2(k, {0, 0, 0, 0});
    CHECK(k.process_event(OpRmsNorm(in2.view(contiguous({2, 2, 1, 1})), out2.view(contiguous({2, 2, 1, 1})), 1.0f)).is_ok(),
          "rms ok");
    CHECK(same(out2.read(), {0.8164966f, 1.0886621f, 0.0f, 1.1547005f}), "rms values");
    Result r = k.process_event(OpNorm(in.view(contiguous({3, 2, 1, 1})), out.view(contiguous({3, 2, 1, 1})), NAN));
    CHECK(!r.is_ok() && r.error() == NormalizationError::InvalidParameters, "nan epsilon rejected");
}

// reductions.rs:58-102
static void reductions_known_answers(Kernel& k) {
    Buf in(k, {1, 2, 3, 4, 5, 6}), scalar(k, {0}), rows(k, {0, 0});
    Layout src = contiguous({3, 2, 1, 1}), one = contiguous({1, 1, 1, 1});
    CHECK(k.process_event(OpSum(in.view(src), scalar.view(one))).is_ok() && same(scalar.read(), {21}), "sum");
    CHECK(k.process_event(OpMean(in.view(src), scalar.view(one))).is_ok() && same(scalar.read(), {3.5f}), "mean");
    CHECK(k.process_event(OpArgmax(in.view(src), scalar.view(one))).is_ok() && same(scalar.read(), {5}), "argmax");
    CHECK(k.process_event(OpSumRows(in.view(src), rows.view(contiguous({1, 2, 1, 1})))).is_ok() &&
              same(rows.read(), {6, 15}),
          "sum_rows");
}

// softmax_ops.rs:32-104
static void softmax_rows(Kernel& k) {
    Buf in(k, {1000, 1001, 1002, -1000, -999, -998}), out(k, std::vector<float>(6, 0.0f));
    Layout l = contiguous({3, 2, 1, 1});
    CHECK(k.process_event(OpSoftMax(in.view(l), out.view(l))).is_ok(), "softmax ok");
    auto o = out.read();
    CHECK(std::fabs(o[0] + o[1] + o[2] - 1.0f) < 1e-6f && std::fabs(o[3] + o[4] + o[5] - 1.0f) < 1e-6f, "rows sum to 1");
    CHECK(o[2] > o[1] && o[1] > o[0], "ordered");
    Buf small(k, {1, 2}), dst(k, {9, 9, 9});
    Result r = k.process_event(OpSoftMax(small.view(contiguous({2, 1, 1, 1})), dst.view(contiguous({3, 1, 1, 1}))));
    CHECK(!r.is_ok() && r.error() == ReductionError::ShapeMismatch && same(dst.read(), {9, 9, 9}), "count mismatch");
}

// tools/emel-kernel-flash-attn-parity/src/main.rs:61-104 and its manifest
// (snapshots/parity/kernel-flash-attn): exact output bits; flash_attn_ops.rs:220-250
static void flash_attn_golden(Kernel& k) {
    const std::vector<uint16_t> key{0x3c00, 0, 0, 0, 0, 0x3c00, 0, 0}, value{0x4000, 0x4400, 0x4600, 0x4800};
    DeviceBuffer kb(k, key.size() * 2), vb(k, value.size() * 2);
    kb.upload(key.data(), key.size() * 2);
    vb.upload(value.data(), value.size() * 2);
    Buf q(k, {1, 0, 1, 0}), out(k, std::vector<float>(4, 0.0f));
    Layout ql = contiguous({2, 1, 2, 1});
    Layout kvl = *Layout::contiguous(DType::F16, {2, 2, 1, 1});
    FlashAttnOptions o{1.0f, 2u};
    CHECK(k.process_event(OpFlashAttnExt(q.view(ql), kb.view(kvl), vb.view(kvl), out.view(ql), o)).is_ok(), "attn ok");
    const uint32_t want[4] = {0x4044d668u, 0x40a27a4fu, 0x4044d668u, 0x40a27a4fu};
    auto got = out.read();
    CHECK(std::memcmp(got.data(), want, 16) == 0, "attn golden bits");
    Buf rejected(k, std::vector<float>(4, 9.0f));
    Result r = k.process_event(OpFlashAttnExt(q.view(ql), kb.view(kvl), vb.view(kvl), rejected.view(ql),
                                              FlashAttnOptions{0.0f, 2u}));
    CHECK(!r.is_ok() && r.error() == FlashAttnError::InvalidRequest && same(rejected.read(), {9, 9, 9, 9}),
          "attn invalid scale");
}

int main() {
    Kernel k(0);
    binary_formulas(k);
    binary_rejection_does_not_mutate(k);
    row_broadcast(k);
    normalization_known_answers(k);
    reductions_known_answers(k);
    softmax_rows(k);
    flash_attn_golden(k);
    std::printf("%s: %d failure(s)\n", failures ? "FAILED" : "ok", failures);
    return failures ? 1 : 0;
}
