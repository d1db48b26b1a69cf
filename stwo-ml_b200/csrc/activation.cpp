// Activation lookup tables for the LogUp activation layer.
//
// Semantics of the engine's table functions (gadgets/lookup_table.rs:193-345;
// table sizes and type tags in components/activation.rs:39-96): inputs are
// M31 values read in fixed point with scale 2^16, values above (P-1)/2 count
// as negative; GELU and SiLU are evaluated in binary64 and rounded half away
// from zero.  The reference evaluates these with the platform libm in plain
// IEEE order, so this file is compiled without floating-point contraction
// (-ffp-contract=off) and uses the same libm, giving identical tables.
#include <cmath>
#include <cstdint>
#include <mutex>
#include <vector>

namespace zk {

namespace {

constexpr uint64_t kP = (1ull << 31) - 1;
constexpr uint32_t kHalfP = (1u << 30) - 1;
constexpr double kScale = 65536.0;

double to_real(uint32_t v) {
    return v <= kHalfP ? (double)v / kScale : -((double)(kP - (uint64_t)v)) / kScale;
}

uint32_t from_real(double r) {
    if (r >= 0.0) {
        const uint64_t u = (uint64_t)std::round(r * kScale);
        return (uint32_t)(u < kP - 1 ? u : kP - 1);
    }
    uint64_t neg = (uint64_t)std::round(-r * kScale);
    if (neg > kP - 1) neg = kP - 1;
    return (uint32_t)(kP - neg);
}

uint32_t relu(uint32_t v) { return v <= kHalfP ? v : 0; }

uint32_t gelu(uint32_t v) {
    if (v == 0) return 0;
    const double x = to_real(v);
    const double k = std::sqrt(2.0 / 3.14159265358979311599796346854);
    const double inner = k * (x + 0.044715 * x * x * x);
    return from_real(0.5 * x * (1.0 + std::tanh(inner)));
}

uint32_t sigmoid_step(uint32_t v) {
    if (v > kHalfP) return 0;
    return v == 0 ? 32768u : 65536u;
}

uint32_t softmax_exp(uint32_t v) {
    const uint32_t scale = 1u << 16;
    if (v > kHalfP) {
        const uint32_t neg = ((1u << 31) - 2) - v;
        uint32_t decay = neg / scale;
        if (decay > 20) decay = 20;
        const uint32_t r = scale >> decay;
        return r > 1 ? r : 1;
    }
    if (v == 0) return scale;
    uint32_t growth = v / scale;
    if (growth > 10) growth = 10;
    const uint64_t r = (uint64_t)scale << growth;
    const uint64_t cap = (1ull << 31) - 2;
    return (uint32_t)(r < cap ? r : cap);
}

uint32_t silu(uint32_t v) {
    if (v == 0) return 0;
    const double x = to_real(v);
    return from_real(x / (1.0 + std::exp(-x)));
}

}  // namespace

// recommended_table_log_size (components/activation.rs:39-47)
unsigned activation_table_log_size(int tag) { return tag == 4 ? 20u : 16u; }

bool activation_tag_valid(int tag) { return tag >= 1 && tag <= 5; }

// Host table for a type tag (1 ReLU, 2 GELU, 3 Sigmoid, 4 Softmax, 5 SiLU), built once.
const std::vector<uint32_t>& activation_table(int tag) {
    static std::once_flag once[6];
    static std::vector<uint32_t> tables[6];
    std::call_once(once[tag], [tag] {
        const size_t n = (size_t)1 << activation_table_log_size(tag);
        std::vector<uint32_t>& t = tables[tag];
        t.resize(n);
        for (size_t i = 0; i < n; i++) {
            const uint32_t v = (uint32_t)i;
            switch (tag) {
                case 1: t[i] = relu(v); break;
                case 2: t[i] = gelu(v); break;
                case 3: t[i] = sigmoid_step(v); break;
                case 4: t[i] = softmax_exp(v); break;
                default: t[i] = silu(v); break;
            }
        }
    });
    return tables[tag];
}

// sigmoid_integer (components/integer_math.rs:288-315); C++ division truncates like Rust's.
static int64_t sigmoid_int(int64_t x, int64_t scale) {
    const int64_t x5 = scale * 5, x25 = scale * 5 / 2;
    if (x <= -x5) return 0;
    if (x >= x5) return scale;
    if (x <= -x25) return ((x + x5) * 28) / (1000 * (x5 - x25) / scale);
    if (x >= x25) return scale * 93 / 100 + ((x - x25) * 7) / (100 * (x5 - x25) / scale);
    return scale / 2 + x / 4;
}

// apply_activation_integer (components/integer_math.rs:212-263) for type tag 1..5
// (ReLU, GELU, Sigmoid, Softmax-exp, SiLU): M31 read as signed fixed point with scale
// (p - 1) / 2, integer-only arithmetic, the result mapped back into [0, p).
uint32_t activation_integer(int tag, uint32_t val) {
    const int64_t P31 = 0x7FFFFFFF, half = P31 / 2;
    const int64_t s = val <= (uint32_t)half ? (int64_t)val : (int64_t)val - P31;
    int64_t r;
    switch (tag) {
        case 1: r = s > 0 ? s : 0; break;
        case 2: r = (s * sigmoid_int((s * 1702) / 1000, half)) / half; break;
        case 3: r = sigmoid_int(s, half); break;
        case 4: {  // exp_activation_integer: Taylor terms until one is below 2 in magnitude
            int64_t res = half + s, term = s;
            for (int64_t k = 2; k <= 8; k++) {
                term = (term * s) / (k * half);
                res += term;
                if ((term < 0 ? -term : term) < 2) break;
            }
            r = res > 0 ? res : 0;
            break;
        }
        case 5: r = (s * sigmoid_int(s, half)) / half; break;
        default: r = s;
    }
    return (uint32_t)(((r % P31) + P31) % P31);
}

namespace {
uint64_t mpow_host(uint64_t b, uint64_t e) {
    uint64_t r = 1;
    b %= kP;
    while (e) {
        if (e & 1) r = r * b % kP;
        b = b * b % kP;
        e >>= 1;
    }
    return r;
}
}  // namespace

// PiecewiseLinearCoeffs::for_activation (components/activation.rs:269-316): segment i of
// width 2^27 (the last one ending at p - 1) is the line through its two end points.
void piecewise_coeffs(int tag, uint32_t slopes[16], uint32_t intercepts[16]) {
    for (uint32_t i = 0; i < 16; i++) {
        const uint64_t xs = (uint64_t)i << 27, xe = i == 15 ? kP - 1 : (((uint64_t)i + 1) << 27) - 1;
        const uint64_t ys = activation_integer(tag, (uint32_t)xs), ye = activation_integer(tag, (uint32_t)xe);
        const uint64_t slope = (ye + kP - ys) % kP * mpow_host((xe + kP - xs) % kP, kP - 2) % kP;
        slopes[i] = (uint32_t)slope;
        intercepts[i] = (uint32_t)((ys + kP - slope * xs % kP) % kP);
    }
}

// rsqrt table of the RMSNorm / LayerNorm lookups (components/layernorm.rs:116-136):
// 0 -> 2^16 - 1, x -> min(2^16 / floor(sqrt(x)), p - 1); 2^16 entries, built once.
const std::vector<uint32_t>& rsqrt_table16() {
    static std::once_flag once;
    static std::vector<uint32_t> t;
    std::call_once(once, [] {
        t.resize((size_t)1 << 16);
        t[0] = (1u << 16) - 1;
        uint64_t s = 1;
        for (uint64_t x = 1; x < t.size(); x++) {
            while ((s + 1) * (s + 1) <= x) s++;  // s = floor(sqrt(x)), non-decreasing in x
            const uint64_t r = (1ull << 16) / s;
            t[x] = (uint32_t)(r < kP - 1 ? r : kP - 1);
        }
    });
    return t;
}

}  // namespace zk

#include "../../include/zkml_b200.h"

extern "C" int zkml_activation_table(int tag, uint32_t* out, size_t cap, size_t* out_len) {
    if (!zk::activation_tag_valid(tag) || !out_len) return ZKML_ERR_INVALID_ARG;
    const std::vector<uint32_t>& t = zk::activation_table(tag);
    *out_len = t.size();
    if (!out || cap < t.size()) return ZKML_ERR_INVALID_ARG;
    for (size_t i = 0; i < t.size(); i++) out[i] = t[i];
    return ZKML_OK;
}
