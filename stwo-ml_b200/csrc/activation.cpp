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
