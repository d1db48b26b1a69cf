// C-ABI: the algebraic ReLU reduction (reduce_activation_layer_algebraic,
// gkr/prover.rs:6700-6890), the reference's proof of ReLU layers.
//
// 33 vectors are folded: eq, the input, the indicator b = [x <= (p - 1) / 2] and the 30
// bits of low = x (b = 1) or x - 2^30 (b = 0).  The combined constraint
//   h = e0 b in + e1 b (1 - b) + e2 (in - sum_j 2^j bit_j - 2^30 (1 - b)) + sum_j e_{3+j} bit_j (1 - bit_j)
// (prover.rs:6642-6690, e_j = eta^j) is regrouped as
//   h = e2 in - 2^30 e2 + b (u_b + e0 in - e1 b) + sum_j bit_j (u_j - e_{3+j} bit_j),
//   u_b = e1 + 2^30 e2,  u_j = e_{3+j} - 2^j e2,
// and every pair adds eq(t) h(t) in coefficient form (deg3_terms.cuh), so each round
// kernel returns the round polynomial's coefficients; they equal the reference's Newton
// interpolation of s(0..3).
#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "calldata.hpp"
#include "channel.hpp"
#include "context.hpp"
#include "deg3_terms.cuh"
#include "logup_device.cuh"
#include "relu.hpp"

namespace zk {

namespace {

constexpr int RELU_BITS = 30;
constexpr int RELU_NV = 3 + RELU_BITS;  // eq, input, indicator, bits

struct ReluConsts {
    qm31 u_b, g_b, e_b;  // indicator term (g_b = -e0)
    qm31 u[RELU_BITS], e[RELU_BITS];
    qm31 e2, lin0;       // linear part e2 in - 2^30 e2
};

// V[v * stride + idx] for the 33 vectors of the padded rows x cols input; V[0] (eq) is
// written by the eq-table launch.
__global__ void relu_prepare_kernel(const uint32_t* __restrict__ in, uint32_t rows, uint32_t cols, size_t pc,
                                    size_t n, uint4* __restrict__ V, size_t stride, uint32_t* __restrict__ err) {
    uint32_t bad = 0;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < n; idx += (size_t)gridDim.x * blockDim.x) {
        const size_t i = idx / pc, j = idx % pc;
        uint32_t x = 0;
        if (i < rows && j < cols) {
            x = in[i * cols + j];
            bad |= x;
            x = red32(x);
        }
        const bool nonneg = x <= (P - 1) / 2;
        const uint32_t low = nonneg ? x : x - (1u << 30);
        V[stride + idx] = make_uint4(x, 0, 0, 0);
        V[2 * stride + idx] = make_uint4(nonneg ? 1u : 0u, 0, 0, 0);
#pragma unroll
        for (int b = 0; b < RELU_BITS; b++) V[(3 + b) * stride + idx] = make_uint4((low >> b) & 1u, 0, 0, 0);
    }
    if (bad & 0x80000000u) atomicOr(err, 1u);
}

// One round: with FOLD, fold all vectors 2h -> h in place first; then add the pairs
// (i, i + h/2) (without FOLD: h is the current length).  16 words: c0..c3.
template <bool FOLD>
__global__ void __launch_bounds__(256, 2) relu_round_kernel(uint4* __restrict__ V, size_t stride, size_t h,
                                                            const AlphaRows m, const ReluConsts c, ReduceScratch rs) {
    const size_t q = h / 2;
    qm31 kacc[4] = {qzero(), qzero(), qzero(), qzero()};
    const qm31 one = qm(1, 0, 0, 0);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < q; i += (size_t)gridDim.x * blockDim.x) {
        auto pair_of = [&](int v, qm31& lo, qm31& hi) {
            uint4* b = V + v * stride;
            if (FOLD) {
                lo = fold_qq(ldq4(b + i), ldq4(b + i + h), m);
                hi = fold_qq(ldq4(b + i + q), ldq4(b + i + q + h), m);
                stq4(b + i, lo);
                stq4(b + i + q, hi);
            } else {
                lo = ldq4(b + i);
                hi = ldq4(b + i + q);
            }
        };
        qm31 e0, e1, in0, in1, b0, b1;
        pair_of(0, e0, e1);
        pair_of(1, in0, in1);
        pair_of(2, b0, b1);
        const qm31 eD = qsub(e1, e0), inD = qsub(in1, in0);
        PwAcc a;
        qacc_zero(a.H0);
        qacc_zero(a.H1);
        qacc_zero(a.H2);
        qacc_mul(a.H0, c.e2, in0);
        qacc_mul(a.H0, c.lin0, one);
        qacc_mul(a.H1, c.e2, inD);
        pw_term(a, b0, qsub(b1, b0), c.u_b, &c.g_b, c.e_b, in0, inD);
#pragma unroll 1
        for (int j = 0; j < RELU_BITS; j++) {
            qm31 x0, x1;
            pair_of(3 + j, x0, x1);
            pw_term(a, x0, qsub(x1, x0), c.u[j], nullptr, c.e[j], in0, inD);
        }
        const qm31 h0 = qacc_value(a.H0), h1 = qacc_value(a.H1), h2 = qacc_value(a.H2);
        kacc[0] = qadd(kacc[0], qmul_fr(e0, h0));
        kacc[1] = qadd(kacc[1], qadd(qmul_fr(e0, h1), qmul_fr(eD, h0)));
        kacc[2] = qadd(kacc[2], qadd(qmul_fr(e0, h2), qmul_fr(eD, h1)));
        kacc[3] = qadd(kacc[3], qmul_fr(eD, h2));
    }
    unsigned long long words[16];
#pragma unroll
    for (int t = 0; t < 4; t++) {
        words[4 * t] = kacc[t].a;
        words[4 * t + 1] = kacc[t].b;
        words[4 * t + 2] = kacc[t].c;
        words[4 * t + 3] = kacc[t].d;
    }
    grid_reduce<16>(words, rs);
}

// Last fold (length 2 -> 1) of the 32 non-eq vectors: input, indicator, bits (128 words).
__global__ void relu_final_kernel(const uint4* V, size_t stride, qm31 alpha, uint32_t* out) {
    const int v = threadIdx.x + 1;
    if (blockIdx.x != 0 || v >= RELU_NV) return;
    const qm31 a = ldq4(V + v * stride), b = ldq4(V + v * stride + 1);
    const qm31 r = qadd(a, qmul(alpha, qsub(b, a)));
    out[4 * (v - 1)] = r.a;
    out[4 * (v - 1) + 1] = r.b;
    out[4 * (v - 1) + 2] = r.c;
    out[4 * (v - 1) + 3] = r.d;
}

inline size_t np2(size_t x) {
    size_t p = 1;
    while (p < x) p <<= 1;
    return p;
}
inline unsigned lg2(size_t x) {
    unsigned l = 0;
    while (((size_t)1 << (l + 1)) <= x) l++;
    return l;
}
inline qm31 ldw(const uint32_t* p) { return qm(p[0], p[1], p[2], p[3]); }

}  // namespace

int relu_reduce_dev(zkml_ctx* ctx, const uint32_t* input, size_t rows, size_t cols, const qm31* point,
                    const qm31& claim_value, zkml_channel* chs, Out& o, qm31* next_point, qm31* next_value,
                    bool legacy_record) {
    const size_t pc = np2(cols), n = np2(rows) * pc;
    const unsigned num_vars = lg2(n);
    if (num_vars == 0) return set_error(ZKML_ERR_INVALID_ARG, "activation input needs at least 2 padded elements");
    if (num_vars > MAX_EQ_VARS || n > ((size_t)1 << 32)) return set_error(ZKML_ERR_INVALID_ARG, "activation too large");
    cudaStream_t s = ctx->stream;
    const void* Iv = nullptr;
    int rc = device_view(ctx, input, rows * cols * 4, ctx->a_in, &Iv);
    if (rc) return rc;
    LogupScratch& b = ctx->lu;
    if ((rc = b.pv.ensure(RELU_NV * n * 16)) || (rc = b.outv.ensure(RELU_NV * 16))) return rc;
    uint4* V = b.pv.as<uint4>();
    {
        const unsigned g = (unsigned)std::min<size_t>((n + 255) / 256, (size_t)ctx->num_sms * 16);
        relu_prepare_kernel<<<g, 256, 0, s>>>(static_cast<const uint32_t*>(Iv), (uint32_t)rows, (uint32_t)cols, pc, n,
                                               V, n, ctx->err_flag());
    }
    launch_eq_table(point, num_vars, V, n, s);
    ctx->launches += 2;

    Channel ch(chs);
    ch.mix_u64(0x414354);
    ch.mix_qm31(claim_value);
    const qm31 eta = ch.draw_qm31();
    qm31 ep[RELU_NV];
    ep[0] = qone();
    for (int i = 1; i < RELU_NV; i++) ep[i] = qmul(ep[i - 1], eta);
    ReluConsts c;
    const uint32_t two30 = 1u << 30;
    c.u_b = qadd(ep[1], qmul_m(ep[2], two30));
    c.g_b = qsub(qzero(), ep[0]);
    c.e_b = ep[1];
    for (int j = 0; j < RELU_BITS; j++) {
        c.u[j] = qsub(ep[3 + j], qmul_m(ep[2], 1u << j));
        c.e[j] = ep[3 + j];
    }
    c.e2 = ep[2];
    c.lin0 = qsub(qzero(), qmul_m(ep[2], two30));
    if ((rc = read_err_flag(ctx)) || (rc = check_err_flag(ctx, "reduce_activation_relu"))) return rc;

    RoundScratch rs = ctx->round_scratch();
    rs.sig = ctx->d_sig;
    auto grid = [&](size_t work) {
        size_t g = (work + 255) / 256;
        if (g > (size_t)ctx->max_round_blocks) g = ctx->max_round_blocks;
        return (unsigned)(g ? g : 1);
    };
    uint32_t words[16];
    std::vector<qm31> rps(4 * num_vars);
    size_t len = n;
    rs.seq = ++ctx->sig_seq;
    relu_round_kernel<false><<<grid(len / 2), 256, 0, s>>>(V, n, len, alpha_rows(qzero()), c, rs);
    ctx->launches++;
    ZK_CUDA(cudaGetLastError());
    for (unsigned r = 0; r < num_vars; r++) {
        if ((rc = wait_signal(ctx, rs.seq, words, 16))) return rc;
        for (int t = 0; t < 4; t++) rps[4 * r + t] = ldw(words + 4 * t);
        ch.mix_poly_coeffs_deg3(rps[4 * r], rps[4 * r + 1], rps[4 * r + 2], rps[4 * r + 3]);
        next_point[r] = ch.draw_qm31();
        if (len == 2) {
            relu_final_kernel<<<1, 32, 0, s>>>(V, n, next_point[r], b.outv.as<uint32_t>());
        } else {
            rs.seq = ++ctx->sig_seq;
            relu_round_kernel<true><<<grid(len / 4), 256, 0, s>>>(V, n, len / 2, alpha_rows(next_point[r]), c, rs);
        }
        ctx->launches++;
        ZK_CUDA(cudaGetLastError());
        len /= 2;
    }
    uint32_t fin[4 * (RELU_NV - 1)];
    ZK_CUDA(cudaMemcpyAsync(fin, b.outv.ptr, sizeof(fin), cudaMemcpyDeviceToHost, s));
    ZK_CUDA(cudaStreamSynchronize(s));
    for (int v = 0; v < RELU_NV - 1; v++) ch.mix_qm31(ldw(fin + 4 * v));
    const qm31 input_eval = ldw(fin);
    *next_value = input_eval;

    // LayerProof::Activation with the activation product proof (cairo_serde.rs:1355-1387, 1190-1235)
    const uint64_t zero[4] = {0, 0, 0, 0};
    o.u64(3);
    o.u64(1);  // ReLU type tag
    o.q(input_eval);
    o.q(claim_value);
    o.push(zero);
    o.u64(0);                    // no LogUp proof
    if (!legacy_record) o.u64(0);  // no multiplicity sumcheck
    o.u64(1);                    // activation product proof
    o.u64(num_vars);
    for (unsigned r = 0; r < num_vars; r++) {
        o.q(rps[4 * r]);
        o.q(rps[4 * r + 2]);
        o.q(rps[4 * r + 3]);
    }
    o.q(input_eval);
    o.q(ldw(fin + 4));  // indicator
    o.u64(1);
    o.u64(RELU_BITS);
    for (int j = 0; j < RELU_BITS; j++) o.q(ldw(fin + 8 + 4 * j));
    if (!legacy_record) o.u64(0);  // no piecewise proof
    return ZKML_OK;
}

}  // namespace zk

using namespace zk;

extern "C" int zkml_reduce_activation_relu(zkml_ctx* ctx, const uint32_t* input, size_t rows, size_t cols,
                                           const uint32_t* claim_point, size_t n_point, const uint32_t claim_value[4],
                                           zkml_channel* chs, uint64_t* out_calldata, size_t cap, size_t* out_len,
                                           uint32_t out_input_eval[4], uint32_t* out_point) {
    if (!ctx || !input || !claim_value || !chs || !out_len) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    if (rows == 0 || cols == 0) return set_error(ZKML_ERR_INVALID_ARG, "empty activation input");
    const unsigned num_vars = lg2(np2(rows) * np2(cols));
    if (n_point != num_vars || !claim_point)
        return set_error(ZKML_ERR_INVALID_ARG, "claim point must have log2(padded size) = " +
                                                   std::to_string(num_vars) + " variables");
    ZK_CUDA(cudaSetDevice(ctx->device));
    Out o{out_calldata, out_calldata ? cap : 0};
    std::vector<qm31> nxt(num_vars + 1);
    qm31 value;
    int rc = relu_reduce_dev(ctx, input, rows, cols, reinterpret_cast<const qm31*>(claim_point),
                             qm(claim_value[0], claim_value[1], claim_value[2], claim_value[3]), chs, o, nxt.data(),
                             &value, false);
    if (rc) return rc;
    *out_len = o.len;
    if (out_input_eval) memcpy(out_input_eval, &value, 16);
    if (out_point) memcpy(out_point, nxt.data(), 16 * num_vars);
    if (o.overflow)
        return set_error(ZKML_ERR_INVALID_ARG, "calldata buffer too small: need " + std::to_string(o.len) + " felts");
    return ZKML_OK;
}
