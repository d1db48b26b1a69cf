// C-ABI: the piecewise-linear algebraic activation reduction
// (reduce_activation_layer_piecewise, gkr/prover.rs:7006-7228), the reference's default
// proof for GELU, Sigmoid, Softmax-exp and SiLU layers.
//
// The reference folds 23 vectors (eq, input, output, 16 segment indicators, 4 segment
// bits) and evaluates the combined constraint
//   h = e0 (out - sum_i I_i (a_i in + b_i)) + e1 (sum_i I_i - 1) + sum_i e_{2+i} I_i (1 - I_i)
//       + e18 (sum_k 2^k B_k - sum_i i I_i) + sum_k e_{19+k} B_k (1 - B_k)     (e_j = eta^j)
// at t = 0, 1, 2, 3 for every pair (prover.rs:6935-6998).  Here h is regrouped as
//   h = L - in G - Q,  L = sum_i u_i I_i + sum_k w_k B_k + e0 out - e1,  G = sum_i g_i I_i,
//   Q = sum_i e_{2+i} I_i^2 + sum_k e_{19+k} B_k^2
// (u_i = e1 + e_{2+i} - i e18 - e0 b_i, g_i = e0 a_i, w_k = 2^k e18 + e_{19+k}), i.e.
//   h = e0 out - e1 + sum_i I_i (u_i - g_i in - e_{2+i} I_i) + sum_k B_k (w_k - e_{19+k} B_k);
// every vector
// is linear in t over a pair, so each pair contributes the cubic eq(t) h(t) in coefficient
// form and the kernel returns the round polynomial's coefficients (c0..c3) directly; they
// equal the reference's Newton interpolation of s(0..3) because a cubic is determined by
// four values.  Round 0 derives every vector from the raw input (segment = top 4 bits);
// round 1 folds from the raw input into 23 QM31 vectors; later rounds fold those in place.
#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "calldata.hpp"
#include "channel.hpp"
#include "context.hpp"
#include "deg3_terms.cuh"
#include "logup_device.cuh"

namespace zk {

void piecewise_coeffs(int tag, uint32_t slopes[16], uint32_t intercepts[16]);
bool activation_tag_valid(int tag);

namespace {

constexpr int PW_NV = 23;  // eq, input, output, 16 indicators, 4 segment bits

struct PwConsts {
    qm31 u[16], g[16], e[16];  // per indicator
    qm31 w[4], f[4];           // per segment bit
    qm31 eta0, neg_eta1;
    uint32_t slope[16], icpt[16];
};

// Folded rounds with at least this many pairs run one thread per pair (throughput); shorter
// ones one warp per pair (latency: a pair is ~10k dependent instructions for one thread).
constexpr size_t PW_THREAD_MIN_PAIRS = (size_t)1 << 16;

__device__ __forceinline__ uint32_t pw_seg(uint32_t x) { return min(x >> 27, 15u); }

// Folded rounds (2 and later), one thread per pair: each of the 23 vectors is folded
// 2h -> h in place and its pair (i, i + q), q = h / 2, is added to h(t).
__global__ void __launch_bounds__(256, 2) pw_round_kernel(uint4* __restrict__ V, size_t stride, size_t h,
                                                          const AlphaRows m, const PwConsts c, ReduceScratch rs) {
    const size_t q = h / 2;
    qm31 kacc[4] = {qzero(), qzero(), qzero(), qzero()};  // this thread's coefficient sums
    const qm31 one = qm(1, 0, 0, 0);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < q; i += (size_t)gridDim.x * blockDim.x) {
        auto pair_of = [&](int v, qm31& lo, qm31& hi) {
            uint4* b = V + v * stride;
            lo = fold_qq(ldq4(b + i), ldq4(b + i + h), m);
            hi = fold_qq(ldq4(b + i + q), ldq4(b + i + q + h), m);
            stq4(b + i, lo);
            stq4(b + i + q, hi);
        };
        qm31 e0, e1, in0, in1, o0, o1;
        pair_of(0, e0, e1);
        pair_of(1, in0, in1);
        pair_of(2, o0, o1);
        const qm31 eD = qsub(e1, e0), inD = qsub(in1, in0);
        PwAcc a;
        qacc_zero(a.H0);
        qacc_zero(a.H1);
        qacc_zero(a.H2);
        qacc_mul(a.H0, c.eta0, o0);
        qacc_mul(a.H1, c.eta0, qsub(o1, o0));
        qacc_mul(a.H0, c.neg_eta1, one);
#pragma unroll 1
        for (int s = 0; s < 16; s++) {
            qm31 x0, x1;
            pair_of(3 + s, x0, x1);
            pw_term(a, x0, qsub(x1, x0), c.u[s], &c.g[s], c.e[s], in0, inD);
        }
#pragma unroll 1
        for (int k = 0; k < 4; k++) {
            qm31 x0, x1;
            pair_of(19 + k, x0, x1);
            pw_term(a, x0, qsub(x1, x0), c.w[k], nullptr, c.f[k], in0, inD);
        }
        const qm31 h0 = qacc_value(a.H0), h1 = qacc_value(a.H1), h2 = qacc_value(a.H2);
        kacc[0] = qadd(kacc[0], qmul_f(e0, h0));
        kacc[1] = qadd(kacc[1], qadd(qmul_f(e0, h1), qmul_f(eD, h0)));
        kacc[2] = qadd(kacc[2], qadd(qmul_f(e0, h2), qmul_f(eD, h1)));
        kacc[3] = qadd(kacc[3], qmul_f(eD, h2));
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

// Rounds 0 and 1 read the raw input: the indicators and segment bits are 0/1 there
// (round 0) or fold two 0/1 values (round 1), so only the segments a pair touches (at
// most 2 or 4 of the 16) contribute, and in round 0 every term is a signed sum of
// constants and M31 multiples of constants (no QM31 products but the eq ones).
__device__ __forceinline__ qm31 qneg(const qm31& x) { return qsub(qzero(), x); }
__device__ __forceinline__ qm31 qsign(int s, const qm31& x) { return s > 0 ? x : (s < 0 ? qneg(x) : qzero()); }

// Round 0 term of an indicator / segment bit with 0/1 values x0 (lo), x1 (hi).
__device__ __forceinline__ void pw_term01(qm31 (&H)[3], int x0, int x1, const qm31& u, const qm31* g,
                                          const qm31& e, uint32_t in0, uint32_t ind) {
    const int xd = x1 - x0;
    qm31 y0 = x0 ? qsub(u, e) : u;
    qm31 yd = qsign(-xd, e);
    if (g) {
        y0 = qsub(y0, qmul_m(*g, in0));
        yd = qsub(yd, qmul_m(*g, ind));
    }
    if (x0) {
        H[0] = qadd(H[0], y0);
        H[1] = qadd(H[1], yd);
    }
    H[1] = qadd(H[1], qsign(xd, y0));
    H[2] = qadd(H[2], qsign(xd, yd));
}

__device__ __forceinline__ void pw_term_h(qm31 (&H)[3], const qm31& x0, const qm31& xd, const qm31& u, const qm31* g,
                                        const qm31& e, const qm31& in0, const qm31& ind) {
    qm31 y0 = qsub(u, qmul_f(e, x0)), yd = qneg(qmul_f(e, xd));
    if (g) {
        y0 = qsub(y0, qmul_f(*g, in0));
        yd = qsub(yd, qmul_f(*g, ind));
    }
    H[0] = qadd(H[0], qmul_f(x0, y0));
    H[1] = qadd(H[1], qadd(qmul_f(x0, yd), qmul_f(xd, y0)));
    H[2] = qadd(H[2], qmul_f(xd, yd));
}

template <bool FOLD>
__global__ void __launch_bounds__(256) pw_raw_kernel(const uint32_t* __restrict__ x32, const uint4* __restrict__ E,
                                                     uint4* __restrict__ V, size_t stride, size_t h, const AlphaRows m,
                                                     qm31 alpha, const PwConsts c, ReduceScratch rs) {
    // !FOLD: pairs (i, i + h/2) of the raw length-h input; FOLD: the raw input has length 2h
    // and is folded into V (length h) while the pairs (i, i + h/2) are summed.
    const size_t q = h / 2;
    qm31 kacc[4] = {qzero(), qzero(), qzero(), qzero()};
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < q; i += (size_t)gridDim.x * blockDim.x) {
        qm31 H[3] = {qzero(), qzero(), qzero()};
        qm31 e0, eD;
        if (!FOLD) {
            const uint32_t xa = x32[i], xb = x32[i + q];
            const uint32_t sa = pw_seg(xa), sb = pw_seg(xb);
            e0 = ldq4(E + i);
            eD = qsub(ldq4(E + i + q), e0);
            const uint32_t ind = csub(xb, xa);
            const uint32_t oa = madd(mmul(c.slope[sa], xa), c.icpt[sa]), ob = madd(mmul(c.slope[sb], xb), c.icpt[sb]);
            H[0] = qadd(qmul_m(c.eta0, oa), c.neg_eta1);
            H[1] = qmul_m(c.eta0, csub(ob, oa));
            pw_term01(H, 1, sa == sb, c.u[sa], &c.g[sa], c.e[sa], xa, ind);
            if (sb != sa) pw_term01(H, 0, 1, c.u[sb], &c.g[sb], c.e[sb], xa, ind);
#pragma unroll
            for (int k = 0; k < 4; k++)
                pw_term01(H, (sa >> k) & 1, (sb >> k) & 1, c.w[k], nullptr, c.f[k], xa, ind);
        } else {
            const uint32_t xr[4] = {x32[i], x32[i + q], x32[i + h], x32[i + q + h]};
            uint32_t sg[4], o[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                sg[j] = pw_seg(xr[j]);
                o[j] = madd(mmul(c.slope[sg[j]], xr[j]), c.icpt[sg[j]]);
            }
            e0 = fold_qq(ldq4(E + i), ldq4(E + i + h), m);
            const qm31 e1 = fold_qq(ldq4(E + i + q), ldq4(E + i + q + h), m);
            eD = qsub(e1, e0);
            stq4(V + i, e0);
            stq4(V + i + q, e1);
            const qm31 in0 = fold_mq(xr[0], xr[2], alpha), in1 = fold_mq(xr[1], xr[3], alpha);
            stq4(V + stride + i, in0);
            stq4(V + stride + i + q, in1);
            const qm31 inD = qsub(in1, in0);
            const qm31 o0 = fold_mq(o[0], o[2], alpha), o1 = fold_mq(o[1], o[3], alpha);
            stq4(V + 2 * stride + i, o0);
            stq4(V + 2 * stride + i + q, o1);
            H[0] = qadd(qmul_f(c.eta0, o0), c.neg_eta1);
            H[1] = qmul_f(c.eta0, qsub(o1, o0));
#pragma unroll 1
            for (int sI = 0; sI < 16; sI++) {
                const uint32_t su = (uint32_t)sI;
                const bool l0 = sg[0] == su, l2 = sg[2] == su, h1 = sg[1] == su, h3 = sg[3] == su;
                const qm31 lo = fold_mq(l0, l2, alpha), hi = fold_mq(h1, h3, alpha);
                stq4(V + (3 + sI) * stride + i, lo);
                stq4(V + (3 + sI) * stride + i + q, hi);
                if (l0 | l2 | h1 | h3) pw_term_h(H, lo, qsub(hi, lo), c.u[sI], &c.g[sI], c.e[sI], in0, inD);
            }
#pragma unroll 1
            for (int k = 0; k < 4; k++) {
                const qm31 lo = fold_mq((sg[0] >> k) & 1, (sg[2] >> k) & 1, alpha);
                const qm31 hi = fold_mq((sg[1] >> k) & 1, (sg[3] >> k) & 1, alpha);
                stq4(V + (19 + k) * stride + i, lo);
                stq4(V + (19 + k) * stride + i + q, hi);
                pw_term_h(H, lo, qsub(hi, lo), c.w[k], nullptr, c.f[k], in0, inD);
            }
        }
        kacc[0] = qadd(kacc[0], qmul_f(e0, H[0]));
        kacc[1] = qadd(kacc[1], qadd(qmul_f(e0, H[1]), qmul_f(eD, H[0])));
        kacc[2] = qadd(kacc[2], qadd(qmul_f(e0, H[2]), qmul_f(eD, H[1])));
        kacc[3] = qadd(kacc[3], qmul_f(eD, H[2]));
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

// Folded rounds with one warp per pair: lane v < 23 folds vector v (lo at index i, hi at
// i + q) and adds its term of h; the eq and input values are broadcast from lanes 0 and 1,
// and lane 0 combines the warp's h with eq into the cubic.  A pair's work is spread over 23
// lanes, so the short rounds at the end (a few pairs) do not run one long dependent chain
// per thread.
__global__ void __launch_bounds__(256) pw_fold_warp_kernel(uint4* __restrict__ V, size_t stride, size_t h,
                                                           const AlphaRows m, const PwConsts c, ReduceScratch rs) {
    const size_t q = h / 2;
    const int lane = threadIdx.x & 31;
    const size_t w0 = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
    const size_t nw = ((size_t)gridDim.x * blockDim.x) >> 5;
    qm31 kacc[4] = {qzero(), qzero(), qzero(), qzero()};
    for (size_t i = w0; i < q; i += nw) {
        qm31 lo = qzero(), hi = qzero();
        if (lane < PW_NV) {
            uint4* b = V + lane * stride;
            lo = fold_qq(ldq4(b + i), ldq4(b + i + h), m);
            hi = fold_qq(ldq4(b + i + q), ldq4(b + i + q + h), m);
            stq4(b + i, lo);
            stq4(b + i + q, hi);
        }
        const qm31 d = qsub(hi, lo);
        auto bcast = [&](const qm31& v, int src) {
            return qm(__shfl_sync(0xffffffffu, v.a, src), __shfl_sync(0xffffffffu, v.b, src),
                      __shfl_sync(0xffffffffu, v.c, src), __shfl_sync(0xffffffffu, v.d, src));
        };
        const qm31 in0 = bcast(lo, 1), inD = bcast(d, 1);
        qm31 H[3] = {qzero(), qzero(), qzero()};
        if (lane == 2) {
            H[0] = qadd(qmul_f(c.eta0, lo), c.neg_eta1);
            H[1] = qmul_f(c.eta0, d);
        } else if (lane >= 3 && lane < PW_NV) {
            qm31 y0, yd;
            if (lane < 19) {
                const int s = lane - 3;
                y0 = qsub(qsub(c.u[s], qmul_f(c.e[s], lo)), qmul_f(c.g[s], in0));
                yd = qsub(qsub(qzero(), qmul_f(c.e[s], d)), qmul_f(c.g[s], inD));
            } else {
                const int k = lane - 19;
                y0 = qsub(c.w[k], qmul_f(c.f[k], lo));
                yd = qsub(qzero(), qmul_f(c.f[k], d));
            }
            H[0] = qmul_f(lo, y0);
            H[1] = qadd(qmul_f(lo, yd), qmul_f(d, y0));
            H[2] = qmul_f(d, yd);
        }
#pragma unroll
        for (int t = 0; t < 3; t++)
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) H[t] = qadd(H[t], bcast(H[t], lane ^ off));
        if (lane == 0) {
            const qm31 e0 = lo, eD = d;
            kacc[0] = qadd(kacc[0], qmul_f(e0, H[0]));
            kacc[1] = qadd(kacc[1], qadd(qmul_f(e0, H[1]), qmul_f(eD, H[0])));
            kacc[2] = qadd(kacc[2], qadd(qmul_f(e0, H[2]), qmul_f(eD, H[1])));
            kacc[3] = qadd(kacc[3], qmul_f(eD, H[2]));
        }
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

// Last fold (length 2 -> 1) of the 22 non-eq vectors: input, output, 16 indicators,
// 4 segment bits (88 words to out).
__global__ void pw_final_kernel(const uint32_t* x32, const uint4* V, size_t stride, qm31 alpha, const PwConsts c,
                                uint32_t* out) {
    const int v = threadIdx.x + 1;
    if (blockIdx.x != 0 || v >= PW_NV) return;
    qm31 r;
    if (x32) {
        const uint32_t a = x32[0], b = x32[1];
        auto val = [&](uint32_t x) -> uint32_t {
            const uint32_t s = pw_seg(x);
            if (v == 1) return x;
            if (v == 2) return madd(mmul(c.slope[s], x), c.icpt[s]);
            if (v < 19) return s == (uint32_t)(v - 3) ? 1u : 0u;
            return (s >> (v - 19)) & 1u;
        };
        r = fold_mq(val(a), val(b), alpha);
    } else {
        const qm31 a = ldq4(V + v * stride), b = ldq4(V + v * stride + 1);
        r = qadd(a, qmul(alpha, qsub(b, a)));
    }
    out[4 * (v - 1)] = r.a;
    out[4 * (v - 1) + 1] = r.b;
    out[4 * (v - 1) + 2] = r.c;
    out[4 * (v - 1) + 3] = r.d;
}

// Zero-padded, canonical row-major input (the padded matrix_to_mle order).
__global__ void pw_pad_kernel(const uint32_t* __restrict__ in, uint32_t rows, uint32_t cols, size_t pc, size_t n,
                              uint32_t* __restrict__ out, uint32_t* __restrict__ err) {
    uint32_t bad = 0;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < n; idx += (size_t)gridDim.x * blockDim.x) {
        const size_t i = idx / pc, j = idx % pc;
        uint32_t x = 0;
        if (i < rows && j < cols) {
            x = in[i * cols + j];
            bad |= x;
            x = red32(x);
        }
        out[idx] = x;
    }
    if (bad & 0x80000000u) atomicOr(err, 1u);
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
}  // namespace zk

using namespace zk;

extern "C" int zkml_reduce_activation_piecewise(zkml_ctx* ctx, const uint32_t* input, size_t rows, size_t cols,
                                                int tag, const uint32_t* claim_point, size_t n_point,
                                                const uint32_t claim_value[4], zkml_channel* chs,
                                                uint64_t* out_calldata, size_t cap, size_t* out_len,
                                                uint32_t out_input_eval[4], uint32_t* out_point) {
    if (!ctx || !input || !claim_value || !chs || !out_len) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    if (!activation_tag_valid(tag)) return set_error(ZKML_ERR_INVALID_ARG, "unknown activation type tag");
    if (rows == 0 || cols == 0) return set_error(ZKML_ERR_INVALID_ARG, "empty activation input");
    const size_t pc = np2(cols), n = np2(rows) * pc;
    const unsigned num_vars = lg2(n);
    if (num_vars == 0) return set_error(ZKML_ERR_INVALID_ARG, "activation input needs at least 2 padded elements");
    if (n_point != num_vars || !claim_point)
        return set_error(ZKML_ERR_INVALID_ARG, "claim point must have log2(padded size) = " +
                                                   std::to_string(num_vars) + " variables");
    if (num_vars > MAX_EQ_VARS || n > ((size_t)1 << 32)) return set_error(ZKML_ERR_INVALID_ARG, "activation too large");
    ZK_CUDA(cudaSetDevice(ctx->device));
    cudaStream_t s = ctx->stream;
    const void* Iv = nullptr;
    int rc = device_view(ctx, input, rows * cols * 4, ctx->a_in, &Iv);
    if (rc) return rc;
    LogupScratch& b = ctx->lu;
    const size_t stride = n / 2 > 0 ? n / 2 : 1;
    if ((rc = b.x.ensure(n * 4)) || (rc = b.eq.ensure(n * 16)) || (rc = b.pv.ensure(PW_NV * stride * 16)) ||
        (rc = b.outv.ensure(PW_NV * 16)))
        return rc;
    RoundScratch rs = ctx->round_scratch();
    rs.sig = ctx->d_sig;
    auto next = [&]() { rs.seq = ++ctx->sig_seq; };
    uint32_t words[16];
    Channel ch(chs);
    const qm31* point = reinterpret_cast<const qm31*>(claim_point);

    {
        const unsigned g = (unsigned)std::min<size_t>((n + 255) / 256, (size_t)ctx->num_sms * 16);
        pw_pad_kernel<<<g, 256, 0, s>>>(static_cast<const uint32_t*>(Iv), (uint32_t)rows, (uint32_t)cols, pc, n,
                                         b.x.as<uint32_t>(), ctx->err_flag());
    }
    launch_eq_table(point, num_vars, b.eq.as<uint4>(), n, s);
    ctx->launches += 2;

    // transcript: "PW_ACT", type tag, num_vars, the claim; eta and the constraint constants
    ch.mix_u64(0x50575F414354ull);
    ch.mix_u64((uint64_t)tag);
    ch.mix_u64(num_vars);
    ch.mix_qm31(ldw(claim_value));
    const qm31 eta = ch.draw_qm31();
    qm31 ep[23];
    ep[0] = qone();
    for (int i = 1; i < 23; i++) ep[i] = qmul(ep[i - 1], eta);
    PwConsts c;
    piecewise_coeffs(tag, c.slope, c.icpt);
    for (int i = 0; i < 16; i++) {
        c.g[i] = qmul_m(ep[0], c.slope[i]);
        c.e[i] = ep[2 + i];
        c.u[i] = qsub(qsub(qadd(ep[1], ep[2 + i]), qmul_m(ep[18], (uint32_t)i)), qmul_m(ep[0], c.icpt[i]));
    }
    for (int k = 0; k < 4; k++) {
        c.w[k] = qadd(qmul_m(ep[18], 1u << k), ep[19 + k]);
        c.f[k] = ep[19 + k];
    }
    c.eta0 = ep[0];
    c.neg_eta1 = qsub(qzero(), ep[1]);
    if ((rc = read_err_flag(ctx)) || (rc = check_err_flag(ctx, "reduce_activation_piecewise"))) return rc;

    auto grid = [&](size_t work) {
        size_t g = (work + 255) / 256;
        if (g > (size_t)ctx->max_round_blocks) g = ctx->max_round_blocks;
        return (unsigned)(g ? g : 1);
    };
    std::vector<qm31> rps(4 * num_vars), chal(num_vars);
    size_t len = n;
    next();
    pw_raw_kernel<false><<<grid(len / 2), 256, 0, s>>>(b.x.as<uint32_t>(), b.eq.as<uint4>(), b.pv.as<uint4>(),
                                                       stride, len, alpha_rows(qzero()), qzero(), c, rs);
    ctx->launches++;
    ZK_CUDA(cudaGetLastError());
    for (unsigned r = 0; r < num_vars; r++) {
        if ((rc = wait_signal(ctx, rs.seq, words, 16))) return rc;
        const qm31 c0 = ldw(words), c1 = ldw(words + 4), c2 = ldw(words + 8), c3 = ldw(words + 12);
        rps[4 * r] = c0;
        rps[4 * r + 1] = c1;
        rps[4 * r + 2] = c2;
        rps[4 * r + 3] = c3;
        ch.mix_poly_coeffs_deg3(c0, c1, c2, c3);
        chal[r] = ch.draw_qm31();
        if (len == 2) {
            pw_final_kernel<<<1, 32, 0, s>>>(r == 0 ? b.x.as<uint32_t>() : nullptr, b.pv.as<uint4>(), stride, chal[r],
                                             c, b.outv.as<uint32_t>());
        } else {
            next();
            const size_t h = len / 2;
            if (r == 0)
                pw_raw_kernel<true><<<grid(h / 2), 256, 0, s>>>(b.x.as<uint32_t>(), b.eq.as<uint4>(),
                                                                b.pv.as<uint4>(), stride, h, alpha_rows(chal[r]),
                                                                chal[r], c, rs);
            else if (h / 2 >= PW_THREAD_MIN_PAIRS)
                pw_round_kernel<<<grid(h / 2), 256, 0, s>>>(b.pv.as<uint4>(), stride, h, alpha_rows(chal[r]), c, rs);
            else
                pw_fold_warp_kernel<<<grid(h / 2 * 32), 256, 0, s>>>(b.pv.as<uint4>(), stride, h, alpha_rows(chal[r]),
                                                                    c, rs);
        }
        ctx->launches++;
        ZK_CUDA(cudaGetLastError());
        len /= 2;
    }
    uint32_t fin[88];
    ZK_CUDA(cudaMemcpyAsync(fin, b.outv.ptr, sizeof(fin), cudaMemcpyDeviceToHost, s));
    ZK_CUDA(cudaStreamSynchronize(s));
    for (int v = 0; v < 22; v++) ch.mix_qm31(ldw(fin + 4 * v));
    const qm31 input_eval = ldw(fin);

    // LayerProof::Activation with the piecewise proof (cairo_serde.rs:1355-1387, 1249-1300)
    Out o{out_calldata, out_calldata ? cap : 0};
    const uint64_t zero[4] = {0, 0, 0, 0};
    o.u64(3);
    o.u64((uint64_t)tag);
    o.q(input_eval);
    o.q(ldw(claim_value));
    o.push(zero);
    o.u64(0);  // no LogUp proof
    o.u64(0);  // no multiplicity sumcheck
    o.u64(0);  // no activation product proof
    o.u64(1);  // piecewise proof
    o.u64(num_vars);
    for (unsigned r = 0; r < num_vars; r++) {
        o.q(rps[4 * r]);
        o.q(rps[4 * r + 2]);
        o.q(rps[4 * r + 3]);
    }
    for (int v = 0; v < 18; v++) o.q(ldw(fin + 4 * v));  // input, output, 16 indicators
    o.u64(1);                                              // segment bits present
    for (int v = 18; v < 22; v++) o.q(ldw(fin + 4 * v));
    *out_len = o.len;
    if (out_input_eval) memcpy(out_input_eval, fin, 16);
    if (out_point) memcpy(out_point, chal.data(), 16 * num_vars);
    if (o.overflow)
        return set_error(ZKML_ERR_INVALID_ARG, "calldata buffer too small: need " + std::to_string(o.len) + " felts");
    return ZKML_OK;
}
