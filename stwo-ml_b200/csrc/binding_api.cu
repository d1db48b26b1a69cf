// C-ABI: the aggregated weight binding (prove_aggregated_binding_streaming,
// crypto/aggregated_opening.rs:1647-1719) and the weight commitment it binds to.
//
// The reference runs the mismatch sumcheck R(t) = sum_i beta_i eq(g_i, t) (W(t) - v_i)
// claim by claim: every round evaluates the unified oracle W at one point per claim and
// per t in {0, 1, 2} (aggregated_opening.rs:517-625).  Here the same round values come
// from one product sumcheck over two tables of the global hypercube (2^n_global entries):
//   H(t) = sum_i beta_i eq(g_i, t): claim i's scaled eq table of its evaluation point
//          in the first 2^n_i entries of its selector slot (g_i is zero on the slot's
//          higher local bits, so the rest of the slot is zero);
//   W(t) = the unified oracle on the hypercube: slot k holds matrix k's column-major
//          padded MLE repeated 2^(n_max - n_k) times (the oracle ignores the top local
//          variables of a smaller matrix, aggregated_opening.rs:382-386).
// Folding H by the challenges gives sum_i beta_i eq_prefix_i eq(g_i[rest], .), so
// sum_x H(r, X, x) W(r, X, x) is exactly the reference's sum over claims of
// beta_i eq_prefix_i eq(g_i[j], X) W(r, X, g_i[j+1..]); the constant part
// sum_i beta_i eq_prefix_i eq(g_i[j], X) v_i is subtracted on the host before the
// round polynomial is formed.  The last fold of W is the oracle value at the
// challenge point.  The opening then runs on the zero-padded virtual MLE
// (build_virtual_mle_u32, aggregated_opening.rs:654-679) with the device opening prover.
#include <algorithm>
#include <array>
#include <cstring>
#include <string>
#include <vector>

#include "calldata.hpp"
#include "channel.hpp"
#include "context.hpp"
#include "gkr.cuh"
#include "merkle.cuh"
#include "opening.hpp"

namespace zk {

namespace {

inline size_t p2(size_t x) {
    size_t p = 1;
    while (p < x) p <<= 1;
    return p;
}
inline unsigned l2(size_t x) {
    unsigned l = 0;
    while (((size_t)1 << (l + 1)) <= x) l++;
    return l;
}

// dst[i] += beta * src[i] for i < n (QM31, canonical).
__global__ void qm31_axpy_kernel(uint4* __restrict__ dst, const uint4* __restrict__ src, size_t n, qm31 beta) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const uint4 a = src[i], d = dst[i];
        const qm31 r = qadd(qm(d.x, d.y, d.z, d.w), qmul(beta, qm(a.x, a.y, a.z, a.w)));
        dst[i] = make_uint4(r.a, r.b, r.c, r.d);
    }
}

struct BindingRounds {
    const std::vector<std::vector<qm31>>* g;  // global points
    std::vector<qm31> pre;                    // eq_prefix_i
    const std::vector<qm31>* coef;            // beta_i v_i
};

qm31 eq1(const qm31& g, uint32_t x) {  // g x + (1 - g)(1 - x) for x in {0, 1, 2}
    const qm31 X = qm(x, 0, 0, 0);
    return qadd(qmul(g, X), qmul(qsub(qone(), g), qsub(qone(), X)));
}

void binding_adjust(void* arg, unsigned r, uint32_t s12[12]) {
    BindingRounds* b = static_cast<BindingRounds*>(arg);
    for (uint32_t x = 0; x < 3; x++) {
        qm31 c = qzero();
        for (size_t i = 0; i < b->pre.size(); i++)
            c = qadd(c, qmul(qmul(b->pre[i], eq1((*b->g)[i][r], x)), (*b->coef)[i]));
        const qm31 v = qsub(qm(s12[4 * x], s12[4 * x + 1], s12[4 * x + 2], s12[4 * x + 3]), c);
        s12[4 * x] = v.a;
        s12[4 * x + 1] = v.b;
        s12[4 * x + 2] = v.c;
        s12[4 * x + 3] = v.d;
    }
}

void binding_challenge(void* arg, unsigned r, const qm31& alpha) {
    BindingRounds* b = static_cast<BindingRounds*>(arg);
    for (size_t i = 0; i < b->pre.size(); i++) {
        const qm31 g = (*b->g)[i][r];
        b->pre[i] = qmul(b->pre[i], qadd(qmul(alpha, g), qmul(qsub(qone(), alpha), qsub(qone(), g))));
    }
}

}  // namespace
}  // namespace zk

using namespace zk;

extern "C" {

int zkml_weight_commitment(zkml_ctx* ctx, const uint32_t* weight, size_t rows, size_t cols, uint64_t out_root[4]) {
    if (!ctx || !weight || !out_root || rows == 0 || cols == 0)
        return set_error(ZKML_ERR_INVALID_ARG, "NULL or empty argument");
    if (rows > (1u << 30) || cols > (1u << 30) || p2(rows) * p2(cols) > ((size_t)1 << 32))
        return set_error(ZKML_ERR_INVALID_ARG, "weight matrix too large");
    ZK_CUDA(cudaSetDevice(ctx->device));
    cudaStream_t s = ctx->stream;
    const size_t pr = p2(rows), pc = p2(cols), n = pr * pc;
    const void* B = nullptr;
    int rc = device_view(ctx, weight, rows * cols * 4, ctx->b_in, &B);
    if (rc) return rc;
    DevBuf& mle = ctx->op.bmle;
    if ((rc = mle.ensure(n * 16)) || (rc = ctx->op.nodes.ensure(merkle_node_count(n) * 32))) return rc;
    launch_colmajor_mle(static_cast<const uint32_t*>(B), (uint32_t)rows, (uint32_t)cols, pr, pc, mle.as<uint4>(), s);
    launch_merkle_tree(mle.as<uint4>(), n, ctx->op.nodes.ptr, ctx->num_sms, s);
    ctx->launches += 1 + merkle_tree_launches(n);
    uint32_t root[8];
    ZK_CUDA(cudaMemcpyAsync(root, ctx->op.nodes.as<char>() + 32 * (merkle_node_count(n) - 1), 32,
                            cudaMemcpyDeviceToHost, s));
    ZK_CUDA(cudaStreamSynchronize(s));
    felt f;
    memcpy(f.l, root, 32);
    f_to_canon(f, out_root);
    return ZKML_OK;
}

int zkml_prove_aggregated_binding(zkml_ctx* ctx, const zkml_weight_claim* claims, size_t n_claims, zkml_channel* chs,
                                  size_t n_queries, uint64_t* out_calldata, size_t cap, size_t* out_len) {
    if (!ctx || !claims || !chs || !out_len) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    if (n_claims == 0 || n_claims > 256) return set_error(ZKML_ERR_INVALID_ARG, "need 1 to 256 weight claims");
    // AggregatedBindingConfig::from_claims (aggregated_opening.rs:68-97)
    std::vector<unsigned> nv(n_claims);
    std::vector<size_t> pr(n_claims), pc(n_claims);
    unsigned n_max = 0;
    for (size_t i = 0; i < n_claims; i++) {
        const zkml_weight_claim& c = claims[i];
        if (!c.weight || c.rows == 0 || c.cols == 0 || c.rows > (1u << 30) || c.cols > (1u << 30))
            return set_error(ZKML_ERR_INVALID_ARG, "claim " + std::to_string(i) + ": bad weight matrix");
        pr[i] = p2(c.rows);
        pc[i] = p2(c.cols);
        nv[i] = l2(pr[i] * pc[i]);
        if (nv[i] == 0) return set_error(ZKML_ERR_INVALID_ARG, "claim " + std::to_string(i) + ": 1 x 1 weight");
        if (!c.eval_point) return set_error(ZKML_ERR_INVALID_ARG, "claim " + std::to_string(i) + ": NULL point");
        n_max = nv[i] > n_max ? nv[i] : n_max;
    }
    const size_t m_padded = p2(n_claims);
    const unsigned sb = l2(m_padded), n_global = sb + n_max;
    if (n_global > 32 || n_global > MAX_EQ_VARS)
        return set_error(ZKML_ERR_INVALID_ARG, "virtual oracle too large (2^" + std::to_string(n_global) + ")");
    ZK_CUDA(cudaSetDevice(ctx->device));
    cudaStream_t s = ctx->stream;
    felt_init();

    // build_super_root (aggregated_opening.rs:181-227)
    std::vector<std::array<uint64_t, 4>> zr(n_max + 1), sub(m_padded);
    f_to_canon(felt_of_qm31(qzero()), zr[0].data());
    for (unsigned l = 1; l <= n_max; l++) poseidon_hash_canon(zr[l - 1].data(), zr[l - 1].data(), zr[l].data());
    for (size_t i = 0; i < m_padded; i++) {
        if (i >= n_claims) {
            sub[i] = zr[n_max];
            continue;
        }
        memcpy(sub[i].data(), claims[i].commitment, 32);
        for (unsigned l = nv[i]; l < n_max; l++) poseidon_hash_canon(sub[i].data(), zr[l].data(), sub[i].data());
    }
    std::vector<std::array<uint64_t, 4>> lvl(sub);
    while (lvl.size() > 1) {
        for (size_t i = 0; i < lvl.size() / 2; i++) poseidon_hash_canon(lvl[2 * i].data(), lvl[2 * i + 1].data(), lvl[i].data());
        lvl.resize(lvl.size() / 2);
    }
    const std::array<uint64_t, 4> root = lvl[0];
    Channel ch(chs);
    ch.mix_m(f_from_canon(root.data()));
    // draw_beta_weights (aggregated_opening.rs:395-405)
    const qm31 rho = ch.draw_qm31();
    std::vector<qm31> beta(n_claims), coef(n_claims);
    std::vector<std::vector<qm31>> g(n_claims, std::vector<qm31>(n_global));
    {
        qm31 pw = qone();
        for (size_t i = 0; i < n_claims; i++) {
            beta[i] = pw;
            pw = qmul(pw, rho);
            const uint32_t* v = claims[i].expected_value;
            coef[i] = qmul(beta[i], qm(v[0], v[1], v[2], v[3]));
            // global_point (aggregated_opening.rs:328-358)
            for (unsigned j = 0; j < sb; j++) g[i][j] = qm((uint32_t)((claims[i].matrix_index >> (sb - 1 - j)) & 1), 0, 0, 0);
            for (unsigned j = 0; j < n_max - nv[i]; j++) g[i][sb + j] = qzero();
            const uint32_t* e = claims[i].eval_point;
            for (unsigned j = 0; j < nv[i]; j++)
                g[i][sb + n_max - nv[i] + j] = qm(e[4 * j], e[4 * j + 1], e[4 * j + 2], e[4 * j + 3]);
        }
    }

    // the two tables of the mismatch sumcheck
    const size_t N = (size_t)1 << n_global, slot = (size_t)1 << n_max;
    int rc;
    if ((rc = ctx->fa.ensure(N * 16)) || (rc = ctx->fb.ensure(N * 16)) || (rc = ctx->lu.eq.ensure(slot * 16)))
        return rc;
    uint4* H = ctx->fa.as<uint4>();
    uint4* W = ctx->fb.as<uint4>();
    ZK_CUDA(cudaMemsetAsync(H, 0, N * 16, s));
    ZK_CUDA(cudaMemsetAsync(W, 0, N * 16, s));
    for (size_t i = 0; i < n_claims; i++) {
        const void* B = nullptr;
        if ((rc = device_view(ctx, claims[i].weight, claims[i].rows * claims[i].cols * 4, ctx->b_in, &B))) return rc;
        uint4* ws = W + i * slot;
        launch_colmajor_mle(static_cast<const uint32_t*>(B), (uint32_t)claims[i].rows, (uint32_t)claims[i].cols,
                            pr[i], pc[i], ws, s);
        for (size_t len = (size_t)1 << nv[i]; len < slot; len *= 2)
            ZK_CUDA(cudaMemcpyAsync(ws + len, ws, len * 16, cudaMemcpyDeviceToDevice, s));
        const size_t hs = claims[i].matrix_index & (m_padded - 1);
        const size_t ne = (size_t)1 << nv[i];
        launch_eq_table(reinterpret_cast<const qm31*>(claims[i].eval_point), (int)nv[i], ctx->lu.eq.as<uint4>(), ne,
                        s);
        const unsigned grid = (unsigned)std::min<size_t>((ne + 255) / 256, (size_t)ctx->num_sms * 8);
        qm31_axpy_kernel<<<grid, 256, 0, s>>>(H + hs * slot, ctx->lu.eq.as<uint4>(), ne, beta[i]);
        ctx->launches += 3;
        ZK_CUDA(cudaGetLastError());
    }
    if ((rc = read_err_flag(ctx)) || (rc = check_err_flag(ctx, "prove_aggregated_binding"))) return rc;

    // mismatch sumcheck (aggregated_opening.rs:412-510)
    BindingRounds br{&g, std::vector<qm31>(n_claims, qone()), &coef};
    ClaimHook hook{nullptr, &br};
    hook.adjust = binding_adjust;
    hook.challenge = binding_challenge;
    std::vector<uint32_t> rps(12 * n_global), chal(4 * n_global);
    uint32_t h_fin[4], w_fin[4];
    if ((rc = run_sumcheck(ctx, H, W, nullptr, nullptr, N, chs, rps.data(), chal.data(), h_fin, w_fin, &hook)))
        return rc;
    const qm31 oracle_eval = qm(w_fin[0], w_fin[1], w_fin[2], w_fin[3]);
    ch.mix_felts(&oracle_eval, 1);

    // serialize_aggregated_binding_proof (cairo_serde.rs:3884-3921)
    Out o{out_calldata, out_calldata ? cap : 0};
    o.u64(sb);
    o.u64(n_max);
    o.u64(m_padded);
    o.u64(n_global);
    o.u64(n_claims);
    o.u64(n_global);
    for (size_t j = 0; j < 3 * (size_t)n_global; j++) o.qm(&rps[4 * j]);
    o.q(oracle_eval);
    o.push(root.data());
    o.u64(m_padded);
    for (size_t i = 0; i < m_padded; i++) o.push(sub[i].data());

    // the zero-padded virtual MLE, opened at the challenge point against the super-root
    ZK_CUDA(cudaMemsetAsync(W, 0, N * 16, s));
    for (size_t i = 0; i < n_claims; i++) {
        const void* B = nullptr;
        if ((rc = device_view(ctx, claims[i].weight, claims[i].rows * claims[i].cols * 4, ctx->b_in, &B))) return rc;
        launch_colmajor_mle(static_cast<const uint32_t*>(B), (uint32_t)claims[i].rows, (uint32_t)claims[i].cols,
                            pr[i], pc[i], W + i * slot, s);
        ctx->launches++;
    }
    uint64_t com[4];
    {
        KTimer t(ctx, KC_MERKLE);
        rc = prove_opening_dev(ctx, W, n_global, reinterpret_cast<const qm31*>(chal.data()), chs, n_queries, com, o,
                               nullptr);
    }
    if (rc) return rc;
    if (memcmp(com, root.data(), 32) != 0)
        return set_error(ZKML_ERR_INVALID_ARG, "weight commitments do not match the weight matrices");
    *out_len = o.len;
    if (o.overflow)
        return set_error(ZKML_ERR_INVALID_ARG, "calldata buffer too small: need " + std::to_string(o.len) + " felts");
    return ZKML_OK;
}

}  // extern "C"
