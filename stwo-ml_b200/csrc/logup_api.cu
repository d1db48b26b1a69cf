// C-ABI: the LogUp activation layer reduction (gkr/prover.rs:6390-6600) on the GPU.
//
// Transcript (host): mix "LOG" tag and the activation type tag, draw gamma and
// beta; mix the trace-side sum; one degree-3 eq-sumcheck round polynomial per
// variable; the multiplicity sumcheck (mix c0, c1; draw); finally the input
// evaluation and the output claim.  Everything data-parallel runs on the GPU;
// each reducing kernel publishes its words through mapped host memory.
#include <cstring>
#include <string>
#include <vector>

#include "calldata.hpp"
#include "channel.hpp"
#include "context.hpp"
#include "logup.cuh"

namespace zk {

unsigned activation_table_log_size(int tag);
bool activation_tag_valid(int tag);
const std::vector<uint32_t>& activation_table(int tag);

namespace {

inline size_t next_pow2(size_t x) {
    size_t p = 1;
    while (p < x) p <<= 1;
    return p;
}
inline unsigned ilog2(size_t x) {
    unsigned l = 0;
    while (((size_t)1 << (l + 1)) <= x) l++;
    return l;
}
inline qm31 ldq(const uint32_t* p) { return qm(p[0], p[1], p[2], p[3]); }

}  // namespace
}  // namespace zk

using namespace zk;

extern "C" int zkml_reduce_activation_logup(zkml_ctx* ctx, const uint32_t* input, size_t rows, size_t cols, int tag,
                                            const uint32_t* claim_point, size_t n_point, const uint32_t claim_value[4],
                                            zkml_channel* chs, uint64_t* out_calldata, size_t cap, size_t* out_len,
                                            uint32_t out_input_eval[4]) {
    if (!ctx || !input || !claim_value || !chs || !out_len) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    if (!activation_tag_valid(tag)) return set_error(ZKML_ERR_INVALID_ARG, "unknown activation type tag");
    if (rows == 0 || cols == 0) return set_error(ZKML_ERR_INVALID_ARG, "empty activation input");
    const size_t pr = next_pow2(rows), pc = next_pow2(cols), n = pr * pc;
    const unsigned num_vars = ilog2(n);
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
    // table (host-built once, cached on the device per context)
    const unsigned log_t = activation_table_log_size(tag);
    const size_t tsize = (size_t)1 << log_t;
    DevBuf& tbuf = ctx->act_tables[tag];
    if (!tbuf.ptr) {
        const std::vector<uint32_t>& t = activation_table(tag);
        if ((rc = tbuf.ensure(tsize * 4))) return rc;
        ZK_CUDA(cudaMemcpy(tbuf.ptr, t.data(), tsize * 4, cudaMemcpyHostToDevice));
    }
    LogupScratch& b = ctx->lu;  // kept across calls: allocation would synchronise the device every call
    if ((rc = b.x.ensure(n * 4)) || (rc = b.m_in.ensure(n * 4)) || (rc = b.m_out.ensure(n * 4)) ||
        (rc = b.mult.ensure(tsize * 4)) || (rc = b.eq.ensure(n * 16)) || (rc = b.d.ensure(n * 16)) ||
        (rc = b.w.ensure(n * 16)) || (rc = b.mv.ensure(tsize / 2 * 16)))
        return rc;
    RoundScratch rs = ctx->round_scratch();
    rs.sig = ctx->d_sig;
    auto next = [&]() { rs.seq = ++ctx->sig_seq; };
    uint32_t words[16];
    Channel ch(chs);
    const qm31* point = reinterpret_cast<const qm31*>(claim_point);

    // masked lookups, multiplicities, and the input evaluation at the claim point
    ZK_CUDA(cudaMemsetAsync(b.mult.ptr, 0, tsize * 4, s));
    launch_eq_table(point, num_vars, b.eq.as<uint4>(), n, s);
    launch_logup_prepare(static_cast<const uint32_t*>(Iv), (uint32_t)rows, (uint32_t)cols, pc, n,
                         (uint32_t)(tsize - 1), tbuf.as<uint32_t>(), b.x.as<uint32_t>(), b.m_in.as<uint32_t>(),
                         b.m_out.as<uint32_t>(), b.mult.as<uint32_t>(), ctx->err_flag(), ctx->max_round_blocks, s);
    next();
    launch_eq_dot(b.eq.as<uint4>(), b.x.as<uint32_t>(), nullptr, n, rs, s);
    ctx->launches += 3;
    // LogUp encoding challenges (overlapping the GPU work above)
    ch.mix_u64(0x4C4F47);
    ch.mix_u64((uint64_t)tag);
    const qm31 gamma = ch.draw_qm31();
    const qm31 beta = ch.draw_qm31();
    if ((rc = wait_signal(ctx, rs.seq, words, 4))) return rc;
    const qm31 input_eval = ldq(words);
    if ((rc = read_err_flag(ctx)) || (rc = check_err_flag(ctx, "reduce_activation_logup"))) return rc;

    // denominators, inverse witnesses and both LogUp sums
    next();
    launch_logup_dw(b.m_in.as<uint32_t>(), b.m_out.as<uint32_t>(), n, gamma, beta, b.d.as<uint4>(), b.w.as<uint4>(),
                    rs, s);
    ctx->launches++;
    if ((rc = wait_signal(ctx, rs.seq, words, 4))) return rc;
    const qm31 trace_sum = ldq(words);
    next();
    launch_logup_table_sum(b.mult.as<uint32_t>(), tbuf.as<uint32_t>(), tsize, gamma, beta, rs, s);
    ctx->launches++;
    if ((rc = wait_signal(ctx, rs.seq, words, 4))) return rc;
    if (!qeq(ldq(words), trace_sum))
        return set_error(ZKML_ERR_VERIFY, "activation LogUp sum mismatch (trace side != table side)");
    ch.mix_qm31(trace_sum);

    // degree-3 eq-sumcheck: sum eq(r, x) w(x) d(x) = 1
    static const uint32_t inv2 = minv(2), inv6 = minv(6);
    std::vector<qm31> rps(4 * num_vars), chal(num_vars);
    size_t len = n;
    next();
    launch_logup_round(b.eq.as<uint4>(), b.w.as<uint4>(), b.d.as<uint4>(), len, false, qzero(), rs, s);
    ctx->launches++;
    for (unsigned r = 0; r < num_vars; r++) {
        if ((rc = wait_signal(ctx, rs.seq, words, 16))) return rc;
        const qm31 s0 = ldq(words), s1 = ldq(words + 4), s2 = ldq(words + 8), s3 = ldq(words + 12);
        const qm31 dd1 = qsub(s1, s0);
        const qm31 dd2 = qmul_m(qadd(qsub(qsub(s2, s1), s1), s0), inv2);
        const qm31 dd3 = qmul_m(qsub(qsub(s3, s0), qmul_m(qsub(s2, s1), 3)), inv6);
        const qm31 c0 = s0, c1 = qadd(qsub(dd1, dd2), qmul_m(dd3, 2)), c2 = qsub(dd2, qmul_m(dd3, 3)), c3 = dd3;
        rps[4 * r] = c0;
        rps[4 * r + 1] = c1;
        rps[4 * r + 2] = c2;
        rps[4 * r + 3] = c3;
        ch.mix_poly_coeffs_deg3(c0, c1, c2, c3);
        chal[r] = ch.draw_qm31();
        next();
        if (len == 2)
            launch_logup_final(b.eq.as<uint4>(), b.w.as<uint4>(), b.d.as<uint4>(), chal[r], rs, s);
        else
            launch_logup_round(b.eq.as<uint4>(), b.w.as<uint4>(), b.d.as<uint4>(), len, true, chal[r], rs, s);
        ctx->launches++;
        len /= 2;
    }
    if ((rc = wait_signal(ctx, rs.seq, words, 4))) return rc;
    const qm31 w_eval = ldq(words);
    // masked input / output MLEs at the sumcheck point
    launch_eq_table(chal.data(), num_vars, b.eq.as<uint4>(), n, s);
    next();
    launch_eq_dot(b.eq.as<uint4>(), b.m_in.as<uint32_t>(), b.m_out.as<uint32_t>(), n, rs, s);
    ctx->launches += 2;
    if ((rc = wait_signal(ctx, rs.seq, words, 8))) return rc;
    const qm31 in_eval_s = ldq(words), out_eval_s = ldq(words + 4);

    // multiplicity sumcheck (prover.rs:9449-9515)
    std::vector<qm31> mrp(2 * log_t);
    qm31 m_claim = qzero(), m_final = qzero();
    size_t mlen = tsize;
    next();
    launch_mult_round(b.mult.as<uint32_t>(), b.mv.as<uint4>(), mlen, true, false, qzero(), rs, s);
    ctx->launches++;
    for (unsigned r = 0; r < log_t; r++) {
        if ((rc = wait_signal(ctx, rs.seq, words, 8))) return rc;
        const qm31 lo = ldq(words), hi = ldq(words + 4);
        if (r == 0) m_claim = qadd(lo, hi);
        const qm31 c0 = lo, c1 = qsub(hi, lo);
        mrp[2 * r] = c0;
        mrp[2 * r + 1] = c1;
        ch.mix_qm31(c0);
        ch.mix_qm31(c1);
        const qm31 x = ch.draw_qm31();
        next();
        if (mlen == 2)
            launch_mult_final(r == 0 ? b.mult.as<uint32_t>() : nullptr, b.mv.as<uint4>(), x, rs, s);
        else
            launch_mult_round(b.mult.as<uint32_t>(), b.mv.as<uint4>(), mlen, r == 0, true, x, rs, s);
        ctx->launches++;
        mlen /= 2;
    }
    if ((rc = wait_signal(ctx, rs.seq, words, 4))) return rc;
    m_final = ldq(words);
    std::vector<uint32_t> mult(tsize);
    ZK_CUDA(cudaMemcpyAsync(mult.data(), b.mult.ptr, tsize * 4, cudaMemcpyDeviceToHost, s));
    ZK_CUDA(cudaStreamSynchronize(s));

    // deterministic table commitment, final mixes
    uint64_t tcom[4];
    {
        const uint64_t in[8] = {(uint64_t)tag, 0, 0, 0, log_t, 0, 0, 0};
        poseidon_hash_many_canon(in, 2, tcom);
    }
    ch.mix_qm31(input_eval);
    ch.mix_qm31(ldq(claim_value));

    // LayerProof::Activation as serialize_gkr_model_proof writes it (cairo_serde.rs:1355-1387)
    Out o{out_calldata, out_calldata ? cap : 0};
    o.u64(3);
    o.u64((uint64_t)tag);
    o.q(input_eval);
    o.q(ldq(claim_value));
    o.push(tcom);
    o.u64(1);
    o.q(trace_sum);
    o.u64(num_vars);
    for (unsigned r = 0; r < num_vars; r++) {
        o.q(rps[4 * r]);
        o.q(rps[4 * r + 2]);
        o.q(rps[4 * r + 3]);
    }
    o.q(w_eval);
    o.q(in_eval_s);
    o.q(out_eval_s);
    o.u64(tsize);
    for (size_t j = 0; j < tsize; j++) o.u64(mult[j]);
    o.u64(1);
    o.u64(log_t);
    for (unsigned r = 0; r < log_t; r++) {
        o.q(mrp[2 * r]);
        o.q(mrp[2 * r + 1]);
    }
    o.q(m_final);
    o.q(m_claim);
    o.u64(0);  // no activation product proof
    o.u64(0);  // no piecewise proof
    *out_len = o.len;
    if (out_input_eval) {
        out_input_eval[0] = input_eval.a;
        out_input_eval[1] = input_eval.b;
        out_input_eval[2] = input_eval.c;
        out_input_eval[3] = input_eval.d;
    }
    if (o.overflow)
        return set_error(ZKML_ERR_INVALID_ARG, "calldata buffer too small: need " + std::to_string(o.len) + " felts");
    return ZKML_OK;
}
