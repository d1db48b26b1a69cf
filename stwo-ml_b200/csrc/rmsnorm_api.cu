// C-ABI: the RMSNorm layer reduction (reduce_rmsnorm_layer_with_gamma,
// gkr/prover.rs:8424-8790) on the GPU.
//
// Transcript (host), in the reference's order:
//   Part 0  mix "RQ", n_active, sum_x input(x)^2; per variable the plain
//           sumcheck round (c3 = 0) mixed as a degree-3 polynomial, a draw;
//           mix the folded input.  Skipped entirely when STWO_SKIP_RMS_SQ_PROOF
//           is set in the environment (as the reference does).
//   Part 1  mix "RN", rms^2(r), rsqrt(r), the claim; degree-3 eq-sumcheck of
//           eq(r, x) input(x) scale(x); mix the two final values.
//   Part 2  mix "LOG", "RN", draw gamma, beta; the LogUp of (rms^2, rsqrt)
//           pairs against the rsqrt table: trace sum, degree-3 eq-sumcheck of
//           eq w d, the multiplicity sumcheck (transcript only; the record
//           does not carry it); mix input(r), output(r).
// Every data-parallel pass runs on the GPU; reducing kernels publish their words
// through mapped host memory (LogUp kernels + rmsnorm_kernels.cu).
#include <cstdlib>
#include <string>
#include <vector>

#include "calldata.hpp"
#include "channel.hpp"
#include "context.hpp"
#include "logup.cuh"
#include "relu.hpp"

namespace zk {

const std::vector<uint32_t>& rsqrt_table16();

namespace {

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

int zk::rmsnorm_reduce_dev(zkml_ctx* ctx, const uint32_t* input, size_t rows, size_t cols, size_t dim,
                           const uint32_t* gamma, size_t gamma_len, const uint32_t* claim_point, size_t n_point,
                           const uint32_t claim_value[4], zkml_channel* chs, Out& o, uint32_t out_input_eval[4],
                           bool v1_record) {
    if (!ctx || !input || !claim_value || !chs) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    if (rows == 0 || cols == 0 || dim == 0) return set_error(ZKML_ERR_INVALID_ARG, "empty RMSNorm input or dim 0");
    if (gamma && gamma_len == 0) return set_error(ZKML_ERR_INVALID_ARG, "empty gamma");
    const size_t pr = np2(rows), pc = np2(cols), n = pr * pc;
    const unsigned num_vars = lg2(n);
    if (num_vars == 0) return set_error(ZKML_ERR_INVALID_ARG, "RMSNorm input needs at least 2 padded elements");
    if (n_point != num_vars || !claim_point)
        return set_error(ZKML_ERR_INVALID_ARG, "claim point must have log2(padded size) = " +
                                                   std::to_string(num_vars) + " variables");
    if (num_vars > MAX_EQ_VARS || n > ((size_t)1 << 32) || pc > ((size_t)1 << 31))
        return set_error(ZKML_ERR_INVALID_ARG, "RMSNorm input too large");
    const bool skip_rms_sq = getenv("STWO_SKIP_RMS_SQ_PROOF") != nullptr;
    ZK_CUDA(cudaSetDevice(ctx->device));
    cudaStream_t s = ctx->stream;
    const void* Iv = nullptr;
    int rc = device_view(ctx, input, rows * cols * 4, ctx->a_in, &Iv);
    if (rc) return rc;
    LogupScratch& b = ctx->lu;
    const void* Gv = nullptr;
    if (gamma && (rc = device_view(ctx, gamma, gamma_len * 4, b.gam, &Gv))) return rc;
    const unsigned log_t = 16;
    const size_t tsize = (size_t)1 << log_t;
    if (!ctx->rsqrt_table.ptr) {
        if ((rc = ctx->rsqrt_table.ensure(tsize * 4))) return rc;
        ZK_CUDA(cudaMemcpy(ctx->rsqrt_table.ptr, rsqrt_table16().data(), tsize * 4, cudaMemcpyHostToDevice));
    }
    if ((rc = b.x.ensure(n * 4)) || (rc = b.m_in.ensure(n * 4)) || (rc = b.m_out.ensure(n * 4)) ||
        (rc = b.outv.ensure(n * 4)) || (rc = b.mult.ensure(tsize * 4)) || (rc = b.eq.ensure(n * 16)) ||
        (rc = b.d.ensure(n * 16)) || (rc = b.w.ensure(n * 16)) || (rc = b.pv.ensure(n / 2 * 16)) ||
        (rc = b.mv.ensure(tsize / 2 * 16)) || (rc = b.row_rms.ensure(pr * 4)))
        return rc;
    RoundScratch rs = ctx->round_scratch();
    rs.sig = ctx->d_sig;
    auto next = [&]() { rs.seq = ++ctx->sig_seq; };
    uint32_t words[16];
    Channel ch(chs);
    const qm31* point = reinterpret_cast<const qm31*>(claim_point);
    static const uint32_t inv2 = minv(2), inv6 = minv(6);
    const size_t n_active = dim < pc ? dim : pc;
    const uint32_t inv_n = minv((uint32_t)(n_active % P));

    // per-row rms^2 / rsqrt and every vector below; the four evaluations at the claim point
    ZK_CUDA(cudaMemsetAsync(b.mult.ptr, 0, tsize * 4, s));
    launch_rmsnorm_prepare(static_cast<const uint32_t*>(Iv), (uint32_t)rows, (uint32_t)cols, (uint32_t)pr,
                           (uint32_t)pc, (uint32_t)n_active, inv_n, static_cast<const uint32_t*>(Gv),
                           (uint32_t)gamma_len, ctx->rsqrt_table.as<uint32_t>(), (uint32_t)(tsize - 1),
                           b.x.as<uint32_t>(), b.m_in.as<uint32_t>(), b.m_out.as<uint32_t>(), b.outv.as<uint32_t>(),
                           b.w.as<uint4>(), b.d.as<uint4>(), b.row_rms.as<uint32_t>(), b.mult.as<uint32_t>(),
                           ctx->err_flag(), ctx->max_round_blocks, s);
    launch_eq_table(point, num_vars, b.eq.as<uint4>(), n, s);
    next();
    {
        const uint32_t* xs[4] = {b.x.as<uint32_t>(), b.outv.as<uint32_t>(), b.m_in.as<uint32_t>(),
                                 b.m_out.as<uint32_t>()};
        launch_eq_dot(b.eq.as<uint4>(), xs, 4, n, rs, s);
    }
    ctx->launches += 3;
    if ((rc = wait_signal(ctx, rs.seq, words, 16))) return rc;
    const qm31 input_eval = ldw(words), output_eval = ldw(words + 4);
    const qm31 rms_sq_eval = ldw(words + 8), rsqrt_eval = ldw(words + 12);
    if ((rc = read_err_flag(ctx)) || (rc = check_err_flag(ctx, "reduce_rmsnorm"))) return rc;

    // Part 0: plain sumcheck sum_x input(x)^2 = total (prover.rs:8500-8545)
    std::vector<qm31> rq(3 * num_vars);
    qm31 total_sq = qzero(), rq_final = qzero();
    if (!skip_rms_sq) {
        size_t len = n;
        next();
        launch_sq_round(b.x.as<uint32_t>(), b.pv.as<uint4>(), len, true, false, qzero(), rs, s);
        ctx->launches++;
        for (unsigned r = 0; r < num_vars; r++) {
            if ((rc = wait_signal(ctx, rs.seq, words, 12))) return rc;
            const qm31 s0 = ldw(words), s1 = ldw(words + 4), s2 = ldw(words + 8);
            if (r == 0) {
                total_sq = qadd(s0, s1);
                ch.mix_u64(0x5251);
                ch.mix_u64(n_active);
                ch.mix_qm31(total_sq);
            }
            const qm31 dd1 = qsub(s1, s0);
            const qm31 dd2 = qmul_m(qsub(qsub(s2, s1), dd1), inv2);
            const qm31 c0 = s0, c1 = qsub(dd1, dd2), c2 = dd2;
            rq[3 * r] = c0;
            rq[3 * r + 1] = c2;
            rq[3 * r + 2] = qzero();
            ch.mix_poly_coeffs_deg3(c0, c1, c2, qzero());
            const qm31 x = ch.draw_qm31();
            next();
            if (len == 2)
                launch_mult_final(r == 0 ? b.x.as<uint32_t>() : nullptr, b.pv.as<uint4>(), x, rs, s);
            else
                launch_sq_round(b.x.as<uint32_t>(), b.pv.as<uint4>(), len, r == 0, true, x, rs, s);
            ctx->launches++;
            len /= 2;
        }
        if ((rc = wait_signal(ctx, rs.seq, words, 4))) return rc;
        rq_final = ldw(words);
        ch.mix_qm31(rq_final);
    }

    // Part 1: degree-3 eq-sumcheck of eq(r, x) input(x) scale(x) (prover.rs:8560-8630)
    ch.mix_u64(0x524E);
    ch.mix_qm31(rms_sq_eval);
    ch.mix_qm31(rsqrt_eval);
    ch.mix_qm31(ldw(claim_value));
    auto eq_sumcheck = [&](std::vector<qm31>& rps, std::vector<qm31>& chal, qm31* fin_w, qm31* fin_d) -> int {
        size_t len = n;
        next();
        launch_logup_round(b.eq.as<uint4>(), b.w.as<uint4>(), b.d.as<uint4>(), len, false, qzero(), rs, s);
        ctx->launches++;
        for (unsigned r = 0; r < num_vars; r++) {
            int e = wait_signal(ctx, rs.seq, words, 16);
            if (e) return e;
            const qm31 s0 = ldw(words), s1 = ldw(words + 4), s2 = ldw(words + 8), s3 = ldw(words + 12);
            const qm31 dd1 = qsub(s1, s0);
            const qm31 dd2 = qmul_m(qadd(qsub(qsub(s2, s1), s1), s0), inv2);
            const qm31 dd3 = qmul_m(qsub(qsub(s3, s0), qmul_m(qsub(s2, s1), 3)), inv6);
            const qm31 c0 = s0, c1 = qadd(qsub(dd1, dd2), qmul_m(dd3, 2)), c2 = qsub(dd2, qmul_m(dd3, 3));
            const qm31 c3 = dd3;
            rps[3 * r] = c0;
            rps[3 * r + 1] = c2;
            rps[3 * r + 2] = c3;
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
        int e = wait_signal(ctx, rs.seq, words, 8);
        if (e) return e;
        *fin_w = ldw(words);
        *fin_d = ldw(words + 4);
        return 0;
    };
    std::vector<qm31> lin(3 * num_vars), chal(num_vars);
    qm31 input_final, rsqrt_final;
    if ((rc = eq_sumcheck(lin, chal, &input_final, &rsqrt_final))) return rc;
    ch.mix_qm31(input_final);
    ch.mix_qm31(rsqrt_final);

    // Part 2: LogUp of (rms^2, rsqrt) against the rsqrt table (prover.rs:8632-8720)
    ch.mix_u64(0x4C4F47);
    ch.mix_u64(0x524E);
    const qm31 lgamma = ch.draw_qm31();
    const qm31 lbeta = ch.draw_qm31();
    launch_eq_table(point, num_vars, b.eq.as<uint4>(), n, s);
    next();
    launch_logup_dw(b.m_in.as<uint32_t>(), b.m_out.as<uint32_t>(), n, lgamma, lbeta, b.d.as<uint4>(),
                    b.w.as<uint4>(), rs, s);
    ctx->launches += 2;
    if ((rc = wait_signal(ctx, rs.seq, words, 4))) return rc;
    const qm31 trace_sum = ldw(words);
    next();
    launch_logup_table_sum(b.mult.as<uint32_t>(), ctx->rsqrt_table.as<uint32_t>(), tsize, lgamma, lbeta, rs, s);
    ctx->launches++;
    if ((rc = wait_signal(ctx, rs.seq, words, 4))) return rc;
    if (!qeq(ldw(words), trace_sum))
        return set_error(ZKML_ERR_VERIFY, "RMSNorm LogUp sum mismatch (trace side != table side)");
    ch.mix_qm31(trace_sum);
    std::vector<qm31> lrp(3 * num_vars);
    qm31 w_eval, d_last;
    if ((rc = eq_sumcheck(lrp, chal, &w_eval, &d_last))) return rc;
    launch_eq_table(chal.data(), num_vars, b.eq.as<uint4>(), n, s);
    next();
    launch_eq_dot(b.eq.as<uint4>(), b.m_in.as<uint32_t>(), b.m_out.as<uint32_t>(), n, rs, s);
    ctx->launches += 2;
    if ((rc = wait_signal(ctx, rs.seq, words, 8))) return rc;
    const qm31 rms_s = ldw(words), rsqrt_s = ldw(words + 4);

    // multiplicity sumcheck (prover.rs:9449-9515): in the record only in the V1 layout
    std::vector<qm31> mrp(2 * log_t);
    qm31 m_claim = qzero();
    size_t mlen = tsize;
    next();
    launch_mult_round(b.mult.as<uint32_t>(), b.mv.as<uint4>(), mlen, true, false, qzero(), rs, s);
    ctx->launches++;
    for (unsigned r = 0; r < log_t; r++) {
        if ((rc = wait_signal(ctx, rs.seq, words, 8))) return rc;
        const qm31 lo = ldw(words), hi = ldw(words + 4);
        if (r == 0) m_claim = qadd(lo, hi);
        mrp[2 * r] = lo;
        mrp[2 * r + 1] = qsub(hi, lo);
        ch.mix_qm31(lo);
        ch.mix_qm31(qsub(hi, lo));
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
    const qm31 m_final = ldw(words);
    std::vector<uint32_t> mult(tsize), row_rms(pr);
    ZK_CUDA(cudaMemcpyAsync(mult.data(), b.mult.ptr, tsize * 4, cudaMemcpyDeviceToHost, s));
    ZK_CUDA(cudaMemcpyAsync(row_rms.data(), b.row_rms.ptr, pr * 4, cudaMemcpyDeviceToHost, s));
    ZK_CUDA(cudaStreamSynchronize(s));

    uint64_t tcom[4];
    {
        const uint64_t in[8] = {0x5253, 0, 0, 0, log_t, 0, 0, 0};  // compute_rsqrt_table_commitment
        poseidon_hash_many_canon(in, 2, tcom);
    }
    ch.mix_qm31(input_eval);
    ch.mix_qm31(output_eval);

    // LayerProof::RMSNorm as serialize_gkr_model_proof writes it (cairo_serde.rs:1648-1726)
    o.u64(8);
    o.q(input_eval);
    o.q(output_eval);
    o.q(rms_sq_eval);
    o.q(rsqrt_eval);
    o.push(tcom);
    o.u64(0);  // not SIMD-combined
    if (skip_rms_sq) {
        o.u64(0);
    } else {
        o.u64(1);
        o.u64(n_active);
        o.q(total_sq);
        o.u64(num_vars);
        for (unsigned r = 0; r < num_vars; r++) {
            o.q(rq[3 * r]);
            o.q(rq[3 * r + 1]);
            o.q(rq[3 * r + 2]);
        }
        o.q(rq_final);
    }
    o.u64(num_vars);
    for (unsigned r = 0; r < 3 * num_vars; r++) o.q(lin[r]);
    o.q(input_final);
    o.q(rsqrt_final);
    o.u64(1);  // LogUp proof present
    o.q(trace_sum);
    o.u64(num_vars);
    for (unsigned r = 0; r < 3 * num_vars; r++) o.q(lrp[r]);
    o.q(w_eval);
    o.q(rms_s);
    o.q(rsqrt_s);
    if (v1_record) {
        o.u64(0);  // no multiplicities on chain
        o.u64(1);  // multiplicity sumcheck (serialize_multiplicity_sumcheck, cairo_serde.rs:1138-1156)
        o.u64(log_t);
        for (unsigned r = 0; r < 2 * log_t; r++) o.q(mrp[r]);
        o.q(m_final);
        o.q(m_claim);
    } else {
        o.u64(tsize);
        for (size_t j = 0; j < tsize; j++) o.u64(mult[j]);
    }
    if (pr > 1) {
        o.u64(1);
        o.u64(pr);
        for (size_t i = 0; i < pr; i++) o.u64(row_rms[i]);
    } else {
        o.u64(0);
    }
    if (out_input_eval) {
        out_input_eval[0] = input_eval.a;
        out_input_eval[1] = input_eval.b;
        out_input_eval[2] = input_eval.c;
        out_input_eval[3] = input_eval.d;
    }
    return ZKML_OK;
}

extern "C" int zkml_reduce_rmsnorm(zkml_ctx* ctx, const uint32_t* input, size_t rows, size_t cols, size_t dim,
                                   const uint32_t* gamma, size_t gamma_len, const uint32_t* claim_point,
                                   size_t n_point, const uint32_t claim_value[4], zkml_channel* chs,
                                   uint64_t* out_calldata, size_t cap, size_t* out_len, uint32_t out_input_eval[4]) {
    if (!out_len) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    Out o{out_calldata, out_calldata ? cap : 0};
    int rc = rmsnorm_reduce_dev(ctx, input, rows, cols, dim, gamma, gamma_len, claim_point, n_point, claim_value, chs,
                                o, out_input_eval);
    if (rc) return rc;
    *out_len = o.len;
    if (o.overflow)
        return set_error(ZKML_ERR_INVALID_ARG, "calldata buffer too small: need " + std::to_string(o.len) + " felts");
    return ZKML_OK;
}
