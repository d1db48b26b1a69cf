// C-ABI: a stepwise product sumcheck, for splitting one sumcheck across GPUs.
//
// The sumcheck of reduce_matmul_layer (engine/src/backend.rs:141-178) is
// driven one round at a time: each call folds the two vectors with the
// previous challenge (in place) and returns this round's (s0, s1, s2) over the
// vectors the context holds.  When rank g of G holds the elements whose index
// is g modulo G, every fold partner (i, i + N/2) is on the same rank as long as
// the local length is at least 2, so the local sums of all ranks add up to the
// global round sums: the only exchange per round is those 12 words.  Below a
// size threshold the caller gathers the local vectors (zkml_sumcheck_export)
// and continues on one GPU (zkml_sumcheck_load_qm31).
#include <cstring>
#include <string>

#include "context.hpp"

namespace zk {
namespace {

inline bool is_pow2(size_t x) { return x && !(x & (x - 1)); }

int round_words(zkml_ctx* ctx, const qm31* alpha, uint32_t out[12]) {
    cudaStream_t s = ctx->stream;
    RoundScratch rs = ctx->round_scratch();
    rs.sig = ctx->d_sig;
    rs.seq = ++ctx->sig_seq;
    const size_t len = ctx->sc_len;
    const bool checks_input = ctx->sc_m31 && !alpha;  // only the base-field round validates words
    {
        KTimer t(ctx, KC_ROUND);
        if (!alpha) {
            if (ctx->sc_m31)
                launch_round_m31(ctx->sc_a32, ctx->sc_b32, len, rs, ctx->err_flag(), s);
            else
                launch_round_qm31(ctx->fa.as<uint4>(), ctx->fb.as<uint4>(), len, rs, s);
        } else if (ctx->sc_m31) {
            launch_fold_round_m31(ctx->sc_a32, ctx->sc_b32, len, *alpha, ctx->fa.as<uint4>(), ctx->fb.as<uint4>(),
                                  rs, s);
        } else {
            launch_fold_round_qm31(ctx->fa.as<uint4>(), ctx->fb.as<uint4>(), len, *alpha, rs, s);
        }
    }
    ZK_CUDA(cudaGetLastError());
    ctx->launches++;
    int rc = wait_signal(ctx, rs.seq, out, 12);
    if (rc) return rc;
    if (alpha) {
        ctx->sc_len = len / 2;
        ctx->sc_m31 = false;
    }
    if (!checks_input) return ZKML_OK;
    if ((rc = read_err_flag(ctx))) return rc;
    return check_err_flag(ctx, "sumcheck round");
}

int load(zkml_ctx* ctx, const uint32_t* a, const uint32_t* b, size_t n, bool m31) {
    if (!ctx || !a || !b) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    if (!is_pow2(n) || n < 2) return set_error(ZKML_ERR_INVALID_ARG, "length must be a power of two >= 2");
    ZK_CUDA(cudaSetDevice(ctx->device));
    ctx->sc_len = 0;
    int rc;
    const size_t esz = m31 ? 4 : 16;
    if ((rc = ctx->fa.ensure((m31 ? n / 2 : n) * 16)) || (rc = ctx->fb.ensure((m31 ? n / 2 : n) * 16))) return rc;
    if (m31) {
        const void *A = nullptr, *B = nullptr;
        if ((rc = device_view(ctx, a, n * esz, ctx->sc_a, &A)) || (rc = device_view(ctx, b, n * esz, ctx->sc_b, &B)))
            return rc;
        ctx->sc_a32 = static_cast<const uint32_t*>(A);
        ctx->sc_b32 = static_cast<const uint32_t*>(B);
    } else {
        ZK_CUDA(cudaMemcpyAsync(ctx->fa.ptr, a, n * 16, cudaMemcpyDefault, ctx->stream));
        ZK_CUDA(cudaMemcpyAsync(ctx->fb.ptr, b, n * 16, cudaMemcpyDefault, ctx->stream));
        launch_canon_words(ctx->fa.as<uint32_t>(), 4 * n, ctx->stream);
        launch_canon_words(ctx->fb.as<uint32_t>(), 4 * n, ctx->stream);
        ZK_CUDA(cudaGetLastError());
        ctx->launches += 2;
        ctx->sc_a32 = ctx->sc_b32 = nullptr;
    }
    ctx->sc_m31 = m31;
    ctx->sc_len = n;
    return ZKML_OK;
}

}  // namespace
}  // namespace zk

using namespace zk;

extern "C" {

int zkml_sumcheck_load_m31(zkml_ctx* ctx, const uint32_t* a, const uint32_t* b, size_t n) {
    return load(ctx, a, b, n, true);
}

int zkml_sumcheck_load_qm31(zkml_ctx* ctx, const uint32_t* a, const uint32_t* b, size_t n) {
    return load(ctx, a, b, n, false);
}

size_t zkml_sumcheck_length(const zkml_ctx* ctx) { return ctx ? ctx->sc_len : 0; }

int zkml_sumcheck_round(zkml_ctx* ctx, const uint32_t* alpha, uint32_t out_sums[12]) {
    if (!ctx || !out_sums) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    if (ctx->sc_len < 2 || (alpha && ctx->sc_len < 4))
        return set_error(ZKML_ERR_INVALID_ARG, "no sumcheck loaded, or too short for another round");
    ZK_CUDA(cudaSetDevice(ctx->device));
    const qm31 al = alpha ? qm(alpha[0], alpha[1], alpha[2], alpha[3]) : qzero();
    return round_words(ctx, alpha ? &al : nullptr, out_sums);
}

int zkml_sumcheck_export(zkml_ctx* ctx, uint32_t* out_a, uint32_t* out_b) {
    if (!ctx || !out_a || !out_b) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    if (ctx->sc_len == 0) return set_error(ZKML_ERR_INVALID_ARG, "no sumcheck loaded");
    if (ctx->sc_m31) return set_error(ZKML_ERR_INVALID_ARG, "export needs at least one folded round");
    ZK_CUDA(cudaSetDevice(ctx->device));
    ZK_CUDA(cudaMemcpyAsync(out_a, ctx->fa.ptr, ctx->sc_len * 16, cudaMemcpyDefault, ctx->stream));
    ZK_CUDA(cudaMemcpyAsync(out_b, ctx->fb.ptr, ctx->sc_len * 16, cudaMemcpyDefault, ctx->stream));
    ZK_CUDA(cudaStreamSynchronize(ctx->stream));
    return ZKML_OK;
}

int zkml_sumcheck_finalize(zkml_ctx* ctx, const uint32_t alpha[4], uint32_t out_a[4], uint32_t out_b[4]) {
    if (!ctx || !alpha || !out_a || !out_b) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    if (ctx->sc_len != 2) return set_error(ZKML_ERR_INVALID_ARG, "finalize needs vectors of length 2");
    ZK_CUDA(cudaSetDevice(ctx->device));
    const uint32_t seq = ++ctx->sig_seq;
    launch_final_fold(ctx->fa.as<uint4>(), ctx->fb.as<uint4>(), ctx->sc_m31 ? ctx->sc_a32 : nullptr,
                      ctx->sc_m31 ? ctx->sc_b32 : nullptr, 2, qm(alpha[0], alpha[1], alpha[2], alpha[3]),
                      ctx->out_words(), ctx->d_sig, seq, ctx->stream);
    ZK_CUDA(cudaGetLastError());
    ctx->launches++;
    uint32_t w[8];
    int rc = wait_signal(ctx, seq, w, 8);
    if (rc) return rc;
    memcpy(out_a, w, 16);
    memcpy(out_b, w + 4, 16);
    ctx->sc_len = 1;
    return ZKML_OK;
}

// Queues one look-ahead round kernel that waits for a challenge nobody posts and
// reports how its bounded wait ended: *status_out = 1 when the kernel gave up
// and flagged the timeout (the expected outcome).  Takes a few seconds.
int zkml_selftest_wait_timeout(zkml_ctx* ctx, uint32_t* status_out) {
    if (!ctx || !status_out) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    ZK_CUDA(cudaSetDevice(ctx->device));
    int rc;
    if ((rc = ctx->fa.ensure(64 * 16)) || (rc = ctx->fb.ensure(64 * 16))) return rc;
    ZK_CUDA(cudaMemsetAsync(ctx->fa.ptr, 0, 64 * 16, ctx->stream));
    ZK_CUDA(cudaMemsetAsync(ctx->fb.ptr, 0, 64 * 16, ctx->stream));
    ZK_CUDA(cudaMemsetAsync(ctx->la_status(), 0, 4, ctx->stream));
    RoundScratch rs = ctx->round_scratch();
    rs.sig = ctx->d_sig;
    rs.seq = ++ctx->sig_seq;
    const uint32_t tag = ++ctx->la_msg_seq;  // never posted
    launch_round_lookahead(ctx->fa.as<uint4>(), ctx->fb.as<uint4>(), 32, true, qzero(), rs, ctx->stream,
                           ctx->d_la_msg() + 8 * (tag % zkml_ctx::LA_SLOTS), tag, ctx->la_status(),
                           ctx->la_mailbox());
    ZK_CUDA(cudaGetLastError());
    ctx->launches++;
    uint32_t st = 0;
    ZK_CUDA(cudaMemcpyAsync(&st, ctx->la_status(), 4, cudaMemcpyDeviceToHost, ctx->stream));
    ZK_CUDA(cudaStreamSynchronize(ctx->stream));
    ZK_CUDA(cudaMemsetAsync(ctx->la_status(), 0, 4, ctx->stream));
    *status_out = st;
    return ZKML_OK;
}

}  // extern "C"
