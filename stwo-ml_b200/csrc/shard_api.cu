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
#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include <vector>

#include "channel.hpp"
#include "context.hpp"
#include "mesh.hpp"

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

// Round coefficients from (s0, s1, s2 = s(2)): c0 = s0, c2 = (s2 - 2 s1 + s0) / 2, c1 = s1 - s0 - c2.
void round_coeffs(const uint32_t* s12, qm31& c0, qm31& c1, qm31& c2) {
    static const uint32_t inv2 = minv(2);
    const qm31 s0 = qm(s12[0], s12[1], s12[2], s12[3]), s1 = qm(s12[4], s12[5], s12[6], s12[7]);
    const qm31 s2 = qm(s12[8], s12[9], s12[10], s12[11]);
    c0 = s0;
    c2 = qmul_m(qadd(qsub(qsub(s2, s1), s1), s0), inv2);
    c1 = qsub(qsub(s1, s0), c2);
}

void st4(uint32_t* p, const qm31& x) {
    p[0] = x.a;
    p[1] = x.b;
    p[2] = x.c;
    p[3] = x.d;
}

// out[j * G + g] = in[g * nl + j]: rank-major M31 shards back to global order.
__global__ void interleave_u32_kernel(const uint32_t* __restrict__ in, size_t nl, size_t G, uint32_t* __restrict__ out) {
    const size_t n = nl * G;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = in[(i % G) * nl + i / G];
}

// True when a mesh-reduced round published 0xFFFFFFFF words (a peer timed out).
bool mesh_words_bad(const uint32_t* w) {
    for (int i = 0; i < 12; i++)
        if (w[i] >= P) return true;
    return false;
}

// Copies n words of a host or device buffer to the host.
int to_host(const uint32_t* src, size_t n, std::vector<uint32_t>& dst) {
    dst.resize(n);
    ZK_CUDA(cudaMemcpy(dst.data(), src, n * 4, cudaMemcpyDefault));
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

}  // extern "C"

namespace zk {
namespace {

// The sharded product sumcheck with the per-round exchange and the final gather either through
// a host exchange (ex) or through the peer mesh (mesh), exactly one of them set.
int prove_sharded(zkml_ctx* ctx, const uint32_t* a_local, const uint32_t* b_local, size_t n, size_t gather_local,
                  const zkml_exchange* ex, MeshState* mesh, zkml_channel* chs, uint32_t* out_rp, uint32_t* out_ch,
                  uint32_t out_final_a[4], uint32_t out_final_b[4], size_t* out_gathered_at) {
    const size_t G = ex ? (size_t)ex->world : (size_t)mesh->world;
    const int rank = ex ? ex->rank : mesh->rank;
    if (!is_pow2(n) || n < 2) return set_error(ZKML_ERR_INVALID_ARG, "n must be a power of two >= 2");
    if (G < 1 || !is_pow2(G) || n % G || rank < 0 || (size_t)rank >= G)
        return set_error(ZKML_ERR_INVALID_ARG, "world size must be a power of two dividing n");
    ZK_CUDA(cudaSetDevice(ctx->device));
    const size_t nl = n / G;
    cudaStream_t s = ctx->stream;
    int rc;
    if (G == 1) {  // one rank: the plain product sumcheck on this GPU
        const void *A = nullptr, *B = nullptr;
        if ((rc = device_view(ctx, a_local, n * 4, ctx->sc_a, &A)) || (rc = device_view(ctx, b_local, n * 4, ctx->sc_b, &B)))
            return rc;
        if ((rc = ctx->fa.ensure(n / 2 * 16)) || (rc = ctx->fb.ensure(n / 2 * 16))) return rc;
        ctx->sc_len = 0;
        if (out_gathered_at) *out_gathered_at = n;
        return run_sumcheck(ctx, nullptr, nullptr, static_cast<const uint32_t*>(A), static_cast<const uint32_t*>(B), n,
                            chs, out_rp, out_ch, out_final_a, out_final_b, nullptr);
    }
    if (nl < 4 || nl <= gather_local) {
        // too small to split: every rank proves the whole product
        if ((rc = ctx->sc_a.ensure(n * 4)) || (rc = ctx->sc_b.ensure(n * 4)) || (rc = ctx->fa.ensure(n * 16)) ||
            (rc = ctx->fb.ensure(n * 16)))
            return rc;
        if (mesh) {
            if (nl % 4) return set_error(ZKML_ERR_INVALID_ARG, "mesh gather needs at least 4 elements per rank");
            const void *A = nullptr, *B = nullptr;
            if ((rc = device_view(ctx, a_local, nl * 4, ctx->a_in, &A)) ||
                (rc = device_view(ctx, b_local, nl * 4, ctx->b_in, &B)) || (rc = ctx->mesh_stage.ensure(nl * 8)) ||
                (rc = ctx->gather_dev.ensure(n * 8)))
                return rc;
            ZK_CUDA(cudaMemcpyAsync(ctx->mesh_stage.ptr, A, nl * 4, cudaMemcpyDeviceToDevice, s));
            ZK_CUDA(cudaMemcpyAsync(ctx->mesh_stage.as<uint8_t>() + nl * 4, B, nl * 4, cudaMemcpyDeviceToDevice, s));
            if ((rc = mesh_allgather(ctx, mesh, ctx->mesh_stage.ptr, nl * 8, ctx->gather_dev.ptr))) return rc;
            // rank g's slot holds [a (nl) | b (nl)]: regroup to [a of every rank | b of every rank],
            // then interleave each back to global order
            const unsigned g = (unsigned)std::min<size_t>((n + 255) / 256, 4096);
            {
                // compact the two halves into [a of all ranks | b of all ranks] and interleave each
                DevBuf& tmp = ctx->op.cbuf;
                if ((rc = tmp.ensure(n * 8))) return rc;
                for (size_t r = 0; r < G; r++) {
                    ZK_CUDA(cudaMemcpyAsync(tmp.as<uint32_t>() + r * nl, ctx->gather_dev.as<uint32_t>() + r * 2 * nl,
                                            nl * 4, cudaMemcpyDeviceToDevice, s));
                    ZK_CUDA(cudaMemcpyAsync(tmp.as<uint32_t>() + n + r * nl,
                                            ctx->gather_dev.as<uint32_t>() + r * 2 * nl + nl, nl * 4,
                                            cudaMemcpyDeviceToDevice, s));
                }
                interleave_u32_kernel<<<g, 256, 0, s>>>(tmp.as<uint32_t>(), nl, G, ctx->sc_a.as<uint32_t>());
                interleave_u32_kernel<<<g, 256, 0, s>>>(tmp.as<uint32_t>() + n, nl, G, ctx->sc_b.as<uint32_t>());
                ctx->launches += 2;
                ZK_CUDA(cudaGetLastError());
            }
            ZK_CUDA(cudaStreamSynchronize(s));
            if ((rc = mesh_check(ctx))) return rc;
        } else {
            std::vector<uint32_t> la, lb, ga(n), gb(n), tmp(n);
            if ((rc = to_host(a_local, nl, la)) || (rc = to_host(b_local, nl, lb))) return rc;
            if ((rc = ex->allgather(ex->user, la.data(), tmp.data(), nl * 4))) return rc;
            for (size_t g = 0; g < G; g++)
                for (size_t j = 0; j < nl; j++) ga[j * G + g] = tmp[g * nl + j];
            if ((rc = ex->allgather(ex->user, lb.data(), tmp.data(), nl * 4))) return rc;
            for (size_t g = 0; g < G; g++)
                for (size_t j = 0; j < nl; j++) gb[j * G + g] = tmp[g * nl + j];
            ZK_CUDA(cudaMemcpyAsync(ctx->sc_a.ptr, ga.data(), n * 4, cudaMemcpyHostToDevice, s));
            ZK_CUDA(cudaMemcpyAsync(ctx->sc_b.ptr, gb.data(), n * 4, cudaMemcpyHostToDevice, s));
        }
        ctx->sc_len = 0;
        if (out_gathered_at) *out_gathered_at = n;
        return run_sumcheck(ctx, nullptr, nullptr, ctx->sc_a.as<uint32_t>(), ctx->sc_b.as<uint32_t>(), n, chs, out_rp,
                            out_ch, out_final_a, out_final_b, nullptr);
    }
    // ZKML_SHARD_TRACE=1 prints the phase times of each call to stderr.
    static const bool trace = getenv("ZKML_SHARD_TRACE") && getenv("ZKML_SHARD_TRACE")[0] == '1';
    const auto t_start = std::chrono::steady_clock::now();
    double t_wait = 0, t_ex = 0, t_hash = 0;
    auto now = [] { return std::chrono::steady_clock::now(); };
    auto us = [](std::chrono::steady_clock::time_point a, std::chrono::steady_clock::time_point b) {
        return std::chrono::duration<double, std::micro>(b - a).count();
    };
    // Split phase: round 0 over the local M31 elements, then fused fold + round per challenge.
    const void *A = nullptr, *B = nullptr;
    if ((rc = device_view(ctx, a_local, nl * 4, ctx->sc_a, &A)) || (rc = device_view(ctx, b_local, nl * 4, ctx->sc_b, &B)))
        return rc;
    if ((rc = ctx->fa.ensure(nl / 2 * 16)) || (rc = ctx->fb.ensure(nl / 2 * 16))) return rc;
    ctx->sc_len = 0;
    const uint32_t* A32 = static_cast<const uint32_t*>(A);
    const uint32_t* B32 = static_cast<const uint32_t*>(B);
    Channel ch(chs);
    RoundScratch rs = ctx->round_scratch();
    rs.sig = ctx->d_sig;
    rs.seq = ++ctx->sig_seq;
    if (mesh) rs.mesh = mesh_next(mesh);
    {
        KTimer t(ctx, KC_ROUND);
        launch_round_m31(A32, B32, nl, rs, ctx->err_flag(), s);
    }
    ZK_CUDA(cudaGetLastError());
    ctx->launches++;
    size_t len = nl;
    unsigned r = 0;
    uint32_t words[12];
    for (;; r++) {
        auto t0 = now();
        if ((rc = wait_signal(ctx, rs.seq, words, 12))) return rc;
        auto t1 = now();
        uint32_t s12[12];
        if (mesh) {  // the round kernel already added every rank's words
            if (mesh_words_bad(words)) {
                if ((rc = mesh_check(ctx))) return rc;
                return set_error(ZKML_ERR_TIMEOUT, "mesh: a rank did not arrive within about two seconds");
            }
            memcpy(s12, words, sizeof(s12));
        } else {
            uint64_t w64[12];
            for (int i = 0; i < 12; i++) w64[i] = words[i];
            if ((rc = ex->allreduce_u64(ex->user, w64, 12))) return rc;
            for (int i = 0; i < 12; i++) s12[i] = (uint32_t)(w64[i] % P);
        }
        auto t2 = now();
        t_wait += us(t0, t1);
        t_ex += us(t1, t2);
        qm31 c0, c1, c2, alpha;
        round_coeffs(s12, c0, c1, c2);
        ch.mix_poly_coeffs(c0, c1, c2);
        alpha = ch.draw_qm31();
        t_hash += us(t2, now());
        st4(out_rp + 12 * r, c0);
        st4(out_rp + 12 * r + 4, c1);
        st4(out_rp + 12 * r + 8, c2);
        st4(out_ch + 4 * r, alpha);
        rs.seq = ++ctx->sig_seq;
        const bool last = len / 2 <= gather_local || len / 2 < 4;
        // the last split fold's local sums are not needed (the gathered round recomputes them)
        rs.mesh = (mesh && !last) ? mesh_next(mesh) : MeshArg{nullptr, 0};
        {
            KTimer t(ctx, KC_ROUND);
            if (len == nl)
                launch_fold_round_m31(A32, B32, len, alpha, ctx->fa.as<uint4>(), ctx->fb.as<uint4>(), rs, s);
            else
                launch_fold_round_qm31(ctx->fa.as<uint4>(), ctx->fb.as<uint4>(), len, alpha, rs, s);
        }
        ZK_CUDA(cudaGetLastError());
        ctx->launches++;
        len /= 2;
        if (last) break;
    }
    if ((rc = wait_signal(ctx, rs.seq, words, 12))) return rc;
    if ((rc = read_err_flag(ctx)) || (rc = check_err_flag(ctx, "prove_product_sharded"))) return rc;
    const size_t glen = len * G;
    const size_t local_bytes = len * 32;
    if (mesh) {
        // [fa | fb] of this rank into every rank's inbox, collected rank-major, interleaved on the GPU
        if ((rc = ctx->mesh_stage.ensure(local_bytes)) || (rc = ctx->gather_dev.ensure(G * local_bytes))) return rc;
        ZK_CUDA(cudaMemcpyAsync(ctx->mesh_stage.ptr, ctx->fa.ptr, len * 16, cudaMemcpyDeviceToDevice, s));
        ZK_CUDA(cudaMemcpyAsync(ctx->mesh_stage.as<uint8_t>() + len * 16, ctx->fb.ptr, len * 16,
                                cudaMemcpyDeviceToDevice, s));
        if ((rc = mesh_allgather(ctx, mesh, ctx->mesh_stage.ptr, local_bytes, ctx->gather_dev.ptr))) return rc;
        if ((rc = ctx->fa.ensure(glen * 16)) || (rc = ctx->fb.ensure(glen * 16))) return rc;
    } else {
        const size_t need = local_bytes * (1 + G);
        if (ctx->h_stage_bytes < need) {
            if (ctx->h_stage) cudaFreeHost(ctx->h_stage);
            ctx->h_stage = nullptr;
            ctx->h_stage_bytes = 0;
            ZK_CUDA(cudaMallocHost(&ctx->h_stage, need));
            ctx->h_stage_bytes = need;
        }
        uint8_t* hl = ctx->h_stage;                  // this rank: A part then B part
        uint8_t* hall = ctx->h_stage + local_bytes;  // every rank, rank-major
        ZK_CUDA(cudaMemcpyAsync(hl, ctx->fa.ptr, len * 16, cudaMemcpyDeviceToHost, s));
        ZK_CUDA(cudaMemcpyAsync(hl + len * 16, ctx->fb.ptr, len * 16, cudaMemcpyDeviceToHost, s));
        ZK_CUDA(cudaStreamSynchronize(s));
        if ((rc = ex->allgather(ex->user, hl, hall, local_bytes))) return rc;
        if ((rc = ctx->gather_dev.ensure(G * local_bytes)) || (rc = ctx->fa.ensure(glen * 16)) ||
            (rc = ctx->fb.ensure(glen * 16)))
            return rc;
        ZK_CUDA(cudaMemcpyAsync(ctx->gather_dev.ptr, hall, G * local_bytes, cudaMemcpyHostToDevice, s));
    }
    launch_interleave_gather(ctx->gather_dev.as<uint4>(), len, G, ctx->fa.as<uint4>(), ctx->fb.as<uint4>(), s);
    ZK_CUDA(cudaGetLastError());
    ctx->launches++;
    if (out_gathered_at) *out_gathered_at = glen;
    const unsigned done = r + 1;
    const auto t_gather = now();
    rc = run_sumcheck(ctx, ctx->fa.as<uint4>(), ctx->fb.as<uint4>(), nullptr, nullptr, glen, chs, out_rp + 12 * done,
                      out_ch + 4 * done, out_final_a, out_final_b, nullptr);
    if (!rc && mesh) rc = mesh_check(ctx);  // a gather that timed out leaves zeros: fail the call
    if (trace)
        fprintf(stderr,
                "[zkml shard rank %d] split rounds %u: gpu wait %.1f us, exchange %.1f us, transcript %.1f us; "
                "until gather end %.1f us; gathered tail (%zu) %.1f us\n",
                rank, done, t_wait, t_ex, t_hash, us(t_start, t_gather), glen, us(t_gather, now()));
    return rc;
}

}  // namespace
}  // namespace zk

extern "C" {

int zkml_prove_product_sharded(zkml_ctx* ctx, const uint32_t* a_local, const uint32_t* b_local, size_t n,
                               size_t gather_local, const zkml_exchange* ex, zkml_channel* chs,
                               uint32_t* out_rp, uint32_t* out_ch, uint32_t out_final_a[4], uint32_t out_final_b[4],
                               size_t* out_gathered_at) {
    if (!ctx || !a_local || !b_local || !ex || !ex->allreduce_u64 || !ex->allgather || !chs || !out_rp || !out_ch ||
        !out_final_a || !out_final_b)
        return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    return prove_sharded(ctx, a_local, b_local, n, gather_local, ex, nullptr, chs, out_rp, out_ch, out_final_a,
                         out_final_b, out_gathered_at);
}

int zkml_prove_product_sharded_mesh(zkml_ctx* ctx, const uint32_t* a_local, const uint32_t* b_local, size_t n,
                                    size_t gather_local, zkml_channel* chs, uint32_t* out_rp, uint32_t* out_ch,
                                    uint32_t out_final_a[4], uint32_t out_final_b[4], size_t* out_gathered_at) {
    if (!ctx || !a_local || !b_local || !chs || !out_rp || !out_ch || !out_final_a || !out_final_b)
        return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    MeshState* m = mesh_of(ctx);
    if (!m) return set_error(ZKML_ERR_INVALID_ARG, "no peer mesh is open on this context's device");
    return prove_sharded(ctx, a_local, b_local, n, gather_local, nullptr, m, chs, out_rp, out_ch, out_final_a,
                         out_final_b, out_gathered_at);
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
