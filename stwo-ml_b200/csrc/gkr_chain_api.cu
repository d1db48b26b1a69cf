// C-ABI: the GKR proof of a sequential chain of Linear, ReLU and RMSNorm layers
// (prove_gkr_with_cache, gkr/prover.rs:1500-2251, for GraphBuilder::new((m, k0)) followed
// by .linear(n) / .activation(ReLU) layers) in Sequential weight-binding mode, serialized
// by serialize_gkr_model_proof (cairo_serde.rs:1307-1772).
//
// Forward pass on the GPU (tensor-pipe M31 GEMM, ReLU), then the transcript: depth, input
// shape, optional policy commitment, the output claim at a drawn point, the walk from the
// output layer to the input (matmul layers through zkml_reduce_matmul_layer_gkr, ReLU
// layers through the algebraic reduction, RMSNorm layers through the RMSNorm reduction),
// the input claim, one MLE opening per weight on
// the main channel in walk order, and the io commitment.
#include <algorithm>
#include <array>
#include <cstring>
#include <string>
#include <vector>

#include "calldata.hpp"
#include "channel.hpp"
#include "context.hpp"
#include "gkr.cuh"
#include "logup.cuh"
#include "opening.hpp"
#include "relu.hpp"

namespace zk {

const std::vector<uint32_t>& rsqrt_table16();

namespace {

__global__ void relu_forward_kernel(const uint32_t* __restrict__ x, size_t n, uint32_t* __restrict__ y) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const uint32_t v = red32(x[i]);
        y[i] = v <= (P - 1) / 2 ? v : 0u;
    }
}

// Zero-padded row-major copy (rows x cols -> pr x pc) of an M31 matrix.
__global__ void pad_rows_cols_kernel(const uint32_t* __restrict__ x, size_t rows, size_t cols, size_t pc, size_t n,
                                     uint32_t* __restrict__ y) {
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < n; idx += (size_t)gridDim.x * blockDim.x) {
        const size_t i = idx / pc, j = idx % pc;
        y[idx] = (i < rows && j < cols) ? red32(x[i * cols + j]) : 0u;
    }
}

// apply_rmsnorm_detailed (compiler/prove.rs:1115-1180) with dim = cols: one block per
// row, rms^2 = sum x^2 / cols masked to 16 bits, out = x * rsqrt(rms^2).
__global__ void __launch_bounds__(256) rmsnorm_forward_kernel(const uint32_t* __restrict__ x, uint32_t rows,
                                                              uint32_t cols, uint32_t inv_n,
                                                              const uint32_t* __restrict__ table,
                                                              uint32_t* __restrict__ y) {
    __shared__ unsigned long long part[8];
    __shared__ uint32_t s_rs;
    for (uint32_t i = blockIdx.x; i < rows; i += gridDim.x) {
        const uint32_t* row = x + (size_t)i * cols;
        unsigned long long sq = 0;
        for (uint32_t j = threadIdx.x; j < cols; j += blockDim.x) {
            const uint32_t v = red32(row[j]);
            sq += red64((uint64_t)v * v);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
        if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sq;
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned long long t = 0;
            for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += part[w];
            s_rs = table[mmul(red64(t), inv_n) & 0xFFFFu];
        }
        __syncthreads();
        const uint32_t rs = s_rs;
        for (uint32_t j = threadIdx.x; j < cols; j += blockDim.x) y[(size_t)i * cols + j] = mmul(red32(row[j]), rs);
        __syncthreads();
    }
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
inline unsigned blocks_for(size_t n) { return (unsigned)std::min<size_t>((n + 255) / 256, 8192); }

}  // namespace
}  // namespace zk

using namespace zk;

extern "C" int zkml_prove_gkr_chain(zkml_ctx* ctx, const uint32_t* input, size_t m, size_t k0,
                                    const zkml_chain_layer* layers, size_t n_layers, const uint64_t* policy,
                                    size_t n_queries, int flags, uint64_t* out_calldata, size_t cap, size_t* out_len,
                                    uint64_t out_digest[4], uint64_t out_io[4]) {
    if (!ctx || !input || !layers || !out_len || !out_digest || !out_io)
        return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    if (m == 0 || k0 == 0 || n_layers == 0 || n_layers > 1024) return set_error(ZKML_ERR_INVALID_ARG, "empty chain");
    if (m > (1u << 30) || k0 > (1u << 30)) return set_error(ZKML_ERR_INVALID_ARG, "input too large");
    ZK_CUDA(cudaSetDevice(ctx->device));
    cudaStream_t s = ctx->stream;
    int rc;
    // forward pass: acts[l] is layer l's input (m x width[l]) in device memory
    std::vector<size_t> width(n_layers + 1);
    width[0] = k0;
    for (size_t l = 0; l < n_layers; l++) {
        if (layers[l].type == ZKML_LAYER_LINEAR) {
            if (!layers[l].weight || layers[l].n == 0 || layers[l].n > (1u << 30))
                return set_error(ZKML_ERR_INVALID_ARG, "layer " + std::to_string(l) + ": bad Linear layer");
            width[l + 1] = layers[l].n;
        } else if (layers[l].type == ZKML_LAYER_RELU || layers[l].type == ZKML_LAYER_RMSNORM) {
            width[l + 1] = width[l];
        } else {
            return set_error(ZKML_ERR_INVALID_ARG, "layer " + std::to_string(l) + ": unsupported layer type");
        }
    }
    std::vector<DevBuf> acts(n_layers + 1);
    struct Release {
        std::vector<DevBuf>& v;
        ~Release() {
            for (DevBuf& b : v) b.release();
        }
    } release{acts};
    for (size_t l = 0; l <= n_layers; l++)
        if ((rc = acts[l].ensure(m * width[l] * 4))) return rc;
    {
        const void* Iv = nullptr;
        if ((rc = device_view(ctx, input, m * k0 * 4, ctx->a_in, &Iv))) return rc;
        pad_rows_cols_kernel<<<blocks_for(m * k0), 256, 0, s>>>(static_cast<const uint32_t*>(Iv), m, k0, k0, m * k0,
                                                                acts[0].as<uint32_t>());
        ctx->launches++;
    }
    for (size_t l = 0; l < n_layers; l++) {
        if (layers[l].type == ZKML_LAYER_LINEAR) {
            if ((rc = zkml_matmul_m31(ctx, acts[l].as<uint32_t>(), m, width[l], layers[l].weight, width[l + 1],
                                      acts[l + 1].as<uint32_t>())))
                return rc;
        } else if (layers[l].type == ZKML_LAYER_RMSNORM) {
            if (!ctx->rsqrt_table.ptr) {
                if ((rc = ctx->rsqrt_table.ensure(4u << 16))) return rc;
                ZK_CUDA(cudaMemcpy(ctx->rsqrt_table.ptr, rsqrt_table16().data(), 4u << 16, cudaMemcpyHostToDevice));
            }
            rmsnorm_forward_kernel<<<(unsigned)std::min<size_t>(m, 8192), 256, 0, s>>>(
                acts[l].as<uint32_t>(), (uint32_t)m, (uint32_t)width[l], minv((uint32_t)(width[l] % P)),
                ctx->rsqrt_table.as<uint32_t>(), acts[l + 1].as<uint32_t>());
            ctx->launches++;
        } else {
            relu_forward_kernel<<<blocks_for(m * width[l]), 256, 0, s>>>(acts[l].as<uint32_t>(), m * width[l],
                                                                         acts[l + 1].as<uint32_t>());
            ctx->launches++;
        }
    }
    ZK_CUDA(cudaGetLastError());

    zkml_channel chs;
    zkml_channel_init(&chs);
    Channel ch(&chs);
    ch.mix_u64(n_layers);
    ch.mix_u64(m);
    ch.mix_u64(k0);
    if (policy && (policy[0] | policy[1] | policy[2] | policy[3])) ch.mix_m(f_from_canon(policy));
    // output claim (prover.rs:1543-1561)
    const size_t wout = width[n_layers];
    const size_t pm = np2(m), pout = np2(wout), nout = pm * pout;
    const unsigned log_m = lg2(pm), nvo = log_m + lg2(pout);
    std::vector<qm31> point(64);
    for (unsigned i = 0; i < nvo; i++) point[i] = ch.draw_qm31();
    qm31 value;
    {
        LogupScratch& b = ctx->lu;
        if ((rc = b.x.ensure(nout * 4)) || (rc = b.eq.ensure(nout * 16))) return rc;
        pad_rows_cols_kernel<<<blocks_for(nout), 256, 0, s>>>(acts[n_layers].as<uint32_t>(), m, wout, pout, nout,
                                                              b.x.as<uint32_t>());
        launch_eq_table(point.data(), nvo, b.eq.as<uint4>(), nout, s);
        RoundScratch rs = ctx->round_scratch();
        rs.sig = ctx->d_sig;
        rs.seq = ++ctx->sig_seq;
        launch_eq_dot(b.eq.as<uint4>(), b.x.as<uint32_t>(), nullptr, nout, rs, s);
        ctx->launches += 3;
        uint32_t w[4];
        if ((rc = wait_signal(ctx, rs.seq, w, 4))) return rc;
        value = qm(w[0], w[1], w[2], w[3]);
    }
    ch.mix_qm31(value);
    unsigned npt = nvo;

    Out o{out_calldata, out_calldata ? cap : 0};
    o.u64(n_layers);
    struct WeightClaim {
        size_t layer;
        std::vector<qm31> point;
        qm31 value;
    };
    std::vector<WeightClaim> wclaims;
    for (size_t li = n_layers; li-- > 0;) {
        const size_t w = width[li];
        if (layers[li].type == ZKML_LAYER_LINEAR) {
            const size_t n = width[li + 1];
            const unsigned log_k = lg2(np2(w)), log_n = lg2(np2(n));
            std::vector<uint32_t> rp(12 * (log_k + 1)), nxt(4 * (log_m + log_k + 1));
            uint32_t fa[4], fb[4], cv[4] = {value.a, value.b, value.c, value.d};
            if ((rc = zkml_reduce_matmul_layer_gkr(ctx, reinterpret_cast<const uint32_t*>(point.data()), npt, cv,
                                                   acts[li].as<uint32_t>(), m, w, layers[li].weight, n, &chs,
                                                   rp.data(), fa, fb, nxt.data())))
                return rc;
            o.u64(0);  // tag MatMul
            o.u64(log_k);
            for (unsigned r = 0; r < log_k; r++) {
                o.qm(&rp[12 * r]);
                o.qm(&rp[12 * r + 8]);
            }
            o.qm(fa);
            o.qm(fb);
            // weight claim: r_j || sumcheck challenges (prover.rs:1465-1483)
            WeightClaim wc{li, std::vector<qm31>(log_n + log_k), qm(fb[0], fb[1], fb[2], fb[3])};
            for (unsigned i = 0; i < log_n; i++) wc.point[i] = point[log_m + i];
            memcpy(wc.point.data() + log_n, nxt.data() + 4 * log_m, 16 * log_k);
            wclaims.push_back(std::move(wc));
            memcpy(point.data(), nxt.data(), 16 * (log_m + log_k));
            npt = log_m + log_k;
            value = qm(fa[0], fa[1], fa[2], fa[3]);
        } else if (layers[li].type == ZKML_LAYER_RMSNORM) {
            uint32_t cv[4] = {value.a, value.b, value.c, value.d}, ie[4];
            if ((rc = rmsnorm_reduce_dev(ctx, acts[li].as<uint32_t>(), m, w, w, nullptr, 0,
                                         reinterpret_cast<const uint32_t*>(point.data()), npt, cv, &chs, o, ie)))
                return rc;
            value = qm(ie[0], ie[1], ie[2], ie[3]);  // the point is unchanged
        } else {
            std::vector<qm31> nxt(64);
            qm31 nval;
            if ((rc = relu_reduce_dev(ctx, acts[li].as<uint32_t>(), m, w, point.data(), value, &chs, o, nxt.data(),
                                      &nval, (flags & ZKML_CHAIN_LEGACY_ACTIVATION_RECORD) != 0)))
                return rc;
            npt = lg2(pm * np2(w));
            memcpy(point.data(), nxt.data(), 16 * npt);
            value = nval;
        }
    }
    o.u64(npt);  // input claim
    for (unsigned i = 0; i < npt; i++) o.q(point[i]);
    o.q(value);
    // Sequential weight openings on the main channel, in walk order (prover.rs:2140-2171)
    std::vector<std::array<uint64_t, 4>> coms(wclaims.size());
    std::vector<std::vector<uint64_t>> obufs(wclaims.size());
    std::vector<size_t> olens(wclaims.size());
    for (size_t i = 0; i < wclaims.size(); i++) {
        const WeightClaim& wc = wclaims[i];
        const size_t l = wc.layer, k = width[l], n = width[l + 1];
        const size_t pk = np2(k), pn = np2(n);
        const void* Bv = nullptr;
        if ((rc = device_view(ctx, layers[l].weight, k * n * 4, ctx->b_in, &Bv))) return rc;
        DevBuf& bmle = ctx->op.bmle;
        if ((rc = bmle.ensure(pk * pn * 16))) return rc;
        launch_colmajor_mle(static_cast<const uint32_t*>(Bv), (uint32_t)k, (uint32_t)n, pk, pn, bmle.as<uint4>(), s);
        ctx->launches++;
        const unsigned nv = (unsigned)wc.point.size();
        const size_t qcap = 64 + (n_queries + 1) * (2 + (size_t)nv * (10 + 2 * (nv + 1)));
        obufs[i].resize(qcap * 4);
        Out oo{obufs[i].data(), qcap};
        {
            KTimer t(ctx, KC_MERKLE);
            if ((rc = prove_opening_dev(ctx, bmle.as<uint4>(), nv, wc.point.data(), &chs, n_queries, coms[i].data(), oo,
                                        nullptr)))
                return rc;
        }
        olens[i] = oo.len;
    }
    o.u64(wclaims.size());
    for (auto& c : coms) o.push(c.data());
    o.u64(wclaims.size());
    for (size_t i = 0; i < wclaims.size(); i++) {
        o.u64(wclaims[i].point.size());
        for (const qm31& p : wclaims[i].point) o.q(p);
        o.q(wclaims[i].value);
        for (size_t j = 0; j < olens[i]; j++) o.push(&obufs[i][4 * j]);
    }
    // io commitment (aggregation.rs:235-254) of the model input and output
    std::vector<uint32_t> hin(m * k0), hout(m * wout);
    ZK_CUDA(cudaMemcpyAsync(hin.data(), acts[0].ptr, m * k0 * 4, cudaMemcpyDeviceToHost, s));
    ZK_CUDA(cudaMemcpyAsync(hout.data(), acts[n_layers].ptr, m * wout * 4, cudaMemcpyDeviceToHost, s));
    ZK_CUDA(cudaStreamSynchronize(s));
    if ((rc = zkml_io_commitment(hin.data(), m, k0, hout.data(), m, wout, out_io))) return rc;
    o.push(out_io);
    memcpy(out_digest, chs.digest, 32);
    *out_len = o.len;
    if (o.overflow)
        return set_error(ZKML_ERR_INVALID_ARG, "calldata buffer too small: need " + std::to_string(o.len) + " felts");
    return ZKML_OK;
}
