// C-ABI: the GKR proof of a layered circuit of Linear, ReLU, RMSNorm, Add and Mul layers
// (prove_gkr_with_cache, gkr/prover.rs:1500-2251, for GraphBuilder::new((m, k0)) followed
// by .linear(n) / .activation(ReLU) / .rms_norm() / .add_from(fork) / .mul_from(fork)) in
// Sequential weight-binding mode, serialized by serialize_gkr_model_proof
// (cairo_serde.rs:1307-1772) or as the verify_model_gkr calldata (starknet.rs:3143-3345).
//
// Forward pass on the GPU (tensor-pipe M31 GEMM, ReLU), then the transcript: depth, input
// shape, optional policy commitment, the output claim at a drawn point, the walk from the
// output layer to the input (matmul layers through zkml_reduce_matmul_layer_gkr, ReLU
// layers through the algebraic reduction, RMSNorm layers through the RMSNorm reduction, Add
// layers by two MLE evaluations, Mul layers by a degree-3 eq-sumcheck on the LogUp round
// kernels; Add / Mul defer their skip branch), the deferred MatMul proofs, the input claim,
// one MLE opening per weight on the main channel (deferred first, then walk order), and the
// io commitment.
#include <algorithm>
#include <array>
#include <cstring>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <thread>
#include <vector>

#include "calldata.hpp"
#include "channel.hpp"
#include "context.hpp"
#include "gkr.cuh"
#include "logup.cuh"
#include "mesh.hpp"
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

// ActivationType::as_fn (gadgets/lookup_table.rs:193-345) applied to full M31 values, as the
// reference's forward pass does (compiler/prove.rs:1893-1899): fixed point with scale 2^16,
// values above (P - 1) / 2 read as negative; GELU (tanh form) and SiLU in binary64, rounded
// half away from zero and clamped to [0, P - 1] / [-(P - 1), 0]; Sigmoid a step; Softmax-exp a
// shift.  The binary64 evaluation uses the device exp / tanh; they round to nearest within an
// ulp of the host libm's, which decides a result only when x * 2^16 lands within ~1e-9 of a
// half-integer.
__device__ __forceinline__ double act_real(uint32_t v) {
    return v <= 0x3FFFFFFFu ? (double)v / 65536.0 : -((double)((uint64_t)P - v)) / 65536.0;
}
__device__ __forceinline__ uint32_t act_from_real(double r) {
    const uint64_t pm1 = (uint64_t)P - 1;
    if (r >= 0.0) {
        const uint64_t u = (uint64_t)round(r * 65536.0);
        return (uint32_t)(u < pm1 ? u : pm1);
    }
    uint64_t neg = (uint64_t)round(-r * 65536.0);
    if (neg > pm1) neg = pm1;
    return (uint32_t)((uint64_t)P - neg);
}
__device__ uint32_t act_value(int tag, uint32_t v) {
    switch (tag) {
        case 2: {  // GELU
            if (v == 0) return 0;
            const double x = act_real(v);
            const double c = sqrt(2.0 / 3.14159265358979311599796346854);
            const double inner = __dmul_rn(c, __dadd_rn(x, __dmul_rn(__dmul_rn(__dmul_rn(0.044715, x), x), x)));
            return act_from_real(__dmul_rn(__dmul_rn(0.5, x), __dadd_rn(1.0, tanh(inner))));
        }
        case 3:  // Sigmoid step
            if (v > 0x3FFFFFFFu) return 0;
            return v == 0 ? 32768u : 65536u;
        case 4: {  // Softmax exp
            if (v > 0x3FFFFFFFu) {
                uint32_t decay = (((1u << 31) - 2) - v) / 65536u;
                if (decay > 20) decay = 20;
                const uint32_t r = 65536u >> decay;
                return r > 1 ? r : 1;
            }
            if (v == 0) return 65536u;
            uint32_t growth = v / 65536u;
            if (growth > 10) growth = 10;
            const uint64_t r = (uint64_t)65536u << growth, cap = (1ull << 31) - 2;
            return (uint32_t)(r < cap ? r : cap);
        }
        default: {  // SiLU
            if (v == 0) return 0;
            const double x = act_real(v);
            return act_from_real(__ddiv_rn(x, __dadd_rn(1.0, exp(-x))));
        }
    }
}
__global__ void act_forward_kernel(const uint32_t* __restrict__ x, size_t n, int tag, uint32_t* __restrict__ y) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = act_value(tag, red32(x[i]));
}

// Zero-padded row-major copy (rows x cols -> pr x pc) of an M31 matrix.
__global__ void pad_rows_cols_kernel(const uint32_t* __restrict__ x, size_t rows, size_t cols, size_t pc, size_t n,
                                     uint32_t* __restrict__ y) {
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < n; idx += (size_t)gridDim.x * blockDim.x) {
        const size_t i = idx / pc, j = idx % pc;
        y[idx] = (i < rows && j < cols) ? red32(x[i * cols + j]) : 0u;
    }
}

// elementwise_add / elementwise_mul (compiler/prove.rs:875-925): y = lhs + rhs or lhs * rhs.
__global__ void elementwise_kernel(const uint32_t* __restrict__ a, const uint32_t* __restrict__ b, size_t n, bool mul,
                                   uint32_t* __restrict__ y) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = mul ? mmul(red32(a[i]), red32(b[i])) : madd(red32(a[i]), red32(b[i]));
}

// Zero-padded row-major MLE (rows x cols -> pr x pc) of an M31 matrix as QM31 values.
__global__ void lift_pad_kernel(const uint32_t* __restrict__ x, size_t rows, size_t cols, size_t pc, size_t n,
                                uint4* __restrict__ y) {
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < n; idx += (size_t)gridDim.x * blockDim.x) {
        const size_t i = idx / pc, j = idx % pc;
        y[idx] = make_uint4((i < rows && j < cols) ? red32(x[i * cols + j]) : 0u, 0u, 0u, 0u);
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

// The proof of the circuit; with model_id (V1 layout only) the whole verify_model_gkr
// calldata: model_id, raw io, circuit depth, proof layer count, matmul dims, dequantize bits.
static int prove_chain(zkml_ctx* ctx, const uint64_t* model_id, const uint32_t* input, size_t m, size_t k0,
                       const zkml_chain_layer* layers, size_t n_layers, const uint64_t* policy, size_t n_queries,
                       int flags, uint64_t* out_calldata, size_t cap, size_t* out_len, uint64_t out_digest[4],
                       uint64_t out_io[4]) {
    if (!ctx || !input || !layers || !out_len || !out_digest || !out_io)
        return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    if (m == 0 || k0 == 0 || n_layers == 0 || n_layers > 1024) return set_error(ZKML_ERR_INVALID_ARG, "empty chain");
    if (m > (1u << 30) || k0 > (1u << 30)) return set_error(ZKML_ERR_INVALID_ARG, "input too large");
    ZK_CUDA(cudaSetDevice(ctx->device));
    cudaStream_t s = ctx->stream;
    int rc;
    // ZKML_CHAIN_TRACE=1 prints the host wall time of each phase and layer kind to stderr.
    static const bool trace = getenv("ZKML_CHAIN_TRACE") && getenv("ZKML_CHAIN_TRACE")[0] == '1';
    auto now = [] { return std::chrono::steady_clock::now(); };
    auto ms_since = [](std::chrono::steady_clock::time_point t) {
        return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t).count();
    };
    const auto t_call = now();
    double t_kind[8] = {0, 0, 0, 0, 0, 0, 0, 0}, t_forward = 0, t_open = 0, t_io_wait = 0;
    MeshState* mesh = nullptr;
    if (flags & ZKML_CHAIN_MESH) {
        mesh = mesh_of(ctx);
        if (!mesh) return set_error(ZKML_ERR_INVALID_ARG, "ZKML_CHAIN_MESH: no peer mesh is open on this device");
    }
    // outs[0] is the model input, outs[l + 1] layer l's output (m x width[l + 1]), in device memory
    std::vector<size_t> width(n_layers + 1);
    std::vector<long long> src(n_layers);
    width[0] = k0;
    for (size_t l = 0; l < n_layers; l++) {
        const std::string at = "layer " + std::to_string(l) + ": ";
        src[l] = layers[l].src == ZKML_CHAIN_PREV ? (long long)l - 1 : layers[l].src;
        if (src[l] < -1 || src[l] >= (long long)l) return set_error(ZKML_ERR_INVALID_ARG, at + "bad input layer");
        const size_t w = width[src[l] + 1];
        const int t = layers[l].type;
        if (t == ZKML_LAYER_LINEAR) {
            if (!layers[l].weight || layers[l].n == 0 || layers[l].n > (1u << 30))
                return set_error(ZKML_ERR_INVALID_ARG, at + "bad Linear layer");
            width[l + 1] = layers[l].n;
        } else if (t == ZKML_LAYER_RELU || t == ZKML_LAYER_RMSNORM || t == ZKML_LAYER_LAYERNORM) {
            width[l + 1] = w;
        } else if (t == ZKML_LAYER_ACTIVATION) {
            if (layers[l].n < 2 || layers[l].n > 5)
                return set_error(ZKML_ERR_INVALID_ARG, at + "Activation tag must be 2 (GELU), 3 (Sigmoid), 4 (Softmax) "
                                                            "or 5 (SiLU); ReLU is ZKML_LAYER_RELU");
            width[l + 1] = w;
        } else if (t == ZKML_LAYER_ADD || t == ZKML_LAYER_MUL) {
            if (layers[l].lhs < 0 || layers[l].lhs >= (long long)l || width[layers[l].lhs + 1] != w)
                return set_error(ZKML_ERR_INVALID_ARG, at + "bad lhs layer (a lower layer of the same width)");
            width[l + 1] = w;
        } else {
            return set_error(ZKML_ERR_INVALID_ARG, at + "unsupported layer type");
        }
    }
    std::vector<DevBuf> outs(n_layers + 1);
    struct Release {
        std::vector<DevBuf>& v;
        ~Release() {
            for (DevBuf& b : v) b.release();
        }
    } release{outs};
    for (size_t l = 0; l <= n_layers; l++)
        if ((rc = outs[l].ensure(m * width[l] * 4))) return rc;
    {
        const void* Iv = nullptr;
        if ((rc = device_view(ctx, input, m * k0 * 4, ctx->a_in, &Iv))) return rc;
        pad_rows_cols_kernel<<<blocks_for(m * k0), 256, 0, s>>>(static_cast<const uint32_t*>(Iv), m, k0, k0, m * k0,
                                                                outs[0].as<uint32_t>());
        ctx->launches++;
    }
    auto in_of = [&](size_t l) { return outs[src[l] + 1].as<uint32_t>(); };
    for (size_t l = 0; l < n_layers; l++) {
        const size_t w = width[src[l] + 1];
        const int t = layers[l].type;
        if (t == ZKML_LAYER_LINEAR) {
            if ((rc = zkml_matmul_m31(ctx, in_of(l), m, w, layers[l].weight, width[l + 1], outs[l + 1].as<uint32_t>())))
                return rc;
        } else if (t == ZKML_LAYER_RMSNORM) {
            if (!ctx->rsqrt_table.ptr) {
                if ((rc = ctx->rsqrt_table.ensure(4u << 16))) return rc;
                ZK_CUDA(cudaMemcpy(ctx->rsqrt_table.ptr, rsqrt_table16().data(), 4u << 16, cudaMemcpyHostToDevice));
            }
            rmsnorm_forward_kernel<<<(unsigned)std::min<size_t>(m, 8192), 256, 0, s>>>(
                in_of(l), (uint32_t)m, (uint32_t)w, minv((uint32_t)(w % P)), ctx->rsqrt_table.as<uint32_t>(),
                outs[l + 1].as<uint32_t>());
            ctx->launches++;
        } else if (t == ZKML_LAYER_LAYERNORM) {
            if (!ctx->rsqrt_table.ptr) {
                if ((rc = ctx->rsqrt_table.ensure(4u << 16))) return rc;
                ZK_CUDA(cudaMemcpy(ctx->rsqrt_table.ptr, rsqrt_table16().data(), 4u << 16, cudaMemcpyHostToDevice));
            }
            launch_layernorm_forward(in_of(l), (uint32_t)m, (uint32_t)w, minv((uint32_t)(w % P)),
                                     ctx->rsqrt_table.as<uint32_t>(), outs[l + 1].as<uint32_t>(), s);
            ctx->launches++;
        } else if (t == ZKML_LAYER_RELU) {
            relu_forward_kernel<<<blocks_for(m * w), 256, 0, s>>>(in_of(l), m * w, outs[l + 1].as<uint32_t>());
            ctx->launches++;
        } else if (t == ZKML_LAYER_ACTIVATION) {
            act_forward_kernel<<<blocks_for(m * w), 256, 0, s>>>(in_of(l), m * w, (int)layers[l].n,
                                                                 outs[l + 1].as<uint32_t>());
            ctx->launches++;
        } else {
            elementwise_kernel<<<blocks_for(m * w), 256, 0, s>>>(outs[layers[l].lhs + 1].as<uint32_t>(), in_of(l),
                                                                 m * w, t == ZKML_LAYER_MUL,
                                                                 outs[l + 1].as<uint32_t>());
            ctx->launches++;
        }
    }
    ZK_CUDA(cudaGetLastError());

    // io commitment (aggregation.rs:235-254) of the model input and output: a sequential
    // Poseidon sponge over every element (one permutation per two elements), known as soon as
    // the forward pass is done, so it runs on a host thread of its own beside the proof
    const size_t wout0 = width[n_layers];
    std::vector<uint32_t> hin(m * k0), hout(m * wout0);
    ZK_CUDA(cudaMemcpyAsync(hin.data(), outs[0].ptr, m * k0 * 4, cudaMemcpyDeviceToHost, s));
    ZK_CUDA(cudaMemcpyAsync(hout.data(), outs[n_layers].ptr, m * wout0 * 4, cudaMemcpyDeviceToHost, s));
    ZK_CUDA(cudaStreamSynchronize(s));
    felt_init();
    int io_rc = ZKML_OK;
    std::thread io_thread(
        [&] { io_rc = zkml_io_commitment(hin.data(), m, k0, hout.data(), m, wout0, out_io); });
    // the thread must be joined on every return path
    struct Joiner {
        std::thread& t;
        ~Joiner() {
            if (t.joinable()) t.join();
        }
    } joiner{io_thread};

    t_forward = ms_since(t_call);
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
    LogupScratch& b = ctx->lu;
    RoundScratch rs = ctx->round_scratch();
    rs.sig = ctx->d_sig;
    uint32_t words[16];
    qm31 value;
    {
        if ((rc = b.x.ensure(nout * 4)) || (rc = b.eq.ensure(nout * 16))) return rc;
        pad_rows_cols_kernel<<<blocks_for(nout), 256, 0, s>>>(outs[n_layers].as<uint32_t>(), m, wout, pout, nout,
                                                              b.x.as<uint32_t>());
        launch_eq_table(point.data(), nvo, b.eq.as<uint4>(), nout, s);
        rs.seq = ++ctx->sig_seq;
        launch_eq_dot(b.eq.as<uint4>(), b.x.as<uint32_t>(), nullptr, nout, rs, s);
        ctx->launches += 3;
        if ((rc = wait_signal(ctx, rs.seq, words, 4))) return rc;
        value = qm(words[0], words[1], words[2], words[3]);
    }
    ch.mix_qm31(value);
    unsigned npt = nvo;

    const bool v1 = (flags & ZKML_CHAIN_V1_CALLDATA) != 0;
    std::vector<uint64_t> lay_buf(4 * std::max<size_t>(cap, 1));
    Out lay{lay_buf.data(), cap};
    size_t n_proofs = 0;
    struct WeightClaim {
        size_t layer;
        std::vector<qm31> point;
        qm31 value;
    };
    struct Deferred {
        std::vector<qm31> point;
        qm31 value;
        size_t layer;
    };
    std::vector<WeightClaim> wclaims;
    std::vector<Deferred> defs;
    std::vector<char> skip(n_layers, 0);
    static const uint32_t inv2 = minv(2), inv6 = minv(6);
    for (size_t li = n_layers; li-- > 0;) {
        if (skip[li]) continue;
        n_proofs++;
        const size_t w = width[src[li] + 1];
        const int t = layers[li].type;
        const auto t_layer = now();
        struct KindTimer {
            double* acc;
            std::chrono::steady_clock::time_point t0;
            bool on;
            ~KindTimer() {
                if (on) *acc += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
            }
        } kind_timer{&t_kind[t & 7], t_layer, trace};
        if (t == ZKML_LAYER_LINEAR) {
            const size_t n = width[li + 1];
            const unsigned log_k = lg2(np2(w)), log_n = lg2(np2(n));
            std::vector<uint32_t> rp(12 * (log_k + 1)), nxt(4 * (log_m + log_k + 1));
            uint32_t fa[4], fb[4], cv[4] = {value.a, value.b, value.c, value.d};
            if ((rc = zkml_reduce_matmul_layer_gkr(ctx, reinterpret_cast<const uint32_t*>(point.data()), npt, cv,
                                                   in_of(li), m, w, layers[li].weight, n, &chs, rp.data(), fa, fb,
                                                   nxt.data())))
                return rc;
            lay.u64(0);  // tag MatMul
            lay.u64(log_k);
            for (unsigned r = 0; r < log_k; r++) {
                lay.qm(&rp[12 * r]);
                lay.qm(&rp[12 * r + 8]);
            }
            lay.qm(fa);
            lay.qm(fb);
            // weight claim: r_j || sumcheck challenges (prover.rs:1465-1483)
            WeightClaim wc{li, std::vector<qm31>(log_n + log_k), qm(fb[0], fb[1], fb[2], fb[3])};
            for (unsigned i = 0; i < log_n; i++) wc.point[i] = point[log_m + i];
            memcpy(wc.point.data() + log_n, nxt.data() + 4 * log_m, 16 * log_k);
            wclaims.push_back(std::move(wc));
            memcpy(point.data(), nxt.data(), 16 * (log_m + log_k));
            npt = log_m + log_k;
            value = qm(fa[0], fa[1], fa[2], fa[3]);
        } else if (t == ZKML_LAYER_RMSNORM) {
            uint32_t cv[4] = {value.a, value.b, value.c, value.d}, ie[4];
            if ((rc = rmsnorm_reduce_dev(ctx, in_of(li), m, w, w, nullptr, 0,
                                         reinterpret_cast<const uint32_t*>(point.data()), npt, cv, &chs, lay, ie, v1)))
                return rc;
            value = qm(ie[0], ie[1], ie[2], ie[3]);  // the point is unchanged
        } else if (t == ZKML_LAYER_LAYERNORM) {
            uint32_t cv[4] = {value.a, value.b, value.c, value.d}, ie[4];
            if ((rc = layernorm_reduce_dev(ctx, in_of(li), m, w, w, reinterpret_cast<const uint32_t*>(point.data()),
                                           npt, cv, &chs, lay, ie, v1)))
                return rc;
            value = qm(ie[0], ie[1], ie[2], ie[3]);  // the point is unchanged
        } else if (t == ZKML_LAYER_ACTIVATION) {
            // prover.rs:1765-1790: piecewise by default, LogUp under STWO_PIECEWISE_ACTIVATION=0
            const bool logup = (flags & ZKML_CHAIN_ACTIVATION_LOGUP) != 0;
            const int tag = (int)layers[li].n;
            const unsigned nv = lg2(pm * np2(w));
            if (npt != nv)
                return set_error(ZKML_ERR_INVALID_ARG, "layer " + std::to_string(li) + ": claim point size mismatch");
            const size_t tcap = (logup ? ((size_t)1 << (tag == 4 ? 20 : 16)) : 0) + 200 + 40 * (size_t)(nv + 2);
            std::vector<uint64_t> tbuf(4 * tcap);
            size_t tlen = 0;
            uint32_t cv[4] = {value.a, value.b, value.c, value.d}, ie[4];
            std::vector<qm31> nxt(64);
            if (logup)
                rc = zkml_reduce_activation_logup(ctx, in_of(li), m, w, tag,
                                                  reinterpret_cast<const uint32_t*>(point.data()), npt, cv, &chs,
                                                  tbuf.data(), tcap, &tlen, ie);
            else
                rc = zkml_reduce_activation_piecewise(ctx, in_of(li), m, w, tag,
                                                      reinterpret_cast<const uint32_t*>(point.data()), npt, cv, &chs,
                                                      tbuf.data(), tcap, &tlen, ie,
                                                      reinterpret_cast<uint32_t*>(nxt.data()));
            if (rc) return rc;
            // the on-chain record (cairo_serde.rs:1862-1890) drops the LogUp multiplicities
            const size_t mpos = 29 + 12 * (size_t)nv;
            for (size_t i = 0; i < tlen; i++) {
                if (v1 && logup && i == mpos) {
                    lay.u64(0);
                    i += (size_t)tbuf[4 * i];
                    continue;
                }
                lay.push(&tbuf[4 * i]);
            }
            if (!logup) memcpy(point.data(), nxt.data(), 16 * nv);
            value = qm(ie[0], ie[1], ie[2], ie[3]);
        } else if (t == ZKML_LAYER_RELU) {
            std::vector<qm31> nxt(64);
            qm31 nval;
            if ((rc = relu_reduce_dev(ctx, in_of(li), m, w, point.data(), value, &chs, lay, nxt.data(), &nval,
                                      (flags & ZKML_CHAIN_LEGACY_ACTIVATION_RECORD) != 0)))
                return rc;
            npt = lg2(pm * np2(w));
            memcpy(point.data(), nxt.data(), 16 * npt);
            value = nval;
        } else {
            // binary op: input_layers = [lhs, rhs], the trunk is the higher layer index
            const long long il0 = layers[li].lhs, il1 = src[li];
            const bool rhs_trunk = il1 > il0;
            const size_t pw = np2(w), n = pm * pw;
            const unsigned nv = lg2(n);
            if (npt != nv || nv == 0)
                return set_error(ZKML_ERR_INVALID_ARG, "layer " + std::to_string(li) + ": claim point size mismatch");
            const uint32_t* lv = outs[il0 + 1].as<uint32_t>();
            const uint32_t* rv = in_of(li);
            if ((rc = b.eq.ensure(n * 16))) return rc;
            qm31 le, re;
            if (t == ZKML_LAYER_ADD) {
                // reduce_add_layer (prover.rs:6103-6146): both MLEs at the claim point
                if ((rc = b.x.ensure(n * 4)) || (rc = b.m_in.ensure(n * 4))) return rc;
                pad_rows_cols_kernel<<<blocks_for(n), 256, 0, s>>>(lv, m, w, pw, n, b.x.as<uint32_t>());
                pad_rows_cols_kernel<<<blocks_for(n), 256, 0, s>>>(rv, m, w, pw, n, b.m_in.as<uint32_t>());
                launch_eq_table(point.data(), nv, b.eq.as<uint4>(), n, s);
                rs.seq = ++ctx->sig_seq;
                launch_eq_dot(b.eq.as<uint4>(), b.x.as<uint32_t>(), b.m_in.as<uint32_t>(), n, rs, s);
                ctx->launches += 4;
                if ((rc = wait_signal(ctx, rs.seq, words, 8))) return rc;
                le = qm(words[0], words[1], words[2], words[3]);
                re = qm(words[4], words[5], words[6], words[7]);
                ch.mix_qm31(le);
                ch.mix_qm31(re);
                (void)ch.draw_qm31();
                lay.u64(1);  // tag Add
                lay.q(le);
                lay.q(re);
                lay.u64(rhs_trunk ? 1 : 0);
                // process_add_deferred (prover.rs:1424-1463)
                defs.push_back({std::vector<qm31>(point.begin(), point.begin() + npt), rhs_trunk ? le : re,
                                (size_t)(rhs_trunk ? il0 : il1)});
                value = rhs_trunk ? re : le;
            } else {
                // reduce_mul_layer (prover.rs:6172-6280): degree-3 eq-sumcheck of eq(r, x) lhs(x) rhs(x)
                if ((rc = b.w.ensure(n * 16)) || (rc = b.d.ensure(n * 16))) return rc;
                lift_pad_kernel<<<blocks_for(n), 256, 0, s>>>(lv, m, w, pw, n, b.w.as<uint4>());
                lift_pad_kernel<<<blocks_for(n), 256, 0, s>>>(rv, m, w, pw, n, b.d.as<uint4>());
                launch_eq_table(point.data(), nv, b.eq.as<uint4>(), n, s);
                ctx->launches += 3;
                ch.mix_u64(0x4D554C);
                ch.mix_qm31(value);
                std::vector<qm31> rps(3 * nv);
                size_t len = n;
                rs.seq = ++ctx->sig_seq;
                launch_logup_round(b.eq.as<uint4>(), b.w.as<uint4>(), b.d.as<uint4>(), len, false, qzero(), rs, s);
                ctx->launches++;
                for (unsigned r = 0; r < nv; r++) {
                    if ((rc = wait_signal(ctx, rs.seq, words, 16))) return rc;
                    const qm31 s0 = qm(words[0], words[1], words[2], words[3]);
                    const qm31 s1 = qm(words[4], words[5], words[6], words[7]);
                    const qm31 s2 = qm(words[8], words[9], words[10], words[11]);
                    const qm31 s3 = qm(words[12], words[13], words[14], words[15]);
                    const qm31 dd1 = qsub(s1, s0);
                    const qm31 dd2 = qmul_m(qadd(qsub(qsub(s2, s1), s1), s0), inv2);
                    const qm31 dd3 = qmul_m(qsub(qsub(s3, s0), qmul_m(qsub(s2, s1), 3)), inv6);
                    const qm31 c0 = s0, c1 = qadd(qsub(dd1, dd2), qmul_m(dd3, 2)), c2 = qsub(dd2, qmul_m(dd3, 3));
                    rps[3 * r] = c0;
                    rps[3 * r + 1] = c2;
                    rps[3 * r + 2] = dd3;
                    ch.mix_poly_coeffs_deg3(c0, c1, c2, dd3);
                    const qm31 x = ch.draw_qm31();
                    rs.seq = ++ctx->sig_seq;
                    if (len == 2)
                        launch_logup_final(b.eq.as<uint4>(), b.w.as<uint4>(), b.d.as<uint4>(), x, rs, s);
                    else
                        launch_logup_round(b.eq.as<uint4>(), b.w.as<uint4>(), b.d.as<uint4>(), len, true, x, rs, s);
                    ctx->launches++;
                    len /= 2;
                }
                if ((rc = wait_signal(ctx, rs.seq, words, 8))) return rc;
                le = qm(words[0], words[1], words[2], words[3]);
                re = qm(words[4], words[5], words[6], words[7]);
                ch.mix_qm31(le);
                ch.mix_qm31(re);
                (void)ch.draw_qm31();
                lay.u64(2);  // tag Mul
                lay.u64(nv);
                for (unsigned r = 0; r < nv; r++) {
                    lay.q(rps[3 * r]);
                    lay.q(rps[3 * r + 1]);
                    lay.q(rps[3 * r + 2]);
                }
                lay.q(le);
                lay.q(re);
                // the branched Mul (prover.rs:1719-1760): the deferred claim carries rhs_eval, the
                // skip layer leaves the walk, the walk goes on at the same point
                const long long sk = rhs_trunk ? il0 : il1;
                defs.push_back({std::vector<qm31>(point.begin(), point.begin() + npt), re, (size_t)sk});
                skip[sk] = 1;
                value = rhs_trunk ? re : le;
            }
            if ((rc = read_err_flag(ctx)) || (rc = check_err_flag(ctx, "binary layer"))) return rc;
        }
    }

    // one Sequential MLE opening of a weight at a point on the main channel
    auto open_weight = [&](size_t l, const std::vector<qm31>& wpt, uint64_t com[4], std::vector<uint64_t>& obuf,
                           size_t* olen) -> int {
        const size_t k = width[src[l] + 1], n = width[l + 1];
        const size_t pk = np2(k), pn = np2(n);
        const void* Bv = nullptr;
        int e;
        if ((e = device_view(ctx, layers[l].weight, k * n * 4, ctx->b_in, &Bv))) return e;
        DevBuf& bmle = ctx->op.bmle;
        if ((e = bmle.ensure(pk * pn * 16))) return e;
        launch_colmajor_mle(static_cast<const uint32_t*>(Bv), (uint32_t)k, (uint32_t)n, pk, pn, bmle.as<uint4>(), s);
        ctx->launches++;
        const unsigned nv = (unsigned)wpt.size();
        const size_t qcap = 64 + (n_queries + 1) * (2 + (size_t)nv * (10 + 2 * (nv + 1)));
        obuf.resize(qcap * 4);
        Out oo{obuf.data(), qcap};
        KTimer tm(ctx, KC_MERKLE);
        if ((e = prove_opening_dev(ctx, bmle.as<uint4>(), nv, wpt.data(), &chs, n_queries, com, oo, nullptr, mesh)))
            return e;
        *olen = oo.len;
        return 0;
    };

    // deferred proofs of the skip branches and their openings (prover.rs:1918-2047)
    std::vector<uint64_t> dsec_buf(4 * std::max<size_t>(cap, 1));
    Out dsec{dsec_buf.data(), cap};
    dsec.u64(defs.size());
    std::vector<std::array<uint64_t, 4>> dcoms(defs.size());
    std::vector<std::vector<uint64_t>> dobufs(defs.size());
    std::vector<size_t> dolens(defs.size());
    for (size_t i = 0; i < defs.size(); i++) {
        const Deferred& d = defs[i];
        const size_t L = d.layer;
        if (layers[L].type != ZKML_LAYER_LINEAR)
            return set_error(ZKML_ERR_INVALID_ARG, "deferred proof not yet supported for layer " + std::to_string(L) +
                                                       " (only Linear skip branches)");
        const size_t w = width[src[L] + 1], n = width[L + 1];
        const unsigned log_k = lg2(np2(w)), log_n = lg2(np2(n));
        ch.mix_qm31(d.value);
        std::vector<uint32_t> rp(12 * (log_k + 1)), nxt(4 * (log_m + log_k + 1));
        uint32_t fa[4], fb[4], cv[4] = {d.value.a, d.value.b, d.value.c, d.value.d};
        if ((rc = zkml_reduce_matmul_layer_gkr(ctx, reinterpret_cast<const uint32_t*>(d.point.data()), d.point.size(),
                                               cv, in_of(L), m, w, layers[L].weight, n, &chs, rp.data(), fa, fb,
                                               nxt.data())))
            return rc;
        std::vector<qm31> wpt(log_n + log_k);
        for (unsigned j = 0; j < log_n; j++) wpt[j] = d.point[log_m + j];
        memcpy(wpt.data() + log_n, nxt.data() + 4 * log_m, 16 * log_k);
        if ((rc = open_weight(L, wpt, dcoms[i].data(), dobufs[i], &dolens[i]))) return rc;
        // serialize_gkr_proof_data_only's deferred record (cairo_serde.rs:2238-2276)
        dsec.q(d.value);
        dsec.u64(0);  // kind MatMul
        dsec.u64(m);
        dsec.u64(w);
        dsec.u64(n);
        dsec.u64(log_k);
        for (unsigned r = 0; r < log_k; r++) {
            dsec.qm(&rp[12 * r]);
            dsec.qm(&rp[12 * r + 8]);
        }
        dsec.qm(fa);
        dsec.qm(fb);
        dsec.push(dcoms[i].data());
    }
    const auto t_open0 = now();
    // the walk's Sequential weight openings on the main channel, in walk order (prover.rs:2140-2171)
    std::vector<std::array<uint64_t, 4>> coms(wclaims.size());
    std::vector<std::vector<uint64_t>> obufs(wclaims.size());
    std::vector<size_t> olens(wclaims.size());
    for (size_t i = 0; i < wclaims.size(); i++)
        if ((rc = open_weight(wclaims[i].layer, wclaims[i].point, coms[i].data(), obufs[i], &olens[i]))) return rc;

    t_open = ms_since(t_open0);
    const auto t_join = now();
    io_thread.join();
    t_io_wait = ms_since(t_join);
    if ((rc = io_rc)) return rc;
    if (trace)
        fprintf(stderr,
                "[zkml chain] forward %.2f ms; walk: linear %.2f, relu %.2f, rmsnorm %.2f, add %.2f, mul %.2f, "
                "layernorm %.2f, activation %.2f ms; deferred+openings %.2f ms; io wait %.2f ms; total %.2f ms\n",
                t_forward, t_kind[0], t_kind[1], t_kind[2], t_kind[3], t_kind[4], t_kind[5], t_kind[6], t_open,
                t_io_wait, ms_since(t_call));

    Out o{out_calldata, out_calldata ? cap : 0};
    if (v1 && model_id) {
        o.push(model_id);
        // raw_io_data (serialize_raw_io, cairo_serde.rs:3714-3732)
        o.u64(6 + m * k0 + m * wout);
        o.u64(m);
        o.u64(k0);
        o.u64(m * k0);
        for (uint32_t v : hin) o.u64(v);
        o.u64(m);
        o.u64(wout);
        o.u64(m * wout);
        for (uint32_t v : hout) o.u64(v);
        o.u64(n_layers);  // circuit_depth
        o.u64(n_proofs);  // num_layers: the proof's layer records
        size_t n_lin = 0;
        for (size_t l = 0; l < n_layers; l++) n_lin += layers[l].type == ZKML_LAYER_LINEAR;
        o.u64(3 * n_lin);  // matmul_dims in walk order (extract_matmul_dims, starknet.rs:1557-1569)
        for (size_t l = n_layers; l-- > 0;)
            if (layers[l].type == ZKML_LAYER_LINEAR) {
                o.u64(m);
                o.u64(width[src[l] + 1]);
                o.u64(width[l + 1]);
            }
        o.u64(0);  // dequantize_bits
    }
    auto append = [&](const Out& from) {
        for (size_t j = 0; j < from.len && j < from.cap; j++) o.push(from.buf + 4 * j);
    };
    if (v1) {
        o.u64(lay.len + dsec.len);  // proof_data
        append(lay);
        append(dsec);
        o.u64(wclaims.size() + defs.size());  // weight commitments: the walk's, then the deferred
        for (auto& c : coms) o.push(c.data());
        for (auto& c : dcoms) o.push(c.data());
        o.u64(wclaims.size() + defs.size());  // opening proofs, same order
        for (size_t i = 0; i < wclaims.size(); i++)
            for (size_t j = 0; j < olens[i]; j++) o.push(&obufs[i][4 * j]);
        for (size_t i = 0; i < defs.size(); i++)
            for (size_t j = 0; j < dolens[i]; j++) o.push(&dobufs[i][4 * j]);
    } else {
        o.u64(n_proofs);
        append(lay);
        o.u64(npt);  // input claim
        for (unsigned i = 0; i < npt; i++) o.q(point[i]);
        o.q(value);
        o.u64(wclaims.size());
        for (auto& c : coms) o.push(c.data());
        o.u64(wclaims.size());
        for (size_t i = 0; i < wclaims.size(); i++) {
            o.u64(wclaims[i].point.size());
            for (const qm31& p : wclaims[i].point) o.q(p);
            o.q(wclaims[i].value);
            for (size_t j = 0; j < olens[i]; j++) o.push(&obufs[i][4 * j]);
        }
    }
    if (!v1) o.push(out_io);
    memcpy(out_digest, chs.digest, 32);
    *out_len = o.len;
    if (o.overflow || lay.overflow || dsec.overflow)
        return set_error(ZKML_ERR_INVALID_ARG, "calldata buffer too small: need more than " + std::to_string(o.len) +
                                                   " felts");
    return ZKML_OK;
}

extern "C" int zkml_prove_gkr_chain(zkml_ctx* ctx, const uint32_t* input, size_t m, size_t k0,
                                    const zkml_chain_layer* layers, size_t n_layers, const uint64_t* policy,
                                    size_t n_queries, int flags, uint64_t* out_calldata, size_t cap, size_t* out_len,
                                    uint64_t out_digest[4], uint64_t out_io[4]) {
    return prove_chain(ctx, nullptr, input, m, k0, layers, n_layers, policy, n_queries, flags, out_calldata, cap,
                       out_len, out_digest, out_io);
}

extern "C" int zkml_build_verify_model_gkr_calldata(zkml_ctx* ctx, const uint64_t model_id[4], const uint32_t* input,
                                                    size_t m, size_t k0, const zkml_chain_layer* layers,
                                                    size_t n_layers, const uint64_t* policy, size_t n_queries,
                                                    int flags, uint64_t* out_calldata, size_t cap, size_t* out_len,
                                                    uint64_t out_digest[4], uint64_t out_io[4]) {
    if (!model_id) return set_error(ZKML_ERR_INVALID_ARG, "NULL model_id");
    return prove_chain(ctx, model_id, input, m, k0, layers, n_layers, policy, n_queries,
                       flags | ZKML_CHAIN_V1_CALLDATA, out_calldata, cap, out_len, out_digest, out_io);
}
