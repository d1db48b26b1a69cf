// Forward M31 matrix product C = A * B mod P on the integer tensor pipe
// (replaces gpu_matmul_m31_full, engine/src/gpu_sumcheck.rs:3104-3196, the
// forward pass that produces the GraphExecution the GKR prover walks).
//
// Both operands are split into byte planes (imma.cuh): C = sum_{a,b} 256^(a+b)
// A_a B_b, each A_a B_b an exact u8 GEMM on mma.m16n8k32.  A (m x k, row major)
// is read as is: four consecutive k of a row are one 16-byte load whose byte
// planes are A fragments; B (k x n, row major) is read in place, four rows at a
// time, and split into planes in registers.  The sixteen plane pairs share seven accumulators
// by weight w = a + b (at most four pairs per weight, each below
// 255^2 * 8192 per K chunk, so a chunk of 8192 stays below 2^31); every K
// chunk ends with sum_w 256^w acc_w mod P added to 64-bit lazy sums.
#include <cuda_runtime.h>

#include <cstdlib>

#include "context.hpp"
#include "gkr.cuh"
#include "imma.cuh"
#include "round_arith.cuh"

namespace zk {

constexpr uint32_t GEMM_KCHUNK = 8192;

// One block = 4 x NT x KS warps over a 64-row group and 8 NT output columns:
// warp w takes row tile w % 4 (16 rows), N-tile (w / 4) % NT and K part
// w / (4 NT); K parts meet in shared memory at the end.  B is read in place (row major): the four
// values B[t .. t+3][j] a B-fragment word needs are four 4-byte loads whose
// byte planes are the four planes' words; the lanes of a warp cover 8
// consecutive columns x 4 rows per load, so every 32-byte sector is used.
// The next K step's loads are issued before this step's MMAs.
constexpr int GEMM_NT = 1;  // 8-column N-tiles per block
constexpr int GEMM_KS = 2;  // K splits per block

struct GemmLoads {
    uint4 a[4];      // A: rows r0 / r1, k = t + 4 tg (+16)
    uint32_t b[8];   // B: rows t + 4 tg + e (e < 4) and t + 16 + 4 tg + e, column j
};

__device__ __forceinline__ void gemm_load(GemmLoads& L, const uint4* a0p, const uint4* a1p, bool v0, bool v1,
                                          const uint32_t* __restrict__ B, uint32_t k, uint32_t n, uint32_t j,
                                          bool wj, uint32_t t, uint32_t tg) {
    const uint32_t ta = t + 4 * tg, tb = ta + 16;
    const uint4 z = make_uint4(0, 0, 0, 0);
    L.a[0] = (v0 && ta < k) ? __ldg(a0p + ta / 4) : z;
    L.a[1] = (v1 && ta < k) ? __ldg(a1p + ta / 4) : z;
    L.a[2] = (v0 && tb < k) ? __ldg(a0p + tb / 4) : z;
    L.a[3] = (v1 && tb < k) ? __ldg(a1p + tb / 4) : z;
#pragma unroll
    for (int e = 0; e < 4; e++) {
        L.b[e] = (wj && ta + e < k) ? __ldg(B + (size_t)(ta + e) * n + j) : 0u;
        L.b[4 + e] = (wj && tb + e < k) ? __ldg(B + (size_t)(tb + e) * n + j) : 0u;
    }
}

template <int NT, int KS>
__global__ void __launch_bounds__(4 * NT * KS * 32) m31_gemm_tc_kernel(const uint32_t* __restrict__ A,
                                                                     const uint32_t* __restrict__ B,
                                                                     uint32_t* __restrict__ Cm, uint32_t m, uint32_t k,
                                                                     uint32_t n, uint32_t* __restrict__ err) {
    __shared__ uint64_t part[KS > 1 ? 4 * NT : 1][32][4];
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, tg = lane & 3;
    const uint32_t rt = warp & 3, nt = (warp >> 2) % NT, half = warp / (4 * NT);
    const uint32_t r0 = blockIdx.y * 64 + rt * 16 + g, r1 = r0 + 8;
    const uint32_t j0 = blockIdx.x * 8 * NT + 8 * nt, j = j0 + g;
    const bool v0 = r0 < m, v1 = r1 < m, wj = j < n;
    const uint4* a0p = reinterpret_cast<const uint4*>(A + (size_t)(v0 ? r0 : 0) * k);
    const uint4* a1p = reinterpret_cast<const uint4*>(A + (size_t)(v1 ? r1 : 0) * k);
    // this warp's half of the K steps
    const uint32_t steps = (k + 31) / 32, per = (steps + KS - 1) / KS;
    const uint32_t s_begin = min(steps, half * per), s_end = min(steps, s_begin + per);
    uint64_t tot[4] = {0, 0, 0, 0};
    uint32_t bad = 0;
    GemmLoads cur, nxt;
    if (s_begin < s_end) gemm_load(cur, a0p, a1p, v0, v1, B, k, n, j, wj, 32 * s_begin, tg);
    for (uint32_t c0 = s_begin; c0 < s_end; c0 += GEMM_KCHUNK / 32) {
        const uint32_t c_end = min(s_end, c0 + GEMM_KCHUNK / 32);
        int acc[7][4];
#pragma unroll
        for (int w = 0; w < 7; w++)
#pragma unroll
            for (int e = 0; e < 4; e++) acc[w][e] = 0;
        for (uint32_t st = c0; st < c_end; st++) {
            if (st + 1 < s_end) gemm_load(nxt, a0p, a1p, v0, v1, B, k, n, j, wj, 32 * (st + 1), tg);
            uint32_t pa[4][4], pb[4][2];
#pragma unroll
            for (int f = 0; f < 4; f++) {
                bad |= cur.a[f].x | cur.a[f].y | cur.a[f].z | cur.a[f].w;
                byte_planes(cur.a[f], pa[0][f], pa[1][f], pa[2][f], pa[3][f]);
            }
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const uint4 bw = make_uint4(cur.b[4 * h], cur.b[4 * h + 1], cur.b[4 * h + 2], cur.b[4 * h + 3]);
                bad |= bw.x | bw.y | bw.z | bw.w;
                byte_planes(bw, pb[0][h], pb[1][h], pb[2][h], pb[3][h]);
            }
#pragma unroll
            for (int a = 0; a < 4; a++)
#pragma unroll
                for (int b = 0; b < 4; b++) mma_u8(acc[a + b], pa[a], pb[b][0], pb[b][1]);
            cur = nxt;
        }
#pragma unroll
        for (int e = 0; e < 4; e++) {
            uint64_t sum = 0;
#pragma unroll
            for (int w = 0; w < 7; w++) sum = acc_fold(sum, mul_wide((uint32_t)acc[w][e], pow256(w)));
            tot[e] = acc_fold(tot[e], (uint64_t)canon64(sum));
        }
    }
    static_assert(KS == 1 || KS == 2, "K split");
    if (bad & 0x80000000u) atomicOr(err, 1u);
    if (KS > 1) {  // K halves meet in shared memory
        if (half) {
#pragma unroll
            for (int e = 0; e < 4; e++) part[warp % (4 * NT)][lane][e] = tot[e];
        }
        __syncthreads();
        if (half) return;
#pragma unroll
        for (int e = 0; e < 4; e++) tot[e] = acc_fold(tot[e], part[warp][lane][e]);
    }
    {
        // C fragment: e = 0, 1 -> row r0, columns 2 tg, 2 tg + 1; e = 2, 3 -> row r1
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const uint32_t row = e < 2 ? r0 : r1, col = j0 + 2 * tg + (e & 1);
            if (row < m && col < n) Cm[(size_t)row * n + col] = canon64(tot[e]);
        }
    }
}

}  // namespace zk

using namespace zk;

extern "C" int zkml_matmul_m31(zkml_ctx* ctx, const uint32_t* a, size_t m, size_t k, const uint32_t* b, size_t n,
                               uint32_t* c) {
    if (!ctx || !a || !b || !c) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    if (m == 0 || k == 0 || n == 0) return set_error(ZKML_ERR_INVALID_ARG, "empty matrix");
    if (m > (1u << 30) || k > (1u << 30) || n > (1u << 30) || m * k > ((size_t)1 << 34) || k * n > ((size_t)1 << 34))
        return set_error(ZKML_ERR_INVALID_ARG, "matrix too large");
    ZK_CUDA(cudaSetDevice(ctx->device));
    cudaStream_t s = ctx->stream;
    const void *A = nullptr, *B = nullptr;
    int rc = device_view(ctx, a, m * k * 4, ctx->a_in, &A);
    if (!rc) rc = device_view(ctx, b, k * n * 4, ctx->b_in, &B);
    if (rc) return rc;
    // output: in place when c is device memory of this GPU, else staged and copied back
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, c) != cudaSuccess) {
        cudaGetLastError();
        attr.type = cudaMemoryTypeUnregistered;
    }
    const bool dev_out = attr.type == cudaMemoryTypeDevice && attr.device == ctx->device;
    uint32_t* C = c;
    if (!dev_out) {
        if ((rc = ctx->op.cbuf.ensure(m * n * 4))) return rc;
        C = ctx->op.cbuf.as<uint32_t>();
    }
    const uint32_t* Ad = static_cast<const uint32_t*>(A);
    static const bool tc_on = !(getenv("ZKML_GEMM_TC") && getenv("ZKML_GEMM_TC")[0] == '0');  // 0: CUDA cores
    if (tc_on && k % 4 == 0 && (reinterpret_cast<uintptr_t>(Ad) & 15) == 0) {
        dim3 gg((unsigned)((n + 8 * GEMM_NT - 1) / (8 * GEMM_NT)), (unsigned)((m + 63) / 64));
        m31_gemm_tc_kernel<GEMM_NT, GEMM_KS><<<gg, 4 * GEMM_NT * GEMM_KS * 32, 0, s>>>(Ad, static_cast<const uint32_t*>(B), C, (uint32_t)m,
                                                           (uint32_t)k, (uint32_t)n, ctx->err_flag());
        ctx->launches++;
    } else {
        launch_m31_gemm(Ad, static_cast<const uint32_t*>(B), C, (uint32_t)m, (uint32_t)k, (uint32_t)n, s);
        ctx->launches++;
    }
    ZK_CUDA(cudaGetLastError());
    if (!dev_out) ZK_CUDA(cudaMemcpyAsync(c, C, m * n * 4, cudaMemcpyDeviceToHost, s));
    if ((rc = read_err_flag(ctx)) || (rc = check_err_flag(ctx, "matmul_m31"))) return rc;
    return ZKML_OK;
}
