// Forward M31 matrix product C = A * B mod P on the integer tensor pipe
// (replaces gpu_matmul_m31_full, engine/src/gpu_sumcheck.rs:3104-3196, the
// forward pass that produces the GraphExecution the GKR prover walks).
//
// Both operands are split into byte planes (imma.cuh): C = sum_{a,b} 256^(a+b)
// A_a B_b, each A_a B_b an exact u8 GEMM on mma.m16n8k32.  A (m x k, row major)
// is read as is: four consecutive k of a row are one 16-byte load whose byte
// planes are A fragments.  B (k x n, row major) is first packed into four
// planes (in the order the B fragments are read, bp_offset) by a shared-memory
// transpose.  The sixteen plane pairs share seven accumulators
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

// Packed right operand, laid out in the order the B fragments are read: for
// column j, K step s (32 values of t) and fragment lane tg (0..3), 32 bytes =
// for each plane b the two fragment words (t = 32 s + 4 tg + [0, 4) and
// t = 32 s + 16 + 4 tg + [0, 4)), so a lane fetches all four planes of one K
// step with two 16-byte loads.  Entries with t >= k are zero.
__device__ __forceinline__ size_t bp_offset(uint32_t j, uint32_t s, uint32_t tg, uint32_t ksteps) {
    return (((size_t)j * ksteps + s) * 4 + tg) * 32;
}

__global__ void __launch_bounds__(256) pack_b_planes_kernel(const uint32_t* __restrict__ B, uint32_t k, uint32_t n,
                                                            uint32_t kpad, uint8_t* __restrict__ Bp,
                                                            uint32_t* __restrict__ err) {
    __shared__ uint32_t tile[32][33];
    const uint32_t j0 = blockIdx.x * 32, s = blockIdx.y, t0 = s * 32;
    const uint32_t tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    uint32_t bad = 0;
    for (uint32_t r = ty; r < 32; r += 8) {
        const uint32_t t = t0 + r, j = j0 + tx;
        uint32_t v = 0;
        if (t < k && j < n) v = B[(size_t)t * n + j];
        bad |= v;
        tile[r][tx] = v;
    }
    __syncthreads();
    if (threadIdx.x < 128) {  // thread -> (column j0 + jl, fragment lane tg)
        const uint32_t jl = threadIdx.x >> 2, tg = threadIdx.x & 3, j = j0 + jl;
        if (j < n) {
            uint32_t p0[4], p1[4];
            byte_planes(make_uint4(tile[4 * tg][jl], tile[4 * tg + 1][jl], tile[4 * tg + 2][jl], tile[4 * tg + 3][jl]),
                        p0[0], p0[1], p0[2], p0[3]);
            byte_planes(make_uint4(tile[16 + 4 * tg][jl], tile[17 + 4 * tg][jl], tile[18 + 4 * tg][jl],
                                   tile[19 + 4 * tg][jl]),
                        p1[0], p1[1], p1[2], p1[3]);
            uint4* dst = reinterpret_cast<uint4*>(Bp + bp_offset(j, s, tg, kpad / 32));
            dst[0] = make_uint4(p0[0], p1[0], p0[1], p1[1]);
            dst[1] = make_uint4(p0[2], p1[2], p0[3], p1[3]);
        }
    }
    if (bad & 0x80000000u) atomicOr(err, 1u);
}

// One block: 4 warps x 16 rows (a 64-row group) by 16 columns; warp w takes
// rows 64 * blockIdx.y + 16 w ...  All warps of a block read the same B plane
// words, so B comes from DRAM once and from L1 for the other warps.
__global__ void __launch_bounds__(128) m31_gemm_tc_kernel(const uint32_t* __restrict__ A, const uint8_t* __restrict__ Bp,
                                                          uint32_t* __restrict__ Cm, uint32_t m, uint32_t k, uint32_t n,
                                                          uint32_t kpad, uint32_t* __restrict__ err) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, tg = lane & 3;
    const uint32_t r0 = blockIdx.y * 64 + warp * 16 + g, r1 = r0 + 8;
    const uint32_t j0 = blockIdx.x * 16;
    const bool v0 = r0 < m, v1 = r1 < m;
    const uint4* a0p = reinterpret_cast<const uint4*>(A + (size_t)(v0 ? r0 : 0) * k);
    const uint4* a1p = reinterpret_cast<const uint4*>(A + (size_t)(v1 ? r1 : 0) * k);
    const uint32_t ksteps = kpad / 32;
    const uint32_t jb0 = j0 + g, jb1 = j0 + 8 + g;  // B fragment columns of the two N-tiles
    const bool w0 = jb0 < n, w1 = jb1 < n;
    uint64_t tot[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
    uint32_t bad = 0;
    for (uint32_t c0 = 0; c0 < kpad; c0 += GEMM_KCHUNK) {
        const uint32_t c_end = min(kpad, c0 + GEMM_KCHUNK);
        int acc[7][2][4];
#pragma unroll
        for (int w = 0; w < 7; w++)
#pragma unroll
            for (int q = 0; q < 2; q++)
#pragma unroll
                for (int e = 0; e < 4; e++) acc[w][q][e] = 0;
        for (uint32_t t = c0; t < c_end; t += 32) {
            const uint32_t ta = t + 4 * tg, tb = ta + 16;
            const uint4 z = make_uint4(0, 0, 0, 0);
            uint4 x[4];
            x[0] = (v0 && ta < k) ? __ldg(a0p + ta / 4) : z;
            x[1] = (v1 && ta < k) ? __ldg(a1p + ta / 4) : z;
            x[2] = (v0 && tb < k) ? __ldg(a0p + tb / 4) : z;
            x[3] = (v1 && tb < k) ? __ldg(a1p + tb / 4) : z;
            uint32_t pa[4][4];
#pragma unroll
            for (int f = 0; f < 4; f++) {
                bad |= x[f].x | x[f].y | x[f].z | x[f].w;
                byte_planes(x[f], pa[0][f], pa[1][f], pa[2][f], pa[3][f]);
            }
            uint32_t bb[2][4][2];
            const uint32_t ks = t / 32;
#pragma unroll
            for (int q = 0; q < 2; q++) {
                const bool ok = q ? w1 : w0;
                uint4 u0 = make_uint4(0, 0, 0, 0), u1 = u0;
                if (ok) {
                    const uint4* src = reinterpret_cast<const uint4*>(Bp + bp_offset(q ? jb1 : jb0, ks, tg, ksteps));
                    u0 = __ldg(src);
                    u1 = __ldg(src + 1);
                }
                bb[q][0][0] = u0.x; bb[q][0][1] = u0.y; bb[q][1][0] = u0.z; bb[q][1][1] = u0.w;
                bb[q][2][0] = u1.x; bb[q][2][1] = u1.y; bb[q][3][0] = u1.z; bb[q][3][1] = u1.w;
            }
#pragma unroll
            for (int q = 0; q < 2; q++)
#pragma unroll
                for (int a = 0; a < 4; a++)
#pragma unroll
                    for (int b = 0; b < 4; b++) mma_u8(acc[a + b][q], pa[a], bb[q][b][0], bb[q][b][1]);
        }
#pragma unroll
        for (int q = 0; q < 2; q++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                uint64_t sum = 0;
#pragma unroll
                for (int w = 0; w < 7; w++) sum = acc_fold(sum, mul_wide((uint32_t)acc[w][q][e], pow256(w)));
                tot[q][e] = acc_fold(tot[q][e], (uint64_t)canon64(sum));
            }
    }
    // C fragment: e = 0, 1 -> row r0, columns 2 tg, 2 tg + 1 of N-tile q; e = 2, 3 -> row r1
#pragma unroll
    for (int q = 0; q < 2; q++)
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const uint32_t row = e < 2 ? r0 : r1, col = j0 + 8 * q + 2 * tg + (e & 1);
            if (row < m && col < n) Cm[(size_t)row * n + col] = canon64(tot[q][e]);
        }
    if (bad & 0x80000000u) atomicOr(err, 1u);
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
        const size_t kpad = (k + 31) / 32 * 32;
        if ((rc = ctx->gemm_planes.ensure(4 * n * kpad))) return rc;
        dim3 pg((unsigned)((n + 31) / 32), (unsigned)(kpad / 32));
        pack_b_planes_kernel<<<pg, 256, 0, s>>>(static_cast<const uint32_t*>(B), (uint32_t)k, (uint32_t)n,
                                                 (uint32_t)kpad, ctx->gemm_planes.as<uint8_t>(), ctx->err_flag());
        dim3 gg((unsigned)((n + 15) / 16), (unsigned)((m + 63) / 64));
        m31_gemm_tc_kernel<<<gg, 128, 0, s>>>(Ad, ctx->gemm_planes.as<uint8_t>(), C, (uint32_t)m, (uint32_t)k,
                                               (uint32_t)n, (uint32_t)kpad, ctx->err_flag());
        ctx->launches += 2;
    } else {
        launch_m31_gemm(Ad, static_cast<const uint32_t*>(B), C, (uint32_t)m, (uint32_t)k, (uint32_t)n, s);
        ctx->launches++;
    }
    ZK_CUDA(cudaGetLastError());
    if (!dev_out) ZK_CUDA(cudaMemcpyAsync(c, C, m * n * 4, cudaMemcpyDeviceToHost, s));
    if ((rc = read_err_flag(ctx)) || (rc = check_err_flag(ctx, "matmul_m31"))) return rc;
    return ZKML_OK;
}
