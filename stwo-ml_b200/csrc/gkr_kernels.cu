// Layout and forward-pass kernels used by the single-layer GKR proof:
//  * the column-major padded weight MLE (components/matmul.rs:227-262,
//    matrix_to_mle_col_major_padded): out[j * pk + i] = B[i][j] as QM31,
//    written through 32 x 32 shared-memory tiles so both the row-major reads
//    and the column-major writes are coalesced;
//  * the M31 matrix product C = A . B (components/matmul.rs:572-627) that the
//    IO commitment hashes, as a 64 x 64 register-tiled CUDA-core kernel with
//    64-bit lazy accumulation (reduced every four products).
#include <cuda_runtime.h>

#include "gkr.cuh"
#include "qm31.cuh"

namespace zk {

__global__ void colmajor_mle_kernel(const uint32_t* __restrict__ B, uint32_t k, uint32_t n, size_t pk, size_t pn,
                                    uint4* __restrict__ out) {
    __shared__ uint32_t tile[32][33];
    const size_t i0 = (size_t)blockIdx.y * 32, j0 = (size_t)blockIdx.x * 32;  // tile of rows i, cols j
    const int tx = threadIdx.x, ty = threadIdx.y;                            // 32 x 8 threads
    for (int r = ty; r < 32; r += 8) {
        const size_t i = i0 + r, j = j0 + tx;
        tile[r][tx] = (i < k && j < n) ? red32(B[i * n + j]) : 0u;
    }
    __syncthreads();
    for (int c = ty; c < 32; c += 8) {
        const size_t j = j0 + c, i = i0 + tx;
        if (j < pn && i < pk) out[j * pk + i] = make_uint4(tile[tx][c], 0, 0, 0);
    }
}

void launch_colmajor_mle(const uint32_t* B, uint32_t k, uint32_t n, size_t pk, size_t pn, uint4* out,
                         cudaStream_t s) {
    dim3 grid((unsigned)((pn + 31) / 32), (unsigned)((pk + 31) / 32));
    colmajor_mle_kernel<<<grid, dim3(32, 8), 0, s>>>(B, k, n, pk, pn, out);
}

// C[i][j] = sum_l A[i][l] B[l][j] mod P; 64 x 64 tile per 256-thread block,
// each thread a 4 x 4 sub-tile; K staged in chunks of 16 through shared memory.
__global__ void __launch_bounds__(256) m31_gemm_kernel(const uint32_t* __restrict__ A, const uint32_t* __restrict__ B,
                                                       uint32_t* __restrict__ Cm, uint32_t m, uint32_t k, uint32_t n) {
    __shared__ uint32_t As[16][64 + 1];
    __shared__ uint32_t Bs[16][64 + 1];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const uint32_t row0 = blockIdx.y * 64, col0 = blockIdx.x * 64;
    unsigned long long acc[4][4];
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
        for (int b = 0; b < 4; b++) acc[a][b] = 0;
    for (uint32_t l0 = 0; l0 < k; l0 += 16) {
        for (int e = threadIdx.x; e < 16 * 64; e += 256) {
            const int rr = e / 16, ll = e % 16;  // A tile: 64 rows x 16 k
            const uint32_t gi = row0 + rr, gl = l0 + ll;
            As[ll][rr] = (gi < m && gl < k) ? red32(A[(size_t)gi * k + gl]) : 0u;
            const int bl = e / 64, bc = e % 64;  // B tile: 16 k x 64 cols
            const uint32_t gbl = l0 + bl, gbc = col0 + bc;
            Bs[bl][bc] = (gbl < k && gbc < n) ? red32(B[(size_t)gbl * n + gbc]) : 0u;
        }
        __syncthreads();
#pragma unroll
        for (int ll = 0; ll < 16; ll++) {
            uint32_t av[4], bv[4];
#pragma unroll
            for (int a = 0; a < 4; a++) av[a] = As[ll][ty * 4 + a];
#pragma unroll
            for (int b = 0; b < 4; b++) bv[b] = Bs[ll][tx * 4 + b];
#pragma unroll
            for (int a = 0; a < 4; a++)
#pragma unroll
                for (int b = 0; b < 4; b++) acc[a][b] += (unsigned long long)av[a] * bv[b];
            if ((ll & 3) == 3) {
#pragma unroll
                for (int a = 0; a < 4; a++)
#pragma unroll
                    for (int b = 0; b < 4; b++) acc[a][b] = (acc[a][b] & P) + (acc[a][b] >> 31);
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
        for (int b = 0; b < 4; b++) {
            const uint32_t i = row0 + ty * 4 + a, j = col0 + tx * 4 + b;
            if (i < m && j < n) Cm[(size_t)i * n + j] = red64(acc[a][b]);
        }
}

void launch_m31_gemm(const uint32_t* A, const uint32_t* B, uint32_t* C, uint32_t m, uint32_t k, uint32_t n,
                     cudaStream_t s) {
    dim3 grid((n + 63) / 64, (m + 63) / 64);
    m31_gemm_kernel<<<grid, 256, 0, s>>>(A, B, C, m, k, n);
}

// Row-major padded MLE of a matrix (matrix_to_mle on the padded matrix).
__global__ void rowmajor_mle_kernel(const uint32_t* __restrict__ M, uint32_t rows, uint32_t cols, size_t pc,
                                    size_t total, uint4* __restrict__ out) {
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
         idx += (size_t)gridDim.x * blockDim.x) {
        const size_t i = idx / pc, j = idx % pc;
        const uint32_t v = (i < rows && j < cols) ? red32(M[i * cols + j]) : 0u;
        out[idx] = make_uint4(v, 0, 0, 0);
    }
}

void launch_rowmajor_mle(const uint32_t* M, uint32_t rows, uint32_t cols, size_t pr, size_t pc, uint4* out,
                         cudaStream_t s) {
    const size_t total = pr * pc;
    size_t blocks = (total + 255) / 256;
    if (blocks > 8192) blocks = 8192;
    if (blocks == 0) blocks = 1;
    rowmajor_mle_kernel<<<(unsigned)blocks, 256, 0, s>>>(M, rows, cols, pc, total, out);
}

}  // namespace zk
