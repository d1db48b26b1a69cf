// Host launchers for gkr_kernels.cu (single-layer GKR proof helpers).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace zk {

// out[j * pk + i] = (B[i][j], 0, 0, 0) for i < k, j < n; zero elsewhere (pk x pn total).
void launch_colmajor_mle(const uint32_t* B, uint32_t k, uint32_t n, size_t pk, size_t pn, uint4* out,
                         cudaStream_t s);
// out[i * pc + j] = (M[i][j], 0, 0, 0), zero padded to pr x pc.
void launch_rowmajor_mle(const uint32_t* M, uint32_t rows, uint32_t cols, size_t pr, size_t pc, uint4* out,
                         cudaStream_t s);
// C = A . B over M31 (row-major).
void launch_m31_gemm(const uint32_t* A, const uint32_t* B, uint32_t* C, uint32_t m, uint32_t k, uint32_t n,
                     cudaStream_t s);

}  // namespace zk
