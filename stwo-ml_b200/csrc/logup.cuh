// Host launchers for the LogUp activation kernels (logup_kernels.cu).  Every
// reducing launcher leaves its result words in rs.out (device) and, when
// rs.sig is set, publishes them to mapped host memory with sequence rs.seq.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.cuh"
#include "qm31.cuh"

namespace zk {

typedef RoundScratch ReduceScratch;  // partials must hold max_blocks * 16 words

// Padded row-major input -> x (M31), masked input, table output, multiplicity histogram.
void launch_logup_prepare(const uint32_t* input, uint32_t rows, uint32_t cols, size_t pc, size_t n, uint32_t mask,
                          const uint32_t* table, uint32_t* x_out, uint32_t* m_in, uint32_t* m_out, uint32_t* mult,
                          uint32_t* err, int max_blocks, cudaStream_t s);
// d, w = 1/d and sum w (4 words).
void launch_logup_dw(const uint32_t* m_in, const uint32_t* m_out, size_t n, qm31 gamma, qm31 beta, uint4* d,
                     uint4* w, const ReduceScratch& rs, cudaStream_t s);
// sum over table entries with nonzero multiplicity (4 words).
void launch_logup_table_sum(const uint32_t* mult, const uint32_t* table, size_t tsize, qm31 gamma, qm31 beta,
                            const ReduceScratch& rs, cudaStream_t s);
// sum eq * x0 (and eq * x1 if x1) (4 or 8 words).
void launch_eq_dot(const uint4* eq, const uint32_t* x0, const uint32_t* x1, size_t n, const ReduceScratch& rs,
                   cudaStream_t s);
// sum eq * xs[v] for nv (1..4) vectors (4 * nv words).
void launch_eq_dot(const uint4* eq, const uint32_t* const* xs, int nv, size_t n, const ReduceScratch& rs,
                   cudaStream_t s);
// Degree-3 round over (eq, w, d) of length len (after the optional fold), 16 words.
void launch_logup_round(uint4* E, uint4* W, uint4* D, size_t len, bool fold, qm31 alpha, const ReduceScratch& rs,
                        cudaStream_t s);
// Last fold of length-2 vectors: w then d (8 words).
void launch_logup_final(const uint4* E, const uint4* W, const uint4* D, qm31 alpha, const ReduceScratch& rs,
                        cudaStream_t s);
// Degree-1 multiplicity rounds: len is the current length before the optional fold.
void launch_mult_round(const uint32_t* src32, uint4* V, size_t len, bool first, bool fold, qm31 alpha,
                       const ReduceScratch& rs, cudaStream_t s);
void launch_mult_final(const uint32_t* src32, const uint4* V, qm31 alpha, const ReduceScratch& rs, cudaStream_t s);

// RMSNorm (rmsnorm_kernels.cu).  Per padded row: rms^2 = (sum of squares of the
// first n_active columns) / n_active masked to the table, its rsqrt, the
// multiplicity histogram (pc per row) and row_rms[row]; per element: x (M31),
// m_in = rms^2, m_out = rsqrt, W = x and D = scale (QM31), out = the RMSNorm output.
void launch_rmsnorm_prepare(const uint32_t* input, uint32_t rows, uint32_t cols, uint32_t pr, uint32_t pc,
                            uint32_t n_active, uint32_t inv_n, const uint32_t* gamma, uint32_t gamma_len,
                            const uint32_t* table, uint32_t mask, uint32_t* x_out, uint32_t* m_in, uint32_t* m_out,
                            uint32_t* outv, uint4* W, uint4* D, uint32_t* row_rms, uint32_t* mult, uint32_t* err,
                            int max_blocks, cudaStream_t s);
// Plain sumcheck round of sum_x v(x)^2: s(0), s(1), s(2) (12 words).  len is the
// current length before the optional fold; the first fold reads the M31 vector src32.
void launch_sq_round(const uint32_t* src32, uint4* V, size_t len, bool first, bool fold, qm31 alpha,
                     const ReduceScratch& rs, cudaStream_t s);

// LayerNorm (layernorm_kernels.cu).  Per padded row: mean, variance masked to the table,
// rsqrt, the multiplicity histogram (pc per row), row_mean / row_var; per element: x,
// centered, mean, variance, rsqrt (M31) and the output centered * rsqrt.
void launch_layernorm_prepare(const uint32_t* input, uint32_t rows, uint32_t cols, uint32_t pr, uint32_t pc,
                              uint32_t n_active, uint32_t inv_n, const uint32_t* table, uint32_t mask,
                              uint32_t* x_out, uint32_t* cen, uint32_t* mean_v, uint32_t* var_v, uint32_t* rs_v,
                              uint32_t* outv, uint32_t* row_mean, uint32_t* row_var, uint32_t* mult, uint32_t* err,
                              int max_blocks, cudaStream_t s);
// Batched mean / variance round: s(0..2) of sum eta0 in + eta1 c^2 (12 words); len is the
// current length before the optional fold of the input, centered and mean vectors.
void launch_mv_round(const uint32_t* x32, const uint32_t* c32, const uint32_t* m32, uint4* IN, uint4* C, uint4* M,
                     size_t len, bool first, bool fold, qm31 alpha, qm31 eta0, qm31 eta1, const ReduceScratch& rs,
                     cudaStream_t s);
// Last fold of the length-2 input and mean vectors (M31 sources when non-null): 8 words.
void launch_mv_final(const uint32_t* x32, const uint32_t* m32, const uint4* IN, const uint4* M, qm31 alpha,
                     const ReduceScratch& rs, cudaStream_t s);
void launch_lift2(const uint32_t* a, const uint32_t* b, size_t n, uint4* W, uint4* D, cudaStream_t s);
void launch_layernorm_forward(const uint32_t* x, uint32_t rows, uint32_t cols, uint32_t inv_n, const uint32_t* table,
                              uint32_t* y, cudaStream_t s);

}  // namespace zk
