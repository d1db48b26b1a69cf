// Layer reductions on the device shared with the GKR chain driver: the algebraic ReLU
// (relu_api.cu) and the RMSNorm reduction (rmsnorm_api.cu).
#pragma once
#include "calldata.hpp"
#include "context.hpp"

namespace zk {

// reduce_activation_layer_algebraic (gkr/prover.rs:6700-6890) on the rows x cols input
// (host or device memory); appends the LayerProof::Activation record to `o` (without the
// multiplicity-sumcheck and piecewise flags when legacy_record) and writes the next claim
// (point: log2(padded size) QM31, value).
int relu_reduce_dev(::zkml_ctx* ctx, const uint32_t* input, size_t rows, size_t cols, const qm31* point,
                    const qm31& claim_value, zkml_channel* chs, Out& o, qm31* next_point, qm31* next_value,
                    bool legacy_record);

// reduce_rmsnorm_layer_with_gamma (gkr/prover.rs:8424-8790) on the rows x cols input;
// appends the LayerProof::RMSNorm record to `o` (rmsnorm_api.cu), as serialize_gkr_model_proof
// writes it or, with v1_record, as serialize_gkr_proof_data_only does (no multiplicities, the
// multiplicity sumcheck included).  The next claim keeps the point; its value is written to
// out_input_eval.
int rmsnorm_reduce_dev(::zkml_ctx* ctx, const uint32_t* input, size_t rows, size_t cols, size_t dim,
                       const uint32_t* gamma, size_t gamma_len, const uint32_t* claim_point, size_t n_point,
                       const uint32_t claim_value[4], zkml_channel* chs, Out& o, uint32_t out_input_eval[4],
                       bool v1_record = false);

// reduce_layernorm_layer (gkr/prover.rs:7944-8354) on the rows x cols input; appends the
// LayerProof::LayerNorm record to `o` (layernorm_api.cu); v1_record leaves out the LogUp
// multiplicities (serialize_gkr_proof_data_only).  The next claim keeps the point; its value
// is written to out_input_eval.
int layernorm_reduce_dev(::zkml_ctx* ctx, const uint32_t* input, size_t rows, size_t cols, size_t dim,
                         const uint32_t* claim_point, size_t n_point, const uint32_t claim_value[4],
                         zkml_channel* chs, Out& o, uint32_t out_input_eval[4], bool v1_record = false);

}  // namespace zk
