// The algebraic ReLU reduction on the device (relu_api.cu), shared with the GKR chain driver.
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

}  // namespace zk
