// MLE opening on the device (opening_api.cu), shared by the entry points that open an MLE.
#pragma once
#include <cstdint>

#include "calldata.hpp"
#include "context.hpp"

namespace zk {

// Proves the opening of the MLE `evals` (device, 2^n_vars QM31) at `point`
// (prove_mle_opening_with_commitment, crypto/mle_opening.rs:1654-1916), appending the
// serialized MleOpeningProof to `out`; writes the commitment (canonical limbs) and,
// if final_out is set, the final folded value.  Advances `chs`.  With a peer mesh (not null,
// two or more ranks) the Merkle hashing is split across the ranks, which must all make the
// same call; the proof is the same on every rank and equal to the one-GPU proof.
struct MeshState;
int prove_opening_dev(::zkml_ctx* ctx, const uint4* evals, unsigned n_vars, const qm31* point, zkml_channel* chs,
                      size_t n_queries_cfg, uint64_t commitment[4], FeltOut& out, uint32_t final_out[4],
                      MeshState* mesh = nullptr);

}  // namespace zk
