/*
 * CPU oracle for the GKR matmul-sumcheck path of stwo-ml (obelyzk engine).
 *
 * TEST INFRASTRUCTURE ONLY.  This library restates the reference's CPU prover
 * (Rust, engine/src/...) in plain C so that the CUDA product can be checked
 * bit for bit.  It is loaded by tests/, by __graft_entry__.smoke() and by the
 * cpu_baseline / --impl reference legs of bench.py, and by nothing else: the
 * product library never links or calls it.
 *
 * Parity pin: the oracle reproduces engine/tests/artifacts/sp3_matmul_only_proof.json
 * (calldata, weight commitment, weight opening calldata, io_commitment and the
 * final channel digest) and the Poseidon known answers of
 * engine/src/crypto/poseidon_channel.rs:1619-1637 and
 * stwo-gpu/crates/stwo/src/core/channel/poseidon252.rs:230-253.
 *
 * Representations:
 *   felt252 : 4 x uint64_t little-endian limbs of the canonical integer (< p_stark)
 *   QM31    : 4 x uint32_t [a, b, c, d] = (a + b i) + (c + d i) u, i^2 = -1, u^2 = 2 + i
 *   M31     : uint32_t in [0, 2^31 - 1)
 */
#ifndef ZKML_ORACLE_H
#define ZKML_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    uint64_t digest[4];
    uint32_t n_draws;
    uint32_t reserved;
    uint64_t hash_count;
} orc_channel;

/* felt252 / Poseidon (starknet-crypto 0.6.2 semantics) */
void orc_felt_mul(const uint64_t a[4], const uint64_t b[4], uint64_t out[4]);
void orc_hades(uint64_t state[12]);
void orc_poseidon_hash(const uint64_t a[4], const uint64_t b[4], uint64_t out[4]);
void orc_poseidon_hash_many(const uint64_t *in, size_t n, uint64_t out[4]);

/* PoseidonChannel (engine/src/crypto/poseidon_channel.rs:83-306) */
void orc_ch_init(orc_channel *ch);
void orc_ch_mix_u64(orc_channel *ch, uint64_t v);
void orc_ch_mix_felt(orc_channel *ch, const uint64_t v[4]);
void orc_ch_draw_felt(orc_channel *ch, uint64_t out[4]);
void orc_ch_draw_qm31(orc_channel *ch, uint32_t out[4]);
void orc_ch_mix_poly_coeffs(orc_channel *ch, const uint32_t c[12]);
void orc_ch_mix_poly_coeffs_deg3(orc_channel *ch, const uint32_t c[16]);
void orc_ch_mix_felts(orc_channel *ch, const uint32_t *qm31s, size_t n);
void orc_securefield_to_felt(const uint32_t v[4], uint64_t out[4]);

/* QM31 helpers exposed for tests */
void orc_qm31_mul(const uint32_t a[4], const uint32_t b[4], uint32_t out[4]);
void orc_qm31_inv(const uint32_t a[4], uint32_t out[4]);

/* MLE helpers (engine/src/components/matmul.rs:118-356) */
void orc_lagrange_basis(const uint32_t *challenges, size_t v, uint32_t *out /* 2^v QM31 */);
void orc_evaluate_mle(const uint32_t *evals, size_t n_vars, const uint32_t *point, uint32_t out[4]);
void orc_restrict_mle(const uint32_t *evals, size_t n_evals, const uint32_t *assign, size_t n_assign,
                      uint32_t *out /* n_evals >> n_assign */);

/* ZkmlOps::reduce_matmul_layer for SimdBackend (engine/src/backend.rs:110-197).
 * mode 0 = materialised pad + MLE + restrict_mle, exactly as backend.rs:127-134;
 * mode 1 = fused unpadded restriction (components/matmul.rs:470-566).
 * Both give identical results. Returns 0 on success. */
int orc_reduce_matmul_layer(const uint32_t *a, size_t a_rows, size_t a_cols,
                            const uint32_t *b, size_t b_rows, size_t b_cols,
                            const uint32_t *r_i, size_t n_ri, const uint32_t *r_j, size_t n_rj,
                            size_t pk, orc_channel *ch,
                            uint32_t *out_round_polys /* 12 per round */,
                            uint32_t *out_challenges /* 4 per round */,
                            uint32_t out_final_a[4], uint32_t out_final_b[4],
                            int mode, int threads);

/* reduce_matmul_layer_with_backend (engine/src/gkr/prover.rs:5959-6073): the transcript
 * wrapper.  claim_point has log2(pm)+log2(pn) QM31.  next_point receives
 * log2(pm)+log2(pk) QM31; next_value = final_a. */
int orc_reduce_matmul_gkr(const uint32_t *claim_point, size_t n_point, const uint32_t claim_value[4],
                          const uint32_t *a, size_t m, size_t k, const uint32_t *b, size_t n,
                          orc_channel *ch, uint32_t *out_round_polys, uint32_t out_final_a[4],
                          uint32_t out_final_b[4], uint32_t *next_point, int mode, int threads);

/* Poseidon Merkle (engine/src/crypto/poseidon_merkle.rs:91-280): root of the tree
 * whose leaves are securefield_to_felt(evals[i]), zero-padded to a power of two (min 2). */
void orc_merkle_root_qm31(const uint32_t *evals, size_t n, uint64_t out[4], int threads);
/* Auth path of leaf `index` (bottom-up siblings, log2(padded n) felts). */
void orc_merkle_path_qm31(const uint32_t *evals, size_t n, size_t index, uint64_t *out_siblings,
                          int threads);
int orc_merkle_verify(const uint64_t root[4], size_t index, const uint64_t leaf[4],
                      const uint64_t *siblings, size_t n_siblings);

/* MLE opening (engine/src/crypto/mle_opening.rs:1654-1916), serialized as
 * cairo_serde::serialize_mle_opening_proof (cairo_serde.rs:341-370). */
int orc_prove_mle_opening(const uint32_t *evals, size_t n_vars, const uint32_t *point,
                          orc_channel *ch, size_t n_queries, uint64_t commitment[4],
                          uint64_t *calldata, size_t cap, size_t *out_len, int threads);
int orc_verify_mle_opening(const uint64_t commitment[4], const uint64_t *calldata, size_t len,
                           const uint32_t *point, size_t n_vars, orc_channel *ch,
                           size_t n_queries, uint32_t out_final[4]);

/* Single-MatMul GKR proof: prove_gkr_with_cache (gkr/prover.rs:1500-2251) for the
 * circuit GraphBuilder::new((m,k)).linear(n) in Sequential weight-binding mode,
 * serialized with cairo_serde::serialize_gkr_model_proof (cairo_serde.rs:1307-1772).
 * policy may be NULL (no policy mix).  Writes calldata felts, the final channel
 * digest and the io commitment. */
int orc_prove_gkr_matmul(const uint32_t *input, size_t m, size_t k, const uint32_t *weight,
                         size_t n, const uint64_t *policy, size_t n_queries, uint64_t *calldata,
                         size_t cap, size_t *out_len, uint64_t digest[4], uint64_t io[4],
                         int threads);
/* Verifier replay of a proof produced by orc_prove_gkr_matmul
 * (gkr/verifier.rs:2675-2788 + mle_opening.rs:1918-2029).  Returns 1 if accepted. */
int orc_verify_gkr_matmul(const uint32_t *input, size_t m, size_t k, const uint32_t *weight,
                          size_t n, const uint64_t *policy, size_t n_queries,
                          const uint64_t *calldata, size_t len, uint64_t digest[4]);

void orc_io_commitment(const uint32_t *input, size_t in_rows, size_t in_cols,
                       const uint32_t *output, size_t out_rows, size_t out_cols, uint64_t out[4]);

/* Activation lookup tables (gadgets/lookup_table.rs:193-345, components/activation.rs:39-96).
 * tag: 1 ReLU, 2 GELU, 3 Sigmoid, 4 Softmax(exp), 5 SiLU.  Fills out[2^log_size]. */
int orc_activation_table(int tag, unsigned log_size, uint32_t *out);
unsigned orc_activation_table_log_size(int tag);

/* reduce_activation_layer, the LogUp path (gkr/prover.rs:6390-6600), serialized as the
 * LayerProof::Activation record of serialize_gkr_model_proof (cairo_serde.rs:1355-1387,
 * multiplicities included).  The activation input is rows x cols (padded to powers of two),
 * the output claim has log2(padded size) variables. */
int orc_reduce_activation_logup(const uint32_t *input, size_t rows, size_t cols, int tag,
                                const uint32_t *claim_point, size_t n_point,
                                const uint32_t claim_value[4], orc_channel *ch, uint64_t *calldata,
                                size_t cap, size_t *out_len, uint32_t out_input_eval[4]);
/* verify_activation_reduction (gkr/verifier.rs:3058-3287) + verify_multiplicity_sumcheck
 * (verifier.rs:5818-5842) on such a record.  Returns 1 if accepted. */
int orc_verify_activation_logup(const uint64_t *calldata, size_t len, const uint32_t *claim_point,
                                size_t n_point, const uint32_t claim_value[4], orc_channel *ch,
                                uint32_t out_input_eval[4]);

/* rsqrt table of the RMSNorm / LayerNorm lookups (components/layernorm.rs:116-136). */
int orc_rsqrt_table(unsigned log_size, uint32_t *out);
/* reduce_rmsnorm_layer_with_gamma (gkr/prover.rs:8424-8790): RMS^2 plain sumcheck, the
 * degree-3 eq-sumcheck output = input x scale, and the rsqrt LogUp, serialized as the
 * LayerProof::RMSNorm record (cairo_serde.rs:1648-1726).  gamma (gamma_len values) is the
 * optional affine scale (NULL for none); skip_rms_sq mirrors STWO_SKIP_RMS_SQ_PROOF. */
int orc_reduce_rmsnorm(const uint32_t *input, size_t rows, size_t cols, size_t dim,
                       const uint32_t *gamma, size_t gamma_len, int skip_rms_sq,
                       const uint32_t *claim_point, size_t n_point, const uint32_t claim_value[4],
                       orc_channel *ch, uint64_t *calldata, size_t cap, size_t *out_len,
                       uint32_t out_input_eval[4]);
/* verify_rmsnorm_reduction (gkr/verifier.rs:4693-5080) on such a record; the multiplicity
 * sumcheck, absent from the calldata, is replayed from the multiplicities.  Returns 1 if accepted. */
int orc_verify_rmsnorm(const uint64_t *calldata, size_t len, size_t dim, const uint32_t *claim_point,
                       size_t n_point, const uint32_t claim_value[4], orc_channel *ch,
                       uint32_t out_input_eval[4]);

/* A weight claim of the aggregated binding (crypto/aggregated_opening.rs:99-112): the
 * weight matrix (rows x cols M31, row major; its MLE is the column-major padded one,
 * local_n_vars = log2(padded rows * padded cols)), its index in the binding, the
 * evaluation point (local_n_vars QM31), the claimed value and the Merkle commitment. */
typedef struct {
    const uint32_t *weight;
    size_t rows, cols;
    size_t matrix_index;
    const uint32_t *eval_point;
    uint32_t expected_value[4];
    uint64_t commitment[4];
} orc_weight_claim;
/* commit_mle_root_only of matrix_to_mle_col_major_padded (gkr/prover.rs:1137-1139). */
void orc_weight_commitment(const uint32_t *weight, size_t rows, size_t cols, uint64_t out[4], int threads);
/* prove_aggregated_binding (aggregated_opening.rs:681-730), serialized by
 * serialize_aggregated_binding_proof (cairo_serde.rs:3884-3921).  Returns 4 if the
 * commitments do not match the weights. */
int orc_prove_aggregated_binding(const orc_weight_claim *claims, size_t m, orc_channel *ch, size_t n_queries,
                                 uint64_t *calldata, size_t cap, size_t *out_len, int threads);
/* verify_aggregated_binding (aggregated_opening.rs:1774-1905) on such a record (weights unused). */
int orc_verify_aggregated_binding(const orc_weight_claim *claims, size_t m, const uint64_t *calldata,
                                  size_t len, orc_channel *ch, size_t n_queries);

/* apply_activation_integer (components/integer_math.rs:212-263), act 0..4 = ReLU..SiLU. */
uint32_t orc_activation_integer(int act, uint32_t val);
/* PiecewiseLinearCoeffs::for_activation (components/activation.rs:269-316), tag 1..5. */
int orc_piecewise_coeffs(int tag, uint32_t slopes[16], uint32_t intercepts[16]);
/* reduce_activation_layer_piecewise (gkr/prover.rs:7006-7228), serialized as
 * LayerProof::Activation with the piecewise proof (cairo_serde.rs:1355-1387, 1249-1300).
 * out_point (num_vars QM31, may be NULL) receives the next claim's point. */
int orc_reduce_activation_piecewise(const uint32_t *input, size_t rows, size_t cols, int tag,
                                    const uint32_t *claim_point, size_t n_point,
                                    const uint32_t claim_value[4], orc_channel *ch, uint64_t *calldata,
                                    size_t cap, size_t *out_len, uint32_t out_input_eval[4],
                                    uint32_t *out_point);
/* verify_piecewise_activation_reduction (gkr/verifier.rs:3298-3480).  Returns 1 if accepted. */
int orc_verify_activation_piecewise(const uint64_t *calldata, size_t len, const uint32_t *claim_point,
                                    size_t n_point, const uint32_t claim_value[4], orc_channel *ch,
                                    uint32_t out_input_eval[4]);

/* reduce_layernorm_layer (gkr/prover.rs:7944-8354): the batched mean / variance plain
 * sumcheck, the eq-sumcheck of centered x rsqrt with the centered binding, the LogUp of
 * (variance, rsqrt) against the 2^16 rsqrt table and its multiplicity sumcheck; serialized as
 * LayerProof::LayerNorm (cairo_serde.rs:1389-1483).  The next claim is (point, input eval). */
int orc_reduce_layernorm(const uint32_t *input, size_t rows, size_t cols, size_t dim, const uint32_t *claim_point,
                         size_t n_point, const uint32_t claim_value[4], orc_channel *ch, uint64_t *calldata,
                         size_t cap, size_t *out_len, uint32_t out_input_eval[4]);

/* One layer of a GKR circuit (LayeredCircuit::from_graph, gkr/circuit.rs:140-225, for the
 * GraphBuilder ops linear / activation(ReLU) / rms_norm / add_from / mul_from):
 * type 0 = Linear (weight: rows = the layer's input width, n columns, row major), 1 = ReLU,
 * 2 = RMSNorm over the full width, 3 = Add, 4 = Mul (element-wise, M31), 5 = LayerNorm over
 * the full width.
 * src: the layer whose output is this layer's input (for Add / Mul the rhs operand);
 * ORC_CHAIN_PREV = the previous layer (the model input for layer 0), -1 = the model input.
 * lhs: Add / Mul only, the layer whose output is the lhs operand (the saved fork). */
#define ORC_CHAIN_PREV (-2)
typedef struct {
    int type;
    const uint32_t *weight;
    size_t n;
    long long src;
    long long lhs;
} orc_chain_layer;
/* prove_gkr_with_cache (gkr/prover.rs:1500-2251) for such a circuit on an m x k0 input:
 * the walk from the output with DAG Add / Mul layers (prover.rs:1424-1463, 1705-1760), the
 * deferred MatMul proofs of their skip branches (prover.rs:1918-2047), Sequential weight
 * binding (deferred openings first, then the walk's, all on the main channel).  Output:
 *   flags bit 1 clear: serialize_gkr_model_proof (cairo_serde.rs:1307-1772), which carries
 *     neither the deferred proofs nor their openings;
 *   flags bit 1 set: the verify_model_gkr calldata (starknet.rs:3143-3345, layout V1) from
 *     proof_data on: proof_data (serialize_gkr_proof_data_only, cairo_serde.rs:1816-2277,
 *     deferred proofs included), weight commitments (walk, then deferred), opening proofs.
 * flags bit 0: the earlier Activation record layout without the multiplicity-sumcheck and
 * piecewise flags (the layout of engine/tests/artifacts/sp3_mlp_proof.json).
 * flags bit 2: Activation layers (type 6, tag in .n: 2 GELU, 3 Sigmoid, 4 Softmax, 5 SiLU)
 * take the LogUp reduction (STWO_PIECEWISE_ACTIVATION=0); clear: the piecewise reduction
 * (the reference's default), gkr/prover.rs:1765-1790.  At most 1024 layers.
 * Writes the final digest and the io commitment.  Returns 4 for a deferred branch that is
 * not a Linear layer (the reference's "deferred proof not yet supported"). */
int orc_prove_gkr_chain(const uint32_t *input, size_t m, size_t k0, const orc_chain_layer *layers, size_t n_layers,
                        const uint64_t *policy, size_t n_queries, int flags, uint64_t *calldata, size_t cap,
                        size_t *out_len, uint64_t digest[4], uint64_t io[4], int threads);

/* verify_gkr (gkr/verifier.rs) on a chain proof of Linear, Activation (GELU / Sigmoid / Softmax /
 * SiLU; flags bit 2 as for orc_prove_gkr_chain) and RMSNorm layers, each fed by the previous
 * one: the output recomputed from the input and weights, every layer record replayed with its
 * verifier, the input claim, the weight commitments and Sequential openings, the io commitment.
 * Writes the verifier channel's final digest.  Returns 1 if accepted. */
int orc_verify_gkr_chain(const uint32_t *input, size_t m, size_t k0, const orc_chain_layer *layers, size_t n_layers,
                         const uint64_t *policy, size_t n_queries, int flags, const uint64_t *calldata, size_t len,
                         uint64_t digest[4], int threads);

/* reduce_activation_layer_algebraic (gkr/prover.rs:6700-6890), the ReLU proof, serialized as
 * LayerProof::Activation with the activation product proof (cairo_serde.rs:1355-1387,
 * 1190-1235).  out_point receives the next claim's point (the sumcheck challenges). */
int orc_reduce_activation_relu(const uint32_t *input, size_t rows, size_t cols, const uint32_t *claim_point,
                               size_t n_point, const uint32_t claim_value[4], orc_channel *ch, uint64_t *calldata,
                               size_t cap, size_t *out_len, uint32_t out_input_eval[4], uint32_t *out_point);

/* M31 matmul C = A.B mod p (components/matmul.rs:572-627) */
void orc_matmul_m31(const uint32_t *a, size_t m, size_t k, const uint32_t *b, size_t n,
                    uint32_t *c, int threads);

#ifdef __cplusplus
}
#endif
#endif
