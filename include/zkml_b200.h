/*
 * zkml_b200.h -- C ABI of the B200-native GKR matmul-sumcheck prover.
 *
 * This is the drop-in boundary for the stwo-ml engine's `ZkmlOps` backend trait
 * (engine/src/backend.rs:85-107) and the GKR layer-prover entry points that sit
 * on it.  Plain pointers and sizes only: no CUDA or torch types cross it.
 *
 * Conventions
 *   M31     uint32_t, canonical value in [0, 2^31 - 1); values >= 2^31 are
 *           rejected with ZKML_ERR_INVALID_ARG (detected on the GPU).
 *   QM31    4 x uint32_t [a, b, c, d] = (a + b i) + (c + d i) u  (i^2 = -1,
 *           u^2 = 2 + i), the SecureField AoS layout of
 *           engine/src/gpu_sumcheck.rs:3614-3630.
 *   felt252 4 x uint64_t little-endian limbs of the canonical integer < p_stark.
 *   Matrices are row-major and unpadded, like M31Matrix
 *           (engine/src/components/matmul.rs:85-116); padding to powers of two
 *           is logical.
 *   Matrix/MLE input pointers may be host memory (pageable or pinned; copied to
 *   the device inside the call) or device memory of the context's GPU (used in
 *   place, never modified).  All outputs are host pointers.
 *   Every function returns 0 (ZKML_OK) or a zkml_status; zkml_last_error()
 *   gives the message for the calling thread.  There is no CPU fallback: a
 *   missing or failing GPU is an error.
 *   A context drives one GPU from one host thread at a time.
 */
#ifndef ZKML_B200_H
#define ZKML_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ZKML_ABI_VERSION 1

typedef enum {
    ZKML_OK = 0,
    ZKML_ERR_INVALID_ARG = 1,
    ZKML_ERR_OOM = 2,
    ZKML_ERR_CUDA = 3,
    ZKML_ERR_NCCL = 4,
    ZKML_ERR_TIMEOUT = 5,
    ZKML_ERR_UNSUPPORTED = 6,
    ZKML_ERR_VERIFY = 7
} zkml_status;

/* Lossless PoseidonChannel state (engine/src/crypto/poseidon_channel.rs:83-88).
 * Unlike the reference's to_gpu_state/from_gpu_state pair
 * (poseidon_channel.rs:109-138) it keeps n_draws. */
typedef struct zkml_channel {
    uint64_t digest[4];
    uint32_t n_draws;
    uint32_t reserved;
    uint64_t hash_count;
} zkml_channel;

typedef struct zkml_ctx zkml_ctx;

int zkml_abi_version(void);
const char *zkml_last_error(void);

/* GpuSumcheckExecutor::cached (engine/src/gpu_sumcheck.rs:1365-1385): one
 * context per device, owning its stream and reusable device scratch. */
int zkml_ctx_create(int device, zkml_ctx **out);
int zkml_ctx_destroy(zkml_ctx *ctx);
int zkml_ctx_device(const zkml_ctx *ctx);
/* Kernel launches of this context so far (instrumentation for benchmarks). */
uint64_t zkml_ctx_kernel_launches(const zkml_ctx *ctx);
/* Host -> device bytes of the input-matrix uploads of this context so far (instrumentation for
 * benchmarks).  B of zkml_reduce_matmul_layer / _gkr in host memory with at least 2^22 words
 * (ZKML_PACK_MIN) crosses PCIe in chunks of 2^18 words packed by host threads into one byte per
 * word when every word of the chunk is the M31 image of a signed byte (x >= 0 ? x : p + x, the
 * reference's int8 quantisation); other chunks are copied as they are.  The device receives the
 * same field elements either way.  ZKML_PACK_H2D=0 turns the packing off. */
uint64_t zkml_ctx_h2d_bytes(const zkml_ctx *ctx);
/* Per-kernel device timing with CUDA events (off by default).  `enable` is 0
 * (off), -1 (every class) or a bit mask of classes in the order listed below
 * (bit 0 = "restrict_cols").  Each launch of a timed class is bracketed by events on the
 * context's stream; zkml_ctx_kernel_time returns the accumulated milliseconds
 * and launch count.  Kernel classes: "restrict_cols", "restrict_rows",
 * "sumcheck_round", "merkle"; and two host-side phases timed by wall clock:
 * "host_sync" (waiting for round results) and "host_channel" (Fiat-Shamir). */
int zkml_ctx_enable_timing(zkml_ctx *ctx, int enable);
int zkml_ctx_kernel_time(zkml_ctx *ctx, const char *kernel, double *out_ms, uint64_t *out_launches);
/* Replace the context's stream with a caller-owned cudaStream_t (NULL = own stream). */
int zkml_ctx_set_stream(zkml_ctx *ctx, void *cuda_stream);

/* ---- Poseidon / Fiat-Shamir channel (host; poseidon_channel.rs:83-306) ----- */
void zkml_channel_init(zkml_channel *ch);                                       /* PoseidonChannel::new */
void zkml_channel_mix_u64(zkml_channel *ch, uint64_t v);                        /* mix_u64 */
void zkml_channel_mix_felt(zkml_channel *ch, const uint64_t v[4]);              /* mix_felt */
void zkml_channel_mix_qm31(zkml_channel *ch, const uint32_t v[4]);              /* gkr::prover mix_secure_field */
void zkml_channel_draw_felt252(zkml_channel *ch, uint64_t out[4]);              /* draw_felt252 */
void zkml_channel_draw_qm31(zkml_channel *ch, uint32_t out[4]);                 /* draw_qm31 */
void zkml_channel_mix_poly_coeffs(zkml_channel *ch, const uint32_t c[12]);      /* mix_poly_coeffs */
void zkml_channel_mix_poly_coeffs_deg3(zkml_channel *ch, const uint32_t c[16]); /* mix_poly_coeffs_deg3 */
void zkml_channel_mix_felts(zkml_channel *ch, const uint32_t *qm31s, size_t n); /* mix_felts */
/* starknet_crypto::{poseidon_permute_comp, poseidon_hash, poseidon_hash_many}
 * (engine/src/crypto/hades.rs:21-23). */
void zkml_hades_permutation(uint64_t state[12]);
void zkml_poseidon_hash(const uint64_t a[4], const uint64_t b[4], uint64_t out[4]);
void zkml_poseidon_hash_many(const uint64_t *in, size_t n, uint64_t out[4]);
/* securefield_to_felt (poseidon_channel.rs:60-69) */
void zkml_securefield_to_felt(const uint32_t v[4], uint64_t out[4]);

/* ---- ZkmlOps (engine/src/backend.rs:85-107) -------------------------------- */

/* ZkmlOps::reduce_matmul_layer (backend.rs:87-94; CPU impl 110-197, reference
 * GPU impl gpu_sumcheck.rs:2692-2873).  Restricts A's rows by r_i and B's
 * columns by r_j (A: a_rows x a_cols, B: b_rows x b_cols, a_cols == b_rows),
 * then runs log2(pk) degree-2 sumcheck rounds, advancing `ch` on the host.
 * n_ri == log2(next_pow2(a_rows)), n_rj == log2(next_pow2(b_cols)),
 * pk == next_pow2(a_cols).
 * Outputs: out_round_polys  log2(pk) x 3 QM31 (c0, c1, c2 per round)
 *          out_challenges   log2(pk) QM31
 *          out_final_a/b    the folded A and B values (MatMulReduction). */
int zkml_reduce_matmul_layer(zkml_ctx *ctx, const uint32_t *a, size_t a_rows, size_t a_cols,
                             const uint32_t *b, size_t b_rows, size_t b_cols,
                             const uint32_t *r_i, size_t n_ri, const uint32_t *r_j, size_t n_rj,
                             size_t pk, zkml_channel *ch, uint32_t *out_round_polys,
                             uint32_t *out_challenges, uint32_t out_final_a[4],
                             uint32_t out_final_b[4]);

/* ZkmlOps::evaluate_mle_at_point (backend.rs:97-100): MLE of 2^n_vars QM31. */
int zkml_evaluate_mle(zkml_ctx *ctx, const uint32_t *mle, size_t n_vars, const uint32_t *point,
                      uint32_t out[4]);

/* ZkmlOps::restrict_mle (backend.rs:103-106): fix the first n_assign variables
 * (most significant index bits) of an MLE of n_evals = 2^k QM31;
 * out receives n_evals >> n_assign QM31. */
int zkml_restrict_mle(zkml_ctx *ctx, const uint32_t *mle, size_t n_evals, const uint32_t *assign,
                      size_t n_assign, uint32_t *out);

/* ---- GKR layer prover entry points (engine/src/gkr/prover.rs) --------------- */

/* reduce_matmul_layer_with_backend (gkr/prover.rs:5959-6073): mixes the
 * unpadded (m, k, n) and the claimed value, runs zkml_reduce_matmul_layer with
 * r_i = claim_point[..log m], r_j = claim_point[log m..], then mixes
 * final_a and final_b.  out_next_point receives log2(pm) + log2(pk) QM31
 * (r_i || challenges); the next claim's value is final_a. */
int zkml_reduce_matmul_layer_gkr(zkml_ctx *ctx, const uint32_t *claim_point, size_t n_point,
                                 const uint32_t claim_value[4], const uint32_t *a, size_t m,
                                 size_t k, const uint32_t *b, size_t n, zkml_channel *ch,
                                 uint32_t *out_round_polys, uint32_t out_final_a[4],
                                 uint32_t out_final_b[4], uint32_t *out_next_point);

/* ---- Poseidon-252 Merkle commitment and MLE opening (engine/src/crypto) ----- */

/* commit_mle_root_only (crypto/mle_opening.rs:630-642): root of the Poseidon
 * Merkle tree whose leaves are securefield_to_felt(evals[i]), zero-padded to a
 * power of two (at least 2); internal node = poseidon_hash(left, right)
 * (crypto/poseidon_merkle.rs:91-130). */
int zkml_commit_mle_root(zkml_ctx *ctx, const uint32_t *evals, size_t n, uint64_t out_root[4]);

/* prove_mle_opening_with_commitment (crypto/mle_opening.rs:1654-1916) for an
 * MLE of 2^n_vars QM31 at `point` (n_vars QM31).  Mixes the commitment and the
 * intermediate roots into `ch`, draws min(n_queries, 2^(n_vars-1)) queries
 * (STWO_MLE_N_QUERIES, default 10) and writes the proof serialized as
 * cairo_serde::serialize_mle_opening_proof (cairo_serde.rs:341-369) into
 * out_calldata (cap felts; *out_len receives the felt count, also when the
 * buffer is too small, which returns ZKML_ERR_INVALID_ARG). */
int zkml_prove_mle_opening(zkml_ctx *ctx, const uint32_t *evals, size_t n_vars, const uint32_t *point,
                           zkml_channel *ch, size_t n_queries, uint64_t out_commitment[4],
                           uint64_t *out_calldata, size_t cap, size_t *out_len);

/* compute_io_commitment (engine/src/aggregation.rs:235-254). Host only. */
int zkml_io_commitment(const uint32_t *input, size_t in_rows, size_t in_cols, const uint32_t *output,
                       size_t out_rows, size_t out_cols, uint64_t out[4]);

/* prove_gkr (gkr/prover.rs:1500-2251) for the one-layer circuit
 * GraphBuilder::new((m, k)).linear(n) with Sequential weight binding, from a
 * fresh PoseidonChannel: seeding (depth, input shape, optional policy
 * commitment; pass NULL to skip it, as STWO_SKIP_POLICY_COMMITMENT does),
 * output claim, the MatMul reduction, the weight-MLE opening and the IO
 * commitment.  The proof is written as cairo_serde::serialize_gkr_model_proof
 * (cairo_serde.rs:1307-1772) into out_calldata; out_digest receives the final
 * channel digest and out_io the IO commitment. */
int zkml_prove_gkr_matmul(zkml_ctx *ctx, const uint32_t *input, size_t m, size_t k, const uint32_t *weight,
                          size_t n, const uint64_t *policy, size_t n_queries, uint64_t *out_calldata,
                          size_t cap, size_t *out_len, uint64_t out_digest[4], uint64_t out_io[4]);

/* ---- Column-block sharded matmul layer -----------------------------------------
 * The config-2/4 layer split by column blocks of B across ranks (one GPU each): rank g
 * restricts its block B[:, col_offset .. col_offset + n_block) with the weights
 * L_{col_offset + j}(r_j) of the full padded column space into 4 k canonical u64 words
 * (out_words, device memory of the context's GPU); the ranks add their words (an int64
 * SUM all-reduce, e.g. NCCL); every rank then runs the layer from the summed words
 * (zkml_reduce_matmul_layer_gkr_fb), whose outputs equal zkml_reduce_matmul_layer_gkr's
 * on the whole B.  col_offset must be a multiple of 64. */
int zkml_restrict_cols_block(zkml_ctx *ctx, const uint32_t *b_block, size_t k, size_t n_block, size_t col_offset,
                             const uint32_t *r_j, size_t n_rj, uint64_t *out_words);
int zkml_reduce_matmul_layer_gkr_fb(zkml_ctx *ctx, const uint32_t *claim_point, size_t n_point,
                                    const uint32_t claim_value[4], const uint32_t *a, size_t m, size_t k,
                                    const uint64_t *fb_words, size_t n, zkml_channel *ch, uint32_t *out_round_polys,
                                    uint32_t out_final_a[4], uint32_t out_final_b[4], uint32_t *out_next_point);

/* The same split layer with the partial-word exchange over peer memory (NVLink) instead
 * of a collective library.  Each rank (one process per GPU, distinct GPUs of one node)
 * creates an inbox for a given k and exports its CUDA IPC handle (64 bytes); after the
 * ranks have exchanged the handles, each opens the others'.  Per layer call, with an
 * epoch that starts at 1 and increases by one per call (epoch 0, a skipped or repeated
 * epoch, and a scatter before the previous call's gather return ZKML_ERR_INVALID_ARG;
 * both calls go on the context's stream, gather(e) before scatter(e + 1), which is what
 * makes the inbox's double buffer safe): zkml_restrict_cols_block_p2p restricts the block
 * and stores the canonical partial words straight into every rank's inbox, then publishes
 * the epoch there; zkml_reduce_matmul_layer_gkr_p2p waits (bounded: ZKML_ERR_TIMEOUT after
 * about two seconds) for every rank's words, adds them and runs the layer.  Two ranks
 * must not share a GPU (their kernels would wait on each other). */
int zkml_p2p_inbox_create(zkml_ctx *ctx, size_t k, int world, int rank, uint8_t out_handle[64]);
int zkml_p2p_open(zkml_ctx *ctx, const uint8_t *handles /* world x 64 bytes */, int world);
int zkml_p2p_close(zkml_ctx *ctx);
int zkml_restrict_cols_block_p2p(zkml_ctx *ctx, const uint32_t *b_block, size_t k, size_t n_block, size_t col_offset,
                                 const uint32_t *r_j, size_t n_rj, uint32_t epoch);
int zkml_reduce_matmul_layer_gkr_p2p(zkml_ctx *ctx, const uint32_t *claim_point, size_t n_point,
                                     const uint32_t claim_value[4], const uint32_t *a, size_t m, size_t k, size_t n,
                                     uint32_t epoch, zkml_channel *ch, uint32_t *out_round_polys,
                                     uint32_t out_final_a[4], uint32_t out_final_b[4], uint32_t *out_next_point);

/* ---- LogUp activation layer ------------------------------------------------- */

/* reduce_activation_layer, LogUp path (gkr/prover.rs:6390-6600; reference GPU
 * variant prover.rs:4594-4816): proves that every (masked input, table output)
 * pair of the rows x cols activation input (zero-padded to powers of two) lies
 * in the activation table of `tag` (1 ReLU, 2 GELU, 3 Sigmoid, 4 Softmax-exp,
 * 5 SiLU; components/activation.rs:39-71), with a degree-3 eq-sumcheck and the
 * multiplicity sumcheck (prover.rs:9449-9515).  claim_point has
 * log2(padded size) QM31; claim_value is the output claim.  Writes the
 * LayerProof::Activation record of serialize_gkr_model_proof
 * (cairo_serde.rs:1355-1387, multiplicities included) and the input
 * evaluation that becomes the next claim's value.  Returns ZKML_ERR_VERIFY if
 * the trace-side and table-side LogUp sums differ. */
/* PrecomputedTable::build of the activation `tag` (gadgets/lookup_table.rs:30-49,
 * 193-345): out[i] = f(i) for i < 2^table_log_size.  Host only; *out_len receives
 * the table size (also when cap is too small, which returns ZKML_ERR_INVALID_ARG). */
int zkml_activation_table(int tag, uint32_t *out, size_t cap, size_t *out_len);

int zkml_reduce_activation_logup(zkml_ctx *ctx, const uint32_t *input, size_t rows, size_t cols, int tag,
                                 const uint32_t *claim_point, size_t n_point, const uint32_t claim_value[4],
                                 zkml_channel *ch, uint64_t *out_calldata, size_t cap, size_t *out_len,
                                 uint32_t out_input_eval[4]);

/* reduce_rmsnorm_layer_with_gamma (gkr/prover.rs:8424-8790): the RMSNorm layer
 * output = input * rsqrt(rms^2) (* gamma) over the rows x cols input (zero-padded to
 * powers of two; rms^2 over the first min(dim, padded cols) columns of each row).
 * Proves sum_x input(x)^2 (plain sumcheck; left out when STWO_SKIP_RMS_SQ_PROOF is
 * set, as in the reference), output(r) = sum_x eq(r, x) input(x) scale(x)
 * (degree-3 eq-sumcheck) and that every (rms^2, rsqrt) pair lies in the 2^16-entry
 * rsqrt table (LogUp + multiplicity sumcheck).  gamma (gamma_len values, host or
 * device memory) is the optional learned per-column scale, NULL for none.  Writes
 * the LayerProof::RMSNorm record of serialize_gkr_model_proof
 * (cairo_serde.rs:1648-1726) and the input evaluation (the next claim's value). */
int zkml_reduce_rmsnorm(zkml_ctx *ctx, const uint32_t *input, size_t rows, size_t cols, size_t dim,
                        const uint32_t *gamma, size_t gamma_len, const uint32_t *claim_point, size_t n_point,
                        const uint32_t claim_value[4], zkml_channel *ch, uint64_t *out_calldata, size_t cap,
                        size_t *out_len, uint32_t out_input_eval[4]);

/* reduce_activation_layer_piecewise (gkr/prover.rs:7006-7228), the default proof of a
 * non-ReLU activation layer (STWO_PIECEWISE_ACTIVATION unset): the activation as 16
 * linear segments of the M31 domain (components/activation.rs:269-358), one degree-3
 * eq-sumcheck over the combined segment constraints with eta powers.  Writes the
 * LayerProof::Activation record with the piecewise proof (cairo_serde.rs:1355-1387,
 * 1249-1300), the input evaluation and, if out_point is set, the next claim's point
 * (log2(padded size) QM31: the sumcheck challenges). */
int zkml_reduce_activation_piecewise(zkml_ctx *ctx, const uint32_t *input, size_t rows, size_t cols, int tag,
                                     const uint32_t *claim_point, size_t n_point, const uint32_t claim_value[4],
                                     zkml_channel *ch, uint64_t *out_calldata, size_t cap, size_t *out_len,
                                     uint32_t out_input_eval[4], uint32_t *out_point);

/* reduce_activation_layer_algebraic (gkr/prover.rs:6700-6890), the proof of a ReLU layer:
 * product + indicator + 30-bit decomposition constraints in one degree-3 eq-sumcheck.
 * Writes the LayerProof::Activation record with the activation product proof
 * (cairo_serde.rs:1355-1387, 1190-1235), the input evaluation and, if out_point is set,
 * the next claim's point (the sumcheck challenges). */
int zkml_reduce_activation_relu(zkml_ctx *ctx, const uint32_t *input, size_t rows, size_t cols,
                                const uint32_t *claim_point, size_t n_point, const uint32_t claim_value[4],
                                zkml_channel *ch, uint64_t *out_calldata, size_t cap, size_t *out_len,
                                uint32_t out_input_eval[4], uint32_t *out_point);

/* reduce_layernorm_layer (gkr/prover.rs:7944-8354) on a rows x cols M31 input over its
 * first dim columns: the batched mean / variance plain sumcheck, the eq-sumcheck of
 * centered x rsqrt with the centered binding, the LogUp of (variance, rsqrt) against the
 * 2^16 rsqrt table and its multiplicity sumcheck, advancing ch; writes the
 * LayerProof::LayerNorm record (cairo_serde.rs:1389-1483).  The next claim is the claim
 * point with value out_input_eval. */
int zkml_reduce_layernorm(zkml_ctx *ctx, const uint32_t *input, size_t rows, size_t cols, size_t dim,
                          const uint32_t *claim_point, size_t n_point, const uint32_t claim_value[4],
                          zkml_channel *ch, uint64_t *out_calldata, size_t cap, size_t *out_len,
                          uint32_t out_input_eval[4]);

/* ---- GKR proof of a layered circuit (Linear / ReLU / Activation / RMSNorm / LayerNorm /
 *      Add / Mul) */

#define ZKML_LAYER_LINEAR 0
#define ZKML_LAYER_RELU 1
#define ZKML_LAYER_RMSNORM 2 /* RMSNorm over the full layer width, no affine scale */
#define ZKML_LAYER_ADD 3     /* element-wise lhs + rhs (GraphBuilder::add_from) */
#define ZKML_LAYER_MUL 4     /* element-wise lhs * rhs (GraphBuilder::mul_from) */
#define ZKML_LAYER_LAYERNORM 5 /* LayerNorm over the full layer width (GraphBuilder::layer_norm) */
/* GraphBuilder::activation(GELU / Sigmoid / Softmax / SiLU): zkml_chain_layer.n holds the type
 * tag (2 GELU, 3 Sigmoid, 4 Softmax, 5 SiLU); the forward pass applies ActivationType::as_fn
 * to the full M31 values (compiler/prove.rs:1893-1899) */
#define ZKML_LAYER_ACTIVATION 6
/* zkml_chain_layer.src: the previous layer's output (the model input for layer 0) */
#define ZKML_CHAIN_PREV (-2)
/* flags: the Activation record without the multiplicity-sumcheck and piecewise flags, the
 * layout of the reference's engine/tests/artifacts/sp3_mlp_proof.json */
#define ZKML_CHAIN_LEGACY_ACTIVATION_RECORD 1
/* flags: emit the verify_model_gkr calldata (starknet.rs:3143-3345, layout V1) from
 * proof_data on, instead of serialize_gkr_model_proof */
#define ZKML_CHAIN_V1_CALLDATA 2
/* flags: Activation layers take the LogUp reduction (gkr/prover.rs:6400-6600), as the
 * reference does under STWO_PIECEWISE_ACTIVATION=0; without it the piecewise-algebraic
 * reduction (prover.rs:7006-7228), the reference's default (prover.rs:1765-1790) */
#define ZKML_CHAIN_ACTIVATION_LOGUP 4
/* flags: split the weight openings' Merkle hashing across the ranks of the peer mesh open on
 * the context's device (zkml_mesh_create / zkml_mesh_open): every rank of the mesh makes the
 * same call with the same inputs and gets the same proof, equal to the one-GPU proof; each
 * hashes 1/world of every large tree (see zkml_prove_product_sharded_mesh for the mesh) */
#define ZKML_CHAIN_MESH 8

/* One layer of the circuit (LayeredCircuit::from_graph, gkr/circuit.rs:140-225); layer i's
 * index is its circuit layer index. */
typedef struct {
    int type;               /* ZKML_LAYER_* */
    const uint32_t *weight; /* Linear: (input width) x n, row major, host or device memory */
    size_t n;               /* Linear: output width */
    long long src;          /* the layer whose output feeds this one (Add / Mul: the rhs operand);
                               ZKML_CHAIN_PREV, -1 = the model input, or a lower layer index */
    long long lhs;          /* Add / Mul: the layer whose output is the lhs operand (the fork) */
} zkml_chain_layer;

/* prove_gkr_with_cache (gkr/prover.rs:1500-2251) for such a circuit on an m x k0 input, from
 * a fresh PoseidonChannel: the walk from the output layer (Add layers defer their skip branch,
 * prover.rs:1424-1463; Mul layers run the degree-3 eq-sumcheck of reduce_mul_layer,
 * prover.rs:6172-6280, and defer and skip theirs, prover.rs:1719-1760), the deferred MatMul
 * proofs (prover.rs:1918-2047), Sequential weight binding (one MLE opening per weight,
 * n_queries queries, deferred openings first, all on the main channel).  The forward pass runs
 * on the GPU.  Output: serialize_gkr_model_proof (cairo_serde.rs:1307-1772; it carries no
 * deferred proofs), or with ZKML_CHAIN_V1_CALLDATA the verify_model_gkr calldata from
 * proof_data on.  policy may be NULL (no policy mix).  Writes the final channel digest and the
 * io commitment.  A deferred branch that is not a Linear layer fails with
 * ZKML_ERR_INVALID_ARG, as the reference's prover does. */
int zkml_prove_gkr_chain(zkml_ctx *ctx, const uint32_t *input, size_t m, size_t k0, const zkml_chain_layer *layers,
                         size_t n_layers, const uint64_t *policy, size_t n_queries, int flags,
                         uint64_t *out_calldata, size_t cap, size_t *out_len, uint64_t out_digest[4],
                         uint64_t out_io[4]);

/* build_verify_model_gkr_calldata (starknet.rs:2837-2852, 3143-3345; layout V1, Sequential
 * weight binding) for the same circuit: model_id, raw_io_data (serialize_raw_io of the input
 * and the GPU forward pass's output), circuit depth, proof layer count, matmul dims in walk
 * order, dequantize bits (none), proof_data, weight commitments and opening proofs. */
int zkml_build_verify_model_gkr_calldata(zkml_ctx *ctx, const uint64_t model_id[4], const uint32_t *input, size_t m,
                                         size_t k0, const zkml_chain_layer *layers, size_t n_layers,
                                         const uint64_t *policy, size_t n_queries, int flags,
                                         uint64_t *out_calldata, size_t cap, size_t *out_len,
                                         uint64_t out_digest[4], uint64_t out_io[4]);

/* ---- Aggregated weight binding ------------------------------------------------ */

/* A weight claim of the GKR walk (AggregatedWeightClaim, crypto/aggregated_opening.rs:99-112).
 * The weight is rows x cols M31, row major, host or device memory; its MLE is the
 * column-major padded one (matrix_to_mle_col_major_padded) with
 * n = log2(padded rows * padded cols) variables; eval_point holds n QM31; commitment
 * is that MLE's Poseidon Merkle root (zkml_weight_commitment), canonical limbs. */
typedef struct {
    const uint32_t *weight;
    size_t rows, cols;
    size_t matrix_index;
    const uint32_t *eval_point;
    uint32_t expected_value[4];
    uint64_t commitment[4];
} zkml_weight_claim;

/* commit_mle_root_only(matrix_to_mle_col_major_padded(weight)) (gkr/prover.rs:1137-1139). */
int zkml_weight_commitment(zkml_ctx *ctx, const uint32_t *weight, size_t rows, size_t cols, uint64_t out_root[4]);

/* prove_aggregated_binding_streaming (crypto/aggregated_opening.rs:1647-1719): super-root
 * of the claims' commitments, beta weights, the mismatch sumcheck over
 * log2(next_pow2(n_claims)) + max n variables, the oracle value at the challenge point and
 * one MLE opening (n_queries queries) of the virtual MLE against the super-root.  Writes
 * serialize_aggregated_binding_proof (cairo_serde.rs:3884-3921).  Returns
 * ZKML_ERR_INVALID_ARG if a commitment does not match its weight. */
int zkml_prove_aggregated_binding(zkml_ctx *ctx, const zkml_weight_claim *claims, size_t n_claims,
                                  zkml_channel *ch, size_t n_queries, uint64_t *out_calldata, size_t cap,
                                  size_t *out_len);

/* ---- Forward pass --------------------------------------------------------------
 * C = A * B mod p for M31 matrices (m x k times k x n, row major): the forward
 * GEMM that produces a layer's output (gpu_matmul_m31_full,
 * engine/src/gpu_sumcheck.rs:3104-3196).  Exact, on the integer tensor pipe
 * (byte planes, u8 MMAs) when k % 4 == 0 and A is 16-byte aligned, else on CUDA
 * cores.  c may be host memory or device memory of the context's GPU. */
int zkml_matmul_m31(zkml_ctx *ctx, const uint32_t *a, size_t m, size_t k, const uint32_t *b, size_t n, uint32_t *c);

/* ---- Stepwise product sumcheck (multi-GPU building block) -------------------
 * The round loop of ZkmlOps::reduce_matmul_layer (backend.rs:141-178) one round
 * at a time, so that a caller can split one sumcheck across GPUs: rank g of G
 * loads the elements with index = g (mod G); local round sums of all ranks add
 * up to the global ones while the local length is >= 2 (fold partners stay on
 * one rank), and below a threshold the local vectors are exported, gathered
 * (global[j*G + g] = local_g[j]) and loaded on one GPU.  The Fiat-Shamir
 * channel stays with the caller. */
/* Load two M31 (u32) or QM31 (4 x u32) vectors of length n (power of two >= 2). */
int zkml_sumcheck_load_m31(zkml_ctx *ctx, const uint32_t *a, const uint32_t *b, size_t n);
int zkml_sumcheck_load_qm31(zkml_ctx *ctx, const uint32_t *a, const uint32_t *b, size_t n);
/* Current vector length (0 without a session). */
size_t zkml_sumcheck_length(const zkml_ctx *ctx);
/* If alpha != NULL, fold both vectors with it first (length halves); then write
 * (s0, s1, s2) = (sum a_lo b_lo, sum a_hi b_hi, sum (2a_hi - a_lo)(2b_hi - b_lo)). */
int zkml_sumcheck_round(zkml_ctx *ctx, const uint32_t *alpha, uint32_t out_sums[12]);
/* Copy the current (folded, QM31) vectors to a and b (host or device). */
int zkml_sumcheck_export(zkml_ctx *ctx, uint32_t *out_a, uint32_t *out_b);
/* Fold length-2 vectors with alpha into the final values. */
int zkml_sumcheck_finalize(zkml_ctx *ctx, const uint32_t alpha[4], uint32_t out_a[4], uint32_t out_b[4]);

/* ---- Sharded product sumcheck, native round loop ------------------------------
 * One degree-2 product sumcheck over M31 vectors of global length n split across
 * `world` ranks (one process and context per GPU): rank g holds the elements
 * whose index is g (mod world), in order.  Per round the ranks all-reduce the
 * 12 round words through `ex`, every rank runs the same host transcript (no
 * challenge broadcast), and once the local length is at most gather_local the
 * folded vectors are all-gathered, interleaved back to global order and the
 * remaining rounds run on every rank's GPU.  The proof (round polynomials,
 * challenges, final values) is identical on every rank and equal to
 * zkml_reduce_matmul_layer on the 1 x n and n x 1 matrices.  The round loop of
 * engine/src/backend.rs:141-178, split as the north star's multi-GPU plan asks. */
typedef struct zkml_exchange {
    void *user;
    /* element-wise sum of n u64 words over all ranks, in place */
    int (*allreduce_u64)(void *user, uint64_t *words, int n);
    /* every rank's `bytes` from `local` into out, rank-major */
    int (*allgather)(void *user, const void *local, void *out, size_t bytes);
    int world;
    int rank;
} zkml_exchange;

/* A zkml_exchange over a POSIX shared-memory segment for the ranks of one node
 * (rank 0 creates it under `name`).  job_nonce must be the same on every rank and
 * differ between jobs (rank 0 draws it and broadcasts it): a segment an earlier,
 * crashed job left under the same name carries another nonce and is never joined.
 * max_gather_bytes bounds one rank's allgather contribution.  All waits are
 * bounded (60 s -> ZKML_ERR_TIMEOUT). */
int zkml_shm_exchange_open(const char *name, int world, int rank, size_t max_gather_bytes, uint64_t job_nonce,
                           zkml_exchange *out);
int zkml_shm_exchange_close(zkml_exchange *ex);

/* The same sharded proof with the exchange on the GPUs' own data path: a peer-memory mesh
 * over NVLink / NVSwitch between the ranks of one node, one process per distinct GPU.
 * zkml_mesh_create allocates this rank's inbox (max_gather_bytes bounds one rank's share of
 * the gather: 32 x gather_local bytes for the folded vectors, 8 x n / world when the vectors
 * are too short to split) and returns its CUDA IPC handle; once the ranks have exchanged the
 * handles (e.g. an all-gather over their process group), zkml_mesh_open maps every peer's
 * inbox.  zkml_prove_product_sharded_mesh then runs the loop of zkml_prove_product_sharded
 * with each split round's 12 words added across the ranks inside the round kernel (peer
 * stores, a release flag per rank, a bounded acquire wait in the grid's last block) and the
 * folded vectors gathered by peer stores into every inbox, with no host step and no
 * collective library.  Every rank must make the same sequence of calls on its context's
 * stream.  A rank that does not arrive within about two seconds makes the others' calls
 * return ZKML_ERR_TIMEOUT with the GPU usable; the mesh must then be closed and re-created.
 * No TMA and no multicast touch peer memory. */
int zkml_mesh_create(zkml_ctx *ctx, int world, int rank, size_t max_gather_bytes, uint8_t out_handle[64]);
int zkml_mesh_open(zkml_ctx *ctx, const uint8_t *handles /* world x 64 bytes */, int world);
int zkml_mesh_close(zkml_ctx *ctx);
int zkml_prove_product_sharded_mesh(zkml_ctx *ctx, const uint32_t *a_local, const uint32_t *b_local, size_t n,
                                    size_t gather_local, zkml_channel *ch, uint32_t *out_round_polys,
                                    uint32_t *out_challenges, uint32_t out_final_a[4], uint32_t out_final_b[4],
                                    size_t *out_gathered_at);

/* a_local, b_local: this rank's n / world M31 elements (host or device).
 * out_round_polys: log2(n) x 12 words, out_challenges: log2(n) x 4 words;
 * *out_gathered_at: global length at which the vectors were gathered. */
int zkml_prove_product_sharded(zkml_ctx *ctx, const uint32_t *a_local, const uint32_t *b_local, size_t n,
                               size_t gather_local, const zkml_exchange *ex, zkml_channel *ch,
                               uint32_t *out_round_polys, uint32_t *out_challenges, uint32_t out_final_a[4],
                               uint32_t out_final_b[4], size_t *out_gathered_at);

/* Self-test of the bounded waits: queues one round kernel whose challenge is
 * never posted; *status_out = 1 when its wait ran out and it flagged the
 * timeout instead of hanging.  Takes a few seconds; no GPU fault is involved. */
int zkml_selftest_wait_timeout(zkml_ctx *ctx, uint32_t *status_out);

/* ---- Allocation-free restriction ------------------------------------------- */

/* No counterpart in the reference: an extra entry point for callers that
 * cannot allocate GPU memory (code running inside a memory pool it does not
 * own, allocator callbacks, embedders with a fixed memory budget).  It computes
 * the column restriction f[i] = sum_j B[i][j] * eq(r_j, j) of a rows x cols
 * row-major M31 matrix -- the f_b that zkml_reduce_matmul_layer starts from --
 * and allocates nothing: its scratch is one fixed-size array in the library's
 * device code (about 2.3 MiB, held on every GPU that loads the library until
 * the process exits).
 *   b, out   device memory of the current GPU; out receives out_len QM31
 *            (rows of them, zero-padded to out_len >= rows).
 *   r_j      host, log2(next_pow2(cols)) QM31 challenges (first = most
 *            significant column bit).
 *   stream   cudaStream_t to run on (NULL = default stream); the call
 *            synchronises that stream before returning.
 * Limits: rows <= ZKML_NOALLOC_MAX_ROWS, cols <= ZKML_NOALLOC_MAX_COLS; larger
 * sizes return ZKML_ERR_INVALID_ARG.  The first call on each device resolves
 * the array's device address.  All calls share the one array, so calls whose GPU work overlaps (other
 * threads, other streams) race and must be serialised by the caller. */
#define ZKML_NOALLOC_MAX_ROWS 65536
#define ZKML_NOALLOC_MAX_COLS (1 << 20)
int zkml_restrict_cols_noalloc(const uint32_t *b, size_t rows, size_t cols, const uint32_t *r_j, size_t n_rj,
                               uint32_t *out, size_t out_len, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* ZKML_B200_H */
