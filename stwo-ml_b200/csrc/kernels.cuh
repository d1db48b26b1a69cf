// Declarations of the sm_100a kernels of the matmul-sumcheck path and their
// host launchers (all launchers are asynchronous on the given stream).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "mesh.cuh"
#include "qm31.cuh"

namespace zk {

constexpr int MAX_EQ_VARS = 40;

struct EqChallenges {  // passed by value as a kernel parameter
    qm31 c[MAX_EQ_VARS];
    int v;
};

// ---- eq / Lagrange tables (components/matmul.rs:342-356) --------------------
// table[idx] = prod_l ((bit_{v-1-l}(idx)) ? c_l : 1 - c_l), first challenge on the MSB.
void launch_eq_table(const qm31* c, int v, uint4* table, size_t table_len, cudaStream_t s);

// ---- restriction W . eq(r) (components/matmul.rs:470-566) --------------------
// Column restriction of a row-major k x n M31 matrix: acc[i] += sum_j B[i][j] L_j,
// with L_j = lhi[j >> 6] * llo[j & 63] (llo zero-padded to 64 entries); acc is 4 x u64
// per row, zeroed by the caller.
// Tensor-pipe column restriction (see restrict_cols_tc_kernel); needs restrict_cols_tc_ok(B, n).
bool restrict_cols_tc_ok(const uint32_t* B, uint32_t n);
// The eq weights come straight from r_j (hi_vars high + lo_vars low challenges, lo_vars <= 6);
// hi_base is the first 64-column stripe of B within the full column range.
void launch_restrict_cols_tc(const uint32_t* B, uint32_t k, uint32_t n, const qm31* r_j, unsigned hi_vars,
                             unsigned lo_vars, uint32_t hi_base, unsigned long long* acc, uint32_t* err, int num_sms,
                             cudaStream_t s);
void launch_restrict_cols(const uint32_t* B, uint32_t k, uint32_t n, const uint4* lhi, const uint4* llo,
                          unsigned long long* acc, uint32_t* err, int num_sms, cudaStream_t s);
// Row restriction of a row-major m x k M31 matrix: acc[j] += sum_i A[i][j] L_i.
void launch_restrict_rows(const uint32_t* A, uint32_t m, uint32_t k, const uint4* L,
                          unsigned long long* acc, uint32_t* err, cudaStream_t s);
// f_a (pk entries, zero past k) from an m x k M31 matrix and the n_ri <= 8 row
// challenges in one launch, plus f_b[i] = acc_b[i] mod P (i < k_b, zero up to pk)
// when acc_b is set.  Returns nonzero (nothing launched) outside those bounds.
int launch_restrict_rows_fused(const uint32_t* A, uint32_t m, uint32_t k, const qm31* r_i, int n_ri,
                               const unsigned long long* acc_b, size_t k_b, uint4* fa, uint4* fb, size_t pk,
                               uint32_t* err, cudaStream_t s);
// out[i] = acc[i] mod P for i < n_rows, zero for n_rows <= i < out_len.
void launch_acc_finalize(const unsigned long long* acc, size_t n_rows, uint4* out, size_t out_len,
                         cudaStream_t s);
// Embed M31 values as QM31 (a, 0, 0, 0) with zero padding to out_len.
void launch_m31_to_qm31(const uint32_t* in, size_t n, uint4* out, size_t out_len, uint32_t* err,
                        cudaStream_t s);

// ---- sumcheck rounds (backend.rs:145-178) ------------------------------------
// All round launchers leave the 12 u32 (s0, s1, s2) QM31 sums of the *current*
// round in out12 (device), reduced across the grid in the same launch.
struct RoundScratch {
    uint32_t* partials;  // >= max_blocks * 12
    unsigned int* ticket;  // zero-initialised
    uint32_t* out;       // >= 16 u32
    int max_blocks;
    // Optional host signal: device alias of mapped pinned host memory.  When
    // set, the grid's last block also writes the result words to sig[1..] and
    // then publishes `seq` in sig[0] (system-scope release), so the host can
    // spin on sig[0] instead of synchronising the stream.
    uint32_t* sig;
    uint32_t seq;
    // Optional peer mesh (launch_round_m31, launch_fold_round_m31 / _qm31, launch_round_qm31):
    // the last block adds every rank's 12 words before it stores or publishes them.
    MeshArg mesh{nullptr, 0};
    // Look-ahead rounds: LA_WORDS zero-initialised 64-bit accumulators (left zero
    // by every launch_round_lookahead kernel).
    unsigned long long* la_acc = nullptr;
};
// Reduce n u32 words in place to [0, P) (the round kernels need canonical QM31 input).
void launch_canon_words(uint32_t* w, size_t n, cudaStream_t s);
// Reduce n u64 words in place to [0, P).
void launch_canon_u64(unsigned long long* w, size_t n, cudaStream_t s);
// Round sums over QM31 vectors of length len (no fold).
void launch_round_qm31(uint4* A, uint4* B, size_t len, const RoundScratch& rs, cudaStream_t s);
// Fold A, B in place with alpha (len -> len/2) and emit the next round's sums.
void launch_fold_round_qm31(uint4* A, uint4* B, size_t len, qm31 alpha, const RoundScratch& rs,
                            cudaStream_t s);
// Round sums over M31 vectors (base-field first round of a product sumcheck).
void launch_round_m31(const uint32_t* A, const uint32_t* B, size_t len, const RoundScratch& rs,
                      uint32_t* err, cudaStream_t s);
// Fold M31 vectors into QM31 outputs (len -> len/2) and emit the next round's sums.
void launch_fold_round_m31(const uint32_t* A, const uint32_t* B, size_t len, qm31 alpha, uint4* Ao,
                           uint4* Bo, const RoundScratch& rs, cudaStream_t s);
// Look-ahead round over QM31 vectors: optionally fold V_{r-1} (length 2L) with
// alpha into V_r (length L, in place), then publish 40 words (L >= 4: the sums
// [Q0 Q1 Q2 Q3 T D0 D1 U W UW] from which the host forms round r's sums and round
// r+1's sums as quadratics in the next challenge) or 28 words (L = 2:
// [P0 P1 T A0 A1 B0 B1]).  partials must hold max_blocks * 16 words.
// With wait_msg != null the kernel may be queued before the challenge exists:
// thread 0 of every block polls the 8-word slot wait_msg (mapped host memory)
// until word 0 equals wait_seq, then folds with words 1-4; a set word 5 (abort)
// or a poll that runs past its limit skips the arithmetic (the latter also sets
// *status), and the kernel still publishes so that the queue drains.  Only
// block 0 polls host memory; it forwards the slot to the other blocks through
// `mailbox` (6 words of device memory).  With err_word, the last round (L = 2)
// also publishes *err_word and *status as words 40-41.  pdl launches it as a
// programmatic dependent of the stream's previous kernel (resident early): only
// for a kernel that waits for a challenge the host posts after the previous
// kernel published, since the vectors are read after that challenge is seen.
void launch_round_lookahead(uint4* A, uint4* B, size_t L, bool fold, qm31 alpha, const RoundScratch& rs,
                            cudaStream_t s, const uint32_t* wait_msg = nullptr, uint32_t wait_seq = 0,
                            uint32_t* status = nullptr, uint32_t* mailbox = nullptr,
                            const uint32_t* err_word = nullptr, bool pdl = false);
// All remaining look-ahead rounds in one single-block launch (vectors in shared
// memory).  The L0 input elements (L0 <= 2 * LA_TAIL_MAX) are folded first when
// fold0 is set, with alpha0 or, if wait0, with the challenge posted to round
// 0's slot.  Round j publishes sequence seq_base + j and (j > 0, or j = 0 with
// wait0) waits for tag tag_base + j in the 8-word slot (tag_base + j) % slots
// of msg.  With err_word, the last round also publishes *err_word and *status
// as words 40-41.  pdl as for launch_round_lookahead (wait0 set).  Returns
// nonzero if the launch could not be configured.
constexpr size_t LA_TAIL_MAX = 2048;
// Word 6 of a posted challenge slot: tag ^ words 1-5 ^ LA_SLOT_MIX (the kernels read
// the slot in one PCIe round trip and retry a read that straddles a post).
constexpr uint32_t LA_SLOT_MIX = 0x9E3779B9u;
void la_stamps_enable(bool on);
void la_stamps_print(uint32_t lo, uint32_t hi);
int launch_lookahead_tail(const uint4* A, const uint4* B, size_t L0, bool fold0, bool wait0, qm31 alpha0,
                          uint32_t* sig, uint32_t seq_base, const uint32_t* msg, uint32_t tag_base, int slots,
                          uint32_t* status, cudaStream_t s, const uint32_t* err_word = nullptr,
                          bool pdl = false);
// Rank-major gathered shards [g][A: len | B: len] -> fa, fb in global order
// (global[j * G + g] = local_g[j]).
void launch_interleave_gather(const uint4* in, size_t len, size_t G, uint4* fa, uint4* fb, cudaStream_t s);
// Final fold of length-2 vectors to one value each: out[0..4) = a, out[4..8) = b.
// src_m31 selects M31 inputs (A32, B32) instead of QM31 (A, B).
void launch_final_fold(const uint4* A, const uint4* B, const uint32_t* A32, const uint32_t* B32,
                       size_t len, qm31 alpha, uint32_t* out, uint32_t* sig, uint32_t seq, cudaStream_t s);

// ---- persistent round loop ----------------------------------------------------
// One cooperative launch runs every round of a degree-2 sumcheck: per round the
// grid computes (s0, s1, s2) (with the previous fold fused in), block 0 publishes
// them to the host (sig, sequence seq_base + r), waits for the host's challenge
// in hostmsg (sequence word, then 4 challenge words, then an abort word), and a
// grid barrier hands the challenge to all blocks.  After the last round block 0
// publishes the final (a, b) with sequence seq_base + log_k.  All waits are
// bounded; on a timeout the kernel sets status and exits.
struct PersistArgs {
    uint4* A;             // QM31 vectors (or fold targets in M31 mode)
    uint4* B;
    const uint32_t* A32;  // M31 inputs (M31 mode), else null
    const uint32_t* B32;
    size_t len;
    int log_k;
    uint32_t* partials;     // >= gridDim * 12 words
    unsigned int* bar;      // [0] arrival count, [1] generation (zeroed)
    uint4* alpha_dev;       // challenge broadcast slot
    uint32_t* status;       // bit 0: barrier timeout, bit 1: host timeout / abort
    uint32_t* sig;          // mapped host words written by the GPU
    const uint32_t* hostmsg;  // mapped host words written by the host
    uint32_t seq_base;
};
// Returns the grid size it launched (0 if a cooperative launch is not possible).
int launch_sumcheck_persistent(const PersistArgs& a, int num_sms, cudaStream_t s, cudaError_t* err);

// ---- generic MLE ops (ZkmlOps::evaluate_mle_at_point / restrict_mle) ----------
// dst[i] = src[i] + r (src[i + h] - src[i]) for i < h (dst may alias src).
void launch_mle_fold(const uint4* src, uint4* dst, size_t h, qm31 r, cudaStream_t s);

}  // namespace zk
