// Internal definition of zkml_ctx: one GPU, one stream, reusable device scratch.
#pragma once
#include <cuda_runtime.h>

#include <string>
#include <vector>

#include "../../include/zkml_b200.h"
#include "kernels.cuh"

namespace zk {

// Records a status + message for zkml_last_error() and returns the status.
int set_error(int status, const std::string& msg);
int cuda_error(cudaError_t e, const char* what);

#define ZK_CUDA(call)                                              \
    do {                                                           \
        cudaError_t _e = (call);                                   \
        if (_e != cudaSuccess) return ::zk::cuda_error(_e, #call); \
    } while (0)

// A growable device allocation.
struct DevBuf {
    void* ptr = nullptr;
    size_t bytes = 0;
    int ensure(size_t need);  // returns 0 or a zkml status
    void release();
    template <class T>
    T* as() const {
        return static_cast<T*>(ptr);
    }
};

// Called once with the claimed sum of the reduction (p(0) + p(1) of round 0,
// or f_a * f_b when there are no rounds) before any round touches the channel.
// `overlap`, if set, runs on the host right after the first GPU launches
// (before the host waits for the first round), for transcript work that does
// not depend on GPU results.
// `adjust`, if set, edits round r's sums (s(0), s(1), s(2), 12 words) before they are
// interpolated and mixed, and `challenge` receives round r's challenge: together they let a
// caller run a sumcheck of (sum A B) - (a host-known polynomial of degree <= 2 per round).
struct ClaimHook {
    void (*fn)(void* arg, const qm31& claimed_sum);
    void* arg;
    void (*overlap)(void* arg) = nullptr;
    void (*adjust)(void* arg, unsigned r, uint32_t s12[12]) = nullptr;
    void (*challenge)(void* arg, unsigned r, const qm31& alpha) = nullptr;
};

int reduce_matmul_internal(::zkml_ctx* ctx, const uint32_t* a, size_t a_rows, size_t a_cols, const uint32_t* b,
                           size_t b_rows, size_t b_cols, const uint32_t* r_i, size_t n_ri, const uint32_t* r_j,
                           size_t n_rj, size_t pk, zkml_channel* ch, uint32_t* out_round_polys,
                           uint32_t* out_challenges, uint32_t out_final_a[4], uint32_t out_final_b[4],
                           const ClaimHook* hook, const uint64_t* fb_words = nullptr);

// The sumcheck round loop (matmul_api.cu): M31 inputs (A32, B32) or QM31 (A, B)
// of length len; writes log2(len) round polynomials and challenges.
int run_sumcheck(::zkml_ctx* ctx, uint4* A, uint4* B, const uint32_t* A32, const uint32_t* B32, size_t len,
                 zkml_channel* chs, uint32_t* out_rp, uint32_t* out_ch, uint32_t* fa_out, uint32_t* fb_out,
                 const ClaimHook* hook);

// Shared host helpers (matmul_api.cu).
// device_view: `p` itself if it is device memory of the context's GPU, else a copy in `stage`.
int device_view(::zkml_ctx* ctx, const void* p, size_t bytes, DevBuf& stage, const void** out);
// device_view of an M31 matrix of `count` words: a large host matrix goes through
// upload_m31_packed (values that fit a signed byte cross PCIe as bytes; ZKML_PACK_H2D=0 turns it
// off, ZKML_PACK_MIN sets the size in words from which it is used, default 2^22).
int matrix_view(::zkml_ctx* ctx, const uint32_t* p, size_t count, DevBuf& stage, const void** out);
int upload_m31_packed(::zkml_ctx* ctx, const uint32_t* host, size_t count, DevBuf& dst, const void** out);
// Spin (bounded) until a kernel publishes `seq` in the mapped signal words; copy n words.
int wait_signal(::zkml_ctx* ctx, uint32_t seq, uint32_t* words, int n);
int read_err_flag(::zkml_ctx* ctx);
int check_err_flag(::zkml_ctx* ctx, const char* what);

enum KernelClass { KC_RESTRICT_COLS = 0, KC_RESTRICT_ROWS = 1, KC_ROUND = 2, KC_MERKLE = 3, KC_HOST_SYNC = 4,
                   KC_HOST_CHANNEL = 5 };

// Brackets one launch of a kernel class with events when timing is enabled.
struct KTimer {
    ::zkml_ctx* ctx;
    int cls;
    KTimer(::zkml_ctx* c, int k, bool enabled = true);  // enabled = false: record nothing
    ~KTimer();
};

}  // namespace zk

namespace zk {
// Device scratch of the LogUp activation and RMSNorm reductions, kept by the context (grown on demand).
struct LogupScratch {
    DevBuf x, m_in, m_out, mult, eq, d, w, mv;
    DevBuf outv, row_rms, pv, gam;  // RMSNorm: output, per-row rms^2, plain-sumcheck vector, affine scale
    DevBuf cen, meanv, row_var;     // LayerNorm: centered input, per-element mean, per-row variance
    void release() {
        DevBuf* all[] = {&x, &m_in, &m_out, &mult, &eq, &d, &w, &mv, &outv, &row_rms, &pv, &gam, &cen, &meanv, &row_var};
        for (DevBuf* b : all) b->release();
    }
};
// Device scratch of the Merkle commitment and the MLE opening (grown on demand).
struct OpeningScratch {
    DevBuf layers, trees, idx, gathered, qvals, nodes, cbuf, bmle;
    DevBuf adig;   // signed byte digits of the forward GEMM's left operand
    DevBuf gpart;  // the forward GEMM's per-K-split partial products
    void release() {
        DevBuf* all[] = {&layers, &trees, &idx, &gathered, &qvals, &nodes, &cbuf, &bmle, &adig, &gpart};
        for (DevBuf* b : all) b->release();
    }
};
}  // namespace zk

struct zkml_ctx {
    int device = 0;
    int num_sms = 148;
    cudaStream_t stream = nullptr;
    cudaStream_t own_stream = nullptr;
    // The row side of a restriction runs on side_stream under the column side
    // (fork / join events; off with ZKML_ROW_SIDE_STREAM=0 or while the row class is timed).
    cudaStream_t side_stream = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    bool row_side_stream = true;
    bool rows_fused = true;  // launch_restrict_rows_fused for A of at most 2^8 rows (ZKML_ROWS_FUSED=0: off; off while the row class is timed)
    // Queued look-ahead kernels that wait for a challenge launch as programmatic
    // dependents of the kernel before them (ZKML_LA_PDL=0: plain launches).
    bool la_pdl = true;
    uint64_t launches = 0;
    // scratch
    zk::DevBuf a_in, b_in;          // device copies of host inputs
    zk::DevBuf fa, fb;              // QM31 sumcheck vectors
    zk::DevBuf acc_a, acc_b;        // u64 restriction accumulators
    zk::DevBuf eq_a, eq_hi, eq_lo;  // eq tables
    zk::DevBuf partials;            // per-block round partials
    zk::DevBuf small;               // ticket + out words + error flag
    zk::DevBuf act_tables[6];       // activation lookup tables by type tag (device copies)
    zk::DevBuf rsqrt_table;         // RMSNorm rsqrt table (device copy)
    zk::LogupScratch lu;
    zk::OpeningScratch op;
    zk::DevBuf gather_dev;          // gathered shards of the sharded product sumcheck
    zk::DevBuf mesh_stage;          // this rank's contribution to a mesh gather
    uint8_t* h_stage = nullptr;     // pinned host staging for the sharded gather
    size_t h_stage_bytes = 0;
    // packed upload of host matrices (h2d_pack.cu)
    uint8_t* pack_host = nullptr;   // pinned byte staging
    size_t pack_host_bytes = 0;
    zk::DevBuf pack_dev;            // packed bytes on the device
    cudaEvent_t pack_event = nullptr;  // after the last upload's copies
    uint64_t h2d_bytes = 0;         // host -> device bytes of the matrix uploads
    // stepwise product-sumcheck session (zkml_sumcheck_*)
    zk::DevBuf sc_a, sc_b;          // staged M31 inputs
    const uint32_t* sc_a32 = nullptr;
    const uint32_t* sc_b32 = nullptr;
    size_t sc_len = 0;              // current vector length (0 = no session)
    bool sc_m31 = false;            // vectors are still the M31 inputs
    uint32_t* h_small = nullptr;    // pinned host mirror of `small`
    uint32_t* h_sig = nullptr;      // mapped pinned host words the round kernels publish to
    uint32_t* d_sig = nullptr;      // device alias of h_sig
    uint32_t sig_seq = 0;           // last sequence number handed to a kernel
    size_t lookahead_max = size_t(1) << 16;  // look-ahead rounds for vectors up to this length (ZKML_LOOKAHEAD_MAX)
    bool persistent = false;        // run sumcheck rounds in one cooperative launch (ZKML_PERSISTENT_ROUNDS=1)
    int max_round_blocks = 0;
    // optional per-kernel-class event timing
    bool timing = false;
    unsigned timing_mask = 0;  // bit i: time kernel class i
    struct KTime {
        double ms = 0;
        uint64_t launches = 0;
    };
    KTime ktime[6];  // restrict_cols, restrict_rows, sumcheck_round, merkle, host_sync, host_channel
    // Event pairs recorded but not yet read; read after the next stream sync so
    // timing never adds a host wait of its own.
    struct PendingEv {
        int cls;
        cudaEvent_t e0, e1;
    };
    std::vector<PendingEv> pending;
    std::vector<cudaEvent_t> ev_pool;

    unsigned int* ticket() const { return small.as<unsigned int>(); }
    uint32_t* out_words() const { return small.as<uint32_t>() + 16; }  // 32 words
    uint32_t* err_flag() const { return small.as<uint32_t>() + 48; }
    unsigned int* grid_bar() const { return small.as<unsigned int>() + 52; }       // 2 words
    uint4* alpha_slot() const { return reinterpret_cast<uint4*>(small.as<uint32_t>() + 56); }
    uint32_t* persist_status() const { return small.as<uint32_t>() + 60; }
    uint32_t* la_mailbox() const { return small.as<uint32_t>() + 4; }  // words 4-9
    uint32_t* la_status() const { return small.as<uint32_t>() + 61; }  // look-ahead wait timed out
    // 40 u64 look-ahead accumulators, words 64-143 (zero between kernels)
    unsigned long long* la_acc() const { return reinterpret_cast<unsigned long long*>(small.as<uint32_t>() + 64); }
    // challenge slots of the pre-queued look-ahead kernels: LA_SLOTS x 8 words
    // (sequence tag, 4 challenge words, abort) from word 256 of the mapped page
    static constexpr int LA_SLOTS = 32;
    uint32_t* h_la_msg() const { return h_sig + 256; }
    uint32_t* d_la_msg() const { return d_sig + 256; }
    uint32_t la_msg_seq = 0;
    bool restrict_tc = true;  // tensor-pipe column restriction when the layout allows (ZKML_RESTRICT_TC=0: off)
    bool la_queue = true;  // queue look-ahead kernels up front (ZKML_LA_QUEUE=0 turns it off)
    bool la_tail = true;  // single-block tail for the last look-ahead rounds (ZKML_LOOKAHEAD_TAIL=0 turns it off)
    size_t la_tail_max = zk::LA_TAIL_MAX;  // vectors up to this length go to the tail (ZKML_LOOKAHEAD_TAIL_MAX)
    uint32_t* h_msg() const { return h_sig + 64; }  // host -> GPU words (own cache lines)
    uint32_t* d_msg() const { return d_sig + 64; }
    zk::RoundScratch round_scratch() const {
        zk::RoundScratch r;
        r.partials = partials.as<uint32_t>();
        r.ticket = ticket();
        r.out = out_words();
        r.max_blocks = max_round_blocks;
        r.sig = nullptr;
        r.seq = 0;
        r.la_acc = la_acc();
        return r;
    }
};
