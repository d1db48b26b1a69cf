// C-ABI: context management and the ZkmlOps / GKR matmul entry points.
//
// Host side of the B200 matmul-sumcheck prover.  The Fiat-Shamir channel is
// advanced here, on the host, between kernel launches; each sumcheck round is
// one kernel (fold of the previous round fused with this round's sums, grid
// reduction included) followed by a 48-byte device-to-host read.
#include <atomic>
#include <chrono>
#include <x86intrin.h>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "channel.hpp"
#include "context.hpp"
#include "merkle.cuh"

// ZKML_LAYER_TRACE=1: the host timeline of each matmul layer reduction, printed to stderr
// (microseconds since the call entered the library).
namespace {
struct LayerTrace {
    bool on = getenv("ZKML_LAYER_TRACE") && getenv("ZKML_LAYER_TRACE")[0] == '1';
    std::chrono::steady_clock::time_point t0;
    std::vector<std::pair<const char*, double>> marks;
    void start() {
        if (!on) return;
        marks.clear();
        t0 = std::chrono::steady_clock::now();
    }
    void mark(const char* what) {
        if (on)
            marks.emplace_back(what, std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - t0).count());
    }
    void print() {
        if (!on) return;
        fprintf(stderr, "[zkml layer]");
        for (auto& m : marks) fprintf(stderr, " %s %.1f", m.first, m.second);
        fprintf(stderr, "\n");
    }
};
LayerTrace g_trace;
}  // namespace

namespace zk {

static thread_local std::string g_last_error;

int set_error(int status, const std::string& msg) {
    g_last_error = msg;
    return status;
}

int cuda_error(cudaError_t e, const char* what) {
    cudaGetLastError();  // clear a sticky launch error where possible
    int st = (e == cudaErrorMemoryAllocation) ? ZKML_ERR_OOM : ZKML_ERR_CUDA;
    return set_error(st, std::string("CUDA error in ") + what + ": " + cudaGetErrorString(e));
}

int DevBuf::ensure(size_t need) {
    if (need <= bytes && ptr) return ZKML_OK;
    release();
    size_t sz = need < 256 ? 256 : need;
    cudaError_t e = cudaMalloc(&ptr, sz);
    if (e != cudaSuccess) {
        ptr = nullptr;
        bytes = 0;
        return cuda_error(e, "cudaMalloc");
    }
    bytes = sz;
    return ZKML_OK;
}

void DevBuf::release() {
    if (ptr) cudaFree(ptr);
    ptr = nullptr;
    bytes = 0;
}

static cudaEvent_t pool_event(zkml_ctx* ctx) {
    if (!ctx->ev_pool.empty()) {
        cudaEvent_t e = ctx->ev_pool.back();
        ctx->ev_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

KTimer::KTimer(zkml_ctx* c, int k, bool enabled) : ctx(c), cls(k) {
    if (!enabled || !ctx->timing || !(ctx->timing_mask & (1u << k))) {
        cls = -1;
        return;
    }
    zkml_ctx::PendingEv p;
    p.cls = k;
    p.e0 = pool_event(ctx);
    p.e1 = pool_event(ctx);
    cudaEventRecord(p.e0, ctx->stream);
    ctx->pending.push_back(p);
}

KTimer::~KTimer() {
    if (cls < 0) return;
    cudaEventRecord(ctx->pending.back().e1, ctx->stream);
}

// Accumulate the timings of completed event pairs (call after a stream sync).
static void drain_timers(zkml_ctx* ctx) {
    for (auto& p : ctx->pending) {
        float ms = 0;
        if (cudaEventElapsedTime(&ms, p.e0, p.e1) == cudaSuccess) {
            ctx->ktime[p.cls].ms += ms;
            ctx->ktime[p.cls].launches++;
        } else {
            cudaGetLastError();
        }
        ctx->ev_pool.push_back(p.e0);
        ctx->ev_pool.push_back(p.e1);
    }
    ctx->pending.clear();
}

// Accumulate the event pairs whose end event has completed, without a stream sync;
// the others stay pending.
static void drain_done_timers(zkml_ctx* ctx) {
    std::vector<zkml_ctx::PendingEv> keep;
    for (auto& p : ctx->pending) {
        const cudaError_t q = cudaEventQuery(p.e1);
        if (q == cudaErrorNotReady) {
            keep.push_back(p);
            continue;
        }
        float ms = 0;
        if (q == cudaSuccess && cudaEventElapsedTime(&ms, p.e0, p.e1) == cudaSuccess) {
            ctx->ktime[p.cls].ms += ms;
            ctx->ktime[p.cls].launches++;
        } else {
            cudaGetLastError();
        }
        ctx->ev_pool.push_back(p.e0);
        ctx->ev_pool.push_back(p.e1);
    }
    ctx->pending.swap(keep);
}

// Host wall-time accumulator for a pseudo kernel class (timing mode only).
struct HostTimer {
    zkml_ctx* ctx;
    int cls;
    std::chrono::steady_clock::time_point t0;
    HostTimer(zkml_ctx* c, int k) : ctx(c), cls(k) {
        if (!ctx->timing || !(ctx->timing_mask & (1u << k))) cls = -1;
        else t0 = std::chrono::steady_clock::now();
    }
    ~HostTimer() {
        if (cls < 0) return;
        ctx->ktime[cls].ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        ctx->ktime[cls].launches++;
    }
};

static inline bool is_pow2(size_t x) { return x && !(x & (x - 1)); }
static inline size_t next_pow2(size_t x) {
    size_t p = 1;
    while (p < x) p <<= 1;
    return p;
}
static inline unsigned ilog2(size_t x) {
    unsigned l = 0;
    while (((size_t)1 << (l + 1)) <= x) l++;
    return l;
}

// Returns a device pointer for `p` (count bytes): p itself when it is device
// memory of the current GPU, otherwise a copy in `stage`.
int device_view(zkml_ctx* ctx, const void* p, size_t bytes, DevBuf& stage, const void** out) {
    cudaPointerAttributes attr;
    cudaError_t e = cudaPointerGetAttributes(&attr, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        attr.type = cudaMemoryTypeUnregistered;
    }
    if (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged) {
        if (attr.type == cudaMemoryTypeDevice && attr.device != ctx->device)
            return set_error(ZKML_ERR_INVALID_ARG, "input pointer is device memory of another GPU");
        *out = p;
        return ZKML_OK;
    }
    int rc = stage.ensure(bytes);
    if (rc) return rc;
    ZK_CUDA(cudaMemcpyAsync(stage.ptr, p, bytes, cudaMemcpyHostToDevice, ctx->stream));
    ctx->h2d_bytes += bytes;
    *out = stage.ptr;
    return ZKML_OK;
}

int matrix_view(zkml_ctx* ctx, const uint32_t* p, size_t count, DevBuf& stage, const void** out) {
    const char* on = getenv("ZKML_PACK_H2D");
    const char* mn = getenv("ZKML_PACK_MIN");
    const size_t min_words = mn ? (size_t)strtoull(mn, nullptr, 10) : ((size_t)1 << 22);
    if ((on && on[0] == '0') || count < min_words || count == 0) return device_view(ctx, p, count * 4, stage, out);
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
        cudaGetLastError();
        attr.type = cudaMemoryTypeUnregistered;
    }
    if (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged)
        return device_view(ctx, p, count * 4, stage, out);
    return upload_m31_packed(ctx, p, count, stage, out);
}

int check_err_flag(zkml_ctx* ctx, const char* what) {
    if (ctx->h_small[61]) {  // a queued look-ahead kernel gave up waiting for its challenge
        ctx->h_small[61] = 0;
        ZK_CUDA(cudaMemsetAsync(ctx->la_status(), 0, 4, ctx->stream));
        return set_error(ZKML_ERR_TIMEOUT, std::string(what) + ": a round kernel timed out waiting for its challenge");
    }
    if (ctx->h_small[48]) {
        ctx->h_small[48] = 0;
        ZK_CUDA(cudaMemsetAsync(ctx->err_flag(), 0, 4, ctx->stream));
        return set_error(ZKML_ERR_INVALID_ARG, std::string(what) + ": input value >= 2^31 is not an M31 element");
    }
    return ZKML_OK;
}

static inline qm31 ldq(const uint32_t* p) { return qm(p[0], p[1], p[2], p[3]); }
static inline void stq(uint32_t* p, const qm31& x) {
    p[0] = x.a;
    p[1] = x.b;
    p[2] = x.c;
    p[3] = x.d;
}

// Round polynomial from its values at 0, 1, 2 (backend.rs:163-166).
static void interpolate(const uint32_t* s12, qm31& c0, qm31& c1, qm31& c2) {
    static const uint32_t inv2 = minv(2);
    qm31 s0 = ldq(s12), s1 = ldq(s12 + 4), s2 = ldq(s12 + 8);
    c0 = s0;
    c2 = qmul_m(qadd(qsub(qsub(s2, s1), s1), s0), inv2);
    c1 = qsub(qsub(s1, s0), c2);
}

// Waits until a kernel publishes `seq` in the mapped signal words, then copies
// `n` result words out.  Polls the stream for errors while waiting and gives up
// after a bounded time, so a failed launch never leaves the host spinning.
int wait_signal(zkml_ctx* ctx, uint32_t seq, uint32_t* words, int n) {
    HostTimer ht(ctx, KC_HOST_SYNC);
    volatile uint32_t* sig = ctx->h_sig;
    const auto t0 = std::chrono::steady_clock::now();
    for (uint64_t it = 0; sig[0] != seq; it++) {
        _mm_pause();
        if ((it & 1023) == 1023) {
            cudaError_t e = cudaStreamQuery(ctx->stream);
            if (e != cudaSuccess && e != cudaErrorNotReady) return cuda_error(e, "round kernel");
            const double waited = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
            if (e == cudaSuccess && sig[0] != seq && waited > 1.0)
                return set_error(ZKML_ERR_CUDA, "round kernel finished without publishing its result");
            if (waited > 120.0) return set_error(ZKML_ERR_TIMEOUT, "timed out waiting for a round kernel");
        }
    }
    std::atomic_thread_fence(std::memory_order_acquire);
    for (int i = 0; i < n; i++) words[i] = sig[1 + i];
    return ZKML_OK;
}

// Reads the device error flag (one synchronisation).
int read_err_flag(zkml_ctx* ctx) {
    ZK_CUDA(cudaMemcpyAsync(ctx->h_small + 48, ctx->err_flag(), 16 * 4, cudaMemcpyDeviceToHost, ctx->stream));
    ZK_CUDA(cudaStreamSynchronize(ctx->stream));
    if (!ctx->pending.empty()) drain_timers(ctx);
    return ZKML_OK;
}

// Hands the round-r challenge to the persistent kernel (or tells it to stop).
static void post_challenge(zkml_ctx* ctx, uint32_t seq, const qm31& alpha, bool abort) {
    volatile uint32_t* m = ctx->h_msg();
    m[1] = alpha.a;
    m[2] = alpha.b;
    m[3] = alpha.c;
    m[4] = alpha.d;
    m[5] = abort ? 1u : 0u;
    std::atomic_thread_fence(std::memory_order_release);
    m[0] = seq;
}

// All rounds in one cooperative launch; the host only waits for round words
// and posts challenges.  Returns ZKML_ERR_UNSUPPORTED if the launch is refused.
static int run_sumcheck_persistent(zkml_ctx* ctx, uint4* A, uint4* B, const uint32_t* A32, const uint32_t* B32,
                                   size_t len, zkml_channel* chs, uint32_t* out_rp, uint32_t* out_ch,
                                   uint32_t* fa_out, uint32_t* fb_out, const ClaimHook* hook) {
    Channel ch(chs);
    cudaStream_t s = ctx->stream;
    const unsigned log_k = ilog2(len);
    PersistArgs pa;
    pa.A = A32 ? ctx->fa.as<uint4>() : A;
    pa.B = B32 ? ctx->fb.as<uint4>() : B;
    pa.A32 = A32;
    pa.B32 = B32;
    pa.len = len;
    pa.log_k = (int)log_k;
    pa.partials = ctx->partials.as<uint32_t>();
    pa.bar = ctx->grid_bar();
    pa.alpha_dev = ctx->alpha_slot();
    pa.status = ctx->persist_status();
    pa.sig = ctx->d_sig;
    pa.hostmsg = ctx->d_msg();
    pa.seq_base = ctx->sig_seq + 1;
    ctx->sig_seq += log_k + 1;
    ZK_CUDA(cudaMemsetAsync(ctx->persist_status(), 0, 4, s));
    ZK_CUDA(cudaMemsetAsync(ctx->grid_bar(), 0, 8, s));
    ctx->h_msg()[5] = 0;
    cudaError_t e = cudaSuccess;
    int grid;
    {
        KTimer t(ctx, KC_ROUND);
        grid = launch_sumcheck_persistent(pa, ctx->num_sms, s, &e);
    }
    if (!grid) {
        cudaGetLastError();
        return ZKML_ERR_UNSUPPORTED;
    }
    ctx->launches++;
    if (hook && hook->overlap) hook->overlap(hook->arg);
    uint32_t words[12];
    int rc = ZKML_OK;
    for (unsigned r = 0; r < log_k; r++) {
        if ((rc = wait_signal(ctx, pa.seq_base + r, words, 12))) break;
        if (r == 0 && hook && hook->fn) hook->fn(hook->arg, qadd(ldq(words), ldq(words + 4)));
        if (hook && hook->adjust) hook->adjust(hook->arg, r, words);
        qm31 c0, c1, c2, alpha;
        {
            HostTimer ht(ctx, KC_HOST_CHANNEL);
            interpolate(words, c0, c1, c2);
            ch.mix_poly_coeffs(c0, c1, c2);
            alpha = ch.draw_qm31();
        }
        if (hook && hook->challenge) hook->challenge(hook->arg, r, alpha);
        post_challenge(ctx, pa.seq_base + r, alpha, false);
        if (out_rp) {
            stq(out_rp + 12 * r, c0);
            stq(out_rp + 12 * r + 4, c1);
            stq(out_rp + 12 * r + 8, c2);
        }
        if (out_ch) stq(out_ch + 4 * r, alpha);
    }
    if (!rc) rc = wait_signal(ctx, pa.seq_base + log_k, words, 8);
    if (rc) {
        // release the kernel (it exits on the abort word) before reporting
        post_challenge(ctx, pa.seq_base, qzero(), true);
        cudaStreamSynchronize(s);
        return rc;
    }
    memcpy(fa_out, words, 16);
    memcpy(fb_out, words + 4, 16);
    uint32_t status = 0;
    ZK_CUDA(cudaMemcpyAsync(&status, ctx->persist_status(), 4, cudaMemcpyDeviceToHost, s));
    if ((rc = read_err_flag(ctx))) return rc;
    if (status) return set_error(ZKML_ERR_TIMEOUT, "sumcheck round kernel timed out waiting (status " +
                                                       std::to_string(status) + ")");
    return check_err_flag(ctx, "reduce_matmul_layer");
}

// The sumcheck round loop over (A, B).  In M31 mode A32/B32 hold the base-field
// vectors (length len) and the first fold writes QM31 into ctx->fa / fb.
// Host side of the look-ahead rounds (launch_round_lookahead).
constexpr int LA_WORDS_HOST = 42;  // 40 words + the last round's two error words

// Round r's own sums from its look-ahead words (len = |V_r|).
static void la_round_sums(const uint32_t* w, size_t len, uint32_t s12[12]) {
    if (len == 2) {
        memcpy(s12, w, 48);
        return;
    }
    stq(s12, qadd(ldq(w), ldq(w + 4)));
    stq(s12 + 4, qadd(ldq(w + 8), ldq(w + 12)));
    stq(s12 + 8, ldq(w + 16));
}

// Round r+1's sums from round r's look-ahead words, at the challenge x of round r.
static void la_next_sums(const uint32_t* w, const qm31& x, uint32_t s12[12]) {
    auto quad = [&](const qm31& c0, const qm31& both, const qm31& c2) {
        const qm31 c1 = qsub(qsub(both, c0), c2);
        return qadd(c0, qmul(x, qadd(c1, qmul(x, c2))));
    };
    stq(s12, quad(ldq(w), ldq(w + 8), ldq(w + 20)));
    stq(s12 + 4, quad(ldq(w + 4), ldq(w + 12), ldq(w + 24)));
    stq(s12 + 8, quad(ldq(w + 28), ldq(w + 36), ldq(w + 32)));
}

// The look-ahead kernels of one sumcheck.  Queued mode (the default) puts them
// all on the stream up front: kernel 0 needs no challenge (or is given it),
// kernel j > 0 waits for the host to post the challenge of the round before it
// into its slot, and the rounds whose vectors fit LA_TAIL_MAX run in one
// resident block.  Every queued kernel either gets its challenge or an abort,
// so the queue always drains.  Unqueued mode (ZKML_LA_QUEUE=0, and always under
// Nsight Compute, which serialises launches and would otherwise leave a queued
// kernel waiting for a post that cannot come) launches kernel j when its
// challenge is known.
struct LaQueue {
    static constexpr int MAX = 40;
    zkml_ctx* ctx;
    uint4 *A = nullptr, *B = nullptr;
    RoundScratch rs;
    cudaStream_t stream = nullptr;
    bool queued = true;
    int n = 0, posted = 1;
    uint32_t seq[MAX], tag[MAX];
    int slot[MAX];
    size_t len[MAX];

    explicit LaQueue(zkml_ctx* c) : ctx(c), queued(c->la_queue) {}

    int enqueue(uint4* A_, uint4* B_, size_t L0, bool fold0, const qm31& alpha0, RoundScratch rs_, cudaStream_t s) {
        A = A_;
        B = B_;
        rs = rs_;
        stream = s;
        n = 0;
        posted = 1;
        for (size_t L = L0; L >= 2 && n < MAX; L /= 2) len[n++] = L;
        if (!queued) return launch_one(0, fold0, alpha0, nullptr, 0);
        for (int j = 0; j < n; j++) {
            seq[j] = ++ctx->sig_seq;
            if (j > 0) {
                tag[j] = ++ctx->la_msg_seq;
                slot[j] = (int)(tag[j] % zkml_ctx::LA_SLOTS);
            }
        }
        for (int j = 0; j < n; j++) {
            if (ctx->la_tail && len[j] <= ctx->la_tail_max) {  // the remaining rounds in one resident block
                const bool wait0 = j > 0;
                const bool f0 = wait0 || fold0;
                const uint32_t tag_base = wait0 ? tag[j] : (n > 1 ? tag[1] - 1 : 0);
                if (launch_lookahead_tail(A, B, f0 ? 2 * len[j] : len[j], f0, wait0, alpha0, rs.sig, seq[j],
                                          ctx->d_la_msg(), tag_base, zkml_ctx::LA_SLOTS, ctx->la_status(), s,
                                          ctx->err_flag(), wait0 && ctx->la_pdl))
                    return set_error(ZKML_ERR_CUDA, "cannot configure the look-ahead tail kernel");
                ZK_CUDA(cudaGetLastError());
                ctx->launches++;
                return ZKML_OK;
            }
            int rc = j == 0 ? launch_one(0, fold0, alpha0, nullptr, 0)
                            : launch_one(j, true, qzero(), ctx->d_la_msg() + 8 * slot[j], tag[j]);
            if (rc) return rc;
        }
        return ZKML_OK;
    }
    int launch_one(int j, bool fold, const qm31& alpha, const uint32_t* wait_msg, uint32_t wait_tag) {
        if (!queued) seq[j] = ++ctx->sig_seq;
        rs.seq = seq[j];
        {
            KTimer t(ctx, KC_ROUND, wait_msg == nullptr);
            launch_round_lookahead(A, B, len[j], fold, alpha, rs, stream, wait_msg, wait_tag, ctx->la_status(),
                                   ctx->la_mailbox(), ctx->err_flag(), queued && wait_msg && ctx->la_pdl);
        }
        ZK_CUDA(cudaGetLastError());
        ctx->launches++;
        return ZKML_OK;
    }
    // Hands round j its challenge (the one drawn in round j - 1).
    int post(int j, const qm31& a, bool abort) {
        if (!queued) return abort ? ZKML_OK : launch_one(j, true, a, nullptr, 0);
        volatile uint32_t* m = ctx->h_la_msg() + 8 * slot[j];
        const uint32_t ab = abort ? 1u : 0u;
        m[1] = a.a;
        m[2] = a.b;
        m[3] = a.c;
        m[4] = a.d;
        m[5] = ab;
        m[6] = tag[j] ^ a.a ^ a.b ^ a.c ^ a.d ^ ab ^ LA_SLOT_MIX;  // lets the GPU take the slot in one read
        std::atomic_thread_fence(std::memory_order_release);
        m[0] = tag[j];
        return ZKML_OK;
    }
    void abort_rest() {
        for (; posted < n; posted++) post(posted, qzero(), true);
    }
};

int run_sumcheck(zkml_ctx* ctx, uint4* A, uint4* B, const uint32_t* A32, const uint32_t* B32, size_t len,
                 zkml_channel* chs, uint32_t* out_rp, uint32_t* out_ch, uint32_t* fa_out, uint32_t* fb_out,
                 const ClaimHook* hook) {
    Channel ch(chs);
    cudaStream_t s = ctx->stream;
    RoundScratch rs = ctx->round_scratch();
    rs.sig = ctx->d_sig;
    const unsigned log_k = ilog2(len);
    bool m31 = A32 != nullptr;
    int rc;
    if (log_k == 0) {
        if (m31) {
            uint32_t v[2];
            ZK_CUDA(cudaMemcpyAsync(&v[0], A32, 4, cudaMemcpyDeviceToHost, s));
            ZK_CUDA(cudaMemcpyAsync(&v[1], B32, 4, cudaMemcpyDeviceToHost, s));
            ZK_CUDA(cudaStreamSynchronize(s));
            stq(fa_out, qm(red32(v[0]), 0, 0, 0));
            stq(fb_out, qm(red32(v[1]), 0, 0, 0));
        } else {
            ZK_CUDA(cudaMemcpyAsync(fa_out, A, 16, cudaMemcpyDeviceToHost, s));
            ZK_CUDA(cudaMemcpyAsync(fb_out, B, 16, cudaMemcpyDeviceToHost, s));
            ZK_CUDA(cudaStreamSynchronize(s));
        }
        if ((rc = read_err_flag(ctx)) || (rc = check_err_flag(ctx, "reduce_matmul_layer"))) return rc;
        if (hook && hook->overlap) hook->overlap(hook->arg);
        if (hook && hook->fn) hook->fn(hook->arg, qmul(ldq(fa_out), ldq(fb_out)));
        return ZKML_OK;
    }
    if (ctx->persistent) {
        rc = run_sumcheck_persistent(ctx, A, B, A32, B32, len, chs, out_rp, out_ch, fa_out, fb_out, hook);
        if (rc != ZKML_ERR_UNSUPPORTED) return rc;
        ctx->persistent = false;  // cooperative launch unavailable: use one launch per round
    }
    // Vectors of at most lookahead_max elements run the look-ahead rounds
    // (launch_round_lookahead): a round's kernel runs while the host hashes the
    // previous round, and the host evaluates the next round's sums itself.
    const size_t la_max = ctx->lookahead_max;
    bool la = false;
    if (m31 && len <= la_max) {  // small base-field product: lift to QM31 first
        if ((rc = ctx->fa.ensure(len * 16)) || (rc = ctx->fb.ensure(len * 16))) return rc;
        launch_m31_to_qm31(A32, len, ctx->fa.as<uint4>(), len, ctx->err_flag(), s);
        launch_m31_to_qm31(B32, len, ctx->fb.as<uint4>(), len, ctx->err_flag(), s);
        ctx->launches += 2;
        A = ctx->fa.as<uint4>();
        B = ctx->fb.as<uint4>();
        m31 = false;
    }
    LaQueue laq(ctx);
    if (!m31 && len <= la_max) {
        if ((rc = laq.enqueue(A, B, len, false, qzero(), rs, s))) return rc;
        la = true;
    } else {
        rs.seq = ++ctx->sig_seq;
        {
            KTimer t(ctx, KC_ROUND);
            if (m31)
                launch_round_m31(A32, B32, len, rs, ctx->err_flag(), s);
            else
                launch_round_qm31(A, B, len, rs, s);
        }
        ZK_CUDA(cudaGetLastError());
        ctx->launches++;
    }
    g_trace.mark("queued");
    if (hook && hook->overlap) hook->overlap(hook->arg);  // host transcript work while the GPU runs
    g_trace.mark("overlap");
    uint32_t words[LA_WORDS_HOST];
    uint32_t s12[12];
    uint32_t la_w[LA_WORDS_HOST];  // the previous look-ahead words (this round's sums as a quadratic)
    qm31 alpha_prev = qzero();
    int j = 0;  // look-ahead kernel whose words belong to this round
    for (unsigned r = 0; r < log_k; r++) {
        if (la && j > 0) {
            la_next_sums(la_w, alpha_prev, s12);  // this round's kernel may still be running
        } else {
            rc = wait_signal(ctx, la ? laq.seq[0] : rs.seq, words, la ? LA_WORDS_HOST : 12);
            g_trace.mark("w0");
            if (rc) {
                laq.abort_rest();
                return rc;
            }
            if (la)
                la_round_sums(words, laq.len[0], s12);
            else
                memcpy(s12, words, sizeof(s12));
        }
        if (r == 0 && hook && hook->fn) hook->fn(hook->arg, qadd(ldq(s12), ldq(s12 + 4)));
        qm31 c0, c1, c2, alpha;
        {
            HostTimer ht(ctx, KC_HOST_CHANNEL);
            uint32_t adj[12];  // s12 stays the raw sums: the look-ahead check compares them
            memcpy(adj, s12, sizeof(adj));
            if (hook && hook->adjust) hook->adjust(hook->arg, r, adj);
            interpolate(adj, c0, c1, c2);
            ch.mix_poly_coeffs(c0, c1, c2);
            alpha = ch.draw_qm31();
        }
        g_trace.mark("r");
        if (hook && hook->challenge) hook->challenge(hook->arg, r, alpha);
        if (out_rp) {
            stq(out_rp + 12 * r, c0);
            stq(out_rp + 12 * r + 4, c1);
            stq(out_rp + 12 * r + 8, c2);
        }
        if (out_ch) stq(out_ch + 4 * r, alpha);
        if (la) {
            if (j > 0) {  // this round's words: check them against the quadratic (read before the next post)
                if ((rc = wait_signal(ctx, laq.seq[j], words, LA_WORDS_HOST))) {
                    laq.abort_rest();
                    return rc;
                }
                uint32_t plain[12];
                la_round_sums(words, laq.len[j], plain);
                if (memcmp(plain, s12, sizeof(plain)) != 0) {
                    laq.abort_rest();
                    // invalid input words or a timed-out wait surface as a disagreement: report them first
                    if ((rc = read_err_flag(ctx)) || (rc = check_err_flag(ctx, "reduce_matmul_layer"))) return rc;
                    return set_error(ZKML_ERR_CUDA, "look-ahead round sums disagree with the round kernel");
                }
            }
            if (laq.len[j] == 2) {  // final values from the last round's words
                const qm31 a0 = ldq(words + 12), a1 = ldq(words + 16), b0 = ldq(words + 20), b1 = ldq(words + 24);
                stq(fa_out, qadd(a0, qmul(alpha, qsub(a1, a0))));
                stq(fb_out, qadd(b0, qmul(alpha, qsub(b1, b0))));
                g_trace.mark("last");
                // The last kernel read the error words after every earlier kernel of the
                // stream had ended: both clear means no read-back (and no stream wait).
                if (words[40] == 0 && words[41] == 0) {
                    if (!ctx->pending.empty()) drain_done_timers(ctx);
                    if (ctx->pending.empty()) return ZKML_OK;
                }
                if ((rc = read_err_flag(ctx))) return rc;
                return check_err_flag(ctx, "reduce_matmul_layer");
            }
            memcpy(la_w, words, sizeof(la_w));
            alpha_prev = alpha;
            if ((rc = laq.post(++j, alpha, false))) {  // releases (or launches) the next round's kernel
                laq.abort_rest();
                return rc;
            }
            laq.posted = j + 1;
            continue;
        }
        if (len == 2) {
            rs.seq = ++ctx->sig_seq;
            {
                KTimer t(ctx, KC_ROUND);
                launch_final_fold(A, B, m31 ? A32 : nullptr, m31 ? B32 : nullptr, len, alpha, ctx->out_words(),
                                  rs.sig, rs.seq, s);
            }
        } else if (!m31 && len / 2 <= la_max) {
            if ((rc = laq.enqueue(A, B, len / 2, true, alpha, rs, s))) return rc;
            la = true;
            j = 0;
            len /= 2;
            continue;
        } else {
            rs.seq = ++ctx->sig_seq;
            KTimer t(ctx, KC_ROUND);
            if (m31) {
                A = ctx->fa.as<uint4>();
                B = ctx->fb.as<uint4>();
                launch_fold_round_m31(A32, B32, len, alpha, A, B, rs, s);
                m31 = false;
            } else {
                launch_fold_round_qm31(A, B, len, alpha, rs, s);
            }
        }
        ZK_CUDA(cudaGetLastError());
        ctx->launches++;
        len /= 2;
    }
    if ((rc = wait_signal(ctx, rs.seq, words, 8))) return rc;
    memcpy(fa_out, words, 16);
    memcpy(fb_out, words + 4, 16);
    if ((rc = read_err_flag(ctx))) return rc;
    return check_err_flag(ctx, "reduce_matmul_layer");
}

// Restriction of A (rows by r_i) and B (columns by r_j) into ctx->fa / fb (length pk).
static int restrict_ab(zkml_ctx* ctx, const uint32_t* A, size_t m, size_t k, const uint32_t* B, size_t n,
                       const qm31* r_i, unsigned n_ri, const qm31* r_j, unsigned n_rj, size_t pk,
                       const uint64_t* fb_words) {
    cudaStream_t s = ctx->stream;
    int rc;
    if ((rc = ctx->fa.ensure(pk * 16)) || (rc = ctx->fb.ensure(pk * 16))) return rc;
    uint4* fa = ctx->fa.as<uint4>();
    uint4* fb = ctx->fb.as<uint4>();
    // The row side (small) runs on the side stream under the column side's weight stream; it
    // forks after every earlier operation of the stream (e.g. an input copy) and joins
    // before the round kernels.
    // Up to 2^8 rows: the row side and the finalisations are one launch after the column
    // restriction (launch_restrict_rows_fused); larger A runs its own row pass.
    const bool rows_timed = ctx->timing && (ctx->timing_mask & (1u << KC_RESTRICT_ROWS));
    const bool fused = n_ri >= 1 && n_ri <= 8 && ctx->rows_fused && !rows_timed;
    const bool side = n_ri != 0 && !fused && ctx->row_side_stream && !rows_timed && ctx->side_stream;
    if (side) ZK_CUDA(cudaEventRecord(ctx->ev_fork, s));
    bool acc_b_pending = false;  // f_b still in acc_b (finalised by the fused row launch)
    // f_b first: the column restriction streams the whole weight and is the long kernel, so it
    // goes to the GPU before the host spends time launching the row side
    if (fb_words) {  // f_b from column-block partial sums added across ranks (zkml_restrict_cols_block)
        launch_acc_finalize(reinterpret_cast<const unsigned long long*>(fb_words), k, fb, pk, s);
        ctx->launches++;
    } else if (n_rj == 0) {  // n == 1: f_b is B's single column (contiguous)
        launch_m31_to_qm31(B, k, fb, pk, ctx->err_flag(), s);
        ctx->launches++;
    } else {
        const unsigned lo_vars = n_rj < 6 ? n_rj : 6;
        const unsigned hi_vars = n_rj - lo_vars;
        const bool tc = ctx->restrict_tc && restrict_cols_tc_ok(B, (uint32_t)n);
        if ((rc = ctx->acc_b.ensure(k * 32))) return rc;
        if (!tc) {  // the tensor-pipe kernel forms its eq weights from r_j itself
            if ((rc = ctx->eq_hi.ensure(((size_t)16) << hi_vars)) || (rc = ctx->eq_lo.ensure(64 * 16))) return rc;
            launch_eq_table(r_j, hi_vars, ctx->eq_hi.as<uint4>(), (size_t)1 << hi_vars, s);
            launch_eq_table(r_j + hi_vars, lo_vars, ctx->eq_lo.as<uint4>(), 64, s);
            ctx->launches += 2;
        }
        ZK_CUDA(cudaMemsetAsync(ctx->acc_b.ptr, 0, k * 32, s));
        {
            KTimer t(ctx, KC_RESTRICT_COLS);
            if (tc)
                launch_restrict_cols_tc(B, (uint32_t)k, (uint32_t)n, r_j, hi_vars, lo_vars, 0,
                                        ctx->acc_b.as<unsigned long long>(), ctx->err_flag(), ctx->num_sms, s);
            else
                launch_restrict_cols(B, (uint32_t)k, (uint32_t)n, ctx->eq_hi.as<uint4>(), ctx->eq_lo.as<uint4>(),
                                     ctx->acc_b.as<unsigned long long>(), ctx->err_flag(), ctx->num_sms, s);
        }
        ctx->launches++;
        if (!fused) {
            launch_acc_finalize(ctx->acc_b.as<unsigned long long>(), k, fb, pk, s);
            ctx->launches++;
        }
        acc_b_pending = true;
    }
    if (fused) {
        if (launch_restrict_rows_fused(A, (uint32_t)m, (uint32_t)k, r_i, (int)n_ri,
                                       acc_b_pending ? ctx->acc_b.as<unsigned long long>() : nullptr, k, fa, fb, pk,
                                       ctx->err_flag(), s))
            return set_error(ZKML_ERR_INVALID_ARG, "row restriction bounds");
        ZK_CUDA(cudaGetLastError());
        ctx->launches++;
    } else if (n_ri == 0) {  // m == 1: f_a is A's single row
        launch_m31_to_qm31(A, k, fa, pk, ctx->err_flag(), s);
        ctx->launches++;
    } else {
        if ((rc = ctx->eq_a.ensure(((size_t)16) << n_ri)) || (rc = ctx->acc_a.ensure(k * 32))) return rc;
        cudaStream_t rs = s;
        if (side) {
            rs = ctx->side_stream;
            ZK_CUDA(cudaStreamWaitEvent(rs, ctx->ev_fork, 0));
        }
        launch_eq_table(r_i, n_ri, ctx->eq_a.as<uint4>(), (size_t)1 << n_ri, rs);
        ZK_CUDA(cudaMemsetAsync(ctx->acc_a.ptr, 0, k * 32, rs));
        {
            KTimer t(ctx, KC_RESTRICT_ROWS);
            launch_restrict_rows(A, (uint32_t)m, (uint32_t)k, ctx->eq_a.as<uint4>(),
                                 ctx->acc_a.as<unsigned long long>(), ctx->err_flag(), rs);
        }
        launch_acc_finalize(ctx->acc_a.as<unsigned long long>(), k, fa, pk, rs);
        ctx->launches += 3;
        if (side) {
            ZK_CUDA(cudaEventRecord(ctx->ev_join, rs));
            ZK_CUDA(cudaStreamWaitEvent(s, ctx->ev_join, 0));
        }
    }
    return ZKML_OK;
}

}  // namespace zk

using namespace zk;

extern "C" {

int zkml_abi_version(void) { return ZKML_ABI_VERSION; }
const char* zkml_last_error(void) { return g_last_error.c_str(); }

int zkml_ctx_create(int device, zkml_ctx** out) {
    if (!out) return set_error(ZKML_ERR_INVALID_ARG, "out is NULL");
    *out = nullptr;
    felt_init();
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0)
        return set_error(ZKML_ERR_CUDA, std::string("no CUDA device: ") + cudaGetErrorString(e));
    if (device < 0 || device >= n) return set_error(ZKML_ERR_INVALID_ARG, "device ordinal out of range");
    ZK_CUDA(cudaSetDevice(device));
    int major = 0;
    ZK_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
    if (major != 10)
        return set_error(ZKML_ERR_UNSUPPORTED, "this build targets sm_100a (B200); device has compute capability " +
                                                   std::to_string(major) + ".x");
    zkml_ctx* ctx = new zkml_ctx();
    ctx->device = device;
    cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, device);
    {
        const char* pv = getenv("ZKML_PERSISTENT_ROUNDS");
        if (pv) ctx->persistent = pv[0] == '1';
        const char* lv = getenv("ZKML_LOOKAHEAD_MAX");
        if (lv) ctx->lookahead_max = strtoull(lv, nullptr, 10);
        const char* tv = getenv("ZKML_LOOKAHEAD_TAIL");
        if (tv) ctx->la_tail = tv[0] != '0';
        const char* tm = getenv("ZKML_LOOKAHEAD_TAIL_MAX");  // a power of two in [2, LA_TAIL_MAX]
        if (tm) {
            const size_t v = strtoull(tm, nullptr, 10);
            if (v >= 2 && v <= LA_TAIL_MAX && !(v & (v - 1))) ctx->la_tail_max = v;
        }
        const char* rv = getenv("ZKML_RESTRICT_TC");
        if (rv) ctx->restrict_tc = rv[0] != '0';
        const char* qv = getenv("ZKML_LA_QUEUE");
        if (qv) ctx->la_queue = qv[0] != '0';
        // A profiler that serialises launches would hold a queued kernel back from the post it waits
        // for; Nsight Compute marks its target processes with these variables.
        if (getenv("NV_TPS_LAUNCH_TOKEN") || getenv("NV_NSIGHT_INJECTION_TRANSPORT_TYPE") ||
            getenv("CUDA_INJECTION64_PATH"))
            ctx->la_queue = false;
    }
    ctx->max_round_blocks = ctx->num_sms * 8;
    int rc = ZKML_OK;
    e = cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) rc = cuda_error(e, "cudaStreamCreate");
    ctx->stream = ctx->own_stream;
    if (!rc && (e = cudaStreamCreateWithFlags(&ctx->side_stream, cudaStreamNonBlocking)) != cudaSuccess)
        rc = cuda_error(e, "cudaStreamCreate");
    if (!rc && ((e = cudaEventCreateWithFlags(&ctx->ev_fork, cudaEventDisableTiming)) != cudaSuccess ||
                (e = cudaEventCreateWithFlags(&ctx->ev_join, cudaEventDisableTiming)) != cudaSuccess))
        rc = cuda_error(e, "cudaEventCreate");
    {
        const char* rv = getenv("ZKML_ROW_SIDE_STREAM");
        if (rv) ctx->row_side_stream = rv[0] != '0';
        const char* pv = getenv("ZKML_LA_PDL");
        if (pv) ctx->la_pdl = pv[0] != '0';
        const char* fv = getenv("ZKML_ROWS_FUSED");
        if (fv) ctx->rows_fused = fv[0] != '0';
    }
    if (!rc) rc = ctx->partials.ensure((size_t)ctx->max_round_blocks * 16 * 4);
    if (!rc) rc = ctx->small.ensure(256 * 4);
    if (!rc && (e = cudaMemset(ctx->small.ptr, 0, 256 * 4)) != cudaSuccess) rc = cuda_error(e, "cudaMemset");
    if (!rc && (e = cudaMallocHost(&ctx->h_small, 64 * 4)) != cudaSuccess) rc = cuda_error(e, "cudaMallocHost");
    if (!rc && (e = cudaHostAlloc(&ctx->h_sig, 4096, cudaHostAllocMapped)) != cudaSuccess)
        rc = cuda_error(e, "cudaHostAlloc(mapped)");
    if (!rc) {
        memset(ctx->h_sig, 0, 4096);
        if ((e = cudaHostGetDevicePointer((void**)&ctx->d_sig, ctx->h_sig, 0)) != cudaSuccess)
            rc = cuda_error(e, "cudaHostGetDevicePointer");
    }
    if (!rc) {
        // Hades round keys and Montgomery constants into this device's constant bank
        const felt two = f_from_u64(2);
        if ((e = upload_hades_constants(HADES_RC, &F_R2, &two, &F_ONE)) != cudaSuccess) rc = cuda_error(e, "upload constants");
    }
    if (rc) {
        zkml_ctx_destroy(ctx);
        return rc;
    }
    memset(ctx->h_small, 0, 64 * 4);
    *out = ctx;
    return ZKML_OK;
}

int zkml_ctx_destroy(zkml_ctx* ctx) {
    if (!ctx) return ZKML_OK;
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    DevBuf* bufs[] = {&ctx->a_in, &ctx->b_in, &ctx->fa,    &ctx->fb,       &ctx->acc_a, &ctx->acc_b,
                      &ctx->eq_a, &ctx->eq_hi, &ctx->eq_lo, &ctx->partials, &ctx->small};
    for (DevBuf* b : bufs) b->release();
    for (DevBuf& t : ctx->act_tables) t.release();
    ctx->rsqrt_table.release();
    ctx->lu.release();
    ctx->op.release();
    ctx->gather_dev.release();
    ctx->mesh_stage.release();
    if (ctx->h_stage) cudaFreeHost(ctx->h_stage);
    ctx->pack_dev.release();
    if (ctx->pack_host) cudaFreeHost(ctx->pack_host);
    if (ctx->pack_event) cudaEventDestroy(ctx->pack_event);
    ctx->sc_a.release();
    ctx->sc_b.release();
    if (ctx->h_small) cudaFreeHost(ctx->h_small);
    if (ctx->h_sig) cudaFreeHost(ctx->h_sig);
    drain_timers(ctx);
    for (cudaEvent_t e : ctx->ev_pool) cudaEventDestroy(e);
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    if (ctx->side_stream) cudaStreamSynchronize(ctx->side_stream), cudaStreamDestroy(ctx->side_stream);
    if (ctx->ev_fork) cudaEventDestroy(ctx->ev_fork);
    if (ctx->ev_join) cudaEventDestroy(ctx->ev_join);
    delete ctx;
    return ZKML_OK;
}

int zkml_ctx_device(const zkml_ctx* ctx) { return ctx ? ctx->device : -1; }
uint64_t zkml_ctx_kernel_launches(const zkml_ctx* ctx) { return ctx ? ctx->launches : 0; }
uint64_t zkml_ctx_h2d_bytes(const zkml_ctx* ctx) { return ctx ? ctx->h2d_bytes : 0; }

int zkml_ctx_enable_timing(zkml_ctx* ctx, int enable) {
    if (!ctx) return set_error(ZKML_ERR_INVALID_ARG, "ctx is NULL");
    ZK_CUDA(cudaSetDevice(ctx->device));
    ZK_CUDA(cudaStreamSynchronize(ctx->stream));
    drain_timers(ctx);
    ctx->timing = enable != 0;
    ctx->timing_mask = enable < 0 ? ~0u : (unsigned)enable;
    for (auto& k : ctx->ktime) k = zkml_ctx::KTime();
    return ZKML_OK;
}

int zkml_ctx_kernel_time(zkml_ctx* ctx, const char* kernel, double* out_ms, uint64_t* out_launches) {
    if (!ctx || !kernel) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    static const char* names[6] = {"restrict_cols", "restrict_rows", "sumcheck_round",
                                   "merkle",        "host_sync",     "host_channel"};
    if (!ctx->pending.empty()) {
        ZK_CUDA(cudaStreamSynchronize(ctx->stream));
        drain_timers(ctx);
    }
    for (int i = 0; i < 6; i++)
        if (!strcmp(kernel, names[i])) {
            if (out_ms) *out_ms = ctx->ktime[i].ms;
            if (out_launches) *out_launches = ctx->ktime[i].launches;
            return ZKML_OK;
        }
    return set_error(ZKML_ERR_INVALID_ARG, std::string("unknown kernel class ") + kernel);
}

int zkml_ctx_set_stream(zkml_ctx* ctx, void* stream) {
    if (!ctx) return set_error(ZKML_ERR_INVALID_ARG, "ctx is NULL");
    ctx->stream = stream ? static_cast<cudaStream_t>(stream) : ctx->own_stream;
    return ZKML_OK;
}

int zkml_reduce_matmul_layer(zkml_ctx* ctx, const uint32_t* a, size_t a_rows, size_t a_cols, const uint32_t* b,
                             size_t b_rows, size_t b_cols, const uint32_t* r_i, size_t n_ri, const uint32_t* r_j,
                             size_t n_rj, size_t pk, zkml_channel* ch, uint32_t* out_round_polys,
                             uint32_t* out_challenges, uint32_t out_final_a[4], uint32_t out_final_b[4]) {
    return zk::reduce_matmul_internal(ctx, a, a_rows, a_cols, b, b_rows, b_cols, r_i, n_ri, r_j, n_rj, pk, ch,
                                      out_round_polys, out_challenges, out_final_a, out_final_b, nullptr);
}

}  // extern "C"

namespace zk {
int reduce_matmul_internal(zkml_ctx* ctx, const uint32_t* a, size_t a_rows, size_t a_cols, const uint32_t* b,
                           size_t b_rows, size_t b_cols, const uint32_t* r_i, size_t n_ri, const uint32_t* r_j,
                           size_t n_rj, size_t pk, zkml_channel* ch, uint32_t* out_round_polys,
                           uint32_t* out_challenges, uint32_t out_final_a[4], uint32_t out_final_b[4],
                           const ClaimHook* hook, const uint64_t* fb_words) {
    if (!ctx || !a || !(b || fb_words) || !ch || !out_final_a || !out_final_b)
        return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    if (a_rows == 0 || a_cols == 0 || b_cols == 0) return set_error(ZKML_ERR_INVALID_ARG, "empty matrix");
    if (a_cols != b_rows) return set_error(ZKML_ERR_INVALID_ARG, "A.cols must equal B.rows");
    if (a_rows > (1u << 30) || a_cols > (1u << 30) || b_cols > (1u << 30))
        return set_error(ZKML_ERR_INVALID_ARG, "matrix dimension exceeds 2^30");
    if (pk != next_pow2(a_cols)) return set_error(ZKML_ERR_INVALID_ARG, "pk must be next_pow2(A.cols)");
    if (n_ri != ilog2(next_pow2(a_rows)) || n_rj != ilog2(next_pow2(b_cols)))
        return set_error(ZKML_ERR_INVALID_ARG, "r_i / r_j length does not match the padded dimensions");
    if (a_rows * a_cols > ((size_t)1 << 32) || b_rows * b_cols > ((size_t)1 << 34))
        return set_error(ZKML_ERR_INVALID_ARG, "matrix too large");
    if ((n_ri && !r_i) || (n_rj && !r_j)) return set_error(ZKML_ERR_INVALID_ARG, "NULL challenge point");
    if (n_rj > MAX_EQ_VARS || n_ri > MAX_EQ_VARS) return set_error(ZKML_ERR_INVALID_ARG, "too many variables");
    g_trace.mark("checks");
    ZK_CUDA(cudaSetDevice(ctx->device));
    g_trace.mark("setdev");
    const void* A = nullptr;
    const void* B = nullptr;
    int rc = device_view(ctx, a, a_rows * a_cols * 4, ctx->a_in, &A);
    g_trace.mark("viewA");
    if (!rc && !fb_words) rc = matrix_view(ctx, b, b_rows * b_cols, ctx->b_in, &B);
    if (rc) return rc;
    const uint32_t* Ad = static_cast<const uint32_t*>(A);
    const uint32_t* Bd = static_cast<const uint32_t*>(B);
    if (fb_words) {
        cudaPointerAttributes attr;
        if (cudaPointerGetAttributes(&attr, fb_words) != cudaSuccess || attr.type != cudaMemoryTypeDevice ||
            attr.device != ctx->device) {
            cudaGetLastError();
            return set_error(ZKML_ERR_INVALID_ARG, "f_b partial words must be device memory of the context's GPU");
        }
    }
    // Product sumcheck (1 x k times k x 1, k a power of two): stay in M31 for round 0.
    if (!fb_words && n_ri == 0 && n_rj == 0 && pk == a_cols && pk >= 4) {
        if ((rc = ctx->fa.ensure(pk / 2 * 16)) || (rc = ctx->fb.ensure(pk / 2 * 16))) return rc;
        return run_sumcheck(ctx, nullptr, nullptr, Ad, Bd, pk, ch, out_round_polys, out_challenges, out_final_a,
                            out_final_b, hook);
    }
    g_trace.mark("views");
    rc = restrict_ab(ctx, Ad, a_rows, a_cols, Bd, b_cols, reinterpret_cast<const qm31*>(r_i), (unsigned)n_ri,
                     reinterpret_cast<const qm31*>(r_j), (unsigned)n_rj, pk, fb_words);
    if (rc) return rc;
    g_trace.mark("restrict");
    rc = run_sumcheck(ctx, ctx->fa.as<uint4>(), ctx->fb.as<uint4>(), nullptr, nullptr, pk, ch, out_round_polys,
                      out_challenges, out_final_a, out_final_b, hook);
    if (rc) return rc;
    g_trace.mark("rounds");
    return check_err_flag(ctx, "reduce_matmul_layer");
}
}  // namespace zk

static int matmul_layer_gkr(zkml_ctx* ctx, const uint32_t* claim_point, size_t n_point,
                            const uint32_t claim_value[4], const uint32_t* a, size_t m, size_t k, const uint32_t* b,
                            size_t n, const uint64_t* fb_words, zkml_channel* chs, uint32_t* out_round_polys,
                            uint32_t out_final_a[4], uint32_t out_final_b[4], uint32_t* out_next_point) {
    if (!ctx || !claim_value || !chs || (n_point && !claim_point)) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    if (m == 0 || k == 0 || n == 0) return set_error(ZKML_ERR_INVALID_ARG, "empty matrix");
    const size_t pm = next_pow2(m), pk = next_pow2(k), pn = next_pow2(n);
    const unsigned log_m = ilog2(pm), log_n = ilog2(pn), log_k = ilog2(pk);
    if (n_point != log_m + log_n)
        return set_error(ZKML_ERR_INVALID_ARG, "output claim has " + std::to_string(n_point) +
                                                   " vars, expected exactly " + std::to_string(log_m + log_n));
    // Seeding mixes (gkr/prover.rs:5996-5999) run on the host while the GPU restricts.
    struct Seed {
        zkml_channel* ch;
        size_t m, k, n;
        const uint32_t* value;
    } seed{chs, m, k, n, claim_value};
    ClaimHook hook;
    hook.fn = nullptr;
    hook.arg = &seed;
    hook.overlap = [](void* arg) {
        Seed* sd = static_cast<Seed*>(arg);
        Channel c(sd->ch);
        c.mix_u64(sd->m);
        c.mix_u64(sd->k);
        c.mix_u64(sd->n);
        c.mix_qm31(ldq(sd->value));
    };
    std::vector<uint32_t> chal(4 * (log_k + 1));
    if (g_trace.on) la_stamps_enable(true);  // synchronous copies: before the timeline starts
    const uint32_t seq_lo = ctx->sig_seq + 1;
    g_trace.start();
    int rc = reduce_matmul_internal(ctx, a, m, k, b, k, n, claim_point, log_m, claim_point + 4 * log_m, log_n, pk,
                                    chs, out_round_polys, chal.data(), out_final_a, out_final_b, &hook, fb_words);
    if (rc) return rc;
    g_trace.mark("sumcheck");
    Channel ch(chs);
    ch.mix_qm31(ldq(out_final_a));
    ch.mix_qm31(ldq(out_final_b));
    g_trace.mark("final");
    g_trace.print();
    if (g_trace.on) la_stamps_print(seq_lo, ctx->sig_seq);
    if (out_next_point) {
        memcpy(out_next_point, claim_point, 16 * log_m);
        memcpy(out_next_point + 4 * log_m, chal.data(), 16 * log_k);
    }
    return ZKML_OK;
}

extern "C" {

int zkml_reduce_matmul_layer_gkr(zkml_ctx* ctx, const uint32_t* claim_point, size_t n_point,
                                 const uint32_t claim_value[4], const uint32_t* a, size_t m, size_t k,
                                 const uint32_t* b, size_t n, zkml_channel* chs, uint32_t* out_round_polys,
                                 uint32_t out_final_a[4], uint32_t out_final_b[4], uint32_t* out_next_point) {
    if (!b) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    return matmul_layer_gkr(ctx, claim_point, n_point, claim_value, a, m, k, b, n, nullptr, chs, out_round_polys,
                            out_final_a, out_final_b, out_next_point);
}

int zkml_reduce_matmul_layer_gkr_fb(zkml_ctx* ctx, const uint32_t* claim_point, size_t n_point,
                                    const uint32_t claim_value[4], const uint32_t* a, size_t m, size_t k,
                                    const uint64_t* fb_words, size_t n, zkml_channel* chs, uint32_t* out_round_polys,
                                    uint32_t out_final_a[4], uint32_t out_final_b[4], uint32_t* out_next_point) {
    if (!fb_words) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    return matmul_layer_gkr(ctx, claim_point, n_point, claim_value, a, m, k, nullptr, n, fb_words, chs,
                            out_round_polys, out_final_a, out_final_b, out_next_point);
}

int zkml_restrict_cols_block(zkml_ctx* ctx, const uint32_t* b_block, size_t k, size_t n_block, size_t col_offset,
                             const uint32_t* r_j, size_t n_rj, uint64_t* out_words) {
    if (!ctx || !b_block || !out_words || (n_rj && !r_j)) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    if (k == 0 || n_block == 0 || k > (1u << 30) || k * n_block > ((size_t)1 << 34))
        return set_error(ZKML_ERR_INVALID_ARG, "bad block shape");
    if (n_rj > MAX_EQ_VARS || col_offset + n_block > ((size_t)1 << n_rj))
        return set_error(ZKML_ERR_INVALID_ARG, "block exceeds the padded column space of r_j");
    if (col_offset % 64 != 0) return set_error(ZKML_ERR_INVALID_ARG, "col_offset must be a multiple of 64");
    ZK_CUDA(cudaSetDevice(ctx->device));
    cudaStream_t s = ctx->stream;
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, out_words) != cudaSuccess || attr.type != cudaMemoryTypeDevice ||
        attr.device != ctx->device) {
        cudaGetLastError();
        return set_error(ZKML_ERR_INVALID_ARG, "out_words must be device memory of the context's GPU");
    }
    const void* Bv = nullptr;
    int rc = device_view(ctx, b_block, k * n_block * 4, ctx->b_in, &Bv);
    if (rc) return rc;
    const uint32_t* B = static_cast<const uint32_t*>(Bv);
    // L_{col_offset + j} = eq_hi[(col_offset >> 6) + (j >> 6)] * eq_lo[j & 63]
    const unsigned lo_vars = n_rj < 6 ? (unsigned)n_rj : 6u;
    const unsigned hi_vars = (unsigned)n_rj - lo_vars;
    const qm31* rj = reinterpret_cast<const qm31*>(r_j);
    const bool tc = ctx->restrict_tc && restrict_cols_tc_ok(B, (uint32_t)n_block);
    if (!tc) {  // the tensor-pipe kernel forms its eq weights from r_j itself
        if ((rc = ctx->eq_hi.ensure(((size_t)16) << hi_vars)) || (rc = ctx->eq_lo.ensure(64 * 16))) return rc;
        launch_eq_table(rj, (int)hi_vars, ctx->eq_hi.as<uint4>(), (size_t)1 << hi_vars, s);
        launch_eq_table(rj + hi_vars, (int)lo_vars, ctx->eq_lo.as<uint4>(), 64, s);
        ctx->launches += 2;
    }
    unsigned long long* acc = reinterpret_cast<unsigned long long*>(out_words);
    ZK_CUDA(cudaMemsetAsync(acc, 0, k * 32, s));
    {
        KTimer t(ctx, KC_RESTRICT_COLS);
        if (tc)
            launch_restrict_cols_tc(B, (uint32_t)k, (uint32_t)n_block, rj, hi_vars, lo_vars,
                                    (uint32_t)(col_offset >> 6), acc, ctx->err_flag(), ctx->num_sms, s);
        else
            launch_restrict_cols(B, (uint32_t)k, (uint32_t)n_block, ctx->eq_hi.as<uint4>() + (col_offset >> 6),
                                 ctx->eq_lo.as<uint4>(), acc, ctx->err_flag(), ctx->num_sms, s);
    }
    // partial sums to canonical words (so that adding them across ranks cannot overflow)
    launch_canon_u64(acc, 4 * k, s);
    ctx->launches += 2;
    ZK_CUDA(cudaGetLastError());
    if ((rc = read_err_flag(ctx)) || (rc = check_err_flag(ctx, "restrict_cols_block"))) return rc;
    return ZKML_OK;
}

int zkml_evaluate_mle(zkml_ctx* ctx, const uint32_t* mle, size_t n_vars, const uint32_t* point, uint32_t out[4]) {
    if (!ctx || !mle || !out || (n_vars && !point)) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    if (n_vars > 34) return set_error(ZKML_ERR_INVALID_ARG, "too many variables");
    const size_t n = (size_t)1 << n_vars;
    if (n_vars == 0) {
        ZK_CUDA(cudaSetDevice(ctx->device));
        const void* M = nullptr;
        int rc = device_view(ctx, mle, 16, ctx->a_in, &M);
        if (rc) return rc;
        ZK_CUDA(cudaMemcpyAsync(out, M, 16, cudaMemcpyDeviceToHost, ctx->stream));
        ZK_CUDA(cudaStreamSynchronize(ctx->stream));
        return ZKML_OK;
    }
    int rc = ZKML_OK;
    ZK_CUDA(cudaSetDevice(ctx->device));
    const void* M = nullptr;
    if ((rc = device_view(ctx, mle, n * 16, ctx->a_in, &M))) return rc;
    if ((rc = ctx->fa.ensure(n / 2 * 16))) return rc;
    const qm31* pt = reinterpret_cast<const qm31*>(point);
    const uint4* src = static_cast<const uint4*>(M);
    size_t h = n / 2;
    for (size_t r = 0; r < n_vars; r++, h /= 2) {
        launch_mle_fold(src, ctx->fa.as<uint4>(), h, pt[r], ctx->stream);
        ctx->launches++;
        src = ctx->fa.as<uint4>();
    }
    ZK_CUDA(cudaMemcpyAsync(out, ctx->fa.ptr, 16, cudaMemcpyDeviceToHost, ctx->stream));
    ZK_CUDA(cudaStreamSynchronize(ctx->stream));
    return ZKML_OK;
}

int zkml_restrict_mle(zkml_ctx* ctx, const uint32_t* mle, size_t n_evals, const uint32_t* assign, size_t n_assign,
                      uint32_t* out) {
    if (!ctx || !mle || !out || (n_assign && !assign)) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    if (!is_pow2(n_evals) || ((size_t)1 << n_assign) > n_evals)
        return set_error(ZKML_ERR_INVALID_ARG, "n_evals must be a power of two >= 2^n_assign");
    ZK_CUDA(cudaSetDevice(ctx->device));
    const void* M = nullptr;
    int rc = device_view(ctx, mle, n_evals * 16, ctx->a_in, &M);
    if (rc) return rc;
    const size_t out_len = n_evals >> n_assign;
    if (n_assign == 0) {
        ZK_CUDA(cudaMemcpyAsync(out, M, n_evals * 16, cudaMemcpyDeviceToHost, ctx->stream));
        ZK_CUDA(cudaStreamSynchronize(ctx->stream));
        return ZKML_OK;
    }
    if ((rc = ctx->fa.ensure(n_evals / 2 * 16))) return rc;
    const qm31* pt = reinterpret_cast<const qm31*>(assign);
    const uint4* src = static_cast<const uint4*>(M);
    size_t h = n_evals / 2;
    for (size_t r = 0; r < n_assign; r++, h /= 2) {
        launch_mle_fold(src, ctx->fa.as<uint4>(), h, pt[r], ctx->stream);
        ctx->launches++;
        src = ctx->fa.as<uint4>();
    }
    ZK_CUDA(cudaMemcpyAsync(out, ctx->fa.ptr, out_len * 16, cudaMemcpyDeviceToHost, ctx->stream));
    ZK_CUDA(cudaStreamSynchronize(ctx->stream));
    return ZKML_OK;
}

}  // extern "C"
