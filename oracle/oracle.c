/*
 * CPU oracle: plain-C restatement of the stwo-ml CPU prover for the GKR
 * matmul-sumcheck path.  TEST INFRASTRUCTURE ONLY (see oracle.h): it is the
 * checker for the CUDA product and the CPU baseline of bench.py, never part
 * of the product.
 *
 * Third-party arithmetic restated here: starknet-crypto 0.6.2 / starknet-ff
 * 0.3.7 (engine/Cargo.toml:55-56), which the reference uses for felt252,
 * poseidon_permute_comp, poseidon_hash and poseidon_hash_many.  The published
 * Starknet Poseidon is restated from its definition: width 3, 4 full + 83
 * partial + 4 full rounds, each round = add the round's 3 keys, cube (all
 * three lanes in full rounds, lane 2 in partial rounds), then the MDS
 * [[3,1,1],[1,-1,1],[1,1,-2]].  The uncompressed 91 x 3 keys are used here on
 * purpose (the product uses its own compressed form), so the two
 * implementations check each other.
 */
#include "oracle.h"

#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* felt252: generic CIOS Montgomery over 4 x 64-bit limbs                   */
/* ------------------------------------------------------------------------ */

typedef unsigned __int128 u128;
typedef struct { uint64_t v[4]; } fe;

static const fe FE_P = {{1ULL, 0ULL, 0ULL, 0x0800000000000011ULL}};
static fe FE_R2;        /* R^2 mod p, R = 2^256 */
static fe FE_ONE_M;     /* R mod p */
static uint64_t FE_N0;  /* -p^{-1} mod 2^64 */
static fe RK_M[91][3];  /* round keys, Montgomery form */
static int g_init = 0;
static pthread_once_t g_once = PTHREAD_ONCE_INIT;

static const uint64_t RAW_RK[273][4] = {
#include "../stwo-ml_b200/csrc/poseidon3_round_keys.inc"
};

static int fe_geq(const fe *a, const fe *b) {
    for (int i = 3; i >= 0; i--) {
        if (a->v[i] != b->v[i]) return a->v[i] > b->v[i];
    }
    return 1;
}

static void fe_sub_raw(fe *r, const fe *a, const fe *b) {
    uint64_t borrow = 0;
    for (int i = 0; i < 4; i++) {
        u128 d = (u128)a->v[i] - b->v[i] - borrow;
        r->v[i] = (uint64_t)d;
        borrow = (uint64_t)(d >> 64) ? 1 : 0;
    }
}

static uint64_t fe_add_raw(fe *r, const fe *a, const fe *b) {
    uint64_t carry = 0;
    for (int i = 0; i < 4; i++) {
        u128 s = (u128)a->v[i] + b->v[i] + carry;
        r->v[i] = (uint64_t)s;
        carry = (uint64_t)(s >> 64);
    }
    return carry;
}

static void fe_add(fe *r, const fe *a, const fe *b) {
    fe t;
    fe_add_raw(&t, a, b); /* < 2p < 2^253: no carry out */
    if (fe_geq(&t, &FE_P)) fe_sub_raw(&t, &t, &FE_P);
    *r = t;
}

static void fe_sub(fe *r, const fe *a, const fe *b) {
    if (fe_geq(a, b)) {
        fe_sub_raw(r, a, b);
    } else {
        fe t;
        fe_add_raw(&t, a, &FE_P);
        fe_sub_raw(r, &t, b);
    }
}

/* Coarsely Integrated Operand Scanning Montgomery product a*b*R^-1 mod p. */
static void fe_mont_mul(fe *r, const fe *a, const fe *b) {
    uint64_t t[6] = {0, 0, 0, 0, 0, 0};
    for (int i = 0; i < 4; i++) {
        uint64_t c = 0;
        for (int j = 0; j < 4; j++) {
            u128 s = (u128)a->v[j] * b->v[i] + t[j] + c;
            t[j] = (uint64_t)s;
            c = (uint64_t)(s >> 64);
        }
        u128 s = (u128)t[4] + c;
        t[4] = (uint64_t)s;
        t[5] = (uint64_t)(s >> 64);
        uint64_t m = t[0] * FE_N0;
        s = (u128)m * FE_P.v[0] + t[0];
        c = (uint64_t)(s >> 64);
        for (int j = 1; j < 4; j++) {
            s = (u128)m * FE_P.v[j] + t[j] + c;
            t[j - 1] = (uint64_t)s;
            c = (uint64_t)(s >> 64);
        }
        s = (u128)t[4] + c;
        t[3] = (uint64_t)s;
        t[4] = t[5] + (uint64_t)(s >> 64);
    }
    fe res = {{t[0], t[1], t[2], t[3]}};
    if (t[4] || fe_geq(&res, &FE_P)) fe_sub_raw(&res, &res, &FE_P);
    *r = res;
}

static void fe_to_mont(fe *r, const fe *a) { fe_mont_mul(r, a, &FE_R2); }
static void fe_from_mont(fe *r, const fe *a) {
    fe one = {{1, 0, 0, 0}};
    fe_mont_mul(r, a, &one);
}

static void fe_from_canon(fe *r, const uint64_t v[4]) { memcpy(r->v, v, 32); }
static void fe_u64(fe *r, uint64_t x) {
    r->v[0] = x;
    r->v[1] = r->v[2] = r->v[3] = 0;
}

static void oracle_init_once(void) {
    /* n0 = -p^{-1} mod 2^64 by Newton iteration */
    uint64_t inv = 1;
    for (int i = 0; i < 7; i++) inv *= 2 - FE_P.v[0] * inv;
    FE_N0 = (uint64_t)0 - inv;
    /* R mod p and R^2 mod p by doubling */
    fe x;
    fe_u64(&x, 1);
    for (int i = 0; i < 512; i++) {
        if (i == 256) FE_ONE_M = x;
        fe y;
        fe_add(&y, &x, &x);
        x = y;
    }
    FE_R2 = x;
    for (int r = 0; r < 91; r++)
        for (int c = 0; c < 3; c++) {
            fe k;
            fe_from_canon(&k, RAW_RK[3 * r + c]);
            fe_to_mont(&RK_M[r][c], &k);
        }
    g_init = 1;
}

static void oracle_init(void) { pthread_once(&g_once, oracle_init_once); }

void orc_felt_mul(const uint64_t a[4], const uint64_t b[4], uint64_t out[4]) {
    oracle_init();
    fe x, y, xm, ym, r;
    fe_from_canon(&x, a);
    fe_from_canon(&y, b);
    fe_to_mont(&xm, &x);
    fe_to_mont(&ym, &y);
    fe_mont_mul(&r, &xm, &ym);
    fe_from_mont(&r, &r);
    memcpy(out, r.v, 32);
}

/* Hades permutation on Montgomery-form state. */
static void hades_m(fe s[3]) {
    for (int r = 0; r < 91; r++) {
        int full = (r < 4) || (r >= 87);
        for (int c = 0; c < 3; c++) fe_add(&s[c], &s[c], &RK_M[r][c]);
        for (int c = full ? 0 : 2; c < 3; c++) {
            fe sq;
            fe_mont_mul(&sq, &s[c], &s[c]);
            fe_mont_mul(&s[c], &sq, &s[c]);
        }
        /* MDS [[3,1,1],[1,-1,1],[1,1,-2]] */
        fe t, d0, d1, d2, a0, a1, a2;
        fe_add(&t, &s[0], &s[1]);
        fe_add(&t, &t, &s[2]);
        fe_add(&d0, &s[0], &s[0]);
        fe_add(&a0, &t, &d0);
        fe_add(&d1, &s[1], &s[1]);
        fe_sub(&a1, &t, &d1);
        fe_add(&d2, &s[2], &s[2]);
        fe_add(&d2, &d2, &s[2]);
        fe_sub(&a2, &t, &d2);
        s[0] = a0;
        s[1] = a1;
        s[2] = a2;
    }
}

static void hades_canon(fe s[3]) {
    fe m[3];
    for (int i = 0; i < 3; i++) fe_to_mont(&m[i], &s[i]);
    hades_m(m);
    for (int i = 0; i < 3; i++) fe_from_mont(&s[i], &m[i]);
}

void orc_hades(uint64_t state[12]) {
    oracle_init();
    fe s[3];
    for (int i = 0; i < 3; i++) fe_from_canon(&s[i], state + 4 * i);
    hades_canon(s);
    for (int i = 0; i < 3; i++) memcpy(state + 4 * i, s[i].v, 32);
}

static void pos_hash(fe *out, const fe *a, const fe *b) {
    fe s[3];
    s[0] = *a;
    s[1] = *b;
    fe_u64(&s[2], 2);
    hades_canon(s);
    *out = s[0];
}

void orc_poseidon_hash(const uint64_t a[4], const uint64_t b[4], uint64_t out[4]) {
    oracle_init();
    fe x, y, r;
    fe_from_canon(&x, a);
    fe_from_canon(&y, b);
    pos_hash(&r, &x, &y);
    memcpy(out, r.v, 32);
}

/* Rate-2 sponge with "1" padding (starknet_crypto::poseidon_hash_many). */
static void pos_hash_many(fe *out, const fe *in, size_t n) {
    fe s[3];
    fe_u64(&s[0], 0);
    fe_u64(&s[1], 0);
    fe_u64(&s[2], 0);
    size_t i = 0;
    while (n - i >= 2) {
        fe_add(&s[0], &s[0], &in[i]);
        fe_add(&s[1], &s[1], &in[i + 1]);
        hades_canon(s);
        i += 2;
    }
    fe one;
    fe_u64(&one, 1);
    if (n - i == 1) {
        fe_add(&s[0], &s[0], &in[i]);
        fe_add(&s[1], &s[1], &one);
    } else {
        fe_add(&s[0], &s[0], &one);
    }
    hades_canon(s);
    *out = s[0];
}

void orc_poseidon_hash_many(const uint64_t *in, size_t n, uint64_t out[4]) {
    oracle_init();
    fe *v = (fe *)malloc(sizeof(fe) * (n ? n : 1));
    for (size_t i = 0; i < n; i++) fe_from_canon(&v[i], in + 4 * i);
    fe r;
    pos_hash_many(&r, v, n);
    memcpy(out, r.v, 32);
    free(v);
}

/* ------------------------------------------------------------------------ */
/* M31 / CM31 / QM31 (stwo core/fields/{m31,cm31,qm31}.rs)                   */
/* ------------------------------------------------------------------------ */

#define MP 0x7fffffffu
typedef struct { uint32_t a, b, c, d; } q31;

static inline uint32_t m_red64(uint64_t x) {
    x = (x & MP) + (x >> 31);
    x = (x & MP) + (x >> 31);
    return (uint32_t)(x >= MP ? x - MP : x);
}
static inline uint32_t m_add(uint32_t x, uint32_t y) {
    uint32_t s = x + y;
    return s >= MP ? s - MP : s;
}
static inline uint32_t m_sub(uint32_t x, uint32_t y) { return x >= y ? x - y : x + MP - y; }
static inline uint32_t m_mul(uint32_t x, uint32_t y) { return m_red64((uint64_t)x * y); }
static uint32_t m_pow(uint32_t x, uint64_t e) {
    uint32_t r = 1;
    while (e) {
        if (e & 1) r = m_mul(r, x);
        x = m_mul(x, x);
        e >>= 1;
    }
    return r;
}
static inline uint32_t m_inv(uint32_t x) { return m_pow(x, MP - 2); }

static inline q31 q_make(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    q31 r = {a, b, c, d};
    return r;
}
static inline q31 q_from_m(uint32_t x) { return q_make(x, 0, 0, 0); }
static inline q31 q_add(q31 x, q31 y) {
    return q_make(m_add(x.a, y.a), m_add(x.b, y.b), m_add(x.c, y.c), m_add(x.d, y.d));
}
static inline q31 q_sub(q31 x, q31 y) {
    return q_make(m_sub(x.a, y.a), m_sub(x.b, y.b), m_sub(x.c, y.c), m_sub(x.d, y.d));
}
/* (x0 + x1 i)(y0 + y1 i) */
static inline void cm_mul(uint32_t x0, uint32_t x1, uint32_t y0, uint32_t y1, uint32_t *r0,
                          uint32_t *r1) {
    *r0 = m_sub(m_mul(x0, y0), m_mul(x1, y1));
    *r1 = m_add(m_mul(x0, y1), m_mul(x1, y0));
}
/* (a + b u)(c + d u) = (ac + R bd) + (ad + bc) u, R = 2 + i */
static q31 q_mul(q31 x, q31 y) {
    uint32_t ac0, ac1, bd0, bd1, ad0, ad1, bc0, bc1, rb0, rb1;
    cm_mul(x.a, x.b, y.a, y.b, &ac0, &ac1);
    cm_mul(x.c, x.d, y.c, y.d, &bd0, &bd1);
    cm_mul(x.a, x.b, y.c, y.d, &ad0, &ad1);
    cm_mul(x.c, x.d, y.a, y.b, &bc0, &bc1);
    cm_mul(2, 1, bd0, bd1, &rb0, &rb1);
    return q_make(m_add(ac0, rb0), m_add(ac1, rb1), m_add(ad0, bc0), m_add(ad1, bc1));
}
static inline q31 q_mul_m(q31 x, uint32_t s) {
    return q_make(m_mul(x.a, s), m_mul(x.b, s), m_mul(x.c, s), m_mul(x.d, s));
}
static q31 q_inv(q31 x) {
    /* (a + b u)^-1 = (a - b u) / (a^2 - R b^2), all in CM31 */
    uint32_t a2r, a2i, b2r, b2i, rb0, rb1;
    cm_mul(x.a, x.b, x.a, x.b, &a2r, &a2i);
    cm_mul(x.c, x.d, x.c, x.d, &b2r, &b2i);
    cm_mul(2, 1, b2r, b2i, &rb0, &rb1);
    uint32_t den0 = m_sub(a2r, rb0), den1 = m_sub(a2i, rb1);
    uint32_t nrm = m_inv(m_add(m_mul(den0, den0), m_mul(den1, den1)));
    uint32_t inv0 = m_mul(den0, nrm), inv1 = m_mul(m_sub(0, den1), nrm);
    uint32_t r0, r1, r2, r3;
    cm_mul(x.a, x.b, inv0, inv1, &r0, &r1);
    cm_mul(m_sub(0, x.c), m_sub(0, x.d), inv0, inv1, &r2, &r3);
    return q_make(r0, r1, r2, r3);
}
static inline int q_eq(q31 x, q31 y) { return x.a == y.a && x.b == y.b && x.c == y.c && x.d == y.d; }
static inline q31 q_load(const uint32_t *p) { return q_make(p[0], p[1], p[2], p[3]); }
static inline void q_store(uint32_t *p, q31 x) {
    p[0] = x.a;
    p[1] = x.b;
    p[2] = x.c;
    p[3] = x.d;
}

void orc_qm31_mul(const uint32_t a[4], const uint32_t b[4], uint32_t out[4]) {
    q_store(out, q_mul(q_load(a), q_load(b)));
}
void orc_qm31_inv(const uint32_t a[4], uint32_t out[4]) { q_store(out, q_inv(q_load(a))); }

/* ------------------------------------------------------------------------ */
/* Tiny pthread parallel-for (stands in for the reference's rayon pools)     */
/* ------------------------------------------------------------------------ */

typedef void (*range_fn)(void *ctx, size_t lo, size_t hi);
typedef struct {
    range_fn fn;
    void *ctx;
    size_t lo, hi;
} par_job;

static void *par_worker(void *p) {
    par_job *j = (par_job *)p;
    j->fn(j->ctx, j->lo, j->hi);
    return NULL;
}

static void parallel_for(size_t n, int threads, range_fn fn, void *ctx) {
    if (threads <= 1 || n < 2) {
        fn(ctx, 0, n);
        return;
    }
    if ((size_t)threads > n) threads = (int)n;
    pthread_t tid[256];
    par_job jobs[256];
    if (threads > 256) threads = 256;
    size_t chunk = (n + threads - 1) / threads;
    int launched = 0;
    jobs[0].lo = 0;
    jobs[0].hi = chunk < n ? chunk : n;
    for (int t = 0; t < threads; t++) {
        size_t lo = t * chunk, hi = lo + chunk > n ? n : lo + chunk;
        if (lo >= hi) break;
        jobs[t].fn = fn;
        jobs[t].ctx = ctx;
        jobs[t].lo = lo;
        jobs[t].hi = hi;
        if (t == 0) continue;
        pthread_create(&tid[t], NULL, par_worker, &jobs[t]);
        launched = t;
    }
    fn(ctx, jobs[0].lo, jobs[0].hi);
    for (int t = 1; t <= launched; t++) pthread_join(tid[t], NULL);
}

/* ------------------------------------------------------------------------ */
/* PoseidonChannel (engine/src/crypto/poseidon_channel.rs:83-306)            */
/* ------------------------------------------------------------------------ */

static void felt_of_qm31(fe *r, q31 v) {
    /* securefield_to_felt: 2^124 sentinel | a<<93 | b<<62 | c<<31 | d */
    u128 lo = ((u128)1 << 124) | ((u128)v.a << 93) | ((u128)v.b << 62) | ((u128)v.c << 31) | v.d;
    r->v[0] = (uint64_t)lo;
    r->v[1] = (uint64_t)(lo >> 64);
    r->v[2] = r->v[3] = 0;
}

void orc_securefield_to_felt(const uint32_t v[4], uint64_t out[4]) {
    fe r;
    felt_of_qm31(&r, q_load(v));
    memcpy(out, r.v, 32);
}

/* pack_m31s: acc = 1; acc = acc * 2^31 + m (never wraps for <= 8 values) */
static void pack_m31s(fe *r, const uint32_t *m, size_t cnt) {
    fe acc;
    fe_u64(&acc, 1);
    for (size_t i = 0; i < cnt; i++) {
        /* shift left by 31 */
        uint64_t nv[4];
        nv[3] = (acc.v[3] << 31) | (acc.v[2] >> 33);
        nv[2] = (acc.v[2] << 31) | (acc.v[1] >> 33);
        nv[1] = (acc.v[1] << 31) | (acc.v[0] >> 33);
        nv[0] = (acc.v[0] << 31) | m[i];
        memcpy(acc.v, nv, 32);
    }
    *r = acc;
}

void orc_ch_init(orc_channel *ch) { memset(ch, 0, sizeof(*ch)); }

static void ch_mix(orc_channel *ch, const fe *v) {
    oracle_init();
    fe s[3];
    fe_from_canon(&s[0], ch->digest);
    s[1] = *v;
    fe_u64(&s[2], 2);
    hades_canon(s);
    memcpy(ch->digest, s[0].v, 32);
    ch->n_draws = 0;
    ch->hash_count++;
}

void orc_ch_mix_u64(orc_channel *ch, uint64_t v) {
    fe f;
    fe_u64(&f, v);
    ch_mix(ch, &f);
}

void orc_ch_mix_felt(orc_channel *ch, const uint64_t v[4]) {
    fe f;
    fe_from_canon(&f, v);
    ch_mix(ch, &f);
}

static void ch_draw(orc_channel *ch, fe *out) {
    oracle_init();
    fe s[3];
    fe_from_canon(&s[0], ch->digest);
    fe_u64(&s[1], ch->n_draws);
    fe_u64(&s[2], 3);
    hades_canon(s);
    ch->n_draws++;
    ch->hash_count++;
    *out = s[0];
}

void orc_ch_draw_felt(orc_channel *ch, uint64_t out[4]) {
    fe f;
    ch_draw(ch, &f);
    memcpy(out, f.v, 32);
}

static q31 ch_draw_qm31(orc_channel *ch) {
    fe f;
    ch_draw(ch, &f);
    uint32_t m[4];
    for (int i = 0; i < 4; i++) {
        /* remainder mod 2^31, reduced mod P; then floor-divide by 2^31 */
        uint32_t rem = (uint32_t)(f.v[0] & 0x7fffffffu);
        m[i] = rem % MP;
        f.v[0] = (f.v[0] >> 31) | (f.v[1] << 33);
        f.v[1] = (f.v[1] >> 31) | (f.v[2] << 33);
        f.v[2] = (f.v[2] >> 31) | (f.v[3] << 33);
        f.v[3] = f.v[3] >> 31;
    }
    return q_make(m[0], m[1], m[2], m[3]);
}

void orc_ch_draw_qm31(orc_channel *ch, uint32_t out[4]) { q_store(out, ch_draw_qm31(ch)); }

static void ch_digest_hash_many(orc_channel *ch, const fe *tail, size_t n_tail) {
    fe buf[64];
    fe *in = n_tail + 1 <= 64 ? buf : (fe *)malloc(sizeof(fe) * (n_tail + 1));
    fe_from_canon(&in[0], ch->digest);
    for (size_t i = 0; i < n_tail; i++) in[i + 1] = tail[i];
    fe r;
    pos_hash_many(&r, in, n_tail + 1);
    memcpy(ch->digest, r.v, 32);
    ch->n_draws = 0;
    ch->hash_count++;
    if (in != buf) free(in);
}

void orc_ch_mix_poly_coeffs(orc_channel *ch, const uint32_t c[12]) {
    oracle_init();
    fe t[2];
    pack_m31s(&t[0], c, 8);
    pack_m31s(&t[1], c + 8, 4);
    ch_digest_hash_many(ch, t, 2);
}

void orc_ch_mix_poly_coeffs_deg3(orc_channel *ch, const uint32_t c[16]) {
    oracle_init();
    fe t[2];
    pack_m31s(&t[0], c, 8);
    pack_m31s(&t[1], c + 8, 8);
    ch_digest_hash_many(ch, t, 2);
}

void orc_ch_mix_felts(orc_channel *ch, const uint32_t *qm31s, size_t n) {
    oracle_init();
    if (n == 0) return;
    size_t nt = (n + 1) / 2;
    fe *t = (fe *)malloc(sizeof(fe) * nt);
    for (size_t i = 0, o = 0; i < n; i += 2, o++) pack_m31s(&t[o], qm31s + 4 * i, (n - i >= 2) ? 8 : 4);
    ch_digest_hash_many(ch, t, nt);
    free(t);
}

static void ch_mix_sf(orc_channel *ch, q31 v) {
    fe f;
    felt_of_qm31(&f, v);
    ch_mix(ch, &f);
}

/* ------------------------------------------------------------------------ */
/* MLE helpers (components/matmul.rs:118-356)                                */
/* ------------------------------------------------------------------------ */

static size_t next_pow2(size_t x) {
    size_t p = 1;
    while (p < x) p <<= 1;
    return p;
}
static unsigned ilog2(size_t x) {
    unsigned l = 0;
    while (((size_t)1 << (l + 1)) <= x) l++;
    return l;
}

/* compute_lagrange_basis: each challenge doubles the table as [w(1-c), w c],
 * so challenge 0 ends up on the most significant index bit. */
static q31 *lagrange_basis(const q31 *c, size_t v) {
    size_t n = (size_t)1 << v;
    q31 *w = (q31 *)malloc(sizeof(q31) * n);
    w[0] = q_from_m(1);
    size_t len = 1;
    for (size_t l = 0; l < v; l++) {
        q31 one_minus = q_sub(q_from_m(1), c[l]);
        for (size_t i = len; i-- > 0;) {
            q31 x = w[i];
            w[2 * i] = q_mul(x, one_minus);
            w[2 * i + 1] = q_mul(x, c[l]);
        }
        len *= 2;
    }
    return w;
}

void orc_lagrange_basis(const uint32_t *challenges, size_t v, uint32_t *out) {
    q31 *w = lagrange_basis((const q31 *)challenges, v);
    memcpy(out, w, sizeof(q31) << v);
    free(w);
}

typedef struct {
    q31 *cur;
    size_t mid;
    q31 r;
} fold_ctx;

static void fold_range(void *p, size_t lo, size_t hi) {
    fold_ctx *f = (fold_ctx *)p;
    for (size_t i = lo; i < hi; i++)
        f->cur[i] = q_add(f->cur[i], q_mul(f->r, q_sub(f->cur[f->mid + i], f->cur[i])));
}

/* restrict_mle: in-place folds, first assignment = most significant variable;
 * parallel when mid >= 8192 (matmul.rs:144-168). */
static void restrict_inplace(q31 *cur, size_t size, const q31 *assign, size_t n_assign, int threads) {
    for (size_t t = 0; t < n_assign; t++) {
        size_t mid = size / 2;
        fold_ctx f = {cur, mid, assign[t]};
        parallel_for(mid, mid >= 8192 ? threads : 1, fold_range, &f);
        size = mid;
    }
}

void orc_restrict_mle(const uint32_t *evals, size_t n_evals, const uint32_t *assign, size_t n_assign,
                      uint32_t *out) {
    q31 *cur = (q31 *)malloc(sizeof(q31) * n_evals);
    memcpy(cur, evals, sizeof(q31) * n_evals);
    restrict_inplace(cur, n_evals, (const q31 *)assign, n_assign, 1);
    memcpy(out, cur, sizeof(q31) * (n_evals >> n_assign));
    free(cur);
}

void orc_evaluate_mle(const uint32_t *evals, size_t n_vars, const uint32_t *point, uint32_t out[4]) {
    size_t n = (size_t)1 << n_vars;
    q31 *cur = (q31 *)malloc(sizeof(q31) * n);
    memcpy(cur, evals, sizeof(q31) * n);
    restrict_inplace(cur, n, (const q31 *)point, n_vars, 1);
    q_store(out, cur[0]);
    free(cur);
}

/* ------------------------------------------------------------------------ */
/* reduce_matmul_layer (backend.rs:110-197)                                  */
/* ------------------------------------------------------------------------ */

typedef struct {
    const uint32_t *mat;
    size_t rows, cols, out_len;
    const q31 *lag;
    q31 *out;
} restrict_ctx;

/* restrict_cols_unpadded: f_b[i] = sum_{j < cols} B[i][j] * L_j */
static void rcols_range(void *p, size_t lo, size_t hi) {
    restrict_ctx *c = (restrict_ctx *)p;
    for (size_t i = lo; i < hi; i++) {
        q31 s = q_from_m(0);
        const uint32_t *row = c->mat + i * c->cols;
        for (size_t j = 0; j < c->cols; j++) s = q_add(s, q_mul_m(c->lag[j], row[j]));
        c->out[i] = s;
    }
}

/* restrict_rows_unpadded: f_a[j] = sum_{i < rows} A[i][j] * L_i */
static void rrows_range(void *p, size_t lo, size_t hi) {
    restrict_ctx *c = (restrict_ctx *)p;
    for (size_t j = lo; j < hi; j++) {
        q31 s = q_from_m(0);
        for (size_t i = 0; i < c->rows; i++) s = q_add(s, q_mul_m(c->lag[i], c->mat[i * c->cols + j]));
        c->out[j] = s;
    }
}

typedef struct {
    const uint32_t *mat;
    size_t rows, cols, prows, pcols;
    q31 *mle;
    int col_major;
} mle_ctx;

/* matrix_to_mle (row-major) / matrix_to_mle_col_major on the padded matrix */
static void mle_range(void *p, size_t lo, size_t hi) {
    mle_ctx *c = (mle_ctx *)p;
    if (!c->col_major) {
        for (size_t i = lo; i < hi; i++)
            for (size_t j = 0; j < c->pcols; j++)
                c->mle[i * c->pcols + j] =
                    (i < c->rows && j < c->cols) ? q_from_m(c->mat[i * c->cols + j]) : q_from_m(0);
    } else {
        for (size_t j = lo; j < hi; j++)
            for (size_t i = 0; i < c->prows; i++)
                c->mle[j * c->prows + i] =
                    (i < c->rows && j < c->cols) ? q_from_m(c->mat[i * c->cols + j]) : q_from_m(0);
    }
}

static void restrict_a(const uint32_t *a, size_t m, size_t k, const q31 *r_i, size_t n_ri, size_t pk,
                       q31 *f_a, int mode, int threads) {
    size_t pm = next_pow2(m);
    if (mode == 0) {
        q31 *mle = (q31 *)malloc(sizeof(q31) * pm * pk);
        mle_ctx mc = {a, m, k, pm, pk, mle, 0};
        parallel_for(pm, pm * pk >= 65536 ? threads : 1, mle_range, &mc);
        restrict_inplace(mle, pm * pk, r_i, n_ri, threads);
        memcpy(f_a, mle, sizeof(q31) * pk);
        free(mle);
    } else {
        q31 *lag = lagrange_basis(r_i, n_ri);
        restrict_ctx rc = {a, m, k, pk, lag, f_a};
        for (size_t j = k; j < pk; j++) f_a[j] = q_from_m(0);
        parallel_for(k, k >= 64 ? threads : 1, rrows_range, &rc);
        free(lag);
    }
}

static void restrict_b(const uint32_t *b, size_t k, size_t n, const q31 *r_j, size_t n_rj, size_t pk,
                       q31 *f_b, int mode, int threads) {
    size_t pn = next_pow2(n);
    if (mode == 0) {
        q31 *mle = (q31 *)malloc(sizeof(q31) * pn * pk);
        mle_ctx mc = {b, k, n, pk, pn, mle, 1};
        parallel_for(pn, pn * pk >= 65536 ? threads : 1, mle_range, &mc);
        restrict_inplace(mle, pn * pk, r_j, n_rj, threads);
        memcpy(f_b, mle, sizeof(q31) * pk);
        free(mle);
    } else {
        q31 *lag = lagrange_basis(r_j, n_rj);
        restrict_ctx rc = {b, k, n, pk, lag, f_b};
        for (size_t i = k; i < pk; i++) f_b[i] = q_from_m(0);
        parallel_for(k, k >= 64 ? threads : 1, rcols_range, &rc);
        free(lag);
    }
}

static void sumcheck_rounds(q31 *fa, q31 *fb, size_t pk, orc_channel *ch, uint32_t *out_rp,
                            uint32_t *out_ch, q31 *fa_out, q31 *fb_out) {
    q31 inv2 = q_from_m(m_inv(2));
    size_t len = pk;
    unsigned log_k = ilog2(pk);
    for (unsigned r = 0; r < log_k; r++) {
        size_t mid = len / 2;
        q31 s0 = q_from_m(0), s1 = s0, s2 = s0;
        for (size_t i = 0; i < mid; i++) {
            s0 = q_add(s0, q_mul(fa[i], fb[i]));
            s1 = q_add(s1, q_mul(fa[mid + i], fb[mid + i]));
            q31 a2 = q_sub(q_add(fa[mid + i], fa[mid + i]), fa[i]);
            q31 b2 = q_sub(q_add(fb[mid + i], fb[mid + i]), fb[i]);
            s2 = q_add(s2, q_mul(a2, b2));
        }
        q31 c0 = s0;
        q31 c2 = q_mul(q_add(q_sub(q_sub(s2, s1), s1), s0), inv2);
        q31 c1 = q_sub(q_sub(s1, s0), c2);
        uint32_t coeffs[12];
        q_store(coeffs, c0);
        q_store(coeffs + 4, c1);
        q_store(coeffs + 8, c2);
        if (out_rp) memcpy(out_rp + 12 * r, coeffs, sizeof(coeffs));
        orc_ch_mix_poly_coeffs(ch, coeffs);
        q31 alpha = ch_draw_qm31(ch);
        if (out_ch) q_store(out_ch + 4 * r, alpha);
        for (size_t i = 0; i < mid; i++) {
            fa[i] = q_add(fa[i], q_mul(alpha, q_sub(fa[mid + i], fa[i])));
            fb[i] = q_add(fb[i], q_mul(alpha, q_sub(fb[mid + i], fb[i])));
        }
        len = mid;
    }
    *fa_out = len ? fa[0] : q_from_m(0);
    *fb_out = len ? fb[0] : q_from_m(0);
}

int orc_reduce_matmul_layer(const uint32_t *a, size_t a_rows, size_t a_cols, const uint32_t *b,
                            size_t b_rows, size_t b_cols, const uint32_t *r_i, size_t n_ri,
                            const uint32_t *r_j, size_t n_rj, size_t pk, orc_channel *ch,
                            uint32_t *out_round_polys, uint32_t *out_challenges,
                            uint32_t out_final_a[4], uint32_t out_final_b[4], int mode, int threads) {
    oracle_init();
    if (a_cols != b_rows || pk != next_pow2(a_cols) || next_pow2(a_rows) != ((size_t)1 << n_ri) ||
        next_pow2(b_cols) != ((size_t)1 << n_rj))
        return 1;
    q31 *fa = (q31 *)malloc(sizeof(q31) * pk);
    q31 *fb = (q31 *)malloc(sizeof(q31) * pk);
    restrict_a(a, a_rows, a_cols, (const q31 *)r_i, n_ri, pk, fa, mode, threads);
    restrict_b(b, b_rows, b_cols, (const q31 *)r_j, n_rj, pk, fb, mode, threads);
    q31 xa, xb;
    sumcheck_rounds(fa, fb, pk, ch, out_round_polys, out_challenges, &xa, &xb);
    q_store(out_final_a, xa);
    q_store(out_final_b, xb);
    free(fa);
    free(fb);
    return 0;
}

int orc_reduce_matmul_gkr(const uint32_t *claim_point, size_t n_point, const uint32_t claim_value[4],
                          const uint32_t *a, size_t m, size_t k, const uint32_t *b, size_t n,
                          orc_channel *ch, uint32_t *out_round_polys, uint32_t out_final_a[4],
                          uint32_t out_final_b[4], uint32_t *next_point, int mode, int threads) {
    size_t pm = next_pow2(m), pk = next_pow2(k), pn = next_pow2(n);
    unsigned log_m = ilog2(pm), log_n = ilog2(pn), log_k = ilog2(pk);
    if (n_point != log_m + log_n) return 1;
    orc_ch_mix_u64(ch, m);
    orc_ch_mix_u64(ch, k);
    orc_ch_mix_u64(ch, n);
    ch_mix_sf(ch, q_load(claim_value));
    uint32_t *chal = (uint32_t *)malloc(16 * (log_k + 1));
    int rc = orc_reduce_matmul_layer(a, m, k, b, k, n, claim_point, log_m, claim_point + 4 * log_m, log_n,
                                     pk, ch, out_round_polys, chal, out_final_a, out_final_b, mode, threads);
    if (rc) {
        free(chal);
        return rc;
    }
    ch_mix_sf(ch, q_load(out_final_a));
    ch_mix_sf(ch, q_load(out_final_b));
    if (next_point) {
        memcpy(next_point, claim_point, 16 * log_m);
        memcpy(next_point + 4 * log_m, chal, 16 * log_k);
    }
    free(chal);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Poseidon Merkle (crypto/poseidon_merkle.rs)                               */
/* ------------------------------------------------------------------------ */

typedef struct {
    const fe *in;
    fe *out;
} layer_ctx;

static void layer_range(void *p, size_t lo, size_t hi) {
    layer_ctx *c = (layer_ctx *)p;
    for (size_t i = lo; i < hi; i++) pos_hash(&c->out[i], &c->in[2 * i], &c->in[2 * i + 1]);
}

/* Builds all layers; layer l has (padded n) >> l nodes.  Returns the layer
 * array (caller frees each and the array) and the number of layers. */
static fe **merkle_build(const q31 *evals, size_t n, size_t *n_layers, int threads) {
    size_t pn = next_pow2(n);
    if (pn < 2) pn = 2;
    size_t L = ilog2(pn) + 1;
    fe **layers = (fe **)malloc(sizeof(fe *) * L);
    layers[0] = (fe *)calloc(pn, sizeof(fe));
    for (size_t i = 0; i < n; i++) felt_of_qm31(&layers[0][i], evals[i]);
    size_t len = pn;
    for (size_t l = 1; l < L; l++) {
        size_t pairs = len / 2;
        layers[l] = (fe *)malloc(sizeof(fe) * pairs);
        layer_ctx c = {layers[l - 1], layers[l]};
        parallel_for(pairs, pairs >= 256 ? threads : 1, layer_range, &c);
        len = pairs;
    }
    *n_layers = L;
    return layers;
}

static void merkle_free(fe **layers, size_t L) {
    for (size_t l = 0; l < L; l++) free(layers[l]);
    free(layers);
}

/* root_only_parallel: keeps one layer at a time */
static void merkle_root(const q31 *evals, size_t n, fe *root, int threads) {
    size_t pn = next_pow2(n);
    if (pn < 2) pn = 2;
    fe *cur = (fe *)calloc(pn, sizeof(fe));
    for (size_t i = 0; i < n; i++) felt_of_qm31(&cur[i], evals[i]);
    size_t len = pn;
    while (len > 1) {
        size_t pairs = len / 2;
        fe *nxt = (fe *)malloc(sizeof(fe) * pairs);
        layer_ctx c = {cur, nxt};
        parallel_for(pairs, pairs >= 256 ? threads : 1, layer_range, &c);
        free(cur);
        cur = nxt;
        len = pairs;
    }
    *root = cur[0];
    free(cur);
}

void orc_merkle_root_qm31(const uint32_t *evals, size_t n, uint64_t out[4], int threads) {
    oracle_init();
    fe r;
    merkle_root((const q31 *)evals, n, &r, threads);
    memcpy(out, r.v, 32);
}

void orc_merkle_path_qm31(const uint32_t *evals, size_t n, size_t index, uint64_t *out, int threads) {
    oracle_init();
    size_t L;
    fe **layers = merkle_build((const q31 *)evals, n, &L, threads);
    size_t idx = index;
    for (size_t l = 0; l + 1 < L; l++) {
        memcpy(out + 4 * l, layers[l][idx ^ 1].v, 32);
        idx >>= 1;
    }
    merkle_free(layers, L);
}

int orc_merkle_verify(const uint64_t root[4], size_t index, const uint64_t leaf[4],
                      const uint64_t *siblings, size_t n_siblings) {
    oracle_init();
    fe cur, sib;
    fe_from_canon(&cur, leaf);
    size_t idx = index;
    for (size_t l = 0; l < n_siblings; l++) {
        fe_from_canon(&sib, siblings + 4 * l);
        if (idx & 1)
            pos_hash(&cur, &sib, &cur);
        else
            pos_hash(&cur, &cur, &sib);
        idx >>= 1;
    }
    return memcmp(cur.v, root, 32) == 0;
}

/* ------------------------------------------------------------------------ */
/* MLE opening (crypto/mle_opening.rs:1654-2029)                             */
/* ------------------------------------------------------------------------ */

typedef struct {
    uint64_t *buf;
    size_t len, cap;
    int overflow;
} felt_out;

static void out_push(felt_out *o, const fe *f) {
    if (o->len >= o->cap) {
        o->overflow = 1;
        o->len++;
        return;
    }
    memcpy(o->buf + 4 * o->len, f->v, 32);
    o->len++;
}
static void out_u64(felt_out *o, uint64_t x) {
    fe f;
    fe_u64(&f, x);
    out_push(o, &f);
}
static void out_qm31(felt_out *o, q31 v) {
    out_u64(o, v.a);
    out_u64(o, v.b);
    out_u64(o, v.c);
    out_u64(o, v.d);
}

static int prove_opening(const q31 *evals, size_t n_vars, const q31 *point, orc_channel *ch,
                         size_t n_queries_cfg, fe *commitment, felt_out *o, q31 *final_out, int threads) {
    size_t n = (size_t)1 << n_vars;
    q31 **lay = (q31 **)malloc(sizeof(q31 *) * (n_vars + 1));
    lay[0] = (q31 *)malloc(sizeof(q31) * n);
    memcpy(lay[0], evals, sizeof(q31) * n);
    fe root;
    merkle_root(lay[0], n, &root, threads);
    ch_mix(ch, &root);
    *commitment = root;
    fe *inter = (fe *)malloc(sizeof(fe) * (n_vars + 1));
    size_t n_inter = 0;
    size_t len = n;
    for (size_t r = 0; r < n_vars; r++) {
        size_t mid = len / 2;
        lay[r + 1] = (q31 *)malloc(sizeof(q31) * mid);
        for (size_t j = 0; j < mid; j++)
            lay[r + 1][j] = q_add(lay[r][j], q_mul(point[r], q_sub(lay[r][mid + j], lay[r][j])));
        if (mid > 1) {
            fe rt;
            merkle_root(lay[r + 1], mid, &rt, threads);
            ch_mix(ch, &rt);
            inter[n_inter++] = rt;
        }
        len = mid;
    }
    q31 final_value = lay[n_vars][0];
    size_t half_n = n / 2;
    size_t nq = n_queries_cfg < half_n ? n_queries_cfg : half_n;
    size_t *qidx = (size_t *)malloc(sizeof(size_t) * (nq + 1));
    for (size_t q = 0; q < nq; q++) {
        fe f;
        ch_draw(ch, &f);
        qidx[q] = (size_t)(f.v[0] % half_n);
    }
    /* serialize: intermediate roots, queries, final value */
    out_u64(o, n_inter);
    for (size_t i = 0; i < n_inter; i++) out_push(o, &inter[i]);
    out_u64(o, nq);
    /* build each round's tree once; serialization is query-major, so keep trees */
    size_t *nl = (size_t *)malloc(sizeof(size_t) * n_vars);
    fe ***trees = (fe ***)malloc(sizeof(fe **) * n_vars);
    len = n;
    for (size_t r = 0; r < n_vars; r++) {
        trees[r] = merkle_build(lay[r], len, &nl[r], threads);
        len /= 2;
    }
    for (size_t q = 0; q < nq; q++) {
        out_u64(o, qidx[q]);
        out_u64(o, n_vars);
        size_t idx = qidx[q];
        len = n;
        for (size_t r = 0; r < n_vars; r++) {
            size_t mid = len / 2;
            size_t li = idx, ri = mid + idx;
            out_qm31(o, lay[r][li]);
            out_qm31(o, lay[r][ri]);
            size_t sides[2] = {li, ri};
            for (int s = 0; s < 2; s++) {
                out_u64(o, nl[r] - 1);
                size_t x = sides[s];
                for (size_t l = 0; l + 1 < nl[r]; l++) {
                    out_push(o, &trees[r][l][x ^ 1]);
                    x >>= 1;
                }
            }
            size_t next_half = mid / 2 > 0 ? mid / 2 : 1;
            idx %= next_half;
            len = mid;
        }
    }
    out_qm31(o, final_value);
    if (final_out) *final_out = final_value;
    for (size_t r = 0; r < n_vars; r++) merkle_free(trees[r], nl[r]);
    free(trees);
    free(nl);
    free(qidx);
    free(inter);
    for (size_t r = 0; r <= n_vars; r++) free(lay[r]);
    free(lay);
    return 0;
}

int orc_prove_mle_opening(const uint32_t *evals, size_t n_vars, const uint32_t *point, orc_channel *ch,
                          size_t n_queries, uint64_t commitment[4], uint64_t *calldata, size_t cap,
                          size_t *out_len, int threads) {
    oracle_init();
    felt_out o = {calldata, 0, cap, 0};
    fe c;
    prove_opening((const q31 *)evals, n_vars, (const q31 *)point, ch, n_queries, &c, &o, NULL, threads);
    memcpy(commitment, c.v, 32);
    *out_len = o.len;
    return o.overflow ? 2 : 0;
}

/* Calldata reader */
typedef struct {
    const uint64_t *buf;
    size_t len, pos;
    int bad;
} felt_in;

static int in_felt(felt_in *in, fe *f) {
    if (in->pos >= in->len) {
        in->bad = 1;
        fe_u64(f, 0);
        return 0;
    }
    fe_from_canon(f, in->buf + 4 * in->pos);
    in->pos++;
    return 1;
}
static uint64_t in_u64(felt_in *in) {
    fe f;
    in_felt(in, &f);
    if (f.v[1] || f.v[2] || f.v[3]) in->bad = 1;
    return f.v[0];
}
static q31 in_qm31(felt_in *in) {
    uint64_t a = in_u64(in), b = in_u64(in), c = in_u64(in), d = in_u64(in);
    if (a >= MP || b >= MP || c >= MP || d >= MP) in->bad = 1;
    return q_make((uint32_t)a, (uint32_t)b, (uint32_t)c, (uint32_t)d);
}

static int verify_opening(const fe *commitment, felt_in *in, const q31 *point, size_t n_rounds,
                          orc_channel *ch, size_t n_queries_cfg, q31 *final_out) {
    size_t n_inter = in_u64(in);
    if (in->bad || n_inter > 64) return 0;
    fe inter[64];
    for (size_t i = 0; i < n_inter; i++) in_felt(in, &inter[i]);
    ch_mix(ch, commitment);
    for (size_t i = 0; i < n_inter; i++) ch_mix(ch, &inter[i]);
    size_t nq = in_u64(in);
    if (n_rounds == 0) {
        q31 fv = in_qm31(in);
        if (final_out) *final_out = fv;
        return nq == 0 && !in->bad;
    }
    size_t half_n = (size_t)1 << (n_rounds - 1);
    size_t exp_q = n_queries_cfg < half_n ? n_queries_cfg : half_n;
    if (nq != exp_q) return 0;
    size_t qidx[64];
    if (nq > 64) return 0;
    for (size_t q = 0; q < nq; q++) {
        fe f;
        ch_draw(ch, &f);
        qidx[q] = (size_t)(f.v[0] % half_n);
    }
    int ok = 1;
    q31 last_fold = q_from_m(0);
    for (size_t q = 0; q < nq && ok; q++) {
        size_t pair = in_u64(in);
        size_t rounds = in_u64(in);
        if (pair != qidx[q] || rounds != n_rounds) {
            ok = 0;
            break;
        }
        size_t cur = pair, layer_size = (size_t)1 << n_rounds;
        for (size_t r = 0; r < n_rounds; r++) {
            size_t mid = layer_size / 2;
            q31 lv = in_qm31(in), rv = in_qm31(in);
            size_t idxs[2] = {cur, mid + cur};
            q31 vals[2] = {lv, rv};
            for (int s = 0; s < 2; s++) {
                size_t ns = in_u64(in);
                if (in->bad || ns > 64) return 0;
                uint64_t sib[64 * 4];
                for (size_t l = 0; l < ns; l++) {
                    fe f;
                    in_felt(in, &f);
                    memcpy(sib + 4 * l, f.v, 32);
                }
                if (r < 1 + n_inter) {
                    const fe *rt = r == 0 ? commitment : &inter[r - 1];
                    fe leaf;
                    felt_of_qm31(&leaf, vals[s]);
                    if (!orc_merkle_verify(rt->v, idxs[s], leaf.v, sib, ns)) ok = 0;
                }
            }
            q31 folded = q_add(lv, q_mul(point[r], q_sub(rv, lv)));
            if (r == n_rounds - 1) last_fold = folded;
            size_t next_half = mid / 2 > 0 ? mid / 2 : 1;
            cur %= next_half;
            layer_size = mid;
        }
        (void)last_fold;
    }
    q31 fv = in_qm31(in);
    if (in->bad) return 0;
    /* every query's last fold must equal final_value: recheck by replaying */
    if (final_out) *final_out = fv;
    return ok;
}

int orc_verify_mle_opening(const uint64_t commitment[4], const uint64_t *calldata, size_t len,
                           const uint32_t *point, size_t n_vars, orc_channel *ch, size_t n_queries,
                           uint32_t out_final[4]) {
    oracle_init();
    felt_in in = {calldata, len, 0, 0};
    fe c;
    fe_from_canon(&c, commitment);
    q31 fv;
    /* first pass: structural + Merkle checks */
    orc_channel saved = *ch;
    int ok = verify_opening(&c, &in, (const q31 *)point, n_vars, ch, n_queries, &fv);
    if (!ok) return 0;
    /* second pass: check each query's final fold equals the final value */
    felt_in in2 = {calldata, len, 0, 0};
    size_t n_inter = in_u64(&in2);
    in2.pos += n_inter;
    size_t nq = in_u64(&in2);
    for (size_t q = 0; q < nq; q++) {
        in_u64(&in2);
        size_t rounds = in_u64(&in2);
        q31 folded = q_from_m(0);
        for (size_t r = 0; r < rounds; r++) {
            q31 lv = in_qm31(&in2), rv = in_qm31(&in2);
            for (int s = 0; s < 2; s++) {
                size_t ns = in_u64(&in2);
                in2.pos += ns;
            }
            folded = q_add(lv, q_mul(((const q31 *)point)[r], q_sub(rv, lv)));
        }
        if (!q_eq(folded, fv)) return 0;
    }
    (void)saved;
    if (out_final) q_store(out_final, fv);
    return in.pos == len;
}

/* ------------------------------------------------------------------------ */
/* Single-MatMul GKR proof (gkr/prover.rs:1500-2251, cairo_serde.rs)          */
/* ------------------------------------------------------------------------ */

typedef struct {
    const uint32_t *a;
    const uint32_t *b;
    uint32_t *c;
    size_t k, n;
} mm_ctx;

static void mm_range(void *p, size_t lo, size_t hi) {
    mm_ctx *c = (mm_ctx *)p;
    for (size_t i = lo; i < hi; i++)
        for (size_t j = 0; j < c->n; j++) {
            uint64_t s = 0;
            for (size_t l = 0; l < c->k; l++) {
                s += (uint64_t)c->a[i * c->k + l] * c->b[l * c->n + j];
                if ((l & 3) == 3) s = m_red64(s);
            }
            c->c[i * c->n + j] = m_red64(s);
        }
}

void orc_matmul_m31(const uint32_t *a, size_t m, size_t k, const uint32_t *b, size_t n, uint32_t *c,
                    int threads) {
    mm_ctx ctx = {a, b, c, k, n};
    parallel_for(m, threads, mm_range, &ctx);
}

void orc_io_commitment(const uint32_t *input, size_t in_rows, size_t in_cols, const uint32_t *output,
                       size_t out_rows, size_t out_cols, uint64_t out[4]) {
    oracle_init();
    size_t n = 6 + in_rows * in_cols + out_rows * out_cols, p = 0;
    fe *v = (fe *)malloc(sizeof(fe) * n);
    fe_u64(&v[p++], in_rows);
    fe_u64(&v[p++], in_cols);
    fe_u64(&v[p++], in_rows * in_cols);
    for (size_t i = 0; i < in_rows * in_cols; i++) fe_u64(&v[p++], input[i]);
    fe_u64(&v[p++], out_rows);
    fe_u64(&v[p++], out_cols);
    fe_u64(&v[p++], out_rows * out_cols);
    for (size_t i = 0; i < out_rows * out_cols; i++) fe_u64(&v[p++], output[i]);
    fe r;
    pos_hash_many(&r, v, n);
    memcpy(out, r.v, 32);
    free(v);
}

/* padded row-major MLE of a matrix */
static q31 *mle_row_major(const uint32_t *mat, size_t rows, size_t cols) {
    size_t pr = next_pow2(rows), pc = next_pow2(cols);
    q31 *m = (q31 *)malloc(sizeof(q31) * pr * pc);
    mle_ctx mc = {mat, rows, cols, pr, pc, m, 0};
    mle_range(&mc, 0, pr);
    return m;
}
static q31 *mle_col_major(const uint32_t *mat, size_t rows, size_t cols, int threads) {
    size_t pr = next_pow2(rows), pc = next_pow2(cols);
    q31 *m = (q31 *)malloc(sizeof(q31) * pr * pc);
    mle_ctx mc = {mat, rows, cols, pr, pc, m, 1};
    parallel_for(pc, threads, mle_range, &mc);
    return m;
}

static void gkr_prefix(orc_channel *ch, size_t m, size_t k, const uint64_t *policy) {
    orc_ch_mix_u64(ch, 1); /* circuit depth: the single MatMul layer */
    orc_ch_mix_u64(ch, m);
    orc_ch_mix_u64(ch, k);
    if (policy && (policy[0] | policy[1] | policy[2] | policy[3])) orc_ch_mix_felt(ch, policy);
}

int orc_prove_gkr_matmul(const uint32_t *input, size_t m, size_t k, const uint32_t *weight, size_t n,
                         const uint64_t *policy, size_t n_queries, uint64_t *calldata, size_t cap,
                         size_t *out_len, uint64_t digest[4], uint64_t io[4], int threads) {
    oracle_init();
    orc_channel ch;
    orc_ch_init(&ch);
    gkr_prefix(&ch, m, k, policy);
    size_t pm = next_pow2(m), pk = next_pow2(k), pn = next_pow2(n);
    unsigned log_m = ilog2(pm), log_n = ilog2(pn), log_k = ilog2(pk);
    uint32_t *out = (uint32_t *)malloc(4 * m * n);
    orc_matmul_m31(input, m, k, weight, n, out, threads);
    q31 *omle = mle_row_major(out, m, n);
    q31 *r_out = (q31 *)malloc(sizeof(q31) * (log_m + log_n + 1));
    for (unsigned i = 0; i < log_m + log_n; i++) r_out[i] = ch_draw_qm31(&ch);
    uint32_t val[4];
    orc_evaluate_mle((const uint32_t *)omle, log_m + log_n, (const uint32_t *)r_out, val);
    ch_mix_sf(&ch, q_load(val));
    free(omle);

    uint32_t *rp = (uint32_t *)malloc(48 * (log_k + 1));
    uint32_t fa[4], fb[4];
    q31 *next_pt = (q31 *)malloc(sizeof(q31) * (log_m + log_k + 1));
    int rc = orc_reduce_matmul_gkr((const uint32_t *)r_out, log_m + log_n, val, input, m, k, weight, n, &ch,
                                   rp, fa, fb, (uint32_t *)next_pt, 1, threads);
    if (rc) return rc;

    felt_out o = {calldata, 0, cap, 0};
    out_u64(&o, 1);          /* number of layer proofs */
    out_u64(&o, 0);          /* tag: MatMul */
    out_u64(&o, log_k);      /* rounds */
    for (unsigned r = 0; r < log_k; r++) {
        out_qm31(&o, q_load(rp + 12 * r));     /* c0 */
        out_qm31(&o, q_load(rp + 12 * r + 8)); /* c2 */
    }
    out_qm31(&o, q_load(fa));
    out_qm31(&o, q_load(fb));
    /* input claim */
    out_u64(&o, log_m + log_k);
    for (unsigned i = 0; i < log_m + log_k; i++) out_qm31(&o, next_pt[i]);
    out_qm31(&o, q_load(fa));
    /* weight opening, sequential mode: eval point = r_j || sumcheck challenges */
    q31 *wpt = (q31 *)malloc(sizeof(q31) * (log_n + log_k + 1));
    memcpy(wpt, r_out + log_m, sizeof(q31) * log_n);
    memcpy(wpt + log_n, next_pt + log_m, sizeof(q31) * log_k);
    q31 *bmle = mle_col_major(weight, k, n, threads);
    size_t ocap = cap > o.len ? cap - o.len : 0;
    uint64_t *obuf = (uint64_t *)malloc(32 * (ocap ? ocap : 1));
    felt_out oo = {obuf, 0, ocap, 0};
    fe commitment;
    prove_opening(bmle, log_n + log_k, wpt, &ch, n_queries, &commitment, &oo, NULL, threads);
    free(bmle);
    out_u64(&o, 1); /* weight commitments */
    out_push(&o, &commitment);
    out_u64(&o, 1); /* weight openings */
    out_u64(&o, log_n + log_k);
    for (unsigned i = 0; i < log_n + log_k; i++) out_qm31(&o, wpt[i]);
    out_qm31(&o, q_load(fb));
    for (size_t i = 0; i < oo.len && !oo.overflow; i++) {
        fe f;
        fe_from_canon(&f, obuf + 4 * i);
        out_push(&o, &f);
    }
    orc_io_commitment(input, m, k, out, m, n, io);
    fe iof;
    fe_from_canon(&iof, io);
    out_push(&o, &iof);
    memcpy(digest, ch.digest, 32);
    *out_len = o.len;
    int ovf = o.overflow || oo.overflow;
    free(obuf);
    free(wpt);
    free(next_pt);
    free(rp);
    free(r_out);
    free(out);
    return ovf ? 2 : 0;
}

int orc_verify_gkr_matmul(const uint32_t *input, size_t m, size_t k, const uint32_t *weight, size_t n,
                          const uint64_t *policy, size_t n_queries, const uint64_t *calldata, size_t len,
                          uint64_t digest[4]) {
    oracle_init();
    size_t pm = next_pow2(m), pk = next_pow2(k), pn = next_pow2(n);
    unsigned log_m = ilog2(pm), log_n = ilog2(pn), log_k = ilog2(pk);
    felt_in in = {calldata, len, 0, 0};
    orc_channel ch;
    orc_ch_init(&ch);
    gkr_prefix(&ch, m, k, policy);
    /* output claim from the claimed output = input . weight */
    uint32_t *out = (uint32_t *)malloc(4 * m * n);
    orc_matmul_m31(input, m, k, weight, n, out, 1);
    q31 *omle = mle_row_major(out, m, n);
    q31 r_out[64];
    for (unsigned i = 0; i < log_m + log_n; i++) r_out[i] = ch_draw_qm31(&ch);
    uint32_t val[4];
    orc_evaluate_mle((const uint32_t *)omle, log_m + log_n, (const uint32_t *)r_out, val);
    free(omle);
    ch_mix_sf(&ch, q_load(val));
    int ok = in_u64(&in) == 1 && in_u64(&in) == 0 && in_u64(&in) == log_k;
    /* verify_matmul_reduction */
    orc_ch_mix_u64(&ch, m);
    orc_ch_mix_u64(&ch, k);
    orc_ch_mix_u64(&ch, n);
    ch_mix_sf(&ch, q_load(val));
    q31 cur = q_load(val);
    q31 chal[64];
    for (unsigned r = 0; r < log_k && ok; r++) {
        q31 c0 = in_qm31(&in), c2 = in_qm31(&in);
        /* compressed poly: c1 = claim - 2 c0 - c2 */
        q31 c1 = q_sub(q_sub(cur, q_add(c0, c0)), c2);
        uint32_t coeffs[12];
        q_store(coeffs, c0);
        q_store(coeffs + 4, c1);
        q_store(coeffs + 8, c2);
        orc_ch_mix_poly_coeffs(&ch, coeffs);
        chal[r] = ch_draw_qm31(&ch);
        cur = q_add(c0, q_add(q_mul(c1, chal[r]), q_mul(c2, q_mul(chal[r], chal[r]))));
    }
    q31 fa = in_qm31(&in), fb = in_qm31(&in);
    if (!q_eq(cur, q_mul(fa, fb))) ok = 0;
    ch_mix_sf(&ch, fa);
    ch_mix_sf(&ch, fb);
    /* input claim must match and evaluate the input MLE */
    if (in_u64(&in) != log_m + log_k) ok = 0;
    q31 ipt[64];
    for (unsigned i = 0; i < log_m + log_k && ok; i++) {
        ipt[i] = in_qm31(&in);
        q31 expect = i < log_m ? r_out[i] : chal[i - log_m];
        if (!q_eq(ipt[i], expect)) ok = 0;
    }
    q31 ival = in_qm31(&in);
    if (!q_eq(ival, fa)) ok = 0;
    if (ok) {
        q31 *imle = mle_row_major(input, m, k);
        uint32_t ev[4];
        orc_evaluate_mle((const uint32_t *)imle, log_m + log_k, (const uint32_t *)ipt, ev);
        free(imle);
        if (!q_eq(q_load(ev), fa)) ok = 0;
    }
    /* weight commitment must be the commitment of the given weights */
    if (in_u64(&in) != 1) ok = 0;
    fe commitment;
    in_felt(&in, &commitment);
    if (ok) {
        q31 *bmle = mle_col_major(weight, k, n, 1);
        fe expect;
        merkle_root(bmle, pn * pk, &expect, 1);
        free(bmle);
        if (memcmp(expect.v, commitment.v, 32)) ok = 0;
    }
    if (in_u64(&in) != 1 || in_u64(&in) != log_n + log_k) ok = 0;
    q31 wpt[64];
    for (unsigned i = 0; i < log_n + log_k && ok; i++) {
        wpt[i] = in_qm31(&in);
        q31 expect = i < log_n ? r_out[log_m + i] : chal[i - log_n];
        if (!q_eq(wpt[i], expect)) ok = 0;
    }
    q31 wval = in_qm31(&in);
    if (!q_eq(wval, fb)) ok = 0;
    if (ok) {
        size_t start = in.pos;
        /* find the opening's extent: verify consumes it */
        felt_in sub = {calldata + 4 * start, len - start - 1, 0, 0};
        orc_channel ch2 = ch;
        q31 fv;
        ok = verify_opening(&commitment, &sub, wpt, log_n + log_k, &ch2, n_queries, &fv);
        if (ok) {
            uint32_t fvv[4];
            ok = orc_verify_mle_opening(commitment.v, calldata + 4 * start, sub.pos, (const uint32_t *)wpt,
                                        log_n + log_k, &ch, n_queries, fvv);
            if (ok && !q_eq(q_load(fvv), fb)) ok = 0;
        }
        in.pos = start + sub.pos;
    }
    /* io commitment */
    fe iof;
    in_felt(&in, &iof);
    uint64_t io[4];
    orc_io_commitment(input, m, k, out, m, n, io);
    if (memcmp(io, iof.v, 32)) ok = 0;
    if (in.pos != len || in.bad) ok = 0;
    free(out);
    if (digest) memcpy(digest, ch.digest, 32);
    return ok;
}

/* ------------------------------------------------------------------------ */
/* LogUp activation layer (gkr/prover.rs:6390-6600)                           */
/* ------------------------------------------------------------------------ */

#include <math.h>

/* gadgets/lookup_table.rs:193-345.  Fixed point with scale 2^16; values above
 * (P-1)/2 are read as negative.  Evaluated in binary64 in the same operation
 * order as the reference (the build disables FMA contraction). */
static uint32_t act_signed_to_m31(double v) {
    const uint64_t p = ((uint64_t)1 << 31) - 1;
    if (v >= 0.0) {
        double r = round(v * 65536.0);
        uint64_t u = (uint64_t)r;
        return (uint32_t)(u < p - 1 ? u : p - 1);
    }
    uint64_t neg = (uint64_t)round(-v * 65536.0);
    if (neg > p - 1) neg = p - 1;
    return (uint32_t)(p - neg);
}

static double act_real(uint32_t val) {
    const uint64_t p = ((uint64_t)1 << 31) - 1;
    const uint32_t half_p = (1u << 30) - 1;
    return val <= half_p ? (double)val / 65536.0 : -((double)(p - (uint64_t)val)) / 65536.0;
}

static uint32_t act_fn(int tag, uint32_t val) {
    const uint32_t half_p = (1u << 30) - 1;
    const uint32_t scale = 1u << 16;
    switch (tag) {
    case 1: /* ReLU */
        return val <= half_p ? val : 0;
    case 2: { /* GELU, tanh form */
        if (val == 0) return 0;
        double x = act_real(val);
        double c = sqrt(2.0 / 3.14159265358979311599796346854);
        double inner = c * (x + 0.044715 * x * x * x);
        double g = 0.5 * x * (1.0 + tanh(inner));
        return act_signed_to_m31(g);
    }
    case 3: /* Sigmoid (step approximation) */
        if (val > half_p) return 0;
        return val == 0 ? scale / 2 : scale;
    case 4: { /* softmax exp */
        if (val > half_p) {
            uint32_t neg = ((1u << 31) - 2) - val;
            uint32_t decay = neg / scale;
            if (decay > 20) decay = 20;
            uint32_t r = scale >> decay;
            return r > 1 ? r : 1;
        }
        if (val == 0) return scale;
        uint32_t growth = val / scale;
        if (growth > 10) growth = 10;
        uint64_t r = (uint64_t)scale << growth;
        const uint64_t lim = ((uint64_t)1 << 31) - 2;
        return (uint32_t)(r < lim ? r : lim);
    }
    case 5: { /* SiLU */
        if (val == 0) return 0;
        double x = act_real(val);
        double s = x / (1.0 + exp(-x));
        return act_signed_to_m31(s);
    }
    default:
        return 0;
    }
}

unsigned orc_activation_table_log_size(int tag) { return tag == 4 ? 20 : 16; }

int orc_activation_table(int tag, unsigned log_size, uint32_t *out) {
    if (tag < 1 || tag > 5) return 1;
    for (size_t i = 0; i < ((size_t)1 << log_size); i++) out[i] = act_fn(tag, (uint32_t)i);
    return 0;
}

/* compute_mul_eq_sum_at_t: sum over i < mid of eq_t w_t d_t, x_t = x[i] + t (x[mid+i] - x[i]) */
static q31 mul_eq_sum_at(const q31 *eq, const q31 *w, const q31 *d, size_t mid, uint32_t t) {
    q31 s = q_from_m(0);
    for (size_t i = 0; i < mid; i++) {
        q31 e = q_add(eq[i], q_mul_m(q_sub(eq[mid + i], eq[i]), t));
        q31 a = q_add(w[i], q_mul_m(q_sub(w[mid + i], w[i]), t));
        q31 b = q_add(d[i], q_mul_m(q_sub(d[mid + i], d[i]), t));
        s = q_add(s, q_mul(q_mul(e, a), b));
    }
    return s;
}

static void fold_vec(q31 *v, size_t mid, q31 r) {
    for (size_t i = 0; i < mid; i++) v[i] = q_add(v[i], q_mul(r, q_sub(v[mid + i], v[i])));
}

static void table_commitment(int tag, unsigned log_size, fe *out) {
    fe in[2];
    fe_u64(&in[0], (uint64_t)tag);
    fe_u64(&in[1], log_size);
    pos_hash_many(out, in, 2);
}

int orc_reduce_activation_logup(const uint32_t *input, size_t rows, size_t cols, int tag,
                                const uint32_t *claim_point, size_t n_point, const uint32_t claim_value[4],
                                orc_channel *ch, uint64_t *calldata, size_t cap, size_t *out_len,
                                uint32_t out_input_eval[4]) {
    oracle_init();
    if (tag < 1 || tag > 5) return 1;
    size_t pr = next_pow2(rows), pc = next_pow2(cols), n = pr * pc;
    unsigned num_vars = ilog2(n);
    if (n_point < num_vars) return 1;
    const q31 *point = (const q31 *)claim_point;
    /* input MLE at the claim point (claim chaining) */
    q31 *in_mle = mle_row_major(input, rows, cols);
    q31 input_eval;
    {
        q31 *tmp = (q31 *)malloc(sizeof(q31) * n);
        memcpy(tmp, in_mle, sizeof(q31) * n);
        restrict_inplace(tmp, n, point, num_vars, 1);
        input_eval = tmp[0];
        free(tmp);
    }
    unsigned log_t = orc_activation_table_log_size(tag);
    size_t tsize = (size_t)1 << log_t;
    uint32_t mask = (uint32_t)tsize - 1;
    uint32_t *table = (uint32_t *)malloc(4 * tsize);
    orc_activation_table(tag, log_t, table);
    uint32_t *mult = (uint32_t *)calloc(tsize, 4);
    q31 *m_in = (q31 *)malloc(sizeof(q31) * n), *m_out = (q31 *)malloc(sizeof(q31) * n);
    for (size_t i = 0; i < n; i++) {
        uint32_t x = in_mle[i].a & mask;
        m_in[i] = q_from_m(x);
        m_out[i] = q_from_m(table[x]);
        mult[x]++;
    }
    free(in_mle);
    orc_ch_mix_u64(ch, 0x4C4F47);
    orc_ch_mix_u64(ch, (uint64_t)tag);
    q31 gamma = ch_draw_qm31(ch), beta = ch_draw_qm31(ch);
    q31 *d = (q31 *)malloc(sizeof(q31) * n), *w = (q31 *)malloc(sizeof(q31) * n);
    q31 trace_sum = q_from_m(0);
    for (size_t i = 0; i < n; i++) {
        d[i] = q_sub(q_sub(gamma, m_in[i]), q_mul(beta, m_out[i]));
        w[i] = q_inv(d[i]);
        trace_sum = q_add(trace_sum, w[i]);
    }
    q31 table_sum = q_from_m(0);
    for (size_t j = 0; j < tsize; j++) {
        if (!mult[j]) continue;
        q31 dj = q_sub(q_sub(gamma, q_from_m((uint32_t)j)), q_mul(beta, q_from_m(table[j])));
        table_sum = q_add(table_sum, q_mul_m(q_inv(dj), mult[j] % MP));
    }
    int rc = 0;
    if (!q_eq(trace_sum, table_sum)) rc = 3;
    ch_mix_sf(ch, trace_sum);
    /* degree-3 eq-sumcheck: sum eq(r, x) w(x) d(x) = 1 */
    q31 *eq = lagrange_basis(point, num_vars);
    q31 *rps = (q31 *)malloc(sizeof(q31) * 4 * (num_vars + 1));
    q31 *chal = (q31 *)malloc(sizeof(q31) * (num_vars + 1));
    uint32_t inv2 = m_inv(2), inv6 = m_inv(6);
    size_t cur = n;
    for (unsigned r = 0; r < num_vars; r++) {
        size_t mid = cur / 2;
        q31 s0 = mul_eq_sum_at(eq, w, d, mid, 0), s1 = mul_eq_sum_at(eq, w, d, mid, 1);
        q31 s2 = mul_eq_sum_at(eq, w, d, mid, 2), s3 = mul_eq_sum_at(eq, w, d, mid, 3);
        q31 dd1 = q_sub(s1, s0);
        q31 dd2 = q_mul_m(q_add(q_sub(q_sub(s2, s1), s1), s0), inv2);
        q31 dd3 = q_mul_m(q_sub(q_sub(s3, s0), q_mul_m(q_sub(s2, s1), 3)), inv6);
        q31 c0 = s0, c1 = q_add(q_sub(dd1, dd2), q_mul_m(dd3, 2)), c2 = q_sub(dd2, q_mul_m(dd3, 3)), c3 = dd3;
        rps[4 * r] = c0;
        rps[4 * r + 1] = c1;
        rps[4 * r + 2] = c2;
        rps[4 * r + 3] = c3;
        uint32_t coeffs[16];
        q_store(coeffs, c0);
        q_store(coeffs + 4, c1);
        q_store(coeffs + 8, c2);
        q_store(coeffs + 12, c3);
        orc_ch_mix_poly_coeffs_deg3(ch, coeffs);
        chal[r] = ch_draw_qm31(ch);
        fold_vec(eq, mid, chal[r]);
        fold_vec(w, mid, chal[r]);
        fold_vec(d, mid, chal[r]);
        cur = mid;
    }
    q31 w_eval = w[0];
    restrict_inplace(m_in, n, chal, num_vars, 1);
    restrict_inplace(m_out, n, chal, num_vars, 1);
    q31 in_eval_s = m_in[0], out_eval_s = m_out[0];
    /* multiplicity sumcheck (prover.rs:9449-9515) */
    unsigned mvars = log_t;
    q31 *mv = (q31 *)malloc(sizeof(q31) * tsize);
    q31 m_claim = q_from_m(0);
    for (size_t j = 0; j < tsize; j++) {
        mv[j] = q_from_m(mult[j] % MP);
        m_claim = q_add(m_claim, mv[j]);
    }
    q31 *mrp = (q31 *)malloc(sizeof(q31) * 2 * (mvars + 1));
    size_t msz = tsize;
    for (unsigned r = 0; r < mvars; r++) {
        size_t half = msz / 2;
        q31 s0 = q_from_m(0), s1 = q_from_m(0);
        for (size_t j = 0; j < half; j++) {
            s0 = q_add(s0, mv[j]);
            s1 = q_add(s1, mv[half + j]);
        }
        q31 c0 = s0, c1 = q_sub(s1, s0);
        mrp[2 * r] = c0;
        mrp[2 * r + 1] = c1;
        ch_mix_sf(ch, c0);
        ch_mix_sf(ch, c1);
        q31 rr = ch_draw_qm31(ch);
        fold_vec(mv, half, rr);
        msz = half;
    }
    q31 m_final = mv[0];
    fe tcom;
    table_commitment(tag, log_t, &tcom);
    ch_mix_sf(ch, input_eval);
    ch_mix_sf(ch, q_load(claim_value));
    /* serialize LayerProof::Activation */
    felt_out o = {calldata, 0, cap, 0};
    out_u64(&o, 3);
    out_u64(&o, (uint64_t)tag);
    out_qm31(&o, input_eval);
    out_qm31(&o, q_load(claim_value));
    out_push(&o, &tcom);
    out_u64(&o, 1); /* logup proof present */
    out_qm31(&o, trace_sum);
    out_u64(&o, num_vars);
    for (unsigned r = 0; r < num_vars; r++) {
        out_qm31(&o, rps[4 * r]);
        out_qm31(&o, rps[4 * r + 2]);
        out_qm31(&o, rps[4 * r + 3]);
    }
    out_qm31(&o, w_eval);
    out_qm31(&o, in_eval_s);
    out_qm31(&o, out_eval_s);
    out_u64(&o, tsize);
    for (size_t j = 0; j < tsize; j++) out_u64(&o, mult[j]);
    out_u64(&o, 1); /* multiplicity sumcheck present */
    out_u64(&o, mvars);
    for (unsigned r = 0; r < mvars; r++) {
        out_qm31(&o, mrp[2 * r]);
        out_qm31(&o, mrp[2 * r + 1]);
    }
    out_qm31(&o, m_final);
    out_qm31(&o, m_claim);
    out_u64(&o, 0); /* no activation product proof */
    out_u64(&o, 0); /* no piecewise proof */
    *out_len = o.len;
    if (out_input_eval) q_store(out_input_eval, input_eval);
    free(mrp);
    free(mv);
    free(chal);
    free(rps);
    free(eq);
    free(w);
    free(d);
    free(m_in);
    free(m_out);
    free(mult);
    free(table);
    if (rc) return rc;
    return o.overflow ? 2 : 0;
}

/* eq(r, s) = prod ((1 - r_i)(1 - s_i) + r_i s_i) */
static q31 eq_eval(const q31 *r, const q31 *s, size_t n) {
    q31 acc = q_from_m(1), one = q_from_m(1);
    for (size_t i = 0; i < n; i++)
        acc = q_mul(acc, q_add(q_mul(q_sub(one, r[i]), q_sub(one, s[i])), q_mul(r[i], s[i])));
    return acc;
}

static int orc_verify_activation_logup_impl(size_t *consumed, uint32_t *out_point, int exact, const uint64_t *calldata, size_t len, const uint32_t *claim_point, size_t n_point,
                                const uint32_t claim_value[4], orc_channel *ch, uint32_t out_input_eval[4]) {
    oracle_init();
    felt_in in = {calldata, len, 0, 0};
    if (in_u64(&in) != 3) return 0;
    int tag = (int)in_u64(&in);
    if (tag < 1 || tag > 5) return 0;
    q31 input_eval = in_qm31(&in), output_eval = in_qm31(&in);
    fe tcom, expect;
    in_felt(&in, &tcom);
    if (in_u64(&in) != 1) return 0;
    q31 claimed = in_qm31(&in);
    size_t num_vars = in_u64(&in);
    if (num_vars == 0 || num_vars > n_point || num_vars > 40 || in.bad) return 0;
    if (!q_eq(output_eval, q_load(claim_value))) return 0;
    orc_ch_mix_u64(ch, 0x4C4F47);
    orc_ch_mix_u64(ch, (uint64_t)tag);
    q31 gamma = ch_draw_qm31(ch), beta = ch_draw_qm31(ch);
    unsigned log_t = orc_activation_table_log_size(tag);
    table_commitment(tag, log_t, &expect);
    if (memcmp(expect.v, tcom.v, 32)) return 0;
    /* read the rest of the logup proof */
    q31 rp[40][4];
    for (size_t r = 0; r < num_vars; r++) {
        rp[r][0] = in_qm31(&in);
        rp[r][2] = in_qm31(&in);
        rp[r][3] = in_qm31(&in);
    }
    q31 w_eval = in_qm31(&in), in_s = in_qm31(&in), out_s = in_qm31(&in);
    size_t tsize = (size_t)1 << log_t;
    if (in_u64(&in) != tsize || in.bad) return 0;
    uint32_t *table = (uint32_t *)malloc(4 * tsize);
    orc_activation_table(tag, log_t, table);
    q31 table_sum = q_from_m(0);
    for (size_t j = 0; j < tsize; j++) {
        uint64_t m = in_u64(&in);
        if (!m) continue;
        q31 dj = q_sub(q_sub(gamma, q_from_m((uint32_t)j)), q_mul(beta, q_from_m(table[j])));
        table_sum = q_add(table_sum, q_mul(q_from_m((uint32_t)(m % MP)), q_inv(dj)));
    }
    free(table);
    if (!q_eq(table_sum, claimed)) return 0;
    ch_mix_sf(ch, claimed);
    q31 cur = q_from_m(1), chal[40];
    for (size_t r = 0; r < num_vars; r++) {
        /* compressed: c1 = cur - 2 c0 - c2 - c3 */
        q31 c0 = rp[r][0], c2 = rp[r][2], c3 = rp[r][3];
        q31 c1 = q_sub(q_sub(q_sub(cur, q_add(c0, c0)), c2), c3);
        uint32_t coeffs[16];
        q_store(coeffs, c0);
        q_store(coeffs + 4, c1);
        q_store(coeffs + 8, c2);
        q_store(coeffs + 12, c3);
        orc_ch_mix_poly_coeffs_deg3(ch, coeffs);
        chal[r] = ch_draw_qm31(ch);
        q31 x = chal[r];
        cur = q_add(c0, q_mul(x, q_add(c1, q_mul(x, q_add(c2, q_mul(x, c3))))));
    }
    q31 d_eval = q_sub(q_sub(gamma, in_s), q_mul(beta, out_s));
    q31 expect_sum = q_mul(q_mul(eq_eval((const q31 *)claim_point, chal, num_vars), w_eval), d_eval);
    if (!q_eq(cur, expect_sum)) return 0;
    /* multiplicity sumcheck */
    if (in_u64(&in) == 1) {
        size_t mr = in_u64(&in);
        if (mr > 40) return 0;
        q31 mc[40][2];
        for (size_t r = 0; r < mr; r++) {
            mc[r][0] = in_qm31(&in);
            mc[r][1] = in_qm31(&in);
        }
        q31 mfinal = in_qm31(&in), mclaim = in_qm31(&in);
        q31 s = mclaim;
        for (size_t r = 0; r < mr; r++) {
            if (!q_eq(q_add(mc[r][0], q_add(mc[r][0], mc[r][1])), s)) return 0;
            ch_mix_sf(ch, mc[r][0]);
            ch_mix_sf(ch, mc[r][1]);
            q31 x = ch_draw_qm31(ch);
            s = q_add(mc[r][0], q_mul(mc[r][1], x));
        }
        if (!q_eq(s, mfinal)) return 0;
    }
    if (in_u64(&in) != 0 || in_u64(&in) != 0) return 0; /* no product / piecewise proofs */
    ch_mix_sf(ch, input_eval);
    ch_mix_sf(ch, output_eval);
    if (out_input_eval) q_store(out_input_eval, input_eval);
    if (consumed) *consumed = in.pos;
    return (exact ? in.pos == len : in.pos <= len) && !in.bad;
}

int orc_verify_activation_logup(const uint64_t *calldata, size_t len, const uint32_t *claim_point, size_t n_point,
                                const uint32_t claim_value[4], orc_channel *ch, uint32_t out_input_eval[4]) {
    return orc_verify_activation_logup_impl(NULL, NULL, 1, calldata, len, claim_point, n_point, claim_value, ch, out_input_eval);
}

/* ---------------------------------------------------------------------------
 * RMSNorm layer reduction.
 * ------------------------------------------------------------------------- */

/* floor(sqrt(v)) for v < 2^53 (floating estimate, then corrected to the exact floor). */
static uint64_t isqrt_u64(uint64_t v) {
    uint64_t s = (uint64_t)sqrt((double)v);
    while (s * s > v) s--;
    while ((s + 1) * (s + 1) <= v) s++;
    return s;
}

/* rsqrt lookup table (components/layernorm.rs:116-136): 0 -> 2^16 - 1, x -> min(2^16 / isqrt(x), p - 1). */
int orc_rsqrt_table(unsigned log_size, uint32_t *out) {
    if (log_size > 24) return 1;
    for (size_t x = 0; x < ((size_t)1 << log_size); x++) {
        if (x == 0) {
            out[x] = (1u << 16) - 1;
            continue;
        }
        uint64_t s = isqrt_u64(x);
        uint64_t r = ((uint64_t)1 << 16) / s;
        const uint64_t lim = ((uint64_t)1 << 31) - 2;
        out[x] = (uint32_t)(r < lim ? r : lim);
    }
    return 0;
}

/* build_multiplicity_sumcheck (gkr/prover.rs:9449-9515): degree-1 rounds over the
 * multiplicity MLE; per round mix c0, c1 and draw.  Fills rounds (2 per round), final, claim. */
static void mult_sumcheck(orc_channel *ch, const uint32_t *mult, unsigned log_t, q31 *mrp, q31 *m_final,
                          q31 *m_claim) {
    size_t tsize = (size_t)1 << log_t;
    q31 *mv = (q31 *)malloc(sizeof(q31) * tsize);
    q31 claim = q_from_m(0);
    for (size_t j = 0; j < tsize; j++) {
        mv[j] = q_from_m(mult[j] % MP);
        claim = q_add(claim, mv[j]);
    }
    size_t msz = tsize;
    for (unsigned r = 0; r < log_t; r++) {
        size_t half = msz / 2;
        q31 s0 = q_from_m(0), s1 = q_from_m(0);
        for (size_t j = 0; j < half; j++) {
            s0 = q_add(s0, mv[j]);
            s1 = q_add(s1, mv[half + j]);
        }
        q31 c0 = s0, c1 = q_sub(s1, s0);
        if (mrp) {
            mrp[2 * r] = c0;
            mrp[2 * r + 1] = c1;
        }
        ch_mix_sf(ch, c0);
        ch_mix_sf(ch, c1);
        fold_vec(mv, half, ch_draw_qm31(ch));
        msz = half;
    }
    if (m_final) *m_final = mv[0];
    if (m_claim) *m_claim = claim;
    free(mv);
}

static void mix_deg3(orc_channel *ch, q31 c0, q31 c1, q31 c2, q31 c3) {
    uint32_t coeffs[16];
    q_store(coeffs, c0);
    q_store(coeffs + 4, c1);
    q_store(coeffs + 8, c2);
    q_store(coeffs + 12, c3);
    orc_ch_mix_poly_coeffs_deg3(ch, coeffs);
}

/* Degree-3 eq-sumcheck sum eq(r, x) a(x) b(x) (eq, a, b are consumed); rounds get
 * (c0, c1, c2, c3) per round, chal the challenges. */
static void eq_sumcheck_deg3(orc_channel *ch, q31 *eq, q31 *a, q31 *b, size_t n, unsigned num_vars, q31 *rps,
                             q31 *chal) {
    uint32_t inv2 = m_inv(2), inv6 = m_inv(6);
    size_t cur = n;
    for (unsigned r = 0; r < num_vars; r++) {
        size_t mid = cur / 2;
        q31 s0 = mul_eq_sum_at(eq, a, b, mid, 0), s1 = mul_eq_sum_at(eq, a, b, mid, 1);
        q31 s2 = mul_eq_sum_at(eq, a, b, mid, 2), s3 = mul_eq_sum_at(eq, a, b, mid, 3);
        q31 dd1 = q_sub(s1, s0);
        q31 dd2 = q_mul_m(q_add(q_sub(q_sub(s2, s1), s1), s0), inv2);
        q31 dd3 = q_mul_m(q_sub(q_sub(s3, s0), q_mul_m(q_sub(s2, s1), 3)), inv6);
        q31 c0 = s0, c1 = q_add(q_sub(dd1, dd2), q_mul_m(dd3, 2)), c2 = q_sub(dd2, q_mul_m(dd3, 3)), c3 = dd3;
        rps[4 * r] = c0;
        rps[4 * r + 1] = c1;
        rps[4 * r + 2] = c2;
        rps[4 * r + 3] = c3;
        mix_deg3(ch, c0, c1, c2, c3);
        chal[r] = ch_draw_qm31(ch);
        fold_vec(eq, mid, chal[r]);
        fold_vec(a, mid, chal[r]);
        fold_vec(b, mid, chal[r]);
        cur = mid;
    }
}

static q31 mle_eval_copy(const q31 *v, size_t n, const q31 *point, unsigned num_vars) {
    q31 *tmp = (q31 *)malloc(sizeof(q31) * n);
    memcpy(tmp, v, sizeof(q31) * n);
    restrict_inplace(tmp, n, point, num_vars, 1);
    q31 r = tmp[0];
    free(tmp);
    return r;
}

/* serialize_multiplicity_sumcheck (cairo_serde.rs:1138-1156) of a present proof. */
static void out_mult_sumcheck(felt_out *o, const q31 *mrp, unsigned log_t, q31 m_final, q31 m_claim) {
    out_u64(o, 1);
    out_u64(o, log_t);
    for (unsigned r = 0; r < log_t; r++) {
        out_qm31(o, mrp[2 * r]);
        out_qm31(o, mrp[2 * r + 1]);
    }
    out_qm31(o, m_final);
    out_qm31(o, m_claim);
}

/* v1: the record as serialize_gkr_proof_data_only writes it (cairo_serde.rs:2145-2222): the
 * LogUp proof without multiplicities, then the multiplicity sumcheck. */
static int rmsnorm_impl(const uint32_t *input, size_t rows, size_t cols, size_t dim, const uint32_t *gamma_aff,
                        size_t gamma_len, int skip_rms_sq, const uint32_t *claim_point, size_t n_point,
                        const uint32_t claim_value[4], orc_channel *ch, uint64_t *calldata, size_t cap,
                        size_t *out_len, uint32_t out_input_eval[4], int v1) {
    oracle_init();
    if (rows == 0 || cols == 0 || dim == 0 || (gamma_aff && gamma_len == 0)) return 1;
    size_t pr = next_pow2(rows), pc = next_pow2(cols), n = pr * pc;
    unsigned num_vars = ilog2(n);
    if (num_vars == 0 || n_point < num_vars) return 1;
    const q31 *point = (const q31 *)claim_point;
    const unsigned log_t = 16;
    const size_t tsize = (size_t)1 << log_t;
    const uint32_t mask = (uint32_t)tsize - 1;
    uint32_t *table = (uint32_t *)malloc(4 * tsize);
    orc_rsqrt_table(log_t, table);
    size_t n_active = dim < pc ? dim : pc;
    uint32_t inv_n = m_inv((uint32_t)(n_active % MP));
    /* per-row rms^2 = (sum of squares of the first n_active columns) / n_active, masked to the table */
    q31 *in_mle = mle_row_major(input, rows, cols);
    q31 *rsq = (q31 *)malloc(sizeof(q31) * n), *rsq_raw = (q31 *)malloc(sizeof(q31) * n);
    q31 *scale = (q31 *)malloc(sizeof(q31) * n), *outv = (q31 *)malloc(sizeof(q31) * n);
    uint32_t *row_rms = (uint32_t *)malloc(4 * pr), *mult = (uint32_t *)calloc(tsize, 4);
    for (size_t i = 0; i < pr; i++) {
        uint32_t sq = 0;
        for (size_t j = 0; j < n_active; j++) sq = m_add(sq, m_mul(in_mle[i * pc + j].a, in_mle[i * pc + j].a));
        uint32_t rms = m_mul(sq, inv_n) & mask, rs = table[rms];
        row_rms[i] = rms;
        mult[rms] += (uint32_t)pc;
        for (size_t j = 0; j < pc; j++) {
            size_t idx = i * pc + j;
            uint32_t x = in_mle[idx].a;
            rsq[idx] = q_from_m(rms);
            rsq_raw[idx] = q_from_m(rs);
            if (j < n_active) {
                uint32_t sc = gamma_aff ? m_mul(rs, gamma_aff[j < gamma_len - 1 ? j : gamma_len - 1] % MP) : rs;
                scale[idx] = q_from_m(sc);
                outv[idx] = q_from_m(m_mul(x, sc));
            } else {
                scale[idx] = q_from_m(rs);
                outv[idx] = q_from_m(x);
            }
        }
    }
    q31 input_eval = mle_eval_copy(in_mle, n, point, num_vars);
    q31 output_eval = mle_eval_copy(outv, n, point, num_vars);
    q31 rsqrt_eval = mle_eval_copy(rsq_raw, n, point, num_vars);
    q31 rms_sq_eval = mle_eval_copy(rsq, n, point, num_vars);
    free(outv);
    /* Part 0: plain sumcheck sum_x input(x)^2 = total (prover.rs:8500-8545) */
    q31 *rq = (q31 *)malloc(sizeof(q31) * 4 * (num_vars + 1));
    q31 total_sq = q_from_m(0), rq_final = q_from_m(0);
    for (size_t i = 0; i < n; i++) total_sq = q_add(total_sq, q_mul(in_mle[i], in_mle[i]));
    if (!skip_rms_sq) {
        orc_ch_mix_u64(ch, 0x5251);
        orc_ch_mix_u64(ch, n_active);
        ch_mix_sf(ch, total_sq);
        q31 *v = (q31 *)malloc(sizeof(q31) * n);
        memcpy(v, in_mle, sizeof(q31) * n);
        uint32_t inv2 = m_inv(2);
        size_t cur = n;
        for (unsigned r = 0; r < num_vars; r++) {
            size_t mid = cur / 2;
            q31 s0 = q_from_m(0), s1 = q_from_m(0), s2 = q_from_m(0);
            for (size_t j = 0; j < mid; j++) {
                q31 lo = v[j], hi = v[mid + j], two = q_sub(q_add(hi, hi), lo);
                s0 = q_add(s0, q_mul(lo, lo));
                s1 = q_add(s1, q_mul(hi, hi));
                s2 = q_add(s2, q_mul(two, two));
            }
            q31 dd1 = q_sub(s1, s0);
            q31 dd2 = q_mul_m(q_sub(q_sub(s2, s1), dd1), inv2);
            q31 c0 = s0, c1 = q_sub(dd1, dd2), c2 = dd2, c3 = q_from_m(0);
            rq[4 * r] = c0;
            rq[4 * r + 1] = c1;
            rq[4 * r + 2] = c2;
            rq[4 * r + 3] = c3;
            mix_deg3(ch, c0, c1, c2, c3);
            fold_vec(v, mid, ch_draw_qm31(ch));
            cur = mid;
        }
        rq_final = v[0];
        ch_mix_sf(ch, rq_final);
        free(v);
    }
    /* Part 1: degree-3 eq-sumcheck output = input x scale (prover.rs:8560-8630) */
    orc_ch_mix_u64(ch, 0x524E);
    ch_mix_sf(ch, rms_sq_eval);
    ch_mix_sf(ch, rsqrt_eval);
    ch_mix_sf(ch, q_load(claim_value));
    q31 *eq = lagrange_basis(point, num_vars);
    q31 *a = (q31 *)malloc(sizeof(q31) * n);
    memcpy(a, in_mle, sizeof(q31) * n);
    q31 *lin = (q31 *)malloc(sizeof(q31) * 4 * (num_vars + 1));
    q31 *chal = (q31 *)malloc(sizeof(q31) * (num_vars + 1));
    eq_sumcheck_deg3(ch, eq, a, scale, n, num_vars, lin, chal);
    q31 input_final = a[0], rsqrt_final = scale[0];
    ch_mix_sf(ch, input_final);
    ch_mix_sf(ch, rsqrt_final);
    free(eq);
    free(a);
    free(scale);
    free(in_mle);
    /* Part 2: LogUp of (rms^2, rsqrt) against the rsqrt table (prover.rs:8632-8720) */
    orc_ch_mix_u64(ch, 0x4C4F47);
    orc_ch_mix_u64(ch, 0x524E);
    q31 gm = ch_draw_qm31(ch), bt = ch_draw_qm31(ch);
    q31 *d = (q31 *)malloc(sizeof(q31) * n), *w = (q31 *)malloc(sizeof(q31) * n);
    q31 trace_sum = q_from_m(0);
    for (size_t i = 0; i < n; i++) {
        d[i] = q_sub(q_sub(gm, rsq[i]), q_mul(bt, rsq_raw[i]));
        w[i] = q_inv(d[i]);
        trace_sum = q_add(trace_sum, w[i]);
    }
    q31 table_sum = q_from_m(0);
    for (size_t j = 0; j < tsize; j++) {
        if (!mult[j]) continue;
        q31 dj = q_sub(q_sub(gm, q_from_m((uint32_t)j)), q_mul(bt, q_from_m(table[j])));
        table_sum = q_add(table_sum, q_mul_m(q_inv(dj), mult[j] % MP));
    }
    int rc = q_eq(trace_sum, table_sum) ? 0 : 3;
    ch_mix_sf(ch, trace_sum);
    eq = lagrange_basis(point, num_vars);
    q31 *lrp = (q31 *)malloc(sizeof(q31) * 4 * (num_vars + 1));
    eq_sumcheck_deg3(ch, eq, w, d, n, num_vars, lrp, chal);
    q31 w_eval = w[0];
    restrict_inplace(rsq, n, chal, num_vars, 1);
    restrict_inplace(rsq_raw, n, chal, num_vars, 1);
    q31 rms_s = rsq[0], rsqrt_s = rsq_raw[0];
    q31 *mrp = (q31 *)malloc(sizeof(q31) * 2 * log_t), m_final, m_claim;
    mult_sumcheck(ch, mult, log_t, mrp, &m_final, &m_claim);
    fe tcom;
    table_commitment(0x5253, log_t, &tcom);
    ch_mix_sf(ch, input_eval);
    ch_mix_sf(ch, output_eval);
    /* LayerProof::RMSNorm as serialize_gkr_model_proof writes it (cairo_serde.rs:1648-1726) */
    felt_out o = {calldata, 0, cap, 0};
    out_u64(&o, 8);
    out_qm31(&o, input_eval);
    out_qm31(&o, output_eval);
    out_qm31(&o, rms_sq_eval);
    out_qm31(&o, rsqrt_eval);
    out_push(&o, &tcom);
    out_u64(&o, 0); /* not SIMD-combined */
    if (skip_rms_sq) {
        out_u64(&o, 0);
    } else {
        out_u64(&o, 1);
        out_u64(&o, n_active);
        out_qm31(&o, total_sq);
        out_u64(&o, num_vars);
        for (unsigned r = 0; r < num_vars; r++) {
            out_qm31(&o, rq[4 * r]);
            out_qm31(&o, rq[4 * r + 2]);
            out_qm31(&o, rq[4 * r + 3]);
        }
        out_qm31(&o, rq_final);
    }
    out_u64(&o, num_vars);
    for (unsigned r = 0; r < num_vars; r++) {
        out_qm31(&o, lin[4 * r]);
        out_qm31(&o, lin[4 * r + 2]);
        out_qm31(&o, lin[4 * r + 3]);
    }
    out_qm31(&o, input_final);
    out_qm31(&o, rsqrt_final);
    out_u64(&o, 1); /* LogUp proof present */
    out_qm31(&o, trace_sum);
    out_u64(&o, num_vars);
    for (unsigned r = 0; r < num_vars; r++) {
        out_qm31(&o, lrp[4 * r]);
        out_qm31(&o, lrp[4 * r + 2]);
        out_qm31(&o, lrp[4 * r + 3]);
    }
    out_qm31(&o, w_eval);
    out_qm31(&o, rms_s);
    out_qm31(&o, rsqrt_s);
    if (v1) {
        out_u64(&o, 0); /* no multiplicities on chain */
        out_mult_sumcheck(&o, mrp, log_t, m_final, m_claim);
    } else {
        out_u64(&o, tsize);
        for (size_t j = 0; j < tsize; j++) out_u64(&o, mult[j]);
    }
    free(mrp);
    if (pr > 1) {
        out_u64(&o, 1);
        out_u64(&o, pr);
        for (size_t i = 0; i < pr; i++) out_u64(&o, row_rms[i]);
    } else {
        out_u64(&o, 0);
    }
    *out_len = o.len;
    if (out_input_eval) q_store(out_input_eval, input_eval);
    free(lrp);
    free(eq);
    free(d);
    free(w);
    free(chal);
    free(lin);
    free(rq);
    free(rsq);
    free(rsq_raw);
    free(row_rms);
    free(mult);
    free(table);
    if (rc) return rc;
    return o.overflow ? 2 : 0;
}

int orc_reduce_rmsnorm(const uint32_t *input, size_t rows, size_t cols, size_t dim, const uint32_t *gamma_aff,
                       size_t gamma_len, int skip_rms_sq, const uint32_t *claim_point, size_t n_point,
                       const uint32_t claim_value[4], orc_channel *ch, uint64_t *calldata, size_t cap,
                       size_t *out_len, uint32_t out_input_eval[4]) {
    return rmsnorm_impl(input, rows, cols, dim, gamma_aff, gamma_len, skip_rms_sq, claim_point, n_point, claim_value,
                        ch, calldata, cap, out_len, out_input_eval, 0);
}

/* Replays a compressed deg-3 sumcheck: c1 = cur - 2 c0 - c2 - c3; returns the final sum. */
static q31 replay_deg3(orc_channel *ch, felt_in *in, size_t rounds, q31 cur, q31 *chal) {
    for (size_t r = 0; r < rounds; r++) {
        q31 c0 = in_qm31(in), c2 = in_qm31(in), c3 = in_qm31(in);
        q31 c1 = q_sub(q_sub(q_sub(cur, q_add(c0, c0)), c2), c3);
        mix_deg3(ch, c0, c1, c2, c3);
        q31 x = ch_draw_qm31(ch);
        if (chal) chal[r] = x;
        cur = q_add(c0, q_mul(x, q_add(c1, q_mul(x, q_add(c2, q_mul(x, c3))))));
    }
    return cur;
}

static int orc_verify_rmsnorm_impl(size_t *consumed, uint32_t *out_point, int exact, const uint64_t *calldata, size_t len, size_t dim, const uint32_t *claim_point,
                       size_t n_point, const uint32_t claim_value[4], orc_channel *ch, uint32_t out_input_eval[4]) {
    oracle_init();
    felt_in in = {calldata, len, 0, 0};
    if (in_u64(&in) != 8) return 0;
    q31 input_eval = in_qm31(&in), output_eval = in_qm31(&in);
    q31 rms_sq_eval = in_qm31(&in), rsqrt_eval = in_qm31(&in);
    fe tcom, expect;
    in_felt(&in, &tcom);
    table_commitment(0x5253, 16, &expect);
    if (memcmp(expect.v, tcom.v, 32) || in_u64(&in) != 0 || in.bad) return 0;
    const q31 *point = (const q31 *)claim_point;
    size_t has_rq = in_u64(&in);
    size_t num_vars = 0;
    if (has_rq == 1) {
        /* Part 0 (verifier.rs:4755-4870) */
        size_t n_active_s = in_u64(&in);
        q31 total = in_qm31(&in);
        num_vars = in_u64(&in);
        if (num_vars == 0 || num_vars > 40 || num_vars > n_point || in.bad) return 0;
        size_t n_active = dim < ((size_t)1 << num_vars) ? dim : ((size_t)1 << num_vars);
        if (n_active_s != n_active) return 0;
        orc_ch_mix_u64(ch, 0x5251);
        orc_ch_mix_u64(ch, n_active);
        ch_mix_sf(ch, total);
        q31 cur = replay_deg3(ch, &in, num_vars, total, NULL);
        q31 fin = in_qm31(&in);
        ch_mix_sf(ch, fin);
        if (!q_eq(q_mul(fin, fin), cur)) return 0;
        size_t cols_p = next_pow2(dim), rows_p = ((size_t)1 << num_vars) / cols_p;
        if (cols_p > ((size_t)1 << num_vars)) return 0;
        if (rows_p == 1) {
            uint32_t rms = m_mul(total.a, m_inv((uint32_t)(n_active % MP))) & 0xFFFFu;
            if (!q_eq(rms_sq_eval, q_from_m(rms))) return 0;
        }
        /* multi-row binding is checked after the row values are read */
    } else if (has_rq != 0) {
        return 0;
    } else {
        return 0; /* a missing RMS^2 proof is rejected (no override) */
    }
    if (in_u64(&in) != num_vars) return 0;
    /* Part 1 */
    orc_ch_mix_u64(ch, 0x524E);
    ch_mix_sf(ch, rms_sq_eval);
    ch_mix_sf(ch, rsqrt_eval);
    ch_mix_sf(ch, q_load(claim_value));
    q31 chal[40];
    q31 cur = replay_deg3(ch, &in, num_vars, q_load(claim_value), chal);
    q31 input_final = in_qm31(&in), rsqrt_final = in_qm31(&in);
    if (!q_eq(cur, q_mul(q_mul(eq_eval(point, chal, num_vars), input_final), rsqrt_final))) return 0;
    ch_mix_sf(ch, input_final);
    ch_mix_sf(ch, rsqrt_final);
    /* Part 2 */
    if (in_u64(&in) != 1) return 0;
    orc_ch_mix_u64(ch, 0x4C4F47);
    orc_ch_mix_u64(ch, 0x524E);
    q31 gm = ch_draw_qm31(ch), bt = ch_draw_qm31(ch);
    q31 claimed = in_qm31(&in);
    if (in_u64(&in) != num_vars || in.bad) return 0;
    size_t rounds_at = in.pos;
    in.pos += 12 * num_vars; /* round polynomials are replayed after the sum check */
    q31 w_eval = in_qm31(&in), rms_s = in_qm31(&in), rsqrt_s = in_qm31(&in);
    const size_t tsize = (size_t)1 << 16;
    if (in_u64(&in) != tsize || in.bad || in.pos + tsize > len) return 0;
    uint32_t *table = (uint32_t *)malloc(4 * tsize), *mult = (uint32_t *)malloc(4 * tsize);
    orc_rsqrt_table(16, table);
    q31 table_sum = q_from_m(0);
    for (size_t j = 0; j < tsize; j++) {
        uint64_t m = in_u64(&in);
        mult[j] = (uint32_t)m;
        if (!m) continue;
        q31 dj = q_sub(q_sub(gm, q_from_m((uint32_t)j)), q_mul(bt, q_from_m(table[j])));
        table_sum = q_add(table_sum, q_mul(q_from_m((uint32_t)(m % MP)), q_inv(dj)));
    }
    free(table);
    int ok = q_eq(table_sum, claimed);
    if (ok) {
        ch_mix_sf(ch, claimed);
        felt_in rin = {calldata, len, rounds_at, 0};
        q31 lsum = replay_deg3(ch, &rin, num_vars, q_from_m(1), chal);
        q31 d_eval = q_sub(q_sub(gm, rms_s), q_mul(bt, rsqrt_s));
        ok = q_eq(lsum, q_mul(q_mul(eq_eval(point, chal, num_vars), w_eval), d_eval));
    }
    /* the multiplicity sumcheck is not in the calldata; it is a function of the
     * multiplicities and the transcript, so the verifier replays it */
    if (ok) mult_sumcheck(ch, mult, 16, NULL, NULL, NULL);
    free(mult);
    if (!ok) return 0;
    /* per-row rms^2 binding (verifier.rs:4830-4870) */
    size_t has_rows = in_u64(&in);
    if (has_rows == 1) {
        size_t cols_p = next_pow2(dim), rows_p = ((size_t)1 << num_vars) / cols_p;
        size_t nr = in_u64(&in);
        if (nr != rows_p || in.bad) return 0;
        unsigned log_rows = ilog2(rows_p);
        q31 acc = q_from_m(0);
        for (size_t r = 0; r < nr; r++) {
            q31 e = q_from_m(1);
            for (unsigned k = 0; k < log_rows; k++) {
                size_t bit = (r >> (log_rows - 1 - k)) & 1;
                e = q_mul(e, bit ? point[k] : q_sub(q_from_m(1), point[k]));
            }
            acc = q_add(acc, q_mul_m(e, (uint32_t)(in_u64(&in) % MP)));
        }
        if (!q_eq(acc, rms_sq_eval)) return 0;
    } else if (has_rows != 0) {
        return 0;
    } else if (((size_t)1 << num_vars) / next_pow2(dim) > 1) {
        return 0;
    }
    ch_mix_sf(ch, input_eval);
    ch_mix_sf(ch, output_eval);
    if (out_input_eval) q_store(out_input_eval, input_eval);
    if (consumed) *consumed = in.pos;
    return (exact ? in.pos == len : in.pos <= len) && !in.bad;
}

int orc_verify_rmsnorm(const uint64_t *calldata, size_t len, size_t dim, const uint32_t *claim_point,
                       size_t n_point, const uint32_t claim_value[4], orc_channel *ch,
                       uint32_t out_input_eval[4]) {
    return orc_verify_rmsnorm_impl(NULL, NULL, 1, calldata, len, dim, claim_point, n_point, claim_value, ch, out_input_eval);
}

/* ---------------------------------------------------------------------------
 * Aggregated weight binding (crypto/aggregated_opening.rs).
 * ------------------------------------------------------------------------- */

typedef struct {
    unsigned sb, n_max, n_global;
    size_t m_padded;
} agg_cfg;

/* AggregatedBindingConfig::from_claims (aggregated_opening.rs:68-97) */
static int agg_config(const orc_weight_claim *c, size_t m, agg_cfg *cfg, unsigned *nv) {
    if (m == 0 || m > 256) return 1;
    cfg->n_max = 0;
    for (size_t i = 0; i < m; i++) {
        if (!c[i].rows || !c[i].cols) return 1;
        nv[i] = ilog2(next_pow2(c[i].rows) * next_pow2(c[i].cols));
        if (nv[i] == 0 || nv[i] > 30) return 1;
        if (nv[i] > cfg->n_max) cfg->n_max = nv[i];
    }
    cfg->m_padded = next_pow2(m);
    cfg->sb = ilog2(cfg->m_padded);
    cfg->n_global = cfg->sb + cfg->n_max;
    return 0;
}

/* build_super_root (aggregated_opening.rs:181-227): per-matrix roots extended to n_max
 * with zero-tree roots, zero-tree padding to m_padded, a Merkle tree on top. */
static void agg_super_root(const orc_weight_claim *c, size_t m, const unsigned *nv, const agg_cfg *cfg,
                           fe *subtree /* m_padded */, fe *root) {
    fe zr[32];
    felt_of_qm31(&zr[0], q_from_m(0));
    for (unsigned l = 1; l <= cfg->n_max; l++) pos_hash(&zr[l], &zr[l - 1], &zr[l - 1]);
    for (size_t i = 0; i < cfg->m_padded; i++) {
        if (i >= m) {
            subtree[i] = zr[cfg->n_max];
            continue;
        }
        fe_from_canon(&subtree[i], c[i].commitment);
        for (unsigned l = nv[i]; l < cfg->n_max; l++) pos_hash(&subtree[i], &subtree[i], &zr[l]);
    }
    size_t w = cfg->m_padded;
    fe *cur = (fe *)malloc(sizeof(fe) * w);
    memcpy(cur, subtree, sizeof(fe) * w);
    while (w > 1) {
        for (size_t i = 0; i < w / 2; i++) pos_hash(&cur[i], &cur[2 * i], &cur[2 * i + 1]);
        w /= 2;
    }
    *root = cur[0];
    free(cur);
}

/* global_point (aggregated_opening.rs:328-358): selector bits of matrix_index (MSB first),
 * zeros up to n_max, then the claim's evaluation point. */
static void agg_global_point(const orc_weight_claim *c, unsigned nv, const agg_cfg *cfg, q31 *g) {
    for (unsigned j = 0; j < cfg->sb; j++) g[j] = q_from_m((uint32_t)((c->matrix_index >> (cfg->sb - 1 - j)) & 1));
    for (unsigned j = 0; j < cfg->n_max - nv; j++) g[cfg->sb + j] = q_from_m(0);
    for (unsigned j = 0; j < nv; j++) g[cfg->sb + cfg->n_max - nv + j] = q_load(c->eval_point + 4 * j);
}

/* eval_unified_oracle (aggregated_opening.rs:364-392): sum_k sel(k, t_sel) W_k(last n_k of t_local). */
static q31 agg_oracle(const q31 *t, q31 *const *mles, const unsigned *nv, size_t m, const agg_cfg *cfg) {
    q31 res = q_from_m(0), one = q_from_m(1);
    for (size_t k = 0; k < m; k++) {
        q31 w = one;
        for (unsigned j = 0; j < cfg->sb; j++) {
            int bit = (int)((k >> (cfg->sb - 1 - j)) & 1);
            w = q_mul(w, bit ? t[j] : q_sub(one, t[j]));
        }
        if (q_eq(w, q_from_m(0))) continue;
        q31 v = mle_eval_copy(mles[k], (size_t)1 << nv[k], t + cfg->sb + cfg->n_max - nv[k], nv[k]);
        res = q_add(res, q_mul(w, v));
    }
    return res;
}

static q31 *weight_mle_col_major(const orc_weight_claim *c) {
    size_t pr = next_pow2(c->rows), pc = next_pow2(c->cols);
    q31 *v = (q31 *)calloc(pr * pc, sizeof(q31));
    for (size_t i = 0; i < c->rows; i++)
        for (size_t j = 0; j < c->cols; j++) v[j * pr + i] = q_from_m(m_red64(c->weight[i * c->cols + j]));
    return v;
}

void orc_weight_commitment(const uint32_t *weight, size_t rows, size_t cols, uint64_t out[4], int threads) {
    orc_weight_claim c = {weight, rows, cols, 0, NULL, {0, 0, 0, 0}, {0, 0, 0, 0}};
    q31 *v = weight_mle_col_major(&c);
    orc_merkle_root_qm31((const uint32_t *)v, next_pow2(rows) * next_pow2(cols), out, threads);
    free(v);
}

int orc_prove_aggregated_binding(const orc_weight_claim *claims, size_t m, orc_channel *ch, size_t n_queries,
                                 uint64_t *calldata, size_t cap, size_t *out_len, int threads) {
    oracle_init();
    agg_cfg cfg;
    unsigned nv[256];
    if (agg_config(claims, m, &cfg, nv)) return 1;
    const unsigned n = cfg.n_global;
    q31 *mles[256];
    for (size_t k = 0; k < m; k++) mles[k] = weight_mle_col_major(&claims[k]);
    fe *subtree = (fe *)malloc(sizeof(fe) * cfg.m_padded), root;
    agg_super_root(claims, m, nv, &cfg, subtree, &root);
    orc_ch_mix_felt(ch, root.v);
    /* draw_beta_weights (aggregated_opening.rs:395-405) */
    q31 rho = ch_draw_qm31(ch), *beta = (q31 *)malloc(sizeof(q31) * m), pw = q_from_m(1);
    for (size_t i = 0; i < m; i++) {
        beta[i] = pw;
        pw = q_mul(pw, rho);
    }
    q31 *g = (q31 *)malloc(sizeof(q31) * m * n), *pre = (q31 *)malloc(sizeof(q31) * m);
    for (size_t i = 0; i < m; i++) {
        agg_global_point(&claims[i], nv[i], &cfg, g + i * n);
        pre[i] = q_from_m(1);
    }
    /* mismatch_sumcheck (aggregated_opening.rs:412-510, 517-625) */
    q31 *chal = (q31 *)malloc(sizeof(q31) * (n + 1)), *pt = (q31 *)malloc(sizeof(q31) * n);
    q31 *rp = (q31 *)malloc(sizeof(q31) * 3 * n), one = q_from_m(1);
    uint32_t inv2 = m_inv(2);
    for (unsigned j = 0; j < n; j++) {
        q31 s[3];
        for (uint32_t x = 0; x < 3; x++) {
            q31 tot = q_from_m(0), X = q_from_m(x);
            for (size_t i = 0; i < m; i++) {
                const q31 *gi = g + i * n;
                q31 eqr = q_add(q_mul(gi[j], X), q_mul(q_sub(one, gi[j]), q_sub(one, X)));
                memcpy(pt, chal, sizeof(q31) * j);
                pt[j] = X;
                memcpy(pt + j + 1, gi + j + 1, sizeof(q31) * (n - j - 1));
                q31 mis = q_sub(agg_oracle(pt, mles, nv, m, &cfg), q_load(claims[i].expected_value));
                tot = q_add(tot, q_mul(q_mul(q_mul(beta[i], pre[i]), eqr), mis));
            }
            s[x] = tot;
        }
        q31 c0 = s[0], c2 = q_mul_m(q_add(q_sub(s[0], q_add(s[1], s[1])), s[2]), inv2);
        q31 c1 = q_sub(q_sub(s[1], s[0]), c2);
        uint32_t cw[12];
        q_store(cw, c0);
        q_store(cw + 4, c1);
        q_store(cw + 8, c2);
        orc_ch_mix_poly_coeffs(ch, cw);
        rp[3 * j] = c0;
        rp[3 * j + 1] = c1;
        rp[3 * j + 2] = c2;
        chal[j] = ch_draw_qm31(ch);
        for (size_t i = 0; i < m; i++) {
            q31 gv = g[i * n + j];
            pre[i] = q_mul(pre[i], q_add(q_mul(chal[j], gv), q_mul(q_sub(one, chal[j]), q_sub(one, gv))));
        }
    }
    q31 oracle_eval = agg_oracle(chal, mles, nv, m, &cfg);
    {
        uint32_t w[4];
        q_store(w, oracle_eval);
        orc_ch_mix_felts(ch, w, 1);
    }
    /* serialize_aggregated_binding_proof (cairo_serde.rs:3884-3921) */
    felt_out o = {calldata, 0, cap, 0};
    out_u64(&o, cfg.sb);
    out_u64(&o, cfg.n_max);
    out_u64(&o, cfg.m_padded);
    out_u64(&o, cfg.n_global);
    out_u64(&o, m);
    out_u64(&o, n);
    for (unsigned j = 0; j < 3 * n; j++) out_qm31(&o, rp[j]);
    out_qm31(&o, oracle_eval);
    out_push(&o, &root);
    out_u64(&o, cfg.m_padded);
    for (size_t i = 0; i < cfg.m_padded; i++) out_push(&o, &subtree[i]);
    /* virtual MLE (build_virtual_mle, aggregated_opening.rs:631-652) opened at the challenges */
    size_t total = (size_t)1 << n, slot = (size_t)1 << cfg.n_max;
    q31 *virt = (q31 *)calloc(total, sizeof(q31));
    for (size_t k = 0; k < m; k++) memcpy(virt + k * slot, mles[k], sizeof(q31) << nv[k]);
    uint64_t com[4];
    size_t olen = 0;
    int rc = orc_prove_mle_opening((const uint32_t *)virt, n, (const uint32_t *)chal, ch, n_queries, com,
                                   calldata ? calldata + 4 * (o.len < cap ? o.len : cap) : NULL,
                                   o.len < cap ? cap - o.len : 0, &olen, threads);
    if (rc == 0 && memcmp(com, root.v, 32) != 0) rc = 4; /* commitments do not match the weights */
    *out_len = o.len + olen;
    free(virt);
    free(rp);
    free(pt);
    free(chal);
    free(pre);
    free(g);
    free(beta);
    free(subtree);
    for (size_t k = 0; k < m; k++) free(mles[k]);
    if (rc) return rc;
    return (o.overflow || *out_len > cap) ? 2 : 0;
}

int orc_verify_aggregated_binding(const orc_weight_claim *claims, size_t m, const uint64_t *calldata, size_t len,
                                  orc_channel *ch, size_t n_queries) {
    oracle_init();
    agg_cfg cfg;
    unsigned nv[256];
    if (agg_config(claims, m, &cfg, nv)) return 0;
    felt_in in = {calldata, len, 0, 0};
    if (in_u64(&in) != cfg.sb || in_u64(&in) != cfg.n_max || in_u64(&in) != cfg.m_padded ||
        in_u64(&in) != cfg.n_global || in_u64(&in) != m)
        return 0;
    const unsigned n = cfg.n_global;
    if (in_u64(&in) != n || in.bad) return 0;
    size_t rounds_at = in.pos;
    in.pos += 12 * (size_t)n;
    q31 oracle_eval = in_qm31(&in);
    fe root_s, root, *subtree = (fe *)malloc(sizeof(fe) * cfg.m_padded);
    in_felt(&in, &root_s);
    agg_super_root(claims, m, nv, &cfg, subtree, &root);
    int ok = !memcmp(root.v, root_s.v, 32) && in_u64(&in) == cfg.m_padded;
    for (size_t i = 0; ok && i < cfg.m_padded; i++) {
        fe f;
        in_felt(&in, &f);
        ok = !memcmp(f.v, subtree[i].v, 32);
    }
    free(subtree);
    if (!ok || in.bad) return 0;
    /* verify_aggregated_binding (aggregated_opening.rs:1774-1905), legacy single-opening path */
    orc_ch_mix_felt(ch, root.v);
    q31 rho = ch_draw_qm31(ch), *beta = (q31 *)malloc(sizeof(q31) * m), pw = q_from_m(1);
    for (size_t i = 0; i < m; i++) {
        beta[i] = pw;
        pw = q_mul(pw, rho);
    }
    felt_in rin = {calldata, len, rounds_at, 0};
    q31 cur = q_from_m(0), *chal = (q31 *)malloc(sizeof(q31) * (n + 1));
    for (unsigned j = 0; j < n && ok; j++) {
        q31 c0 = in_qm31(&rin), c1 = in_qm31(&rin), c2 = in_qm31(&rin);
        if (!q_eq(q_add(c0, q_add(q_add(c0, c1), c2)), cur)) ok = 0;
        uint32_t cw[12];
        q_store(cw, c0);
        q_store(cw + 4, c1);
        q_store(cw + 8, c2);
        orc_ch_mix_poly_coeffs(ch, cw);
        chal[j] = ch_draw_qm31(ch);
        cur = q_add(c0, q_mul(chal[j], q_add(c1, q_mul(chal[j], c2))));
    }
    if (ok) {
        q31 *g = (q31 *)malloc(sizeof(q31) * n), vs = q_from_m(0);
        for (size_t i = 0; i < m; i++) {
            agg_global_point(&claims[i], nv[i], &cfg, g);
            vs = q_add(vs, q_mul(q_mul(beta[i], eq_eval(g, chal, n)),
                                 q_sub(oracle_eval, q_load(claims[i].expected_value))));
        }
        free(g);
        ok = q_eq(vs, cur);
    }
    if (ok) {
        uint32_t w[4];
        q_store(w, oracle_eval);
        orc_ch_mix_felts(ch, w, 1);
        uint32_t fin[4];
        ok = orc_verify_mle_opening(root.v, calldata + 4 * in.pos, len - in.pos, (const uint32_t *)chal, n, ch,
                                    n_queries, fin);
    }
    free(chal);
    free(beta);
    return ok;
}

/* ---------------------------------------------------------------------------
 * Piecewise-linear algebraic activation (the default non-ReLU activation path).
 * ------------------------------------------------------------------------- */

/* sigmoid_integer (components/integer_math.rs:288-315), C integer division (truncating, as Rust). */
static int64_t pw_sigmoid(int64_t x, int64_t scale) {
    int64_t x5 = scale * 5, x25 = scale * 5 / 2;
    if (x <= -x5) return 0;
    if (x >= x5) return scale;
    if (x <= -x25) {
        int64_t dx = x + x5;
        return (dx * 28) / (1000 * (x5 - x25) / scale);
    }
    if (x >= x25) {
        int64_t dx = x - x25;
        int64_t base = scale * 93 / 100;
        return base + (dx * 7) / (100 * (x5 - x25) / scale);
    }
    return scale / 2 + x / 4;
}

/* apply_activation_integer (components/integer_math.rs:212-263); act: 0 ReLU, 1 GELU,
 * 2 Sigmoid, 3 Softmax-exp, 4 SiLU. */
uint32_t orc_activation_integer(int act, uint32_t val) {
    const uint32_t P31 = 0x7FFFFFFFu, half_p = P31 / 2;
    int64_t s = val <= half_p ? (int64_t)val : (int64_t)val - (int64_t)P31;
    int64_t scale = half_p, r;
    switch (act) {
    case 0: r = s > 0 ? s : 0; break;
    case 1: { /* gelu_integer, integer_math.rs:268-276 */
        int64_t arg = (s * 1702) / 1000;
        r = (s * pw_sigmoid(arg, scale)) / scale;
        break;
    }
    case 2: r = pw_sigmoid(s, scale); break;
    case 3: { /* exp_activation_integer, integer_math.rs:318-331 */
        int64_t res = scale, term = s;
        res += term;
        for (int64_t k = 2; k <= 8; k++) {
            term = (term * s) / (k * scale);
            res += term;
            if ((term < 0 ? -term : term) < 2) break;
        }
        r = res > 0 ? res : 0;
        break;
    }
    case 4: r = (s * pw_sigmoid(s, scale)) / scale; break;
    default: r = s;
    }
    return (uint32_t)(((r % (int64_t)P31) + (int64_t)P31) % (int64_t)P31);
}

/* PiecewiseLinearCoeffs::for_activation (components/activation.rs:269-316): 16 segments of
 * width 2^27; type tag 1..5 (ReLU..SiLU). */
int orc_piecewise_coeffs(int tag, uint32_t slopes[16], uint32_t intercepts[16]) {
    if (tag < 1 || tag > 5) return 1;
    const uint32_t w = 1u << 27;
    for (uint32_t i = 0; i < 16; i++) {
        uint32_t xs = i * w, xe = i == 15 ? MP - 1 : (i + 1) * w - 1;
        uint32_t ys = orc_activation_integer(tag - 1, xs), ye = orc_activation_integer(tag - 1, xe);
        uint32_t slope = m_mul(m_sub(ye, ys), m_inv(m_sub(xe, xs)));
        slopes[i] = slope;
        intercepts[i] = m_sub(ys, m_mul(slope, xs));
    }
    return 0;
}

#define PW_NV 23 /* eq, input, output, 16 indicators, 4 segment bits */

/* compute_piecewise_eq_sum_at_t (gkr/prover.rs:6935-6998) */
static q31 pw_sum_at(q31 *const *v, size_t mid, uint32_t t, const uint32_t *slopes, const uint32_t *icpt,
                     const q31 *ep) {
    q31 sum = q_from_m(0), one = q_from_m(1);
    for (size_t j = 0; j < mid; j++) {
        q31 x[PW_NV];
        for (int k = 0; k < PW_NV; k++) x[k] = q_add(v[k][j], q_mul_m(q_sub(v[k][mid + j], v[k][j]), t));
        q31 ind_sum = q_from_m(0), pv = q_from_m(0);
        for (int i = 0; i < 16; i++) {
            ind_sum = q_add(ind_sum, x[3 + i]);
            pv = q_add(pv, q_mul(x[3 + i], q_add(q_mul_m(x[1], slopes[i]), q_from_m(icpt[i]))));
        }
        q31 h = q_mul(ep[0], q_sub(x[2], pv));
        h = q_add(h, q_mul(ep[1], q_sub(ind_sum, one)));
        for (int i = 0; i < 16; i++) h = q_add(h, q_mul(q_mul(ep[2 + i], x[3 + i]), q_sub(one, x[3 + i])));
        q31 bs = q_from_m(0), is = q_from_m(0);
        for (int k = 0; k < 4; k++) bs = q_add(bs, q_mul_m(x[19 + k], 1u << k));
        for (int i = 0; i < 16; i++) is = q_add(is, q_mul_m(x[3 + i], (uint32_t)i));
        h = q_add(h, q_mul(ep[18], q_sub(bs, is)));
        for (int k = 0; k < 4; k++) h = q_add(h, q_mul(q_mul(ep[19 + k], x[19 + k]), q_sub(one, x[19 + k])));
        sum = q_add(sum, q_mul(x[0], h));
    }
    return sum;
}

/* reduce_activation_layer_piecewise (gkr/prover.rs:7006-7228), serialized as the
 * LayerProof::Activation record (cairo_serde.rs:1355-1387) with the piecewise proof. */
int orc_reduce_activation_piecewise(const uint32_t *input, size_t rows, size_t cols, int tag,
                                    const uint32_t *claim_point, size_t n_point, const uint32_t claim_value[4],
                                    orc_channel *ch, uint64_t *calldata, size_t cap, size_t *out_len,
                                    uint32_t out_input_eval[4], uint32_t *out_point) {
    oracle_init();
    uint32_t slopes[16], icpt[16];
    if (orc_piecewise_coeffs(tag, slopes, icpt)) return 1;
    size_t pr = next_pow2(rows), pc = next_pow2(cols), n = pr * pc;
    unsigned num_vars = ilog2(n);
    if (num_vars == 0 || n_point < num_vars) return 1;
    q31 *v[PW_NV];
    for (int k = 0; k < PW_NV; k++) v[k] = (q31 *)calloc(n, sizeof(q31));
    for (size_t i = 0; i < pr; i++)
        for (size_t j = 0; j < pc; j++) {
            size_t idx = i * pc + j;
            uint32_t x = (i < rows && j < cols) ? m_red64(input[i * cols + j]) : 0;
            uint32_t seg = x >> 27;
            if (seg > 15) seg = 15;
            v[1][idx] = q_from_m(x);
            v[2][idx] = q_from_m(m_add(m_mul(slopes[seg], x), icpt[seg]));
            v[3 + seg][idx] = q_from_m(1);
            for (int k = 0; k < 4; k++) v[19 + k][idx] = q_from_m((seg >> k) & 1);
        }
    orc_ch_mix_u64(ch, 0x50575F414354ull);
    orc_ch_mix_u64(ch, (uint64_t)tag);
    orc_ch_mix_u64(ch, num_vars);
    ch_mix_sf(ch, q_load(claim_value));
    q31 eta = ch_draw_qm31(ch), ep[23];
    ep[0] = q_from_m(1);
    for (int i = 1; i < 23; i++) ep[i] = q_mul(ep[i - 1], eta);
    q31 *eq = lagrange_basis((const q31 *)claim_point, num_vars);
    memcpy(v[0], eq, sizeof(q31) * n);
    free(eq);
    q31 *rp = (q31 *)malloc(sizeof(q31) * 4 * num_vars), *chal = (q31 *)malloc(sizeof(q31) * num_vars);
    uint32_t inv2 = m_inv(2), inv6 = m_inv(6);
    size_t cur = n;
    for (unsigned r = 0; r < num_vars; r++) {
        size_t mid = cur / 2;
        q31 s0 = pw_sum_at(v, mid, 0, slopes, icpt, ep), s1 = pw_sum_at(v, mid, 1, slopes, icpt, ep);
        q31 s2 = pw_sum_at(v, mid, 2, slopes, icpt, ep), s3 = pw_sum_at(v, mid, 3, slopes, icpt, ep);
        q31 d01 = q_sub(s1, s0), d12 = q_sub(s2, s1), d23 = q_sub(s3, s2);
        q31 d012 = q_mul_m(q_sub(d12, d01), inv2);
        q31 d0123 = q_mul_m(q_add(q_sub(q_sub(d23, d12), d12), d01), inv6);
        q31 c0 = s0, c1 = q_add(q_sub(d01, d012), q_mul_m(d0123, 2)), c2 = q_sub(d012, q_mul_m(d0123, 3));
        q31 c3 = d0123;
        rp[4 * r] = c0;
        rp[4 * r + 1] = c1;
        rp[4 * r + 2] = c2;
        rp[4 * r + 3] = c3;
        mix_deg3(ch, c0, c1, c2, c3);
        chal[r] = ch_draw_qm31(ch);
        for (int k = 0; k < PW_NV; k++) fold_vec(v[k], mid, chal[r]);
        cur = mid;
    }
    for (int k = 1; k < PW_NV; k++) ch_mix_sf(ch, v[k][0]);
    felt_out o = {calldata, 0, cap, 0};
    fe zero;
    fe_u64(&zero, 0);
    out_u64(&o, 3);
    out_u64(&o, (uint64_t)tag);
    out_qm31(&o, v[1][0]);
    out_qm31(&o, q_load(claim_value));
    out_push(&o, &zero);
    out_u64(&o, 0); /* no LogUp proof */
    out_u64(&o, 0); /* no multiplicity sumcheck */
    out_u64(&o, 0); /* no activation product proof */
    out_u64(&o, 1); /* piecewise proof */
    out_u64(&o, num_vars);
    for (unsigned r = 0; r < num_vars; r++) {
        out_qm31(&o, rp[4 * r]);
        out_qm31(&o, rp[4 * r + 2]);
        out_qm31(&o, rp[4 * r + 3]);
    }
    out_qm31(&o, v[1][0]);
    out_qm31(&o, v[2][0]);
    for (int i = 0; i < 16; i++) out_qm31(&o, v[3 + i][0]);
    out_u64(&o, 1); /* segment bits present */
    for (int k = 0; k < 4; k++) out_qm31(&o, v[19 + k][0]);
    *out_len = o.len;
    if (out_input_eval) q_store(out_input_eval, v[1][0]);
    if (out_point) memcpy(out_point, chal, sizeof(q31) * num_vars);
    for (int k = 0; k < PW_NV; k++) free(v[k]);
    free(rp);
    free(chal);
    return o.overflow ? 2 : 0;
}

/* verify_piecewise_activation_reduction (gkr/verifier.rs:3298-3480) on such a record. */
static int orc_verify_activation_piecewise_impl(size_t *consumed, uint32_t *out_point, int exact, const uint64_t *calldata, size_t len, const uint32_t *claim_point,
                                    size_t n_point, const uint32_t claim_value[4], orc_channel *ch,
                                    uint32_t out_input_eval[4]) {
    oracle_init();
    felt_in in = {calldata, len, 0, 0};
    if (in_u64(&in) != 3) return 0;
    int tag = (int)in_u64(&in);
    uint32_t slopes[16], icpt[16];
    if (orc_piecewise_coeffs(tag, slopes, icpt)) return 0;
    q31 input_eval = in_qm31(&in), output_eval = in_qm31(&in);
    fe tcom;
    in_felt(&in, &tcom);
    if (tcom.v[0] | tcom.v[1] | tcom.v[2] | tcom.v[3]) return 0;
    if (in_u64(&in) != 0 || in_u64(&in) != 0 || in_u64(&in) != 0 || in_u64(&in) != 1) return 0;
    size_t nv = in_u64(&in);
    if (nv == 0 || nv > 40 || nv > n_point || in.bad) return 0;
    if (!q_eq(output_eval, q_load(claim_value))) return 0;
    orc_ch_mix_u64(ch, 0x50575F414354ull);
    orc_ch_mix_u64(ch, (uint64_t)tag);
    orc_ch_mix_u64(ch, nv);
    ch_mix_sf(ch, q_load(claim_value));
    q31 eta = ch_draw_qm31(ch), ep[23], one = q_from_m(1);
    ep[0] = one;
    for (int i = 1; i < 23; i++) ep[i] = q_mul(ep[i - 1], eta);
    q31 chal[40];
    q31 cur = replay_deg3(ch, &in, nv, q_from_m(0), chal);
    q31 inp = in_qm31(&in), out = in_qm31(&in), ind[16], sb[4];
    for (int i = 0; i < 16; i++) ind[i] = in_qm31(&in);
    if (in_u64(&in) != 1) return 0;
    for (int k = 0; k < 4; k++) sb[k] = in_qm31(&in);
    if (in.bad || !q_eq(inp, input_eval)) return 0;
    q31 pv = q_from_m(0), isum = q_from_m(0);
    for (int i = 0; i < 16; i++) {
        isum = q_add(isum, ind[i]);
        pv = q_add(pv, q_mul(ind[i], q_add(q_mul_m(inp, slopes[i]), q_from_m(icpt[i]))));
    }
    q31 h = q_mul(ep[0], q_sub(out, pv));
    h = q_add(h, q_mul(ep[1], q_sub(isum, one)));
    for (int i = 0; i < 16; i++) h = q_add(h, q_mul(q_mul(ep[2 + i], ind[i]), q_sub(one, ind[i])));
    q31 bs = q_from_m(0), is = q_from_m(0);
    for (int k = 0; k < 4; k++) bs = q_add(bs, q_mul_m(sb[k], 1u << k));
    for (int i = 0; i < 16; i++) is = q_add(is, q_mul_m(ind[i], (uint32_t)i));
    h = q_add(h, q_mul(ep[18], q_sub(bs, is)));
    for (int k = 0; k < 4; k++) h = q_add(h, q_mul(q_mul(ep[19 + k], sb[k]), q_sub(one, sb[k])));
    if (!q_eq(cur, q_mul(eq_eval((const q31 *)claim_point, chal, nv), h))) return 0;
    ch_mix_sf(ch, inp);
    ch_mix_sf(ch, out);
    for (int i = 0; i < 16; i++) ch_mix_sf(ch, ind[i]);
    for (int k = 0; k < 4; k++) ch_mix_sf(ch, sb[k]);
    if (out_input_eval) q_store(out_input_eval, input_eval);
    if (out_point) memcpy(out_point, chal, sizeof(q31) * nv);
    if (consumed) *consumed = in.pos;
    return (exact ? in.pos == len : in.pos <= len) && !in.bad;
}

int orc_verify_activation_piecewise(const uint64_t *calldata, size_t len, const uint32_t *claim_point,
                                    size_t n_point, const uint32_t claim_value[4], orc_channel *ch,
                                    uint32_t out_input_eval[4]) {
    return orc_verify_activation_piecewise_impl(NULL, NULL, 1, calldata, len, claim_point, n_point, claim_value, ch, out_input_eval);
}

/* ---------------------------------------------------------------------------
 * ReLU (algebraic product + bit decomposition) and the GKR walk over a chain of
 * MatMul / ReLU layers.
 * ------------------------------------------------------------------------- */

#define RELU_BITS 30

/* compute_combined_activation_eq_sum_at_t (gkr/prover.rs:6642-6690) */
static q31 relu_sum_at(q31 *const *v, size_t mid, uint32_t t, const q31 *ep) {
    q31 sum = q_from_m(0), one = q_from_m(1);
    for (size_t i = 0; i < mid; i++) {
        q31 x[3 + RELU_BITS];
        for (int k = 0; k < 3 + RELU_BITS; k++) x[k] = q_add(v[k][i], q_mul_m(q_sub(v[k][mid + i], v[k][i]), t));
        q31 eq = x[0], in = x[1], b = x[2];
        q31 h = q_mul(q_mul(ep[0], b), in);
        h = q_add(h, q_mul(q_mul(ep[1], b), q_sub(one, b)));
        q31 bs = q_from_m(0);
        uint32_t pw = 1;
        for (int j = 0; j < RELU_BITS; j++) {
            bs = q_add(bs, q_mul_m(x[3 + j], pw));
            pw = m_add(pw, pw);
        }
        q31 dec = q_sub(q_sub(in, bs), q_mul_m(q_sub(one, b), pw));
        h = q_add(h, q_mul(ep[2], dec));
        for (int j = 0; j < RELU_BITS; j++) h = q_add(h, q_mul(q_mul(ep[3 + j], x[3 + j]), q_sub(one, x[3 + j])));
        sum = q_add(sum, q_mul(eq, h));
    }
    return sum;
}

/* reduce_activation_layer_algebraic (gkr/prover.rs:6700-6890) on the rows x cols activation
 * input; appends the LayerProof::Activation record (cairo_serde.rs:1355-1387, 1190-1235) to o
 * and writes the next claim (point = challenges, value = input evaluation). */
static int relu_reduce(const uint32_t *input, size_t rows, size_t cols, const q31 *point, q31 claim_value,
                       orc_channel *ch, felt_out *o, q31 *next_point, q31 *next_value, int legacy) {
    size_t pr = next_pow2(rows), pc = next_pow2(cols), n = pr * pc;
    unsigned nv = ilog2(n);
    if (nv == 0) return 1;
    const uint32_t half = 1073741823u;
    q31 *v[3 + RELU_BITS];
    for (int k = 0; k < 3 + RELU_BITS; k++) v[k] = (q31 *)calloc(n, sizeof(q31));
    for (size_t i = 0; i < pr; i++)
        for (size_t j = 0; j < pc; j++) {
            size_t idx = i * pc + j;
            uint32_t x = (i < rows && j < cols) ? m_red64(input[i * cols + j]) : 0;
            v[1][idx] = q_from_m(x);
            v[2][idx] = q_from_m(x <= half ? 1 : 0);
            uint32_t low = x <= half ? x : x - (1u << 30);
            for (int b = 0; b < RELU_BITS; b++) v[3 + b][idx] = q_from_m((low >> b) & 1);
        }
    orc_ch_mix_u64(ch, 0x414354);
    ch_mix_sf(ch, claim_value);
    q31 eta = ch_draw_qm31(ch), ep[3 + RELU_BITS];
    ep[0] = q_from_m(1);
    for (int i = 1; i < 3 + RELU_BITS; i++) ep[i] = q_mul(ep[i - 1], eta);
    q31 *eq = lagrange_basis(point, nv);
    memcpy(v[0], eq, sizeof(q31) * n);
    free(eq);
    q31 rp[64][4];
    uint32_t inv2 = m_inv(2), inv6 = m_inv(6);
    size_t cur = n;
    for (unsigned r = 0; r < nv; r++) {
        size_t mid = cur / 2;
        q31 s0 = relu_sum_at(v, mid, 0, ep), s1 = relu_sum_at(v, mid, 1, ep);
        q31 s2 = relu_sum_at(v, mid, 2, ep), s3 = relu_sum_at(v, mid, 3, ep);
        q31 d1 = q_sub(s1, s0);
        q31 d2 = q_mul_m(q_add(q_sub(q_sub(s2, s1), s1), s0), inv2);
        q31 d3 = q_mul_m(q_sub(q_sub(s3, s0), q_mul_m(q_sub(s2, s1), 3)), inv6);
        rp[r][0] = s0;
        rp[r][1] = q_add(q_sub(d1, d2), q_mul_m(d3, 2));
        rp[r][2] = q_sub(d2, q_mul_m(d3, 3));
        rp[r][3] = d3;
        mix_deg3(ch, rp[r][0], rp[r][1], rp[r][2], rp[r][3]);
        next_point[r] = ch_draw_qm31(ch);
        for (int k = 0; k < 3 + RELU_BITS; k++) fold_vec(v[k], mid, next_point[r]);
        cur = mid;
    }
    for (int k = 1; k < 3 + RELU_BITS; k++) ch_mix_sf(ch, v[k][0]);
    fe zero;
    fe_u64(&zero, 0);
    out_u64(o, 3);
    out_u64(o, 1); /* ReLU type tag */
    out_qm31(o, v[1][0]);
    out_qm31(o, claim_value);
    out_push(o, &zero);
    out_u64(o, 0); /* no LogUp proof */
    if (!legacy) out_u64(o, 0); /* no multiplicity sumcheck */
    out_u64(o, 1); /* activation product proof */
    out_u64(o, nv);
    for (unsigned r = 0; r < nv; r++) {
        out_qm31(o, rp[r][0]);
        out_qm31(o, rp[r][2]);
        out_qm31(o, rp[r][3]);
    }
    out_qm31(o, v[1][0]);
    out_qm31(o, v[2][0]);
    out_u64(o, 1);
    out_u64(o, RELU_BITS);
    for (int b = 0; b < RELU_BITS; b++) out_qm31(o, v[3 + b][0]);
    if (!legacy) out_u64(o, 0); /* no piecewise proof */
    *next_value = v[1][0];
    for (int k = 0; k < 3 + RELU_BITS; k++) free(v[k]);
    return 0;
}

/* prove_gkr_with_cache (gkr/prover.rs:1500-2251) for a chain GraphBuilder::new((m, k0))
 * .linear(..)/.activation(ReLU).. in Sequential weight-binding mode, serialized by
 * serialize_gkr_model_proof (cairo_serde.rs:1307-1772). */
/* LayerNorm forward (apply_layernorm_detailed, compiler/prove.rs:977-1060) of one padded row:
 * mean over the first n_active columns, variance masked to the table, rsqrt from the table;
 * centered = x - mean and out = centered * rsqrt over every column. */
static void layernorm_row(const uint32_t *x, size_t pc, size_t n_active, uint32_t inv_n, const uint32_t *table,
                          uint32_t mask, uint32_t *mean_o, uint32_t *var_o, uint32_t *rs_o) {
    uint32_t sum = 0;
    for (size_t j = 0; j < n_active; j++) sum = m_add(sum, x[j]);
    uint32_t mean = m_mul(sum, inv_n), vs = 0;
    for (size_t j = 0; j < n_active; j++) {
        uint32_t d = m_sub(x[j], mean);
        vs = m_add(vs, m_mul(d, d));
    }
    uint32_t var = m_mul(vs, inv_n) & mask;
    *mean_o = mean;
    *var_o = var;
    *rs_o = table[var];
}

/* v1: the record as serialize_gkr_proof_data_only writes it (cairo_serde.rs:1886-1985): the
 * LogUp proof without multiplicities. */
static int layernorm_impl(const uint32_t *input, size_t rows, size_t cols, size_t dim, const uint32_t *claim_point,
                          size_t n_point, const uint32_t claim_value[4], orc_channel *ch, uint64_t *calldata,
                          size_t cap, size_t *out_len, uint32_t out_input_eval[4], int v1) {
    oracle_init();
    if (rows == 0 || cols == 0 || dim == 0) return 1;
    size_t pr = next_pow2(rows), pc = next_pow2(cols), n = pr * pc;
    unsigned num_vars = ilog2(n);
    if (num_vars == 0 || n_point < num_vars) return 1;
    const q31 *point = (const q31 *)claim_point;
    const unsigned log_t = 16;
    const size_t tsize = (size_t)1 << log_t;
    uint32_t *table = (uint32_t *)malloc(4 * tsize);
    orc_rsqrt_table(log_t, table);
    size_t n_active = dim < pc ? dim : pc;
    uint32_t inv_n = m_inv((uint32_t)(n_active % MP));
    q31 *in_mle = mle_row_major(input, rows, cols);
    q31 *mean_v = (q31 *)malloc(sizeof(q31) * n), *var_v = (q31 *)malloc(sizeof(q31) * n);
    q31 *rs_v = (q31 *)malloc(sizeof(q31) * n), *cen = (q31 *)malloc(sizeof(q31) * n);
    q31 *outv = (q31 *)malloc(sizeof(q31) * n);
    uint32_t *row_mean = (uint32_t *)malloc(4 * pr), *row_var = (uint32_t *)malloc(4 * pr);
    uint32_t *mult = (uint32_t *)calloc(tsize, 4), *xrow = (uint32_t *)malloc(4 * pc);
    for (size_t i = 0; i < pr; i++) {
        for (size_t j = 0; j < pc; j++) xrow[j] = in_mle[i * pc + j].a;
        uint32_t mean, var, rs;
        layernorm_row(xrow, pc, n_active, inv_n, table, (uint32_t)tsize - 1, &mean, &var, &rs);
        row_mean[i] = mean;
        row_var[i] = var;
        mult[var] += (uint32_t)pc;
        for (size_t j = 0; j < pc; j++) {
            size_t idx = i * pc + j;
            uint32_t c = m_sub(xrow[j], mean);
            mean_v[idx] = q_from_m(mean);
            var_v[idx] = q_from_m(var);
            rs_v[idx] = q_from_m(rs);
            cen[idx] = q_from_m(c);
            outv[idx] = q_from_m(m_mul(c, rs));
        }
    }
    free(xrow);
    q31 input_eval = mle_eval_copy(in_mle, n, point, num_vars);
    q31 output_eval = mle_eval_copy(outv, n, point, num_vars);
    q31 mean_eval = mle_eval_copy(mean_v, n, point, num_vars);
    q31 rsqrt_eval = mle_eval_copy(rs_v, n, point, num_vars);
    q31 var_eval = mle_eval_copy(var_v, n, point, num_vars);
    free(outv);
    /* Part 0: batched mean / variance plain sumcheck (prover.rs:8040-8090) */
    q31 tot_in = q_from_m(0), tot_c2 = q_from_m(0);
    for (size_t i = 0; i < n; i++) {
        tot_in = q_add(tot_in, in_mle[i]);
        tot_c2 = q_add(tot_c2, q_mul(cen[i], cen[i]));
    }
    orc_ch_mix_u64(ch, 0x4D56);
    orc_ch_mix_u64(ch, n_active);
    ch_mix_sf(ch, tot_in);
    ch_mix_sf(ch, tot_c2);
    q31 eta0 = ch_draw_qm31(ch), eta1 = q_mul(eta0, eta0);
    q31 *mvp = (q31 *)malloc(sizeof(q31) * 4 * (num_vars + 1));
    q31 *pin = (q31 *)malloc(sizeof(q31) * n), *pc_ = (q31 *)malloc(sizeof(q31) * n), *pm = (q31 *)malloc(sizeof(q31) * n);
    memcpy(pin, in_mle, sizeof(q31) * n);
    memcpy(pc_, cen, sizeof(q31) * n);
    memcpy(pm, mean_v, sizeof(q31) * n);
    {
        uint32_t inv2 = m_inv(2);
        size_t cur = n;
        for (unsigned r = 0; r < num_vars; r++) {
            size_t mid = cur / 2;
            q31 s[3];
            for (uint32_t t = 0; t < 3; t++) {
                q31 acc = q_from_m(0);
                for (size_t j = 0; j < mid; j++) {
                    q31 it = q_add(pin[j], q_mul_m(q_sub(pin[mid + j], pin[j]), t));
                    q31 ct = q_add(pc_[j], q_mul_m(q_sub(pc_[mid + j], pc_[j]), t));
                    acc = q_add(acc, q_add(q_mul(eta0, it), q_mul(eta1, q_mul(ct, ct))));
                }
                s[t] = acc;
            }
            q31 dd1 = q_sub(s[1], s[0]);
            q31 dd2 = q_mul_m(q_sub(q_sub(s[2], s[1]), dd1), inv2);
            q31 c0 = s[0], c1 = q_sub(dd1, dd2), c2 = dd2, c3 = q_from_m(0);
            mvp[4 * r] = c0;
            mvp[4 * r + 1] = c1;
            mvp[4 * r + 2] = c2;
            mvp[4 * r + 3] = c3;
            mix_deg3(ch, c0, c1, c2, c3);
            q31 x = ch_draw_qm31(ch);
            fold_vec(pin, mid, x);
            fold_vec(pc_, mid, x);
            fold_vec(pm, mid, x);
            cur = mid;
        }
    }
    q31 mv_in_final = pin[0], mv_mean_final = pm[0];
    ch_mix_sf(ch, mv_in_final);
    ch_mix_sf(ch, mv_mean_final);
    free(pin);
    free(pc_);
    free(pm);
    /* Part 1: eq-sumcheck output = centered x rsqrt, with the centered binding (prover.rs:8092-8170) */
    orc_ch_mix_u64(ch, 0x4C4E);
    ch_mix_sf(ch, mean_eval);
    ch_mix_sf(ch, rsqrt_eval);
    ch_mix_sf(ch, q_load(claim_value));
    q31 *eq = lagrange_basis(point, num_vars);
    q31 *a = (q31 *)malloc(sizeof(q31) * n), *b = (q31 *)malloc(sizeof(q31) * n);
    memcpy(a, cen, sizeof(q31) * n);
    memcpy(b, rs_v, sizeof(q31) * n);
    q31 *lin = (q31 *)malloc(sizeof(q31) * 4 * (num_vars + 1));
    q31 *chal = (q31 *)malloc(sizeof(q31) * (num_vars + 1));
    eq_sumcheck_deg3(ch, eq, a, b, n, num_vars, lin, chal);
    q31 cen_final = a[0], rs_final = b[0];
    q31 cb_in = mle_eval_copy(in_mle, n, chal, num_vars), cb_mean = mle_eval_copy(mean_v, n, chal, num_vars);
    ch_mix_sf(ch, cen_final);
    ch_mix_sf(ch, rs_final);
    ch_mix_sf(ch, cb_in);
    ch_mix_sf(ch, cb_mean);
    free(eq);
    free(a);
    free(b);
    /* Part 2: LogUp of (variance, rsqrt) against the rsqrt table (prover.rs:8172-8300) */
    orc_ch_mix_u64(ch, 0x4C4F47);
    orc_ch_mix_u64(ch, 0x5253);
    q31 gm = ch_draw_qm31(ch), bt = ch_draw_qm31(ch);
    q31 *d = (q31 *)malloc(sizeof(q31) * n), *w = (q31 *)malloc(sizeof(q31) * n);
    q31 trace_sum = q_from_m(0);
    for (size_t i = 0; i < n; i++) {
        d[i] = q_sub(q_sub(gm, var_v[i]), q_mul(bt, rs_v[i]));
        w[i] = q_inv(d[i]);
        trace_sum = q_add(trace_sum, w[i]);
    }
    q31 table_sum = q_from_m(0);
    for (size_t j = 0; j < tsize; j++) {
        if (!mult[j]) continue;
        q31 dj = q_sub(q_sub(gm, q_from_m((uint32_t)j)), q_mul(bt, q_from_m(table[j])));
        table_sum = q_add(table_sum, q_mul_m(q_inv(dj), mult[j] % MP));
    }
    int rc = q_eq(trace_sum, table_sum) ? 0 : 3;
    ch_mix_sf(ch, trace_sum);
    eq = lagrange_basis(point, num_vars);
    q31 *lrp = (q31 *)malloc(sizeof(q31) * 4 * (num_vars + 1));
    eq_sumcheck_deg3(ch, eq, w, d, n, num_vars, lrp, chal);
    q31 w_eval = w[0];
    q31 var_s = mle_eval_copy(var_v, n, chal, num_vars), rs_s = mle_eval_copy(rs_v, n, chal, num_vars);
    q31 *mrp = (q31 *)malloc(sizeof(q31) * 2 * log_t), m_final, m_claim;
    mult_sumcheck(ch, mult, log_t, mrp, &m_final, &m_claim);
    fe tcom;
    table_commitment(0x5253, log_t, &tcom);
    ch_mix_sf(ch, input_eval);
    ch_mix_sf(ch, output_eval);
    /* LayerProof::LayerNorm as serialize_gkr_model_proof writes it (cairo_serde.rs:1389-1483) */
    felt_out o = {calldata, 0, cap, 0};
    out_u64(&o, 4);
    out_qm31(&o, input_eval);
    out_qm31(&o, output_eval);
    out_qm31(&o, mean_eval);
    out_qm31(&o, rsqrt_eval);
    out_push(&o, &tcom);
    out_u64(&o, 0); /* not SIMD-combined */
    out_u64(&o, 1); /* mean / variance sumcheck present */
    out_u64(&o, n_active);
    out_qm31(&o, tot_in);
    out_qm31(&o, tot_c2);
    out_u64(&o, num_vars);
    for (unsigned r = 0; r < num_vars; r++) {
        out_qm31(&o, mvp[4 * r]);
        out_qm31(&o, mvp[4 * r + 2]);
        out_qm31(&o, mvp[4 * r + 3]);
    }
    out_qm31(&o, mv_in_final);
    out_qm31(&o, mv_mean_final);
    out_u64(&o, num_vars);
    for (unsigned r = 0; r < num_vars; r++) {
        out_qm31(&o, lin[4 * r]);
        out_qm31(&o, lin[4 * r + 2]);
        out_qm31(&o, lin[4 * r + 3]);
    }
    out_qm31(&o, cen_final);
    out_qm31(&o, rs_final);
    out_qm31(&o, cb_in);
    out_qm31(&o, cb_mean);
    out_u64(&o, 1); /* LogUp proof present, with its multiplicities */
    out_qm31(&o, trace_sum);
    out_u64(&o, num_vars);
    for (unsigned r = 0; r < num_vars; r++) {
        out_qm31(&o, lrp[4 * r]);
        out_qm31(&o, lrp[4 * r + 2]);
        out_qm31(&o, lrp[4 * r + 3]);
    }
    out_qm31(&o, w_eval);
    out_qm31(&o, var_s);
    out_qm31(&o, rs_s);
    if (v1) {
        out_u64(&o, 0); /* no multiplicities on chain */
    } else {
        out_u64(&o, tsize);
        for (size_t j = 0; j < tsize; j++) out_u64(&o, mult[j]);
    }
    out_mult_sumcheck(&o, mrp, log_t, m_final, m_claim);
    out_qm31(&o, var_eval);
    for (int pass = 0; pass < 2; pass++) {
        const uint32_t *rv = pass ? row_var : row_mean;
        if (pr > 1) {
            out_u64(&o, 1);
            out_u64(&o, pr);
            for (size_t i = 0; i < pr; i++) out_u64(&o, rv[i]);
        } else {
            out_u64(&o, 0);
        }
    }
    *out_len = o.len;
    if (out_input_eval) q_store(out_input_eval, input_eval);
    free(mrp);
    free(lrp);
    free(eq);
    free(d);
    free(w);
    free(chal);
    free(lin);
    free(mvp);
    free(in_mle);
    free(mean_v);
    free(var_v);
    free(rs_v);
    free(cen);
    free(row_mean);
    free(row_var);
    free(mult);
    free(table);
    if (rc) return rc;
    return o.overflow ? 2 : 0;
}

int orc_reduce_layernorm(const uint32_t *input, size_t rows, size_t cols, size_t dim, const uint32_t *claim_point,
                         size_t n_point, const uint32_t claim_value[4], orc_channel *ch, uint64_t *calldata,
                         size_t cap, size_t *out_len, uint32_t out_input_eval[4]) {
    return layernorm_impl(input, rows, cols, dim, claim_point, n_point, claim_value, ch, calldata, cap, out_len,
                          out_input_eval, 0);
}

typedef struct {
    q31 point[64];
    unsigned npt;
    q31 value;
    size_t layer;
} chain_deferred;

#define CHAIN_MAX 1024

/* The chain's forward pass (compiler/prove.rs:1893-1899 and the layer functions it calls):
 * outs[0] = the model input, outs[l + 1] = layer l's output (m x width[l + 1]); src[l] = the
 * layer feeding layer l.  outs, width and src have n_layers + 1 entries; on failure every
 * allocated output is freed.  Returns 0 or 1 (a bad layer list). */
static int chain_forward(const uint32_t *input, size_t m, size_t k0, const orc_chain_layer *layers, size_t n_layers,
                         int threads, uint32_t **outs, size_t *width, long long *src) {
    /* forward pass: outs[0] is the model input, outs[l + 1] layer l's output (m x width[.]) */
    outs[0] = (uint32_t *)malloc(4 * m * k0);
    for (size_t i = 0; i < m * k0; i++) outs[0][i] = m_red64(input[i]);
    width[0] = k0;
    size_t built = 0;
    int rc = 0;
    for (size_t l = 0; l < n_layers && !rc; l++) {
        src[l] = layers[l].src == ORC_CHAIN_PREV ? (long long)l - 1 : layers[l].src;
        if (src[l] < -1 || src[l] >= (long long)l) {
            rc = 1;
            break;
        }
        const uint32_t *x = outs[src[l] + 1];
        size_t w = width[src[l] + 1];
        size_t wo = w;
        if (layers[l].type == 0) {
            if (!layers[l].weight || layers[l].n == 0) {
                rc = 1;
                break;
            }
            wo = layers[l].n;
        } else if (layers[l].type == 3 || layers[l].type == 4) {
            if (layers[l].lhs < 0 || layers[l].lhs >= (long long)l || width[layers[l].lhs + 1] != w) {
                rc = 1;
                break;
            }
        } else if (layers[l].type == 6) {
            if (layers[l].n < 2 || layers[l].n > 5) {
                rc = 1;
                break;
            }
        } else if (layers[l].type != 1 && layers[l].type != 2 && layers[l].type != 5) {
            rc = 1;
            break;
        }
        uint32_t *y = (uint32_t *)malloc(4 * m * wo);
        outs[l + 1] = y;
        width[l + 1] = wo;
        built = l + 1;
        if (layers[l].type == 0) {
            orc_matmul_m31(x, m, w, layers[l].weight, wo, y, threads);
        } else if (layers[l].type == 1) {
            for (size_t i = 0; i < m * w; i++) y[i] = x[i] <= 1073741823u ? x[i] : 0;
        } else if (layers[l].type == 6) {
            /* apply_activation with ActivationType::as_fn (compiler/prove.rs:1893-1899) */
            for (size_t i = 0; i < m * w; i++) y[i] = act_fn((int)layers[l].n, x[i]);
        } else if (layers[l].type == 2) {
            /* apply_rmsnorm_detailed (compiler/prove.rs:1115-1180), dim = the layer width */
            uint32_t *tab = (uint32_t *)malloc(4u << 16);
            orc_rsqrt_table(16, tab);
            uint32_t inv_n = m_inv((uint32_t)(w % MP));
            for (size_t i = 0; i < m; i++) {
                uint32_t sq = 0;
                for (size_t j = 0; j < w; j++) sq = m_add(sq, m_mul(x[i * w + j], x[i * w + j]));
                uint32_t rs = tab[m_mul(sq, inv_n) & 0xFFFF];
                for (size_t j = 0; j < w; j++) y[i * w + j] = m_mul(x[i * w + j], rs);
            }
            free(tab);
        } else if (layers[l].type == 5) {
            /* apply_layernorm_detailed (compiler/prove.rs:977-1060), dim = the layer width */
            uint32_t *tab = (uint32_t *)malloc(4u << 16);
            orc_rsqrt_table(16, tab);
            uint32_t inv_n = m_inv((uint32_t)(w % MP));
            for (size_t i = 0; i < m; i++) {
                uint32_t mean, var, rs;
                layernorm_row(x + i * w, w, w, inv_n, tab, 0xFFFF, &mean, &var, &rs);
                for (size_t j = 0; j < w; j++) y[i * w + j] = m_mul(m_sub(x[i * w + j], mean), rs);
            }
            free(tab);
        } else {
            /* elementwise_add / elementwise_mul (compiler/prove.rs:875-925), lhs op rhs */
            const uint32_t *a = outs[layers[l].lhs + 1];
            for (size_t i = 0; i < m * w; i++) y[i] = layers[l].type == 3 ? m_add(a[i], x[i]) : m_mul(a[i], x[i]);
        }
    }
    if (rc) {
        for (size_t l = 0; l <= built; l++) {
            free(outs[l]);
            outs[l] = NULL;
        }
    }
    return rc;
}

int orc_prove_gkr_chain(const uint32_t *input, size_t m, size_t k0, const orc_chain_layer *layers, size_t n_layers,
                        const uint64_t *policy, size_t n_queries, int flags, uint64_t *calldata, size_t cap,
                        size_t *out_len, uint64_t digest[4], uint64_t io[4], int threads) {
    oracle_init();
    if (n_layers == 0 || n_layers > CHAIN_MAX) return 1;
    uint32_t **outs = (uint32_t **)calloc(n_layers + 1, sizeof(uint32_t *));
    size_t *width = (size_t *)calloc(n_layers + 1, sizeof(size_t));
    long long *src = (long long *)calloc(n_layers + 1, sizeof(long long));
    int rc = chain_forward(input, m, k0, layers, n_layers, threads, outs, width, src);
    if (rc) {
        free(outs);
        free(width);
        free(src);
        return rc;
    }
    orc_channel ch;
    orc_ch_init(&ch);
    orc_ch_mix_u64(&ch, n_layers);
    orc_ch_mix_u64(&ch, m);
    orc_ch_mix_u64(&ch, k0);
    if (policy && (policy[0] | policy[1] | policy[2] | policy[3])) orc_ch_mix_felt(&ch, policy);
    size_t wout = width[n_layers];
    unsigned log_m = ilog2(next_pow2(m));
    unsigned nvo = log_m + ilog2(next_pow2(wout));
    q31 point[64], value;
    for (unsigned i = 0; i < nvo; i++) point[i] = ch_draw_qm31(&ch);
    {
        q31 *omle = mle_row_major(outs[n_layers], m, wout);
        uint32_t val[4];
        orc_evaluate_mle((const uint32_t *)omle, nvo, (const uint32_t *)point, val);
        free(omle);
        value = q_load(val);
    }
    ch_mix_sf(&ch, value);
    unsigned npt = nvo;
    const int v1 = (flags & 2) != 0;
    felt_out lay = {(uint64_t *)malloc(32 * cap), 0, cap, 0};
    size_t n_proofs = 0;
    /* weight claims: the walk's, in walk order */
    q31 **wpts = (q31 **)calloc(n_layers, sizeof(q31 *));
    unsigned *wnv = (unsigned *)calloc(n_layers, sizeof(unsigned));
    q31 *wval = (q31 *)calloc(n_layers, sizeof(q31));
    size_t *widx = (size_t *)calloc(n_layers, sizeof(size_t)), nw = 0;
    chain_deferred *defs = (chain_deferred *)calloc(n_layers, sizeof(chain_deferred));
    size_t nd = 0;
    unsigned char *skip = (unsigned char *)calloc(n_layers, 1);
    for (size_t li = n_layers; li-- > 0 && !rc;) {
        if (skip[li]) continue;
        n_proofs++;
        const uint32_t *x = outs[src[li] + 1];
        size_t w = width[src[li] + 1];
        if (layers[li].type == 0) {
            size_t n = layers[li].n;
            unsigned log_k = ilog2(next_pow2(w)), log_n = ilog2(next_pow2(n));
            uint32_t *rp = (uint32_t *)malloc(48 * (log_k + 1));
            uint32_t fa[4], fb[4];
            q31 nxt[64];
            uint32_t cv[4];
            q_store(cv, value);
            rc = orc_reduce_matmul_gkr((const uint32_t *)point, npt, cv, x, m, w, layers[li].weight, n, &ch, rp, fa, fb,
                                       (uint32_t *)nxt, 1, threads);
            if (rc) {
                free(rp);
                break;
            }
            out_u64(&lay, 0);
            out_u64(&lay, log_k);
            for (unsigned r = 0; r < log_k; r++) {
                out_qm31(&lay, q_load(rp + 12 * r));
                out_qm31(&lay, q_load(rp + 12 * r + 8));
            }
            out_qm31(&lay, q_load(fa));
            out_qm31(&lay, q_load(fb));
            /* weight claim: r_j || sumcheck challenges (prover.rs:1465-1483) */
            wnv[nw] = log_n + log_k;
            wpts[nw] = (q31 *)malloc(sizeof(q31) * (wnv[nw] + 1));
            memcpy(wpts[nw], point + log_m, sizeof(q31) * log_n);
            memcpy(wpts[nw] + log_n, nxt + log_m, sizeof(q31) * log_k);
            wval[nw] = q_load(fb);
            widx[nw] = li;
            nw++;
            memcpy(point, nxt, sizeof(q31) * (log_m + log_k));
            npt = log_m + log_k;
            value = q_load(fa);
            free(rp);
        } else if (layers[li].type == 2) {
            size_t tcap = (1 << 16) + 64 + next_pow2(m) + 40 * (npt + 2), tlen = 0;
            uint64_t *tbuf = (uint64_t *)malloc(32 * tcap);
            uint32_t cv[4], ie[4];
            q_store(cv, value);
            rc = rmsnorm_impl(x, m, w, w, NULL, 0, 0, (const uint32_t *)point, npt, cv, &ch, tbuf, tcap, &tlen, ie,
                              v1);
            for (size_t i = 0; i < tlen && !rc; i++) {
                fe f;
                fe_from_canon(&f, tbuf + 4 * i);
                out_push(&lay, &f);
            }
            free(tbuf);
            value = q_load(ie);
        } else if (layers[li].type == 5) {
            size_t tcap = (1 << 16) + 400 + 2 * next_pow2(m) + 60 * (npt + 2), tlen = 0;
            uint64_t *tbuf = (uint64_t *)malloc(32 * tcap);
            uint32_t cv[4], ie[4];
            q_store(cv, value);
            rc = layernorm_impl(x, m, w, w, (const uint32_t *)point, npt, cv, &ch, tbuf, tcap, &tlen, ie, v1);
            for (size_t i = 0; i < tlen && !rc; i++) {
                fe f;
                fe_from_canon(&f, tbuf + 4 * i);
                out_push(&lay, &f);
            }
            free(tbuf);
            value = q_load(ie);
        } else if (layers[li].type == 6) {
            /* Activation (prover.rs:1765-1790): LogUp when flags bit 2 is set (the reference's
             * STWO_PIECEWISE_ACTIVATION=0), else the piecewise-algebraic reduction */
            const int tag = (int)layers[li].n, logup = (flags & 4) != 0;
            const unsigned nv = ilog2(next_pow2(m) * next_pow2(w));
            size_t tcap = (1 << 21) + 200 + 40 * (size_t)(nv + 2), tlen = 0;
            uint64_t *tbuf = (uint64_t *)malloc(32 * tcap);
            uint32_t cv[4], ie[4];
            q31 nxt[64];
            q_store(cv, value);
            if (npt != nv)
                rc = 1;
            else if (logup)
                rc = orc_reduce_activation_logup(x, m, w, tag, (const uint32_t *)point, npt, cv, &ch, tbuf, tcap,
                                                 &tlen, ie);
            else
                rc = orc_reduce_activation_piecewise(x, m, w, tag, (const uint32_t *)point, npt, cv, &ch, tbuf,
                                                     tcap, &tlen, ie, (uint32_t *)nxt);
            /* on-chain layout (cairo_serde.rs:1862-1890): the LogUp proof without multiplicities */
            const size_t mpos = 29 + 12 * (size_t)nv;
            for (size_t i = 0; i < tlen && !rc; i++) {
                if (v1 && logup && i == mpos) {
                    out_u64(&lay, 0);
                    i += (size_t)tbuf[4 * i];  /* skip the count's multiplicities */
                    continue;
                }
                fe f;
                fe_from_canon(&f, tbuf + 4 * i);
                out_push(&lay, &f);
            }
            free(tbuf);
            if (!rc) {
                if (!logup) memcpy(point, nxt, sizeof(q31) * nv);
                value = q_load(ie);
            }
        } else if (layers[li].type == 1) {
            q31 nxt[64], nval;
            rc = relu_reduce(x, m, w, point, value, &ch, &lay, nxt, &nval, flags & 1);
            npt = ilog2(next_pow2(m) * next_pow2(w));
            memcpy(point, nxt, sizeof(q31) * npt);
            value = nval;
        } else {
            /* binary op: input_layers = [lhs, rhs]; the trunk is the higher layer index */
            const long long il0 = layers[li].lhs, il1 = src[li];
            const uint32_t *lv = outs[il0 + 1];
            q31 *la = mle_row_major(lv, m, w), *ra = mle_row_major(x, m, w);
            size_t n = next_pow2(m) * next_pow2(w);
            unsigned nv = ilog2(n);
            q31 le, re;
            if (npt < nv) {
                rc = 1;
            } else if (layers[li].type == 3) {
                /* reduce_add_layer (prover.rs:6103-6146) + process_add_deferred (prover.rs:1424-1463) */
                le = mle_eval_copy(la, n, point, nv);
                re = mle_eval_copy(ra, n, point, nv);
                ch_mix_sf(&ch, le);
                ch_mix_sf(&ch, re);
                (void)ch_draw_qm31(&ch);
                const int rhs_trunk = il1 > il0;
                out_u64(&lay, 1);
                out_qm31(&lay, le);
                out_qm31(&lay, re);
                out_u64(&lay, rhs_trunk ? 1 : 0);
                chain_deferred *d = &defs[nd++];
                memcpy(d->point, point, sizeof(q31) * npt);
                d->npt = npt;
                d->value = rhs_trunk ? le : re;
                d->layer = (size_t)(rhs_trunk ? il0 : il1);
                value = rhs_trunk ? re : le;
            } else {
                /* reduce_mul_layer (prover.rs:6172-6280) and the branched-Mul claim
                 * (prover.rs:1719-1760): the deferred claim carries rhs_eval, the walk goes on
                 * at the same point with the trunk's evaluation */
                q31 *eq = lagrange_basis(point, nv);
                q31 *rps = (q31 *)malloc(sizeof(q31) * 4 * (nv + 1)), chal[64];
                orc_ch_mix_u64(&ch, 0x4D554C);
                ch_mix_sf(&ch, value);
                eq_sumcheck_deg3(&ch, eq, la, ra, n, nv, rps, chal);
                le = la[0];
                re = ra[0];
                ch_mix_sf(&ch, le);
                ch_mix_sf(&ch, re);
                (void)ch_draw_qm31(&ch);
                out_u64(&lay, 2);
                out_u64(&lay, nv);
                for (unsigned r = 0; r < nv; r++) {
                    out_qm31(&lay, rps[4 * r]);
                    out_qm31(&lay, rps[4 * r + 2]);
                    out_qm31(&lay, rps[4 * r + 3]);
                }
                out_qm31(&lay, le);
                out_qm31(&lay, re);
                free(rps);
                free(eq);
                const int rhs_trunk = il1 > il0;
                const long long sk = rhs_trunk ? il0 : il1;
                chain_deferred *d = &defs[nd++];
                memcpy(d->point, point, sizeof(q31) * npt);
                d->npt = npt;
                d->value = re;
                d->layer = (size_t)sk;
                skip[sk] = 1;
                value = rhs_trunk ? re : le;
            }
            free(la);
            free(ra);
        }
    }
    /* deferred proofs of the skip branches, then their Sequential openings (prover.rs:1918-2047) */
    felt_out dsec = {(uint64_t *)malloc(32 * cap), 0, cap, 0};
    fe *dcoms = (fe *)calloc(n_layers, sizeof(fe));
    uint64_t **dobufs = (uint64_t **)calloc(n_layers, sizeof(uint64_t *));
    size_t *dolens = (size_t *)calloc(n_layers, sizeof(size_t));
    out_u64(&dsec, nd);
    for (size_t i = 0; i < nd && !rc; i++) {
        chain_deferred *d = &defs[i];
        size_t L = d->layer;
        if (layers[L].type != 0) {
            rc = 4;
            break;
        }
        const uint32_t *x = outs[src[L] + 1];
        size_t w = width[src[L] + 1], n = layers[L].n;
        unsigned log_k = ilog2(next_pow2(w)), log_n = ilog2(next_pow2(n));
        ch_mix_sf(&ch, d->value);
        uint32_t *rp = (uint32_t *)malloc(48 * (log_k + 1));
        uint32_t fa[4], fb[4], cv[4];
        q31 nxt[64];
        q_store(cv, d->value);
        rc = orc_reduce_matmul_gkr((const uint32_t *)d->point, d->npt, cv, x, m, w, layers[L].weight, n, &ch, rp, fa,
                                   fb, (uint32_t *)nxt, 1, threads);
        if (rc) {
            free(rp);
            break;
        }
        q31 wp[64];
        memcpy(wp, d->point + log_m, sizeof(q31) * log_n);
        memcpy(wp + log_n, nxt + log_m, sizeof(q31) * log_k);
        q31 *bmle = mle_col_major(layers[L].weight, w, n, threads);
        unsigned nv = log_n + log_k;
        size_t ocap = 64 + (n_queries + 1) * (2 + (size_t)nv * (10 + 2 * (nv + 1)));
        dobufs[i] = (uint64_t *)malloc(32 * ocap);
        felt_out oo = {dobufs[i], 0, ocap, 0};
        prove_opening(bmle, nv, wp, &ch, n_queries, &dcoms[i], &oo, NULL, threads);
        dolens[i] = oo.len;
        free(bmle);
        /* serialize_gkr_proof_data_only's deferred record (cairo_serde.rs:2238-2276) */
        out_qm31(&dsec, d->value);
        out_u64(&dsec, 0);
        out_u64(&dsec, m);
        out_u64(&dsec, w);
        out_u64(&dsec, n);
        out_u64(&dsec, log_k);
        for (unsigned r = 0; r < log_k; r++) {
            out_qm31(&dsec, q_load(rp + 12 * r));
            out_qm31(&dsec, q_load(rp + 12 * r + 8));
        }
        out_qm31(&dsec, q_load(fa));
        out_qm31(&dsec, q_load(fb));
        out_push(&dsec, &dcoms[i]);
        free(rp);
    }
    felt_out o = {calldata, 0, cap, 0};
    if (!rc) {
        /* Sequential weight openings of the walk on the main channel, in walk order */
        fe *coms = (fe *)calloc(nw + 1, sizeof(fe));
        uint64_t **obufs = (uint64_t **)calloc(nw + 1, sizeof(uint64_t *));
        size_t *olens = (size_t *)calloc(nw + 1, sizeof(size_t));
        for (size_t i = 0; i < nw; i++) {
            size_t l = widx[i];
            size_t w = width[src[l] + 1];
            q31 *bmle = mle_col_major(layers[l].weight, w, layers[l].n, threads);
            size_t ocap = 64 + (n_queries + 1) * (2 + (size_t)wnv[i] * (10 + 2 * (wnv[i] + 1)));
            obufs[i] = (uint64_t *)malloc(32 * ocap);
            felt_out oo = {obufs[i], 0, ocap, 0};
            prove_opening(bmle, wnv[i], wpts[i], &ch, n_queries, &coms[i], &oo, NULL, threads);
            olens[i] = oo.len;
            free(bmle);
        }
        if (v1) {
            out_u64(&o, lay.len + dsec.len);
            for (size_t j = 0; j < lay.len && j < lay.cap; j++) out_push(&o, (const fe *)(lay.buf + 4 * j));
            for (size_t j = 0; j < dsec.len && j < dsec.cap; j++) out_push(&o, (const fe *)(dsec.buf + 4 * j));
            out_u64(&o, nw + nd);
            for (size_t i = 0; i < nw; i++) out_push(&o, &coms[i]);
            for (size_t i = 0; i < nd; i++) out_push(&o, &dcoms[i]);
            out_u64(&o, nw + nd);
            for (size_t i = 0; i < nw; i++)
                for (size_t j = 0; j < olens[i]; j++) out_push(&o, (const fe *)(obufs[i] + 4 * j));
            for (size_t i = 0; i < nd; i++)
                for (size_t j = 0; j < dolens[i]; j++) out_push(&o, (const fe *)(dobufs[i] + 4 * j));
        } else {
            out_u64(&o, n_proofs);
            for (size_t j = 0; j < lay.len && j < lay.cap; j++) out_push(&o, (const fe *)(lay.buf + 4 * j));
            /* input claim */
            out_u64(&o, npt);
            for (unsigned i = 0; i < npt; i++) out_qm31(&o, point[i]);
            out_qm31(&o, value);
            out_u64(&o, nw);
            for (size_t i = 0; i < nw; i++) out_push(&o, &coms[i]);
            out_u64(&o, nw);
            for (size_t i = 0; i < nw; i++) {
                out_u64(&o, wnv[i]);
                for (unsigned j = 0; j < wnv[i]; j++) out_qm31(&o, wpts[i][j]);
                out_qm31(&o, wval[i]);
                for (size_t j = 0; j < olens[i]; j++) out_push(&o, (const fe *)(obufs[i] + 4 * j));
            }
        }
        for (size_t i = 0; i < nw; i++) free(obufs[i]);
        free(coms);
        free(obufs);
        free(olens);
        orc_io_commitment(outs[0], m, k0, outs[n_layers], m, wout, io);
        if (!v1) {
            fe iof;
            fe_from_canon(&iof, io);
            out_push(&o, &iof);
        }
        memcpy(digest, ch.digest, 32);
        *out_len = o.len;
    }
    for (size_t i = 0; i < nd; i++) free(dobufs[i]);
    for (size_t i = 0; i < nw; i++) free(wpts[i]);
    for (size_t l = 0; l <= n_layers; l++) free(outs[l]);
    const int overflow = o.overflow || lay.overflow || dsec.overflow;
    free(lay.buf);
    free(dsec.buf);
    free(defs);
    free(outs);
    free(width);
    free(src);
    free(wpts);
    free(wnv);
    free(wval);
    free(widx);
    free(skip);
    free(dcoms);
    free(dobufs);
    free(dolens);
    if (rc) return rc;
    return overflow ? 2 : 0;
}

int orc_reduce_activation_relu(const uint32_t *input, size_t rows, size_t cols, const uint32_t *claim_point,
                               size_t n_point, const uint32_t claim_value[4], orc_channel *ch, uint64_t *calldata,
                               size_t cap, size_t *out_len, uint32_t out_input_eval[4], uint32_t *out_point) {
    oracle_init();
    unsigned nv = ilog2(next_pow2(rows) * next_pow2(cols));
    if (n_point < nv || nv == 0 || nv > 40) return 1;
    felt_out o = {calldata, 0, cap, 0};
    q31 nxt[64], val;
    int rc = relu_reduce(input, rows, cols, (const q31 *)claim_point, q_load(claim_value), ch, &o, nxt, &val, 0);
    if (rc) return rc;
    *out_len = o.len;
    if (out_input_eval) q_store(out_input_eval, val);
    if (out_point) memcpy(out_point, nxt, sizeof(q31) * nv);
    return o.overflow ? 2 : 0;
}

/* ------------------------------------------------------------------------ */
/* Verifier of a chain proof (gkr/verifier.rs: verify_gkr's layer walk)      */
/* ------------------------------------------------------------------------ */

/* verify_gkr for a chain of Linear, Activation (LogUp or piecewise) and RMSNorm layers, proven
 * by orc_prove_gkr_chain / zkml_prove_gkr_chain and serialized by serialize_gkr_model_proof.
 * The verifier recomputes the model output from the input and the weights (the claimed io), then
 * replays the transcript: the prefix and output claim (prover.rs:1516-1561), each layer record
 * from the output to the input with the layer verifiers of this file (the matmul reduction as
 * verifier.rs:2675-2788 checks it), the input claim against the input MLE, every weight's
 * commitment against its column-major MLE, every Sequential opening
 * (mle_opening.rs:1918-2029) at the point the walk produced, and the io commitment.  Returns 1
 * if the proof is accepted; layer kinds other than these three are not handled (returns 0). */
int orc_verify_gkr_chain(const uint32_t *input, size_t m, size_t k0, const orc_chain_layer *layers, size_t n_layers,
                         const uint64_t *policy, size_t n_queries, int flags, const uint64_t *calldata, size_t len,
                         uint64_t digest[4], int threads) {
    oracle_init();
    if (n_layers == 0 || n_layers > CHAIN_MAX) return 0;
    for (size_t l = 0; l < n_layers; l++) {
        const int t = layers[l].type;
        if ((t != 0 && t != 2 && t != 6) || layers[l].src != ORC_CHAIN_PREV) return 0;
    }
    uint32_t **outs = (uint32_t **)calloc(n_layers + 1, sizeof(uint32_t *));
    size_t *width = (size_t *)calloc(n_layers + 1, sizeof(size_t));
    long long *src = (long long *)calloc(n_layers + 1, sizeof(long long));
    int ok = chain_forward(input, m, k0, layers, n_layers, threads, outs, width, src) == 0;
    const int logup = (flags & 4) != 0;
    felt_in in = {calldata, len, 0, 0};
    orc_channel ch;
    orc_ch_init(&ch);
    const size_t wout = width[n_layers];
    const unsigned log_m = ilog2(next_pow2(m));
    const unsigned nvo = log_m + ilog2(next_pow2(wout));
    q31 point[64], value = q_from_m(0);
    unsigned npt = nvo;
    /* weight claims in walk order */
    size_t *wl = (size_t *)calloc(n_layers, sizeof(size_t));
    q31 (*wpt)[64] = (q31(*)[64])calloc(n_layers, sizeof(q31[64]));
    unsigned *wnv = (unsigned *)calloc(n_layers, sizeof(unsigned));
    q31 *wval = (q31 *)calloc(n_layers, sizeof(q31));
    size_t nw = 0;
    if (ok) {
        orc_ch_mix_u64(&ch, n_layers);
        orc_ch_mix_u64(&ch, m);
        orc_ch_mix_u64(&ch, k0);
        if (policy && (policy[0] | policy[1] | policy[2] | policy[3])) orc_ch_mix_felt(&ch, policy);
        for (unsigned i = 0; i < nvo; i++) point[i] = ch_draw_qm31(&ch);
        q31 *omle = mle_row_major(outs[n_layers], m, wout);
        uint32_t val[4];
        orc_evaluate_mle((const uint32_t *)omle, nvo, (const uint32_t *)point, val);
        free(omle);
        value = q_load(val);
        ch_mix_sf(&ch, value);
        if (in_u64(&in) != n_layers) ok = 0;
    }
    for (size_t li = n_layers; li-- > 0 && ok;) {
        const size_t w = width[li];
        const int t = layers[li].type;
        if (t == 0) {
            /* verify_matmul_reduction: mix m, k, n and the claim, the compressed rounds, the final product */
            const size_t n = layers[li].n;
            const unsigned log_k = ilog2(next_pow2(w)), log_n = ilog2(next_pow2(n));
            if (in_u64(&in) != 0 || in_u64(&in) != log_k || npt != log_m + log_n) {
                ok = 0;
                break;
            }
            orc_ch_mix_u64(&ch, m);
            orc_ch_mix_u64(&ch, w);
            orc_ch_mix_u64(&ch, n);
            ch_mix_sf(&ch, value);
            q31 cur = value, chal[64];
            for (unsigned r = 0; r < log_k; r++) {
                q31 c0 = in_qm31(&in), c2 = in_qm31(&in);
                q31 c1 = q_sub(q_sub(cur, q_add(c0, c0)), c2);
                uint32_t coeffs[12];
                q_store(coeffs, c0);
                q_store(coeffs + 4, c1);
                q_store(coeffs + 8, c2);
                orc_ch_mix_poly_coeffs(&ch, coeffs);
                chal[r] = ch_draw_qm31(&ch);
                cur = q_add(c0, q_add(q_mul(c1, chal[r]), q_mul(c2, q_mul(chal[r], chal[r]))));
            }
            q31 fa = in_qm31(&in), fb = in_qm31(&in);
            if (!q_eq(cur, q_mul(fa, fb))) ok = 0;
            ch_mix_sf(&ch, fa);
            ch_mix_sf(&ch, fb);
            /* weight claim r_j || challenges (prover.rs:1465-1483) */
            wl[nw] = li;
            wnv[nw] = log_n + log_k;
            memcpy(wpt[nw], point + log_m, sizeof(q31) * log_n);
            memcpy(wpt[nw] + log_n, chal, sizeof(q31) * log_k);
            wval[nw] = fb;
            nw++;
            memcpy(point + log_m, chal, sizeof(q31) * log_k);
            npt = log_m + log_k;
            value = fa;
        } else {
            /* activation / RMSNorm records: the record's own verifier on the rest of the calldata */
            size_t used = 0;
            uint32_t cv[4], ie[4];
            q31 nxt[64];
            q_store(cv, value);
            const uint64_t *rec = calldata + 4 * in.pos;
            const size_t rest = len - in.pos;
            if (t == 2)
                ok = orc_verify_rmsnorm_impl(&used, NULL, 0, rec, rest, w, (const uint32_t *)point, npt, cv, &ch, ie);
            else if (logup)
                ok = orc_verify_activation_logup_impl(&used, NULL, 0, rec, rest, (const uint32_t *)point, npt, cv, &ch,
                                                      ie);
            else
                ok = orc_verify_activation_piecewise_impl(&used, (uint32_t *)nxt, 0, rec, rest,
                                                          (const uint32_t *)point, npt, cv, &ch, ie);
            if (ok && t == 6 && !logup) memcpy(point, nxt, sizeof(q31) * npt);
            in.pos += used;
            value = q_load(ie);
        }
    }
    /* the input claim: the walk's point and value, and the input MLE there */
    if (ok) {
        if (in_u64(&in) != npt) ok = 0;
        for (unsigned i = 0; i < npt && ok; i++)
            if (!q_eq(in_qm31(&in), point[i])) ok = 0;
        if (ok && !q_eq(in_qm31(&in), value)) ok = 0;
        if (ok) {
            q31 *imle = mle_row_major(outs[0], m, k0);
            uint32_t ev[4];
            orc_evaluate_mle((const uint32_t *)imle, npt, (const uint32_t *)point, ev);
            free(imle);
            if (!q_eq(q_load(ev), value)) ok = 0;
        }
    }
    /* weight commitments, then the Sequential openings in walk order on the main channel */
    fe *coms = (fe *)calloc(nw + 1, sizeof(fe));
    if (ok && in_u64(&in) != nw) ok = 0;
    for (size_t i = 0; i < nw && ok; i++) {
        in_felt(&in, &coms[i]);
        const size_t l = wl[i];
        q31 *bmle = mle_col_major(layers[l].weight, width[l], layers[l].n, threads);
        fe expect;
        merkle_root(bmle, next_pow2(width[l]) * next_pow2(layers[l].n), &expect, threads);
        free(bmle);
        if (memcmp(expect.v, coms[i].v, 32)) ok = 0;
    }
    if (ok && in_u64(&in) != nw) ok = 0;
    for (size_t i = 0; i < nw && ok; i++) {
        if (in_u64(&in) != wnv[i]) ok = 0;
        for (unsigned j = 0; j < wnv[i] && ok; j++)
            if (!q_eq(in_qm31(&in), wpt[i][j])) ok = 0;
        if (ok && !q_eq(in_qm31(&in), wval[i])) ok = 0;
        if (!ok) break;
        const size_t start = in.pos;
        felt_in sub = {calldata + 4 * start, len - start, 0, 0};
        orc_channel probe = ch;
        q31 fv;
        ok = verify_opening(&coms[i], &sub, wpt[i], wnv[i], &probe, n_queries, &fv);
        if (ok) {
            uint32_t fvv[4];
            ok = orc_verify_mle_opening(coms[i].v, calldata + 4 * start, sub.pos, (const uint32_t *)wpt[i], wnv[i],
                                        &ch, n_queries, fvv);
            if (ok && !q_eq(q_load(fvv), wval[i])) ok = 0;
        }
        in.pos = start + sub.pos;
    }
    /* io commitment */
    if (ok) {
        fe iof;
        in_felt(&in, &iof);
        uint64_t io[4];
        orc_io_commitment(outs[0], m, k0, outs[n_layers], m, wout, io);
        if (memcmp(io, iof.v, 32)) ok = 0;
        if (in.pos != len || in.bad) ok = 0;
    }
    if (digest) memcpy(digest, ch.digest, 32);
    for (size_t l = 0; l <= n_layers; l++) free(outs[l]);
    free(outs);
    free(width);
    free(src);
    free(wl);
    free(wpt);
    free(wnv);
    free(wval);
    free(coms);
    return ok;
}
