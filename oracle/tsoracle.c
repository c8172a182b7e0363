/*
 * tsoracle.c -- CPU oracle (TEST INFRASTRUCTURE ONLY) for the TenSafe CKKS
 * hot path.  A line-by-line C restatement of the reference Rust crate
 * `tensafe-he/crates/tensafe-he-core` and the ZeRo-MOAI glue in
 * `demonstrator/server/inference_engine.py`.  Each function cites the
 * reference file:line it follows.  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline / reference arm load this library; the product
 * never does.
 *
 * Build: gcc -O2 -ffp-contract=off (no FMA contraction, no fast-math), glibc
 * libm for cos/sin/log/sqrt/round -- the same calls Rust's f64 methods make on
 * linux-gnu, so the floating-point steps round identically.
 */
#include "tsoracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

typedef unsigned __int128 u128;

#ifndef M_PI
#define M_PI 3.14159265358979323846
#endif
static const double OR_PI = 3.141592653589793; /* std::f64::consts::PI */

/* ======================================================================== */
/* params.rs                                                                */
/* ======================================================================== */

/* params.rs:31-44 -- Barrett constant floor((2^128-1)/q) as (hi, lo). */
void or_modulus_new(uint64_t value, uint32_t bits, or_modulus *out) {
    u128 full = (~(u128)0) / (u128)value;
    out->value = value;
    out->bits = bits;
    out->barrett_hi = (uint64_t)(full >> 64);
    out->barrett_lo = (uint64_t)full;
}

/* params.rs:66-126 (n8192 / n16384 / n32768), selected as for_degree
 * (params.rs:129-136). */
int or_params_preset(uint32_t n, uint64_t *moduli_out, uint32_t *bits_out) {
    static const uint64_t p8192[4] = {1152921504606830593ULL, 1099511480321ULL,
                                      1099510890497ULL, 1152921504606601217ULL};
    static const uint64_t p16384[4] = {1152921504606748673ULL, 1099510054913ULL,
                                       1099508121601ULL, 1152921504606683137ULL};
    static const uint64_t p32768[4] = {1152921504606584833ULL, 1099507695617ULL,
                                       1099506515969ULL, 1152921504598720513ULL};
    static const uint32_t bits[4] = {60, 40, 40, 60};
    const uint64_t *p;
    switch (n) {
    case 8192: p = p8192; break;
    case 16384: p = p16384; break;
    case 32768: p = p32768; break;
    default: return -1;
    }
    for (int i = 0; i < 4; i++) {
        moduli_out[i] = p[i];
        if (bits_out) bits_out[i] = bits[i];
    }
    return 4;
}

/* params.rs:308-326 -- 6k+-1 trial division. */
int or_is_prime_u64(uint64_t n) {
    if (n < 2) return 0;
    if (n == 2 || n == 3) return 1;
    if (n % 2 == 0 || n % 3 == 0) return 0;
    uint64_t i = 5;
    for (;;) {
        /* i.saturating_mul(i) <= n */
        u128 sq = (u128)i * i;
        if (sq > (u128)n) break;
        if (n % i == 0 || n % (i + 2) == 0) return 0;
        i += 6;
    }
    return 1;
}

/* params.rs:169-193 -- largest bits-bit prime == 1 mod two_n, searched
 * downward from 2^bits - 1.  Every equal width therefore yields the same
 * prime (the reference's duplicate-prime behaviour is reproduced). */
uint64_t or_find_ntt_friendly_prime(uint32_t bits, uint64_t two_n) {
    uint64_t upper = bits >= 64 ? UINT64_MAX : ((1ULL << bits) - 1);
    uint64_t lower = 1ULL << (bits - 1);
    uint64_t candidate = upper - (upper % two_n) + 1;
    if (candidate > upper) candidate -= two_n;
    while (candidate >= lower) {
        if (or_is_prime_u64(candidate)) return candidate;
        candidate = candidate - two_n; /* wrapping_sub */
        if (candidate < lower) break;
    }
    return 0; /* reference panics */
}

/* ======================================================================== */
/* rns.rs                                                                   */
/* ======================================================================== */

/* rns.rs:11-18 */
uint64_t or_mod_add(uint64_t a, uint64_t b, uint64_t q) {
    uint64_t sum = a + b;
    return sum >= q ? sum - q : sum;
}

/* rns.rs:23-29 */
uint64_t or_mod_sub(uint64_t a, uint64_t b, uint64_t q) {
    return a >= b ? a - b : q - b + a;
}

/* rns.rs:34-36 */
uint64_t or_mod_mul(uint64_t a, uint64_t b, uint64_t q) {
    return (uint64_t)(((u128)a * (u128)b) % (u128)q);
}

/* rns.rs:46-87 -- Barrett reduction with the (hi, lo) constant; the
 * a_lo*b_lo carry is dropped exactly as in the reference. */
static uint64_t barrett_reduce(u128 a, const or_modulus *m) {
    uint64_t q = m->value;
    uint64_t a_lo = (uint64_t)a;
    uint64_t a_hi = (uint64_t)(a >> 64);
    if (a_hi == 0) return a_lo % q;
    u128 p_hh = (u128)a_hi * (u128)m->barrett_hi;
    u128 p_hl = (u128)a_hi * (u128)m->barrett_lo;
    u128 p_lh = (u128)a_lo * (u128)m->barrett_hi;
    u128 mid_sum = (p_hl >> 64) + (p_lh >> 64);
    u128 mid_lo_sum = (u128)(uint64_t)p_hl + (u128)(uint64_t)p_lh;
    u128 mid_carry = mid_lo_sum >> 64;
    uint64_t approx_quot = (uint64_t)(p_hh + mid_sum + mid_carry);
    uint64_t r = a_lo - approx_quot * q; /* wrapping */
    if (r >= q) r -= q;
    if (r >= q) r -= q;
    return r;
}

/* rns.rs:92-95 */
uint64_t or_mod_mul_barrett(uint64_t a, uint64_t b, const or_modulus *m) {
    return barrett_reduce((u128)a * (u128)b, m);
}

/* rns.rs:99-110 */
uint64_t or_mod_pow(uint64_t base, uint64_t exp, uint64_t q) {
    uint64_t result = 1;
    base %= q;
    while (exp > 0) {
        if (exp & 1) result = or_mod_mul(result, base, q);
        exp >>= 1;
        base = or_mod_mul(base, base, q);
    }
    return result;
}

/* rns.rs:114-117 */
uint64_t or_mod_inv(uint64_t a, uint64_t q) { return or_mod_pow(a, q - 2, q); }

/* rns.rs:124-154 -- smallest g >= 2 whose psi = g^((q-1)/2N) has psi^N = -1. */
uint64_t or_find_primitive_root(size_t n, uint64_t q) {
    uint64_t two_n = (uint64_t)(2 * n);
    if (q % two_n != 1) return 0;
    uint64_t exponent = (q - 1) / two_n;
    for (uint64_t g = 2; g < 10000; g++) {
        if (g >= q) break;
        uint64_t psi = or_mod_pow(g, exponent, q);
        if (psi <= 1) continue;
        uint64_t psi_n = or_mod_pow(psi, (uint64_t)n, q);
        if (psi_n == q - 1) return psi;
    }
    return 0;
}

/* rns.rs:189-196 */
uint32_t or_bit_reverse(uint32_t x, uint32_t bits) {
    uint32_t result = 0;
    for (uint32_t i = 0; i < bits; i++) {
        result = (result << 1) | (x & 1);
        x >>= 1;
    }
    return result;
}

static uint32_t log2_size(size_t n) {
    uint32_t l = 0;
    while (((size_t)1 << l) < n) l++;
    return l;
}

/* rns.rs:161-171 -- fw[brv(i)] = psi^i. */
static void compute_twiddle_factors(size_t n, uint64_t psi, uint64_t q, uint64_t *tw) {
    uint32_t log_n = log2_size(n);
    for (size_t i = 0; i < n; i++) {
        uint32_t rev = or_bit_reverse((uint32_t)i, log_n);
        tw[rev] = or_mod_pow(psi, (uint64_t)i, q);
    }
}

/* rns.rs:175-185 -- iw[brv(i)] = psi^{-i}. */
static void compute_inv_twiddle_factors(size_t n, uint64_t psi, uint64_t q, uint64_t *tw) {
    uint64_t psi_inv = or_mod_inv(psi, q);
    uint32_t log_n = log2_size(n);
    for (size_t i = 0; i < n; i++) {
        uint32_t rev = or_bit_reverse((uint32_t)i, log_n);
        tw[rev] = or_mod_pow(psi_inv, (uint64_t)i, q);
    }
}

/* ======================================================================== */
/* ntt.rs                                                                   */
/* ======================================================================== */

/* ntt.rs:38-65 */
int or_ntt_tables_init(or_ntt_tables *t, size_t n, uint64_t q) {
    memset(t, 0, sizeof(*t));
    uint32_t log_n = (uint32_t)__builtin_ctzll((unsigned long long)n);
    if (((size_t)1 << log_n) != n) return -1;
    uint64_t psi = or_find_primitive_root(n, q);
    if (psi == 0) return -2;
    t->forward_twiddles = (uint64_t *)malloc(n * sizeof(uint64_t));
    t->inverse_twiddles = (uint64_t *)malloc(n * sizeof(uint64_t));
    if (!t->forward_twiddles || !t->inverse_twiddles) return -3;
    t->psi = psi;
    t->psi_inv = or_mod_inv(psi, q);
    compute_twiddle_factors(n, psi, q, t->forward_twiddles);
    compute_inv_twiddle_factors(n, psi, q, t->inverse_twiddles);
    t->n_inv = or_mod_inv((uint64_t)n, q);
    t->q = q;
    or_modulus_new(q, 64 - (uint32_t)__builtin_clzll(q), &t->modulus);
    t->log_n = log_n;
    t->n = n;
    return 0;
}

void or_ntt_tables_free(or_ntt_tables *t) {
    free(t->forward_twiddles);
    free(t->inverse_twiddles);
    t->forward_twiddles = t->inverse_twiddles = NULL;
}

/* ntt.rs:79-102 -- CT, t = N/2..1, m = 1..N/2, w = fw[m+i]. */
void or_ntt_forward(uint64_t *a, const or_ntt_tables *t) {
    size_t n = t->n;
    uint64_t q = t->q;
    size_t tt = n >> 1, m = 1;
    for (uint32_t s = 0; s < t->log_n; s++) {
        for (size_t i = 0; i < m; i++) {
            uint64_t w = t->forward_twiddles[m + i];
            size_t j1 = 2 * i * tt;
            for (size_t j = j1; j < j1 + tt; j++) {
                uint64_t u = a[j];
                uint64_t v = or_mod_mul_barrett(a[j + tt], w, &t->modulus);
                a[j] = or_mod_add(u, v, q);
                a[j + tt] = or_mod_sub(u, v, q);
            }
        }
        tt >>= 1;
        m <<= 1;
    }
}

/* ntt.rs:113-141 -- GS, t = 1..N/2, m = N/2..1, w = iw[m+i], then x N^-1. */
void or_ntt_inverse(uint64_t *a, const or_ntt_tables *t) {
    size_t n = t->n;
    uint64_t q = t->q;
    size_t tt = 1, m = n >> 1;
    for (uint32_t s = 0; s < t->log_n; s++) {
        for (size_t i = 0; i < m; i++) {
            uint64_t w = t->inverse_twiddles[m + i];
            size_t j1 = 2 * i * tt;
            for (size_t j = j1; j < j1 + tt; j++) {
                uint64_t u = a[j];
                uint64_t v = a[j + tt];
                a[j] = or_mod_add(u, v, q);
                a[j + tt] = or_mod_mul_barrett(or_mod_sub(u, v, q), w, &t->modulus);
            }
        }
        tt <<= 1;
        m >>= 1;
    }
    for (size_t i = 0; i < n; i++) a[i] = or_mod_mul_barrett(a[i], t->n_inv, &t->modulus);
}

int or_ntt_forward_nq(uint64_t *a, size_t n, uint64_t q) {
    or_ntt_tables t;
    int rc = or_ntt_tables_init(&t, n, q);
    if (rc) { or_ntt_tables_free(&t); return rc; }
    or_ntt_forward(a, &t);
    or_ntt_tables_free(&t);
    return 0;
}

int or_ntt_inverse_nq(uint64_t *a, size_t n, uint64_t q) {
    or_ntt_tables t;
    int rc = or_ntt_tables_init(&t, n, q);
    if (rc) { or_ntt_tables_free(&t); return rc; }
    or_ntt_inverse(a, &t);
    or_ntt_tables_free(&t);
    return 0;
}

int or_ntt_tables_export(size_t n, uint64_t q, uint64_t *fw, uint64_t *iw,
                         uint64_t *psi_out, uint64_t *n_inv_out) {
    or_ntt_tables t;
    int rc = or_ntt_tables_init(&t, n, q);
    if (rc) { or_ntt_tables_free(&t); return rc; }
    if (fw) memcpy(fw, t.forward_twiddles, n * sizeof(uint64_t));
    if (iw) memcpy(iw, t.inverse_twiddles, n * sizeof(uint64_t));
    if (psi_out) *psi_out = t.psi;
    if (n_inv_out) *n_inv_out = t.n_inv;
    or_ntt_tables_free(&t);
    return 0;
}

/* ======================================================================== */
/* rng.rs                                                                   */
/* ======================================================================== */

static inline uint32_t rotl32(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }

/* rng.rs:190-206 */
static inline void quarter_round(uint32_t *s, int a, int b, int c, int d) {
    s[a] += s[b]; s[d] ^= s[a]; s[d] = rotl32(s[d], 16);
    s[c] += s[d]; s[b] ^= s[c]; s[b] = rotl32(s[b], 12);
    s[a] += s[b]; s[d] ^= s[a]; s[d] = rotl32(s[d], 8);
    s[c] += s[d]; s[b] ^= s[c]; s[b] = rotl32(s[b], 7);
}

/* rng.rs:163-186 -- 10 double rounds, then add the input state. */
void or_chacha20_block(const uint32_t state[16], uint32_t out[16]) {
    uint32_t w[16];
    memcpy(w, state, sizeof(w));
    for (int i = 0; i < 10; i++) {
        quarter_round(w, 0, 4, 8, 12);
        quarter_round(w, 1, 5, 9, 13);
        quarter_round(w, 2, 6, 10, 14);
        quarter_round(w, 3, 7, 11, 15);
        quarter_round(w, 0, 5, 10, 15);
        quarter_round(w, 1, 6, 11, 12);
        quarter_round(w, 2, 7, 8, 13);
        quarter_round(w, 3, 4, 9, 14);
    }
    for (int i = 0; i < 16; i++) out[i] = w[i] + state[i];
}

/* rng.rs:79-84 */
static void rng_refill(or_rng *r) {
    or_chacha20_block(r->state, r->buffer);
    r->index = 0;
    r->state[12] += 1;
}

/* rng.rs:38-68 -- key = (lo, hi) x 4, counter 0, nonce 0, refilled at
 * construction (so block 0 is consumed first). */
void or_rng_from_seed(or_rng *r, uint64_t seed) {
    uint32_t lo = (uint32_t)seed, hi = (uint32_t)(seed >> 32);
    memset(r, 0, sizeof(*r));
    r->state[0] = 0x61707865u;
    r->state[1] = 0x3320646eu;
    r->state[2] = 0x79622d32u;
    r->state[3] = 0x6b206574u;
    for (int i = 0; i < 4; i++) {
        r->state[4 + i * 2] = lo;
        r->state[5 + i * 2] = hi;
    }
    r->index = 16;
    rng_refill(r);
}

/* rng.rs:88-95 */
uint32_t or_rng_next_u32(or_rng *r) {
    if (r->index >= 16) rng_refill(r);
    return r->buffer[r->index++];
}

/* rng.rs:99-103 -- low word first. */
uint64_t or_rng_next_u64(or_rng *r) {
    uint64_t lo = or_rng_next_u32(r);
    uint64_t hi = or_rng_next_u32(r);
    return (hi << 32) | lo;
}

/* rng.rs:109-120 */
uint32_t or_rng_range_u32(or_rng *r, uint32_t max) {
    uint32_t threshold = (UINT32_MAX - max + 1) % max;
    for (;;) {
        uint32_t v = or_rng_next_u32(r);
        if (v >= threshold) return v % max;
    }
}

/* rng.rs:124-133 */
uint64_t or_rng_range_u64(or_rng *r, uint64_t max) {
    uint64_t threshold = (UINT64_MAX - max + 1) % max;
    for (;;) {
        uint64_t v = or_rng_next_u64(r);
        if (v >= threshold) return v % max;
    }
}

/* rng.rs:139-144 */
double or_rng_next_f64(or_rng *r) {
    uint64_t bits = or_rng_next_u64(r) >> 11;
    return ((double)bits + 0.5) / (double)(1ULL << 53);
}

/* rng.rs:152-157 -- Box-Muller, cosine branch only. */
double or_rng_gaussian(or_rng *r, double sigma) {
    double u1 = or_rng_next_f64(r);
    double u2 = or_rng_next_f64(r);
    double z = sqrt(-2.0 * log(u1)) * cos(2.0 * OR_PI * u2);
    return z * sigma;
}

/* ======================================================================== */
/* sampling.rs                                                              */
/* ======================================================================== */

/* sampling.rs:17-29 -- 0 -> q-1, 1 -> 0, 2 -> 1. */
void or_sample_ternary(or_rng *r, size_t n, uint64_t q, uint64_t *out) {
    for (size_t i = 0; i < n; i++) {
        uint32_t v = or_rng_range_u32(r, 3);
        out[i] = v == 0 ? q - 1 : (v == 1 ? 0 : 1);
    }
}

/* Rust `f64 as i64`: saturating, NaN -> 0. */
static int64_t f64_to_i64_sat(double x) {
    if (x != x) return 0;
    if (x >= 9223372036854775808.0) return INT64_MAX;
    if (x < -9223372036854775808.0) return INT64_MIN;
    return (int64_t)x;
}

/* sampling.rs:51-58 */
void or_sample_gaussian_signed(or_rng *r, size_t n, double sigma, int64_t *out) {
    for (size_t i = 0; i < n; i++) out[i] = f64_to_i64_sat(round(or_rng_gaussian(r, sigma)));
}

/* sampling.rs:62-64 */
void or_sample_uniform(or_rng *r, size_t n, uint64_t q, uint64_t *out) {
    for (size_t i = 0; i < n; i++) out[i] = or_rng_range_u64(r, q);
}

/* signed -> residue as in encoding.rs:198-202 / ciphertext.rs:196-201 */
static inline uint64_t signed_to_residue(int64_t v, uint64_t q) {
    if (v >= 0) return ((uint64_t)v) % q;
    return q - (((uint64_t)0 - (uint64_t)v) % q);
}

/* ======================================================================== */
/* encoding.rs + ciphertext.rs context                                      */
/* ======================================================================== */

struct or_ctx {
    uint32_t n, num_slots, log_n, num_limbs, scale_bits;
    double scale;
    or_modulus moduli[OR_MAX_LIMBS];
    or_ntt_tables ntt[OR_MAX_LIMBS];
    /* FftTables (encoding.rs:25-36) */
    double *twist_re, *twist_im;
    uint32_t *bit_rev;
    double *tw_re, *tw_im; /* stage s, k -> [(1<<s) + k] */
};

/* encoding.rs:38-80 */
static int fft_tables_init(or_ctx *c) {
    size_t n = c->n;
    uint32_t log_n = c->log_n;
    c->twist_re = (double *)malloc(n * sizeof(double));
    c->twist_im = (double *)malloc(n * sizeof(double));
    c->bit_rev = (uint32_t *)malloc(n * sizeof(uint32_t));
    c->tw_re = (double *)calloc(n, sizeof(double));
    c->tw_im = (double *)calloc(n, sizeof(double));
    if (!c->twist_re || !c->twist_im || !c->bit_rev || !c->tw_re || !c->tw_im) return -1;
    for (size_t j = 0; j < n; j++) {
        double angle = OR_PI * (double)j / (double)n;
        c->twist_re[j] = cos(angle);
        c->twist_im[j] = sin(angle);
    }
    for (size_t i = 0; i < n; i++) {
        size_t rev = 0, val = i;
        for (uint32_t b = 0; b < log_n; b++) {
            rev = (rev << 1) | (val & 1);
            val >>= 1;
        }
        c->bit_rev[i] = (uint32_t)rev;
    }
    for (uint32_t s = 0; s < log_n; s++) {
        size_t half_len = (size_t)1 << s;
        for (size_t k = 0; k < half_len; k++) {
            double angle = -2.0 * OR_PI * (double)k / (double)(2 * half_len);
            c->tw_re[half_len + k] = cos(angle);
            c->tw_im[half_len + k] = sin(angle);
        }
    }
    return 0;
}

/* ciphertext.rs:61-74 */
or_ctx *or_ctx_new(uint32_t n, const uint64_t *moduli, uint32_t num_limbs,
                   uint32_t scale_bits) {
    if (num_limbs == 0 || num_limbs > OR_MAX_LIMBS) return NULL;
    if (n < 4 || (n & (n - 1))) return NULL;
    or_ctx *c = (or_ctx *)calloc(1, sizeof(or_ctx));
    if (!c) return NULL;
    c->n = n;
    c->num_slots = n / 2;
    c->log_n = (uint32_t)__builtin_ctz(n);
    c->num_limbs = num_limbs;
    c->scale_bits = scale_bits;
    /* encode/encrypt/decrypt use the crate constant SCALE = 2^40
     * (params.rs:9-12, encoding.rs:196, ciphertext.rs:227, :350) whatever
     * scale_bits a custom parameter set records. */
    c->scale = (double)(1ULL << 40);
    for (uint32_t l = 0; l < num_limbs; l++) {
        uint64_t q = moduli[l];
        or_modulus_new(q, 64 - (uint32_t)__builtin_clzll(q), &c->moduli[l]);
        if (or_ntt_tables_init(&c->ntt[l], n, q) != 0) {
            or_ctx_free(c);
            return NULL;
        }
    }
    if (fft_tables_init(c) != 0) {
        or_ctx_free(c);
        return NULL;
    }
    return c;
}

void or_ctx_free(or_ctx *c) {
    if (!c) return;
    for (uint32_t l = 0; l < OR_MAX_LIMBS; l++) or_ntt_tables_free(&c->ntt[l]);
    free(c->twist_re);
    free(c->twist_im);
    free(c->bit_rev);
    free(c->tw_re);
    free(c->tw_im);
    free(c);
}

uint32_t or_ctx_num_limbs(const or_ctx *c) { return c->num_limbs; }

int or_ctx_fft_tables(const or_ctx *c, double *twist_re, double *twist_im,
                      double *tw_re, double *tw_im) {
    size_t n = c->n;
    if (twist_re) memcpy(twist_re, c->twist_re, n * sizeof(double));
    if (twist_im) memcpy(twist_im, c->twist_im, n * sizeof(double));
    if (tw_re) memcpy(tw_re, c->tw_re, n * sizeof(double));
    if (tw_im) memcpy(tw_im, c->tw_im, n * sizeof(double));
    return 0;
}

/* encoding.rs:83-120 -- bit-reversal swap, then radix-2 DIT stages. */
void or_fft(const or_ctx *c, double *re, double *im) {
    size_t n = c->n;
    for (size_t i = 0; i < n; i++) {
        size_t j = c->bit_rev[i];
        if (i < j) {
            double t = re[i]; re[i] = re[j]; re[j] = t;
            t = im[i]; im[i] = im[j]; im[j] = t;
        }
    }
    for (uint32_t s = 0; s < c->log_n; s++) {
        size_t half_len = (size_t)1 << s;
        size_t full_len = half_len << 1;
        for (size_t gs = 0; gs < n; gs += full_len) {
            for (size_t k = 0; k < half_len; k++) {
                double w_re = c->tw_re[half_len + k];
                double w_im = c->tw_im[half_len + k];
                size_t i0 = gs + k, i1 = i0 + half_len;
                double v_re = w_re * re[i1] - w_im * im[i1];
                double v_im = w_re * im[i1] + w_im * re[i1];
                double u_re = re[i0], u_im = im[i0];
                re[i0] = u_re + v_re;
                im[i0] = u_im + v_im;
                re[i1] = u_re - v_re;
                im[i1] = u_im - v_im;
            }
        }
    }
}

/* encoding.rs:250-278 -- conj-symmetric fill, FFT, x1/N, untwist. */
static void inverse_canonical_embedding(const or_ctx *c, const double *z, double *coeffs) {
    size_t n = c->n, s = c->num_slots;
    double *re = (double *)calloc(n, sizeof(double));
    double *im = (double *)calloc(n, sizeof(double));
    for (size_t k = 0; k < s; k++) {
        re[k] = z[k];
        re[n - 1 - k] = z[k];
    }
    or_fft(c, re, im);
    double inv_n = 1.0 / (double)n;
    for (size_t j = 0; j < n; j++) {
        double a_re = re[j] * inv_n;
        double a_im = im[j] * inv_n;
        coeffs[j] = a_re * c->twist_re[j] + a_im * c->twist_im[j];
    }
    free(re);
    free(im);
}

/* encoding.rs:173-207, returning the rounded signed coefficients. */
int or_encode_coeffs(const or_ctx *c, const double *z, size_t len, int64_t *out) {
    if (len > c->num_slots) return -1; /* reference asserts */
    size_t n = c->n;
    double *zf = (double *)calloc(c->num_slots, sizeof(double));
    double *coeffs = (double *)malloc(n * sizeof(double));
    if (len) memcpy(zf, z, len * sizeof(double));
    inverse_canonical_embedding(c, zf, coeffs);
    for (size_t i = 0; i < n; i++) out[i] = f64_to_i64_sat(round(coeffs[i] * c->scale));
    free(zf);
    free(coeffs);
    return 0;
}

/* encoding.rs:173-207 */
int or_encode(const or_ctx *c, const double *z, size_t len, uint64_t *out_poly) {
    size_t n = c->n;
    int64_t *r = (int64_t *)malloc(n * sizeof(int64_t));
    int rc = or_encode_coeffs(c, z, len, r);
    if (rc) { free(r); return rc; }
    for (uint32_t l = 0; l < c->num_limbs; l++) {
        uint64_t q = c->moduli[l].value;
        for (size_t i = 0; i < n; i++) out_poly[(size_t)l * n + i] = signed_to_residue(r[i], q);
    }
    free(r);
    return 0;
}

/* encoding.rs:295-315 */
static void canonical_embedding(const or_ctx *c, const double *coeffs, double *out_slots) {
    size_t n = c->n;
    double *re = (double *)malloc(n * sizeof(double));
    double *im = (double *)malloc(n * sizeof(double));
    for (size_t j = 0; j < n; j++) {
        re[j] = coeffs[j] * c->twist_re[j];
        im[j] = -coeffs[j] * c->twist_im[j];
    }
    or_fft(c, re, im);
    memcpy(out_slots, re, c->num_slots * sizeof(double));
    free(re);
    free(im);
}

/* encoding.rs:282-284 */
void or_decode_coefficients(const or_ctx *c, const double *coeffs, double *out_slots) {
    canonical_embedding(c, coeffs, out_slots);
}

/* encoding.rs:219-239 -- limb-0 centring / scale. */
static void decode_limb0_coeffs(const or_ctx *c, const uint64_t *poly, double scale,
                                double *coeffs) {
    uint64_t q = c->moduli[0].value;
    uint64_t half_q = q / 2;
    for (size_t j = 0; j < c->n; j++) {
        uint64_t v = poly[j];
        double sgn = v > half_q ? -((double)(q - v)) : (double)v;
        coeffs[j] = sgn / scale;
    }
}

void or_decode(const or_ctx *c, const uint64_t *poly, double scale, double *out_slots) {
    double *coeffs = (double *)malloc(c->n * sizeof(double));
    decode_limb0_coeffs(c, poly, scale, coeffs);
    canonical_embedding(c, coeffs, out_slots);
    free(coeffs);
}

/* ======================================================================== */
/* ciphertext.rs                                                            */
/* ======================================================================== */

/* ciphertext.rs:77-103 -- sample_ternary(rng, n, 3) gives {2, 0, 1} for
 * draws {0, 1, 2}; the per-limb match then maps 0 -> q-1, 1 -> 0, 2 -> 1. */
void or_keygen(const or_ctx *c, or_rng *r, uint64_t *sk_ntt) {
    size_t n = c->n;
    uint64_t *tern = (uint64_t *)malloc(n * sizeof(uint64_t));
    or_sample_ternary(r, n, 3, tern);
    for (uint32_t l = 0; l < c->num_limbs; l++) {
        uint64_t q = c->moduli[l].value;
        uint64_t *limb = sk_ntt + (size_t)l * n;
        for (size_t i = 0; i < n; i++)
            limb[i] = tern[i] == 0 ? q - 1 : (tern[i] == 1 ? 0 : 1);
        or_ntt_forward(limb, &c->ntt[l]);
    }
    free(tern);
}

/* ciphertext.rs:114-154 */
void or_keygen_public(const or_ctx *c, const uint64_t *sk_ntt, or_rng *r,
                      uint64_t *pk_b, uint64_t *pk_a) {
    size_t n = c->n;
    uint32_t L = c->num_limbs;
    for (uint32_t l = 0; l < L; l++) {
        uint64_t *a = pk_a + (size_t)l * n;
        or_sample_uniform(r, n, c->moduli[l].value, a);
        or_ntt_forward(a, &c->ntt[l]);
    }
    int64_t *e = (int64_t *)malloc(n * sizeof(int64_t));
    uint64_t *en = (uint64_t *)malloc(n * sizeof(uint64_t));
    or_sample_gaussian_signed(r, n, OR_ERROR_STD_DEV, e);
    for (uint32_t l = 0; l < L; l++) {
        uint64_t q = c->moduli[l].value;
        for (size_t i = 0; i < n; i++) en[i] = signed_to_residue(e[i], q);
        or_ntt_forward(en, &c->ntt[l]);
        const uint64_t *a = pk_a + (size_t)l * n;
        const uint64_t *s = sk_ntt + (size_t)l * n;
        uint64_t *b = pk_b + (size_t)l * n;
        for (size_t i = 0; i < n; i++) {
            uint64_t as = or_mod_mul_barrett(a[i], s[i], &c->moduli[l]);
            uint64_t neg_as = as == 0 ? 0 : q - as;
            b[i] = or_mod_add(neg_as, en[i], q);
        }
    }
    free(e);
    free(en);
}

/* ciphertext.rs:167-229 */
int or_encrypt(const or_ctx *c, const double *z, size_t len, const uint64_t *sk_ntt,
               or_rng *r, uint64_t *c0, uint64_t *c1, double *scale) {
    size_t n = c->n;
    uint32_t L = c->num_limbs;
    uint64_t *m = (uint64_t *)malloc((size_t)L * n * sizeof(uint64_t));
    int rc = or_encode(c, z, len, m);
    if (rc) { free(m); return rc; }
    for (uint32_t l = 0; l < L; l++) or_ntt_forward(m + (size_t)l * n, &c->ntt[l]);
    for (uint32_t l = 0; l < L; l++) {
        uint64_t *a = c1 + (size_t)l * n;
        or_sample_uniform(r, n, c->moduli[l].value, a);
        or_ntt_forward(a, &c->ntt[l]);
    }
    int64_t *e = (int64_t *)malloc(n * sizeof(int64_t));
    uint64_t *en = (uint64_t *)malloc(n * sizeof(uint64_t));
    or_sample_gaussian_signed(r, n, OR_ERROR_STD_DEV, e);
    for (uint32_t l = 0; l < L; l++) {
        uint64_t q = c->moduli[l].value;
        for (size_t i = 0; i < n; i++) en[i] = signed_to_residue(e[i], q);
        or_ntt_forward(en, &c->ntt[l]);
        const uint64_t *a = c1 + (size_t)l * n;
        const uint64_t *s = sk_ntt + (size_t)l * n;
        const uint64_t *ml = m + (size_t)l * n;
        uint64_t *o = c0 + (size_t)l * n;
        for (size_t i = 0; i < n; i++) {
            uint64_t neg_as = or_mod_sub(0, or_mod_mul_barrett(a[i], s[i], &c->moduli[l]), q);
            o[i] = or_mod_add(neg_as, or_mod_add(ml[i], en[i], q), q);
        }
    }
    free(e);
    free(en);
    free(m);
    *scale = c->scale;
    return 0;
}

/* ciphertext.rs:240-319 */
int or_encrypt_pk(const or_ctx *c, const double *z, size_t len, const uint64_t *pk_b,
                  const uint64_t *pk_a, or_rng *r, uint64_t *c0, uint64_t *c1,
                  double *scale) {
    size_t n = c->n;
    uint32_t L = c->num_limbs;
    uint64_t *m = (uint64_t *)malloc((size_t)L * n * sizeof(uint64_t));
    int rc = or_encode(c, z, len, m);
    if (rc) { free(m); return rc; }
    for (uint32_t l = 0; l < L; l++) or_ntt_forward(m + (size_t)l * n, &c->ntt[l]);
    uint64_t *tern = (uint64_t *)malloc(n * sizeof(uint64_t));
    or_sample_ternary(r, n, 3, tern);
    uint64_t *u = (uint64_t *)malloc((size_t)L * n * sizeof(uint64_t));
    for (uint32_t l = 0; l < L; l++) {
        uint64_t q = c->moduli[l].value;
        uint64_t *ul = u + (size_t)l * n;
        for (size_t i = 0; i < n; i++) ul[i] = tern[i] == 0 ? q - 1 : (tern[i] == 1 ? 0 : 1);
        or_ntt_forward(ul, &c->ntt[l]);
    }
    int64_t *e0 = (int64_t *)malloc(n * sizeof(int64_t));
    int64_t *e1 = (int64_t *)malloc(n * sizeof(int64_t));
    or_sample_gaussian_signed(r, n, OR_ERROR_STD_DEV, e0);
    or_sample_gaussian_signed(r, n, OR_ERROR_STD_DEV, e1);
    uint64_t *e0n = (uint64_t *)malloc(n * sizeof(uint64_t));
    uint64_t *e1n = (uint64_t *)malloc(n * sizeof(uint64_t));
    for (uint32_t l = 0; l < L; l++) {
        uint64_t q = c->moduli[l].value;
        for (size_t i = 0; i < n; i++) {
            e0n[i] = signed_to_residue(e0[i], q);
            e1n[i] = signed_to_residue(e1[i], q);
        }
        or_ntt_forward(e0n, &c->ntt[l]);
        or_ntt_forward(e1n, &c->ntt[l]);
        const uint64_t *b = pk_b + (size_t)l * n, *a = pk_a + (size_t)l * n;
        const uint64_t *ul = u + (size_t)l * n, *ml = m + (size_t)l * n;
        uint64_t *o0 = c0 + (size_t)l * n, *o1 = c1 + (size_t)l * n;
        for (size_t i = 0; i < n; i++) {
            uint64_t bu = or_mod_mul_barrett(b[i], ul[i], &c->moduli[l]);
            o0[i] = or_mod_add(bu, or_mod_add(e0n[i], ml[i], q), q);
            uint64_t au = or_mod_mul_barrett(a[i], ul[i], &c->moduli[l]);
            o1[i] = or_mod_add(au, e1n[i], q);
        }
    }
    free(m); free(tern); free(u); free(e0); free(e1); free(e0n); free(e1n);
    *scale = c->scale;
    return 0;
}

/* u128 -> f64 with round-to-nearest, ties-to-even (Rust `u128 as f64`). */
double or_u128_to_f64(uint64_t hi, uint64_t lo) {
    if (hi == 0) return (double)lo; /* u64 -> f64 conversion is RNE in C */
    int lz = __builtin_clzll(hi);
    int nbits = 128 - lz;             /* 65..128 */
    /* top 64 bits of the value, MSB at bit 63 */
    uint64_t top = lz ? ((hi << lz) | (lo >> (64 - lz))) : hi;
    uint64_t rest = lz ? (lo << lz) : lo; /* bits below the top 64 */
    uint64_t mant = top >> 11;            /* 53 bits */
    uint64_t rbit = (top >> 10) & 1;
    int sticky = ((top & 0x3FF) != 0) || (rest != 0);
    if (rbit && (sticky || (mant & 1))) mant++;
    /* value = mant * 2^(nbits - 53) (mant may be 2^53 -> exact power) */
    return ldexp((double)mant, nbits - 53);
}

/* ciphertext.rs:327-400, stopping before the canonical embedding. */
void or_decrypt_coeffs(const or_ctx *c, const uint64_t *c0, const uint64_t *c1,
                       uint32_t num_limbs, double scale, const uint64_t *sk_ntt,
                       double *out_coeffs) {
    size_t n = c->n;
    uint64_t *m = (uint64_t *)malloc((size_t)num_limbs * n * sizeof(uint64_t));
    for (uint32_t l = 0; l < num_limbs; l++) {
        uint64_t q = c->moduli[l].value;
        const uint64_t *a0 = c0 + (size_t)l * n, *a1 = c1 + (size_t)l * n;
        const uint64_t *s = sk_ntt + (size_t)l * n;
        uint64_t *ml = m + (size_t)l * n;
        for (size_t i = 0; i < n; i++) {
            uint64_t c1s = or_mod_mul_barrett(a1[i], s[i], &c->moduli[l]);
            ml[i] = or_mod_add(a0[i], c1s, q);
        }
    }
    for (uint32_t l = 0; l < num_limbs; l++) or_ntt_inverse(m + (size_t)l * n, &c->ntt[l]);
    if (scale > c->scale * 1.5 && num_limbs >= 2) {
        uint64_t q0 = c->moduli[0].value, q1 = c->moduli[1].value;
        uint64_t q0_inv_mod_q1 = or_mod_inv(q0 % q1, q1);
        u128 q_product = (u128)q0 * (u128)q1;
        u128 half_product = q_product / 2;
        for (size_t i = 0; i < n; i++) {
            uint64_t m0 = m[i], m1 = m[n + i];
            uint64_t m0_mod_q1 = (uint64_t)((u128)m0 % (u128)q1);
            uint64_t diff = m1 >= m0_mod_q1 ? m1 - m0_mod_q1 : q1 - m0_mod_q1 + m1;
            uint64_t k = (uint64_t)(((u128)diff * (u128)q0_inv_mod_q1) % (u128)q1);
            u128 mu = (u128)m0 + (u128)k * (u128)q0;
            if (mu >= q_product) mu = mu % q_product;
            double v;
            if (mu > half_product) {
                u128 d = q_product - mu;
                v = -or_u128_to_f64((uint64_t)(d >> 64), (uint64_t)d);
            } else {
                v = or_u128_to_f64((uint64_t)(mu >> 64), (uint64_t)mu);
            }
            out_coeffs[i] = v / scale;
        }
    } else {
        decode_limb0_coeffs(c, m, scale, out_coeffs);
    }
    free(m);
}

/* ciphertext.rs:327-400 */
void or_decrypt(const or_ctx *c, const uint64_t *c0, const uint64_t *c1,
                uint32_t num_limbs, double scale, const uint64_t *sk_ntt,
                double *out_slots) {
    double *coeffs = (double *)malloc(c->n * sizeof(double));
    or_decrypt_coeffs(c, c0, c1, num_limbs, scale, sk_ntt, coeffs);
    canonical_embedding(c, coeffs, out_slots);
    free(coeffs);
}

/* ciphertext.rs:539-545 */
int or_encode_to_ntt(const or_ctx *c, const double *z, size_t len, uint64_t *out) {
    int rc = or_encode(c, z, len, out);
    if (rc) return rc;
    for (uint32_t l = 0; l < c->num_limbs; l++) or_ntt_forward(out + (size_t)l * c->n, &c->ntt[l]);
    return 0;
}

/* ciphertext.rs:422-429 (hadamard over the ciphertext's limbs, rns.rs:243-253) */
void or_ct_pt_mul_ntt(const or_ctx *c, const uint64_t *c0, const uint64_t *c1,
                      uint32_t num_limbs, const uint64_t *pt_ntt, uint64_t *o0,
                      uint64_t *o1) {
    size_t n = c->n;
    for (uint32_t l = 0; l < num_limbs; l++) {
        const or_modulus *md = &c->moduli[l];
        for (size_t i = 0; i < n; i++) {
            size_t x = (size_t)l * n + i;
            o0[x] = or_mod_mul_barrett(c0[x], pt_ntt[x], md);
            o1[x] = or_mod_mul_barrett(c1[x], pt_ntt[x], md);
        }
    }
}

/* ciphertext.rs:408-418 */
int or_ct_pt_mul(const or_ctx *c, const uint64_t *c0, const uint64_t *c1,
                 uint32_t num_limbs, const double *pt, size_t len, uint64_t *o0,
                 uint64_t *o1) {
    uint64_t *p = (uint64_t *)malloc((size_t)c->num_limbs * c->n * sizeof(uint64_t));
    int rc = or_encode_to_ntt(c, pt, len, p);
    if (!rc) or_ct_pt_mul_ntt(c, c0, c1, num_limbs, p, o0, o1);
    free(p);
    return rc;
}

/* ciphertext.rs:435-448 (rns.rs:217-227) */
void or_ct_add(const or_ctx *c, const uint64_t *a0, const uint64_t *a1,
               const uint64_t *b0, const uint64_t *b1, uint32_t num_limbs,
               uint64_t *o0, uint64_t *o1) {
    size_t n = c->n;
    for (uint32_t l = 0; l < num_limbs; l++) {
        uint64_t q = c->moduli[l].value;
        for (size_t i = 0; i < n; i++) {
            size_t x = (size_t)l * n + i;
            o0[x] = or_mod_add(a0[x], b0[x], q);
            o1[x] = or_mod_add(a1[x], b1[x], q);
        }
    }
}

/* ciphertext.rs:453-466 (rns.rs:230-240) */
void or_ct_sub(const or_ctx *c, const uint64_t *a0, const uint64_t *a1,
               const uint64_t *b0, const uint64_t *b1, uint32_t num_limbs,
               uint64_t *o0, uint64_t *o1) {
    size_t n = c->n;
    for (uint32_t l = 0; l < num_limbs; l++) {
        uint64_t q = c->moduli[l].value;
        for (size_t i = 0; i < n; i++) {
            size_t x = (size_t)l * n + i;
            o0[x] = or_mod_sub(a0[x], b0[x], q);
            o1[x] = or_mod_sub(a1[x], b1[x], q);
        }
    }
}

/* ciphertext.rs:476-535 -- outputs are (num_limbs-1) limbs. */
int or_rescale(const or_ctx *c, const uint64_t *c0, const uint64_t *c1,
               uint32_t num_limbs, uint64_t *o0, uint64_t *o1) {
    if (num_limbs < 2) return -1;
    size_t n = c->n;
    uint32_t last = num_limbs - 1;
    uint64_t last_q = c->moduli[last].value;
    uint64_t *c0l = (uint64_t *)malloc(n * sizeof(uint64_t));
    uint64_t *c1l = (uint64_t *)malloc(n * sizeof(uint64_t));
    uint64_t *t0 = (uint64_t *)malloc(n * sizeof(uint64_t));
    uint64_t *t1 = (uint64_t *)malloc(n * sizeof(uint64_t));
    memcpy(c0l, c0 + (size_t)last * n, n * sizeof(uint64_t));
    memcpy(c1l, c1 + (size_t)last * n, n * sizeof(uint64_t));
    or_ntt_inverse(c0l, &c->ntt[last]);
    or_ntt_inverse(c1l, &c->ntt[last]);
    for (uint32_t l = 0; l < last; l++) {
        uint64_t ql = c->moduli[l].value;
        uint64_t inv = or_mod_inv(last_q % ql, ql);
        memcpy(t0, c0 + (size_t)l * n, n * sizeof(uint64_t));
        memcpy(t1, c1 + (size_t)l * n, n * sizeof(uint64_t));
        or_ntt_inverse(t0, &c->ntt[l]);
        or_ntt_inverse(t1, &c->ntt[l]);
        uint64_t *r0 = o0 + (size_t)l * n, *r1 = o1 + (size_t)l * n;
        for (size_t i = 0; i < n; i++) {
            uint64_t lm0 = c0l[i] % ql;
            uint64_t d0 = t0[i] >= lm0 ? t0[i] - lm0 : ql - lm0 + t0[i];
            r0[i] = or_mod_mul_barrett(d0, inv, &c->moduli[l]);
            uint64_t lm1 = c1l[i] % ql;
            uint64_t d1 = t1[i] >= lm1 ? t1[i] - lm1 : ql - lm1 + t1[i];
            r1[i] = or_mod_mul_barrett(d1, inv, &c->moduli[l]);
        }
        or_ntt_forward(r0, &c->ntt[l]);
        or_ntt_forward(r1, &c->ntt[l]);
    }
    free(c0l); free(c1l); free(t0); free(t1);
    return 0;
}

/* ======================================================================== */
/* Wire format: serialize.rs:14-93                                           */
/* ======================================================================== */

/* u64::to_le_bytes / from_le_bytes, independent of the host's byte order. */
static void le_put(uint8_t *o, uint64_t x) {
    for (int b = 0; b < 8; b++) o[b] = (uint8_t)(x >> (8 * b));
}

static uint64_t le_get(const uint8_t *o) {
    uint64_t x = 0;
    for (int b = 0; b < 8; b++) x |= (uint64_t)o[b] << (8 * b);
    return x;
}

/* serialize.rs:14-23 */
void or_rns_poly_to_bytes(const uint64_t *poly, size_t n, uint32_t L, uint8_t *out) {
    for (uint32_t l = 0; l < L; l++)
        for (size_t i = 0; i < n; i++) le_put(out + ((size_t)l * n + i) * 8, poly[(size_t)l * n + i]);
}

/* serialize.rs:26-44 */
int or_rns_poly_from_bytes(const uint8_t *bytes, size_t len, size_t n, uint32_t L, uint64_t *poly) {
    if (len != (size_t)L * n * 8) return -1;
    size_t off = 0;
    for (uint32_t l = 0; l < L; l++)
        for (size_t i = 0; i < n; i++, off += 8) poly[(size_t)l * n + i] = le_get(bytes + off);
    return 0;
}

/* serialize.rs:48-52 */
void or_pk_to_bytes(const uint64_t *b, const uint64_t *a, size_t n, uint32_t L, uint8_t *out) {
    or_rns_poly_to_bytes(b, n, L, out);
    or_rns_poly_to_bytes(a, n, L, out + (size_t)L * n * 8);
}

/* serialize.rs:55-67 */
int or_pk_from_bytes(const uint8_t *bytes, size_t len, size_t n, uint32_t L, uint64_t *b, uint64_t *a) {
    const size_t poly = (size_t)L * n * 8;
    if (len != 2 * poly) return -1;
    if (or_rns_poly_from_bytes(bytes, poly, n, L, b)) return -1;
    return or_rns_poly_from_bytes(bytes + poly, poly, n, L, a);
}

/* serialize.rs:71-77 */
void or_ct_to_bytes(double scale, const uint64_t *c0, const uint64_t *c1, size_t n, uint32_t L, uint8_t *out) {
    uint64_t sb;
    memcpy(&sb, &scale, 8); /* f64::to_le_bytes: the IEEE bits, little-endian */
    le_put(out, sb);
    or_rns_poly_to_bytes(c0, n, L, out + 8);
    or_rns_poly_to_bytes(c1, n, L, out + 8 + (size_t)L * n * 8);
}

/* serialize.rs:80-93 */
int or_ct_from_bytes(const uint8_t *bytes, size_t len, size_t n, uint32_t L, double *scale, uint64_t *c0,
                     uint64_t *c1) {
    const size_t poly = (size_t)L * n * 8;
    if (len != 8 + 2 * poly) return -1;
    const uint64_t sb = le_get(bytes);
    memcpy(scale, &sb, 8);
    if (or_rns_poly_from_bytes(bytes + 8, poly, n, L, c0)) return -1;
    return or_rns_poly_from_bytes(bytes + 8 + poly, poly, n, L, c1);
}

/* ======================================================================== */
/* ZeRo-MOAI delta: inference_engine.py:1244-1392                           */
/* ======================================================================== */

int or_lora_delta_cached(const or_ctx *c, const uint64_t *sk_ntt, const double *h,
                         uint32_t d, const float *lora_a, const float *lora_b, uint32_t r,
                         uint64_t enc_seed, int mode, const uint64_t *pt_cache, double *delta,
                         double *intermediate);

/* _precompute_he_cache (inference_engine.py:1037-1074) taken one step
 * further, as ct_pt_mul_ntt's cached-plaintext fast path intends
 * (ciphertext.rs:420-429): NTT(encode(packed_pt_b)) for each batch b,
 * out [n_batches][L][n]. */
int or_lora_pack(const or_ctx *c, const float *lora_a, uint32_t r, uint32_t d, uint64_t *out) {
    size_t S = c->num_slots;
    if (d == 0 || d > S || r == 0) return -1;
    size_t cols = S / d, nb = (r + cols - 1) / cols;
    double *pt = (double *)malloc(S * sizeof(double));
    int rc = 0;
    for (size_t b = 0; b < nb && !rc; b++) {
        size_t r0 = b * cols, r1 = r0 + cols < r ? r0 + cols : r;
        memset(pt, 0, S * sizeof(double));
        for (size_t i = 0; i < r1 - r0; i++)
            for (size_t j = 0; j < d; j++) pt[i * d + j] = (double)lora_a[(r0 + i) * d + j];
        rc = or_encode_to_ntt(c, pt, S, out + b * (size_t)c->num_limbs * c->n);
    }
    free(pt);
    return rc;
}

int or_lora_delta(const or_ctx *c, const uint64_t *sk_ntt, const double *h,
                  uint32_t d, const float *lora_a, const float *lora_b, uint32_t r,
                  uint64_t enc_seed, int mode, double *delta, double *intermediate) {
    return or_lora_delta_cached(c, sk_ntt, h, d, lora_a, lora_b, r, enc_seed, mode, NULL, delta,
                                intermediate);
}

int or_lora_delta_cached(const or_ctx *c, const uint64_t *sk_ntt, const double *h,
                         uint32_t d, const float *lora_a, const float *lora_b, uint32_t r,
                         uint64_t enc_seed, int mode, const uint64_t *pt_cache, double *delta,
                         double *intermediate) {
    size_t n = c->n, S = c->num_slots;
    uint32_t L = c->num_limbs;
    if (d == 0 || d > S || r == 0) return -1;
    size_t cols = S / d;                              /* :1258 (max(1, S//d)) */
    if (cols < 1) cols = 1;
    size_t n_batches = (r + cols - 1) / cols;         /* :1259 */
    double *rep = (double *)calloc(S, sizeof(double)); /* :1267-1269 */
    for (size_t i = 0; i < cols; i++) memcpy(rep + i * d, h, d * sizeof(double));
    size_t poly = (size_t)L * n;
    uint64_t *c0 = (uint64_t *)malloc(poly * sizeof(uint64_t));
    uint64_t *c1 = (uint64_t *)malloc(poly * sizeof(uint64_t));
    uint64_t *p0 = (uint64_t *)malloc(poly * sizeof(uint64_t));
    uint64_t *p1 = (uint64_t *)malloc(poly * sizeof(uint64_t));
    double *pt = (double *)malloc(S * sizeof(double));
    double *dec = (double *)malloc(S * sizeof(double));
    double scale;
    or_rng rng;
    or_rng_from_seed(&rng, enc_seed);
    int rc = or_encrypt(c, rep, S, sk_ntt, &rng, c0, c1, &scale); /* :1272 */
    or_ctx *obj_ctx = NULL;
    if (!rc && mode == 1) {
        /* lib.rs:322-328 -- ensure_ctx rebuilds a CkksContext for the new
         * ciphertext object on its first `*`. */
        uint64_t moduli[OR_MAX_LIMBS];
        for (uint32_t l = 0; l < L; l++) moduli[l] = c->moduli[l].value;
        obj_ctx = or_ctx_new(c->n, moduli, L, c->scale_bits);
        if (!obj_ctx) rc = -2;
    }
    uint64_t *ptn = (uint64_t *)malloc(poly * sizeof(uint64_t));
    for (size_t b = 0; !rc && b < n_batches; b++) {
        size_t r0 = b * cols, r1 = r0 + cols < r ? r0 + cols : r;
        memset(pt, 0, S * sizeof(double));            /* :1299-1303 */
        for (size_t i = 0; i < r1 - r0; i++)
            for (size_t j = 0; j < d; j++) pt[i * d + j] = (double)lora_a[(r0 + i) * d + j];
        if (mode == 1) {
            rc = or_ct_pt_mul(obj_ctx, c0, c1, L, pt, S, p0, p1); /* :1311 */
        } else if (pt_cache) {
            or_ct_pt_mul_ntt(c, c0, c1, L, pt_cache + b * poly, p0, p1);
        } else {
            rc = or_encode_to_ntt(c, pt, S, ptn);
            if (!rc) or_ct_pt_mul_ntt(c, c0, c1, L, ptn, p0, p1);
        }
        if (rc) break;
        or_decrypt(c, p0, p1, L, scale * scale, sk_ntt, dec); /* :1315 */
        for (size_t i = 0; i < r1 - r0; i++) {          /* :1382-1386 */
            double s = 0.0;
            for (size_t j = 0; j < d; j++) s += dec[i * d + j];
            intermediate[r0 + i] = s;
        }
    }
    if (!rc) {
        for (size_t i = 0; i < d; i++) {                /* :1392 */
            double s = 0.0;
            for (size_t k = 0; k < r; k++) s += (double)lora_b[i * r + k] * intermediate[k];
            delta[i] = s;
        }
    }
    or_ctx_free(obj_ctx);
    free(rep); free(c0); free(c1); free(p0); free(p1); free(pt); free(dec); free(ptn);
    return rc;
}

/* ======================================================================== */
/* Test helper: find seeds whose stream exercises the rejection branches.   */
/* ======================================================================== */
/* kind 0: encrypt's uniform segments -- L x n range_u64(q_l) draws
 *         (ciphertext.rs:185-191, rng.rs:124-133);
 * kind 1: keygen's n range_u32(3) draws (sampling.rs:17-29, rng.rs:109-120).
 * Returns the first seed in [start, start+count) that rejects at least one
 * candidate, or UINT64_MAX. */
uint64_t or_find_reject_seed(const uint64_t *moduli, uint32_t L, size_t n, uint64_t start,
                             uint64_t count, int kind) {
    for (uint64_t s = start; s < start + count; s++) {
        or_rng r;
        or_rng_from_seed(&r, s);
        if (kind == 1) {
            for (size_t i = 0; i < n; i++)
                if (or_rng_next_u32(&r) < 1u) return s;
            continue;
        }
        for (uint32_t l = 0; l < L; l++) {
            uint64_t q = moduli[l];
            uint64_t thr = (UINT64_MAX - q + 1) % q;
            for (size_t i = 0; i < n; i++)
                if (or_rng_next_u64(&r) < thr) return s;
        }
    }
    return UINT64_MAX;
}
