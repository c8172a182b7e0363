/*
 * tsoracle.h -- CPU oracle for the TenSafe CKKS hot path (TEST INFRASTRUCTURE).
 *
 * This is a plain-C restatement of the reference Rust crate
 * `tensafe-he/crates/tensafe-he-core` (params.rs, rns.rs, ntt.rs, rng.rs,
 * sampling.rs, encoding.rs, ciphertext.rs) plus the ZeRo-MOAI glue of
 * `demonstrator/server/inference_engine.py:1244-1392`.  It exists only so
 * that tests, the smoke check and the bench's CPU-baseline leg can check and
 * time the CUDA product path.  Nothing in the product (`provenloop_b200/`)
 * links, loads or calls it.
 *
 * Parity pinning: the reference Rust cannot be built in this image (no
 * cargo/rustc, no crate registry), so this restatement is pinned against the
 * reference's own known-answer tests (RFC 8439 ChaCha20 block, the NTT
 * round-trip and negacyclic-product KATs, prime/root properties, encode and
 * encrypt tolerances) -- see tests/test_oracle_kats.py.
 *
 * Layouts: an RNS polynomial is `num_limbs * n` uint64, limb-major
 * (limb l occupies [l*n, (l+1)*n)), exactly like `RnsPoly.limbs` flattened.
 */
#ifndef TSORACLE_H
#define TSORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OR_MAX_LIMBS 16

/* ---- params.rs ---------------------------------------------------------- */
typedef struct {
    uint64_t value;
    uint32_t bits;
    uint64_t barrett_hi;
    uint64_t barrett_lo;
} or_modulus;

void or_modulus_new(uint64_t value, uint32_t bits, or_modulus *out);
/* Hard-coded 4-prime chains (params.rs:66-126). Returns number of limbs or -1. */
int or_params_preset(uint32_t n, uint64_t *moduli_out, uint32_t *bits_out);
/* params.rs:169-193 (descending search, trial division). */
uint64_t or_find_ntt_friendly_prime(uint32_t bits, uint64_t two_n);
int or_is_prime_u64(uint64_t n);

/* ---- rns.rs -------------------------------------------------------------- */
uint64_t or_mod_add(uint64_t a, uint64_t b, uint64_t q);
uint64_t or_mod_sub(uint64_t a, uint64_t b, uint64_t q);
uint64_t or_mod_mul(uint64_t a, uint64_t b, uint64_t q);
uint64_t or_mod_mul_barrett(uint64_t a, uint64_t b, const or_modulus *m);
uint64_t or_mod_pow(uint64_t base, uint64_t exp, uint64_t q);
uint64_t or_mod_inv(uint64_t a, uint64_t q);
uint64_t or_find_primitive_root(size_t n, uint64_t q);
uint32_t or_bit_reverse(uint32_t x, uint32_t bits);

/* ---- ntt.rs -------------------------------------------------------------- */
typedef struct {
    uint64_t *forward_twiddles;
    uint64_t *inverse_twiddles;
    uint64_t psi, psi_inv, n_inv, q;
    or_modulus modulus;
    uint32_t log_n;
    size_t n;
} or_ntt_tables;

int or_ntt_tables_init(or_ntt_tables *t, size_t n, uint64_t q);
void or_ntt_tables_free(or_ntt_tables *t);
void or_ntt_forward(uint64_t *a, const or_ntt_tables *t);
void or_ntt_inverse(uint64_t *a, const or_ntt_tables *t);
/* Convenience for KATs: build tables for (n, q), transform in place. */
int or_ntt_forward_nq(uint64_t *a, size_t n, uint64_t q);
int or_ntt_inverse_nq(uint64_t *a, size_t n, uint64_t q);
/* Export tables (n entries each) for table-level checks. */
int or_ntt_tables_export(size_t n, uint64_t q, uint64_t *fw, uint64_t *iw,
                         uint64_t *psi_out, uint64_t *n_inv_out);

/* ---- rng.rs -------------------------------------------------------------- */
typedef struct {
    uint32_t state[16];
    uint32_t buffer[16];
    uint32_t index;
} or_rng;

void or_chacha20_block(const uint32_t state[16], uint32_t out[16]);
void or_rng_from_seed(or_rng *r, uint64_t seed);
uint32_t or_rng_next_u32(or_rng *r);
uint64_t or_rng_next_u64(or_rng *r);
uint32_t or_rng_range_u32(or_rng *r, uint32_t max);
uint64_t or_rng_range_u64(or_rng *r, uint64_t max);
double or_rng_next_f64(or_rng *r);
double or_rng_gaussian(or_rng *r, double sigma);

/* ---- sampling.rs --------------------------------------------------------- */
#define OR_ERROR_STD_DEV 3.19
void or_sample_ternary(or_rng *r, size_t n, uint64_t q, uint64_t *out);
void or_sample_gaussian_signed(or_rng *r, size_t n, double sigma, int64_t *out);
void or_sample_uniform(or_rng *r, size_t n, uint64_t q, uint64_t *out);

/* ---- ciphertext.rs / encoding.rs: context ------------------------------- */
typedef struct or_ctx or_ctx;

or_ctx *or_ctx_new(uint32_t n, const uint64_t *moduli, uint32_t num_limbs,
                   uint32_t scale_bits);
void or_ctx_free(or_ctx *c);
uint32_t or_ctx_num_limbs(const or_ctx *c);
/* FFT tables (encoding.rs:38-80): twist_re/im[n], stage twiddles packed as
 * tw[(1<<s) + k] for stage s, k < 2^s (entry 0 unused). */
int or_ctx_fft_tables(const or_ctx *c, double *twist_re, double *twist_im,
                      double *tw_re, double *tw_im);

/* encoding.rs */
int or_encode(const or_ctx *c, const double *z, size_t len, uint64_t *out_poly);
/* encode, but also return the rounded signed coefficients (i64[n]). */
int or_encode_coeffs(const or_ctx *c, const double *z, size_t len, int64_t *out);
void or_decode(const or_ctx *c, const uint64_t *poly, double scale, double *out_slots);
void or_decode_coefficients(const or_ctx *c, const double *coeffs, double *out_slots);
void or_fft(const or_ctx *c, double *re, double *im);

/* ciphertext.rs: keys and ciphertexts. sk/ct polys are [L][n]. */
void or_keygen(const or_ctx *c, or_rng *r, uint64_t *sk_ntt);
void or_keygen_public(const or_ctx *c, const uint64_t *sk_ntt, or_rng *r,
                      uint64_t *pk_b, uint64_t *pk_a);
int or_encrypt(const or_ctx *c, const double *z, size_t len, const uint64_t *sk_ntt,
               or_rng *r, uint64_t *c0, uint64_t *c1, double *scale);
int or_encrypt_pk(const or_ctx *c, const double *z, size_t len, const uint64_t *pk_b,
                  const uint64_t *pk_a, or_rng *r, uint64_t *c0, uint64_t *c1,
                  double *scale);
void or_decrypt(const or_ctx *c, const uint64_t *c0, const uint64_t *c1,
                uint32_t num_limbs, double scale, const uint64_t *sk_ntt,
                double *out_slots);
/* Decrypt up to (and excluding) the canonical embedding: the f64
 * coefficients that feed decode (CRT branch or limb-0 centring). */
void or_decrypt_coeffs(const or_ctx *c, const uint64_t *c0, const uint64_t *c1,
                       uint32_t num_limbs, double scale, const uint64_t *sk_ntt,
                       double *out_coeffs);
int or_encode_to_ntt(const or_ctx *c, const double *z, size_t len, uint64_t *out);
void or_ct_pt_mul_ntt(const or_ctx *c, const uint64_t *c0, const uint64_t *c1,
                      uint32_t num_limbs, const uint64_t *pt_ntt, uint64_t *o0,
                      uint64_t *o1);
int or_ct_pt_mul(const or_ctx *c, const uint64_t *c0, const uint64_t *c1,
                 uint32_t num_limbs, const double *pt, size_t len, uint64_t *o0,
                 uint64_t *o1);
void or_ct_add(const or_ctx *c, const uint64_t *a0, const uint64_t *a1,
               const uint64_t *b0, const uint64_t *b1, uint32_t num_limbs,
               uint64_t *o0, uint64_t *o1);
void or_ct_sub(const or_ctx *c, const uint64_t *a0, const uint64_t *a1,
               const uint64_t *b0, const uint64_t *b1, uint32_t num_limbs,
               uint64_t *o0, uint64_t *o1);
int or_rescale(const or_ctx *c, const uint64_t *c0, const uint64_t *c1,
               uint32_t num_limbs, uint64_t *o0, uint64_t *o1);

/* ---- wire format (serialize.rs:14-93) ----------------------------------- */
/* RnsPoly: limb-major, every u64 little-endian (L*n*8 bytes). */
void or_rns_poly_to_bytes(const uint64_t *poly, size_t n, uint32_t L, uint8_t *out);
/* -1 unless len == L*n*8 (the reference's assert_eq!). */
int or_rns_poly_from_bytes(const uint8_t *bytes, size_t len, size_t n, uint32_t L, uint64_t *poly);
/* PublicKey: [b | a] (2*L*n*8 bytes). */
void or_pk_to_bytes(const uint64_t *b, const uint64_t *a, size_t n, uint32_t L, uint8_t *out);
int or_pk_from_bytes(const uint8_t *bytes, size_t len, size_t n, uint32_t L, uint64_t *b, uint64_t *a);
/* Ciphertext: [scale f64 LE | c0 | c1] (8 + 2*L*n*8 bytes). */
void or_ct_to_bytes(double scale, const uint64_t *c0, const uint64_t *c1, size_t n, uint32_t L, uint8_t *out);
int or_ct_from_bytes(const uint8_t *bytes, size_t len, size_t n, uint32_t L, double *scale, uint64_t *c0,
                     uint64_t *c1);

/* u128 -> f64, round-to-nearest-even (Rust `as f64`). */
double or_u128_to_f64(uint64_t hi, uint64_t lo);

/* ---- ZeRo-MOAI delta (inference_engine.py:1244-1392) --------------------- */
/* mode 0 = "core-optimal": cached context, pt encoded once per batch via
 *          encode_to_ntt and multiplied with ct_pt_mul_ntt;
 * mode 1 = "as invoked": what the PyO3 binding does per `ct * pt`
 *          (tensafe-he-python/src/lib.rs:322-350): a CkksContext rebuilt on
 *          the first `*` of the ciphertext object, pt re-encoded each call.
 * h: f64[d]; lora_a: f32[r][d]; lora_b: f32[d][r]; out delta f64[d],
 * out intermediate f64[r]. */
int or_lora_delta(const or_ctx *c, const uint64_t *sk_ntt, const double *h,
                  uint32_t d, const float *lora_a, const float *lora_b, uint32_t r,
                  uint64_t enc_seed, int mode, double *delta, double *intermediate);

/* NTT(plaintext) of each packed LoRA-A batch: out [n_batches][L][n]. */
int or_lora_pack(const or_ctx *c, const float *lora_a, uint32_t r, uint32_t d, uint64_t *out);
/* or_lora_delta with an optional pt cache from or_lora_pack (mode 0 only):
 * the fastest CPU form, ct_pt_mul_ntt on cached plaintexts. */
int or_lora_delta_cached(const or_ctx *c, const uint64_t *sk_ntt, const double *h,
                         uint32_t d, const float *lora_a, const float *lora_b, uint32_t r,
                         uint64_t enc_seed, int mode, const uint64_t *pt_cache, double *delta,
                         double *intermediate);

/* Test helper: first seed in [start, start+count) whose encrypt (kind 0) or
 * keygen (kind 1) stream hits a rejection; UINT64_MAX if none. */
uint64_t or_find_reject_seed(const uint64_t *moduli, uint32_t L, size_t n, uint64_t start,
                             uint64_t count, int kind);

#ifdef __cplusplus
}
#endif
#endif
