// common.cuh -- device arithmetic shared by every tsgpu kernel (sm_100a).
//
// 64-bit modular arithmetic for the RNS limbs of the reference parameter sets
// (tensafe-he-core/src/params.rs:66-126: 60- and 40-bit primes, all < 2^62):
//   * Shoup's precomputed-quotient product (V. Shoup, NTL) for a fixed
//     operand w with companion w' = floor(w * 2^64 / q): the result is
//     a*w mod q in [0, 2q) for any a < 2^64 -- used for NTT twiddles.
//   * Barrett reduction with mu = floor(2^(2k) / q), k = bitlen(q), for
//     products of two canonical residues -- used for data x data products
//     (ct x pt, c1 * s, a * s).
// Both give the exact residue, so results equal the reference's u128 Barrett
// (rns.rs:46-95) bit for bit.
//
// ChaCha20 (RFC 8439 block function) keyed the way the reference seeds it
// (rng.rs:38-68): key words = (seed_lo, seed_hi) x 4, counter in word 12,
// nonce 0.  The reference refills block 0 at construction, so stream word w
// is word (w mod 16) of the block with counter w / 16.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace tsg {

constexpr int kMaxLimbs = 8;

// ----------------------------------------------------------------- 64-bit mod
__device__ __forceinline__ uint64_t mulhi64(uint64_t a, uint64_t b) { return __umul64hi(a, b); }

// a*w mod q, lazily reduced to [0, 2q); valid for any a < 2^64 when q < 2^63.
__device__ __forceinline__ uint64_t mul_shoup_lazy(uint64_t a, uint64_t w, uint64_t wp, uint64_t q) {
    uint64_t qh = mulhi64(a, wp);
    return a * w - qh * q;
}

__device__ __forceinline__ uint64_t reduce_2q(uint64_t x, uint64_t q) { return x >= q ? x - q : x; }

// a*w mod q lazily reduced to [0, 4q), for any a < 2^64 (q < 2^62).
// Shoup's quotient floor(a*wp / 2^64) is estimated from three of the four
// 32x32 partial products (a1*w1 and the high halves of a1*w0, a0*w1); the
// dropped terms (a0*w0 and the carry of the middle sum) each add less than
// one to the exact quotient, so the estimate is low by at most 2 and the
// remainder a*w - qh*q lies in [0, 4q).
__device__ __forceinline__ uint64_t mul_shoup4(uint64_t a, uint64_t w, uint64_t wp, uint64_t q) {
    const uint32_t a0 = (uint32_t)a, a1 = (uint32_t)(a >> 32);
    const uint32_t w0 = (uint32_t)wp, w1 = (uint32_t)(wp >> 32);
    uint64_t qh = (uint64_t)a1 * w1;
    qh += __umulhi(a1, w0);
    qh += __umulhi(a0, w1);
    return a * w - qh * q;
}

// Per-limb constants for Barrett: mu = floor(2^(2k)/q), k = bitlen(q) <= 62.
struct BarrettConst {
    uint64_t q;
    uint64_t mu;
    int k;
};

// Exact (a*b) mod q for a, b < q.
__device__ __forceinline__ uint64_t mul_barrett(uint64_t a, uint64_t b, uint64_t q, uint64_t mu, int k) {
    uint64_t lo = a * b;
    uint64_t hi = mulhi64(a, b);
    // q1 = P >> (k-1), fits in k+1 bits
    uint64_t q1 = (hi << (65 - k)) | (lo >> (k - 1));
    uint64_t t_lo = q1 * mu;
    uint64_t t_hi = mulhi64(q1, mu);
    uint64_t q3 = (t_hi << (63 - k)) | (t_lo >> (k + 1));
    uint64_t r = lo - q3 * q;
    if (r >= q) r -= q;
    if (r >= q) r -= q;
    return r;
}

__device__ __forceinline__ uint64_t add_mod(uint64_t a, uint64_t b, uint64_t q) {
    uint64_t s = a + b;
    return s >= q ? s - q : s;
}

__device__ __forceinline__ uint64_t sub_mod(uint64_t a, uint64_t b, uint64_t q) {
    return a >= b ? a - b : a + q - b;
}

// x mod q for any 64-bit x, with mu64 = floor((2^64-1)/q).
__device__ __forceinline__ uint64_t mod_u64(uint64_t x, uint64_t q, uint64_t mu64) {
    uint64_t qt = mulhi64(x, mu64);
    uint64_t r = x - qt * q;
    if (r >= q) r -= q;
    if (r >= q) r -= q;
    return r;
}

// Residue of a signed coefficient exactly as the reference maps it
// (encoding.rs:198-202, ciphertext.rs:196-201): v >= 0 -> v % q, else
// q - ((-v) % q).  The negative branch yields q (not 0) when q | v, which
// the reference also does.
// Branch-free, so that callers' loads are not serialised behind divergent
// branches.
__device__ __forceinline__ uint64_t signed_residue(int64_t v, uint64_t q, uint64_t mu64) {
    const bool neg = v < 0;
    const uint64_t r = mod_u64(neg ? (uint64_t)0 - (uint64_t)v : (uint64_t)v, q, mu64);
    return neg ? q - r : r;
}

// ----------------------------------------------------------------- ChaCha20
__device__ __forceinline__ uint32_t rotl32(uint32_t x, int r) { return __funnelshift_l(x, x, r); }

#define TSG_QR(a, b, c, d)                     \
    a += b; d ^= a; d = rotl32(d, 16);          \
    c += d; b ^= c; b = rotl32(b, 12);          \
    a += b; d ^= a; d = rotl32(d, 8);           \
    c += d; b ^= c; b = rotl32(b, 7);

// Block with the given counter for the reference seed expansion.
__device__ __forceinline__ void chacha_block(uint64_t seed, uint32_t counter, uint32_t out[16]) {
    const uint32_t lo = (uint32_t)seed, hi = (uint32_t)(seed >> 32);
    uint32_t x0 = 0x61707865u, x1 = 0x3320646eu, x2 = 0x79622d32u, x3 = 0x6b206574u;
    uint32_t x4 = lo, x5 = hi, x6 = lo, x7 = hi, x8 = lo, x9 = hi, x10 = lo, x11 = hi;
    uint32_t x12 = counter, x13 = 0, x14 = 0, x15 = 0;
#pragma unroll
    for (int i = 0; i < 10; i++) {
        TSG_QR(x0, x4, x8, x12)
        TSG_QR(x1, x5, x9, x13)
        TSG_QR(x2, x6, x10, x14)
        TSG_QR(x3, x7, x11, x15)
        TSG_QR(x0, x5, x10, x15)
        TSG_QR(x1, x6, x11, x12)
        TSG_QR(x2, x7, x8, x13)
        TSG_QR(x3, x4, x9, x14)
    }
    out[0] = x0 + 0x61707865u; out[1] = x1 + 0x3320646eu; out[2] = x2 + 0x79622d32u; out[3] = x3 + 0x6b206574u;
    out[4] = x4 + lo; out[5] = x5 + hi; out[6] = x6 + lo; out[7] = x7 + hi;
    out[8] = x8 + lo; out[9] = x9 + hi; out[10] = x10 + lo; out[11] = x11 + hi;
    out[12] = x12 + counter; out[13] = x13; out[14] = x14; out[15] = x15;
}
#undef TSG_QR

// Single stream word (slow path: one block per call).
__device__ __forceinline__ uint32_t chacha_word(uint64_t seed, uint64_t w) {
    uint32_t b[16];
    chacha_block(seed, (uint32_t)(w >> 4), b);
    uint32_t r = b[0];
#pragma unroll
    for (int i = 1; i < 16; i++)
        if ((uint32_t)(w & 15) == (uint32_t)i) r = b[i];
    return r;
}

// next_f64 of the reference (rng.rs:139-144): ((u64 >> 11) + 0.5) / 2^53.
__device__ __forceinline__ double u64_to_unit(uint64_t u) {
    return __dmul_rn(__dadd_rn((double)(u >> 11), 0.5), 1.0 / 9007199254740992.0);
}

// Box-Muller, cosine branch, times sigma (rng.rs:152-157), evaluated with
// CUDA's log/cos/sqrt (sqrt is correctly rounded; log/cos are within a few
// ulp of glibc's).  Rounded to the nearest integer, half away from zero
// (f64::round).  *near_tie is set when the product lies within 1e-9 of a
// half-integer, the only case where an ulp-level difference from glibc could
// change the rounded integer.
__device__ __forceinline__ int gaussian_round(uint64_t u1w, uint64_t u2w, double sigma, bool* near_tie) {
    double u1 = u64_to_unit(u1w);
    double u2 = u64_to_unit(u2w);
    const double two_pi = 6.283185307179586;  // 2.0 * PI, exact doubling
    double z = __dmul_rn(sqrt(__dmul_rn(-2.0, log(u1))), cos(__dmul_rn(two_pi, u2)));
    double v = __dmul_rn(z, sigma);
    double a = fabs(v);
    double f = a - floor(a);
    *near_tie = fabs(f - 0.5) < 1e-9;
    return (int)round(v);
}

// The encryption's error sample round(3.19 * z) (sampling.rs:10, :51-58;
// rng.rs:152-157) with the transcendental work in float32 first.  CUDA's
// logf (at most 1 ulp), cosf (at most 2 ulp) and sqrtf (correctly rounded),
// with the rounding of u1, u2, 2*pi and 3.19 to float and of the products,
// put the float value v within 4.4e-5 of the exact 3.19 * z whenever
// |3.19 * z| >= 0.4, and below 0.402 in magnitude otherwise.  So when |v|
// lies more than kGaussGuard (5.7x that bound) from a half-integer, round(v)
// is the rounding of the reference's f64 value; the rest (about one sample
// in 2000) take the f64 evaluation, gaussian_round, with its near-tie count.
constexpr float kGaussGuard = 2.5e-4f;

__device__ __forceinline__ int gaussian_round_e(uint64_t u1w, uint64_t u2w, bool* near_tie) {
    const float u1 = __double2float_rn(u64_to_unit(u1w));
    const float u2 = __double2float_rn(u64_to_unit(u2w));
    const float v = __fmul_rn(__fmul_rn(sqrtf(__fmul_rn(-2.0f, logf(u1))), cosf(__fmul_rn(6.2831855f, u2))), 3.19f);
    const float a = fabsf(v);
    if (fabsf(a - floorf(a) - 0.5f) > kGaussGuard) {
        *near_tie = false;
        return (int)roundf(v);
    }
    return gaussian_round(u1w, u2w, 3.19, near_tie);
}

// ----------------------------------------------------------------- L2 prefetch
// Asks the TMA unit to pull [p, p + bytes) into L2 (p 16-byte aligned, bytes
// a multiple of 16); a hint that neither blocks nor touches shared memory.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// ----------------------------------------------------------------- u128 -> f64
// Round-to-nearest-even conversion of the 128-bit integer (hi, lo), as Rust's
// `u128 as f64` (used by the CRT branch of decrypt, ciphertext.rs:379-383).
// Branch-free: both the hi == 0 and the general result are formed and one
// is selected.
__device__ __forceinline__ double u128_to_f64(uint64_t hi, uint64_t lo) {
    const int lz = __clzll((long long)hi) & 63;  // (hi == 0 selects the other result)
    const int nbits = 128 - lz;
    const uint64_t top = lz ? ((hi << lz) | (lo >> (64 - lz))) : hi;
    const uint64_t rest = lz ? (lo << lz) : lo;
    uint64_t mant = top >> 11;
    const uint64_t rbit = (top >> 10) & 1;
    const bool sticky = ((top & 0x3FF) != 0) || (rest != 0);
    mant += (rbit && (sticky || (mant & 1))) ? 1 : 0;
    // mant < 2^54; scale by 2^(nbits-53) (exact)
    const double big =
        __dmul_rn(__ull2double_rn(mant), __longlong_as_double((long long)(1023 + nbits - 53) << 52));
    return hi ? big : __ull2double_rn(lo);
}

// Rust `f64 as i64` (saturating, NaN -> 0).
__device__ __forceinline__ int64_t f64_to_i64_sat(double x) {
    if (x != x) return 0;
    if (x >= 9223372036854775808.0) return INT64_MAX;
    if (x < -9223372036854775808.0) return INT64_MIN;
    return (int64_t)x;
}

}  // namespace tsg
