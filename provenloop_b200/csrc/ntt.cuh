// ntt.cuh -- negacyclic NTT / INTT device cores for one poly-limb per CTA.
//
// Computes exactly the transforms of tensafe-he-core/src/ntt.rs:
//   forward (ntt.rs:79-102): Cooley-Tukey, stage s has m = 2^s groups of
//     half-size t = N >> (s+1); group i uses twiddle fw[m + i], where
//     fw[brv(i)] = psi^i (rns.rs:161-171).  Output in bit-reversed order.
//   inverse (ntt.rs:113-141): Gentleman-Sande, t = 1 .. N/2, m = N/(2t),
//     twiddle iw[m + i] (iw[brv(i)] = psi^-i), then a final x N^-1.
// Any evaluation order of these exact modular butterflies yields the same
// canonical outputs, so the results are bit-identical to the reference.
//
// B200 layout: the whole poly-limb (N u64, 128 KiB at N = 16384) lives in
// one CTA's shared memory, padded to element j -> j + j/16 (136 KiB), which
// keeps every pass's access pattern bank-conflict free and turns each
// thread's 2^R addresses into one base plus compile-time offsets.  N/E
// threads each own E values in registers (E = 32 from N = 8192, else 16) and
// run radix-2^R passes (R up to log2 E: 5, 5, 4 stages at N = 16384) with one
// shared-memory exchange between passes.  Global memory is touched only in
// coalesced order j = tid + k*(N/E): the forward transform reads its input
// straight into the first pass and stages its bit-reversed output through
// shared memory; the inverse stages its input and writes its last pass
// straight out.  Callers supply the element loader and storer, so fused
// kernels transform on load and combine on store.
//
// Butterflies: Harvey-style lazy reduction with Shoup twiddle products whose
// quotient comes from three 32x32 partial products (remainder in [0, 4q));
// values stay in [0, 8q) forward and [0, 4q) inverse, which needs q < 2^61
// (the reference's primes are <= 60 bits).  Inverse transforms of limbs
// with headroom (q < 2^(61 - log2 N), the 40-bit primes) skip the per-stage
// corrections entirely (the NC variants below).
// Each twiddle and its companion are one 16-byte load.  N^-1 is folded into
// the last inverse stage.
//
// N = 32768 (256 KiB per poly-limb) spans a cluster of two CTAs (CL = 2):
// CTA h holds elements [h*N/2, (h+1)*N/2) in its own padded shared memory
// and 512 threads x 32 values.  Of the three radix-32 passes, the one whose
// butterflies cross the halves (spans N/32 .. N/2: the forward's first, the
// inverse's last) is split by sets, each CTA taking half of the 1024 sets
// and reaching the partner's elements through distributed shared memory;
// the other two passes are local.  The kernel must then be launched with
// cluster dimension 2 along x, and block pairs see the same work item.
// The same split is available from N = 8192 (CL = 2 as a template argument),
// which halves the work of a lone transform's CTA when a small batch leaves
// most SMs idle.  Below N = 32768 a pair keeps 16 values per thread (radix-16
// passes, N/32 threads per CTA), so each CTA still has 16 warps to hide the
// latency of its loads.
#pragma once
#include <cooperative_groups.h>

#include <type_traits>

#include "common.cuh"

namespace tsg {

// Per-limb device constants (one entry per RNS limb, in global memory).
struct LimbTab {
    const uint64_t* tw;  // [2][n][2]: (fw, fw') pairs then (iw, iw') pairs, x' = Shoup companion
    uint64_t q;
    uint64_t ninv, ninvs;  // N^-1 mod q and companion
    uint64_t iw1n, iw1ns;  // iw[1] * N^-1 mod q and companion
    uint64_t mu64;         // floor((2^64 - 1) / q)
    uint64_t bmu;          // Barrett floor(2^(2k) / q)
    uint64_t thresh;       // 2^64 mod q: range_u64 rejection threshold (rng.rs:126)
    int bk;                // bitlen(q)
    int fp;                // q < 2^50: the transforms run in FP64 (below); tables at tw + 4n; 2: q < 2^44, lazy
};

// Padded shared-memory index of element j.
__device__ __forceinline__ int pad(int j) { return j + (j >> 4); }

// CTAs per transform by default: two from N = 32768 (a poly-limb no longer
// fits one CTA).  Smaller transforms may also be split over a pair (CL = 2
// from N = 8192) to halve the latency of a lone transform.
__host__ __device__ constexpr int ntt_default_cl(int logn) { return logn >= 15 ? 2 : 1; }

template <int LOGN, int CL_ = ntt_default_cl(LOGN)>
struct NttCfg {
    static constexpr int N = 1 << LOGN;
    static constexpr int CL = CL_;                  // CTAs per transform (cluster size)
    static constexpr int H = N / CL;                // elements held by one CTA
    // values per thread: 32 from N = 8192 on one CTA; a pair holds 16, so
    // that its CTAs keep 512 threads (N = 8192, 16384; two CTAs per SM) or
    // 1024 (N = 32768, whose shares allow one CTA per SM) to hide latency
    static constexpr int E = LOGN >= 13 && CL_ == 1 ? 32 : 16;
    static constexpr int NT = H / E;                // threads per CTA
    static constexpr int JS = N / E;                // element stride of a first-pass set
    static constexpr int RMAX = E == 32 ? 5 : 4;    // stages per pass
    static constexpr int SMEM_WORDS = H + H / 16;   // padded share of the poly-limb
    static constexpr int NPASS = (LOGN + RMAX - 1) / RMAX;
    // stages of forward pass p: RMAX each, the last pass the remainder
    __host__ __device__ static constexpr int fwd_r(int p) { return p < NPASS - 1 ? RMAX : LOGN - RMAX * (NPASS - 1); }
    __host__ __device__ static constexpr int fwd_s0(int p) { return p * RMAX; }
    static_assert(CL == 1 || (CL == 2 && LOGN >= 13), "pairs from N = 8192");
};

// Geometry of a radix-2^R pass whose smallest butterfly span is 2^TLOG:
// set sigma = (g, o), g = sigma >> TLOG, o = sigma & (2^TLOG - 1); its k-th
// element is j = j0 + (k << TLOG) with j0 = (g << (TLOG + R)) + o.  Thread
// tid owns sets sigma = tid + NT*u, u < SETS.  j0 and k << TLOG occupy
// disjoint bits, so pad(j0 + (k << TLOG)) = pad(j0) + K + K/16 with
// K = k << TLOG: one base register plus a compile-time offset.
//
// With CL = 2 the CTA of rank h takes sets h*NT*SETS .. (h+1)*NT*SETS - 1.
// In a local pass (TLOG + R < LOGN) those are exactly the sets whose
// elements lie in half h, and pbase gives the local padded address.
template <int LOGN, int R, int TLOG, int CL = ntt_default_cl(LOGN)>
struct Geo {
    static constexpr int N = 1 << LOGN;
    static constexpr int NT = NttCfg<LOGN, CL>::NT;
    static constexpr int H = NttCfg<LOGN, CL>::H;
    static constexpr int SETS = NttCfg<LOGN, CL>::E >> R;
    __device__ __forceinline__ static int sigma(int h, int tid, int u) { return h * NT * SETS + tid + NT * u; }
    __device__ __forceinline__ static int pbase(int sg) {
        return pad((((sg >> TLOG) << (TLOG + R)) + (sg & ((1 << TLOG) - 1))) & (H - 1));
    }
    __host__ __device__ static constexpr int koff(int k) { return (k << TLOG) + ((k << TLOG) >> 4); }
};

// Values of a transform: u64 residues (integer modes) or FP64 integers
// (FP64 mode); shared memory holds their 64-bit patterns either way.
constexpr int kModeInt = 0, kModeNC = 1, kModeFp = 2, kModeFpLazy = 3;
__host__ __device__ constexpr bool is_fp(int m) { return m == kModeFp || m == kModeFpLazy; }
template <int M>
using NttV = typename std::conditional<is_fp(M), double, uint64_t>::type;
__device__ __forceinline__ uint64_t vbits(uint64_t x) { return x; }
__device__ __forceinline__ uint64_t vbits(double x) { return (uint64_t)__double_as_longlong(x); }
template <class V>
__device__ __forceinline__ V vfrom(uint64_t b) {
    if constexpr (std::is_same<V, double>::value) return __longlong_as_double((long long)b);
    else return b;
}

template <int LOGN, int R, int TLOG, int CL, class V>
__device__ __forceinline__ void smem_load(const uint64_t* sm, V* v, int h, int tid) {
    using G = Geo<LOGN, R, TLOG, CL>;
#pragma unroll
    for (int u = 0; u < G::SETS; u++) {
        const uint64_t* b = sm + G::pbase(G::sigma(h, tid, u));
#pragma unroll
        for (int k = 0; k < (1 << R); k++) v[u * (1 << R) + k] = vfrom<V>(b[G::koff(k)]);
    }
}

template <int LOGN, int R, int TLOG, int CL, class V>
__device__ __forceinline__ void smem_store(uint64_t* sm, const V* v, int h, int tid) {
    using G = Geo<LOGN, R, TLOG, CL>;
#pragma unroll
    for (int u = 0; u < G::SETS; u++) {
        uint64_t* b = sm + G::pbase(G::sigma(h, tid, u));
#pragma unroll
        for (int k = 0; k < (1 << R); k++) b[G::koff(k)] = vbits(v[u * (1 << R) + k]);
    }
}

// Cluster helpers (CL = 2).  The rank, and shared memory of either CTA of
// the pair as a generic pointer.
__device__ __forceinline__ int cluster_rank() { return (int)cooperative_groups::this_cluster().block_rank(); }
__device__ __forceinline__ void cluster_sync() { cooperative_groups::this_cluster().sync(); }
__device__ __forceinline__ uint64_t* cluster_smem(uint64_t* sm, int rank) {
    return cooperative_groups::this_cluster().map_shared_rank(sm, rank);
}
// A transform pair is cluster ranks (2i, 2i + 1): a cluster may hold several
// pairs (one per limb), which then take the same barriers in step.
__device__ __forceinline__ int pair_base() { return cluster_rank() & ~1; }

// Padded local offset of element k*JS of a cross-half set, k < E/2.  A
// set base sigma < JS has no bits in common with k*JS (a multiple of JS), so
// pad(sigma + k*JS) = pad(sigma) + xoff(k): one base register per half plus
// compile-time offsets.
template <int LOGN, int CL>
__host__ __device__ constexpr int xoff(int k) {
    return k * NttCfg<LOGN, CL>::JS + ((k * NttCfg<LOGN, CL>::JS) >> 4);
}

// Rank of this CTA within its transform (0 unless CL = 2).
template <int LOGN, int CL = ntt_default_cl(LOGN)>
__device__ __forceinline__ int ntt_rank() {
    if constexpr (CL == 2) return cluster_rank() & 1;
    return 0;
}

// One forward CT stage (sub-stage r of a radix-2^R pass starting at stage
// S0) on the 2^R values x of set-group g.  Template recursion keeps every
// loop bound a compile-time constant so x stays in registers.
// NC ("no correction") drops the X >= 4q step: each stage then adds at most
// 4q to the bound, so inputs < 8q stay below 8q + 4q*LOGN <= 64q, which fits
// 64 bits for q < 2^57 (the 40/50-bit limbs).
template <int R, int S0, int r, bool NC>
__device__ __forceinline__ void fwd_stage(uint64_t* x, int g, const ulonglong2* __restrict__ fw, uint64_t q,
                                          uint64_t q4) {
    constexpr int half = 1 << (R - 1 - r);
#pragma unroll
    for (int gi = 0; gi < (1 << r); gi++) {
        const ulonglong2 w = __ldg(fw + (1 << (S0 + r)) + (g << r) + gi);
#pragma unroll
        for (int kk = 0; kk < half; kk++) {
            const int k = gi * 2 * half + kk;
            uint64_t X = x[k];
            if constexpr (!NC) X = X >= q4 ? X - q4 : X;             // [0, 4q)
            const uint64_t T = mul_shoup4(x[k + half], w.x, w.y, q);  // [0, 4q)
            x[k] = X + T;                                             // [0, 8q) (NC: bound + 4q)
            x[k + half] = X + q4 - T;                                 // (0, 8q) (NC: bound + 4q)
        }
    }
    if constexpr (r + 1 < R) fwd_stage<R, S0, r + 1, NC>(x, g, fw, q, q4);
}

// ---------------------------------------------------------------- FP64 mode
// Limbs with q < 2^50 run their butterflies on the FP64 pipe, which issues
// these products at about 2.5x the rate of the 64-bit integer Shoup product
// (measured on register-resident radix-32 passes, 50-bit modulus).  Values
// are integers held exactly in doubles, balanced around 0; twiddles are
// balanced too (|w| <= q/2) and stored with wq = fl(w / q).
//
// fp_mulmod(y, w, wq): b = the integer nearest y*wq, T = y*w - b*q with
// y*w = h + l split exactly by an FMA (h = fl(y*w), l = fma(y, w, -h)).
// b comes from the round-to-integer constant R = 1.5 * 2^52: for |t| < 2^51,
// fl(t + R) lies in [2^52, 2^53), where the spacing of doubles is 1, so
// fl(fma(y, wq, R)) - R is y*wq rounded once to the nearest integer (two
// full-rate FP64 operations; no separate round-to-integer instruction).
// For |y| <= 2^52 and q < 2^50: |y*wq - y*w/q| <= |y| * 2^-54, so
// |T| <= q(1/2 + |y|2^-54) <= q; h - b*q is an integer below 2^53 in
// magnitude, hence fma(-b, q, h) and the final + l are exact.  T is
// congruent to y*w mod q, so every butterfly is exact modular arithmetic,
// and the canonical outputs equal the integer path's bit for bit.
//
// Bounds (B = largest |value|, q < 2^50 so q * 2^-53 < 1/8):
//   forward CT: B' = B + q(1/2 + B 2^-53).  From B = q/2 at the start of a
//     pass, five stages reach 1.06q, 1.70q, 2.41q, 3.21q, 4.11q: products
//     see |y| <= 3.21q <= 2^52, and every value stays below 2^53.
//   inverse GS: the sums double per stage, so the sum outputs of the
//     second and fourth stage of a pass are reduced; products then see
//     |y| <= 3.5q.
// Every pass ends with a reduction to |v| <= q/2 (plus a rounding sliver),
// so each pass starts from the same bound.
// Lazy mode (kModeFpLazy, q < 2^44): the forward transform reduces after its
// last pass only, and the inverse only at the end of each pass.  Forward:
// each of at most 15 stages adds at most q(1/2 + |y|2^-54) <= 0.52q, so
// values stay below 8.5q.  Inverse: sums double within a pass of at most
// five stages, so they stay below 16q.  Products then see |y| <= 16q, so
// |y*wq| <= 8q < 2^51 (the rounding constant's range) and
// |y|q2^-54 <= q2^-6; every value stays far below 2^53, and the products
// keep |T| <= 0.52q.  Removing the reductions saves three FP64 operations
// per element and pass (forward) or per sum of two stages (inverse).
constexpr double kFpRound = 6755399441055744.0;  // 1.5 * 2^52

// nearest integer to x*y (ties to even) for |x*y| < 2^51, one rounding
__device__ __forceinline__ double fp_round_mul(double x, double y) {
    return __dsub_rn(__fma_rn(x, y, kFpRound), kFpRound);
}

__device__ __forceinline__ double fp_mulmod(double y, double w, double wq, double q) {
    const double h = __dmul_rn(y, w);
    const double l = __fma_rn(y, w, -h);
    const double b = fp_round_mul(y, wq);
    return __dadd_rn(__fma_rn(-b, q, h), l);
}

// v - q*round(v/q): |result| <= q/2 + a sliver, exact (an integer < 2^53);
// an NTT prime exceeds 2N >= 2^13, so |v/q| < 2^40, far inside 2^51
__device__ __forceinline__ double fp_reduce(double v, double q, double qinv) {
    return __fma_rn(-fp_round_mul(v, qinv), q, v);
}

// Per-transform FP64 constants, derived from the limb's table entry: the
// (w, w/q) pairs at tw + 4n (forward) and tw + 6n (inverse), q, fl(1/q),
// and the last inverse stage's N^-1 and iw[1]*N^-1, balanced, with their
// quotients by q.
struct FpK {
    const double2* fw;
    const double2* iw;
    double q, qinv, ninv, ninvq, iw1n, iw1nq;
};

__device__ __forceinline__ double fp_bal(uint64_t x, uint64_t q) {
    return x > q / 2 ? -__ull2double_rn(q - x) : __ull2double_rn(x);
}

template <int N>
__device__ __forceinline__ FpK fp_consts(const LimbTab& T) {
    FpK F;
    F.fw = reinterpret_cast<const double2*>(T.tw + 4 * N);
    F.iw = reinterpret_cast<const double2*>(T.tw + 6 * N);
    F.q = __ull2double_rn(T.q);
    F.qinv = __drcp_rn(F.q);
    F.ninv = fp_bal(T.ninv, T.q);
    F.ninvq = __ddiv_rn(F.ninv, F.q);
    F.iw1n = fp_bal(T.iw1n, T.q);
    F.iw1nq = __ddiv_rn(F.iw1n, F.q);
    return F;
}

// u64 residue (< 2^53) -> balanced FP64 value
__device__ __forceinline__ double fp_in(uint64_t x, const FpK& F) {
    return fp_reduce(__ull2double_rn(x), F.q, F.qinv);
}

// balanced FP64 value (|v| < q) -> canonical u64 residue
__device__ __forceinline__ uint64_t fp_out(double v, const FpK& F) {
    return __double2ull_rn(v < 0.0 ? __dadd_rn(v, F.q) : v);
}

template <int R, int S0, int r>
__device__ __forceinline__ void fwd_stage_fp(double* x, int g, const double2* __restrict__ fw, double q) {
    constexpr int half = 1 << (R - 1 - r);
#pragma unroll
    for (int gi = 0; gi < (1 << r); gi++) {
        const double2 w = __ldg(fw + (1 << (S0 + r)) + (g << r) + gi);
#pragma unroll
        for (int kk = 0; kk < half; kk++) {
            const int k = gi * 2 * half + kk;
            const double X = x[k];
            const double Tv = fp_mulmod(x[k + half], w.x, w.y, q);
            x[k] = __dadd_rn(X, Tv);
            x[k + half] = __dsub_rn(X, Tv);
        }
    }
    if constexpr (r + 1 < R) fwd_stage_fp<R, S0, r + 1>(x, g, fw, q);
}

// K: the LimbTab (integer modes) or the FpK (FP64 mode) of the transform.
template <int LOGN, int R, int S0, int M, int CL, class K>
__device__ __forceinline__ void fwd_compute(NttV<M>* v, const K& T, int h, int tid) {
    constexpr int TLOG = LOGN - S0 - R;
    using G = Geo<LOGN, R, TLOG, CL>;
    if constexpr (is_fp(M)) {
#pragma unroll
        for (int u = 0; u < G::SETS; u++)
            fwd_stage_fp<R, S0, 0>(v + u * (1 << R), G::sigma(h, tid, u) >> TLOG, T.fw, T.q);
        // the lazy mode reduces after the last pass only
        if constexpr (M == kModeFp || S0 + R == LOGN) {
#pragma unroll
            for (int k = 0; k < NttCfg<LOGN, CL>::E; k++) v[k] = fp_reduce(v[k], T.q, T.qinv);
        }
    } else {
        const ulonglong2* fw = reinterpret_cast<const ulonglong2*>(T.tw);
#pragma unroll
        for (int u = 0; u < G::SETS; u++)
            fwd_stage<R, S0, 0, M == kModeNC>(v + u * (1 << R), G::sigma(h, tid, u) >> TLOG, fw, T.q, 4 * T.q);
    }
}

// One inverse GS stage (span 2^(TLOG+r)) on values in [0, 4q); the stage of
// span N/2 folds N^-1 into both outputs.
// NC drops the X + Y >= 4q step: the bound then doubles per stage, from 4q
// before global stage 0 to 4q * 2^s before stage s, and the difference
// branch adds that bound instead of 4q.  Everything stays below 2^64 for
// q < 2^(61 - LOGN) (the 40-bit limbs).
template <int LOGN, int R, int TLOG, int r, bool NC>
__device__ __forceinline__ void inv_stage(uint64_t* x, int g, const ulonglong2* __restrict__ iw, const LimbTab& T,
                                          uint64_t q4) {
    constexpr int span = 1 << r;
    constexpr int m = 1 << (LOGN - TLOG - r - 1);
    constexpr bool last = (TLOG + r == LOGN - 1);
    const uint64_t q = T.q;
    const uint64_t off = NC ? q4 << (TLOG + r) : q4;  // bound of the inputs of this stage
#pragma unroll
    for (int gi = 0; gi < ((1 << R) >> (r + 1)); gi++) {
        ulonglong2 w;
        if constexpr (last) {
            w.x = T.iw1n;
            w.y = T.iw1ns;
        } else {
            w = __ldg(iw + m + (g << (R - r - 1)) + gi);
        }
#pragma unroll
        for (int kk = 0; kk < span; kk++) {
            const int k = gi * 2 * span + kk;
            const uint64_t X = x[k], Y = x[k + span];
            if constexpr (last) {
                x[k] = mul_shoup4(X + Y, T.ninv, T.ninvs, q);
            } else if constexpr (NC) {
                x[k] = X + Y;
            } else {
                const uint64_t s = X + Y;
                x[k] = s >= q4 ? s - q4 : s;
            }
            x[k + span] = mul_shoup4(X + off - Y, w.x, w.y, q);
        }
    }
    if constexpr (r + 1 < R) inv_stage<LOGN, R, TLOG, r + 1, NC>(x, g, iw, T, q4);
}

// FP64 inverse stage: sums of the pass's second and fourth stage (r = 1, 3)
// are reduced, which keeps every product input below 3.5q (bounds above).
template <int LOGN, int R, int TLOG, int r, bool LAZY>
__device__ __forceinline__ void inv_stage_fp(double* x, int g, const double2* __restrict__ iw, const FpK& T) {
    constexpr int span = 1 << r;
    constexpr int m = 1 << (LOGN - TLOG - r - 1);
    constexpr bool last = (TLOG + r == LOGN - 1);
    const double q = T.q;
#pragma unroll
    for (int gi = 0; gi < ((1 << R) >> (r + 1)); gi++) {
        double2 w;
        if constexpr (last) {
            w.x = T.iw1n;
            w.y = T.iw1nq;
        } else {
            w = __ldg(iw + m + (g << (R - r - 1)) + gi);
        }
#pragma unroll
        for (int kk = 0; kk < span; kk++) {
            const int k = gi * 2 * span + kk;
            const double X = x[k], Y = x[k + span];
            const double s = __dadd_rn(X, Y);
            if constexpr (last) x[k] = fp_mulmod(s, T.ninv, T.ninvq, q);
            else if constexpr ((r & 1) && !LAZY) x[k] = fp_reduce(s, q, T.qinv);
            else x[k] = s;
            x[k + span] = fp_mulmod(__dsub_rn(X, Y), w.x, w.y, q);
        }
    }
    if constexpr (r + 1 < R) inv_stage_fp<LOGN, R, TLOG, r + 1, LAZY>(x, g, iw, T);
}

template <int LOGN, int R, int TLOG, int M, int CL, class K>
__device__ __forceinline__ void inv_compute(NttV<M>* v, const K& T, int h, int tid) {
    using G = Geo<LOGN, R, TLOG, CL>;
    if constexpr (is_fp(M)) {
#pragma unroll
        for (int u = 0; u < G::SETS; u++)
            inv_stage_fp<LOGN, R, TLOG, 0, M == kModeFpLazy>(v + u * (1 << R), G::sigma(h, tid, u) >> TLOG, T.iw, T);
#pragma unroll
        for (int k = 0; k < NttCfg<LOGN, CL>::E; k++) v[k] = fp_reduce(v[k], T.q, T.qinv);
    } else {
        const ulonglong2* iw = reinterpret_cast<const ulonglong2*>(T.tw) + NttCfg<LOGN, CL>::N;
#pragma unroll
        for (int u = 0; u < G::SETS; u++)
            inv_stage<LOGN, R, TLOG, 0, M == kModeNC>(v + u * (1 << R), G::sigma(h, tid, u) >> TLOG, iw, T,
                                                      4 * T.q);
    }
}

// [0, 8q) -> [0, q)
__device__ __forceinline__ uint64_t canon8(uint64_t x, uint64_t q) {
    x = x >= 4 * q ? x - 4 * q : x;
    x = x >= 2 * q ? x - 2 * q : x;
    return x >= q ? x - q : x;
}

// [0, 4q) -> [0, q)
__device__ __forceinline__ uint64_t canon4(uint64_t x, uint64_t q) {
    x = x >= 2 * q ? x - 2 * q : x;
    return x >= q ? x - q : x;
}

// A loaded residue as a value of mode M, and a final value as a canonical
// residue (forward: from shared memory, [0, 8q) for the integer modes).
template <int M, class K>
__device__ __forceinline__ NttV<M> ntt_in(uint64_t x, const K& T) {
    if constexpr (is_fp(M)) return fp_in(x, T);
    else return x;
}

// An exact integer-valued double (|x| < 2^52) as a value of an FP64 mode:
// reduced like fp_in reduces a residue (|x * fl(1/q)| stays far inside the
// rounding constant's 2^51, and x - q*round(x/q) is an exact integer).
template <int M, class K>
__device__ __forceinline__ NttV<M> ntt_in(double x, const K& T) {
    static_assert(is_fp(M), "signed double inputs enter the FP64 modes only");
    return fp_reduce(x, T.q, T.qinv);
}

// The transform's constants for mode M: the table entry itself, or FpK.
template <int LOGN, int M>
__device__ __forceinline__ auto ntt_consts(const LimbTab& T) {
    if constexpr (is_fp(M)) return fp_consts<(1 << LOGN)>(T);
    else return T;
}

// Forward pass P (stages fwd_s0(P) ..) and the ones after it.  Pass 0's
// values are already in v; every pass stores its results back to the
// positions it read (its own sets), so one barrier between passes suffices.
template <int LOGN, int P, int M, int CL, class K>
__device__ __forceinline__ void fwd_passes(uint64_t* sm, NttV<M>* v, const K& T, int h, int tid) {
    using C = NttCfg<LOGN, CL>;
    constexpr int R = C::fwd_r(P), S0 = C::fwd_s0(P), TLOG = LOGN - S0 - R;
    if constexpr (P > 0) {
        if constexpr (C::CL == 2 && P == 1) cluster_sync();  // both halves written
        else __syncthreads();
        smem_load<LOGN, R, TLOG, CL>(sm, v, h, tid);
    }
    fwd_compute<LOGN, R, S0, M, CL>(v, T, h, tid);
    if constexpr (C::CL == 2 && P == 0) {
        // the first pass's sets span both halves: element sigma + k*JS goes
        // to CTA k / (E/2).  The partner must be done reading its shared
        // memory (the previous transform, or a loader that reads it) first.
        static_assert((1 << R) == C::E, "the cross-half pass holds a whole set per thread");
        cluster_sync();
        const int sg = Geo<LOGN, R, TLOG, CL>::sigma(h, tid, 0);
        uint64_t* s0 = cluster_smem(sm, pair_base()) + pad(sg);
        uint64_t* s1 = cluster_smem(sm, pair_base() + 1) + pad(sg);
#pragma unroll
        for (int k = 0; k < C::E; k++) (k < C::E / 2 ? s0 : s1)[xoff<LOGN, CL>(k & (C::E / 2 - 1))] = vbits(v[k]);
    } else {
        smem_store<LOGN, R, TLOG, CL>(sm, v, h, tid);
    }
    if constexpr (P + 1 < C::NPASS) fwd_passes<LOGN, P + 1, M, CL>(sm, v, T, h, tid);
}

// Forward transform of one poly-limb.  ld(j) returns element j (< 8q, e.g.
// canonical) for j = sigma + k*JS, sigma = rank*NT + tid (rank 0 unless
// CL = 2); st(j, v) receives canonical output j for j = rank*H + tid + k*NT,
// coalesced.  `sm` holds NttCfg<LOGN>::SMEM_WORDS u64.  All NT threads of
// the block (both blocks of the cluster for CL = 2) must call this; a caller
// that reuses `sm` afterwards must __syncthreads() first.  A caller whose
// input is staged in shared memory uses ntt_forward_from_smem instead.
// first(k, sigma) supplies element sigma + k*JS of the first-pass set
// (k is a compile-time constant after unrolling).
template <int LOGN, int M, int CL = ntt_default_cl(LOGN), class First, class St>
__device__ __forceinline__ void ntt_forward_core(uint64_t* sm, const LimbTab& T, First& first, St& st) {
    using C = NttCfg<LOGN, CL>;
    static_assert(LOGN >= 10 && LOGN <= 15, "NTT supports N in [1024, 32768]");
    static_assert(C::fwd_r(0) == C::RMAX, "the first pass takes RMAX stages");
    const int tid = threadIdx.x;
    const int h = ntt_rank<LOGN, CL>();
    const auto K = ntt_consts<LOGN, M>(T);
    NttV<M> v[C::E];
    // first pass: one set per thread, elements sigma + k*JS
    const int sg = h * C::NT + tid;
#pragma unroll
    for (int k = 0; k < C::E; k++) v[k] = ntt_in<M>(first(k, sg), K);
    fwd_passes<LOGN, 0, M, CL>(sm, v, K, h, tid);
    __syncthreads();
    // own share, coalesced: j = h*H + tid + k*NT
#pragma unroll
    for (int k = 0; k < C::E; k++) {
        const int jl = tid + k * C::NT;
        uint64_t y;
        if constexpr (is_fp(M)) y = fp_out(vfrom<double>(sm[pad(jl)]), K);
        else if constexpr (M == kModeNC) y = mod_u64(sm[pad(jl)], T.q, T.mu64);
        else y = canon8(sm[pad(jl)], T.q);
        st(h * C::H + jl, y);
    }
}

// FP64 forward transform: the lazy mode for limbs the table marks (fp == 2,
// q < 2^44), else the reducing one (a uniform branch per CTA).
template <int LOGN, int CL, class First, class St>
__device__ __forceinline__ void ntt_forward_fp(uint64_t* sm, const LimbTab& T, First& first, St& st) {
    if (T.fp == 2)
        ntt_forward_core<LOGN, kModeFpLazy, CL>(sm, T, first, st);
    else
        ntt_forward_core<LOGN, kModeFp, CL>(sm, T, first, st);
}

// Forward transform of the loader's elements: FP64 for limbs with q < 2^50,
// integer otherwise (a uniform branch per CTA).  The correction-free integer
// variant measured no faster here: the forward integer butterfly is bound by
// the IMAD pipe, not by the ALU instructions NC removes.
// FPOK = false keeps a kernel integer-only (less code and fewer registers
// where the FP64 mode does not pay).
template <int LOGN, int CL = ntt_default_cl(LOGN), bool FPOK = true, class Ld, class St>
__device__ __forceinline__ void ntt_forward_block(uint64_t* sm, const LimbTab& T, Ld ld, St st) {
    auto first = [&](int k, int sg) { return ld(sg + k * NttCfg<LOGN, CL>::JS); };
    if (FPOK && T.fp)
        ntt_forward_fp<LOGN, CL>(sm, T, first, st);
    else
        ntt_forward_core<LOGN, kModeInt, CL>(sm, T, first, st);
}

// Forward transform of the signed integers x_j = m_j + e_j (ldm(j): the
// i64 coefficient m_j; lde(j): the small error |e_j| < 128), congruent to the
// residue the reference forms per limb, signed_residue(m) + residue(e) mod q
// (encoding.rs:198-202, ciphertext.rs:196-201).  The FP64 modes take x_j as
// an exact double when |m_j| < 2^52 (their input reduction does the rest);
// the integer modes take x_j or q + x_j when |m_j| < q - 128.  Coefficients
// outside those ranges go through the exact 64-bit reduction.  The outputs
// equal those of ntt_forward_block on the reference's residues.
template <int LOGN, int CL = ntt_default_cl(LOGN), bool FPOK = true, class Ldm, class Lde, class St>
__device__ __forceinline__ void ntt_forward_signed(uint64_t* sm, const LimbTab& T, Ldm ldm, Lde lde, St st) {
    using C = NttCfg<LOGN, CL>;
    auto slow = [&](int64_t m, int e) {  // the reference's two residues, added mod q
        return add_mod(signed_residue(m, T.q, T.mu64), e >= 0 ? (uint64_t)e : T.q + e, T.q);
    };
    if (FPOK && T.fp) {
        auto first = [&](int k, int sg) -> double {
            const int j = sg + k * C::JS;
            const int64_t m = ldm(j);
            const int e = lde(j);
            if (m > -(1LL << 52) && m < (1LL << 52)) return (double)(m + e);  // exact below 2^53
            return __ull2double_rn(slow(m, e));                              // < q < 2^50: exact
        };
        ntt_forward_fp<LOGN, CL>(sm, T, first, st);
    } else {
        const int64_t lim = (int64_t)T.q - 128;
        auto first = [&](int k, int sg) -> uint64_t {
            const int j = sg + k * C::JS;
            const int64_t m = ldm(j);
            const int e = lde(j);
            if (m > -lim && m < lim) {
                const int64_t x = m + e;  // |x| < q
                return x >= 0 ? (uint64_t)x : T.q - (uint64_t)(-x);
            }
            return slow(m, e);
        };
        ntt_forward_core<LOGN, kModeInt, CL>(sm, T, first, st);
    }
}

// Forward transform of a poly-limb already staged in shared memory (u64
// residues): each CTA's share at its own padded local positions, complete
// (__syncthreads, or cluster_sync for CL = 2) before the call.  The first
// pass reads it with the half chosen at compile time, so no per-element
// address selection.
// DBL: for limbs in an FP64 mode the staged words are the bits of exact
// integer-valued doubles (|x| < 2^52) instead of u64 residues.
template <int LOGN, int CL = ntt_default_cl(LOGN), bool FPOK = true, bool DBL = false, class St>
__device__ __forceinline__ void ntt_forward_from_smem(uint64_t* sm, const LimbTab& T, St st) {
    using C = NttCfg<LOGN, CL>;
    if constexpr (CL == 2) {
        const int sg0 = ntt_rank<LOGN, CL>() * C::NT + threadIdx.x;
        const uint64_t* s0 = cluster_smem(sm, pair_base()) + pad(sg0);
        const uint64_t* s1 = cluster_smem(sm, pair_base() + 1) + pad(sg0);
        auto first = [&](int k, int) { return (k < C::E / 2 ? s0 : s1)[xoff<LOGN, CL>(k & (C::E / 2 - 1))]; };
        if (FPOK && T.fp) {
            if constexpr (DBL) {
                auto firstd = [&](int k, int sg) { return vfrom<double>(first(k, sg)); };
                ntt_forward_fp<LOGN, CL>(sm, T, firstd, st);
            } else {
                ntt_forward_fp<LOGN, CL>(sm, T, first, st);
            }
        } else {
            ntt_forward_core<LOGN, kModeInt, CL>(sm, T, first, st);
        }
    } else {
        auto first = [&](int k, int sg) { return sm[pad(sg + k * C::JS)]; };
        if (FPOK && T.fp) {
            if constexpr (DBL) {
                auto firstd = [&](int k, int sg) { return vfrom<double>(first(k, sg)); };
                ntt_forward_fp<LOGN, CL>(sm, T, firstd, st);
            } else {
                ntt_forward_fp<LOGN, CL>(sm, T, first, st);
            }
        } else {
            ntt_forward_core<LOGN, kModeInt, CL>(sm, T, first, st);
        }
    }
}

// Inverse pass P in GS order (spans 1 .. N/2) mirrors forward pass
// NPASS-1-P.  Its values are in shared memory on entry; the last pass keeps
// its results (elements tid + k*NT) in v.
template <int LOGN, int P, int M, int CL, class K>
__device__ __forceinline__ void inv_passes(uint64_t* sm, NttV<M>* v, const K& T, int h, int tid) {
    using C = NttCfg<LOGN, CL>;
    constexpr int FP = C::NPASS - 1 - P;
    constexpr int R = C::fwd_r(FP), TLOG = LOGN - C::fwd_s0(FP) - R;
    if constexpr (C::CL == 2 && FP == 0) {
        // the last pass's sets span both halves: element sigma + k*JS is in
        // CTA k / (E/2); once both CTAs hold their values in registers the
        // partner may reuse its shared memory
        static_assert((1 << R) == C::E, "the cross-half pass holds a whole set per thread");
        cluster_sync();
        const int sg = Geo<LOGN, R, TLOG, CL>::sigma(h, tid, 0);
        const uint64_t* s0 = cluster_smem(sm, pair_base()) + pad(sg);
        const uint64_t* s1 = cluster_smem(sm, pair_base() + 1) + pad(sg);
#pragma unroll
        for (int k = 0; k < C::E; k++)
            v[k] = vfrom<NttV<M>>((k < C::E / 2 ? s0 : s1)[xoff<LOGN, CL>(k & (C::E / 2 - 1))]);
        cluster_sync();
    } else {
        __syncthreads();
        smem_load<LOGN, R, TLOG, CL>(sm, v, h, tid);
    }
    inv_compute<LOGN, R, TLOG, M, CL>(v, T, h, tid);
    if constexpr (P + 1 < C::NPASS) {
        smem_store<LOGN, R, TLOG, CL>(sm, v, h, tid);
        inv_passes<LOGN, P + 1, M, CL>(sm, v, T, h, tid);
    }
}

// Inverse transform (including x N^-1) of one poly-limb; ld(j) returns
// element j (< 4q) for j = rank*H + tid + k*NT.  A caller that reuses `sm`
// afterwards must __syncthreads() first.  sink(k, sigma, x) receives
// canonical output sigma + k*JS, sigma = rank*NT + tid.
template <int LOGN, int M, int CL = ntt_default_cl(LOGN), class Ld, class Sink>
__device__ __forceinline__ void ntt_inverse_core(uint64_t* sm, const LimbTab& T, Ld& ld, Sink& sink) {
    using C = NttCfg<LOGN, CL>;
    static_assert(LOGN >= 10 && LOGN <= 15, "NTT supports N in [1024, 32768]");
    const int tid = threadIdx.x;
    const int h = ntt_rank<LOGN, CL>();
    const auto K = ntt_consts<LOGN, M>(T);
    NttV<M> v[C::E];
    // own share: j = h*H + tid + k*NT
#pragma unroll
    for (int k = 0; k < C::E; k++) {
        const int jl = tid + k * C::NT;
        sm[pad(jl)] = vbits(ntt_in<M>(ld(h * C::H + jl), K));
    }
    inv_passes<LOGN, 0, M, CL>(sm, v, K, h, tid);
    // last-pass set: elements sigma + k*JS (for CL = 1, sigma = tid)
    const int sg = h * C::NT + tid;
#pragma unroll
    for (int k = 0; k < C::E; k++) {
        if constexpr (is_fp(M)) sink(k, sg, fp_out(v[k], K));
        else sink(k, sg, canon4(v[k], T.q));
    }
}

// FP64 inverse transform, lazy or reducing as for the forward one.
template <int LOGN, int CL, class Ld, class Sink>
__device__ __forceinline__ void ntt_inverse_fp(uint64_t* sm, const LimbTab& T, Ld& ld, Sink& sink) {
    if (T.fp == 2)
        ntt_inverse_core<LOGN, kModeFpLazy, CL>(sm, T, ld, sink);
    else
        ntt_inverse_core<LOGN, kModeFp, CL>(sm, T, ld, sink);
}

// Inverse transform of mode NC (integer limbs: correction-free or not), or
// FP64 for limbs with q < 2^50 whatever NC says (a uniform branch per CTA).
template <int LOGN, int NC, int CL = ntt_default_cl(LOGN), bool FPOK = true, class Ld, class St>
__device__ __forceinline__ void ntt_inverse_impl(uint64_t* sm, const LimbTab& T, Ld& ld, St& st) {
    auto sink = [&](int k, int sg, uint64_t x) { st(sg + k * NttCfg<LOGN, CL>::JS, x); };
    if (FPOK && T.fp)
        ntt_inverse_fp<LOGN, CL>(sm, T, ld, sink);
    else
        ntt_inverse_core<LOGN, NC ? kModeNC : kModeInt, CL>(sm, T, ld, sink);
}

// Inverse transform whose canonical output is parked in shared memory: each
// CTA's share at its own padded local positions (through DSMEM for CL = 2,
// complete on return; for CL = 1 a thread's outputs are the positions
// pad(tid + k*NT) it alone reads afterwards).
template <int LOGN, int NC, int CL = ntt_default_cl(LOGN), bool FPOK = true, class Ld>
__device__ __forceinline__ void ntt_inverse_to_smem(uint64_t* sm, const LimbTab& T, Ld& ld) {
    using C = NttCfg<LOGN, CL>;
    if constexpr (CL == 2) {
        const int sg0 = ntt_rank<LOGN, CL>() * C::NT + threadIdx.x;
        uint64_t* s0 = cluster_smem(sm, pair_base()) + pad(sg0);
        uint64_t* s1 = cluster_smem(sm, pair_base() + 1) + pad(sg0);
        auto sink = [&](int k, int, uint64_t x) { (k < C::E / 2 ? s0 : s1)[xoff<LOGN, CL>(k & (C::E / 2 - 1))] = x; };
        if (FPOK && T.fp)
            ntt_inverse_fp<LOGN, CL>(sm, T, ld, sink);
        else
            ntt_inverse_core<LOGN, NC ? kModeNC : kModeInt, CL>(sm, T, ld, sink);
        cluster_sync();
    } else {
        auto sink = [&](int k, int sg, uint64_t x) { sm[pad(sg + k * C::JS)] = x; };
        if (FPOK && T.fp)
            ntt_inverse_fp<LOGN, CL>(sm, T, ld, sink);
        else
            ntt_inverse_core<LOGN, NC ? kModeNC : kModeInt, CL>(sm, T, ld, sink);
    }
}

// Inverse transform: FP64 for q < 2^50 (when FPOK); otherwise integer,
// correction-free when 4q * 2^LOGN * 2 fits 64 bits.
template <int LOGN, int CL = ntt_default_cl(LOGN), bool FPOK = true, class Ld, class St>
__device__ __forceinline__ void ntt_inverse_block(uint64_t* sm, const LimbTab& T, Ld ld, St st) {
    if (!(FPOK && T.fp) && T.q < (1ULL << (61 - LOGN)))
        ntt_inverse_impl<LOGN, true, CL, FPOK>(sm, T, ld, st);
    else
        ntt_inverse_impl<LOGN, false, CL, FPOK>(sm, T, ld, st);
}

}  // namespace tsg
