// fft.cuh -- canonical-embedding FFT device code, bit-identical to the
// reference's f64 FFT (tensafe-he-core/src/encoding.rs:83-120).
//
// The reference runs a radix-2 DIT FFT: bit-reversal permutation, then
// stages s = 0 .. log2(N)-1 with twiddle (cos, sin)(-2 pi k / 2^(s+1)),
// butterfly v = w * x[i1] computed as (wr*re1 - wi*im1, wr*im1 + wi*re1).
// Every butterfly here evaluates that same expression with round-to-nearest
// intrinsics (__dmul_rn/__dadd_rn/__dsub_rn: no FMA contraction), on the
// same host-computed glibc tables, so each output rounds exactly as the
// reference's.  The order of independent butterflies within a stage does not
// change any result.
//
// Layout: a vector of N complex f64 (256 KiB at N = 16384) does not fit one
// CTA, so pass A permutes and runs the first min(log2 N, 13) stages inside
// 8192-point blocks held in shared memory (128 KiB), and pass B runs the
// remaining (log2 N - 13) stages in registers on columns
// {c, c + 8192, ...} and applies the encode or decode epilogue.
#pragma once
#include "common.cuh"

namespace tsg {

// f64 tables (host-computed with glibc, encoding.rs:38-80):
//   twist_re/twist_im[j] = cos/sin(pi j / N); stage twiddles packed as
//   tw_re/tw_im[2^s + k] = cos/sin(-2 pi k / 2^(s+1)).
struct FftTab {
    const double* twist_re;
    const double* twist_im;
    const double* tw_re;
    const double* tw_im;
};

__device__ __forceinline__ void fft_bfly(double& ur, double& ui, double& vr, double& vi, double wr, double wi) {
    const double tr = __dsub_rn(__dmul_rn(wr, vr), __dmul_rn(wi, vi));
    const double ti = __dadd_rn(__dmul_rn(wr, vi), __dmul_rn(wi, vr));
    const double ar = ur, ai = ui;
    ur = __dadd_rn(ar, tr);
    ui = __dadd_rn(ai, ti);
    vr = __dsub_rn(ar, tr);
    vi = __dsub_rn(ai, ti);
}

template <int LOGN>
struct FftGeo {
    static constexpr int N = 1 << LOGN;
    static constexpr int LB = LOGN < 13 ? LOGN : 13;  // in-smem stages
    static constexpr int BLK = 1 << LB;
    static constexpr int NB = N / BLK;                // columns' height
    static constexpr int NS = LOGN - LB;              // register stages (0..2)
};

__device__ __forceinline__ int brev_n(int p, int logn) { return (int)(__brev((unsigned)p) >> (32 - logn)); }

// Pass A for one block of one vector.  gen(i, re, im) produces input element
// i (pre-permutation index).  Output: block positions written to
// out_re/out_im (the vector's base), positions blk*BLK .. +BLK.
// Requires 2*BLK doubles of shared memory and blockDim.x == 1024.
template <int LOGN, class Gen>
__device__ __forceinline__ void fft_pass_a(double* sre, double* sim, int blk, Gen gen, double* out_re, double* out_im,
                                           const FftTab& T) {
    using G = FftGeo<LOGN>;
    const int tid = threadIdx.x;
    for (int pp = tid; pp < G::BLK; pp += blockDim.x) {
        const int p = blk * G::BLK + pp;
        double re, im;
        gen(brev_n(p, LOGN), re, im);
        sre[pp] = re;
        sim[pp] = im;
    }
    __syncthreads();
    for (int s = 0; s < G::LB; s++) {
        const int half = 1 << s;
        for (int b = tid; b < G::BLK / 2; b += blockDim.x) {
            const int k = b & (half - 1);
            const int i0 = ((b >> s) << (s + 1)) | k;
            const int i1 = i0 + half;
            const double wr = __ldg(T.tw_re + half + k), wi = __ldg(T.tw_im + half + k);
            double ur = sre[i0], ui = sim[i0], vr = sre[i1], vi = sim[i1];
            fft_bfly(ur, ui, vr, vi, wr, wi);
            sre[i0] = ur;
            sim[i0] = ui;
            sre[i1] = vr;
            sim[i1] = vi;
        }
        __syncthreads();
    }
    for (int pp = tid; pp < G::BLK; pp += blockDim.x) {
        out_re[blk * G::BLK + pp] = sre[pp];
        out_im[blk * G::BLK + pp] = sim[pp];
    }
}

// Pass B register stages on one column c (elements c + b*BLK, b < NB).
template <int LOGN>
__device__ __forceinline__ void fft_pass_b_col(double* re, double* im, int c, const FftTab& T) {
    using G = FftGeo<LOGN>;
#pragma unroll
    for (int s = G::LB; s < LOGN; s++) {
        const int hb = 1 << (s - G::LB);  // half-length in column units
#pragma unroll
        for (int b = 0; b < G::NB; b++) {
            if (b & hb) continue;
            const int k = c + (b & (hb - 1)) * G::BLK;  // i0 mod 2^s
            const int half = 1 << s;
            const double wr = __ldg(T.tw_re + half + k), wi = __ldg(T.tw_im + half + k);
            fft_bfly(re[b], im[b], re[b + hb], im[b + hb], wr, wi);
        }
    }
}

}  // namespace tsg
