// k_decrypt.cu -- decrypt, decode and the fused ZeRo-MOAI decrypt kernels (sm_100a).
#include <cooperative_groups.h>

#include "launch.cuh"

namespace cg = cooperative_groups;

namespace tsg {

// ======================================================================
// Decrypt front half: (ct x pt) then c0 + c1*s, INTT (ciphertext.rs:327-349)
// ======================================================================
template <int LOGN, int CLX = ntt_default_cl(LOGN)>
__global__ void __launch_bounds__(NttCfg<LOGN, CLX>::NT, 1)
    k_decrypt_limb(uint64_t* __restrict__ M, int nl, const uint64_t* __restrict__ cts, long long ct_stride, int ct_limbs,
                   const uint64_t* __restrict__ sk, const uint64_t* __restrict__ sks, const int* __restrict__ sk_of,
                   const uint64_t* __restrict__ pt, const uint64_t* __restrict__ pts, const int* __restrict__ pt_sel,
                   int per_ct, const LimbTab* __restrict__ tabs, int L) {
    extern __shared__ __align__(16) uint64_t sm[];
    const int limb = blockIdx.x / NttCfg<LOGN, CLX>::CL, v = blockIdx.y;
    const LimbTab T = tabs[limb];
    const int ci = v / per_ct;
    const uint64_t* c0 = cts + (size_t)ci * ct_stride + ((size_t)limb << LOGN);
    const uint64_t* c1 = cts + (size_t)ci * ct_stride + ((size_t)(ct_limbs + limb) << LOGN);
    const size_t so = ((size_t)(sk_of ? sk_of[ci] : 0) * L + limb) << LOGN;
    const uint64_t* s = sk + so;
    const uint64_t* sp = sks + so;
    const uint64_t* p = nullptr;
    const uint64_t* pp = nullptr;
    if (pt) {
        const int pv = (pt_sel ? pt_sel[ci] : 0) * per_ct + v % per_ct;
        p = pt + (((size_t)pv * L + limb) << LOGN);
        if (pts) pp = pts + (((size_t)pv * L + limb) << LOGN);
    }
    uint64_t* out = M + (((size_t)v * nl + limb) << LOGN);
    ntt_inverse_block<LOGN, CLX, kPairFp<LOGN, CLX>>(
        sm, T,
        [&](int j) {
            if (pp)  // p*(c0 + c1*s) = c0*p + (c1*p)*s: two Shoup products, in [0, 4q)
                return mul_shoup4(c0[j] + mul_shoup4(c1[j], s[j], sp[j], T.q), p[j], pp[j], T.q);
            uint64_t a0 = c0[j], a1 = c1[j];
            if (p) {
                const uint64_t pj = p[j];
                a0 = mul_barrett(a0, pj, T.q, T.bmu, T.bk);
                a1 = mul_barrett(a1, pj, T.q, T.bmu, T.bk);
            }
            return a0 + canon4(mul_shoup4(a1, s[j], sp[j], T.q), T.q);  // < 2q
        },
        [&](int j, uint64_t x) { out[j] = x; });
}

template <int LG, int CL>
cudaError_t launch_decrypt_limbs_cl(const DevCtx& c, uint64_t* M, int nl, const uint64_t* cts, long long ct_stride,
                                    int ct_limbs, const uint64_t* sk, const uint64_t* sks, const int* sk_of,
                                    const uint64_t* pt, const int* pt_sel, int per_ct, int nvec, cudaStream_t s,
                                    const uint64_t* pts, const char* scope) {
    constexpr size_t smem = (size_t)NttCfg<LG, CL>::SMEM_WORDS * 8;
    cudaError_t er = ensure_smem(k_decrypt_limb<LG, CL>, smem);
    if (er != cudaSuccess) return er;
    KScope ks(scope, s);
    return launch_cl(CL, k_decrypt_limb<LG, CL>, dim3(nl * CL, nvec), NttCfg<LG, CL>::NT, smem, s, M, nl, cts, ct_stride,
                     ct_limbs, sk, sks, sk_of, pt, pts, pt_sel, per_ct, c.tabs, c.L);
}

cudaError_t launch_decrypt_limbs(const DevCtx& c, uint64_t* M, int nl, const uint64_t* cts, long long ct_stride,
                                 int ct_limbs, const uint64_t* sk, const uint64_t* sks, const int* sk_of,
                                 const uint64_t* pt, const int* pt_sel, int per_ct, int nvec, cudaStream_t s,
                                 const uint64_t* pts, const char* scope) {
    if (nvec <= 0) return cudaSuccess;
    TSG_LOGN_SWITCH(c.logn, {
        // a batch that leaves SMs idle runs each N >= 8192 transform on a CTA
        // pair (half the latency); N = 32768 always does
        constexpr int CLP = LG >= 13 ? 2 : NttCfg<LG>::CL;
        if (CLP != NttCfg<LG>::CL && (long long)nvec * nl * CLP <= c.sms)
            return launch_decrypt_limbs_cl<LG, CLP>(c, M, nl, cts, ct_stride, ct_limbs, sk, sks, sk_of, pt, pt_sel,
                                                    per_ct, nvec, s, pts, scope);
        return launch_decrypt_limbs_cl<LG, NttCfg<LG>::CL>(c, M, nl, cts, ct_stride, ct_limbs, sk, sks, sk_of, pt,
                                                           pt_sel, per_ct, nvec, s, pts, scope);
    });
    return cudaGetLastError();
}

// ======================================================================
// Decrypt back half: CRT / centring, / scale, canonical embedding
// (ciphertext.rs:351-399, encoding.rs:219-239, :295-315)
// ======================================================================
__device__ __forceinline__ double crt_coeff(uint64_t m0, uint64_t m1, const CrtConst& K) {
    const uint64_t m0q1 = mod_u64(m0, K.q1, K.mu64_1);
    const uint64_t diff = m1 >= m0q1 ? m1 - m0q1 : K.q1 - m0q1 + m1;
    const uint64_t k = canon4(mul_shoup4(diff, K.q0inv, K.q0inv_s, K.q1), K.q1);
    // mu = m0 + k*q0 (< q0*q1 < 2^101)
    uint64_t lo = k * K.q0;
    uint64_t hi = mulhi64(k, K.q0);
    lo += m0;
    hi += (lo < m0) ? 1 : 0;
    // (the reference's "mu >= Q -> mu % Q" branch cannot trigger: mu < Q)
    const bool neg = (hi > K.H_hi) || (hi == K.H_hi && lo > K.H_lo);
    // |mu - Q| for the negative half, selected without a branch
    const uint64_t dlo = K.Q_lo - lo;
    const uint64_t dhi = K.Q_hi - hi - (K.Q_lo < lo ? 1 : 0);
    const double mag = u128_to_f64(neg ? dhi : hi, neg ? dlo : lo);
    return neg ? -mag : mag;
}

// The same CRT for the segment functionals, on the FP64 pipe (K.q1d != 0,
// i.e. q1 < 2^50).  k = (m1 - m0) q0^-1 mod q1 is formed exactly (fp_mulmod
// is an exact modular product below 2^50), and so is the centring decision:
// Q = q0 q1 is odd, so mu = m0 + k q0 > Q/2 exactly when k > (q1 - 1)/2, or
// k = (q1 - 1)/2 and m0 > q0/2.  The centred value m0 + k' q0 (k' = k, or
// k - q1) is then formed with three roundings, within 2^9 + ulp/2 of the
// exact value, where crt_coeff rounds the 128-bit value once: the
// functionals sum thousands of terms of magnitude ~2^80 in f64 anyway (an
// absolute error of 2^-71 per term after / Delta^2).
__device__ __forceinline__ double crt_coeff_fp(uint64_t m0, uint64_t m1, const CrtConst& K) {
    // exact u64 -> double for values below 2^52: the bits of 2^52 + x, minus 2^52
    const double R52 = 4503599627370496.0;
    const double h = __dsub_rn(__longlong_as_double((long long)(0x4330000000000000ULL | (m0 >> 30))), R52);
    const double l = __dsub_rn(__longlong_as_double((long long)(0x4330000000000000ULL | (m0 & 0x3fffffffULL))), R52);
    const double m1d = __dsub_rn(__longlong_as_double((long long)(0x4330000000000000ULL | m1)), R52);
    // m0 = h 2^30 + l = h (2^30 mod q1) + l (mod q1); |t| <= q1
    const double t = fp_mulmod(h, K.r30, K.r30q, K.q1d);
    const double x = __dsub_rn(__dsub_rn(m1d, t), l);  // = m1 - m0 (mod q1); |x| < 2 q1 + 2^30, exact
    double k = fp_mulmod(x, K.q0invd, K.q0invq, K.q1d);  // |k| <= q1
    k = k < 0.0 ? __dadd_rn(k, K.q1d) : k;
    k = k >= K.q1d ? __dsub_rn(k, K.q1d) : k;  // [0, q1)
    const bool neg = k > K.t_half || (k == K.t_half && m0 > K.q0_half);
    const double kc = neg ? __dsub_rn(k, K.q1d) : k;
    // m0 + kc (q0_hi + q0_lo): |kc q0_lo| < 2^48, m0 rounded once to 53 bits
    return __fma_rn(kc, K.q0_hi, __fma_rn(kc, K.q0_lo, __fma_rn(h, 1073741824.0, l)));
}

// The coefficient for the functionals: the FP64 form where the moduli allow.
template <bool FPC>
__device__ __forceinline__ double crt_seg_coeff(uint64_t m0, uint64_t m1, const CrtConst& K) {
    if constexpr (FPC) return crt_coeff_fp(m0, m1, K);
    else return crt_coeff(m0, m1, K);
}

template <int LOGN>
__global__ void __launch_bounds__(1024, 1)
    k_decode_a(const uint64_t* __restrict__ M, int nl, int crt, double scale, CrtConst K, uint64_t q0, FftTab T,
               double* scr) {
    extern __shared__ __align__(16) double smd[];
    using G = FftGeo<LOGN>;
    constexpr int N = G::N;
    const int v = blockIdx.y, blk = blockIdx.x;
    const uint64_t* m0p = M + ((size_t)v * nl << LOGN);
    const uint64_t* m1p = m0p + N;
    double* ore = scr + (size_t)v * 2 * N;
    double* oim = ore + N;
    const uint64_t half_q = q0 / 2;
    auto gen = [&](int i, double& re, double& im) {
        double sgn;
        if (crt) {
            sgn = crt_coeff(m0p[i], m1p[i], K);
        } else {
            const uint64_t x = m0p[i];
            sgn = x > half_q ? -__ull2double_rn(q0 - x) : __ull2double_rn(x);
        }
        const double coeff = __ddiv_rn(sgn, scale);
        re = __dmul_rn(coeff, __ldg(T.twist_re + i));
        im = __dmul_rn(-coeff, __ldg(T.twist_im + i));
    };
    fft_pass_a<LOGN>(smd, smd + G::BLK, blk, gen, ore, oim, T);
}

// Pass B of the decode: remaining stages; slot j < N/2 is Re(X[j]).  Either
// store every slot or reduce `seg_cols` segments of `seg_d` slots (the
// ZeRo-MOAI segment sums, inference_engine.py:1382-1386) deterministically.
template <int LOGN>
__global__ void __launch_bounds__(1024, 1)
    k_decode_b(const double* __restrict__ scr, FftTab T, double* __restrict__ out_slots, double* __restrict__ seg_out,
               int seg_d, int seg_cols) {
    extern __shared__ __align__(16) double slots[];
    using G = FftGeo<LOGN>;
    constexpr int N = G::N, S = N / 2;
    const int v = blockIdx.x;
    const double* ire = scr + (size_t)v * 2 * N;
    const double* iim = ire + N;
    for (int c0 = 4 * threadIdx.x; c0 < G::BLK; c0 += 4 * blockDim.x) {
#pragma unroll
        for (int cc = 0; cc < 4; cc++) {
            const int c = c0 + cc;
            if (G::NS == 0) {
                if (c < S) {
                    const double x = ire[c];
                    if (seg_out) slots[c] = x;
                    else out_slots[(size_t)v * S + c] = x;
                }
                continue;
            }
            double re[G::NB], im[G::NB];
#pragma unroll
            for (int b = 0; b < G::NB; b++) {
                re[b] = ire[c + b * G::BLK];
                im[b] = iim[c + b * G::BLK];
            }
            fft_pass_b_col<LOGN>(re, im, c, T);
#pragma unroll
            for (int b = 0; b < G::NB; b++) {
                const int j = c + b * G::BLK;
                if (j < S) {
                    if (seg_out) slots[j] = re[b];
                    else out_slots[(size_t)v * S + j] = re[b];
                }
            }
        }
    }
    if (!seg_out) return;
    __syncthreads();
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int sgi = wid; sgi < seg_cols; sgi += nw) {
        double acc = 0.0;
        for (int t = lane; t < seg_d; t += 32) acc += slots[sgi * seg_d + t];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) seg_out[(size_t)v * seg_cols + sgi] = acc;
    }
}

cudaError_t launch_decode(const DevCtx& c, const uint64_t* M, int nl, bool crt, double scale, int nvec,
                          double* out_slots, double* seg_out, int seg_d, int seg_cols, double* scratch, cudaStream_t s) {
    if (nvec <= 0) return cudaSuccess;
    if (crt && nl < 2) return cudaErrorInvalidValue;
    const CrtConst K = c.crt;
    cudaError_t er;
    TSG_LOGN_SWITCH(c.logn, {
        using G = FftGeo<LG>;
        const size_t smem_a = (size_t)2 * G::BLK * sizeof(double);
        er = ensure_smem(k_decode_a<LG>, smem_a);
        if (er != cudaSuccess) return er;
        {
        KScope ks("decode_a", s);
        k_decode_a<LG><<<dim3(G::NB, nvec), 1024, smem_a, s>>>(M, nl, crt ? 1 : 0, scale, K, K.q0, c.fft, scratch);
        }
        const size_t smem_b = seg_out ? (size_t)(G::N / 2) * sizeof(double) : 0;
        er = ensure_smem(k_decode_b<LG>, smem_b);
        if (er != cudaSuccess) return er;
        KScope ks("decode_b", s);
        k_decode_b<LG><<<nvec, 1024, smem_b, s>>>(scratch, c.fft, out_slots, seg_out, seg_d, seg_cols);
    });
    return cudaGetLastError();
}

// ======================================================================
// Fused decrypt + decode + segment sums for the ZeRo-MOAI delta
// (ciphertext.rs:408-429, :327-399; encoding.rs:295-315;
//  inference_engine.py:1382-1386)
// ======================================================================
// NC0 / NC1: correction-free INTT for limb 0 / limb 1 (chosen by the host
// from the moduli, so each instantiation holds only two transforms).
template <int LOGN, bool NC0, bool NC1>
__global__ void __launch_bounds__(NttCfg<LOGN>::NT, 1)
    k_dec_fused(const uint64_t* __restrict__ cts, long long ct_stride, int ct_limbs, const uint64_t* __restrict__ sk,
                const uint64_t* __restrict__ sks, const int* __restrict__ sk_of, const uint64_t* __restrict__ pt,
                const uint64_t* __restrict__ pts, const int* __restrict__ pt_sel, int per_ct, int nvec,
                const LimbTab* __restrict__ tabs, int L, CrtConst K, double inv_scale, const double* __restrict__ W,
                int cols, uint64_t* __restrict__ M0, double* __restrict__ seg_out) {
    extern __shared__ __align__(16) uint64_t sm[];
    using C = NttCfg<LOGN>;
    constexpr int N = C::N, NT = C::NT, CL = C::CL;
    const int tid = threadIdx.x;
    // persistent over transform groups (one CTA, or a cluster pair for
    // CL = 2); each group keeps one limb-0 buffer, reused for every vector,
    // so the round trip stays in L2
    const int grp = blockIdx.x / CL, ngrp = gridDim.x / CL;
    const int h = ntt_rank<LOGN>();
    uint64_t* m0v = M0 + ((size_t)grp << LOGN);
    for (int v = grp; v < nvec; v += ngrp) {
        const int ci = v / per_ct;
        const int pv = (pt_sel ? pt_sel[ci] : 0) * per_ct + v % per_ct;
        const size_t key = (size_t)(sk_of ? sk_of[ci] : 0) * L;
        const uint64_t* ctb = cts + (size_t)ci * ct_stride;
        if (tid == 0 && v + ngrp < nvec) {
            // limbs 0-1 of both components of the next vector's ciphertext
            const uint64_t* nx = cts + (size_t)((v + ngrp) / per_ct) * ct_stride;
            prefetch_l2(nx, 2u << (LOGN + 3));
            prefetch_l2(nx + ((size_t)ct_limbs << LOGN), 2u << (LOGN + 3));
        }
        // phase 1: limb 0 -> scratch (each element written and later re-read
        // by the same thread)
        {
            const LimbTab T = tabs[0];
            const uint64_t* c0 = ctb;
            const uint64_t* c1 = ctb + ((size_t)ct_limbs << LOGN);
            const uint64_t* s = sk + (key << LOGN);
            const uint64_t* sp = sks + (key << LOGN);
            const uint64_t* p = pt + ((size_t)pv * L << LOGN);
            const uint64_t* pp = pts + ((size_t)pv * L << LOGN);
            // p*(c0 + c1*s): c0 + c1*s < 5q, the product lies in [0, 4q)
            auto ld = [&](int j) {
                return mul_shoup4(c0[j] + mul_shoup4(c1[j], s[j], sp[j], T.q), p[j], pp[j], T.q);
            };
            auto st = [&](int j, uint64_t x) { m0v[j] = x; };
            ntt_inverse_impl<LOGN, NC0, NttCfg<LOGN>::CL, false>(sm, T, ld, st);
        }
        __syncthreads();
        double acc[kMaxSegCols];
#pragma unroll
        for (int c = 0; c < kMaxSegCols; c++) acc[c] = 0.0;
        // phase 2: limb 1
        {
            const LimbTab T = tabs[1];
            const uint64_t* c0 = ctb + ((size_t)1 << LOGN);
            const uint64_t* c1 = ctb + ((size_t)(ct_limbs + 1) << LOGN);
            const uint64_t* s = sk + ((key + 1) << LOGN);
            const uint64_t* sp = sks + ((key + 1) << LOGN);
            const uint64_t* p = pt + (((size_t)pv * L + 1) << LOGN);
            const uint64_t* pp = pts + (((size_t)pv * L + 1) << LOGN);
            auto ld = [&](int j) {
                return mul_shoup4(c0[j] + mul_shoup4(c1[j], s[j], sp[j], T.q), p[j], pp[j], T.q);
            };
            // the last pass parks element j in the shared memory of the CTA
            // that holds j (its own for CL = 1, either for CL = 2); for CL = 2
            // both CTAs' parks (and limb-0 writes) are complete on return
            ntt_inverse_to_smem<LOGN, NC1, NttCfg<LOGN>::CL, false>(sm, T, ld);
        }
        // CRT, / Delta^2 and the segment functionals over this CTA's share
        // j = h*H + tid + k*NT; limb-0 loads issued in groups of 8 ahead of
        // their arithmetic
        {
            constexpr int G = 8;
#pragma unroll 1
            for (int k0 = 0; k0 < C::E; k0 += G) {
                uint64_t m0r[G];
#pragma unroll
                for (int kk = 0; kk < G; kk++) m0r[kk] = m0v[h * C::H + tid + (k0 + kk) * NT];
#pragma unroll
                for (int kk = 0; kk < G; kk++) {
                    const int jl = tid + (k0 + kk) * NT;
                    const int j = h * C::H + jl;
                    const double coeff = __dmul_rn(K.q1d != 0.0 ? crt_coeff_fp(m0r[kk], sm[pad(jl)], K)
                                                                  : crt_coeff(m0r[kk], sm[pad(jl)], K),
                                                   inv_scale);
#pragma unroll
                    for (int c = 0; c < kMaxSegCols; c++)
                        if (c < cols) acc[c] = fma(coeff, __ldg(W + (size_t)c * N + j), acc[c]);
                }
            }
        }
        // deterministic reduction of acc[0 .. cols): warps, then (CL = 2)
        // the two CTAs in rank order
        __syncthreads();
        double* red = reinterpret_cast<double*>(sm);  // [NT/32][kMaxSegCols]
        const int lane = tid & 31, wid = tid >> 5;
#pragma unroll
        for (int c = 0; c < kMaxSegCols; c++) {
            double a = acc[c];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
            if (lane == 0) red[wid * kMaxSegCols + c] = a;
        }
        if constexpr (CL == 1) {
            __syncthreads();
            if (tid < cols) {
                double a = 0.0;
                for (int w = 0; w < NT / 32; w++) a += red[w * kMaxSegCols + tid];
                seg_out[(size_t)v * cols + tid] = a;
            }
            __syncthreads();
        } else {
            cluster_sync();
            if (ntt_rank<LOGN>() == 0 && tid < cols) {
                double a = 0.0;
                for (int r = 0; r < CL; r++) {
                    const double* rr = reinterpret_cast<const double*>(cluster_smem(sm, r));
                    for (int w = 0; w < NT / 32; w++) a += rr[w * kMaxSegCols + tid];
                }
                seg_out[(size_t)v * cols + tid] = a;
            }
            cluster_sync();
        }
    }
}

// The fused decrypt from N = 8192 (two CTAs per SM below N = 32768, one at
// it), split in two kernels.  With both
// limbs' INTTs in one four-CTA cluster (an FP64 pair for the 40-bit limb 1
// beside an integer pair for the 60-bit limb 0) the FP64 pair finished well
// before the integer pair and waited at the cluster barrier, holding its SM
// slots (4.34 ms against 1.52 + 2.45 ms per C1 step for the split form).
// Here each kernel's CTA pairs do one kind of transform:
//   k_dec_limb1: p*(c0 + c1*s) and the INTT of limb 1 for every vector
//     (FP64 butterflies), canonical results to M1 [nvec][N];
//   k_dec_pair: the same for limb 0 (IMAD butterflies), parked in shared
//     memory, then the CRT with M1, / Delta^2 and the segment functionals
//     over the pair's positions; rank 0 adds the two CTAs' partials in rank
//     order.
// u = c0 + c1*s (in [0, 5q)) of limb `limb` of ciphertext ci on the elements
// this thread later loads into its transforms (j = h*H + tid + k*NT), to the
// ciphertext's row of U.  The same thread reads them back for every batch,
// so the row stays in L2 and needs no barrier.
template <int LOGN>
__device__ __forceinline__ void dec_u_row(uint64_t* __restrict__ u, const uint64_t* __restrict__ c0,
                                          const uint64_t* __restrict__ c1, const uint64_t* __restrict__ s,
                                          const uint64_t* __restrict__ sp, uint64_t q) {
    using C = NttCfg<LOGN, 2>;
    const int base = ntt_rank<LOGN, 2>() * C::H + (int)threadIdx.x;
#pragma unroll 4
    for (int k = 0; k < C::E; k++) {
        const int j = base + k * C::NT;
        u[j] = c0[j] + mul_shoup4(c1[j], s[j], sp[j], q);
    }
}

// One batch of k_dec_limb1: INTT of p*u (p*u = p*(c0 + c1*s) = c0*p +
// (c1*p)*s mod q, in [0, 4q)) to out.  Kept out of line, so that the batch
// loop's state and the transform's registers are allocated apart.
template <int LOGN>
__device__ __noinline__ void dec_limb1_batch(uint64_t* sm, const LimbTab* tab, const uint64_t* __restrict__ u,
                                             const uint64_t* __restrict__ p, const uint64_t* __restrict__ pp,
                                             uint64_t* __restrict__ out) {
    const LimbTab T = *tab;
    ntt_inverse_block<LOGN, 2>(
        sm, T, [&](int j) { return mul_shoup4(u[j], p[j], pp[j], T.q); }, [&](int j, uint64_t x) { out[j] = x; });
}

// CTAs per SM of the split decrypt: two up to N = 16384, one at N = 32768
// (a pair's shares fill two SMs' shared memory).
constexpr int dec_minb(int logn) { return logn >= 15 ? 1 : 2; }

template <int LOGN>
__global__ void __launch_bounds__(NttCfg<LOGN, 2>::NT, dec_minb(LOGN))
    k_dec_limb1(uint64_t* __restrict__ M1, uint64_t* __restrict__ U, const uint64_t* __restrict__ cts,
                long long ct_stride, int ct_limbs, const uint64_t* __restrict__ sk, const uint64_t* __restrict__ sks,
                const int* __restrict__ sk_of, const uint64_t* __restrict__ pt, const uint64_t* __restrict__ pts,
                const int* __restrict__ pt_sel, int per_ct, int bpp, const LimbTab* __restrict__ tabs, int L) {
    extern __shared__ __align__(16) uint64_t sm[];
    // CTA pair g of ciphertext ci takes batches [g*bpp, g*bpp + bpp): all of
    // them when there are enough ciphertexts to fill the GPU, fewer otherwise
    const int ngrp = (per_ct + bpp - 1) / bpp;
    const int ci = (blockIdx.x >> 1) / ngrp, b0 = ((blockIdx.x >> 1) % ngrp) * bpp;
    const int b1 = b0 + bpp < per_ct ? b0 + bpp : per_ct;
    const size_t key = (size_t)(sk_of ? sk_of[ci] : 0) * L;
    // limb 0's row for k_dec_pair (this kernel's IMAD pipe is otherwise
    // idle; the first group writes it), then limb 1's, which this pair's
    // transforms read (each group writes the same values and reads back its
    // own threads' writes)
    if (b0 == 0)
        dec_u_row<LOGN>(U + ((size_t)ci * 2 << LOGN), cts + (size_t)ci * ct_stride,
                        cts + (size_t)ci * ct_stride + ((size_t)ct_limbs << LOGN), sk + (key << LOGN),
                        sks + (key << LOGN), tabs[0].q);
    uint64_t* u = U + (((size_t)ci * 2 + 1) << LOGN);
    dec_u_row<LOGN>(u, cts + (size_t)ci * ct_stride + ((size_t)1 << LOGN),
                    cts + (size_t)ci * ct_stride + ((size_t)(ct_limbs + 1) << LOGN), sk + ((key + 1) << LOGN),
                    sks + ((key + 1) << LOGN), tabs[1].q);
#pragma unroll 1
    for (int b = b0; b < b1; b++) {
        const int v = ci * per_ct + b;
        const int pv = (pt_sel ? pt_sel[ci] : 0) * per_ct + b;
        dec_limb1_batch<LOGN>(sm, tabs + 1, u, pt + (((size_t)pv * L + 1) << LOGN),
                              pts + (((size_t)pv * L + 1) << LOGN), M1 + ((size_t)v << LOGN));
        __syncthreads();
    }
}

template <int LOGN, int MAXC, bool FPC>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NttCfg<LOGN, 2>::NT, dec_minb(LOGN))
    k_dec_pair(const uint64_t* __restrict__ M1, const uint64_t* __restrict__ U, const uint64_t* __restrict__ pt,
               const uint64_t* __restrict__ pts, const int* __restrict__ pt_sel, int per_ct,
               const LimbTab* __restrict__ tabs, int L, CrtConst K, double inv_scale, const double* __restrict__ W,
               int cols, double* __restrict__ seg_out) {
    extern __shared__ __align__(16) uint64_t sm[];
    using C = NttCfg<LOGN, 2>;
    constexpr int N = C::N, NT = C::NT, H = C::H;
    __shared__ double red[NT / 32][MAXC];
    const int tid = threadIdx.x, v = blockIdx.x >> 1, h = cluster_rank();
    const int ci = v / per_ct;
    const int pv = (pt_sel ? pt_sel[ci] : 0) * per_ct + v % per_ct;
    {
        const LimbTab T = tabs[0];
        const uint64_t* u = U + ((size_t)ci * 2 << LOGN);  // c0 + c1*s of limb 0, from k_dec_limb1
        const uint64_t* p = pt + ((size_t)pv * L << LOGN);
        const uint64_t* pp = pts + ((size_t)pv * L << LOGN);
        auto ld = [&](int j) { return mul_shoup4(u[j], p[j], pp[j], T.q); };
        ntt_inverse_to_smem<LOGN, false, 2>(sm, T, ld);  // this CTA's half at its padded local positions
    }
    const uint64_t* m1 = M1 + ((size_t)v << LOGN) + (size_t)h * H;
    double acc[MAXC];
#pragma unroll
    for (int c = 0; c < MAXC; c++) acc[c] = 0.0;
#pragma unroll 2
    for (int k = 0; k < C::E; k++) {
        const int jl = tid + k * NT;
        const int j = h * H + jl;
        const double coeff = __dmul_rn(crt_seg_coeff<FPC>(sm[pad(jl)], m1[jl], K), inv_scale);
#pragma unroll
        for (int c = 0; c < MAXC; c++)
            if (c < cols) acc[c] = fma(coeff, __ldg(W + (size_t)c * N + j), acc[c]);
    }
    const int lane = tid & 31, wid = tid >> 5;
#pragma unroll
    for (int c = 0; c < MAXC; c++) {
        double a = acc[c];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        if (lane == 0) red[wid][c] = a;
    }
    cluster_sync();  // both CTAs' partials written
    if (h == 0 && tid < cols) {
        double a = 0.0;
        for (int r = 0; r < 2; r++) {
            const double* rr = cooperative_groups::this_cluster().map_shared_rank(&red[0][0], r);
            for (int w = 0; w < NT / 32; w++) a += rr[w * MAXC + tid];
        }
        seg_out[(size_t)v * cols + tid] = a;
    }
    cluster_sync();  // keep the partials alive until rank 0 has read them
}

cudaError_t launch_dec_fused(const DevCtx& c, const uint64_t* cts, long long ct_stride, int ct_limbs,
                             const uint64_t* sk, const uint64_t* sks, const int* sk_of, const uint64_t* pt,
                             const uint64_t* pts, const int* pt_sel, int per_ct,
                             int nvec, double inv_scale, const double* W, int seg_cols, uint64_t* M0, uint64_t* U,
                             double* seg_out, cudaStream_t s) {
    if (nvec <= 0) return cudaSuccess;
    if (seg_cols < 1 || seg_cols > kMaxSegCols || c.L < 2) return cudaErrorInvalidValue;
    // correction-free INTT where the modulus leaves the headroom (as in
    // ntt_inverse_block); this kernel stays integer-only (its FP64 variant
    // spilled 648 bytes and ran 15% slower)
    const bool nc0 = c.q0 < (1ULL << (61 - c.logn)), nc1 = c.q1 < (1ULL << (61 - c.logn));
    TSG_LOGN_SWITCH(c.logn, {
        // N = 8192 .. 32768: the split form on CTA pairs (LQ: other sizes
        // never take it)
        constexpr int LQ = LG >= 13 ? LG : 14;
        if (LG >= 13) {
            // split form: limb-1 INTTs to M0 (nvec x N words), then limb 0 + CRT
            constexpr size_t smemq = (size_t)NttCfg<LQ, 2>::SMEM_WORDS * 8;
            cudaError_t er = ensure_smem(k_dec_limb1<LQ>, smemq);
            if (er != cudaSuccess) return er;
            // u rows once per ciphertext where the ciphertexts alone fill two
            // waves of CTA pairs; otherwise batches spread over more pairs
            const int nct = nvec / per_ct;
            int bpp = nvec / (dec_minb(LG) * c.sms);
            bpp = bpp < 1 ? 1 : (bpp > per_ct ? per_ct : bpp);
            const unsigned pairs = (unsigned)nct * (unsigned)((per_ct + bpp - 1) / bpp);
            {
                KScope ks("dec_limb1", s);
                er = launch_cl(2, k_dec_limb1<LQ>, dim3(pairs * 2), NttCfg<LQ, 2>::NT, smemq, s, M0, U, cts, ct_stride,
                               ct_limbs, sk, sks, sk_of, pt, pts, pt_sel, per_ct, bpp, c.tabs, c.L);
                if (er != cudaSuccess) return er;
            }
            // accumulators for at most 5 segment columns where that suffices
            const bool fpc = c.crt.q1d != 0.0;
            auto kp = seg_cols <= 5 ? (fpc ? k_dec_pair<LQ, 5, true> : k_dec_pair<LQ, 5, false>)
                                    : (fpc ? k_dec_pair<LQ, kMaxSegCols, true> : k_dec_pair<LQ, kMaxSegCols, false>);
            er = ensure_smem(kp, smemq);
            if (er != cudaSuccess) return er;
            KScope ks("dec_fused", s);
            kp<<<dim3((unsigned)nvec * 2), NttCfg<LQ, 2>::NT, smemq, s>>>(M0, U, pt, pts, pt_sel, per_ct, c.tabs,
                                                                         c.L, c.crt, inv_scale, W, seg_cols, seg_out);
            return cudaGetLastError();
        }
        constexpr size_t smem = ntt_smem_bytes<LG>();
        constexpr int CL = NttCfg<LG>::CL;
        // one CTA per SM (the padded share fills most of shared memory); M0
        // holds one limb per group (CTA, or cluster pair)
        const int groups = nvec < c.sms / CL ? nvec : c.sms / CL;
        auto kern = nc0 ? (nc1 ? k_dec_fused<LG, true, true> : k_dec_fused<LG, true, false>)
                        : (nc1 ? k_dec_fused<LG, false, true> : k_dec_fused<LG, false, false>);
        cudaError_t er = ensure_smem(kern, smem);
        if (er != cudaSuccess) return er;
        KScope ks("dec_fused", s);
        return launch_cl(CL, kern, dim3(groups * CL), NttCfg<LG>::NT, smem, s, cts, ct_stride, ct_limbs, sk, sks,
                         sk_of, pt, pts, pt_sel, per_ct, nvec, c.tabs, c.L, c.crt, inv_scale, W, seg_cols, M0, seg_out);
    });
    return cudaGetLastError();
}

// CRT of limbs 0/1, / scale and the segment functionals, for decrypts whose
// INTT ran separately (N = 32768, and small batches at any N).  One cluster
// of kCrtCl CTAs per vector v of M [nvec][2][n]: each CTA takes an n/kCrtCl
// slice, reduces it in shared memory, and cluster rank 0 adds the kCrtCl
// partials in rank order through distributed shared memory, so the sum order
// is fixed.  A small batch (the decode step's 7 vectors) thus spreads over
// 8x the SMs instead of running one block per vector.
constexpr int kCrtCl = 8;

template <bool FPC>
__global__ void __launch_bounds__(256)
    k_crt_seg(const uint64_t* __restrict__ M, int logn, CrtConst K, double inv_scale, const double* __restrict__ W,
              int cols, double* __restrict__ seg_out) {
    const int n = 1 << logn, tid = threadIdx.x;
    const int v = blockIdx.x / kCrtCl, rank = blockIdx.x % kCrtCl;
    const int slice = n / kCrtCl, j0 = rank * slice;
    const uint64_t* m0 = M + ((size_t)v * 2 << logn);
    const uint64_t* m1 = m0 + n;
    double acc[kMaxSegCols];
#pragma unroll
    for (int c = 0; c < kMaxSegCols; c++) acc[c] = 0.0;
    for (int j = j0 + tid; j < j0 + slice; j += blockDim.x) {
        const double coeff = __dmul_rn(crt_seg_coeff<FPC>(m0[j], m1[j], K), inv_scale);
#pragma unroll
        for (int c = 0; c < kMaxSegCols; c++)
            if (c < cols) acc[c] = fma(coeff, __ldg(W + (size_t)c * n + j), acc[c]);
    }
    __shared__ double red[8][kMaxSegCols];
    __shared__ double part[kMaxSegCols];
    const int lane = tid & 31, wid = tid >> 5;
#pragma unroll
    for (int c = 0; c < kMaxSegCols; c++) {
        double a = acc[c];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        if (lane == 0) red[wid][c] = a;
    }
    __syncthreads();
    if (tid < cols) {
        double a = 0.0;
        for (int w = 0; w < 8; w++) a += red[w][tid];
        part[tid] = a;
    }
    cg::cluster_group cl = cg::this_cluster();
    cl.sync();  // every slice's partial is in its CTA's shared memory
    if (rank == 0 && tid < cols) {
        double a = 0.0;
        for (int r = 0; r < kCrtCl; r++) a += cl.map_shared_rank(part, r)[tid];
        seg_out[(size_t)v * cols + tid] = a;
    }
    cl.sync();  // the other CTAs keep their shared memory until rank 0 has read it
}

cudaError_t launch_crt_seg(const DevCtx& c, const uint64_t* M, int nvec, double inv_scale, const double* W,
                           int seg_cols, double* seg_out, cudaStream_t s, const char* scope) {
    if (nvec <= 0) return cudaSuccess;
    if (seg_cols < 1 || seg_cols > kMaxSegCols || c.L < 2 || (c.n % kCrtCl) != 0) return cudaErrorInvalidValue;
    KScope ks(scope, s);
    return launch_cl(kCrtCl, c.crt.q1d != 0.0 ? k_crt_seg<true> : k_crt_seg<false>, dim3((unsigned)(nvec * kCrtCl)),
                     256, 0, s, M, c.logn, c.crt, inv_scale, W, seg_cols, seg_out);
}


}  // namespace tsg
