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
// one CTA's shared memory; N/E threads each own E = 16 (N <= 8192) or 32
// (N = 16384) values in registers and run radix-16 passes (4 butterfly stages per pass) with one shared-memory
// exchange between passes.  The shared-memory address of element j is
// swizzled so that every pass's access pattern is bank-conflict free.
// Butterflies use Harvey's lazy reduction (values kept in [0, 4q) forward,
// [0, 2q) inverse) with Shoup twiddle products; N^-1 is folded into the last
// inverse stage.  The first pass reads through a caller functor (global
// memory, or shared memory a sampler filled) and the last pass writes through
// a caller functor, so fused kernels can transform on load and combine on
// store without extra passes over HBM.
#pragma once
#include "common.cuh"

namespace tsg {

// Per-limb device constants (one entry per RNS limb, in global memory).
struct LimbTab {
    const uint64_t* tw;  // [4][n]: fw, fw', iw, iw'  (x' = Shoup companion)
    uint64_t q;
    uint64_t ninv, ninvs;  // N^-1 mod q and companion
    uint64_t iw1n, iw1ns;  // iw[1] * N^-1 mod q and companion
    uint64_t mu64;         // floor((2^64 - 1) / q)
    uint64_t bmu;          // Barrett floor(2^(2k) / q)
    uint64_t thresh;       // 2^64 mod q: range_u64 rejection threshold (rng.rs:126)
    int bk;                // bitlen(q)
    int pad;
};

__device__ __forceinline__ int swz(int j) { return j ^ ((((j >> 6) & 3) << 2) | ((j >> 4) & 3)); }

// Geometry of a radix-2^R pass whose smallest butterfly span is TL = 2^TLOG:
// set sigma = (g, o), g = sigma >> TLOG, o = sigma & (TL-1); its k-th element
// is j = (g << (TLOG + R)) + o + (k << TLOG).  Thread tid owns sets
// sigma = tid + NT*u, u < SETS.
// Values per thread: 16 up to N = 8192, 32 at N = 16384 (512 threads with
// up to 128 registers each).
template <int LOGN>
struct NttCfg {
    static constexpr int N = 1 << LOGN;
    static constexpr int E = LOGN >= 14 ? 32 : 16;
    static constexpr int NT = N / E;
};

template <int LOGN, int R, int TLOG>
struct Geo {
    static constexpr int N = 1 << LOGN;
    static constexpr int NT = NttCfg<LOGN>::NT;
    static constexpr int SETS = NttCfg<LOGN>::E >> R;
    __device__ __forceinline__ static int sigma(int tid, int u) { return tid + NT * u; }
    __device__ __forceinline__ static int elem(int sg, int k) {
        return ((sg >> TLOG) << (TLOG + R)) + (sg & ((1 << TLOG) - 1)) + (k << TLOG);
    }
};

template <int LOGN, int R, int TLOG>
__device__ __forceinline__ void smem_load(const uint64_t* sm, uint64_t* v, int tid) {
    using G = Geo<LOGN, R, TLOG>;
#pragma unroll
    for (int u = 0; u < G::SETS; u++)
#pragma unroll
        for (int k = 0; k < (1 << R); k++) v[u * (1 << R) + k] = sm[swz(G::elem(G::sigma(tid, u), k))];
}

template <int LOGN, int R, int TLOG>
__device__ __forceinline__ void smem_store(uint64_t* sm, const uint64_t* v, int tid) {
    using G = Geo<LOGN, R, TLOG>;
#pragma unroll
    for (int u = 0; u < G::SETS; u++)
#pragma unroll
        for (int k = 0; k < (1 << R); k++) sm[swz(G::elem(G::sigma(tid, u), k))] = v[u * (1 << R) + k];
}

// One forward CT stage (sub-stage r of a radix-2^R pass starting at stage
// S0) on the 2^R values x of set-group g.  Template recursion keeps every
// loop bound a compile-time constant so x stays in registers.
template <int R, int S0, int r>
__device__ __forceinline__ void fwd_stage(uint64_t* x, int g, const uint64_t* __restrict__ fw,
                                          const uint64_t* __restrict__ fws, uint64_t q, uint64_t q2) {
    constexpr int half = 1 << (R - 1 - r);
#pragma unroll
    for (int gi = 0; gi < (1 << r); gi++) {
        const int ti = (1 << (S0 + r)) + (g << r) + gi;
        const uint64_t w = __ldg(fw + ti), wp = __ldg(fws + ti);
#pragma unroll
        for (int kk = 0; kk < half; kk++) {
            const int k = gi * 2 * half + kk;
            uint64_t X = x[k];
            X = X >= q2 ? X - q2 : X;
            const uint64_t T = mul_shoup_lazy(x[k + half], w, wp, q);
            x[k] = X + T;
            x[k + half] = X - T + q2;
        }
    }
    if constexpr (r + 1 < R) fwd_stage<R, S0, r + 1>(x, g, fw, fws, q, q2);
}

// Forward CT butterflies for stages S0 .. S0+R-1 on the thread's sets.
template <int LOGN, int R, int S0>
__device__ __forceinline__ void fwd_compute(uint64_t* v, const uint64_t* __restrict__ fw,
                                            const uint64_t* __restrict__ fws, uint64_t q, int tid) {
    constexpr int TLOG = LOGN - S0 - R;
    using G = Geo<LOGN, R, TLOG>;
#pragma unroll
    for (int u = 0; u < G::SETS; u++)
        fwd_stage<R, S0, 0>(v + u * (1 << R), G::sigma(tid, u) >> TLOG, fw, fws, q, 2 * q);
}

// One inverse GS stage (span 2^(TLOG+r)); the stage of span N/2 folds N^-1.
template <int LOGN, int R, int TLOG, int r>
__device__ __forceinline__ void inv_stage(uint64_t* x, int g, const uint64_t* __restrict__ iw,
                                          const uint64_t* __restrict__ iws, const LimbTab& T, uint64_t q2) {
    constexpr int span = 1 << r;
    constexpr int m = 1 << (LOGN - TLOG - r - 1);
    constexpr bool last = (TLOG + r == LOGN - 1);
    const uint64_t q = T.q;
#pragma unroll
    for (int gi = 0; gi < ((1 << R) >> (r + 1)); gi++) {
        uint64_t w, wp;
        if constexpr (last) {
            w = T.iw1n;
            wp = T.iw1ns;
        } else {
            const int ti = m + (g << (R - r - 1)) + gi;
            w = __ldg(iw + ti);
            wp = __ldg(iws + ti);
        }
#pragma unroll
        for (int kk = 0; kk < span; kk++) {
            const int k = gi * 2 * span + kk;
            const uint64_t X = x[k], Y = x[k + span];
            if constexpr (last) {
                x[k] = mul_shoup_lazy(X + Y, T.ninv, T.ninvs, q);
            } else {
                const uint64_t s = X + Y;
                x[k] = s >= q2 ? s - q2 : s;
            }
            x[k + span] = mul_shoup_lazy(X - Y + q2, w, wp, q);
        }
    }
    if constexpr (r + 1 < R) inv_stage<LOGN, R, TLOG, r + 1>(x, g, iw, iws, T, q2);
}

// Inverse GS butterflies for spans TL .. TL*2^(R-1) (TL = 2^TLOG).
template <int LOGN, int R, int TLOG>
__device__ __forceinline__ void inv_compute(uint64_t* v, const uint64_t* __restrict__ iw,
                                            const uint64_t* __restrict__ iws, const LimbTab& T, int tid) {
    using G = Geo<LOGN, R, TLOG>;
#pragma unroll
    for (int u = 0; u < G::SETS; u++)
        inv_stage<LOGN, R, TLOG, 0>(v + u * (1 << R), G::sigma(tid, u) >> TLOG, iw, iws, T, 2 * T.q);
}

__device__ __forceinline__ uint64_t canon4(uint64_t x, uint64_t q) {
    const uint64_t q2 = 2 * q;
    x = x >= q2 ? x - q2 : x;
    return x >= q ? x - q : x;
}

// Forward transform of one poly-limb.  ld(j) returns canonical element j
// (any source); st(j, v) receives canonical output element j.  `sm` must
// hold N u64.  All NttCfg<LOGN>::NT threads of the block must call this.
template <int LOGN, class Ld, class St>
__device__ __forceinline__ void ntt_forward_block(uint64_t* sm, const LimbTab& T, Ld ld, St st) {
    constexpr int N = 1 << LOGN, NT = NttCfg<LOGN>::NT, E = NttCfg<LOGN>::E;
    static_assert(LOGN >= 10 && LOGN <= 14, "single-CTA NTT supports N in [1024, 16384]");
    const int tid = threadIdx.x;
    const uint64_t* fw = T.tw;
    const uint64_t* fws = T.tw + N;
    uint64_t v[E];
#pragma unroll
    for (int u = 0; u < E / 16; u++)
#pragma unroll
        for (int k = 0; k < 16; k++) v[u * 16 + k] = ld(tid + NT * u + k * (N / 16));
    fwd_compute<LOGN, 4, 0>(v, fw, fws, T.q, tid);
    smem_store<LOGN, 4, LOGN - 4>(sm, v, tid);
    __syncthreads();
    // pass 2: stages 4..7
    smem_load<LOGN, 4, LOGN - 8>(sm, v, tid);
    fwd_compute<LOGN, 4, 4>(v, fw, fws, T.q, tid);
    constexpr int R3 = (LOGN - 8) < 4 ? (LOGN - 8) : 4;  // stages 8 .. 8+R3-1
    smem_store<LOGN, 4, LOGN - 8>(sm, v, tid);
    __syncthreads();
    smem_load<LOGN, R3, LOGN - 8 - R3>(sm, v, tid);
    fwd_compute<LOGN, R3, 8>(v, fw, fws, T.q, tid);
    if constexpr (LOGN - 8 - R3 == 0) {
        using G = Geo<LOGN, R3, 0>;
#pragma unroll
        for (int u = 0; u < G::SETS; u++)
#pragma unroll
            for (int k = 0; k < (1 << R3); k++)
                st(G::elem(G::sigma(tid, u), k), canon4(v[u * (1 << R3) + k], T.q));
    } else {
        constexpr int R4 = LOGN - 12;  // 1 or 2
        smem_store<LOGN, R3, LOGN - 8 - R3>(sm, v, tid);
        __syncthreads();
        smem_load<LOGN, R4, 0>(sm, v, tid);
        fwd_compute<LOGN, R4, 12>(v, fw, fws, T.q, tid);
        using G = Geo<LOGN, R4, 0>;
#pragma unroll
        for (int u = 0; u < G::SETS; u++)
#pragma unroll
            for (int k = 0; k < (1 << R4); k++)
                st(G::elem(G::sigma(tid, u), k), canon4(v[u * (1 << R4) + k], T.q));
    }
}

// Inverse transform (including x N^-1) of one poly-limb; ld returns
// canonical inputs, st receives canonical outputs.
template <int LOGN, class Ld, class St>
__device__ __forceinline__ void ntt_inverse_block(uint64_t* sm, const LimbTab& T, Ld ld, St st) {
    constexpr int N = 1 << LOGN, NT = NttCfg<LOGN>::NT, E = NttCfg<LOGN>::E;
    static_assert(LOGN >= 10 && LOGN <= 14, "single-CTA NTT supports N in [1024, 16384]");
    const int tid = threadIdx.x;
    const uint64_t* iw = T.tw + 2 * N;
    const uint64_t* iws = T.tw + 3 * N;
    uint64_t v[E];
    constexpr int R3 = (LOGN - 8) < 4 ? (LOGN - 8) : 4;
    if constexpr (LOGN - 8 - R3 == 0) {
        // passes: (R3, span 1), (4, span 2^R3), (4, span 2^(R3+4))
        using G = Geo<LOGN, R3, 0>;
#pragma unroll
        for (int u = 0; u < G::SETS; u++)
#pragma unroll
            for (int k = 0; k < (1 << R3); k++) v[u * (1 << R3) + k] = ld(G::elem(G::sigma(tid, u), k));
        inv_compute<LOGN, R3, 0>(v, iw, iws, T, tid);
        smem_store<LOGN, R3, 0>(sm, v, tid);
    } else {
        constexpr int R4 = LOGN - 12;
        using G = Geo<LOGN, R4, 0>;
#pragma unroll
        for (int u = 0; u < G::SETS; u++)
#pragma unroll
            for (int k = 0; k < (1 << R4); k++) v[u * (1 << R4) + k] = ld(G::elem(G::sigma(tid, u), k));
        inv_compute<LOGN, R4, 0>(v, iw, iws, T, tid);
        smem_store<LOGN, R4, 0>(sm, v, tid);
        __syncthreads();
        smem_load<LOGN, R3, R4>(sm, v, tid);
        inv_compute<LOGN, R3, R4>(v, iw, iws, T, tid);
        smem_store<LOGN, R3, R4>(sm, v, tid);
    }
    __syncthreads();
    smem_load<LOGN, 4, LOGN - 8>(sm, v, tid);
    inv_compute<LOGN, 4, LOGN - 8>(v, iw, iws, T, tid);
    smem_store<LOGN, 4, LOGN - 8>(sm, v, tid);
    __syncthreads();
    smem_load<LOGN, 4, LOGN - 4>(sm, v, tid);
    inv_compute<LOGN, 4, LOGN - 4>(v, iw, iws, T, tid);
#pragma unroll
    for (int u = 0; u < E / 16; u++)
#pragma unroll
        for (int k = 0; k < 16; k++) {
            const uint64_t x = v[u * 16 + k];
            st(tid + NT * u + k * (N / 16), x >= T.q ? x - T.q : x);
        }
}

}  // namespace tsg
