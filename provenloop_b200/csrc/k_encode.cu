// k_encode.cu -- CKKS encode (canonical-embedding inverse) kernels (sm_100a).
#include <cooperative_groups.h>

#include "launch.cuh"

namespace cg = cooperative_groups;

namespace tsg {

// ======================================================================
// Encode (encoding.rs:173-207 + :250-278) and the encryption's Gaussian
// ======================================================================
__device__ __forceinline__ double slot_value(const SlotSrc& s, int v, int k) {
    long long idx;
    if (s.rep_cols > 0) {
        if (k >= s.rep_cols * s.rep_d) return 0.0;
        idx = (long long)v * s.stride + (k % s.rep_d);
    } else {
        if (k >= s.len) return 0.0;
        idx = (long long)v * s.stride + k;
    }
    return s.is_f32 ? (double)__ldg(static_cast<const float*>(s.src) + idx)
                    : __ldg(static_cast<const double*>(s.src) + idx);
}

template <int LOGN>
__global__ void __launch_bounds__(1024, 1) k_encode_a(SlotSrc src, FftTab T, double* scr) {
    extern __shared__ __align__(16) double smd[];
    using G = FftGeo<LOGN>;
    const int v = blockIdx.y, blk = blockIdx.x;
    constexpr int N = G::N, S = N / 2;
    double* ore = scr + (size_t)v * 2 * N;
    double* oim = ore + N;
    // conjugate-symmetric real input: re[k] = re[N-1-k] = z[k], im = 0
    auto gen = [&](int i, double& re, double& im) {
        const int k = i < S ? i : N - 1 - i;
        re = slot_value(src, v, k);
        im = 0.0;
    };
    fft_pass_a<LOGN>(smd, smd + G::BLK, blk, gen, ore, oim, T);
}

// Pass B of the encode: final FFT stages, x 1/N, untwist, x Delta, round;
// optionally the Gaussian error of the same encryption (rng.rs:152-157,
// sampling.rs:51-58) from words gauss_off + 4j of the vector's stream.
template <int LOGN>
__global__ void __launch_bounds__(1024, 1)
    k_encode_b(const double* __restrict__ scr, FftTab T, int64_t* __restrict__ m, int8_t* __restrict__ e,
               const uint64_t* __restrict__ seeds, uint64_t gauss_off, unsigned long long* stats) {
    using G = FftGeo<LOGN>;
    constexpr int N = G::N;
    const int v = blockIdx.x;
    const double* ire = scr + (size_t)v * 2 * N;
    const double* iim = ire + N;
    const double inv_n = 1.0 / (double)N;
    const double scale = 1099511627776.0;  // SCALE = 2^40
    const uint64_t seed = e ? seeds[v] : 0;
    int ties = 0;
    for (int c0 = 4 * threadIdx.x; c0 < G::BLK; c0 += 4 * blockDim.x) {
        double re[4][G::NB], im[4][G::NB];
#pragma unroll
        for (int cc = 0; cc < 4; cc++) {
#pragma unroll
            for (int b = 0; b < G::NB; b++) {
                re[cc][b] = ire[c0 + cc + b * G::BLK];
                im[cc][b] = iim[c0 + cc + b * G::BLK];
            }
            fft_pass_b_col<LOGN>(re[cc], im[cc], c0 + cc, T);
        }
#pragma unroll
        for (int b = 0; b < G::NB; b++) {
            const int j0 = c0 + b * G::BLK;
            uint32_t w[16];
            if (e) chacha_block(seed, (uint32_t)((gauss_off + 4ULL * j0) >> 4), w);
#pragma unroll
            for (int cc = 0; cc < 4; cc++) {
                const int j = j0 + cc;
                const double a_re = __dmul_rn(re[cc][b], inv_n);
                const double a_im = __dmul_rn(im[cc][b], inv_n);
                const double coeff =
                    __dadd_rn(__dmul_rn(a_re, __ldg(T.twist_re + j)), __dmul_rn(a_im, __ldg(T.twist_im + j)));
                m[(size_t)v * N + j] = f64_to_i64_sat(round(__dmul_rn(coeff, scale)));
                if (e) {
                    bool tie;
                    const uint64_t u1 = (uint64_t)w[4 * cc] | ((uint64_t)w[4 * cc + 1] << 32);
                    const uint64_t u2 = (uint64_t)w[4 * cc + 2] | ((uint64_t)w[4 * cc + 3] << 32);
                    e[(size_t)v * N + j] = (int8_t)gaussian_round_e(u1, u2, &tie);
                    ties += tie ? 1 : 0;
                }
            }
        }
    }
    if (ties && stats) atomicAdd(stats + STAT_NEAR_TIE, (unsigned long long)ties);
}

// ----------------------------------------------------------------------
// Single-kernel encode at N = 16384: a cluster of two CTAs per vector, each
// holding one 8192-point half of the FFT in padded shared memory.  Stages
// 0-11 run as radix-16 register passes (16 complex values per thread, one
// shared-memory exchange per pass); stages 12 and 13 combine the halves
// through distributed shared memory, and the encode epilogue (1/N, untwist,
// x Delta, round) and the encryption's Gaussian error follow in the same
// kernel.  Every butterfly is fft_bfly on the same twiddles as the reference
// (encoding.rs:83-120), so m is bit-identical to the two-pass kernels.
// ----------------------------------------------------------------------
namespace enc1 {
constexpr int LOGN = 14, N = 1 << LOGN, S = N / 2, HALF = N / 2;  // HALF points per CTA
constexpr int NT = 512, E = 16, R = 4;                           // radix-16 passes
constexpr int SM_WORDS = HALF + HALF / 16;                       // padded half (doubles)
constexpr size_t SMEM = (size_t)2 * SM_WORDS * sizeof(double);  // re and im

// One radix-2^R pass over stages TLOG .. TLOG+R-1 on the 16-point set with
// local base j0 (positions j0 + k*2^TLOG); all twiddle indexes are local to
// the half because every stage here has 2^s <= 2^11 < HALF.
template <int TLOG, int rr>
__device__ __forceinline__ void pass_stage(double* re, double* im, int j0, const FftTab& T) {
    constexpr int span = 1 << rr;
    constexpr int half = 1 << (TLOG + rr);
#pragma unroll
    for (int k = 0; k < E; k++) {
        if (k & span) continue;
        const int ktw = (j0 + k * (1 << TLOG)) & (half - 1);
        const double wr = __ldg(T.tw_re + half + ktw), wi = __ldg(T.tw_im + half + ktw);
        fft_bfly(re[k], im[k], re[k + span], im[k + span], wr, wi);
    }
    if constexpr (rr + 1 < R) pass_stage<TLOG, rr + 1>(re, im, j0, T);
}

template <int TLOG>
__device__ __forceinline__ int set_base(int sigma) {
    return ((sigma >> TLOG) << (TLOG + R)) + (sigma & ((1 << TLOG) - 1));
}

// Stages TL .. TL+3 on this thread's set of stride 2^TL, through the CTA's
// padded shared memory (the previous pass's stores complete first).
template <int TL>
__device__ __forceinline__ void smem_pass(double* re, double* im, double* sre, double* sim, int tid,
                                          const FftTab& T) {
    __syncthreads();
    const int j0 = set_base<TL>(tid);
#pragma unroll
    for (int k = 0; k < E; k++) {
        re[k] = sre[pad(j0 + k * (1 << TL))];
        im[k] = sim[pad(j0 + k * (1 << TL))];
    }
    pass_stage<TL, 0>(re, im, j0, T);
#pragma unroll
    for (int k = 0; k < E; k++) {
        sre[pad(j0 + k * (1 << TL))] = re[k];
        sim[pad(j0 + k * (1 << TL))] = im[k];
    }
}
}  // namespace enc1

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(enc1::NT, 1)
    k_encode_n16k(SlotSrc src, FftTab T, int64_t* __restrict__ m, int8_t* __restrict__ e,
                  const uint64_t* __restrict__ seeds, uint64_t gauss_off, unsigned long long* stats) {
    using namespace enc1;
    extern __shared__ __align__(16) double smd[];
    double* sre = smd;
    double* sim = smd + SM_WORDS;
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();  // which half of the positions
    const int v = blockIdx.x >> 1, tid = threadIdx.x;
    double re[E], im[E];
    // pass 0: stages 0-3 on 16 consecutive positions, loaded in bit-reversed
    // order from the conjugate-symmetric input (re[k] = re[N-1-k] = z[k])
    {
        const int j0 = tid * E;
#pragma unroll
        for (int k = 0; k < E; k++) {
            const int i = brev_n(rank * HALF + j0 + k, LOGN);
            re[k] = slot_value(src, v, i < S ? i : N - 1 - i);
            im[k] = 0.0;
        }
        pass_stage<0, 0>(re, im, j0, T);
#pragma unroll
        for (int k = 0; k < E; k++) {
            sre[pad(j0 + k)] = re[k];
            sim[pad(j0 + k)] = im[k];
        }
    }
    // passes 1 and 2: stages 4-7 and 8-11 (sets of stride 16 and 256)
    smem_pass<4>(re, im, sre, sim, tid, T);
    smem_pass<8>(re, im, sre, sim, tid, T);
    // both halves complete before either reads the other's
    cluster.sync();
    // stages 12 and 13: positions p, p+4096 (half 0) and p+8192, p+12288
    // (half 1); this CTA takes p in [rank*2048, rank*2048 + 2048)
    const double* re0 = cluster.map_shared_rank(sre, 0);
    const double* im0 = cluster.map_shared_rank(sim, 0);
    const double* re1 = cluster.map_shared_rank(sre, 1);
    const double* im1 = cluster.map_shared_rank(sim, 1);
    const double inv_n = 1.0 / (double)N;
    const double scale = 1099511627776.0;  // SCALE = 2^40
    int64_t* mv = m + (size_t)v * N;
    for (int p = rank * 2048 + tid; p < rank * 2048 + 2048; p += NT) {
        double ar = re0[pad(p)], ai = im0[pad(p)];
        double br = re0[pad(p + 4096)], bi = im0[pad(p + 4096)];
        double cr = re1[pad(p)], ci = im1[pad(p)];
        double dr = re1[pad(p + 4096)], di = im1[pad(p + 4096)];
        {
            const double wr = __ldg(T.tw_re + 4096 + p), wi = __ldg(T.tw_im + 4096 + p);
            fft_bfly(ar, ai, br, bi, wr, wi);  // stage 12: (p, p+4096)
            fft_bfly(cr, ci, dr, di, wr, wi);  // stage 12: (p+8192, p+12288)
        }
        {
            const double wr = __ldg(T.tw_re + 8192 + p), wi = __ldg(T.tw_im + 8192 + p);
            fft_bfly(ar, ai, cr, ci, wr, wi);  // stage 13: (p, p+8192)
        }
        {
            const double wr = __ldg(T.tw_re + 8192 + p + 4096), wi = __ldg(T.tw_im + 8192 + p + 4096);
            fft_bfly(br, bi, dr, di, wr, wi);  // stage 13: (p+4096, p+12288)
        }
        // encode epilogue (encoding.rs:250-278)
        const double xr[4] = {ar, br, cr, dr}, xi[4] = {ai, bi, ci, di};
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int j = p + q * 4096;
            const double a_re = __dmul_rn(xr[q], inv_n);
            const double a_im = __dmul_rn(xi[q], inv_n);
            const double coeff =
                __dadd_rn(__dmul_rn(a_re, __ldg(T.twist_re + j)), __dmul_rn(a_im, __ldg(T.twist_im + j)));
            mv[j] = f64_to_i64_sat(round(__dmul_rn(coeff, scale)));
        }
    }
    // the encryption's Gaussian error (rng.rs:152-157, sampling.rs:51-58):
    // sample j from words gauss_off + 4j, four samples per ChaCha block
    if (e) {
        const uint64_t seed = seeds[v];
        int ties = 0;
        for (int b = rank * (HALF / 4) + tid; b < (rank + 1) * (HALF / 4); b += NT) {
            uint32_t w[16];
            chacha_block(seed, (uint32_t)((gauss_off >> 4) + (uint64_t)b), w);
            char4 o;
            bool tie;
            o.x = (signed char)gaussian_round_e((uint64_t)w[0] | ((uint64_t)w[1] << 32),
                                              (uint64_t)w[2] | ((uint64_t)w[3] << 32), &tie);
            ties += tie;
            o.y = (signed char)gaussian_round_e((uint64_t)w[4] | ((uint64_t)w[5] << 32),
                                              (uint64_t)w[6] | ((uint64_t)w[7] << 32), &tie);
            ties += tie;
            o.z = (signed char)gaussian_round_e((uint64_t)w[8] | ((uint64_t)w[9] << 32),
                                              (uint64_t)w[10] | ((uint64_t)w[11] << 32), &tie);
            ties += tie;
            o.w = (signed char)gaussian_round_e((uint64_t)w[12] | ((uint64_t)w[13] << 32),
                                              (uint64_t)w[14] | ((uint64_t)w[15] << 32), &tie);
            ties += tie;
            reinterpret_cast<char4*>(e + (size_t)v * N)[b] = o;
        }
        if (ties && stats) atomicAdd(stats + STAT_NEAR_TIE, (unsigned long long)ties);
    }
    // keep this CTA's shared memory alive until the partner has read it
    cluster.sync();
}

// ----------------------------------------------------------------------
// Single-kernel encode at N = 32768: a cluster of four CTAs per vector, each
// holding one 8192-point quarter (CTA r: positions r*8192 .. r*8192 + 8191)
// in padded shared memory.  Stages 0-11 are local to a quarter and run as in
// k_encode_n16k; stages 12-14 combine the quarters through distributed
// shared memory, eight points per column (positions p and p + 4096 of every
// quarter), followed by the encode epilogue.  The butterflies and twiddles
// are those of the stage-by-stage FFT (encoding.rs:83-120), so m is
// bit-identical to the two-pass kernels'.
// ----------------------------------------------------------------------
__global__ void __cluster_dims__(4, 1, 1) __launch_bounds__(enc1::NT, 1)
    k_encode_n32k(SlotSrc src, FftTab T, int64_t* __restrict__ m, int8_t* __restrict__ e,
                  const uint64_t* __restrict__ seeds, uint64_t gauss_off, unsigned long long* stats) {
    using namespace enc1;
    constexpr int LG = 15, NN = 1 << LG, SS = NN / 2, Q = HALF;  // Q = 8192 points per CTA
    extern __shared__ __align__(16) double smd[];
    double* sre = smd;
    double* sim = smd + SM_WORDS;
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();  // which quarter of the positions
    const int v = blockIdx.x >> 2, tid = threadIdx.x;
    double re[E], im[E];
    {
        const int j0 = tid * E;
#pragma unroll
        for (int k = 0; k < E; k++) {
            const int i = brev_n(rank * Q + j0 + k, LG);
            re[k] = slot_value(src, v, i < SS ? i : NN - 1 - i);
            im[k] = 0.0;
        }
        pass_stage<0, 0>(re, im, j0, T);
#pragma unroll
        for (int k = 0; k < E; k++) {
            sre[pad(j0 + k)] = re[k];
            sim[pad(j0 + k)] = im[k];
        }
    }
    smem_pass<4>(re, im, sre, sim, tid, T);
    smem_pass<8>(re, im, sre, sim, tid, T);
    cluster.sync();  // all four quarters complete before any CTA reads another's
    const double* qre[4];
    const double* qim[4];
#pragma unroll
    for (int r = 0; r < 4; r++) {
        qre[r] = cluster.map_shared_rank(sre, r);
        qim[r] = cluster.map_shared_rank(sim, r);
    }
    const double inv_n = 1.0 / (double)NN;
    const double scale = 1099511627776.0;  // SCALE = 2^40
    int64_t* mv = m + (size_t)v * NN;
    // column p (this CTA: p in [rank*1024, rank*1024 + 1024)): x[r][o] is
    // position r*Q + p + o*4096
    for (int p = rank * 1024 + tid; p < rank * 1024 + 1024; p += NT) {
        double xr[4][2], xi[4][2];
#pragma unroll
        for (int r = 0; r < 4; r++)
#pragma unroll
            for (int o = 0; o < 2; o++) {
                xr[r][o] = qre[r][pad(p + o * 4096)];
                xi[r][o] = qim[r][pad(p + o * 4096)];
            }
        {  // stage 12: (p, p + 4096) within each quarter
            const double wr = __ldg(T.tw_re + 4096 + p), wi = __ldg(T.tw_im + 4096 + p);
#pragma unroll
            for (int r = 0; r < 4; r++) fft_bfly(xr[r][0], xi[r][0], xr[r][1], xi[r][1], wr, wi);
        }
#pragma unroll
        for (int o = 0; o < 2; o++) {  // stage 13: quarters (0, 1) and (2, 3)
            const double wr = __ldg(T.tw_re + 8192 + p + o * 4096), wi = __ldg(T.tw_im + 8192 + p + o * 4096);
            fft_bfly(xr[0][o], xi[0][o], xr[1][o], xi[1][o], wr, wi);
            fft_bfly(xr[2][o], xi[2][o], xr[3][o], xi[3][o], wr, wi);
        }
#pragma unroll
        for (int o = 0; o < 2; o++) {  // stage 14: quarters (0, 2) and (1, 3)
            const int j = p + o * 4096;
            fft_bfly(xr[0][o], xi[0][o], xr[2][o], xi[2][o], __ldg(T.tw_re + 16384 + j), __ldg(T.tw_im + 16384 + j));
            fft_bfly(xr[1][o], xi[1][o], xr[3][o], xi[3][o], __ldg(T.tw_re + 16384 + 8192 + j),
                     __ldg(T.tw_im + 16384 + 8192 + j));
        }
        // encode epilogue (encoding.rs:250-278)
#pragma unroll
        for (int r = 0; r < 4; r++)
#pragma unroll
            for (int o = 0; o < 2; o++) {
                const int j = r * Q + p + o * 4096;
                const double a_re = __dmul_rn(xr[r][o], inv_n);
                const double a_im = __dmul_rn(xi[r][o], inv_n);
                const double coeff =
                    __dadd_rn(__dmul_rn(a_re, __ldg(T.twist_re + j)), __dmul_rn(a_im, __ldg(T.twist_im + j)));
                mv[j] = f64_to_i64_sat(round(__dmul_rn(coeff, scale)));
            }
    }
    // the encryption's Gaussian error, as in k_encode_n16k (this CTA: a
    // quarter of the samples, four per ChaCha20 block)
    if (e) {
        const uint64_t seed = seeds[v];
        int ties = 0;
        for (int b = rank * (Q / 4) + tid; b < (rank + 1) * (Q / 4); b += NT) {
            uint32_t w[16];
            chacha_block(seed, (uint32_t)((gauss_off >> 4) + (uint64_t)b), w);
            char4 o;
            bool tie;
            o.x = (signed char)gaussian_round_e((uint64_t)w[0] | ((uint64_t)w[1] << 32),
                                              (uint64_t)w[2] | ((uint64_t)w[3] << 32), &tie);
            ties += tie;
            o.y = (signed char)gaussian_round_e((uint64_t)w[4] | ((uint64_t)w[5] << 32),
                                              (uint64_t)w[6] | ((uint64_t)w[7] << 32), &tie);
            ties += tie;
            o.z = (signed char)gaussian_round_e((uint64_t)w[8] | ((uint64_t)w[9] << 32),
                                              (uint64_t)w[10] | ((uint64_t)w[11] << 32), &tie);
            ties += tie;
            o.w = (signed char)gaussian_round_e((uint64_t)w[12] | ((uint64_t)w[13] << 32),
                                              (uint64_t)w[14] | ((uint64_t)w[15] << 32), &tie);
            ties += tie;
            reinterpret_cast<char4*>(e + (size_t)v * NN)[b] = o;
        }
        if (ties && stats) atomicAdd(stats + STAT_NEAR_TIE, (unsigned long long)ties);
    }
    // keep this CTA's shared memory alive until the others have read it
    cluster.sync();
}

bool encode_cluster_supported(int logn) {
    if (logn != 14 && logn != 15) return false;
    auto kern = logn == 14 ? k_encode_n16k : k_encode_n32k;
    if (ensure_smem(kern, enc1::SMEM) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(logn == 14 ? 2 : 4, 1, 1);
    cfg.blockDim = dim3(enc1::NT, 1, 1);
    cfg.dynamicSmemBytes = enc1::SMEM;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return clusters > 0;
}

cudaError_t launch_encode(const DevCtx& c, const SlotSrc& src, int nvec, int64_t* m, int8_t* e,
                          const uint64_t* seeds, uint64_t gauss_off, double* scratch, cudaStream_t s) {
    if (nvec <= 0) return cudaSuccess;
    if (e && (gauss_off & 15)) return cudaErrorInvalidValue;
    if (c.logn == 14 && c.encode_cluster) {
        cudaError_t er = ensure_smem(k_encode_n16k, enc1::SMEM);
        if (er != cudaSuccess) return er;
        KScope ks("encode", s);
        k_encode_n16k<<<2 * nvec, enc1::NT, enc1::SMEM, s>>>(src, c.fft, m, e, seeds, gauss_off, c.stats);
        return cudaGetLastError();
    }
    if (c.logn == 15 && c.encode_cluster) {
        cudaError_t er = ensure_smem(k_encode_n32k, enc1::SMEM);
        if (er != cudaSuccess) return er;
        KScope ks("encode", s);
        k_encode_n32k<<<4 * nvec, enc1::NT, enc1::SMEM, s>>>(src, c.fft, m, e, seeds, gauss_off, c.stats);
        return cudaGetLastError();
    }
    TSG_LOGN_SWITCH(c.logn, {
        using G = FftGeo<LG>;
        const size_t smem = (size_t)2 * G::BLK * sizeof(double);
        cudaError_t er = ensure_smem(k_encode_a<LG>, smem);
        if (er != cudaSuccess) return er;
        {
            KScope ks("encode_a", s);
            k_encode_a<LG><<<dim3(G::NB, nvec), 1024, smem, s>>>(src, c.fft, scratch);
        }
        KScope ks("encode_b", s);
        k_encode_b<LG><<<nvec, 1024, 0, s>>>(scratch, c.fft, m, e, seeds, gauss_off, c.stats);
    });
    return cudaGetLastError();
}

// pt_ntt = NTT(encode(z)) (ciphertext.rs:539-545): signed residues per limb
// (the residue can be q itself in the reference's negative branch; the lazy
// NTT accepts it and reduces it like 0).

}  // namespace tsg
