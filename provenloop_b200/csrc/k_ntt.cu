// k_ntt.cu -- plain batched NTT / INTT, key generation, the signed-input NTT of
// encode_to_ntt, and public-key encryption (sm_100a).
#include <cooperative_groups.h>

#include "launch.cuh"

namespace cg = cooperative_groups;

namespace tsg {

// ======================================================================
// Plain batched NTT / INTT (ntt.rs:79-141)
// ======================================================================
// MINB CTAs per SM: 2 for the CTA-pair form below N = 32768 (half a
// poly-limb each, 64 registers per thread), so one CTA's loads and stores
// overlap the other's butterflies.
template <int LOGN, bool INV, int CLX = ntt_default_cl(LOGN), int MINB = 1>
__global__ void __launch_bounds__(NttCfg<LOGN, CLX>::NT, MINB)
    k_ntt(uint64_t* __restrict__ data, const LimbTab* __restrict__ tabs, int lmod, int l0) {
    extern __shared__ __align__(16) uint64_t sm[];
    const long long p = blockIdx.x / CLX;
    const LimbTab T = tabs[l0 + (int)(p % lmod)];
    uint64_t* a = data + (p << LOGN);
    auto ld = [&](int j) { return a[j]; };
    auto st = [&](int j, uint64_t x) { a[j] = x; };
    if (INV)
        ntt_inverse_block<LOGN, CLX>(sm, T, ld, st);
    else
        ntt_forward_block<LOGN, CLX>(sm, T, ld, st);
}

cudaError_t launch_ntt(const DevCtx& c, uint64_t* data, long long P, int lmod, int l0, bool inverse, cudaStream_t s) {
    if (P <= 0) return cudaSuccess;
    TSG_LOGN_SWITCH(c.logn, {
        constexpr int CL = LG >= 13 ? 2 : NttCfg<LG>::CL;
        constexpr int MINB = (CL == 2 && LG < 15) ? 2 : 1;
        constexpr size_t smem = (size_t)NttCfg<LG, CL>::SMEM_WORDS * 8;
        auto kern = inverse ? k_ntt<LG, true, CL, MINB> : k_ntt<LG, false, CL, MINB>;
        cudaError_t e = ensure_smem(kern, smem);
        if (e != cudaSuccess) return e;
        KScope ks(inverse ? "ntt_inverse" : "ntt_forward", s);
        return launch_cl(CL, kern, dim3((unsigned)(P * CL)), NttCfg<LG, CL>::NT, smem, s, data, c.tabs, lmod, l0);
    });
    return cudaGetLastError();
}

// ======================================================================
// Key generation (ciphertext.rs:77-103, sampling.rs:17-29)
// ======================================================================
// Draw r (range_u32(3), word i of the stream) maps through sample_ternary
// (q = 3) and then the per-limb match to the secret coefficient:
// r = 0 -> +1, r = 1 -> -1 (q-1), r = 2 -> 0.
__device__ __forceinline__ uint64_t ternary_coeff(uint32_t r, uint64_t q) {
    const uint32_t v = r % 3u;
    return v == 0 ? 1ULL : (v == 1 ? q - 1 : 0ULL);
}

template <int LOGN>
__global__ void __launch_bounds__(NttCfg<LOGN>::NT, 1)
    k_keygen(uint64_t* __restrict__ sk, const uint64_t* __restrict__ seeds, const LimbTab* __restrict__ tabs, int L,
             int nkeys, uint32_t* flags, const StreamPlan* __restrict__ plans, int plan_mode) {
    extern __shared__ __align__(16) uint64_t sm[];
    using C = NttCfg<LOGN>;
    constexpr int NT = C::NT, H = C::H;
    const int limb = blockIdx.x / C::CL, tid = threadIdx.x;
    const int h0 = ntt_rank<LOGN>() * H;  // first element of this CTA's share
    const LimbTab T = tabs[limb];
    const int nwork = plan_mode ? (int)flags[nkeys] : 1;
    for (int it = blockIdx.y; it < (plan_mode ? nwork : (int)blockIdx.y + 1); it += gridDim.y) {
        const int key = plan_mode ? (int)flags[nkeys + 1 + it] : it;
        const uint64_t seed = seeds[key];
        if (!plan_mode) {
            // word i = sample i; block b holds samples 16b .. 16b+15 (this
            // CTA draws the blocks of its share)
            bool rej = false;
            for (int b = h0 / 16 + tid; b < (h0 + H) / 16; b += NT) {
                uint32_t w[16];
                chacha_block(seed, (uint32_t)b, w);
#pragma unroll
                for (int c = 0; c < 16; c++) {
                    rej |= (w[c] == 0u);  // range_u32(3) threshold is 1 (rng.rs:112)
                    sm[pad(16 * b + c - h0)] = ternary_coeff(w[c], T.q);
                }
            }
            if (rej && limb == 0) flag_stream(flags, nkeys, key);
        } else {
            const StreamPlan& P = plans[key];
            for (int i = h0 + tid; i < h0 + H; i += NT) {
                const uint32_t ci = cand_index((uint32_t)i, P.rej[0], P.nrej[0]);
                sm[pad(i - h0)] = ternary_coeff(chacha_word(seed, P.off[0] + ci), T.q);
            }
        }
        if constexpr (C::CL == 2) cluster_sync();  // the transform reads both shares
        else __syncthreads();
        uint64_t* out = sk + (((size_t)key * L + limb) << LOGN);
        ntt_forward_from_smem<LOGN>(sm, T, [&](int j, uint64_t x) { out[j] = x; });
        __syncthreads();
    }
}

cudaError_t launch_keygen(const DevCtx& c, uint64_t* sk, const uint64_t* seeds, int nkeys, uint32_t* flags,
                          StreamPlan* plans, cudaStream_t s) {
    TSG_LOGN_SWITCH(c.logn, {
        constexpr size_t smem = ntt_smem_bytes<LG>();
        constexpr int CL = NttCfg<LG>::CL;
        cudaError_t e = ensure_smem(k_keygen<LG>, smem);
        if (e != cudaSuccess) return e;
        KScope ks("keygen", s);
        return launch_cl(CL, k_keygen<LG>, dim3(c.L * CL, nkeys), NttCfg<LG>::NT, smem, s, sk, seeds, c.tabs, c.L,
                         nkeys, flags, plans, 0);
    });
    return cudaGetLastError();
}

cudaError_t launch_keygen_fix(const DevCtx& c, uint64_t* sk, const uint64_t* seeds, int nkeys, const uint32_t* flags,
                              const StreamPlan* plans, cudaStream_t s) {
    TSG_LOGN_SWITCH(c.logn, {
        constexpr size_t smem = ntt_smem_bytes<LG>();
        constexpr int CL = NttCfg<LG>::CL;
        cudaError_t e = ensure_smem(k_keygen<LG>, smem);
        if (e != cudaSuccess) return e;
        KScope ks("keygen_fix", s);
        const int gy = nkeys < 8 ? nkeys : 8;
        return launch_cl(CL, k_keygen<LG>, dim3(c.L * CL, gy), NttCfg<LG>::NT, smem, s, sk, seeds, c.tabs, c.L, nkeys,
                         const_cast<uint32_t*>(flags), plans, 1);
    });
    return cudaGetLastError();
}

template <int LOGN>
__global__ void __launch_bounds__(NttCfg<LOGN>::NT, 1)
    k_ntt_signed(uint64_t* __restrict__ out, const int64_t* __restrict__ m, const LimbTab* __restrict__ tabs, int L) {
    extern __shared__ __align__(16) uint64_t sm[];
    const int limb = blockIdx.x / NttCfg<LOGN>::CL, v = blockIdx.y;
    const LimbTab T = tabs[limb];
    const int64_t* mv = m + ((size_t)v << LOGN);
    uint64_t* o = out + (((size_t)v * L + limb) << LOGN);
    ntt_forward_block<LOGN>(
        sm, T, [&](int j) { return signed_residue(mv[j], T.q, T.mu64); }, [&](int j, uint64_t x) { o[j] = x; });
}

cudaError_t launch_ntt_signed(const DevCtx& c, uint64_t* out, const int64_t* m, int nvec, cudaStream_t s) {
    if (nvec <= 0) return cudaSuccess;
    TSG_LOGN_SWITCH(c.logn, {
        constexpr size_t smem = ntt_smem_bytes<LG>();
        constexpr int CL = NttCfg<LG>::CL;
        cudaError_t e = ensure_smem(k_ntt_signed<LG>, smem);
        if (e != cudaSuccess) return e;
        KScope ks("ntt_signed", s);
        return launch_cl(CL, k_ntt_signed<LG>, dim3(c.L * CL, nvec), NttCfg<LG>::NT, smem, s, out, m, c.tabs, c.L);
    });
    return cudaGetLastError();
}

// ======================================================================
// Public-key encryption (ciphertext.rs:240-319): c0 = b*u + NTT(m + e0),
// c1 = a*u + NTT(e1), with u = NTT(ternary) computed by the key-generation
// kernel from the same stream (the reference's u mapping composed with its
// ternary sampler equals keygen's: draw 0 -> 1, 1 -> q-1, 2 -> 0).
// ======================================================================
// Gaussian samples j = 4b .. 4b+3 of vector v from words off + 16b (off a
// multiple of 16): one ChaCha block per thread.
__global__ void k_gauss_gen(int8_t* __restrict__ e, const uint64_t* __restrict__ seeds, int N, uint64_t off,
                            unsigned long long* stats) {
    const int v = blockIdx.y;
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    int ties = 0;
    if (b < N / 4) {
        uint32_t w[16];
        chacha_block(seeds[v], (uint32_t)((off >> 4) + (uint64_t)b), w);
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

cudaError_t launch_gauss_gen(const DevCtx& c, int8_t* e, const uint64_t* seeds, int nvec, uint64_t off,
                             cudaStream_t s) {
    if (nvec <= 0) return cudaSuccess;
    if (off & 15) return cudaErrorInvalidValue;
    KScope ks("gauss_gen", s);
    k_gauss_gen<<<dim3((c.n / 4 + 255) / 256, nvec), 256, 0, s>>>(e, seeds, c.n, off, c.stats);
    return cudaGetLastError();
}

// Component comp = blockIdx.z of ciphertext v, limb blockIdx.x / CL.
template <int LOGN>
__global__ void __launch_bounds__(NttCfg<LOGN>::NT, 1)
    k_enc_pk(uint64_t* __restrict__ ct, const int64_t* __restrict__ m, const int8_t* __restrict__ e0,
             const int8_t* __restrict__ e1, const uint64_t* __restrict__ U, const uint64_t* __restrict__ pk,
             const uint64_t* __restrict__ pks, const LimbTab* __restrict__ tabs, int L) {
    extern __shared__ __align__(16) uint64_t sm[];
    const int limb = blockIdx.x / NttCfg<LOGN>::CL, v = blockIdx.y, comp = blockIdx.z;
    const LimbTab T = tabs[limb];
    uint64_t* out = ct + (((size_t)v * 2 * L + (size_t)comp * L + limb) << LOGN);
    // pk layout [2][L][n]: b then a; u of this vector and limb
    const uint64_t* P = pk + (((size_t)(comp ? L : 0) + limb) << LOGN);
    const uint64_t* Ps = pks + (((size_t)(comp ? L : 0) + limb) << LOGN);
    const uint64_t* u = U + (((size_t)v * L + limb) << LOGN);
    const int64_t* mv = m + ((size_t)v << LOGN);
    const int8_t* ev = (comp ? e1 : e0) + ((size_t)v << LOGN);
    ntt_forward_block<LOGN>(
        sm, T,
        [&](int j) {
            // |e| < q: the reference's residue of a negative e is q + e
            const int ej = ev[j];
            const uint64_t er = ej >= 0 ? (uint64_t)ej : T.q + ej;
            return comp ? er : add_mod(signed_residue(mv[j], T.q, T.mu64), er, T.q);
        },
        [&](int j, uint64_t x) { out[j] = canon8(x + mul_shoup4(u[j], P[j], Ps[j], T.q), T.q); });
}

cudaError_t launch_enc_pk(const DevCtx& c, uint64_t* ct, const int64_t* m, const int8_t* e0, const int8_t* e1,
                          const uint64_t* U, const uint64_t* pk, const uint64_t* pks, int nvec, cudaStream_t s) {
    if (nvec <= 0) return cudaSuccess;
    TSG_LOGN_SWITCH(c.logn, {
        constexpr size_t smem = ntt_smem_bytes<LG>();
        constexpr int CL = NttCfg<LG>::CL;
        cudaError_t er = ensure_smem(k_enc_pk<LG>, smem);
        if (er != cudaSuccess) return er;
        KScope ks("enc_pk", s);
        return launch_cl(CL, k_enc_pk<LG>, dim3(c.L * CL, nvec, 2), NttCfg<LG>::NT, smem, s, ct, m, e0, e1, U, pk, pks,
                         c.tabs, c.L);
    });
    return cudaGetLastError();
}

}  // namespace tsg
