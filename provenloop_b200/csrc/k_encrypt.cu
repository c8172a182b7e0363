// k_encrypt.cu -- secret-key encryption per (ciphertext, limb) (sm_100a).
#include <cooperative_groups.h>

#include "launch.cuh"

namespace cg = cooperative_groups;

namespace tsg {

// ======================================================================
// Encryption per (ciphertext, limb) (ciphertext.rs:167-229)
// ======================================================================
// Candidates per window round of k_enc_a's plan mode (2 words each); the
// window of 2 * kEncPlanRound + 16 words follows the NTT buffer.
constexpr int kEncPlanRound = 4096;
constexpr size_t kEncPlanWinBytes = (2 * kEncPlanRound + 16) * 4;

// Staging of c1 = NTT(a)'s input in the speculative pass: this CTA's share
// of limb `limb`'s candidates (h0 .. h0 + H - 1, 8 per ChaCha20 block) into
// shared memory.  Returns whether any of them fell in the rejection zone.
template <int LOGN, int CLX, int MINB>
__device__ __forceinline__ bool enc_a_stage(uint64_t* sm, uint64_t seed, const LimbTab& T, int limb, int h0, int tid) {
    using C = NttCfg<LOGN, CLX>;
    constexpr int N = 1 << LOGN, NT = C::NT, H = C::H;
    // two CTAs per SM (k_enc_fused below N = 32768): FP64 limbs' draws are
    // staged as exact doubles; the other forms stage residues
    constexpr bool kDblStage = MINB == 2 && kPairFp<LOGN, CLX, MINB>;
    // this CTA's share: candidates h0 .. h0 + H - 1, 8 per block
    const uint32_t blk0 = (uint32_t)limb * (N / 8);
    bool rej = false;
    if (kDblStage && T.fp) {  // (kDblStage: every staged FP64-limb word is a double)
        // FP64 limb: u = hi 2^32 + lo = hi (2^32 mod q) + lo (mod q),
        // staged as the exact double fp_mulmod(hi, 2^32 mod q) + lo
        // (|x| <= q + 2^32), which the transform's input reduction
        // takes like the residue; the IMAD pipe is the busier one here
        const double q = __ull2double_rn(T.q);
        const uint64_t r = ((uint64_t)1 << 32) % T.q;
        const double r32 = r > T.q / 2 ? -__ull2double_rn(T.q - r) : __ull2double_rn(r);
        const double r32q = __ddiv_rn(r32, q);
        for (int b = h0 / 8 + tid; b < (h0 + H) / 8; b += NT) {
            uint32_t w[16];
            chacha_block(seed, blk0 + (uint32_t)b, w);
#pragma unroll
            for (int c = 0; c < 8; c++) {
                const uint64_t u = (uint64_t)w[2 * c] | ((uint64_t)w[2 * c + 1] << 32);
                rej |= (u < T.thresh);  // range_u64 rejection zone [0, 2^64 mod q)
                const double x = __dadd_rn(fp_mulmod(__uint2double_rn(w[2 * c + 1]), r32, r32q, q),
                                           __uint2double_rn(w[2 * c]));
                sm[pad(8 * b + c - h0)] = vbits(x);
            }
        }
    } else {
        for (int b = h0 / 8 + tid; b < (h0 + H) / 8; b += NT) {
            uint32_t w[16];
            chacha_block(seed, blk0 + (uint32_t)b, w);
#pragma unroll
            for (int c = 0; c < 8; c++) {
                const uint64_t u = (uint64_t)w[2 * c] | ((uint64_t)w[2 * c + 1] << 32);
                rej |= (u < T.thresh);  // range_u64 rejection zone [0, 2^64 mod q)
                sm[pad(8 * b + c - h0)] = mod_u64(u, T.q, T.mu64);
            }
        }
    }
    return rej;
}

// Two single-transform kernels (each fits in registers):
//   k_enc_a: c1 = NTT(a), a = range_u64(q_l) draws (sampling.rs:62-64);
//   k_enc_u: c0 = NTT(m + e mod q_l) - c1 * s.
// NTT(m) + NTT(e) of the reference equals NTT(m + e) exactly (the transform
// is linear mod q and both results are canonical).  Stream layout
// (speculative, no rejection): limb l's candidate i at words 2*l*N + 2i, low
// word first; the Gaussian block follows at 2*L*N.  In list mode the CTAs
// walk the flagged streams only, using their exact plans.
template <int LOGN, int CLX = ntt_default_cl(LOGN), int MINB = 1>
__global__ void __launch_bounds__(NttCfg<LOGN, CLX>::NT, MINB)
    k_enc_a(uint64_t* __restrict__ ct, const uint64_t* __restrict__ seeds, const LimbTab* __restrict__ tabs, int L,
            int nvec, uint32_t* flags, const StreamPlan* __restrict__ plans, int plan_mode) {
    extern __shared__ __align__(16) uint64_t sm[];
    using C = NttCfg<LOGN, CLX>;
    constexpr int N = 1 << LOGN, NT = C::NT, H = C::H;
    // a two-per-SM pair form would stage FP64 limbs' draws as exact doubles
    // (as k_enc_fused does); the forms launched here (repair, small batch,
    // MINB = 1) stage residues
    constexpr bool kDblStage = MINB == 2 && kPairFp<LOGN, CLX, MINB>;
    const int limb = blockIdx.x / C::CL, tid = threadIdx.x;
    const int h0 = ntt_rank<LOGN, CLX>() * H;  // first element of this CTA's share
    const LimbTab T = tabs[limb];
    if (kDblStage) plan_mode = 0;  // the throughput form is launched for the speculative pass only
    const int nwork = plan_mode ? (int)flags[nvec] : 1;
    for (int it = blockIdx.y; it < (plan_mode ? nwork : (int)blockIdx.y + 1); it += gridDim.y) {
        const int v = plan_mode ? (int)flags[nvec + 1 + it] : it;
        const uint64_t seed = seeds[v];
        uint64_t* c1 = ct + (((size_t)v * 2 * L + L + limb) << LOGN);
        if (!plan_mode) {
            if (enc_a_stage<LOGN, CLX, MINB>(sm, seed, T, limb, h0, tid)) flag_stream(flags, nvec, v);
        } else {
            // exact plan: candidates 0 .. N + nrej - 1 of this limb's segment
            // at words off + 2*cidx; the rejected ones are skipped and
            // accepted candidate cidx lands at output cidx - (# rejected
            // before it).  Words come through a window behind the NTT buffer.
            const StreamPlan& P = plans[v];
            uint32_t* win = reinterpret_cast<uint32_t*>(sm + C::SMEM_WORDS);
            const uint32_t nrej = P.nrej[limb];
            const uint32_t* rej = P.rej[limb];
            const int ncand = N + (int)nrej;
            for (int c0 = 0; c0 < ncand; c0 += kEncPlanRound) {
                const int cnt = ncand - c0 < kEncPlanRound ? ncand - c0 : kEncPlanRound;
                const uint64_t ws = P.off[limb] + 2ULL * c0;
                const int sh = (int)(ws & 15);
                __syncthreads();
                chacha_window(seed, ws >> 4, (sh + 2 * cnt + 15) >> 4, win);
                __syncthreads();
                for (int cl = tid; cl < cnt; cl += NT) {
                    const uint32_t cidx = (uint32_t)(c0 + cl);
                    uint32_t before = 0;
                    bool rejected = false;
                    for (uint32_t t = 0; t < nrej; t++) {
                        before += rej[t] < cidx;
                        rejected |= rej[t] == cidx;
                    }
                    const int i = (int)(cidx - before);
                    if (!rejected && i >= h0 && i < h0 + H) {  // outputs of this CTA's share
                        const int o = sh + 2 * cl;
                        const uint64_t u = (uint64_t)win[o] | ((uint64_t)win[o + 1] << 32);
                        sm[pad(i - h0)] = mod_u64(u, T.q, T.mu64);
                    }
                }
            }
        }
        if constexpr (C::CL == 2) cluster_sync();  // the transform reads both shares
        else __syncthreads();
        ntt_forward_from_smem<LOGN, CLX, kPairFp<LOGN, CLX, MINB>, kDblStage>(sm, T,
                                                                              [&](int j, uint64_t x) { c1[j] = x; });
        __syncthreads();
    }
}

template <int LOGN, int CLX = ntt_default_cl(LOGN), int MINB = 1>
__global__ void __launch_bounds__(NttCfg<LOGN, CLX>::NT, MINB)
    k_enc_u(uint64_t* __restrict__ ct, const int64_t* __restrict__ m, const int8_t* __restrict__ e,
            const uint64_t* __restrict__ sk, const uint64_t* __restrict__ sks, const int* __restrict__ sk_of,
            const LimbTab* __restrict__ tabs, int L,
            int nvec, const uint32_t* __restrict__ flags, int list_mode, int sub) {
    extern __shared__ __align__(16) uint64_t sm[];
    using C = NttCfg<LOGN, CLX>;
    const int limb = blockIdx.x / C::CL;
    const int h0 = ntt_rank<LOGN, CLX>() * C::H;
    const LimbTab T = tabs[limb];
    const int nwork = list_mode ? (int)flags[nvec] : 1;
    for (int it = blockIdx.y; it < (list_mode ? nwork : (int)blockIdx.y + 1); it += gridDim.y) {
        const int v = list_mode ? (int)flags[nvec + 1 + it] : it;
        uint64_t* c0 = ct + (((size_t)v * 2 * L + limb) << LOGN);
        const uint64_t* c1 = ct + (((size_t)v * 2 * L + L + limb) << LOGN);
        const size_t so = ((size_t)(sk_of ? sk_of[v] : 0) * L + limb) << LOGN;
        const uint64_t* s = sk + so;
        const uint64_t* sp = sks + so;
        const int64_t* mv = m + ((size_t)v << LOGN);
        const int8_t* ev = e + ((size_t)v << LOGN);
        if (sub && threadIdx.x == 0) prefetch_l2(c1 + h0, (unsigned)C::H * 8u);  // this CTA's share, read by the epilogue
        ntt_forward_signed<LOGN, CLX, kPairFp<LOGN, CLX, MINB>>(
            sm, T, [&](int j) { return mv[j]; }, [&](int j) { return (int)ev[j]; },
            [&](int j, uint64_t x) {
                if (!sub) {  // x alone; k_enc_combine subtracts c1*s later
                    c0[j] = x;
                    return;
                }
                // x - c1*s with the product in [0, 4q): x + 4q - as lies in [1, 5q)
                const uint64_t as = mul_shoup4(c1[j], s[j], sp[j], T.q);
                c0[j] = canon8(x + 4 * T.q - as, T.q);
            });
        __syncthreads();
    }
}

// Both transforms of a (ciphertext, limb) on one CTA pair, one after the
// other (the throughput form from N = 8192: two CTAs per SM below N = 32768,
// one at it).  c1 = NTT(a) is stored, and t = c1*s goes to c0's place; then
// c0 = NTT(m + e) - t.  Every forward transform stores element
// h*H + tid + k*NT from thread tid, so each thread reads back only the t it
// wrote itself, one transform later, while it is still in L2: the c1 round
// trip through HBM that k_enc_a + k_enc_u make is gone.  c1 and the final c0
// are streaming stores (evicted first).
// A stream that met a rejection is flagged and redone by the repair pass
// (k_enc_a's plan mode, then k_enc_u's list mode, which reads c1).
//
// Phase 1 of k_enc_fused: c1 = NTT(a) stored, t = c1*s into c0's place.
// Out of line, like phase 2, so each transform is register-allocated alone.
// MINB: CTAs per SM (2 up to N = 16384, where the FP64 limbs' draws are
// staged as doubles; 1 at N = 32768, whose shares fill an SM's shared memory).
template <int LOGN, int MINB>
__device__ __noinline__ void enc_fused_c1(uint64_t* sm, uint64_t seed, const LimbTab* __restrict__ tabs, int limb,
                                          uint64_t* c0, uint64_t* c1, const uint64_t* __restrict__ s,
                                          const uint64_t* __restrict__ sp, uint32_t* flags, int nvec, int v) {
    using C = NttCfg<LOGN, 2>;
    constexpr bool kFp = kPairFp<LOGN, 2, MINB>;
    constexpr bool kDbl = MINB == 2 && kFp;  // FP64 limbs' draws staged as doubles (as enc_a_stage does)
    const LimbTab T = tabs[limb];
    const int h0 = ntt_rank<LOGN, 2>() * C::H;
    if (enc_a_stage<LOGN, 2, MINB>(sm, seed, T, limb, h0, (int)threadIdx.x)) flag_stream(flags, nvec, v);
    cluster_sync();  // the transform reads both shares
    ntt_forward_from_smem<LOGN, 2, kFp, kDbl>(sm, T, [&](int j, uint64_t x) {
        __stcs(reinterpret_cast<unsigned long long*>(c1 + j), (unsigned long long)x);
        c0[j] = mul_shoup4(x, s[j], sp[j], T.q);  // t, in [0, 4q)
    });
}

// Phase 2 of k_enc_fused: c0 = NTT(m + e) - t.
template <int LOGN, int MINB>
__device__ __noinline__ void enc_fused_c0(uint64_t* sm, const LimbTab* __restrict__ tabs, int limb, uint64_t* c0,
                                          const int64_t* __restrict__ mv, const int8_t* __restrict__ ev) {
    constexpr bool kFp = kPairFp<LOGN, 2, MINB>;
    const LimbTab T = tabs[limb];
    ntt_forward_signed<LOGN, 2, kFp>(
        sm, T, [&](int j) { return mv[j]; }, [&](int j) { return (int)ev[j]; },
        [&](int j, uint64_t x) {
            // x - t with t in [0, 4q): x + 4q - t lies in [1, 5q)
            const uint64_t t = __ldcs(reinterpret_cast<const unsigned long long*>(c0 + j));
            __stcs(reinterpret_cast<unsigned long long*>(c0 + j), (unsigned long long)canon8(x + 4 * T.q - t, T.q));
        });
}

template <int LOGN, int MINB>
__global__ void __launch_bounds__(NttCfg<LOGN, 2>::NT, MINB)
    k_enc_fused(uint64_t* __restrict__ ct, const uint64_t* __restrict__ seeds, const int64_t* __restrict__ m,
                const int8_t* __restrict__ e, const uint64_t* __restrict__ sk, const uint64_t* __restrict__ sks,
                const int* __restrict__ sk_of, const LimbTab* __restrict__ tabs, int L, int nvec, uint32_t* flags) {
    extern __shared__ __align__(16) uint64_t sm[];
    using C = NttCfg<LOGN, 2>;
    const int limb = blockIdx.x / C::CL, v = blockIdx.y;
    uint64_t* c0 = ct + (((size_t)v * 2 * L + limb) << LOGN);
    uint64_t* c1 = c0 + ((size_t)L << LOGN);
    const size_t so = ((size_t)(sk_of ? sk_of[v] : 0) * L + limb) << LOGN;
    if (threadIdx.x == 0) {  // phase 2's inputs (this CTA's half of the m and e rows) into L2 meanwhile
        const size_t o = ((size_t)v << LOGN) + (size_t)ntt_rank<LOGN, 2>() * C::H;
        prefetch_l2(m + o, (uint32_t)C::H * 8u);
        prefetch_l2(e + o, (uint32_t)C::H);
    }
    enc_fused_c1<LOGN, MINB>(sm, seeds[v], tabs, limb, c0, c1, sk + so, sks + so, flags, nvec, v);
    __syncthreads();
    enc_fused_c0<LOGN, MINB>(sm, tabs, limb, c0, m + ((size_t)v << LOGN), e + ((size_t)v << LOGN));
}

// c0 -= c1*s over every limb of nvec ciphertexts, c0 holding NTT(m + e)
// (the second half of k_enc_u when the two transforms ran concurrently).
__global__ void k_enc_combine(uint64_t* __restrict__ ct, const uint64_t* __restrict__ sk,
                              const uint64_t* __restrict__ sks, const int* __restrict__ sk_of,
                              const LimbTab* __restrict__ tabs, int L, int logn, long long total) {
    for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
         t += (long long)gridDim.x * blockDim.x) {
        const int j = (int)(t & ((1 << logn) - 1));
        const long long vl = t >> logn;
        const int l = (int)(vl % L);
        const long long v = vl / L;
        const uint64_t q = tabs[l].q;
        uint64_t* c0 = ct + ((v * 2 * L + l) << logn);
        const uint64_t* c1 = ct + ((v * 2 * L + L + l) << logn);
        const size_t so = ((size_t)(sk_of ? sk_of[v] : 0) * L + l) << logn;
        const uint64_t as = mul_shoup4(c1[j], sk[so + j], sks[so + j], q);
        c0[j] = canon8(c0[j] + 4 * q - as, q);
    }
}

cudaError_t launch_encrypt_limbs(const DevCtx& c, uint64_t* ct, const int64_t* m, const int8_t* e, const uint64_t* sk,
                                 const uint64_t* sks, const int* sk_of, const uint64_t* seeds, int nvec, uint32_t* flags,
                                 const StreamPlan* plans, bool plan_mode, cudaStream_t s) {
    if (nvec <= 0) return cudaSuccess;
    TSG_LOGN_SWITCH(c.logn, {
        constexpr size_t smem = ntt_smem_bytes<LG>();
        constexpr int CL = NttCfg<LG>::CL;
        // (LP: the pair form exists from N = 8192; other sizes never take it)
        constexpr int LP = (LG == 13 || LG == 14) ? LG : 14;
        if (LG == 13 || LG == 14) {
            // speculative pass over every stream: CTA pairs, two CTAs per SM
            // (as the plain NTT), so one CTA's loads overlap the other's
            // butterflies
            if (!plan_mode) {
                constexpr size_t smem2 = (size_t)NttCfg<LP, 2>::SMEM_WORDS * 8;
                cudaError_t er = ensure_smem(k_enc_fused<LP, 2>, smem2);
                if (er != cudaSuccess) return er;
                KScope ks("enc_fused", s);
                return launch_cl(2, k_enc_fused<LP, 2>, dim3(c.L * 2, nvec), NttCfg<LP, 2>::NT, smem2, s, ct, seeds,
                                 m, e, sk, sks, sk_of, c.tabs, c.L, nvec, flags);
            }
            // the repair of the flagged streams (about one per 2048 deltas at
            // C1): each transform on a CTA pair, which halves its latency.
            // Small batches (a decode step) almost never have one, and there
            // the one-CTA form below is cheaper to launch and exit.
            if ((int)(nvec * c.L * 2) > c.sms) {
                constexpr size_t smemp = (size_t)NttCfg<LP, 2>::SMEM_WORDS * 8;
                cudaError_t er = ensure_smem(k_enc_a<LP, 2>, smemp + kEncPlanWinBytes);
                if (er != cudaSuccess) return er;
                er = ensure_smem(k_enc_u<LP, 2>, smemp);
                if (er != cudaSuccess) return er;
                const int gyp = nvec < 16 ? nvec : 16;
                {
                    KScope ks("enc_a_fix", s);
                    er = launch_cl(2, k_enc_a<LP, 2>, dim3(c.L * 2, gyp), NttCfg<LP, 2>::NT,
                                   smemp + kEncPlanWinBytes, s, ct, seeds, c.tabs, c.L, nvec, flags, plans, 1);
                    if (er != cudaSuccess) return er;
                }
                KScope ks("enc_u_fix", s);
                return launch_cl(2, k_enc_u<LP, 2>, dim3(c.L * 2, gyp), NttCfg<LP, 2>::NT, smemp, s, ct, m, e, sk,
                                 sks, sk_of, c.tabs, c.L, nvec, (const uint32_t*)flags, 1, 1);
            }
        }
        if (LG == 15 && !plan_mode) {
            // N = 32768: the same fused form at one CTA per SM (a pair's
            // shares fill the shared memory of two SMs)
            constexpr int L15 = LG == 15 ? LG : 15;
            cudaError_t er = ensure_smem(k_enc_fused<L15, 1>, smem);
            if (er != cudaSuccess) return er;
            KScope ks("enc_fused", s);
            return launch_cl(2, k_enc_fused<L15, 1>, dim3(c.L * 2, nvec), NttCfg<L15, 2>::NT, smem, s, ct, seeds, m,
                             e, sk, sks, sk_of, c.tabs, c.L, nvec, flags);
        }
        const size_t smem_a = plan_mode ? smem + kEncPlanWinBytes : smem;
        cudaError_t er = ensure_smem(k_enc_a<LG>, smem + kEncPlanWinBytes);
        if (er != cudaSuccess) return er;
        er = ensure_smem(k_enc_u<LG>, smem);
        if (er != cudaSuccess) return er;
        const int gy = plan_mode ? (nvec < 16 ? nvec : 16) : nvec;
        {
            KScope ks(plan_mode ? "enc_a_fix" : "enc_a", s);
            er = launch_cl(CL, k_enc_a<LG>, dim3(c.L * CL, gy), NttCfg<LG>::NT, smem_a, s, ct, seeds, c.tabs, c.L, nvec,
                           flags, plans, plan_mode ? 1 : 0);
            if (er != cudaSuccess) return er;
        }
        KScope ks(plan_mode ? "enc_u_fix" : "enc_u", s);
        return launch_cl(CL, k_enc_u<LG>, dim3(c.L * CL, gy), NttCfg<LG>::NT, smem, s, ct, m, e, sk, sks, sk_of, c.tabs,
                         c.L, nvec, (const uint32_t*)flags, plan_mode ? 1 : 0, 1);
    });
    return cudaGetLastError();
}

cudaError_t launch_encrypt_split(const DevCtx& c, uint64_t* ct, const int64_t* m, const int8_t* e, const uint64_t* sk,
                                 const uint64_t* sks, const int* sk_of, const uint64_t* seeds, int nvec,
                                 uint32_t* flags, const StreamPlan* plans, cudaStream_t s_a, cudaStream_t s_x) {
    if (nvec <= 0) return cudaSuccess;
    TSG_LOGN_SWITCH(c.logn, {
        // each transform on a CTA pair from N = 8192: a small batch leaves
        // most SMs idle, and the pair halves a transform's latency
        constexpr int CL = LG >= 13 ? 2 : NttCfg<LG>::CL;
        constexpr size_t smem = (size_t)NttCfg<LG, CL>::SMEM_WORDS * 8;
        cudaError_t er = ensure_smem(k_enc_a<LG, CL>, smem);
        if (er != cudaSuccess) return er;
        er = ensure_smem(k_enc_u<LG, CL>, smem);
        if (er != cudaSuccess) return er;
        {
            KScope ks("enc_a", s_a);
            er = launch_cl(CL, k_enc_a<LG, CL>, dim3(c.L * CL, nvec), NttCfg<LG, CL>::NT, smem, s_a, ct, seeds, c.tabs,
                           c.L, nvec, flags, plans, 0);
            if (er != cudaSuccess) return er;
        }
        KScope ks("enc_x", s_x);
        return launch_cl(CL, k_enc_u<LG, CL>, dim3(c.L * CL, nvec), NttCfg<LG, CL>::NT, smem, s_x, ct, m, e, sk, sks,
                         sk_of, c.tabs, c.L, nvec, (const uint32_t*)flags, 0, 0);
    });
    return cudaGetLastError();
}

cudaError_t launch_enc_combine(const DevCtx& c, uint64_t* ct, const uint64_t* sk, const uint64_t* sks,
                               const int* sk_of, int nvec, cudaStream_t s) {
    if (nvec <= 0) return cudaSuccess;
    const long long total = (long long)nvec * c.L << c.logn;
    const long long blocks = (total + 255) / 256;
    KScope ks("enc_combine", s);
    k_enc_combine<<<(int)(blocks < 8 * 148 ? blocks : 8 * 148), 256, 0, s>>>(ct, sk, sks, sk_of, c.tabs, c.L, c.logn,
                                                                             total);
    return cudaGetLastError();
}


}  // namespace tsg
