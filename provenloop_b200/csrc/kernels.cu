// kernels.cu -- CUDA kernels of the tsgpu CKKS engine (sm_100a).
//
// Every kernel reproduces a step of tensafe-he-core (cited per kernel) with
// exact integer arithmetic and, for the f64 FFT, the same rounding sequence,
// so ciphertexts and NTT outputs are bit-identical to the reference's.
#include <cooperative_groups.h>
#include <atomic>
#include <cstring>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <utility>
#include <vector>

#include "kernels.cuh"

namespace cg = cooperative_groups;

namespace tsg {

namespace {

std::mutex g_attr_mu;
std::map<std::pair<const void*, int>, size_t> g_attr_done;  // (kernel, device) -> dynamic smem limit set

// Raises a kernel's dynamic shared-memory limit to at least `bytes` on the
// current device (launchers of one kernel may need different sizes).
template <class K>
cudaError_t ensure_smem(K* kernel, size_t bytes) {
    if (bytes <= 48 * 1024) return cudaSuccess;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> g(g_attr_mu);
    auto key = std::make_pair((const void*)kernel, dev);
    auto it = g_attr_done.find(key);
    if (it != g_attr_done.end() && it->second >= bytes) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) g_attr_done[key] = bytes;
    return e;
}

// Flag list of a batch of `count` streams: flags[0..count) per-stream
// flags, flags[count] the number of flagged streams, flags[count+1 ..] their
// indexes (each stream listed once).  Repair kernels walk only the list.
__device__ __forceinline__ void flag_stream(uint32_t* flags, int count, int v) {
    if (atomicOr(flags + v, 1u) == 0u) {
        const uint32_t slot = atomicAdd(flags + count, 1u);
        flags[count + 1 + slot] = (uint32_t)v;
    }
}

// Candidate index of the i-th accepted draw given the ascending list of
// rejected candidate indexes (the reference's rejection loops skip them).
__device__ __forceinline__ uint32_t cand_index(uint32_t i, const uint32_t* rej, uint32_t nrej) {
    uint32_t c = i;
    for (uint32_t t = 0; t < nrej; t++)
        if (rej[t] <= c) c++;
    return c;
}

__device__ __forceinline__ uint64_t word64(uint64_t seed, uint64_t w) {
    return (uint64_t)chacha_word(seed, w) | ((uint64_t)chacha_word(seed, w + 1) << 32);
}

// Stream words [16*b0, 16*(b0 + nblk)) of `seed` into win (16-byte
// aligned, nblk*16 words): one ChaCha block per thread and round, instead of
// one block per word.
__device__ __forceinline__ void chacha_window(uint64_t seed, uint64_t b0, int nblk, uint32_t* win) {
    for (int b = threadIdx.x; b < nblk; b += blockDim.x) {
        uint32_t w[16];
        chacha_block(seed, (uint32_t)(b0 + b), w);
        uint4* o = reinterpret_cast<uint4*>(win + 16 * b);
        o[0] = make_uint4(w[0], w[1], w[2], w[3]);
        o[1] = make_uint4(w[4], w[5], w[6], w[7]);
        o[2] = make_uint4(w[8], w[9], w[10], w[11]);
        o[3] = make_uint4(w[12], w[13], w[14], w[15]);
    }
}

// Block-wide exclusive scan of one int per thread (blockDim.x <= 1024).
__device__ int block_exclusive_scan(int x, int* total) {
    __shared__ int warp_sums[33];  // 32 exclusive warp offsets, then the total
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    int incl = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) warp_sums[wid] = incl;
    __syncthreads();
    if (wid == 0) {
        const int nw = (blockDim.x + 31) >> 5;
        int v = lane < nw ? warp_sums[lane] : 0;
        int vi = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, vi, o);
            if (lane >= o) vi += y;
        }
        if (lane < nw) warp_sums[lane] = vi - v;
        if (lane == 31) warp_sums[32] = vi;  // total over all nw <= 32 warps
    }
    __syncthreads();
    const int res = incl - x + warp_sums[wid];
    *total = warp_sums[32];
    __syncthreads();
    return res;
}

std::atomic<uint64_t> g_launches{0};
std::atomic<bool> g_prof_on{false};
std::mutex g_prof_mu;
struct ProfEntry {
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> ev;
    double ms = 0.0;
    uint64_t launches = 0;
};
std::map<std::string, ProfEntry> g_prof;
std::vector<cudaEvent_t> g_event_pool;

cudaEvent_t pool_event() {
    if (!g_event_pool.empty()) {
        cudaEvent_t e = g_event_pool.back();
        g_event_pool.pop_back();
        return e;
    }
    cudaEvent_t e;
    cudaEventCreate(&e);
    return e;
}

// Counts the kernels launched in its scope and, when profiling is on,
// brackets them with an event pair on the launch stream.
struct KScope {
    const char* name;
    cudaStream_t s;
    int kernels;
    cudaEvent_t a = nullptr, b = nullptr;
    KScope(const char* n, cudaStream_t st, int k = 1) : name(n), s(st), kernels(k) {
        if (g_prof_on.load(std::memory_order_relaxed)) {
            std::lock_guard<std::mutex> g(g_prof_mu);
            a = pool_event();
            b = pool_event();
            cudaEventRecord(a, s);
        }
    }
    ~KScope() {
        g_launches.fetch_add((uint64_t)kernels, std::memory_order_relaxed);
        if (a) {
            cudaEventRecord(b, s);
            std::lock_guard<std::mutex> g(g_prof_mu);
            g_prof[name].ev.emplace_back(a, b);
        }
    }
};

}  // namespace

uint64_t launch_count() { return g_launches.load(); }

void prof_enable(bool on) { g_prof_on.store(on); }

void prof_reset() {
    std::lock_guard<std::mutex> g(g_prof_mu);
    for (auto& kv : g_prof) {
        for (auto& pr : kv.second.ev) {
            cudaEventSynchronize(pr.second);
            g_event_pool.push_back(pr.first);
            g_event_pool.push_back(pr.second);
        }
    }
    g_prof.clear();
}

bool prof_read(const char* name, double* ms, uint64_t* launches) {
    std::lock_guard<std::mutex> g(g_prof_mu);
    auto it = g_prof.find(name);
    if (it == g_prof.end()) return false;
    ProfEntry& P = it->second;
    for (auto& pr : P.ev) {
        float t = 0.f;
        cudaEventSynchronize(pr.second);
        cudaEventElapsedTime(&t, pr.first, pr.second);
        P.ms += t;
        P.launches += 1;
        g_event_pool.push_back(pr.first);
        g_event_pool.push_back(pr.second);
    }
    P.ev.clear();
    *ms = P.ms;
    *launches = P.launches;
    return true;
}

#define TSG_LOGN_SWITCH(logn, ...)                                \
    switch (logn) {                                               \
        case 10: { constexpr int LG = 10; __VA_ARGS__; } break;   \
        case 11: { constexpr int LG = 11; __VA_ARGS__; } break;   \
        case 12: { constexpr int LG = 12; __VA_ARGS__; } break;   \
        case 13: { constexpr int LG = 13; __VA_ARGS__; } break;   \
        case 14: { constexpr int LG = 14; __VA_ARGS__; } break;   \
        case 15: { constexpr int LG = 15; __VA_ARGS__; } break;   \
        default: return cudaErrorInvalidValue;                    \
    }

// Launch of an NTT kernel whose transforms span `cl` CTAs along x: a plain
// launch for cl = 1, a cluster launch (cluster dimension cl along x) else.
template <class... KArgs, class... Args>
cudaError_t launch_cl(int cl, void (*kern)(KArgs...), dim3 grid, unsigned block, size_t smem, cudaStream_t s,
                      Args... args) {
    if (cl == 1) {
        kern<<<grid, block, smem, s>>>(args...);
        return cudaGetLastError();
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(block, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = (unsigned)cl;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Whether a kernel instantiation carries the FP64 transform mode: yes for
// the throughput instantiations; no for the CTA-pair variants below
// N = 32768, which serve small batches, where the second code path's
// instruction fetches cost more than its faster butterflies save.
template <int LOGN, int CL, int MINB = 1>
constexpr bool kPairFp = CL == ntt_default_cl(LOGN) || MINB == 2;

// Shared-memory bytes of one NTT CTA (its padded share of a poly-limb).
template <int LOGN>
constexpr size_t ntt_smem_bytes() {
    return (size_t)NttCfg<LOGN>::SMEM_WORDS * 8;
}

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
// Element-wise limb ops (rns.rs:217-253)
// ======================================================================
__global__ void k_elementwise(uint64_t* __restrict__ out, const uint64_t* __restrict__ a,
                              const uint64_t* __restrict__ b, long long total, int logn, int L, int bcast, int op,
                              const LimbTab* __restrict__ tabs) {
    const long long stride = (long long)gridDim.x * blockDim.x * 2;
    for (long long idx = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 2; idx < total; idx += stride) {
        const long long p = idx >> logn;
        const int limb = (int)(p % L);
        const long long bi = bcast ? (((long long)limb << logn) + (idx & ((1LL << logn) - 1))) : idx;
        const uint64_t q = __ldg(&tabs[limb].q);
        const ulonglong2 av = *reinterpret_cast<const ulonglong2*>(a + idx);
        const ulonglong2 bv = *reinterpret_cast<const ulonglong2*>(b + bi);
        ulonglong2 o;
        if (op == EW_MUL) {
            const uint64_t mu = __ldg(&tabs[limb].bmu);
            const int k = __ldg(&tabs[limb].bk);
            o.x = mul_barrett(av.x, bv.x, q, mu, k);
            o.y = mul_barrett(av.y, bv.y, q, mu, k);
        } else if (op == EW_ADD) {
            o.x = add_mod(av.x, bv.x, q);
            o.y = add_mod(av.y, bv.y, q);
        } else {
            o.x = sub_mod(av.x, bv.x, q);
            o.y = sub_mod(av.y, bv.y, q);
        }
        *reinterpret_cast<ulonglong2*>(out + idx) = o;
    }
}

cudaError_t launch_elementwise(const DevCtx& c, uint64_t* out, const uint64_t* a, const uint64_t* b, long long P,
                               int L, bool b_bcast, EwOp op, cudaStream_t s) {
    const long long total = P << c.logn;
    if (total <= 0) return cudaSuccess;
    long long blocks = (total / 2 + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    KScope ks(op == EW_MUL ? "hadamard" : "add_sub", s);
    k_elementwise<<<(unsigned)blocks, 256, 0, s>>>(out, a, b, total, c.logn, L, b_bcast ? 1 : 0, (int)op, c.tabs);
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
                    e[(size_t)v * N + j] = (int8_t)gaussian_round(u1, u2, 3.19, &tie);
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
#define TSG_ENC_PASS(TL)                                                       \
    {                                                                          \
        __syncthreads();                                                       \
        const int j0 = set_base<TL>(tid);                                      \
        _Pragma("unroll") for (int k = 0; k < E; k++) {                        \
            re[k] = sre[pad(j0 + k * (1 << TL))];                              \
            im[k] = sim[pad(j0 + k * (1 << TL))];                              \
        }                                                                      \
        pass_stage<TL, 0>(re, im, j0, T);                                      \
        _Pragma("unroll") for (int k = 0; k < E; k++) {                        \
            sre[pad(j0 + k * (1 << TL))] = re[k];                              \
            sim[pad(j0 + k * (1 << TL))] = im[k];                              \
        }                                                                      \
    }
    TSG_ENC_PASS(4)
    TSG_ENC_PASS(8)
#undef TSG_ENC_PASS
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
            o.x = (signed char)gaussian_round((uint64_t)w[0] | ((uint64_t)w[1] << 32),
                                              (uint64_t)w[2] | ((uint64_t)w[3] << 32), 3.19, &tie);
            ties += tie;
            o.y = (signed char)gaussian_round((uint64_t)w[4] | ((uint64_t)w[5] << 32),
                                              (uint64_t)w[6] | ((uint64_t)w[7] << 32), 3.19, &tie);
            ties += tie;
            o.z = (signed char)gaussian_round((uint64_t)w[8] | ((uint64_t)w[9] << 32),
                                              (uint64_t)w[10] | ((uint64_t)w[11] << 32), 3.19, &tie);
            ties += tie;
            o.w = (signed char)gaussian_round((uint64_t)w[12] | ((uint64_t)w[13] << 32),
                                              (uint64_t)w[14] | ((uint64_t)w[15] << 32), 3.19, &tie);
            ties += tie;
            reinterpret_cast<char4*>(e + (size_t)v * N)[b] = o;
        }
        if (ties && stats) atomicAdd(stats + STAT_NEAR_TIE, (unsigned long long)ties);
    }
    // keep this CTA's shared memory alive until the partner has read it
    cluster.sync();
}

bool encode_cluster_supported() {
    if (ensure_smem(k_encode_n16k, enc1::SMEM) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(enc1::NT, 1, 1);
    cfg.dynamicSmemBytes = enc1::SMEM;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, k_encode_n16k, &cfg) != cudaSuccess) {
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
// Shoup companions of fixed operands (secret keys, cached plaintexts)
// ======================================================================
__global__ void k_shoup_companion(uint64_t* __restrict__ out, const uint64_t* __restrict__ in,
                                  const LimbTab* __restrict__ tabs, int L, int logn, long long total) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const uint64_t q = tabs[(int)((i >> logn) % L)].q;
        // restoring division of in * 2^64 by q (q < 2^61, so 2r never overflows)
        uint64_t r = in[i] % q, quo = 0;
        for (int b = 0; b < 64; b++) {
            r <<= 1;
            quo <<= 1;
            if (r >= q) {
                r -= q;
                quo |= 1;
            }
        }
        out[i] = quo;
    }
}

cudaError_t launch_shoup_companion(const DevCtx& c, uint64_t* out, const uint64_t* in, long long polys,
                                   cudaStream_t s) {
    if (polys <= 0) return cudaSuccess;
    const long long total = polys << c.logn;
    const long long blocks = (total + 255) / 256;
    KScope ks("shoup_companion", s);
    k_shoup_companion<<<(int)(blocks < 4 * 148 ? blocks : 4 * 148), 256, 0, s>>>(out, in, c.tabs, c.L, c.logn, total);
    return cudaGetLastError();
}

// ======================================================================
// Encryption per (ciphertext, limb) (ciphertext.rs:167-229)
// ======================================================================
// Candidates per window round of k_enc_a's plan mode (2 words each); the
// window of 2 * kEncPlanRound + 16 words follows the NTT buffer.
constexpr int kEncPlanRound = 4096;
constexpr size_t kEncPlanWinBytes = (2 * kEncPlanRound + 16) * 4;

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
    const int limb = blockIdx.x / C::CL, tid = threadIdx.x;
    const int h0 = ntt_rank<LOGN, CLX>() * H;  // first element of this CTA's share
    const LimbTab T = tabs[limb];
    const int nwork = plan_mode ? (int)flags[nvec] : 1;
    for (int it = blockIdx.y; it < (plan_mode ? nwork : (int)blockIdx.y + 1); it += gridDim.y) {
        const int v = plan_mode ? (int)flags[nvec + 1 + it] : it;
        const uint64_t seed = seeds[v];
        uint64_t* c1 = ct + (((size_t)v * 2 * L + L + limb) << LOGN);
        if (!plan_mode) {
            // this CTA's share: candidates h0 .. h0 + H - 1, 8 per block
            const uint32_t blk0 = (uint32_t)limb * (N / 8);
            bool rej = false;
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
            if (rej) flag_stream(flags, nvec, v);
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
        ntt_forward_from_smem<LOGN, CLX, kPairFp<LOGN, CLX, MINB>>(sm, T, [&](int j, uint64_t x) { c1[j] = x; });
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
        ntt_forward_block<LOGN, CLX, kPairFp<LOGN, CLX, MINB>>(
            sm, T,
            [&](int j) {
                // |e| < q: the reference's residue of a negative e is q + e
                const int ej = ev[j];
                return add_mod(signed_residue(mv[j], T.q, T.mu64), ej >= 0 ? (uint64_t)ej : T.q + ej, T.q);
            },
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
                cudaError_t er = ensure_smem(k_enc_a<LP, 2, 2>, smem2);
                if (er != cudaSuccess) return er;
                er = ensure_smem(k_enc_u<LP, 2, 2>, smem2);
                if (er != cudaSuccess) return er;
                {
                    KScope ks("enc_a", s);
                    er = launch_cl(2, k_enc_a<LP, 2, 2>, dim3(c.L * 2, nvec), NttCfg<LP, 2>::NT, smem2, s, ct, seeds,
                                   c.tabs, c.L, nvec, flags, plans, 0);
                    if (er != cudaSuccess) return er;
                }
                KScope ks("enc_u", s);
                return launch_cl(2, k_enc_u<LP, 2, 2>, dim3(c.L * 2, nvec), NttCfg<LP, 2>::NT, smem2, s, ct, m, e, sk,
                                 sks, sk_of, c.tabs, c.L, nvec, (const uint32_t*)flags, 0, 1);
            }
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

// ======================================================================
// L2 warm-up for latency-bound small batches.  A decode step runs one delta
// per layer between weight streams that evict L2, so a small batch would
// otherwise take an HBM round trip on every dependent twiddle, key and
// plaintext load of its one-CTA-per-limb kernels.  Pieces of kL2Piece bytes
// are spread over the grid; each is one cp.async.bulk.prefetch.L2 (16-byte
// aligned start and length, rounded inwards).
// ======================================================================
constexpr long long kL2Piece = 8192;

__device__ __forceinline__ long long l2_pieces(const L2Range& R) {
    return (long long)R.rows * R.reps * ((R.bytes + kL2Piece - 1) / kL2Piece);
}

__global__ void __launch_bounds__(128) k_prefetch_l2(L2List L) {
    long long first[kMaxL2Ranges + 1];
    first[0] = 0;
    for (int k = 0; k < L.n; k++) first[k + 1] = first[k] + l2_pieces(L.r[k]);
    const long long total = first[L.n];
    for (long long p = (long long)blockIdx.x * blockDim.x + threadIdx.x; p < total;
         p += (long long)gridDim.x * blockDim.x) {
        int k = 0;
        while (p >= first[k + 1]) k++;
        const L2Range& R = L.r[k];
        long long q = p - first[k];
        const long long chunks = (R.bytes + kL2Piece - 1) / kL2Piece;
        const long long chunk = q % chunks;
        q /= chunks;
        const int rep = (int)(q % R.reps), row = (int)(q / R.reps);
        long long off = (long long)rep * R.rep_stride + chunk * kL2Piece;
        if (R.idx) {
            const int i = R.idx[row];
            if (i < 0 || i >= R.idx_max) continue;
            off += (long long)i * R.idx_stride;
        }
        const long long len = R.bytes - chunk * kL2Piece < kL2Piece ? R.bytes - chunk * kL2Piece : kL2Piece;
        const size_t a = __cvta_generic_to_global(static_cast<const char*>(R.base) + off);
        const size_t lo = (a + 15) & ~(size_t)15, hi = (a + (size_t)len) & ~(size_t)15;
        if (hi > lo)
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(lo), "r"((unsigned)(hi - lo)) : "memory");
    }
}

cudaError_t launch_prefetch_l2(const L2List& list, cudaStream_t s) {
    if (list.n <= 0) return cudaSuccess;
    if (list.n > kMaxL2Ranges) return cudaErrorInvalidValue;
    long long total = 0;
    for (int k = 0; k < list.n; k++) {
        const L2Range& R = list.r[k];
        if (!R.base || R.rows < 1 || R.reps < 1 || R.bytes < 0 || (!R.idx && R.rows != 1)) return cudaErrorInvalidValue;
        total += (long long)R.rows * R.reps * ((R.bytes + kL2Piece - 1) / kL2Piece);
    }
    if (total == 0) return cudaSuccess;
    const long long blocks = (total + 127) / 128;
    KScope ks("prefetch_l2", s);
    k_prefetch_l2<<<(int)(blocks < 148 ? blocks : 148), 128, 0, s>>>(list);
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
        o.x = (signed char)gaussian_round((uint64_t)w[0] | ((uint64_t)w[1] << 32),
                                          (uint64_t)w[2] | ((uint64_t)w[3] << 32), 3.19, &tie);
        ties += tie;
        o.y = (signed char)gaussian_round((uint64_t)w[4] | ((uint64_t)w[5] << 32),
                                          (uint64_t)w[6] | ((uint64_t)w[7] << 32), 3.19, &tie);
        ties += tie;
        o.z = (signed char)gaussian_round((uint64_t)w[8] | ((uint64_t)w[9] << 32),
                                          (uint64_t)w[10] | ((uint64_t)w[11] << 32), 3.19, &tie);
        ties += tie;
        o.w = (signed char)gaussian_round((uint64_t)w[12] | ((uint64_t)w[13] << 32),
                                          (uint64_t)w[14] | ((uint64_t)w[15] << 32), 3.19, &tie);
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

// ======================================================================
// Rescale (ciphertext.rs:476-535), coefficient-domain step: for limbs
// l < nl-1 of both components, (x_l - (x_last mod q_l)) * q_last^-1 mod q_l.
// ======================================================================
__global__ void k_rescale_combine(uint64_t* __restrict__ out, const uint64_t* __restrict__ in, int nl, int logn,
                                  long long total, const LimbTab* __restrict__ tabs, RescaleInv inv) {
    const int n = 1 << logn;
    for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
         t += (long long)gridDim.x * blockDim.x) {
        // t indexes out [count][2][nl-1][n]
        const int i = (int)(t & (n - 1));
        const long long pl = t >> logn;
        const int l = (int)(pl % (nl - 1));
        const long long vc = pl / (nl - 1);  // vector * 2 + component
        const LimbTab& T = tabs[l];
        const uint64_t x = in[((vc * nl + l) << logn) + i];
        const uint64_t y = mod_u64(in[((vc * nl + nl - 1) << logn) + i], T.q, T.mu64);
        const uint64_t d = x >= y ? x - y : T.q - y + x;
        out[t] = mul_barrett(d, inv.v[l], T.q, T.bmu, T.bk);
    }
}

cudaError_t launch_rescale_combine(const DevCtx& c, uint64_t* out, const uint64_t* in, int count, int nl,
                                   const RescaleInv& inv, cudaStream_t s) {
    if (count <= 0 || nl < 2) return cudaErrorInvalidValue;
    const long long total = (long long)count * 2 * (nl - 1) << c.logn;
    const long long blocks = (total + 255) / 256;
    KScope ks("rescale", s);
    k_rescale_combine<<<(int)(blocks < 8 * 148 ? blocks : 8 * 148), 256, 0, s>>>(out, in, nl, c.logn, total, c.tabs,
                                                                                 inv);
    return cudaGetLastError();
}

// ======================================================================
// Exact stream plans for streams that hit a rejection (rng.rs:109-133)
// ======================================================================
// Candidates each plan thread tests per round, and the window that holds
// their words (up to 2 words per candidate, 1024 threads, plus one block
// of misalignment).
constexpr int kPlanCand = 4;
constexpr int kPlanWin = kPlanCand * 1024 * 2 + 16;

__device__ void plan_one(const uint64_t* __restrict__ seeds, int v, StreamPlan* plans, const SegList& segs,
                         const LimbTab* __restrict__ tabs, int N, unsigned long long* stats, int tid, uint64_t base) {
    __shared__ uint32_t s_nrej;
    __shared__ uint32_t s_rej[kMaxRej + 1];
    __shared__ uint32_t s_overflow;
    __shared__ __align__(16) uint32_t win[kPlanWin];
    StreamPlan& P = plans[v];
    const uint64_t seed = seeds[v];
    uint64_t off = base;  // first word of this stream's segments
    if (tid == 0) s_overflow = 0;
    for (int sg = 0; sg < segs.count; sg++) {
        const int kind = segs.kind[sg];
        if (tid == 0) {
            P.off[sg] = off;
            P.nrej[sg] = 0;
            s_nrej = 0;
        }
        __syncthreads();
        if (kind == SEG_GAUSS) {
            off += 4ULL * N;
            continue;
        }
        const int wpc = kind == SEG_UNIFORM ? 2 : 1;
        const uint64_t thr = kind == SEG_UNIFORM ? tabs[segs.limb[sg]].thresh : 1ULL;
        const int per_round = kPlanCand * (int)blockDim.x;
        long long accepted = 0, base = 0;
        // bounded: a segment that needs more than 4N candidates is reported
        // as an overflow instead of scanning on
        while (accepted < N && base < 4LL * N) {
            // candidates base .. base + per_round - 1 sit at words ws + wpc*i
            const uint64_t ws = off + (uint64_t)wpc * (uint64_t)base;
            const int sh = (int)(ws & 15);
            chacha_window(seed, ws >> 4, (sh + wpc * per_round + 15) >> 4, win);
            __syncthreads();
            int ok[kPlanCand], cnt = 0;
#pragma unroll
            for (int t = 0; t < kPlanCand; t++) {
                const int o = sh + wpc * (tid * kPlanCand + t);
                const uint64_t val = wpc == 2 ? ((uint64_t)win[o] | ((uint64_t)win[o + 1] << 32)) : (uint64_t)win[o];
                ok[t] = val >= thr;
                cnt += ok[t];
            }
            int total;
            const int pre = block_exclusive_scan(cnt, &total);
            int run = pre;
#pragma unroll
            for (int t = 0; t < kPlanCand; t++) {
                if (!ok[t] && accepted + run < N) {
                    const uint32_t slot = atomicAdd(&s_nrej, 1u);
                    if (slot < kMaxRej) s_rej[slot] = (uint32_t)(base + (long long)tid * kPlanCand + t);
                    else s_overflow = 1;
                }
                run += ok[t];
            }
            accepted += total;
            base += per_round;
            __syncthreads();
        }
        if (tid == 0 && accepted < N) s_overflow = 1;
        __syncthreads();
        if (tid == 0) {
            const uint32_t nr = s_nrej < kMaxRej ? s_nrej : kMaxRej;
            // sort ascending (tiny list)
            for (uint32_t a = 1; a < nr; a++) {
                uint32_t x = s_rej[a];
                int b = (int)a - 1;
                while (b >= 0 && s_rej[b] > x) {
                    s_rej[b + 1] = s_rej[b];
                    b--;
                }
                s_rej[b + 1] = x;
            }
            for (uint32_t a = 0; a < nr; a++) P.rej[sg][a] = s_rej[a];
            P.nrej[sg] = nr;
        }
        __syncthreads();
        off += (uint64_t)wpc * ((uint64_t)N + s_nrej);
        __syncthreads();
    }
    if (tid == 0) {
        P.status = s_overflow;
        if (stats) {
            atomicAdd(stats + STAT_REJECT, 1ULL);
            if (s_overflow) atomicAdd(stats + STAT_PLAN_FAIL, 1ULL);
        }
    }
    __syncthreads();
}

__global__ void __launch_bounds__(1024, 1)
    k_plan(const uint64_t* __restrict__ seeds, int nstreams, const uint32_t* __restrict__ flags, StreamPlan* plans,
           SegList segs, const LimbTab* __restrict__ tabs, int N, unsigned long long* stats,
           const uint64_t* __restrict__ bases) {
    const int tid = threadIdx.x;
    const int nwork = (int)flags[nstreams];
    for (int it = blockIdx.x; it < nwork; it += gridDim.x) {
        const int v = (int)flags[nstreams + 1 + it];
        plan_one(seeds, v, plans, segs, tabs, N, stats, tid, bases ? bases[v] : 0);
    }
}

cudaError_t launch_plan(const DevCtx& c, const uint64_t* seeds, int nstreams, const uint32_t* flags, StreamPlan* plans,
                        const SegList& segs, cudaStream_t s, const uint64_t* bases) {
    if (nstreams <= 0) return cudaSuccess;
    KScope ks("plan", s);
    k_plan<<<nstreams < 32 ? nstreams : 32, 1024, 0, s>>>(seeds, nstreams, flags, plans, segs, c.tabs, c.n, c.stats,
                                                          bases);
    return cudaGetLastError();
}

// Gaussian samples per window round of k_gauss_fix (4 words each).
constexpr int kGaussRound = 2048;

__global__ void __launch_bounds__(512)
    k_gauss_fix(int8_t* __restrict__ e, const uint64_t* __restrict__ seeds, int N, int nvec,
                const uint32_t* __restrict__ flags, const StreamPlan* __restrict__ plans, int seg,
                unsigned long long* stats) {
    __shared__ __align__(16) uint32_t win[4 * kGaussRound + 16];
    const int nwork = (int)flags[nvec];
    for (int it = blockIdx.x; it < nwork; it += gridDim.x) {
        const int v = (int)flags[nvec + 1 + it];
        const uint64_t seed = seeds[v];
        const uint64_t off = plans[v].off[seg];
        int ties = 0;
        for (int j0 = 0; j0 < N; j0 += kGaussRound) {
            const int cnt = N - j0 < kGaussRound ? N - j0 : kGaussRound;
            // sample j uses words off + 4j .. off + 4j + 3 (two u64 draws)
            const uint64_t ws = off + 4ULL * j0;
            const int sh = (int)(ws & 15);
            __syncthreads();
            chacha_window(seed, ws >> 4, (sh + 4 * cnt + 15) >> 4, win);
            __syncthreads();
            for (int jj = threadIdx.x; jj < cnt; jj += blockDim.x) {
                const int o = sh + 4 * jj;
                const uint64_t u1 = (uint64_t)win[o] | ((uint64_t)win[o + 1] << 32);
                const uint64_t u2 = (uint64_t)win[o + 2] | ((uint64_t)win[o + 3] << 32);
                bool tie;
                e[(size_t)v * N + j0 + jj] = (int8_t)gaussian_round(u1, u2, 3.19, &tie);
                ties += tie;
            }
        }
        if (ties && stats) atomicAdd(stats + STAT_NEAR_TIE, (unsigned long long)ties);
        __syncthreads();
    }
}

cudaError_t launch_gauss_fix(const DevCtx& c, int8_t* e, const uint64_t* seeds, int nvec, const uint32_t* flags,
                             const StreamPlan* plans, int seg, cudaStream_t s) {
    if (nvec <= 0) return cudaSuccess;
    KScope ks("gauss_fix", s);
    k_gauss_fix<<<nvec < 32 ? nvec : 32, 512, 0, s>>>(e, seeds, c.n, nvec, flags, plans, seg, c.stats);
    return cudaGetLastError();
}

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
                    const double coeff = __dmul_rn(crt_coeff(m0r[kk], sm[pad(jl)], K), inv_scale);
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

// The same decrypt for N = 8192 and 16384 on a cluster of four CTAs per
// (delta, batch) vector, two CTAs per SM: one pair of ranks (0-1 in even
// clusters, 2-3 in odd ones) runs the limb-0 INTT, the other pair the limb-1
// INTT (each CTA half a poly-limb; FP64 butterflies for a limb below 2^50),
// both parked in shared memory.  Then CTA (l, h) takes the l-th half of half
// h's positions, reading both limbs through DSMEM, into the CRT, / Delta^2
// and the segment functionals; rank 0 adds the four CTAs' partials in
// (limb, half) order.
// No limb-0 round trip through memory, and one CTA's loads overlap the
// other's butterflies on each SM.
template <int LOGN, int MAXC>
__global__ void __cluster_dims__(4, 1, 1) __launch_bounds__(NttCfg<LOGN, 2>::NT, 2)
    k_dec_quad(const uint64_t* __restrict__ cts, long long ct_stride, int ct_limbs, const uint64_t* __restrict__ sk,
               const uint64_t* __restrict__ sks, const int* __restrict__ sk_of, const uint64_t* __restrict__ pt,
               const uint64_t* __restrict__ pts, const int* __restrict__ pt_sel, int per_ct,
               const LimbTab* __restrict__ tabs, int L, CrtConst K, double inv_scale, const double* __restrict__ W,
               int cols, double* __restrict__ seg_out) {
    extern __shared__ __align__(16) uint64_t sm[];
    using C = NttCfg<LOGN, 2>;
    constexpr int N = C::N, NT = C::NT, H = C::H;
    __shared__ double red[NT / 32][kMaxSegCols];
    const int tid = threadIdx.x;
    const int v = blockIdx.x >> 2;
    // The scheduler puts the four CTAs of a cluster on four SMs and refills a
    // finished cluster's slots with the next cluster in the same rank order,
    // so with fixed roles an SM would host limb-0 CTAs (IMAD butterflies)
    // only, or limb-1 CTAs (FP64 butterflies) only.  Odd clusters swap which
    // pair takes limb 0, which mixes the two pipes' work on an SM.
    const int swap = v & 1;
    const int rank = cluster_rank(), limb = (rank >> 1) ^ swap, h = rank & 1;
    const int ci = v / per_ct;
    const int pv = (pt_sel ? pt_sel[ci] : 0) * per_ct + v % per_ct;
    const size_t key = (size_t)(sk_of ? sk_of[ci] : 0) * L;
    {
        const LimbTab T = tabs[limb];
        const uint64_t* c0 = cts + (size_t)ci * ct_stride + ((size_t)limb << LOGN);
        const uint64_t* c1 = cts + (size_t)ci * ct_stride + ((size_t)(ct_limbs + limb) << LOGN);
        const uint64_t* s = sk + ((key + limb) << LOGN);
        const uint64_t* sp = sks + ((key + limb) << LOGN);
        const uint64_t* p = pt + (((size_t)pv * L + limb) << LOGN);
        const uint64_t* pp = pts + (((size_t)pv * L + limb) << LOGN);
        // p*(c0 + c1*s): c0 + c1*s < 5q, the product lies in [0, 4q)
        auto ld = [&](int j) { return mul_shoup4(c0[j] + mul_shoup4(c1[j], s[j], sp[j], T.q), p[j], pp[j], T.q); };
        ntt_inverse_to_smem<LOGN, false, 2>(sm, T, ld);  // ends with a cluster barrier
    }
    const uint64_t* m0 = cluster_smem(sm, (swap << 1) + h);
    const uint64_t* m1 = cluster_smem(sm, ((swap ^ 1) << 1) + h);
    double acc[MAXC];  // MAXC >= cols: 5 covers N = 16384 at d >= 1366
#pragma unroll
    for (int c = 0; c < MAXC; c++) acc[c] = 0.0;
    constexpr int Q = H / 2;  // positions per CTA
#pragma unroll 2  // (4 spilled more at 64 registers)
    for (int jq = tid; jq < Q; jq += NT) {
        const int jl = limb * Q + jq;
        const int j = h * H + jl;
        const double coeff = __dmul_rn(crt_coeff(m0[pad(jl)], m1[pad(jl)], K), inv_scale);
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
    cluster_sync();  // every CTA done reading the parked limbs; partials written
    if (rank == 0 && tid < cols) {
        double a = 0.0;
        for (int role = 0; role < 4; role++) {  // (limb, half) order, whichever rank took it
            const int r = ((((role >> 1) ^ swap) << 1) | (role & 1));
            const double* rr = cooperative_groups::this_cluster().map_shared_rank(&red[0][0], r);
            for (int w = 0; w < NT / 32; w++) a += rr[w * kMaxSegCols + tid];
        }
        seg_out[(size_t)v * cols + tid] = a;
    }
    cluster_sync();  // keep the partials alive until rank 0 has read them
}

cudaError_t launch_dec_fused(const DevCtx& c, const uint64_t* cts, long long ct_stride, int ct_limbs,
                             const uint64_t* sk, const uint64_t* sks, const int* sk_of, const uint64_t* pt,
                             const uint64_t* pts, const int* pt_sel, int per_ct,
                             int nvec, double inv_scale, const double* W, int seg_cols, uint64_t* M0, double* seg_out,
                             cudaStream_t s) {
    if (nvec <= 0) return cudaSuccess;
    if (seg_cols < 1 || seg_cols > kMaxSegCols || c.L < 2) return cudaErrorInvalidValue;
    // correction-free INTT where the modulus leaves the headroom (as in
    // ntt_inverse_block); this kernel stays integer-only (its FP64 variant
    // spilled 648 bytes and ran 15% slower)
    const bool nc0 = c.q0 < (1ULL << (61 - c.logn)), nc1 = c.q1 < (1ULL << (61 - c.logn));
    TSG_LOGN_SWITCH(c.logn, {
        // N = 8192, 16384: four-CTA clusters (LQ: other sizes never take it)
        constexpr int LQ = (LG == 13 || LG == 14) ? LG : 14;
        if (LG == 13 || LG == 14) {
            constexpr size_t smemq = (size_t)NttCfg<LQ, 2>::SMEM_WORDS * 8;
            // accumulators for at most 5 segment columns where that suffices
            auto kq = seg_cols <= 5 ? k_dec_quad<LQ, 5> : k_dec_quad<LQ, kMaxSegCols>;
            cudaError_t er = ensure_smem(kq, smemq);
            if (er != cudaSuccess) return er;
            KScope ks("dec_fused", s);
            kq<<<dim3((unsigned)nvec * 4), NttCfg<LQ, 2>::NT, smemq, s>>>(
                cts, ct_stride, ct_limbs, sk, sks, sk_of, pt, pts, pt_sel, per_ct, c.tabs, c.L, c.crt, inv_scale, W,
                seg_cols, seg_out);
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
        const double coeff = __dmul_rn(crt_coeff(m0[j], m1[j], K), inv_scale);
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
    return launch_cl(kCrtCl, k_crt_seg, dim3((unsigned)(nvec * kCrtCl)), 256, 0, s, M, c.logn, c.crt, inv_scale, W,
                     seg_cols, seg_out);
}

// ======================================================================
// ZeRo-MOAI tail: gather segment sums, B @ intermediate
// ======================================================================
__global__ void k_gather_inter(const double* __restrict__ seg, double* __restrict__ inter, int ndelta, int nb,
                               int cols, int r) {
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (long long)ndelta * r) return;
    const int i = (int)(t / r), k = (int)(t % r);
    const int b = k / cols, c = k % cols;
    inter[t] = seg[((size_t)i * nb + b) * cols + c];
}

cudaError_t launch_gather_inter(const double* seg, double* inter, int ndelta, int nb, int cols, int r, cudaStream_t s) {
    const long long tot = (long long)ndelta * r;
    if (tot <= 0) return cudaSuccess;
    KScope ks("gather_inter", s);
    k_gather_inter<<<(unsigned)((tot + 255) / 256), 256, 0, s>>>(seg, inter, ndelta, nb, cols, r);
    return cudaGetLastError();
}

// delta[i][row] = sum_k B[row][k] * inter[i][k], one FMA chain in k order.
__global__ void k_bmat(const float* __restrict__ B, const double* __restrict__ inter, double* __restrict__ delta,
                       int nvec, int d, int r, const int* __restrict__ b_sel, long long b_stride) {
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (long long)nvec * d) return;
    const int i = (int)(t / d), row = (int)(t % d);
    const float* Bm = B + (b_sel ? (long long)b_sel[i] * b_stride : 0) + (long long)row * r;
    const double* x = inter + (size_t)i * r;
    double acc = 0.0;
    for (int k = 0; k < r; k++) acc = fma((double)__ldg(Bm + k), x[k], acc);
    delta[t] = acc;
}

// The same products for small batches, one warp per output: the lanes load
// 32 consecutive k of the row (one coalesced line) and every lane runs the
// k-order FMA chain on broadcast values, so the result is bit-identical to
// k_bmat's while the loads of a row are one request instead of r.
__global__ void k_bmat_warp(const float* __restrict__ B, const double* __restrict__ inter, double* __restrict__ delta,
                            int nvec, int d, int r, const int* __restrict__ b_sel, long long b_stride) {
    const long long t = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (t >= (long long)nvec * d) return;
    const int i = (int)(t / d), row = (int)(t % d);
    const float* Bm = B + (b_sel ? (long long)b_sel[i] * b_stride : 0) + (long long)row * r;
    const double* x = inter + (size_t)i * r;
    double acc = 0.0;
    for (int k0 = 0; k0 < r; k0 += 32) {
        const int kn = r - k0 < 32 ? r - k0 : 32;
        const double bl = lane < kn ? (double)__ldg(Bm + k0 + lane) : 0.0;
        const double xl = lane < kn ? x[k0 + lane] : 0.0;
        for (int k = 0; k < kn; k++)
            acc = fma(__shfl_sync(0xffffffffu, bl, k), __shfl_sync(0xffffffffu, xl, k), acc);
    }
    if (lane == 0) delta[t] = acc;
}

cudaError_t launch_bmat(const float* B, const double* inter, double* delta, int nvec, int d, int r, const int* b_sel,
                        long long b_stride, cudaStream_t s) {
    const long long tot = (long long)nvec * d;
    if (tot <= 0) return cudaSuccess;
    KScope ks("bmat", s);
    if (tot <= 16384) {  // up to ~10 deltas: latency, not throughput
        k_bmat_warp<<<(unsigned)((tot * 32 + 255) / 256), 256, 0, s>>>(B, inter, delta, nvec, d, r, b_sel, b_stride);
    } else {
        k_bmat<<<(unsigned)((tot + 255) / 256), 256, 0, s>>>(B, inter, delta, nvec, d, r, b_sel, b_stride);
    }
    return cudaGetLastError();
}

// ======================================================================
// DP Gaussian noise (inference_engine.py:1436-1456)
// ======================================================================
__global__ void k_dp_noise(double* __restrict__ h, int d, double clip, double sigma, const uint64_t* __restrict__ seeds) {
    __shared__ double red[32];
    const int v = blockIdx.x;
    double* x = h + (size_t)v * d;
    double acc = 0.0;
    for (int j = threadIdx.x; j < d; j += blockDim.x) acc += x[j] * x[j];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
        double y = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) y += __shfl_xor_sync(0xffffffffu, y, o);
        if (threadIdx.x == 0) red[0] = y;
    }
    __syncthreads();
    const double norm = sqrt(red[0]);
    const double f = norm > clip ? clip / norm : 1.0;
    const uint64_t seed = seeds[v];
    for (int j = threadIdx.x; j < d; j += blockDim.x) {
        // Box-Muller draw j uses words 4j..4j+3 of the stream (rng.rs:152-157)
        const uint64_t w = 4ULL * j;
        uint32_t b[16];
        chacha_block(seed, (uint32_t)(w >> 4), b);
        const int o = (int)(w & 15);
        uint32_t a0 = 0, a1 = 0, a2 = 0, a3 = 0;
#pragma unroll
        for (int t = 0; t < 16; t += 4)
            if (t == o) {
                a0 = b[t];
                a1 = b[t + 1];
                a2 = b[t + 2];
                a3 = b[t + 3];
            }
        const double u1 = u64_to_unit((uint64_t)a0 | ((uint64_t)a1 << 32));
        const double u2 = u64_to_unit((uint64_t)a2 | ((uint64_t)a3 << 32));
        const double z = sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
        const double xv = norm > clip ? x[j] * f : x[j];
        x[j] = xv + z * sigma;
    }
}

cudaError_t launch_dp_noise(double* h, int nvec, int d, double clip, double sigma, const uint64_t* seeds,
                            cudaStream_t s) {
    if (nvec <= 0) return cudaSuccess;
    KScope ks("dp_noise", s);
    k_dp_noise<<<nvec, 256, 0, s>>>(h, d, clip, sigma, seeds);
    return cudaGetLastError();
}

}  // namespace tsg
