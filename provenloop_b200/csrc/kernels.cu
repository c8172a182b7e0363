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

#include "launch.cuh"

namespace cg = cooperative_groups;

namespace tsg {

namespace {

std::mutex g_attr_mu;
std::map<std::pair<const void*, int>, size_t> g_attr_done;  // (kernel, device) -> dynamic smem limit set

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


}  // namespace

cudaError_t ensure_smem_raw(const void* kernel, size_t bytes) {
    if (bytes <= 48 * 1024) return cudaSuccess;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> g(g_attr_mu);
    auto key = std::make_pair(kernel, dev);
    auto it = g_attr_done.find(key);
    if (it != g_attr_done.end() && it->second >= bytes) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) g_attr_done[key] = bytes;
    return e;
}

KScope::KScope(const char* n, cudaStream_t st, int k) : name(n), s(st), kernels(k) {
    if (g_prof_on.load(std::memory_order_relaxed)) {
        std::lock_guard<std::mutex> g(g_prof_mu);
        a = pool_event();
        b = pool_event();
        cudaEventRecord(a, s);
    }
}

KScope::~KScope() {
    g_launches.fetch_add((uint64_t)kernels, std::memory_order_relaxed);
    if (a) {
        cudaEventRecord(b, s);
        std::lock_guard<std::mutex> g(g_prof_mu);
        g_prof[name].ev.emplace_back(a, b);
    }
}

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
                e[(size_t)v * N + j0 + jj] = (int8_t)gaussian_round_e(u1, u2, &tie);
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
    if ((r & 3) == 0 && ((reinterpret_cast<uintptr_t>(B) | (uintptr_t)(b_stride * 4)) & 15) == 0) {
        // the row as 16-byte loads (a row per thread: four floats per load
        // instead of one); the same k-order FMA chain
        const float4* B4 = reinterpret_cast<const float4*>(Bm);
        for (int k4 = 0; k4 < (r >> 2); k4++) {
            const float4 b = __ldg(B4 + k4);
            acc = fma((double)b.x, x[4 * k4], acc);
            acc = fma((double)b.y, x[4 * k4 + 1], acc);
            acc = fma((double)b.z, x[4 * k4 + 2], acc);
            acc = fma((double)b.w, x[4 * k4 + 3], acc);
        }
    } else {
        for (int k = 0; k < r; k++) acc = fma((double)__ldg(Bm + k), x[k], acc);
    }
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
