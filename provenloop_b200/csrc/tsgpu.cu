// tsgpu.cu -- host side of the C ABI declared in include/tsgpu.h.
//
// Owns contexts (parameter set, tables on the device, stream, scratch),
// key / ciphertext / plaintext objects, and drives the kernels of
// kernels.cu.  Parameter and table construction restates
// tensafe-he-core/src/params.rs, rns.rs and encoding.rs (cited inline); all
// per-ciphertext arithmetic runs on the GPU.
#include <atomic>
#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/tsgpu.h"
#include "kernels.cuh"

using namespace tsg;
typedef unsigned __int128 u128;

// =====================================================================
// errors
// =====================================================================
static thread_local std::string t_err;

static int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_err = buf;
    return code;
}

static bool aligned(const void* p, size_t a) { return ((uintptr_t)p % a) == 0; }

#define CU(expr)                                                                               \
    do {                                                                                       \
        cudaError_t _e = (expr);                                                               \
        if (_e != cudaSuccess) {                                                               \
            return fail(_e == cudaErrorMemoryAllocation ? TS_ERR_OOM : TS_ERR_CUDA, "%s: %s (%s:%d)", \
                        #expr, cudaGetErrorString(_e), __FILE__, __LINE__);                    \
        }                                                                                      \
    } while (0)

// =====================================================================
// host number theory (params.rs, rns.rs)
// =====================================================================
static uint64_t mulmod(uint64_t a, uint64_t b, uint64_t q) { return (uint64_t)(((u128)a * b) % q); }

static uint64_t powmod(uint64_t b, uint64_t e, uint64_t q) {  // rns.rs:99-110
    uint64_t r = 1;
    b %= q;
    while (e) {
        if (e & 1) r = mulmod(r, b, q);
        e >>= 1;
        b = mulmod(b, b, q);
    }
    return r;
}

// Deterministic Miller-Rabin for 64-bit n (bases 2..37 are exact below
// 3.3e24).  Decides primality exactly, like the reference's trial division
// (params.rs:308-326), so the prime search returns the same prime.
static bool is_prime(uint64_t n) {
    if (n < 2) return false;
    static const uint64_t small[] = {2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37};
    for (uint64_t p : small) {
        if (n % p == 0) return n == p;
    }
    uint64_t d = n - 1;
    int s = 0;
    while ((d & 1) == 0) {
        d >>= 1;
        s++;
    }
    for (uint64_t a : small) {
        uint64_t x = powmod(a, d, n);
        if (x == 1 || x == n - 1) continue;
        bool comp = true;
        for (int r = 1; r < s; r++) {
            x = mulmod(x, x, n);
            if (x == n - 1) {
                comp = false;
                break;
            }
        }
        if (comp) return false;
    }
    return true;
}

// params.rs:169-193: largest `bits`-bit prime == 1 mod two_n, searching down.
static uint64_t find_ntt_prime(uint32_t bits, uint64_t two_n) {
    uint64_t upper = bits >= 64 ? UINT64_MAX : ((1ULL << bits) - 1);
    uint64_t lower = 1ULL << (bits - 1);
    uint64_t c = upper - (upper % two_n) + 1;
    if (c > upper) c -= two_n;
    while (c >= lower) {
        if (is_prime(c)) return c;
        c -= two_n;
        if (c < lower) break;
    }
    return 0;
}

// rns.rs:124-154: smallest g >= 2 with psi = g^((q-1)/2N) != 1 and psi^N = -1.
static uint64_t find_psi(uint64_t n, uint64_t q) {
    if (q % (2 * n) != 1) return 0;
    uint64_t e = (q - 1) / (2 * n);
    for (uint64_t g = 2; g < 10000 && g < q; g++) {
        uint64_t psi = powmod(g, e, q);
        if (psi <= 1) continue;
        if (powmod(psi, n, q) == q - 1) return psi;
    }
    return 0;
}

static uint32_t brv(uint32_t x, int bits) {
    uint32_t r = 0;
    for (int i = 0; i < bits; i++) {
        r = (r << 1) | (x & 1);
        x >>= 1;
    }
    return r;
}

static uint64_t shoup(uint64_t w, uint64_t q) { return (uint64_t)(((u128)w << 64) / q); }

static const double kPi = 3.141592653589793;  // std::f64::consts::PI

// fw[brv(i)] = psi^i, iw[brv(i)] = psi^-i (rns.rs:161-185, ntt.rs:38-65).
static bool ntt_tables(uint32_t n, uint64_t q, uint64_t* fw, uint64_t* iw) {
    const int logn = __builtin_ctz(n);
    const uint64_t psi = find_psi(n, q);
    if (!psi) return false;
    const uint64_t psi_inv = powmod(psi, q - 2, q);
    uint64_t pf = 1, pi = 1;
    for (uint32_t i = 0; i < n; i++) {
        const uint32_t r = brv(i, logn);
        fw[r] = pf;
        iw[r] = pi;
        pf = mulmod(pf, psi, q);
        pi = mulmod(pi, psi_inv, q);
    }
    return true;
}

// FFT tables (encoding.rs:38-80), same expressions and glibc cos/sin.
static void fft_tables(uint32_t n, double* twist_re, double* twist_im, double* tw_re, double* tw_im) {
    const int logn = __builtin_ctz(n);
    for (uint32_t j = 0; j < n; j++) {
        volatile double angle = kPi * (double)j / (double)n;
        twist_re[j] = cos(angle);
        twist_im[j] = sin(angle);
    }
    tw_re[0] = tw_im[0] = 0.0;
    for (int s = 0; s < logn; s++) {
        const uint32_t half = 1u << s;
        for (uint32_t k = 0; k < half; k++) {
            volatile double angle = -2.0 * kPi * (double)k / (double)(2 * half);
            tw_re[half + k] = cos(angle);
            tw_im[half + k] = sin(angle);
        }
    }
}

namespace tsg_host {
void noalloc_prepare(int device);  // noalloc.cu
}

// =====================================================================
// objects
// =====================================================================
struct ts_ctx {
    std::mutex mu;
    // One reference for the context handle and one per live key, public key,
    // ciphertext, plaintext and adapter object: the context's memory is
    // released when the last of them is destroyed, in whatever order that
    // happens (a garbage collector may destroy a context before its objects).
    std::atomic<int> refs{1};
    int device = 0;
    uint32_t n = 0, slots = 0, L = 0, scale_bits = 40;
    int logn = 0;
    uint64_t q[kMaxLimbs] = {};
    // host copies of the tables (tests / export)
    std::vector<uint64_t> h_fw, h_iw;  // [L][n]
    std::vector<double> h_twist_re, h_twist_im, h_tw_re, h_tw_im;
    // device
    uint64_t* d_tw = nullptr;  // [L][8][n]: integer (w, w') pairs, then FP64 (w, w/q) pairs, forward then inverse
    LimbTab* d_tabs = nullptr;
    double* d_fft = nullptr;   // [4][n]
    unsigned long long* d_stats = nullptr;
    DevCtx dc{};
    cudaStream_t own = nullptr, stream = nullptr;
    // second stream and fork / join events of the small-batch encryption,
    // and a third stream for the decrypt side's code warm-up; created by
    // their first use
    cudaStream_t side = nullptr, warm = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr, ev_gauss = nullptr, ev_warm0 = nullptr, ev_warm1 = nullptr;
    // copy streams and events of the pipelined host-buffer delta path: the
    // H2D of chunk k+1 and the D2H of chunk k-1 overlap chunk k's kernels
    cudaStream_t s_h2d = nullptr, s_d2h = nullptr;
    cudaEvent_t ev_start = nullptr, ev_h2d[2] = {}, ev_comp[2] = {}, ev_d2h[2] = {};
    // grow-only scratch
    void* scratch = nullptr;
    size_t scratch_bytes = 0;
    // Ring of pinned staging slots for the small per-call inputs (seeds,
    // indexes).  A call takes the next slot and waits only until that slot's
    // previous copy has left it, so back-to-back calls (one per layer of a
    // decode step) do not wait for the GPU.
    static constexpr int kPinnedSlots = 8;
    void* pinned[kPinnedSlots] = {};
    size_t pinned_bytes[kPinnedSlots] = {};
    cudaEvent_t pinned_free[kPinnedSlots] = {};  // recorded after the copy out of the slot
    int pinned_next = 0;
};

struct ts_sk {
    ts_ctx* ctx;
    uint32_t count;
    uint64_t* d;  // [count][L][n] residues, then [count][L][n] Shoup companions
};

// Shoup companions of a key set (floor(s * 2^64 / q_l) per coefficient).
static const uint64_t* sk_shoup(const ts_sk* sk) { return sk->d + (size_t)sk->count * sk->ctx->L * sk->ctx->n; }

struct ts_pk {
    ts_ctx* ctx;
    uint64_t* d;  // [2][L][n] = (b, a), NTT domain, then [2][L][n] Shoup companions
};

struct ts_ct {
    ts_ctx* ctx;
    uint32_t count, limbs;
    double scale;
    uint64_t* d;  // [count][2][limbs][n]
};

struct ts_pt {
    ts_ctx* ctx;
    uint32_t count;
    uint64_t* d;  // [count][L][n]
};

struct ts_lora {
    ts_ctx* ctx;
    uint32_t experts, r, d, cols, batches;
    uint64_t* d_pt;  // [experts][batches][L][n] residues, then as many Shoup companions
    float* d_b;      // [experts][d][r]
    double* d_w;     // [cols][n] segment functionals, or null (cols > kMaxSegCols)
};

namespace {

struct Lock {
    std::lock_guard<std::mutex> g;
    explicit Lock(ts_ctx* c) : g(c->mu) {}
};

int set_device(ts_ctx* c) {
    CU(cudaSetDevice(c->device));
    return TS_OK;
}

// Carve aligned sub-buffers out of the context's grow-only scratch.
struct Carve {
    std::vector<size_t> sizes;
    size_t add(size_t bytes) {
        sizes.push_back((bytes + 255) & ~(size_t)255);
        return sizes.size() - 1;
    }
    size_t total() const {
        size_t t = 0;
        for (size_t s : sizes) t += s;
        return t;
    }
    template <class T>
    T* at(void* base, size_t idx) const {
        size_t off = 0;
        for (size_t i = 0; i < idx; i++) off += sizes[i];
        return reinterpret_cast<T*>(static_cast<char*>(base) + off);
    }
};

int ensure_scratch(ts_ctx* c, size_t bytes) {
    if (bytes <= c->scratch_bytes) return TS_OK;
    if (c->scratch) {
        CU(cudaFreeAsync(c->scratch, c->stream));
        c->scratch = nullptr;
        c->scratch_bytes = 0;
    }
    size_t want = bytes + bytes / 4;
    CU(cudaMallocAsync(&c->scratch, want, c->stream));
    c->scratch_bytes = want;
    return TS_OK;
}

// Pinned staging buffer for small per-call inputs; waits until the previous
// asynchronous copy out of it has executed before it is reused.
// Next pinned staging slot of at least `bytes`; *slot receives its index.
// The caller records pinned_free[*slot] after its copy out of the slot.
int ensure_pinned(ts_ctx* c, size_t bytes, int* slot) {
    const int k = c->pinned_next;
    c->pinned_next = (k + 1) % ts_ctx::kPinnedSlots;
    if (!c->pinned_free[k]) CU(cudaEventCreateWithFlags(&c->pinned_free[k], cudaEventDisableTiming));
    CU(cudaEventSynchronize(c->pinned_free[k]));
    *slot = k;
    if (bytes <= c->pinned_bytes[k]) return TS_OK;
    if (c->pinned[k]) {
        CU(cudaFreeHost(c->pinned[k]));
        c->pinned[k] = nullptr;
        c->pinned_bytes[k] = 0;
    }
    CU(cudaMallocHost(&c->pinned[k], bytes));
    c->pinned_bytes[k] = bytes;
    return TS_OK;
}

int dev_alloc(ts_ctx* c, void** p, size_t bytes) {
    cudaError_t e = cudaMallocAsync(p, bytes, c->stream);
    if (e != cudaSuccess) return fail(TS_ERR_OOM, "device allocation of %zu bytes failed: %s", bytes, cudaGetErrorString(e));
    return TS_OK;
}

SegList encrypt_segs(uint32_t L) {
    SegList s{};
    for (uint32_t l = 0; l < L; l++) {
        s.kind[s.count] = SEG_UNIFORM;
        s.limb[s.count] = (int)l;
        s.count++;
    }
    s.kind[s.count++] = SEG_GAUSS;
    return s;
}

int build_ctx(uint32_t n, const uint64_t* moduli, uint32_t L, uint32_t scale_bits, int device, ts_ctx** out) {
    if (!out) return fail(TS_ERR_ARG, "out is NULL");
    *out = nullptr;
    if (n < 1024 || n > 32768 || (n & (n - 1)))
        return fail(TS_ERR_UNSUPPORTED, "Unsupported poly_mod_degree: %u (this build supports 1024..32768)", n);
    if (L < 1 || L > (uint32_t)kMaxLimbs) return fail(TS_ERR_ARG, "num_limbs %u out of range [1, %d]", L, kMaxLimbs);
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return fail(TS_ERR_NODEVICE, "no CUDA device");
    if (device < 0 || device >= ndev) return fail(TS_ERR_ARG, "device %d out of range (%d devices)", device, ndev);
    ts_ctx* c = new ts_ctx();
    c->device = device;
    c->n = n;
    c->slots = n / 2;
    c->L = L;
    c->scale_bits = scale_bits;
    c->logn = __builtin_ctz(n);
    const int logn = c->logn;
    std::vector<LimbTab> tabs(L);
    std::vector<uint64_t> tw((size_t)L * 8 * n);
    c->h_fw.assign((size_t)L * n, 0);
    c->h_iw.assign((size_t)L * n, 0);
    for (uint32_t l = 0; l < L; l++) {
        const uint64_t q = moduli[l];
        // the lazy NTT keeps values below 8q < 2^64
        if (q < 3 || q >= (1ULL << 61) || q % (2 * n) != 1) {
            delete c;
            return fail(TS_ERR_ARG, "modulus %llu is not an NTT-friendly prime below 2^61 for N=%u",
                        (unsigned long long)q, n);
        }
        c->q[l] = q;
        uint64_t* fw = c->h_fw.data() + (size_t)l * n;
        uint64_t* iw = c->h_iw.data() + (size_t)l * n;
        if (!ntt_tables(n, q, fw, iw)) {
            delete c;
            return fail(TS_ERR_ARG, "no primitive 2N-th root for q=%llu", (unsigned long long)q);
        }
        // device layout per limb: (fw, fw') pairs, then (iw, iw') pairs; then
        // the FP64 mode's (w, w/q) pairs with w balanced into (-q/2, q/2]
        uint64_t* dst = tw.data() + (size_t)l * 8 * n;
        const double qd = (double)q;
        auto bal = [q](uint64_t w) { return w > q / 2 ? (double)(int64_t)(w - q) : (double)w; };
        auto put = [](uint64_t* d, double x) { memcpy(d, &x, 8); };
        for (uint32_t i = 0; i < n; i++) {
            dst[2 * i] = fw[i];
            dst[2 * i + 1] = shoup(fw[i], q);
            dst[2 * (size_t)n + 2 * i] = iw[i];
            dst[2 * (size_t)n + 2 * i + 1] = shoup(iw[i], q);
            put(dst + 4 * (size_t)n + 2 * i, bal(fw[i]));
            put(dst + 4 * (size_t)n + 2 * i + 1, bal(fw[i]) / qd);
            put(dst + 6 * (size_t)n + 2 * i, bal(iw[i]));
            put(dst + 6 * (size_t)n + 2 * i + 1, bal(iw[i]) / qd);
        }
        LimbTab& T = tabs[l];
        T.q = q;
        T.ninv = powmod(n, q - 2, q);  // ntt.rs:48
        T.ninvs = shoup(T.ninv, q);
        T.iw1n = mulmod(iw[1], T.ninv, q);  // last inverse stage twiddle with N^-1 folded in
        T.iw1ns = shoup(T.iw1n, q);
        T.mu64 = UINT64_MAX / q;
        T.bk = 64 - __builtin_clzll(q);
        T.bmu = (uint64_t)(((u128)1 << (2 * T.bk)) / q);
        T.thresh = (uint64_t)(((u128)1 << 64) % q);  // (u64::MAX - q + 1) % q, rng.rs:126
        T.fp = q < (1ULL << 44) ? 2 : q < (1ULL << 50) ? 1 : 0;  // 2: the lazy FP64 mode
    }
    c->h_twist_re.assign(n, 0.0);
    c->h_twist_im.assign(n, 0.0);
    c->h_tw_re.assign(n, 0.0);
    c->h_tw_im.assign(n, 0.0);
    fft_tables(n, c->h_twist_re.data(), c->h_twist_im.data(), c->h_tw_re.data(), c->h_tw_im.data());
    // CRT constants (ciphertext.rs:351-356)
    CrtConst K{};
    if (L >= 2) {
        const uint64_t q0 = c->q[0], q1 = c->q[1];
        K.q0 = q0;
        K.q1 = q1;
        K.mu64_1 = tabs[1].mu64;
        K.bmu1 = tabs[1].bmu;
        K.bk1 = tabs[1].bk;
        K.q0inv = powmod(q0 % q1, q1 - 2, q1);
        K.q0inv_s = (uint64_t)(((u128)K.q0inv << 64) / q1);
        const u128 Q = (u128)q0 * q1;
        const u128 H = Q / 2;
        K.Q_lo = (uint64_t)Q;
        K.Q_hi = (uint64_t)(Q >> 64);
        K.H_lo = (uint64_t)H;
        K.H_hi = (uint64_t)(H >> 64);
        if (q1 < (1ULL << 50)) {  // the FP64 form needs exact products mod q1
            auto bal = [q1](uint64_t w) { return w > q1 / 2 ? -(double)(q1 - w) : (double)w; };
            K.q1d = (double)q1;
            K.r30 = bal((1ULL << 30) % q1);
            K.r30q = K.r30 / K.q1d;
            K.q0invd = bal(K.q0inv);
            K.q0invq = K.q0invd / K.q1d;
            K.t_half = (double)((q1 - 1) / 2);
            K.q0_hi = (double)q0;
            K.q0_lo = (double)(int64_t)(q0 - (uint64_t)K.q0_hi);  // |q0 - fl(q0)| <= 2^7
            K.q0_half = q0 / 2;
        }
    } else {
        K.q0 = c->q[0];
    }
    // device upload
    int rc = TS_OK;
    do {
        cudaError_t e = cudaSetDevice(device);
        if (e != cudaSuccess) { rc = fail(TS_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(e)); break; }
        // keep freed stream-ordered allocations in the pool for reuse
        cudaMemPool_t pool;
        if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
            uint64_t thr = UINT64_MAX;
            cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
        }
        e = cudaStreamCreateWithFlags(&c->own, cudaStreamNonBlocking);
        if (e != cudaSuccess) { rc = fail(TS_ERR_CUDA, "stream: %s", cudaGetErrorString(e)); break; }
        c->stream = c->own;
        if (cudaMalloc(&c->d_tw, tw.size() * 8) != cudaSuccess || cudaMalloc(&c->d_tabs, L * sizeof(LimbTab)) != cudaSuccess ||
            cudaMalloc(&c->d_fft, (size_t)4 * n * sizeof(double)) != cudaSuccess ||
            cudaMalloc(&c->d_stats, STAT_COUNT * sizeof(unsigned long long)) != cudaSuccess) {
            rc = fail(TS_ERR_OOM, "table allocation failed");
            break;
        }
        for (uint32_t l = 0; l < L; l++) tabs[l].tw = c->d_tw + (size_t)l * 8 * n;
        cudaMemcpy(c->d_tw, tw.data(), tw.size() * 8, cudaMemcpyHostToDevice);
        cudaMemcpy(c->d_tabs, tabs.data(), L * sizeof(LimbTab), cudaMemcpyHostToDevice);
        cudaMemcpy(c->d_fft, c->h_twist_re.data(), n * 8, cudaMemcpyHostToDevice);
        cudaMemcpy(c->d_fft + n, c->h_twist_im.data(), n * 8, cudaMemcpyHostToDevice);
        cudaMemcpy(c->d_fft + 2 * (size_t)n, c->h_tw_re.data(), n * 8, cudaMemcpyHostToDevice);
        cudaMemcpy(c->d_fft + 3 * (size_t)n, c->h_tw_im.data(), n * 8, cudaMemcpyHostToDevice);
        cudaMemset(c->d_stats, 0, STAT_COUNT * sizeof(unsigned long long));
        e = cudaDeviceSynchronize();
        if (e != cudaSuccess) { rc = fail(TS_ERR_CUDA, "table upload: %s", cudaGetErrorString(e)); break; }
        // load ts_decrypt_noalloc's fixed array on this device now (lazy
        // module loading would otherwise allocate it at its first call)
        tsg_host::noalloc_prepare(device);
    } while (0);
    if (rc != TS_OK) {
        ts_ctx_destroy(c);
        return rc;
    }
    c->dc.logn = logn;
    c->dc.q0 = c->q[0];
    c->dc.encode_cluster = encode_cluster_supported(logn) ? 1 : 0;
    c->dc.q1 = L >= 2 ? c->q[1] : 0;
    c->dc.sms = 148;
    {
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, c->device) == cudaSuccess && sms > 0)
            c->dc.sms = sms;
    }
    c->dc.n = (int)n;
    c->dc.L = (int)L;
    c->dc.tabs = c->d_tabs;
    c->dc.fft.twist_re = c->d_fft;
    c->dc.fft.twist_im = c->d_fft + n;
    c->dc.fft.tw_re = c->d_fft + 2 * (size_t)n;
    c->dc.fft.tw_im = c->d_fft + 3 * (size_t)n;
    c->dc.scale = 1099511627776.0;
    c->dc.crt = K;
    c->dc.stats = c->d_stats;
    *out = c;
    return TS_OK;
}

// H2D of a row-strided host matrix (rows x len doubles) into dst [rows][len].
int h2d_rows(ts_ctx* c, double* dst, const double* src, size_t rows, size_t len, size_t stride) {
    if (rows == 0 || len == 0) return TS_OK;
    CU(cudaMemcpy2DAsync(dst, len * 8, src, stride * 8, len * 8, rows, cudaMemcpyHostToDevice, c->stream));
    return TS_OK;
}

template <class T>
int h2d_small(ts_ctx* c, T* dst, const T* src, size_t count) {
    if (count == 0) return TS_OK;
    CU(cudaMemcpyAsync(dst, src, count * sizeof(T), cudaMemcpyHostToDevice, c->stream));
    return TS_OK;
}

int check_stats(ts_ctx* c) {
    unsigned long long st[STAT_COUNT];
    CU(cudaMemcpyAsync(st, c->d_stats, sizeof(st), cudaMemcpyDeviceToHost, c->stream));
    CU(cudaStreamSynchronize(c->stream));
    if (st[STAT_PLAN_FAIL])
        return fail(TS_ERR_STATE, "a sampling stream rejected more than %d candidates in one segment", kMaxRej);
    return TS_OK;
}

// Work buffers of one encryption pass over up to `cap` vectors.
struct EncWork {
    int64_t* m;       // [cap][n] rounded coefficients
    int8_t* e;        // [cap][n] Gaussian error
    double* f;        // [cap][2][n] FFT scratch
    uint32_t* fl;     // [cap] rejection flags
    StreamPlan* pl;   // [cap] exact stream plans
    size_t cap;
};

void carve_enc(Carve& cv, size_t cap, size_t n, size_t idx[5]) {
    idx[0] = cv.add(cap * n * 8);
    idx[1] = cv.add(cap * n);
    idx[2] = cv.add(cap * 2 * n * 8);
    idx[3] = cv.add((2 * cap + 1) * 4);
    idx[4] = cv.add(cap * sizeof(StreamPlan));
}

EncWork enc_work(const Carve& cv, void* base, size_t cap, const size_t idx[5]) {
    return EncWork{cv.at<int64_t>(base, idx[0]), cv.at<int8_t>(base, idx[1]), cv.at<double>(base, idx[2]),
                   cv.at<uint32_t>(base, idx[3]), cv.at<StreamPlan>(base, idx[4]), cap};
}

// The side streams and events of the small-batch forms (first use).
int ensure_side_streams(ts_ctx* c) {
    if (c->side) return TS_OK;
    CU(cudaStreamCreateWithFlags(&c->warm, cudaStreamNonBlocking));
    for (cudaEvent_t* e : {&c->ev_fork, &c->ev_join, &c->ev_gauss, &c->ev_warm0, &c->ev_warm1})
        CU(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
    CU(cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking));
    return TS_OK;
}

// The copy streams and events of the pipelined host-buffer delta path
// (first use).
int ensure_copy_streams(ts_ctx* c) {
    if (c->s_h2d) return TS_OK;
    for (cudaEvent_t* e : {&c->ev_start, &c->ev_h2d[0], &c->ev_h2d[1], &c->ev_comp[0], &c->ev_comp[1], &c->ev_d2h[0],
                           &c->ev_d2h[1]})
        CU(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
    CU(cudaStreamCreateWithFlags(&c->s_d2h, cudaStreamNonBlocking));
    CU(cudaStreamCreateWithFlags(&c->s_h2d, cudaStreamNonBlocking));
    return TS_OK;
}

// Core of every secret-key encryption: `count` vectors already on the device
// (SlotSrc), seeds / key indexes on the device, output ct [count][2][L][n].
// Uses only the work buffers in `w` (callers own the scratch layout).
// `warm` (optional) lists tables the caller's later kernels read; in the
// small-batch branch they are prefetched into L2 on the side stream ahead of
// c1 = NTT(a), together with the encryption's own tables.
int encrypt_core(ts_ctx* c, const SlotSrc& src, size_t count, const uint64_t* d_seeds, const int* d_skof,
                 const uint64_t* d_sk, const uint64_t* d_sks, uint64_t* d_ct, const EncWork& w,
                 const L2List* warm = nullptr) {
    const size_t n = c->n;
    for (size_t v0 = 0; v0 < count; v0 += w.cap) {
        const size_t nv = count - v0 < w.cap ? count - v0 : w.cap;
        SlotSrc s = src;
        s.src = static_cast<const char*>(src.src) + (size_t)v0 * src.stride * (src.is_f32 ? 4 : 8);
        const uint64_t* seeds = d_seeds + v0;
        const int* skof = d_skof ? d_skof + v0 : nullptr;
        uint64_t* ct = d_ct + v0 * 2 * c->L * n;
        CU(cudaMemsetAsync(w.fl, 0, (2 * nv + 1) * 4, c->stream));
        const int cl = c->logn >= 15 ? 2 : 1;
        if ((int)(nv * c->L * cl * 2) <= c->dc.sms) {
            // small batch (a decode step): latency, not throughput, matters.
            // c1 = NTT(a) runs on a side stream while the encode and
            // NTT(m + e) run on the context's stream; c0 -= c1*s after the join
            if (int rc = ensure_side_streams(c)) return rc;
            CU(cudaEventRecord(c->ev_fork, c->stream));
            CU(cudaStreamWaitEvent(c->side, c->ev_fork, 0));
            {
                // NTT twiddles, FFT tables and the key(s), then the caller's
                L2List pl = warm ? *warm : L2List{};
                const int room = kMaxL2Ranges - pl.n;
                if (room >= 4) {
                    const long long limb = (long long)n * 8;
                    pl.r[pl.n++] = L2Range{c->d_fft, nullptr, 0, 0, 1, 1, 0, 4 * limb};
                    // the small-batch kernels below N = 32768 are integer-only:
                    // their half of each limb's tables
                    pl.r[pl.n++] = c->logn >= 15 ? L2Range{c->d_tw, nullptr, 0, 0, 1, 1, 0, 8 * (long long)c->L * limb}
                                                 : L2Range{c->d_tw, nullptr, 0, 0, 1, (int)c->L, 8 * limb, 4 * limb};
                    if (!d_skof) {  // one key for the whole batch
                        pl.r[pl.n++] = L2Range{d_sk, nullptr, 0, 0, 1, 1, 0, (long long)c->L * limb};
                        pl.r[pl.n++] = L2Range{d_sks, nullptr, 0, 0, 1, 1, 0, (long long)c->L * limb};
                    }
                }
                CU(launch_prefetch_l2(pl, c->side));
            }
            // the Gaussian error (words 2LN.. of each stream) on the side
            // stream too, off the encode's critical path
            CU(launch_gauss_gen(c->dc, w.e, seeds, (int)nv, 2ULL * c->L * n, c->side));
            CU(cudaEventRecord(c->ev_gauss, c->side));
            CU(launch_encode(c->dc, s, (int)nv, w.m, nullptr, seeds, 0, w.f, c->stream));
            CU(cudaStreamWaitEvent(c->stream, c->ev_gauss, 0));
            CU(launch_encrypt_split(c->dc, ct, w.m, w.e, d_sk, d_sks, skof, seeds, (int)nv, w.fl, w.pl, c->side,
                                    c->stream));
            CU(cudaEventRecord(c->ev_join, c->side));
            CU(cudaStreamWaitEvent(c->stream, c->ev_join, 0));
            CU(launch_enc_combine(c->dc, ct, d_sk, d_sks, skof, (int)nv, c->stream));
        } else {
            // the Gaussian error (words 2LN.. of each stream) in its own
            // kernel: ChaCha20 and Box-Muller at full occupancy, where the
            // encode's FFT holds one CTA per SM
            CU(launch_encode(c->dc, s, (int)nv, w.m, nullptr, seeds, 0, w.f, c->stream));
            CU(launch_gauss_gen(c->dc, w.e, seeds, (int)nv, 2ULL * c->L * n, c->stream));
            CU(launch_encrypt_limbs(c->dc, ct, w.m, w.e, d_sk, d_sks, skof, seeds, (int)nv, w.fl, w.pl, false,
                                    c->stream));
        }
        // exact repair of the (rare) streams that met a rejection
        CU(launch_plan(c->dc, seeds, (int)nv, w.fl, w.pl, encrypt_segs(c->L), c->stream));
        CU(launch_gauss_fix(c->dc, w.e, seeds, (int)nv, w.fl, w.pl, (int)c->L, c->stream));
        CU(launch_encrypt_limbs(c->dc, ct, w.m, w.e, d_sk, d_sks, skof, seeds, (int)nv, w.fl, w.pl, true, c->stream));
    }
    return TS_OK;
}

int new_ct(ts_ctx* c, uint32_t count, uint32_t limbs, double scale, ts_ct** out) {
    ts_ct* ct = new ts_ct{c, count, limbs, scale, nullptr};
    int rc = dev_alloc(c, (void**)&ct->d, (size_t)count * 2 * limbs * c->n * 8);
    if (rc) {
        delete ct;
        return rc;
    }
    *out = ct;
    return TS_OK;
}

}  // namespace

// =====================================================================
// C ABI
// =====================================================================
extern "C" {

const char* ts_last_error(void) { return t_err.c_str(); }

int ts_launch_count(uint64_t* out) {
    if (!out) return fail(TS_ERR_ARG, "out is NULL");
    *out = launch_count();
    return TS_OK;
}

int ts_profile_enable(int on) {
    prof_enable(on != 0);
    return TS_OK;
}

int ts_profile_reset(void) {
    prof_reset();
    return TS_OK;
}

int ts_profile_read(const char* kernel, double* ms, uint64_t* launches) {
    if (!kernel || !ms || !launches) return fail(TS_ERR_ARG, "NULL argument");
    if (!prof_read(kernel, ms, launches)) return fail(TS_ERR_ARG, "kernel %s was not profiled", kernel);
    return TS_OK;
}

int ts_params_custom(uint32_t poly_degree, const uint32_t* bits, uint32_t L, uint64_t* out) {
    if (!bits || !out || L == 0) return fail(TS_ERR_ARG, "bad arguments");
    if (poly_degree == 0 || (poly_degree & (poly_degree - 1))) return fail(TS_ERR_ARG, "poly_degree must be a power of 2");
    for (uint32_t i = 0; i < L; i++) {
        if (bits[i] < 2 || bits[i] > 61) return fail(TS_ERR_ARG, "modulus width %u unsupported (2..61)", bits[i]);
        out[i] = find_ntt_prime(bits[i], 2ULL * poly_degree);
        if (!out[i]) return fail(TS_ERR_ARG, "No %u-bit NTT-friendly prime found for 2N=%u", bits[i], 2 * poly_degree);
    }
    return TS_OK;
}

int ts_host_tables(uint32_t n, uint64_t q, uint64_t* fw, uint64_t* iw, double* twr, double* twi, double* tr,
                   double* ti) {
    if (n < 4 || (n & (n - 1))) return fail(TS_ERR_ARG, "n must be a power of 2 >= 4");
    if (fw || iw) {
        std::vector<uint64_t> a(n), b(n);
        if (!ntt_tables(n, q, a.data(), b.data()))
            return fail(TS_ERR_ARG, "q=%llu is not NTT-friendly for N=%u", (unsigned long long)q, n);
        if (fw) memcpy(fw, a.data(), n * 8);
        if (iw) memcpy(iw, b.data(), n * 8);
    }
    if (twr || twi || tr || ti) {
        std::vector<double> A(n), B(n), Cc(n), D(n);
        fft_tables(n, A.data(), B.data(), Cc.data(), D.data());
        if (twr) memcpy(twr, A.data(), n * 8);
        if (twi) memcpy(twi, B.data(), n * 8);
        if (tr) memcpy(tr, Cc.data(), n * 8);
        if (ti) memcpy(ti, D.data(), n * 8);
    }
    return TS_OK;
}

int ts_version(void) { return 10000; }

int ts_device_count(int* out) {
    if (!out) return fail(TS_ERR_ARG, "out is NULL");
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) n = 0;
    *out = n;
    return TS_OK;
}

int ts_ctx_create(uint32_t poly_mod_degree, int device, ts_ctx** out) {
    // params.rs:66-126
    static const uint64_t p8192[4] = {1152921504606830593ULL, 1099511480321ULL, 1099510890497ULL,
                                      1152921504606601217ULL};
    static const uint64_t p16384[4] = {1152921504606748673ULL, 1099510054913ULL, 1099508121601ULL,
                                       1152921504606683137ULL};
    static const uint64_t p32768[4] = {1152921504606584833ULL, 1099507695617ULL, 1099506515969ULL,
                                       1152921504598720513ULL};
    const uint64_t* p = nullptr;
    switch (poly_mod_degree) {
        case 8192: p = p8192; break;
        case 16384: p = p16384; break;
        case 32768: p = p32768; break;
        default:
            return fail(TS_ERR_UNSUPPORTED, "Unsupported poly_mod_degree: %u. Use 8192, 16384, or 32768.",
                        poly_mod_degree);
    }
    return build_ctx(poly_mod_degree, p, 4, 40, device, out);
}

int ts_ctx_create_custom(uint32_t poly_degree, const uint32_t* modulus_bits, uint32_t num_limbs, uint32_t scale_bits,
                         int device, ts_ctx** out) {
    if (!modulus_bits || num_limbs == 0 || num_limbs > (uint32_t)kMaxLimbs)
        return fail(TS_ERR_ARG, "bad modulus_bits / num_limbs");
    if (poly_degree == 0 || (poly_degree & (poly_degree - 1))) return fail(TS_ERR_ARG, "poly_degree must be a power of 2");
    uint64_t q[kMaxLimbs];
    for (uint32_t i = 0; i < num_limbs; i++) {
        if (modulus_bits[i] < 2 || modulus_bits[i] > 61)
            return fail(TS_ERR_ARG, "modulus width %u unsupported (2..61)", modulus_bits[i]);
        q[i] = find_ntt_prime(modulus_bits[i], 2ULL * poly_degree);
        if (!q[i])
            return fail(TS_ERR_ARG, "No %u-bit NTT-friendly prime found for 2N=%u", modulus_bits[i], 2 * poly_degree);
    }
    return build_ctx(poly_degree, q, num_limbs, scale_bits, device, out);
}

int ts_ctx_create_moduli(uint32_t poly_degree, const uint64_t* moduli, uint32_t num_limbs, int device, ts_ctx** out) {
    if (!moduli) return fail(TS_ERR_ARG, "moduli is NULL");
    return build_ctx(poly_degree, moduli, num_limbs, 40, device, out);
}

}  // extern "C"

namespace {

void ctx_free(ts_ctx* c) {
    cudaSetDevice(c->device);
    if (c->own) cudaStreamSynchronize(c->own);
    if (c->stream && c->stream != c->own) cudaStreamSynchronize(c->stream);
    if (c->scratch) cudaFree(c->scratch);
    for (int k = 0; k < ts_ctx::kPinnedSlots; k++) {
        if (c->pinned[k]) cudaFreeHost(c->pinned[k]);
        if (c->pinned_free[k]) cudaEventDestroy(c->pinned_free[k]);
    }
    cudaFree(c->d_tw);
    cudaFree(c->d_tabs);
    cudaFree(c->d_fft);
    cudaFree(c->d_stats);
    for (cudaStream_t st : {c->side, c->warm, c->s_h2d, c->s_d2h})
        if (st) {
            cudaStreamSynchronize(st);
            cudaStreamDestroy(st);
        }
    for (cudaEvent_t e : {c->ev_fork, c->ev_join, c->ev_gauss, c->ev_warm0, c->ev_warm1, c->ev_start, c->ev_h2d[0],
                          c->ev_h2d[1], c->ev_comp[0], c->ev_comp[1], c->ev_d2h[0], c->ev_d2h[1]})
        if (e) cudaEventDestroy(e);
    if (c->own) cudaStreamDestroy(c->own);
    delete c;
}

}  // namespace

// Reference bookkeeping of child objects (see ts_ctx::refs).
template <class T>
T* ctx_adopt(T* o) {
    o->ctx->refs.fetch_add(1);
    return o;
}

void ctx_release(ts_ctx* c) {
    if (c->refs.fetch_sub(1) == 1) ctx_free(c);
}

extern "C" {

int ts_ctx_destroy(ts_ctx* c) {
    if (!c) return TS_OK;
    ctx_release(c);
    return TS_OK;
}

int ts_ctx_info(const ts_ctx* c, uint32_t* n, uint32_t* slots, uint32_t* L, uint64_t* moduli) {
    if (!c) return fail(TS_ERR_ARG, "ctx is NULL");
    if (n) *n = c->n;
    if (slots) *slots = c->slots;
    if (L) *L = c->L;
    if (moduli)
        for (uint32_t l = 0; l < c->L; l++) moduli[l] = c->q[l];
    return TS_OK;
}

int ts_ctx_get_stream(ts_ctx* c, void** s) {
    if (!c || !s) return fail(TS_ERR_ARG, "NULL argument");
    *s = (void*)c->stream;
    return TS_OK;
}

int ts_ctx_set_stream(ts_ctx* c, void* s) {
    if (!c) return fail(TS_ERR_ARG, "ctx is NULL");
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    CU(cudaStreamSynchronize(c->stream));
    c->stream = (cudaStream_t)s;  // 0 is the legacy default stream
    return TS_OK;
}

int ts_ctx_reset_stream(ts_ctx* c) {
    if (!c) return fail(TS_ERR_ARG, "ctx is NULL");
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    CU(cudaStreamSynchronize(c->stream));
    c->stream = c->own;
    return TS_OK;
}

int ts_ctx_synchronize(ts_ctx* c) {
    if (!c) return fail(TS_ERR_ARG, "ctx is NULL");
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    return check_stats(c);
}

int ts_ctx_stats(ts_ctx* c, uint64_t out[4]) {
    if (!c || !out) return fail(TS_ERR_ARG, "NULL argument");
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    unsigned long long st[STAT_COUNT];
    CU(cudaMemcpyAsync(st, c->d_stats, sizeof(st), cudaMemcpyDeviceToHost, c->stream));
    CU(cudaStreamSynchronize(c->stream));
    for (int i = 0; i < 4; i++) out[i] = st[i];
    return TS_OK;
}

int ts_ctx_tables(const ts_ctx* c, uint32_t limb, uint64_t* fw, uint64_t* iw, double* twr, double* twi, double* tr,
                  double* ti) {
    if (!c || limb >= c->L) return fail(TS_ERR_ARG, "bad ctx / limb");
    const size_t n = c->n;
    if (fw) memcpy(fw, c->h_fw.data() + limb * n, n * 8);
    if (iw) memcpy(iw, c->h_iw.data() + limb * n, n * 8);
    if (twr) memcpy(twr, c->h_twist_re.data(), n * 8);
    if (twi) memcpy(twi, c->h_twist_im.data(), n * 8);
    if (tr) memcpy(tr, c->h_tw_re.data(), n * 8);
    if (ti) memcpy(ti, c->h_tw_im.data(), n * 8);
    return TS_OK;
}

// ------------------------------------------------------------------ keys
int ts_keygen_batch(ts_ctx* c, const uint64_t* seeds, uint32_t count, ts_sk** out) {
    if (!c || !seeds || !out || count == 0) return fail(TS_ERR_ARG, "bad arguments to ts_keygen_batch");
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    ts_sk* sk = new ts_sk{c, count, nullptr};
    rc = dev_alloc(c, (void**)&sk->d, 2 * (size_t)count * c->L * c->n * 8);
    if (rc) {
        delete sk;
        return rc;
    }
    Carve cv;
    const size_t i_s = cv.add(count * 8), i_f = cv.add((2 * (size_t)count + 1) * 4),
                 i_p = cv.add(count * sizeof(StreamPlan));
    rc = ensure_scratch(c, cv.total());
    if (rc) {
        cudaFreeAsync(sk->d, c->stream);
        delete sk;
        return rc;
    }
    uint64_t* ds = cv.at<uint64_t>(c->scratch, i_s);
    uint32_t* fl = cv.at<uint32_t>(c->scratch, i_f);
    StreamPlan* pl = cv.at<StreamPlan>(c->scratch, i_p);
    SegList segs{};
    segs.count = 1;
    segs.kind[0] = SEG_TERNARY;
    rc = h2d_small(c, ds, seeds, count);
    if (!rc) {
        cudaError_t e = cudaMemsetAsync(fl, 0, (2 * (size_t)count + 1) * 4, c->stream);
        if (e == cudaSuccess) e = launch_keygen(c->dc, sk->d, ds, (int)count, fl, pl, c->stream);
        if (e == cudaSuccess) e = launch_plan(c->dc, ds, (int)count, fl, pl, segs, c->stream);
        if (e == cudaSuccess) e = launch_keygen_fix(c->dc, sk->d, ds, (int)count, fl, pl, c->stream);
        if (e == cudaSuccess)
            e = launch_shoup_companion(c->dc, sk->d + (size_t)count * c->L * c->n, sk->d, (long long)count * c->L,
                                       c->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
        if (e != cudaSuccess) rc = fail(TS_ERR_CUDA, "keygen: %s", cudaGetErrorString(e));
    }
    if (rc) {
        cudaFreeAsync(sk->d, c->stream);
        delete sk;
        return rc;
    }
    *out = ctx_adopt(sk);
    return TS_OK;
}

int ts_keygen(ts_ctx* c, uint64_t seed, ts_sk** out) { return ts_keygen_batch(c, &seed, 1, out); }

int ts_sk_destroy(ts_sk* sk) {
    if (!sk) return TS_OK;
    ts_ctx* c = sk->ctx;
    {
        Lock lk(c);
        cudaSetDevice(c->device);
        cudaFreeAsync(sk->d, c->stream);
        delete sk;
    }
    ctx_release(c);
    return TS_OK;
}

int ts_sk_count(const ts_sk* sk, uint32_t* count) {
    if (!sk || !count) return fail(TS_ERR_ARG, "NULL argument");
    *count = sk->count;
    return TS_OK;
}

int ts_sk_export(const ts_sk* sk, uint32_t index, uint64_t* host) {
    if (!sk || !host || index >= sk->count) return fail(TS_ERR_ARG, "bad sk export arguments");
    ts_ctx* c = sk->ctx;
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    const size_t words = (size_t)c->L * c->n;
    CU(cudaMemcpyAsync(host, sk->d + index * words, words * 8, cudaMemcpyDeviceToHost, c->stream));
    CU(cudaStreamSynchronize(c->stream));
    return TS_OK;
}

// ------------------------------------------------------------------ encrypt
static int encrypt_impl(ts_ctx* c, const ts_sk* sk, const double* data, size_t count, size_t len, size_t stride,
                        const uint64_t* seeds, const int32_t* sk_index, int on_device, ts_ct** out) {
    if (!c || !sk || !out || !seeds || count == 0 || (!data && len)) return fail(TS_ERR_ARG, "bad encrypt arguments");
    if (sk->ctx != c) return fail(TS_ERR_ARG, "secret key belongs to another context");
    if (len > c->slots) len = c->slots;  // lib.rs:124-126 pads / truncates
    if (stride < len) stride = len;
    if (on_device && !aligned(data, 8)) return fail(TS_ERR_ARG, "device data must be 8-byte aligned");
    int rc = set_device(c);
    if (rc) return rc;
    if (sk_index)
        for (size_t i = 0; i < count; i++)
            if (sk_index[i] < 0 || (uint32_t)sk_index[i] >= sk->count) return fail(TS_ERR_ARG, "sk_index out of range");
    ts_ct* ct = nullptr;
    rc = new_ct(c, (uint32_t)count, c->L, c->dc.scale, &ct);
    if (rc) return rc;
    // inputs to the device (persistent buffer for this call)
    void* buf = nullptr;
    const size_t data_bytes = on_device ? 0 : count * (len ? len : 1) * 8;
    const size_t bytes = data_bytes + count * 8 + count * 4 + 512;
    rc = dev_alloc(c, &buf, bytes);
    if (rc) {
        cudaFreeAsync(ct->d, c->stream);
        delete ct;
        return rc;
    }
    double* d_data = on_device ? const_cast<double*>(data) : static_cast<double*>(buf);
    uint64_t* d_seeds = reinterpret_cast<uint64_t*>(static_cast<char*>(buf) + ((data_bytes + 255) & ~(size_t)255));
    int* d_skof = reinterpret_cast<int*>(d_seeds + count);
    if (!on_device) rc = h2d_rows(c, d_data, data, count, len, stride);
    if (!rc) rc = h2d_small(c, d_seeds, seeds, count);
    if (!rc && sk_index) rc = h2d_small(c, d_skof, (const int*)sk_index, count);
    SlotSrc src{d_data, 0, (int)len, (long long)(on_device ? stride : len), 0, 0};
    if (!rc) {
        const size_t cap = count < 256 ? count : 256;
        Carve cv;
        size_t idx[5];
        carve_enc(cv, cap, c->n, idx);
        rc = ensure_scratch(c, cv.total());
        if (!rc) rc = encrypt_core(c, src, count, d_seeds, sk_index ? d_skof : nullptr, sk->d, sk_shoup(sk), ct->d,
                                   enc_work(cv, c->scratch, cap, idx));
    }
    cudaFreeAsync(buf, c->stream);
    if (!rc) rc = check_stats(c);
    if (rc) {
        cudaFreeAsync(ct->d, c->stream);
        delete ct;
        return rc;
    }
    *out = ctx_adopt(ct);
    return TS_OK;
}

int ts_encrypt(ts_ctx* c, const ts_sk* sk, const double* data, size_t len, uint64_t seed, ts_ct** out) {
    if (!c) return fail(TS_ERR_ARG, "ctx is NULL");
    Lock lk(c);
    return encrypt_impl(c, sk, data, 1, len, len, &seed, nullptr, 0, out);
}

int ts_encrypt_batch(ts_ctx* c, const ts_sk* sk, const double* data, size_t count, size_t len, size_t stride,
                     const uint64_t* seeds, const int32_t* sk_index, int data_on_device, ts_ct** out) {
    if (!c) return fail(TS_ERR_ARG, "ctx is NULL");
    Lock lk(c);
    return encrypt_impl(c, sk, data, count, len, stride, seeds, sk_index, data_on_device, out);
}

int ts_ct_destroy(ts_ct* ct) {
    if (!ct) return TS_OK;
    ts_ctx* c = ct->ctx;
    {
        Lock lk(c);
        cudaSetDevice(c->device);
        cudaFreeAsync(ct->d, c->stream);
        delete ct;
    }
    ctx_release(c);
    return TS_OK;
}

int ts_ct_info(const ts_ct* ct, uint32_t* count, uint32_t* limbs, double* scale) {
    if (!ct) return fail(TS_ERR_ARG, "ct is NULL");
    if (count) *count = ct->count;
    if (limbs) *limbs = ct->limbs;
    if (scale) *scale = ct->scale;
    return TS_OK;
}

int ts_ct_export(const ts_ct* ct, uint32_t index, uint64_t* c0, uint64_t* c1) {
    if (!ct || index >= ct->count) return fail(TS_ERR_ARG, "bad ct export arguments");
    ts_ctx* c = ct->ctx;
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    const size_t words = (size_t)ct->limbs * c->n;
    const uint64_t* base = ct->d + (size_t)index * 2 * words;
    if (c0) CU(cudaMemcpyAsync(c0, base, words * 8, cudaMemcpyDeviceToHost, c->stream));
    if (c1) CU(cudaMemcpyAsync(c1, base + words, words * 8, cudaMemcpyDeviceToHost, c->stream));
    CU(cudaStreamSynchronize(c->stream));
    return TS_OK;
}

int ts_ct_import(ts_ctx* c, const uint64_t* c0, const uint64_t* c1, uint32_t limbs, double scale, ts_ct** out) {
    if (!c || !c0 || !c1 || !out || limbs == 0 || limbs > c->L) return fail(TS_ERR_ARG, "bad ct import arguments");
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    ts_ct* ct = nullptr;
    rc = new_ct(c, 1, limbs, scale, &ct);
    if (rc) return rc;
    const size_t words = (size_t)limbs * c->n;
    CU(cudaMemcpyAsync(ct->d, c0, words * 8, cudaMemcpyHostToDevice, c->stream));
    CU(cudaMemcpyAsync(ct->d + words, c1, words * 8, cudaMemcpyHostToDevice, c->stream));
    CU(cudaStreamSynchronize(c->stream));
    *out = ctx_adopt(ct);
    return TS_OK;
}

int ts_ct_select(ts_ctx* c, const ts_ct* ct, uint32_t index, ts_ct** out) {
    if (!c || !ct || !out || index >= ct->count) return fail(TS_ERR_ARG, "bad ct select arguments");
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    ts_ct* o = nullptr;
    rc = new_ct(c, 1, ct->limbs, ct->scale, &o);
    if (rc) return rc;
    const size_t words = (size_t)2 * ct->limbs * c->n;
    CU(cudaMemcpyAsync(o->d, ct->d + index * words, words * 8, cudaMemcpyDeviceToDevice, c->stream));
    *out = ctx_adopt(o);
    return TS_OK;
}

// ------------------------------------------------------------------ wire format
// serialize.rs:14-93: an RnsPoly is limb-major little-endian u64; a
// ciphertext is [scale f64 LE | c0 | c1], a public key [b | a].  The device
// layout of a ciphertext object, [count][2][limbs][n], is already the wire
// layout of c0 | c1 (and a key's [2][L][n] that of b | a), so each direction
// is one copy; a batch of ciphertexts is their blobs back to back (one
// strided copy).
static_assert(__BYTE_ORDER__ == __ORDER_LITTLE_ENDIAN__, "the wire format and the device are little-endian");

// Every u64 of `polys` polynomials of `limbs` limbs at p (unaligned bytes)
// must be at most q_l: canonical residues, or q itself, which the
// reference's encode can emit (its negative branch when q divides a
// coefficient).  Larger words would break the kernels' lazy-reduction
// bounds, so they are refused instead of being reduced silently.
static int check_wire_residues(const ts_ctx* c, const uint8_t* p, size_t polys, uint32_t limbs, const char* what) {
    for (size_t k = 0; k < polys; k++)
        for (uint32_t l = 0; l < limbs; l++) {
            const uint64_t q = c->q[l];
            const uint8_t* w = p + ((k * limbs + l) * (size_t)c->n) * 8;
            for (uint32_t i = 0; i < c->n; i++) {
                uint64_t x;
                memcpy(&x, w + (size_t)i * 8, 8);
                if (x > q)
                    return fail(TS_ERR_ARG, "%s: word %u of limb %u is %llu, not a residue mod %llu", what, i, l,
                                (unsigned long long)x, (unsigned long long)q);
            }
        }
    return TS_OK;
}

int ts_ct_to_bytes(const ts_ct* ct, uint8_t* out, size_t out_len, size_t* written) {
    if (!ct || !out) return fail(TS_ERR_ARG, "bad ct_to_bytes arguments");
    ts_ctx* c = ct->ctx;
    const size_t body = (size_t)2 * ct->limbs * c->n * 8, blob = 8 + body, total = blob * ct->count;
    if (out_len < total) return fail(TS_ERR_ARG, "ct_to_bytes: %zu bytes needed, the buffer holds %zu", total, out_len);
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    for (uint32_t i = 0; i < ct->count; i++) memcpy(out + (size_t)i * blob, &ct->scale, 8);
    if (ct->count == 1)
        CU(cudaMemcpyAsync(out + 8, ct->d, body, cudaMemcpyDeviceToHost, c->stream));
    else
        CU(cudaMemcpy2DAsync(out + 8, blob, ct->d, body, body, ct->count, cudaMemcpyDeviceToHost, c->stream));
    CU(cudaStreamSynchronize(c->stream));
    if (written) *written = total;
    return TS_OK;
}

int ts_ct_from_bytes(ts_ctx* c, const uint8_t* bytes, size_t len, uint32_t num_limbs, ts_ct** out) {
    if (!c || !bytes || !out) return fail(TS_ERR_ARG, "bad ct_from_bytes arguments");
    if (num_limbs == 0 || num_limbs > c->L)
        return fail(TS_ERR_ARG, "ct_from_bytes: num_limbs %u out of range [1, %u]", num_limbs, c->L);
    const size_t body = (size_t)2 * num_limbs * c->n * 8, blob = 8 + body;
    if (len == 0 || len % blob != 0)
        return fail(TS_ERR_ARG, "Expected a multiple of %zu bytes for Ciphertext(n=%u, L=%u), got %zu", blob, c->n,
                    num_limbs, len);
    const size_t count = len / blob;
    if (count > UINT32_MAX) return fail(TS_ERR_ARG, "ct_from_bytes: too many ciphertexts");
    double scale = 0.0;
    memcpy(&scale, bytes, 8);
    for (size_t i = 0; i < count; i++) {
        if (memcmp(bytes + i * blob, bytes, 8) != 0)
            return fail(TS_ERR_ARG, "ct_from_bytes: ciphertext %zu has another scale than ciphertext 0", i);
        int rc = check_wire_residues(c, bytes + i * blob + 8, 2, num_limbs, "ct_from_bytes");
        if (rc) return rc;
    }
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    ts_ct* ct = nullptr;
    rc = new_ct(c, (uint32_t)count, num_limbs, scale, &ct);
    if (rc) return rc;
    cudaError_t e = count == 1 ? cudaMemcpyAsync(ct->d, bytes + 8, body, cudaMemcpyHostToDevice, c->stream)
                               : cudaMemcpy2DAsync(ct->d, body, bytes + 8, blob, body, count, cudaMemcpyHostToDevice,
                                                   c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) {
        cudaFreeAsync(ct->d, c->stream);
        delete ct;
        return fail(TS_ERR_CUDA, "ct_from_bytes: %s", cudaGetErrorString(e));
    }
    *out = ctx_adopt(ct);
    return TS_OK;
}

int ts_pk_to_bytes(const ts_pk* pk, uint8_t* out, size_t out_len, size_t* written) {
    if (!pk || !out) return fail(TS_ERR_ARG, "bad pk_to_bytes arguments");
    ts_ctx* c = pk->ctx;
    const size_t total = (size_t)2 * c->L * c->n * 8;
    if (out_len < total) return fail(TS_ERR_ARG, "pk_to_bytes: %zu bytes needed, the buffer holds %zu", total, out_len);
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    CU(cudaMemcpyAsync(out, pk->d, total, cudaMemcpyDeviceToHost, c->stream));
    CU(cudaStreamSynchronize(c->stream));
    if (written) *written = total;
    return TS_OK;
}

int ts_pk_from_bytes(ts_ctx* c, const uint8_t* bytes, size_t len, ts_pk** out) {
    if (!c || !bytes || !out) return fail(TS_ERR_ARG, "bad pk_from_bytes arguments");
    const size_t words = (size_t)c->L * c->n;
    if (len != 2 * words * 8) return fail(TS_ERR_ARG, "Expected %zu bytes for PublicKey, got %zu", 2 * words * 8, len);
    int rc = check_wire_residues(c, bytes, 2, c->L, "pk_from_bytes");
    if (rc) return rc;
    Lock lk(c);
    rc = set_device(c);
    if (rc) return rc;
    ts_pk* pk = new ts_pk{c, nullptr};
    rc = dev_alloc(c, (void**)&pk->d, 4 * words * 8);
    if (rc) {
        delete pk;
        return rc;
    }
    cudaError_t e = cudaMemcpyAsync(pk->d, bytes, 2 * words * 8, cudaMemcpyHostToDevice, c->stream);
    // Shoup companions of b and a, as keygen_public makes them
    if (e == cudaSuccess) e = launch_shoup_companion(c->dc, pk->d + 2 * words, pk->d, 2LL * c->L, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) {
        cudaFreeAsync(pk->d, c->stream);
        delete pk;
        return fail(TS_ERR_CUDA, "pk_from_bytes: %s", cudaGetErrorString(e));
    }
    *out = ctx_adopt(pk);
    return TS_OK;
}

// ------------------------------------------------------------------ decrypt
static int decrypt_core(ts_ctx* c, const ts_ct* ct, const uint64_t* d_sk, const uint64_t* d_sks, const int* d_skof,
                        double* d_out) {
    const size_t n = c->n;
    const bool crt = ct->scale > c->dc.scale * 1.5 && ct->limbs >= 2;  // ciphertext.rs:351
    const int nl = crt ? 2 : 1;
    const size_t CH = 256;
    for (size_t v0 = 0; v0 < ct->count; v0 += CH) {
        const size_t nv = ct->count - v0 < CH ? ct->count - v0 : CH;
        Carve cv;
        const size_t i_M = cv.add(nv * nl * n * 8), i_f = cv.add(nv * 2 * n * 8);
        int rc = ensure_scratch(c, cv.total());
        if (rc) return rc;
        uint64_t* M = cv.at<uint64_t>(c->scratch, i_M);
        double* f = cv.at<double>(c->scratch, i_f);
        const long long stride = (long long)2 * ct->limbs * n;
        CU(launch_decrypt_limbs(c->dc, M, nl, ct->d + v0 * stride, stride, (int)ct->limbs, d_sk, d_sks,
                                d_skof ? d_skof + v0 : nullptr, nullptr, nullptr, 1, (int)nv, c->stream));
        CU(launch_decode(c->dc, M, nl, crt, ct->scale, (int)nv, d_out + v0 * c->slots, nullptr, 0, 0, f, c->stream));
    }
    return TS_OK;
}

int ts_decrypt(ts_ctx* c, const ts_ct* ct, const ts_sk* sk, const int32_t* sk_index, double* out, int out_on_device) {
    if (!c || !ct || !sk || !out) return fail(TS_ERR_ARG, "bad decrypt arguments");
    if (ct->ctx != c || sk->ctx != c) return fail(TS_ERR_ARG, "objects belong to another context");
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    if (sk_index)
        for (uint32_t i = 0; i < ct->count; i++)
            if (sk_index[i] < 0 || (uint32_t)sk_index[i] >= sk->count) return fail(TS_ERR_ARG, "sk_index out of range");
    const size_t out_bytes = (size_t)ct->count * c->slots * 8;
    void* buf = nullptr;
    rc = dev_alloc(c, &buf, (out_on_device ? 0 : out_bytes) + ct->count * 4 + 256);
    if (rc) return rc;
    double* d_out = out_on_device ? out : static_cast<double*>(buf);
    int* d_skof = reinterpret_cast<int*>(static_cast<char*>(buf) + (out_on_device ? 0 : ((out_bytes + 255) & ~(size_t)255)));
    if (sk_index) rc = h2d_small(c, d_skof, (const int*)sk_index, ct->count);
    if (!rc) rc = decrypt_core(c, ct, sk->d, sk_shoup(sk), sk_index ? d_skof : nullptr, d_out);
    if (!rc && !out_on_device) {
        cudaError_t e = cudaMemcpyAsync(out, d_out, out_bytes, cudaMemcpyDeviceToHost, c->stream);
        if (e != cudaSuccess) rc = fail(TS_ERR_CUDA, "D2H: %s", cudaGetErrorString(e));
    }
    cudaFreeAsync(buf, c->stream);
    if (!rc) {
        cudaError_t e = cudaStreamSynchronize(c->stream);
        if (e != cudaSuccess) rc = fail(TS_ERR_CUDA, "decrypt: %s", cudaGetErrorString(e));
    }
    return rc;
}

// ------------------------------------------------------------------ ct x pt
static int encode_ntt_core(ts_ctx* c, const double* d_pts, size_t count, size_t len, size_t stride, uint64_t* d_out) {
    const size_t n = c->n;
    const size_t CH = 256;
    for (size_t v0 = 0; v0 < count; v0 += CH) {
        const size_t nv = count - v0 < CH ? count - v0 : CH;
        Carve cv;
        const size_t i_m = cv.add(nv * n * 8), i_f = cv.add(nv * 2 * n * 8);
        int rc = ensure_scratch(c, cv.total());
        if (rc) return rc;
        int64_t* m = cv.at<int64_t>(c->scratch, i_m);
        double* f = cv.at<double>(c->scratch, i_f);
        SlotSrc s{d_pts + v0 * stride, 0, (int)len, (long long)stride, 0, 0};
        CU(launch_encode(c->dc, s, (int)nv, m, nullptr, nullptr, 0, f, c->stream));
        CU(launch_ntt_signed(c->dc, d_out + v0 * c->L * n, m, (int)nv, c->stream));
    }
    return TS_OK;
}

int ts_encode_ntt(ts_ctx* c, const double* pts, size_t count, size_t len, size_t stride, int on_device, ts_pt** out) {
    if (!c || !out || count == 0 || (!pts && len)) return fail(TS_ERR_ARG, "bad encode arguments");
    if (len > c->slots) return fail(TS_ERR_ARG, "Input length %zu exceeds slot count %u", len, c->slots);
    if (stride < len) stride = len;
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    ts_pt* pt = new ts_pt{c, (uint32_t)count, nullptr};
    rc = dev_alloc(c, (void**)&pt->d, count * c->L * c->n * 8);
    if (rc) {
        delete pt;
        return rc;
    }
    double* d_in = nullptr;
    size_t st = stride;
    if (!on_device) {
        rc = dev_alloc(c, (void**)&d_in, count * (len ? len : 1) * 8);
        if (!rc) rc = h2d_rows(c, d_in, pts, count, len, stride);
        st = len ? len : 1;
    } else {
        d_in = const_cast<double*>(pts);
    }
    if (!rc) rc = encode_ntt_core(c, d_in, count, len, st, pt->d);
    if (!on_device && d_in) cudaFreeAsync(d_in, c->stream);
    if (!rc) {
        cudaError_t e = cudaStreamSynchronize(c->stream);
        if (e != cudaSuccess) rc = fail(TS_ERR_CUDA, "encode: %s", cudaGetErrorString(e));
    }
    if (rc) {
        cudaFreeAsync(pt->d, c->stream);
        delete pt;
        return rc;
    }
    *out = ctx_adopt(pt);
    return TS_OK;
}

int ts_pt_destroy(ts_pt* pt) {
    if (!pt) return TS_OK;
    ts_ctx* c = pt->ctx;
    {
        Lock lk(c);
        cudaSetDevice(c->device);
        cudaFreeAsync(pt->d, c->stream);
        delete pt;
    }
    ctx_release(c);
    return TS_OK;
}

int ts_pt_export(const ts_pt* pt, uint32_t index, uint64_t* host) {
    if (!pt || !host || index >= pt->count) return fail(TS_ERR_ARG, "bad pt export arguments");
    ts_ctx* c = pt->ctx;
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    const size_t words = (size_t)c->L * c->n;
    CU(cudaMemcpyAsync(host, pt->d + index * words, words * 8, cudaMemcpyDeviceToHost, c->stream));
    CU(cudaStreamSynchronize(c->stream));
    return TS_OK;
}

static int ct_pt_mul_dev(ts_ctx* c, const ts_ct* ct, const uint64_t* d_pt, ts_ct** out) {
    ts_ct* o = nullptr;
    int rc = new_ct(c, ct->count, ct->limbs, ct->scale * ct->scale, &o);  // ciphertext.rs:427
    if (rc) return rc;
    cudaError_t e = launch_elementwise(c->dc, o->d, ct->d, d_pt, (long long)ct->count * 2 * ct->limbs,
                                       (int)ct->limbs, true, EW_MUL, c->stream);
    if (e != cudaSuccess) {
        cudaFreeAsync(o->d, c->stream);
        delete o;
        return fail(TS_ERR_CUDA, "ct_pt_mul: %s", cudaGetErrorString(e));
    }
    *out = ctx_adopt(o);
    return TS_OK;
}

int ts_ct_pt_mul_ntt(ts_ctx* c, const ts_ct* ct, const ts_pt* pt, uint32_t pt_index, ts_ct** out) {
    if (!c || !ct || !pt || !out || pt_index >= pt->count) return fail(TS_ERR_ARG, "bad ct_pt_mul_ntt arguments");
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    return ct_pt_mul_dev(c, ct, pt->d + (size_t)pt_index * c->L * c->n, out);
}

int ts_ct_pt_mul(ts_ctx* c, const ts_ct* ct, const double* pt, size_t len, ts_ct** out) {
    if (!c || !ct || !out || (!pt && len)) return fail(TS_ERR_ARG, "bad ct_pt_mul arguments");
    if (len > c->slots) len = c->slots;  // lib.rs:345-347 pads / truncates
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    void* buf = nullptr;
    const size_t words = (size_t)c->L * c->n;
    rc = dev_alloc(c, &buf, words * 8 + (len ? len : 1) * 8 + 256);
    if (rc) return rc;
    uint64_t* d_pt = static_cast<uint64_t*>(buf);
    double* d_in = reinterpret_cast<double*>(d_pt + words);
    rc = h2d_rows(c, d_in, pt, 1, len, len);
    if (!rc) rc = encode_ntt_core(c, d_in, 1, len, len ? len : 1, d_pt);
    if (!rc) rc = ct_pt_mul_dev(c, ct, d_pt, out);
    cudaFreeAsync(buf, c->stream);
    if (!rc) {
        cudaError_t e = cudaStreamSynchronize(c->stream);
        if (e != cudaSuccess) rc = fail(TS_ERR_CUDA, "ct_pt_mul: %s", cudaGetErrorString(e));
    }
    return rc;
}

static int ct_addsub(ts_ctx* c, const ts_ct* a, const ts_ct* b, ts_ct** out, bool sub) {
    if (!c || !a || !b || !out) return fail(TS_ERR_ARG, "bad ct_add/ct_sub arguments");
    if (std::fabs(a->scale - b->scale) >= 1.0)  // ciphertext.rs:436-441
        return fail(TS_ERR_SCALE, "Scale mismatch in %s: %g vs %g", sub ? "ct_sub" : "ct_add", a->scale, b->scale);
    if (a->count != b->count || a->limbs != b->limbs) return fail(TS_ERR_ARG, "ciphertext shapes differ");
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    ts_ct* o = nullptr;
    rc = new_ct(c, a->count, a->limbs, a->scale, &o);
    if (rc) return rc;
    cudaError_t e = launch_elementwise(c->dc, o->d, a->d, b->d, (long long)a->count * 2 * a->limbs, (int)a->limbs, false,
                                       sub ? EW_SUB : EW_ADD, c->stream);
    if (e != cudaSuccess) {
        cudaFreeAsync(o->d, c->stream);
        delete o;
        return fail(TS_ERR_CUDA, "ct_add: %s", cudaGetErrorString(e));
    }
    *out = ctx_adopt(o);
    return TS_OK;
}

int ts_ct_add(ts_ctx* c, const ts_ct* a, const ts_ct* b, ts_ct** out) { return ct_addsub(c, a, b, out, false); }
int ts_ct_sub(ts_ctx* c, const ts_ct* a, const ts_ct* b, ts_ct** out) { return ct_addsub(c, a, b, out, true); }

// ------------------------------------------------------------------ raw kernels
int ts_ntt_forward(ts_ctx* c, uint64_t* data, size_t n_polys, uint32_t limb_count, uint32_t limb_offset) {
    if (!c || !data || limb_count == 0 || limb_offset + limb_count > c->L) return fail(TS_ERR_ARG, "bad NTT arguments");
    if (!aligned(data, 8)) return fail(TS_ERR_ARG, "data must be 8-byte aligned");
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    CU(launch_ntt(c->dc, data, (long long)n_polys * limb_count, (int)limb_count, (int)limb_offset, false, c->stream));
    return TS_OK;
}

int ts_ntt_inverse(ts_ctx* c, uint64_t* data, size_t n_polys, uint32_t limb_count, uint32_t limb_offset) {
    if (!c || !data || limb_count == 0 || limb_offset + limb_count > c->L) return fail(TS_ERR_ARG, "bad NTT arguments");
    if (!aligned(data, 8)) return fail(TS_ERR_ARG, "data must be 8-byte aligned");
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    CU(launch_ntt(c->dc, data, (long long)n_polys * limb_count, (int)limb_count, (int)limb_offset, true, c->stream));
    return TS_OK;
}

int ts_hadamard(ts_ctx* c, uint64_t* out, const uint64_t* a, const uint64_t* b, size_t n_polys, uint32_t limb_count,
                int b_bcast) {
    if (!c || !out || !a || !b || limb_count == 0 || limb_count > c->L) return fail(TS_ERR_ARG, "bad hadamard arguments");
    if (!aligned(out, 16) || !aligned(a, 16) || !aligned(b, 16))
        return fail(TS_ERR_ARG, "hadamard operands must be 16-byte aligned");
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    CU(launch_elementwise(c->dc, out, a, b, (long long)n_polys * limb_count, (int)limb_count, b_bcast != 0, EW_MUL,
                          c->stream));
    return TS_OK;
}

// ------------------------------------------------------------------ ZeRo-MOAI
// Packed plaintext rows of one adapter (inference_engine.py:1060-1068): row
// b holds A's rows b*cols .. b*cols + cols - 1, row i of them at slots
// i*d .. i*d + d - 1; out [nb][slots] must be zero on entry.
static void pack_lora_rows(const float* A, uint32_t r, uint32_t d, uint32_t cols, uint32_t nb, uint32_t slots,
                           double* out) {
    for (uint32_t b = 0; b < nb; b++) {
        double* row = out + (size_t)b * slots;
        for (uint32_t i = 0; i < cols && b * cols + i < r; i++) {
            const float* a_row = A + ((size_t)b * cols + i) * d;
            for (uint32_t j = 0; j < d; j++) row[(size_t)i * d + j] = (double)a_row[j];
        }
    }
}

int ts_lora_load(ts_ctx* c, const float* A, const float* B, uint32_t experts, uint32_t r, uint32_t d, ts_lora** out) {
    if (!c || !A || !B || !out || experts == 0 || r == 0 || d == 0) return fail(TS_ERR_ARG, "bad lora_load arguments");
    if (d > c->slots) return fail(TS_ERR_ARG, "d_model %u exceeds slot count %u", d, c->slots);
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    const uint32_t cols = c->slots / d > 0 ? c->slots / d : 1;  // inference_engine.py:1057
    const uint32_t nb = (r + cols - 1) / cols;                 // :1058
    std::vector<double> packed((size_t)experts * nb * c->slots, 0.0);
    for (uint32_t e = 0; e < experts; e++)
        pack_lora_rows(A + (size_t)e * r * d, r, d, cols, nb, c->slots, packed.data() + (size_t)e * nb * c->slots);
    ts_lora* lo = new ts_lora{c, experts, r, d, cols, nb, nullptr, nullptr, nullptr};
    double* d_in = nullptr;
    // Segment functionals of the decode (encoding.rs:295-315): slot k of a
    // decoded polynomial is sum_j coeff_j cos(pi j (2k+1) / N), so the sum
    // over segment c (slots c*d .. c*d+d-1) is sum_j coeff_j W[c][j] with
    //   W[c][j] = sin(d t) cos(t (2 c d + d)) / sin(t),  t = pi j / N  (W[c][0] = d),
    // evaluated in long double.
    std::vector<double> W;
    if (cols <= (uint32_t)kMaxSegCols && c->L >= 2) {
        W.resize((size_t)cols * c->n);
        const long double pi = 3.141592653589793238462643383279502884L;
        for (uint32_t cc = 0; cc < cols; cc++)
            for (uint32_t j = 0; j < c->n; j++) {
                if (j == 0) {
                    W[(size_t)cc * c->n] = (double)d;
                    continue;
                }
                const long double t = pi * (long double)j / (long double)c->n;
                W[(size_t)cc * c->n + j] =
                    (double)(sinl((long double)d * t) * cosl(t * (long double)(2ULL * cc * d + d)) / sinl(t));
            }
    }
    const size_t pt_words = (size_t)experts * nb * c->L * c->n;
    rc = dev_alloc(c, (void**)&lo->d_pt, 2 * pt_words * 8);
    if (!rc) rc = dev_alloc(c, (void**)&lo->d_b, (size_t)experts * d * r * 4);
    if (!rc && !W.empty()) rc = dev_alloc(c, (void**)&lo->d_w, W.size() * 8);
    if (!rc && !W.empty()) rc = h2d_small(c, lo->d_w, W.data(), W.size());
    if (!rc) rc = dev_alloc(c, (void**)&d_in, packed.size() * 8);
    if (!rc) rc = h2d_small(c, d_in, packed.data(), packed.size());
    if (!rc) rc = h2d_small(c, lo->d_b, B, (size_t)experts * d * r);
    if (!rc) rc = encode_ntt_core(c, d_in, (size_t)experts * nb, c->slots, c->slots, lo->d_pt);
    if (!rc) {
        cudaError_t e = launch_shoup_companion(c->dc, lo->d_pt + pt_words, lo->d_pt, (long long)experts * nb * c->L,
                                               c->stream);
        if (e != cudaSuccess) rc = fail(TS_ERR_CUDA, "lora_load: %s", cudaGetErrorString(e));
    }
    if (d_in) cudaFreeAsync(d_in, c->stream);
    if (!rc) {
        cudaError_t e = cudaStreamSynchronize(c->stream);
        if (e != cudaSuccess) rc = fail(TS_ERR_CUDA, "lora_load: %s", cudaGetErrorString(e));
    }
    if (rc) {
        if (lo->d_pt) cudaFreeAsync(lo->d_pt, c->stream);
        if (lo->d_b) cudaFreeAsync(lo->d_b, c->stream);
        if (lo->d_w) cudaFreeAsync(lo->d_w, c->stream);
        delete lo;
        return rc;
    }
    *out = ctx_adopt(lo);
    return TS_OK;
}

// Hot swap of one expert (inference_engine.py:879-959 swap_adapter, with the
// NTT(plaintext) cache of :1037-1074): the expert's cached plaintexts, their
// Shoup companions and its B are rebuilt in place, so device pointers held
// elsewhere (a captured decode-step graph) stay valid.  The rebuild is
// ordered on the context's stream and complete when the call returns; work
// enqueued on that stream before the call sees the old adapter, work after
// it the new one.
int ts_lora_set_expert(ts_ctx* c, ts_lora* lo, uint32_t expert, const float* A, const float* B) {
    if (!c || !lo || !A || !B) return fail(TS_ERR_ARG, "bad lora_set_expert arguments");
    if (lo->ctx != c) return fail(TS_ERR_ARG, "adapter belongs to another context");
    if (expert >= lo->experts) return fail(TS_ERR_ARG, "expert %u out of range (%u experts)", expert, lo->experts);
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    const uint32_t nb = lo->batches, r = lo->r, d = lo->d;
    std::vector<double> packed((size_t)nb * c->slots, 0.0);
    pack_lora_rows(A, r, d, lo->cols, nb, c->slots, packed.data());
    const size_t pt_words = (size_t)lo->experts * nb * c->L * c->n;
    const size_t off = (size_t)expert * nb * c->L * c->n;
    double* d_in = nullptr;
    rc = dev_alloc(c, (void**)&d_in, packed.size() * 8);
    if (!rc) rc = h2d_small(c, d_in, packed.data(), packed.size());
    if (!rc) rc = h2d_small(c, lo->d_b + (size_t)expert * d * r, B, (size_t)d * r);
    if (!rc) rc = encode_ntt_core(c, d_in, nb, c->slots, c->slots, lo->d_pt + off);
    if (!rc) {
        cudaError_t e = launch_shoup_companion(c->dc, lo->d_pt + pt_words + off, lo->d_pt + off,
                                               (long long)nb * c->L, c->stream);
        if (e != cudaSuccess) rc = fail(TS_ERR_CUDA, "lora_set_expert: %s", cudaGetErrorString(e));
    }
    if (d_in) cudaFreeAsync(d_in, c->stream);
    if (!rc) {
        cudaError_t e = cudaStreamSynchronize(c->stream);
        if (e != cudaSuccess) rc = fail(TS_ERR_CUDA, "lora_set_expert: %s", cudaGetErrorString(e));
    }
    return rc;
}

int ts_lora_destroy(ts_lora* lo) {
    if (!lo) return TS_OK;
    ts_ctx* c = lo->ctx;
    {
        Lock lk(c);
        cudaSetDevice(c->device);
        cudaFreeAsync(lo->d_pt, c->stream);
        cudaFreeAsync(lo->d_b, c->stream);
        if (lo->d_w) cudaFreeAsync(lo->d_w, c->stream);
        delete lo;
    }
    ctx_release(c);
    return TS_OK;
}

int ts_lora_info(const ts_lora* lo, uint32_t* experts, uint32_t* r, uint32_t* d, uint32_t* cols, uint32_t* batches) {
    if (!lo) return fail(TS_ERR_ARG, "lora is NULL");
    if (experts) *experts = lo->experts;
    if (r) *r = lo->r;
    if (d) *d = lo->d;
    if (cols) *cols = lo->cols;
    if (batches) *batches = lo->batches;
    return TS_OK;
}

int ts_lora_delta_batch(ts_ctx* c, const ts_sk* sk, const ts_lora* lo, const double* h, uint32_t n,
                        const int32_t* expert, const int32_t* sk_index, const uint64_t* seeds, double* delta,
                        double* inter, int io_on_device) {
    if (!c || !sk || !lo || !h || !seeds || !delta || n == 0) return fail(TS_ERR_ARG, "bad lora_delta arguments");
    if (sk->ctx != c || lo->ctx != c) return fail(TS_ERR_ARG, "objects belong to another context");
    if (io_on_device && (!aligned(h, 8) || !aligned(delta, 8) || !aligned(inter, 8)))
        return fail(TS_ERR_ARG, "device buffers must be 8-byte aligned");
    if (c->L < 2) return fail(TS_ERR_ARG, "the ct x pt decrypt needs at least 2 limbs (CRT)");
    if (io_on_device < 0 || io_on_device > 2) return fail(TS_ERR_ARG, "io_on_device must be 0, 1 or 2");
    // io_on_device == 2: seeds / expert / sk_index are device arrays too (the
    // call then issues stream work only, with no host copy or wait)
    const bool idx_dev = io_on_device == 2;
    for (uint32_t i = 0; !idx_dev && expert && i < n; i++)
        if (expert[i] < 0 || (uint32_t)expert[i] >= lo->experts) return fail(TS_ERR_ARG, "expert index out of range");
    for (uint32_t i = 0; !idx_dev && sk_index && i < n; i++)
        if (sk_index[i] < 0 || (uint32_t)sk_index[i] >= sk->count) return fail(TS_ERR_ARG, "sk_index out of range");
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    const size_t N = c->n, L = c->L, d = lo->d, r = lo->r, cols = lo->cols, nb = lo->batches;
    // Passes of at most 2048 deltas: large enough that every kernel's grid
    // spans many waves.  With host buffers and more than 1024 deltas the
    // passes are pipelined: the H2D of pass k+1 and the D2H of pass k-1 run on
    // the context's copy streams while pass k's kernels run, and the first
    // and last passes are 256 deltas, so that only their copies are exposed.
    const bool pipe = !io_on_device && n > 1024;
    std::vector<size_t> pass_start;
    {
        const size_t edge = pipe ? 256 : 0, mid = n - 2 * edge, per = (mid + 2047) / 2048;
        if (pipe) pass_start.push_back(0);
        for (size_t i = 0; i < per; i++) pass_start.push_back(edge + mid * i / per);
        if (pipe) pass_start.push_back(n - edge);
        pass_start.push_back(n);
    }
    size_t cap = 0;  // scratch is carved once, for the largest pass
    for (size_t i = 0; i + 1 < pass_start.size(); i++)
        cap = std::max(cap, pass_start[i + 1] - pass_start[i]);
    const size_t nbuf = pipe ? 2 : 1;  // host-facing buffers per pass (double-buffered when pipelined)
    const double scale2 = c->dc.scale * c->dc.scale;
    // small per-delta inputs: staged once through pinned memory (async H2D)
    void* small = nullptr;
    const uint64_t* d_seeds_all = seeds;
    const int* d_ex_all = expert;
    const int* d_sk_all = sk_index;
    if (!idx_dev) {
        const size_t sm_bytes = (size_t)n * 8 + (size_t)n * 4 * 2 + 512;
        int slot = 0;
        rc = ensure_pinned(c, sm_bytes, &slot);
        if (rc) return rc;
        uint64_t* p_seeds = static_cast<uint64_t*>(c->pinned[slot]);
        int* p_ex = reinterpret_cast<int*>(p_seeds + n);
        int* p_sk = p_ex + n;
        memcpy(p_seeds, seeds, (size_t)n * 8);
        if (expert) memcpy(p_ex, expert, (size_t)n * 4);
        if (sk_index) memcpy(p_sk, sk_index, (size_t)n * 4);
        rc = dev_alloc(c, &small, sm_bytes);
        if (rc) return rc;
        CU(cudaMemcpyAsync(small, c->pinned[slot], sm_bytes - 512, cudaMemcpyHostToDevice, c->stream));
        CU(cudaEventRecord(c->pinned_free[slot], c->stream));
        d_seeds_all = static_cast<uint64_t*>(small);
        d_ex_all = reinterpret_cast<const int*>(d_seeds_all + n);
        d_sk_all = d_ex_all + n;
    }
    if (pipe) {
        rc = ensure_copy_streams(c);
        if (rc) return rc;
    }
    for (size_t k = 0; k + 1 < pass_start.size() && !rc; k++) {
        const size_t v0 = pass_start[k], nv = pass_start[k + 1] - v0;
        const bool last_pass = k + 2 == pass_start.size();
        const size_t b = pipe ? (k & 1) : 0;  // host-facing buffer of this pass
        Carve cv;
        const size_t i_h = cv.add(io_on_device ? 0 : nbuf * cap * d * 8),
                     i_o = cv.add(io_on_device ? 0 : nbuf * cap * d * 8), i_in = cv.add(nbuf * cap * r * 8),
                     i_ct = cv.add(cap * 2 * L * N * 8), i_m = cv.add(cap * N * 8), i_e = cv.add(cap * N),
                     i_fe = cv.add(cap * 2 * N * 8), i_fl = cv.add((2 * cap + 1) * 4),
                     i_pl = cv.add(cap * sizeof(StreamPlan)),
                     // fused decrypt: limb 1 of every vector at N = 8192 / 16384 (split
                     // form; both limbs when the pass is small enough for the per-limb
                     // path), one limb-0 buffer per CTA below; otherwise both limbs of
                     // every vector (N = 32768: the per-limb path of small passes, of
                     // which the split form uses half; and the FFT scratch of the decode)
                     i_M = cv.add(lo->d_w && (c->logn == 13 || c->logn == 14)
                                      ? cap * nb * N * 8 * ((int)(cap * nb * 2) <= c->dc.sms ? 2 : 1)
                                  : lo->d_w && c->logn < 13 ? (size_t)c->dc.sms * N * 8 : cap * nb * 2 * N * 8),
                     i_fd = cv.add(lo->d_w ? 0 : cap * nb * 2 * N * 8), i_sg = cv.add(cap * nb * cols * 8),
                     // the split decrypt's c0 + c1*s rows of limbs 0 and 1
                     i_U = cv.add(lo->d_w && c->logn >= 13 ? cap * 2 * N * 8 : 0);
        // Small batches (a decode step): the weight stream of the model
        // between two calls evicts the kernels' code from L2, and a lone
        // transform's CTA then stalls on instruction fetches from HBM.  A
        // copy of the decrypt-side kernels on one vector of this call's
        // buffers (outputs to scratch) runs on a third stream from the start
        // of the call and brings their code back into L2 before the real
        // launches need it.
        const int cl = c->logn >= 15 ? 2 : 1;
        const bool code_warm = !pipe && lo->d_w && (int)(nv * L * cl * 2) <= c->dc.sms &&
                          (c->logn == 15 || (c->logn >= 13 && (int)(nv * nb * 2 * 2) <= c->dc.sms));
        const size_t i_wm = cv.add(code_warm ? 2 * N * 8 + kMaxSegCols * 8 : 0);
        rc = ensure_scratch(c, cv.total());  // grows on the first pass only
        if (rc) break;
        void* S = c->scratch;
        double* dh = io_on_device ? const_cast<double*>(h) + v0 * d : cv.at<double>(S, i_h) + b * cap * d;
        double* dout = io_on_device ? delta + v0 * d : cv.at<double>(S, i_o) + b * cap * d;
        double* dinter = (io_on_device && inter) ? inter + v0 * r : cv.at<double>(S, i_in) + b * cap * r;
        const uint64_t* ds = d_seeds_all + v0;
        const int* dex = expert ? d_ex_all + v0 : nullptr;
        const int* dsk = sk_index ? d_sk_all + v0 : nullptr;
        uint64_t* ct = cv.at<uint64_t>(S, i_ct);
        uint64_t* M = cv.at<uint64_t>(S, i_M);
        double* fd = cv.at<double>(S, i_fd);
        double* sg = cv.at<double>(S, i_sg);
        if (pipe) {
            double* dh0 = cv.at<double>(S, i_h);
            if (k == 0) {
                // the scratch (and the staged seeds) are ready in the context's
                // stream order; pass 0's hidden states go first
                CU(cudaEventRecord(c->ev_start, c->stream));
                CU(cudaStreamWaitEvent(c->s_h2d, c->ev_start, 0));
                CU(cudaMemcpyAsync(dh0, h, nv * d * 8, cudaMemcpyHostToDevice, c->s_h2d));
                CU(cudaEventRecord(c->ev_h2d[0], c->s_h2d));
            }
            if (!last_pass) {
                // pass k+1's hidden states into the other buffer, once pass k-1
                // (its last reader) has run
                const size_t v1 = pass_start[k + 1], nv1 = pass_start[k + 2] - v1;
                const size_t b1 = (k + 1) & 1;
                if (k >= 1) CU(cudaStreamWaitEvent(c->s_h2d, c->ev_comp[b1], 0));
                CU(cudaMemcpyAsync(dh0 + b1 * cap * d, h + v1 * d, nv1 * d * 8, cudaMemcpyHostToDevice, c->s_h2d));
                CU(cudaEventRecord(c->ev_h2d[b1], c->s_h2d));
            }
            CU(cudaStreamWaitEvent(c->stream, c->ev_h2d[b], 0));
            if (k >= 2) CU(cudaStreamWaitEvent(c->stream, c->ev_d2h[b], 0));  // pass k-2 has left dout / dinter
        } else if (!io_on_device) {
            rc = h2d_small(c, dh, h + v0 * d, nv * d);
            if (rc) break;
        }
        if (code_warm) {
            rc = ensure_side_streams(c);
            if (rc) break;
            uint64_t* wm = cv.at<uint64_t>(S, i_wm);
            CU(cudaEventRecord(c->ev_warm0, c->stream));
            CU(cudaStreamWaitEvent(c->warm, c->ev_warm0, 0));
            CU(launch_decrypt_limbs(c->dc, wm, 2, ct, (long long)2 * L * N, (int)L, sk->d, sk_shoup(sk), nullptr,
                                    lo->d_pt, nullptr, (int)nb, 1, c->warm,
                                    lo->d_pt + (size_t)lo->experts * nb * L * N, "warm_decrypt_limb"));
            CU(launch_crt_seg(c->dc, wm, 1, 1.0 / scale2, lo->d_w, (int)cols, reinterpret_cast<double*>(wm + 2 * N),
                              c->warm, "warm_crt_seg"));
            CU(cudaEventRecord(c->ev_warm1, c->warm));
        }
        // 1. encrypt the cols-fold replicated hidden states (:1267-1272)
        SlotSrc src{dh, 0, (int)d, (long long)d, (int)d, (int)cols};
        const size_t eidx[5] = {i_m, i_e, i_fe, i_fl, i_pl};
        // tables of the decrypt side, warmed into L2 during the encryption
        // when the batch is small: limbs 0/1 of the routed expert's packed
        // plaintexts and their companions, the segment functionals, B
        L2List warm{};
        {
            const int rows = expert ? (int)nv : 1;
            const long long limb = (long long)N * 8, lstride = (long long)L * limb;
            const long long per_expert = (long long)nb * lstride, bbytes = (long long)(d * r * 4);
            const uint64_t* pts = lo->d_pt + (size_t)lo->experts * nb * L * N;
            const int* ex = expert ? dex : nullptr;
            warm.r[warm.n++] = L2Range{lo->d_pt, ex, per_expert, (int)lo->experts, rows, (int)nb, lstride, 2 * limb};
            warm.r[warm.n++] = L2Range{pts, ex, per_expert, (int)lo->experts, rows, (int)nb, lstride, 2 * limb};
            if (lo->d_w) warm.r[warm.n++] = L2Range{lo->d_w, nullptr, 0, 0, 1, 1, 0, (long long)cols * limb};
            warm.r[warm.n++] = L2Range{lo->d_b, ex, bbytes, (int)lo->experts, rows, 1, 0, bbytes};
        }
        rc = encrypt_core(c, src, nv, ds, sk_index ? dsk : nullptr, sk->d, sk_shoup(sk), ct,
                          enc_work(cv, S, nv, eidx), &warm);
        if (rc) break;
        if (lo->d_w && (int)(nv * nb * 2 * cl) <= c->dc.sms) {
            // a batch too small to fill the GPU: the limb-0 and
            // limb-1 INTTs of every (delta, batch) run as separate CTAs
            // (cluster pairs at N = 32768), then one light kernel does the
            // CRT and the segment functionals (:1311-1386)
            CU(launch_decrypt_limbs(c->dc, M, 2, ct, (long long)2 * L * N, (int)L, sk->d, sk_shoup(sk),
                                    sk_index ? dsk : nullptr, lo->d_pt, expert ? dex : nullptr, (int)nb,
                                    (int)(nv * nb), c->stream, lo->d_pt + (size_t)lo->experts * nb * L * N));
            CU(launch_crt_seg(c->dc, M, (int)(nv * nb), 1.0 / scale2, lo->d_w, (int)cols, sg, c->stream));
        } else if (lo->d_w) {
            // 2+3. per (delta, batch): ct x packed_pt (limbs 0/1), c0 + c1*s, INTT,
            // CRT / Delta^2 and the segment sums of the decoded slots (:1311-1386)
            CU(launch_dec_fused(c->dc, ct, (long long)2 * L * N, (int)L, sk->d, sk_shoup(sk), sk_index ? dsk : nullptr,
                                lo->d_pt, lo->d_pt + (size_t)lo->experts * nb * L * N,
                                expert ? dex : nullptr, (int)nb, (int)(nv * nb), 1.0 / scale2, lo->d_w, (int)cols, M,
                                cv.at<uint64_t>(S, i_U), sg, c->stream));
        } else {
            // 2. ct x packed_pt (limbs 0/1) fused with decrypt's c0 + c1*s, INTT (:1311-1315)
            CU(launch_decrypt_limbs(c->dc, M, 2, ct, (long long)2 * L * N, (int)L, sk->d, sk_shoup(sk),
                                    sk_index ? dsk : nullptr,
                                    lo->d_pt, expert ? dex : nullptr, (int)nb, (int)(nv * nb), c->stream));
            // 3. CRT, / Delta^2, canonical embedding, segment sums (:1382-1386)
            CU(launch_decode(c->dc, M, 2, true, scale2, (int)(nv * nb), nullptr, sg, (int)d, (int)cols, fd,
                             c->stream));
        }
        if (code_warm) CU(cudaStreamWaitEvent(c->stream, c->ev_warm1, 0));  // join the warm-up stream
        CU(launch_gather_inter(sg, dinter, (int)nv, (int)nb, (int)cols, (int)r, c->stream));
        // 4. delta = B @ intermediate (:1392)
        CU(launch_bmat(lo->d_b, dinter, dout, (int)nv, (int)d, (int)r, expert ? dex : nullptr, (long long)d * r,
                       c->stream));
        if (pipe) {
            // pass k's results leave on the D2H stream while pass k+1 runs
            CU(cudaEventRecord(c->ev_comp[b], c->stream));
            CU(cudaStreamWaitEvent(c->s_d2h, c->ev_comp[b], 0));
            CU(cudaMemcpyAsync(delta + v0 * d, dout, nv * d * 8, cudaMemcpyDeviceToHost, c->s_d2h));
            if (inter) CU(cudaMemcpyAsync(inter + v0 * r, dinter, nv * r * 8, cudaMemcpyDeviceToHost, c->s_d2h));
            CU(cudaEventRecord(c->ev_d2h[b], c->s_d2h));
            if (last_pass) CU(cudaStreamWaitEvent(c->stream, c->ev_d2h[b], 0));  // the call ends after the last copy
        } else if (!io_on_device) {
            CU(cudaMemcpyAsync(delta + v0 * d, dout, nv * d * 8, cudaMemcpyDeviceToHost, c->stream));
            if (inter) CU(cudaMemcpyAsync(inter + v0 * r, dinter, nv * r * 8, cudaMemcpyDeviceToHost, c->stream));
        }
    }
    if (small) cudaFreeAsync(small, c->stream);
    if (rc) return rc;
    if (!io_on_device) return check_stats(c);
    return TS_OK;
}

int ts_dp_noise(ts_ctx* c, double* h, uint32_t n, uint32_t d, double clip, double sigma, const uint64_t* seeds,
                int on_device) {
    if (!c || !h || !seeds || n == 0 || d == 0) return fail(TS_ERR_ARG, "bad dp_noise arguments");
    if (on_device < 0 || on_device > 2) return fail(TS_ERR_ARG, "on_device must be 0, 1 or 2");
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    if (on_device == 2) {  // h and seeds on the device: stream work only
        cudaError_t e = launch_dp_noise(h, (int)n, (int)d, clip, sigma, seeds, c->stream);
        return e == cudaSuccess ? TS_OK : fail(TS_ERR_CUDA, "dp_noise: %s", cudaGetErrorString(e));
    }
    void* buf = nullptr;
    rc = dev_alloc(c, &buf, (on_device ? 0 : (size_t)n * d * 8) + n * 8 + 256);
    if (rc) return rc;
    double* dh = on_device ? h : static_cast<double*>(buf);
    uint64_t* ds = reinterpret_cast<uint64_t*>(static_cast<char*>(buf) + (on_device ? 0 : (((size_t)n * d * 8 + 255) & ~(size_t)255)));
    if (!on_device) rc = h2d_small(c, dh, h, (size_t)n * d);
    // seeds through a pinned slot, so that device-resident calls never wait
    int slot = 0;
    if (!rc) rc = ensure_pinned(c, (size_t)n * 8, &slot);
    if (!rc) {
        memcpy(c->pinned[slot], seeds, (size_t)n * 8);
        cudaError_t e = cudaMemcpyAsync(ds, c->pinned[slot], (size_t)n * 8, cudaMemcpyHostToDevice, c->stream);
        if (e == cudaSuccess) e = cudaEventRecord(c->pinned_free[slot], c->stream);
        if (e == cudaSuccess) e = launch_dp_noise(dh, (int)n, (int)d, clip, sigma, ds, c->stream);
        if (e == cudaSuccess && !on_device) {
            e = cudaMemcpyAsync(h, dh, (size_t)n * d * 8, cudaMemcpyDeviceToHost, c->stream);
            if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
        }
        if (e != cudaSuccess) rc = fail(TS_ERR_CUDA, "dp_noise: %s", cudaGetErrorString(e));
    }
    cudaFreeAsync(buf, c->stream);
    return rc;
}

// ------------------------------------------------------------------ public key
int ts_keygen_public(ts_ctx* c, const ts_sk* sk, uint32_t sk_index, uint64_t seed, ts_pk** out) {
    if (!c || !sk || !out) return fail(TS_ERR_ARG, "bad keygen_public arguments");
    if (sk->ctx != c) return fail(TS_ERR_ARG, "secret key belongs to another context");
    if (sk_index >= sk->count) return fail(TS_ERR_ARG, "sk_index out of range");
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    const size_t words = (size_t)c->L * c->n;
    ts_pk* pk = new ts_pk{c, nullptr};
    rc = dev_alloc(c, (void**)&pk->d, 4 * words * 8);
    if (rc) {
        delete pk;
        return rc;
    }
    // pk = (b, a) is exactly a secret-key encryption of the zero message
    // under the same stream layout (ciphertext.rs:114-154 against :167-229:
    // a limbs, then e; b = -a*s + e), so it reuses the encryption pipeline.
    Carve cv;
    size_t idx[5];
    carve_enc(cv, 1, c->n, idx);
    const size_t i_seed = cv.add(8);
    rc = ensure_scratch(c, cv.total());
    uint64_t* d_seed = rc ? nullptr : cv.at<uint64_t>(c->scratch, i_seed);
    if (!rc) rc = h2d_small(c, d_seed, &seed, 1);
    if (!rc) {
        SlotSrc zero{d_seed, 0, 0, 1, 0, 0};  // len 0: every slot is 0
        rc = encrypt_core(c, zero, 1, d_seed, nullptr, sk->d + sk_index * words, sk_shoup(sk) + sk_index * words,
                          pk->d, enc_work(cv, c->scratch, 1, idx));
    }
    if (!rc) {
        cudaError_t e = launch_shoup_companion(c->dc, pk->d + 2 * words, pk->d, 2LL * c->L, c->stream);
        if (e != cudaSuccess) rc = fail(TS_ERR_CUDA, "keygen_public: %s", cudaGetErrorString(e));
    }
    if (!rc) rc = check_stats(c);
    if (rc) {
        cudaFreeAsync(pk->d, c->stream);
        delete pk;
        return rc;
    }
    *out = ctx_adopt(pk);
    return TS_OK;
}

int ts_pk_destroy(ts_pk* pk) {
    if (!pk) return TS_OK;
    ts_ctx* c = pk->ctx;
    {
        Lock lk(c);
        cudaSetDevice(c->device);
        cudaFreeAsync(pk->d, c->stream);
        delete pk;
    }
    ctx_release(c);
    return TS_OK;
}

int ts_pk_export(const ts_pk* pk, uint64_t* b, uint64_t* a) {
    if (!pk) return fail(TS_ERR_ARG, "pk is NULL");
    ts_ctx* c = pk->ctx;
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    const size_t words = (size_t)c->L * c->n;
    if (b) CU(cudaMemcpyAsync(b, pk->d, words * 8, cudaMemcpyDeviceToHost, c->stream));
    if (a) CU(cudaMemcpyAsync(a, pk->d + words, words * 8, cudaMemcpyDeviceToHost, c->stream));
    CU(cudaStreamSynchronize(c->stream));
    return TS_OK;
}

int ts_encrypt_pk(ts_ctx* c, const ts_pk* pk, const double* data, size_t count, size_t len, size_t stride,
                  const uint64_t* seeds, int data_on_device, ts_ct** out) {
    if (!c || !pk || !out || !seeds || count == 0 || (!data && len)) return fail(TS_ERR_ARG, "bad encrypt_pk arguments");
    if (pk->ctx != c) return fail(TS_ERR_ARG, "public key belongs to another context");
    Lock lk(c);
    if (len > c->slots) len = c->slots;  // lib.rs:142-164 pads / truncates like encrypt
    if (stride < len) stride = len;
    if (data_on_device && !aligned(data, 8)) return fail(TS_ERR_ARG, "device data must be 8-byte aligned");
    int rc = set_device(c);
    if (rc) return rc;
    const size_t n = c->n, L = c->L, words = L * n;
    ts_ct* ct = nullptr;
    rc = new_ct(c, (uint32_t)count, c->L, c->dc.scale, &ct);
    if (rc) return rc;
    void* buf = nullptr;
    const size_t data_bytes = data_on_device ? 0 : count * (len ? len : 1) * 8;
    rc = dev_alloc(c, &buf, data_bytes + count * 8 + 512);
    if (rc) {
        cudaFreeAsync(ct->d, c->stream);
        delete ct;
        return rc;
    }
    double* d_data = data_on_device ? const_cast<double*>(data) : static_cast<double*>(buf);
    uint64_t* d_seeds = reinterpret_cast<uint64_t*>(static_cast<char*>(buf) + ((data_bytes + 255) & ~(size_t)255));
    if (!data_on_device) rc = h2d_rows(c, d_data, data, count, len, stride);
    if (!rc) rc = h2d_small(c, d_seeds, seeds, count);
    // stream layout (ciphertext.rs:240-319): ternary u (N words, rejecting
    // 0), then e0 and e1 (4N words each)
    SegList segs{};
    segs.count = 3;
    segs.kind[0] = SEG_TERNARY;
    segs.kind[1] = SEG_GAUSS;
    segs.kind[2] = SEG_GAUSS;
    const size_t cap = count < 256 ? count : 256;
    Carve cv;
    size_t idx[5];
    carve_enc(cv, cap, n, idx);
    const size_t i_e1 = cv.add(cap * n), i_u = cv.add(cap * words * 8);
    if (!rc) rc = ensure_scratch(c, cv.total());
    for (size_t v0 = 0; v0 < count && !rc; v0 += cap) {
        const size_t nv = count - v0 < cap ? count - v0 : cap;
        const EncWork w = enc_work(cv, c->scratch, cap, idx);
        int8_t* e1 = cv.at<int8_t>(c->scratch, i_e1);
        uint64_t* U = cv.at<uint64_t>(c->scratch, i_u);
        const uint64_t* sd = d_seeds + v0;
        SlotSrc src{d_data + v0 * (data_on_device ? stride : len), 0, (int)len,
                    (long long)(data_on_device ? stride : len), 0, 0};
        CU(cudaMemsetAsync(w.fl, 0, (2 * nv + 1) * 4, c->stream));
        CU(launch_encode(c->dc, src, (int)nv, w.m, w.e, sd, n, w.f, c->stream));  // m, e0 at word N
        CU(launch_gauss_gen(c->dc, e1, sd, (int)nv, 5 * n, c->stream));          // e1 at word 5N
        CU(launch_keygen(c->dc, U, sd, (int)nv, w.fl, w.pl, c->stream));         // NTT(u), flags
        // exact repair of streams whose ternary segment rejected a draw
        CU(launch_plan(c->dc, sd, (int)nv, w.fl, w.pl, segs, c->stream));
        CU(launch_keygen_fix(c->dc, U, sd, (int)nv, w.fl, w.pl, c->stream));
        CU(launch_gauss_fix(c->dc, w.e, sd, (int)nv, w.fl, w.pl, 1, c->stream));
        CU(launch_gauss_fix(c->dc, e1, sd, (int)nv, w.fl, w.pl, 2, c->stream));
        CU(launch_enc_pk(c->dc, ct->d + v0 * 2 * words, w.m, w.e, e1, U, pk->d, pk->d + 2 * words, (int)nv,
                         c->stream));
    }
    cudaFreeAsync(buf, c->stream);
    if (!rc) rc = check_stats(c);
    if (rc) {
        cudaFreeAsync(ct->d, c->stream);
        delete ct;
        return rc;
    }
    *out = ctx_adopt(ct);
    return TS_OK;
}

// ------------------------------------------------------------------ rescale
int ts_rescale(ts_ctx* c, const ts_ct* ct, ts_ct** out) {
    if (!c || !ct || !out) return fail(TS_ERR_ARG, "bad rescale arguments");
    if (ct->ctx != c) return fail(TS_ERR_ARG, "ciphertext belongs to another context");
    if (ct->limbs < 2) return fail(TS_ERR_ARG, "Cannot rescale: only 1 limb left");  // ciphertext.rs:479
    Lock lk(c);
    int rc = set_device(c);
    if (rc) return rc;
    const uint32_t nl = ct->limbs;
    const uint64_t q_last = c->q[nl - 1];
    RescaleInv inv{};
    for (uint32_t l = 0; l + 1 < nl; l++) {
        // rns.rs:114-117 asserts a != 0: a chain that repeats its last prime
        // (custom(..) duplicates) cannot be rescaled
        if (q_last % c->q[l] == 0) return fail(TS_ERR_ARG, "Cannot invert zero (limb %u repeats the last prime)", l);
        inv.v[l] = powmod(q_last % c->q[l], c->q[l] - 2, c->q[l]);
    }
    const size_t n = c->n, words = (size_t)ct->count * 2 * nl * n;
    ts_ct* o = nullptr;
    rc = new_ct(c, ct->count, nl - 1, ct->scale / (double)q_last, &o);  // ciphertext.rs:531
    if (rc) return rc;
    rc = ensure_scratch(c, words * 8);
    if (!rc) {
        uint64_t* t = static_cast<uint64_t*>(c->scratch);
        cudaError_t e = cudaMemcpyAsync(t, ct->d, words * 8, cudaMemcpyDeviceToDevice, c->stream);
        if (e == cudaSuccess) e = launch_ntt(c->dc, t, (long long)ct->count * 2 * nl, (int)nl, 0, true, c->stream);
        if (e == cudaSuccess) e = launch_rescale_combine(c->dc, o->d, t, (int)ct->count, (int)nl, inv, c->stream);
        if (e == cudaSuccess)
            e = launch_ntt(c->dc, o->d, (long long)ct->count * 2 * (nl - 1), (int)nl - 1, 0, false, c->stream);
        if (e != cudaSuccess) rc = fail(TS_ERR_CUDA, "rescale: %s", cudaGetErrorString(e));
    }
    if (rc) {
        cudaFreeAsync(o->d, c->stream);
        delete o;
        return rc;
    }
    *out = ctx_adopt(o);
    return TS_OK;
}

// batch_encrypt (lib.rs:231-258): the arrays consume ONE stream in order, so
// array i starts where array i-1 stopped.  Array i takes 2(L*N + R_i) + 4N
// words, R_i = its uniform rejections, so its start depends on every earlier
// array's rejections.  The starts are found by fixed-point iteration: plan
// every array from the starts implied by the previous round's rejection
// counts (round 0: none) until they repeat -- each round settles at least
// the first array whose start moved, and rejections are rare, so one or two
// rounds suffice.  Every array is then encrypted from its exact plan.
int ts_encrypt_stream(ts_ctx* c, const ts_sk* sk, const double* data, size_t count, size_t len, size_t stride,
                      uint64_t seed, ts_ct** out) {
    if (!c || !sk || !out || count == 0 || (!data && len)) return fail(TS_ERR_ARG, "bad batch_encrypt arguments");
    if (sk->ctx != c) return fail(TS_ERR_ARG, "secret key belongs to another context");
    Lock lk(c);
    if (len > c->slots) len = c->slots;  // lib.rs:244-250 pads / truncates each array
    if (stride < len) stride = len;
    int rc = set_device(c);
    if (rc) return rc;
    const size_t n = c->n, L = c->L, words = L * n;
    ts_ct* ct = nullptr;
    rc = new_ct(c, (uint32_t)count, c->L, c->dc.scale, &ct);
    if (rc) return rc;
    Carve cb;
    const size_t b_data = cb.add(count * (len ? len : 1) * 8), b_seed = cb.add(count * 8), b_base = cb.add(count * 8),
                 b_fl = cb.add((2 * count + 1) * 4), b_pl = cb.add(count * sizeof(StreamPlan));
    void* buf = nullptr;
    rc = dev_alloc(c, &buf, cb.total());
    if (rc) {
        cudaFreeAsync(ct->d, c->stream);
        delete ct;
        return rc;
    }
    double* d_data = cb.at<double>(buf, b_data);
    uint64_t* d_seeds = cb.at<uint64_t>(buf, b_seed);
    uint64_t* d_base = cb.at<uint64_t>(buf, b_base);
    uint32_t* d_fl = cb.at<uint32_t>(buf, b_fl);
    StreamPlan* d_pl = cb.at<StreamPlan>(buf, b_pl);
    std::vector<uint64_t> hseed(count, seed), base(count), nbase(count);
    std::vector<uint32_t> hfl(2 * count + 1);
    for (size_t v = 0; v < count; v++) {
        hfl[v] = 1;
        hfl[count + 1 + v] = (uint32_t)v;
    }
    hfl[count] = (uint32_t)count;
    rc = h2d_rows(c, d_data, data, count, len, stride);
    if (!rc) rc = h2d_small(c, d_seeds, hseed.data(), count);
    if (!rc) rc = h2d_small(c, d_fl, hfl.data(), hfl.size());
    const SegList segs = encrypt_segs(c->L);
    std::vector<StreamPlan> hp(count);
    for (size_t v = 0; v < count; v++) base[v] = v * (2 * words + 4 * n);  // no rejections
    for (size_t round = 0; !rc; round++) {
        if (round > count) {
            rc = fail(TS_ERR_STATE, "batch_encrypt: stream offsets did not settle");
            break;
        }
        rc = h2d_small(c, d_base, base.data(), count);
        if (rc) break;
        CU(launch_plan(c->dc, d_seeds, (int)count, d_fl, d_pl, segs, c->stream, d_base));
        CU(cudaMemcpyAsync(hp.data(), d_pl, count * sizeof(StreamPlan), cudaMemcpyDeviceToHost, c->stream));
        CU(cudaStreamSynchronize(c->stream));
        nbase[0] = 0;
        for (size_t v = 0; v < count; v++) {
            if (hp[v].status) {
                rc = fail(TS_ERR_STATE, "a sampling stream rejected more than %d candidates in one segment", kMaxRej);
                break;
            }
            if (v + 1 < count) {
                uint64_t rej = 0;
                for (uint32_t l = 0; l < L; l++) rej += hp[v].nrej[l];
                nbase[v + 1] = nbase[v] + 2 * (words + rej) + 4 * n;
            }
        }
        if (rc || nbase == base) break;
        base = nbase;
    }
    // encrypt every array from its plan, in chunks
    const size_t cap = count < 256 ? count : 256;
    Carve cv;
    size_t idx[5];
    carve_enc(cv, cap, n, idx);
    if (!rc) rc = ensure_scratch(c, cv.total());
    for (size_t v0 = 0; v0 < count && !rc; v0 += cap) {
        const size_t nv = count - v0 < cap ? count - v0 : cap;
        const EncWork w = enc_work(cv, c->scratch, cap, idx);
        std::vector<uint32_t> cfl(2 * nv + 1);  // every array of the chunk flagged
        for (size_t v = 0; v < nv; v++) {
            cfl[v] = 1;
            cfl[nv + 1 + v] = (uint32_t)v;
        }
        cfl[nv] = (uint32_t)nv;
        rc = h2d_small(c, w.fl, cfl.data(), cfl.size());
        if (rc) break;
        SlotSrc src{d_data + v0 * len, 0, (int)len, (long long)len, 0, 0};
        CU(launch_encode(c->dc, src, (int)nv, w.m, w.e, d_seeds, 2 * words, w.f, c->stream));
        CU(launch_gauss_fix(c->dc, w.e, d_seeds + v0, (int)nv, w.fl, d_pl + v0, (int)L, c->stream));
        CU(launch_encrypt_limbs(c->dc, ct->d + v0 * 2 * words, w.m, w.e, sk->d, sk_shoup(sk), nullptr, d_seeds + v0,
                                (int)nv, w.fl, d_pl + v0, true, c->stream));
    }
    cudaFreeAsync(buf, c->stream);
    if (!rc) rc = check_stats(c);
    if (rc) {
        cudaFreeAsync(ct->d, c->stream);
        delete ct;
        return rc;
    }
    *out = ctx_adopt(ct);
    return TS_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------
// Read-only accessors for noalloc.cu (the opaque structs are defined here).
// ---------------------------------------------------------------------
namespace tsg_host {
int noalloc_ctx(ts_ctx* c, int* device, const DevCtx** dc, cudaStream_t* stream, uint32_t* n, uint32_t* slots,
                std::mutex** mu) {
    *device = c->device;
    *dc = &c->dc;
    *stream = c->stream;
    *n = c->n;
    *slots = c->slots;
    *mu = &c->mu;
    return TS_OK;
}
int noalloc_ct(const ts_ct* ct, const ts_ctx** owner, uint32_t* count, uint32_t* limbs, double* scale,
               const uint64_t** d) {
    *owner = ct->ctx;
    *count = ct->count;
    *limbs = ct->limbs;
    *scale = ct->scale;
    *d = ct->d;
    return TS_OK;
}
int noalloc_sk(const ts_sk* sk, const ts_ctx** owner, uint32_t* count, const uint64_t** d, const uint64_t** ds) {
    *owner = sk->ctx;
    *count = sk->count;
    *d = sk->d;
    *ds = sk_shoup(sk);
    return TS_OK;
}
int noalloc_fail(int code, const char* msg) { return fail(code, "%s", msg); }
}  // namespace tsg_host
