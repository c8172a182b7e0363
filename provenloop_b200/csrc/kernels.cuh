// kernels.cuh -- internal launcher interface between the host API
// (tsgpu.cu) and the CUDA kernels (kernels.cu).  Not part of the public ABI.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "ntt.cuh"
#include "fft.cuh"

namespace tsg {

// Random-stream segments consumed by one keygen / encrypt call, in the
// reference's order (ciphertext.rs:77-103, :167-229, :114-154, :240-319).
enum SegKind : int { SEG_UNIFORM = 0, SEG_TERNARY = 1, SEG_GAUSS = 2 };
constexpr int kMaxSeg = 10;
constexpr int kMaxRej = 16;

struct SegList {
    int count;
    int kind[kMaxSeg];
    int limb[kMaxSeg];  // modulus index for SEG_UNIFORM
};

// Exact stream layout of one call: word offset of each segment and the
// candidate indexes the reference's rejection loops discarded.
struct StreamPlan {
    uint64_t off[kMaxSeg];
    uint32_t nrej[kMaxSeg];
    uint32_t rej[kMaxSeg][kMaxRej];
    uint32_t status;  // 0 ok, 1 more than kMaxRej rejections in a segment
    uint32_t pad;
};

// Device counters (unsigned long long each).
enum Stat : int {
    STAT_NEAR_TIE = 0,    // Gaussian samples within 1e-9 of a half-integer
    STAT_REJECT = 1,      // streams that needed the exact-plan repair
    STAT_PLAN_FAIL = 2,   // streams whose rejections exceeded kMaxRej
    STAT_COUNT = 4
};

// CRT(q0, q1) constants of decrypt (ciphertext.rs:351-356).
struct CrtConst {
    uint64_t q0, q1, mu64_1, q0inv, q0inv_s, bmu1;  // q0inv_s: Shoup companion of q0^-1 mod q1
    int bk1;
    int pad;
    uint64_t Q_lo, Q_hi;  // q0*q1
    uint64_t H_lo, H_hi;  // (q0*q1)/2
    // FP64 form of the same CRT for the segment functionals (crt_coeff_fp):
    // q1, (2^30 mod q1) and (q0^-1 mod q1) balanced with their quotients by
    // q1, (q1 - 1)/2, q0 = q0_hi + q0_lo (q0_hi = fl(q0)), floor(q0 / 2)
    double q1d, r30, r30q, q0invd, q0invq, t_half, q0_hi, q0_lo;
    uint64_t q0_half;
};

struct DevCtx {
    int logn, n, L;
    int sms;              // streaming multiprocessors of the context's device
    uint64_t q0, q1;      // moduli of limbs 0 and 1 (host copies, for kernel selection)
    int encode_cluster;   // the device runs the cluster encode (2 CTAs at N = 16384, 4 at N = 32768)
    const LimbTab* tabs;  // device array [L]
    FftTab fft;
    double scale;         // Delta = 2^40 (params.rs:9-12)
    CrtConst crt;
    unsigned long long* stats;  // device [STAT_COUNT]
};

// Where slot values come from for an encode (one "vector" per encode):
// slot k of vector v is
//   rep_cols > 0 : (k < rep_cols*rep_d) ? src[v*stride + k % rep_d] : 0
//   otherwise    : (k < len) ? src[v*stride + k] : 0
struct SlotSrc {
    const void* src;
    int is_f32;
    int len;
    long long stride;
    int rep_d;
    int rep_cols;
};

// ---------------------------------------------------------------- profiling
// Process-wide count of kernels launched by this library, and optional
// per-kernel CUDA-event timing of every launch (diagnostics for the bench).
uint64_t launch_count();
void prof_enable(bool on);
void prof_reset();
// Sum of event-timed milliseconds and number of launches of kernel `name`
// (waits for the recorded events).  Returns false if `name` was not seen.
bool prof_read(const char* name, double* ms, uint64_t* launches);

// ---------------------------------------------------------------- launchers
// In-place forward/inverse NTT of P poly-limbs of `data` ([P][n]); the limb of
// poly-limb p is l0 + p % lmod.
cudaError_t launch_ntt(const DevCtx& c, uint64_t* data, long long P, int lmod, int l0, bool inverse,
                       cudaStream_t s);
// out[p][i] = a[p][i] (*|+|-) b[bp][i] mod q_{p % L}, bp = b_bcast ? p % L : p.
enum EwOp : int { EW_MUL = 0, EW_ADD = 1, EW_SUB = 2 };
cudaError_t launch_elementwise(const DevCtx& c, uint64_t* out, const uint64_t* a, const uint64_t* b, long long P,
                               int L, bool b_bcast, EwOp op, cudaStream_t s);

// Secret keys: sk[k][L][n] from seeds[k] (ciphertext.rs:77-103).
cudaError_t launch_keygen(const DevCtx& c, uint64_t* sk, const uint64_t* seeds, int nkeys, uint32_t* flags,
                          StreamPlan* plans, cudaStream_t s);

// Encode slot vectors -> rounded coefficients m[v][n] (int64); when e != null,
// also the encryption's Gaussian e[v][n] (int8) at word offset gauss_off of
// stream seeds[v] (speculative: assumes no earlier rejection).
// Encode-kernel probe: whether the 2-CTA cluster encode can be resident on
// the current device (sets its shared-memory limit as a side effect).
bool encode_cluster_supported(int logn);
cudaError_t launch_encode(const DevCtx& c, const SlotSrc& src, int nvec, int64_t* m, int8_t* e,
                          const uint64_t* seeds, uint64_t gauss_off, double* scratch_cplx, cudaStream_t s);

// pt_ntt[v][L][n] = NTT(residues of m[v]) (ciphertext.rs:539-545).
cudaError_t launch_ntt_signed(const DevCtx& c, uint64_t* out, const int64_t* m, int nvec, cudaStream_t s);

// The speculative encryption split for latency (small batches): c1 = NTT(a)
// on stream s_a concurrently with c0 = NTT(m + e) on stream s_x; the caller
// joins the streams and runs launch_enc_combine (c0 -= c1*s) after both.
cudaError_t launch_encrypt_split(const DevCtx& c, uint64_t* ct, const int64_t* m, const int8_t* e, const uint64_t* sk,
                                 const uint64_t* sks, const int* sk_of, const uint64_t* seeds, int nvec,
                                 uint32_t* flags, const StreamPlan* plans, cudaStream_t s_a, cudaStream_t s_x);
cudaError_t launch_enc_combine(const DevCtx& c, uint64_t* ct, const uint64_t* sk, const uint64_t* sks,
                               const int* sk_of, int nvec, cudaStream_t s);

// L2 warm-up of the tables a small batch reads (latency mode): each range is
// `rows` x `reps` blocks of `bytes` at base + idx[row]*idx_stride +
// rep*rep_stride (idx[row] outside [0, idx_max) skips the row; idx null:
// row 0 only, no offset).  Issued as bulk L2 prefetches, so it moves no data
// through the SMs and has no visible effect besides cache state.
constexpr int kMaxL2Ranges = 12;
struct L2Range {
    const void* base;
    const int* idx;
    long long idx_stride;
    int idx_max;
    int rows;
    int reps;
    long long rep_stride;
    long long bytes;
};
struct L2List {
    L2Range r[kMaxL2Ranges];
    int n;
};
cudaError_t launch_prefetch_l2(const L2List& list, cudaStream_t s);

// Shoup companions out[i] = floor(in[i] * 2^64 / q_l) of canonical
// residues, for `polys` consecutive poly-limbs whose limb index is poly % L.
cudaError_t launch_shoup_companion(const DevCtx& c, uint64_t* out, const uint64_t* in, long long polys,
                                   cudaStream_t s);

// Secret-key encryption of nvec vectors into ct[v][2][L][n]
// (ciphertext.rs:167-229).  sk_of[v] selects the key (sk + sk_of[v]*L*n,
// Shoup companions at the same offset from sks); when plan_mode, only
// streams with flags[v] != 0 are (re)computed using plans[v].
cudaError_t launch_encrypt_limbs(const DevCtx& c, uint64_t* ct, const int64_t* m, const int8_t* e,
                                 const uint64_t* sk, const uint64_t* sks, const int* sk_of, const uint64_t* seeds,
                                 int nvec,
                                 uint32_t* flags, const StreamPlan* plans, bool plan_mode, cudaStream_t s);

// Gaussian errors e[v][j] from stream words off + 4j (off a multiple of 16)
// of seeds[v] (sampling.rs:51-58), for every vector.
cudaError_t launch_gauss_gen(const DevCtx& c, int8_t* e, const uint64_t* seeds, int nvec, uint64_t off,
                             cudaStream_t s);
// Public-key encryption (ciphertext.rs:240-319) of nvec vectors into
// ct[v][2][L][n] from m, e0, e1, U = NTT(u) [v][L][n] and pk = (b, a)
// [2][L][n] with Shoup companions pks.
cudaError_t launch_enc_pk(const DevCtx& c, uint64_t* ct, const int64_t* m, const int8_t* e0, const int8_t* e1,
                          const uint64_t* U, const uint64_t* pk, const uint64_t* pks, int nvec, cudaStream_t s);

// q_last^-1 mod q_l for the limbs kept by a rescale.
struct RescaleInv {
    uint64_t v[kMaxLimbs];
};
// Rescale's coefficient-domain step (ciphertext.rs:499-521): in is
// INTT(ct) [count][2][nl][n], out [count][2][nl-1][n] (still coefficients).
cudaError_t launch_rescale_combine(const DevCtx& c, uint64_t* out, const uint64_t* in, int count, int nl,
                                   const RescaleInv& inv, cudaStream_t s);

// Flag buffers hold (2*count + 1) uint32: per-stream flags, the number of
// flagged streams, and their indexes; zero them before the speculative pass.
// Exact plans for flagged streams (CTAs walk the flagged list).  Stream v's
// segments start at word bases[v] (0 when bases is null).
cudaError_t launch_plan(const DevCtx& c, const uint64_t* seeds, int nstreams, const uint32_t* flags,
                        StreamPlan* plans, const SegList& segs, cudaStream_t s, const uint64_t* bases = nullptr);
// Recompute the Gaussian e[v] of flagged streams from plan segment `seg`.
cudaError_t launch_gauss_fix(const DevCtx& c, int8_t* e, const uint64_t* seeds, int nvec, const uint32_t* flags,
                             const StreamPlan* plans, int seg, cudaStream_t s);
// Redo keygen of flagged keys using their plans.
cudaError_t launch_keygen_fix(const DevCtx& c, uint64_t* sk, const uint64_t* seeds, int nkeys,
                              const uint32_t* flags, const StreamPlan* plans, cudaStream_t s);

// Decrypt front half: M[v][j][n] = INTT( c0 (+) c1*s ) for limbs j < nl, where
// the ciphertext of vector v is cts + ct_of(v)*ct_stride and, when pt !=
// null, both components are first multiplied by pt + pt_of(v)*L*n
// (ct x pt fused into decrypt; ciphertext.rs:408-429 then :327-349).  With
// pts (the plaintexts' Shoup companions) the product is formed as
// p*(c0 + c1*s) with two Shoup products.
// ct_of(v) = v / per_ct, pt_of(v) = (pt_sel ? pt_sel[v / per_ct] : 0)*per_ct + v % per_ct.
// sks holds the keys' Shoup companions.
// `scope` names the launch in the per-kernel profile.
cudaError_t launch_decrypt_limbs(const DevCtx& c, uint64_t* M, int nl, const uint64_t* cts, long long ct_stride,
                                 int ct_limbs, const uint64_t* sk, const uint64_t* sks, const int* sk_of,
                                 const uint64_t* pt, const int* pt_sel, int per_ct, int nvec, cudaStream_t s,
                                 const uint64_t* pts = nullptr, const char* scope = "decrypt_limb");

// Decrypt back half (ciphertext.rs:351-399 + encoding.rs:219-315): CRT of
// limbs 0/1 (crt) or limb-0 centring, / scale, canonical embedding.
// Outputs either all slots (out_slots[v][S]) or, when seg_out != null, sums of
// `seg_cols` consecutive `seg_d`-slot segments: seg_out[v*seg_cols + c].
cudaError_t launch_decode(const DevCtx& c, const uint64_t* M, int nl, bool crt, double scale, int nvec,
                          double* out_slots, double* seg_out, int seg_d, int seg_cols, double* scratch_cplx,
                          cudaStream_t s);

// Fused decrypt side of the ZeRo-MOAI delta, one CTA per vector v (a
// ciphertext-plaintext product): INTT of limbs 0 and 1 of
// c0*p + (c1*p)*s = p*(c0 + c1*s), CRT to f64 / scale, and the segment sums
// of the decoded slots as the linear functional seg[c] = sum_j coeff_j W[c][j]
// (W[c][j] = sum over the segment's slots k of cos(pi j (2k+1) / N)).
// sks / pts hold the Shoup companions of the keys / plaintexts.
// Supports seg_cols <= kMaxSegCols.  M0 is u64 scratch: [nvec][n] from
// N = 8192 (the split form's limb-1 INTT outputs), else [min(nvec, sms)][n]
// (one limb per persistent group); U (from N = 8192 only) is
// [nvec / per_ct][2][n], the rows of c0 + c1*s of limbs 0 and 1.
constexpr int kMaxSegCols = 10;
cudaError_t launch_dec_fused(const DevCtx& c, const uint64_t* cts, long long ct_stride, int ct_limbs,
                             const uint64_t* sk, const uint64_t* sks, const int* sk_of, const uint64_t* pt,
                             const uint64_t* pts, const int* pt_sel, int per_ct,
                             int nvec, double inv_scale, const double* W, int seg_cols, uint64_t* M0, uint64_t* U,
                             double* seg_out, cudaStream_t s);

// seg_out[v][c] = sum_j CRT(M[v][0][j], M[v][1][j]) * inv_scale * W[c][j]:
// the back half of the fused decrypt for INTT outputs already in M.
cudaError_t launch_crt_seg(const DevCtx& c, const uint64_t* M, int nvec, double inv_scale, const double* W,
                           int seg_cols, double* seg_out, cudaStream_t s, const char* scope = "crt_seg");

// delta[i][d] = sum_k B[d][k] * inter[i][k] (inference_engine.py:1392).
cudaError_t launch_bmat(const float* B, const double* inter, double* delta, int nvec, int d, int r,
                        const int* b_sel, long long b_stride, cudaStream_t s);

// Gather per-batch segment sums into intermediate[i][r].
cudaError_t launch_gather_inter(const double* seg, double* inter, int ndelta, int nb, int cols, int r,
                                cudaStream_t s);

// DP noise (inference_engine.py:1436-1456): clip ||h||_2 <= C, add N(0, sigma^2)
// from the stream of seeds[v]; h is [nvec][d] f64 (in place).
cudaError_t launch_dp_noise(double* h, int nvec, int d, double clip, double sigma, const uint64_t* seeds,
                            cudaStream_t s);

}  // namespace tsg
