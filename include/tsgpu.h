/*
 * tsgpu.h -- C ABI of the B200-native CKKS engine for TenSafe's encrypted
 * LoRA-delta hot path (libtsgpu.so).
 *
 * The entry points replace the PyO3 binding `tensafe_he`
 * (tensafe-he/crates/tensafe-he-python/src/lib.rs) method for method, and
 * add batched / device-pointer entry points for the ZeRo-MOAI delta
 * (demonstrator/server/inference_engine.py:1197-1405).  Everything runs as
 * CUDA kernels on the context's device; there is no CPU compute fallback.
 *
 * Conventions
 *   - Every function returns TS_OK (0) or a negative TS_ERR_* code; the
 *     message of the calling thread's last error is in ts_last_error().
 *   - Polynomials are uint64 residues, limb-major: [num_limbs][n].  A
 *     ciphertext object holds `count` ciphertexts, each [2][num_limbs][n]
 *     (c0 then c1), NTT domain, as in ciphertext.rs:18-27.
 *   - Host pointers unless a parameter is named *_dev or a flag says so.
 *   - Calls on one context are serialized by the context (internal lock);
 *     distinct contexts may be used concurrently from different threads.
 *   - Results written to host memory are complete when the call returns;
 *     results written to device memory are ordered on the context's stream
 *     (ts_ctx_get_stream / ts_ctx_set_stream).
 */
#ifndef TSGPU_H
#define TSGPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TS_OK 0
#define TS_ERR_ARG (-1)         /* invalid argument / size (Rust assert!)   */
#define TS_ERR_OOM (-2)         /* device allocation failed                  */
#define TS_ERR_CUDA (-3)        /* CUDA runtime error                        */
#define TS_ERR_UNSUPPORTED (-4) /* unsupported degree (PyValueError)         */
#define TS_ERR_SCALE (-5)       /* scale mismatch in ct_add/ct_sub           */
#define TS_ERR_STATE (-6)       /* sampling plan overflow, bad handle state  */
#define TS_ERR_NODEVICE (-7)    /* no CUDA device                            */

typedef struct ts_ctx ts_ctx; /* CkksContext            lib.rs:19-24          */
typedef struct ts_sk ts_sk;   /* TenSafeSecretKey       lib.rs:298-301 (xN)   */
typedef struct ts_pk ts_pk;   /* TenSafePublicKey       lib.rs:304-307        */
typedef struct ts_ct ts_ct;   /* TenSafeCiphertext      lib.rs:310-317 (xN)   */
typedef struct ts_pt ts_pt;   /* cached NTT(plaintext)  ciphertext.rs:539-545 */
typedef struct ts_lora ts_lora; /* packed LoRA-A plaintexts + B, per expert
                                   inference_engine.py:1037-1074            */

/* ------------------------------------------------------------ library */
const char* ts_last_error(void);
int ts_version(void);
int ts_device_count(int* out);

/* Diagnostics: kernels this library launched in the process so far, and
 * optional CUDA-event timing of every launch by kernel name ("encrypt_limb",
 * "decrypt_limb", "ntt_forward", "decode_a", ...). */
int ts_launch_count(uint64_t* out);
int ts_profile_enable(int on);
int ts_profile_reset(void);
/* Total event-timed ms and launches of `kernel` since the last reset;
 * TS_ERR_ARG if it was not launched. */
int ts_profile_read(const char* kernel, double* ms, uint64_t* launches);

/* ------------------------------------------------------------ host-only */
/* CkksParams::custom prime chain (params.rs:142-193) without a device. */
int ts_params_custom(uint32_t poly_degree, const uint32_t* modulus_bits, uint32_t num_limbs, uint64_t* moduli_out);
/* The tables a context would upload for (N, q): fw / iw [n] (rns.rs:161-185)
 * and the FFT twist / stage tables [n] (encoding.rs:38-80).  No device
 * needed.  Any pointer may be NULL. */
int ts_host_tables(uint32_t poly_degree, uint64_t q, uint64_t* fw, uint64_t* iw, double* twist_re,
                   double* twist_im, double* tw_re, double* tw_im);

/* ------------------------------------------------------------ context */
/* CkksContext(poly_mod_degree) -- lib.rs:35-56 (CkksParams::for_degree,
 * params.rs:66-136): N in {8192, 16384, 32768}, else TS_ERR_UNSUPPORTED. */
int ts_ctx_create(uint32_t poly_mod_degree, int device, ts_ctx** out);
/* CkksParams::custom -- params.rs:142-193: one descending NTT-friendly prime
 * search per width (equal widths repeat the same prime, as there). */
int ts_ctx_create_custom(uint32_t poly_degree, const uint32_t* modulus_bits, uint32_t num_limbs,
                         uint32_t scale_bits, int device, ts_ctx** out);
/* Explicit prime chain (test and benchmark parameter sets). */
int ts_ctx_create_moduli(uint32_t poly_degree, const uint64_t* moduli, uint32_t num_limbs, int device,
                         ts_ctx** out);
int ts_ctx_destroy(ts_ctx* ctx);
/* num_slots / poly_mod_degree getters (lib.rs:78-88), get_backend_info
 * (lib.rs:282-294).  moduli may be NULL. */
int ts_ctx_info(const ts_ctx* ctx, uint32_t* poly_degree, uint32_t* num_slots, uint32_t* num_limbs,
                uint64_t* moduli);
int ts_ctx_get_stream(ts_ctx* ctx, void** cuda_stream);
/* Issue all work on an external cudaStream_t from now on (0 is the legacy
 * default stream); ts_ctx_reset_stream returns to the context's own
 * non-blocking stream. */
int ts_ctx_set_stream(ts_ctx* ctx, void* cuda_stream);
int ts_ctx_reset_stream(ts_ctx* ctx);
int ts_ctx_synchronize(ts_ctx* ctx);
/* Device counters: [0] near-tie Gaussian samples, [1] streams repaired after
 * a rejection, [2] plan overflows, [3] reserved. */
int ts_ctx_stats(ts_ctx* ctx, uint64_t out[4]);
/* Export the host-computed tables (tests): fw, iw [n] for `limb`, FFT
 * twist/stage tables [n] each.  Any pointer may be NULL. */
int ts_ctx_tables(const ts_ctx* ctx, uint32_t limb, uint64_t* fw, uint64_t* iw, double* twist_re,
                  double* twist_im, double* tw_re, double* tw_im);

/* ------------------------------------------------------------ keys */
/* keygen(seed) -- lib.rs:91-99, ciphertext.rs:77-103.  ts_keygen_batch makes
 * `count` independent keys (one per seed) in one object. */
int ts_keygen(ts_ctx* ctx, uint64_t seed, ts_sk** out);
int ts_keygen_batch(ts_ctx* ctx, const uint64_t* seeds, uint32_t count, ts_sk** out);
int ts_sk_destroy(ts_sk* sk);
int ts_sk_count(const ts_sk* sk, uint32_t* count);
/* Copy key `index` ([L][n], NTT domain) to host memory (tests). */
int ts_sk_export(const ts_sk* sk, uint32_t index, uint64_t* host);

/* ------------------------------------------------------------ ciphertexts */
/* encrypt(data, sk, seed) -- lib.rs:116-138, ciphertext.rs:167-229: data is
 * padded / truncated to num_slots.  One fresh stream per call. */
int ts_encrypt(ts_ctx* ctx, const ts_sk* sk, const double* data, size_t len, uint64_t seed, ts_ct** out);
/* `count` vectors (row stride `stride` doubles), independent seeds[i]; key
 * sk_index[i] of sk (NULL: key 0).  data_on_device: data is a device ptr. */
int ts_encrypt_batch(ts_ctx* ctx, const ts_sk* sk, const double* data, size_t count, size_t len, size_t stride,
                     const uint64_t* seeds, const int32_t* sk_index, int data_on_device, ts_ct** out);
/* batch_encrypt(arrays, sk, seed) -- lib.rs:231-258: ONE stream shared by
 * the arrays in order (the i-th array starts where the (i-1)-th stopped). */
int ts_encrypt_stream(ts_ctx* ctx, const ts_sk* sk, const double* data, size_t count, size_t len, size_t stride,
                      uint64_t seed, ts_ct** out);
/* Public-key path.  CkksContext::keygen_public (ciphertext.rs:114-154;
 * lib.rs:102-110): pk = (b, a) with a uniform and b = -a*s + e, both NTT
 * domain, from TenSafeRng::from_seed(seed); key sk_index of sk. */
int ts_keygen_public(ts_ctx* ctx, const ts_sk* sk, uint32_t sk_index, uint64_t seed, ts_pk** out);
int ts_pk_destroy(ts_pk* pk);
/* Copy b and a ([L][n] each, NTT domain) to host memory (either may be NULL). */
int ts_pk_export(const ts_pk* pk, uint64_t* b_host, uint64_t* a_host);
/* CkksContext::encrypt_pk (ciphertext.rs:240-319; lib.rs:142-164), batched:
 * `count` vectors (row stride `stride`), independent seeds[i];
 * c0 = b*u + m + e0, c1 = a*u + e1. */
int ts_encrypt_pk(ts_ctx* ctx, const ts_pk* pk, const double* data, size_t count, size_t len, size_t stride,
                  const uint64_t* seeds, int data_on_device, ts_ct** out);
/* CkksContext::rescale (ciphertext.rs:476-535; lib.rs:218-225): drop the last
 * limb, dividing by its modulus; scale / q_last.  TS_ERR_ARG with 1 limb. */
int ts_rescale(ts_ctx* ctx, const ts_ct* ct, ts_ct** out);
int ts_ct_destroy(ts_ct* ct);
int ts_ct_info(const ts_ct* ct, uint32_t* count, uint32_t* num_limbs, double* scale);
/* Copy ciphertext `index` to host: c0, c1 [num_limbs][n] (either may be NULL). */
int ts_ct_export(const ts_ct* ct, uint32_t index, uint64_t* c0, uint64_t* c1);
/* Build a one-ciphertext object from host residues. */
int ts_ct_import(ts_ctx* ctx, const uint64_t* c0, const uint64_t* c1, uint32_t num_limbs, double scale,
                 ts_ct** out);
/* Ciphertext `index` of a batch as its own object (device copy). */
int ts_ct_select(ts_ctx* ctx, const ts_ct* ct, uint32_t index, ts_ct** out);

/* Wire format (tensafe-he-core serialize.rs:14-93; no PyO3 method): an
 * RnsPoly is limb-major little-endian u64, a ciphertext [scale f64 LE | c0 |
 * c1], a public key [b | a].
 * ts_ct_to_bytes -- serialize.rs:71-77 ct_to_bytes, for every ciphertext of
 * the object, blobs back to back (count * (8 + 2 * num_limbs * n * 8) bytes;
 * TS_ERR_ARG if out_len is smaller).  *written (may be NULL) gets the size. */
int ts_ct_to_bytes(const ts_ct* ct, uint8_t* out, size_t out_len, size_t* written);
/* serialize.rs:80-93 ct_from_bytes(bytes, n, num_limbs): len must be a
 * positive multiple of 8 + 2 * num_limbs * n * 8 (TS_ERR_ARG otherwise, the
 * reference's assert_eq!); several blobs give one object of as many
 * ciphertexts, which must share their scale.  Words above q_l are refused
 * (TS_ERR_ARG), where the reference would accept and compute on them. */
int ts_ct_from_bytes(ts_ctx* ctx, const uint8_t* bytes, size_t len, uint32_t num_limbs, ts_ct** out);
/* serialize.rs:48-52 pk_to_bytes: 2 * L * n * 8 bytes. */
int ts_pk_to_bytes(const ts_pk* pk, uint8_t* out, size_t out_len, size_t* written);
/* serialize.rs:55-67 pk_from_bytes(bytes, n, L): len must be 2 * L * n * 8;
 * words above q_l are refused. */
int ts_pk_from_bytes(ts_ctx* ctx, const uint8_t* bytes, size_t len, ts_pk** out);

/* decrypt(ct, sk) -- lib.rs:167-175, ciphertext.rs:327-400: writes
 * count * num_slots doubles (row i = ciphertext i).  sk_index as above. */
int ts_decrypt(ts_ctx* ctx, const ts_ct* ct, const ts_sk* sk, const int32_t* sk_index, double* out,
               int out_on_device);

/* Decrypt without allocating -- no counterpart in the reference.  For
 * callers that cannot allocate device memory while serving (a server that
 * reserves the whole device for its model and KV cache at start-up, or a
 * plugin host whose device heap belongs to another framework's allocator):
 * same result as ts_decrypt with key 0 of `sk`, written to out_dev (device
 * memory, count * num_slots doubles), with all temporaries in one fixed
 * 2 MiB device array that the library holds on every GPU it is loaded on.
 * At N = 16384 that fits 4 ciphertexts after ct x pt (CRT, 2 limbs) or 5
 * fresh ones per call; larger requests fail with TS_ERR_ARG.  The work is
 * queued on the context's stream and the call returns without waiting.
 * ts_ctx_create resolves the array's address on its device
 * (cudaGetSymbolAddress), which also loads the array under CUDA's lazy
 * module loading: create the context at start-up, before the host reserves
 * the rest of the device.  If that early resolve failed, the first call on
 * the device retries it, so make that first call before any stream capture.
 * Calls share the array: calls that overlap on the GPU race. */
int ts_decrypt_noalloc(ts_ctx* ctx, const ts_ct* ct, const ts_sk* sk, double* out_dev);

/* ct_pt_mul(ct, plaintext) -- lib.rs:178-195 / __mul__ lib.rs:336-356 /
 * ciphertext.rs:408-418: the plaintext (len <= num_slots doubles) is encoded
 * and transformed on the device, then multiplied into every ciphertext. */
int ts_ct_pt_mul(ts_ctx* ctx, const ts_ct* ct, const double* pt, size_t len, ts_ct** out);
/* encode_to_ntt -- ciphertext.rs:539-545, for `count` plaintext rows. */
int ts_encode_ntt(ts_ctx* ctx, const double* pts, size_t count, size_t len, size_t stride, int on_device,
                  ts_pt** out);
int ts_pt_destroy(ts_pt* pt);
int ts_pt_export(const ts_pt* pt, uint32_t index, uint64_t* host);
/* ct_pt_mul_ntt -- ciphertext.rs:422-429 with plaintext row pt_index. */
int ts_ct_pt_mul_ntt(ts_ctx* ctx, const ts_ct* ct, const ts_pt* pt, uint32_t pt_index, ts_ct** out);
/* ct_add / ct_sub -- ciphertext.rs:435-466 (TS_ERR_SCALE on mismatch). */
int ts_ct_add(ts_ctx* ctx, const ts_ct* a, const ts_ct* b, ts_ct** out);
int ts_ct_sub(ts_ctx* ctx, const ts_ct* a, const ts_ct* b, ts_ct** out);

/* ------------------------------------------------------------ raw kernels */
/* In-place batched NTT of n_polys polynomials [n_polys][limb_count][n] on the
 * device, limbs limb_offset .. limb_offset+limb_count-1 (ntt.rs:79-141). */
int ts_ntt_forward(ts_ctx* ctx, uint64_t* data_dev, size_t n_polys, uint32_t limb_count, uint32_t limb_offset);
int ts_ntt_inverse(ts_ctx* ctx, uint64_t* data_dev, size_t n_polys, uint32_t limb_count, uint32_t limb_offset);
/* out = a (.) b per limb (rns.rs:243-253); b_bcast: b is one [L][n] poly
 * applied to every poly of a. */
int ts_hadamard(ts_ctx* ctx, uint64_t* out_dev, const uint64_t* a_dev, const uint64_t* b_dev, size_t n_polys,
                uint32_t limb_count, int b_bcast);

/* ------------------------------------------------------------ ZeRo-MOAI */
/* Load `experts` LoRA adapters: lora_a [experts][r][d] f32, lora_b
 * [experts][d][r] f32 (host).  Packs A column-wise into cols = S / d rows per
 * plaintext (inference_engine.py:1037-1074) and caches NTT(plaintext) of all
 * limbs on the device. */
int ts_lora_load(ts_ctx* ctx, const float* lora_a, const float* lora_b, uint32_t experts, uint32_t r, uint32_t d,
                 ts_lora** out);
int ts_lora_destroy(ts_lora* lora);
/* Hot swap of expert `expert` -- swap_adapter, inference_engine.py:879-959
 * (the NTT(plaintext) cache rebuild of :1037-1074): lora_a [r][d] and
 * lora_b [d][r] f32 (host; the adapter's r and d) replace the expert's
 * packed plaintexts and B in place, so pointers a captured CUDA graph holds
 * stay valid.  Ordered on the context's stream and complete on return: work
 * queued on that stream before the call uses the old adapter, work after it
 * the new one.  Do not swap while another stream's work reads the adapter. */
int ts_lora_set_expert(ts_ctx* ctx, ts_lora* lora, uint32_t expert, const float* lora_a, const float* lora_b);
int ts_lora_info(const ts_lora* lora, uint32_t* experts, uint32_t* r, uint32_t* d, uint32_t* cols,
                 uint32_t* batches);
/* Encrypted LoRA deltas for n hidden states h [n][d] (f64): per state,
 * replicate h cols times, encrypt (seed seeds[i], key sk_index[i]), multiply
 * by expert expert[i]'s packed plaintexts, decrypt, sum each d-slot segment,
 * and apply B (inference_engine.py:1244-1392).  delta [n][d] f64,
 * intermediate [n][r] f64 (may be NULL).  expert / sk_index may be NULL (0).
 * io_on_device: 1 -- h / delta / intermediate are device pointers (the call
 * returns once the work is queued on the context's stream); 2 -- seeds,
 * expert and sk_index are device arrays as well, and the call then only
 * enqueues stream work (no host copies or waits, so it can be captured in a
 * CUDA graph once a first call has sized the context's scratch); their
 * values are not range-checked on the host. */
int ts_lora_delta_batch(ts_ctx* ctx, const ts_sk* sk, const ts_lora* lora, const double* h, uint32_t n,
                        const int32_t* expert, const int32_t* sk_index, const uint64_t* seeds, double* delta,
                        double* intermediate, int io_on_device);

/* Post-transformer DP noise (inference_engine.py:1436-1456) on the device:
 * clip each row of h [n][d] to L2 norm <= clip, add N(0, sigma^2) drawn from
 * the ChaCha20 stream of seeds[i] (Box-Muller as rng.rs:152-157).  With
 * on_device = 1, h is a device pointer and the call returns without waiting:
 * the result is ready in stream order on the context's stream; with
 * on_device = 2 the seeds are a device array too (stream work only). */
int ts_dp_noise(ts_ctx* ctx, double* h, uint32_t n, uint32_t d, double clip, double sigma, const uint64_t* seeds,
                int on_device);

#ifdef __cplusplus
}
#endif
#endif
