// noalloc.cu -- decrypt for callers that must not allocate device memory.
//
// Some hosts cannot call cudaMalloc (or any allocating routine) once they are
// serving: an inference server that reserves all device memory for the model
// and its KV cache at start-up and forbids later allocations, or a plugin
// host whose device heap is owned by another framework's caching allocator
// (an allocation there can fail under memory pressure or block on the
// allocator's lock in the middle of a token).  ts_decrypt_noalloc gives them
// the decrypt of ts_decrypt with every temporary buffer taken from one
// fixed, file-scope device array instead of from an allocator.
//
// The array (kScratchBytes = 2 MiB) is part of the library image: every GPU
// that loads this code holds it until the process exits.  Under CUDA's lazy
// module loading (the default from CUDA 12.2) a module is loaded, and its
// __device__ arrays allocated, on first use; ts_ctx_create therefore
// resolves the array's address on the context's device (noalloc_prepare),
// so the 2 MiB are taken when the context is made at start-up, not at the
// first decrypt.  If that early resolve fails (the device was already full),
// context creation still succeeds and the first ts_decrypt_noalloc call on
// that device retries it.  All calls share
// it and it keeps the last call's contents; nothing in it has to start at
// zero, because each call writes every byte it later reads.  Calls that
// overlap on the GPU (two streams, or two contexts on one device) race on
// the array and must be serialized by the caller.
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/tsgpu.h"
#include "kernels.cuh"

using namespace tsg;

namespace {

constexpr size_t kScratchBytes = 2u << 20;  // 2 MiB per device
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_sym_mu;
void* g_sym_addr[64] = {};  // device address of g_noalloc_scratch, per device

// Device address of the array on `device`, which must be current; resolved
// once per device and cached.
cudaError_t scratch_address(int device, void** out) {
    if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> g(g_sym_mu);
    if (!g_sym_addr[device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        g_sym_addr[device] = p;
    }
    *out = g_sym_addr[device];
    return cudaSuccess;
}

}  // namespace

namespace tsg_host {
// Called by context creation with `device` current: loads the array on that
// device.  A failure is not fatal there (the error is cleared and the first
// ts_decrypt_noalloc call on the device tries again).
void noalloc_prepare(int device) {
    void* p = nullptr;
    if (scratch_address(device, &p) != cudaSuccess) cudaGetLastError();
}
}  // namespace tsg_host

// Accessors implemented in tsgpu.cu (the opaque structs live there).
namespace tsg_host {
int noalloc_ctx(ts_ctx* c, int* device, const DevCtx** dc, cudaStream_t* stream, uint32_t* n, uint32_t* slots,
                std::mutex** mu);
int noalloc_ct(const ts_ct* ct, const ts_ctx** owner, uint32_t* count, uint32_t* limbs, double* scale,
               const uint64_t** d);
int noalloc_sk(const ts_sk* sk, const ts_ctx** owner, uint32_t* count, const uint64_t** d, const uint64_t** ds);
int noalloc_fail(int code, const char* msg);
}  // namespace tsg_host

extern "C" int ts_decrypt_noalloc(ts_ctx* ctx, const ts_ct* ct, const ts_sk* sk, double* out_dev) {
    using namespace tsg_host;
    if (!ctx || !ct || !sk || !out_dev) return noalloc_fail(TS_ERR_ARG, "ts_decrypt_noalloc: NULL argument");
    int device = 0;
    const DevCtx* dc = nullptr;
    cudaStream_t stream = nullptr;
    uint32_t n = 0, slots = 0, count = 0, limbs = 0, kcount = 0;
    double scale = 0.0;
    std::mutex* mu = nullptr;
    const ts_ctx *ct_owner = nullptr, *sk_owner = nullptr;
    const uint64_t *d_ct = nullptr, *d_sk = nullptr, *d_sks = nullptr;
    int rc = noalloc_ctx(ctx, &device, &dc, &stream, &n, &slots, &mu);
    if (rc == TS_OK) rc = noalloc_ct(ct, &ct_owner, &count, &limbs, &scale, &d_ct);
    if (rc == TS_OK) rc = noalloc_sk(sk, &sk_owner, &kcount, &d_sk, &d_sks);
    if (rc != TS_OK) return noalloc_fail(rc, "ts_decrypt_noalloc: could not read the context, ciphertext or key");
    if (ct_owner != ctx || sk_owner != ctx)
        return noalloc_fail(TS_ERR_ARG, "ts_decrypt_noalloc: objects belong to another context");
    if (kcount < 1 || !d_sk || !d_ct || count < 1)
        return noalloc_fail(TS_ERR_ARG, "ts_decrypt_noalloc: empty key set or ciphertext");
    if (reinterpret_cast<uintptr_t>(out_dev) % 8)
        return noalloc_fail(TS_ERR_ARG, "ts_decrypt_noalloc: out_dev must be 8-byte aligned");
    // same CRT rule as ts_decrypt (ciphertext.rs:351)
    const bool crt = scale > dc->scale * 1.5 && limbs >= 2;
    const int nl = crt ? 2 : 1;
    const size_t m_bytes = ((size_t)count * nl * n * 8 + 255) & ~(size_t)255;
    const size_t f_bytes = (size_t)count * 2 * n * 8;
    if (m_bytes + f_bytes > kScratchBytes) {
        char msg[256];
        snprintf(msg, sizeof(msg),
                 "ts_decrypt_noalloc: %u ciphertexts at N=%u need %zu scratch bytes, above the fixed %zu-byte "
                 "buffer; decrypt fewer ciphertexts per call",
                 count, n, m_bytes + f_bytes, kScratchBytes);
        return noalloc_fail(TS_ERR_ARG, msg);
    }
    std::lock_guard<std::mutex> lk(*mu);
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return noalloc_fail(TS_ERR_CUDA, cudaGetErrorString(e));
    // the array's device address on this device (resolved by context
    // creation; resolved here, with the device current, if that failed)
    if (device < 0 || device >= 64) return noalloc_fail(TS_ERR_ARG, "ts_decrypt_noalloc: device id >= 64");
    void* base = nullptr;
    e = scratch_address(device, &base);
    if (e != cudaSuccess) return noalloc_fail(TS_ERR_CUDA, cudaGetErrorString(e));
    uint64_t* M = static_cast<uint64_t*>(base);
    double* fft = reinterpret_cast<double*>(static_cast<char*>(base) + m_bytes);
    e = launch_decrypt_limbs(*dc, M, nl, d_ct, (long long)2 * limbs * n, (int)limbs, d_sk, d_sks, nullptr, nullptr, nullptr, 1,
                             (int)count, stream);
    if (e == cudaSuccess)
        e = launch_decode(*dc, M, nl, crt, scale, (int)count, out_dev, nullptr, 0, 0, fft, stream);
    if (e != cudaSuccess) return noalloc_fail(TS_ERR_CUDA, cudaGetErrorString(e));
    return TS_OK;
}
