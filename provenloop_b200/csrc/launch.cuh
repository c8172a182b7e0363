// launch.cuh -- helpers shared by the kernel translation units (kernels.cu,
// k_ntt.cu, k_encode.cu, k_encrypt.cu, k_decrypt.cu): launch bookkeeping,
// cluster launches, and the device-side stream-flag / ChaCha-window / scan
// helpers.  The sources are split so that nvcc compiles them in parallel;
// each kernel still compiles whole within its own file.
#pragma once
#include <cooperative_groups.h>

#include "kernels.cuh"

namespace tsg {

// Raises a kernel's dynamic shared-memory limit to at least `bytes` on the
// current device (launchers of one kernel may need different sizes); the
// limits already set are remembered per (kernel, device) in kernels.cu.
cudaError_t ensure_smem_raw(const void* kernel, size_t bytes);
template <class K>
inline cudaError_t ensure_smem(K* kernel, size_t bytes) {
    return ensure_smem_raw(reinterpret_cast<const void*>(kernel), bytes);
}

// Counts the kernels launched in its scope and, when profiling is on,
// brackets them with an event pair on the launch stream (kernels.cu).
struct KScope {
    const char* name;
    cudaStream_t s;
    int kernels;
    cudaEvent_t a = nullptr, b = nullptr;
    KScope(const char* n, cudaStream_t st, int k = 1);
    ~KScope();
    KScope(const KScope&) = delete;
    KScope& operator=(const KScope&) = delete;
};

namespace {

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

}  // namespace

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

}  // namespace tsg
