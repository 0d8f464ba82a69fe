// peak.cu -- throughput ceilings measured on the device this library runs on.
//
// The roofline of the 3xTF32 SGEMM needs the tensor core's kind::tf32 rate,
// and that of the exact SIMT kernels the FP32 FFMA rate; neither is the cuBLAS
// bf16 figure.  These kernels measure them the way the reference measured its
// own FMA ceiling with a microbenchmark (lakitu12/vkblas test/fma_peak.c,
// test/fma_peak.comp): nothing but the instruction under test, in a loop,
// timed by the caller with CUDA events.
//
//   PEAK_FFMA        fp32 FFMA: 8 independent fmaf chains per thread, every SM.
//   PEAK_TF32        tcgen05.mma.cta_group::1.kind::tf32, M=128 N=256 K=8
//   PEAK_TF32_PAIR   tcgen05.mma.cta_group::2.kind::tf32, M=256 N=256 K=8
//   PEAK_F16         tcgen05.mma.cta_group::1.kind::f16,  M=128 N=256 K=16
//   PEAK_F16_PAIR    tcgen05.mma.cta_group::2.kind::f16,  M=256 N=256 K=16
//
// MMA kernels: one CTA per SM (one 2-CTA cluster per SM pair), operands are a
// fixed K-major SWIZZLE_128B tile in shared memory filled with finite values,
// and one thread issues `iters` rounds of 4 MMAs (one 128-byte k block) into
// two alternating TMEM accumulators.  The only wait is the final commit,
// bounded like every wait of this library: on timeout a status code is
// recorded and the CTA leaves.
#include "common.cuh"
#include "umma.cuh"
#include "vkblas_b200.h"

namespace vkb {
namespace {

using namespace umma;

constexpr uint64_t PEAK_WAIT_NS = 2000000000ull;        // 2 s
constexpr uint32_t PEAK_SMEM = 160u * 1024u;            // forces one CTA per SM

__global__ void __launch_bounds__(256) peak_ffma_kernel(uint32_t iters, float seed, int* sink) {
    float a[8];
#pragma unroll
    for (int i = 0; i < 8; i++) a[i] = seed + (float)(threadIdx.x + i);
    const float m = 0.999999f, c = 1e-7f;
    for (uint32_t it = 0; it < iters; it++) {
#pragma unroll
        for (int u = 0; u < 16; u++)
#pragma unroll
            for (int i = 0; i < 8; i++) a[i] = fmaf(a[i], m, c);
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) s += a[i];
    // The chains stay positive, so this never adds; the test keeps them alive.
    if (s < 0.f) atomicAdd(sink, 0);
}

// kind: 0 = tf32, 1 = f16.  PAIR: cta_group::2 on a 2-CTA cluster.
template <int KIND, bool PAIR>
__global__ void __launch_bounds__(128, 1) peak_mma_kernel(uint32_t iters, int* status) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t pad = (1024u - (raw & 1023u)) & 1023u;
    uint8_t* smem = smem_raw + pad;
    const uint32_t sA = raw + pad;                       // 128 rows x 128 B
    const uint32_t sB = sA + 128u * 128u;                // 256 (128 per CTA of a pair) rows x 128 B
    constexpr uint32_t B_ROWS = PAIR ? 128u : 256u;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 128u * 128u + B_ROWS * 128u);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
    const uint32_t bar_a = smem_u32(bar);
    const int warp = threadIdx.x >> 5;

    // Operand tiles: finite values of magnitude < 1 (tf32: fp32 words with the
    // low 13 bits clear; f16: pairs of halves).
    uint32_t* w = reinterpret_cast<uint32_t*>(smem);
    const uint32_t words = (128u + B_ROWS) * 128u / 4u;
    for (uint32_t i = threadIdx.x; i < words; i += blockDim.x) {
        const uint32_t h = (i * 2654435761u) ^ (blockIdx.x * 40503u);
        if (KIND == 0) {
            w[i] = (0x3E000000u | (h & 0x007FE000u)) ^ ((h & 1u) << 31);   // +-[0.125, 0.25)
        } else {
            const uint32_t lo = 0x3000u | (h & 0x03FFu), hi = 0x3000u | ((h >> 10) & 0x03FFu);
            w[i] = lo | (hi << 16) | ((h & 1u) << 15);                       // +-[0.125, 0.25)
        }
    }
    if (threadIdx.x == 0) {
        mbar_init(bar_a, 1);
        fence_barrier_init();
    }
    fence_proxy_async_smem();
    if (warp == 0) {
        if constexpr (PAIR) {
            tmem_alloc_pair(smem_u32(tmem_slot), 512);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(smem_u32(tmem_slot), 512);
            tmem_relinquish();
        }
    }
    __syncthreads();
    if constexpr (PAIR) cluster_sync();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const bool issuer = !PAIR || cluster_ctarank() == 0;
    if (threadIdx.x == 0 && issuer) {
        constexpr uint32_t M = PAIR ? 256u : 128u;
        const uint32_t idesc = instr_desc(KIND == 0 ? 2u : 0u, false, false, M, 256u);
        uint64_t ad[4], bd[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            ad[j] = smem_desc_sw128(sA + j * 32, 16, 1024);
            bd[j] = smem_desc_sw128(sB + j * 32, 16, 1024);
        }
        for (uint32_t it = 0; it < iters; it++) {
            const uint32_t d = tmem + (it & 1u) * 256u;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const uint32_t acc = (it < 2 && j == 0) ? 0u : 1u;
                if constexpr (KIND == 0) {
                    if constexpr (PAIR) mma_tf32_pair(d, ad[j], bd[j], idesc, acc);
                    else mma_tf32(d, ad[j], bd[j], idesc, acc);
                } else {
                    if constexpr (PAIR) mma_f16_pair(d, ad[j], bd[j], idesc, acc);
                    else mma_f16(d, ad[j], bd[j], idesc, acc);
                }
            }
        }
        if constexpr (PAIR) tc_commit_pair_mc(bar_a, 0x3);
        else tc_commit(bar_a);
    }
    // Every CTA waits for the commit (both CTAs of a pair receive it).
    if (threadIdx.x == 0) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(bar_a, 0)) {
            if (globaltimer_ns() - t0 > PEAK_WAIT_NS) {
                atomicCAS(status, 0, DS_TIMEOUT_MMA);
                break;
            }
        }
    }
    __syncthreads();
    if constexpr (PAIR) cluster_sync();
    if (warp == 0) {
        tc_fence_after();
        if constexpr (PAIR) tmem_dealloc_pair(tmem, 512);
        else tmem_dealloc(tmem, 512);
    }
}

template <int KIND, bool PAIR>
cudaError_t launch_peak_mma(uint32_t iters, int num_sms, int* status, cudaStream_t s) {
    auto kern = peak_mma_kernel<KIND, PAIR>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)PEAK_SMEM);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(PAIR ? (uint32_t)(num_sms & ~1) : (uint32_t)num_sms);
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = PEAK_SMEM;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = PAIR ? 2 : 1;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, iters, status);
}

}  // namespace
}  // namespace vkb

extern "C" __attribute__((visibility("default"))) vkblas_status_t vkblas_b200_peak_launch(
    int which, uint32_t iters, void* stream, int* status, double* flops) {
    using namespace vkb;
    if (iters == 0 || !status || !flops) return VKBLAS_ERR_PARAM;
    int dev = 0, sms = 0, major = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        major != 10) {
        cudaGetLastError();
        return VKBLAS_ERR_INIT;
    }
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e;
    const int pairs_sms = sms & ~1;
    switch (which) {
        case VKBLAS_PEAK_FFMA: {
            const uint32_t blocks = (uint32_t)sms * 8u;          // 2048 threads per SM
            peak_ffma_kernel<<<blocks, 256, 0, s>>>(iters, 1.0f, status);
            e = cudaGetLastError();
            *flops = 2.0 * 8 * 16 * (double)iters * blocks * 256;
            break;
        }
        case VKBLAS_PEAK_TF32:
            e = launch_peak_mma<0, false>(iters, sms, status, s);
            *flops = 2.0 * 128 * 256 * 32 * (double)iters * sms;
            break;
        case VKBLAS_PEAK_TF32_PAIR:
            e = launch_peak_mma<0, true>(iters, sms, status, s);
            *flops = 2.0 * 128 * 256 * 32 * (double)iters * pairs_sms;
            break;
        case VKBLAS_PEAK_F16:
            e = launch_peak_mma<1, false>(iters, sms, status, s);
            *flops = 2.0 * 128 * 256 * 64 * (double)iters * sms;
            break;
        case VKBLAS_PEAK_F16_PAIR:
            e = launch_peak_mma<1, true>(iters, sms, status, s);
            *flops = 2.0 * 128 * 256 * 64 * (double)iters * pairs_sms;
            break;
        default:
            return VKBLAS_ERR_PARAM;
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return VKBLAS_ERR_INIT;
    }
    return VKBLAS_OK;
}
