// The bf16 tensor-core ("fast") value network: tcgen05 MMAs with operands in
// 128-byte-swizzled shared memory and fp32 accumulators in TMEM, epilogues on
// the CUDA cores (bias, residual, LayerNorm, tanh-GELU).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "device.h"
#include "kernels.h"
#include "umma.cuh"

namespace wcdev {

// ---------------------------------------------------------------- selftest
// D[128, N] = A[128, K] * B[N, K]^T through one CTA's tcgen05 path: checks the
// descriptors, the swizzle and the TMEM read-out against a host product.
__global__ void k_umma_selftest(const __nv_bfloat16* __restrict__ A, const __nv_bfloat16* __restrict__ B, int K,
                                int N, float* __restrict__ D, int* __restrict__ status) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t mbar;
    __shared__ uint32_t tmem_slot;
    uint8_t* smem = smem_raw + ((1024u - (umma::smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sA = smem;
    uint8_t* sB = smem + 128 * K * 2;
    const int tid = threadIdx.x, warp = tid / 32;
    // stage operands, 8 bf16 (16 bytes) at a time
    for (int q = tid; q < 128 * K / 8; q += blockDim.x) {
        int r = q / (K / 8), k = (q % (K / 8)) * 8;
        *reinterpret_cast<uint4*>(sA + umma::sw128_offset(128, r, k)) =
            *reinterpret_cast<const uint4*>(A + (size_t)r * K + k);
    }
    for (int q = tid; q < N * K / 8; q += blockDim.x) {
        int r = q / (K / 8), k = (q % (K / 8)) * 8;
        *reinterpret_cast<uint4*>(sB + umma::sw128_offset(N, r, k)) =
            *reinterpret_cast<const uint4*>(B + (size_t)r * K + k);
    }
    if (tid == 0) {
        umma::mbar_init(&mbar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    uint32_t ncols = 32;
    while (ncols < (uint32_t)N) ncols <<= 1;
    if (warp == 0) umma::tmem_alloc(&tmem_slot, ncols);
    umma::fence_async_smem();
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = tmem_slot;
    if (tid == 0) {
        const uint32_t idesc = umma::idesc_bf16(128, N);
        for (int k0 = 0; k0 < K; k0 += 16)
            umma::mma_bf16(tmem, umma::desc_at(umma::smem_u32(sA), 128, k0), umma::desc_at(umma::smem_u32(sB), N, k0),
                           idesc, k0 > 0);
        umma::commit(&mbar);
    }
    bool ok = umma::mbar_wait(&mbar, 0);
    umma::fence_after_sync();
    if (!ok) {
        if (tid == 0) *status = 1;
    } else {
        float v[32];
        for (int c = 0; c < N; c += 32) {
            umma::tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + c, v);
            for (int j = 0; j < 32 && c + j < N; ++j) D[(size_t)tid * N + c + j] = v[j];
        }
    }
    umma::fence_before_sync();
    __syncthreads();
    if (warp == 0) umma::tmem_dealloc(tmem, ncols);
}

int umma_selftest(const uint16_t* A, const uint16_t* B, int K, int N, float* D) {
    if (K % 64 || N % 16 || N < 16 || N > 256) return 1;
    __nv_bfloat16 *dA, *dB;
    float* dD;
    int* dS;
    cudaMalloc(&dA, 128ull * K * 2);
    cudaMalloc(&dB, (size_t)N * K * 2);
    cudaMalloc(&dD, 128ull * N * 4);
    cudaMalloc(&dS, 4);
    cudaMemcpy(dA, A, 128ull * K * 2, cudaMemcpyHostToDevice);
    cudaMemcpy(dB, B, (size_t)N * K * 2, cudaMemcpyHostToDevice);
    cudaMemset(dS, 0, 4);
    size_t smem = 128ull * K * 2 + (size_t)N * K * 2 + 1024;
    cudaFuncSetAttribute(k_umma_selftest, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_umma_selftest<<<1, 128, smem>>>(dA, dB, K, N, dD, dS);
    int status = 0;
    cudaError_t e = cudaDeviceSynchronize();
    cudaMemcpy(D, dD, 128ull * N * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(&status, dS, 4, cudaMemcpyDeviceToHost);
    cudaFree(dA);
    cudaFree(dB);
    cudaFree(dD);
    cudaFree(dS);
    if (e != cudaSuccess) return 2;
    return status ? 3 : 0;
}

}  // namespace wcdev
