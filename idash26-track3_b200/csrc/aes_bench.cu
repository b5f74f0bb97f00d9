// AES throughput probe: the ceiling the DCF kernels are measured against.
// Each thread hashes its own chain of `iters` blocks with the tree-hash key
// (one fixed-key AES per step, exactly the per-level work of a DCF level).
#include "aes_dev.cuh"
#include "common.cuh"
#include "gates.cuh"

namespace ddg {

template <bool IMAD>
__global__ void __launch_bounds__(256, 3) aes_chain_kernel(uint64_t threads, int iters, uint32_t *out)
{
    extern __shared__ uint32_t smem_tab[];
    aes_stage_tables(smem_tab);
    __syncthreads();
    AesLane A(smem_tab);
    for (uint64_t t = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < threads; t += uint64_t(gridDim.x) * blockDim.x) {
        Blk b;
        b.w[0] = uint32_t(t), b.w[1] = uint32_t(t >> 32), b.w[2] = 0x9e3779b9u, b.w[3] = 0x7f4a7c15u;
#pragma unroll 1
        for (int i = 0; i < iters; i++) b = A.ccr<IMAD>(b, c_fixed.h.rk);
        out[t] = b.w[0] ^ b.w[1] ^ b.w[2] ^ b.w[3];
    }
}

// variant: 0 = the build's default round, 1 = shifts/PRMT only, 2 = multiply-add offload
int aes_chain(uint64_t threads, int iters, uint32_t *out, cudaStream_t st, int variant)
{
    DDG_TRY(aes_device_init());
    const bool imad = variant == 0 ? bool(DDG_AES_IMAD) : variant == 2;
    auto kern = imad ? aes_chain_kernel<true> : aes_chain_kernel<false>;
    DDG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, AES_SMEM_BYTES));
    int sms = device_sms();
    uint64_t need = (threads + 255) / 256, full = uint64_t(sms) * 3;
    kern<<<int(need < full ? need : full), 256, AES_SMEM_BYTES, st>>>(threads, iters, out);
    note_launch();
    DDG_CUDA(cudaGetLastError());
    return DDG_OK;
}

}  // namespace ddg
