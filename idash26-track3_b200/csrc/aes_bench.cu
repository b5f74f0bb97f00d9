// AES throughput probe: the ceiling the DCF kernels are measured against.
// Each thread hashes its own chain of `iters` blocks with the tree-hash key
// (one fixed-key AES per step, exactly the per-level work of a DCF level).
#include "aes_dev.cuh"
#include "common.cuh"
#include "gates.cuh"

namespace ddg {

template <class E>
__global__ void __launch_bounds__(E::THREADS, E::CTAS) aes_chain_kernel(uint64_t threads, int iters, uint32_t *out)
{
    extern __shared__ uint32_t smem_tab[];
    E::stage(smem_tab);
    __syncthreads();
    E A(smem_tab);
    for (uint64_t t = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < threads; t += uint64_t(gridDim.x) * blockDim.x) {
        Blk b;
        b.w[0] = uint32_t(t), b.w[1] = uint32_t(t >> 32), b.w[2] = 0x9e3779b9u, b.w[3] = 0x7f4a7c15u;
#pragma unroll 1
        for (int i = 0; i < iters; i++) b = A.hash_h(b);
        out[t] = b.w[0] ^ b.w[1] ^ b.w[2] ^ b.w[3];
    }
}

template <class E>
static int chain_launch(uint64_t threads, int iters, uint32_t *out, cudaStream_t st)
{
    DDG_CUDA(cudaFuncSetAttribute(aes_chain_kernel<E>, cudaFuncAttributeMaxDynamicSharedMemorySize, E::SMEM));
    aes_chain_kernel<E><<<aes_blocks<E>(threads), E::THREADS, E::SMEM, st>>>(threads, iters, out);
    return DDG_OK;
}

// variant: 0 = the engine the library currently uses, 2 / 4 = that many staged tables
int aes_chain(uint64_t threads, int iters, uint32_t *out, cudaStream_t st, int variant)
{
    DDG_TRY(aes_device_init());
    const int nt = variant == 0 ? aes_tables() : variant;
    DDG_TRY((nt == 4 ? chain_launch<AesLane4>(threads, iters, out, st) : chain_launch<AesLane2>(threads, iters, out, st)));
    note_launch();
    DDG_CUDA(cudaGetLastError());
    return DDG_OK;
}

}  // namespace ddg
