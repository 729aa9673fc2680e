// Instantiations of the batch-1 NF4 tensor-pipe GEMV (register load pipeline
// of depth 2, 3 or 4; deeper spills).
#include "b4_gemv_nf4_mma.cuh"

void* b4::gemv_kernel_nf4_mma(int depth)
{
    switch (depth) {
        case 2: return (void*)&b4::b4_gemv_nf4_mma_kernel<2>;
        case 3: return (void*)&b4::b4_gemv_nf4_mma_kernel<3>;
        case 4: return (void*)&b4::b4_gemv_nf4_mma_kernel<4>;
    }
    return nullptr;
}

// the row-parallel shard with the all-reduce fused in (b4_tp_gemv_p2p)
void* b4::gemv_kernel_nf4_mma_p2p(int depth)
{
    switch (depth) {
        case 2: return (void*)&b4::b4_gemv_nf4_mma_kernel<2, 1>;
        case 3: return (void*)&b4::b4_gemv_nf4_mma_kernel<3, 1>;
        case 4: return (void*)&b4::b4_gemv_nf4_mma_kernel<4, 1>;
    }
    return nullptr;
}
