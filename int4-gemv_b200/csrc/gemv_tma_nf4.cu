// Instantiations of the streaming (bulk-copy ring) NF4 GEMV kernel.
#include "b4_gemv_tma_nf4.cuh"

void* b4::gemv_kernel_nf4_tma(int rw, int vw, int stages)
{
#define B4_TMA_NF4_PICK(RW, VW, ST) \
    if (rw == RW && vw == VW && stages == ST) return (void*)&b4::b4_gemv_tma_nf4_kernel<RW, VW, ST>;
    B4_TMA_NF4_PICK(4, 2, 4)
    B4_TMA_NF4_PICK(4, 2, 8)
    B4_TMA_NF4_PICK(8, 2, 4)
    B4_TMA_NF4_PICK(8, 2, 6)
    B4_TMA_NF4_PICK(16, 2, 4)
    B4_TMA_NF4_PICK(4, 4, 4)
    B4_TMA_NF4_PICK(8, 4, 4)
#undef B4_TMA_NF4_PICK
    return nullptr;
}
