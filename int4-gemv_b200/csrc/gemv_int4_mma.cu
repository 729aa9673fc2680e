// Instantiations of the tensor-pipe INT4 GEMV kernel.
#include "b4_gemv_mma.cuh"

void* b4::gemv_kernel_int4_mma(int rt, int nt)
{
    if (rt == 1 && nt == 1) return (void*)&b4::b4_gemv_mma_kernel<1, 1>;
    if (rt == 2 && nt == 1) return (void*)&b4::b4_gemv_mma_kernel<2, 1>;
    if (rt == 1 && nt == 2) return (void*)&b4::b4_gemv_mma_kernel<1, 2>;
    if (rt == 2 && nt == 2) return (void*)&b4::b4_gemv_mma_kernel<2, 2>;
    return nullptr;
}
