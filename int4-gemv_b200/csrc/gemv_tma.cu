// Instantiations of the streaming (bulk-copy ring) INT4 GEMV kernel, and the
// reader of this translation unit's device error flag.
#include "b4_gemv_tma.cuh"

void* b4::gemv_kernel_int4_tma(int nt, int stages, int kcg)
{
#define B4_TMA_PICK(NT, ST, KCG) \
    if (nt == NT && stages == ST && kcg == KCG) return (void*)&b4::b4_gemv_tma_mma_kernel<NT, ST, KCG>;
    B4_TMA_PICK(1, 4, 4)
    B4_TMA_PICK(1, 3, 4)
    B4_TMA_PICK(1, 6, 4)
    B4_TMA_PICK(1, 4, 2)
    B4_TMA_PICK(1, 4, 8)
    B4_TMA_PICK(1, 8, 2)
    B4_TMA_PICK(2, 4, 4)
#undef B4_TMA_PICK
    return nullptr;
}

int b4::gemv_tma_device_error(int clear)
{
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return -1;
    if (clear && v) {
        const int z = 0;
        cudaMemcpyToSymbol(g_device_error, &z, sizeof(int));
    }
    return v;
}
