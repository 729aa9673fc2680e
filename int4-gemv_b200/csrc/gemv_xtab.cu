// Instantiations of the batch-1 NF4 GEMV from x-pair product tables (register
// load pipeline of depth 2, 3 or 4), and the reader of this translation
// unit's device error flag.
#include "b4_gemv_xtab.cuh"

void* b4::gemv_kernel_xtab(int depth)
{
    switch (depth) {
        case 2: return (void*)&b4::b4_gemv_xtab_kernel<2>;
        case 3: return (void*)&b4::b4_gemv_xtab_kernel<3>;
        case 4: return (void*)&b4::b4_gemv_xtab_kernel<4>;
    }
    return nullptr;
}

int b4::xtab_device_error(int clear)
{
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_xtab_error, sizeof(int)) != cudaSuccess) return -1;
    if (clear && v) {
        const int z = 0;
        cudaMemcpyToSymbol(g_xtab_error, &z, sizeof(int));
    }
    return v;
}
