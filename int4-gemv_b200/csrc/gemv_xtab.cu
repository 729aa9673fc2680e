// Instantiations of the batch-1 NF4 GEMV from x-pair product tables (warps per
// CTA x batches each warp keeps in flight in registers; one CTA per SM, within
// the registers of one CTA per SM without spills), and the reader of this
// translation unit's device error flag.
#include "b4_gemv_xtab.cuh"

void* b4::gemv_kernel_xtab(int warps, int stages)
{
#define B4_XTAB_PICK(NW, P) \
    if (warps == NW && stages == P) return (void*)&b4::b4_gemv_xtab_kernel<NW, P>;
    B4_XTAB_PICK(8, 4)
    B4_XTAB_PICK(12, 2)
    B4_XTAB_PICK(12, 3)
    B4_XTAB_PICK(16, 2)
    B4_XTAB_PICK(20, 1)
    B4_XTAB_PICK(24, 1)
#undef B4_XTAB_PICK
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
