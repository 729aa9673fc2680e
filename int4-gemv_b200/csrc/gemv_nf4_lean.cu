// Instantiations of the lean batch-1 NF4 GEMV kernel.
#include "b4_gemv_lean_nf4.cuh"

void* b4::gemv_kernel_nf4_lean(int depth, int rw, int vw, int lut)
{
#define B4_NF4_LEAN(D, RW, VW, LUT) \
    if (depth == D && rw == RW && vw == VW && lut == LUT) return (void*)&b4::b4_gemv_lean_nf4_kernel<D, RW, VW, LUT>;
    B4_NF4_LEAN(4, 4, 2, 0)
    B4_NF4_LEAN(4, 8, 2, 0)
    B4_NF4_LEAN(6, 4, 2, 0)
    B4_NF4_LEAN(4, 4, 4, 0)
    B4_NF4_LEAN(4, 4, 2, 2)
    B4_NF4_LEAN(4, 8, 2, 2)
    B4_NF4_LEAN(6, 4, 2, 2)
    B4_NF4_LEAN(8, 4, 2, 2)
    B4_NF4_LEAN(4, 4, 4, 2)
#undef B4_NF4_LEAN
    return nullptr;
}
