// Instantiations of the GEMV kernel for format nf4, 1-word lane loads.
#include "b4_gemv_kernel.cuh"

void* b4::gemv_kernel_nf4_v1(int rw, int mb, int lut)
{
    B4_GEMV_PICK(b4::kNf4, 1, 1, 1, 0)
    B4_GEMV_PICK(b4::kNf4, 1, 4, 1, 0)
    B4_GEMV_PICK(b4::kNf4, 1, 1, 1, 1)
    B4_GEMV_PICK(b4::kNf4, 1, 4, 1, 1)
    return nullptr;
}
