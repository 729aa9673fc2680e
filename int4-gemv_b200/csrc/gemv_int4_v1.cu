// Instantiations of the GEMV kernel for format int4, 1-word lane loads.
#include "b4_gemv_kernel.cuh"

void* b4::gemv_kernel_int4_v1(int rw, int mb, int lut)
{
    B4_GEMV_PICK(b4::kInt4, 1, 1, 1, 0)
    B4_GEMV_PICK(b4::kInt4, 1, 4, 1, 0)
    return nullptr;
}
