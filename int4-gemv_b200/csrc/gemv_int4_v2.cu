// Instantiations of the GEMV kernel for format int4, 2-word lane loads.
#include "b4_gemv_kernel.cuh"

void* b4::gemv_kernel_int4_v2(int rw, int mb, int lut)
{
    B4_GEMV_PICK(b4::kInt4, 2, 1, 1, 0)
    B4_GEMV_PICK(b4::kInt4, 2, 2, 1, 0)
    B4_GEMV_PICK(b4::kInt4, 2, 4, 1, 0)
    B4_GEMV_PICK(b4::kInt4, 2, 8, 1, 0)
    B4_GEMV_PICK(b4::kInt4, 2, 1, 2, 0)
    B4_GEMV_PICK(b4::kInt4, 2, 2, 2, 0)
    B4_GEMV_PICK(b4::kInt4, 2, 4, 2, 0)
    B4_GEMV_PICK(b4::kInt4, 2, 8, 2, 0)
    B4_GEMV_PICK(b4::kInt4, 2, 1, 4, 0)
    B4_GEMV_PICK(b4::kInt4, 2, 2, 4, 0)
    B4_GEMV_PICK(b4::kInt4, 2, 4, 4, 0)
    return nullptr;
}
