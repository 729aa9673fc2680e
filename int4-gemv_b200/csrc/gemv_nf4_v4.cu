// Instantiations of the GEMV kernel for format nf4, 4-word lane loads.
#include "b4_gemv_kernel.cuh"

void* b4::gemv_kernel_nf4_v4(int rw, int mb, int lut)
{
    B4_GEMV_PICK(b4::kNf4, 4, 1, 1, 0)
    B4_GEMV_PICK(b4::kNf4, 4, 2, 1, 0)
    B4_GEMV_PICK(b4::kNf4, 4, 4, 1, 0)
    B4_GEMV_PICK(b4::kNf4, 4, 8, 1, 0)
    B4_GEMV_PICK(b4::kNf4, 4, 1, 2, 0)
    B4_GEMV_PICK(b4::kNf4, 4, 2, 2, 0)
    B4_GEMV_PICK(b4::kNf4, 4, 4, 2, 0)
    B4_GEMV_PICK(b4::kNf4, 4, 8, 2, 0)
    B4_GEMV_PICK(b4::kNf4, 4, 1, 4, 0)
    B4_GEMV_PICK(b4::kNf4, 4, 2, 4, 0)
    B4_GEMV_PICK(b4::kNf4, 4, 4, 4, 0)
    B4_GEMV_PICK(b4::kNf4, 4, 1, 1, 1)
    B4_GEMV_PICK(b4::kNf4, 4, 2, 1, 1)
    B4_GEMV_PICK(b4::kNf4, 4, 4, 1, 1)
    B4_GEMV_PICK(b4::kNf4, 4, 8, 1, 1)
    B4_GEMV_PICK(b4::kNf4, 4, 1, 2, 1)
    B4_GEMV_PICK(b4::kNf4, 4, 2, 2, 1)
    B4_GEMV_PICK(b4::kNf4, 4, 4, 2, 1)
    B4_GEMV_PICK(b4::kNf4, 4, 8, 2, 1)
    B4_GEMV_PICK(b4::kNf4, 4, 1, 4, 1)
    B4_GEMV_PICK(b4::kNf4, 4, 2, 4, 1)
    B4_GEMV_PICK(b4::kNf4, 4, 4, 4, 1)
    return nullptr;
}
