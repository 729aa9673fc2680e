// Instantiations of the lean batch-1 INT4 tensor-pipe GEMV kernel.
#include "b4_gemv_lean.cuh"

void* b4::gemv_kernel_int4_lean(int depth)
{
    switch (depth) {
        case 2: return (void*)&b4::b4_gemv_lean_kernel<2>;
        case 3: return (void*)&b4::b4_gemv_lean_kernel<3>;
        case 4: return (void*)&b4::b4_gemv_lean_kernel<4>;
        case 6: return (void*)&b4::b4_gemv_lean_kernel<6>;
    }
    return nullptr;
}
