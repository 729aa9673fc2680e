// Instantiations of the small-batch NF4 tensor-pipe GEMV: register pipeline of
// depth 2 or 3 x one, two or four 8-column MMA blocks (4, 8 or 16 batch rows),
// plain or k-sliced (B4_FLAG_KSLICE).
#include "b4_gemv_nf4_mma_mb.cuh"

void* b4::gemv_kernel_nf4_mma_mb(int depth, int nb, int sliced)
{
    if (sliced) {
        switch (nb * 10 + depth) {
            case 12: return (void*)&b4::b4_gemv_nf4_mma_mb_kernel<2, 1, 1>;
            case 13: return (void*)&b4::b4_gemv_nf4_mma_mb_kernel<3, 1, 1>;
            case 22: return (void*)&b4::b4_gemv_nf4_mma_mb_kernel<2, 2, 1>;
            case 23: return (void*)&b4::b4_gemv_nf4_mma_mb_kernel<3, 2, 1>;
            case 42: return (void*)&b4::b4_gemv_nf4_mma_mb_kernel<2, 4, 1>;
            case 43: return (void*)&b4::b4_gemv_nf4_mma_mb_kernel<3, 4, 1>;
        }
        return nullptr;
    }
    switch (nb * 10 + depth) {
        case 12: return (void*)&b4::b4_gemv_nf4_mma_mb_kernel<2, 1>;
        case 13: return (void*)&b4::b4_gemv_nf4_mma_mb_kernel<3, 1>;
        case 22: return (void*)&b4::b4_gemv_nf4_mma_mb_kernel<2, 2>;
        case 23: return (void*)&b4::b4_gemv_nf4_mma_mb_kernel<3, 2>;
        case 42: return (void*)&b4::b4_gemv_nf4_mma_mb_kernel<2, 4>;
        case 43: return (void*)&b4::b4_gemv_nf4_mma_mb_kernel<3, 4>;
    }
    return nullptr;
}
