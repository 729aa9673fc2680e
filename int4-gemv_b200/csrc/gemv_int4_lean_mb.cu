// Instantiations of the small-batch lean INT4 kernel: (stages, groups per
// stage) x (one or two 8-column blocks of batch rows); `wide`: the 16-warp
// CTA for two blocks (9..16 batch rows); `sliced`: the k-sliced form
// (B4_FLAG_KSLICE).
#include "b4_gemv_lean_mb.cuh"

void* b4::gemv_kernel_int4_lean_mb(int depth, int groups, int nb, int wide, int sliced)
{
    if (wide) {
        if (nb != 2 || groups != 1 || depth != 4) return nullptr;
        return sliced ? (void*)&b4::b4_gemv_lean_mb_kernel<4, 1, 2, 512, 1> : (void*)&b4::b4_gemv_lean_mb_kernel<4, 1, 2, 512>;
    }
    if (sliced) {
        switch (nb * 1000 + groups * 100 + depth) {
            case 1402: return (void*)&b4::b4_gemv_lean_mb_kernel<2, 4, 1, 256, 1>;
            case 1203: return (void*)&b4::b4_gemv_lean_mb_kernel<3, 2, 1, 256, 1>;
            case 1104: return (void*)&b4::b4_gemv_lean_mb_kernel<4, 1, 1, 256, 1>;
            case 2402: return (void*)&b4::b4_gemv_lean_mb_kernel<2, 4, 2, 256, 1>;
            case 2203: return (void*)&b4::b4_gemv_lean_mb_kernel<3, 2, 2, 256, 1>;
            case 2104: return (void*)&b4::b4_gemv_lean_mb_kernel<4, 1, 2, 256, 1>;
        }
        return nullptr;
    }
    switch (nb * 1000 + groups * 100 + depth) {
        case 1402: return (void*)&b4::b4_gemv_lean_mb_kernel<2, 4, 1>;
        case 1203: return (void*)&b4::b4_gemv_lean_mb_kernel<3, 2, 1>;
        case 1104: return (void*)&b4::b4_gemv_lean_mb_kernel<4, 1, 1>;
        case 2402: return (void*)&b4::b4_gemv_lean_mb_kernel<2, 4, 2>;
        case 2203: return (void*)&b4::b4_gemv_lean_mb_kernel<3, 2, 2>;
        case 2104: return (void*)&b4::b4_gemv_lean_mb_kernel<4, 1, 2>;
    }
    return nullptr;
}
