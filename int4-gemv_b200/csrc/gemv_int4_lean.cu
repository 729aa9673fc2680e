// Instantiations of the lean batch-1 INT4 tensor-pipe GEMV kernel: register
// load pipeline (depth 2..6) or per-lane cp.async ring (depth 4..12).
#include "b4_gemv_lean.cuh"

void* b4::gemv_kernel_int4_lean(int depth, int async_ring)
{
    if (!async_ring) {
        switch (depth) {
            case 2: return (void*)&b4::b4_gemv_lean_kernel<2, 0>;
            case 3: return (void*)&b4::b4_gemv_lean_kernel<3, 0>;
            case 4: return (void*)&b4::b4_gemv_lean_kernel<4, 0>;
            case 6: return (void*)&b4::b4_gemv_lean_kernel<6, 0>;
        }
    } else {
        switch (depth) {
            case 4: return (void*)&b4::b4_gemv_lean_kernel<4, 1>;
            case 6: return (void*)&b4::b4_gemv_lean_kernel<6, 1>;
            case 8: return (void*)&b4::b4_gemv_lean_kernel<8, 1>;
            case 12: return (void*)&b4::b4_gemv_lean_kernel<12, 1>;
        }
    }
    return nullptr;
}
