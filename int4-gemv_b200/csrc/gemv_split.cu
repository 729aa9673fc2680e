// Instantiations of the split batch-1 GEMVs (b4_gemv_split.cuh): INT4 with a
// cp.async ring of depth x groups per stage, NF4 with a register pipeline.
#include "b4_gemv_split.cuh"

void* b4::gemv_kernel_split_int4(int depth, int groups)
{
    switch (groups * 100 + depth) {
        case 104: return (void*)&b4::b4_gemv_split_int4_kernel<4, 1>;
        case 106: return (void*)&b4::b4_gemv_split_int4_kernel<6, 1>;
        case 203: return (void*)&b4::b4_gemv_split_int4_kernel<3, 2>;
        case 204: return (void*)&b4::b4_gemv_split_int4_kernel<4, 2>;
        case 402: return (void*)&b4::b4_gemv_split_int4_kernel<2, 4>;
        case 403: return (void*)&b4::b4_gemv_split_int4_kernel<3, 4>;
    }
    return nullptr;
}

void* b4::gemv_kernel_split_nf4(int depth)
{
    switch (depth) {
        case 2: return (void*)&b4::b4_gemv_split_nf4_kernel<2>;
        case 3: return (void*)&b4::b4_gemv_split_nf4_kernel<3>;
        case 4: return (void*)&b4::b4_gemv_split_nf4_kernel<4>;
    }
    return nullptr;
}
