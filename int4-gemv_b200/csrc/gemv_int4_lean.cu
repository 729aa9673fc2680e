// Instantiations of the lean batch-1 INT4 tensor-pipe GEMV kernel: per-lane
// cp.async ring of depth x groups per stage as listed.
#include "b4_gemv_lean.cuh"

void* b4::gemv_kernel_int4_lean(int depth, int groups)
{
    switch (groups * 100 + depth) {
        case 104: return (void*)&b4::b4_gemv_lean_kernel<4, 1>;
        case 106: return (void*)&b4::b4_gemv_lean_kernel<6, 1>;
        case 108: return (void*)&b4::b4_gemv_lean_kernel<8, 1>;
        case 203: return (void*)&b4::b4_gemv_lean_kernel<3, 2>;
        case 204: return (void*)&b4::b4_gemv_lean_kernel<4, 2>;
        case 206: return (void*)&b4::b4_gemv_lean_kernel<6, 2>;
        case 402: return (void*)&b4::b4_gemv_lean_kernel<2, 4>;
        case 403: return (void*)&b4::b4_gemv_lean_kernel<3, 4>;
    }
    return nullptr;
}

// Row-parallel tensor-parallel shards with the peer-memory all-reduce in the
// epilogue (the batch-1 dispatch's variants).
void* b4::gemv_kernel_int4_lean_p2p(int depth, int groups)
{
    switch (groups * 100 + depth) {
        case 104: return (void*)&b4::b4_gemv_lean_kernel<4, 1, 1>;
        case 203: return (void*)&b4::b4_gemv_lean_kernel<3, 2, 1>;
        case 402: return (void*)&b4::b4_gemv_lean_kernel<2, 4, 1>;
    }
    return nullptr;
}
