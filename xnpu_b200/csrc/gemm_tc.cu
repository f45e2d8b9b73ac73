// gemm_tc.cu -- K2: batched-decode / prefill dequant-GEMM (m >= 16).
#include <cuda_runtime.h>
#include "xq4_internal.h"
#include "xq4_device.cuh"

cudaError_t xq4_launch_gemm(const uint8_t *pack, int n, int k, const void *x, int m, void *y, int out_f32,
                            cudaStream_t st)
{
    return xq4_launch_gemv(pack, n, k, x, m, y, out_f32, st);
}

unsigned int xq4_take_fault_gemm()
{
    unsigned int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_xq4_fault, sizeof v) != cudaSuccess) return ~0u;
    cudaMemcpyToSymbol(g_xq4_fault, &zero, sizeof zero);
    return v;
}
