// unit_kernels.cu -- TEST INFRASTRUCTURE ONLY: exposes single device helpers
// of the product kernel (fmha_native_b200/csrc/sm100_ptx.cuh) through a C ABI
// so tests can check them against CUDA's own functions on a GPU.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../fmha_native_b200/csrc/sm100_ptx.cuh"

using namespace fmha_sm100;

namespace {

// y_poly[i] = exp2_poly2 of x[i] (pairs), y_mufu = ex2.approx.ftz, y_ref =
// CUDA's exp2f.
__global__ void exp2_kernel(const float* x, float* y_poly, float* y_mufu, float* y_ref, int n) {
    const int i = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
    if (i + 1 >= n) return;
    const float2 p = exp2_poly2(make_float2(x[i], x[i + 1]));
    y_poly[i] = p.x;
    y_poly[i + 1] = p.y;
    y_mufu[i] = ex2_approx(x[i]);
    y_mufu[i + 1] = ex2_approx(x[i + 1]);
    y_ref[i] = exp2f(x[i]);
    y_ref[i + 1] = exp2f(x[i + 1]);
}

// out[i] = pack_bf16_trunc / pack_bf16_rne of the pair (x[2i], x[2i+1]).
__global__ void pack_kernel(const float* x, uint32_t* trunc, uint32_t* rne, int npairs) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= npairs) return;
    trunc[i] = pack_bf16_trunc(x[2 * i], x[2 * i + 1]);
    rne[i] = pack_bf16_rne(x[2 * i], x[2 * i + 1]);
}

}  // namespace

extern "C" {

int unit_exp2(const float* x, float* y_poly, float* y_mufu, float* y_ref, int n) {
    if (n <= 0 || (n & 1)) return 1;
    exp2_kernel<<<(n / 2 + 255) / 256, 256>>>(x, y_poly, y_mufu, y_ref, n);
    return (int)cudaGetLastError();
}

int unit_pack_bf16(const float* x, uint32_t* trunc, uint32_t* rne, int npairs) {
    if (npairs <= 0) return 1;
    pack_kernel<<<(npairs + 255) / 256, 256>>>(x, trunc, rne, npairs);
    return (int)cudaGetLastError();
}

}  // extern "C"
