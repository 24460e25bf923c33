// Exhaustive check of the kernels' fast normalisation against IEEE-754 division.
//
// normalise_fast() divides by a channel's std with div_markstein (a multiply and four fused
// multiply-adds from RN(1/std)) instead of a division. This kernel evaluates both for every
// single-precision value v in [0, 256) and for -0 — every input the letterbox, crop and NV12
// paths can hand to normalisation, since their blended and converted pixels lie in [0, 255] —
// and counts the inputs whose results differ in any bit. When the std allows the one-correction
// form (markstein_one_step_ok: the crop kernel then uses div_markstein2_1), that form is checked
// on the same inputs too, and an input counts if either form differs.
#include "common.cuh"
#include "kernels.h"

namespace shipk {

namespace {

constexpr uint32_t kEnd = 0x43800000u;  // bit pattern of 256.0f: every float in [0, 256) is below

__global__ void normalise_check_kernel(float mean, float stdv, float rcp, bool one_step,
                                       unsigned long long* result) {
    unsigned long long local = 0;
    uint32_t first = 0xffffffffu;
    const uint32_t stride = gridDim.x * blockDim.x;
    const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
    // thread 0 takes -0 (bit pattern 0x80000000) before its share of [0, 256)
    for (uint32_t u = t == 0 ? 0x80000000u : t; u < kEnd || u == 0x80000000u;
         u = u == 0x80000000u ? 0u : u + stride) {
        const float v = __uint_as_float(u);
        const float ref = normalise(v, mean, stdv);
        const float fast = normalise_fast(v, mean, stdv, rcp, true);
        bool differs = __float_as_uint(ref) != __float_as_uint(fast);
        if (one_step) {  // normalise_fast's decision with div_markstein_1 for div_markstein
            const float x = __fsub_rn(v, mean);
            const float fast1 = tiny_nonzero(x, 8.67361737988403547e-19f) ? __fdiv_rn(x, stdv)
                                                                           : div_markstein_1(x, stdv, rcp);
            differs |= __float_as_uint(ref) != __float_as_uint(fast1);
        }
        if (differs) {
            ++local;
            first = min(first, u);
        }
    }
    if (local) {
        atomicAdd(result, local);
        atomicMin(result + 1, (unsigned long long)first);
    }
}

}  // namespace

Status launch_normalise_check(float mean, float stdv, unsigned long long* result, cudaStream_t stream) {
    if (!normalise_arith_ok(mean, stdv))
        return Status{SHIPK_ERANGE, "mean/std outside the range where the kernels use the fast division"};
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) sms = 148;
    normalise_check_kernel<<<sms * 8, 256, 0, stream>>>(mean, stdv, 1.0f / stdv, markstein_one_step_ok(stdv),
                                                         result);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return Status{SHIPK_ECUDA, cudaGetErrorString(e)};
    return Status{SHIPK_OK, nullptr};
}

}  // namespace shipk
