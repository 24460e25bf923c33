// Shared device helpers for the shipk kernels (sm_100a).
//
// Arithmetic here is written with explicit round-to-nearest intrinsics (__fmaf_rn,
// __fmul_rn, __fadd_rn, __fsub_rn, __fdiv_rn) wherever the reference result depends on
// whether a multiply and an add are fused: the intrinsics are never contracted or
// re-associated by the compiler, so the kernels compute exactly the formulation they name.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace shipk {

// ---- bilinear taps, torch's F.interpolate(align_corners=False) CUDA formulation ---------
// src = ratio * (d + 0.5) - 0.5 as one fused multiply-add, clamped at 0;
// i0 = (int)src, i1 = i0 + (i0 < in - 1); l1 = src - i0, l0 = 1 - l1.
// Reference call site: TorchImageOps._letterbox, src/shipinfer/runtime/ops/torch_ops.py:389.
struct Tap {
    int i0, i1;
    float l0, l1;
};

__host__ __device__ __forceinline__ Tap interp_tap(float ratio, int d, int in_size) {
    Tap t;
#ifdef __CUDA_ARCH__
    float s = __fmaf_rn(ratio, __fadd_rn((float)d, 0.5f), -0.5f);
#else
    float s = fmaf(ratio, (float)d + 0.5f, -0.5f);
#endif
    s = s < 0.f ? 0.f : s;
    t.i0 = (int)s;
    if (t.i0 > in_size - 1) t.i0 = in_size - 1;
    t.i1 = t.i0 + (t.i0 < in_size - 1 ? 1 : 0);
#ifdef __CUDA_ARCH__
    t.l1 = __fsub_rn(s, (float)t.i0);
    t.l0 = __fsub_rn(1.f, t.l1);
#else
    t.l1 = s - (float)t.i0;
    t.l0 = 1.f - t.l1;
#endif
    return t;
}

// h0 * (w0*p00 + w1*p01) + h1 * (w0*p10 + w1*p11), each "a*b + c*d" as fma(a, b, c*d).
__device__ __forceinline__ float interp_blend(const Tap& ty, const Tap& tx, float p00,
                                              float p01, float p10, float p11) {
    float top = __fmaf_rn(tx.l0, p00, __fmul_rn(tx.l1, p01));
    float bottom = __fmaf_rn(tx.l0, p10, __fmul_rn(tx.l1, p11));
    return __fmaf_rn(ty.l0, top, __fmul_rn(ty.l1, bottom));
}

// (v - mean) / std, each step rounded: canvas.sub_(mean).div_(std), torch_ops.py:401-402.
__device__ __forceinline__ float normalise(float v, float mean, float stdv) {
    return __fdiv_rn(__fsub_rn(v, mean), stdv);
}

// ---- output element stores -------------------------------------------------------------
template <typename T>
struct OutVec;

template <>
struct OutVec<float> {
    static constexpr int kVec = 4;  // 16 bytes
    __device__ __forceinline__ static void store(float* p, const float (&v)[4]) {
        __stcs(reinterpret_cast<float4*>(p), make_float4(v[0], v[1], v[2], v[3]));
    }
    __device__ __forceinline__ static void store1(float* p, float v) { __stcs(p, v); }
};

template <>
struct OutVec<__half> {
    static constexpr int kVec = 8;  // 16 bytes
    __device__ __forceinline__ static void store(__half* p, const float (&v)[8]) {
        __half2 h0 = __floats2half2_rn(v[0], v[1]);
        __half2 h1 = __floats2half2_rn(v[2], v[3]);
        __half2 h2 = __floats2half2_rn(v[4], v[5]);
        __half2 h3 = __floats2half2_rn(v[6], v[7]);
        uint4 u;
        u.x = *reinterpret_cast<uint32_t*>(&h0);
        u.y = *reinterpret_cast<uint32_t*>(&h1);
        u.z = *reinterpret_cast<uint32_t*>(&h2);
        u.w = *reinterpret_cast<uint32_t*>(&h3);
        __stcs(reinterpret_cast<uint4*>(p), u);
    }
    __device__ __forceinline__ static void store1(__half* p, float v) {
        __half h = __float2half_rn(v);
        *p = h;
    }
};

// ---- staging a byte range of global memory into shared memory --------------------------
// Copies src[0, nbytes) so that byte k lands at dst[(src & 15) + k]: shared and global then
// agree modulo 16, so the aligned middle moves as 16-byte vectors (ld.global.nc.v4) while
// the unaligned head and tail move byte by byte. Every global access stays inside
// [src, src + nbytes). `dst` must be 16-byte aligned with nbytes + 16 bytes of room.
// Returns the shared pointer to byte 0 of the copied range.
__device__ __forceinline__ const uint8_t* stage_bytes(uint8_t* dst, const uint8_t* src,
                                                      int nbytes, int tid, int nthreads) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(src);
    const int mis = static_cast<int>(a & 15);
    uint8_t* base = dst + mis;  // base[k] mirrors src[k]
    const int head = mis == 0 ? 0 : min(16 - mis, nbytes);
    const int body_vecs = (nbytes - head) >> 4;
    const int tail_start = head + (body_vecs << 4);
    // aligned middle: 16-byte vectors, global and shared both 16-byte aligned
    const uint4* gsrc = reinterpret_cast<const uint4*>(src + head);
    uint4* sdst = reinterpret_cast<uint4*>(base + head);
    for (int v = tid; v < body_vecs; v += nthreads) sdst[v] = __ldg(gsrc + v);
    // head and tail bytes
    const int edge = head + (nbytes - tail_start);
    for (int e = tid; e < edge; e += nthreads) {
        const int k = e < head ? e : tail_start + (e - head);
        base[k] = __ldg(src + k);
    }
    return base;
}

}  // namespace shipk
