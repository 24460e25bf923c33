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

// Correctly rounded x / d by one multiply and four fused multiply-adds, given y = RN(1/d).
// Markstein's theorem (P. Markstein, "Computation of elementary functions on the IBM RISC
// System/6000 processor", IBM J. Res. Dev. 34(1), 1990; restated in Muller et al., Handbook of
// Floating-Point Arithmetic, ch. 4): if y is within half an ulp of 1/d and q is a faithful
// rounding of x/d, then r = x - d*q is exact in one FMA and RN(q + r*y) is RN(x/d), barring
// underflow and overflow. q0 = RN(x*y) can be 1.5 ulp off, so one correction comes first:
// q0 + r0*y = x/d + (x/d - q0)*(y*d - 1) is within 2^-23 ulp of x/d before its one rounding,
// which makes q1 faithful; the second correction is the theorem's step. A zero numerator
// returns q0, which is the quotient's correctly signed zero (the corrections would turn -0 into
// +0). Callers establish the no-underflow range on the host (normalise_arith_ok) and the tests
// compare this against __fdiv_rn for every single-precision value in [0, 256) and for -0.
__device__ __forceinline__ float div_markstein(float x, float d, float y) {
    const float q0 = __fmul_rn(x, y);
    const float r0 = __fmaf_rn(-q0, d, x);
    const float q1 = __fmaf_rn(r0, y, q0);
    const float r1 = __fmaf_rn(-q1, d, x);
    const float q2 = __fmaf_rn(r1, y, q1);
    return x == 0.f ? q0 : q2;
}

// normalise() of a group of N pixels (three channels) in place, through div_markstein when
// `arith` (the host checked the constants' range). A group with a nonzero numerator below
// 2^-60 in magnitude (values no pixel blend produces), where a quotient could be subnormal and
// outside the theorem, takes the division instead. One decision per group, not per value,
// keeps the common path a single block the compiler can interleave. `skip[k]` marks pixels
// whose values the caller replaces (pad columns): they do not steer the decision.
__device__ __forceinline__ bool tiny_nonzero(float x, float tiny) { return x != 0.f && fabsf(x) < tiny; }

template <int N>
__device__ __forceinline__ void normalise_group(float (&c0)[N], float (&c1)[N], float (&c2)[N], const bool (&skip)[N],
                                                const float mean[3], const float stdv[3], const float rcp[3],
                                                bool arith) {
    constexpr float kTiny = 8.67361737988403547e-19f;  // 2^-60
    bool slow = !arith;
#pragma unroll
    for (int k = 0; k < N; ++k) {
        c0[k] = __fsub_rn(c0[k], mean[0]);
        c1[k] = __fsub_rn(c1[k], mean[1]);
        c2[k] = __fsub_rn(c2[k], mean[2]);
        slow |= !skip[k] && (tiny_nonzero(c0[k], kTiny) || tiny_nonzero(c1[k], kTiny) || tiny_nonzero(c2[k], kTiny));
    }
    if (!slow) {
#pragma unroll
        for (int k = 0; k < N; ++k) {
            c0[k] = div_markstein(c0[k], stdv[0], rcp[0]);
            c1[k] = div_markstein(c1[k], stdv[1], rcp[1]);
            c2[k] = div_markstein(c2[k], stdv[2], rcp[2]);
        }
    } else {
#pragma unroll
        for (int k = 0; k < N; ++k) {
            c0[k] = __fdiv_rn(c0[k], stdv[0]);
            c1[k] = __fdiv_rn(c1[k], stdv[1]);
            c2[k] = __fdiv_rn(c2[k], stdv[2]);
        }
    }
}

// One value, for the exhaustive check: the decision normalise_group makes for a lone pixel.
__device__ __forceinline__ float normalise_fast(float v, float mean, float stdv, float rcp, bool arith) {
    const float x = __fsub_rn(v, mean);
    if (!arith || tiny_nonzero(x, 8.67361737988403547e-19f)) return __fdiv_rn(x, stdv);
    return div_markstein(x, stdv, rcp);
}

// Host: may div_markstein stand in for division by `stdv` of (v - mean), v in [0, 255]? With
// |x| >= 2^-60 (normalise_fast) it keeps every quotient and remainder normal and every value
// finite: |std| and |mean| within [2^-20, 2^20] (mean may also be 0), 1/std a normal number.
inline bool normalise_arith_ok(float mean, float stdv) {
    const float lo = 9.5367431640625e-07f, hi = 1048576.0f;  // 2^-20, 2^20
    const float as = stdv < 0 ? -stdv : stdv, am = mean < 0 ? -mean : mean;
    if (!(as >= lo && as <= hi)) return false;  // also rejects NaN
    if (!(mean == 0.f || (am >= lo && am <= hi))) return false;
    const float y = 1.0f / stdv;
    const float ay = y < 0 ? -y : y;
    return ay >= 1.17549435e-38f && ay <= 3.4e38f;
}

// ---- programmatic dependent launch (sm_90+) ------------------------------------------------
// A kernel launched with cudaLaunchAttributeProgrammaticStreamSerialization may start before the
// stream's previous kernel has finished. griddep_wait() returns once the grids it depends on have
// completed and their memory is visible: nothing before it may touch global memory those grids
// could write or read. griddep_launch_dependents() lets the stream's next such kernel launch.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

// Launch `kernel` on `stream` as a programmatic dependent of the stream's previous kernel.
template <typename Kernel, typename Params>
inline cudaError_t launch_dependent(Kernel kernel, dim3 grid, dim3 block, int smem, cudaStream_t stream,
                                   const Params& params) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, params);
}

// A uint8 as float without the conversion pipe: 2^23 + b has the exact integer b in its low
// mantissa bits, and subtracting 2^23 leaves exactly b.
__device__ __forceinline__ float u8f(uint32_t b) {
    return __fsub_rn(__uint_as_float(0x4b000000u | b), 8388608.0f);
}

// ---- NV12 conversion ---------------------------------------------------------------------
// Conversion constants: limited-range YCbCr -> R'G'B', six decimals, as the reference's
// nv12_to_bgr (csrc/shipinfer/runtime/ops.cu:159-166) writes BT.601; BT.709 is the same
// construction from Kr = 0.2126, Kb = 0.0722.
struct YuvMatrix {
    float ys, cbu, cgu, cgv, crv;
};

__device__ __forceinline__ YuvMatrix yuv_matrix(int matrix) {
    YuvMatrix m;
    m.ys = 1.164383f;
    if (matrix == 709) {
        m.cbu = 2.112402f; m.cgu = 0.213249f; m.cgv = 0.532909f; m.crv = 1.792741f;
    } else {
        m.cbu = 2.017232f; m.cgu = 0.391762f; m.cgv = 0.812968f; m.crv = 1.596027f;
    }
    return m;
}

// fminf(255, fmaxf(0, v)) for a finite v that is not -0, as one integer instruction on its bit
// pattern: non-negative floats order as their patterns do as integers, a negative float's
// pattern is a negative integer (min.relu clamps it to 0, the pattern of +0), and 0x437f0000
// is 255.0f. The colour conversions below meet no -0 and no NaN: Y' = (Y - 16) * ys is +0 or
// nonzero, and a fused sum whose exact value is 0 rounds to +0 unless both its addends are -0.
__device__ __forceinline__ float clamp255(float v) {
    int r;
    asm("min.relu.s32 %0, %1, %2;" : "=r"(r) : "r"(__float_as_int(v)), "r"(0x437f0000));
    return __int_as_float(r);
}

// One pixel to BGR: Y' = (Y - 16) * ys; B = Y' + cbu*U; G = Y' - cgu*U - cgv*V;
// R = Y' + crv*V, each sum fused as nvcc contracts the reference's expressions, clamped.
__device__ __forceinline__ void yuv_to_bgr(const YuvMatrix& m, const uint8_t* yrow,
                                           const uint8_t* uvrow, int xi, float bgr[3]) {
    const float Y = __fmul_rn(__fsub_rn(u8f(yrow[xi]), 16.f), m.ys);
    const int cx = (xi >> 1) << 1;
    const float U = __fsub_rn(u8f(uvrow[cx]), 128.f);
    const float V = __fsub_rn(u8f(uvrow[cx + 1]), 128.f);
    const float b = __fmaf_rn(m.cbu, U, Y);
    const float g = __fmaf_rn(-m.cgv, V, __fmaf_rn(-m.cgu, U, Y));
    const float r = __fmaf_rn(m.crv, V, Y);
    bgr[0] = clamp255(b);
    bgr[1] = clamp255(g);
    bgr[2] = clamp255(r);
}

// ---- packed fp32 pairs (sm_100) ------------------------------------------------------------
// __ffma2_rn / __fadd2_rn / __fmul2_rn compute two lanes per instruction, each rounded exactly as
// __fmaf_rn / __fadd_rn / __fmul_rn round it, so a pair of pixels costs one instruction where
// the scalar form costs two and the bits are the same. Subtraction is addition of the negation
// (exact); negated constants are prepared by the host.
__device__ __forceinline__ float2 splat2(float a) { return make_float2(a, a); }

// 2^23 + b as a float: b's value in the low mantissa bits (one logic operation).
__device__ __forceinline__ float u8_biased(uint32_t b) { return __uint_as_float(0x4b000000u | b); }

// u8f of two bytes.
__device__ __forceinline__ float2 u8f2(uint32_t a, uint32_t b) {
    return __fadd2_rn(make_float2(u8_biased(a), u8_biased(b)), splat2(-8388608.0f));
}

// interp_blend of two pixels: row weights shared, column weights per pixel.
__device__ __forceinline__ float2 interp_blend2(float2 ly0, float2 ly1, float2 lx0, float2 lx1, float2 p00,
                                                float2 p01, float2 p10, float2 p11) {
    const float2 top = __ffma2_rn(lx0, p00, __fmul2_rn(lx1, p01));
    const float2 bottom = __ffma2_rn(lx0, p10, __fmul2_rn(lx1, p11));
    return __ffma2_rn(ly0, top, __fmul2_rn(ly1, bottom));
}

// div_markstein of two numerators by one divisor d, given nd = -d and y = RN(1/d); fma(-q, d, x)
// is written fma(q, -d, x), the same exact product. Without div_markstein's zero select: for
// x = +0 every correction adds +0 and the result is q0, so this equals div_markstein for every
// numerator but -0, which no pixel value minus a mean produces (blends of non-negative values
// and clamped conversions are never -0, and an exact zero difference rounds to +0).
__device__ __forceinline__ float2 div_markstein2(float2 x, float2 nd, float2 y) {
    const float2 q0 = __fmul2_rn(x, y);
    const float2 r0 = __ffma2_rn(q0, nd, x);
    const float2 q1 = __ffma2_rn(r0, y, q0);
    const float2 r1 = __ffma2_rn(q1, nd, x);
    return __ffma2_rn(r1, y, q1);
}

// Markstein's step applied to q0 directly, for a divisor whose y = RN(1/d) is closer to 1/d
// than RN guarantees: |y*d - 1| <= 2^-25 (markstein_one_step_ok). Then x*y differs from x/d by
// at most |x/d| * 2^-25, which is below half an ulp of x/d, and q0 = RN(x*y) adds at most half
// an ulp more (at a binade edge RN lands on the power of two between them), so q0 is within
// one ulp of x/d: a faithful rounding, which is all the theorem asks of q. One multiply and two
// fused multiply-adds. Same range conditions as div_markstein; +0 stays +0 as there.
__device__ __forceinline__ float div_markstein_1(float x, float d, float y) {
    const float q0 = __fmul_rn(x, y);
    const float r0 = __fmaf_rn(-q0, d, x);
    const float q1 = __fmaf_rn(r0, y, q0);
    return x == 0.f ? q0 : q1;
}

__device__ __forceinline__ float2 div_markstein2_1(float2 x, float2 nd, float2 y) {
    const float2 q0 = __fmul2_rn(x, y);
    const float2 r0 = __ffma2_rn(q0, nd, x);
    return __ffma2_rn(r0, y, q0);
}

// Host: does d allow div_markstein_1, |RN(1/d)*d - 1| <= 2^-25? The product of two floats is
// exact in double, so is its difference from 1, and the test is exact.
inline bool markstein_one_step_ok(float d) {
    const float y = 1.0f / d;
    const double e = (double)y * (double)d - 1.0;
    return (e < 0 ? -e : e) <= 2.98023223876953125e-08;  // 2^-25
}

// Per-channel constants of the packed normalisation, each twice.
struct Norm2 {
    float2 nmean[3], nstd[3], rcp[3];  // -mean, -std, RN(1/std)
};

inline Norm2 make_norm2(const float mean[3], const float stdv[3], const float rcp[3]) {
    Norm2 n;
    for (int c = 0; c < 3; ++c) {
        n.nmean[c] = make_float2(-mean[c], -mean[c]);
        n.nstd[c] = make_float2(-stdv[c], -stdv[c]);
        n.rcp[c] = make_float2(rcp[c], rcp[c]);
    }
    return n;
}

// normalise_group with N even, two pixels per packed instruction: the same decisions (one per
// group) and the same bits for every value that is not -0. `guard` false: the caller has shown
// that no numerator is a nonzero below 2^-60, so the group-level test is skipped.
template <int N>
__device__ __forceinline__ void normalise_group2(float (&c0)[N], float (&c1)[N], float (&c2)[N], const bool (&skip)[N],
                                                 const Norm2& n, const float stdv[3], bool arith, bool guard) {
    static_assert(N % 2 == 0, "pairs");
    constexpr float kTiny = 8.67361737988403547e-19f;  // 2^-60, as normalise_group
    bool slow = !arith;
    float2 x[3][N / 2];
#pragma unroll
    for (int i = 0; i < N / 2; ++i) {
        x[0][i] = __fadd2_rn(make_float2(c0[2 * i], c0[2 * i + 1]), n.nmean[0]);
        x[1][i] = __fadd2_rn(make_float2(c1[2 * i], c1[2 * i + 1]), n.nmean[1]);
        x[2][i] = __fadd2_rn(make_float2(c2[2 * i], c2[2 * i + 1]), n.nmean[2]);
        if (guard) {
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                slow |= !skip[2 * i] && tiny_nonzero(x[c][i].x, kTiny);
                slow |= !skip[2 * i + 1] && tiny_nonzero(x[c][i].y, kTiny);
            }
        }
    }
    if (!slow) {
#pragma unroll
        for (int c = 0; c < 3; ++c)
#pragma unroll
            for (int i = 0; i < N / 2; ++i) x[c][i] = div_markstein2(x[c][i], n.nstd[c], n.rcp[c]);
    } else {
#pragma unroll
        for (int c = 0; c < 3; ++c)
#pragma unroll
            for (int i = 0; i < N / 2; ++i) {
                x[c][i].x = __fdiv_rn(x[c][i].x, stdv[c]);
                x[c][i].y = __fdiv_rn(x[c][i].y, stdv[c]);
            }
    }
#pragma unroll
    for (int i = 0; i < N / 2; ++i) {
        c0[2 * i] = x[0][i].x;
        c0[2 * i + 1] = x[0][i].y;
        c1[2 * i] = x[1][i].x;
        c1[2 * i + 1] = x[1][i].y;
        c2[2 * i] = x[2][i].x;
        c2[2 * i + 1] = x[2][i].y;
    }
}

// Conversion constants of yuv_to_bgr, each twice, the subtracted ones negated.
struct Yuv2 {
    float2 ys, cbu, ncgu, ncgv, crv;
};

__device__ __forceinline__ Yuv2 yuv2(const YuvMatrix& m) {
    Yuv2 k;
    k.ys = splat2(m.ys);
    k.cbu = splat2(m.cbu);
    k.ncgu = splat2(-m.cgu);
    k.ncgv = splat2(-m.cgv);
    k.crv = splat2(m.crv);
    return k;
}

// yuv_to_bgr of two pixels: the same operations (u8f(y) - 16 and u8f(u) - 128 are exact, done
// here as one subtraction from 2^23 + b), two per packed instruction; the clamps are clamp255.
__device__ __forceinline__ void yuv_to_bgr2(const Yuv2& k, const uint8_t* yrow, const uint8_t* uvrow, int xa,
                                            int xb, float2 bgr[3]) {
    const int ca = (xa >> 1) << 1, cb = (xb >> 1) << 1;
    const float2 Y = __fmul2_rn(__fadd2_rn(make_float2(u8_biased(yrow[xa]), u8_biased(yrow[xb])),
                                           splat2(-8388624.0f)), k.ys);  // 2^23 + 16
    const float2 U = __fadd2_rn(make_float2(u8_biased(uvrow[ca]), u8_biased(uvrow[cb])), splat2(-8388736.0f));
    const float2 V = __fadd2_rn(make_float2(u8_biased(uvrow[ca + 1]), u8_biased(uvrow[cb + 1])),
                                splat2(-8388736.0f));  // 2^23 + 128
    const float2 b = __ffma2_rn(k.cbu, U, Y);
    const float2 g = __ffma2_rn(k.ncgv, V, __ffma2_rn(k.ncgu, U, Y));
    const float2 r = __ffma2_rn(k.crv, V, Y);
    bgr[0] = make_float2(clamp255(b.x), clamp255(b.y));
    bgr[1] = make_float2(clamp255(g.x), clamp255(g.y));
    bgr[2] = make_float2(clamp255(r.x), clamp255(r.y));
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
    // eight values held with their halves exchanged (v[0..3] are elements 4..7 when `swapped`)
    __device__ __forceinline__ static void store_swapped(__half* p, const float (&v)[8], bool swapped) {
        __half2 h0 = __floats2half2_rn(v[0], v[1]);
        __half2 h1 = __floats2half2_rn(v[2], v[3]);
        __half2 h2 = __floats2half2_rn(v[4], v[5]);
        __half2 h3 = __floats2half2_rn(v[6], v[7]);
        const uint32_t w0 = *reinterpret_cast<uint32_t*>(&h0), w1 = *reinterpret_cast<uint32_t*>(&h1);
        const uint32_t w2 = *reinterpret_cast<uint32_t*>(&h2), w3 = *reinterpret_cast<uint32_t*>(&h3);
        uint4 u;
        u.x = swapped ? w2 : w0;
        u.y = swapped ? w3 : w1;
        u.z = swapped ? w0 : w2;
        u.w = swapped ? w1 : w3;
        __stcs(reinterpret_cast<uint4*>(p), u);
    }
    // four values as one 8-byte store
    __device__ __forceinline__ static void store(__half* p, const float (&v)[4]) {
        __half2 h0 = __floats2half2_rn(v[0], v[1]);
        __half2 h1 = __floats2half2_rn(v[2], v[3]);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&h0);
        u.y = *reinterpret_cast<uint32_t*>(&h1);
        __stcs(reinterpret_cast<uint2*>(p), u);
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
