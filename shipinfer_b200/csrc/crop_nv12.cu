// Batched ROI crop-resize straight from NV12 decoder surfaces: every box of every frame in one
// launch.
//
// Reference semantics: nv12_crop_resize_kernel / nv12_crop_resize_into,
// csrc/shipinfer/runtime/ops.cu:260-318 and :402-416 (one frame per call there), as nvcc
// compiles it with its default contraction:
//   * box corners clipped to [0, W-1] / [0, H-1] in float and truncated; a non-positive extent
//     gives a crop of zeros;
//   * per axis lx = max(0, ((x + 0.5) * box_w) / dst_w - 0.5) with every step rounded,
//     px0 = min((int)lx, box_w - 1), px1 = min(px0 + 1, box_w - 1), wx = lx - px0;
//   * the four taps converted to BGR (BT.601 limited range, as nv12_to_bgr) and blended:
//     value = (p00*(1-wx) + p01*wx)*(1-wy) + (p10*(1-wx) + p11*wx)*wy, each "a*b + c*d" fused
//     as fma(a, b, c*d); channel order flipped by swap_rb; value / 255.
//
// Layout: the crop kernel's (crop.cu). One warp per task (box, strip of 32 x V output columns,
// chunk of 16 output rows), no shared memory, no barriers. The blend is separable in the same
// way: the inner sum h(row, x) = fma(q(row, px0), 1-wx, q(row, px1)*wx) depends only on a source
// row and an output column, so the warp walks its rows holding h of the (at most two) source
// rows the current output row reads, and each distinct source row is converted and blended once
// per chunk; the outer fma per output row follows. Float work runs on packed fp32 pairs (two
// columns per instruction, each lane rounded as the scalar operation is).
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <cstring>

namespace shipk {

namespace {

// warps per CTA: one, so that the task's values are visibly uniform across the CTA (the crop
// kernel's reason). The launch bounds ask for 22 CTAs per SM: the compiler then fits the kernel
// in 80 registers with no spill (25 one-warp CTAs fit an SM either way); asked for 24 it spilled
// 4 bytes, read once per output row. The NV12 workload: 55.7 us, against 56.2 with the spill and
// 57.2 with four-warp CTAs at 122 registers.
constexpr int kWarps = 1;
constexpr int kChunk = 16;  // output rows per warp task (at most 32: lane j derives row j's taps)

struct Nv12CropFrame {
    const uint8_t* luma;
    int64_t pitch, uv_offset;
    int h, w;
    int uv16;  // chroma rows start at even addresses: U and V of a pixel in one 16-bit load
};

struct Nv12CropParams {
    const float* boxes;
    const int32_t* box_frame;
    void* out;
    int n_boxes, n_frames;
    int dst_h, dst_w;
    int strips, chunks;  // column strips (32 * V columns) and row chunks (kChunk rows) per box
    long long tasks;     // n_boxes * strips * chunks
    int plane_of[3];     // output plane of B, G, R: c, or 2 - c with swap_rb
    Norm2 n2;            // value / 255: mean 0, std 255, RN(1/255), in pairs
    Nv12CropFrame f[kMaxBatch];
};

__device__ __forceinline__ int clip_trunc_nv12(float v, float hi) { return (int)fminf(fmaxf(v, 0.f), hi); }

// The reference's tap along one axis (ops.cu:284-297).
__device__ __forceinline__ void tap_axis(int d, int box_len, int dst_len, int& p0, int& p1, float& w) {
    float l = __fsub_rn(__fdiv_rn(__fmul_rn(__fadd_rn((float)d, 0.5f), (float)box_len), (float)dst_len), 0.5f);
    l = fmaxf(0.f, l);
    p0 = min((int)l, box_len - 1);
    p1 = min(p0 + 1, box_len - 1);
    w = __fsub_rn(l, (float)p0);
}

// yuv_to_bgr of two luma columns of one source row, read through the read-only cache.
__device__ __forceinline__ void convert_pair(const Yuv2& k, const uint8_t* yrow, const uint8_t* uvrow, bool uv16,
                                             int xa, int xb, float2 bgr[3]) {
    const int ca = (xa >> 1) << 1, cb = (xb >> 1) << 1;
    float ua, va, ub, vb;
    if (uv16) {
        const uint32_t a = __ldg(reinterpret_cast<const unsigned short*>(uvrow + ca));
        const uint32_t b = __ldg(reinterpret_cast<const unsigned short*>(uvrow + cb));
        ua = __uint_as_float(__byte_perm(a, 0x4b000000u, 0x7440u));
        va = __uint_as_float(__byte_perm(a, 0x4b000000u, 0x7441u));
        ub = __uint_as_float(__byte_perm(b, 0x4b000000u, 0x7440u));
        vb = __uint_as_float(__byte_perm(b, 0x4b000000u, 0x7441u));
    } else {
        ua = u8_biased(__ldg(uvrow + ca));
        va = u8_biased(__ldg(uvrow + ca + 1));
        ub = u8_biased(__ldg(uvrow + cb));
        vb = u8_biased(__ldg(uvrow + cb + 1));
    }
    // u8f(y) - 16 and u8f(u) - 128 are exact: one subtraction each from 2^23 + byte
    const float2 Y = __fmul2_rn(__fadd2_rn(make_float2(u8_biased(__ldg(yrow + xa)), u8_biased(__ldg(yrow + xb))),
                                           splat2(-8388624.0f)), k.ys);
    const float2 U = __fadd2_rn(make_float2(ua, ub), splat2(-8388736.0f));
    const float2 V = __fadd2_rn(make_float2(va, vb), splat2(-8388736.0f));
    const float2 b = __ffma2_rn(k.cbu, U, Y);
    const float2 g = __ffma2_rn(k.ncgv, V, __ffma2_rn(k.ncgu, U, Y));
    const float2 r = __ffma2_rn(k.crv, V, Y);
    bgr[0] = make_float2(clamp255(b.x), clamp255(b.y));
    bgr[1] = make_float2(clamp255(g.x), clamp255(g.y));
    bgr[2] = make_float2(clamp255(r.x), clamp255(r.y));
}

// h(row, x) at the lane's V columns: fma(q(px0), 1 - wx, q(px1) * wx) per channel.
template <int V>
__device__ __forceinline__ void source_row_blends(const Yuv2& k, const uint8_t* yrow, const uint8_t* uvrow, bool uv16,
                                                  const int (&sx0)[V], const int (&sx1)[V], const float2 (&omx)[V / 2],
                                                  const float2 (&wx)[V / 2], float2 (&h)[3][V / 2]) {
#pragma unroll
    for (int i = 0; i < V / 2; ++i) {
        float2 q0[3], q1[3];
        convert_pair(k, yrow, uvrow, uv16, sx0[2 * i], sx0[2 * i + 1], q0);
        convert_pair(k, yrow, uvrow, uv16, sx1[2 * i], sx1[2 * i + 1], q1);
#pragma unroll
        for (int c = 0; c < 3; ++c) h[c][i] = __ffma2_rn(q0[c], omx[i], __fmul2_rn(q1[c], wx[i]));
    }
}

// V values (V/2 pairs) of one output row of one plane: one vector store (VS), or one store per
// column left of dst_w.
template <typename OutT, int V, bool VS>
__device__ __forceinline__ void store_cols(OutT* o, const float2 (&v)[V / 2], int x, int dst_w) {
    if constexpr (VS) {
        if constexpr (sizeof(OutT) == 4) {
            if constexpr (V == 4) __stcs(reinterpret_cast<float4*>(o), make_float4(v[0].x, v[0].y, v[1].x, v[1].y));
            else __stcs(reinterpret_cast<float2*>(o), v[0]);
        } else {
            uint32_t u[V / 2];
#pragma unroll
            for (int i = 0; i < V / 2; ++i) {
                __half2 hv = __float22half2_rn(v[i]);
                u[i] = *reinterpret_cast<uint32_t*>(&hv);
            }
            if constexpr (V == 4) __stcs(reinterpret_cast<uint2*>(o), make_uint2(u[0], u[1]));
            else __stcs(reinterpret_cast<unsigned int*>(o), u[0]);
        }
    } else {
#pragma unroll
        for (int i = 0; i < V / 2; ++i) {
            if (x + 2 * i < dst_w) OutVec<OutT>::store1(o + 2 * i, v[i].x);
            if (x + 2 * i + 1 < dst_w) OutVec<OutT>::store1(o + 2 * i + 1, v[i].y);
        }
    }
}

template <typename OutT, int V, bool VS>
__global__ void __launch_bounds__(kWarps * 32, 22)
crop_nv12_kernel(const __grid_constant__ Nv12CropParams p) {
    static_assert(V % 2 == 0, "columns are handled in pairs");
    const int lane = threadIdx.x & 31;
    const long long task = (long long)blockIdx.x * kWarps + (threadIdx.x >> 5);
    if (task >= p.tasks) return;
    const int per_box = p.strips * p.chunks;
    const int box = (int)(task / per_box);
    const int rem = (int)(task - (long long)box * per_box);
    const int strip = rem / p.chunks, chunk = rem - strip * p.chunks;
    const int xb = strip * 32 * V + lane * V;  // the lane's first column
    const bool live = xb < p.dst_w;
    const int yb = chunk * kChunk, nrows = min(kChunk, p.dst_h - yb);

    // ---- geometry (every lane: four broadcast loads) ----
    const float* bp = p.boxes + (int64_t)box * 4;
    const int fi = p.box_frame ? __ldg(p.box_frame + box) : 0;
    const bool bad_frame = fi < 0 || fi >= p.n_frames;
    const Nv12CropFrame& F = p.f[bad_frame ? 0 : fi];
    const uint8_t* const luma = F.luma;
    const uint8_t* const uv = F.luma + F.uv_offset;
    const int64_t pitch = F.pitch;
    const int fw = F.w, fh = F.h;
    const bool uv16 = F.uv16 != 0;
    const int x1 = clip_trunc_nv12(__ldg(bp), (float)fw - 1.f);
    const int y1 = clip_trunc_nv12(__ldg(bp + 1), (float)fh - 1.f);
    const int bw = clip_trunc_nv12(__ldg(bp + 2), (float)fw - 1.f) - x1;
    const int bh = clip_trunc_nv12(__ldg(bp + 3), (float)fh - 1.f) - y1;
    const bool degenerate = bad_frame || bw <= 0 || bh <= 0;

    const int64_t plane = (int64_t)p.dst_h * p.dst_w;
    OutT* const out = static_cast<OutT*>(p.out) + (int64_t)box * 3 * plane + (int64_t)yb * p.dst_w + xb;

    if (degenerate) {  // a crop of zeros (0 / 255)
        if (!live) return;
        float2 z[V / 2];
#pragma unroll
        for (int i = 0; i < V / 2; ++i) z[i] = make_float2(0.f, 0.f);
        for (int j = 0; j < nrows; ++j)
#pragma unroll
            for (int c = 0; c < 3; ++c) store_cols<OutT, V, VS>(out + c * plane + (int64_t)j * p.dst_w, z, xb, p.dst_w);
        return;
    }

    OutT* dst[3];
#pragma unroll
    for (int c = 0; c < 3; ++c) dst[c] = out + p.plane_of[c] * plane;

    // the lane's columns; columns past the right edge repeat the last one and store nothing
    int sx0[V], sx1[V];
    float2 wx[V / 2], omx[V / 2];
    float wmin = 1.f;  // the smallest nonzero column weight of the lane
#pragma unroll
    for (int k = 0; k < V; ++k) {
        int p0, p1;
        float w;
        tap_axis(min(xb + k, p.dst_w - 1), bw, p.dst_w, p0, p1, w);
        sx0[k] = min(fw - 1, x1 + p0);
        sx1[k] = min(fw - 1, x1 + p1);
        const float om = __fsub_rn(1.f, w);
        if (k & 1) {
            wx[k / 2].y = w;
            omx[k / 2].y = om;
        } else {
            wx[k / 2].x = w;
            omx[k / 2].x = om;
        }
        if (w != 0.f) wmin = fminf(wmin, fminf(w, om));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) wmin = fminf(wmin, __shfl_xor_sync(0xffffffffu, wmin, o));
    // lane j: the vertical taps of the chunk's row j; a row whose weight is 0 reads one source
    // row (s1 = s0): its value is fma(top, 1, bot * 0) = top
    int my_s0 = 0, my_s1 = 0;
    float my_w = 0.f;
    if (lane < nrows) {
        int p0, p1;
        tap_axis(yb + lane, bh, p.dst_h, p0, p1, my_w);
        my_s0 = min(fh - 1, y1 + p0);
        my_s1 = my_w != 0.f ? min(fh - 1, y1 + p1) : my_s0;
    }
    // Lane j asks for the strip's luma and chroma bytes of row j's source rows now (into L1):
    // luma columns [lo, hi], chroma bytes [lo, hi + 1] (U and V of the even column at or below
    // each one), every address inside its row.
    {
        const int lo = (__shfl_sync(0xffffffffu, sx0[0], 0) >> 1) << 1;
        const int hi = __shfl_sync(0xffffffffu, sx1[V - 1], 31);
        if (lane < nrows && hi - lo < 16 * 128) {
            const uint8_t* rows[4] = {luma + (int64_t)my_s0 * pitch + lo, luma + (int64_t)my_s1 * pitch + lo,
                                      uv + (int64_t)(my_s0 >> 1) * pitch + lo, uv + (int64_t)(my_s1 >> 1) * pitch + lo};
            const int last[2] = {hi - lo, ((hi >> 1) << 1) + 1 - lo};
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                if ((r & 1) && my_s1 == my_s0) continue;
                const int n = last[r >> 1];
                const int skip = (int)(reinterpret_cast<uintptr_t>(rows[r]) & 127);
                for (int b = 0; b <= n; b = (b == 0 ? 128 - skip : b + 128))
                    asm volatile("prefetch.global.L1 [%0];" ::"l"(rows[r] + b));
            }
        }
    }

    const Yuv2 k2 = yuv2(yuv_matrix(601));
    float2 top[3][V / 2], bot[3][V / 2];
    int held0 = -1, held1 = -1;  // the source rows whose blends top and bot hold
    for (int j = 0; j < nrows; ++j) {
        const int s0 = __shfl_sync(0xffffffffu, my_s0, j);
        const int s1 = __shfl_sync(0xffffffffu, my_s1, j);
        const float wy = __shfl_sync(0xffffffffu, my_w, j);
        if (s0 != held0) {
            if (s0 == held1) {
#pragma unroll
                for (int c = 0; c < 3; ++c)
#pragma unroll
                    for (int i = 0; i < V / 2; ++i) top[c][i] = bot[c][i];
            } else {
                source_row_blends<V>(k2, luma + (int64_t)s0 * pitch, uv + (int64_t)(s0 >> 1) * pitch, uv16, sx0, sx1,
                                     omx, wx, top);
            }
            held0 = s0;
        }
        float2 v[3][V / 2];
        if (wy == 0.f) {
#pragma unroll
            for (int c = 0; c < 3; ++c)
#pragma unroll
                for (int i = 0; i < V / 2; ++i) v[c][i] = top[c][i];
        } else {
            if (s1 != held1) {
                if (s1 == s0) {  // both taps in one row (the box's last): bot is top
#pragma unroll
                    for (int c = 0; c < 3; ++c)
#pragma unroll
                        for (int i = 0; i < V / 2; ++i) bot[c][i] = top[c][i];
                } else {
                    source_row_blends<V>(k2, luma + (int64_t)s1 * pitch, uv + (int64_t)(s1 >> 1) * pitch, uv16, sx0,
                                         sx1, omx, wx, bot);
                }
                held1 = s1;
            }
            const float2 wy2 = splat2(wy), omy2 = splat2(__fsub_rn(1.f, wy));
#pragma unroll
            for (int c = 0; c < 3; ++c)
#pragma unroll
                for (int i = 0; i < V / 2; ++i) v[c][i] = __ffma2_rn(top[c][i], omy2, __fmul2_rn(bot[c][i], wy2));
        }
        if (live) {
            // value / 255. Converted taps are 0 or at least 2^-25 (multiples of it) and the
            // weights 0 or at least the row's and the warp's smallest nonzero ones, so a blend is
            // 0 or at least 2^-25 * wx * wy less three roundings; only below 2^-58 may a
            // numerator fall under normalise_group's 2^-60 bound.
            const float wyr = wy != 0.f ? fminf(wy, __fsub_rn(1.f, wy)) : 1.f;
            const bool guard = !(2.98023223876953125e-08f * wmin * wyr >= 3.469446951953614e-18f);
            float c0[V], c1[V], c2[V];
            bool none[V];
#pragma unroll
            for (int i = 0; i < V / 2; ++i) {
                c0[2 * i] = v[0][i].x;
                c0[2 * i + 1] = v[0][i].y;
                c1[2 * i] = v[1][i].x;
                c1[2 * i + 1] = v[1][i].y;
                c2[2 * i] = v[2][i].x;
                c2[2 * i + 1] = v[2][i].y;
                none[2 * i] = none[2 * i + 1] = false;
            }
            const float stdv[3] = {255.f, 255.f, 255.f};
            normalise_group2<V>(c0, c1, c2, none, p.n2, stdv, true, guard);
#pragma unroll
            for (int i = 0; i < V / 2; ++i) {
                v[0][i] = make_float2(c0[2 * i], c0[2 * i + 1]);
                v[1][i] = make_float2(c1[2 * i], c1[2 * i + 1]);
                v[2][i] = make_float2(c2[2 * i], c2[2 * i + 1]);
            }
            const int64_t off = (int64_t)j * p.dst_w;
#pragma unroll
            for (int c = 0; c < 3; ++c) store_cols<OutT, V, VS>(dst[c] + off, v[c], xb, p.dst_w);
        }
    }
}

template <typename OutT, int V, bool VS>
cudaError_t launch_t(const Nv12CropParams& p, int grid, cudaStream_t stream) {
    crop_nv12_kernel<OutT, V, VS><<<grid, kWarps * 32, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace

Status launch_crop_nv12(const FrameView* frames, int n_frames, const float* boxes, const int32_t* box_frame,
                        int n_boxes, void* out, int out_dtype, int dst_h, int dst_w, int swap_rb,
                        cudaStream_t stream) {
    if (n_boxes == 0) return Status{SHIPK_OK, nullptr};
    if (n_frames > kMaxBatch) return Status{SHIPK_ERANGE, "more than 64 frames in one crop call"};
    Nv12CropParams p;
    std::memset(&p, 0, sizeof(p));
    p.boxes = boxes;
    p.box_frame = box_frame;
    p.out = out;
    p.n_boxes = n_boxes;
    p.n_frames = n_frames;
    p.dst_h = dst_h;
    p.dst_w = dst_w;
    // the reference's value / 255 is normalise() with mean 0 and std 255 (0 - 0 is exact)
    const float mean[3] = {0.f, 0.f, 0.f}, stdv[3] = {255.f, 255.f, 255.f};
    const float r = 1.0f / 255.0f;
    const float rcp[3] = {r, r, r};
    p.n2 = make_norm2(mean, stdv, rcp);
    for (int c = 0; c < 3; ++c) p.plane_of[c] = swap_rb ? 2 - c : c;
    for (int i = 0; i < n_frames; ++i) {
        p.f[i].luma = frames[i].data;
        p.f[i].pitch = frames[i].pitch;
        p.f[i].uv_offset = frames[i].uv_offset;
        p.f[i].h = frames[i].height;
        p.f[i].w = frames[i].width;
        p.f[i].uv16 = ((reinterpret_cast<uintptr_t>(frames[i].data) + (uint64_t)frames[i].uv_offset) % 2 == 0 &&
                       frames[i].pitch % 2 == 0) ? 1 : 0;
    }
    // Four columns per lane with one vector store per plane row when every row starts aligned
    // for it; else two columns per lane, stored as a pair or one at a time.
    const size_t elt = out_dtype == SHIPK_DTYPE_F32 ? 4 : 2;
    const uintptr_t o = reinterpret_cast<uintptr_t>(out);
    const int mode = (dst_w % 4 == 0 && o % (4 * elt) == 0) ? 4 : (dst_w % 2 == 0 && o % (2 * elt) == 0) ? 2 : 1;
    const int V = mode == 4 ? 4 : 2;
    p.strips = (dst_w + 32 * V - 1) / (32 * V);
    p.chunks = (dst_h + kChunk - 1) / kChunk;
    p.tasks = (long long)n_boxes * p.strips * p.chunks;
    const long long grid = (p.tasks + kWarps - 1) / kWarps;
    if (grid > 0x7fffffffLL) return Status{SHIPK_ERANGE, "too many boxes for one launch"};
    cudaError_t e;
    if (out_dtype == SHIPK_DTYPE_F32)
        e = mode == 4 ? launch_t<float, 4, true>(p, (int)grid, stream)
          : mode == 2 ? launch_t<float, 2, true>(p, (int)grid, stream)
                      : launch_t<float, 2, false>(p, (int)grid, stream);
    else
        e = mode == 4 ? launch_t<__half, 4, true>(p, (int)grid, stream)
          : mode == 2 ? launch_t<__half, 2, true>(p, (int)grid, stream)
                      : launch_t<__half, 2, false>(p, (int)grid, stream);
    if (e != cudaSuccess) return Status{SHIPK_ECUDA, cudaGetErrorString(e)};
    return Status{SHIPK_OK, nullptr};
}

}  // namespace shipk
