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
// Layout: one CTA per (box, tile of output rows); a thread per group of output pixels computes
// its taps directly (the boxes are small and the taps hit L1), and writes 16-byte vectors.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <cstring>

namespace shipk {

namespace {

constexpr int kThreads = 256;

struct Nv12CropFrame {
    const uint8_t* luma;
    int64_t pitch, uv_offset;
    int h, w;
};

struct Nv12CropParams {
    const float* boxes;
    const int32_t* box_frame;
    void* out;
    int n_boxes, n_frames;
    int dst_h, dst_w;
    int rows, tiles;  // output rows per CTA, row tiles per box
    int swap_rb;
    float rcp255;     // RN(1 / 255)
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

template <typename OutT, int VEC>
__global__ void __launch_bounds__(kThreads) crop_nv12_kernel(const __grid_constant__ Nv12CropParams p) {
    const int box = blockIdx.x / p.tiles;
    const int tile = blockIdx.x - box * p.tiles;
    const int groups = (p.dst_w + VEC - 1) / VEC;
    const int y0 = tile * p.rows;
    const int nrows = min(p.rows, p.dst_h - y0);

    const float* bp = p.boxes + (int64_t)box * 4;
    const int fi = p.box_frame ? __ldg(p.box_frame + box) : 0;
    const bool bad_frame = fi < 0 || fi >= p.n_frames;
    const Nv12CropFrame& F = p.f[bad_frame ? 0 : fi];
    const int x1 = clip_trunc_nv12(__ldg(bp), (float)F.w - 1.f);
    const int y1 = clip_trunc_nv12(__ldg(bp + 1), (float)F.h - 1.f);
    const int bw = clip_trunc_nv12(__ldg(bp + 2), (float)F.w - 1.f) - x1;
    const int bh = clip_trunc_nv12(__ldg(bp + 3), (float)F.h - 1.f) - y1;
    const bool degenerate = bad_frame || bw <= 0 || bh <= 0;

    const int64_t plane = (int64_t)p.dst_h * p.dst_w;
    OutT* crop_out = static_cast<OutT*>(p.out) + (int64_t)box * 3 * plane;
    const YuvMatrix m = yuv_matrix(601);
    const uint8_t* uv = F.luma + F.uv_offset;
    const float means[3] = {0.f, 0.f, 0.f}, stdv[3] = {255.f, 255.f, 255.f};
    const float rcp[3] = {p.rcp255, p.rcp255, p.rcp255};

    for (int it = threadIdx.x; it < nrows * groups; it += kThreads) {
        const int r = it / groups;
        const int x0 = (it - r * groups) * VEC;
        const int y = y0 + r;
        float v0[VEC], v1[VEC], v2[VEC];
        bool none[VEC];
        if (degenerate) {
#pragma unroll
            for (int k = 0; k < VEC; ++k) v0[k] = v1[k] = v2[k] = 0.f;
        } else {
            int py0, py1;
            float wy;
            tap_axis(y, bh, p.dst_h, py0, py1, wy);
            const int sy0 = min(F.h - 1, y1 + py0), sy1 = min(F.h - 1, y1 + py1);
            const uint8_t* yr0 = F.luma + (int64_t)sy0 * F.pitch;
            const uint8_t* yr1 = F.luma + (int64_t)sy1 * F.pitch;
            const uint8_t* cr0 = uv + (int64_t)(sy0 >> 1) * F.pitch;
            const uint8_t* cr1 = uv + (int64_t)(sy1 >> 1) * F.pitch;
            const float omy = __fsub_rn(1.f, wy);
#pragma unroll
            for (int k = 0; k < VEC; ++k) {
                const int x = min(x0 + k, p.dst_w - 1);
                int px0, px1;
                float wx;
                tap_axis(x, bw, p.dst_w, px0, px1, wx);
                const int sx0 = min(F.w - 1, x1 + px0), sx1 = min(F.w - 1, x1 + px1);
                float q00[3], q01[3], q10[3], q11[3];
                yuv_to_bgr(m, yr0, cr0, sx0, q00);
                yuv_to_bgr(m, yr0, cr0, sx1, q01);
                yuv_to_bgr(m, yr1, cr1, sx0, q10);
                yuv_to_bgr(m, yr1, cr1, sx1, q11);
                const float omx = __fsub_rn(1.f, wx);
                float val[3];
#pragma unroll
                for (int c = 0; c < 3; ++c) {
                    const float top = __fmaf_rn(q00[c], omx, __fmul_rn(q01[c], wx));
                    const float bot = __fmaf_rn(q10[c], omx, __fmul_rn(q11[c], wx));
                    val[c] = __fmaf_rn(top, omy, __fmul_rn(bot, wy));
                }
                v0[k] = p.swap_rb ? val[2] : val[0];
                v1[k] = val[1];
                v2[k] = p.swap_rb ? val[0] : val[2];
            }
#pragma unroll
            for (int k = 0; k < VEC; ++k) none[k] = false;
            // value / 255, correctly rounded (div_markstein, checked against IEEE division on
            // every float in [0, 256) by shipk_normalise_check)
            normalise_group<VEC>(v0, v1, v2, none, means, stdv, rcp, true);
        }
        OutT* o = crop_out + (int64_t)y * p.dst_w + x0;
        if constexpr (VEC > 1) {
            OutVec<OutT>::store(o, v0);
            OutVec<OutT>::store(o + plane, v1);
            OutVec<OutT>::store(o + 2 * plane, v2);
        } else {
            OutVec<OutT>::store1(o, v0[0]);
            OutVec<OutT>::store1(o + plane, v1[0]);
            OutVec<OutT>::store1(o + 2 * plane, v2[0]);
        }
    }
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
    p.swap_rb = swap_rb;
    p.rcp255 = 1.0f / 255.0f;
    for (int i = 0; i < n_frames; ++i) {
        p.f[i].luma = frames[i].data;
        p.f[i].pitch = frames[i].pitch;
        p.f[i].uv_offset = frames[i].uv_offset;
        p.f[i].h = frames[i].height;
        p.f[i].w = frames[i].width;
    }
    const bool aligned = (reinterpret_cast<uintptr_t>(out) & 15) == 0;
    const int vec = out_dtype == SHIPK_DTYPE_F32 ? ((aligned && dst_w % 4 == 0) ? 4 : 1)
                                                 : ((aligned && dst_w % 8 == 0) ? 8 : 1);
    const int groups = (dst_w + vec - 1) / vec;
    p.rows = std::max(1, std::min(dst_h, kThreads / std::max(1, groups)));
    p.tiles = (dst_h + p.rows - 1) / p.rows;
    const long long grid = (long long)n_boxes * p.tiles;
    if (grid > 0x7fffffffLL) return Status{SHIPK_ERANGE, "too many boxes for one launch"};
    if (out_dtype == SHIPK_DTYPE_F32) {
        if (vec == 4) crop_nv12_kernel<float, 4><<<(int)grid, kThreads, 0, stream>>>(p);
        else crop_nv12_kernel<float, 1><<<(int)grid, kThreads, 0, stream>>>(p);
    } else {
        if (vec == 8) crop_nv12_kernel<__half, 8><<<(int)grid, kThreads, 0, stream>>>(p);
        else crop_nv12_kernel<__half, 1><<<(int)grid, kThreads, 0, stream>>>(p);
    }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return Status{SHIPK_ECUDA, cudaGetErrorString(e)};
    return Status{SHIPK_OK, nullptr};
}

}  // namespace shipk
