// Batched ROI crop-resize: every box of every frame in one launch.
//
// Reference formulation: TorchImageOps.crop_batch and _bilinear_axis,
// src/shipinfer/runtime/ops/torch_ops.py:405-507 and :574-614:
//   * clip x to [0, W-1] and y to [0, H-1] in float32, truncate to int (numpy's cast);
//   * the patch is [x1, x2) x [y1, y2); a non-positive extent is a degenerate box whose crop
//     is 0 before normalisation;
//   * per axis, in float32 with every step rounded (numpy does not fuse):
//       scale = f32(max(ext,1)) / f32(dst); src = max(scale * (d + 0.5) - 0.5, 0);
//       i0 = min(int(src), ext-1); w1 = src - i0; i1 = min(i0 + 1, ext-1);
//   * two torch.lerp across (top row, bottom row), one torch.lerp down;
//   * channel gather [2,1,0] when swap_rb, then (v - mean) / std per output channel.
//
// Layout: one CTA per (box, tile of output rows). Thread 0 derives the box geometry and the
// distinct source rows the tile reads (rows whose vertical weight is exactly 0 are not
// read); the CTA stages the box's span of each of those rows into shared memory with
// 16-byte loads, then each thread writes 16-byte vectors of one output row for all three
// planes. A tile whose rows do not fit the shared budget reads the same bytes through the
// read-only cache instead.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <cmath>
#include <cstring>

namespace shipk {

namespace {

constexpr int kThreads = 256;
constexpr int kMaxRows = 32;
constexpr int kMaxSlots = 2 * kMaxRows;
constexpr int kSmemBytes = 48 * 1024;

struct CropFrame {
    const uint8_t* src;
    const int32_t* row_map;  // staged row of each source row, or null (identity)
    int64_t pitch;
    int h, w;
};

struct CropParams {
    const float* boxes;
    const int32_t* box_frame;
    void* out;
    int n_boxes, n_frames;
    int dst_h, dst_w;
    int rows, tiles;
    float mean[3], stdv[3], zero_out[3];
    int swap_rb;
    CropFrame f[kMaxBatch];
};

struct CropAxis {
    int i0, i1;
    float w1;
};

// _bilinear_axis for one destination index, torch_ops.py:602-614.
__device__ __forceinline__ CropAxis crop_axis(float scale, int last, int d) {
    CropAxis a;
    float src = __fsub_rn(__fmul_rn(scale, __fadd_rn((float)d, 0.5f)), 0.5f);
    src = src < 0.f ? 0.f : src;
    a.i0 = min((int)src, last);
    a.w1 = __fsub_rn(src, (float)a.i0);
    a.i1 = min(a.i0 + 1, last);
    return a;
}

// at::lerp: |w| < 0.5 ? a + w*(b-a) : b - (b-a)*(1-w), one rounding per branch (fused).
__device__ __forceinline__ float lerp_t(float a, float b, float w) {
    const float d = __fsub_rn(b, a);
    return fabsf(w) < 0.5f ? __fmaf_rn(w, d, a) : __fmaf_rn(-d, __fsub_rn(1.f, w), b);
}

// numpy's clip-then-cast, with a NaN coordinate clipping to 0 (undefined in the reference).
__device__ __forceinline__ int clip_trunc(float v, float hi) {
    return (int)fminf(fmaxf(v, 0.f), hi);
}

struct CropTile {
    int degenerate;
    int x1, ew;
    float scale_x;
    int last_x;
    int nslots;
    int slot_row[kMaxSlots];
    int s0[kMaxRows], s1[kMaxRows];
    CropAxis ay[kMaxRows];
    int staged;
    int frame;
};

template <typename OutT, int VEC>
__global__ void __launch_bounds__(kThreads)
crop_kernel(const __grid_constant__ CropParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ CropTile t;
    __shared__ const uint8_t* slot_ptr[kMaxSlots];

    const int box = blockIdx.x / p.tiles;
    const int tile = blockIdx.x - box * p.tiles;
    const int y0 = tile * p.rows;
    const int nrows = min(p.rows, p.dst_h - y0);

    if (threadIdx.x == 0) {
        const float* bp = p.boxes + (int64_t)box * 4;
        const float4 b = make_float4(__ldg(bp), __ldg(bp + 1), __ldg(bp + 2), __ldg(bp + 3));
        const int fi = p.box_frame ? p.box_frame[box] : 0;
        t.frame = fi;
        t.nslots = 0;
        t.staged = 0;
        if (fi < 0 || fi >= p.n_frames) {
            t.degenerate = 1;
        } else {
            const CropFrame& F = p.f[fi];
            const int x1 = clip_trunc(b.x, (float)(F.w - 1));
            const int y1 = clip_trunc(b.y, (float)(F.h - 1));
            const int x2 = clip_trunc(b.z, (float)(F.w - 1));
            const int y2 = clip_trunc(b.w, (float)(F.h - 1));
            const int ew = x2 - x1, eh = y2 - y1;
            t.degenerate = ew <= 0 || eh <= 0;
            if (!t.degenerate) {
                t.x1 = x1;
                t.ew = ew;
                t.scale_x = __fdiv_rn((float)ew, (float)p.dst_w);
                t.last_x = ew - 1;
                const float scale_y = __fdiv_rn((float)eh, (float)p.dst_h);
                for (int r = 0; r < nrows; ++r) {
                    const CropAxis a = crop_axis(scale_y, eh - 1, y0 + r);
                    t.ay[r] = a;
                    int rows[2] = {y1 + a.i0, y1 + a.i1};
                    int* slots[2] = {&t.s0[r], &t.s1[r]};
                    t.s1[r] = -1;
                    for (int k = 0; k < (a.w1 != 0.f ? 2 : 1); ++k) {
                        int s = 0;
                        while (s < t.nslots && t.slot_row[s] != rows[k]) ++s;
                        if (s == t.nslots) t.slot_row[t.nslots++] = rows[k];
                        *slots[k] = s;
                    }
                }
                const int seg = ((ew * 3 + 16 + 15) / 16) * 16;
                t.staged = t.nslots * seg <= kSmemBytes;
            }
        }
    }
    __syncthreads();

    OutT* out = static_cast<OutT*>(p.out);
    const int64_t plane = (int64_t)p.dst_h * p.dst_w;
    OutT* crop_out = out + (int64_t)box * 3 * plane;
    const int groups = (p.dst_w + VEC - 1) / VEC;
    const int items = nrows * groups;

    if (t.degenerate) {
        for (int it = threadIdx.x; it < items; it += kThreads) {
            const int r = it / groups;
            const int x0 = (it - r * groups) * VEC;
            float v0[VEC], v1[VEC], v2[VEC];
#pragma unroll
            for (int k = 0; k < VEC; ++k) {
                v0[k] = p.zero_out[0];
                v1[k] = p.zero_out[1];
                v2[k] = p.zero_out[2];
            }
            OutT* o = crop_out + (int64_t)(y0 + r) * p.dst_w + x0;
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
        return;
    }

    const CropFrame& F = p.f[t.frame];
    const int seg_bytes = t.ew * 3;
    const int seg_stride = ((seg_bytes + 16 + 15) / 16) * 16;
    for (int s = 0; s < t.nslots; ++s) {
        const int row = F.row_map ? F.row_map[t.slot_row[s]] : t.slot_row[s];
        const uint8_t* g = F.src + (int64_t)row * F.pitch + t.x1 * 3;
        if (t.staged) {
            const uint8_t* base = stage_bytes(smem + s * seg_stride, g, seg_bytes, threadIdx.x, kThreads);
            if (threadIdx.x == 0) slot_ptr[s] = base;
        } else if (threadIdx.x == 0) {
            slot_ptr[s] = g;
        }
    }
    __syncthreads();

    const int c_src0 = p.swap_rb ? 2 : 0, c_src2 = p.swap_rb ? 0 : 2;
    const float scale_x = t.scale_x;
    const int last_x = t.last_x;
    for (int it = threadIdx.x; it < items; it += kThreads) {
        const int r = it / groups;
        const int x0 = (it - r * groups) * VEC;
        const CropAxis ay = t.ay[r];
        const uint8_t* r0 = slot_ptr[t.s0[r]];
        const uint8_t* r1 = t.s1[r] >= 0 ? slot_ptr[t.s1[r]] : r0;
        float v0[VEC], v1[VEC], v2[VEC];
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
            const int x = min(x0 + k, p.dst_w - 1);
            const CropAxis ax = crop_axis(scale_x, last_x, x);
            const int a0 = ax.i0 * 3;
            const int a1 = ax.w1 != 0.f ? ax.i1 * 3 : a0;  // weight 0: lerp returns a exactly
            float px[3];
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                const float top = lerp_t((float)r0[a0 + c], (float)r0[a1 + c], ax.w1);
                const float bot = lerp_t((float)r1[a0 + c], (float)r1[a1 + c], ax.w1);
                px[c] = lerp_t(top, bot, ay.w1);
            }
            v0[k] = normalise(px[c_src0], p.mean[0], p.stdv[0]);
            v1[k] = normalise(px[1], p.mean[1], p.stdv[1]);
            v2[k] = normalise(px[c_src2], p.mean[2], p.stdv[2]);
        }
        OutT* o = crop_out + (int64_t)(y0 + r) * p.dst_w + x0;
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

template <typename OutT, int VEC>
cudaError_t launch_crop_t(const CropParams& p, int grid, cudaStream_t stream) {
    // 48 KB of dynamic shared memory on top of the static tile table needs the opt-in.
    cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(crop_kernel<OutT, VEC>), kSmemBytes);
    if (e != cudaSuccess) return e;
    crop_kernel<OutT, VEC><<<grid, kThreads, kSmemBytes, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace

void crop_rows_needed(const float* box, int h, int w, int dst_h, unsigned char* needed) {
    // The kernel's own geometry (clip_trunc, crop_axis) in host float arithmetic.
    auto clip = [](float v, float hi) { return (int)std::fmin(std::fmax(v, 0.f), hi); };
    const int y1 = clip(box[1], (float)(h - 1));
    const int y2 = clip(box[3], (float)(h - 1));
    const int x1 = clip(box[0], (float)(w - 1));
    const int x2 = clip(box[2], (float)(w - 1));
    const int eh = y2 - y1;
    if (x2 - x1 <= 0 || eh <= 0) return;
    const float scale = (float)eh / (float)dst_h;
    for (int d = 0; d < dst_h; ++d) {
        volatile float prod = scale * ((float)d + 0.5f);
        float src = prod - 0.5f;
        src = src < 0.f ? 0.f : src;
        const int i0 = std::min((int)src, eh - 1);
        const float w1 = src - (float)i0;
        needed[y1 + i0] = 1;
        if (w1 != 0.f) needed[y1 + std::min(i0 + 1, eh - 1)] = 1;
    }
}

Status launch_crop(const FrameView* frames, int n_frames, const float* boxes,
                   const int32_t* box_frame, int n_boxes, void* out, int out_dtype, int dst_h,
                   int dst_w, const float mean[3], const float stdv[3], int swap_rb,
                   cudaStream_t stream) {
    if (n_boxes == 0) return Status{SHIPK_OK, nullptr};
    if (n_frames > kMaxBatch) return Status{SHIPK_ERANGE, "more than 64 frames in one crop call"};
    CropParams p;
    std::memset(&p, 0, sizeof(p));
    p.boxes = boxes;
    p.box_frame = box_frame;
    p.out = out;
    p.n_boxes = n_boxes;
    p.n_frames = n_frames;
    p.dst_h = dst_h;
    p.dst_w = dst_w;
    p.swap_rb = swap_rb;
    for (int c = 0; c < 3; ++c) {
        p.mean[c] = mean[c];
        p.stdv[c] = stdv[c];
        p.zero_out[c] = (0.f - mean[c]) / stdv[c];
    }
    for (int i = 0; i < n_frames; ++i) {
        p.f[i].src = frames[i].data;
        p.f[i].row_map = frames[i].row_map;
        p.f[i].pitch = frames[i].pitch;
        p.f[i].h = frames[i].height;
        p.f[i].w = frames[i].width;
    }
    const bool aligned = (reinterpret_cast<uintptr_t>(out) & 15) == 0;
    const int vec = out_dtype == SHIPK_DTYPE_F32 ? ((aligned && dst_w % 4 == 0) ? 4 : 1)
                                                 : ((aligned && dst_w % 8 == 0) ? 8 : 1);
    const int groups = (dst_w + vec - 1) / vec;
    p.rows = std::max(1, std::min(kMaxRows, kThreads / groups));
    p.rows = std::min(p.rows, dst_h);
    p.tiles = (dst_h + p.rows - 1) / p.rows;
    const long long grid = (long long)n_boxes * p.tiles;
    if (grid > 0x7fffffffLL) return Status{SHIPK_ERANGE, "too many boxes for one launch"};
    cudaError_t e;
    if (out_dtype == SHIPK_DTYPE_F32)
        e = vec == 4 ? launch_crop_t<float, 4>(p, (int)grid, stream)
                     : launch_crop_t<float, 1>(p, (int)grid, stream);
    else
        e = vec == 8 ? launch_crop_t<__half, 8>(p, (int)grid, stream)
                     : launch_crop_t<__half, 1>(p, (int)grid, stream);
    if (e != cudaSuccess) return Status{SHIPK_ECUDA, cudaGetErrorString(e)};
    return Status{SHIPK_OK, nullptr};
}

}  // namespace shipk
