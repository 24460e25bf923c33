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
// Layout: one CTA per (box, tile of output rows). Every thread derives the box geometry (a
// broadcast load of four floats); `rows` threads derive the vertical taps of their output row
// in parallel. The CTA stages the box's span of each source row its rows read (a row whose
// vertical weight is exactly 0 is not read) into shared memory with 16-byte cp.async copies,
// then each thread writes 16-byte vectors of one output row for all three planes. A tile whose
// spans do not fit the shared budget reads the same bytes through the read-only cache.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <cmath>
#include <cstring>

namespace shipk {

namespace {

constexpr int kThreads = 256;
constexpr int kMaxRows = 32;
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
__host__ __device__ __forceinline__ int clip_trunc(float v, float hi) {
    return (int)fminf(fmaxf(v, 0.f), hi);
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem_src) : "memory");
}

// src[0, nbytes) into dst with shared and global agreeing modulo 16; cp.async for the aligned
// middle, byte loads for the ragged ends; every global access stays inside the range.
__device__ __forceinline__ const uint8_t* stage_async(uint8_t* dst, const uint8_t* src, int nbytes,
                                                      int tid, int nthreads) {
    const int mis = static_cast<int>(reinterpret_cast<uintptr_t>(src) & 15);
    uint8_t* base = dst + mis;
    const int head = mis == 0 ? 0 : min(16 - mis, nbytes);
    const int body_vecs = (nbytes - head) >> 4;
    const int tail_start = head + (body_vecs << 4);
    for (int v = tid; v < body_vecs; v += nthreads) cp_async16(base + head + 16 * v, src + head + 16 * v);
    const int edge = head + (nbytes - tail_start);
    for (int e = tid; e < edge; e += nthreads) {
        const int k = e < head ? e : tail_start + (e - head);
        base[k] = __ldg(src + k);
    }
    return base;
}

struct CropRow {
    CropAxis ay;
    int src0, src1;  // source rows (frame coordinates) read by this output row; src1 -1: weight 0
};

template <typename OutT, int VEC>
__device__ __forceinline__ void store3(OutT* o, int64_t plane, const float (&v0)[VEC],
                                       const float (&v1)[VEC], const float (&v2)[VEC]) {
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

template <typename OutT, int VEC>
__global__ void __launch_bounds__(kThreads)
crop_kernel(const __grid_constant__ CropParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ CropRow rows[kMaxRows];
    __shared__ const uint8_t* slot_ptr[2 * kMaxRows];

    const int tid = threadIdx.x;
    const int box = blockIdx.x / p.tiles;
    const int tile = blockIdx.x - box * p.tiles;
    const int y0 = tile * p.rows;
    const int nrows = min(p.rows, p.dst_h - y0);

    // the box's geometry, derived by every thread from one broadcast read
    const float* bp = p.boxes + (int64_t)box * 4;
    const float bx1 = __ldg(bp), by1 = __ldg(bp + 1), bx2 = __ldg(bp + 2), by2 = __ldg(bp + 3);
    const int fi = p.box_frame ? __ldg(p.box_frame + box) : 0;
    bool degenerate = fi < 0 || fi >= p.n_frames;
    const CropFrame& F = p.f[degenerate ? 0 : fi];
    const int x1 = clip_trunc(bx1, (float)(F.w - 1));
    const int y1 = clip_trunc(by1, (float)(F.h - 1));
    const int ew = clip_trunc(bx2, (float)(F.w - 1)) - x1;
    const int eh = clip_trunc(by2, (float)(F.h - 1)) - y1;
    degenerate = degenerate || ew <= 0 || eh <= 0;

    OutT* crop_out = static_cast<OutT*>(p.out) + (int64_t)box * 3 * (int64_t)p.dst_h * p.dst_w;
    const int64_t plane = (int64_t)p.dst_h * p.dst_w;
    const int groups = (p.dst_w + VEC - 1) / VEC;
    const int items = nrows * groups;

    if (degenerate) {
        float v0[VEC], v1[VEC], v2[VEC];
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
            v0[k] = p.zero_out[0];
            v1[k] = p.zero_out[1];
            v2[k] = p.zero_out[2];
        }
        for (int it = tid; it < items; it += kThreads) {
            const int r = it / groups;
            const int x0 = (it - r * groups) * VEC;
            store3<OutT, VEC>(crop_out + (int64_t)(y0 + r) * p.dst_w + x0, plane, v0, v1, v2);
        }
        return;
    }

    const float scale_x = __fdiv_rn((float)ew, (float)p.dst_w);
    if (tid < 2 * kMaxRows) slot_ptr[tid] = smem;  // an unstaged slot is never a stale address
    if (tid < nrows) {
        const float scale_y = __fdiv_rn((float)eh, (float)p.dst_h);
        const CropAxis a = crop_axis(scale_y, eh - 1, y0 + tid);
        CropRow& cr = rows[tid];
        cr.ay = a;
        cr.src0 = y1 + a.i0;
        cr.src1 = a.w1 != 0.f ? y1 + a.i1 : -1;
    }
    __syncthreads();

    const int seg_bytes = ew * 3;
    const int seg_stride = ((seg_bytes + 16 + 15) / 16) * 16;
    const bool staged = 2 * nrows * seg_stride <= kSmemBytes;
    for (int s = 0; s < 2 * nrows; ++s) {
        const int sr = (s & 1) ? rows[s >> 1].src1 : rows[s >> 1].src0;
        if (sr < 0) continue;
        const int row = F.row_map ? __ldg(F.row_map + sr) : sr;
        const uint8_t* g = F.src + (int64_t)row * F.pitch + x1 * 3;
        if (staged) {
            const uint8_t* base = stage_async(smem + s * seg_stride, g, seg_bytes, tid, kThreads);
            if (tid == 0) slot_ptr[s] = base;
        } else if (tid == 0) {
            slot_ptr[s] = g;
        }
    }
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
    __syncthreads();

    const int last_x = ew - 1;
    for (int it = tid; it < items; it += kThreads) {
        const int r = it / groups;
        const int x0 = (it - r * groups) * VEC;
        const CropAxis ay = rows[r].ay;
        const uint8_t* r0 = slot_ptr[2 * r];
        const uint8_t* r1 = rows[r].src1 >= 0 ? slot_ptr[2 * r + 1] : r0;
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
            v0[k] = normalise(p.swap_rb ? px[2] : px[0], p.mean[0], p.stdv[0]);
            v1[k] = normalise(px[1], p.mean[1], p.stdv[1]);
            v2[k] = normalise(p.swap_rb ? px[0] : px[2], p.mean[2], p.stdv[2]);
        }
        store3<OutT, VEC>(crop_out + (int64_t)(y0 + r) * p.dst_w + x0, plane, v0, v1, v2);
    }
}

template <typename OutT, int VEC>
cudaError_t launch_crop_t(const CropParams& p, int grid, cudaStream_t stream) {
    // 48 KB of dynamic shared memory on top of the static row table needs the opt-in.
    cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(crop_kernel<OutT, VEC>), kSmemBytes);
    if (e != cudaSuccess) return e;
    crop_kernel<OutT, VEC><<<grid, kThreads, kSmemBytes, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace

void crop_rows_needed(const float* box, int h, int w, int dst_h, unsigned char* needed) {
    // The kernel's own geometry (clip_trunc, crop_axis) in host float arithmetic.
    const int y1 = clip_trunc(box[1], (float)(h - 1));
    const int y2 = clip_trunc(box[3], (float)(h - 1));
    const int x1 = clip_trunc(box[0], (float)(w - 1));
    const int x2 = clip_trunc(box[2], (float)(w - 1));
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
