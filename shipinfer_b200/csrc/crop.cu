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
// Layout: one warp per task (box, strip of 32 x V output columns, chunk of 16 output rows);
// warps never wait on one another, and no shared memory is used. Lane l owns V adjacent output
// columns. The warp walks its rows top to bottom keeping in registers the horizontal lerps of
// the (at most two) source rows the current output row reads: output rows that share a source
// row — every upscaled box's do — reuse its lerps, so each distinct source row is interpolated
// once per chunk. A source row's lerps read each column's two taps as two or three aligned
// 32-bit words through the read-only cache (both taps' six bytes, never a byte outside the
// frame row) and fold each channel into one fused multiply-add; the vertical lerp, the
// channel gather, normalisation and the V-wide stores follow per output row.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <cmath>
#include <cstring>

namespace shipk {

namespace {

constexpr int kWarps = 4;   // warps per CTA
constexpr int kChunk = 16;  // output rows per warp task (at most 32: lane j derives row j's taps)

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
    int strips, chunks;        // column strips (32 * V columns) and row chunks (kChunk rows) per box
    long long tasks;           // n_boxes * strips * chunks
    float mean[3], stdv[3], rcp[3], zero_out[3];  // per output channel
    float rcp_w, rcp_h;        // RN(1 / dst_w), RN(1 / dst_h)
    int arith;                 // normalise by div_markstein (the host checked the constants' range)
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

// numpy's clip-then-cast, with a NaN coordinate clipping to 0 (undefined in the reference).
__host__ __device__ __forceinline__ int clip_trunc(float v, float hi) {
    return (int)fminf(fmaxf(v, 0.f), hi);
}

// V values of one output row of one plane.
template <typename OutT, int V>
__device__ __forceinline__ void store_row(OutT* o, const float (&v)[V]) {
    if constexpr (V == 4) {
        if constexpr (sizeof(OutT) == 4) {
            __stcs(reinterpret_cast<float4*>(o), make_float4(v[0], v[1], v[2], v[3]));
        } else {
            __half2 h0 = __floats2half2_rn(v[0], v[1]), h1 = __floats2half2_rn(v[2], v[3]);
            uint2 u;
            u.x = *reinterpret_cast<uint32_t*>(&h0);
            u.y = *reinterpret_cast<uint32_t*>(&h1);
            __stcs(reinterpret_cast<uint2*>(o), u);
        }
    } else {
        OutVec<OutT>::store1(o, v[0]);
    }
}

// The horizontal lerps of one source row at the lane's V columns, all three channels.
// torch.lerp(a, b, w) is a + w*(b - a) for w < 0.5 and b - (b - a)*(1 - w) otherwise, one
// rounding each (fused); both are fma(W, Q - P, P) with (P, Q, W) = (a, b, w) or (b, a, 1 - w),
// and Q - P is exact for bytes. A column whose two taps are one pixel has W = 0 (P = a): the
// lerp of a pixel with itself is the pixel. Column k's left tap starts at byte a0[k] of the
// row; its right neighbour, three bytes on, is inside the frame row too (the box's right edge
// is clipped to width - 1), so the three aligned words covering both taps hold only bytes of
// that row plus the neighbouring bytes of their own words. 2^23 + b is b's float with the
// integer in the low mantissa bits, made with one byte permute.
template <int V>
__device__ __forceinline__ void source_row_lerps(const uint8_t* row, const int (&a0)[V], const float (&W)[V],
                                                 const bool (&left)[V], float (&h)[3][V]) {
#pragma unroll
    for (int k = 0; k < V; ++k) {
        const uintptr_t a = reinterpret_cast<uintptr_t>(row + a0[k]);
        const uint32_t o = static_cast<uint32_t>(a) & 3u;
        const uint32_t* wp = reinterpret_cast<const uint32_t*>(a - o);
        const uint32_t w0 = __ldg(wp), w1 = __ldg(wp + 1);
        const uint32_t w2 = o == 3u ? __ldg(wp + 2) : 0u;  // the right tap reaches byte 8 only from o = 3
        const uint32_t lt = __funnelshift_r(w0, w1, 8 * o);                        // bytes o .. o+3
        const uint32_t rt = __funnelshift_r(o ? w1 : w0, o ? w2 : w1, 8 * o + 24);  // bytes o+3 .. o+6
        const uint32_t P = left[k] ? lt : rt, Q = left[k] ? rt : lt;
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            const float pf = __uint_as_float(__byte_perm(P, 0x4b000000u, 0x7440u + c));
            const float qf = __uint_as_float(__byte_perm(Q, 0x4b000000u, 0x7440u + c));
            h[c][k] = __fmaf_rn(W[k], __fsub_rn(qf, pf), __fsub_rn(pf, 8388608.0f));
        }
    }
}

// (v - mean) / std for a crop value, correctly rounded. With `arith` (the host checked the
// constants' range) this is div_markstein without its two guards, which no crop value reaches:
//  * every weight is 0 or in [2^-24, 0.5]: w = src - i0 is 0, or RN(t - 0.5) with t >= 0.5 a
//    float (a multiple of 2^-24), or src - i0 with 1 <= i0 <= src (exact, a multiple of
//    2^-23); 1 - w for w >= 0.5 is exact and at least 2^-24;
//  * so a lerp of bytes is +0 or at least 2^-24 (a lerp a + W*(b - a) with a >= 1 stays above
//    a / 2), and the lerp of two such values is +0 or at least 2^-48; never -0, since an exact
//    zero sum rounds to +0;
//  * x = v - mean is then +0 or at least 2^-48 in magnitude: v itself when mean is 0, and for
//    |mean| >= 2^-20 either +0 (v == mean), or at least 2^-21, or a nonzero multiple of the
//    ulp of both v and mean (v within a factor 2 of mean), which is at least 2^-44.
// So no numerator is below 2^-60 (where a quotient could leave the theorem's range) and none is
// -0 (the one zero whose sign the corrections lose; +0 keeps q0's). Without `arith`, IEEE
// division.
template <int V>
__device__ __forceinline__ void crop_normalise(float (&v)[3][V], const float (&mean)[3], const float (&stdv)[3],
                                               const float (&rcp)[3], bool arith) {
    if (arith) {
#pragma unroll
        for (int c = 0; c < 3; ++c)
#pragma unroll
            for (int k = 0; k < V; ++k) {
                const float x = __fsub_rn(v[c][k], mean[c]);
                const float q0 = __fmul_rn(x, rcp[c]);
                const float r0 = __fmaf_rn(-q0, stdv[c], x);
                const float q1 = __fmaf_rn(r0, rcp[c], q0);
                const float r1 = __fmaf_rn(-q1, stdv[c], x);
                v[c][k] = __fmaf_rn(r1, rcp[c], q1);
            }
    } else {
#pragma unroll
        for (int c = 0; c < 3; ++c)
#pragma unroll
            for (int k = 0; k < V; ++k) v[c][k] = normalise(v[c][k], mean[c], stdv[c]);
    }
}

template <typename OutT, int V>
__global__ void __launch_bounds__(kWarps * 32)
crop_kernel(const __grid_constant__ CropParams p) {
    const int lane = threadIdx.x & 31;
    const long long task = (long long)blockIdx.x * kWarps + (threadIdx.x >> 5);
    // Launched as a programmatic dependent of the stream's previous kernel: the boxes, frames
    // and output are touched only once that kernel has completed.
    griddep_wait();
    griddep_launch_dependents();
    if (task >= p.tasks) return;
    const int per_box = p.strips * p.chunks;
    const int box = (int)(task / per_box);
    const int rem = (int)(task - (long long)box * per_box);
    const int strip = rem / p.chunks, chunk = rem - strip * p.chunks;
    const int xb = strip * 32 * V + lane * V;  // the lane's first column; V divides dst_w
    const bool live = xb < p.dst_w;
    const int yb = chunk * kChunk, nrows = min(kChunk, p.dst_h - yb);

    // ---- geometry (every lane: four broadcast loads) ----
    const float* bp = p.boxes + (int64_t)box * 4;
    const float bx1 = __ldg(bp), by1 = __ldg(bp + 1), bx2 = __ldg(bp + 2), by2 = __ldg(bp + 3);
    const int fi = p.box_frame ? __ldg(p.box_frame + box) : 0;
    bool degenerate = fi < 0 || fi >= p.n_frames;
    const CropFrame& F = p.f[degenerate ? 0 : fi];
    const uint8_t* const src = F.src;
    const int32_t* const row_map = F.row_map;
    const int64_t pitch = F.pitch;
    const int fw = F.w, fh = F.h;
    const int x1 = clip_trunc(bx1, (float)(fw - 1));
    const int y1 = clip_trunc(by1, (float)(fh - 1));
    const int ew = clip_trunc(bx2, (float)(fw - 1)) - x1;
    const int eh = clip_trunc(by2, (float)(fh - 1)) - y1;
    degenerate = degenerate || ew <= 0 || eh <= 0;

    const int64_t plane = (int64_t)p.dst_h * p.dst_w;
    OutT* const out = static_cast<OutT*>(p.out) + (int64_t)box * 3 * plane + (int64_t)yb * p.dst_w + xb;

    if (degenerate) {  // a crop of zeros, normalised
        if (!live) return;
        float z[3][V];
#pragma unroll
        for (int c = 0; c < 3; ++c)
#pragma unroll
            for (int k = 0; k < V; ++k) z[c][k] = p.zero_out[c];
        for (int j = 0; j < nrows; ++j)
#pragma unroll
            for (int c = 0; c < 3; ++c) store_row<OutT, V>(out + c * plane + (int64_t)j * p.dst_w, z[c]);
        return;
    }

    // source channel c (the frame's B, G, R bytes) lands in output channel c, or 2 - c with swap_rb
    OutT* dst[3];
    float mean[3], stdv[3], rcp[3];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        const int oc = p.swap_rb ? 2 - c : c;
        dst[c] = out + oc * plane;
        mean[c] = p.mean[oc];
        stdv[c] = p.stdv[oc];
        rcp[c] = p.rcp[oc];
    }

    // the lane's columns (numpy's float32 ew / dst_w, correctly rounded: div_markstein of two
    // positive integers); lanes past the right edge compute the last column and store nothing
    int a0[V];
    float W[V];
    bool left[V];
    const float scale_x = div_markstein((float)ew, (float)p.dst_w, p.rcp_w);
#pragma unroll
    for (int k = 0; k < V; ++k) {
        const CropAxis a = crop_axis(scale_x, ew - 1, min(xb + k, p.dst_w - 1));
        const bool same = a.i1 == a.i0;
        left[k] = same || a.w1 < 0.5f;
        W[k] = same ? 0.f : (left[k] ? a.w1 : __fsub_rn(1.f, a.w1));
        a0[k] = (x1 + a.i0) * 3;
    }
    // lane j: the vertical taps of the chunk's row j; a row whose weight is 0, or whose two taps
    // are one row, reads one source row (s1 == s0)
    int my_s0 = 0, my_s1 = 0;
    float my_w = 0.f;
    if (lane < nrows) {
        const CropAxis a = crop_axis(div_markstein((float)eh, (float)p.dst_h, p.rcp_h), eh - 1, yb + lane);
        my_s0 = a.i0;
        my_s1 = a.w1 != 0.f ? a.i1 : a.i0;
        my_w = a.w1;
    }
    auto row_ptr = [&](int s) {
        const int r = y1 + s;
        return src + (int64_t)(row_map ? __ldg(row_map + r) : r) * pitch;
    };

    float top[3][V], bot[3][V];
    int held0 = -1, held1 = -1;  // the source rows whose lerps top and bot hold
    for (int j = 0; j < nrows; ++j) {
        const int s0 = __shfl_sync(0xffffffffu, my_s0, j);
        const int s1 = __shfl_sync(0xffffffffu, my_s1, j);
        const float wy = __shfl_sync(0xffffffffu, my_w, j);
        if (s0 != held0) {
            if (s0 == held1) {
#pragma unroll
                for (int c = 0; c < 3; ++c)
#pragma unroll
                    for (int k = 0; k < V; ++k) top[c][k] = bot[c][k];
            } else {
                source_row_lerps<V>(row_ptr(s0), a0, W, left, top);
            }
            held0 = s0;
        }
        float v[3][V];
        if (s1 == s0) {
#pragma unroll
            for (int c = 0; c < 3; ++c)
#pragma unroll
                for (int k = 0; k < V; ++k) v[c][k] = top[c][k];
        } else {
            if (s1 != held1) {
                source_row_lerps<V>(row_ptr(s1), a0, W, left, bot);
                held1 = s1;
            }
            // torch.lerp down, the weight the same for the whole warp
            if (wy < 0.5f) {
#pragma unroll
                for (int c = 0; c < 3; ++c)
#pragma unroll
                    for (int k = 0; k < V; ++k) v[c][k] = __fmaf_rn(wy, __fsub_rn(bot[c][k], top[c][k]), top[c][k]);
            } else {
                const float omw = __fsub_rn(1.f, wy);
#pragma unroll
                for (int c = 0; c < 3; ++c)
#pragma unroll
                    for (int k = 0; k < V; ++k)
                        v[c][k] = __fmaf_rn(-__fsub_rn(bot[c][k], top[c][k]), omw, bot[c][k]);
            }
        }
        if (live) {
            crop_normalise<V>(v, mean, stdv, rcp, p.arith);
            const int64_t off = (int64_t)j * p.dst_w;
#pragma unroll
            for (int c = 0; c < 3; ++c) store_row<OutT, V>(dst[c] + off, v[c]);
        }
    }
}

template <typename OutT, int V>
cudaError_t launch_crop_t(const CropParams& p, int grid, cudaStream_t stream) {
    return launch_dependent(crop_kernel<OutT, V>, dim3(grid), dim3(kWarps * 32), 0, stream, p);
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
    p.arith = 1;
    p.rcp_w = 1.0f / (float)dst_w;
    p.rcp_h = 1.0f / (float)dst_h;
    for (int c = 0; c < 3; ++c) {
        p.mean[c] = mean[c];
        p.stdv[c] = stdv[c];
        p.rcp[c] = 1.0f / stdv[c];
        p.zero_out[c] = (0.f - mean[c]) / stdv[c];
        p.arith &= normalise_arith_ok(mean[c], stdv[c]) ? 1 : 0;
    }
    for (int i = 0; i < n_frames; ++i) {
        p.f[i].src = frames[i].data;
        p.f[i].row_map = frames[i].row_map;
        p.f[i].pitch = frames[i].pitch;
        p.f[i].h = frames[i].height;
        p.f[i].w = frames[i].width;
    }
    // four columns per lane (16-byte float / 8-byte fp16 stores) when every row starts aligned
    const size_t elt = out_dtype == SHIPK_DTYPE_F32 ? 4 : 2;
    const bool aligned = (reinterpret_cast<uintptr_t>(out) & (4 * elt - 1)) == 0;
    const int vec = (aligned && dst_w % 4 == 0) ? 4 : 1;
    p.strips = (dst_w + 32 * vec - 1) / (32 * vec);
    p.chunks = (dst_h + kChunk - 1) / kChunk;
    p.tasks = (long long)n_boxes * p.strips * p.chunks;
    const long long grid = (p.tasks + kWarps - 1) / kWarps;
    if (grid > 0x7fffffffLL) return Status{SHIPK_ERANGE, "too many boxes for one launch"};
    cudaError_t e;
    if (out_dtype == SHIPK_DTYPE_F32)
        e = vec == 4 ? launch_crop_t<float, 4>(p, (int)grid, stream) : launch_crop_t<float, 1>(p, (int)grid, stream);
    else
        e = vec == 4 ? launch_crop_t<__half, 4>(p, (int)grid, stream) : launch_crop_t<__half, 1>(p, (int)grid, stream);
    if (e != cudaSuccess) return Status{SHIPK_ECUDA, cudaGetErrorString(e)};
    return Status{SHIPK_OK, nullptr};
}

}  // namespace shipk
