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

// warps per CTA: one, so that every value derived from the task (geometry, the row loop's held
// source rows) is visibly the same for all the CTA's threads; the compiler then branches on it
// without reconvergence bookkeeping and keeps it off the per-thread registers (config 3:
// 42.9 -> 40.4 us against four-warp CTAs, no spills at 80 registers instead of 20 bytes)
constexpr int kWarps = 1;
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
    float zero_out[3];         // a degenerate box's normalised zero, per output channel
    int plane_of[3];           // output plane of source channel c: c, or 2 - c with swap_rb
    float2 nmean2[3], nstd2[3], rcp2[3];  // -mean, -std, RN(1/std) of source channel c's plane, twice
    float rcp_w, rcp_h;        // RN(1 / dst_w), RN(1 / dst_h)
    int arith;                 // normalise by div_markstein (the host checked the constants' range)
    int one_step;              // ... by div_markstein_1 (markstein_one_step_ok for every channel's std)
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

__device__ __forceinline__ float2 neg2(float2 a) { return make_float2(-a.x, -a.y); }

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
                __half2 h = __float22half2_rn(v[i]);
                u[i] = *reinterpret_cast<uint32_t*>(&h);
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

// The horizontal lerps of one source row at the lane's V columns, all three channels, two
// columns per packed instruction (each lane of a packed fp32 operation rounds as the scalar
// one does). torch.lerp(a, b, w) is a + w*(b - a) for w < 0.5 and b - (b - a)*(1 - w)
// otherwise, one rounding each (fused); both are fma(W, Q - P, P) with (P, Q, W) = (a, b, w) or
// (b, a, 1 - w), and Q - P is exact for bytes. A column whose two taps are one pixel has W = 0
// (P = a): the lerp of a pixel with itself is the pixel. Column k's left tap starts at byte
// a0[k] of the row; its right neighbour, three bytes on, is inside the frame row too (the
// box's right edge is clipped to width - 1), so the three aligned words covering both taps
// hold only bytes of that row plus the neighbouring bytes of their own words. 2^23 + b is b's
// float with the integer in the low mantissa bits, made with one byte permute.
template <int V>
__device__ __forceinline__ void source_row_lerps(const uint8_t* row, const int (&a0)[V], const float2 (&W)[V / 2],
                                                 const bool (&left)[V], float2 (&h)[3][V / 2]) {
    uint32_t P[V], Q[V];
#pragma unroll
    for (int k = 0; k < V; ++k) {
        const uintptr_t a = reinterpret_cast<uintptr_t>(row + a0[k]);
        const uint32_t o = static_cast<uint32_t>(a) & 3u;
        const uint32_t* wp = reinterpret_cast<const uint32_t*>(a & ~static_cast<uintptr_t>(3));
        const uint32_t w0 = __ldg(wp), w1 = __ldg(wp + 1);
        const uint32_t w2 = o == 3u ? __ldg(wp + 2) : 0u;  // the right tap reaches byte 8 only from o = 3
        const uint32_t lt = __funnelshift_r(w0, w1, 8 * o);   // bytes o .. o+3
        const uint32_t nx = __funnelshift_r(w1, w2, 8 * o);   // bytes o+4 .. o+7
        const uint32_t rt = __funnelshift_r(lt, nx, 24);      // bytes o+3 .. o+6
        P[k] = left[k] ? lt : rt;
        Q[k] = left[k] ? rt : lt;
    }
    const float2 m23 = make_float2(-8388608.0f, -8388608.0f);
#pragma unroll
    for (int c = 0; c < 3; ++c)
#pragma unroll
        for (int i = 0; i < V / 2; ++i) {
            const float2 pf = make_float2(__uint_as_float(__byte_perm(P[2 * i], 0x4b000000u, 0x7440u + c)),
                                          __uint_as_float(__byte_perm(P[2 * i + 1], 0x4b000000u, 0x7440u + c)));
            const float2 qf = make_float2(__uint_as_float(__byte_perm(Q[2 * i], 0x4b000000u, 0x7440u + c)),
                                          __uint_as_float(__byte_perm(Q[2 * i + 1], 0x4b000000u, 0x7440u + c)));
            h[c][i] = __ffma2_rn(W[i], __fadd2_rn(qf, neg2(pf)), __fadd2_rn(pf, m23));
        }
}

// (v - mean) / std for crop values, correctly rounded, two per packed instruction. With
// `arith` (the host checked the constants' range) this is div_markstein without its two
// guards, which no crop value reaches:
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
// -0 (the one zero whose sign the corrections lose; +0 keeps q0's). fma(-q, d, x) is written
// fma(q, -d, x), the same exact product. With `one_step` as well (every std's RN(1/std) within
// 2^-25 relative of 1/std, true of the ImageNet constants) q0 is already faithful and the one
// correction of div_markstein_1 suffices. Without `arith`, IEEE division.
template <int V>
__device__ __forceinline__ void crop_normalise(float2 (&v)[3][V / 2], const CropParams& p) {
    if (p.one_step) {
#pragma unroll
        for (int c = 0; c < 3; ++c)
#pragma unroll
            for (int i = 0; i < V / 2; ++i)
                v[c][i] = div_markstein2_1(__fadd2_rn(v[c][i], p.nmean2[c]), p.nstd2[c], p.rcp2[c]);
    } else if (p.arith) {
#pragma unroll
        for (int c = 0; c < 3; ++c)
#pragma unroll
            for (int i = 0; i < V / 2; ++i) {
                const float2 x = __fadd2_rn(v[c][i], p.nmean2[c]);
                const float2 q0 = __fmul2_rn(x, p.rcp2[c]);
                const float2 r0 = __ffma2_rn(q0, p.nstd2[c], x);
                const float2 q1 = __ffma2_rn(r0, p.rcp2[c], q0);
                const float2 r1 = __ffma2_rn(q1, p.nstd2[c], x);
                v[c][i] = __ffma2_rn(r1, p.rcp2[c], q1);
            }
    } else {
#pragma unroll
        for (int c = 0; c < 3; ++c)
#pragma unroll
            for (int i = 0; i < V / 2; ++i) {
                v[c][i].x = __fdiv_rn(__fadd_rn(v[c][i].x, p.nmean2[c].x), -p.nstd2[c].x);
                v[c][i].y = __fdiv_rn(__fadd_rn(v[c][i].y, p.nmean2[c].y), -p.nstd2[c].y);
            }
    }
}

// 24 warps per SM at the 80 registers that allows: more warps hide more of the loads' latency
// than the unconstrained 90 registers did (20 warps per SM: 4% slower on config 3; 28, at 72
// registers: 3% slower).
template <typename OutT, int V, bool VS>
__global__ void __launch_bounds__(kWarps * 32, 24)
crop_kernel(const __grid_constant__ CropParams p) {
    static_assert(V % 2 == 0, "columns are handled in pairs");
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
    const int xb = strip * 32 * V + lane * V;  // the lane's first column
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
        for (int j = 0; j < nrows; ++j)
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                float2 z[V / 2];
#pragma unroll
                for (int i = 0; i < V / 2; ++i) z[i] = make_float2(p.zero_out[c], p.zero_out[c]);
                store_cols<OutT, V, VS>(out + c * plane + (int64_t)j * p.dst_w, z, xb, p.dst_w);
            }
        return;
    }

    // source channel c (the frame's B, G, R bytes) lands in output plane p.plane_of[c]
    OutT* dst[3];
#pragma unroll
    for (int c = 0; c < 3; ++c) dst[c] = out + p.plane_of[c] * plane;

    // the lane's columns (numpy's float32 ew / dst_w, correctly rounded: div_markstein of two
    // positive integers); columns past the right edge repeat the last one and store nothing
    int a0[V];
    float2 W[V / 2];
    bool left[V];
    const float scale_x = div_markstein((float)ew, (float)p.dst_w, p.rcp_w);
#pragma unroll
    for (int k = 0; k < V; ++k) {
        const CropAxis a = crop_axis(scale_x, ew - 1, min(xb + k, p.dst_w - 1));
        const bool same = a.i1 == a.i0;
        left[k] = same || a.w1 < 0.5f;
        const float w = same ? 0.f : (left[k] ? a.w1 : __fsub_rn(1.f, a.w1));
        if (k & 1) W[k / 2].y = w;
        else W[k / 2].x = w;
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
    // Lane j asks for the strip's bytes of row j's source rows now (into L1), so that the row
    // loop's loads of them do not each wait out a DRAM round trip. Strips wider than 16 lines
    // are left to the loads.
    {
        const int lo = __shfl_sync(0xffffffffu, a0[0], 0);
        const int hi = __shfl_sync(0xffffffffu, a0[V - 1], 31) + 5;
        if (lane < nrows && hi - lo < 16 * 128) {
            const uint8_t* r0 = row_ptr(my_s0) + lo;
            const uint8_t* r1 = row_ptr(my_s1) + lo;
            const int n = hi - lo;
            const int skip = (int)(reinterpret_cast<uintptr_t>(r0) & 127);  // r0's offset in its line
            for (int b = 0; b <= n; b = (b == 0 ? 128 - skip : b + 128)) {
                asm volatile("prefetch.global.L1 [%0];" ::"l"(r0 + b));
                if (my_s1 != my_s0) asm volatile("prefetch.global.L1 [%0];" ::"l"(r1 + b));
            }
        }
    }

    float2 top[3][V / 2], bot[3][V / 2];
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
                    for (int i = 0; i < V / 2; ++i) top[c][i] = bot[c][i];
            } else {
                source_row_lerps<V>(row_ptr(s0), a0, W, left, top);
            }
            held0 = s0;
        }
        float2 v[3][V / 2];
        if (s1 == s0) {
#pragma unroll
            for (int c = 0; c < 3; ++c)
#pragma unroll
                for (int i = 0; i < V / 2; ++i) v[c][i] = top[c][i];
        } else {
            if (s1 != held1) {
                source_row_lerps<V>(row_ptr(s1), a0, W, left, bot);
                held1 = s1;
            }
            // torch.lerp down, the weight the same for the whole warp: fma(w, d, top), or
            // fma(-d, 1 - w, bot) written fma(-(1 - w), d, bot), the same exact product
            if (wy < 0.5f) {
                const float2 w2 = make_float2(wy, wy);
#pragma unroll
                for (int c = 0; c < 3; ++c)
#pragma unroll
                    for (int i = 0; i < V / 2; ++i)
                        v[c][i] = __ffma2_rn(w2, __fadd2_rn(bot[c][i], neg2(top[c][i])), top[c][i]);
            } else {
                const float nomw = -__fsub_rn(1.f, wy);
                const float2 w2 = make_float2(nomw, nomw);
#pragma unroll
                for (int c = 0; c < 3; ++c)
#pragma unroll
                    for (int i = 0; i < V / 2; ++i)
                        v[c][i] = __ffma2_rn(w2, __fadd2_rn(bot[c][i], neg2(top[c][i])), bot[c][i]);
            }
        }
        if (live) {
            crop_normalise<V>(v, p);
            const int64_t off = (int64_t)j * p.dst_w;
#pragma unroll
            for (int c = 0; c < 3; ++c) store_cols<OutT, V, VS>(dst[c] + off, v[c], xb, p.dst_w);
        }
    }
}

template <typename OutT, int V, bool VS>
cudaError_t launch_crop_t(const CropParams& p, int grid, cudaStream_t stream) {
    return launch_dependent(crop_kernel<OutT, V, VS>, dim3(grid), dim3(kWarps * 32), 0, stream, p);
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
    p.arith = 1;
    p.rcp_w = 1.0f / (float)dst_w;
    p.rcp_h = 1.0f / (float)dst_h;
    for (int c = 0; c < 3; ++c) {
        const int oc = swap_rb ? 2 - c : c;
        p.plane_of[c] = oc;
        p.nmean2[c] = make_float2(-mean[oc], -mean[oc]);
        p.nstd2[c] = make_float2(-stdv[oc], -stdv[oc]);
        const float r = 1.0f / stdv[oc];
        p.rcp2[c] = make_float2(r, r);
        p.zero_out[c] = (0.f - mean[c]) / stdv[c];
        p.arith &= normalise_arith_ok(mean[c], stdv[c]) ? 1 : 0;
    }
    p.one_step = p.arith && markstein_one_step_ok(stdv[0]) && markstein_one_step_ok(stdv[1]) &&
                 markstein_one_step_ok(stdv[2]);
    for (int i = 0; i < n_frames; ++i) {
        p.f[i].src = frames[i].data;
        p.f[i].row_map = frames[i].row_map;
        p.f[i].pitch = frames[i].pitch;
        p.f[i].h = frames[i].height;
        p.f[i].w = frames[i].width;
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
        e = mode == 4 ? launch_crop_t<float, 4, true>(p, (int)grid, stream)
          : mode == 2 ? launch_crop_t<float, 2, true>(p, (int)grid, stream)
                      : launch_crop_t<float, 2, false>(p, (int)grid, stream);
    else
        e = mode == 4 ? launch_crop_t<__half, 4, true>(p, (int)grid, stream)
          : mode == 2 ? launch_crop_t<__half, 2, true>(p, (int)grid, stream)
                      : launch_crop_t<__half, 2, false>(p, (int)grid, stream);
    if (e != cudaSuccess) return Status{SHIPK_ECUDA, cudaGetErrorString(e)};
    return Status{SHIPK_OK, nullptr};
}

}  // namespace shipk
