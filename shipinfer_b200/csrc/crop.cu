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
// Layout: one CTA per (box, tile of R output rows, tile of up to 128 output columns), three
// steps with a barrier between each:
//   1. every thread derives the box geometry (a broadcast load of four floats); the CTA's
//      threads tabulate the horizontal taps of its columns, and one warp derives the vertical
//      taps of its R rows and the distinct source rows they read (at most 2R; a row whose
//      vertical weight is exactly 0 reads one) by a ballot over the row list;
//   2. each distinct source row is interpolated horizontally ONCE per output column (the first
//      two lerps, kept as floats in shared memory) — output rows that share a source row, as
//      every upscaled box's do, share its lerps;
//   3. each thread takes one group of VEC output pixels: the vertical lerp of two tabulated
//      rows, the channel gather, normalisation, and 16-byte stores to the three planes.
// Source bytes are read once per CTA through the read-only path; the output is written once.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <cmath>
#include <cstring>

namespace shipk {

namespace {

constexpr int kThreads = 256;
constexpr int kMaxRows = 32;   // output rows per CTA
constexpr int kMaxCols = 128;  // output columns per CTA

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
    int rows, cols;            // output rows and columns per CTA
    int row_tiles, col_tiles;  // tiles per box
    int tstride;               // floats per row of the horizontal-lerp table (cols, or more for VEC 8)
    int hl_bytes;              // shared bytes of the horizontal-lerp table: 2 rows x 3 x tstride floats
    float mean[3], stdv[3], rcp[3], zero_out[3];
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

// at::lerp: |w| < 0.5 ? a + w*(b-a) : b - (b-a)*(1-w), one rounding per branch (fused).
__device__ __forceinline__ float lerp_t(float a, float b, float w) {
    const float d = __fsub_rn(b, a);
    return fabsf(w) < 0.5f ? __fmaf_rn(w, d, a) : __fmaf_rn(-d, __fsub_rn(1.f, w), b);
}

// numpy's clip-then-cast, with a NaN coordinate clipping to 0 (undefined in the reference).
__host__ __device__ __forceinline__ int clip_trunc(float v, float hi) {
    return (int)fminf(fmaxf(v, 0.f), hi);
}


struct alignas(16) ColTap {
    int a0, a1;  // byte offsets of the two taps in the box's row segment; a1 == a0 at weight 0
    float w1;
    int unused;
};

struct alignas(16) RowTap {
    int h0, h1;  // entries of the horizontal-lerp table read by this output row
    float w1;
    int unused;
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

// The horizontal-lerp table holds, per entry and channel, one float per output column of the
// tile. Thread (g, r) of the CTA reads the VEC columns [g*VEC, g*VEC + VEC) as 16-byte chunks.
// With VEC = 8 a thread's two chunks would sit 32 bytes apart and its warp's 16-byte loads
// would meet two to a bank; so the even chunks of a row come first and the odd ones after them,
// which puts every load of one instruction on consecutive chunks. The odd half starts at a chunk
// index = 4 (mod 8), so that the 32 single-float stores of a warp (32 consecutive columns: four
// even and four odd chunks) fall on 32 different banks.
__host__ __device__ __forceinline__ int odd_base(int cols) { return (cols >> 3) + ((4 - (cols >> 3)) & 7); }

template <int VEC>
__device__ __forceinline__ int chunk_pos(int k, int cols) {
    if constexpr (VEC == 8) return (k & 1) ? odd_base(cols) + (k >> 1) : (k >> 1);
    else return k;
}

// Position of column x in a table row.
template <int VEC>
__device__ __forceinline__ int cell_pos(int x, int cols) {
    if constexpr (VEC % 4 == 0) return 4 * chunk_pos<VEC>(x >> 2, cols) + (x & 3);
    else return x;
}

template <int VEC>
__device__ __forceinline__ void get_group(const float* row, int g, int cols, float (&v)[VEC]) {
    if constexpr (VEC % 4 == 0) {
#pragma unroll
        for (int q = 0; q < VEC / 4; ++q) {
            const float4 u = *reinterpret_cast<const float4*>(row + 4 * chunk_pos<VEC>(g * (VEC / 4) + q, cols));
            v[4 * q] = u.x;
            v[4 * q + 1] = u.y;
            v[4 * q + 2] = u.z;
            v[4 * q + 3] = u.w;
        }
    } else {
#pragma unroll
        for (int q = 0; q < VEC; ++q) v[q] = row[g * VEC + q];
    }
}

// CTA: blockDim = (cols / VEC, rows'), thread (g, r) owns pixel group g of output row r.
template <typename OutT, int VEC>
__global__ void __launch_bounds__(kThreads)
crop_kernel(const __grid_constant__ CropParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ RowTap rowt[kMaxRows];
    __shared__ const uint8_t* src_ptr[2 * kMaxRows];  // byte 0 of each entry's row segment
    __shared__ int n_src_shared;

    const int g = threadIdx.x, r = threadIdx.y;
    const int tid = r * blockDim.x + g, nt = blockDim.x * blockDim.y;
    const int per_box = p.row_tiles * p.col_tiles;
    const int box = blockIdx.x / per_box;
    const int rem = blockIdx.x - box * per_box;
    const int rtile = rem / p.col_tiles, ctile = rem - rtile * p.col_tiles;
    const int y0 = rtile * p.rows, nrows = min(p.rows, p.dst_h - y0);
    const int xc0 = ctile * p.cols, ncols = min(p.cols, p.dst_w - xc0);
    const bool mine = g * VEC < ncols;  // ncols is a multiple of VEC (the host picks VEC > 1 only then)

    // ---- 1. geometry ----
    // Launched as a programmatic dependent of the stream's previous kernel: the boxes, frames
    // and output are touched only once that kernel has completed.
    griddep_wait();
    griddep_launch_dependents();
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

    const int64_t plane = (int64_t)p.dst_h * p.dst_w;
    OutT* tile_out = static_cast<OutT*>(p.out) + (int64_t)box * 3 * plane + (int64_t)y0 * p.dst_w + xc0;

    if (degenerate) {
        float v0[VEC], v1[VEC], v2[VEC];
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
            v0[k] = p.zero_out[0];
            v1[k] = p.zero_out[1];
            v2[k] = p.zero_out[2];
        }
        if (mine && r < nrows) store3<OutT, VEC>(tile_out + (int64_t)r * p.dst_w + g * VEC, plane, v0, v1, v2);
        return;
    }

    float* hl = reinterpret_cast<float*>(smem);  // [2 * rows][3][tstride]
    ColTap* colt = reinterpret_cast<ColTap*>(smem + p.hl_bytes);
    // numpy's float32 ew / dst_w, correctly rounded (div_markstein: both are positive integers)
    const float scale_x = div_markstein((float)ew, (float)p.dst_w, p.rcp_w);
    for (int x = tid; x < ncols; x += nt) {
        const CropAxis a = crop_axis(scale_x, ew - 1, xc0 + x);
        colt[x] = ColTap{a.i0 * 3, (a.w1 != 0.f ? a.i1 : a.i0) * 3, a.w1, 0};  // weight 0: lerp returns a
    }
    if (tid < 32) {
        // The distinct source rows of the tile's rows, ascending, by one warp (lane q: row q).
        // Row q reads s0 and s1, with s0 non-decreasing in q and s1 in {s0, s0 + 1}. Let M be
        // the largest row read by rows before q: s0 is new exactly when s0 > M (otherwise it is
        // s0 of row q-1, or M itself), and s1 != s0 is new exactly when s1 > M. New rows appear
        // in ascending order, so a repeated row's entry is the last one (M == it) or the one
        // before (M == it + 1).
        const int q = tid;
        const bool live = q < nrows;
        int s0 = 0x7fffffff, s1 = -1;
        float w1 = 0.f;
        if (live) {
            const CropAxis a = crop_axis(div_markstein((float)eh, (float)p.dst_h, p.rcp_h), eh - 1, y0 + q);
            s0 = a.i0;
            s1 = a.w1 != 0.f ? a.i1 : a.i0;
            w1 = a.w1;
        }
        int run = s1;  // inclusive running max of s1 over lanes 0..q
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int o = __shfl_up_sync(0xffffffffu, run, d);
            if (q >= d) run = max(run, o);
        }
        int m = __shfl_up_sync(0xffffffffu, run, 1);  // M: rows before q
        if (q == 0) m = -1;
        const bool new0 = live && s0 > m;
        const bool new1 = live && s1 != s0 && s1 > m;
        const unsigned b0 = __ballot_sync(0xffffffffu, new0), b1 = __ballot_sync(0xffffffffu, new1);
        const unsigned below = (1u << q) - 1u;
        const int before = __popc(b0 & below) + __popc(b1 & below);
        const int e0 = new0 ? before : (m == s0 ? before - 1 : before - 2);
        const int e1 = s1 == s0 ? e0 : (new1 ? before + (int)new0 : before - 1);
        auto segment = [&](int sr) {
            const int row = F.row_map ? __ldg(F.row_map + sr) : sr;
            return F.src + (int64_t)row * F.pitch + (int64_t)x1 * 3;
        };
        if (new0) src_ptr[before] = segment(y1 + s0);
        if (new1) src_ptr[before + (int)new0] = segment(y1 + s1);
        if (live) rowt[q] = RowTap{e0, e1, w1, 0};
        if (q == 0) n_src_shared = __popc(b0) + __popc(b1);
    }
    __syncthreads();

    // ---- 2. horizontal lerps of each distinct source row, once per output column ----
    // Items (entry j, column x) dealt to the CTA's threads in order; each thread walks its items
    // by a fixed step (one division to start), four at a time: the bytes of all four are
    // requested before any is used, so their cache latencies overlap.
    const int n_src = n_src_shared;
    {
        constexpr int kU = 4;
        int j = tid / ncols, x = tid - j * ncols;
        const int dj = nt / ncols, dx = nt - dj * ncols;
        while (j < n_src) {
            int jj[kU], xx[kU];
            bool ok[kU];
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                ok[u] = j < n_src;
                jj[u] = ok[u] ? j : 0;  // entry 0 exists: this loop runs only when n_src >= 1
                xx[u] = ok[u] ? x : 0;
                x += dx;
                j += dj;
                if (x >= ncols) {
                    x -= ncols;
                    ++j;
                }
            }
            uint32_t b0[kU][3], b1[kU][3];
            float w1[kU];
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const ColTap t = colt[xx[u]];
                const uint8_t* src = src_ptr[jj[u]];
                w1[u] = t.w1;
#pragma unroll
                for (int c = 0; c < 3; ++c) {
                    b0[u][c] = __ldg(src + t.a0 + c);
                    b1[u][c] = __ldg(src + t.a1 + c);
                }
            }
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                if (!ok[u]) continue;
                float* dst = hl + (jj[u] * 3) * p.tstride + cell_pos<VEC>(xx[u], p.cols);
#pragma unroll
                for (int c = 0; c < 3; ++c) dst[c * p.tstride] = lerp_t(u8f(b0[u][c]), u8f(b1[u][c]), w1[u]);
            }
        }
    }
    __syncthreads();

    // ---- 3. vertical lerp, gather, normalise, store ----
    if (!mine || r >= nrows) return;
    const RowTap rt = rowt[r];
    float v[3][VEC];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        float top[VEC], bot[VEC];
        get_group<VEC>(hl + (rt.h0 * 3 + c) * p.tstride, g, p.cols, top);
        get_group<VEC>(hl + (rt.h1 * 3 + c) * p.tstride, g, p.cols, bot);
#pragma unroll
        for (int k = 0; k < VEC; ++k) v[c][k] = lerp_t(top[k], bot[k], rt.w1);
    }
    float v0[VEC], v1[VEC], v2[VEC];
    bool none[VEC];
#pragma unroll
    for (int k = 0; k < VEC; ++k) {
        v0[k] = p.swap_rb ? v[2][k] : v[0][k];
        v1[k] = v[1][k];
        v2[k] = p.swap_rb ? v[0][k] : v[2][k];
        none[k] = false;
    }
    normalise_group<VEC>(v0, v1, v2, none, p.mean, p.stdv, p.rcp, p.arith);
    store3<OutT, VEC>(tile_out + (int64_t)r * p.dst_w + g * VEC, plane, v0, v1, v2);
}

template <typename OutT, int VEC>
cudaError_t launch_crop_t(const CropParams& p, int grid, dim3 block, int smem, cudaStream_t stream) {
    cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(crop_kernel<OutT, VEC>), smem);
    if (e != cudaSuccess) return e;
    return launch_dependent(crop_kernel<OutT, VEC>, dim3(grid), block, smem, stream, p);
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
    const bool aligned = (reinterpret_cast<uintptr_t>(out) & 15) == 0;
    const int vec = out_dtype == SHIPK_DTYPE_F32 ? ((aligned && dst_w % 4 == 0) ? 4 : 1)
                                                 : ((aligned && dst_w % 8 == 0) ? 8 : 1);
    // Tiles: up to 128 columns (a multiple of vec) and as many rows as give 256 threads one
    // group each, at most 32.
    p.cols = std::min(dst_w, kMaxCols);
    const int gpr = p.cols / vec;
    p.rows = std::max(1, std::min({kMaxRows, kThreads / gpr, dst_h}));
    p.row_tiles = (dst_h + p.rows - 1) / p.rows;
    p.col_tiles = (dst_w + p.cols - 1) / p.cols;
    p.tstride = vec == 8 ? 4 * (odd_base(p.cols) + p.cols / 8) : p.cols;
    p.hl_bytes = (2 * p.rows * 3 * p.tstride * (int)sizeof(float) + 15) / 16 * 16;
    const int smem = p.hl_bytes + p.cols * (int)sizeof(ColTap);
    // thread (g, r): group g of row r; at least one full warp (it derives the row taps)
    const dim3 block(gpr, std::max(p.rows, (32 + gpr - 1) / gpr));
    const long long grid = (long long)n_boxes * p.row_tiles * p.col_tiles;
    if (grid > 0x7fffffffLL) return Status{SHIPK_ERANGE, "too many boxes for one launch"};
    cudaError_t e;
    if (out_dtype == SHIPK_DTYPE_F32)
        e = vec == 4 ? launch_crop_t<float, 4>(p, (int)grid, block, smem, stream)
                     : launch_crop_t<float, 1>(p, (int)grid, block, smem, stream);
    else
        e = vec == 8 ? launch_crop_t<__half, 8>(p, (int)grid, block, smem, stream)
                     : launch_crop_t<__half, 1>(p, (int)grid, block, smem, stream);
    if (e != cudaSuccess) return Status{SHIPK_ECUDA, cudaGetErrorString(e)};
    return Status{SHIPK_OK, nullptr};
}

}  // namespace shipk
