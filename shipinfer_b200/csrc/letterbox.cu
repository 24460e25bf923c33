// Fused letterbox: bilinear resize (half-pixel centres) + pad + BGR->RGB + normalise +
// NHWC->NCHW in one pass, for a whole batch of frames in one launch. BGR uint8 frames, and
// NV12 surfaces (BT.601 / BT.709 limited range, nearest or bilinear).
//
// Reference formulation: TorchImageOps._letterbox, src/shipinfer/runtime/ops/torch_ops.py:
// 349-403 (F.interpolate bilinear, align_corners=False, then paste, flip, sub, div); for NV12
// the reference's nv12_letterbox_kernel, csrc/shipinfer/runtime/ops.cu:148-194.
//
// Layout. The canvas is cut into tiles of `rows` output rows of one frame; a persistent grid
// (a whole number of CTAs per SM) walks the tiles. For each tile, `rows` threads derive the
// vertical taps of their row in parallel; the CTA stages every source row with a non-zero
// vertical weight (one row in three at 1080p -> 640) into shared memory with 16-byte cp.async
// copies, then each thread writes 16-byte streaming stores of one pixel group for all three
// planes. Pad rows never touch the source. HBM traffic is the compulsory bytes: the output
// and the contributing source rows.
//
// Exact taps. Where both tap weights of a pixel are exactly 0 and 1 (every pixel at 1080p ->
// 640: the ratio is exactly 3), the bilinear value IS the integer source pixel, so its
// normalised value comes from a 3 x 256 table built per CTA with the same normalise() — the
// same function of the same integer, hence the same bits — instead of a divide per element.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

namespace shipk {

namespace {

constexpr int kThreads = 256;
constexpr int kMaxRows = 8;            // output rows per tile (upper bound)
constexpr int kMaxSpr = 4;             // staged rows per output row: NV12 bilinear needs 4
constexpr int kSmemTarget = 32 * 1024; // staging per CTA the planner aims for (occupancy)
constexpr int kSmemMax = 200 * 1024;   // hard ceiling for very wide frames

struct LbFrame {
    const uint8_t* src;      // BGR rows, or NV12 luma
    const int32_t* row_map;  // staged row of each source row, or null (identity)
    int64_t pitch;
    int64_t uv_offset;       // NV12 only
    int src_h, src_w;
    int new_h, new_w, pad_y, pad_x;
    float rh, rw;            // (float)src / (float)new, as torch computes its ratio
};

struct LbParams {
    void* out;
    int n, dst_h, dst_w;
    int rows;                // output rows per tile
    int tiles;               // tiles per frame
    int total_tiles;
    int spr;                 // staged source rows per output row (1, 2 or 4)
    int slot_bytes;          // bytes per staged row in shared memory (multiple of 16)
    float mean[3], stdv[3], pad_out[3];
    int swap_rb;
    int matrix, sampling;    // NV12 only
    LbFrame f[kMaxBatch];
};

struct RowInfo {
    Tap ty;
    int inside;
    int src[kMaxSpr];  // source row per staged slot (NV12: luma i0, luma i1, chroma i0, chroma i1), -1: unused
};

// ---- shared helpers ------------------------------------------------------------------------

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
}

// Stage src[0, nbytes) into dst so that shared and global agree modulo 16 (byte k at
// dst[(src & 15) + k]); the aligned middle moves by 16-byte cp.async, the ragged head and tail
// by byte loads. Every global access stays inside [src, src + nbytes).
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

// ---- BGR uint8 ---------------------------------------------------------------------------

template <typename OutT, int VEC>
__global__ void __launch_bounds__(kThreads)
letterbox_u8_kernel(const __grid_constant__ LbParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ RowInfo rows[kMaxRows];
    __shared__ const uint8_t* slot_ptr[kMaxRows * kMaxSpr];
    __shared__ float lut[3][256];

    const int tid = threadIdx.x;
    for (int k = tid; k < 3 * 256; k += kThreads) {
        const int c = k >> 8;
        lut[c][k & 255] = normalise((float)(k & 255), p.mean[c], p.stdv[c]);
    }
    const int64_t plane = (int64_t)p.dst_h * p.dst_w;
    const int groups = (p.dst_w + VEC - 1) / VEC;
    const int c_src0 = p.swap_rb ? 2 : 0, c_src2 = p.swap_rb ? 0 : 2;
    const float pad0 = p.pad_out[0], pad1 = p.pad_out[1], pad2 = p.pad_out[2];

    for (int tile_id = blockIdx.x; tile_id < p.total_tiles; tile_id += gridDim.x) {
        const int img = tile_id / p.tiles;
        const int y0 = (tile_id - img * p.tiles) * p.rows;
        const int nrows = min(p.rows, p.dst_h - y0);
        const LbFrame& F = p.f[img];

        __syncthreads();  // the previous tile is done with rows[] and the staging
        // An unstaged slot points at the (harmless) staging base, never at a stale address.
        if (tid < kMaxRows * kMaxSpr) slot_ptr[tid] = smem;
        if (tid < nrows) {
            RowInfo& ri = rows[tid];
            const int dy = y0 + tid - F.pad_y;
            const int inside = dy >= 0 && dy < F.new_h;
            ri.inside = inside;
            ri.src[0] = -1;
            ri.src[1] = -1;
            if (inside) {
                const Tap ty = interp_tap(F.rh, dy, F.src_h);
                ri.ty = ty;
                ri.src[0] = ty.i0;
                // the planner saw the same taps and gave this launch 2 slots per row
                if (ty.l1 != 0.f && p.spr > 1) ri.src[1] = ty.i1;
            }
        }
        __syncthreads();
        const int row_bytes = F.src_w * 3;
        for (int s = 0; s < nrows * p.spr; ++s) {
            const int r = s / p.spr, k = s - r * p.spr;
            const int sr = rows[r].src[k];
            if (sr < 0) continue;
            const int row = F.row_map ? __ldg(F.row_map + sr) : sr;
            const uint8_t* base = stage_async(smem + s * p.slot_bytes, F.src + (int64_t)row * F.pitch,
                                              row_bytes, tid, kThreads);
            if (tid == 0) slot_ptr[s] = base;
        }
        cp_async_wait_all();
        __syncthreads();

        OutT* img_out = static_cast<OutT*>(p.out) + (int64_t)img * 3 * plane;
        const int items = nrows * groups;
        for (int it = tid; it < items; it += kThreads) {
            const int r = it / groups;
            const int x0 = (it - r * groups) * VEC;
            float v0[VEC], v1[VEC], v2[VEC];
            if (!rows[r].inside) {
#pragma unroll
                for (int k = 0; k < VEC; ++k) {
                    v0[k] = pad0;
                    v1[k] = pad1;
                    v2[k] = pad2;
                }
            } else {
                const Tap ty = rows[r].ty;
                const uint8_t* s0 = slot_ptr[r * p.spr];
                const uint8_t* s1 = rows[r].src[1] >= 0 ? slot_ptr[r * p.spr + 1] : nullptr;
#pragma unroll
                for (int k = 0; k < VEC; ++k) {
                    const int dx = x0 + k - F.pad_x;
                    if (dx < 0 || dx >= F.new_w) {
                        v0[k] = pad0;
                        v1[k] = pad1;
                        v2[k] = pad2;
                        continue;
                    }
                    const Tap tx = interp_tap(F.rw, dx, F.src_w);
                    const int a0 = tx.i0 * 3;
                    if (s1 == nullptr && tx.l1 == 0.f) {
                        // both weights are exactly 1 and 0: the value is the integer pixel
                        v0[k] = lut[0][s0[a0 + c_src0]];
                        v1[k] = lut[1][s0[a0 + 1]];
                        v2[k] = lut[2][s0[a0 + c_src2]];
                        continue;
                    }
                    const int a1 = tx.i1 * 3;
                    const bool right = tx.l1 != 0.f;
                    float px[3];
#pragma unroll
                    for (int c = 0; c < 3; ++c) {
                        // a tap whose weight is exactly 0 contributes exactly 0: not read
                        const float p00 = s0[a0 + c];
                        const float p01 = right ? (float)s0[a1 + c] : 0.f;
                        const float p10 = s1 ? (float)s1[a0 + c] : 0.f;
                        const float p11 = (s1 && right) ? (float)s1[a1 + c] : 0.f;
                        px[c] = interp_blend(ty, tx, p00, p01, p10, p11);
                    }
                    v0[k] = normalise(p.swap_rb ? px[2] : px[0], p.mean[0], p.stdv[0]);
                    v1[k] = normalise(px[1], p.mean[1], p.stdv[1]);
                    v2[k] = normalise(p.swap_rb ? px[0] : px[2], p.mean[2], p.stdv[2]);
                }
            }
            store3<OutT, VEC>(img_out + (int64_t)(y0 + r) * p.dst_w + x0, plane, v0, v1, v2);
        }
    }
}

// ---- NV12 --------------------------------------------------------------------------------
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

// One pixel to BGR: Y' = (Y - 16) * ys; B = Y' + cbu*U; G = Y' - cgu*U - cgv*V;
// R = Y' + crv*V, each sum fused as nvcc contracts the reference's expressions, clamped.
__device__ __forceinline__ void yuv_to_bgr(const YuvMatrix& m, const uint8_t* yrow,
                                           const uint8_t* uvrow, int xi, float bgr[3]) {
    const float Y = __fmul_rn(__fsub_rn((float)yrow[xi], 16.f), m.ys);
    const int cx = (xi >> 1) << 1;
    const float U = __fsub_rn((float)uvrow[cx], 128.f);
    const float V = __fsub_rn((float)uvrow[cx + 1], 128.f);
    const float b = __fmaf_rn(m.cbu, U, Y);
    const float g = __fmaf_rn(-m.cgv, V, __fmaf_rn(-m.cgu, U, Y));
    const float r = __fmaf_rn(m.crv, V, Y);
    bgr[0] = fminf(255.f, fmaxf(0.f, b));
    bgr[1] = fminf(255.f, fmaxf(0.f, g));
    bgr[2] = fminf(255.f, fmaxf(0.f, r));
}

// The reference NV12 kernel's source coordinate, ops.cu:167-172: max(0, ((d + .5) * in) /
// out - .5) with every step rounded.
__host__ __device__ __forceinline__ int ref_nearest(int d, int in_size, int out_size) {
#ifdef __CUDA_ARCH__
    float a = __fadd_rn((float)d, 0.5f);
    float b = __fmul_rn(a, (float)in_size);
    float c = __fdiv_rn(b, (float)out_size);
    float r = fmaxf(0.f, __fsub_rn(c, 0.5f));
#else
    float a = (float)d + 0.5f;
    float b = a * (float)in_size;
    float c = b / (float)out_size;
    float r = std::max(0.f, c - 0.5f);
#endif
    return min((int)r, in_size - 1);
}

template <typename OutT, int VEC>
__global__ void __launch_bounds__(kThreads)
letterbox_nv12_kernel(const __grid_constant__ LbParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ RowInfo rows[kMaxRows];
    __shared__ const uint8_t* slot_ptr[kMaxRows * kMaxSpr];

    const int tid = threadIdx.x;
    const bool nearest = p.sampling == 0;
    const int half = p.spr >> 1;  // first chroma slot of a row
    const YuvMatrix m = yuv_matrix(p.matrix);
    const int64_t plane = (int64_t)p.dst_h * p.dst_w;
    const int groups = (p.dst_w + VEC - 1) / VEC;

    for (int tile_id = blockIdx.x; tile_id < p.total_tiles; tile_id += gridDim.x) {
        const int img = tile_id / p.tiles;
        const int y0 = (tile_id - img * p.tiles) * p.rows;
        const int nrows = min(p.rows, p.dst_h - y0);
        const LbFrame& F = p.f[img];

        __syncthreads();
        // An unstaged slot points at the (harmless) staging base, never at a stale address.
        if (tid < kMaxRows * kMaxSpr) slot_ptr[tid] = smem;
        if (tid < nrows) {
            RowInfo& ri = rows[tid];
            const int dy = y0 + tid - F.pad_y;
            const int inside = dy >= 0 && dy < F.new_h;
            ri.inside = inside;
            ri.src[0] = ri.src[1] = ri.src[2] = ri.src[3] = -1;
            if (inside) {
                int luma0, luma1 = -1;
                if (nearest) {
                    luma0 = ref_nearest(dy, F.src_h, F.new_h);
                } else {
                    const Tap ty = interp_tap(F.rh, dy, F.src_h);
                    ri.ty = ty;
                    luma0 = ty.i0;
                    if (ty.l1 != 0.f && half == 2) luma1 = ty.i1;  // the planner gave 4 slots per row
                }
                ri.src[0] = luma0;
                if (half == 2) {
                    ri.src[1] = luma1;
                    ri.src[2] = luma0 >> 1;
                    ri.src[3] = luma1 >= 0 ? luma1 >> 1 : -1;
                } else {
                    ri.src[1] = luma0 >> 1;
                }
            }
        }
        __syncthreads();
        const int luma_bytes = F.src_w;
        const int chroma_bytes = ((F.src_w + 1) >> 1) << 1;
        for (int s = 0; s < nrows * p.spr; ++s) {
            const int r = s / p.spr, k = s - r * p.spr;
            const int sr = rows[r].src[k];
            if (sr < 0) continue;
            const bool chroma = k >= half;
            const uint8_t* g = chroma ? F.src + F.uv_offset + (int64_t)sr * F.pitch : F.src + (int64_t)sr * F.pitch;
            const uint8_t* base = stage_async(smem + s * p.slot_bytes, g, chroma ? chroma_bytes : luma_bytes,
                                              tid, kThreads);
            if (tid == 0) slot_ptr[s] = base;
        }
        cp_async_wait_all();
        __syncthreads();

        OutT* img_out = static_cast<OutT*>(p.out) + (int64_t)img * 3 * plane;
        const int items = nrows * groups;
        for (int it = tid; it < items; it += kThreads) {
            const int r = it / groups;
            const int x0 = (it - r * groups) * VEC;
            const RowInfo& ri = rows[r];
            float v0[VEC], v1[VEC], v2[VEC];
#pragma unroll
            for (int k = 0; k < VEC; ++k) {
                const int dx = x0 + k - F.pad_x;
                if (!ri.inside || dx < 0 || dx >= F.new_w) {
                    v0[k] = p.pad_out[0];
                    v1[k] = p.pad_out[1];
                    v2[k] = p.pad_out[2];
                    continue;
                }
                float px[3];
                const uint8_t* y0p = slot_ptr[r * p.spr];
                const uint8_t* u0p = slot_ptr[r * p.spr + half];
                if (nearest) {
                    yuv_to_bgr(m, y0p, u0p, ref_nearest(dx, F.src_w, F.new_w), px);
                } else {
                    const Tap ty = ri.ty;
                    const Tap tx = interp_tap(F.rw, dx, F.src_w);
                    const bool right = tx.l1 != 0.f;
                    // a second luma row exists only in the 4-slot layout; in the 2-slot one,
                    // slot 1 is the chroma row
                    const bool below = half == 2 && ri.src[1] >= 0;
                    float q00[3], q01[3] = {0.f, 0.f, 0.f}, q10[3] = {0.f, 0.f, 0.f}, q11[3] = {0.f, 0.f, 0.f};
                    yuv_to_bgr(m, y0p, u0p, tx.i0, q00);
                    if (right) yuv_to_bgr(m, y0p, u0p, tx.i1, q01);
                    if (below) {
                        const uint8_t* y1p = slot_ptr[r * p.spr + 1];
                        const uint8_t* u1p = slot_ptr[r * p.spr + 3];
                        yuv_to_bgr(m, y1p, u1p, tx.i0, q10);
                        if (right) yuv_to_bgr(m, y1p, u1p, tx.i1, q11);
                    }
#pragma unroll
                    for (int c = 0; c < 3; ++c) px[c] = interp_blend(ty, tx, q00[c], q01[c], q10[c], q11[c]);
                }
                v0[k] = normalise(p.swap_rb ? px[2] : px[0], p.mean[0], p.stdv[0]);
                v1[k] = normalise(px[1], p.mean[1], p.stdv[1]);
                v2[k] = normalise(p.swap_rb ? px[0] : px[2], p.mean[2], p.stdv[2]);
            }
            store3<OutT, VEC>(img_out + (int64_t)(y0 + r) * p.dst_w + x0, plane, v0, v1, v2);
        }
    }
}

// ---- host-side planning --------------------------------------------------------------------

// Does any output row of this frame blend two source rows (a non-zero lower weight)?
bool needs_second_row(const LbFrame& f) {
    for (int dy = 0; dy < f.new_h; ++dy)
        if (interp_tap(f.rh, dy, f.src_h).l1 != 0.f) return true;
    return false;
}

struct Plan {
    LbParams p;
    int smem;
};

const char* plan_letterbox(const FrameView* frames, int n, void* out, int dst_h, int dst_w,
                           const float mean[3], const float stdv[3], int swap_rb,
                           float pad_value, bool nv12, int matrix, int sampling, Plan* plan) {
    LbParams& p = plan->p;
    std::memset(&p, 0, sizeof(p));
    p.out = out;
    p.n = n;
    p.dst_h = dst_h;
    p.dst_w = dst_w;
    p.swap_rb = swap_rb;
    p.matrix = matrix;
    p.sampling = sampling;
    for (int c = 0; c < 3; ++c) {
        p.mean[c] = mean[c];
        p.stdv[c] = stdv[c];
        p.pad_out[c] = (pad_value - mean[c]) / stdv[c];
    }
    int max_row_bytes = 16;
    bool second = false;
    for (int i = 0; i < n; ++i) {
        LbFrame& f = p.f[i];
        Fit fit;
        letterbox_fit(frames[i].height, frames[i].width, dst_h, dst_w, &fit);
        f.src = frames[i].data;
        f.row_map = frames[i].row_map;
        f.pitch = frames[i].pitch;
        f.uv_offset = frames[i].uv_offset;
        f.src_h = frames[i].height;
        f.src_w = frames[i].width;
        f.new_h = fit.new_h;
        f.new_w = fit.new_w;
        f.pad_y = fit.pad_y;
        f.pad_x = fit.pad_x;
        f.rh = (float)f.src_h / (float)f.new_h;
        f.rw = (float)f.src_w / (float)f.new_w;
        const int rb = nv12 ? (((f.src_w + 1) >> 1) << 1) : f.src_w * 3;
        max_row_bytes = std::max(max_row_bytes, rb);
        if (!(nv12 && sampling == 0)) second = second || needs_second_row(f);
    }
    // Slots per output row. BGR: i0 [, i1]. NV12: luma i0 [, luma i1], then chroma i0 [, i1]
    // (the first chroma slot is at spr / 2).
    p.spr = nv12 ? (second && sampling != 0 ? 4 : 2) : (second ? 2 : 1);
    p.slot_bytes = ((max_row_bytes + 16 + 15) / 16) * 16;
    int rows = kMaxRows;
    while (rows > 1 && rows * p.spr * p.slot_bytes > kSmemTarget) rows >>= 1;
    if (rows * p.spr * p.slot_bytes > kSmemMax) return "source rows are too wide to stage in shared memory";
    p.rows = std::min(rows, dst_h);
    p.tiles = (dst_h + p.rows - 1) / p.rows;
    p.total_tiles = n * p.tiles;
    plan->smem = p.rows * p.spr * p.slot_bytes;
    return nullptr;
}

int sm_count() {
    static std::mutex mu;
    static std::map<int, int> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(dev);
    if (it != cache.end()) return it->second;
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
    cache[dev] = sms;
    return sms;
}

// Resident CTAs per SM for this kernel at this dynamic shared memory size.
int occupancy(const void* kernel, int smem) {
    static std::mutex mu;
    static std::map<std::tuple<const void*, int, int>, int> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    auto key = std::make_tuple(kernel, smem, dev);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    int blocks = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, kThreads, smem) != cudaSuccess || blocks < 1)
        blocks = 1;
    cache[key] = blocks;
    return blocks;
}

template <typename OutT, int VEC, bool NV12>
cudaError_t launch_one(const Plan& plan, cudaStream_t stream) {
    auto kernel = NV12 ? letterbox_nv12_kernel<OutT, VEC> : letterbox_u8_kernel<OutT, VEC>;
    const void* fn = reinterpret_cast<const void*>(kernel);
    cudaError_t e = ensure_smem_attr(fn, kSmemMax);
    if (e != cudaSuccess) return e;
    const int resident = occupancy(fn, plan.smem) * sm_count();
    const int grid = std::max(1, std::min(plan.p.total_tiles, resident));
    kernel<<<grid, kThreads, plan.smem, stream>>>(plan.p);
    return cudaGetLastError();
}

template <bool NV12>
cudaError_t launch_plan(const Plan& plan, int out_dtype, cudaStream_t stream) {
    const bool aligned = (reinterpret_cast<uintptr_t>(plan.p.out) & 15) == 0;
    if (out_dtype == SHIPK_DTYPE_F32)
        return aligned && plan.p.dst_w % 4 == 0 ? launch_one<float, 4, NV12>(plan, stream)
                                                : launch_one<float, 1, NV12>(plan, stream);
    return aligned && plan.p.dst_w % 8 == 0 ? launch_one<__half, 8, NV12>(plan, stream)
                                            : launch_one<__half, 1, NV12>(plan, stream);
}

}  // namespace

int letterbox_fit(int src_h, int src_w, int dst_h, int dst_w, Fit* out) {
    if (src_h <= 0 || src_w <= 0 || dst_h <= 0 || dst_w <= 0) return SHIPK_EINVAL;
    // torch_ops.py:374-378, in Python's double precision; nearbyint() rounds half to even.
    const double sh = (double)dst_h / (double)src_h;
    const double sw = (double)dst_w / (double)src_w;
    const double s = std::min(sh, sw);
    const double nh = std::nearbyint((double)src_h * s);
    const double nw = std::nearbyint((double)src_w * s);
    out->new_h = nh < 1.0 ? 1 : (int)nh;
    out->new_w = nw < 1.0 ? 1 : (int)nw;
    out->pad_y = (dst_h - out->new_h) / 2;  // dst >= new, so C and floor division agree
    out->pad_x = (dst_w - out->new_w) / 2;
    out->scale = (float)s;
    return SHIPK_OK;
}

void letterbox_rows_needed(int src_h, int new_h, unsigned char* needed) {
    const float rh = (float)src_h / (float)new_h;
    for (int r = 0; r < src_h; ++r) needed[r] = 0;
    for (int dy = 0; dy < new_h; ++dy) {
        const Tap t = interp_tap(rh, dy, src_h);
        needed[t.i0] = 1;
        if (t.l1 != 0.f) needed[t.i1] = 1;
    }
}

Status launch_letterbox(const FrameView* frames, int n, void* out, int out_dtype, int dst_h,
                        int dst_w, const float mean[3], const float stdv[3], int swap_rb,
                        float pad_value, bool nv12, int matrix, int sampling,
                        cudaStream_t stream) {
    const size_t elem = out_dtype == SHIPK_DTYPE_F32 ? 4 : 2;
    const size_t per_image = (size_t)3 * dst_h * dst_w * elem;
    for (int start = 0; start < n; start += kMaxBatch) {
        const int count = std::min(kMaxBatch, n - start);
        Plan plan;
        const char* why = plan_letterbox(frames + start, count,
                                         static_cast<uint8_t*>(out) + per_image * start, dst_h,
                                         dst_w, mean, stdv, swap_rb, pad_value, nv12, matrix,
                                         sampling, &plan);
        if (why) return Status{SHIPK_ERANGE, why};
        cudaError_t e = nv12 ? launch_plan<true>(plan, out_dtype, stream)
                             : launch_plan<false>(plan, out_dtype, stream);
        if (e != cudaSuccess) return Status{SHIPK_ECUDA, cudaGetErrorString(e)};
    }
    return Status{SHIPK_OK, nullptr};
}

}  // namespace shipk
