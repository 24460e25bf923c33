// Fused letterbox: bilinear resize (half-pixel centres) + pad + BGR->RGB + normalise +
// NHWC->NCHW in one pass, for a whole batch of frames in one launch.
//
// Reference formulation: TorchImageOps._letterbox, src/shipinfer/runtime/ops/torch_ops.py:
// 349-403 (F.interpolate bilinear, align_corners=False, then paste, flip, sub, div).
//
// Layout: one CTA per (frame, tile of kRows output rows). The CTA first works out which
// source rows its output rows read (the row with non-zero vertical weight only: at
// 1080p -> 640 that is one source row in three), stages each distinct row once into shared
// memory with 16-byte coalesced loads, then writes every output element of its tile with
// 16-byte streaming stores, three planes per pixel group. Pad rows never touch the source.
// HBM traffic is therefore the compulsory bytes: the output, plus the contributing rows.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <cmath>
#include <cstring>

namespace shipk {

namespace {

constexpr int kThreads = 256;
constexpr int kMaxRows = 8;               // output rows per CTA (upper bound)
constexpr int kMaxSlots = 4 * kMaxRows;   // distinct source rows per CTA (NV12: 2 luma + 2 chroma per row)
constexpr int kSmemBudget = 200 * 1024;   // dynamic shared memory per CTA

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
    int rows;                // output rows per CTA
    int tiles;               // CTAs per frame
    int slot_bytes;          // bytes per staged row in shared memory (multiple of 16)
    int max_slots;           // rows the dynamic shared memory holds; any further row is read
                             // from global memory in place (never taken when the host plan and
                             // the device agree, which they do: both use interp_tap)
    float mean[3], stdv[3], pad_out[3];
    int swap_rb;
    int matrix, sampling;    // NV12 only
    LbFrame f[kMaxBatch];
};

struct TileRows {
    int nslots;
    int slot_row[kMaxSlots];   // source row staged in each slot
    int slot_uv[kMaxSlots];    // NV12: 1 when the slot holds a chroma row
    int s0[kMaxRows], s1[kMaxRows];     // slot of tap row i0 / i1 (-1: weight 0, not read)
    int c0[kMaxRows], c1[kMaxRows];     // NV12 chroma slots
    Tap ty[kMaxRows];
    int inside[kMaxRows];
};

__device__ __forceinline__ int find_or_add(TileRows& t, int row, int uv) {
    for (int s = 0; s < t.nslots; ++s)
        if (t.slot_row[s] == row && t.slot_uv[s] == uv) return s;
    t.slot_row[t.nslots] = row;
    t.slot_uv[t.nslots] = uv;
    return t.nslots++;
}

// ---- BGR uint8 ---------------------------------------------------------------------------

template <typename OutT, int VEC>
__global__ void __launch_bounds__(kThreads)
letterbox_u8_kernel(const __grid_constant__ LbParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ TileRows t;
    __shared__ const uint8_t* slot_ptr[kMaxSlots];

    const int img = blockIdx.x / p.tiles;
    const int tile = blockIdx.x - img * p.tiles;
    const LbFrame& F = p.f[img];
    const int y0 = tile * p.rows;
    const int nrows = min(p.rows, p.dst_h - y0);

    if (threadIdx.x == 0) {
        t.nslots = 0;
        for (int r = 0; r < nrows; ++r) {
            const int dy = y0 + r - F.pad_y;
            t.inside[r] = dy >= 0 && dy < F.new_h;
            t.s0[r] = t.s1[r] = -1;
            if (!t.inside[r]) continue;
            Tap ty = interp_tap(F.rh, dy, F.src_h);
            t.ty[r] = ty;
            t.s0[r] = find_or_add(t, ty.i0, 0);
            if (ty.l1 != 0.f) t.s1[r] = find_or_add(t, ty.i1, 0);
        }
    }
    __syncthreads();

    const int row_bytes = F.src_w * 3;
    for (int s = 0; s < t.nslots; ++s) {
        const int row = F.row_map ? F.row_map[t.slot_row[s]] : t.slot_row[s];
        const uint8_t* g = F.src + (int64_t)row * F.pitch;
        if (s < p.max_slots) {
            const uint8_t* base =
                stage_bytes(smem + s * p.slot_bytes, g, row_bytes, threadIdx.x, kThreads);
            if (threadIdx.x == 0) slot_ptr[s] = base;
        } else if (threadIdx.x == 0) {
            slot_ptr[s] = g;
        }
    }
    __syncthreads();

    OutT* out = static_cast<OutT*>(p.out);
    const int64_t plane = (int64_t)p.dst_h * p.dst_w;
    OutT* img_out = out + (int64_t)img * 3 * plane;
    const int groups = (p.dst_w + VEC - 1) / VEC;
    const int items = nrows * groups;
    const float pad0 = p.pad_out[0], pad1 = p.pad_out[1], pad2 = p.pad_out[2];
    const int c_src0 = p.swap_rb ? 2 : 0, c_src2 = p.swap_rb ? 0 : 2;

    for (int it = threadIdx.x; it < items; it += kThreads) {
        const int r = it / groups;
        const int g = it - r * groups;
        const int y = y0 + r;
        const int x0 = g * VEC;
        float v0[VEC], v1[VEC], v2[VEC];
        if (!t.inside[r]) {
#pragma unroll
            for (int k = 0; k < VEC; ++k) {
                v0[k] = pad0;
                v1[k] = pad1;
                v2[k] = pad2;
            }
        } else {
            const Tap ty = t.ty[r];
            const uint8_t* s0 = slot_ptr[t.s0[r]];
            const uint8_t* s1 = t.s1[r] >= 0 ? slot_ptr[t.s1[r]] : nullptr;
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
                const int a0 = tx.i0 * 3, a1 = tx.i1 * 3;
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
                v0[k] = normalise(px[c_src0], p.mean[0], p.stdv[0]);
                v1[k] = normalise(px[1], p.mean[1], p.stdv[1]);
                v2[k] = normalise(px[c_src2], p.mean[2], p.stdv[2]);
            }
        }
        OutT* o = img_out + (int64_t)y * p.dst_w + x0;
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
__device__ __forceinline__ int ref_nearest(int d, int in_size, int out_size) {
    float a = __fadd_rn((float)d, 0.5f);
    float b = __fmul_rn(a, (float)in_size);
    float c = __fdiv_rn(b, (float)out_size);
    float r = fmaxf(0.f, __fsub_rn(c, 0.5f));
    return min((int)r, in_size - 1);
}

template <typename OutT, int VEC>
__global__ void __launch_bounds__(kThreads)
letterbox_nv12_kernel(const __grid_constant__ LbParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ TileRows t;
    __shared__ const uint8_t* slot_ptr[kMaxSlots];

    const int img = blockIdx.x / p.tiles;
    const int tile = blockIdx.x - img * p.tiles;
    const LbFrame& F = p.f[img];
    const int y0 = tile * p.rows;
    const int nrows = min(p.rows, p.dst_h - y0);
    const bool nearest = p.sampling == 0;

    if (threadIdx.x == 0) {
        t.nslots = 0;
        for (int r = 0; r < nrows; ++r) {
            const int dy = y0 + r - F.pad_y;
            t.inside[r] = dy >= 0 && dy < F.new_h;
            t.s0[r] = t.s1[r] = t.c0[r] = t.c1[r] = -1;
            if (!t.inside[r]) continue;
            if (nearest) {
                const int yi = ref_nearest(dy, F.src_h, F.new_h);
                t.s0[r] = find_or_add(t, yi, 0);
                t.c0[r] = find_or_add(t, yi >> 1, 1);
            } else {
                Tap ty = interp_tap(F.rh, dy, F.src_h);
                t.ty[r] = ty;
                t.s0[r] = find_or_add(t, ty.i0, 0);
                t.c0[r] = find_or_add(t, ty.i0 >> 1, 1);
                if (ty.l1 != 0.f) {
                    t.s1[r] = find_or_add(t, ty.i1, 0);
                    t.c1[r] = find_or_add(t, ty.i1 >> 1, 1);
                }
            }
        }
    }
    __syncthreads();

    const int luma_bytes = F.src_w;
    const int chroma_bytes = ((F.src_w + 1) >> 1) << 1;
    for (int s = 0; s < t.nslots; ++s) {
        const uint8_t* g = t.slot_uv[s] ? F.src + F.uv_offset + (int64_t)t.slot_row[s] * F.pitch
                                        : F.src + (int64_t)t.slot_row[s] * F.pitch;
        if (s < p.max_slots) {
            const uint8_t* base = stage_bytes(smem + s * p.slot_bytes, g,
                                              t.slot_uv[s] ? chroma_bytes : luma_bytes,
                                              threadIdx.x, kThreads);
            if (threadIdx.x == 0) slot_ptr[s] = base;
        } else if (threadIdx.x == 0) {
            slot_ptr[s] = g;
        }
    }
    __syncthreads();

    const YuvMatrix m = yuv_matrix(p.matrix);
    OutT* out = static_cast<OutT*>(p.out);
    const int64_t plane = (int64_t)p.dst_h * p.dst_w;
    OutT* img_out = out + (int64_t)img * 3 * plane;
    const int groups = (p.dst_w + VEC - 1) / VEC;
    const int items = nrows * groups;
    const int c_src0 = p.swap_rb ? 2 : 0, c_src2 = p.swap_rb ? 0 : 2;

    for (int it = threadIdx.x; it < items; it += kThreads) {
        const int r = it / groups;
        const int g = it - r * groups;
        const int y = y0 + r;
        const int x0 = g * VEC;
        float v0[VEC], v1[VEC], v2[VEC];
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
            const int dx = x0 + k - F.pad_x;
            if (!t.inside[r] || dx < 0 || dx >= F.new_w) {
                v0[k] = p.pad_out[0];
                v1[k] = p.pad_out[1];
                v2[k] = p.pad_out[2];
                continue;
            }
            float px[3];
            if (nearest) {
                const int xi = ref_nearest(dx, F.src_w, F.new_w);
                yuv_to_bgr(m, slot_ptr[t.s0[r]], slot_ptr[t.c0[r]], xi, px);
            } else {
                const Tap ty = t.ty[r];
                const Tap tx = interp_tap(F.rw, dx, F.src_w);
                const bool right = tx.l1 != 0.f;
                const bool below = t.s1[r] >= 0;
                float q00[3], q01[3] = {0.f, 0.f, 0.f}, q10[3] = {0.f, 0.f, 0.f},
                               q11[3] = {0.f, 0.f, 0.f};
                const uint8_t* y0p = slot_ptr[t.s0[r]];
                const uint8_t* u0p = slot_ptr[t.c0[r]];
                yuv_to_bgr(m, y0p, u0p, tx.i0, q00);
                if (right) yuv_to_bgr(m, y0p, u0p, tx.i1, q01);
                if (below) {
                    const uint8_t* y1p = slot_ptr[t.s1[r]];
                    const uint8_t* u1p = slot_ptr[t.c1[r]];
                    yuv_to_bgr(m, y1p, u1p, tx.i0, q10);
                    if (right) yuv_to_bgr(m, y1p, u1p, tx.i1, q11);
                }
#pragma unroll
                for (int c = 0; c < 3; ++c) px[c] = interp_blend(ty, tx, q00[c], q01[c], q10[c], q11[c]);
            }
            v0[k] = normalise(px[c_src0], p.mean[0], p.stdv[0]);
            v1[k] = normalise(px[1], p.mean[1], p.stdv[1]);
            v2[k] = normalise(px[c_src2], p.mean[2], p.stdv[2]);
        }
        OutT* o = img_out + (int64_t)y * p.dst_w + x0;
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

// ---- host-side planning --------------------------------------------------------------------

int max_slots_for(const LbFrame& f, int dst_h, int rows, bool nv12, bool nearest) {
    // Distinct staged rows in the busiest tile, computed with the kernel's own tap math.
    int worst = 0;
    for (int y0 = 0; y0 < dst_h; y0 += rows) {
        int list[kMaxSlots * 2];
        int n = 0;
        auto add = [&](int key) {
            for (int i = 0; i < n; ++i)
                if (list[i] == key) return;
            list[n++] = key;
        };
        for (int r = 0; r < rows && y0 + r < dst_h; ++r) {
            const int dy = y0 + r - f.pad_y;
            if (dy < 0 || dy >= f.new_h) continue;
            if (nv12 && nearest) {
                float a = (float)dy + 0.5f;
                volatile float b = a * (float)f.src_h;
                volatile float c = b / (float)f.new_h;
                float rr = std::max(0.f, c - 0.5f);
                int yi = std::min((int)rr, f.src_h - 1);
                add(2 * yi);
                add(2 * (yi >> 1) + 1);
                continue;
            }
            Tap ty = interp_tap(f.rh, dy, f.src_h);
            add(2 * ty.i0);
            if (nv12) add(2 * (ty.i0 >> 1) + 1);
            if (ty.l1 != 0.f) {
                add(2 * ty.i1);
                if (nv12) add(2 * (ty.i1 >> 1) + 1);
            }
        }
        worst = std::max(worst, n);
    }
    return worst;
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

namespace {

struct Plan {
    LbParams p;
    int smem;
    int grid;
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
    }
    p.slot_bytes = ((max_row_bytes + 16 + 15) / 16) * 16;
    // Largest row tile whose staging fits the shared-memory budget.
    for (int rows = kMaxRows; rows >= 1; rows >>= 1) {
        int slots = 0;
        for (int i = 0; i < n; ++i)
            slots = std::max(slots, max_slots_for(p.f[i], dst_h, rows, nv12, sampling == 0));
        const int smem = std::max(slots, 1) * p.slot_bytes;
        if (smem <= kSmemBudget) {
            p.rows = rows;
            p.tiles = (dst_h + rows - 1) / rows;
            p.max_slots = std::max(slots, 1);
            plan->smem = smem;
            plan->grid = n * p.tiles;
            return nullptr;
        }
    }
    return "source rows are too wide to stage in shared memory";
}

template <typename OutT, int VEC, bool NV12>
cudaError_t launch_one(const Plan& plan, cudaStream_t stream) {
    auto kernel = NV12 ? letterbox_nv12_kernel<OutT, VEC> : letterbox_u8_kernel<OutT, VEC>;
    cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kernel), kSmemBudget);
    if (e != cudaSuccess) return e;
    kernel<<<plan.grid, kThreads, plan.smem, stream>>>(plan.p);
    return cudaGetLastError();
}

template <bool NV12>
cudaError_t launch_plan(const Plan& plan, int out_dtype, cudaStream_t stream) {
    const bool vec_f32 = plan.p.dst_w % 4 == 0 && (reinterpret_cast<uintptr_t>(plan.p.out) & 15) == 0;
    const bool vec_f16 = plan.p.dst_w % 8 == 0 && (reinterpret_cast<uintptr_t>(plan.p.out) & 15) == 0;
    if (out_dtype == SHIPK_DTYPE_F32)
        return vec_f32 ? launch_one<float, 4, NV12>(plan, stream) : launch_one<float, 1, NV12>(plan, stream);
    return vec_f16 ? launch_one<__half, 8, NV12>(plan, stream) : launch_one<__half, 1, NV12>(plan, stream);
}

}  // namespace

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
