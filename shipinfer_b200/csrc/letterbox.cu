// Fused letterbox: bilinear resize (half-pixel centres) + pad + BGR->RGB + normalise +
// NHWC->NCHW in one pass, for a whole batch of frames in one launch. BGR uint8 frames, and
// NV12 surfaces (BT.601 / BT.709 limited range, nearest or bilinear).
//
// Reference formulation: TorchImageOps._letterbox, src/shipinfer/runtime/ops/torch_ops.py:
// 349-403 (F.interpolate bilinear, align_corners=False, then paste, flip, sub, div); for NV12
// the reference's nv12_letterbox_kernel, csrc/shipinfer/runtime/ops.cu:148-194.
//
// Layout: a persistent grid of large CTAs (about one per SM). The batch's output rows
// (frame-major) are cut into chunks of `rp` rows; CTA b takes chunks b, b + grid, b + 2 grid, ...
// (so pad rows and image rows spread evenly over the SMs), one chunk per step, one thread per
// 16-byte group of output pixels, and keeps the source rows of the next
// kStages-1 steps in flight in a shared-memory ring filled by 16-byte cp.async copies (one warp
// per source row), so that HBM reads for later rows overlap the stores of the current ones.
// Only source rows with a non-zero vertical weight are fetched (one row in three at 1080p ->
// 640); pad rows fetch nothing. Per step, `rp` threads derive the vertical taps of the step's
// rows once; the horizontal taps of every output column, and a flag per pixel group saying
// whether all its taps are exact, are tabulated once per CTA for each distinct frame geometry
// of the batch. HBM traffic is the compulsory bytes: the output and the contributing rows.
//
// Exact taps. Where both tap weights of a pixel are exactly 1 and 0 (every pixel at 1080p ->
// 640: the ratio is exactly 3), the bilinear value IS the integer source pixel, so its
// normalised value comes from a 3 x 256 table of (k - mean[c]) / std[c], computed on the host
// with the same two IEEE-754 single-precision operations as normalise() — the same function of
// the same integer, hence the same bits — instead of a divide per element.
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

constexpr int kMaxThreads = 1024;
constexpr int kStages = 3;             // ring depth: steps in flight
constexpr int kMaxRp = 16;             // rows per step (upper bound)
constexpr int kMaxTables = 4;          // distinct frame geometries tabulated per launch
constexpr int kSmemMax = 220 * 1024;   // dynamic shared memory ceiling
constexpr int kTableMax = 4096;        // widest canvas whose column taps are tabulated

struct LbFrame {
    const uint8_t* src;      // BGR rows, or NV12 luma
    const int32_t* row_map;  // staged row of each source row, or null (identity)
    int64_t pitch;
    int64_t uv_offset;       // NV12 only
    int src_h, src_w;
    int new_h, new_w, pad_y, pad_x;
    float rh, rw;            // (float)src / (float)new, as torch computes its ratio
    int table;               // column table of this frame's geometry, -1: taps per pixel
};

struct LbParams {
    void* out;
    int n, dst_h, dst_w;
    int total_rows;          // n * dst_h
    int rp;                  // rows per step: CTA b takes the chunks of rp rows b, b + grid, ...
    int gthreads;            // threads per row: one pixel group each
    int spr;                 // source rows per output row in a ring slot (1, 2 or 4)
    int slot_bytes;          // bytes per source row in shared memory (multiple of 16)
    int stage_bytes;         // rp * spr * slot_bytes
    int ntables;             // column tables (distinct geometries), 0: taps per pixel
    int table_off;           // byte offset of the tables in dynamic shared memory
    int tstride;             // entries per column array (dst_w rounded up to 8)
    int table_bytes;         // bytes per table
    int table_frame[kMaxTables];  // a frame of each geometry, to build its table from
    float mean[3], stdv[3], pad_out[3];
    int swap_rb;
    int matrix, sampling;    // NV12 only
    float lut[3][256];       // (k - mean[c]) / std[c] for integer pixels (BGR only)
    LbFrame f[kMaxBatch];
};

struct RowInfo {
    Tap ty;
    int inside;
    int img;
    int y;
    int off[4];  // shared offset of each staged row (slot base + 16-byte misalignment), -1: none
};

// ---- shared helpers ------------------------------------------------------------------------

__device__ __forceinline__ void cp_async16(uint32_t smem_dst, const void* gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_dst), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// Stage src[0, nbytes) into shared memory at byte `base` (which already carries src's
// 16-byte misalignment, so shared and global agree modulo 16): the aligned middle moves by
// 16-byte cp.async, the ragged head and tail by byte loads. Every global access stays inside
// [src, src + nbytes). `lane`/`nlanes` split the work.
__device__ __forceinline__ void stage_row(uint8_t* smem, int base, const uint8_t* src, int nbytes, int lane,
                                          int nlanes) {
    const int mis = static_cast<int>(reinterpret_cast<uintptr_t>(src) & 15);
    const int head = mis == 0 ? 0 : min(16 - mis, nbytes);
    const int body_vecs = (nbytes - head) >> 4;
    const int tail_start = head + (body_vecs << 4);
    const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(smem)) + base + head;
    for (int v = lane; v < body_vecs; v += nlanes) cp_async16(sbase + 16 * v, src + head + 16 * v);
    const int edge = head + (nbytes - tail_start);
    for (int e = lane; e < edge; e += nlanes) {
        const int k = e < head ? e : tail_start + (e - head);
        smem[base + k] = __ldg(src + k);
    }
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

// VEC consecutive entries of a shared int or float array starting at x0 (16-byte loads when
// VEC is a multiple of 4).
template <int VEC>
__device__ __forceinline__ void load_vec(const int* a, int x0, int (&v)[VEC]) {
    if constexpr (VEC % 4 == 0) {
#pragma unroll
        for (int q = 0; q < VEC; q += 4) {
            const int4 u = *reinterpret_cast<const int4*>(a + x0 + q);
            v[q] = u.x;
            v[q + 1] = u.y;
            v[q + 2] = u.z;
            v[q + 3] = u.w;
        }
    } else {
#pragma unroll
        for (int q = 0; q < VEC; ++q) v[q] = a[x0 + q];
    }
}
template <int VEC>
__device__ __forceinline__ void load_vec(const float* a, int x0, float (&v)[VEC]) {
    if constexpr (VEC % 4 == 0) {
#pragma unroll
        for (int q = 0; q < VEC; q += 4) {
            const float4 u = *reinterpret_cast<const float4*>(a + x0 + q);
            v[q] = u.x;
            v[q + 1] = u.y;
            v[q + 2] = u.z;
            v[q + 3] = u.w;
        }
    } else {
#pragma unroll
        for (int q = 0; q < VEC; ++q) v[q] = a[x0 + q];
    }
}

// A uint8 as float without the conversion pipe: 2^23 + b has the exact integer b in its low
// mantissa bits, and subtracting 2^23 leaves exactly b.
__device__ __forceinline__ float u8f(uint32_t b) {
    return __fsub_rn(__uint_as_float(0x4b000000u | b), 8388608.0f);
}

// ---- taps ------------------------------------------------------------------------------------

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

// The horizontal taps of output column x: (first, second) source column times `scale` (3 for
// BGR bytes, 1 for NV12 luma) and the second's weight; a0 = -1 for a pad column. Nearest (the
// reference NV12 kernel): the truncated reference coordinate, weight 0.
__device__ __forceinline__ void column_tap(const LbFrame& F, int x, int scale, bool nearest,
                                           int& a0, int& a1, float& l1) {
    const int dx = x - F.pad_x;
    if (dx < 0 || dx >= F.new_w) {
        a0 = a1 = -1;
        l1 = 0.f;
        return;
    }
    if (nearest) {
        a0 = a1 = ref_nearest(dx, F.src_w, F.new_w) * scale;
        l1 = 0.f;
        return;
    }
    const Tap t = interp_tap(F.rw, dx, F.src_w);
    a0 = t.i0 * scale;
    a1 = t.i1 * scale;
    l1 = t.l1;
}

// Shared pointers of one column table: a0/a1/l1 per column, an exactness flag per group.
struct Table {
    int* a0;
    int* a1;
    float* l1;
    int* gflag;
};

__device__ __forceinline__ Table table_at(uint8_t* smem, const LbParams& p, int t) {
    Table T;
    T.a0 = reinterpret_cast<int*>(smem + p.table_off + t * p.table_bytes);
    T.a1 = T.a0 + p.tstride;
    T.l1 = reinterpret_cast<float*>(T.a1 + p.tstride);
    T.gflag = reinterpret_cast<int*>(T.l1 + p.tstride);
    return T;
}

template <int VEC>
__device__ __forceinline__ void build_table(const LbFrame& F, int dst_w, int scale, bool nearest,
                                            const Table& T, int tid, int nt) {
    const int groups = (dst_w + VEC - 1) / VEC;
    for (int g = tid; g < groups; g += nt) {
        int exact = 1;
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
            const int x = g * VEC + k;
            if (x < dst_w) {
                int a0, a1;
                float l1;
                column_tap(F, x, scale, nearest, a0, a1, l1);
                T.a0[x] = a0;
                T.a1[x] = a1;
                T.l1[x] = l1;
                exact &= (a0 >= 0) & (l1 == 0.f);
            }
        }
        T.gflag[g] = exact;
    }
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
    bgr[0] = fminf(255.f, fmaxf(0.f, b));
    bgr[1] = fminf(255.f, fmaxf(0.f, g));
    bgr[2] = fminf(255.f, fmaxf(0.f, r));
}

// ---- the kernel ----------------------------------------------------------------------------

template <typename OutT, int VEC, bool NV12>
__global__ void __launch_bounds__(kMaxThreads)
letterbox_kernel(const __grid_constant__ LbParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ float lut[NV12 ? 1 : 3][256];
    __shared__ RowInfo rinfo[kStages][kMaxRp];

    const int tid = threadIdx.x, nt = blockDim.x;
    const int warp = tid >> 5, lane = tid & 31, nwarps = nt >> 5;
    const int nchunks = (p.total_rows + p.rp - 1) / p.rp;
    const int nsteps = (nchunks - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
    if (nsteps <= 0) return;

    if constexpr (!NV12) {
        for (int k = tid; k < 3 * 256; k += nt) lut[k >> 8][k & 255] = p.lut[k >> 8][k & 255];
    }
    const bool nearest = NV12 && p.sampling == 0;
    const bool second = NV12 ? p.spr == 4 : p.spr == 2;
    const int half = NV12 ? p.spr >> 1 : 0;  // first chroma row of a slot
    for (int t = 0; t < p.ntables; ++t)
        build_table<VEC>(p.f[p.table_frame[t]], p.dst_w, NV12 ? 1 : 3, nearest, table_at(smem, p, t), tid, nt);

    // Derive the rows of step s (threads < rp, one row each) and issue their copies.
    auto prepare = [&](int s) {
        const int st = s % kStages;
        if (tid < p.rp) {
            RowInfo& ri = rinfo[st][tid];
            const int q = ((int)blockIdx.x + s * (int)gridDim.x) * p.rp + tid;
            ri.inside = 0;
            ri.img = -1;
            ri.off[0] = ri.off[1] = ri.off[2] = ri.off[3] = -1;
            if (q < p.total_rows) {
                const int img = q / p.dst_h;
                const int y = q - img * p.dst_h;
                const LbFrame& F = p.f[img];
                ri.img = img;
                ri.y = y;
                const int dy = y - F.pad_y;
                if (dy >= 0 && dy < F.new_h) {
                    ri.inside = 1;
                    int r0, r1 = -1;
                    if (nearest) {
                        r0 = ref_nearest(dy, F.src_h, F.new_h);
                        ri.ty = Tap{0, 0, 1.f, 0.f};
                    } else {
                        const Tap ty = interp_tap(F.rh, dy, F.src_h);
                        ri.ty = ty;
                        r0 = ty.i0;
                        if (ty.l1 != 0.f && second) r1 = ty.i1;  // the planner saw the same taps
                    }
                    const int slot = st * p.stage_bytes + tid * p.spr * p.slot_bytes;
                    auto offset = [&](int k, const uint8_t* g) {
                        return slot + k * p.slot_bytes + (int)(reinterpret_cast<uintptr_t>(g) & 15);
                    };
                    if constexpr (NV12) {
                        ri.off[0] = offset(0, F.src + (int64_t)r0 * F.pitch);
                        ri.off[half] = offset(half, F.src + F.uv_offset + (int64_t)(r0 >> 1) * F.pitch);
                        if (r1 >= 0) {
                            ri.off[1] = offset(1, F.src + (int64_t)r1 * F.pitch);
                            ri.off[3] = offset(3, F.src + F.uv_offset + (int64_t)(r1 >> 1) * F.pitch);
                        }
                    } else {
                        const int m0 = F.row_map ? __ldg(F.row_map + r0) : r0;
                        ri.off[0] = offset(0, F.src + (int64_t)m0 * F.pitch);
                        if (r1 >= 0) {
                            const int m1 = F.row_map ? __ldg(F.row_map + r1) : r1;
                            ri.off[1] = offset(1, F.src + (int64_t)m1 * F.pitch);
                        }
                    }
                    // remember the source rows for the copy below
                    ri.ty.i0 = r0;
                    ri.ty.i1 = r1;
                }
            }
        }
        __syncthreads();  // rinfo of step s is visible
        // one warp per staged source row
        for (int job = warp; job < p.rp * p.spr; job += nwarps) {
            const int r = job / p.spr, k = job - r * p.spr;
            const RowInfo& ri = rinfo[st][r];
            const int off = ri.off[k];
            if (off < 0) continue;
            const LbFrame& F = p.f[ri.img];
            const uint8_t* g;
            int bytes;
            if constexpr (NV12) {
                const bool chroma = k >= half;
                const int sr = (k == 0 || k == half) ? ri.ty.i0 : ri.ty.i1;
                g = chroma ? F.src + F.uv_offset + (int64_t)(sr >> 1) * F.pitch : F.src + (int64_t)sr * F.pitch;
                bytes = chroma ? ((F.src_w + 1) >> 1) << 1 : F.src_w;
            } else {
                const int sr = k == 0 ? ri.ty.i0 : ri.ty.i1;
                const int row = F.row_map ? __ldg(F.row_map + sr) : sr;
                g = F.src + (int64_t)row * F.pitch;
                bytes = F.src_w * 3;
            }
            stage_row(smem, off, g, bytes, lane, 32);
        }
    };

    const int64_t plane = (int64_t)p.dst_h * p.dst_w;
    const int groups = (p.dst_w + VEC - 1) / VEC;
    const int cs0 = p.swap_rb ? 2 : 0, cs2 = p.swap_rb ? 0 : 2;
    const int rsub = tid / p.gthreads, gi = tid - rsub * p.gthreads;
    const YuvMatrix m = yuv_matrix(p.matrix);

#pragma unroll
    for (int s = 0; s < kStages - 1; ++s) {
        if (s < nsteps) prepare(s);
        cp_async_commit();
    }
    for (int s = 0; s < nsteps; ++s) {
        if (s + kStages - 1 < nsteps) prepare(s + kStages - 1);
        cp_async_commit();
        cp_async_wait<kStages - 1>();  // this thread's copies for step s have landed
        __syncthreads();                // everyone's have (and the tables, the first time)

        const RowInfo& ri = rinfo[s % kStages][rsub < p.rp ? rsub : 0];
        if (rsub < p.rp && ri.img >= 0) {
            const LbFrame& F = p.f[ri.img];
            OutT* orow = static_cast<OutT*>(p.out) + (int64_t)ri.img * 3 * plane + (int64_t)ri.y * p.dst_w;
            if (!ri.inside) {
                float v0[VEC], v1[VEC], v2[VEC];
#pragma unroll
                for (int k = 0; k < VEC; ++k) {
                    v0[k] = p.pad_out[0];
                    v1[k] = p.pad_out[1];
                    v2[k] = p.pad_out[2];
                }
                for (int g = gi; g < groups; g += p.gthreads) store3<OutT, VEC>(orow + g * VEC, plane, v0, v1, v2);
            } else {
                const Tap ty = Tap{0, 0, ri.ty.l0, ri.ty.l1};
                const bool use_table = F.table >= 0;
                const Table T = table_at(smem, p, use_table ? F.table : 0);
                if constexpr (!NV12) {
                    const uint8_t* s0 = smem + ri.off[0];
                    const bool below = ri.off[1] >= 0;
                    const uint8_t* s1 = smem + (below ? ri.off[1] : ri.off[0]);
                    for (int g = gi; g < groups; g += p.gthreads) {
                        const int x0 = g * VEC;
                        float v0[VEC], v1[VEC], v2[VEC];
                        if (use_table && !below && T.gflag[g]) {
                            // every tap of the group is exact: the value is the integer pixel itself
                            int a0[VEC];
                            load_vec<VEC>(T.a0, x0, a0);
#pragma unroll
                            for (int k = 0; k < VEC; ++k) {
                                const uint8_t* qp = s0 + a0[k];
                                v0[k] = lut[0][qp[cs0]];
                                v1[k] = lut[1][qp[1]];
                                v2[k] = lut[2][qp[cs2]];
                            }
                        } else {
                            int a0[VEC], a1[VEC];
                            float l1[VEC];
                            if (use_table) {
                                load_vec<VEC>(T.a0, x0, a0);
                                load_vec<VEC>(T.a1, x0, a1);
                                load_vec<VEC>(T.l1, x0, l1);
                            } else {
#pragma unroll
                                for (int k = 0; k < VEC; ++k)
                                    column_tap(F, min(x0 + k, p.dst_w - 1), 3, false, a0[k], a1[k], l1[k]);
                            }
#pragma unroll
                            for (int k = 0; k < VEC; ++k) {
                                if (a0[k] < 0) {
                                    v0[k] = p.pad_out[0];
                                    v1[k] = p.pad_out[1];
                                    v2[k] = p.pad_out[2];
                                    continue;
                                }
                                Tap tx;
                                tx.l1 = l1[k];
                                tx.l0 = __fsub_rn(1.f, l1[k]);
                                const bool right = l1[k] != 0.f;
                                float px[3];
#pragma unroll
                                for (int c = 0; c < 3; ++c) {
                                    // a tap whose weight is exactly 0 contributes exactly 0: not read
                                    const float p00 = u8f(s0[a0[k] + c]);
                                    const float p01 = right ? u8f(s0[a1[k] + c]) : 0.f;
                                    const float p10 = below ? u8f(s1[a0[k] + c]) : 0.f;
                                    const float p11 = (below && right) ? u8f(s1[a1[k] + c]) : 0.f;
                                    px[c] = interp_blend(ty, tx, p00, p01, p10, p11);
                                }
                                v0[k] = normalise(p.swap_rb ? px[2] : px[0], p.mean[0], p.stdv[0]);
                                v1[k] = normalise(px[1], p.mean[1], p.stdv[1]);
                                v2[k] = normalise(p.swap_rb ? px[0] : px[2], p.mean[2], p.stdv[2]);
                            }
                        }
                        store3<OutT, VEC>(orow + x0, plane, v0, v1, v2);
                    }
                } else {
                    const uint8_t* y0p = smem + ri.off[0];
                    const uint8_t* u0p = smem + ri.off[half];
                    const bool below = half == 2 && ri.off[1] >= 0;
                    const uint8_t* y1p = below ? smem + ri.off[1] : y0p;
                    const uint8_t* u1p = below ? smem + ri.off[3] : u0p;
                    for (int g = gi; g < groups; g += p.gthreads) {
                        const int x0 = g * VEC;
                        float v0[VEC], v1[VEC], v2[VEC];
                        if (use_table && !below && T.gflag[g]) {
                            // one tap with weight 1 per pixel: the blend is the converted pixel itself
                            int a0[VEC];
                            load_vec<VEC>(T.a0, x0, a0);
#pragma unroll
                            for (int k = 0; k < VEC; ++k) {
                                float px[3];
                                yuv_to_bgr(m, y0p, u0p, a0[k], px);
                                v0[k] = normalise(p.swap_rb ? px[2] : px[0], p.mean[0], p.stdv[0]);
                                v1[k] = normalise(px[1], p.mean[1], p.stdv[1]);
                                v2[k] = normalise(p.swap_rb ? px[0] : px[2], p.mean[2], p.stdv[2]);
                            }
                        } else {
                            int a0[VEC], a1[VEC];
                            float l1[VEC];
                            if (use_table) {
                                load_vec<VEC>(T.a0, x0, a0);
                                load_vec<VEC>(T.a1, x0, a1);
                                load_vec<VEC>(T.l1, x0, l1);
                            } else {
#pragma unroll
                                for (int k = 0; k < VEC; ++k)
                                    column_tap(F, min(x0 + k, p.dst_w - 1), 1, nearest, a0[k], a1[k], l1[k]);
                            }
#pragma unroll
                            for (int k = 0; k < VEC; ++k) {
                                if (a0[k] < 0) {
                                    v0[k] = p.pad_out[0];
                                    v1[k] = p.pad_out[1];
                                    v2[k] = p.pad_out[2];
                                    continue;
                                }
                                float px[3];
                                if (nearest || (!below && l1[k] == 0.f)) {
                                    // one tap with weight 1: the blend returns the converted pixel itself
                                    yuv_to_bgr(m, y0p, u0p, a0[k], px);
                                } else {
                                    Tap tx;
                                    tx.l1 = l1[k];
                                    tx.l0 = __fsub_rn(1.f, l1[k]);
                                    const bool right = l1[k] != 0.f;
                                    float q00[3], q01[3] = {0.f, 0.f, 0.f}, q10[3] = {0.f, 0.f, 0.f},
                                                  q11[3] = {0.f, 0.f, 0.f};
                                    yuv_to_bgr(m, y0p, u0p, a0[k], q00);
                                    if (right) yuv_to_bgr(m, y0p, u0p, a1[k], q01);
                                    if (below) {
                                        yuv_to_bgr(m, y1p, u1p, a0[k], q10);
                                        if (right) yuv_to_bgr(m, y1p, u1p, a1[k], q11);
                                    }
#pragma unroll
                                    for (int c = 0; c < 3; ++c) px[c] = interp_blend(ty, tx, q00[c], q01[c], q10[c], q11[c]);
                                }
                                v0[k] = normalise(p.swap_rb ? px[2] : px[0], p.mean[0], p.stdv[0]);
                                v1[k] = normalise(px[1], p.mean[1], p.stdv[1]);
                                v2[k] = normalise(p.swap_rb ? px[0] : px[2], p.mean[2], p.stdv[2]);
                            }
                        }
                        store3<OutT, VEC>(orow + x0, plane, v0, v1, v2);
                    }
                }
            }
        }
        __syncthreads();  // stage s % kStages is free for the prefetch of step s + kStages
    }
    cp_async_wait<0>();
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
    int threads;
};

const char* plan_letterbox(const FrameView* frames, int n, void* out, int dst_h, int dst_w, int vec,
                           const float mean[3], const float stdv[3], int swap_rb,
                           float pad_value, bool nv12, int matrix, int sampling, Plan* plan) {
    LbParams& p = plan->p;
    std::memset(&p, 0, sizeof(p));
    p.out = out;
    p.n = n;
    p.dst_h = dst_h;
    p.dst_w = dst_w;
    p.total_rows = n * dst_h;
    p.swap_rb = swap_rb;
    p.matrix = matrix;
    p.sampling = sampling;
    for (int c = 0; c < 3; ++c) {
        p.mean[c] = mean[c];
        p.stdv[c] = stdv[c];
        p.pad_out[c] = (pad_value - mean[c]) / stdv[c];
        // two IEEE-754 single-precision operations, as normalise() performs them on the device
        for (int k = 0; k < 256; ++k) p.lut[c][k] = ((float)k - mean[c]) / stdv[c];
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
        f.table = -1;
        const int rb = nv12 ? (((f.src_w + 1) >> 1) << 1) : f.src_w * 3;
        max_row_bytes = std::max(max_row_bytes, rb);
        if (!(nv12 && sampling == 0)) second = second || needs_second_row(f);
    }
    // Column tables, one per distinct horizontal geometry (up to kMaxTables).
    if (dst_w <= kTableMax) {
        for (int i = 0; i < n; ++i) {
            LbFrame& f = p.f[i];
            for (int t = 0; t < p.ntables && f.table < 0; ++t) {
                const LbFrame& g = p.f[p.table_frame[t]];
                if (g.src_w == f.src_w && g.new_w == f.new_w && g.pad_x == f.pad_x) f.table = t;
            }
            if (f.table < 0 && p.ntables < kMaxTables) {
                p.table_frame[p.ntables] = i;
                f.table = p.ntables++;
            }
        }
    }
    // Rows per ring slot. BGR: i0 [, i1]. NV12: luma i0 [, luma i1], then chroma i0 [, i1]
    // (the first chroma row is at spr / 2).
    p.spr = nv12 ? (second && sampling != 0 ? 4 : 2) : (second ? 2 : 1);
    p.slot_bytes = ((max_row_bytes + 16 + 15) / 16) * 16;
    const int groups = (dst_w + vec - 1) / vec;
    p.gthreads = std::min(kMaxThreads, ((groups + 31) / 32) * 32);
    p.tstride = ((dst_w + 7) / 8) * 8;
    const int gstride = ((groups + 3) / 4) * 4;
    p.table_bytes = (3 * p.tstride + gstride) * 4;
    // Rows per step: as many as the threads and the shared budget allow. Column tables give way
    // first (their frames then derive taps per pixel) until at least 4 rows fit.
    const int per_row = kStages * p.spr * p.slot_bytes;
    auto fits = [&](int rows, int ntab) { return (int64_t)rows * per_row + (int64_t)ntab * p.table_bytes <= kSmemMax; };
    const int rp_cap = std::min({kMaxRp, kMaxThreads / p.gthreads, dst_h * n});
    const int rp_want = std::min(rp_cap, 4);
    while (p.ntables > 0 && !fits(rp_want, p.ntables)) {
        --p.ntables;
        for (int i = 0; i < n; ++i)
            if (p.f[i].table == p.ntables) p.f[i].table = -1;
    }
    int rp = rp_cap;
    while (rp > 1 && !fits(rp, p.ntables)) --rp;
    if (!fits(rp, p.ntables)) return "source rows are too wide to stage in shared memory";
    p.rp = rp;
    p.stage_bytes = rp * p.spr * p.slot_bytes;
    p.table_off = kStages * p.stage_bytes;
    plan->smem = p.table_off + p.ntables * p.table_bytes;
    plan->threads = rp * p.gthreads;
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

// Resident CTAs per SM for this kernel at this block size and dynamic shared memory size.
int occupancy(const void* kernel, int threads, int smem) {
    static std::mutex mu;
    static std::map<std::tuple<const void*, int, int, int>, int> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    auto key = std::make_tuple(kernel, threads, smem, dev);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    int blocks = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, threads, smem) != cudaSuccess || blocks < 1)
        blocks = 1;
    cache[key] = blocks;
    return blocks;
}

template <typename OutT, int VEC, bool NV12>
cudaError_t launch_one(Plan& plan, cudaStream_t stream) {
    auto kernel = letterbox_kernel<OutT, VEC, NV12>;
    const void* fn = reinterpret_cast<const void*>(kernel);
    cudaError_t e = ensure_smem_attr(fn, kSmemMax);
    if (e != cudaSuccess) return e;
    const int resident = occupancy(fn, plan.threads, plan.smem) * sm_count();
    const int chunks = (plan.p.total_rows + plan.p.rp - 1) / plan.p.rp;
    const int grid = std::max(1, std::min(chunks, resident));
    kernel<<<grid, plan.threads, plan.smem, stream>>>(plan.p);
    return cudaGetLastError();
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
        void* chunk_out = static_cast<uint8_t*>(out) + per_image * start;
        const bool aligned = (reinterpret_cast<uintptr_t>(chunk_out) & 15) == 0;
        const int vec = out_dtype == SHIPK_DTYPE_F32 ? (aligned && dst_w % 4 == 0 ? 4 : 1)
                                                     : (aligned && dst_w % 8 == 0 ? 8 : 1);
        Plan plan;
        const char* why = plan_letterbox(frames + start, count, chunk_out, dst_h, dst_w, vec, mean, stdv,
                                         swap_rb, pad_value, nv12, matrix, sampling, &plan);
        if (why) return Status{SHIPK_ERANGE, why};
        cudaError_t e;
        if (out_dtype == SHIPK_DTYPE_F32) {
            if (nv12) e = vec == 4 ? launch_one<float, 4, true>(plan, stream) : launch_one<float, 1, true>(plan, stream);
            else e = vec == 4 ? launch_one<float, 4, false>(plan, stream) : launch_one<float, 1, false>(plan, stream);
        } else {
            if (nv12) e = vec == 8 ? launch_one<__half, 8, true>(plan, stream) : launch_one<__half, 1, true>(plan, stream);
            else e = vec == 8 ? launch_one<__half, 8, false>(plan, stream) : launch_one<__half, 1, false>(plan, stream);
        }
        if (e != cudaSuccess) return Status{SHIPK_ECUDA, cudaGetErrorString(e)};
    }
    return Status{SHIPK_OK, nullptr};
}

}  // namespace shipk
