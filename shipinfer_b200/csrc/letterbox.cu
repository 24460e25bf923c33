// Fused letterbox: bilinear resize (half-pixel centres) + pad + BGR->RGB + normalise +
// NHWC->NCHW in one pass, for a whole batch of frames in one launch. BGR uint8 frames, and
// NV12 surfaces (BT.601 / BT.709 limited range, nearest or bilinear).
//
// Reference formulation: TorchImageOps._letterbox, src/shipinfer/runtime/ops/torch_ops.py:
// 349-403 (F.interpolate bilinear, align_corners=False, then paste, flip, sub, div); for NV12
// the reference's nv12_letterbox_kernel, csrc/shipinfer/runtime/ops.cu:148-194.
//
// Layout: a persistent grid, one CTA per SM, whose warps are independent row pipelines. The
// batch's output rows (frame-major) are dealt to the grid's warps round-robin (warp w takes rows
// w, w + W, w + 2W, ...), warps numbered across CTAs first, so pad rows and image rows spread
// evenly over the SMs. A warp writes a whole output
// row at a time, its lanes striding over groups of 4 or 8 output pixels, and owns a private
// ring of D shared-memory slots into which 16-byte cp.async copies bring the source rows of its
// next D image rows. For BGR frames it writes its image rows first and its pad rows (which read
// nothing) last: every warp's reads start at once, and the pad rows' stores fill the end of the
// launch, when no reads remain (NV12 frames keep row order, which measured faster there).
// Nothing is shared between warps after set-up, so no CTA-wide barrier sits on the data path:
// each warp waits only on its own copies. Only source rows with a non-zero vertical weight are
// fetched (one row in three at 1080p -> 640), so HBM traffic is the compulsory bytes: the
// output and the contributing rows. Each launch is a programmatic dependent of the previous
// kernel in its stream: its set-up, and an L2 prefetch of each warp's first source rows, run
// while that kernel drains, so the launch's first reads do not start from an idle DRAM.
//
// The horizontal taps of every output column, and a flag per pixel group saying whether all
// its taps are exact, are tabulated once per CTA for each distinct frame geometry of the batch.
//
// Exact taps. Where both tap weights of a pixel are exactly 1 and 0 (every pixel at 1080p ->
// 640: the ratio is exactly 3), the bilinear value IS the integer source pixel, so its
// normalised value comes from a 3 x 256 table of normalise(k) built by each CTA — the same
// function of the same integer, hence the same bits — instead of a divide per element.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <type_traits>

namespace shipk {

namespace {

constexpr int kMaxWarps = 16;          // warps per SM (up to 128 registers each)
constexpr int kMaxDepth = 3;           // ring slots per warp
constexpr int kMaxTables = 4;          // distinct frame geometries tabulated per launch
constexpr int kSmemMax = 220 * 1024;   // dynamic shared memory per SM

// The CTA shape: CTAS CTAs per SM of kMaxWarps / CTAS warps, each with a 1 / CTAS share of the
// shared-memory budget. BGR frames to float32 run as two 8-warp CTAs per SM: a CTA that finishes
// frees its share of the SM for the next launch's CTA sooner (config 1: 11.12 -> 11.03 us on one
// box, 10.79 -> 10.72 on another); NV12 and float16 output run as one 16-warp CTA, whose deeper
// rings and single copy of the column tables measured faster there (config 5: 94.3 against
// 97.3 us; config 4's letterbox 29.4 against 30.5 us).
template <int CTAS>
constexpr int cta_smem() { return CTAS == 1 ? kSmemMax : 100 * 1024; }
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
    int half_a0;             // byte offset of column 0's first tap when every column is a half-weight
                             // pair of adjacent pixels two pixels after the previous one, else -1
};

struct LbParams {
    void* out;
    int n, dst_h, dst_w;
    int total_rows;          // n * dst_h
    int depth;               // ring slots per warp (1..kMaxDepth)
    int spr;                 // source rows per slot (1, 2 or 4)
    int slot_bytes;          // bytes per source row in shared memory (multiple of 16)
    int warp_bytes;          // depth * spr * slot_bytes
    int ntables;             // column tables (distinct geometries), 0: taps per pixel
    int table_off;           // byte offset of the tables in dynamic shared memory
    int tstride;             // entries per column array (dst_w rounded up to 8)
    int table_bytes;         // bytes per table
    int table_frame[kMaxTables];  // a frame of each geometry, to build its table from
    float mean[3], stdv[3], pad_out[3];
    float rcp[3];            // RN(1 / std[c])
    Norm2 n2;                // the same constants in pairs, for the packed paths
    int arith;               // normalise by div_markstein (the host checked the constants' range)
    int mean_zero;           // some channel's mean is 0: tiny numerators are possible
    int exact_arith;         // div_markstein equals normalise() on every integer 0..255 (host-checked)
    int exact_one;           // ... and so does div_markstein_1 (one correction)
    int half_mode;           // half-weight rows: 1 div_markstein_1, 2 div_markstein, 0 none equals
                             // normalise() on every quarter-integer 0..255 (host-checked)
    int half_fold;           // every channel's 2^21 + mean is a float: one fma gives S/4 - mean
    float2 half_c[3];        // -(2^21 + mean) (half_fold) or -mean, twice
    int swap_rb;
    int matrix, sampling;    // NV12 only
    LbFrame f[kMaxBatch];
};

// ---- shared helpers ------------------------------------------------------------------------

__device__ __forceinline__ void cp_async16(uint32_t smem_dst, const void* gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_dst), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// Wait until at most `pending` of this thread's most recent copy groups are still in flight.
__device__ __forceinline__ void cp_async_wait_dyn(int pending) {
    if (pending <= 0) cp_async_wait<0>();
    else if (pending == 1) cp_async_wait<1>();
    else cp_async_wait<2>();  // pending <= kMaxDepth - 1
}

// Stage src[0, nbytes) into shared memory at byte `base` (which already carries src's
// 16-byte misalignment, so shared and global agree modulo 16): the aligned middle moves by
// 16-byte cp.async, the ragged head and tail by byte loads. Every global access stays inside
// [src, src + nbytes). The 32 lanes of the calling warp split the work.
__device__ __forceinline__ void stage_row(uint8_t* smem, int base, const uint8_t* src, int nbytes, int lane) {
    const int mis = static_cast<int>(reinterpret_cast<uintptr_t>(src) & 15);
    const int head = mis == 0 ? 0 : min(16 - mis, nbytes);
    const int body_vecs = (nbytes - head) >> 4;
    const int tail_start = head + (body_vecs << 4);
    const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(smem)) + base + head;
    const uint8_t* gbase = src + head;
    for (int v = lane; v < body_vecs; v += 32) cp_async16(sbase + 16 * v, gbase + 16 * v);
    const int edge = head + (nbytes - tail_start);
    for (int e = lane; e < edge; e += 32) {
        const int k = e < head ? e : tail_start + (e - head);
        smem[base + k] = __ldg(src + k);
    }
}

template <typename OutT, int VEC>
__device__ __forceinline__ void store3(OutT* o, int64_t plane, const float (&v0)[VEC],
                                       const float (&v1)[VEC], const float (&v2)[VEC], int rot = 0) {
    if constexpr (VEC == 8 && std::is_same_v<OutT, __half>) {
        OutVec<OutT>::store_swapped(o, v0, rot != 0);
        OutVec<OutT>::store_swapped(o + plane, v1, rot != 0);
        OutVec<OutT>::store_swapped(o + 2 * plane, v2, rot != 0);
    } else if constexpr (VEC > 1) {
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
// VEC is a multiple of 4). With rot = 4 (VEC 8), v holds entries 4..7 then 0..3.
template <int VEC, typename T>
__device__ __forceinline__ void load_vec(const T* a, int x0, T (&v)[VEC], int rot = 0) {
    if constexpr (VEC % 4 == 0) {
#pragma unroll
        for (int q = 0; q < VEC; q += 4) {
            const int4 u = *reinterpret_cast<const int4*>(a + x0 + (q ^ rot));
            v[q] = __builtin_bit_cast(T, u.x);
            v[q + 1] = __builtin_bit_cast(T, u.y);
            v[q + 2] = __builtin_bit_cast(T, u.z);
            v[q + 3] = __builtin_bit_cast(T, u.w);
        }
    } else {
#pragma unroll
        for (int q = 0; q < VEC; ++q) v[q] = a[x0 + q];
    }
}

// The 24 bytes of a 4-pixel half-weight group as six 32-bit words (three 8-byte loads; the group
// starts 8-byte aligned).
__device__ __forceinline__ void load_words(const uint8_t* q, uint32_t (&w)[6]) {
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        const uint2 u = reinterpret_cast<const uint2*>(q)[i];
        w[2 * i] = u.x;
        w[2 * i + 1] = u.y;
    }
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
    const int* a0;
    const int* a1;
    const float* l1;
    const int* gflag;
};

__device__ __forceinline__ Table table_at(const uint8_t* smem, const LbParams& p, int t) {
    Table T;
    T.a0 = reinterpret_cast<const int*>(smem + p.table_off + t * p.table_bytes);
    T.a1 = T.a0 + p.tstride;
    T.l1 = reinterpret_cast<const float*>(T.a1 + p.tstride);
    T.gflag = reinterpret_cast<const int*>(T.l1 + p.tstride);
    return T;
}

// Returns whether every group this thread tabulated is exact; lowers wmin to the smallest
// nonzero tap weight (l0 or l1) of its image columns.
template <int VEC>
__device__ __forceinline__ int build_table(const LbFrame& F, int dst_w, int scale, bool nearest,
                                           uint8_t* base, int tstride, int tid, int nt, float& wmin) {
    int* a0s = reinterpret_cast<int*>(base);
    int* a1s = a0s + tstride;
    float* l1s = reinterpret_cast<float*>(a1s + tstride);
    int* gflag = reinterpret_cast<int*>(l1s + tstride);
    const int groups = (dst_w + VEC - 1) / VEC;
    int mine = 1;
    for (int g = tid; g < groups; g += nt) {
        int exact = 1;
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
            const int x = g * VEC + k;
            if (x < dst_w) {
                int a0, a1;
                float l1;
                column_tap(F, x, scale, nearest, a0, a1, l1);
                a0s[x] = a0;
                a1s[x] = a1;
                l1s[x] = l1;
                exact &= (a0 >= 0) & (l1 == 0.f);
                if (a0 >= 0 && l1 != 0.f) wmin = fminf(wmin, fminf(l1, __fsub_rn(1.f, l1)));
            }
        }
        gflag[g] = exact;
        mine &= exact;
    }
    return mine;
}

// ---- one output row's geometry ---------------------------------------------------------------

struct RowGeo {
    int img, y;
    bool inside;   // an image row (reads source rows); otherwise a pad row
    float l0, l1;  // vertical weights
    int r0, r1;    // source rows of the two taps; r1 = -1 when the second is not read
};

// A warp's walk over output rows q, q + W, q + 2W, ... as (frame, row) without a division per
// step: W = wi * dst_h + wr.
struct RowCursor {
    int img, y;
    __device__ __forceinline__ void advance(int wi, int wr, int dst_h) {
        img += wi;
        y += wr;
        if (y >= dst_h) {
            y -= dst_h;
            ++img;
        }
    }
};

__device__ __forceinline__ RowGeo row_geo(const LbParams& p, const RowCursor& c, bool nearest, bool second) {
    RowGeo g;
    g.img = c.img;
    g.y = c.y;
    const LbFrame& F = p.f[g.img];
    const int dy = g.y - F.pad_y;
    g.inside = dy >= 0 && dy < F.new_h;
    g.l0 = 1.f;
    g.l1 = 0.f;
    g.r0 = 0;
    g.r1 = -1;
    if (g.inside) {
        if (nearest) {
            g.r0 = ref_nearest(dy, F.src_h, F.new_h);
        } else {
            const Tap ty = interp_tap(F.rh, dy, F.src_h);
            g.l0 = ty.l0;
            g.l1 = ty.l1;
            g.r0 = ty.i0;
            if (ty.l1 != 0.f && second) g.r1 = ty.i1;  // the planner saw the same taps
        }
    }
    return g;
}

// Source bytes of staged row k of an output row's slot. BGR: k = 0 tap r0, k = 1 tap r1.
// NV12 (chroma from slot `half` on): luma r0 [, luma r1], chroma of r0 [, chroma of r1].
template <bool NV12>
__device__ __forceinline__ const uint8_t* staged_src(const LbFrame& F, const RowGeo& g, int k, int half,
                                                     int& bytes) {
    if constexpr (NV12) {
        const bool chroma = k >= half;
        const int sr = (k == 0 || k == half) ? g.r0 : g.r1;
        bytes = chroma ? ((F.src_w + 1) >> 1) << 1 : F.src_w;
        return chroma ? F.src + F.uv_offset + (int64_t)(sr >> 1) * F.pitch : F.src + (int64_t)sr * F.pitch;
    } else {
        const int sr = k == 0 ? g.r0 : g.r1;
        const int row = F.row_map ? __ldg(F.row_map + sr) : sr;
        bytes = F.src_w * 3;
        return F.src + (int64_t)row * F.pitch;
    }
}

// The source rows of a warp's first `depth` image rows (walking its rows from `c`), into L2:
// each lane prefetches every 32nd 128-byte line of each staged row. Stops at the first frame
// with a row map (staged host frames).
template <bool NV12>
__device__ __forceinline__ void prefetch_rows(const LbParams& p, RowCursor c, int nrows, int wi, int wr,
                                              bool nearest, bool second, int half, int lane) {
    int got = 0;
    for (int j = 0; j < nrows && got < p.depth; ++j, c.advance(wi, wr, p.dst_h)) {
        const RowGeo g = row_geo(p, c, nearest, second);
        if (!g.inside) continue;
        const LbFrame& F = p.f[g.img];
        if (F.row_map) return;
#pragma unroll
        for (int k = 0; k < (NV12 ? 4 : 2); ++k) {
            if (k >= p.spr) break;
            const bool tap2 = NV12 ? (half == 2 && (k == 1 || k == 3)) : k == 1;
            if (tap2 && g.r1 < 0) continue;
            int bytes;
            const uint8_t* src = staged_src<NV12>(F, g, k, half, bytes);
            // every line of [src, src + bytes): the last prefetch lands on the row's last byte
            for (int off = lane * 128; off < bytes + 127; off += 32 * 128)
                asm volatile("prefetch.global.L2 [%0];" ::"l"(src + min(off, bytes - 1)));
        }
        ++got;
    }
}

// ---- the kernel ----------------------------------------------------------------------------

template <typename OutT, int VEC, bool NV12, int CTAS>
__global__ void __launch_bounds__(kMaxWarps / CTAS * 32, CTAS)
letterbox_kernel(const __grid_constant__ LbParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ float lut[NV12 ? 1 : 3][256];
    __shared__ int all_exact[kMaxTables];  // every group of the table is exact
    __shared__ int wmin_bits[kMaxTables];  // smallest nonzero column weight of the table (float bits)

    const int tid = threadIdx.x, nt = blockDim.x;
    const int warp = tid >> 5, lane = tid & 31, nwarps = nt >> 5;
    const bool nearest = NV12 && p.sampling == 0;
    const bool second = NV12 ? p.spr == 4 : p.spr == 2;
    const int half = NV12 ? p.spr >> 1 : 0;  // first chroma row of a slot

    // ---- set-up shared by the CTA's warps, from the parameters alone ----
    if constexpr (!NV12) {
        // The exact path's values are normalise() of integer pixels. div_markstein gives them
        // when the host found it equal to normalise() on all 768 (channel, value) inputs; else
        // a table of normalise(k) does: the same operations on the same inputs as the per-pixel
        // path, so the same bits. (Built here rather than read from the parameter block, whose
        // constant-bank loads serialise when a warp's lanes index different entries.)
        if (!p.exact_arith) {
            for (int k = tid; k < 3 * 256; k += nt) {
                const int c = k >> 8;
                lut[c][k & 255] = normalise((float)(k & 255), p.mean[c], p.stdv[c]);
            }
        }
    }
    if (tid < kMaxTables) wmin_bits[tid] = __float_as_int(1.f);
    __syncthreads();
    for (int t = 0; t < p.ntables; ++t) {
        float wmin = 1.f;
        const int mine = build_table<VEC>(p.f[p.table_frame[t]], p.dst_w, NV12 ? 1 : 3, nearest,
                                          smem + p.table_off + t * p.table_bytes, p.tstride, tid, nt, wmin);
        atomicMin(&wmin_bits[t], __float_as_int(wmin));  // positive floats order as their bits
        const int all = __syncthreads_and(mine);
        if (tid == 0) all_exact[t] = all;
    }
    __syncthreads();

    // ---- this warp's rows: gw, gw + W, gw + 2W, ... ----
    // Warp w of CTA b is number b + grid * w: a CTA's warps start 'grid' rows apart, so every
    // CTA samples the whole batch evenly and gets the same mix of pad and image rows.
    const int gw = blockIdx.x + gridDim.x * warp;
    const int W = gridDim.x * nwarps;
    const int nrows = gw < p.total_rows ? (p.total_rows - gw + W - 1) / W : 0;
    const int depth = p.depth;
    const int wi = W / p.dst_h, wr = W - wi * p.dst_h;
    RowCursor at_fetch{gw / p.dst_h, gw % p.dst_h};

    // Launched as a programmatic dependent of the stream's previous kernel: everything above
    // reads only the parameters and may overlap that kernel's tail. So may an L2 prefetch of the
    // source rows of this warp's first `depth` image rows: a prefetch changes no value any
    // thread observes (L2 is the point of coherence for global memory, and the copies below
    // read it only after the dependency has resolved), and it starts the launch's DRAM reads
    // while the previous kernel drains (config 1: 11.44 -> 9.90 us per step). Rows of staged
    // host frames are not prefetched: their row map is written by the copy this launch waits on.
    // Everything else in global memory (frames, row maps, the output) is touched only after the
    // previous kernel has completed and its writes are visible.
    prefetch_rows<NV12>(p, at_fetch, nrows, wi, wr, nearest, second, half, lane);
    griddep_wait();
    griddep_launch_dependents();
    if (nrows == 0) return;
    uint8_t* ring = smem + warp * p.warp_bytes;
    const int slot_stride = p.spr * p.slot_bytes;
    RowCursor at_row = at_fetch;

    int fetch_j = 0, fetched = 0, consumed = 0;
    // Keep the next `depth` image rows of this warp in flight (pad rows are skipped: they read
    // nothing). One copy group per image row, committed in row order.
    auto fetch_more = [&]() {
        while (fetch_j < nrows && fetched - consumed < depth) {
            const RowGeo g = row_geo(p, at_fetch, nearest, second);
            ++fetch_j;
            at_fetch.advance(wi, wr, p.dst_h);
            if (!g.inside) continue;
            const LbFrame& F = p.f[g.img];
            const int slot = (fetched % depth) * slot_stride;
#pragma unroll
            for (int k = 0; k < (NV12 ? 4 : 2); ++k) {
                if (k >= p.spr) break;
                // rows of the second vertical tap: BGR row 1; NV12 rows 1 and 3 of a 4-row slot
                const bool tap2 = NV12 ? (half == 2 && (k == 1 || k == 3)) : k == 1;
                if (tap2 && g.r1 < 0) continue;
                int bytes;
                const uint8_t* src = staged_src<NV12>(F, g, k, half, bytes);
                stage_row(ring, slot + k * p.slot_bytes + (int)(reinterpret_cast<uintptr_t>(src) & 15), src,
                          bytes, lane);
            }
            cp_async_commit();
            ++fetched;
        }
    };

    const int64_t plane = (int64_t)p.dst_h * p.dst_w;
    const int groups = (p.dst_w + VEC - 1) / VEC;
    const int cs0 = p.swap_rb ? 2 : 0, cs2 = p.swap_rb ? 0 : 2;
    const YuvMatrix m = yuv_matrix(p.matrix);
    const Yuv2 k2 = yuv2(m);

    // ---- packed forms (VEC even): two pixels per fp32 instruction, the same bits ----
    // Output channel values i (pixels 2i, 2i+1) from a BGR triple of pairs, channels gathered.
    auto put_pair = [&](float (&v0)[VEC], float (&v1)[VEC], float (&v2)[VEC], int i, const float2 (&px)[3]) {
        const float2 c0 = p.swap_rb ? px[2] : px[0], c2 = p.swap_rb ? px[0] : px[2];
        v0[2 * i] = c0.x;
        v0[2 * i + 1] = c0.y;
        v1[2 * i] = px[1].x;
        v1[2 * i + 1] = px[1].y;
        v2[2 * i] = c2.x;
        v2[2 * i + 1] = c2.y;
    };
    // normalise() of integer pixels (every tap exact) by div_markstein, or by div_markstein_1
    // with `one` (the host checked the form against normalise() on every integer 0..255).
    auto exact_pairs = [&](auto one, const uint8_t* s, const int (&a)[VEC], float (&v0)[VEC], float (&v1)[VEC],
                           float (&v2)[VEC]) {
        constexpr bool kOne = decltype(one)::value;
#pragma unroll
        for (int i = 0; i < VEC / 2; ++i) {
            const uint8_t* qa = s + a[2 * i];
            const uint8_t* qb = s + a[2 * i + 1];
            float2 px[3];
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                const int sc = c == 0 ? cs0 : (c == 2 ? cs2 : 1);
                const float2 x = __fadd2_rn(u8f2(qa[sc], qb[sc]), p.n2.nmean[c]);
                px[c] = kOne ? div_markstein2_1(x, p.n2.nstd[c], p.n2.rcp[c])
                             : div_markstein2(x, p.n2.nstd[c], p.n2.rcp[c]);
            }
            v0[2 * i] = px[0].x;
            v0[2 * i + 1] = px[0].y;
            v1[2 * i] = px[1].x;
            v1[2 * i + 1] = px[1].y;
            v2[2 * i] = px[2].x;
            v2[2 * i + 1] = px[2].y;
        }
    };
    // The BGR blend of a group, channels gathered. Every tap is read: a weight of exactly 0 times
    // a finite pixel adds +0, as the scalar form's unread 0 does. With no second row (its weight
    // is 0 and the first's 1) the blend is the top row's sum itself.
    auto blend_pairs = [&](const uint8_t* s0, const uint8_t* s1, bool below, const Tap& ty, const int (&a0)[VEC],
                           const int (&a1)[VEC], const float (&l1)[VEC], bool (&padc)[VEC], float (&v0)[VEC],
                           float (&v1)[VEC], float (&v2)[VEC]) {
        const float2 ly0 = splat2(ty.l0), ly1 = splat2(ty.l1);
#pragma unroll
        for (int i = 0; i < VEC / 2; ++i) {
            const int ka = 2 * i, kb = 2 * i + 1;
            padc[ka] = a0[ka] < 0;  // a pad column: its value is replaced by the caller
            padc[kb] = a0[kb] < 0;
            const int ia0 = padc[ka] ? 0 : a0[ka], ia1 = padc[ka] ? 0 : a1[ka];
            const int ib0 = padc[kb] ? 0 : a0[kb], ib1 = padc[kb] ? 0 : a1[kb];
            const float2 lx1 = make_float2(l1[ka], l1[kb]);
            const float2 lx0 = __fadd2_rn(splat2(1.f), make_float2(-l1[ka], -l1[kb]));
            float2 px[3];
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                const int sc = c == 0 ? cs0 : (c == 2 ? cs2 : 1);
                const float2 p00 = u8f2(s0[ia0 + sc], s0[ib0 + sc]);
                const float2 p01 = u8f2(s0[ia1 + sc], s0[ib1 + sc]);
                if (below) {
                    const float2 p10 = u8f2(s1[ia0 + sc], s1[ib0 + sc]);
                    const float2 p11 = u8f2(s1[ia1 + sc], s1[ib1 + sc]);
                    px[c] = interp_blend2(ly0, ly1, lx0, lx1, p00, p01, p10, p11);
                } else {
                    px[c] = __ffma2_rn(lx0, p00, __fmul2_rn(lx1, p01));
                }
            }
            v0[ka] = px[0].x;
            v0[kb] = px[0].y;
            v1[ka] = px[1].x;
            v1[kb] = px[1].y;
            v2[ka] = px[2].x;
            v2[kb] = px[2].y;
        }
    };
    // The NV12 blend of a group: nearest sampling converts one tap (weight 1); bilinear converts
    // every tap of a pair (weights of exactly 0 add +0: converted pixels are finite and >= 0),
    // the second row's only when it is read.
    auto nv12_pairs = [&](const uint8_t* y0p, const uint8_t* u0p, const uint8_t* y1p, const uint8_t* u1p,
                          bool below, const Tap& ty, const int (&a0)[VEC], const int (&a1)[VEC],
                          const float (&l1)[VEC], bool (&padc)[VEC], float (&v0)[VEC], float (&v1)[VEC],
                          float (&v2)[VEC]) {
        const float2 ly0 = splat2(ty.l0), ly1 = splat2(ty.l1);
#pragma unroll
        for (int i = 0; i < VEC / 2; ++i) {
            const int ka = 2 * i, kb = 2 * i + 1;
            padc[ka] = a0[ka] < 0;
            padc[kb] = a0[kb] < 0;
            const int ia0 = padc[ka] ? 0 : a0[ka], ia1 = padc[ka] ? 0 : a1[ka];
            const int ib0 = padc[kb] ? 0 : a0[kb], ib1 = padc[kb] ? 0 : a1[kb];
            float2 px[3];
            float2 q00[3];
            yuv_to_bgr2(k2, y0p, u0p, ia0, ib0, q00);
            if (nearest) {
#pragma unroll
                for (int c = 0; c < 3; ++c) px[c] = q00[c];
            } else {
                const float2 lx1 = make_float2(l1[ka], l1[kb]);
                const float2 lx0 = __fadd2_rn(splat2(1.f), make_float2(-l1[ka], -l1[kb]));
                float2 q01[3];
                yuv_to_bgr2(k2, y0p, u0p, ia1, ib1, q01);
                if (below) {
                    float2 q10[3], q11[3];
                    yuv_to_bgr2(k2, y1p, u1p, ia0, ib0, q10);
                    yuv_to_bgr2(k2, y1p, u1p, ia1, ib1, q11);
#pragma unroll
                    for (int c = 0; c < 3; ++c) px[c] = interp_blend2(ly0, ly1, lx0, lx1, q00[c], q01[c], q10[c], q11[c]);
                } else {
#pragma unroll
                    for (int c = 0; c < 3; ++c) px[c] = __ffma2_rn(lx0, q00[c], __fmul2_rn(lx1, q01[c]));
                }
            }
            put_pair(v0, v1, v2, i, px);
        }
    };

    // A pad row: the pad value in every channel.
    auto pad_row = [&](const RowGeo& g) {
        OutT* orow = static_cast<OutT*>(p.out) + (int64_t)g.img * 3 * plane + (int64_t)g.y * p.dst_w;
        float v0[VEC], v1[VEC], v2[VEC];
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
            v0[k] = p.pad_out[0];
            v1[k] = p.pad_out[1];
            v2[k] = p.pad_out[2];
        }
        for (int x = lane; x < groups; x += 32) store3<OutT, VEC>(orow + x * VEC, plane, v0, v1, v2);
    };

    // BGR: image rows first, pad rows after them (below); NV12: rows in order (measured: pad rows
    // last is 0.7% slower there, 1.7% faster for BGR).
    const RowCursor first_row = at_row;
    for (int j = 0; j < nrows; ++j, at_row.advance(wi, wr, p.dst_h)) {
        fetch_more();
        const RowGeo g = row_geo(p, at_row, nearest, second);
        if (!g.inside) {
            if constexpr (NV12) pad_row(g);
            continue;
        }
        OutT* orow = static_cast<OutT*>(p.out) + (int64_t)g.img * 3 * plane + (int64_t)g.y * p.dst_w;
        cp_async_wait_dyn(fetched - consumed - 1);  // this row's group has landed (own lanes)
        __syncwarp();                                // ... and every lane's
        const LbFrame& F = p.f[g.img];
        const uint8_t* slot = ring + (consumed % depth) * slot_stride;
        const bool below = g.r1 >= 0 && (!NV12 || half == 2);
        const bool use_table = F.table >= 0;
        const Table T = table_at(smem, p, use_table ? F.table : 0);
        Tap ty;
        ty.l0 = g.l0;
        ty.l1 = g.l1;
        // May a blended value of this row be a nonzero below 2^-60 (where normalise_group's
        // guard takes IEEE division)? Only with a zero mean (else x = v - mean is 0 or at least
        // 2^-44). A blend of values that are 0 or at least qmin (a byte; a clamped NV12
        // conversion is a multiple of 2^-26) with tap weights 0 or at least wx, wy is 0 or at
        // least qmin * wx * wy, less three roundings.
        bool guard = p.mean_zero != 0;
        if (guard && use_table) {
            const float qmin = NV12 ? 1.4901161193847656e-08f : 1.f;  // 2^-26
            const float wx = __int_as_float(wmin_bits[F.table]);
            const float wy = below ? fminf(g.l0, g.l1) : 1.f;
            guard = !(qmin * wx * wy >= 3.469446951953614e-18f);  // 2^-58
        }
        int bytes;
        if constexpr (!NV12) {
            const uint8_t* s0 = slot + (int)(reinterpret_cast<uintptr_t>(staged_src<false>(F, g, 0, 0, bytes)) & 15);
            const uint8_t* s1 = below
                ? slot + p.slot_bytes + (int)(reinterpret_cast<uintptr_t>(staged_src<false>(F, g, 1, 0, bytes)) & 15)
                : s0;
            // Half-weight rows: every column's taps are adjacent pixels with weights 1/2, two
            // pixels on from the previous column's (an exact 2:1 reduction across), and the row
            // blends two rows with weights 1/2 or reads one with weight 1. Every step of the blend
            // is then exact and its value is S / 4, S the integer sum of the four taps (a single
            // row counted twice). A group of 4 pixels reads 24 contiguous bytes per row, as
            // 32-bit words (8-byte loads, lanes 24 bytes apart: no bank conflicts); S comes from byte permutes into 16-bit lanes and byte dot products,
            // 2^23 + S is S's float with 2^23 added (its bits: 0x4b000000 + S), and one fma
            // scales it by 1/4 and subtracts the mean (and 2^21) with one rounding. The host
            // checked the division form against normalise() on every S of every channel.
            const bool half = VEC == 4 && p.half_mode != 0 && F.half_a0 >= 0 &&
                              (!below || (g.l0 == 0.5f && g.l1 == 0.5f)) &&
                              ((reinterpret_cast<uintptr_t>(s0 + F.half_a0) |
                                reinterpret_cast<uintptr_t>(s1 + F.half_a0)) & 7) == 0;
            if (half) {
                auto half_row = [&](auto one) {
                    if constexpr (VEC == 4) {
                        constexpr bool kOne = decltype(one)::value;
                        constexpr int kW = 6;  // words per row per group
                        const uint8_t* r0 = s0 + F.half_a0;
                        const uint8_t* r1 = s1 + F.half_a0;
                        for (int gi = lane; gi < groups; gi += 32) {
                            uint32_t w[kW], u[kW];
                            load_words(r0 + gi * 24, w);
                            load_words(r1 + gi * 24, u);
                            float v0[VEC], v1[VEC], v2[VEC];
#pragma unroll
                            for (int i = 0; i < VEC / 2; ++i) {
                                // output pixels A = 2i and B = 2i + 1 read the twelve bytes
                                // [B0 G0 R0 B1 | G1 R1 B2 G2 | R2 B3 G3 R3] of each row
                                const uint32_t a0 = w[3 * i], a1 = w[3 * i + 1], a2 = w[3 * i + 2];
                                const uint32_t b0 = u[3 * i], b1 = u[3 * i + 1], b2 = u[3 * i + 2];
                                // (A.G, A.R) and (B.B, B.G) in 16-bit lanes (each at most 1020)
                                const uint32_t gr = __byte_perm(a0, 0u, 0x4241) + __byte_perm(a1, 0u, 0x4140) +
                                                    __byte_perm(b0, 0u, 0x4241) + __byte_perm(b1, 0u, 0x4140);
                                const uint32_t bg = __byte_perm(a1, 0u, 0x4342) + __byte_perm(a2, 0u, 0x4241) +
                                                    __byte_perm(b1, 0u, 0x4342) + __byte_perm(b2, 0u, 0x4241);
                                // A.B = bytes 0 + 3 of word 0, B.R = bytes 0 + 3 of word 2
                                const uint32_t ab = __dp4a(a0, 0x01000001u, __dp4a(b0, 0x01000001u, 0x4b000000u));
                                const uint32_t br = __dp4a(a2, 0x01000001u, __dp4a(b2, 0x01000001u, 0x4b000000u));
                                const float2 sB = make_float2(__uint_as_float(ab),
                                                              __uint_as_float(__byte_perm(bg, 0x4b000000u, 0x7410)));
                                const float2 sG = make_float2(__uint_as_float(__byte_perm(gr, 0x4b000000u, 0x7410)),
                                                              __uint_as_float(__byte_perm(bg, 0x4b000000u, 0x7432)));
                                const float2 sR = make_float2(__uint_as_float(__byte_perm(gr, 0x4b000000u, 0x7432)),
                                                              __uint_as_float(br));
                                float2 px[3];
#pragma unroll
                                for (int c = 0; c < 3; ++c) {
                                    const float2 sv = c == 1 ? sG : ((c == 0) != (p.swap_rb != 0) ? sB : sR);
                                    // (2^23 + S) / 4 = 2^21 + S/4 exactly
                                    const float2 x = p.half_fold
                                        ? __ffma2_rn(sv, splat2(0.25f), p.half_c[c])
                                        : __ffma2_rn(__fadd2_rn(sv, splat2(-8388608.0f)), splat2(0.25f), p.half_c[c]);
                                    px[c] = kOne ? div_markstein2_1(x, p.n2.nstd[c], p.n2.rcp[c])
                                                 : div_markstein2(x, p.n2.nstd[c], p.n2.rcp[c]);
                                }
                                v0[2 * i] = px[0].x;
                                v0[2 * i + 1] = px[0].y;
                                v1[2 * i] = px[1].x;
                                v1[2 * i + 1] = px[1].y;
                                v2[2 * i] = px[2].x;
                                v2[2 * i + 1] = px[2].y;
                            }
                            store3<OutT, VEC>(orow + gi * VEC, plane, v0, v1, v2);
                        }
                    }
                };
                if (p.half_mode == 1) half_row(std::true_type{});
                else half_row(std::false_type{});
            } else if (use_table && !below && all_exact[F.table]) {
                // Every tap of the row is exact: each value is normalise() of the integer pixel,
                // by div_markstein (checked against normalise() on every integer above) or the
                // table. Two groups per lane per pass, so their shared-memory loads overlap.
                auto exact_row = [&](auto arith, auto one) {
                    constexpr bool kArith = decltype(arith)::value;
                    auto value = [&](const uint8_t* q, int cs, int c) {
                        if constexpr (kArith) return div_markstein(__fsub_rn(u8f(q[cs]), p.mean[c]), p.stdv[c], p.rcp[c]);
                        else return lut[c][q[cs]];
                    };
                    for (int gi = lane; gi < groups; gi += 64) {
                        const bool two = gi + 32 < groups;
                        const int gj = two ? gi + 32 : gi;
                        int a0[VEC], b0[VEC];
                        load_vec<VEC>(T.a0, gi * VEC, a0);
                        load_vec<VEC>(T.a0, gj * VEC, b0);
                        float v0[VEC], v1[VEC], v2[VEC], w0[VEC], w1[VEC], w2[VEC];
                        if constexpr (kArith && VEC % 2 == 0) {
                            exact_pairs(one, s0, a0, v0, v1, v2);
                            exact_pairs(one, s0, b0, w0, w1, w2);
                        } else {
#pragma unroll
                        for (int k = 0; k < VEC; ++k) {
                            const uint8_t* qp = s0 + a0[k];
                            const uint8_t* qq = s0 + b0[k];
                            v0[k] = value(qp, cs0, 0);
                            v1[k] = value(qp, 1, 1);
                            v2[k] = value(qp, cs2, 2);
                            w0[k] = value(qq, cs0, 0);
                            w1[k] = value(qq, 1, 1);
                            w2[k] = value(qq, cs2, 2);
                        }
                        }
                        store3<OutT, VEC>(orow + gi * VEC, plane, v0, v1, v2);
                        if (two) store3<OutT, VEC>(orow + gj * VEC, plane, w0, w1, w2);
                    }
                };
                if (p.exact_one) exact_row(std::true_type{}, std::true_type{});
                else if (p.exact_arith) exact_row(std::true_type{}, std::false_type{});
                else exact_row(std::false_type{}, std::false_type{});
            } else
            for (int gi = lane; gi < groups; gi += 32) {
                const int x0 = gi * VEC;
                float v0[VEC], v1[VEC], v2[VEC];
                if (use_table && !below && T.gflag[gi]) {
                    // every tap of the group is exact: the value is normalise() of the integer
                    // pixel, by div_markstein or the table as in the all-exact rows above
                    int a0[VEC];
                    load_vec<VEC>(T.a0, x0, a0);
                    if (p.exact_arith) {
                        if constexpr (VEC % 2 == 0) {
                            exact_pairs(std::false_type{}, s0, a0, v0, v1, v2);
                        } else {
#pragma unroll
                        for (int k = 0; k < VEC; ++k) {
                            const uint8_t* qp = s0 + a0[k];
                            v0[k] = div_markstein(__fsub_rn(u8f(qp[cs0]), p.mean[0]), p.stdv[0], p.rcp[0]);
                            v1[k] = div_markstein(__fsub_rn(u8f(qp[1]), p.mean[1]), p.stdv[1], p.rcp[1]);
                            v2[k] = div_markstein(__fsub_rn(u8f(qp[cs2]), p.mean[2]), p.stdv[2], p.rcp[2]);
                        }
                        }
                    } else {
#pragma unroll
                        for (int k = 0; k < VEC; ++k) {
                            const uint8_t* qp = s0 + a0[k];
                            v0[k] = lut[0][qp[cs0]];
                            v1[k] = lut[1][qp[1]];
                            v2[k] = lut[2][qp[cs2]];
                        }
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
                    bool padc[VEC];
                    if constexpr (VEC % 2 == 0) {
                        blend_pairs(s0, s1, below, ty, a0, a1, l1, padc, v0, v1, v2);
                        normalise_group2<VEC>(v0, v1, v2, padc, p.n2, p.stdv, p.arith, guard);
                    } else {
#pragma unroll
                    for (int k = 0; k < VEC; ++k) {
                        padc[k] = a0[k] < 0;  // a pad column: its value is replaced below
                        const int i0 = padc[k] ? 0 : a0[k], i1 = padc[k] ? 0 : a1[k];
                        Tap tx;
                        tx.l1 = l1[k];
                        tx.l0 = __fsub_rn(1.f, l1[k]);
                        const bool right = l1[k] != 0.f;
                        float px[3];
#pragma unroll
                        for (int c = 0; c < 3; ++c) {
                            // a tap whose weight is exactly 0 contributes exactly 0: not read
                            const float p00 = u8f(s0[i0 + c]);
                            const float p01 = right ? u8f(s0[i1 + c]) : 0.f;
                            const float p10 = below ? u8f(s1[i0 + c]) : 0.f;
                            const float p11 = (below && right) ? u8f(s1[i1 + c]) : 0.f;
                            px[c] = interp_blend(ty, tx, p00, p01, p10, p11);
                        }
                        v0[k] = p.swap_rb ? px[2] : px[0];
                        v1[k] = px[1];
                        v2[k] = p.swap_rb ? px[0] : px[2];
                    }
                    normalise_group<VEC>(v0, v1, v2, padc, p.mean, p.stdv, p.rcp, p.arith);
                    }
#pragma unroll
                    for (int k = 0; k < VEC; ++k) {
                        if (padc[k]) {
                            v0[k] = p.pad_out[0];
                            v1[k] = p.pad_out[1];
                            v2[k] = p.pad_out[2];
                        }
                    }
                }
                store3<OutT, VEC>(orow + x0, plane, v0, v1, v2);
            }
        } else {
            auto at = [&](int k) {
                return slot + k * p.slot_bytes +
                       (int)(reinterpret_cast<uintptr_t>(staged_src<true>(F, g, k, half, bytes)) & 15);
            };
            const uint8_t* y0p = at(0);
            const uint8_t* u0p = at(half);
            const uint8_t* y1p = below ? at(1) : y0p;
            const uint8_t* u1p = below ? at(3) : u0p;
            // Eight pixels a lane (fp16): the upper half-warp takes its group's pixels 4..7 first,
            // so that at each step the two half-warps read source bytes half a group apart, not a
            // whole multiple of 16 groups (whose byte offsets share a bank at 2:1, 3:1 and 6:1
            // ratios); the store puts the halves back.
            const int rot = VEC == 8 && lane >= 16 ? 4 : 0;
            for (int gi = lane; gi < groups; gi += 32) {
                const int x0 = gi * VEC;
                float v0[VEC], v1[VEC], v2[VEC];
                if (use_table && !below && T.gflag[gi]) {
                    // one tap with weight 1 per pixel: the blend is the converted pixel itself
                    int a0[VEC];
                    load_vec<VEC>(T.a0, x0, a0, rot);
                    bool none[VEC];
#pragma unroll
                    for (int k = 0; k < VEC; ++k) none[k] = false;
                    if constexpr (VEC % 2 == 0) {
#pragma unroll
                        for (int i = 0; i < VEC / 2; ++i) {
                            float2 px[3];
                            yuv_to_bgr2(k2, y0p, u0p, a0[2 * i], a0[2 * i + 1], px);
                            put_pair(v0, v1, v2, i, px);
                        }
                        normalise_group2<VEC>(v0, v1, v2, none, p.n2, p.stdv, p.arith, guard);
                    } else {
#pragma unroll
                    for (int k = 0; k < VEC; ++k) {
                        float px[3];
                        yuv_to_bgr(m, y0p, u0p, a0[k], px);
                        v0[k] = p.swap_rb ? px[2] : px[0];
                        v1[k] = px[1];
                        v2[k] = p.swap_rb ? px[0] : px[2];
                    }
                    normalise_group<VEC>(v0, v1, v2, none, p.mean, p.stdv, p.rcp, p.arith);
                    }
                } else {
                    int a0[VEC], a1[VEC];
                    float l1[VEC];
                    if (use_table) {
                        load_vec<VEC>(T.a0, x0, a0, rot);
                        load_vec<VEC>(T.a1, x0, a1, rot);
                        load_vec<VEC>(T.l1, x0, l1, rot);
                    } else {
#pragma unroll
                        for (int k = 0; k < VEC; ++k)
                            column_tap(F, min(x0 + (k ^ rot), p.dst_w - 1), 1, nearest, a0[k], a1[k], l1[k]);
                    }
                    bool padc[VEC];
                    if constexpr (VEC % 2 == 0) {
                        nv12_pairs(y0p, u0p, y1p, u1p, below, ty, a0, a1, l1, padc, v0, v1, v2);
                        normalise_group2<VEC>(v0, v1, v2, padc, p.n2, p.stdv, p.arith, guard);
                    } else {
#pragma unroll
                    for (int k = 0; k < VEC; ++k) {
                        padc[k] = a0[k] < 0;  // a pad column: its value is replaced below
                        const int i0 = padc[k] ? 0 : a0[k], i1 = padc[k] ? 0 : a1[k];
                        float px[3];
                        if (nearest || (!below && l1[k] == 0.f)) {
                            // one tap with weight 1: the blend returns the converted pixel itself
                            yuv_to_bgr(m, y0p, u0p, i0, px);
                        } else {
                            Tap tx;
                            tx.l1 = l1[k];
                            tx.l0 = __fsub_rn(1.f, l1[k]);
                            const bool right = l1[k] != 0.f;
                            float q00[3], q01[3] = {0.f, 0.f, 0.f}, q10[3] = {0.f, 0.f, 0.f},
                                          q11[3] = {0.f, 0.f, 0.f};
                            yuv_to_bgr(m, y0p, u0p, i0, q00);
                            if (right) yuv_to_bgr(m, y0p, u0p, i1, q01);
                            if (below) {
                                yuv_to_bgr(m, y1p, u1p, i0, q10);
                                if (right) yuv_to_bgr(m, y1p, u1p, i1, q11);
                            }
#pragma unroll
                            for (int c = 0; c < 3; ++c) px[c] = interp_blend(ty, tx, q00[c], q01[c], q10[c], q11[c]);
                        }
                        v0[k] = p.swap_rb ? px[2] : px[0];
                        v1[k] = px[1];
                        v2[k] = p.swap_rb ? px[0] : px[2];
                    }
                    normalise_group<VEC>(v0, v1, v2, padc, p.mean, p.stdv, p.rcp, p.arith);
                    }
#pragma unroll
                    for (int k = 0; k < VEC; ++k) {
                        if (padc[k]) {
                            v0[k] = p.pad_out[0];
                            v1[k] = p.pad_out[1];
                            v2[k] = p.pad_out[2];
                        }
                    }
                }
                store3<OutT, VEC>(orow + x0, plane, v0, v1, v2, rot);
            }
        }
        __syncwarp();  // every lane is done with the slot before a later fetch refills it
        ++consumed;
    }
    // BGR: then this warp's pad rows (11.05 -> 10.86 us for config 1 against writing them in row
    // order, between the image rows).
    if constexpr (!NV12) {
        RowCursor c = first_row;
        for (int j = 0; j < nrows; ++j, c.advance(wi, wr, p.dst_h)) {
            const RowGeo g = row_geo(p, c, nearest, second);
            if (!g.inside) pad_row(g);
        }
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
    int warps;
};

// Does div_markstein give normalise()'s bits for every integer pixel value of every channel?
// Host IEEE-754 single precision (-ffp-contract=off) and fmaf are the operations the device
// performs, so this is the device's answer.
bool markstein_exact_on_bytes(const float mean[3], const float stdv[3], const float rcp[3]) {
    for (int c = 0; c < 3; ++c) {
        for (int k = 0; k < 256; ++k) {
            const float x = (float)k - mean[c];
            const float ref = x / stdv[c];
            const float q0 = x * rcp[c];
            const float r0 = std::fmaf(-q0, stdv[c], x);
            const float q1 = std::fmaf(r0, rcp[c], q0);
            const float r1 = std::fmaf(-q1, stdv[c], x);
            const float q2 = std::fmaf(r1, rcp[c], q1);
            const float fast = x == 0.f ? q0 : q2;
            if (std::memcmp(&fast, &ref, sizeof(float)) != 0) return false;
        }
    }
    return true;
}

// Does a division form give normalise()'s bits, (v - mean) / std, for every v = k / den with
// k = 0..kmax and every channel? Form 1 is div_markstein_1 (one correction), form 2
// div_markstein's two corrections without its zero select (the packed form; no numerator here is
// -0). The host's IEEE single operations and fmaf are the device's, so this is the device's
// answer; constants that are not finite are left to the general path.
bool division_form_exact(int form, const float mean[3], const float stdv[3], const float rcp[3], int kmax,
                         float den) {
    for (int c = 0; c < 3; ++c) {
        if (!std::isfinite(mean[c]) || !std::isfinite(stdv[c]) || !std::isfinite(rcp[c])) return false;
        for (int k = 0; k <= kmax; ++k) {
            const float x = (float)k / den - mean[c];  // k / den is exact (den 1 or 4)
            const float ref = x / stdv[c];
            const float q0 = x * rcp[c];
            const float q1 = std::fmaf(std::fmaf(-q0, stdv[c], x), rcp[c], q0);
            const float got = form == 1 ? q1 : std::fmaf(std::fmaf(-q1, stdv[c], x), rcp[c], q1);
            if (std::memcmp(&got, &ref, sizeof(float)) != 0) return false;
        }
    }
    return true;
}

// Byte offset of column 0's first tap when every output column x is an image column whose taps
// are source pixels i0 + 2x and i0 + 2x + 1 with weights exactly 1/2 (a 2:1 reduction across,
// 1280 -> 640 for instance), else -1.
int half_first_tap(const LbFrame& f, int dst_w) {
    if (f.pad_x != 0 || f.new_w != dst_w) return -1;
    const Tap t0 = interp_tap(f.rw, 0, f.src_w);
    for (int x = 0; x < dst_w; ++x) {
        const Tap t = interp_tap(f.rw, x, f.src_w);
        if (t.l0 != 0.5f || t.l1 != 0.5f || t.i1 != t.i0 + 1 || t.i0 != t0.i0 + 2 * x) return -1;
    }
    return t0.i0 * 3;
}

const char* plan_letterbox(const FrameView* frames, int n, void* out, int dst_h, int dst_w, int vec, int max_warps,
                           int smem_max,
                           const float mean[3], const float stdv[3], int swap_rb,
                           float pad_value, const float* pad_out, bool nv12, int matrix, int sampling,
                           Plan* plan) {
    LbParams& p = plan->p;
    std::memset(&p, 0, sizeof(p));
    p.out = out;
    p.n = n;
    p.dst_h = dst_h;
    p.dst_w = dst_w;
    p.total_rows = n * dst_h;
    p.swap_rb = swap_rb;
    p.arith = normalise_arith_ok(mean[0], stdv[0]) && normalise_arith_ok(mean[1], stdv[1]) &&
              normalise_arith_ok(mean[2], stdv[2]);
    p.matrix = matrix;
    p.sampling = sampling;
    for (int c = 0; c < 3; ++c) {
        p.mean[c] = mean[c];
        p.stdv[c] = stdv[c];
        p.pad_out[c] = pad_out ? pad_out[c] : (pad_value - mean[c]) / stdv[c];
        p.rcp[c] = 1.0f / stdv[c];
    }
    p.n2 = make_norm2(p.mean, p.stdv, p.rcp);
    p.mean_zero = (mean[0] == 0.f || mean[1] == 0.f || mean[2] == 0.f) ? 1 : 0;
    p.exact_arith = markstein_exact_on_bytes(p.mean, p.stdv, p.rcp) ? 1 : 0;
    p.exact_one = p.exact_arith && division_form_exact(1, p.mean, p.stdv, p.rcp, 255, 1.f) ? 1 : 0;
    // Half-weight rows' values are quarter integers S / 4, S = 0..1020.
    p.half_mode = nv12 ? 0
                : division_form_exact(1, p.mean, p.stdv, p.rcp, 1020, 4.f) ? 1
                : division_form_exact(2, p.mean, p.stdv, p.rcp, 1020, 4.f) ? 2 : 0;
    p.half_fold = 1;
    for (int c = 0; c < 3; ++c) {
        // is 2^21 + mean a float? (both sides exact in double for |mean| <= 2^20)
        const float t = 2097152.0f + mean[c];
        if (!(std::fabs(mean[c]) <= 1048576.0f) || (double)t - 2097152.0 != (double)mean[c]) p.half_fold = 0;
    }
    for (int c = 0; c < 3; ++c) {
        const float k = p.half_fold ? -(2097152.0f + mean[c]) : -mean[c];
        p.half_c[c] = make_float2(k, k);
    }
    int max_row_bytes = 16;
    bool second = false;
    for (int i = 0; i < n; ++i) {
        LbFrame& f = p.f[i];
        Fit fit;
        frame_fit(frames[i], dst_h, dst_w, &fit);
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
        f.half_a0 = (!nv12 && vec == 4) ? half_first_tap(f, dst_w) : -1;
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
    // Rows per slot. BGR: i0 [, i1]. NV12: luma i0 [, luma i1], then chroma i0 [, i1]
    // (the first chroma row is at spr / 2).
    p.spr = nv12 ? (second && sampling != 0 ? 4 : 2) : (second ? 2 : 1);
    p.slot_bytes = ((max_row_bytes + 16 + 15) / 16) * 16;
    p.tstride = ((dst_w + 7) / 8) * 8;
    const int groups = (dst_w + vec - 1) / vec;
    const int gstride = ((groups + 3) / 4) * 4;
    p.table_bytes = (3 * p.tstride + gstride) * 4;
    // Ring depth and warps per CTA from the shared budget: the deepest ring that still gives
    // max_warps warps, else depth 1; column tables give way before failing.
    const int64_t slot = (int64_t)p.spr * p.slot_bytes;
    auto warps_for = [&](int depth, int ntab) {
        const int64_t room = (int64_t)smem_max - (int64_t)ntab * p.table_bytes;
        return room <= 0 ? 0 : (int)std::min<int64_t>(max_warps, room / (depth * slot));
    };
    int depth = kMaxDepth;
    while (depth > 1 && warps_for(depth, p.ntables) < max_warps) --depth;
    while (p.ntables > 0 && warps_for(depth, p.ntables) < 1) {
        --p.ntables;
        for (int i = 0; i < n; ++i)
            if (p.f[i].table == p.ntables) p.f[i].table = -1;
    }
    const int warps = warps_for(depth, p.ntables);
    if (warps < 1) return "source rows are too wide to stage in shared memory";
    p.depth = depth;
    p.warp_bytes = (int)(depth * slot);
    plan->warps = warps;
    p.table_off = warps * p.warp_bytes;
    plan->smem = p.table_off + p.ntables * p.table_bytes;
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

template <typename OutT, int VEC, bool NV12, int CTAS>
cudaError_t launch_one(const Plan& plan, cudaStream_t stream) {
    auto kernel = letterbox_kernel<OutT, VEC, NV12, CTAS>;
    cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kernel), cta_smem<CTAS>());
    if (e != cudaSuccess) return e;
    // CTAS CTAs per SM (fewer when the batch has fewer rows than the grid has warps).
    const int rows = plan.p.total_rows;
    const int grid = std::max(1, std::min(CTAS * sm_count(), (rows + plan.warps - 1) / plan.warps));
    return launch_dependent(kernel, dim3(grid), dim3(plan.warps * 32), plan.smem, stream, plan.p);
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

int letterbox_fit_f32(int src_h, int src_w, int dst_h, int dst_w, Fit* out) {
    if (src_h <= 0 || src_w <= 0 || dst_h <= 0 || dst_w <= 0) return SHIPK_EINVAL;
    // ops.cu:341-356: float32 throughout; nearbyint() rounds half to even.
    const float s = std::min((float)dst_w / (float)src_w, (float)dst_h / (float)src_h);
    const float nw = std::nearbyint((float)src_w * s);
    const float nh = std::nearbyint((float)src_h * s);
    out->new_w = nw < 1.0f ? 1 : (int)nw;
    out->new_h = nh < 1.0f ? 1 : (int)nh;
    out->pad_x = (dst_w - out->new_w) / 2;
    out->pad_y = (dst_h - out->new_h) / 2;
    out->scale = s;
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
                        cudaStream_t stream, const float* pad_out) {
    const size_t elem = out_dtype == SHIPK_DTYPE_F32 ? 4 : 2;
    const size_t per_image = (size_t)3 * dst_h * dst_w * elem;
    for (int start = 0; start < n; start += kMaxBatch) {
        const int count = std::min(kMaxBatch, n - start);
        void* chunk_out = static_cast<uint8_t*>(out) + per_image * start;
        const bool aligned = (reinterpret_cast<uintptr_t>(chunk_out) & 15) == 0;
        // fp16: groups of 8 pixels (16-byte stores) for NV12; groups of 4 (8-byte stores) for BGR,
        // whose byte loads then sit 36 bytes apart across lanes instead of 72, free of bank
        // conflicts (config 4's letterbox: 30.1 -> 29.4 us; NV12 was 1% slower with 4)
        const int vec = out_dtype == SHIPK_DTYPE_F32 ? (aligned && dst_w % 4 == 0 ? 4 : 1)
                        : nv12                       ? (aligned && dst_w % 8 == 0 ? 8 : 1)
                                                     : (aligned && dst_w % 4 == 0 ? 4 : 1);
        // BGR to float32 runs as two CTAs per SM, everything else as one (cta_smem)
        const int ctas = out_dtype == SHIPK_DTYPE_F32 && !nv12 ? 2 : 1;
        Plan plan;
        const char* why = plan_letterbox(frames + start, count, chunk_out, dst_h, dst_w, vec, kMaxWarps / ctas,
                                         ctas == 1 ? cta_smem<1>() : cta_smem<2>(), mean, stdv, swap_rb, pad_value,
                                         pad_out, nv12, matrix, sampling, &plan);
        if (why) return Status{SHIPK_ERANGE, why};
        cudaError_t e;
        if (out_dtype == SHIPK_DTYPE_F32) {
            if (nv12) e = vec == 4 ? launch_one<float, 4, true, 1>(plan, stream) : launch_one<float, 1, true, 1>(plan, stream);
            else e = vec == 4 ? launch_one<float, 4, false, 2>(plan, stream) : launch_one<float, 1, false, 2>(plan, stream);
        } else {
            if (nv12) e = vec == 8 ? launch_one<__half, 8, true, 1>(plan, stream) : launch_one<__half, 1, true, 1>(plan, stream);
            else e = vec == 4 ? launch_one<__half, 4, false, 1>(plan, stream) : launch_one<__half, 1, false, 1>(plan, stream);
        }
        if (e != cudaSuccess) return Status{SHIPK_ECUDA, cudaGetErrorString(e)};
    }
    return Status{SHIPK_OK, nullptr};
}

}  // namespace shipk
