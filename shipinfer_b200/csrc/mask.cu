// Mask area per crop: the segmenter's fold from prototype masks to one area per object.
//
// Reference semantics: mask_area_into / mask_area_kernel, csrc/shipinfer/runtime/ops.cu:196-255
// and :418-458, per crop:
//   * the strongest candidate row: a scan from row 0 keeping the first strict maximum of the
//     score column (so a NaN score in row 0 stays chosen, and NaN scores elsewhere never win);
//   * a score below score_threshold: area 0;
//   * else the prototype cells whose logit, the coefficients of that row against the planes
//     accumulated in channel order as one fused multiply-add per channel, reaches
//     cut = log(t / (1 - t)) (t the mask threshold; the host computes it as the reference's host
//     code does), counted, times crop_height * crop_width / cells.
//
// Layout: a thread-block cluster of kCluster CTAs per crop, each CTA taking a slice of the
// cells (16-byte loads of four consecutive cells per channel where the bank's rows allow it);
// the CTAs' counts meet in CTA 0's shared memory through distributed shared memory, and CTA 0
// writes the area. The prototype bank (3.3 MB per crop at 32 x 160 x 160) is read once, by
// 8 x 256 threads instead of the reference's one 256-thread block.
#include "common.cuh"
#include "kernels.h"

#include <cooperative_groups.h>

#include <algorithm>
#include <cmath>

namespace cg = cooperative_groups;

namespace shipk {

namespace {

constexpr int kCluster = 8;
// 256 threads per CTA: smaller CTAs spread a batch's clusters more evenly over the SMs than 512
// did (40.3 against 44.7 us for 64 crops; 128 and 192 were slower, so were 16-CTA clusters).
constexpr int kThreads = 256;
constexpr int kMaxChannels = 256;

struct MaskArgs {
    const float* rows;    // [crops, candidates, stride]
    int candidates, stride, prefix;
    const float* protos;  // [crops, channels, cells]
    int channels, cells;
    int vec;              // cells % 4 == 0 and protos 16-byte aligned: four cells per load
    float score_thr, cut, cell_px;
    float* areas;         // [crops]
};

__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kThreads)
mask_area_kernel(const __grid_constant__ MaskArgs a) {
    __shared__ float coef[kMaxChannels];
    __shared__ int warp_sum[kThreads / 32];
    __shared__ int cta_sum[kCluster];
    __shared__ int s_best;

    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int crop = blockIdx.x / kCluster;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float* cand = a.rows + (int64_t)crop * a.candidates * a.stride;

    // ---- the strongest row (every CTA of the cluster finds the same one)
    if (warp == 0) {
        // each lane: the first strict maximum over its rows, NaN scores never winning
        int best = -1;
        float best_s = 0.f;
        for (int c = lane; c < a.candidates; c += 32) {
            const float s = __ldg(cand + (int64_t)c * a.stride + 4);
            if (s != s) continue;
            if (best < 0 || s > best_s) {
                best = c;
                best_s = s;
            }
        }
        // across lanes: the larger score, the lower row on equal scores (-0.0 == +0.0)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const int ob = __shfl_xor_sync(0xffffffffu, best, o);
            const float os = __shfl_xor_sync(0xffffffffu, best_s, o);
            if (ob >= 0 && (best < 0 || os > best_s || (os == best_s && ob < best))) {
                best = ob;
                best_s = os;
            }
        }
        if (lane == 0) {
            const float s0 = __ldg(cand + 4);
            // row 0 starts the reference's scan: a NaN there is never displaced, and when every
            // score is NaN the scan ends where it began
            s_best = (s0 != s0 || best < 0) ? 0 : best;
        }
    }
    __syncthreads();
    const float* chosen = cand + (int64_t)s_best * a.stride;
    const bool found = !(__ldg(chosen + 4) < a.score_thr);
    for (int m = tid; m < a.channels; m += kThreads) coef[m] = __ldg(chosen + a.prefix + m);
    __syncthreads();

    // ---- this CTA's slice of the cells
    int inside = 0;
    if (found) {
        const float* planes = a.protos + (int64_t)crop * a.channels * a.cells;
        const int span = (((a.cells + kCluster - 1) / kCluster) + 3) & ~3;
        const int c0 = rank * span, c1 = min(a.cells, c0 + span);
        if (a.vec) {
            for (int cell = c0 + 4 * tid; cell < c1; cell += 4 * kThreads) {  // c0, c1 multiples of 4
                float l0 = 0.f, l1 = 0.f, l2 = 0.f, l3 = 0.f;
                for (int m = 0; m < a.channels; ++m) {
                    const float4 v = __ldg(reinterpret_cast<const float4*>(planes + (int64_t)m * a.cells + cell));
                    const float w = coef[m];
                    l0 = __fmaf_rn(w, v.x, l0);
                    l1 = __fmaf_rn(w, v.y, l1);
                    l2 = __fmaf_rn(w, v.z, l2);
                    l3 = __fmaf_rn(w, v.w, l3);
                }
                inside += (l0 >= a.cut) + (l1 >= a.cut) + (l2 >= a.cut) + (l3 >= a.cut);
            }
        } else {
            for (int cell = c0 + tid; cell < c1; cell += kThreads) {
                float l = 0.f;
                for (int m = 0; m < a.channels; ++m) l = __fmaf_rn(coef[m], __ldg(planes + (int64_t)m * a.cells + cell), l);
                inside += l >= a.cut;
            }
        }
    }

    // ---- counts: warp, CTA, then the cluster's CTA 0 through distributed shared memory
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) inside += __shfl_xor_sync(0xffffffffu, inside, o);
    if (lane == 0) warp_sum[warp] = inside;
    __syncthreads();
    if (warp == 0) {
        int v = lane < kThreads / 32 ? warp_sum[lane] : 0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) {
            int* dst = cluster.map_shared_rank(cta_sum, 0);
            dst[rank] = v;
        }
    }
    cluster.sync();  // every CTA's count is in CTA 0, and no CTA exits while its smem is addressed
    if (rank == 0 && tid == 0) {
        int total = 0;
        for (int r = 0; r < kCluster; ++r) total += cta_sum[r];
        a.areas[crop] = found ? __fmul_rn((float)total, a.cell_px) : 0.f;
    }
}

}  // namespace

Status launch_mask_area(const float* rows, int crops, int candidates, int stride, int prefix,
                        const float* protos, int channels, int cells, float score_threshold,
                        float mask_threshold, int crop_height, int crop_width, float* areas,
                        cudaStream_t stream) {
    if (crops <= 0) return Status{SHIPK_OK, nullptr};
    if (channels > kMaxChannels) return Status{SHIPK_ERANGE, "more than 256 mask channels"};
    MaskArgs a;
    a.rows = rows;
    a.candidates = candidates;
    a.stride = stride;
    a.prefix = prefix;
    a.protos = protos;
    a.channels = channels;
    a.cells = cells;
    a.vec = (cells % 4 == 0) && (reinterpret_cast<uintptr_t>(protos) & 15) == 0;
    a.score_thr = score_threshold;
    // the reference's host arithmetic (ops.cu:444-447): float log of the odds, and the area of
    // one cell in crop pixels
    a.cut = std::log(mask_threshold / (1.f - mask_threshold));
    a.cell_px = static_cast<float>(crop_height) * static_cast<float>(crop_width) / static_cast<float>(cells);
    a.areas = areas;
    if ((long long)crops * kCluster > 0x7fffffffLL) return Status{SHIPK_ERANGE, "too many crops for one launch"};
    mask_area_kernel<<<crops * kCluster, kThreads, 0, stream>>>(a);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return Status{SHIPK_ECUDA, cudaGetErrorString(e)};
    return Status{SHIPK_OK, nullptr};
}

}  // namespace shipk
