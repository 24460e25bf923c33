// Device NMS, batched and optionally class-aware, in one launch with no host round trip.
//
// Reference semantics: NumpyImageOps.nms, src/shipinfer/runtime/ops/numpy_ops.py:120-155,
// in numpy 2's float32 arithmetic:
//   candidates: scores >= f32(score_threshold); visiting order: score descending, ties to
//   the lower index (a stable argsort of -scores);
//   areas = max(0, x2-x1) * max(0, y2-y1);
//   inter = max(0, min(x2a,x2b) - max(x1a,x1b)) * max(0, min(y2a,y2b) - max(y1a,y1b));
//   iou   = inter / max(area_a + area_b - inter, f32(1e-9)); a candidate survives a kept box
//   when iou <= f32(iou_threshold); np.maximum / np.minimum propagate NaN.
// Class-aware: the same per class, then the survivors of all classes merged by (score
// descending, index ascending) and cut to max_det.
//
// Layout: one 1024-thread CTA per segment (image, or image x class). The CTA
//   1. scans the image's scores (and classes) once with 16-byte loads, appending every
//      eligible candidate's 64-bit key (score order bits << 32 | ~index) to shared memory
//      with warp-aggregated atomics; a segment larger than kCap is processed kCap keys at a
//      time, each chunk chosen exactly by an 8-pass radix select below the previous chunk;
//   2. bitonic-sorts the keys descending, which is exactly the reference's visiting order;
//   3. gathers the boxes of the first kPre sorted candidates into shared memory in one round;
//   4. walks the order 32 candidates at a time: every warp checks the tile against a strided
//      share of the kept boxes (shared memory), the tile's own upper-triangle IoU masks come
//      from one __ballot_sync per row, and one warp resolves the tile greedily with __ffs /
//      __shfl_sync; it stops as soon as max_det boxes are kept.
// In class-aware mode each segment publishes its survivors, and the last segment of an image
// to finish (an atomic arrival count after a __threadfence) merges them: each survivor's rank
// is its position in its own list plus, per other list, a binary-searched count of keys
// above it, searched in shared memory.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace shipk {

namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kCap = 8192;  // keys sorted in shared memory at once
constexpr int kPre = 1024;  // sorted candidates whose boxes are gathered into shared memory
constexpr int kTile = 32;
constexpr int kMaxClassesMerged = 1024;  // lists merged in shared memory (more: global search)

struct NmsParams {
    const float* boxes;
    const float* scores;
    const int32_t* classes;
    int n, segs, class_aware;
    float iou_thr, score_thr;
    int max_det;
    int vec;             // scores/classes rows are 16-byte aligned with n % 4 == 0
    int64_t* keep;
    int32_t* counts;
    int32_t* seg_idx;   // [batch * segs, max_det]
    int32_t* seg_cnt;   // [batch * segs]
    int32_t* arrivals;  // [batch], zero on entry; the merging CTA leaves it zero
};

__device__ __forceinline__ uint64_t cand_key(float s, int idx) {
    uint32_t u = __float_as_uint(s);
    if ((u & 0x7fffffffu) == 0) u = 0;  // -0.0 sorts with +0.0, as the argsort compares them
    const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((uint64_t)ord << 32) | (uint64_t)(0xffffffffu - (uint32_t)idx);
}
__device__ __forceinline__ int key_index(uint64_t k) {
    return (int)(0xffffffffu - (uint32_t)(k & 0xffffffffu));
}

// np.maximum / np.minimum: NaN in either operand gives NaN.
__device__ __forceinline__ float nmax(float a, float b) {
    return (a != a || b != b) ? __int_as_float(0x7fc00000) : (a > b ? a : b);
}
__device__ __forceinline__ float nmin(float a, float b) {
    return (a != a || b != b) ? __int_as_float(0x7fc00000) : (a < b ? a : b);
}

__device__ __forceinline__ float box_area(float4 b) {
    return __fmul_rn(nmax(0.f, __fsub_rn(b.z, b.x)), nmax(0.f, __fsub_rn(b.w, b.y)));
}

// True when `a` (kept) removes `b`: !(iou <= thr), numpy's survivor test negated.
__device__ __forceinline__ bool suppresses(float4 a, float area_a, float4 b, float area_b,
                                           float thr) {
    const float iw = nmax(0.f, __fsub_rn(nmin(a.z, b.z), nmax(a.x, b.x)));
    const float ih = nmax(0.f, __fsub_rn(nmin(a.w, b.w), nmax(a.y, b.y)));
    const float inter = __fmul_rn(iw, ih);
    const float denom = nmax(__fsub_rn(__fadd_rn(area_a, area_b), inter), 1e-9f);
    if (inter == 0.f && denom == denom) return !(0.f <= thr);  // 0 / denom is +-0
    return !(__fdiv_rn(inter, denom) <= thr);
}

__device__ __forceinline__ float4 load_box(const float* bx, int idx) {
    const float* q = bx + (int64_t)idx * 4;
    return make_float4(__ldg(q), __ldg(q + 1), __ldg(q + 2), __ldg(q + 3));
}

// Warp-aggregated append to a shared counter; returns this lane's slot (or -1). Every lane
// of the warp must call it.
__device__ __forceinline__ int warp_append(int* counter, bool take) {
    const unsigned m = __ballot_sync(0xffffffffu, take);
    if (m == 0) return -1;
    const int lane = threadIdx.x & 31;
    const int leader = __ffs(m) - 1;
    int base = 0;
    if (lane == leader) base = atomicAdd(counter, __popc(m));
    base = __shfl_sync(0xffffffffu, base, leader);
    return take ? base + __popc(m & ((1u << lane) - 1u)) : -1;
}

__global__ void __launch_bounds__(kThreads, 1) nms_kernel(const __grid_constant__ NmsParams p) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint64_t* keys = reinterpret_cast<uint64_t*>(smem_raw);
    float4* cbox = reinterpret_cast<float4*>(keys + kCap);
    float* carea = reinterpret_cast<float*>(cbox + kPre);
    float4* kbox = reinterpret_cast<float4*>(carea + kPre);
    float* karea = reinterpret_cast<float*>(kbox + p.max_det);
    int* kidx = reinterpret_cast<int*>(karea + p.max_det);

    __shared__ float4 tbox[kTile];
    __shared__ float tarea[kTile];
    __shared__ int tidx[kTile];
    __shared__ unsigned trow[kTile];
    __shared__ unsigned tsupp;
    __shared__ int s_count, s_nkept, s_last;
    __shared__ unsigned hist[256];
    __shared__ unsigned long long s_prefix;
    __shared__ int s_want;
    __shared__ int s_off[kMaxClassesMerged + 1];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int seg = blockIdx.x;
    const int img = seg / p.segs;
    const int cls = seg - img * p.segs;
    const int n = p.n;
    const float* sc = p.scores + (int64_t)img * n;
    const int32_t* cl = p.classes ? p.classes + (int64_t)img * n : nullptr;
    const float* bx = p.boxes + (int64_t)img * n * 4;
    const float score_thr = p.score_thr, iou_thr = p.iou_thr;
    const bool aware = p.class_aware != 0;

    // Append the keys of candidates below `boundary` (and at or above `floor_key`) to keys[]
    // in any order; returns the count (which may exceed kCap: only the first kCap are kept).
    auto collect = [&](uint64_t boundary, uint64_t floor_key) -> int {
        if (tid == 0) s_count = 0;
        __syncthreads();
        const int groups = (n + 3) >> 2;
        for (int g0 = 0; g0 < groups; g0 += kThreads) {
            const int g = g0 + tid;
            float s4[4] = {0.f, 0.f, 0.f, 0.f};
            int c4[4] = {0, 0, 0, 0};
            const int i0 = g * 4;
            if (g < groups) {
                if (p.vec) {
                    const float4 v = __ldg(reinterpret_cast<const float4*>(sc) + g);
                    s4[0] = v.x; s4[1] = v.y; s4[2] = v.z; s4[3] = v.w;
                    if (aware) {
                        const int4 c = __ldg(reinterpret_cast<const int4*>(cl) + g);
                        c4[0] = c.x; c4[1] = c.y; c4[2] = c.z; c4[3] = c.w;
                    }
                } else {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        if (i0 + q < n) {
                            s4[q] = __ldg(sc + i0 + q);
                            if (aware) c4[q] = __ldg(cl + i0 + q);
                        }
                    }
                }
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int i = i0 + q;
                bool take = false;
                uint64_t k = 0;
                if (g < groups && i < n && s4[q] >= score_thr && (!aware || c4[q] == cls)) {
                    k = cand_key(s4[q], i);
                    take = k < boundary && k >= floor_key;
                }
                const int pos = warp_append(&s_count, take);
                if (take && pos < kCap) keys[pos] = k;
            }
        }
        __syncthreads();
        const int count = s_count;
        __syncthreads();  // every thread has read s_count before anyone resets it
        return count;
    };

    if (tid == 0) s_nkept = 0;
    uint64_t boundary = ~0ull;  // still to visit: keys below this
    for (;;) {
        int m = collect(boundary, 0);
        if (m == 0 || s_nkept >= p.max_det) break;
        int mc = m;
        if (m > kCap) {
            // exactly the kCap largest keys below the boundary: an 8-pass radix select
            uint64_t prefix = 0;
            int want = kCap;
            for (int shift = 56; shift >= 0; shift -= 8) {
                if (tid < 256) hist[tid] = 0;
                __syncthreads();
                for (int i = tid; i < n; i += kThreads) {
                    const float s = __ldg(sc + i);
                    if (!(s >= score_thr) || (aware && __ldg(cl + i) != cls)) continue;
                    const uint64_t k = cand_key(s, i);
                    if (k >= boundary) continue;
                    if (shift < 56 && (k >> (shift + 8)) != (prefix >> (shift + 8))) continue;
                    atomicAdd(&hist[(k >> shift) & 255u], 1u);
                }
                __syncthreads();
                if (warp == 0) {
                    // lane L owns digits 255-8L .. 248-8L (high to low)
                    unsigned c[8];
                    unsigned sum = 0;
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        c[q] = hist[255 - 8 * lane - q];
                        sum += c[q];
                    }
                    unsigned incl = sum;
                    for (int o = 1; o < 32; o <<= 1) {
                        const unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
                        if (lane >= o) incl += v;
                    }
                    const unsigned excl = incl - sum;
                    const unsigned hit = __ballot_sync(0xffffffffu, excl < (unsigned)want &&
                                                                        incl >= (unsigned)want);
                    const int owner = __ffs(hit) - 1;
                    if (lane == owner) {
                        unsigned cum = excl;
                        for (int q = 0; q < 8; ++q) {
                            if (cum + c[q] >= (unsigned)want) {
                                const unsigned digit = 255u - 8u * lane - q;
                                s_prefix = prefix | ((uint64_t)digit << shift);
                                s_want = want - (int)cum;
                                break;
                            }
                            cum += c[q];
                        }
                    }
                }
                __syncthreads();
                prefix = s_prefix;
                want = s_want;
            }
            mc = min(collect(boundary, prefix), kCap);  // the kCap largest, prefix included
        }
        if (mc == 0) break;  // unreachable when m > 0; keeps `boundary` below in range

        int P = 2;
        while (P < mc) P <<= 1;
        for (int i = mc + tid; i < P; i += kThreads) keys[i] = 0;  // 0 sorts last
        __syncthreads();

        // ---- bitonic sort, descending
        for (int k = 2; k <= P; k <<= 1) {
            for (int j = k >> 1; j > 0; j >>= 1) {
                for (int q = tid; q < (P >> 1); q += kThreads) {
                    const int i = ((q & ~(j - 1)) << 1) | (q & (j - 1));
                    const int l = i + j;
                    const uint64_t a = keys[i], b = keys[l];
                    const bool desc = (i & k) == 0;
                    if (desc ? (a < b) : (a > b)) {
                        keys[i] = b;
                        keys[l] = a;
                    }
                }
                __syncthreads();
            }
        }

        // ---- the boxes of the leading candidates, in one round of gathers
        const int pre = min(mc, kPre);
        for (int q = tid; q < pre; q += kThreads) {
            const float4 b = load_box(bx, key_index(keys[q]));
            cbox[q] = b;
            carea[q] = box_area(b);
        }
        __syncthreads();

        // ---- greedy walk, a tile of 32 candidates at a time
        for (int base = 0; base < mc; base += kTile) {
            const int K = s_nkept;
            if (K >= p.max_det) break;
            const int cnt = min(kTile, mc - base);
            if (warp == 0) {
                if (lane < cnt) {
                    const int q = base + lane;
                    const int idx = key_index(keys[q]);
                    float4 b;
                    float a;
                    if (q < kPre) {
                        b = cbox[q];
                        a = carea[q];
                    } else {
                        b = load_box(bx, idx);
                        a = box_area(b);
                    }
                    tbox[lane] = b;
                    tarea[lane] = a;
                    tidx[lane] = idx;
                }
                if (lane == 0) tsupp = 0;
            }
            __syncthreads();
            // against every box kept so far: warp w takes kept boxes w, w+32, ...
            bool sup = false;
            if (lane < cnt) {
                const float4 me = tbox[lane];
                const float ma = tarea[lane];
                for (int j = warp; j < K; j += kWarps) {
                    if (suppresses(kbox[j], karea[j], me, ma, iou_thr)) {
                        sup = true;
                        break;
                    }
                }
            }
            const unsigned bal = __ballot_sync(0xffffffffu, sup);
            if (lane == 0 && bal) atomicOr(&tsupp, bal);
            // inside the tile: row w = the later candidates that candidate w would remove
            if (warp < cnt) {
                bool s2 = false;
                if (lane > warp && lane < cnt)
                    s2 = suppresses(tbox[warp], tarea[warp], tbox[lane], tarea[lane], iou_thr);
                const unsigned row = __ballot_sync(0xffffffffu, s2);
                if (lane == 0) trow[warp] = row;
            }
            __syncthreads();
            if (warp == 0) {
                const unsigned valid = cnt == 32 ? 0xffffffffu : ((1u << cnt) - 1u);
                unsigned alive = valid & ~tsupp;
                const unsigned myrow = lane < cnt ? trow[lane] : 0u;
                unsigned kept = 0;
                int room = p.max_det - K;
                while (alive && room > 0) {
                    const int i = __ffs(alive) - 1;
                    kept |= 1u << i;
                    --room;
                    alive &= ~(__shfl_sync(0xffffffffu, myrow, i) | (1u << i));
                }
                if ((kept >> lane) & 1u) {
                    const int pos = K + __popc(kept & ((1u << lane) - 1u));
                    kbox[pos] = tbox[lane];
                    karea[pos] = tarea[lane];
                    kidx[pos] = tidx[lane];
                }
                if (lane == 0) s_nkept = K + __popc(kept);
            }
            __syncthreads();
        }
        if (mc == m || s_nkept >= p.max_det) break;
        boundary = keys[mc - 1];
        __syncthreads();
    }
    __syncthreads();
    const int nkept = s_nkept;

    if (!aware) {
        int64_t* out = p.keep + (int64_t)img * p.max_det;
        for (int i = tid; i < p.max_det; i += kThreads) out[i] = i < nkept ? kidx[i] : -1;
        if (tid == 0) p.counts[img] = nkept;
        return;
    }

    // ---- class-aware: publish this class's survivors; the image's last class merges
    int32_t* mine = p.seg_idx + (int64_t)seg * p.max_det;
    for (int i = tid; i < nkept; i += kThreads) mine[i] = kidx[i];
    if (tid == 0) p.seg_cnt[seg] = nkept;
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(p.arrivals + img, 1) == p.segs - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();

    const int first = img * p.segs;
    int64_t* out = p.keep + (int64_t)img * p.max_det;
    if (tid == 0) {
        int total = 0;
        for (int c = 0; c < p.segs && c < kMaxClassesMerged; ++c) {
            s_off[c] = total;
            total += __ldcg(p.seg_cnt + first + c);
        }
        s_off[min(p.segs, kMaxClassesMerged)] = total;
        s_count = total;
    }
    __syncthreads();
    const bool in_smem = p.segs <= kMaxClassesMerged && s_count <= kCap;
    int total = 0;
    if (in_smem) {
        total = s_count;
        // every survivor's key, list after list, each list already in descending order
        for (int c = 0; c < p.segs; ++c) {
            const int off = s_off[c], cnt = s_off[c + 1] - off;
            const int32_t* list = p.seg_idx + (int64_t)(first + c) * p.max_det;
            for (int q = tid; q < cnt; q += kThreads) {
                const int idx = __ldcg(list + q);
                keys[off + q] = cand_key(__ldg(sc + idx), idx);
            }
        }
        __syncthreads();
        const int out_n = min(total, p.max_det);
        for (int e = tid; e < total; e += kThreads) {
            int c = 0;  // the list holding element e
            while (s_off[c + 1] <= e) ++c;
            const uint64_t key = keys[e];
            int rank = e - s_off[c];
            for (int o = 0; o < p.segs; ++o) {
                if (o == c) continue;
                int lo = s_off[o], hi = s_off[o + 1];  // first position in list o not above key
                while (lo < hi) {
                    const int mid = (lo + hi) >> 1;
                    if (keys[mid] > key) lo = mid + 1;
                    else hi = mid;
                }
                rank += lo - s_off[o];
            }
            if (rank < out_n) out[rank] = key_index(key);
        }
    } else {
        for (int c = 0; c < p.segs; ++c) total += __ldcg(p.seg_cnt + first + c);
        const int out_n = min(total, p.max_det);
        for (int c = 0; c < p.segs; ++c) {
            const int cnt = __ldcg(p.seg_cnt + first + c);
            const int32_t* list = p.seg_idx + (int64_t)(first + c) * p.max_det;
            for (int q = tid; q < cnt; q += kThreads) {
                const int idx = __ldcg(list + q);
                const uint64_t key = cand_key(__ldg(sc + idx), idx);
                int rank = q;
                for (int o = 0; o < p.segs; ++o) {
                    if (o == c) continue;
                    const int ocnt = __ldcg(p.seg_cnt + first + o);
                    const int32_t* other = p.seg_idx + (int64_t)(first + o) * p.max_det;
                    int lo = 0, hi = ocnt;
                    while (lo < hi) {
                        const int mid = (lo + hi) >> 1;
                        const int oi = __ldcg(other + mid);
                        if (cand_key(__ldg(sc + oi), oi) > key) lo = mid + 1;
                        else hi = mid;
                    }
                    rank += lo;
                }
                if (rank < out_n) out[rank] = idx;
            }
        }
    }
    const int out_n = min(total, p.max_det);
    for (int i = out_n + tid; i < p.max_det; i += kThreads) out[i] = -1;
    if (tid == 0) {
        p.counts[img] = out_n;
        p.arrivals[img] = 0;
    }
}

struct Layout {
    size_t seg_idx, seg_cnt, arrivals, total;
};

Layout nms_layout(int batch, int segs, int max_det) {
    auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
    Layout l;
    const size_t S = (size_t)batch * segs;
    l.seg_idx = 0;
    l.seg_cnt = up(S * (size_t)std::max(max_det, 1) * 4);
    l.arrivals = l.seg_cnt + up(S * 4);
    l.total = l.arrivals + up((size_t)batch * 4);
    return l;
}

constexpr int kNmsMaxDet = 4096;

int smem_bytes(int max_det) { return kCap * 8 + kPre * (16 + 4) + max_det * (16 + 4 + 4); }

}  // namespace

size_t nms_workspace_bytes(int batch, int n, int num_classes, int class_aware, int max_det) {
    (void)n;
    const int segs = class_aware ? std::max(num_classes, 1) : 1;
    return nms_layout(std::max(batch, 0), segs, max_det).total;
}

Status launch_nms(const float* boxes, const float* scores, const int32_t* classes, int batch,
                  int n, int num_classes, int class_aware, float iou_thr, float score_thr,
                  int max_det, int64_t* keep, int32_t* counts, void* workspace,
                  size_t workspace_bytes, bool zero_arrivals, cudaStream_t stream) {
    if (max_det > kNmsMaxDet) return Status{SHIPK_ERANGE, "max_det above 4096"};
    if (batch == 0) return Status{SHIPK_OK, nullptr};
    if (max_det <= 0 || n == 0) {
        cudaError_t e = cudaSuccess;
        if (max_det > 0)
            e = cudaMemsetAsync(keep, 0xff, (size_t)batch * max_det * sizeof(int64_t), stream);
        if (e == cudaSuccess) e = cudaMemsetAsync(counts, 0, (size_t)batch * sizeof(int32_t), stream);
        if (e != cudaSuccess) return Status{SHIPK_ECUDA, cudaGetErrorString(e)};
        return Status{SHIPK_OK, nullptr};
    }
    const int segs = class_aware ? num_classes : 1;
    const Layout l = nms_layout(batch, segs, max_det);
    if (workspace_bytes < l.total) return Status{SHIPK_ENOMEM, "NMS workspace is too small"};
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    NmsParams p;
    p.boxes = boxes;
    p.scores = scores;
    p.classes = classes;
    p.n = n;
    p.segs = segs;
    p.class_aware = class_aware ? 1 : 0;
    p.iou_thr = iou_thr;
    p.score_thr = score_thr;
    p.max_det = max_det;
    const bool aligned = (reinterpret_cast<uintptr_t>(scores) & 15) == 0 &&
                         (!class_aware || (reinterpret_cast<uintptr_t>(classes) & 15) == 0);
    p.vec = aligned && n % 4 == 0;
    p.keep = keep;
    p.counts = counts;
    p.seg_idx = reinterpret_cast<int32_t*>(ws + l.seg_idx);
    p.seg_cnt = reinterpret_cast<int32_t*>(ws + l.seg_cnt);
    p.arrivals = reinterpret_cast<int32_t*>(ws + l.arrivals);
    if (zero_arrivals && class_aware) {
        cudaError_t e = cudaMemsetAsync(p.arrivals, 0, (size_t)batch * sizeof(int32_t), stream);
        if (e != cudaSuccess) return Status{SHIPK_ECUDA, cudaGetErrorString(e)};
    }
    {
        cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(nms_kernel), smem_bytes(kNmsMaxDet));
        if (e != cudaSuccess) return Status{SHIPK_ECUDA, cudaGetErrorString(e)};
    }
    const long long grid = (long long)batch * segs;
    if (grid > 0x7fffffffLL) return Status{SHIPK_ERANGE, "too many NMS segments"};
    nms_kernel<<<(int)grid, kThreads, smem_bytes(max_det), stream>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return Status{SHIPK_ECUDA, cudaGetErrorString(e)};
    return Status{SHIPK_OK, nullptr};
}

}  // namespace shipk
