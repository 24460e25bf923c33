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
// Layout: one 1024-thread CTA per segment (image, or image x class), the leader, with up to 7
// helper CTAs in the same thread-block cluster when the device has SMs to spare. The visiting
// order is the descending order of 64-bit keys (score order bits << 32 | ~index). Every CTA of
// a segment
//   1. scans the image's scores (and classes) once with 16-byte loads, placing every eligible
//      key in shared memory by a block-wide prefix sum (more than kCap eligible keys: the kCap
//      largest, chosen by an exact radix select over global memory, and the rest in later
//      rounds), and records the score bits all of them share;
//   2. takes the kSort largest unvisited keys in descending order: in the first round from the
//      scan's counts of the keys in 2,048 buckets (a prefix sum over the buckets, a scatter of
//      the needed buckets' keys, a rank within each small bucket); otherwise (and when a
//      needed bucket is large) by an exact radix select over shared memory whose 8-bit digits
//      start below the shared bits, and a sort, one key per thread: each warp sorts a run of 32
//      with a bitonic network over __shfl_xor_sync, and the runs merge pairwise, a key's merged
//      position being its place in its run plus a binary-searched count of the partner run's
//      keys above it;
//   3. gathers those candidates' boxes into shared memory in one round;
//   4. (first round) computes its share of the suppression bits of every pair among the first
//      M = max_det + a margin candidates, as columns (for candidate b, which earlier
//      candidates would remove it), storing them into the leader's shared memory across the
//      cluster. After one cluster barrier the helpers are done; the leader settles the greedy
//      set over the columns with parallel passes (each candidate recomputed from the previous
//      pass's kept set, until a pass changes nothing);
//   5. (leader) walks any further candidates 32 at a time while fewer than max_det are kept:
//      every warp checks the tile against a strided share of the kept boxes, one
//      __ballot_sync per row gives the tile's own upper-triangle suppression masks, and one
//      warp resolves the tile, iterating only over candidates that can remove another.
// In class-aware mode with up to 8 classes the image's segments share one cluster, and after a
// cluster barrier the first leader merges every segment's kept keys through distributed shared
// memory; with more classes each segment publishes its survivors and the last segment of an
// image to finish (an atomic arrival count after a __threadfence) merges them. Either way a
// survivor's rank is its position in its own list plus, per other list, a binary-searched count
// of keys above it, searched in shared memory.
#include "common.cuh"
#include "kernels.h"

#include <cooperative_groups.h>

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <type_traits>

namespace shipk {

namespace {

namespace cg = cooperative_groups;

constexpr int kThreads = 1024;
constexpr int kMaxCluster = 8;  // portable thread-block cluster size: segments merged in a cluster
constexpr int kWarps = kThreads / 32;
constexpr int kCap = 8192;   // eligible keys held in shared memory at once
constexpr int kSort = 512;   // keys sorted and walked per round (one per thread of the first half)
constexpr int kTile = 32;
constexpr int kMaxClassesMerged = 1024;  // lists merged in shared memory (more: global search)
constexpr int kBlockMaxDet = 1024;  // max_det up to which the first round starts with a block resolve
constexpr int kMaskStride = 17;     // words per column of the block's suppression bits (odd: no bank conflicts)
constexpr int kMaxPasses = 16;      // parallel passes of the block resolve before the word-by-word form
constexpr int kScanGroups = 3;      // groups of four candidates a thread loads per scan step (8400 in one)
// The first round's bucket sort: keys counted by kBucketBits bits below the bits they all share;
// a bucket the round needs may hold at most kBucketMax keys (else the radix select and sort).
constexpr int kBucketBits = 11;
constexpr int kBuckets = 1 << kBucketBits;  // two per thread
constexpr int kBucketMax = 64;
constexpr int kRecvKeys = 2048;  // class merge in a cluster: segments' kept keys pushed to its first leader
// A pool key that a kept box removes. No candidate has this key: it would need a score whose
// order bits are all ones, a NaN, which never passes the score threshold.
constexpr uint64_t kRemoved = ~0ull;

struct NmsParams {
    const float* boxes;
    const float* scores;
    const int32_t* classes;
    int n, segs, class_aware;
    float iou_thr, score_thr;
    double iou_mid;      // midpoint of iou_thr and the next float above it (exact in double)
    int iou_even;        // iou_thr's last significand bit is 0 (a tie at the midpoint rounds to it)
    float iou_half;      // mid - thr (a power of two) when the single-precision test is exact, else 0
    int max_det;
    int vec;             // score/class rows are 16-byte aligned with n % 4 == 0
    int64_t* keep;
    int32_t* counts;
    int32_t* seg_idx;   // [batch * segs, max_det]
    int32_t* seg_cnt;   // [batch * segs]
    int32_t* arrivals;  // [batch], zero on entry; the merging CTA leaves it zero
    int cluster;        // an image's segments form one thread-block cluster: merge through its
                        // distributed shared memory (no seg_idx, seg_cnt or arrivals)
    int block_cap;      // candidates resolved at once at the start of the first round (0: none)
    int split;          // CTAs per segment: the leader and split - 1 helpers sharing the block's pair
                        // tests, one cluster (blockIdx.x = segment * split + part)
};

// A score's order bits: the key's upper half.
__device__ __forceinline__ uint32_t score_ord(float s) {
    uint32_t u = __float_as_uint(s);
    if ((u & 0x7fffffffu) == 0) u = 0;  // -0.0 sorts with +0.0, as the argsort compares them
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ uint64_t cand_key(float s, int idx) {
    return ((uint64_t)score_ord(s) << 32) | (uint64_t)(0xffffffffu - (uint32_t)idx);
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

__device__ __forceinline__ bool finite4(float4 b) {
    return isfinite(b.x) && isfinite(b.y) && isfinite(b.z) && isfinite(b.w);
}

// The IoU threshold as the survivor test uses it: thr itself, and for finite pairs the exact
// real-number form of RN(inter / denom) <= thr (below).
struct IouThr {
    float thr;
    double mid;  // (thr + next float above thr) / 2, exact in double
    bool even;   // thr's last significand bit is 0
    float half;  // mid - thr, or 0: no single-precision test
};

// True when `a` (kept) removes `b`: !(iou <= thr), numpy's survivor test negated. `both_finite`:
// neither box has a NaN or infinite coordinate, so a pair that does not overlap has inter = +-0
// and a finite denominator, hence iou = +-0 — decided without the full computation.
// For finite pairs the float32 quotient is not formed: with denom > 0, RN(inter/denom) <= thr
// exactly when inter < mid * denom, or inter == mid * denom and the tie rounds to thr (its last
// significand bit is 0), where mid is the midpoint between thr and the next float. mid has at
// most 25 significant bits and denom 24, so their product is exact in double, and so is the
// comparison.
__device__ __forceinline__ bool suppresses(float4 a, float area_a, float4 b, float area_b, const IouThr& t,
                                           bool both_finite) {
    if (both_finite && (fminf(a.z, b.z) <= fmaxf(a.x, b.x) || fminf(a.w, b.w) <= fmaxf(a.y, b.y)))
        return !(0.f <= t.thr);
    const float iw = nmax(0.f, __fsub_rn(nmin(a.z, b.z), nmax(a.x, b.x)));
    const float ih = nmax(0.f, __fsub_rn(nmin(a.w, b.w), nmax(a.y, b.y)));
    const float inter = __fmul_rn(iw, ih);
    const float denom = nmax(__fsub_rn(__fadd_rn(area_a, area_b), inter), 1e-9f);
    if (inter == 0.f && denom == denom) return !(0.f <= t.thr);  // 0 / denom is +-0
    if (both_finite) {
        const double prod = __dmul_rn(t.mid, (double)denom);
        const double in = (double)inter;
        return !(in < prod || (in == prod && t.even));
    }
    return !(__fdiv_rn(inter, denom) <= t.thr);
}

// suppresses() for two "tame" boxes (finite coordinates and a finite area), without a branch
// (a warp's lanes meet overlapping and disjoint pairs alike): a disjoint pair has inter = +0,
// and +0 < mid * denom holds exactly when 0 <= thr, the survivor test for iou = +0.
// Differences of finite values are never NaN, so plain min/max serve; and with finite areas
// the overlap's sides are at most each box's (rounding is monotonic), so inter is at most
// either area, the denominator area_a + area_b - inter is not NaN (at worst +inf), and
// np.maximum's NaN rule reduces to fmaxf there too.
// The comparison inter vs mid * denom first runs in single precision: with h = mid - thr (a
// power of two; the host sets it only where h * denom can neither underflow nor overflow, so
// hd = h * denom is exact), inter - mid * denom has the sign of D - hd where D = inter -
// thr * denom, and e = fma(-thr, denom, inter) = RN(D). RN is monotonic and hd is a float, so
// e < hd implies D < hd (survives) and e > hd implies D > hd (removed); only e == hd (a tie or
// a near-tie) and NaN take the double-precision test.
struct PairTerms {
    float inter, denom;
};
// kFloor = false leaves out the 1e-9 floor of the denominator, a no-op when area_a >= 2e-9: with
// inter <= min(area_a, area_b) (tame boxes), area_a + area_b - inter rounds to at least
// max(area_a, area_b) * (1 - 2^-22).
template <bool kFloor = true>
__device__ __forceinline__ PairTerms pair_terms(float4 a, float area_a, float4 b, float area_b) {
    const float iw = fmaxf(0.f, __fsub_rn(fminf(a.z, b.z), fmaxf(a.x, b.x)));
    const float ih = fmaxf(0.f, __fsub_rn(fminf(a.w, b.w), fmaxf(a.y, b.y)));
    const float inter = __fmul_rn(iw, ih);
    const float d = __fsub_rn(__fadd_rn(area_a, area_b), inter);
    return PairTerms{inter, kFloor ? fmaxf(d, 1e-9f) : d};
}
// The exact comparison inter vs mid * denom, in double precision.
__device__ __forceinline__ bool removes_exact(PairTerms pt, const IouThr& t) {
    const double prod = __dmul_rn(t.mid, (double)pt.denom);
    const double in = (double)pt.inter;
    return !(in < prod || (in == prod && t.even));
}
__device__ __forceinline__ bool suppresses_finite(float4 a, float area_a, float4 b, float area_b, const IouThr& t) {
    const PairTerms pt = pair_terms(a, area_a, b, area_b);
    if (t.half != 0.f) {
        const float e = __fmaf_rn(-t.thr, pt.denom, pt.inter);
        const float hd = __fmul_rn(t.half, pt.denom);
        if (e < hd) return false;
        if (e > hd) return true;
    }
    return removes_exact(pt, t);
}

// Either form, by whether both boxes are tame.
__device__ __forceinline__ bool suppresses_any(float4 a, float area_a, float4 b, float area_b, const IouThr& t,
                                               bool both_finite) {
    bool r = suppresses_finite(a, area_a, b, area_b, t);
    if (!both_finite) r = suppresses(a, area_a, b, area_b, t, false);
    return r;
}

__device__ __forceinline__ float4 load_box(const float* bx, int idx) {
    const float* q = bx + (int64_t)idx * 4;
    return make_float4(__ldg(q), __ldg(q + 1), __ldg(q + 2), __ldg(q + 3));
}

struct Smem {
    unsigned hist[256];
    unsigned long long prefix;
    unsigned kor[kWarps], kand[kWarps];  // per warp: OR and AND of the score halves of the keys the last collect appended
    int wsum[kWarps];                    // per warp: offsets of a block-wide prefix sum
    int want, done;
    int count, nkept, last, tmpn;
    float4 tbox[kTile];
    float tarea[kTile];
    int tidx[kTile];
    int tfin[kTile];
    unsigned trow[kTile];
    unsigned tsupp;
    unsigned kw[16];  // the block resolve's kept set, a word per 32 candidates
    int segn[kMaxCluster];  // class merge by pushes: each segment's kept count
    int off[kMaxClassesMerged + 1];
};

// One digit step of an MSB radix select, run by warp 0 over hist[]: finds the digit whose
// bucket holds the want-th largest key, and records whether that bucket holds exactly `want`.
__device__ __forceinline__ void radix_digit(Smem& s, uint64_t prefix, int want, int shift, int lane) {
    unsigned c[8];
    unsigned sum = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) {  // lane L owns digits 255-8L .. 248-8L (high to low)
        c[q] = s.hist[255 - 8 * lane - q];
        sum += c[q];
    }
    unsigned incl = sum;
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    const unsigned excl = incl - sum;
    const unsigned hit = __ballot_sync(0xffffffffu, excl < (unsigned)want && incl >= (unsigned)want);
    const int owner = __ffs(hit) - 1;
    if (lane == owner) {
        unsigned cum = excl;
        for (int q = 0; q < 8; ++q) {
            if (cum + c[q] >= (unsigned)want) {
                const unsigned digit = 255u - 8u * lane - q;
                s.prefix = prefix | ((uint64_t)digit << shift);
                s.want = want - (int)cum;
                s.done = c[q] == (unsigned)(want - (int)cum);  // the whole bucket is taken
                break;
            }
            cum += c[q];
        }
    }
}

// Cluster barrier halves (all threads of every CTA of the cluster take part, converged): an
// arrival without memory ordering, a wait, and a full release / acquire barrier.
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.aligned;\n\tbarrier.cluster.wait.aligned;\n" ::: "memory");
}

// Drops from the pool (keys[0, mg)) every live key below sboundary that a kept box in
// [kfrom, s.nkept) removes, setting it to kRemoved (at or above every sboundary, so no select or
// compaction takes it again). Every kept box comes before every pool key in the visiting order,
// so the greedy walk would remove that candidate too. On one CTA each thread works through its
// own keys (i = tid, tid + kThreads, ...), testing the current one against the next kept box at
// every step and moving on once one removes it or none is left, so the lanes of a warp do not
// wait for one another; the next key's box is loaded while the current one is tested. With
// replicas (nrep > 1) the batches of 32 keys are dealt over every replica's warps: a batch's
// live keys meet the kept boxes 8 at a time, one per lane of each 8-lane group, four keys per
// step, a ballot deciding each, and each removal is written into every replica's pool, between
// two cluster barriers (before: every replica is done reading its pool for the round; after:
// every removal is in place). Returns the pool's live count below sboundary. Called by every
// thread.
__device__ __forceinline__ int filter_pool_fn(uint64_t* keys, int mg, uint64_t sboundary, const float4* kbox,
                                           const float* karea, const int* kfin, int kfrom, const float* bx,
                                           const IouThr iou_thr, Smem& s, int part, int nrep, int lead_rank,
                                           cg::cluster_group cluster) {
    const int tid = threadIdx.x, lane = tid & 31;
    const int kto = s.nkept;  // kfrom < kto: every caller has a new kept box
    if (nrep > 1) {
        cluster_sync_all();  // every replica is done reading its pool for the round
        const int warp = tid >> 5, gl = lane & 7, grp = lane >> 3;
        for (int b0 = (part * kWarps + warp) * 32; b0 < mg; b0 += nrep * kWarps * 32) {
            const int i = b0 + lane;
            const uint64_t k = i < mg ? keys[i] : kRemoved;
            const float4 mb = k < sboundary ? load_box(bx, key_index(k)) : make_float4(0.f, 0.f, 0.f, 0.f);
            const float ma = box_area(mb);
            const bool mf = finite4(mb) && isfinite(ma);
            unsigned alive = __ballot_sync(0xffffffffu, k < sboundary);
            for (int c0 = kfrom; c0 < kto && alive; c0 += 8) {
                const bool kval = c0 + gl < kto;
                const float4 kb = kval ? kbox[c0 + gl] : make_float4(0.f, 0.f, 0.f, 0.f);
                const float ka = kval ? karea[c0 + gl] : 0.f;
                const bool kf = !kval || kfin[c0 + gl] != 0;
                const bool tame_k = __all_sync(0xffffffffu, kf);
                unsigned todo = alive;
                while (todo) {
                    unsigned t = todo;
                    for (int q = 0; q < grp && t; ++q) t &= t - 1;
                    const int pick = t ? __ffs(t) - 1 : -1;
                    for (int q = 0; q < 4 && todo; ++q) todo &= todo - 1;
                    const int src = pick < 0 ? 0 : pick;
                    const float4 cb = make_float4(__shfl_sync(0xffffffffu, mb.x, src), __shfl_sync(0xffffffffu, mb.y, src),
                                                  __shfl_sync(0xffffffffu, mb.z, src), __shfl_sync(0xffffffffu, mb.w, src));
                    const float ca = __shfl_sync(0xffffffffu, ma, src);
                    const bool cf = __shfl_sync(0xffffffffu, (int)mf, src) != 0;
                    bool r = false;
                    if (pick >= 0 && kval)
                        r = tame_k && cf ? suppresses_finite(kb, ka, cb, ca, iou_thr)
                                         : suppresses_any(kb, ka, cb, ca, iou_thr, kf && cf);
                    const unsigned vote = __ballot_sync(0xffffffffu, r);
#pragma unroll
                    for (int g = 0; g < 4; ++g) {
                        const int pg = __shfl_sync(0xffffffffu, pick, 8 * g);
                        if (pg >= 0 && ((vote >> (8 * g)) & 0xffu)) alive &= ~(1u << pg);
                    }
                }
            }
            if (k < sboundary && !((alive >> lane) & 1u))
                for (int q = 0; q < nrep; ++q) cluster.map_shared_rank(keys, lead_rank + q)[i] = kRemoved;
        }
    } else {
        const int stride = kThreads;
        auto next_live = [&](int i) {
            while (i < mg && keys[i] >= sboundary) i += stride;
            return i;
        };
        int mine = 0;  // keys this thread leaves live
        int i = next_live(tid);
        bool have = i < mg;
        float4 cb = have ? load_box(bx, key_index(keys[i])) : make_float4(0.f, 0.f, 0.f, 0.f);
        float ca = box_area(cb);
        bool cf = finite4(cb) && isfinite(ca);
        int nxt = have ? next_live(i + stride) : mg;
        float4 nb = nxt < mg ? load_box(bx, key_index(keys[nxt])) : make_float4(0.f, 0.f, 0.f, 0.f);
        int j = kfrom;
        while (__any_sync(0xffffffffu, have)) {
            if (have) {
                const bool r = suppresses_any(kbox[j], karea[j], cb, ca, iou_thr, cf && kfin[j]);
                ++j;
                if (r || j >= kto) {  // this key is settled
                    if (r) keys[i] = kRemoved;
                    i = nxt;
                    have = i < mg;
                    if (have) {
                        cb = nb;
                        ca = box_area(cb);
                        cf = finite4(cb) && isfinite(ca);
                        j = kfrom;
                        nxt = next_live(i + stride);
                        if (nxt < mg) nb = load_box(bx, key_index(keys[nxt]));
                    }
                }
            }
        }
    }
    if (nrep > 1) cluster_sync_all();  // every replica's removals are in place
    else __syncthreads();
    int mine = 0;  // keys this thread leaves live, over the whole pool
    for (int q = tid; q < mg; q += kThreads) mine += keys[q] < sboundary;
    const int w = __reduce_add_sync(0xffffffffu, mine);
    if (tid == 0) s.count = 0;
    __syncthreads();
    if (lane == 0 && w) atomicAdd(&s.count, w);
    __syncthreads();
    const int live = s.count;
    __syncthreads();  // every thread has read the count before anyone resets it
    return live;
}

// Whether dropping what `fresh` new kept boxes remove from a pool of `live` keys is likely to
// save more work than it costs. A round of `used` candidates kept `fresh`: the rest of the pool is
// taken to be removed at the round's rate. Walking a candidate costs a tile's share (about 200
// pair tests' time); the filter tests a removed key a few times and a live one against every
// new kept box; and the walk would visit about `needed` / keep rate more candidates.
__device__ __forceinline__ bool filter_pays(int live, int fresh, int used, int needed) {
    if (fresh <= 0 || live <= 0 || needed <= 0) return false;
    const float keep = fminf(1.f, (float)fresh / (float)max(used, 1));
    const float removed = 1.f - keep;
    const float visits = fminf((float)needed / keep, (float)live);
    const float cost = (float)live * (keep * (float)fresh + removed * 5.f);
    const float saved = visits * removed * 200.f;
    return saved > cost;
}


// kReplicas: the launch's helpers may stay as replicas (clusters of one segment with helpers);
// without it the replica paths are compiled out of the kernel.
template <bool kReplicas>
__global__ void __launch_bounds__(kThreads, 1) nms_kernel(const __grid_constant__ NmsParams p) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint64_t* keys = reinterpret_cast<uint64_t*>(smem_raw);     // [kCap] eligible keys
    uint64_t* sbuf = keys + kCap;                                 // [kSort] sorted round
    float4* cbox = reinterpret_cast<float4*>(sbuf + kSort);       // [kSort] their boxes
    float* carea = reinterpret_cast<float*>(cbox + kSort);        // [kSort]
    int* cfin = reinterpret_cast<int*>(carea + kSort);            // [kSort] tame: finite coordinates and area
    float4* kbox = reinterpret_cast<float4*>(cfin + kSort);       // [max_det] kept boxes
    uint64_t* kkey = reinterpret_cast<uint64_t*>(kbox + p.max_det);  // [max_det] their keys
    float* karea = reinterpret_cast<float*>(kkey + p.max_det);
    int* kfin = reinterpret_cast<int*>(karea + p.max_det);
    unsigned* mask = reinterpret_cast<unsigned*>(kfin + p.max_det);  // [kSort, kMaskStride] when block_cap
    unsigned* bstart = mask + kSort * kMaskStride;  // [kBuckets] bucket counts, then starts (when block_cap)
    unsigned* bcur = bstart + kBuckets;             // [kBuckets] scatter cursors (when block_cap)
    uint64_t* mrecv = reinterpret_cast<uint64_t*>(bcur + kBuckets);  // [kRecvKeys] (when block_cap)
    __shared__ Smem s;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int part = blockIdx.x % p.split;  // 0: the segment's leader; else a helper of its block resolve
    const int seg = blockIdx.x / p.split;
    cg::cluster_group cluster = cg::this_cluster();
    // Helpers of a cluster that holds one segment stay to the end as replicas: they take every
    // step the leader takes, on the same data, so they hold the same pool and kept set, and share
    // the work of the block's pair tests and of dropping removed keys from the pool (each writes
    // its results into every replica); only the leader writes the output. In a cluster of several
    // segments (the class merge) helpers leave after the block, since the segments' later rounds
    // differ and the cluster barriers the replicas need would not match.
    const bool replicas = kReplicas && p.split > 1 && !p.cluster;
    const int nrep = replicas ? p.split : 1;
    const int lead_rank = (int)cluster.block_rank() - part;
    // With helpers, every CTA passes the cluster barrier twice around the block resolve (or, if its
    // segment never gets there, just before the output): the first arrival is here, so that the
    // wait before the first store into another CTA's shared memory knows the cluster is running.
    if (p.split > 1) cluster_arrive_relaxed();
    bool block_done = false;   // this CTA has passed the block resolve's cluster barriers
    bool helper_exit = false;  // a helper whose share of the block is done
    // Launched as a programmatic dependent of the stream's previous kernel: boxes, scores and
    // classes are read only after it has completed.
    griddep_wait();
    griddep_launch_dependents();
    const int img = seg / p.segs;
    const int cls = seg - img * p.segs;
    const int n = p.n;
    const float* sc = p.scores + (int64_t)img * n;
    const int32_t* cl = p.classes ? p.classes + (int64_t)img * n : nullptr;
    const float* bx = p.boxes + (int64_t)img * n * 4;
    const float score_thr = p.score_thr;
    const IouThr iou_thr{p.iou_thr, p.iou_mid, p.iou_even != 0, p.iou_half};
    const bool aware = p.class_aware != 0;

    // Exclusive prefix sum of `mine` over the block, in thread order; s.count gets the total.
    // Two barriers; every thread calls it, and reads s.count before the next call.
    auto block_offset = [&](int mine) -> int {
        int incl = mine;  // inclusive prefix sum of the warp's counts
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        if (lane == 31) s.wsum[warp] = incl;
        __syncthreads();
        if (warp == 0) {  // the warps' totals, scanned
            const int t = s.wsum[lane];
            int wi = t;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int u = __shfl_up_sync(0xffffffffu, wi, o);
                if (lane >= o) wi += u;
            }
            s.wsum[lane] = wi - t;
            if (lane == 31) s.count = wi;
        }
        __syncthreads();
        return s.wsum[warp] + incl - mine;
    };

    int bucket_shift = -1;  // the last collect counted its keys into buckets by this shift (-1: none)

    // Append the keys of candidates in [floor_key, boundary) to keys[] in any order; returns
    // how many there are (only the first kCap are stored). In steps of kScanGroups x kThreads
    // groups of four candidates: every thread loads its groups' scores (and classes) at once,
    // counts its keys, and one block-wide prefix sum places them (no shared counter that the
    // warps would take in turn). With `bucket` (the first collect of a segment that has a block
    // resolve, all its candidates in one step) it also counts the keys into kBuckets buckets by
    // the kBucketBits bits below the score bits they all share, and sets bucket_shift.
    auto collect = [&](uint64_t boundary, uint64_t floor_key, bool bucket) -> int {
        const int groups = (n + 3) >> 2;
        bucket = bucket && p.block_cap > 0 && groups <= kScanGroups * kThreads;
        bucket_shift = -1;
        if (bucket) {
            bstart[tid] = 0;
            bstart[tid + kThreads] = 0;
        }
        unsigned kor = 0, kand = ~0u;  // this thread's appended keys: the score bits they all share
        auto fetch = [&](int g, float4& v, int4& c) {
            v = make_float4(0.f, 0.f, 0.f, 0.f);
            c = make_int4(0, 0, 0, 0);
            if (g >= groups) return;
            if (p.vec) {
                v = __ldg(reinterpret_cast<const float4*>(sc) + g);
                if (aware) c = __ldg(reinterpret_cast<const int4*>(cl) + g);
            } else {
                const int i0 = g * 4;
                if (i0 < n) { v.x = __ldg(sc + i0); if (aware) c.x = __ldg(cl + i0); }
                if (i0 + 1 < n) { v.y = __ldg(sc + i0 + 1); if (aware) c.y = __ldg(cl + i0 + 1); }
                if (i0 + 2 < n) { v.z = __ldg(sc + i0 + 2); if (aware) c.z = __ldg(cl + i0 + 2); }
                if (i0 + 3 < n) { v.w = __ldg(sc + i0 + 3); if (aware) c.w = __ldg(cl + i0 + 3); }
            }
        };
        // candidate e of a group: taken when eligible (score, class) and, for a bounded collect,
        // its key is in [floor_key, boundary). The first collect of a segment has no bounds, so
        // its count needs no keys; keys are formed once, for the taken candidates only.
        const bool bounded = boundary != ~0ull || floor_key != 0;
        auto taken = [&](int g, const float4& v, const int4& c, int e) -> bool {
            const float sv = e == 0 ? v.x : e == 1 ? v.y : e == 2 ? v.z : v.w;
            const int cv = e == 0 ? c.x : e == 1 ? c.y : e == 2 ? c.z : c.w;
            const int i = g * 4 + e;
            bool t = g < groups && i < n && sv >= score_thr && (!aware || cv == cls);
            if (bounded && t) {
                const uint64_t k = cand_key(sv, i);
                t = k < boundary && k >= floor_key;
            }
            return t;
        };
        int total = 0;  // keys found in earlier steps (the same in every thread)
        for (int g0 = 0; g0 < groups; g0 += kScanGroups * kThreads) {
            float4 v[kScanGroups];
            int4 c[kScanGroups];
#pragma unroll
            for (int q = 0; q < kScanGroups; ++q) fetch(g0 + q * kThreads + tid, v[q], c[q]);
            unsigned tmask = 0;  // bit 4q + e: candidate e of group q is taken
#pragma unroll
            for (int q = 0; q < kScanGroups; ++q)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const bool t = taken(g0 + q * kThreads + tid, v[q], c[q], e);
                    tmask |= (unsigned)t << (4 * q + e);
                    if (t) {
                        const unsigned o = score_ord(e == 0 ? v[q].x : e == 1 ? v[q].y : e == 2 ? v[q].z : v[q].w);
                        kor |= o;
                        kand &= o;
                    }
                }
            int shift = 0;
            if (bucket) {  // the score bits every key shares, before the prefix sum's barriers
                const unsigned wor = __reduce_or_sync(0xffffffffu, kor);
                const unsigned wand = __reduce_and_sync(0xffffffffu, kand);
                if (lane == 0) {
                    s.kor[warp] = wor;
                    s.kand[warp] = wand;
                }
            }
            int pos = total + block_offset(__popc(tmask));
            if (bucket) {
                const unsigned diff = __reduce_or_sync(0xffffffffu, s.kor[lane]) ^
                                      __reduce_and_sync(0xffffffffu, s.kand[lane]);
                // highest key bit where keys may differ: in the score half, or (one score for all)
                // among the index bits, ~index for index < n differing only below n - 1's top bit
                const int top = diff ? 63 - __clz((int)diff) : (n > 1 ? 31 - __clz(n - 1) : 0);
                shift = max(top + 1 - kBucketBits, 0);
                bucket_shift = shift;
            }
#pragma unroll
            for (int q = 0; q < kScanGroups; ++q)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    if ((tmask >> (4 * q + e)) & 1u) {
                        const float sv = e == 0 ? v[q].x : e == 1 ? v[q].y : e == 2 ? v[q].z : v[q].w;
                        const uint64_t k = cand_key(sv, (g0 + q * kThreads + tid) * 4 + e);
                        if (pos < kCap) keys[pos] = k;
                        ++pos;
                        if (bucket) atomicAdd(&bstart[(unsigned)(k >> shift) & (kBuckets - 1)], 1u);
                    }
                }
            total += s.count;
            __syncthreads();  // every thread has read wsum and count before the next step rewrites them
        }
        {
            const unsigned wor = __reduce_or_sync(0xffffffffu, kor);
            const unsigned wand = __reduce_and_sync(0xffffffffu, kand);
            if (lane == 0) {
                s.kor[warp] = wor;
                s.kand[warp] = wand;
            }
        }
        __syncthreads();
        return total;
    };

    // The want-th largest key of a set, by an exact MSB radix select: returns a floor such that
    // exactly `want` keys of the set are >= it. for_keys(f) calls f(k) for every key of the set (a
    // subset of the last collect's keys). The digits start below the score bits those keys all
    // share (with one score for all, at the index half's top): any start whose higher bits are
    // common to the set gives the same floor.
    auto radix_select = [&](int want, auto&& for_keys) -> uint64_t {
        // every warp reduces the per-warp words itself: no barrier
        const unsigned all_or = __reduce_or_sync(0xffffffffu, s.kor[lane]);
        const unsigned all_and = __reduce_and_sync(0xffffffffu, s.kand[lane]);
        const unsigned diff = all_or ^ all_and;
        const int top = diff ? 63 - __clz((int)diff) : 31;  // the highest key bit where keys may differ
        const uint64_t low = top >= 63 ? ~0ull : ((1ull << (top + 1)) - 1);
        uint64_t prefix = ((uint64_t)all_and << 32) & ~low;
        int width = min(8, top + 1), shift = top + 1 - width;
        for (;;) {
            if (tid < 256) s.hist[tid] = 0;
            __syncthreads();
            const int hi = shift + width;
            const unsigned dmask = (1u << width) - 1u;
            for_keys([&](uint64_t k) {
                if (hi < 64 && (k >> hi) != (prefix >> hi)) return;
                atomicAdd(&s.hist[(unsigned)(k >> shift) & dmask], 1u);
            });
            __syncthreads();
            if (warp == 0) radix_digit(s, prefix, want, shift, lane);
            __syncthreads();
            prefix = s.prefix;
            want = s.want;
            if (s.done || shift == 0) break;  // done: the bucket is taken whole, its lower bits are free
            width = min(8, shift);
            shift -= width;
        }
        return prefix;
    };

    auto filter_pool = [&](int kfrom, int mg, uint64_t sboundary) -> int {
        bucket_shift = -1;  // the bucket counts no longer match the pool
        return filter_pool_fn(keys, mg, sboundary, kbox, karea, kfin, kfrom, bx, iou_thr, s, part, nrep, lead_rank,
                              cluster);
    };

    // Counts the pool's live keys (below sboundary) into the buckets, by the bits below the score
    // bits they all share, as the scan does for a segment's first round; sets bucket_shift.
    auto bucket_count = [&](int mg, uint64_t sboundary) {
        unsigned o = 0, a = ~0u;
        for (int i = tid; i < mg; i += kThreads) {
            const uint64_t k = keys[i];
            if (k < sboundary) {
                o |= (unsigned)(k >> 32);
                a &= (unsigned)(k >> 32);
            }
        }
        bstart[tid] = 0;
        bstart[tid + kThreads] = 0;
        o = __reduce_or_sync(0xffffffffu, o);
        a = __reduce_and_sync(0xffffffffu, a);
        if (lane == 0) {
            s.kor[warp] = o;
            s.kand[warp] = a;
        }
        __syncthreads();
        const unsigned diff = __reduce_or_sync(0xffffffffu, s.kor[lane]) ^ __reduce_and_sync(0xffffffffu, s.kand[lane]);
        const int top = diff ? 63 - __clz((int)diff) : (n > 1 ? 31 - __clz(n - 1) : 0);
        const int shift = max(top + 1 - kBucketBits, 0);
        for (int i = tid; i < mg; i += kThreads) {
            const uint64_t k = keys[i];
            if (k < sboundary) atomicAdd(&bstart[(unsigned)(k >> shift) & (kBuckets - 1)], 1u);
        }
        __syncthreads();
        bucket_shift = shift;
    };

    // The first round from the scan's bucket counts: the `want` largest keys of the pool
    // keys[0, mg), in descending order, into sbuf. A bucket's keys all share the bits above its
    // digit, so buckets in descending digit order hold the keys in descending order: a prefix sum
    // over the counts gives each bucket's first position, the keys of the buckets that start
    // below `want` are scattered to their bucket's range (any order within it), and each key's
    // place is its bucket's start plus the count of its bucket's keys above it. Returns false,
    // leaving sbuf untouched, when a needed bucket holds more than kBucketMax keys.
    auto bucket_round = [&](int want, int mg, uint64_t sboundary) -> bool {
        const int d0 = kBuckets - 1 - 2 * tid, d1 = d0 - 1;  // this thread's two digits, high first
        const int c0 = (int)bstart[d0], c1 = (int)bstart[d1];
        const int st0 = block_offset(c0 + c1), st1 = st0 + c0;
        const bool bad = (st0 < want && c0 > kBucketMax) || (st1 < want && c1 > kBucketMax);
        // the bucket holding position want - 1 ends the scattered keys
        if (c0 > 0 && st0 < want && want <= st0 + c0) s.tmpn = st0 + c0;
        if (c1 > 0 && st1 < want && want <= st1 + c1) s.tmpn = st1 + c1;
        bstart[d0] = st0;  // every count was read before block_offset's barriers
        bstart[d1] = st1;
        bcur[d0] = st0;
        bcur[d1] = st1;
        if (__syncthreads_or(bad)) return false;
        uint64_t* tmp = reinterpret_cast<uint64_t*>(cbox);  // free until the gather
        const int shift = bucket_shift;
        for (int i = tid; i < mg; i += kThreads) {
            const uint64_t k = keys[i];
            const unsigned d = (unsigned)(k >> shift) & (kBuckets - 1);
            if (k < sboundary && (int)bstart[d] < want) tmp[atomicAdd(&bcur[d], 1u)] = k;
        }
        __syncthreads();
        if (tid < s.tmpn) {  // at most want + kBucketMax keys
            const uint64_t k = tmp[tid];
            const unsigned d = (unsigned)(k >> shift) & (kBuckets - 1);
            const int b0 = (int)bstart[d], b1 = (int)bcur[d];
            int r = 0;
            for (int i = b0; i < b1; ++i) r += tmp[i] > k;
            if (b0 + r < want) sbuf[b0 + r] = k;
        }
        __syncthreads();
        return true;
    };

    if (tid == 0) s.nkept = 0;
    int visited = 0;             // candidates consumed by rounds so far
    uint64_t gboundary = ~0ull;  // unvisited candidates outside shared memory: keys below this
    for (;;) {
        const int m = collect(gboundary, 0, true);
        if (m == 0 || s.nkept >= p.max_det) break;
        int mg = m;
        uint64_t pool_floor = 0;  // the pool holds every eligible key in [pool_floor, gboundary)
        if (m > kCap) {
            // the kCap largest keys below gboundary, by an exact radix select over global memory
            const uint64_t prefix = radix_select(kCap, [&](auto&& f) {
                if (p.vec) {  // four candidates per 16-byte load, as the scan reads them
                    for (int g = tid; g < (n >> 2); g += kThreads) {
                        const float4 v = __ldg(reinterpret_cast<const float4*>(sc) + g);
                        const int4 c = aware ? __ldg(reinterpret_cast<const int4*>(cl) + g) : make_int4(cls, cls, cls, cls);
                        const float vv[4] = {v.x, v.y, v.z, v.w};
                        const int cc[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            if (!(vv[e] >= score_thr) || cc[e] != cls) continue;
                            const uint64_t k = cand_key(vv[e], 4 * g + e);
                            if (k < gboundary) f(k);
                        }
                    }
                    return;
                }
                for (int i = tid; i < n; i += kThreads) {
                    const float v = __ldg(sc + i);
                    if (!(v >= score_thr) || (aware && __ldg(cl + i) != cls)) continue;
                    const uint64_t k = cand_key(v, i);
                    if (k < gboundary) f(k);
                }
            });
            mg = min(collect(gboundary, prefix, false), kCap);
            pool_floor = prefix;
        }

        // ---- rounds over the keys held in shared memory. A key that a kept box removes is set
        // to kRemoved (filter_pool); the live keys are those below sboundary.
        uint64_t sboundary = ~0ull;
        int live = mg;
        // a later pool: what the boxes kept so far remove, when that pays (rates over all visits)
        if (s.nkept > 0 && filter_pays(live, s.nkept, visited, p.max_det - s.nkept))
            live = filter_pool(0, mg, sboundary);
        while (live > 0 && s.nkept < p.max_det) {
            const int remaining = live;
            const int K0 = s.nkept;
            // the scan's buckets, when it counted this pool and a needed bucket is small; else an
            // exact radix select of the round, its compaction and a sort
            int cs = 0;
            // a later round of more than two warp runs: count the live keys into the buckets first
            if (bucket_shift < 0 && p.block_cap > 0 && remaining > 64) bucket_count(mg, sboundary);
            const bool from_buckets = bucket_shift >= 0 && bucket_round(min(remaining, kSort), mg, sboundary);
            bucket_shift = -1;
            if (from_buckets) {
                cs = min(remaining, kSort);
            } else {
                uint64_t floor_key = 0;
                if (remaining > kSort) {
                    floor_key = radix_select(kSort, [&](auto&& f) {
                        for (int i = tid; i < mg; i += kThreads) {
                            const uint64_t k = keys[i];
                            if (k < sboundary) f(k);
                        }
                    });
                }
                // compact the round: keys in [floor_key, sboundary), placed by one block-wide prefix sum
                {
                    int mine = 0;
                    for (int i = tid; i < mg; i += kThreads) {
                        const uint64_t k = keys[i];
                        mine += k < sboundary && k >= floor_key;
                    }
                    int pos = block_offset(mine);
                    for (int i = tid; i < mg; i += kThreads) {
                        const uint64_t k = keys[i];
                        if (k < sboundary && k >= floor_key) {
                            if (pos < kSort) sbuf[pos] = k;
                            ++pos;
                        }
                    }
                }
                __syncthreads();
                cs = min(s.count, kSort);
                if (cs == 0) break;  // unreachable while keys remain; keeps the walk below in range

                // ---- sort the round descending. Each warp sorts a run of 32 keys with a bitonic
                // network over shuffles; then runs merge pairwise, level by level: a key's place in
                // the merged pair is its place in its own run plus the count of keys above it in the
                // partner run (a binary search). Keys are distinct and real keys nonzero; the zero
                // padding sits at the end of the last run, and a run with no partner (past P) is
                // copied as it is.
                const int P = (cs + 31) & ~31;  // whole warps: a warp is either all in or all out
                uint64_t v = tid < cs ? sbuf[tid] : 0;
                if (tid < P) {
                    for (int k = 2; k <= 32; k <<= 1) {
                        for (int j = k >> 1; j > 0; j >>= 1) {
                            const uint32_t lo = __shfl_xor_sync(0xffffffffu, (uint32_t)v, j);
                            const uint32_t hi = __shfl_xor_sync(0xffffffffu, (uint32_t)(v >> 32), j);
                            const uint64_t w = ((uint64_t)hi << 32) | lo;
                            const bool keep_max = ((lane & j) == 0) == ((lane & k) == 0);
                            v = keep_max ? (v > w ? v : w) : (v < w ? v : w);
                        }
                    }
                }
                __syncthreads();  // every key has been read before the runs are written back
                if (tid < P) sbuf[tid] = v;
                __syncthreads();
                {
                    uint64_t* src = sbuf;
                    uint64_t* dst = reinterpret_cast<uint64_t*>(cbox);  // free until the gather below
                    for (int L = 32; L < P; L <<= 1) {  // runs of L keys merge into runs of 2L
                        if (tid < P) {
                            const int r = tid / L, in_run = tid - r * L;
                            const int pair = (r >> 1) * 2 * L;
                            const int partner = (r ^ 1) * L;
                            const int plen = max(0, min(L, P - partner));  // 0: no partner run
                            const uint64_t key = src[tid];
                            int lo = 0, hi = plen;  // partner run is descending: count its keys above key
                            while (lo < hi) {
                                const int mid = (lo + hi) >> 1;
                                if (src[partner + mid] > key) lo = mid + 1;
                                else hi = mid;
                            }
                            dst[pair + in_run + lo] = key;
                        }
                        __syncthreads();
                        uint64_t* t = src;
                        src = dst;
                        dst = t;
                    }
                    if (src != sbuf) {
                        if (tid < P) sbuf[tid] = src[tid];
                        __syncthreads();
                    }
                }
            }

            // ---- the round's boxes, in one round of gathers
            for (int q = tid; q < cs; q += kThreads) {
                const float4 b = load_box(bx, key_index(sbuf[q]));
                cbox[q] = b;
                carea[q] = box_area(b);
                cfin[q] = finite4(b) && isfinite(carea[q]);  // tame: suppresses_finite's form applies
            }
            __syncthreads();

            // ---- block resolve of the first M candidates while nothing is kept yet. Every pair's
            // suppression bit goes into shared memory as columns (candidate b: the earlier
            // candidates of each 32-word that would remove it), computed in one pass by all warps of
            // the segment's CTAs (helpers store theirs into the leader's shared memory across the
            // cluster); then the leader settles the greedy choice over the columns in parallel. The
            // columns hold exactly the tests the walk below would make, so the kept set is the
            // walk's. The round consumes its first M candidates; the rest stay in the pool.
            int used = cs;
            if (p.block_cap > 0 && s.nkept == 0 && !block_done) {
                const int M = min(cs, p.block_cap);
                const int W = (M + 31) >> 5;
                // every candidate tame: suppresses_finite alone decides each pair
                const bool tame = __syncthreads_and(tid >= M || cfin[tid]) != 0;
                // helpers store their columns into the leader's; replicas each into their own, and
                // after the barrier each takes the others' from them
                unsigned* cmask = mask;
                if (p.split > 1) {
                    cluster_wait();  // the kernel-entry arrival: every CTA of the cluster is running
                    if (!replicas) cmask = cluster.map_shared_rank(mask, lead_rank);
                }
                auto put = [&](int idx, unsigned w) { cmask[idx] = w; };
                // the pairs (u, b), b in [32u, M), u-major, P of them; warp g of the segment's
                // split x kWarps takes the g-th of equal contiguous shares
                const int P = W * M - 16 * W * (W - 1);
                const int G = p.split * kWarps, g = part * kWarps + warp;
                int off = (int)((long long)P * g / G);
                int left = (int)((long long)P * (g + 1) / G) - off;
                int u = 0;
                while (u < W && off >= M - 32 * u) {
                    off -= M - 32 * u;
                    ++u;
                }
                while (left > 0) {
                    const int a = 32 * u + lane;  // this lane's remover: candidate a of word u
                    const bool ain = a < M;
                    const float4 ab = ain ? cbox[a] : make_float4(0.f, 0.f, 0.f, 0.f);
                    const float aa = ain ? carea[a] : 0.f;
                    const bool af = ain && cfin[a];
                    const int run = min(left, M - 32 * u - off);
                    const int b0 = 32 * u + off;
                    int i = 0;
                    if (tame && iou_thr.half != 0.f) {
                        // four candidates at a time, branch-free: suppresses_finite's single-precision
                        // decision for all four, and its double-precision one only where a lane of the
                        // warp meets a tie or near-tie. Past this word's own candidates every lane's
                        // remover comes first (a < b needs no test); the denominator's floor is left
                        // out when every lane's remover has an area of at least 2e-9.
                        auto four = [&](auto diag, auto floor, int limit) {
                            for (; i + 4 <= limit; i += 4) {
                                PairTerms pt[4];
                                bool r[4], tie = false;
#pragma unroll
                                for (int j = 0; j < 4; ++j) {
                                    const int b = b0 + i + j;
                                    pt[j] = pair_terms<decltype(floor)::value>(ab, aa, cbox[b], carea[b]);
                                    const float e = __fmaf_rn(-iou_thr.thr, pt[j].denom, pt[j].inter);
                                    const float hd = __fmul_rn(iou_thr.half, pt[j].denom);
                                    r[j] = e > hd;
                                    tie |= !(e < hd) && !(e > hd);
                                }
                                if (__any_sync(0xffffffffu, tie)) {
#pragma unroll
                                    for (int j = 0; j < 4; ++j) {
                                        const float e = __fmaf_rn(-iou_thr.thr, pt[j].denom, pt[j].inter);
                                        const float hd = __fmul_rn(iou_thr.half, pt[j].denom);
                                        if (!(e < hd) && !(e > hd)) r[j] = removes_exact(pt[j], iou_thr);
                                    }
                                }
                                unsigned w4[4];
#pragma unroll
                                for (int j = 0; j < 4; ++j)
                                    w4[j] = __ballot_sync(0xffffffffu, r[j] && (!decltype(diag)::value || a < b0 + i + j));
                                if (lane == 0) {
#pragma unroll
                                    for (int j = 0; j < 4; ++j) put((b0 + i + j) * kMaskStride + u, w4[j]);
                                }
                            }
                        };
                        using yes = std::true_type;
                        using no = std::false_type;
                        const int diag_end = min(run, 32 * (u + 1) - b0 + 3);  // groups reaching into word u
                        four(yes{}, yes{}, diag_end);
                        if (__all_sync(0xffffffffu, aa >= 2e-9f)) four(no{}, no{}, run);
                        else four(no{}, yes{}, run);
                    }
                    for (; i < run; ++i) {
                        const int b = b0 + i;
                        bool r = tame ? suppresses_finite(ab, aa, cbox[b], carea[b], iou_thr)
                                      : suppresses_any(ab, aa, cbox[b], carea[b], iou_thr, af && cfin[b]);
                        r = r && a < b;
                        const unsigned word = __ballot_sync(0xffffffffu, r);
                        if (lane == 0) put(b * kMaskStride + u, word);
                    }
                    left -= run;
                    ++u;
                    off = 0;
                }
                if (p.split > 1) cluster_sync_all();  // the helpers' columns are in place
                else __syncthreads();
                if (replicas) {
                    // the words other replicas computed: pair e of the u-major order (word u of
                    // column b) is warp gw's when P * gw / G <= e < P * (gw + 1) / G, and warp gw is
                    // replica gw / kWarps's
                    for (int e = tid; e < P; e += kThreads) {
                        int gw = (int)((long long)e * G / P);
                        while (gw > 0 && (long long)P * gw / G > e) --gw;
                        while (gw + 1 < G && (long long)P * (gw + 1) / G <= e) ++gw;
                        const int owner = gw / kWarps;
                        if (owner == part) continue;
                        int uu = 0, rem = e;
                        while (rem >= M - 32 * uu) {
                            rem -= M - 32 * uu;
                            ++uu;
                        }
                        const int idx = (32 * uu + rem) * kMaskStride + uu;
                        mask[idx] = cluster.map_shared_rank(mask, lead_rank + owner)[idx];
                    }
                    // every replica has read what it needs before any leaves the block or changes it
                    cluster_sync_all();
                }
                block_done = true;
                if (part != 0 && !replicas) {  // a helper: its share is done
                    helper_exit = true;
                    break;
                }
                // The greedy set: b is kept exactly when no kept a < b removes it. From "all kept",
                // each pass recomputes every candidate from the previous pass's set. A candidate
                // whose removers are all settled is settled one pass later, so the passes reach the
                // greedy set (the only fixed point: removal only runs forward) after the longest
                // chain of removals, and stop at the first pass that changes nothing.
                if (tid < 16)
                    s.kw[tid] = tid >= W ? 0u : ((tid == W - 1 && (M & 31)) ? (1u << (M & 31)) - 1u : 0xffffffffu);
                __syncthreads();
                bool settled = false;
                for (int pass = 0; pass < kMaxPasses; ++pass) {
                    unsigned hit = 0;
                    if (tid < M) {
#pragma unroll
                        for (int uu = 0; uu < 16; ++uu)
                            if (uu <= warp) hit |= mask[tid * kMaskStride + uu] & s.kw[uu];
                    }
                    const unsigned nk = __ballot_sync(0xffffffffu, tid < M && hit == 0);
                    const bool changed = warp < W && nk != s.kw[warp];
                    __syncthreads();  // every read of kw is done
                    if (warp < W && lane == 0) s.kw[warp] = nk;
                    if (!__syncthreads_or(changed)) {
                        settled = true;
                        break;
                    }
                }
                if (!settled) {
                    // long chains: warp 0 settles word after word; inside a word the same passes,
                    // which settle 32 candidates in at most 33
                    if (warp == 0) {
                        unsigned kw = 0;  // lane c: the settled word c
                        for (int c = 0; c < W; ++c) {
                            const int b = 32 * c + lane;
                            const bool bin = b < M;
                            unsigned hit = 0;
                            for (int uu = 0; uu < c; ++uu) {
                                const unsigned k = __shfl_sync(0xffffffffu, kw, uu);
                                if (bin) hit |= mask[b * kMaskStride + uu] & k;
                            }
                            const unsigned diag = bin ? mask[b * kMaskStride + c] : 0u;
                            const unsigned alive = __ballot_sync(0xffffffffu, bin && hit == 0);
                            unsigned k = alive;
                            for (int it = 0; it < 34; ++it) {
                                const unsigned nk = __ballot_sync(0xffffffffu, ((alive >> lane) & 1u) && (diag & k) == 0);
                                if (nk == k) break;
                                k = nk;
                            }
                            if (lane == c) kw = k;
                        }
                        if (lane < 16) s.kw[lane] = kw;
                    }
                    __syncthreads();
                }
                // the first max_det of the greedy set, in order
                if (tid < M && ((s.kw[warp] >> lane) & 1u)) {
                    int pos = __popc(s.kw[warp] & ((1u << lane) - 1u));
#pragma unroll
                    for (int uu = 0; uu < 16; ++uu)
                        if (uu < warp) pos += __popc(s.kw[uu]);
                    if (pos < p.max_det) {
                        kbox[pos] = cbox[tid];
                        karea[pos] = carea[tid];
                        kkey[pos] = sbuf[tid];
                        kfin[pos] = cfin[tid];
                    }
                }
                if (warp == 0) {
                    const int total = __reduce_add_sync(0xffffffffu, lane < W ? __popc(s.kw[lane]) : 0);
                    if (lane == 0) s.nkept = min(total, p.max_det);
                }
                used = M;
            }

            // ---- greedy walk, a tile of 32 candidates at a time: candidates are read in place;
            // two barriers per tile (after the checks, after the keeps)
            if (tid == 0) s.tsupp = 0;
            __syncthreads();
            for (int base = 0; used == cs && base < cs; base += kTile) {
                const int K = s.nkept;
                if (K >= p.max_det) break;
                const int cnt = min(kTile, cs - base);
                // against every box kept so far: warp w takes kept boxes w, w+32, ..., four at a time
                bool sup = false;
                if (lane < cnt) {
                    const int q = base + lane;
                    const float4 me = cbox[q];
                    const float ma = carea[q];
                    const bool mf = cfin[q];
                    int j = warp;
                    for (; j + 3 * kWarps < K && !sup; j += 4 * kWarps) {
                        const bool s0 = suppresses_any(kbox[j], karea[j], me, ma, iou_thr, mf && kfin[j]);
                        const bool s1 = suppresses_any(kbox[j + kWarps], karea[j + kWarps], me, ma, iou_thr,
                                                       mf && kfin[j + kWarps]);
                        const bool s2 = suppresses_any(kbox[j + 2 * kWarps], karea[j + 2 * kWarps], me, ma,
                                                       iou_thr, mf && kfin[j + 2 * kWarps]);
                        const bool s3 = suppresses_any(kbox[j + 3 * kWarps], karea[j + 3 * kWarps], me, ma,
                                                       iou_thr, mf && kfin[j + 3 * kWarps]);
                        sup = s0 | s1 | s2 | s3;
                    }
                    for (; j < K && !sup; j += kWarps)
                        sup = suppresses_any(kbox[j], karea[j], me, ma, iou_thr, mf && kfin[j]);
                }
                const unsigned bal = __ballot_sync(0xffffffffu, sup);
                if (lane == 0 && bal) atomicOr(&s.tsupp, bal);
                // inside the tile: row w = the later candidates that candidate w would remove
                if (warp < cnt) {
                    bool s2 = false;
                    if (lane > warp && lane < cnt) {
                        const int a = base + warp, b = base + lane;
                        s2 = suppresses_any(cbox[a], carea[a], cbox[b], carea[b], iou_thr, cfin[a] && cfin[b]);
                    }
                    const unsigned row = __ballot_sync(0xffffffffu, s2);
                    if (lane == 0) s.trow[warp] = row;
                }
                __syncthreads();
                if (warp == 0) {
                    const unsigned valid = cnt == 32 ? 0xffffffffu : ((1u << cnt) - 1u);
                    unsigned alive = valid & ~s.tsupp;
                    const unsigned myrow = lane < cnt ? s.trow[lane] : 0u;
                    // only candidates that would remove a later live one need visiting, in order
                    unsigned todo = __ballot_sync(0xffffffffu, ((alive >> lane) & 1u) && (myrow & alive));
                    while (todo) {
                        const int i = __ffs(todo) - 1;
                        todo &= todo - 1;
                        const unsigned row_i = __shfl_sync(0xffffffffu, myrow, i);
                        if ((alive >> i) & 1u) {  // final: only earlier candidates remove it
                            alive &= ~row_i;
                            todo &= alive;
                        }
                    }
                    // keep the first `room` live candidates, in order
                    const int room = p.max_det - K;
                    unsigned kept = alive;
                    if (__popc(kept) > room) {
                        for (int c = __popc(kept) - room; c > 0; --c) kept &= ~(1u << (31 - __clz(kept)));
                    }
                    if ((kept >> lane) & 1u) {
                        const int pos = K + __popc(kept & ((1u << lane) - 1u));
                        const int q = base + lane;
                        kbox[pos] = cbox[q];
                        karea[pos] = carea[q];
                        kkey[pos] = sbuf[q];
                        kfin[pos] = cfin[q];
                    }
                    if (lane == 0) {
                        s.nkept = K + __popc(kept);
                        s.tsupp = 0;
                    }
                }
                __syncthreads();
            }
            live -= used;
            sboundary = sbuf[used - 1];
            __syncthreads();
            // a round that kept at most half its candidates: what its kept boxes remove is likely a
            // large part of the pool too, so drop it before the next round's select
            const int kept_now = s.nkept - K0;
            visited += used;
            if (s.nkept < p.max_det && filter_pays(live, kept_now, used, p.max_det - s.nkept))
                live = filter_pool(K0, mg, sboundary);
        }
        if (helper_exit || mg == m || s.nkept >= p.max_det) break;
        gboundary = pool_floor;  // the pool's keys are all visited or removed
        __syncthreads();
    }
    __syncthreads();
    if (p.split > 1 && !block_done) {  // the block resolve's two cluster barriers, if not passed yet
        cluster_wait();
        cluster_sync_all();
    }
    const int nkept = s.nkept;

    if (!aware) {
        if (part != 0) return;
        int64_t* out = p.keep + (int64_t)img * p.max_det;
        for (int i = tid; i < p.max_det; i += kThreads) out[i] = i < nkept ? key_index(kkey[i]) : -1;
        if (tid == 0) p.counts[img] = nkept;
        return;
    }

    // ---- class-aware. In a cluster (an image's segments, one CTA each): every CTA's survivors
    // stay in its shared memory, and after the cluster barrier CTA 0 merges them through
    // distributed shared memory; a second barrier keeps the others resident until it has read
    // them. No global publish, no arrival counter, nothing to clear between calls.
    const int first = img * p.segs;
    int64_t* out = p.keep + (int64_t)img * p.max_det;
    if (p.cluster) {
        // With room in the first leader's receive area, every segment leader stores its kept keys
        // and count there before the barrier, and the merge reads them locally; otherwise the
        // first leader reads every leader's lists across the cluster after it.
        const bool push = p.block_cap > 0 && p.segs * p.max_det <= kRecvKeys;
        if (push && part == 0) {
            uint64_t* recv = cluster.map_shared_rank(mrecv, 0) + cls * p.max_det;
            for (int q = tid; q < nkept; q += kThreads) recv[q] = kkey[q];
            if (tid == 0) cluster.map_shared_rank(&s, 0)->segn[cls] = nkept;
        }
        cluster.sync();  // every segment's kept keys are final and visible to the cluster
        if (cluster.block_rank() == 0) {  // segment 0's leader; segment c's leader is rank c * split
            if (tid == 0) {
                int total = 0;
                for (int c = 0; c < p.segs; ++c) {
                    s.off[c] = total;
                    total += push ? s.segn[c] : cluster.map_shared_rank(&s, c * p.split)->nkept;
                }
                s.off[p.segs] = total;
                s.count = total;
            }
            __syncthreads();
            const int total = s.count;  // segs x max_det <= kCap: the host launches a cluster only then
            // list c: its keys at lbase(c), s.off[c + 1] - s.off[c] of them, in descending order
            const uint64_t* lists = push ? mrecv : keys;
            auto lbase = [&](int c) { return push ? c * p.max_det : s.off[c]; };
            if (!push) {
                for (int c = 0; c < p.segs; ++c) {
                    const int off = s.off[c], cnt = s.off[c + 1] - off;
                    const uint64_t* list = cluster.map_shared_rank(kkey, c * p.split);
                    for (int q = tid; q < cnt; q += kThreads) keys[off + q] = list[q];
                }
                __syncthreads();
            }
            const int out_n = min(total, p.max_det);
            for (int e = tid; e < total; e += kThreads) {
                int c = 0;  // the list holding element e
                while (s.off[c + 1] <= e) ++c;
                const int q = e - s.off[c];
                const uint64_t key = lists[lbase(c) + q];
                int rank = q;
                for (int o = 0; o < p.segs; ++o) {
                    if (o == c) continue;
                    const int b = lbase(o);
                    int lo = 0, hi = s.off[o + 1] - s.off[o];  // first position in list o not above key
                    while (lo < hi) {
                        const int mid = (lo + hi) >> 1;
                        if (lists[b + mid] > key) lo = mid + 1;
                        else hi = mid;
                    }
                    rank += lo;
                }
                if (rank < out_n) out[rank] = key_index(key);
            }
            for (int i = out_n + tid; i < p.max_det; i += kThreads) out[i] = -1;
            if (tid == 0) p.counts[img] = out_n;
        }
        cluster.sync();  // no CTA leaves while CTA 0 may still read its shared memory
        return;
    }

    // Not in a cluster: publish this class's survivors; the image's last class merges.
    if (part != 0) return;
    int32_t* mine = p.seg_idx + (int64_t)seg * p.max_det;
    for (int i = tid; i < nkept; i += kThreads) mine[i] = key_index(kkey[i]);
    if (tid == 0) p.seg_cnt[seg] = nkept;
    __threadfence();
    __syncthreads();
    if (tid == 0) s.last = atomicAdd(p.arrivals + img, 1) == p.segs - 1;
    __syncthreads();
    if (!s.last) return;
    __threadfence();

    if (tid == 0) {
        int total = 0;
        for (int c = 0; c < p.segs && c < kMaxClassesMerged; ++c) {
            s.off[c] = total;
            total += __ldcg(p.seg_cnt + first + c);
        }
        s.off[min(p.segs, kMaxClassesMerged)] = total;
        s.count = total;
    }
    __syncthreads();
    const bool in_smem = p.segs <= kMaxClassesMerged && s.count <= kCap;
    int total = 0;
    if (in_smem) {
        total = s.count;
        // every survivor's key, list after list, each list already in descending order
        for (int c = 0; c < p.segs; ++c) {
            const int off = s.off[c], cnt = s.off[c + 1] - off;
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
            while (s.off[c + 1] <= e) ++c;
            const uint64_t key = keys[e];
            int rank = e - s.off[c];
            for (int o = 0; o < p.segs; ++o) {
                if (o == c) continue;
                int lo = s.off[o], hi = s.off[o + 1];  // first position in list o not above key
                while (lo < hi) {
                    const int mid = (lo + hi) >> 1;
                    if (keys[mid] > key) lo = mid + 1;
                    else hi = mid;
                }
                rank += lo - s.off[o];
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

// The midpoint between thr and the next float above it, and whether thr's last significand bit
// is 0 — the real-number form of the survivor test RN(inter / denom) <= thr (suppresses()).
void iou_midpoint(float thr, double* mid, int* even) {
    uint32_t bits;
    std::memcpy(&bits, &thr, sizeof(bits));
    *even = (bits & 1u) == 0;
    if (std::isnan(thr)) {
        *mid = std::nan("");
    } else if (std::isinf(thr)) {
        *mid = thr > 0 ? HUGE_VAL : -HUGE_VAL;
    } else if (thr == FLT_MAX) {
        *mid = std::ldexp(1.0, 128) - std::ldexp(1.0, 103);  // quotients from here on round to inf
    } else {
        *mid = ((double)thr + (double)std::nextafterf(thr, INFINITY)) / 2.0;
    }
}

// mid - thr as a float when suppresses_finite's single-precision comparison is exact: thr finite
// with |thr| <= 2^20 (so h <= 2^-4 and h * denom cannot overflow) and h * 1e-9 normal (denom
// is at least 1e-9, so h * denom cannot underflow); else 0.
float iou_half(float thr, double mid) {
    if (!std::isfinite(thr) || std::fabs(thr) > 1048576.0f) return 0.f;
    const double h = mid - (double)thr;  // half the gap to the next float: a power of two, exact
    if (!(h * 1e-9 >= (double)FLT_MIN)) return 0.f;
    return (float)h;
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

// Candidates resolved at once at the start of the first round: max_det and a margin for the
// candidates suppressed on the way (a sixteenth, and 16), in whole words, at most one round.
int block_cap(int max_det) {
    if (max_det > kBlockMaxDet) return 0;
    return std::min(kSort, (max_det + max_det / 16 + 16 + 31) & ~31);
}

int smem_bytes(int max_det) {
    return kCap * 8 + kSort * 8 + kSort * (16 + 4 + 4) + max_det * (16 + 8 + 4 + 4) +
           (block_cap(max_det) ? kSort * kMaskStride * 4 + 2 * kBuckets * 4 + kRecvKeys * 8 : 0);
}

int smem_limit() { return std::max(smem_bytes(kNmsMaxDet), smem_bytes(kBlockMaxDet)); }

// How many clusters of `size` CTAs with `smem` bytes of dynamic shared memory can be resident on
// the current device at once (cudaOccupancyMaxActiveClusters), cached per device and shape.
int max_active_clusters(int size, int smem) {
    static std::mutex mu;
    static std::map<std::tuple<int, int, int>, int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_tuple(dev, size, smem);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)size);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = (size_t)smem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = (unsigned)size;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, reinterpret_cast<const void*>(nms_kernel<false>), &cfg) != cudaSuccess) {
        cudaGetLastError();  // not fatal: no helpers
        n = 0;
    }
    cache[key] = n;
    return n;
}

int device_sms() {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    return sms;
}

// CTAs per segment for the block resolve: the most (up to a portable cluster of 8 with the class
// merge's segments) for which every cluster of the launch is resident at once, so the helpers
// cost no second wave; 1 when the block is small or the segments alone fill the device.
int choose_split(long long segments, int merge_segs, int cap, int smem) {
    if (cap < 128) return 1;
    const int sms = device_sms();
    for (int split = kMaxCluster / merge_segs; split >= 2; --split) {
        if (segments * split > sms) continue;
        const int size = merge_segs * split;
        if (segments / merge_segs <= max_active_clusters(size, smem)) return split;
    }
    return 1;
}

}  // namespace

// Scratch of the allocation-free entry point (shipk_nms_static): one per device, in the
// library's own module image, so using it allocates nothing. Its address is taken once per
// device with that device current.
constexpr size_t kStaticScratchBytes = size_t(1) << 20;
static __device__ __align__(256) unsigned char g_nms_scratch[kStaticScratchBytes];

size_t nms_static_capacity() { return kStaticScratchBytes; }

Status nms_static_scratch(void** out) {
    static std::mutex mu;
    static std::map<int, void*> addr;  // device -> address of g_nms_scratch there
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return Status{SHIPK_ECUDA, cudaGetErrorString(e)};
    std::lock_guard<std::mutex> lock(mu);
    auto it = addr.find(dev);
    if (it == addr.end()) {
        void* ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_nms_scratch);
        if (e != cudaSuccess) return Status{SHIPK_ECUDA, cudaGetErrorString(e)};
        it = addr.emplace(dev, ptr).first;
    }
    *out = it->second;
    return Status{SHIPK_OK, nullptr};
}

// The launch's shape: whether an image's classes merge inside a cluster, the block size of the
// first round, and the CTAs per segment (needs the kernel's shared-memory limit set first).
struct NmsShape {
    int segs, cluster, block_cap, split, smem;
};
NmsShape nms_shape(int batch, int num_classes, int class_aware, int max_det) {
    NmsShape sh;
    sh.segs = class_aware ? num_classes : 1;
    // An image's segments as one cluster when they fit a portable cluster and their merged lists
    // fit the key buffer (the merge then needs nothing from the workspace and nothing cleared);
    // otherwise the arrival-counter merge through the workspace.
    sh.cluster = class_aware && sh.segs >= 2 && sh.segs <= kMaxCluster && (long long)sh.segs * max_det <= kCap ? 1 : 0;
    sh.block_cap = block_cap(max_det);
    sh.smem = smem_bytes(max_det);
    sh.split = choose_split((long long)batch * sh.segs, sh.cluster ? sh.segs : 1, sh.block_cap, sh.smem);
    return sh;
}

Status nms_launch_shape(int batch, int num_classes, int class_aware, int max_det, int* ctas, int* cluster) {
    if (max_det > kNmsMaxDet) return Status{SHIPK_ERANGE, "max_det above 4096"};
    *ctas = 0;
    *cluster = 1;
    if (batch == 0 || max_det <= 0) return Status{SHIPK_OK, nullptr};
    cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(nms_kernel<false>), smem_limit());
    if (e == cudaSuccess) e = ensure_smem_attr(reinterpret_cast<const void*>(nms_kernel<true>), smem_limit());
    if (e != cudaSuccess) return Status{SHIPK_ECUDA, cudaGetErrorString(e)};
    const NmsShape sh = nms_shape(batch, num_classes, class_aware, max_det);
    const long long grid = (long long)batch * sh.segs * sh.split;
    *ctas = grid > 0x7fffffffLL ? -1 : (int)grid;
    *cluster = (sh.cluster ? sh.segs : 1) * sh.split;
    return Status{SHIPK_OK, nullptr};
}

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
    {
        cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(nms_kernel<false>), smem_limit());
        if (e == cudaSuccess) e = ensure_smem_attr(reinterpret_cast<const void*>(nms_kernel<true>), smem_limit());
        if (e != cudaSuccess) return Status{SHIPK_ECUDA, cudaGetErrorString(e)};
    }
    const NmsShape sh = nms_shape(batch, num_classes, class_aware, max_det);
    const int segs = sh.segs;
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
    iou_midpoint(iou_thr, &p.iou_mid, &p.iou_even);
    p.iou_half = iou_half(iou_thr, p.iou_mid);
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
    p.block_cap = sh.block_cap;
    p.cluster = sh.cluster;
    p.split = sh.split;
    if (zero_arrivals && class_aware && !p.cluster) {
        cudaError_t e = cudaMemsetAsync(p.arrivals, 0, (size_t)batch * sizeof(int32_t), stream);
        if (e != cudaSuccess) return Status{SHIPK_ECUDA, cudaGetErrorString(e)};
    }
    const int smem = sh.smem;
    const int merge_segs = p.cluster ? segs : 1;
    const long long grid = (long long)batch * segs * p.split;
    if (grid > 0x7fffffffLL) return Status{SHIPK_ERANGE, "too many NMS segments"};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (merge_segs * p.split > 1) {
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = (unsigned)(merge_segs * p.split);
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        cfg.numAttrs = 2;
    }
    cudaError_t e = p.split > 1 && !p.cluster ? cudaLaunchKernelEx(&cfg, nms_kernel<true>, p)
                                              : cudaLaunchKernelEx(&cfg, nms_kernel<false>, p);
    if (e != cudaSuccess) return Status{SHIPK_ECUDA, cudaGetErrorString(e)};
    return Status{SHIPK_OK, nullptr};
}

}  // namespace shipk
