// Detector decode on the device: a batch of frames' detector rows -> source-frame detections.
//
// Reference semantics: decode_detections, src/shipinfer/topology/elements/detections.py:423-515,
// in numpy 2 float32, per frame:
//   1. truncate to `count` rows when the detector reports how many it filled;
//   2. keep rows with score >= f32(score_threshold) (a NaN score fails);
//   3. cap at max_detections and order the kept rows by score descending, ties to the HIGHER
//      row first (the reference reverses a stable ascending argsort);
//   4. un-letterbox each coordinate: (v - pad) * float32(1.0 / scale), the reciprocal taken in
//      double (1.0 when scale is 0), then clip to [0, width] / [0, height] as np.clip does
//      (x < lo ? lo : x > hi ? hi : x, which keeps -0.0 and NaN); class float -> int32 as numpy
//      casts on x86-64 (truncation; INT_MIN for NaN, infinities and out-of-range values); a NaN
//      coordinate keeps its payload, as x86-64 arithmetic keeps it.
//
// Layout: one 1024-thread CTA per frame. Rows are visited as 64-bit keys
// ord(score) << 32 | row, whose descending order is step 3's order. When more rows pass the
// threshold than the cap, an exact MSB radix select (12-bit digits over the scores staged in
// shared memory, from the highest bit in which the passing rows' scores differ, stopping as soon
// as a digit's bucket is taken whole) finds the
// smallest key kept; the kept keys are appended to shared memory, sorted by a bitonic network
// there, and each thread writes the detections of its keys.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace shipk {

namespace {

constexpr int kThreads = 1024;
constexpr int kMaxDet = 4096;  // kept detections per frame (the sort runs in shared memory)
constexpr int kStage = 16384;  // frames of up to this many rows have their scores staged in shared memory
constexpr int kMergeMax = 1024;  // up to this many kept keys sort by warp runs and merges
constexpr int kDigitBits = 12;   // radix select digit
constexpr int kDigits = 1 << kDigitBits;
constexpr int kWhole = 32;       // a boundary bucket of up to this many keys is collected whole
static_assert(kDigits == 4 * kThreads, "each thread scans four buckets");
static_assert(kDigits * sizeof(unsigned) <= kMaxDet * sizeof(uint64_t), "the buckets fit in the keys' memory");

struct DecodeArgs {
    const float* rows;        // [batch, R, 6]
    int R;
    const int32_t* counts;    // [batch] or null
    const float* scales;      // [batch]
    const float* pads;        // [batch, 2] (x, y)
    const int32_t* frame_hw;  // [batch, 2] (h, w) or null: no clip
    float score_thr;
    int max_det;
    float* boxes;             // [batch, max_det, 4]
    float* scores;            // [batch, max_det]
    int32_t* classes;         // [batch, max_det]
    int32_t* out_counts;      // [batch]
    int32_t* discarded;       // [batch]
    int staged;               // R <= kStage: each frame's scores are copied to shared memory first
};

// Score order bits: larger floats give larger codes; -0.0 and +0.0 the same (numpy's sort
// finds them equal, so the row index decides).
__device__ __forceinline__ uint64_t row_key(float s, int row) {
    uint32_t u = __float_as_uint(s);
    if ((u & 0x7fffffffu) == 0) u = 0;
    const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((uint64_t)ord << 32) | (uint32_t)row;
}

__device__ __forceinline__ int32_t f32_to_i32_numpy(float v) {
    if (v != v || v >= 2147483648.0f || v < -2147483648.0f) return INT32_MIN;
    return __float2int_rz(v);
}

__device__ __forceinline__ float clip_numpy(float v, float hi) { return v < 0.f ? 0.f : (v > hi ? hi : v); }

// a - b and a * b with NaN results as x86-64 SSE/AVX produce them, which is what numpy computes
// on: a NaN operand propagates (the first one, quieted, payload and sign kept), and an invalid
// operation on other operands (inf - inf, 0 * inf) gives the default NaN 0xffc00000. (The GPU's
// arithmetic returns one canonical NaN, 0x7fffffff, for all of these.)
__device__ __forceinline__ float nan_first(float a, float b, float r) {
    if (a != a) return __uint_as_float(__float_as_uint(a) | 0x00400000u);
    if (b != b) return __uint_as_float(__float_as_uint(b) | 0x00400000u);
    if (r != r) return __uint_as_float(0xffc00000u);
    return r;
}
__device__ __forceinline__ float sub_x86(float a, float b) { return nan_first(a, b, __fsub_rn(a, b)); }
__device__ __forceinline__ float mul_x86(float a, float b) { return nan_first(a, b, __fmul_rn(a, b)); }

__global__ void __launch_bounds__(kThreads) decode_kernel(const __grid_constant__ DecodeArgs a) {
    extern __shared__ float staged_scores[];  // [R] when a.staged
    __shared__ uint64_t keys[kMaxDet];
    __shared__ uint64_t merge_buf[kMergeMax];
    __shared__ unsigned wsum[kThreads / 32];
    __shared__ uint64_t s_prefix;
    __shared__ int s_want, s_done, s_total, s_count;
    __shared__ unsigned s_or, s_and;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int img = blockIdx.x;
    const int total = a.counts ? max(0, min(__ldg(a.counts + img), a.R)) : a.R;
    const float* rows = a.rows + (int64_t)img * a.R * 6;
    const float thr = a.score_thr;
    // Every pass below reads each row's score: from shared memory once they are staged there
    // (one strided pass over the 24-byte rows), else from global memory each time. The first
    // pass also counts the rows that pass the threshold and takes the OR and AND of their order
    // bits (one shared atomic per warp for each).
    if (tid == 0) {
        s_total = 0;
        s_or = 0;
        s_and = ~0u;
    }
    __syncthreads();
    {
        unsigned kor = 0, kand = ~0u, npass = 0;
        for (int i = tid; i < total; i += kThreads) {
            const float s = __ldg(rows + (int64_t)i * 6 + 4);
            if (a.staged) staged_scores[i] = s;
            if (s >= thr) {
                const unsigned o = (unsigned)(row_key(s, 0) >> 32);
                kor |= o;
                kand &= o;
                ++npass;
            }
        }
        kor = __reduce_or_sync(0xffffffffu, kor);
        kand = __reduce_and_sync(0xffffffffu, kand);
        npass = __reduce_add_sync(0xffffffffu, npass);
        if (lane == 0 && npass) {
            atomicOr(&s_or, kor);
            atomicAnd(&s_and, kand);
            atomicAdd(&s_total, (int)npass);
        }
        __syncthreads();
    }
    auto score = [&](int i) { return a.staged ? staged_scores[i] : __ldg(rows + (int64_t)i * 6 + 4); };

    // ---- the smallest kept key: 0 (every passing row) unless more than max_det pass. An MSB
    // radix select in digits of up to kDigitBits bits, the bits at and above `hi` fixed in
    // `prefix`; its buckets live in the keys' shared memory, which is written only after the
    // select. It starts below the bits that every passing row shares: a digit there would put
    // all the rows in one bucket (thousands of shared atomics on one counter) and only append
    // those bits to the prefix, which is set here instead. Scores in [0.25, 1) then spread over
    // 4096 buckets, and the first digit usually ends the select.
    unsigned* const hist = reinterpret_cast<unsigned*>(keys);
    uint64_t prefix = 0;
    int want = a.max_det;
    bool select = a.max_det > 0 && s_total > want;  // a cap of 0 keeps nothing: no select
    int hi = 64;
    if (select) {
        const unsigned diff = s_or ^ s_and;  // order bits in which passing rows differ
        hi = diff == 0 ? 32 : 33 + (31 - __clz((int)diff));
        if (hi < 64) prefix = ((uint64_t)s_and << 32) & ~((1ull << hi) - 1);
    }
    while (hi > 0 && select) {
        const int w = min(kDigitBits, hi), shift = hi - w;
        for (int d = tid; d < kDigits; d += kThreads) hist[d] = 0;
        __syncthreads();
        for (int i = tid; i < total; i += kThreads) {
            const float s = score(i);
            if (!(s >= thr)) continue;
            const uint64_t k = row_key(s, i);
            if (hi < 64 && (k >> hi) != (prefix >> hi)) continue;
            atomicAdd(&hist[(unsigned)(k >> shift) & ((1u << w) - 1u)], 1u);
        }
        __syncthreads();
        // thread t holds digits kDigits-1-4t .. kDigits-4-4t (the top digits first); a prefix
        // sum over the threads finds the digit at which the count from the top reaches `want`
        unsigned c[4], sum = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            c[q] = hist[kDigits - 1 - 4 * tid - q];
            sum += c[q];
        }
        unsigned incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        if (lane == 31) wsum[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            const unsigned t = wsum[lane];
            unsigned wi = t;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned v = __shfl_up_sync(0xffffffffu, wi, o);
                if (lane >= o) wi += v;
            }
            wsum[lane] = wi - t;
        }
        __syncthreads();
        const unsigned excl = wsum[warp] + incl - sum;
        if (excl < (unsigned)want && excl + sum >= (unsigned)want) {
            unsigned cum = excl;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                if (cum + c[q] >= (unsigned)want) {
                    const unsigned digit = kDigits - 1 - 4 * tid - q;
                    const unsigned extra = cum + c[q] - (unsigned)want;  // the bucket's keys past the cap
                    s_prefix = prefix | ((uint64_t)digit << shift);
                    s_want = want - (int)cum;
                    // The bucket is taken whole when it holds just the keys still wanted, or when
                    // it is small: its keys past the cap are then collected too, the sort puts
                    // them after the kept ones, and no further pass over the rows is needed.
                    s_done = extra == 0 || (c[q] <= (unsigned)kWhole && a.max_det + (int)extra <= kMaxDet);
                    break;
                }
                cum += c[q];
            }
        }
        __syncthreads();
        prefix = s_prefix;
        want = s_want;
        select = !s_done;
        hi = shift;
        __syncthreads();  // every thread has read the shared state before the next pass resets it
    }
    __syncthreads();
    const int m = min(s_total, a.max_det);

    // ---- the kept keys (m of them, then any keys of a small boundary bucket taken whole; keys
    // are distinct), appended in any order
    if (tid == 0) s_count = 0;
    __syncthreads();
    for (int base = 0; base < total; base += kThreads) {
        const int i = base + tid;
        bool take = false;
        uint64_t k = 0;
        if (i < total) {
            const float s = score(i);
            if (s >= thr) {
                k = row_key(s, i);
                take = k >= prefix;
            }
        }
        const unsigned bal = __ballot_sync(0xffffffffu, take);
        int slot = 0;
        if (lane == 0 && bal) slot = atomicAdd(&s_count, __popc(bal));
        slot = __shfl_sync(0xffffffffu, slot, 0) + __popc(bal & ((1u << lane) - 1u));
        if (take && slot < kMaxDet) keys[slot] = k;
    }
    __syncthreads();

    const int n = m == 0 ? 0 : min(s_count, kMaxDet);
    // ---- sort keys[0, n) descending (n: the keys collected; the first m are kept). Up to
    // kMergeMax keys: one key per thread, 32-key runs sorted by a bitonic network over warp
    // shuffles, then merged pairwise level by level (a
    // key's place in a merged pair is its place in its run plus the count of keys above it in
    // the partner run, by binary search). Keys are distinct and nonzero; zero padding sits at
    // the end of the last run.
    if (n <= kMergeMax) {
        const int P = (n + 31) & ~31;  // whole warps
        uint64_t v = tid < n ? keys[tid] : 0;
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
        if (tid < P) keys[tid] = v;
        __syncthreads();
        uint64_t* src = keys;
        uint64_t* dst = merge_buf;
        for (int L = 32; L < P; L <<= 1) {
            if (tid < P) {
                const int r = tid / L, in_run = tid - r * L;
                const int pair = (r >> 1) * 2 * L;
                const int partner = (r ^ 1) * L;
                const int plen = max(0, min(L, P - partner));  // 0: no partner run
                const uint64_t key = src[tid];
                int lo = 0, hi = plen;
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
        if (src != keys) {
            if (tid < P) keys[tid] = src[tid];
            __syncthreads();
        }
    } else {
    // bitonic sort of keys[0, P) descending; slots past n hold 0, below every real key
    int P = 1;
    while (P < n) P <<= 1;
    for (int i = n + tid; i < P; i += kThreads) keys[i] = 0;
    __syncthreads();
    for (int k = 2; k <= P; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int t = tid; t < (P >> 1); t += kThreads) {
                const int lo = 2 * t - (t & (j - 1));
                const int hi = lo + j;
                const uint64_t x = keys[lo], y = keys[hi];
                const bool desc = (lo & k) == 0;
                if (desc ? (x < y) : (x > y)) {
                    keys[lo] = y;
                    keys[hi] = x;
                }
            }
            __syncthreads();
        }
    }
    }

    // ---- the detections, in key order
    const float scale = __ldg(a.scales + img);
    const float inv = scale != 0.f ? __double2float_rn(__ddiv_rn(1.0, (double)scale)) : 1.0f;
    const float pad_x = __ldg(a.pads + 2 * img), pad_y = __ldg(a.pads + 2 * img + 1);
    const bool clip = a.frame_hw != nullptr;
    const float fh = clip ? (float)__ldg(a.frame_hw + 2 * img) : 0.f;
    const float fw = clip ? (float)__ldg(a.frame_hw + 2 * img + 1) : 0.f;
    float* ob = a.boxes + (int64_t)img * a.max_det * 4;
    float* os = a.scores + (int64_t)img * a.max_det;
    int32_t* oc = a.classes + (int64_t)img * a.max_det;
    for (int q = tid; q < a.max_det; q += kThreads) {
        if (q < m) {
            const int row = (int)(uint32_t)(keys[q] & 0xffffffffu);
            const float* r = rows + (int64_t)row * 6;
            float v[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                float x = mul_x86(sub_x86(__ldg(r + c), (c & 1) ? pad_y : pad_x), inv);
                if (clip) x = clip_numpy(x, (c & 1) ? fh : fw);
                v[c] = x;
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) ob[4 * q + c] = v[c];
            os[q] = __ldg(r + 4);
            oc[q] = f32_to_i32_numpy(__ldg(r + 5));
        } else {  // past the kept detections: zeros and class -1
#pragma unroll
            for (int c = 0; c < 4; ++c) ob[4 * q + c] = 0.f;
            os[q] = 0.f;
            oc[q] = -1;
        }
    }
    if (tid == 0) {
        a.out_counts[img] = m;
        a.discarded[img] = total - m;
    }
}

}  // namespace

Status launch_decode(const float* rows, int batch, int R, const int32_t* counts, const float* scales,
                     const float* pads, const int32_t* frame_hw, float score_threshold, int max_det,
                     float* boxes, float* scores, int32_t* classes, int32_t* out_counts, int32_t* discarded,
                     cudaStream_t stream) {
    if (max_det > kMaxDet) return Status{SHIPK_ERANGE, "max_detections above 4096"};
    if (batch == 0) return Status{SHIPK_OK, nullptr};
    DecodeArgs a;
    a.rows = rows;
    a.R = R;
    a.counts = counts;
    a.scales = scales;
    a.pads = pads;
    a.frame_hw = frame_hw;
    a.score_thr = score_threshold;
    a.max_det = std::max(max_det, 0);
    a.boxes = boxes;
    a.scores = scores;
    a.classes = classes;
    a.out_counts = out_counts;
    a.discarded = discarded;
    a.staged = R <= kStage ? 1 : 0;
    const int smem = a.staged ? R * (int)sizeof(float) : 0;
    cudaError_t e0 = ensure_smem_attr(reinterpret_cast<const void*>(decode_kernel), kStage * (int)sizeof(float));
    if (e0 != cudaSuccess) return Status{SHIPK_ECUDA, cudaGetErrorString(e0)};
    decode_kernel<<<batch, kThreads, smem, stream>>>(a);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return Status{SHIPK_ECUDA, cudaGetErrorString(e)};
    return Status{SHIPK_OK, nullptr};
}

}  // namespace shipk
