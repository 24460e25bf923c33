/*
 * TEST INFRASTRUCTURE ONLY: the CPU oracle for the image-ops hot path. Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline arm use it, and only as the checker
 * (or the timed CPU baseline), never as the product path.
 *
 * Compiled with -ffp-contract=off: every float operation below rounds on its own, except
 * the ones written as fmaf(), which are the steps the reference's CUDA/torch formulation
 * fuses (nvcc contracts a*b+c by default; torch's vectorised CPU lerp uses fmadd).
 *
 * Parity is pinned by tests/golden/ (outputs of the reference's own TorchImageOps and
 * NumpyImageOps, imported from the reference source tree by tests/golden/make_golden.py).
 */
#include "oracle.h"

#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------------------------------
 * Letterbox placement. Reference: src/shipinfer/runtime/ops/torch_ops.py:373-379
 *   scale = min(dst_h / src_h, dst_w / src_w)        (Python floats, i.e. double)
 *   new   = max(1, round(src * scale))               (round half to even)
 *   pad   = (dst - new) // 2
 * nearbyint() under the default rounding mode is round-half-to-even, as Python's round().
 * ------------------------------------------------------------------------------------- */
orc_fit_t orc_letterbox_fit(int src_h, int src_w, int dst_h, int dst_w) {
    orc_fit_t f;
    double sh = (double)dst_h / (double)src_h;
    double sw = (double)dst_w / (double)src_w;
    double s = sh < sw ? sh : sw;
    double nh = nearbyint((double)src_h * s);
    double nw = nearbyint((double)src_w * s);
    f.new_h = nh < 1.0 ? 1 : (int)nh;
    f.new_w = nw < 1.0 ? 1 : (int)nw;
    /* Python floor division; dst >= new always holds for this scale, so this is C division
     * on a non-negative value, but floor it anyway for a degenerate destination. */
    int dy = dst_h - f.new_h, dx = dst_w - f.new_w;
    f.pad_y = dy >= 0 ? dy / 2 : -((-dy + 1) / 2);
    f.pad_x = dx >= 0 ? dx / 2 : -((-dx + 1) / 2);
    f.scale = (float)s;
    return f;
}

/* The C++ data plane's placement. Reference: csrc/shipinfer/runtime/ops.cu:341-356
 *   scale = min(float(dst_w) / float(src_w), float(dst_h) / float(src_h))   (float32)
 *   new   = max(1, nearbyint(float(src) * scale))                            (float32 product)
 *   pad   = (dst - new) / 2
 * Some sizes place differently from orc_letterbox_fit (180x1280 -> 224x224: 32 rows, not 31). */
orc_fit_t orc_letterbox_fit_f32(int src_h, int src_w, int dst_h, int dst_w) {
    orc_fit_t f;
    float sw = (float)dst_w / (float)src_w;
    float sh = (float)dst_h / (float)src_h;
    float s = sw < sh ? sw : sh;
    float nw = nearbyintf((float)src_w * s);
    float nh = nearbyintf((float)src_h * s);
    f.new_w = nw < 1.f ? 1 : (int)nw;
    f.new_h = nh < 1.f ? 1 : (int)nh;
    f.pad_x = (dst_w - f.new_w) / 2;
    f.pad_y = (dst_h - f.new_h) / 2;
    f.scale = s;
    return f;
}

static orc_fit_t orc_fit_of(int cpp_fit, int src_h, int src_w, int dst_h, int dst_w) {
    return cpp_fit ? orc_letterbox_fit_f32(src_h, src_w, dst_h, dst_w)
                   : orc_letterbox_fit(src_h, src_w, dst_h, dst_w);
}

/* ---------------------------------------------------------------------------------------
 * F.interpolate(mode="bilinear", align_corners=False), CUDA formulation.
 * The reference calls it at torch_ops.py:389-391 on a float32 copy of the uint8 frame.
 *   ratio   = (float)in / (float)out                      (host-side, one rounding)
 *   src     = ratio * (d + 0.5) - 0.5, clamped at 0        (fused multiply-add)
 *   i0      = (int)src; i1 = i0 + (i0 < in - 1)
 *   l1      = src - i0; l0 = 1 - l1
 *   value   = h0 * (w0 * p00 + w1 * p01) + h1 * (w0 * p10 + w1 * p11)
 * with each "a*b + c*d" fused as fma(a, b, c*d).
 * ------------------------------------------------------------------------------------- */
typedef struct {
    int i0, i1;
    float l0, l1;
} orc_tap_t;

static orc_tap_t orc_source_tap(float ratio, int d, int in_size) {
    orc_tap_t t;
    float s = fmaf(ratio, (float)d + 0.5f, -0.5f);
    if (s < 0.f) s = 0.f;
    t.i0 = (int)s;
    if (t.i0 > in_size - 1) t.i0 = in_size - 1; /* never taken for s < in_size - 0.5 */
    t.i1 = t.i0 + (t.i0 < in_size - 1 ? 1 : 0);
    t.l1 = s - (float)t.i0;
    t.l0 = 1.f - t.l1;
    return t;
}

static float orc_blend(orc_tap_t ty, orc_tap_t tx, float p00, float p01, float p10,
                       float p11) {
    float top = fmaf(tx.l0, p00, tx.l1 * p01);
    float bottom = fmaf(tx.l0, p10, tx.l1 * p11);
    return fmaf(ty.l0, top, ty.l1 * bottom);
}

static int orc_threads(int threads) {
#ifdef _OPENMP
    return threads > 0 ? threads : omp_get_max_threads();
#else
    (void)threads;
    return 1;
#endif
}

/* ---------------------------------------------------------------------------------------
 * TorchImageOps._letterbox, torch_ops.py:349-403:
 *   canvas.fill_(pad); canvas[i, :, py:py+nh, px:px+nw] = interpolate(frame);
 *   canvas.flip(1) if swap_rb; canvas.sub_(mean).div_(std)        (per OUTPUT channel)
 * ------------------------------------------------------------------------------------- */
void orc_letterbox_u8(const orc_frame_t* frames, int n, int dst_h, int dst_w,
                      const float mean[3], const float stdv[3], int swap_rb, float pad_value,
                      float* out, int threads) {
    orc_letterbox_u8_fit(frames, n, dst_h, dst_w, mean, stdv, swap_rb, pad_value, 0, out, threads);
}

void orc_letterbox_u8_fit(const orc_frame_t* frames, int n, int dst_h, int dst_w,
                          const float mean[3], const float stdv[3], int swap_rb, float pad_value,
                          int cpp_fit, float* out, int threads) {
    const size_t plane = (size_t)dst_h * (size_t)dst_w;
    float pad_out[3];
    for (int c = 0; c < 3; ++c) pad_out[c] = (pad_value - mean[c]) / stdv[c];
    int nt = orc_threads(threads);
#pragma omp parallel for collapse(2) schedule(static) num_threads(nt)
    for (int i = 0; i < n; ++i) {
        for (int y = 0; y < dst_h; ++y) {
            const orc_frame_t fr = frames[i];
            orc_fit_t fit = orc_fit_of(cpp_fit, fr.h, fr.w, dst_h, dst_w);
            float rh = (float)fr.h / (float)fit.new_h;
            float rw = (float)fr.w / (float)fit.new_w;
            float* img = out + (size_t)i * 3 * plane;
            int inside_y = y >= fit.pad_y && y < fit.pad_y + fit.new_h;
            orc_tap_t ty = {0, 0, 0.f, 0.f};
            if (inside_y) ty = orc_source_tap(rh, y - fit.pad_y, fr.h);
            for (int x = 0; x < dst_w; ++x) {
                int inside = inside_y && x >= fit.pad_x && x < fit.pad_x + fit.new_w;
                if (!inside) {
                    for (int c = 0; c < 3; ++c) img[c * plane + (size_t)y * dst_w + x] = pad_out[c];
                    continue;
                }
                orc_tap_t tx = orc_source_tap(rw, x - fit.pad_x, fr.w);
                const uint8_t* r0 = fr.data + (int64_t)ty.i0 * fr.pitch;
                const uint8_t* r1 = fr.data + (int64_t)ty.i1 * fr.pitch;
                for (int c = 0; c < 3; ++c) {
                    int sc = swap_rb ? 2 - c : c;
                    float v = orc_blend(ty, tx, (float)r0[tx.i0 * 3 + sc], (float)r0[tx.i1 * 3 + sc],
                                        (float)r1[tx.i0 * 3 + sc], (float)r1[tx.i1 * 3 + sc]);
                    img[c * plane + (size_t)y * dst_w + x] = (v - mean[c]) / stdv[c];
                }
            }
        }
    }
}

/* ---------------------------------------------------------------------------------------
 * TorchImageOps.crop_batch, torch_ops.py:405-507, and _bilinear_axis, :574-614.
 *   clip x to [0, W-1], y to [0, H-1] in float32, then truncate (numpy float->int64 cast);
 *   extent = x2 - x1 (patch [x1, x2)); axis table in float32 WITHOUT fusion (numpy):
 *     scale = f32(max(ext,1)) / f32(dst);  src = max(scale * (d + 0.5) - 0.5, 0)
 *     i0 = min(int(src), ext-1); w1 = src - i0; i1 = min(i0 + 1, ext-1)
 *   top = lerp(p[r0][c0], p[r0][c1], wx); bottom = lerp(p[r1][c0], p[r1][c1], wx);
 *   v = lerp(top, bottom, wy)      (torch.lerp; see orc_lerp)
 *   degenerate (ext <= 0 on either axis) -> v = 0 before normalisation
 *   channel gather [2,1,0] if swap_rb, then (v - mean[c]) / std[c].
 * NaN box coordinates are undefined in the reference (numpy casts NaN to INT64_MIN); here,
 * as in the CUDA kernel, a NaN coordinate clips to 0 (fmaxf semantics).
 * ------------------------------------------------------------------------------------- */

/* at::lerp: |w| < 0.5 ? a + w*(b-a) : b - (b-a)*(1-w), each branch one fused multiply-add
 * (torch's CUDA lerp under nvcc contraction; its AVX2/AVX-512 CPU lerp uses fmadd). */
static float orc_lerp(float a, float b, float w) {
    float d = b - a;
    return fabsf(w) < 0.5f ? fmaf(w, d, a) : fmaf(-d, 1.f - w, b);
}

static int orc_clip_trunc(float v, float hi) {
    float c = fmaxf(v, 0.f); /* fmaxf(NaN, 0) = 0 */
    c = fminf(c, hi);
    return (int)c;
}

typedef struct {
    int i0, i1;
    float w1;
} orc_axis_t;

static orc_axis_t orc_crop_axis(int ext, int d, int dst) {
    orc_axis_t a;
    int ext_safe = ext > 1 ? ext : 1;
    float scale = (float)ext_safe / (float)dst;
    float prod = scale * ((float)d + 0.5f);
    float src = prod - 0.5f;
    if (src < 0.f) src = 0.f; /* np.maximum(src, 0) */
    int last = ext_safe - 1;
    int i0 = (int)src;
    if (i0 > last) i0 = last;
    a.w1 = src - (float)i0;
    a.i1 = i0 + 1 < last ? i0 + 1 : last;
    a.i0 = i0;
    return a;
}

void orc_crop_u8(const orc_frame_t* frames, int n_frames, const float* boxes,
                 const int32_t* frame_idx, int n_boxes, int dst_h, int dst_w,
                 const float mean[3], const float stdv[3], int swap_rb, float* out,
                 int threads) {
    const size_t plane = (size_t)dst_h * (size_t)dst_w;
    int nt = orc_threads(threads);
#pragma omp parallel for schedule(dynamic, 1) num_threads(nt)
    for (int b = 0; b < n_boxes; ++b) {
        int f = frame_idx ? frame_idx[b] : 0;
        float* crop = out + (size_t)b * 3 * plane;
        const float* bx = boxes + (size_t)b * 4;
        int valid_frame = f >= 0 && f < n_frames;
        orc_frame_t fr = valid_frame ? frames[f] : frames[0];
        int x1 = orc_clip_trunc(bx[0], (float)(fr.w - 1));
        int y1 = orc_clip_trunc(bx[1], (float)(fr.h - 1));
        int x2 = orc_clip_trunc(bx[2], (float)(fr.w - 1));
        int y2 = orc_clip_trunc(bx[3], (float)(fr.h - 1));
        int ew = x2 - x1, eh = y2 - y1;
        int degenerate = !valid_frame || ew <= 0 || eh <= 0;
        for (int y = 0; y < dst_h; ++y) {
            orc_axis_t ay = orc_crop_axis(eh, y, dst_h);
            const uint8_t* r0 = fr.data + (int64_t)(y1 + ay.i0) * fr.pitch;
            const uint8_t* r1 = fr.data + (int64_t)(y1 + ay.i1) * fr.pitch;
            for (int x = 0; x < dst_w; ++x) {
                float v[3] = {0.f, 0.f, 0.f};
                if (!degenerate) {
                    orc_axis_t ax = orc_crop_axis(ew, x, dst_w);
                    int c0 = (x1 + ax.i0) * 3, c1 = (x1 + ax.i1) * 3;
                    for (int s = 0; s < 3; ++s) {
                        float top = orc_lerp((float)r0[c0 + s], (float)r0[c1 + s], ax.w1);
                        float bot = orc_lerp((float)r1[c0 + s], (float)r1[c1 + s], ax.w1);
                        v[s] = orc_lerp(top, bot, ay.w1);
                    }
                }
                for (int c = 0; c < 3; ++c) {
                    int sc = swap_rb ? 2 - c : c;
                    crop[c * plane + (size_t)y * dst_w + x] = (v[sc] - mean[c]) / stdv[c];
                }
            }
        }
    }
}

/* ---------------------------------------------------------------------------------------
 * NumpyImageOps.nms, numpy_ops.py:120-155, in numpy 2's float32 semantics:
 *   candidates = scores >= f32(score_threshold); order = stable argsort(-scores)
 *   areas = max(0, x2-x1) * max(0, y2-y1)
 *   inter = max(0, min(x2b,x2r) - max(x1b,x1r)) * max(0, min(y2b,y2r) - max(y1b,y1r))
 *   iou = inter / max(areas_b + areas_r - inter, f32(1e-9)); survivors: iou <= f32(thr)
 * np.maximum / np.minimum propagate NaN, so these helpers do too.
 * ------------------------------------------------------------------------------------- */
static float orc_nmax(float a, float b) {
    if (a != a) return a;
    if (b != b) return b;
    return a > b ? a : b;
}
static float orc_nmin(float a, float b) {
    if (a != a) return a;
    if (b != b) return b;
    return a < b ? a : b;
}

typedef struct {
    float score;
    int32_t idx;
} orc_cand_t;

static int orc_cand_cmp(const void* pa, const void* pb) {
    const orc_cand_t* a = (const orc_cand_t*)pa;
    const orc_cand_t* b = (const orc_cand_t*)pb;
    /* descending score (-0.0 == 0.0, as the argsort's < sees them), ties by index */
    if (a->score > b->score) return -1;
    if (a->score < b->score) return 1;
    return a->idx < b->idx ? -1 : (a->idx > b->idx ? 1 : 0);
}

static int orc_nms_subset(const float* boxes, const float* scores, const int32_t* subset,
                          int m, float iou_thr, float score_thr, int max_output,
                          int32_t* kept) {
    if (max_output <= 0) return 0;
    orc_cand_t* order = (orc_cand_t*)malloc(sizeof(orc_cand_t) * (size_t)(m > 0 ? m : 1));
    int n_order = 0;
    for (int j = 0; j < m; ++j) {
        int i = subset ? subset[j] : j;
        if (scores[i] >= score_thr) {
            order[n_order].score = scores[i];
            order[n_order].idx = i;
            ++n_order;
        }
    }
    qsort(order, (size_t)n_order, sizeof(orc_cand_t), orc_cand_cmp);
    const float eps = 1e-9f;
    int n_kept = 0;
    while (n_order > 0 && n_kept < max_output) {
        int best = order[0].idx;
        kept[n_kept++] = best;
        if (n_order == 1) break;
        const float* bb = boxes + (size_t)best * 4;
        float area_b = orc_nmax(0.f, bb[2] - bb[0]) * orc_nmax(0.f, bb[3] - bb[1]);
        int w = 0;
        for (int r = 1; r < n_order; ++r) {
            const float* rb = boxes + (size_t)order[r].idx * 4;
            float area_r = orc_nmax(0.f, rb[2] - rb[0]) * orc_nmax(0.f, rb[3] - rb[1]);
            float iw = orc_nmax(0.f, orc_nmin(bb[2], rb[2]) - orc_nmax(bb[0], rb[0]));
            float ih = orc_nmax(0.f, orc_nmin(bb[3], rb[3]) - orc_nmax(bb[1], rb[1]));
            float inter = iw * ih;
            float denom = orc_nmax(area_b + area_r - inter, eps);
            float iou = inter / denom;
            if (iou <= iou_thr) order[w++] = order[r];
        }
        n_order = w;
    }
    free(order);
    return n_kept;
}

int orc_nms(const float* boxes, const float* scores, int n, float iou_threshold,
            float score_threshold, int max_output, int64_t* keep) {
    int32_t* kept = (int32_t*)malloc(sizeof(int32_t) * (size_t)(max_output > 0 ? max_output : 1));
    int k = orc_nms_subset(boxes, scores, NULL, n, iou_threshold, score_threshold, max_output,
                           kept);
    for (int i = 0; i < k; ++i) keep[i] = kept[i];
    free(kept);
    return k;
}

void orc_nms_batched(const float* boxes, const float* scores, const int32_t* classes, int B,
                     int n, int num_classes, int class_aware, float iou_threshold,
                     float score_threshold, int max_output, int64_t* keep, int32_t* counts,
                     int threads) {
    int nt = orc_threads(threads);
#pragma omp parallel for schedule(dynamic, 1) num_threads(nt)
    for (int b = 0; b < B; ++b) {
        const float* bx = boxes + (size_t)b * n * 4;
        const float* sc = scores + (size_t)b * n;
        int64_t* out = keep + (size_t)b * (max_output > 0 ? max_output : 0);
        for (int k = 0; k < max_output; ++k) out[k] = -1;
        if (max_output <= 0) {
            counts[b] = 0;
            continue;
        }
        if (!class_aware) {
            int32_t* kept = (int32_t*)malloc(sizeof(int32_t) * (size_t)max_output);
            int k = orc_nms_subset(bx, sc, NULL, n, iou_threshold, score_threshold, max_output,
                                   kept);
            for (int i = 0; i < k; ++i) out[i] = kept[i];
            counts[b] = k;
            free(kept);
            continue;
        }
        /* per class: idx_c = nonzero(cls == c), NMS on the subset, then merge the survivors
         * by (score desc, index asc) and keep the first max_output. */
        const int32_t* cl = classes + (size_t)b * n;
        int32_t* subset = (int32_t*)malloc(sizeof(int32_t) * (size_t)(n > 0 ? n : 1));
        orc_cand_t* merged =
            (orc_cand_t*)malloc(sizeof(orc_cand_t) * (size_t)max_output * (size_t)num_classes + 1);
        int32_t* kept = (int32_t*)malloc(sizeof(int32_t) * (size_t)max_output);
        int n_merged = 0;
        for (int c = 0; c < num_classes; ++c) {
            int m = 0;
            for (int i = 0; i < n; ++i)
                if (cl[i] == c) subset[m++] = i;
            int k = orc_nms_subset(bx, sc, subset, m, iou_threshold, score_threshold,
                                   max_output, kept);
            for (int i = 0; i < k; ++i) {
                merged[n_merged].score = sc[kept[i]];
                merged[n_merged].idx = kept[i];
                ++n_merged;
            }
        }
        qsort(merged, (size_t)n_merged, sizeof(orc_cand_t), orc_cand_cmp);
        int k = n_merged < max_output ? n_merged : max_output;
        for (int i = 0; i < k; ++i) out[i] = merged[i].idx;
        counts[b] = k;
        free(subset);
        free(merged);
        free(kept);
    }
}

/* ---------------------------------------------------------------------------------------
 * NV12 -> RGB. Reference nv12_to_bgr: csrc/shipinfer/runtime/ops.cu:148-166 (BT.601
 * limited range, co-sited chroma taken at (x/2*2, y/2)). Its constants are the limited-range
 * matrix rounded to six decimals; BT.709 uses the same construction from Kr = 0.2126,
 * Kb = 0.0722 (ITU-R BT.709-6), also rounded to six decimals:
 *   Y' = (Y - 16) * 255/219;  B = Y' + cbu*U;  G = Y' - cgu*U - cgv*V;  R = Y' + crv*V
 * Under nvcc contraction "Y + k*U" is fma(k, U, Y) and "Y - a*U - b*V" is
 * fma(-b, V, fma(-a, U, Y)); each channel is clamped to [0, 255].
 * ------------------------------------------------------------------------------------- */
typedef struct {
    float ys, cbu, cgu, cgv, crv;
} orc_yuv_t;

static orc_yuv_t orc_matrix(int matrix) {
    orc_yuv_t m;
    m.ys = 1.164383f;
    if (matrix == 709) {
        m.cbu = 2.112402f;
        m.cgu = 0.213249f;
        m.cgv = 0.532909f;
        m.crv = 1.792741f;
    } else {
        m.cbu = 2.017232f;
        m.cgu = 0.391762f;
        m.cgv = 0.812968f;
        m.crv = 1.596027f;
    }
    return m;
}

static void orc_nv12_bgr(const orc_nv12_t* f, orc_yuv_t m, int yi, int xi, float bgr[3]) {
    const uint8_t* uv = f->data + f->uv_offset;
    float Y = ((float)f->data[(int64_t)yi * f->pitch + xi] - 16.f) * m.ys;
    int cx = (xi / 2) * 2, cy = yi / 2;
    float U = (float)uv[(int64_t)cy * f->pitch + cx + 0] - 128.f;
    float V = (float)uv[(int64_t)cy * f->pitch + cx + 1] - 128.f;
    float b = fmaf(m.cbu, U, Y);
    float g = fmaf(-m.cgv, V, fmaf(-m.cgu, U, Y));
    float r = fmaf(m.crv, V, Y);
    bgr[0] = fminf(255.f, fmaxf(0.f, b));
    bgr[1] = fminf(255.f, fmaxf(0.f, g));
    bgr[2] = fminf(255.f, fmaxf(0.f, r));
}

/* The reference NV12 kernel's own source coordinate (ops.cu:167-172):
 * max(0, ((d + 0.5) * in) / out - 0.5), each step rounded (a division sits in the middle,
 * so nothing contracts). Nearest sampling truncates it. */
static float orc_ref_source(int d, int in_size, int out_size) {
    float a = (float)d + 0.5f;
    float b = a * (float)in_size;
    float c = b / (float)out_size;
    float r = c - 0.5f;
    return fmaxf(0.f, r);
}

void orc_letterbox_nv12(const orc_nv12_t* frames, int n, int dst_h, int dst_w,
                        const float mean[3], const float stdv[3], int swap_rb, float pad_value,
                        int matrix, int sampling, float* out, int threads) {
    orc_letterbox_nv12_fit(frames, n, dst_h, dst_w, mean, stdv, swap_rb, pad_value, matrix, sampling, 0, out,
                           threads);
}

void orc_letterbox_nv12_fit(const orc_nv12_t* frames, int n, int dst_h, int dst_w,
                            const float mean[3], const float stdv[3], int swap_rb, float pad_value,
                            int matrix, int sampling, int cpp_fit, float* out, int threads) {
    const size_t plane = (size_t)dst_h * (size_t)dst_w;
    orc_yuv_t m = orc_matrix(matrix);
    float pad_out[3];
    for (int c = 0; c < 3; ++c) pad_out[c] = (pad_value - mean[c]) / stdv[c];
    int nt = orc_threads(threads);
#pragma omp parallel for collapse(2) schedule(static) num_threads(nt)
    for (int i = 0; i < n; ++i) {
        for (int y = 0; y < dst_h; ++y) {
            const orc_nv12_t* fr = &frames[i];
            orc_fit_t fit = orc_fit_of(cpp_fit, fr->h, fr->w, dst_h, dst_w);
            float rh = (float)fr->h / (float)fit.new_h;
            float rw = (float)fr->w / (float)fit.new_w;
            float* img = out + (size_t)i * 3 * plane;
            int inside_y = y >= fit.pad_y && y < fit.pad_y + fit.new_h;
            for (int x = 0; x < dst_w; ++x) {
                int inside = inside_y && x >= fit.pad_x && x < fit.pad_x + fit.new_w;
                if (!inside) {
                    for (int c = 0; c < 3; ++c) img[c * plane + (size_t)y * dst_w + x] = pad_out[c];
                    continue;
                }
                float v[3];
                if (sampling == 0) {
                    float sy = orc_ref_source(y - fit.pad_y, fr->h, fit.new_h);
                    float sx = orc_ref_source(x - fit.pad_x, fr->w, fit.new_w);
                    int yi = (int)sy, xi = (int)sx;
                    if (yi > fr->h - 1) yi = fr->h - 1;
                    if (xi > fr->w - 1) xi = fr->w - 1;
                    orc_nv12_bgr(fr, m, yi, xi, v);
                } else {
                    orc_tap_t ty = orc_source_tap(rh, y - fit.pad_y, fr->h);
                    orc_tap_t tx = orc_source_tap(rw, x - fit.pad_x, fr->w);
                    float p00[3], p01[3], p10[3], p11[3];
                    orc_nv12_bgr(fr, m, ty.i0, tx.i0, p00);
                    orc_nv12_bgr(fr, m, ty.i0, tx.i1, p01);
                    orc_nv12_bgr(fr, m, ty.i1, tx.i0, p10);
                    orc_nv12_bgr(fr, m, ty.i1, tx.i1, p11);
                    for (int s = 0; s < 3; ++s) v[s] = orc_blend(ty, tx, p00[s], p01[s], p10[s], p11[s]);
                }
                for (int c = 0; c < 3; ++c) {
                    int sc = swap_rb ? 2 - c : c;
                    img[c * plane + (size_t)y * dst_w + x] = (v[sc] - mean[c]) / stdv[c];
                }
            }
        }
    }
}

/* ---------------------------------------------------------------------------------------
 * Detector decode. Reference: src/shipinfer/topology/elements/detections.py:423-515
 *   rows[:count]; keep = flatnonzero(scores >= thr)         (float32 compare; NaN fails)
 *   cap: argsort(scores[keep], stable)[::-1][:max]           (ties: the HIGHER row first)
 *   order = keep[argsort(scores[keep], stable)[::-1]]        (the same order)
 *   xs -= pad_x; xs *= inv   with inv = 1.0 / scale in double, used as a float32 (numpy 2
 *                            takes a Python float operand as a float32 for a float32 array)
 *   np.clip(xs, 0.0, width): x < lo ? lo : (x > hi ? hi : x)  (keeps -0.0 and NaN)
 *   class: float32 -> int32, INT_MIN for NaN, infinities and values out of range (as numpy
 *   does on x86-64).
 * ------------------------------------------------------------------------------------- */
typedef struct {
    float score;
    int idx;
} orc_rank_t;

static int orc_rank_desc(const void* a, const void* b) {
    const orc_rank_t* x = (const orc_rank_t*)a;
    const orc_rank_t* y = (const orc_rank_t*)b;
    if (x->score > y->score) return -1;
    if (x->score < y->score) return 1;
    return x->idx > y->idx ? -1 : (x->idx < y->idx ? 1 : 0); /* -0.0 == +0.0: by index */
}

static float orc_clip(float v, float hi) { return v < 0.0f ? 0.0f : (v > hi ? hi : v); }

static int32_t orc_f32_to_i32(float v) {
    if (v != v || v >= 2147483648.0f || v < -2147483648.0f) return INT32_MIN;
    return (int32_t)v; /* truncation toward zero */
}

int orc_decode(const float* rows, int R, int count, float scale, float pad_x, float pad_y,
               int frame_h, int frame_w, float score_threshold, int max_det, float* boxes,
               float* scores, int32_t* class_ids, int* discarded) {
    const int total = count < 0 ? R : (count > R ? R : count);
    orc_rank_t* e = (orc_rank_t*)malloc(sizeof(orc_rank_t) * (size_t)(total > 0 ? total : 1));
    int n = 0;
    for (int i = 0; i < total; ++i) {
        const float s = rows[(size_t)i * 6 + 4];
        if (s >= score_threshold) {
            e[n].score = s;
            e[n].idx = i;
            ++n;
        }
    }
    qsort(e, (size_t)n, sizeof(orc_rank_t), orc_rank_desc);
    const int m = n < max_det ? n : (max_det > 0 ? max_det : 0);
    const double invd = scale != 0.0f ? 1.0 / (double)scale : 1.0;
    const float inv = (float)invd;
    for (int q = 0; q < m; ++q) {
        const float* r = rows + (size_t)e[q].idx * 6;
        for (int c = 0; c < 4; ++c) {
            float v = r[c] - ((c & 1) ? pad_y : pad_x);
            v = v * inv;
            if (frame_h >= 0) v = orc_clip(v, (c & 1) ? (float)frame_h : (float)frame_w);
            boxes[(size_t)q * 4 + c] = v;
        }
        scores[q] = r[4];
        class_ids[q] = orc_f32_to_i32(r[5]);
    }
    free(e);
    *discarded = total - m;
    return m;
}

/* ---------------------------------------------------------------------------------------
 * Mask area. Reference: csrc/shipinfer/runtime/ops.cu:196-255 (mask_area_kernel) and
 * :418-458 (mask_area_into)
 *   best = 0; for c: if (score[c] > score[best]) best = c      (first strict maximum)
 *   score[best] < score_threshold -> area 0
 *   cut = std::log(t / (1 - t)) in float; cell_px = float(h) * float(w) / float(cells)
 *   logit = 0; for m: logit += coef[m] * plane[m][cell]       (nvcc fuses: one fma per m)
 *   area = float(count of logit >= cut) * cell_px
 * ------------------------------------------------------------------------------------- */
void orc_mask_area(const float* rows, int crops, int candidates, int stride, int prefix,
                   const float* protos, int channels, int cells, float score_threshold,
                   float mask_threshold, int crop_height, int crop_width, float* areas, int threads) {
    const float cut = logf(mask_threshold / (1.f - mask_threshold));
    const float cell_px = (float)crop_height * (float)crop_width / (float)cells;
    int nt = orc_threads(threads);
    (void)nt;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nt)
    for (int k = 0; k < crops; ++k) {
        const float* cand = rows + (size_t)k * candidates * stride;
        int best = 0;
        for (int c = 1; c < candidates; ++c)
            if (cand[(size_t)c * stride + 4] > cand[(size_t)best * stride + 4]) best = c;
        const float* chosen = cand + (size_t)best * stride;
        if (chosen[4] < score_threshold) {
            areas[k] = 0.f;
            continue;
        }
        const float* planes = protos + (size_t)k * channels * cells;
        int inside = 0;
        for (int cell = 0; cell < cells; ++cell) {
            float logit = 0.f;
            for (int m = 0; m < channels; ++m) logit = fmaf(chosen[prefix + m], planes[(size_t)m * cells + cell], logit);
            if (logit >= cut) ++inside;
        }
        areas[k] = (float)inside * cell_px;
    }
}

void orc_decode_batched(const float* rows, int B, int R, const int32_t* counts, const float* scales,
                        const float* pads, const int32_t* frame_hw, float score_threshold,
                        int max_det, float* boxes, float* scores, int32_t* class_ids,
                        int32_t* out_counts, int32_t* discarded, int threads) {
    const int cap = max_det > 0 ? max_det : 0;
    int nt = orc_threads(threads);
    (void)nt;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nt)
    for (int b = 0; b < B; ++b) {
        int d = 0;
        const int m = orc_decode(rows + (size_t)b * R * 6, R, counts ? counts[b] : -1, scales[b], pads[2 * b],
                                 pads[2 * b + 1], frame_hw ? frame_hw[2 * b] : -1,
                                 frame_hw ? frame_hw[2 * b + 1] : -1, score_threshold, max_det,
                                 boxes + (size_t)b * cap * 4, scores + (size_t)b * cap,
                                 class_ids + (size_t)b * cap, &d);
        out_counts[b] = m;
        discarded[b] = d;
    }
}

/* ---------------------------------------------------------------------------------------
 * NV12 crop-resize. Reference: csrc/shipinfer/runtime/ops.cu:260-318 (nv12_crop_resize_kernel)
 *   corners clipped to [0, W-1] / [0, H-1] in float, truncated; non-positive extent: zeros
 *   l = max(0, ((d + 0.5) * extent) / dst - 0.5), p0 = min((int)l, extent - 1),
 *   p1 = min(p0 + 1, extent - 1), w = l - p0
 *   value = (p00*(1-wx) + p01*wx)*(1-wy) + (p10*(1-wx) + p11*wx)*wy, where nvcc fuses each
 *   "a*b + c*d" into fma(a, b, c*d); out = value / 255, channel order flipped by swap_rb.
 * Boxes per frame as box_frame gives (out of range: zeros). out: float32 [n,3,dst_h,dst_w].
 * ------------------------------------------------------------------------------------- */
static int orc_clip_i(float v, float hi) { return (int)fminf(fmaxf(v, 0.f), hi); }

void orc_crop_nv12(const orc_nv12_t* frames, int n_frames, const float* boxes,
                   const int32_t* box_frame, int n_boxes, int dst_h, int dst_w, int swap_rb,
                   float* out, int threads) {
    const orc_yuv_t m = orc_matrix(601);
    const int64_t plane = (int64_t)dst_h * dst_w;
    int nt = orc_threads(threads);
    (void)nt;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nt)
    for (int n = 0; n < n_boxes; ++n) {
        float* o = out + (int64_t)n * 3 * plane;
        const int fi = box_frame ? box_frame[n] : 0;
        if (fi < 0 || fi >= n_frames) {
            memset(o, 0, sizeof(float) * 3 * (size_t)plane);
            continue;
        }
        const orc_nv12_t* f = &frames[fi];
        const float* b = boxes + (size_t)n * 4;
        const int x1 = orc_clip_i(b[0], (float)f->w - 1.f), y1 = orc_clip_i(b[1], (float)f->h - 1.f);
        const int bw = orc_clip_i(b[2], (float)f->w - 1.f) - x1, bh = orc_clip_i(b[3], (float)f->h - 1.f) - y1;
        if (bw <= 0 || bh <= 0) {
            memset(o, 0, sizeof(float) * 3 * (size_t)plane);
            continue;
        }
        for (int y = 0; y < dst_h; ++y) {
            const float ly = fmaxf(0.f, orc_ref_source(y, bh, dst_h));
            const int py0 = (int)ly < bh - 1 ? (int)ly : bh - 1;
            const int py1 = py0 + 1 < bh - 1 ? py0 + 1 : bh - 1;
            const float wy = ly - (float)py0, omy = 1.f - wy;
            for (int x = 0; x < dst_w; ++x) {
                const float lx = fmaxf(0.f, orc_ref_source(x, bw, dst_w));
                const int px0 = (int)lx < bw - 1 ? (int)lx : bw - 1;
                const int px1 = px0 + 1 < bw - 1 ? px0 + 1 : bw - 1;
                const float wx = lx - (float)px0, omx = 1.f - wx;
                float q00[3], q01[3], q10[3], q11[3];
                orc_nv12_bgr(f, m, y1 + py0, x1 + px0, q00);
                orc_nv12_bgr(f, m, y1 + py0, x1 + px1, q01);
                orc_nv12_bgr(f, m, y1 + py1, x1 + px0, q10);
                orc_nv12_bgr(f, m, y1 + py1, x1 + px1, q11);
                for (int c = 0; c < 3; ++c) {
                    const int sc = swap_rb ? 2 - c : c;
                    const float top = fmaf(q00[sc], omx, q01[sc] * wx);
                    const float bot = fmaf(q10[sc], omx, q11[sc] * wx);
                    const float value = fmaf(top, omy, bot * wy);
                    o[c * plane + (int64_t)y * dst_w + x] = value / 255.f;
                }
            }
        }
    }
}
