/*
 * shipk — B200-native (sm_100a) data-plane image kernels for ShipInfer, behind a C ABI.
 *
 * This header is the drop-in boundary. Every entry point is plain C: pointers, sizes and
 * status codes, no C++ or torch types. The ShipInfer image-ops seam (the `ImageOps` ABC in
 * the reference, src/shipinfer/runtime/ops/base.py:71-180) reaches these functions through
 * the Python shim in shipinfer_b200/ (or through any FFI that can call C).
 *
 * Conventions
 *   - Every call returns SHIPK_OK (0) or a positive SHIPK_E* code. On failure,
 *     shipk_last_error() returns a message for the calling thread. No exception ever
 *     crosses this boundary.
 *   - Device pointers must belong to the calling thread's current CUDA device. Calls that
 *     launch kernels enqueue them on `stream` (a cudaStream_t; NULL is the legacy default
 *     stream) and return without synchronising, unless documented otherwise.
 *   - Frames are uint8 BGR, HWC, rows `pitch` bytes apart (pitch >= 3 * width).
 *   - Outputs are NCHW, channel order RGB when swap_rb != 0 (the source is BGR), and every
 *     output value is (v - mean[c]) / std[c] with v in the 0-255 pixel scale, as
 *     NormalizeParams defines it (reference base.py:32-44).
 *   - Nothing here allocates device memory except shipk_ctx_create() and the staging it
 *     grows for host-frame calls; all other scratch is passed in by the caller.
 */
#ifndef SHIPK_H
#define SHIPK_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SHIPK_API __attribute__((visibility("default")))
#else
#define SHIPK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define SHIPK_OK 0
#define SHIPK_EINVAL 1   /* an argument is out of its documented range */
#define SHIPK_EDEVICE 2  /* a pointer is not device memory of the current device */
#define SHIPK_ECUDA 3    /* a CUDA runtime call failed; the message names it */
#define SHIPK_ERANGE 4   /* a size exceeds what this build supports */
#define SHIPK_ENOMEM 5   /* a caller-provided buffer is too small */

#define SHIPK_DTYPE_F32 0
#define SHIPK_DTYPE_F16 1

/* One uint8 BGR HWC frame in device memory. */
typedef struct {
    const uint8_t* data;
    int32_t height;
    int32_t width;
    int64_t pitch; /* bytes between rows */
} shipk_frame_u8;

/* One NV12 frame in device memory: a luma plane of `height` rows, then an interleaved UV
 * plane of ceil(height/2) rows starting `uv_offset` bytes after `luma`; both planes use
 * `pitch` bytes per row. */
typedef struct {
    const uint8_t* luma;
    int32_t height;
    int32_t width;
    int64_t pitch;
    int64_t uv_offset;
} shipk_frame_nv12;

/* Where a frame landed on the letterbox canvas (reference LetterboxMap, ops.h:30-36, and
 * TorchImageOps' (scale, pad, extent) triple, torch_ops.py:373-394). */
typedef struct {
    float scale;   /* min(dst_h / src_h, dst_w / src_w), computed in double, stored float */
    int32_t pad_x; /* (dst_w - new_w) // 2 */
    int32_t pad_y; /* (dst_h - new_h) // 2 */
    int32_t new_w; /* max(1, round_half_even(src_w * scale)) */
    int32_t new_h;
} shipk_letterbox_map;

/* ---- probes: reference runtime/native.py:96-150 reads these off shipvision._C ---------- */

/* Version string of this build (static storage). Replaces `shipvision._C.__version__`. */
SHIPK_API const char* shipk_version(void);
/* 1 when this build has sm_100a kernels and a device can run them, else 0.
 * Replaces `shipvision._C.cuda_available()` (native.py:129-148, native_ops.py:112-124). */
SHIPK_API int shipk_cuda_available(void);
/* Visible CUDA devices (0 when none). Replaces `shipvision._C.device_count()`. */
SHIPK_API int shipk_device_count(void);
/* Copy the calling thread's last error message into buf (always NUL-terminated when
 * len > 0). Returns the full message length. */
SHIPK_API size_t shipk_last_error(char* buf, size_t len);

/* ---- geometry -------------------------------------------------------------------------- */

/* The letterbox placement alone. Replaces `letterbox_fit` (reference ops.h:38-39) with the
 * Python plane's arithmetic (torch_ops.py:373-379: double precision, round half to even). */
SHIPK_API int shipk_letterbox_fit(int src_h, int src_w, int dst_h, int dst_w, shipk_letterbox_map* out);

/* ---- fused letterbox ------------------------------------------------------------------- */

/* Letterbox n device frames into `out` (NCHW [n,3,dst_h,dst_w] of out_dtype, contiguous,
 * out_nbytes >= its size): bilinear resize with half-pixel centres, pad, BGR->RGB if
 * swap_rb, normalise, in one launch. pad_value is in the 0-255 pixel scale and is
 * normalised like a pixel. maps_out (host, nullable) receives n placements.
 * Replaces `shipvision._C.ImageOps.letterbox_into` (reference native_ops.py:159-170) and
 * the C++ plane's `letterbox_into` (ops.h:41-43, ops.cu:363-374), batched. */
SHIPK_API int shipk_letterbox_u8(const shipk_frame_u8* frames, int n, void* out, int out_dtype,
                       size_t out_nbytes, int dst_h, int dst_w, const float mean[3],
                       const float std[3], int swap_rb, float pad_value,
                       shipk_letterbox_map* maps_out, void* stream);

/* NV12 frames -> letterboxed RGB. matrix: 601 or 709 (limited range). sampling:
 * 0 = nearest at the reference NV12 kernel's source coordinate (its parity mode),
 * 1 = bilinear with half-pixel centres, taps converted to RGB then blended.
 * Layout is refused, as the reference refuses it (ops.cu:325-339), when pitch < width or
 * uv_offset < pitch * height.
 * Replaces the C++ plane's `nv12_letterbox_into` (ops.h:67-70, ops.cu:388-401), batched. */
SHIPK_API int shipk_letterbox_nv12(const shipk_frame_nv12* frames, int n, void* out, int out_dtype,
                         size_t out_nbytes, int dst_h, int dst_w, const float mean[3],
                         const float std[3], int swap_rb, float pad_value, int matrix,
                         int sampling, shipk_letterbox_map* maps_out, void* stream);

/* ---- batched ROI crop-resize ----------------------------------------------------------- */

/* Crop box i ([x1,y1,x2,y2] float32 in frame pixels, device array [n_boxes,4]) out of
 * frames[box_frame[i]] (device int32 [n_boxes]; NULL means every box is on frames[0]) and
 * resize it to dst_h x dst_w into out (NCHW [n_boxes,3,dst_h,dst_w]). Geometry of
 * TorchImageOps.crop_batch (torch_ops.py:405-507): clip then truncate, patch [x1,x2),
 * half-pixel centres in patch coordinates, far neighbour clamped inside the patch, torch.lerp
 * blending; a degenerate box (or a box_frame out of [0, n_frames)) yields (0 - mean) / std.
 * One launch for every box of every frame.
 * Replaces `shipvision._C.ImageOps.crop_batch` (native_ops.py:199-215) and the C++ plane's
 * `crop_resize_into` (ops.h:52-54, ops.cu:376-386). */
SHIPK_API int shipk_crop_u8(const shipk_frame_u8* frames, int n_frames, const float* boxes,
                  const int32_t* box_frame, int n_boxes, void* out, int out_dtype,
                  size_t out_nbytes, int dst_h, int dst_w, const float mean[3],
                  const float std[3], int swap_rb, void* stream);

/* Crops straight from NV12 decoder surfaces, every box of every frame in one launch. Replaces
 * the reference's nv12_crop_resize_into (csrc/shipinfer/runtime/ops.h:86-89, ops.cu:260-318
 * and 402-416), which takes one frame per call: same box geometry, taps, BT.601 conversion,
 * blend (as nvcc contracts it) and value / 255, bit for bit. frames: NV12 surfaces with the
 * reference's layout rule (stride >= width, uv_offset >= stride * height; SHIPK_EINVAL else);
 * boxes: device float [n_boxes,4] xyxy; box_frame: device int32 [n_boxes] frame of each box
 * (NULL: all frame 0; out of range: a crop of zeros). out: device [n_boxes,3,dst_h,dst_w]
 * float32 (or float16, rounded from the float32 value). */
SHIPK_API int shipk_crop_nv12(const shipk_frame_nv12* frames, int n_frames, const float* boxes,
                              const int32_t* box_frame, int n_boxes, void* out, int out_dtype,
                              size_t out_nbytes, int dst_h, int dst_w, int swap_rb, void* stream);

/* ---- device NMS ------------------------------------------------------------------------ */

/* Scratch bytes shipk_nms needs for this shape. */
SHIPK_API size_t shipk_nms_workspace_bytes(int batch, int n, int num_classes, int class_aware,
                                 int max_det);

/* Greedy NMS over `batch` images of `n` candidates (device arrays: boxes [batch,n,4] xyxy,
 * scores [batch,n], classes [batch,n] int32 or NULL). Semantics of NumpyImageOps.nms
 * (reference numpy_ops.py:120-155) in float32: candidates are scores >= score_threshold,
 * visited by score descending with ties to the lower index, a candidate survives when its
 * IoU with every kept box is <= iou_threshold. class_aware != 0 suppresses within each class
 * in [0, num_classes) (other class ids are ignored) and merges the survivors by (score
 * descending, index ascending). keep (device int64 [batch,max_det]) is -1 padded; counts
 * (device int32 [batch]). workspace: device scratch of shipk_nms_workspace_bytes(). Class-aware
 * with 2..8 classes and num_classes x max_det <= 8192 merges each image's classes inside one
 * thread-block cluster and leaves the workspace untouched; otherwise the classes meet through
 * the workspace, whose arrival counters the call clears on `stream` first. One launch (after
 * that clear, when there is one); no host round trip. Replaces `shipvision._C.ImageOps.nms`
 * (native_ops.py:217-232), batched and class-aware. */
SHIPK_API int shipk_nms(const float* boxes, const float* scores, const int32_t* classes, int batch,
              int n, int num_classes, int class_aware, float iou_threshold,
              float score_threshold, int max_det, int64_t* keep, int32_t* counts,
              void* workspace, size_t workspace_bytes, void* stream);

/* The launch shipk_nms (and shipk_nms_static) makes for this shape on the current device, for
 * capacity planning: *ctas thread blocks of 1024 threads, in thread-block clusters of *cluster
 * (1: no cluster). An image x class segment runs on one CTA, joined by up to 7 helper CTAs that
 * share its first round's pair tests while the launch's clusters all fit on the device at once.
 * 0 CTAs: nothing is launched (batch, n or max_det is 0). No reference counterpart. */
SHIPK_API int shipk_nms_launch_shape(int batch, int n, int num_classes, int class_aware, int max_det,
                           int* ctas, int* cluster);

/* ---- detector decode ------------------------------------------------------------------- */

/* Detector output -> source-frame detections for a batch of frames, on the device: the
 * reference's decode_detections (src/shipinfer/topology/elements/detections.py:423-515) per
 * frame, in its numpy float32 arithmetic. rows: device float [batch, rows_per_frame, 6]
 * ([x1,y1,x2,y2,score,class] in letterboxed pixels). counts: device int32 [batch], rows the
 * detector filled (truncation), or NULL. scales [batch], pads [batch,2] (x, y): the letterbox
 * placement the preprocess reported (shipk_letterbox_map). frame_hw: device int32 [batch,2]
 * source (h, w) to clip to, or NULL. Keeps score >= score_threshold, caps at max_detections
 * (<= 4096, else SHIPK_ERANGE) by score descending with ties to the higher row, writes boxes
 * [batch,max_detections,4] as (v - pad) * float(1/scale) clipped, scores, class_ids (float ->
 * int32 as numpy casts), out_counts [batch] and discarded [batch] (rows not kept); slots past
 * a frame's count hold zeros and class -1. Replaces the host loop of detect.py:146-178 (and
 * stages.cpp:153-172's C++ twin) with one launch. */
SHIPK_API int shipk_decode_detections(const float* rows, int batch, int rows_per_frame,
                                      const int32_t* counts, const float* scales, const float* pads,
                                      const int32_t* frame_hw, float score_threshold,
                                      int max_detections, float* boxes, float* scores,
                                      int32_t* class_ids, int32_t* out_counts, int32_t* discarded,
                                      void* stream);

/* ---- segmenter mask area --------------------------------------------------------------- */

/* One area per crop from a segmenter's outputs, on the device. Replaces the reference's
 * mask_area_into (csrc/shipinfer/runtime/ops.h:117-120, ops.cu:196-255 and 418-458): same
 * arguments, same refusals (SHIPK_EINVAL where it throws ConfigError), same results. rows:
 * device float [count, candidates, stride], score in column 4, mask coefficients in
 * [prefix, stride); protos: device float [count, channels, cells] with channels = stride -
 * prefix. Per crop: the strongest row (first strict maximum of the scores); a score below
 * score_threshold gives 0; else the number of cells whose logit (coefficients against planes,
 * one fused multiply-add per channel in order) is >= log(t / (1 - t)), t = mask_threshold in
 * (0, 1), times crop_height * crop_width / cells, into areas (device float [count]). Channels
 * <= 256 (else SHIPK_ERANGE). Beyond the reference's refusals, a negative prefix or a row of
 * fewer than 5 floats is SHIPK_EINVAL (reads outside the rows). A cluster of 8 CTAs per crop;
 * one launch for the batch. */
SHIPK_API int shipk_mask_area(const float* rows, int candidates, int stride, int prefix,
                              const float* protos, int channels, int cells, int count,
                              float score_threshold, float mask_threshold, int crop_height,
                              int crop_width, float* areas, void* stream);

/* ---- verification ---------------------------------------------------------------------- */

/* No counterpart in the reference. The kernels normalise (v - mean) / std with a correctly
 * rounded division built from RN(1/std) and fused multiply-adds (Markstein's method) when
 * mean and std lie in [2^-20, 2^20] in magnitude (mean may be 0), else with IEEE division.
 * This evaluates both for every float v in [0, 256) — every value normalisation can receive —
 * (and, for a std whose RN(1/std) is within 2^-25 relative of 1/std, the shorter one-correction
 * form the crop kernel then uses, an input counting if either form differs)
 * and adds to result[0] (device uint64) the number of inputs whose results differ in any bit,
 * lowering result[1] to the bit pattern of the first. The caller zeroes result[0] and sets
 * result[1] to UINT64_MAX. SHIPK_ERANGE when (mean, std) is outside the fast range. About a
 * millisecond on a B200. */
SHIPK_API int shipk_normalise_check(float mean, float std, unsigned long long* result, void* stream);

/* Allocation-free variant of shipk_nms. No counterpart in the reference. For callers that
 * hold no device buffer to lend as a workspace and may not make one per call: a C++ stage on a
 * decoder thread bound to a fixed memory budget, or a real-time loop that cannot afford
 * cudaMalloc's implicit device synchronisation. Same arguments, semantics and results as
 * shipk_nms, minus the workspace: the scratch is a static device array of 1 MiB per device
 * inside this library (enough for batch x segments x max_det up to about 260,000, e.g. 16
 * images x 2 classes x 4096, or 64 x 4 x 1000); a call that needs more returns SHIPK_ERANGE
 * and changes nothing. The first call on a device takes the scratch's address
 * (cudaGetSymbolAddress) with that device current and sets the kernel's shared-memory limit:
 * make it before any stream capture on that device. When the classes meet through the scratch
 * (see shipk_nms), each call clears the scratch's arrival counters on `stream` (cudaMemsetAsync)
 * before the launch; nothing else must start at zero.
 * One scratch per device: calls that overlap on one device (concurrent streams or host threads)
 * race on it and must be serialised by the caller. Nothing here allocates. The scratch's
 * address and the shared-memory setting are kept per device for the life of the process: a
 * cudaDeviceReset destroys the context they belong to, so do not call this across one. */
SHIPK_API int shipk_nms_static(const float* boxes, const float* scores, const int32_t* classes,
                               int batch, int n, int num_classes, int class_aware,
                               float iou_threshold, float score_threshold, int max_det,
                               int64_t* keep, int32_t* counts, void* stream);

/* ---- the C++ data plane's per-frame calls -----------------------------------------------
 * C twins of the reference's C++ data-plane functions (csrc/shipinfer/runtime/ops.h:38-120,
 * ops.cu:359-416), argument for argument, for its callers (pipeline/graph/pixels.cpp:18-43):
 * one device frame per call (BGR frames tight, pitch = width * 3), float32 NCHW out (the
 * caller's TensorRT binding, no size given: the caller guarantees [count or 1, 3, dst_h,
 * dst_w]), value / 255, `pad_value` the bars' OUTPUT value. shipinfer_b200/dataplane/
 * ops_shipk.cpp implements ops.h on these. Numerics: the BGR calls compute the Python plane's
 * formulation (TorchImageOps, torch_ops.py:349-507), which the reference's C++ kernels
 * approximate (their own comments name it as the one to agree with); the NV12 calls are the
 * reference kernels' own arithmetic, bit for bit (BT.601 limited range, nearest for the
 * letterbox). NV12 layout refusals are the reference's require_nv12_layout, wording included
 * (SHIPK_EINVAL where it throws ConfigError); count <= 0 is a no-op before any check, as there.
 * mask_area_into's twin is shipk_mask_area (same arguments). The letterbox calls place the frame
 * with the data plane's float32 rule (shipk_dp_letterbox_fit) and return that placement. */
/* The data plane's letterbox placement. Replaces `letterbox_fit` / `fit` of the C++ plane
 * (reference ops.h:38-39, ops.cu:341-356): float32 scale min(dst_w/src_w, dst_h/src_h), extents
 * max(1, nearbyint(float(src) * scale)), bars (dst - new) / 2. It differs from
 * shipk_letterbox_fit (the Python plane's double-precision rule) for some sizes: 180x1280 into
 * 224x224 is 31 rows there and 32 here. */
SHIPK_API int shipk_dp_letterbox_fit(int src_h, int src_w, int dst_h, int dst_w, shipk_letterbox_map* out);
SHIPK_API int shipk_dp_letterbox_into(const uint8_t* src_device, int src_h, int src_w, float* dst_device,
                                      int dst_h, int dst_w, int swap_rb, float pad_value,
                                      shipk_letterbox_map* map_out, void* stream);
SHIPK_API int shipk_dp_crop_resize_into(const uint8_t* src_device, int src_h, int src_w,
                                        const float* boxes_device, int count, float* dst_device, int dst_h,
                                        int dst_w, int swap_rb, void* stream);
SHIPK_API int shipk_dp_nv12_letterbox_into(const uint8_t* nv12_device, int src_h, int src_w, int stride,
                                           size_t uv_offset, float* dst_device, int dst_h, int dst_w,
                                           int swap_rb, float pad_value, shipk_letterbox_map* map_out,
                                           void* stream);
SHIPK_API int shipk_dp_nv12_crop_resize_into(const uint8_t* nv12_device, int src_h, int src_w, int stride,
                                             size_t uv_offset, const float* boxes_device, int count,
                                             float* dst_device, int dst_h, int dst_w, int swap_rb,
                                             void* stream);

/* ---- host-frame entry points (the shipvision._C surface takes numpy frames) ------------- */

typedef struct shipk_ctx shipk_ctx;

/* A per-thread context bound to one device: owns its device staging for host frames and
 * an event to order reuse. Reference: one ImageOps per thread (thread_local.py:14-24). */
SHIPK_API int shipk_ctx_create(int device, shipk_ctx** out);
SHIPK_API void shipk_ctx_destroy(shipk_ctx* ctx);

/* One uint8 BGR HWC frame in host memory (pinned memory makes the copy asynchronous). */
typedef struct {
    const uint8_t* data;
    int32_t height;
    int32_t width;
    int64_t pitch;
} shipk_host_frame_u8;

/* Letterbox host frames into device `out`: copies to the device only the source rows the
 * resize reads (e.g. one row in three at 1080p -> 640), then runs shipk_letterbox_u8 on
 * `stream`. Returns once the copies and the launch are enqueued; the frames must stay valid
 * and unmodified until `stream` reaches this work (pageable frames are copied synchronously
 * by CUDA and are safe to reuse on return). The context's staging is reused by its next
 * call only after this call's kernel has finished with it.
 * Replaces `shipvision._C.ImageOps.letterbox_into` with host frames (native_ops.py:159-170). */
SHIPK_API int shipk_ctx_letterbox_host(shipk_ctx* ctx, const shipk_host_frame_u8* frames, int n,
                             void* out, int out_dtype, size_t out_nbytes, int dst_h, int dst_w,
                             const float mean[3], const float std[3], int swap_rb,
                             float pad_value, shipk_letterbox_map* maps_out, void* stream);

/* Crop from one host frame with host boxes into device `out`. Copies only the frame rows
 * the boxes' samples read. Replaces `shipvision._C.ImageOps.crop_batch` (native_ops.py:
 * 199-215) up to the result's trip home, which the caller chooses. */
SHIPK_API int shipk_ctx_crop_host(shipk_ctx* ctx, const shipk_host_frame_u8* frame, const float* boxes,
                        int n_boxes, void* out, int out_dtype, size_t out_nbytes, int dst_h,
                        int dst_w, const float mean[3], const float std[3], int swap_rb,
                        void* stream);

/* Class-agnostic or class-aware NMS on host arrays for `batch` images, returning host
 * results: keep (host int64 [batch,max_det], -1 padded) and counts (host int32 [batch]).
 * Synchronises `stream` before returning. Replaces `shipvision._C.ImageOps.nms`
 * (native_ops.py:217-232). */
SHIPK_API int shipk_ctx_nms_host(shipk_ctx* ctx, const float* boxes, const float* scores,
                       const int32_t* classes, int batch, int n, int num_classes,
                       int class_aware, float iou_threshold, float score_threshold,
                       int max_det, int64_t* keep, int32_t* counts, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SHIPK_H */
