// Internal launch interface between the C ABI (abi.cu) and the kernel files.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/shipk.h"

namespace shipk {

constexpr int kMaxBatch = 64;  // frames per launch; larger letterbox batches are split

struct Status {
    int code;
    const char* message;  // static string, or null when code == SHIPK_OK
};

// One source frame as the kernels see it: BGR rows, or an NV12 luma plane with its chroma
// plane uv_offset bytes later. row_map, when set, is a device array giving for each source
// row the row of `data` that holds it (frames staged from the host carry only the rows the
// resize reads).
// fit_f32 selects the placement rule: 0 is the Python plane's (letterbox_fit), 1 the C++ data
// plane's (letterbox_fit_f32).
struct FrameView {
    const uint8_t* data;
    const int32_t* row_map;
    int height, width;
    int64_t pitch;
    int64_t uv_offset;
    int fit_f32;
};

struct Fit {
    float scale;
    int pad_x, pad_y, new_w, new_h;
};

// The Python plane's placement (torch_ops.py:373-379), in double precision as Python computes it.
int letterbox_fit(int src_h, int src_w, int dst_h, int dst_w, Fit* out);
// The C++ data plane's placement (csrc/shipinfer/runtime/ops.cu:341-356), in float32: the scale
// is min(dst_w/src_w, dst_h/src_h) in float and each extent nearbyint(float(src) * scale). The
// two rules give different extents for some sizes (180x1280 -> 224x224: 31 rows in double, 32
// in float32).
int letterbox_fit_f32(int src_h, int src_w, int dst_h, int dst_w, Fit* out);
// The placement rule a frame view asks for.
inline int frame_fit(const FrameView& f, int dst_h, int dst_w, Fit* out) {
    return f.fit_f32 ? letterbox_fit_f32(f.height, f.width, dst_h, dst_w, out)
                     : letterbox_fit(f.height, f.width, dst_h, dst_w, out);
}

// pad_out: when set, the bars' output values per channel as given (the C++ data plane's
// pad_value is an output value); else (pad_value - mean) / std.
Status launch_letterbox(const FrameView* frames, int n, void* out, int out_dtype, int dst_h,
                        int dst_w, const float mean[3], const float stdv[3], int swap_rb,
                        float pad_value, bool nv12, int matrix, int sampling,
                        cudaStream_t stream, const float* pad_out = nullptr);

Status launch_crop(const FrameView* frames, int n_frames, const float* boxes,
                   const int32_t* box_frame, int n_boxes, void* out, int out_dtype, int dst_h,
                   int dst_w, const float mean[3], const float stdv[3], int swap_rb,
                   cudaStream_t stream);

// Crops straight from NV12 surfaces (the reference's nv12_crop_resize_into), batched over frames.
Status launch_crop_nv12(const FrameView* frames, int n_frames, const float* boxes, const int32_t* box_frame,
                        int n_boxes, void* out, int out_dtype, int dst_h, int dst_w, int swap_rb,
                        cudaStream_t stream);

size_t nms_workspace_bytes(int batch, int n, int num_classes, int class_aware, int max_det);

// The CTAs and cluster size launch_nms uses for this shape on the current device.
Status nms_launch_shape(int batch, int num_classes, int class_aware, int max_det, int* ctas, int* cluster);

// zero_arrivals: clear the class-aware arrival counters on `stream` before the launch.
Status launch_nms(const float* boxes, const float* scores, const int32_t* classes, int batch,
                  int n, int num_classes, int class_aware, float iou_thr, float score_thr,
                  int max_det, int64_t* keep, int32_t* counts, void* workspace,
                  size_t workspace_bytes, bool zero_arrivals, cudaStream_t stream);

// Detector rows [batch, R, 6] -> detections [batch, max_det] (decode_detections per frame).
Status launch_decode(const float* rows, int batch, int R, const int32_t* counts, const float* scales,
                     const float* pads, const int32_t* frame_hw, float score_threshold, int max_det,
                     float* boxes, float* scores, int32_t* classes, int32_t* out_counts, int32_t* discarded,
                     cudaStream_t stream);

// Mask area per crop (the reference's mask_area_into); cut and cell area computed here.
Status launch_mask_area(const float* rows, int crops, int candidates, int stride, int prefix,
                        const float* protos, int channels, int cells, float score_threshold,
                        float mask_threshold, int crop_height, int crop_width, float* areas,
                        cudaStream_t stream);

// The allocation-free NMS entry point's scratch: a static device array of
// nms_static_capacity() bytes, its address on the current device (taken once per device).
size_t nms_static_capacity();
Status nms_static_scratch(void** out);

// Count the v in [0, 256) where normalise_fast() and normalise() differ for (mean, stdv):
// result[0] += mismatches, result[1] = min(result[1], bit pattern of the first). Device
// pointer to two uint64 the caller set to {0, UINT64_MAX}.
Status launch_normalise_check(float mean, float stdv, unsigned long long* result, cudaStream_t stream);

// Opt a kernel into more than 48 KB of dynamic shared memory on the current device, once.
cudaError_t ensure_smem_attr(const void* func, int bytes);

// Taps of the letterbox resize along one axis, computed on the host with the kernel's own
// arithmetic; used to decide which source rows a host-frame call must upload.
void letterbox_rows_needed(int src_h, int new_h, unsigned char* needed);

// The source rows a crop of `box` (host float[4]) reads from an h x w frame, marked in
// needed[0, h), with the crop kernel's own geometry.
void crop_rows_needed(const float* box, int h, int w, int dst_h, unsigned char* needed);

}  // namespace shipk
