// The C++ data plane's per-frame pixel calls, declared as its callers use them
// (reference csrc/shipinfer/runtime/ops.h:30-120; pipeline/graph/pixels.cpp:18-43), for
// building ops_shipk.cpp outside the reference tree. Inside it, the reference's own ops.h
// declares the same functions and this header is not on the include path: the names, argument
// lists and the LetterboxMap layout must stay as they are for ops_shipk.cpp to link there.
#pragma once

#include <cstddef>
#include <cstdint>

#include "shipinfer/core/platform.h"

namespace shipinfer {

// Where a frame landed on the canvas: scale = min(dst/src), the resized extent
// max(1, round-half-even(src * scale)), bars (dst - new) // 2.
struct LetterboxMap {
    float scale = 1.0f;
    int pad_x = 0;
    int pad_y = 0;
    int new_w = 0;
    int new_h = 0;
};

LetterboxMap letterbox_fit(int src_h, int src_w, int dst_h, int dst_w);

// One uint8 HWC BGR device frame -> float NCHW [3, dst_h, dst_w], value / 255, bars = pad_value.
LetterboxMap letterbox_into(const uint8_t* src_device, int src_h, int src_w, float* dst_device, int dst_h,
                            int dst_w, bool swap_rb, float pad_value, gpuStream_t stream);

// `count` boxes ([x1, y1, x2, y2] frame pixels on the device) of one uint8 HWC BGR device
// frame -> float NCHW [count, 3, dst_h, dst_w], value / 255; a degenerate box is black.
void crop_resize_into(const uint8_t* src_device, int src_h, int src_w, const float* boxes_device, int count,
                      float* dst_device, int dst_h, int dst_w, bool swap_rb, gpuStream_t stream);

// The same two from an NV12 surface (chroma at `uv_offset` bytes from the luma); ConfigError
// for a layout whose rows or planes overlap.
LetterboxMap nv12_letterbox_into(const uint8_t* nv12_device, int src_h, int src_w, int stride, size_t uv_offset,
                                 float* dst_device, int dst_h, int dst_w, bool swap_rb, float pad_value,
                                 gpuStream_t stream);
void nv12_crop_resize_into(const uint8_t* nv12_device, int src_h, int src_w, int stride, size_t uv_offset,
                           const float* boxes_device, int count, float* dst_device, int dst_h, int dst_w,
                           bool swap_rb, gpuStream_t stream);

// One area per crop from a segmenter's rows and prototype planes (all on the device).
void mask_area_into(const float* rows_device, int candidates, int stride, int prefix, const float* protos_device,
                    int channels, int cells, int count, float score_threshold, float mask_threshold,
                    int crop_height, int crop_width, float* areas_device, gpuStream_t stream);

}  // namespace shipinfer
