// TEST INFRASTRUCTURE ONLY. An extern "C" face for the reference's own CUDA kernels
// (csrc/shipinfer/runtime/ops.cu in the reference tree), compiled from the reference sources
// where they lie by oracle/Makefile.ref into oracle/_ref/. GPU parity tests load it, when it
// is present, as a second oracle for the NV12 path, which has no CPU twin in the reference
// outside its C++ test binary. Nothing in the product links it.
#include <cstdint>
#include <exception>

#include "shipinfer/runtime/ops.h"

extern "C" {

// Returns 0 on success, 1 if the reference refused the call (its ConfigError).
int ref_nv12_letterbox(const uint8_t* nv12, int src_h, int src_w, int stride,
                       unsigned long long uv_offset, float* dst, int dst_h, int dst_w,
                       int swap_rb, float pad_value, void* stream, int* map_out) {
    try {
        shipinfer::LetterboxMap m = shipinfer::nv12_letterbox_into(
            nv12, src_h, src_w, stride, static_cast<size_t>(uv_offset), dst, dst_h, dst_w,
            swap_rb != 0, pad_value, static_cast<cudaStream_t>(stream));
        if (map_out) {
            map_out[0] = m.pad_x;
            map_out[1] = m.pad_y;
            map_out[2] = m.new_w;
            map_out[3] = m.new_h;
        }
        return 0;
    } catch (const std::exception&) {
        return 1;
    }
}

// The reference's own host-side placement (ops.cu:341-361); needs no device.
void ref_letterbox_fit(int src_h, int src_w, int dst_h, int dst_w, int* map_out) {
    shipinfer::LetterboxMap m = shipinfer::letterbox_fit(src_h, src_w, dst_h, dst_w);
    map_out[0] = m.pad_x;
    map_out[1] = m.pad_y;
    map_out[2] = m.new_w;
    map_out[3] = m.new_h;
}

int ref_letterbox(const uint8_t* src, int src_h, int src_w, float* dst, int dst_h, int dst_w,
                  int swap_rb, float pad_value, void* stream) {
    try {
        shipinfer::letterbox_into(src, src_h, src_w, dst, dst_h, dst_w, swap_rb != 0, pad_value,
                                  static_cast<cudaStream_t>(stream));
        return 0;
    } catch (const std::exception&) {
        return 1;
    }
}

int ref_mask_area(const float* rows, int candidates, int stride, int prefix, const float* protos,
                  int channels, int cells, int count, float score_threshold, float mask_threshold,
                  int crop_height, int crop_width, float* areas, void* stream) {
    try {
        shipinfer::mask_area_into(rows, candidates, stride, prefix, protos, channels, cells, count,
                                  score_threshold, mask_threshold, crop_height, crop_width, areas,
                                  static_cast<cudaStream_t>(stream));
        return 0;
    } catch (const std::exception&) {
        return 1;
    }
}

int ref_nv12_crop(const uint8_t* nv12, int src_h, int src_w, int stride, unsigned long long uv_offset,
                  const float* boxes, int count, float* dst, int dst_h, int dst_w, int swap_rb,
                  void* stream) {
    try {
        shipinfer::nv12_crop_resize_into(nv12, src_h, src_w, stride, static_cast<size_t>(uv_offset),
                                         boxes, count, dst, dst_h, dst_w, swap_rb != 0,
                                         static_cast<cudaStream_t>(stream));
        return 0;
    } catch (const std::exception&) {
        return 1;
    }
}

int ref_crop(const uint8_t* src, int src_h, int src_w, const float* boxes, int count,
             float* dst, int dst_h, int dst_w, int swap_rb, void* stream) {
    try {
        shipinfer::crop_resize_into(src, src_h, src_w, boxes, count, dst, dst_h, dst_w,
                                    swap_rb != 0, static_cast<cudaStream_t>(stream));
        return 0;
    } catch (const std::exception&) {
        return 1;
    }
}
}
