// The reference C++ data plane's pixel calls (csrc/shipinfer/runtime/ops.h) on libshipk: a
// drop-in for ops.cu. Compile this file in its place, with the tree's own include path, and
// link libshipk.so; the callers (pipeline/graph/pixels.cpp, graph stages) are unchanged.
//
// Each call is one launch of the sm_100a kernels through the C ABI (include/shipk.h):
//   letterbox_into / nv12_letterbox_into -> shipk_dp_letterbox_into / shipk_dp_nv12_letterbox_into
//   crop_resize_into / nv12_crop_resize_into -> shipk_dp_crop_resize_into / shipk_dp_nv12_crop_resize_into
//   mask_area_into -> shipk_mask_area;  letterbox_fit -> shipk_dp_letterbox_fit (the plane's float32
//   placement, ops.cu:341-356, which every letterbox call here also uses)
// A refused argument (SHIPK_EINVAL, SHIPK_ERANGE, SHIPK_ENOMEM) throws ConfigError, as the
// reference's require_nv12_layout and mask_area_into refusals do; a device failure
// (SHIPK_ECUDA, SHIPK_EDEVICE) throws BackendError, as its GPU_CHECK does. Messages are
// shipk_last_error()'s.
#include <string>

#include "shipinfer/runtime/ops.h"
#include "shipk.h"

namespace shipinfer {

namespace {

[[noreturn]] void raise(int rc) {
    char msg[512];
    shipk_last_error(msg, sizeof(msg));
    if (rc == SHIPK_ECUDA || rc == SHIPK_EDEVICE) throw BackendError(msg);
    throw ConfigError(msg);
}

LetterboxMap to_map(const shipk_letterbox_map& m) {
    LetterboxMap out;
    out.scale = m.scale;
    out.pad_x = m.pad_x;
    out.pad_y = m.pad_y;
    out.new_w = m.new_w;
    out.new_h = m.new_h;
    return out;
}

void* as_handle(gpuStream_t stream) { return reinterpret_cast<void*>(stream); }

}  // namespace

LetterboxMap letterbox_fit(int src_h, int src_w, int dst_h, int dst_w) {
    shipk_letterbox_map m;
    const int rc = shipk_dp_letterbox_fit(src_h, src_w, dst_h, dst_w, &m);
    if (rc) raise(rc);
    return to_map(m);
}

LetterboxMap letterbox_into(const uint8_t* src_device, int src_h, int src_w, float* dst_device, int dst_h,
                            int dst_w, bool swap_rb, float pad_value, gpuStream_t stream) {
    shipk_letterbox_map m;
    const int rc = shipk_dp_letterbox_into(src_device, src_h, src_w, dst_device, dst_h, dst_w, swap_rb ? 1 : 0,
                                           pad_value, &m, as_handle(stream));
    if (rc) raise(rc);
    return to_map(m);
}

void crop_resize_into(const uint8_t* src_device, int src_h, int src_w, const float* boxes_device, int count,
                      float* dst_device, int dst_h, int dst_w, bool swap_rb, gpuStream_t stream) {
    const int rc = shipk_dp_crop_resize_into(src_device, src_h, src_w, boxes_device, count, dst_device, dst_h,
                                             dst_w, swap_rb ? 1 : 0, as_handle(stream));
    if (rc) raise(rc);
}

LetterboxMap nv12_letterbox_into(const uint8_t* nv12_device, int src_h, int src_w, int stride, size_t uv_offset,
                                 float* dst_device, int dst_h, int dst_w, bool swap_rb, float pad_value,
                                 gpuStream_t stream) {
    shipk_letterbox_map m;
    const int rc = shipk_dp_nv12_letterbox_into(nv12_device, src_h, src_w, stride, uv_offset, dst_device, dst_h,
                                                dst_w, swap_rb ? 1 : 0, pad_value, &m, as_handle(stream));
    if (rc) raise(rc);
    return to_map(m);
}

void nv12_crop_resize_into(const uint8_t* nv12_device, int src_h, int src_w, int stride, size_t uv_offset,
                           const float* boxes_device, int count, float* dst_device, int dst_h, int dst_w,
                           bool swap_rb, gpuStream_t stream) {
    const int rc = shipk_dp_nv12_crop_resize_into(nv12_device, src_h, src_w, stride, uv_offset, boxes_device,
                                                  count, dst_device, dst_h, dst_w, swap_rb ? 1 : 0,
                                                  as_handle(stream));
    if (rc) raise(rc);
}

void mask_area_into(const float* rows_device, int candidates, int stride, int prefix, const float* protos_device,
                    int channels, int cells, int count, float score_threshold, float mask_threshold,
                    int crop_height, int crop_width, float* areas_device, gpuStream_t stream) {
    const int rc = shipk_mask_area(rows_device, candidates, stride, prefix, protos_device, channels, cells, count,
                                   score_threshold, mask_threshold, crop_height, crop_width, areas_device,
                                   as_handle(stream));
    if (rc) raise(rc);
}

}  // namespace shipinfer
