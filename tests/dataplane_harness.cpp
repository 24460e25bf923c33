// Test harness: C entry points over the C++ data-plane drop-in (shipinfer_b200/dataplane/
// ops_shipk.cpp), so the tests can call the reference's C++ API (csrc/shipinfer/runtime/ops.h)
// through ctypes. Each returns 0, 1 for a ConfigError or 2 for a BackendError (its message in
// `err`); a LetterboxMap comes back as five floats (scale, pad_x, pad_y, new_w, new_h).
#include <cstring>

#include "shipinfer/runtime/ops.h"

namespace {

template <class F>
int guard(char* err, int len, F&& f) {
    try {
        f();
        return 0;
    } catch (const shipinfer::ConfigError& e) {
        std::strncpy(err, e.what(), len - 1);
        err[len - 1] = 0;
        return 1;
    } catch (const shipinfer::BackendError& e) {
        std::strncpy(err, e.what(), len - 1);
        err[len - 1] = 0;
        return 2;
    }
}

void put(const shipinfer::LetterboxMap& m, float* out) {
    out[0] = m.scale;
    out[1] = (float)m.pad_x;
    out[2] = (float)m.pad_y;
    out[3] = (float)m.new_w;
    out[4] = (float)m.new_h;
}

gpuStream_t st(void* s) { return reinterpret_cast<gpuStream_t>(s); }

}  // namespace

extern "C" {

int h_letterbox_fit(int sh, int sw, int dh, int dw, float* map, char* err, int len) {
    return guard(err, len, [&] { put(shipinfer::letterbox_fit(sh, sw, dh, dw), map); });
}

int h_letterbox_into(const void* src, int sh, int sw, void* dst, int dh, int dw, int swap_rb, float pad,
                     float* map, void* stream, char* err, int len) {
    return guard(err, len, [&] {
        put(shipinfer::letterbox_into(static_cast<const uint8_t*>(src), sh, sw, static_cast<float*>(dst), dh, dw,
                                      swap_rb != 0, pad, st(stream)),
            map);
    });
}

int h_crop_resize_into(const void* src, int sh, int sw, const void* boxes, int count, void* dst, int dh, int dw,
                       int swap_rb, void* stream, char* err, int len) {
    return guard(err, len, [&] {
        shipinfer::crop_resize_into(static_cast<const uint8_t*>(src), sh, sw, static_cast<const float*>(boxes), count,
                                    static_cast<float*>(dst), dh, dw, swap_rb != 0, st(stream));
    });
}

int h_nv12_letterbox_into(const void* nv12, int sh, int sw, int stride, unsigned long long uv_offset, void* dst,
                          int dh, int dw, int swap_rb, float pad, float* map, void* stream, char* err, int len) {
    return guard(err, len, [&] {
        put(shipinfer::nv12_letterbox_into(static_cast<const uint8_t*>(nv12), sh, sw, stride, (size_t)uv_offset,
                                           static_cast<float*>(dst), dh, dw, swap_rb != 0, pad, st(stream)),
            map);
    });
}

int h_nv12_crop_resize_into(const void* nv12, int sh, int sw, int stride, unsigned long long uv_offset,
                            const void* boxes, int count, void* dst, int dh, int dw, int swap_rb, void* stream,
                            char* err, int len) {
    return guard(err, len, [&] {
        shipinfer::nv12_crop_resize_into(static_cast<const uint8_t*>(nv12), sh, sw, stride, (size_t)uv_offset,
                                         static_cast<const float*>(boxes), count, static_cast<float*>(dst), dh, dw,
                                         swap_rb != 0, st(stream));
    });
}

int h_mask_area_into(const void* rows, int candidates, int stride, int prefix, const void* protos, int channels,
                     int cells, int count, float score_thr, float mask_thr, int crop_h, int crop_w, void* areas,
                     void* stream, char* err, int len) {
    return guard(err, len, [&] {
        shipinfer::mask_area_into(static_cast<const float*>(rows), candidates, stride, prefix,
                                  static_cast<const float*>(protos), channels, cells, count, score_thr, mask_thr,
                                  crop_h, crop_w, static_cast<float*>(areas), st(stream));
    });
}

}  // extern "C"
