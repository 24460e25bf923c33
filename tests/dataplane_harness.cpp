// Test harness: C entry points over the C++ data-plane drop-in (shipinfer_b200/dataplane/
// ops_shipk.cpp), so the tests can call the reference's C++ API (csrc/shipinfer/runtime/ops.h)
// through ctypes. Each returns 0, 1 for a ConfigError or 2 for a BackendError (its message in
// `err`); a LetterboxMap comes back as five floats (scale, pad_x, pad_y, new_w, new_h).
#include <cstring>
#include <vector>

#include "crop_batch.h"
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

// The batched crop stage over flat arrays. Frame f: bgr[f] or nv12[f] (the other null), h[f] x
// w[f], stride[f] and uv[f] for NV12, its ndet[f] detections next in the flat arrays (boxes
// 4 floats, class, index). Set s: cls[s], sh[s] x sw[s], dst[s]. Outputs: rows[s] and, set
// after set, each row's frame and detection index; launches of the run. select_only: the host
// selection alone (no device), dst may be null.
int h_batched_crop(int nframes, void* const* bgr, void* const* nv12, const int* h, const int* w,
                   const int* stride, const unsigned long long* uv, const int* ndet, const float* boxes,
                   const int* classes, const int* index, int nsets, const int* cls, const int* sh, const int* sw,
                   void* const* dst, int select_only, int device, void* stream, int* rows, int* frame_of_row,
                   int* object_indices, int* launches, char* err, int len) {
    return guard(err, len, [&] {
        std::vector<shipinfer::Detection> dets;
        int total = 0;
        for (int f = 0; f < nframes; ++f) total += ndet[f];
        dets.resize(total);
        for (int i = 0; i < total; ++i) {
            dets[i].x1 = boxes[4 * i];
            dets[i].y1 = boxes[4 * i + 1];
            dets[i].x2 = boxes[4 * i + 2];
            dets[i].y2 = boxes[4 * i + 3];
            dets[i].class_id = classes[i];
            dets[i].index = index[i];
        }
        std::vector<shipinfer::BatchedCropFrame> frames(nframes);
        int at = 0;
        for (int f = 0; f < nframes; ++f) {
            frames[f].bgr = static_cast<const uint8_t*>(bgr[f]);
            frames[f].nv12 = static_cast<const uint8_t*>(nv12[f]);
            frames[f].height = h[f];
            frames[f].width = w[f];
            frames[f].stride = stride[f];
            frames[f].uv_offset = static_cast<size_t>(uv[f]);
            frames[f].detections = ndet[f] ? dets.data() + at : nullptr;
            frames[f].detection_count = ndet[f];
            at += ndet[f];
        }
        std::vector<shipinfer::BatchedCropSet> sets(nsets);
        for (int s = 0; s < nsets; ++s) {
            sets[s].class_id = cls[s];
            sets[s].height = sh[s];
            sets[s].width = sw[s];
            sets[s].dst = static_cast<float*>(dst ? dst[s] : nullptr);
        }
        std::vector<shipinfer::BatchedCropRows> out;
        if (select_only) {
            for (const auto& set : sets) out.push_back(shipinfer::select_crop_rows(frames, set));
            *launches = 0;
        } else {
            shipinfer::BatchedCropStage stage(device, stream);
            out = stage.run(frames, sets);
            *launches = stage.launches();
        }
        int k = 0;
        for (int s = 0; s < nsets; ++s) {
            rows[s] = out[s].rows;
            for (int r = 0; r < out[s].rows; ++r, ++k) {
                frame_of_row[k] = out[s].frame_of_row[r];
                object_indices[k] = out[s].object_indices[r];
            }
        }
    });
}

}  // extern "C"
