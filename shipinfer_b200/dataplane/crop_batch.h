// Crops for a batch of frames on the C++ data plane: the reference's CropStage
// (csrc/shipinfer/pipeline/graph/stages.cpp:195-245) run over many frames at once.
//
// The reference crops one frame at a time: per frame and per crop set it selects the frame's
// detections of the set's class, uploads their boxes, launches crop_frame (pixels.cpp:31-43;
// the NV12 or the BGR kernel by the frame's representation) and synchronises the stream before
// the next set. Here every frame of a batch is handled together: the rows of every set go up in
// one host-to-device copy (boxes plus each row's frame), each set and pixel representation takes
// one launch over all its frames (shipk_crop_u8 / shipk_crop_nv12 with a per-row frame index),
// and the whole batch synchronises once. The rows, selection rule and values are CropStage's: a
// row per detection whose class is the set's (CropSpec::kAnyClass takes every row,
// CropSpec::kNoClass none), value / 255, BGR -> RGB, clip-then-truncate boxes and black
// degenerate crops — bit for bit the per-frame calls' output.
#pragma once

#include <cstddef>
#include <cstdint>
#include <vector>

#include "shipinfer/core/types.h"  // Detection, ConfigError, BackendError
#include "shipk.h"

namespace shipinfer {

// One frame of a batch, in either of pixels.h's representations: a host-uploaded BGR image on
// the device (tight rows: stride = width * 3) or an NVDEC NV12 surface. Exactly one of `bgr`
// and `nv12` is set.
struct BatchedCropFrame {
    const uint8_t* bgr = nullptr;
    const uint8_t* nv12 = nullptr;
    int height = 0;
    int width = 0;
    int stride = 0;          // NV12 only: bytes per luma and chroma row
    size_t uv_offset = 0;    // NV12 only: bytes from the luma plane to the UV plane
    const Detection* detections = nullptr;
    int detection_count = 0;
};

// A crop set: CropSpec's selection (class_id, with kAnyClass = -1 and kNoClass = -2) and output
// size; dst is a device float buffer with room for every selected row of the batch
// ([rows, 3, height, width]).
struct BatchedCropSet {
    static constexpr int kAnyClass = -1;
    static constexpr int kNoClass = -2;
    int class_id = kAnyClass;
    int height = 256;
    int width = 128;
    float* dst = nullptr;
};

// What one set produced: `rows` crops in dst, row r cut from frame frame_of_row[r] for its
// detection object_indices[r] (Detection::index) at boxes[4r .. 4r+3]. Rows of BGR frames come
// first, then rows of NV12 frames; within each, frame by frame in batch order and, within a
// frame, in detection order (CropStage's order for that frame).
struct BatchedCropRows {
    int rows = 0;
    std::vector<int> frame_of_row;
    std::vector<int> object_indices;
    std::vector<float> boxes;
};

// The rows a set selects, in output order, with nothing launched (the host half of run()).
BatchedCropRows select_crop_rows(const std::vector<BatchedCropFrame>& frames, const BatchedCropSet& set);

// Owns the device and pinned host staging for the boxes of a batch (grown as needed, reused
// across batches) and runs on the stream it is given. One instance per worker thread, as the
// reference's WorkerScratch is. Throws ConfigError for a refused argument, BackendError for a
// device failure.
class BatchedCropStage {
  public:
    BatchedCropStage(int device, void* stream);
    ~BatchedCropStage();
    BatchedCropStage(const BatchedCropStage&) = delete;
    BatchedCropStage& operator=(const BatchedCropStage&) = delete;

    // Every set over every frame: one upload, one launch per set and pixel representation, one
    // synchronise. The result has one entry per set, in order.
    std::vector<BatchedCropRows> run(const std::vector<BatchedCropFrame>& frames,
                                     const std::vector<BatchedCropSet>& sets);

    int launches() const { return launches_; }  // kernel launches of the last run()

  private:
    void reserve(size_t bytes);
    int device_;
    void* stream_;
    uint8_t* device_stage_ = nullptr;
    uint8_t* host_stage_ = nullptr;
    size_t capacity_ = 0;
    int launches_ = 0;
};

}  // namespace shipinfer
