// The C++ data plane's crop stage over a batch of frames; see crop_batch.h.
#include "crop_batch.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <string>

namespace shipinfer {

namespace {

constexpr int kFramesPerLaunch = 64;  // the crop kernels' frame table (include/shipk.h)
const float kMean[3] = {0.f, 0.f, 0.f};
const float kStd[3] = {255.f, 255.f, 255.f};  // the data plane's value / 255

[[noreturn]] void raise(int rc) {
    char msg[512];
    shipk_last_error(msg, sizeof(msg));
    if (rc == SHIPK_ECUDA || rc == SHIPK_EDEVICE) throw BackendError(msg);
    throw ConfigError(msg);
}

void check_cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw BackendError(std::string("BatchedCropStage: ") + what + ": " + cudaGetErrorString(e));
}

// The device current for the duration of a scope, restored after.
struct DeviceScope {
    int previous = -1;
    explicit DeviceScope(int device) {
        check_cuda(cudaGetDevice(&previous), "cudaGetDevice");
        check_cuda(cudaSetDevice(device), "cudaSetDevice");
    }
    ~DeviceScope() {
        if (previous >= 0) cudaSetDevice(previous);
    }
};

// CropStage's selection (stages.cpp:199-206): every row for kAnyClass, else the rows of the
// set's class (kNoClass is an id no detector emits, so it selects nothing).
bool selects(const BatchedCropSet& set, int class_id) {
    return set.class_id == BatchedCropSet::kAnyClass || class_id == set.class_id;
}

void check_frames(const std::vector<BatchedCropFrame>& frames) {
    for (size_t f = 0; f < frames.size(); ++f) {
        const BatchedCropFrame& fr = frames[f];
        if ((fr.bgr == nullptr) == (fr.nv12 == nullptr))
            throw ConfigError("BatchedCropStage: frame " + std::to_string(f) +
                              " must carry exactly one of a BGR image and an NV12 surface");
        if (fr.height < 1 || fr.width < 1)
            throw ConfigError("BatchedCropStage: frame " + std::to_string(f) + " has no pixels");
        if (fr.detection_count < 0 || (fr.detection_count > 0 && fr.detections == nullptr))
            throw ConfigError("BatchedCropStage: frame " + std::to_string(f) + " has no detection array");
    }
}

size_t round16(size_t v) { return (v + 15) & ~size_t(15); }

}  // namespace

BatchedCropRows select_crop_rows(const std::vector<BatchedCropFrame>& frames, const BatchedCropSet& set) {
    check_frames(frames);
    BatchedCropRows out;
    for (int nv12 = 0; nv12 < 2; ++nv12) {  // BGR frames' rows first, then NV12 frames'
        for (size_t f = 0; f < frames.size(); ++f) {
            const BatchedCropFrame& fr = frames[f];
            if ((fr.nv12 != nullptr) != (nv12 == 1)) continue;
            for (int d = 0; d < fr.detection_count; ++d) {
                const Detection& det = fr.detections[d];
                if (!selects(set, det.class_id)) continue;
                out.frame_of_row.push_back(static_cast<int>(f));
                out.object_indices.push_back(det.index);
                out.boxes.insert(out.boxes.end(), {det.x1, det.y1, det.x2, det.y2});
            }
        }
    }
    out.rows = static_cast<int>(out.frame_of_row.size());
    return out;
}

BatchedCropStage::BatchedCropStage(int device, void* stream) : device_(device), stream_(stream) {}

BatchedCropStage::~BatchedCropStage() {
    if (capacity_ == 0) return;
    int previous = -1;
    cudaGetDevice(&previous);
    cudaSetDevice(device_);
    cudaFree(device_stage_);
    cudaFreeHost(host_stage_);
    if (previous >= 0) cudaSetDevice(previous);
}

void BatchedCropStage::reserve(size_t bytes) {
    if (bytes <= capacity_) return;
    const size_t want = std::max(bytes, capacity_ * 2);
    if (capacity_) {
        check_cuda(cudaFree(device_stage_), "cudaFree");
        check_cuda(cudaFreeHost(host_stage_), "cudaFreeHost");
        device_stage_ = host_stage_ = nullptr;
        capacity_ = 0;
    }
    check_cuda(cudaMalloc(reinterpret_cast<void**>(&device_stage_), want), "cudaMalloc");
    check_cuda(cudaHostAlloc(reinterpret_cast<void**>(&host_stage_), want, cudaHostAllocDefault), "cudaHostAlloc");
    capacity_ = want;
}

std::vector<BatchedCropRows> BatchedCropStage::run(const std::vector<BatchedCropFrame>& frames,
                                                   const std::vector<BatchedCropSet>& sets) {
    launches_ = 0;
    std::vector<BatchedCropRows> result;
    result.reserve(sets.size());
    // per set, in the staging buffer: its boxes (16 bytes a row), then its rows' frame indices
    // within their launch's frame table (4 bytes a row, padded to 16)
    std::vector<size_t> offset(sets.size());
    size_t total = 0;
    for (size_t s = 0; s < sets.size(); ++s) {
        const BatchedCropSet& set = sets[s];
        if (set.height < 1 || set.width < 1)
            throw ConfigError("BatchedCropStage: crop set " + std::to_string(s) + " has no output size");
        result.push_back(select_crop_rows(frames, set));
        if (result.back().rows > 0 && set.dst == nullptr)
            throw ConfigError("BatchedCropStage: crop set " + std::to_string(s) + " selects rows but has no dst");
        offset[s] = total;
        total += (size_t)result.back().rows * 16 + round16((size_t)result.back().rows * 4);
    }
    if (total == 0) return result;  // no row anywhere: nothing to launch, nothing to wait for

    // each frame's place in its representation's frame table
    std::vector<int> slot(frames.size());
    std::vector<shipk_frame_u8> bgr;
    std::vector<shipk_frame_nv12> nv12;
    for (size_t f = 0; f < frames.size(); ++f) {
        const BatchedCropFrame& fr = frames[f];
        if (fr.bgr) {
            slot[f] = static_cast<int>(bgr.size());
            bgr.push_back(shipk_frame_u8{fr.bgr, fr.height, fr.width, (int64_t)fr.width * 3});
        } else {
            slot[f] = static_cast<int>(nv12.size());
            nv12.push_back(shipk_frame_nv12{fr.nv12, fr.height, fr.width, fr.stride, (int64_t)fr.uv_offset});
        }
    }

    DeviceScope scope(device_);
    reserve(total);
    for (size_t s = 0; s < sets.size(); ++s) {
        const BatchedCropRows& r = result[s];
        float* boxes = reinterpret_cast<float*>(host_stage_ + offset[s]);
        int32_t* index = reinterpret_cast<int32_t*>(host_stage_ + offset[s] + (size_t)r.rows * 16);
        std::copy(r.boxes.begin(), r.boxes.end(), boxes);
        for (int i = 0; i < r.rows; ++i) index[i] = slot[r.frame_of_row[i]] % kFramesPerLaunch;
    }
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    check_cuda(cudaMemcpyAsync(device_stage_, host_stage_, total, cudaMemcpyHostToDevice, stream), "cudaMemcpyAsync");

    for (size_t s = 0; s < sets.size(); ++s) {
        const BatchedCropSet& set = sets[s];
        const BatchedCropRows& r = result[s];
        const size_t row_elems = (size_t)3 * set.height * set.width;
        const float* dev_boxes = reinterpret_cast<const float*>(device_stage_ + offset[s]);
        const int32_t* dev_index = reinterpret_cast<const int32_t*>(device_stage_ + offset[s] + (size_t)r.rows * 16);
        // rows run frame after frame within each representation: one launch over each run of
        // rows whose frames share a representation and a frame table of kFramesPerLaunch
        int i = 0;
        while (i < r.rows) {
            const int f0 = r.frame_of_row[i];
            const bool is_nv12 = frames[f0].nv12 != nullptr;
            const int chunk = slot[f0] / kFramesPerLaunch;
            int j = i;
            while (j < r.rows && (frames[r.frame_of_row[j]].nv12 != nullptr) == is_nv12 &&
                   slot[r.frame_of_row[j]] / kFramesPerLaunch == chunk)
                ++j;
            const int n = j - i;
            const int first = chunk * kFramesPerLaunch;
            float* out = set.dst + (size_t)i * row_elems;
            const size_t nbytes = (size_t)n * row_elems * sizeof(float);
            int rc;
            if (is_nv12) {
                const int nf = std::min<int>(kFramesPerLaunch, (int)nv12.size() - first);
                rc = shipk_crop_nv12(nv12.data() + first, nf, dev_boxes + (size_t)i * 4, dev_index + i, n, out,
                                     SHIPK_DTYPE_F32, nbytes, set.height, set.width, 1, stream_);
            } else {
                const int nf = std::min<int>(kFramesPerLaunch, (int)bgr.size() - first);
                rc = shipk_crop_u8(bgr.data() + first, nf, dev_boxes + (size_t)i * 4, dev_index + i, n, out,
                                   SHIPK_DTYPE_F32, nbytes, set.height, set.width, kMean, kStd, 1, stream_);
            }
            if (rc) raise(rc);
            ++launches_;
            i = j;
        }
    }
    check_cuda(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
    return result;
}

}  // namespace shipinfer
