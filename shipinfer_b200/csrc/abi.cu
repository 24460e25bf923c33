// The C ABI declared in include/shipk.h: argument validation, error reporting, and the
// per-thread context that stages host frames. Every entry point returns a status code; no
// C++ exception crosses the boundary.
#include "kernels.h"

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <new>
#include <set>
#include <string>
#include <utility>
#include <vector>

namespace shipk {
namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int fail_status(const Status& s, const char* who) {
    return fail(s.code, "%s: %s", who, s.message ? s.message : "failed");
}

int fail_cuda(cudaError_t e, const char* who, const char* what) {
    return fail(SHIPK_ECUDA, "%s: %s failed: %s", who, what, cudaGetErrorString(e));
}

// A pointer must be device (or managed) memory of the current device.
int check_device_ptr(const void* ptr, const char* who, const char* name) {
    if (ptr == nullptr) return fail(SHIPK_EINVAL, "%s: %s is null", who, name);
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail_cuda(e, who, "cudaGetDevice");
    cudaPointerAttributes attr;
    e = cudaPointerGetAttributes(&attr, ptr);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(SHIPK_EDEVICE, "%s: %s is not a CUDA pointer (%s)", who, name,
                    cudaGetErrorString(e));
    }
    if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged)
        return fail(SHIPK_EDEVICE, "%s: %s is host memory; this call takes device memory", who,
                    name);
    if (attr.device != dev)
        return fail(SHIPK_EDEVICE,
                    "%s: %s is on cuda:%d but the current device is cuda:%d; a cross-device "
                    "write is refused",
                    who, name, attr.device, dev);
    return SHIPK_OK;
}

int check_common(const char* who, int n, int dst_h, int dst_w, int out_dtype,
                 const float* mean, const float* stdv) {
    if (n < 1) return fail(SHIPK_EINVAL, "%s: needs at least one frame", who);
    if (dst_h < 1 || dst_w < 1 || dst_h > 32768 || dst_w > 32768)
        return fail(SHIPK_EINVAL, "%s: destination %dx%d is outside 1..32768", who, dst_h, dst_w);
    if (out_dtype != SHIPK_DTYPE_F32 && out_dtype != SHIPK_DTYPE_F16)
        return fail(SHIPK_EINVAL, "%s: out_dtype %d is neither F32 nor F16", who, out_dtype);
    if (!mean || !stdv) return fail(SHIPK_EINVAL, "%s: mean and std are required", who);
    for (int c = 0; c < 3; ++c)
        if (stdv[c] == 0.f) return fail(SHIPK_EINVAL, "%s: normalisation std must be non-zero", who);
    return SHIPK_OK;
}

size_t out_bytes(int rows, int dst_h, int dst_w, int out_dtype) {
    return (size_t)rows * 3 * dst_h * dst_w * (out_dtype == SHIPK_DTYPE_F32 ? 4 : 2);
}

int check_u8_frame(const char* who, int i, const uint8_t* data, int h, int w, int64_t pitch) {
    if (data == nullptr) return fail(SHIPK_EINVAL, "%s: frame %d has no data", who, i);
    if (h < 1 || w < 1 || h > 32768 || w > 32768)
        return fail(SHIPK_EINVAL, "%s: frame %d is %dx%d; expected 1..32768 per side", who, i, h, w);
    if (pitch < (int64_t)w * 3)
        return fail(SHIPK_EINVAL, "%s: frame %d pitch %lld is narrower than its %d BGR pixels",
                    who, i, (long long)pitch, w);
    return SHIPK_OK;
}

}  // namespace

// Once per (function, device): the attribute belongs to the function on a device context.
cudaError_t ensure_smem_attr(const void* func, int bytes) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, int> granted;  // (kernel, device) -> bytes
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    auto it = granted.find({func, dev});
    if (it != granted.end() && it->second >= bytes) return cudaSuccess;
    e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    // These kernels keep their working set in shared memory and barely use L1 otherwise: ask
    // for the largest shared carveout, or the driver may pick one that fits fewer CTAs.
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(func, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 cudaSharedmemCarveoutMaxShared);
    if (e == cudaSuccess) granted[{func, dev}] = bytes;
    return e;
}

}  // namespace shipk

using namespace shipk;

// ---- host-frame context ---------------------------------------------------------------------

struct shipk_ctx {
    int device = 0;
    cudaEvent_t done = nullptr;    // recorded after the last kernel that reads the staging
    bool pending = false;
    uint8_t* staging = nullptr;    // device copy of the source rows a call reads
    size_t staging_bytes = 0;
    int32_t* row_map = nullptr;    // device: staged row of each source row, all frames
    size_t row_map_bytes = 0;
    int32_t* host_rows = nullptr;  // pinned: the row maps on their way to the device
    size_t host_rows_bytes = 0;
    float* boxes = nullptr;        // device boxes for host crops
    size_t boxes_bytes = 0;
    float* host_boxes = nullptr;   // pinned
    size_t host_boxes_bytes = 0;
    uint8_t* nms_in = nullptr;     // device NMS inputs and outputs + workspace
    size_t nms_in_bytes = 0;
    uint8_t* nms_host = nullptr;   // pinned NMS inputs and outputs
    size_t nms_host_bytes = 0;
};

namespace {

struct DeviceGuard {
    int prev = -1;
    cudaError_t err = cudaSuccess;
    explicit DeviceGuard(int dev) {
        err = cudaGetDevice(&prev);
        if (err == cudaSuccess && prev != dev) err = cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

template <typename T>
cudaError_t grow_device(T** ptr, size_t* have, size_t need) {
    if (*have >= need) return cudaSuccess;
    if (*ptr) cudaFree(*ptr);
    *ptr = nullptr;
    *have = 0;
    const size_t size = std::max(need, (size_t)1) + need / 4;
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(ptr), size);
    if (e == cudaSuccess) *have = size;
    return e;
}

template <typename T>
cudaError_t grow_pinned(T** ptr, size_t* have, size_t need) {
    if (*have >= need) return cudaSuccess;
    if (*ptr) cudaFreeHost(*ptr);
    *ptr = nullptr;
    *have = 0;
    const size_t size = std::max(need, (size_t)1) + need / 4;
    cudaError_t e = cudaMallocHost(reinterpret_cast<void**>(ptr), size);
    if (e == cudaSuccess) *have = size;
    return e;
}

// Wait until the previous call's kernel has finished reading this context's staging.
int ctx_quiesce(shipk_ctx* ctx, const char* who) {
    if (!ctx->pending) return SHIPK_OK;
    cudaError_t e = cudaEventSynchronize(ctx->done);
    if (e != cudaSuccess) return fail_cuda(e, who, "cudaEventSynchronize");
    ctx->pending = false;
    return SHIPK_OK;
}

// Copy the marked rows of one host frame into consecutive staging rows, one 2-D copy per
// run of rows at a constant stride (one copy for 1080p -> 640, where every third row is
// read). Fills row_map for the marked rows.
int upload_rows(const char* who, const uint8_t* host, int64_t pitch, int h, int row_bytes,
                const unsigned char* needed, uint8_t* dst, int64_t dst_pitch, int32_t* row_map,
                cudaStream_t stream) {
    int staged = 0;
    int r = 0;
    while (r < h) {
        if (!needed[r]) {
            row_map[r] = 0;
            ++r;
            continue;
        }
        int next = r + 1;
        while (next < h && !needed[next]) ++next;
        const int stride = next < h ? next - r : 1;
        int count = 1;
        int last = r;
        // extend the run while the next marked row sits `stride` further on
        for (;;) {
            int cand = last + stride;
            if (cand >= h || !needed[cand]) break;
            bool gap_clear = true;
            for (int q = last + 1; q < cand; ++q)
                if (needed[q]) {
                    gap_clear = false;
                    break;
                }
            if (!gap_clear) break;
            last = cand;
            ++count;
        }
        for (int q = r; q <= last; ++q) row_map[q] = needed[q] ? staged + (q - r) / stride : 0;
        cudaError_t e = cudaMemcpy2DAsync(dst + (int64_t)staged * dst_pitch, dst_pitch,
                                          host + (int64_t)r * pitch, pitch * stride, row_bytes,
                                          count, cudaMemcpyHostToDevice, stream);
        if (e != cudaSuccess) return fail_cuda(e, who, "cudaMemcpy2DAsync");
        staged += count;
        r = last + 1;
    }
    return SHIPK_OK;
}

}  // namespace

extern "C" {

const char* shipk_version(void) { return "0.1.0+sm100a"; }

int shipk_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

int shipk_cuda_available(void) {
    const int n = shipk_device_count();
    for (int d = 0; d < n; ++d) {
        cudaDeviceProp prop;
        if (cudaGetDeviceProperties(&prop, d) != cudaSuccess) {
            cudaGetLastError();
            continue;
        }
        if (prop.major == 10 && prop.minor == 0) return 1;  // sm_100a code runs on cc 10.0
    }
    return 0;
}

size_t shipk_last_error(char* buf, size_t len) {
    const std::string& s = g_last_error;
    if (buf && len) {
        const size_t k = std::min(len - 1, s.size());
        std::memcpy(buf, s.data(), k);
        buf[k] = '\0';
    }
    return s.size();
}

int shipk_letterbox_fit(int src_h, int src_w, int dst_h, int dst_w, shipk_letterbox_map* out) {
    if (!out) return fail(SHIPK_EINVAL, "shipk_letterbox_fit: out is null");
    Fit f;
    if (letterbox_fit(src_h, src_w, dst_h, dst_w, &f) != SHIPK_OK)
        return fail(SHIPK_EINVAL, "shipk_letterbox_fit: sizes must be positive (%dx%d -> %dx%d)",
                    src_h, src_w, dst_h, dst_w);
    out->scale = f.scale;
    out->pad_x = f.pad_x;
    out->pad_y = f.pad_y;
    out->new_w = f.new_w;
    out->new_h = f.new_h;
    return SHIPK_OK;
}

int shipk_dp_letterbox_fit(int src_h, int src_w, int dst_h, int dst_w, shipk_letterbox_map* out) {
    if (!out) return fail(SHIPK_EINVAL, "letterbox_fit: out is null");
    Fit f;
    if (letterbox_fit_f32(src_h, src_w, dst_h, dst_w, &f) != SHIPK_OK)
        return fail(SHIPK_EINVAL, "letterbox_fit: sizes must be positive (%dx%d -> %dx%d)", src_h, src_w, dst_h,
                    dst_w);
    *out = shipk_letterbox_map{f.scale, f.pad_x, f.pad_y, f.new_w, f.new_h};
    return SHIPK_OK;
}

static void fill_maps(const FrameView* frames, int n, int dst_h, int dst_w, shipk_letterbox_map* maps) {
    if (!maps) return;
    for (int i = 0; i < n; ++i) {
        Fit f;
        frame_fit(frames[i], dst_h, dst_w, &f);
        maps[i] = shipk_letterbox_map{f.scale, f.pad_x, f.pad_y, f.new_w, f.new_h};
    }
}

int shipk_letterbox_u8(const shipk_frame_u8* frames, int n, void* out, int out_dtype,
                       size_t out_nbytes, int dst_h, int dst_w, const float mean[3],
                       const float std_[3], int swap_rb, float pad_value,
                       shipk_letterbox_map* maps_out, void* stream) {
    static const char* who = "shipk_letterbox_u8";
    int rc = check_common(who, n, dst_h, dst_w, out_dtype, mean, std_);
    if (rc) return rc;
    if (!frames) return fail(SHIPK_EINVAL, "%s: frames is null", who);
    if (out_nbytes < out_bytes(n, dst_h, dst_w, out_dtype))
        return fail(SHIPK_ENOMEM, "%s: out holds %zu bytes, the batch needs %zu", who, out_nbytes,
                    out_bytes(n, dst_h, dst_w, out_dtype));
    if ((rc = check_device_ptr(out, who, "out"))) return rc;
    std::vector<FrameView> views(n);
    for (int i = 0; i < n; ++i) {
        const shipk_frame_u8& f = frames[i];
        if ((rc = check_u8_frame(who, i, f.data, f.height, f.width, f.pitch))) return rc;
        if ((rc = check_device_ptr(f.data, who, "frame data"))) return rc;
        views[i] = FrameView{f.data, nullptr, f.height, f.width, f.pitch, 0};
    }
    Status s = launch_letterbox(views.data(), n, out, out_dtype, dst_h, dst_w, mean, std_, swap_rb,
                                pad_value, false, 601, 1, static_cast<cudaStream_t>(stream));
    if (s.code) return fail_status(s, who);
    fill_maps(views.data(), n, dst_h, dst_w, maps_out);
    return SHIPK_OK;
}

int shipk_letterbox_nv12(const shipk_frame_nv12* frames, int n, void* out, int out_dtype,
                         size_t out_nbytes, int dst_h, int dst_w, const float mean[3],
                         const float std_[3], int swap_rb, float pad_value, int matrix,
                         int sampling, shipk_letterbox_map* maps_out, void* stream) {
    static const char* who = "shipk_letterbox_nv12";
    int rc = check_common(who, n, dst_h, dst_w, out_dtype, mean, std_);
    if (rc) return rc;
    if (!frames) return fail(SHIPK_EINVAL, "%s: frames is null", who);
    if (matrix != 601 && matrix != 709)
        return fail(SHIPK_EINVAL, "%s: matrix %d is neither 601 nor 709", who, matrix);
    if (sampling != 0 && sampling != 1)
        return fail(SHIPK_EINVAL, "%s: sampling %d is neither 0 (nearest) nor 1 (bilinear)", who,
                    sampling);
    if (out_nbytes < out_bytes(n, dst_h, dst_w, out_dtype))
        return fail(SHIPK_ENOMEM, "%s: out holds %zu bytes, the batch needs %zu", who, out_nbytes,
                    out_bytes(n, dst_h, dst_w, out_dtype));
    if ((rc = check_device_ptr(out, who, "out"))) return rc;
    std::vector<FrameView> views(n);
    for (int i = 0; i < n; ++i) {
        const shipk_frame_nv12& f = frames[i];
        if (!f.luma) return fail(SHIPK_EINVAL, "%s: frame %d has no data", who, i);
        if (f.height < 1 || f.width < 1 || f.height > 32768 || f.width > 32768)
            return fail(SHIPK_EINVAL, "%s: frame %d is %dx%d; expected 1..32768 per side", who, i,
                        f.height, f.width);
        // The reference's layout rule (ops.cu:325-339), plus room for the last chroma pair of
        // an odd width.
        const int64_t chroma_row = ((int64_t)(f.width + 1) / 2) * 2;
        if (f.pitch < f.width || f.pitch < chroma_row)
            return fail(SHIPK_EINVAL,
                        "%s: frame %d stride %lld is narrower than the width %d; a row cannot "
                        "fit, so every row would read into the next",
                        who, i, (long long)f.pitch, f.width);
        if (f.uv_offset < f.pitch * f.height)
            return fail(SHIPK_EINVAL,
                        "%s: frame %d uv_offset %lld is inside the luma plane (%lld x %d); pass "
                        "`stride * height` for a tight buffer",
                        who, i, (long long)f.uv_offset, (long long)f.pitch, f.height);
        if ((rc = check_device_ptr(f.luma, who, "frame data"))) return rc;
        views[i] = FrameView{f.luma, nullptr, f.height, f.width, f.pitch, f.uv_offset};
    }
    Status s = launch_letterbox(views.data(), n, out, out_dtype, dst_h, dst_w, mean, std_, swap_rb,
                                pad_value, true, matrix, sampling, static_cast<cudaStream_t>(stream));
    if (s.code) return fail_status(s, who);
    fill_maps(views.data(), n, dst_h, dst_w, maps_out);
    return SHIPK_OK;
}

int shipk_crop_u8(const shipk_frame_u8* frames, int n_frames, const float* boxes,
                  const int32_t* box_frame, int n_boxes, void* out, int out_dtype,
                  size_t out_nbytes, int dst_h, int dst_w, const float mean[3],
                  const float std_[3], int swap_rb, void* stream) {
    static const char* who = "shipk_crop_u8";
    int rc = check_common(who, n_frames, dst_h, dst_w, out_dtype, mean, std_);
    if (rc) return rc;
    if (n_frames > kMaxBatch)
        return fail(SHIPK_ERANGE, "%s: %d frames; one call takes at most %d", who, n_frames, kMaxBatch);
    if (n_boxes < 0) return fail(SHIPK_EINVAL, "%s: n_boxes is negative", who);
    if (!frames) return fail(SHIPK_EINVAL, "%s: frames is null", who);
    if (n_boxes == 0) return SHIPK_OK;
    if (out_nbytes < out_bytes(n_boxes, dst_h, dst_w, out_dtype))
        return fail(SHIPK_ENOMEM, "%s: out holds %zu bytes, %d crops need %zu", who, out_nbytes,
                    n_boxes, out_bytes(n_boxes, dst_h, dst_w, out_dtype));
    if ((rc = check_device_ptr(out, who, "out"))) return rc;
    if ((rc = check_device_ptr(boxes, who, "boxes"))) return rc;
    if (box_frame && (rc = check_device_ptr(box_frame, who, "box_frame"))) return rc;
    std::vector<FrameView> views(n_frames);
    for (int i = 0; i < n_frames; ++i) {
        const shipk_frame_u8& f = frames[i];
        if ((rc = check_u8_frame(who, i, f.data, f.height, f.width, f.pitch))) return rc;
        if ((rc = check_device_ptr(f.data, who, "frame data"))) return rc;
        views[i] = FrameView{f.data, nullptr, f.height, f.width, f.pitch, 0};
    }
    Status s = launch_crop(views.data(), n_frames, boxes, box_frame, n_boxes, out, out_dtype, dst_h,
                           dst_w, mean, std_, swap_rb, static_cast<cudaStream_t>(stream));
    if (s.code) return fail_status(s, who);
    return SHIPK_OK;
}

size_t shipk_nms_workspace_bytes(int batch, int n, int num_classes, int class_aware, int max_det) {
    return nms_workspace_bytes(batch, n, num_classes, class_aware, max_det);
}

static int check_nms_args(const char* who, int batch, int n, int num_classes, int class_aware,
                          int max_det) {
    if (batch < 0 || n < 0) return fail(SHIPK_EINVAL, "%s: batch and n must be >= 0", who);
    if (class_aware && num_classes < 1)
        return fail(SHIPK_EINVAL, "%s: class-aware NMS needs num_classes >= 1", who);
    if (max_det < 0) return fail(SHIPK_EINVAL, "%s: max_det is negative", who);
    if (max_det > 4096) return fail(SHIPK_ERANGE, "%s: max_det %d is above 4096", who, max_det);
    return SHIPK_OK;
}

int shipk_nms_launch_shape(int batch, int n, int num_classes, int class_aware, int max_det, int* ctas,
                           int* cluster) {
    static const char* who = "shipk_nms_launch_shape";
    int rc = check_nms_args(who, batch, n, num_classes, class_aware, max_det);
    if (rc) return rc;
    if (!ctas || !cluster) return fail(SHIPK_EINVAL, "%s: ctas and cluster must not be NULL", who);
    if (n == 0) {
        *ctas = 0;
        *cluster = 1;
        return SHIPK_OK;
    }
    Status s = nms_launch_shape(batch, num_classes, class_aware, max_det, ctas, cluster);
    if (s.code) return fail_status(s, who);
    return SHIPK_OK;
}

int shipk_nms(const float* boxes, const float* scores, const int32_t* classes, int batch, int n,
              int num_classes, int class_aware, float iou_threshold, float score_threshold,
              int max_det, int64_t* keep, int32_t* counts, void* workspace,
              size_t workspace_bytes, void* stream) {
    static const char* who = "shipk_nms";
    int rc = check_nms_args(who, batch, n, num_classes, class_aware, max_det);
    if (rc) return rc;
    if (batch == 0) return SHIPK_OK;
    if ((rc = check_device_ptr(counts, who, "counts"))) return rc;
    if (max_det > 0 && (rc = check_device_ptr(keep, who, "keep"))) return rc;
    if (n > 0 && max_det > 0) {
        if ((rc = check_device_ptr(boxes, who, "boxes"))) return rc;
        if ((rc = check_device_ptr(scores, who, "scores"))) return rc;
        if (class_aware && (rc = check_device_ptr(classes, who, "classes"))) return rc;
        if ((rc = check_device_ptr(workspace, who, "workspace"))) return rc;
    }
    Status s = launch_nms(boxes, scores, classes, batch, n, num_classes, class_aware, iou_threshold,
                          score_threshold, max_det, keep, counts, workspace, workspace_bytes, true,
                          static_cast<cudaStream_t>(stream));
    if (s.code) return fail_status(s, who);
    return SHIPK_OK;
}

int shipk_nms_static(const float* boxes, const float* scores, const int32_t* classes, int batch,
                     int n, int num_classes, int class_aware, float iou_threshold,
                     float score_threshold, int max_det, int64_t* keep, int32_t* counts,
                     void* stream) {
    static const char* who = "shipk_nms_static";
    int rc = check_nms_args(who, batch, n, num_classes, class_aware, max_det);
    if (rc) return rc;
    if (batch == 0) return SHIPK_OK;
    const size_t need = nms_workspace_bytes(batch, n, num_classes, class_aware, max_det);
    if (need > nms_static_capacity())
        return fail(SHIPK_ERANGE,
                    "%s: %d images x %d segments x max_det %d need %zu bytes of scratch, above the "
                    "%zu-byte static scratch; use shipk_nms with a workspace",
                    who, batch, class_aware ? num_classes : 1, max_det, need, nms_static_capacity());
    if ((rc = check_device_ptr(counts, who, "counts"))) return rc;
    if (max_det > 0 && (rc = check_device_ptr(keep, who, "keep"))) return rc;
    if (n > 0 && max_det > 0) {
        if ((rc = check_device_ptr(boxes, who, "boxes"))) return rc;
        if ((rc = check_device_ptr(scores, who, "scores"))) return rc;
        if (class_aware && (rc = check_device_ptr(classes, who, "classes"))) return rc;
    }
    void* scratch = nullptr;
    Status s = nms_static_scratch(&scratch);
    if (s.code) return fail_status(s, who);
    // zero_arrivals: the arrival counters in the scratch are cleared on `stream` first
    s = launch_nms(boxes, scores, classes, batch, n, num_classes, class_aware, iou_threshold,
                   score_threshold, max_det, keep, counts, scratch, nms_static_capacity(), true,
                   static_cast<cudaStream_t>(stream));
    if (s.code) return fail_status(s, who);
    return SHIPK_OK;
}

int shipk_crop_nv12(const shipk_frame_nv12* frames, int n_frames, const float* boxes,
                    const int32_t* box_frame, int n_boxes, void* out, int out_dtype, size_t out_nbytes,
                    int dst_h, int dst_w, int swap_rb, void* stream) {
    static const char* who = "shipk_crop_nv12";
    if (n_boxes < 0 || n_frames < 0) return fail(SHIPK_EINVAL, "%s: negative box or frame count", who);
    if (n_boxes == 0) return SHIPK_OK;  // a frame with no detections is not an error (ops.cu:407)
    if (dst_h < 1 || dst_w < 1) return fail(SHIPK_EINVAL, "%s: output %dx%d is empty", who, dst_h, dst_w);
    if (out_dtype != SHIPK_DTYPE_F32 && out_dtype != SHIPK_DTYPE_F16)
        return fail(SHIPK_EINVAL, "%s: out_dtype %d is neither f32 nor f16", who, out_dtype);
    if (n_frames < 1 || !frames) return fail(SHIPK_EINVAL, "%s: no frames for %d boxes", who, n_boxes);
    if (out_nbytes < out_bytes(n_boxes, dst_h, dst_w, out_dtype))
        return fail(SHIPK_ENOMEM, "%s: out holds %zu bytes, %d crops need %zu", who, out_nbytes, n_boxes,
                    out_bytes(n_boxes, dst_h, dst_w, out_dtype));
    int rc;
    if ((rc = check_device_ptr(out, who, "out"))) return rc;
    if ((rc = check_device_ptr(boxes, who, "boxes"))) return rc;
    if (box_frame && (rc = check_device_ptr(box_frame, who, "box_frame"))) return rc;
    std::vector<FrameView> views(n_frames);
    for (int i = 0; i < n_frames; ++i) {
        const shipk_frame_nv12& f = frames[i];
        if (!f.luma) return fail(SHIPK_EINVAL, "%s: frame %d has no data", who, i);
        if (f.height < 1 || f.width < 1 || f.height > 32768 || f.width > 32768)
            return fail(SHIPK_EINVAL, "%s: frame %d is %dx%d; expected 1..32768 per side", who, i, f.height,
                        f.width);
        // the reference's layout rule (require_nv12_layout, ops.cu:325-339)
        const int64_t chroma_row = ((int64_t)(f.width + 1) / 2) * 2;
        if (f.pitch < f.width || f.pitch < chroma_row)
            return fail(SHIPK_EINVAL, "%s: frame %d stride %lld is narrower than the width %d", who, i,
                        (long long)f.pitch, f.width);
        if (f.uv_offset < f.pitch * f.height)
            return fail(SHIPK_EINVAL, "%s: frame %d uv_offset %lld is inside the luma plane (%lld x %d)", who, i,
                        (long long)f.uv_offset, (long long)f.pitch, f.height);
        if ((rc = check_device_ptr(f.luma, who, "frame data"))) return rc;
        views[i] = FrameView{f.luma, nullptr, f.height, f.width, f.pitch, f.uv_offset};
    }
    Status s = launch_crop_nv12(views.data(), n_frames, boxes, box_frame, n_boxes, out, out_dtype, dst_h, dst_w,
                                swap_rb, static_cast<cudaStream_t>(stream));
    if (s.code) return fail_status(s, who);
    return SHIPK_OK;
}

int shipk_decode_detections(const float* rows, int batch, int rows_per_frame, const int32_t* counts,
                            const float* scales, const float* pads, const int32_t* frame_hw,
                            float score_threshold, int max_detections, float* boxes, float* scores,
                            int32_t* class_ids, int32_t* out_counts, int32_t* discarded, void* stream) {
    static const char* who = "shipk_decode_detections";
    if (batch < 0 || rows_per_frame < 0)
        return fail(SHIPK_EINVAL, "%s: batch %d and rows %d must not be negative", who, batch, rows_per_frame);
    if (max_detections < 0) return fail(SHIPK_EINVAL, "%s: max_detections is negative", who);
    if (max_detections > 4096)
        return fail(SHIPK_ERANGE, "%s: max_detections %d is above 4096", who, max_detections);
    if (batch == 0) return SHIPK_OK;
    int rc;
    if ((rc = check_device_ptr(scales, who, "scales"))) return rc;
    if ((rc = check_device_ptr(pads, who, "pads"))) return rc;
    if ((rc = check_device_ptr(out_counts, who, "out_counts"))) return rc;
    if ((rc = check_device_ptr(discarded, who, "discarded"))) return rc;
    if (rows_per_frame > 0 && (rc = check_device_ptr(rows, who, "rows"))) return rc;
    if (counts && (rc = check_device_ptr(counts, who, "counts"))) return rc;
    if (frame_hw && (rc = check_device_ptr(frame_hw, who, "frame_hw"))) return rc;
    if (max_detections > 0) {
        if ((rc = check_device_ptr(boxes, who, "boxes"))) return rc;
        if ((rc = check_device_ptr(scores, who, "scores"))) return rc;
        if ((rc = check_device_ptr(class_ids, who, "class_ids"))) return rc;
    }
    Status s = launch_decode(rows, batch, rows_per_frame, counts, scales, pads, frame_hw, score_threshold,
                             max_detections, boxes, scores, class_ids, out_counts, discarded,
                             static_cast<cudaStream_t>(stream));
    if (s.code) return fail_status(s, who);
    return SHIPK_OK;
}

int shipk_mask_area(const float* rows, int candidates, int stride, int prefix, const float* protos,
                    int channels, int cells, int count, float score_threshold, float mask_threshold,
                    int crop_height, int crop_width, float* areas, void* stream) {
    static const char* who = "shipk_mask_area";
    if (count <= 0) return SHIPK_OK;  // no crops is not an error (ops.cu:421)
    // the reference's refusals, ops.cu:422-442
    if (candidates <= 0 || channels <= 0 || cells <= 0 || stride <= prefix || prefix < 0)
        return fail(SHIPK_EINVAL,
                    "%s: candidates, channels and cells must be positive and stride must exceed the prefix", who);
    // beyond the reference, for memory safety: the score column 4 and the coefficients must lie
    // inside a row
    if (stride < 5) return fail(SHIPK_EINVAL, "%s: a row of %d floats has no score column 4", who, stride);
    if (stride - prefix != channels)
        return fail(SHIPK_EINVAL,
                    "%s: the rows carry %d mask coefficient(s) and the bank has %d plane(s); the basis "
                    "would be truncated or overrun", who, stride - prefix, channels);
    if (!(mask_threshold > 0.f) || !(mask_threshold < 1.f))
        return fail(SHIPK_EINVAL, "%s: mask_threshold is a probability in (0, 1), so its logit exists", who);
    int rc;
    if ((rc = check_device_ptr(rows, who, "rows"))) return rc;
    if ((rc = check_device_ptr(protos, who, "protos"))) return rc;
    if ((rc = check_device_ptr(areas, who, "areas"))) return rc;
    Status s = launch_mask_area(rows, count, candidates, stride, prefix, protos, channels, cells, score_threshold,
                                mask_threshold, crop_height, crop_width, areas, static_cast<cudaStream_t>(stream));
    if (s.code) return fail_status(s, who);
    return SHIPK_OK;
}

// ---- the C++ data plane's per-frame calls (reference csrc/shipinfer/runtime/ops.h:38-120) ----

namespace {

// The reference's require_nv12_layout (ops.cu:325-339), with its wording, plus room for the last
// chroma pair of an odd width.
int check_nv12_layout(const char* who, int src_h, int src_w, int64_t stride, uint64_t uv_offset) {
    if (src_h < 1 || src_w < 1 || src_h > 32768 || src_w > 32768)
        return fail(SHIPK_EINVAL, "%s: frame is %dx%d; expected 1..32768 per side", who, src_h, src_w);
    const int64_t chroma_row = ((int64_t)(src_w + 1) / 2) * 2;
    if (stride < src_w || stride < chroma_row)
        return fail(SHIPK_EINVAL,
                    "%s: stride %lld is narrower than the width %d; a row cannot fit, so every row "
                    "would read into the next",
                    who, (long long)stride, src_w);
    if (uv_offset < (uint64_t)stride * (uint64_t)src_h)
        return fail(SHIPK_EINVAL,
                    "%s: uv_offset %llu is inside the luma plane (%lld x %d); pass `stride * src_h` "
                    "-- which is the answer for a tight buffer and for a mapped decoder surface alike",
                    who, (unsigned long long)uv_offset, (long long)stride, src_h);
    return SHIPK_OK;
}

const float kDpMean[3] = {0.f, 0.f, 0.f};
const float kDpStd[3] = {255.f, 255.f, 255.f};  // the data plane's value / 255

}  // namespace

int shipk_dp_letterbox_into(const uint8_t* src, int src_h, int src_w, float* dst, int dst_h, int dst_w,
                            int swap_rb, float pad_value, shipk_letterbox_map* map_out, void* stream) {
    static const char* who = "shipk_dp_letterbox_into";
    int rc = check_common(who, 1, dst_h, dst_w, SHIPK_DTYPE_F32, kDpMean, kDpStd);
    if (rc) return rc;
    if ((rc = check_u8_frame(who, 0, src, src_h, src_w, (int64_t)src_w * 3))) return rc;
    if ((rc = check_device_ptr(src, who, "src_device"))) return rc;
    if ((rc = check_device_ptr(dst, who, "dst_device"))) return rc;
    // the data plane's float32 placement (ops.cu:341-356), returned in map_out as the reference does
    const FrameView view{src, nullptr, src_h, src_w, (int64_t)src_w * 3, 0, 1};
    const float pad_out[3] = {pad_value, pad_value, pad_value};
    Status s = launch_letterbox(&view, 1, dst, SHIPK_DTYPE_F32, dst_h, dst_w, kDpMean, kDpStd, swap_rb, 0.f,
                                false, 601, 1, static_cast<cudaStream_t>(stream), pad_out);
    if (s.code) return fail_status(s, who);
    fill_maps(&view, 1, dst_h, dst_w, map_out);
    return SHIPK_OK;
}

int shipk_dp_crop_resize_into(const uint8_t* src, int src_h, int src_w, const float* boxes, int count,
                              float* dst, int dst_h, int dst_w, int swap_rb, void* stream) {
    static const char* who = "shipk_dp_crop_resize_into";
    if (count <= 0) return SHIPK_OK;  // no boxes is not an error (ops.cu:379)
    int rc = check_common(who, 1, dst_h, dst_w, SHIPK_DTYPE_F32, kDpMean, kDpStd);
    if (rc) return rc;
    if ((rc = check_u8_frame(who, 0, src, src_h, src_w, (int64_t)src_w * 3))) return rc;
    if ((rc = check_device_ptr(src, who, "src_device"))) return rc;
    if ((rc = check_device_ptr(boxes, who, "boxes_device"))) return rc;
    if ((rc = check_device_ptr(dst, who, "dst_device"))) return rc;
    const FrameView view{src, nullptr, src_h, src_w, (int64_t)src_w * 3, 0};
    Status s = launch_crop(&view, 1, boxes, nullptr, count, dst, SHIPK_DTYPE_F32, dst_h, dst_w, kDpMean, kDpStd,
                           swap_rb, static_cast<cudaStream_t>(stream));
    if (s.code) return fail_status(s, who);
    return SHIPK_OK;
}

int shipk_dp_nv12_letterbox_into(const uint8_t* nv12, int src_h, int src_w, int stride, size_t uv_offset,
                                 float* dst, int dst_h, int dst_w, int swap_rb, float pad_value,
                                 shipk_letterbox_map* map_out, void* stream) {
    static const char* who = "nv12_letterbox_into";
    int rc = check_nv12_layout(who, src_h, src_w, stride, uv_offset);
    if (rc) return rc;
    if ((rc = check_common(who, 1, dst_h, dst_w, SHIPK_DTYPE_F32, kDpMean, kDpStd))) return rc;
    if ((rc = check_device_ptr(nv12, who, "nv12_device"))) return rc;
    if ((rc = check_device_ptr(dst, who, "dst_device"))) return rc;
    // the data plane's float32 placement (ops.cu:341-356), as the reference kernel is launched with
    const FrameView view{nv12, nullptr, src_h, src_w, stride, (int64_t)uv_offset, 1};
    const float pad_out[3] = {pad_value, pad_value, pad_value};
    // BT.601 limited range, nearest tap at the reference kernel's source coordinate: the
    // reference's own nv12_letterbox_kernel, bit for bit
    Status s = launch_letterbox(&view, 1, dst, SHIPK_DTYPE_F32, dst_h, dst_w, kDpMean, kDpStd, swap_rb, 0.f,
                                true, 601, 0, static_cast<cudaStream_t>(stream), pad_out);
    if (s.code) return fail_status(s, who);
    fill_maps(&view, 1, dst_h, dst_w, map_out);
    return SHIPK_OK;
}

int shipk_dp_nv12_crop_resize_into(const uint8_t* nv12, int src_h, int src_w, int stride, size_t uv_offset,
                                   const float* boxes, int count, float* dst, int dst_h, int dst_w, int swap_rb,
                                   void* stream) {
    static const char* who = "nv12_crop_resize_into";
    if (count <= 0) return SHIPK_OK;  // no boxes is not an error (ops.cu:407)
    int rc = check_nv12_layout(who, src_h, src_w, stride, uv_offset);
    if (rc) return rc;
    if ((rc = check_common(who, 1, dst_h, dst_w, SHIPK_DTYPE_F32, kDpMean, kDpStd))) return rc;
    if ((rc = check_device_ptr(nv12, who, "nv12_device"))) return rc;
    if ((rc = check_device_ptr(boxes, who, "boxes_device"))) return rc;
    if ((rc = check_device_ptr(dst, who, "dst_device"))) return rc;
    const FrameView view{nv12, nullptr, src_h, src_w, stride, (int64_t)uv_offset};
    Status s = launch_crop_nv12(&view, 1, boxes, nullptr, count, dst, SHIPK_DTYPE_F32, dst_h, dst_w, swap_rb,
                                static_cast<cudaStream_t>(stream));
    if (s.code) return fail_status(s, who);
    return SHIPK_OK;
}

int shipk_normalise_check(float mean, float std_, unsigned long long* result, void* stream) {
    static const char* who = "shipk_normalise_check";
    if (!result) return fail(SHIPK_EINVAL, "%s: result is null", who);
    int rc = check_device_ptr(result, who, "result");
    if (rc) return rc;
    Status s = launch_normalise_check(mean, std_, result, static_cast<cudaStream_t>(stream));
    if (s.code) return fail_status(s, who);
    return SHIPK_OK;
}

int shipk_ctx_create(int device, shipk_ctx** out) {
    static const char* who = "shipk_ctx_create";
    if (!out) return fail(SHIPK_EINVAL, "%s: out is null", who);
    *out = nullptr;
    const int count = shipk_device_count();
    if (device < 0 || device >= count)
        return fail(SHIPK_EINVAL, "%s: device %d is not one of the %d visible devices", who, device,
                    count);
    DeviceGuard guard(device);
    if (guard.err != cudaSuccess) return fail_cuda(guard.err, who, "cudaSetDevice");
    shipk_ctx* ctx = new (std::nothrow) shipk_ctx();
    if (!ctx) return fail(SHIPK_ENOMEM, "%s: out of host memory", who);
    ctx->device = device;
    cudaError_t e = cudaEventCreateWithFlags(&ctx->done, cudaEventDisableTiming);
    if (e != cudaSuccess) {
        delete ctx;
        return fail_cuda(e, who, "cudaEventCreate");
    }
    *out = ctx;
    return SHIPK_OK;
}

void shipk_ctx_destroy(shipk_ctx* ctx) {
    if (!ctx) return;
    DeviceGuard guard(ctx->device);
    if (ctx->pending) cudaEventSynchronize(ctx->done);
    cudaFree(ctx->staging);
    cudaFree(ctx->row_map);
    cudaFree(ctx->boxes);
    cudaFree(ctx->nms_in);
    cudaFreeHost(ctx->host_rows);
    cudaFreeHost(ctx->host_boxes);
    cudaFreeHost(ctx->nms_host);
    cudaEventDestroy(ctx->done);
    delete ctx;
}

int shipk_ctx_letterbox_host(shipk_ctx* ctx, const shipk_host_frame_u8* frames, int n, void* out,
                             int out_dtype, size_t out_nbytes, int dst_h, int dst_w,
                             const float mean[3], const float std_[3], int swap_rb,
                             float pad_value, shipk_letterbox_map* maps_out, void* stream) {
    static const char* who = "shipk_ctx_letterbox_host";
    if (!ctx) return fail(SHIPK_EINVAL, "%s: ctx is null", who);
    int rc = check_common(who, n, dst_h, dst_w, out_dtype, mean, std_);
    if (rc) return rc;
    if (!frames) return fail(SHIPK_EINVAL, "%s: frames is null", who);
    if (out_nbytes < out_bytes(n, dst_h, dst_w, out_dtype))
        return fail(SHIPK_ENOMEM, "%s: out holds %zu bytes, the batch needs %zu", who, out_nbytes,
                    out_bytes(n, dst_h, dst_w, out_dtype));
    DeviceGuard guard(ctx->device);
    if (guard.err != cudaSuccess) return fail_cuda(guard.err, who, "cudaSetDevice");
    if ((rc = check_device_ptr(out, who, "out"))) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    // Which rows each frame's resize reads, and where they go in the staging buffer.
    std::vector<std::vector<unsigned char>> needed(n);
    std::vector<int64_t> stage_off(n), stage_pitch(n), map_off(n);
    int64_t stage_total = 0, map_total = 0;
    for (int i = 0; i < n; ++i) {
        const shipk_host_frame_u8& f = frames[i];
        if ((rc = check_u8_frame(who, i, f.data, f.height, f.width, f.pitch))) return rc;
        Fit fit;
        letterbox_fit(f.height, f.width, dst_h, dst_w, &fit);
        needed[i].assign(f.height, 0);
        letterbox_rows_needed(f.height, fit.new_h, needed[i].data());
        int64_t rows = 0;
        for (unsigned char v : needed[i]) rows += v;
        stage_pitch[i] = ((int64_t)f.width * 3 + 15) / 16 * 16;
        stage_off[i] = stage_total;
        stage_total += rows * stage_pitch[i];
        map_off[i] = map_total;
        map_total += f.height;
    }
    if ((rc = ctx_quiesce(ctx, who))) return rc;
    cudaError_t e = grow_device(&ctx->staging, &ctx->staging_bytes, (size_t)stage_total);
    if (e == cudaSuccess) e = grow_device(&ctx->row_map, &ctx->row_map_bytes, (size_t)map_total * 4);
    if (e == cudaSuccess) e = grow_pinned(&ctx->host_rows, &ctx->host_rows_bytes, (size_t)map_total * 4);
    if (e != cudaSuccess) return fail_cuda(e, who, "staging allocation");

    std::vector<FrameView> views(n);
    for (int i = 0; i < n; ++i) {
        const shipk_host_frame_u8& f = frames[i];
        rc = upload_rows(who, f.data, f.pitch, f.height, f.width * 3, needed[i].data(),
                         ctx->staging + stage_off[i], stage_pitch[i], ctx->host_rows + map_off[i], st);
        if (rc) return rc;
        views[i] = FrameView{ctx->staging + stage_off[i], ctx->row_map + map_off[i], f.height,
                             f.width, stage_pitch[i], 0};
    }
    e = cudaMemcpyAsync(ctx->row_map, ctx->host_rows, (size_t)map_total * 4, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return fail_cuda(e, who, "cudaMemcpyAsync(row map)");
    Status s = launch_letterbox(views.data(), n, out, out_dtype, dst_h, dst_w, mean, std_, swap_rb,
                                pad_value, false, 601, 1, st);
    if (s.code) return fail_status(s, who);
    e = cudaEventRecord(ctx->done, st);
    if (e != cudaSuccess) return fail_cuda(e, who, "cudaEventRecord");
    ctx->pending = true;
    fill_maps(views.data(), n, dst_h, dst_w, maps_out);
    return SHIPK_OK;
}

int shipk_ctx_crop_host(shipk_ctx* ctx, const shipk_host_frame_u8* frame, const float* boxes,
                        int n_boxes, void* out, int out_dtype, size_t out_nbytes, int dst_h,
                        int dst_w, const float mean[3], const float std_[3], int swap_rb,
                        void* stream) {
    static const char* who = "shipk_ctx_crop_host";
    if (!ctx) return fail(SHIPK_EINVAL, "%s: ctx is null", who);
    int rc = check_common(who, 1, dst_h, dst_w, out_dtype, mean, std_);
    if (rc) return rc;
    if (!frame) return fail(SHIPK_EINVAL, "%s: frame is null", who);
    if (n_boxes < 0) return fail(SHIPK_EINVAL, "%s: n_boxes is negative", who);
    if ((rc = check_u8_frame(who, 0, frame->data, frame->height, frame->width, frame->pitch))) return rc;
    if (n_boxes == 0) return SHIPK_OK;
    if (!boxes) return fail(SHIPK_EINVAL, "%s: boxes is null", who);
    if (out_nbytes < out_bytes(n_boxes, dst_h, dst_w, out_dtype))
        return fail(SHIPK_ENOMEM, "%s: out holds %zu bytes, %d crops need %zu", who, out_nbytes,
                    n_boxes, out_bytes(n_boxes, dst_h, dst_w, out_dtype));
    DeviceGuard guard(ctx->device);
    if (guard.err != cudaSuccess) return fail_cuda(guard.err, who, "cudaSetDevice");
    if ((rc = check_device_ptr(out, who, "out"))) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    const int h = frame->height, w = frame->width;
    std::vector<unsigned char> needed(h, 0);
    for (int b = 0; b < n_boxes; ++b) crop_rows_needed(boxes + 4 * (size_t)b, h, w, dst_h, needed.data());
    int64_t rows = 0;
    for (unsigned char v : needed) rows += v;
    const int64_t pitch = ((int64_t)w * 3 + 15) / 16 * 16;
    if ((rc = ctx_quiesce(ctx, who))) return rc;
    const size_t box_bytes = (size_t)n_boxes * 16;
    cudaError_t e = grow_device(&ctx->staging, &ctx->staging_bytes, (size_t)std::max<int64_t>(rows, 1) * pitch);
    if (e == cudaSuccess) e = grow_device(&ctx->row_map, &ctx->row_map_bytes, (size_t)h * 4);
    if (e == cudaSuccess) e = grow_pinned(&ctx->host_rows, &ctx->host_rows_bytes, (size_t)h * 4);
    if (e == cudaSuccess) e = grow_device(&ctx->boxes, &ctx->boxes_bytes, box_bytes);
    if (e == cudaSuccess) e = grow_pinned(&ctx->host_boxes, &ctx->host_boxes_bytes, box_bytes);
    if (e != cudaSuccess) return fail_cuda(e, who, "staging allocation");
    rc = upload_rows(who, frame->data, frame->pitch, h, w * 3, needed.data(), ctx->staging, pitch,
                     ctx->host_rows, st);
    if (rc) return rc;
    std::memcpy(ctx->host_boxes, boxes, box_bytes);
    e = cudaMemcpyAsync(ctx->row_map, ctx->host_rows, (size_t)h * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(ctx->boxes, ctx->host_boxes, box_bytes, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return fail_cuda(e, who, "cudaMemcpyAsync");
    FrameView view{ctx->staging, ctx->row_map, h, w, pitch, 0};
    Status s = launch_crop(&view, 1, ctx->boxes, nullptr, n_boxes, out, out_dtype, dst_h, dst_w, mean,
                           std_, swap_rb, st);
    if (s.code) return fail_status(s, who);
    e = cudaEventRecord(ctx->done, st);
    if (e != cudaSuccess) return fail_cuda(e, who, "cudaEventRecord");
    ctx->pending = true;
    return SHIPK_OK;
}

int shipk_ctx_nms_host(shipk_ctx* ctx, const float* boxes, const float* scores,
                       const int32_t* classes, int batch, int n, int num_classes, int class_aware,
                       float iou_threshold, float score_threshold, int max_det, int64_t* keep,
                       int32_t* counts, void* stream) {
    static const char* who = "shipk_ctx_nms_host";
    if (!ctx) return fail(SHIPK_EINVAL, "%s: ctx is null", who);
    int rc = check_nms_args(who, batch, n, num_classes, class_aware, max_det);
    if (rc) return rc;
    if (batch == 0) return SHIPK_OK;
    if (!counts || (max_det > 0 && !keep)) return fail(SHIPK_EINVAL, "%s: keep/counts are null", who);
    if (n > 0 && max_det > 0 && (!boxes || !scores || (class_aware && !classes)))
        return fail(SHIPK_EINVAL, "%s: boxes/scores/classes are null", who);
    DeviceGuard guard(ctx->device);
    if (guard.err != cudaSuccess) return fail_cuda(guard.err, who, "cudaSetDevice");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
    const size_t nb = (size_t)batch * n;
    const size_t o_boxes = 0, o_scores = up(nb * 16), o_classes = o_scores + up(nb * 4);
    const size_t o_keep = o_classes + up(class_aware ? nb * 4 : 0);
    const size_t o_counts = o_keep + up((size_t)batch * max_det * 8);
    const size_t o_ws = o_counts + up((size_t)batch * 4);
    const size_t ws = nms_workspace_bytes(batch, n, num_classes, class_aware, max_det);
    const size_t total = o_ws + ws;
    if ((rc = ctx_quiesce(ctx, who))) return rc;
    cudaError_t e = grow_device(&ctx->nms_in, &ctx->nms_in_bytes, total);
    if (e == cudaSuccess) e = grow_pinned(&ctx->nms_host, &ctx->nms_host_bytes, o_ws);
    if (e != cudaSuccess) return fail_cuda(e, who, "NMS buffer allocation");
    uint8_t* d = ctx->nms_in;
    uint8_t* h = ctx->nms_host;
    if (nb) {
        std::memcpy(h + o_boxes, boxes, nb * 16);
        std::memcpy(h + o_scores, scores, nb * 4);
        if (class_aware) std::memcpy(h + o_classes, classes, nb * 4);
        e = cudaMemcpyAsync(d, h, o_keep, cudaMemcpyHostToDevice, st);
        if (e != cudaSuccess) return fail_cuda(e, who, "cudaMemcpyAsync(inputs)");
    }
    Status s = launch_nms(reinterpret_cast<float*>(d + o_boxes), reinterpret_cast<float*>(d + o_scores),
                          class_aware ? reinterpret_cast<int32_t*>(d + o_classes) : nullptr, batch, n,
                          num_classes, class_aware, iou_threshold, score_threshold, max_det,
                          reinterpret_cast<int64_t*>(d + o_keep), reinterpret_cast<int32_t*>(d + o_counts),
                          d + o_ws, ws, true, st);
    if (s.code) return fail_status(s, who);
    e = cudaMemcpyAsync(h + o_keep, d + o_keep, o_ws - o_keep, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return fail_cuda(e, who, "result copy");
    if (max_det > 0) std::memcpy(keep, h + o_keep, (size_t)batch * max_det * 8);
    std::memcpy(counts, h + o_counts, (size_t)batch * 4);
    return SHIPK_OK;
}

}  // extern "C"
