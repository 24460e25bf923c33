// The types the C++ data plane's pixel calls use, for building ops_shipk.cpp and crop_batch.cpp
// outside the reference tree. Inside it, the reference's own core/types.h (types.h:60-75)
// provides them with the same names, fields and bases, and this header is not on the include
// path.
#pragma once

#include <stdexcept>

namespace shipinfer {

// One detection of a frame, as the decode writes it (reference core/types.h:60-65): the box in
// frame pixels, its score and class, and its position within the frame.
struct Detection {
    float x1 = 0, y1 = 0, x2 = 0, y2 = 0;
    float score = 0;
    int class_id = 0;
    int index = 0;
};

// A caller's argument or a frame's layout is unusable: fix the call, not the device.
struct ConfigError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

// The device or its runtime failed the call.
struct BackendError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

}  // namespace shipinfer
