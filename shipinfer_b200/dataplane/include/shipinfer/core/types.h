// The two error types the C++ data plane's pixel calls throw, for building ops_shipk.cpp
// outside the reference tree. Inside it, the reference's own core/types.h (types.h:70-75)
// provides them with the same names and bases, and this header is not on the include path.
#pragma once

#include <stdexcept>

namespace shipinfer {

// A caller's argument or a frame's layout is unusable: fix the call, not the device.
struct ConfigError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

// The device or its runtime failed the call.
struct BackendError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

}  // namespace shipinfer
