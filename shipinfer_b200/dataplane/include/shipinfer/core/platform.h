// The stream type of the C++ data plane's calls, for building ops_shipk.cpp outside the
// reference tree (whose core/platform.h defines gpuStream_t for its CUDA build the same way).
#pragma once

#include <cuda_runtime.h>

#include "shipinfer/core/types.h"

using gpuStream_t = cudaStream_t;
