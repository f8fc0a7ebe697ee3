// Internal declarations shared by the library's translation units.
#pragma once
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "../../include/q4gpu.h"

// Blocks of the persistent LM-head kernel (3 resident CTAs on each of 148 SMs).
#define Q4GPU_LM_HEAD_BLOCKS 444
// Devices the library keeps per-device state for.
#define Q4GPU_MAX_DEVICES 64

// Record an error message for q4gpu_last_error() and return `code`.
int q4gpu_fail(int code, const char* fmt, ...);
// Check the last kernel launch; returns Q4GPU_OK or Q4GPU_ERR_CUDA.
int q4gpu_check_launch();
