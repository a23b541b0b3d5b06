// TEST INFRASTRUCTURE: HIP half-precision header -> CUDA's (see hip_runtime.h).
#pragma once
#include <cuda_fp16.h>
