// TEST INFRASTRUCTURE.  Minimal HIP -> CUDA name shim, used only to compile the
// reference's own csrc/nova_winograd.hip with nvcc into oracle/_ref/ so that
// the reference kernels themselves can check the CPU oracle on a GPU.  Nothing
// in the product library includes this file.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#define hipError_t cudaError_t
#define hipSuccess cudaSuccess
#define hipGetErrorString cudaGetErrorString
#define hipMalloc cudaMalloc
#define hipFree cudaFree
#define hipMemcpy cudaMemcpy
#define hipMemcpyHostToDevice cudaMemcpyHostToDevice
#define hipMemcpyDeviceToHost cudaMemcpyDeviceToHost
#define hipMemcpyToSymbol cudaMemcpyToSymbol
#define hipGetLastError cudaGetLastError
#define hipDeviceSynchronize cudaDeviceSynchronize
#define hipStream_t cudaStream_t
#define hipLaunchKernelGGL(kernel, grid, block, smem, stream, ...) \
  kernel<<<(grid), (block), (smem), (stream)>>>(__VA_ARGS__)

// AMD wavefronts are 64 lanes wide and the reference's multi-tile kernels
// exchange values across all 64 lanes with __shfl(v, lane, 64).  A CUDA warp
// has 32 lanes, so the exchange goes through shared memory instead: each
// 64-thread group of the block synchronises on its own named barrier (ids
// 1..16; the group either runs the exchange with all 64 threads or has
// returned as a whole, which is how those kernels are written), publishes its
// value and reads the source lane's.  The values exchanged are exact, so the
// kernels compute what they compute on a 64-lane wavefront.
__device__ __forceinline__ float nova_ref_wave64_shfl(float v, int src, int width) {
  __shared__ float xch[1024];
  const unsigned group = threadIdx.x >> 6;
  asm volatile("bar.sync %0, 64;" ::"r"(group + 1u) : "memory");
  xch[threadIdx.x] = v;
  asm volatile("bar.sync %0, 64;" ::"r"(group + 1u) : "memory");
  return xch[(threadIdx.x & ~63u) + (unsigned)(src & (width - 1))];
}
#define __shfl nova_ref_wave64_shfl
