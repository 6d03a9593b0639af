// surf_cuda.cuh — shared helpers for the framework's CUDA libraries.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

#define SURF_EXPORT extern "C" __attribute__((visibility("default")))

// Launch-status convention of every exported entry point: 0 on success,
// otherwise the cudaError_t of the failed launch/call.
#define SURF_RETURN_LAUNCH() return static_cast<int>(cudaGetLastError())

namespace surfk {

inline __host__ __device__ int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Device error flag (one int per device, shared by the kernels and read by
// the host after a step): the first error code wins. Codes 1-5 are the GEMM
// pipeline's bounded waits; the index checks of the data-driven gathers use
// the codes below (the offending access is skipped, its output zeroed).
enum ErrCode : int { kErrGatherIndex = 0x100, kErrStackIndex = 0x101, kErrLossIndex = 0x102 };
__device__ __forceinline__ void report_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ float bf16_to_f32(uint16_t h) { return __uint_as_float(static_cast<uint32_t>(h) << 16); }

// Round-to-nearest-even float -> bf16 bits (NaN kept quiet).
__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x7fffffu)) return static_cast<uint16_t>((u >> 16) | 0x40);
  u += 0x7fffu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

// Two floats -> packed bf16 pair (lo in the low half), round to nearest even:
// one hardware conversion instead of two integer sequences.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Bricked voxel addressing: 4x4x4 bricks of 64 elements, brick-major.
struct BrickGrid {
  int nx, ny, nz;          // logical dims
  int bx, by, bz;          // brick counts (dims rounded up to 4)
  __host__ __device__ int64_t index(int ix, int iy, int iz) const {
    int64_t brick = (static_cast<int64_t>(iz >> 2) * by + (iy >> 2)) * bx + (ix >> 2);
    return brick * 64 + (((iz & 3) << 4) | ((iy & 3) << 2) | (ix & 3));
  }
  __host__ __device__ int64_t size() const { return static_cast<int64_t>(bx) * by * bz * 64; }
};

inline BrickGrid make_brick_grid(int nx, int ny, int nz) {
  return BrickGrid{nx, ny, nz, (nx + 3) / 4, (ny + 3) / 4, (nz + 3) / 4};
}

}  // namespace surfk
