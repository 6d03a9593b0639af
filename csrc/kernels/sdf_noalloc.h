// sdf_noalloc.h — the allocation-free exact distance transform of libsurf_vision.so.
//
// This entry point has no counterpart in the reference project, which computes
// its distance field on the host with scipy. It is an addition of this library
// for callers that must not allocate GPU memory: a plugin running inside a
// host program that reserved the whole device for its own pool up front (so a
// cudaMalloc from the plugin fails or steals from the host's budget), or a
// real-time loop that rules out allocation after start-up because cudaMalloc
// and cudaFree can stall the device. Such a caller passes device buffers it
// already owns; the function allocates nothing (no cudaMalloc, no cudaFree, no
// allocating library call) and keeps its per-line scratch in a file-scope
// device array compiled into the library.
//
// Contract:
//   occ     device pointer, uint8 [nz][ny][nx], 1 = solid voxel, 0 = free;
//   out     device pointer, float32 [nz][ny][nx]: the Euclidean distance (map
//           units, voxel pitch `cell`) from each voxel centre to the nearest
//           solid voxel centre, space outside the grid counting as solid; the
//           same values as the allocating surf_edt;
//   stream  the cudaStream_t to launch on (nullptr = the legacy default stream).
//   Returns 0 on success, otherwise a cudaError_t value; nothing is launched
//   when an argument is rejected (cudaErrorInvalidValue).
//
// Limits:
//   * every axis of the grid at most SURF_EDT_NOALLOC_MAX_LINE voxels; larger
//     grids, empty axes and null pointers are rejected;
//   * the scratch array is 1024 lines x (3 * 256 + 8) ints, about 3.2 MB, held
//     by every GPU that loads the library until the process exits;
//   * the first call on a device looks up the array's device address
//     (cudaGetSymbolAddress, with that device current) and caches it; make
//     that first call before any stream capture begins. The cache does not
//     survive cudaDeviceReset: do not call this function after a device reset
//     in the same process;
//   * every call on a device shares the one scratch array and leaves its own
//     contents in it (no part of it needs to start at zero: each line is
//     written before it is read). Calls that can overlap on the GPU, such as
//     calls on two streams without ordering between them, race and corrupt
//     each other's results; calls ordered on one stream are safe.
#pragma once

#include <stdint.h>

#define SURF_EDT_NOALLOC_MAX_LINE 256

#ifdef __cplusplus
extern "C" {
#endif

int surf_edt_noalloc(const uint8_t* occ, int nx, int ny, int nz, float cell, float* out, void* stream);

#ifdef __cplusplus
}
#endif
