// hd.hpp — what lets the simulator's per-player code compile twice: as host
// C++ (g++, the CPU env batch) and as CUDA device code (nvcc, the GPU env
// batch, one thread per env). Every function on that path is SURF_HD and
// reads the map through MapView's plain pointers, so both builds run the
// same source, operation for operation.
#pragma once
#include <cstdint>

#if defined(__CUDACC__)
#define SURF_HD __host__ __device__
#else
#define SURF_HD
#endif
// Device code: keep one out-of-line copy (one stack frame) of a function that
// would otherwise be inlined at every call site with its own local arrays.
#if defined(__CUDA_ARCH__)
#define SURF_HD_NOINLINE __noinline__
#else
#define SURF_HD_NOINLINE inline
#endif

namespace surf {

// Read-only array view (host or device memory).
template <typename T>
struct Span {
  const T* p = nullptr;
  int32_t n = 0;
  SURF_HD int32_t size() const { return n; }
  SURF_HD bool empty() const { return n == 0; }
  SURF_HD const T& operator[](int32_t i) const { return p[i]; }
  SURF_HD const T* begin() const { return p; }
  SURF_HD const T* end() const { return p + n; }
  SURF_HD const T* data() const { return p; }
};

// Player hull boxes by pmove "usehull" (0 stand, 1 duck, 2 point, 3 large)
// and clip-hull boxes by BSP hull index (0 point, 1 human, 2 large, 3
// crouch): GoldSrc engine constants, as functions so device code can read them.
SURF_HD inline float player_mins(int usehull, int k) {
  const float t[4][3] = {{-16, -16, -36}, {-16, -16, -18}, {0, 0, 0}, {-32, -32, -32}};
  return t[usehull][k];
}
SURF_HD inline float player_maxs(int usehull, int k) {
  const float t[4][3] = {{16, 16, 36}, {16, 16, 18}, {0, 0, 0}, {32, 32, 32}};
  return t[usehull][k];
}
SURF_HD inline float hull_mins(int bsp_hull, int k) {
  const float t[4][3] = {{0, 0, 0}, {-16, -16, -36}, {-32, -32, -32}, {-16, -16, -18}};
  return t[bsp_hull][k];
}
SURF_HD inline float hull_maxs(int bsp_hull, int k) {
  const float t[4][3] = {{0, 0, 0}, {16, 16, 36}, {32, 32, 32}, {16, 16, 18}};
  return t[bsp_hull][k];
}

}  // namespace surf
