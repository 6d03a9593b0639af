// sdf.cu — GPU bake of the vision/goal occupancy grid and its Euclidean
// distance field (sm_100a).
//
// Occupancy (reference: src/env.c:673-698 plus python/surfgym/vision.py:
// 346-406): a voxel is solid when its centre is SOLID or SKY in the world's
// point hull (hull 0) or inside a solid brush entity. "Slab" sampling ORs in
// samples shifted by k*cell/4 (k = +-1, +-2) along each axis so that geometry
// thinner than a voxel cannot slip between centres. The reference samples the
// C tracer on CPU threads (13 full-grid passes); here one thread walks the
// clip tree for all samples of its voxel.
//
// Distance (reference: scipy.ndimage.distance_transform_edt on the padded
// occupancy, python/surfgym/vision.py:409-439): exact Euclidean distance from
// each free voxel centre to the nearest solid voxel centre, outside the grid
// counting as solid. Computed with the separable lower-envelope-of-parabolas
// transform of Felzenszwalb & Huttenlocher ("Distance Transforms of Sampled
// Functions", Theory of Computing 8, 2012): three 1-D passes (x, y, z), one
// thread per grid line.
#include <cuda_fp16.h>

#include <atomic>

#include "sdf_noalloc.h"
#include "surf_cuda.cuh"

namespace {

constexpr int kSolid = -2, kSky = -6, kEmpty = -1;

struct TreeView {
  const float4* planes;   // normal xyz, dist
  const int* ptype;       // 0..2 axial, 3..5 general
  const int3* nodes;      // plane, child0, child1
};

__device__ __forceinline__ int tree_contents(const TreeView& t, int num, float x, float y, float z) {
  int guard = 0;
  while (num >= 0 && guard++ < 4096) {
    const int3 nd = t.nodes[num];
    const float4 pl = t.planes[nd.x];
    const int ty = t.ptype[nd.x];
    const float d = ty == 0 ? x - pl.w : ty == 1 ? y - pl.w : ty == 2 ? z - pl.w : (x * pl.x + y * pl.y + z * pl.z) - pl.w;
    num = d >= 0.0f ? nd.y : nd.z;
  }
  return num < 0 ? num : kEmpty;
}

struct SolidEnt { int head; float ox, oy, oz; float lo[3], hi[3]; };

__global__ void occupancy_kernel(TreeView t, int world_head, const SolidEnt* ents, int n_ents, float mnx, float mny,
                                 float mnz, float cell, int nx, int ny, int nz, int slab, uint8_t* out) {
  const int64_t total = static_cast<int64_t>(nx) * ny * nz;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int ix = static_cast<int>(i % nx);
    const int iy = static_cast<int>((i / nx) % ny);
    const int iz = static_cast<int>(i / (static_cast<int64_t>(nx) * ny));
    const float cx = mnx + (ix + 0.5f) * cell, cy = mny + (iy + 0.5f) * cell, cz = mnz + (iz + 0.5f) * cell;
    const int nsamp = slab ? 13 : 1;
    bool solid = false;
    for (int s = 0; s < nsamp && !solid; ++s) {
      float x = cx, y = cy, z = cz;
      if (s > 0) {
        const int axis = (s - 1) >> 2, which = (s - 1) & 3;
        const float off = (which < 2 ? which - 2 : which - 1) * 0.25f * cell;   // -2,-1,+1,+2 quarters
        if (axis == 0) x += off; else if (axis == 1) y += off; else z += off;
      }
      const int c = tree_contents(t, world_head, x, y, z);
      if (c == kSolid || c == kSky) { solid = true; break; }
      for (int e = 0; e < n_ents; ++e) {
        const SolidEnt& se = ents[e];
        if (x < se.lo[0] || x > se.hi[0] || y < se.lo[1] || y > se.hi[1] || z < se.lo[2] || z > se.hi[2]) continue;
        if (tree_contents(t, se.head, x - se.ox, y - se.oy, z - se.oz) == kSolid) { solid = true; break; }
      }
    }
    out[i] = solid ? 1 : 0;
  }
}

constexpr int kMaxLine = 8192;
constexpr float kInf = 1e20f;
constexpr int kEdtBlocks = 148 * 4, kEdtThreads = 64;   // fixed grid: workspace is per thread

// Per-thread workspace of one line transform.
struct LineWs { int* v; float* zb; float* tmp; };

__device__ __forceinline__ LineWs line_ws(int* base, int maxn) {
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  int* p = base + tid * static_cast<int64_t>(3 * maxn + 8);
  return LineWs{p, reinterpret_cast<float*>(p + maxn + 2), reinterpret_cast<float*>(p + 2 * maxn + 5)};
}

// 1-D squared distance transform of one line: f[q] (squared distances in
// voxel units, 0 = solid site, kInf = no site) -> out[q * stride], with a
// solid site just outside each end of the line.
template <typename F, typename Out>
__device__ void edt_line(F fval_in, Out* out, int64_t stride, int n, LineWs ws) {
  int* v = ws.v;
  float* zb = ws.zb;
  auto fval = [&](int q) -> float { return (q < 0 || q >= n) ? 0.0f : fval_in(q); };
  int k = 0;
  v[0] = -1;
  zb[0] = -kInf;
  zb[1] = kInf;
  for (int q = 0; q <= n; ++q) {
    const float fq = fval(q);
    if (fq >= kInf) continue;
    float s;
    for (;;) {
      const int p = v[k];
      const float fp = fval(p);
      s = ((fq + static_cast<float>(q) * q) - (fp + static_cast<float>(p) * p)) / (2.0f * static_cast<float>(q - p));
      if (s <= zb[k] && k > 0) { --k; continue; }
      break;
    }
    if (s <= zb[k]) k = -1;          // k == 0 and the new parabola dominates everywhere
    ++k;
    v[k] = q;
    zb[k] = (k == 0) ? -kInf : s;
    zb[k + 1] = kInf;
  }
  k = 0;
  for (int q = 0; q < n; ++q) {
    while (zb[k + 1] < static_cast<float>(q)) ++k;
    const int p = v[k];
    const float d = static_cast<float>(q - p);
    out[q * stride] = d * d + fval(p);
  }
}

// pass over x lines: occupancy -> squared distance along x
__global__ void __launch_bounds__(kEdtThreads) edt_x_kernel(const uint8_t* occ, float* d2, int nx, int ny, int nz,
                                                             int* ws, int maxn) {
  const LineWs w = line_ws(ws, maxn);
  const int64_t lines = static_cast<int64_t>(ny) * nz;
  for (int64_t l = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; l < lines;
       l += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint8_t* in = occ + l * nx;
    for (int q = 0; q < nx; ++q) w.tmp[q] = in[q] ? 0.0f : kInf;
    edt_line([&](int q) { return w.tmp[q]; }, d2 + l * nx, 1, nx, w);
  }
}

// pass over y (axis=1) or z (axis=2) lines, in place
__global__ void __launch_bounds__(kEdtThreads) edt_yz_kernel(float* d2, int nx, int ny, int nz, int axis, int* ws,
                                                              int maxn) {
  const LineWs w = line_ws(ws, maxn);
  const int n = axis == 1 ? ny : nz;
  const int64_t stride = axis == 1 ? nx : static_cast<int64_t>(nx) * ny;
  const int64_t lines = static_cast<int64_t>(nx) * (axis == 1 ? nz : ny);
  for (int64_t l = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; l < lines;
       l += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int ix = static_cast<int>(l % nx);
    const int64_t other = l / nx;
    const int64_t base = axis == 1 ? (other * static_cast<int64_t>(ny) * nx + ix) : (other * nx + ix);
    for (int q = 0; q < n; ++q) w.tmp[q] = d2[base + q * stride];
    edt_line([&](int q) { return w.tmp[q]; }, d2 + base, stride, n, w);
  }
}

__global__ void finish_kernel(const float* d2, float cell, int64_t total, float* out_f32, __half* out_f16) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float d = sqrtf(d2[i]) * cell;
    if (out_f32) out_f32[i] = d;
    if (out_f16) out_f16[i] = __float2half_rn(fminf(d, 65504.0f));
  }
}

int grid_blocks(int64_t work, int threads) {
  int64_t b = surfk::ceil_div(work, threads);
  return static_cast<int>(b < 148 * 32 ? (b < 1 ? 1 : b) : 148 * 32);
}

}  // namespace

// Occupancy of an nx*ny*nz grid of `cell` voxels starting at mins (voxel
// centres at mins + (i + 0.5) * cell). ents: n_ents records of 10 floats
// (head as float bits, origin xyz, absmin xyz, absmax xyz) for solid brush
// entities. slab != 0 adds the 12 shifted samples per voxel.
SURF_EXPORT int surf_occupancy(const float* planes4, const int* ptype, const int* nodes3, int world_head,
                               const void* ents, int n_ents, float mnx, float mny, float mnz, float cell, int nx,
                               int ny, int nz, int slab, uint8_t* out, void* stream) {
  TreeView t{reinterpret_cast<const float4*>(planes4), ptype, reinterpret_cast<const int3*>(nodes3)};
  const int64_t total = static_cast<int64_t>(nx) * ny * nz;
  occupancy_kernel<<<grid_blocks(total, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      t, world_head, static_cast<const SolidEnt*>(ents), n_ents, mnx, mny, mnz, cell, nx, ny, nz, slab, out);
  SURF_RETURN_LAUNCH();
}

SURF_EXPORT int64_t surf_edt_workspace_bytes(int nx, int ny, int nz) {
  int maxn = nx > ny ? nx : ny;
  maxn = maxn > nz ? maxn : nz;
  return static_cast<int64_t>(kEdtBlocks) * kEdtThreads * (3 * maxn + 8) * 4;
}

// Exact EDT of the free space of `occ` (uint8, [nz][ny][nx]), distances in
// map units (voxel distance * cell). d2: float workspace of nx*ny*nz
// elements; ws: surf_edt_workspace_bytes bytes. Outputs (either may be
// null): float32 linear, fp16 linear.
SURF_EXPORT int surf_edt(const uint8_t* occ, int nx, int ny, int nz, float cell, float* d2, void* ws,
                         float* out_f32, void* out_f16, void* stream) {
  if (nx > kMaxLine || ny > kMaxLine || nz > kMaxLine) return static_cast<int>(cudaErrorInvalidValue);
  int maxn = nx > ny ? nx : ny;
  maxn = maxn > nz ? maxn : nz;
  auto s = static_cast<cudaStream_t>(stream);
  int* w = static_cast<int*>(ws);
  edt_x_kernel<<<kEdtBlocks, kEdtThreads, 0, s>>>(occ, d2, nx, ny, nz, w, maxn);
  edt_yz_kernel<<<kEdtBlocks, kEdtThreads, 0, s>>>(d2, nx, ny, nz, 1, w, maxn);
  edt_yz_kernel<<<kEdtBlocks, kEdtThreads, 0, s>>>(d2, nx, ny, nz, 2, w, maxn);
  const int64_t total = static_cast<int64_t>(nx) * ny * nz;
  finish_kernel<<<grid_blocks(total, 256), 256, 0, s>>>(d2, cell, total, out_f32, static_cast<__half*>(out_f16));
  SURF_RETURN_LAUNCH();
}

// ---------------------------------------------------------------------------
// surf_edt_noalloc — the exact EDT without any device allocation.
//
// Declared, with its full contract, in sdf_noalloc.h; it has no counterpart in
// the reference project (which runs its distance transform through scipy on
// the host). It serves callers that must not allocate GPU memory: a plugin in
// a host program that reserved the whole device for its own pool, or a
// real-time loop that forbids cudaMalloc/cudaFree after start-up because they
// can stall the device. The caller passes the occupancy grid and the float32
// output; the output doubles as the squared-distance buffer of the three
// passes, and the per-line scratch lives in the file-scope array below.
//
// Limits and behaviour:
//   * every grid axis must be <= SURF_EDT_NOALLOC_MAX_LINE (256) voxels;
//     larger grids, empty axes and null pointers return cudaErrorInvalidValue
//     without launching anything;
//   * the scratch is a static device array of 1024 lines x (3*256+8) ints
//     (about 3.2 MB); every GPU that loads this library keeps it until the
//     process exits;
//   * its device address is looked up once per device (cudaGetSymbolAddress,
//     with that device current) by the first call made on the device, so that
//     first call should happen before any stream capture begins. Two host
//     threads making that first call together both look it up and store the
//     same value (atomic per-device slots). The cached address is not valid
//     after cudaDeviceReset;
//   * every call on a device shares the one scratch array: calls that can
//     overlap on the GPU (different streams without ordering) race and corrupt
//     each other's results. Calls on one stream are safe. No part of the
//     scratch needs to start at zero (each line is written before it is read).
// ---------------------------------------------------------------------------
namespace {
constexpr int kNoAllocMaxLine = SURF_EDT_NOALLOC_MAX_LINE;
constexpr int kNoAllocBlocks = 16;                        // x kEdtThreads = 1024 concurrent lines
constexpr int kNoAllocInts = kNoAllocBlocks * kEdtThreads * (3 * kNoAllocMaxLine + 8);
static __device__ __align__(256) int g_edt_noalloc_ws[kNoAllocInts];

constexpr int kMaxDevices = 64;
std::atomic<int*> g_ws_addr[kMaxDevices];                 // zero-initialised (static storage)
}  // namespace

SURF_EXPORT int surf_edt_noalloc(const uint8_t* occ, int nx, int ny, int nz, float cell, float* out, void* stream) {
  if (!occ || !out || nx < 1 || ny < 1 || nz < 1 || nx > kNoAllocMaxLine || ny > kNoAllocMaxLine ||
      nz > kNoAllocMaxLine)
    return static_cast<int>(cudaErrorInvalidValue);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (dev < 0 || dev >= kMaxDevices) return static_cast<int>(cudaErrorInvalidDevice);
  int* ws = g_ws_addr[dev].load(std::memory_order_acquire);
  if (!ws) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_edt_noalloc_ws);
    if (e != cudaSuccess) return static_cast<int>(e);
    ws = static_cast<int*>(p);
    g_ws_addr[dev].store(ws, std::memory_order_release);
  }
  auto s = static_cast<cudaStream_t>(stream);
  edt_x_kernel<<<kNoAllocBlocks, kEdtThreads, 0, s>>>(occ, out, nx, ny, nz, ws, kNoAllocMaxLine);
  edt_yz_kernel<<<kNoAllocBlocks, kEdtThreads, 0, s>>>(out, nx, ny, nz, 1, ws, kNoAllocMaxLine);
  edt_yz_kernel<<<kNoAllocBlocks, kEdtThreads, 0, s>>>(out, nx, ny, nz, 2, ws, kNoAllocMaxLine);
  const int64_t total = static_cast<int64_t>(nx) * ny * nz;
  finish_kernel<<<grid_blocks(total, 256), 256, 0, s>>>(out, cell, total, out, nullptr);
  SURF_RETURN_LAUNCH();
}

// ---------------------------------------------------------------------------
// Surface slope mask: per voxel, |n_z| * 127 of the solid face the voxel holds
// (reference: python/surfgym/surfmask.py:112-179, the second lidar channel).
// Depth alone cannot tell floor (n_z = 1), surf ramp (~0.3-0.7) and wall (0)
// apart; the march reads this byte at the voxel where it stopped.
//
// Claims follow the reference's rules, resolved in one pass with a 64-bit
// atomicMax instead of two ordered host passes: a triangle claims every voxel
// of its dilated box whose centre lies within the margin radius
// 0.5*cell*(|nx|+|ny|+|nz|) + 0.5*cell of its plane, EXACT when also within
// the tight radius 0.5*cell*(|nx|+|ny|+|nz|). Key = exact (bit 63) | float32
// bits of twice the area (bits 31..62) | triangle index (bits 7..30) | value
// (bits 0..6), so an exact claim beats a margin claim, then the larger area
// wins, then the later triangle (the reference's stable ascending-area write
// order). The mesh here is the hull-0 solid-leaf polyhedra, which include
// faces between two solid cells: a triangle whose outward side is solid at
// all four probe points (centroid and the three centroid-vertex midpoints,
// 0.25 units out) is inside geometry and claims nothing.
namespace {

__device__ bool outside_solid(const TreeView& t, int world_head, const SolidEnt* ents, int n_ents, float x, float y,
                              float z) {
  const int c = tree_contents(t, world_head, x, y, z);
  if (c == kSolid || c == kSky) return true;
  for (int e = 0; e < n_ents; ++e) {
    const SolidEnt& se = ents[e];
    if (x < se.lo[0] || x > se.hi[0] || y < se.lo[1] || y > se.hi[1] || z < se.lo[2] || z > se.hi[2]) continue;
    if (tree_contents(t, se.head, x - se.ox, y - se.oy, z - se.oz) == kSolid) return true;
  }
  return false;
}

__global__ void __launch_bounds__(256) surfnz_claim_kernel(const float* tris, int n_tris, TreeView tv, int world_head,
                                                           const SolidEnt* ents, int n_ents, double mnx, double mny,
                                                           double mnz, double cell, int nx, int ny, int nz,
                                                           unsigned long long* keys) {
  const int ti = blockIdx.x;
  if (ti >= n_tris) return;
  const float* v = tris + 9 * static_cast<int64_t>(ti);
  const double ax = v[0], ay = v[1], az = v[2], bx = v[3], by = v[4], bz = v[5], cx = v[6], cy = v[7], cz = v[8];
  const double ux = bx - ax, uy = by - ay, uz = bz - az, wx = cx - ax, wy = cy - ay, wz = cz - az;
  // explicit round-to-nearest products and sums (no FMA contraction): every
  // decision below is reproducible bit for bit by a float64 host oracle
  const double crx = __dsub_rn(__dmul_rn(uy, wz), __dmul_rn(uz, wy));
  const double cry = __dsub_rn(__dmul_rn(uz, wx), __dmul_rn(ux, wz));
  const double crz = __dsub_rn(__dmul_rn(ux, wy), __dmul_rn(uy, wx));
  const double area2 = sqrt(__dadd_rn(__dadd_rn(__dmul_rn(crx, crx), __dmul_rn(cry, cry)), __dmul_rn(crz, crz)));
  if (!(area2 > 1e-9)) return;                              // degenerate fan triangle
  const double n0 = crx / area2, n1 = cry / area2, n2 = crz / area2;
  const unsigned val = static_cast<unsigned>(rint(fabs(n2) * 127.0));
  const double tight = __dmul_rn(0.5 * cell, fabs(n0) + fabs(n1) + fabs(n2));
  const double margin = tight + 0.5 * cell;
  const double pd = __dadd_rn(__dadd_rn(__dmul_rn(n0, ax), __dmul_rn(n1, ay)), __dmul_rn(n2, az));
  const double lo_v[3] = {fmin(ax, fmin(bx, cx)), fmin(ay, fmin(by, cy)), fmin(az, fmin(bz, cz))};
  const double hi_v[3] = {fmax(ax, fmax(bx, cx)), fmax(ay, fmax(by, cy)), fmax(az, fmax(bz, cz))};
  const double mn[3] = {mnx, mny, mnz};
  const int dim[3] = {nx, ny, nz};
  int lo[3], span[3];
  for (int a = 0; a < 3; ++a) {
    const double l = floor((lo_v[a] - cell - mn[a]) / cell), h = floor((hi_v[a] + cell - mn[a]) / cell) + 1.0;
    const int li = static_cast<int>(fmin(fmax(l, 0.0), static_cast<double>(dim[a])));
    const int hi = static_cast<int>(fmin(fmax(h, 0.0), static_cast<double>(dim[a])));
    lo[a] = li;
    span[a] = hi - li;
    if (span[a] <= 0) return;                               // entirely outside the grid
  }
  const unsigned long long base = (static_cast<unsigned long long>(__float_as_uint(static_cast<float>(area2))) << 31) |
                                  (static_cast<unsigned long long>(ti & 0xFFFFFF) << 7) | val;
  const int64_t plane = static_cast<int64_t>(span[0]) * span[1];
  const int64_t total = plane * span[2];
  if (blockIdx.y * static_cast<int64_t>(blockDim.x) >= total) return;   // no voxels for this slice
  if (tv.nodes) {                                           // internal face filter
    const double gx = (ax + bx + cx) / 3.0, gy = (ay + by + cy) / 3.0, gz = (az + bz + cz) / 3.0;
    bool open = false;
    for (int s = 0; s < 4 && !open; ++s) {
      double px = gx, py = gy, pz = gz;
      if (s > 0) {
        const float* q = v + 3 * (s - 1);
        px = 0.5 * (gx + q[0]); py = 0.5 * (gy + q[1]); pz = 0.5 * (gz + q[2]);
      }
      open = !outside_solid(tv, world_head, ents, n_ents, static_cast<float>(px + 0.25 * n0),
                            static_cast<float>(py + 0.25 * n1), static_cast<float>(pz + 0.25 * n2));
    }
    if (!open) return;
  }
  for (int64_t i = blockIdx.y * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.y) * blockDim.x) {
    const int x = lo[0] + static_cast<int>(i % span[0]);
    const int y = lo[1] + static_cast<int>((i / span[0]) % span[1]);
    const int z = lo[2] + static_cast<int>(i / plane);
    const double pz = __dmul_rn(__dadd_rn(__dmul_rn(z + 0.5, cell), mnz), n2);
    const double py = __dmul_rn(__dadd_rn(__dmul_rn(y + 0.5, cell), mny), n1);
    const double px = __dmul_rn(__dadd_rn(__dmul_rn(x + 0.5, cell), mnx), n0);
    const double dist = __dsub_rn(__dadd_rn(__dadd_rn(pz, py), px), pd);
    const double ad = fabs(dist);
    if (ad > margin) continue;
    const unsigned long long key = base | (ad <= tight ? (1ull << 63) : 0ull);
    atomicMax(keys + (static_cast<int64_t>(z) * ny + y) * nx + x, key);
  }
}

__global__ void surfnz_finish_kernel(const unsigned long long* keys, int nx, int ny, int nz, surfk::BrickGrid g,
                                     int8_t* linear, int8_t* bricked) {
  const int64_t total = static_cast<int64_t>(nx) * ny * nz;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const unsigned long long k = keys[i];
    const int8_t v = static_cast<int8_t>(k ? (k & 127ull) : 0ull);
    if (linear) linear[i] = v;
    if (bricked) {
      const int ix = static_cast<int>(i % nx), iy = static_cast<int>((i / nx) % ny);
      const int iz = static_cast<int>(i / (static_cast<int64_t>(nx) * ny));
      bricked[g.index(ix, iy, iz)] = v;
    }
  }
}

}  // namespace

// Bake the slope mask. tris: n_tris x 9 float32 (three xyz vertices, outward
// winding). planes4/ptype/nodes3/world_head/ents: the hull-0 tree and solid
// entities (the occupancy bake's inputs) for the internal-face filter; pass
// nodes3 = NULL to skip the filter. keys: nx*ny*nz uint64 workspace. Outputs
// (either may be NULL): linear int8 [nz][ny][nx] and the 4x4x4-bricked int8
// grid (surf_brick_size(nx, ny, nz) bytes, padding voxels zero).
SURF_EXPORT int surf_surfnz_bake(const float* tris, int n_tris, const float* planes4, const int* ptype,
                                 const int* nodes3, int world_head, const void* ents, int n_ents, double mnx,
                                 double mny, double mnz, double cell, int nx, int ny, int nz, void* keys,
                                 int8_t* linear, int8_t* bricked, void* stream) {
  if (n_tris < 0 || n_tris > (1 << 24) || nx < 1 || ny < 1 || nz < 1 || !keys || !(cell > 0.0))
    return static_cast<int>(cudaErrorInvalidValue);
  auto s = static_cast<cudaStream_t>(stream);
  const int64_t total = static_cast<int64_t>(nx) * ny * nz;
  cudaError_t e = cudaMemsetAsync(keys, 0, static_cast<size_t>(total) * 8, s);
  if (e != cudaSuccess) return static_cast<int>(e);
  const surfk::BrickGrid g = surfk::make_brick_grid(nx, ny, nz);
  if (bricked) {
    e = cudaMemsetAsync(bricked, 0, static_cast<size_t>(g.size()), s);
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  TreeView tv{reinterpret_cast<const float4*>(planes4), ptype, reinterpret_cast<const int3*>(nodes3)};
  if (n_tris > 0) {
    surfnz_claim_kernel<<<dim3(static_cast<unsigned>(n_tris), 8), 256, 0, s>>>(
        tris, n_tris, tv, world_head, static_cast<const SolidEnt*>(ents), n_ents, mnx, mny, mnz, cell, nx, ny, nz,
        static_cast<unsigned long long*>(keys));
    e = cudaGetLastError();
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  surfnz_finish_kernel<<<grid_blocks(total, 256), 256, 0, s>>>(static_cast<const unsigned long long*>(keys), nx, ny,
                                                                nz, g, linear, bricked);
  SURF_RETURN_LAUNCH();
}
