// march.cu — SDF sphere-traced depth camera for every env (sm_100a).
//
// Behaviour (reference: python/surfgym/vision.py:59-265, the three Triton
// march kernels): per ray, eye = origin + 17 (12 ducked) up; direction from
// yaw/pitch plus a per-pixel angle (equiangular) or a tangent-plane offset
// (pinhole); march t over a nearest-voxel unsigned distance field: a ray stops
// once d <= 0.6*cell or t >= range, otherwise t += max(0.9*d, 0.3*cell), up to
// max_steps; encode depth as min(t,near)/near + 0.25*(1 - exp(-max(t-near,0)/2500)).
//
// B200 design (not a translation of the Triton kernels):
//   * one thread per ray, each warp a 16x2 pixel patch of one env: the 32
//     rays of a warp stay within a few voxels of each other, so a step's 32
//     gathers hit one or two 128-byte lines;
//   * the SDF is stored in 4x4x4 fp16 bricks (one brick = one 128 B line),
//     which keeps vertical and diagonal steps in the same line, unlike a
//     linear z-y-x layout where a z step is nx*ny*2 bytes away;
//   * per-thread early exit (a warp retires when its last ray stops);
//   * the pose is read straight from the env's step record, and the depth is
//     written in the policy's input dtype and layout (NHW, or the 4x4
//     space-to-depth layout that turns conv1's 8x8/stride-4 filter into a
//     2x2/stride-1 one), directly into a rollout buffer row.
#include <cuda_fp16.h>

#include "surf_cuda.cuh"

using surfk::BrickGrid;

namespace {

struct MarchParams {
  const float* pose;      // per env row: x, y, z, yaw_deg, pitch_deg, ducked
  int64_t pose_stride;    // floats between env rows
  int n_env, H, W;
  const __half* sdf;      // bricked distances (map units)
  BrickGrid grid;
  float mnx, mny, mnz, cell, inv_cell;
  const float* col_off;   // per column: yaw offset (rad) | pinhole u
  const float* row_off;   // per row: pitch offset (rad) | pinhole v
  float range, near_range;
  int max_steps;
  void* out;              // depth (float or bf16)
  int64_t out_stride;     // elements between env images
  const int8_t* surf_nz;  // optional bricked |n_z|*127 grid (second channel)
  int exit_outside;       // grid padded by >= 1 free layer: skip loads once a ray leaves it
  int flags;              // bit 2: 64-bit voxel addressing even for small grids (timing comparisons)
  int idx32;              // the bricked grid has < 2^31 elements: 32-bit voxel addressing
  uint8_t* steps;         // optional per-ray step census [n_env, H, W]
  const int32_t* env_order;  // optional: the env each run of blocks renders (a permutation of [0, n_env))
};

enum Layout : int { kNHW = 0, kS2D4 = 1 };

template <typename T> __device__ __forceinline__ void store(T* p, float v);
template <> __device__ __forceinline__ void store<float>(float* p, float v) { *p = v; }
template <> __device__ __forceinline__ void store<uint16_t>(uint16_t* p, float v) { *p = surfk::f32_to_bf16(v); }

__device__ __forceinline__ int voxel(float p, float mn, float inv, int n) {
  float f = (p - mn) * inv;
  f = fminf(fmaxf(f, 0.0f), static_cast<float>(n - 1));
  return static_cast<int>(f);
}

template <int kPinhole, typename OutT, int kLayout, bool kSurfNz>
__global__ void __launch_bounds__(128) march_kernel(MarchParams p) {
  const int tiles_w = (p.W + 15) >> 4;
  const int tiles = tiles_w * ((p.H + 7) >> 3);
  const int nb = blockIdx.x / tiles;
  const int tile = blockIdx.x - nb * tiles;
  // with env_order, consecutive envs of the launch are spatial neighbours
  // (the host env's Morton order): their rays share SDF bricks in L2
  const int n = p.env_order ? __ldg(p.env_order + nb) : nb;
  if (n < 0) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = (tile % tiles_w) * 16 + (lane & 15);
  const int r = (tile / tiles_w) * 8 + warp * 2 + (lane >> 4);
  if (n >= p.n_env || r >= p.H || c >= p.W) return;

  const float* pz = p.pose + n * p.pose_stride;
  const float ex = __ldg(pz + 0), ey = __ldg(pz + 1);
  const float ez = __ldg(pz + 2) + (__ldg(pz + 5) != 0.0f ? 12.0f : 17.0f);
  const float d2r = 0.017453292519943295f;
  const float yaw = __ldg(pz + 3) * d2r, pitch = __ldg(pz + 4) * d2r;
  float dx, dy, dz;
  if (kPinhole) {
    // forward + u*right + v*up with right = (sin y, -cos y, 0) and
    // up = (-sin p cos y, -sin p sin y, cos p); col 0 looks left, row 0 up.
    float sy, cy, sp, cp;
    sincosf(yaw, &sy, &cy);
    sincosf(pitch, &sp, &cp);
    const float u = __ldg(p.col_off + c), v = __ldg(p.row_off + r);
    dx = cp * cy + u * sy - v * sp * cy;
    dy = cp * sy - u * cy - v * sp * sy;
    dz = sp + v * cp;
    const float inv = rsqrtf(dx * dx + dy * dy + dz * dz);
    dx *= inv; dy *= inv; dz *= inv;
  } else {
    float sy, cy, sp, cp;
    sincosf(yaw + __ldg(p.col_off + c), &sy, &cy);
    sincosf(pitch + __ldg(p.row_off + r), &sp, &cp);
    dx = cp * cy;
    dy = cp * sy;
    dz = sp;
  }
  const float hit_eps = 0.6f * p.cell, min_step = 0.3f * p.cell;
  // Grid box in voxel units. A ray that has left it samples clamped
  // boundary-layer voxels only; the grid is padded by at least one free
  // layer, so every such voxel holds the same distance (one cell). From the
  // first outside sample on, d is frozen and the loop continues with the
  // same step arithmetic but no memory traffic: outputs are unchanged.
  const float gx = static_cast<float>(p.grid.nx), gy = static_cast<float>(p.grid.ny), gz = static_cast<float>(p.grid.nz);
  float t = 0.0f, d = 0.0f;
  bool outside = false;
  int k = 0;
  for (; k < p.max_steps; ++k) {
    if (!outside) {
      const float fx = (ex + dx * t - p.mnx) * p.inv_cell;
      const float fy = (ey + dy * t - p.mny) * p.inv_cell;
      const float fz = (ez + dz * t - p.mnz) * p.inv_cell;
      const bool inside = fx >= 0.0f && fx < gx && fy >= 0.0f && fy < gy && fz >= 0.0f && fz < gz;
      int ix, iy, iz;
      if (inside) {
        // 0 <= f < n: the clamp below would change nothing (int(f) <= n - 1)
        ix = static_cast<int>(fx);
        iy = static_cast<int>(fy);
        iz = static_cast<int>(fz);
      } else {
        ix = static_cast<int>(fminf(fmaxf(fx, 0.0f), gx - 1.0f));
        iy = static_cast<int>(fminf(fmaxf(fy, 0.0f), gy - 1.0f));
        iz = static_cast<int>(fminf(fmaxf(fz, 0.0f), gz - 1.0f));
      }
      // 32-bit brick addressing when the grid has < 2^31 voxels (the host checks)
      const int64_t vi = p.idx32 ? static_cast<int64_t>(
                                       ((static_cast<uint32_t>(iz >> 2) * p.grid.by + static_cast<uint32_t>(iy >> 2)) *
                                            p.grid.bx + static_cast<uint32_t>(ix >> 2)) << 6 |
                                       ((iz & 3) << 4) | ((iy & 3) << 2) | (ix & 3))
                                 : p.grid.index(ix, iy, iz);
      d = __half2float(__ldg(p.sdf + vi));
      outside = p.exit_outside && !inside;
    }
    if (!(d > hit_eps && t < p.range)) break;
    t += fmaxf(d * 0.9f, min_step);
  }
  t = fminf(t, p.range);
  const float enc = fminf(t, p.near_range) / p.near_range +
                    0.25f * (1.0f - expf(-fmaxf(t - p.near_range, 0.0f) / 2500.0f));
  constexpr int C = kSurfNz ? 2 : 1;
  int64_t pix;
  if (kLayout == kS2D4) pix = (static_cast<int64_t>(r >> 2) * (p.W >> 2) + (c >> 2)) * 16 + ((r & 3) << 2) + (c & 3);
  else pix = static_cast<int64_t>(r) * p.W + c;
  OutT* o = static_cast<OutT*>(p.out) + n * p.out_stride + pix * C;
  store<OutT>(o, enc);
  if (kSurfNz) {
    // the march stops inside the surface voxel (hit_eps < one cell): re-derive it
    const int ix = voxel(ex + dx * t, p.mnx, p.inv_cell, p.grid.nx);
    const int iy = voxel(ey + dy * t, p.mny, p.inv_cell, p.grid.ny);
    const int iz = voxel(ez + dz * t, p.mnz, p.inv_cell, p.grid.nz);
    store<OutT>(o + 1, static_cast<float>(__ldg(p.surf_nz + p.grid.index(ix, iy, iz))) * (1.0f / 127.0f));
  }
  if (p.steps) p.steps[(static_cast<int64_t>(n) * p.H + r) * p.W + c] = static_cast<uint8_t>(k > 255 ? 255 : k);
}

template <int kPinhole, typename OutT, int kLayout, bool kSurfNz>
int launch(const MarchParams& p, cudaStream_t s) {
  const int tiles = ((p.W + 15) >> 4) * ((p.H + 7) >> 3);
  const int64_t blocks = static_cast<int64_t>(tiles) * p.n_env;
  if (blocks == 0) return 0;
  march_kernel<kPinhole, OutT, kLayout, kSurfNz><<<static_cast<unsigned>(blocks), 128, 0, s>>>(p);
  SURF_RETURN_LAUNCH();
}

template <int kPinhole, typename OutT>
int dispatch_layout(const MarchParams& p, int layout, cudaStream_t s) {
  const bool nz = p.surf_nz != nullptr;
  if (layout == kS2D4) return nz ? launch<kPinhole, OutT, kS2D4, true>(p, s) : launch<kPinhole, OutT, kS2D4, false>(p, s);
  return nz ? launch<kPinhole, OutT, kNHW, true>(p, s) : launch<kPinhole, OutT, kNHW, false>(p, s);
}

// linear [nz][ny][nx] (float or half) -> bricked half
template <typename T>
__global__ void brick_kernel(const T* src, __half* dst, BrickGrid g) {
  const int64_t total = g.size();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t brick = i >> 6;
    const int w = static_cast<int>(i & 63);
    const int bxi = static_cast<int>(brick % g.bx);
    const int64_t rest = brick / g.bx;
    const int byi = static_cast<int>(rest % g.by);
    const int bzi = static_cast<int>(rest / g.by);
    const int ix = bxi * 4 + (w & 3), iy = byi * 4 + ((w >> 2) & 3), iz = bzi * 4 + (w >> 4);
    float v = 0.0f;
    if (ix < g.nx && iy < g.ny && iz < g.nz)
      v = static_cast<float>(src[(static_cast<int64_t>(iz) * g.ny + iy) * g.nx + ix]);
    dst[i] = __float2half_rn(v);
  }
}

}  // namespace

// Render depth for n_env poses. camera: 0 equiangular, 1 pinhole. out_dtype:
// 0 float32, 1 bfloat16. layout: 0 NHW, 1 space-to-depth 4x4 (H, W % 4 == 0).
// flags bit 0: the grid has >= 1 free boundary layer (enables the
// outside-the-grid shortcut, which leaves every output unchanged).
// env_order (optional, int32 [n_env], a permutation): the order the envs are
// rendered in; every env's output is the same in any order.
SURF_EXPORT int surf_march(const float* pose, int64_t pose_stride, int n_env, int H, int W, const void* sdf_bricked,
                           int nx, int ny, int nz, float mnx, float mny, float mnz, float cell, const float* col_off,
                           const float* row_off, float range, float near_range, int max_steps, int camera,
                           void* out, int64_t out_stride, int out_dtype, int layout, const int8_t* surf_nz,
                           uint8_t* steps, int flags, const int32_t* env_order, void* stream) {
  MarchParams p;
  p.pose = pose;
  p.pose_stride = pose_stride;
  p.n_env = n_env;
  p.H = H;
  p.W = W;
  p.sdf = static_cast<const __half*>(sdf_bricked);
  p.grid = surfk::make_brick_grid(nx, ny, nz);
  p.mnx = mnx; p.mny = mny; p.mnz = mnz;
  p.cell = cell;
  p.inv_cell = 1.0f / cell;
  p.col_off = col_off;
  p.row_off = row_off;
  p.range = range;
  p.near_range = near_range > 0 ? near_range : range;
  p.max_steps = max_steps;
  p.out = out;
  p.out_stride = out_stride;
  p.surf_nz = surf_nz;
  p.steps = steps;
  p.env_order = env_order;
  p.exit_outside = flags & 1;
  p.flags = flags;
  p.idx32 = p.grid.size() < (int64_t(1) << 31) && !(flags & 4);
  if (layout == kS2D4 && ((H & 3) || (W & 3))) return static_cast<int>(cudaErrorInvalidValue);
  auto s = static_cast<cudaStream_t>(stream);
  if (camera == 1) return out_dtype == 1 ? dispatch_layout<1, uint16_t>(p, layout, s) : dispatch_layout<1, float>(p, layout, s);
  return out_dtype == 1 ? dispatch_layout<0, uint16_t>(p, layout, s) : dispatch_layout<0, float>(p, layout, s);
}

SURF_EXPORT int64_t surf_brick_size(int nx, int ny, int nz) { return surfk::make_brick_grid(nx, ny, nz).size(); }

// src_dtype: 0 float32, 1 float16.
SURF_EXPORT int surf_brick_sdf(const void* src, int src_dtype, void* dst, int nx, int ny, int nz, void* stream) {
  BrickGrid g = surfk::make_brick_grid(nx, ny, nz);
  const int blocks = static_cast<int>(surfk::ceil_div(g.size(), 256) < 148 * 64 ? surfk::ceil_div(g.size(), 256) : 148 * 64);
  auto s = static_cast<cudaStream_t>(stream);
  if (src_dtype == 1) brick_kernel<__half><<<blocks, 256, 0, s>>>(static_cast<const __half*>(src), static_cast<__half*>(dst), g);
  else brick_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(src), static_cast<__half*>(dst), g);
  SURF_RETURN_LAUNCH();
}

// Same bricking for an int8 per-voxel grid (the |n_z| surfability channel).
__global__ void brick_i8_kernel(const int8_t* src, int8_t* dst, BrickGrid g) {
  const int64_t total = g.size();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t brick = i >> 6;
    const int w = static_cast<int>(i & 63);
    const int bxi = static_cast<int>(brick % g.bx);
    const int64_t rest = brick / g.bx;
    const int byi = static_cast<int>(rest % g.by);
    const int bzi = static_cast<int>(rest / g.by);
    const int ix = bxi * 4 + (w & 3), iy = byi * 4 + ((w >> 2) & 3), iz = bzi * 4 + (w >> 4);
    dst[i] = (ix < g.nx && iy < g.ny && iz < g.nz) ? src[(static_cast<int64_t>(iz) * g.ny + iy) * g.nx + ix] : 0;
  }
}

SURF_EXPORT int surf_brick_i8(const int8_t* src, int8_t* dst, int nx, int ny, int nz, void* stream) {
  BrickGrid g = surfk::make_brick_grid(nx, ny, nz);
  const int blocks = static_cast<int>(surfk::ceil_div(g.size(), 256) < 148 * 64 ? surfk::ceil_div(g.size(), 256) : 148 * 64);
  brick_i8_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(src, dst, g);
  SURF_RETURN_LAUNCH();
}
