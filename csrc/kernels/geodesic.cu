// geodesic.cu — multi-source shortest paths over free voxels (sm_100a).
//
// The race reward shapes on the geodesic distance from every free voxel to
// the finish zone along the 26-connected voxel graph (edge cost = centre
// distance: cell * {1, sqrt 2, sqrt 3}); solid voxels never relax.
// Reference: python/surfgym/goalfield.py:221-298, which runs Bellman-Ford as
// 26 shifted full-grid tensor ops per sweep (up to 8000 sweeps).
//
// Here the grid is cut into 8x8x8 tiles. A pass runs a persistent grid over a
// compacted worklist of ACTIVE tiles: each tile plus a one-voxel halo is
// staged in shared memory and relaxed to local convergence (a wavefront
// crosses the whole tile inside one pass); a tile that changed marks itself,
// and a dilation step appends it and its 26 neighbours to the next worklist.
// Passes repeat until no tile changes, so the work follows the wavefront
// instead of re-sweeping the whole volume.
#include <cstdint>

#include "surf_cuda.cuh"

namespace {

constexpr int T = 8;               // tile edge
constexpr int H = T + 2;           // with halo
constexpr float kInf = 3.0e38f;

struct Grid { int nx, ny, nz, tx, ty, tz; float w1, w2, w3; };

__device__ void relax_tile(float* dist, const uint8_t* solid, uint8_t* changed, const Grid& g, int* any_changed,
                           int64_t tile) {
  const int tx = static_cast<int>(tile % g.tx), ty = static_cast<int>((tile / g.tx) % g.ty),
            tz = static_cast<int>(tile / (static_cast<int64_t>(g.tx) * g.ty));
  __shared__ float d[H][H][H];
  __shared__ uint8_t sol[H][H][H];
  // stage tile + halo
  for (int i = threadIdx.x; i < H * H * H; i += blockDim.x) {
    const int lx = i % H, ly = (i / H) % H, lz = i / (H * H);
    const int gx = tx * T + lx - 1, gy = ty * T + ly - 1, gz = tz * T + lz - 1;
    float v = kInf;
    uint8_t s = 1;
    if (gx >= 0 && gy >= 0 && gz >= 0 && gx < g.nx && gy < g.ny && gz < g.nz) {
      const int64_t k = (static_cast<int64_t>(gz) * g.ny + gy) * g.nx + gx;
      v = dist[k];
      s = solid[k];
    }
    d[lz][ly][lx] = v;
    sol[lz][ly][lx] = s;
  }
  __syncthreads();
  const int lx = threadIdx.x % T + 1, ly = (threadIdx.x / T) % T + 1, lz = threadIdx.x / (T * T) + 1;
  const int gx = tx * T + lx - 1, gy = ty * T + ly - 1, gz = tz * T + lz - 1;
  const bool inside = gx < g.nx && gy < g.ny && gz < g.nz;
  const bool free_v = inside && !sol[lz][ly][lx];
  bool mine = false;
  for (int it = 0; it < 3 * T; ++it) {
    float best = d[lz][ly][lx];
    if (free_v) {
      for (int oz = -1; oz <= 1; ++oz)
        for (int oy = -1; oy <= 1; ++oy)
          for (int ox = -1; ox <= 1; ++ox) {
            const int m = (ox != 0) + (oy != 0) + (oz != 0);
            if (m == 0) continue;
            const float w = m == 1 ? g.w1 : (m == 2 ? g.w2 : g.w3);
            best = fminf(best, d[lz + oz][ly + oy][lx + ox] + w);
          }
    }
    __syncthreads();
    const bool upd = free_v && best < d[lz][ly][lx];
    if (upd) { d[lz][ly][lx] = best; mine = true; }
    if (!__syncthreads_or(upd)) break;
  }
  if (inside && mine) dist[(static_cast<int64_t>(gz) * g.ny + gy) * g.nx + gx] = d[lz][ly][lx];
  if (__syncthreads_or(mine) && threadIdx.x == 0) {
    changed[tile] = 1;
    atomicOr(any_changed, 1);
  }
  __syncthreads();          // shared tile is reused by the next worklist entry
}

__global__ void __launch_bounds__(512) relax_kernel(float* dist, const uint8_t* solid, const int64_t* work,
                                                    const int* count, uint8_t* changed, Grid g, int* any_changed) {
  const int n = *count;
  for (int w = blockIdx.x; w < n; w += gridDim.x) relax_tile(dist, solid, changed, g, any_changed, work[w]);
}

// next worklist = changed tiles and their 26 neighbours (from `changed`, or
// from `seedflags` when non-null)
__global__ void dilate_kernel(const uint8_t* changed, int64_t* work, int* count, Grid g, int self_only) {
  const int64_t n = static_cast<int64_t>(g.tx) * g.ty * g.tz;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < n;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int tx = static_cast<int>(t % g.tx), ty = static_cast<int>((t / g.tx) % g.ty),
              tz = static_cast<int>(t / (static_cast<int64_t>(g.tx) * g.ty));
    uint8_t a = self_only ? changed[t] : 0;
    for (int oz = -1; oz <= 1 && !a && !self_only; ++oz)
      for (int oy = -1; oy <= 1 && !a; ++oy)
        for (int ox = -1; ox <= 1 && !a; ++ox) {
          const int x = tx + ox, y = ty + oy, z = tz + oz;
          if (x < 0 || y < 0 || z < 0 || x >= g.tx || y >= g.ty || z >= g.tz) continue;
          a = changed[(static_cast<int64_t>(z) * g.ty + y) * g.tx + x];
        }
    if (a) work[atomicAdd(count, 1)] = t;
  }
}

__global__ void clear_kernel(uint8_t* p, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    p[i] = 0;
}

// seeds: free voxels in [lo, hi] get 0; every other voxel +inf; tiles holding a seed start active
__global__ void seed_kernel(float* dist, const uint8_t* solid, uint8_t* seeded_tiles, Grid g, int x0, int y0, int z0, int x1,
                            int y1, int z1, int* n_seed) {
  const int64_t n = static_cast<int64_t>(g.nx) * g.ny * g.nz;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int x = static_cast<int>(i % g.nx), y = static_cast<int>((i / g.nx) % g.ny),
              z = static_cast<int>(i / (static_cast<int64_t>(g.nx) * g.ny));
    const bool seed = !solid[i] && x >= x0 && x <= x1 && y >= y0 && y <= y1 && z >= z0 && z <= z1;
    dist[i] = seed ? 0.0f : kInf;
    if (seed) {
      seeded_tiles[(static_cast<int64_t>(z / T) * g.ty + y / T) * g.tx + x / T] = 1;
      atomicAdd(n_seed, 1);
    }
  }
}

// uint16 quantisation with a sentinel for solid / unreachable voxels
__global__ void quantize_kernel(const float* dist, int64_t n, float quant, float sentinel, uint16_t* out) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float v = dist[i];
    if (!(v < 1e30f)) v = sentinel;
    out[i] = static_cast<uint16_t>(fminf(rintf(v / quant), 65535.0f));
  }
}

__global__ void max_finite_kernel(const float* dist, int64_t n, unsigned int* out_bits) {
  float m = 0.0f;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float v = dist[i];
    if (v < 1e30f) m = fmaxf(m, v);
  }
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out_bits, __float_as_uint(m));    // non-negative floats order as uints
}

Grid make_grid(int nx, int ny, int nz, float cell) {
  return Grid{nx, ny, nz, (nx + T - 1) / T, (ny + T - 1) / T, (nz + T - 1) / T, cell, cell * 1.41421356f,
              cell * 1.73205081f};
}

int blocks_for(int64_t n) {
  const int64_t b = surfk::ceil_div(n, 256);
  return static_cast<int>(b < 1 ? 1 : (b > 148 * 32 ? 148 * 32 : b));
}

}  // namespace

SURF_EXPORT int64_t surf_geodesic_tiles(int nx, int ny, int nz) {
  Grid g = make_grid(nx, ny, nz, 1.0f);
  return static_cast<int64_t>(g.tx) * g.ty * g.tz;
}

// Workspace: flags (tiles bytes), two worklists (2 x tiles int64) and two
// counters (int[2]), all caller-allocated. Initialise: dist (float
// [nz,ny,nx]) = 0 on free voxels of the seed box (voxel indices,
// inclusive), +inf elsewhere; worklist 0 = the seeded tiles. *n_seed counts
// the seeded voxels (zeroed by the caller).
SURF_EXPORT int surf_geodesic_init(float* dist, const uint8_t* solid, uint8_t* flags, int64_t* work, int* counts,
                                   int nx, int ny, int nz, float cell, int x0, int y0, int z0, int x1, int y1, int z1,
                                   int* n_seed, void* stream) {
  Grid g = make_grid(nx, ny, nz, cell);
  const int64_t tiles = static_cast<int64_t>(g.tx) * g.ty * g.tz;
  auto s = static_cast<cudaStream_t>(stream);
  clear_kernel<<<blocks_for(tiles), 256, 0, s>>>(flags, tiles);
  cudaMemsetAsync(counts, 0, 2 * sizeof(int), s);
  seed_kernel<<<blocks_for(static_cast<int64_t>(nx) * ny * nz), 256, 0, s>>>(dist, solid, flags, g, x0, y0, z0, x1, y1,
                                                                            z1, n_seed);
  dilate_kernel<<<blocks_for(tiles), 256, 0, s>>>(flags, work, counts, g, 1);
  SURF_RETURN_LAUNCH();
}

// One pass: relax the tiles of worklist `cur` (0/1), then build worklist
// 1-cur from the tiles that changed and their neighbours. *any_changed is
// set when some tile improved (the caller zeroes it).
SURF_EXPORT int surf_geodesic_pass(float* dist, const uint8_t* solid, uint8_t* flags, int64_t* work, int* counts,
                                   int cur, int nx, int ny, int nz, float cell, int* any_changed, void* stream) {
  Grid g = make_grid(nx, ny, nz, cell);
  const int64_t tiles = static_cast<int64_t>(g.tx) * g.ty * g.tz;
  auto s = static_cast<cudaStream_t>(stream);
  int64_t* w_cur = work + cur * tiles;
  int64_t* w_next = work + (1 - cur) * tiles;
  clear_kernel<<<blocks_for(tiles), 256, 0, s>>>(flags, tiles);
  relax_kernel<<<148 * 4, 512, 0, s>>>(dist, solid, w_cur, counts + cur, flags, g, any_changed);
  cudaMemsetAsync(counts + (1 - cur), 0, sizeof(int), s);
  dilate_kernel<<<blocks_for(tiles), 256, 0, s>>>(flags, w_next, counts + (1 - cur), g, 0);
  SURF_RETURN_LAUNCH();
}

// Largest finite distance (as float bits in *out, zeroed by the caller) and
// the uint16 quantisation.
SURF_EXPORT int surf_geodesic_finish(const float* dist, int nx, int ny, int nz, unsigned int* max_bits, float quant,
                                     float sentinel, uint16_t* out, void* stream) {
  const int64_t n = static_cast<int64_t>(nx) * ny * nz;
  auto s = static_cast<cudaStream_t>(stream);
  if (max_bits) max_finite_kernel<<<blocks_for(n), 256, 0, s>>>(dist, n, max_bits);
  if (out) quantize_kernel<<<blocks_for(n), 256, 0, s>>>(dist, n, quant, sentinel, out);
  SURF_RETURN_LAUNCH();
}
