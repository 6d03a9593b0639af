// geodesic.cpp — host multi-source shortest path over the free voxels of an
// occupancy grid (26-connected; edge cost cell, cell*sqrt2, cell*sqrt3), the
// CPU path of the race goal field.
//
// The reference relaxes the whole grid Bellman-Ford style on the GPU
// (python/surfgym/goalfield.py:158-260); the GPU path of this framework does
// the same (csrc/kernels/geodesic.cu). On the host, a wavefront sweep costs
// one full-grid pass per voxel of path length, so this is Dijkstra's
// algorithm on an indexed 4-ary heap instead: every free voxel is settled
// once. Distances are float32 sums in path order, d[v] = d[u] + w, so the
// result is the same fixed point the relaxation reaches (a neighbour settled
// later cannot improve a settled voxel: weights are positive and float
// rounding is monotone).
#include <cmath>
#include <cstdint>
#include <vector>

#define SURFSIM_API extern "C" __attribute__((visibility("default")))

namespace {

constexpr float kInf = 3.0e38f;
constexpr uint32_t kNone = 0xFFFFFFFFu;

struct Entry { float d; uint32_t v; };

// 4-ary min-heap of (distance, voxel) with a voxel -> slot index for
// decrease-key; keys live in the entries so sifting stays in one array.
struct Heap4 {
  std::vector<Entry> items;
  std::vector<uint32_t> pos;     // voxel -> heap slot (kNone: not queued)

  void place(size_t i, const Entry& e) {
    items[i] = e;
    pos[e.v] = static_cast<uint32_t>(i);
  }
  void up(size_t i, Entry e) {
    while (i > 0) {
      const size_t p = (i - 1) >> 2;
      if (!(e.d < items[p].d)) break;
      place(i, items[p]);
      i = p;
    }
    place(i, e);
  }
  void down(size_t i, Entry e) {
    const size_t n = items.size();
    for (;;) {
      const size_t c0 = 4 * i + 1;
      if (c0 >= n) break;
      size_t best = c0;
      float bd = items[c0].d;
      const size_t cend = c0 + 4 < n ? c0 + 4 : n;
      for (size_t c = c0 + 1; c < cend; ++c)
        if (items[c].d < bd) { bd = items[c].d; best = c; }
      if (!(bd < e.d)) break;
      place(i, items[best]);
      i = best;
    }
    place(i, e);
  }
  void push_or_decrease(uint32_t v, float d) {
    if (pos[v] == kNone) {
      items.push_back(Entry{d, v});
      up(items.size() - 1, Entry{d, v});
    } else {
      up(pos[v], Entry{d, v});
    }
  }
  Entry pop() {
    const Entry top = items[0];
    pos[top.v] = kNone;
    const Entry last = items.back();
    items.pop_back();
    if (!items.empty()) down(0, last);
    return top;
  }
};

}  // namespace

// occ: uint8 [nz][ny][nx] (non-zero = solid); lo3/hi3: inclusive seed box
// (x, y, z voxel indices, clipped to the grid). out: float32 [nz][ny][nx],
// 3e38 on solid and unreachable voxels. Returns the number of reached voxels,
// or -1 for a grid too large for 32-bit voxel indices.
SURFSIM_API int64_t surfsim_geodesic(const uint8_t* occ, int32_t nx, int32_t ny, int32_t nz, float cell,
                                     const int32_t* lo3, const int32_t* hi3, float* out) {
  const int64_t n = static_cast<int64_t>(nx) * ny * nz;
  if (nx < 1 || ny < 1 || nz < 1 || n >= static_cast<int64_t>(kNone)) return -1;
  for (int64_t i = 0; i < n; ++i) out[i] = kInf;
  const float w[4] = {0.0f, cell, cell * 1.41421356f, cell * 1.73205081f};
  Heap4 h;
  h.pos.assign(static_cast<size_t>(n), kNone);
  const int32_t dim[3] = {nx, ny, nz};
  int32_t lo[3], hi[3];
  for (int a = 0; a < 3; ++a) {
    lo[a] = lo3[a] < 0 ? 0 : lo3[a];
    hi[a] = hi3[a] >= dim[a] ? dim[a] - 1 : hi3[a];
  }
  for (int32_t z = lo[2]; z <= hi[2]; ++z)
    for (int32_t y = lo[1]; y <= hi[1]; ++y)
      for (int32_t x = lo[0]; x <= hi[0]; ++x) {
        const uint32_t v = static_cast<uint32_t>((static_cast<int64_t>(z) * ny + y) * nx + x);
        if (occ[v]) continue;
        out[v] = 0.0f;
        h.push_or_decrease(v, 0.0f);
      }
  std::vector<uint8_t> done(static_cast<size_t>(n), 0);
  int64_t reached = 0;
  const int64_t plane = static_cast<int64_t>(nx) * ny;
  while (!h.items.empty()) {
    const Entry e = h.pop();
    const uint32_t u = e.v;
    done[u] = 1;
    ++reached;
    const float du = e.d;
    const int32_t x = static_cast<int32_t>(u % nx), y = static_cast<int32_t>((u / nx) % ny);
    const int32_t z = static_cast<int32_t>(u / plane);
    for (int dz = -1; dz <= 1; ++dz) {
      const int32_t zz = z + dz;
      if (zz < 0 || zz >= nz) continue;
      for (int dy = -1; dy <= 1; ++dy) {
        const int32_t yy = y + dy;
        if (yy < 0 || yy >= ny) continue;
        for (int dx = -1; dx <= 1; ++dx) {
          const int32_t xx = x + dx;
          if (xx < 0 || xx >= nx) continue;
          const int m = (dz != 0) + (dy != 0) + (dx != 0);
          if (m == 0) continue;
          const uint32_t v = static_cast<uint32_t>((static_cast<int64_t>(zz) * ny + yy) * nx + xx);
          if (occ[v] || done[v]) continue;
          const float nd = du + w[m];
          if (nd < out[v]) {
            out[v] = nd;
            h.push_or_decrease(v, nd);
          }
        }
      }
    }
  }
  return reached;
}
