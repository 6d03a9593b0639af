// map.hpp — a loaded collision map: planes, hull trees for every brush model,
// and the entities the movement simulation reacts to.
//
// Behaviour parity with the reference loader (src/bsp.c:168-336): hull 0 is
// rebuilt from the render NODES/LEAFS (Mod_MakeHull0), hulls 1-3 come from
// CLIPNODES, and the entity lump is parsed for spawns, trigger_teleport /
// trigger_hurt / trigger_push, solid brush entities and contents volumes.
#pragma once
#include <climits>
#include <cstdint>
#include <string>
#include <vector>

#include "bspfile.hpp"

namespace surf {

// Start-node grid of one clip tree (an acceleration structure of this build;
// the engine always descends from the root): a uniform grid of power-of-two
// cells over the tree's bounds, in the tree's coordinates. A cell holds the
// deepest node that the descent reaches, with the same plane-side decisions,
// from EVERY point of the cell (or the leaf contents it reaches). A point
// query takes exactly that root-to-node path, so it may start there. So may
// a segment whose endpoints lie in one cell (the cell is convex), or in two
// cells holding the same internal node that has a single path from the root
// (kShared marks nodes with several parents -- a compiler may share
// subtrees -- and leaf contents are not unique either). Either way the
// result is bit-identical to a descent from the root. Axial planes decide
// a cell exactly (cell bounds are floats and p - d keeps the sign of p - d);
// sloped planes only when every corner clears the plane by a margin far
// above the float error of dot(p, n) - d.
struct HullGrid {
  static constexpr int32_t kNone = INT32_MIN;
  static constexpr int32_t kShared = 1 << 30;   // flag on a cell's node: reachable along several paths
  const int32_t* cells = nullptr;   // null: no grid (descents start at the root)
  float mn[3] = {0, 0, 0};          // grid origin: a multiple of the cell size
  float size = 0, inv = 0;          // cell size (a power of two) and its inverse
  int32_t n[3] = {0, 0, 0};

  // The node of the cell containing p, or kNone (no grid, p outside it, or p
  // on the far side of a rounding boundary of the index estimate); *cell
  // receives the cell's index.
  SURF_HD int32_t lookup(const float p[3], int64_t* cell = nullptr) const {
    if (!cells) return kNone;
    int32_t idx[3];
    for (int k = 0; k < 3; ++k) {
      const float f = (p[k] - mn[k]) * inv;
      if (!(f >= 0.f) || f >= static_cast<float>(n[k])) return kNone;
      const int32_t i = static_cast<int32_t>(f);
      const float lo = mn[k] + static_cast<float>(i) * size;    // exact: integer multiples of a power of two
      if (p[k] < lo || p[k] >= lo + size) return kNone;
      idx[k] = i;
    }
    const int64_t c = (static_cast<int64_t>(idx[2]) * n[1] + idx[1]) * n[0] + idx[0];
    if (cell) *cell = c;
    return cells[c];
  }

  SURF_HD static int32_t node_of(int32_t v) { return v >= 0 ? (v & ~kShared) : v; }

  // Where a point query at p may start (kNone: at the root).
  SURF_HD int32_t point_start(const float p[3]) const {
    const int32_t v = lookup(p);
    return v == kNone ? kNone : node_of(v);
  }

  // Where a descent of the segment a -> b may start: the node of their one
  // cell, or the single-path internal node both cells hold; else kNone.
  SURF_HD int32_t segment_start(const float a[3], const float b[3]) const {
    int64_t ca = -1, cb = -2;
    const int32_t va = lookup(a, &ca);
    if (va == kNone) return kNone;
    const int32_t vb = lookup(b, &cb);
    if (vb != va) return kNone;
    if (va >= 0 && !(va & kShared)) return va;
    return ca == cb ? node_of(va) : kNone;
  }
};

// One BSP clip tree view: nodes + planes + the box the tree was expanded by.
struct HullView {
  const Clipnode* nodes = nullptr;
  const Plane* planes = nullptr;
  int first = 0, last = 0;          // root node index, last valid node index
  float clip_mins[3] = {0, 0, 0};
  float clip_maxs[3] = {0, 0, 0};
  HullGrid grid;                    // start-node grid (the world model only)
};

enum class TriggerKind : int32_t { kTeleport = 0, kHurt = 1, kPush = 2 };

struct Trigger {
  TriggerKind kind = TriggerKind::kTeleport;
  int32_t model = 0;
  float origin[3] = {0, 0, 0};
  float absmin[3] = {0, 0, 0}, absmax[3] = {0, 0, 0};  // model bounds + origin, padded by 1
  bool has_dest = false;             // teleport: target resolved to a point entity
  float dest[3] = {0, 0, 0};
  float dest_yaw = 0;
  float damage = 10;                 // hurt
  float push_velocity[3] = {0, 0, 0};  // push: movedir * speed
  bool push_once = false;
};

struct BrushEntity {                 // solid brush entity or contents volume
  int32_t model = 0;
  float origin[3] = {0, 0, 0};
  int32_t contents = kSolid;         // contents volumes: skin value (or kLadder)
  float absmin[3] = {0, 0, 0}, absmax[3] = {0, 0, 0};
};

struct SpawnPoint { float origin[3]; float yaw; };

// Plain-pointer view of a loaded map: what the per-player simulation code
// reads (traces, contents, triggers). The host builds it over Map's vectors;
// the GPU env builds the same struct over device copies of those arrays.
struct MapView {
  Span<Plane> planes;
  Span<Clipnode> clipnodes;           // hulls 1..3 of every model
  Span<Clipnode> hull0;               // render nodes mirrored into clipnode form
  Span<Model> models;
  Span<BrushEntity> solids;
  Span<BrushEntity> volumes;
  Span<Trigger> triggers;
  Span<SpawnPoint> spawns;
  float world_mins[3] = {0, 0, 0}, world_maxs[3] = {0, 0, 0};
  HullGrid world_grid[4];             // start-node grids of the world model's hulls
  // false when no point of the map can have liquid contents (no hull-0 leaf
  // and no contents volume is water, slime, lava, sky or a current): the
  // movement's water checks then skip their point-contents probes, whose
  // result could not change anything
  bool any_liquid = true;

  SURF_HD HullView hull(int model, int bsp_hull) const {
    HullView v;
    v.planes = planes.data();
    const Model& m = models[model];
    if (bsp_hull == 0) {
      v.nodes = hull0.data();
      v.last = hull0.size() - 1;
    } else {
      v.nodes = clipnodes.data();
      v.last = clipnodes.size() - 1;
    }
    v.first = m.headnode[bsp_hull];
    for (int k = 0; k < 3; ++k) { v.clip_mins[k] = hull_mins(bsp_hull, k); v.clip_maxs[k] = hull_maxs(bsp_hull, k); }
    if (model == 0) v.grid = world_grid[bsp_hull];
    return v;
  }
};

class Map {
 public:
  // Parse a BSP v30 image. Returns false and fills *err on malformed input.
  bool load_memory(const uint8_t* data, size_t size, std::string* err);
  bool load_file(const std::string& path, std::string* err);

  HullView hull(int model, int bsp_hull) const { return view().hull(model, bsp_hull); }
  // Views over the vectors below (valid while the map is alive; a loaded map
  // never changes).
  MapView view() const;

  std::vector<DPlane> planes;
  std::vector<DClipnode> clipnodes;   // hulls 1..3 of every model
  std::vector<DClipnode> hull0;       // render nodes mirrored into clipnode form
  std::vector<DModel> models;
  std::string entities;

  std::vector<BrushEntity> solids;    // collide like world geometry
  std::vector<BrushEntity> volumes;   // water / ladder / other contents volumes
  std::vector<Trigger> triggers;
  std::vector<SpawnPoint> spawns;

  float world_mins[3] = {0, 0, 0}, world_maxs[3] = {0, 0, 0};
  bool any_liquid = true;             // see MapView::any_liquid

  // Start-node grids of the world model's hulls 0 (point), 1 (standing) and
  // 3 (crouched), built at load; at most kGridCells cells each.
  static constexpr int64_t kGridCells = int64_t(1) << 21;
  std::vector<int32_t> grid_cells[4];
  HullGrid grid_meta[4];

 private:
  bool parse_entities();
  void build_grids();
  void find_liquids();
};

}  // namespace surf
