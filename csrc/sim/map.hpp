// map.hpp — a loaded collision map: planes, hull trees for every brush model,
// and the entities the movement simulation reacts to.
//
// Behaviour parity with the reference loader (src/bsp.c:168-336): hull 0 is
// rebuilt from the render NODES/LEAFS (Mod_MakeHull0), hulls 1-3 come from
// CLIPNODES, and the entity lump is parsed for spawns, trigger_teleport /
// trigger_hurt / trigger_push, solid brush entities and contents volumes.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

#include "bspfile.hpp"

namespace surf {

// One BSP clip tree view: nodes + planes + the box the tree was expanded by.
struct HullView {
  const Clipnode* nodes = nullptr;
  const Plane* planes = nullptr;
  int first = 0, last = 0;          // root node index, last valid node index
  float clip_mins[3] = {0, 0, 0};
  float clip_maxs[3] = {0, 0, 0};
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

 private:
  bool parse_entities();
};

}  // namespace surf
