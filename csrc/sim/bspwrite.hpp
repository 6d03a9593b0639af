// bspwrite.hpp — compile convex brushes into a BSP v30 collision file.
//
// The procedural map generator (Python) describes a map as convex brushes
// (intersections of half-spaces n.x <= d) grouped into brush models (model 0 =
// world, others = brush entities such as trigger volumes) plus an entity lump.
// This writer produces everything the GoldSrc collision code reads:
//   * PLANES (axial planes stored positive-facing, as the engine requires),
//   * hull 0 as render NODES + LEAFS (solid / empty / water leaves),
//   * hulls 1..3 as CLIPNODES, each brush expanded by the hull box with axial
//     bevel planes (the hlcsg rule), so a point query in hull h answers "does a
//     player box of that size at this origin overlap geometry",
//   * MODELS with per-hull head nodes and bounds, and ENTITIES.
// Tree construction: axis-aligned splits at brush bounds (chosen to duplicate
// the fewest brushes) until few brushes remain, then each brush becomes a
// chain of its planes whose outside branches share the subtree of the
// remaining brushes; identical nodes are merged. The result is a DAG, which
// the engine's child-index walk handles like a tree. The format caps node
// indices at 32767 (int16 children), which bounds the brush count per map.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

#include "bspfile.hpp"

namespace surf {

struct BrushPlane { float n[3]; float d; };   // solid where n.x <= d
struct Brush {
  int model = 0;
  int contents = kSolid;                      // kSolid or a liquid contents code
  std::vector<BrushPlane> planes;
};

class BspWriter {
 public:
  void add_brush(const Brush& b) { brushes_.push_back(b); }
  void set_entities(const std::string& text) { entities_ = text; }
  // Also compile hull 2 (the 64u monster box). Players use hulls 0, 1 and 3,
  // so by default hull 2 is written as an empty tree to save clipnodes.
  void set_large_hull(bool on) { large_hull_ = on; }
  // Build the file image. Returns false (and *err) if a BSP limit is exceeded.
  bool build(std::vector<uint8_t>* out, std::string* err);

 private:
  std::vector<Brush> brushes_;
  std::string entities_;
  bool large_hull_ = false;
};

}  // namespace surf
