// bspfile.hpp — on-disk layout of GoldSrc BSP version 30 (the lumps this
// framework reads and writes).
//
// The byte layout is fixed by the file format, so these structs are packed and
// their sizes are asserted. Only the collision-relevant lumps are modelled:
// ENTITIES (0), PLANES (1), NODES (5), CLIPNODES (9), LEAFS (10), MODELS (14).
// Reference parity: src/sim.h:33-58 (reference reads the same lumps).
#pragma once
#include <cstdint>

#include "hd.hpp"

namespace surf {

constexpr int32_t kBspVersion = 30;
constexpr int kNumLumps = 15;
enum LumpId : int {
  kLumpEntities = 0, kLumpPlanes = 1, kLumpTextures = 2, kLumpVertexes = 3,
  kLumpVisibility = 4, kLumpNodes = 5, kLumpTexinfo = 6, kLumpFaces = 7,
  kLumpLighting = 8, kLumpClipnodes = 9, kLumpLeafs = 10, kLumpMarksurfaces = 11,
  kLumpEdges = 12, kLumpSurfedges = 13, kLumpModels = 14,
};

// GoldSrc contents codes (negative leaf/clipnode children).
enum Contents : int {
  kEmpty = -1, kSolid = -2, kWater = -3, kSlime = -4, kLava = -5, kSky = -6,
  kCurrent0 = -9, kCurrentDown = -14, kTranslucent = -15, kLadder = -16,
};

// pm_shared's liquid test (water, slime, lava, sky and the contents between
// them): the contents for which CheckWater raises the water level
SURF_HD inline bool contents_liquid(int c) { return c <= kWater && c > kTranslucent; }

#pragma pack(push, 1)
struct DLump { int32_t offset, length; };
struct DHeader { int32_t version; DLump lumps[kNumLumps]; };
struct DPlane { float normal[3]; float dist; int32_t type; };  // type 0..2 axial, 3..5 nearest axis
struct DClipnode { int32_t plane; int16_t child[2]; };          // child < 0 -> contents
struct DNode {
  int32_t plane; int16_t child[2];                               // child < 0 -> -(leaf+1)
  int16_t mins[3], maxs[3]; uint16_t first_face, num_faces;
};
struct DLeaf {
  int32_t contents, vis_offset; int16_t mins[3], maxs[3];
  uint16_t first_mark, num_marks; uint8_t ambient[4];
};
struct DModel {
  float mins[3], maxs[3], origin[3];
  int32_t headnode[4]; int32_t visleafs, first_face, num_faces;
};
#pragma pack(pop)

// Naturally aligned mirrors of the packed records with identical layouts
// (every field is a 4- or 2-byte value at an aligned offset): the types the
// simulation code reads through MapView / HullView, so device code loads
// whole words instead of single bytes.
struct alignas(4) Plane { float normal[3]; float dist; int32_t type; };
struct alignas(4) Clipnode { int32_t plane; int16_t child[2]; };
struct alignas(4) Model {
  float mins[3], maxs[3], origin[3];
  int32_t headnode[4]; int32_t visleafs, first_face, num_faces;
};

static_assert(sizeof(DHeader) == 124, "BSP header");
static_assert(sizeof(DPlane) == 20, "BSP plane");
static_assert(sizeof(DClipnode) == 8, "BSP clipnode");
static_assert(sizeof(DNode) == 24, "BSP node");
static_assert(sizeof(DLeaf) == 28, "BSP leaf");
static_assert(sizeof(DModel) == 64, "BSP model");
static_assert(sizeof(Plane) == sizeof(DPlane) && sizeof(Clipnode) == sizeof(DClipnode) &&
                  sizeof(Model) == sizeof(DModel), "aligned mirrors keep the packed layouts");

// Player hull boxes by pmove "usehull" (0 stand, 1 duck, 2 point, 3 large).
// GoldSrc engine constants (pm_shared player_mins/maxs).
extern const float kPlayerMins[4][3];
extern const float kPlayerMaxs[4][3];
// Clip-hull boxes by BSP hull index (0 point, 1 human, 2 large, 3 crouch).
extern const float kHullMins[4][3];
extern const float kHullMaxs[4][3];
// pmove usehull -> BSP hull index.
SURF_HD inline int bsp_hull_of_usehull(int usehull) {
  return usehull == 1 ? 3 : usehull == 2 ? 0 : usehull == 3 ? 2 : 1;
}

}  // namespace surf
