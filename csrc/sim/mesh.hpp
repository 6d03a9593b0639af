// mesh.hpp — triangle mesh of a map's solid geometry (data export).
#pragma once
#include <cstdint>
#include <vector>

#include "map.hpp"

namespace surf {

// Boundary polygons of every solid leaf of `model`'s hull 0 (the convex cell
// cut out by the splitting planes on the leaf's path, clipped to the world
// bounds grown by `margin`), fan-triangulated with outward winding. Faces
// that lie on the artificial bounding box are dropped. Appends to verts
// (xyz) / tris (3 indices each).
void solid_mesh(const Map& map, int model, const float offset[3], float margin, std::vector<float>& verts,
                std::vector<int32_t>& tris);

}  // namespace surf
