// mesh.cpp — solid-leaf polyhedra of a hull-0 tree as a triangle mesh.
//
// The reference exports the render faces of a BSP (tools/export_map.py);
// maps written by this framework's BSP writer carry collision hulls only, so
// the mesh is rebuilt from the tree itself: each solid leaf is the
// intersection of the half-spaces chosen on its path from the root; every
// bounding plane of that cell yields a face polygon (a large quad on the
// plane clipped by all the other half-spaces, Sutherland-Hodgman).
#include "mesh.hpp"

#include <array>
#include <cmath>

namespace surf {
namespace {

struct Half { double n[3]; double d; bool box; };   // n . x <= d
using Poly = std::vector<std::array<double, 3>>;

double dot3(const double* a, const double* b) { return a[0] * b[0] + a[1] * b[1] + a[2] * b[2]; }

Poly clip(const Poly& in, const Half& h) {
  Poly out;
  const size_t n = in.size();
  for (size_t i = 0; i < n; ++i) {
    const auto& a = in[i];
    const auto& b = in[(i + 1) % n];
    const double da = dot3(h.n, a.data()) - h.d, db = dot3(h.n, b.data()) - h.d;
    const bool ia = da <= 1e-6, ib = db <= 1e-6;
    if (ia) out.push_back(a);
    if (ia != ib) {
      const double t = da / (da - db);
      out.push_back({a[0] + t * (b[0] - a[0]), a[1] + t * (b[1] - a[1]), a[2] + t * (b[2] - a[2])});
    }
  }
  return out;
}

void emit_cell(const std::vector<Half>& hs, std::vector<float>& verts, std::vector<int32_t>& tris) {
  constexpr double R = 1 << 18;
  for (size_t i = 0; i < hs.size(); ++i) {
    const Half& f = hs[i];
    if (f.box) continue;
    // basis on the plane: u perpendicular to the normal, v = n x u (u x v = n)
    const double* n = f.n;
    const int ax = std::fabs(n[0]) < std::fabs(n[1]) ? (std::fabs(n[0]) < std::fabs(n[2]) ? 0 : 2)
                                                     : (std::fabs(n[1]) < std::fabs(n[2]) ? 1 : 2);
    double a[3] = {0, 0, 0};
    a[ax] = 1.0;
    double u[3] = {n[1] * a[2] - n[2] * a[1], n[2] * a[0] - n[0] * a[2], n[0] * a[1] - n[1] * a[0]};
    const double ul = std::sqrt(dot3(u, u));
    for (double& c : u) c /= ul;
    const double v[3] = {n[1] * u[2] - n[2] * u[1], n[2] * u[0] - n[0] * u[2], n[0] * u[1] - n[1] * u[0]};
    const double c[3] = {n[0] * f.d, n[1] * f.d, n[2] * f.d};
    Poly p;
    const double su[4] = {-1, 1, 1, -1}, sv[4] = {-1, -1, 1, 1};
    for (int k = 0; k < 4; ++k)
      p.push_back({c[0] + R * (su[k] * u[0] + sv[k] * v[0]), c[1] + R * (su[k] * u[1] + sv[k] * v[1]),
                   c[2] + R * (su[k] * u[2] + sv[k] * v[2])});
    for (size_t j = 0; j < hs.size() && p.size() >= 3; ++j)
      if (j != i) p = clip(p, hs[j]);
    if (p.size() < 3) continue;
    const int32_t base = static_cast<int32_t>(verts.size() / 3);
    for (const auto& q : p)
      for (int k = 0; k < 3; ++k) verts.push_back(static_cast<float>(q[k]));
    for (size_t k = 1; k + 1 < p.size(); ++k) {
      tris.push_back(base);
      tris.push_back(base + static_cast<int32_t>(k));
      tris.push_back(base + static_cast<int32_t>(k + 1));
    }
  }
}

}  // namespace

static void walk(const Map& map, const HullView& hv, int node, const float offset[3], std::vector<Half>& path,
          std::vector<float>& verts, std::vector<int32_t>& tris) {
  if (node < 0) {
    if (node == kSolid) emit_cell(path, verts, tris);
    return;
  }
  const Clipnode& cn = hv.nodes[node];
  const DPlane& pl = map.planes[static_cast<size_t>(cn.plane)];
  const double d = static_cast<double>(pl.dist) + pl.normal[0] * static_cast<double>(offset[0]) +
                   pl.normal[1] * static_cast<double>(offset[1]) + pl.normal[2] * static_cast<double>(offset[2]);
  path.push_back(Half{{-pl.normal[0], -pl.normal[1], -pl.normal[2]}, -d, false});   // front: n.x >= d
  walk(map, hv, cn.child[0], offset, path, verts, tris);
  path.back() = Half{{pl.normal[0], pl.normal[1], pl.normal[2]}, d, false};         // back: n.x < d
  walk(map, hv, cn.child[1], offset, path, verts, tris);
  path.pop_back();
}

void solid_mesh(const Map& map, int model, const float offset[3], float margin, std::vector<float>& verts,
                std::vector<int32_t>& tris) {
  const HullView hv = map.hull(model, 0);
  const DModel& md = map.models[static_cast<size_t>(model)];
  std::vector<Half> path;
  for (int k = 0; k < 3; ++k) {   // the model's bounds (+ margin) close every cell
    Half lo{}, hi{};
    lo.n[k] = -1.0;
    lo.d = -(static_cast<double>(md.mins[k]) + offset[k] - margin);
    lo.box = true;
    hi.n[k] = 1.0;
    hi.d = static_cast<double>(md.maxs[k]) + offset[k] + margin;
    hi.box = true;
    path.push_back(lo);
    path.push_back(hi);
  }
  walk(map, hv, hv.first, offset, path, verts, tris);
}

}  // namespace surf
