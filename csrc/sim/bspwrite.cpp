// bspwrite.cpp — brush compiler for procedural maps. See bspwrite.hpp.
#include "bspwrite.hpp"

#include <algorithm>
#include <array>
#include <cmath>
#include <cstring>
#include <map>
#include <tuple>

namespace surf {
namespace {

struct Box { double lo[3], hi[3]; };

struct XBrush {                    // a brush expanded for one hull
  std::vector<BrushPlane> planes;
  double lo[3], hi[3];
  int contents;
};

struct GNode { int plane; int child[2]; Box region; };   // child < 0 = contents

class PlaneTable {
 public:
  // Index of plane n.x = d in engine form; *flip set when the stored plane
  // faces the opposite way (axial planes must face +axis).
  int index(const float n[3], float d, bool* flip) {
    float nn[3] = {n[0], n[1], n[2]};
    float dd = d;
    *flip = false;
    for (int a = 0; a < 3; ++a) {
      if (nn[a] == -1.f && nn[(a + 1) % 3] == 0.f && nn[(a + 2) % 3] == 0.f) {
        nn[a] = 1.f; dd = -dd; *flip = true;
      }
    }
    for (int a = 0; a < 3; ++a) if (nn[a] == 0.f) nn[a] = 0.f;    // scrub -0
    auto key = std::make_tuple(nn[0], nn[1], nn[2], dd);
    auto it = lut_.find(key);
    if (it != lut_.end()) return it->second;
    DPlane p;
    for (int a = 0; a < 3; ++a) p.normal[a] = nn[a];
    p.dist = dd;
    int type = 3;
    for (int a = 0; a < 3; ++a)
      if (nn[a] == 1.f && nn[(a + 1) % 3] == 0.f && nn[(a + 2) % 3] == 0.f) type = a;
    if (type == 3) {
      float ax = std::fabs(nn[0]), ay = std::fabs(nn[1]), az = std::fabs(nn[2]);
      type = (ax >= ay && ax >= az) ? 3 : (ay >= az ? 4 : 5);
    }
    p.type = type;
    int id = static_cast<int>(planes.size());
    planes.push_back(p);
    lut_[key] = id;
    return id;
  }
  std::vector<DPlane> planes;

 private:
  std::map<std::tuple<float, float, float, float>, int> lut_;
};

bool brush_bounds(const Brush& b, double lo[3], double hi[3]) {
  const size_t np = b.planes.size();
  bool any = false;
  for (int a = 0; a < 3; ++a) { lo[a] = 1e30; hi[a] = -1e30; }
  for (size_t i = 0; i < np; ++i)
    for (size_t j = i + 1; j < np; ++j)
      for (size_t k = j + 1; k < np; ++k) {
        const float* a = b.planes[i].n;
        const float* c = b.planes[j].n;
        const float* e = b.planes[k].n;
        double det = a[0] * (double(c[1]) * e[2] - double(c[2]) * e[1]) - a[1] * (double(c[0]) * e[2] - double(c[2]) * e[0]) +
                     a[2] * (double(c[0]) * e[1] - double(c[1]) * e[0]);
        if (std::fabs(det) < 1e-9) continue;
        double d1 = b.planes[i].d, d2 = b.planes[j].d, d3 = b.planes[k].d;
        // Cramer's rule
        double x = (d1 * (double(c[1]) * e[2] - double(c[2]) * e[1]) - a[1] * (d2 * e[2] - double(c[2]) * d3) +
                    a[2] * (d2 * e[1] - double(c[1]) * d3)) / det;
        double y = (a[0] * (d2 * e[2] - double(c[2]) * d3) - d1 * (double(c[0]) * e[2] - double(c[2]) * e[0]) +
                    a[2] * (double(c[0]) * d3 - d2 * e[0])) / det;
        double z = (a[0] * (double(c[1]) * d3 - d2 * e[1]) - a[1] * (double(c[0]) * d3 - d2 * e[0]) +
                    d1 * (double(c[0]) * e[1] - double(c[1]) * e[0])) / det;
        double p[3] = {x, y, z};
        bool inside = true;
        for (size_t q = 0; q < np && inside; ++q) {
          const BrushPlane& pl = b.planes[q];
          if (pl.n[0] * p[0] + pl.n[1] * p[1] + pl.n[2] * p[2] - pl.d > 1e-3) inside = false;
        }
        if (!inside) continue;
        any = true;
        for (int t = 0; t < 3; ++t) { lo[t] = std::min(lo[t], p[t]); hi[t] = std::max(hi[t], p[t]); }
      }
  return any;
}

XBrush expand(const Brush& b, const double blo[3], const double bhi[3], const float hmin[3], const float hmax[3]) {
  XBrush x;
  x.contents = b.contents;
  for (const BrushPlane& p : b.planes) {
    BrushPlane q = p;
    double d = p.d;
    for (int a = 0; a < 3; ++a) d -= p.n[a] > 0 ? p.n[a] * hmin[a] : p.n[a] * hmax[a];
    q.d = static_cast<float>(d);
    x.planes.push_back(q);
  }
  for (int a = 0; a < 3; ++a) {                      // axial bevels
    for (int s = 0; s < 2; ++s) {
      float sign = s == 0 ? 1.f : -1.f;
      bool have = false;
      for (const BrushPlane& p : b.planes)
        if (p.n[a] == sign && p.n[(a + 1) % 3] == 0.f && p.n[(a + 2) % 3] == 0.f) have = true;
      if (have) continue;
      BrushPlane q{{0, 0, 0}, 0};
      q.n[a] = sign;
      q.d = static_cast<float>(sign > 0 ? bhi[a] - hmin[a] : -blo[a] + hmax[a]);
      x.planes.push_back(q);
    }
  }
  for (int a = 0; a < 3; ++a) { x.lo[a] = blo[a] - hmax[a]; x.hi[a] = bhi[a] - hmin[a]; }
  return x;
}

// Signed distance range of a box against plane n.x - d.
void box_plane_range(const Box& r, const BrushPlane& p, double* mn, double* mx) {
  double lo = -p.d, hi = -p.d;
  for (int a = 0; a < 3; ++a) {
    double u = p.n[a] * r.lo[a], v = p.n[a] * r.hi[a];
    lo += std::min(u, v);
    hi += std::max(u, v);
  }
  *mn = lo;
  *mx = hi;
}

class TreeBuilder {
 public:
  TreeBuilder(const std::vector<XBrush>& brushes, PlaneTable* planes, std::vector<GNode>* nodes)
      : br_(brushes), planes_(planes), nodes_(nodes) {}

  int build(std::vector<int> ids, const Box& region, int depth) {
    ids.erase(std::remove_if(ids.begin(), ids.end(), [&](int i) { return !overlaps(br_[i], region); }), ids.end());
    if (ids.empty()) return kEmpty;
    if (ids.size() > kLeafBrushes && depth < 48) {
      // Candidate splits: brush bound coordinates on every axis. Pick the one
      // that duplicates the fewest brushes into both children, then the most
      // balanced; a split must shrink both sides.
      int best_axis = -1;
      double best_split = 0, best_cost = 1e30;
      for (int a = 0; a < 3; ++a) {
        std::vector<double> cand;
        for (int i : ids) { cand.push_back(std::floor(br_[i].lo[a])); cand.push_back(std::ceil(br_[i].hi[a])); }
        std::sort(cand.begin(), cand.end());
        cand.erase(std::unique(cand.begin(), cand.end()), cand.end());
        const size_t stride = std::max<size_t>(1, cand.size() / 64);
        for (size_t ci = 0; ci < cand.size(); ci += stride) {
          double split = cand[ci];
          if (split <= region.lo[a] + 1 || split >= region.hi[a] - 1) continue;
          size_t nf = 0, nb = 0;
          for (int i : ids) {
            if (br_[i].hi[a] >= split) ++nf;
            if (br_[i].lo[a] <= split) ++nb;
          }
          if (nf == ids.size() || nb == ids.size()) continue;
          double cost = static_cast<double>(nf + nb) + 0.25 * std::fabs(static_cast<double>(nf) - static_cast<double>(nb));
          if (cost < best_cost) { best_cost = cost; best_axis = a; best_split = split; }
        }
      }
      if (best_axis >= 0) {
        const int a = best_axis;
        const double split = best_split;
        std::vector<int> front, back;
        for (int i : ids) {
          if (br_[i].hi[a] >= split) front.push_back(i);
          if (br_[i].lo[a] <= split) back.push_back(i);
        }
        Box fr = region, bk = region;
        fr.lo[a] = split;
        bk.hi[a] = split;
        float n[3] = {0, 0, 0};
        n[a] = 1.f;
        bool flip;
        int pl = planes_->index(n, static_cast<float>(split), &flip);
        int cf = build(front, fr, depth + 1);
        int cb = build(back, bk, depth + 1);
        return make(pl, cf, cb, region);
      }
    }
    std::stable_sort(ids.begin(), ids.end(), [&](int x, int y) {
      return (br_[x].contents == kSolid) > (br_[y].contents == kSolid);   // solid wins over liquids
    });
    return chain(ids, 0, region);
  }

 private:
  static bool overlaps(const XBrush& b, const Box& r) {
    for (int a = 0; a < 3; ++a)
      if (b.hi[a] < r.lo[a] || b.lo[a] > r.hi[a]) return false;
    return true;
  }
  // Create (or reuse an identical) node; identical subtrees collapse.
  int make(int plane, int front, int back, const Box& region) {
    auto key = std::make_tuple(plane, front, back);
    auto it = memo_.find(key);
    if (it != memo_.end()) return it->second;
    GNode g;
    g.plane = plane;
    g.child[0] = front;
    g.child[1] = back;
    g.region = region;
    nodes_->push_back(g);
    int id = static_cast<int>(nodes_->size()) - 1;
    memo_[key] = id;
    return id;
  }
  int chain(const std::vector<int>& ids, size_t k, const Box& region) {
    if (k == ids.size()) return kEmpty;
    int rest = chain(ids, k + 1, region);
    const XBrush& b = br_[ids[k]];
    std::vector<const BrushPlane*> cut;
    for (const BrushPlane& p : b.planes) {
      double mn, mx;
      box_plane_range(region, p, &mn, &mx);
      if (mn > 0) return rest;             // region wholly outside this brush
      if (mx <= 0) continue;               // plane does not cut the region
      cut.push_back(&p);
    }
    int cur = b.contents;
    for (auto it = cut.rbegin(); it != cut.rend(); ++it) {
      bool flip;
      int pl = planes_->index((*it)->n, (*it)->d, &flip);
      // unflipped: front (n.x >= d) is outside -> rest; back -> deeper in the brush
      cur = flip ? make(pl, cur, rest, region) : make(pl, rest, cur, region);
    }
    return cur;
  }
  static constexpr size_t kLeafBrushes = 3;
  const std::vector<XBrush>& br_;
  PlaneTable* planes_;
  std::vector<GNode>* nodes_;
  std::map<std::tuple<int, int, int>, int> memo_;
};

template <typename T>
void append_lump(std::vector<uint8_t>* out, DHeader* h, int lump, const T* data, size_t count) {
  while (out->size() % 4) out->push_back(0);
  h->lumps[lump].offset = static_cast<int32_t>(out->size());
  h->lumps[lump].length = static_cast<int32_t>(count * sizeof(T));
  const uint8_t* p = reinterpret_cast<const uint8_t*>(data);
  out->insert(out->end(), p, p + count * sizeof(T));
}

int16_t clamp16(double v) { return static_cast<int16_t>(std::max(-32767.0, std::min(32767.0, v))); }

}  // namespace

bool BspWriter::build(std::vector<uint8_t>* out, std::string* err) {
  int nmodels = 1;
  for (const Brush& b : brushes_) nmodels = std::max(nmodels, b.model + 1);
  PlaneTable planes;
  std::vector<GNode> hull0_nodes, clip_nodes;
  std::vector<DModel> models(static_cast<size_t>(nmodels));
  // leaf 0 = solid, 1 = empty; liquids get their own leaves
  std::vector<int> leaf_contents = {kSolid, kEmpty};

  for (int m = 0; m < nmodels; ++m) {
    std::vector<const Brush*> mb;
    std::vector<std::array<double, 6>> bounds;
    double mlo[3] = {1e30, 1e30, 1e30}, mhi[3] = {-1e30, -1e30, -1e30};
    for (const Brush& b : brushes_) {
      if (b.model != m) continue;
      double lo[3], hi[3];
      if (!brush_bounds(b, lo, hi)) continue;
      mb.push_back(&b);
      bounds.push_back({lo[0], lo[1], lo[2], hi[0], hi[1], hi[2]});
      for (int a = 0; a < 3; ++a) { mlo[a] = std::min(mlo[a], lo[a]); mhi[a] = std::max(mhi[a], hi[a]); }
    }
    DModel& dm = models[static_cast<size_t>(m)];
    std::memset(&dm, 0, sizeof dm);
    if (mb.empty()) {
      for (int a = 0; a < 3; ++a) mlo[a] = mhi[a] = 0;
    }
    for (int a = 0; a < 3; ++a) { dm.mins[a] = static_cast<float>(mlo[a]); dm.maxs[a] = static_cast<float>(mhi[a]); }
    for (int hull = 0; hull < 4; ++hull) {
      std::vector<XBrush> xb;
      for (size_t i = 0; i < mb.size(); ++i) {
        if (hull > 0 && mb[i]->contents != kSolid) continue;      // liquids are not clip geometry
        if (hull == 2 && !large_hull_) continue;                    // monster-size hull: players never use it
        double lo[3] = {bounds[i][0], bounds[i][1], bounds[i][2]};
        double hi[3] = {bounds[i][3], bounds[i][4], bounds[i][5]};
        xb.push_back(expand(*mb[i], lo, hi, kHullMins[hull], kHullMaxs[hull]));
      }
      Box region;
      for (int a = 0; a < 3; ++a) { region.lo[a] = mlo[a] - 64 - 1; region.hi[a] = mhi[a] + 64 + 1; }
      std::vector<int> ids(xb.size());
      for (size_t i = 0; i < xb.size(); ++i) ids[i] = static_cast<int>(i);
      std::vector<GNode>& nodes = hull == 0 ? hull0_nodes : clip_nodes;
      TreeBuilder tb(xb, &planes, &nodes);
      int root = tb.build(ids, region, 0);
      if (root < 0) {
        // An empty (or all-liquid) tree still needs a node: one plane, both sides `root`.
        float n[3] = {0, 0, 1};
        bool flip;
        GNode g;
        g.plane = planes.index(n, static_cast<float>(mlo[2]), &flip);
        g.child[0] = g.child[1] = root;
        g.region = region;
        nodes.push_back(g);
        root = static_cast<int>(nodes.size()) - 1;
      }
      dm.headnode[hull] = root;
    }
  }
  // A trailing filler node: the engine treats a tree whose head is the last
  // node of the lump as empty, so no head may sit there.
  for (auto* nodes : {&hull0_nodes, &clip_nodes}) {
    GNode g;
    g.plane = 0;
    g.child[0] = g.child[1] = kEmpty;
    g.region = Box{{0, 0, 0}, {0, 0, 0}};
    if (planes.planes.empty()) {
      float n[3] = {0, 0, 1};
      bool flip;
      planes.index(n, 0.f, &flip);
    }
    nodes->push_back(g);
  }
  if (clip_nodes.size() > 32767 || hull0_nodes.size() > 32767) {
    *err = "BSP node limit exceeded (" + std::to_string(clip_nodes.size()) + " clipnodes, " +
           std::to_string(hull0_nodes.size()) + " nodes); use fewer or larger brushes";
    return false;
  }
  std::vector<DClipnode> dclip(clip_nodes.size());
  for (size_t i = 0; i < clip_nodes.size(); ++i) {
    dclip[i].plane = clip_nodes[i].plane;
    dclip[i].child[0] = static_cast<int16_t>(clip_nodes[i].child[0]);
    dclip[i].child[1] = static_cast<int16_t>(clip_nodes[i].child[1]);
  }
  auto leaf_of = [&](int contents) {
    for (size_t i = 0; i < leaf_contents.size(); ++i)
      if (leaf_contents[i] == contents) return static_cast<int>(i);
    leaf_contents.push_back(contents);
    return static_cast<int>(leaf_contents.size()) - 1;
  };
  std::vector<DNode> dnodes(hull0_nodes.size());
  for (size_t i = 0; i < hull0_nodes.size(); ++i) {
    const GNode& g = hull0_nodes[i];
    DNode& d = dnodes[i];
    std::memset(&d, 0, sizeof d);
    d.plane = g.plane;
    for (int s = 0; s < 2; ++s)
      d.child[s] = static_cast<int16_t>(g.child[s] >= 0 ? g.child[s] : -1 - leaf_of(g.child[s]));
    for (int a = 0; a < 3; ++a) { d.mins[a] = clamp16(g.region.lo[a]); d.maxs[a] = clamp16(g.region.hi[a]); }
  }
  std::vector<DLeaf> dleafs(leaf_contents.size());
  for (size_t i = 0; i < leaf_contents.size(); ++i) {
    std::memset(&dleafs[i], 0, sizeof(DLeaf));
    dleafs[i].contents = leaf_contents[i];
    dleafs[i].vis_offset = -1;
  }
  DHeader h;
  std::memset(&h, 0, sizeof h);
  h.version = kBspVersion;
  out->assign(sizeof(DHeader), 0);
  std::string ents = entities_;
  ents.push_back('\0');
  for (int l = 0; l < kNumLumps; ++l) { h.lumps[l].offset = static_cast<int32_t>(out->size()); h.lumps[l].length = 0; }
  append_lump(out, &h, kLumpEntities, ents.data(), ents.size());
  append_lump(out, &h, kLumpPlanes, planes.planes.data(), planes.planes.size());
  append_lump(out, &h, kLumpNodes, dnodes.data(), dnodes.size());
  append_lump(out, &h, kLumpClipnodes, dclip.data(), dclip.size());
  append_lump(out, &h, kLumpLeafs, dleafs.data(), dleafs.size());
  append_lump(out, &h, kLumpModels, models.data(), models.size());
  for (int l = 0; l < kNumLumps; ++l)
    if (h.lumps[l].length == 0) h.lumps[l].offset = static_cast<int32_t>(out->size());
  std::memcpy(out->data(), &h, sizeof h);
  return true;
}

}  // namespace surf
