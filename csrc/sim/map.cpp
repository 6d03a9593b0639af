// map.cpp — BSP v30 reader and entity-lump interpreter.
//
// Entity semantics follow the reference loader (src/bsp.c:168-298) so the same
// file yields the same triggers/solids/volumes in both simulators: see the
// per-class notes below. Unlike the reference there are no fixed-size tables.
#include "map.hpp"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iterator>
#include <map>
#include <utility>

namespace surf {

const float kPlayerMins[4][3] = {{-16, -16, -36}, {-16, -16, -18}, {0, 0, 0}, {-32, -32, -32}};
const float kPlayerMaxs[4][3] = {{16, 16, 36}, {16, 16, 18}, {0, 0, 0}, {32, 32, 32}};
const float kHullMins[4][3] = {{0, 0, 0}, {-16, -16, -36}, {-32, -32, -32}, {-16, -16, -18}};
const float kHullMaxs[4][3] = {{0, 0, 0}, {16, 16, 36}, {32, 32, 32}, {16, 16, 18}};

namespace {

template <typename T>
bool read_lump(const uint8_t* data, size_t size, const DLump& lump, std::vector<T>* out,
               std::string* err) {
  if (lump.offset < 0 || lump.length < 0 ||
      static_cast<uint64_t>(lump.offset) + static_cast<uint64_t>(lump.length) > size) {
    *err = "lump out of file bounds";
    return false;
  }
  if (lump.length % static_cast<int32_t>(sizeof(T)) != 0) {
    *err = "lump size not a multiple of its element size";
    return false;
  }
  out->resize(static_cast<size_t>(lump.length) / sizeof(T));
  if (lump.length) std::memcpy(out->data(), data + lump.offset, static_cast<size_t>(lump.length));
  return true;
}

// One entity: ordered key/value pairs (first occurrence of a key wins).
struct Entity {
  std::vector<std::pair<std::string, std::string>> kv;
  const char* get(const char* key) const {
    for (auto& p : kv)
      if (p.first == key) return p.second.c_str();
    return nullptr;
  }
  float number(const char* key, float fallback) const {
    const char* v = get(key);
    return v ? static_cast<float>(std::atof(v)) : fallback;
  }
  void vec3(const char* key, float out[3]) const {
    out[0] = out[1] = out[2] = 0.f;
    if (const char* v = get(key)) std::sscanf(v, "%f %f %f", &out[0], &out[1], &out[2]);
  }
  int model_index() const {               // "*N" -> N, otherwise -1
    const char* v = get("model");
    return (v && v[0] == '*') ? std::atoi(v + 1) : -1;
  }
  float yaw() const {                     // "angles" pitch/yaw/roll, else legacy "angle"
    if (const char* a = get("angles")) {
      float v[3] = {0, 0, 0};
      std::sscanf(a, "%f %f %f", &v[0], &v[1], &v[2]);
      return v[1];
    }
    return number("angle", 0.f);
  }
};

// Split the entity lump into { "k" "v" ... } blocks. Keys are truncated to 39
// and values to 519 characters, as the engine's fixed buffers do.
std::vector<Entity> tokenize_entities(const std::string& text) {
  std::vector<Entity> out;
  size_t i = 0, n = text.size();
  auto at = [&](size_t k) { return k < n ? text[k] : '\0'; };
  while (true) {
    while (i < n && text[i] && text[i] != '{') ++i;
    if (i >= n || !text[i]) break;
    ++i;
    Entity e;
    while (true) {
      while (i < n && text[i] && text[i] != '"' && text[i] != '}') ++i;
      if (i >= n || !text[i] || text[i] == '}') {
        if (at(i) == '}') ++i;
        break;
      }
      size_t ks = ++i;
      while (i < n && text[i] && text[i] != '"') ++i;
      std::string key = text.substr(ks, i - ks);
      if (i < n) ++i;
      while (i < n && text[i] && text[i] != '"') ++i;
      if (i >= n || !text[i]) break;
      size_t vs = ++i;
      while (i < n && text[i] && text[i] != '"') ++i;
      std::string val = text.substr(vs, i - vs);
      if (i < n) ++i;
      if (e.kv.size() < 40) {
        if (key.size() > 39) key.resize(39);
        if (val.size() > 519) val.resize(519);
        e.kv.emplace_back(std::move(key), std::move(val));
      }
    }
    out.push_back(std::move(e));
  }
  return out;
}

// SetMovedir: the two "up"/"down" angle codes, otherwise the forward vector
// of the entity angles (computed in double, stored as float).
void movedir_from_angles(const float ang[3], float out[3]) {
  if (ang[0] == 0 && ang[1] == -1 && ang[2] == 0) { out[0] = 0; out[1] = 0; out[2] = 1; return; }
  if (ang[0] == 0 && ang[1] == -2 && ang[2] == 0) { out[0] = 0; out[1] = 0; out[2] = -1; return; }
  const double deg = 3.14159265358979323846 * 2 / 360;
  double p = ang[0] * deg, y = ang[1] * deg;
  out[0] = static_cast<float>(std::cos(p) * std::cos(y));
  out[1] = static_cast<float>(std::cos(p) * std::sin(y));
  out[2] = static_cast<float>(-std::sin(p));
}

bool is_solid_class(const char* c) {
  static const char* kClasses[] = {"func_wall", "func_breakable", "func_pushable",
                                   "func_button", "func_train", "func_conveyor",
                                   "func_wall_toggle", "func_rotating",
                                   "func_door_rotating", "func_door"};
  for (const char* k : kClasses)
    if (!std::strcmp(c, k)) return true;
  return false;
}

}  // namespace

bool Map::load_file(const std::string& path, std::string* err) {
  std::ifstream f(path, std::ios::binary);
  if (!f) { *err = "cannot open bsp file"; return false; }
  std::vector<uint8_t> buf((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  return load_memory(buf.data(), buf.size(), err);
}

bool Map::load_memory(const uint8_t* data, size_t size, std::string* err) {
  if (size < sizeof(DHeader)) { *err = "file too small"; return false; }
  DHeader h;
  std::memcpy(&h, data, sizeof h);
  if (h.version != kBspVersion) { *err = "not a BSP v30 file"; return false; }
  std::vector<DNode> nodes;
  std::vector<DLeaf> leafs;
  std::vector<char> ents;
  if (!read_lump(data, size, h.lumps[kLumpPlanes], &planes, err) ||
      !read_lump(data, size, h.lumps[kLumpClipnodes], &clipnodes, err) ||
      !read_lump(data, size, h.lumps[kLumpNodes], &nodes, err) ||
      !read_lump(data, size, h.lumps[kLumpLeafs], &leafs, err) ||
      !read_lump(data, size, h.lumps[kLumpModels], &models, err) ||
      !read_lump(data, size, h.lumps[kLumpEntities], &ents, err))
    return false;
  entities.assign(ents.begin(), ents.end());
  // Hull 0: render nodes become clipnodes, leaf children become leaf contents.
  hull0.resize(nodes.size());
  for (size_t i = 0; i < nodes.size(); ++i) {
    hull0[i].plane = nodes[i].plane;
    for (int s = 0; s < 2; ++s) {
      int c = nodes[i].child[s];
      if (c >= 0) { hull0[i].child[s] = static_cast<int16_t>(c); continue; }
      int leaf = -1 - c;
      if (leaf < 0 || leaf >= static_cast<int>(leafs.size())) { *err = "bad leaf ref"; return false; }
      hull0[i].child[s] = static_cast<int16_t>(leafs[leaf].contents);
    }
  }
  if (models.empty()) { *err = "no models"; return false; }
  for (int k = 0; k < 3; ++k) { world_mins[k] = models[0].mins[k]; world_maxs[k] = models[0].maxs[k]; }
  if (!parse_entities()) return false;
  build_grids();
  find_liquids();
  return true;
}

// Every value point_contents can return is a hull-0 leaf's contents (a
// current mapped to water) or a contents volume's: if none is a liquid, no
// probe of CheckWater can raise the water level.
void Map::find_liquids() {
  any_liquid = false;
  for (const DClipnode& n : hull0)
    for (int s = 0; s < 2; ++s) {
      int c = n.child[s];
      if (c >= 0) continue;
      if (c <= kCurrent0 && c >= kCurrentDown) c = kWater;
      any_liquid |= contents_liquid(c);
    }
  for (const BrushEntity& v : volumes) any_liquid |= contents_liquid(v.contents);
}

namespace {

// Which child every point of the box [lo, hi) takes at this plane, decided
// as the descent computes plane_side in float: 0 front (side >= 0), 1 back
// (side < 0), -1 undecided. Axial planes are exact. For a sloped plane the
// side is a float evaluation of dot(p, n) - d, whose error is below
// 4 u (|p||n|_1 + |d|) with u = 2^-24; the margin is 16 times that bound.
int classify_box(const Plane& pl, const double lo[3], const double hi[3]) {
  const double d = pl.dist;
  if (pl.type < 3) {
    if (lo[pl.type] >= d) return 0;
    if (hi[pl.type] <= d) return 1;
    return -1;
  }
  double tmin = 1e300, tmax = -1e300, pmax = 0, n1 = 0;
  for (int k = 0; k < 3; ++k) {
    n1 += std::fabs(static_cast<double>(pl.normal[k]));
    pmax = std::max(pmax, std::max(std::fabs(lo[k]), std::fabs(hi[k])));
  }
  for (int c = 0; c < 8; ++c) {
    double t = -d;
    for (int k = 0; k < 3; ++k) t += static_cast<double>(pl.normal[k]) * ((c >> k) & 1 ? hi[k] : lo[k]);
    tmin = std::min(tmin, t);
    tmax = std::max(tmax, t);
  }
  const double margin = 64.0 * 5.960464477539063e-08 * (n1 * pmax + std::fabs(d)) + 1e-3;
  if (tmin > margin) return 0;
  if (tmax < -margin) return 1;
  return -1;
}

struct GridFill {
  const Clipnode* nodes;
  const Plane* planes;
  const HullGrid* g;
  int32_t* cells;
  const std::vector<uint8_t>* shared;     // per node: reachable from the root along several paths
  // Descend with the box of cell range [i0, i1) while every point agrees;
  // assign the node reached, or split the range and go on from there.
  void fill(int32_t node, const int32_t i0[3], const int32_t i1[3]) {
    double lo[3], hi[3];
    for (int k = 0; k < 3; ++k) {
      lo[k] = static_cast<double>(g->mn[k]) + static_cast<double>(i0[k]) * g->size;
      hi[k] = static_cast<double>(g->mn[k]) + static_cast<double>(i1[k]) * g->size;
    }
    while (node >= 0) {
      const Clipnode& cn = nodes[node];
      const int c = classify_box(planes[cn.plane], lo, hi);
      if (c < 0) break;
      node = cn.child[c];
    }
    int ax = 0;
    for (int k = 1; k < 3; ++k)
      if (i1[k] - i0[k] > i1[ax] - i0[ax]) ax = k;
    if (node < 0 || i1[ax] - i0[ax] == 1) {
      const int32_t v = node >= 0 && (*shared)[node] ? (node | HullGrid::kShared) : node;
      for (int32_t z = i0[2]; z < i1[2]; ++z)
        for (int32_t y = i0[1]; y < i1[1]; ++y)
          for (int32_t x = i0[0]; x < i1[0]; ++x)
            cells[(static_cast<int64_t>(z) * g->n[1] + y) * g->n[0] + x] = v;
      return;
    }
    const int32_t mid = i0[ax] + (i1[ax] - i0[ax]) / 2;
    int32_t a1[3] = {i1[0], i1[1], i1[2]}, b0[3] = {i0[0], i0[1], i0[2]};
    a1[ax] = mid;
    b0[ax] = mid;
    fill(node, i0, a1);
    fill(node, b0, i1);
  }
};

}  // namespace

void Map::build_grids() {
  const MapView v = view();
  for (int hull : {0, 1, 3}) {
    grid_cells[hull].clear();
    grid_meta[hull] = HullGrid();
    const HullView h = v.hull(0, hull);
    if (h.first < 0 || h.first >= h.last) continue;
    // tree coordinates of the world model (origin 0): its bounds, padded
    double lo[3], hi[3], ext = 0;
    for (int k = 0; k < 3; ++k) {
      lo[k] = static_cast<double>(world_mins[k]) - 64.0;
      hi[k] = static_cast<double>(world_maxs[k]) + 64.0;
      ext = std::max(ext, std::max(std::fabs(lo[k]), std::fabs(hi[k])));
    }
    if (!(ext < 1048576.0)) continue;      // cell bounds must stay exact floats
    double size = 8.0;
    int32_t n[3];
    for (;;) {
      int64_t total = 1;
      for (int k = 0; k < 3; ++k) {
        const double a = std::floor(lo[k] / size) * size;
        n[k] = static_cast<int32_t>(std::ceil((hi[k] - a) / size));
        total *= n[k];
      }
      if (total <= kGridCells) break;
      size *= 2.0;
    }
    HullGrid& g = grid_meta[hull];
    for (int k = 0; k < 3; ++k) {
      g.mn[k] = static_cast<float>(std::floor(lo[k] / size) * size);
      g.n[k] = n[k];
    }
    g.size = static_cast<float>(size);
    g.inv = static_cast<float>(1.0 / size);
    // nodes with more than one path from the root (a parent reached along
    // several paths, or several parents): a segment's two endpoints reaching
    // one of them may have taken different paths
    const int nn = h.last + 1;
    std::vector<int32_t> indeg(nn, 0);
    std::vector<uint8_t> seen(nn, 0), shared(nn, 0);
    std::vector<int32_t> order, stack{h.first};
    while (!stack.empty()) {
      const int32_t x = stack.back();
      stack.pop_back();
      if (x < 0 || x >= nn || seen[x]) continue;
      seen[x] = 1;
      order.push_back(x);
      for (int c = 0; c < 2; ++c) {
        const int32_t ch = h.nodes[x].child[c];
        if (ch >= 0 && ch < nn) {
          ++indeg[ch];
          stack.push_back(ch);
        }
      }
    }
    // propagate down to a fixed point (the graph is acyclic)
    for (int32_t x : order) if (indeg[x] > 1) shared[x] = 1;
    for (bool changed = true; changed;) {
      changed = false;
      for (int32_t x : order) {
        if (!shared[x]) continue;
        for (int c = 0; c < 2; ++c) {
          const int32_t ch = h.nodes[x].child[c];
          if (ch >= 0 && ch < nn && !shared[ch]) { shared[ch] = 1; changed = true; }
        }
      }
    }
    grid_cells[hull].assign(static_cast<size_t>(n[0]) * n[1] * n[2], HullGrid::kNone);
    GridFill f{h.nodes, h.planes, &g, grid_cells[hull].data(), &shared};
    const int32_t i0[3] = {0, 0, 0};
    f.fill(h.first, i0, n);
  }
}

namespace {
template <typename T>
Span<T> span_of(const std::vector<T>& v) {
  Span<T> s;
  s.p = v.data();
  s.n = static_cast<int32_t>(v.size());
  return s;
}
// The aligned mirror of a packed record array (same bytes; vector storage is
// at least 8-byte aligned).
template <typename A, typename D>
Span<A> span_as(const std::vector<D>& v) {
  static_assert(sizeof(A) == sizeof(D), "layout");
  Span<A> s;
  s.p = reinterpret_cast<const A*>(v.data());
  s.n = static_cast<int32_t>(v.size());
  return s;
}
}  // namespace

MapView Map::view() const {
  MapView v;
  v.planes = span_as<Plane>(planes);
  v.clipnodes = span_as<Clipnode>(clipnodes);
  v.hull0 = span_as<Clipnode>(hull0);
  v.models = span_as<Model>(models);
  v.solids = span_of(solids);
  v.volumes = span_of(volumes);
  v.triggers = span_of(triggers);
  v.spawns = span_of(spawns);
  for (int k = 0; k < 3; ++k) { v.world_mins[k] = world_mins[k]; v.world_maxs[k] = world_maxs[k]; }
  v.any_liquid = any_liquid;
  for (int h = 0; h < 4; ++h) {
    v.world_grid[h] = grid_meta[h];
    v.world_grid[h].cells = grid_cells[h].empty() ? nullptr : grid_cells[h].data();
  }
  return v;
}

bool Map::parse_entities() {
  auto ents = tokenize_entities(entities);
  struct Target { std::string name; float origin[3]; float yaw; };
  std::vector<Target> targets;
  std::vector<std::pair<size_t, std::string>> pending;     // trigger index -> target name
  solids.clear(); volumes.clear(); triggers.clear(); spawns.clear();

  auto bounds = [&](int model, const float org[3], float lo[3], float hi[3]) {
    const DModel& m = models[static_cast<size_t>(model)];
    for (int k = 0; k < 3; ++k) { lo[k] = m.mins[k] + org[k] - 1.f; hi[k] = m.maxs[k] + org[k] + 1.f; }
  };

  for (const Entity& e : ents) {
    const char* cls = e.get("classname");
    if (!cls) continue;
    int model = e.model_index();
    if (model >= static_cast<int>(models.size())) continue;        // malformed "*N"
    float origin[3];
    e.vec3("origin", origin);

    if (!std::strncmp(cls, "info_player_start", 17) || !std::strncmp(cls, "info_player_deathmatch", 22)) {
      SpawnPoint sp{{origin[0], origin[1], origin[2]}, e.yaw()};
      spawns.push_back(sp);
    } else if (model >= 0 && !std::strcmp(cls, "trigger_teleport")) {
      Trigger t;
      t.kind = TriggerKind::kTeleport; t.model = model;
      for (int k = 0; k < 3; ++k) t.origin[k] = origin[k];
      bounds(model, origin, t.absmin, t.absmax);
      if (const char* tgt = e.get("target")) pending.emplace_back(triggers.size(), std::string(tgt).substr(0, 63));
      triggers.push_back(t);
    } else if (model >= 0 && !std::strcmp(cls, "trigger_hurt")) {
      Trigger t;
      t.kind = TriggerKind::kHurt; t.model = model;
      for (int k = 0; k < 3; ++k) t.origin[k] = origin[k];
      bounds(model, origin, t.absmin, t.absmax);
      t.damage = e.number("dmg", 10.f);
      triggers.push_back(t);
    } else if (model >= 0 && !std::strcmp(cls, "trigger_push")) {
      Trigger t;
      t.kind = TriggerKind::kPush; t.model = model;
      for (int k = 0; k < 3; ++k) t.origin[k] = origin[k];
      bounds(model, origin, t.absmin, t.absmax);
      float ang[3];
      e.vec3("angles", ang);
      if (!e.get("angles") && e.get("angle")) { ang[0] = ang[2] = 0; ang[1] = e.number("angle", 0.f); }
      if (ang[0] == 0 && ang[1] == 0 && ang[2] == 0) ang[1] = 360.f;   // CTriggerPush::Spawn
      float dir[3];
      movedir_from_angles(ang, dir);
      float speed = e.number("speed", 0.f);
      if (speed == 0.f) speed = 100.f;
      for (int k = 0; k < 3; ++k) t.push_velocity[k] = dir[k] * speed;
      t.push_once = (static_cast<int>(e.number("spawnflags", 0)) & 1) != 0;
      triggers.push_back(t);
    } else if (model >= 0 &&
               (!std::strcmp(cls, "func_water") || !std::strcmp(cls, "func_ladder") ||
                (!std::strcmp(cls, "func_illusionary") && e.number("skin", -1.f) < -1.f) ||
                (!std::strcmp(cls, "func_door") && e.number("skin", 0.f) < -1.f))) {
      // Non-solid contents volumes: the brush carries its skin as contents.
      BrushEntity v;
      v.model = model;
      for (int k = 0; k < 3; ++k) v.origin[k] = origin[k];
      v.contents = !std::strcmp(cls, "func_ladder") ? kLadder : static_cast<int32_t>(e.number("skin", -3.f));
      bounds(model, origin, v.absmin, v.absmax);
      volumes.push_back(v);
    } else if (model >= 0) {
      bool solid = is_solid_class(cls);
      // SF_CONVEYOR_NOTSOLID (2) turns a func_conveyor into decoration.
      if (solid && !std::strcmp(cls, "func_conveyor") && (static_cast<int>(e.number("spawnflags", 0)) & 2))
        solid = false;
      if (solid) {
        BrushEntity s;
        s.model = model;
        for (int k = 0; k < 3; ++k) s.origin[k] = origin[k];
        bounds(model, origin, s.absmin, s.absmax);
        solids.push_back(s);
      }
    } else if (const char* tn = e.get("targetname")) {
      Target t{std::string(tn).substr(0, 63), {origin[0], origin[1], origin[2]}, e.yaw()};
      targets.push_back(t);
    }
  }
  for (auto& p : pending) {
    for (auto& t : targets) {
      if (t.name == p.second) {
        Trigger& tr = triggers[p.first];
        tr.has_dest = true;
        for (int k = 0; k < 3; ++k) tr.dest[k] = t.origin[k];
        tr.dest_yaw = t.yaw;
        break;
      }
    }
  }
  return true;
}

}  // namespace surf
